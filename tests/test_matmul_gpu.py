"""Projection GEMVs (g4a_matmul / g4a_matmul_group) through the C ABI, bit for bit against the
oracle's restatement of the reference shaders (matmul_quant*.wgsl, matmul_q8*.wgsl,
matmul_q4k*.wgsl).  Shapes: the Gemma 4 E2B projections (hidden 1536; q 2048 / 4096, k and v
256 / 512, o back to 1536: src/config/gemma4-e2b.ts:31-53), ragged N (the f16 scalar path and a
partial last 256-element step), M not a multiple of the 8 rows a CTA takes per pass, a long
grid-stride run, zero-size and invalid calls, and the Q/K/V group of one launch."""
import numpy as np
import pytest
import torch

from g4attn import G4AError, _lib, quant
from gpu_helpers import dev, host, same_bits

pytestmark = pytest.mark.gpu

F16, Q8, Q4K = _lib.WEIGHT_F16, _lib.WEIGHT_Q8, _lib.WEIGHT_Q4K


def _pack(fmt, w):
    """(device weight, device scales or None, host weight, host scales)."""
    if fmt == F16:
        wq = w.astype(np.float16).view(np.uint16)
        return dev(wq.view(np.int16)), None, wq, None
    if fmt == Q8:
        wq, sc = quant.quantize_q8(w)
    else:
        wq, sc = quant.quantize_q4k(w)
    return dev(wq.view(np.int32)), dev(sc.view(np.int16)), wq, sc


def _inputs(seed, M, N, scale=0.05):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(N).astype(np.float32)
    w = (rng.standard_normal((M, N)) * scale).astype(np.float32)
    return x, w


@pytest.mark.parametrize("fmt", [F16, Q8, Q4K])
@pytest.mark.parametrize("M,N", [(2048, 1536), (256, 1536), (1536, 2048), (4096, 1536), (512, 1536),
                                 (1536, 4096), (13, 256), (1, 512), (1003, 768)])
def test_matmul_bit_exact(ctx, oracle, fmt, M, N):
    x, w = _inputs(M * 7 + N + fmt, M, N)
    wd, sd, wq, sc = _pack(fmt, w)
    out = torch.full((M,), float("nan"), device="cuda")
    ctx.matmul(fmt, dev(x), wd, sd, out, M=M, N=N)
    ctx.sync()
    ref = oracle.matmul(fmt, x, wq, sc, M, N)
    assert same_bits(host(out), ref), f"fmt {fmt} M {M} N {N}: max diff {np.abs(host(out) - ref).max()}"


@pytest.mark.parametrize("fmt,N", [(F16, 100), (F16, 1000), (F16, 1544), (F16, 8), (Q8, 544), (Q8, 32),
                                   (Q8, 1056)])
def test_matmul_ragged_n(ctx, oracle, fmt, N):
    M = 37
    x, w = _inputs(N, M, N, scale=1.0)
    wd, sd, wq, sc = _pack(fmt, w)
    out = torch.full((M,), float("nan"), device="cuda")
    ctx.matmul(fmt, dev(x), wd, sd, out, M=M, N=N)
    ctx.sync()
    assert same_bits(host(out), oracle.matmul(fmt, x, wq, sc, M, N))


def test_matmul_f16_unaligned_weight_uses_the_scalar_path(ctx, oracle):
    M, N = 19, 512
    x, w = _inputs(5, M, N)
    wq = w.astype(np.float16).view(np.uint16)
    buf = dev(np.concatenate([np.zeros(1, np.uint16), wq.reshape(-1)]).view(np.int16))
    out = torch.empty((M,), device="cuda")
    ctx.matmul(F16, dev(x), buf[1:], None, out, M=M, N=N)  # 2-byte aligned, not 16
    ctx.sync()
    assert same_bits(host(out), oracle.matmul(F16, x, wq, None, M, N))


def test_matmul_long_grid_stride_and_large_n(ctx, oracle):
    M, N = 40000, 256  # more rows than one pass of the grid covers
    x, w = _inputs(11, M, N)
    for fmt in (F16, Q4K):
        wd, sd, wq, sc = _pack(fmt, w)
        out = torch.empty((M,), device="cuda")
        ctx.matmul(fmt, dev(x), wd, sd, out, M=M, N=N)
        ctx.sync()
        assert same_bits(host(out), oracle.matmul(fmt, x, wq, sc, M, N))
    # streaming-sized row counts take the register-resident input variant (Q8 and 4-bit)
    M, N = 70000, 1536
    x, w = _inputs(13, M, N)
    for fmt in (Q8, Q4K):
        wd, sd, wq, sc = _pack(fmt, w)
        out = torch.empty((M,), device="cuda")
        ctx.matmul(fmt, dev(x), wd, sd, out, M=M, N=N)
        ctx.sync()
        assert same_bits(host(out), oracle.matmul(fmt, x, wq, sc, M, N)), fmt
    M, N = 64, 12288  # the widest reference matmul input (FFN down of the double-wide layers)
    x, w = _inputs(12, M, N)
    for fmt in (F16, Q8, Q4K):
        wd, sd, wq, sc = _pack(fmt, w)
        out = torch.empty((M,), device="cuda")
        ctx.matmul(fmt, dev(x), wd, sd, out, M=M, N=N)
        ctx.sync()
        assert same_bits(host(out), oracle.matmul(fmt, x, wq, sc, M, N))


def test_matmul_special_values(ctx, oracle):
    """Zero rows and blocks (scale 0), signed zeros and inf/nan in the input propagate as in f32."""
    M, N = 8, 512
    x, w = _inputs(13, M, N)
    w[0] = 0.0
    w[1, :32] = 0.0
    x[5] = -0.0
    xi = x.copy()
    xi[7] = np.inf
    for fmt in (F16, Q8, Q4K):
        wd, sd, wq, sc = _pack(fmt, w)
        for xx in (x, xi):
            out = torch.empty((M,), device="cuda")
            ctx.matmul(fmt, dev(xx), wd, sd, out, M=M, N=N)
            ctx.sync()
            got, ref = host(out), oracle.matmul(fmt, xx, wq, sc, M, N)
            assert np.array_equal(np.isnan(got), np.isnan(ref))
            ok = ~np.isnan(ref)
            assert same_bits(got[ok], ref[ok])


@pytest.mark.parametrize("fmt", [F16, Q8, Q4K])
def test_matmul_group_qkv(ctx, oracle, fmt):
    """Q (2048), K (256) and V (256) rows of one layer from the same normed input in one launch."""
    N = 1536
    rng = np.random.default_rng(fmt)
    x = rng.standard_normal(N).astype(np.float32)
    jobs, refs, outs = [], [], []
    for i, M in enumerate((2048, 256, 256)):
        w = (rng.standard_normal((M, N)) * 0.05).astype(np.float32)
        wd, sd, wq, sc = _pack(fmt, w)
        o = torch.full((M,), float("nan"), device="cuda")
        jobs.append((wd, sd, o, M))
        outs.append(o)
        refs.append(oracle.matmul(fmt, x, wq, sc, M, N))
        jobs[-1] = (wd, sd, o, M)
    ctx.matmul_group(fmt, dev(x), N, jobs)
    ctx.sync()
    for o, r in zip(outs, refs):
        assert same_bits(host(o), r)


def test_matmul_zero_sizes_and_errors(ctx):
    x = torch.zeros(256, device="cuda")
    w = torch.zeros(256 * 4, dtype=torch.int16, device="cuda")
    out = torch.full((4,), 7.0, device="cuda")
    ctx.matmul(F16, x, w, None, out, M=0, N=256)  # nothing to do
    ctx.sync()
    assert same_bits(host(out), np.full(4, 7.0, np.float32))
    ctx.matmul(F16, x, w, None, out, M=4, N=0)  # empty dot products are 0
    ctx.sync()
    assert same_bits(host(out), np.zeros(4, np.float32))
    q = torch.zeros(1024, dtype=torch.int32, device="cuda")
    s = torch.zeros(1024, dtype=torch.int16, device="cuda")
    with pytest.raises(G4AError, match="N % 32"):
        ctx.matmul(Q8, x, q, s, out, M=4, N=48)
    with pytest.raises(G4AError, match="N % 256"):
        ctx.matmul(Q4K, x, q, s, out, M=4, N=288)
    with pytest.raises(G4AError, match="16-byte aligned"):
        ctx.matmul(Q8, x, q[1:], s, out, M=4, N=64)
    with pytest.raises(G4AError, match="null scales"):
        ctx.matmul(Q8, x, q, None, out, M=4, N=64)
    with pytest.raises(G4AError, match="weight_format"):
        ctx.matmul(3, x, q, s, out, M=4, N=64)
    with pytest.raises(G4AError, match="num_jobs"):
        ctx.matmul_group(F16, x, 256, [(w, None, out, 4)] * 5)
    ctx.sync()
