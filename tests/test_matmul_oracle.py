"""CPU checks of the projection-matmul oracle and of the reference's weight packing (no GPU).

* g4attn.quant mirrors createQ8Buffers / createQ4KBuffers (src/engine.ts:638-674, 699-739) and
  the truncating f32ToF16 (src/gguf.ts:440-455): known bit patterns, JS Math.round halves, the
  dequantisation error bound, and the packing order the shaders read (matmul_q8.wgsl:25-28,
  47; matmul_q4k.wgsl:46-47).
* orc_matmul_* (the shaders' 256-thread order in f32) against a float64 dot product of the
  dequantised weights: the restatement computes the right thing; its bit-level order is what
  the GPU tests then hold the kernels to.
"""
import numpy as np
import pytest

from g4attn import quant


def test_f32_to_f16_trunc_known_values():
    vals = np.array([0.0, -0.0, 1.0, -2.0, 65504.0, 1e6, 1.0 + 0.75 * 2.0**-10, 2.0**-14, 2.0**-24, 2.0**-26,
                     float("inf"), 1e-40], dtype=np.float64)
    got = quant.f32_to_f16_trunc(vals)
    want = [0x0000, 0x8000, 0x3C00, 0xC000, 0x7BFF, 0x7C00, 0x3C00, 0x0400, 0x0001, 0x0000, 0x7C00, 0x0000]
    assert [int(g) for g in got] == want
    assert int(quant.f32_to_f16_trunc(np.array([float("nan")]))[0]) & 0x7C00 == 0x7C00


def test_js_round_halves_go_up():
    w = np.zeros((1, 32), dtype=np.float32)
    w[0, 0] = 127.0          # scale 1
    w[0, 1] = -2.5           # Math.round(-2.5) = -2 (numpy's rint would give -2 too; -3.5 -> -3 differs)
    w[0, 2] = -3.5
    w[0, 3] = 2.5
    q, s = quant.quantize_q8(w)
    qb = q.view(np.int8)
    assert list(qb[:4]) == [127, -2, -3, 3]
    assert int(s[0, 0]) == 0x3C00


@pytest.mark.parametrize("M,N", [(3, 32), (7, 1536), (16, 2048)])
def test_q8_roundtrip_and_layout(M, N):
    rng = np.random.default_rng(M * N)
    w = (rng.standard_normal((M, N)) * 0.05).astype(np.float32)
    q, s = quant.quantize_q8(w)
    assert q.dtype == np.uint32 and q.size == M * N // 4 and s.shape == (M, N // 32)
    deq = quant.dequantize_q8(q, s, M, N)
    scale = s.view(np.float16).astype(np.float64).repeat(32, axis=1)
    assert np.all(np.abs(deq - w) <= 0.5 * scale * (1 + 2.0**-9) + 127 * scale * 2.0**-10 + 1e-12)
    # element k of row m is byte (m N + k) % 4 of word (m N + k) / 4
    m, k = M - 1, N - 3
    gi = m * N + k
    b = (int(q[gi >> 2]) >> (8 * (gi & 3))) & 0xFF
    qv = b - 256 if b >= 128 else b
    assert qv == int(np.floor(w[m, k] / (np.abs(w[m, (k // 32) * 32:(k // 32) * 32 + 32]).max() / 127.0) + 0.5))


@pytest.mark.parametrize("M,N", [(2, 256), (5, 1536)])
def test_q4k_roundtrip_and_layout(M, N):
    rng = np.random.default_rng(M + N)
    w = (rng.standard_normal((M, N)) * 0.05 + 0.01).astype(np.float32)
    q, meta = quant.quantize_q4k(w)
    assert q.dtype == np.uint32 and q.size == M * N // 8 and meta.shape == (M, N // 256, 16)
    deq = quant.dequantize_q4k(q, meta, M, N)
    m16 = meta.view(np.float16).astype(np.float64)
    scale = np.repeat(m16[..., :8], 32, axis=2).reshape(M, N)
    mn = np.repeat(m16[..., 8:], 32, axis=2).reshape(M, N)
    assert np.all(np.abs(deq - w) <= 0.5 * scale * (1 + 2.0**-9) + 15 * scale * 2.0**-10 + np.abs(mn) * 2.0**-9
                  + 1e-7)
    # nibble (m N + k) % 8 of word (m N + k) / 8
    m, k = M - 1, 37
    fi = m * N + k
    nib = (int(q[fi >> 3]) >> (4 * (fi & 7))) & 0xF
    sub = w[m, 32:64].astype(np.float64)
    sc = (sub.max() - sub.min()) / 15.0
    assert nib == min(15, max(0, int(np.floor((w[m, k] - sub.min()) / sc + 0.5))))


def _ref64(x, deq):
    return deq.astype(np.float64) @ x.astype(np.float64)


@pytest.mark.parametrize("fmt,M,N", [(0, 9, 1536), (0, 4, 100), (1, 9, 1536), (1, 3, 544), (2, 6, 1536),
                                     (2, 2, 256)])
def test_oracle_matmul_against_float64(oracle, fmt, M, N):
    rng = np.random.default_rng(fmt * 1000 + N)
    x = rng.standard_normal(N).astype(np.float32)
    w = (rng.standard_normal((M, N)) * 0.05).astype(np.float32)
    if fmt == 0:
        wq = w.astype(np.float16).view(np.uint16)
        sc = None
        deq = wq.view(np.float16).astype(np.float32)
    elif fmt == 1:
        wq, sc = quant.quantize_q8(w)
        deq = quant.dequantize_q8(wq, sc, M, N)
    else:
        wq, sc = quant.quantize_q4k(w)
        deq = quant.dequantize_q4k(wq, sc, M, N)
    got = oracle.matmul(fmt, x, wq, sc, M, N)
    ref = _ref64(x, deq)
    scale = np.abs(deq).astype(np.float64) @ np.abs(x).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * scale + 1e-6)


def test_oracle_matmul_order_is_the_workgroup_tree(oracle):
    """The f16 restatement's bits equal an explicit transcription of matmul_quant.wgsl:29-52."""
    rng = np.random.default_rng(3)
    M, N = 3, 700
    x = rng.standard_normal(N).astype(np.float32)
    w = rng.standard_normal((M, N)).astype(np.float16)
    got = oracle.matmul(0, x, w.view(np.uint16), None, M, N)
    for m in range(M):
        p = np.zeros(256, dtype=np.float32)
        for t in range(256):
            acc = np.float32(0.0)
            for k in range(t, N, 256):
                acc = np.float32(acc + np.float32(np.float32(w[m, k]) * x[k]))
            p[t] = acc
        st = 128
        while st:
            p[:st] = (p[:st] + p[st:2 * st]).astype(np.float32)
            st >>= 1
        assert np.float32(p[0]).view(np.uint32) == np.float32(got[m]).view(np.uint32)
