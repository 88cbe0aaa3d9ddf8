"""Decode attention (g4a_decode_attn) against the fp64 oracle: max |diff| <= 2e-3 and per-head
cosine >= 0.9999, exact sliding-window masking, GQA mapping, zero length, determinism."""
import numpy as np
import pytest
import torch

from g4attn import G4AError, synth
from gpu_helpers import EPS, assert_attention_close, dev, gpu_build_cache, host

pytestmark = pytest.mark.gpu


def _layer(ctx, oracle, L, hd=256, theta=1e4, window=0, seed=0, nqh=8, nkh=1):
    """Cache for positions 0..L-1 built by the producer kernels, and the normed+roped q at L-1."""
    raw = synth.raw_layer(seed, max(L, 1), nqh=nqh, nkh=nkh, hd=hd, theta=theta, window=window)
    kc, vc = gpu_build_cache(ctx, raw.k, raw.v, raw.k_w, theta=theta)
    q = oracle.norm_rope(raw.q[0], raw.q_w, None, num_heads=nqh, head_dim=hd, eps=EPS, position=max(L - 1, 0),
                         theta=theta)
    return q, kc, vc


def _run(ctx, q, kc, vc, L, hd, window, nqh=8, nkh=1, scale=1.0):
    out = torch.full((nqh, hd), float("nan"), device="cuda")
    ctx.decode_attn(dev(q), kc, vc, out, num_q_heads=nqh, num_kv_heads=nkh, head_dim=hd, seq_len=L, scale=scale,
                    sliding_window=window)
    ctx.sync()
    return host(out)


def test_config0_sliding_decode(ctx, oracle):
    """L=512 cache, q at position 511, theta 1e4, window 512, seed 0."""
    q, kc, vc = _layer(ctx, oracle, 512, theta=1e4, window=512, seed=0)
    ours = _run(ctx, q, kc, vc, 512, 256, 512)
    k, v = host(kc), host(vc)
    ref = oracle.decode_attn_f64(q, k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=512,
                                 sliding_window=512)
    assert_attention_close(ours, ref, what="config0 vs fp64")
    wgsl = oracle.decode_chain_f32(q, k.astype(np.float32), v.astype(np.float32), num_q_heads=8, num_kv_heads=1,
                                   head_dim=256, seq_len=512, sliding_window=512)
    assert_attention_close(ours, wgsl, what="config0 vs WGSL-order f32 chain")


@pytest.mark.parametrize("L", [1, 2, 3, 31, 32, 33, 63, 64, 65, 100, 511, 512, 513, 1000, 4097])
@pytest.mark.parametrize("W", [0, 512, 16])
def test_decode_lengths_and_windows(ctx, oracle, L, W):
    q, kc, vc = _layer(ctx, oracle, L, theta=1e4 if W else 1e6, window=W, seed=L)
    ours = _run(ctx, q, kc, vc, L, 256, W)
    ref = oracle.decode_attn_f64(q, host(kc), host(vc), num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=L,
                                 sliding_window=W)
    assert_attention_close(ours, ref, what=f"L={L} W={W}")


@pytest.mark.parametrize("hd", [128, 512])
@pytest.mark.parametrize("L,W", [(1, 0), (77, 0), (700, 512), (3000, 0)])
def test_decode_head_dims(ctx, oracle, hd, L, W):
    q, kc, vc = _layer(ctx, oracle, L, hd=hd, theta=1e6, window=W, seed=hd + L)
    ours = _run(ctx, q, kc, vc, L, hd, W)
    ref = oracle.decode_attn_f64(q, host(kc), host(vc), num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L,
                                 sliding_window=W)
    assert_attention_close(ours, ref, what=f"hd={hd} L={L} W={W}")


@pytest.mark.parametrize("L", [4096, 32768, 131072])
def test_config1_global_decode(ctx, oracle, L):
    """global layer, theta 1e6, no window, q at the true position."""
    q, kc, vc = _layer(ctx, oracle, L, theta=1e6, window=0, seed=1)
    ours = _run(ctx, q, kc, vc, L, 256, 0)
    ref = oracle.decode_attn_f64(q, host(kc), host(vc), num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=L)
    assert_attention_close(ours, ref, what=f"config1 L={L}")


def test_zero_length_gives_zeros(ctx):
    kc = torch.zeros((4, 1, 256), dtype=torch.float16, device="cuda")
    ours = _run(ctx, np.ones((8, 256), np.float32), kc, kc, 0, 256, 0)
    assert not ours.any()


@pytest.mark.parametrize("L,W", [(700, 512), (2049, 100), (300, 0)])
def test_mask_is_exact(ctx, oracle, L, W):
    """Rows before max(0, L-W) and rows >= L are never read: poisoning them with NaN/Inf leaves
    the output bit-identical."""
    q, kc, vc = _layer(ctx, oracle, L, window=W, seed=5)
    cap = L + 40
    k2 = torch.full((cap, 1, 256), float("nan"), dtype=torch.float16, device="cuda")
    v2 = torch.full_like(k2, float("inf"))
    ws = max(L - W, 0) if W else 0
    k2[ws:L] = kc[ws:L]
    v2[ws:L] = vc[ws:L]
    clean = _run(ctx, q, kc, vc, L, 256, W)
    poisoned = _run(ctx, q, k2, v2, L, 256, W)
    assert np.array_equal(clean.view(np.uint32), poisoned.view(np.uint32))


def test_deterministic(ctx, oracle):
    q, kc, vc = _layer(ctx, oracle, 20000, theta=1e6, seed=9)
    a = _run(ctx, q, kc, vc, 20000, 256, 0)
    b = _run(ctx, q, kc, vc, 20000, 256, 0)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_scale_parameter(ctx, oracle):
    q, kc, vc = _layer(ctx, oracle, 900, seed=4)
    ours = _run(ctx, q, kc, vc, 900, 256, 0, scale=1.0 / 16)
    ref = oracle.decode_attn_f64(q, host(kc), host(vc), num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=900,
                                 scale=1.0 / 16)
    assert_attention_close(ours, ref, what="scale 1/16")


@pytest.mark.parametrize("nqh,nkh,hd", [(16, 2, 128), (8, 1, 96), (4, 1, 64), (6, 3, 80), (16, 2, 256)])
def test_gqa_and_generic_shapes(ctx, oracle, nqh, nkh, hd):
    """kv head of q head h is h*NKH/NQH; shapes off the 8:1 fast path run the generic kernel."""
    L = 777
    rng = np.random.default_rng(nqh * 100 + hd)
    q = rng.standard_normal((nqh, hd)).astype(np.float32)
    q /= np.sqrt((q * q).mean(-1, keepdims=True))
    k = oracle.f32_to_f16(rng.standard_normal((L, nkh, hd)).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal((L, nkh, hd)).astype(np.float32))
    kd = dev(k.view(np.uint16)).view(torch.float16)
    vd = dev(v.view(np.uint16)).view(torch.float16)
    for W in (0, 300):
        ours = _run(ctx, q, kd, vd, L, hd, W, nqh=nqh, nkh=nkh)
        ref = oracle.decode_attn_f64(q, k, v, num_q_heads=nqh, num_kv_heads=nkh, head_dim=hd, kv_len=L,
                                     sliding_window=W)
        assert_attention_close(ours, ref, what=f"nqh={nqh} nkh={nkh} hd={hd} W={W}")


def test_bad_arguments_are_rejected(ctx):
    kc = torch.zeros((64, 1, 256), dtype=torch.float16, device="cuda")
    q = torch.zeros(8 * 256 + 1, device="cuda")
    out = torch.zeros(8 * 256, device="cuda")
    from g4attn._lib import call
    from g4attn import _ptr

    with pytest.raises(G4AError) as ei:  # q misaligned by 4 bytes
        call("g4a_decode_attn", ctx.handle, _ptr(q.data_ptr() + 4), _ptr(kc), _ptr(kc), _ptr(out), 8, 1, 256, 10,
             1.0, 0)
    assert ei.value.status_name == "G4A_EINVAL"
    with pytest.raises(G4AError):  # head_dim not a multiple of 8
        call("g4a_decode_attn", ctx.handle, _ptr(q), _ptr(kc), _ptr(kc), _ptr(out), 8, 1, 100, 10, 1.0, 0)
    with pytest.raises(G4AError):  # nkh > nqh
        call("g4a_decode_attn", ctx.handle, _ptr(q), _ptr(kc), _ptr(kc), _ptr(out), 1, 2, 256, 10, 1.0, 0)
    with pytest.raises(G4AError):  # slot beyond the cache
        ctx.kv_store(out[:256], out[:256], kc, kc, num_kv_heads=1, head_dim=256, position=64, max_seq_len=64)
    ctx.sync()
