"""The CUDA path against HF transformers' Gemma 4 attention, through the C ABI.

Same fixtures and bars as tests/test_hf_parity.py (HF Gemma4TextAttention, fp32 eager, a sliding
layer at head_dim 256 and a global layer at head_dim 512 with proportional RoPE), here for the
kernels: the producer kernels (norm+RoPE, v_norm, f16 store), the split-KV decode on HF's own q
and f16 cache, the whole decode layer entry (g4a_attn_decode_layer: producers and attention in
one call), and the prefill kernels (tcgen05 at head_dim 256, the head_dim 512 kernel) over the
whole prompt.  Attention tolerance: max abs <= 2e-3, per-head cosine >= 0.9999 on the same f16
cache; against HF's fp32-cache forward: per-head cosine >= 0.99999, max abs <= 2e-2.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import assert_attention_close, dev, host
from hf_fixture import EPS, NAMES, Fixture

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=NAMES)
def fx(request):
    f = Fixture(request.param)
    assert f.inputs_match()
    return f


def _weights(f):
    qw = dev(f.q_w16.view(np.uint16)).view(torch.float16)
    kw = dev(f.k_w16.view(np.uint16)).view(torch.float16)
    rf = dev(f.rope_freqs.view(np.uint16)).view(torch.float16) if f.rope_freqs is not None else None
    return qw, kw, rf


def _prep_all(ctx, f):
    """Producer kernels over the whole prompt: q16 [T, 8, hd] and the f16 caches [T, 1, hd]."""
    qw, kw, rf = _weights(f)
    T, hd = f.T, f.hd
    q16 = torch.zeros((T, 8, hd), dtype=torch.float16, device="cuda")
    kc = torch.zeros((T, 1, hd), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    ctx.prefill_qkv_prep(dev(f.inp["q"]), dev(f.inp["k"][:, None]), dev(f.inp["v"][:, None]), qw, kw, rf, q16, kc, vc,
                         T=T, start_pos=0, max_seq_len=T, num_q_heads=8, num_kv_heads=1, head_dim=hd, eps=EPS,
                         theta=f.theta, apply_divisor=f.apply_divisor)
    ctx.sync()
    return q16, kc, vc


def test_producer_kernels_match_hf(ctx, fx):
    qw, kw, rf = _weights(fx)
    for n, p in enumerate(fx.rows):
        q = dev(fx.inp["q"][p].reshape(-1))
        ctx.norm_rope(q, qw, rf, num_heads=8, head_dim=fx.hd, eps=EPS, position=p, theta=fx.theta,
                      apply_divisor=fx.apply_divisor)
        got = host(q).reshape(8, fx.hd)
        assert np.abs(got - fx.d["q_rot"][n]).max() <= 1e-4, p
    _, kc, vc = _prep_all(ctx, fx)
    hk, hv = fx.hf_cache()
    for ours, hf in ((host(kc), hk), (host(vc), hv)):
        d = ours.view(np.uint16).astype(np.int32) - hf.astype(np.int32)
        assert np.abs(d).max() <= 2
        assert np.count_nonzero(d) <= d.size // 1000


def test_decode_on_hf_cache_matches_hf(ctx, fx):
    hk, hv = fx.hf_cache()
    kc = dev(hk.view(np.float16))
    vc = dev(hv.view(np.float16))
    for n, p in enumerate(fx.rows):
        out = torch.full((8, fx.hd), float("nan"), device="cuda")
        ctx.decode_attn(dev(fx.d["q_rot"][n]), kc, vc, out, num_q_heads=8, num_kv_heads=1, head_dim=fx.hd,
                        seq_len=p + 1, sliding_window=fx.W)
        ctx.sync()
        assert_attention_close(host(out), fx.d["attn_k16"][n].astype(np.float64), what=f"{fx.name} row {p}")


def test_decode_layer_entry_matches_hf_forward(ctx, fx):
    """g4a_attn_decode_layer for the token at each tested row: it norms and ropes the token's q
    and k, normalises v, stores k / v at slot p of a cache that holds rows 0..p-1 from the
    producer kernels, and attends over rows 0..p (the engine's per-token dispatch order)."""
    qw, kw, rf = _weights(fx)
    _, kc_all, vc_all = _prep_all(ctx, fx)
    for n, p in enumerate(fx.rows):
        kc = kc_all.clone()
        vc = vc_all.clone()
        kc[p:] = 0
        vc[p:] = 0
        q = dev(fx.inp["q"][p].reshape(-1))
        k = dev(fx.inp["k"][p])
        v = dev(fx.inp["v"][p])
        out = torch.full((8, fx.hd), float("nan"), device="cuda")
        ctx.attn_decode_layer(q, k, v, qw, kw, rf, kc, vc, out, num_q_heads=8, num_kv_heads=1, head_dim=fx.hd,
                              eps=EPS, position=p, slot=p, kv_len=p + 1, max_seq_len=fx.T, theta=fx.theta,
                              apply_divisor=fx.apply_divisor, sliding_window=fx.W)
        ctx.sync()
        assert_attention_close(host(out), fx.d["attn_fp32"][n].reshape(8, fx.hd).astype(np.float64), max_abs=2e-2,
                               cos=0.99999, what=f"{fx.name} layer row {p}")
        assert_attention_close(host(out), fx.d["attn_k16"][n].astype(np.float64), max_abs=2e-3,
                               what=f"{fx.name} layer row {p} vs HF on the f16 cache")


def test_prefill_matches_hf(ctx, fx):
    q16, kc, vc = _prep_all(ctx, fx)
    out = torch.full((fx.T, 8, fx.hd), float("nan"), device="cuda")
    ctx.prefill_attn(q16, kc, vc, out, T=fx.T, start_pos=0, num_q_heads=8, num_kv_heads=1, head_dim=fx.hd,
                     sliding_window=fx.W)
    ctx.sync()
    got = host(out)
    assert np.isfinite(got).all()
    for n, p in enumerate(fx.prefill_rows):
        assert_attention_close(got[p], fx.d["attn_prefill"][n].astype(np.float64), what=f"{fx.name} prefill row {p}")
