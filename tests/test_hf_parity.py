"""The oracle against HF transformers' Gemma 4 attention (the reference's own ground truth).

The reference checks its engine against HF transformers' Gemma 4 forward, captured with module
hooks (reference/pytorch/probe_layer0.py:88-116).  The fixtures hold HF's Gemma4TextAttention
(transformers 5.5.0, fp32, eager) on seeded inputs for a sliding layer (head_dim 256, theta
1e4, window 512, rows 14 / 511 / 512 / 513 / 700) and a global layer (head_dim 512, theta 1e6,
proportional RoPE = the rope_freqs divisor, rows 14 / 255 / 256 / 399).  Bars:
  - mask: the keys HF's mask allows for each row are exactly [kv_len - W, kv_len) of
    attn_score.wgsl:23-30 (no off-by-one between HF and the WGSL window);
  - producers (fused_per_head_norm_rope.wgsl, per_head_rms_norm_no_weight.wgsl): post-RoPE q / k
    and v_norm within 1e-4 abs; the f16 caches differ from HF's by at most 2 f16 ulps on at
    most 0.1% of the elements (f32 rounding of the RoPE angle, then round-to-nearest f16);
  - attention over the same f16 cache: max abs <= 2e-3 and per-head cosine >= 0.9999 (measured
    ~2e-5 and 1.0), fp64 oracle and the WGSL-order f32 chain;
  - the whole chain from the raw projections (our producers, f16 cache, attention) against HF's
    fp32 forward, which keeps K / V in f32: per-head cosine >= 0.99999 and max abs <= 2e-2; the
    gap is the f16 rounding of the cache (the reference keeps f32 caches, src/engine.ts:1420).
"""
import numpy as np
import pytest

from g4attn.crosslab import attention_parity, head_cosines
from hf_fixture import EPS, NAMES, Fixture


@pytest.fixture(scope="module", params=NAMES)
def fx(request):
    return Fixture(request.param)


def _oracle_producers(orc, f, p):
    q = orc.norm_rope(f.inp["q"][p].reshape(-1), f.q_w16, f.rope_freqs, num_heads=8, head_dim=f.hd, eps=EPS,
                      position=p, theta=f.theta, apply_divisor=f.apply_divisor).reshape(8, f.hd)
    k = orc.norm_rope(f.inp["k"][p], f.k_w16, f.rope_freqs, num_heads=1, head_dim=f.hd, eps=EPS, position=p,
                      theta=f.theta, apply_divisor=f.apply_divisor)
    v = orc.rms_norm_no_weight(f.inp["v"][p], num_heads=1, head_dim=f.hd, eps=EPS)
    return q, k, v


def test_fixture_inputs_are_the_generated_ones(fx):
    assert fx.inputs_match(), "numpy's generator no longer reproduces the fixture inputs"


def test_window_matches_hf_mask(fx, oracle):
    for n, p in enumerate(fx.rows):
        L = p + 1
        assert oracle.window_start(L, fx.W) == int(fx.d["mask_lo"][n]), (p, fx.W)
        assert L - 1 == int(fx.d["mask_hi"][n])


def test_producers_match_hf(fx, oracle):
    for n, p in enumerate(fx.rows):
        q, k, v = _oracle_producers(oracle, fx, p)
        assert np.abs(q - fx.d["q_rot"][n]).max() <= 1e-4, p
        assert head_cosines(q, fx.d["q_rot"][n]).min() >= 0.999999, p
        assert np.abs(k - fx.d["k_rot"][n]).max() <= 1e-4, p
        assert np.abs(v - fx.d["v_norm"][n]).max() <= 1e-5, p


def test_f16_cache_matches_hf(fx, oracle):
    kc, vc = oracle.build_cache(fx.inp["k"][:, None], fx.inp["v"][:, None], fx.k_w16, theta=fx.theta,
                                apply_divisor=fx.apply_divisor, rope_freqs=fx.rope_freqs)
    hk, hv = fx.hf_cache()
    for ours, hf in ((kc, hk), (vc, hv)):
        d = ours.view(np.uint16).astype(np.int32) - hf.astype(np.int32)
        assert np.abs(d).max() <= 2
        assert np.count_nonzero(d) <= d.size // 1000


def test_attention_on_hf_cache_matches_hf(fx, oracle):
    hk, hv = fx.hf_cache()
    kf, vf = oracle.f16_to_f32(hk), oracle.f16_to_f32(hv)
    for n, p in enumerate(fx.rows):
        ref = fx.d["attn_k16"][n].astype(np.float64)
        o64 = oracle.decode_attn_f64(fx.d["q_rot"][n], hk, hv, num_q_heads=8, num_kv_heads=1, head_dim=fx.hd,
                                     kv_len=p + 1, sliding_window=fx.W)
        r = attention_parity(o64, ref)
        assert r["ok"] and r["max_abs"] <= 1e-4, (p, r)
        o32 = oracle.decode_chain_f32(fx.d["q_rot"][n], kf[:p + 1], vf[:p + 1], num_q_heads=8, num_kv_heads=1,
                                      head_dim=fx.hd, seq_len=p + 1, sliding_window=fx.W)
        r = attention_parity(o32, ref)
        assert r["ok"] and r["max_abs"] <= 1e-4, (p, r)


def test_prefill_rows_match_hf(fx, oracle):
    """Row i of a prompt prefill = decode at kv_len i + 1 over q rounded to f16 (the prefill
    kernels' input), against HF's eager attention on the same f16 q and cache."""
    kc, vc = oracle.build_cache(fx.inp["k"][:, None], fx.inp["v"][:, None], fx.k_w16, theta=fx.theta,
                                apply_divisor=fx.apply_divisor, rope_freqs=fx.rope_freqs)
    for n, p in enumerate(fx.prefill_rows):
        q, _, _ = _oracle_producers(oracle, fx, p)
        q16 = oracle.f16_to_f32(oracle.f32_to_f16(q))
        o = oracle.decode_attn_f64(q16, kc, vc, num_q_heads=8, num_kv_heads=1, head_dim=fx.hd, kv_len=p + 1,
                                   sliding_window=fx.W)
        r = attention_parity(o, fx.d["attn_prefill"][n].astype(np.float64))
        assert r["ok"], (p, r)


def test_whole_chain_matches_hf_fp32_forward(fx, oracle):
    kc, vc = oracle.build_cache(fx.inp["k"][:, None], fx.inp["v"][:, None], fx.k_w16, theta=fx.theta,
                                apply_divisor=fx.apply_divisor, rope_freqs=fx.rope_freqs)
    for n, p in enumerate(fx.rows):
        q, _, _ = _oracle_producers(oracle, fx, p)
        o = oracle.decode_attn_f64(q, kc, vc, num_q_heads=8, num_kv_heads=1, head_dim=fx.hd, kv_len=p + 1,
                                   sliding_window=fx.W)
        r = attention_parity(o, fx.d["attn_fp32"][n].astype(np.float64), max_abs_tol=2e-2, cos_tol=0.99999)
        assert r["ok"], (p, r)
