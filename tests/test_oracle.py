"""CPU tests of the oracle: pinned against the reference's own golden data and an independent
numpy restatement.  No GPU needed."""
from pathlib import Path

import numpy as np
import pytest

from g4attn import synth
from g4attn.crosslab import attention_parity, cross_lab_diff, head_cosines
from g4attn.gemma import gemma_rope_freqs

GOLDEN = Path(__file__).resolve().parent / "golden" / "vnorm_layer0.npz"


def test_f16_roundtrip_all_halves(oracle):
    h = np.arange(65536, dtype=np.uint16).view(np.float16)
    f = oracle.f16_to_f32(h)
    ref = h.astype(np.float32)
    same = (f == ref) | (np.isnan(f) & np.isnan(ref))
    assert same.all()


def test_f32_to_f16_round_nearest_even(oracle):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(200000) * np.float32(300)).astype(np.float32)
    edge = np.array([65504, 65519.99, 65520, -65520, 6e-8, 3e-8, 2.98e-8, 1e-5, 0.0, -0.0, np.inf, -np.inf],
                    dtype=np.float32)
    x = np.concatenate([x, edge, rng.standard_normal(1000).astype(np.float32) * np.float32(1e-6)])
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16)
    assert (oracle.f32_to_f16(x).view(np.uint16) == ref.view(np.uint16)).all()


def test_vnorm_known_answer_from_reference_fixture(oracle):
    """Weightless RMSNorm of the reference's layer-0 v projection equals HF's v_norm output
    (public/ref/layer_0_detail.npz, bf16 source => loose abs tolerance, tight cosine)."""
    g = np.load(GOLDEN)
    v = g["v_proj"].reshape(1, 256)
    ours = oracle.rms_norm_no_weight(v, num_heads=1, head_dim=256, eps=1e-6).reshape(-1)
    rep = cross_lab_diff(ours, g["v_norm"])
    assert rep["cosineSimilarity"] > 0.99999
    assert rep["maxAbsDiff"] < 1e-2
    assert abs(np.sqrt(np.mean(ours.astype(np.float64) ** 2)) - 1.0) < 1e-5


def test_golden_q_norm_is_rmsnorm_times_shared_weight(oracle):
    """q_norm outputs of the fixture are per-head RMSNorm * one shared weight: dividing them by
    the weightless norm of the q projection gives the same per-dim ratio for all 8 heads."""
    g = np.load(GOLDEN)
    qp = g["q_proj"].reshape(8, 256)
    qn = g["q_norm"].reshape(8, 256)
    normed = oracle.rms_norm_no_weight(qp, num_heads=8, head_dim=256, eps=1e-6)
    ratio = qn / np.where(np.abs(normed) > 1e-2, normed, np.nan)
    med = np.nanmedian(ratio, axis=0)
    spread = np.nanmedian(np.abs(ratio - med[None]), axis=0)
    assert np.nanmedian(spread / np.abs(med)) < 0.02


def test_rope_base_freq_definition(oracle):
    for theta in (1e4, 1e6):
        for hd in (256, 512):
            for i in range(hd // 2):
                e = np.float32(2 * i) / np.float32(hd)
                p = np.float32(np.float64(theta) ** np.float64(e))
                assert oracle.rope_base_freq(theta, i, hd) == np.float32(1.0) / p


def _np_norm_rope(x, w, pos, theta, rf=None, eps=1e-6):
    x = x.astype(np.float64)
    hd = x.shape[-1]
    rms = np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    y = x * w.astype(np.float64) / rms
    half = hd // 2
    i = np.arange(half)
    freq = 1.0 / theta ** (2 * i / hd)
    if rf is not None:
        freq = freq / rf.astype(np.float64)
    ang = pos * freq
    c, s = np.cos(ang), np.sin(ang)
    out = y.copy()
    out[..., :half] = y[..., :half] * c - y[..., half:] * s
    out[..., half:] = y[..., :half] * s + y[..., half:] * c
    return out


@pytest.mark.parametrize("hd,pos,theta", [(256, 0, 1e4), (256, 511, 1e4), (512, 4095, 1e6), (256, 17, 1e6)])
def test_norm_rope_matches_float64_math(oracle, hd, pos, theta):
    rng = np.random.default_rng(hd + pos)
    x = rng.standard_normal((8, hd)).astype(np.float32)
    w = synth.norm_weight(rng, hd)
    ours = oracle.norm_rope(x, w, None, num_heads=8, head_dim=hd, eps=1e-6, position=pos, theta=theta)
    ref = _np_norm_rope(x, w, pos, theta)
    # the reference rounds angle = f32(pos) * freq to f32: error up to ~ulp(pos) radians
    tol = 2e-5 + 2.0 * np.spacing(np.float32(max(pos, 1))) * np.abs(ref).max()
    assert np.abs(ours - ref).max() < tol


def test_norm_rope_divisor_table_leaves_trailing_pairs_unrotated(oracle):
    rng = np.random.default_rng(3)
    hd = 512
    x = rng.standard_normal((1, hd)).astype(np.float32)
    w = synth.norm_weight(rng, hd)
    rf = gemma_rope_freqs(hd, 64)
    assert np.isinf(rf[64:].astype(np.float32)).all()
    a = oracle.norm_rope(x, w, rf, num_heads=1, head_dim=hd, eps=1e-6, position=1000, theta=1e6, apply_divisor=1)
    plain = oracle.norm_rope(x, w, None, num_heads=1, head_dim=hd, eps=1e-6, position=0, theta=1e6)
    assert np.array_equal(a[0, 64:256], plain[0, 64:256])
    assert np.array_equal(a[0, 256 + 64:], plain[0, 256 + 64:])
    assert not np.array_equal(a[0, :64], plain[0, :64])


@pytest.mark.parametrize("L,W", [(1, 0), (37, 0), (300, 0), (100, 512), (512, 512), (513, 512), (700, 512),
                                 (64, 16)])
def test_chain_orders_agree(oracle, L, W):
    """The WGSL-order f32 chain, the fp64 golden and the numpy twin agree on the same f16 cache."""
    rng = np.random.default_rng(L * 7 + W)
    hd = 256
    q = rng.standard_normal((8, hd)).astype(np.float32)
    q /= np.sqrt((q * q).mean(-1, keepdims=True))
    k = oracle.f32_to_f16(rng.standard_normal((L, 1, hd)).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal((L, 1, hd)).astype(np.float32))
    f64 = oracle.decode_attn_f64(q, k, v, num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L, sliding_window=W)
    f32 = oracle.decode_chain_f32(q, oracle.f16_to_f32(k), oracle.f16_to_f32(v), num_q_heads=8, num_kv_heads=1,
                                  head_dim=hd, seq_len=L, sliding_window=W)
    tw = oracle.decode_numpy_f64(q, k.astype(np.float32), v.astype(np.float32), L, W)
    assert attention_parity(f32, f64)["ok"]
    assert np.abs(tw - f64).max() < 1e-5


def test_window_mask_is_exact_in_oracle(oracle):
    """Keys before max(0, L-W) never influence the output: poison them with inf/nan."""
    rng = np.random.default_rng(11)
    L, W, hd = 700, 512, 256
    q = rng.standard_normal((8, hd)).astype(np.float32)
    k = oracle.f32_to_f16(rng.standard_normal((L, 1, hd)).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal((L, 1, hd)).astype(np.float32))
    a = oracle.decode_attn_f64(q, k, v, num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L, sliding_window=W)
    k2, v2 = k.copy(), v.copy()
    k2[: L - W] = np.float16(np.inf)
    v2[: L - W] = np.float16(np.nan)
    b = oracle.decode_attn_f64(q, k2, v2, num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L, sliding_window=W)
    assert np.array_equal(a, b)
    assert oracle.window_start(L, W) == L - W
    assert oracle.window_start(W, W) == 0
    assert oracle.window_start(W + 1, W) == 1
    assert oracle.window_start(0, W) == 0


def test_zero_length_gives_zeros(oracle):
    q = np.ones((8, 256), np.float32)
    k = np.zeros((1, 1, 256), np.float16)
    out = oracle.decode_attn_f64(q, k, k, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=0)
    assert not out.any()
    out2 = oracle.decode_chain_f32(q, k.astype(np.float32), k.astype(np.float32), num_q_heads=8, num_kv_heads=1,
                                   head_dim=256, seq_len=0)
    assert not out2.any()


def test_gqa_mapping_in_oracle(oracle):
    """kv head of q head h is h*NKH/NQH (attn_score.wgsl:31): with 16 q heads and 2 kv heads,
    heads 0-7 read kv head 0 and heads 8-15 kv head 1."""
    rng = np.random.default_rng(9)
    L, hd = 50, 128
    q = rng.standard_normal((16, hd)).astype(np.float32)
    k = oracle.f32_to_f16(rng.standard_normal((L, 2, hd)).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal((L, 2, hd)).astype(np.float32))
    full = oracle.decode_attn_f64(q, k, v, num_q_heads=16, num_kv_heads=2, head_dim=hd, kv_len=L)
    tw = oracle.decode_numpy_f64(q, k.astype(np.float32), v.astype(np.float32), L, 0, nkh=2)
    assert np.abs(full - tw).max() < 1e-5
    lo = oracle.decode_attn_f64(q[:8], np.ascontiguousarray(k[:, :1]), np.ascontiguousarray(v[:, :1]),
                                num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L)
    assert np.abs(full[:8] - lo).max() < 1e-6


def test_partials_merge_to_full(oracle):
    from g4attn.dist import merge_partials_host, splitkv_ranges

    rng = np.random.default_rng(21)
    L, hd = 1000, 256
    q = rng.standard_normal((8, hd)).astype(np.float32)
    q /= np.sqrt((q * q).mean(-1, keepdims=True))
    k = oracle.f32_to_f16(rng.standard_normal((L, 1, hd)).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal((L, 1, hd)).astype(np.float32))
    full = oracle.decode_attn_f64(q, k, v, num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L)
    for n in (1, 2, 3, 8):
        parts = []
        for (b, e) in splitkv_ranges(L, n):
            m, l_, o = oracle.decode_partial_f64(q, k, v, num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_begin=b,
                                                 kv_end=e, kv_len=L)
            # natural -> base-2 units, as the GPU partial format stores them
            m2, o2, l2 = m / np.log(2.0), o, l_
            parts.append(np.concatenate([m2, l2, o2.reshape(-1)]))
        merged = merge_partials_host(np.stack(parts), 8, hd)
        assert np.abs(merged - full).max() < 1e-5


def test_prefill_row_is_decode_at_prefix(oracle):
    rng = np.random.default_rng(4)
    T, hd = 40, 256
    q = oracle.f16_to_f32(oracle.f32_to_f16(rng.standard_normal((T, 8, hd)).astype(np.float32)))
    k = oracle.f32_to_f16(rng.standard_normal((T, 1, hd)).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal((T, 1, hd)).astype(np.float32))
    rows = oracle.prefill_rows_f64(q, k, v, list(range(T)), start_pos=0, num_q_heads=8, num_kv_heads=1, head_dim=hd,
                                   sliding_window=16)
    k2 = k.copy()
    k2[21:] = np.float16(3.0)
    rows2 = oracle.prefill_rows_f64(q, k2, v, list(range(21)), start_pos=0, num_q_heads=8, num_kv_heads=1,
                                    head_dim=hd, sliding_window=16)
    assert np.array_equal(rows[:21], rows2)
    assert abs(head_cosines(rows[5], rows[5]).min() - 1.0) < 1e-12


def test_build_cache_is_producer_path(oracle):
    raw = synth.raw_layer(0, 8, hd=256, theta=1e4)
    kc, vc = oracle.build_cache(raw.k, raw.v, raw.k_w, theta=1e4)
    for t in (0, 7):
        kn = oracle.norm_rope(raw.k[t], raw.k_w, None, num_heads=1, head_dim=256, eps=1e-6, position=t, theta=1e4)
        assert np.array_equal(kc[t], kn.astype(np.float16))
        vn = oracle.rms_norm_no_weight(raw.v[t], num_heads=1, head_dim=256, eps=1e-6)
        assert np.array_equal(vc[t], vn.astype(np.float16))
