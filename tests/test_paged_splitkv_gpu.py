"""Batched paged decode and split-KV partials + log-sum-exp merge against the fp64 oracle."""
import numpy as np
import pytest
import torch

from g4attn import G4AError, dist, synth
from gpu_helpers import EPS, assert_attention_close, dev, gpu_build_cache, host

pytestmark = pytest.mark.gpu


def _paged_setup(ctx, oracle, lengths, page_size, theta, seed, hd=256):
    """Build each sequence's cache with the producer kernels, then scatter its rows into a
    randomly permuted page pool."""
    lengths = np.asarray(lengths, dtype=np.int32)
    table, npages = synth.page_assignment(seed, lengths, page_size, extra_pages=3)
    kp = torch.zeros((npages, page_size, 1, hd), dtype=torch.float16, device="cuda")
    vp = torch.zeros_like(kp)
    qs, caches = [], []
    for b, L in enumerate(lengths):
        raw = synth.raw_layer(seed * 1000 + b, max(int(L), 1), hd=hd, theta=theta)
        kc, vc = gpu_build_cache(ctx, raw.k, raw.v, raw.k_w, theta=theta)
        n = (int(L) + page_size - 1) // page_size
        for j in range(n):
            r0, r1 = j * page_size, min((j + 1) * page_size, int(L))
            kp[table[b, j], : r1 - r0] = kc[r0:r1]
            vp[table[b, j], : r1 - r0] = vc[r0:r1]
        qs.append(oracle.norm_rope(raw.q[0], raw.q_w, None, num_heads=8, head_dim=hd, eps=EPS,
                                   position=max(int(L) - 1, 0), theta=theta))
        caches.append((host(kc), host(vc)))
    return np.stack(qs), kp, vp, table, caches


@pytest.mark.parametrize("page_size", [64, 16, 128, 8, 48])
@pytest.mark.parametrize("W", [0, 512])
def test_paged_batch_matches_oracle(ctx, oracle, page_size, W):
    rng = np.random.default_rng(page_size + W)
    lengths = rng.integers(1, 3000, size=12).astype(np.int32)
    lengths[3] = 0
    lengths[5] = 1
    lengths[7] = page_size
    q, kp, vp, table, caches = _paged_setup(ctx, oracle, lengths, page_size, 1e4 if W else 1e6, seed=page_size)
    out = torch.full((len(lengths), 8, 256), float("nan"), device="cuda")
    for host_lens in (lengths, None):
        ctx.decode_attn_paged(dev(q), kp, vp, dev(table), dev(lengths), out, num_q_heads=8, num_kv_heads=1,
                              head_dim=256, page_size=page_size, sliding_window=W, host_kv_lens=host_lens)
        ctx.sync()
        ours = host(out)
        for b, L in enumerate(lengths):
            if L == 0:
                assert not ours[b].any()
                continue
            k, v = caches[b]
            ref = oracle.decode_attn_f64(q[b], k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=int(L),
                                         sliding_window=W)
            assert_attention_close(ours[b], ref, what=f"seq {b} L={L} ps={page_size} W={W}")


@pytest.mark.parametrize("W", [0, 512])
def test_paged_long_sequence_among_short(ctx, oracle, W):
    """One sequence long enough to be split over many CTAs (two-level merge) next to short and
    empty ones; run twice in a row so that the merge counters are seen to reset."""
    lengths = np.array([1, 70000, 0, 2500, 700, 64], dtype=np.int32)
    q, kp, vp, table, caches = _paged_setup(ctx, oracle, lengths, 64, 1e4 if W else 1e6, seed=21)
    for rep in range(2):
        out = torch.full((len(lengths), 8, 256), float("nan"), device="cuda")
        ctx.decode_attn_paged(dev(q), kp, vp, dev(table), dev(lengths), out, num_q_heads=8, num_kv_heads=1,
                              head_dim=256, page_size=64, sliding_window=W, host_kv_lens=lengths)
        ctx.sync()
        ours = host(out)
        for b, L in enumerate(lengths):
            if L == 0:
                assert not ours[b].any()
                continue
            k, v = caches[b]
            ref = oracle.decode_attn_f64(q[b], k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=int(L),
                                         sliding_window=W)
            assert_attention_close(ours[b], ref, what=f"rep {rep} seq {b} L={L} W={W}")


def test_config3_shape_reduced(ctx, oracle):
    """64 sequences, 64-token pages in a seeded random order, one sliding and one global layer."""
    lengths = synth.batched_lengths(2, 64, 1024, 4096)
    for W, theta in ((512, 1e4), (0, 1e6)):
        q, kp, vp, table, caches = _paged_setup(ctx, oracle, lengths, 64, theta, seed=2)
        out = torch.zeros((64, 8, 256), device="cuda")
        ctx.decode_attn_paged(dev(q), kp, vp, dev(table), dev(lengths), out, num_q_heads=8, num_kv_heads=1,
                              head_dim=256, page_size=64, sliding_window=W, host_kv_lens=lengths)
        ctx.sync()
        ours = host(out)
        for b in range(0, 64, 7):
            k, v = caches[b]
            ref = oracle.decode_attn_f64(q[b], k, v, num_q_heads=8, num_kv_heads=1, head_dim=256,
                                         kv_len=int(lengths[b]), sliding_window=W)
            assert_attention_close(ours[b], ref, what=f"config3 seq {b} W={W}")


def test_bad_page_id_is_reported_not_read(ctx, oracle):
    lengths = np.array([300, 200], dtype=np.int32)
    q, kp, vp, table, caches = _paged_setup(ctx, oracle, lengths, 64, 1e6, seed=11)
    table = table.copy()
    table[0, 2] = 10_000  # outside the pool
    out = torch.zeros((2, 8, 256), device="cuda")
    ctx.decode_attn_paged(dev(q), kp, vp, dev(table), dev(lengths), out, num_q_heads=8, num_kv_heads=1,
                          head_dim=256, page_size=64, host_kv_lens=lengths)
    with pytest.raises(G4AError) as ei:
        ctx.sync()
    assert "page id" in str(ei.value)
    ctx.sync()  # the error word is cleared; the context stays usable
    k, v = caches[1]
    ref = oracle.decode_attn_f64(q[1], k, v, num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=200)
    assert_attention_close(host(out)[1], ref, what="healthy sequence next to a bad one")


@pytest.mark.parametrize("n,align", [(1, 32), (2, 32), (3, 32), (8, 32), (3, 1), (5, 7)])
@pytest.mark.parametrize("L,W", [(5000, 0), (2000, 512), (100000, 0)])
def test_splitkv_partials_merge(ctx, oracle, n, align, L, W):
    """Emulates n ranks on one GPU: each slice's partial over its own buffer, then the merge."""
    raw = synth.raw_layer(7, L, hd=256, theta=1e6)
    kc, vc = gpu_build_cache(ctx, raw.k, raw.v, raw.k_w, theta=1e6)
    q = oracle.norm_rope(raw.q[0], raw.q_w, None, num_heads=8, head_dim=256, eps=EPS, position=L - 1, theta=1e6)
    qd = dev(q)
    pf = dist.partial_floats(8, 256)
    parts = torch.zeros((n, pf), device="cuda")
    for r, (b, e) in enumerate(dist.splitkv_ranges(L, n, align)):
        ks = kc[b:e].contiguous()
        vs = vc[b:e].contiguous()
        ctx.decode_attn_partial(qd, ks, vs, parts[r], num_q_heads=8, num_kv_heads=1, head_dim=256, kv_begin=b,
                                kv_end=e, kv_len_total=L, sliding_window=W)
    out = torch.zeros((8, 256), device="cuda")
    ctx.lse_merge(parts, n, out, num_q_heads=8, head_dim=256)
    ctx.sync()
    ref = oracle.decode_attn_f64(q, host(kc), host(vc), num_q_heads=8, num_kv_heads=1, head_dim=256, kv_len=L,
                                 sliding_window=W)
    assert_attention_close(host(out), ref, what=f"split n={n} L={L} W={W}")
    # the host restatement of the merge agrees with the kernel
    assert_attention_close(dist.merge_partials_host(host(parts), 8, 256), ref, what="host merge")
    # partial semantics: l * 2^m equals the oracle's sum of exp over the slice
    ph = host(parts)
    for r, (b, e) in enumerate(dist.splitkv_ranges(L, n, align)):
        m, l_, o = oracle.decode_partial_f64(q, host(kc), host(vc), num_q_heads=8, num_kv_heads=1, head_dim=256,
                                             kv_begin=b, kv_end=e, kv_len=L, sliding_window=W)
        mg, lg = ph[r, :8].astype(np.float64), ph[r, 8:16].astype(np.float64)
        for h in range(8):
            if not np.isfinite(m[h]):
                assert lg[h] == 0.0 and mg[h] == -np.inf
                continue
            lhs = np.log(lg[h]) + mg[h] * np.log(2.0)
            rhs = np.log(l_[h]) + m[h]
            assert abs(lhs - rhs) < 1e-4
