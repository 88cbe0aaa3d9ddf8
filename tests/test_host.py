"""Host-side logic: Gemma layer rules, the synthetic recipe, sharding and the crossLabDiff report."""
import numpy as np

from g4attn import dist, synth
from g4attn.crosslab import attention_parity, cross_lab_diff
from g4attn.gemma import GemmaAttnConfig, gemma_rope_freqs, ring_slot_and_len


def test_gemma_layer_pattern():
    c = GemmaAttnConfig()
    globals_ = [i for i in range(35) if not c.is_swa_layer(i)]
    assert globals_ == [4, 9, 14, 19, 24, 29, 34]
    assert c.head_dim(0) == 256 and c.head_dim(4) == 512
    assert c.rope_theta(0) == 1e4 and c.rope_theta(4) == 1e6
    assert c.window(0) == 512 and c.window(4) == 0
    assert c.apply_divisor(0) == 0 and c.apply_divisor(4) == 1
    assert c.attn_scale(3) == 1.0


def test_kv_producer_map():
    c = GemmaAttnConfig()
    m = c.kv_producer_for_layer()
    assert m[:15] == list(range(15))
    # consumers read the last unshared layer of their type: 13 (sliding) or 14 (global)
    for i in range(15, 35):
        assert m[i] == (13 if c.is_swa_layer(i) else 14)
    assert c.is_kv_producer_layer(14) and not c.is_kv_producer_layer(20)


def test_rope_freqs_table():
    t = gemma_rope_freqs(512, 64)
    assert t.dtype == np.float16 and t.shape == (256,)
    assert (t[:64] == 1).all() and np.isinf(t[64:].astype(np.float32)).all()


def test_ring_mapping():
    # before the ring is active: slot == position, kv_len == seq_len
    assert ring_slot_and_len(10, 11, None, 0) == (10, 11)
    assert ring_slot_and_len(10, 11, 8, 4) == (10, 11)
    # after wrap: slot cycles in [P, P + W), kv_len capped at P + W
    assert ring_slot_and_len(13, 14, 8, 4) == (9, 12)
    assert ring_slot_and_len(16, 17, 8, 4) == (8, 12)


def test_synth_is_seeded():
    a = synth.raw_layer(0, 16)
    b = synth.raw_layer(0, 16)
    assert np.array_equal(a.k, b.k) and np.array_equal(a.q_w, b.q_w)
    assert not np.array_equal(synth.raw_layer(1, 16).k, a.k)
    L = synth.batched_lengths(2, 64)
    assert L.min() >= 1024 and L.max() <= 32768 and len(L) == 64
    assert np.array_equal(L, synth.batched_lengths(2, 64))


def test_page_assignment_is_a_permutation():
    L = np.array([1, 64, 65, 1000, 0], dtype=np.int32)
    table, npages = synth.page_assignment(2, L, 64)
    used = []
    for b, n in enumerate((L + 63) // 64):
        used += list(table[b, :n])
    assert sorted(used) == list(range(npages))


def test_work_figures():
    assert synth.kv_bytes_decode(512, 512) == 540_672
    assert synth.kv_bytes_decode(32768, 0) == 33_570_816
    assert synth.prefill_flops(4096, 0) == 68_736_253_952
    assert synth.prefill_flops(4096, 512) == 4 * 8 * 256 * 1_966_336


def test_lpt_shard_balances_and_partitions():
    L = synth.batched_lengths(2, 64)
    cost = dist.decode_cost_bytes(L)
    for n in (1, 2, 4, 8):
        bins = dist.lpt_shard(cost, n)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(64))
        loads = [cost[b].sum() for b in bins]
        assert max(loads) <= cost.sum() / n + cost.max()


def test_splitkv_ranges():
    r = dist.splitkv_ranges(1_048_576, 8)
    assert r[0][0] == 0 and r[-1][1] == 1_048_576
    assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
    assert all((e - b) == 131072 for b, e in r)
    r = dist.splitkv_ranges(100, 3)
    assert r[0][0] == 0 and r[-1][1] == 100


def test_host_merge_of_empty_parts_is_zero():
    parts = np.zeros((2, 8 * (256 + 2)), np.float32)
    parts[:, :8] = -np.inf
    assert not dist.merge_partials_host(parts, 8, 256).any()


def test_cross_lab_diff_report():
    ref = np.arange(100, dtype=np.float32)
    ours = ref.copy()
    ours[7] += 1.0
    r = cross_lab_diff(ours, ref)
    assert r["maxAbsDiff"] == 1.0 and r["firstOverIndex"] == 7 and r["overCount"] == 1
    assert r["concentration"]["top1PctFraction"] == 1.0
    p = attention_parity(ref.reshape(4, 25), ref.reshape(4, 25))
    assert p["ok"] and p["max_abs"] == 0.0
    assert not attention_parity(ours.reshape(4, 25), ref.reshape(4, 25))["ok"]
