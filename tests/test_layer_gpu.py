"""The whole per-layer decode block (g4a_attn_decode_layer) against the oracle run in the
reference's dispatch order (src/engine.ts:2061-2094): v_norm, q/k norm+RoPE, store, attention."""
import numpy as np
import pytest
import torch

from g4attn import synth
from g4attn.gemma import GemmaAttnConfig, gemma_rope_freqs
from gpu_helpers import EPS, assert_attention_close, dev, gpu_build_cache, host, same_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layer", [0, 4])
@pytest.mark.parametrize("L", [1, 600, 5000])
def test_producer_layer_decode_step(ctx, oracle, layer, L):
    cfg = GemmaAttnConfig()
    hd, theta, W, div = cfg.head_dim(layer), cfg.rope_theta(layer), cfg.window(layer), cfg.apply_divisor(layer)
    rf = gemma_rope_freqs(512, 64) if div else None
    raw = synth.raw_layer(L + layer, L, hd=hd, theta=theta)
    max_seq = L + 8
    # history: positions 0..L-2 through the producer kernels
    kc, vc = gpu_build_cache(ctx, raw.k[: L - 1], raw.v[: L - 1], raw.k_w, theta=theta, apply_divisor=div,
                             rope_freqs=rf, max_seq=max_seq) if L > 1 else (
        torch.zeros((max_seq, 1, hd), dtype=torch.float16, device="cuda"),
        torch.zeros((max_seq, 1, hd), dtype=torch.float16, device="cuda"))
    pos = L - 1
    qd, kd, vd = dev(raw.q[0]), dev(raw.k[pos]), dev(raw.v[pos])
    f16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
    out = torch.zeros((8, hd), device="cuda")
    ctx.attn_decode_layer(qd, kd, vd, f16(raw.q_w), f16(raw.k_w), f16(rf) if rf is not None else None, kc, vc, out,
                          num_q_heads=8, num_kv_heads=1, head_dim=hd, eps=EPS, position=pos, slot=pos, kv_len=L,
                          max_seq_len=max_seq, theta=theta, apply_divisor=div, scale=cfg.attn_scale(layer),
                          sliding_window=W, is_producer=1)
    ctx.sync()
    # oracle in the reference's order
    vn = oracle.rms_norm_no_weight(raw.v[pos], num_heads=1, head_dim=hd, eps=EPS)
    qn = oracle.norm_rope(raw.q[0], raw.q_w, rf, num_heads=8, head_dim=hd, eps=EPS, position=pos, theta=theta,
                          apply_divisor=div)
    kn = oracle.norm_rope(raw.k[pos], raw.k_w, rf, num_heads=1, head_dim=hd, eps=EPS, position=pos, theta=theta,
                          apply_divisor=div)
    assert same_bits(host(qd), qn)
    assert same_bits(host(kd), kn)
    assert same_bits(host(vd), vn)
    kh, vh = host(kc), host(vc)
    assert same_bits(kh[pos], oracle.f32_to_f16(kn)) and same_bits(vh[pos], oracle.f32_to_f16(vn))
    ref = oracle.decode_attn_f64(qn, kh, vh, num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L, sliding_window=W)
    assert_attention_close(host(out), ref, what=f"layer {layer} L={L}")


def test_consumer_layer_reads_shared_cache(ctx, oracle):
    """A consumer layer (is_producer = 0) only runs q norm+RoPE and attention over the
    producer's cache, which it must not modify."""
    L, hd = 700, 256
    raw = synth.raw_layer(3, L, hd=hd, theta=1e4)
    kc, vc = gpu_build_cache(ctx, raw.k, raw.v, raw.k_w, theta=1e4)
    before = host(kc).copy()
    f16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
    qd = dev(raw.q[0])
    out = torch.zeros((8, hd), device="cuda")
    dummy = torch.zeros(hd, device="cuda")
    ctx.attn_decode_layer(qd, dummy, dummy, f16(raw.q_w), f16(raw.k_w), None, kc, vc, out, num_q_heads=8,
                          num_kv_heads=1, head_dim=hd, eps=EPS, position=L - 1, slot=L - 1, kv_len=L, max_seq_len=L,
                          theta=1e4, sliding_window=512, is_producer=0)
    ctx.sync()
    assert same_bits(host(kc), before)
    qn = oracle.norm_rope(raw.q[0], raw.q_w, None, num_heads=8, head_dim=hd, eps=EPS, position=L - 1, theta=1e4)
    ref = oracle.decode_attn_f64(qn, before, host(vc), num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L,
                                 sliding_window=512)
    assert_attention_close(host(out), ref, what="consumer layer")


@pytest.mark.parametrize("layer,producer,pinned", [(0, 1, True), (4, 1, True), (5, 0, True), (0, 1, False),
                                                   (4, 1, "in")])
def test_layer_io_entry_matches_device_path(ctx, layer, producer, pinned):
    """g4a_attn_decode_layer_io (host q | k | v in, host output back, one call) gives the same bits
    as the copy-in, g4a_attn_decode_layer, copy-out sequence, for the caches too; a consumer
    layer copies only q and leaves the shared cache alone.  With both host buffers pinned the
    kernels read and write host memory directly; otherwise the call copies."""
    cfg = GemmaAttnConfig()
    hd, theta, W, div = cfg.head_dim(layer), cfg.rope_theta(layer), cfg.window(layer), cfg.apply_divisor(layer)
    rf = gemma_rope_freqs(512, 64) if div else None
    L = 700
    raw = synth.raw_layer(L + layer, L, hd=hd, theta=theta)
    f16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
    kc0, vc0 = gpu_build_cache(ctx, raw.k[: L - 1], raw.v[: L - 1], raw.k_w, theta=theta, apply_divisor=div,
                               rope_freqs=rf, max_seq=L + 4)
    pos = L - 1
    kw = dict(num_q_heads=8, num_kv_heads=1, head_dim=hd, eps=EPS, position=pos, slot=pos, kv_len=L,
              max_seq_len=L + 4, theta=theta, apply_divisor=div, scale=1.0, sliding_window=W, is_producer=producer)
    qkv = np.concatenate([raw.q[0].reshape(-1), raw.k[pos].reshape(-1), raw.v[pos].reshape(-1)]).astype(np.float32)
    # device path
    kc1, vc1 = kc0.clone(), vc0.clone()
    qd, kd, vd = dev(raw.q[0]), dev(raw.k[pos]), dev(raw.v[pos])
    out1 = torch.zeros((8, hd), device="cuda")
    ctx.attn_decode_layer(qd, kd, vd, f16(raw.q_w), f16(raw.k_w), f16(rf) if rf is not None else None, kc1, vc1,
                          out1, **kw)
    # host-buffer entry, twice in a row into the same pinned output
    kc2, vc2 = kc0.clone(), vc0.clone()
    hin = torch.from_numpy(qkv)
    hout = torch.full((8, hd), float("nan"))
    if pinned is True:
        hin, hout = hin.pin_memory(), hout.pin_memory()  # no copies: kernels reach host memory
    elif pinned == "in":
        hin = hin.pin_memory()  # a mapped input with a pageable output: the copy path
    qkv_dev = torch.empty(qkv.size, device="cuda")
    out_dev = torch.empty((8, hd), device="cuda")
    for _ in range(2):
        ctx.attn_decode_layer_io(hin, qkv_dev, out_dev, hout, f16(raw.q_w), f16(raw.k_w),
                                 f16(rf) if rf is not None else None, kc2, vc2, **kw)
    ctx.sync()
    assert same_bits(hout.numpy(), host(out1))
    assert same_bits(host(qkv_dev[: 8 * hd]), host(qd).reshape(-1))
    assert same_bits(host(kc2), host(kc1)) and same_bits(host(vc2), host(vc1))
    if not producer:
        assert same_bits(host(kc2), host(kc0))
