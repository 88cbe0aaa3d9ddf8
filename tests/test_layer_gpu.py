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
