"""Gemma's real layer pattern through the C ABI, against the oracle in the reference's order.

* One decode token through all 35 attention layers of the E2B config (src/config/gemma4-e2b.ts:
  20-53, 159-178): 15 producer layers with their own caches (sliding layers head_dim 256 /
  theta 1e4 / window 512, global layers head_dim 512 / theta 1e6 / rope_freqs divisor), then 20
  consumer layers that read the cache of the last producer of their type (src/engine.ts:
  1519-1522) and never write it.
* The R-SWA ring mapping (src/engine.ts:1962-1969): past the prefix P the store slot wraps
  over a ring of W rows while RoPE keeps the true position and attention covers the
  min(seq_len, P + W) valid rows; twenty-odd consecutive decode steps wrap the ring twice.
* Prompt prefill over the same pattern: sliding layers on the tensor-core kernel, global
  layers (head_dim 512) through the decode kernels."""
import numpy as np
import pytest
import torch

from g4attn import synth
from g4attn.gemma import GemmaAttnConfig, gemma_rope_freqs, ring_slot_and_len
from gpu_helpers import EPS, assert_attention_close, dev, gpu_build_cache, host, same_bits

pytestmark = pytest.mark.gpu


def _f16(a):
    return dev(np.ascontiguousarray(a).view(np.uint16)).view(torch.float16)


def test_decode_token_through_all_layers(ctx, oracle):
    cfg = GemmaAttnConfig()
    L = 600  # position L - 1; the history 0 .. L-2 is in the producers' caches
    pos = L - 1
    producer_of = cfg.kv_producer_for_layer()
    rf = gemma_rope_freqs(512, 64)
    caches = {}  # producer layer -> (device k, device v, raw layer)
    for il in range(cfg.num_layers):
        hd, theta, W = cfg.head_dim(il), cfg.rope_theta(il), cfg.window(il)
        div = cfg.apply_divisor(il)
        rfl = rf if div else None
        prod = producer_of[il]
        if prod == il:
            raw = synth.raw_layer(100 + il, L, hd=hd, theta=theta)
            kc, vc = gpu_build_cache(ctx, raw.k[:pos], raw.v[:pos], raw.k_w, theta=theta, apply_divisor=div,
                                     rope_freqs=rfl, max_seq=L + 4)
            caches[il] = (kc, vc, raw)
            q_raw, q_w = raw.q[0], raw.q_w
            kd, vd = dev(raw.k[pos]), dev(raw.v[pos])
        else:
            # a consumer: its own q and q_norm weight, the producer's cache (and k_norm weight unused)
            rawq = synth.raw_layer(100 + il, 1, hd=hd, theta=theta)
            q_raw, q_w = rawq.q[0], rawq.q_w
            kd = vd = torch.zeros(hd, device="cuda")
        kc, vc, praw = caches[prod]
        before = host(kc).copy() if prod != il else None
        qd = dev(q_raw)
        out = torch.full((8, hd), float("nan"), device="cuda")
        ctx.attn_decode_layer(qd, kd, vd, _f16(q_w), _f16(praw.k_w), _f16(rfl) if rfl is not None else None, kc, vc,
                              out, num_q_heads=8, num_kv_heads=1, head_dim=hd, eps=EPS, position=pos, slot=pos,
                              kv_len=L, max_seq_len=L + 4, theta=theta, apply_divisor=div,
                              scale=cfg.attn_scale(il), sliding_window=W, is_producer=int(prod == il))
        ctx.sync()
        if before is not None:
            assert same_bits(host(kc), before), f"consumer layer {il} wrote the shared cache"
        qn = oracle.norm_rope(q_raw, q_w, rfl, num_heads=8, head_dim=hd, eps=EPS, position=pos, theta=theta,
                              apply_divisor=div)
        assert same_bits(host(qd), qn), f"layer {il} q norm+RoPE"
        ref = oracle.decode_attn_f64(qn, host(kc), host(vc), num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=L,
                                     sliding_window=W)
        assert_attention_close(host(out), ref, what=f"layer {il} (producer {prod}, hd {hd}, W {W})")


@pytest.mark.parametrize("hd,window", [(256, 0), (256, 512), (512, 0)])
def test_ring_decode_steps(ctx, oracle, hd, window):
    P, Wr, steps = 5, 12, 31  # the ring wraps at positions 17 and 29
    theta = 1e4 if hd == 256 else 1e6
    div = 0 if hd == 256 else 1
    rf = gemma_rope_freqs(512, 64) if div else None
    raw = synth.raw_layer(7 + hd, steps, hd=hd, theta=theta, Tq=steps)
    rows = P + Wr
    kc = torch.zeros((rows, 1, hd), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    kh = np.zeros((rows, 1, hd), dtype=np.float16)
    vh = np.zeros_like(kh)
    for pos in range(steps):
        slot, kv_len = ring_slot_and_len(pos, pos + 1, P, Wr)
        qd, kd, vd = dev(raw.q[pos]), dev(raw.k[pos]), dev(raw.v[pos])
        out = torch.full((8, hd), float("nan"), device="cuda")
        ctx.attn_decode_layer(qd, kd, vd, _f16(raw.q_w), _f16(raw.k_w), _f16(rf) if rf is not None else None, kc, vc,
                              out, num_q_heads=8, num_kv_heads=1, head_dim=hd, eps=EPS, position=pos, slot=slot,
                              kv_len=kv_len, max_seq_len=rows, theta=theta, apply_divisor=div, sliding_window=window,
                              is_producer=1)
        ctx.sync()
        # oracle: RoPE at the true position, store at the ring slot, attend to kv_len rows
        qn = oracle.norm_rope(raw.q[pos], raw.q_w, rf, num_heads=8, head_dim=hd, eps=EPS, position=pos, theta=theta,
                              apply_divisor=div)
        kn = oracle.norm_rope(raw.k[pos], raw.k_w, rf, num_heads=1, head_dim=hd, eps=EPS, position=pos, theta=theta,
                              apply_divisor=div)
        vn = oracle.rms_norm_no_weight(raw.v[pos], num_heads=1, head_dim=hd, eps=EPS)
        kh[slot] = oracle.f32_to_f16(kn).reshape(1, hd)
        vh[slot] = oracle.f32_to_f16(vn).reshape(1, hd)
        assert same_bits(host(kc), kh) and same_bits(host(vc), vh), f"cache after position {pos}"
        ref = oracle.decode_attn_f64(qn, kh, vh, num_q_heads=8, num_kv_heads=1, head_dim=hd, kv_len=kv_len,
                                     sliding_window=window)
        assert_attention_close(host(out), ref, what=f"ring pos {pos} slot {slot} kv_len {kv_len}")


def test_prompt_prefill_over_the_layer_pattern(ctx, oracle):
    """One sliding (tensor cores) and one global (head_dim 512, decode kernels) producer layer of a
    130-token prompt at start_pos 70, every row against the oracle."""
    cfg = GemmaAttnConfig()
    T, start = 130, 70
    for il in (0, 4):
        hd, theta, W, div = cfg.head_dim(il), cfg.rope_theta(il), cfg.window(il), cfg.apply_divisor(il)
        rf = gemma_rope_freqs(512, 64) if div else None
        raw = synth.raw_layer(40 + il, start + T, hd=hd, theta=theta, Tq=T)
        kc, vc = gpu_build_cache(ctx, raw.k, raw.v, raw.k_w, theta=theta, apply_divisor=div, rope_freqs=rf)
        qn = np.stack([oracle.norm_rope(raw.q[i], raw.q_w, rf, num_heads=8, head_dim=hd, eps=EPS, position=start + i,
                                        theta=theta, apply_divisor=div).reshape(8, hd) for i in range(T)])
        q16 = oracle.f32_to_f16(qn).reshape(T, 8, hd)
        out = torch.full((T, 8, hd), float("nan"), device="cuda")
        ctx.prefill_attn(_f16(q16), kc, vc, out, T=T, start_pos=start, num_q_heads=8, num_kv_heads=1, head_dim=hd,
                         sliding_window=W)
        ctx.sync()
        ref = oracle.prefill_rows_f64(oracle.f16_to_f32(q16), host(kc), host(vc), list(range(T)), start_pos=start,
                                      num_q_heads=8, num_kv_heads=1, head_dim=hd, sliding_window=W)
        assert_attention_close(host(out), ref, what=f"prefill layer {il} (hd {hd}, W {W})")
