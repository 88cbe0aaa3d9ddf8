"""Shared helpers of the GPU parity tests (device buffers from numpy, cache building)."""
import numpy as np
import torch

from g4attn.crosslab import attention_parity

EPS = 1e-6


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t) -> np.ndarray:
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def same_bits(a, b) -> bool:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.dtype == np.float16:
        return np.array_equal(a.view(np.uint16), b.astype(np.float16).view(np.uint16))
    return np.array_equal(a.astype(np.float32).view(np.uint32), b.astype(np.float32).view(np.uint32))


def gpu_build_cache(ctx, raw_k, raw_v, k_w, *, theta, apply_divisor=0, rope_freqs=None, max_seq=None,
                    start_pos=0):
    """Run the producer kernels (g4a_prefill_qkv_prep with no q heads) over raw K/V rows for
    positions start_pos.. and return device f16 caches [max_seq, nkh, hd]."""
    L, nkh, hd = raw_k.shape
    max_seq = max_seq or (start_pos + L)
    kc = torch.zeros((max_seq, nkh, hd), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    k = dev(raw_k)
    v = dev(raw_v)
    kw = dev(k_w.view(np.uint16)).view(torch.float16)
    rf = dev(rope_freqs.view(np.uint16)).view(torch.float16) if rope_freqs is not None else None
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda")
    dummy16 = torch.zeros(16, dtype=torch.float16, device="cuda")
    for c0 in range(0, L, 32768):
        T = min(32768, L - c0)
        ctx.prefill_qkv_prep(dummy, k[c0:c0 + T], v[c0:c0 + T], kw, kw, rf, dummy16, kc, vc, T=T,
                             start_pos=start_pos + c0, max_seq_len=max_seq, num_q_heads=0, num_kv_heads=nkh,
                             head_dim=hd, eps=EPS, theta=theta, apply_divisor=apply_divisor)
    ctx.sync()
    return kc, vc


def assert_attention_close(ours, ref, max_abs=2e-3, cos=0.9999, what=""):
    r = attention_parity(ours, ref, max_abs, cos)
    assert r["ok"], f"{what}: max_abs={r['max_abs']:.3e} min_head_cos={r['min_head_cos']:.8f}"
    return r
