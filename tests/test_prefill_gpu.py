"""Tensor-core prefill attention (g4a_prefill_attn) against the oracle.

The reference prefills token by token (prefillBatched, src/engine.ts:2460-2479), so row i of
prefill attention must equal decode attention at kv_len = start_pos + i + 1 with the window
measured from that kv_len.  Q is the f16 output of the prep kernel (the kernel's input format),
so the oracle runs on the same f16-valued q.  Tolerance: max abs <= 2e-3 and per-head cosine
>= 0.9999 against the fp64 oracle (small shapes, every row) and against a torch fp32 reference
on the GPU (the full 4096-token config, every row)."""
import numpy as np
import pytest
import torch

from g4attn import G4AError, synth
from gpu_helpers import EPS, assert_attention_close, dev, host

pytestmark = pytest.mark.gpu


def _setup(ctx, T, start_pos, hd, nkh, theta, seed):
    """Cache rows 0 .. start_pos+T-1 and the f16 q of the last T tokens, built by the prep kernel
    (history first, then the prompt chunk, as a chunked prefill would)."""
    nqh = 8 * nkh
    L = start_pos + T
    rng = np.random.default_rng(seed)
    qw = dev(synth.norm_weight(rng, hd).view(np.uint16)).view(torch.float16)
    kw = dev(synth.norm_weight(rng, hd).view(np.uint16)).view(torch.float16)
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((L, nkh, hd), generator=g, device="cuda")
    v = torch.randn((L, nkh, hd), generator=g, device="cuda")
    q = torch.randn((T, nqh, hd), generator=g, device="cuda")
    kc = torch.zeros((L, nkh, hd), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    q16 = torch.zeros((T, nqh, hd), dtype=torch.float16, device="cuda")
    dummy = torch.zeros(16, device="cuda")
    dummy16 = torch.zeros(16, dtype=torch.float16, device="cuda")
    if start_pos:
        ctx.prefill_qkv_prep(dummy, k[:start_pos], v[:start_pos], qw, kw, None, dummy16, kc, vc, T=start_pos,
                             start_pos=0, max_seq_len=L, num_q_heads=0, num_kv_heads=nkh, head_dim=hd, eps=EPS,
                             theta=theta)
    ctx.prefill_qkv_prep(q, k[start_pos:], v[start_pos:], qw, kw, None, q16, kc, vc, T=T, start_pos=start_pos,
                         max_seq_len=L, num_q_heads=nqh, num_kv_heads=nkh, head_dim=hd, eps=EPS, theta=theta)
    ctx.sync()
    return q16, kc, vc


def _run(ctx, q16, kc, vc, T, start_pos, hd, nkh, W):
    out = torch.full((T, 8 * nkh, hd), float("nan"), device="cuda")
    ctx.prefill_attn(q16, kc, vc, out, T=T, start_pos=start_pos, num_q_heads=8 * nkh, num_kv_heads=nkh, head_dim=hd,
                     scale=1.0, sliding_window=W)
    ctx.sync()
    return out


def _torch_ref(q16, kc, vc, start_pos, W, rows_per_chunk=256):
    """fp32 masked softmax attention on the GPU, in chunks of query rows."""
    T, nqh, hd = q16.shape
    nkh = kc.shape[1]
    g = nqh // nkh
    K = kc.float()
    V = vc.float()
    out = torch.empty((T, nqh, hd), device="cuda")
    keys = torch.arange(K.shape[0], device="cuda")
    for c0 in range(0, T, rows_per_chunk):
        c1 = min(T, c0 + rows_per_chunk)
        hi = start_pos + torch.arange(c0, c1, device="cuda") + 1           # [n]
        lo = torch.clamp(hi - W, min=0) if W else torch.zeros_like(hi)
        mask = (keys[None, :] >= lo[:, None]) & (keys[None, :] < hi[:, None])  # [n, L]
        q = q16[c0:c1].float()                                              # [n, nqh, hd]
        for kvh in range(nkh):
            qs = q[:, kvh * g:(kvh + 1) * g]                                # [n, g, hd]
            s = torch.einsum("ngd,ld->ngl", qs, K[:, kvh])
            s = s.masked_fill(~mask[:, None, :], float("-inf"))
            p = torch.softmax(s, dim=-1)
            out[c0:c1, kvh * g:(kvh + 1) * g] = torch.einsum("ngl,ld->ngd", p, V[:, kvh])
    return out


SMALL = [  # T, start_pos, W, hd, nkh
    (1, 0, 0, 256, 1),
    (5, 0, 0, 256, 1),
    (16, 0, 0, 256, 1),
    (17, 0, 0, 256, 1),
    (100, 0, 0, 256, 1),
    (300, 0, 40, 256, 1),
    (200, 37, 0, 256, 1),
    (130, 500, 64, 256, 1),
    (77, 0, 0, 128, 1),
    (129, 0, 512, 128, 1),
    (64, 10, 0, 256, 2),
    (40, 1000, 512, 256, 1),
]


@pytest.mark.parametrize("T,start_pos,W,hd,nkh", SMALL)
def test_prefill_every_row_matches_oracle(ctx, oracle, T, start_pos, W, hd, nkh):
    theta = 1e4 if W else 1e6
    q16, kc, vc = _setup(ctx, T, start_pos, hd, nkh, theta, seed=T * 31 + start_pos + hd + nkh)
    ours = host(_run(ctx, q16, kc, vc, T, start_pos, hd, nkh, W))
    ref = oracle.prefill_rows_f64(host(q16).astype(np.float32), host(kc), host(vc), list(range(T)),
                                  start_pos=start_pos, num_q_heads=8 * nkh, num_kv_heads=nkh, head_dim=hd,
                                  sliding_window=W)
    assert_attention_close(ours, ref, what=f"T={T} start={start_pos} W={W} hd={hd} nkh={nkh}")


@pytest.mark.parametrize("W,theta", [(0, 1e6), (512, 1e4)])
def test_prefill_config3_full_size(ctx, oracle, W, theta):
    """T = 4096, 8 q heads / 1 kv head, head_dim 256; every row against the
    torch fp32 reference, tile-boundary and random rows against the fp64 oracle."""
    T = 4096
    q16, kc, vc = _setup(ctx, T, 0, 256, 1, theta, seed=3)
    out = _run(ctx, q16, kc, vc, T, 0, 256, 1, W)
    ref = _torch_ref(q16, kc, vc, 0, W)
    assert_attention_close(host(out), host(ref), what=f"config3 W={W} vs torch fp32")
    rng = np.random.default_rng(W)
    rows = sorted(set([0, 1, 15, 16, 17, 63, 64, 65, 511, 512, 513, 1023, 2048, 4031, 4080, 4095]
                      + rng.integers(0, T, size=16).tolist()))
    ours = host(out)[rows]
    ref64 = oracle.prefill_rows_f64(host(q16).astype(np.float32), host(kc), host(vc), rows, start_pos=0,
                                    num_q_heads=8, num_kv_heads=1, head_dim=256, sliding_window=W)
    assert_attention_close(ours, ref64, what=f"config3 W={W} vs oracle")


def test_prefill_repeatable(ctx):
    """Two runs on the same inputs give the same bits (no races between the warp roles)."""
    q16, kc, vc = _setup(ctx, 700, 0, 256, 1, 1e6, seed=5)
    a = host(_run(ctx, q16, kc, vc, 700, 0, 256, 1, 0))
    b = host(_run(ctx, q16, kc, vc, 700, 0, 256, 1, 0))
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# head_dim 512 with GQA 8:1 (Gemma's global layers) runs on the tensor-core kernel as CTA pairs
# (each CTA of a cluster owns 256 of the 512 dims and the two exchange partial scores); other
# shapes run through the decode kernels (the fast decode path for head_dim 512 with other ratios
# is not used; GQA 4:1 and 3:1 take the generic kernel).
FALLBACK = [
    (70, 0, 0, 512, 1, 8),      # Gemma global layer: head_dim 512, causal
    (90, 300, 512, 512, 1, 8),  # head_dim 512, sliding, after a prefix
    (1, 0, 0, 512, 1, 8),       # one token
    (7, 0, 0, 512, 1, 8),       # a partial tile
    (16, 0, 0, 512, 1, 8),      # exactly one tile (16 tokens x 8 heads)
    (17, 3, 0, 512, 1, 8),      # one row past a tile, after a prefix
    (257, 40, 33, 512, 2, 16),  # two kv heads (two tiles per token group), window not a multiple of 64
    (200, 0, 64, 512, 1, 8),    # window of exactly one key block
    (130, 1000, 64, 512, 1, 8), # long prefix, small window
    (33, 5, 0, 256, 1, 4),      # GQA 4:1 (generic kernel)
    (48, 0, 16, 64, 2, 6),      # GQA 3:1, small head_dim, tiny window
    (40, 0, 0, 512, 1, 4),      # head_dim 512 at GQA 4:1 (decode kernels)
]


@pytest.mark.parametrize("T,start_pos,W,hd,nkh,nqh", FALLBACK)
def test_prefill_other_shapes_match_oracle(ctx, oracle, T, start_pos, W, hd, nkh, nqh):
    rng = np.random.default_rng(T + hd + nqh)
    L = start_pos + T
    q = rng.standard_normal((T, nqh, hd)).astype(np.float32).astype(np.float16)
    k = rng.standard_normal((L, nkh, hd)).astype(np.float32).astype(np.float16)
    v = rng.standard_normal((L, nkh, hd)).astype(np.float32).astype(np.float16)
    q /= np.float16(np.sqrt(hd) / 4)  # keep the scores in a moderate range
    q16 = dev(q.view(np.uint16)).view(torch.float16)
    kc = dev(k.view(np.uint16)).view(torch.float16)
    vc = dev(v.view(np.uint16)).view(torch.float16)
    out = torch.full((T, nqh, hd), float("nan"), device="cuda")
    ctx.prefill_attn(q16, kc, vc, out, T=T, start_pos=start_pos, num_q_heads=nqh, num_kv_heads=nkh, head_dim=hd,
                     sliding_window=W)
    ctx.sync()
    ref = oracle.prefill_rows_f64(q.astype(np.float32), k, v, list(range(T)), start_pos=start_pos, num_q_heads=nqh,
                                  num_kv_heads=nkh, head_dim=hd, sliding_window=W)
    assert_attention_close(host(out), ref, what=f"T={T} start={start_pos} W={W} hd={hd} nkh={nkh} nqh={nqh}")


@pytest.mark.parametrize("W,theta", [(0, 1e6), (512, 1e4)])
def test_prefill_head_dim_512_full_size(ctx, oracle, W, theta):
    """T = 4096 at head_dim 512 (a Gemma global layer's prompt): every row against the torch fp32
    reference, tile-boundary and random rows against the fp64 oracle; two runs give the same bits."""
    T = 4096
    q16, kc, vc = _setup(ctx, T, 0, 512, 1, theta, seed=11)
    out = _run(ctx, q16, kc, vc, T, 0, 512, 1, W)
    again = _run(ctx, q16, kc, vc, T, 0, 512, 1, W)
    assert np.array_equal(host(out).view(np.uint32), host(again).view(np.uint32))
    ref = _torch_ref(q16, kc, vc, 0, W, rows_per_chunk=128)
    assert_attention_close(host(out), host(ref), what=f"hd512 W={W} vs torch fp32")
    rows = [0, 1, 7, 8, 9, 15, 16, 17, 31, 32, 33, 63, 64, 65, 511, 512, 513, 2047, 4080, 4088, 4095]
    ref64 = oracle.prefill_rows_f64(host(q16).astype(np.float32), host(kc), host(vc), rows, start_pos=0,
                                    num_q_heads=8, num_kv_heads=1, head_dim=512, sliding_window=W)
    assert_attention_close(host(out)[rows], ref64, what=f"hd512 W={W} vs oracle")


def test_prefill_rejects_invalid_shapes(ctx):
    q16 = torch.zeros((4, 8, 520), dtype=torch.float16, device="cuda")
    kc = torch.zeros((4, 1, 520), dtype=torch.float16, device="cuda")
    out = torch.zeros((4, 8, 520), device="cuda")
    with pytest.raises(G4AError) as ei:
        ctx.prefill_attn(q16, kc, kc, out, T=4, start_pos=0, num_q_heads=8, num_kv_heads=1, head_dim=520)
    assert "head_dim" in str(ei.value)
    with pytest.raises(G4AError):
        ctx.prefill_attn(q16, kc, kc, out, T=4, start_pos=0, num_q_heads=1, num_kv_heads=2, head_dim=256)
    ctx.prefill_attn(q16, kc, kc, out, T=0, start_pos=0, num_q_heads=8, num_kv_heads=1, head_dim=256)
    ctx.sync()
