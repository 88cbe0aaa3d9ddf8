"""The allocation-free decode entry (g4a_decode_attn_noalloc) against g4a_decode_attn and the oracle.

It runs the same kernels with the split-KV scratch in a fixed static device area instead of
the context's growable workspace, so its output must agree with g4a_decode_attn on the same
inputs, and both with the fp64-accumulated CPU oracle (orc_decode_attn_f64), within the
attention tolerance (max abs <= 2e-3, per-head cosine >= 0.9999), on two calls in a row; calls
after the first must not change the device's free memory.  The file builds all its own state,
so it passes alone in a fresh process as well as after the others.
"""
import numpy as np
import pytest
import torch

import g4attn
from g4attn import G4AError
from g4attn.crosslab import attention_parity

pytestmark = pytest.mark.gpu

SHAPES = [  # (kv_len, sliding_window, head_dim, num_kv_heads)
    (32768, 0, 256, 1),
    (5000, 512, 256, 1),
    (3000, 0, 512, 1),
    (700, 0, 128, 2),
    (1, 0, 256, 1),
    (0, 0, 256, 1),
]


def _inputs(seed, L, hd, nkh):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn((8 * nkh, hd), generator=g)
    q = q / q.pow(2).mean(-1, keepdim=True).sqrt()
    k = torch.randn((max(L, 1), nkh, hd), generator=g).half()
    v = torch.randn((max(L, 1), nkh, hd), generator=g).half()
    return q.cuda(), k.cuda(), v.cuda()


@pytest.mark.parametrize("L,W,hd,nkh", SHAPES)
def test_noalloc_matches_decode_attn(L, W, hd, nkh, oracle):
    q, k, v = _inputs(L * 7 + hd + nkh, L, hd, nkh)
    kw = dict(num_q_heads=8 * nkh, num_kv_heads=nkh, head_dim=hd, seq_len=L, sliding_window=W, scale=1.0)
    with g4attn.Context(0) as ctx:
        ref = torch.zeros((8 * nkh, hd), device="cuda")
        ctx.decode_attn(q, k, v, ref, **kw)
        ctx.sync()
        want = ref.cpu().numpy()
    with g4attn.Context(0) as ctx:
        outs = [torch.full((8 * nkh, hd), float("nan"), device="cuda") for _ in range(3)]
        ctx.decode_attn_noalloc(q, k, v, outs[0], **kw)  # first call: looks up the scratch address
        ctx.sync()
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        for o in outs[1:]:  # two calls in a row
            ctx.decode_attn_noalloc(q, k, v, o, **kw)
        ctx.sync()
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        got = [o.cpu().numpy() for o in outs]
    assert free_after == free_before, (free_before, free_after)
    gold = None
    if L > 0:
        gold = oracle.decode_attn_f64(q.cpu().numpy(), k.cpu().numpy().view(np.uint16), v.cpu().numpy().view(np.uint16),
                                      num_q_heads=8 * nkh, num_kv_heads=nkh, head_dim=hd, kv_len=L,
                                      sliding_window=W).astype(np.float64)
        r = attention_parity(want, gold)
        assert r["ok"], ("g4a_decode_attn vs oracle", r)
    for i, g in enumerate(got):
        assert np.isfinite(g).all(), i
        if L == 0:
            assert not g.any() and not want.any()
            continue
        r = attention_parity(g, want.astype(np.float64))
        assert r["ok"], (i, r)
        r = attention_parity(g, gold)
        assert r["ok"], (i, "vs oracle", r)


def test_noalloc_rejects_shape_beyond_scratch():
    """128 kv heads at head_dim 512 need more split-KV scratch than the fixed area holds: the call
    fails on the host with a message naming the sizes, before anything is launched."""
    nkh, hd, L = 128, 512, 64
    q = torch.zeros((8 * nkh, hd), device="cuda")
    k = torch.zeros((L, nkh, hd), dtype=torch.float16, device="cuda")
    v = torch.zeros_like(k)
    out = torch.full((8 * nkh, hd), 7.0, device="cuda")
    with g4attn.Context(0) as ctx:
        with pytest.raises(G4AError) as ei:
            ctx.decode_attn_noalloc(q, k, v, out, num_q_heads=8 * nkh, num_kv_heads=nkh, head_dim=hd, seq_len=L)
        assert "scratch" in str(ei.value) and "bytes" in str(ei.value)
        ctx.sync()
    assert bool((out == 7.0).all())


def test_noalloc_refuses_while_profiling():
    q, k, v = _inputs(3, 100, 256, 1)
    out = torch.zeros((8, 256), device="cuda")
    with g4attn.Context(0) as ctx:
        ctx.profile_enable(True)
        with pytest.raises(G4AError):
            ctx.decode_attn_noalloc(q, k, v, out, num_q_heads=8, num_kv_heads=1, head_dim=256, seq_len=100)
        ctx.profile_enable(False)
        ctx.decode_attn_noalloc(q, k, v, out, num_q_heads=8, num_kv_heads=1, head_dim=256, seq_len=100)
        ctx.sync()
    assert np.isfinite(out.cpu().numpy()).all()
