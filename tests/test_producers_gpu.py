"""Producer kernels (norm+RoPE, v_norm, KV store, prefill input stage) are bit-exact against
the oracle's restatement of fused_per_head_norm_rope.wgsl, per_head_rms_norm_no_weight.wgsl
and kv_cache_store.wgsl."""
from pathlib import Path

import numpy as np
import pytest
import torch

from g4attn import synth
from g4attn.gemma import gemma_rope_freqs
from gpu_helpers import EPS, dev, gpu_build_cache, host, same_bits

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "vnorm_layer0.npz"


@pytest.mark.parametrize("hd", [256, 512])
@pytest.mark.parametrize("pos", [0, 1, 511, 4095, 131071, 1048575])
@pytest.mark.parametrize("theta", [1e4, 1e6])
def test_norm_rope_bit_exact(ctx, oracle, hd, pos, theta):
    rng = np.random.default_rng(hd * 7 + pos)
    x = rng.standard_normal((8, hd)).astype(np.float32)
    w = synth.norm_weight(rng, hd)
    ref = oracle.norm_rope(x, w, None, num_heads=8, head_dim=hd, eps=EPS, position=pos, theta=theta)
    xd = dev(x)
    ctx.norm_rope(xd, dev(w.view(np.uint16)).view(torch.float16), None, num_heads=8, head_dim=hd, eps=EPS,
                  position=pos, theta=theta)
    assert same_bits(host(xd), ref)


@pytest.mark.parametrize("pos", [3, 70000, 1048575])
def test_norm_rope_divisor_table_bit_exact(ctx, oracle, pos):
    rng = np.random.default_rng(pos)
    hd = 512
    x = rng.standard_normal((1, hd)).astype(np.float32)
    w = synth.norm_weight(rng, hd)
    rf = gemma_rope_freqs(hd, 64)
    ref = oracle.norm_rope(x, w, rf, num_heads=1, head_dim=hd, eps=EPS, position=pos, theta=1e6, apply_divisor=1)
    xd = dev(x)
    ctx.norm_rope(xd, dev(w.view(np.uint16)).view(torch.float16), dev(rf.view(np.uint16)).view(torch.float16),
                  num_heads=1, head_dim=hd, eps=EPS, position=pos, theta=1e6, apply_divisor=1)
    assert same_bits(host(xd), ref)


@pytest.mark.parametrize("hd,nh", [(256, 1), (512, 1), (256, 8), (100, 3)])
def test_rms_norm_no_weight_bit_exact(ctx, oracle, hd, nh):
    x = np.random.default_rng(hd + nh).standard_normal((nh, hd)).astype(np.float32) * 3
    ref = oracle.rms_norm_no_weight(x, num_heads=nh, head_dim=hd, eps=EPS)
    xd = dev(x)
    ctx.rms_norm_no_weight(xd, num_heads=nh, head_dim=hd, eps=EPS)
    assert same_bits(host(xd), ref)


def test_vnorm_golden_fixture_on_gpu(ctx, oracle):
    g = np.load(GOLDEN)
    xd = dev(g["v_proj"].reshape(1, 256))
    ctx.rms_norm_no_weight(xd, num_heads=1, head_dim=256, eps=EPS)
    ours = host(xd).reshape(-1)
    assert same_bits(ours, oracle.rms_norm_no_weight(g["v_proj"].reshape(1, 256), num_heads=1, head_dim=256,
                                                     eps=EPS).reshape(-1))
    c = float(np.dot(ours, g["v_norm"]) / np.linalg.norm(ours) / np.linalg.norm(g["v_norm"]))
    assert c > 0.99999


@pytest.mark.parametrize("fuse", [0, 1])
def test_kv_store_bit_exact(ctx, oracle, fuse):
    rng = np.random.default_rng(fuse)
    nkh, hd, max_seq, slot = 2, 256, 40, 17
    k = rng.standard_normal((nkh, hd)).astype(np.float32)
    v = rng.standard_normal((nkh, hd)).astype(np.float32) * 5
    kc = torch.full((max_seq, nkh, hd), 7.0, dtype=torch.float16, device="cuda")
    vc = torch.full_like(kc, 7.0)
    kd, vd = dev(k), dev(v)
    ctx.kv_store(kd, vd, kc, vc, num_kv_heads=nkh, head_dim=hd, position=slot, max_seq_len=max_seq,
                 eps=EPS, fuse_v_norm=fuse)
    vn = oracle.rms_norm_no_weight(v, num_heads=nkh, head_dim=hd, eps=EPS) if fuse else v
    kch, vch = host(kc), host(vc)
    assert same_bits(kch[slot], oracle.f32_to_f16(k))
    assert same_bits(vch[slot], oracle.f32_to_f16(vn))
    assert same_bits(host(vd), vn)
    others = np.delete(np.arange(max_seq), slot)
    assert (kch[others] == 7).all() and (vch[others] == 7).all()


@pytest.mark.parametrize("hd,theta,div", [(256, 1e4, 0), (512, 1e6, 1)])
def test_prefill_qkv_prep_bit_exact(ctx, oracle, hd, theta, div):
    T, start, max_seq = 50, 7, 64
    raw = synth.raw_layer(3, T, hd=hd, theta=theta, Tq=T)
    rf = gemma_rope_freqs(hd, 64) if div else None
    q16 = torch.zeros((T, 8, hd), dtype=torch.float16, device="cuda")
    kc = torch.zeros((max_seq, 1, hd), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    qd, kd, vd = dev(raw.q), dev(raw.k), dev(raw.v)
    ctx.prefill_qkv_prep(qd, kd, vd, dev(raw.q_w.view(np.uint16)).view(torch.float16),
                         dev(raw.k_w.view(np.uint16)).view(torch.float16),
                         dev(rf.view(np.uint16)).view(torch.float16) if rf is not None else None, q16, kc, vc, T=T,
                         start_pos=start, max_seq_len=max_seq, num_q_heads=8, num_kv_heads=1, head_dim=hd, eps=EPS,
                         theta=theta, apply_divisor=div)
    kref, vref = oracle.build_cache(raw.k, raw.v, raw.k_w, theta=theta, apply_divisor=div, rope_freqs=rf,
                                    positions=np.arange(start, start + T))
    assert same_bits(host(kc)[start:start + T], kref)
    assert same_bits(host(vc)[start:start + T], vref)
    for i in (0, 13, T - 1):
        qref = oracle.norm_rope(raw.q[i], raw.q_w, rf, num_heads=8, head_dim=hd, eps=EPS, position=start + i,
                                theta=theta, apply_divisor=div)
        assert same_bits(host(q16)[i], oracle.f32_to_f16(qref))
    assert same_bits(host(qd), raw.q)  # inputs untouched


def test_gpu_cache_builder_matches_oracle(ctx, oracle):
    raw = synth.raw_layer(0, 300, hd=256, theta=1e4)
    kc, vc = gpu_build_cache(ctx, raw.k, raw.v, raw.k_w, theta=1e4)
    kref, vref = oracle.build_cache(raw.k, raw.v, raw.k_w, theta=1e4)
    assert same_bits(host(kc), kref) and same_bits(host(vc), vref)


def test_prefill_prep_rejects_head_dim_off_the_warp_layout(ctx):
    """The prefill input stage takes head_dim in multiples of 64 (<= 512); others fail on the host."""
    from g4attn import G4AError

    T, hd = 4, 96
    f = torch.zeros((T, 1, hd), device="cuda")
    h = torch.zeros((T, 1, hd), dtype=torch.float16, device="cuda")
    w = torch.ones(hd, dtype=torch.float16, device="cuda")
    with pytest.raises(G4AError) as ei:
        ctx.prefill_qkv_prep(f, f, f, w, w, None, h, h, h, T=T, start_pos=0, max_seq_len=T, num_q_heads=1,
                             num_kv_heads=1, head_dim=hd, eps=EPS, theta=1e4)
    assert "multiple of 64" in str(ei.value)
