"""Generate the HF-attention fixtures: Gemma 4 text attention as HF transformers computes it.

The reference validates its engine against HF transformers' Gemma 4 forward pass captured with
module hooks (reference/pytorch/probe_layer0.py:88-116, smoke_test.py:31-36; methodology in
docs/methodology.md).  This script builds HF's own Gemma4TextAttention module (transformers
5.5.0, transformers.models.gemma4) in float32 with eager attention, for one sliding layer
(head_dim 256, theta 1e4, window 512) and one global layer (head_dim 512, theta 1e6,
proportional RoPE), feeds it the seeded inputs of tests/golden/hf_inputs.py through identity
projections (so the q / k / v projection outputs ARE those inputs), and records with hooks:

  q_rot, k_rot   post-RoPE q and k (HF's apply_rotary_pos_emb on the q_norm / k_norm outputs with
                 HF's rotary cos/sin) at the tested rows
  v_norm         HF's weightless v_norm output at the tested rows
  k16, v16       post-RoPE k and v_norm of every position, rounded to f16 (the f16 KV cache)
  attn_fp32      the attention output (o_proj input) of HF's full fp32 forward at the tested rows
  attn_k16       HF's eager attention (its own function and its own 4-D mask) over the f16 cache:
                 the common-input reference for the decode tests
  attn_prefill   the same with q rounded to f16 too, at prefill_rows (the prefill kernels take f16 q)
  mask_lo/hi     first and last key HF's mask lets each tested row attend

Only this script needs transformers; the tests read the .npz files.  Run it here:
    python tests/golden/make_attn_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import hf_inputs  # noqa: E402


def build_case(name: str) -> dict:
    from transformers import masking_utils
    from transformers.models.gemma4 import modeling_gemma4 as hf
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    c = hf_inputs.CASES[name]
    hd, T, nqh = c["head_dim"], c["T"], hf_inputs.NQH
    inp = hf_inputs.raw_inputs(name)
    H = (nqh + 2) * hd  # hidden = [q (8 hd) | k (hd) | v (hd)]
    cfg = Gemma4TextConfig(hidden_size=H, num_attention_heads=nqh, num_key_value_heads=1, head_dim=256,
                           global_head_dim=512, sliding_window=512, rms_norm_eps=1e-6,
                           layer_types=["sliding_attention", "full_attention"], num_hidden_layers=2,
                           vocab_size=16, intermediate_size=32, num_kv_shared_layers=0)
    cfg._attn_implementation = "eager"
    attn = hf.Gemma4TextAttention(cfg, c["layer_idx"]).float().eval()
    assert attn.head_dim == hd and attn.scaling == 1.0 and attn.num_key_value_groups == nqh
    assert attn.is_sliding == (c["window"] > 0)
    ltype = attn.layer_type
    with torch.no_grad():
        eye = torch.eye(H)
        attn.q_proj.weight.copy_(eye[: nqh * hd])
        attn.k_proj.weight.copy_(eye[nqh * hd:(nqh + 1) * hd])
        attn.v_proj.weight.copy_(eye[(nqh + 1) * hd:])
        attn.q_norm.weight.copy_(torch.from_numpy(inp["q_w"]))
        attn.k_norm.weight.copy_(torch.from_numpy(inp["k_w"]))
    hidden = torch.from_numpy(np.concatenate([inp["q"].reshape(T, nqh * hd), inp["k"], inp["v"]], axis=1))[None]
    pid = torch.arange(T)[None]
    cos, sin = hf.Gemma4TextRotaryEmbedding(cfg)(hidden, pid, ltype)
    make_mask = masking_utils.create_sliding_window_causal_mask if attn.is_sliding else masking_utils.create_causal_mask
    mask = make_mask(cfg, hidden, None, past_key_values=None, position_ids=pid)

    cap = {}
    hooks = [attn.q_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("q_proj", o.detach())),
             attn.k_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("k_proj", o.detach())),
             attn.v_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("v_proj", o.detach())),
             attn.q_norm.register_forward_hook(lambda m, i, o: cap.__setitem__("q_norm", o.detach())),
             attn.k_norm.register_forward_hook(lambda m, i, o: cap.__setitem__("k_norm", o.detach())),
             attn.v_norm.register_forward_hook(lambda m, i, o: cap.__setitem__("v_norm", o.detach())),
             attn.o_proj.register_forward_pre_hook(lambda m, i: cap.__setitem__("attn", i[0].detach()))]
    with torch.no_grad():
        attn(hidden, (cos, sin), mask)
        for h in hooks:
            h.remove()
        # the projections are exact copies of the inputs (identity weights, no bias)
        assert torch.equal(cap["q_proj"][0], torch.from_numpy(inp["q"].reshape(T, nqh * hd)))
        assert torch.equal(cap["k_proj"][0], torch.from_numpy(inp["k"]))
        assert torch.equal(cap["v_proj"][0], torch.from_numpy(inp["v"]))
        q_rot = hf.apply_rotary_pos_emb(cap["q_norm"], cos, sin, unsqueeze_dim=2)  # [1, T, 8, hd]
        k_rot = hf.apply_rotary_pos_emb(cap["k_norm"], cos, sin, unsqueeze_dim=2)  # [1, T, 1, hd]
        vn = cap["v_norm"]                                                          # [1, T, 1, hd]
        # the module's own output is HF's eager attention over these tensors (sanity: bit-equal)
        again, _ = hf.eager_attention_forward(attn, q_rot.transpose(1, 2), k_rot.transpose(1, 2),
                                              vn.transpose(1, 2), mask, scaling=1.0)
        assert torch.equal(again.reshape(1, T, -1), cap["attn"]), "HF forward is not eager attention on q_rot/k_rot"
        k16 = k_rot[0, :, 0].half()
        v16 = vn[0, :, 0].half()
        a16, _ = hf.eager_attention_forward(attn, q_rot.transpose(1, 2), k16.float()[None, None],
                                            v16.float()[None, None], mask, scaling=1.0)
        ap16, _ = hf.eager_attention_forward(attn, q_rot.half().float().transpose(1, 2), k16.float()[None, None],
                                             v16.float()[None, None], mask, scaling=1.0)
    rows = np.array(c["rows"], dtype=np.int64)
    prow = np.array(c["prefill_rows"], dtype=np.int64)
    m = mask[0, 0].numpy()
    allowed = m == 0
    mask_lo = np.array([np.flatnonzero(allowed[r]).min() for r in rows], dtype=np.int64)
    mask_hi = np.array([np.flatnonzero(allowed[r]).max() for r in rows], dtype=np.int64)
    return dict(
        transformers_version=np.array(__import__("transformers").__version__),
        inputs_sha256=np.array(hf_inputs.checksum(inp)),
        head_dim=np.int64(hd), T=np.int64(T), theta=np.float64(c["theta"]), window=np.int64(c["window"]),
        rows=rows, prefill_rows=prow,
        q_rot=q_rot[0].numpy()[rows].astype(np.float32),
        k_rot=k_rot[0, :, 0].numpy()[rows].astype(np.float32),
        v_norm=vn[0, :, 0].numpy()[rows].astype(np.float32),
        k16=k16.numpy().view(np.uint16), v16=v16.numpy().view(np.uint16),
        attn_fp32=cap["attn"][0].numpy()[rows].reshape(len(rows), nqh, hd).astype(np.float32),
        attn_k16=a16[0].numpy()[rows].astype(np.float32),
        attn_prefill=ap16[0].numpy()[prow].astype(np.float32),
        mask_lo=mask_lo, mask_hi=mask_hi,
    )


def main() -> int:
    torch.manual_seed(0)
    for name in hf_inputs.CASES:
        d = build_case(name)
        out = HERE / f"hf_attn_{name}.npz"
        np.savez_compressed(out, **d)
        print(f"wrote {out} ({out.stat().st_size} bytes): rows {d['rows'].tolist()}, "
              f"mask [lo, hi] {list(zip(d['mask_lo'].tolist(), d['mask_hi'].tolist()))}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
