"""Regenerate the committed golden fixture from the reference project's own data.

Run in a container that has the reference checkout (it is not needed at test time):
    python tests/golden/make_golden.py /path/to/reference

vnorm_layer0.npz: from public/ref/layer_0_detail.npz, written by the reference's
reference/pytorch/probe_layer0.py:88-116 (HF transformers 5.5.4, bf16 eager, Gemma 4 E2B,
layer 0 = sliding, head_dim 256, position 14).  It holds the v projection output and HF's
v_norm output for the same token: a known-answer pair for the weightless per-head RMSNorm
(shaders/per_head_rms_norm_no_weight.wgsl), plus the q/k projections and q_norm/k_norm outputs
(one shared norm weight across the 8 q heads), and the attention output (o_proj input).
"""
import sys
from pathlib import Path

import numpy as np

if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
ref = Path(sys.argv[1])
d = np.load(ref / "public/ref/layer_0_detail.npz")
out = Path(__file__).resolve().parent / "vnorm_layer0.npz"
np.savez_compressed(
    out,
    v_proj=d["L0_self_attn.v_proj_output"].astype(np.float32),
    v_norm=d["L0_self_attn.v_norm_output"].astype(np.float32).reshape(-1),
    k_proj=d["L0_self_attn.k_proj_output"].astype(np.float32),
    k_norm=d["L0_self_attn.k_norm_output"].astype(np.float32).reshape(-1),
    q_proj=d["L0_self_attn.q_proj_output"].astype(np.float32),
    q_norm=d["L0_self_attn.q_norm_output"].astype(np.float32),
    attn_out=d["L0_self_attn_o_proj_input"].astype(np.float32),
    position=np.int32(d["position"]),
    source=np.array("public/ref/layer_0_detail.npz (reference/pytorch/probe_layer0.py)"),
)
print("wrote", out)
