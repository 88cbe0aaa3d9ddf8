"""Seeded raw inputs of the HF-attention fixtures (hf_attn_sliding.npz, hf_attn_global.npz).

Shared by tests/golden/make_attn_golden.py (which feeds them to HF transformers' Gemma 4
attention) and by the parity tests (which feed them to the oracle and the CUDA kernels).  Every
value is f16-representable, so the f16 norm weights and the f32 projections of both sides hold
identical numbers.  The fixture stores a SHA-256 of these arrays; the tests recompute it, so a
change of numpy's generator stream fails loudly instead of comparing different inputs.

Recipe (BASELINE config recipe): q, k, v ~ N(0, 1); q_norm / k_norm weights 1 + N(0, 0.05).
"""
from __future__ import annotations

import hashlib

import numpy as np

NQH = 8

CASES = {
    # Gemma 4 sliding layer: head_dim 256, RoPE theta 1e4, window 512 (src/config/gemma4-e2b.ts).
    # Rows 511 / 512 / 513 straddle the window edge; 700 has a window start of 189.
    "sliding": dict(layer_idx=0, head_dim=256, T=701, rows=[14, 511, 512, 513, 700], theta=1e4, window=512,
                    prefill_rows=[0, 1, 13, 14, 100, 255, 256, 511, 512, 513, 600, 700], seed=4001),
    # Gemma 4 global layer: head_dim 512, theta 1e6, proportional RoPE over the first quarter of
    # the pairs (HF rope_type "proportional", partial_rotary_factor 0.25) = the engine's rope_freqs
    # divisor table (1 for pairs 0..63, +inf after: src/engine.ts:571-576).
    "global": dict(layer_idx=1, head_dim=512, T=400, rows=[14, 255, 256, 399], theta=1e6, window=0,
                   prefill_rows=[0, 1, 14, 100, 255, 256, 300, 399], seed=4002),
}


def f16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def raw_inputs(case: str) -> dict:
    """q [T, 8, hd], k [T, hd], v [T, hd] (one kv head), q_w [hd], k_w [hd]: f32 holding f16 values."""
    c = CASES[case]
    hd, T = c["head_dim"], c["T"]
    rng = np.random.default_rng(c["seed"])
    q = f16_round(rng.standard_normal((T, NQH, hd)))
    k = f16_round(rng.standard_normal((T, hd)))
    v = f16_round(rng.standard_normal((T, hd)))
    q_w = f16_round(1.0 + 0.05 * rng.standard_normal(hd))
    k_w = f16_round(1.0 + 0.05 * rng.standard_normal(hd))
    return {"q": q, "k": k, "v": v, "q_w": q_w, "k_w": k_w}


def checksum(inputs: dict) -> str:
    h = hashlib.sha256()
    for name in ("q", "k", "v", "q_w", "k_w"):
        h.update(np.ascontiguousarray(inputs[name], dtype=np.float32).tobytes())
    return h.hexdigest()
