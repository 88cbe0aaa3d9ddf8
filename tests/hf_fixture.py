"""Loading of the HF-attention fixtures (tests/golden/hf_attn_*.npz, made by
tests/golden/make_attn_golden.py from HF transformers' Gemma4TextAttention) and their inputs."""
import sys
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))
import hf_inputs  # noqa: E402

from g4attn.gemma import gemma_rope_freqs  # noqa: E402

NAMES = list(hf_inputs.CASES)
EPS = 1e-6


class Fixture:
    def __init__(self, name: str):
        self.name = name
        self.d = np.load(GOLDEN / f"hf_attn_{name}.npz")
        self.inp = hf_inputs.raw_inputs(name)
        self.hd = int(self.d["head_dim"])
        self.T = int(self.d["T"])
        self.W = int(self.d["window"])
        self.theta = float(self.d["theta"])
        self.rows = [int(r) for r in self.d["rows"]]
        self.prefill_rows = [int(r) for r in self.d["prefill_rows"]]
        # global layers: proportional RoPE = the rope_freqs divisor table (src/engine.ts:571-576)
        self.apply_divisor = 1 if self.W == 0 else 0
        self.rope_freqs = gemma_rope_freqs(512, 64) if self.apply_divisor else None
        self.q_w16 = self.inp["q_w"].astype(np.float16)
        self.k_w16 = self.inp["k_w"].astype(np.float16)

    def inputs_match(self) -> bool:
        return str(self.d["inputs_sha256"]) == hf_inputs.checksum(self.inp)

    def hf_cache(self):
        """HF's f16 K / V cache as [T, 1, hd] uint16."""
        return (self.d["k16"].reshape(self.T, 1, self.hd), self.d["v16"].reshape(self.T, 1, self.hd))
