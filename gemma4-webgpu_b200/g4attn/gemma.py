"""Gemma 4 E2B attention-layer shape rules, restated from the reference's config helpers.

These decide, per layer, the arguments of the attention entry points: head_dim, RoPE theta,
sliding window, whether the rope_freqs divisor applies, and which layer's KV cache a consumer
layer reads.  Sources: src/config/gemma4-e2b.ts:16-60 (defaults), :159-178 (producer map),
src/types.ts:140-162 (isSwaLayer / getRopeTheta / getHeadDim / isKvProducerLayer),
src/engine.ts:548-590 (per-layer uniforms: scale 1.0, apply_divisor on global layers).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class GemmaAttnConfig:
    num_layers: int = 35
    num_q_heads: int = 8
    num_kv_heads: int = 1
    head_dim_local: int = 256
    head_dim_global: int = 512
    rms_norm_eps: float = 1e-6
    rope_theta_global: float = 1_000_000.0
    rope_theta_swa: float = 10_000.0
    sliding_window: int = 512
    num_unshared_layers: int = 15
    context_length: int = 2048
    attention_is_sliding: list[bool] = field(default_factory=list)

    def __post_init__(self):
        if not self.attention_is_sliding:
            s = [True] * self.num_layers
            for i in (4, 9, 14, 19, 24, 29, 34):  # every fifth layer is global (gemma4-e2b.ts:20-21)
                if i < self.num_layers:
                    s[i] = False
            self.attention_is_sliding = s

    # src/types.ts:140-162
    def is_swa_layer(self, il: int) -> bool:
        return self.attention_is_sliding[il]

    def rope_theta(self, il: int) -> float:
        return self.rope_theta_swa if self.is_swa_layer(il) else self.rope_theta_global

    def head_dim(self, il: int) -> int:
        return self.head_dim_local if self.is_swa_layer(il) else self.head_dim_global

    def window(self, il: int) -> int:
        """Params.sliding_window of attn_score (src/engine.ts:554)."""
        return self.sliding_window if self.is_swa_layer(il) else 0

    def apply_divisor(self, il: int) -> int:
        """rope_freqs divisor on global layers only (src/engine.ts:571-576)."""
        return 0 if self.is_swa_layer(il) else 1

    def attn_scale(self, il: int) -> float:
        return 1.0  # Gemma: q_norm/k_norm make heads unit-RMS (src/engine.ts:555-561)

    def kv_producer_for_layer(self) -> list[int]:
        """Consumers share the cache of the last unshared layer of their type (gemma4-e2b.ts:159-178)."""
        last_local, last_global = -1, -1
        for i in range(self.num_unshared_layers):
            if self.attention_is_sliding[i]:
                last_local = i
            else:
                last_global = i
        out = []
        for i in range(self.num_layers):
            if i < self.num_unshared_layers:
                out.append(i)
            else:
                out.append(last_local if self.attention_is_sliding[i] else last_global)
        return out

    def is_kv_producer_layer(self, il: int) -> bool:
        return self.kv_producer_for_layer()[il] == il


def gemma_rope_freqs(head_dim_global: int = 512, rotated_pairs: int = 64) -> np.ndarray:
    """The GGUF rope_freqs table as the engine holds it: f16, 1.0 for the first `rotated_pairs`
    entries and 1e30 (= +inf in f16) after, so trailing pairs are not rotated
    (shaders/fused_per_head_norm_rope.wgsl:4-11)."""
    t = np.full(head_dim_global // 2, 1e30, dtype=np.float32)
    t[:rotated_pairs] = 1.0
    with np.errstate(over="ignore"):
        return t.astype(np.float16)


def ring_slot_and_len(position: int, seq_len: int, ring_prefix: int | None, ring_window: int) -> tuple[int, int]:
    """R-SWA ring mapping of the deepseek-ocr long-doc mode (src/engine.ts:1962-1969): the cache
    slot written and the number of valid cache entries for a token at `position`."""
    active = ring_window > 0 and ring_prefix is not None and position >= ring_prefix
    slot = ring_prefix + ((position - ring_prefix) % ring_window) if active else position
    kv_len = min(seq_len, ring_prefix + ring_window) if active else seq_len
    return slot, kv_len
