"""Seeded synthetic inputs with the shapes of the benchmark configurations.

No model weights or prompts are involved: every configuration is a synthetic shape.  The
recipe for all configurations: raw q/k/v rows ~ N(0, 1) (f32); q and k go through the per-head
RMSNorm with an f16 weight 1 + N(0, 0.05) and RoPE at their true positions (theta per layer);
v goes through the weightless RMSNorm; K/V land in the f16 cache.  Those transforms are exactly
the producer kernels of the hot path, so the raw arrays generated here are fed to the producer
entry points (GPU) and to the CPU oracle alike.

Seeds: numpy ``default_rng(seed)``, seed 0 for the sliding-decode config and the config index
otherwise.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

EPS = 1e-6


@dataclass
class RawLayer:
    q: np.ndarray        # [Tq, nqh, hd] f32 raw (pre-norm) queries
    k: np.ndarray        # [L, nkh, hd] f32 raw keys for positions 0..L-1
    v: np.ndarray        # [L, nkh, hd] f32 raw values
    q_w: np.ndarray      # [hd] f16 q_norm weight
    k_w: np.ndarray      # [hd] f16 k_norm weight
    theta: float
    window: int
    q_pos0: int          # position of q row 0


def norm_weight(rng: np.random.Generator, hd: int) -> np.ndarray:
    return (1.0 + 0.05 * rng.standard_normal(hd)).astype(np.float32).astype(np.float16)


def raw_layer(seed: int, L: int, nqh: int = 8, nkh: int = 1, hd: int = 256, theta: float = 1e4,
              window: int = 0, Tq: int = 1, q_pos0: int | None = None) -> RawLayer:
    """Raw inputs of one attention layer: a KV history of L tokens and Tq query rows.

    By default the query rows sit at the last Tq positions (decode of the last token)."""
    rng = np.random.default_rng(seed)
    q_w = norm_weight(rng, hd)
    k_w = norm_weight(rng, hd)
    k = rng.standard_normal((L, nkh, hd), dtype=np.float32)
    v = rng.standard_normal((L, nkh, hd), dtype=np.float32)
    q = rng.standard_normal((Tq, nqh, hd), dtype=np.float32)
    if q_pos0 is None:
        q_pos0 = max(L - Tq, 0)
    return RawLayer(q=q, k=k, v=v, q_w=q_w, k_w=k_w, theta=theta, window=window, q_pos0=q_pos0)


def batched_lengths(seed: int = 2, batch: int = 64, lo: int = 1024, hi: int = 32768) -> np.ndarray:
    """Context lengths of the batched-decode config: U[lo, hi] inclusive, seeded."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=batch).astype(np.int32)


def page_assignment(seed: int, lengths: np.ndarray, page_size: int = 64, extra_pages: int = 0):
    """Page table for a paged cache: every sequence's pages drawn from one seeded random
    permutation of the pool.  Returns (page_table [B, max_pages] int32, num_pages)."""
    rng = np.random.default_rng(seed + 1000)
    pages_per = (lengths.astype(np.int64) + page_size - 1) // page_size
    total = int(pages_per.sum()) + extra_pages
    perm = rng.permutation(max(total, 1)).astype(np.int32)
    max_pages = int(pages_per.max()) if len(pages_per) else 1
    table = np.zeros((len(lengths), max(max_pages, 1)), dtype=np.int32)
    off = 0
    for b, n in enumerate(pages_per):
        table[b, :n] = perm[off:off + n]
        off += n
    return table, max(total, 1)


def kv_bytes_decode(L: int, window: int, nkh: int = 1, hd: int = 256, nqh: int = 8) -> int:
    """Algorithmic bytes of one decode layer-call: visible K and V rows (f16) + q in + out (f32)."""
    vis = min(L, window) if window else L
    return 2 * vis * nkh * hd * 2 + 2 * nqh * hd * 4


def prefill_flops(T: int, window: int, nqh: int = 8, hd: int = 256, start_pos: int = 0) -> int:
    """Algorithmic FLOPs of prefill attention (QK^T and PV over visible pairs only)."""
    kv = np.arange(start_pos + 1, start_pos + T + 1, dtype=np.int64)
    pairs = np.minimum(kv, window).sum() if window else kv.sum()
    return int(4 * nqh * hd * pairs)
