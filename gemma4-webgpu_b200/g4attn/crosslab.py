"""crossLabDiff metrics: the reference's numeric comparison between two captures of a tensor.

Restates the statistics of src/diagnostics/cross-lab-diff.ts:76-194 (max/mean/stddev of the
absolute difference, first index over a threshold, norms, cosine similarity, and the
concentration of the difference mass) so that the B200 kernels are judged with the same report
the reference uses against its HF captures.  Adds the per-head cosine that the attention-path
tolerance is stated in.
"""
from __future__ import annotations

import numpy as np


def cross_lab_diff(ours, ref, threshold: float = 0.05, top_k: int = 20) -> dict:
    o = np.asarray(ours, dtype=np.float64).reshape(-1)
    r = np.asarray(ref, dtype=np.float64).reshape(-1)
    if o.shape != r.shape:
        raise ValueError(f"length mismatch: ours={o.size} ref={r.size}")
    n = o.size
    d = o - r
    ad = np.abs(d)
    over = np.nonzero(ad > threshold)[0]
    sum_abs = ad.sum()
    order = np.argsort(-ad, kind="stable")

    def cutoff(pct):
        k = max(1, int(np.ceil(n * pct / 100)))
        return float(ad[order[:k]].sum() / sum_abs) if sum_abs > 0 else 0.0

    sum_abs_sq = (ad * ad).sum()
    eff = (sum_abs * sum_abs) / sum_abs_sq if sum_abs_sq > 0 else 0.0
    mean = sum_abs / n if n else 0.0
    var = (d * d).sum() / n - mean * mean if n else 0.0
    cos = float((o * r).sum() / (np.sqrt((r * r).sum()) * np.sqrt((o * o).sum()) + 1e-30))
    return {
        "length": n,
        "maxAbsDiff": float(ad.max()) if n else 0.0,
        "meanAbsDiff": float(mean),
        "stddevDiff": float(np.sqrt(max(0.0, var))),
        "firstOverIndex": int(over[0]) if over.size else -1,
        "firstOverThreshold": threshold,
        "overCount": int(over.size),
        "refNorm": float(np.sqrt((r * r).sum())),
        "ourNorm": float(np.sqrt((o * o).sum())),
        "cosineSimilarity": cos,
        "topDiffs": [{"index": int(i), "ref": float(r[i]), "ours": float(o[i]), "diff": float(d[i])}
                     for i in order[:min(top_k, n)]],
        "concentration": {
            "top1PctFraction": cutoff(1),
            "top10PctFraction": cutoff(10),
            "top50PctFraction": cutoff(50),
            "participationRatio": eff / n if n else 0.0,
            "effectiveDimCount": eff,
        },
    }


def _cos_rows(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    num = (a * b).sum(axis=-1)
    den = np.sqrt((a * a).sum(axis=-1)) * np.sqrt((b * b).sum(axis=-1))
    with np.errstate(invalid="ignore", divide="ignore"):
        c = np.where(den > 0, num / np.where(den > 0, den, 1.0), np.where((a == b).all(axis=-1), 1.0, 0.0))
    return c


def head_cosines(ours, ref) -> np.ndarray:
    """Cosine of each head row: inputs [..., head_dim] (e.g. [nqh, hd] or [T, nqh, hd])."""
    a = np.asarray(ours, dtype=np.float64)
    b = np.asarray(ref, dtype=np.float64)
    return _cos_rows(a.reshape(-1, a.shape[-1]), b.reshape(-1, b.shape[-1]))


def attention_parity(ours, ref, max_abs_tol: float = 2e-3, cos_tol: float = 0.9999) -> dict:
    """The attention-path parity bar: max |diff| <= 2e-3 and every head's cosine >= 0.9999."""
    a = np.asarray(ours, dtype=np.float64)
    b = np.asarray(ref, dtype=np.float64)
    cos = head_cosines(a, b)
    mad = float(np.abs(a - b).max()) if a.size else 0.0
    finite = bool(np.isfinite(a).all())
    return {"max_abs": mad, "min_head_cos": float(cos.min()) if cos.size else 1.0,
            "ok": bool(finite and mad <= max_abs_tol and (cos.size == 0 or cos.min() >= cos_tol)),
            "max_abs_tol": max_abs_tol, "cos_tol": cos_tol}
