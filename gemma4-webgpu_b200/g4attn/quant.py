"""Host-side weight packing for the projection GEMVs (g4a_matmul), as the reference builds it.

The reference requantises each f32 weight [M, N] at load time into one of its in-shader storage
modes (src/engine.ts:107 `weightQuant`):

* Q8 (createQ8Buffers, src/engine.ts:638-674): symmetric int8 with one f16 scale per 32-element
  block; scale = amax / 127, q = round(v / scale) clamped to [-127, 127], packed 4 per uint32
  little-endian.
* Q4K (createQ4KBuffers, src/engine.ts:699-739): per 32-element sub-block an affine 4-bit grid,
  scale = (max - min) / 15, q = round((v - min) / scale) clamped to [0, 15], packed 8 per
  uint32 (nibble i at bits 4i); f16 meta per 256-element super-block: 8 scales then 8 mins.

The arithmetic follows the TypeScript: values are JS doubles, Math.round rounds halves towards
+inf (floor(x + 0.5)), and the f16 meta goes through the scalar f32ToF16 (src/gguf.ts:440-455),
which rounds the double to f32 and then truncates the mantissa (f32 subnormals become signed
zeros).  The packed arrays are what g4a_matmul takes.
"""
from __future__ import annotations

import numpy as np

__all__ = ["f32_to_f16_trunc", "quantize_q8", "quantize_q4k", "dequantize_q8", "dequantize_q4k"]


def f32_to_f16_trunc(v) -> np.ndarray:
    """The reference's scalar f32 -> f16 bit conversion (src/gguf.ts:440-455), elementwise."""
    bits = np.asarray(v, dtype=np.float64).astype(np.float32).view(np.uint32).astype(np.int64)
    sign = (bits >> 16) & 0x8000
    exp_raw = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    new_exp = exp_raw - 127 + 15
    out = sign | (new_exp << 10) | (mant >> 13)                              # normal range
    sub_shift = np.clip(1 - new_exp + 13, 0, 63)
    sub = sign | ((mant | 0x800000) >> sub_shift)                           # f16 subnormal
    out = np.where(new_exp <= 0, np.where(new_exp < -10, sign, sub), out)
    out = np.where(new_exp >= 0x1F, sign | 0x7C00, out)                     # overflow -> inf
    out = np.where(exp_raw == 0, sign, out)                                 # zero / f32 subnormal
    out = np.where(exp_raw == 0xFF, sign | 0x7C00 | np.where(mant != 0, 0x200, 0), out)
    return out.astype(np.uint16)


def _js_round(x: np.ndarray) -> np.ndarray:
    return np.floor(x + 0.5)


def quantize_q8(w: np.ndarray):
    """f32 [M, N] (N % 32 == 0) -> (qweight uint32 [M*N/4], qscale uint16 [M, N/32])."""
    w = np.asarray(w, dtype=np.float32)
    M, N = w.shape
    if N % 32:
        raise ValueError("Q8 needs N % 32 == 0")
    blk = w.astype(np.float64).reshape(M, N // 32, 32)
    amax = np.abs(blk).max(axis=2)
    scale = amax / 127.0
    with np.errstate(divide="ignore"):
        inv = np.where(scale > 0, 1.0 / np.where(scale > 0, scale, 1.0), 0.0)
    q = np.clip(_js_round(blk * inv[..., None]), -127, 127).astype(np.int64)
    qbytes = (q & 0xFF).astype(np.uint8).reshape(-1)
    return qbytes.view(np.uint32).copy(), f32_to_f16_trunc(scale)


def quantize_q4k(w: np.ndarray):
    """f32 [M, N] (N % 256 == 0) -> (qweight uint32 [M*N/8], qmeta uint16 [M, N/256, 16])."""
    w = np.asarray(w, dtype=np.float32)
    M, N = w.shape
    if N % 256:
        raise ValueError("Q4K needs N % 256 == 0")
    sub = w.astype(np.float64).reshape(M, N // 256, 8, 32)
    mn = sub.min(axis=3)
    mx = sub.max(axis=3)
    scale = (mx - mn) / 15.0
    with np.errstate(divide="ignore"):
        inv = np.where(scale > 0, 1.0 / np.where(scale > 0, scale, 1.0), 0.0)
    q = np.clip(_js_round((sub - mn[..., None]) * inv[..., None]), 0, 15).astype(np.uint32).reshape(-1)
    words = np.zeros(q.size // 8, dtype=np.uint32)
    for i in range(8):
        words |= q[i::8] << np.uint32(4 * i)
    meta = np.concatenate([f32_to_f16_trunc(scale), f32_to_f16_trunc(mn)], axis=2)  # [M, nsb, 16]
    return words, meta


def dequantize_q8(qweight: np.ndarray, qscale: np.ndarray, M: int, N: int) -> np.ndarray:
    q = np.asarray(qweight, dtype=np.uint32).view(np.int8).astype(np.float32).reshape(M, N // 32, 32)
    s = np.asarray(qscale, dtype=np.uint16).view(np.float16).astype(np.float32).reshape(M, N // 32, 1)
    return (q * s).reshape(M, N)


def dequantize_q4k(qweight: np.ndarray, qmeta: np.ndarray, M: int, N: int) -> np.ndarray:
    words = np.asarray(qweight, dtype=np.uint32)
    nib = np.stack([(words >> np.uint32(4 * i)) & np.uint32(0xF) for i in range(8)], axis=1).reshape(-1)
    nib = nib.astype(np.float32).reshape(M, N // 256, 8, 32)
    meta = np.asarray(qmeta, dtype=np.uint16).view(np.float16).astype(np.float32).reshape(M, N // 256, 16)
    return (meta[..., :8, None] * nib + meta[..., 8:, None]).reshape(M, N)
