"""Python front-end of the CPU oracle (oracle.c).  TEST INFRASTRUCTURE ONLY.

Only the test-suite, the smoke check and the benchmark's CPU-baseline leg import this module;
the product path never does.  It wraps the C restatement of the reference's WGSL attention
chain and adds the glue the tests need: building f16 caches from raw inputs with the
reference's producer order, gathering a paged cache back to a contiguous one, prefill as a
loop of decode steps (src/engine.ts:2460-2479), and a numpy twin of the attention math.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_size_t, c_uint16, c_uint32
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
            build()
        L = ctypes.CDLL(str(LIB))
        f32p, u16p, f64p = POINTER(c_float), POINTER(c_uint16), POINTER(c_double)
        u = c_uint32
        L.orc_half_to_float.argtypes = [c_uint16]
        L.orc_half_to_float.restype = c_float
        L.orc_float_to_half.argtypes = [c_float]
        L.orc_float_to_half.restype = c_uint16
        L.orc_f32_to_f16_array.argtypes = [f32p, u16p, c_size_t]
        L.orc_f16_to_f32_array.argtypes = [u16p, f32p, c_size_t]
        L.orc_rope_base_freq.argtypes = [c_float, u, u]
        L.orc_rope_base_freq.restype = c_float
        L.orc_norm_rope.argtypes = [f32p, u16p, u16p, u, u, c_float, u, c_float, u]
        L.orc_rms_norm_no_weight.argtypes = [f32p, u, u, c_float]
        L.orc_kv_cache_store_f32.argtypes = [f32p, f32p, f32p, f32p, u, u, u]
        L.orc_kv_cache_store_f16.argtypes = [f32p, f32p, u16p, u16p, u, u, u]
        L.orc_window_start.argtypes = [u, u]
        L.orc_window_start.restype = u
        L.orc_attn_score.argtypes = [f32p, f32p, f32p, u, u, u, u, c_float, u]
        L.orc_softmax.argtypes = [f32p, u, u]
        L.orc_attn_output.argtypes = [f32p, f32p, f32p, u, u, u, u]
        L.orc_decode_chain_f32.argtypes = [f32p, f32p, f32p, f32p, f32p, u, u, u, u, c_float, u]
        L.orc_decode_attn_f64.argtypes = [f32p, u16p, u16p, f32p, u, u, u, u, c_float, u]
        L.orc_decode_partial_f64.argtypes = [f32p, u16p, u16p, u, u, u, u, u, u, c_float, u, f64p, f64p, f64p]
        L.orc_prefill_attn_f64.argtypes = [f32p, u16p, u16p, f32p, u, u, u, u, u, c_float, u]
        u32p = POINTER(c_uint32)
        L.orc_matmul_f16.argtypes = [f32p, u16p, f32p, u, u]
        L.orc_matmul_q8.argtypes = [f32p, u32p, u16p, f32p, u, u]
        L.orc_matmul_q4k.argtypes = [f32p, u32p, u16p, f32p, u, u]
        L.orc_num_threads.restype = c_int
        L.orc_set_num_threads.argtypes = [c_int]
        _lib = L
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(POINTER(c_float))


def _u16(a):
    if a is None:
        return None, None
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    a = np.ascontiguousarray(a, dtype=np.uint16)
    return a, a.ctypes.data_as(POINTER(c_uint16))


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


# ------------------------------------------------------------------ f16
def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x, px = _f32(x)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_array(px, out.ctypes.data_as(POINTER(c_uint16)), x.size)
    return out.view(np.float16)


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h, ph = _u16(h)
    out = np.empty(h.shape, dtype=np.float32)
    lib().orc_f16_to_f32_array(ph, out.ctypes.data_as(POINTER(c_float)), h.size)
    return out


# ------------------------------------------------------------------ producers
def rope_base_freq(theta: float, i: int, head_dim: int) -> float:
    return lib().orc_rope_base_freq(theta, i, head_dim)


def norm_rope(x, weight, rope_freqs, *, num_heads, head_dim, eps, position, theta, apply_divisor=0):
    """fused_per_head_norm_rope.wgsl on a copy of x (f32 [num_heads, head_dim])."""
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    w, pw = _u16(weight)
    rf, prf = _u16(rope_freqs) if rope_freqs is not None else (None, None)
    lib().orc_norm_rope(x.ctypes.data_as(POINTER(c_float)), pw, prf, num_heads, head_dim, eps, position, theta,
                        apply_divisor)
    return x


def rms_norm_no_weight(x, *, num_heads, head_dim, eps):
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().orc_rms_norm_no_weight(x.ctypes.data_as(POINTER(c_float)), num_heads, head_dim, eps)
    return x


def build_cache(raw_k, raw_v, k_w, *, theta, eps=1e-6, apply_divisor=0, rope_freqs=None, positions=None):
    """Producer path for every cached token: k -> norm+RoPE at its position, v -> v_norm, both
    stored f16 (src/engine.ts:2061-2091 per token).  raw_k/raw_v: [L, nkh, hd].
    Returns (k_cache f16 [L, nkh, hd], v_cache f16 [L, nkh, hd])."""
    L, nkh, hd = raw_k.shape
    kc = np.empty((L, nkh, hd), dtype=np.float16)
    vc = np.empty((L, nkh, hd), dtype=np.float16)
    for t in range(L):
        pos = t if positions is None else int(positions[t])
        kn = norm_rope(raw_k[t], k_w, rope_freqs, num_heads=nkh, head_dim=hd, eps=eps, position=pos, theta=theta,
                       apply_divisor=apply_divisor)
        vn = rms_norm_no_weight(raw_v[t], num_heads=nkh, head_dim=hd, eps=eps)
        kc[t] = f32_to_f16(kn)
        vc[t] = f32_to_f16(vn)
    return kc, vc


def window_start(seq_len: int, sliding_window: int) -> int:
    return lib().orc_window_start(seq_len, sliding_window)


# ------------------------------------------------------------------ attention
def decode_chain_f32(q, k_cache_f32, v_cache_f32, *, num_q_heads, num_kv_heads, head_dim, seq_len, scale=1.0,
                     sliding_window=0):
    """The reference chain in WGSL order over f32 caches (attn_score, softmax, attn_output)."""
    q, pq = _f32(q)
    k, pk = _f32(k_cache_f32)
    v, pv = _f32(v_cache_f32)
    out = np.zeros(num_q_heads * head_dim, dtype=np.float32)
    work = np.zeros(max(num_q_heads * seq_len, 1), dtype=np.float32)
    lib().orc_decode_chain_f32(pq, pk, pv, out.ctypes.data_as(POINTER(c_float)),
                               work.ctypes.data_as(POINTER(c_float)), num_q_heads, num_kv_heads, head_dim, seq_len,
                               scale, sliding_window)
    return out.reshape(num_q_heads, head_dim)


def decode_attn_f64(q, k_cache, v_cache, *, num_q_heads, num_kv_heads, head_dim, kv_len, scale=1.0,
                    sliding_window=0):
    """fp64-accumulated golden over f16 caches ([>=kv_len, nkh, hd])."""
    q, pq = _f32(q)
    k, pk = _u16(k_cache)
    v, pv = _u16(v_cache)
    out = np.zeros(num_q_heads * head_dim, dtype=np.float32)
    lib().orc_decode_attn_f64(pq, pk, pv, out.ctypes.data_as(POINTER(c_float)), num_q_heads, num_kv_heads,
                              head_dim, kv_len, scale, sliding_window)
    return out.reshape(num_q_heads, head_dim)


def decode_partial_f64(q, k_cache, v_cache, *, num_q_heads, num_kv_heads, head_dim, kv_begin, kv_end, kv_len,
                       scale=1.0, sliding_window=0):
    """(m, l, o) in natural-log units over positions [kv_begin, kv_end) of a full cache."""
    q, pq = _f32(q)
    k, pk = _u16(k_cache)
    v, pv = _u16(v_cache)
    m = np.zeros(num_q_heads, dtype=np.float64)
    l_ = np.zeros(num_q_heads, dtype=np.float64)
    o = np.zeros(num_q_heads * head_dim, dtype=np.float64)
    dp = POINTER(c_double)
    lib().orc_decode_partial_f64(pq, pk, pv, num_q_heads, num_kv_heads, head_dim, kv_begin, kv_end, kv_len, scale,
                                 sliding_window, m.ctypes.data_as(dp), l_.ctypes.data_as(dp), o.ctypes.data_as(dp))
    return m, l_, o.reshape(num_q_heads, head_dim)


def prefill_rows_f64(q, k_cache, v_cache, rows, *, start_pos, num_q_heads, num_kv_heads, head_dim, scale=1.0,
                     sliding_window=0):
    """Selected rows of prefill attention: row i is decode at kv_len = start_pos + i + 1.
    q: [T, nqh, hd] f32 (f16-valued when the kernel takes f16 Q)."""
    out = np.zeros((len(rows), num_q_heads, head_dim), dtype=np.float32)
    for n, i in enumerate(rows):
        out[n] = decode_attn_f64(q[i], k_cache, v_cache, num_q_heads=num_q_heads, num_kv_heads=num_kv_heads,
                                 head_dim=head_dim, kv_len=start_pos + i + 1, scale=scale,
                                 sliding_window=sliding_window)
    return out


def gather_pages(pages: np.ndarray, page_table_row: np.ndarray, kv_len: int, page_size: int) -> np.ndarray:
    """Contiguous [kv_len, nkh, hd] copy of one sequence of a paged pool [num_pages, page_size, nkh, hd]."""
    n = (kv_len + page_size - 1) // page_size
    rows = pages[page_table_row[:n]].reshape(n * page_size, *pages.shape[2:])
    return np.ascontiguousarray(rows[:kv_len])


# ------------------------------------------------------------------ numpy twin
def decode_numpy_f64(q, k_cache, v_cache, kv_len, window=0, scale=1.0, nkh=1):
    """Independent numpy restatement (float64) of decode attention, for cross-checking the C oracle."""
    nqh, hd = q.shape
    ws = 0 if (window == 0 or kv_len <= window) else kv_len - window
    out = np.zeros((nqh, hd), dtype=np.float64)
    if kv_len == 0:
        return out.astype(np.float32)
    K = k_cache[ws:kv_len].astype(np.float64)
    V = v_cache[ws:kv_len].astype(np.float64)
    for h in range(nqh):
        kvh = h * nkh // nqh
        s = (K[:, kvh, :] @ q[h].astype(np.float64)) * scale
        p = np.exp(s - s.max())
        out[h] = (p @ V[:, kvh, :]) / p.sum()
    return out.astype(np.float32)


def matmul(weight_format: int, x, weight, scales, M: int, N: int) -> np.ndarray:
    """out[m] = sum_k W[m, k] x[k] in the reference shaders' order (orc_matmul_*).
    weight_format 0 = f16 (weight uint16 [M, N]), 1 = Q8 (weight uint32 [M*N/4], scales uint16
    [M, N/32]), 2 = Q4K (weight uint32 [M*N/8], scales uint16 [M, N/256, 16])."""
    x, px = _f32(np.asarray(x).reshape(-1))
    assert x.size >= N
    out = np.zeros(M, dtype=np.float32)
    pout = out.ctypes.data_as(POINTER(c_float))
    w = np.ascontiguousarray(weight).reshape(-1)
    if weight_format == 0:
        w, pw = _u16(w.view(np.uint16))
        lib().orc_matmul_f16(px, pw, pout, M, N)
    else:
        w = np.ascontiguousarray(w.view(np.uint32))
        s, ps = _u16(np.ascontiguousarray(scales).reshape(-1).view(np.uint16))
        fn = lib().orc_matmul_q8 if weight_format == 1 else lib().orc_matmul_q4k
        fn(px, w.ctypes.data_as(POINTER(c_uint32)), ps, pout, M, N)
    return out
