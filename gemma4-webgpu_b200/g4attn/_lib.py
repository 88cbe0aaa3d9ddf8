"""ctypes binding of libg4attn.so (the C ABI declared in include/g4attn.h).

The library is loaded from this package directory.  There is no fallback: if the shared
library is missing or fails to load, importing the binding raises, so a GPU run can never
silently compute on the CPU.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_size_t, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libg4attn.so"

G4A_OK = 0
STATUS_NAMES = {
    0: "G4A_OK",
    1: "G4A_EINVAL",
    2: "G4A_ECUDA",
    3: "G4A_ENOMEM",
    4: "G4A_ETIMEOUT",
    5: "G4A_ENCCL",
    6: "G4A_EUNSUPPORTED",
}


class G4AError(RuntimeError):
    """A libg4attn call returned a non-OK status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        self.status_name = STATUS_NAMES.get(status, str(status))
        self.func = func
        super().__init__(f"{func}: {self.status_name}: {message}")


WEIGHT_F16, WEIGHT_Q8, WEIGHT_Q4K = 0, 1, 2  # G4A_WEIGHT_* of g4a_matmul
MATMUL_MAX_JOBS = 4
DIST_ID_BYTES = 128  # G4A_DIST_ID_BYTES


class MatmulJob(ctypes.Structure):
    """g4a_matmul_job: one matrix of a g4a_matmul_group call."""

    _fields_ = [("weight", c_void_p), ("scales", c_void_p), ("out", c_void_p), ("M", c_uint32)]


# (name, argtypes) for every g4a_status entry point.
_u32 = c_uint32
_f = c_float
_p = c_void_p
SIGNATURES: dict[str, list] = {
    "g4a_create": [c_int, POINTER(c_void_p)],
    "g4a_destroy": [_p],
    "g4a_set_stream": [_p, _p],
    "g4a_use_own_stream": [_p],
    "g4a_sync": [_p, _u32],
    "g4a_alloc": [_p, c_size_t, POINTER(c_void_p)],
    "g4a_free": [_p, _p],
    "g4a_memcpy_h2d": [_p, _p, _p, c_size_t],
    "g4a_memcpy_d2h": [_p, _p, _p, c_size_t],
    "g4a_memset": [_p, _p, c_int, c_size_t],
    "g4a_reserve_workspace": [_p, _u32, _u32, _u32],
    "g4a_profile_enable": [_p, c_int],
    "g4a_profile_reset": [_p],
    "g4a_profile_read": [_p, c_char_p, POINTER(ctypes.c_double), POINTER(ctypes.c_uint64)],
    "g4a_norm_rope": [_p, _p, _p, _p, _u32, _u32, _f, _u32, _f, _u32],
    "g4a_rms_norm_no_weight": [_p, _p, _u32, _u32, _f],
    "g4a_kv_store": [_p, _p, _p, _p, _p, _u32, _u32, _u32, _u32, _f, _u32],
    "g4a_decode_attn": [_p, _p, _p, _p, _p, _u32, _u32, _u32, _u32, _f, _u32],
    "g4a_decode_attn_noalloc": [_p, _p, _p, _p, _p, _u32, _u32, _u32, _u32, _f, _u32],
    "g4a_decode_attn_paged": [_p, _p, _p, _p, _p, _p, _p, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _f, _u32, _p],
    "g4a_decode_attn_partial": [_p, _p, _p, _p, _u32, _u32, _u32, _u32, _u32, _u32, _f, _u32, _p],
    "g4a_lse_merge": [_p, _p, _u32, _u32, _u32, _p],
    "g4a_attn_decode_layer": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _u32, _u32, _u32, _f, _u32, _u32, _u32,
                              _u32, _f, _u32, _f, _u32, _u32],
    "g4a_attn_decode_layer_io": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _u32, _u32, _u32, _f, _u32, _u32, _u32,
                                 _u32, _f, _u32, _f, _u32, _u32],
    "g4a_prefill_qkv_prep": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _u32, _u32, _u32, _u32, _u32, _u32, _f, _f,
                             _u32],
    "g4a_prefill_attn": [_p, _p, _p, _p, _p, _u32, _u32, _u32, _u32, _u32, _f, _u32],
    "g4a_ipc_get_handle": [_p, _p, _p],
    "g4a_ipc_open_handle": [_p, _p, POINTER(c_void_p)],
    "g4a_ipc_close_handle": [_p, _p],
    "g4a_splitkv_exchange_merge": [_p, _p, POINTER(c_void_p), _u32, _u32, _u32, _u32, _u32, _p],
    "g4a_dist_unique_id": [_p],
    "g4a_dist_init": [_p, c_int, c_int, _p, _u32],
    "g4a_dist_destroy": [_p],
    "g4a_dist_info": [_p, POINTER(c_int), POINTER(c_int)],
    "g4a_allgather_partials": [_p, _p, _p, c_size_t, _u32],
    "g4a_decode_attn_splitkv": [_p, _p, _p, _p, _u32, _u32, _u32, _u32, _u32, _u32, _f, _u32, _p, _p, _u32],
    "g4a_dist_allgather_host": [_p, _p, _p, c_size_t, _u32],
    "g4a_dist_poll_selftest": [c_int, _u32, POINTER(c_int)],
    "g4a_matmul": [_p, _u32, _p, _p, _p, _p, _u32, _u32],
    "g4a_matmul_group": [_p, _u32, _p, _u32, POINTER(MatmulJob), _u32],
}
EXTRA_SYMBOLS = {"g4a_last_error": ([], c_char_p), "g4a_version": ([], c_char_p),
                 "g4a_get_stream": ([c_void_p], c_void_p),
                 "g4a_exchange_buffer_bytes": ([c_uint32, c_uint32, c_uint32], c_size_t)}

_lib = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the shared library with argtypes set."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"libg4attn.so not found at {p}; build it with `python gemma4-webgpu_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = c_int
    for name, (argtypes, restype) in EXTRA_SYMBOLS.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    if path is None:
        _lib = lib
    return lib


def call(name: str, *args) -> None:
    """Call an entry point and raise G4AError on a non-OK status."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != G4A_OK:
        msg = lib.g4a_last_error()
        raise G4AError(st, name, msg.decode() if msg else "")


def exported_symbols() -> list[str]:
    return sorted(list(SIGNATURES) + list(EXTRA_SYMBOLS))
