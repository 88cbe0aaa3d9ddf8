"""The C ABI library loads, exports every symbol include/g4attn.h declares, and the Python
binding's argument lists match the header.  No GPU compute is run here."""
import ctypes
import re
from pathlib import Path

import pytest

import g4attn
from g4attn import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "g4attn.h"


def header_decls() -> dict[str, int]:
    """name -> number of parameters of every function declared in the header."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"^[\w\s\*]*?\b(g4a_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.M | re.S):
        name, args = m.group(1), m.group(2).strip()
        out[name] = 0 if args in ("", "void") else len(args.split(","))
    return out


def test_library_loads_and_reports_version():
    lib = _lib.load()
    assert g4attn.version().startswith("g4attn ")
    assert "sm_100a" in g4attn.version()
    assert lib.g4a_last_error() is not None


def test_every_declared_symbol_is_exported():
    decls = header_decls()
    assert len(decls) >= 25
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in decls if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_matches_header_arity():
    decls = header_decls()
    bound = {**{k: len(v) for k, v in _lib.SIGNATURES.items()},
             **{k: len(v[0]) for k, v in _lib.EXTRA_SYMBOLS.items()}}
    assert set(bound) == set(decls), (set(decls) ^ set(bound))
    for name, n in decls.items():
        assert bound[name] == n, (name, bound[name], n)


def test_null_context_is_rejected_without_a_gpu():
    lib = _lib.load()
    st = lib.g4a_decode_attn(None, None, None, None, None, 8, 1, 256, 10, 1.0, 0)
    assert st == 1  # G4A_EINVAL
    assert b"null context" in lib.g4a_last_error()
    assert lib.g4a_sync(None, 0) == 1
    assert lib.g4a_destroy(None) == 0


def test_status_error_carries_message():
    with pytest.raises(g4attn.G4AError) as ei:
        _lib.call("g4a_norm_rope", None, None, None, None, 1, 256, 1e-6, 0, 1e4, 0)
    assert ei.value.status_name == "G4A_EINVAL"
    assert "null context" in str(ei.value)


def test_create_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = _lib.load().g4a_create(0, ctypes.byref(h))
    assert st != 0 and not h.value
    assert _lib.load().g4a_last_error()


def test_every_context_entry_rejects_a_null_context():
    """Every entry point that takes a context checks it before anything else: with a null context
    (and null / zero for the rest) it returns G4A_EINVAL with a message and touches no device."""
    lib = _lib.load()
    # create, the NCCL unique id and the communicator self-test take no context; destroy(NULL)
    # is a no-op
    skip = {"g4a_create", "g4a_destroy", "g4a_dist_unique_id", "g4a_dist_poll_selftest"}
    checked = 0
    for name, argtypes in _lib.SIGNATURES.items():
        if name in skip:
            continue
        args = []
        for t in argtypes:
            if t in (ctypes.c_float, ctypes.c_double):
                args.append(t(0.0))
            elif t in (ctypes.c_uint32, ctypes.c_int, ctypes.c_size_t):
                args.append(t(0))
            else:
                args.append(None)
        st = getattr(lib, name)(*args)
        assert st == 1, (name, st)
        assert b"null context" in lib.g4a_last_error(), name
        checked += 1
    assert checked >= 25
