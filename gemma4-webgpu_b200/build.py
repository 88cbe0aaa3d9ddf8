"""Build libg4attn.so (sm_100a) in-tree with nvcc.

Objects go to gemma4-webgpu_b200/_build/, the shared library to
gemma4-webgpu_b200/g4attn/libg4attn.so next to its Python host module, so it travels
with a snapshot of the repository.  Recompiles only sources newer than their object.

    python gemma4-webgpu_b200/build.py [--force] [-v] [--ptxas-v]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "g4attn" / "libg4attn.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install CUDA 12.9)")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    cc = nvcc()
    hdr = _headers_mtime()
    objs = []
    changed = force or not LIB.exists()
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            cmd = [cc] + NVCC_FLAGS + (extra_flags or []) + ["-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
            changed = True
    if changed or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [cc] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else None
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose, extra_flags=extra))
    return 0


if __name__ == "__main__":
    sys.exit(main())
