"""Ahead-of-time build of the layer's CUDA library for sm_100a.

The reference JIT-compiles its extension on the first call
(``solution/python/kernel.py:57-92``); here ``nvcc`` builds one plain C-ABI
shared library, ``libmoe_fp8_ds.so``, next to this file before any call, so
no compiler runs on the serving path.
"""

from __future__ import annotations

import os
import pathlib
import shutil
import subprocess

PKG_DIR = pathlib.Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_NAME = "libmoe_fp8_ds.so"
LIB_PATH = PKG_DIR / LIB_NAME
SOURCES = ("api.cu", "route_permute.cu", "gemm_fp8.cu", "gemm_tm.cu", "noalloc.cu", "ep.cu")
HEADERS = ("common.cuh", "kernels.cuh")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _inputs():
    inc = PKG_DIR.parent / "include" / "moe_fp8_ds.h"
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [inc]


STAMP_PATH = PKG_DIR / (LIB_NAME + ".stamp")


def sources_digest() -> str:
    """sha256 over the build inputs and flags (the stamp a build leaves next to the library)."""
    import hashlib
    h = hashlib.sha256(" ".join(ARG_FLAGS_FOR_STAMP()).encode())
    for p in _inputs():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def ARG_FLAGS_FOR_STAMP():
    return ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17"]


def is_stale() -> bool:
    """True when the library is missing or was built from different sources."""
    if not LIB_PATH.exists() or not STAMP_PATH.exists():
        return True
    return STAMP_PATH.read_text().strip() != sources_digest()


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compile ``libmoe_fp8_ds.so`` (sm_100a) if missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    cmd = [_nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "-o", str(LIB_PATH) + ".tmp", *[str(CSRC / s) for s in SOURCES], "-lcudart"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=str(PKG_DIR))
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    STAMP_PATH.write_text(sources_digest() + "\n")
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
