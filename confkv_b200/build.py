"""Build the in-tree sm_100a library ``confkv_b200/libgpu_aesgcm.so``.

One nvcc invocation compiles the CUDA kernels, the host key schedule / GHASH
table code and the C-ABI (``include/gpu_aesgcm_api.h``) into a shared object
that the ctypes binding loads. Usage: ``python -m confkv_b200.build [-v]``.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_NAME = "libgpu_aesgcm.so"
LIB_PATH = PKG / LIB_NAME

SOURCES = [CSRC / "gpu_aesgcm.cu", CSRC / "host_crypto.cpp"]
HEADERS = [CSRC / "kernels.cuh", CSRC / "tiles.cuh", CSRC / "batch.cuh", CSRC / "host_crypto.h", INCLUDE / "gpu_aesgcm_api.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    mtime = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in SOURCES + HEADERS + [Path(__file__)])


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and not needs_build():
        return LIB_PATH
    cmd = [
        nvcc(),
        "-O3",
        "-std=c++17",
        "-lineinfo",
        "--shared",
        "-Xcompiler=-fPIC",
        *ARCH_FLAGS,
        "-I",
        str(INCLUDE),
        "-I",
        str(CSRC),
        *(["-Xptxas", "-v"] if verbose else []),
        *[str(s) for s in SOURCES],
        "-o",
        str(LIB_PATH) + ".tmp",
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force=True))
