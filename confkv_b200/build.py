"""Build the in-tree sm_100a library ``confkv_b200/libgpu_aesgcm.so``.

nvcc compiles the CUDA kernels and C-ABI (gpu_aesgcm.cu: per-object calls;
batch.cu: batched calls) and the host key schedule / GHASH table code in
parallel, then links them into the shared object that the ctypes binding
loads (``include/gpu_aesgcm_api.h``). Usage: ``python -m confkv_b200.build [-v]``.
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

SOURCES = [CSRC / "gpu_aesgcm.cu", CSRC / "batch.cu", CSRC / "host_crypto.cpp"]
HEADERS = [CSRC / "kernels.cuh", CSRC / "clmul.cuh", CSRC / "gh5.cuh", CSRC / "tiles.cuh", CSRC / "batch.cuh", CSRC / "small.cuh", CSRC / "host_common.h",
           CSRC / "host_crypto.h", INCLUDE / "gpu_aesgcm_api.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    mtime = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in SOURCES + HEADERS + [Path(__file__)])


def _compile_cmd(src: Path, obj: Path, verbose: bool) -> list[str]:
    return [nvcc(), "-O3", "-std=c++17", "-lineinfo", "-c", "-Xcompiler=-fPIC", *ARCH_FLAGS,
            "-I", str(INCLUDE), "-I", str(CSRC), *(["-Xptxas", "-v"] if verbose else []), str(src), "-o", str(obj)]


PIPE_RATES_SRC = CSRC / "pipe_rates.cu"
PIPE_RATES_LIB = PKG / "libpipe_rates.so"


def build_pipe_rates(force: bool = False) -> Path:
    """The issue-rate microbenchmark (csrc/pipe_rates.cu) as its own shared
    library: a measurement tool, not part of the seal/open C-ABI."""
    if not force and PIPE_RATES_LIB.exists() and PIPE_RATES_LIB.stat().st_mtime >= PIPE_RATES_SRC.stat().st_mtime:
        return PIPE_RATES_LIB
    cmd = [nvcc(), "-O3", "-std=c++17", "-lineinfo", "--shared", "-Xcompiler=-fPIC", *ARCH_FLAGS,
           str(PIPE_RATES_SRC), "-o", str(PIPE_RATES_LIB) + ".tmp"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"pipe_rates build failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(str(PIPE_RATES_LIB) + ".tmp", PIPE_RATES_LIB)
    return PIPE_RATES_LIB


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile each source to an object in parallel, then link the shared
    library next to this file (atomically replaced)."""
    if not force and not needs_build():
        return LIB_PATH
    import tempfile

    with tempfile.TemporaryDirectory(prefix="confkv_b200_build_") as tmp:
        objs = [Path(tmp) / (src.stem + ".o") for src in SOURCES]
        procs = [subprocess.Popen(_compile_cmd(src, obj, verbose), stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                  text=True) for src, obj in zip(SOURCES, objs)]
        errors = []
        for src, p in zip(SOURCES, procs):
            out, err = p.communicate()
            if verbose:
                sys.stderr.write(err)
            if p.returncode != 0:
                errors.append(f"{src.name}: nvcc failed ({p.returncode}):\n{out}\n{err}")
        if errors:
            raise RuntimeError("\n".join(errors))
        link = [nvcc(), "--shared", *ARCH_FLAGS, *[str(o) for o in objs], "-o", str(LIB_PATH) + ".tmp"]
        res = subprocess.run(link, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force=True))
    print(build_pipe_rates(force=True))
