"""Measured issue rates of the instructions the seal/open kernels use.

Runs the microbenchmark in ``csrc/pipe_rates.cu`` (``libpipe_rates.so``) on
the current CUDA device and reports, per instruction, how many are executed
per SM per SM clock (counted in threads: one 32-lane warp instruction = 32).
These are the peaks of the integer-pipe and shared-memory bounds bench.py
reports; `python -m confkv_b200.pipe_rates` prints them as JSON.

Each kernel runs one CTA of 1024 threads per SM, 8 independent dependency
chains per thread, 128 instructions per loop iteration, and times its loop
with %clock64 on every SM.
"""

from __future__ import annotations

import ctypes
import json

from . import build

OPS = ("lop3", "iadd", "prmt", "shf", "imad", "imad_wide", "imad_hi", "lds32", "lds128", "lop3_imad_mix", "shfl",
       "lds32_shfl_mix")


def _lib():
    lib = ctypes.CDLL(str(build.build_pipe_rates()))
    lib.pipe_rates_run.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                   ctypes.POINTER(ctypes.c_double)]
    lib.pipe_rates_run.restype = ctypes.c_int
    return lib


def measure(iters: int = 2048) -> dict:
    """{op: {"per_sm_clk": threads' instructions per SM per clock, "cycles": loop cycles}}."""
    lib = _lib()
    out = {}
    for i, name in enumerate(OPS):
        rate, cyc = ctypes.c_double(), ctypes.c_double()
        rc = lib.pipe_rates_run(i, iters, ctypes.byref(rate), ctypes.byref(cyc))
        if rc != 0:
            raise RuntimeError(f"pipe_rates_run({name}) failed: rc {rc}")
        out[name] = {"per_sm_clk": round(rate.value, 2), "cycles": round(cyc.value)}
    return out


if __name__ == "__main__":
    import torch

    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    print(json.dumps({"gpu": props.name, "sms": props.multi_processor_count, "rates": measure()}))


def model_peaks(rates: dict) -> dict:
    """Per-SM-per-clock peaks of the units the seal/open kernels load, from
    measured rates: shared-memory wavefronts (one LDS.32 warp instruction on
    32 banks is one wavefront), ALU-pipe instructions (LOP3), FMA-pipe
    instructions (IMAD) and issued instructions (LOP3 and IMAD interleaved),
    all in threads (one warp instruction = 32)."""
    r = {k: v["per_sm_clk"] for k, v in rates.items()}
    return {"l1_wavefronts": r["lds32"] / 32.0, "alu": r["lop3"], "fma": r["imad"], "issue": r["lop3_imad_mix"]}
