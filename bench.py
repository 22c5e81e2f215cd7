#!/usr/bin/env python3
"""Benchmark: AES-128-GCM seal + authenticated open of Llama-3-8B KV chunks.

One step = seal a batch of 32 KV objects [2, 32 layers, 256 tokens, 8 KV heads,
128] bf16 (32 MiB each, N(0,1), seeded; inputs resident in HBM) into frames
[1 | IV | ct | tag], then open all 32 frames with tag verification. Each GPU
(one process per GPU under torchrun) seals its own 32 objects: no collective
on the data path, weak scaling. value = plaintext bytes sealed + opened by all
ranks / max-over-ranks device time, through one batched seal call and one
batched open call per step; the same step through one seal_async / open_async
call per object (the reference's C-ABI) is reported beside it ("per_object"),
and e2e (host buffers, copies timed) goes through the per-object calls.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--api both|batched|per_object]

--impl reference times the reference's own OpenSSL CPU backend
(lmcache_aes128gcm_seal/open from oracle/_ref/libcpu_seal.so, driven by the
native pthread loop oracle/_ref/libcpu_threads.so) on the host cores with one
thread per core, on the same objects, metric and unit.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
from pathlib import Path


ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "AES-GCM seal/open GB/s (32 MiB KV objects) at 1/2/4/8 B200 vs OpenSSL host"
UNIT = "GB/s"
SHAPE = (2, 32, 256, 8, 128)  # workloads.BENCH_SHAPE
OBJECTS = 32  # objects per GPU per step in the benchmarked workload (workloads.BENCH_OBJECTS)
WORKLOAD = "llama3_8b_kv_chunk_32MiB_x32_seal_then_open"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--api", choices=["both", "batched", "per_object"], default="both",
                    help="both: value from the batched calls, per-object calls reported beside it")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg (profiling runs)")
    ap.add_argument("--objects", type=int, default=OBJECTS, help="objects per GPU per step (profiling runs)")
    ap.add_argument("--cpu-sample-objects", type=int, default=0,
                    help="objects per OpenSSL thread in the cpu_baseline sample (0 = auto)")
    ap.add_argument("--cpu-sweep", action="store_true",
                    help="with --impl reference: also time seal and open of single objects 4 KiB..1 GiB "
                         "on all host cores (the CPU side of the size sweep), one JSON line per size")
    return ap.parse_args()


def dist_env():
    from confkv_b200.multigpu import rank_env

    return rank_env()


def load_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


KERNEL_PROFILE = "batched_kernels_kv_llama8b.md"
PIPE_RATES_PROFILE = "pipe_rates_b200.md"
SEAL_TWO_PASS_MIN_BYTES = 80 << 20  # kSealTwoPassMinBytes: per-object seals from this size take two launches


def kernel_profile(name: str = KERNEL_PROFILE) -> dict:
    """Per-kernel costs per 16-byte block from a committed ncu summary under
    profiles/: lines `kernel <name> call=<seal|open> wavefronts=<L1 data-pipe
    wavefronts> alu=<ALU-pipe instructions> fma=<FMA-pipe busy SM clocks>
    issue=<instructions> dram=<DRAM bytes>` (instructions in threads)."""
    p = ROOT / "profiles" / name
    out = {}
    if not p.exists():
        return out
    for line in p.read_text().splitlines():
        parts = line.strip().split()
        if len(parts) < 3 or parts[0] != "kernel":
            continue
        rec = {}
        for kv in parts[2:]:
            k, _, v = kv.partition("=")
            try:
                rec[k] = float(v)
            except ValueError:
                rec[k] = v
        out[parts[1]] = rec
    return out


def committed_pipe_peaks() -> dict | None:
    """`peak <unit>=<per SM per clock>` lines of the committed microbenchmark summary."""
    p = ROOT / "profiles" / PIPE_RATES_PROFILE
    if not p.exists():
        return None
    out = {}
    for line in p.read_text().splitlines():
        parts = line.strip().split()
        if parts and parts[0] == "peak":
            for kv in parts[1:]:
                k, _, v = kv.partition("=")
                out[k] = float(v)
    return out or None


def pipe_roofline(prof: dict, call: str, peaks: dict, n_sm: int, sm_hz: float, achieved_gbs: float) -> dict:
    """Ceiling of one call (its kernels run one after another) from the
    per-block costs of its kernels at the measured per-SM peaks: each kernel
    needs max over units of (units per block / units per SM per clock) SM
    clocks per block; the call needs their sum."""
    kernels = {}
    total = 0.0
    for name, rec in prof.items():
        if rec.get("call") != call:
            continue
        # fma: FMA-pipe busy clocks per block as ncu counts them (an IMAD.WIDE
        # holds the pipe about two cycles, so instructions / rate would undercount)
        clk = {"l1_wavefronts": rec["wavefronts"] / peaks["l1_wavefronts"], "alu": rec["alu"] / peaks["alu"],
               "fma": rec["fma"], "issue": rec["issue"] / peaks["issue"]}
        bind = max(clk, key=clk.get)
        kernels[name] = {"clocks_per_block": {u: round(v, 3) for u, v in clk.items()}, "binding": bind}
        total += clk[bind]
    if total == 0.0:
        return {}
    ceiling = n_sm * sm_hz / total * 16 / 1e9
    return {"kernels": kernels, "ceiling_plaintext_gbs": round(ceiling, 1),
            "achieved_plaintext_gbs": round(achieved_gbs, 1), "frac": round(achieved_gbs / ceiling, 3)}


# ----------------------------------------------------------------- ours

def run_ours(args, rank, world, local):
    import torch

    from confkv_b200 import build, workloads
    from confkv_b200.batch import DeviceBatch
    from confkv_b200.gpu_aesgcm import GpuAes128GcmKey, GpuAesGcmLibrary

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if rank == 0:
        build.build()
    if world > 1:
        torch.distributed.barrier()
    lib = GpuAesGcmLibrary()

    nobj = args.objects
    case = workloads.bench_case(rank, nobj, device=dev)  # this rank's objects, resident in HBM
    P = case.object_bytes
    frame_len = P + 29
    stride = case.frame_stride
    key_bytes, ivs, plain_u8 = case.key, case.ivs, case.plain
    key = GpuAes128GcmKey(lib, key_bytes, device=local)
    key.reserve(P)
    frames = torch.empty((nobj, stride), dtype=torch.uint8, device=dev)
    opened = torch.empty((nobj, P), dtype=torch.uint8, device=dev)
    auth = torch.zeros((nobj,), dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream

    # per-object calls: the reference's C-ABI, one seal_async / open_async each
    def seal_each():
        for k in range(nobj):
            key.seal_async(src_ptr=plain_u8[k].data_ptr(), plaintext_len=P, dst_ptr=frames[k].data_ptr(),
                           dst_capacity=stride, iv=ivs[k], stream_ptr=sp)

    def open_each():
        for k in range(nobj):
            key.open_async(src_ptr=frames[k].data_ptr(), frame_len=frame_len, dst_ptr=opened[k].data_ptr(),
                           plaintext_len=P, auth_ok_ptr=auth[k:k + 1].data_ptr(), stream_ptr=sp)

    # batched calls: one seal_batch_async / open_batch_async per step over the
    # same objects; the descriptor arrays are device-resident like the inputs
    bseal = DeviceBatch(lib, nobj, dev)
    bopen = DeviceBatch(lib, nobj, dev)
    bseal.seal(key, [(plain_u8[k].data_ptr(), frames[k].data_ptr(), P, stride, ivs[k]) for k in range(nobj)], stream)
    bopen.open(key, [(frames[k].data_ptr(), opened[k].data_ptr(), P, frame_len, auth.data_ptr() + 4 * k)
                     for k in range(nobj)], stream)

    def seal_batched():
        key.seal_batch_async(items_ptr=bseal.items.data_ptr(), count=nobj, workspace_ptr=bseal.workspace.data_ptr(),
                             workspace_bytes=bseal.workspace_bytes, stream_ptr=sp)

    def open_batched():
        key.open_batch_async(items_ptr=bopen.items.data_ptr(), count=nobj, workspace_ptr=bopen.workspace.data_ptr(),
                             workspace_bytes=bopen.workspace_bytes, stream_ptr=sp)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    def measure(seal_fn, open_fn):
        """W warm-up steps, then K steps timed with events on the launching
        stream; checks every object's round trip afterwards."""
        opened.zero_()
        auth.zero_()
        barrier()
        for _ in range(args.warmup):
            seal_fn()
            open_fn()
        barrier()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        barrier()
        with torch.cuda.stream(stream):
            for s in range(args.steps):
                ev[s][0].record(stream)
                seal_fn()
                ev[s][1].record(stream)
                open_fn()
                ev[s][2].record(stream)
        barrier()
        seal_ms = [e[0].elapsed_time(e[1]) for e in ev]
        open_ms = [e[1].elapsed_time(e[2]) for e in ev]
        ok = bool((auth == 1).all()) and torch.equal(opened, plain_u8)
        return seal_ms, open_ms, ok

    from confkv_b200 import multigpu
    from confkv_b200.clocks import ClockSampler

    # the headline call style is measured last, so `frames` holds its last
    # timed step's output for the OpenSSL comparison below
    apis = ["per_object", "batched"] if args.api == "both" else [args.api]
    clocks = ClockSampler(local)
    clocks.start()
    results = {}
    for api in apis:
        seal_ms, open_ms, ok = measure(seal_batched, open_batched) if api == "batched" else \
            measure(seal_each, open_each)
        tot, ssum, osum = multigpu.reduce_max([sum(a + b for a, b in zip(seal_ms, open_ms)), sum(seal_ms),
                                               sum(open_ms)], device=dev)
        results[api] = (tot, ssum, osum, multigpu.all_ok(ok, device=dev))
    clk = clocks.stop()
    frames_check = frames_match_openssl(frames, plain_u8, ivs, key_bytes, P)
    frames_check["match"] = multigpu.all_ok(bool(frames_check["match"]), device=dev)
    frames_check["api"] = apis[-1]

    # e2e through the public API: pinned host plaintext -> H2D -> seal -> D2H
    # frames, then open -> D2H auth flags; copies overlapped across objects.
    e2e = {"ms": float("nan"), "gbs": float("nan"), "h2d": 0, "d2h": 0} if args.no_e2e else \
        run_e2e(torch, key, plain_u8, ivs, P, stride, dev, args, barrier)
    (e2e_ms, copy_ms) = multigpu.reduce_max([e2e["ms"], e2e.get("copy_ms", float("nan"))], device=dev)

    if rank == 0:
        head = apis[-1]
        total_ms, seal_sum, open_sum, ok = results[head]
        bytes_per_step = 2 * nobj * P * world  # sealed + opened plaintext, all ranks

        def gbs(ms_sum, nbytes):
            return nbytes / (ms_sum / args.steps * 1e-3) / 1e9

        ms_per_step = total_ms / args.steps
        value = gbs(total_ms, bytes_per_step)
        peak, peak_kind = load_peaks()
        launches_per_step = (3 + 3) if head == "batched" else 3 * nobj
        # HBM roofline of the seal call. Batched: one seal_batch_async per
        # step = the plan kernel, seal_batch_kernel (encrypts; for this
        # workload the plan picks the two-pass seal) and seal_ghash_batch_kernel
        # (hashes, writes tags), timed together by the events around the call;
        # per object: one seal_kernel launch per object. Algorithmic bytes per
        # object: read P + write P + 29.
        kernel = ("seal_batch_async: batch_plan_kernel + seal_batch_kernel + seal_ghash_batch_kernel"
                  if head == "batched" else "seal_kernel")
        objs_per_launch = nobj if head == "batched" else 1
        launch_ms = seal_sum / args.steps / (1 if head == "batched" else nobj)
        achieved = objs_per_launch * (2 * P + 29) / (launch_ms * 1e-3) / 1e9
        prof = kernel_profile()
        blocks = objs_per_launch * (P // 16)
        traffic = None
        if head == "batched" and prof:
            traffic = round(sum(r["dram"] for r in prof.values() if r.get("call") == "seal") * blocks)
        sm_hz = (clk["sm_mhz"] if clk else 1965.0) * 1e6
        n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
        seal_gbs_dev = nobj * P / (seal_sum / args.steps * 1e-3) / 1e9
        open_gbs_dev = nobj * P / (open_sum / args.steps * 1e-3) / 1e9
        peaks, peaks_src = None, None
        try:
            from confkv_b200 import pipe_rates

            peaks = pipe_rates.model_peaks(pipe_rates.measure())
            peaks_src = "measured in this run (confkv_b200.pipe_rates)"
        except Exception as exc:  # noqa: BLE001 - fall back to the committed measurement
            peaks = committed_pipe_peaks()
            peaks_src = f"profiles/{PIPE_RATES_PROFILE} ({exc.__class__.__name__} live)"
        pipes = {}
        if head == "batched" and prof and peaks:
            pipes = {"unit": "plaintext GB/s", "per_sm_clk_peaks": {k: round(v, 2) for k, v in peaks.items()},
                     "peaks_source": peaks_src, "costs_source": f"profiles/{KERNEL_PROFILE}",
                     "sm_mhz": sm_hz / 1e6,
                     "seal": pipe_roofline(prof, "seal", peaks, n_sm, sm_hz, seal_gbs_dev),
                     "open": pipe_roofline(prof, "open", peaks, n_sm, sm_hz, open_gbs_dev)}
            binds = [k["binding"] for c in ("seal", "open") for k in pipes[c].get("kernels", {}).values()]
            pipes["bound"] = max(set(binds), key=binds.count) if binds else None
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u8",
            "data": "synthetic: bf16 N(0,1) KV chunks from fixed seeds, resident in HBM",
            "config": bench_config(nobj, P, world),
            "api": ("one seal_batch_async + one open_batch_async call per step" if head == "batched"
                    else "one seal_async + one open_async call per object"),
            "seal_gbs": round(gbs(seal_sum, nobj * P * world), 2),
            "open_gbs": round(gbs(open_sum, nobj * P * world), 2),
            "round_trip_ok": ok,
            "frames_match_openssl": frames_check["match"],
            "frames_check": frames_check,
            "roofline": {"bound": "hbm", "kernel": kernel, "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s",
                         "algorithmic_bytes_per_launch": objs_per_launch * (2 * P + 29),
                         "traffic": traffic,
                         "traffic_source": f"profiles/{KERNEL_PROFILE}: DRAM bytes per block of the call's kernels "
                                           "x blocks" if traffic is not None else None},
            "pipe_roofline": pipes,
            "e2e": {"value": round(e2e["gbs"] * world, 2) if world == 1 else
                    round(2 * nobj * P * world / (e2e_ms * 1e-3) / 1e9, 2),
                    "unit": UNIT, "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                    "what": "pinned host plaintext -> H2D -> seal_async -> D2H frames; open_async -> D2H auth; "
                            "copies overlapped across objects (streams: H2D, seal, open, D2H)",
                    "copy_only": round(2 * nobj * P * world / (copy_ms * 1e-3) / 1e9, 2),
                    "copy_only_what": "the same copies on the same streams with no kernels (host-link bound "
                                      "of the step, same byte accounting)"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if "per_object" in results and head != "per_object":
            t, ss, os_, okp = results["per_object"]
            line["per_object"] = {"value": round(gbs(t, bytes_per_step), 2),
                                  "ms_per_step": round(t / args.steps, 4),
                                  "seal_gbs": round(gbs(ss, nobj * P * world), 2),
                                  "open_gbs": round(gbs(os_, nobj * P * world), 2),
                                  "round_trip_ok": okp,
                                  "gpu_launches": ((2 if P >= SEAL_TWO_PASS_MIN_BYTES else 1) + 2) * nobj * args.steps,
                                  "api": "one seal_async + one open_async call per object (reference C-ABI)"}
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(args, plain_u8, key_bytes)
        print(json.dumps(line), flush=True)

    key.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def bench_config(nobj: int, P: int, world: int) -> dict:
    """The workload, identical in both arms' JSON lines."""
    return {"workload": WORKLOAD, "objects_per_gpu": nobj, "object_shape": list(SHAPE), "object_bytes": P,
            "step": f"seal {nobj} objects then open {nobj} frames with tag check (per GPU)",
            "l2": "inputs larger than L2 (1 GiB plaintext per GPU)",
            "parallelism": f"independent objects per GPU x{world}, no collective"}


def frames_match_openssl(frames, plain_u8, ivs, key: bytes, P: int) -> dict:
    """SHA-256 of each object's frame as the GPU wrote it against that of the
    frame OpenSSL writes for the same key, IV and plaintext (pyca
    `cryptography` AESGCM, stock LMCache's call: 0x01 + IV +
    encrypt(IV, P, None)). Runs after the timed steps."""
    import hashlib

    try:
        from cryptography.hazmat.primitives.ciphers.aead import AESGCM
    except ImportError as exc:
        return {"match": False, "error": f"pyca cryptography unavailable: {exc}"}
    aes = AESGCM(key)
    host_plain = plain_u8.cpu().numpy()
    host_frames = frames[:, :P + 29].cpu().numpy()
    bad = []
    for k in range(host_plain.shape[0]):
        want = hashlib.sha256(b"\x01" + ivs[k] + aes.encrypt(ivs[k], host_plain[k].tobytes(), None)).digest()
        if hashlib.sha256(host_frames[k].tobytes()).digest() != want:
            bad.append(k)
    return {"match": not bad, "objects": int(host_plain.shape[0]), "mismatched": bad,
            "how": "sha256 of each GPU frame vs pyca AESGCM (OpenSSL) frame for the same key, IV, plaintext"}


def run_e2e(torch, key, plain_u8, ivs, P, stride, dev, args, barrier):
    """Same step through the public API with host buffers and copies timed.
    Every rank runs each timed phase at the same time (barrier before each):
    the ranks share the host's memory and links."""
    n = plain_u8.shape[0]
    host_in = torch.empty((n, P), dtype=torch.uint8, pin_memory=True)
    host_in.copy_(plain_u8.cpu())
    host_frames = torch.empty((n, stride), dtype=torch.uint8, pin_memory=True)
    host_auth = torch.empty((2, n), dtype=torch.int32, pin_memory=True)
    d_in = torch.empty_like(plain_u8)
    # frames and verdicts alternate between two buffers by step, so a step's
    # seals never overwrite frames the previous step's opens still read
    d_frames = torch.empty((2, n, stride), dtype=torch.uint8, device=dev)
    d_out = torch.empty_like(plain_u8)
    d_auth = torch.zeros((2, n), dtype=torch.int32, device=dev)
    s_h2d, s_cmp, s_open, s_d2h = (torch.cuda.Stream(device=dev) for _ in range(4))
    frame_len = P + 29
    parity = [0]
    opened = [None, None]   # event after the opens that last used buffer set b
    sealed = [None] * n     # event after the last seal of object k (it read d_in[k])

    def step():
        b = parity[0]
        parity[0] ^= 1
        frames, auth = d_frames[b], d_auth[b]
        # the opens that last read this buffer set (two steps back) must be
        # done; the previous step's opens (other set) may still run
        if opened[b] is not None:
            s_cmp.wait_event(opened[b])
        for k in range(n):
            e_in = torch.cuda.Event()
            if sealed[k] is not None:
                s_h2d.wait_event(sealed[k])
            with torch.cuda.stream(s_h2d):
                d_in[k].copy_(host_in[k], non_blocking=True)
                e_in.record(s_h2d)
            s_cmp.wait_event(e_in)
            key.seal_async(src_ptr=d_in[k].data_ptr(), plaintext_len=P, dst_ptr=frames[k].data_ptr(),
                           dst_capacity=stride, iv=ivs[k], stream_ptr=s_cmp.cuda_stream)
            e_seal = torch.cuda.Event()
            e_seal.record(s_cmp)
            sealed[k] = e_seal
            s_d2h.wait_event(e_seal)
            with torch.cuda.stream(s_d2h):
                host_frames[k].copy_(frames[k], non_blocking=True)
            # each open follows its seal on its own stream, so the next
            # object's seal and the frame copies never wait for it
            s_open.wait_event(e_seal)
            key.open_async(src_ptr=frames[k].data_ptr(), frame_len=frame_len, dst_ptr=d_out[k].data_ptr(),
                           plaintext_len=P, auth_ok_ptr=auth[k:k + 1].data_ptr(), stream_ptr=s_open.cuda_stream)
        e_open = torch.cuda.Event()
        e_open.record(s_open)
        opened[b] = e_open
        # the verdicts go back on the open stream: the frame stream (the
        # host link's busy direction) does not wait for the opens
        with torch.cuda.stream(s_open):
            host_auth[b].copy_(auth, non_blocking=True)

    def copies_only():
        # the same copies in the same order and streams, no kernels: the
        # host-link bound of this step
        for k in range(n):
            e_in = torch.cuda.Event()
            with torch.cuda.stream(s_h2d):
                d_in[k].copy_(host_in[k], non_blocking=True)
                e_in.record(s_h2d)
            s_d2h.wait_event(e_in)
            with torch.cuda.stream(s_d2h):
                host_frames[k].copy_(d_frames[0, k], non_blocking=True)
        with torch.cuda.stream(s_d2h):
            host_auth[0].copy_(d_auth[0], non_blocking=True)

    def timed_steps(fn, steps):
        for _ in range(2):
            fn()
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(s_h2d)
        for st in (s_cmp, s_open, s_d2h):
            st.wait_event(t0)
        for _ in range(steps):
            fn()
        for st in (s_cmp, s_open, s_d2h):
            e = torch.cuda.Event()
            e.record(st)
            s_h2d.wait_event(e)
        t1.record(s_h2d)
        torch.cuda.synchronize(dev)
        return t0.elapsed_time(t1) / steps

    steps = max(2, min(args.steps, 5))
    copy_ms = timed_steps(copies_only, steps)
    ms = timed_steps(step, steps)
    assert bool((host_auth == 1).all()), "e2e open rejected a frame"
    return {"ms": ms, "gbs": 2 * n * P / (ms * 1e-3) / 1e9, "h2d": n * P, "d2h": n * (stride) + 4 * n,
            "copy_ms": copy_ms}


# ------------------------------------------------------- CPU (reference)

def load_ref_lib():
    """The native pthread driver around the reference's OpenSSL backend
    (oracle/_ref/libcpu_threads.so linked to oracle/_ref/libcpu_seal.so)."""
    so = ROOT / "oracle" / "_ref" / "libcpu_threads.so"
    if not so.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "ref"], capture_output=True)
    if not so.exists():
        return None
    lib = ctypes.CDLL(str(so))
    dp = ctypes.POINTER(ctypes.c_double)
    lib.cpu_threads_sweep.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_long, dp, dp]
    lib.cpu_threads_sweep.restype = ctypes.c_int
    vpp = ctypes.POINTER(ctypes.c_void_p)
    lib.cpu_threads_objects.argtypes = [ctypes.c_void_p, vpp, vpp, vpp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                                        dp, dp]
    lib.cpu_threads_objects.restype = ctypes.c_int
    return lib


class HostObjects:
    """Distinct objects in host memory, each with its own frame and output
    buffer, for the reference backend's native thread driver."""

    def __init__(self, objs):
        import numpy as np

        self.objs = np.ascontiguousarray(objs)            # [count, P] uint8
        count, P = self.objs.shape
        self.P, self.count = int(P), int(count)
        self.frames = np.empty((count, P + 29), dtype=np.uint8)
        self.outs = np.empty((count, P), dtype=np.uint8)
        arr = ctypes.c_void_p * count
        self._src = arr(*[self.objs[k].ctypes.data for k in range(count)])
        self._fr = arr(*[self.frames[k].ctypes.data for k in range(count)])
        self._out = arr(*[self.outs[k].ctypes.data for k in range(count)])
        # touch every page before anything is timed
        self.frames.fill(0)
        self.outs.fill(0)

    def run(self, lib, key: bytes, threads: int) -> tuple[float, float]:
        """Seal every object, then open every frame (reference
        lmcache_aes128gcm_seal/open, object k on thread k mod threads);
        returns the wall seconds of the seal leg and of the open leg."""
        ts, to = ctypes.c_double(), ctypes.c_double()
        kb = (ctypes.c_uint8 * 16).from_buffer_copy(key)
        rc = lib.cpu_threads_objects(kb, self._src, self._fr, self._out, self.P, self.count, threads,
                                     ctypes.byref(ts), ctypes.byref(to))
        assert rc == 0, "reference backend failed or a round trip differed"
        return ts.value, to.value


def openssl_threads_run(lib, key: bytes, per: int, threads: int, P: int) -> tuple[float, float]:
    """`threads` native threads each seal `per` objects of P bytes, then open
    them `per` times (reference lmcache_aes128gcm_seal/open); returns the wall
    seconds of the seal leg and of the open leg."""
    ts, to = ctypes.c_double(), ctypes.c_double()
    kb = (ctypes.c_uint8 * 16).from_buffer_copy(key)
    rc = lib.cpu_threads_sweep(kb, P, threads, per, ctypes.byref(ts), ctypes.byref(to))
    assert rc == 0, "reference backend failed"
    return ts.value, to.value


SINGLE_CORE_OBJECTS = 4  # objects of the single-core sample (128 MiB each way at 32 MiB)


def single_core(lib, objs, key: bytes) -> dict:
    """The reference backend on one native thread over the first objects of
    the step, sealed then opened (after one untimed pass): the figure the
    reference's own single-core CPU table is comparable with."""
    host = HostObjects(objs[:SINGLE_CORE_OBJECTS])
    host.run(lib, key, 1)
    ts, to = host.run(lib, key, 1)
    nbytes = host.count * host.P
    return {"seal_gbs": round(nbytes / ts / 1e9, 2), "open_gbs": round(nbytes / to / 1e9, 2),
            "value": round(2 * nbytes / (ts + to) / 1e9, 2), "cores": 1,
            "sample": f"{host.count} objects of {host.P} B sealed then opened on one native thread"}


def cpu_baseline(args, plain_u8, key: bytes) -> dict:
    """The reference OpenSSL backend on all host threads, sealing then
    opening this rank's objects (copied to host memory), once: a bounded
    sample of the step (1 GiB each way at the default 32 objects)."""
    lib = load_ref_lib()
    if lib is None:
        return {"unavailable": "oracle/_ref/libcpu_threads.so missing"}
    threads = len(os.sched_getaffinity(0))
    count = plain_u8.shape[0] if not args.cpu_sample_objects else min(args.cpu_sample_objects, plain_u8.shape[0])
    host = HostObjects(plain_u8[:count].cpu().numpy())
    host.run(lib, key, threads)  # warm-up: caches, page tables
    ts, to = host.run(lib, key, threads)
    gbs = 2 * host.count * host.P / (ts + to) / 1e9
    return {"value": round(gbs, 2), "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"the step's {host.count} objects of {host.P} B (bf16 KV, same bytes as the GPU run) sealed "
                      f"then opened once on {threads} native threads, reference lmcache_aes128gcm_seal/open "
                      f"(OpenSSL EVP)",
            "single_core": single_core(lib, host.objs, key)}


def cpu_sweep_sizes(lib, key: bytes, threads: int) -> None:
    """Seal and open of single objects of 2^k bytes (k = 12..30) with the
    reference OpenSSL backend on `threads` native host threads (fewer for
    large objects so the buffers stay under ~8 GiB), ~2 GiB of plaintext per
    leg."""
    for k in range(12, 31):
        P = 1 << k
        nth = max(1, min(threads, (8 << 30) // (3 * P)))
        per = max(1, min(1 << 19, (2 << 30) // (P * nth)))
        ts, to = openssl_threads_run(lib, key, per, nth, P)
        total = P * per * nth
        print(json.dumps({"sweep": "cpu_reference", "object_bytes": P, "threads": nth, "objects": per * nth,
                          "seal_gbs": round(total / ts / 1e9, 2), "open_gbs": round(total / to / 1e9, 2),
                          "impl": "reference (OpenSSL EVP lmcache_aes128gcm_seal/open), native threads"}),
              flush=True)


def run_reference(args, rank, world):
    """The reference's OpenSSL CPU backend on this host's cores, over the
    same objects the GPU run seals: every rank's 32 bf16 KV objects (the whole
    job of `world` GPUs), each in its own host buffer, sealed then opened per
    step. Objects are drawn with torch's CUDA generator like the GPU run's
    (then copied to host memory) when a GPU is present."""
    if rank != 0:
        return
    lib = load_ref_lib()
    if lib is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference OpenSSL backend could not be built"}))
        return
    import numpy as np
    import torch

    from confkv_b200 import workloads

    draw = "cuda" if torch.cuda.is_available() else "cpu"
    cases = [workloads.bench_case(r, args.objects, device=draw) for r in range(world)]
    objs = np.concatenate([c.plain.cpu().numpy() for c in cases])
    del cases
    if draw == "cuda":
        torch.cuda.empty_cache()
    key = workloads.make_key(workloads.BENCH_SEED)
    host = HostObjects(objs)
    del objs
    threads = len(os.sched_getaffinity(0))
    for _ in range(args.warmup):
        host.run(lib, key, threads)
    times = [sum(host.run(lib, key, threads)) for _ in range(args.steps)]
    ms = statistics.mean(times) * 1e3
    value = 2 * host.count * host.P / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8",
        "data": f"synthetic: the GPU run's bf16 N(0,1) KV objects (drawn on {draw}), one host buffer each",
        "config": bench_config(args.objects, host.P, world),
        "impl": "reference",
        "api": "reference lmcache_aes128gcm_seal / lmcache_aes128gcm_open, one call per object, native threads",
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": f"all {host.count} objects of the step ({world} GPU(s) x {args.objects}) "
                                   f"sealed then opened, object k on thread k mod {threads}",
                         "single_core": single_core(lib, host.objs, key)},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    if args.cpu_sweep:
        cpu_sweep_sizes(lib, key, threads)


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
