"""Throughput of seal / open over object sizes and KV workloads (one GPU).

    python -m confkv_b200.sweep [--min-log2 12] [--max-log2 30] [--device 0]

Prints one JSON line per measurement:

* size sweep: single bf16 N(0,1) objects of 2^k bytes, k = min..max. Each
  line times a batch of objects of that size (enough for >= 64 MiB or at least
  4 objects) launched back to back on one stream: seal GB/s, open GB/s (tag
  check included), and seal with the frame copied to pinned host memory on a
  side stream overlapped with the next seal (the persistent-store path).
* workloads: 64 x 2 MiB kv_small objects and 64 x 10 MiB Llama-3-70B TP-8
  KV-head shards (seal then open).
* batches (--batch): the ragged workload (4096 objects, log-uniform 4 KiB ..
  1 MiB, odd lengths, packed back to back), 8192 x 4 KiB and 32 x 32 MiB,
  each sealed and opened once per object (seal_async / open_async) and once
  per call (seal_batch / open_batch).

All numbers are CUDA-event device times; GB/s counts plaintext bytes.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import workloads
from .gpu_aesgcm import GpuAes128GcmKey, GpuAesGcmLibrary


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def measure_batch(key: GpuAes128GcmKey, plain: torch.Tensor, reps: int, warmup: int = 2) -> dict:
    """plain: [count, P] uint8 on the device. Returns GB/s for seal, open and
    seal + overlapped pinned D2H of every frame."""
    dev = plain.device
    count, P = plain.shape
    stride = (P + 29 + 255) // 256 * 256
    frames = torch.empty((count, stride), dtype=torch.uint8, device=dev)
    out = torch.empty_like(plain)
    auth = torch.zeros((count,), dtype=torch.int32, device=dev)
    host = torch.empty((count, stride), dtype=torch.uint8, pin_memory=True)
    s, s_copy = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ivs = workloads.make_ivs(P, count)

    def seal(k):
        key.seal_async(src_ptr=plain[k].data_ptr(), plaintext_len=P, dst_ptr=frames[k].data_ptr(),
                       dst_capacity=stride, iv=ivs[k], stream_ptr=s.cuda_stream)

    def open_(k):
        key.open_async(src_ptr=frames[k].data_ptr(), frame_len=P + 29, dst_ptr=out[k].data_ptr(),
                       plaintext_len=P, auth_ok_ptr=auth[k:k + 1].data_ptr(), stream_ptr=s.cuda_stream)

    def timed(body):
        for _ in range(warmup):
            body()
        torch.cuda.synchronize(dev)
        a, b = _events()
        a.record(s)
        for _ in range(reps):
            body()
        b.record(s)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / reps

    seal_ms = timed(lambda: [seal(k) for k in range(count)])
    open_ms = timed(lambda: [open_(k) for k in range(count)])
    assert bool((auth == 1).all()) and torch.equal(out, plain), "round trip failed"

    def seal_d2h():
        for k in range(count):
            seal(k)
            e = torch.cuda.Event()
            e.record(s)
            s_copy.wait_event(e)
            with torch.cuda.stream(s_copy):
                host[k, :P + 29].copy_(frames[k, :P + 29], non_blocking=True)
        e = torch.cuda.Event()
        e.record(s_copy)
        s.wait_event(e)

    d2h_ms = timed(seal_d2h)
    total = count * P
    return {"objects": count, "object_bytes": P,
            "seal_gbs": round(total / (seal_ms * 1e-3) / 1e9, 2),
            "open_gbs": round(total / (open_ms * 1e-3) / 1e9, 2),
            "seal_d2h_gbs": round(total / (d2h_ms * 1e-3) / 1e9, 2),
            "seal_us_per_object": round(seal_ms * 1e3 / count, 2),
            "open_us_per_object": round(open_ms * 1e3 / count, 2)}


def measure_batch_api(lib: GpuAesGcmLibrary, key: GpuAes128GcmKey, lens, seed: int, reps: int,
                      warmup: int = 2) -> dict:
    """Per-object calls vs one batched call over objects packed back to back
    (plaintexts and frames at arbitrary byte offsets)."""
    from .batch import DeviceBatch

    dev = torch.device("cuda", key.device)
    lens = [int(x) for x in lens]
    pt_off, fr_off, p, f = [], [], 0, 0
    for n in lens:
        pt_off.append(p)
        fr_off.append(f)
        p += n
        f += n + 29
    g = torch.Generator(device=dev).manual_seed(seed)
    plain = torch.randint(0, 256, (p + 16,), dtype=torch.uint8, device=dev, generator=g)
    frames = torch.empty(f + 16, dtype=torch.uint8, device=dev)
    out = torch.empty(p + 16, dtype=torch.uint8, device=dev)
    auth = torch.zeros(len(lens), dtype=torch.int32, device=dev)
    ivs = workloads.make_ivs(seed, len(lens))
    s = torch.cuda.Stream(device=dev)
    pb, fb, ob, ab = plain.data_ptr(), frames.data_ptr(), out.data_ptr(), auth.data_ptr()
    seal_entries = [(pb + pt_off[i], fb + fr_off[i], n, n + 29, ivs[i]) for i, n in enumerate(lens)]
    open_entries = [(fb + fr_off[i], ob + pt_off[i], n, n + 29, ab + 4 * i) for i, n in enumerate(lens)]
    # one DeviceBatch per direction: descriptors are uploaded by the first
    # (warm-up) call; the timed region is the batched launches alone
    bseal = DeviceBatch(lib, len(lens), dev)
    bopen = DeviceBatch(lib, len(lens), dev)

    def per_object_seal():
        for i, n in enumerate(lens):
            key.seal_async(src_ptr=pb + pt_off[i], plaintext_len=n, dst_ptr=fb + fr_off[i], dst_capacity=n + 29,
                           iv=ivs[i], stream_ptr=s.cuda_stream)

    def per_object_open():
        for i, n in enumerate(lens):
            key.open_async(src_ptr=fb + fr_off[i], frame_len=n + 29, dst_ptr=ob + pt_off[i], plaintext_len=n,
                           auth_ok_ptr=ab + 4 * i, stream_ptr=s.cuda_stream)

    def batched(fn, b):
        def run():
            fn(items_ptr=b.items.data_ptr(), count=len(lens), workspace_ptr=b.workspace.data_ptr(),
               workspace_bytes=b.workspace_bytes, stream_ptr=s.cuda_stream)
        return run

    def timed(body):
        for _ in range(warmup):
            body()
        torch.cuda.synchronize(dev)
        a, b = _events()
        a.record(s)
        for _ in range(reps):
            body()
        b.record(s)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / reps

    def check_open():
        assert bool((auth == 1).all()) and torch.equal(out[:p], plain[:p]), "round trip failed"

    r = {}

    def record(name, ms):
        r[name + "_gbs"] = round(sum(lens) / (ms * 1e-3) / 1e9, 2)
        r[name + "_ms"] = round(ms, 4)

    record("per_object_seal", timed(per_object_seal))
    ref_frames = frames[:f].clone()
    frames.zero_()
    torch.cuda.synchronize(dev)   # default-stream work above, stream `s` below
    bseal.seal(key, seal_entries, s)
    record("batch_seal", timed(batched(key.seal_batch_async, bseal)))
    assert torch.equal(frames[:f], ref_frames), "batched seal frames differ from per-object frames"
    record("per_object_open", timed(per_object_open))
    check_open()
    out.zero_()
    auth.zero_()
    torch.cuda.synchronize(dev)
    bopen.open(key, open_entries, s)
    record("batch_open", timed(batched(key.open_batch_async, bopen)))
    check_open()
    return {"objects": len(lens), "bytes": sum(lens), **r}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-log2", type=int, default=12)
    ap.add_argument("--max-log2", type=int, default=30)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--batch", action="store_true", help="only the batched-call comparison")
    args = ap.parse_args()
    torch.cuda.set_device(args.device)
    dev = torch.device("cuda", args.device)
    lib = GpuAesGcmLibrary()
    with GpuAes128GcmKey(lib, workloads.make_key(5), device=args.device) as key:
        if args.batch:
            ragged = workloads.ragged_case(4096, seed=3).lengths
            for name, lens in (("ragged_4096", ragged), ("small_8192x4KiB", [4096] * 8192),
                               ("kv_llama8b_32x32MiB", [32 << 20] * 32)):
                r = measure_batch_api(lib, key, lens, seed=13, reps=args.reps)
                print(json.dumps({"sweep": "batch", "workload": name, **r}), flush=True)
            return
        for k in range(args.min_log2, args.max_log2 + 1):
            P = 1 << k
            count = max(4, min(4096, (64 << 20) // P))
            plain = workloads.bf16_batch((P // 2,), count, seed=k, device=dev).view(torch.uint8).reshape(count, P)
            r = measure_batch(key, plain, reps=args.reps)
            print(json.dumps({"sweep": "size", "log2": k, **r}), flush=True)
            del plain
            torch.cuda.empty_cache()
        for name, count in (("kv_small", 64), ("kv_llama70b_tp8_shard", 64)):
            shape = workloads.SHAPES[name]
            P = workloads.nbytes_of(shape)
            plain = workloads.bf16_batch(shape, count, seed=7, device=dev).view(torch.uint8).reshape(count, P)
            r = measure_batch(key, plain, reps=args.reps)
            print(json.dumps({"sweep": "workload", "workload": name, **r}), flush=True)
            del plain
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
