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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-log2", type=int, default=12)
    ap.add_argument("--max-log2", type=int, default=30)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    torch.cuda.set_device(args.device)
    dev = torch.device("cuda", args.device)
    lib = GpuAesGcmLibrary()
    with GpuAes128GcmKey(lib, workloads.make_key(5), device=args.device) as key:
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
