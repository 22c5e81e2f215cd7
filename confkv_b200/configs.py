"""The five benchmarked configurations on 1..8 GPUs of one node.

    python -m confkv_b200.configs --config kv_small|kv_llama8b|ragged|tp8|sweep [--api both|per_object|batched]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m confkv_b200.configs --config tp8

  kv_small    64 objects [2,4,256,8,64] bf16 N(0,1) (2 MiB), round-robin over the GPUs
  kv_llama8b  32 objects [2,32,256,8,128] bf16 (32 MiB) per GPU
  ragged      4096 objects, lengths log-uniform in [4 KiB, 1 MiB] with odd remainders,
              random bytes, round-robin over the GPUs
  tp8         64 Llama-3-70B KV chunks split by KV head: every GPU seals its own
              64 shards [2,80,256,1,128] (10 MiB), generated on that GPU
  sweep       single objects of 2^k bytes, k = 12..30, round-robin over the GPUs;
              also seal with each frame copied to pinned host memory on a side stream

Call styles (--api): per_object (one seal_async / open_async per object, the
reference C-ABI), per_object_graph (the same calls captured once into a CUDA
graph and replayed; objects up to 64 KiB in the sweep) and batched (one
seal_batch_async / open_batch_async per rank).

One process per GPU, each with its own key handle and stream; no data crosses
GPUs. Every timed iteration starts after a barrier and runs INNER back-to-back
calls; each rank times its own work with CUDA events on its stream and the
per-iteration times are reduced with MAX over ranks (the job takes as long as
its slowest GPU). Reported: median and p95 over the iterations of the time per
call, GB/s = plaintext bytes of all ranks / median max-over-ranks time. Every
round trip is checked after timing.
"""

from __future__ import annotations

import argparse
import json
import math
import statistics

import torch

from . import hostmem, multigpu, workloads
from .batch import DeviceBatch
from .clocks import ClockSampler
from .gpu_aesgcm import GpuAes128GcmKey, GpuAesGcmLibrary

ALIGN = 256
INNER = 4  # calls per timed iteration


class RankWork:
    """This rank's objects packed into one plaintext buffer (starts 256-B
    aligned unless `packed`), frames and outputs likewise, plus descriptor
    arrays for the batched calls."""

    def __init__(self, lib, key, lens, plain: torch.Tensor, offsets, stream, ivs, packed=False):
        dev = plain.device
        self.key, self.lens, self.stream = key, [int(n) for n in lens], stream
        self.plain, self.pt_off = plain, [int(o) for o in offsets]
        self.fr_off, pos = [], 0
        for n in self.lens:
            self.fr_off.append(pos)
            pos += n + 29 if packed else (n + 29 + ALIGN - 1) // ALIGN * ALIGN
        self.frames = torch.zeros(pos + 16, dtype=torch.uint8, device=dev)
        self.out = torch.zeros(plain.numel() + 16, dtype=torch.uint8, device=dev)
        self.auth = torch.zeros(max(1, len(self.lens)), dtype=torch.int32, device=dev)
        self.ivs = ivs
        pb, fb, ob, ab = plain.data_ptr(), self.frames.data_ptr(), self.out.data_ptr(), self.auth.data_ptr()
        self.seal_entries = [(pb + self.pt_off[i], fb + self.fr_off[i], n, n + 29, ivs[i])
                             for i, n in enumerate(self.lens)]
        self.open_entries = [(fb + self.fr_off[i], ob + self.pt_off[i], n, n + 29, ab + 4 * i)
                             for i, n in enumerate(self.lens)]
        self.bseal = self.bopen = None
        if self.lens:
            self.bseal = DeviceBatch(lib, len(self.lens), dev)
            self.bopen = DeviceBatch(lib, len(self.lens), dev)
            self.bseal.seal(key, self.seal_entries, stream)     # uploads the descriptors
            self.bopen.open(key, self.open_entries, stream)
        self.host = None

    @property
    def nbytes(self) -> int:
        return sum(self.lens)

    def seal_each(self):
        sp = self.stream.cuda_stream
        for s, d, n, c, iv in self.seal_entries:
            self.key.seal_async(src_ptr=s, plaintext_len=n, dst_ptr=d, dst_capacity=c, iv=iv, stream_ptr=sp)

    def open_each(self):
        sp = self.stream.cuda_stream
        for f, d, n, fl, a in self.open_entries:
            self.key.open_async(src_ptr=f, frame_len=fl, dst_ptr=d, plaintext_len=n, auth_ok_ptr=a, stream_ptr=sp)

    def seal_batched(self):
        if self.bseal is not None:
            b = self.bseal
            self.key.seal_batch_async(items_ptr=b.items.data_ptr(), count=len(self.lens),
                                      workspace_ptr=b.workspace.data_ptr(), workspace_bytes=b.workspace_bytes,
                                      stream_ptr=self.stream.cuda_stream)

    def open_batched(self):
        if self.bopen is not None:
            b = self.bopen
            self.key.open_batch_async(items_ptr=b.items.data_ptr(), count=len(self.lens),
                                      workspace_ptr=b.workspace.data_ptr(), workspace_bytes=b.workspace_bytes,
                                      stream_ptr=self.stream.cuda_stream)

    def graphed(self, fn):
        """Capture `fn` (a sequence of calls on this rank's stream) into a CUDA
        graph; returns its replay. Key handles, descriptors and device set-up
        exist before capture, so the captured calls allocate nothing."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            fn()
        self._graphs = getattr(self, "_graphs", []) + [g]

        def replay():
            with torch.cuda.stream(self.stream):
                g.replay()
        return replay

    def seal_each_to_host(self):
        """Per-object seal with each frame written straight into pinned host
        memory (device-mapped, no copy afterwards). Requires
        hostmem.device_mapped(self.host_ptr())."""
        base = self.host_ptr()
        sp = self.stream.cuda_stream
        for i, (s, d, n, c, iv) in enumerate(self.seal_entries):
            self.key.seal_async(src_ptr=s, plaintext_len=n, dst_ptr=base + self.fr_off[i], dst_capacity=c, iv=iv,
                                stream_ptr=sp)

    def host_ptr(self) -> int:
        if self.host is None:
            self.host = torch.empty(self.frames.numel(), dtype=torch.uint8, pin_memory=True)
        return self.host.data_ptr()

    def seal_each_d2h(self, side: torch.cuda.Stream):
        """Per-object seal with each frame copied to pinned host memory on
        `side` as soon as it is sealed (the persistent-store path)."""
        if self.host is None:
            self.host = torch.empty(self.frames.numel(), dtype=torch.uint8, pin_memory=True)
        sp = self.stream.cuda_stream
        for i, (s, d, n, c, iv) in enumerate(self.seal_entries):
            self.key.seal_async(src_ptr=s, plaintext_len=n, dst_ptr=d, dst_capacity=c, iv=iv, stream_ptr=sp)
            e = torch.cuda.Event()
            e.record(self.stream)
            side.wait_event(e)
            a = self.fr_off[i]
            with torch.cuda.stream(side):
                self.host[a:a + n + 29].copy_(self.frames[a:a + n + 29], non_blocking=True)
        e = torch.cuda.Event()
        e.record(side)
        self.stream.wait_event(e)

    def open_each_from_host(self, side: torch.cuda.Stream):
        """Per-object open of frames held in pinned host memory (the load path
        from host storage): each frame is copied in on `side` and opened on the
        work stream as soon as it has arrived, so copies overlap the opens of
        earlier objects. The copies start after the work stream's earlier
        work, whose opens may still read the frame buffer."""
        if self.host is None:
            raise RuntimeError("no host frames: seal_each_d2h or seal_each_to_host first")
        e = torch.cuda.Event()
        e.record(self.stream)
        side.wait_event(e)
        sp = self.stream.cuda_stream
        for i, (f, d, n, fl, a) in enumerate(self.open_entries):
            o = self.fr_off[i]
            with torch.cuda.stream(side):
                self.frames[o:o + n + 29].copy_(self.host[o:o + n + 29], non_blocking=True)
            e = torch.cuda.Event()
            e.record(side)
            self.stream.wait_event(e)
            self.key.open_async(src_ptr=f, frame_len=fl, dst_ptr=d, plaintext_len=n, auth_ok_ptr=a, stream_ptr=sp)

    def reset_outputs(self):
        self.out.zero_()
        self.auth.zero_()

    def round_trip_ok(self) -> bool:
        if not self.lens:
            return True
        if not bool((self.auth[:len(self.lens)] == 1).all()):
            return False
        return all(torch.equal(self.out[a:a + n], self.plain[a:a + n]) for a, n in zip(self.pt_off, self.lens))


def barrier(world, dev):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)


def timed(fn, stream, warmup, iters, world, dev, inner=INNER) -> dict:
    """Per-call device time: each iteration times `inner` back-to-back calls
    (so host submission overlaps the previous call's GPU work instead of
    being counted) and divides by `inner`."""
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        barrier(world, dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(inner):
            fn()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b) / inner)
    times = multigpu.reduce_max(times, device=dev)
    srt = sorted(times)
    return {"median_ms": statistics.median(times), "p95_ms": srt[min(len(srt) - 1, math.ceil(0.95 * len(srt)) - 1)],
            "mean_ms": statistics.fmean(times)}


def measure(work: RankWork, apis, warmup, iters, world, dev, d2h=False) -> list[dict]:
    total = int(multigpu.reduce_sum([work.nbytes], device=dev)[0])
    out = []
    for api in apis:
        if api == "per_object":
            seal_fn, open_fn = work.seal_each, work.open_each
        elif api == "per_object_graph":
            barrier(world, dev)
            seal_fn, open_fn = work.graphed(work.seal_each), work.graphed(work.open_each)
        else:
            seal_fn, open_fn = work.seal_batched, work.open_batched
        work.reset_outputs()
        barrier(world, dev)
        clocks = ClockSampler(dev.index if dev.index is not None else 0)
        clocks.start()
        rs = timed(seal_fn, work.stream, warmup, iters, world, dev)
        ro = timed(open_fn, work.stream, warmup, iters, world, dev)
        clk = clocks.stop()
        barrier(world, dev)
        ok = multigpu.all_ok(work.round_trip_ok(), device=dev)
        r = {"api": api, "bytes_all_ranks": total, "round_trip_ok": ok, "clocks": clk}
        for name, t in (("seal", rs), ("open", ro)):
            r[f"{name}_gbs"] = round(total / (t["median_ms"] * 1e-3) / 1e9, 2)
            r[f"{name}_ms_median"] = round(t["median_ms"], 4)
            r[f"{name}_ms_p95"] = round(t["p95_ms"], 4)
        out.append(r)
    if d2h:
        side = torch.cuda.Stream(device=dev)
        t = timed(lambda: work.seal_each_d2h(side), work.stream, warmup, iters, world, dev)
        out[0]["seal_d2h_gbs"] = round(total / (t["median_ms"] * 1e-3) / 1e9, 2)
        out[0]["seal_d2h_ms_median"] = round(t["median_ms"], 4)
        # the same frames written by the seal kernel straight into pinned host
        # memory (checked to be device-mapped on the host first)
        if hostmem.device_mapped(work.host_ptr()):
            torch.cuda.synchronize(dev)
            work.host.fill_(0)
            t = timed(work.seal_each_to_host, work.stream, warmup, iters, world, dev)
            torch.cuda.synchronize(dev)
            same = all(torch.equal(work.host[a:a + n + 29].to(dev), work.frames[a:a + n + 29])
                       for a, n in zip(work.fr_off, work.lens))
            out[0]["seal_to_host_gbs"] = round(total / (t["median_ms"] * 1e-3) / 1e9, 2)
            out[0]["seal_to_host_ms_median"] = round(t["median_ms"], 4)
            out[0]["seal_to_host_frames_ok"] = bool(multigpu.all_ok(same, device=dev))
        # the load path: frames from pinned host memory -> H2D -> gated open
        torch.cuda.synchronize(dev)
        work.reset_outputs()
        t = timed(lambda: work.open_each_from_host(side), work.stream, warmup, iters, world, dev)
        torch.cuda.synchronize(dev)
        out[0]["open_h2d_gbs"] = round(total / (t["median_ms"] * 1e-3) / 1e9, 2)
        out[0]["open_h2d_ms_median"] = round(t["median_ms"], 4)
        out[0]["open_h2d_round_trip_ok"] = bool(multigpu.all_ok(work.round_trip_ok(), device=dev))
    return out


def packed_offsets(lens, packed=False):
    offs, pos = [], 0
    for n in lens:
        offs.append(pos)
        pos += int(n) if packed else (int(n) + ALIGN - 1) // ALIGN * ALIGN
    return offs, pos


def random_plain(lens, seed, dev, packed=False):
    offs, total = packed_offsets(lens, packed)
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randint(0, 256, (total + 16,), dtype=torch.uint8, device=dev, generator=g), offs


def bf16_plain(shape, count, seed, dev):
    P = workloads.nbytes_of(shape)
    t = workloads.bf16_batch(shape, count, seed=seed, device=dev).view(torch.uint8).reshape(-1)
    return t, [k * P for k in range(count)], [P] * count


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True, choices=["kv_small", "kv_llama8b", "ragged", "tp8", "sweep"])
    ap.add_argument("--api", default="both", choices=["both", "all", "per_object", "per_object_graph", "batched"],
                    help="both = per_object + batched; all adds per-object calls replayed from a CUDA graph")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--min-log2", type=int, default=12)
    ap.add_argument("--max-log2", type=int, default=30)
    args = ap.parse_args()
    rank, world, local = multigpu.rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    apis = {"both": ["per_object", "batched"], "all": ["per_object", "per_object_graph", "batched"]}.get(
        args.api, [args.api])
    lib = GpuAesGcmLibrary()
    key = GpuAes128GcmKey(lib, workloads.make_key(40), device=local)
    stream = torch.cuda.Stream(device=dev)

    def emit(extra, results):
        if rank == 0:
            for r in results:
                print(json.dumps({"config": args.config, "n_gpus": world, **extra, **r}), flush=True)

    def run(lens, plain, offs, extra, packed=False, d2h=False, iters=None, graph=True):
        ivs = workloads.make_ivs(1000 + rank, len(lens))
        work = RankWork(lib, key, lens, plain, offs, stream, ivs, packed=packed)
        use = [a for a in apis if graph or a != "per_object_graph"]
        emit(extra, measure(work, use, args.warmup, iters or args.iters, world, dev, d2h=d2h))

    try:
        if args.config in ("kv_small", "kv_llama8b", "tp8"):
            name = {"kv_small": "kv_small", "kv_llama8b": "kv_llama8b", "tp8": "kv_llama70b_tp8_shard"}[args.config]
            shape = workloads.SHAPES[name]
            if args.config == "kv_small":
                mine = multigpu.round_robin(64, rank, world)       # 64 objects over the GPUs
            else:
                mine = list(range(32 if args.config == "kv_llama8b" else 64))   # per GPU
            plain, offs, lens = bf16_plain(shape, len(mine), seed=50 + rank, dev=dev)
            run(lens, plain, offs, {"object_shape": list(shape), "objects_per_gpu": len(mine),
                                    "objects_all_gpus": len(mine) * world if args.config != "kv_small" else 64})
        elif args.config == "ragged":
            case = workloads.ragged_case(4096, seed=3)
            mine = multigpu.round_robin(len(case.lengths), rank, world)
            lens = [int(case.lengths[i]) for i in mine]
            plain, offs = random_plain(lens, seed=60 + rank, dev=dev, packed=True)
            run(lens, plain, offs, {"objects_all_gpus": len(case.lengths), "packing": "back to back"}, packed=True)
        else:
            for k in range(args.min_log2, args.max_log2 + 1):
                P = 1 << k
                total_objects = max(world, min(4096 * world, (64 << 20) * world // P))
                mine = multigpu.round_robin(total_objects, rank, world)
                lens = [P] * len(mine)
                plain, offs = random_plain(lens, seed=70 + k, dev=dev)
                run(lens, plain, offs, {"object_bytes": P, "objects_all_gpus": total_objects}, d2h=True,
                    iters=min(args.iters, 10), graph=P <= (64 << 10))
                del plain
                torch.cuda.empty_cache()
    finally:
        key.close()
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
