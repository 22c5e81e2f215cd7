"""Seeded synthetic KV-cache objects for the seal/open workloads.

No public dataset is involved: every workload is bf16 N(0,1) KV tensors (or
random bytes) drawn from fixed seeds, with the shapes of the benchmarked
configurations:

* ``kv_small``  - [2 (K,V), 4 layers, 256 tokens, 8 heads, 64 dim] bf16, 2 MiB
* ``kv_llama8b`` - [2, 32 layers, 256 tokens, 8 KV heads, 128 dim] bf16, 32 MiB
  (one LMCache chunk of Llama-3-8B)
* ``kv_llama70b_tp8_shard`` - [2, 80, 256, 1, 128] bf16, 10 MiB (one KV head
  of a Llama-3-70B chunk, the per-rank shard under 8-way tensor parallelism)
* ragged: lengths log-uniform in [4 KiB, 1 MiB], half of them with a 1-15 byte
  remainder, random uint8 payloads, 1% tampered and 1% opened with a wrong key.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

SHAPES = {
    "kv_small": (2, 4, 256, 8, 64),
    "kv_llama8b": (2, 32, 256, 8, 128),
    "kv_llama70b_tp8_shard": (2, 80, 256, 1, 128),
}


def nbytes_of(shape) -> int:
    return int(np.prod(shape)) * 2  # bf16


def make_key(seed: int) -> bytes:
    return np.random.default_rng([seed, 0x6B6579]).bytes(16)


def make_ivs(seed: int, count: int) -> list[bytes]:
    rng = np.random.default_rng([seed, 0x6976])
    return [rng.bytes(12) for _ in range(count)]


def bf16_objects(shape, count: int, seed: int, device="cpu"):
    """`count` bf16 N(0,1) tensors of `shape` from torch generators seeded
    (seed, k). Returned as a list of contiguous tensors on `device`."""
    import torch

    out = []
    for k in range(count):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 1000003 + k)
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
        out.append(t.contiguous())
    return out


def bf16_batch(shape, count: int, seed: int, device="cpu"):
    """One [count, *shape] bf16 tensor; object k is row k (N(0,1), one seed)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn((count, *shape), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


# The benchmarked workload (Llama-3-8B KV chunks): per rank, 32 objects
# [2, 32, 256, 8, 128] bf16 (32 MiB each) under one key, each with its own IV;
# frames laid out at a 256-byte stride (the ciphertext at frame + 13).
BENCH_SHAPE = SHAPES["kv_llama8b"]
BENCH_OBJECTS = 32
BENCH_SEED = 2


@dataclass
class BenchCase:
    key: bytes
    ivs: list                  # 12-byte IVs, one per object
    plain: object              # torch uint8 [count, P] on the device it was drawn on
    object_bytes: int
    frame_stride: int


def bench_case(rank: int = 0, count: int = BENCH_OBJECTS, device="cuda") -> BenchCase:
    """The inputs rank `rank` seals in the benchmark: the key is shared by all
    ranks, the objects and IVs are the rank's own. The objects are drawn with
    torch's generator on `device` (CUDA draws differ from CPU draws for the
    same seed), so a host-side consumer that wants the GPU run's bytes draws
    them on a GPU and copies them to the host."""
    import torch

    P = nbytes_of(BENCH_SHAPE)
    plain = bf16_batch(BENCH_SHAPE, count, seed=BENCH_SEED * 100 + rank, device=device).view(torch.uint8)
    plain = plain.reshape(count, P)
    return BenchCase(key=make_key(BENCH_SEED), ivs=make_ivs(BENCH_SEED * 100 + rank, count), plain=plain,
                     object_bytes=P, frame_stride=(P + 29 + 255) // 256 * 256)


@dataclass
class RaggedCase:
    lengths: np.ndarray        # plaintext bytes per object
    payload_seed: int
    tamper: dict               # object index -> ("iv" | "ct" | "tag", bit index within that field)
    wrong_key: set             # object indices opened with a wrong key


def ragged_case(count: int = 4096, seed: int = 3, lo: int = 4096, hi: int = 1 << 20) -> RaggedCase:
    rng = np.random.default_rng([seed, 0x7261])
    raw = np.floor(np.exp(rng.uniform(math.log(lo), math.log(hi), size=count))).astype(np.int64)
    lengths = (raw // 16) * 16
    odd = rng.random(count) < 0.5
    lengths = np.where(odd, lengths + rng.integers(1, 16, size=count), lengths)
    lengths = np.clip(lengths, lo, hi + 15)
    n_bad = max(1, count // 100)
    picks = rng.permutation(count)
    tamper_idx = picks[:n_bad]
    wrong_idx = picks[n_bad:2 * n_bad]
    tamper = {}
    for i in tamper_idx:
        field = ("iv", "ct", "tag")[int(rng.integers(0, 3))]
        width = {"iv": 96, "tag": 128, "ct": int(lengths[i]) * 8}[field]
        tamper[int(i)] = (field, int(rng.integers(0, width)))
    return RaggedCase(lengths=lengths, payload_seed=seed, tamper=tamper, wrong_key={int(i) for i in wrong_idx})


def ragged_payload(case: RaggedCase, index: int) -> np.ndarray:
    rng = np.random.default_rng([case.payload_seed, 0x706C, index])
    return rng.integers(0, 256, size=int(case.lengths[index]), dtype=np.uint8)


def flip_bit(frame: np.ndarray, plen: int, field: str, bit: int) -> None:
    """Flip one bit of the IV, ciphertext or tag of a frame in place."""
    start = {"iv": 1, "ct": 13, "tag": 13 + plen}[field]
    frame[start + bit // 8] ^= np.uint8(1 << (bit % 8))
