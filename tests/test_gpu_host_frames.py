"""Frames in pinned host memory: the store and load paths.

Pinned host memory (cudaHostAlloc, torch `pin_memory=True`) is mapped into the
device's address space at the same address, so seal_async and
seal_batch_async can write frames directly into it: the persistent-store path
without a separate device-to-host copy. The frames must equal the OpenSSL EVP
frames; the host-side check (`hostmem.device_mapped`) must hold first. The
load path copies frames from pinned host memory in on a side stream and opens
each one as soon as it has arrived; tampered frames are rejected and zeroed.
"""

import numpy as np
import pytest
import torch

from confkv_b200 import hostmem, workloads
from confkv_b200.batch import DeviceBatch
from confkv_b200.configs import RankWork, random_plain
from confkv_b200.gpu_aesgcm import GpuAes128GcmKey

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 17, 4096, 16 * 1024 + 16, (1 << 20) + 3, (5 << 20) + 11]


def _layout(sizes, pad=7):
    offs, pos = [], 0
    for n in sizes:
        offs.append(pos)
        pos += n + 29 + pad
    return offs, pos


def test_seal_async_into_pinned_host(gpu_lib, oracle):
    key = workloads.make_key(31)
    ivs = workloads.make_ivs(31, len(SIZES))
    rng = np.random.default_rng(31)
    pts = [rng.integers(0, 256, size=n, dtype=np.uint8) for n in SIZES]
    offs, total = _layout(SIZES)
    host = torch.full((total,), 0xAB, dtype=torch.uint8, pin_memory=True)
    assert hostmem.device_mapped(host.data_ptr())
    d_pts = [torch.from_numpy(p).cuda() if len(p) else torch.empty(16, dtype=torch.uint8, device="cuda")
             for p in pts]
    s = torch.cuda.Stream()
    with GpuAes128GcmKey(gpu_lib, key) as k:
        for i, n in enumerate(SIZES):
            k.seal_async(src_ptr=d_pts[i].data_ptr(), plaintext_len=n, dst_ptr=host.data_ptr() + offs[i],
                         dst_capacity=n + 29, iv=ivs[i], stream_ptr=s.cuda_stream)
        s.synchronize()
    frames = host.numpy()
    expected = oracle.evp_seal_many(key, ivs, pts)
    mask = np.zeros(total, dtype=bool)
    for i, n in enumerate(SIZES):
        assert np.array_equal(frames[offs[i]:offs[i] + n + 29], expected[i]), (i, n)
        mask[offs[i]:offs[i] + n + 29] = True
    assert (frames[~mask] == 0xAB).all()


def test_seal_batch_into_pinned_host(gpu_lib, oracle):
    key = workloads.make_key(32)
    ivs = workloads.make_ivs(32, len(SIZES))
    rng = np.random.default_rng(32)
    pts = [rng.integers(0, 256, size=n, dtype=np.uint8) for n in SIZES]
    offs, total = _layout(SIZES)
    pt_offs, pt_total = [], 0
    for n in SIZES:
        pt_offs.append(pt_total)
        pt_total += n + 3
    d_plain = torch.zeros(pt_total + 16, dtype=torch.uint8, device="cuda")
    for i, p in enumerate(pts):
        if len(p):
            d_plain[pt_offs[i]:pt_offs[i] + len(p)].copy_(torch.from_numpy(p))
    host = torch.full((total,), 0xAB, dtype=torch.uint8, pin_memory=True)
    assert hostmem.device_mapped(host.data_ptr())
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, len(SIZES))
    with GpuAes128GcmKey(gpu_lib, key) as k:
        batch.seal(k, [(d_plain.data_ptr() + pt_offs[i], host.data_ptr() + offs[i], n, n + 29, ivs[i])
                       for i, n in enumerate(SIZES)], s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert not batch.statuses().any()
    frames = host.numpy()
    expected = oracle.evp_seal_many(key, ivs, pts)
    for i, n in enumerate(SIZES):
        assert np.array_equal(frames[offs[i]:offs[i] + n + 29], expected[i]), (i, n)


def test_device_mapped_rejects_pageable_memory():
    a = np.zeros(4096, dtype=np.uint8)
    assert not hostmem.device_mapped(a.ctypes.data)


def test_open_frames_from_pinned_host(gpu_lib, oracle):
    """RankWork.open_each_from_host: OpenSSL frames placed in pinned host
    memory open on the GPU after their H2D copies; one tampered frame in
    three is rejected with a zeroed output, the rest round-trip."""
    dev = torch.device("cuda", 0)
    key = workloads.make_key(33)
    lens = [n for n in SIZES for _ in range(3)]
    ivs = workloads.make_ivs(33, len(lens))
    plain, offs = random_plain(lens, seed=33, dev=dev)
    s = torch.cuda.Stream()
    with GpuAes128GcmKey(gpu_lib, key) as k:
        w = RankWork(gpu_lib, k, lens, plain, offs, s, ivs)   # runs one batched seal + open on s
        s.synchronize()
        host_plain = plain.cpu().numpy()
        expected = oracle.evp_seal_many(key, ivs, [host_plain[o:o + n] for o, n in zip(offs, lens)])
        w.host_ptr()
        bad = set(range(2, len(lens), 3))
        for i, (o, n) in enumerate(zip(w.fr_off, lens)):
            f = expected[i].copy()
            if i in bad:
                f[13 + (7 * i) % (n + 16)] ^= 0x04
            w.host[o:o + n + 29].copy_(torch.from_numpy(f))
        side = torch.cuda.Stream()
        w.out.fill_(0xCC)
        w.auth.fill_(7)
        torch.cuda.synchronize()
        w.open_each_from_host(side)
        w.open_each_from_host(side)   # a second pass over the same buffers
        s.synchronize()
        auth = w.auth.cpu().numpy()
        out = w.out.cpu().numpy()
        for i, (o, n) in enumerate(zip(offs, lens)):
            if i in bad:
                assert auth[i] == 0 and not out[o:o + n].any(), (i, n)
            else:
                assert auth[i] == 1 and np.array_equal(out[o:o + n], host_plain[o:o + n]), (i, n)
