"""Seal straight into pinned host memory.

Pinned host memory (cudaHostAlloc, torch `pin_memory=True`) is mapped into the
device's address space at the same address, so seal_async and
seal_batch_async can write frames directly into it: the persistent-store path
without a separate device-to-host copy. The frames must equal the OpenSSL EVP
frames; the host-side check (`hostmem.device_mapped`) must hold first.
"""

import numpy as np
import pytest
import torch

from confkv_b200 import hostmem, workloads
from confkv_b200.batch import DeviceBatch
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
