"""lmcache_gpu_aes128gcm_seal_noalloc against the keyed seal.

This entry point is for callers that cannot call cudaMalloc at the moment
they seal: a KV-cache server whose memory pool already owns the device's
memory, or a pipeline thread that must not take cudaMalloc's implicit device
synchronisation. It takes the raw key and keeps its working memory (key
tables, accumulation slot) in one static device array shared by every call;
a small kernel ahead of each seal checks, on the device, which key the array's
tables belong to and rebuilds them on a key change. Consecutive calls must
therefore still produce frames byte-identical to
lmcache_gpu_aes128gcm_seal_async's, even though each call inherits the array
the previous call left behind (same key: tables kept; another key, or a
return to an earlier one: tables rebuilt).

This file is named to be collected last, and passes both alone in a fresh
process and after the rest of the suite.
"""

import ctypes
import threading

import numpy as np
import pytest
import torch

from confkv_b200.gpu_aesgcm import GpuAes128GcmKey

pytestmark = pytest.mark.gpu


def _seal_noalloc(lib):
    f = lib.lib.lmcache_gpu_aes128gcm_seal_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                  ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _keyed_frame(lib, key: bytes, plain: torch.Tensor, src_off: int, size: int, iv: bytes, stream) -> torch.Tensor:
    """The frame lmcache_gpu_aes128gcm_seal_async writes for the same inputs."""
    out = torch.full((size + 29,), 0x5A, dtype=torch.uint8, device="cuda")
    with GpuAes128GcmKey(lib, key) as k:
        k.seal_async(src_ptr=plain.data_ptr() + src_off, plaintext_len=size, dst_ptr=out.data_ptr(),
                     dst_capacity=size + 29, iv=iv, stream_ptr=stream.cuda_stream)
        stream.synchronize()
    return out


def test_noalloc_seal_matches_keyed_seal_on_consecutive_calls(gpu_lib):
    seal_noalloc = _seal_noalloc(gpu_lib)
    rng = np.random.default_rng(2026)
    key_a, key_b = rng.bytes(16), rng.bytes(16)
    stream = torch.cuda.Stream()
    # (key, plaintext bytes, source offset, frame offset): call 2 reuses key
    # A's tables, call 3 switches to B, call 4 returns to A (tables rebuilt
    # again), calls 3 and 5 read a misaligned source, call 6 is empty.
    calls = [(key_a, (32 << 20) + 5, 0, 0), (key_a, 2 << 20, 0, 3), (key_b, 100_003, 7, 0),
             (key_a, (1 << 20) + 9, 0, 5), (key_a, 65_536 * 3 + 1, 13, 11), (key_b, 0, 0, 0)]
    for n_call, (key, size, src_off, off) in enumerate(calls):
        g = torch.Generator(device="cuda")
        g.manual_seed(n_call)
        plain = torch.randint(0, 256, (max(size, 1) + src_off,), generator=g, device="cuda", dtype=torch.uint8)
        iv = rng.bytes(12)
        expected = _keyed_frame(gpu_lib, key, plain, src_off, size, iv, stream)
        got = torch.full((off + size + 29,), 0xA5, dtype=torch.uint8, device="cuda")
        iv_buf = (ctypes.c_uint8 * 12).from_buffer_copy(iv)
        rc = seal_noalloc(key, 16, ctypes.c_void_p(plain.data_ptr() + src_off), size,
                          ctypes.c_void_p(got.data_ptr() + off), size + 29, iv_buf, torch.cuda.current_device(),
                          ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, gpu_lib.error_string(rc)
        stream.synchronize()
        assert torch.equal(got[off:], expected), f"call {n_call}: frame differs from the keyed seal"
        assert bool((got[:off] == 0xA5).all()), f"call {n_call}: wrote before the frame"


def test_noalloc_seal_two_threads_alternating_keys_on_one_stream(gpu_lib):
    """Two host threads issue calls with different keys on the same stream at
    once; every frame must still be the keyed seal's frame for its own key."""
    seal_noalloc = _seal_noalloc(gpu_lib)
    rng = np.random.default_rng(77)
    keys = [rng.bytes(16), rng.bytes(16)]
    stream = torch.cuda.Stream()
    calls_per_thread = 24
    size = (1 << 20) + 3
    plain = torch.randint(0, 256, (size,), dtype=torch.uint8, device="cuda")
    ivs = [[rng.bytes(12) for _ in range(calls_per_thread)] for _ in keys]
    frames = [[torch.zeros(size + 29, dtype=torch.uint8, device="cuda") for _ in range(calls_per_thread)]
              for _ in keys]
    dev = torch.cuda.current_device()
    errors = []
    start = threading.Barrier(len(keys))

    def worker(t):
        try:
            start.wait()
            for k in range(calls_per_thread):
                iv_buf = (ctypes.c_uint8 * 12).from_buffer_copy(ivs[t][k])
                rc = seal_noalloc(keys[t], 16, ctypes.c_void_p(plain.data_ptr()), size,
                                  ctypes.c_void_p(frames[t][k].data_ptr()), size + 29, iv_buf, dev,
                                  ctypes.c_void_p(stream.cuda_stream))
                if rc != 0:
                    errors.append((t, k, rc))
        except Exception as exc:  # pragma: no cover - reported below
            errors.append((t, -1, repr(exc)))

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(len(keys))]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    stream.synchronize()
    assert not errors, errors
    for t, key in enumerate(keys):
        for k in range(calls_per_thread):
            expected = _keyed_frame(gpu_lib, key, plain, 0, size, ivs[t][k], stream)
            assert torch.equal(frames[t][k], expected), f"thread {t} call {k}: frame differs from the keyed seal"


def test_noalloc_seal_rejects_objects_above_its_limit(gpu_lib):
    seal_noalloc = _seal_noalloc(gpu_lib)
    iv_buf = (ctypes.c_uint8 * 12)()
    p = ctypes.c_void_p(0x1000)
    big = (1 << 30) + 1
    assert seal_noalloc(bytes(16), 16, p, big, p, big + 29, iv_buf, 0, None) == -1
