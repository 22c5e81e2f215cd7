"""lmcache_gpu_aes128gcm_seal_noalloc against the keyed seal.

This entry point is for callers that cannot call cudaMalloc at the moment
they seal: a KV-cache server whose memory pool already owns the device's
memory, or a pipeline thread that must not take cudaMalloc's implicit device
synchronisation. It takes the raw key and keeps its working memory (key
tables, accumulation slot) in one static device array shared by every call.
Consecutive calls must therefore still produce frames byte-identical to
lmcache_gpu_aes128gcm_seal_async's, even though each call inherits the array
the previous call left behind (same key: cached tables; new key: re-upload).

This file is named to be collected last, and passes both alone in a fresh
process and after the rest of the suite.
"""

import ctypes

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


def test_noalloc_seal_matches_keyed_seal_on_consecutive_calls(gpu_lib):
    seal_noalloc = _seal_noalloc(gpu_lib)
    rng = np.random.default_rng(2026)
    key_a, key_b = rng.bytes(16), rng.bytes(16)
    stream = torch.cuda.Stream()
    # (key, plaintext bytes, frame offset in its buffer): calls 1 and 2 reuse
    # key A's tables left in the array, call 3 switches key, call 4 is empty.
    calls = [(key_a, (32 << 20) + 5, 0), (key_a, 2 << 20, 3), (key_b, 100_003, 0), (key_b, 0, 0)]
    for n_call, (key, size, off) in enumerate(calls):
        g = torch.Generator(device="cuda")
        g.manual_seed(n_call)
        plain = torch.randint(0, 256, (max(size, 1),), generator=g, device="cuda", dtype=torch.uint8)
        iv = rng.bytes(12)
        expected = torch.full((off + size + 29,), 0x5A, dtype=torch.uint8, device="cuda")
        got = torch.full((off + size + 29,), 0xA5, dtype=torch.uint8, device="cuda")
        with GpuAes128GcmKey(gpu_lib, key) as k:
            k.seal_async(src_ptr=plain.data_ptr(), plaintext_len=size, dst_ptr=expected.data_ptr() + off,
                         dst_capacity=size + 29, iv=iv, stream_ptr=stream.cuda_stream)
            stream.synchronize()
        iv_buf = (ctypes.c_uint8 * 12).from_buffer_copy(iv)
        rc = seal_noalloc(key, 16, ctypes.c_void_p(plain.data_ptr()), size, ctypes.c_void_p(got.data_ptr() + off),
                          size + 29, iv_buf, torch.cuda.current_device(), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, gpu_lib.error_string(rc)
        stream.synchronize()
        assert torch.equal(got[off:], expected[off:]), f"call {n_call}: frame differs from the keyed seal"
        assert bool((got[:off] == 0xA5).all()), f"call {n_call}: wrote before the frame"


def test_noalloc_seal_rejects_objects_above_its_limit(gpu_lib):
    seal_noalloc = _seal_noalloc(gpu_lib)
    iv_buf = (ctypes.c_uint8 * 12)()
    p = ctypes.c_void_p(0x1000)
    big = (1 << 30) + 1
    assert seal_noalloc(bytes(16), 16, p, big, p, big + 29, iv_buf, 0, None) == -1
