"""Key handles bound to a device other than the caller's current one.

The reference binds a key to `device` at key_create and makes that device
current for every call, restoring the caller's device afterwards
(experiments/gpu_kv_seal/gpu/gpu_aesgcm.cu:1239-1263, used at :1506). These
tests create a key on device 1 while device 0 is current, seal and open on
device 1 through the per-object and batched calls, compare with OpenSSL, and
check that device 0 is still current after every call; then two host threads
create keys on devices 0 and 1 at once and seal concurrently. They need two
GPUs and are skipped with fewer.
"""

import ctypes
import threading

import numpy as np
import pytest
import torch

from confkv_b200.batch import DeviceBatch
from confkv_b200.gpu_aesgcm import GpuAes128GcmKey

pytestmark = pytest.mark.gpu


@pytest.fixture
def two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    torch.cuda.set_device(0)
    yield
    torch.cuda.set_device(0)


def _current() -> int:
    """The CUDA runtime's current device, read through the runtime itself."""
    return torch.cuda.current_device()


def test_key_on_other_device_per_object_and_batched(gpu_lib, oracle, two_gpus):
    rng = np.random.default_rng(4242)
    key = rng.bytes(16)
    d1 = torch.device("cuda", 1)
    sizes = [0, 17, 4096, (1 << 20) + 5, 32 << 20]
    pts = [rng.integers(0, 256, size=n, dtype=np.uint8) for n in sizes]
    ivs = [rng.bytes(12) for _ in sizes]
    srcs = [torch.from_numpy(np.concatenate([p, np.zeros(16, np.uint8)])).to(d1) for p in pts]
    frames = [torch.zeros(n + 29, dtype=torch.uint8, device=d1) for n in sizes]
    outs = [torch.full((n + 16,), 0xCC, dtype=torch.uint8, device=d1) for n in sizes]
    auth = torch.zeros(len(sizes), dtype=torch.int32, device=d1)
    s1 = torch.cuda.Stream(device=d1)
    torch.cuda.synchronize(d1)
    assert _current() == 0
    with GpuAes128GcmKey(gpu_lib, key, device=1) as k:
        assert _current() == 0, "key_create left another device current"
        for f, src, n, iv in zip(frames, srcs, sizes, ivs):
            k.seal_async(src_ptr=src.data_ptr(), plaintext_len=n, dst_ptr=f.data_ptr(), dst_capacity=n + 29, iv=iv,
                         stream_ptr=s1.cuda_stream)
        assert _current() == 0, "seal_async left another device current"
        for i, (f, o, n) in enumerate(zip(frames, outs, sizes)):
            k.open_async(src_ptr=f.data_ptr(), frame_len=n + 29, dst_ptr=o.data_ptr(), plaintext_len=n,
                         auth_ok_ptr=auth.data_ptr() + 4 * i, stream_ptr=s1.cuda_stream)
        assert _current() == 0, "open_async left another device current"
        s1.synchronize()
        assert auth.cpu().tolist() == [1] * len(sizes)
        for f, p, iv, o in zip(frames, pts, ivs, outs):
            assert f.cpu().numpy().tobytes() == oracle.evp_seal(key, iv, p).tobytes()
            assert o[:p.size].cpu().numpy().tobytes() == p.tobytes()

        # the batched calls on device 1, descriptors and workspace there too
        bframes = [torch.zeros(n + 29, dtype=torch.uint8, device=d1) for n in sizes]
        bouts = [torch.full((n + 16,), 0xCC, dtype=torch.uint8, device=d1) for n in sizes]
        bauth = torch.zeros(len(sizes), dtype=torch.int32, device=d1)
        torch.cuda.synchronize(d1)
        batch = DeviceBatch(gpu_lib, len(sizes), d1)
        batch.seal(k, [(s.data_ptr(), f.data_ptr(), n, n + 29, iv) for s, f, n, iv in zip(srcs, bframes, sizes, ivs)],
                   s1)
        assert _current() == 0, "seal_batch_async left another device current"
        batch.open(k, [(f.data_ptr(), o.data_ptr(), n, n + 29, bauth.data_ptr() + 4 * i)
                       for i, (f, o, n) in enumerate(zip(bframes, bouts, sizes))], s1)
        assert _current() == 0, "open_batch_async left another device current"
        s1.synchronize()
        assert int(batch.fault()) == 0
        assert bauth.cpu().tolist() == [1] * len(sizes)
        for f, bf in zip(frames, bframes):
            assert torch.equal(f, bf)
        for p, o in zip(pts, bouts):
            assert o[:p.size].cpu().numpy().tobytes() == p.tobytes()
    assert _current() == 0, "key_destroy left another device current"


def test_noalloc_seal_on_other_device(gpu_lib, oracle, two_gpus):
    f = gpu_lib.lib.lmcache_gpu_aes128gcm_seal_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                  ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    f.restype = ctypes.c_int
    rng = np.random.default_rng(99)
    key, iv = rng.bytes(16), rng.bytes(12)
    d1 = torch.device("cuda", 1)
    pt = rng.integers(0, 256, size=(3 << 20) + 1, dtype=np.uint8)
    src = torch.from_numpy(pt).to(d1)
    frame = torch.zeros(pt.size + 29, dtype=torch.uint8, device=d1)
    s1 = torch.cuda.Stream(device=d1)
    torch.cuda.synchronize(d1)
    rc = f(key, 16, ctypes.c_void_p(src.data_ptr()), pt.size, ctypes.c_void_p(frame.data_ptr()), pt.size + 29,
           (ctypes.c_uint8 * 12).from_buffer_copy(iv), 1, ctypes.c_void_p(s1.cuda_stream))
    assert rc == 0, gpu_lib.error_string(rc)
    assert _current() == 0
    s1.synchronize()
    assert frame.cpu().numpy().tobytes() == oracle.evp_seal(key, iv, pt).tobytes()


def test_keys_created_on_both_devices_from_two_threads(gpu_lib, oracle, two_gpus):
    rng = np.random.default_rng(7)
    keys = [rng.bytes(16), rng.bytes(16)]
    pts = [rng.integers(0, 256, size=(2 << 20) + 3 * d, dtype=np.uint8) for d in range(2)]
    ivs = [[rng.bytes(12) for _ in range(8)] for _ in range(2)]
    results = [None, None]
    errors = []
    start = threading.Barrier(2)

    def worker(d):
        try:
            dev = torch.device("cuda", d)
            src = torch.from_numpy(pts[d]).to(dev)
            frames = [torch.zeros(pts[d].size + 29, dtype=torch.uint8, device=dev) for _ in ivs[d]]
            s = torch.cuda.Stream(device=dev)
            torch.cuda.synchronize(dev)
            start.wait()
            with GpuAes128GcmKey(gpu_lib, keys[d], device=d) as k:
                for f, iv in zip(frames, ivs[d]):
                    k.seal_async(src_ptr=src.data_ptr(), plaintext_len=pts[d].size, dst_ptr=f.data_ptr(),
                                 dst_capacity=f.numel(), iv=iv, stream_ptr=s.cuda_stream)
                s.synchronize()
            results[d] = [f.cpu().numpy().tobytes() for f in frames]
        except Exception as exc:  # pragma: no cover - reported below
            errors.append((d, repr(exc)))

    threads = [threading.Thread(target=worker, args=(d,)) for d in range(2)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    for d in range(2):
        for got, iv in zip(results[d], ivs[d]):
            assert got == oracle.evp_seal(keys[d], iv, pts[d]).tobytes()
