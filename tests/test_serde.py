"""LMCache serde backend switch with the GPU backend (confkv_b200.serde).

LMCache itself is absent from this image, so the "aesgcm" serde type with its
stock / native backends comes from the test-only stand-in under
tests/fake_lmcache (rebuilt from ConfKV's call sites). Ports:
  - scripts/test_backend_switch.py:41-187  (stock <-> native, now <-> gpu)
  - scripts/test_native_async_serde.py:115-289 (registration, estimate, async
    round trip, async tamper -> False + zeroed output)
  - scripts/test_native_security.py:104-271 (wrong tenant, flips in ct/tag/IV)
and the persistent-store path: device KV tensor -> GPU seal -> host frame ->
GPU open into a device tensor.
"""

import ctypes
import os
import sys
import time
from pathlib import Path

import numpy as np
import pytest

FAKE = Path(__file__).resolve().parent / "fake_lmcache"
if str(FAKE) not in sys.path:
    sys.path.insert(0, str(FAKE))

from lmcache.v1.distributed.api import MemoryLayoutDesc, ObjectKey  # noqa: E402
from lmcache.v1.distributed.serde.base import SerdeConfig  # noqa: E402
from lmcache.v1.distributed.serde.factory import (  # noqa: E402
    create_serde_processor,
    get_registered_serde_types,
)

import confkv_b200.serde as gpu_serde  # noqa: E402,F401  (registers "gpu_aesgcm")

SIZE = 4 * 1024 * 1024
MASTER = b"paper-benchmark-master-key-32bytes!!"
KEY = ObjectKey(chunk_hash=b"\x11" * 32, model_name="paper-benchmark", kv_rank=0, cache_salt="tenant-a")
OTHER_TENANT = ObjectKey(chunk_hash=b"\x11" * 32, model_name="paper-benchmark", kv_rank=0, cache_salt="tenant-b")


class Buf:
    """Host MemoryObj stand-in (scripts/test_native_async_serde.py:36-74)."""

    def __init__(self, capacity):
        self._arr = (ctypes.c_ubyte * capacity)()
        self._capacity = capacity
        self._used = capacity

    @property
    def byte_array(self):
        return memoryview(self._arr)[:self._used]

    @property
    def address(self):
        return ctypes.addressof(self._arr)

    def bytes(self):
        return bytes(memoryview(self._arr)[:self._used])


class DevObj:
    """Device MemoryObj stand-in: exposes `.tensor`."""

    def __init__(self, tensor):
        self.tensor = tensor


@pytest.fixture
def key_path(tmp_path):
    p = tmp_path / "master.key"
    p.write_bytes(MASTER)
    return str(p)


def processor(backend, key_path, **extra):
    os.environ["LMCACHE_AESGCM_BACKEND"] = backend
    try:
        return create_serde_processor(SerdeConfig(type="aesgcm", kwargs={
            "master_key_path": key_path, "aes_bits": 128, "max_workers": 1, **extra}))
    finally:
        os.environ.pop("LMCACHE_AESGCM_BACKEND", None)


def wait(query, task):
    deadline = time.monotonic() + 30
    while time.monotonic() < deadline:
        r = query(task)
        if r is not None:
            return r
        time.sleep(0.001)
    raise TimeoutError


def run_ser(proc, src, dst, key=KEY):
    return wait(proc.query_serialize_result, proc.submit_serialize([src], [dst], [key]))


def run_de(proc, src, dst, key=KEY):
    return wait(proc.query_deserialize_result, proc.submit_deserialize([src], [dst], [key]))


# --------------------------------------------------------------- CPU-only

def test_gpu_type_registered_and_estimate():
    assert "gpu_aesgcm" in get_registered_serde_types()
    assert "aesgcm" in get_registered_serde_types()
    layout = MemoryLayoutDesc(shapes=[__import__("torch").Size([SIZE // 2])],
                              dtypes=[__import__("torch").bfloat16])
    ctx = gpu_serde.GpuSerdeContext(key_provider=None)
    assert gpu_serde.GpuAesGcmSerializer(ctx).estimate_serialized_size(layout) == SIZE + 29


def test_gpu_factory_validates_config(key_path):
    with pytest.raises(ValueError):
        gpu_serde.create_gpu_aesgcm_serde({"master_key_path": key_path, "aes_bits": 256})
    with pytest.raises(ValueError):
        gpu_serde.create_gpu_aesgcm_serde({"aes_bits": 128})


def test_backend_switch_values(key_path):
    from lmcache.v1.distributed.serde import aesgcm

    for v in ("stock", "native", "gpu", "GPU "):
        os.environ["LMCACHE_AESGCM_BACKEND"] = v
        assert aesgcm.backend_name() == v.strip().lower()
    os.environ["LMCACHE_AESGCM_BACKEND"] = "tpu"
    with pytest.raises(ValueError):
        aesgcm.backend_name()
    os.environ.pop("LMCACHE_AESGCM_BACKEND")
    assert aesgcm.backend_name() == "stock"


# --------------------------------------------------------------- GPU

@pytest.mark.gpu
@pytest.mark.parametrize("other", ["stock", "native"])
def test_backend_switch_cross_open(key_path, other):
    src = Buf(SIZE)
    ctypes.memset(src.address, 0xA5, SIZE)
    gpu = processor("gpu", key_path)
    cpu = processor(other, key_path)
    try:
        # other seal -> gpu open
        frame = Buf(cpu.estimate_serialized_size(MemoryLayoutDesc([__import__("torch").Size([SIZE])],
                                                                   [__import__("torch").uint8])))
        assert run_ser(cpu, src, frame) is True
        out = Buf(SIZE)
        assert run_de(gpu, frame, out) is True
        assert out.bytes() == src.bytes()
        # gpu seal -> other open
        frame2 = Buf(SIZE + 29)
        assert run_ser(gpu, src, frame2) is True
        assert frame2.bytes()[0] == 1
        out2 = Buf(SIZE)
        assert run_de(cpu, frame2, out2) is True
        assert out2.bytes() == src.bytes()
    finally:
        gpu.close()
        cpu.close()


@pytest.mark.gpu
def test_async_gpu_serde_round_trip_and_tamper(key_path):
    proc = create_serde_processor(SerdeConfig(type="gpu_aesgcm", kwargs={
        "master_key_path": key_path, "aes_bits": 128, "max_workers": 2}))
    try:
        src = Buf(SIZE)
        ctypes.memset(src.address, 0xA5, SIZE)
        frame = Buf(SIZE + 29)
        assert run_ser(proc, src, frame) is True
        out = Buf(SIZE)
        assert run_de(proc, frame, out) is True
        assert out.bytes() == src.bytes()
        memoryview(frame._arr).cast("B")[13 + SIZE // 2] ^= 0x01
        ctypes.memset(out.address, 0xCC, SIZE)
        assert run_de(proc, frame, out) is False
        assert not any(out.bytes())
    finally:
        proc.close()


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["wrong_tenant", "ciphertext", "tag", "iv", "version"])
def test_gpu_serde_security(key_path, case):
    stock = processor("stock", key_path)
    gpu = processor("gpu", key_path)
    try:
        src = Buf(SIZE)
        ctypes.memset(src.address, 0x5A, SIZE)
        frame = Buf(SIZE + 29)
        assert run_ser(stock, src, frame) is True
        fv = memoryview(frame._arr).cast("B")
        key = KEY
        if case == "wrong_tenant":
            key = OTHER_TENANT
        elif case == "ciphertext":
            fv[13 + SIZE // 2] ^= 0x01
        elif case == "tag":
            fv[-1] ^= 0x01
        elif case == "iv":
            fv[1] ^= 0x01
        else:
            fv[0] = 2
        out = Buf(SIZE)
        ctypes.memset(out.address, 0xCC, SIZE)
        assert run_de(gpu, frame, out, key) is False
        assert not any(out.bytes())
    finally:
        stock.close()
        gpu.close()


@pytest.mark.gpu
def test_device_kv_tensor_to_host_frame_and_back(key_path):
    """The persistent-store path: bf16 KV tensor in HBM -> GPU seal -> host
    frame (what storage receives) -> GPU open back into an HBM tensor."""
    import torch

    from confkv_b200 import workloads

    kv = workloads.bf16_batch(workloads.SHAPES["kv_small"], 1, seed=11, device="cuda")[0]
    P = kv.numel() * kv.element_size()
    gpu = processor("gpu", key_path)
    native = processor("native", key_path)
    try:
        frame = Buf(P + 29)
        assert run_ser(gpu, DevObj(kv), frame) is True
        # storage-side check with the reference's OpenSSL backend
        host_out = Buf(P)
        assert run_de(native, frame, host_out) is True
        assert host_out.bytes() == kv.view(torch.uint8).cpu().numpy().tobytes()
        restored = torch.empty_like(kv)
        assert run_de(gpu, frame, DevObj(restored)) is True
        assert torch.equal(restored.view(torch.uint8), kv.view(torch.uint8))
        # device frame destination too (seal into HBM, e.g. before a batched D2H)
        dframe = torch.empty(P + 29, dtype=torch.uint8, device="cuda")
        assert run_ser(gpu, DevObj(kv), DevObj(dframe)) is True
        restored2 = torch.zeros_like(kv)
        assert run_de(gpu, DevObj(dframe), DevObj(restored2)) is True
        assert torch.equal(restored2, kv)
        dframe[13 + 100] ^= 1
        assert run_de(gpu, DevObj(dframe), DevObj(restored2)) is False
        assert not bool(restored2.view(torch.uint8).any())
    finally:
        gpu.close()
        native.close()


def run_ser_many(proc, srcs, dsts, keys):
    return wait(proc.query_serialize_result, proc.submit_serialize(srcs, dsts, keys))


def run_de_many(proc, srcs, dsts, keys):
    return wait(proc.query_deserialize_result, proc.submit_deserialize(srcs, dsts, keys))


@pytest.mark.gpu
def test_gpu_serde_multi_object_batches(key_path):
    """A multi-object submit runs as one batched call per data-encryption key
    (two tenants here): frames open with the reference's native backend, and
    a batched open of native frames restores every object; one tampered
    frame makes the task report False with only that object zeroed."""
    import torch

    sizes = [1, 17, 4096, (1 << 20) + 3, SIZE, 33]
    keys = [KEY if i % 2 == 0 else OTHER_TENANT for i in range(len(sizes))]
    rng = np.random.default_rng(5)
    srcs = []
    for n in sizes:
        b = Buf(n)
        ctypes.memmove(b.address, rng.integers(0, 256, size=n, dtype=np.uint8).tobytes(), n)
        srcs.append(b)
    gpu = processor("gpu", key_path)
    native = processor("native", key_path)
    try:
        frames = [Buf(n + 29) for n in sizes]
        assert run_ser_many(gpu, srcs, frames, keys) is True
        for s, f, k in zip(srcs, frames, keys):
            out = Buf(len(s.bytes()))
            assert run_de(native, f, out, k) is True
            assert out.bytes() == s.bytes()
        # native seal -> GPU batched open, host and device destinations mixed
        nframes = [Buf(n + 29) for n in sizes]
        for s, f, k in zip(srcs, nframes, keys):
            assert run_ser(native, s, f, k) is True
        outs = [Buf(n) if i % 3 else DevObj(torch.zeros(n, dtype=torch.uint8, device="cuda"))
                for i, n in enumerate(sizes)]
        assert run_de_many(gpu, nframes, outs, keys) is True
        for s, o in zip(srcs, outs):
            got = o.bytes() if isinstance(o, Buf) else o.tensor.cpu().numpy().tobytes()
            assert got == s.bytes()
        # one tampered frame: task False, that object zeroed, the rest restored
        memoryview(nframes[3]._arr).cast("B")[13 + 1000] ^= 0x10
        outs = [Buf(n) for n in sizes]
        for o in outs:
            ctypes.memset(o.address, 0xCC, len(o.bytes()))
        assert run_de_many(gpu, nframes, outs, keys) is False
        for i, (s, o) in enumerate(zip(srcs, outs)):
            if i == 3:
                assert not any(o.bytes())
            else:
                assert o.bytes() == s.bytes()
    finally:
        gpu.close()
        native.close()
