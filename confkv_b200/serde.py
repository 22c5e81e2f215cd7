"""LMCache serde backend on the B200 AES-128-GCM engine.

Drop-in counterpart of ConfKV's CPU serde plugins
(experiments/gpu_kv_seal/integration/native_aesgcm_serde.py:104-298): the same
Serializer / Deserializer interface, the same HKDF key lookup per object
(info prefix b"lmcache-l2-aesgcm-v1", key = provider.get_key(key.cache_salt)),
a fresh os.urandom IV per frame, the same frame [1 | IV | C | T] and P + 29
size estimate, InvalidTag on authentication failure with the destination
zeroed. What changes is where the work runs:

    GPU plaintext KV (MemoryObj.tensor on cuda)
      -> seal on the GPU -> device frame -> (if the destination is host memory)
         D2H copy on the same stream -> storage

and the reverse for deserialize (host frame -> H2D -> authenticated open ->
plaintext written to the device tensor only after the tag verified).

Objects are duck-typed like LMCache's MemoryObj: `.tensor` (a contiguous
torch tensor on a CUDA device or on the host) if present, else `.byte_array`
(a host buffer). Registered as serde type "gpu_aesgcm"; ConfKV's
LMCACHE_AESGCM_BACKEND switch selects it with the value "gpu".
"""

from __future__ import annotations

import itertools
import os
import threading
from collections import defaultdict
from concurrent.futures import ThreadPoolExecutor

from cryptography.exceptions import InvalidTag
from lmcache.v1.distributed.serde.async_processor import AsyncSerdeProcessor
from lmcache.v1.distributed.serde.base import Deserializer, Serializer
from lmcache.v1.distributed.serde.factory import register_serde_factory
from lmcache.v1.distributed.serde.key_provider import HkdfKeyProvider

from .gpu_aesgcm import FRAME_OVERHEAD, GpuAes128GcmKey, GpuAesGcmLibrary

HKDF_INFO_PREFIX = b"lmcache-l2-aesgcm-v1"
SERDE_TYPE = "gpu_aesgcm"


def _bytes_view(obj):
    """uint8 torch view of a MemoryObj-like object (no copy)."""
    import torch

    t = getattr(obj, "tensor", None)
    if t is not None:
        if not t.is_contiguous():
            raise ValueError("gpu aesgcm: tensor must be contiguous")
        return t.reshape(-1).view(torch.uint8)
    mv = memoryview(obj.byte_array).cast("B")
    if len(mv) == 0:
        return torch.empty(0, dtype=torch.uint8)
    return torch.frombuffer(mv, dtype=torch.uint8)


def _plaintext_bytes(layout_desc) -> int:
    import torch

    total = 0
    for shape, dtype in zip(layout_desc.shapes, layout_desc.dtypes, strict=True):
        n = 1
        for d in shape:
            n *= int(d)
        total += n * torch.empty((), dtype=dtype).element_size()
    return total


class GpuSerdeContext:
    """State shared by a serializer/deserializer pair: the device, one key
    handle per data-encryption key, and one CUDA stream per worker thread."""

    def __init__(self, key_provider, device: int | None = None, library: GpuAesGcmLibrary | None = None):
        self.keys = key_provider
        self._device = device
        self._library = library
        self._handles: dict[bytes, GpuAes128GcmKey] = {}
        self._lock = threading.Lock()
        self._local = threading.local()

    @property
    def device(self) -> int:
        if self._device is None:
            import torch

            self._device = torch.cuda.current_device()
        return self._device

    def handle(self, dek: bytes) -> GpuAes128GcmKey:
        if len(dek) != 16:
            raise ValueError("gpu aesgcm supports AES-128 only")
        with self._lock:
            h = self._handles.get(dek)
            if h is None:
                if self._library is None:
                    self._library = GpuAesGcmLibrary()
                h = GpuAes128GcmKey(self._library, dek, device=self.device)
                self._handles[dek] = h
            return h

    def stream(self):
        import torch

        s = getattr(self._local, "stream", None)
        if s is None:
            s = torch.cuda.Stream(device=self.device)
            self._local.stream = s
        return s

    def batch(self, count: int):
        """This thread's DeviceBatch with room for `count` objects (grown by
        doubling; the descriptor array and workspace are reused)."""
        from .batch import DeviceBatch

        b = getattr(self._local, "batch", None)
        if b is None or b.capacity < count:
            cap = max(count, 2 * b.capacity if b is not None else 64)
            if self._library is None:
                self._library = GpuAesGcmLibrary()
            b = DeviceBatch(self._library, cap, self.device)
            self._local.batch = b
        return b

    def close(self) -> None:
        with self._lock:
            for h in self._handles.values():
                h.close()
            self._handles.clear()


class GpuAesGcmSerializer(Serializer):
    def __init__(self, ctx: GpuSerdeContext):
        self._ctx = ctx

    def serialize(self, src, dst, key) -> int:
        import torch

        ctx = self._ctx
        src_t, dst_t = _bytes_view(src), _bytes_view(dst)
        plaintext_len = src_t.numel()
        frame_len = plaintext_len + FRAME_OVERHEAD
        if dst_t.numel() < frame_len:
            raise ValueError("gpu aesgcm: destination too small")
        gkey = ctx.handle(ctx.keys.get_key(key.cache_salt))
        iv = os.urandom(12)
        stream = ctx.stream()
        dev = torch.device("cuda", ctx.device)
        with torch.cuda.stream(stream):
            if plaintext_len == 0:
                src_d = torch.empty(1, dtype=torch.uint8, device=dev)
            elif src_t.is_cuda:
                src_d = src_t
            else:
                src_d = src_t.to(dev, non_blocking=True)
            frame_d = dst_t if dst_t.is_cuda else torch.empty(frame_len, dtype=torch.uint8, device=dev)
            gkey.seal_async(src_ptr=src_d.data_ptr(), plaintext_len=plaintext_len, dst_ptr=frame_d.data_ptr(),
                            dst_capacity=frame_d.numel(), iv=iv, stream_ptr=stream.cuda_stream)
            if not dst_t.is_cuda:
                dst_t[:frame_len].copy_(frame_d[:frame_len], non_blocking=True)
        stream.synchronize()
        return frame_len

    def estimate_serialized_size(self, layout_desc) -> int:
        return _plaintext_bytes(layout_desc) + FRAME_OVERHEAD


class GpuAesGcmDeserializer(Deserializer):
    def __init__(self, ctx: GpuSerdeContext):
        self._ctx = ctx

    def deserialize(self, src, dst, key) -> None:
        import torch

        ctx = self._ctx
        src_t, dst_t = _bytes_view(src), _bytes_view(dst)
        plaintext_len = dst_t.numel()
        frame_len = plaintext_len + FRAME_OVERHEAD
        if src_t.numel() < frame_len:
            raise ValueError("gpu aesgcm: malformed frame")
        gkey = ctx.handle(ctx.keys.get_key(key.cache_salt))
        stream = ctx.stream()
        dev = torch.device("cuda", ctx.device)
        with torch.cuda.stream(stream):
            frame_d = src_t if src_t.is_cuda else src_t[:frame_len].to(dev, non_blocking=True)
            out_d = dst_t if dst_t.is_cuda and plaintext_len else torch.empty(max(plaintext_len, 1),
                                                                               dtype=torch.uint8, device=dev)
            auth = torch.zeros(1, dtype=torch.int32, device=dev)
            gkey.open_async(src_ptr=frame_d.data_ptr(), frame_len=frame_len, dst_ptr=out_d.data_ptr(),
                            plaintext_len=plaintext_len, auth_ok_ptr=auth.data_ptr(), stream_ptr=stream.cuda_stream)
            if plaintext_len and not dst_t.is_cuda:
                dst_t.copy_(out_d[:plaintext_len], non_blocking=True)
            auth_h = auth.to("cpu", non_blocking=True)
        stream.synchronize()
        if int(auth_h.item()) != 1:
            # the kernel zero-filled the plaintext destination
            raise InvalidTag("gpu aesgcm authentication failed")


def _device_view(t, dev, n: int):
    """`t` itself when it is on the device, else a device copy of its first n
    bytes (a 1-byte placeholder when n == 0)."""
    import torch

    if n == 0:
        return torch.empty(1, dtype=torch.uint8, device=dev)
    return t if t.is_cuda else t[:n].to(dev, non_blocking=True)


class GpuAesGcmSerdeProcessor(AsyncSerdeProcessor):
    """AsyncSerdeProcessor whose multi-object submits run as one batched
    seal / open call per data-encryption key (lmcache_gpu_aes128gcm_*_batch_async)
    instead of one call per object; single-object submits take the
    per-object path. A batched deserialize reports False when any object
    fails authentication; every failed object's destination is zeroed and the
    authentic ones are written. Also releases the GPU key handles on close."""

    def __init__(self, ctx: GpuSerdeContext, max_workers: int = 1):
        super().__init__(GpuAesGcmSerializer(ctx), GpuAesGcmDeserializer(ctx), max_workers=max_workers)
        self._ctx = ctx
        self._bpool = ThreadPoolExecutor(max_workers=max(1, int(max_workers)))
        self._bids = itertools.count(1 << 40)   # disjoint from the base class's task ids
        self._btasks = {}
        self._block = threading.Lock()

    # ---- batched tasks
    def _bsubmit(self, fn, srcs, dsts, keys):
        tid = next(self._bids)
        with self._block:
            self._btasks[tid] = self._bpool.submit(fn, list(srcs), list(dsts), list(keys))
        return tid

    def _bquery(self, tid):
        with self._block:
            fut = self._btasks.get(tid)
        if fut is None or not fut.done():
            return None
        with self._block:
            self._btasks.pop(tid, None)
        return fut.exception() is None

    def _groups(self, keys):
        groups = defaultdict(list)
        for i, k in enumerate(keys):
            groups[self._ctx.keys.get_key(k.cache_salt)].append(i)
        return groups

    def _seal_many(self, srcs, dsts, keys):
        import torch

        ctx = self._ctx
        dev = torch.device("cuda", ctx.device)
        stream = ctx.stream()
        for dek, idx in self._groups(keys).items():
            handle = ctx.handle(dek)
            keep, copies, entries = [], [], []
            with torch.cuda.stream(stream):
                for i in idx:
                    src_t, dst_t = _bytes_view(srcs[i]), _bytes_view(dsts[i])
                    P = src_t.numel()
                    F = P + FRAME_OVERHEAD
                    if dst_t.numel() < F:
                        raise ValueError("gpu aesgcm: destination too small")
                    src_d = _device_view(src_t, dev, P)
                    frame_d = dst_t if dst_t.is_cuda else torch.empty(F, dtype=torch.uint8, device=dev)
                    entries.append((src_d.data_ptr(), frame_d.data_ptr(), P, frame_d.numel(), os.urandom(12)))
                    keep += [src_d, frame_d]
                    if not dst_t.is_cuda:
                        copies.append((dst_t, frame_d, F))
                batch = ctx.batch(len(entries))
                batch.seal(handle, entries, stream)
                for dst_t, frame_d, F in copies:
                    dst_t[:F].copy_(frame_d[:F], non_blocking=True)
                status = batch.statuses().to("cpu", non_blocking=True)
            stream.synchronize()
            if bool(status.any()):
                raise ValueError("gpu aesgcm: an object descriptor was rejected")
        return True

    def _open_many(self, srcs, dsts, keys):
        import torch

        ctx = self._ctx
        dev = torch.device("cuda", ctx.device)
        stream = ctx.stream()
        failed = False
        for dek, idx in self._groups(keys).items():
            handle = ctx.handle(dek)
            keep, copies, entries = [], [], []
            with torch.cuda.stream(stream):
                auth = torch.zeros(len(idx), dtype=torch.int32, device=dev)
                for j, i in enumerate(idx):
                    src_t, dst_t = _bytes_view(srcs[i]), _bytes_view(dsts[i])
                    P = dst_t.numel()
                    F = P + FRAME_OVERHEAD
                    if src_t.numel() < F:
                        raise ValueError("gpu aesgcm: malformed frame")
                    frame_d = _device_view(src_t, dev, F)
                    out_d = dst_t if dst_t.is_cuda and P else torch.empty(max(P, 1), dtype=torch.uint8, device=dev)
                    entries.append((frame_d.data_ptr(), out_d.data_ptr(), P, F, auth.data_ptr() + 4 * j))
                    keep += [frame_d, out_d]
                    if P and not dst_t.is_cuda:
                        copies.append((dst_t, out_d, P))
                batch = ctx.batch(len(entries))
                batch.open(handle, entries, stream)
                for dst_t, out_d, P in copies:
                    dst_t.copy_(out_d[:P], non_blocking=True)
                auth_h = auth.to("cpu", non_blocking=True)
                status = batch.statuses().to("cpu", non_blocking=True)
            stream.synchronize()
            if bool(status.any()):
                raise ValueError("gpu aesgcm: an object descriptor was rejected")
            failed = failed or bool((auth_h != 1).any())
        if failed:
            # the kernels zero-filled every rejected object's plaintext
            raise InvalidTag("gpu aesgcm authentication failed")
        return True

    # ---- SerdeProcessor interface
    def submit_serialize(self, srcs, dsts, keys):
        if len(srcs) < 2:
            return super().submit_serialize(srcs, dsts, keys)
        return self._bsubmit(self._seal_many, srcs, dsts, keys)

    def submit_deserialize(self, srcs, dsts, keys):
        if len(srcs) < 2:
            return super().submit_deserialize(srcs, dsts, keys)
        return self._bsubmit(self._open_many, srcs, dsts, keys)

    def query_serialize_result(self, tid):
        if tid in self._btasks:
            return self._bquery(tid)
        return super().query_serialize_result(tid)

    def query_deserialize_result(self, tid):
        if tid in self._btasks:
            return self._bquery(tid)
        return super().query_deserialize_result(tid)

    def close(self):
        self._bpool.shutdown(wait=True)
        super().close()
        self._ctx.close()


def create_gpu_aesgcm_serde(kwargs: dict) -> GpuAesGcmSerdeProcessor:
    """Factory with the kwargs of native_aesgcm_serde.py:236-292 plus
    `device` (CUDA ordinal; default the current device)."""
    if int(kwargs.get("aes_bits", 128)) != 128:
        raise ValueError("gpu aesgcm supports aes_bits=128 only")
    master_key_path = str(kwargs.get("master_key_path", ""))
    if not master_key_path:
        raise ValueError("gpu_aesgcm requires master_key_path")
    with open(master_key_path, "rb") as f:
        master_key = f.read()
    provider = HkdfKeyProvider(master_key, key_len=16, info_prefix=HKDF_INFO_PREFIX)
    device = kwargs.get("device")
    ctx = GpuSerdeContext(provider, device=None if device is None else int(device))
    return GpuAesGcmSerdeProcessor(ctx, max_workers=int(kwargs.get("max_workers", 1)))


register_serde_factory(SERDE_TYPE, create_gpu_aesgcm_serde)
