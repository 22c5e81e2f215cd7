"""ctypes binding for the B200 AES-128-GCM library (``libgpu_aesgcm.so``).

Same classes, constants, keyword arguments and error behaviour as ConfKV's
binding (experiments/gpu_kv_seal/gpu/gpu_aesgcm.py:9-326): device pointers and
CUDA streams are plain integer addresses, a non-zero rc raises
``GpuAesGcmError`` carrying ``lmcache_gpu_aesgcm_strerror(rc)``, and
``GpuAes128GcmKey`` owns one native key handle. There is no CPU fallback: a
missing library raises ``FileNotFoundError``.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

FRAME_OVERHEAD = 29
IV_LEN = 12
KEY_LEN = 16
VERSION = 1
HEADER_LEN = 1 + IV_LEN
TAG_LEN = 16

DEFAULT_LIBRARY = Path(__file__).with_name("libgpu_aesgcm.so")

EXPORTED_SYMBOLS = (
    "lmcache_gpu_aesgcm_frame_size",
    "lmcache_gpu_aes128gcm_key_create",
    "lmcache_gpu_aes128gcm_key_destroy",
    "lmcache_gpu_aes128gcm_reserve",
    "lmcache_gpu_aes128gcm_seal_async",
    "lmcache_gpu_aes128gcm_open_async",
    "lmcache_gpu_aesgcm_strerror",
)


# Entry points beyond the reference ABI (include/gpu_aesgcm_api.h marks each
# as an extension): the seal that allocates nothing and batched seal/open.
EXTENSION_SYMBOLS = (
    "lmcache_gpu_aes128gcm_seal_noalloc",
    "lmcache_gpu_aes128gcm_batch_workspace_size",
    "lmcache_gpu_aes128gcm_seal_batch_async",
    "lmcache_gpu_aes128gcm_open_batch_async",
)


class GpuAesGcmError(RuntimeError):
    pass


class BatchItem(ctypes.Structure):
    """lmcache_gpu_aesgcm_batch_item: one object of a batched seal/open.
    Pointers are device addresses; `status` is written by the device."""

    _fields_ = [
        ("src", ctypes.c_uint64),
        ("dst", ctypes.c_uint64),
        ("plaintext_len", ctypes.c_uint64),
        ("capacity", ctypes.c_uint64),
        ("auth_ok", ctypes.c_uint64),
        ("iv", ctypes.c_uint8 * IV_LEN),
        ("status", ctypes.c_int32),
        ("reserved", ctypes.c_uint64),
    ]


assert ctypes.sizeof(BatchItem) == 64


def pack_batch_items(items) -> bytes:
    """Descriptor bytes for a batch. `items` yields tuples
    (src_ptr, dst_ptr, plaintext_len, capacity, auth_ok_ptr, iv) with iv 12
    bytes (seal) or None (open) and auth_ok_ptr 0 for seal."""
    items = list(items)
    arr = (BatchItem * len(items))()
    for k, (src, dst, plen, cap, auth, iv) in enumerate(items):
        e = arr[k]
        e.src, e.dst, e.plaintext_len, e.capacity, e.auth_ok = src, dst, plen, cap, auth
        if iv is not None:
            if len(iv) != IV_LEN:
                raise ValueError("AES-GCM IV must be exactly 12 bytes")
            ctypes.memmove(e.iv, bytes(iv), IV_LEN)
        e.status = 0
        e.reserved = 0
    return bytes(arr)


class GpuAesGcmLibrary:
    """Loads the shared library and declares the C-ABI signatures."""

    def __init__(self, path: str | Path | None = None):
        self.path = Path(path if path is not None else DEFAULT_LIBRARY).resolve()
        if not self.path.exists():
            raise FileNotFoundError(f"GPU AES-GCM library not found: {self.path}")
        self.lib = ctypes.CDLL(str(self.path))
        self._configure_abi()

    def _configure_abi(self) -> None:
        lib = self.lib
        c_size, c_int, c_vp = ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p
        u8p = ctypes.POINTER(ctypes.c_uint8)

        lib.lmcache_gpu_aesgcm_frame_size.argtypes = [c_size]
        lib.lmcache_gpu_aesgcm_frame_size.restype = c_size

        lib.lmcache_gpu_aes128gcm_key_create.argtypes = [u8p, c_size, c_int, ctypes.POINTER(c_vp)]
        lib.lmcache_gpu_aes128gcm_key_create.restype = c_int

        lib.lmcache_gpu_aes128gcm_key_destroy.argtypes = [c_vp]
        lib.lmcache_gpu_aes128gcm_key_destroy.restype = c_int

        lib.lmcache_gpu_aes128gcm_reserve.argtypes = [c_vp, c_size]
        lib.lmcache_gpu_aes128gcm_reserve.restype = c_int

        lib.lmcache_gpu_aes128gcm_seal_async.argtypes = [c_vp, c_vp, c_size, c_vp, c_size, u8p, c_vp]
        lib.lmcache_gpu_aes128gcm_seal_async.restype = c_int

        lib.lmcache_gpu_aes128gcm_open_async.argtypes = [c_vp, c_vp, c_size, c_vp, c_size, c_vp, c_vp]
        lib.lmcache_gpu_aes128gcm_open_async.restype = c_int

        lib.lmcache_gpu_aesgcm_strerror.argtypes = [c_int]
        lib.lmcache_gpu_aesgcm_strerror.restype = ctypes.c_char_p

        lib.lmcache_gpu_aes128gcm_batch_workspace_size.argtypes = [c_size]
        lib.lmcache_gpu_aes128gcm_batch_workspace_size.restype = c_size
        for name in ("lmcache_gpu_aes128gcm_seal_batch_async", "lmcache_gpu_aes128gcm_open_batch_async"):
            fn = getattr(lib, name)
            fn.argtypes = [c_vp, c_vp, c_size, c_vp, c_size, c_vp]
            fn.restype = c_int

    def frame_size(self, plaintext_len: int) -> int:
        if plaintext_len < 0:
            raise ValueError("plaintext_len must be non-negative")
        return int(self.lib.lmcache_gpu_aesgcm_frame_size(plaintext_len))

    def error_string(self, rc: int) -> str:
        p = self.lib.lmcache_gpu_aesgcm_strerror(rc)
        if not p:
            return f"error {rc}"
        return p.decode("utf-8", errors="replace")

    def batch_workspace_size(self, count: int) -> int:
        """Device workspace bytes for a batch of `count` objects (0 = too many)."""
        return int(self.lib.lmcache_gpu_aes128gcm_batch_workspace_size(count))

    def check(self, rc: int, operation: str) -> None:
        if rc == 0:
            return
        raise GpuAesGcmError(f"{operation} failed: rc={rc} ({self.error_string(rc)})")


class GpuAes128GcmKey:
    """Owner of one native AES-128-GCM key handle bound to a CUDA device.

    Device pointers and streams are integer addresses (``tensor.data_ptr()``,
    ``torch.cuda.Stream.cuda_stream``), so the binding itself needs no torch.
    """

    def __init__(self, library: GpuAesGcmLibrary, key: bytes, device: int = 0):
        if len(key) != KEY_LEN:
            raise ValueError("AES-128 key must be exactly 16 bytes")
        self.library = library
        self.device = int(device)
        self._handle = ctypes.c_void_p()
        key_buf = (ctypes.c_uint8 * KEY_LEN).from_buffer_copy(key)
        rc = library.lib.lmcache_gpu_aes128gcm_key_create(
            key_buf, KEY_LEN, self.device, ctypes.byref(self._handle)
        )
        library.check(rc, "key_create")
        if not self._handle.value:
            raise GpuAesGcmError("key_create succeeded but returned NULL handle")

    @property
    def handle(self) -> int:
        if not self._handle.value:
            raise GpuAesGcmError("GPU AES-GCM key has been closed")
        return int(self._handle.value)

    def reserve(self, max_plaintext_len: int) -> None:
        rc = self.library.lib.lmcache_gpu_aes128gcm_reserve(self._handle, max_plaintext_len)
        self.library.check(rc, "reserve")

    def seal_async(
        self,
        *,
        src_ptr: int,
        plaintext_len: int,
        dst_ptr: int,
        dst_capacity: int,
        iv: bytes,
        stream_ptr: int,
    ) -> None:
        if len(iv) != IV_LEN:
            raise ValueError("AES-GCM IV must be exactly 12 bytes")
        iv_buf = (ctypes.c_uint8 * IV_LEN).from_buffer_copy(iv)
        rc = self.library.lib.lmcache_gpu_aes128gcm_seal_async(
            self._handle,
            ctypes.c_void_p(src_ptr),
            plaintext_len,
            ctypes.c_void_p(dst_ptr),
            dst_capacity,
            iv_buf,
            ctypes.c_void_p(stream_ptr),
        )
        self.library.check(rc, "seal_async")

    def open_async(
        self,
        *,
        src_ptr: int,
        frame_len: int,
        dst_ptr: int,
        plaintext_len: int,
        auth_ok_ptr: int,
        stream_ptr: int,
    ) -> None:
        rc = self.library.lib.lmcache_gpu_aes128gcm_open_async(
            self._handle,
            ctypes.c_void_p(src_ptr),
            frame_len,
            ctypes.c_void_p(dst_ptr),
            plaintext_len,
            ctypes.c_void_p(auth_ok_ptr),
            ctypes.c_void_p(stream_ptr),
        )
        self.library.check(rc, "open_async")

    def seal_batch_async(self, *, items_ptr: int, count: int, workspace_ptr: int, workspace_bytes: int,
                         stream_ptr: int) -> None:
        """Enqueue seal of `count` objects described by the device array at
        items_ptr (pack_batch_items layout); per-object status on the device."""
        rc = self.library.lib.lmcache_gpu_aes128gcm_seal_batch_async(
            self._handle, ctypes.c_void_p(items_ptr), count, ctypes.c_void_p(workspace_ptr), workspace_bytes,
            ctypes.c_void_p(stream_ptr))
        self.library.check(rc, "seal_batch_async")

    def open_batch_async(self, *, items_ptr: int, count: int, workspace_ptr: int, workspace_bytes: int,
                         stream_ptr: int) -> None:
        """Enqueue authentication-gated open of `count` frames; each object's
        verdict goes to its auth_ok pointer."""
        rc = self.library.lib.lmcache_gpu_aes128gcm_open_batch_async(
            self._handle, ctypes.c_void_p(items_ptr), count, ctypes.c_void_p(workspace_ptr), workspace_bytes,
            ctypes.c_void_p(stream_ptr))
        self.library.check(rc, "open_batch_async")

    def close(self) -> None:
        if not self._handle.value:
            return
        rc = self.library.lib.lmcache_gpu_aes128gcm_key_destroy(self._handle)
        self._handle = ctypes.c_void_p()
        self.library.check(rc, "key_destroy")

    def __enter__(self) -> "GpuAes128GcmKey":
        return self

    def __exit__(self, exc_type, exc, tb) -> None:
        self.close()

    def __del__(self):
        # Never raise from __del__.
        try:
            if getattr(self, "_handle", None) is not None and self._handle.value:
                self.library.lib.lmcache_gpu_aes128gcm_key_destroy(self._handle)
                self._handle = ctypes.c_void_p()
        except Exception:
            pass
