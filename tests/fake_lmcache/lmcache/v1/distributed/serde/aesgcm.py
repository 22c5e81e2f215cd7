"""Test-only stand-in for ConfKV's lmcache.v1.distributed.serde.aesgcm.

Reproduces, from the call sites in experiments/gpu_kv_seal/, the "aesgcm"
serde type and its backend switch LMCACHE_AESGCM_BACKEND
(scripts/test_backend_switch.py:41-53, MODIFICATIONS.md:9-20):

* stock  - pyca AESGCM, os.urandom IV, AAD None, frame 0x01|iv|ct|tag
           (scripts/bench_seal_worker.py:101-149)
* native - the reference's OpenSSL backend lmcache_aes128gcm_seal/open
           (integration/native_aesgcm_serde.py), library from
           LMCACHE_AESGCM_NATIVE_LIB or oracle/_ref/libcpu_seal.so
* gpu    - the B200 engine (confkv_b200.serde); the fork's real aesgcm.py
           gains the same branch.
"""

import ctypes
import os
from pathlib import Path

from cryptography.exceptions import InvalidTag
from cryptography.hazmat.primitives.ciphers.aead import AESGCM

from .async_processor import AsyncSerdeProcessor
from .base import Deserializer, Serializer
from .factory import register_serde_factory
from .key_provider import HkdfKeyProvider

FRAME_OVERHEAD = 29
HKDF_INFO_PREFIX = b"lmcache-l2-aesgcm-v1"


def _view(obj):
    return memoryview(obj.byte_array).cast("B")


def plaintext_bytes(layout_desc) -> int:
    import torch

    total = 0
    for shape, dtype in zip(layout_desc.shapes, layout_desc.dtypes, strict=True):
        n = 1
        for d in shape:
            n *= int(d)
        total += n * torch.empty((), dtype=dtype).element_size()
    return total


class AesGcmSerializer(Serializer):
    def __init__(self, key_provider):
        self._keys = key_provider

    def serialize(self, src, dst, key) -> int:
        dek = self._keys.get_key(key.cache_salt)
        iv = os.urandom(12)
        plain = bytes(src.byte_array)
        ct = AESGCM(dek).encrypt(iv, plain, None)
        out = _view(dst)
        out[0:1] = b"\x01"
        out[1:13] = iv
        out[13:13 + len(ct)] = ct
        return 13 + len(ct)

    def estimate_serialized_size(self, layout_desc) -> int:
        return plaintext_bytes(layout_desc) + FRAME_OVERHEAD


class AesGcmDeserializer(Deserializer):
    def __init__(self, key_provider):
        self._keys = key_provider

    def deserialize(self, src, dst, key) -> None:
        frame = _view(src)
        out = _view(dst)
        n = len(out)
        if len(frame) < n + FRAME_OVERHEAD or frame[0] != 1:
            raise InvalidTag("malformed frame")
        dek = self._keys.get_key(key.cache_salt)
        try:
            plain = AESGCM(dek).decrypt(bytes(frame[1:13]), bytes(frame[13:13 + n + 16]), None)
        except InvalidTag:
            out[:] = bytes(n)
            raise
        out[:] = plain


def _native_lib():
    path = os.environ.get("LMCACHE_AESGCM_NATIVE_LIB") or str(
        Path(__file__).resolve().parents[6] / "oracle" / "_ref" / "libcpu_seal.so")
    lib = ctypes.CDLL(path)
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    for name in ("lmcache_aes128gcm_seal", "lmcache_aes128gcm_open"):
        fn = getattr(lib, name)
        fn.argtypes = [vp, vp, sz, vp, sz]
        fn.restype = ctypes.c_int
    return lib


def _addr(view):
    return ctypes.addressof(ctypes.c_ubyte.from_buffer(view))


class NativeAesGcmSerializer(AesGcmSerializer):
    def serialize(self, src, dst, key) -> int:
        s, d = _view(src), _view(dst)
        dek = self._keys.get_key(key.cache_salt)
        rc = _native_lib().lmcache_aes128gcm_seal(dek, _addr(s), len(s), _addr(d), len(d))
        if rc != 0:
            raise RuntimeError(f"native aesgcm seal failed: rc={rc}")
        return len(s) + FRAME_OVERHEAD


class NativeAesGcmDeserializer(AesGcmDeserializer):
    def deserialize(self, src, dst, key) -> None:
        s, d = _view(src), _view(dst)
        dek = self._keys.get_key(key.cache_salt)
        rc = _native_lib().lmcache_aes128gcm_open(dek, _addr(s), len(d) + FRAME_OVERHEAD, _addr(d), len(d))
        if rc == -11:
            raise InvalidTag("native aesgcm authentication failed")
        if rc != 0:
            raise ValueError(f"native aesgcm open failed: rc={rc}")


def backend_name() -> str:
    name = os.environ.get("LMCACHE_AESGCM_BACKEND", "stock").strip().lower()
    if name not in ("stock", "native", "gpu"):
        raise ValueError(f"unknown LMCACHE_AESGCM_BACKEND {name!r}")
    return name


def create_aesgcm_serde(kwargs):
    backend = backend_name()
    if backend == "gpu":
        from confkv_b200.serde import create_gpu_aesgcm_serde

        return create_gpu_aesgcm_serde(kwargs)
    if int(kwargs.get("aes_bits", 128)) != 128:
        raise ValueError("aes_bits=128 only")
    path = str(kwargs.get("master_key_path", ""))
    if not path:
        raise ValueError("aesgcm requires master_key_path")
    with open(path, "rb") as f:
        provider = HkdfKeyProvider(f.read(), key_len=16, info_prefix=HKDF_INFO_PREFIX)
    if backend == "native":
        ser, de = NativeAesGcmSerializer(provider), NativeAesGcmDeserializer(provider)
    else:
        ser, de = AesGcmSerializer(provider), AesGcmDeserializer(provider)
    return AsyncSerdeProcessor(ser, de, max_workers=int(kwargs.get("max_workers", 1)))


register_serde_factory("aesgcm", create_aesgcm_serde)
