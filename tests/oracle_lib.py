"""ctypes wrappers for the CPU checkers under oracle/ (test infrastructure).

* ``oracle/liboracle_aesgcm.so``: plain-C AES-128-GCM restatement
  (``oracle_gcm_seal`` / ``oracle_gcm_open``) and the OpenSSL EVP seal with an
  injected IV (``oracle_evp_seal_iv``).
* ``oracle/_ref/libcpu_seal.so``: the reference's own OpenSSL backend
  (``lmcache_aes128gcm_seal`` draws a random IV; ``lmcache_aes128gcm_open``
  returns -11 and cleanses dst on authentication failure).

Large inputs go through the EVP functions (AES-NI); the plain-C restatement
is used where sizes keep it to seconds.
"""

from __future__ import annotations

import ctypes
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
ORACLE_DIR = ROOT / "oracle"
ORACLE_SO = ORACLE_DIR / "liboracle_aesgcm.so"
REF_SO = ORACLE_DIR / "_ref" / "libcpu_seal.so"


def _ptr(buf) -> int:
    if isinstance(buf, np.ndarray):
        return buf.ctypes.data
    if isinstance(buf, (bytes, bytearray, memoryview)):
        arr = np.frombuffer(buf, dtype=np.uint8)
        return arr.ctypes.data
    raise TypeError(type(buf))


class Oracle:
    _inst: "Oracle | None" = None

    def __init__(self):
        if not ORACLE_SO.exists():
            subprocess.run(["make", "-C", str(ORACLE_DIR), "oracle"], check=True, capture_output=True)
        o = ctypes.CDLL(str(ORACLE_SO))
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        o.oracle_gcm_seal.argtypes = [vp, vp, vp, sz, vp, sz]
        o.oracle_gcm_seal.restype = ctypes.c_int
        o.oracle_gcm_open.argtypes = [vp, vp, sz, vp, sz]
        o.oracle_gcm_open.restype = ctypes.c_int
        o.oracle_evp_seal_iv.argtypes = [vp, vp, vp, sz, vp, sz]
        o.oracle_evp_seal_iv.restype = ctypes.c_int
        o.oracle_gf128_mul.argtypes = [vp, vp, vp]
        o.oracle_gf128_mul.restype = None
        o.oracle_ghash_ct.argtypes = [vp, vp, sz, vp]
        o.oracle_ghash_ct.restype = None
        o.oracle_aes128_encrypt.argtypes = [vp, vp, vp]
        o.oracle_aes128_encrypt.restype = None
        o.oracle_sbox.argtypes = [ctypes.c_uint8]
        o.oracle_sbox.restype = ctypes.c_uint8
        self.o = o
        self.ref = None
        if REF_SO.exists():
            r = ctypes.CDLL(str(REF_SO))
            r.lmcache_aes128gcm_seal.argtypes = [vp, vp, sz, vp, sz]
            r.lmcache_aes128gcm_seal.restype = ctypes.c_int
            r.lmcache_aes128gcm_open.argtypes = [vp, vp, sz, vp, sz]
            r.lmcache_aes128gcm_open.restype = ctypes.c_int
            self.ref = r

    @classmethod
    def load(cls) -> "Oracle":
        if cls._inst is None:
            cls._inst = cls()
        return cls._inst

    # ---- plain-C restatement
    def seal(self, key: bytes, iv: bytes, pt) -> bytes:
        pt = np.frombuffer(bytes(pt), dtype=np.uint8) if not isinstance(pt, np.ndarray) else pt
        out = np.empty(pt.size + 29, dtype=np.uint8)
        rc = self.o.oracle_gcm_seal(key, iv, _ptr(pt) if pt.size else None, pt.size, out.ctypes.data, out.size)
        assert rc == 0, rc
        return out.tobytes()

    def open(self, key: bytes, frame: bytes, plen: int) -> tuple[int, bytes]:
        fr = np.frombuffer(frame, dtype=np.uint8)
        out = np.full(max(plen, 1), 0xCC, dtype=np.uint8)
        rc = self.o.oracle_gcm_open(key, fr.ctypes.data, fr.size, out.ctypes.data, plen)
        return rc, out[:plen].tobytes()

    def gf_mul(self, a: bytes, b: bytes) -> bytes:
        out = ctypes.create_string_buffer(16)
        self.o.oracle_gf128_mul(a, b, out)
        return out.raw

    def ghash_ct(self, h: bytes, data: bytes) -> bytes:
        out = ctypes.create_string_buffer(16)
        d = np.frombuffer(data, dtype=np.uint8)
        self.o.oracle_ghash_ct(h, d.ctypes.data if d.size else None, d.size, out)
        return out.raw

    def aes_block(self, key: bytes, block: bytes) -> bytes:
        out = ctypes.create_string_buffer(16)
        self.o.oracle_aes128_encrypt(key, block, out)
        return out.raw

    # ---- OpenSSL EVP with injected IV (fast; same EVP sequence as the reference)
    def evp_seal(self, key: bytes, iv: bytes, pt: np.ndarray) -> np.ndarray:
        pt = np.ascontiguousarray(pt).view(np.uint8).reshape(-1)
        out = np.empty(pt.size + 29, dtype=np.uint8)
        rc = self.o.oracle_evp_seal_iv(key, iv, pt.ctypes.data if pt.size else None, pt.size, out.ctypes.data, out.size)
        assert rc == 0, rc
        return out

    def evp_seal_many(self, key: bytes, ivs, pts, threads: int = 8) -> list[np.ndarray]:
        with ThreadPoolExecutor(threads) as ex:
            return list(ex.map(lambda a: self.evp_seal(key, a[0], a[1]), zip(ivs, pts)))

    # ---- the reference's own backend
    def ref_open(self, key: bytes, frame: np.ndarray) -> tuple[int, np.ndarray]:
        assert self.ref is not None, "oracle/_ref/libcpu_seal.so not built"
        fr = np.ascontiguousarray(frame).view(np.uint8).reshape(-1)
        plen = fr.size - 29
        out = np.full(max(plen, 1), 0xCC, dtype=np.uint8)
        rc = self.ref.lmcache_aes128gcm_open(key, fr.ctypes.data, fr.size, out.ctypes.data, out.size)
        return rc, out[:plen]

    def ref_seal(self, key: bytes, pt: np.ndarray) -> np.ndarray:
        assert self.ref is not None, "oracle/_ref/libcpu_seal.so not built"
        pt = np.ascontiguousarray(pt).view(np.uint8).reshape(-1)
        out = np.empty(pt.size + 29, dtype=np.uint8)
        rc = self.ref.lmcache_aes128gcm_seal(key, pt.ctypes.data, pt.size, out.ctypes.data, out.size)
        assert rc == 0, rc
        return out
