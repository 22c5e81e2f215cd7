"""Test-only stand-in for lmcache.v1.distributed.serde.key_provider.

The real HkdfKeyProvider is not available here, so its derivation is not
pinned: this one uses HKDF-SHA256(master, salt=None, info=prefix + cache_salt).
The seal/open path only ever receives the derived 16-byte key."""

from cryptography.hazmat.primitives import hashes
from cryptography.hazmat.primitives.kdf.hkdf import HKDF


class KeyProvider:
    def get_key(self, cache_salt) -> bytes:
        raise NotImplementedError


class HkdfKeyProvider(KeyProvider):
    def __init__(self, master_key: bytes, key_len: int = 16, info_prefix: bytes = b""):
        self._master = bytes(master_key)
        self._len = int(key_len)
        self._prefix = bytes(info_prefix)
        self._cache = {}

    def get_key(self, cache_salt) -> bytes:
        salt = (cache_salt or "").encode() if not isinstance(cache_salt, bytes) else cache_salt
        if salt not in self._cache:
            self._cache[salt] = HKDF(algorithm=hashes.SHA256(), length=self._len, salt=None,
                                     info=self._prefix + b"|" + salt).derive(self._master)
        return self._cache[salt]
