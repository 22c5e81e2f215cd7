"""Test-only stand-in for lmcache.v1.distributed.api: the two types the
ConfKV serde code uses (experiments/gpu_kv_seal/integration/
native_aesgcm_serde.py:8, scripts/test_native_async_serde.py:140-159)."""

from dataclasses import dataclass, field


@dataclass(frozen=True)
class ObjectKey:
    chunk_hash: bytes
    model_name: str
    kv_rank: int
    cache_salt: str = ""


@dataclass
class MemoryLayoutDesc:
    shapes: list = field(default_factory=list)
    dtypes: list = field(default_factory=list)
