"""Test-only stand-in for lmcache.v1.distributed.serde.base: abstract
Serializer / Deserializer / SerdeProcessor and SerdeConfig as used by
native_aesgcm_serde.py:104-292 and test_backend_switch.py:44-53."""

from dataclasses import dataclass, field


class Serializer:
    def serialize(self, src, dst, key) -> int:
        raise NotImplementedError

    def estimate_serialized_size(self, layout_desc) -> int:
        raise NotImplementedError


class Deserializer:
    def deserialize(self, src, dst, key) -> None:
        raise NotImplementedError


class SerdeProcessor:
    def estimate_serialized_size(self, layout_desc) -> int:
        raise NotImplementedError

    def close(self) -> None:
        pass


@dataclass
class SerdeConfig:
    type: str
    kwargs: dict = field(default_factory=dict)
