"""Test-only stand-in for lmcache.v1.distributed.serde.factory: a name ->
factory registry (native_aesgcm_serde.py:295-298,
test_native_async_serde.py:115-138)."""

_FACTORIES = {}


def register_serde_factory(name, fn):
    _FACTORIES[name] = fn


def get_registered_serde_types():
    _ensure_builtin()
    return sorted(_FACTORIES)


def create_serde_processor(config):
    _ensure_builtin()
    if config.type not in _FACTORIES:
        raise ValueError(f"unknown serde type {config.type!r}")
    return _FACTORIES[config.type](dict(config.kwargs))


def _ensure_builtin():
    from . import aesgcm  # noqa: F401  (registers "aesgcm")
