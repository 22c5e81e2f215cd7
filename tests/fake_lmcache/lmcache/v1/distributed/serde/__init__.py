"""Test-only stand-in for lmcache.v1.distributed.serde."""
