"""Test-only stand-in for the LMCache package (the real one is not vendored here)."""
