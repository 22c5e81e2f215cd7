"""Authentication gating: tampered, wrong-key and wrong-version frames give
auth_ok == 0 and an all-zero dst. Ports experiments/gpu_kv_seal/scripts/
test_gpu_security.py:28-249 (SIZE 4 MiB, IV 00112233445566778899aabb, flips at
ciphertext byte 113, IV byte 1, last tag byte, version = 2, wrong key =
reversed(range(16))) and adds more positions and sizes."""

import numpy as np
import pytest
from cryptography.hazmat.primitives.ciphers.aead import AESGCM

from gpu_helpers import GpuKey

pytestmark = pytest.mark.gpu

KEY = bytes(range(16))
WRONG_KEY = bytes(reversed(range(16)))
SIZE = 4 * 1024 * 1024
IV = bytes.fromhex("00112233445566778899aabb")


@pytest.fixture(scope="module")
def plain():
    return bytes(range(256)) * (SIZE // 256)


@pytest.fixture(scope="module")
def good_frame(plain):
    return b"\x01" + IV + AESGCM(KEY).encrypt(IV, plain, None)


@pytest.fixture(scope="module")
def gkey(gpu_lib):
    k = GpuKey(gpu_lib, KEY)
    k.key.reserve(SIZE)
    yield k
    k.close()


def tampered(frame: bytes, pos: int, value=None) -> bytes:
    x = bytearray(frame)
    if value is None:
        x[pos] ^= 0x01
    else:
        x[pos] = value
    return bytes(x)


def test_valid_frame(gkey, good_frame, plain):
    assert gkey.open(good_frame, SIZE) == (1, plain)


@pytest.mark.parametrize("name,pos,value", [
    ("ciphertext", 13 + 100, None),
    ("iv", 1, None),
    ("tag", -1, None),
    ("version", 0, 2),
    ("ciphertext_first", 13, None),
    ("ciphertext_last", 13 + SIZE - 1, None),
    ("tag_first", 13 + SIZE, None),
    ("iv_last", 12, None),
])
def test_tamper_rejected_and_zeroised(gkey, good_frame, name, pos, value):
    pos = pos if pos >= 0 else len(good_frame) + pos
    auth, out = gkey.open(tampered(good_frame, pos, value), SIZE)
    assert auth == 0, name
    assert out == bytes(SIZE), name


def test_wrong_key_rejected_and_zeroised(gpu_lib, good_frame):
    wrong = GpuKey(gpu_lib, WRONG_KEY)
    try:
        auth, out = wrong.open(good_frame, SIZE)
        assert auth == 0
        assert out == bytes(SIZE)
    finally:
        wrong.close()


@pytest.mark.parametrize("size", [0, 1, 15, 16, 17, 333, 65536 + 3])
def test_small_sizes_tamper(gkey, oracle, size):
    rng = np.random.default_rng(size + 1)
    pt, iv = rng.bytes(size), rng.bytes(12)
    frame = oracle.seal(KEY, iv, pt)
    assert gkey.open(frame, size) == (1, pt)
    for pos in sorted({0, 1, 12, 13, 13 + size // 2, len(frame) - 16, len(frame) - 1}):
        if pos == 13 + size // 2 and size == 0:
            continue
        auth, out = gkey.open(tampered(frame, pos), size)
        assert auth == 0 and out == bytes(size), (size, pos)


def test_gpu_sealed_frame_rejected_after_tamper(gkey, oracle, plain):
    frame = bytearray(gkey.seal(plain, IV))
    frame[13 + SIZE // 2] ^= 0x80
    rc, out = oracle.open(KEY, bytes(frame), SIZE)
    assert rc == 0
    auth, out = gkey.open(bytes(frame), SIZE)
    assert auth == 0 and out == bytes(SIZE)
