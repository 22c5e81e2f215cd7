"""GPU seal <-> CPU open and CPU seal -> GPU open, bit-exact.

Ports experiments/gpu_kv_seal/scripts/test_gpu_interop.py:28-230 (KEY = 0..15,
pattern plaintext, IV = size as 12 big-endian bytes, expected frame from pyca
AESGCM, output pre-filled with 0xCC) and extends it to every length 0..64,
the committed golden frames, P = 0, and every destination / source alignment.
"""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
from cryptography.hazmat.primitives.ciphers.aead import AESGCM

from gpu_helpers import GpuKey

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).parent / "golden" / "golden_frames.json").read_text())
KEY = bytes(range(16))


def pattern(size: int) -> bytes:
    return (bytes(range(256)) * ((size + 255) // 256))[:size]


@pytest.fixture(scope="module")
def gkey(gpu_lib):
    k = GpuKey(gpu_lib, KEY)
    k.key.reserve(4 << 20)
    yield k
    k.close()


@pytest.mark.parametrize("size", [0, 1, 15, 16, 17, 31, 32, 33, 4096, 4 << 20])
def test_reference_interop_sizes(gkey, size):
    plain = pattern(size)
    iv = size.to_bytes(12, "big")
    expected = b"\x01" + iv + AESGCM(KEY).encrypt(iv, plain, None)
    frame = gkey.seal(plain, iv)
    assert frame == expected, f"GPU frame mismatch at size={size}"
    assert AESGCM(KEY).decrypt(frame[1:13], frame[13:], None) == plain
    auth, out = gkey.open(expected, size)
    assert auth == 1
    assert out == plain


def test_reference_interop_golden(gkey):
    for v in GOLDEN["reference_interop"]:
        size = v["size"]
        assert gkey.seal(pattern(size), bytes.fromhex(v["iv"])) == bytes.fromhex(v["frame"])
    for d in GOLDEN["digests"]:
        if d["name"] == "ref_interop_4MiB":
            fr = gkey.seal(pattern(d["plen"]), bytes.fromhex(d["iv"]))
            assert hashlib.sha256(fr).hexdigest() == d["frame_sha256"]


def test_golden_small_vectors_seal_and_open(gpu_lib):
    for v in GOLDEN["small"]:
        key, iv, pt = bytes.fromhex(v["key"]), bytes.fromhex(v["iv"]), bytes.fromhex(v["pt"])
        frame = bytes.fromhex(v["frame"])
        k = GpuKey(gpu_lib, key)
        try:
            assert k.seal(pt, iv) == frame, len(pt)
            assert k.open(frame, len(pt)) == (1, pt), len(pt)
        finally:
            k.close()


@pytest.mark.parametrize("dst_off", range(16))
def test_every_frame_alignment(gkey, oracle, dst_off):
    rng = np.random.default_rng(dst_off)
    for size in (1, 13, 16, 29, 100, 511, 512, 513, 8192 + 3, 100000):
        pt = rng.bytes(size)
        iv = rng.bytes(12)
        expected = oracle.seal(KEY, iv, pt)
        assert gkey.seal(pt, iv, dst_off=dst_off) == expected, (size, dst_off)
        assert gkey.open(expected, size, frame_off=dst_off) == (1, pt), (size, dst_off)


@pytest.mark.parametrize("src_off", [1, 3, 8, 15])
def test_unaligned_plaintext_buffers(gkey, oracle, src_off):
    rng = np.random.default_rng(100 + src_off)
    for size in (5, 64, 1000, 70001):
        pt, iv = rng.bytes(size), rng.bytes(12)
        expected = oracle.seal(KEY, iv, pt)
        assert gkey.seal(pt, iv, src_off=src_off, dst_off=(src_off * 7) % 16) == expected
        assert gkey.open(expected, size, dst_off=src_off) == (1, pt)


def test_padded_frames_open(gkey, oracle):
    pt = pattern(5000)
    frame = oracle.seal(KEY, bytes(12), pt)
    for pad in (1, 16, 333):
        assert gkey.open(frame, len(pt), pad=pad) == (1, pt)


@pytest.mark.parametrize("size", [16 * 256 * 148 - 1, 16 * 256 * 148, 16 * 256 * 148 + 1,
                                  (2 << 20) + 7, (32 << 20) + 13])
def test_grid_boundaries(gkey, oracle, size):
    rng = np.random.default_rng(size)
    pt = rng.integers(0, 256, size=size, dtype=np.uint8)
    iv = rng.bytes(12)
    expected = oracle.evp_seal(KEY, iv, pt).tobytes()
    frame = gkey.seal(pt, iv, dst_off=size % 16)
    assert frame == expected
    assert gkey.open(expected, size) == (1, pt.tobytes())


# Per-object open switches its GHASH kernel at 48 MiB (kOpenWindowMinBytes:
# two 4-bit table chains below, the window-table / integer-pipe split from
# there on); both sides of the switch, every ciphertext alignment class and
# the gating on a corrupted frame.
@pytest.mark.parametrize("size,frame_off", [((48 << 20) - 1, 0), (48 << 20, 0), ((48 << 20) + 3, 5),
                                            ((64 << 20) + 13, 3), ((96 << 20) + 5, 8), ((64 << 20) + 16, 1)])
def test_large_object_open_both_ghash_designs(gkey, oracle, size, frame_off):
    rng = np.random.default_rng(size + frame_off)
    pt = rng.integers(0, 256, size=size, dtype=np.uint8)
    iv = rng.bytes(12)
    expected = oracle.evp_seal(KEY, iv, pt).tobytes()
    assert gkey.open(expected, size, frame_off=frame_off) == (1, pt.tobytes())
    if frame_off == 0:
        assert gkey.seal(pt, iv, dst_off=3) == expected
    zeros = bytes(size)
    for pos in (13 + size // 2, 13 + size - 1, 13 + size + 15):   # ciphertext middle, last byte, tag
        bad = bytearray(expected)
        bad[pos] ^= 0x10
        assert gkey.open(bytes(bad), size, frame_off=frame_off) == (0, zeros)


# Per-object seal switches to two passes (CTR kernel, then the window-table
# GHASH kernel writing the tag) at 80 MiB (kSealTwoPassMinBytes): both sides,
# every ciphertext store class (dst offset 0, 1, 3, 7, 11, 15 -> frame + 13
# at 13, 14, 0, 4, 8, 12 mod 16) and a misaligned plaintext.
@pytest.mark.parametrize("size,src_off,dst_off", [((80 << 20) - 3, 0, 0), (80 << 20, 0, 3), ((80 << 20) + 1, 5, 0),
                                                  ((96 << 20) + 13, 0, 1), ((96 << 20) + 7, 0, 7),
                                                  ((96 << 20) + 16, 9, 11), ((112 << 20) + 5, 0, 15)])
def test_large_object_seal_both_designs(gkey, oracle, size, src_off, dst_off):
    rng = np.random.default_rng(size * 7 + dst_off)
    pt = rng.integers(0, 256, size=size, dtype=np.uint8)
    iv = rng.bytes(12)
    expected = oracle.evp_seal(KEY, iv, pt).tobytes()
    assert gkey.seal(pt, iv, src_off=src_off, dst_off=dst_off) == expected
