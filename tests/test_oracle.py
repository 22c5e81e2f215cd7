"""Pin the CPU oracle: golden frames, pyca cryptography, the EVP injected-IV
shim and the reference's own OpenSSL backend (oracle/_ref/libcpu_seal.so)."""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
from cryptography.hazmat.primitives.ciphers.aead import AESGCM

from confkv_b200 import workloads

GOLDEN = json.loads((Path(__file__).parent / "golden" / "golden_frames.json").read_text())


def pattern(size: int) -> bytes:
    return (bytes(range(256)) * ((size + 255) // 256))[:size]


def test_oracle_small_golden(oracle):
    for v in GOLDEN["small"]:
        key, iv, pt = bytes.fromhex(v["key"]), bytes.fromhex(v["iv"]), bytes.fromhex(v["pt"])
        frame = bytes.fromhex(v["frame"])
        assert oracle.seal(key, iv, pt) == frame
        assert oracle.open(key, frame, len(pt)) == (1, pt)
        assert oracle.evp_seal(key, iv, np.frombuffer(pt, np.uint8)).tobytes() == frame


def test_oracle_reference_interop_golden(oracle):
    key = bytes(range(16))
    for v in GOLDEN["reference_interop"]:
        size = v["size"]
        iv = bytes.fromhex(v["iv"])
        assert iv == size.to_bytes(12, "big")
        assert oracle.seal(key, iv, pattern(size)) == bytes.fromhex(v["frame"])


def test_oracle_digests_4mib(oracle):
    for d in GOLDEN["digests"]:
        if not d["name"].startswith("ref_"):
            continue
        key, iv = bytes.fromhex(d["key"]), bytes.fromhex(d["iv"])
        pt = pattern(d["plen"])
        assert hashlib.sha256(pt).hexdigest() == d["pt_sha256"]
        assert hashlib.sha256(oracle.seal(key, iv, pt)).hexdigest() == d["frame_sha256"]


def test_kv_small_digests_evp(oracle):
    import torch

    shape = workloads.SHAPES["kv_small"]
    key = workloads.make_key(1)
    ivs = workloads.make_ivs(1, 64)
    objs = workloads.bf16_objects(shape, 64, seed=1)
    digests = {d["name"]: d for d in GOLDEN["digests"]}
    for k, (iv, t) in enumerate(zip(ivs, objs)):
        d = digests[f"kv_small_{k}"]
        pt = t.view(torch.uint8).numpy().reshape(-1)
        assert hashlib.sha256(pt.tobytes()).hexdigest() == d["pt_sha256"]
        fr = oracle.evp_seal(key, iv, pt)
        assert hashlib.sha256(fr.tobytes()).hexdigest() == d["frame_sha256"]


@pytest.mark.parametrize("size", [0, 1, 7, 15, 16, 17, 100, 1023, 4096, 65536 + 5])
def test_oracle_vs_pyca_random(oracle, size):
    rng = np.random.default_rng(size)
    key, iv, pt = rng.bytes(16), rng.bytes(12), rng.bytes(size)
    expected = b"\x01" + iv + AESGCM(key).encrypt(iv, pt, None)
    assert oracle.seal(key, iv, pt) == expected


def test_oracle_gf_and_aes_consistency(oracle):
    """GHASH over ciphertext and E_K(J0) reproduce the tag of a pyca frame."""
    rng = np.random.default_rng(5)
    key, iv, pt = rng.bytes(16), rng.bytes(12), rng.bytes(333)
    frame = b"\x01" + iv + AESGCM(key).encrypt(iv, pt, None)
    h = oracle.aes_block(key, bytes(16))
    s = oracle.ghash_ct(h, frame[13:-16])
    ej0 = oracle.aes_block(key, iv + b"\x00\x00\x00\x01")
    assert bytes(a ^ b for a, b in zip(s, ej0)) == frame[-16:]
    one = b"\x80" + bytes(15)
    assert oracle.gf_mul(h, one) == h
    assert oracle.gf_mul(one, h) == h


@pytest.mark.parametrize("field", ["version", "iv", "ct_first", "ct_mid", "ct_last", "tag_first", "tag_last"])
def test_oracle_rejects_tamper_and_zeroises(oracle, field):
    rng = np.random.default_rng(11)
    key, iv, pt = rng.bytes(16), rng.bytes(12), rng.bytes(4096 + 7)
    frame = bytearray(oracle.seal(key, iv, pt))
    pos = {"version": 0, "iv": 5, "ct_first": 13, "ct_mid": 13 + 2048, "ct_last": 13 + len(pt) - 1,
           "tag_first": 13 + len(pt), "tag_last": len(frame) - 1}[field]
    frame[pos] ^= 0x01 if field != "version" else 0x03
    rc, out = oracle.open(key, bytes(frame), len(pt))
    assert rc == 0
    assert out == bytes(len(pt))


def test_oracle_wrong_key_and_padded_frame(oracle):
    key = bytes(range(16))
    wrong = bytes(reversed(range(16)))
    pt = pattern(1000)
    frame = oracle.seal(key, bytes(12), pt)
    assert oracle.open(wrong, frame, len(pt)) == (0, bytes(len(pt)))
    # padded frames are accepted; the tag is read at 13 + P
    assert oracle.open(key, frame + b"\xee" * 37, len(pt)) == (1, pt)


def test_reference_backend_cross(oracle):
    if oracle.ref is None:
        pytest.skip("oracle/_ref/libcpu_seal.so not built (reference tree absent)")
    rng = np.random.default_rng(9)
    for size in (1, 15, 16, 17, 4096, (2 << 20) + 7):
        key = rng.bytes(16)
        pt = rng.integers(0, 256, size=size, dtype=np.uint8)
        # reference seal (random IV) -> oracle open
        fr = oracle.ref_seal(key, pt)
        assert oracle.open(key, fr.tobytes(), size) == (1, pt.tobytes())
        # oracle seal -> reference open
        iv = rng.bytes(12)
        fr2 = np.frombuffer(oracle.seal(key, iv, pt.tobytes()) if size < 100000
                            else oracle.evp_seal(key, iv, pt).tobytes(), np.uint8).copy()
        rc, out = oracle.ref_open(key, fr2)
        assert rc == 0 and out.tobytes() == pt.tobytes()
        fr2[13 + size // 2] ^= 1
        rc, out = oracle.ref_open(key, fr2)
        assert rc == -11 and not out.any()
