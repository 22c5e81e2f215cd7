"""Generate the committed golden AES-128-GCM frames (tests/golden/*.json).

Expected frames come from pyca ``cryptography``'s ``AESGCM(key).encrypt(iv,
pt, None)`` framed as ``b"\\x01" + iv + ct_tag`` -- the exact call of stock
LMCache's serializer and of the reference's GPU interop test
(experiments/gpu_kv_seal/scripts/test_gpu_interop.py:95-107). The script also
checks every frame with the reference's own OpenSSL backend
(oracle/_ref/libcpu_seal.so, lmcache_aes128gcm_open) when it is built.

Run from the repo root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
from cryptography import __version__ as crypto_version
from cryptography.hazmat.primitives.ciphers.aead import AESGCM

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from confkv_b200 import workloads  # noqa: E402


def frame_of(key: bytes, iv: bytes, pt: bytes) -> bytes:
    return b"\x01" + iv + AESGCM(key).encrypt(iv, pt, None)


def pattern(size: int) -> bytes:
    return (bytes(range(256)) * ((size + 255) // 256))[:size]


def ref_check(frame: bytes, key: bytes, pt: bytes) -> bool:
    so = ROOT / "oracle" / "_ref" / "libcpu_seal.so"
    if not so.exists() or len(pt) == 0:
        return True
    lib = ctypes.CDLL(str(so))
    out = ctypes.create_string_buffer(len(pt))
    rc = lib.lmcache_aes128gcm_open(key, frame, ctypes.c_size_t(len(frame)), out, ctypes.c_size_t(len(pt)))
    return rc == 0 and out.raw == pt


def main() -> None:
    doc = {
        "generator": "pyca cryptography AESGCM(key).encrypt(iv, pt, None), framed 0x01|iv|ct|tag",
        "cryptography_version": crypto_version,
        "small": [],
        "reference_interop": [],
        "digests": [],
    }

    # 1. Seeded small vectors with full bytes: every length 0..64, ragged sizes.
    rng = np.random.default_rng(20261201)
    for size in list(range(0, 65)) + [127, 128, 129, 255, 256, 257, 1000, 4096 + 13]:
        key, iv, pt = rng.bytes(16), rng.bytes(12), rng.bytes(size)
        fr = frame_of(key, iv, pt)
        assert ref_check(fr, key, pt)
        doc["small"].append({"key": key.hex(), "iv": iv.hex(), "pt": pt.hex(), "frame": fr.hex()})

    # 2. The reference GPU interop test's inputs: KEY = 0..15, pattern
    #    plaintext, IV = size as 12 big-endian bytes (test_gpu_interop.py:28-107).
    key = bytes(range(16))
    for size in (1, 15, 16, 17, 31, 32, 33, 4096):
        iv = size.to_bytes(12, "big")
        fr = frame_of(key, iv, pattern(size))
        assert ref_check(fr, key, pattern(size))
        doc["reference_interop"].append({"size": size, "iv": iv.hex(), "frame": fr.hex()})

    # 3. Digests of larger frames.
    def add_digest(name, key, iv, pt):
        fr = frame_of(key, iv, pt)
        assert ref_check(fr, key, pt)
        doc["digests"].append(
            {"name": name, "key": key.hex(), "iv": iv.hex(), "plen": len(pt),
             "pt_sha256": hashlib.sha256(pt).hexdigest(), "frame_sha256": hashlib.sha256(fr).hexdigest()}
        )

    add_digest("ref_interop_4MiB", key, (4 << 20).to_bytes(12, "big"), pattern(4 << 20))
    add_digest("ref_security_4MiB", key, bytes.fromhex("00112233445566778899aabb"), pattern(4 << 20))

    # 4. kv_small objects (64 x 2 MiB bf16 N(0,1)), seeds as in tests and bench.
    shape = workloads.SHAPES["kv_small"]
    kkey = workloads.make_key(1)
    ivs = workloads.make_ivs(1, 64)
    objs = workloads.bf16_objects(shape, 64, seed=1)
    for k, (iv, t) in enumerate(zip(ivs, objs)):
        pt = t.view(__import__("torch").uint8).numpy().tobytes()
        add_digest(f"kv_small_{k}", kkey, iv, pt)

    out = HERE / "golden_frames.json"
    out.write_text(json.dumps(doc, indent=1) + "\n")
    print(f"wrote {out} ({out.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
