"""The integer-pipe GF(2^128) multiply (confkv_b200/csrc/clmul.cuh) and the
window tables of the batched GHASH passes (confkv_b200/csrc/gh5.cuh with the product's host table
builder), compiled for the host, against the oracle's bit-serial SP 800-38D
multiply (reference gpu_aesgcm.cu:195-248) and GHASH. The GPU kernels compile
the same headers, so these CPU checks cover their arithmetic; the GPU tests
cover the kernels that use them."""

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def clmul(tmp_path_factory):
    so = tmp_path_factory.mktemp("clmul") / "libclmul_check.so"
    subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wextra",
                    "-I", str(ROOT / "confkv_b200" / "csrc"), str(ROOT / "tests" / "native" / "clmul_check.cpp"),
                    "-o", str(so)], check=True)
    lib = ctypes.CDLL(str(so))
    lib.clmul_check_mul.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
    lib.clmul_check_mul.restype = None
    lib.clmul_check_ghash.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p,
                                      ctypes.c_int]
    lib.clmul_check_ghash.restype = None
    return lib


HOLES = [pytest.param(0, id="spacing4"), pytest.param(1, id="spacing5")]


def _mul(lib, a: bytes, m: bytes, h5: int = 0) -> bytes:
    out = ctypes.create_string_buffer(16)
    lib.clmul_check_mul(a, m, out, h5)
    return out.raw


def _edge_blocks():
    one = bytes([0x80]) + bytes(15)            # x^0
    top = bytes(15) + bytes([0x01])            # x^127
    yield bytes(16)
    yield one
    yield top
    yield b"\xff" * 16
    for bit in (1, 7, 8, 31, 32, 63, 64, 95, 96, 120, 121, 126):
        b = bytearray(16)
        b[bit // 8] = 0x80 >> (bit % 8)
        yield bytes(b)


@pytest.mark.parametrize("h5", HOLES)
def test_mul_matches_bit_serial_multiply(clmul, oracle, h5):
    rng = np.random.default_rng(128)
    cases = [(rng.bytes(16), rng.bytes(16)) for _ in range(2000)]
    edges = list(_edge_blocks())
    cases += [(a, m) for a in edges for m in edges]
    cases += [(a, rng.bytes(16)) for a in edges for _ in range(8)]
    for a, m in cases:
        assert _mul(clmul, a, m, h5) == oracle.gf_mul(a, m), (a.hex(), m.hex())


@pytest.mark.parametrize("h5", HOLES)
def test_mul_by_one_is_identity(clmul, h5):
    rng = np.random.default_rng(5)
    one = bytes([0x80]) + bytes(15)
    for _ in range(100):
        a = rng.bytes(16)
        assert _mul(clmul, a, one, h5) == a


@pytest.mark.parametrize("h5", HOLES)
def test_horner_chain_matches_ghash(clmul, oracle, h5):
    rng = np.random.default_rng(9)
    for nblocks in (1, 2, 3, 17, 256):
        h = rng.bytes(16)
        data = rng.bytes(16 * nblocks)
        # the oracle's GHASH ends with the length block [0^64 || 8 len]
        length_block = (0).to_bytes(8, "big") + (8 * len(data)).to_bytes(8, "big")
        out = ctypes.create_string_buffer(16)
        clmul.clmul_check_ghash(h, data + length_block, nblocks + 1, out, h5)
        assert out.raw == oracle.ghash_ct(h, data)


@pytest.fixture(scope="module", params=[5, 6], ids=["window5", "window6"])
def gh5(request, tmp_path_factory):
    so = tmp_path_factory.mktemp("gh5") / f"libgh5_check_w{request.param}.so"
    csrc = ROOT / "confkv_b200" / "csrc"
    subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wextra", "-I", str(csrc),
                    f"-DCONFKV_GH_WINDOW={request.param}", str(ROOT / "tests" / "native" / "gh5_check.cpp"),
                    str(csrc / "host_crypto.cpp"), "-o", str(so)],
                   check=True)
    lib = ctypes.CDLL(str(so))
    lib.gh5_check_mul.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p]
    lib.gh5_check_mul.restype = None
    return lib


def test_window_tables_match_bit_serial_multiply(gh5, oracle):
    rng = np.random.default_rng(55)
    edges = list(_edge_blocks())
    cases = [(rng.bytes(16), rng.bytes(16)) for _ in range(300)]
    cases += [(a, m) for a in edges for m in edges[:6]]
    for x, m in cases:
        out = ctypes.create_string_buffer(16)
        gh5.gh5_check_mul(x, m, out)
        assert out.raw == oracle.gf_mul(x, m), (x.hex(), m.hex())
