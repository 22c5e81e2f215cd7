"""C-ABI checks that need no GPU: exported symbols, frame size, error strings,
argument validation (which returns before any device access) and the
host-side allocation-failure hook. Ports experiments/gpu_kv_seal/scripts/
test_gpu_abi.py:30-73 and adds the argument-error paths of
gpu_aesgcm.cu:1287-1293,1465-1499,1640-1660."""

import ctypes
import os
import re
from pathlib import Path

import pytest

from confkv_b200.gpu_aesgcm import EXPORTED_SYMBOLS, EXTENSION_SYMBOLS, FRAME_OVERHEAD

HEADER = Path(__file__).resolve().parents[1] / "include" / "gpu_aesgcm_api.h"

OK, ERR_ARG, ERR_ALLOC, ERR_CUDA, ERR_INTERNAL = 0, -1, -2, -3, -4
FAKE_HANDLE = ctypes.c_void_p(0x1000)  # never dereferenced on argument-error paths


def header_functions():
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:size_t|int|const char\*)\s+(lmcache_\w+)\s*\(", text, re.M))


NOALLOC_SYMBOL = "lmcache_gpu_aes128gcm_seal_noalloc"


def test_header_declares_the_reference_abi():
    # the reference's seven entry points plus the extensions (the seal that
    # allocates nothing, batched seal/open)
    assert NOALLOC_SYMBOL in EXTENSION_SYMBOLS
    assert header_functions() == set(EXPORTED_SYMBOLS) | set(EXTENSION_SYMBOLS)


def test_library_exports_every_header_symbol(cpu_lib):
    for name in header_functions():
        assert hasattr(cpu_lib.lib, name), name


@pytest.mark.parametrize("size", [0, 1, 15, 16, 17, 1024, 4 << 20, 18 << 20, 36 << 20, 72 << 20, 1 << 30])
def test_frame_size(cpu_lib, size):
    assert cpu_lib.frame_size(size) == size + FRAME_OVERHEAD


def test_error_strings(cpu_lib):
    assert cpu_lib.error_string(OK) == "success"
    assert cpu_lib.error_string(ERR_ARG) == "invalid argument"
    assert cpu_lib.error_string(ERR_ALLOC) == "GPU allocation failure"
    assert cpu_lib.error_string(ERR_CUDA) == "CUDA failure"
    assert cpu_lib.error_string(ERR_INTERNAL) == "internal error"
    assert cpu_lib.error_string(-99) == "unknown error"


def test_key_create_argument_errors(cpu_lib):
    lib = cpu_lib.lib
    out = ctypes.c_void_p()
    key = (ctypes.c_uint8 * 16)(*range(16))
    assert lib.lmcache_gpu_aes128gcm_key_create(None, 16, 0, ctypes.byref(out)) == ERR_ARG
    assert lib.lmcache_gpu_aes128gcm_key_create(key, 16, 0, None) == ERR_ARG
    for bad_len in (0, 15, 17, 24, 32):
        assert lib.lmcache_gpu_aes128gcm_key_create(key, bad_len, 0, ctypes.byref(out)) == ERR_ARG
    assert out.value is None


def test_key_create_alloc_fault_injection(cpu_lib):
    os.environ["CONFKV_B200_FAIL_ALLOC"] = "1"
    out = ctypes.c_void_p()
    key = (ctypes.c_uint8 * 16)(*range(16))
    assert cpu_lib.lib.lmcache_gpu_aes128gcm_key_create(key, 16, 0, ctypes.byref(out)) == ERR_ALLOC
    assert out.value is None


def test_destroy_and_reserve_null(cpu_lib):
    assert cpu_lib.lib.lmcache_gpu_aes128gcm_key_destroy(None) == OK
    assert cpu_lib.lib.lmcache_gpu_aes128gcm_reserve(None, 1 << 20) == ERR_ARG


def test_seal_argument_errors(cpu_lib):
    lib = cpu_lib.lib
    iv = (ctypes.c_uint8 * 12)()
    p = ctypes.c_void_p(0x2000)
    seal = lib.lmcache_gpu_aes128gcm_seal_async
    assert seal(None, p, 16, p, 45, iv, None) == ERR_ARG
    assert seal(FAKE_HANDLE, None, 16, p, 45, iv, None) == ERR_ARG
    assert seal(FAKE_HANDLE, p, 16, None, 45, iv, None) == ERR_ARG
    assert seal(FAKE_HANDLE, p, 16, p, 45, None, None) == ERR_ARG
    # dst_capacity must hold P + 29
    assert seal(FAKE_HANDLE, p, 16, p, 44, iv, None) == ERR_ARG
    assert seal(FAKE_HANDLE, p, 0, p, 28, iv, None) == ERR_ARG
    # at most 2^32 - 2 counter blocks (gpu_aesgcm.cu:1494-1499)
    big = 16 * 0xFFFFFFFF
    assert seal(FAKE_HANDLE, p, big, p, big + 29, iv, None) == ERR_ARG
    # size_t overflow of P + 29
    assert seal(FAKE_HANDLE, p, (1 << 64) - 1, p, (1 << 64) - 1, iv, None) == ERR_ARG


def test_open_argument_errors(cpu_lib):
    lib = cpu_lib.lib
    p = ctypes.c_void_p(0x2000)
    op = lib.lmcache_gpu_aes128gcm_open_async
    assert op(None, p, 45, p, 16, p, None) == ERR_ARG
    assert op(FAKE_HANDLE, None, 45, p, 16, p, None) == ERR_ARG
    assert op(FAKE_HANDLE, p, 45, None, 16, p, None) == ERR_ARG
    assert op(FAKE_HANDLE, p, 45, p, 16, None, None) == ERR_ARG
    # frame must hold P + 29 bytes (padded frames are fine, short ones are not)
    assert op(FAKE_HANDLE, p, 44, p, 16, p, None) == ERR_ARG
    big = 16 * 0xFFFFFFFF
    assert op(FAKE_HANDLE, p, big + 29, p, big, p, None) == ERR_ARG


def test_seal_noalloc_argument_errors(cpu_lib):
    f = getattr(cpu_lib.lib, NOALLOC_SYMBOL)
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    f.argtypes = [vp, sz, vp, sz, vp, sz, vp, ctypes.c_int, vp]
    f.restype = ctypes.c_int
    key = bytes(16)
    iv = (ctypes.c_uint8 * 12)()
    p = ctypes.c_void_p(0x2000)
    assert f(None, 16, p, 16, p, 45, iv, 0, None) == ERR_ARG
    assert f(key, 15, p, 16, p, 45, iv, 0, None) == ERR_ARG
    assert f(key, 16, None, 16, p, 45, iv, 0, None) == ERR_ARG
    assert f(key, 16, p, 16, None, 45, iv, 0, None) == ERR_ARG
    assert f(key, 16, p, 16, p, 45, None, 0, None) == ERR_ARG
    assert f(key, 16, p, 16, p, 44, iv, 0, None) == ERR_ARG
    assert f(key, 16, p, (1 << 30) + 1, p, (1 << 30) + 30, iv, 0, None) == ERR_ARG
    assert f(key, 16, p, 16, p, 45, iv, -1, None) == ERR_ARG


def test_batch_workspace_size(cpu_lib):
    ws = cpu_lib.batch_workspace_size
    # header 256 B, one 32-B slot per object (rounded to 256 B), a 16-B
    # tile-object record per object plus a sentinel (rounded to 256 B), a
    # 16-B record for each of at most 1024 chunks plus a sentinel, and four
    # small-object list regions (one per size bucket) of a 4-B entry per object
    r256 = lambda x: (x + 255) // 256 * 256
    for count in (1, 7, 8, 9, 4096, 1 << 20):
        assert ws(count) == 256 + r256(count * 32) + r256((count + 1) * 16) + 1025 * 16 + 5 * count * 4
    assert ws((1 << 20) + 1) == 0


def test_batch_argument_errors(cpu_lib):
    lib = cpu_lib.lib
    p = ctypes.c_void_p(0x2000)
    for f in (lib.lmcache_gpu_aes128gcm_seal_batch_async, lib.lmcache_gpu_aes128gcm_open_batch_async):
        need = cpu_lib.batch_workspace_size(4)
        assert f(None, p, 4, p, need, None) == ERR_ARG
        assert f(FAKE_HANDLE, p, 0, None, 0, None) == OK           # empty batch: no-op
        assert f(FAKE_HANDLE, None, 4, p, need, None) == ERR_ARG
        assert f(FAKE_HANDLE, p, 4, None, need, None) == ERR_ARG
        assert f(FAKE_HANDLE, p, 4, p, need - 1, None) == ERR_ARG  # short workspace
        assert f(FAKE_HANDLE, ctypes.c_void_p(0x2008), 4, p, need, None) == ERR_ARG  # items not 16-B aligned
        assert f(FAKE_HANDLE, p, 4, ctypes.c_void_p(0x2004), need, None) == ERR_ARG  # workspace not 16-B aligned
        assert f(FAKE_HANDLE, p, (1 << 20) + 1, p, 1 << 40, None) == ERR_ARG


def test_batch_item_layout():
    from confkv_b200.gpu_aesgcm import BatchItem, pack_batch_items

    assert ctypes.sizeof(BatchItem) == 64
    offs = {name: getattr(BatchItem, name).offset for name, _ in BatchItem._fields_}
    assert offs == {"src": 0, "dst": 8, "plaintext_len": 16, "capacity": 24, "auth_ok": 32, "iv": 40,
                    "status": 52, "reserved": 56}
    raw = pack_batch_items([(1, 2, 3, 32, 0, bytes(range(12))), (5, 6, 7, 36, 0x99, None)])
    assert len(raw) == 128
    assert raw[40:52] == bytes(range(12)) and raw[64 + 32] == 0x99 and raw[64 + 40:64 + 52] == bytes(12)
    with pytest.raises(ValueError):
        pack_batch_items([(1, 2, 3, 32, 0, b"short")])


def test_binding_rejects_bad_lengths(cpu_lib):
    from confkv_b200.gpu_aesgcm import GpuAes128GcmKey

    with pytest.raises(ValueError):
        GpuAes128GcmKey(cpu_lib, b"\x00" * 15)
    with pytest.raises(ValueError):
        cpu_lib.frame_size(-1)


def test_missing_library_fails_loudly(tmp_path):
    from confkv_b200.gpu_aesgcm import GpuAesGcmLibrary

    with pytest.raises(FileNotFoundError):
        GpuAesGcmLibrary(tmp_path / "nope.so")
