"""Parity on the benchmarked workloads, through the C-ABI.

* kv_small: 64 x 2 MiB bf16 KV objects -> frames byte-identical to the
  committed golden digests (pyca / stock-LMCache frames).
* kv_llama8b: 32 x 32 MiB objects -> frames identical to OpenSSL EVP frames,
  reference lmcache_aes128gcm_open accepts them, GPU open round-trips.
* ragged: 4096 objects, 4 KiB..1 MiB with 1-15 byte remainders; 1% tampered
  (IV / ciphertext / tag bit) and 1% opened with a wrong key must give
  auth_ok = 0 and a zeroed output, the rest round-trip bit-exactly.
* sweep: single objects 4 KiB .. 1 GiB (powers of two), frames vs OpenSSL and
  open round trip.
"""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from confkv_b200 import workloads
from confkv_b200.gpu_aesgcm import GpuAes128GcmKey
from gpu_helpers import GpuKey

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).parent / "golden" / "golden_frames.json").read_text())


def test_kv_small_frames_match_golden(gpu_lib):
    shape = workloads.SHAPES["kv_small"]
    key = workloads.make_key(1)
    ivs = workloads.make_ivs(1, 64)
    objs = workloads.bf16_objects(shape, 64, seed=1)
    digests = {d["name"]: d for d in GOLDEN["digests"]}
    k = GpuKey(gpu_lib, key)
    try:
        for i, (iv, t) in enumerate(zip(ivs, objs)):
            pt = t.view(torch.uint8).numpy().reshape(-1)
            frame = k.seal(pt, iv)
            assert hashlib.sha256(frame).hexdigest() == digests[f"kv_small_{i}"]["frame_sha256"], i
            auth, out = k.open(frame, pt.size)
            assert auth == 1 and out == pt.tobytes()
    finally:
        k.close()


def test_kv_llama8b_batch(gpu_lib, oracle):
    shape = workloads.SHAPES["kv_llama8b"]
    P = workloads.nbytes_of(shape)
    n = 32
    key = workloads.make_key(2)
    ivs = workloads.make_ivs(2, n)
    plain = workloads.bf16_batch(shape, n, seed=2, device="cuda").view(torch.uint8).reshape(n, P)
    stride = (P + 29 + 255) // 256 * 256
    frames = torch.zeros((n, stride), dtype=torch.uint8, device="cuda")
    opened = torch.zeros((n, P), dtype=torch.uint8, device="cuda")
    auth = torch.zeros((n,), dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with GpuAes128GcmKey(gpu_lib, key) as k:
        for i in range(n):
            k.seal_async(src_ptr=plain[i].data_ptr(), plaintext_len=P, dst_ptr=frames[i].data_ptr(),
                         dst_capacity=stride, iv=ivs[i], stream_ptr=s.cuda_stream)
        for i in range(n):
            k.open_async(src_ptr=frames[i].data_ptr(), frame_len=P + 29, dst_ptr=opened[i].data_ptr(),
                         plaintext_len=P, auth_ok_ptr=auth[i:i + 1].data_ptr(), stream_ptr=s.cuda_stream)
        s.synchronize()
    assert bool((auth == 1).all())
    assert torch.equal(opened, plain)
    host_plain = plain.cpu().numpy()
    host_frames = frames[:, :P + 29].cpu().numpy()
    expected = oracle.evp_seal_many(key, ivs, list(host_plain))
    for i in range(n):
        assert np.array_equal(host_frames[i], expected[i]), i
    if oracle.ref is not None:
        for i in (0, n - 1):
            rc, out = oracle.ref_open(key, host_frames[i])
            assert rc == 0 and np.array_equal(out, host_plain[i])


def test_ragged_adversarial_batch(gpu_lib, oracle):
    case = workloads.ragged_case(4096, seed=3)
    key = workloads.make_key(3)
    wrong = bytes(b ^ 0x5A for b in key)
    ivs = workloads.make_ivs(3, len(case.lengths))
    lens = case.lengths.astype(np.int64)
    pts = [workloads.ragged_payload(case, i) for i in range(len(lens))]
    # pack plaintexts and frames back to back (frames deliberately unaligned)
    pt_off = np.concatenate([[0], np.cumsum(lens)])
    fr_off = np.concatenate([[0], np.cumsum(lens + 29)])
    d_plain = torch.from_numpy(np.concatenate(pts)).cuda()
    d_frames = torch.zeros(int(fr_off[-1]), dtype=torch.uint8, device="cuda")
    d_out = torch.full((int(pt_off[-1]),), 0xCC, dtype=torch.uint8, device="cuda")
    d_auth = torch.full((len(lens),), 7, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    kgood = GpuAes128GcmKey(gpu_lib, key)
    kwrong = GpuAes128GcmKey(gpu_lib, wrong)
    try:
        for i in range(len(lens)):
            kgood.seal_async(src_ptr=d_plain.data_ptr() + int(pt_off[i]), plaintext_len=int(lens[i]),
                             dst_ptr=d_frames.data_ptr() + int(fr_off[i]), dst_capacity=int(lens[i]) + 29,
                             iv=ivs[i], stream_ptr=s.cuda_stream)
        s.synchronize()
        host_frames = d_frames.cpu().numpy()
        expected = oracle.evp_seal_many(key, ivs, pts)
        for i in range(len(lens)):
            assert np.array_equal(host_frames[fr_off[i]:fr_off[i + 1]], expected[i]), i
        # tamper 1% in place, on the host copy, then upload
        for i, (field, bit) in case.tamper.items():
            workloads.flip_bit(host_frames[fr_off[i]:fr_off[i + 1]], int(lens[i]), field, bit)
        d_frames.copy_(torch.from_numpy(host_frames))
        for i in range(len(lens)):
            k = kwrong if i in case.wrong_key else kgood
            k.open_async(src_ptr=d_frames.data_ptr() + int(fr_off[i]), frame_len=int(lens[i]) + 29,
                         dst_ptr=d_out.data_ptr() + int(pt_off[i]), plaintext_len=int(lens[i]),
                         auth_ok_ptr=d_auth[i:i + 1].data_ptr(), stream_ptr=s.cuda_stream)
        s.synchronize()
    finally:
        kgood.close()
        kwrong.close()
    auth = d_auth.cpu().numpy()
    out = d_out.cpu().numpy()
    bad = set(case.tamper) | case.wrong_key
    assert len(bad) == 2 * (len(lens) // 100)
    for i in range(len(lens)):
        seg = out[pt_off[i]:pt_off[i + 1]]
        if i in bad:
            assert auth[i] == 0, i
            assert not seg.any(), i
        else:
            assert auth[i] == 1, i
            assert np.array_equal(seg, pts[i]), i


@pytest.mark.parametrize("log2", list(range(12, 31, 2)) + [29, 30])
def test_size_sweep(gpu_lib, oracle, log2):
    size = 1 << log2
    rng = np.random.default_rng(log2)
    key, iv = rng.bytes(16), rng.bytes(12)
    g = torch.Generator(device="cuda")
    g.manual_seed(log2)
    plain = torch.randn(size // 2, generator=g, device="cuda").to(torch.bfloat16).view(torch.uint8)
    frame = torch.empty(size + 29, dtype=torch.uint8, device="cuda")
    out = torch.empty(size, dtype=torch.uint8, device="cuda")
    auth = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with GpuAes128GcmKey(gpu_lib, key) as k:
        k.seal_async(src_ptr=plain.data_ptr(), plaintext_len=size, dst_ptr=frame.data_ptr(),
                     dst_capacity=size + 29, iv=iv, stream_ptr=s.cuda_stream)
        k.open_async(src_ptr=frame.data_ptr(), frame_len=size + 29, dst_ptr=out.data_ptr(),
                     plaintext_len=size, auth_ok_ptr=auth.data_ptr(), stream_ptr=s.cuda_stream)
        s.synchronize()
    assert int(auth.item()) == 1
    assert torch.equal(out, plain)
    hp = plain.cpu().numpy()
    assert np.array_equal(frame.cpu().numpy(), oracle.evp_seal(key, iv, hp))
