"""The benchmarked calls pinned directly to OpenSSL, through the C-ABI.

* The bench workload exactly as bench.py runs it on rank 0: 32 Llama-3-8B KV
  chunks [2, 32, 256, 8, 128] bf16 (32 MiB) under the bench key and IVs,
  frames at a 256-byte stride (ciphertext at frame + 13), sealed by ONE
  seal_batch_async call and opened by ONE open_batch_async call with the same
  descriptors as the bench; every frame is compared with OpenSSL EVP's.
* The Llama-3-70B TP-8 shard configuration as the config runner builds it:
  64 shards [2, 80, 256, 1, 128] bf16 (10 MiB), batched and per-object calls.
* The seal -> pinned-host store path (RankWork.seal_each_d2h: each frame
  copied to pinned host memory on a side stream as soon as it is sealed),
  objects of 1 B .. 64 MiB: every host frame against OpenSSL, every byte
  between frames untouched; then the load path back (open_each_from_host).
"""

import numpy as np
import pytest
import torch

from confkv_b200 import configs, workloads
from confkv_b200.batch import DeviceBatch
from confkv_b200.gpu_aesgcm import GpuAes128GcmKey

pytestmark = pytest.mark.gpu


def _assert_frames_match(oracle, key, ivs, host_plain, host_frames):
    expected = oracle.evp_seal_many(key, ivs, list(host_plain))
    for i, want in enumerate(expected):
        assert np.array_equal(host_frames[i], want), f"object {i}: frame differs from OpenSSL EVP"


def test_bench_workload_batched_frames_match_openssl(gpu_lib, oracle):
    case = workloads.bench_case(0, workloads.BENCH_OBJECTS, device="cuda")
    n, P, stride = len(case.ivs), case.object_bytes, case.frame_stride
    frames = torch.full((n, stride), 0x5A, dtype=torch.uint8, device="cuda")
    opened = torch.zeros((n, P), dtype=torch.uint8, device="cuda")
    auth = torch.zeros((n,), dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()  # inputs were written on the default stream
    with GpuAes128GcmKey(gpu_lib, case.key) as k:
        bseal, bopen = DeviceBatch(gpu_lib, n), DeviceBatch(gpu_lib, n)
        bseal.seal(k, [(case.plain[i].data_ptr(), frames[i].data_ptr(), P, stride, case.ivs[i]) for i in range(n)], s)
        bopen.open(k, [(frames[i].data_ptr(), opened[i].data_ptr(), P, P + 29, auth.data_ptr() + 4 * i)
                       for i in range(n)], s)
        s.synchronize()
        assert int(bseal.fault()) == 0 and int(bopen.fault()) == 0
        assert bseal.statuses().cpu().tolist() == [0] * n
    assert bool((auth == 1).all())
    assert torch.equal(opened, case.plain)
    host_frames = frames.cpu().numpy()
    assert (host_frames[:, P + 29:] == 0x5A).all(), "bytes past a frame were written"
    host_plain = case.plain.cpu().numpy()
    _assert_frames_match(oracle, case.key, case.ivs, host_plain, host_frames[:, :P + 29])
    if oracle.ref is not None:
        for i in (0, n // 2, n - 1):
            rc, out = oracle.ref_open(case.key, host_frames[i, :P + 29])
            assert rc == 0 and np.array_equal(out, host_plain[i])


def test_tp8_shard_config_matches_openssl(gpu_lib, oracle):
    shape = workloads.SHAPES["kv_llama70b_tp8_shard"]
    key = workloads.make_key(40)
    plain, offs, lens = configs.bf16_plain(shape, 64, seed=50, dev=torch.device("cuda", 0))
    ivs = workloads.make_ivs(1000, len(lens))
    s = torch.cuda.Stream()
    with GpuAes128GcmKey(gpu_lib, key) as k:
        work = configs.RankWork(gpu_lib, k, lens, plain, offs, s, ivs)  # its constructor runs one batched call
        torch.cuda.synchronize()
        host_plain = [plain[a:a + n].cpu().numpy() for a, n in zip(offs, lens)]
        for call in ("batched", "per_object"):
            work.frames.fill_(0)
            work.reset_outputs()
            torch.cuda.synchronize()  # the fills ran on the default stream
            (work.seal_batched if call == "batched" else work.seal_each)()
            (work.open_batched if call == "batched" else work.open_each)()
            s.synchronize()
            assert work.round_trip_ok(), call
            frames = work.frames.cpu().numpy()
            got = [frames[o:o + n + 29] for o, n in zip(work.fr_off, lens)]
            _assert_frames_match(oracle, key, ivs, host_plain, got)
        assert int(work.bseal.fault()) == 0 and int(work.bopen.fault()) == 0


def test_seal_each_d2h_host_frames_match_openssl(gpu_lib, oracle):
    sizes = [1, 15, 16, 17, 4096 + 3, 65536, (1 << 20) + 7, 3 << 20, (8 << 20) + 13, 64 << 20]
    dev = torch.device("cuda", 0)
    plain, offs = configs.random_plain(sizes, seed=91, dev=dev)
    ivs = workloads.make_ivs(92, len(sizes))
    key = workloads.make_key(93)
    s, side = torch.cuda.Stream(), torch.cuda.Stream()
    with GpuAes128GcmKey(gpu_lib, key) as k:
        work = configs.RankWork(gpu_lib, k, sizes, plain, offs, s, ivs)
        torch.cuda.synchronize()
        work.host_ptr()
        work.host.fill_(0x5C)
        torch.cuda.synchronize()
        work.seal_each_d2h(side)
        s.synchronize()
        side.synchronize()
        host = work.host.numpy().copy()
        host_plain = [plain[a:a + n].cpu().numpy() for a, n in zip(offs, sizes)]
        got = [host[o:o + n + 29] for o, n in zip(work.fr_off, sizes)]
        _assert_frames_match(oracle, key, ivs, host_plain, got)
        covered = np.zeros(host.size, dtype=bool)
        for o, n in zip(work.fr_off, sizes):
            covered[o:o + n + 29] = True
        assert (host[~covered] == 0x5C).all(), "the store path wrote outside the frames"
        # and back: frames from pinned host memory -> H2D -> gated open
        work.frames.fill_(0)
        work.reset_outputs()
        torch.cuda.synchronize()
        work.open_each_from_host(side)
        s.synchronize()
        assert work.round_trip_ok()


SEAL_TWO_PASS_OFFSET = 60  # BatchHeader.seal_two_pass: the plan's choice of seal design


@pytest.mark.parametrize("big,expect_two_pass", [((64 << 20) + 5, 1), ((1 << 20) + 3, 0)])
def test_batched_seal_both_designs_match_openssl(gpu_lib, oracle, big, expect_two_pass):
    """A batch of eight large objects with 300 small and mid objects mixed
    in: with 64 MiB objects the plan picks the two-pass seal (CTR pass, then
    the GHASH pass writes the tags), with 1 MiB objects the fused seal. Every
    frame must equal OpenSSL's either way, and the opens must round-trip."""
    rng = np.random.default_rng(big)
    lens = [big] * 8 + [int(x) for x in rng.integers(0, 40 << 10, size=300)]
    order = rng.permutation(len(lens))
    lens = [lens[i] for i in order]
    dev = torch.device("cuda", 0)
    plain, offs = configs.random_plain(lens, seed=17, dev=dev, packed=True)
    ivs = workloads.make_ivs(18, len(lens))
    key = workloads.make_key(19)
    s = torch.cuda.Stream()
    with GpuAes128GcmKey(gpu_lib, key) as k:
        work = configs.RankWork(gpu_lib, k, lens, plain, offs, s, ivs, packed=True)
        torch.cuda.synchronize()
        work.frames.fill_(0)
        work.reset_outputs()
        torch.cuda.synchronize()
        work.seal_batched()
        s.synchronize()
        mode = int(work.bseal.workspace[SEAL_TWO_PASS_OFFSET:SEAL_TWO_PASS_OFFSET + 4].view(torch.int32).item())
        assert mode == expect_two_pass
        assert int(work.bseal.fault()) == 0
        work.open_batched()
        s.synchronize()
        assert work.round_trip_ok()
        frames = work.frames.cpu().numpy()
        host_plain = [plain[a:a + n].cpu().numpy() for a, n in zip(offs, lens)]
        got = [frames[o:o + n + 29] for o, n in zip(work.fr_off, lens)]
        _assert_frames_match(oracle, key, ivs, host_plain, got)
