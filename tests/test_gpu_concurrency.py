"""One key handle used from several host threads and streams at once.

The reference forbids concurrent use of a handle on different streams; here
each stream a handle is used on gets its own accumulation slot (the calls of
one stream are ordered on the device and share it), so four threads, each
with its own stream, may seal and open through one handle at the same time.
Every frame must equal the OpenSSL EVP frame and every open must authenticate
and restore the plaintext. Far more calls than slots may be outstanding; a
handle used on more distinct streams than it has slots refuses the extra
stream's call with ERR_ALLOC instead of sharing a slot.
"""

import threading

import numpy as np
import pytest
import torch

from confkv_b200 import workloads
from confkv_b200.gpu_aesgcm import GpuAes128GcmKey

pytestmark = pytest.mark.gpu

THREADS = 4
PER_THREAD = 24
SIZES = [1, 4096, 65536 + 5, (1 << 20) + 3, (3 << 20) + 17, 16 * 512 * 148 + 1]


def test_one_handle_four_threads_four_streams(gpu_lib, oracle):
    key = workloads.make_key(51)
    rng = np.random.default_rng(51)
    jobs = []
    for t in range(THREADS):
        sizes = [SIZES[(t + j) % len(SIZES)] for j in range(PER_THREAD)]
        ivs = workloads.make_ivs(100 + t, PER_THREAD)
        pts = [rng.integers(0, 256, size=n, dtype=np.uint8) for n in sizes]
        jobs.append((sizes, ivs, pts))
    expected = [oracle.evp_seal_many(key, ivs, pts) for sizes, ivs, pts in jobs]
    results = [None] * THREADS
    errors = []

    with GpuAes128GcmKey(gpu_lib, key) as k:
        barrier = threading.Barrier(THREADS)

        def run(t):
            try:
                sizes, ivs, pts = jobs[t]
                s = torch.cuda.Stream()
                d_pt = [torch.from_numpy(p).cuda() for p in pts]
                d_fr = [torch.zeros(n + 29, dtype=torch.uint8, device="cuda") for n in sizes]
                d_out = [torch.full((n,), 0xCC, dtype=torch.uint8, device="cuda") for n in sizes]
                d_auth = torch.zeros(PER_THREAD, dtype=torch.int32, device="cuda")
                torch.cuda.synchronize()
                barrier.wait()
                for j, n in enumerate(sizes):
                    k.seal_async(src_ptr=d_pt[j].data_ptr(), plaintext_len=n, dst_ptr=d_fr[j].data_ptr(),
                                 dst_capacity=n + 29, iv=ivs[j], stream_ptr=s.cuda_stream)
                for j, n in enumerate(sizes):
                    k.open_async(src_ptr=d_fr[j].data_ptr(), frame_len=n + 29, dst_ptr=d_out[j].data_ptr(),
                                 plaintext_len=n, auth_ok_ptr=d_auth[j:j + 1].data_ptr(), stream_ptr=s.cuda_stream)
                s.synchronize()
                results[t] = ([f.cpu().numpy() for f in d_fr], [o.cpu().numpy() for o in d_out],
                              d_auth.cpu().numpy())
            except Exception as e:  # reported below
                errors.append(e)

        workers = [threading.Thread(target=run, args=(t,)) for t in range(THREADS)]
        for w in workers:
            w.start()
        for w in workers:
            w.join()
    assert not errors, errors
    for t in range(THREADS):
        sizes, ivs, pts = jobs[t]
        frames, outs, auth = results[t]
        assert (auth == 1).all(), t
        for j in range(PER_THREAD):
            assert np.array_equal(frames[j], expected[t][j]), (t, j)
            assert np.array_equal(outs[j], pts[j]), (t, j)


def test_more_outstanding_calls_than_slots_on_two_streams(gpu_lib, oracle):
    """1,100 seals queued on two streams before any completes (more calls
    in flight than the handle has slots): each stream keeps its own slot, so
    every frame is still right."""
    key = workloads.make_key(52)
    rng = np.random.default_rng(52)
    n_calls = 1100
    size = 100_003
    pt = rng.integers(0, 256, size=size, dtype=np.uint8)
    ivs = workloads.make_ivs(53, n_calls)
    d_pt = torch.from_numpy(pt).cuda()
    d_fr = torch.zeros((n_calls, size + 29), dtype=torch.uint8, device="cuda")
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    gate = torch.cuda.Event()
    torch.cuda.synchronize()
    with GpuAes128GcmKey(gpu_lib, key) as k:
        # hold both streams behind a long kernel so the calls pile up
        spin = torch.cuda.Stream()
        with torch.cuda.stream(spin):
            torch.cuda._sleep(50_000_000)
            gate.record(spin)
        for s in streams:
            s.wait_event(gate)
        for j in range(n_calls):
            k.seal_async(src_ptr=d_pt.data_ptr(), plaintext_len=size, dst_ptr=d_fr[j].data_ptr(),
                         dst_capacity=size + 29, iv=ivs[j], stream_ptr=streams[j % 2].cuda_stream)
        torch.cuda.synchronize()
    frames = d_fr.cpu().numpy()
    expected = oracle.evp_seal_many(key, ivs, [pt] * n_calls)
    for j in range(n_calls):
        assert np.array_equal(frames[j], expected[j]), j


def test_stream_beyond_the_slot_count_is_refused(gpu_lib):
    """Each distinct stream takes one of the handle's 1024 slots; the call on
    a 1025th stream fails with ERR_ALLOC (-2) rather than sharing a slot.
    The streams come from the CUDA runtime itself (torch.cuda.Stream hands out
    a small pool of streams over and over)."""
    from cuda.bindings import runtime as rt

    from confkv_b200.gpu_aesgcm import GpuAesGcmError

    key = workloads.make_key(54)
    size = 4096
    d_pt = torch.zeros(size, dtype=torch.uint8, device="cuda")
    d_fr = torch.zeros(size + 29, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    streams = []
    try:
        for _ in range(1025):
            err, st = rt.cudaStreamCreateWithFlags(rt.cudaStreamNonBlocking)
            assert err == rt.cudaError_t.cudaSuccess, err
            streams.append(st)
        ptrs = [int(st) for st in streams]
        assert len(set(ptrs)) == 1025
        with GpuAes128GcmKey(gpu_lib, key) as k:
            for sp in ptrs[:1024]:
                k.seal_async(src_ptr=d_pt.data_ptr(), plaintext_len=size, dst_ptr=d_fr.data_ptr(),
                             dst_capacity=size + 29, iv=bytes(12), stream_ptr=sp)
                assert rt.cudaStreamSynchronize(sp)[0] == rt.cudaError_t.cudaSuccess
            with pytest.raises(GpuAesGcmError, match="allocation"):
                k.seal_async(src_ptr=d_pt.data_ptr(), plaintext_len=size, dst_ptr=d_fr.data_ptr(),
                             dst_capacity=size + 29, iv=bytes(12), stream_ptr=ptrs[1024])
            # a stream that already holds a slot keeps working
            k.seal_async(src_ptr=d_pt.data_ptr(), plaintext_len=size, dst_ptr=d_fr.data_ptr(),
                         dst_capacity=size + 29, iv=bytes(12), stream_ptr=ptrs[0])
            assert rt.cudaStreamSynchronize(ptrs[0])[0] == rt.cudaError_t.cudaSuccess
    finally:
        for st in streams:
            rt.cudaStreamDestroy(st)
