"""One key handle used from several host threads and streams at once.

The reference forbids concurrent use of a handle on different streams; here
each seal/open call takes its own entry of the handle's slot ring, so four
threads, each with its own stream, may seal and open through one handle at
the same time. Every frame must equal the OpenSSL EVP frame and every open
must authenticate and restore the plaintext.
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
