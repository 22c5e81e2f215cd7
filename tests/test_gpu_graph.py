"""Seal / open calls captured into CUDA graphs.

Key handles and descriptor arrays are created before capture; the captured
calls (per-object seal_async / open_async, launched with programmatic stream
serialization, and the batched calls) allocate nothing and synchronise
nothing, so a graph of them replays the same work. Replays must write the
same frames as eager calls and open them, repeatedly.
"""

import numpy as np
import pytest
import torch

from confkv_b200 import workloads
from confkv_b200.batch import DeviceBatch
from confkv_b200.gpu_aesgcm import GpuAes128GcmKey

pytestmark = pytest.mark.gpu


def _buffers(lens, seed):
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    foffs = np.concatenate([[0], np.cumsum(np.asarray(lens) + 29)]).astype(np.int64)
    g = torch.Generator(device="cuda").manual_seed(seed)
    plain = torch.randint(0, 256, (int(offs[-1]) + 16,), dtype=torch.uint8, device="cuda", generator=g)
    return offs, foffs, plain


@pytest.mark.parametrize("style", ["per_object", "batched"])
def test_graph_replay_matches_eager(gpu_lib, style):
    rng = np.random.default_rng(31)
    lens = [int(x) for x in rng.integers(0, 70000, size=200)] + [0, 1, 4096, 65536, 3 << 20]
    ivs = workloads.make_ivs(31, len(lens))
    offs, foffs, plain = _buffers(lens, 31)
    eager = torch.zeros(int(foffs[-1]) + 16, dtype=torch.uint8, device="cuda")
    frames = torch.zeros_like(eager)
    out = torch.zeros_like(plain)
    auth = torch.zeros(len(lens), dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    pb, eb, fb, ob, ab = plain.data_ptr(), eager.data_ptr(), frames.data_ptr(), out.data_ptr(), auth.data_ptr()
    with GpuAes128GcmKey(gpu_lib, workloads.make_key(31)) as k:
        for i, n in enumerate(lens):
            k.seal_async(src_ptr=pb + int(offs[i]), plaintext_len=n, dst_ptr=eb + int(foffs[i]),
                         dst_capacity=n + 29, iv=ivs[i], stream_ptr=s.cuda_stream)
        s.synchronize()
        seal_items = [(pb + int(offs[i]), fb + int(foffs[i]), n, n + 29, ivs[i]) for i, n in enumerate(lens)]
        open_items = [(fb + int(foffs[i]), ob + int(offs[i]), n, n + 29, ab + 4 * i) for i, n in enumerate(lens)]
        if style == "batched":
            bs, bo = DeviceBatch(gpu_lib, len(lens)), DeviceBatch(gpu_lib, len(lens))
            bs.seal(k, seal_items, s)
            bo.open(k, open_items, s)
            s.synchronize()

            def body():
                k.seal_batch_async(items_ptr=bs.items.data_ptr(), count=len(lens), workspace_ptr=bs.workspace.data_ptr(),
                                   workspace_bytes=bs.workspace_bytes, stream_ptr=s.cuda_stream)
                k.open_batch_async(items_ptr=bo.items.data_ptr(), count=len(lens), workspace_ptr=bo.workspace.data_ptr(),
                                   workspace_bytes=bo.workspace_bytes, stream_ptr=s.cuda_stream)
        else:
            def body():
                for src, dst, n, cap, iv in seal_items:
                    k.seal_async(src_ptr=src, plaintext_len=n, dst_ptr=dst, dst_capacity=cap, iv=iv,
                                 stream_ptr=s.cuda_stream)
                for f, d, n, fl, a in open_items:
                    k.open_async(src_ptr=f, frame_len=fl, dst_ptr=d, plaintext_len=n, auth_ok_ptr=a,
                                 stream_ptr=s.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            body()
        for _ in range(3):
            frames.zero_()
            out.zero_()
            auth.zero_()
            torch.cuda.synchronize()
            with torch.cuda.stream(s):
                g.replay()
            s.synchronize()
            assert torch.equal(frames, eager)
            assert (auth == 1).all()
            for i, n in enumerate(lens):
                a = int(offs[i])
                assert torch.equal(out[a:a + n], plain[a:a + n]), i
        del g
