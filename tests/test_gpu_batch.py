"""Batched seal / open (lmcache_gpu_aes128gcm_{seal,open}_batch_async).

Every frame a batch call writes must equal the OpenSSL EVP frame for the same
key, IV and plaintext (and so the per-object seal_async frame); batched open
must accept exactly the authentic frames, restore their plaintext and zero
the rest. Cases: the ragged adversarial workload (4096 objects, log-uniform
4 KiB .. 1 MiB, odd lengths, 1% tampered, 1% opened under a wrong key),
edge sizes with every 16-byte misalignment class of source and frame,
objects spanning many tiles, invalid descriptors, and workspace reuse.
"""

import numpy as np
import pytest
import torch

from confkv_b200 import workloads
from confkv_b200.batch import DeviceBatch
from confkv_b200.gpu_aesgcm import GpuAes128GcmKey

pytestmark = pytest.mark.gpu


def _packed(lens, align=1, pad=0):
    """Offsets of objects packed back to back (start rounded to `align`)."""
    offs, pos = [], 0
    for n in lens:
        pos = (pos + align - 1) // align * align
        offs.append(pos)
        pos += int(n) + pad
    return np.array(offs, dtype=np.int64), pos


def _seal_entries(d_plain, pt_off, d_frames, fr_off, lens, ivs):
    return [(d_plain.data_ptr() + int(pt_off[i]), d_frames.data_ptr() + int(fr_off[i]), int(lens[i]),
             int(lens[i]) + 29, ivs[i]) for i in range(len(lens))]


def _open_entries(d_frames, fr_off, d_out, pt_off, lens, d_auth, idx):
    return [(d_frames.data_ptr() + int(fr_off[i]), d_out.data_ptr() + int(pt_off[i]), int(lens[i]),
             int(lens[i]) + 29, d_auth.data_ptr() + 4 * int(i)) for i in idx]


def test_batch_ragged_adversarial(gpu_lib, oracle):
    case = workloads.ragged_case(4096, seed=5)
    key = workloads.make_key(5)
    wrong = bytes(b ^ 0x3C for b in key)
    lens = case.lengths.astype(np.int64)
    ivs = workloads.make_ivs(5, len(lens))
    pts = [workloads.ragged_payload(case, i) for i in range(len(lens))]
    pt_off, pt_total = _packed(lens)
    fr_off, fr_total = _packed(lens + 29)
    d_plain = torch.from_numpy(np.concatenate(pts)).cuda()
    d_frames = torch.full((fr_total + 64,), 0xAB, dtype=torch.uint8, device="cuda")
    d_out = torch.full((pt_total + 64,), 0xCC, dtype=torch.uint8, device="cuda")
    d_auth = torch.full((len(lens),), 7, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, len(lens))
    with GpuAes128GcmKey(gpu_lib, key) as kgood, GpuAes128GcmKey(gpu_lib, wrong) as kwrong:
        batch.seal(kgood, _seal_entries(d_plain, pt_off, d_frames, fr_off, lens, ivs), s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert not batch.statuses().any()
        host_frames = d_frames.cpu().numpy()
        assert (host_frames[fr_total:] == 0xAB).all()
        expected = oracle.evp_seal_many(key, ivs, pts)
        for i in range(len(lens)):
            assert np.array_equal(host_frames[fr_off[i]:fr_off[i] + lens[i] + 29], expected[i]), i
        for i, (field, bit) in case.tamper.items():
            workloads.flip_bit(host_frames[fr_off[i]:fr_off[i] + lens[i] + 29], int(lens[i]), field, bit)
        d_frames.copy_(torch.from_numpy(host_frames))
        good_idx = [i for i in range(len(lens)) if i not in case.wrong_key]
        batch.open(kgood, _open_entries(d_frames, fr_off, d_out, pt_off, lens, d_auth, good_idx), s)
        s.synchronize()
        assert int(batch.fault()) == 0
        batch.open(kwrong, _open_entries(d_frames, fr_off, d_out, pt_off, lens, d_auth, sorted(case.wrong_key)), s)
        s.synchronize()
        assert int(batch.fault()) == 0
    auth = d_auth.cpu().numpy()
    out = d_out.cpu().numpy()
    assert (out[pt_total:] == 0xCC).all()
    bad = set(case.tamper) | case.wrong_key
    for i in range(len(lens)):
        seg = out[pt_off[i]:pt_off[i] + lens[i]]
        if i in bad:
            assert auth[i] == 0, i
            assert not seg.any(), i
        else:
            assert auth[i] == 1, i
            assert np.array_equal(seg, pts[i]), i


EDGE_SIZES = [0, 1, 15, 16, 17, 31, 255, 256, 4095, 4096, 8191, 8192, 8193, 16 * 512 - 1, 16 * 512,
              16 * 512 + 1, 16 * 1024 * 3 + 5, (1 << 20) + 3, (5 << 20) + 7]


@pytest.mark.parametrize("src_mis,dst_mis", [(0, 0), (0, 3), (5, 0), (7, 11), (1, 15), (12, 2), (3, 8), (9, 6)])
def test_batch_edge_sizes_alignments(gpu_lib, oracle, src_mis, dst_mis):
    rng = np.random.default_rng(src_mis * 16 + dst_mis)
    key = rng.bytes(16)
    lens = np.array(EDGE_SIZES, dtype=np.int64)
    ivs = [rng.bytes(12) for _ in lens]
    pts = [rng.integers(0, 256, size=int(n), dtype=np.uint8) for n in lens]
    # every object starts at `mis` bytes past a 256-byte boundary
    pt_off, pt_total = _packed(lens, align=256, pad=256)
    fr_off, fr_total = _packed(lens + 29, align=256, pad=256)
    pt_off, fr_off = pt_off + src_mis, fr_off + dst_mis
    d_plain = torch.zeros(pt_total + 512, dtype=torch.uint8, device="cuda")
    for i, p in enumerate(pts):
        if len(p):
            d_plain[pt_off[i]:pt_off[i] + len(p)].copy_(torch.from_numpy(p))
    d_frames = torch.full((fr_total + 512,), 0xAB, dtype=torch.uint8, device="cuda")
    d_out = torch.full((pt_total + 512,), 0xCC, dtype=torch.uint8, device="cuda")
    d_auth = torch.full((len(lens),), 7, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, 64)
    with GpuAes128GcmKey(gpu_lib, key) as k:
        batch.seal(k, _seal_entries(d_plain, pt_off, d_frames, fr_off, lens, ivs), s)
        s.synchronize()
        assert int(batch.fault()) == 0
        frames = d_frames.cpu().numpy()
        expected = oracle.evp_seal_many(key, ivs, pts)
        mask = np.zeros(frames.size, dtype=bool)
        for i in range(len(lens)):
            assert np.array_equal(frames[fr_off[i]:fr_off[i] + lens[i] + 29], expected[i]), (i, lens[i])
            mask[fr_off[i]:fr_off[i] + lens[i] + 29] = True
        assert (frames[~mask] == 0xAB).all()
        batch.open(k, _open_entries(d_frames, fr_off, d_out, pt_off, lens, d_auth, range(len(lens))), s)
        s.synchronize()
        assert int(batch.fault()) == 0
    assert (d_auth.cpu().numpy() == 1).all()
    out = d_out.cpu().numpy()
    mask = np.zeros(out.size, dtype=bool)
    for i in range(len(lens)):
        assert np.array_equal(out[pt_off[i]:pt_off[i] + lens[i]], pts[i]), i
        mask[pt_off[i]:pt_off[i] + lens[i]] = True
    assert (out[~mask] == 0xCC).all()


def test_batch_multi_tile_objects_match_single_seal(gpu_lib):
    """A few large objects: each spans many tiles (the batch is small, so the
    tile height is small); frames equal seal_async's, and the same workspace
    serves two calls in a row."""
    key = workloads.make_key(9)
    lens = np.array([(32 << 20), (33 << 20) + 5, (7 << 20) + 9, 123457], dtype=np.int64)
    ivs = workloads.make_ivs(9, len(lens))
    pt_off, pt_total = _packed(lens, align=16)
    fr_off, fr_total = _packed(lens + 29, align=16)
    g = torch.Generator(device="cuda").manual_seed(9)
    d_plain = torch.randint(0, 256, (pt_total,), dtype=torch.uint8, device="cuda", generator=g)
    d_batch = torch.zeros(fr_total, dtype=torch.uint8, device="cuda")
    d_single = torch.zeros(fr_total, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, 8)
    with GpuAes128GcmKey(gpu_lib, key) as k:
        for _ in range(2):
            d_batch.zero_()
            batch.seal(k, _seal_entries(d_plain, pt_off, d_batch, fr_off, lens, ivs), s)
            for i in range(len(lens)):
                k.seal_async(src_ptr=d_plain.data_ptr() + int(pt_off[i]), plaintext_len=int(lens[i]),
                             dst_ptr=d_single.data_ptr() + int(fr_off[i]), dst_capacity=int(lens[i]) + 29,
                             iv=ivs[i], stream_ptr=s.cuda_stream)
            s.synchronize()
            assert int(batch.fault()) == 0
            assert torch.equal(d_batch, d_single)
        d_out = torch.zeros_like(d_plain)
        d_auth = torch.zeros(len(lens), dtype=torch.int32, device="cuda")
        batch.open(k, _open_entries(d_batch, fr_off, d_out, pt_off, lens, d_auth, range(len(lens))), s)
        s.synchronize()
        assert int(batch.fault()) == 0
    assert (d_auth == 1).all()
    for i in range(len(lens)):
        a, n = int(pt_off[i]), int(lens[i])
        assert torch.equal(d_out[a:a + n], d_plain[a:a + n]), i


def test_batch_invalid_descriptors_are_skipped(gpu_lib):
    key = workloads.make_key(11)
    n = 4096
    d_plain = torch.arange(4 * n, dtype=torch.int64, device="cuda").to(torch.uint8)
    d_frames = torch.full((4 * (n + 29) + 64,), 0xAB, dtype=torch.uint8, device="cuda")
    base_p, base_f = d_plain.data_ptr(), d_frames.data_ptr()
    iv = bytes(12)
    entries = [
        (base_p, base_f, n, n + 29, iv),                      # valid
        (0, base_f + (n + 29), n, n + 29, iv),                # null source
        (base_p, base_f + 2 * (n + 29), n, n + 28, iv),       # capacity one byte short
        (base_p, base_f + 3 * (n + 29), n, n + 29, iv),       # valid
    ]
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, 4)
    with GpuAes128GcmKey(gpu_lib, key) as k:
        batch.seal(k, entries, s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert batch.statuses().cpu().tolist() == [0, -1, -1, 0]
        frames = d_frames.cpu().numpy()
        assert (frames[n + 29:3 * (n + 29)] == 0xAB).all()
        assert frames[0] == 1 and frames[3 * (n + 29)] == 1
        assert np.array_equal(frames[:n + 29], frames[3 * (n + 29):4 * (n + 29)])
        # open: a null auth_ok pointer and a short frame length are skipped
        d_out = torch.full((4 * n,), 0xCC, dtype=torch.uint8, device="cuda")
        d_auth = torch.full((4,), 7, dtype=torch.int32, device="cuda")
        o = [(base_f, d_out.data_ptr(), n, n + 29, d_auth.data_ptr()),
             (base_f, d_out.data_ptr() + n, n, n + 29, 0),
             (base_f, d_out.data_ptr() + 2 * n, n, n + 28, d_auth.data_ptr() + 8),
             (base_f + 3 * (n + 29), d_out.data_ptr() + 3 * n, n, n + 29, d_auth.data_ptr() + 12)]
        batch.open(k, o, s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert batch.statuses().cpu().tolist() == [0, -1, -1, 0]
    # the rejected descriptor with an auth_ok pointer gets 0, not the stale 7
    assert d_auth.cpu().tolist() == [1, 7, 0, 1]
    out = d_out.cpu().numpy()
    assert (out[n:3 * n] == 0xCC).all()
    pl = d_plain[:n].cpu().numpy()
    assert np.array_equal(out[:n], pl) and np.array_equal(out[3 * n:], pl)


def test_batch_many_small_objects(gpu_lib, oracle):
    """8192 objects of 4 KiB and 8192 of 0..64 bytes in one call each."""
    rng = np.random.default_rng(21)
    key = rng.bytes(16)
    for lens in (np.full(8192, 4096, dtype=np.int64), rng.integers(0, 65, size=8192).astype(np.int64)):
        ivs = [rng.bytes(12) for _ in lens]
        pts = [rng.integers(0, 256, size=int(n), dtype=np.uint8) for n in lens]
        pt_off, pt_total = _packed(lens)
        fr_off, fr_total = _packed(lens + 29)
        d_plain = torch.from_numpy(np.concatenate(pts + [np.zeros(16, np.uint8)])).cuda()
        d_frames = torch.zeros(fr_total + 16, dtype=torch.uint8, device="cuda")
        s = torch.cuda.Stream()
        batch = DeviceBatch(gpu_lib, len(lens))
        with GpuAes128GcmKey(gpu_lib, key) as k:
            batch.seal(k, _seal_entries(d_plain, pt_off, d_frames, fr_off, lens, ivs), s)
            s.synchronize()
            assert int(batch.fault()) == 0
        frames = d_frames.cpu().numpy()
        expected = oracle.evp_seal_many(key, ivs, pts)
        for i in range(len(lens)):
            assert np.array_equal(frames[fr_off[i]:fr_off[i] + lens[i] + 29], expected[i]), (i, lens[i])


def _plan_counts(batch):
    """(tile objects, warp-path objects) of the last call, as the device plan
    recorded them in the workspace header (BatchHeader: tile_objects at byte
    20, small_count at byte 24)."""
    h = batch.workspace[:32].cpu().numpy().view(np.uint32)
    return int(h[5]), int(h[6])


def _expected_counts(lens, routed):
    blocks = [-(-int(n) // 16) for n in lens]
    warp = sum(1 for n in blocks if n <= 1024 or (routed and n <= 2048))
    return len(lens) - warp, warp


@pytest.mark.parametrize("per_sm", [0, 10, 16])
def test_batch_mid_objects_both_routes(gpu_lib, oracle, per_sm):
    """Objects of 1025..2048 blocks (16-32 KiB) take one warp each when the
    batch has enough of them, else they are tile objects: 300 objects stay
    tiles, 10 per SM take warps in open only, 16 per SM in both directions
    (the plan's rule, replayed by tests/schedules.py). Both routes give
    OpenSSL's frames and open's gating. Sizes cover both ends of the range
    and the first size above it, every alignment class; one object in 50 is
    tampered."""
    from schedules import mid_routed

    sms = min(torch.cuda.get_device_properties(0).multi_processor_count, 256)
    count = per_sm * sms + 7 if per_sm else 300
    rng = np.random.default_rng(88 + per_sm)
    key = rng.bytes(16)
    edges = [16 * 1024 + 1, 16 * 1025, 16 * 2048 - 1, 16 * 2048, 16 * 2048 + 1, 16 * 2049, 4096, 0]
    lens = np.concatenate([edges, rng.integers(16 * 1024 + 1, 16 * 2048 + 1, size=count - len(edges))]).astype(np.int64)
    routes = (mid_routed(lens.tolist(), sms), mid_routed(lens.tolist(), sms, open_=True))
    assert routes == {0: (False, False), 10: (False, True), 16: (True, True)}[per_sm]
    ivs = [rng.bytes(12) for _ in lens]
    pts = [rng.integers(0, 256, size=int(n), dtype=np.uint8) for n in lens]
    pt_off, pt_total = _packed(lens, pad=3)
    fr_off, fr_total = _packed(lens + 29, pad=5)
    d_plain = torch.zeros(pt_total + 16, dtype=torch.uint8, device="cuda")
    d_plain[:pt_total].copy_(torch.from_numpy(np.concatenate(
        [np.concatenate([p, np.zeros(3, np.uint8)]) for p in pts])))
    d_frames = torch.full((fr_total + 16,), 0xAB, dtype=torch.uint8, device="cuda")
    d_out = torch.full((pt_total + 16,), 0xCC, dtype=torch.uint8, device="cuda")
    d_auth = torch.full((len(lens),), 7, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, len(lens))
    with GpuAes128GcmKey(gpu_lib, key) as k:
        batch.seal(k, _seal_entries(d_plain, pt_off, d_frames, fr_off, lens, ivs), s)
        s.synchronize()
        assert int(batch.fault()) == 0 and not batch.statuses().any()
        assert _plan_counts(batch) == _expected_counts(lens, routes[0])
        frames = d_frames.cpu().numpy()
        expected = oracle.evp_seal_many(key, ivs, pts)
        for i in range(len(lens)):
            assert np.array_equal(frames[fr_off[i]:fr_off[i] + lens[i] + 29], expected[i]), (i, lens[i])
        bad = set(range(3, len(lens), 50))
        for i in bad:
            frames[fr_off[i] + 13 + int(rng.integers(0, lens[i] + 16))] ^= 0x10
        d_frames.copy_(torch.from_numpy(frames))
        batch.open(k, _open_entries(d_frames, fr_off, d_out, pt_off, lens, d_auth, range(len(lens))), s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert _plan_counts(batch) == _expected_counts(lens, routes[1])
    auth = d_auth.cpu().numpy()
    out = d_out.cpu().numpy()
    for i in range(len(lens)):
        seg = out[pt_off[i]:pt_off[i] + lens[i]]
        if i in bad:
            assert auth[i] == 0 and not seg.any(), i
        else:
            assert auth[i] == 1 and np.array_equal(seg, pts[i]), i
        assert (out[pt_off[i] + lens[i]:pt_off[i] + lens[i] + 3] == 0xCC).all(), i


def test_batch_two_hundred_thousand_tiny_objects(gpu_lib, oracle):
    """200,000 objects of 0..256 bytes in one seal and one open call (the
    warp-per-object path, a plan over hundreds of objects per thread); every
    frame equals OpenSSL's; one object in 1,000 is tampered and rejected."""
    rng = np.random.default_rng(77)
    count = 200_000
    lens = rng.integers(0, 257, size=count).astype(np.int64)
    key = rng.bytes(16)
    ivs = [rng.bytes(12) for _ in range(count)]
    pt_all = rng.integers(0, 256, size=int(lens.sum()) + 16, dtype=np.uint8)
    pt_off, pt_total = _packed(lens)
    fr_off, fr_total = _packed(lens + 29)
    pts = [pt_all[pt_off[i]:pt_off[i] + lens[i]] for i in range(count)]
    d_plain = torch.from_numpy(pt_all).cuda()
    d_frames = torch.zeros(fr_total + 16, dtype=torch.uint8, device="cuda")
    d_out = torch.full((pt_total + 16,), 0xCC, dtype=torch.uint8, device="cuda")
    d_auth = torch.full((count,), 7, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, count)
    with GpuAes128GcmKey(gpu_lib, key) as k:
        batch.seal(k, _seal_entries(d_plain, pt_off, d_frames, fr_off, lens, ivs), s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert not batch.statuses().any()
        frames = d_frames.cpu().numpy()
        expected = oracle.evp_seal_many(key, ivs, pts)
        for i in range(count):
            assert np.array_equal(frames[fr_off[i]:fr_off[i] + lens[i] + 29], expected[i]), i
        bad = set(int(x) for x in rng.choice(count, size=count // 1000, replace=False))
        for i in bad:
            frames[fr_off[i] + 13 + int(lens[i]) + int(rng.integers(0, 16))] ^= 0x20   # a tag byte
        d_frames.copy_(torch.from_numpy(frames))
        batch.open(k, _open_entries(d_frames, fr_off, d_out, pt_off, lens, d_auth, range(count)), s)
        s.synchronize()
        assert int(batch.fault()) == 0
    auth = d_auth.cpu().numpy()
    out = d_out.cpu().numpy()
    for i in range(count):
        seg = out[pt_off[i]:pt_off[i] + lens[i]]
        if i in bad:
            assert auth[i] == 0 and not seg.any(), i
        else:
            assert auth[i] == 1 and np.array_equal(seg, pts[i]), i


def _seal_single(k, d_plain, pt_off, d_frames, fr_off, lens, ivs, s):
    for i in range(len(lens)):
        k.seal_async(src_ptr=d_plain.data_ptr() + int(pt_off[i]), plaintext_len=int(lens[i]),
                     dst_ptr=d_frames.data_ptr() + int(fr_off[i]), dst_capacity=int(lens[i]) + 29,
                     iv=ivs[i], stream_ptr=s.cuda_stream)


@pytest.mark.parametrize("lens", [
    # one large object cut by many chunk boundaries, tile objects of 3 rows, warp-path
    # objects and an empty one, at odd offsets
    [(64 << 20) + 7] + [20 * 1024 + 3] * 6 + [4096, 0, (1 << 20) + 1],
    # fewer rows than SMs: one-row chunks, so every 3-row object is three segments and
    # the first one holds a single block (1025 blocks = 3 rows, row 0 partial)
    [16 * 1024 + 16] * 3,
    [16 * 1024 + 16, 40 * 1024, 16 * 1024 + 1],
])
def test_batch_chunk_boundaries_and_gating(gpu_lib, lens):
    """Segments of one object run on different CTAs: the frames equal
    seal_async's, and a tampered object is rejected and zero-filled in every
    segment while its neighbours in the same chunks open."""
    key = workloads.make_key(21)
    lens = np.array(lens, dtype=np.int64)
    ivs = workloads.make_ivs(21, len(lens))
    pt_off, pt_total = _packed(lens, align=1, pad=3)
    fr_off, fr_total = _packed(lens + 29, align=1, pad=5)
    g = torch.Generator(device="cuda").manual_seed(21)
    d_plain = torch.randint(0, 256, (pt_total + 16,), dtype=torch.uint8, device="cuda", generator=g)
    d_batch = torch.zeros(fr_total + 16, dtype=torch.uint8, device="cuda")
    d_single = torch.zeros(fr_total + 16, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, len(lens))
    with GpuAes128GcmKey(gpu_lib, key) as k:
        batch.seal(k, _seal_entries(d_plain, pt_off, d_batch, fr_off, lens, ivs), s)
        _seal_single(k, d_plain, pt_off, d_single, fr_off, lens, ivs, s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert not batch.statuses().any()
        assert torch.equal(d_batch, d_single)
        # tamper the middle of the largest object's ciphertext and the tag of the last one
        big = int(np.argmax(lens))
        mid = int(fr_off[big]) + 13 + int(lens[big]) // 2
        d_batch[mid] ^= 0x10
        last = len(lens) - 1
        d_batch[int(fr_off[last]) + 13 + int(lens[last])] ^= 0x01
        d_out = torch.full((pt_total + 16,), 0xCC, dtype=torch.uint8, device="cuda")
        d_auth = torch.full((len(lens),), 7, dtype=torch.int32, device="cuda")
        batch.open(k, _open_entries(d_batch, fr_off, d_out, pt_off, lens, d_auth, range(len(lens))), s)
        s.synchronize()
        assert int(batch.fault()) == 0
    auth = d_auth.cpu().tolist()
    for i in range(len(lens)):
        a, n = int(pt_off[i]), int(lens[i])
        if i in (big, last):
            assert auth[i] == 0, i
            assert not d_out[a:a + n].any(), i
        else:
            assert auth[i] == 1, i
            assert torch.equal(d_out[a:a + n], d_plain[a:a + n]), i


def test_batch_handoff_wait_runs_out_without_hanging(gpu_lib, monkeypatch):
    """Host-side stall injection (CONFKV_B200_TEST_HANDOFF_STALL=1): the seal
    power warps take no hand-off, so the row warps' bounded waits run out
    after 50 ms. The call must return with the batch's fault word set, and the
    next call in the same context must be correct."""
    import time

    key = workloads.make_key(41)
    lens = np.array([40 * 1024] * 1200, dtype=np.int64)   # 5-row tile objects: many segments per CTA
    ivs = workloads.make_ivs(41, len(lens))
    pt_off, pt_total = _packed(lens, align=16)
    fr_off, fr_total = _packed(lens + 29, align=16)
    g = torch.Generator(device="cuda").manual_seed(41)
    d_plain = torch.randint(0, 256, (pt_total,), dtype=torch.uint8, device="cuda", generator=g)
    d_batch = torch.zeros(fr_total, dtype=torch.uint8, device="cuda")
    d_single = torch.zeros(fr_total, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, len(lens))
    entries = _seal_entries(d_plain, pt_off, d_batch, fr_off, lens, ivs)
    with GpuAes128GcmKey(gpu_lib, key) as k:
        monkeypatch.setenv("CONFKV_B200_TEST_HANDOFF_STALL", "1")
        t0 = time.monotonic()
        batch.seal(k, entries, s)
        s.synchronize()
        elapsed = time.monotonic() - t0
        assert int(batch.fault()) != 0
        assert elapsed < 10.0
        monkeypatch.delenv("CONFKV_B200_TEST_HANDOFF_STALL")
        batch.seal(k, entries, s)
        _seal_single(k, d_plain, pt_off, d_single, fr_off, lens, ivs, s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert torch.equal(d_batch, d_single)


@pytest.mark.parametrize("mixed", [False, True])
def test_batch_chunk_count_matches_replay(gpu_lib, oracle, mixed):
    """A batch of many tile objects per SM takes one chunk per SM when its
    objects are about the same size (the largest at most twice the rows of
    the smallest) and four per SM when they are mixed; the device plan's chunk
    count (BatchHeader.chunks, byte 8 of the workspace) must equal the CPU
    replay's (tests/schedules.py). Both give OpenSSL's frames and open back."""
    from schedules import chunk_plan

    sms = min(torch.cuda.get_device_properties(0).multi_processor_count, 256)
    count = 5 * sms
    rng = np.random.default_rng(97 + mixed)
    key = rng.bytes(16)
    if mixed:
        lens = np.array([(1 << 20) + int(rng.integers(0, 16)) if i % 2 else 65536 + int(rng.integers(1, 16))
                         for i in range(count)], dtype=np.int64)
    else:
        # 64-65 rows each: enough rows for four chunks per SM, one for a uniform batch
        lens = np.array([524288 + (i % 7) for i in range(count)], dtype=np.int64)
    plan = chunk_plan(lens.tolist(), sms)
    assert plan["M"] == (4 * sms if mixed else sms)
    ivs = [rng.bytes(12) for _ in lens]
    pts = [rng.integers(0, 256, size=int(n), dtype=np.uint8) for n in lens]
    pt_off, pt_total = _packed(lens, align=256)
    fr_off, fr_total = _packed(lens + 29, align=256)
    d_plain = torch.zeros(pt_total + 16, dtype=torch.uint8, device="cuda")
    d_plain[:pt_total].copy_(torch.from_numpy(np.concatenate(
        [np.concatenate([p, np.zeros(int(pt_off[i + 1] - pt_off[i]) - len(p) if i + 1 < len(pts) else 0, np.uint8)])
         for i, p in enumerate(pts)])))
    d_frames = torch.zeros(fr_total + 16, dtype=torch.uint8, device="cuda")
    d_out = torch.zeros(pt_total + 16, dtype=torch.uint8, device="cuda")
    d_auth = torch.full((len(lens),), 7, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    batch = DeviceBatch(gpu_lib, len(lens))
    with GpuAes128GcmKey(gpu_lib, key) as k:
        batch.seal(k, _seal_entries(d_plain, pt_off, d_frames, fr_off, lens, ivs), s)
        s.synchronize()
        assert int(batch.fault()) == 0 and not batch.statuses().any()
        chunks = int(batch.workspace[8:12].cpu().numpy().view(np.uint32)[0])
        assert chunks == plan["M"]
        frames = d_frames.cpu().numpy()
        expected = oracle.evp_seal_many(key, ivs, pts)
        for i in range(len(lens)):
            assert np.array_equal(frames[fr_off[i]:fr_off[i] + lens[i] + 29], expected[i]), (i, lens[i])
        batch.open(k, _open_entries(d_frames, fr_off, d_out, pt_off, lens, d_auth, range(len(lens))), s)
        s.synchronize()
        assert int(batch.fault()) == 0
        assert int(batch.workspace[8:12].cpu().numpy().view(np.uint32)[0]) == plan["M"]
        assert bool((d_auth == 1).all())
        out = d_out.cpu().numpy()
        for i in range(len(lens)):
            assert np.array_equal(out[pt_off[i]:pt_off[i] + lens[i]], pts[i]), (i, lens[i])
