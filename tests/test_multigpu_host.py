"""Multi-GPU host logic on CPU: world-size-2 gloo process group exercising the
object partition, the max-over-ranks timing reduction and the all-ranks-ok
check that bench.py uses under torchrun (on GPUs the same calls run on NCCL).
"""

import os
import socket

import pytest
import torch.multiprocessing as mp

from confkv_b200 import multigpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        mine = multigpu.round_robin(37, rank, world)
        times = [10.0 + rank, 5.0 * (world - rank)]
        mx = multigpu.reduce_max(times)
        sm = multigpu.reduce_sum([len(mine)])
        ok_all = multigpu.all_ok(True)
        ok_one_bad = multigpu.all_ok(rank != 1)
        q.put((rank, mine, (mx, sm), ok_all, ok_one_bad))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_partition_and_reductions():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, mine, mx, ok_all, ok_one_bad = q.get(timeout=120)
        results[rank] = (mine, mx, ok_all, ok_one_bad)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    covered = sorted(results[0][0] + results[1][0])
    assert covered == list(range(37))
    assert not set(results[0][0]) & set(results[1][0])
    for rank in range(world):
        assert results[rank][1] == ([11.0, 10.0], [37.0])
        assert results[rank][2] is True
        assert results[rank][3] is False


def test_single_process_helpers():
    assert multigpu.round_robin(5, 0, 1) == [0, 1, 2, 3, 4]
    assert multigpu.reduce_max([1.5, 2.0]) == [1.5, 2.0]
    assert multigpu.reduce_sum([3]) == [3.0]
    assert multigpu.all_ok(True) and not multigpu.all_ok(False)
    assert list(multigpu.kv_head_shard(8, 3, 8)) == [3]
    with pytest.raises(ValueError):
        multigpu.round_robin(5, 2, 2)
    with pytest.raises(ValueError):
        multigpu.kv_head_shard(8, 0, 3)
