"""Host logic of the sharded stack run: the even split of sequences over ranks and the next-token id
gather, on two gloo ranks (CPU)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from anemll_b200.stack import nccl_id_gather, shard


def test_shard_splits_evenly():
    assert [shard(128, r, 8) for r in (0, 7)] == [(0, 16), (112, 128)]
    assert shard(128, 0, 1) == (0, 128)
    with pytest.raises(ValueError):
        shard(10, 0, 4)


def _rank(r, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=r, world_size=2)
    try:
        lo, hi = shard(6, r, 2)
        job = torch.arange(100, 106)
        gather = nccl_id_gather()
        got = [gather(job[lo:hi] + s) for s in range(3)]  # three steps of this rank's ids
        q.put((r, [g.tolist() for g in got]))
    finally:
        dist.destroy_process_group()


def test_id_gather_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert res[r] == [[100 + s + i for i in range(6)] for s in range(3)]
