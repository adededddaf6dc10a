"""Multi-rank host logic on CPU (gloo, world size 2 and 4): the shards cover every
(sequence, value head) unit exactly once, key-head pairs stay together, and the
max-over-ranks reduction the benchmark uses gives the slowest rank's time."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from anemll_b200 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_seqs, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        sh = shard.prefill_shard(world, rank, n_seqs, 16, 32)
        units = [(s, h) for s in range(sh.seq_start, sh.seq_start + sh.seq_count)
                 for h in range(sh.v_head_start, sh.v_head_start + sh.v_head_count)]
        pairs_ok = all(h // 2 in range(sh.k_head_start, sh.k_head_start + sh.k_head_count)
                       for _, h in units)
        gathered = [None] * world
        dist.all_gather_object(gathered, units)
        t = torch.tensor([float(10 + rank)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((gathered, pairs_ok, float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_seqs", [(2, 8), (4, 2)])
def test_prefill_shards_cover_all_units_once(world, n_seqs):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_seqs, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, pairs_ok, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    allu = [u for g in gathered for u in g]
    assert sorted(allu) == [(s, h) for s in range(n_seqs) for h in range(32)]
    assert len(allu) == len(set(allu))
    assert pairs_ok
    assert tmax == 10.0 + world - 1


def test_shard_rules():
    assert shard.prefill_shard(8, 3, 8, 16, 32) == shard.PrefillShard(3, 1, 0, 16, 0, 32)
    s = shard.prefill_shard(8, 5, 2, 16, 32)  # 4 head groups per sequence
    assert (s.seq_start, s.k_head_start, s.k_head_count, s.v_head_start, s.v_head_count) == (1, 4, 4, 8, 8)
    with pytest.raises(ValueError):
        shard.prefill_shard(3, 0, 8, 16, 32)
    assert shard.kv_head_shard(2, 1, 2) == (1, 1)
    assert shard.kv_head_shard(8, 5, 2) == (1, 1)
    assert shard.decode_seed(1, 3) == 3001
