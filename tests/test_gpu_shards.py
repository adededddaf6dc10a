"""Multi-GPU sharding, emulated on one device.

The path has no exchange between ranks: under torchrun every rank runs the same library calls on its
own share of the job (``anemll_b200.shard``), exactly as ``bench.py`` does.  So the multi-GPU parity
property is that each rank's share, run on its own, reproduces its slice of the unsharded run.  These
tests check that for 2, 4, 8 and 16 ranks on one GPU:

* GDN chunked prefill (sequences, then value-head groups with their key heads): output and final
  state bit-identical to the slice of the one-launch run;
* GDN recurrent decode (weak scaling: each rank its own batch of sequences): bit-identical;
* KV-cache attention (kv heads, with the query heads of each group; ranks beyond the kv heads
  replicate a group): the new cache rows bit-identical, the output within the parity bar (the
  split-KV plan may differ with the number of heads in one call).
"""
import pytest
import torch

from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _sl(t, dim, start, n):
    return t.narrow(dim, start, n).contiguous()


@pytest.mark.parametrize("world", [2, 4, 8, 16])
def test_chunked_prefill_shards_reproduce_the_full_run(world):
    from anemll_b200 import gdn, inputs, shard
    B, T, Hqk, Hv, d = 8, 256, 16, 32, 128
    w = inputs.gdn_prefill_device(seed=11, B=B, T=T, device=DEV, Hqk=Hqk, Hv=Hv)
    q, k, v, g, beta = w["q"], w["k"], w["v"], w["g"], w["beta"]
    s_full = torch.zeros(B, Hv, d, d, device=DEV)
    o_full = gdn.chunk_gated_delta_rule_(q, k, v, g, beta, s_full)
    covered = torch.zeros(B, Hv, dtype=torch.int32)
    for rank in range(world):
        sh = shard.prefill_shard(world, rank, B, Hqk, Hv)
        s0, ns, k0, nk, v0, nv = (sh.seq_start, sh.seq_count, sh.k_head_start, sh.k_head_count, sh.v_head_start,
                                  sh.v_head_count)
        qs, ks = (_sl(_sl(t, 0, s0, ns), 2, k0, nk) for t in (q, k))
        vs = _sl(_sl(v, 0, s0, ns), 2, v0, nv)
        gs, bs = (_sl(_sl(t, 0, s0, ns), 2, v0, nv) for t in (g, beta))
        st = torch.zeros(ns, nv, d, d, device=DEV)
        o = gdn.chunk_gated_delta_rule_(qs, ks, vs, gs, bs, st)
        assert torch.equal(o, o_full[s0:s0 + ns, :, v0:v0 + nv]), f"rank {rank}/{world}: output"
        assert torch.equal(st, s_full[s0:s0 + ns, v0:v0 + nv]), f"rank {rank}/{world}: state"
        covered[s0:s0 + ns, v0:v0 + nv] += 1
    assert bool((covered == 1).all()), "every (sequence, value head) owned by exactly one rank"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_recurrent_decode_shards_reproduce_the_full_batch(world):
    from anemll_b200 import gdn, inputs
    B, steps = 64, 3
    w = inputs.gdn_decode(seed=12, B=B, steps=steps)
    cuda = {n: t.to(DEV) for n, t in w.items() if torch.is_tensor(t)}
    s_full = cuda["state"].clone()
    outs = [gdn.recurrent_gated_delta_rule_(cuda["q"][i], cuda["k"][i], cuda["v"][i], cuda["g"][i],
                                            cuda["beta"][i], s_full) for i in range(steps)]
    per = B // world
    for rank in range(world):
        b0 = rank * per
        st = cuda["state"][b0:b0 + per].clone()
        for i in range(steps):
            o = gdn.recurrent_gated_delta_rule_(*(_sl(cuda[n][i], 0, b0, per) for n in ("q", "k", "v", "g", "beta")),
                                                st)
            assert torch.equal(o, outs[i][b0:b0 + per]), f"rank {rank}/{world}, step {i}: output"
        assert torch.equal(st, s_full[b0:b0 + per]), f"rank {rank}/{world}: state"


@pytest.mark.parametrize("world", [2, 4])
def test_kv_attention_shards_reproduce_the_full_call(world):
    from anemll_b200 import attention, shard
    Hq, Hkv, hd, ctx, G = 16, 2, 256, 1024, 8
    gen = torch.Generator().manual_seed(13)
    cache = torch.zeros(2, 1, Hkv, ctx, hd)
    cache[:, :, :, :512] = torch.randn(2, 1, Hkv, 512, hd, generator=gen)
    cache = cache.half().to(DEV)
    # a 64-token prefill chunk at 512, then a decode step at 576
    calls = []
    for pos, S in ((512, 64), (576, 1)):
        calls.append((pos, torch.randn(1, Hq, S, hd, generator=gen).half().to(DEV),
                      torch.randn(1, Hkv, S, hd, generator=gen).half().to(DEV),
                      torch.randn(1, Hkv, S, hd, generator=gen).half().to(DEV),
                      torch.randn(1, S, Hq * hd, generator=gen).half().to(DEV)))
    Kf, Vf = cache[0].clone(), cache[1].clone()
    full = [attention.kv_attention(q, Kf, Vf, pos, k_new=k, v_new=v, gate=gt) for pos, q, k, v, gt in calls]
    for rank in range(world):
        kv0, nkv = shard.kv_head_shard(world, rank, Hkv)
        hq0, nq = kv0 * G, nkv * G
        K, V = _sl(cache[0], 1, kv0, nkv), _sl(cache[1], 1, kv0, nkv)
        for (pos, q, k, v, gt), of in zip(calls, full):
            S = q.shape[2]
            gs = gt.view(1, S, Hq, hd)[:, :, hq0:hq0 + nq].reshape(1, S, nq * hd).contiguous()
            o = attention.kv_attention(_sl(q, 1, hq0, nq), K, V, pos, k_new=_sl(k, 1, kv0, nkv),
                                       v_new=_sl(v, 1, kv0, nkv), gate=gs)
            ref = of.view(1, S, Hq, hd)[:, :, hq0:hq0 + nq].reshape(1, S, nq * hd)
            assert_close(o.float().cpu(), ref.float().cpu(), f"kv rank {rank}/{world} pos {pos}")
        assert torch.equal(K, Kf[:, kv0:kv0 + nkv]) and torch.equal(V, Vf[:, kv0:kv0 + nkv]), \
            f"rank {rank}/{world}: cache rows"
