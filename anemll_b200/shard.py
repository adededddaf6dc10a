"""How the hot path splits over GPUs: independent units, no exchange inside an op.

Every (sequence, value head) recurrence of the gated delta rule and every
(sequence, kv head) attention is independent, so the work splits over ranks
with no collective on the data path:

* prefill: the sequences split evenly over the ranks; with more ranks than
  sequences each sequence's value heads split further, keeping the two value
  heads that read one key head together;
* decode (weak scaling): each rank owns its own batch, seeded by rank;
* KV attention: kv heads split first (each carries its H_q/H_kv query heads);
  beyond that, ranks are replicas.

The only cross-rank step the benchmark makes is one max-reduction of the timed
duration.  The reference is single-device and has no counterpart.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class PrefillShard:
    seq_start: int
    seq_count: int
    k_head_start: int
    k_head_count: int
    v_head_start: int
    v_head_count: int


def prefill_shard(world: int, rank: int, n_seqs: int, H_qk: int, H_v: int) -> PrefillShard:
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if H_v % H_qk:
        raise ValueError("H_v must be a multiple of H_qk")
    if world <= n_seqs:
        if n_seqs % world:
            raise ValueError(f"{n_seqs} sequences do not split evenly over {world} ranks")
        per = n_seqs // world
        return PrefillShard(rank * per, per, 0, H_qk, 0, H_v)
    if world % n_seqs:
        raise ValueError(f"{world} ranks do not split {n_seqs} sequences evenly")
    parts = world // n_seqs  # head groups per sequence
    if H_qk % parts:
        raise ValueError(f"{H_qk} key heads do not split into {parts} groups")
    seq = rank // parts
    grp = rank % parts
    kq = H_qk // parts
    rep = H_v // H_qk
    return PrefillShard(seq, 1, grp * kq, kq, grp * kq * rep, kq * rep)


def decode_seed(base_seed: int, rank: int) -> int:
    """Weak scaling: rank r decodes its own batch drawn from seed base + 1000 r."""
    return base_seed + 1000 * rank


def kv_head_shard(world: int, rank: int, H_kv: int):
    """(first kv head, count) owned by `rank`; ranks beyond H_kv replicate a head group."""
    if world <= H_kv:
        if H_kv % world:
            raise ValueError("kv heads do not split evenly")
        per = H_kv // world
        return rank * per, per
    return rank % H_kv, 1
