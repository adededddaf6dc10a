"""Generate ``cache_ops.pt``: golden vectors of the cache-management ops, from the reference itself.

Runs, on the CPU, the reference's own functions from the read-only checkout (``--reference PATH``
or the ``ANEMLL_REFERENCE`` environment variable):

* ``Gemma3Model._apply_update_mask`` / ``_apply_update_mask_batch``
  (``anemll/models/gemma3_model.py:932-965``), which use no model state, called unbound;
* ``Gemma3Model._update_kv_local`` (1024-1066) and ``_update_kv_local_prefill`` (1167-1204), called on a
  stand-in object that carries only the attributes they read (``config.sliding_window``,
  ``config.batch_size``, ``_local_layer_indices``, ``kv_cache_local``);
* ``transition_kv_state`` / ``compact_kv_state`` (``anemll/utils/state_transition.py:62-357``).

All tensors are fp16, the reference's cache dtype, except the dtype-converting transition case.
Usage: ``python tests/golden/make_cache_ops.py --reference PATH``.
"""
from __future__ import annotations

import argparse
import os
import sys
from types import SimpleNamespace

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root):
    sys.path.insert(0, ref_root)
    from anemll.models.gemma3_model import Gemma3Model
    from anemll.utils.state_transition import compact_kv_state, transition_kv_state

    g = torch.Generator().manual_seed(21)

    def rnd(*shape):
        return torch.randn(*shape, generator=g).half()

    fx = {}
    # ---- update-mask writes: one token, then a batch of tokens ----
    H, L, d = 2, 32, 64
    single = []
    for p in (0, 7, 31):
        cache = rnd(1, H, L, d)
        new = rnd(1, H, 1, d)
        mask = torch.zeros(1, 1, L, 1, dtype=torch.half)
        mask[0, 0, p, 0] = 1
        out = Gemma3Model._apply_update_mask(None, cache.clone(), new, mask)
        single.append(dict(cache=cache, new=new, mask=mask, out=out))
    fx["update_mask_single"] = single
    batch = []
    for start, S in ((0, 8), (20, 8), (5, 1)):
        cache = rnd(1, H, L, d)
        new = rnd(1, H, S, d)
        mask = torch.zeros(1, 1, L, S, dtype=torch.half)
        for s in range(S):
            mask[0, 0, start + s, s] = 1
        out = Gemma3Model._apply_update_mask_batch(None, cache.clone(), new, mask)
        batch.append(dict(cache=cache, new=new, mask=mask, out=out))
    fx["update_mask_batch"] = batch

    # ---- rotating sliding-window cache (split local cache of 2 local layers) ----
    sw, nloc = 32, 2
    rot = []
    for layer_idx, shift in ((0, 1), (1, 1), (0, 8), (1, 8)):
        kv = rnd(2 * nloc, H, sw, d)
        key = rnd(1, H, shift, d)
        val = rnd(1, H, shift, d)
        me = SimpleNamespace(config=SimpleNamespace(sliding_window=sw, batch_size=shift),
                             _local_layer_indices=list(range(nloc)), kv_cache_local=kv.clone())
        if shift == 1:
            Gemma3Model._update_kv_local(me, layer_idx, key, val)
        else:
            Gemma3Model._update_kv_local_prefill(me, layer_idx, key, val, shift)
        rot.append(dict(layer_idx=layer_idx, num_local=nloc, shift=shift, before=kv, key=key, value=val,
                        after=me.kv_cache_local))
    fx["rotate"] = rot

    # ---- KV-state transition (expand) and compaction ----
    trans = []
    src = rnd(3, 2, 16, 32)
    for tgt, pos, pad, dt in ((40, 10, 0.0, None), (40, None, 0.5, None), (16, 9, -1.0, None),
                              (24, 16, 0.0, torch.float32)):
        out = transition_kv_state(src, tgt, current_position=pos, pad_value=pad, dtype=dt)
        trans.append(dict(src=src, target=tgt, pos=pos, pad=pad, dtype=dt, out=out))
    big = rnd(3, 2, 48, 32)
    comp = []
    for tgt, pos in ((16, 10), (48, 48), (20, 0)):
        comp.append(dict(src=big, target=tgt, pos=pos, out=compact_kv_state(big, tgt, current_position=pos)))
    fx["transition"] = trans
    fx["compact"] = comp
    torch.save(fx, os.path.join(HERE, "cache_ops.pt"))
    print("cache_ops.pt", os.path.getsize(os.path.join(HERE, "cache_ops.pt")))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ANEMLL_REFERENCE"),
                    required="ANEMLL_REFERENCE" not in os.environ,
                    help="checkout of the reference repository (or set ANEMLL_REFERENCE)")
    main(ap.parse_args().reference)
