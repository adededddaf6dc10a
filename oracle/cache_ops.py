"""CPU oracle of the cache-management ops (test infrastructure only; the product never imports it).

Restates, in plain torch on the CPU, the reference's
* update-mask cache writes: ``Gemma3Model._apply_update_mask`` and ``_apply_update_mask_batch``
  (``anemll/models/gemma3_model.py:932-965``): ``cache * (1 - min(sum_s mask, 1)) + sum_s new_s * mask_s``;
* rotating sliding-window updates: ``_update_kv_local`` (1024-1066, shift left by one, append the new
  row) and ``_update_kv_local_prefill`` (1167-1204, shift left by the batch, append the batch);
* KV-state transition and compaction between context sizes: ``transition_kv_state`` /
  ``compact_kv_state`` (``anemll/utils/state_transition.py:62-152, 153-357``): a target of the new
  length filled with the pad value (zero for compaction), positions ``[0, current_position)`` copied
  and converted to the target dtype.

The pin is the reference itself: ``tests/golden/make_cache_ops.py`` runs those reference functions and
records their outputs in ``tests/golden/cache_ops.pt``.
"""
from __future__ import annotations

import torch


def update_mask_write(cache, new, mask):
    """``cache [..., L, d]``, ``new [..., S, d]``, ``mask [L, S]`` (1 at the write positions).

    Returns ``cache * (1 - min(sum_s mask, 1)) + sum_s new[s] * mask[:, s]`` in fp32 (the values of the
    reference's formula for 0/1 masks)."""
    m = mask.float()
    msum = torch.clamp(m.sum(-1), max=1.0)  # [L]
    upd = torch.einsum("...sd,ls->...ld", new.float(), m)
    return cache.float() * (1.0 - msum)[:, None] + upd


def rotate_append(cache, new, n):
    """Shift ``cache [..., L, d]`` left by ``n`` rows and append ``new[..., :n, :]`` at the end."""
    L = cache.shape[-2]
    if not 0 < n <= L:
        raise ValueError(f"shift {n} outside (0, {L}]")
    return torch.cat([cache[..., n:, :], new[..., :n, :]], dim=-2)


def transition_state(src, target_len, current_position, pad_value=0.0, dtype=None):
    """``src [L, H, S_src, d]`` -> ``[L, H, target_len, d]``: rows ``[0, current_position)`` from
    ``src`` (converted to ``dtype``), the rest ``pad_value``."""
    L, H, S, d = src.shape
    out_dtype = dtype if dtype is not None else src.dtype
    out = torch.full((L, H, target_len, d), pad_value, dtype=out_dtype)
    if current_position > 0:
        out[:, :, :current_position] = src[:, :, :current_position].to(out_dtype)
    return out
