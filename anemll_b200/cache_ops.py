"""Cache-management ops on the device, behind the reference's function names and arguments.

* ``apply_update_mask_`` — the one-hot update-mask write of ``Gemma3Model._apply_update_mask`` and
  ``_apply_update_mask_batch`` (``anemll/models/gemma3_model.py:932-965``), applied in place.
* ``rotate_append_`` — the rotating sliding-window update of ``_update_kv_local`` (shift by one,
  1024-1066) and ``_update_kv_local_prefill`` (shift by the batch, 1167-1204), in place.
* ``update_kv_local_`` — that update on the reference's split local cache ``kv_cache_local``
  ``[2 * num_local, H_kv, sliding_window, hd]`` (key slot ``i``, value slot ``i + num_local``).
* ``transition_kv_state`` / ``compact_kv_state`` — the KV-state resize between context sizes of
  ``anemll/utils/state_transition.py`` (62-152, 153-357), with the same argument checks and errors.

All tensors are CUDA tensors; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["apply_update_mask_", "rotate_append_", "update_kv_local_", "transition_kv_state", "compact_kv_state"]


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("anemll_b200 ops take CUDA tensors (no CPU path)")


def _slabs(x, L, d):
    """(number of slabs, slab stride) of a tensor whose last two dims are [L, d], rows contiguous."""
    if x.shape[-2] != L or x.shape[-1] != d or x.stride(-1) != 1 or x.stride(-2) != d:
        raise ValueError("the last two dims must be contiguous rows [L, d]")
    lead = x.shape[:-2]
    n = 1
    for s in lead:
        n *= s
    if n == 1:
        return 1, L * d
    # the leading dims must collapse to one uniform stride
    stride = x.stride(-3)
    expect = stride
    for dim in range(x.dim() - 3, -1, -1):
        if x.shape[dim] != 1 and x.stride(dim) != expect:
            raise ValueError("leading dims must collapse into one slab stride")
        expect *= x.shape[dim]
    return n, stride


def apply_update_mask_(cache_slice, new_states, update_mask):
    """Write ``new_states`` into ``cache_slice`` where ``update_mask`` is 1, in place; returns the cache.

    ``cache_slice [..., L, d]``, ``new_states [..., S, d]`` (same leading dims), ``update_mask``
    ``[1, 1, L, S]`` (``S == 1``: the single-token form ``[1, 1, L, 1]``)."""
    _need_cuda(cache_slice, new_states, update_mask)
    L, d = cache_slice.shape[-2], cache_slice.shape[-1]
    S = new_states.shape[-2]
    if new_states.shape[:-2] != cache_slice.shape[:-2] or new_states.shape[-1] != d:
        raise ValueError("new_states must match cache_slice except in the row count")
    if new_states.dtype != cache_slice.dtype:
        raise TypeError("new_states and cache_slice must share a dtype")
    m = update_mask.reshape(update_mask.shape[-2], update_mask.shape[-1])
    if m.shape != (L, S):
        raise ValueError(f"update_mask must be [1, 1, {L}, {S}]")
    if m.stride(-1) != 1:
        m = m.contiguous()
    new = new_states.contiguous()
    n, cs = _slabs(cache_slice, L, d)
    _, ns = _slabs(new, S, d)
    rc = _lib.load().anemll_kv_update_mask(_lib.ptr(cache_slice), _lib.ptr(new), _lib.dtype_code(cache_slice.dtype),
                                           _lib.ptr(m), _lib.dtype_code(m.dtype), m.stride(0), n, L, S, d, cs, ns,
                                           _lib.stream_ptr(cache_slice.device))
    _lib.check(rc, "anemll_kv_update_mask")
    return cache_slice


def rotate_append_(cache_slice, new_states, n=None):
    """Shift every ``[L, d]`` slab of ``cache_slice`` left by ``n`` rows and store ``new_states[..., :n, :]``
    at the end, in place; ``n`` defaults to the number of new rows.  Returns the cache."""
    _need_cuda(cache_slice, new_states)
    L, d = cache_slice.shape[-2], cache_slice.shape[-1]
    n = new_states.shape[-2] if n is None else int(n)
    if new_states.shape[:-2] != cache_slice.shape[:-2] or new_states.shape[-1] != d or new_states.shape[-2] < n:
        raise ValueError("new_states must match cache_slice except in the row count (>= n)")
    if new_states.dtype != cache_slice.dtype:
        raise TypeError("new_states and cache_slice must share a dtype")
    new = new_states.contiguous()
    nslab, cs = _slabs(cache_slice, L, d)
    _, ns = _slabs(new, new.shape[-2], d)
    rc = _lib.load().anemll_kv_rotate_append(_lib.ptr(cache_slice), _lib.ptr(new), _lib.dtype_code(cache_slice.dtype),
                                             nslab, L, n, d, cs, ns, _lib.stream_ptr(cache_slice.device))
    _lib.check(rc, "anemll_kv_rotate_append")
    return cache_slice


def update_kv_local_(kv_cache_local, local_index, num_local, key_states, value_states, shift=None):
    """The reference's rotating update of its split local cache, in place: key slot ``local_index``
    and value slot ``local_index + num_local`` of ``kv_cache_local [2 num_local, H_kv, sw, hd]`` are
    shifted left by ``shift`` (default: the number of new rows) and receive the new rows."""
    rotate_append_(kv_cache_local[local_index:local_index + 1], key_states, shift)
    rotate_append_(kv_cache_local[local_index + num_local:local_index + num_local + 1], value_states, shift)
    return kv_cache_local


def _resize(source_state, target_seq_length, current_position, pad_value, dtype):
    _need_cuda(source_state)
    L, H, S, d = source_state.shape
    out_dtype = dtype if dtype is not None else source_state.dtype
    src = source_state.contiguous()
    out = torch.empty(L, H, target_seq_length, d, dtype=out_dtype, device=source_state.device)
    rc = _lib.load().anemll_kv_state_transition(_lib.ptr(src), _lib.dtype_code(src.dtype), _lib.ptr(out),
                                                _lib.dtype_code(out_dtype), L * H, S, target_seq_length, d,
                                                int(current_position), float(pad_value),
                                                _lib.stream_ptr(source_state.device))
    _lib.check(rc, "anemll_kv_state_transition")
    return out


def transition_kv_state(source_state, target_seq_length, current_position=None, pad_value=0.0, dtype=None):
    """Expand ``source_state [num_layers, num_kv_heads, seq, head_dim]`` to ``target_seq_length``
    rows: rows ``[0, current_position)`` copied (converted to ``dtype``), the rest ``pad_value``."""
    if source_state.dim() != 4:
        raise ValueError(f"Expected 4D state tensor [num_layers, num_kv_heads, seq_length, head_dim], "
                         f"got shape {tuple(source_state.shape)}")
    S = source_state.shape[2]
    if target_seq_length < S:
        raise ValueError(f"Target sequence length ({target_seq_length}) must be >= source sequence length ({S})")
    if current_position is None:
        current_position = S
    elif current_position > S:
        raise ValueError(f"current_position ({current_position}) cannot exceed source sequence length ({S})")
    if target_seq_length == S and current_position == S:
        return source_state
    return _resize(source_state, target_seq_length, current_position, pad_value, dtype)


def compact_kv_state(source_state, target_seq_length, current_position, dtype=None):
    """Shrink ``source_state`` to ``target_seq_length`` rows, keeping rows ``[0, current_position)``
    and zero-filling the rest; ``current_position`` must fit in the target."""
    if source_state.dim() != 4:
        raise ValueError(f"Expected 4D state tensor [num_layers, num_kv_heads, seq_length, head_dim], "
                         f"got shape {tuple(source_state.shape)}")
    S = source_state.shape[2]
    if current_position > target_seq_length:
        raise ValueError(f"Cannot compact: current_position ({current_position}) exceeds target_seq_length "
                         f"({target_seq_length}). The processed tokens won't fit in the smaller state.")
    if current_position > S:
        raise ValueError(f"current_position ({current_position}) cannot exceed source sequence length ({S})")
    return _resize(source_state, target_seq_length, current_position, 0.0, dtype)
