"""CPU oracle: fixed-shape KV-cache softmax attention — TEST INFRASTRUCTURE ONLY.

Restates, in fp32 (or fp64), what the reference computes in
``anemll/models/qwen_model.py``:

* cache write (``process_layer_prefill`` 669-675, ``process_layer_regular``
  733-745): the unified cache ``kv_cache_0`` is ``[2L, H_kv, ctx, hd]``; layer
  ``l`` keeps K at index ``l`` and V at index ``l + L`` (``get_kv_cache_idx``
  88-93); new rows land at ``[pos, pos + S)``;
* attention (``forward_prefill`` 509-546 / ``forward_regular`` 469-507):
  query head ``h`` reads kv head ``h // (H_q / H_kv)`` (``repeat_kv``
  351-360), scores are ``q k^T / sqrt(hd)`` plus an additive mask over the
  full fixed cache width, softmax over keys, times V;
* masks: causal (``tests/chat.py`` ``make_causal_mask`` 977-983: key ``j`` is
  visible to the query at absolute position ``p`` iff ``j <= p``) and the
  sliding window of ``anemll/models/gemma3_model.py`` ``_kv_slice`` 906-926
  (additionally ``j > p - W``);
* the Qwen3.5 sigmoid output gate (third-party ``transformers==5.5.0``
  ``modeling_qwen3_5.py:632-689``): ``out * sigmoid(gate)`` before ``o_proj``.

The hot path's output is the gated attention output ``[B, S, H_q*hd]``, i.e.
everything before ``o_proj``.  A batch dimension is added for the multi-
sequence stack; ``B = 1`` is exactly the reference's layout.
"""
from __future__ import annotations

import math

import torch

__all__ = ["visibility_mask", "additive_mask", "write_cache", "attend", "kv_attention_step"]


def visibility_mask(S: int, ctx: int, pos: int, window: int = 0, chunk_aligned: bool = False) -> torch.Tensor:
    """Boolean ``[S, ctx]``: True where key ``j`` is visible to query ``i`` at position ``pos+i``.

    Causal: ``j <= pos+i``.  Sliding window ``W > 0``: per query ``j > pos+i-W``;
    with ``chunk_aligned`` the whole chunk shares the start
    ``max(0, min(pos+S, ctx) - W)`` (``gemma3_model.py:923-926``).
    """
    p = pos + torch.arange(S).unsqueeze(1)
    j = torch.arange(ctx).unsqueeze(0)
    vis = j <= p
    if window > 0:
        if chunk_aligned:
            vis &= j >= max(0, min(pos + S, ctx) - window)
        else:
            vis &= j > p - window
    return vis


def additive_mask(S: int, ctx: int, pos: int, window: int = 0, dtype=torch.float32,
                  chunk_aligned: bool = False) -> torch.Tensor:
    """The reference's additive mask ``[1, 1, S, ctx]``: 0 where visible, -inf elsewhere."""
    vis = visibility_mask(S, ctx, pos, window, chunk_aligned)
    m = torch.zeros(S, ctx, dtype=dtype)
    m.masked_fill_(~vis, float("-inf"))
    return m.view(1, 1, S, ctx)


def write_cache(kv_cache: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                layer_idx: int, num_layers: int, pos: int) -> None:
    """In-place cache write.  ``kv_cache`` is ``[2L, H_kv, ctx, hd]`` (reference
    layout) or ``[2L, B, H_kv, ctx, hd]``; ``k_new, v_new`` are ``[B, H_kv, S, hd]``."""
    S = k_new.shape[2]
    if kv_cache.dim() == 4:
        kv_cache[layer_idx, :, pos:pos + S, :] = k_new[0].to(kv_cache.dtype)
        kv_cache[layer_idx + num_layers, :, pos:pos + S, :] = v_new[0].to(kv_cache.dtype)
    else:
        kv_cache[layer_idx, :, :, pos:pos + S, :] = k_new.to(kv_cache.dtype)
        kv_cache[layer_idx + num_layers, :, :, pos:pos + S, :] = v_new.to(kv_cache.dtype)


def attend(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, mask: torch.Tensor | None,
           gate: torch.Tensor | None = None, dtype=torch.float32) -> torch.Tensor:
    """``q [B,H_q,S,hd]``, ``K, V [B,H_kv,ctx,hd]``, additive ``mask [.., S, ctx]``,
    ``gate [B,S,H_q*hd]`` pre-activation.  Returns ``[B, S, H_q*hd]``."""
    B, Hq, S, hd = q.shape
    Hkv = K.shape[1]
    rep = Hq // Hkv
    q = q.to(dtype)
    Kr = K.to(dtype).repeat_interleave(rep, dim=1)
    Vr = V.to(dtype).repeat_interleave(rep, dim=1)
    scores = torch.einsum("bhqd,bhkd->bhqk", q, Kr) * (1.0 / math.sqrt(hd))
    if mask is not None:
        scores = scores + mask.to(dtype)[..., :S, :K.shape[2]]
    p = torch.softmax(scores, dim=-1)
    o = torch.einsum("bhqk,bhkd->bhqd", p, Vr)
    o = o.transpose(1, 2).reshape(B, S, Hq * hd)
    if gate is not None:
        o = o * torch.sigmoid(gate.to(dtype))
    return o


def kv_attention_step(q, k_new, v_new, gate, kv_cache, layer_idx, num_layers, pos, window=0,
                      mask=None, dtype=torch.float32, chunk_aligned=False):
    """One prefill chunk (``S > 1``) or decode step (``S == 1``): write the cache
    in place, then attend over the full fixed cache width.

    ``mask``: explicit additive mask ``[1,1,S,ctx]``; when ``None`` the causal
    (``window == 0``) or sliding-window mask is built from ``pos``.
    """
    write_cache(kv_cache, k_new, v_new, layer_idx, num_layers, pos)
    if kv_cache.dim() == 4:
        K = kv_cache[layer_idx].unsqueeze(0)
        V = kv_cache[layer_idx + num_layers].unsqueeze(0)
    else:
        K = kv_cache[layer_idx]
        V = kv_cache[layer_idx + num_layers]
    S = q.shape[2]
    ctx = K.shape[2]
    if mask is None:
        mask = additive_mask(S, ctx, pos, window, dtype, chunk_aligned)
    return attend(q, K, V, mask, gate, dtype)
