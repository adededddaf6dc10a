"""Fixed-shape KV-cache attention on the sm_100a kernel, behind the reference's signatures.

``kv_attention`` is the fused op (cache write + GQA attention + sigmoid gate).
``QwenAttentionB200`` keeps the method signatures of the reference's
``QwenAttention`` (``anemll/models/qwen_model.py``):
``forward_prefill(hidden_states, query_states, kv_cache_layer, causal_mask)``
(509-546) and ``forward_regular(hidden_states, query_states, kv_cache_layer,
causal_mask, current_pos)`` (469-507), where the caller has already written
the cache (``process_layer_prefill`` 669-675 / ``process_layer_regular``
733-745); ``process_layer_step`` does write + attend in one launch on the
unified cache ``kv_cache_0`` [2L, H_kv, ctx, hd].  Outputs are the attention
output before ``o_proj`` (``o_proj`` stays a torch GEMM in the caller).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib

__all__ = ["kv_attention", "kv_attention_workspace_size", "kv_device_error", "unified_cache_layer",
           "QwenAttentionB200"]

_ws_cache: dict = {}


def kv_attention_workspace_size(B, S, H_q, H_kv, head_dim, ctx) -> int:
    return int(_lib.load().anemll_kv_attention_workspace_size(B, S, H_q, H_kv, head_dim, ctx))


def kv_device_error(reset=True) -> int:
    """Non-zero if a TMA-fed KV launch stopped on a bounded wait (synchronous)."""
    return int(_lib.load().anemll_kv_attention_error(int(bool(reset))))


def _workspace(device, nbytes):
    """Per-device scratch, grown on demand and reused (ops never free it)."""
    if nbytes == 0:
        return None
    key = torch.device(device)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def unified_cache_layer(kv_cache, layer_idx, num_layers):
    """K and V views of one layer of the unified cache (``get_kv_cache_idx``, qwen_model.py:88-93)."""
    return kv_cache[layer_idx], kv_cache[layer_idx + num_layers]


def kv_attention(query_states, k_cache, v_cache, current_pos, k_new=None, v_new=None, gate=None,
                 causal_mask=None, window=0, window_chunk_aligned=False, out=None, workspace=None):
    """One prefill chunk or decode step.

    ``query_states`` [B,H_q,S,hd]; ``k_cache, v_cache`` [H_kv,ctx,hd] (reference
    layout, B=1) or [B,H_kv,ctx,hd] (unit stride on the last two dims);
    ``k_new, v_new`` [B,H_kv,S,hd] written at ``[current_pos, current_pos+S)``
    (``None``: already written); ``gate`` [B,S,H_q*hd] sigmoid pre-activation;
    ``causal_mask``: the reference's additive mask [1,1,>=S,>=ctx] — when given it
    decides visibility, otherwise causal / sliding ``window`` from positions.
    Returns ``[B, S, H_q*hd]``.
    """
    q = query_states
    for t in (q, k_cache, v_cache, k_new, v_new, gate, causal_mask):
        if t is not None and not t.is_cuda:
            raise RuntimeError("anemll_b200 ops take CUDA tensors (no CPU path)")
    if not q.is_contiguous():
        q = q.contiguous()
    B, Hq, S, hd = q.shape
    if k_cache.dim() == 3:
        k_cache = k_cache.unsqueeze(0)
        v_cache = v_cache.unsqueeze(0)
    if k_cache.shape != v_cache.shape or k_cache.shape[0] not in (1, B):
        raise ValueError("k_cache / v_cache shape mismatch")
    _, Hkv, ctx, hd2 = k_cache.shape
    if hd2 != hd:
        raise ValueError("head_dim mismatch between query and cache")
    if k_cache.stride(-1) != 1 or k_cache.stride(-2) != hd or v_cache.stride() != k_cache.stride():
        raise ValueError("cache rows must be contiguous [.., ctx, hd] with equal K/V strides")
    bstride = k_cache.stride(0) if k_cache.shape[0] == B and B > 1 else 0
    dt = q.dtype
    for t in (k_new, v_new, gate):
        if t is not None and t.dtype != dt:
            raise TypeError("query, k_new, v_new and gate must share a dtype")
    if k_cache.dtype != dt:
        raise TypeError("cache dtype must match the query dtype")
    if k_new is not None:
        if k_cache.shape[0] != B:
            raise ValueError("writing new rows needs one cache per sequence (cache batch == query batch)")
        k_new = k_new.contiguous()
        v_new = v_new.contiguous()
        if tuple(k_new.shape) != (B, Hkv, S, hd) or k_new.shape != v_new.shape:
            raise ValueError("k_new / v_new must be [B, H_kv, S, hd]")
    if gate is not None:
        gate = gate.contiguous()
    mask = None
    mask_dt, mask_ld = 0, 0
    if causal_mask is not None:
        m = causal_mask
        while m.dim() > 2:
            m = m[0]
        m = m[:S]
        if m.stride(-1) != 1:
            m = m.contiguous()
        mask = m
        mask_dt = _lib.dtype_code(m.dtype)
        mask_ld = m.stride(0)
        if m.shape[1] < ctx or m.shape[0] < S:
            raise ValueError("causal_mask must cover [S, ctx]")
    if out is None:
        out = torch.empty(B, S, Hq * hd, dtype=dt, device=q.device)
    need = kv_attention_workspace_size(B, S, Hq, Hkv, hd, ctx)
    if workspace is None:
        workspace = _workspace(q.device, need)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = _lib.load().anemll_kv_attention(
        _lib.ptr(q), _lib.ptr(k_new), _lib.ptr(v_new), _lib.ptr(gate), _lib.ptr(k_cache), _lib.ptr(v_cache),
        bstride, k_cache.stride(1), _lib.ptr(mask), mask_dt, mask_ld, _lib.ptr(out), _lib.dtype_code(dt),
        B, S, Hq, Hkv, hd, ctx, int(current_pos), int(window), int(bool(window_chunk_aligned)),
        _lib.ptr(workspace), ws_bytes, _lib.stream_ptr(q.device))
    _lib.check(rc, "anemll_kv_attention")
    return out


def kv_attention_qkv(qkv, q_norm, k_norm, cos, sin, eps, k_cache, v_cache, current_pos, H_q, H_kv, head_dim,
                     window=0, window_chunk_aligned=False, out=None, workspace=None):
    """One attention call with the layer's prologue fused in (``anemll_kv_attention_qkv``).

    ``qkv`` [B, S, H_q*2*hd + 2*H_kv*hd] is the fused projection output (per head ``[query | gate]``,
    then k, then v; rows may be spaced by a stride); ``q_norm``/``k_norm`` fp32 [hd]; ``cos``/``sin``
    fp32 [>= pos+S, hd].  The new K/V rows are written into ``k_cache``/``v_cache`` [B, H_kv, ctx, hd].
    Returns the gated output [B, S, H_q*hd], or None when the shape needs the separate
    ``anemll_qk_norm_rope`` kernel (see the C ABI)."""
    for t in (qkv, q_norm, k_norm, cos, sin, k_cache, v_cache):
        if not t.is_cuda:
            raise RuntimeError("anemll_b200 ops take CUDA tensors (no CPU path)")
    B, S, width = qkv.shape
    if qkv.stride(-1) != 1 or (S > 1 and B > 1 and qkv.stride(0) != qkv.stride(1) * S):
        raise ValueError("qkv rows must be dense with a uniform token stride")
    ld = qkv.stride(1) if S > 1 else (qkv.stride(0) if B > 1 else width)
    if k_cache.dim() == 3:
        k_cache, v_cache = k_cache.unsqueeze(0), v_cache.unsqueeze(0)
    _, Hkv2, ctx, hd2 = k_cache.shape
    if Hkv2 != H_kv or hd2 != head_dim or k_cache.stride() != v_cache.stride():
        raise ValueError("cache shape does not match the head configuration")
    bstride = k_cache.stride(0) if k_cache.shape[0] == B and B > 1 else 0
    if out is None:
        out = torch.empty(B, S, H_q * head_dim, dtype=qkv.dtype, device=qkv.device)
    need = kv_attention_workspace_size(B, S, H_q, H_kv, head_dim, ctx)
    if workspace is None:
        workspace = _workspace(qkv.device, need)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = _lib.load().anemll_kv_attention_qkv(
        qkv.data_ptr(), ld, _lib.ptr(q_norm), _lib.ptr(k_norm), _lib.ptr(cos), _lib.ptr(sin), float(eps),
        _lib.ptr(k_cache), _lib.ptr(v_cache), bstride, k_cache.stride(1), _lib.ptr(out), _lib.dtype_code(qkv.dtype),
        B, S, H_q, H_kv, head_dim, ctx, int(current_pos), int(window), int(bool(window_chunk_aligned)),
        _lib.ptr(workspace), ws_bytes, _lib.stream_ptr(qkv.device))
    if rc == _lib.EUNSUPPORTED:
        return None
    _lib.check(rc, "anemll_kv_attention_qkv")
    return out


class QwenAttentionB200(nn.Module):
    """The attention core of ``QwenAttention`` with the reference's method signatures.

    Holds no weights: projections, q/k norms and RoPE (``get_new_kv_cache*``,
    qwen_model.py:362-415) and ``o_proj`` stay torch GEMMs in the caller, so the
    methods return the attention output before ``o_proj`` ([B, S, H_q*hd]).
    ``window`` > 0 selects the sliding-window rule when no mask is given.
    """

    def __init__(self, num_heads, num_kv_heads, head_dim, window=0, window_chunk_aligned=False):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.window, self.window_chunk_aligned = window, window_chunk_aligned

    def forward_prefill(self, hidden_states, query_states, kv_cache_layer=None, causal_mask=None, gate=None,
                        current_pos=0):
        K, V = kv_cache_layer
        return kv_attention(query_states, K, V, current_pos, gate=gate, causal_mask=causal_mask,
                            window=self.window, window_chunk_aligned=self.window_chunk_aligned)

    def forward_regular(self, hidden_states, query_states, kv_cache_layer=None, causal_mask=None, current_pos=None,
                        gate=None):
        K, V = kv_cache_layer
        pos = int(current_pos) if current_pos is not None else 0
        return kv_attention(query_states, K, V, pos, gate=gate, causal_mask=causal_mask, window=self.window,
                            window_chunk_aligned=self.window_chunk_aligned)

    def process_layer_step(self, kv_cache, layer_idx, num_layers, query_states, key_states, value_states,
                           current_pos, gate=None, causal_mask=None):
        """Fused cache write + attention on the unified cache (one launch)."""
        K, V = unified_cache_layer(kv_cache, layer_idx, num_layers)
        return kv_attention(query_states, K, V, int(current_pos), k_new=key_states, v_new=value_states, gate=gate,
                            causal_mask=causal_mask, window=self.window,
                            window_chunk_aligned=self.window_chunk_aligned)
