"""Fixed-shape KV-cache attention on the sm_100a kernel, behind the reference's signatures.

``kv_attention`` is the fused op (cache write + GQA attention + sigmoid gate).
``QwenAttentionB200`` keeps the method signatures and results of the
reference's ``QwenAttention`` (``anemll/models/qwen_model.py``):
``forward_prefill(hidden_states, query_states, kv_cache_layer, causal_mask)``
(509-546) and ``forward_regular(hidden_states, query_states, kv_cache_layer,
causal_mask, current_pos)`` (469-507), where the caller has already written
the cache (``process_layer_prefill`` 669-675 / ``process_layer_regular``
733-745), both ending in ``o_proj`` (a torch GEMM on the kernel's output);
``process_layer_step`` does write + attend in one launch on the unified cache
``kv_cache_0`` [2L, H_kv, ctx, hd].
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

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
    """``QwenAttention``'s attention methods with the reference's signatures and results.

    ``forward_prefill(hidden_states, query_states, kv_cache_layer, causal_mask)``
    (qwen_model.py:509-546) and ``forward_regular(hidden_states, query_states,
    kv_cache_layer, causal_mask, current_pos)`` (469-507) attend over the
    caller's fixed-shape cache (``kv_cache_layer`` = (K [H_kv, ctx, hd],
    V [H_kv, ctx, hd]), already written by ``process_layer_*``, 669-675 /
    733-745) and end in ``o_proj``, so they return what the reference returns:
    [B, S, hidden].  ``o_proj`` is the reference's 1x1 ``Conv2d``
    ([hidden, H_q*hd, 1, 1] weight), an ``nn.Linear``, or a weight tensor of
    either shape; it runs as a torch GEMM on the kernel's output.
    ``from_reference(attn)`` shares a reference module's ``o_proj``.  Without
    ``o_proj`` the projection is the identity.  ``attention(...)`` is the
    pre-projection core ([B, S, H_q*hd]).  ``window`` > 0 selects the
    sliding-window rule when no mask is given; ``gate`` (optional) is the
    sigmoid output gate's pre-activation [B, S, H_q*hd].
    """

    def __init__(self, num_heads, num_kv_heads, head_dim, window=0, window_chunk_aligned=False, o_proj=None):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.window, self.window_chunk_aligned = window, window_chunk_aligned
        self.o_proj = o_proj
        self._w = None  # o_proj weight as [hidden, H_q*hd] in the activation dtype (cached)

    @classmethod
    def from_reference(cls, attn, window=0, window_chunk_aligned=False):
        """Wrap a reference ``QwenAttention`` (its head shape and its ``o_proj`` module)."""
        return cls(attn.num_heads, attn.num_kv_heads, attn.head_dim, window, window_chunk_aligned, attn.o_proj)

    def _proj_weight(self, dtype, device):
        p = self.o_proj
        w = p if isinstance(p, torch.Tensor) else p.weight
        qd = self.num_heads * self.head_dim
        if w.dim() == 4:
            if tuple(w.shape[1:]) != (qd, 1, 1):
                raise ValueError(f"o_proj Conv2d weight must be [hidden, {qd}, 1, 1]")
            w = w.reshape(w.shape[0], qd)
        if w.dim() != 2 or w.shape[1] != qd:
            raise ValueError(f"o_proj weight must be [hidden, {qd}]")
        c = self._w
        if c is None or c[0] is not w or c[1].dtype != dtype or c[1].device != device:
            self._w = c = (w, w.detach().to(device=device, dtype=dtype).contiguous())
        return c[1]

    def project(self, attn_output):
        """``o_proj`` of the attention output [B, S, H_q*hd] (identity without one)."""
        if self.o_proj is None:
            return attn_output
        bias = getattr(self.o_proj, "bias", None)
        return F.linear(attn_output, self._proj_weight(attn_output.dtype, attn_output.device),
                        None if bias is None else bias.to(attn_output.dtype))

    def attention(self, query_states, kv_cache_layer, causal_mask=None, current_pos=0, gate=None):
        K, V = kv_cache_layer
        return kv_attention(query_states, K, V, _position(current_pos), gate=gate, causal_mask=causal_mask,
                            window=self.window, window_chunk_aligned=self.window_chunk_aligned)

    def forward_prefill(self, hidden_states, query_states, kv_cache_layer=None, causal_mask=None, gate=None,
                        current_pos=0):
        return self.project(self.attention(query_states, kv_cache_layer, causal_mask, current_pos, gate))

    def forward_regular(self, hidden_states, query_states, kv_cache_layer=None, causal_mask=None, current_pos=None,
                        gate=None):
        return self.project(self.attention(query_states, kv_cache_layer, causal_mask,
                                           0 if current_pos is None else current_pos, gate))

    def process_layer_step(self, kv_cache, layer_idx, num_layers, query_states, key_states, value_states,
                           current_pos, gate=None, causal_mask=None):
        """Fused cache write + attention on the unified cache (one launch), then ``o_proj``."""
        K, V = unified_cache_layer(kv_cache, layer_idx, num_layers)
        return self.project(kv_attention(query_states, K, V, _position(current_pos), k_new=key_states,
                                         v_new=value_states, gate=gate, causal_mask=causal_mask, window=self.window,
                                         window_chunk_aligned=self.window_chunk_aligned))


def _position(current_pos) -> int:
    """``current_pos`` as an int: the reference passes positions as one-element int tensors."""
    if isinstance(current_pos, torch.Tensor):
        if current_pos.numel() != 1:
            raise ValueError("current_pos must hold one position")
        return int(current_pos.reshape(()).item())
    return int(current_pos)
