"""CPU oracle: Qwen3.5 gated delta-rule (GDN) layer — TEST INFRASTRUCTURE ONLY.

Restated from the mathematics, not from any implementation.  Per sequence
``b`` and value head ``h`` the layer keeps a state ``S`` of shape
``[d_k, d_v]`` and, for every token with key ``k``, query ``q`` (both
l2-normalised, ``q`` scaled by ``1/sqrt(d_k)``), value ``v``, write strength
``beta`` and log-decay ``g``::

    S   <- exp(g) * S
    d    = beta * (v - S^T k)
    S   <- S + k d^T
    o    = S^T q

Argument meaning, the l2-norm epsilon, the gate formula and the conv-state
layout follow the third-party ``transformers==5.5.0`` module
``transformers/models/qwen3_5/modeling_qwen3_5.py`` (line numbers cited per
function).  Value head ``j`` reads key head ``j // (H_v / H_qk)``, the same
pairing as ``repeat_interleave`` at ``modeling_qwen3_5.py:495-496``.

Tensor layouts are token-major, as in that module: ``q, k`` are
``[B, T, H_qk, d_k]``, ``v`` is ``[B, T, H_v, d_v]``, ``g`` and ``beta`` are
``[B, T, H_v]``, the recurrent state is ``[B, H_v, d_k, d_v]``.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

__all__ = [
    "l2norm",
    "gates",
    "causal_conv1d_prefill",
    "causal_conv1d_update",
    "prologue",
    "recurrent_gated_delta_rule",
    "chunk_gated_delta_rule",
    "gated_rmsnorm",
    "gdn_layer_prefill",
    "gdn_layer_decode",
]


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``x * rsqrt(sum(x^2) + eps)`` over the last dim (``modeling_qwen3_5.py:228-231``)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor | None):
    """``beta = sigmoid(b)``, ``g = -exp(A_log) * softplus(a + dt_bias)``.

    ``modeling_qwen3_5.py:491-493``.  ``a, b`` are ``[B, T, H_v]``.
    """
    a = a.float()
    if dt_bias is not None:
        a = a + dt_bias.float()
    beta = torch.sigmoid(b.float())
    g = -torch.exp(A_log.float()) * F.softplus(a)
    return g, beta


def causal_conv1d_prefill(x: torch.Tensor, weight: torch.Tensor, conv_state: torch.Tensor | None):
    """Depthwise causal conv over time + SiLU, with optional history.

    ``x`` is ``[B, T, C]`` (token-major), ``weight`` is ``[C, K]``,
    ``conv_state`` (optional, ``[B, C, K]``) holds the last ``K`` raw inputs
    before this call, newest at index ``K-1``; zeros when absent (the prefill
    path of ``modeling_qwen3_5.py:463-474`` starts from zero history).
    Returns ``(y [B, T, C], new_conv_state [B, C, K])`` where the new state
    is the last ``K`` columns of ``cat(history, x)``
    (``modeling_qwen3_5.py:217-218``).
    """
    B, T, C = x.shape
    K = weight.shape[1]
    xt = x.float().transpose(1, 2)  # [B, C, T]
    if conv_state is None:
        hist = torch.zeros(B, C, K, dtype=xt.dtype)
    else:
        hist = conv_state.float()
    full = torch.cat([hist, xt], dim=-1)  # [B, C, K+T]
    w = weight.float()
    # y[t] = sum_j w[j] * full[t + 1 + j]   (taps on the K most recent inputs)
    y = torch.zeros(B, C, T, dtype=xt.dtype)
    for j in range(K):
        y += w[:, j].view(1, C, 1) * full[:, :, 1 + j: 1 + j + T]
    y = F.silu(y)
    new_state = full[:, :, -K:].clone()
    return y.transpose(1, 2).contiguous(), new_state


def causal_conv1d_update(x: torch.Tensor, weight: torch.Tensor, conv_state: torch.Tensor):
    """Decode form of :func:`causal_conv1d_prefill` (``modeling_qwen3_5.py:210-226``)."""
    return causal_conv1d_prefill(x, weight, conv_state)


def prologue(mixed_qkv, a, b, conv_w, A_log, dt_bias, conv_state, H_qk, H_v, d_k, d_v):
    """conv1d+SiLU, split into q/k/v, l2-normalise q/k, gates.

    ``mixed_qkv`` is the raw ``in_proj_qkv`` output ``[B, T, 2*H_qk*d_k + H_v*d_v]``.
    Returns ``q, k [B,T,H_qk,d_k]`` (l2-normalised, unscaled), ``v [B,T,H_v,d_v]``,
    ``g, beta [B,T,H_v]``, new conv state.  Follows ``modeling_qwen3_5.py:453-496``
    with the l2-norm that the core applies in-kernel moved here.
    """
    B, T, _ = mixed_qkv.shape
    y, new_state = causal_conv1d_prefill(mixed_qkv, conv_w, conv_state)
    kd = H_qk * d_k
    q = y[..., :kd].reshape(B, T, H_qk, d_k)
    k = y[..., kd:2 * kd].reshape(B, T, H_qk, d_k)
    v = y[..., 2 * kd:].reshape(B, T, H_v, d_v)
    q = l2norm(q)
    k = l2norm(k)
    g, beta = gates(a, b, A_log, dt_bias)
    return q, k, v, g, beta, new_state


def _expand_heads(x: torch.Tensor, H_v: int) -> torch.Tensor:
    """``[B,T,H_qk,d] -> [B,T,H_v,d]``: value head j reads key head j // (H_v/H_qk)."""
    rep = H_v // x.shape[2]
    return x.repeat_interleave(rep, dim=2) if rep > 1 else x


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, scale=None,
                               use_qk_l2norm=False, dtype=torch.float32):
    """Token-by-token delta rule (``modeling_qwen3_5.py:314-353`` semantics).

    Returns ``(o [B,T,H_v,d_v], final_state [B,H_v,d_k,d_v])`` in ``dtype``.
    """
    B, T, H_v, d_v = v.shape
    d_k = q.shape[-1]
    q = q.to(dtype)
    k = k.to(dtype)
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    q = _expand_heads(q, H_v) * (scale if scale is not None else 1.0 / math.sqrt(d_k))
    k = _expand_heads(k, H_v)
    v = v.to(dtype)
    g = g.to(dtype)
    beta = beta.to(dtype)
    S = (torch.zeros(B, H_v, d_k, d_v, dtype=dtype) if initial_state is None
         else initial_state.to(dtype).clone())
    out = torch.empty(B, T, H_v, d_v, dtype=dtype)
    for t in range(T):
        S = S * torch.exp(g[:, t]).view(B, H_v, 1, 1)
        kt = k[:, t]  # [B,H,dk]
        pred = torch.einsum("bhkv,bhk->bhv", S, kt)
        d = beta[:, t].unsqueeze(-1) * (v[:, t] - pred)
        S = S + kt.unsqueeze(-1) * d.unsqueeze(-2)
        out[:, t] = torch.einsum("bhkv,bhk->bhv", S, q[:, t])
    return out, S


def chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=None, scale=None,
                           use_qk_l2norm=False, dtype=torch.float32):
    """Chunkwise (WY / UT) form of the same recurrence.

    Within a chunk of ``c <= chunk_size`` tokens, with ``G`` the in-chunk
    cumulative sum of ``g`` and ``Gam[i,j] = exp(G_i - G_j)``::

        L   = strict_lower(diag(beta) (K K^T * Gam))
        D   = (I + L)^-1 (diag(beta) V - diag(beta e^G) K S0)      # per-token deltas
        O   = diag(e^G) Q S0 + lower_incl_diag(Q K^T * Gam) D
        S1  = e^{G_c} S0 + K^T diag(e^{G_c - G}) D

    The unit-lower-triangular system is solved with
    ``torch.linalg.solve_triangular``.  A ragged last chunk is just a shorter
    chunk, which equals the zero padding of ``modeling_qwen3_5.py:247-254``.
    """
    B, T, H_v, d_v = v.shape
    d_k = q.shape[-1]
    q = q.to(dtype)
    k = k.to(dtype)
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    q = _expand_heads(q, H_v) * (scale if scale is not None else 1.0 / math.sqrt(d_k))
    k = _expand_heads(k, H_v)
    # [B,H,T,d]
    q = q.transpose(1, 2)
    k = k.transpose(1, 2)
    v = v.to(dtype).transpose(1, 2)
    g = g.to(dtype).transpose(1, 2)
    beta = beta.to(dtype).transpose(1, 2)
    S = (torch.zeros(B, H_v, d_k, d_v, dtype=dtype) if initial_state is None
         else initial_state.to(dtype).clone())
    out = torch.empty(B, H_v, T, d_v, dtype=dtype)
    for s in range(0, T, chunk_size):
        e = min(T, s + chunk_size)
        c = e - s
        Q, Kc, V = q[:, :, s:e], k[:, :, s:e], v[:, :, s:e]
        bt = beta[:, :, s:e]
        G = torch.cumsum(g[:, :, s:e], dim=-1)  # [B,H,c]
        diff = G.unsqueeze(-1) - G.unsqueeze(-2)  # [B,H,c,c]  G_i - G_j
        lower_incl = torch.tril(torch.ones(c, c, dtype=torch.bool))
        strict = torch.tril(torch.ones(c, c, dtype=torch.bool), diagonal=-1)
        Gam = torch.where(lower_incl, torch.exp(torch.where(lower_incl, diff, torch.zeros_like(diff))),
                          torch.zeros_like(diff))
        KK = Kc @ Kc.transpose(-1, -2)
        L = torch.where(strict, bt.unsqueeze(-1) * KK * Gam, torch.zeros_like(KK))
        I = torch.eye(c, dtype=dtype).expand_as(L)
        eG = torch.exp(G).unsqueeze(-1)
        rhs = bt.unsqueeze(-1) * V - (bt.unsqueeze(-1) * eG * Kc) @ S
        D = torch.linalg.solve_triangular(I + L, rhs, upper=False, unitriangular=True)
        QK = torch.where(lower_incl, (Q @ Kc.transpose(-1, -2)) * Gam, torch.zeros_like(KK))
        out[:, :, s:e] = eG * (Q @ S) + QK @ D
        Gl = G[..., -1:]  # [B,H,1]
        S = torch.exp(Gl).unsqueeze(-1) * S + (Kc * torch.exp(Gl - G).unsqueeze(-1)).transpose(-1, -2) @ D
    return out.transpose(1, 2).contiguous(), S


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """``weight * x * rsqrt(mean(x^2) + eps) * silu(z)`` over the last dim.

    ``modeling_qwen3_5.py:175-190`` (norm before gate), in fp32.
    """
    x = x.float()
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return weight.float() * y * F.silu(z.float())


def gdn_layer_prefill(mixed_qkv, z, a, b, params, H_qk, H_v, d_k, d_v, chunk_size=64,
                      conv_state=None, recurrent_state=None, dtype=torch.float32):
    """GDN layer between the input and output projections, prefill form.

    ``mixed_qkv, z, a, b`` are the projection outputs (the hot path's
    inputs).  ``params``: ``conv_w [C,K]``, ``A_log [H_v]``, ``dt_bias [H_v]`` or
    ``None``, ``norm_w [d_v]``, ``eps``.  Returns ``(core_out [B,T,H_v,d_v],
    normed [B,T,H_v,d_v], new_conv_state, final_state)``.
    """
    q, k, v, g, beta, new_conv = prologue(mixed_qkv, a, b, params["conv_w"], params["A_log"],
                                          params.get("dt_bias"), conv_state, H_qk, H_v, d_k, d_v)
    o, S = chunk_gated_delta_rule(q, k, v, g, beta, chunk_size, recurrent_state, dtype=dtype)
    B, T = o.shape[:2]
    normed = gated_rmsnorm(o, z.reshape(B, T, H_v, d_v), params["norm_w"], params.get("eps", 1e-6))
    return o, normed, new_conv, S


def gdn_layer_decode(mixed_qkv, z, a, b, params, H_qk, H_v, d_k, d_v,
                     conv_state, recurrent_state, dtype=torch.float32):
    """Single-token (or few-token) decode form of :func:`gdn_layer_prefill`."""
    q, k, v, g, beta, new_conv = prologue(mixed_qkv, a, b, params["conv_w"], params["A_log"],
                                          params.get("dt_bias"), conv_state, H_qk, H_v, d_k, d_v)
    o, S = recurrent_gated_delta_rule(q, k, v, g, beta, recurrent_state, dtype=dtype)
    B, T = o.shape[:2]
    normed = gated_rmsnorm(o, z.reshape(B, T, H_v, d_v), params["norm_w"], params.get("eps", 1e-6))
    return o, normed, new_conv, S
