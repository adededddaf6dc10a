"""Gated delta-rule (GDN) ops and the drop-in layer, on the sm_100a kernels.

Functional ops mirror the third-party interface the Qwen3.5 layer calls
(transformers 5.5.0 ``modeling_qwen3_5.py``; the reference snapshot has no GDN
code): ``recurrent_gated_delta_rule`` (314-353), ``causal_conv1d_update`` +
gates (210-226, 453-496) and ``Qwen3_5RMSNormGated`` (175-190), with the
same argument names and meaning.  Differences, all deliberate:

* ``query``/``key`` may stay at ``H_qk`` heads (value head ``j`` reads key
  head ``j // (H_v/H_qk)``), so the ``repeat_interleave`` copy of
  ``modeling_qwen3_5.py:495-496`` is never materialised;
* the ``*_`` variants update ``state`` in place (the caller owns it, like the
  reference's mutable cache buffers); the plain variants clone first and
  return the final state, as the third-party functions do.

Every op runs a CUDA kernel from ``libanemll_b200.so``; there is no CPU path.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib

__all__ = [
    "recurrent_gated_delta_rule",
    "recurrent_gated_delta_rule_",
    "chunk_gated_delta_rule",
    "chunk_gated_delta_rule_",
    "gated_delta_rule_norm_",
    "chunked_device_error",
    "gdn_prologue",
    "gated_rmsnorm",
    "GatedDeltaNet",
]


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("anemll_b200 ops take CUDA tensors (no CPU path)")


def _need_contig(name, t):
    if t is not None and not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def recurrent_gated_delta_rule_(query, key, value, g, beta, state, scale=None,
                                use_qk_l2norm_in_kernel=False, out=None, out_dtype=None):
    """Token-by-token delta rule, updating ``state`` [B,H_v,d_k,d_v] fp32 in place.

    ``query, key`` [B,T,H_qk,d_k]; ``value`` [B,T,H_v,d_v]; ``g, beta`` [B,T,H_v] fp32.
    Returns ``out`` [B,T,H_v,d_v] (dtype ``out_dtype``, default ``query.dtype``).
    """
    _need_cuda(query, key, value, g, beta, state)
    for n, t in (("query", query), ("key", key), ("value", value), ("g", g), ("beta", beta), ("state", state)):
        _need_contig(n, t)
    if g.dtype != torch.float32 or beta.dtype != torch.float32 or state.dtype != torch.float32:
        raise TypeError("g, beta and state must be float32")
    if query.dtype != key.dtype or key.dtype != value.dtype:
        raise TypeError("query, key and value must share a dtype")
    B, T, H_qk, d_k = query.shape
    H_v, d_v = value.shape[2], value.shape[3]
    if key.shape != query.shape or value.shape[:2] != (B, T) or tuple(state.shape) != (B, H_v, d_k, d_v):
        raise ValueError("shape mismatch between query/key/value/state")
    if tuple(g.shape) != (B, T, H_v) or tuple(beta.shape) != (B, T, H_v):
        raise ValueError("g and beta must be [B, T, H_v]")
    out_dtype = out_dtype or query.dtype
    if out is None:
        out = torch.empty(B, T, H_v, d_v, dtype=out_dtype, device=query.device)
    rc = _lib.load().anemll_gdn_recurrent(
        _lib.ptr(query), _lib.ptr(key), _lib.ptr(value), _lib.dtype_code(query.dtype), _lib.ptr(g), _lib.ptr(beta),
        _lib.ptr(state), _lib.ptr(out), _lib.dtype_code(out.dtype), B, T, H_qk, H_v, d_k, d_v,
        float(scale) if scale is not None else 0.0, int(bool(use_qk_l2norm_in_kernel)), _lib.stream_ptr(query.device))
    _lib.check(rc, "anemll_gdn_recurrent")
    return out


def recurrent_gated_delta_rule(query, key, value, g, beta, initial_state=None, output_final_state=False,
                               use_qk_l2norm_in_kernel=False, scale=None):
    """Functional form with the third-party signature; returns ``(out, final_state or None)``."""
    B, T, _, d_k = query.shape
    H_v, d_v = value.shape[2], value.shape[3]
    if initial_state is None:
        state = torch.zeros(B, H_v, d_k, d_v, dtype=torch.float32, device=query.device)
    else:
        state = initial_state.to(torch.float32).clone()
    out = recurrent_gated_delta_rule_(query, key, value, g.float().contiguous(), beta.float().contiguous(), state,
                                      scale, use_qk_l2norm_in_kernel)
    return out, (state if output_final_state else None)


def chunk_gated_delta_rule_(query, key, value, g, beta, state, scale=None, use_qk_l2norm_in_kernel=False,
                            chunk_size=64, out=None, out_dtype=None):
    """Chunked (WY/UT) delta rule on the tensor cores, updating ``state`` in place.

    Same layouts as :func:`recurrent_gated_delta_rule_`; ``query/key/value`` are
    fp16 or bf16 (converted to fp16 operands inside the kernel).
    """
    _need_cuda(query, key, value, g, beta, state)
    for n, t in (("query", query), ("key", key), ("value", value), ("g", g), ("beta", beta), ("state", state)):
        _need_contig(n, t)
    if g.dtype != torch.float32 or beta.dtype != torch.float32 or state.dtype != torch.float32:
        raise TypeError("g, beta and state must be float32")
    if query.dtype != key.dtype or key.dtype != value.dtype:
        raise TypeError("query, key and value must share a dtype")
    B, T, H_qk, d_k = query.shape
    H_v, d_v = value.shape[2], value.shape[3]
    if key.shape != query.shape or value.shape[:2] != (B, T) or tuple(state.shape) != (B, H_v, d_k, d_v):
        raise ValueError("shape mismatch between query/key/value/state")
    if tuple(g.shape) != (B, T, H_v) or tuple(beta.shape) != (B, T, H_v):
        raise ValueError("g and beta must be [B, T, H_v]")
    out_dtype = out_dtype or query.dtype
    if out is None:
        out = torch.empty(B, T, H_v, d_v, dtype=out_dtype, device=query.device)
    rc = _lib.load().anemll_gdn_chunked_prefill(
        _lib.ptr(query), _lib.ptr(key), _lib.ptr(value), _lib.dtype_code(query.dtype), _lib.ptr(g), _lib.ptr(beta),
        _lib.ptr(state), _lib.ptr(out), _lib.dtype_code(out.dtype), B, T, H_qk, H_v, d_k, d_v, int(chunk_size),
        float(scale) if scale is not None else 0.0, int(bool(use_qk_l2norm_in_kernel)),
        _lib.stream_ptr(query.device))
    _lib.check(rc, "anemll_gdn_chunked_prefill")
    return out


def _z_rows(z, B, T, H, d):
    """``z`` [B, T, H, d] as (tensor, token row stride in elements): dense heads with a uniform token
    stride (a column slice of a wider projection output is read in place), else a contiguous copy."""
    if z.is_contiguous():
        return z, H * d
    if z.dim() == 4 and z.stride(-1) == 1 and z.stride(-2) == d:
        ld = z.stride(1) if T > 1 else z.stride(0)
        if B == 1 or T == 1 or z.stride(0) == ld * T:
            return z, ld
    return z.contiguous(), H * d


def gated_delta_rule_norm_(query, key, value, g, beta, state, z, norm_weight, eps=1e-6, chunked=True,
                           chunk_size=64, scale=None, use_qk_l2norm_in_kernel=False, out=None, out_dtype=None,
                           core_out=None):
    """The delta rule followed by the layer's gated RMSNorm: returns
    ``norm_weight * o * rsqrt(mean(o^2) + eps) * silu(z)`` [B, T, H_v, d_v] (``out_dtype``, default
    ``z.dtype``: fp16 or bf16), where ``o`` is the core output of :func:`chunk_gated_delta_rule_`
    (``chunked``) or :func:`recurrent_gated_delta_rule_`.  The chunked prefill applies the norm in its
    epilogue, so ``o`` never goes through HBM; the recurrent form runs the recurrent kernel and then
    :func:`gated_rmsnorm` (fused recurrent forms measured slower: the norm's sum over d_v spans the
    CTAs that split a head's state).  ``state`` is updated in place; ``core_out`` (fp32
    [B, T, H_v, d_v], optional) also receives ``o``.  ``z`` [B, T, H_v, d_v] may be a column slice of
    the layer's fused projection output.  Replaces the core call and ``self.norm`` of
    ``Qwen3_5GatedDeltaNet.forward`` (modeling_qwen3_5.py:497-523, 175-190)."""
    _need_cuda(query, key, value, g, beta, state, z, norm_weight, core_out)
    for n, t in (("query", query), ("key", key), ("value", value), ("g", g), ("beta", beta), ("state", state)):
        _need_contig(n, t)
    if g.dtype != torch.float32 or beta.dtype != torch.float32 or state.dtype != torch.float32:
        raise TypeError("g, beta and state must be float32")
    if query.dtype != key.dtype or key.dtype != value.dtype:
        raise TypeError("query, key and value must share a dtype")
    B, T, H_qk, d_k = query.shape
    H_v, d_v = value.shape[2], value.shape[3]
    if key.shape != query.shape or value.shape[:2] != (B, T) or tuple(state.shape) != (B, H_v, d_k, d_v):
        raise ValueError("shape mismatch between query/key/value/state")
    if tuple(g.shape) != (B, T, H_v) or tuple(beta.shape) != (B, T, H_v):
        raise ValueError("g and beta must be [B, T, H_v]")
    if tuple(z.shape) != (B, T, H_v, d_v) or tuple(norm_weight.shape) != (d_v,):
        raise ValueError("z must be [B, T, H_v, d_v] and norm_weight [d_v]")
    out_dtype = out_dtype or z.dtype
    if out_dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("the gated output is fp16 or bf16")
    if z.dtype != out_dtype:
        z = z.to(out_dtype)
    if not chunked:
        o = core_out if core_out is not None else torch.empty(B, T, H_v, d_v, dtype=torch.float32,
                                                              device=query.device)
        recurrent_gated_delta_rule_(query, key, value, g, beta, state, scale, use_qk_l2norm_in_kernel, out=o)
        return gated_rmsnorm(o, z, norm_weight, eps, out_dtype=out_dtype, out=out)
    z, z_ld = _z_rows(z, B, T, H_v, d_v)
    if chunked and (z_ld * z.element_size()) % 16:
        z, z_ld = z.contiguous(), H_v * d_v
    w = norm_weight.float().contiguous()
    if out is None:
        out = torch.empty(B, T, H_v, d_v, dtype=out_dtype, device=query.device)
    if core_out is not None and (core_out.dtype != torch.float32 or tuple(core_out.shape) != (B, T, H_v, d_v)
                                 or not core_out.is_contiguous()):
        raise ValueError("core_out must be a contiguous fp32 [B, T, H_v, d_v] tensor")
    lib = _lib.load()
    args = (_lib.ptr(query), _lib.ptr(key), _lib.ptr(value), _lib.dtype_code(query.dtype), _lib.ptr(g), _lib.ptr(beta),
            _lib.ptr(state), _lib.ptr(z), int(z_ld), _lib.ptr(w), float(eps), _lib.ptr(out), _lib.dtype_code(out.dtype),
            _lib.ptr(core_out), B, T, H_qk, H_v, d_k, d_v)
    tail = (float(scale) if scale is not None else 0.0, int(bool(use_qk_l2norm_in_kernel)),
            _lib.stream_ptr(query.device))
    rc = lib.anemll_gdn_chunked_prefill_gated(*args, int(chunk_size), *tail)
    _lib.check(rc, "anemll_gdn_chunked_prefill_gated")
    return out


def chunk_gated_delta_rule(query, key, value, g, beta, chunk_size=64, initial_state=None, output_final_state=False,
                           use_qk_l2norm_in_kernel=False, scale=None):
    """Functional form with the third-party signature; returns ``(out, final_state or None)``."""
    B, T, _, d_k = query.shape
    H_v, d_v = value.shape[2], value.shape[3]
    if initial_state is None:
        state = torch.zeros(B, H_v, d_k, d_v, dtype=torch.float32, device=query.device)
    else:
        state = initial_state.to(torch.float32).clone()
    out = chunk_gated_delta_rule_(query, key, value, g.float().contiguous(), beta.float().contiguous(), state,
                                  scale, use_qk_l2norm_in_kernel, chunk_size)
    return out, (state if output_final_state else None)


def chunked_device_error(reset=True) -> int:
    """Non-zero if a chunked-prefill launch stopped on a bounded wait (synchronous)."""
    return int(_lib.load().anemll_gdn_chunked_error(int(bool(reset))))


def _token_stride(t):
    """Elements between consecutive token rows of a [B, T, width] tensor whose rows are dense (unit
    stride along the width) with one uniform token stride, e.g. a column slice of a wider projection
    output; None for any other layout."""
    B, T, W = t.shape
    if t.stride(2) != 1 and W > 1:
        return None
    if T > 1:
        ld = t.stride(1)
        if B > 1 and t.stride(0) != ld * T:
            return None
    else:
        ld = t.stride(0) if B > 1 else W
    return ld if ld >= W else None


def _rows_for_kernel(t, align):
    """``t`` and its token stride, copied to a dense aligned tensor when its layout or alignment
    (``align`` bytes for the pointer and the row stride) does not suit the kernel."""
    ld = _token_stride(t)
    if ld is None or t.data_ptr() % align or (ld * t.element_size()) % align:
        t = t.contiguous()
        if t.data_ptr() % align:
            t = t.clone()
        ld = t.shape[2]
    return t, ld


def gdn_prologue(mixed_qkv, conv_weight, conv_state, a, b, A_log, dt_bias, num_k_heads, num_v_heads,
                 head_k_dim=128, head_v_dim=128, use_state=True, out_dtype=torch.float16):
    """conv1d(+SiLU) over ``mixed_qkv`` [B,T,C], split, l2-normalise q/k, gates.

    ``conv_weight`` [C, K] fp32; ``conv_state`` [B, C, K] (dtype of ``mixed_qkv``)
    is read as history when ``use_state`` and always receives the last K raw
    inputs.  ``mixed_qkv``, ``a`` and ``b`` may be column slices of one wider
    projection output (dense rows, uniform token stride).  Returns ``q, k``
    [B,T,H_qk,d_k], ``v`` [B,T,H_v,d_v] (``out_dtype``), ``g, beta`` [B,T,H_v] fp32.
    """
    _need_cuda(mixed_qkv, conv_weight, conv_state, a, b, A_log, dt_bias)
    for n, t in (("conv_weight", conv_weight), ("conv_state", conv_state), ("A_log", A_log)):
        _need_contig(n, t)
    B, T, C = mixed_qkv.shape
    K = conv_weight.shape[1]
    if C != 2 * num_k_heads * head_k_dim + num_v_heads * head_v_dim:
        raise ValueError("mixed_qkv width does not match the head configuration")
    if conv_state.dtype != mixed_qkv.dtype or tuple(conv_state.shape) != (B, C, K):
        raise ValueError("conv_state must be [B, C, K] in the dtype of mixed_qkv")
    if conv_weight.dtype != torch.float32 or A_log.dtype != torch.float32:
        raise TypeError("conv_weight and A_log must be float32")
    if a.dtype != b.dtype:
        raise TypeError("a and b must share a dtype")
    mixed_qkv, x_ld = _rows_for_kernel(mixed_qkv, 16)
    a, a_ld = _rows_for_kernel(a, 1)
    b, b_ld = _rows_for_kernel(b, 1)
    if a_ld != b_ld:
        a, b = a.contiguous(), b.contiguous()
        a_ld = num_v_heads
    dev = mixed_qkv.device
    q = torch.empty(B, T, num_k_heads, head_k_dim, dtype=out_dtype, device=dev)
    k = torch.empty_like(q)
    v = torch.empty(B, T, num_v_heads, head_v_dim, dtype=out_dtype, device=dev)
    g = torch.empty(B, T, num_v_heads, dtype=torch.float32, device=dev)
    beta = torch.empty_like(g)
    dtb = None if dt_bias is None else dt_bias.float().contiguous()
    rc = _lib.load().anemll_gdn_prologue(
        _lib.ptr(mixed_qkv), _lib.dtype_code(mixed_qkv.dtype), _lib.ptr(conv_weight), _lib.ptr(conv_state),
        _lib.ptr(a), _lib.ptr(b), _lib.dtype_code(a.dtype), _lib.ptr(A_log), _lib.ptr(dtb),
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(out_dtype), _lib.ptr(g), _lib.ptr(beta),
        B, T, num_k_heads, num_v_heads, head_k_dim, head_v_dim, K, int(bool(use_state)), x_ld, a_ld,
        _lib.stream_ptr(dev))
    _lib.check(rc, "anemll_gdn_prologue")
    return q, k, v, g, beta


def gated_rmsnorm(x, z, weight, eps=1e-6, out_dtype=None, out=None):
    """``weight * x * rsqrt(mean(x^2)+eps) * silu(z)`` over the last dim.  ``z`` may be a column slice
    of a wider projection output: [B, T, H, d] with dense heads and a uniform token stride."""
    _need_cuda(x, z, weight)
    _need_contig("x", x)
    d = x.shape[-1]
    if z.shape != x.shape or weight.shape != (d,):
        raise ValueError("gated_rmsnorm: shape mismatch")
    z_heads, z_ld = 0, 0
    if not z.is_contiguous():
        ok = z.dim() == 4 and z.stride(-1) == 1 and z.stride(-2) == d
        if ok:
            B, T, H = z.shape[:3]
            z_ld = z.stride(1) if T > 1 else z.stride(0)
            ok = (B == 1 or T == 1 or z.stride(0) == z_ld * T)
            z_heads = H
        if not ok:
            z, z_heads, z_ld = z.contiguous(), 0, 0
    w = weight.float().contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    elif out.shape != x.shape or not out.is_contiguous():
        raise ValueError("gated_rmsnorm: out must be a contiguous tensor of x's shape")
    rc = _lib.load().anemll_gated_rmsnorm(_lib.ptr(x), _lib.dtype_code(x.dtype), _lib.ptr(z), _lib.dtype_code(z.dtype),
                                          _lib.ptr(w), _lib.ptr(out), _lib.dtype_code(out.dtype), x.numel() // d, d,
                                          float(eps), z_heads, z_ld, _lib.stream_ptr(x.device))
    _lib.check(rc, "anemll_gated_rmsnorm")
    return out


class GatedDeltaNet(nn.Module):
    """Drop-in Qwen3.5 gated-DeltaNet layer (``Qwen3_5GatedDeltaNet``, modeling_qwen3_5.py:356-533).

    Same parameters and projections; the state lives in caller-owned tensors
    that ``forward(hidden_states, current_pos, conv_state, recurrent_state)``
    mutates in place (the reference's mutable-buffer convention, like its
    ``kv_cache_0`` buffer): ``conv_state`` [B, C, K] in the activation dtype and
    ``recurrent_state`` [B, H_v, d_k, d_v] fp32.  ``current_pos`` is the
    position of the first token of ``hidden_states`` (an int or a one-element
    tensor): 0 starts a sequence (zero conv history, the recurrent state is
    reset), a later position continues from the states.  Calls of 16 tokens
    or more run the chunked prefill kernel, shorter ones the recurrent kernel.
    """

    def __init__(self, hidden_size=2048, num_k_heads=16, num_v_heads=32, head_k_dim=128, head_v_dim=128,
                 conv_kernel=4, eps=1e-6, dtype=torch.bfloat16, core_dtype=torch.float16, chunk_size=64,
                 device=None):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_k_heads, self.num_v_heads = num_k_heads, num_v_heads
        self.head_k_dim, self.head_v_dim = head_k_dim, head_v_dim
        self.key_dim = num_k_heads * head_k_dim
        self.value_dim = num_v_heads * head_v_dim
        self.conv_dim = 2 * self.key_dim + self.value_dim
        self.conv_kernel = conv_kernel
        self.eps = eps
        self.core_dtype = core_dtype
        self.chunk_size = chunk_size
        fk = dict(device=device, dtype=dtype)
        # the four input projections are views of one [qkv | z | b | a] weight: one GEMM, whose column
        # slices the prologue and the gated norm read in place
        widths = (self.conv_dim, self.value_dim, num_v_heads, num_v_heads)
        self.w_in = torch.empty(sum(widths), hidden_size, **fk)
        off = 0
        for name, n in zip(("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a"), widths):
            lin = nn.Linear(hidden_size, n, bias=False, device="meta")
            lin.weight = nn.Parameter(self.w_in[off:off + n])
            setattr(self, name, lin)
            off += n
        self.conv_weight = nn.Parameter(torch.zeros(self.conv_dim, conv_kernel, device=device, dtype=torch.float32))
        self.dt_bias = nn.Parameter(torch.zeros(num_v_heads, device=device, dtype=torch.float32))
        self.A_log = nn.Parameter(torch.zeros(num_v_heads, device=device, dtype=torch.float32))
        self.norm_weight = nn.Parameter(torch.ones(head_v_dim, device=device, dtype=torch.float32))
        self.out_proj = nn.Linear(self.value_dim, hidden_size, bias=False, **fk)

    def new_states(self, batch_size, device=None, dtype=None):
        device = device or self.in_proj_qkv.weight.device
        dtype = dtype or self.in_proj_qkv.weight.dtype
        conv = torch.zeros(batch_size, self.conv_dim, self.conv_kernel, device=device, dtype=dtype)
        rec = torch.zeros(batch_size, self.num_v_heads, self.head_k_dim, self.head_v_dim, device=device,
                          dtype=torch.float32)
        return conv, rec

    CHUNKED_MIN_TOKENS = 16  # calls with at least this many tokens run the chunked prefill kernel

    def core(self, mixed_qkv, z, a, b, conv_state, recurrent_state, current_pos=0, return_core=False):
        """Everything between the input and output projections (the hot path): the prologue, then the
        chunked or recurrent kernel with the gated RMSNorm in its epilogue.  Returns the gated-normed
        output (activation dtype), or with ``return_core`` the pair (fp32 core output, normed output)
        from the same launch."""
        B, T, _ = mixed_qkv.shape
        cont = _position(current_pos) > 0
        if not cont:
            recurrent_state.zero_()
        q, k, v, g, beta = gdn_prologue(mixed_qkv, self.conv_weight, conv_state, a, b, self.A_log, self.dt_bias,
                                        self.num_k_heads,
                                        self.num_v_heads, self.head_k_dim, self.head_v_dim,
                                        use_state=cont, out_dtype=self.core_dtype)
        o = None
        if return_core:
            o = torch.empty(B, T, self.num_v_heads, self.head_v_dim, dtype=torch.float32, device=mixed_qkv.device)
        normed = gated_delta_rule_norm_(q, k, v, g, beta, recurrent_state,
                                        z.reshape(B, T, self.num_v_heads, self.head_v_dim), self.norm_weight,
                                        self.eps, chunked=T >= self.CHUNKED_MIN_TOKENS, chunk_size=self.chunk_size,
                                        out_dtype=mixed_qkv.dtype, core_out=o)
        return (o, normed) if return_core else normed

    def forward(self, hidden_states, current_pos, conv_state, recurrent_state):
        B, T, _ = hidden_states.shape
        proj = F.linear(hidden_states, self.w_in)  # [B, T, conv_dim + value_dim + 2 H_v]
        c, v = self.conv_dim, self.value_dim
        mixed_qkv, z = proj[..., :c], proj[..., c:c + v]
        b, a = proj[..., c + v:c + v + self.num_v_heads], proj[..., c + v + self.num_v_heads:]
        normed = self.core(mixed_qkv, z, a, b, conv_state, recurrent_state, current_pos)
        return F.linear(normed.reshape(B, T, self.value_dim), self.out_proj.weight)


def _position(current_pos) -> int:
    """``current_pos`` as an int: the reference passes positions as one-element int tensors."""
    if isinstance(current_pos, torch.Tensor):
        if current_pos.numel() != 1:
            raise ValueError("current_pos must hold one position")
        return int(current_pos.reshape(()).item())
    return int(current_pos)
