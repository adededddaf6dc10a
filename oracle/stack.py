"""CPU oracle of the 24-layer hybrid stack's layers (test infrastructure only).

Each layer is restated in fp32 from its weights (copied from the device model), rounding to bf16
exactly where the device path materialises bf16 tensors (GEMM outputs, norms, rotary outputs,
residual sums), so that a comparison isolates the library's kernels and the wiring:

* gated-DeltaNet layer: torch projections, then the CPU restatement of the layer core
  (:func:`oracle.gdn.gdn_layer_prefill` / :func:`oracle.gdn.gdn_layer_decode`, the semantics of
  ``Qwen3_5GatedDeltaNet``), then ``out_proj``;
* gated full attention: q/k/v/gate projections, per-head RMSNorm of q and k (``QwenHeadNorm``,
  ``anemll/models/qwen_model.py:143-184``), rotary embedding (186-261), the cache write and
  attention of :func:`oracle.kv_attention.attend` over the whole cache with the causal mask, the
  sigmoid gate, ``o_proj``;
* SwiGLU MLP and RMSNorm.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import gdn as og
from . import kv_attention as ok


def bf(x):
    return x.to(torch.bfloat16).float()


def rms_norm(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope(x, cos, sin):
    h = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., h:], x[..., :h]], dim=-1) * sin


def _w(p):
    return p.detach().float().cpu()


def attention_core(m, cfg, qkv, kc, vc, pos, cos, sin, with_k=False):
    """The attention call of a gated full-attention layer on its fused projection output ``qkv``
    [B, T, H_q*2*hd + 2*H_kv*hd] (per query head ``[query | gate]``, then k, then v; bf16-valued fp32):
    per-head RMSNorm of q and k, RoPE, the cache write into ``kc``/``vc`` [B, H_kv, ctx, hd] (fp32,
    updated in place), attention over the cache with the causal mask and the sigmoid gate.  Returns
    the gated output [B, T, H_q*hd] in fp32, before its bf16 rounding and ``o_proj`` (and with
    ``with_k`` also the new K rows [B, H_kv, T, hd] before their bf16 rounding and the normed K rows
    that entered RoPE, bf16-valued, in the same layout)."""
    B, T, _ = qkv.shape
    n_q, n_kv = cfg.H_q * 2 * cfg.head_dim, cfg.H_kv * cfg.head_dim
    qg = qkv[..., :n_q].reshape(B, T, cfg.H_q, 2 * cfg.head_dim)
    q, gate = qg[..., :cfg.head_dim], qg[..., cfg.head_dim:]
    k = qkv[..., n_q:n_q + n_kv].reshape(B, T, cfg.H_kv, cfg.head_dim)
    v = qkv[..., n_q + n_kv:].reshape(B, T, cfg.H_kv, cfg.head_dim)
    q = bf(rms_norm(q, _w(m.q_norm), cfg.eps)).transpose(1, 2)
    k = bf(rms_norm(k, _w(m.k_norm), cfg.eps)).transpose(1, 2)
    q = bf(rope(q, cos, sin))
    k_f = rope(k, cos, sin)
    kc[:, :, pos:pos + T] = bf(k_f)
    vc[:, :, pos:pos + T] = v.transpose(1, 2)
    o = ok.attend(q, kc, vc, ok.additive_mask(T, cfg.ctx, pos), gate.reshape(B, T, -1))
    return (o, k_f, k) if with_k else o


def attention_layer(m, cfg, h, kc, vc, pos, cos, sin):
    """h [B, T, hidden] (bf16-valued fp32) -> o_proj output; kc/vc [B, H_kv, ctx, hd] fp32, updated."""
    qkv = bf(torch.cat([F.linear(h, _w(m.q_proj.weight)), F.linear(h, _w(m.k_proj.weight)),
                        F.linear(h, _w(m.v_proj.weight))], dim=-1))
    o = attention_core(m, cfg, qkv, kc, vc, pos, cos, sin)
    return bf(F.linear(bf(o), _w(m.o_proj.weight)))


def gdn_layer(m, cfg, h, conv, S, pos):
    """h [B, T, hidden] -> (out_proj output, conv state, recurrent state)."""
    B, T, _ = h.shape
    mixed = bf(F.linear(h, _w(m.in_proj_qkv.weight)))
    z = bf(F.linear(h, _w(m.in_proj_z.weight)))
    b = bf(F.linear(h, _w(m.in_proj_b.weight)))
    a = bf(F.linear(h, _w(m.in_proj_a.weight)))
    params = dict(conv_w=_w(m.conv_weight), A_log=_w(m.A_log), dt_bias=_w(m.dt_bias), norm_w=_w(m.norm_weight),
                  eps=m.eps)
    if pos == 0:
        _, normed, conv, S = og.gdn_layer_prefill(mixed, z, a, b, params, cfg.H_qk, cfg.H_v, cfg.d_k, cfg.d_v)
    else:
        _, normed, conv, S = og.gdn_layer_decode(mixed, z, a, b, params, cfg.H_qk, cfg.H_v, cfg.d_k, cfg.d_v, conv, S)
    out = bf(F.linear(bf(normed).reshape(B, T, -1), _w(m.out_proj.weight)))
    return out, conv, S


def layer(model, i, x, state, pos, with_mixer=False):
    """One layer of ``model`` (an ``anemll_b200.stack.HybridStack``) on x [B, T, hidden] (bf16-valued
    fp32, CPU); ``state`` is this layer's oracle state (a mutable list).  Returns the layer output (and
    the mixer output before the residual add when ``with_mixer``)."""
    cfg = model.cfg
    T = x.shape[1]
    h = bf(rms_norm(x, _w(model.norm1[i]), cfg.eps))
    if cfg.is_attention(i):
        cos = model.cos[pos:pos + T].cpu()
        sin = model.sin[pos:pos + T].cpu()
        h = attention_layer(model.mixers[i], cfg, h, state[0], state[1], pos, cos, sin)
    else:
        h, state[0], state[1] = gdn_layer(model.mixers[i], cfg, h, state[0], state[1], pos)
    x = bf(x + h)
    gu = bf(F.linear(bf(rms_norm(x, _w(model.norm2[i]), cfg.eps)), _w(model.gate_up[i].weight)))
    gate, up = gu.chunk(2, dim=-1)
    y = bf(x + bf(F.linear(bf(bf(F.silu(gate)) * up), _w(model.down[i].weight))))
    return (y, h) if with_mixer else y


def host_model(model):
    """An fp32 copy of a device ``HybridStack`` on the host (built once; the layer functions above then
    read its weights without device copies)."""
    from anemll_b200.stack import HybridStack
    host = HybridStack(model.cfg, device="meta", dtype=torch.float32).to_empty(device="cpu")
    with torch.no_grad():
        src = dict(model.named_parameters())
        for name, p in host.named_parameters():
            p.copy_(src[name].detach().float().cpu())
    host.cos, host.sin = model.cos.cpu(), model.sin.cpu()
    return host


def new_state(model, B):
    cfg = model.cfg
    st = []
    for i in range(cfg.n_layers):
        if cfg.is_attention(i):
            st.append([torch.zeros(B, cfg.H_kv, cfg.ctx, cfg.head_dim), torch.zeros(B, cfg.H_kv, cfg.ctx, cfg.head_dim)])
        else:
            st.append([None, None])
    return st
