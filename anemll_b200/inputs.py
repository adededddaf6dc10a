"""Seeded synthetic workloads for the five benchmark configurations.

No public dataset drives this path; every input is drawn from the stated
distributions with ``torch.manual_seed(seed)`` on the CPU generator (so the
values do not depend on the device), rounded to the kernel dtype, and the
oracle consumes the rounded values upcast to fp32.

* gdn_layer       (seed 0) one gated-DeltaNet layer, B=1, H_qk=16, H_v=32,
                  d=128, hidden 2048: hidden ~ N(0,1); projections ~ N(0,0.02);
                  conv1d kernel 4 ~ N(0,0.1); A_log ~ U(log 1, log 16);
                  dt_bias = 0; state zero.
* gdn_decode      (seed 1) B=64 decode: state ~ N(0, 0.01) fp32
                  [64,32,128,128]; q, k ~ N(0,1) l2-normalised then bf16;
                  v ~ N(0,1) bf16; beta = sigmoid(N(0,1));
                  g = -softplus(N(0,1)) * exp(A_log), A_log ~ U(log 1, log 16).
* kv_attention    (seed 2) H_q=16, H_kv=2, hd=256, ctx=4096, fp16: cache
                  prefilled ~ N(0,1) at 0..2047; new q/k/v ~ N(0,1) for
                  positions 2048..4095; gate pre-activation ~ N(0,1).
* gdn_prefill     (seed 3) B=8 x T=32768 chunked prefill, bf16 q/k/v with the
                  gdn_decode distributions; generated on the device (4 GiB).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

H_QK, H_V, D_K, D_V, HIDDEN = 16, 32, 128, 128, 2048


def _gates(gen_shape, A_log):
    beta = torch.sigmoid(torch.randn(gen_shape))
    g = -F.softplus(torch.randn(gen_shape)) * torch.exp(A_log)
    return g.float(), beta.float()


def _A_log(H):
    return torch.empty(H).uniform_(math.log(1.0), math.log(16.0))


def gdn_layer(seed=0, B=1, T_prefill=512, T_decode=64, dtype=torch.bfloat16):
    """Weights and hidden states of the single-layer workload (CPU tensors)."""
    torch.manual_seed(seed)
    C = 2 * H_QK * D_K + H_V * D_V
    w = dict(
        in_proj_qkv=(0.02 * torch.randn(C, HIDDEN)).to(dtype),
        in_proj_z=(0.02 * torch.randn(H_V * D_V, HIDDEN)).to(dtype),
        in_proj_b=(0.02 * torch.randn(H_V, HIDDEN)).to(dtype),
        in_proj_a=(0.02 * torch.randn(H_V, HIDDEN)).to(dtype),
        out_proj=(0.02 * torch.randn(HIDDEN, H_V * D_V)).to(dtype),
        conv_w=(0.1 * torch.randn(C, 4)).float(),
        A_log=_A_log(H_V).float(),
        dt_bias=torch.zeros(H_V),
        norm_w=torch.ones(D_V),
    )
    hidden = torch.randn(B, T_prefill + T_decode, HIDDEN).to(dtype)
    return w, hidden


def gdn_decode(seed=1, B=64, steps=256, dtype=torch.bfloat16, state=True):
    """Decode workload: returns dict of CPU tensors (state optional: 128 MiB at B=64)."""
    torch.manual_seed(seed)
    A_log = _A_log(H_V)
    S0 = 0.01 * torch.randn(B, H_V, D_K, D_V) if state else None
    q = F.normalize(torch.randn(steps, B, 1, H_QK, D_K), dim=-1).to(dtype)
    k = F.normalize(torch.randn(steps, B, 1, H_QK, D_K), dim=-1).to(dtype)
    v = torch.randn(steps, B, 1, H_V, D_V).to(dtype)
    g, beta = _gates((steps, B, 1, H_V), A_log)
    return dict(state=S0, q=q, k=k, v=v, g=g, beta=beta, A_log=A_log)


def kv_attention(seed=2, Hq=16, Hkv=2, hd=256, ctx=4096, prefill_from=2048, prefill_to=4032, chunk=64,
                 dtype=torch.float16):
    torch.manual_seed(seed)
    cache = torch.zeros(2, Hkv, ctx, hd)
    cache[:, :, :prefill_from] = torch.randn(2, Hkv, prefill_from, hd)
    n_new = ctx - prefill_from
    q = torch.randn(1, Hq, n_new, hd)
    k = torch.randn(1, Hkv, n_new, hd)
    v = torch.randn(1, Hkv, n_new, hd)
    gate = torch.randn(1, n_new, Hq * hd)
    return dict(cache=cache.to(dtype), q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), gate=gate.to(dtype),
                prefill_from=prefill_from, prefill_to=prefill_to, chunk=chunk)


def gdn_prefill_device(seed=3, B=8, T=32768, device="cuda", dtype=torch.bfloat16, Hqk=H_QK, Hv=H_V):
    """Long-prefill workload generated on the device with a seeded CUDA generator."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    A_log = torch.empty(Hv, device=device).uniform_(math.log(1.0), math.log(16.0), generator=gen)
    q = F.normalize(torch.randn(B, T, Hqk, D_K, device=device, generator=gen), dim=-1).to(dtype)
    k = F.normalize(torch.randn(B, T, Hqk, D_K, device=device, generator=gen), dim=-1).to(dtype)
    v = torch.randn(B, T, Hv, D_V, device=device, generator=gen).to(dtype)
    beta = torch.sigmoid(torch.randn(B, T, Hv, device=device, generator=gen))
    g = -F.softplus(torch.randn(B, T, Hv, device=device, generator=gen)) * torch.exp(A_log)
    return dict(q=q, k=k, v=v, g=g.float(), beta=beta.float())
