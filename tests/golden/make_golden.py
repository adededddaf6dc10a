"""Generate the golden fixtures in this directory (run once, in the build container).

Sources of truth:

* KV-cache attention: the reference itself, ``anemll/models/qwen_model.py`` from
  the read-only reference checkout (``--reference PATH`` or the
  ``ANEMLL_REFERENCE`` environment variable), imported with ``MODEL_DTYPE = torch.float32`` so the
  whole attention path runs in fp32 on fp16-rounded inputs.
  ``QwenAttention.forward_prefill`` (509-546) and ``forward_regular`` (469-507)
  are called with ``o_proj`` set to the identity, so the recorded output is the
  pre-projection attention output; ``kv_attention_oproj.pt`` records the same
  methods with a random ``o_proj``, i.e. the reference's full return value.  The cache write is recorded by running
  ``QwenModel.process_layer_prefill`` (647-696) / ``process_layer_regular``
  (698-839) on a tiny random model and capturing ``kv_cache_0`` before and after.
  Masks: ``tests/chat.py`` ``make_causal_mask`` (977-983) rule; sliding windows
  by the per-query rule and by the chunk-aligned rule of
  ``anemll/models/gemma3_model.py`` ``_kv_slice`` (923-926).

* Gated delta rule: the reference has no implementation, so the pin is the
  third-party ``transformers==5.5.0`` module
  ``transformers/models/qwen3_5/modeling_qwen3_5.py``:
  ``torch_chunk_gated_delta_rule`` (234-311),
  ``torch_recurrent_gated_delta_rule`` (314-353),
  ``torch_causal_conv1d_update`` (210-226), the prefill conv of
  ``Qwen3_5GatedDeltaNet.forward`` (463-474) and ``Qwen3_5RMSNormGated``
  (175-190), all on CPU in fp32 (the chunk/recurrent rules in fp64 as well).

Usage: ``python tests/golden/make_golden.py --reference PATH``.
The GPU tests and the oracle tests read only the ``.pt`` files written here.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _r16(x):
    return x.to(torch.float16).to(torch.float32)


def causal_mask_ref_rule(S, ctx, pos):
    """``make_causal_mask(ctx, 0)`` rows ``[pos, pos+S)`` (``tests/chat.py:977-983``, row-sliced at 1058)."""
    row = torch.arange(ctx).view(ctx, 1)
    col = torch.arange(ctx).view(1, ctx)
    m = torch.full((ctx, ctx), float("-inf"))
    m[col <= row] = 0.0
    return m[pos:pos + S].view(1, 1, S, ctx)


def window_mask(S, ctx, pos, W, chunk_aligned):
    m = causal_mask_ref_rule(S, ctx, pos).clone()
    j = torch.arange(ctx).view(1, ctx)
    p = pos + torch.arange(S).view(S, 1)
    if chunk_aligned:
        start = max(0, min(pos + S, ctx) - W)  # gemma3_model.py:923-926
        lo = torch.full((S, 1), start)
        hide = j < lo
    else:
        hide = j <= p - W
    m[0, 0][hide] = float("-inf")
    return m


def make_kv(ref_root):
    sys.path.insert(0, ref_root)
    import anemll.models.qwen_model as qm  # noqa: E402

    qm.MODEL_DTYPE = torch.float32
    torch.manual_seed(20)
    Hq, Hkv, hd, ctx = 4, 2, 64, 256
    cfg = qm.QwenConfig(hidden_size=Hq * hd, num_attention_heads=Hq, num_key_value_heads=Hkv,
                        head_dim=hd, context_length=ctx, state_length=ctx, num_hidden_layers=1,
                        intermediate_size=64, vocab_size=32)
    attn = qm.QwenAttention(cfg)
    with torch.no_grad():
        attn.o_proj.weight.copy_(torch.eye(Hq * hd).view(Hq * hd, Hq * hd, 1, 1))
    cases = []
    specs = [
        ("prefill_causal", 16, 100, 0, False),
        ("prefill_causal_pos0", 16, 0, 0, False),
        ("decode_causal", 1, 200, 0, False),
        ("decode_last", 1, ctx - 1, 0, False),
        ("prefill_swa", 16, 150, 64, False),
        ("prefill_swa_chunk_aligned", 16, 150, 64, True),
        ("decode_swa", 1, 200, 64, False),
    ]
    for name, S, pos, W, aligned in specs:
        K = torch.zeros(Hkv, ctx, hd)
        V = torch.zeros(Hkv, ctx, hd)
        K[:, :pos + S] = _r16(torch.randn(Hkv, pos + S, hd))
        V[:, :pos + S] = _r16(torch.randn(Hkv, pos + S, hd))
        q = _r16(torch.randn(1, Hq, S, hd))
        mask = window_mask(S, ctx, pos, W, aligned) if W else causal_mask_ref_rule(S, ctx, pos)
        hidden = torch.zeros(1, S, Hq * hd)
        with torch.no_grad():
            if S == 1:
                out = attn.forward_regular(hidden, q, (K, V), mask, torch.tensor([pos]))
            else:
                out = attn.forward_prefill(hidden, q, (K, V), mask)
        cases.append(dict(name=name, S=S, pos=pos, window=W, chunk_aligned=aligned,
                          q=q.half(), K=K[:, :pos + S].half(), V=V[:, :pos + S].half(),
                          visible=(mask[0, 0] == 0), out=out.float()))
    torch.save(dict(Hq=Hq, Hkv=Hkv, hd=hd, ctx=ctx, cases=cases), os.path.join(HERE, "kv_attention.pt"))

    # ---- cache write through the reference model (bit-exact target) ----
    torch.manual_seed(21)
    L, Hq, Hkv, hd, ctx = 2, 4, 2, 64, 64
    cfg = qm.QwenConfig(hidden_size=128, num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=hd,
                        context_length=ctx, state_length=ctx, num_hidden_layers=L,
                        intermediate_size=64, vocab_size=32)
    model = qm.QwenModel(cfg)
    writes = []
    for name, layer_idx, S, pos in [("prefill_l1", 1, 8, 20), ("decode_l0", 0, 1, 40), ("prefill_l0_end", 0, 8, ctx - 8)]:
        with torch.no_grad():
            model.kv_cache_0.copy_(_r16(torch.randn_like(model.kv_cache_0)))
            before = model.kv_cache_0.clone()
            hidden = torch.randn(1, S, 128)
            layer = model.layers[layer_idx]
            normed = layer.input_layernorm(hidden)
            pos_ids = torch.arange(pos, pos + S)
            if S == 1:
                rot = model.get_rotary_embeddings_s(pos)
                q, k, v = layer.self_attn.get_new_kv_cache(normed, torch.tensor([pos]), rot)
                mask = causal_mask_ref_rule(1, ctx, pos)
                model.process_layer_regular(layer_idx, hidden, pos_ids, mask, torch.tensor([pos]), rot, 0)
            else:
                rot = model.get_rotary_embedding_prefill(pos_ids)
                q, k, v = layer.self_attn.get_new_kv_cache_prefill(normed, torch.tensor([pos]), rot)
                mask = causal_mask_ref_rule(S, ctx, pos)
                model.process_layer_prefill(layer_idx, hidden, pos_ids, mask, torch.tensor([pos]), rot, 0)
            after = model.kv_cache_0.clone()
        # the fp32 cache copy commutes with rounding to fp16, so fp16 views are the target
        writes.append(dict(name=name, layer_idx=layer_idx, num_layers=L, S=S, pos=pos,
                           k=k.half(), v=v.half(), before=before.half(), after=after.half()))
    torch.save(dict(writes=writes), os.path.join(HERE, "kv_cache_write.pt"))


def make_gdn():
    from transformers.models.qwen3_5 import modeling_qwen3_5 as m

    torch.manual_seed(30)
    B, T, Hqk, Hv, dk, dv = 1, 130, 2, 4, 128, 128
    rep = Hv // Hqk
    q = torch.randn(B, T, Hqk, dk).to(torch.float16)
    k = torch.randn(B, T, Hqk, dk).to(torch.float16)
    v = torch.randn(B, T, Hv, dv).to(torch.float16)
    beta = torch.sigmoid(torch.randn(B, T, Hv))
    A_log = torch.empty(Hv).uniform_(0.0, float(torch.log(torch.tensor(16.0))))
    g = -F.softplus(torch.randn(B, T, Hv)) * torch.exp(A_log)
    S0 = 0.01 * torch.randn(B, Hv, dk, dv)

    def run(fn, dtype, **kw):
        qq = q.to(dtype).repeat_interleave(rep, dim=2)
        kk = k.to(dtype).repeat_interleave(rep, dim=2)
        o, s = fn(qq, kk, v.to(dtype), g=g.to(dtype), beta=beta.to(dtype), initial_state=S0.to(dtype),
                  output_final_state=True, use_qk_l2norm_in_kernel=True, **kw)
        return o, s

    o_chunk, s_chunk = run(m.torch_chunk_gated_delta_rule, torch.float64, chunk_size=64)
    o_rec, s_rec = run(m.torch_recurrent_gated_delta_rule, torch.float64)
    gdn = dict(B=B, T=T, Hqk=Hqk, Hv=Hv, dk=dk, dv=dv, q=q, k=k, v=v, g=g, beta=beta, S0=S0,
               out_chunk=o_chunk.float(), state_chunk=s_chunk.float(),
               out_recurrent=o_rec.float(), state_recurrent=s_rec.float())

    # conv prologue: prefill from zero history, then a decode update
    torch.manual_seed(31)
    C, K, Tp = 3 * 64 + 2 * 64, 4, 7  # 2 key heads + 2 value heads of 64... any C works
    w = 0.1 * torch.randn(C, K)
    x = torch.randn(2, Tp, C).to(torch.float16)
    xt = x.float().transpose(1, 2)
    conv = torch.nn.Conv1d(C, C, K, groups=C, padding=K - 1, bias=False)
    with torch.no_grad():
        conv.weight.copy_(w.unsqueeze(1))
        y_prefill = F.silu(conv(xt)[:, :, :Tp])  # modeling_qwen3_5.py:474
    state_prefill = F.pad(xt, (K - Tp, 0)) if Tp < K else xt[:, :, -K:]  # 463-464
    x1 = torch.randn(2, 1, C).to(torch.float16)
    st = state_prefill.clone()
    y_dec = m.torch_causal_conv1d_update(x1.float().transpose(1, 2), st, w, None, "silu")
    conv_fx = dict(C=C, K=K, w=w, x=x, y_prefill=y_prefill.transpose(1, 2).contiguous(),
                   state_prefill=state_prefill.clone(), x1=x1, y_decode=y_dec.transpose(1, 2).contiguous(),
                   state_decode=st.clone())

    torch.manual_seed(32)
    xn = torch.randn(5, 3, 128)
    z = torch.randn(5, 3, 128)
    norm = m.Qwen3_5RMSNormGated(128, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(1.0 + 0.1 * torch.randn(128))
        yn = norm(xn, z)
    norm_fx = dict(x=xn, z=z, weight=norm.weight.detach().clone(), y=yn)
    torch.save(dict(gdn=gdn, conv=conv_fx, norm=norm_fx), os.path.join(HERE, "gdn.pt"))


def make_kv_oproj(ref_root):
    """``kv_attention_oproj.pt``: the reference's ``QwenAttention.forward_prefill`` / ``forward_regular``
    with a random ``o_proj`` (a 1x1 Conv2d from H_q*hd = 256 to hidden 320), so the drop-in module's
    projected output is compared with exactly what the reference returns."""
    sys.path.insert(0, ref_root)
    import anemll.models.qwen_model as qm  # noqa: E402

    qm.MODEL_DTYPE = torch.float32
    torch.manual_seed(23)
    Hq, Hkv, hd, ctx, hidden = 4, 2, 64, 256, 320
    cfg = qm.QwenConfig(hidden_size=hidden, num_attention_heads=Hq, num_key_value_heads=Hkv,
                        head_dim=hd, context_length=ctx, state_length=ctx, num_hidden_layers=1,
                        intermediate_size=64, vocab_size=32)
    attn = qm.QwenAttention(cfg)
    with torch.no_grad():  # fp16-representable weights, so both sides project with the same values
        attn.o_proj.weight.copy_(_r16(0.05 * torch.randn_like(attn.o_proj.weight)))
    cases = []
    for name, S, pos in [("prefill", 16, 100), ("decode", 1, 200)]:
        K = torch.zeros(Hkv, ctx, hd)
        V = torch.zeros(Hkv, ctx, hd)
        K[:, :pos + S] = _r16(torch.randn(Hkv, pos + S, hd))
        V[:, :pos + S] = _r16(torch.randn(Hkv, pos + S, hd))
        q = _r16(torch.randn(1, Hq, S, hd))
        mask = causal_mask_ref_rule(S, ctx, pos)
        hs = torch.zeros(1, S, hidden)
        with torch.no_grad():
            if S == 1:
                out = attn.forward_regular(hs, q, (K, V), mask, torch.tensor([pos]))
            else:
                out = attn.forward_prefill(hs, q, (K, V), mask)
        cases.append(dict(name=name, S=S, pos=pos, q=q.half(), K=K[:, :pos + S].half(), V=V[:, :pos + S].half(),
                          out=out.float()))
    torch.save(dict(Hq=Hq, Hkv=Hkv, hd=hd, ctx=ctx, hidden=hidden,
                    o_proj_weight=attn.o_proj.weight.detach().clone(), cases=cases),
               os.path.join(HERE, "kv_attention_oproj.pt"))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ANEMLL_REFERENCE"),
                    required="ANEMLL_REFERENCE" not in os.environ,
                    help="checkout of the reference repository (or set ANEMLL_REFERENCE)")
    args = ap.parse_args()
    make_kv(args.reference)
    make_kv_oproj(args.reference)
    make_gdn()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
