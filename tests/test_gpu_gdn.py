"""GPU parity of the gated delta-rule kernels against the CPU oracle (through the C ABI)."""
import os

import pytest
import torch
import torch.nn.functional as F

from anemll_b200 import gdn, inputs
from oracle import gdn as og
from tests.conftest import GOLDEN
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def gold():
    return torch.load(os.path.join(GOLDEN, "gdn.pt"))["gdn"]


def test_recurrent_prefill_matches_golden(gold):
    d = gold
    state = d["S0"].to(DEV).contiguous()
    out = gdn.recurrent_gated_delta_rule_(d["q"].to(DEV), d["k"].to(DEV), d["v"].to(DEV), d["g"].to(DEV),
                                          d["beta"].to(DEV), state, use_qk_l2norm_in_kernel=True,
                                          out_dtype=torch.float32)
    assert_close(out, d["out_recurrent"], "out")
    assert_close(state, d["state_recurrent"], "state")


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_decode_full_batch_few_steps(out_dtype):
    w = inputs.gdn_decode(B=64, steps=3)
    S_ref = w["state"].clone()
    state = w["state"].to(DEV)
    for t in range(3):
        q, k, v, g, b = (w[n][t] for n in ("q", "k", "v", "g", "beta"))
        out = gdn.recurrent_gated_delta_rule_(q.to(DEV), k.to(DEV), v.to(DEV), g.to(DEV), b.to(DEV), state,
                                              out_dtype=out_dtype)
        o_ref, S_ref = og.recurrent_gated_delta_rule(q, k, v, g, b, S_ref)
        if out_dtype == torch.bfloat16:
            o_ref = o_ref.to(torch.bfloat16).float()  # the output rounding is part of the contract
            assert_close(out.float(), o_ref, f"out step {t}", rel_l2=5e-3)
        else:
            assert_close(out, o_ref, f"out step {t}")
    assert_close(state, S_ref, "state")


def test_decode_256_steps_small_batch():
    w = inputs.gdn_decode(B=2, steps=256)
    S_ref = w["state"].clone()
    state = w["state"].to(DEV)
    outs, refs = [], []
    for t in range(256):
        q, k, v, g, b = (w[n][t] for n in ("q", "k", "v", "g", "beta"))
        outs.append(gdn.recurrent_gated_delta_rule_(q.to(DEV), k.to(DEV), v.to(DEV), g.to(DEV), b.to(DEV), state,
                                                    out_dtype=torch.float32))
    q, k, v, g, b = (w[n].squeeze(2).transpose(0, 1).contiguous() for n in ("q", "k", "v", "g", "beta"))
    o_ref, S_ref = og.recurrent_gated_delta_rule(q, k, v, g, b, S_ref)
    assert_close(torch.cat(outs, 1), o_ref, "outputs")
    assert_close(state, S_ref, "state")


def test_multi_token_launch_equals_token_launches_bit_exact():
    """Size-independent property at the full decode shape: T tokens in one launch
    (state kept in registers) == T single-token launches (state through HBM)."""
    w = inputs.gdn_decode(B=64, steps=2)
    q, k, v, g, b = (w[n].squeeze(2).transpose(0, 1).contiguous().to(DEV) for n in ("q", "k", "v", "g", "beta"))
    s1 = w["state"].to(DEV)
    s2 = s1.clone()
    o1 = gdn.recurrent_gated_delta_rule_(q, k, v, g, b, s1, out_dtype=torch.float32)
    o2 = torch.cat([gdn.recurrent_gated_delta_rule_(q[:, t:t + 1].contiguous(), k[:, t:t + 1].contiguous(),
                                                    v[:, t:t + 1].contiguous(), g[:, t:t + 1].contiguous(),
                                                    b[:, t:t + 1].contiguous(), s2, out_dtype=torch.float32)
                    for t in range(2)], 1)
    assert torch.equal(o1, o2)
    assert torch.equal(s1, s2)


def test_zero_write_keeps_state_bit_exact():
    """beta = 0 and g = 0: the state must come back bit-identical and out = S^T q."""
    w = inputs.gdn_decode(B=64, steps=1)
    q, k, v = (w[n][0].to(DEV) for n in ("q", "k", "v"))
    z = torch.zeros(64, 1, 32, device=DEV)
    s = w["state"].to(DEV)
    s0 = s.clone()
    out = gdn.recurrent_gated_delta_rule_(q, k, v, z, z, s, out_dtype=torch.float32)
    assert torch.equal(s, s0)
    qe = q.float().repeat_interleave(2, dim=2)[:, 0] / (128 ** 0.5)
    ref = torch.einsum("bhkv,bhk->bhv", s0, qe)
    assert_close(out[:, 0], ref, "S^T q")


def test_equal_heads_and_empty_sequence():
    torch.manual_seed(5)
    B, T, H = 2, 5, 4
    q = F.normalize(torch.randn(B, T, H, 128), dim=-1).half()
    k = F.normalize(torch.randn(B, T, H, 128), dim=-1).half()
    v = torch.randn(B, T, H, 128).half()
    g = -F.softplus(torch.randn(B, T, H))
    b = torch.sigmoid(torch.randn(B, T, H))
    o, s = gdn.recurrent_gated_delta_rule(q.to(DEV), k.to(DEV), v.to(DEV), g.to(DEV), b.to(DEV),
                                          output_final_state=True)
    o_ref, s_ref = og.recurrent_gated_delta_rule(q, k, v, g, b)
    assert_close(o.float(), o_ref.half().float(), "out", rel_l2=2e-3)
    assert_close(s, s_ref, "state")
    st = torch.randn(B, H, 128, 128, device=DEV)
    st0 = st.clone()
    gdn.recurrent_gated_delta_rule_(q[:, :0].to(DEV), k[:, :0].to(DEV), v[:, :0].to(DEV), g[:, :0].to(DEV),
                                    b[:, :0].to(DEV), st)
    assert torch.equal(st, st0)


def test_invalid_arguments_raise():
    q = torch.zeros(1, 1, 1, 64, device=DEV, dtype=torch.half)
    with pytest.raises(RuntimeError, match="d_k"):
        gdn.recurrent_gated_delta_rule_(q, q, q, torch.zeros(1, 1, 1, device=DEV), torch.zeros(1, 1, 1, device=DEV),
                                        torch.zeros(1, 1, 64, 64, device=DEV))


def _prologue_case(B, T, use_state, seed, K=4):
    torch.manual_seed(seed)
    Hqk, Hv = 16, 32
    C = 2 * Hqk * 128 + Hv * 128
    x = torch.randn(B, T, C).bfloat16()
    w = 0.1 * torch.randn(C, K)
    cs = torch.randn(B, C, K).bfloat16() if use_state else torch.zeros(B, C, K).bfloat16()
    a = torch.randn(B, T, Hv).bfloat16()
    bb = torch.randn(B, T, Hv).bfloat16()
    A_log = torch.empty(Hv).uniform_(0, 2.77)
    dtb = 0.1 * torch.randn(Hv)
    return Hqk, Hv, x, w, cs, a, bb, A_log, dtb


@pytest.mark.parametrize("B,T,use_state,K", [(1, 512, False, 4), (2, 37, True, 4), (3, 1, True, 4), (1, 2, True, 4),
                                             (2, 3, False, 4), (2, 20, True, 6), (1, 3, True, 2), (2, 17, False, 8),
                                             (18, 1, True, 4), (33, 2, True, 4), (16, 4, False, 4)])
def test_prologue_matches_oracle(B, T, use_state, K):
    Hqk, Hv, x, w, cs, a, bb, A_log, dtb = _prologue_case(B, T, use_state, 10 + T, K)
    cs_dev = cs.to(DEV)
    q, k, v, g, beta = gdn.gdn_prologue(x.to(DEV), w.to(DEV), cs_dev, a.to(DEV), bb.to(DEV), A_log.to(DEV),
                                        dtb.to(DEV), Hqk, Hv, use_state=use_state, out_dtype=torch.float32)
    rq, rk, rv, rg, rb, rstate = og.prologue(x, a, bb, w, A_log, dtb, cs if use_state else None, Hqk, Hv, 128, 128)
    assert_close(q, rq, "q", rel_l2=1e-5, max_abs=1e-5)
    assert_close(k, rk, "k", rel_l2=1e-5, max_abs=1e-5)
    assert_close(v, rv, "v", rel_l2=1e-5, max_abs=1e-5)
    assert_close(g, rg, "g", rel_l2=1e-5, max_abs=1e-4)
    assert_close(beta, rb, "beta", rel_l2=1e-5, max_abs=1e-5)
    assert torch.equal(cs_dev.cpu(), rstate.to(torch.bfloat16)), "conv state must be bit-exact"


def test_gated_rmsnorm_matches_golden():
    n = torch.load(os.path.join(GOLDEN, "gdn.pt"))["norm"]
    y = gdn.gated_rmsnorm(n["x"].to(DEV), n["z"].to(DEV), n["weight"].to(DEV))
    assert_close(y, n["y"], "gated rmsnorm", rel_l2=1e-5, max_abs=1e-5)


def test_gdn_layer_prefill_then_decode_matches_oracle():
    """Single layer, B=1: 512-token prefill then 64 decode steps; the hot path's
    inputs are the device's own projection outputs, which the oracle re-uses."""
    w, hidden = inputs.gdn_layer()
    layer = gdn.GatedDeltaNet(dtype=torch.bfloat16, device=DEV)
    with torch.no_grad():
        for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
            getattr(layer, n).weight.copy_(w[n])
        layer.conv_weight.copy_(w["conv_w"])
        layer.A_log.copy_(w["A_log"])
        layer.dt_bias.copy_(w["dt_bias"])
        layer.norm_weight.copy_(w["norm_w"])
    params = dict(conv_w=w["conv_w"], A_log=w["A_log"], dt_bias=w["dt_bias"], norm_w=w["norm_w"])
    conv_state, rec_state = layer.new_states(1)
    h = hidden.to(DEV)
    ref_conv, ref_state = None, None
    with torch.no_grad():
        for step, (s, e) in enumerate([(0, 512)] + [(512 + i, 513 + i) for i in range(64)]):
            x = h[:, s:e]
            mixed, z, a, b = layer.in_proj_qkv(x), layer.in_proj_z(x), layer.in_proj_a(x), layer.in_proj_b(x)
            o, normed = layer.core(mixed, z, a, b, conv_state, rec_state,
                                   current_pos=0 if step == 0 else 512 + step - 1, return_core=True)
            if step == 0:
                ro, rn, ref_conv, ref_state = og.gdn_layer_prefill(mixed.cpu(), z.cpu(), a.cpu(), b.cpu(), params,
                                                                   16, 32, 128, 128)
            else:
                ro, rn, ref_conv, ref_state = og.gdn_layer_decode(mixed.cpu(), z.cpu(), a.cpu(), b.cpu(), params,
                                                                  16, 32, 128, 128, ref_conv, ref_state)
            if step in (0, 1, 64):
                assert_close(o, ro, f"core output step {step}")
                zz = z.reshape(o.shape).contiguous()
                normed32 = gdn.gated_rmsnorm(o, zz, layer.norm_weight, out_dtype=torch.float32)
                # the absolute 2e-3 bar applies to the core output and the state (checked above and
                # below); the gated-norm output is rescaled to unit RMS, so its absolute bar scales too
                assert_close(normed32, rn, f"normed step {step}", max_abs=1e-2)
                # the layer's own bf16 output: values are O(1), so one bf16 ulp is ~1e-2 absolute
                assert_close(normed.float(), rn.to(torch.bfloat16).float(), f"normed bf16 step {step}",
                             rel_l2=5e-3, max_abs=6.25e-2)
                assert torch.equal(conv_state.cpu(), ref_conv.to(torch.bfloat16)), "conv state"
                assert_close(rec_state, ref_state, f"state step {step}")


@pytest.mark.parametrize("T", [1, 3])
def test_short_prologue_batch_equals_single_sequences(T):
    """The decode-length prologue takes four sequences per CTA at batches of 16 or more: a batch of
    21 (a ragged last group) gives bit for bit what 21 one-sequence calls give."""
    B = 21
    Hqk, Hv, x, w, cs, a, bb, A_log, dtb = _prologue_case(B, T, True, 70 + T)
    args = (w.to(DEV), A_log.to(DEV), dtb.to(DEV))
    cs_all = cs.to(DEV)
    got = gdn.gdn_prologue(x.to(DEV), args[0], cs_all, a.to(DEV), bb.to(DEV), args[1], args[2], Hqk, Hv,
                           use_state=True)
    for b in range(B):
        cs_b = cs[b:b + 1].to(DEV)
        ref = gdn.gdn_prologue(x[b:b + 1].to(DEV), args[0], cs_b, a[b:b + 1].to(DEV), bb[b:b + 1].to(DEV), args[1],
                               args[2], Hqk, Hv, use_state=True)
        for g_, r_ in zip(got, ref):
            assert torch.equal(g_[b:b + 1], r_), f"sequence {b}"
        assert torch.equal(cs_all[b:b + 1], cs_b), f"conv state {b}"


@pytest.mark.parametrize("T,use_state", [(1, True), (3, True), (200, False)])
def test_prologue_and_gated_norm_read_projection_slices(T, use_state):
    """The layer's fused [qkv | z | b | a] projection output read in place (token-strided column
    slices) gives bit-for-bit the results of dense copies of the same slices."""
    Hqk, Hv, x, w, cs, a, bb, A_log, dtb = _prologue_case(2, T, use_state, 50 + T)
    C = x.shape[-1]
    z = torch.randn(2, T, Hv * 128).bfloat16()
    fused = torch.cat([x, z, bb, a], dim=-1).to(DEV)
    xs, zs = fused[..., :C], fused[..., C:C + Hv * 128]
    bs, as_ = fused[..., C + Hv * 128:C + Hv * 128 + Hv], fused[..., C + Hv * 128 + Hv:]
    cs1, cs2 = cs.to(DEV), cs.to(DEV)
    args = (w.to(DEV), A_log.to(DEV), dtb.to(DEV))
    got = gdn.gdn_prologue(xs, args[0], cs1, as_, bs, args[1], args[2], Hqk, Hv, use_state=use_state)
    ref = gdn.gdn_prologue(xs.contiguous(), args[0], cs2, as_.contiguous(), bs.contiguous(), args[1], args[2], Hqk,
                           Hv, use_state=use_state)
    for g_, r_ in zip(got, ref):
        assert torch.equal(g_, r_)
    assert torch.equal(cs1, cs2)
    o = torch.randn(2, T, Hv, 128, device=DEV)
    nw = torch.rand(128, device=DEV) + 0.5
    n1 = gdn.gated_rmsnorm(o, zs.view(2, T, Hv, 128), nw, out_dtype=torch.bfloat16)
    n2 = gdn.gated_rmsnorm(o, zs.contiguous().view(2, T, Hv, 128), nw, out_dtype=torch.bfloat16)
    assert torch.equal(n1, n2)


def test_layer_continues_a_prefill_from_its_states():
    """``current_pos`` > 0 continues from the caller's states: a 512-token prefill split into calls at
    positions 0 and 256 (chunk-aligned) gives bit for bit the core outputs, conv state and recurrent
    state of one call; the position may be a one-element tensor, as the reference passes it."""
    w, hidden = inputs.gdn_layer()
    layer = gdn.GatedDeltaNet(dtype=torch.bfloat16, device=DEV)
    with torch.no_grad():
        layer.w_in.copy_(torch.cat([w["in_proj_qkv"], w["in_proj_z"], w["in_proj_b"], w["in_proj_a"]]))
        layer.conv_weight.copy_(w["conv_w"])
        layer.A_log.copy_(w["A_log"])
        proj = F.linear(hidden[:, :512].to(DEV), layer.w_in)
        c, v, H = layer.conv_dim, layer.value_dim, layer.num_v_heads
        parts = lambda s, e: (proj[:, s:e, :c], proj[:, s:e, c:c + v], proj[:, s:e, c + v + H:],
                              proj[:, s:e, c + v:c + v + H])
        one = layer.new_states(1)
        o1, n1 = layer.core(*parts(0, 512), *one, current_pos=0, return_core=True)
        two = layer.new_states(1)
        two[1].fill_(1.0)  # position 0 resets the recurrent state
        oa, na = layer.core(*parts(0, 256), *two, current_pos=0, return_core=True)
        ob, nb = layer.core(*parts(256, 512), *two, current_pos=torch.tensor([256], dtype=torch.int32),
                            return_core=True)
    assert torch.equal(torch.cat([oa, ob], 1), o1) and torch.equal(torch.cat([na, nb], 1), n1)
    assert torch.equal(two[0], one[0]) and torch.equal(two[1], one[1])
