"""The torch operator registrations (``torch.ops.anemll_b200.*``) give bit for bit what the direct
calls through the C ABI give, and update the declared state in place."""
import pytest
import torch
import torch.nn.functional as F

import anemll_b200.ops  # noqa: F401
from anemll_b200 import attention, gdn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _gdn_inputs(T, seed):
    g = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(2, T, 2, 128, generator=g), dim=-1).half().to(DEV)
    k = F.normalize(torch.randn(2, T, 2, 128, generator=g), dim=-1).half().to(DEV)
    v = torch.randn(2, T, 4, 128, generator=g).half().to(DEV)
    gg = (-F.softplus(torch.randn(2, T, 4, generator=g))).to(DEV)
    beta = torch.sigmoid(torch.randn(2, T, 4, generator=g)).to(DEV)
    s0 = (0.01 * torch.randn(2, 4, 128, 128, generator=g)).to(DEV)
    return q, k, v, gg, beta, s0


@pytest.mark.parametrize("op,T", [("gdn_chunked_prefill", 130), ("gdn_recurrent", 3)])
def test_gdn_ops_equal_direct_calls(op, T):
    q, k, v, g, beta, s0 = _gdn_inputs(T, T)
    s_op, s_dir = s0.clone(), s0.clone()
    o_op = getattr(torch.ops.anemll_b200, op)(q, k, v, g, beta, s_op)
    direct = gdn.chunk_gated_delta_rule_ if op == "gdn_chunked_prefill" else gdn.recurrent_gated_delta_rule_
    o_dir = direct(q, k, v, g, beta, s_dir)
    assert torch.equal(o_op, o_dir) and torch.equal(s_op, s_dir)
    assert not torch.equal(s_op, s0)


def test_prologue_and_kv_ops_equal_direct_calls():
    g = torch.Generator().manual_seed(5)
    Hqk, Hv, B, T = 2, 4, 2, 8
    C = 2 * Hqk * 128 + Hv * 128
    x = torch.randn(B, T, C, generator=g).bfloat16().to(DEV)
    w = (0.1 * torch.randn(C, 4, generator=g)).to(DEV)
    a = torch.randn(B, T, Hv, generator=g).bfloat16().to(DEV)
    b = torch.randn(B, T, Hv, generator=g).bfloat16().to(DEV)
    A_log = torch.rand(Hv, generator=g).to(DEV)
    cs = torch.randn(B, C, 4, generator=g).bfloat16().to(DEV)
    cs_op, cs_dir = cs.clone(), cs.clone()
    r_op = torch.ops.anemll_b200.gdn_prologue(x, w, cs_op, a, b, A_log, None, Hqk, Hv)
    r_dir = gdn.gdn_prologue(x, w, cs_dir, a, b, A_log, None, Hqk, Hv)
    assert all(torch.equal(u, v) for u, v in zip(r_op, r_dir)) and torch.equal(cs_op, cs_dir)
    Hq, Hkv, hd, ctx, S, pos = 8, 2, 128, 256, 16, 40
    cache = torch.randn(2, 1, Hkv, ctx, hd, generator=g).half().to(DEV)
    qa = torch.randn(1, Hq, S, hd, generator=g).half().to(DEV)
    kn, vn = (torch.randn(1, Hkv, S, hd, generator=g).half().to(DEV) for _ in range(2))
    c_op, c_dir = cache.clone(), cache.clone()
    o_op = torch.ops.anemll_b200.kv_attention(qa, c_op[0], c_op[1], pos, kn, vn)
    o_dir = attention.kv_attention(qa, c_dir[0], c_dir[1], pos, k_new=kn, v_new=vn)
    assert torch.equal(o_op, o_dir) and torch.equal(c_op, c_dir)
