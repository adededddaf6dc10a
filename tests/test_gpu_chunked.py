"""GPU parity of the tcgen05 chunked-prefill kernel (through the C ABI)."""
import math
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


def _no_device_error():
    torch.cuda.synchronize()
    assert gdn.chunked_device_error(reset=True) == 0, "a bounded wait ran out inside the chunked kernel"


def _case(B, T, Hqk, Hv, seed, dtype=torch.bfloat16, s0=0.0):
    torch.manual_seed(seed)
    A_log = torch.empty(Hv).uniform_(0.0, math.log(16.0))
    q = F.normalize(torch.randn(B, T, Hqk, 128), dim=-1).to(dtype)
    k = F.normalize(torch.randn(B, T, Hqk, 128), dim=-1).to(dtype)
    v = torch.randn(B, T, Hv, 128).to(dtype)
    g = (-F.softplus(torch.randn(B, T, Hv)) * torch.exp(A_log)).float()
    beta = torch.sigmoid(torch.randn(B, T, Hv)).float()
    S0 = s0 * torch.randn(B, Hv, 128, 128)
    return q, k, v, g, beta, S0


def _run(q, k, v, g, beta, S0, l2=False, out_dtype=torch.float32):
    st = S0.to(DEV).contiguous()
    o = gdn.chunk_gated_delta_rule_(q.to(DEV), k.to(DEV), v.to(DEV), g.to(DEV), beta.to(DEV), st,
                                    use_qk_l2norm_in_kernel=l2, out_dtype=out_dtype)
    _no_device_error()
    return o, st


def test_matches_golden_fixture():
    d = torch.load(os.path.join(GOLDEN, "gdn.pt"))["gdn"]
    o, st = _run(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], l2=True)
    assert_close(o, d["out_chunk"], "out")
    assert_close(st, d["state_chunk"], "state")


@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
def test_ragged_lengths_match_oracle(T):
    q, k, v, g, beta, S0 = _case(2, T, 2, 4, 100 + T, s0=0.01)
    o, st = _run(q, k, v, g, beta, S0)
    ro, rs = og.chunk_gated_delta_rule(q, k, v, g, beta, 64, S0)
    assert_close(o, ro, f"out T={T}")
    assert_close(st, rs, f"state T={T}")


def test_full_head_shape_long_sequence():
    """H_qk=16, H_v=32, d=128, one 4096-token sequence (bf16 inputs, fp32 carry)."""
    q, k, v, g, beta, S0 = _case(1, 4096, 16, 32, 3)
    o, st = _run(q, k, v, g, beta, S0)
    ro, rs = og.chunk_gated_delta_rule(q, k, v, g, beta, 64, S0)
    assert_close(o, ro, "out")
    assert_close(st, rs, "state")


@pytest.mark.parametrize("dtype,s0", [(torch.bfloat16, 0.0), (torch.float16, 0.01)])
def test_long_prefill_full_sequence_matches_oracle(dtype, s0):
    """One whole sequence of the long-prefill workload: 32768 tokens (512 chunks of state carry) with
    all 32 value heads, seed 3, against the fp32 oracle.  bf16 inputs from a zero state (the
    workload's own form), and fp16 inputs from a non-zero state (the gated-DeltaNet layer feeds the
    kernel fp16 q/k/v)."""
    q, k, v, g, beta, S0 = _case(1, 32768, 16, 32, 3, dtype=dtype, s0=s0)
    o, st = _run(q, k, v, g, beta, S0)
    ro, rs = og.chunk_gated_delta_rule(q, k, v, g, beta, 64, S0)
    assert_close(o, ro, "out")
    assert_close(st, rs, "state")


def test_fp16_and_bf16_outputs():
    q, k, v, g, beta, S0 = _case(1, 256, 2, 4, 9, dtype=torch.float16, s0=0.01)
    ro, rs = og.chunk_gated_delta_rule(q, k, v, g, beta, 64, S0)
    o16, _ = _run(q, k, v, g, beta, S0, out_dtype=torch.float16)
    assert_close(o16.float(), ro.half().float(), "fp16 out")
    ob, _ = _run(q, k, v, g, beta, S0, out_dtype=torch.bfloat16)
    assert_close(ob.float(), ro.bfloat16().float(), "bf16 out", rel_l2=5e-3)


def test_split_at_chunk_boundary_is_bit_exact():
    """Size-independent property: T tokens in one call == the first 64*m tokens,
    then the rest with the carried state (identical chunk arithmetic)."""
    q, k, v, g, beta, S0 = _case(4, 1000, 4, 8, 11, s0=0.01)
    o1, s1 = _run(q, k, v, g, beta, S0)
    st = S0.to(DEV).contiguous()
    cut = 640
    parts = []
    for a, b in ((0, cut), (cut, 1000)):
        parts.append(gdn.chunk_gated_delta_rule_(*(x[:, a:b].contiguous().to(DEV) for x in (q, k, v, g, beta)), st,
                                                 out_dtype=torch.float32))
    _no_device_error()
    assert torch.equal(o1, torch.cat(parts, 1))
    assert torch.equal(s1, st)


def test_chunked_agrees_with_recurrent_kernel_at_full_prefill_shape():
    """The long-prefill head shape on the device only (no CPU oracle): B=8 sequences of 8192
    tokens, chunked vs token-recurrent kernel, both against each other."""
    w = inputs.gdn_prefill_device(B=8, T=8192)
    s_c = torch.zeros(8, 32, 128, 128, device=DEV)
    s_r = torch.zeros_like(s_c)
    o_c = gdn.chunk_gated_delta_rule_(w["q"], w["k"], w["v"], w["g"], w["beta"], s_c, out_dtype=torch.float32)
    o_r = gdn.recurrent_gated_delta_rule_(w["q"], w["k"], w["v"], w["g"], w["beta"], s_r, out_dtype=torch.float32)
    _no_device_error()
    assert_close(o_c, o_r, "out")
    assert_close(s_c, s_r, "state")


def test_empty_and_invalid():
    st = torch.randn(1, 2, 128, 128, device=DEV)
    s0 = st.clone()
    e = torch.empty(1, 0, 1, 128, device=DEV, dtype=torch.half)
    gdn.chunk_gated_delta_rule_(e, e, torch.empty(1, 0, 2, 128, device=DEV, dtype=torch.half),
                                torch.empty(1, 0, 2, device=DEV), torch.empty(1, 0, 2, device=DEV), st)
    assert torch.equal(st, s0)
    q = torch.zeros(1, 4, 1, 128, device=DEV)
    with pytest.raises(RuntimeError, match="f16 or bf16"):
        gdn.chunk_gated_delta_rule_(q, q, torch.zeros(1, 4, 2, 128, device=DEV), torch.zeros(1, 4, 2, device=DEV),
                                    torch.zeros(1, 4, 2, device=DEV), st)


@pytest.mark.parametrize("B,T,Hqk,Hv,l2,dtype", [(2, 300, 2, 4, False, torch.bfloat16), (1, 130, 2, 4, True, torch.float16),
                                                 (1, 2048, 16, 32, False, torch.bfloat16)])
def test_pipelined_and_two_chain_kernels_agree_bitwise(B, T, Hqk, Hv, l2, dtype):
    """The one-chain-per-SM kernel (the next chunk's state-independent work pipelined under the current
    chunk's state chain) and the two-chains-per-SM kernel run the same arithmetic: outputs and final
    states are equal bit for bit, in the plain and the gated form, with ragged last chunks and the
    in-kernel l2 norm."""
    from anemll_b200 import _lib
    lib = _lib.load()
    q, k, v, g, beta, S0 = _case(B, T, Hqk, Hv, seed=T, dtype=dtype, s0=0.01)
    if l2:
        q, k = (2.0 * q.float()).to(dtype), (0.5 * k.float()).to(dtype)
    z = torch.randn(B, T, Hv, 128).to(dtype).to(DEV)
    w = (1.0 + 0.1 * torch.randn(128)).to(DEV)
    prev = lib.anemll_gdn_chunked_mode(0)
    try:
        res = {}
        for mode in (1, 2):
            lib.anemll_gdn_chunked_mode(mode)
            o, st = _run(q, k, v, g, beta, S0, l2=l2)
            s2 = S0.to(DEV).contiguous()
            y = gdn.gated_delta_rule_norm_(q.to(DEV), k.to(DEV), v.to(DEV), g.to(DEV), beta.to(DEV), s2, z, w,
                                           chunked=True, use_qk_l2norm_in_kernel=l2)
            _no_device_error()
            res[mode] = (o, st, y, s2)
    finally:
        lib.anemll_gdn_chunked_mode(prev)
    for a, b_ in zip(res[1], res[2]):
        assert torch.equal(a, b_)
