"""The delta rule followed by the layer's gated RMSNorm (``gated_delta_rule_norm_``: the chunked
prefill with the norm in its epilogue, ``anemll_gdn_chunked_prefill_gated``, and the recurrent kernel
followed by ``anemll_gated_rmsnorm``) against the unfused calls and the CPU oracle.

* The core output the fused launch also writes (``core_out``) and the updated state are bit for bit
  those of the plain kernel: the epilogue only adds the norm.
* The normed output against the oracle's fp32 gated RMSNorm of that core output: within the parity
  bar beyond the rounding of the 2-byte output itself (rel-L2 at most the rounding floor + 1e-3,
  every element within one ulp of the output type + 2e-3).
* The unfused path (plain kernel, then ``gated_rmsnorm``) and the fused one differ only in the order
  of the sum of squares: every element within one ulp of the output type.
* z read in place as a column slice of a wider projection output gives the contiguous result.

Shapes cover the chunked kernels (the pipelined one-chain-per-SM kernel at these chain counts) with
a ragged last chunk, and the recurrent path with its narrow (16-column) and wide (32-column) slice
grids, one and several tokens per launch.
"""
import pytest
import torch
import torch.nn.functional as F

import anemll_b200.ops  # noqa: F401
from anemll_b200 import gdn
from oracle import gdn as og
from tests.tolerance import errors

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ulp(x, dtype):
    """Spacing of ``dtype`` numbers at |x| (normal range)."""
    mant = 8 if dtype == torch.bfloat16 else 11
    _, e = torch.frexp(x.float())
    return torch.ldexp(torch.ones_like(x.float()), e - mant)


def _inputs(B, T, Hqk, Hv, seed, dtype=torch.bfloat16, wide_z=True):
    g = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(B, T, Hqk, 128, generator=g), dim=-1).to(dtype).to(DEV)
    k = F.normalize(torch.randn(B, T, Hqk, 128, generator=g), dim=-1).to(dtype).to(DEV)
    v = torch.randn(B, T, Hv, 128, generator=g).to(dtype).to(DEV)
    A = torch.empty(Hv).uniform_(0.0, 2.77, generator=g)  # log 1 .. log 16
    gg = (-F.softplus(torch.randn(B, T, Hv, generator=g)) * A.exp()).to(DEV)
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=g)).to(DEV)
    s0 = (0.01 * torch.randn(B, Hv, 128, 128, generator=g)).to(DEV)
    # z as a column slice of a [B, T, extra | H_v*128 | extra] projection output (token rows 16-byte aligned)
    proj = torch.randn(B, T, 64 + Hv * 128 + 64, generator=g).to(dtype).to(DEV)
    z = proj[..., 64:64 + Hv * 128].reshape(B, T, Hv, 128) if wide_z else proj[..., 64:64 + Hv * 128].contiguous().reshape(B, T, Hv, 128)
    w = (1.0 + 0.1 * torch.randn(128, generator=g)).to(DEV)
    return q, k, v, gg, beta, s0, z, w


CASES = [  # (B, T, H_qk, H_v, chunked)
    (2, 200, 2, 4, True),     # two full chunks and a ragged one
    (1, 64, 16, 32, True),    # the full head shape, one chunk
    (2, 1, 2, 4, False),      # narrow recurrent grid (16-column slices)
    (3, 5, 2, 4, False),      # several tokens per launch
    (4, 1, 16, 32, False),    # wide grid (32-column slices)
]


@pytest.mark.parametrize("B,T,Hqk,Hv,chunked", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_gated_norm_matches_plain_kernel_and_oracle(B, T, Hqk, Hv, chunked, dtype):
    q, k, v, g, beta, s0, z, w = _inputs(B, T, Hqk, Hv, seed=B * 1000 + T, dtype=dtype)
    eps = 1e-6
    s_plain, s_fused = s0.clone(), s0.clone()
    plain = gdn.chunk_gated_delta_rule_ if chunked else gdn.recurrent_gated_delta_rule_
    o = plain(q, k, v, g, beta, s_plain, out_dtype=torch.float32)
    core = torch.empty(B, T, Hv, 128, dtype=torch.float32, device=DEV)
    y = gdn.gated_delta_rule_norm_(q, k, v, g, beta, s_fused, z, w, eps, chunked=chunked, core_out=core)
    torch.cuda.synchronize()
    assert y.dtype == dtype and y.shape == (B, T, Hv, 128)
    assert torch.equal(core, o), "core output differs from the plain kernel's"
    assert torch.equal(s_fused, s_plain), "state differs from the plain kernel's"
    # against the oracle's fp32 gated norm of the same core output
    want = og.gated_rmsnorm(o.cpu(), z.float().cpu(), w.cpu(), eps)
    got = y.float().cpu()
    rel_floor, _ = errors(want.to(dtype), want)
    rel, _ = errors(got, want)
    assert rel <= rel_floor + 1e-3, f"rel_l2 {rel:.3e} (rounding floor {rel_floor:.3e})"
    over = ((got - want).abs() - _ulp(want, dtype) - 2e-3).max().item()
    assert over <= 0, f"an element {over:.3e} beyond one ulp + 2e-3"
    # against the unfused path: same values up to the order of the sum of squares
    y_unfused = gdn.gated_rmsnorm(o, z, w, eps, out_dtype=dtype)
    d = (y.float() - y_unfused.float()).abs()
    assert (d <= _ulp(torch.maximum(y.float().abs(), y_unfused.float().abs()), dtype)).all()
    if chunked and gdn.chunked_device_error(reset=True):
        raise AssertionError("chunked kernel reported a wait time-out")


@pytest.mark.parametrize("chunked", [True, False])
def test_z_column_slice_equals_contiguous_z(chunked):
    T = 130 if chunked else 2
    args = _inputs(2, T, 2, 4, seed=7)
    q, k, v, g, beta, s0, z, w = args
    zc = z.contiguous()
    assert not z.is_contiguous()
    s1, s2 = s0.clone(), s0.clone()
    y1 = gdn.gated_delta_rule_norm_(q, k, v, g, beta, s1, z, w, chunked=chunked)
    y2 = gdn.gated_delta_rule_norm_(q, k, v, g, beta, s2, zc, w, chunked=chunked)
    assert torch.equal(y1, y2) and torch.equal(s1, s2)


def test_torch_op_equals_direct_call():
    q, k, v, g, beta, s0, z, w = _inputs(2, 70, 2, 4, seed=9)
    s1, s2 = s0.clone(), s0.clone()
    y1 = torch.ops.anemll_b200.gdn_gated_delta_rule_norm(q, k, v, g, beta, s1, z, w, 1e-6, True)
    y2 = gdn.gated_delta_rule_norm_(q, k, v, g, beta, s2, z, w, 1e-6, chunked=True)
    assert torch.equal(y1, y2) and torch.equal(s1, s2)
