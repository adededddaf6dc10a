"""The stack's fused epilogue kernels against the CPU oracle's restatement of the framework ops they
replace (through the C ABI).  Moves and residual sums are bit-exact; normalised outputs are rounded
to bf16 once on both sides from fp32 values that differ only in summation order, so they agree to
bf16 rounding."""
import pytest
import torch
import torch.nn.functional as F

from oracle import stack as ost
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_RTOL, BF16_ATOL = 4e-3, 3e-2  # one bf16 rounding flip is 2^-8 relative


@pytest.mark.parametrize("rows,d", [(1, 2048), (37, 2048), (300, 512), (5, 4096), (3, 264)])
def test_rmsnorm_and_residual_add(rows, d):
    from anemll_b200.stack import rms_norm
    g = torch.Generator().manual_seed(rows + d)
    x = torch.randn(rows, d, generator=g).bfloat16()
    r = torch.randn(rows, d, generator=g).bfloat16()
    w = 1 + 0.1 * torch.randn(d, generator=g)
    out = rms_norm(x.to(DEV), w.to(DEV), 1e-6)
    assert_close(out.float().cpu(), ost.bf(ost.rms_norm(x.float(), w, 1e-6)), "rmsnorm", BF16_RTOL, BF16_ATOL)
    s, out = rms_norm(x.to(DEV), w.to(DEV), 1e-6, residual=r.to(DEV))
    ref_s = ost.bf(x.float() + r.float())
    assert torch.equal(s.float().cpu(), ref_s)
    assert_close(out.float().cpu(), ost.bf(ost.rms_norm(ref_s, w, 1e-6)), "add+rmsnorm", BF16_RTOL, BF16_ATOL)


def test_silu_mul():
    from anemll_b200.stack import silu_mul
    g = torch.Generator().manual_seed(3)
    gu = (3 * torch.randn(2, 7, 2 * 6144, generator=g)).bfloat16()
    out = silu_mul(gu.to(DEV))
    gate, up = gu.float().chunk(2, dim=-1)
    assert_close(out.float().cpu(), ost.bf(ost.bf(F.silu(gate)) * up), "silu_mul", BF16_RTOL, BF16_ATOL)


@pytest.mark.parametrize("hd,T,pos", [(256, 1, 1000), (256, 37, 0), (128, 9, 77)])
def test_qk_norm_rope_matches_oracle(hd, T, pos):
    from anemll_b200 import _lib
    from anemll_b200.stack import rope_tables
    g = torch.Generator().manual_seed(hd + T)
    B, Hq, Hkv, eps = 2, 16, 2, 1e-6
    n_q, n_kv = Hq * 2 * hd, Hkv * hd
    qkv = torch.randn(B, T, n_q + 2 * n_kv, generator=g).bfloat16()
    qw = 1 + 0.1 * torch.randn(hd, generator=g)
    kw = 1 + 0.1 * torch.randn(hd, generator=g)
    cos, sin = rope_tables(hd, 2048, 1e7, "cpu")
    d = {n: t.to(DEV) for n, t in dict(qkv=qkv, qw=qw, kw=kw, cos=cos, sin=sin).items()}
    q = torch.empty(B, Hq, T, hd, dtype=torch.bfloat16, device=DEV)
    k = torch.empty(B, Hkv, T, hd, dtype=torch.bfloat16, device=DEV)
    v = torch.empty_like(k)
    gate = torch.empty(B, T, Hq * hd, dtype=torch.bfloat16, device=DEV)
    base, es, ld = d["qkv"].data_ptr(), 2, qkv.shape[-1]
    rc = _lib.load().anemll_qk_norm_rope(base, ld, base + n_q * es, ld, base + (n_q + n_kv) * es, ld,
                                         _lib.ptr(d["qw"]), _lib.ptr(d["kw"]), _lib.ptr(d["cos"]), _lib.ptr(d["sin"]),
                                         _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(gate), _lib.BF16, B, T, Hq,
                                         Hkv, hd, pos, eps, _lib.stream_ptr(DEV))
    _lib.check(rc, "anemll_qk_norm_rope")
    f = qkv.float()
    qg = f[..., :n_q].view(B, T, Hq, 2 * hd)
    rq = ost.bf(ost.rms_norm(qg[..., :hd], qw, eps)).transpose(1, 2)
    rk = ost.bf(ost.rms_norm(f[..., n_q:n_q + n_kv].view(B, T, Hkv, hd), kw, eps)).transpose(1, 2)
    c, s = cos[pos:pos + T], sin[pos:pos + T]
    assert_close(q.float().cpu(), ost.bf(ost.rope(rq, c, s)), "q", BF16_RTOL, BF16_ATOL)
    assert_close(k.float().cpu(), ost.bf(ost.rope(rk, c, s)), "k", BF16_RTOL, BF16_ATOL)
    assert torch.equal(v.float().cpu(), f[..., n_q + n_kv:].view(B, T, Hkv, hd).transpose(1, 2))
    assert torch.equal(gate.float().cpu(), qg[..., hd:].reshape(B, T, Hq * hd))


def test_stack_op_errors():
    from anemll_b200.stack import rms_norm
    with pytest.raises(RuntimeError, match="multiple of 8"):
        rms_norm(torch.zeros(2, 12, device=DEV, dtype=torch.bfloat16), torch.ones(12, device=DEV), 1e-6)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        rms_norm(torch.zeros(2, 16), torch.ones(16), 1e-6)


@pytest.mark.parametrize("S,pos,B", [(64, 0, 2), (32, 100, 2), (1, 300, 3), (1, 0, 1), (256, 512, 1)])
def test_fused_attention_prologue_is_bit_exact(S, pos, B):
    """anemll_kv_attention_qkv (head norm + RoPE inside the attention call) gives the bits of the
    separate prologue kernel followed by anemll_kv_attention: output and cache."""
    from anemll_b200 import attention
    from anemll_b200.stack import rope_tables
    g = torch.Generator().manual_seed(S * 7 + pos)
    Hq, Hkv, hd, ctx, eps = 16, 2, 256, 1024, 1e-6
    n_q, n_kv = Hq * 2 * hd, Hkv * hd
    wide = torch.randn(B, S, n_q + 2 * n_kv + 16, generator=g).bfloat16().to(DEV)  # rows spaced by 16 extra
    qkv = wide[..., :n_q + 2 * n_kv]
    qw = (1 + 0.1 * torch.randn(hd, generator=g)).to(DEV)
    kw = (1 + 0.1 * torch.randn(hd, generator=g)).to(DEV)
    cos, sin = (t.to(DEV) for t in rope_tables(hd, ctx, 1e7, "cpu"))
    cache = torch.randn(2, B, Hkv, ctx, hd, generator=g).bfloat16().to(DEV)
    ca, cb = cache.clone(), cache.clone()
    out = attention.kv_attention_qkv(qkv, qw, kw, cos, sin, eps, ca[0], ca[1], pos, Hq, Hkv, hd)
    assert out is not None
    q = torch.empty(B, Hq, S, hd, dtype=torch.bfloat16, device=DEV)
    k = torch.empty(B, Hkv, S, hd, dtype=torch.bfloat16, device=DEV)
    v = torch.empty_like(k)
    gate = torch.empty(B, S, Hq * hd, dtype=torch.bfloat16, device=DEV)
    from anemll_b200 import _lib
    base, ld = qkv.data_ptr(), qkv.stride(1) if S > 1 else qkv.stride(0)
    rc = _lib.load().anemll_qk_norm_rope(base, ld, base + n_q * 2, ld, base + (n_q + n_kv) * 2, ld, _lib.ptr(qw),
                                         _lib.ptr(kw), _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(q), _lib.ptr(k),
                                         _lib.ptr(v), _lib.ptr(gate), _lib.BF16, B, S, Hq, Hkv, hd, pos, eps,
                                         _lib.stream_ptr(DEV))
    _lib.check(rc, "anemll_qk_norm_rope")
    ref = attention.kv_attention(q, cb[0], cb[1], pos, k_new=k, v_new=v, gate=gate)
    assert torch.equal(out, ref)
    assert torch.equal(ca, cb)
    assert attention.kv_device_error() == 0


def test_fused_attention_prologue_declines_other_shapes():
    from anemll_b200 import attention
    from anemll_b200.stack import rope_tables
    Hq, Hkv, hd, ctx = 16, 2, 256, 256
    qkv = torch.zeros(1, 4, Hq * 2 * hd + 2 * Hkv * hd, dtype=torch.bfloat16, device=DEV)  # 4 tokens: neither path
    cos, sin = (t.to(DEV) for t in rope_tables(hd, ctx, 1e7, "cpu"))
    cache = torch.zeros(2, 1, Hkv, ctx, hd, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(hd, device=DEV)
    assert attention.kv_attention_qkv(qkv, w, w, cos, sin, 1e-6, cache[0], cache[1], 0, Hq, Hkv, hd) is None
