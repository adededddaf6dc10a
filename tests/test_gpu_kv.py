"""GPU parity of the fused KV-cache attention kernel against the oracle (through the C ABI)."""
import os

import pytest
import torch

from anemll_b200 import attention, inputs
from oracle import kv_attention as ok
from tests.conftest import GOLDEN
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def gold():
    return torch.load(os.path.join(GOLDEN, "kv_attention.pt"))


@pytest.mark.parametrize("use_mask", [True, False])
def test_matches_reference_golden(gold, use_mask):
    hd, ctx, Hkv = gold["hd"], gold["ctx"], gold["Hkv"]
    for c in gold["cases"]:
        S, pos = c["S"], c["pos"]
        K = torch.zeros(Hkv, ctx, hd, dtype=torch.half)
        V = torch.zeros(Hkv, ctx, hd, dtype=torch.half)
        K[:, :pos + S] = c["K"]
        V[:, :pos + S] = c["V"]
        mask = None
        if use_mask:
            mask = torch.zeros(1, 1, S, ctx).masked_fill(~c["visible"].view(1, 1, S, ctx), float("-inf")).half()
            mask = mask.to(DEV)
        att = attention.QwenAttentionB200(gold["Hq"], Hkv, hd, window=c["window"],
                                          window_chunk_aligned=c["chunk_aligned"])
        args = (None, c["q"].to(DEV), (K.to(DEV), V.to(DEV)), mask)
        if S == 1:
            out = att.forward_regular(*args, current_pos=pos)
        else:
            out = att.forward_prefill(*args, current_pos=pos)
        assert_close(out.float(), c["out"], c["name"])


@pytest.mark.parametrize("o_proj_form", ["conv2d", "weight"])
def test_drop_in_module_returns_the_reference_projected_output(o_proj_form):
    """The module built around the reference's own o_proj (a 1x1 Conv2d, or its weight) returns what
    QwenAttention.forward_prefill / forward_regular return: o_proj(attention), [B, S, hidden]
    (golden from the reference with a random o_proj), with the reference's own argument forms: the
    additive causal mask and current_pos as a one-element tensor."""
    fx = torch.load(os.path.join(GOLDEN, "kv_attention_oproj.pt"))
    Hq, Hkv, hd, ctx, hidden = fx["Hq"], fx["Hkv"], fx["hd"], fx["ctx"], fx["hidden"]
    conv = torch.nn.Conv2d(Hq * hd, hidden, 1, bias=False).to(DEV)
    with torch.no_grad():
        conv.weight.copy_(fx["o_proj_weight"])
    att = attention.QwenAttentionB200(Hq, Hkv, hd, o_proj=conv if o_proj_form == "conv2d" else conv.weight)
    for c in fx["cases"]:
        S, pos = c["S"], c["pos"]
        K = torch.zeros(Hkv, ctx, hd, dtype=torch.half)
        V = torch.zeros(Hkv, ctx, hd, dtype=torch.half)
        K[:, :pos + S] = c["K"]
        V[:, :pos + S] = c["V"]
        mask = ok.additive_mask(S, ctx, pos).half().to(DEV)
        hs = torch.zeros(1, S, hidden, dtype=torch.half, device=DEV)
        args = (hs, c["q"].to(DEV), (K.to(DEV), V.to(DEV)), mask)
        if S == 1:
            out = att.forward_regular(*args, torch.tensor([pos], dtype=torch.int32))
        else:
            out = att.forward_prefill(*args)
        assert out.shape == (1, S, hidden)
        assert_close(out.float(), c["out"], c["name"])
        core = att.attention(c["q"].to(DEV), (K.to(DEV), V.to(DEV)), mask, pos)
        assert torch.equal(att.project(core), out)


def test_fused_cache_write_bit_exact_vs_reference():
    fx = torch.load(os.path.join(GOLDEN, "kv_cache_write.pt"))
    for w in fx["writes"]:
        cache = w["before"].to(DEV)
        L, Hkv, ctx, hd = cache.shape[0] // 2, cache.shape[1], cache.shape[2], cache.shape[3]
        S = w["S"]
        q = torch.randn(1, 4, S, hd, dtype=torch.half, device=DEV)
        att = attention.QwenAttentionB200(4, Hkv, hd)
        att.process_layer_step(cache, w["layer_idx"], w["num_layers"], q, w["k"].to(DEV), w["v"].to(DEV), w["pos"])
        assert torch.equal(cache.cpu(), w["after"]), w["name"]


@pytest.mark.parametrize("window", [0, 512])
def test_chunked_prefill_and_decode_over_a_4096_cache(window):
    """H_q=16, H_kv=2, hd=256, ctx 4096, fp16: 31 x 64-token chunks at 2048..4031, then
    64 decode steps at 4032..4095, causal and 512-token sliding window; every
    output within tolerance, the final cache bit-exact."""
    d = inputs.kv_attention()
    cache_dev = d["cache"].clone().to(DEV)  # [2, Hkv, ctx, hd]: a one-layer unified cache
    cache_ref = d["cache"].float().clone()
    att = attention.QwenAttentionB200(16, 2, 256, window=window)
    pos = d["prefill_from"]
    steps = [(p, 64) for p in range(pos, d["prefill_to"], 64)] + [(p, 1) for p in range(d["prefill_to"], 4096)]
    worst = 0.0
    for i, (p, S) in enumerate(steps):
        j = p - pos
        q = d["q"][:, :, j:j + S]
        k = d["k"][:, :, j:j + S]
        v = d["v"][:, :, j:j + S]
        gte = d["gate"][:, j:j + S]
        out = att.process_layer_step(cache_dev, 0, 1, q.to(DEV), k.to(DEV), v.to(DEV), p, gate=gte.to(DEV))
        if i % 4 == 0 or S == 1 and i % 8 == 0 or i == len(steps) - 1:
            ref = ok.kv_attention_step(q, k, v, gte, cache_ref, 0, 1, p, window)
            rel, _ = assert_close(out.float(), ref, f"step {i} pos {p}")
            worst = max(worst, rel)
        else:
            ok.write_cache(cache_ref, k, v, 0, 1, p)
    assert torch.equal(cache_dev.cpu(), cache_ref.half())
    assert attention.kv_device_error() == 0


def test_batched_cache_and_workspace_errors():
    torch.manual_seed(7)
    B, Hq, Hkv, hd, ctx, S, pos = 3, 8, 2, 128, 512, 16, 200
    kc = torch.randn(B, Hkv, ctx, hd).half()
    vc = torch.randn(B, Hkv, ctx, hd).half()
    q = torch.randn(B, Hq, S, hd).half()
    kn = torch.randn(B, Hkv, S, hd).half()
    vn = torch.randn(B, Hkv, S, hd).half()
    kd, vd = kc.to(DEV), vc.to(DEV)
    out = attention.kv_attention(q.to(DEV), kd, vd, pos, k_new=kn.to(DEV), v_new=vn.to(DEV))
    kr, vr = kc.float().clone(), vc.float().clone()
    kr[:, :, pos:pos + S] = kn.float()
    vr[:, :, pos:pos + S] = vn.float()
    ref = ok.attend(q, kr, vr, ok.additive_mask(S, ctx, pos))
    assert_close(out.float(), ref, "batched")
    assert torch.equal(kd.cpu().float(), kr) and torch.equal(vd.cpu().float(), vr)
    with pytest.raises(RuntimeError, match="exceed"):
        attention.kv_attention(q.to(DEV), kd, vd, ctx - 4, k_new=kn.to(DEV), v_new=vn.to(DEV))
    tiny = torch.empty(16, dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="workspace"):
        attention.kv_attention(q[:, :, :1].contiguous().to(DEV), kd, vd, 400, workspace=tiny)


def test_bf16_cache():
    torch.manual_seed(8)
    Hq, Hkv, hd, ctx, S, pos = 16, 2, 256, 1024, 64, 512
    kc = torch.randn(Hkv, ctx, hd).bfloat16()
    vc = torch.randn(Hkv, ctx, hd).bfloat16()
    q = torch.randn(1, Hq, S, hd).bfloat16()
    gate = torch.randn(1, S, Hq * hd).bfloat16()
    out = attention.kv_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), pos, gate=gate.to(DEV))
    ref = ok.attend(q, kc.unsqueeze(0), vc.unsqueeze(0), ok.additive_mask(S, ctx, pos), gate)
    # bf16 probabilities feed the PV product: its 8-bit mantissa sets this bound
    assert_close(out.float(), ref, "bf16", rel_l2=5e-3, max_abs=1e-2)


def _aligned4_out(B, S, width, dt):
    """An output view whose address is 4- but not 8-byte aligned: the library then takes its
    generic split-KV kernel instead of the TMA decode kernel."""
    buf = torch.empty(B * S * width + 2, dtype=dt, device=DEV)
    out = buf[2:].view(B, S, width)
    assert out.data_ptr() % 8 == 4
    return out


@pytest.mark.parametrize("hd", [64, 128, 256])
@pytest.mark.parametrize("dt", [torch.half, torch.bfloat16])
def test_decode_kernels_match_oracle(hd, dt):
    """Decode-shaped calls (S x G <= 16 query rows), batched caches: the TMA decode kernel and
    the generic split-KV kernel both match the oracle under causal, sliding-window and
    explicit masks, with 1, 8 and 16 query heads per kv head; written cache rows bit-exact."""
    torch.manual_seed(11 + hd)
    B, ctx = 2, 1536
    cases = [  # (H_q, H_kv, S, pos, window, explicit mask)
        (16, 2, 1, 1000, 0, False), (16, 2, 1, 1400, 300, False), (16, 2, 2, 777, 0, True),
        (16, 2, 1, 63, 0, False), (32, 2, 1, 1535, 0, False), (4, 4, 3, 500, 128, False),
    ]
    # bf16 probabilities and outputs carry an 8-bit mantissa: 5e-3 / 1e-2 for bf16
    rel_l2, max_abs = (1e-3, 2e-3) if dt == torch.half else (5e-3, 1e-2)
    for Hq, Hkv, S, pos, window, use_mask in cases:
        kc = torch.randn(B, Hkv, ctx, hd).to(dt)
        vc = torch.randn(B, Hkv, ctx, hd).to(dt)
        q = torch.randn(B, Hq, S, hd).to(dt)
        kn = torch.randn(B, Hkv, S, hd).to(dt)
        vn = torch.randn(B, Hkv, S, hd).to(dt)
        gate = torch.randn(B, S, Hq * hd).to(dt)
        kr, vr = kc.float().clone(), vc.float().clone()
        kr[:, :, pos:pos + S] = kn.float()
        vr[:, :, pos:pos + S] = vn.float()
        amask = ok.additive_mask(S, ctx, pos, window)
        ref = ok.attend(q, kr, vr, amask, gate)
        for generic in (False, True):
            kd, vd = kc.to(DEV), vc.to(DEV)
            out = _aligned4_out(B, S, Hq * hd, dt) if generic else None
            res = attention.kv_attention(q.to(DEV), kd, vd, pos, k_new=kn.to(DEV), v_new=vn.to(DEV),
                                         gate=gate.to(DEV), causal_mask=amask.to(dt).to(DEV) if use_mask else None,
                                         window=0 if use_mask else window, out=out)
            name = f"hd {hd} {dt} Hq {Hq} Hkv {Hkv} S {S} pos {pos} w {window} mask {use_mask} generic {generic}"
            assert_close(res.float().cpu(), ref, name, rel_l2=rel_l2, max_abs=max_abs)
            assert torch.equal(kd.cpu().float(), kr) and torch.equal(vd.cpu().float(), vr), name
    assert attention.kv_device_error() == 0


@pytest.mark.parametrize("hd", [128, 256])
def test_tcgen05_partial_query_tiles_with_key_splits(hd):
    """Prefill chunks on the tcgen05 path whose last 16-token query tile is partial (S = 20, 33, 100,
    130), at positions that give every tile several key splits: the split partials leave each CTA by
    TMA stores that must stop at the chunk's last token (later tokens would land in the next split's
    rows), and the combine merges them.  New rows patched into the tiles (S < 128) and pre-written
    by the copy kernel (S >= 128); causal and a 300-token window; cache bit-exact."""
    torch.manual_seed(31 + hd)
    Hq, Hkv, ctx = 16, 2, 4096
    for S, pos, window in [(20, 2500, 0), (33, 1800, 0), (100, 3000, 300), (130, 2047, 0), (20, 3900, 300)]:
        kc = torch.randn(Hkv, ctx, hd).half()
        vc = torch.randn(Hkv, ctx, hd).half()
        q = torch.randn(1, Hq, S, hd).half()
        kn = torch.randn(1, Hkv, S, hd).half()
        vn = torch.randn(1, Hkv, S, hd).half()
        gate = torch.randn(1, S, Hq * hd).half()
        kr, vr = kc.float().clone(), vc.float().clone()
        kr[:, pos:pos + S] = kn[0].float()
        vr[:, pos:pos + S] = vn[0].float()
        ref = ok.attend(q, kr.unsqueeze(0), vr.unsqueeze(0), ok.additive_mask(S, ctx, pos, window), gate)
        kd, vd = kc.to(DEV), vc.to(DEV)
        out = attention.kv_attention(q.to(DEV), kd, vd, pos, k_new=kn.to(DEV), v_new=vn.to(DEV), gate=gate.to(DEV),
                                     window=window)
        assert_close(out.float().cpu(), ref, f"hd {hd} S {S} pos {pos} window {window}")
        assert torch.equal(kd.cpu().float(), kr) and torch.equal(vd.cpu().float(), vr)
    assert attention.kv_device_error() == 0


def test_unwritten_cache_rows_are_never_read():
    """Cache rows past the visible range may hold anything, NaN included: prefill chunks (tcgen05
    path), decode steps (TMA decode kernel) and the generic kernel read none of them."""
    torch.manual_seed(12)
    for Hq, Hkv, hd, S, pos in [(16, 2, 256, 64, 300), (16, 2, 256, 48, 100), (16, 2, 128, 1, 333),
                                (8, 2, 64, 20, 70), (16, 2, 256, 1, 0)]:
        ctx = 1024
        kc = torch.randn(Hkv, ctx, hd).half()
        vc = torch.randn(Hkv, ctx, hd).half()
        q = torch.randn(1, Hq, S, hd).half()
        gate = torch.randn(1, S, Hq * hd).half()
        ref = ok.attend(q, kc.unsqueeze(0), vc.unsqueeze(0), ok.additive_mask(S, ctx, pos), gate)
        kc[:, pos + S:] = float("nan")
        vc[:, pos + S:] = float("nan")
        out = attention.kv_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), pos, gate=gate.to(DEV))
        assert_close(out.float().cpu(), ref, f"hd {hd} S {S} pos {pos}")


def test_tcgen05_prefill_with_batched_caches():
    """Prefill chunks on the tcgen05 path (8 query heads per kv head, hd 256) over per-sequence caches
    [B, H_kv, ctx, hd] (4-D tensor maps), new rows written in the same call; bit-exact cache, output
    within tolerance, with and without a sliding window."""
    torch.manual_seed(13)
    B, Hq, Hkv, hd, ctx, S = 3, 16, 2, 256, 1024, 64
    for pos, window in ((0, 0), (320, 0), (700, 128)):
        kc = torch.randn(B, Hkv, ctx, hd).half()
        vc = torch.randn(B, Hkv, ctx, hd).half()
        q = torch.randn(B, Hq, S, hd).half()
        kn = torch.randn(B, Hkv, S, hd).half()
        vn = torch.randn(B, Hkv, S, hd).half()
        gate = torch.randn(B, S, Hq * hd).half()
        kd, vd = kc.to(DEV), vc.to(DEV)
        out = attention.kv_attention(q.to(DEV), kd, vd, pos, k_new=kn.to(DEV), v_new=vn.to(DEV), gate=gate.to(DEV),
                                     window=window)
        kr, vr = kc.float().clone(), vc.float().clone()
        kr[:, :, pos:pos + S] = kn.float()
        vr[:, :, pos:pos + S] = vn.float()
        ref = ok.attend(q, kr, vr, ok.additive_mask(S, ctx, pos, window), gate)
        assert_close(out.float().cpu(), ref, f"pos {pos} window {window}")
        assert torch.equal(kd.cpu().float(), kr) and torch.equal(vd.cpu().float(), vr)
    assert attention.kv_device_error() == 0


@pytest.mark.gpu
def test_tcgen05_long_chunk_clips_keys_per_tile():
    """A 512-token chunk on the tcgen05 path: each 16-query tile scans only the keys its queries can
    see (causal prefix, per-query window start) and writes its own new rows into the cache; output
    within tolerance and the cache bit-exact, for the causal, per-query window and chunk-aligned
    window rules, from position 0 and from a later position."""
    torch.manual_seed(17)
    B, Hq, Hkv, hd, ctx, S = 2, 16, 2, 256, 1024, 512
    for pos, window, aligned in ((0, 0, False), (256, 0, False), (0, 200, False), (300, 96, False),
                                 (256, 600, True)):
        kc = torch.randn(B, Hkv, ctx, hd).half()
        vc = torch.randn(B, Hkv, ctx, hd).half()
        q = torch.randn(B, Hq, S, hd).half()
        kn = torch.randn(B, Hkv, S, hd).half()
        vn = torch.randn(B, Hkv, S, hd).half()
        gate = torch.randn(B, S, Hq * hd).half()
        kd, vd = kc.to(DEV), vc.to(DEV)
        out = attention.kv_attention(q.to(DEV), kd, vd, pos, k_new=kn.to(DEV), v_new=vn.to(DEV), gate=gate.to(DEV),
                                     window=window, window_chunk_aligned=aligned)
        kr, vr = kc.float().clone(), vc.float().clone()
        kr[:, :, pos:pos + S] = kn.float()
        vr[:, :, pos:pos + S] = vn.float()
        ref = ok.attend(q, kr, vr, ok.additive_mask(S, ctx, pos, window, chunk_aligned=aligned), gate)
        assert_close(out.float().cpu(), ref, f"pos {pos} window {window} aligned {aligned}")
        assert torch.equal(kd.cpu().float(), kr) and torch.equal(vd.cpu().float(), vr)
    assert attention.kv_device_error() == 0
