"""The CPU oracle against the golden vectors (no GPU).

KV attention is pinned by the reference's own ``QwenAttention`` / ``QwenModel``
run in fp32; the gated delta rule by the third-party transformers 5.5.0 torch
functions (the reference has no GDN code).  See ``tests/golden/make_golden.py``.
"""
import os

import pytest
import torch

from oracle import gdn as og
from oracle import kv_attention as ok
from tests.conftest import GOLDEN


def _rel(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.fixture(scope="module")
def gold_gdn():
    return torch.load(os.path.join(GOLDEN, "gdn.pt"))


@pytest.fixture(scope="module")
def gold_kv():
    return torch.load(os.path.join(GOLDEN, "kv_attention.pt"))


@pytest.fixture(scope="module")
def gold_write():
    return torch.load(os.path.join(GOLDEN, "kv_cache_write.pt"))


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-6), (torch.float32, 2e-5)])
def test_chunk_rule_matches_golden(gold_gdn, dtype, tol):
    d = gold_gdn["gdn"]
    o, s = og.chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], 64, d["S0"],
                                     use_qk_l2norm=True, dtype=dtype)
    assert _rel(o, d["out_chunk"]) < tol
    assert _rel(s, d["state_chunk"]) < tol


@pytest.mark.parametrize("chunk", [16, 32, 64, 100])
def test_chunk_rule_any_chunk_matches_recurrent_golden(gold_gdn, chunk):
    d = gold_gdn["gdn"]
    o, s = og.chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], chunk, d["S0"],
                                     use_qk_l2norm=True, dtype=torch.float64)
    assert _rel(o, d["out_recurrent"]) < 1e-6
    assert _rel(s, d["state_recurrent"]) < 1e-6


def test_recurrent_rule_matches_golden(gold_gdn):
    d = gold_gdn["gdn"]
    o, s = og.recurrent_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"],
                                         use_qk_l2norm=True, dtype=torch.float32)
    assert _rel(o, d["out_recurrent"]) < 2e-5
    assert _rel(s, d["state_recurrent"]) < 2e-5


def test_conv_prologue_matches_golden(gold_gdn):
    c = gold_gdn["conv"]
    y, st = og.causal_conv1d_prefill(c["x"], c["w"], None)
    assert _rel(y, c["y_prefill"]) < 1e-6
    assert torch.equal(st, c["state_prefill"])  # state shift is exact
    y1, st1 = og.causal_conv1d_update(c["x1"], c["w"], st)
    assert _rel(y1, c["y_decode"]) < 1e-6
    assert torch.equal(st1, c["state_decode"])


def test_gated_rmsnorm_matches_golden(gold_gdn):
    n = gold_gdn["norm"]
    y = og.gated_rmsnorm(n["x"], n["z"], n["weight"])
    assert _rel(y, n["y"]) < 1e-6


def test_kv_attention_matches_reference(gold_kv):
    hd, ctx = gold_kv["hd"], gold_kv["ctx"]
    for c in gold_kv["cases"]:
        S, pos = c["S"], c["pos"]
        K = torch.zeros(1, gold_kv["Hkv"], ctx, hd)
        V = torch.zeros(1, gold_kv["Hkv"], ctx, hd)
        K[0, :, :pos + S] = c["K"].float()
        V[0, :, :pos + S] = c["V"].float()
        vis = ok.visibility_mask(S, ctx, pos, c["window"], c["chunk_aligned"])
        assert torch.equal(vis, c["visible"]), c["name"]
        mask = ok.additive_mask(S, ctx, pos, c["window"], chunk_aligned=c["chunk_aligned"])
        out = ok.attend(c["q"], K, V, mask)
        assert _rel(out, c["out"]) < 1e-5, c["name"]


def test_kv_attention_with_o_proj_matches_reference():
    """The oracle's attention followed by the fixture's o_proj weight reproduces the reference's
    projected return value (``kv_attention_oproj.pt``)."""
    fx = torch.load(os.path.join(GOLDEN, "kv_attention_oproj.pt"))
    hd, ctx = fx["hd"], fx["ctx"]
    w = fx["o_proj_weight"].reshape(fx["hidden"], -1)
    for c in fx["cases"]:
        S, pos = c["S"], c["pos"]
        K = torch.zeros(1, fx["Hkv"], ctx, hd)
        V = torch.zeros(1, fx["Hkv"], ctx, hd)
        K[0, :, :pos + S] = c["K"].float()
        V[0, :, :pos + S] = c["V"].float()
        out = torch.nn.functional.linear(ok.attend(c["q"], K, V, ok.additive_mask(S, ctx, pos)), w)
        assert _rel(out, c["out"]) < 1e-5, c["name"]


def test_kv_cache_write_bit_exact(gold_write):
    for w in gold_write["writes"]:
        cache = w["before"].clone()
        ok.write_cache(cache, w["k"], w["v"], w["layer_idx"], w["num_layers"], w["pos"])
        assert torch.equal(cache, w["after"]), w["name"]
