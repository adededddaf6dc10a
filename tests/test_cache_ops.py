"""Cache-management ops: the oracle against the reference's own outputs (CPU), and the device ops
against both (GPU, through the C ABI).  Values must match exactly: these ops only copy, convert
and select."""
import os

import pytest
import torch

from oracle import cache_ops as oc
from tests.conftest import GOLDEN

DEV = "cuda"


@pytest.fixture(scope="module")
def fx():
    return torch.load(os.path.join(GOLDEN, "cache_ops.pt"))


def _rotate_ref(c):
    after = c["before"].clone()
    nl, li = c["num_local"], c["layer_idx"]
    for slot, nw in ((li, c["key"]), (li + nl, c["value"])):
        after[slot:slot + 1] = oc.rotate_append(after[slot:slot + 1], nw, c["shift"])
    return after


# ------------------------------------------------------------------ oracle (CPU) --
def test_oracle_matches_reference_update_mask(fx):
    for c in fx["update_mask_single"] + fx["update_mask_batch"]:
        got = oc.update_mask_write(c["cache"], c["new"], c["mask"][0, 0]).to(c["out"].dtype)
        assert torch.equal(got, c["out"])


def test_oracle_matches_reference_rotation(fx):
    for c in fx["rotate"]:
        assert torch.equal(_rotate_ref(c), c["after"])


def test_oracle_matches_reference_transition_and_compaction(fx):
    for c in fx["transition"]:
        pos = c["pos"] if c["pos"] is not None else c["src"].shape[2]
        assert torch.equal(oc.transition_state(c["src"], c["target"], pos, c["pad"], c["dtype"]), c["out"])
    for c in fx["compact"]:
        assert torch.equal(oc.transition_state(c["src"], c["target"], c["pos"], 0.0), c["out"])


# ---------------------------------------------------------------- device (GPU) --
@pytest.mark.gpu
def test_update_mask_matches_reference(fx):
    from anemll_b200 import cache_ops
    for c in fx["update_mask_single"] + fx["update_mask_batch"]:
        cache = c["cache"].to(DEV)
        cache_ops.apply_update_mask_(cache, c["new"].to(DEV), c["mask"].to(DEV))
        assert torch.equal(cache.cpu(), c["out"])


@pytest.mark.gpu
def test_rotation_matches_reference(fx):
    from anemll_b200 import cache_ops
    for c in fx["rotate"]:
        kv = c["before"].to(DEV)
        cache_ops.update_kv_local_(kv, c["layer_idx"], c["num_local"], c["key"].to(DEV), c["value"].to(DEV),
                                   c["shift"])
        assert torch.equal(kv.cpu(), c["after"]), c["shift"]


@pytest.mark.gpu
def test_transition_and_compaction_match_reference(fx):
    from anemll_b200 import cache_ops
    for c in fx["transition"]:
        out = cache_ops.transition_kv_state(c["src"].to(DEV), c["target"], current_position=c["pos"],
                                            pad_value=c["pad"], dtype=c["dtype"])
        assert out.dtype == c["out"].dtype and torch.equal(out.cpu(), c["out"])
    for c in fx["compact"]:
        out = cache_ops.compact_kv_state(c["src"].to(DEV), c["target"], current_position=c["pos"])
        assert torch.equal(out.cpu(), c["out"])


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
def test_ops_at_model_sizes_match_oracle(dt):
    """Gemma3-like split local cache (18 local layers, 1 kv head, window 512, hd 256) and a 36-layer
    state resize 512 -> 1024 -> 256, every dtype; exact against the oracle."""
    from anemll_b200 import cache_ops
    g = torch.Generator().manual_seed(5)
    nl, H, sw, hd = 18, 1, 512, 256
    kv = torch.randn(2 * nl, H, sw, hd, generator=g).to(dt)
    ref = kv.clone()
    dev = kv.to(DEV)
    for li, shift in ((0, 1), (17, 64), (5, 512)):
        key = torch.randn(1, H, shift, hd, generator=g).to(dt)
        val = torch.randn(1, H, shift, hd, generator=g).to(dt)
        cache_ops.update_kv_local_(dev, li, nl, key.to(DEV), val.to(DEV), shift)
        for slot, nw in ((li, key), (li + nl, val)):
            ref[slot:slot + 1] = oc.rotate_append(ref[slot:slot + 1], nw, shift)
    assert torch.equal(dev.cpu(), ref)
    # one-hot mask writes of a 64-token chunk at positions 100..163 of every local layer
    new = torch.randn(2 * nl, H, 64, hd, generator=g).to(dt)
    mask = torch.zeros(1, 1, sw, 64, dtype=torch.float16)
    for s in range(64):
        mask[0, 0, 100 + s, s] = 1
    cache_ops.apply_update_mask_(dev, new.to(DEV), mask.to(DEV))
    ref = oc.update_mask_write(ref, new, mask[0, 0]).to(dt)
    assert torch.equal(dev.cpu(), ref)
    # state resize
    st = torch.randn(36, 1, 512, 256, generator=g).to(dt)
    big = cache_ops.transition_kv_state(st.to(DEV), 1024, current_position=300)
    assert torch.equal(big.cpu(), oc.transition_state(st, 1024, 300))
    small = cache_ops.compact_kv_state(big, 256, current_position=250, dtype=torch.float16)
    assert torch.equal(small.cpu(), oc.transition_state(oc.transition_state(st, 1024, 300), 256, 250, 0.0,
                                                        torch.float16))


@pytest.mark.gpu
def test_argument_errors_follow_the_reference():
    from anemll_b200 import cache_ops
    s = torch.zeros(2, 1, 64, 32, device=DEV, dtype=torch.half)
    with pytest.raises(ValueError, match="must be >= source"):
        cache_ops.transition_kv_state(s, 32)
    with pytest.raises(ValueError, match="cannot exceed"):
        cache_ops.transition_kv_state(s, 128, current_position=65)
    with pytest.raises(ValueError, match="Cannot compact"):
        cache_ops.compact_kv_state(s, 16, current_position=20)
    assert cache_ops.transition_kv_state(s, 64) is s  # nothing to do: the input itself, as in the reference
    with pytest.raises(RuntimeError, match="shift"):
        cache_ops.rotate_append_(s, torch.zeros(2, 1, 65, 32, device=DEV, dtype=torch.half), 65)
    wide = torch.zeros(1, 1, 8192, 64, device=DEV, dtype=torch.half)
    with pytest.raises(RuntimeError, match="strip"):
        cache_ops.rotate_append_(wide, torch.zeros(1, 1, 1, 64, device=DEV, dtype=torch.half))
