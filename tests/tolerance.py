"""The parity bar: relative L2 error <= 1e-3 and max abs error <= 2e-3 against
the fp32 oracle run on the same rounded inputs; cache and state index updates
must be bit-exact (compared with torch.equal)."""
import torch

REL_L2 = 1e-3
MAX_ABS = 2e-3


def errors(got, want):
    got = got.detach().float().cpu().double()
    want = want.detach().float().cpu().double()
    diff = got - want
    rel = float(diff.norm() / want.norm().clamp_min(1e-30))
    mx = float(diff.abs().max()) if diff.numel() else 0.0
    return rel, mx


def assert_close(got, want, what="", rel_l2=REL_L2, max_abs=MAX_ABS):
    assert got.shape == want.shape, f"{what}: shape {tuple(got.shape)} != {tuple(want.shape)}"
    assert torch.isfinite(got.float()).all(), f"{what}: non-finite values"
    rel, mx = errors(got, want)
    assert rel <= rel_l2 and mx <= max_abs, f"{what}: rel_l2={rel:.3e} (<= {rel_l2}) max_abs={mx:.3e} (<= {max_abs})"
    return rel, mx
