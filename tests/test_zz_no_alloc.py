"""The allocation-free KV-attention entry point, called through the C ABI (GPU).

Callers that cannot allocate device memory at call time (an engine that has
reserved all GPU memory up front, or a loop that cannot afford the device-wide
synchronisation of cudaMalloc) use anemll_kv_attention_noalloc, which takes its
split-KV scratch from a fixed array inside the library.  This file checks that
it produces what anemll_kv_attention produces with a caller workspace, on two
calls in a row (the second call reuses the scratch the first one left behind),
and that a shape beyond the built-in maximum is refused.  It sorts last so a
run that stops at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

from anemll_b200 import _lib
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
HQ, HKV, HD, CTX = 16, 2, 256, 4096


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call(lib, noalloc, q, kn, vn, gate, K, V, out, pos, ws=None):
    S = q.shape[2]
    common = (_p(q), _p(kn), _p(vn), _p(gate), _p(K), _p(V), 0, K.stride(0), None, 0, 0, _p(out), _lib.F16,
              1, S, HQ, HKV, HD, CTX, pos, 0, 0)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        return lib.anemll_kv_attention_noalloc(*common, stream)
    return lib.anemll_kv_attention(*common, _p(ws), ws.numel(), stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    lib = _lib.load()
    torch.manual_seed(42)
    cache = torch.zeros(2, HKV, CTX, HD, dtype=torch.half)
    cache[:, :, :3000] = torch.randn(2, HKV, 3000, HD).half()
    cache_a = cache.to(DEV)  # regular entry point
    cache_b = cache.clone().to(DEV)  # allocation-free entry point
    need = lib.anemll_kv_attention_workspace_size(1, 1, HQ, HKV, HD, CTX)
    assert 0 < need <= lib.anemll_kv_attention_noalloc_max_scratch()
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    for pos in (3000, 3001):  # two decode steps in a row, each split over the keys
        q = torch.randn(1, HQ, 1, HD, dtype=torch.half, device=DEV)
        kn = torch.randn(1, HKV, 1, HD, dtype=torch.half, device=DEV)
        vn = torch.randn(1, HKV, 1, HD, dtype=torch.half, device=DEV)
        gate = torch.randn(1, 1, HQ * HD, dtype=torch.half, device=DEV)
        out_a = torch.empty(1, 1, HQ * HD, dtype=torch.half, device=DEV)
        out_b = torch.full_like(out_a, float("nan"))
        _lib.check(_call(lib, False, q, kn, vn, gate, cache_a[0], cache_a[1], out_a, pos, ws), "regular")
        _lib.check(_call(lib, True, q, kn, vn, gate, cache_b[0], cache_b[1], out_b, pos), "noalloc")
        torch.cuda.synchronize()
        assert_close(out_b.float(), out_a.float(), f"decode at {pos}")
        assert torch.equal(cache_a, cache_b), "cache writes differ"


def test_noalloc_matches_workspace_entry_point_on_prefill_chunks():
    """16-token chunks take the tcgen05 prefill path, whose partial rows sit at offsets set by its own
    split count inside the scratch; two chunks in a row against the workspace entry point, at a shape
    whose scratch fits the built-in array (8 query heads on one kv head, hd 128, 1024-row cache)."""
    lib = _lib.load()
    torch.manual_seed(43)
    S, hq, hkv, hd, ctx = 16, 8, 1, 128, 1024
    cache = torch.zeros(2, hkv, ctx, hd, dtype=torch.half)
    cache[:, :, :512] = torch.randn(2, hkv, 512, hd).half()
    cache_a, cache_b = cache.to(DEV), cache.clone().to(DEV)
    need = lib.anemll_kv_attention_workspace_size(1, S, hq, hkv, hd, ctx)
    assert 0 < need <= lib.anemll_kv_attention_noalloc_max_scratch()
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for pos in (512, 512 + S):
        q = torch.randn(1, hq, S, hd, dtype=torch.half, device=DEV)
        kn = torch.randn(1, hkv, S, hd, dtype=torch.half, device=DEV)
        vn = torch.randn(1, hkv, S, hd, dtype=torch.half, device=DEV)
        gate = torch.randn(1, S, hq * hd, dtype=torch.half, device=DEV)
        out_a = torch.empty(1, S, hq * hd, dtype=torch.half, device=DEV)
        out_b = torch.full_like(out_a, float("nan"))
        for noalloc, cc, out in ((False, cache_a, out_a), (True, cache_b, out_b)):
            args = (_p(q), _p(kn), _p(vn), _p(gate), _p(cc[0]), _p(cc[1]), 0, cc[0].stride(0), None, 0, 0, _p(out),
                    _lib.F16, 1, S, hq, hkv, hd, ctx, pos, 0, 0)
            rc = (lib.anemll_kv_attention_noalloc(*args, stream) if noalloc
                  else lib.anemll_kv_attention(*args, _p(ws), ws.numel(), stream))
            _lib.check(rc, "noalloc" if noalloc else "regular")
        torch.cuda.synchronize()
        assert_close(out_b.float(), out_a.float(), f"chunk at {pos}")
        assert torch.equal(cache_a, cache_b), "cache writes differ"


def test_noalloc_rejects_positions_past_the_cache():
    lib = _lib.load()
    cache = torch.zeros(2, HKV, CTX, HD, dtype=torch.half, device=DEV)
    q = torch.zeros(1, HQ, 1, HD, dtype=torch.half, device=DEV)
    kn = torch.zeros(1, HKV, 1, HD, dtype=torch.half, device=DEV)
    out = torch.empty(1, 1, HQ * HD, dtype=torch.half, device=DEV)
    for pos in (CTX, 2**31 - 1):  # the second would overflow a 32-bit pos + S
        assert _call(lib, True, q, kn, kn, None, cache[0], cache[1], out, pos) == -1
        assert _call(lib, False, q, kn, kn, None, cache[0], cache[1], out, pos,
                     torch.empty(1 << 20, dtype=torch.uint8, device=DEV)) == -1


def test_noalloc_rejects_scratch_beyond_its_maximum():
    lib = _lib.load()
    # a 64-token prefill chunk of this shape needs about 18 MB of split-KV scratch
    S, pos = 64, 2048
    cache = torch.zeros(2, HKV, CTX, HD, dtype=torch.half, device=DEV)
    q = torch.zeros(1, HQ, S, HD, dtype=torch.half, device=DEV)
    kn = torch.zeros(1, HKV, S, HD, dtype=torch.half, device=DEV)
    out = torch.empty(1, S, HQ * HD, dtype=torch.half, device=DEV)
    before = cache.clone()
    rc = _call(lib, True, q, kn, kn, None, cache[0], cache[1], out, pos)
    assert rc == -4
    assert b"maximum" in lib.anemll_last_error()
    torch.cuda.synchronize()
    assert torch.equal(cache, before), "a refused call must not launch"
