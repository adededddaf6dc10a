"""CPU checks of the C-ABI boundary: the library loads and exports every symbol
that include/anemll_b200.h declares, and argument validation rejects bad calls
before any launch (no GPU needed: validation returns before touching CUDA)."""
import ctypes
import os
import re

import pytest
import torch

from anemll_b200 import _lib
from tests.conftest import ROOT


def _declared():
    txt = open(os.path.join(ROOT, "include", "anemll_b200.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(anemll_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert declared, "no entry points parsed from the header"
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_lib.exported_symbols()), "ctypes table and header disagree"


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.anemll_version() >= 1
    assert isinstance(lib.anemll_last_error(), bytes)


def test_recurrent_rejects_bad_head_dim():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    rc = lib.anemll_gdn_recurrent(p, p, p, 2, p, p, p, p, 2, 1, 1, 1, 2, 64, 128, 0.0, 1, None)
    assert rc < 0
    assert b"d_k" in lib.anemll_last_error()


def test_recurrent_rejects_null_and_head_ratio():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.anemll_gdn_recurrent(None, p, p, 2, p, p, p, p, 2, 1, 1, 1, 2, 128, 128, 0.0, 1, None) < 0
    assert lib.anemll_gdn_recurrent(p, p, p, 2, p, p, p, p, 2, 1, 1, 3, 4, 128, 128, 0.0, 1, None) < 0


def test_gated_prefill_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # the gated output (and z) is fp16 or bf16
    rc = lib.anemll_gdn_chunked_prefill_gated(p, p, p, 2, p, p, p, p, 0, p, 1e-6, p, 0, None, 1, 64, 1, 2, 128, 128,
                                              64, 0.0, 0, None)
    assert rc < 0 and b"out" in lib.anemll_last_error()
    rc = lib.anemll_gdn_chunked_prefill_gated(p, p, p, 2, p, p, p, p, 0, p, 1e-6, p, 2, None, 1, 64, 1, 2, 128, 256,
                                              64, 0.0, 0, None)
    assert rc < 0 and b"d_v" in lib.anemll_last_error()
    # z rows shorter than H_v * d_v
    rc = lib.anemll_gdn_chunked_prefill_gated(p, p, p, 2, p, p, p, p, 64, p, 1e-6, p, 2, None, 1, 64, 1, 2, 128, 128,
                                              64, 0.0, 0, None)
    assert rc < 0 and b"stride" in lib.anemll_last_error()
    rc = lib.anemll_gdn_chunked_prefill_gated(p, p, p, 2, p, p, p, None, 0, p, 1e-6, p, 2, None, 1, 64, 1, 2, 128, 128,
                                              64, 0.0, 0, None)
    assert rc < 0 and b"null" in lib.anemll_last_error()


def test_kv_attention_validation():
    lib = _lib.load()
    p = ctypes.c_void_p(1 << 20)
    # positions beyond the cache
    rc = lib.anemll_kv_attention(p, p, p, None, p, p, 0, 4096 * 256, None, 0, 0, p, 1,
                                 1, 64, 16, 2, 256, 4096, 4090, 0, 0, None, 0, None)
    assert rc < 0 and b"exceed" in lib.anemll_last_error()
    # unsupported head dim
    rc = lib.anemll_kv_attention(p, p, p, None, p, p, 0, 4096 * 96, None, 0, 0, p, 1,
                                 1, 1, 16, 2, 96, 4096, 0, 0, 0, None, 0, None)
    assert rc < 0
    # missing workspace when splits are needed
    need = lib.anemll_kv_attention_workspace_size(1, 1, 16, 2, 256, 4096)
    assert need > 0
    rc = lib.anemll_kv_attention(p, p, p, None, p, p, 0, 4096 * 256, None, 0, 0, p, 1,
                                 1, 1, 16, 2, 256, 4096, 4000, 0, 0, None, 0, None)
    assert rc == -4 and b"workspace" in lib.anemll_last_error()


def test_product_fails_loudly_without_cuda():
    torch = pytest.importorskip("torch")
    from anemll_b200 import gdn
    q = torch.zeros(1, 1, 1, 128)
    with pytest.raises(RuntimeError):
        gdn.recurrent_gated_delta_rule(q, q, q, torch.zeros(1, 1, 1), torch.zeros(1, 1, 1))


def test_torch_ops_are_registered_and_refuse_cpu_tensors():
    import anemll_b200.ops  # noqa: F401  (registers torch.ops.anemll_b200.*)
    for name in ("gdn_chunked_prefill", "gdn_recurrent", "gdn_gated_delta_rule_norm", "gdn_prologue", "kv_attention"):
        assert hasattr(torch.ops.anemll_b200, name)
    z = torch.zeros(1, 1, 1, 128, dtype=torch.half)
    with pytest.raises(NotImplementedError):
        torch.ops.anemll_b200.gdn_recurrent(z, z, z, torch.zeros(1, 1, 1), torch.zeros(1, 1, 1),
                                            torch.zeros(1, 1, 128, 128))
