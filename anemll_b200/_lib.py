"""ctypes binding of the C ABI in ``include/anemll_b200.h``.

The library is the in-tree ``anemll_b200/lib/libanemll_b200.so`` built by
``anemll_b200.build``.  There is no fallback: if the library is missing every
op raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import build as _build

F32, F16, BF16 = 0, 1, 2
EUNSUPPORTED = -2  # ANEMLL_EUNSUPPORTED: the entry point does not take this shape
_DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

_c_int, _c_i64, _c_float, _vp, _c_size = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t

_SIGS = {
    "anemll_last_error": ([], ctypes.c_char_p),
    "anemll_version": ([], _c_int),
    "anemll_launch_count": ([], ctypes.c_longlong),
    "anemll_gdn_recurrent": ([_vp, _vp, _vp, _c_int, _vp, _vp, _vp, _vp, _c_int,
                              _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _vp], _c_int),
    "anemll_gdn_chunked_prefill": ([_vp, _vp, _vp, _c_int, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                    _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _vp], _c_int),
    "anemll_gdn_chunked_error": ([_c_int], _c_int),
    "anemll_gdn_chunked_mode": ([_c_int], _c_int),
    "anemll_gdn_chunked_prefill_gated": ([_vp, _vp, _vp, _c_int, _vp, _vp, _vp, _vp, _c_i64, _vp, _c_float, _vp,
                                          _c_int, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                          _c_float, _c_int, _vp], _c_int),
    "anemll_gdn_prologue": ([_vp, _c_int, _vp, _vp, _vp, _vp, _c_int, _vp, _vp, _vp, _vp, _vp, _c_int, _vp, _vp,
                             _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_i64, _vp],
                            _c_int),
    "anemll_gated_rmsnorm": ([_vp, _c_int, _vp, _c_int, _vp, _vp, _c_int, _c_i64, _c_int, _c_float, _c_i64, _c_i64,
                              _vp], _c_int),
    "anemll_kv_attention_workspace_size": ([_c_int, _c_int, _c_int, _c_int, _c_int, _c_int], _c_size),
    "anemll_kv_attention": ([_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _vp, _c_int, _c_i64, _vp, _c_int,
                             _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                             _vp, _c_size, _vp], _c_int),
    "anemll_kv_attention_qkv": ([_vp, _c_i64, _vp, _vp, _vp, _vp, _c_float, _vp, _vp, _c_i64, _c_i64, _vp, _c_int,
                                 _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_size,
                                 _vp], _c_int),
    "anemll_kv_attention_noalloc_max_scratch": ([], _c_size),
    "anemll_kv_attention_error": ([_c_int], _c_int),
    "anemll_kv_update_mask": ([_vp, _vp, _c_int, _vp, _c_int, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_i64, _c_i64,
                               _vp], _c_int),
    "anemll_kv_rotate_append": ([_vp, _vp, _c_int, _c_i64, _c_int, _c_int, _c_int, _c_i64, _c_i64, _vp], _c_int),
    "anemll_rmsnorm": ([_vp, _vp, _vp, _vp, _vp, _c_int, _c_i64, _c_int, _c_float, _vp], _c_int),
    "anemll_silu_mul": ([_vp, _vp, _c_int, _c_i64, _c_int, _vp], _c_int),
    "anemll_qk_norm_rope": ([_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int,
                             _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _vp], _c_int),
    "anemll_kv_state_transition": ([_vp, _c_int, _vp, _c_int, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_float,
                                    _vp], _c_int),
    "anemll_kv_attention_noalloc": ([_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _vp, _c_int, _c_i64, _vp, _c_int,
                                     _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp],
                                    _c_int),
}

_lib = None


def lib_path() -> str:
    return _build.LIB


def load() -> ctypes.CDLL:
    """Load the shared library (once).  Raises ``RuntimeError`` if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise RuntimeError(
            f"anemll_b200 CUDA library not found at {path}; build it with `python -m anemll_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (args, res) in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def exported_symbols():
    return list(_SIGS)


def launch_count() -> int:
    """Kernel launches issued through the library so far in this process (graph replays excluded)."""
    return int(load().anemll_launch_count())


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().anemll_last_error().decode(errors="replace")
        kind = "invalid argument" if rc < 0 else "CUDA error"
        raise RuntimeError(f"{what} failed ({kind} {rc}): {msg}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError as e:
        raise TypeError(f"unsupported dtype {t}") from e


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
