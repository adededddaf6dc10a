"""``torch.ops.anemll_b200.*``: the hot-path entry points registered as torch operators.

Each operator is a thin registration over the C ABI (``include/anemll_b200.h``) through the Python
mirrors in :mod:`anemll_b200.gdn` and :mod:`anemll_b200.attention`: same argument meaning, the
mutated state declared to the dispatcher (``mutates_args``), CUDA tensors only (no CPU kernel is
registered, so a CPU tensor fails in the dispatcher).  Importing this module registers them.

=====================================  =========================================================
operator                               replaces
=====================================  =========================================================
``gdn_chunked_prefill(q, k, v, g,      ``torch_chunk_gated_delta_rule`` (transformers 5.5.0
beta, state, scale, use_qk_l2norm)``   ``modeling_qwen3_5.py:234-311``); ``state`` updated
``gdn_recurrent(q, k, v, g, beta,      ``torch_recurrent_gated_delta_rule`` (314-353)
state, scale, use_qk_l2norm)``
``gdn_gated_delta_rule_norm(q, k, v,   the core call and ``self.norm`` (``Qwen3_5RMSNormGated``)
g, beta, state, z, norm_weight, eps,   of ``Qwen3_5GatedDeltaNet.forward`` (497-523, 175-190):
chunked, scale, use_qk_l2norm)``       the chunked prefill with the norm in its epilogue, or the
                                       recurrent kernel followed by the norm kernel
``gdn_prologue(mixed_qkv, conv_weight, the conv/split/l2-norm/gate part of
conv_state, a, b, A_log, dt_bias,      ``Qwen3_5GatedDeltaNet.forward`` (453-496);
H_qk, H_v, d_k, d_v, use_state)``      ``conv_state`` updated
``kv_attention(query_states, k_cache,  ``QwenAttention.forward_prefill`` / ``forward_regular``
v_cache, current_pos, k_new, v_new,    (``anemll/models/qwen_model.py:469-546``) before
gate, causal_mask, window,             ``o_proj``, with the cache write of ``process_layer_*``
window_chunk_aligned)``                (669-675, 733-745); the caches updated in place
=====================================  =========================================================
"""
from __future__ import annotations

from typing import Optional

import torch

from . import attention, gdn

__all__ = ["gdn_chunked_prefill", "gdn_recurrent", "gdn_gated_delta_rule_norm", "gdn_prologue", "kv_attention"]


@torch.library.custom_op("anemll_b200::gdn_chunked_prefill", mutates_args=("state",), device_types="cuda")
def gdn_chunked_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                        state: torch.Tensor, scale: float = 0.0, use_qk_l2norm: bool = False) -> torch.Tensor:
    return gdn.chunk_gated_delta_rule_(q, k, v, g, beta, state, scale=scale if scale > 0 else None,
                                       use_qk_l2norm_in_kernel=use_qk_l2norm)


@torch.library.custom_op("anemll_b200::gdn_recurrent", mutates_args=("state",), device_types="cuda")
def gdn_recurrent(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                  state: torch.Tensor, scale: float = 0.0, use_qk_l2norm: bool = False) -> torch.Tensor:
    return gdn.recurrent_gated_delta_rule_(q, k, v, g, beta, state, scale=scale if scale > 0 else None,
                                           use_qk_l2norm_in_kernel=use_qk_l2norm)


@torch.library.custom_op("anemll_b200::gdn_gated_delta_rule_norm", mutates_args=("state",), device_types="cuda")
def gdn_gated_delta_rule_norm(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                              beta: torch.Tensor, state: torch.Tensor, z: torch.Tensor, norm_weight: torch.Tensor,
                              eps: float = 1e-6, chunked: bool = True, scale: float = 0.0,
                              use_qk_l2norm: bool = False) -> torch.Tensor:
    return gdn.gated_delta_rule_norm_(q, k, v, g, beta, state, z, norm_weight, eps, chunked=chunked,
                                      scale=scale if scale > 0 else None, use_qk_l2norm_in_kernel=use_qk_l2norm)


@torch.library.custom_op("anemll_b200::gdn_prologue", mutates_args=("conv_state",), device_types="cuda")
def gdn_prologue(mixed_qkv: torch.Tensor, conv_weight: torch.Tensor, conv_state: torch.Tensor, a: torch.Tensor,
                 b: torch.Tensor, A_log: torch.Tensor, dt_bias: Optional[torch.Tensor], H_qk: int, H_v: int,
                 d_k: int = 128, d_v: int = 128, use_state: bool = True
                 ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return gdn.gdn_prologue(mixed_qkv, conv_weight, conv_state, a, b, A_log, dt_bias, H_qk, H_v, d_k, d_v,
                            use_state=use_state)


@torch.library.custom_op("anemll_b200::kv_attention", mutates_args=("k_cache", "v_cache"), device_types="cuda")
def kv_attention(query_states: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, current_pos: int,
                 k_new: Optional[torch.Tensor] = None, v_new: Optional[torch.Tensor] = None,
                 gate: Optional[torch.Tensor] = None, causal_mask: Optional[torch.Tensor] = None, window: int = 0,
                 window_chunk_aligned: bool = False) -> torch.Tensor:
    return attention.kv_attention(query_states, k_cache, v_cache, current_pos, k_new=k_new, v_new=v_new, gate=gate,
                                  causal_mask=causal_mask, window=window, window_chunk_aligned=window_chunk_aligned)
