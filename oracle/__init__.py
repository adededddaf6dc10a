"""CPU oracle for the attention hot path — TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it.  The product path (``anemll_b200``) never calls into it and fails
loudly when its CUDA library is missing.

Two halves, both fp32 (optionally fp64) CPU restatements:

* ``oracle.gdn`` — the Qwen3.5 gated delta-rule layer (causal conv1d
  prologue, gates, chunked and recurrent delta rule, gated RMSNorm).  The
  reference snapshot (slimwangyue/Anemll) has no gated-DeltaNet code, so this
  is written from the published mathematics (Yang, Kautz & Hatamizadeh,
  "Gated Delta Networks", ICLR 2025; the chunkwise WY/UT form of Yang et al.,
  "Parallelizing Linear Transformers with the Delta Rule", NeurIPS 2024).
  Its semantics (argument meaning, l2-norm epsilon, gate formula, conv-state
  layout) follow the third-party module the reference's model family uses:
  ``transformers==5.5.0``, ``transformers/models/qwen3_5/modeling_qwen3_5.py``
  (``l2norm`` 228-231, ``torch_causal_conv1d_update`` 210-226,
  ``torch_chunk_gated_delta_rule`` 234-311,
  ``torch_recurrent_gated_delta_rule`` 314-353, ``Qwen3_5RMSNormGated``
  175-190, gate lines 491-493).  Parity of this restatement is pinned by the
  golden vectors in ``tests/golden/`` that were produced by that third-party
  code (see ``tests/golden/make_golden.py``); the reference itself pins
  nothing for this half.

* ``oracle.kv_attention`` — the fixed-shape KV-cache attention of
  ``anemll/models/qwen_model.py`` (``QwenAttention.forward_prefill``
  509-546, ``forward_regular`` 469-507, cache writes 669-675 / 733-745), the
  sliding-window visibility rule of ``anemll/models/gemma3_model.py``
  (``_kv_slice`` 906-926) and the Qwen3.5 sigmoid output gate
  (``modeling_qwen3_5.py`` 632-689).  Pinned against the reference's own
  ``QwenAttention`` run in fp32 (golden vectors in ``tests/golden/``).
"""
