/*
 * anemll_b200 — C ABI of the B200 (sm_100a) attention hot path.
 *
 * Plain pointers and sizes only.  Every tensor pointer is device memory owned
 * by the caller; nothing here allocates persistent memory.  `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  All calls are
 * asynchronous and stream-ordered.
 *
 * Return value: 0 = success; negative = invalid argument (shape, dtype,
 * alignment, null pointer — nothing was launched); positive = a CUDA error
 * code from the launch.  anemll_last_error() returns a message for the last
 * failing call on the calling host thread.
 *
 * Layouts (row-major, contiguous unless a stride argument says otherwise):
 *   GDN   q, k        [B, T, H_qk, d_k]     value head j reads key head j / (H_v / H_qk)
 *         v, out      [B, T, H_v,  d_v]
 *         g, beta     [B, T, H_v]           fp32; g is the log-decay (<= 0)
 *         state       [B, H_v, d_k, d_v]    fp32, updated in place
 *         mixed_qkv   [B, T, 2*H_qk*d_k + H_v*d_v]   (q | k | v channels)
 *         conv_state  [B, 2*H_qk*d_k + H_v*d_v, conv_k]  same dtype as mixed_qkv
 *   KV    q           [B, H_q, S, hd]
 *         k_new,v_new [B, H_kv, S, hd]
 *         gate        [B, S, H_q*hd]        sigmoid-gate pre-activation (may be NULL)
 *         out         [B, S, H_q*hd]        attention output before o_proj
 *         k/v_cache   [B, H_kv, ctx, hd] with explicit batch/head element strides
 *                     (token stride = hd); one layer of the reference's unified
 *                     cache [2L, H_kv, ctx, hd] is batch_stride = 0,
 *                     head_stride = ctx*hd.
 */
#ifndef ANEMLL_B200_H
#define ANEMLL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define ANEMLL_F32 0
#define ANEMLL_F16 1
#define ANEMLL_BF16 2

/* status */
#define ANEMLL_OK 0
#define ANEMLL_EINVAL (-1)
#define ANEMLL_EUNSUPPORTED (-2)
#define ANEMLL_EALIGN (-3)
#define ANEMLL_EWORKSPACE (-4)

const char* anemll_last_error(void);
int anemll_version(void);
/* Kernel launches this process has issued through the library (successful launches; a launch
 * recorded into a CUDA graph counts once, when captured, not per replay). */
long long anemll_launch_count(void);

/*
 * Gated delta rule, token-by-token form: decode (T == 1) and recurrent prefill.
 * Replaces the recurrent core called from Qwen3_5GatedDeltaNet.forward
 * (third-party transformers 5.5.0, modeling_qwen3_5.py:314-353,
 * torch_recurrent_gated_delta_rule; the reference snapshot has no GDN code).
 * scale <= 0 selects 1/sqrt(d_k).  qk_l2norm != 0 l2-normalises q and k
 * (eps 1e-6) first, as use_qk_l2norm_in_kernel=True does there.
 * qkv_dtype / out_dtype: ANEMLL_F32, ANEMLL_F16 or ANEMLL_BF16.  d_k == 128,
 * d_v % 32 == 0, H_v % H_qk == 0.
 */
int anemll_gdn_recurrent(const void* q, const void* k, const void* v, int qkv_dtype,
                         const float* g, const float* beta, float* state,
                         void* out, int out_dtype,
                         int B, int T, int H_qk, int H_v, int d_k, int d_v,
                         float scale, int qk_l2norm, void* stream);

/*
 * Gated delta rule, chunked prefill: chunks of chunk_size tokens in the WY/UT
 * form on the tcgen05 tensor cores (q/k/v as given; the derived operands that
 * multiply them split into hi and lo parts of the same type; fp32
 * accumulators), the fp32 state carried across chunks in tensor memory.  Replaces
 * torch_chunk_gated_delta_rule (transformers 5.5.0 modeling_qwen3_5.py:234-311).
 * q/k/v are ANEMLL_F16 or ANEMLL_BF16; T may be any length (a ragged last
 * chunk is a shorter chunk).  chunk_size == 64, d_k == d_v == 128.
 */
int anemll_gdn_chunked_prefill(const void* q, const void* k, const void* v, int qkv_dtype,
                               const float* g, const float* beta, float* state,
                               void* out, int out_dtype,
                               int B, int T, int H_qk, int H_v, int d_k, int d_v,
                               int chunk_size, float scale, int qk_l2norm, void* stream);

/*
 * The chunked prefill with the layer's gated RMSNorm in its epilogue:
 * out = norm_weight * o * rsqrt(mean(o^2) + eps) * silu(z) over d_v, o being
 * the core output the plain call would return.  Replaces the core call together
 * with self.norm (Qwen3_5RMSNormGated) in Qwen3_5GatedDeltaNet.forward
 * (transformers 5.5.0 modeling_qwen3_5.py:497-523, the norm 175-190), so that o
 * never travels through HBM.  z [B, T, H_v, d_v] has the output's dtype
 * (ANEMLL_F16 or ANEMLL_BF16) with dense heads and token rows z_row_stride
 * elements apart (0: H_v * d_v; 16-byte aligned), so it may be a column slice
 * of the layer's fused projection output; norm_weight [d_v] fp32 (16-byte
 * aligned).  core_out (fp32 [B, T, H_v, d_v], 16-byte aligned, or NULL) also
 * receives o.  Other arguments as anemll_gdn_chunked_prefill.  (Decode keeps the
 * recurrent kernel and anemll_gated_rmsnorm: the fused recurrent forms measured
 * slower.)
 */
int anemll_gdn_chunked_prefill_gated(const void* q, const void* k, const void* v, int qkv_dtype,
                                     const float* g, const float* beta, float* state,
                                     const void* z, int64_t z_row_stride, const float* norm_weight, float eps,
                                     void* out, int out_dtype, float* core_out,
                                     int B, int T, int H_qk, int H_v, int d_k, int d_v,
                                     int chunk_size, float scale, int qk_l2norm, void* stream);

/*
 * Which kernel runs the chunked prefill (and its gated form): 0 (default)
 * chooses by the number of (sequence, value head) chains: one chain per SM
 * with the next chunk's state-independent work pipelined under the current
 * chunk's state chain while the chains fit one wave of SMs, two chains per
 * SM beyond that; 1 always the pipelined kernel; 2 always the two-chain
 * kernel.  Both give the same results bit for bit.  Returns the previous
 * mode; other values only query it.  No counterpart in the reference (a
 * choice between this build's kernels).
 */
int anemll_gdn_chunked_mode(int mode);

/*
 * Device-side status of the chunked kernel: non-zero if a bounded wait on the
 * tensor core ran out (the kernel then stopped early and its outputs are
 * invalid).  Synchronous; reset != 0 clears the flag.  Returns -1 on a CUDA
 * error.  No counterpart in the reference (diagnostics of this build).
 */
int anemll_gdn_chunked_error(int reset);

/*
 * Fused GDN prologue: depthwise causal conv1d (conv_k taps) + SiLU over the
 * mixed q|k|v channels, split, l2-normalise q and k (eps 1e-6), and the gates
 * beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias).
 * Replaces the conv/split/gate part of Qwen3_5GatedDeltaNet.forward
 * (modeling_qwen3_5.py:453-496, torch_causal_conv1d_update 210-226).
 * use_state == 0: history is zero (fresh prefill); != 0: history is read from
 * conv_state.  conv_state always receives the last conv_k raw inputs.
 * conv_w [C, conv_k] fp32; A_log, dt_bias [H_v] fp32 (dt_bias may be NULL);
 * a, b [B, T, H_v] in ab_dtype.  q/k/v outputs in out_dtype, g/beta fp32.
 * Token rows of mixed_qkv are x_row_stride elements apart (0: C, dense; a
 * multiple of 16 bytes), those of a and b ab_row_stride (0: H_v), so that all
 * four can be column slices of one fused projection output.
 */
int anemll_gdn_prologue(const void* mixed_qkv, int in_dtype, const float* conv_w, void* conv_state,
                        const void* a, const void* b, int ab_dtype,
                        const float* A_log, const float* dt_bias,
                        void* q_out, void* k_out, void* v_out, int out_dtype,
                        float* g_out, float* beta_out,
                        int B, int T, int H_qk, int H_v, int d_k, int d_v, int conv_k,
                        int use_state, int64_t x_row_stride, int64_t ab_row_stride, void* stream);

/*
 * Gated RMSNorm: out = weight * x * rsqrt(mean(x^2) + eps) * silu(z) over rows
 * of length d.  Replaces Qwen3_5RMSNormGated (modeling_qwen3_5.py:175-190).
 * x and out are dense [rows][d].  z is dense too when z_heads == 0; otherwise
 * row r of z is head r % z_heads of token r / z_heads, token rows
 * z_row_stride elements apart (a column slice of a fused projection output).
 */
int anemll_gated_rmsnorm(const void* x, int x_dtype, const void* z, int z_dtype,
                         const float* weight, void* out, int out_dtype,
                         int64_t rows, int d, float eps, int64_t z_heads, int64_t z_row_stride,
                         void* stream);

/*
 * KV-cache attention with the cache write fused in (one call = one prefill
 * chunk of S tokens or one decode step, S == 1).  Writes k_new/v_new at
 * positions [current_pos, current_pos + S) of k_cache / v_cache (for the
 * reference's unified cache: k_cache = kv_cache[layer_idx], v_cache =
 * kv_cache[layer_idx + num_layers], get_kv_cache_idx qwen_model.py:88-93),
 * then attends each query at position current_pos + i over keys 0..ctx-1.
 * k_new and v_new may both be NULL: the caller already wrote the cache (the
 * reference's own order: process_layer_* writes, then forward_* attends).
 * Replaces QwenAttention.forward_prefill (anemll/models/qwen_model.py:509-546)
 * plus the write at 669-675, and forward_regular (469-507) plus the write at
 * 733-745, with the Qwen3.5 sigmoid gate (modeling_qwen3_5.py:689).
 * Visibility: if `mask` is non-NULL it is the reference's additive mask
 * ([S, mask_row_stride] elements of mask_dtype; -inf hides a key).  Otherwise
 * key j is visible to position p iff j <= p and, when window > 0, j > p - window
 * (window_chunk_aligned != 0: j >= max(0, min(current_pos + S, ctx) - window)
 * for the whole chunk, gemma3_model.py:923-926).
 * dtype: ANEMLL_F16 or ANEMLL_BF16 for q, k_new, v_new, gate, cache and out.
 * workspace: device scratch of at least anemll_kv_attention_workspace_size()
 * bytes (may be NULL when that size is 0).
 */
size_t anemll_kv_attention_workspace_size(int B, int S, int H_q, int H_kv, int head_dim, int ctx);

int anemll_kv_attention(const void* q, const void* k_new, const void* v_new, const void* gate,
                        void* k_cache, void* v_cache, int64_t cache_batch_stride, int64_t cache_head_stride,
                        const void* mask, int mask_dtype, int64_t mask_row_stride,
                        void* out, int dtype,
                        int B, int S, int H_q, int H_kv, int head_dim, int ctx,
                        int current_pos, int window, int window_chunk_aligned,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Device-side status of the TMA-fed KV kernels (prefill chunks on the tensor
 * cores, decode steps): non-zero if a bounded wait for a K/V tile ran out (the
 * kernel then stopped early and that call's outputs are invalid).
 * Synchronous; reset != 0 clears the flag.  Returns -1 on a CUDA error.  No
 * counterpart in the reference (diagnostics of this library).
 */
int anemll_kv_attention_error(int reset);

/*
 * Allocation-free form of anemll_kv_attention (no counterpart in the
 * reference).  For callers that cannot allocate device memory when they call
 * in — an engine that reserves all GPU memory at start-up and forbids later
 * cudaMalloc, or a loop that cannot pay for the device-wide synchronisation
 * of cudaMalloc/cudaFree — the split-KV scratch comes from a fixed array
 * inside the library (anemll_kv_attention_noalloc_max_scratch() bytes, 8 MiB,
 * held on every GPU that loads the library until the process exits).
 * Same arguments as anemll_kv_attention minus the workspace; calls whose
 * scratch need exceeds the maximum return ANEMLL_EWORKSPACE without launching.
 * The size check uses the split count of the generic split-KV plan, the largest
 * any path of the call can take, so a call whose chosen path needs less can
 * still be refused.  The first call on a device (with that device current)
 * looks up the array's device address and caches it; make it before any stream
 * capture, and do not use the entry point after a cudaDeviceReset in the same
 * process.  All calls share the array: calls that overlap on the GPU race.
 * Allocates nothing.
 */
size_t anemll_kv_attention_noalloc_max_scratch(void);

int anemll_kv_attention_noalloc(const void* q, const void* k_new, const void* v_new, const void* gate,
                                void* k_cache, void* v_cache, int64_t cache_batch_stride,
                                int64_t cache_head_stride,
                                const void* mask, int mask_dtype, int64_t mask_row_stride,
                                void* out, int dtype,
                                int B, int S, int H_q, int H_kv, int head_dim, int ctx,
                                int current_pos, int window, int window_chunk_aligned, void* stream);

/*
 * Cache-management ops: ANEMLL-format caches (linear rows, oldest first) updated on the device.
 * A "slab" is one (layer, kv head) slice of L rows x d elements; slabs are cache_slab_stride
 * elements apart (new rows: new_slab_stride).  dtype: ANEMLL_F32 / F16 / BF16.
 *
 * anemll_kv_update_mask: the reference's one-hot update-mask write, in place:
 *   cache[l] = cache[l] * (1 - min(sum_s mask[l][s], 1)) + sum_s new[s] * mask[l][s]  (fp32 math),
 * with mask [L, S] (mask_row_stride elements between rows) shared by every slab.  Replaces
 * Gemma3Model._apply_update_mask / _apply_update_mask_batch (anemll/models/gemma3_model.py:932-965)
 * as used by _fill_kv_local / _store_kv_local_prefill_masked (967-1022).  For 0/1 masks the values
 * equal the reference's (a zero may differ in sign); rows the mask does not touch are not written.
 */
int anemll_kv_update_mask(void* cache, const void* new_rows, int dtype, const void* mask, int mask_dtype,
                          int64_t mask_row_stride, int64_t n_slabs, int L, int S, int d,
                          int64_t cache_slab_stride, int64_t new_slab_stride, void* stream);

/*
 * Rotating sliding-window update, in place: every slab is shifted left by n rows (the oldest n
 * dropped) and new rows [0, n) are stored at rows [L - n, L).  Replaces Gemma3Model._update_kv_local
 * (n = 1, gemma3_model.py:1024-1066) and _update_kv_local_prefill (n = the prefill batch, 1167-1204).
 * Windows up to 6400 rows (each CTA stages a 32-byte-wide strip of the L rows in shared memory);
 * pointers and slab strides 16-byte aligned, rows whole 16-byte units.
 */
int anemll_kv_rotate_append(void* cache, const void* new_rows, int dtype, int64_t n_slabs, int L, int n, int d,
                            int64_t cache_slab_stride, int64_t new_slab_stride, void* stream);

/*
 * KV-state transition between context sizes: dst [n_slabs][dst_len][d] receives rows
 * [0, current_position) of src [n_slabs][src_len][d] converted to dst_dtype (round to nearest)
 * and pad_value (an fp32 value, converted the same way) everywhere else.  Covers
 * transition_kv_state (expand, anemll/utils/state_transition.py:62-152) and compact_kv_state
 * (shrink with zero padding, 153-357).  dst must not overlap src; both contiguous.
 */
int anemll_kv_state_transition(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n_slabs,
                               int src_len, int dst_len, int d, int current_position, float pad_value, void* stream);

/*
 * anemll_kv_attention with the attention layer's prologue fused in: qkv is one q/k/v projection
 * output, per token H_q x [query | gate] head_dim each, then H_kv x k, then H_kv x v (row stride
 * qkv_row_stride elements, 16-byte units).  Query and key heads get their RMSNorm (q_norm / k_norm
 * fp32 [head_dim], eps; QwenHeadNorm, qwen_model.py:143-184) and rotary embedding at their
 * positions (fp32 cos/sin tables [>= current_pos + S][head_dim]; apply_rotary_pos_emb, 186-261)
 * inside the attention call: the tcgen05 prefill kernel reads its query tile from qkv by TMA and
 * normalises it in shared memory, the new K rows are normed on their way into the cache, the decode
 * kernel normalises its query and key rows as it loads them, and the gate is read in place.  The
 * arithmetic is that of anemll_qk_norm_rope, bit for bit.  Shapes: 8 query heads per kv head with
 * head_dim 128 or 256 and S >= 16 (prefill chunks), or S == 1 (decode); anything else returns
 * ANEMLL_EUNSUPPORTED (use anemll_qk_norm_rope + anemll_kv_attention).  No explicit mask.
 */
int anemll_kv_attention_qkv(const void* qkv, int64_t qkv_row_stride, const float* q_norm, const float* k_norm,
                            const float* cos_table, const float* sin_table, float eps,
                            void* k_cache, void* v_cache, int64_t cache_batch_stride, int64_t cache_head_stride,
                            void* out, int dtype, int B, int S, int H_q, int H_kv, int head_dim, int ctx,
                            int current_pos, int window, int window_chunk_aligned,
                            void* workspace, size_t workspace_bytes, void* stream);

/* ---- decoder-stack epilogues (the hybrid stack's glue between its GEMMs) ---- */

/*
 * RMSNorm over rows of d elements: out = x * rsqrt(mean(x^2) + eps) * weight (fp32 arithmetic, one
 * rounding to dtype).  With residual != NULL the norm is of s = x + residual (rounded to dtype),
 * and s is stored to sum_out (which may be x itself).  The stack's pre-norms and final norm
 * (QwenRMSNorm, anemll/models/qwen_model.py:101-141, with the residual adds of QwenDecoderLayer,
 * 559-577).  weight fp32 [d]; d a multiple of 8, at most 4096; pointers 16-byte aligned.
 */
int anemll_rmsnorm(const void* x, const void* residual, void* sum_out, const float* weight, void* out,
                   int dtype, int64_t rows, int d, float eps, void* stream);

/*
 * SwiGLU activation of a [rows][2 ffn] gate|up GEMM output: out[r][j] = silu(gate) * up, with
 * silu rounded to dtype before the product (QwenMLP.forward, qwen_model.py:286-298).
 */
int anemll_silu_mul(const void* gate_up, void* out, int dtype, int64_t rows, int ffn, void* stream);

/*
 * Attention-layer prologue after the q/k/v projections: per-head RMSNorm of q and k (QwenHeadNorm,
 * qwen_model.py:143-184), rotary embedding at positions [pos, pos + T) from fp32 cos/sin tables
 * [>= pos + T][head_dim] (apply_rotary_pos_emb, 186-261), and the layout change to the attention
 * op's inputs.  q_gate: per token H_q x [query | gate] head_dim each (row stride qg_row_stride
 * elements); k, v: per token H_kv x head_dim.  Outputs q [B][H_q][T][hd], k and v [B][H_kv][T][hd],
 * gate [B][T][H_q hd].  fp16/bf16; head_dim 128 or 256; 16-byte aligned rows.
 */
int anemll_qk_norm_rope(const void* q_gate, int64_t qg_row_stride, const void* k, int64_t k_row_stride,
                        const void* v, int64_t v_row_stride, const float* q_norm, const float* k_norm,
                        const float* cos_table, const float* sin_table, void* q_out, void* k_out, void* v_out,
                        void* gate_out, int dtype, int B, int T, int H_q, int H_kv, int head_dim, int pos,
                        float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ANEMLL_B200_H */
