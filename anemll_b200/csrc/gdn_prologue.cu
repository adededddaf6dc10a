// Fused GDN prologue: causal depthwise conv1d + SiLU, q/k l2-norm, gates.
//
// Grid: x = token tiles of TT tokens, y = 128-channel head groups
// (H_qk q-heads, H_qk k-heads, H_v v-heads) plus one gate group, z = batch.
// One thread per channel walks the tile's TT tokens with a conv_k-deep sliding
// window in registers; the per-token l2 norm of a q/k head is a 128-channel
// block reduction.  Reads and writes are coalesced along channels.
//
// The conv state (last conv_k raw inputs, newest last) is read only by the
// tile-0 CTA of each channel group, which is also the only writer, so the
// in-place update has no cross-CTA hazard; the copy is of raw input values and
// therefore bit-exact.  Semantics: modeling_qwen3_5.py:210-226 (update),
// 453-496 (prefill conv, split, gates) of transformers 5.5.0.
#include "common.cuh"

namespace anemll {
namespace {

constexpr int CH = 128;     // channels per head group == threads per CTA
constexpr int TT = 16;      // tokens per CTA
constexpr int MAXK = 8;     // largest supported conv kernel

template <typename TIn, typename TAB, typename TOut>
__global__ void __launch_bounds__(CH)
gdn_prologue_kernel(const TIn* __restrict__ x, const float* __restrict__ w, TIn* __restrict__ conv_state,
                    const TAB* __restrict__ a, const TAB* __restrict__ bgate,
                    const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                    TOut* __restrict__ qo, TOut* __restrict__ ko, TOut* __restrict__ vo,
                    float* __restrict__ go, float* __restrict__ betao,
                    int T, int Hqk, int Hv, int K, int use_state) {
  const int tile = blockIdx.x;
  const int grp = blockIdx.y;
  const int b = blockIdx.z;
  const int c = threadIdx.x;
  const int t0 = tile * TT;
  const int ngroups = 2 * Hqk + Hv;

  if (grp == ngroups) {  // gates
    for (int i = c; i < TT * Hv; i += CH) {
      const int t = t0 + i / Hv;
      const int h = i % Hv;
      if (t >= T) continue;
      const size_t idx = ((size_t)b * T + t) * Hv + h;
      float av = to_f32(a[idx]);
      if (dt_bias) av += dt_bias[h];
      const float bv = to_f32(bgate[idx]);
      go[idx] = -expf(A_log[h]) * softplus(av);
      betao[idx] = 1.0f / (1.0f + expf(-bv));
    }
    return;
  }

  const int C = ngroups * CH;
  const int ch = grp * CH + c;
  const float* wc = w + (size_t)ch * K;
  float wr[MAXK];
#pragma unroll
  for (int j = 0; j < MAXK; ++j) wr[j] = j < K ? wc[j] : 0.f;

  // history: raw inputs at relative positions t0-K+1 .. t0-1 (window slots 1..K-1)
  float win[MAXK];
  TIn* cs = conv_state + ((size_t)b * C + ch) * K;
  TIn old_state[MAXK];
  if (tile == 0) {
#pragma unroll
    for (int j = 0; j < MAXK; ++j) old_state[j] = j < K && use_state ? cs[j] : from_f32<TIn>(0.f);
  }
#pragma unroll
  for (int j = 0; j < MAXK; ++j) {
    // slot j holds position t0 - K + j  (slot K-1 is the newest before t0)
    const int pos = t0 - K + j;
    float val = 0.f;
    if (j < K) {
      if (pos >= 0) val = to_f32(x[((size_t)b * T + pos) * C + ch]);
      else if (use_state) val = to_f32(old_state[K + pos]);  // pos in [-K, -1]; only tile 0 reaches here
    }
    win[j] = val;
  }

  float y[TT];
#pragma unroll
  for (int i = 0; i < TT; ++i) {
    const int t = t0 + i;
    const float xn = t < T ? to_f32(x[((size_t)b * T + t) * C + ch]) : 0.f;
    // shift the window left by one and append x[t]
#pragma unroll
    for (int j = 0; j < MAXK - 1; ++j) win[j] = (j + 1 < K) ? win[j + 1] : win[j];
    if (K - 1 < MAXK) {
#pragma unroll
      for (int j = 0; j < MAXK; ++j) if (j == K - 1) win[j] = xn;
    }
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < MAXK; ++j) if (j < K) acc += wr[j] * win[j];
    y[i] = silu(acc);
  }

  const bool is_q = grp < Hqk;
  const bool is_k = !is_q && grp < 2 * Hqk;
  if (is_q || is_k) {
    __shared__ float part[CH / 32][TT];
    const int lane = c & 31, warp = c >> 5;
#pragma unroll
    for (int i = 0; i < TT; ++i) {
      const float ss = warp_sum(y[i] * y[i]);
      if (lane == 0) part[warp][i] = ss;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < TT; ++i) {
      float ss = 0.f;
#pragma unroll
      for (int ww = 0; ww < CH / 32; ++ww) ss += part[ww][i];
      y[i] *= rsqrtf(ss + 1e-6f);
    }
    const int h = is_q ? grp : grp - Hqk;
    TOut* dst = is_q ? qo : ko;
#pragma unroll
    for (int i = 0; i < TT; ++i) {
      const int t = t0 + i;
      if (t < T) dst[(((size_t)b * T + t) * Hqk + h) * CH + c] = from_f32<TOut>(y[i]);
    }
  } else {
    const int h = grp - 2 * Hqk;
#pragma unroll
    for (int i = 0; i < TT; ++i) {
      const int t = t0 + i;
      if (t < T) vo[(((size_t)b * T + t) * Hv + h) * CH + c] = from_f32<TOut>(y[i]);
    }
  }

  if (tile == 0) {
    // new state = last K entries of cat(history, x): relative positions T-K .. T-1
#pragma unroll
    for (int j = 0; j < MAXK; ++j) {
      if (j >= K) break;
      const int pos = T - K + j;
      TIn val;
      if (pos >= 0) val = x[((size_t)b * T + pos) * C + ch];
      else val = old_state[K + pos];
      cs[j] = val;
    }
  }
}

template <typename TIn, typename TAB, typename TOut>
int launch_prologue(const void* x, const float* w, void* cs, const void* a, const void* bg, const float* A_log,
                    const float* dt_bias, void* qo, void* ko, void* vo, float* go, float* bo, int B, int T,
                    int Hqk, int Hv, int K, int use_state, cudaStream_t st) {
  dim3 grid((T + TT - 1) / TT, 2 * Hqk + Hv + 1, B);
  gdn_prologue_kernel<TIn, TAB, TOut><<<grid, CH, 0, st>>>(
      (const TIn*)x, w, (TIn*)cs, (const TAB*)a, (const TAB*)bg, A_log, dt_bias, (TOut*)qo, (TOut*)ko,
      (TOut*)vo, go, bo, T, Hqk, Hv, K, use_state);
  return launch_status("gdn_prologue");
}

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_gdn_prologue(const void* mixed_qkv, int in_dtype, const float* conv_w, void* conv_state,
                                   const void* a, const void* b, int ab_dtype,
                                   const float* A_log, const float* dt_bias,
                                   void* q_out, void* k_out, void* v_out, int out_dtype,
                                   float* g_out, float* beta_out,
                                   int B, int T, int H_qk, int H_v, int d_k, int d_v, int conv_k,
                                   int use_state, void* stream) {
  ANEMLL_REQUIRE(mixed_qkv && conv_w && conv_state && a && b && A_log && q_out && k_out && v_out && g_out &&
                     beta_out,
                 ANEMLL_EINVAL, "gdn_prologue: null pointer");
  ANEMLL_REQUIRE(B > 0 && T > 0 && H_qk > 0 && H_v > 0, ANEMLL_EINVAL, "gdn_prologue: bad sizes");
  ANEMLL_REQUIRE(d_k == CH && d_v == CH, ANEMLL_EUNSUPPORTED, "gdn_prologue: d_k and d_v must be 128");
  ANEMLL_REQUIRE(conv_k >= 1 && conv_k <= MAXK, ANEMLL_EUNSUPPORTED, "gdn_prologue: conv_k must be in [1, %d]", MAXK);
  ANEMLL_REQUIRE(dtype_ok(in_dtype) && dtype_ok(ab_dtype) && dtype_ok(out_dtype), ANEMLL_EUNSUPPORTED,
                 "gdn_prologue: bad dtype");
  cudaStream_t st = (cudaStream_t)stream;
  return ANEMLL_DISPATCH_DTYPE(in_dtype, TIn, [&] {
    return ANEMLL_DISPATCH_DTYPE(ab_dtype, TAB, [&] {
      return ANEMLL_DISPATCH_DTYPE(out_dtype, TOut, [&] {
        return launch_prologue<TIn, TAB, TOut>(mixed_qkv, conv_w, conv_state, a, b, A_log, dt_bias, q_out, k_out,
                                               v_out, g_out, beta_out, B, T, H_qk, H_v, conv_k, use_state, st);
      });
    });
  });
}
