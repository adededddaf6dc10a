// Fused GDN prologue: causal depthwise conv1d + SiLU, q/k l2-norm, gates.
//
// Channels come in 128-channel head groups (H_qk q-heads, H_qk k-heads, H_v v-heads).  Two kernels:
//
// * Tile kernel (T > DEC_T): a CTA of 128 threads owns one sequence, one head group and TT = 32
//   tokens.  Its input rows (the tile plus the conv_k - 1 rows before it) are copied into shared
//   memory with 16-byte cp.async; each thread then runs the conv + SiLU of a channel pair over half
//   the tile from shared memory into an fp32 tile, and the four warps finish row by row (a warp per
//   token: the q/k l2 norm is a warp reduction, stores are whole 256-byte row segments).
// * Short kernel (T <= DEC_T and conv_k == 4, the decode steps): a thread per channel, the conv
//   window, weights and state in registers (one vector access each), the head's l2 norm a block
//   reduction; one instantiation per T.
//
// The gates (g, beta) are computed by extra CTAs at the end of either grid.  The conv state (last
// conv_k raw inputs per channel, newest last) is read only by the CTA that holds token 0, which is
// also its only writer, so the in-place update has no cross-CTA hazard; the copy is of raw input
// values and therefore bit-exact.  Semantics: modeling_qwen3_5.py:210-226 (update), 453-496
// (prefill conv, split, gates) of transformers 5.5.0.
#include "common.cuh"
#include "mma_sync.cuh"

namespace anemll {
namespace {

constexpr int HDIM = 128;  // channels per head group (d_k == d_v); threads per CTA
constexpr int TT = 32;     // tokens per tile (32: eight CTAs, 32 warps per SM)
constexpr int MAXK = 8;    // largest supported conv kernel
constexpr int DEC_T = 4;   // longest call served by the short kernel
constexpr int SHORT_SB_MIN_B = 16;  // batches from which the short kernel takes four sequences per CTA

__device__ __forceinline__ float load_any(const void* p, int dt, long long i) {
  return dt == ANEMLL_F32 ? reinterpret_cast<const float*>(p)[i]
       : dt == ANEMLL_F16 ? __half2float(reinterpret_cast<const __half*>(p)[i])
                          : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) for one (token, v-head); a and b rows
// (tokens) are ab_ld elements apart, g and beta are dense
__device__ __forceinline__ void gate_elem(long long idx, int Hv, const void* a, const void* bgate, int ab_dt,
                                          long long ab_ld, const float* A_log, const float* dt_bias, float* go,
                                          float* betao) {
  const int h = (int)(idx % Hv);
  const long long src = (idx / Hv) * ab_ld + h;
  float av = load_any(a, ab_dt, src);
  if (dt_bias) av += dt_bias[h];
  const float bv = load_any(bgate, ab_dt, src);
  go[idx] = -expf(A_log[h]) * softplus(av);
  betao[idx] = 1.0f / (1.0f + expf(-bv));
}

// x / (1 + e^-x) with the fast division (relative error a few ulp; the conv output is not rounded
// to a storage type before the l2 norm, so this stays far inside fp32 tolerances)
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// two consecutive elements (4-byte aligned for 2-byte types, 8-byte for fp32) as fp32
template <typename T>
__device__ __forceinline__ float2 ld2f(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return *reinterpret_cast<const float2*>(p);
  } else {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
    return make_float2(to_f32(h[0]), to_f32(h[1]));
  }
}

struct Dst {
  void* p;
  int H, h;
};

__device__ __forceinline__ Dst group_dst(int grp, int Hqk, int Hv, void* qo, void* ko, void* vo) {
  if (grp < Hqk) return {qo, Hqk, grp};
  if (grp < 2 * Hqk) return {ko, Hqk, grp - Hqk};
  return {vo, Hv, grp - 2 * Hqk};
}

// ------------------------------------------------------------------ tile --
// KT: conv_k as a compile-time constant (4, the conv of every Qwen3.5 size), or 0 for a runtime K.
template <typename TIn, typename TOut, int KT>
__global__ void __launch_bounds__(HDIM)
prologue_tile_kernel(const TIn* __restrict__ x, const float* __restrict__ w, TIn* __restrict__ conv_state,
                     const void* __restrict__ a, const void* __restrict__ bgate, int ab_dt, const float* __restrict__ A_log,
                     const float* __restrict__ dt_bias, TOut* __restrict__ qo, TOut* __restrict__ ko,
                     TOut* __restrict__ vo, float* __restrict__ go, float* __restrict__ betao, int B, int T, int Hqk,
                     int Hv, int K, int use_state, int n_tiles, int conv_ctas, long long x_ld, long long ab_ld) {
  if ((int)blockIdx.x >= conv_ctas) {
    const long long idx = (long long)(blockIdx.x - conv_ctas) * HDIM + threadIdx.x;
    if (idx < (long long)B * T * Hv) gate_elem(idx, Hv, a, bgate, ab_dt, ab_ld, A_log, dt_bias, go, betao);
    return;
  }
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int ROWB = HDIM * sizeof(TIn);  // bytes of one input row segment
  TIn* X = reinterpret_cast<TIn*>(smem);    // [TT + MAXK - 1][HDIM]: row r = position t0 - (K-1) + r
  float* Y = reinterpret_cast<float*>(smem + (TT + MAXK - 1) * ROWB);  // [TT][HDIM]

  const int ngroups = 2 * Hqk + Hv;
  const int C = ngroups * HDIM;
  // head groups fastest: neighbouring CTAs read neighbouring 256-byte segments of the same token rows
  const int grp = blockIdx.x % ngroups;
  const int tile = (blockIdx.x / ngroups) % n_tiles;
  const int b = blockIdx.x / (n_tiles * ngroups);
  const int c = threadIdx.x;
  const int t0 = tile * TT, nt = min(TT, T - t0);
  const int nrows = nt + K - 1;
  const TIn* xg = x + (long long)b * T * x_ld + grp * HDIM;  // token rows are x_ld elements apart
  TIn* cs = conv_state + ((long long)b * C + grp * HDIM) * K;

  // rows from x: 16-byte asynchronous copies; rows before token 0: the old state (or zeros)
  constexpr int CPR = ROWB / 16;  // 16-byte chunks per row
  for (int i = c; i < nrows * CPR; i += HDIM) {
    const int r = i / CPR, ch = i % CPR;
    const int pos = t0 - (K - 1) + r;
    if (pos >= 0) cp_async16(reinterpret_cast<uint8_t*>(X) + r * ROWB + ch * 16,
                             reinterpret_cast<const uint8_t*>(xg + (long long)pos * x_ld) + ch * 16);
  }
  cp_async_commit();
  if (t0 == 0) {
    for (int r = 0; r < K - 1; ++r)  // position r - (K-1) = state slot r + 1
      X[r * HDIM + c] = use_state ? cs[(long long)c * K + r + 1] : from_f32<TIn>(0.f);
  }
  // phase 1: thread = (channel pair cc, cc+1; half of the tile's tokens)
  const int cc = 2 * (c & (HDIM / 2 - 1)), half = c / (HDIM / 2);
  float2 wr[MAXK];
#pragma unroll
  for (int j = 0; j < MAXK; ++j)
    wr[j] = j < K ? make_float2(w[(long long)(grp * HDIM + cc) * K + j], w[(long long)(grp * HDIM + cc + 1) * K + j])
                  : make_float2(0.f, 0.f);
  cp_async_wait<0>();
  __syncthreads();

  // conv + SiLU over the tile from shared memory (taps j read rows t + j)
  const int tb = half * (TT / 2), te = min(nt, tb + TT / 2);  // uniform per warp
  if constexpr (KT == 4) {
    // a register window over the rows: one shared-memory load per token
    float2 x0 = ld2f(X + (tb + 0) * HDIM + cc), x1 = ld2f(X + (tb + 1) * HDIM + cc);
    float2 x2 = ld2f(X + (tb + 2) * HDIM + cc);
#pragma unroll
    for (int i = 0; i < TT / 2; ++i) {
      const int t = tb + i;
      if (t < te) {
        const float2 x3 = ld2f(X + (t + 3) * HDIM + cc);
        float a0 = wr[0].x * x0.x, a1 = wr[0].y * x0.y;
        a0 += wr[1].x * x1.x; a1 += wr[1].y * x1.y;
        a0 += wr[2].x * x2.x; a1 += wr[2].y * x2.y;
        a0 += wr[3].x * x3.x; a1 += wr[3].y * x3.y;
        *reinterpret_cast<float2*>(Y + t * HDIM + cc) = make_float2(silu_fast(a0), silu_fast(a1));
        x0 = x1; x1 = x2; x2 = x3;
      }
    }
  } else {
    for (int t = tb; t < te; ++t) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int j = 0; j < MAXK; ++j) {
        if (j < K) {
          const float2 xv = ld2f(X + (t + j) * HDIM + cc);
          a0 += wr[j].x * xv.x;
          a1 += wr[j].y * xv.y;
        }
      }
      *reinterpret_cast<float2*>(Y + t * HDIM + cc) = make_float2(silu_fast(a0), silu_fast(a1));
    }
  }
  if (t0 == 0) {
    // new state = last K entries of cat(old state, x): positions T-K .. T-1; the old state's are in
    // X rows 0 .. K-2 (only reached when T < K, and then the whole sequence is this tile)
    TIn nv[MAXK];
#pragma unroll
    for (int j = 0; j < MAXK; ++j) {
      if (j < K) {
        const int pos = T - K + j;
        nv[j] = pos >= 0 ? xg[(long long)pos * x_ld + c] : X[(pos + K - 1) * HDIM + c];
      }
    }
#pragma unroll
    for (int j = 0; j < MAXK; ++j)
      if (j < K) cs[(long long)c * K + j] = nv[j];
  }
  __syncthreads();

  // rows: warp per token, 4 channels per lane
  const int lane = c & 31, warp = c >> 5;
  const bool norm = grp < 2 * Hqk;
  const Dst d = group_dst(grp, Hqk, Hv, qo, ko, vo);
  TOut* dst = reinterpret_cast<TOut*>(d.p);
  for (int t = warp; t < nt; t += HDIM / 32) {
    float4 v = *reinterpret_cast<const float4*>(Y + t * HDIM + lane * 4);
    if (norm) {
      const float r = rsqrtf(warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w) + 1e-6f);
      v.x *= r; v.y *= r; v.z *= r; v.w *= r;
    }
    TOut* o = dst + (((long long)b * T + t0 + t) * d.H + d.h) * HDIM + lane * 4;
    if constexpr (sizeof(TOut) == 4) {
      *reinterpret_cast<float4*>(o) = v;
    } else {
      TOut h4[4] = {from_f32<TOut>(v.x), from_f32<TOut>(v.y), from_f32<TOut>(v.z), from_f32<TOut>(v.w)};
      *reinterpret_cast<uint2*>(o) = *reinterpret_cast<const uint2*>(h4);
    }
  }
}

// ----------------------------------------------------------------- short --
// conv_k == 4, TS = T tokens (1 .. DEC_T): raw slot s holds position s - 4 (the old state in slots
// 0..3, x[t] in slot 4 + t), so token t's taps are slots t+1 .. t+4 and the new state is slots
// TS .. TS+3, all static register indices.  A CTA takes one channel group of SB sequences (a
// thread per channel): every sequence's loads are issued before the first is used, and the conv
// weights are loaded once for all of them; each sequence's arithmetic (and its norm's reduction
// order) is the same whatever SB is.
template <typename TIn, typename TOut, int TS, int SB>
__global__ void __launch_bounds__(HDIM)
prologue_short_kernel(const TIn* __restrict__ x, const float* __restrict__ w, TIn* __restrict__ conv_state,
                      const void* __restrict__ a, const void* __restrict__ bgate, int ab_dt,
                      const float* __restrict__ A_log, const float* __restrict__ dt_bias, TOut* __restrict__ qo,
                      TOut* __restrict__ ko, TOut* __restrict__ vo, float* __restrict__ go, float* __restrict__ betao,
                      int B, int Hqk, int Hv, int use_state, int conv_ctas, long long x_ld, long long ab_ld) {
  if ((int)blockIdx.x >= conv_ctas) {
    const long long idx = (long long)(blockIdx.x - conv_ctas) * HDIM + threadIdx.x;
    if (idx < (long long)B * TS * Hv) gate_elem(idx, Hv, a, bgate, ab_dt, ab_ld, A_log, dt_bias, go, betao);
    return;
  }
  constexpr int K = 4;
  const int ngroups = 2 * Hqk + Hv;
  const int C = ngroups * HDIM;
  const int grp = blockIdx.x % ngroups, b0 = (blockIdx.x / ngroups) * SB;
  const int c = threadIdx.x, ch = grp * HDIM + c;
  const float4 w4 = *reinterpret_cast<const float4*>(w + (long long)ch * K);

  TIn raw[SB][K + TS];
#pragma unroll
  for (int s = 0; s < SB; ++s) {
    const int b = b0 + s;
#pragma unroll
    for (int j = 0; j < K + TS; ++j) raw[s][j] = from_f32<TIn>(0.f);
    if (b < B) {
      const TIn* cs = conv_state + ((long long)b * C + ch) * K;
      if constexpr (sizeof(TIn) == 2) {
        if (use_state) {
          const uint2 u = *reinterpret_cast<const uint2*>(cs);  // 4 x 2 bytes, 8-byte aligned
          const TIn* s4 = reinterpret_cast<const TIn*>(&u);
#pragma unroll
          for (int j = 0; j < K; ++j) raw[s][j] = s4[j];
        }
      } else {
        if (use_state) {
#pragma unroll
          for (int j = 0; j < K; ++j) raw[s][j] = cs[j];
        }
      }
      const TIn* xg = x + (long long)b * TS * x_ld + ch;
#pragma unroll
      for (int t = 0; t < TS; ++t) raw[s][K + t] = xg[(long long)t * x_ld];
    }
  }

  float y[SB][TS];
#pragma unroll
  for (int s = 0; s < SB; ++s)
#pragma unroll
    for (int t = 0; t < TS; ++t)
      y[s][t] = silu_fast(w4.x * to_f32(raw[s][t + 1]) + w4.y * to_f32(raw[s][t + 2]) +
                          w4.z * to_f32(raw[s][t + 3]) + w4.w * to_f32(raw[s][t + 4]));

  if (grp < 2 * Hqk) {  // q/k head: l2 norm over the 128 channels (4 warps), per sequence and token
    __shared__ float part[HDIM / 32][SB][TS];
    const int lane = c & 31, warp = c >> 5;
#pragma unroll
    for (int s = 0; s < SB; ++s)
#pragma unroll
      for (int t = 0; t < TS; ++t) {
        const float ss = warp_sum(y[s][t] * y[s][t]);
        if (lane == 0) part[warp][s][t] = ss;
      }
    __syncthreads();
#pragma unroll
    for (int s = 0; s < SB; ++s)
#pragma unroll
      for (int t = 0; t < TS; ++t)
        y[s][t] *= rsqrtf(part[0][s][t] + part[1][s][t] + part[2][s][t] + part[3][s][t] + 1e-6f);
  }
  const Dst d = group_dst(grp, Hqk, Hv, qo, ko, vo);
  TOut* dst = reinterpret_cast<TOut*>(d.p);
#pragma unroll
  for (int s = 0; s < SB; ++s) {
    const int b = b0 + s;
    if (b >= B) break;
#pragma unroll
    for (int t = 0; t < TS; ++t) dst[(((long long)b * TS + t) * d.H + d.h) * HDIM + c] = from_f32<TOut>(y[s][t]);
    TIn* cs = conv_state + ((long long)b * C + ch) * K;
    if constexpr (sizeof(TIn) == 2) {  // new state: slots TS .. TS + 3
      const TIn s4[4] = {raw[s][TS], raw[s][TS + 1], raw[s][TS + 2], raw[s][TS + 3]};
      *reinterpret_cast<uint2*>(cs) = *reinterpret_cast<const uint2*>(s4);
    } else {
#pragma unroll
      for (int j = 0; j < K; ++j) cs[j] = raw[s][TS + j];
    }
  }
}

template <typename TIn, typename TOut>
int launch_prologue(const void* x, const float* w, void* cs, const void* a, const void* bg, int ab_dt,
                    const float* A_log, const float* dt_bias, void* qo, void* ko, void* vo, float* go, float* bo,
                    int B, int T, int Hqk, int Hv, int K, int use_state, long long x_ld, long long ab_ld,
                    cudaStream_t st) {
  const int ngroups = 2 * Hqk + Hv;
  const long long gate_ctas = ((long long)B * T * Hv + HDIM - 1) / HDIM;
  if (T <= DEC_T && K == 4) {
    // four sequences per CTA once there are enough of them to fill the SMs
    const int sb = B >= SHORT_SB_MIN_B ? 4 : 1;
    const long long conv_ctas = (long long)((B + sb - 1) / sb) * ngroups;
    ANEMLL_REQUIRE(conv_ctas + gate_ctas < (1LL << 31), ANEMLL_EINVAL, "gdn_prologue: problem too large");
    const unsigned grid = (unsigned)(conv_ctas + gate_ctas);
    auto go_short = [&](auto kern) {
      kern<<<grid, HDIM, 0, st>>>((const TIn*)x, w, (TIn*)cs, a, bg, ab_dt, A_log, dt_bias, (TOut*)qo, (TOut*)ko,
                                  (TOut*)vo, go, bo, B, Hqk, Hv, use_state, (int)conv_ctas, x_ld, ab_ld);
    };
    if (sb == 4) {
      switch (T) {
        case 1: go_short(prologue_short_kernel<TIn, TOut, 1, 4>); break;
        case 2: go_short(prologue_short_kernel<TIn, TOut, 2, 4>); break;
        case 3: go_short(prologue_short_kernel<TIn, TOut, 3, 4>); break;
        default: go_short(prologue_short_kernel<TIn, TOut, 4, 4>); break;
      }
    } else {
      switch (T) {
        case 1: go_short(prologue_short_kernel<TIn, TOut, 1, 1>); break;
        case 2: go_short(prologue_short_kernel<TIn, TOut, 2, 1>); break;
        case 3: go_short(prologue_short_kernel<TIn, TOut, 3, 1>); break;
        default: go_short(prologue_short_kernel<TIn, TOut, 4, 1>); break;
      }
    }
  } else {
    const int n_tiles = (T + TT - 1) / TT;
    const long long conv_ctas = (long long)B * ngroups * n_tiles;
    ANEMLL_REQUIRE(conv_ctas + gate_ctas < (1LL << 31), ANEMLL_EINVAL, "gdn_prologue: problem too large");
    const size_t smem = (size_t)(TT + MAXK - 1) * HDIM * sizeof(TIn) + (size_t)TT * HDIM * sizeof(float);
    auto go_tile = [&](auto kern) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      kern<<<(unsigned)(conv_ctas + gate_ctas), HDIM, smem, st>>>(
          (const TIn*)x, w, (TIn*)cs, a, bg, ab_dt, A_log, dt_bias, (TOut*)qo, (TOut*)ko, (TOut*)vo, go, bo, B, T,
          Hqk, Hv, K, use_state, n_tiles, (int)conv_ctas, x_ld, ab_ld);
    };
    if (K == 4) go_tile(prologue_tile_kernel<TIn, TOut, 4>);
    else go_tile(prologue_tile_kernel<TIn, TOut, 0>);
  }
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
                                   int use_state, int64_t x_row_stride, int64_t ab_row_stride, void* stream) {
  ANEMLL_REQUIRE(mixed_qkv && conv_w && conv_state && a && b && A_log && q_out && k_out && v_out && g_out &&
                     beta_out,
                 ANEMLL_EINVAL, "gdn_prologue: null pointer");
  ANEMLL_REQUIRE(B > 0 && T > 0 && H_qk > 0 && H_v > 0, ANEMLL_EINVAL, "gdn_prologue: bad sizes");
  ANEMLL_REQUIRE(d_k == HDIM && d_v == HDIM, ANEMLL_EUNSUPPORTED, "gdn_prologue: d_k and d_v must be 128");
  ANEMLL_REQUIRE(conv_k >= 1 && conv_k <= MAXK, ANEMLL_EUNSUPPORTED, "gdn_prologue: conv_k must be in [1, %d]", MAXK);
  ANEMLL_REQUIRE(dtype_ok(in_dtype) && dtype_ok(ab_dtype) && dtype_ok(out_dtype), ANEMLL_EUNSUPPORTED,
                 "gdn_prologue: bad dtype");
  const long long C = (2LL * H_qk + H_v) * HDIM;
  const long long x_ld = x_row_stride ? x_row_stride : C, ab_ld = ab_row_stride ? ab_row_stride : H_v;
  ANEMLL_REQUIRE(x_ld >= C && ab_ld >= H_v, ANEMLL_EINVAL, "gdn_prologue: row strides shorter than the rows");
  ANEMLL_REQUIRE(x_ld * dtype_size(in_dtype) % 16 == 0, ANEMLL_EINVAL,
                 "gdn_prologue: the mixed_qkv row stride must be a multiple of 16 bytes");
  ANEMLL_REQUIRE(aligned(mixed_qkv, 16) && aligned(conv_w, 16) && aligned(conv_state, 8) && aligned(q_out, 16) &&
                     aligned(k_out, 16) && aligned(v_out, 16),
                 ANEMLL_EINVAL, "gdn_prologue: mixed_qkv, conv_w and the outputs must be 16-byte aligned, "
                                "conv_state 8-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  return ANEMLL_DISPATCH_DTYPE(in_dtype, TIn, [&] {
    return ANEMLL_DISPATCH_DTYPE(out_dtype, TOut, [&] {
      return launch_prologue<TIn, TOut>(mixed_qkv, conv_w, conv_state, a, b, ab_dtype, A_log, dt_bias, q_out, k_out,
                                        v_out, g_out, beta_out, B, T, H_qk, H_v, conv_k, use_state, x_ld, ab_ld, st);
    });
  });
}
