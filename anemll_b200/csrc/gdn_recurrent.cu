// Gated delta rule, token-by-token form (decode, and recurrent prefill).
//
// Per (sequence b, value head h) the fp32 state S[d_k=128][d_v] is streamed
// from HBM once per launch, kept in registers across the launch's T tokens,
// and written back once.  One CTA owns a DVT-column slice of one state: the
// columns of S evolve independently (column j only needs v[j]), so a slice is
// a complete sub-problem.  Each thread holds RPT rows x 4 columns (float4), a
// warp reads whole 4*CG-float row segments, so loads and stores are 16-byte
// vectors on contiguous 64/128-byte runs.
//
// Per token, with q, k l2-normalised and q scaled:
//   pk = S^T k, pq = S^T q            (one pass over the register tile)
//   delta = beta * (v - e^g pk)
//   o     = e^g pq + delta * (k . q)  (= S_new^T q without a second pass)
//   S     = e^g S + k delta^T
// Semantics follow torch_recurrent_gated_delta_rule (transformers 5.5.0,
// modeling_qwen3_5.py:314-353).
#include "common.cuh"

namespace anemll {
namespace {

constexpr int DK = 128;

template <typename TIn, typename TOut, int DVT, int NT>
__global__ void __launch_bounds__(NT)
gdn_recurrent_kernel(const TIn* __restrict__ q, const TIn* __restrict__ k, const TIn* __restrict__ v,
                     const float* __restrict__ g, const float* __restrict__ beta,
                     float* __restrict__ state, TOut* __restrict__ out,
                     int T, int Hqk, int Hv, int dv, float scale, int l2norm) {
  constexpr int CG = DVT / 4;   // float4 column groups per row
  constexpr int RG = NT / CG;   // row groups
  constexpr int RPT = DK / RG;  // rows per thread
  constexpr int NWARP = NT / 32;
  static_assert(CG <= 32 && (32 % CG) == 0, "column groups must tile a warp");
  static_assert(DK % RG == 0, "rows must split evenly");

  const int slice = blockIdx.x;
  const int hv = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = hv / (Hv / Hqk);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int cg = tid % CG;
  const int rg = tid / CG;
  const int col0 = slice * DVT + cg * 4;

  float* S = state + (size_t)(b * Hv + hv) * DK * dv;
  float4 s[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg + i * RG;
    s[i] = *reinterpret_cast<const float4*>(S + (size_t)r * dv + col0);
  }

  // double-buffered by token parity: a thread can be at most one token ahead
  __shared__ float sq[2][DK];
  __shared__ float sk[2][DK];
  __shared__ float red[2][2][NWARP][DVT];
  __shared__ float scal[2][4];

  for (int t = 0; t < T; ++t) {
    const int p = t & 1;
    const size_t tok = (size_t)b * T + t;
    const TIn* qt = q + (tok * Hqk + hk) * DK;
    const TIn* kt = k + (tok * Hqk + hk) * DK;
    for (int i = tid; i < DK; i += NT) {
      sq[p][i] = to_f32(qt[i]);
      sk[p][i] = to_f32(kt[i]);
    }
    const float gt = g[tok * Hv + hv];
    const float bt = beta[tok * Hv + hv];
    float vv[4];
    const TIn* vt = v + (tok * Hv + hv) * dv + col0;
#pragma unroll
    for (int c = 0; c < 4; ++c) vv[c] = to_f32(vt[c]);
    __syncthreads();
    if (warp == 0) {
      float a = 0.f, bb = 0.f, c = 0.f;
#pragma unroll
      for (int i = lane; i < DK; i += 32) {
        const float x = sq[p][i], y = sk[p][i];
        a += x * x;
        bb += y * y;
        c += x * y;
      }
      a = warp_sum(a);
      bb = warp_sum(bb);
      c = warp_sum(c);
      if (lane == 0) {
        const float rq = l2norm ? rsqrtf(a + 1e-6f) : 1.f;
        const float rk = l2norm ? rsqrtf(bb + 1e-6f) : 1.f;
        scal[p][0] = rq * scale;
        scal[p][1] = rk;
        scal[p][2] = c * rq * scale * rk;
      }
    }
    __syncthreads();
    const float qs = scal[p][0], ks = scal[p][1], kq = scal[p][2];
    float pk[4] = {0.f, 0.f, 0.f, 0.f}, pq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg + i * RG;
      const float kr = sk[p][r] * ks, qr = sq[p][r] * qs;
      pk[0] += s[i].x * kr; pk[1] += s[i].y * kr; pk[2] += s[i].z * kr; pk[3] += s[i].w * kr;
      pq[0] += s[i].x * qr; pq[1] += s[i].y * qr; pq[2] += s[i].z * qr; pq[3] += s[i].w * qr;
    }
#pragma unroll
    for (int o = CG; o < 32; o <<= 1) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        pk[c] += __shfl_xor_sync(0xffffffffu, pk[c], o);
        pq[c] += __shfl_xor_sync(0xffffffffu, pq[c], o);
      }
    }
    if (lane < CG) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        red[p][0][warp][cg * 4 + c] = pk[c];
        red[p][1][warp][cg * 4 + c] = pq[c];
      }
    }
    __syncthreads();
    const float dec = __expf(gt);
    float delta[4], o[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float a = 0.f, bb = 0.f;
#pragma unroll
      for (int w = 0; w < NWARP; ++w) {
        a += red[p][0][w][cg * 4 + c];
        bb += red[p][1][w][cg * 4 + c];
      }
      delta[c] = bt * (vv[c] - dec * a);
      o[c] = dec * bb + delta[c] * kq;
    }
    if (rg == 0) {
      TOut* ot = out + (tok * Hv + hv) * dv + col0;
#pragma unroll
      for (int c = 0; c < 4; ++c) ot[c] = from_f32<TOut>(o[c]);
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg + i * RG;
      const float kr = sk[p][r] * ks;
      s[i].x = dec * s[i].x + kr * delta[0];
      s[i].y = dec * s[i].y + kr * delta[1];
      s[i].z = dec * s[i].z + kr * delta[2];
      s[i].w = dec * s[i].w + kr * delta[3];
    }
  }

#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg + i * RG;
    *reinterpret_cast<float4*>(S + (size_t)r * dv + col0) = s[i];
  }
}

template <typename TIn, typename TOut>
int launch_recurrent(const void* q, const void* k, const void* v, const float* g, const float* beta,
                     float* state, void* out, int B, int T, int Hqk, int Hv, int dv, float scale,
                     int l2norm, cudaStream_t st) {
  // Narrow slices when there are few (b, h) pairs so the grid still covers the SMs.
  const long pairs = (long)B * Hv;
  const bool narrow = pairs * (dv / 32) < 2 * 148 && (dv % 16) == 0;
  if (narrow) {
    dim3 grid(dv / 16, Hv, B);
    gdn_recurrent_kernel<TIn, TOut, 16, 128><<<grid, 128, 0, st>>>(
        (const TIn*)q, (const TIn*)k, (const TIn*)v, g, beta, state, (TOut*)out, T, Hqk, Hv, dv, scale, l2norm);
  } else {
    dim3 grid(dv / 32, Hv, B);
    gdn_recurrent_kernel<TIn, TOut, 32, 128><<<grid, 128, 0, st>>>(
        (const TIn*)q, (const TIn*)k, (const TIn*)v, g, beta, state, (TOut*)out, T, Hqk, Hv, dv, scale, l2norm);
  }
  return launch_status("gdn_recurrent");
}

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_gdn_recurrent(const void* q, const void* k, const void* v, int qkv_dtype,
                                    const float* g, const float* beta, float* state,
                                    void* out, int out_dtype,
                                    int B, int T, int H_qk, int H_v, int d_k, int d_v,
                                    float scale, int qk_l2norm, void* stream) {
  ANEMLL_REQUIRE(state && (T == 0 || (q && k && v && g && beta && out)), ANEMLL_EINVAL,
                 "gdn_recurrent: null pointer");
  ANEMLL_REQUIRE(B > 0 && T >= 0 && H_qk > 0 && H_v > 0, ANEMLL_EINVAL,
                 "gdn_recurrent: bad sizes B=%d T=%d H_qk=%d H_v=%d", B, T, H_qk, H_v);
  ANEMLL_REQUIRE(H_v % H_qk == 0, ANEMLL_EINVAL, "gdn_recurrent: H_v (%d) must be a multiple of H_qk (%d)", H_v, H_qk);
  ANEMLL_REQUIRE(d_k == DK, ANEMLL_EUNSUPPORTED, "gdn_recurrent: d_k must be 128 (got %d)", d_k);
  ANEMLL_REQUIRE(d_v > 0 && d_v % 32 == 0, ANEMLL_EUNSUPPORTED, "gdn_recurrent: d_v must be a multiple of 32 (got %d)", d_v);
  ANEMLL_REQUIRE(dtype_ok(qkv_dtype) && dtype_ok(out_dtype), ANEMLL_EUNSUPPORTED, "gdn_recurrent: bad dtype");
  ANEMLL_REQUIRE(aligned(state, 16), ANEMLL_EALIGN, "gdn_recurrent: state must be 16-byte aligned");
  if (T == 0) return ANEMLL_OK;
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)d_k);
  cudaStream_t st = (cudaStream_t)stream;
  return ANEMLL_DISPATCH_DTYPE(qkv_dtype, TIn, [&] {
    return ANEMLL_DISPATCH_DTYPE(out_dtype, TOut, [&] {
      return launch_recurrent<TIn, TOut>(q, k, v, g, beta, state, out, B, T, H_qk, H_v, d_v, scale, qk_l2norm, st);
    });
  });
}
