// Fused elementwise/normalisation kernels between the decoder stack's GEMMs: they replace chains of
// small framework kernels (fp32 conversions, reductions, rotations, copies), each HBM-bound, one
// pass over their rows, 16-byte vectors.
//
//   rmsnorm      out = bf(x * rsqrt(mean(x^2) + eps) * w), optionally after the residual add
//                s = bf(x + r) (s written back); a CTA per row (a warp per row for rows of at
//                most 256 elements);
//   silu_mul     out = bf(bf(silu(gate)) * up) for a [gate | up] GEMM output (SwiGLU; the fast
//                exponential and division, whose few-ulp error vanishes in the rounding to bf16);
//   qk_norm_rope per-head RMSNorm of q and k (QwenHeadNorm, anemll/models/qwen_model.py:143-184)
//                then the rotary embedding x cos + rotate_half(x) sin (apply_rotary_pos_emb,
//                qwen_model.py:186-261), q/k/v moved to the head-major layout the attention op
//                reads and the output gate split off, one pass.
//
// Rounding follows the framework ops they replace: fp32 arithmetic, one rounding to the storage
// type per materialised tensor (the rotation's products and sum are rounded separately in fp32, as
// two elementwise kernels would).
#include "common.cuh"

namespace anemll {
namespace {

constexpr int NT = 256;

// ---------------------------------------------------------------- RMSNorm --
// Raw 16-byte vectors of 8 elements (two for fp32), so that all of a lane's loads are issued before
// the first is used.
template <typename T> struct V8 { uint4 u; };
template <> struct V8<float> { float4 a, b; };
template <typename T>
__device__ __forceinline__ V8<T> ldv8(const T* p) {
  V8<T> r;
  if constexpr (sizeof(T) == 4) {
    r.a = reinterpret_cast<const float4*>(p)[0];
    r.b = reinterpret_cast<const float4*>(p)[1];
  } else {
    r.u = *reinterpret_cast<const uint4*>(p);
  }
  return r;
}
template <typename T>
__device__ __forceinline__ void cvt8(const V8<T>& r, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = r.a.x; f[1] = r.a.y; f[2] = r.a.z; f[3] = r.a.w; f[4] = r.b.x; f[5] = r.b.y; f[6] = r.b.z; f[7] = r.b.w;
  } else {
    const T* h = reinterpret_cast<const T*>(&r.u);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = to_f32(h[e]);
  }
}

// The row's 8-element chunks ch = first, first + step, ... (at most NC of them) held in registers.
// sum_out may alias x (in-place residual add): every element is read before it is written, by the
// same thread.  Returns the partial sum of squares.
template <typename T, int NC>
__device__ __forceinline__ float rms_load(const T* x, const T* res, int d, int first, int step, float (&v)[NC][8]) {
  V8<T> rx[NC], rr[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (first + c * step) * 8;
    if (col < d) {
      rx[c] = ldv8(x + col);
      if (res) rr[c] = ldv8(res + col);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (first + c * step) * 8;
    if (col < d) {
      cvt8(rx[c], v[c]);
      if (res) {
        float r8[8];
        cvt8(rr[c], r8);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[c][e] = to_f32(from_f32<T>(v[c][e] + r8[e]));  // the stored sum
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[c][e] * v[c][e];
    }
  }
  return ss;
}

template <typename T, int NC>
__device__ __forceinline__ void rms_store(T* sum_out, bool has_res, const float* __restrict__ w, T* out, int d,
                                          int first, int step, float r, const float (&v)[NC][8]) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (first + c * step) * 8;
    if (col < d) {
      if (has_res) store8(sum_out + col, v[c]);
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(__fmul_rn(v[c][e], r), w[col + e]);
      store8(out + col, o);
    }
  }
}

// short rows: a warp per row
template <typename T, int NC>
__global__ void __launch_bounds__(NT)
rmsnorm_kernel(const T* x, const T* res, T* sum_out, const float* __restrict__ w, T* __restrict__ out,
               long long rows, int d, float eps) {
  const long long row = (long long)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[NC][8];
  const float ss = warp_sum(rms_load<T, NC>(x + row * d, res ? res + row * d : nullptr, d, lane, 32, v));
  const float r = rsqrtf(ss / (float)d + eps);
  rms_store<T, NC>(res ? sum_out + row * d : nullptr, res != nullptr, w, out + row * d, d, lane, 32, r, v);
}

// a CTA per row: eight warps share the row, so that few rows (decode) spread over the SMs and many
// rows keep several loads in flight per thread at low register use
template <typename T>
__global__ void __launch_bounds__(NT)
rmsnorm_row_kernel(const T* x, const T* res, T* sum_out, const float* __restrict__ w, T* __restrict__ out, int d,
                   float eps) {
  constexpr int NC = 2;  // d <= 2 * 8 * NT
  const long long row = blockIdx.x;
  __shared__ float part[NT / 32];
  float v[NC][8];
  float ss = warp_sum(rms_load<T, NC>(x + row * d, res ? res + row * d : nullptr, d, threadIdx.x, NT, v));
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) ss += part[i];
  const float r = rsqrtf(ss / (float)d + eps);
  rms_store<T, NC>(res ? sum_out + row * d : nullptr, res != nullptr, w, out + row * d, d, threadIdx.x, NT, r, v);
}

// --------------------------------------------------------------- SiLU * up --
template <typename T>
__global__ void __launch_bounds__(NT)
silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ out, long long rows, int ffn) {
  const int per_row = ffn / 8;
  const long long i = (long long)blockIdx.x * NT + threadIdx.x;
  if (i >= rows * per_row) return;
  const long long row = i / per_row;
  const int col = (int)(i % per_row) * 8;
  float g[8], u[8], o[8];
  load8(gu + row * 2 * ffn + col, g);
  load8(gu + row * 2 * ffn + ffn + col, u);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float s = to_f32(from_f32<T>(__fdividef(g[e], 1.0f + __expf(-g[e]))));  // rounded to T, as stored
    o[e] = s * u[e];
  }
  store8(out + row * ffn + col, o);
}

// ------------------------------------------------- head norm + RoPE + layout --
// One CTA per token; warp w takes rows w, w+8, ... of the token's 2 H_q + 2 H_kv rows:
// q heads, k heads (normed and rotated), v heads (moved), gate slices (moved).
// EPL = head_dim / 32 elements per lane; lane l holds [l*EPL, (l+1)*EPL), and the rotation's
// partner elements (i +- head_dim/2) sit in lane l ^ 16.
template <typename T, int EPL>
__global__ void __launch_bounds__(NT)
qk_norm_rope_kernel(const T* __restrict__ qg, long long qg_ld, const T* __restrict__ kin, long long k_ld,
                    const T* __restrict__ vin, long long v_ld, const float* __restrict__ qw,
                    const float* __restrict__ kw, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                    T* __restrict__ qo, T* __restrict__ ko, T* __restrict__ vo, T* __restrict__ go,
                    int T_len, int Hq, int Hkv, int pos, float eps) {
  constexpr int HD = EPL * 32;
  const long long tok = blockIdx.x;  // b * T + t
  const int b = (int)(tok / T_len), t = (int)(tok % T_len);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nrows = 2 * Hq + 2 * Hkv;
  const float* cr = cos_t + (long long)(pos + t) * HD;
  const float* sr = sin_t + (long long)(pos + t) * HD;
  for (int r = warp; r < nrows; r += NT / 32) {
    const T* src;
    T* dst;
    const float* nw = nullptr;
    if (r < Hq) {
      src = qg + tok * qg_ld + (long long)r * 2 * HD;
      dst = qo + (((long long)b * Hq + r) * T_len + t) * HD;
      nw = qw;
    } else if (r < Hq + Hkv) {
      const int h = r - Hq;
      src = kin + tok * k_ld + (long long)h * HD;
      dst = ko + (((long long)b * Hkv + h) * T_len + t) * HD;
      nw = kw;
    } else if (r < Hq + 2 * Hkv) {
      const int h = r - Hq - Hkv;
      src = vin + tok * v_ld + (long long)h * HD;
      dst = vo + (((long long)b * Hkv + h) * T_len + t) * HD;
    } else {
      const int h = r - Hq - 2 * Hkv;
      src = qg + tok * qg_ld + (long long)h * 2 * HD + HD;
      dst = go + (tok * Hq + h) * HD;
    }
    float x[EPL];
    if constexpr (EPL == 8) {
      load8(src + lane * 8, x);
    } else {
#pragma unroll
      for (int e = 0; e < EPL; ++e) x[e] = to_f32(src[lane * EPL + e]);
    }
    if (nw) head_norm_rope_warp<T, EPL>(x, nw, cr, sr, eps, lane);
    if constexpr (EPL == 8) {
      store8(dst + lane * 8, x);
    } else {
#pragma unroll
      for (int e = 0; e < EPL; ++e) dst[lane * EPL + e] = from_f32<T>(x[e]);
    }
  }
}

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_rmsnorm(const void* x, const void* residual, void* sum_out, const float* weight, void* out,
                              int dtype, int64_t rows, int d, float eps, void* stream) {
  ANEMLL_REQUIRE(x && weight && out, ANEMLL_EINVAL, "rmsnorm: null pointer");
  ANEMLL_REQUIRE(!residual || sum_out, ANEMLL_EINVAL, "rmsnorm: a residual needs sum_out");
  ANEMLL_REQUIRE(rows >= 0 && rows < (1LL << 31) && d > 0 && d % 8 == 0 && d <= 4096, ANEMLL_EUNSUPPORTED,
                 "rmsnorm: d must be a multiple of 8 and at most 4096 (got %d)", d);
  ANEMLL_REQUIRE(dtype_ok(dtype), ANEMLL_EUNSUPPORTED, "rmsnorm: bad dtype");
  ANEMLL_REQUIRE(aligned(x, 16) && aligned(out, 16) && (!residual || (aligned(residual, 16) && aligned(sum_out, 16))),
                 ANEMLL_EINVAL, "rmsnorm: tensors must be 16-byte aligned");
  if (rows == 0) return ANEMLL_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned blocks = (unsigned)((rows + NT / 32 - 1) / (NT / 32));
  const int nc = (d + 255) / 256;
  return ANEMLL_DISPATCH_DTYPE(dtype, T, [&] {
    const T* xx = (const T*)x;
    const T* rr = (const T*)residual;
    // rows of more than 256 elements: a CTA per row (8 warps, a few loads in flight per thread, low
    // register use); shorter rows: a warp per row
    if (nc > 1)
      rmsnorm_row_kernel<T><<<(unsigned)rows, NT, 0, st>>>(xx, rr, (T*)sum_out, weight, (T*)out, d, eps);
    else
      rmsnorm_kernel<T, 1><<<blocks, NT, 0, st>>>(xx, rr, (T*)sum_out, weight, (T*)out, rows, d, eps);
    return launch_status("rmsnorm");
  });
}

extern "C" int anemll_silu_mul(const void* gate_up, void* out, int dtype, int64_t rows, int ffn, void* stream) {
  ANEMLL_REQUIRE(gate_up && out, ANEMLL_EINVAL, "silu_mul: null pointer");
  ANEMLL_REQUIRE(rows >= 0 && ffn > 0 && ffn % 8 == 0, ANEMLL_EUNSUPPORTED, "silu_mul: ffn must be a multiple of 8");
  ANEMLL_REQUIRE(dtype_ok(dtype), ANEMLL_EUNSUPPORTED, "silu_mul: bad dtype");
  ANEMLL_REQUIRE(aligned(gate_up, 16) && aligned(out, 16), ANEMLL_EINVAL, "silu_mul: tensors must be 16-byte aligned");
  if (rows == 0) return ANEMLL_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const long long n = rows * (ffn / 8);
  ANEMLL_REQUIRE((n + NT - 1) / NT < (1LL << 31), ANEMLL_EINVAL, "silu_mul: too many rows");
  return ANEMLL_DISPATCH_DTYPE(dtype, T, [&] {
    silu_mul_kernel<T><<<(unsigned)((n + NT - 1) / NT), NT, 0, st>>>((const T*)gate_up, (T*)out, rows, ffn);
    return launch_status("silu_mul");
  });
}

extern "C" int anemll_qk_norm_rope(const void* q_gate, int64_t qg_row_stride, const void* k, int64_t k_row_stride,
                                   const void* v, int64_t v_row_stride, const float* q_norm, const float* k_norm,
                                   const float* cos_table, const float* sin_table, void* q_out, void* k_out,
                                   void* v_out, void* gate_out, int dtype, int B, int T, int H_q, int H_kv,
                                   int head_dim, int pos, float eps, void* stream) {
  ANEMLL_REQUIRE(q_gate && k && v && q_norm && k_norm && cos_table && sin_table && q_out && k_out && v_out && gate_out,
                 ANEMLL_EINVAL, "qk_norm_rope: null pointer");
  ANEMLL_REQUIRE(B > 0 && T > 0 && H_q > 0 && H_kv > 0 && pos >= 0, ANEMLL_EINVAL, "qk_norm_rope: bad sizes");
  ANEMLL_REQUIRE(head_dim == 128 || head_dim == 256, ANEMLL_EUNSUPPORTED,
                 "qk_norm_rope: head_dim must be 128 or 256 (got %d)", head_dim);
  ANEMLL_REQUIRE(qg_row_stride >= 2LL * H_q * head_dim && k_row_stride >= (long long)H_kv * head_dim &&
                     v_row_stride >= (long long)H_kv * head_dim,
                 ANEMLL_EINVAL, "qk_norm_rope: row strides too small");
  ANEMLL_REQUIRE(dtype == ANEMLL_F16 || dtype == ANEMLL_BF16, ANEMLL_EUNSUPPORTED, "qk_norm_rope: fp16 or bf16 only");
  ANEMLL_REQUIRE(aligned(q_gate, 16) && aligned(k, 16) && aligned(v, 16) && aligned(q_out, 16) && aligned(k_out, 16) &&
                     aligned(v_out, 16) && aligned(gate_out, 16) && qg_row_stride % 8 == 0 && k_row_stride % 8 == 0 &&
                     v_row_stride % 8 == 0,
                 ANEMLL_EINVAL, "qk_norm_rope: tensors and row strides must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  return ANEMLL_DISPATCH_HALF(dtype, T_, [&] {
    const unsigned grid = (unsigned)((long long)B * T);
    if (head_dim == 256)
      qk_norm_rope_kernel<T_, 8><<<grid, NT, 0, st>>>(
          (const T_*)q_gate, qg_row_stride, (const T_*)k, k_row_stride, (const T_*)v, v_row_stride, q_norm, k_norm,
          cos_table, sin_table, (T_*)q_out, (T_*)k_out, (T_*)v_out, (T_*)gate_out, T, H_q, H_kv, pos, eps);
    else
      qk_norm_rope_kernel<T_, 4><<<grid, NT, 0, st>>>(
          (const T_*)q_gate, qg_row_stride, (const T_*)k, k_row_stride, (const T_*)v, v_row_stride, q_norm, k_norm,
          cos_table, sin_table, (T_*)q_out, (T_*)k_out, (T_*)v_out, (T_*)gate_out, T, H_q, H_kv, pos, eps);
    return launch_status("qk_norm_rope");
  });
}
