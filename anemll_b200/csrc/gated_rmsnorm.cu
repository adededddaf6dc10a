// Gated RMSNorm over rows: out = weight * x * rsqrt(mean(x^2) + eps) * silu(z).
// Semantics of Qwen3_5RMSNormGated (transformers 5.5.0, modeling_qwen3_5.py:175-190), evaluated in
// fp32.  Rows of up to 512 elements (d_v = 128 in every Qwen3.5 size): a half-warp per row, 8
// elements per lane as 16-byte vectors, every load issued before the first use.  Longer rows: a
// warp per row, element by element.
#include "common.cuh"

namespace anemll {
namespace {

// z row r: dense (zh == 0), or head r % zh of token r / zh with token rows z_ld elements apart
__device__ __forceinline__ int64_t z_offset(int64_t r, int d, int64_t zh, int64_t z_ld) {
  return zh ? (r / zh) * z_ld + (r % zh) * d : r * d;
}

template <typename TX, typename TZ, typename TO>
__global__ void __launch_bounds__(256)
gated_rmsnorm_kernel(const TX* __restrict__ x, const TZ* __restrict__ z, const float* __restrict__ w,
                     TO* __restrict__ out, int64_t rows, int d, float eps, int64_t zh, int64_t z_ld) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const TX* xr = x + row * d;
  const TZ* zr = z + z_offset(row, d, zh, z_ld);
  float ss = 0.f;
  for (int i = lane; i < d; i += 32) {
    const float xv = to_f32(xr[i]);
    ss += xv * xv;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)d + eps);
  TO* orow = out + row * d;
  for (int i = lane; i < d; i += 32) {
    orow[i] = from_f32<TO>(w[i] * to_f32(xr[i]) * r * silu(to_f32(zr[i])));
  }
}

// rows of d <= 16 * 8 * NC elements, d % 8 == 0; 16 rows per 256-thread CTA
template <typename TX, typename TZ, typename TO, int NC>
__global__ void __launch_bounds__(256)
gated_rmsnorm_vec_kernel(const TX* __restrict__ x, const TZ* __restrict__ z, const float* __restrict__ w,
                         TO* __restrict__ out, int64_t rows, int d, float eps, int64_t zh, int64_t z_ld) {
  const int64_t row = (int64_t)blockIdx.x * 16 + (threadIdx.x >> 4);
  const int l = threadIdx.x & 15;
  const unsigned hmask = 0xffffu << (threadIdx.x & 16);
  if (row >= rows) return;  // whole half-warps leave together
  float xv[NC][8], zv[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 16 + l) * 8;
    if (col < d) {
      load8(x + row * d + col, xv[c]);
      load8(z + z_offset(row, d, zh, z_ld) + col, zv[c]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 16 + l) * 8;
    if (col < d) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += xv[c][e] * xv[c][e];
    }
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(hmask, ss, off);
  const float r = rsqrtf(ss / (float)d + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 16 + l) * 8;
    if (col < d) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        o[e] = w[col + e] * xv[c][e] * r * __fdividef(zv[c][e], 1.0f + __expf(-zv[c][e]));  // silu(z)
      store8(out + row * d + col, o);
    }
  }
}

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_gated_rmsnorm(const void* x, int x_dtype, const void* z, int z_dtype,
                                    const float* weight, void* out, int out_dtype,
                                    int64_t rows, int d, float eps, int64_t z_heads, int64_t z_row_stride,
                                    void* stream) {
  ANEMLL_REQUIRE(x && z && weight && out, ANEMLL_EINVAL, "gated_rmsnorm: null pointer");
  ANEMLL_REQUIRE(rows >= 0 && d > 0, ANEMLL_EINVAL, "gated_rmsnorm: bad sizes");
  ANEMLL_REQUIRE(z_heads >= 0 && (z_heads == 0 || z_row_stride >= z_heads * d), ANEMLL_EINVAL,
                 "gated_rmsnorm: z row stride shorter than z_heads * d");
  ANEMLL_REQUIRE(dtype_ok(x_dtype) && dtype_ok(z_dtype) && dtype_ok(out_dtype), ANEMLL_EUNSUPPORTED,
                 "gated_rmsnorm: bad dtype");
  if (rows == 0) return ANEMLL_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  const bool z_vec_ok = z_heads == 0 || (z_row_stride * dtype_size(z_dtype)) % 16 == 0;
  return ANEMLL_DISPATCH_DTYPE(x_dtype, TX, [&] {
    return ANEMLL_DISPATCH_DTYPE(z_dtype, TZ, [&] {
      return ANEMLL_DISPATCH_DTYPE(out_dtype, TO, [&] {
        const bool vec = d % 8 == 0 && d <= 512 && aligned(x, 16) && aligned(z, 16) && aligned(out, 16) && z_vec_ok;
        const unsigned vblocks = (unsigned)((rows + 15) / 16);
        if (vec && d <= 128)
          gated_rmsnorm_vec_kernel<TX, TZ, TO, 1><<<vblocks, 256, 0, st>>>((const TX*)x, (const TZ*)z, weight,
                                                                          (TO*)out, rows, d, eps, z_heads,
                                                                          z_row_stride);
        else if (vec)
          gated_rmsnorm_vec_kernel<TX, TZ, TO, 4><<<vblocks, 256, 0, st>>>((const TX*)x, (const TZ*)z, weight,
                                                                          (TO*)out, rows, d, eps, z_heads,
                                                                          z_row_stride);
        else
          gated_rmsnorm_kernel<TX, TZ, TO><<<blocks, 256, 0, st>>>((const TX*)x, (const TZ*)z, weight, (TO*)out,
                                                                   rows, d, eps, z_heads, z_row_stride);
        return launch_status("gated_rmsnorm");
      });
    });
  });
}
