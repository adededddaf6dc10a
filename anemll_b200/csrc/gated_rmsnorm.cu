// Gated RMSNorm over rows: out = weight * x * rsqrt(mean(x^2) + eps) * silu(z).
// One warp per row; semantics of Qwen3_5RMSNormGated (transformers 5.5.0,
// modeling_qwen3_5.py:175-190), evaluated in fp32.
#include "common.cuh"

namespace anemll {
namespace {

template <typename TX, typename TZ, typename TO>
__global__ void __launch_bounds__(256)
gated_rmsnorm_kernel(const TX* __restrict__ x, const TZ* __restrict__ z, const float* __restrict__ w,
                     TO* __restrict__ out, int64_t rows, int d, float eps) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const TX* xr = x + row * d;
  const TZ* zr = z + row * d;
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

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_gated_rmsnorm(const void* x, int x_dtype, const void* z, int z_dtype,
                                    const float* weight, void* out, int out_dtype,
                                    int64_t rows, int d, float eps, void* stream) {
  ANEMLL_REQUIRE(x && z && weight && out, ANEMLL_EINVAL, "gated_rmsnorm: null pointer");
  ANEMLL_REQUIRE(rows >= 0 && d > 0, ANEMLL_EINVAL, "gated_rmsnorm: bad sizes");
  if (rows == 0) return ANEMLL_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  return ANEMLL_DISPATCH_DTYPE(x_dtype, TX, [&] {
    return ANEMLL_DISPATCH_DTYPE(z_dtype, TZ, [&] {
      return ANEMLL_DISPATCH_DTYPE(out_dtype, TO, [&] {
        gated_rmsnorm_kernel<TX, TZ, TO><<<blocks, 256, 0, st>>>((const TX*)x, (const TZ*)z, weight, (TO*)out,
                                                                 rows, d, eps);
        return launch_status("gated_rmsnorm");
      });
    });
  });
}
