// Shared helpers for the anemll_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/anemll_b200.h"

namespace anemll {

// ---------------------------------------------------------------- errors ----
void set_error(const char* fmt, ...);

#define ANEMLL_REQUIRE(cond, code, ...)      \
  do {                                       \
    if (!(cond)) {                           \
      ::anemll::set_error(__VA_ARGS__);      \
      return (code);                         \
    }                                        \
  } while (0)

// Map a launch/runtime error to the positive status range (success: counts one kernel launch).
int launch_status(const char* what);

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int dtype_size(int dt) { return dt == ANEMLL_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == ANEMLL_F32 || dt == ANEMLL_F16 || dt == ANEMLL_BF16; }

// ------------------------------------------------------------ conversions --
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// ------------------------------------------------------------ reductions ---
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }
// 1 / (1 + e^-x) with the fast exponential and reciprocal (a few ulp; the IEEE division is a long
// instruction sequence, and gates are applied to every output element)
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// 2^x with the hardware approximation instruction (PTX ex2.approx.ftz.f32;
// relative error about 2^-22, -inf -> 0): the softmax exponent.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Programmatic dependent launch (PTX griddepcontrol): a kernel launched with programmatic stream
// serialisation may start while the previous kernel of the stream is still running; it must call
// griddep_wait() before it reads or writes global memory (the wait returns once the previous grid has
// completed and its writes are visible; without that launch attribute it returns at once).
// griddep_launch_dependents() lets the next such kernel start launching early.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ float softplus(float x) {
  // log(1 + e^x), evaluated without overflow (same threshold behaviour as torch's softplus, beta=1, threshold=20)
  return x > 20.0f ? x : log1pf(__expf(x));
}

// 8 consecutive elements <-> fp32, as one 16-byte (2-byte types) or two 16-byte (fp32) accesses
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* f) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = to_f32(h[e]);
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float* f) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    uint4 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(f[e]);
    *reinterpret_cast<uint4*>(p) = u;
  }
}


// ---- per-head RMSNorm + rotary embedding (QwenHeadNorm then apply_rotary_pos_emb) ----
// x = T(x * rsqrt(mean(x^2) + eps) * w) (fp32, one rounding to the storage type), then
// y = x cos + rotate_half(x) sin with the products and the sum rounded separately in fp32.  The sum
// of squares is a fixed tree: 32 partial sums of EPL consecutive squares (one per lane of a warp
// that holds the row, lane l owning [l EPL, (l+1) EPL)), combined like warp_sum.  Every caller
// (a warp per row, or one thread per row) follows it, so all produce the same bits.
template <typename T>
__device__ __forceinline__ float head_norm_round(float x, float rn, float w) {
  return to_f32(from_f32<T>(__fmul_rn(__fmul_rn(x, rn), w)));
}
__device__ __forceinline__ float rope_one(float x, float partner_rot, float c, float s) {
  return __fadd_rn(__fmul_rn(x, c), __fmul_rn(partner_rot, s));
}

// A warp holds the row: lane l has x[0..EPL) = elements [l EPL, (l+1) EPL); the rotation partner of
// element i (i +- HD/2) sits in lane l ^ 16.  w, cr, sr point at element 0 of the weight and of this
// position's cos/sin rows.
template <typename T, int EPL>
__device__ __forceinline__ void head_norm_rope_warp(float* x, const float* w, const float* cr, const float* sr,
                                                    float eps, int lane) {
  constexpr int HD = EPL * 32;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) ss += x[e] * x[e];
  ss = warp_sum(ss);
  const float rn = rsqrtf(ss / (float)HD + eps);
#pragma unroll
  for (int e = 0; e < EPL; ++e) x[e] = head_norm_round<T>(x[e], rn, w[lane * EPL + e]);
  const bool lower = lane < 16;  // first half: rotate_half gives -x[i + HD/2]
  float y[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
    y[e] = rope_one(x[e], lower ? -partner : partner, cr[lane * EPL + e], sr[lane * EPL + e]);
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) x[e] = y[e];
}

// The same result from one thread: rsqrt(mean(x^2) + eps) of a row given its 32 partial sums
// (partial l = the sum of squares of elements [l EPL, (l+1) EPL), accumulated in order).
__device__ __forceinline__ float head_norm_scale(float* part, int HD, float eps) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < o; ++i) part[i] = part[i] + part[i + o];
  return rsqrtf(part[0] / (float)HD + eps);
}
}  // namespace anemll

// Dispatch an element type code to a C++ type alias `T`.
#define ANEMLL_DISPATCH_DTYPE(code, T, ...)                     \
  [&]() -> int {                                                \
    switch (code) {                                             \
      case ANEMLL_F32: { using T = float; return __VA_ARGS__(); }          \
      case ANEMLL_F16: { using T = __half; return __VA_ARGS__(); }         \
      case ANEMLL_BF16: { using T = __nv_bfloat16; return __VA_ARGS__(); } \
      default:                                                  \
        ::anemll::set_error("unsupported dtype code %d", (int)(code)); \
        return ANEMLL_EUNSUPPORTED;                             \
    }                                                           \
  }()

#define ANEMLL_DISPATCH_HALF(code, T, ...)                      \
  [&]() -> int {                                                \
    switch (code) {                                             \
      case ANEMLL_F16: { using T = __half; return __VA_ARGS__(); }         \
      case ANEMLL_BF16: { using T = __nv_bfloat16; return __VA_ARGS__(); } \
      default:                                                  \
        ::anemll::set_error("dtype code %d unsupported here (f16/bf16 only)", (int)(code)); \
        return ANEMLL_EUNSUPPORTED;                             \
    }                                                           \
  }()
