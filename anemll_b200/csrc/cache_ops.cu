// Cache-management ops on the device: the reference's one-hot update-mask writes, the rotating
// sliding-window update of its split local cache, and KV-state transition / compaction between
// context sizes.  All three are HBM-bound copies: 16-byte vectors, coalesced rows, one pass.
//
// Reference semantics: anemll/models/gemma3_model.py _apply_update_mask / _apply_update_mask_batch
// (932-965), _update_kv_local (1024-1066), _update_kv_local_prefill (1167-1204);
// anemll/utils/state_transition.py transition_kv_state (62-152), compact_kv_state (153-357).
#include "common.cuh"

namespace anemll {
namespace {

__device__ __forceinline__ float mask_at(const void* m, int mdt, long long i) {
  return mdt == ANEMLL_F32 ? reinterpret_cast<const float*>(m)[i]
       : mdt == ANEMLL_F16 ? __half2float(reinterpret_cast<const __half*>(m)[i])
                           : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(m)[i]);
}

// One warp per (row l, slab).  The lanes read the mask row together; a row the mask leaves untouched
// (all weights zero) is left alone, with no cache traffic.  For a touched row the lanes rewrite the
// slab's d elements in 8-element groups: cache = cache (1 - min(sum_s m, 1)) + sum_s new_s m_s (fp32);
// a ballot walks only the columns s with a non-zero weight.
template <typename T>
__global__ void update_mask_kernel(T* __restrict__ cache, const T* __restrict__ nw, const void* __restrict__ mask,
                                   int mdt, long long mld, long long n_slabs, int L, int S, int d, long long cs,
                                   long long ns) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  if (warp_id >= (long long)L * n_slabs) return;  // warp-uniform
  const int l = (int)(warp_id % L);
  const long long slab = warp_id / L;
  const void* mrow = mask;
  float msum = 0.f;
  bool touched = false;
  for (int s = lane; s < S; s += 32) {
    const float m = mask_at(mrow, mdt, (long long)l * mld + s);
    msum += m;
    touched |= m != 0.f;
  }
  if (!__any_sync(0xffffffffu, touched)) return;  // warp-uniform
  msum = warp_sum(msum);
  const float keep = 1.f - fminf(msum, 1.f);
  const int groups = d / 8;
  for (int gbase = 0; gbase < groups; gbase += 32) {  // warp-uniform loop
    const int gi = gbase + lane;
    const bool act = gi < groups;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < S; s0 += 32) {  // warp-uniform loop
      const int sl = s0 + lane;
      unsigned nz = __ballot_sync(0xffffffffu, sl < S && mask_at(mrow, mdt, (long long)l * mld + sl) != 0.f);
      while (nz) {
        const int s = s0 + __ffs(nz) - 1;
        nz &= nz - 1;
        if (act) {
          const float w = mask_at(mrow, mdt, (long long)l * mld + s);
          float x[8];
          load8(nw + slab * ns + (long long)s * d + gi * 8, x);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += x[e] * w;
        }
      }
    }
    if (act) {
      T* dst = cache + slab * cs + (long long)l * d + gi * 8;
      float c[8];
      load8(dst, c);
#pragma unroll
      for (int e = 0; e < 8; ++e) c[e] = c[e] * keep + acc[e];
      store8(dst, c);
    }
  }
}

// One CTA per (slab, 32-byte column strip): the strip's L rows are staged in shared memory before any
// is rewritten, so the in-place shift never reads a row it has already overwritten; 32-byte rows of
// the strip are whole DRAM sectors.
constexpr int ROT_W = 32;
__global__ void rotate_append_kernel(uint8_t* __restrict__ cache, const uint8_t* __restrict__ nw, int L, int n,
                                     int row_bytes, long long cs_bytes, long long ns_bytes) {
  extern __shared__ __align__(16) uint8_t strip[];
  const long long slab = blockIdx.y;
  const int col0 = blockIdx.x * ROT_W;
  const int chunks = min(ROT_W, row_bytes - col0) / 16;  // 16-byte chunks of this strip (1 or 2)
  uint8_t* base = cache + slab * cs_bytes + col0;
  const uint8_t* nbase = nw + slab * ns_bytes + col0;
  for (int i = threadIdx.x; i < L * chunks; i += blockDim.x) {
    const int r = i / chunks, c = i % chunks;
    const uint8_t* src =
        r < L - n ? base + (long long)(r + n) * row_bytes : nbase + (long long)(r - (L - n)) * row_bytes;
    *reinterpret_cast<uint4*>(strip + r * ROT_W + c * 16) = *reinterpret_cast<const uint4*>(src + c * 16);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < L * chunks; i += blockDim.x) {
    const int r = i / chunks, c = i % chunks;
    *reinterpret_cast<uint4*>(base + (long long)r * row_bytes + c * 16) =
        *reinterpret_cast<const uint4*>(strip + r * ROT_W + c * 16);
  }
}

// One thread per 8 consecutive destination elements (16- or 32-byte accesses).
template <typename TS, typename TD>
__global__ void transition_kernel(const TS* __restrict__ src, TD* __restrict__ dst, long long n_slabs, int src_len,
                                  int dst_len, int d, int pos, float pad) {
  const int groups = d / 8;
  const long long total = n_slabs * dst_len * groups;
  const float padv = to_f32(from_f32<TD>(pad));
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int gi = (int)(t % groups);
    const int r = (int)((t / groups) % dst_len);
    const long long slab = t / ((long long)groups * dst_len);
    float v[8];
    if (r < pos) {
      load8(src + (slab * src_len + r) * d + gi * 8, v);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = padv;
    }
    store8(dst + (slab * dst_len + r) * d + gi * 8, v);
  }
}

int grid_for(long long work, int block) {
  const long long b = (work + block - 1) / block;
  return (int)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

constexpr int ROTATE_MAX_STRIP = 200 * 1024;

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_kv_update_mask(void* cache, const void* new_rows, int dtype, const void* mask, int mask_dtype,
                                     int64_t mask_row_stride, int64_t n_slabs, int L, int S, int d,
                                     int64_t cache_slab_stride, int64_t new_slab_stride, void* stream) {
  ANEMLL_REQUIRE(cache && new_rows && mask, ANEMLL_EINVAL, "kv_update_mask: null pointer");
  ANEMLL_REQUIRE(n_slabs > 0 && L > 0 && S > 0 && d > 0 && mask_row_stride >= S, ANEMLL_EINVAL,
                 "kv_update_mask: bad sizes");
  ANEMLL_REQUIRE(d % 8 == 0, ANEMLL_EUNSUPPORTED, "kv_update_mask: d must be a multiple of 8 (got %d)", d);
  ANEMLL_REQUIRE(dtype_ok(mask_dtype), ANEMLL_EUNSUPPORTED, "kv_update_mask: bad mask dtype");
  ANEMLL_REQUIRE(cache_slab_stride >= (int64_t)L * d && new_slab_stride >= (int64_t)S * d, ANEMLL_EINVAL,
                 "kv_update_mask: slab strides smaller than a slab");
  cudaStream_t st = (cudaStream_t)stream;
  ANEMLL_REQUIRE(aligned(cache, 16) && aligned(new_rows, 16) && (cache_slab_stride * dtype_size(dtype)) % 16 == 0 &&
                     (new_slab_stride * dtype_size(dtype)) % 16 == 0,
                 ANEMLL_EALIGN, "kv_update_mask: cache / new rows and their slab strides must be 16-byte aligned");
  ANEMLL_REQUIRE((int64_t)L * n_slabs <= ((int64_t)1 << 36), ANEMLL_EINVAL, "kv_update_mask: too many rows");
  return ANEMLL_DISPATCH_DTYPE(dtype, T, [&] {
    const long long warps = n_slabs * L;  // one warp per (row, slab)
    const long long blocks = (warps * 32 + 255) / 256;
    update_mask_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<T*>(cache),
                                                            reinterpret_cast<const T*>(new_rows), mask, mask_dtype,
                                                            mask_row_stride, n_slabs, L, S, d, cache_slab_stride,
                                                            new_slab_stride);
    return launch_status("kv_update_mask");
  });
}

extern "C" int anemll_kv_rotate_append(void* cache, const void* new_rows, int dtype, int64_t n_slabs, int L, int n,
                                       int d, int64_t cache_slab_stride, int64_t new_slab_stride, void* stream) {
  ANEMLL_REQUIRE(cache && new_rows, ANEMLL_EINVAL, "kv_rotate_append: null pointer");
  ANEMLL_REQUIRE(dtype_ok(dtype), ANEMLL_EUNSUPPORTED, "kv_rotate_append: bad dtype");
  ANEMLL_REQUIRE(n_slabs > 0 && n_slabs <= 65535 && L > 0 && d > 0, ANEMLL_EINVAL, "kv_rotate_append: bad sizes");
  ANEMLL_REQUIRE(n > 0 && n <= L, ANEMLL_EINVAL, "kv_rotate_append: shift %d outside (0, %d]", n, L);
  const int es = dtype_size(dtype);
  const int row_bytes = d * es;
  ANEMLL_REQUIRE(row_bytes % 16 == 0, ANEMLL_EUNSUPPORTED, "kv_rotate_append: rows must be whole 16-byte units");
  ANEMLL_REQUIRE((cache_slab_stride * es) % 16 == 0 && (new_slab_stride * es) % 16 == 0 && aligned(cache, 16) &&
                     aligned(new_rows, 16),
                 ANEMLL_EALIGN, "kv_rotate_append: pointers and slab strides must be 16-byte aligned");
  ANEMLL_REQUIRE(cache_slab_stride >= (int64_t)L * d && new_slab_stride >= (int64_t)n * d, ANEMLL_EINVAL,
                 "kv_rotate_append: slab strides smaller than a slab");
  const size_t smem = (size_t)L * ROT_W;
  ANEMLL_REQUIRE(smem <= (size_t)ROTATE_MAX_STRIP, ANEMLL_EUNSUPPORTED,
                 "kv_rotate_append: window of %d rows exceeds the %d-row shared-memory strip", L,
                 ROTATE_MAX_STRIP / ROT_W);
  cudaFuncSetAttribute(rotate_append_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((row_bytes + ROT_W - 1) / ROT_W, (unsigned)n_slabs);
  rotate_append_kernel<<<grid, 256, smem, (cudaStream_t)stream>>>(
      reinterpret_cast<uint8_t*>(cache), reinterpret_cast<const uint8_t*>(new_rows), L, n, row_bytes,
      cache_slab_stride * es, new_slab_stride * es);
  return launch_status("kv_rotate_append");
}

extern "C" int anemll_kv_state_transition(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n_slabs,
                                          int src_len, int dst_len, int d, int current_position, float pad_value,
                                          void* stream) {
  ANEMLL_REQUIRE(src && dst, ANEMLL_EINVAL, "kv_state_transition: null pointer");
  ANEMLL_REQUIRE(n_slabs > 0 && src_len > 0 && dst_len > 0 && d > 0, ANEMLL_EINVAL, "kv_state_transition: bad sizes");
  ANEMLL_REQUIRE(current_position >= 0 && current_position <= src_len && current_position <= dst_len, ANEMLL_EINVAL,
                 "kv_state_transition: current_position %d outside [0, min(%d, %d)]", current_position, src_len,
                 dst_len);
  ANEMLL_REQUIRE(d % 8 == 0, ANEMLL_EUNSUPPORTED, "kv_state_transition: d must be a multiple of 8 (got %d)", d);
  ANEMLL_REQUIRE(aligned(src, 16) && aligned(dst, 16), ANEMLL_EALIGN, "kv_state_transition: 16-byte aligned pointers");
  cudaStream_t st = (cudaStream_t)stream;
  return ANEMLL_DISPATCH_DTYPE(src_dtype, TS, [&] {
    return ANEMLL_DISPATCH_DTYPE(dst_dtype, TD, [&] {
      const long long work = n_slabs * dst_len * (d / 8);
      transition_kernel<TS, TD><<<grid_for(work, 256), 256, 0, st>>>(
          reinterpret_cast<const TS*>(src), reinterpret_cast<TD*>(dst), n_slabs, src_len, dst_len, d,
          current_position, pad_value);
      return launch_status("kv_state_transition");
    });
  });
}
