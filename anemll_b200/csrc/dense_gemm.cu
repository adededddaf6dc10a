// Y[M][N] = X[M][K] . W[N][K]^T for few rows (the decode steps' projections: M = the batch), bf16 or
// fp16 operands, fp32 accumulation, output in the operand type.
//
// At M <= 128 these GEMMs are weight-streaming: every weight byte is read once and used M times.
// One CTA computes a 128 x 128 output tile (UMMA M = 128 rows of X, N = 128 rows of W) over a slice
// of K; the K slices of one tile are a thread-block cluster of S CTAs (S = 1, 2, 4, 8), chosen so
// that narrow outputs (N = 2048, K up to 6144) still occupy the whole GPU in one wave.  The launch
// allows programmatic dependent launch: a CTA initialises its barriers, TMEM and tensor maps while
// the previous kernel drains, and waits for it only before the first load.  Per CTA:
//   * one thread streams 64-element K chunks of X and W into a 6-stage ring with TMA (128-byte
//     swizzle); one thread of another warp issues 4 tcgen05.mma (K = 16 each) per chunk into a TMEM
//     accumulator (128 lanes x 128 fp32 columns) and frees each slot with tcgen05.commit;
//   * S == 1: the four warps read the accumulator (a row per thread) and store it;
//   * S > 1: CTA rank r owns rows [r 128/S, (r+1) 128/S) of the tile; every CTA pushes its fp32
//     partial rows from registers into the owners' shared memory (distributed shared memory stores),
//     and each owner sums the S partials in rank order (deterministic) and stores its rows.
// Waits on mbarriers are bounded; a CTA that gives up records an error and still takes part in both
// cluster barriers, so no CTA of the cluster waits forever.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace anemll {
namespace {

namespace cg = cooperative_groups;

constexpr int BM = 128, BN = 128, BK = 64;       // BK elements = one 128-byte swizzle row
constexpr int STAGES = 6;                        // 192 KB in flight: one CTA per SM
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // 32 KB
constexpr int PLD = BN + 4;                      // fp32 partial tile row stride (bank spread)
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
static_assert(BM * PLD * 4 <= STAGES * STAGE_BYTES, "the received partial rows reuse the stage ring");

__device__ int g_gemm_error = 0;

template <typename T>
__global__ void __launch_bounds__(128)
dense_gemm_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mw, T* __restrict__ y,
                  int M, int N, int ldy, int total_chunks, int chunks_per_split) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[STAGES], empty[STAGES], done;
  __shared__ uint32_t tmem_slot;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * BN, split = blockIdx.y, S = gridDim.y, m0 = blockIdx.z * BM;
  const int c0 = split * chunks_per_split, c1 = min(total_chunks, c0 + chunks_per_split);
  const int nk = max(0, c1 - c0);
  const uint32_t sbase = tc::smem_u32(sm);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(&done, 1);
    tc::fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&mx) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&mw) : "memory");
  }
  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, BN);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_slot;

  // warp 0 lane 0 streams the chunks, warp 1 lane 0 issues the MMAs; their other lanes wait at the
  // warp barrier (parked, not polling), the other warps at the CTA barrier below
  __shared__ int issued, consumed;
  bool ok = true;
  if (warp == 0) {
    if (lane == 0) {
      griddep_wait();  // the previous kernel's outputs (X) are complete
      int j = 0;
      for (; j < nk; ++j) {
        const int s = j % STAGES;
        if (j >= STAGES) {  // the slot's previous chunk has been read by its MMAs
          ok = tc::mbar_wait(tc::smem_u32(&empty[s]), (uint32_t)((j / STAGES - 1) & 1));
          if (!ok) break;
        }
        const uint32_t bar = tc::smem_u32(&full[s]);
        const uint32_t a = sbase + s * STAGE_BYTES;
        tc::mbar_arrive_expect_tx(bar, STAGE_BYTES);
        tc::tma_load_2d(a, &mx, (c0 + j) * BK, m0, bar);
        tc::tma_load_2d(a + A_BYTES, &mw, (c0 + j) * BK, n0, bar);
      }
      issued = j;
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id = tc::idesc_f16(BM, BN, false, false, false, std::is_same<T, __nv_bfloat16>::value);
      int j = 0;
      for (; j < nk; ++j) {
        const int s = j % STAGES;
        ok = tc::mbar_wait(tc::smem_u32(&full[s]), (uint32_t)((j / STAGES) & 1));
        if (!ok) break;
        tc::fence_after();
        const uint32_t a = sbase + s * STAGE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc::mma_f16(tmem, tc::sdesc_sw128(a + kk * 32, 16, 1024), tc::sdesc_sw128(a + A_BYTES + kk * 32, 16, 1024),
                      id, (j > 0 || kk > 0) ? 1u : 0u);
        tc::commit(tc::smem_u32(&empty[s]));  // the slot is free once these MMAs have read it
      }
      consumed = j;
      if (nk > 0) tc::commit(tc::smem_u32(&done));  // arrives when every MMA issued above has completed
    }
    __syncwarp();
  }
  const bool loops_ok = __syncthreads_and(ok ? 1 : 0);
  griddep_launch_dependents();
  if (!loops_ok && tid == 0) {
    atomicExch(&g_gemm_error, 1);
    // wait (bounded) for loads still in flight before the ring is reused
    for (int j = consumed; j < issued; ++j)
      tc::mbar_wait(tc::smem_u32(&full[j % STAGES]), (uint32_t)((j / STAGES) & 1), 1u << 16);
  }
  // the accumulator is complete (bounded); the outcome is made CTA-uniform, since the TMEM reads
  // below are warp-collective
  bool mine = true;
  if (nk > 0 && !tc::mbar_wait(tc::smem_u32(&done), 0)) {
    atomicExch(&g_gemm_error, 1);
    mine = false;
  }
  const bool have = nk > 0 && __syncthreads_and(loops_ok && mine);
  tc::fence_after();
  griddep_wait();  // (a K slice with no chunks writes too: never before the previous kernel is done)

  const int row = warp * 32 + lane;  // TMEM lane = output row within the tile
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
  if (S == 1) {
    const int gr = m0 + row;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      if (have) {
        tc::tmem_ld32(taddr + c * 32, v);
        tc::tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
      }
      if (gr < M) {
        T* dst = y + (long long)gr * ldy + n0 + c * 32;
        const int ncols = min(32, N - (n0 + c * 32));
        if (ncols == 32) {
#pragma unroll
          for (int q = 0; q < 4; ++q) store8(dst + q * 8, v + q * 8);
        } else {
          for (int e = 0; e < ncols; ++e) dst[e] = from_f32<T>(v[e]);
        }
      }
    }
  } else {
    // split-K: CTA rank q owns output rows [q R, (q+1) R), R = 128 / S.  Every CTA pushes each of its
    // partial rows from registers straight into the owner's receive buffer (remote shared-memory
    // stores, slab = the sender's rank), then each owner sums its S slabs in rank order.
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every CTA's ring is free (its MMAs have completed): it may receive
    const int rank = (int)cluster.block_rank();
    const int R = BM / S;
    float* recv = reinterpret_cast<float*>(sm);  // [S][R][PLD]
    float* dst_buf = cluster.map_shared_rank(recv, row / R) + ((size_t)rank * R + row % R) * PLD;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      if (have) {
        tc::tmem_ld32(taddr + c * 32, v);
        tc::tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(dst_buf + c * 32 + q * 4) = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2],
                                                                           v[q * 4 + 3]);
    }
    cluster.sync();  // every slab has arrived; no remote access follows
    for (int i = tid; i < R * (BN / 4); i += 128) {
      const int r = i / (BN / 4), col = (i % (BN / 4)) * 4;
      float4 acc = *reinterpret_cast<const float4*>(recv + (size_t)r * PLD + col);
#pragma unroll 7
      for (int q = 1; q < S; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(recv + ((size_t)q * R + r) * PLD + col);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      const int gr = m0 + rank * R + r, gc = n0 + col;
      if (gr < M && gc < N) {
        T* dst = y + (long long)gr * ldy + gc;
        const float o4[4] = {acc.x, acc.y, acc.z, acc.w};
        if (gc + 4 <= N) {
          T h4[4] = {from_f32<T>(o4[0]), from_f32<T>(o4[1]), from_f32<T>(o4[2]), from_f32<T>(o4[3])};
          *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(h4);
        } else {
          for (int e = 0; e < N - gc; ++e) dst[e] = from_f32<T>(o4[e]);
        }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, BN);
}

PFN_cuTensorMapEncodeTiled_v12000 gemm_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// [rows][K] row-major operand, row stride ld elements: 64-element x 128-row boxes, 128-byte swizzle;
// rows past `rows` and columns past K read as zeros
int gemm_map(CUtensorMap* m, const void* base, long long rows, long long K, long long ld) {
  auto enc = gemm_map_encoder();
  ANEMLL_REQUIRE(enc, ANEMLL_EUNSUPPORTED, "gemm: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {BK, 128};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  ANEMLL_REQUIRE(r == CUDA_SUCCESS, ANEMLL_EINVAL, "gemm: tensor map encoding failed (%d)", (int)r);
  return ANEMLL_OK;
}

template <typename T>
int launch_gemm(const void* x, long long ldx, const void* w, long long ldw, void* y, long long ldy, int M, int N,
                int K, cudaStream_t st) {
  CUtensorMap mx, mw;
  int rc = gemm_map(&mx, x, M, K, ldx);
  if (!rc) rc = gemm_map(&mw, w, N, K, ldw);
  if (rc) return rc;
  const int n_tiles = (N + BN - 1) / BN, m_tiles = (M + BM - 1) / BM;
  const int total_chunks = (K + BK - 1) / BK;
  // K splits: one wave of one CTA per SM, at least 4 chunks per split
  int S = 1;
  while (S < 8 && (long long)n_tiles * m_tiles * S * 2 <= 148 && total_chunks >= 4 * S * 2) S *= 2;
  const int per = (total_chunks + S - 1) / S;
  auto kern = dense_gemm_kernel<T>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_tiles, S, m_tiles);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = S;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mx, mw, (T*)y, M, N, (int)ldy, total_chunks, per);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("gemm: launch failed, CUDA error %d (%s)", (int)e, cudaGetErrorString(e));
    return (int)e;
  }
  return launch_status("gemm");
}

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M, int N,
                           int K, int dtype, void* stream) {
  ANEMLL_REQUIRE(x && w && y, ANEMLL_EINVAL, "gemm: null pointer");
  ANEMLL_REQUIRE(M > 0 && N > 0 && K > 0, ANEMLL_EINVAL, "gemm: bad sizes");
  ANEMLL_REQUIRE(dtype == ANEMLL_F16 || dtype == ANEMLL_BF16, ANEMLL_EUNSUPPORTED, "gemm: fp16 or bf16 only");
  ANEMLL_REQUIRE(ldx >= K && ldw >= K && ldy >= N, ANEMLL_EINVAL, "gemm: leading dimensions shorter than the rows");
  ANEMLL_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(y, 16) && ldx % 8 == 0 && ldw % 8 == 0 && ldy % 8 == 0,
                 ANEMLL_EINVAL, "gemm: operands 16-byte aligned with rows whole 16-byte units");
  ANEMLL_REQUIRE((long long)((M + BM - 1) / BM) < 65536, ANEMLL_EINVAL, "gemm: too many rows");
  cudaStream_t st = (cudaStream_t)stream;
  return ANEMLL_DISPATCH_HALF(dtype, T, [&] { return launch_gemm<T>(x, ldx, w, ldw, y, ldy, M, N, K, st); });
}

extern "C" int anemll_gemm_error(int reset) {
  int h = 0;
  cudaMemcpyFromSymbol(&h, g_gemm_error, sizeof(int));
  if (reset && h) {
    const int z = 0;
    cudaMemcpyToSymbol(g_gemm_error, &z, sizeof(int));
  }
  return h;
}
