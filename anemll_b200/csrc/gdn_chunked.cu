// Gated delta rule, chunked prefill on the 5th-generation tensor cores.
//
// One CTA owns one (sequence b, value head h) and walks its chunks of C = 64
// tokens in order; the fp32 state S [d_k=128, d_v=128] lives in tensor memory
// (TMEM) as S^T (lane = d_v index, column = d_k index) for the whole sequence
// and leaves the SM only after the last chunk.  With G the in-chunk cumulative
// log-decay and Gam[i,j] = exp(G_i - G_j), per chunk:
//
//   D1   = [Q;K] K^T                         (tcgen05, M=128 N=64 K=128)
//   P    = lower_incl(Q K^T * Gam)           (CUDA cores, fp16 to smem)
//   A    = strict_lower(diag(beta) K K^T * Gam), T = (I + A)^-1   (CUDA cores, fp32, blockwise)
//   U^T  = V^T (T diag(beta))^T              (tcgen05, M=128 N=64 K=64)
//   W^T  = K^T (T diag(beta e^G))^T          (tcgen05, M=128 N=64 K=64)
//   Vn^T = U^T - S^T W^T                     (tcgen05, A negated, accumulates on U)
//   O1^T = S^T Q^T,  O2^T = Vn^T P^T         (tcgen05; O = diag(e^G) O1 + O2 at readout)
//   S^T  = e^{G_c} S^T + (diag(e^{G_c - G}) Vn)^T K   (e^{G_c} applied in TMEM, then tcgen05)
//
// Every product is arranged so that M = 128 (d_v or d_k on TMEM lanes).  All
// operands are fp16 in 128-byte-swizzled shared memory; accumulators are fp32
// in TMEM.  fp16 (10-bit mantissa) operands keep the result within 1e-3
// relative L2 of an fp32 evaluation; bf16 inputs are converted to fp16 in
// place.  The attention scale multiplies O in fp32 at the end (O is linear in q).
//
// Occupancy: two CTAs per SM (128 threads, 256 TMEM columns and ~109 KB of
// shared memory each), so two heads' latency-bound phases interleave on the
// SM.  Shared memory is reused phase by phase (see the map below).  q/k/v
// tiles arrive by TMA (3-D tensor maps over [d, head, token], 64-token x
// 64-element boxes, 128-byte swizzle done by the copy engine); the next chunk's
// copies are issued as soon as the state update has released the tiles.
// T = (I + A)^-1 is built blockwise: four 16x16 diagonal blocks by forward
// substitution, then 16 -> 32 -> 64 merges T21 = -T22 (A21 T11) as small fp32
// matrix products over all threads.
//
// Semantics: torch_chunk_gated_delta_rule of transformers 5.5.0
// (modeling_qwen3_5.py:234-311); chunk (WY/UT) form of Yang et al. (2024).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "mma_sync.cuh"
#include "tcgen05.cuh"

namespace anemll {
namespace {

constexpr int C = 64;
constexpr int D = 128;
constexpr int NT = 128;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t COL_S = 0, COL_U = 128, COL_R = 192;  // U: U -> Vn -> O2;  R: D1 -> W -> O1

// shared memory map (bytes from a 1024-byte aligned base) and lifetimes within a chunk:
//   QK (TMA): rows 0-63 Q, 64-127 K                     [load .. S update]
//   V  (TMA) V -> W [tok][d_k] -> Vn^T [d_v][tok]      (W after U/W, Vn after V'/O1)
//   VD (dec Vn)^T                                       [Vn readout .. S update]
//   P                                                   [P/A .. O2]
//   X: A fp32 | T fp32 -> T1,T2 (over A) -> S^T fp16 (after U/W) -> O staging (after V'/O1)
constexpr int QK_BLK = 128 * 128;  // one 64-column block of a 128-row tile
constexpr int T64_BLK = 64 * 128;  // one 64-column block of a 64-row tile
constexpr int LDF = 68;            // fp32 row pitch (floats) of A and T
constexpr int OFF_QK = 0;
constexpr int OFF_V = OFF_QK + 2 * QK_BLK;
constexpr int OFF_VD = OFF_V + 2 * T64_BLK;
constexpr int OFF_P = OFF_VD + 2 * T64_BLK;
constexpr int OFF_X = OFF_P + T64_BLK;
constexpr int OFF_A = OFF_X, OFF_T = OFF_X + 64 * LDF * 4;
constexpr int OFF_T1 = OFF_X, OFF_T2 = OFF_X + T64_BLK;
constexpr int OFF_ST = OFF_X, OFF_OST = OFF_X;
constexpr int OFF_GB = OFF_X + 2 * 64 * LDF * 4;  // raw g[64], beta[64]
constexpr int OFF_MISC = OFF_GB + 128 * 4;        // G, beta, e^G, dec [64] each, gamma
constexpr int SMEM_BYTES = OFF_MISC + 4 * 64 * 4 + 16 + 1024;
constexpr uint32_t TILE_TX_BYTES = 2 * QK_BLK + 2 * T64_BLK;  // six 8 KB boxes per chunk
static_assert(OFF_X % 1024 == 0 && OFF_V % 1024 == 0, "tile alignment");
static_assert(2 * QK_BLK <= 2 * 64 * LDF * 4, "S^T must fit in the A|T region");
static_assert(SMEM_BYTES <= 113 * 1024, "two CTAs per SM");

struct TileMaps {
  CUtensorMap q, k, v;
};

__device__ int g_chunked_error = 0;

// byte offset of 16-byte chunk `ch` (0..7) of row `r` inside a 128-byte-row swizzled block
// (the TMA 128-byte swizzle: chunk index XOR row index mod 8, 1024-byte aligned blocks)
__device__ __forceinline__ uint32_t sw(int r, int ch) { return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4)); }
__device__ __forceinline__ uint32_t sw_elem(int r, int c) { return sw(r, c >> 3) + (uint32_t)((c & 7) << 1); }

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32(h[i]);
}

__device__ __forceinline__ uint4 pack8_f16(const float* f) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Rewrite the chunk's tiles in place as fp16: convert from TIn, l2-normalise q
// and k rows if asked, zero the rows at and past `nvalid`.
template <typename TIn>
__device__ __forceinline__ void convert_tiles(uint8_t* qk, uint8_t* vt, int nvalid, int l2norm, int tid) {
  const int ch = tid & 15;
  const int blk = ch >> 3, cb = ch & 7;
#pragma unroll 1
  for (int it = 0; it < 8; ++it) {
    const int r = (tid >> 4) + it * 8;
    uint4* pq = reinterpret_cast<uint4*>(qk + blk * QK_BLK + sw(r, cb));
    uint4* pk = reinterpret_cast<uint4*>(qk + blk * QK_BLK + sw(64 + r, cb));
    uint4* pv = reinterpret_cast<uint4*>(vt + blk * T64_BLK + sw(r, cb));
    float fq[8], fk[8], fv[8];
    if (r < nvalid) {
      unpack8<TIn>(*pq, fq);
      unpack8<TIn>(*pk, fk);
      unpack8<TIn>(*pv, fv);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) fq[i] = fk[i] = fv[i] = 0.f;
    }
    if (l2norm) {
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) { sq += fq[i] * fq[i]; sk += fk[i] * fk[i]; }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
      }
      const float rq = rsqrtf(sq + 1e-6f), rk = rsqrtf(sk + 1e-6f);
#pragma unroll
      for (int i = 0; i < 8; ++i) { fq[i] *= rq; fk[i] *= rk; }
    }
    *pq = pack8_f16(fq);
    *pk = pack8_f16(fk);
    *pv = pack8_f16(fv);
  }
}

template <typename TIn, typename TOut>
__global__ void __launch_bounds__(NT, 2)
gdn_chunked_kernel(const __grid_constant__ TileMaps maps, const float* __restrict__ g, const float* __restrict__ beta,
                   float* __restrict__ state, TOut* __restrict__ out, int T, int Hqk, int Hv, float scale,
                   int l2norm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sG = reinterpret_cast<float*>(sm + OFF_MISC);
  float* sBeta = sG + 64;
  float* sEG = sG + 128;
  float* sDec = sG + 192;
  float* sGamma = sG + 256;
  float* sA = reinterpret_cast<float*>(sm + OFF_A);
  float* sT = reinterpret_cast<float*>(sm + OFF_T);
  const float* sGB = reinterpret_cast<const float*>(sm + OFF_GB);
  __shared__ uint64_t mbar;  // tensor-core completions
  __shared__ uint64_t tbar;  // TMA arrivals
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;  // thread tid reads TMEM lane tid
  const int bh = blockIdx.x;
  const int b = bh / Hv, hv = bh % Hv;
  const int hk = hv / (Hv / Hqk);
  const uint32_t sbase = tc::smem_u32(sm);
  const uint32_t bar = tc::smem_u32(&mbar);
  const uint32_t tb = tc::smem_u32(&tbar);
  const int nchunks = (T + C - 1) / C;
  // fp16 inputs without l2-norm need no rewrite except for a ragged last chunk
  const bool always_convert = !std::is_same<TIn, __half>::value || l2norm;

  auto issue_loads = [&](int cc) {
    const int tok0 = b * T + cc * C;
    if (tid == 0) {
      tc::mbar_arrive_expect_tx(tb, TILE_TX_BYTES);
      const uint32_t qk = sbase + OFF_QK, vt = sbase + OFF_V;
      tc::tma_load_3d(qk, &maps.q, 0, hk, tok0, tb);
      tc::tma_load_3d(qk + QK_BLK, &maps.q, 64, hk, tok0, tb);
      tc::tma_load_3d(qk + 64 * 128, &maps.k, 0, hk, tok0, tb);
      tc::tma_load_3d(qk + QK_BLK + 64 * 128, &maps.k, 64, hk, tok0, tb);
      tc::tma_load_3d(vt, &maps.v, 0, hv, tok0, tb);
      tc::tma_load_3d(vt + T64_BLK, &maps.v, 64, hv, tok0, tb);
    }
    const int r = tid & 63;
    if (cc * C + r < T) {
      const size_t idx = ((size_t)b * T + cc * C + r) * Hv + hv;
      cp_async4(sm + OFF_GB + (tid >> 6) * 256 + r * 4, (tid >> 6) ? beta + idx : g + idx);
    }
    cp_async_commit();
  };

  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init(&tbar, 1);
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  issue_loads(0);
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's TMEM lane quarter
  uint32_t phase = 0;
  int pending_chunk = 0;  // chunk whose tiles were requested and not yet waited for (-1: none)

  // ---- initial state: thread d holds column d of S (row d of S^T) ----
  float* Sg = state + (size_t)bh * D * D;
  {
    float buf[32];
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int i = 0; i < 32; ++i) buf[i] = Sg[(size_t)(j * 32 + i) * D + tid];
      tc::tmem_st32(lane_addr + COL_S + j * 32, buf);
    }
    tc::tmem_wait_st();
  }

  auto fail = [&]() {
    atomicExch(&g_chunked_error, 1);
    abort_flag = 1;
  };
  auto sync_mma = [&]() -> bool {
    // every thread: wait until the MMAs committed so far have completed
    const bool ok = __syncthreads_and(tc::mbar_wait(bar, phase));  // block-uniform outcome
    phase ^= 1u;
    if (!ok) fail();
    tc::fence_after();
    return ok;
  };
  auto sync_smem_for_mma = [&]() {
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  };

#pragma unroll 1
  for (int c = 0; c < nchunks && !abort_flag; ++c) {
    const int t0 = c * C;
    const int nvalid = min(C, T - t0);
    // ---------------- tiles and gates of this chunk ----------------
    if (!__syncthreads_and(tc::mbar_wait(tb, (uint32_t)(c & 1)))) {
      fail();
      break;
    }
    pending_chunk = -1;
    cp_async_wait<0>();
    __syncthreads();
    if (always_convert || nvalid < C) convert_tiles<TIn>(sm + OFF_QK, sm + OFF_V, nvalid, l2norm, tid);
    if (warp == 0) {
      const int i0 = 2 * lane, i1 = 2 * lane + 1;
      const float g0 = i0 < nvalid ? sGB[i0] : 0.f, g1 = i1 < nvalid ? sGB[i1] : 0.f;
      const float b0 = i0 < nvalid ? sGB[64 + i0] : 0.f, b1 = i1 < nvalid ? sGB[64 + i1] : 0.f;
      float s = g0 + g1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += n;
      }
      const float G1 = s, G0 = s - g1;
      const float Glast = __shfl_sync(0xffffffffu, G1, 31);
      sG[i0] = G0;
      sG[i1] = G1;
      sBeta[i0] = b0;
      sBeta[i1] = b1;
      sEG[i0] = __expf(G0);
      sEG[i1] = __expf(G1);
      sDec[i0] = __expf(Glast - G0);
      sDec[i1] = __expf(Glast - G1);
      if (lane == 0) *sGamma = __expf(Glast);
    }
    sync_smem_for_mma();

    // ---------------- D1 = [Q;K] K^T ----------------
    if (tid == 0) {
      constexpr uint32_t id = tc::idesc_f16(128, 64, false, false);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t koff = (uint32_t)((s >> 2) * QK_BLK + (s & 3) * 32);
        const uint64_t ad = tc::sdesc_sw128(sbase + OFF_QK + koff, 16, 1024);
        const uint64_t bd = tc::sdesc_sw128(sbase + OFF_QK + 64 * 128 + koff, 16, 1024);
        tc::mma_f16(tmem + COL_R, ad, bd, id, s > 0);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- P (rows 0-63), A (rows 64-127) ----------------
    {
      const int i = tid & 63;
      const float Gi = sG[i];
      float r0[32], r1[32];
      tc::tmem_ld32(lane_addr + COL_R, r0);
      tc::tmem_ld32(lane_addr + COL_R + 32, r1);
      tc::tmem_wait_ld();
      if (tid < 64) {
#pragma unroll
        for (int cb = 0; cb < 8; ++cb) {
          const float4 ga = ld4(sG + cb * 8), gb = ld4(sG + cb * 8 + 4);
          const float gj[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
          float p8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = cb * 8 + e;
            const float x = j < 32 ? r0[j] : r1[j - 32];
            p8[e] = j <= i ? x * __expf(Gi - gj[e]) : 0.f;
          }
          *reinterpret_cast<uint4*>(sm + OFF_P + sw(i, cb)) = pack8_f16(p8);
        }
      } else {
        const float bi = sBeta[i];
        float* arow = sA + i * LDF;
#pragma unroll
        for (int j4 = 0; j4 < 16; ++j4) {
          const float4 g4 = ld4(sG + j4 * 4);
          const float gj[4] = {g4.x, g4.y, g4.z, g4.w};
          float a4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = j4 * 4 + e;
            const float x = j < 32 ? r0[j] : r1[j - 32];
            a4[e] = j < i ? bi * x * __expf(Gi - gj[e]) : 0.f;
          }
          *reinterpret_cast<float4*>(arow + j4 * 4) = make_float4(a4[0], a4[1], a4[2], a4[3]);
        }
      }
    }
    tc::fence_before();
    __syncthreads();

    // ---------------- T = (I + A)^-1, blockwise ----------------
    // (1) diagonal 16x16 blocks: thread (blk, j) solves column j by right-looking substitution;
    //     the upper blocks T[0:16,16:32] and T[32:48,48:64] that the merges read are zeroed
    {
      const int z = tid * 4, sel = z >> 8, w = z & 255;
      const int zr = (sel ? 32 : 0) + (w >> 4), zc = (sel ? 48 : 16) + (w & 15);
      *reinterpret_cast<float4*>(sT + zr * LDF + zc) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (tid < 64) {
      const int o = (tid >> 4) * 16, j = tid & 15;
      float xs[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) xs[i] = i == j ? 1.f : 0.f;
#pragma unroll
      for (int kk = 0; kk < 15; ++kk) {
        const float xk = xs[kk];
#pragma unroll
        for (int i = kk + 1; i < 16; ++i) xs[i] -= sA[(o + i) * LDF + o + kk] * xk;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) sT[(o + i) * LDF + o + j] = xs[i];
    }
    __syncthreads();
    // (2) 16 -> 32: X = A_{r,c} T_{c,c} (kept in A's unused upper block), T_{r,c} = -T_{r,r} X
    {
      const int m = tid >> 6, idx = tid & 63, r = idx >> 2, c0 = (idx & 3) * 4;
      const int ro = m ? 48 : 16, co = m ? 32 : 0;  // block rows ro.., block cols co..
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const float a = sA[(ro + r) * LDF + co + kk];
        const float4 t4 = ld4(sT + (co + kk) * LDF + co + c0);
        acc[0] += a * t4.x; acc[1] += a * t4.y; acc[2] += a * t4.z; acc[3] += a * t4.w;
      }
      *reinterpret_cast<float4*>(sA + (ro - 16 + r) * LDF + co + 16 + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      __syncthreads();
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const float t = sT[(ro + r) * LDF + ro + kk];
        const float4 x4 = ld4(sA + (ro - 16 + kk) * LDF + co + 16 + c0);
        acc[0] += t * x4.x; acc[1] += t * x4.y; acc[2] += t * x4.z; acc[3] += t * x4.w;
      }
      *reinterpret_cast<float4*>(sT + (ro + r) * LDF + co + c0) = make_float4(-acc[0], -acc[1], -acc[2], -acc[3]);
    }
    __syncthreads();
    // (3) 32 -> 64: Y = A[32:64, 0:32] T[0:32, 0:32] (kept in A[0:32, 32:64]); T[32:64, 0:32] = -T[32:64, 32:64] Y
    {
      const int r = tid >> 2, c0 = (tid & 3) * 8;
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll 8
      for (int kk = 0; kk < 32; ++kk) {
        const float a = sA[(32 + r) * LDF + kk];
        const float4 t0 = ld4(sT + kk * LDF + c0), t1 = ld4(sT + kk * LDF + c0 + 4);
        acc[0] += a * t0.x; acc[1] += a * t0.y; acc[2] += a * t0.z; acc[3] += a * t0.w;
        acc[4] += a * t1.x; acc[5] += a * t1.y; acc[6] += a * t1.z; acc[7] += a * t1.w;
      }
      *reinterpret_cast<float4*>(sA + r * LDF + 32 + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(sA + r * LDF + 36 + c0) = make_float4(acc[4], acc[5], acc[6], acc[7]);
      __syncthreads();
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll 8
      for (int kk = 0; kk < 32; ++kk) {
        const float t = sT[(32 + r) * LDF + 32 + kk];
        const float4 y0 = ld4(sA + kk * LDF + 32 + c0), y1 = ld4(sA + kk * LDF + 36 + c0);
        acc[0] += t * y0.x; acc[1] += t * y0.y; acc[2] += t * y0.z; acc[3] += t * y0.w;
        acc[4] += t * y1.x; acc[5] += t * y1.y; acc[6] += t * y1.z; acc[7] += t * y1.w;
      }
      *reinterpret_cast<float4*>(sT + (32 + r) * LDF + c0) = make_float4(-acc[0], -acc[1], -acc[2], -acc[3]);
      *reinterpret_cast<float4*>(sT + (32 + r) * LDF + c0 + 4) = make_float4(-acc[4], -acc[5], -acc[6], -acc[7]);
    }
    __syncthreads();
    // T1 = T diag(beta), T2 = T diag(beta e^G): fp16, swizzled, over A's (now dead) storage
    {
      const int r = tid >> 1, cq = (tid & 1) * 4;  // four 8-column chunks per thread
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        const int c8 = (cq + cb) * 8;
        const float4 ta = ld4(sT + r * LDF + c8), tb4 = ld4(sT + r * LDF + c8 + 4);
        const float4 ba = ld4(sBeta + c8), bb = ld4(sBeta + c8 + 4);
        const float4 ea = ld4(sEG + c8), eb = ld4(sEG + c8 + 4);
        const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb4.x, tb4.y, tb4.z, tb4.w};
        const float bv[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
        const float ev[8] = {ea.x, ea.y, ea.z, ea.w, eb.x, eb.y, eb.z, eb.w};
        float t1[8], t2[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float t = c8 + e <= r ? tv[e] : 0.f;
          t1[e] = t * bv[e];
          t2[e] = t1[e] * ev[e];
        }
        *reinterpret_cast<uint4*>(sm + OFF_T1 + sw(r, cq + cb)) = pack8_f16(t1);
        *reinterpret_cast<uint4*>(sm + OFF_T2 + sw(r, cq + cb)) = pack8_f16(t2);
      }
    }
    sync_smem_for_mma();

    // ---------------- U^T = V^T T1^T ; W^T = K^T T2^T ----------------
    if (tid == 0) {
      constexpr uint32_t id = tc::idesc_f16(128, 64, true, false);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint64_t av = tc::sdesc_sw128(sbase + OFF_V + s * 2048, T64_BLK, 1024);
        const uint64_t b1 = tc::sdesc_sw128(sbase + OFF_T1 + s * 32, 16, 1024);
        tc::mma_f16(tmem + COL_U, av, b1, id, s > 0);
        const uint64_t ak = tc::sdesc_sw128(sbase + OFF_QK + 64 * 128 + s * 2048, QK_BLK, 1024);
        const uint64_t b2 = tc::sdesc_sw128(sbase + OFF_T2 + s * 32, 16, 1024);
        tc::mma_f16(tmem + COL_R, ak, b2, id, s > 0);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- W readout (into the V region) and state readout (into X) ----------------
    {
      float r0[32], r1[32];
      tc::tmem_ld32(lane_addr + COL_R, r0);
      tc::tmem_ld32(lane_addr + COL_R + 32, r1);
      tc::tmem_wait_ld();
      uint8_t* wb = sm + OFF_V + (tid >> 6) * T64_BLK;  // W [token][d_k], two 64-column blocks
#pragma unroll
      for (int t = 0; t < 64; ++t)
        *reinterpret_cast<__half*>(wb + sw_elem(t, tid & 63)) = __float2half_rn(t < 32 ? r0[t] : r1[t - 32]);
      const float gamma = *sGamma;
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
        float s32[32];
        tc::tmem_ld32(lane_addr + COL_S + j * 32, s32);
        tc::tmem_wait_ld();
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          const int kc = j * 4 + cb;  // 16-byte chunk index 0..15 along d_k
          *reinterpret_cast<uint4*>(sm + OFF_ST + (kc >> 3) * QK_BLK + sw(tid, kc & 7)) = pack8_f16(s32 + cb * 8);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) s32[e] *= gamma;
        tc::tmem_st32(lane_addr + COL_S + j * 32, s32);
      }
      tc::tmem_wait_st();
    }
    sync_smem_for_mma();

    // ---------------- Vn^T = U^T - S^T W^T ; O1^T = S^T Q^T ----------------
    if (tid == 0) {
      constexpr uint32_t idn = tc::idesc_f16(128, 64, false, false, true);
      constexpr uint32_t id = tc::idesc_f16(128, 64, false, false);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint64_t as = tc::sdesc_sw128(sbase + OFF_ST + (s >> 2) * QK_BLK + (s & 3) * 32, 16, 1024);
        const uint64_t bw = tc::sdesc_sw128(sbase + OFF_V + (s >> 2) * T64_BLK + (s & 3) * 32, 16, 1024);
        tc::mma_f16(tmem + COL_U, as, bw, idn, 1);
        const uint64_t bq = tc::sdesc_sw128(sbase + OFF_QK + (s >> 2) * QK_BLK + (s & 3) * 32, 16, 1024);
        tc::mma_f16(tmem + COL_R, as, bq, id, s > 0);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- Vn readout: lane = d_v index, columns = tokens ----------------
    {
      float r0[32], r1[32];
      tc::tmem_ld32(lane_addr + COL_U, r0);
      tc::tmem_ld32(lane_addr + COL_U + 32, r1);
      tc::tmem_wait_ld();
#pragma unroll
      for (int cb = 0; cb < 8; ++cb) {
        float x[8], y[8];
        const float4 d0 = ld4(sDec + cb * 8), d1 = ld4(sDec + cb * 8 + 4);
        const float dd[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int t = cb * 8 + e;
          x[e] = t < 32 ? r0[t] : r1[t - 32];
          y[e] = x[e] * dd[e];
        }
        *reinterpret_cast<uint4*>(sm + OFF_V + sw(tid, cb)) = pack8_f16(x);
        *reinterpret_cast<uint4*>(sm + OFF_VD + sw(tid, cb)) = pack8_f16(y);
      }
    }
    sync_smem_for_mma();

    // ---------------- O2^T = Vn^T P^T (into U's columns) ; S^T += (dec Vn)^T K ----------------
    if (tid == 0) {
      constexpr uint32_t id64 = tc::idesc_f16(128, 64, false, false);
      constexpr uint32_t id128 = tc::idesc_f16(128, 128, false, true);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint64_t av = tc::sdesc_sw128(sbase + OFF_V + s * 32, 16, 1024);
        const uint64_t bp = tc::sdesc_sw128(sbase + OFF_P + s * 32, 16, 1024);
        tc::mma_f16(tmem + COL_U, av, bp, id64, s > 0);
        const uint64_t ad = tc::sdesc_sw128(sbase + OFF_VD + s * 32, 16, 1024);
        const uint64_t bk = tc::sdesc_sw128(sbase + OFF_QK + 64 * 128 + s * 2048, QK_BLK, 1024);
        tc::mma_f16(tmem + COL_S, ad, bk, id128, 1);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;
    // the tiles are free: start the next chunk's copies while O drains
    if (c + 1 < nchunks) {
      issue_loads(c + 1);
      pending_chunk = c + 1;
    }

    // ---------------- O = (e^G O1 + O2) * scale -> global ----------------
    {
      float o1[32], o2[32];
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        tc::tmem_ld32(lane_addr + COL_R + hh * 32, o1);
        tc::tmem_ld32(lane_addr + COL_U + hh * 32, o2);
        tc::tmem_wait_ld();
        if constexpr (sizeof(TOut) == 2) {
          TOut* ost = reinterpret_cast<TOut*>(sm + OFF_OST);  // [token][d_v] staging over X
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int tt = hh * 32 + t;
            ost[tt * D + tid] = from_f32<TOut>((sEG[tt] * o1[t] + o2[t]) * scale);
          }
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int tt = hh * 32 + t;
            if (tt < nvalid)
              out[(((size_t)b * T + t0 + tt) * Hv + hv) * D + tid] = from_f32<TOut>((sEG[tt] * o1[t] + o2[t]) * scale);
          }
        }
      }
      if constexpr (sizeof(TOut) == 2) {
        __syncthreads();
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int r = (tid >> 4) + it * 8, ch = tid & 15;
          if (r < nvalid)
            *reinterpret_cast<uint4*>(out + (((size_t)b * T + t0 + r) * Hv + hv) * D + ch * 8) =
                *reinterpret_cast<const uint4*>(sm + OFF_OST + r * 256 + ch * 16);
        }
      }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  }

  cp_async_wait<0>();
  // a stopped CTA still lets the tiles it requested land before it leaves (bounded)
  if (pending_chunk >= 0) tc::mbar_wait(tb, (uint32_t)(pending_chunk & 1));
  // ---- final state ----
  if (!abort_flag) {
    float buf[32];
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      tc::tmem_ld32(lane_addr + COL_S + j * 32, buf);
      tc::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) Sg[(size_t)(j * 32 + i) * D + tid] = buf[i];
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
}

// ------------------------------------------------------------ tensor maps ----
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [d = 128, heads, tokens] view of a [B*T, heads, 128] 2-byte tensor; box 64 x 1 x 64, 128-byte swizzle.
int encode_rows_map(CUtensorMap* m, const void* base, int heads, long long tokens) {
  auto enc = tensor_map_encoder();
  ANEMLL_REQUIRE(enc, ANEMLL_EUNSUPPORTED, "gdn_chunked_prefill: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)tokens};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)heads * D * 2};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)C};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  ANEMLL_REQUIRE(r == CUDA_SUCCESS, ANEMLL_EINVAL, "gdn_chunked_prefill: tensor map encoding failed (%d)", (int)r);
  return ANEMLL_OK;
}

template <typename TIn, typename TOut>
int launch_chunked(const void* q, const void* k, const void* v, const float* g, const float* beta, float* state,
                   void* out, int B, int T, int Hqk, int Hv, float scale, int l2norm, cudaStream_t st) {
  TileMaps maps;
  const long long tokens = (long long)B * T;
  int rc = encode_rows_map(&maps.q, q, Hqk, tokens);
  if (!rc) rc = encode_rows_map(&maps.k, k, Hqk, tokens);
  if (!rc) rc = encode_rows_map(&maps.v, v, Hv, tokens);
  if (rc) return rc;
  auto kern = gdn_chunked_kernel<TIn, TOut>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  kern<<<B * Hv, NT, SMEM_BYTES, st>>>(maps, g, beta, state, (TOut*)out, T, Hqk, Hv, scale, l2norm);
  return launch_status("gdn_chunked_prefill");
}

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_gdn_chunked_prefill(const void* q, const void* k, const void* v, int qkv_dtype,
                                          const float* g, const float* beta, float* state,
                                          void* out, int out_dtype,
                                          int B, int T, int H_qk, int H_v, int d_k, int d_v,
                                          int chunk_size, float scale, int qk_l2norm, void* stream) {
  ANEMLL_REQUIRE(state && (T == 0 || (q && k && v && g && beta && out)), ANEMLL_EINVAL,
                 "gdn_chunked_prefill: null pointer");
  ANEMLL_REQUIRE(B > 0 && T >= 0 && H_qk > 0 && H_v > 0 && H_v % H_qk == 0, ANEMLL_EINVAL,
                 "gdn_chunked_prefill: bad sizes B=%d T=%d H_qk=%d H_v=%d", B, T, H_qk, H_v);
  ANEMLL_REQUIRE(d_k == D && d_v == D, ANEMLL_EUNSUPPORTED, "gdn_chunked_prefill: d_k and d_v must be 128");
  ANEMLL_REQUIRE(chunk_size == C, ANEMLL_EUNSUPPORTED, "gdn_chunked_prefill: chunk_size must be 64");
  ANEMLL_REQUIRE(qkv_dtype == ANEMLL_F16 || qkv_dtype == ANEMLL_BF16, ANEMLL_EUNSUPPORTED,
                 "gdn_chunked_prefill: q/k/v must be f16 or bf16");
  ANEMLL_REQUIRE(dtype_ok(out_dtype), ANEMLL_EUNSUPPORTED, "gdn_chunked_prefill: bad out dtype");
  if (T == 0) return ANEMLL_OK;
  ANEMLL_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(g, 4) && aligned(beta, 4) &&
                     (dtype_size(out_dtype) == 4 || aligned(out, 16)),
                 ANEMLL_EALIGN, "gdn_chunked_prefill: q/k/v (and 2-byte outputs) must be 16-byte aligned");
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)d_k);
  cudaStream_t st = (cudaStream_t)stream;
  return ANEMLL_DISPATCH_HALF(qkv_dtype, TIn, [&] {
    return ANEMLL_DISPATCH_DTYPE(out_dtype, TOut, [&] {
      return launch_chunked<TIn, TOut>(q, k, v, g, beta, state, out, B, T, H_qk, H_v, scale, qk_l2norm, st);
    });
  });
}

extern "C" int anemll_gdn_chunked_error(int reset) {
  int h = 0;
  if (cudaMemcpyFromSymbol(&h, g_chunked_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && h) {
    const int z = 0;
    cudaMemcpyToSymbol(g_chunked_error, &z, sizeof(int));
  }
  return h;
}
