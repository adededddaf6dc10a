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
//   [X1|X2] = -S^T [W;Q]^T                   (tcgen05, one N=128 product, A negated)
//   Vn^T = U^T + X1,  O2^T = Vn^T P^T        (O = diag(e^G) (-X2) + O2 at readout)
//   S^T  = e^{G_c} S^T + (diag(e^{G_c - G}) Vn)^T K   (e^{G_c} applied in TMEM, then tcgen05)
//
// Every product is arranged so that M = 128 (d_v or d_k on TMEM lanes).  All
// operands are fp16 in 128-byte-swizzled shared memory; accumulators are fp32
// in TMEM.  fp16 (10-bit mantissa) operands keep the result within 1e-3
// relative L2 of an fp32 evaluation; bf16 inputs are converted to fp16 in
// place.  The attention scale multiplies O in fp32 at the end (O is linear in q).
//
// Data movement: q/k/v tiles arrive by TMA (3-D tensor maps over [d, head,
// token], 64-token x 64-element boxes, 128-byte swizzle done by the copy
// engine) into two tile buffers: chunk c computes from one while chunk c+1
// lands in the other; the in-place conversion of chunk c+1 (bf16 -> fp16,
// optional l2-norm, zeroing of rows past the sequence end) runs while the
// tensor core works on chunk c.  256 threads: warps w and w+4 read the same
// TMEM lane quarter and split its columns.  T = (I + A)^-1 is built blockwise:
// four 16x16 diagonal blocks by forward substitution, then 16 -> 32 -> 64
// merges T21 = -T22 (A21 T11) as small fp32 matrix products over all threads.
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
constexpr int NT = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0, COL_U = 128, COL_X = 192, COL_O2 = 320, COL_D = 384;  // X: [X1 | X2]

// shared memory map (bytes from a 1024-byte aligned base); lifetimes in a chunk:
//   WQK[x]: rows 0-63 W (written per chunk), 64-127 Q and 128-191 K (TMA) [prep .. S update]
//   V[x] (TMA): V [.. U/W] -> Vn^T [Vn .. S update] -> O staging
//   VD: (dec Vn)^T [Vn .. S update]      R1: A fp32 [P/A .. T] -> T1,T2 [.. U/W]
constexpr int QK_BLK = 128 * 128;   // one 64-column block of a 128-row tile (S^T)
constexpr int WQK_BLK = 192 * 128;  // one 64-column block of the [W;Q;K] tile
constexpr int T64_BLK = 64 * 128;   // one 64-column block of a 64-row tile
constexpr int WQK_BYTES = 2 * WQK_BLK, V_BYTES = 2 * T64_BLK;
constexpr int ROW_Q = 64, ROW_K = 128;
constexpr int LDF = 68;  // fp32 row pitch (floats) of A and T
constexpr int OFF_WQK0 = 0;
constexpr int OFF_V0 = OFF_WQK0 + 2 * WQK_BYTES;
constexpr int OFF_VD = OFF_V0 + 2 * V_BYTES;
constexpr int OFF_P = OFF_VD + 2 * T64_BLK;
constexpr int OFF_ST = OFF_P + T64_BLK;
constexpr int OFF_R1 = OFF_ST + 2 * QK_BLK;
constexpr int OFF_T1 = OFF_R1, OFF_T2 = OFF_R1 + T64_BLK;
constexpr int OFF_T = OFF_R1 + 64 * LDF * 4;
constexpr int OFF_GB = OFF_T + 64 * LDF * 4;    // raw g, beta per buffer: [2][128] floats
constexpr int OFF_MISC = OFF_GB + 2 * 128 * 4;  // G, beta, e^G, dec [64] each, gamma
constexpr int SMEM_BYTES = OFF_MISC + 4 * 64 * 4 + 16 + 1024;
constexpr uint32_t TILE_TX_BYTES = 2 * 2 * 64 * 128 + V_BYTES;  // bytes one chunk's six boxes deliver
static_assert(OFF_R1 % 1024 == 0 && OFF_ST % 1024 == 0, "tile alignment");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

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

// Rewrite one chunk's tiles in place as fp16: convert from TIn, l2-normalise q
// and k rows if asked, zero the rows at and past `nvalid`.
template <typename TIn>
__device__ __forceinline__ void convert_tiles(uint8_t* wqk, uint8_t* vt, int nvalid, int l2norm, int tid) {
  const int ch = tid & 15;
  const int blk = ch >> 3, cb = ch & 7;
#pragma unroll 1
  for (int it = 0; it < 4; ++it) {
    const int r = (tid >> 4) + it * 16;
    uint4* pq = reinterpret_cast<uint4*>(wqk + blk * WQK_BLK + sw(ROW_Q + r, cb));
    uint4* pk = reinterpret_cast<uint4*>(wqk + blk * WQK_BLK + sw(ROW_K + r, cb));
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
__global__ void __launch_bounds__(NT, 1)
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
  float* sA = reinterpret_cast<float*>(sm + OFF_R1);
  float* sT = reinterpret_cast<float*>(sm + OFF_T);
  __shared__ uint64_t mbar;       // tensor-core completions
  __shared__ uint64_t tbar[2];    // TMA arrivals per tile buffer
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = tid & 127;   // TMEM lane this thread reads (warps w and w+4 share a lane quarter)
  const int half = tid >> 7;   // which half of the columns it reads
  const int bh = blockIdx.x;
  const int b = bh / Hv, hv = bh % Hv;
  const int hk = hv / (Hv / Hqk);
  const uint32_t sbase = tc::smem_u32(sm);
  const uint32_t bar = tc::smem_u32(&mbar);
  const uint32_t tb0 = tc::smem_u32(&tbar[0]);
  const int nchunks = (T + C - 1) / C;
  // fp16 inputs without l2-norm need no rewrite except for a ragged last chunk
  constexpr bool kConvert = sizeof(TIn) == 2 && !std::is_same<TIn, __half>::value;
  const bool always_convert = kConvert || l2norm;

  // chunk cc -> buffer cc & 1: six TMA boxes plus the gates by cp.async
  auto issue_loads = [&](int cc) {
    const int x = cc & 1;
    const int tok0 = b * T + cc * C;
    if (tid == 0) {
      const uint32_t tb = tb0 + 8u * x;
      tc::mbar_arrive_expect_tx(tb, TILE_TX_BYTES);
      const uint32_t w = sbase + OFF_WQK0 + x * WQK_BYTES, vt = sbase + OFF_V0 + x * V_BYTES;
      tc::tma_load_3d(w + ROW_Q * 128, &maps.q, 0, hk, tok0, tb);
      tc::tma_load_3d(w + WQK_BLK + ROW_Q * 128, &maps.q, 64, hk, tok0, tb);
      tc::tma_load_3d(w + ROW_K * 128, &maps.k, 0, hk, tok0, tb);
      tc::tma_load_3d(w + WQK_BLK + ROW_K * 128, &maps.k, 64, hk, tok0, tb);
      tc::tma_load_3d(vt, &maps.v, 0, hv, tok0, tb);
      tc::tma_load_3d(vt + T64_BLK, &maps.v, 64, hv, tok0, tb);
    }
    if (tid < 128) {
      const int r = tid & 63;
      if (cc * C + r < T) {
        const size_t idx = ((size_t)b * T + cc * C + r) * Hv + hv;
        cp_async4(sm + OFF_GB + x * 512 + (tid >> 6) * 256 + r * 4, (tid >> 6) ? beta + idx : g + idx);
      }
    }
    cp_async_commit();
  };

  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init(&tbar[0], 1);
    tc::mbar_init(&tbar[1], 1);
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
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's TMEM lane quarter
  uint32_t phase = 0;
  int pending_chunk = 0;  // chunk whose tiles were requested and not yet waited for (-1: none)

  // ---- initial state: thread (row d, half) holds S[half*64 .. +64, d] (row d of S^T) ----
  float* Sg = state + (size_t)bh * D * D;
  {
    float buf[32];
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int k0 = half * 64 + j * 32;
#pragma unroll
      for (int i = 0; i < 32; ++i) buf[i] = Sg[(size_t)(k0 + i) * D + row];
      tc::tmem_st32(lane_addr + COL_S + k0, buf);
    }
    tc::tmem_wait_st();
  }

  auto fail = [&]() {
    atomicExch(&g_chunked_error, 1);
    abort_flag = 1;
  };
  auto sync_mma = [&]() -> bool {
    // every thread: wait until the MMAs committed so far have completed
    const bool ok = tc::mbar_wait(bar, phase);
    phase ^= 1u;
    if (!ok) fail();
    tc::fence_after();
    return ok;
  };
  auto wait_tiles = [&](int cc) -> bool {
    const bool ok = tc::mbar_wait(tb0 + 8u * (cc & 1), (uint32_t)((cc >> 1) & 1));
    if (!ok) fail();
    else pending_chunk = -1;
    return ok;
  };
  auto sync_smem_for_mma = [&]() {
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  };

  if (wait_tiles(0) && (always_convert || T < C))
    convert_tiles<TIn>(sm + OFF_WQK0, sm + OFF_V0, min(C, T), l2norm, tid);

#pragma unroll 1
  for (int c = 0; c < nchunks && !abort_flag; ++c) {
    const int x = c & 1;
    const int t0 = c * C;
    const int nvalid = min(C, T - t0);
    const uint32_t wqk_a = sbase + OFF_WQK0 + x * WQK_BYTES;
    const int wqk_off = OFF_WQK0 + x * WQK_BYTES;
    const uint32_t v_a = sbase + OFF_V0 + x * V_BYTES;
    const int v_off = OFF_V0 + x * V_BYTES;
    cp_async_wait<0>();
    __syncthreads();

    // ---------------- gates: cumulative log decay (padding tokens: g = beta = 0) ----------------
    if (warp == 0) {
      const float* gb = reinterpret_cast<const float*>(sm + OFF_GB + x * 512);
      const int i0 = 2 * lane, i1 = 2 * lane + 1;
      const float g0 = i0 < nvalid ? gb[i0] : 0.f, g1 = i1 < nvalid ? gb[i1] : 0.f;
      const float b0 = i0 < nvalid ? gb[64 + i0] : 0.f, b1 = i1 < nvalid ? gb[64 + i1] : 0.f;
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
    if (c + 1 < nchunks) {  // the other buffer was released by chunk c-1
      issue_loads(c + 1);
      pending_chunk = c + 1;
    }

    // ---------------- D1 = [Q;K] K^T ----------------
    if (tid == 0) {
      constexpr uint32_t id = tc::idesc_f16(128, 64, false, false);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t koff = (uint32_t)((s >> 2) * WQK_BLK + (s & 3) * 32);
        const uint64_t ad = tc::sdesc_sw128(wqk_a + ROW_Q * 128 + koff, 16, 1024);
        const uint64_t bd = tc::sdesc_sw128(wqk_a + ROW_K * 128 + koff, 16, 1024);
        tc::mma_f16(tmem + COL_D, ad, bd, id, s > 0);
      }
      tc::commit(bar);
    }

    // state readout (independent of D1): S^T row -> fp16 operand, then scale the accumulator by gamma
    {
      const float gamma = *sGamma;
#pragma unroll 1
      for (int j = 0; j < 2; ++j) {
        const int k0 = half * 64 + j * 32;
        float s32[32];
        tc::tmem_ld32(lane_addr + COL_S + k0, s32);
        tc::tmem_wait_ld();
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          const int kc = (k0 >> 3) + cb;  // 16-byte chunk index 0..15 along d_k
          *reinterpret_cast<uint4*>(sm + OFF_ST + (kc >> 3) * QK_BLK + sw(row, kc & 7)) = pack8_f16(s32 + cb * 8);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) s32[e] *= gamma;
        tc::tmem_st32(lane_addr + COL_S + k0, s32);
      }
      tc::tmem_wait_st();
    }
    if (!sync_mma()) break;

    // ---------------- P (rows 0-63), A (rows 64-127): each thread 32 columns ----------------
    {
      const int i = row & 63;
      const float Gi = sG[i];
      float r32[32];
      tc::tmem_ld32(lane_addr + COL_D + half * 32, r32);
      tc::tmem_wait_ld();
      if (row < 64) {
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          float p8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = half * 32 + cb * 8 + e;
            p8[e] = j <= i ? r32[cb * 8 + e] * __expf(Gi - sG[j]) : 0.f;
          }
          *reinterpret_cast<uint4*>(sm + OFF_P + sw(i, half * 4 + cb)) = pack8_f16(p8);
        }
      } else {
        const float bi = sBeta[i];
        float* arow = sA + i * LDF + half * 32;
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          float a4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = half * 32 + j4 * 4 + e;
            a4[e] = j < i ? bi * r32[j4 * 4 + e] * __expf(Gi - sG[j]) : 0.f;
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
      const int z = tid * 2, sel = z >> 8, w = z & 255;
      const int zr = (sel ? 32 : 0) + (w >> 4), zc = (sel ? 48 : 16) + (w & 15);
      *reinterpret_cast<float2*>(sT + zr * LDF + zc) = make_float2(0.f, 0.f);
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
      const int m = tid >> 7, idx = tid & 127, r = idx >> 3, c0 = (idx & 7) * 2;
      const int ro = m ? 48 : 16, co = m ? 32 : 0;  // block rows ro.., block cols co..
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const float a = sA[(ro + r) * LDF + co + kk];
        const float2 t2 = *reinterpret_cast<const float2*>(sT + (co + kk) * LDF + co + c0);
        a0 += a * t2.x;
        a1 += a * t2.y;
      }
      *reinterpret_cast<float2*>(sA + (ro - 16 + r) * LDF + co + 16 + c0) = make_float2(a0, a1);
      __syncthreads();
      a0 = a1 = 0.f;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const float t = sT[(ro + r) * LDF + ro + kk];
        const float2 x2 = *reinterpret_cast<const float2*>(sA + (ro - 16 + kk) * LDF + co + 16 + c0);
        a0 += t * x2.x;
        a1 += t * x2.y;
      }
      *reinterpret_cast<float2*>(sT + (ro + r) * LDF + co + c0) = make_float2(-a0, -a1);
    }
    __syncthreads();
    // (3) 32 -> 64: Y = A[32:64, 0:32] T[0:32, 0:32] (kept in A[0:32, 32:64]); T[32:64, 0:32] = -T[32:64, 32:64] Y
    {
      const int r = tid >> 3, c0 = (tid & 7) * 4;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
      for (int kk = 0; kk < 32; ++kk) {
        const float a = sA[(32 + r) * LDF + kk];
        const float4 t4 = *reinterpret_cast<const float4*>(sT + kk * LDF + c0);
        acc[0] += a * t4.x; acc[1] += a * t4.y; acc[2] += a * t4.z; acc[3] += a * t4.w;
      }
      *reinterpret_cast<float4*>(sA + r * LDF + 32 + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      __syncthreads();
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll 8
      for (int kk = 0; kk < 32; ++kk) {
        const float t = sT[(32 + r) * LDF + 32 + kk];
        const float4 y4 = *reinterpret_cast<const float4*>(sA + kk * LDF + 32 + c0);
        acc[0] += t * y4.x; acc[1] += t * y4.y; acc[2] += t * y4.z; acc[3] += t * y4.w;
      }
      *reinterpret_cast<float4*>(sT + (32 + r) * LDF + c0) = make_float4(-acc[0], -acc[1], -acc[2], -acc[3]);
    }
    __syncthreads();
    // T1 = T diag(beta), T2 = T diag(beta e^G): fp16, swizzled, over A's (now dead) storage
    {
      const int r = tid >> 2, cq = (tid & 3) * 2;  // two 8-column chunks per thread
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        float t1[8], t2[8];
        const int c8 = (cq + cb) * 8;
        const float4 ta = *reinterpret_cast<const float4*>(sT + r * LDF + c8);
        const float4 tb = *reinterpret_cast<const float4*>(sT + r * LDF + c8 + 4);
        const float4 ba = *reinterpret_cast<const float4*>(sBeta + c8), bb = *reinterpret_cast<const float4*>(sBeta + c8 + 4);
        const float4 ea = *reinterpret_cast<const float4*>(sEG + c8), eb = *reinterpret_cast<const float4*>(sEG + c8 + 4);
        const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
        const float bv[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
        const float ev[8] = {ea.x, ea.y, ea.z, ea.w, eb.x, eb.y, eb.z, eb.w};
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
        const uint64_t av = tc::sdesc_sw128(v_a + s * 2048, T64_BLK, 1024);
        const uint64_t b1 = tc::sdesc_sw128(sbase + OFF_T1 + s * 32, 16, 1024);
        tc::mma_f16(tmem + COL_U, av, b1, id, s > 0);
        const uint64_t ak = tc::sdesc_sw128(wqk_a + ROW_K * 128 + s * 2048, WQK_BLK, 1024);
        const uint64_t b2 = tc::sdesc_sw128(sbase + OFF_T2 + s * 32, 16, 1024);
        tc::mma_f16(tmem + COL_D, ak, b2, id, s > 0);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- W readout: lane = d_k index, 32 token columns per thread ----------------
    {
      uint8_t* wb = sm + wqk_off + (row >> 6) * WQK_BLK;  // rows 0-63 of [W;Q;K]
      float r32[32];
      tc::tmem_ld32(lane_addr + COL_D + half * 32, r32);
      tc::tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < 32; ++t)
        *reinterpret_cast<__half*>(wb + sw_elem(half * 32 + t, row & 63)) = __float2half_rn(r32[t]);
    }
    sync_smem_for_mma();

    // ---------------- [X1 | X2] = -S^T [W;Q]^T : one N=128 product ----------------
    if (tid == 0) {
      constexpr uint32_t idn = tc::idesc_f16(128, 128, false, false, true);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint64_t as = tc::sdesc_sw128(sbase + OFF_ST + (s >> 2) * QK_BLK + (s & 3) * 32, 16, 1024);
        const uint64_t bwq = tc::sdesc_sw128(wqk_a + (s >> 2) * WQK_BLK + (s & 3) * 32, 16, 1024);
        tc::mma_f16(tmem + COL_X, as, bwq, idn, s > 0);
      }
      tc::commit(bar);
    }
    // while the tensor core works: land and rewrite the next chunk's tiles
    if (c + 1 < nchunks) {
      const int nv1 = min(C, T - (c + 1) * C);
      if (wait_tiles(c + 1) && (always_convert || nv1 < C))
        convert_tiles<TIn>(sm + OFF_WQK0 + (x ^ 1) * WQK_BYTES, sm + OFF_V0 + (x ^ 1) * V_BYTES, nv1, l2norm, tid);
    }
    if (!sync_mma()) break;

    // ---------------- Vn readout: lane = d_v index, 32 token columns per thread ----------------
    {
      float r32[32], x32[32];
      tc::tmem_ld32(lane_addr + COL_U + half * 32, r32);
      tc::tmem_ld32(lane_addr + COL_X + half * 32, x32);
      tc::tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) r32[e] += x32[e];
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float y[8];
        const float4 d0 = *reinterpret_cast<const float4*>(sDec + half * 32 + cb * 8);
        const float4 d1 = *reinterpret_cast<const float4*>(sDec + half * 32 + cb * 8 + 4);
        const float dd[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = r32[cb * 8 + e] * dd[e];
        *reinterpret_cast<uint4*>(sm + v_off + sw(row, half * 4 + cb)) = pack8_f16(r32 + cb * 8);
        *reinterpret_cast<uint4*>(sm + OFF_VD + sw(row, half * 4 + cb)) = pack8_f16(y);
      }
    }
    sync_smem_for_mma();

    // ---------------- O2^T = Vn^T P^T ; S^T += (dec Vn)^T K ----------------
    if (tid == 0) {
      constexpr uint32_t id64 = tc::idesc_f16(128, 64, false, false);
      constexpr uint32_t id128 = tc::idesc_f16(128, 128, false, true);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint64_t av = tc::sdesc_sw128(v_a + s * 32, 16, 1024);
        const uint64_t bp = tc::sdesc_sw128(sbase + OFF_P + s * 32, 16, 1024);
        tc::mma_f16(tmem + COL_O2, av, bp, id64, s > 0);
        const uint64_t ad = tc::sdesc_sw128(sbase + OFF_VD + s * 32, 16, 1024);
        const uint64_t bk = tc::sdesc_sw128(wqk_a + ROW_K * 128 + s * 2048, WQK_BLK, 1024);
        tc::mma_f16(tmem + COL_S, ad, bk, id128, 1);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- O = (e^G O1 + O2) * scale -> global ----------------
    {
      float o1[32], o2[32];
      tc::tmem_ld32(lane_addr + COL_X + 64 + half * 32, o1);
      tc::tmem_ld32(lane_addr + COL_O2 + half * 32, o2);
      tc::tmem_wait_ld();
      if constexpr (sizeof(TOut) == 2) {
        // stage [token][d_v] in this chunk's V region, then write whole 256-byte rows
        TOut* ost = reinterpret_cast<TOut*>(sm + v_off);
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int tt = half * 32 + t;
          ost[tt * D + row] = from_f32<TOut>((o2[t] - sEG[tt] * o1[t]) * scale);
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int r = (tid >> 4) + it * 16, ch = tid & 15;
          if (r < nvalid)
            *reinterpret_cast<uint4*>(out + (((size_t)b * T + t0 + r) * Hv + hv) * D + ch * 8) =
                *reinterpret_cast<const uint4*>(sm + v_off + r * 256 + ch * 16);
        }
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int tt = half * 32 + t;
          if (tt < nvalid)
            out[(((size_t)b * T + t0 + tt) * Hv + hv) * D + row] = from_f32<TOut>((o2[t] - sEG[tt] * o1[t]) * scale);
        }
      }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  }

  cp_async_wait<0>();
  // a stopped CTA still lets the tiles it requested land before it leaves (bounded)
  if (pending_chunk >= 0) tc::mbar_wait(tb0 + 8u * (pending_chunk & 1), (uint32_t)((pending_chunk >> 1) & 1));
  // ---- final state ----
  if (!abort_flag) {
    float buf[32];
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int k0 = half * 64 + j * 32;
      tc::tmem_ld32(lane_addr + COL_S + k0, buf);
      tc::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) Sg[(size_t)(k0 + i) * D + row] = buf[i];
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
