// Gated delta rule, chunked prefill on the 5th-generation tensor cores.
//
// One CTA owns one (sequence b, value head h) and walks its chunks of C = 64
// tokens in order; the fp32 state S [d_k=128, d_v=128] lives in tensor memory
// (TMEM) as S^T (lane = d_v index, column = d_k index) for the whole sequence
// and leaves the SM only after the last chunk.  With G the in-chunk cumulative
// log-decay, Gam[i,j] = exp(G_i - G_j), and rq, rk the reciprocal l2 norms of
// the q and k rows (1 when the caller normalised them already), per chunk:
//
//   D1   = [Q;K] [Q;K]^T                          (tcgen05, M=128 N=128 K=128; its
//                                                  diagonal gives the row norms)
//   P    = lower_incl(rq rk^T (Q K^T) * Gam)      (CUDA cores, fp16 to smem)
//   A    = strict_lower(diag(beta rk) K K^T diag(rk) * Gam)
//   T    = (I + A)^-1: 16x16 diagonal blocks by forward substitution (fp32),
//          16 -> 32 -> 64 merges T21 = -T22 (A21 T11) on mma.sync (fp16 operands)
//   U^T  = V^T (T diag(beta))^T                   (tcgen05, M=128 N=64 K=64)
//   W^T  = K^T (T diag(beta e^G rk))^T            (tcgen05)
//   Vn^T = U^T - S^T W^T                          (tcgen05, A negated, accumulates on U)
//   O1^T = S^T Q^T,  O2^T = Vn^T P^T              (tcgen05; O = diag(e^G rq) O1 + O2 at readout,
//                                                  the attention scale folded into P and the O1 factor)
//   S^T  = e^{G_c} S^T + (diag(e^{G_c - G} rk) Vn)^T K   (e^{G_c} applied in TMEM)
//
// Operand precision.  q, k and v are used as they arrive (fp16 or bf16) — no
// conversion pass.  The derived operands that multiply them, T diag(beta),
// T diag(beta e^G rk) and the decayed Vn, are split into a hi and a lo part of
// the input type (x = hi + lo, about 16 significant bits) and enter their
// products as two accumulating MMAs; S^T and W^T are single-precision-of-the-
// input-type operands; the Vn P^T product runs in fp16.  A CPU emulation of
// every rounding point gives output rel-L2 ~3e-4 and state rel-L2 ~3e-6
// against an fp64 recurrence (bf16 inputs, the layer's input and gate distributions).
//
// Occupancy: two CTAs per SM (256 threads, 256 TMEM columns and ~112 KB of
// shared memory each).  Warps w and w + 4 share TMEM lane quarter w and split
// every row readout by columns, so four warps per scheduler hide the latency
// of the tensor-memory loads, the exponentials and the barriers.  Shared memory
// is reused phase by phase (map below); the first half of the state readout
// runs while the tensor core forms U and W.
// q/k tiles and v tiles arrive by TMA on separate barriers (3-D tensor maps
// over [d, head, token], 64-token x 64-element boxes, 128-byte swizzle): the
// next chunk's v is requested once U has been formed, its q/k once the state
// update has read k.
//
// Semantics: torch_chunk_gated_delta_rule of transformers 5.5.0
// (modeling_qwen3_5.py:234-311); chunk (WY/UT) form of Yang et al. (2024).
//
// Gated form (anemll_gdn_chunked_prefill_gated): the layer's gated RMSNorm
// (Qwen3_5RMSNormGated, modeling_qwen3_5.py:175-190) runs in the epilogue.  A
// CTA holds all d_v columns of its head, so the chunk's fp32 output tile is
// staged in shared memory and four threads per token reduce its sum of squares
// and write weight * o * rsqrt(mean(o^2) + eps) * silu(z) directly.
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
constexpr uint32_t TMEM_COLS = 256;
// S^T: cols 0-127.  D1: cols 128-255.  Then U -> Vn -> O2 at 128-191, W -> O1 at 192-255.
constexpr uint32_t COL_S = 0, COL_D1 = 128, COL_U = 128, COL_W = 192;

// Shared memory (bytes from a 1024-byte aligned base) and lifetimes within a chunk:
//   QK (TMA)  rows 0-63 Q, 64-127 K, two 64-column blocks          [load .. state update]
//   V  (TMA)  two 64-column blocks                                   [load .. U]
//   P  fp16 [i][j]                                                   [P/A .. O2]
//   R1 32 KB: T1 hi|lo, T2 hi|lo [i][j]  ->  W^T [d_k][tok] | S^T copy, d_k 64-127  ->  decayed Vn hi|lo [d_v][tok]
//   R2 16 KB: A fp16 | T fp16 [i][j]  ->  S^T copy, d_k 0-63 [d_v][64]  ->  Vn fp16 [d_v][tok]  ->  O staging
//   AD fp32 diagonal 16x16 blocks of A
constexpr int QK_BLK = 128 * 128;  // one 64-column block of a 128-row tile
constexpr int T64_BLK = 64 * 128;  // one 64-column block of a 64-row tile
constexpr int OFF_QK = 0;
constexpr int OFF_V = OFF_QK + 2 * QK_BLK;
constexpr int OFF_P = OFF_V + 2 * T64_BLK;
constexpr int OFF_R1 = OFF_P + T64_BLK;
constexpr int OFF_T1H = OFF_R1, OFF_T1L = OFF_R1 + T64_BLK, OFF_T2H = OFF_R1 + 2 * T64_BLK,
              OFF_T2L = OFF_R1 + 3 * T64_BLK;
constexpr int OFF_W = OFF_R1;                           // W^T [d_k 128][tok 64], MN-major operand
constexpr int OFF_SB1 = OFF_R1 + QK_BLK;                // S^T copy, d_k 64-127: [d_v 128][64]
constexpr int OFF_DH = OFF_R1, OFF_DL = OFF_R1 + QK_BLK;  // [d_v 128][tok 64]
constexpr int OFF_R2 = OFF_R1 + 4 * T64_BLK;
constexpr int OFF_A16 = OFF_R2, OFF_T16 = OFF_R2 + T64_BLK;
constexpr int OFF_SB0 = OFF_R2;  // S^T copy, d_k 0-63
constexpr int OFF_VN = OFF_R2;   // Vn^T [d_v 128][tok 64]
constexpr int OFF_OST = OFF_R2;  // [tok 64][d_v 128] 2-byte staging
constexpr int OFF_AD = OFF_R2 + QK_BLK;
constexpr int AD_BLK = 16 * 16 + 16;  // floats per diagonal block of A, column-major, padded (bank spread)
constexpr int OFF_MISC = OFF_AD + 4 * AD_BLK * 4;
// MISC (floats), per token of the chunk unless noted:
//   raw g[64] beta[64] | G log2e | beta | dec rk (dec = e^{G_c - G}) | O1 factor e^G rq scale |
//   T2 column scale beta e^G rk | log2 column factor Gk = G log2e - log2 rk |
//   log2 row factors of P (G log2e + log2(rq scale)) and of A (G log2e + log2(beta rk)) | gamma, G_c log2e
constexpr int M_GB = 0, M_GL = 128, M_BETA = 192, M_DK = 256, M_OF = 320, M_T2S = 384, M_GK = 448, M_GQ = 512,
              M_GA = 576, M_GAMMA = 640, M_GLL = 641;
constexpr int SMEM_BYTES = OFF_MISC + 644 * 4 + 1024;  // + slack for the 1024-byte alignment of the base
constexpr uint32_t QK_TX_BYTES = 2 * QK_BLK, V_TX_BYTES = 2 * T64_BLK;
static_assert(OFF_V % 1024 == 0 && OFF_P % 1024 == 0 && OFF_R1 % 1024 == 0 && OFF_R2 % 1024 == 0, "tile alignment");
// two CTAs per SM: each also holds 1 KB of static shared memory (the aligned dynamic base pads the
// static section to 1 KB) and the 1 KB the hardware reserves per CTA, out of 228 KB per SM
static_assert(2 * (SMEM_BYTES + 1024 + 1024) <= 228 * 1024, "two CTAs per SM");

struct TileMaps {
  CUtensorMap q, k, v;
};

// The gated RMSNorm's extra operands: z rows (token row b*T + t, z_ld elements apart, heads dense,
// 16-byte aligned), the weight [d_v], eps, and an optional fp32 copy of the core output (NULL: not
// written).
template <typename TZ>
struct GatedNorm {
  const TZ* z;
  long long z_ld;
  const float* w;
  float eps;
  float* core_out;
};

__device__ int g_chunked_error = 0;

// byte offset of 16-byte chunk `ch` (0..7) of row `r` inside a 128-byte-row swizzled block
// (the TMA 128-byte swizzle: chunk index XOR row index mod 8, 1024-byte aligned blocks)
__device__ __forceinline__ uint32_t sw(int r, int ch) { return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4)); }
// byte offset of 2-byte element (r, c), c in 0..63
__device__ __forceinline__ uint32_t sw_elem(int r, int c) { return sw(r, c >> 3) + (uint32_t)((c & 7) << 1); }

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = pack2<T>(f[2 * i], f[2 * i + 1]);
  return u;
}

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w);
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// x = hi + lo with hi, lo of type T (lo = the rounding remainder of hi)
template <typename T>
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack2<T>(a, b);
  const float2 h = unpack2<T>(hi);
  lo = pack2<T>(a - h.x, b - h.y);
}

template <typename T>
__device__ __forceinline__ void pack8_hilo(const float* f, uint4& hi, uint4& lo) {
  uint32_t* h = reinterpret_cast<uint32_t*>(&hi);
  uint32_t* l = reinterpret_cast<uint32_t*>(&lo);
#pragma unroll
  for (int i = 0; i < 4; ++i) split2<T>(f[2 * i], f[2 * i + 1], h[i], l[i]);
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// lane-indexed element of a 32-register row (the diagonal of a 32x32 TMEM block)
__device__ __forceinline__ float pick_lane(const float* r, int lane) {
  float d = 0.f;
#pragma unroll
  for (int e = 0; e < 32; ++e) d = e == lane ? r[e] : d;
  return d;
}

template <typename TIn, typename TOut, bool GATED>
__global__ void __launch_bounds__(NT, 2)
gdn_chunked_kernel(const __grid_constant__ TileMaps maps, const float* __restrict__ g, const float* __restrict__ beta,
                   float* __restrict__ state, TOut* __restrict__ out, int T, int Hqk, int Hv, float scale,
                   int l2norm, const GatedNorm<TOut> gn) {
  constexpr bool kBF = std::is_same<TIn, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* misc = reinterpret_cast<float*>(sm + OFF_MISC);
  float* sGB = misc + M_GB;
  float* sGl = misc + M_GL;
  float* sBeta = misc + M_BETA;
  float* sDk = misc + M_DK;
  float* sOf = misc + M_OF;
  float* sT2s = misc + M_T2S;
  float* sGk = misc + M_GK;
  float* sGq = misc + M_GQ;
  float* sGa = misc + M_GA;
  float* sAd = reinterpret_cast<float*>(sm + OFF_AD);
  __shared__ uint64_t mbar;           // tensor-core completions
  __shared__ uint64_t qkbar, vbar;    // TMA arrivals of the q/k and v tiles
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2;  // TMEM lane quarter, column half
  const int row = tid & 127;                // the TMEM lane (tile row) this thread reads
  const int bh = blockIdx.x;
  const int b = bh / Hv, hv = bh % Hv;
  const int hk = hv / (Hv / Hqk);
  const uint32_t sbase = tc::smem_u32(sm);
  const uint32_t bar = tc::smem_u32(&mbar);
  const uint32_t qkb = tc::smem_u32(&qkbar), vb = tc::smem_u32(&vbar);
  const int nchunks = (T + C - 1) / C;

  auto issue_qk = [&](int cc) {
    const int tok0 = b * T + cc * C;
    if (tid == 0) {
      tc::mbar_arrive_expect_tx(qkb, QK_TX_BYTES);
      const uint32_t qk = sbase + OFF_QK;
      tc::tma_load_3d(qk, &maps.q, 0, hk, tok0, qkb);
      tc::tma_load_3d(qk + QK_BLK, &maps.q, 64, hk, tok0, qkb);
      tc::tma_load_3d(qk + 64 * 128, &maps.k, 0, hk, tok0, qkb);
      tc::tma_load_3d(qk + QK_BLK + 64 * 128, &maps.k, 64, hk, tok0, qkb);
    }
    const int r = tid & 63;
    if (tid < 128 && cc * C + r < T) {
      const size_t idx = ((size_t)b * T + cc * C + r) * Hv + hv;
      cp_async4(sGB + (tid >> 6) * 64 + r, (tid >> 6) ? beta + idx : g + idx);
    }
    cp_async_commit();
  };
  auto issue_v = [&](int cc) {
    if (tid == 0) {
      const int tok0 = b * T + cc * C;
      tc::mbar_arrive_expect_tx(vb, V_TX_BYTES);
      tc::tma_load_3d(sbase + OFF_V, &maps.v, 0, hv, tok0, vb);
      tc::tma_load_3d(sbase + OFF_V + T64_BLK, &maps.v, 64, hv, tok0, vb);
    }
  };

  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init(&qkbar, 1);
    tc::mbar_init(&vbar, 1);
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
  issue_qk(0);
  issue_v(0);
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);  // this warp's TMEM lane quarter
  uint32_t phase = 0;
  int pending_qk = 0, pending_v = 0;  // chunk whose tiles were requested and not yet waited for (-1: none)

  // ---- initial state: thread (row d, half hf) holds S[64 hf .. 64 hf + 63][d] (row d of S^T) ----
  float* Sg = state + (size_t)bh * D * D;
  {
    float buf[32];
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int k0 = 64 * hf + 32 * j;
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
  constexpr uint32_t ID_D1 = tc::idesc_f16(128, 128, false, false, false, kBF);
  constexpr uint32_t ID_VN = tc::idesc_f16(128, 64, false, true, true, kBF);
  constexpr uint32_t ID_O1 = tc::idesc_f16(128, 64, false, false, false, kBF);
  constexpr uint32_t ID_SU = tc::idesc_f16(128, 128, false, true, false, kBF);

#pragma unroll 1
  for (int c = 0; c < nchunks && !abort_flag; ++c) {
    const int t0 = c * C;
    const int nvalid = min(C, T - t0);
    // ---------------- tiles and gates of this chunk ----------------
    if (!__syncthreads_and(tc::mbar_wait(qkb, (uint32_t)(c & 1)))) {
      fail();
      break;
    }
    pending_qk = -1;
    cp_async_wait<0>();
    // ---------------- D1 = [Q;K] [Q;K]^T (issued before the gates are formed) ----------------
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t koff = (uint32_t)((s >> 2) * QK_BLK + (s & 3) * 32);
        const uint64_t d = tc::sdesc_sw128(sbase + OFF_QK + koff, 16, 1024);
        tc::mma_f16(tmem + COL_D1, d, d, ID_D1, s > 0);
      }
      tc::commit(bar);
    }
    __syncthreads();  // raw g / beta of every thread visible
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
      constexpr float L2E = 1.4426950408889634f;
      const float Gl1 = s * L2E, Gl0 = (s - g1) * L2E;
      const float Gll = __shfl_sync(0xffffffffu, Gl1, 31);
      sGl[i0] = Gl0;
      sGl[i1] = Gl1;
      sBeta[i0] = b0;
      sBeta[i1] = b1;
      if (lane == 0) {
        misc[M_GAMMA] = fast_exp2(Gll);
        misc[M_GLL] = Gll;
      }
      if (!l2norm) {  // rq = rk = 1
        const float e0 = fast_exp2(Gl0), e1 = fast_exp2(Gl1), d0 = fast_exp2(Gll - Gl0), d1 = fast_exp2(Gll - Gl1);
        const float ls = log2f(scale);
        sDk[i0] = d0;
        sDk[i1] = d1;
        sOf[i0] = e0 * scale;
        sOf[i1] = e1 * scale;
        sT2s[i0] = b0 * e0;
        sT2s[i1] = b1 * e1;
        sGk[i0] = Gl0;
        sGk[i1] = Gl1;
        sGq[i0] = Gl0 + ls;
        sGq[i1] = Gl1 + ls;
        sGa[i0] = Gl0 + log2f(b0);
        sGa[i1] = Gl1 + log2f(b1);
      }
    }
    if (!sync_mma()) break;  // D1 done; gates visible

    // ---------------- P (rows 0-63), A (rows 64-127) ----------------
    // P_ij = x_ij 2^(Gq_i - Gk_j) (j <= i), A_ij = x_ij 2^(Ga_i - Gk_j) (j < i): the norms, beta and the
    // attention scale ride in the log2 row / column factors
    {
      const bool qrow = row < 64;
      const int i = row & 63;
      float r0[32];  // D1 columns 64 + 32 hf ..: row . k_j for j in [32 hf, 32 hf + 32)
      tc::tmem_ld32(lane_addr + COL_D1 + 64 + 32 * hf, r0);
      if (l2norm) {
        const float Gli = sGl[i];
        if (qrow) {
          if (hf == 0) {  // |q_i|^2 sits in column i of the QQ^T block
            float rd[32];
            tc::tmem_ld32(lane_addr + COL_D1 + (qd & 1) * 32, rd);
            tc::tmem_wait_ld();
            const float rq = rsqrtf(pick_lane(rd, lane) + 1e-6f);
            sOf[i] = fast_exp2(Gli) * rq * scale;
            sGq[i] = Gli + log2f(rq * scale);
          } else {
            tc::tmem_wait_ld();
          }
        } else {
          tc::tmem_wait_ld();
          if (hf == (qd & 1)) {  // |k_i|^2 sits in column 64 + i, held by this half
            const float rk = rsqrtf(pick_lane(r0, lane) + 1e-6f);
            const float bi = sBeta[i];
            sDk[i] = fast_exp2(misc[M_GLL] - Gli) * rk;
            sT2s[i] = bi * fast_exp2(Gli) * rk;
            sGk[i] = Gli - log2f(rk);
            sGa[i] = Gli + log2f(bi * rk);
          }
        }
        __syncthreads();
      } else {
        tc::tmem_wait_ld();
      }
      const float Gr = qrow ? sGq[i] : sGa[i];
      const int lim = qrow ? i : i - 1;  // last visible column
      const bool above = hf > (qd & 1);  // this warp's columns lie wholly above its rows
      const int blk = i >> 4;
      uint8_t* dst = sm + (qrow ? OFF_P : OFF_A16);
      // (blocks above the diagonal are never read: the products that use P and A skip them)
#pragma unroll
      for (int cl = 0; cl < 4 && !above; ++cl) {
        const int cb = 4 * hf + cl;
        float v8[8];
        {
          const float4 ga = ld4(sGk + cb * 8), gb = ld4(sGk + cb * 8 + 4);
          const float gk[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = cb * 8 + e;
            const float v = r0[cl * 8 + e] * fast_exp2(Gr - gk[e]);
            v8[e] = j <= lim ? v : 0.f;
          }
          if (!qrow && (cb >> 1) == blk) {  // the diagonal 16x16 block, fp32, column-major
            float* ad = sAd + blk * AD_BLK + (cb & 1) * 8 * 16 + (i & 15);
#pragma unroll
            for (int e = 0; e < 8; ++e) ad[e * 16] = v8[e];
          }
        }
        *reinterpret_cast<uint4*>(dst + sw(i, cb)) = pack8<__half>(v8);
      }
    }
    __syncthreads();

    // ---------------- T = (I + A)^-1 -> T1 = T diag(beta), T2 = T diag(beta e^G rk), hi|lo ----------------
    // (1) diagonal 16x16 blocks by right-looking substitution: four adjacent lanes own column j of
    //     block blk (rows q, q + 4, q + 8, q + 12 each), the row that has just become final is shuffled
    //     to them step by step; each thread writes its four rows to T (fp16) and T1, T2 (hi|lo)
    {
      const int blk = tid >> 6, j = (tid >> 2) & 15, q = tid & 3, o = blk * 16;
      const float* ab = sAd + blk * AD_BLK;  // column kk at ab + 16 kk
      float xs[4];                          // rows q, q + 4, q + 8, q + 12 of column j
#pragma unroll
      for (int i = 0; i < 4; ++i) xs[i] = 4 * i + q == j ? 1.f : 0.f;
#pragma unroll
      for (int kk = 0; kk < 15; ++kk) {
        const float xk = __shfl_sync(0xffffffffu, xs[kk >> 2], (lane & ~3) | (kk & 3));  // row kk, now final
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (4 * i + q > kk) xs[i] -= ab[kk * 16 + 4 * i + q] * xk;
      }
      const int col = o + j;
      const float s1 = sBeta[col], s2 = sT2s[col];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = 4 * i + q;
        const uint32_t off = sw_elem(o + r, col);
        *reinterpret_cast<__half*>(sm + OFF_T16 + off) = __float2half_rn(xs[i]);
        const float v1 = xs[i] * s1, v2 = xs[i] * s2;
        const TIn h1 = from_f32<TIn>(v1), h2 = from_f32<TIn>(v2);
        *reinterpret_cast<TIn*>(sm + OFF_T1H + off) = h1;
        *reinterpret_cast<TIn*>(sm + OFF_T1L + off) = from_f32<TIn>(v1 - to_f32(h1));
        *reinterpret_cast<TIn*>(sm + OFF_T2H + off) = h2;
        *reinterpret_cast<TIn*>(sm + OFF_T2L + off) = from_f32<TIn>(v2 - to_f32(h2));
      }
    }
    __syncthreads();
    const int g8 = lane >> 2, t4 = lane & 3;  // mma.sync fragment coordinates
    // (2) 16 -> 32 -> 64 in one pass (warps 0-3; warp = (row half mt, column half nh) of
    //     T[32:64, 0:32]):  Y^T = T[0:32,0:32]^T A[32:64,0:32]^T (rows 16 nh.. of Y^T) and
    //     T[32+16mt.., 16nh..] = -T[32+16mt.., 32:64] Y.  The 16 -> 32 blocks are formed in registers by
    //     the warps that need them: T10 = -T11' (A10 T00') by the warps with nh = 0 (as the transposed
    //     A operand of Y^T, via movmatrix), T32 = -T33' (A32 T22') by the warps with mt = 1 (as the
    //     A operand of the second product).  The zero blocks (0,1), (2,3) of T are skipped, not read.
    if (warp < 4) {
      const int nh = warp & 1, mt = warp >> 1;
      // -T_rr (A_rc T_cc) for the 16x16 block (rr0, cc0), as C fragments
      auto level1 = [&](int rr0, int cc0, float (&c)[2][4]) {
        uint32_t at[4], bA[4], aR[4];
        ldmatrix_x4_trans(at, sm + OFF_T16 + sw(cc0 + (lane & 7) + ((lane >> 4) << 3), (cc0 >> 3) + ((lane >> 3) & 1)));
        ldmatrix_x4(bA, sm + OFF_A16 + sw(rr0 + (lane & 7) + ((lane >> 4) << 3), (cc0 >> 3) + ((lane >> 3) & 1)));
        ldmatrix_x4(aR, sm + OFF_T16 + sw(rr0 + (lane & 15), (rr0 >> 3) + (lane >> 4)));
        float xt[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // X^T = T_cc^T A_rc^T
        mma_16816<__half>(xt[0], at, bA[0], bA[1]);
        mma_16816<__half>(xt[1], at, bA[2], bA[3]);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
          mma_16816<__half>(c[nt], aR, pack2<__half>(xt[0][2 * nt], xt[0][2 * nt + 1]),
                            pack2<__half>(xt[1][2 * nt], xt[1][2 * nt + 1]));
#pragma unroll
          for (int e = 0; e < 4; ++e) c[nt][e] = -c[nt][e];
        }
      };
      // T1, T2 (hi|lo) of the 16x16 block at (r0, c0) from C fragments
      auto store_t12 = [&](const float (&c)[2][4], int r0, int c0) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int col = c0 + 8 * nt + 2 * t4;
          const float s1a = sBeta[col], s1b = sBeta[col + 1], s2a = sT2s[col], s2b = sT2s[col + 1];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float va = c[nt][2 * hh], vb = c[nt][2 * hh + 1];
            const uint32_t off = sw_elem(r0 + g8 + 8 * hh, col);
            uint32_t hi, lo;
            split2<TIn>(va * s1a, vb * s1b, hi, lo);
            *reinterpret_cast<uint32_t*>(sm + OFF_T1H + off) = hi;
            *reinterpret_cast<uint32_t*>(sm + OFF_T1L + off) = lo;
            split2<TIn>(va * s2a, vb * s2b, hi, lo);
            *reinterpret_cast<uint32_t*>(sm + OFF_T2H + off) = hi;
            *reinterpret_cast<uint32_t*>(sm + OFF_T2L + off) = lo;
          }
        }
      };
      // Y^T rows 16 nh..: k-steps over k = rows of T[0:32,0:32] (16 each) against A[32:64,0:32]^T
      float yt[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n) yt[n][0] = yt[n][1] = yt[n][2] = yt[n][3] = 0.f;
      auto y_step = [&](const uint32_t (&aT)[4], int ks) {
#pragma unroll
        for (int ap = 0; ap < 2; ++ap) {
          uint32_t bA[4];
          ldmatrix_x4(bA, sm + OFF_A16 + sw(32 + 16 * ap + (lane & 7) + ((lane >> 4) << 3), 2 * ks + ((lane >> 3) & 1)));
          mma_16816<__half>(yt[2 * ap], aT, bA[0], bA[1]);
          mma_16816<__half>(yt[2 * ap + 1], aT, bA[2], bA[3]);
        }
      };
      if (nh == 0) {
        float t10[2][4];
        level1(16, 0, t10);
        if (mt == 0) store_t12(t10, 16, 0);
        uint32_t at[4];  // k = 0..15: diagonal block 0, transposed
        ldmatrix_x4_trans(at, sm + OFF_T16 + sw((lane & 7) + ((lane >> 4) << 3), (lane >> 3) & 1));
        y_step(at, 0);
        const uint32_t a1[4] = {movmatrix_trans(pack2<__half>(t10[0][0], t10[0][1])),
                                movmatrix_trans(pack2<__half>(t10[1][0], t10[1][1])),
                                movmatrix_trans(pack2<__half>(t10[0][2], t10[0][3])),
                                movmatrix_trans(pack2<__half>(t10[1][2], t10[1][3]))};  // k = 16..31: T10^T
        y_step(a1, 1);
      } else {
        uint32_t at[4];  // k = 0..15: block (0,1) = 0;  k = 16..31: diagonal block 1, transposed
        ldmatrix_x4_trans(at, sm + OFF_T16 + sw(16 + (lane & 7) + ((lane >> 4) << 3), 2 + ((lane >> 3) & 1)));
        y_step(at, 1);
      }
      float o4[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      auto t_step = [&](const uint32_t (&aR)[4], int ks) {  // k = Y rows 16 ks..16 ks + 15
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          mma_16816<__half>(o4[nt], aR, pack2<__half>(yt[2 * ks][2 * nt], yt[2 * ks][2 * nt + 1]),
                            pack2<__half>(yt[2 * ks + 1][2 * nt], yt[2 * ks + 1][2 * nt + 1]));
      };
      if (mt == 0) {
        uint32_t aR[4];  // rows 32-47: diagonal block 2; block (2,3) = 0
        ldmatrix_x4(aR, sm + OFF_T16 + sw(32 + (lane & 15), 4 + (lane >> 4)));
        t_step(aR, 0);
      } else {
        float t32[2][4];
        level1(48, 32, t32);
        if (nh == 1) store_t12(t32, 48, 32);
        const uint32_t a0[4] = {pack2<__half>(t32[0][0], t32[0][1]), pack2<__half>(t32[0][2], t32[0][3]),
                                pack2<__half>(t32[1][0], t32[1][1]), pack2<__half>(t32[1][2], t32[1][3])};
        t_step(a0, 0);
        uint32_t aR[4];  // rows 48-63, k = 16..31: diagonal block 3
        ldmatrix_x4(aR, sm + OFF_T16 + sw(48 + (lane & 15), 6 + (lane >> 4)));
        t_step(aR, 1);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o4[nt][e] = -o4[nt][e];
      store_t12(o4, 32 + 16 * mt, 16 * nh);
    }
    // v of this chunk must have landed before U
    if (!__syncthreads_and(tc::mbar_wait(vb, (uint32_t)(c & 1)))) {
      fail();
      break;
    }
    pending_v = -1;
    sync_smem_for_mma();

    // ---------------- U^T = V^T T1^T ; W^T = K^T T2^T (hi and lo parts) ----------------
    // T1, T2 are lower triangular: k-step s (tokens j in [16 s, 16 s + 16)) only reaches output
    // tokens i >= 16 s, so it runs with N = 64 - 16 s on B rows and D columns from 16 s
    if (tid == 0) {
#pragma unroll
      for (int part = 0; part < 2; ++part) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint32_t id = tc::idesc_f16(128, 64 - 16 * s, true, false, false, kBF);
          const uint64_t av = tc::sdesc_sw128(sbase + OFF_V + s * 2048, T64_BLK, 1024);
          const uint64_t b1 = tc::sdesc_sw128(sbase + (part ? OFF_T1L : OFF_T1H) + s * 2048 + s * 32, 16, 1024);
          tc::mma_f16(tmem + COL_U + 16 * s, av, b1, id, part > 0 || s > 0);
          const uint64_t ak = tc::sdesc_sw128(sbase + OFF_QK + 64 * 128 + s * 2048, QK_BLK, 1024);
          const uint64_t b2 = tc::sdesc_sw128(sbase + (part ? OFF_T2L : OFF_T2H) + s * 2048 + s * 32, 16, 1024);
          tc::mma_f16(tmem + COL_W + 16 * s, ak, b2, id, part > 0 || s > 0);
        }
      }
      tc::commit(bar);
    }
    // meanwhile: S^T columns 0-63 -> the first block of the S^T copy; S^T *= gamma there
    {
      float s32[32];
      tc::tmem_ld32(lane_addr + COL_S + 32 * hf, s32);
      tc::tmem_wait_ld();
#pragma unroll
      for (int cb = 0; cb < 4; ++cb)
        *reinterpret_cast<uint4*>(sm + OFF_SB0 + sw(row, 4 * hf + cb)) = pack8<TIn>(s32 + cb * 8);
      const float gamma = misc[M_GAMMA];
#pragma unroll
      for (int e = 0; e < 32; ++e) s32[e] *= gamma;
      tc::tmem_st32(lane_addr + COL_S + 32 * hf, s32);
      tc::tmem_wait_st();
    }
    if (!sync_mma()) break;
    // v is free: request the next chunk's v tile
    if (c + 1 < nchunks) {
      issue_v(c + 1);
      pending_v = c + 1;
    }

    // ---------------- W^T readout (MN-major operand) and S^T columns 64-127 (copy, then S^T *= gamma) ----------------
    {
      float r0[32];
      tc::tmem_ld32(lane_addr + COL_W + 32 * hf, r0);
      tc::tmem_wait_ld();
#pragma unroll
      for (int cb = 0; cb < 4; ++cb)
        *reinterpret_cast<uint4*>(sm + OFF_W + sw(row, 4 * hf + cb)) = pack8<TIn>(r0 + cb * 8);
      float s32[32];
      tc::tmem_ld32(lane_addr + COL_S + 64 + 32 * hf, s32);
      tc::tmem_wait_ld();
#pragma unroll
      for (int cb = 0; cb < 4; ++cb)
        *reinterpret_cast<uint4*>(sm + OFF_SB1 + sw(row, 4 * hf + cb)) = pack8<TIn>(s32 + cb * 8);
      const float gamma = misc[M_GAMMA];
#pragma unroll
      for (int e = 0; e < 32; ++e) s32[e] *= gamma;
      tc::tmem_st32(lane_addr + COL_S + 64 + 32 * hf, s32);
      tc::tmem_wait_st();
    }
    sync_smem_for_mma();

    // ---------------- Vn^T = U^T - S^T W^T ; O1^T = S^T Q^T ----------------
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint64_t as = tc::sdesc_sw128(sbase + ((s >> 2) ? OFF_SB1 : OFF_SB0) + (s & 3) * 32, 16, 1024);
        const uint64_t bw = tc::sdesc_sw128(sbase + OFF_W + s * 2048, 8192, 1024);
        tc::mma_f16(tmem + COL_U, as, bw, ID_VN, 1);
        const uint64_t bq = tc::sdesc_sw128(sbase + OFF_QK + (s >> 2) * QK_BLK + (s & 3) * 32, 16, 1024);
        tc::mma_f16(tmem + COL_W, as, bq, ID_O1, s > 0);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- Vn readout: Vn (fp16) and the decayed Vn diag(dec rk) (hi|lo) ----------------
    {
      float r0[32];
      tc::tmem_ld32(lane_addr + COL_U + 32 * hf, r0);
      tc::tmem_wait_ld();
#pragma unroll
      for (int cl = 0; cl < 4; ++cl) {
        const int cb = 4 * hf + cl;
        float y[8];
        const float4 d0 = ld4(sDk + cb * 8), d1 = ld4(sDk + cb * 8 + 4);
        const float dd[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = r0[cl * 8 + e] * dd[e];
        *reinterpret_cast<uint4*>(sm + OFF_VN + sw(row, cb)) = pack8<__half>(r0 + cl * 8);
        uint4 hi, lo;
        pack8_hilo<TIn>(y, hi, lo);
        *reinterpret_cast<uint4*>(sm + OFF_DH + sw(row, cb)) = hi;
        *reinterpret_cast<uint4*>(sm + OFF_DL + sw(row, cb)) = lo;
      }
    }
    sync_smem_for_mma();

    // ---------------- O2^T = Vn^T P^T (into U's columns) ; S^T += (dec Vn)^T K (hi and lo) ----------------
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < 4; ++s) {  // P is lower triangular: k-step s reaches tokens i >= 16 s only
        const uint32_t id = tc::idesc_f16(128, 64 - 16 * s, false, false, false, false);
        const uint64_t av = tc::sdesc_sw128(sbase + OFF_VN + s * 32, 16, 1024);
        const uint64_t bp = tc::sdesc_sw128(sbase + OFF_P + s * 2048 + s * 32, 16, 1024);
        tc::mma_f16(tmem + COL_U + 16 * s, av, bp, id, s > 0);
      }
#pragma unroll
      for (int part = 0; part < 2; ++part) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint64_t ad = tc::sdesc_sw128(sbase + (part ? OFF_DL : OFF_DH) + s * 32, 16, 1024);
          const uint64_t bk = tc::sdesc_sw128(sbase + OFF_QK + 64 * 128 + s * 2048, QK_BLK, 1024);
          tc::mma_f16(tmem + COL_S, ad, bk, ID_SU, 1);
        }
      }
      tc::commit(bar);
    }
    float o1[32];  // O1 (untouched by these MMAs) is read while they run
    tc::tmem_ld32(lane_addr + COL_W + 32 * hf, o1);
    tc::tmem_wait_ld();
    if (!sync_mma()) break;
    // q/k are free: start the next chunk's copies while O drains
    if (c + 1 < nchunks) {
      issue_qk(c + 1);
      pending_qk = c + 1;
    }

    // ---------------- O = e^G rq scale O1 + O2 -> global (tokens 32 hf .. 32 hf + 31 of row d_v) ----------------
    {
      float o2[32];
      tc::tmem_ld32(lane_addr + COL_U + 32 * hf, o2);
      tc::tmem_wait_ld();
      float of[32];  // per-token O1 factor e^G rq scale (O2 arrives scaled through P)
#pragma unroll
      for (int q4 = 0; q4 < 8; ++q4) {
        const float4 f = ld4(sOf + 32 * hf + q4 * 4);
        of[q4 * 4] = f.x;
        of[q4 * 4 + 1] = f.y;
        of[q4 * 4 + 2] = f.z;
        of[q4 * 4 + 3] = f.w;
      }
      if constexpr (GATED) {
        // fp32 [token][d_v] staging in R1 (free once the state update has read the decayed Vn); the
        // low three bits of each row's 16-byte chunk index are XORed with the chunk's 32-column
        // quarter and the token's parity, so neither the column writes nor the row reads conflict
        float* ost = reinterpret_cast<float*>(sm + OFF_R1);
        const int cw = row >> 2;
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int tok = 32 * hf + t;
          ost[tok * D + ((cw ^ (((cw >> 3) & 3) ^ ((tok & 1) << 2))) << 2) + (row & 3)] = fmaf(of[t], o1[t], o2[t]);
        }
        __syncthreads();
        // thread (token, quarter): 32 columns of one token; the token's four threads are adjacent lanes
        const int tok = tid >> 2, qq = tid & 3;
        const int swz = qq ^ ((tok & 1) << 2);
        float x[32];
        float ss = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const float4 f = ld4(ost + tok * D + (((8 * qq + kk) ^ swz) << 2));
          x[4 * kk] = f.x;
          x[4 * kk + 1] = f.y;
          x[4 * kk + 2] = f.z;
          x[4 * kk + 3] = f.w;
          ss += f.x * f.x + f.y * f.y + f.z * f.z + f.w * f.w;
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        const float rn = rsqrtf(ss / (float)D + gn.eps);
        if (tok < nvalid) {
          const size_t trow = (size_t)b * T + t0 + tok;
          const size_t obase = (trow * Hv + hv) * D + 32 * qq;
          if (gn.core_out) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              *reinterpret_cast<float4*>(gn.core_out + obase + 4 * kk) =
                  make_float4(x[4 * kk], x[4 * kk + 1], x[4 * kk + 2], x[4 * kk + 3]);
          }
          const TOut* zp = gn.z + (long long)trow * gn.z_ld + (long long)hv * D + 32 * qq;
          const float* wp = gn.w + 32 * qq;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float zf[8], y[8];
            load8(zp + 8 * j, zf);
            const float4 wa = __ldg(reinterpret_cast<const float4*>(wp + 8 * j));
            const float4 wb = __ldg(reinterpret_cast<const float4*>(wp + 8 * j + 4));
            const float wf[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e)
              y[e] = wf[e] * x[8 * j + e] * rn * __fdividef(zf[e], 1.0f + __expf(-zf[e]));
            store8(out + obase + 8 * j, y);
          }
        }
      } else if constexpr (sizeof(TOut) == 2) {
        TOut* ost = reinterpret_cast<TOut*>(sm + OFF_OST);  // [token][d_v] staging
#pragma unroll
        for (int t = 0; t < 32; ++t) ost[(32 * hf + t) * D + row] = from_f32<TOut>(fmaf(of[t], o1[t], o2[t]));
        __syncthreads();
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int idx = tid + it * NT, r = idx >> 4, ch = idx & 15;
          if (r < nvalid)
            *reinterpret_cast<uint4*>(out + (((size_t)b * T + t0 + r) * Hv + hv) * D + ch * 8) =
                *reinterpret_cast<const uint4*>(sm + OFF_OST + r * 256 + ch * 16);
        }
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int tt = 32 * hf + t;
          if (tt < nvalid) out[(((size_t)b * T + t0 + tt) * Hv + hv) * D + row] = fmaf(of[t], o1[t], o2[t]);
        }
      }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  }

  cp_async_wait<0>();
  // a stopped CTA still lets the tiles it requested land before it leaves (bounded)
  if (pending_qk >= 0) tc::mbar_wait(qkb, (uint32_t)(pending_qk & 1));
  if (pending_v >= 0) tc::mbar_wait(vb, (uint32_t)(pending_v & 1));
  // ---- final state ----
  if (!abort_flag) {
    float buf[32];
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int k0 = 64 * hf + 32 * j;
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

// ------------------------------------------------------------------------------------------------
// Pipelined form: one chain per SM, 512 threads in two warp groups, and the next chunk's
// state-independent work (D1, P/A, T, U/W) under the current chunk's state chain.
//   intra group (warps 0-7):  chunk c + 1: D1, gates, P/A readout, T
//   state group (warps 8-15): chunk c:     U/W products, S and W readouts, Vn/O1, Vn readout, O2 and
//                                          the state update, output
// TMEM (512 columns): S^T 0-127, U|W of even chunks 128-255, of odd chunks 256-383, D1 384-511.
// Shared memory: the q/k tiles, P and the state factors (dec rk, the O1 factor, gamma) are
// double-buffered by chunk parity; T1/T2, A/T (fp16) and A's diagonal blocks belong to the intra
// group, the W^T and S^T copies -> Vn and the decayed Vn -> output staging to the state group.
// Hand-offs (mbarriers): chunk c's T1/T2, P, factors and v tile ready (intra -> state, which issues
// the U/W products itself and reads S^T under them); chunk c's U/W products done (their commit: the
// intra group waits for it before it rewrites T1/T2 for chunk c + 1); U|W, P and factors of chunk c
// free again (state -> intra, before chunk c + 2 reuses them).  The v tiles are double-buffered too.  The state group requests
// chunk c + 2's q/k tile as soon as its state update has read k.  The arithmetic is the two-CTA
// kernel's, phase for phase, so both give the same results bit for bit.
constexpr int PT = 512;
constexpr uint32_t PCOL_S = 0, PCOL_UW = 128, PCOL_D1 = 384;
constexpr int PP_QK = 0;                          // [2][2 * QK_BLK]
constexpr int PP_V = 4 * QK_BLK;                  // [2][2 * T64_BLK]
constexpr int PP_P = PP_V + 4 * T64_BLK;          // [2][T64_BLK]
constexpr int PP_T1H = PP_P + 2 * T64_BLK, PP_T1L = PP_T1H + T64_BLK, PP_T2H = PP_T1H + 2 * T64_BLK,
              PP_T2L = PP_T1H + 3 * T64_BLK;
constexpr int PP_A16 = PP_T1H + 4 * T64_BLK, PP_T16 = PP_A16 + T64_BLK;
constexpr int PP_AD = PP_T16 + T64_BLK;
constexpr int PP_ST = (PP_AD + 4 * AD_BLK * 4 + 1023) / 1024 * 1024;  // state group: 48 KB
constexpr int PP_W = PP_ST, PP_SB0 = PP_ST + QK_BLK, PP_SB1 = PP_ST + 2 * QK_BLK;  // before Vn/O1
constexpr int PP_VN = PP_ST, PP_DH = PP_ST + QK_BLK, PP_DL = PP_ST + 2 * QK_BLK;   // before O2/SU
constexpr int PP_OST = PP_ST;                                                      // output staging
constexpr int PP_MISC = PP_ST + 3 * QK_BLK;
// misc (floats): raw g|beta [2][128] | G log2e | beta | T2 column scale | Gk | Gq | Ga | G_c log2e |
// per parity: dec rk [2][64], O1 factor [2][64] | gamma [2]
constexpr int PM2_GB = 0, PM2_GL = 256, PM2_BETA = 320, PM2_T2S = 384, PM2_GK = 448, PM2_GQ = 512, PM2_GA = 576,
              PM2_GLL = 640, PM2_DK = 648, PM2_OF = 776, PM2_GAM = 904;
constexpr int SMEM_PIPE = PP_MISC + 908 * 4 + 1024;
static_assert(PP_ST % 1024 == 0 && PP_P % 1024 == 0 && PP_T1H % 1024 == 0 && PP_A16 % 1024 == 0, "tile alignment");
static_assert(SMEM_PIPE + 1024 <= 227 * 1024, "one pipelined CTA per SM");

// named barriers of one 256-thread group (ids 1 and 2; 0 is __syncthreads)
__device__ __forceinline__ void group_sync(int id) { asm volatile("bar.sync %0, 256;\n" ::"r"(id) : "memory"); }
__device__ __forceinline__ bool group_and(int id, bool v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 256, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((int)v), "r"(id)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

template <typename TIn, typename TOut, bool GATED>
__global__ void __launch_bounds__(PT, 1)
gdn_chunked_pipe_kernel(const __grid_constant__ TileMaps maps, const float* __restrict__ g,
                        const float* __restrict__ beta, float* __restrict__ state, TOut* __restrict__ out, int T,
                        int Hqk, int Hv, float scale, int l2norm, const GatedNorm<TOut> gn) {
  constexpr bool kBF = std::is_same<TIn, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* misc = reinterpret_cast<float*>(sm + PP_MISC);
  float* sGl = misc + PM2_GL;
  float* sBeta = misc + PM2_BETA;
  float* sT2s = misc + PM2_T2S;
  float* sGk = misc + PM2_GK;
  float* sGq = misc + PM2_GQ;
  float* sGa = misc + PM2_GA;
  float* sAd = reinterpret_cast<float*>(sm + PP_AD);
  __shared__ uint64_t qkbar[2], vbar[2], mbarI, mbarS, iready[2], uwdone[2], sfree[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag, qk_issued, qk_done, v_issued, v_done, uw_issued;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool intra = tid < 256;
  const int ti = tid & 255;                 // thread index within its group
  const int gid = intra ? 1 : 2;            // the group's named barrier
  const int qd = warp & 3, hf = (ti >> 5) >> 2;  // TMEM lane quarter, column half
  const int row = ti & 127;                 // the TMEM lane (tile row) this thread reads
  const int bh = blockIdx.x;
  const int b = bh / Hv, hv = bh % Hv;
  const int hk = hv / (Hv / Hqk);
  const uint32_t sbase = tc::smem_u32(sm);
  const int nchunks = (T + C - 1) / C;

  auto issue_qk = [&](int cc) {  // one thread
    const int tok0 = b * T + cc * C;
    const uint32_t bb = tc::smem_u32(&qkbar[cc & 1]);
    const uint32_t qk = sbase + PP_QK + (cc & 1) * 2 * QK_BLK;
    tc::mbar_arrive_expect_tx(bb, QK_TX_BYTES);
    tc::tma_load_3d(qk, &maps.q, 0, hk, tok0, bb);
    tc::tma_load_3d(qk + QK_BLK, &maps.q, 64, hk, tok0, bb);
    tc::tma_load_3d(qk + 64 * 128, &maps.k, 0, hk, tok0, bb);
    tc::tma_load_3d(qk + QK_BLK + 64 * 128, &maps.k, 64, hk, tok0, bb);
    qk_issued = cc;
  };
  auto issue_v = [&](int cc) {  // one thread
    const int tok0 = b * T + cc * C;
    const uint32_t vb = tc::smem_u32(&vbar[cc & 1]);
    const uint32_t vd = sbase + PP_V + (cc & 1) * 2 * T64_BLK;
    tc::mbar_arrive_expect_tx(vb, V_TX_BYTES);
    tc::tma_load_3d(vd, &maps.v, 0, hv, tok0, vb);
    tc::tma_load_3d(vd + T64_BLK, &maps.v, 64, hv, tok0, vb);
    v_issued = cc;
  };
  auto issue_gb = [&](int cc) {  // intra threads 0-127: raw g, beta of chunk cc into its parity's slot
    const int r = ti & 63;
    if (ti < 128 && cc * C + r < T) {
      const size_t idx = ((size_t)b * T + cc * C + r) * Hv + hv;
      cp_async4(misc + PM2_GB + (cc & 1) * 128 + (ti >> 6) * 64 + r, (ti >> 6) ? beta + idx : g + idx);
    }
    cp_async_commit();
  };

  if (tid == 0) {
    tc::mbar_init(&qkbar[0], 1);
    tc::mbar_init(&qkbar[1], 1);
    tc::mbar_init(&vbar[0], 1);
    tc::mbar_init(&vbar[1], 1);
    tc::mbar_init(&mbarI, 1);
    tc::mbar_init(&mbarS, 1);
    tc::mbar_init(&iready[0], 1);
    tc::mbar_init(&iready[1], 1);
    tc::mbar_init(&uwdone[0], 1);
    tc::mbar_init(&uwdone[1], 1);
    tc::mbar_init(&sfree[0], 1);
    tc::mbar_init(&sfree[1], 1);
    tc::fence_mbar_init();
    abort_flag = 0;
    qk_issued = qk_done = v_issued = v_done = uw_issued = -1;
  }
  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (tid == 0) {
    issue_qk(0);
    if (nchunks > 1) issue_qk(1);
    issue_v(0);
    if (nchunks > 1) issue_v(1);
  }
  if (intra) issue_gb(0);
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);  // this warp's TMEM lane quarter
  float* Sg = state + (size_t)bh * D * D;
  if (!intra) {  // ---- initial state: thread (row d, half hf) holds S[64 hf .. 64 hf + 63][d] ----
    float buf[32];
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int k0 = 64 * hf + 32 * j;
#pragma unroll
      for (int i = 0; i < 32; ++i) buf[i] = Sg[(size_t)(k0 + i) * D + row];
      tc::tmem_st32(lane_addr + PCOL_S + k0, buf);
    }
    tc::tmem_wait_st();
  }
  auto fail = [&]() {
    atomicExch(&g_chunked_error, 1);
    abort_flag = 1;
  };
  uint32_t phase = 0;  // this group's MMA barrier phase
  const uint32_t mbar = tc::smem_u32(intra ? &mbarI : &mbarS);
  auto sync_mma = [&]() -> bool {
    const bool ok = group_and(gid, tc::mbar_wait(mbar, phase));  // group-uniform outcome
    phase ^= 1u;
    if (!ok) fail();
    tc::fence_after();
    return ok;
  };
  auto sync_smem_for_mma = [&]() {
    tc::fence_async_smem();
    tc::fence_before();
    group_sync(gid);
    tc::fence_after();
  };
  constexpr uint32_t ID_D1 = tc::idesc_f16(128, 128, false, false, false, kBF);
  constexpr uint32_t ID_VN = tc::idesc_f16(128, 64, false, true, true, kBF);
  constexpr uint32_t ID_O1 = tc::idesc_f16(128, 64, false, false, false, kBF);
  constexpr uint32_t ID_SU = tc::idesc_f16(128, 128, false, true, false, kBF);

  if (intra) {
    // ================= intra group: chunk c's state-independent work =================
#pragma unroll 1
    for (int c = 0; c < nchunks && !abort_flag; ++c) {
      const int buf = c & 1;
      const int t0 = c * C;
      const int nvalid = min(C, T - t0);
      const uint32_t col_u = PCOL_UW + 128u * (uint32_t)buf;
      float* sGB = misc + PM2_GB + buf * 128;
      float* sDk = misc + PM2_DK + buf * 64;
      float* sOf = misc + PM2_OF + buf * 64;
      // the q/k tile of this chunk; its raw g, beta (requested a chunk ahead)
      if (!group_and(1, tc::mbar_wait(tc::smem_u32(&qkbar[buf]), (uint32_t)((c >> 1) & 1)))) {
        fail();
        break;
      }
      if (ti == 0) qk_done = c;
      cp_async_wait<0>();
      if (c + 1 < nchunks) issue_gb(c + 1);
      // U|W, P and the factors of this parity are free once chunk c - 2's state chain has read them
      if (c >= 2 && !group_and(1, tc::mbar_wait(tc::smem_u32(&sfree[buf]), (uint32_t)(((c - 2) >> 1) & 1)))) {
        fail();
        break;
      }
      // ---------------- D1 = [Q;K] [Q;K]^T (issued before the gates are formed) ----------------
      if (ti == 0) {
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t koff = (uint32_t)((s >> 2) * QK_BLK + (s & 3) * 32);
          const uint64_t d = tc::sdesc_sw128(sbase + (PP_QK + buf * 2 * QK_BLK) + koff, 16, 1024);
          tc::mma_f16(tmem + PCOL_D1, d, d, ID_D1, s > 0);
        }
        tc::commit(mbar);
      }
      group_sync(1);  // raw g / beta of every thread visible
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
        constexpr float L2E = 1.4426950408889634f;
        const float Gl1 = s * L2E, Gl0 = (s - g1) * L2E;
        const float Gll = __shfl_sync(0xffffffffu, Gl1, 31);
        sGl[i0] = Gl0;
        sGl[i1] = Gl1;
        sBeta[i0] = b0;
        sBeta[i1] = b1;
        if (lane == 0) {
          misc[PM2_GAM + buf] = fast_exp2(Gll);
          misc[PM2_GLL] = Gll;
        }
        if (!l2norm) {  // rq = rk = 1
          const float e0 = fast_exp2(Gl0), e1 = fast_exp2(Gl1), d0 = fast_exp2(Gll - Gl0), d1 = fast_exp2(Gll - Gl1);
          const float ls = log2f(scale);
          sDk[i0] = d0;
          sDk[i1] = d1;
          sOf[i0] = e0 * scale;
          sOf[i1] = e1 * scale;
          sT2s[i0] = b0 * e0;
          sT2s[i1] = b1 * e1;
          sGk[i0] = Gl0;
          sGk[i1] = Gl1;
          sGq[i0] = Gl0 + ls;
          sGq[i1] = Gl1 + ls;
          sGa[i0] = Gl0 + log2f(b0);
          sGa[i1] = Gl1 + log2f(b1);
        }
      }
      if (!sync_mma()) break;  // D1 done; gates visible
      // ---------------- P (rows 0-63), A (rows 64-127) ----------------
      // P_ij = x_ij 2^(Gq_i - Gk_j) (j <= i), A_ij = x_ij 2^(Ga_i - Gk_j) (j < i): the norms, beta and the
      // attention scale ride in the log2 row / column factors
      {
        const bool qrow = row < 64;
        const int i = row & 63;
        float r0[32];  // D1 columns 64 + 32 hf ..: row . k_j for j in [32 hf, 32 hf + 32)
        tc::tmem_ld32(lane_addr + PCOL_D1 + 64 + 32 * hf, r0);
        if (l2norm) {
          const float Gli = sGl[i];
          if (qrow) {
            if (hf == 0) {  // |q_i|^2 sits in column i of the QQ^T block
              float rd[32];
              tc::tmem_ld32(lane_addr + PCOL_D1 + (qd & 1) * 32, rd);
              tc::tmem_wait_ld();
              const float rq = rsqrtf(pick_lane(rd, lane) + 1e-6f);
              sOf[i] = fast_exp2(Gli) * rq * scale;
              sGq[i] = Gli + log2f(rq * scale);
            } else {
              tc::tmem_wait_ld();
            }
          } else {
            tc::tmem_wait_ld();
            if (hf == (qd & 1)) {  // |k_i|^2 sits in column 64 + i, held by this half
              const float rk = rsqrtf(pick_lane(r0, lane) + 1e-6f);
              const float bi = sBeta[i];
              sDk[i] = fast_exp2(misc[PM2_GLL] - Gli) * rk;
              sT2s[i] = bi * fast_exp2(Gli) * rk;
              sGk[i] = Gli - log2f(rk);
              sGa[i] = Gli + log2f(bi * rk);
            }
          }
          group_sync(1);
        } else {
          tc::tmem_wait_ld();
        }
        const float Gr = qrow ? sGq[i] : sGa[i];
        const int lim = qrow ? i : i - 1;  // last visible column
        const bool above = hf > (qd & 1);  // this warp's columns lie wholly above its rows
        const int blk = i >> 4;
        uint8_t* dst = sm + (qrow ? (PP_P + buf * T64_BLK) : PP_A16);
        // (blocks above the diagonal are never read: the products that use P and A skip them)
#pragma unroll
        for (int cl = 0; cl < 4 && !above; ++cl) {
          const int cb = 4 * hf + cl;
          float v8[8];
          {
            const float4 ga = ld4(sGk + cb * 8), gb = ld4(sGk + cb * 8 + 4);
            const float gk[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int j = cb * 8 + e;
              const float v = r0[cl * 8 + e] * fast_exp2(Gr - gk[e]);
              v8[e] = j <= lim ? v : 0.f;
            }
            if (!qrow && (cb >> 1) == blk) {  // the diagonal 16x16 block, fp32, column-major
              float* ad = sAd + blk * AD_BLK + (cb & 1) * 8 * 16 + (i & 15);
#pragma unroll
              for (int e = 0; e < 8; ++e) ad[e * 16] = v8[e];
            }
          }
          *reinterpret_cast<uint4*>(dst + sw(i, cb)) = pack8<__half>(v8);
        }
      }
      group_sync(1);

      // chunk c - 1's U/W products (the state group issues them) have read T1/T2 and their v tile:
      // request chunk c + 1's v there
      if (c >= 1) {
        if (!group_and(1, tc::mbar_wait(tc::smem_u32(&uwdone[buf ^ 1]), (uint32_t)(((c - 1) >> 1) & 1)))) {
          fail();
          break;
        }
        if (ti == 0 && c + 1 < nchunks) issue_v(c + 1);
      }
      // ---------------- T = (I + A)^-1 -> T1 = T diag(beta), T2 = T diag(beta e^G rk), hi|lo ----------------
      // (1) threads 0-63: diagonal 16x16 blocks, thread (blk, j) solves column j by right-looking
      //     substitution and writes it to T (fp16) and T1, T2 (hi|lo)
      {
        const int blk = ti >> 6, j = (ti >> 2) & 15, q = ti & 3, o = blk * 16;
        const float* ab = sAd + blk * AD_BLK;  // column kk at ab + 16 kk
        float xs[4];                          // rows q, q + 4, q + 8, q + 12 of column j
#pragma unroll
        for (int i = 0; i < 4; ++i) xs[i] = 4 * i + q == j ? 1.f : 0.f;
#pragma unroll
        for (int kk = 0; kk < 15; ++kk) {
          const float xk = __shfl_sync(0xffffffffu, xs[kk >> 2], (lane & ~3) | (kk & 3));  // row kk, now final
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (4 * i + q > kk) xs[i] -= ab[kk * 16 + 4 * i + q] * xk;
        }
        const int col = o + j;
        const float s1 = sBeta[col], s2 = sT2s[col];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = 4 * i + q;
          const uint32_t off = sw_elem(o + r, col);
          *reinterpret_cast<__half*>(sm + PP_T16 + off) = __float2half_rn(xs[i]);
          const float v1 = xs[i] * s1, v2 = xs[i] * s2;
          const TIn h1 = from_f32<TIn>(v1), h2 = from_f32<TIn>(v2);
          *reinterpret_cast<TIn*>(sm + PP_T1H + off) = h1;
          *reinterpret_cast<TIn*>(sm + PP_T1L + off) = from_f32<TIn>(v1 - to_f32(h1));
          *reinterpret_cast<TIn*>(sm + PP_T2H + off) = h2;
          *reinterpret_cast<TIn*>(sm + PP_T2L + off) = from_f32<TIn>(v2 - to_f32(h2));
        }
      }
      group_sync(1);
      const int g8 = lane >> 2, t4 = lane & 3;  // mma.sync fragment coordinates
      // (2) 16 -> 32 -> 64 in one pass (warps 0-3; warp = (row half mt, column half nh) of
      //     T[32:64, 0:32]):  Y^T = T[0:32,0:32]^T A[32:64,0:32]^T (rows 16 nh.. of Y^T) and
      //     T[32+16mt.., 16nh..] = -T[32+16mt.., 32:64] Y.  The 16 -> 32 blocks are formed in registers by
      //     the warps that need them: T10 = -T11' (A10 T00') by the warps with nh = 0 (as the transposed
      //     A operand of Y^T, via movmatrix), T32 = -T33' (A32 T22') by the warps with mt = 1 (as the
      //     A operand of the second product).  The zero blocks (0,1), (2,3) of T are skipped, not read.
      if (warp < 4) {
        const int nh = warp & 1, mt = warp >> 1;
        // -T_rr (A_rc T_cc) for the 16x16 block (rr0, cc0), as C fragments
        auto level1 = [&](int rr0, int cc0, float (&c)[2][4]) {
          uint32_t at[4], bA[4], aR[4];
          ldmatrix_x4_trans(at, sm + PP_T16 + sw(cc0 + (lane & 7) + ((lane >> 4) << 3), (cc0 >> 3) + ((lane >> 3) & 1)));
          ldmatrix_x4(bA, sm + PP_A16 + sw(rr0 + (lane & 7) + ((lane >> 4) << 3), (cc0 >> 3) + ((lane >> 3) & 1)));
          ldmatrix_x4(aR, sm + PP_T16 + sw(rr0 + (lane & 15), (rr0 >> 3) + (lane >> 4)));
          float xt[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // X^T = T_cc^T A_rc^T
          mma_16816<__half>(xt[0], at, bA[0], bA[1]);
          mma_16816<__half>(xt[1], at, bA[2], bA[3]);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
            mma_16816<__half>(c[nt], aR, pack2<__half>(xt[0][2 * nt], xt[0][2 * nt + 1]),
                              pack2<__half>(xt[1][2 * nt], xt[1][2 * nt + 1]));
#pragma unroll
            for (int e = 0; e < 4; ++e) c[nt][e] = -c[nt][e];
          }
        };
        // T1, T2 (hi|lo) of the 16x16 block at (r0, c0) from C fragments
        auto store_t12 = [&](const float (&c)[2][4], int r0, int c0) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int col = c0 + 8 * nt + 2 * t4;
            const float s1a = sBeta[col], s1b = sBeta[col + 1], s2a = sT2s[col], s2b = sT2s[col + 1];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float va = c[nt][2 * hh], vb = c[nt][2 * hh + 1];
              const uint32_t off = sw_elem(r0 + g8 + 8 * hh, col);
              uint32_t hi, lo;
              split2<TIn>(va * s1a, vb * s1b, hi, lo);
              *reinterpret_cast<uint32_t*>(sm + PP_T1H + off) = hi;
              *reinterpret_cast<uint32_t*>(sm + PP_T1L + off) = lo;
              split2<TIn>(va * s2a, vb * s2b, hi, lo);
              *reinterpret_cast<uint32_t*>(sm + PP_T2H + off) = hi;
              *reinterpret_cast<uint32_t*>(sm + PP_T2L + off) = lo;
            }
          }
        };
        // Y^T rows 16 nh..: k-steps over k = rows of T[0:32,0:32] (16 each) against A[32:64,0:32]^T
        float yt[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n) yt[n][0] = yt[n][1] = yt[n][2] = yt[n][3] = 0.f;
        auto y_step = [&](const uint32_t (&aT)[4], int ks) {
#pragma unroll
          for (int ap = 0; ap < 2; ++ap) {
            uint32_t bA[4];
            ldmatrix_x4(bA, sm + PP_A16 + sw(32 + 16 * ap + (lane & 7) + ((lane >> 4) << 3), 2 * ks + ((lane >> 3) & 1)));
            mma_16816<__half>(yt[2 * ap], aT, bA[0], bA[1]);
            mma_16816<__half>(yt[2 * ap + 1], aT, bA[2], bA[3]);
          }
        };
        if (nh == 0) {
          float t10[2][4];
          level1(16, 0, t10);
          if (mt == 0) store_t12(t10, 16, 0);
          uint32_t at[4];  // k = 0..15: diagonal block 0, transposed
          ldmatrix_x4_trans(at, sm + PP_T16 + sw((lane & 7) + ((lane >> 4) << 3), (lane >> 3) & 1));
          y_step(at, 0);
          const uint32_t a1[4] = {movmatrix_trans(pack2<__half>(t10[0][0], t10[0][1])),
                                  movmatrix_trans(pack2<__half>(t10[1][0], t10[1][1])),
                                  movmatrix_trans(pack2<__half>(t10[0][2], t10[0][3])),
                                  movmatrix_trans(pack2<__half>(t10[1][2], t10[1][3]))};  // k = 16..31: T10^T
          y_step(a1, 1);
        } else {
          uint32_t at[4];  // k = 0..15: block (0,1) = 0;  k = 16..31: diagonal block 1, transposed
          ldmatrix_x4_trans(at, sm + PP_T16 + sw(16 + (lane & 7) + ((lane >> 4) << 3), 2 + ((lane >> 3) & 1)));
          y_step(at, 1);
        }
        float o4[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        auto t_step = [&](const uint32_t (&aR)[4], int ks) {  // k = Y rows 16 ks..16 ks + 15
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
            mma_16816<__half>(o4[nt], aR, pack2<__half>(yt[2 * ks][2 * nt], yt[2 * ks][2 * nt + 1]),
                              pack2<__half>(yt[2 * ks + 1][2 * nt], yt[2 * ks + 1][2 * nt + 1]));
        };
        if (mt == 0) {
          uint32_t aR[4];  // rows 32-47: diagonal block 2; block (2,3) = 0
          ldmatrix_x4(aR, sm + PP_T16 + sw(32 + (lane & 15), 4 + (lane >> 4)));
          t_step(aR, 0);
        } else {
          float t32[2][4];
          level1(48, 32, t32);
          if (nh == 1) store_t12(t32, 48, 32);
          const uint32_t a0[4] = {pack2<__half>(t32[0][0], t32[0][1]), pack2<__half>(t32[0][2], t32[0][3]),
                                  pack2<__half>(t32[1][0], t32[1][1]), pack2<__half>(t32[1][2], t32[1][3])};
          t_step(a0, 0);
          uint32_t aR[4];  // rows 48-63, k = 16..31: diagonal block 3
          ldmatrix_x4(aR, sm + PP_T16 + sw(48 + (lane & 15), 6 + (lane >> 4)));
          t_step(aR, 1);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) o4[nt][e] = -o4[nt][e];
        store_t12(o4, 32 + 16 * mt, 16 * nh);
      }

      // v of this chunk must have landed before U
      if (!group_and(1, tc::mbar_wait(tc::smem_u32(&vbar[buf]), (uint32_t)((c >> 1) & 1)))) {
        fail();
        break;
      }
      if (ti == 0) v_done = c;
      tc::fence_async_smem();  // T1/T2 and P are operands of the state group's products
      // chunk c's T1/T2, P, factors and v tile are ready for the state group
      tc::fence_before();
      group_sync(1);
      if (ti == 0) mbar_arrive(tc::smem_u32(&iready[buf]));
    }
  } else {
    // ================= state group: chunk c's state chain and output =================
#pragma unroll 1
    for (int c = 0; c < nchunks && !abort_flag; ++c) {
      const int buf = c & 1;
      const int t0 = c * C;
      const int nvalid = min(C, T - t0);
      const uint32_t col_u = PCOL_UW + 128u * (uint32_t)buf;
      const float* sDk = misc + PM2_DK + buf * 64;
      const float* sOf = misc + PM2_OF + buf * 64;
      if (!group_and(2, tc::mbar_wait(tc::smem_u32(&iready[buf]), (uint32_t)((c >> 1) & 1)))) {
        fail();
        break;
      }
      tc::fence_after();
      // ---------------- U^T = V^T T1^T ; W^T = K^T T2^T (hi and lo parts) ----------------
      // T1, T2 are lower triangular: k-step s (tokens j in [16 s, 16 s + 16)) only reaches output
      // tokens i >= 16 s, so it runs with N = 64 - 16 s on B rows and D columns from 16 s
      if (ti == 0) {
#pragma unroll
        for (int part = 0; part < 2; ++part) {
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint32_t id = tc::idesc_f16(128, 64 - 16 * s, true, false, false, kBF);
            const uint64_t av = tc::sdesc_sw128(sbase + PP_V + buf * 2 * T64_BLK + s * 2048, T64_BLK, 1024);
            const uint64_t b1 = tc::sdesc_sw128(sbase + (part ? PP_T1L : PP_T1H) + s * 2048 + s * 32, 16, 1024);
            tc::mma_f16(tmem + col_u + 16 * s, av, b1, id, part > 0 || s > 0);
            const uint64_t ak = tc::sdesc_sw128(sbase + (PP_QK + buf * 2 * QK_BLK) + 64 * 128 + s * 2048, QK_BLK, 1024);
            const uint64_t b2 = tc::sdesc_sw128(sbase + (part ? PP_T2L : PP_T2H) + s * 2048 + s * 32, 16, 1024);
            tc::mma_f16(tmem + col_u + 64 + 16 * s, ak, b2, id, part > 0 || s > 0);
          }
        }
        tc::commit(tc::smem_u32(&uwdone[buf]));
        uw_issued = c;
      }

      // ---------------- meanwhile: S^T -> the S^T copy (S^T *= gamma in TMEM) ----------------
      {
        const float gamma = misc[PM2_GAM + buf];
        float s32[32];
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          tc::tmem_ld32(lane_addr + PCOL_S + 64 * hh + 32 * hf, s32);
          tc::tmem_wait_ld();
#pragma unroll
          for (int cb = 0; cb < 4; ++cb)
            *reinterpret_cast<uint4*>(sm + (hh ? PP_SB1 : PP_SB0) + sw(row, 4 * hf + cb)) = pack8<TIn>(s32 + cb * 8);
#pragma unroll
          for (int e = 0; e < 32; ++e) s32[e] *= gamma;
          tc::tmem_st32(lane_addr + PCOL_S + 64 * hh + 32 * hf, s32);
        }
        tc::tmem_wait_st();
      }
      // ---------------- W^T readout (MN-major operand) once the U/W products are done ----------------
      if (!group_and(2, tc::mbar_wait(tc::smem_u32(&uwdone[buf]), (uint32_t)((c >> 1) & 1)))) {
        fail();
        break;
      }
      tc::fence_after();
      {
        float r0[32];
        tc::tmem_ld32(lane_addr + col_u + 64 + 32 * hf, r0);
        tc::tmem_wait_ld();
#pragma unroll
        for (int cb = 0; cb < 4; ++cb)
          *reinterpret_cast<uint4*>(sm + PP_W + sw(row, 4 * hf + cb)) = pack8<TIn>(r0 + cb * 8);
      }
      sync_smem_for_mma();

      // ---------------- Vn^T = U^T - S^T W^T ; O1^T = S^T Q^T ----------------
      if (ti == 0) {
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint64_t as = tc::sdesc_sw128(sbase + ((s >> 2) ? PP_SB1 : PP_SB0) + (s & 3) * 32, 16, 1024);
          const uint64_t bw = tc::sdesc_sw128(sbase + PP_W + s * 2048, 8192, 1024);
          tc::mma_f16(tmem + col_u, as, bw, ID_VN, 1);
          const uint64_t bq = tc::sdesc_sw128(sbase + (PP_QK + buf * 2 * QK_BLK) + (s >> 2) * QK_BLK + (s & 3) * 32, 16, 1024);
          tc::mma_f16(tmem + col_u + 64, as, bq, ID_O1, s > 0);
        }
        tc::commit(mbar);
      }
      if (!sync_mma()) break;

      // ---------------- Vn readout: Vn (fp16) and the decayed Vn diag(dec rk) (hi|lo) ----------------
      {
        float r0[32];
        tc::tmem_ld32(lane_addr + col_u + 32 * hf, r0);
        tc::tmem_wait_ld();
#pragma unroll
        for (int cl = 0; cl < 4; ++cl) {
          const int cb = 4 * hf + cl;
          float y[8];
          const float4 d0 = ld4(sDk + cb * 8), d1 = ld4(sDk + cb * 8 + 4);
          const float dd[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = r0[cl * 8 + e] * dd[e];
          *reinterpret_cast<uint4*>(sm + PP_VN + sw(row, cb)) = pack8<__half>(r0 + cl * 8);
          uint4 hi, lo;
          pack8_hilo<TIn>(y, hi, lo);
          *reinterpret_cast<uint4*>(sm + PP_DH + sw(row, cb)) = hi;
          *reinterpret_cast<uint4*>(sm + PP_DL + sw(row, cb)) = lo;
        }
      }
      sync_smem_for_mma();

      // ---------------- O2^T = Vn^T P^T (into U's columns) ; S^T += (dec Vn)^T K (hi and lo) ----------------
      if (ti == 0) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {  // P is lower triangular: k-step s reaches tokens i >= 16 s only
          const uint32_t id = tc::idesc_f16(128, 64 - 16 * s, false, false, false, false);
          const uint64_t av = tc::sdesc_sw128(sbase + PP_VN + s * 32, 16, 1024);
          const uint64_t bp = tc::sdesc_sw128(sbase + (PP_P + buf * T64_BLK) + s * 2048 + s * 32, 16, 1024);
          tc::mma_f16(tmem + col_u + 16 * s, av, bp, id, s > 0);
        }
#pragma unroll
        for (int part = 0; part < 2; ++part) {
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint64_t ad = tc::sdesc_sw128(sbase + (part ? PP_DL : PP_DH) + s * 32, 16, 1024);
            const uint64_t bk = tc::sdesc_sw128(sbase + (PP_QK + buf * 2 * QK_BLK) + 64 * 128 + s * 2048, QK_BLK, 1024);
            tc::mma_f16(tmem + PCOL_S, ad, bk, ID_SU, 1);
          }
        }
        tc::commit(mbar);
      }
      float o1[32];  // O1 (untouched by these MMAs) is read while they run
      tc::tmem_ld32(lane_addr + col_u + 64 + 32 * hf, o1);
      tc::tmem_wait_ld();
      if (!sync_mma()) break;

      // q/k of this chunk are free: request chunk c + 2's tile into this parity's buffer
      if (ti == 0 && c + 2 < nchunks) issue_qk(c + 2);
      // ---------------- O = e^G rq scale O1 + O2 -> global (tokens 32 hf .. 32 hf + 31 of row d_v) ----------------
      {
        float o2[32];
        tc::tmem_ld32(lane_addr + col_u + 32 * hf, o2);
        tc::tmem_wait_ld();
        float of[32];  // per-token O1 factor e^G rq scale (O2 arrives scaled through P)
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          const float4 f = ld4(sOf + 32 * hf + q4 * 4);
          of[q4 * 4] = f.x;
          of[q4 * 4 + 1] = f.y;
          of[q4 * 4 + 2] = f.z;
          of[q4 * 4 + 3] = f.w;
        }
        // this chunk's U|W, P and factors are no longer read: chunk c + 2 may reuse them
        tc::fence_before();
        group_sync(2);
        if (ti == 0) mbar_arrive(tc::smem_u32(&sfree[buf]));
      if constexpr (GATED) {
        // fp32 [token][d_v] staging in R1 (free once the state update has read the decayed Vn); the
        // low three bits of each row's 16-byte chunk index are XORed with the chunk's 32-column
        // quarter and the token's parity, so neither the column writes nor the row reads conflict
        float* ost = reinterpret_cast<float*>(sm + PP_OST);
        const int cw = row >> 2;
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int tok = 32 * hf + t;
          ost[tok * D + ((cw ^ (((cw >> 3) & 3) ^ ((tok & 1) << 2))) << 2) + (row & 3)] = fmaf(of[t], o1[t], o2[t]);
        }
        group_sync(2);
        // thread (token, quarter): 32 columns of one token; the token's four threads are adjacent lanes
        const int tok = ti >> 2, qq = ti & 3;
        const int swz = qq ^ ((tok & 1) << 2);
        float x[32];
        float ss = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const float4 f = ld4(ost + tok * D + (((8 * qq + kk) ^ swz) << 2));
          x[4 * kk] = f.x;
          x[4 * kk + 1] = f.y;
          x[4 * kk + 2] = f.z;
          x[4 * kk + 3] = f.w;
          ss += f.x * f.x + f.y * f.y + f.z * f.z + f.w * f.w;
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        const float rn = rsqrtf(ss / (float)D + gn.eps);
        if (tok < nvalid) {
          const size_t trow = (size_t)b * T + t0 + tok;
          const size_t obase = (trow * Hv + hv) * D + 32 * qq;
          if (gn.core_out) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              *reinterpret_cast<float4*>(gn.core_out + obase + 4 * kk) =
                  make_float4(x[4 * kk], x[4 * kk + 1], x[4 * kk + 2], x[4 * kk + 3]);
          }
          const TOut* zp = gn.z + (long long)trow * gn.z_ld + (long long)hv * D + 32 * qq;
          const float* wp = gn.w + 32 * qq;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float zf[8], y[8];
            load8(zp + 8 * j, zf);
            const float4 wa = __ldg(reinterpret_cast<const float4*>(wp + 8 * j));
            const float4 wb = __ldg(reinterpret_cast<const float4*>(wp + 8 * j + 4));
            const float wf[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e)
              y[e] = wf[e] * x[8 * j + e] * rn * __fdividef(zf[e], 1.0f + __expf(-zf[e]));
            store8(out + obase + 8 * j, y);
          }
        }
      } else if constexpr (sizeof(TOut) == 2) {
        TOut* ost = reinterpret_cast<TOut*>(sm + PP_OST);  // [token][d_v] staging
#pragma unroll
        for (int t = 0; t < 32; ++t) ost[(32 * hf + t) * D + row] = from_f32<TOut>(fmaf(of[t], o1[t], o2[t]));
        group_sync(2);
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int idx = ti + it * NT, r = idx >> 4, ch = idx & 15;
          if (r < nvalid)
            *reinterpret_cast<uint4*>(out + (((size_t)b * T + t0 + r) * Hv + hv) * D + ch * 8) =
                *reinterpret_cast<const uint4*>(sm + PP_OST + r * 256 + ch * 16);
        }
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int tt = 32 * hf + t;
          if (tt < nvalid) out[(((size_t)b * T + t0 + tt) * Hv + hv) * D + row] = fmaf(of[t], o1[t], o2[t]);
        }
      }
    }
      tc::fence_before();
      group_sync(2);
      tc::fence_after();
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // both groups have left their loops
  if (tid == 0) {
    // loads still in flight after a stopped run land before the CTA leaves (bounded waits)
    for (int cc = qk_done + 1; cc <= qk_issued; ++cc)
      tc::mbar_wait(tc::smem_u32(&qkbar[cc & 1]), (uint32_t)((cc >> 1) & 1));
    for (int cc = v_done + 1; cc <= v_issued; ++cc)
      tc::mbar_wait(tc::smem_u32(&vbar[cc & 1]), (uint32_t)((cc >> 1) & 1));
    // U/W products of a stopped run complete before TMEM is released
    if (abort_flag && uw_issued >= 0)
      tc::mbar_wait(tc::smem_u32(&uwdone[uw_issued & 1]), (uint32_t)((uw_issued >> 1) & 1));
  }
  // ---- final state (state group) ----
  if (!intra && !abort_flag) {
    float buf32[32];
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int k0 = 64 * hf + 32 * j;
      tc::tmem_ld32(lane_addr + PCOL_S + k0, buf32);
      tc::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) Sg[(size_t)(k0 + i) * D + row] = buf32[i];
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
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

// The pipelined form runs one chain per SM: it is used while the chains fit one wave of SMs; beyond
// that two chains per SM (the two-CTA kernel) hide more of each chain's latency.
static int g_pipe_mode = 0;  // 0: by chain count, 1: always pipelined, 2: never
bool use_pipelined(int chains) {
  if (g_pipe_mode) return g_pipe_mode == 1;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return chains <= sms;
}

template <typename TIn, typename TOut, bool GATED>
int launch_chunked(const void* q, const void* k, const void* v, const float* g, const float* beta, float* state,
                   void* out, int B, int T, int Hqk, int Hv, float scale, int l2norm, const GatedNorm<TOut>& gn,
                   cudaStream_t st) {
  TileMaps maps;
  const long long tokens = (long long)B * T;
  int rc = encode_rows_map(&maps.q, q, Hqk, tokens);
  if (!rc) rc = encode_rows_map(&maps.k, k, Hqk, tokens);
  if (!rc) rc = encode_rows_map(&maps.v, v, Hv, tokens);
  if (rc) return rc;
  if (use_pipelined(B * Hv)) {
    auto kern = gdn_chunked_pipe_kernel<TIn, TOut, GATED>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_PIPE);
    kern<<<B * Hv, PT, SMEM_PIPE, st>>>(maps, g, beta, state, (TOut*)out, T, Hqk, Hv, scale, l2norm, gn);
  } else {
    auto kern = gdn_chunked_kernel<TIn, TOut, GATED>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    kern<<<B * Hv, NT, SMEM_BYTES, st>>>(maps, g, beta, state, (TOut*)out, T, Hqk, Hv, scale, l2norm, gn);
  }
  return launch_status(GATED ? "gdn_chunked_prefill_gated" : "gdn_chunked_prefill");
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
      const GatedNorm<TOut> none{nullptr, 0, nullptr, 0.f, nullptr};
      return launch_chunked<TIn, TOut, false>(q, k, v, g, beta, state, out, B, T, H_qk, H_v, scale, qk_l2norm, none,
                                              st);
    });
  });
}

extern "C" int anemll_gdn_chunked_prefill_gated(const void* q, const void* k, const void* v, int qkv_dtype,
                                                const float* g, const float* beta, float* state,
                                                const void* z, int64_t z_row_stride, const float* norm_weight,
                                                float eps, void* out, int out_dtype, float* core_out,
                                                int B, int T, int H_qk, int H_v, int d_k, int d_v,
                                                int chunk_size, float scale, int qk_l2norm, void* stream) {
  ANEMLL_REQUIRE(state && (T == 0 || (q && k && v && g && beta && z && norm_weight && out)), ANEMLL_EINVAL,
                 "gdn_chunked_prefill_gated: null pointer");
  ANEMLL_REQUIRE(B > 0 && T >= 0 && H_qk > 0 && H_v > 0 && H_v % H_qk == 0, ANEMLL_EINVAL,
                 "gdn_chunked_prefill_gated: bad sizes B=%d T=%d H_qk=%d H_v=%d", B, T, H_qk, H_v);
  ANEMLL_REQUIRE(d_k == D && d_v == D, ANEMLL_EUNSUPPORTED, "gdn_chunked_prefill_gated: d_k and d_v must be 128");
  ANEMLL_REQUIRE(chunk_size == C, ANEMLL_EUNSUPPORTED, "gdn_chunked_prefill_gated: chunk_size must be 64");
  ANEMLL_REQUIRE(qkv_dtype == ANEMLL_F16 || qkv_dtype == ANEMLL_BF16, ANEMLL_EUNSUPPORTED,
                 "gdn_chunked_prefill_gated: q/k/v must be f16 or bf16");
  ANEMLL_REQUIRE(out_dtype == ANEMLL_F16 || out_dtype == ANEMLL_BF16, ANEMLL_EUNSUPPORTED,
                 "gdn_chunked_prefill_gated: out (and z) must be f16 or bf16");
  if (z_row_stride == 0) z_row_stride = (int64_t)H_v * d_v;
  ANEMLL_REQUIRE(z_row_stride >= (int64_t)H_v * d_v, ANEMLL_EINVAL,
                 "gdn_chunked_prefill_gated: z row stride shorter than H_v * d_v");
  if (T == 0) return ANEMLL_OK;
  ANEMLL_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(g, 4) && aligned(beta, 4) &&
                     aligned(out, 16) && aligned(z, 16) && (z_row_stride * 2) % 16 == 0 && aligned(norm_weight, 16) &&
                     (core_out == nullptr || aligned(core_out, 16)),
                 ANEMLL_EALIGN,
                 "gdn_chunked_prefill_gated: q/k/v, out, z (and its row stride), the weight and core_out must be "
                 "16-byte aligned");
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)d_k);
  cudaStream_t st = (cudaStream_t)stream;
  return ANEMLL_DISPATCH_HALF(qkv_dtype, TIn, [&] {
    return ANEMLL_DISPATCH_HALF(out_dtype, TOut, [&] {
      const GatedNorm<TOut> gn{(const TOut*)z, (long long)z_row_stride, norm_weight, eps, core_out};
      return launch_chunked<TIn, TOut, true>(q, k, v, g, beta, state, out, B, T, H_qk, H_v, scale, qk_l2norm, gn,
                                             st);
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

// Selects the chunked prefill's kernel: 0 by the number of (sequence, value head) chains (the
// pipelined one-chain-per-SM kernel while they fit one wave of SMs), 1 always pipelined, 2 always
// the two-chains-per-SM kernel.  Returns the previous mode.  Both give the same results bit for bit.
extern "C" int anemll_gdn_chunked_mode(int mode) {
  const int prev = anemll::g_pipe_mode;
  if (mode >= 0 && mode <= 2) anemll::g_pipe_mode = mode;
  return prev;
}
