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
//   A    = strict_lower(diag(beta) K K^T * Gam), T = (I + A)^-1   (CUDA cores)
//   U^T  = V^T (T diag(beta))^T              (tcgen05, M=128 N=64 K=64)
//   W^T  = K^T (T diag(beta e^G))^T          (tcgen05, M=128 N=64 K=64)
//   Vn^T = U^T - S^T W^T                     (tcgen05, A negated, accumulates on U)
//   O^T  = S^T (diag(e^G) Q)^T + Vn^T P^T    (tcgen05, two products, one accumulator)
//   S^T  = e^{G_c} S^T + (diag(e^{G_c - G}) Vn)^T K   (e^{G_c} applied in TMEM, then tcgen05)
//
// Every product is arranged so that M = 128 (d_v or d_k on TMEM lanes).  All
// operands are fp16 in 128-byte-swizzled shared memory; accumulators are fp32
// in TMEM.  fp16 (10-bit mantissa) operands keep the result within 1e-3
// relative L2 of an fp32 evaluation; bf16 inputs convert to fp16 on load.  The
// attention scale multiplies O in fp32 at the end (O is linear in q).
//
// Semantics: torch_chunk_gated_delta_rule of transformers 5.5.0
// (modeling_qwen3_5.py:234-311); chunk (WY/UT) form of Yang et al. (2024).
#include "common.cuh"
#include "tcgen05.cuh"

namespace anemll {
namespace {

constexpr int C = 64;
constexpr int D = 128;
constexpr int NT = 128;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t COL_S = 0, COL_O = 128, COL_U = 192;

// shared memory map (bytes from a 1024-byte aligned base)
constexpr int QK_BLK = 128 * 128;            // one 64-column block of a 128-row tile
constexpr int T64_BLK = 64 * 128;            // one 64-column block of a 64-row tile
constexpr int OFF_QK = 0;                    // [2][128 rows][128 B]: rows 0-63 Q, 64-127 K
constexpr int OFF_QT = OFF_QK + 2 * QK_BLK;  // diag(e^G) Q: [2][64][128 B]
constexpr int OFF_V = OFF_QT + 2 * T64_BLK;  // V [2][64][128 B]; later Vn^T [128][128 B]
constexpr int OFF_VD = OFF_V + 2 * T64_BLK;  // (dec * Vn)^T [128][128 B]
constexpr int OFF_P = OFF_VD + 128 * 128;    // P [64][128 B]
constexpr int OFF_T1 = OFF_P + 64 * 128;     // T diag(beta)
constexpr int OFF_T2 = OFF_T1 + 64 * 128;    // T diag(beta e^G)
constexpr int OFF_W = OFF_T2 + 64 * 128;     // W [2][64][128 B]
constexpr int OFF_ST = OFF_W + 2 * T64_BLK;  // S^T [2][128][128 B]
constexpr int OFF_A = OFF_ST + 2 * QK_BLK;   // fp32 A [64][A_LD]
constexpr int A_LD = 68;                     // row pitch: conflict-free float4 row stores
constexpr int OFF_MISC = OFF_A + 64 * A_LD * 4;
constexpr int SMEM_BYTES = OFF_MISC + 6 * 64 * 4 + 64 + 1024;

__device__ int g_chunked_error = 0;

// byte offset of 16-byte chunk `ch` (0..7) of row `r` inside a 128-byte-row swizzled block
__device__ __forceinline__ uint32_t sw(int r, int ch) { return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4)); }
__device__ __forceinline__ uint32_t sw_elem(int r, int c) { return sw(r, c >> 3) + (uint32_t)((c & 7) << 1); }

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* f) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
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

template <typename TIn, typename TOut>
__global__ void __launch_bounds__(NT, 1)
gdn_chunked_kernel(const TIn* __restrict__ q, const TIn* __restrict__ k, const TIn* __restrict__ v,
                   const float* __restrict__ g, const float* __restrict__ beta, float* __restrict__ state,
                   TOut* __restrict__ out, int T, int Hqk, int Hv, float scale, int l2norm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sG = reinterpret_cast<float*>(sm + OFF_MISC);
  float* sBeta = sG + 64;
  float* sEG = sG + 128;
  float* sDec = sG + 192;
  float* sA = reinterpret_cast<float*>(sm + OFF_A);
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x;
  const int b = bh / Hv, hv = bh % Hv;
  const int hk = hv / (Hv / Hqk);
  const uint32_t sbase = tc::smem_u32(sm);
  const uint32_t bar = tc::smem_u32(&mbar);

  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's TMEM sub-partition
  uint32_t phase = 0;

  // ---- initial state: thread d holds column d of S (row d of S^T) ----
  float* Sg = state + (size_t)bh * D * D;
  {
    float buf[32];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int i = 0; i < 32; ++i) buf[i] = Sg[(size_t)(j * 32 + i) * D + tid];
      tc::tmem_st32(lane_addr + COL_S + j * 32, buf);
    }
    tc::tmem_wait_st();
  }

  auto sync_mma = [&]() -> bool {
    // every thread: wait until the MMAs committed so far have completed
    const bool ok = tc::mbar_wait(bar, phase);
    phase ^= 1u;
    if (!ok) {
      atomicExch(&g_chunked_error, 1);
      abort_flag = 1;
    }
    tc::fence_after();
    return ok;
  };

  const int nchunks = (T + C - 1) / C;
  for (int c = 0; c < nchunks && !abort_flag; ++c) {
    const int t0 = c * C;
    const int nvalid = min(C, T - t0);
    // ---------------- gates: cumulative log decay (padding tokens: g = beta = 0) ----------------
    if (warp == 0) {
      float g0 = 0.f, g1 = 0.f, b0 = 0.f, b1 = 0.f;
      const int i0 = 2 * lane, i1 = 2 * lane + 1;
      const size_t base = ((size_t)b * T + t0) * Hv + hv;
      if (i0 < nvalid) { g0 = g[base + (size_t)i0 * Hv]; b0 = beta[base + (size_t)i0 * Hv]; }
      if (i1 < nvalid) { g1 = g[base + (size_t)i1 * Hv]; b1 = beta[base + (size_t)i1 * Hv]; }
      float s = g0 + g1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += n;
      }
      const float G1 = s, G0 = s - g1;
      sG[i0] = G0;
      sG[i1] = G1;
      sBeta[i0] = b0;
      sBeta[i1] = b1;
      const float Glast = __shfl_sync(0xffffffffu, G1, 31);
      sEG[i0] = __expf(G0);
      sEG[i1] = __expf(G1);
      sDec[i0] = __expf(Glast - G0);
      sDec[i1] = __expf(Glast - G1);
      if (lane == 0) sG[256] = __expf(Glast);  // gamma, after the four 64-float arrays
    }
    __syncthreads();

    // ---------------- tiles: Q, diag(e^G) Q, K, V (fp16, swizzled) ----------------
    {
      const int ch = tid & 15;  // 16-byte chunk of the 256-byte row
      const int blk = ch >> 3, cb = ch & 7;
#pragma unroll 2
      for (int it = 0; it < 8; ++it) {
        const int r = (tid >> 4) + it * 8;  // token row 0..63
        const bool valid = r < nvalid;
        const size_t tok = (size_t)b * T + t0 + r;
        float fq[8], fk[8], fv[8];
        if (valid) {
          load8(q + (tok * Hqk + hk) * D + ch * 8, fq);
          load8(k + (tok * Hqk + hk) * D + ch * 8, fk);
          load8(v + (tok * Hv + hv) * D + ch * 8, fv);
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
        *reinterpret_cast<uint4*>(sm + OFF_QK + blk * QK_BLK + sw(r, cb)) = pack8_f16(fq);
        *reinterpret_cast<uint4*>(sm + OFF_QK + blk * QK_BLK + sw(64 + r, cb)) = pack8_f16(fk);
        *reinterpret_cast<uint4*>(sm + OFF_V + blk * T64_BLK + sw(r, cb)) = pack8_f16(fv);
        const float e = sEG[r];
#pragma unroll
        for (int i = 0; i < 8; ++i) fq[i] *= e;
        *reinterpret_cast<uint4*>(sm + OFF_QT + blk * T64_BLK + sw(r, cb)) = pack8_f16(fq);
      }
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

    // ---------------- D1 = [Q;K] K^T ----------------
    if (tid == 0) {
      constexpr uint32_t id = tc::idesc_f16(128, 64, false, false);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t koff = (uint32_t)((s >> 2) * QK_BLK + (s & 3) * 32);
        const uint64_t ad = tc::sdesc_sw128(sbase + OFF_QK + koff, 16, 1024);
        const uint64_t bd = tc::sdesc_sw128(sbase + OFF_QK + 64 * 128 + koff, 16, 1024);
        tc::mma_f16(tmem + COL_O, ad, bd, id, s > 0);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- P, A; state readout ----------------
    {
      float r0[32], r1[32];
      tc::tmem_ld32(lane_addr + COL_O, r0);
      tc::tmem_ld32(lane_addr + COL_O + 32, r1);
      tc::tmem_wait_ld();
      if (tid < 64) {
        const int i = tid;
        const float Gi = sG[i];
        float p[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float x = j < 32 ? r0[j] : r1[j - 32];
          p[j] = j <= i ? x * __expf(Gi - sG[j]) : 0.f;
        }
#pragma unroll
        for (int cb = 0; cb < 8; ++cb)
          *reinterpret_cast<uint4*>(sm + OFF_P + sw(i, cb)) = pack8_f16(p + cb * 8);
      } else {
        const int i = tid - 64;
        const float Gi = sG[i], bi = sBeta[i];
        float* arow = sA + i * A_LD;
#pragma unroll
        for (int j4 = 0; j4 < 16; ++j4) {
          float a4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = j4 * 4 + e;
            const float x = j < 32 ? r0[j] : r1[j - 32];
            a4[e] = j < i ? bi * x * __expf(Gi - sG[j]) : 0.f;
          }
          *reinterpret_cast<float4*>(arow + j4 * 4) = make_float4(a4[0], a4[1], a4[2], a4[3]);
        }
      }
      // S^T row (lane = d_v index) -> fp16 operand; then scale the accumulator by gamma
      const float gamma = sG[256];
#pragma unroll
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
        for (int i = 0; i < 32; ++i) s32[i] *= gamma;
        tc::tmem_st32(lane_addr + COL_S + j * 32, s32);
      }
      tc::tmem_wait_st();
    }
    tc::fence_before();
    __syncthreads();

    // ---------------- T = (I + A)^-1 by forward substitution (thread j: column j) ----------------
    if (tid < 64) {
      const int j = tid;
      float t[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        float acc = (i == j) ? 1.f : 0.f;
        const float* arow = sA + i * A_LD;
#pragma unroll
        for (int kk = 0; kk < i; ++kk) acc -= arow[kk] * t[kk];
        t[i] = acc;
      }
      const float bj = sBeta[j], bej = sBeta[j] * sEG[j];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        *reinterpret_cast<__half*>(sm + OFF_T1 + sw_elem(i, j)) = __float2half_rn(t[i] * bj);
        *reinterpret_cast<__half*>(sm + OFF_T2 + sw_elem(i, j)) = __float2half_rn(t[i] * bej);
      }
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

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
        tc::mma_f16(tmem + COL_O, ak, b2, id, s > 0);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- W readout: lane = d_k index, columns = tokens ----------------
    {
      float r0[32], r1[32];
      tc::tmem_ld32(lane_addr + COL_O, r0);
      tc::tmem_ld32(lane_addr + COL_O + 32, r1);
      tc::tmem_wait_ld();
      const int d = tid;
      uint8_t* wb = sm + OFF_W + (d >> 6) * T64_BLK;
#pragma unroll
      for (int t = 0; t < 64; ++t) {
        const float x = t < 32 ? r0[t] : r1[t - 32];
        *reinterpret_cast<__half*>(wb + sw_elem(t, d & 63)) = __float2half_rn(x);
      }
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

    // ---------------- Vn^T = U^T - S^T W^T ; O^T = S^T Qt^T ----------------
    if (tid == 0) {
      constexpr uint32_t idn = tc::idesc_f16(128, 64, false, false, true);
      constexpr uint32_t id = tc::idesc_f16(128, 64, false, false);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint64_t as = tc::sdesc_sw128(sbase + OFF_ST + (s >> 2) * QK_BLK + (s & 3) * 32, 16, 1024);
        const uint64_t bw = tc::sdesc_sw128(sbase + OFF_W + (s >> 2) * T64_BLK + (s & 3) * 32, 16, 1024);
        tc::mma_f16(tmem + COL_U, as, bw, idn, 1);
        const uint64_t bq = tc::sdesc_sw128(sbase + OFF_QT + (s >> 2) * T64_BLK + (s & 3) * 32, 16, 1024);
        tc::mma_f16(tmem + COL_O, as, bq, id, s > 0);
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
      const int d = tid;
#pragma unroll
      for (int cb = 0; cb < 8; ++cb) {
        float x[8], y[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int t = cb * 8 + e;
          x[e] = t < 32 ? r0[t] : r1[t - 32];
          y[e] = x[e] * sDec[t];
        }
        *reinterpret_cast<uint4*>(sm + OFF_V + sw(d, cb)) = pack8_f16(x);
        *reinterpret_cast<uint4*>(sm + OFF_VD + sw(d, cb)) = pack8_f16(y);
      }
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

    // ---------------- O^T += Vn^T P^T ; S^T += (dec Vn)^T K ----------------
    if (tid == 0) {
      constexpr uint32_t id64 = tc::idesc_f16(128, 64, false, false);
      constexpr uint32_t id128 = tc::idesc_f16(128, 128, false, true);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint64_t av = tc::sdesc_sw128(sbase + OFF_V + s * 32, 16, 1024);
        const uint64_t bp = tc::sdesc_sw128(sbase + OFF_P + s * 32, 16, 1024);
        tc::mma_f16(tmem + COL_O, av, bp, id64, 1);
        const uint64_t ad = tc::sdesc_sw128(sbase + OFF_VD + s * 32, 16, 1024);
        const uint64_t bk = tc::sdesc_sw128(sbase + OFF_QK + 64 * 128 + s * 2048, QK_BLK, 1024);
        tc::mma_f16(tmem + COL_S, ad, bk, id128, 1);
      }
      tc::commit(bar);
    }
    if (!sync_mma()) break;

    // ---------------- O readout -> global ----------------
    {
      float r0[32], r1[32];
      tc::tmem_ld32(lane_addr + COL_O, r0);
      tc::tmem_ld32(lane_addr + COL_O + 32, r1);
      tc::tmem_wait_ld();
      const int d = tid;
#pragma unroll
      for (int t = 0; t < 64; ++t) {
        if (t < nvalid) {
          const float x = (t < 32 ? r0[t] : r1[t - 32]) * scale;
          out[(((size_t)b * T + t0 + t) * Hv + hv) * D + d] = from_f32<TOut>(x);
        }
      }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  }

  // ---- final state ----
  if (!abort_flag) {
    float buf[32];
#pragma unroll
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

template <typename TIn, typename TOut>
int launch_chunked(const void* q, const void* k, const void* v, const float* g, const float* beta, float* state,
                   void* out, int B, int T, int Hqk, int Hv, float scale, int l2norm, cudaStream_t st) {
  auto kern = gdn_chunked_kernel<TIn, TOut>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  kern<<<B * Hv, NT, SMEM_BYTES, st>>>((const TIn*)q, (const TIn*)k, (const TIn*)v, g, beta, state, (TOut*)out, T,
                                       Hqk, Hv, scale, l2norm);
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
  ANEMLL_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16), ANEMLL_EALIGN,
                 "gdn_chunked_prefill: q/k/v must be 16-byte aligned");
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
