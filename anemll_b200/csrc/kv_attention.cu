// Fixed-shape KV-cache attention with the cache write fused in.
//
// One launch handles one prefill chunk (S tokens) or one decode step (S = 1)
// of one layer.  The G = H_q / H_kv query heads of a kv head are packed into
// the rows of one tile (row r = token r / G, head r % G), so every K/V tile
// read from HBM serves all G heads (GQA without the reference's repeat_kv
// copy).  Keys are split across CTAs (split-KV); each CTA runs an online
// softmax over its key range with fp32 accumulators and either finishes the
// rows itself (one split) or leaves unnormalised partials plus (max, sum) in
// the caller's workspace for kv_combine_kernel.  Only the visible key range
// [key_lo, key_hi) is visited when the mask is derived from positions.
//
// The new rows [pos, pos + S) are read straight from k_new / v_new by the CTA
// whose split contains them, and row-tile-0 CTAs store them into the cache,
// so no CTA ever reads a cache row that is being written.
//
// Reference semantics: anemll/models/qwen_model.py forward_prefill 509-546,
// forward_regular 469-507, cache writes 669-675 / 733-745; sigmoid gate of
// transformers 5.5.0 modeling_qwen3_5.py:689.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "mma_sync.cuh"
#include "tcgen05.cuh"

namespace anemll {
namespace {

constexpr int NB = 32;  // keys per block

struct KvParams {
  const void* q;
  const void* k_new;
  const void* v_new;
  const void* gate;
  void* kc;
  void* vc;
  long long bs, hs;
  const void* mask;
  int mask_dtype;
  long long mask_ld;
  void* out;
  int B, S, Hq, Hkv, ctx, pos, window, aligned, has_new;
  int key_lo, key_hi, n_splits, ks;
  float* ws_o;
  float* ws_ml;
  float scale_log2;
  long long gate_ts, gate_hs;  // gate element (b, s, head, d) at (b S + s) gate_ts + head gate_hs + d
  // fused head norm + RoPE: q, k_new, v_new and gate are column slices of one q/k/v projection output
  // whose token rows are qkv_ld elements apart; q and k_new are normed and rotated on the way in
  int fused;
  long long qkv_ld;
  const float* qnw;
  const float* knw;
  const float* cos_t;
  const float* sin_t;
  float eps;
};

// gate element (b, s, head hq, column d)
__device__ __forceinline__ long long gate_index(const KvParams& p, int b, int s, int hq, int d) {
  return ((long long)b * p.S + s) * p.gate_ts + (long long)hq * p.gate_hs + d;
}

__device__ __forceinline__ int swz(int row, int chunk) { return chunk ^ (row & 7); }

template <typename T, int HD>
__device__ __forceinline__ void load_rows_async(T* smem, int nrows, const T* const* src_rows, int tid, int nthreads) {
  constexpr int CPR = HD / 8;  // 16-byte chunks per row
  for (int i = tid; i < nrows * CPR; i += nthreads) {
    const int r = i / CPR, c = i % CPR;
    T* dst = smem + r * HD + swz(r, c) * 8;
    const T* s = src_rows[r];
    if (s) cp_async16(dst, s + c * 8);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
}

template <typename T, int HD, int MW>
__global__ void __launch_bounds__(MW * 32)
kv_attn_kernel(KvParams p) {
  griddep_wait();
  constexpr int ROWS = 16 * MW;
  constexpr int NT = MW * 32;
  constexpr int NTILE_O = HD / 8;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  T* Qs = reinterpret_cast<T*>(smem_raw);
  T* Ks = Qs + ROWS * HD;       // [2][NB][HD]
  T* Vs = Ks + 2 * NB * HD;     // [2][NB][HD]
  __shared__ const T* rowptr[ROWS > NB ? ROWS : NB];
  __shared__ const T* vrowptr[NB];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.Hq / p.Hkv;
  const int R = p.S * G;
  const int bh = blockIdx.z;
  const int b = bh / p.Hkv, kvh = bh % p.Hkv;
  const int split = blockIdx.y;
  const int r0 = blockIdx.x * ROWS;
  const int k_begin = p.key_lo + split * p.ks;
  const int k_end = min(p.key_hi, k_begin + p.ks);

  T* Kc = reinterpret_cast<T*>(p.kc) + (long long)b * p.bs + (long long)kvh * p.hs;
  T* Vc = reinterpret_cast<T*>(p.vc) + (long long)b * p.bs + (long long)kvh * p.hs;
  const T* kn = p.has_new ? reinterpret_cast<const T*>(p.k_new) + (long long)(b * p.Hkv + kvh) * p.S * HD : nullptr;
  const T* vn = p.has_new ? reinterpret_cast<const T*>(p.v_new) + (long long)(b * p.Hkv + kvh) * p.S * HD : nullptr;

  // fused cache write of the new rows that fall in this split
  if (p.has_new && blockIdx.x == 0) {
    const int w0 = max(p.pos, k_begin), w1 = min(p.pos + p.S, k_end);
    constexpr int CPR = HD / 8;
    for (int i = tid; i < (w1 - w0) * CPR * 2; i += NT) {
      const int which = i / ((w1 - w0) * CPR);
      const int rem = i % ((w1 - w0) * CPR);
      const int j = w0 + rem / CPR, c = rem % CPR;
      const T* src = (which ? vn : kn) + (long long)(j - p.pos) * HD + c * 8;
      T* dst = (which ? Vc : Kc) + (long long)j * HD + c * 8;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
  }

  // Q tile
  for (int i = tid; i < ROWS; i += NT) {
    const int r = r0 + i;
    if (r < R) {
      const int s = r / G, h = kvh * G + r % G;
      rowptr[i] = reinterpret_cast<const T*>(p.q) + ((long long)(b * p.Hq + h) * p.S + s) * HD;
    } else {
      rowptr[i] = nullptr;
    }
  }
  __syncthreads();
  load_rows_async<T, HD>(Qs, ROWS, rowptr, tid, NT);
  cp_async_commit();
  __syncthreads();

  auto issue_kv = [&](int kb, int buf) {
    for (int i = tid; i < NB; i += NT) {
      const int j = kb + i;
      const T* kp = nullptr;
      const T* vp = nullptr;
      if (j < k_end) {
        if (p.has_new && j >= p.pos && j < p.pos + p.S) {
          kp = kn + (long long)(j - p.pos) * HD;
          vp = vn + (long long)(j - p.pos) * HD;
        } else {
          kp = Kc + (long long)j * HD;
          vp = Vc + (long long)j * HD;
        }
      }
      rowptr[i] = kp;
      vrowptr[i] = vp;
    }
    __syncthreads();
    load_rows_async<T, HD>(Ks + buf * NB * HD, NB, rowptr, tid, NT);
    load_rows_async<T, HD>(Vs + buf * NB * HD, NB, vrowptr, tid, NT);
    cp_async_commit();
    __syncthreads();
  };

  const int nblk = (k_end - k_begin + NB - 1) / NB;
  // per-thread row state: rows g and g+8 of this warp's 16
  const int g = lane >> 2, t4 = lane & 3;
  const int wr0 = r0 + warp * 16;
  int rows_s[2], rows_lo[2], rows_hi[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = wr0 + g + h * 8;
    const int s = r < R ? r / G : 0;
    rows_s[h] = s;
    const int pq = p.pos + s;
    int lo = 0;
    if (p.window > 0) lo = p.aligned ? max(0, min(p.pos + p.S, p.ctx) - p.window) : pq - p.window + 1;
    rows_lo[h] = lo;
    rows_hi[h] = r < R ? pq : -1;  // inclusive; -1 hides everything for padding rows
  }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o_acc[NTILE_O][4];
#pragma unroll
  for (int i = 0; i < NTILE_O; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;

  if (nblk > 0) issue_kv(k_begin, 0);
  for (int blk = 0; blk < nblk; ++blk) {
    const int buf = blk & 1;
    const int kb = k_begin + blk * NB;
    if (blk + 1 < nblk) {
      issue_kv(kb + NB, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const T* Kb = Ks + buf * NB * HD;
    const T* Vb = Vs + buf * NB * HD;

    // S = Q K^T : 16 rows x NB keys per warp
    float sc[NB / 8][4];
#pragma unroll
    for (int n = 0; n < NB / 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t a[4];
      {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 2 + (lane >> 4);
        ldmatrix_x4(a, Qs + r * HD + swz(r, c) * 8);
      }
#pragma unroll
      for (int n2 = 0; n2 < NB / 16; ++n2) {
        uint32_t bfr[4];
        const int r = n2 * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(bfr, Kb + r * HD + swz(r, c) * 8);
        mma_16816<T>(sc[2 * n2], a, bfr[0], bfr[1]);
        mma_16816<T>(sc[2 * n2 + 1], a, bfr[2], bfr[3]);
      }
    }
    // scale, mask, online softmax (base-2)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < NB / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int j = kb + n * 8 + t4 * 2 + (e & 1);
        float v = sc[n][e] * p.scale_log2;
        bool vis = j < k_end;
        if (p.mask) {
          if (vis && rows_hi[h] >= 0) {
            const long long mi = (long long)rows_s[h] * p.mask_ld + j;
            const float mv = p.mask_dtype == ANEMLL_F32 ? reinterpret_cast<const float*>(p.mask)[mi]
                           : p.mask_dtype == ANEMLL_F16 ? __half2float(reinterpret_cast<const __half*>(p.mask)[mi])
                           : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.mask)[mi]);
            v += mv * 1.4426950408889634f;
          } else {
            vis = false;
          }
          if (v == -INFINITY) vis = false;
        } else {
          vis = vis && j <= rows_hi[h] && j >= rows_lo[h];
        }
        v = vis ? v : -INFINITY;
        sc[n][e] = v;
        mx[h] = fmaxf(mx[h], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float mnew = fmaxf(m_run[h], mx[h]);
      const float base = mnew == -INFINITY ? 0.f : mnew;
      alpha[h] = fast_exp2(m_run[h] - base);
      m_run[h] = mnew;
      mx[h] = base;  // reuse as subtraction base
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[NB / 16][4];
#pragma unroll
    for (int n = 0; n < NB / 8; ++n) {
      const float p0 = fast_exp2(sc[n][0] - mx[0]);
      const float p1 = fast_exp2(sc[n][1] - mx[0]);
      const float p2 = fast_exp2(sc[n][2] - mx[1]);
      const float p3 = fast_exp2(sc[n][3] - mx[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int kk = n >> 1, hi = n & 1;
      pf[kk][hi * 2 + 0] = pack2<T>(p0, p1);
      pf[kk][hi * 2 + 1] = pack2<T>(p2, p3);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      l_run[h] = l_run[h] * alpha[h] + rs[h];
    }
#pragma unroll
    for (int i = 0; i < NTILE_O; ++i) {
      o_acc[i][0] *= alpha[0];
      o_acc[i][1] *= alpha[0];
      o_acc[i][2] *= alpha[1];
      o_acc[i][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < NB / 16; ++kk) {
      // A fragment order: (row g, k lo), (row g+8, k lo), (row g, k hi), (row g+8, k hi)
      uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int n2 = 0; n2 < HD / 16; ++n2) {
        uint32_t bfr[4];
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = n2 * 2 + (lane >> 4);
        ldmatrix_x4_trans(bfr, Vb + r * HD + swz(r, c) * 8);
        mma_16816<T>(o_acc[2 * n2], a, bfr[0], bfr[1]);
        mma_16816<T>(o_acc[2 * n2 + 1], a, bfr[2], bfr[3]);
      }
    }
    __syncthreads();
  }
  griddep_launch_dependents();

  // epilogue
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = wr0 + g + h * 8;
    if (r >= R) continue;
    const int s = r / G, hq = kvh * G + r % G;
    if (p.n_splits == 1) {
      const float inv = 1.f / l_run[h];
      T* orow = reinterpret_cast<T*>(p.out) + ((long long)b * p.S + s) * p.Hq * HD + (long long)hq * HD;
      const T* grow = p.gate ? reinterpret_cast<const T*>(p.gate) + gate_index(p, b, s, hq, 0) : nullptr;
#pragma unroll
      for (int i = 0; i < NTILE_O; ++i) {
        const int d = i * 8 + t4 * 2;
        float v0 = o_acc[i][h * 2] * inv, v1 = o_acc[i][h * 2 + 1] * inv;
        if (grow) {
          v0 *= sigmoid_fast(to_f32(grow[d]));
          v1 *= sigmoid_fast(to_f32(grow[d + 1]));
        }
        *reinterpret_cast<uint32_t*>(orow + d) = pack2<T>(v0, v1);
      }
    } else {
      const long long row_id = ((long long)bh * p.n_splits + split) * R + r;
      float* wo = p.ws_o + row_id * HD;
#pragma unroll
      for (int i = 0; i < NTILE_O; ++i) {
        const int d = i * 8 + t4 * 2;
        *reinterpret_cast<float2*>(wo + d) = make_float2(o_acc[i][h * 2], o_acc[i][h * 2 + 1]);
      }
      if (t4 == 0) {
        p.ws_ml[row_id * 2 + 0] = m_run[h];
        p.ws_ml[row_id * 2 + 1] = l_run[h];
      }
    }
  }
}

// Merge the split partials of each row: out = sum_i w_i O_i / sum_i w_i l_i, w_i = 2^(m_i - max m).
// One CTA per row with CB_WARPS warps: warp w reads splits w, w + CB_WARPS, ... (each lane HD/32
// consecutive columns, so a warp reads whole partial rows), and every one of its partial loads is
// issued before the weights are known, so the kernel waits on a single memory round trip.  The
// warp sums meet in shared memory.
// PER = splits per warp (1, 2, 4, 8 or 16), the smallest that covers n_splits, keeps the registers
// (and so the CTAs per SM) in step with the split count.  NCG > 1 splits each row's columns over NCG
// CTAs (blockIdx.z): decode-shaped calls have few rows, and one CTA pulling every split's whole row
// waits on its own SM's load rate, so a few CTAs per row share the reads.
constexpr int CB_WARPS = 8;
constexpr int CB_MAX_SPLITS = 128;

template <typename T, int HD, int PER, int NCG = 1>
__global__ void __launch_bounds__(CB_WARPS * 32)
kv_combine_kernel(KvParams p) {
  static_assert(PER <= CB_MAX_SPLITS / CB_WARPS, "split count above the combine's limit");
  static_assert(HD % (32 * NCG) == 0 && (HD / NCG / 32) % 2 == 0, "column groups of 64 or more");
  griddep_wait();
  griddep_launch_dependents();
  constexpr int CW = HD / NCG;  // columns of this CTA
  constexpr int VPT = CW / 32;  // columns per lane
  const int G = p.Hq / p.Hkv;
  const int R = p.S * G;
  const int r = blockIdx.x;
  const int bh = blockIdx.y;
  const int c0 = (int)blockIdx.z * CW;
  const int b = bh / p.Hkv, kvh = bh % p.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ float s_w[CB_MAX_SPLITS];
  __shared__ float s_red[CB_WARPS];
  __shared__ __align__(16) float s_acc[CB_WARPS][CW];
  const int ns = p.n_splits;
  const long long row0 = (long long)bh * ns * R + r;  // row id of split 0; split i adds i * R
  const long long step = (long long)R * HD;
  const float* po = p.ws_o + row0 * HD + c0 + lane * VPT;
  float v[PER][VPT];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = warp + CB_WARPS * k;
#pragma unroll
    for (int e = 0; e < VPT; e += 2) {
      float2 x = make_float2(0.f, 0.f);
      if (i < ns) x = *reinterpret_cast<const float2*>(po + i * step + e);
      v[k][e] = x.x;
      v[k][e + 1] = x.y;
    }
  }
  // (max, sum) of the splits: thread t holds split t
  float mt = -INFINITY, lt = 0.f;
  if (tid < ns) {
    mt = p.ws_ml[(row0 + (long long)tid * R) * 2];
    lt = p.ws_ml[(row0 + (long long)tid * R) * 2 + 1];
  }
  float M = warp_max(mt);
  if (lane == 0) s_red[warp] = M;
  __syncthreads();
  M = s_red[0];
#pragma unroll
  for (int w = 1; w < CB_WARPS; ++w) M = fmaxf(M, s_red[w]);
  const float base = M == -INFINITY ? 0.f : M;
  const float wt = tid < ns ? fast_exp2(mt - base) : 0.f;
  if (tid < ns) s_w[tid] = wt;
  const float Lp = warp_sum(wt * lt);
  __syncthreads();  // every s_w written, every read of M from s_red done
  if (lane == 0) s_red[warp] = Lp;
  float acc[VPT];
#pragma unroll
  for (int e = 0; e < VPT; ++e) acc[e] = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = warp + CB_WARPS * k;
    if (i < ns) {
      const float wi = s_w[i];
#pragma unroll
      for (int e = 0; e < VPT; ++e) acc[e] += wi * v[k][e];
    }
  }
#pragma unroll
  for (int e = 0; e < VPT; e += 2) *reinterpret_cast<float2*>(&s_acc[warp][lane * VPT + e]) = make_float2(acc[e], acc[e + 1]);
  __syncthreads();
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < CB_WARPS; ++w) L += s_red[w];
  const int s = r / G, hq = kvh * G + r % G;
  for (int d = tid; d < CW; d += CB_WARPS * 32) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < CB_WARPS; ++w) a += s_acc[w][d];
    const long long o = ((long long)b * p.S + s) * p.Hq * HD + (long long)hq * HD + c0 + d;
    float val = a / L;
    if (p.gate) val *= sigmoid_fast(to_f32(reinterpret_cast<const T*>(p.gate)[gate_index(p, b, s, hq, c0 + d)]));
    reinterpret_cast<T*>(p.out)[o] = from_f32<T>(val);
  }
}

// Launch with programmatic stream serialisation, so that the kernel's launch overlaps the tail of the
// previous kernel in the stream.  Every kernel launched this way calls griddep_wait() before its first
// global-memory access.
template <typename... KArgs, typename... Args>
int launch_pdl(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("%s: launch failed, CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
    return (int)e;
  }
  return launch_status(what);
}

template <typename T, int HD, int NCG>
int launch_combine_ncg(const KvParams& q, cudaStream_t st) {
  const int R = q.S * (q.Hq / q.Hkv);
  const dim3 grid(R, q.B * q.Hkv, NCG), block(CB_WARPS * 32);
  const int per = (q.n_splits + CB_WARPS - 1) / CB_WARPS;
  if (per <= 1) return launch_pdl("kv_combine", kv_combine_kernel<T, HD, 1, NCG>, grid, block, 0, st, q);
  if (per <= 2) return launch_pdl("kv_combine", kv_combine_kernel<T, HD, 2, NCG>, grid, block, 0, st, q);
  if (per <= 4) return launch_pdl("kv_combine", kv_combine_kernel<T, HD, 4, NCG>, grid, block, 0, st, q);
  if (per <= 8) return launch_pdl("kv_combine", kv_combine_kernel<T, HD, 8, NCG>, grid, block, 0, st, q);
  return launch_pdl("kv_combine", kv_combine_kernel<T, HD, 16, NCG>, grid, block, 0, st, q);
}

// Rows x (sequence, kv head) below one CTA per SM: split the columns into 64-wide groups.
template <typename T, int HD>
int launch_combine(const KvParams& q, cudaStream_t st) {
  const long rows = (long)q.S * (q.Hq / q.Hkv) * q.B * q.Hkv;
  if (HD >= 128 && rows < 148) return launch_combine_ncg<T, HD, HD / 64>(q, st);
  return launch_combine_ncg<T, HD, 1>(q, st);
}

struct Plan {
  int key_lo, key_hi, n_splits, ks, mw, row_tiles;
  int max_splits;  // bound on n_splits over every key range of this shape (workspace sizing)
};

Plan make_plan(int B, int S, int Hq, int Hkv, int ctx, int pos, int window, int aligned, bool explicit_mask) {
  Plan pl;
  if (explicit_mask) {
    pl.key_lo = 0;
    pl.key_hi = ctx;
  } else {
    pl.key_hi = min(ctx, pos + S);
    pl.key_lo = 0;
    if (window > 0) pl.key_lo = max(0, aligned ? min(pos + S, ctx) - window : pos - window + 1);
    if (pl.key_lo > pl.key_hi) pl.key_lo = pl.key_hi;
  }
  const int R = S * (Hq / Hkv);
  pl.mw = R <= 16 ? 1 : 4;
  pl.row_tiles = (R + 16 * pl.mw - 1) / (16 * pl.mw);
  const int L = pl.key_hi - pl.key_lo;
  const int nblocks = max(1, (L + NB - 1) / NB);
  const long base = (long)pl.row_tiles * B * Hkv;
  const int want_raw = (int)((2L * 148 + base - 1) / base);
  pl.max_splits = max(1, min(want_raw, min((ctx + NB - 1) / NB, 128)));
  // single-warp CTAs (decode): at most 64 splits, so each CTA reads at least two key blocks
  const int cap = pl.mw == 1 ? 64 : 128;
  const int want = max(1, min(want_raw, min(nblocks, cap)));
  const int bps = (nblocks + want - 1) / want;
  pl.ks = bps * NB;
  pl.n_splits = max(1, (L + pl.ks - 1) / pl.ks);
  return pl;
}

template <typename T, int HD>
int launch_kv(KvParams& p, const Plan& pl, cudaStream_t st) {
  dim3 grid(pl.row_tiles, pl.n_splits, p.B * p.Hkv);
  int rc;
  if (pl.mw == 1) {
    const size_t smem = (size_t)(16 * HD + 4 * NB * HD) * sizeof(T);
    auto kern = kv_attn_kernel<T, HD, 1>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    rc = launch_pdl("kv_attention", kern, grid, dim3(32), smem, st, p);
  } else {
    const size_t smem = (size_t)(64 * HD + 4 * NB * HD) * sizeof(T);
    auto kern = kv_attn_kernel<T, HD, 4>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    rc = launch_pdl("kv_attention", kern, grid, dim3(128), smem, st, p);
  }
  if (rc) return rc;
  if (pl.n_splits > 1) {
    rc = launch_combine<T, HD>(p, st);
  }
  return rc;
}

size_t workspace_bytes_for(int n_splits, int B, int S, int Hq, int Hkv, int hd) {
  if (n_splits <= 1) return 0;
  const size_t R = (size_t)S * (Hq / Hkv);
  return (size_t)B * Hkv * n_splits * R * (hd + 2) * sizeof(float);
}


// ---------------------------------------------------------------------------
// tcgen05 path for prefill chunks (G = H_q/H_kv = 8 query heads per kv head,
// head_dim 128 or 256, S >= 16).  A CTA owns a 128-row query tile (8 heads x
// 16 tokens, rows head-major: row = head * 16 + token) and one key split; K/V
// blocks of 64 keys arrive by TMA (double-buffered) straight from the cache.
// Per block: S = Q K^T into TMEM (tcgen05, M=128 N=64 K=hd), an online softmax
// on CUDA cores writes fp16 P to shared memory, O += P V on the tensor core
// into TMEM (M=128 N=hd K=64).  Two threads share each row (256 threads: warps
// w and w + 4 read TMEM lane quarter w), each taking half of the row's score
// columns, half of O's columns in a rescale and half of the epilogue; the two
// halves meet once per block, on the row maximum.  The running max is kept
// stale until it grows by more than 2^8, so O in TMEM is rescaled only then.
// The new cache rows are copied from k_new / v_new into the landed K/V tiles of
// every CTA whose blocks hold them, and row-tile-0 CTAs store them into the
// cache.  Partials use the same workspace format and combine kernel as the
// mma.sync path; they leave the CTA as one 128-row fp32 tile, staged in shared
// memory and written by TMA stores.
constexpr int TC_KB = 64;  // keys per block
constexpr int TC_NT = 256;  // threads: two per query row

struct KvTcMaps {
  CUtensorMap q, k, v;
  // split partials of the tcgen05 prefill path (n_splits > 1), fp32, as {column, token, head, block =
  // (sequence, kv head, split)}: a {32, 16, 8, 1} box is one 32-column slice of a 128-row tile in the
  // kernel's head-major row order, stored into the workspace's token-major rows (row = token G + head)
  CUtensorMap o;
};

__device__ int g_kv_tc_error = 0;

__device__ __forceinline__ uint32_t swz128(int r, int ch) { return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4)); }

template <typename T, int HD>
__global__ void __launch_bounds__(TC_NT, 1)
kv_attn_tc_kernel(const __grid_constant__ KvTcMaps maps, KvParams p) {
  griddep_wait();
  constexpr int NKB = HD / 64;                 // 64-element column blocks of a row
  constexpr int Q_BLK = 128 * 128;             // [128 rows][128 B]
  constexpr int KV_BLK = TC_KB * 128;          // [64 keys][128 B]
  constexpr int OFF_Q = 0;
  constexpr int OFF_K = OFF_Q + NKB * Q_BLK;   // [2 buffers][NKB blocks]
  constexpr int OFF_V = OFF_K + 2 * NKB * KV_BLK;
  constexpr int OFF_P = OFF_V + 2 * NKB * KV_BLK;
  constexpr uint32_t COL_SB = 0, COL_O = 256;  // S: two 64-column buffers; O: HD columns
  constexpr int SLICES = HD / 32;              // 32-column slices of an O row
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t mbar, qbar, kvbar[2];
  __shared__ uint32_t tmem_slot;
  __shared__ float s_half[2][128];  // per row: each half's block maximum, then its running sum

  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & 127, half = tid >> 7;  // query row (TMEM lane) and which half of its columns
  const int G = p.Hq / p.Hkv;  // == 8
  const int bh = blockIdx.z, b = bh / p.Hkv, kvh = bh % p.Hkv;
  const int tile = blockIdx.x, split = blockIdx.y;
  int k_begin = p.key_lo + split * p.ks;
  int k_end = min(p.key_hi, k_begin + p.ks);
  if (!p.mask) {
    // positional visibility: no key past the tile's last query is visible, nor (per-query window)
    // a key before its first query's window; a long chunk's early tiles scan only their own prefix
    k_end = min(k_end, p.pos + min(p.S, tile * 16 + 16));
    if (p.window > 0 && !p.aligned) k_begin = max(k_begin, p.pos + tile * 16 - p.window + 1);
  }
  const int nblk = k_end > k_begin ? (k_end - k_begin + TC_KB - 1) / TC_KB : 0;
  const uint32_t sbase = tc::smem_u32(sm);
  const uint32_t bar = tc::smem_u32(&mbar), qb = tc::smem_u32(&qbar), kvb0 = tc::smem_u32(&kvbar[0]);

  // this thread's row: head g, token s
  const int g = row >> 4, s = tile * 16 + (row & 15);
  const bool row_valid = s < p.S;
  const int qpos = p.pos + s;
  int lo = 0;
  if (p.window > 0) lo = p.aligned ? max(0, min(p.pos + p.S, p.ctx) - p.window) : qpos - p.window + 1;

  auto issue_kv = [&](int j) {
    const int buf = j & 1;
    const uint32_t kb = kvb0 + 8u * buf;
    tc::mbar_arrive_expect_tx(kb, 2u * NKB * KV_BLK);
    const int key0 = k_begin + j * TC_KB;
#pragma unroll
    for (int c = 0; c < NKB; ++c) {
      const uint32_t dk = sbase + OFF_K + (buf * NKB + c) * KV_BLK;
      const uint32_t dv = sbase + OFF_V + (buf * NKB + c) * KV_BLK;
      if (p.B > 1) {
        tc::tma_load_4d(dk, &maps.k, c * 64, key0, kvh, b, kb);
        tc::tma_load_4d(dv, &maps.v, c * 64, key0, kvh, b, kb);
      } else {
        tc::tma_load_3d(dk, &maps.k, c * 64, key0, kvh, kb);
        tc::tma_load_3d(dv, &maps.v, c * 64, key0, kvh, kb);
      }
    }
  };

  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init(&qbar, 1);
    tc::mbar_init(&kvbar[0], 1);
    tc::mbar_init(&kvbar[1], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  if (tid == 0) {
    tc::mbar_arrive_expect_tx(qb, (uint32_t)(NKB * Q_BLK));
#pragma unroll
    for (int c = 0; c < NKB; ++c) {
      if (p.fused)  // straight from the q/k/v projection output: {column, token, head, sequence}
        tc::tma_load_4d(sbase + OFF_Q + c * Q_BLK, &maps.q, c * 64, tile * 16, kvh * G, b, qb);
      else
        tc::tma_load_3d(sbase + OFF_Q + c * Q_BLK, &maps.q, c * 64, tile * 16, b * p.Hq + kvh * G, qb);
    }
    if (nblk > 0) issue_kv(0);
  }
  // fused head norm: this tile's cos/sin rows and the q_norm weights into shared memory while the Q
  // tile is in flight (the second K and V buffers and the P tile are idle until the key loop)
  constexpr int FLD = HD + 4;  // staged table row stride (floats): 16-byte units, banks spread
  float* f_cos = reinterpret_cast<float*>(sm + OFF_K + NKB * KV_BLK);
  float* f_sin = reinterpret_cast<float*>(sm + OFF_V + NKB * KV_BLK);
  float* f_w = reinterpret_cast<float*>(sm + OFF_P);
  static_assert(16 * FLD * 4 <= NKB * KV_BLK && HD * 4 <= 128 * 128, "staged tables fit the idle buffers");
  if (p.fused) {
    for (int i = tid; i < 2 * 16 * (HD / 4); i += TC_NT) {
      const int tb = i / (16 * (HD / 4)), rem = i % (16 * (HD / 4)), st = rem / (HD / 4), c4 = rem % (HD / 4);
      if (tile * 16 + st < p.S)
        cp_async16((tb ? f_sin : f_cos) + st * FLD + c4 * 4,
                   (tb ? p.sin_t : p.cos_t) + (long long)(p.pos + tile * 16 + st) * HD + c4 * 4);
    }
    for (int i = tid; i < HD / 4; i += TC_NT) cp_async16(f_w + i * 4, p.qnw + i * 4);
    cp_async_commit();
  }
  bool ok = __syncthreads_and(tc::mbar_wait(qb, 0));
  if (p.fused) {
    cp_async_wait<0>();
    __syncthreads();
  }
  if (p.fused && ok) {
    // head norm + RoPE of the query rows, in place in the swizzled tile (the first half's thread
    // owns row `row`: head row / 16, token tile * 16 + row % 16); same arithmetic as
    // head_norm_rope_warp
    if (half == 0 && row_valid) {
      constexpr int EPL = HD / 32, PPC = 8 / EPL;  // elements per partial, partials per 8-element chunk
      float part[32];
#pragma unroll
      for (int k = 0; k < HD / 8; ++k) {
        const uint4 u = *reinterpret_cast<const uint4*>(sm + OFF_Q + (k >> 3) * Q_BLK + swz128(row, k & 7));
        const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int q2 = 0; q2 < PPC; ++q2) {
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const float v = to_f32(h[q2 * EPL + e]);
            ss += v * v;
          }
          part[k * PPC + q2] = ss;
        }
      }
      const float rn = head_norm_scale(part, HD, p.eps);
      const float* cr = f_cos + (row & 15) * FLD;
      const float* sr = f_sin + (row & 15) * FLD;
#pragma unroll 1
      for (int k = 0; k < HD / 16; ++k) {  // chunk k of the first half with chunk k + HD/16
        const int k2 = k + HD / 16;
        uint8_t* pl = sm + OFF_Q + (k >> 3) * Q_BLK + swz128(row, k & 7);
        uint8_t* ph = sm + OFF_Q + (k2 >> 3) * Q_BLK + swz128(row, k2 & 7);
        uint4 ul = *reinterpret_cast<const uint4*>(pl), uh = *reinterpret_cast<const uint4*>(ph);
        T* hl = reinterpret_cast<T*>(&ul);
        T* hh = reinterpret_cast<T*>(&uh);
        float xl[8], xh[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xl[e] = head_norm_round<T>(to_f32(hl[e]), rn, f_w[k * 8 + e]);
          xh[e] = head_norm_round<T>(to_f32(hh[e]), rn, f_w[k2 * 8 + e]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          hl[e] = from_f32<T>(rope_one(xl[e], -xh[e], cr[k * 8 + e], sr[k * 8 + e]));
          hh[e] = from_f32<T>(rope_one(xh[e], xl[e], cr[k2 * 8 + e], sr[k2 * 8 + e]));
        }
        *reinterpret_cast<uint4*>(pl) = ul;
        *reinterpret_cast<uint4*>(ph) = uh;
      }
    }
    tc::fence_async_smem();  // generic writes before the tensor core reads the tile
    __syncthreads();
  }
  uint32_t phase = 0;
  float m_run = -INFINITY, l_run = 0.f;  // l_run: this half's share of the row sum
  int pending = nblk > 0 ? 0 : -1;  // K/V block requested and not yet waited for

#pragma unroll 1
  for (int j = 0; j < nblk && ok; ++j) {
    const int buf = j & 1;
    if (tid == 0 && j + 1 < nblk) issue_kv(j + 1);  // the other buffer was released by block j-1
    ok = __syncthreads_and(tc::mbar_wait(kvb0 + 8u * buf, (uint32_t)((j >> 1) & 1)));  // block-uniform
    if (!ok) break;
    pending = j + 1 < nblk ? j + 1 : -1;
    const int key0 = k_begin + j * TC_KB;
    if (p.has_new && key0 < p.pos + p.S && key0 + TC_KB > p.pos) {  // block-uniform
      // the new rows of this block: from k_new / v_new into the landed tiles, and into the cache by
      // the row tile whose queries they are (every tile's scan covers its own rows; other tiles may
      // have read those cache rows before or while they are written, and their tiles are overwritten
      // here as well)
      const int j0 = max(key0, p.pos), j1 = min(min(key0 + TC_KB, k_end), p.pos + p.S);
      const T* kn = reinterpret_cast<const T*>(p.k_new) + (long long)bh * p.S * HD;
      const T* vn = reinterpret_cast<const T*>(p.v_new) + (long long)bh * p.S * HD;
      T* Kc = reinterpret_cast<T*>(p.kc) + (long long)b * p.bs + (long long)kvh * p.hs;
      T* Vc = reinterpret_cast<T*>(p.vc) + (long long)b * p.bs + (long long)kvh * p.hs;
      // four vectors per thread in flight at a time (loads first, then stores)
      constexpr int PU = 4;
      const int n_items = (j1 - j0) * (HD / 8);
      for (int i0 = tid; i0 < n_items; i0 += PU * TC_NT) {
        uint4 kv[PU], vv[PU];
#pragma unroll
        for (int u = 0; u < PU; ++u) {
          const int i = i0 + u * TC_NT;
          if (i < n_items) {
            const int jj = j0 + i / (HD / 8), ch = i % (HD / 8);
            kv[u] = *reinterpret_cast<const uint4*>(kn + (long long)(jj - p.pos) * HD + ch * 8);
            vv[u] = *reinterpret_cast<const uint4*>(vn + (long long)(jj - p.pos) * HD + ch * 8);
          }
        }
#pragma unroll
        for (int u = 0; u < PU; ++u) {
          const int i = i0 + u * TC_NT;
          if (i < n_items) {
            const int jj = j0 + i / (HD / 8), ch = i % (HD / 8), r = jj - key0;
            *reinterpret_cast<uint4*>(sm + OFF_K + (buf * NKB + (ch >> 3)) * KV_BLK + swz128(r, ch & 7)) = kv[u];
            *reinterpret_cast<uint4*>(sm + OFF_V + (buf * NKB + (ch >> 3)) * KV_BLK + swz128(r, ch & 7)) = vv[u];
            if (tile == (jj - p.pos) >> 4) {
              *reinterpret_cast<uint4*>(Kc + (long long)jj * HD + ch * 8) = kv[u];
              *reinterpret_cast<uint4*>(Vc + (long long)jj * HD + ch * 8) = vv[u];
            }
          }
        }
      }
      tc::fence_async_smem();  // generic writes before the tensor core reads the tiles
      __syncthreads();
    }
    tc::fence_after();
    // S = Q K^T
    if (tid == 0) {
      constexpr uint32_t id = tc::idesc_f16(128, 64, false, false, false, std::is_same<T, __nv_bfloat16>::value);
#pragma unroll
      for (int st = 0; st < HD / 16; ++st) {
        const uint64_t ad = tc::sdesc_sw128(sbase + OFF_Q + (st >> 2) * Q_BLK + (st & 3) * 32, 16, 1024);
        const uint64_t bd =
            tc::sdesc_sw128(sbase + OFF_K + (buf * NKB + (st >> 2)) * KV_BLK + (st & 3) * 32, 16, 1024);
        tc::mma_f16(tmem + COL_SB + buf * 64, ad, bd, id, st > 0);
      }
      tc::commit(bar);
    }
    ok = __syncthreads_and(tc::mbar_wait(bar, phase));
    phase ^= 1u;
    if (!ok) break;
    tc::fence_after();
    // online softmax (base 2): this thread's 32 of the row's 64 scores
    float x[32];
    tc::tmem_ld32(lane_addr + COL_SB + buf * 64 + half * 32, x);
    tc::tmem_wait_ld();
    float mb = -INFINITY;
    if (!p.mask) {
      // keys visible to this row form one interval of the block: [vlo, vhi] (block columns)
      const int vlo = max(lo, key0) - key0 - half * 32;
      const int vhi = (row_valid ? min(qpos, k_end - 1) - key0 : -1) - half * 32;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        x[e] = (e >= vlo && e <= vhi) ? x[e] * p.scale_log2 : -INFINITY;
        mb = fmaxf(mb, x[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int kj = key0 + half * 32 + e;
        float v = x[e] * p.scale_log2;
        bool vis = row_valid && kj < k_end;
        if (vis) {
          const long long mi = (long long)s * p.mask_ld + kj;
          const float mv = p.mask_dtype == ANEMLL_F32 ? reinterpret_cast<const float*>(p.mask)[mi]
                         : p.mask_dtype == ANEMLL_F16 ? __half2float(reinterpret_cast<const __half*>(p.mask)[mi])
                         : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.mask)[mi]);
          v += mv * 1.4426950408889634f;
          vis = v != -INFINITY;
        }
        x[e] = vis ? v : -INFINITY;
        mb = fmaxf(mb, x[e]);
      }
    }
    // the row's block maximum over both halves (the halves then take the same rescale decisions)
    s_half[half][row] = mb;
    __syncthreads();
    mb = fmaxf(s_half[0][row], s_half[1][row]);
    float alpha = 1.f;
    bool rescale = false;
    if (mb > m_run + 8.f) {  // also true when m_run is still -inf
      if (m_run != -INFINITY) {
        alpha = fast_exp2(m_run - mb);
        rescale = true;
      }
      m_run = mb;
    }
    const float base = m_run == -INFINITY ? 0.f : m_run;
    float ls = 0.f;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      float p8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        p8[e] = fast_exp2(x[cb * 8 + e] - base);
        ls += p8[e];
      }
      uint4 u;
      T* h = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(p8[e]);
      *reinterpret_cast<uint4*>(sm + OFF_P + swz128(row, half * 4 + cb)) = u;
    }
    l_run = l_run * alpha + ls;
    if (key0 + TC_KB > k_end) {
      // V rows past the split end (unwritten cache rows, possibly not finite) are zeroed, so that
      // their zero weights give exact zeros in P V
      const int nz = key0 + TC_KB - k_end;
      for (int i = tid; i < nz * NKB * 8; i += TC_NT) {
        const int r = TC_KB - nz + i / (NKB * 8), c = (i / 8) % NKB, u = i % 8;
        *reinterpret_cast<uint4*>(sm + OFF_V + (buf * NKB + c) * KV_BLK + r * 128 + u * 16) =
            make_uint4(0, 0, 0, 0);
      }
    }
    if (__any_sync(0xffffffffu, rescale)) {  // warp-collective TMEM access; alpha = 1 on other lanes
#pragma unroll 1
      for (int c = 0; c < SLICES / 2; ++c) {  // this half's columns of O
        float o[32];
        const uint32_t col = COL_O + (uint32_t)(half * (HD / 2) + c * 32);
        tc::tmem_ld32(lane_addr + col, o);
        tc::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= alpha;
        tc::tmem_st32(lane_addr + col, o);
      }
      tc::tmem_wait_st();
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    // O += P V
    if (tid == 0) {
      constexpr uint32_t id = tc::idesc_f16(128, HD, false, true, false, std::is_same<T, __nv_bfloat16>::value);
#pragma unroll
      for (int st = 0; st < TC_KB / 16; ++st) {
        const uint64_t ad = tc::sdesc_sw128(sbase + OFF_P + st * 32, 16, 1024);
        const uint64_t bd = tc::sdesc_sw128(sbase + OFF_V + buf * NKB * KV_BLK + st * 2048, KV_BLK, 1024);
        tc::mma_f16(tmem + COL_O, ad, bd, id, j > 0 || st > 0);
      }
      tc::commit(bar);
    }
    ok = __syncthreads_and(tc::mbar_wait(bar, phase));
    phase ^= 1u;
    tc::fence_after();
  }
  if (!ok) atomicExch(&g_kv_tc_error, 1);
  if (pending >= 0 && !ok) tc::mbar_wait(kvb0 + 8u * (pending & 1), (uint32_t)((pending >> 1) & 1));
  griddep_launch_dependents();

  if (ok) {
    const int R = p.S * G;
    s_half[half][row] = l_run;  // (every block's reads of s_half are done: barriers since)
    __syncthreads();
    const float l_row = s_half[0][row] + s_half[1][row];
    if (p.n_splits > 1) {
      // ---- partial: the unnormalised 128-row O tile is staged in shared memory in 32-column
      //      slices [slice][128 rows][32 floats] with the 128-byte swizzle (the Q and K regions:
      //      every MMA has completed) and leaves by TMA stores; tokens past S are not written ----
      if (half == 0 && row_valid) {
        const long long row_id = ((long long)bh * p.n_splits + split) * R + (long long)s * G + g;
        p.ws_ml[row_id * 2 + 0] = m_run;
        p.ws_ml[row_id * 2 + 1] = l_row;
      }
      static_assert(SLICES * 128 * 128 <= OFF_V - OFF_Q, "the staged O tile fits in the Q and K regions");
#pragma unroll 1
      for (int c0 = 0; c0 < SLICES / 2; ++c0) {
        const int c = half * (SLICES / 2) + c0;
        float o[32];
        if (nblk > 0) {  // uniform across the CTA: every lane takes part in the warp-wide TMEM load
          tc::tmem_ld32(lane_addr + COL_O + c * 32, o);
          tc::tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0.f;
        }
        uint8_t* dst = sm + OFF_Q + c * (128 * 128);
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4)
          *reinterpret_cast<float4*>(dst + swz128(row, c4)) =
              make_float4(o[c4 * 4], o[c4 * 4 + 1], o[c4 * 4 + 2], o[c4 * 4 + 3]);
      }
      tc::fence_async_smem();  // generic writes before the TMA engine reads the tile
      __syncthreads();
      if (tid == 0) {
#pragma unroll 1
        for (int c = 0; c < SLICES; ++c)
          tc::tma_store_4d(&maps.o, sbase + OFF_Q + c * (128 * 128), c * 32, tile * 16, 0, bh * p.n_splits + split);
        tc::bulk_commit();
        tc::bulk_wait_all();
      }
    } else {
      // ---- final rows: O / l, gated, through shared memory in 32-column slices (the two halves
      //      stage slices 2 c2 and 2 c2 + 1 side by side), so that global stores are whole 64-byte
      //      row segments ----
      const float scale_row = nblk > 0 && l_row > 0.f ? 1.f / l_row : 0.f;
      // the tile's gate rows are copied into shared memory in one go (the Q and K regions are free:
      // every MMA has completed), so that no store of the slices below waits on a global load
      const bool gated = p.gate != nullptr;
      constexpr int GLD = HD + 8;  // staged gate row stride (elements): 16-byte units, banks spread
      T* gs = reinterpret_cast<T*>(sm + OFF_Q);
      static_assert(128 * GLD * (int)sizeof(T) <= OFF_V - OFF_Q, "the gate tile fits in the Q and K regions");
      if (gated) {
        for (int i = tid; i < 128 * (HD / 8); i += TC_NT) {
          const int r = i / (HD / 8), ch = i % (HD / 8);
          const int rs = tile * 16 + (r & 15), hq = kvh * G + (r >> 4);
          if (rs < p.S)
            cp_async16(gs + r * GLD + ch * 8, reinterpret_cast<const T*>(p.gate) + gate_index(p, b, rs, hq, ch * 8));
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
      }
#pragma unroll 1
      for (int c2 = 0; c2 < SLICES / 2; ++c2) {
        {
          const int c = 2 * c2 + half;
          float o[32];
          if (nblk > 0) {
            tc::tmem_ld32(lane_addr + COL_O + c * 32, o);
            tc::tmem_wait_ld();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0.f;
          }
          float* stage = reinterpret_cast<float*>(sm + (half ? OFF_V : OFF_P));  // [128][32], float4 swizzled
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4)
            *reinterpret_cast<float4*>(stage + row * 32 + ((c4 ^ (row & 7)) << 2)) =
                make_float4(o[c4 * 4] * scale_row, o[c4 * 4 + 1] * scale_row, o[c4 * 4 + 2] * scale_row,
                            o[c4 * 4 + 3] * scale_row);
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int idx = tid + it * TC_NT, sl = idx >> 9, r = (idx >> 2) & 127, c8 = idx & 3;
          const int col = (2 * c2 + sl) * 32 + c8 * 8;
          const int rs = tile * 16 + (r & 15), hq = kvh * G + (r >> 4);
          const long long off = ((long long)b * p.S + rs) * p.Hq * HD + (long long)hq * HD + col;
          if (rs < p.S) {
            const float* stage = reinterpret_cast<const float*>(sm + (sl ? OFF_V : OFF_P));
            const float4 a = *reinterpret_cast<const float4*>(stage + r * 32 + (((2 * c8) ^ (r & 7)) << 2));
            const float4 bq = *reinterpret_cast<const float4*>(stage + r * 32 + (((2 * c8 + 1) ^ (r & 7)) << 2));
            float v[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
            if (gated) {
              const uint4 gu = *reinterpret_cast<const uint4*>(gs + r * GLD + col);
              const T* gh = reinterpret_cast<const T*>(&gu);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] *= sigmoid_fast(to_f32(gh[e]));
            }
            uint4 u;
            T* h = reinterpret_cast<T*>(&u);
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[e]);
            *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + off) = u;
          }
        }
        __syncthreads();
      }
    }
  }
  // the other warps' epilogue reads of TMEM must finish before the allocation is released
  __syncwarp();
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// Decode-shaped calls (S * G <= 16 query rows, e.g. one token of 8 GQA heads).
// A CTA owns one (sequence, kv head) and one key split.  K/V chunks of 64 keys
// arrive by TMA (128-byte swizzle, up to MAX_STAGES chunks in flight), and the
// four warps split every chunk: warp w takes keys [16w, 16w + 16) with its own
// online softmax on mma.sync m16n8k16, so a chunk is four independent
// dependency chains instead of one.  At the end the warps' (max, sum, O) are
// merged through shared memory and the CTA writes either the final gated rows
// (one split) or one partial per row for kv_combine_kernel.  The new cache rows
// are copied from k_new / v_new into the landed tiles and into the cache by the
// warp that owns them.  V rows past the split end are zeroed in shared memory.
constexpr int DC_KC = 64;  // keys per chunk: 16 per warp

template <int HD>
struct DcLayout {
  static constexpr int NKB = HD / 64;
  static constexpr int KV_BLK = DC_KC * 128;                    // [64 keys][128 B] per 64-column block
  static constexpr int STAGE = 2 * NKB * KV_BLK;                 // K blocks, then V blocks
  static constexpr int OFF_Q = 0;                                // [NKB][16 rows][128 B]
  static constexpr int OFF_ST = NKB * 16 * 128;                  // stages (and the merge slab after the loop)
  static constexpr int SLAB_LD = HD + 8;                         // floats per merge-slab row (bank spread)
  static constexpr int SLAB = 4 * 16 * SLAB_LD * 4;
  static constexpr int MAX_STAGES = HD == 256 ? 2 : HD == 128 ? 3 : 4;
  static size_t smem_bytes(int stages) {
    const size_t st = (size_t)stages * STAGE;
    return (size_t)OFF_ST + (st > (size_t)SLAB ? st : (size_t)SLAB) + 1024;
  }
};

template <typename T, int HD>
__global__ void __launch_bounds__(128, 1)
kv_decode_kernel(const __grid_constant__ KvTcMaps maps, KvParams p, int n_stages) {
  griddep_wait();
  using L = DcLayout<HD>;
  constexpr int NKB = L::NKB;
  constexpr int NTILE_O = HD / 8;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[L::MAX_STAGES];
  __shared__ float s_m[4][16], s_l[4][16];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int G = p.Hq / p.Hkv;
  const int R = p.S * G;
  const int bh = blockIdx.y, b = bh / p.Hkv, kvh = bh % p.Hkv;
  const int split = blockIdx.x;
  const int k_begin = p.key_lo + split * p.ks;
  const int k_end = min(p.key_hi, k_begin + p.ks);
  const int nch = k_end > k_begin ? (k_end - k_begin + DC_KC - 1) / DC_KC : 0;
  const int NS = n_stages;
  const uint32_t sbase = tc::smem_u32(sm);
  const uint32_t full0 = tc::smem_u32(&full[0]);

  T* Kc = reinterpret_cast<T*>(p.kc) + (long long)b * p.bs + (long long)kvh * p.hs;
  T* Vc = reinterpret_cast<T*>(p.vc) + (long long)b * p.bs + (long long)kvh * p.hs;
  const T* kn = p.has_new ? reinterpret_cast<const T*>(p.k_new) + (long long)bh * p.S * HD : nullptr;
  const T* vn = p.has_new ? reinterpret_cast<const T*>(p.v_new) + (long long)bh * p.S * HD : nullptr;

  auto issue = [&](int c) {  // chunk c into stage c % NS
    const int st = c % NS;
    const uint32_t fb = full0 + 8u * st;
    tc::mbar_arrive_expect_tx(fb, (uint32_t)L::STAGE);
    const int key0 = k_begin + c * DC_KC;
#pragma unroll
    for (int cb = 0; cb < NKB; ++cb) {
      const uint32_t dk = sbase + L::OFF_ST + st * L::STAGE + cb * L::KV_BLK;
      const uint32_t dv = dk + NKB * L::KV_BLK;
      if (p.B > 1) {
        tc::tma_load_4d(dk, &maps.k, cb * 64, key0, kvh, b, fb);
        tc::tma_load_4d(dv, &maps.v, cb * 64, key0, kvh, b, fb);
      } else {
        tc::tma_load_3d(dk, &maps.k, cb * 64, key0, kvh, fb);
        tc::tma_load_3d(dv, &maps.v, cb * 64, key0, kvh, fb);
      }
    }
  };

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) tc::mbar_init(&full[s], 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int c = 0; c < NS && c < nch; ++c) issue(c);

  // Q tile: 16 rows (rows >= R are zero), swizzled like the TMA tiles
  if (p.fused) {  // S == 1: row r = head kvh G + r, read from the projection output, normed and rotated
    constexpr int EPL = HD / 32;
    for (int r = warp; r < 16; r += 4) {
      float x[EPL];
      if (r < R) {
        const T* src = reinterpret_cast<const T*>(p.q) + (long long)b * p.qkv_ld + (long long)(kvh * G + r) * 2 * HD +
                       lane * EPL;
        if constexpr (EPL == 8) {
          load8(src, x);
        } else {
#pragma unroll
          for (int e = 0; e < EPL; ++e) x[e] = to_f32(src[e]);
        }
        head_norm_rope_warp<T, EPL>(x, p.qnw, p.cos_t + (long long)p.pos * HD, p.sin_t + (long long)p.pos * HD, p.eps,
                                    lane);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) x[e] = 0.f;
      }
      const int ch = lane * EPL / 8;  // this lane's 16-byte chunk (half of it when EPL == 4)
      uint8_t* dst = sm + L::OFF_Q + (ch >> 3) * 2048 + swz128(r, ch & 7) + (EPL == 4 ? (lane & 1) * 8 : 0);
      if constexpr (EPL == 8) {
        store8(reinterpret_cast<T*>(dst), x);
      } else {
        T h4[4] = {from_f32<T>(x[0]), from_f32<T>(x[1]), from_f32<T>(x[2]), from_f32<T>(x[3])};
        *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(h4);
      }
    }
  } else
  for (int i = tid; i < 16 * (HD / 8); i += 128) {
    const int r = i / (HD / 8), c = i % (HD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < R) {
      const int s = r / G, h = kvh * G + r % G;
      v = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) + ((long long)(b * p.Hq + h) * p.S + s) * HD +
                                          c * 8);
    }
    *reinterpret_cast<uint4*>(sm + L::OFF_Q + (c >> 3) * 2048 + swz128(r, c & 7)) = v;
  }

  // visibility of this thread's rows g and g + 8
  int rows_s[2], rows_lo[2], rows_hi[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + h * 8;
    const int s = r < R ? r / G : 0;
    rows_s[h] = s;
    const int pq = p.pos + s;
    int lo = 0;
    if (p.window > 0) lo = p.aligned ? max(0, min(p.pos + p.S, p.ctx) - p.window) : pq - p.window + 1;
    rows_lo[h] = lo;
    rows_hi[h] = r < R ? pq : -1;
  }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o_acc[NTILE_O][4];
#pragma unroll
  for (int i = 0; i < NTILE_O; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;

  bool ok = true;
  int c = 0;
#pragma unroll 1
  for (; c < nch; ++c) {
    const int st = c % NS;
    // the barrier also means every warp is done with chunk c - 1, whose stage is then refilled
    // (with NS >= 2 that stage is not the one waited for here; with one stage the refill comes first)
    if (NS == 1 && c >= 1) {  // one stage: every warp is done with chunk c - 1, refill it with chunk c
      __syncthreads();
      if (tid == 0) issue(c);
    }
    ok = __syncthreads_and(tc::mbar_wait(full0 + 8u * st, (uint32_t)((c / NS) & 1)));
    if (!ok) break;
    if (tid == 0 && NS >= 2 && c >= 1 && c - 1 + NS < nch) issue(c - 1 + NS);
    uint8_t* Kt = sm + L::OFF_ST + st * L::STAGE;
    uint8_t* Vt = Kt + NKB * L::KV_BLK;
    const int key0 = k_begin + c * DC_KC;
    const int kw0 = key0 + warp * 16;  // this warp's first key

    // new rows into the landed tiles (and the cache); V rows past the split end zeroed
    bool touched = false;
    if (p.has_new && p.fused) {  // S == 1: the row at pos, K normed and rotated on the way in
      if (p.pos >= kw0 && p.pos < min(kw0 + 16, k_end)) {
        touched = true;
        constexpr int EPL = HD / 32;
        const long long src = (long long)b * p.qkv_ld + (long long)kvh * HD + lane * EPL;
        float x[EPL];
        const T* ks = reinterpret_cast<const T*>(p.k_new) + src;
        const T* vs = reinterpret_cast<const T*>(p.v_new) + src;
        if constexpr (EPL == 8) {
          load8(ks, x);
        } else {
#pragma unroll
          for (int e = 0; e < EPL; ++e) x[e] = to_f32(ks[e]);
        }
        head_norm_rope_warp<T, EPL>(x, p.knw, p.cos_t + (long long)p.pos * HD, p.sin_t + (long long)p.pos * HD,
                                    p.eps, lane);
        const int r = p.pos - key0, ch = lane * EPL / 8;
        const uint32_t so = (ch >> 3) * L::KV_BLK + swz128(r, ch & 7) + (EPL == 4 ? (lane & 1) * 8 : 0);
        T* kc_row = Kc + (long long)p.pos * HD + lane * EPL;
        T* vc_row = Vc + (long long)p.pos * HD + lane * EPL;
        if constexpr (EPL == 8) {
          store8(reinterpret_cast<T*>(Kt + so), x);
          store8(kc_row, x);
          const uint4 vv = *reinterpret_cast<const uint4*>(vs);
          *reinterpret_cast<uint4*>(Vt + so) = vv;
          *reinterpret_cast<uint4*>(vc_row) = vv;
        } else {
          T h4[4] = {from_f32<T>(x[0]), from_f32<T>(x[1]), from_f32<T>(x[2]), from_f32<T>(x[3])};
          *reinterpret_cast<uint2*>(Kt + so) = *reinterpret_cast<const uint2*>(h4);
          *reinterpret_cast<uint2*>(kc_row) = *reinterpret_cast<const uint2*>(h4);
          const uint2 vv = *reinterpret_cast<const uint2*>(vs);
          *reinterpret_cast<uint2*>(Vt + so) = vv;
          *reinterpret_cast<uint2*>(vc_row) = vv;
        }
      }
    } else if (p.has_new) {
      const int j0 = max(kw0, p.pos), j1 = min(min(kw0 + 16, k_end), p.pos + p.S);
      if (j1 > j0) {
        touched = true;
        for (int i = lane; i < (j1 - j0) * (HD / 8); i += 32) {
          const int j = j0 + i / (HD / 8), ch = i % (HD / 8), r = j - key0;
          const uint4 kv = *reinterpret_cast<const uint4*>(kn + (long long)(j - p.pos) * HD + ch * 8);
          const uint4 vv = *reinterpret_cast<const uint4*>(vn + (long long)(j - p.pos) * HD + ch * 8);
          *reinterpret_cast<uint4*>(Kt + (ch >> 3) * L::KV_BLK + swz128(r, ch & 7)) = kv;
          *reinterpret_cast<uint4*>(Vt + (ch >> 3) * L::KV_BLK + swz128(r, ch & 7)) = vv;
          *reinterpret_cast<uint4*>(Kc + (long long)j * HD + ch * 8) = kv;
          *reinterpret_cast<uint4*>(Vc + (long long)j * HD + ch * 8) = vv;
        }
      }
    }
    if (kw0 + 16 > k_end) {
      const int z0 = max(kw0, k_end);
      touched = true;
      for (int i = lane; i < (kw0 + 16 - z0) * NKB * 8; i += 32) {
        const int r = z0 - key0 + i / (NKB * 8), cb = (i / 8) % NKB, u = i % 8;
        *reinterpret_cast<uint4*>(Vt + cb * L::KV_BLK + r * 128 + u * 16) = make_uint4(0, 0, 0, 0);
      }
    }
    if (touched) tc::fence_async_smem();  // these generic writes precede the stage's next TMA refill
    __syncwarp();

    // S = Q K^T: 16 rows x 16 keys, two accumulator sets to halve the dependency chain
    float sc[2][2][4];
#pragma unroll
    for (int a2 = 0; a2 < 2; ++a2)
#pragma unroll
      for (int n = 0; n < 2; ++n) sc[a2][n][0] = sc[a2][n][1] = sc[a2][n][2] = sc[a2][n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t a[4], bfr[4];
      {
        const int r = lane & 15, ch = kk * 2 + (lane >> 4);
        ldmatrix_x4(a, sm + L::OFF_Q + (ch >> 3) * 2048 + swz128(r, ch & 7));
      }
      {
        const int r = warp * 16 + (lane & 7) + ((lane >> 4) << 3), ch = kk * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(bfr, Kt + (ch >> 3) * L::KV_BLK + swz128(r, ch & 7));
      }
      mma_16816<T>(sc[kk & 1][0], a, bfr[0], bfr[1]);
      mma_16816<T>(sc[kk & 1][1], a, bfr[2], bfr[3]);
    }
    // scale, mask, online softmax (base 2)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int j = kw0 + n * 8 + t4 * 2 + (e & 1);
        float v = (sc[0][n][e] + sc[1][n][e]) * p.scale_log2;
        bool vis = j < k_end;
        if (p.mask) {
          if (vis && rows_hi[h] >= 0) {
            const long long mi = (long long)rows_s[h] * p.mask_ld + j;
            const float mv = p.mask_dtype == ANEMLL_F32 ? reinterpret_cast<const float*>(p.mask)[mi]
                           : p.mask_dtype == ANEMLL_F16 ? __half2float(reinterpret_cast<const __half*>(p.mask)[mi])
                           : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.mask)[mi]);
            v += mv * 1.4426950408889634f;
          } else {
            vis = false;
          }
          if (v == -INFINITY) vis = false;
        } else {
          vis = vis && j <= rows_hi[h] && j >= rows_lo[h];
        }
        v = vis ? v : -INFINITY;
        sc[0][n][e] = v;
        mx[h] = fmaxf(mx[h], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float mnew = fmaxf(m_run[h], mx[h]);
      const float base = mnew == -INFINITY ? 0.f : mnew;
      alpha[h] = fast_exp2(m_run[h] - base);
      m_run[h] = mnew;
      mx[h] = base;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const float p0 = fast_exp2(sc[0][n][0] - mx[0]);
      const float p1 = fast_exp2(sc[0][n][1] - mx[0]);
      const float p2 = fast_exp2(sc[0][n][2] - mx[1]);
      const float p3 = fast_exp2(sc[0][n][3] - mx[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      pf[n * 2 + 0] = pack2<T>(p0, p1);
      pf[n * 2 + 1] = pack2<T>(p2, p3);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      l_run[h] = l_run[h] * alpha[h] + rs[h];
    }
    // O = alpha O + P V
#pragma unroll
    for (int n2 = 0; n2 < HD / 16; ++n2) {
      uint32_t bfr[4];
      const int r = warp * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), ch = n2 * 2 + (lane >> 4);
      ldmatrix_x4_trans(bfr, Vt + (ch >> 3) * L::KV_BLK + swz128(r, ch & 7));
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        float* o = o_acc[2 * n2 + q2];
        o[0] *= alpha[0];
        o[1] *= alpha[0];
        o[2] *= alpha[1];
        o[3] *= alpha[1];
        mma_16816<T>(o, pf, bfr[2 * q2], bfr[2 * q2 + 1]);
      }
    }
  }
  if (!ok) {
    atomicExch(&g_kv_tc_error, 1);
    // chunks issued and not consumed, [c, issued_end), may still be landing: wait for them
    // (bounded) before the CTA exits.  Chunks [0, NS) are issued up front and iteration
    // c' >= 1 issues chunk c' - 1 + NS, so issued_end = min(nch, max(NS, c - 1 + NS)); with one
    // stage iteration c issues chunk c itself, before its wait.
    const int issued_end = NS == 1 ? min(nch, c + 1) : min(nch, c == 0 ? NS : c - 1 + NS);
    for (int x = c; x < issued_end; ++x) tc::mbar_wait(full0 + 8u * (x % NS), (uint32_t)((x / NS) & 1));
    return;  // block-uniform: ok came from __syncthreads_and
  }

  griddep_launch_dependents();
  // ---- merge the four warps' partial softmax states through shared memory ----
  if (t4 == 0) {
    s_m[warp][g] = m_run[0];
    s_m[warp][g + 8] = m_run[1];
  }
  __syncthreads();  // also: every warp is done with the stage memory the slab reuses
  float* slab = reinterpret_cast<float*>(sm + L::OFF_ST);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + h * 8;
    float M = s_m[0][r];
#pragma unroll
    for (int w = 1; w < 4; ++w) M = fmaxf(M, s_m[w][r]);
    const float f = m_run[h] == -INFINITY ? 0.f : fast_exp2(m_run[h] - M);
    if (t4 == 0) s_l[warp][r] = l_run[h] * f;
    float* row = slab + (warp * 16 + r) * L::SLAB_LD + t4 * 2;
#pragma unroll
    for (int i = 0; i < NTILE_O; ++i)
      *reinterpret_cast<float2*>(row + i * 8) = make_float2(o_acc[i][2 * h] * f, o_acc[i][2 * h + 1] * f);
  }
  __syncthreads();
  for (int idx = tid; idx < R * (HD / 4); idx += 128) {
    const int r = idx / (HD / 4), d = (idx % (HD / 4)) * 4;
    float4 o = *reinterpret_cast<const float4*>(slab + r * L::SLAB_LD + d);
    float Ls = s_l[0][r], M = s_m[0][r];
#pragma unroll
    for (int w = 1; w < 4; ++w) {
      const float4 x = *reinterpret_cast<const float4*>(slab + (w * 16 + r) * L::SLAB_LD + d);
      o.x += x.x;
      o.y += x.y;
      o.z += x.z;
      o.w += x.w;
      Ls += s_l[w][r];
      M = fmaxf(M, s_m[w][r]);
    }
    if (p.n_splits == 1) {
      const int s = r / G, hq = kvh * G + r % G;
      const long long off = ((long long)b * p.S + s) * p.Hq * HD + (long long)hq * HD + d;
      const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
      float v[4] = {o.x * inv, o.y * inv, o.z * inv, o.w * inv};
      if (p.gate) {
        const uint2 gu = *reinterpret_cast<const uint2*>(reinterpret_cast<const T*>(p.gate) + gate_index(p, b, s, hq, d));
        const T* gh = reinterpret_cast<const T*>(&gu);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] *= sigmoid_fast(to_f32(gh[e]));
      }
      uint2 u;
      T* hh = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) hh[e] = from_f32<T>(v[e]);
      *reinterpret_cast<uint2*>(reinterpret_cast<T*>(p.out) + off) = u;
    } else {
      const long long row_id = ((long long)bh * p.n_splits + split) * R + r;
      *reinterpret_cast<float4*>(p.ws_o + row_id * HD + d) = o;
      if (d == 0) {
        p.ws_ml[row_id * 2 + 0] = M;
        p.ws_ml[row_id * 2 + 1] = Ls;
      }
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 kv_map_encoder() {
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

int kv_encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
              const cuuint32_t* box, CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT16) {
  auto enc = kv_map_encoder();
  ANEMLL_REQUIRE(enc, ANEMLL_EUNSUPPORTED, "kv_attention: cuTensorMapEncodeTiled unavailable");
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides,
                         box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  ANEMLL_REQUIRE(r == CUDA_SUCCESS, ANEMLL_EINVAL, "kv_attention: tensor map encoding failed (%d)", (int)r);
  return ANEMLL_OK;
}

// K and V cache maps: [hd, ctx, H_kv(, B)] with 64-element x 64-key boxes, 128-byte swizzle.
int kv_cache_maps(KvTcMaps& maps, const KvParams& p, int HD) {
  static_assert(TC_KB == DC_KC, "prefill and decode kernels share the 64-key cache box");
  const cuuint32_t bk[4] = {64, (cuuint32_t)TC_KB, 1, 1};
  int rc;
  if (p.B > 1) {
    const cuuint64_t dk[4] = {(cuuint64_t)HD, (cuuint64_t)p.ctx, (cuuint64_t)p.Hkv, (cuuint64_t)p.B};
    const cuuint64_t sk[3] = {(cuuint64_t)HD * 2, (cuuint64_t)p.hs * 2, (cuuint64_t)p.bs * 2};
    rc = kv_encode(&maps.k, p.kc, 4, dk, sk, bk);
    if (!rc) rc = kv_encode(&maps.v, p.vc, 4, dk, sk, bk);
  } else {
    const cuuint64_t dk[3] = {(cuuint64_t)HD, (cuuint64_t)p.ctx, (cuuint64_t)p.Hkv};
    const cuuint64_t sk[2] = {(cuuint64_t)HD * 2, (cuuint64_t)p.hs * 2};
    rc = kv_encode(&maps.k, p.kc, 3, dk, sk, bk);
    if (!rc) rc = kv_encode(&maps.v, p.vc, 3, dk, sk, bk);
  }
  return rc;
}

// Decode kernel: at most 16 query rows, cache strides whole 16-byte units, 8-byte aligned out / gate.
bool dec_eligible(int S, int Hq, int Hkv, long long bs, long long hs, const void* out, const void* gate) {
  return (long long)S * (Hq / Hkv) <= 16 && (hs * 2) % 16 == 0 && (bs * 2) % 16 == 0 && aligned(out, 8) &&
         (!gate || aligned(gate, 8));
}

template <typename T, int HD>
int launch_kv_dec(KvParams& p, const Plan& pl0, cudaStream_t st) {
  using L = DcLayout<HD>;
  // about two CTAs per SM, never more splits than the generic plan (workspace bound)
  const int Lk = p.key_hi - p.key_lo;
  const int nchunks = max(1, (Lk + DC_KC - 1) / DC_KC);
  const long base = (long)p.B * p.Hkv;
  int want = (int)((2L * 148 + base - 1) / base);
  want = max(1, min(want, min(nchunks, pl0.n_splits)));
  const int cps = (nchunks + want - 1) / want;  // chunks per split
  const int ks = cps * DC_KC;
  const int n_splits = max(1, (Lk + ks - 1) / ks);
  // One K/V stage when the grid holds two CTAs per SM at hd 256: two resident CTAs (eight warps)
  // hide each other's loads better than one CTA with a second stage (batch 128: 80 -> 70 us a call).
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool two_per_sm = HD == 256 && (long)n_splits * base >= 2L * sms;
  const int stages = two_per_sm ? 1 : min(cps, L::MAX_STAGES);
  KvParams q = p;
  q.n_splits = n_splits;
  q.ks = ks;
  if (n_splits > 1) {
    const size_t R = (size_t)p.S * (p.Hq / p.Hkv);
    q.ws_ml = q.ws_o + (size_t)p.B * p.Hkv * n_splits * R * HD;
  }
  KvTcMaps maps;
  int rc = kv_cache_maps(maps, p, HD);
  if (rc) return rc;
  const size_t smem = L::smem_bytes(stages);
  auto kern = kv_decode_kernel<T, HD>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(n_splits, p.B * p.Hkv);
  rc = launch_pdl("kv_attention_decode", kern, grid, dim3(128), smem, st, maps, q, stages);
  if (rc) return rc;
  if (n_splits > 1) {
    rc = launch_combine<T, HD>(q, st);
  }
  return rc;
}

// New rows k_new / v_new [B][H_kv][S][HD] -> cache rows [pos, pos + S), 16-byte vectors.  The tcgen05
// prefill path runs this first for chunks of TC_PREWRITE_MIN tokens or more: its attention kernel
// then reads every row, new or old, with TMA and no block has rows to patch.
constexpr int TC_PREWRITE_MIN = 128;

template <typename T, int HD>
__global__ void __launch_bounds__(256)
kv_write_rows_kernel(const T* __restrict__ kn, const T* __restrict__ vn, T* __restrict__ kc, T* __restrict__ vc,
                     int Hkv, int S, int pos, long long bs, long long hs, long long n_vec) {
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  if (i >= n_vec) return;
  constexpr int VPR = HD / 8;  // 16-byte vectors per row
  const long long row = i / VPR;  // (b, h, s)
  const int v = (int)(i % VPR), s = (int)(row % S);
  const long long bh = row / S;
  const int h = (int)(bh % Hkv), b = (int)(bh / Hkv);
  const long long dst = (long long)b * bs + (long long)h * hs + (long long)(pos + s) * HD + v * 8;
  reinterpret_cast<uint4*>(kc + dst)[0] = reinterpret_cast<const uint4*>(kn + row * HD + v * 8)[0];
  reinterpret_cast<uint4*>(vc + dst)[0] = reinterpret_cast<const uint4*>(vn + row * HD + v * 8)[0];
}

// Fused form: a warp per new row; K rows normed (k_norm) and rotated at their position, V rows moved;
// both read in place from the q/k/v projection output.
template <typename T, int HD>
__global__ void __launch_bounds__(256)
kv_write_rows_fused_kernel(KvParams p) {
  constexpr int EPL = HD / 32;
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);  // (b, h, s), s fastest
  const int lane = threadIdx.x & 31;
  if (row >= (long long)p.B * p.Hkv * p.S) return;
  const int s = (int)(row % p.S);
  const long long bh = row / p.S;
  const int h = (int)(bh % p.Hkv), b = (int)(bh / p.Hkv);
  const long long src = ((long long)b * p.S + s) * p.qkv_ld + (long long)h * HD + lane * EPL;
  const long long dst = (long long)b * p.bs + (long long)h * p.hs + (long long)(p.pos + s) * HD + lane * EPL;
  float x[EPL];
  const T* kn = reinterpret_cast<const T*>(p.k_new) + src;
  if constexpr (EPL == 8) {
    load8(kn, x);
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) x[e] = to_f32(kn[e]);
  }
  head_norm_rope_warp<T, EPL>(x, p.knw, p.cos_t + (long long)(p.pos + s) * HD, p.sin_t + (long long)(p.pos + s) * HD,
                              p.eps, lane);
  T* kd = reinterpret_cast<T*>(p.kc) + dst;
  T* vd = reinterpret_cast<T*>(p.vc) + dst;
  const T* vs = reinterpret_cast<const T*>(p.v_new) + src;
  if constexpr (EPL == 8) {
    store8(kd, x);
    *reinterpret_cast<uint4*>(vd) = *reinterpret_cast<const uint4*>(vs);
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      kd[e] = from_f32<T>(x[e]);
      vd[e] = vs[e];
    }
  }
}

template <typename T, int HD>
int launch_kv_write_rows(const KvParams& p, cudaStream_t st) {
  if (p.fused) {
    const long long rows = (long long)p.B * p.Hkv * p.S;
    kv_write_rows_fused_kernel<T, HD><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(p);
    return launch_status("kv_attention_write_rows");
  }
  const long long n_vec = (long long)p.B * p.Hkv * p.S * (HD / 8);
  kv_write_rows_kernel<T, HD><<<(unsigned)((n_vec + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const T*>(p.k_new), reinterpret_cast<const T*>(p.v_new), reinterpret_cast<T*>(p.kc),
      reinterpret_cast<T*>(p.vc), p.Hkv, p.S, p.pos, p.bs, p.hs, n_vec);
  return launch_status("kv_attention_write_rows");
}

bool tc_eligible(int S, int Hq, int Hkv, int hd, long long bs, long long hs, const void* out, const void* gate) {
  return Hq / Hkv == 8 && (hd == 128 || hd == 256) && S >= 16 && (hs * 2) % 16 == 0 && (bs * 2) % 16 == 0 &&
         aligned(out, 16) && (!gate || aligned(gate, 16));
}

template <typename T, int HD>
int launch_kv_tc(KvParams& p, const Plan& pl0, cudaStream_t st) {
  // key split for 128-row tiles: about one wave, never more splits than the generic plan (workspace bound)
  const int row_tiles = (p.S + 15) / 16;
  const int L = p.key_hi - p.key_lo;
  const int nblocks = max(1, (L + TC_KB - 1) / TC_KB);
  const long base = (long)row_tiles * p.B * p.Hkv;
  int want = (int)(148 / base);  // one wave: every CTA holds a whole SM (shared memory)
  want = max(1, min(want, min(nblocks, pl0.n_splits)));
  const int bps = (nblocks + want - 1) / want;
  const int ks = bps * TC_KB;
  const int n_splits = max(1, (L + ks - 1) / ks);
  KvParams q = p;
  q.n_splits = n_splits;
  q.ks = ks;
  if (n_splits > 1) {
    const size_t R = (size_t)p.S * (p.Hq / p.Hkv);
    q.ws_ml = q.ws_o + (size_t)p.B * p.Hkv * n_splits * R * HD;
  }
  KvTcMaps maps;
  {
    int rc;
    if (p.fused) {  // the projection output: {column, token (qkv_ld), head (2 HD), sequence (S qkv_ld)}
      const cuuint64_t dq[4] = {(cuuint64_t)HD, (cuuint64_t)p.S, (cuuint64_t)p.Hq, (cuuint64_t)p.B};
      const cuuint64_t sq[3] = {(cuuint64_t)p.qkv_ld * 2, (cuuint64_t)HD * 4, (cuuint64_t)p.S * p.qkv_ld * 2};
      const cuuint32_t bq[4] = {64, 16, 8, 1};
      rc = kv_encode(&maps.q, p.q, 4, dq, sq, bq);
    } else {
      const cuuint64_t dq[3] = {(cuuint64_t)HD, (cuuint64_t)p.S, (cuuint64_t)p.B * p.Hq};
      const cuuint64_t sq[2] = {(cuuint64_t)HD * 2, (cuuint64_t)p.S * HD * 2};
      const cuuint32_t bq[3] = {64, 16, 8};
      rc = kv_encode(&maps.q, p.q, 3, dq, sq, bq);
    }
    if (!rc) rc = kv_cache_maps(maps, p, HD);
    if (!rc && n_splits > 1) {  // partials {column, token, head, (sequence, kv head, split)}, fp32
      const int G = p.Hq / p.Hkv;
      const cuuint64_t dm[4] = {(cuuint64_t)HD, (cuuint64_t)p.S, (cuuint64_t)G,
                                (cuuint64_t)p.B * p.Hkv * n_splits};
      const cuuint64_t sm4[3] = {(cuuint64_t)G * HD * 4, (cuuint64_t)HD * 4, (cuuint64_t)p.S * G * HD * 4};
      const cuuint32_t bm[4] = {32, 16, 8, 1};
      rc = kv_encode(&maps.o, q.ws_o, 4, dm, sm4, bm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
    }
    if (rc) return rc;
  }
  constexpr int NKB = HD / 64;
  const size_t smem = (size_t)NKB * 128 * 128 + 4 * (size_t)NKB * TC_KB * 128 + 128 * 128 + 1024;
  auto kern = kv_attn_tc_kernel<T, HD>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(row_tiles, n_splits, p.B * p.Hkv);
  int rc = launch_pdl("kv_attention_tc", kern, grid, dim3(TC_NT), smem, st, maps, q);
  if (rc) return rc;
  if (n_splits > 1) {
    rc = launch_combine<T, HD>(q, st);
  }
  return rc;
}

// tcgen05 prefill path: long chunks write their new rows with a copy kernel first (the attention
// kernel, launched dependent on it, waits for it before its first load), short ones patch them in.
template <typename T, int HD>
int launch_kv_tc_rows(KvParams& p, const Plan& pl, cudaStream_t st) {
  if (!p.has_new || (!p.fused && p.S < TC_PREWRITE_MIN)) return launch_kv_tc<T, HD>(p, pl, st);
  int rc = launch_kv_write_rows<T, HD>(p, st);
  if (rc) return rc;
  KvParams q = p;
  q.has_new = 0;
  q.k_new = q.v_new = nullptr;
  return launch_kv_tc<T, HD>(q, pl, st);
}

}  // namespace
}  // namespace anemll

using namespace anemll;

extern "C" int anemll_kv_attention_error(int reset) {
  int h = 0;
  if (cudaMemcpyFromSymbol(&h, g_kv_tc_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && h) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_kv_tc_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return h;
}

extern "C" size_t anemll_kv_attention_workspace_size(int B, int S, int H_q, int H_kv, int head_dim, int ctx) {
  if (B <= 0 || S <= 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv || ctx <= 0) return 0;
  // max_splits bounds the split count of every key range this shape can take
  Plan pl = make_plan(B, S, H_q, H_kv, ctx, 0, 0, 0, true);
  return workspace_bytes_for(pl.max_splits, B, S, H_q, H_kv, head_dim);
}

namespace anemll {
namespace {

// the fused q/k head norm + RoPE inputs of anemll_kv_attention_qkv
struct FusedQkv {
  long long ld;
  const float* qn;
  const float* kn;
  const float* cos_t;
  const float* sin_t;
  float eps;
};

int kv_attention_run(const void* q, const void* k_new, const void* v_new, const void* gate, void* k_cache,
                     void* v_cache, int64_t cache_batch_stride, int64_t cache_head_stride, const void* mask,
                     int mask_dtype, int64_t mask_row_stride, void* out, int dtype, int B, int S, int H_q, int H_kv,
                     int head_dim, int ctx, int current_pos, int window, int window_chunk_aligned, void* workspace,
                     size_t workspace_bytes, void* stream, const FusedQkv* fz) {
  ANEMLL_REQUIRE(q && k_cache && v_cache && out, ANEMLL_EINVAL, "kv_attention: null pointer");
  ANEMLL_REQUIRE((k_new == nullptr) == (v_new == nullptr), ANEMLL_EINVAL,
                 "kv_attention: k_new and v_new must both be given or both be NULL");
  ANEMLL_REQUIRE(B > 0 && S > 0 && H_q > 0 && H_kv > 0 && ctx > 0, ANEMLL_EINVAL, "kv_attention: bad sizes");
  ANEMLL_REQUIRE(H_q % H_kv == 0, ANEMLL_EINVAL, "kv_attention: H_q %% H_kv != 0");
  ANEMLL_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, ANEMLL_EUNSUPPORTED,
                 "kv_attention: head_dim must be 64, 128 or 256 (got %d)", head_dim);
  ANEMLL_REQUIRE(current_pos >= 0 && (int64_t)current_pos + S <= ctx, ANEMLL_EINVAL,
                 "kv_attention: positions [%d, %lld) exceed the cache length %d", current_pos,
                 (long long)current_pos + S, ctx);
  ANEMLL_REQUIRE(!mask || (mask_dtype == ANEMLL_F32 || mask_dtype == ANEMLL_F16 || mask_dtype == ANEMLL_BF16),
                 ANEMLL_EUNSUPPORTED, "kv_attention: bad mask dtype");
  ANEMLL_REQUIRE(!mask || mask_row_stride >= ctx, ANEMLL_EINVAL, "kv_attention: mask row stride < ctx");
  ANEMLL_REQUIRE(aligned(q, 16) && (!k_new || (aligned(k_new, 16) && aligned(v_new, 16))) && aligned(k_cache, 16) &&
                     aligned(v_cache, 16) && aligned(out, 4) && (!gate || aligned(gate, 4)),
                 ANEMLL_EALIGN, "kv_attention: q/k_new/v_new/caches must be 16-byte aligned");
  ANEMLL_REQUIRE(cache_batch_stride % 8 == 0 && cache_head_stride % 8 == 0, ANEMLL_EALIGN,
                 "kv_attention: cache strides must be multiples of 8 elements");
  Plan pl = make_plan(B, S, H_q, H_kv, ctx, current_pos, window, window_chunk_aligned, mask != nullptr);
  const size_t need = workspace_bytes_for(pl.n_splits, B, S, H_q, H_kv, head_dim);
  ANEMLL_REQUIRE(workspace_bytes >= need && (need == 0 || workspace), ANEMLL_EWORKSPACE,
                 "kv_attention: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  ANEMLL_REQUIRE(!workspace || aligned(workspace, 16), ANEMLL_EALIGN, "kv_attention: workspace must be 16-byte aligned");

  KvParams p;
  p.q = q; p.k_new = k_new; p.v_new = v_new; p.gate = gate; p.kc = k_cache; p.vc = v_cache;
  p.bs = cache_batch_stride; p.hs = cache_head_stride;
  p.mask = mask; p.mask_dtype = mask_dtype; p.mask_ld = mask_row_stride;
  p.out = out;
  p.B = B; p.S = S; p.Hq = H_q; p.Hkv = H_kv; p.ctx = ctx;
  p.pos = current_pos; p.window = window; p.aligned = window_chunk_aligned; p.has_new = k_new != nullptr;
  p.key_lo = pl.key_lo; p.key_hi = pl.key_hi; p.n_splits = pl.n_splits; p.ks = pl.ks;
  const size_t R = (size_t)S * (H_q / H_kv);
  p.ws_o = reinterpret_cast<float*>(workspace);
  p.ws_ml = p.ws_o ? p.ws_o + (size_t)B * H_kv * pl.n_splits * R * head_dim : nullptr;
  p.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  p.gate_ts = (long long)H_q * head_dim;
  p.gate_hs = head_dim;
  p.fused = 0;
  p.qkv_ld = 0;
  p.qnw = p.knw = p.cos_t = p.sin_t = nullptr;
  p.eps = 0.f;
  cudaStream_t st = (cudaStream_t)stream;
  const bool use_tc = tc_eligible(S, H_q, H_kv, head_dim, cache_batch_stride, cache_head_stride, out, gate);
  const bool use_dec = !use_tc && dec_eligible(S, H_q, H_kv, cache_batch_stride, cache_head_stride, out, gate);
  if (fz) {
    ANEMLL_REQUIRE(use_tc || (use_dec && S == 1 && head_dim != 64), ANEMLL_EUNSUPPORTED,
                   "kv_attention_qkv: fused head norm needs a tcgen05 prefill chunk (8 query heads per kv head, "
                   "head_dim 128/256, 16+ tokens) or a one-token decode step");
    p.fused = 1;
    p.qkv_ld = fz->ld;
    p.qnw = fz->qn;
    p.knw = fz->kn;
    p.cos_t = fz->cos_t;
    p.sin_t = fz->sin_t;
    p.eps = fz->eps;
    p.gate_ts = fz->ld;  // gate columns of head h follow its query columns
    p.gate_hs = 2LL * head_dim;
  }
  return ANEMLL_DISPATCH_HALF(dtype, T, [&] {
    switch (head_dim) {
      case 64: return use_dec ? launch_kv_dec<T, 64>(p, pl, st) : launch_kv<T, 64>(p, pl, st);
      case 128:
        return use_tc ? launch_kv_tc_rows<T, 128>(p, pl, st)
               : use_dec ? launch_kv_dec<T, 128>(p, pl, st)
                         : launch_kv<T, 128>(p, pl, st);
      default:
        return use_tc ? launch_kv_tc_rows<T, 256>(p, pl, st)
               : use_dec ? launch_kv_dec<T, 256>(p, pl, st)
                         : launch_kv<T, 256>(p, pl, st);
    }
  });
}

}  // namespace
}  // namespace anemll

extern "C" int anemll_kv_attention(const void* q, const void* k_new, const void* v_new, const void* gate,
                                   void* k_cache, void* v_cache, int64_t cache_batch_stride, int64_t cache_head_stride,
                                   const void* mask, int mask_dtype, int64_t mask_row_stride,
                                   void* out, int dtype,
                                   int B, int S, int H_q, int H_kv, int head_dim, int ctx,
                                   int current_pos, int window, int window_chunk_aligned,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  return kv_attention_run(q, k_new, v_new, gate, k_cache, v_cache, cache_batch_stride, cache_head_stride, mask,
                          mask_dtype, mask_row_stride, out, dtype, B, S, H_q, H_kv, head_dim, ctx, current_pos, window,
                          window_chunk_aligned, workspace, workspace_bytes, stream, nullptr);
}

extern "C" int anemll_kv_attention_qkv(const void* qkv, int64_t qkv_row_stride, const float* q_norm,
                                       const float* k_norm, const float* cos_table, const float* sin_table, float eps,
                                       void* k_cache, void* v_cache, int64_t cache_batch_stride,
                                       int64_t cache_head_stride, void* out, int dtype, int B, int S, int H_q,
                                       int H_kv, int head_dim, int ctx, int current_pos, int window,
                                       int window_chunk_aligned, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  ANEMLL_REQUIRE(qkv && q_norm && k_norm && cos_table && sin_table, ANEMLL_EINVAL, "kv_attention_qkv: null pointer");
  ANEMLL_REQUIRE(aligned(q_norm, 16) && aligned(cos_table, 16) && aligned(sin_table, 16), ANEMLL_EALIGN,
                 "kv_attention_qkv: q_norm and the cos/sin tables must be 16-byte aligned");
  ANEMLL_REQUIRE(dtype == ANEMLL_F16 || dtype == ANEMLL_BF16, ANEMLL_EUNSUPPORTED, "kv_attention_qkv: fp16 or bf16");
  ANEMLL_REQUIRE(H_q > 0 && H_kv > 0 && head_dim > 0 &&
                     qkv_row_stride >= 2LL * H_q * head_dim + 2LL * H_kv * head_dim && qkv_row_stride % 8 == 0,
                 ANEMLL_EINVAL, "kv_attention_qkv: the q/k/v row stride is shorter than a row or not 16-byte units");
  const uint8_t* base = reinterpret_cast<const uint8_t*>(qkv);
  const long long es = 2;
  const void* q = base;
  const void* gate = base + (long long)head_dim * es;
  const void* k_new = base + 2LL * H_q * head_dim * es;
  const void* v_new = base + (2LL * H_q + H_kv) * head_dim * es;
  const FusedQkv fz{qkv_row_stride, q_norm, k_norm, cos_table, sin_table, eps};
  return kv_attention_run(q, k_new, v_new, gate, k_cache, v_cache, cache_batch_stride, cache_head_stride, nullptr, 0,
                          0, out, dtype, B, S, H_q, H_kv, head_dim, ctx, current_pos, window, window_chunk_aligned,
                          workspace, workspace_bytes, stream, &fz);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of anemll_kv_attention.
//
// Some callers cannot hand us a workspace or allocate one at call time: engines
// that reserve all device memory when they start and forbid any later
// cudaMalloc, and loops that cannot afford cudaMalloc/cudaFree because those
// calls synchronise the whole device.  This entry point takes the split-KV
// scratch from a fixed array that the library itself owns instead.
//
// - Limit: KV_NOALLOC_SCRATCH_BYTES (8 MiB).  Every GPU that loads this
//   library holds that array until the process exits.  Shapes whose scratch
//   need exceeds it are rejected (ANEMLL_EWORKSPACE) before anything launches.
// - Set-up: the first call on a device, with that device current, looks up the
//   array's device address (cudaGetSymbolAddress) and caches it per device.
//   Make that first call before any stream capture on the device.
// - Sharing: all calls share one array.  Each call fully overwrites the part it
//   reads (every split writes all of its partial rows before the combine reads
//   them), so nothing has to start at zero, but two calls that overlap on the
//   GPU (different streams, or different host threads) race on the array.
// - The size check uses the split count of the generic split-KV plan, the
//   largest any path of this call can take; the tcgen05 and decode paths often
//   use fewer splits, so a call can be refused although its path would fit.
// - The cached address belongs to the device's primary context: do not use this
//   entry point after a cudaDeviceReset in the same process.
// - It never calls cudaMalloc, cudaFree or any allocating library routine.
#include <mutex>

namespace anemll {
namespace {

constexpr size_t KV_NOALLOC_SCRATCH_BYTES = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_kv_noalloc_scratch[KV_NOALLOC_SCRATCH_BYTES];

constexpr int KV_NOALLOC_MAX_DEVICES = 64;
std::mutex g_kv_noalloc_mu;
void* g_kv_noalloc_ptr[KV_NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch array on the current device (host code may not
// use the symbol itself: it is only a host-side stand-in for the device array).
int kv_noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("kv_attention_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return (int)e;
  }
  ANEMLL_REQUIRE(dev >= 0 && dev < KV_NOALLOC_MAX_DEVICES, ANEMLL_EUNSUPPORTED,
                 "kv_attention_noalloc: device ordinal %d beyond the supported %d", dev, KV_NOALLOC_MAX_DEVICES);
  std::lock_guard<std::mutex> lock(g_kv_noalloc_mu);
  if (!g_kv_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_kv_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("kv_attention_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(e));
      return e != cudaSuccess ? (int)e : ANEMLL_EINVAL;
    }
    g_kv_noalloc_ptr[dev] = p;
  }
  *out = g_kv_noalloc_ptr[dev];
  return ANEMLL_OK;
}

}  // namespace
}  // namespace anemll

extern "C" size_t anemll_kv_attention_noalloc_max_scratch(void) { return anemll::KV_NOALLOC_SCRATCH_BYTES; }

extern "C" int anemll_kv_attention_noalloc(const void* q, const void* k_new, const void* v_new, const void* gate,
                                           void* k_cache, void* v_cache, int64_t cache_batch_stride,
                                           int64_t cache_head_stride,
                                           const void* mask, int mask_dtype, int64_t mask_row_stride,
                                           void* out, int dtype,
                                           int B, int S, int H_q, int H_kv, int head_dim, int ctx,
                                           int current_pos, int window, int window_chunk_aligned, void* stream) {
  // sizes the plan needs; everything else is validated by anemll_kv_attention
  ANEMLL_REQUIRE(B > 0 && S > 0 && H_q > 0 && H_kv > 0 && H_q % H_kv == 0 && ctx > 0 && current_pos >= 0,
                 ANEMLL_EINVAL, "kv_attention_noalloc: bad sizes");
  ANEMLL_REQUIRE((int64_t)current_pos + S <= ctx, ANEMLL_EINVAL,
                 "kv_attention_noalloc: positions [%d, %lld) exceed the cache length %d", current_pos,
                 (long long)current_pos + S, ctx);
  ANEMLL_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, ANEMLL_EUNSUPPORTED,
                 "kv_attention_noalloc: head_dim must be 64, 128 or 256 (got %d)", head_dim);
  const Plan pl = make_plan(B, S, H_q, H_kv, ctx, current_pos, window, window_chunk_aligned, mask != nullptr);
  const size_t need = workspace_bytes_for(pl.n_splits, B, S, H_q, H_kv, head_dim);
  ANEMLL_REQUIRE(need <= KV_NOALLOC_SCRATCH_BYTES, ANEMLL_EWORKSPACE,
                 "kv_attention_noalloc: this call needs %zu bytes of scratch, above the built-in %zu-byte maximum; "
                 "use anemll_kv_attention with a caller-provided workspace",
                 need, KV_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int rc = kv_noalloc_scratch(&scratch);
  if (rc) return rc;
  return anemll_kv_attention(q, k_new, v_new, gate, k_cache, v_cache, cache_batch_stride, cache_head_stride, mask,
                             mask_dtype, mask_row_stride, out, dtype, B, S, H_q, H_kv, head_dim, ctx, current_pos,
                             window, window_chunk_aligned, scratch, KV_NOALLOC_SCRATCH_BYTES, stream);
}
