// ffn_kernels.cu -- CUDA kernels of the quantized expert-FFN path (sm_100a)
// and their host-side launchers.
//
// Reference (terox27/Flash1017-Engine, crates/flash-core/src/flash1017.rs):
//   NVFP4 matvec              :2331-2357     ternary matvec            :2602-2621
//   rank-16 Q8 core           :2446-2472     SwiGLU expert             :7537-7561
//   router + top-6            :7277-7376     batched grouping/combine  :8088-8099, 8267-8326
#include <algorithm>

#include "ffn_internal.h"
#include "gemv_tile.cuh"

namespace ffn {

// ============================================================ activations
// One CTA per row.  Optionally RMS-normalises the row first (flash1017.rs:
// 4880-4891: inv = 1 / sqrt(sum(x^2) / n + eps), xn = x * inv * w; with
// seq_norm the sum of squares is taken sequentially in column order, the
// reference's order, so xn is bit-identical to the CPU's), writes xn (f32) when
// asked, then splits x (or xn) into hi/lo f16 of x * 2^-e with
// e = floor(log2 max|x|) - 14, in natural column order (NVFP4 consumers)
// and/or pair order (ternary consumers).
__global__ void __launch_bounds__(256) xprep_loop_kernel(const float *__restrict__ x, int ld_x, int K,
                                                    __half *nh, __half *nl, __half *th,
                                                    __half *tl, int ld_o, int *xe,
                                                    const float *__restrict__ norm_w,
                                                    float norm_eps, int seq_norm, float *xn) {
  pdl_enter();
  const int row = blockIdx.x;
  const float *xr = x + (size_t)row * ld_x;
  __shared__ float red[32];
  __shared__ float s_inv;
  float inv = 1.0f;
  if (norm_w) {
    if (seq_norm) {
      if (threadIdx.x == 0) {
        float ss = 0.f;
        for (int c = 0; c < K; ++c) ss = __fadd_rn(ss, __fmul_rn(xr[c], xr[c]));
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), norm_eps)));
      }
    } else {
      float ss = 0.f;
#pragma unroll 8
      for (int c = threadIdx.x; c < K; c += blockDim.x) ss = fmaf(xr[c], xr[c], ss);
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), norm_eps)));
      }
    }
    __syncthreads();
    inv = s_inv;
  }
  float amax = 0.f;
#pragma unroll 8
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    float v = xr[c];
    if (norm_w) {
      v = __fmul_rn(__fmul_rn(v, inv), norm_w[c]);
      if (xn) xn[(size_t)row * K + c] = v;
    }
    amax = fmaxf(amax, fabsf(v));
  }
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  amax = red[0];
  int e = 0;
  if (amax > 0.f && isfinite(amax)) {
    int ex;
    frexpf(amax, &ex);  // amax = m 2^ex, m in [0.5, 1)
    e = max(-100, min(100, ex - 15));
  }
  const float sc = pow2f(-e);
  const size_t o = (size_t)row * ld_o;
#pragma unroll 8
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    float v = xr[c];
    if (norm_w) v = __fmul_rn(__fmul_rn(v, inv), norm_w[c]);
    __half hi, lo;
    split_f16(v * sc, hi, lo);
    if (nh) { nh[o + c] = hi; nl[o + c] = lo; }
    if (th) { const int p = tern_pos(c); th[o + p] = hi; tl[o + p] = lo; }
  }
  if (threadIdx.x == 0) xe[row] = e;
}

// Rows of up to kXprepV * 1024 columns with 16-byte aligned x (and norm
// weight) rows: each thread holds its 4-column groups in registers, so the row
// is read from memory once and every pass runs on registers.
constexpr int kXprepV = 8;
__global__ void __launch_bounds__(256) xprep_reg_kernel(const float *__restrict__ x, int ld_x, int K,
                                                        __half *nh, __half *nl, __half *th,
                                                        __half *tl, int ld_o, int *xe,
                                                        const float *__restrict__ norm_w,
                                                        float norm_eps, int seq_norm, float *xn) {
  pdl_enter();
  const int row = blockIdx.x;
  const float *xr = x + (size_t)row * ld_x;
  __shared__ float red[32];
  __shared__ float s_inv;
  float4 v[kXprepV];
#pragma unroll
  for (int j = 0; j < kXprepV; ++j) {
    const int c = 4 * (threadIdx.x + 256 * j);
    v[j] = c < K ? __ldg(reinterpret_cast<const float4 *>(xr + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (norm_w) {
    if (seq_norm) {
      if (threadIdx.x == 0) {
        float ss = 0.f;
        for (int c = 0; c < K; ++c) ss = __fadd_rn(ss, __fmul_rn(xr[c], xr[c]));
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), norm_eps)));
      }
    } else {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < kXprepV; ++j)
        ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < 8; ++w) t += red[w];
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), norm_eps)));
      }
    }
    __syncthreads();
    const float inv = s_inv;
#pragma unroll
    for (int j = 0; j < kXprepV; ++j) {
      const int c = 4 * (threadIdx.x + 256 * j);
      if (c < K) {
        const float4 w = __ldg(reinterpret_cast<const float4 *>(norm_w + c));
        v[j].x = __fmul_rn(__fmul_rn(v[j].x, inv), w.x);
        v[j].y = __fmul_rn(__fmul_rn(v[j].y, inv), w.y);
        v[j].z = __fmul_rn(__fmul_rn(v[j].z, inv), w.z);
        v[j].w = __fmul_rn(__fmul_rn(v[j].w, inv), w.w);
        if (xn) *reinterpret_cast<float4 *>(xn + (size_t)row * K + c) = v[j];
      }
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kXprepV; ++j)
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float m = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) red[0] = m;
  }
  __syncthreads();
  amax = red[0];
  int e = 0;
  if (amax > 0.f && isfinite(amax)) {
    int ex;
    frexpf(amax, &ex);  // amax = m 2^ex, m in [0.5, 1)
    e = max(-100, min(100, ex - 15));
  }
  const float sc = pow2f(-e);
  const size_t o = (size_t)row * ld_o;
#pragma unroll
  for (int j = 0; j < kXprepV; ++j) {
    const int c = 4 * (threadIdx.x + 256 * j);
    if (c >= K) continue;
    const float f[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
    __half hi[4], lo[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) split_f16(f[q] * sc, hi[q], lo[q]);
    if (nh) {
      *reinterpret_cast<__half2 *>(nh + o + c) = __halves2half2(hi[0], hi[1]);
      *reinterpret_cast<__half2 *>(nh + o + c + 2) = __halves2half2(hi[2], hi[3]);
      *reinterpret_cast<__half2 *>(nl + o + c) = __halves2half2(lo[0], lo[1]);
      *reinterpret_cast<__half2 *>(nl + o + c + 2) = __halves2half2(lo[2], lo[3]);
    }
    if (th) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int p = tern_pos(c + q);
        th[o + p] = hi[q];
        tl[o + p] = lo[q];
      }
    }
  }
  if (threadIdx.x == 0) xe[row] = e;
}

int launch_xprep(const float *x, int ld_x, int rows, int K, __half *nh, __half *nl, __half *th,
                 __half *tl, int ld_o, int *xe, cudaStream_t st, const float *norm_w,
                 float norm_eps, int seq_norm, float *xn) {
  if (rows <= 0) return 0;
  const bool reg = K <= kXprepV * 1024 && ld_x % 4 == 0 && ld_o % 2 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(norm_w) & 15) == 0;
  if (reg)
    FFN_LAUNCH_PDL(FFN_B200_K_XPREP, st, "xprep_reg_kernel", xprep_reg_kernel, rows, 256, 0, x, ld_x, K, nh, nl, th, tl, ld_o, xe, norm_w, norm_eps, seq_norm, xn);
  else
    FFN_LAUNCH_PDL(FFN_B200_K_XPREP, st, "xprep_loop_kernel", xprep_loop_kernel, rows, 256, 0, x, ld_x, K, nh, nl, th, tl, ld_o, xe, norm_w, norm_eps, seq_norm, xn);
  return 0;
}

// ============================================================ phase kernels
__device__ __forceinline__ float silu_clamped(float g) {
  return fminf(g / (1.0f + expf(-g)), 10.0f);  // flash1017.rs:7539
}
__device__ __forceinline__ float clamp10(float u) {  // Rust f32::clamp(-10, 10)
  if (u < -10.f) u = -10.f;
  if (u > 10.f) u = 10.f;
  return u;
}

// Rank-16 core term sum_r B[row][r] * z[r] (flash1017.rs:2465-2471).
__device__ __forceinline__ float core_term(const int8_t *b, int row, const float *z) {
  const int4 v = __ldg(reinterpret_cast<const int4 *>(b + (size_t)row * 16));
  const int8_t *bb = reinterpret_cast<const int8_t *>(&v);
  float acc = 0.f;
#pragma unroll
  for (int r = 0; r < 16; ++r) acc += (float)bb[r] * z[r];
  return acc;
}

// What a tile needs of one matrix of its expert.
struct MatInfo {
  const uint8_t *w, *s;     // weights / NVFP4 block scales
  float gs;                 // NVFP4 per-tensor scale
  const float *rs;          // ternary row scales
  const int8_t *core_b;     // ternary rank-16 B, or nullptr
};

template <int FMT>
__device__ __forceinline__ MatInfo mat_info(const ffn_b200_expert &E, int mm) {
  MatInfo r;
  if (FMT != FFN_B200_FMT_TERNARY) {  // NVFP4, MXFP4 and MXFP8 (nv[] descriptors)
    r.w = E.nv[mm].w; r.s = E.nv[mm].s; r.gs = E.nv[mm].gs; r.rs = nullptr; r.core_b = nullptr;
  } else {
    r.w = E.tn[mm].p; r.s = E.tn[mm].bs; r.gs = 1.0f; r.rs = E.tn[mm].rs;
    r.core_b = E.tn[mm].core_a ? E.tn[mm].core_b : nullptr;
  }
  return r;
}

// Stages of each warp's cp.async ring (units in flight = STAGES - 1) and
// sub-chunks per unit (2: 256 NVFP4 columns, so a row's block scales for one
// unit are one 16-byte copy).
#ifndef FFN_STAGES
#define FFN_STAGES 2
#endif
#ifndef FFN_SUB
#define FFN_SUB 2
#endif
constexpr int kStages = FFN_STAGES;
constexpr int kSub = FFN_SUB;  // sub-chunks per ring unit

// Rows of one warp task: gate+up tasks carry two matrices, so R = 2 (32 rows);
// single-matrix tasks use R = 4 (64 rows): both have four m-tiles, so every
// activation fragment a lane loads feeds four MMAs per term.
#ifndef FFN_R_GATEUP
#define FFN_R_GATEUP 2
#endif
#ifndef FFN_R_SINGLE
#define FFN_R_SINGLE 4
#endif
template <int PHASE>
__host__ __device__ constexpr int task_r() { return PHASE == 1 ? FFN_R_GATEUP : FFN_R_SINGLE; }

int rows_per_tile(int phase) { return 16 * (phase == 1 ? task_r<1>() : task_r<2>()); }
int chunk_cols(int fmt) {
  return (fmt == FFN_B200_FMT_NVFP4 ? 128 : fmt == FFN_B200_FMT_MXFP8 ? 64 : 256) * kSub;
}

// A task's slice and first row.
__device__ __forceinline__ VExp task_slice(const PhaseArgs &a, int task, int rows_per_task, int &row0) {
  const int v = task / a.blocks, blk = task - v * a.blocks;
  row0 = blk * rows_per_task;
  if (a.vexp) return a.vexp[v];
  VExp ve;
  ve.expert = -1;
  ve.offset = v * kNTok;
  ve.count = min(kNTok, a.n_tok_direct - v * kNTok);
  ve.pad = 0;
  return ve;
}

// Matrix mi (of NMAT) of a task on expert `expert` (-1: the direct expert).
template <int FMT, int PHASE, int NMAT>
__device__ __forceinline__ int task_mat(const PhaseArgs &a, int mi) {
  return PHASE == 1 ? (mi == 0 ? 0 : 1) : (PHASE == 2 ? 2 : a.mat);
}
__device__ __forceinline__ int expert_format(const PhaseArgs &a, int expert) {
  return expert >= 0 ? a.experts[expert].format : a.direct.format;
}
template <int FMT, int PHASE, int NMAT>
__device__ __forceinline__ MatInfo task_info(const PhaseArgs &a, int expert, int mi) {
  return mat_info<FMT>(expert >= 0 ? a.experts[expert] : a.direct, task_mat<FMT, PHASE, NMAT>(a, mi));
}

// PHASE 1: gate+up -> h.  PHASE 2: down -> y / out.  PHASE 0: one matrix -> out.
// Every warp walks its own work items (slice, row block, K-split) with a
// grid-wide stride and streams each item's K-chunks through its cp.async ring;
// warps never wait for one another.  Consecutive warps take consecutive items
// of one slice, so the slice's activation rows are shared in L1.
template <int FMT, int PHASE, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) phase_kernel(const PhaseArgs a) {
  pdl_enter();
  constexpr int NMAT = PHASE == 1 ? 2 : 1;
  constexpr int R = task_r<PHASE>();
  using WE = WarpEngine<FMT, NMAT, R, kStages, kSub>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  uint8_t *ring = smem + warp * WE::RING;
  const int n_vexp = a.vexp ? *a.n_vexp_dev : (a.n_tok_direct + kNTok - 1) / kNTok;
  const int S = a.splits;
  const int n_items = n_vexp * a.blocks * S;
  const int nch = WE::nchunks(a.K);
  const int gw = (int)blockIdx.x * kWarps + warp, nw = (int)gridDim.x * kWarps;
  const int n_mine = n_items > gw ? (n_items - gw + nw - 1) / nw : 0;
  // chunks of split s: [s*nch/S, (s+1)*nch/S)
  auto chunk_lo = [&](int item) { return (int)((long)(item % S) * nch / S); };
  auto chunk_hi = [&](int item) { return (int)((long)(item % S + 1) * nch / S); };

  // producer: issues the units of this warp's items in order (item p_k,
  // chunk p_c), STAGES - 1 units ahead of the consumer
  int p_k = 0, p_c = -1, p_cend = 0, p_slot = 0, p_row0 = 0;
  bool p_sal = false;  // scale rows aligned for one SR-byte copy each
  bool p_mx = false;   // the item's expert is MXFP4 (NVFP4 instance)
  MatRef pm[NMAT];
  auto issue_next = [&]() {
    if (p_k < n_mine) {
      if (p_c < 0) {
        const int item = gw + p_k * nw;
        const VExp ve = task_slice(a, item / S, WE::ROWS, p_row0);
        p_c = chunk_lo(item);
        p_cend = chunk_hi(item);
        p_mx = FMT == FFN_B200_FMT_NVFP4 && expert_format(a, ve.expert) == FFN_B200_FMT_MXFP4;
        const int srb = p_mx ? WE::SR / 2 : WE::SR;  // scale bytes per row and unit
        p_sal = (p_mx ? a.K / 32 : WE::sld_of(a.K)) % srb == 0;
#pragma unroll
        for (int mi = 0; mi < NMAT; ++mi) {
          const MatInfo m = task_info<FMT, PHASE, NMAT>(a, ve.expert, mi);
          pm[mi].w = m.w;
          pm[mi].s = m.s;
          p_sal = p_sal && ((reinterpret_cast<uintptr_t>(m.s) & (srb - 1)) == 0);
        }
      }
      WE::issue(ring + p_slot * WE::UNIT, pm, a.rows, a.K, p_row0, p_c, p_sal, p_mx);
      if (++p_c == p_cend) { p_c = -1; ++p_k; }
    }
    cp_async_commit();
    p_slot = p_slot + 1 == kStages ? 0 : p_slot + 1;
  };
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) issue_next();

  int c_slot = 0;
  for (int k = 0; k < n_mine; ++k) {
    const int item = gw + k * nw, task = item / S;
    int row0;
    const VExp ve = task_slice(a, task, WE::ROWS, row0);
    // ternary matrices with U8 block scales (bit mi)
    uint32_t bs_mask = 0, mxinfo = 0;
    if (FMT == FFN_B200_FMT_TERNARY) {
#pragma unroll
      for (int mi = 0; mi < NMAT; ++mi)
        if (task_info<FMT, PHASE, NMAT>(a, ve.expert, mi).s) bs_mask |= 1u << mi;
    } else if (FMT == FFN_B200_FMT_MXFP8 || expert_format(a, ve.expert) == FFN_B200_FMT_MXFP4) {
      // MXFP4: bit 31, and per matrix the exponent of its power-of-two gs + 128
      mxinfo = 1u << 31;
#pragma unroll
      for (int mi = 0; mi < NMAT; ++mi) {
        const int b = max(-128, min(127, ilogbf(task_info<FMT, PHASE, NMAT>(a, ve.expert, mi).gs)));
        mxinfo |= (uint32_t)(b + 128) << (8 * mi);
      }
    }
    const bool packed = ve.count <= 4;
    // this lane's MMA column: packed: token g&3, hi terms in columns 0-3 and
    // lo terms in 4-7; otherwise token g with separate hi / lo MMAs
    const int tok = packed ? (g & 3) : g;
    const __half *xa = nullptr, *xb = nullptr;
    if (tok < ve.count) {
      const int p = ve.offset + tok;
      const int xr = a.pair_tok ? __ldg(a.pair_tok + p) : p;
      const __half *hrow = a.xh + (size_t)xr * a.ld_x, *lrow = a.xl + (size_t)xr * a.ld_x;
      if (packed) xa = g < 4 ? hrow : lrow;
      else { xa = hrow; xb = lrow; }
    }
    float acc[NMAT][R][4];
#pragma unroll
    for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[mi][i][q] = 0.f;
    const int c_end = chunk_hi(item);
    for (int c = chunk_lo(item); c < c_end; ++c) {
      issue_next();
      cp_async_wait<kStages - 1>();
      __syncwarp();
      const uint8_t *slot = ring + c_slot * WE::UNIT;
      c_slot = c_slot + 1 == kStages ? 0 : c_slot + 1;
      if (packed) WE::template compute<true>(slot, a.K, c, xa, xb, acc, bs_mask, mxinfo);
      else WE::template compute<false>(slot, a.K, c, xa, xb, acc, bs_mask, mxinfo);
      __syncwarp();
    }

    // Lane (g, t) holds rows 16i+g and 16i+g+8, columns 2t and 2t+1.  Packed:
    // token n = column n + column n+4, so lanes t < 2 add their partner lane
    // t+2 and own tokens 2t, 2t+1.
    if (packed) {
#pragma unroll
      for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[mi][i][q] += __shfl_xor_sync(0xffffffffu, acc[mi][i][q], 2);
    }
    const bool owner = !packed || t < 2;
    if (S > 1) {
      // leave this split's sums; the last split of the task adds all of them
      float *pp = a.part + (size_t)task * S * NMAT * a.pt * WE::ROWS;
      const int s = item % S;
#pragma unroll
      for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int n = 2 * t + (q & 1), rl = 16 * i + g + 8 * (q >> 1);
            if (owner && n < ve.count)
              pp[(((size_t)s * NMAT + mi) * a.pt + n) * WE::ROWS + rl] = acc[mi][i][q];
          }
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(a.cnt + task, 1) == S - 1;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence();
      // Lane-parallel reduction: lane L sums values L, L+32, ... of the task
      // over the splits in split order (8 loads in flight per value), writes
      // the totals over split 0's slot, and reads back its own fragment.
      const int V = NMAT * a.pt * WE::ROWS;
      for (int v = lane; v < V; v += 32) {
        float sum = 0.f;
        for (int s0 = 0; s0 < S; s0 += 8) {
          float part8[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) part8[u] = s0 + u < S ? __ldcg(pp + (size_t)(s0 + u) * V + v) : 0.f;
#pragma unroll
          for (int u = 0; u < 8; ++u) sum += part8[u];
        }
        pp[v] = sum;
      }
      __threadfence_block();
      __syncwarp();
#pragma unroll
      for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int n = 2 * t + (q & 1), rl = 16 * i + g + 8 * (q >> 1);
            acc[mi][i][q] = owner && n < ve.count ? __ldcg(pp + ((size_t)mi * a.pt + n) * WE::ROWS + rl) : 0.f;
          }
    }
    if (!owner) continue;

    // epilogue
    MatInfo mat[NMAT];
#pragma unroll
    for (int mi = 0; mi < NMAT; ++mi) mat[mi] = task_info<FMT, PHASE, NMAT>(a, ve.expert, mi);
    const float proj = ve.expert >= 0 ? a.experts[ve.expert].proj_scale : a.direct.proj_scale;
#pragma unroll
    for (int jn = 0; jn < 2; ++jn) {
      const int n = 2 * t + jn;
      if (n >= ve.count) continue;
      const int p = ve.offset + n;
      const int xr = a.pair_tok ? __ldg(a.pair_tok + p) : p;
      const float xsc = a.xe ? pow2f(__ldg(a.xe + xr)) : 1.0f;
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int jr = 0; jr < 2; ++jr) {
          const int row = row0 + 16 * i + g + 8 * jr;
          if (row >= a.rows) continue;
          float val[NMAT];
#pragma unroll
          for (int mi = 0; mi < NMAT; ++mi) {
            float s = acc[mi][i][2 * jr + jn];
            if (FMT != FFN_B200_FMT_TERNARY) {
              s = s * xsc * mat[mi].gs;
            } else {
              const int mm = task_mat<FMT, PHASE, NMAT>(a, mi);
              s = (s * 0.5f) * xsc * __ldg(mat[mi].rs + row);
              if (mat[mi].core_b)
                s += core_term(mat[mi].core_b, row, a.z + ((size_t)p * 3 + mm) * 16);
            }
            val[mi] = s;
          }
          if (PHASE == 1) {
            float gv = val[0], uv = val[NMAT - 1];
            if (FMT == FFN_B200_FMT_TERNARY) { gv *= proj; uv *= proj; }
            const float h = silu_clamped(gv) * clamp10(uv);
            __half hi, lo;
            split_f16(h, hi, lo);
            const int col = FMT != FFN_B200_FMT_TERNARY ? row : tern_pos(row);
            a.hh[(size_t)p * a.ld_h + col] = hi;
            a.hl[(size_t)p * a.ld_h + col] = lo;
          } else {
            float *dst = a.y + (size_t)p * a.ld_y + row;
            if (a.vexp || PHASE == 0) {
              *dst = val[0];
            } else {
              const float wy = a.out_w * val[0];  // flash1017.rs:4900-4905 (dst += scale * src)
              *dst = a.accumulate ? *dst + wy : wy;
            }
          }
        }
    }
  }
  cp_async_wait<0>();
}

constexpr int phase_kind(int fmt, int phase) {
  return phase == 0 ? FFN_B200_K_MATVEC
                    : (fmt != FFN_B200_FMT_TERNARY ? (phase == 1 ? FFN_B200_K_GATEUP_NVFP4 : FFN_B200_K_DOWN_NVFP4)
                                                 : (phase == 1 ? FFN_B200_K_GATEUP_TERNARY : FFN_B200_K_DOWN_TERNARY));
}

// CTAs per SM: what the rings' shared memory allows, capped so that 16 warps
// share an SM (4-warp CTAs: 3 fit the shared memory, at up to 168 registers
// per thread; a lower register cap makes the engine spill).
#ifndef FFN_MAX_CTAS
#define FFN_MAX_CTAS (16 / FFN_WARPS)
#endif
template <int FMT, int PHASE>
constexpr int phase_min_blocks() {
  constexpr size_t smem = WarpEngine<FMT, PHASE == 1 ? 2 : 1, task_r<PHASE>(), kStages, kSub>::SMEM;
  constexpr int by_smem = smem * 3 <= 225 * 1024 ? 3 : (smem * 2 <= 225 * 1024 ? 2 : 1);
  return by_smem < FFN_MAX_CTAS ? by_smem : FFN_MAX_CTAS;
}

template <int FMT, int PHASE>
static int launch_phase_t(const PhaseArgs &a, long long tasks, cudaStream_t st) {
  constexpr int MINB = phase_min_blocks<FMT, PHASE>();
  constexpr size_t smem = WarpEngine<FMT, PHASE == 1 ? 2 : 1, task_r<PHASE>(), kStages, kSub>::SMEM;
  static bool attr_set[64] = {false};
  int dev = 0;
  FFN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "phase_kernel: device index >= 64");
  if (!attr_set[dev]) {
    FFN_CUDA_TRY(cudaFuncSetAttribute(phase_kernel<FMT, PHASE, MINB>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set[dev] = true;
  }
  const long long want = (tasks + kWarps - 1) / kWarps;
  const int grid = (int)std::max<long long>(1, std::min<long long>(want, (long long)MINB * sm_count_of(dev)));
  FFN_LAUNCH_PDL(phase_kind(FMT, PHASE), st, "phase_kernel", (phase_kernel<FMT, PHASE, MINB>), grid, kThreads, smem, a);
  return 0;
}

// `tasks` is an upper bound of the warp work items (slices x row blocks x splits).
int launch_phase(int fmt, int phase, const PhaseArgs &a, long long tasks, cudaStream_t st) {
  if (fmt == FFN_B200_FMT_MXFP8) {
    if (phase == 1) return launch_phase_t<FFN_B200_FMT_MXFP8, 1>(a, tasks, st);
    if (phase == 2) return launch_phase_t<FFN_B200_FMT_MXFP8, 2>(a, tasks, st);
    return launch_phase_t<FFN_B200_FMT_MXFP8, 0>(a, tasks, st);
  }
  if (fmt == FFN_B200_FMT_NVFP4) {
    if (phase == 1) return launch_phase_t<FFN_B200_FMT_NVFP4, 1>(a, tasks, st);
    if (phase == 2) return launch_phase_t<FFN_B200_FMT_NVFP4, 2>(a, tasks, st);
    return launch_phase_t<FFN_B200_FMT_NVFP4, 0>(a, tasks, st);
  }
  if (phase == 1) return launch_phase_t<FFN_B200_FMT_TERNARY, 1>(a, tasks, st);
  if (phase == 2) return launch_phase_t<FFN_B200_FMT_TERNARY, 2>(a, tasks, st);
  return launch_phase_t<FFN_B200_FMT_TERNARY, 0>(a, tasks, st);
}

// ============================================================ rank-16 core z
// z[pair][mat][r] = (sum_c A[r][c] * x[c]) * a_sc[r] * b_sc[r]   (flash1017.rs:2452-2463)
// One CTA of 512 threads per (slice, matrix).  Thread (rg, l) takes core rows
// 4rg..4rg+3 and the 16-column blocks l, l+128, ...: one 16-byte load of A per
// row and block, each activation block loaded once for four rows.  Lane sums
// are combined with shuffles and then across the 4 warps of a row group in a
// fixed order.
constexpr int kCorezThreads = 512;
__global__ void __launch_bounds__(kCorezThreads) corez_kernel(const CoreZArgs a) {
  pdl_enter();
  const int n_vexp = a.vexp ? *a.n_vexp_dev : (a.n_tok_direct + kNTok - 1) / kNTok;
  const int item = blockIdx.x;
  const int v = item / a.nmat, mm = a.mat0 + item % a.nmat;
  if (v >= n_vexp) return;
  VExp ve;
  if (a.vexp) ve = a.vexp[v];
  else { ve.expert = -1; ve.offset = v * kNTok; ve.count = min(kNTok, a.n_tok_direct - v * kNTok); }
  int fmt;
  const int8_t *A;
  const float *asc, *bsc;
  if (ve.expert >= 0) {
    const ffn_b200_expert &E = a.experts[ve.expert];
    fmt = E.format; A = E.tn[mm].core_a; asc = E.tn[mm].core_a_sc; bsc = E.tn[mm].core_b_sc;
  } else {
    fmt = a.direct.format; A = a.direct.tn[mm].core_a;
    asc = a.direct.tn[mm].core_a_sc; bsc = a.direct.tn[mm].core_b_sc;
  }
  if (fmt != FFN_B200_FMT_TERNARY || A == nullptr) return;  // uniform per CTA
  const int rg = threadIdx.x >> 7, l = threadIdx.x & 127;
  float acc[4][kNTok];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int n = 0; n < kNTok; ++n) acc[q][n] = 0.f;
  const int nblk = a.K / 16;
  for (int blk = l; blk < nblk; blk += 128) {
    int4 av[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      av[q] = __ldg(reinterpret_cast<const int4 *>(A + (size_t)(4 * rg + q) * a.K + 16 * blk));
#pragma unroll
    for (int n = 0; n < kNTok; ++n) {
      if (n >= ve.count) break;
      const int p = ve.offset + n;
      float xv[16];
      if (a.xf) {
        const int xr = a.pair_tok ? __ldg(a.pair_tok + p) : p;
        const float *xp = a.xf + (size_t)xr * a.ld_xf + 16 * blk;
        if ((reinterpret_cast<uintptr_t>(xp) & 15) == 0) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 f = __ldg(reinterpret_cast<const float4 *>(xp) + q);
            xv[4 * q] = f.x; xv[4 * q + 1] = f.y; xv[4 * q + 2] = f.z; xv[4 * q + 3] = f.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) xv[i] = __ldg(xp + i);
        }
      } else {
        // pair order: column i (< 8) at 2i, column i + 8 at 2i + 1
        const uint4 *hp = reinterpret_cast<const uint4 *>(a.hh + (size_t)p * a.ld_h + 16 * blk);
        const uint4 *lp = reinterpret_cast<const uint4 *>(a.hl + (size_t)p * a.ld_h + 16 * blk);
        const uint4 h0 = __ldg(hp), h1 = __ldg(hp + 1), l0 = __ldg(lp), l1 = __ldg(lp + 1);
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const __half2 hh = *reinterpret_cast<const __half2 *>(&hw[i]);
          const __half2 ll = *reinterpret_cast<const __half2 *>(&lw[i]);
          xv[i] = __low2float(hh) + __low2float(ll);
          xv[i + 8] = __high2float(hh) + __high2float(ll);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int8_t *ab = reinterpret_cast<const int8_t *>(&av[q]);
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[q][n] = fmaf((float)ab[i], xv[i], acc[q][n]);
      }
    }
  }
  __shared__ float red[4][4][4][kNTok];  // [row group][warp of the group][row][token]
  const int wg = l >> 5;
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int n = 0; n < kNTok; ++n) {
      float s = acc[q][n];
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if ((l & 31) == 0) red[rg][wg][q][n] = s;
    }
  __syncthreads();
  if (threadIdx.x < 16 * kNTok) {
    const int r = threadIdx.x / kNTok, n = threadIdx.x % kNTok;
    if (n < ve.count) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) s += red[r >> 2][w][r & 3][n];
      a.z[((size_t)(ve.offset + n) * 3 + mm) * 16 + r] = s * asc[r] * bsc[r];
    }
  }
}

int launch_corez(const CoreZArgs &a, int max_vexp, cudaStream_t st) {
  if (max_vexp <= 0) return 0;
  FFN_LAUNCH_PDL(FFN_B200_K_COREZ, st, "corez_kernel", corez_kernel, max_vexp * a.nmat, kCorezThreads, 0, a);
  return 0;
}

// ============================================================ router
// EXACT: logits[t][e] = sum_c w[e][c] * x[t][c], summed sequentially in column
// order with separate multiply and add (the CPU loop, flash1017.rs:2216-2222),
// so the logits are bit-identical to the oracle's.  CTA = 32 experts x 8 tokens.
__device__ __forceinline__ float wload(const float *w, size_t i) { return w[i]; }
__device__ __forceinline__ float wload(const uint16_t *w, size_t i) {
  return __uint_as_float((uint32_t)w[i] << 16);  // bf16 -> f32 (flash1017.rs:2220)
}

template <typename WT>
__global__ void __launch_bounds__(256) router_exact_kernel(const WT *__restrict__ w,
                                                           const float *__restrict__ x, int n_tok,
                                                           int n_exp, int H,
                                                           float *__restrict__ logits) {
  pdl_enter();
  __shared__ float ws[32][65];
  __shared__ float xs[8][64];
  const int el = threadIdx.x & 31, tl = threadIdx.x >> 5;
  const int e0 = blockIdx.x * 32, t0 = blockIdx.y * 8;
  float acc = 0.f;
  for (int c0 = 0; c0 < H; c0 += 64) {
    for (int i = threadIdx.x; i < 32 * 64; i += 256) {
      const int er = i >> 6, cc = i & 63;
      const int e = e0 + er, c = c0 + cc;
      ws[er][cc] = (e < n_exp && c < H) ? wload(w, (size_t)e * H + c) : 0.f;
    }
    for (int i = threadIdx.x; i < 8 * 64; i += 256) {
      const int tr = i >> 6, cc = i & 63;
      const int t = t0 + tr, c = c0 + cc;
      xs[tr][cc] = (t < n_tok && c < H) ? x[(size_t)t * H + c] : 0.f;
    }
    __syncthreads();
    const int lim = min(64, H - c0);
    for (int cc = 0; cc < lim; ++cc) acc = __fadd_rn(acc, __fmul_rn(ws[el][cc], xs[tl][cc]));
    __syncthreads();
  }
  const int e = e0 + el, t = t0 + tl;
  if (e < n_exp && t < n_tok) logits[(size_t)t * n_exp + e] = acc;
}

// logits [n_tok, rows] with the exact sequential sum over f32 or bf16 weights.
int launch_exact_matvec(const float *w32, const uint16_t *w16, const float *x, int n_tok,
                        int rows, int H, float *out, cudaStream_t st) {
  if (n_tok <= 0 || rows <= 0) return 0;
  dim3 g1((rows + 31) / 32, (n_tok + 7) / 8);
  if (g1.y > 65535) return fail(FFN_B200_EINVAL, "exact matvec: too many tokens");
  if (w32)
    FFN_LAUNCH_PDL(FFN_B200_K_ROUTER, st, "router_exact_kernel", (router_exact_kernel<float>), g1, 256, 0, w32, x, n_tok, rows, H, out);
  else
    FFN_LAUNCH_PDL(FFN_B200_K_ROUTER, st, "router_exact_kernel", (router_exact_kernel<uint16_t>), g1, 256, 0, w16, x, n_tok, rows, H, out);
  return 0;
}

// TENSOR: logits[t][e] = sum_c w[e][c] x[t][c] on the tensor cores.  The f32
// router weights are split into f16 hi/lo pairs as they are loaded; x enters
// as the hi/lo halves of the per-token normalised row (xprep); three MMAs per
// k-step (wh*xh + wh*xl + wl*xh) leave an error of about 2^-22 relative.  The
// summation order differs from the CPU loop, so selections can differ from the
// reference's only where two biased scores are within that error.
// CTA = 32 experts x 32 tokens x one of gridDim.z K-ranges.  The range is
// streamed through a 3-stage cp.async pipeline of 128-column stages (f32
// weight rows, f16 hi and lo token rows; rows padded so the fragment reads are
// free of bank conflicts); warp w computes k-step w of every stage, and the
// 8 warps' partial tiles are added in warp order through shared memory.  Each
// K-range writes its own partial logits (logits + z * n_tok * n_exp); top-k adds
// the partials in z order.
constexpr int kRouterWarps = 8;  // router_tc_kernel runs 256 threads
// K-ranges of the tensor router (partial logit planes): 12 x 8 x 3 = 288 CTAs of a
// 256-token, 384-expert layer fit one wave at 2 CTAs per SM
constexpr int kRouterKSplit = kRouterPlanes;
constexpr int kRtStages = 3;
constexpr int kRtW = 128 * 4 + 64;   // weight row stride (bytes): 576, rows 16 banks apart
constexpr int kRtX = 128 * 2 + 32;   // token row stride (bytes): 288, rows 8 banks apart
constexpr int kRtStage = 32 * kRtW + 2 * 32 * kRtX;
constexpr int kRtSmem = kRtStages * kRtStage;  // 110,592 bytes: 2 CTAs per SM
static_assert(kRouterWarps * 32 * 33 * 4 <= kRtSmem, "reduction fits the pipeline buffers");
__global__ void __launch_bounds__(256, 2) router_tc_kernel(const float *__restrict__ w,
                                                           const __half *__restrict__ xh,
                                                           const __half *__restrict__ xl,
                                                           const int *__restrict__ xe, int n_tok,
                                                           int n_exp, int H,
                                                           float *__restrict__ logits) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t rt_smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int e0 = blockIdx.x * 32, t0 = blockIdx.y * 32;
  const int ksteps = H / 16, kz = (ksteps + gridDim.z - 1) / gridDim.z;
  const int ks_lo = blockIdx.z * kz, ks_hi = min(ksteps, ks_lo + kz);
  const int n_st = ks_hi > ks_lo ? (ks_hi - ks_lo + 7) / 8 : 0;
  logits += (size_t)blockIdx.z * n_tok * n_exp;

  // copies of stage s: 1024 16-byte weight pieces (32 rows x 32) and 1024 token
  // pieces (hi and lo, 32 rows x 16); pieces of k-steps past the range are skipped
  auto issue = [&](int s) {
    if (s < n_st) {
      uint8_t *sw = rt_smem + (s % kRtStages) * kRtStage, *sx = sw + 32 * kRtW;
      const int kb = ks_lo + 8 * s;  // first k-step of the stage
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int p = tid + 256 * q;
        const int r = p >> 5, pc = p & 31;
        if (kb + (pc >> 2) < ks_hi)
          cp_async16(sw + r * kRtW + pc * 16,
                     w + (size_t)min(e0 + r, n_exp - 1) * H + (size_t)kb * 16 + pc * 4);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int p = tid + 256 * q;
        const int arr = p >> 9, r = (p >> 4) & 31, pc = p & 15;
        if (kb + (pc >> 1) < ks_hi)
          cp_async16(sx + arr * 32 * kRtX + r * kRtX + pc * 16,
                     (arr ? xl : xh) + (size_t)min(t0 + r, n_tok - 1) * H + (size_t)kb * 16 + pc * 8);
      }
    }
    cp_async_commit();
  };

  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.f;
#pragma unroll
  for (int s = 0; s < kRtStages - 1; ++s) issue(s);
  for (int s = 0; s < n_st; ++s) {
    cp_async_wait<kRtStages - 2>();
    __syncthreads();  // stage s visible to all; stage s - 1's slot is free
    issue(s + kRtStages - 1);
    if (ks_lo + 8 * s + warp < ks_hi) {
      const uint8_t *sw = rt_smem + (s % kRtStages) * kRtStage, *sx = sw + 32 * kRtW;
      const int cb = warp * 16 + 4 * t;  // this lane's 4 columns of the warp's k-step
      uint32_t ah[2][4], al[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float4 va = *reinterpret_cast<const float4 *>(sw + (16 * i + g) * kRtW + cb * 4);
        const float4 vb = *reinterpret_cast<const float4 *>(sw + (16 * i + g + 8) * kRtW + cb * 4);
        __half h[8], l[8];
        const float v[8] = {va.x, va.y, vb.x, vb.y, va.z, va.w, vb.z, vb.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) split_f16(v[q], h[q], l[q]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __half2 hh = __halves2half2(h[2 * q], h[2 * q + 1]);
          __half2 ll = __halves2half2(l[2 * q], l[2 * q + 1]);
          ah[i][q] = *reinterpret_cast<uint32_t *>(&hh);
          al[i][q] = *reinterpret_cast<uint32_t *>(&ll);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint2 bh = *reinterpret_cast<const uint2 *>(sx + (8 * j + g) * kRtX + cb * 2);
        const uint2 bl = *reinterpret_cast<const uint2 *>(sx + 32 * kRtX + (8 * j + g) * kRtX + cb * 2);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          mma_f16(acc[i][j], ah[i][0], ah[i][1], ah[i][2], ah[i][3], bh.x, bh.y);
          mma_f16(acc[i][j], ah[i][0], ah[i][1], ah[i][2], ah[i][3], bl.x, bl.y);
          mma_f16(acc[i][j], al[i][0], al[i][1], al[i][2], al[i][3], bh.x, bh.y);
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with the pipeline buffers
  float(*red)[32][33] = reinterpret_cast<float(*)[32][33]>(rt_smem);
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r0 = 16 * i + g, c0 = 8 * j + 2 * t;
      red[warp][r0][c0] = acc[i][j][0];
      red[warp][r0][c0 + 1] = acc[i][j][1];
      red[warp][r0 + 8][c0] = acc[i][j][2];
      red[warp][r0 + 8][c0 + 1] = acc[i][j][3];
    }
  __syncthreads();
  for (int q = threadIdx.x; q < 32 * 32; q += blockDim.x) {
    const int el = q & 31, tl = q >> 5;
    const int e = e0 + el, tok = t0 + tl;
    if (e >= n_exp || tok >= n_tok) continue;
    float sum = 0.f;
#pragma unroll
    for (int wv = 0; wv < kRouterWarps; ++wv) sum += red[wv][el][tl];
    logits[(size_t)tok * n_exp + e] = sum * pow2f(xe[tok]);
  }
}

// Top-k per token, one warp per token (flash1017.rs:7280-7376).  Ties in the
// biased score are broken by the lower expert index.
__device__ __forceinline__ float score_of(float l, int fn) {
  if (fn == FFN_B200_SCORE_REF_SQRTSOFTPLUS) {
    const float sp = l > 20.0f ? l : (l < -20.0f ? expf(l) : logf(1.0f + expf(l)));
    return sqrtf(fmaxf(sp, 0.0f));
  }
  return 1.0f / (1.0f + expf(-l));
}

__global__ void __launch_bounds__(64) topk_kernel(const float *__restrict__ logits,
                                                   const float *__restrict__ bias, int n_tok,
                                                   int n_exp, int top_k, int score_fn,
                                                   int n_part, int32_t *idx, float *wt) {
  pdl_enter();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= n_tok) return;
  const float *lg = logits + (size_t)warp * n_exp;
  const size_t plane = (size_t)n_tok * n_exp;
  // logit of expert e: the partial planes added in order
  auto logit = [&](int e) {
    float l = lg[e];
#pragma unroll
    for (int z = 1; z < kRouterKSplit; ++z)
      if (z < n_part) l += lg[z * plane + e];
    return l;
  };
  // round k's winner is kept by lane k (top_k <= 16 < 32)
  float my_score = 0.f;
  int my_idx = 0;
  float prev_b = INFINITY;
  int prev_i = -1;
  // scores and biased scores of this lane's experts (lane + 32j), computed once
  constexpr int kCache = 16;
  float cs[kCache], cb[kCache];
  const bool cached = n_exp <= 32 * kCache;
  if (cached) {
    // all logit (and bias) loads first, so they are in flight together; then
    // the scores
#pragma unroll
    for (int j = 0; j < kCache; ++j) {
      const int e = lane + 32 * j;
      cs[j] = e < n_exp ? logit(e) : 0.f;
      cb[j] = e < n_exp && bias ? bias[e] : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kCache; ++j) {
      const int e = lane + 32 * j;
      cs[j] = e < n_exp ? score_of(cs[j], score_fn) : 0.f;
      cb[j] = e < n_exp ? cs[j] + cb[j] : -INFINITY;
    }
  }
  if (cached && top_k <= 32) {
    // Each lane keeps the best of its own live experts (lane + 32j); a round
    // takes the warp's best lane head (biased score desc, index asc) and the
    // winning lane retires that expert and rescans its <= 16.  NaN scores are
    // never candidates; if no candidate is left the round yields index
    // 0x7fffffff with score 0.
    uint32_t alive = 0;
#pragma unroll
    for (int j = 0; j < kCache; ++j)
      if (lane + 32 * j < n_exp && cb[j] == cb[j]) alive |= 1u << j;
    float hb = 0.f, hs = 0.f;  // this lane's head: biased score, score, slot
    int hj = -1;
    auto rescan = [&]() {
      hj = -1;
      hb = -INFINITY;
      hs = 0.f;
#pragma unroll
      for (int j = 0; j < kCache; ++j)
        if (((alive >> j) & 1u) && (hj < 0 || cb[j] > hb)) { hb = cb[j]; hs = cs[j]; hj = j; }
    };
    rescan();
    for (int k = 0; k < top_k; ++k) {
      const uint32_t u = __float_as_uint(hb);
      const uint32_t key = hj < 0 ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
      const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
      const uint32_t cand = (key == kmax && hj >= 0) ? (uint32_t)(lane + 32 * hj) : 0x7fffffffu;
      const int bi = (int)__reduce_min_sync(0xffffffffu, cand);
      const float bs = __shfl_sync(0xffffffffu, hs, bi & 31);
      if (lane == k) { my_score = bi == 0x7fffffff ? 0.f : bs; my_idx = bi; }
      if (bi != 0x7fffffff && lane == (bi & 31)) {  // this lane's head won: retire it
        alive &= ~(1u << hj);
        rescan();
      }
    }
  } else {
  for (int k = 0; k < top_k; ++k) {
    // best candidate strictly after (prev_b, prev_i) in (biased desc, index asc) order
    float bb = -INFINITY, bs = 0.f;
    int bi = 0x7fffffff;
    if (cached) {
#pragma unroll
      for (int j = 0; j < kCache; ++j) {
        const int e = lane + 32 * j;
        const float b = cb[j];
        const bool after = b < prev_b || (b == prev_b && e > prev_i);
        const bool better = b > bb || (b == bb && e < bi);
        if (e < n_exp && after && better) { bb = b; bs = cs[j]; bi = e; }
      }
    } else {
      for (int e = lane; e < n_exp; e += 32) {
        const float s = score_of(logit(e), score_fn);
        const float b = s + (bias ? bias[e] : 0.0f);
        const bool after = b < prev_b || (b == prev_b && e > prev_i);
        const bool better = b > bb || (b == bb && e < bi);
        if (after && better) { bb = b; bs = s; bi = e; }
      }
    }
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, bb, o);
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > bb || (ob == bb && oi < bi)) { bb = ob; bs = os; bi = oi; }
    }
    if (lane == k) { my_score = bs; my_idx = bi; }
    prev_b = bb;
    prev_i = bi;
  }
  }
  // sum of the selected scores in selection order (flash1017.rs:7370)
  float sum = 0.f;
  for (int k = 0; k < top_k; ++k) sum += __shfl_sync(0xffffffffu, my_score, k);
  const float num = score_fn == FFN_B200_SCORE_REF_SQRTSOFTPLUS ? 1.5f : 1.0f;
  const float scale = sum > 1e-12f ? num / sum : 0.0f;
  if (lane < top_k) {
    idx[(size_t)warp * top_k + lane] = my_idx;
    wt[(size_t)warp * top_k + lane] = my_score * scale;
  }
}

// The same selection with four warps per token (up to 512 experts, four per
// lane), for a shorter dependent chain than topk_kernel's one warp: each warp
// picks its own top_k in order (biased score desc, index asc) out of its
// experts e = lane + 32 (w + 4 j), then warp 0 of the token merges the four
// sorted lists by the same order.  Every member of the token's top_k is in the
// top_k of its own warp, so the result (set, order, weights) is topk_kernel's.
// Two tokens per 256-thread CTA.
constexpr int kTkWarps = 4;   // warps per token
constexpr int kTkPer = 4;     // experts per lane and warp
constexpr int kTkMaxExp = 32 * kTkWarps * kTkPer;

// biased score -> a key whose unsigned order is the float order
__device__ __forceinline__ uint32_t order_key(float b) {
  const uint32_t u = __float_as_uint(b);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(256) topk4_kernel(const float *__restrict__ logits,
                                                    const float *__restrict__ bias, int n_tok,
                                                    int n_exp, int top_k, int score_fn, int n_part,
                                                    int32_t *idx, float *wt) {
  pdl_enter();
  __shared__ uint32_t s_key[2][kTkWarps][kTopKMax];
  __shared__ int s_idx[2][kTkWarps][kTopKMax];
  __shared__ float s_sc[2][kTkWarps][kTopKMax];
  __shared__ int s_n[2][kTkWarps];
  const int lane = threadIdx.x & 31, w = (threadIdx.x >> 5) & (kTkWarps - 1), g = threadIdx.x >> 7;
  const int tok = blockIdx.x * 2 + g;
  const bool live = tok < n_tok;  // (no early return: the CTA meets at a barrier)
  if (live) {
    const float *lg = logits + (size_t)tok * n_exp;
    const size_t plane = (size_t)n_tok * n_exp;
    float l[kTkPer], bb[kTkPer];
#pragma unroll
    for (int j = 0; j < kTkPer; ++j) {
      const int e = lane + 32 * (w + kTkWarps * j);
      l[j] = e < n_exp ? lg[e] : 0.f;
      bb[j] = e < n_exp && bias ? bias[e] : 0.0f;
    }
    // the partial planes added in order, as topk_kernel does
#pragma unroll
    for (int z = 1; z < kRouterKSplit; ++z)
      if (z < n_part) {
#pragma unroll
        for (int j = 0; j < kTkPer; ++j) {
          const int e = lane + 32 * (w + kTkWarps * j);
          if (e < n_exp) l[j] += lg[z * plane + e];
        }
      }
    float cs[kTkPer];
    uint32_t ck[kTkPer];
    uint32_t alive = 0;
#pragma unroll
    for (int j = 0; j < kTkPer; ++j) {
      const int e = lane + 32 * (w + kTkWarps * j);
      cs[j] = 0.f;
      ck[j] = 0u;
      if (e < n_exp) {
        cs[j] = score_of(l[j], score_fn);
        const float b = cs[j] + bb[j];
        ck[j] = order_key(b);
        if (b == b) alive |= 1u << j;  // NaN is never a candidate
      }
    }
    int n_sel = 0;
    for (int k = 0; k < top_k; ++k) {
      // this lane's head: the largest key, the lowest slot (= lowest index) on ties
      uint32_t hk = 0u;
      float hs = 0.f;
      int hj = -1;
#pragma unroll
      for (int j = 0; j < kTkPer; ++j)
        if (((alive >> j) & 1u) && (hj < 0 || ck[j] > hk)) { hk = ck[j]; hs = cs[j]; hj = j; }
      const uint32_t key = hj < 0 ? 0u : hk;  // non-NaN keys are >= 1
      const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
      const uint32_t cand = (hj >= 0 && key == kmax) ? (uint32_t)(lane + 32 * (w + kTkWarps * hj)) : 0x7fffffffu;
      const uint32_t bi = __reduce_min_sync(0xffffffffu, cand);
      if (bi == 0x7fffffffu) break;  // warp-uniform: no candidate left
      if (lane == (int)(bi & 31u)) {
        alive &= ~(1u << hj);
        s_key[g][w][k] = kmax;
        s_idx[g][w][k] = (int)bi;
        s_sc[g][w][k] = hs;
      }
      n_sel = k + 1;
    }
    if (lane == 0) s_n[g][w] = n_sel;
  }
  __syncthreads();
  if (!live || w != 0) return;
  // merge: candidate slot c = (warp c / top_k, rank c % top_k); lane holds c = lane, lane + 32
  uint32_t mk[2];
  int mi[2];
  float ms[2];
  uint32_t malive = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int c = lane + 32 * h;
    const int ww = c / top_k, kk = c - ww * top_k;
    mk[h] = 0u;
    mi[h] = 0x7fffffff;
    ms[h] = 0.f;
    if (ww < kTkWarps && kk < s_n[g][ww]) {
      mk[h] = s_key[g][ww][kk];
      mi[h] = s_idx[g][ww][kk];
      ms[h] = s_sc[g][ww][kk];
      malive |= 1u << h;
    }
  }
  float my_score = 0.f;
  int my_idx = 0x7fffffff;
  for (int k = 0; k < top_k; ++k) {
    uint32_t hk = 0u;
    int hi = 0x7fffffff, hh = -1;
    float hs = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (((malive >> h) & 1u) && (hh < 0 || mk[h] > hk || (mk[h] == hk && mi[h] < hi))) {
        hk = mk[h]; hi = mi[h]; hs = ms[h]; hh = h;
      }
    const uint32_t key = hh < 0 ? 0u : hk;
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
    const uint32_t cand = (hh >= 0 && key == kmax) ? (uint32_t)hi : 0x7fffffffu;
    const int bi = (int)__reduce_min_sync(0xffffffffu, cand);
    const bool won = bi != 0x7fffffff && hh >= 0 && hi == bi && key == kmax;
    const float bs = __shfl_sync(0xffffffffu, hs, (__ffs(__ballot_sync(0xffffffffu, won)) - 1) & 31);
    if (lane == k) { my_score = bi == 0x7fffffff ? 0.f : bs; my_idx = bi; }
    if (won) malive &= ~(1u << hh);
  }
  // sum of the selected scores in selection order (flash1017.rs:7370)
  float sum = 0.f;
  for (int k = 0; k < top_k; ++k) sum += __shfl_sync(0xffffffffu, my_score, k);
  const float num = score_fn == FFN_B200_SCORE_REF_SQRTSOFTPLUS ? 1.5f : 1.0f;
  const float scale = sum > 1e-12f ? num / sum : 0.0f;
  if (lane < top_k) {
    idx[(size_t)tok * top_k + lane] = my_idx;
    wt[(size_t)tok * top_k + lane] = my_score * scale;
  }
}

int launch_topk(const float *logits, int n_part, const float *bias, int n_tok, int n_exp, int top_k,
                int score_fn, int32_t *idx, float *wt, cudaStream_t st) {
  if (n_exp <= kTkMaxExp) {
    FFN_LAUNCH_PDL(FFN_B200_K_TOPK, st, "topk4_kernel", topk4_kernel, (n_tok + 1) / 2, 256, 0, logits, bias, n_tok, n_exp, top_k, score_fn, n_part, idx, wt);
  } else {
    FFN_LAUNCH_PDL(FFN_B200_K_TOPK, st, "topk_kernel", topk_kernel, (n_tok + 1) / 2, 64, 0, logits, bias, n_tok, n_exp, top_k, score_fn, n_part, idx, wt);
  }
  return 0;
}

int launch_router(const float *w, const float *bias, const float *x, const __half *xh,
                  const __half *xl, const int *xe, int mode, int n_tok, int n_exp, int H,
                  int top_k, int score_fn, float *logits, int32_t *idx, float *wt,
                  cudaStream_t st) {
  int n_part = 1;  // partial logit planes top-k adds up
  if (mode == FFN_B200_ROUTER_EXACT) {
    int rc = launch_exact_matvec(w, nullptr, x, n_tok, n_exp, H, logits, st);
    if (rc) return rc;
  } else {
    n_part = std::max(1, std::min(kRouterKSplit, H / 16 / kRouterWarps));
    dim3 g1((n_exp + 31) / 32, (n_tok + 31) / 32, n_part);
    if (g1.y > 65535) return fail(FFN_B200_EINVAL, "router: too many tokens");
    static bool attr_set[64] = {false};  // > 48 KB of dynamic shared memory, once per device
    int dev = 0;
    FFN_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "router: device index >= 64");
    if (!attr_set[dev]) {
      FFN_CUDA_TRY(cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRtSmem));
      attr_set[dev] = true;
    }
    FFN_LAUNCH_PDL(FFN_B200_K_ROUTER, st, "router_tc_kernel", router_tc_kernel, g1, 256, kRtSmem, w, xh, xl, xe, n_tok, n_exp, H, logits);
  }
  return launch_topk(logits, n_part, bias, n_tok, n_exp, top_k, score_fn, idx, wt, st);
}

// ============================================================ grouping
// Token->expert groups (flash1017.rs:8088-8099 builds the same groups by a
// linear scan).  Single CTA: counts per local expert (shared-memory atomics),
// exclusive scans, pair placement in pair order, and slices of <= 8 tokens per
// expert, listed per weight format.  Shared memory: per-warp counts with a row
// stride of n_exp + 1 words (a warp reading one expert's 32 counts hits 32
// banks), then counts, offsets, the experts' formats and slice bases.
__global__ void __launch_bounds__(1024) group_kernel(const int32_t *__restrict__ idx, int n_pairs,
                                                     int top_k, int n_exp, int e_begin, int e_end,
                                                     const ffn_b200_expert *__restrict__ experts,
                                                     int *counts, int *offsets, int *cursor,
                                                     int *vbase, int32_t *pair_tok, int32_t *inv,
                                                     VExp *vexp_nv, VExp *vexp_tn, int *n_vexp) {
  extern __shared__ int g_smem[];
  const int sp = n_exp + 1;              // row stride of the per-warp counts
  int *s_cnt = g_smem;                   // [32 warps][sp]: counts, then bases
  int *s_counts = g_smem + 32 * sp;      // [n_exp] pairs per expert
  int *s_off = s_counts + n_exp;         // [n_exp] first position of each expert
  int *s_nv = s_off + n_exp;             // [n_exp] 1: NVFP4 / MXFP4 slice list, 0: ternary
  int *s_vb = s_nv + n_exp;              // [n_exp] first slice of each expert in its list
  __shared__ int s_tot[2];
  __shared__ int ws_p[32], ws_n[32], ws_t[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  // nothing here depends on the previous kernel: runs while it finishes
  for (int i = tid; i < 32 * sp; i += blockDim.x) s_cnt[i] = 0;
  for (int e = tid; e < n_exp; e += blockDim.x) s_nv[e] = experts[e].format != FFN_B200_FMT_TERNARY;
  pdl_enter();
  // Warp w owns the pair range [w * span, (w + 1) * span) and walks it in
  // order, 32 pairs per step; lanes holding the same expert find each other
  // with match.any, the lowest of them updates the warp's count.
  const int span = (n_pairs + 31) / 32;
  const int q_lo = wid * span, q_hi = min(n_pairs, q_lo + span);
  __syncthreads();
  constexpr int kU = 8;  // steps whose expert ids are loaded together
  for (int q0 = q_lo; q0 < q_hi; q0 += 32 * kU) {
    int ev[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int q = q0 + 32 * u + lane;
      ev[u] = q < q_hi ? idx[q] : -1;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (q0 + 32 * u >= q_hi) break;  // warp-uniform
      int e = ev[u];
      if (e < e_begin || e >= e_end) e = -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0 && (peers & ((1u << lane) - 1u)) == 0) s_cnt[wid * sp + e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  // per expert (one warp each, lane = counting warp): warp counts -> exclusive
  // bases in warp order, and the total
  for (int e = wid; e < n_exp; e += 32) {
    const int c = s_cnt[lane * sp + e];
    int inc = c;
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += a;
    }
    s_cnt[lane * sp + e] = inc - c;
    if (lane == 31) s_counts[e] = inc;
  }
  __syncthreads();
  // each thread owns a contiguous run of `per` experts
  const int per = (n_exp + blockDim.x - 1) / blockDim.x;
  int loc_pairs = 0, loc_nv = 0, loc_tn = 0;
  for (int i = 0; i < per; ++i) {
    const int e = tid * per + i;
    if (e < n_exp) {
      const int c = s_counts[e], s = (c + kNTok - 1) / kNTok;
      loc_pairs += c;
      if (s_nv[e]) loc_nv += s; else loc_tn += s;
    }
  }
  // block-wide exclusive scans of the three per-thread totals
  int inc_p = loc_pairs, inc_n = loc_nv, inc_t = loc_tn;
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, inc_p, o);
    const int b = __shfl_up_sync(0xffffffffu, inc_n, o);
    const int c = __shfl_up_sync(0xffffffffu, inc_t, o);
    if (lane >= o) { inc_p += a; inc_n += b; inc_t += c; }
  }
  if (lane == 31) { ws_p[wid] = inc_p; ws_n[wid] = inc_n; ws_t[wid] = inc_t; }
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    int a = lane < nw ? ws_p[lane] : 0;
    int b = lane < nw ? ws_n[lane] : 0;
    int c = lane < nw ? ws_t[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int x1 = __shfl_up_sync(0xffffffffu, a, o);
      const int x2 = __shfl_up_sync(0xffffffffu, b, o);
      const int x3 = __shfl_up_sync(0xffffffffu, c, o);
      if (lane >= o) { a += x1; b += x2; c += x3; }
    }
    ws_p[lane] = a; ws_n[lane] = b; ws_t[lane] = c;
    if (lane == 31) { s_tot[0] = b; s_tot[1] = c; }
  }
  __syncthreads();
  int base_p = (wid ? ws_p[wid - 1] : 0) + inc_p - loc_pairs;
  int base_n = (wid ? ws_n[wid - 1] : 0) + inc_n - loc_nv;
  int base_t = (wid ? ws_t[wid - 1] : 0) + inc_t - loc_tn;
  for (int i = 0; i < per; ++i) {
    const int e = tid * per + i;
    if (e < n_exp) {
      const int c = s_counts[e], s = (c + kNTok - 1) / kNTok;
      counts[e] = c;
      offsets[e] = base_p;
      s_off[e] = base_p;
      base_p += c;
      const int vb = s_nv[e] ? base_n : base_t;
      vbase[e] = vb;
      s_vb[e] = vb;
      if (s_nv[e]) base_n += s; else base_t += s;
    }
  }
  __syncthreads();
  // Pair placement in pair order (the reference's linear scan, flash1017.rs:
  // 8088-8099): inside an expert group, tokens are in token order, so every
  // run groups the same tokens into the same slices.  A pair's position = the
  // expert's offset + its expert's pairs in earlier warps' ranges + those
  // earlier in its own warp's walk.
  for (int q0 = q_lo; q0 < q_hi; q0 += 32 * kU) {
    int ev[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int q = q0 + 32 * u + lane;
      ev[u] = q < q_hi ? idx[q] : -1;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (q0 + 32 * u >= q_hi) break;  // warp-uniform
      const int q = q0 + 32 * u + lane;
      int e = ev[u];
      const bool mine = e >= e_begin && e < e_end;
      if (!mine) e = -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      if (mine) {
        const int pos = s_off[e] + s_cnt[wid * sp + e] + rank;
        pair_tok[pos] = q / top_k;
        inv[q] = pos;
      } else if (q < q_hi) {
        inv[q] = -1;
      }
      __syncwarp();
      if (mine && rank == 0) s_cnt[wid * sp + e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  for (int e = tid; e < n_exp; e += blockDim.x) {
    const int c = s_counts[e];
    VExp *dst = s_nv[e] ? vexp_nv : vexp_tn;  // NVFP4, MXFP4 | ternary
    for (int j = 0; j * kNTok < c; ++j) {
      VExp v;
      v.expert = e;
      v.offset = s_off[e] + j * kNTok;
      v.count = min(kNTok, c - j * kNTok);
      v.pad = 0;
      dst[s_vb[e] + j] = v;
    }
  }
  if (tid == 0) { n_vexp[0] = s_tot[0]; n_vexp[1] = s_tot[1]; }
}

// The same groups from per-expert token bitmaps, for up to 32 x 32 tokens:
// bit t of expert e's words = token t routed to e.  A token picks an expert at
// most once, so a pair's position is its expert's offset plus the number of
// the expert's tokens before its own: the pair order of the linear scan.  (A
// token listed twice for one expert by a caller would get one row for both
// pairs, whose outputs are equal, so the weighted sum is unchanged.)
constexpr int kGroupBitsMaxWords = 32;
__global__ void __launch_bounds__(1024) group_bits_kernel(const int32_t *__restrict__ idx, int n_tok,
                                                          int top_k, int n_exp, int e_begin, int e_end,
                                                          const ffn_b200_expert *__restrict__ experts,
                                                          int *counts, int *offsets, int *vbase,
                                                          int32_t *pair_tok, int32_t *inv, VExp *vexp_nv,
                                                          VExp *vexp_tn, int *n_vexp) {
  extern __shared__ uint32_t gb_smem[];
  const int W = (n_tok + 31) >> 5;
  uint32_t *bm = gb_smem;                               // [n_exp][W]
  int *s_counts = reinterpret_cast<int *>(bm + (size_t)n_exp * W);
  int *s_off = s_counts + n_exp;
  int *s_nv = s_off + n_exp;
  int *s_vb = s_nv + n_exp;
  __shared__ int s_tot[2];
  __shared__ int ws_p[32], ws_n[32], ws_t[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  // nothing here depends on the previous kernel: runs while it finishes
  for (int i = tid; i < n_exp * W; i += blockDim.x) bm[i] = 0u;
  for (int e = tid; e < n_exp; e += blockDim.x) s_nv[e] = experts[e].format != FFN_B200_FMT_TERNARY;
  pdl_enter();
  __syncthreads();
  const int n_pairs = n_tok * top_k;
  for (int q = tid; q < n_pairs; q += blockDim.x) {
    const int e = idx[q];
    if (e >= e_begin && e < e_end) {
      const int t = q / top_k;
      atomicOr(&bm[e * W + (t >> 5)], 1u << (t & 31));
    }
  }
  __syncthreads();
  for (int e = tid; e < n_exp; e += blockDim.x) {
    int c = 0;
    for (int w = 0; w < W; ++w) c += __popc(bm[e * W + w]);
    s_counts[e] = c;
  }
  __syncthreads();
  // each thread owns a contiguous run of `per` experts; block-wide exclusive
  // scans of the pairs and of the two slice lists
  const int per = (n_exp + blockDim.x - 1) / blockDim.x;
  int loc_pairs = 0, loc_nv = 0, loc_tn = 0;
  for (int i = 0; i < per; ++i) {
    const int e = tid * per + i;
    if (e < n_exp) {
      const int c = s_counts[e], sl = (c + kNTok - 1) / kNTok;
      loc_pairs += c;
      if (s_nv[e]) loc_nv += sl; else loc_tn += sl;
    }
  }
  int inc_p = loc_pairs, inc_n = loc_nv, inc_t = loc_tn;
  for (int o = 1; o < 32; o <<= 1) {
    const int x1 = __shfl_up_sync(0xffffffffu, inc_p, o);
    const int x2 = __shfl_up_sync(0xffffffffu, inc_n, o);
    const int x3 = __shfl_up_sync(0xffffffffu, inc_t, o);
    if (lane >= o) { inc_p += x1; inc_n += x2; inc_t += x3; }
  }
  if (lane == 31) { ws_p[wid] = inc_p; ws_n[wid] = inc_n; ws_t[wid] = inc_t; }
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    int x1 = lane < nw ? ws_p[lane] : 0, x2 = lane < nw ? ws_n[lane] : 0, x3 = lane < nw ? ws_t[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y1 = __shfl_up_sync(0xffffffffu, x1, o);
      const int y2 = __shfl_up_sync(0xffffffffu, x2, o);
      const int y3 = __shfl_up_sync(0xffffffffu, x3, o);
      if (lane >= o) { x1 += y1; x2 += y2; x3 += y3; }
    }
    ws_p[lane] = x1; ws_n[lane] = x2; ws_t[lane] = x3;
    if (lane == 31) { s_tot[0] = x2; s_tot[1] = x3; }
  }
  __syncthreads();
  int base_p = (wid ? ws_p[wid - 1] : 0) + inc_p - loc_pairs;
  int base_n = (wid ? ws_n[wid - 1] : 0) + inc_n - loc_nv;
  int base_t = (wid ? ws_t[wid - 1] : 0) + inc_t - loc_tn;
  for (int i = 0; i < per; ++i) {
    const int e = tid * per + i;
    if (e < n_exp) {
      const int c = s_counts[e], sl = (c + kNTok - 1) / kNTok;
      counts[e] = c;
      offsets[e] = base_p;
      s_off[e] = base_p;
      base_p += c;
      const int vb = s_nv[e] ? base_n : base_t;
      vbase[e] = vb;
      s_vb[e] = vb;
      if (s_nv[e]) base_n += sl; else base_t += sl;
    }
  }
  __syncthreads();
  for (int q = tid; q < n_pairs; q += blockDim.x) {
    const int e = idx[q];
    if (e >= e_begin && e < e_end) {
      const int t = q / top_k, w = t >> 5;
      const uint32_t *row = bm + e * W;
      int pos = s_off[e] + __popc(row[w] & ((1u << (t & 31)) - 1u));
      for (int w2 = 0; w2 < w; ++w2) pos += __popc(row[w2]);
      pair_tok[pos] = t;
      inv[q] = pos;
    } else {
      inv[q] = -1;
    }
  }
  for (int e = tid; e < n_exp; e += blockDim.x) {
    const int c = s_counts[e];
    VExp *dst = s_nv[e] ? vexp_nv : vexp_tn;  // NVFP4, MXFP4 | ternary
    for (int j = 0; j * kNTok < c; ++j) {
      VExp v;
      v.expert = e;
      v.offset = s_off[e] + j * kNTok;
      v.count = min(kNTok, c - j * kNTok);
      v.pad = 0;
      dst[s_vb[e] + j] = v;
    }
  }
  if (tid == 0) { n_vexp[0] = s_tot[0]; n_vexp[1] = s_tot[1]; }
}

int launch_group(const int32_t *idx, int n_tok, int top_k, int n_exp, int e_begin, int e_end,
                 const ffn_b200_expert *experts, int *ws_int, int32_t *pair_tok, int32_t *inv,
                 VExp *vexp_nv, VExp *vexp_tn, int *n_vexp, cudaStream_t st) {
  const size_t smem = ((size_t)32 * (n_exp + 1) + 4 * (size_t)n_exp) * sizeof(int);
  if (smem > 200 * 1024) return fail(FFN_B200_EUNSUP, "group: too many experts");
  static bool attr_set[64] = {false};
  int dev = 0;
  FFN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "group: device index >= 64");
  if (!attr_set[dev]) {
    FFN_CUDA_TRY(cudaFuncSetAttribute(group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set[dev] = true;
  }
  const int words = (n_tok + 31) / 32;
  const size_t smem_bits = ((size_t)n_exp * words + 4 * (size_t)n_exp) * sizeof(int);
  if (words <= kGroupBitsMaxWords && smem_bits <= 200 * 1024) {
    static bool bits_attr[64] = {false};
    if (!bits_attr[dev]) {
      FFN_CUDA_TRY(cudaFuncSetAttribute(group_bits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      bits_attr[dev] = true;
    }
    FFN_LAUNCH_PDL(FFN_B200_K_GROUP, st, "group_bits_kernel", group_bits_kernel, 1, 1024, smem_bits, idx, n_tok, top_k, n_exp, e_begin, e_end, experts, ws_int, ws_int + n_exp, ws_int + 3 * n_exp, pair_tok, inv, vexp_nv, vexp_tn, n_vexp);
    return 0;
  }
  FFN_LAUNCH_PDL(FFN_B200_K_GROUP, st, "group_kernel", group_kernel, 1, 1024, smem, idx, n_tok * top_k, top_k, n_exp, e_begin, e_end, experts, ws_int, ws_int + n_exp, ws_int + 2 * n_exp, ws_int + 3 * n_exp, pair_tok, inv, vexp_nv, vexp_tn, n_vexp);
  return 0;
}

// ============================================================ combine
// out[t] = residual[t] + sum_k w[t][k] * y[pair(t,k)], the terms added in
// selection order starting from zero with separate multiply and add, as
// flash1017_axpy_f32 does (flash1017.rs:4900-4905, 7546-7547).  Ternary
// experts weigh by w * proj_scale (flash1017.rs:7561).
__global__ void __launch_bounds__(1024) combine_kernel(const float *__restrict__ y, int ld_y,
                                                      const int32_t *__restrict__ idx,
                                                      const float *__restrict__ wt,
                                                      const int32_t *__restrict__ inv, int top_k,
                                                      const ffn_b200_expert *__restrict__ experts,
                                                      const float *residual, float *out, int H,
                                                      const int *err, int n_exp) {
  pdl_enter();
  const int t = blockIdx.x;
  __shared__ float wk[kTopKMax];
  __shared__ int pk[kTopKMax];
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = err && *err;  // an upstream kernel gave up on a wait
  __syncthreads();
  if (threadIdx.x < top_k) {
    const int q = t * top_k + threadIdx.x;
    const int e = idx[q];
    if (e < 0 || e >= n_exp) {  // no expert selected (every score NaN): no table read
      s_bad = 1;
      wk[threadIdx.x] = 0.f;
      pk[threadIdx.x] = -1;
    } else {
      float w = wt[q];
      if (experts[e].format == FFN_B200_FMT_TERNARY) w = w * experts[e].proj_scale;
      wk[threadIdx.x] = w;
      pk[threadIdx.x] = inv[q];
    }
  }
  __syncthreads();
  if (s_bad) {  // make the failure visible
    for (int c = threadIdx.x; c < H; c += blockDim.x) out[(size_t)t * H + c] = __int_as_float(0x7FC00000);
    return;
  }
  if (H % 4 == 0 && ld_y % 4 == 0 && ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(out) |
                                       reinterpret_cast<uintptr_t>(residual)) & 15) == 0) {
    // four columns per thread; the terms' loads issue 8 at a time
    for (int c = 4 * threadIdx.x; c < H; c += 4 * blockDim.x) {
      const float4 r = residual ? *reinterpret_cast<const float4 *>(residual + (size_t)t * H + c)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k0 = 0; k0 < top_k; k0 += 8) {
        float4 yv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int k = k0 + u;
          if (k < top_k && pk[k] >= 0) yv[u] = __ldg(reinterpret_cast<const float4 *>(y + (size_t)pk[k] * ld_y + c));
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int k = k0 + u;
          if (k < top_k && pk[k] >= 0) {
            acc.x = __fadd_rn(acc.x, __fmul_rn(wk[k], yv[u].x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wk[k], yv[u].y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wk[k], yv[u].z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wk[k], yv[u].w));
          }
        }
      }
      if (residual) {
        acc.x = __fadd_rn(r.x, acc.x);
        acc.y = __fadd_rn(r.y, acc.y);
        acc.z = __fadd_rn(r.z, acc.z);
        acc.w = __fadd_rn(r.w, acc.w);
      }
      *reinterpret_cast<float4 *>(out + (size_t)t * H + c) = acc;
    }
    return;
  }
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float acc = 0.f;
    for (int k = 0; k < top_k; ++k) {
      const int p = pk[k];
      if (p >= 0) acc = __fadd_rn(acc, __fmul_rn(wk[k], __ldg(y + (size_t)p * ld_y + c)));
    }
    if (residual) acc = __fadd_rn(residual[(size_t)t * H + c], acc);
    out[(size_t)t * H + c] = acc;
  }
}

int launch_combine(const float *y, int ld_y, const int32_t *idx, const float *wt,
                   const int32_t *inv, int n_tok, int top_k, const ffn_b200_expert *experts,
                   const float *residual, float *out, int H, cudaStream_t st, const int *err, int n_exp) {
  if (n_tok <= 0) return 0;
  FFN_LAUNCH_PDL(FFN_B200_K_COMBINE, st, "combine_kernel", combine_kernel, n_tok, std::min(1024, std::max(32, H / 4)), 0, y, ld_y, idx, wt, inv, top_k, experts, residual, out, H, err, n_exp);
  return 0;
}

// ============================================================ queued routed calls
// out[r] += w[e] * y[pair[e]] for the entries of row r in list order (call
// order), each term rounded as fl(out + fl(w * y)), as the reference's per-call
// axpy does (flash1017.rs:4900-4905, 8297-8303); rows with row_zero[r] start
// from 0 (the queue began with an overwriting call).  Grid: (column blocks,
// out rows); 4 columns per thread (hidden % 64 == 0).
__global__ void __launch_bounds__(256) rows_accum_kernel(const float *__restrict__ y,
                                                         const int32_t *__restrict__ tok_ptr,
                                                         const int32_t *__restrict__ ent_pair,
                                                         const float *__restrict__ ent_w,
                                                         const uint8_t *__restrict__ row_zero, int H,
                                                         float *out) {
  pdl_enter();
  const int r = blockIdx.y;
  const int e0 = __ldg(tok_ptr + r), e1 = __ldg(tok_ptr + r + 1);
  const bool zero = __ldg(row_zero + r) != 0;
  if (e0 == e1 && !zero) return;
  float4 *o4 = reinterpret_cast<float4 *>(out + (size_t)r * H);
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < H / 4; c += gridDim.x * blockDim.x) {
    float4 acc = zero ? make_float4(0.f, 0.f, 0.f, 0.f) : o4[c];
    for (int e = e0; e < e1; ++e) {
      const float w = __ldg(ent_w + e);
      const float4 v = __ldg(reinterpret_cast<const float4 *>(y + (size_t)__ldg(ent_pair + e) * H) + c);
      acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
    }
    o4[c] = acc;
  }
}

int launch_rows_accum(const float *y, const int32_t *tok_ptr, const int32_t *ent_pair,
                      const float *ent_w, const uint8_t *row_zero, int out_rows, int H, float *out,
                      cudaStream_t st) {
  if (out_rows <= 0) return 0;
  if (H % 4) return fail(FFN_B200_EINVAL, "rows_accum: hidden must be a multiple of 4");
  const dim3 grid((unsigned)((H / 4 + 255) / 256), (unsigned)out_rows);
  FFN_LAUNCH_PDL(FFN_B200_K_COMBINE, st, "rows_accum_kernel", rows_accum_kernel, grid, 256, 0, y, tok_ptr,
                 ent_pair, ent_w, row_zero, H, out);
  return 0;
}

// ============================================================ reference-ABI helpers
// Single-row dots of the V1 vtable slots (HA:150-159).  mode 0: f32 . f32,
// 1: i8 . f32, 2: Q4_G32 (int4 - 8, bf16 scale per 32; twin HA:1159-1179),
// 3: ternary 2-bit codes (no scale).  One CTA, fixed-order tree reduction.
__global__ void __launch_bounds__(256) dot_kernel(int mode, const void *a, const void *aux,
                                                  const float *x, size_t len, float *out) {
  float acc = 0.f;
  if (mode == 0) {
    const float *v = (const float *)a;
    for (size_t i = threadIdx.x; i < len; i += 256) acc += v[i] * x[i];
  } else if (mode == 1) {
    const int8_t *v = (const int8_t *)a;
    for (size_t i = threadIdx.x; i < len; i += 256) acc += (float)v[i] * x[i];
  } else if (mode == 2) {
    const uint8_t *nib = (const uint8_t *)a;
    const uint16_t *sc = (const uint16_t *)aux;
    for (size_t g = threadIdx.x; g < len / 32; g += 256) {
      float gs = 0.f;
      for (int k = 0; k < 16; ++k) {
        const uint32_t b = nib[g * 16 + k];
        gs += (float)((int)(b & 15u) - 8) * x[g * 32 + 2 * k] +
              (float)((int)(b >> 4) - 8) * x[g * 32 + 2 * k + 1];
      }
      acc += gs * __uint_as_float((uint32_t)sc[g] << 16);
    }
  } else {
    const uint8_t *p = (const uint8_t *)a;
    for (size_t i = threadIdx.x; i < len / 4; i += 256) {
      const uint32_t b = p[i];
      for (int j = 0; j < 4; ++j) acc += tern_to_f32((b >> (2 * j)) & 3u) * x[4 * i + j];
    }
  }
  __shared__ float red[256];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int o = 128; o; o >>= 1) {
    if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = red[0];
}
int launch_dot(int mode, const void *a, const void *aux, const float *x, size_t len, float *out,
               cudaStream_t st) {
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "dot_kernel", dot_kernel<<<1, 256, 0, st>>>(mode, a, aux, x, len, out));
  return 0;
}

// ============================================================ generators
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t rnd(uint64_t key, uint64_t i) {
  return mix64(key + 0x9E3779B97F4A7C15ULL * (i + 1));
}
__device__ __forceinline__ float normal_at(uint64_t key, uint64_t i) {
  long long s = 0;
  for (int d = 0; d < 3; ++d) {
    const uint64_t r = rnd(key, 3 * i + d);
    s += (long long)(r & 0xFFFF) + (long long)((r >> 16) & 0xFFFF) +
         (long long)((r >> 32) & 0xFFFF) + (long long)(r >> 48);
  }
  return __fmul_rn((float)(s - 393210), 1.0f / 65536.0f);
}
// |N(0,1)| stand-in for block scales: Irwin-Hall sum of the four 16-bit
// uniforms of one draw, scaled to unit variance (same arithmetic as the oracle).
__device__ __forceinline__ float normal4_at(uint64_t key, uint64_t i) {
  const uint64_t r = rnd(key, i);
  const long long s = (long long)(r & 0xFFFF) + (long long)((r >> 16) & 0xFFFF) +
                      (long long)((r >> 32) & 0xFFFF) + (long long)(r >> 48);
  return __fmul_rn((float)(s - 131070), 1.0f / 37837.227f);
}
__device__ __forceinline__ float unit_at(uint64_t key, uint64_t i) {
  return __fmul_rn((float)(uint32_t)(rnd(key, i) >> 40), 1.0f / 16777216.0f);
}
// f32 -> E4M3, round to nearest even, saturating at 448 (integer arithmetic).
__device__ __forceinline__ uint8_t f32_to_e4m3(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t sign = (u >> 24) & 0x80u, a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return (uint8_t)(sign | 0x7Fu);
  if (a >= 0x43E00000u) return (uint8_t)(sign | 0x7Eu);
  const int e = (int)(a >> 23) - 127;
  if (e < -6) {
    if (e < -40 || (a >> 23) == 0) return (uint8_t)sign;  // rounds to zero
    const uint32_t M = (a & 0x7FFFFFu) | 0x800000u;     // value = M * 2^(e-23)
    const int sh = 14 - e;                               // value*2^9 = M >> sh
    const uint32_t q = M >> sh, rem = M & ((1u << sh) - 1u), half = 1u << (sh - 1);
    const uint32_t r = q + ((rem > half || (rem == half && (q & 1u))) ? 1u : 0u);
    return (uint8_t)(sign | r);
  }
  const uint32_t mant = a & 0x7FFFFFu, keep = mant >> 20, rest = mant & 0xFFFFFu;
  uint32_t enc = ((uint32_t)(e + 7) << 3) | keep;
  if (rest > 0x80000u || (rest == 0x80000u && (keep & 1u))) enc++;
  if (enc > 0x7Eu) enc = 0x7Eu;
  return (uint8_t)(sign | enc);
}

// One 64-bit draw per 8 weight bytes (little-endian), one per scale byte.
__global__ void gen_nvfp4_kernel(uint64_t kw, uint64_t ks, size_t nb, size_t ns, uint8_t *w,
                                 uint8_t *s) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t n8 = nb / 8;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += stride)
    reinterpret_cast<uint64_t *>(w)[i] = rnd(kw, i);
  for (size_t i = n8 * 8 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nb; i += stride)
    w[i] = (uint8_t)(rnd(kw, i >> 3) >> (8 * (i & 7)));
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < ns; i += stride)
    s[i] = f32_to_e4m3(__fdiv_rn(fabsf(normal4_at(ks, i)), 6.0f));
}

__global__ void gen_ternary_kernel(uint64_t kp, uint64_t kr, size_t nbytes, size_t rows,
                                   uint8_t *p, float *rs) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < nbytes; b += stride) {
    uint32_t byte = 0;
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = (uint32_t)(rnd(kp, 4 * b + i) >> 32);
      const uint32_t code = u < 1288490189u ? 0u : (u < 3006477107u ? 1u : 2u);
      byte |= code << (2 * i);
    }
    p[b] = (uint8_t)byte;
  }
  for (size_t r = (size_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += stride)
    rs[r] = __fadd_rn(0.01f, __fmul_rn(0.04f, unit_at(kr, r)));
}

__global__ void gen_core_kernel(uint64_t ka, uint64_t kb, uint64_t kas, uint64_t kbs, size_t na,
                                size_t nb, int8_t *a, float *a_sc, int8_t *b, float *b_sc) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (size_t i = i0; i < na; i += stride) a[i] = (int8_t)((int)(rnd(ka, i) % 255u) - 127);
  for (size_t i = i0; i < nb; i += stride) b[i] = (int8_t)((int)(rnd(kb, i) % 255u) - 127);
  if (i0 < 16) {
    a_sc[i0] = __fadd_rn(0.0001f, __fmul_rn(0.0009f, unit_at(kas, i0)));
    b_sc[i0] = __fadd_rn(0.0001f, __fmul_rn(0.0009f, unit_at(kbs, i0)));
  }
}

__global__ void gen_normal_kernel(uint64_t key, size_t n, float stdev, float *out) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = __fmul_rn(normal_at(key, i), stdev);
}

static int gen_grid(size_t n) {
  const size_t b = (n + 255) / 256;
  return (int)std::max<size_t>(1, std::min<size_t>(b, 148 * 16));
}

int launch_gen_nvfp4(uint64_t kw, uint64_t ks, size_t rows, size_t cols, uint8_t *w, uint8_t *s,
                     cudaStream_t st) {
  const size_t nb = rows * cols / 2, ns = rows * cols / 16;
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "gen_nvfp4_kernel", gen_nvfp4_kernel<<<gen_grid(nb), 256, 0, st>>>(kw, ks, nb, ns, w, s));
  return 0;
}
int launch_gen_ternary(uint64_t kp, uint64_t kr, size_t rows, size_t cols, uint8_t *p, float *rs,
                       cudaStream_t st) {
  const size_t nb = rows * cols / 4;
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "gen_ternary_kernel", gen_ternary_kernel<<<gen_grid(nb), 256, 0, st>>>(kp, kr, nb, rows, p, rs));
  return 0;
}
int launch_gen_core(uint64_t ka, uint64_t kb, uint64_t kas, uint64_t kbs, size_t rows,
                    size_t cols, int8_t *a, float *a_sc, int8_t *b, float *b_sc,
                    cudaStream_t st) {
  const size_t na = 16 * cols, nb = rows * 16;
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "gen_core_kernel", gen_core_kernel<<<gen_grid(std::max(na, nb)), 256, 0, st>>>(ka, kb, kas, kbs, na, nb, a, a_sc,
                                                              b, b_sc));
  return 0;
}
int launch_gen_normal(uint64_t key, size_t n, float stdev, float *out, cudaStream_t st) {
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "gen_normal_kernel", gen_normal_kernel<<<gen_grid(n), 256, 0, st>>>(key, n, stdev, out));
  return 0;
}

// ============================================================ decode checks
__global__ void dequant_nvfp4_kernel(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s,
                                     float *out) {
  const size_t n = rows * cols, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const size_t r = i / cols, c = i % cols;
    const uint32_t b = w[r * (cols / 2) + c / 2];
    const float v = e2m1_to_f32((c & 1) ? (b >> 4) : (b & 15u));
    out[i] = v * e4m3_to_f32(s[r * (cols / 16) + c / 16]);
  }
}
__global__ void dequant_ternary_kernel(size_t rows, size_t cols, const uint8_t *p, float *out) {
  const size_t n = rows * cols, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const size_t r = i / cols, c = i % cols;
    const uint32_t b = p[r * (cols / 4) + c / 4];
    out[i] = tern_to_f32((b >> (2 * (c & 3))) & 3u);
  }
}
int launch_dequant_nvfp4(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s, float *out,
                         cudaStream_t st) {
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "dequant_nvfp4_kernel", dequant_nvfp4_kernel<<<gen_grid(rows * cols), 256, 0, st>>>(rows, cols, w, s, out));
  return 0;
}
int launch_dequant_ternary(size_t rows, size_t cols, const uint8_t *p, float *out,
                           cudaStream_t st) {
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "dequant_ternary_kernel", dequant_ternary_kernel<<<gen_grid(rows * cols), 256, 0, st>>>(rows, cols, p, out));
  return 0;
}

}  // namespace ffn
