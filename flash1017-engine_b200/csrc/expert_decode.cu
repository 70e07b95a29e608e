// Batch decode of one NVFP4 or MXFP4 SwiGLU expert for 1..8 tokens, or one
// ternary expert (rank-16 cores, block scales) for 1 token, in two launches
// (a ternary expert with gate/up cores: the cores' z kernel first).
//
//   phase 1  h[t][i] = min(silu(g), 10) * clamp(u, -10, 10),
//            g = (W1 x_t)_i, u = (W3 x_t)_i          (flash1017.rs:7537-7547)
//   phase 2  y[t][r] = (W2 h_t)_r, written as out (+)= out_w * y
//
// The reference issues this shape once per routed expert and token
// (flash1017.rs:7449-7514, the `*_mlp_accum` call sequence), so its cost is
// latency: the 14 MB of a config-size expert stream in ~2.2 us at the HBM
// rate, while a GEMV chain of activation prep, split-K gate/up and down
// launches takes an order of magnitude longer.  Here:
//
// * one CTA per SM (grid = SM count) owns a contiguous run of output rows and
//   pulls ALL of its rows' codes and scales into shared memory at once, with
//   one bulk copy per matrix and batch of 8 rows (mbarrier per batch), before
//   anything else: every byte of the expert is in flight from the start;
// * both phases are launched with programmatic dependent launch and trigger
//   their dependents on entry, so phase 2's CTAs (and the next call's phase 1)
//   become resident next to the running phase, issue their weight copies, and
//   only then wait for the previous grid (griddepcontrol.wait) before reading
//   activations.  The two phases fit on one SM together (<= 64 registers x 512
//   threads each, about 100 KB of shared memory between them), so the down
//   weights stream while gate/up computes;
// * for 1-2 tokens (any format) the arithmetic is f32 on the CUDA cores: a
//   lane owns one 16-column scale group of a row, decodes its 16 codes exactly
//   (cvt.rn.f16x2.e2m1x2; ternary by sign flips and masks), keeps its 16
//   activations per token in registers across the rows it visits, sums code x
//   activation, times the group's scale (flash1017.rs:2331-2357 sums each
//   group, times its scale, over the row, times the matrix scale); NVFP4 from
//   3 tokens runs mma.sync on the tensor cores (compute_rows_mma), whose work
//   does not grow with the tokens; warps reduce through shuffles and shared
//   memory in a fixed order, so results are deterministic.
//
// Weights and scales are read before the wait on the previous kernel: they
// must not be written by a kernel of the same stream that lets this one start
// early (every library kernel that writes weights runs to completion first).
// A batch copy that does not land within the bounded wait turns the CTA's
// outputs into NaN.

#include "ffn_internal.h"
#include "tcgen05.cuh"

namespace ffn {
namespace dec {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kBatchRows = 8;   // rows per mbarrier
constexpr int kMaxRows = 64;    // rows per CTA
constexpr int kMaxBatches = kMaxRows / kBatchRows;
static_assert(kMaxBatches * 8 <= 128, "the batch barriers fit the first 128 bytes");
constexpr int kMaxTok = 8;
constexpr size_t kSmemCap = 110 * 1024;  // per CTA: both phases side by side on one SM


__device__ __forceinline__ float e8m0_f32(uint32_t b) {  // flash1017.rs:1049-1057
  return b == 0xFFu ? __int_as_float(0x7FC00000) : (b == 0u ? __int_as_float(0x00400000) : __int_as_float(b << 23));
}
// E4M3 (flash1017.rs:1031-1045) through the hardware converter: every E4M3
// value, NaN included, is an f16 value
__device__ __forceinline__ float e4m3_f32(uint32_t b) {
  const uint32_t h2 = e4m3x2_to_f16x2((uint16_t)b);
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}
__device__ __forceinline__ float silu10(float g) { return fminf(g / (1.0f + expf(-g)), 10.0f); }
__device__ __forceinline__ float clamp10(float u) {  // Rust f32::clamp(-10, 10): NaN stays NaN
  if (u < -10.f) u = -10.f;
  if (u > 10.f) u = 10.f;
  return u;
}

// Weight formats of the decode kernels.
constexpr int kNv = 0;    // NVFP4: E2M1 pairs, E4M3 scale per 16 columns, matrix scale
constexpr int kMx = 1;    // MXFP4: E2M1 pairs, E8M0 scale per 32 columns
constexpr int kTern = 2;  // ternary: 2-bit codes, row scale, optional U8 scale per 64 columns, rank-16 core

__host__ __device__ constexpr int code_bytes(int F, int K) { return F == kTern ? K / 4 : K / 2; }
__host__ __device__ constexpr int scale_bytes(int F, int K, bool bs) {
  return F == kNv ? K / 16 : (F == kMx ? K / 32 : (bs ? K / 64 : 0));
}

// Shared memory: batch barriers, then per matrix the rows' codes and scales,
// then the reduction slots red[(row * NMAT + m) * T + t][chunk].
// On the tensor-core path (compute_rows_mma) the code rows sit 16 bytes apart
// beyond their length, so the 8 rows of an MMA fragment fall in different
// banks, and each of the 16 warps leaves one partial per row and token.  The
// CUDA-core path keeps dense rows and one partial per 512-column chunk.
struct Layout {
  int nr, cb, cs, sb, ss, nch;  // rows of this CTA; code bytes per row and row stride; the same for
                                // the scales; partials per row and token
  size_t codes[2], scales[2], red, total;
};
// NVFP4 takes the tensor cores from kMmaTok tokens on: they cost a fixed
// amount per 8 tokens, while the CUDA-core sums grow with every token.
constexpr int kMmaTok = 3;
__host__ __device__ constexpr bool use_mma(int F, int T) { return F == kNv && T >= kMmaTok; }
__host__ __device__ inline Layout layout(int F, bool bs, int nmat, int nr, int K, int T, size_t base = 128) {
  Layout l;
  l.nr = nr;
  l.cb = code_bytes(F, K);
  l.cs = use_mma(F, T) ? l.cb + 16 : l.cb;
  l.sb = scale_bytes(F, K, bs);
  l.ss = use_mma(F, T) ? l.sb + 16 : l.sb;
  l.nch = use_mma(F, T) ? kWarps : K / 512;
  size_t o = base;  // after the barriers
  for (int m = 0; m < nmat; ++m) {
    l.codes[m] = o;
    o += (size_t)nr * l.cs;
    l.scales[m] = o;
    o += (size_t)nr * l.ss;
  }
  l.red = (o + 15) & ~(size_t)15;
  l.total = l.red + (size_t)nr * nmat * T * l.nch * sizeof(float);
  return l;
}

// Halving reduction of eight per-lane values over the warp: afterwards lane l
// holds, in v[0], the warp-wide sum of value 4 b4 + 2 b3 + b2 (b_k = bit k of
// l); 9 shuffles for the eight sums.
__device__ __forceinline__ float reduce8(float (&v)[8], int lane) {
#pragma unroll
  for (int n = 8, o = 16; n > 1; n >>= 1, o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? v[i] : v[i + n / 2];
      const float keep = up ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float r = v[0];
  r += __shfl_xor_sync(0xffffffffu, r, 2);
  r += __shfl_xor_sync(0xffffffffu, r, 1);
  return r;
}

// One phase's matrices: gate and up (NMAT 2) or down (NMAT 1).
struct Phase {
  const uint8_t *w[2];      // codes [rows][code_bytes]
  const uint8_t *s[2];      // scales [rows][scale_bytes] (ternary: U8 block scales or null)
  float gs[2];              // NVFP4 matrix scales
  const float *rs[2];       // ternary row scales [rows]
  const int8_t *core_b[2];  // ternary rank-16 core B [rows][16], or null
  const float *z;           // ternary gate/up: z [token][3][16] (core A x, times a_sc b_sc)
  const int8_t *core_a;     // ternary down core A [16][inter], or null: phase 1 writes partial
                            // sums of A h over its rows, phase 2 adds them up
  const float *a_sc, *b_sc; // ... and its scales [16] (phase 2)
  float *zpart;             // [phase-1 CTA][token][16]
  int zparts;               // phase-1 CTAs (phase 2)
  float proj;               // ternary gate/up pre-scale (tier_b_proj_scale), else 1
  int rows, K;
};

// Thread 0: arm this CTA's batch barriers of one phase and issue the bulk
// copies of its rows [r0, r0 + nr) (barriers initialised and fenced already).
template <int NMAT>
__device__ __forceinline__ void issue_rows(const Phase &p, uint8_t *smem, const Layout &L, uint64_t *bar, int r0,
                                           int nr) {
  const size_t cb = (size_t)L.cb;
  const int nb = (nr + kBatchRows - 1) / kBatchRows;
  for (int b = 0; b < nb; ++b) {
    const int i0 = b * kBatchRows, n = min(kBatchRows, nr - i0);
    tc::bar_arrive_tx(&bar[b], (uint32_t)(NMAT * n * (cb + L.sb)));
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      if (L.cs == L.cb) {
        tc::bulk_g2s(smem + L.codes[m] + i0 * cb, p.w[m] + (size_t)(r0 + i0) * cb, (uint32_t)(n * cb), &bar[b]);
      } else {
        for (int i = i0; i < i0 + n; ++i)  // one copy per row into its padded slot
          tc::bulk_g2s(smem + L.codes[m] + (size_t)i * L.cs, p.w[m] + (size_t)(r0 + i) * cb, (uint32_t)cb, &bar[b]);
      }
      if (L.sb && L.ss == L.sb) {
        tc::bulk_g2s(smem + L.scales[m] + (size_t)i0 * L.sb, p.s[m] + (size_t)(r0 + i0) * L.sb,
                     (uint32_t)(n * L.sb), &bar[b]);
      } else if (L.sb) {
        for (int i = i0; i < i0 + n; ++i)
          tc::bulk_g2s(smem + L.scales[m] + (size_t)i * L.ss, p.s[m] + (size_t)(r0 + i) * L.sb, (uint32_t)L.sb,
                       &bar[b]);
      }
    }
  }
}

// Sum over a lane's 16 columns of L(code) x for one row (per token), times
// the group's scale: E2M1 via the hardware f16x2 decode; ternary codes
// (0 -> -1, 1 -> 0, 2 -> +1, 3 -> 0, flash1017.rs:2566) by sign flips and masks.
template <int F, int TQ>
__device__ __forceinline__ void row_group(const uint8_t *cptr, float sc, const float (&xr)[TQ][16],
                                          float (&acc)[TQ]) {
#pragma unroll
  for (int t = 0; t < TQ; ++t) acc[t] = 0.f;
  if (F == kTern) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(cptr);
    const uint32_t neg = ~w & ~(w >> 1) & 0x55555555u;  // bit 2i: code i == 0
    const uint32_t pos = (w >> 1) & ~w & 0x55555555u;   // bit 2i: code i == 2
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t keep = 0u - (((neg | pos) >> (2 * i)) & 1u);  // all ones for +-1
      const uint32_t flip = ((neg >> (2 * i)) & 1u) << 31;
#pragma unroll
      for (int t = 0; t < TQ; ++t)
        acc[t] += __uint_as_float((__float_as_uint(xr[t][i]) ^ flip) & keep);
    }
  } else {
    const uint2 cw = *reinterpret_cast<const uint2 *>(cptr);
#pragma unroll
    for (int hw = 0; hw < 2; ++hw) {
      uint32_t q4[4];
      e2m1x8_to_f16x2(hw ? cw.y : cw.x, q4);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 w2 = __half22float2(*reinterpret_cast<const __half2 *>(&q4[j]));
        const int k = 8 * hw + 2 * j;
#pragma unroll
        for (int t = 0; t < TQ; ++t) acc[t] = fmaf(w2.y, xr[t][k + 1], fmaf(w2.x, xr[t][k], acc[t]));
      }
    }
  }
#pragma unroll
  for (int t = 0; t < TQ; ++t) acc[t] *= sc;
}

// NVFP4 on the tensor cores (mma.sync m16n8k16, f16 in, f32 accumulate): the
// A operand is 16 weight rows, E2M1 codes times their E4M3 block scale in f16
// (exact: at most 6 significant bits, 2^-10 .. 2688); the B operand is the
// tokens (up to 8, one per MMA column) as two f16 terms hi + lo of x 2^-e,
// e per token and warp from the maximum over the warp's columns, so the MMAs
// reproduce f32 products to ~2^-22.  Warp w takes the 128-column blocks
// w, w + 16, ...; in a block, lane (g, q) = (lane / 4, lane % 4) reads the
// 32-bit code word 4v + q (v = 0..3: columns 32v + 8q .. + 7) of rows g and
// g + 8 and feeds them to k16 tiles 2v and 2v + 1 as their columns
// 32v + 8q .. + 3 and + 4 .. + 7 (the k order inside a tile is free as long as
// A and B agree).  Code rows 16 bytes apart beyond their length put the 32
// lanes' words in 32 banks; scale rows likewise.  Each warp leaves one partial
// per row and token, times its 2^e, for finish_rows to add in warp order.
template <int NMAT>
__device__ __forceinline__ bool compute_rows_mma(const Phase &p, const uint8_t *smem, const Layout &L,
                                                 uint64_t *bar, int nr, int T, const float *x, int ld_x,
                                                 int *s_err) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int nblk = p.K / 128, ntile = (nr + 15) / 16, nitem = NMAT * ntile;
  float *red = reinterpret_cast<float *>(const_cast<uint8_t *>(smem) + L.red);
  bool ok = true;
  // the token's scale exponent over this warp's columns (lanes of token g),
  // while the rows' copies are still landing
  const bool have = g < T;
  const float *xrow = x + (size_t)(have ? g : 0) * ld_x + 8 * q;
  float xm = 0.f;
  if (have)
    for (int blk = warp; blk < nblk; blk += kWarps) {
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const float4 *src = reinterpret_cast<const float4 *>(xrow + 128 * blk + 32 * v);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float4 f = __ldcg(src + u);
          xm = fmaxf(xm, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
        }
      }
    }
  xm = fmaxf(xm, __shfl_xor_sync(0xffffffffu, xm, 1));
  xm = fmaxf(xm, __shfl_xor_sync(0xffffffffu, xm, 2));
  int e = 0;
  if (xm > 0.f && isfinite(xm)) {
    int ex;
    frexpf(xm, &ex);  // xm < 2^ex: |x 2^-e| < 2^15 with e = ex - 15
    e = max(-100, min(100, ex - 15));
  }
  const float xs = pow2f(-e);
  // the exponents of this lane's two accumulator columns (tokens 2q, 2q + 1)
  const float c0s = pow2f(__shfl_sync(0xffffffffu, e, 8 * q)), c1s = pow2f(__shfl_sync(0xffffffffu, e, 8 * q + 4));
  const int nb = (nr + kBatchRows - 1) / kBatchRows;
  for (int b = 0; b < nb; ++b) ok = tc::bar_wait(&bar[b], 0u, s_err) && ok;
  for (int it0 = 0; it0 < nitem; it0 += 2) {
    float acc[2][4];
#pragma unroll
    for (int ii = 0; ii < 2; ++ii)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[ii][k] = 0.f;
    for (int blk = warp; blk < nblk; blk += kWarps) {
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        // B: x of token g, columns 32v + 8q .. + 7 (tiles 2v and 2v + 1), hi and lo
        uint32_t bh[4], bl[4];
        {
          float xv[8];
          if (have) {
            const float4 *src = reinterpret_cast<const float4 *>(xrow + 128 * blk + 32 * v);
            const float4 f0 = __ldcg(src), f1 = __ldcg(src + 1);
            xv[0] = f0.x; xv[1] = f0.y; xv[2] = f0.z; xv[3] = f0.w;
            xv[4] = f1.x; xv[5] = f1.y; xv[6] = f1.z; xv[7] = f1.w;
          } else {
#pragma unroll
            for (int u = 0; u < 8; ++u) xv[u] = 0.f;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            __half h0, l0, h1, l1;
            split_f16(xv[2 * u] * xs, h0, l0);
            split_f16(xv[2 * u + 1] * xs, h1, l1);
            bh[u] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            bl[u] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
          }
        }
#pragma unroll
        for (int ii = 0; ii < 2; ++ii) {
          const int it = it0 + ii;
          if (it >= nitem) break;  // warp-uniform
          const int m = it % NMAT, tile = it / NMAT;
          const uint8_t *cbase = smem + (m ? L.codes[NMAT - 1] : L.codes[0]) + 64 * blk + 4 * (4 * v + q);
          const uint8_t *sbase = smem + (m ? L.scales[NMAT - 1] : L.scales[0]) + 8 * blk + 2 * v + (q >> 1);
          const int ra = tile * 16 + g, rb = ra + 8;
          const uint32_t wa = ra < nr ? *reinterpret_cast<const uint32_t *>(cbase + (size_t)ra * L.cs) : 0u;
          const uint32_t wb = rb < nr ? *reinterpret_cast<const uint32_t *>(cbase + (size_t)rb * L.cs) : 0u;
          // the word's 16-column group scale of each row, in both f16 halves
          const uint32_t pa = e4m3x2_to_f16x2(ra < nr ? sbase[(size_t)ra * L.ss] : 0);
          const uint32_t pb = e4m3x2_to_f16x2(rb < nr ? sbase[(size_t)rb * L.ss] : 0);
          const uint32_t sa = (pa & 0xFFFFu) * 0x10001u, sb = (pb & 0xFFFFu) * 0x10001u;
          uint32_t qa[4], qb[4];
          e2m1x8_to_f16x2(wa, qa);
          e2m1x8_to_f16x2(wb, qb);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            __half2 ha = __hmul2(*reinterpret_cast<const __half2 *>(&qa[k]), *reinterpret_cast<const __half2 *>(&sa));
            __half2 hb = __hmul2(*reinterpret_cast<const __half2 *>(&qb[k]), *reinterpret_cast<const __half2 *>(&sb));
            qa[k] = *reinterpret_cast<uint32_t *>(&ha);
            qb[k] = *reinterpret_cast<uint32_t *>(&hb);
          }
          // tile 2v: bytes 0 (k slots 2q, 2q+1) and 1 (2q+8, 2q+9); tile 2v + 1: bytes 2 and 3
          mma_f16(acc[ii], qa[0], qb[0], qa[1], qb[1], bh[0], bh[1]);
          mma_f16(acc[ii], qa[0], qb[0], qa[1], qb[1], bl[0], bl[1]);
          mma_f16(acc[ii], qa[2], qb[2], qa[3], qb[3], bh[2], bh[3]);
          mma_f16(acc[ii], qa[2], qb[2], qa[3], qb[3], bl[2], bl[3]);
        }
      }
    }
#pragma unroll
    for (int ii = 0; ii < 2; ++ii) {
      const int it = it0 + ii;
      if (it >= nitem) break;
      const int m = it % NMAT, tile = it / NMAT;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int row = tile * 16 + g + 8 * (k >> 1), t = 2 * q + (k & 1);
        if (row < nr && t < T)
          red[((size_t)(row * NMAT + m) * T + t) * kWarps + warp] = acc[ii][k] * ((k & 1) ? c1s : c0s);
      }
    }
  }
  return ok;
}

// All warps: the partial sums of this CTA's rows of one phase into the
// reduction slots.  A warp task = one column chunk (512 columns: a 16-column
// group per lane) of RB = 8 / TQ rows of one matrix, for TQ tokens whose
// activations stay in registers; its 8 sums (RB rows x TQ tokens) leave
// through one halving reduction.  Tokens beyond TQ take further passes.
// Returns false when a batch of rows did not land in time.
template <int NMAT, int F, int TQ>
__device__ __forceinline__ bool compute_rows(const Phase &p, const uint8_t *smem, const Layout &L, uint64_t *bar,
                                             int nr, int T, const float *x, int ld_x, int *s_err) {
  if (use_mma(F, T)) return compute_rows_mma<NMAT>(p, smem, L, bar, nr, T, x, ld_x, s_err);
  constexpr int RB = 8 / TQ;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int C = p.K / 512;  // column chunks of 32 groups of 16
  const int c = warp % C, slot = warp / C, nslots = kWarps / C;
  const int g = c * 32 + lane;  // this lane's 16-column group
  const int nrb = (nr + RB - 1) / RB;
  const int ntask = nrb * NMAT;
  float *red = reinterpret_cast<float *>(const_cast<uint8_t *>(smem) + L.red);
  const int vi = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);  // reduce8's value
  const int cg = F == kTern ? 4 * g : 8 * g;                                          // code byte of the group
  const int sg = F == kNv ? g : (F == kMx ? g >> 1 : g >> 2);                         // scale byte of the group
  bool ok = true;
  for (int tp = 0; tp < T; tp += TQ) {
    float xr[TQ][16];
#pragma unroll
    for (int t = 0; t < TQ; ++t) {
      const bool have = tp + t < T;
      const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)(have ? tp + t : 0) * ld_x + 16 * g);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f = have ? __ldcg(src + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        xr[t][4 * q] = f.x; xr[t][4 * q + 1] = f.y; xr[t][4 * q + 2] = f.z; xr[t][4 * q + 3] = f.w;
      }
    }
    for (int task = slot; task < ntask; task += nslots) {
      const int rb = task / NMAT, m = task - rb * NMAT;
      const int i0 = rb * RB;
      ok = tc::bar_wait(&bar[i0 / kBatchRows], 0u, s_err) && ok;  // returns at once after the first time
      const uint8_t *cbase = smem + (m ? L.codes[NMAT - 1] : L.codes[0]) + (size_t)i0 * L.cb + cg;
      const uint8_t *sbase = smem + (m ? L.scales[NMAT - 1] : L.scales[0]) + (size_t)i0 * L.ss + sg;
      float v[8];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        float acc[TQ];
        if (i0 + r < nr) {
          float sc = 1.0f;
          if (F == kNv) sc = e4m3_f32(sbase[r * L.ss]);
          else if (F == kMx) sc = e8m0_f32(sbase[r * L.ss]);
          else if (L.sb) sc = (float)sbase[r * L.ss];
          row_group<F, TQ>(cbase + r * L.cb, sc, xr, acc);
        } else {
#pragma unroll
          for (int t = 0; t < TQ; ++t) acc[t] = 0.f;
        }
#pragma unroll
        for (int t = 0; t < TQ; ++t) v[t * RB + r] = acc[t];
      }
      const float sum = reduce8(v, lane);
      const int t = vi / RB, r = vi - t * RB;
      if ((lane & 3) == 0 && i0 + r < nr && tp + t < T)
        red[((size_t)((i0 + r) * NMAT + m) * T + tp + t) * C + c] = sum;
    }
  }
  return ok;
}

// The rank-16 core's term of a row (flash1017.rs:2465-2472 in the oracle's
// order): sum_r B[row][r] z[r], z already times a_sc b_sc.
__device__ __forceinline__ float core_row(const int8_t *b, int row, const float *z) {
  const int4 v = __ldg(reinterpret_cast<const int4 *>(b + (size_t)row * 16));
  const int8_t *bb = reinterpret_cast<const int8_t *>(&v);
  float acc = 0.f;
#pragma unroll
  for (int r = 0; r < 16; ++r) acc += (float)bb[r] * z[r];
  return acc;
}

// Ternary down core, z[t][r] = (sum_c A[r][c] h[t][c]) a_sc[r] b_sc[r]
// (flash1017.rs:2452-2463), split over the phases: a phase-1 CTA owns h's
// columns [r0, r0 + nr), so it writes the partial sums over them
// (core_partial, from h in shared memory); phase 2 adds the CTAs' partials in
// CTA order (core_sum).
__device__ __forceinline__ void core_partial(const Phase &p, int r0, int nr, int T, const float *s_h) {
  for (int q = threadIdx.x; q < T * 16; q += kThreads) {
    const int t = q >> 4, r = q & 15;
    const int8_t *arow = p.core_a + (size_t)r * p.rows + r0;
    float acc = 0.f;
    for (int i = 0; i < nr; ++i) acc = fmaf((float)__ldg(arow + i), s_h[t * kMaxRows + i], acc);
    p.zpart[((size_t)blockIdx.x * T + t) * 16 + r] = acc;
  }
}
__device__ __forceinline__ void core_sum(const Phase &p, int T, float *s_z) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int item = warp; item < T * 16; item += kWarps) {
    const int t = item >> 4, r = item & 15;
    float acc = 0.f;
    for (int b = lane; b < p.zparts; b += 32) acc += __ldcg(p.zpart + ((size_t)b * T + t) * 16 + r);
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) s_z[t * 16 + r] = acc * __ldg(p.a_sc + r) * __ldg(p.b_sc + r);
  }
}

// After a __syncthreads: each (row, token) sums its chunks in order and
// scales (NVFP4: the matrix scale; ternary: the row scale, then + the core
// term); phase 1 writes h = min(silu(g), 10) * clamp(u, -10, 10) (ternary:
// g, u times proj first), phase 2 out (+)= out_w * y.  NaN where `bad`.
template <int NMAT, int F>
__device__ __forceinline__ void finish_rows(const Phase &p, const uint8_t *smem, const Layout &L, int r0, int nr,
                                            int T, bool bad, const float *s_z, float *s_h, float *h, int ld_h,
                                            float *y, int ld_y, float out_w, int accumulate) {
  const int C = L.nch;
  const float *red = reinterpret_cast<const float *>(smem + L.red);
  for (int idx = threadIdx.x; idx < nr * T; idx += kThreads) {
    const int i = idx / T, t = idx - i * T;
    float v[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const float *rr = red + ((size_t)(i * NMAT + m) * T + t) * C;
      float s = 0.f;
      for (int k = 0; k < C; ++k) s += rr[k];
      if (F == kNv) s *= p.gs[m];
      if (F == kTern) {
        s *= __ldg(p.rs[m] + r0 + i);
        if (p.core_b[m]) s += core_row(p.core_b[m], r0 + i, s_z + (t * NMAT + m) * 16);
      }
      v[m] = s;
    }
    if (NMAT == 2) {
      float gv = v[0], uv = v[NMAT - 1];
      if (F == kTern) { gv *= p.proj; uv *= p.proj; }
      const float hv = bad ? __int_as_float(0x7FC00000) : silu10(gv) * clamp10(uv);
      h[(size_t)t * ld_h + r0 + i] = hv;
      if (s_h) s_h[t * kMaxRows + i] = hv;
    } else {
      float *dst = y + (size_t)t * ld_y + r0 + i;
      const float wy = out_w * v[0];  // flash1017.rs:4900-4905 (dst += scale * src)
      *dst = bad ? __int_as_float(0x7FC00000) : (accumulate ? *dst + wy : wy);
    }
  }
}

__device__ __forceinline__ void rows_of(int rows, int &r0, int &nr) {
  r0 = (int)((long long)blockIdx.x * rows / gridDim.x);
  nr = (int)((long long)(blockIdx.x + 1) * rows / gridDim.x) - r0;
}

struct DecArgs {
  Phase p;
  int T;
  const float *x;  // [T][ld_x] activations (x; h for phase 2)
  int ld_x;
  float *h;        // phase 1 output [T][ld_h]
  int ld_h;
  float *y;        // phase 2 output [T][ld_y]
  int ld_y;
  float out_w;
  int accumulate;
};

// One phase per launch: PHASE 1 gate (matrix 0) and up (matrix 1) -> h,
// PHASE 2 down -> y.
template <int PHASE, int F, int TQ>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(const DecArgs a) {
  constexpr int NMAT = PHASE == 1 ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
  __shared__ int s_err;
  int r0, nr;
  rows_of(a.p.rows, r0, nr);
  const Layout L = layout(F, a.p.s[0] != nullptr, NMAT, nr, a.p.K, a.T);
  const int nb = (nr + kBatchRows - 1) / kBatchRows;
  if (threadIdx.x == 0) {
    s_err = 0;
    for (int b = 0; b < nb; ++b) tc::bar_init(&bar[b], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    issue_rows<NMAT>(a.p, smem, L, bar, r0, nr);
  }
  // the next kernel may now be scheduled; it waits for this grid's completion
  // before it reads what this grid writes
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncthreads();
  // activations (and, for phase 2, h; ternary: z) come from the previous kernels
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float s_z[kMaxTok * 2 * 16];  // ternary cores' z [token][matrix][16]
  if (F == kTern) {
    if (PHASE == 1 && (a.p.core_b[0] || a.p.core_b[1])) {
      for (int q = threadIdx.x; q < a.T * 2 * 16; q += kThreads) {
        const int t = q >> 5, m = (q >> 4) & 1, r = q & 15;
        s_z[q] = __ldcg(a.p.z + ((size_t)t * 3 + m) * 16 + r);
      }
    }
    if (PHASE == 2 && a.p.core_a) core_sum(a.p, a.T, s_z);
  }
  const bool ok = compute_rows<NMAT, F, TQ>(a.p, smem, L, bar, nr, a.T, a.x, a.ld_x, &s_err);
  __syncthreads();
  __shared__ float s_h[F == kTern && PHASE == 1 ? kMaxTok * kMaxRows : 1];  // this CTA's h for the down core
  const bool partial = F == kTern && PHASE == 1 && a.p.core_a != nullptr;
  finish_rows<NMAT, F>(a.p, smem, L, r0, nr, a.T, s_err != 0 || !ok, s_z, partial ? s_h : nullptr, a.h, a.ld_h,
                       a.y, a.ld_y, a.out_w, a.accumulate);
  if (partial) {
    __syncthreads();
    core_partial(a.p, r0, nr, a.T, s_h);
  }
  // no bulk copy may still be landing when the CTA's shared memory is released
  if (threadIdx.x == 0)
    for (int b = 0; b < nb; ++b) tc::bar_wait_drain(&bar[b], 0u);
}

}  // namespace dec

// Device SM count, cached per device.
static int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cache[dev] = n;
  }
  return cache[dev];
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }


// Which decode format an expert takes, or -1: NVFP4 / MXFP4 / ternary with
// the shapes, alignment and shared-memory budget of the kernels.
static int decode_format(const ffn_b200_expert &e, size_t inter, size_t hidden, size_t seq) {
  using namespace dec;
  const int F = e.format == FFN_B200_FMT_NVFP4 ? kNv
                : e.format == FFN_B200_FMT_MXFP4 ? kMx
                : e.format == FFN_B200_FMT_TERNARY ? kTern : -1;
  if (F < 0 || seq < 1 || seq > (size_t)kMaxTok) return -1;
  // ternary: the sign-and-mask decode costs about twice the E2M1 one per
  // value and is repeated per token pass; from 2 tokens on the GEMV engine's
  // tensor-core decode is as fast
  if (F == kTern && seq > 1) return -1;
  if (inter % 512 || hidden % 512 || inter > 8192 || hidden > 8192) return -1;
  if (16 % (inter / 512) || 16 % (hidden / 512)) return -1;  // column chunks split the 16 warps evenly
  const int sms = sm_count();
  if (sms <= 0) return -1;
  bool bs1 = false, bs2 = false;
  if (F == kTern) {
    for (int m = 0; m < 3; ++m) {
      const ffn_b200_ternary_mat &t = e.tn[m];
      if (!t.p || !t.rs || !aligned16(t.p)) return -1;
      if ((t.core_a == nullptr) != (t.core_b == nullptr)) return -1;
      if (t.core_a && (!t.core_a_sc || !t.core_b_sc || !aligned16(t.core_a) || !aligned16(t.core_b))) return -1;
      if (t.bs && !aligned16(t.bs)) return -1;
    }
    if ((e.tn[0].bs == nullptr) != (e.tn[1].bs == nullptr)) return -1;  // gate and up alike
    bs1 = e.tn[0].bs != nullptr;
    bs2 = e.tn[2].bs != nullptr;
    if ((bs1 && hidden % 1024) || (bs2 && inter % 1024)) return -1;  // 16-byte rows of block scales
  } else {
    for (int m = 0; m < 3; ++m)
      if (!e.nv[m].w || !e.nv[m].s || !aligned16(e.nv[m].w) || !aligned16(e.nv[m].s)) return -1;
  }
  const int nr1 = (int)((inter + sms - 1) / sms), nr2 = (int)((hidden + sms - 1) / sms);
  if (nr1 > kMaxRows || nr2 > kMaxRows) return -1;
  const size_t s1 = layout(F, bs1, 2, nr1, (int)hidden, (int)seq).total;
  const size_t s2 = layout(F, bs2, 1, nr2, (int)inter, (int)seq).total;
  return s1 <= kSmemCap && s2 <= kSmemCap && s1 + s2 <= 200 * 1024 ? F : -1;
}

bool expert_decode_fits(const ffn_b200_expert &e, size_t inter, size_t hidden, size_t seq) {
  return decode_format(e, inter, hidden, seq) >= 0;
}

// h [seq][inter] f32, then (ternary cores) z [seq][3][16] f32 and the down
// core's partial sums [phase-1 CTAs <= 1024][seq][16] f32
static size_t h_bytes(size_t inter, size_t seq) { return (seq * inter * sizeof(float) + 15) & ~(size_t)15; }
size_t expert_decode_ws_bytes(size_t inter, size_t seq) {
  return h_bytes(inter, seq) + seq * 48 * sizeof(float) + (size_t)1024 * seq * 16 * sizeof(float);
}

template <int PHASE, int F, int TQ>
static int launch_dec(const dec::DecArgs &a, int grid, size_t smem, cudaStream_t st, int kind, const char *name) {
  static bool attr[64] = {false};
  int dev = 0;
  FFN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "expert decode: device index >= 64");
  if (!attr[dev]) {
    FFN_CUDA_TRY(cudaFuncSetAttribute(dec::decode_kernel<PHASE, F, TQ>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dec::kSmemCap));
    // the largest shared-memory carve-out for both phases, so that a phase-2
    // CTA finds room next to a running phase-1 CTA without a reconfiguration
    FFN_CUDA_TRY(cudaFuncSetAttribute(dec::decode_kernel<PHASE, F, TQ>,
                                      cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    attr[dev] = true;
  }
  FFN_LAUNCH_PDL(kind, st, name, (dec::decode_kernel<PHASE, F, TQ>), grid, dec::kThreads, smem, a);
  return 0;
}

template <int F>
static int run_decode(const ffn_b200_expert &e, int inter, int hidden, int seq, const float *x, float *out,
                      float w, int accumulate, float *h, float *z, float *zpart, cudaStream_t st) {
  using dec::kTern;
  const int sms = sm_count();
  dec::Phase p1{}, p2{};
  p1.rows = inter;
  p1.K = hidden;
  p1.proj = 1.0f;
  p2.rows = hidden;
  p2.K = inter;
  p2.proj = 1.0f;
  if (F == kTern) {
    for (int m = 0; m < 2; ++m) {
      p1.w[m] = e.tn[m].p;
      p1.s[m] = e.tn[m].bs;
      p1.rs[m] = e.tn[m].rs;
      p1.core_b[m] = e.tn[m].core_b;
    }
    p1.z = z;
    p1.proj = e.proj_scale;
    p2.w[0] = e.tn[2].p;
    p2.s[0] = e.tn[2].bs;
    p2.rs[0] = e.tn[2].rs;
    p2.core_b[0] = e.tn[2].core_b;
    p1.core_a = p2.core_a = e.tn[2].core_a;
    p2.a_sc = e.tn[2].core_a_sc;
    p2.b_sc = e.tn[2].core_b_sc;
    p1.zpart = p2.zpart = zpart;
    p2.zparts = min(sms, inter);  // phase 1's grid
    if (e.tn[0].core_a || e.tn[1].core_a) {  // gate/up cores' z from their own kernel
      CoreZArgs c{};
      c.direct = e;
      c.n_tok_direct = seq;
      c.K = hidden;
      c.mat0 = 0;
      c.nmat = 2;
      c.xf = x;
      c.ld_xf = hidden;
      c.z = z;
      if (int rc = launch_corez(c, (seq + kNTok - 1) / kNTok, st)) return rc;
    }
  } else {
    for (int m = 0; m < 2; ++m) {
      p1.w[m] = e.nv[m].w;
      p1.s[m] = e.nv[m].s;
      p1.gs[m] = e.nv[m].gs;
    }
    p2.w[0] = e.nv[2].w;
    p2.s[0] = e.nv[2].s;
    p2.gs[0] = e.nv[2].gs;
  }
  const int g1 = min(sms, inter), g2 = min(sms, hidden);
  const int k1 = F == kTern ? FFN_B200_K_GATEUP_TERNARY : FFN_B200_K_GATEUP_NVFP4;
  const int k2 = F == kTern ? FFN_B200_K_DOWN_TERNARY : FFN_B200_K_DOWN_NVFP4;
  dec::DecArgs a{};
  a.p = p1;
  a.T = seq;
  a.x = x;
  a.ld_x = hidden;
  a.h = h;
  a.ld_h = inter;
  const size_t sm1 = dec::layout(F, p1.s[0] != nullptr, 2, (inter + g1 - 1) / g1, hidden, seq).total;
  int rc = seq == 1 ? launch_dec<1, F, 1>(a, g1, sm1, st, k1, "decode_kernel<1>")
                    : launch_dec<1, F, 2>(a, g1, sm1, st, k1, "decode_kernel<1>");
  if (rc) return rc;
  dec::DecArgs b{};
  b.p = p2;
  b.T = seq;
  b.x = h;
  b.ld_x = inter;
  b.y = out;
  b.ld_y = hidden;
  b.out_w = w;
  b.accumulate = accumulate;
  const size_t sm2 = dec::layout(F, p2.s[0] != nullptr, 1, (hidden + g2 - 1) / g2, inter, seq).total;
  return seq == 1 ? launch_dec<2, F, 1>(b, g2, sm2, st, k2, "decode_kernel<2>")
                  : launch_dec<2, F, 2>(b, g2, sm2, st, k2, "decode_kernel<2>");
}

int launch_expert_decode(const ffn_b200_expert &e, size_t inter, size_t hidden, size_t seq, const float *x,
                         float *out, float accum_weight, int accumulate, void *ws, cudaStream_t st) {
  float *h = static_cast<float *>(ws);
  float *z = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + h_bytes(inter, seq));
  float *zpart = z + seq * 48;
  if (sm_count() > 1024) return fail(FFN_B200_EUNSUP, "expert decode: more than 1024 SMs");
  if (!aligned16(ws) || !aligned16(x) || !aligned16(out) || (hidden % 4))
    return fail(FFN_B200_EUNSUP, "expert decode: x, out and ws must be 16-byte aligned");
  const int I = (int)inter, H = (int)hidden, T = (int)seq;
  switch (decode_format(e, inter, hidden, seq)) {
    case dec::kNv: return run_decode<dec::kNv>(e, I, H, T, x, out, accum_weight, accumulate, h, z, zpart, st);
    case dec::kMx: return run_decode<dec::kMx>(e, I, H, T, x, out, accum_weight, accumulate, h, z, zpart, st);
    case dec::kTern:
      return run_decode<dec::kTern>(e, I, H, T, x, out, accum_weight, accumulate, h, z, zpart, st);
    default: return fail(FFN_B200_EUNSUP, "expert decode: expert or shape not supported");
  }
}

}  // namespace ffn
