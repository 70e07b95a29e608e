// Batch decode of one NVFP4 (or MXFP4) SwiGLU expert for 1..8 tokens in two
// launches and no other device work.
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
// * arithmetic is f32 on the CUDA cores: a lane owns one 16-column scale
//   group of a row, decodes its 16 E2M1 codes exactly (cvt.rn.f16x2.e2m1x2),
//   keeps its 16 activations per token in registers across the rows it visits,
//   sums code x activation, times the group's scale (flash1017.rs:2331-2357
//   sums each group, times its scale, over the row, times the matrix scale);
//   lanes and column-chunk warps reduce through shuffles and shared memory in
//   a fixed order, so results are deterministic.
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

// Shared memory: batch barriers, then per matrix the rows' codes and scales,
// then the reduction slots red[(row * NMAT + m) * T + t][chunk].
struct Layout {
  int nr, sb;              // rows of this CTA, scale bytes per row
  size_t codes[2], scales[2], red, total;
};
__host__ __device__ inline Layout layout(int nmat, int nr, int K, int T, bool mx, size_t base = 128) {
  Layout l;
  l.nr = nr;
  l.sb = mx ? K / 32 : K / 16;
  size_t o = base;  // after the barriers
  for (int m = 0; m < nmat; ++m) {
    l.codes[m] = o;
    o += (size_t)nr * (K / 2);
    l.scales[m] = o;
    o += (size_t)nr * l.sb;
  }
  l.red = (o + 15) & ~(size_t)15;
  l.total = l.red + (size_t)nr * nmat * T * (K / 512) * sizeof(float);
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
  const uint8_t *w[2];
  const uint8_t *s[2];
  float gs[2];
  int rows, K;
};

// Thread 0: arm this CTA's batch barriers of one phase and issue the bulk
// copies of its rows [r0, r0 + nr) (barriers initialised and fenced already).
template <int NMAT>
__device__ __forceinline__ void issue_rows(const Phase &p, uint8_t *smem, const Layout &L, uint64_t *bar, int r0,
                                           int nr) {
  const size_t cb = (size_t)p.K / 2;
  const int nb = (nr + kBatchRows - 1) / kBatchRows;
  for (int b = 0; b < nb; ++b) {
    const int i0 = b * kBatchRows, n = min(kBatchRows, nr - i0);
    tc::bar_arrive_tx(&bar[b], (uint32_t)(NMAT * n * (cb + L.sb)));
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      tc::bulk_g2s(smem + L.codes[m] + i0 * cb, p.w[m] + (size_t)(r0 + i0) * cb, (uint32_t)(n * cb), &bar[b]);
      tc::bulk_g2s(smem + L.scales[m] + (size_t)i0 * L.sb, p.s[m] + (size_t)(r0 + i0) * L.sb, (uint32_t)(n * L.sb),
                   &bar[b]);
    }
  }
}

// All warps: the partial sums of this CTA's rows of one phase into the
// reduction slots.  A warp task = one column chunk (512 columns: a 16-column
// group per lane) of RB = 8 / TQ rows of one matrix, for TQ tokens whose
// activations stay in registers; its 8 sums (RB rows x TQ tokens) leave
// through one halving reduction.  Tokens beyond TQ take further passes.
// Returns false when a batch of rows did not land in time.
template <int NMAT, bool MX, int TQ>
__device__ __forceinline__ bool compute_rows(const Phase &p, const uint8_t *smem, const Layout &L, uint64_t *bar,
                                             int nr, int T, const float *x, int ld_x, int *s_err) {
  constexpr int RB = 8 / TQ;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t cb = (size_t)p.K / 2;
  const int C = p.K / 512;  // column chunks of 32 groups of 16
  const int c = warp % C, slot = warp / C, nslots = kWarps / C;
  const int g = c * 32 + lane;  // this lane's 16-column group
  const int nrb = (nr + RB - 1) / RB;
  const int ntask = nrb * NMAT;
  float *red = reinterpret_cast<float *>(const_cast<uint8_t *>(smem) + L.red);
  const int vi = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);  // reduce8's value
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
      const uint8_t *cbase = smem + (m ? L.codes[NMAT - 1] : L.codes[0]) + (size_t)i0 * cb + 8 * g;
      const uint8_t *sbase = smem + (m ? L.scales[NMAT - 1] : L.scales[0]) + (size_t)i0 * L.sb + (MX ? g >> 1 : g);
      float v[8];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        float acc[TQ];
#pragma unroll
        for (int t = 0; t < TQ; ++t) acc[t] = 0.f;
        if (i0 + r < nr) {
          const uint2 cw = *reinterpret_cast<const uint2 *>(cbase + r * cb);
          const uint32_t sbyte = sbase[r * L.sb];
          const float sc = MX ? e8m0_f32(sbyte) : e4m3_f32(sbyte);
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
#pragma unroll
          for (int t = 0; t < TQ; ++t) acc[t] *= sc;
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

// After a __syncthreads: each (row, token) sums its chunks in order, times the
// matrix scale; phase 1 writes h = min(silu(g), 10) * clamp(u, -10, 10),
// phase 2 out (+)= out_w * y.  NaN where `bad`.
template <int NMAT, bool MX>
__device__ __forceinline__ void finish_rows(const Phase &p, const uint8_t *smem, const Layout &L, int r0, int nr,
                                            int T, bool bad, float *h, int ld_h, float *y, int ld_y, float out_w,
                                            int accumulate) {
  const int C = p.K / 512;
  const float *red = reinterpret_cast<const float *>(smem + L.red);
  for (int idx = threadIdx.x; idx < nr * T; idx += kThreads) {
    const int i = idx / T, t = idx - i * T;
    float v[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const float *rr = red + ((size_t)(i * NMAT + m) * T + t) * C;
      float s = 0.f;
      for (int k = 0; k < C; ++k) s += rr[k];
      v[m] = MX ? s : s * p.gs[m];
    }
    if (NMAT == 2) {
      h[(size_t)t * ld_h + r0 + i] = bad ? __int_as_float(0x7FC00000) : silu10(v[0]) * clamp10(v[NMAT - 1]);
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
template <int PHASE, bool MX, int TQ>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(const DecArgs a) {
  constexpr int NMAT = PHASE == 1 ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
  __shared__ int s_err;
  int r0, nr;
  rows_of(a.p.rows, r0, nr);
  const Layout L = layout(NMAT, nr, a.p.K, a.T, MX);
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
  // activations (and, for phase 2, h) come from the previous kernels
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const bool ok = compute_rows<NMAT, MX, TQ>(a.p, smem, L, bar, nr, a.T, a.x, a.ld_x, &s_err);
  __syncthreads();
  finish_rows<NMAT, MX>(a.p, smem, L, r0, nr, a.T, s_err != 0 || !ok, a.h, a.ld_h, a.y, a.ld_y, a.out_w,
                        a.accumulate);
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


bool expert_decode_fits(const ffn_b200_expert &e, size_t inter, size_t hidden, size_t seq) {
  if (e.format != FFN_B200_FMT_NVFP4 && e.format != FFN_B200_FMT_MXFP4) return false;
  if (seq < 1 || seq > (size_t)dec::kMaxTok) return false;
  if (inter % 512 || hidden % 512 || inter > 8192 || hidden > 8192) return false;
  if (16 % (inter / 512) || 16 % (hidden / 512)) return false;  // column chunks split the 16 warps evenly
  const int sms = sm_count();
  if (sms <= 0) return false;
  const bool mx = e.format == FFN_B200_FMT_MXFP4;
  for (int m = 0; m < 3; ++m)
    if (!e.nv[m].w || !e.nv[m].s || !aligned16(e.nv[m].w) || !aligned16(e.nv[m].s)) return false;
  const int nr1 = (int)((inter + sms - 1) / sms), nr2 = (int)((hidden + sms - 1) / sms);
  if (nr1 > dec::kMaxRows || nr2 > dec::kMaxRows) return false;
  const size_t s1 = dec::layout(2, nr1, (int)hidden, (int)seq, mx).total;
  const size_t s2 = dec::layout(1, nr2, (int)inter, (int)seq, mx).total;
  return s1 <= dec::kSmemCap && s2 <= dec::kSmemCap && s1 + s2 <= 200 * 1024;
}

size_t expert_decode_ws_bytes(size_t inter, size_t seq) { return seq * inter * sizeof(float); }

template <int PHASE, bool MX, int TQ>
static int launch_dec(const dec::DecArgs &a, int grid, size_t smem, cudaStream_t st, int kind, const char *name) {
  static bool attr[64] = {false};
  int dev = 0;
  FFN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "expert decode: device index >= 64");
  if (!attr[dev]) {
    FFN_CUDA_TRY(cudaFuncSetAttribute(dec::decode_kernel<PHASE, MX, TQ>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dec::kSmemCap));
    // the largest shared-memory carve-out for both phases, so that a phase-2
    // CTA finds room next to a running phase-1 CTA without a reconfiguration
    FFN_CUDA_TRY(cudaFuncSetAttribute(dec::decode_kernel<PHASE, MX, TQ>,
                                      cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    attr[dev] = true;
  }
  FFN_LAUNCH_PDL(kind, st, name, (dec::decode_kernel<PHASE, MX, TQ>), grid, dec::kThreads, smem, a);
  return 0;
}

template <bool MX>
static int run_decode(const ffn_b200_expert &e, int inter, int hidden, int seq, const float *x, float *out,
                      float w, int accumulate, float *h, cudaStream_t st) {
  const int sms = sm_count();
  dec::Phase p1{}, p2{};
  for (int m = 0; m < 2; ++m) {
    p1.w[m] = e.nv[m].w;
    p1.s[m] = e.nv[m].s;
    p1.gs[m] = e.nv[m].gs;
  }
  p1.rows = inter;
  p1.K = hidden;
  p2.w[0] = e.nv[2].w;
  p2.s[0] = e.nv[2].s;
  p2.gs[0] = e.nv[2].gs;
  p2.rows = hidden;
  p2.K = inter;
  const int g1 = min(sms, inter), g2 = min(sms, hidden);
  dec::DecArgs a{};
  a.p = p1;
  a.T = seq;
  a.x = x;
  a.ld_x = hidden;
  a.h = h;
  a.ld_h = inter;
  const size_t sm1 = dec::layout(2, (inter + g1 - 1) / g1, hidden, seq, MX).total;
  int rc = seq == 1 ? launch_dec<1, MX, 1>(a, g1, sm1, st, FFN_B200_K_GATEUP_NVFP4, "decode_kernel<1>")
                    : launch_dec<1, MX, 2>(a, g1, sm1, st, FFN_B200_K_GATEUP_NVFP4, "decode_kernel<1>");
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
  const size_t sm2 = dec::layout(1, (hidden + g2 - 1) / g2, inter, seq, MX).total;
  return seq == 1 ? launch_dec<2, MX, 1>(b, g2, sm2, st, FFN_B200_K_DOWN_NVFP4, "decode_kernel<2>")
                  : launch_dec<2, MX, 2>(b, g2, sm2, st, FFN_B200_K_DOWN_NVFP4, "decode_kernel<2>");
}

int launch_expert_decode(const ffn_b200_expert &e, size_t inter, size_t hidden, size_t seq, const float *x,
                         float *out, float accum_weight, int accumulate, void *ws, cudaStream_t st) {
  float *h = static_cast<float *>(ws);
  if (!aligned16(ws) || !aligned16(x) || !aligned16(out) || (hidden % 4))
    return fail(FFN_B200_EUNSUP, "expert decode: x, out and ws must be 16-byte aligned");
  return e.format == FFN_B200_FMT_MXFP4
             ? run_decode<true>(e, (int)inter, (int)hidden, (int)seq, x, out, accum_weight, accumulate, h, st)
             : run_decode<false>(e, (int)inter, (int)hidden, (int)seq, x, out, accum_weight, accumulate, h, st);
}

}  // namespace ffn
