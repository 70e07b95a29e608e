// fp4_gemm.cu -- the MoE layer's NVFP4 experts on tcgen05 block-scaled FP4
// MMAs (kind::mxf4nvf4, UE4M3 scales per 16 K values, TMEM accumulators).
//
// Reference arithmetic (crates/flash-core/src/flash1017.rs): the NVFP4
// matvec y[r] = gs * sum_g e4m3(S[r,g]) * sum_k e2m1(W[r,k]) x[k] (:2331-2357)
// and the SwiGLU expert h = min(silu(g), 10) * clamp(u, -10, 10), y = W2 h
// (:7537-7547, batched :8285-8324).  The weights enter the tensor core exactly
// as stored: the E2M1 nibbles are the MMA's A operand and the E4M3 block
// scales its A scale factors (both are NVFP4 by definition; a scale byte with
// the sign bit set, or the E4M3 NaN 0x7F, is not a UE4M3 value and is
// reported through the error word).  No weight is decoded by the SMs.
//
// Activations: an FP4 MMA multiplies FP4 by FP4, so every activation row x is
// written as a sum of four NVFP4 rows, x ~= sum_t 2^E_t q_t, each with its own
// UE4M3 scale per 16 values and its own power-of-two exponent E_t (term t
// quantises what terms 0 .. t-1 left over).  Four terms leave a relative error
// of about 1e-4 on a dot product (three leave ~1e-3), inside the path's 1e-3
// bound.  The terms are four MMA columns of one token, so one MMA per K-step
// and matrix covers all of them; the epilogue adds the columns with their 2^E_t.
//
// Kernels:
//   q4_kernel        rows of f32 -> 4 NVFP4 terms (codes [row][t][K/2], scales
//                    [row][t][K/16], exponents [row][t]); one CTA per row, one
//                    thread per 16-value block.
//   xq_kernel        the layer input's RMSNorm and router split (xprep's
//                    output) and its four terms in one pass.
//   fp4_gemm_kernel  PH 1: h[p][r] = SwiGLU(gate, up) for 128 rows of W1 and W3;
//                    PH 2: y[p][r] for 256 rows of W2 (two 128-row blocks).
// The gemm is persistent (one CTA per SM walks the (chunk, row block) tiles)
// and warp-specialised (256 threads):
//   warps 0, 1  A producers: 128 weight rows each, 256 K values (128 bytes) per
//               stage by cp.async into the 128-byte-swizzled K-major tile, and
//               the rows' 16 scale bytes per stage into a staging area; the
//               copies' completion arrives on the stage's `landed` barrier by
//               itself, so a producer only ever waits for a free slot.
//   warp 2      B producer: the chunk's 4 x tokens activation rows and scales;
//               kLag stages behind, it transposes each landed stage's scales
//               into the scale-factor atoms and hands the stage over (`full`).
//   warp 3      TMEM owner; lane 0 copies the stage's scale atoms to TMEM
//               (tcgen05.cp) and issues the MMAs (M = 128, N = 4 x tokens
//               rounded to 8, K = 64), committing to the stage and
//               accumulator barriers.
//   warps 4-7   epilogue: thread = TMEM lane = output row of the tile.
// A stage is handed over by the B warp after its copies landed and its atoms
// are written (fence.proxy.async, then mbarrier arrive).  All waits are bounded
// (tcgen05.cuh); a wait that runs out sets the error word, the other roles
// see it and drain, and the combine kernel writes NaN outputs.
#include <algorithm>

#include "ffn_internal.h"
#include "gemv_tile.cuh"
#include "tcgen05.cuh"

namespace ffn {
namespace f4 {

constexpr int kThreads = 256;
constexpr int kStages = 4;
#ifndef F4_LAG
#define F4_LAG 2
#endif
constexpr int kLag = F4_LAG;       // stages the B warp's issue runs ahead of its hand-overs
// kLag <= kStages - 2: one stage of slack between the hand-over of stage j and
// the B warp's wait for slot j + kStages (with kLag = kStages - 1 every stage
// waits for the MMA commit round trip)
static_assert(kLag <= kStages - 2, "the B warp hands a stage over one stage before it needs the slot again");
constexpr int kTileM = 128;
constexpr int kKC = 256;           // K values per stage (128 bytes of a row)
constexpr int kTerms = 4;
constexpr int kNTok = 8;           // tokens per chunk
constexpr int kNMax = kTerms * kNTok;  // MMA columns per chunk (32)

// one pipeline stage in shared memory
constexpr int OFF_A = 0;                        // 2 blocks x 128 rows x 128 B, swizzled
constexpr int OFF_B = 2 * kTileM * 128;         // kNMax rows x 128 B, swizzled
constexpr int OFF_SAS = OFF_B + kNMax * 128;    // A scale staging: 2 x 128 rows x 16 B
constexpr int OFF_SAA = OFF_SAS + 2 * kTileM * 16;  // A scale atoms: 2 blocks x 4 K-steps x 512 B
constexpr int OFF_SBS = OFF_SAA + 2 * 4 * 512;  // B scale staging: kNMax rows x 16 B
constexpr int OFF_SBA = OFF_SBS + kNMax * 16;   // B scale atoms: 4 K-steps x 512 B
constexpr int STAGE = ((OFF_SBA + 4 * 512) + 1023) / 1024 * 1024;
constexpr int SMEM = 1024 + kStages * STAGE;
static_assert(OFF_B % 1024 == 0 && STAGE % 1024 == 0, "swizzled tiles need 1024-byte alignment");
static_assert(SMEM + 1024 <= 227 * 1024, "shared memory");

// TMEM: two accumulator buffers of 2 blocks x kNMax f32 columns, then two
// scale-factor slots (SFA: 2 blocks x 4 K-steps x 4 columns; SFB: 4 x 4)
constexpr int kAccCols = 2 * kNMax;
constexpr int kSfCols = 2 * 16 + 16;
constexpr int kSf0 = 2 * kAccCols;
constexpr int kTmemCols = 256;
static_assert(kSf0 + 2 * kSfCols <= kTmemCols, "TMEM");

// A chunk = the grouping kernel's slice of one expert's routed pairs
// (VExp: expert, first pair, count <= 8).
using Chunk = VExp;
static_assert(kNTok == ::ffn::kNTok, "a slice holds at most kNTok pairs");

struct GemmArgs {
  const ffn_b200_expert *experts;
  const Chunk *chunks;
  const int *n_chunks;
  int K;                    // reduction length
  int rows;                 // output rows
  const uint8_t *qc;        // activation terms: codes [row][4][K/2]
  const uint8_t *qs;        //                   scales [row][4][K/16]
  const int *qe;            //                   exponents [row][4]
  const int32_t *pair_tok;  // phase 1: activation row of pair p; phase 2: nullptr (row = pair)
  float *out;               // phase 1: h [pair][rows]; phase 2: y [pair][rows]
  int ld_out;
  int *err;                 // 1 timed-out wait, 2 scale byte outside UE4M3, 3 misaligned weights
};

__device__ __forceinline__ float silu10(float g) { return fminf(g / (1.0f + expf(-g)), 10.0f); }
__device__ __forceinline__ float clamp10(float u) {  // Rust f32::clamp(-10, 10): NaN stays NaN
  if (u < -10.f) u = -10.f;
  if (u > 10.f) u = 10.f;
  return u;
}

template <int PH>
__global__ void __launch_bounds__(kThreads, 1) fp4_gemm_kernel(const GemmArgs a) {
  pdl_enter();
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t landed[kStages], full[kStages], empty[kStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t s_tmem;
  uint8_t *smem = smem_raw + ((1024 - (tc::sa(smem_raw) & 1023)) & 1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int ROWS = PH == 1 ? kTileM : 2 * kTileM;  // output rows per tile

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::bar_init(&landed[s], 96);  // every A and B producer lane's copies (noinc arrivals)
      tc::bar_init(&full[s], 1);     // the hand-over by the B warp
      tc::bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&acc_full[b], 1);
      tc::bar_init(&acc_empty[b], 4);
    }
    tc::bar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 3) tc::alloc(&s_tmem, kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = s_tmem;

  const int rb_count = a.rows / ROWS;
  const int n_tiles = *a.n_chunks * rb_count;
  const int KT = a.K / kKC;
  const size_t wld = (size_t)a.K / 2, sld = (size_t)a.K / 16;

  if (warp < 2) {
    // ------------------------------------------------------ A producers
    // Issue a stage's copies and move on: the copies' completion arrives on
    // landed[s] by itself (cp.async.mbarrier.arrive.noinc), so a producer waits
    // only for free slots and every free stage can be in flight.
    const int mi = warp;
    int it = 0;
    bool live = true;
    for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x) {
      const Chunk ch = a.chunks[tile / rb_count];
      const int row0 = (tile % rb_count) * ROWS + (PH == 2 ? mi * kTileM : 0);
      const ffn_b200_nvfp4_mat &M = a.experts[ch.expert].nv[PH == 1 ? mi : 2];
      const uint8_t *wb = M.w + (size_t)row0 * wld;
      const uint8_t *sb = M.s + (size_t)row0 * sld;
      const bool s16 = (reinterpret_cast<uintptr_t>(sb) & 15) == 0;
      if ((reinterpret_cast<uintptr_t>(wb) & 15) || (reinterpret_cast<uintptr_t>(sb) & 3)) {
        atomicExch(a.err, 3);
        live = false;
        break;
      }
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % kStages;
        if (!__all_sync(0xffffffffu, tc::bar_wait(&empty[s], ((it / kStages) & 1) ^ 1, a.err))) {
          live = false;
          break;
        }
        uint8_t *st = smem + s * STAGE;
        uint8_t *ta = st + OFF_A + mi * (kTileM * 128);
        // 8 lanes per row, 16 bytes each: one instruction copies 4 whole rows
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
          const int rr = 4 * j + (lane >> 3), pc = lane & 7;
          cp_async16(ta + tc::sw128(rr, pc), wb + (size_t)rr * wld + (size_t)kt * 128 + pc * 16);
        }
        uint8_t *stg = st + OFF_SAS + mi * (kTileM * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int rr = lane + 32 * q;
          const uint8_t *src = sb + (size_t)rr * sld + (size_t)kt * 16;
          if (s16) {
            cp_async16(stg + rr * 16, src);
          } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) cp_async4(stg + rr * 16 + 4 * u, src + 4 * u);
          }
        }
        tc::cp_async_arrive(&landed[s]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------ B producer + hand-over
    // Issues the chunk's activation rows; kLag stages behind, once a stage's
    // copies have all landed, transposes its A and B scales into the
    // scale-factor atoms, fences the async proxy and hands the stage over.
    int it = 0;
    bool live = true;
    auto finish = [&](int j) -> bool {
      const int sj = j % kStages;
      if (!__all_sync(0xffffffffu, tc::bar_wait(&landed[sj], (j / kStages) & 1, a.err))) return false;
      uint8_t *st = smem + sj * STAGE;
      // a byte with the sign bit set or 0x7F is not a UE4M3 scale: flag the
      // layer (NaN outputs) and hand the tensor core a zero scale instead
      uint32_t bad = 0;
      auto clean = [&](uint32_t w) {
        const uint32_t off = (w & 0x80808080u) | __vcmpeq4(w & 0x7F7F7F7Fu, 0x7F7F7F7Fu);
        bad |= off;
        const uint32_t sel = ((off >> 7) & 0x01010101u) * 0xFFu;  // bytes to clear
        return w & ~sel;
      };
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const uint8_t *stg = st + OFF_SAS + mi * (kTileM * 16);
        uint4 r[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) r[q] = *reinterpret_cast<const uint4 *>(stg + (lane + 32 * q) * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) r[q] = make_uint4(clean(r[q].x), clean(r[q].y), clean(r[q].z), clean(r[q].w));
        uint8_t *atoms = st + OFF_SAA + mi * 2048;
        *reinterpret_cast<uint4 *>(atoms + 0 * 512 + lane * 16) = make_uint4(r[0].x, r[1].x, r[2].x, r[3].x);
        *reinterpret_cast<uint4 *>(atoms + 1 * 512 + lane * 16) = make_uint4(r[0].y, r[1].y, r[2].y, r[3].y);
        *reinterpret_cast<uint4 *>(atoms + 2 * 512 + lane * 16) = make_uint4(r[0].z, r[1].z, r[2].z, r[3].z);
        *reinterpret_cast<uint4 *>(atoms + 3 * 512 + lane * 16) = make_uint4(r[0].w, r[1].w, r[2].w, r[3].w);
      }
      if (bad) atomicExch(a.err, 2);
      const uint4 r = *reinterpret_cast<const uint4 *>(st + OFF_SBS + lane * 16);  // row = lane (kNMax = 32)
      uint8_t *atoms = st + OFF_SBA;
      *reinterpret_cast<uint4 *>(atoms + 0 * 512 + lane * 16) = make_uint4(r.x, 0u, 0u, 0u);
      *reinterpret_cast<uint4 *>(atoms + 1 * 512 + lane * 16) = make_uint4(r.y, 0u, 0u, 0u);
      *reinterpret_cast<uint4 *>(atoms + 2 * 512 + lane * 16) = make_uint4(r.z, 0u, 0u, 0u);
      *reinterpret_cast<uint4 *>(atoms + 3 * 512 + lane * 16) = make_uint4(r.w, 0u, 0u, 0u);
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) tc::bar_arrive(&full[sj]);
      return true;
    };
    static_assert(kNMax == 32, "one B row per lane");
    const size_t cld = (size_t)a.K / 2, qsld = (size_t)a.K / 16;
    for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x) {
      const Chunk ch = a.chunks[tile / rb_count];
      // this lane's B row n = lane: token i = n / 4, term t = n % 4
      const int i = lane >> 2, t = lane & 3;
      const bool have = i < ch.count;
      const uint8_t *cb = nullptr, *sbp = nullptr;
      if (have) {
        const int xr = a.pair_tok ? __ldg(a.pair_tok + ch.offset + i) : ch.offset + i;
        cb = a.qc + ((size_t)xr * kTerms + t) * cld;
        sbp = a.qs + ((size_t)xr * kTerms + t) * qsld;
      }
      const int nrows = kTerms * ch.count;
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % kStages;
        if (!__all_sync(0xffffffffu, tc::bar_wait(&empty[s], ((it / kStages) & 1) ^ 1, a.err))) {
          live = false;
          break;
        }
        uint8_t *st = smem + s * STAGE;
#pragma unroll
        for (int j = 0; j < kNMax / 4; ++j) {
          const int n = 4 * j + (lane >> 3), pc = lane & 7;
          const uint8_t *rowp = reinterpret_cast<const uint8_t *>(
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(cb), n));
          if (n < nrows) cp_async16(st + OFF_B + tc::sw128(n, pc), rowp + (size_t)kt * 128 + pc * 16);
        }
        if (have) cp_async16(st + OFF_SBS + lane * 16, sbp + (size_t)kt * 16);
        else *reinterpret_cast<uint4 *>(st + OFF_SBS + lane * 16) = make_uint4(0u, 0u, 0u, 0u);
        tc::cp_async_arrive(&landed[s]);
        if (it >= kLag && !finish(it - kLag)) {
          live = false;
          break;
        }
      }
    }
    if (live)
      for (int j = max(0, it - kLag); j < it; ++j)
        if (!finish(j)) break;
  } else if (warp == 3) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, tcount = 0;
      bool live = true;
      for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x, ++tcount) {
        const Chunk ch = a.chunks[tile / rb_count];
        const int N = (kTerms * ch.count + 7) & ~7;
        const uint32_t id = tc::idesc_nvf4(kTileM, N);
        const int b = tcount & 1, use = tcount >> 1;
        if (!tc::bar_wait(&acc_empty[b], (use & 1) ^ 1, a.err)) break;
        tc::fence_after();
        const uint32_t acc = tmem + b * kAccCols;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % kStages;
          if (!tc::bar_wait(&full[s], (it / kStages) & 1, a.err)) { live = false; break; }
          tc::fence_async_smem();  // the producers' cp.async data, for the tensor core's reads
          tc::fence_after();
          const uint8_t *st = smem + s * STAGE;
          const uint32_t sf = tmem + kSf0 + (it & 1) * kSfCols;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            tc::cp_sf(sf + 4 * k, tc::desc_sf(tc::sa(st + OFF_SAA + k * 512)));
            tc::cp_sf(sf + 16 + 4 * k, tc::desc_sf(tc::sa(st + OFF_SAA + 2048 + k * 512)));
            tc::cp_sf(sf + 32 + 4 * k, tc::desc_sf(tc::sa(st + OFF_SBA + k * 512)));
          }
          const uint32_t ab = tc::sa(st + OFF_A), bb = tc::sa(st + OFF_B);
#pragma unroll
          for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
              tc::mma_nvf4(acc + mi * kNMax, tc::desc_sw128(ab + mi * (kTileM * 128) + 32 * k),
                           tc::desc_sw128(bb + 32 * k), id, sf + 16 * mi + 4 * k, sf + 32 + 4 * k,
                           (kt > 0 || k > 0) ? 1u : 0u);
          tc::commit(&empty[s]);
        }
        if (!live) break;
        tc::commit(&acc_full[b]);
      }
      // every MMA issued here has completed before TMEM is released (issued
      // MMAs always complete, so this wait does not give up on the error word)
      tc::commit(&mma_done);
      tc::bar_wait_drain(&mma_done, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------ epilogue (warps 4-7)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int tcount = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++tcount) {
      const Chunk ch = a.chunks[tile / rb_count];
      const int row0 = (tile % rb_count) * ROWS;
      const int b = tcount & 1, use = tcount >> 1;
      // lane n: 2^E of MMA column n = (token n / 4, term n % 4); 0 when absent
      float csl = 0.f;
      {
        const int i = lane >> 2, t = lane & 3;
        if (i < ch.count) {
          const int xr = a.pair_tok ? __ldg(a.pair_tok + ch.offset + i) : ch.offset + i;
          csl = pow2f(__ldg(a.qe + (size_t)xr * kTerms + t));
        }
      }
      if (!__all_sync(0xffffffffu, tc::bar_wait(&acc_full[b], use & 1, a.err))) break;
      tc::fence_after();
      uint32_t v0[32], v1[32];
      const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + b * kAccCols;
      tc::ld32(tl, v0);
      tc::ld32(tl + kNMax, v1);
      tc::wait_ld();
      const ffn_b200_expert &E = a.experts[ch.expert];
      const float gs0 = E.nv[PH == 1 ? 0 : 2].gs, gs1 = E.nv[PH == 1 ? 1 : 2].gs;
      const int r = 32 * q + lane;
#pragma unroll
      for (int i = 0; i < kNTok; ++i) {
        if (i >= ch.count) break;
        float d0 = 0.f, d1 = 0.f;
#pragma unroll
        for (int t = kTerms - 1; t >= 0; --t) {  // smallest term first
          const float c = __shfl_sync(0xffffffffu, csl, kTerms * i + t);
          d0 += __uint_as_float(v0[kTerms * i + t]) * c;
          d1 += __uint_as_float(v1[kTerms * i + t]) * c;
        }
        float *o = a.out + (size_t)(ch.offset + i) * a.ld_out + row0 + r;
        if (PH == 1) {
          *o = silu10(d0 * gs0) * clamp10(d1 * gs1);
        } else {
          o[0] = d0 * gs0;
          o[kTileM] = d1 * gs1;
        }
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc::bar_arrive(&acc_empty[b]);
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  tc::fence_before();
  __syncthreads();
  if (warp == 3) {
    tc::fence_after();
    tc::dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- quantiser

// Smallest UE4M3 code whose value is >= s (s >= 0), at most 448 (0x7E).
__device__ __forceinline__ uint32_t ue4m3_ceil(float s) {
  if (!(s > 0.f)) return 0u;
  const uint32_t bits = __float_as_uint(s);
  int e = (int)(bits >> 23) - 127;
  if (e >= -6) {
    uint32_t mq = ((bits & 0x7FFFFFu) + 0xFFFFFu) >> 20;  // mantissa rounded up to 3 bits
    if (mq == 8u) { mq = 0u; ++e; }
    if (e > 8) return 0x7Eu;
    const uint32_t c = ((uint32_t)(e + 7) << 3) | mq;
    return c > 0x7Eu ? 0x7Eu : c;
  }
  return (uint32_t)ceilf(s * 512.0f);  // subnormal: units of 2^-9 (8 -> 0x08 = 2^-6)
}
__device__ __forceinline__ float ue4m3_value(uint32_t c) {
  const uint32_t e = c >> 3, m = c & 7u;
  return e == 0u ? (float)m * (1.0f / 512.0f) : (float)(8u + m) * pow2f((int)e - 10);
}
// eight values -> one word of E2M1 codes (round to nearest even, saturated to
// +-6); value 2j in the low nibble of byte j (the NVFP4 packing)
__device__ __forceinline__ uint32_t e2m1x8(const float *f) {
  uint32_t r;
  asm("{ .reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3}; }"
      : "=r"(r)
      : "f"(f[0]), "f"(f[1]), "f"(f[2]), "f"(f[3]), "f"(f[4]), "f"(f[5]), "f"(f[6]), "f"(f[7]));
  return r;
}

// value of an E2M1 code: magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6, bit 3 = sign
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t m = c & 7u;
  const float a = m < 4u ? 0.5f * (float)m : (m == 7u ? 6.0f : (float)(m - 2u));
  return (c & 8u) ? -a : a;
}

// Quantise one 16-value block v of the remainder for term scale 2^e (inv =
// 2^-e, sc = 2^e): block scale = UE4M3 ceiling of max|v| 2^-e / 6, codes =
// E2M1(v 2^-e * (1/s)) with the correctly rounded reciprocal; v becomes the
// new remainder v - 2^e s q.  Writes the 8 code bytes and returns the scale.
__device__ __forceinline__ uint32_t quant_block(float (&v)[16], float inv, float sc, uint2 &codes) {
  float bm = 0.f;
#pragma unroll
  for (int u = 0; u < 16; ++u) bm = fmaxf(bm, fabsf(v[u]));
  const uint32_t code = ue4m3_ceil(__fdiv_rn(bm * inv, 6.0f));
  codes = make_uint2(0u, 0u);
  if (!code) return 0u;
  const float sv = ue4m3_value(code), rcp = __frcp_rn(sv);
  float qv[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) qv[u] = __fmul_rn(__fmul_rn(v[u], inv), rcp);
  codes.x = e2m1x8(qv);
  codes.y = e2m1x8(qv + 8);
  // remainder: the codes' values (exact, from the code words' nibbles) times s 2^e
  const float ss = sv * sc;
#pragma unroll
  for (int u = 0; u < 16; ++u) v[u] -= e2m1_value(((u < 8 ? codes.x : codes.y) >> (4 * (u & 7))) & 15u) * ss;
  return code;
}

// Term exponent from the remainder's max: E = floor(log2 m) - 8 (the largest
// block scale stays below 512/6), 0 for a zero remainder.
__device__ __forceinline__ int term_exp(float m) {
  if (!(m > 0.f) || !isfinite(m)) return 0;
  int ex;
  frexpf(m, &ex);  // m = f 2^ex, f in [0.5, 1)
  return max(-110, min(110, ex - 1 - 8));
}

// The four terms of one row, thread = 16-value block `threadIdx.x` holding
// v (its values; the remainder afterwards).  Term t: one CTA-wide maximum
// (warp shuffles, then the warps' maxima through red[t & 1]), the exponent,
// and one block quantisation per thread.  Every thread of the CTA calls it.
__device__ __forceinline__ void q4_terms(float (&v)[16], bool mine, int row, int K, float (*red)[32],
                                         uint8_t *qc, uint8_t *qs, int *qe) {
  const int blk = threadIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (int)(blockDim.x >> 5);
#pragma unroll 1
  for (int t = 0; t < kTerms; ++t) {
    float am = 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u) am = fmaxf(am, fabsf(v[u]));
    for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if (lane == 0) red[t & 1][wid] = am;
    __syncthreads();  // (the other buffer was last read before the previous term's barrier)
    float m = lane < nw ? red[t & 1][lane] : 0.f;
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int e = term_exp(m);
    if (threadIdx.x == 0) qe[(size_t)row * kTerms + t] = e;
    if (mine) {
      uint2 cw;
      const uint32_t code = quant_block(v, pow2f(-e), pow2f(e), cw);
      *reinterpret_cast<uint2 *>(qc + ((size_t)row * kTerms + t) * (K / 2) + 8 * blk) = cw;
      qs[((size_t)row * kTerms + t) * (K / 16) + blk] = (uint8_t)code;
    }
  }
}

// x row (f32, K values) -> 4 NVFP4 terms.  Term t: E_t = floor(log2 max|r_t|)
// - 8 over the row's remainder r_t, then every 16-value block quantised by
// quant_block.  A zero remainder gives E_t = 0 and zero codes.
// One CTA per row and one thread per 16-value block (blockDim = K / 16 rounded
// up to a warp): each term costs one CTA-wide maximum (warp shuffles, then
// the warps' maxima through shared memory) and one block quantisation per
// thread, so a row's four terms are four short dependent steps.
__global__ void __launch_bounds__(1024) q4_kernel(const float *__restrict__ x, int ld_x, int K,
                                                  uint8_t *qc, uint8_t *qs, int *qe) {
  pdl_enter();
  const int row = blockIdx.x, blk = threadIdx.x;
  const bool mine = blk < K / 16;
  __shared__ float red[2][32];  // warps' maxima, double-buffered by term parity
  float v[16];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float4 f = mine ? __ldg(reinterpret_cast<const float4 *>(x + (size_t)row * ld_x + 16 * blk) + u)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    v[4 * u] = f.x; v[4 * u + 1] = f.y; v[4 * u + 2] = f.z; v[4 * u + 3] = f.w;
  }
  q4_terms(v, mine, row, K, red, qc, qs, qe);
}

// The layer input's preparation and its quantisation in one pass (the FP4
// path's first kernel): per row, the optional RMSNorm (flash1017.rs:4880-4891;
// with seq_norm the sum of squares in column order, as xprep does), xn to
// global only when asked (the exact router reads it), the tensor router's hi/lo
// f16 split of xn 2^-e (e = floor(log2 max|xn|) - 15, xprep's rule), then the
// four NVFP4 terms of xn exactly as q4_kernel forms them.  One CTA per row, one
// thread per 16-value block; the norm weights are read before the wait on the
// previous kernel.
__global__ void __launch_bounds__(1024) xq_kernel(const float *__restrict__ x, int ld_x, int K,
                                                  __half *nh, __half *nl, int ld_o, int *xe,
                                                  const float *__restrict__ norm_w, float norm_eps,
                                                  int seq_norm, float *xn, uint8_t *qc, uint8_t *qs,
                                                  int *qe) {
  const int row = blockIdx.x, blk = threadIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nb = K / 16, nw = (int)(blockDim.x >> 5);
  const bool mine = blk < nb;
  __shared__ float red[2][32];  // term maxima, double-buffered by term parity
  __shared__ float red_a[32];   // sum of squares, then the split's maximum
  __shared__ float s_inv;
  float wv[16];
  if (norm_w) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float4 f = mine ? __ldg(reinterpret_cast<const float4 *>(norm_w + 16 * blk) + u)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      wv[4 * u] = f.x; wv[4 * u + 1] = f.y; wv[4 * u + 2] = f.z; wv[4 * u + 3] = f.w;
    }
  }
  pdl_enter();
  const float *xr = x + (size_t)row * ld_x;
  float v[16];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float4 f = mine ? __ldg(reinterpret_cast<const float4 *>(xr + 16 * blk) + u)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    v[4 * u] = f.x; v[4 * u + 1] = f.y; v[4 * u + 2] = f.z; v[4 * u + 3] = f.w;
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
      for (int u = 0; u < 16; ++u) ss = fmaf(v[u], v[u], ss);
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) red_a[wid] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < nw; ++w) t += red_a[w];
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), norm_eps)));
      }
    }
    __syncthreads();
    const float inv = s_inv;
#pragma unroll
    for (int u = 0; u < 16; ++u) v[u] = __fmul_rn(__fmul_rn(v[u], inv), wv[u]);
    if (xn && mine) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        reinterpret_cast<float4 *>(xn + (size_t)row * K + 16 * blk)[u] =
            make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
    }
  }
  // the tensor router's f16 hi/lo split
  {
    float am = 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u) am = fmaxf(am, fabsf(v[u]));
    for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    __syncthreads();  // (red_a's sums were read before the barrier above)
    if (lane == 0) red_a[wid] = am;
    __syncthreads();
    float m = lane < nw ? red_a[lane] : 0.f;
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int e = 0;
    if (m > 0.f && isfinite(m)) {
      int ex;
      frexpf(m, &ex);  // m = f 2^ex, f in [0.5, 1)
      e = max(-100, min(100, ex - 15));
    }
    if (threadIdx.x == 0) xe[row] = e;
    if (mine) {
      const float sc = pow2f(-e);
      uint32_t wh[8], wl[8];  // f16 pairs, even column in the low half
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        __half h0, l0, h1, l1;
        split_f16(v[2 * u] * sc, h0, l0);
        split_f16(v[2 * u + 1] * sc, h1, l1);
        wh[u] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        wl[u] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
      }
      uint4 *dh = reinterpret_cast<uint4 *>(nh + (size_t)row * ld_o + 16 * blk);
      uint4 *dl = reinterpret_cast<uint4 *>(nl + (size_t)row * ld_o + 16 * blk);
      dh[0] = make_uint4(wh[0], wh[1], wh[2], wh[3]);
      dh[1] = make_uint4(wh[4], wh[5], wh[6], wh[7]);
      dl[0] = make_uint4(wl[0], wl[1], wl[2], wl[3]);
      dl[1] = make_uint4(wl[4], wl[5], wl[6], wl[7]);
    }
  }
  q4_terms(v, mine, row, K, red, qc, qs, qe);  // the four NVFP4 terms, as q4_kernel forms them
}

}  // namespace f4

int launch_xprep_q4(const float *x, int ld_x, int rows, int K, __half *nh, __half *nl, int ld_o, int *xe,
                    const float *norm_w, float norm_eps, int seq_norm, float *xn, uint8_t *qc,
                    uint8_t *qs, int *qe, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (K % 256 || K > 16384 || ld_x % 4 || ld_o % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(norm_w) & 15) || (reinterpret_cast<uintptr_t>(xn) & 15) ||
      ((reinterpret_cast<uintptr_t>(nh) | reinterpret_cast<uintptr_t>(nl)) & 15))
    return fail(FFN_B200_EUNSUP, "xprep_q4: K must be a multiple of 256 up to 16384, rows 16-byte aligned");
  const int threads = (K / 16 + 31) / 32 * 32;
  FFN_LAUNCH_PDL(FFN_B200_K_XPREP, st, "xq_kernel", f4::xq_kernel, rows, threads, 0, x, ld_x, K, nh, nl, ld_o, xe,
                 norm_w, norm_eps, seq_norm, xn, qc, qs, qe);
  return 0;
}

int launch_q4(const float *x, int ld_x, int rows, int K, uint8_t *qc, uint8_t *qs, int *qe, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (K % 256 || K > 16384 || ld_x % 4 || (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(FFN_B200_EUNSUP, "q4: K must be a multiple of 256 up to 16384, rows 16-byte aligned");
  const int threads = (K / 16 + 31) / 32 * 32;  // one thread per 16-value block
  FFN_LAUNCH_PDL(FFN_B200_K_QUANT, st, "q4_kernel", f4::q4_kernel, rows, threads, 0, x, ld_x, K, qc, qs, qe);
  return 0;
}

int launch_fp4_moe(const Fp4Args &g, cudaStream_t st) {
  using namespace f4;
  int dev = 0;
  FFN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "fp4_moe: device index >= 64");
  static bool attr[64] = {false};
  if (!attr[dev]) {
    FFN_CUDA_TRY(cudaFuncSetAttribute(fp4_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    FFN_CUDA_TRY(cudaFuncSetAttribute(fp4_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr[dev] = true;
  }
  const int H = g.hidden, I = g.inter, T = g.n_tok, P = g.n_pairs;
  const int e_loc = g.e_end - g.e_begin;
  const Chunk *chunks = g.slices;
  const int *n_chunks = g.n_slices;
  FFN_CUDA_TRY(cudaMemsetAsync(g.err, 0, sizeof(int), st));
  int rc = 0;
  if (g.x && (rc = launch_q4(g.x, H, T, H, g.xq, g.xs, g.xqe, st))) return rc;  // else quantised already
  const int sms = sm_count_of(dev);
  const long long max_chunks = (long long)P / f4::kNTok + e_loc;
  GemmArgs p{};
  p.experts = g.experts;
  p.chunks = chunks;
  p.n_chunks = n_chunks;
  p.K = H;
  p.rows = I;
  p.qc = g.xq;
  p.qs = g.xs;
  p.qe = g.xqe;
  p.pair_tok = g.pair_tok;
  p.out = g.h;
  p.ld_out = I;
  p.err = g.err;
  int grid = (int)std::max(1LL, std::min<long long>(sms, max_chunks * (I / kTileM)));
  FFN_LAUNCH_PDL(FFN_B200_K_FP4_GATEUP, st, "fp4_gemm_kernel<1>", (fp4_gemm_kernel<1>), grid, f4::kThreads, SMEM, p);
  if ((rc = launch_q4(g.h, I, P, I, g.hq, g.hs, g.hqe, st))) return rc;
  GemmArgs q = p;
  q.K = I;
  q.rows = H;
  q.qc = g.hq;
  q.qs = g.hs;
  q.qe = g.hqe;
  q.pair_tok = nullptr;
  q.out = g.y;
  q.ld_out = H;
  grid = (int)std::max(1LL, std::min<long long>(sms, max_chunks * (H / (2 * kTileM))));
  FFN_LAUNCH_PDL(FFN_B200_K_FP4_DOWN, st, "fp4_gemm_kernel<2>", (fp4_gemm_kernel<2>), grid, f4::kThreads, SMEM, q);
  return 0;
}

}  // namespace ffn

extern "C" {

int ffn_b200_quantize_nvfp4x4(size_t rows, size_t K, const float *x, size_t ld_x, uint8_t *codes,
                              uint8_t *scales, int32_t *exps, void *stream) {
  if (rows == 0) return 0;
  if (!x || !codes || !scales || !exps) return ffn::fail(FFN_B200_EINVAL, "quantize_nvfp4x4: null pointer");
  if (rows > (1u << 24) || ld_x < K || ld_x > (1u << 30))
    return ffn::fail(FFN_B200_EINVAL, "quantize_nvfp4x4: bad rows / ld_x");
  return ffn::launch_q4(x, (int)ld_x, (int)rows, (int)K, codes, scales, exps, (cudaStream_t)stream);
}

}  // extern "C"
