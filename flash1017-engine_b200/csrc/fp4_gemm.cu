// fp4_gemm.cu -- the MoE layer's NVFP4 experts on tcgen05 block-scaled FP4
// MMAs (kind::mxf4nvf4, UE4M3 scales per 16 K values, TMEM accumulators).
//
// Reference arithmetic (crates/flash-core/src/flash1017.rs): the NVFP4
// matvec y[r] = gs * sum_g e4m3(S[r,g]) * sum_k e2m1(W[r,k]) x[k] (:2331-2357)
// and the SwiGLU expert h = min(silu(g), 10) * clamp(u, -10, 10), y = W2 h
// (:7537-7547, batched :8285-8324).  The weights enter the tensor core exactly
// as stored: the E2M1 nibbles are the MMA's A operand and the E4M3 block
// scales its A scale factors (both are NVFP4 by definition; a scale byte with
// the sign bit set, or the E4M3 NaN 0x7F, is not a UE4M3 value and such an
// expert cannot be packed).  No weight is decoded by the SMs.
//
// Packed weights (ffn_b200_pack_nvfp4_expert): the kernel's pipeline stage is
// two 128-row blocks x 256 K values -- the W1 and W3 rows of an output block
// in phase 1, the two halves of a 256-row W2 block in phase 2 -- and packing
// stores every stage's bytes as the image the stage has in shared memory: the
// two blocks' codes as 128-byte-swizzled K-major tiles (16 KB each), then
// their scale-factor atoms (4 K-steps x 512 B each), 36 KB per stage, stages
// ordered (row block, K step).  One non-multicast bulk copy brings a stage in,
// and DRAM streams 36 KB contiguous pieces (the reference layout would be read
// as 128-byte pieces of rows 2 KB apart, which HBM serves markedly slower).
//
// Activations: an FP4 MMA multiplies FP4 by FP4, so every activation row x is
// written as a sum of kTerms NVFP4 rows, x ~= sum_t 2^E_t q_t, each with its own
// UE4M3 scale per 16 values and its own power-of-two exponent E_t (term t
// quantises what terms 0 .. t-1 left over; each term gains about 2.6 bits).
// Six terms keep a 40-layer stack inside the path's 1e-3 bound (four leave
// ~2.6e-4 per layer, which compounds through the stack).  The terms are
// MMA columns of one token, so one MMA per K-step and block covers all of
// them; the epilogue adds the columns with their 2^E_t.
//
// Kernels:
//   q4_kernel        rows of f32 -> NVFP4 terms (codes [row][t][K/2], scales
//                    [row][t][K/16], exponents [row][t]); one CTA per row, one
//                    thread per 16-value block.
//   xq_kernel        the layer input's RMSNorm and router split (xprep's
//                    output) and its terms in one pass.
//   pack_kernel      reference-layout NVFP4 matrices -> stage images.
//   fp4_gemm_kernel  PH 1: h[p][r] = SwiGLU(gate, up) for 128 rows of W1 and W3;
//                    PH 2: y[p][r] for 256 rows of W2 (two 128-row blocks).
// The gemm is persistent (one CTA per SM walks the (chunk, row block) tiles)
// and warp-specialised (256 threads):
//   warp 0      producer: lane 0 waits for a free slot and issues the stage's
//               bulk copy (36 KB, completing on a_full).
//   warp 1      activations: the chunk's kTerms x tokens rows for the stage's
//               K range, and their scales straight into the scale-factor
//               atoms (row n at line n % 32, word n / 32), all by cp.async
//               arriving on b_full when landed: this warp never waits for
//               data.
//   warp 2      TMEM owner; lane 0 copies the stage's atoms to TMEM
//               (tcgen05.cp) and issues the MMAs (M = 128, N = kTerms x tokens
//               rounded to 8, K = 64), committing to the stage and
//               accumulator barriers.
//   warps 4-7   epilogue: thread = TMEM lane = output row of the tile.
// All waits are bounded (tcgen05.cuh); a wait that runs out sets the error
// word, the other roles see it and drain, and the combine kernel writes NaN
// outputs.
#include <algorithm>

#include "ffn_internal.h"
#include "gemv_tile.cuh"
#include "tcgen05.cuh"

namespace ffn {
namespace f4 {

constexpr int kThreads = 256;
constexpr int kStages = 5;
constexpr int kTileM = 128;
constexpr int kKC = 256;                  // K values per stage (128 bytes of a row)
constexpr int kTerms = kFp4Terms;         // activation terms the layer uses
constexpr int kMaxTerms = 8;              // the quantiser's limit
constexpr int kNTok = 8;                  // tokens per chunk
constexpr int kNMax = kTerms * kNTok;     // MMA columns per chunk (48)
static_assert(kNMax <= 64, "B rows: one or two per lane");

// one stage in shared memory: the packed image (bulk copy), then the B rows
// and the B scale atoms
constexpr int kImg = 2 * kTileM * 128 + 2 * 4 * 512;  // 36 KB: codes blk 0, blk 1, atoms blk 0, blk 1
constexpr int OFF_A = 0;
constexpr int OFF_SAA = 2 * kTileM * 128;             // A atoms inside the image
constexpr int OFF_B = kImg;                           // kNMax rows x 128 B, swizzled
constexpr int OFF_SBA = OFF_B + ((kNMax * 128 + 1023) / 1024) * 1024;  // 4 K-steps x 512 B
constexpr int STAGE = ((OFF_SBA + 4 * 512) + 1023) / 1024 * 1024;
constexpr int SMEM = 1024 + kStages * STAGE;
static_assert(OFF_B % 1024 == 0 && STAGE % 1024 == 0, "swizzled tiles need 1024-byte alignment");
static_assert(SMEM <= 227 * 1024, "shared memory");

// TMEM: two accumulator buffers of 2 blocks x kNMax f32 columns, then two
// scale-factor slots (SFA: 2 blocks x 4 K-steps x 4 columns; SFB: 4 x 4);
// every accumulator and slot starts on a 64-column boundary
constexpr int kAccStride = 64;            // columns per block accumulator (kNMax used)
constexpr int kAccCols = 2 * kAccStride;
constexpr int kSfCols = 64;               // slot stride (48 used)
constexpr int kSf0 = 2 * kAccCols;
constexpr int kTmemCols = 512;
static_assert(kNMax <= kAccStride && 2 * 16 + 16 <= kSfCols, "TMEM layout");
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
  const uint8_t *qc;        // activation terms: codes [row][kTerms][K/2]
  const uint8_t *qs;        //                   scales [row][kTerms][K/16]
  const int *qe;            //                   exponents [row][kTerms]
  const int32_t *pair_tok;  // phase 1: activation row of pair p; phase 2: nullptr (row = pair)
  float *out;               // phase 1: h [pair][rows]; phase 2: y [pair][rows]
  int ld_out;
  int *err;                 // 1 timed-out wait, 3 expert not packed
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
  __shared__ __align__(8) uint64_t a_full[kStages], b_full[kStages], empty[kStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t s_tmem;
  uint8_t *smem = smem_raw + ((1024 - (tc::sa(smem_raw) & 1023)) & 1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int ROWS = PH == 1 ? kTileM : 2 * kTileM;  // output rows per tile

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::bar_init(&a_full[s], 1);   // the producer's expect_tx; the bulk copy's bytes complete it
      tc::bar_init(&b_full[s], 32);  // the activation warp's lanes' cp.async (noinc arrivals)
      tc::bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&acc_full[b], 1);
      tc::bar_init(&acc_empty[b], 4);
    }
    tc::bar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) tc::alloc(&s_tmem, kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = s_tmem;

  const int rb_count = a.rows / ROWS;
  const int n_tiles = *a.n_chunks * rb_count;
  const int KT = a.K / kKC;

  if (warp == 0) {
    // ------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0, issued = 0;
      bool live = true;
      for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x) {
        const Chunk ch = a.chunks[tile / rb_count];
        const uint8_t *img = PH == 1 ? a.experts[ch.expert].fp4_gu : a.experts[ch.expert].fp4_dn;
        if (!img || (reinterpret_cast<uintptr_t>(img) & 15)) {
          atomicExch(a.err, 3);
          break;
        }
        img += (size_t)(tile % rb_count) * KT * kImg;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % kStages;
          if (!tc::bar_wait(&empty[s], ((it / kStages) & 1) ^ 1, a.err)) { live = false; break; }
          tc::bar_arrive_tx(&a_full[s], (uint32_t)kImg);
          tc::bulk_g2s(smem + s * STAGE + OFF_A, img + (size_t)kt * kImg, (uint32_t)kImg, &a_full[s]);
          issued = it + 1;
        }
      }
      // before leaving, the copies this thread issued have landed (bounded:
      // a copy always completes; this only guards a shared-memory release)
      for (int j = max(0, issued - kStages); j < issued; ++j)
        tc::bar_wait_drain(&a_full[j % kStages], (j / kStages) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------ activations
    // lane l owns B rows l and l + 32 (when < kNMax): token n / kTerms, term n % kTerms
    for (int i = lane; i < kStages * 4 * 32; i += 32)  // B atom words 2-3 (rows 64-127) stay zero
      reinterpret_cast<uint2 *>(smem + (i / 128) * STAGE + OFF_SBA + (i % 128) * 16)[1] = make_uint2(0u, 0u);
    tc::fence_async_smem();  // (the MMA issuer reads them through the async proxy)
    const size_t cld = (size_t)a.K / 2, qsld = (size_t)a.K / 16;
    int it = 0;
    bool live = true;
    for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x) {
      const Chunk ch = a.chunks[tile / rb_count];
      const uint8_t *cb[2] = {nullptr, nullptr}, *sbp[2] = {nullptr, nullptr};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = lane + 32 * h, i = n / kTerms, t = n - i * kTerms;
        if (n < kNMax && i < ch.count) {
          const int xr = a.pair_tok ? __ldg(a.pair_tok + ch.offset + i) : ch.offset + i;
          cb[h] = a.qc + ((size_t)xr * kTerms + t) * cld;
          sbp[h] = a.qs + ((size_t)xr * kTerms + t) * qsld;
        }
      }
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % kStages;
        if (!__all_sync(0xffffffffu, tc::bar_wait(&empty[s], ((it / kStages) & 1) ^ 1, a.err))) {
          live = false;
          break;
        }
        uint8_t *st = smem + s * STAGE;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (cb[h]) {
            const uint8_t *src = cb[h] + (size_t)kt * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) cp_async16(st + OFF_B + tc::sw128(lane + 32 * h, c), src + c * 16);
          }
        // this K range's 16 scale bytes of row n, 4 per K-step, copied straight
        // to word n / 32 of line n % 32 of the 4 atoms (no wait in this warp;
        // the words of absent rows keep stale values, read only into MMA
        // columns the epilogue never reads)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (sbp[h]) {
            const uint8_t *src = sbp[h] + (size_t)kt * 16;
#pragma unroll
            for (int k = 0; k < 4; ++k) cp_async4(st + OFF_SBA + k * 512 + lane * 16 + 4 * h, src + 4 * k);
          }
        tc::cp_async_arrive(&b_full[s]);
      }
    }
  } else if (warp == 2) {
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
          if (!tc::bar_wait(&a_full[s], (it / kStages) & 1, a.err) ||
              !tc::bar_wait(&b_full[s], (it / kStages) & 1, a.err)) {
            live = false;
            break;
          }
          tc::fence_async_smem();  // the activations' cp.async data, for the tensor core's reads
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
              tc::mma_nvf4(acc + mi * kAccStride, tc::desc_sw128(ab + mi * (kTileM * 128) + 32 * k),
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
  } else if (warp >= 4) {
    // ------------------------------------------------------ epilogue (warps 4-7)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int tcount = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++tcount) {
      const Chunk ch = a.chunks[tile / rb_count];
      const int row0 = (tile % rb_count) * ROWS;
      const int b = tcount & 1, use = tcount >> 1;
      // lane l: 2^E of MMA columns l and l + 32 (token n / kTerms, term n % kTerms); 0 when absent
      float csl[2] = {0.f, 0.f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = lane + 32 * h, i = n / kTerms, t = n - i * kTerms;
        if (n < kNMax && i < ch.count) {
          const int xr = a.pair_tok ? __ldg(a.pair_tok + ch.offset + i) : ch.offset + i;
          csl[h] = pow2f(__ldg(a.qe + (size_t)xr * kTerms + t));
        }
      }
      if (!__all_sync(0xffffffffu, tc::bar_wait(&acc_full[b], use & 1, a.err))) break;
      tc::fence_after();
      uint32_t v0[kNMax], v1[kNMax];
      const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + b * kAccCols;
      static_assert(kNMax == 48, "the epilogue reads 32 + 16 columns per block");
      tc::ld32(tl, *reinterpret_cast<uint32_t(*)[32]>(v0));
      tc::ld16(tl + 32, v0 + 32);
      tc::ld32(tl + kAccStride, *reinterpret_cast<uint32_t(*)[32]>(v1));
      tc::ld16(tl + kAccStride + 32, v1 + 32);
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
          const int n = kTerms * i + t;
          const float c = __shfl_sync(0xffffffffu, csl[n >> 5], n & 31);
          d0 += __uint_as_float(v0[n]) * c;
          d1 += __uint_as_float(v1[n]) * c;
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
  if (warp == 2) {
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

// Quantise one 16-value block v of the remainder for term scale 2^e (inv =
// 2^-e, sc = 2^e): block scale = UE4M3 ceiling of max|v| 2^-e / 6, codes =
// E2M1(v 2^-e * (1/s)) with the correctly rounded reciprocal; v becomes the
// new remainder v - 2^e s q.  Writes the 8 code bytes and returns the scale.
// bm = max|v| over the block (the caller has it already).
__device__ __forceinline__ uint32_t quant_block(float (&v)[16], float bm, float inv, float sc, uint2 &codes) {
  const uint32_t code = ue4m3_ceil(__fdiv_rn(bm * inv, 6.0f));
  codes = make_uint2(0u, 0u);
  if (!code) return 0u;
  const float sv = ue4m3_value(code), rcp = __frcp_rn(sv);
  float qv[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) qv[u] = __fmul_rn(__fmul_rn(v[u], inv), rcp);
  codes.x = e2m1x8(qv);
  codes.y = e2m1x8(qv + 8);
  // remainder: the codes' values (exact, from the code words' nibbles) times
  // s 2^e.  (The hardware E2M1 -> f16x2 decode of these freshly converted code
  // words left the remainder unchanged in a test build; the bit decode below
  // is what the bit-exact tests pin.)
  // A code c = (sign, m) placed as f32 bits (sign << 31) | (m << 22) is
  // exactly its E2M1 value times 2^-126 (m = 1 lands on the subnormal 2^-127),
  // so the decode is shifts and masks and one exact multiply by 2^126.
  const float ss = sv * sc;
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const uint32_t w = u < 8 ? codes.x : codes.y;
    const int k = 4 * (u & 7);  // the nibble's first bit
    const uint32_t mag = (k <= 22 ? w << (22 - k) : w >> (k - 22)) & 0x01C00000u;
    const uint32_t sgn = (w << (28 - k)) & 0x80000000u;
    const float a = __uint_as_float(mag | sgn) * 0x1p126f;
    v[u] -= a * ss;
  }
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

// The `terms` terms of one row, thread = 16-value block `threadIdx.x` holding
// v (its values; the remainder afterwards).  Term t: one CTA-wide maximum
// (warp shuffles, then the warps' maxima through red[t & 1]), the exponent,
// and one block quantisation per thread.  Every thread of the CTA calls it.
__device__ __forceinline__ void q4_terms(float (&v)[16], bool mine, int row, int K, int terms, float (*red)[32],
                                         uint8_t *qc, uint8_t *qs, int *qe) {
  const int blk = threadIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (int)(blockDim.x >> 5);
#pragma unroll 1
  for (int t = 0; t < terms; ++t) {
    float bm = 0.f;  // this thread's block maximum
#pragma unroll
    for (int u = 0; u < 16; ++u) bm = fmaxf(bm, fabsf(v[u]));
    float am = bm;
    for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if (lane == 0) red[t & 1][wid] = am;
    __syncthreads();  // (the other buffer was last read before the previous term's barrier)
    float m = lane < nw ? red[t & 1][lane] : 0.f;
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int e = term_exp(m);
    if (threadIdx.x == 0) qe[(size_t)row * terms + t] = e;
    if (mine) {
      uint2 cw;
      const uint32_t code = quant_block(v, bm, pow2f(-e), pow2f(e), cw);
      *reinterpret_cast<uint2 *>(qc + ((size_t)row * terms + t) * (K / 2) + 8 * blk) = cw;
      qs[((size_t)row * terms + t) * (K / 16) + blk] = (uint8_t)code;
    }
  }
}

// x row (f32, K values) -> `terms` NVFP4 terms.  Term t: E_t = floor(log2 max|r_t|)
// - 8 over the row's remainder r_t, then every 16-value block quantised by
// quant_block.  A zero remainder gives E_t = 0 and zero codes.
// One CTA per row and one thread per 16-value block (blockDim = K / 16 rounded
// up to a warp): each term costs one CTA-wide maximum (warp shuffles, then
// the warps' maxima through shared memory) and one block quantisation per
// thread, so a row's terms are short dependent steps.
__global__ void __launch_bounds__(1024) q4_kernel(const float *__restrict__ x, int ld_x, int K, int terms,
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
  q4_terms(v, mine, row, K, terms, red, qc, qs, qe);
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
  q4_terms(v, mine, row, K, kTerms, red, qc, qs, qe);  // the layer's terms, as q4_kernel forms them
}

// Bytes of a scale word that are not UE4M3 (sign bit set, or 0x7F: its low
// seven bits plus one carry into bit 7), as 0x80 in each such byte.
__device__ __forceinline__ uint32_t not_ue4m3(uint32_t w) {
  return (w | ((w & 0x7F7F7F7Fu) + 0x01010101u)) & 0x80808080u;
}

// Reference-layout NVFP4 matrices -> stage images (the layout is described at
// the top of this file).  One CTA per image (row block rb, K step kt): the two
// blocks' codes (2 x 128 rows x 8 pieces of 16 bytes, moved to their swizzled
// places), then the two blocks' scale atoms (2 x 4 K-steps x 32 lines of 16
// bytes: line l = the 4 scale bytes of rows l, l + 32, l + 64, l + 96).  A
// scale byte that is not UE4M3 is counted in *bad.
struct PackArgs {
  const uint8_t *w0, *w1;  // codes of the matrices holding block 0 and block 1
  const uint8_t *s0, *s1;  // their E4M3 scales
  int row_off1;            // block 1's first row, relative to block 0's
  int rows_per_rb;         // rows between consecutive row blocks
  int K, KT;
  uint8_t *out;
  int *bad;
};
__global__ void __launch_bounds__(256) pack_kernel(const PackArgs a) {
  const int img = blockIdx.x, rb = img / a.KT, kt = img - rb * a.KT;
  uint8_t *o = a.out + (size_t)img * kImg;
  const size_t wld = (size_t)a.K / 2, sld = (size_t)a.K / 16;
  for (int p = threadIdx.x; p < 2 * kTileM * 8; p += blockDim.x) {
    const int blk = p / (kTileM * 8), r = (p / 8) % kTileM, c = p % 8;
    const size_t row = (size_t)rb * a.rows_per_rb + (blk ? a.row_off1 : 0) + r;
    const uint4 v = *reinterpret_cast<const uint4 *>((blk ? a.w1 : a.w0) + row * wld + (size_t)kt * 128 + c * 16);
    *reinterpret_cast<uint4 *>(o + blk * (kTileM * 128) + tc::sw128(r, c)) = v;
  }
  for (int p = threadIdx.x; p < 2 * 4 * 32; p += blockDim.x) {
    const int blk = p / 128, k = (p / 32) % 4, l = p % 32;
    uint32_t w[4], off = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const size_t row = (size_t)rb * a.rows_per_rb + (blk ? a.row_off1 : 0) + l + 32 * q;
      w[q] = *reinterpret_cast<const uint32_t *>((blk ? a.s1 : a.s0) + row * sld + (size_t)kt * 16 + 4 * k);
      off |= not_ue4m3(w[q]);
    }
    *reinterpret_cast<uint4 *>(o + OFF_SAA + blk * 2048 + k * 512 + l * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    if (off) atomicAdd(a.bad, 1);
  }
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

int launch_q4(const float *x, int ld_x, int rows, int K, int terms, uint8_t *qc, uint8_t *qs, int *qe,
              cudaStream_t st) {
  if (rows <= 0) return 0;
  if (K % 256 || K > 16384 || ld_x % 4 || (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(FFN_B200_EUNSUP, "q4: K must be a multiple of 256 up to 16384, rows 16-byte aligned");
  if (terms < 1 || terms > f4::kMaxTerms) return fail(FFN_B200_EINVAL, "q4: terms must be 1..8");
  const int threads = (K / 16 + 31) / 32 * 32;  // one thread per 16-value block
  FFN_LAUNCH_PDL(FFN_B200_K_QUANT, st, "q4_kernel", f4::q4_kernel, rows, threads, 0, x, ld_x, K, terms, qc, qs, qe);
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
  if (g.x && (rc = launch_q4(g.x, H, T, H, kTerms, g.xq, g.xs, g.xqe, st))) return rc;  // else quantised already
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
  if ((rc = launch_q4(g.h, I, P, I, kTerms, g.hq, g.hs, g.hqe, st))) return rc;
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

int ffn_b200_quantize_nvfp4_terms(size_t rows, size_t K, size_t terms, const float *x, size_t ld_x,
                                  uint8_t *codes, uint8_t *scales, int32_t *exps, void *stream) {
  if (rows == 0) return 0;
  if (!x || !codes || !scales || !exps) return ffn::fail(FFN_B200_EINVAL, "quantize_nvfp4: null pointer");
  if (rows > (1u << 24) || ld_x < K || ld_x > (1u << 30))
    return ffn::fail(FFN_B200_EINVAL, "quantize_nvfp4: bad rows / ld_x");
  if (terms < 1 || terms > (size_t)ffn::f4::kMaxTerms) return ffn::fail(FFN_B200_EINVAL, "quantize_nvfp4: terms must be 1..8");
  return ffn::launch_q4(x, (int)ld_x, (int)rows, (int)K, (int)terms, codes, scales, exps, (cudaStream_t)stream);
}

size_t ffn_b200_fp4_pack_bytes(size_t inter, size_t hidden, int which) {
  if (inter % 256 || hidden % 256) return 0;
  return which == 0 ? (inter / 128) * (hidden / 256) * (size_t)ffn::f4::kImg
                    : (hidden / 256) * (inter / 256) * (size_t)ffn::f4::kImg;
}

int ffn_b200_pack_nvfp4_expert(size_t inter, size_t hidden, const ffn_b200_expert *e, uint8_t *gu, uint8_t *dn,
                               void *stream) {
  using namespace ffn;
  if (!e) return fail(FFN_B200_EINVAL, "pack_nvfp4_expert: null expert");
  if (e->format != FFN_B200_FMT_NVFP4) return fail(FFN_B200_EINVAL, "pack_nvfp4_expert: not an NVFP4 expert");
  if (inter % 256 || hidden % 256 || inter == 0 || hidden == 0 || inter > 16384 || hidden > 16384)
    return fail(FFN_B200_EUNSUP, "pack_nvfp4_expert: inter and hidden must be multiples of 256 up to 16384");
  for (int m = 0; m < 3; ++m)
    if (!e->nv[m].w || !e->nv[m].s || (reinterpret_cast<uintptr_t>(e->nv[m].w) & 15) ||
        (reinterpret_cast<uintptr_t>(e->nv[m].s) & 3))
      return fail(FFN_B200_EINVAL, "pack_nvfp4_expert: codes must be 16-byte and scales 4-byte aligned");
  if ((reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(dn)) & 15)
    return fail(FFN_B200_EINVAL, "pack_nvfp4_expert: images must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  int dev = 0;
  FFN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "pack_nvfp4_expert: device index >= 64");
  static int *bad_dev[64] = {nullptr};  // one counter per device (packing is a load-time step)
  if (!bad_dev[dev]) FFN_CUDA_TRY(cudaMalloc(&bad_dev[dev], sizeof(int)));
  FFN_CUDA_TRY(cudaMemsetAsync(bad_dev[dev], 0, sizeof(int), st));
  const int H = (int)hidden, I = (int)inter;
  if (gu) {
    f4::PackArgs p{e->nv[0].w, e->nv[1].w, e->nv[0].s, e->nv[1].s, 0, f4::kTileM, H, H / 256, gu, bad_dev[dev]};
    FFN_LAUNCH(FFN_B200_K_OTHER, st, "pack_kernel", (f4::pack_kernel<<<(I / 128) * (H / 256), 256, 0, st>>>(p)));
  }
  if (dn) {
    f4::PackArgs p{e->nv[2].w, e->nv[2].w, e->nv[2].s, e->nv[2].s, f4::kTileM, 2 * f4::kTileM, I, I / 256, dn,
                   bad_dev[dev]};
    FFN_LAUNCH(FFN_B200_K_OTHER, st, "pack_kernel", (f4::pack_kernel<<<(H / 256) * (I / 256), 256, 0, st>>>(p)));
  }
  int bad = 0;
  FFN_CUDA_TRY(cudaMemcpyAsync(&bad, bad_dev[dev], sizeof(int), cudaMemcpyDeviceToHost, st));
  FFN_CUDA_TRY(cudaStreamSynchronize(st));
  if (bad)
    return fail(FFN_B200_EINVAL, "pack_nvfp4_expert: a scale byte is not UE4M3 (sign bit set or 0x7F); "
                                 "the FP4 path cannot take this expert");
  return 0;
}

int ffn_b200_quantize_nvfp4x4(size_t rows, size_t K, const float *x, size_t ld_x, uint8_t *codes,
                              uint8_t *scales, int32_t *exps, void *stream) {
  return ffn_b200_quantize_nvfp4_terms(rows, K, 4, x, ld_x, codes, scales, exps, stream);
}

}  // extern "C"
