// grouped_gemm.cu -- tensor-core (tcgen05) grouped GEMM for many tokens per
// expert: the MoE prefill path (batched tokens of crates/flash-core/src/
// flash1017.rs:8267-8326, the same arithmetic as the decode path).
//
// Per local expert the routed tokens form chunks of <= 192 pairs.  A tile is
// (chunk, block of 128 output rows); one CTA per SM walks the tiles.
//
//   phase 1:  D_g = W1[rows] . X^T, D_u = W3[rows] . X^T  (K = hidden)
//             h[p][row] = f16( min(silu(g), 10) * clamp(u, -10, 10) ),
//             g = D_g * 2^xe[tok] * gs1, u = D_u * 2^xe[tok] * gs3
//   phase 2:  y[p][row] = (W2[rows] . H^T) * gs2                (K = inter)
//             (a tile covers 256 down rows as two 128-row blocks, so each
//             activation tile feeds as many MMAs as in phase 1)
//
// MMA: tcgen05.mma.cta_group::1.kind::f16, M = 128 weight rows, N = chunk
// tokens rounded up to 16, K = 16 per instruction.  A (the decoded weights)
// comes from TMEM, B (the activations) from shared memory as K-major tiles of
// 64 columns in the 128-byte swizzled canonical layout.  TMEM (512 columns):
// one f32 accumulator buffer of 2 x kMaxN columns (phase 1: gate block, then
// up block), then the decoded A stages, 2 x 32 columns each (lane = weight
// row, column c = f16 pair (2c, 2c + 1) of the K-step's 64 values).
//
// Weights: NVFP4 rows are decoded on the fly into f16 (exact: an E2M1 value
// times an E4M3 scale has at most 6 significant bits, inside f16's range), so
// the tensor core sees the reference's dequantised weights.  Activations:
// phase 1 takes x * 2^-xe as one f16 term (bf16 inputs, config 3, are exact
// there); phase 2 takes h rounded to f16.  Relative error of an output about
// 2^-12 (measured ~2e-4), inside the path's 1e-3 tolerance.
//
// Warp roles (384 threads):
//   warps 0, 1, 3  activation producers: cp.async of the chunk's rows straight
//                  into their swizzled B tile, kXStages-deep ring (L2 hits
//                  mostly).  Producer completion is an mbarrier arrive per
//                  lane (noinc).
//   warp 2         TMEM allocation; lane 0 issues the MMAs and commits them to
//                  the ring / accumulator barriers.
//   warps 4-11     stream their own 32 weight rows (NVFP4 + block scales)
//                  through a private kWStages-deep cp.async ring (kWSteps
//                  K-steps per stage), as the decode GEMV engine does, decode
//                  them (thread = row of A block w / 4 - 1) and store the f16
//                  row to TMEM with tcgen05.st; after a tile's last K-step they
//                  run the epilogue from TMEM (warp w reads TMEM lanes
//                  32 (w % 4) ..., warps 4-7 the first half of the tile's
//                  columns, warps 8-11 the second).
// Every mbarrier wait is bounded; a wait that runs out sets *err and the
// kernel drains and returns (the host turns *err into FFN_B200_ECUDA).
#include <algorithm>

#include "ffn_internal.h"
#include "gemv_tile.cuh"

namespace ffn {
namespace gg {

constexpr int kThreadsGG = 384;
constexpr int kDecWarps = 8;   // warps 4-11: decode + epilogue
#ifndef GG_WSTEPS
#define GG_WSTEPS 2
#endif
#ifndef GG_WSTAGES
#define GG_WSTAGES 5
#endif
#ifndef GG_XSTAGES
#define GG_XSTAGES 3
#endif
constexpr int kWSteps = GG_WSTEPS;    // K-steps per weight stage: 32 kWSteps contiguous bytes of each row
constexpr int kWStages = GG_WSTAGES;  // weight stages per decode warp ring (kWStages - 1 in flight)
constexpr int kXStages = GG_XSTAGES;  // activation tiles per K-step (mostly L2 hits)
static_assert(kWSteps == 1 || kWSteps == 2 || kWSteps == 4, "K is a multiple of 256");
constexpr int kTileM = 128;
constexpr int kTileK = 64;
#ifndef GG_MAXN
#define GG_MAXN 192
#endif
constexpr int kMaxN = GG_MAXN;  // tokens per chunk (MMA N)
// decoded f16 weight tiles (2 blocks x 64 K = 64 TMEM columns each) in the
// TMEM columns the accumulators (2 blocks x kMaxN) leave free
constexpr int kAStages = (512 - 2 * kMaxN) / kTileK;
static_assert(kMaxN % 16 == 0 && kAStages >= 2, "TMEM split");
constexpr int kXLanes = 96;    // warps 0, 1, 3: activation producers
constexpr long long kSpinLimit = 1LL << 22;  // try_wait polls per wait before giving up

// A tile = 2 blocks of 128 weight rows sharing one activation tile: gate and
// up rows (phase 1), or 256 consecutive down rows (phase 2).
template <int PH>
struct Layout {
  static constexpr int NMAT = 2;                                  // A blocks per tile
  static constexpr int ROWS = PH == 1 ? kTileM : 2 * kTileM;      // output rows per tile
  static constexpr int X_STAGE = kMaxN * 128;                    // swizzled B tile (1024-aligned)
  static constexpr int W_W = NMAT * kTileM * 32 * kWSteps;       // NVFP4 bytes of a weight stage
  static constexpr int W_S = NMAT * kTileM * 4 * kWSteps;        // scale bytes of a weight stage
  static constexpr int RB = 32 * kWSteps;                        // weight bytes of a row per stage
  static constexpr int SB = 4 * kWSteps;                         // scale bytes of a row per stage
  static constexpr int PPR = RB / 16;                            // 16-byte pieces per row
  // piece swizzle of row r: rows sharing a 128-byte bank window get distinct slots
  static __device__ __forceinline__ int pswz(int r) { return (r / (128 / RB)) % PPR; }
  static constexpr int WSLOT = 32 * (RB + SB);                   // one decode warp's rows, one stage
  static constexpr int W_STAGE = W_W + W_S;
  static_assert(kDecWarps * WSLOT == W_STAGE, "the decode warps' rings fill the W region");
  static constexpr int OFF_W = kXStages * X_STAGE;
  static constexpr int SMEM = 1024 + OFF_W + kWStages * W_STAGE;
  static_assert(SMEM + 2048 <= 227 * 1024, "shared memory");
  // TMEM: one accumulator buffer (NMAT blocks x kMaxN f32 columns), then the
  // decoded A stages (NMAT blocks x 64 f16 = 32 columns each; lane = row)
  static constexpr int ACC_BUFS = 1;
  static constexpr int ACC_COLS = NMAT * kMaxN;
  static constexpr int A_COL0 = ACC_BUFS * ACC_COLS;
  static constexpr int A_COLS = NMAT * kTileK / 2;
  static constexpr int TMEM_COLS = 512;                          // a power of 2
  static_assert(A_COL0 + kAStages * A_COLS <= TMEM_COLS, "TMEM");
};

struct Chunk {
  int32_t expert, p0, nn, npad;
};

struct GemmArgs {
  const ffn_b200_expert *experts;
  const Chunk *chunks;
  const int *n_chunks;
  int K;                  // reduction length (hidden for phase 1, inter for phase 2)
  int rows;               // output rows (inter for phase 1, hidden for phase 2)
  const __half *x;        // phase 1: xh rows by token; phase 2: h rows by pair
  int ld_x;
  const int32_t *pair_tok;
  const int *xe;
  __half *h;              // phase 1 output [pair][rows]
  int ld_h;
  float *y;               // phase 2 output [pair][rows]
  int ld_y;
  int *err;
};

__device__ __forceinline__ uint32_t sa(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint32_t sw128(int r, int kc) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((kc ^ (r & 7)) << 4));
}
// K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16: f32 accumulate, f16 A and B, both K-major.
__device__ __forceinline__ uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void bar_init(uint64_t *b, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(count));
}
__device__ __forceinline__ void bar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
// Wait for the completion of the phase with parity `par`; false on time-out.
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t par, int *err) {
  uint32_t ok = 0;
  for (long long it = 0; it < kSpinLimit; ++it) {
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(sa(b)), "r"(par) : "memory");
    if (ok) return true;
    if ((it & 1023) == 1023 && *(volatile int *)err) return false;  // another role gave up
  }
  atomicExch(err, 1);
  return false;
}
__device__ __forceinline__ void cp_async_bar_arrive(uint64_t *b) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t *b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
               ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
// A from TMEM (M = 128 lanes = rows, K along columns, two f16 per column)
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
               ::"r"(d), "r"(a), "l"(b), "r"(id), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
// 32 columns of this thread's TMEM lane; complete (wait::st) on return
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
               "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
               ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
                 "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
                 "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
                 "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]),
                 "r"(v[31]) : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// without the wait: several loads in flight, then one tcgen05.wait::ld
__device__ __forceinline__ void tc_ld16_nw(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
               : "r"(taddr) : "memory");
}

// the decode path's SwiGLU (flash1017.rs:7539): min(silu(g), 10) * clamp(u, -10, 10),
// NaN propagating like Rust's f32::clamp
__device__ __forceinline__ float silu10(float g) { return fminf(g / (1.0f + expf(-g)), 10.0f); }
// the same with the hardware exp2 approximation and a fast divide (relative
// error ~1e-6, far inside the path's 1e-3 output tolerance; h is rounded to f16)
__device__ __forceinline__ float silu10_fast(float g) { return fminf(__fdividef(g, 1.0f + __expf(-g)), 10.0f); }
__device__ __forceinline__ float clamp10f(float u) {
  if (u < -10.f) u = -10.f;
  if (u > 10.f) u = 10.f;
  return u;
}

template <int PH>
__global__ void __launch_bounds__(kThreadsGG, 1) gemm_kernel(const GemmArgs a) {
  pdl_enter();
  using L = Layout<PH>;
  constexpr int NMAT = L::NMAT;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t x_full[kXStages], x_empty[kXStages];
  __shared__ __align__(8) uint64_t a_full[kAStages], a_empty[kAStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ float s_xs[2][kMaxN];  // phase 1: 2^xe of the tile's tokens (by tile parity)
  uint8_t *smem = smem_raw + ((1024 - (sa(smem_raw) & 1023)) & 1023);
  uint8_t *xbuf = smem, *wbuf = smem + L::OFF_W;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kXStages; ++s) { bar_init(&x_full[s], kXLanes); bar_init(&x_empty[s], 1); }
    for (int s = 0; s < kAStages; ++s) { bar_init(&a_full[s], kDecWarps); bar_init(&a_empty[s], 1); }
    for (int b = 0; b < 2; ++b) { bar_init(&acc_full[b], 1); bar_init(&acc_empty[b], kDecWarps); }
    bar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&s_tmem)),
                 "r"(L::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  const int n_chunks = *a.n_chunks;
  const int fb_count = a.rows / L::ROWS;
  const int n_tiles = n_chunks * fb_count;
  const int KT = a.K / kTileK;
  const size_t wld = (size_t)a.K / 2, sld = (size_t)a.K / 16;

  if (warp == 0 || warp == 1 || warp == 3) {
    // ------------------------------------------------ activation producers (96 lanes)
    // eight lanes per row (one 16-byte piece each): an instruction covers
    // whole 128-byte rows of 4 tokens
    constexpr int RI = (kMaxN * 8 + kXLanes - 1) / kXLanes;  // rows per lane (rows >= nn skipped)
    const int xl = (warp == 0 ? 0 : warp == 1 ? 32 : 64) + lane;
    const int kc = xl & 7;
    int it = 0;
    bool live = true;
    for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x) {
      const Chunk ch = a.chunks[tile / fb_count];
      const __half *rp[RI];
#pragma unroll
      for (int j = 0; j < RI; ++j) {
        const int n = (xl >> 3) + (kXLanes / 8) * j;
        rp[j] = nullptr;
        if (n < ch.nn) {
          const int p = ch.p0 + n;
          const int xr = PH == 1 ? __ldg(a.pair_tok + p) : p;
          rp[j] = a.x + (size_t)xr * a.ld_x + kc * 8;
        }
      }
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % kXStages;
        if (!bar_wait(&x_empty[s], ((it / kXStages) & 1) ^ 1, a.err)) { live = false; break; }
        uint8_t *st = xbuf + s * L::X_STAGE;
#pragma unroll
        for (int j = 0; j < RI; ++j)
          if (rp[j]) cp_async16(st + sw128((xl >> 3) + (kXLanes / 8) * j, kc), rp[j] + kt * kTileK);
        cp_async_bar_arrive(&x_full[s]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int itx = 0, ita = 0, tcount = 0;
      bool live = true;
      for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x, ++tcount) {
        const Chunk ch = a.chunks[tile / fb_count];
        const uint32_t id = idesc_f16(kTileM, ch.npad);
        const int b = L::ACC_BUFS == 1 ? 0 : (tcount & 1);
        const int use = L::ACC_BUFS == 1 ? tcount : (tcount >> 1);
        if (!bar_wait(&acc_empty[b], (use & 1) ^ 1, a.err)) break;
        tc_fence_after();
        const uint32_t acc_col = tmem + b * L::ACC_COLS;
        for (int kt = 0; kt < KT; ++kt, ++itx, ++ita) {
          const int s3 = itx % kXStages, s2 = ita % kAStages;
          if (!bar_wait(&x_full[s3], (itx / kXStages) & 1, a.err) ||
              !bar_wait(&a_full[s2], (ita / kAStages) & 1, a.err)) { live = false; break; }
          fence_async_smem();
          tc_fence_after();
          const uint32_t xb = sa(xbuf + s3 * L::X_STAGE);
          const uint32_t ab = tmem + L::A_COL0 + s2 * L::A_COLS;
#pragma unroll
          for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
            for (int j = 0; j < kTileK / 16; ++j)
              tc_mma_ts(acc_col + mi * kMaxN, ab + mi * (kTileK / 2) + 8 * j, sdesc(xb + 32 * j), id,
                     (kt > 0 || j > 0) ? 1u : 0u);
          tc_commit(&a_empty[s2]);
          tc_commit(&x_empty[s3]);
        }
        if (!live) break;
        tc_commit(&acc_full[b]);
      }
      // every MMA this thread issued has completed before TMEM is freed
      tc_commit(&mma_done);
      bar_wait(&mma_done, 0, a.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ decode + epilogue (8 warps)
    const int d = tid - 128, half = d >> 7;
    const int r = d & 127;  // tile row = TMEM lane (warp w: quarter w % 4)
    // half h decodes row r of A block h
    const int mi = half;
    // This warp's weight ring: its 32 rows of block mi, kWSteps K-steps per
    // stage; lanes copy four 16-byte pieces of eight rows per instruction and
    // one scale row each; kWStages - 1 stages in flight, across tiles.  Piece
    // c of row r sits at piece slot c ^ pswz(r) of the row, so the decode's
    // 16-byte row reads are free of bank conflicts while each copy
    // instruction still fills 512 contiguous bytes.
    const int dw = warp - 4, rw0 = 32 * (dw & 3);
    uint8_t *ring = wbuf + dw * kWStages * L::WSLOT;
    int p_tile = blockIdx.x, p_kw = 0, p_slot = 0;
    const uint8_t *p_w = nullptr, *p_s = nullptr;
    bool p_s8 = true;
    auto issue_next = [&]() {
      if (p_tile < n_tiles) {
        if (p_kw == 0) {
          const Chunk pc_ = a.chunks[p_tile / fb_count];
          const int prow0 = (p_tile % fb_count) * L::ROWS;
          const ffn_b200_expert &PE = a.experts[pc_.expert];
          p_w = (PH == 1 ? PE.nv[mi].w : PE.nv[2].w + (size_t)mi * kTileM * wld) + (size_t)(prow0 + rw0) * wld;
          p_s = (PH == 1 ? PE.nv[mi].s : PE.nv[2].s + (size_t)mi * kTileM * sld) + (size_t)(prow0 + rw0) * sld;
          p_s8 = ((reinterpret_cast<uintptr_t>(p_s) | (sld * sizeof(uint8_t))) & (L::SB - 1)) == 0;
        }
        uint8_t *slot = ring + p_slot * L::WSLOT;
#pragma unroll
        for (int j = 0; j < 32 * L::PPR / 32; ++j) {
          const int q = lane + 32 * j, rr = q / L::PPR, pc = q % L::PPR;
          cp_async16(slot + rr * L::RB + ((pc ^ L::pswz(rr)) << 4), p_w + (size_t)rr * wld + p_kw * L::RB + pc * 16);
        }
        uint8_t *sd = slot + 32 * L::RB + lane * L::SB;
        const uint8_t *ss = p_s + (size_t)lane * sld + p_kw * L::SB;
        if (p_s8) {
          cp_async_n<L::SB>(sd, ss);
        } else {
#pragma unroll
          for (int q = 0; q < L::SB / 4; ++q) cp_async4(sd + 4 * q, ss + 4 * q);
        }
        if (++p_kw == KT / kWSteps) { p_kw = 0; p_tile += gridDim.x; }
      }
      cp_async_commit();
      p_slot = p_slot + 1 == kWStages ? 0 : p_slot + 1;
    };
#pragma unroll
    for (int q = 0; q < kWStages - 1; ++q) issue_next();
    int itw = 0, ita = 0, tcount = 0;
    bool live = true;
    for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x, ++tcount) {
      const Chunk ch = a.chunks[tile / fb_count];
      const int row0 = (tile % fb_count) * L::ROWS;
      if (PH == 1) {
        // token scales of the tile's columns, read by every epilogue thread;
        // a buffer is rewritten two tiles later, after all decode warps have
        // finished this tile's epilogue (the next tile's MMAs wait for that)
        static_assert(kMaxN <= kDecWarps * 32, "one decode thread per chunk column");
        if (d < kMaxN) s_xs[tcount & 1][d] = d < ch.nn ? pow2f(__ldg(a.xe + __ldg(a.pair_tok + ch.p0 + d))) : 0.f;
        asm volatile("bar.sync 1, %0;" ::"n"(kDecWarps * 32) : "memory");
      }
      for (int kt = 0; kt < KT; ++kt, ++ita) {
        const int sub = kt % kWSteps;  // K-step inside the weight stage
        const int s = itw % kWStages, s2 = ita % kAStages;
        if (sub == 0) {  // refill the slot consumed last, then wait for this stage
          issue_next();
          cp_async_wait<kWStages - 1>();
          __syncwarp();
        }
        const bool ok = bar_wait(&a_empty[s2], ((ita / kAStages) & 1) ^ 1, a.err);
        if (!__all_sync(0xffffffffu, ok)) { live = false; break; }
        const uint8_t *st = ring + s * L::WSLOT;
        tc_fence_after();
        // this warp's 32 lanes of block mi, stage s2
        const uint32_t at = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + L::A_COL0 + s2 * L::A_COLS +
                            mi * (kTileK / 2);
        {
          const uint8_t *wr = st + lane * L::RB;
          const int sw = L::pswz(lane);
          const uint4 w0 = *reinterpret_cast<const uint4 *>(wr + (((2 * sub) ^ sw) << 4));
          const uint4 w1 = *reinterpret_cast<const uint4 *>(wr + (((2 * sub + 1) ^ sw) << 4));
          const uint32_t sc4 = *reinterpret_cast<const uint32_t *>(st + 32 * L::RB + lane * L::SB + sub * 4);
          const uint32_t s01 = e4m3x2_to_f16x2((uint16_t)(sc4 & 0xFFFFu));
          const uint32_t s23 = e4m3x2_to_f16x2((uint16_t)(sc4 >> 16));
          const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          uint32_t o[32];  // TMEM column c = f16 pair (2c, 2c + 1) of the row's 64 K values
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // word j = K values 8j..8j+7
            uint32_t dd[4];
            e2m1x8_to_f16x2(words[j], dd);
            const uint32_t sc = j < 2 ? bcast_lo(s01) : j < 4 ? bcast_hi(s01) : j < 6 ? bcast_lo(s23) : bcast_hi(s23);
#pragma unroll
            for (int q = 0; q < 4; ++q) o[4 * j + q] = hmul2_u32(dd[q], sc);
          }
          tc_st32(at, o);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) bar_arrive(&a_full[s2]);
        if (sub == kWSteps - 1) ++itw;
      }
      if (!live) break;
      // epilogue: this thread's TMEM lane = tile row r
      const int b = L::ACC_BUFS == 1 ? 0 : (tcount & 1);
      const int use = L::ACC_BUFS == 1 ? tcount : (tcount >> 1);
      if (!__all_sync(0xffffffffu, bar_wait(&acc_full[b], use & 1, a.err))) break;
      tc_fence_after();
      const int row = row0 + r;
      const uint32_t tl = tmem + b * L::ACC_COLS + ((uint32_t)(32 * (warp & 3)) << 16);
      const ffn_b200_expert &E = a.experts[ch.expert];
      const float gs0 = E.nv[PH == 1 ? 0 : 2].gs, gs1 = E.nv[PH == 1 ? 1 : 2].gs;
      const int split = ((ch.npad / 16 + 1) / 2) * 16;  // columns [0, split) | [split, npad)
      // 16 columns of both blocks -> h (phase 1) or y (phase 2)
      auto emit = [&](const uint32_t (&v0)[16], const uint32_t (&v1)[16], int n0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = n0 + j;
          if (n >= ch.nn) continue;
          const int p = ch.p0 + n;
          if (PH == 1) {
            const float xs = s_xs[tcount & 1][n];
            const float g = __uint_as_float(v0[j]) * xs * gs0;
            const float u = __uint_as_float(v1[j]) * xs * gs1;
            a.h[(size_t)p * a.ld_h + row] = __float2half_rn(silu10_fast(g) * clamp10f(u));
          } else {
            a.y[(size_t)p * a.ld_y + row] = __uint_as_float(v0[j]) * gs0;
            a.y[(size_t)p * a.ld_y + row + kTileM] = __uint_as_float(v1[j]) * gs1;
          }
        }
      };
      const int n_end = half ? ch.npad : split;
      for (int n0 = half ? split : 0; n0 < n_end; n0 += 32) {
        uint32_t g0[16], u0[16], g1[16], u1[16];
        const bool two = n0 + 16 < n_end;  // warp-uniform
        tc_ld16_nw(tl + n0, g0);
        tc_ld16_nw(tl + kMaxN + n0, u0);
        if (two) {
          tc_ld16_nw(tl + n0 + 16, g1);
          tc_ld16_nw(tl + kMaxN + n0 + 16, u1);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        emit(g0, u0, n0);
        if (two) emit(g1, u1, n0 + 16);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&acc_empty[b]);
    }
  }
  // drain: every cp.async of this thread has landed before the CTA leaves
  asm volatile("cp.async.wait_all;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS));
  }
}

// Chunks of <= kMaxN pairs per local expert, balanced inside an expert
// (c pairs -> ceil(c / kMaxN) chunks of equal size, rounded up to 16 columns).
__global__ void __launch_bounds__(1024) chunk_kernel(const int *__restrict__ counts,
                                                     const int *__restrict__ offsets, int e_begin,
                                                     int e_end, Chunk *chunks, int *n_chunks) {
  pdl_enter();
  __shared__ int warp_sum[32];
  __shared__ int s_base;
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int e0 = e_begin; e0 < e_end; e0 += blockDim.x) {
    const int e = e0 + threadIdx.x;
    const int c = e < e_end ? counts[e] : 0;
    const int nch = (c + kMaxN - 1) / kMaxN;
    int inc = nch;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    if (lane == 31) warp_sum[wid] = inc;
    __syncthreads();
    if (wid == 0) {
      int v = lane < (int)(blockDim.x >> 5) ? warp_sum[lane] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      warp_sum[lane] = v;
    }
    __syncthreads();
    const int base = s_base + (wid ? warp_sum[wid - 1] : 0) + inc - nch;
    if (nch) {
      const int per = (c + nch - 1) / nch;
      for (int j = 0; j < nch; ++j) {
        Chunk ch;
        ch.expert = e;
        ch.p0 = offsets[e] + j * per;
        ch.nn = min(per, c - j * per);
        ch.npad = (ch.nn + 15) & ~15;
        chunks[base + j] = ch;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) s_base += warp_sum[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) *n_chunks = s_base;
}

}  // namespace gg

size_t gg_chunk_bytes(int n_pairs, int n_local) {
  return (size_t)(n_pairs / 16 + n_local + 1) * sizeof(gg::Chunk) + 64;
}

int launch_grouped_moe(const GroupedArgs &g, cudaStream_t st) {
  using namespace gg;
  int dev = 0;
  FFN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "grouped_moe: device index >= 64");
  static bool attr[64] = {false};
  if (!attr[dev]) {
    FFN_CUDA_TRY(cudaFuncSetAttribute(gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<1>::SMEM));
    FFN_CUDA_TRY(cudaFuncSetAttribute(gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<2>::SMEM));
    attr[dev] = true;
  }
  Chunk *chunks = reinterpret_cast<Chunk *>(g.chunk_ws);
  int *n_chunks = reinterpret_cast<int *>(g.chunk_ws + gg_chunk_bytes(g.n_pairs, g.e_end - g.e_begin) - 64);
  FFN_CUDA_TRY(cudaMemsetAsync(g.err, 0, sizeof(int), st));
  FFN_LAUNCH_PDL(FFN_B200_K_GROUP, st, "chunk_kernel", chunk_kernel, 1, 1024, 0, g.counts, g.offsets, g.e_begin, g.e_end, chunks, n_chunks);
  const int sms = sm_count_of(dev);
  const long long max_chunks = g.n_pairs / 16 + (g.e_end - g.e_begin);
  GemmArgs p{};
  p.experts = g.experts;
  p.chunks = chunks;
  p.n_chunks = n_chunks;
  p.pair_tok = g.pair_tok;
  p.xe = g.xe;
  p.err = g.err;
  p.K = g.hidden;
  p.rows = g.inter;
  p.x = g.xh;
  p.ld_x = g.ld_x;
  p.h = g.h;
  p.ld_h = g.inter;
  int grid = (int)std::max(1LL, std::min<long long>(sms, max_chunks * (g.inter / Layout<1>::ROWS)));
  FFN_LAUNCH_PDL(FFN_B200_K_GEMM_GATEUP, st, "grouped gemm_kernel<1>", (gemm_kernel<1>), grid, kThreadsGG, Layout<1>::SMEM, p);
  GemmArgs q = p;
  q.K = g.inter;
  q.rows = g.hidden;
  q.x = g.h;
  q.ld_x = g.inter;
  q.y = g.y;
  q.ld_y = g.hidden;
  grid = (int)std::max(1LL, std::min<long long>(sms, max_chunks * (g.hidden / Layout<2>::ROWS)));
  FFN_LAUNCH_PDL(FFN_B200_K_GEMM_DOWN, st, "grouped gemm_kernel<2>", (gemm_kernel<2>), grid, kThreadsGG, Layout<2>::SMEM, q);
  return 0;
}

}  // namespace ffn
