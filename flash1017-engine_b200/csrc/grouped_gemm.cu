// grouped_gemm.cu -- tensor-core (tcgen05) grouped GEMM for many tokens per
// expert: the MoE prefill path (batched tokens of crates/flash-core/src/
// flash1017.rs:8267-8326, the same arithmetic as the decode path).
//
// Per local expert the routed tokens form chunks of <= 256 pairs.  A tile is
// (chunk, block of 128 output rows); one CTA per SM walks the tiles.
//
//   phase 1:  D_g = W1[rows] . X^T, D_u = W3[rows] . X^T  (K = hidden)
//             h[p][row] = f16( min(silu(g), 10) * clamp(u, -10, 10) ),
//             g = D_g * 2^xe[tok] * gs1, u = D_u * 2^xe[tok] * gs3
//   phase 2:  y[p][row] = (W2[rows] . H^T) * gs2                (K = inter)
//
// MMA: tcgen05.mma.cta_group::1.kind::f16, M = 128 weight rows, N = chunk
// tokens rounded up to 16, K = 16 per instruction, fp32 accumulators in TMEM
// (phase 1: gate in columns [0, 256), up in [256, 512)).  Operands are K-major
// tiles of 64 columns in the 128-byte swizzled canonical layout.
//
// Weights: NVFP4 rows are decoded on the fly into f16 (exact: an E2M1 value
// times an E4M3 scale has at most 6 significant bits, inside f16's range), so
// the tensor core sees the reference's dequantised weights.  Activations:
// phase 1 takes x * 2^-xe as one f16 term (bf16 inputs, config 3, are exact
// there); phase 2 takes h rounded to f16.  Relative error of an output about
// 2^-12 (measured ~2e-4), inside the path's 1e-3 tolerance.
//
// Warp roles (256 threads):
//   warps 0, 1, 3  producers: cp.async of the raw NVFP4 rows + scales of the
//                  tile's K-step into a raw stage, and of the chunk's
//                  activation rows straight into their swizzled B tile;
//                  completion is an mbarrier arrive per lane (noinc).
//   warp 2         TMEM allocation; lane 0 issues the MMAs and commits them to
//                  the stage / accumulator barriers.
//   warps 4-7      decode a raw stage into the f16 A tile(s) (thread = row),
//                  and after a tile's last K-step run the epilogue from TMEM
//                  (warp w reads TMEM lanes 32 (w % 4) ...).
// Every mbarrier wait is bounded; a wait that runs out sets *err and the
// kernel drains and returns (the host turns *err into FFN_B200_ECUDA).
#include <algorithm>

#include "ffn_internal.h"
#include "gemv_tile.cuh"

namespace ffn {
namespace gg {

constexpr int kThreadsGG = 256;
constexpr int kRawStages = 3;
constexpr int kAStages = 2;
constexpr int kTileM = 128;
constexpr int kTileK = 64;
constexpr int kMaxN = 256;
constexpr int kProducerLanes = 96;  // warps 0, 1, 3
constexpr long long kSpinLimit = 1LL << 22;  // try_wait polls per wait before giving up

template <int PH>
struct Layout {
  static constexpr int NMAT = PH == 1 ? 2 : 1;
  static constexpr int RAW_W = NMAT * kTileM * 32;   // NVFP4 bytes of a K-step
  static constexpr int RAW_S = NMAT * kTileM * 4;    // scale bytes of a K-step
  static constexpr int RAW_X = kMaxN * 128;          // activation tile (swizzled)
  static constexpr int RAW = (RAW_X + RAW_W + RAW_S + 1023) & ~1023;  // x first, 1024-aligned stages
  static constexpr int A_TILE = kTileM * 128;        // one f16 A tile
  static constexpr int A_STAGE = NMAT * A_TILE;
  static constexpr int SMEM = 1024 + kRawStages * RAW + kAStages * A_STAGE;
  static constexpr int TMEM_COLS = PH == 1 ? 512 : 256;
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
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// the decode path's SwiGLU (flash1017.rs:7539): min(silu(g), 10) * clamp(u, -10, 10),
// NaN propagating like Rust's f32::clamp
__device__ __forceinline__ float silu10(float g) { return fminf(g / (1.0f + expf(-g)), 10.0f); }
__device__ __forceinline__ float clamp10f(float u) {
  if (u < -10.f) u = -10.f;
  if (u > 10.f) u = 10.f;
  return u;
}

template <int PH>
__global__ void __launch_bounds__(kThreadsGG, 1) gemm_kernel(const GemmArgs a) {
  using L = Layout<PH>;
  constexpr int NMAT = L::NMAT;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t raw_full[kRawStages], raw_empty[kRawStages];
  __shared__ __align__(8) uint64_t a_full[kAStages], a_empty[kAStages];
  __shared__ __align__(8) uint64_t acc_full, acc_empty, mma_done;
  __shared__ uint32_t s_tmem;
  uint8_t *smem = smem_raw + ((1024 - (sa(smem_raw) & 1023)) & 1023);
  uint8_t *raw = smem;
  uint8_t *abuf = smem + kRawStages * L::RAW;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kRawStages; ++s) { bar_init(&raw_full[s], kProducerLanes); bar_init(&raw_empty[s], 5); }
    for (int s = 0; s < kAStages; ++s) { bar_init(&a_full[s], 4); bar_init(&a_empty[s], 1); }
    bar_init(&acc_full, 1);
    bar_init(&acc_empty, 4);
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
  const int fb_count = a.rows / kTileM;
  const int n_tiles = n_chunks * fb_count;
  const int KT = a.K / kTileK;
  const size_t wld = (size_t)a.K / 2, sld = (size_t)a.K / 16;

  if (warp == 0 || warp == 1 || warp == 3) {
    // ------------------------------------------------------------ producers
    const int pl = warp == 3 ? 64 + lane : warp * 32 + lane;  // 0..95
    int it = 0;
    bool live = true;
    for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x) {
      const Chunk ch = a.chunks[tile / fb_count];
      const int row0 = (tile % fb_count) * kTileM;
      const ffn_b200_expert &E = a.experts[ch.expert];
      const uint8_t *wsrc[NMAT], *ssrc[NMAT];
#pragma unroll
      for (int mi = 0; mi < NMAT; ++mi) {
        const ffn_b200_nvfp4_mat &m = E.nv[PH == 1 ? mi : 2];
        wsrc[mi] = m.w + (size_t)row0 * wld;
        ssrc[mi] = m.s + (size_t)row0 * sld;
      }
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % kRawStages;
        if (!bar_wait(&raw_empty[s], ((it / kRawStages) & 1) ^ 1, a.err)) { live = false; break; }
        uint8_t *st = raw + s * L::RAW;
        // activation rows: chunk row n, 16-byte piece kc -> swizzled B tile
        for (int q = pl; q < ch.nn * 8; q += kProducerLanes) {
          const int n = q >> 3, kc = q & 7;
          const int p = ch.p0 + n;
          const int xr = PH == 1 ? __ldg(a.pair_tok + p) : p;
          cp_async16(st + sw128(n, kc), a.x + (size_t)xr * a.ld_x + kt * kTileK + kc * 8);
        }
        // NVFP4 rows: 128 rows x 32 bytes per matrix (2 pieces of 16 bytes)
#pragma unroll
        for (int mi = 0; mi < NMAT; ++mi)
          for (int q = pl; q < kTileM * 2; q += kProducerLanes) {
            const int r = q >> 1, half = q & 1;
            cp_async16(st + L::RAW_X + mi * kTileM * 32 + r * 32 + half * 16,
                       wsrc[mi] + (size_t)r * wld + kt * 32 + half * 16);
          }
        // block scales: 128 rows x 4 bytes per matrix
#pragma unroll
        for (int mi = 0; mi < NMAT; ++mi)
          for (int r = pl; r < kTileM; r += kProducerLanes)
            cp_async4(st + L::RAW_X + L::RAW_W + mi * kTileM * 4 + r * 4, ssrc[mi] + (size_t)r * sld + kt * 4);
        cp_async_bar_arrive(&raw_full[s]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, ait = 0, tcount = 0;
      bool live = true;
      for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x, ++tcount) {
        const Chunk ch = a.chunks[tile / fb_count];
        const uint32_t id = idesc_f16(kTileM, ch.npad);
        if (!bar_wait(&acc_empty, (tcount & 1) ^ 1, a.err)) break;
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt, ++it, ++ait) {
          const int s = it % kRawStages, s2 = ait % kAStages;
          if (!bar_wait(&raw_full[s], (it / kRawStages) & 1, a.err) ||
              !bar_wait(&a_full[s2], (ait / kAStages) & 1, a.err)) { live = false; break; }
          fence_async_smem();
          tc_fence_after();
          const uint32_t xb = sa(raw + s * L::RAW);
          const uint32_t ab = sa(abuf + s2 * L::A_STAGE);
#pragma unroll
          for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
            for (int j = 0; j < kTileK / 16; ++j)
              tc_mma(tmem + mi * 256, sdesc(ab + mi * L::A_TILE + 32 * j), sdesc(xb + 32 * j), id,
                     (kt > 0 || j > 0) ? 1u : 0u);
          tc_commit(&a_empty[s2]);
          tc_commit(&raw_empty[s]);
        }
        if (!live) break;
        tc_commit(&acc_full);
      }
      // every MMA this thread issued has completed before TMEM is freed
      tc_commit(&mma_done);
      bar_wait(&mma_done, 0, a.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ decode + epilogue
    const int r = tid - 128;  // tile row, 0..127 (warps 4-7 = TMEM lane quarters 0-3)
    int it = 0, ait = 0, tcount = 0;
    bool live = true;
    for (int tile = blockIdx.x; tile < n_tiles && live; tile += gridDim.x, ++tcount) {
      const Chunk ch = a.chunks[tile / fb_count];
      const int row0 = (tile % fb_count) * kTileM;
      for (int kt = 0; kt < KT; ++kt, ++it, ++ait) {
        const int s = it % kRawStages, s2 = ait % kAStages;
        const bool ok = bar_wait(&raw_full[s], (it / kRawStages) & 1, a.err) &&
                        bar_wait(&a_empty[s2], ((ait / kAStages) & 1) ^ 1, a.err);
        if (!__all_sync(0xffffffffu, ok)) { live = false; break; }
        const uint8_t *st = raw + s * L::RAW;
        uint8_t *at = abuf + s2 * L::A_STAGE;
#pragma unroll
        for (int mi = 0; mi < NMAT; ++mi) {
          const uint4 w0 = *reinterpret_cast<const uint4 *>(st + L::RAW_X + mi * kTileM * 32 + r * 32);
          const uint4 w1 = *reinterpret_cast<const uint4 *>(st + L::RAW_X + mi * kTileM * 32 + r * 32 + 16);
          const uint32_t sc4 = *reinterpret_cast<const uint32_t *>(st + L::RAW_X + L::RAW_W + mi * kTileM * 4 + r * 4);
          const uint32_t s01 = e4m3x2_to_f16x2((uint16_t)(sc4 & 0xFFFFu));
          const uint32_t s23 = e4m3x2_to_f16x2((uint16_t)(sc4 >> 16));
          const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // word j = columns 8j..8j+7 = 16-byte chunk j
            uint32_t d[4];
            e2m1x8_to_f16x2(words[j], d);
            const uint32_t sc = j < 2 ? bcast_lo(s01) : j < 4 ? bcast_hi(s01) : j < 6 ? bcast_lo(s23) : bcast_hi(s23);
            uint4 o;
            o.x = hmul2_u32(d[0], sc);
            o.y = hmul2_u32(d[1], sc);
            o.z = hmul2_u32(d[2], sc);
            o.w = hmul2_u32(d[3], sc);
            *reinterpret_cast<uint4 *>(at + mi * L::A_TILE + sw128(r, j)) = o;
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) { bar_arrive(&a_full[s2]); bar_arrive(&raw_empty[s]); }
      }
      if (!live) break;
      // epilogue: this thread's TMEM lane = tile row r
      if (!__all_sync(0xffffffffu, bar_wait(&acc_full, tcount & 1, a.err))) break;
      tc_fence_after();
      const int row = row0 + r;
      const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
      const ffn_b200_expert &E = a.experts[ch.expert];
      const float gs0 = E.nv[PH == 1 ? 0 : 2].gs, gs1 = E.nv[1].gs;
      for (int n0 = 0; n0 < ch.npad; n0 += 16) {
        uint32_t v0[16], v1[16];
        tc_ld16(tl + n0, v0);
        if (PH == 1) tc_ld16(tl + 256 + n0, v1);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = n0 + j;
          if (n >= ch.nn) break;
          const int p = ch.p0 + n;
          if (PH == 1) {
            const float xs = pow2f(__ldg(a.xe + __ldg(a.pair_tok + p)));
            const float g = __uint_as_float(v0[j]) * xs * gs0;
            const float u = __uint_as_float(v1[j]) * xs * gs1;
            a.h[(size_t)p * a.ld_h + row] = __float2half_rn(silu10(g) * clamp10f(u));
          } else {
            a.y[(size_t)p * a.ld_y + row] = __uint_as_float(v0[j]) * gs0;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&acc_empty);
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

// Chunks of <= 256 pairs per local expert, balanced inside an expert
// (c pairs -> ceil(c / 256) chunks of equal size, rounded up to 16 columns).
__global__ void __launch_bounds__(1024) chunk_kernel(const int *__restrict__ counts,
                                                     const int *__restrict__ offsets, int e_begin,
                                                     int e_end, Chunk *chunks, int *n_chunks) {
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
  FFN_LAUNCH(FFN_B200_K_GROUP, st, "chunk_kernel",
             chunk_kernel<<<1, 1024, 0, st>>>(g.counts, g.offsets, g.e_begin, g.e_end, chunks, n_chunks));
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
  int grid = (int)std::max(1LL, std::min<long long>(sms, max_chunks * (g.inter / kTileM)));
  FFN_LAUNCH(FFN_B200_K_GEMM_GATEUP, st, "grouped gemm_kernel<1>",
             (gemm_kernel<1><<<grid, kThreadsGG, Layout<1>::SMEM, st>>>(p)));
  GemmArgs q = p;
  q.K = g.inter;
  q.rows = g.hidden;
  q.x = g.h;
  q.ld_x = g.inter;
  q.y = g.y;
  q.ld_y = g.hidden;
  grid = (int)std::max(1LL, std::min<long long>(sms, max_chunks * (g.hidden / kTileM)));
  FFN_LAUNCH(FFN_B200_K_GEMM_DOWN, st, "grouped gemm_kernel<2>",
             (gemm_kernel<2><<<grid, kThreadsGG, Layout<2>::SMEM, st>>>(q)));
  return 0;
}

}  // namespace ffn
