// gemv_tile.cuh -- grouped low-token-count GEMM tile engine for NVFP4 and
// packed ternary weights on sm_100a.
//
// One CTA computes a tile of ROWS = 16*R output rows of NMAT matrices that
// share those rows (gate+up, or a single matrix) for up to 8 tokens, over the
// whole reduction dimension K.  The 8 warps split K chunk-wise; each warp keeps
// its partial sums in mma accumulators and the CTA reduces them through shared
// memory in a fixed warp order (deterministic results).
//
// Weights stream from HBM with 128-bit non-allocating loads and are decoded in
// registers straight into mma.sync m16n8k16 A fragments:
//   NVFP4   cvt.rn.f16x2.e2m1x2 gives the E2M1 values exactly; one HMUL2 by the
//           E4M3 block scale (also exact in f16: <= 6 significant bits, range
//           2^-10..2688) folds the block scale into A.  The per-tensor scale is
//           applied in f32 in the epilogue.
//   ternary the 2-bit code of each element is moved to bits 15:14 of an f16 and
//           inverted, giving exactly 2*v; the factor 1/2 and the row scale are
//           applied in the epilogue.
// Activations enter as two f16 terms (hi = f16(x), lo = f16(x - hi)) of a
// per-token power-of-two normalised row, so the two MMAs reproduce fp32
// products to about 2^-22 relative; accumulation is fp32.
//
// Column <-> MMA-k mapping.  NVFP4: chunk c = 128 columns; thread t of a quad
// owns columns [c*128 + 32t, +32) = 16 bytes of each row = 8 MMA k-steps; step
// j uses bytes 2j (k = 2t, 2t+1) and 2j+1 (k = 2t+8, 2t+9), i.e. columns
// 4j..4j+3, and the B fragment is the 4 consecutive activation halves at those
// columns.  Ternary: chunk = 256 columns; thread t owns [c*256 + 64t, +64) =
// 16 bytes = four 16-column words; step s of word q uses code pairs 2s and
// 2s+1 (columns {2s, 2s+8} and {2s+1, 2s+9}); activations are stored in
// "pair order" (column i at 2i, column i+8 at 2i+1 inside each 16 block) so the
// B fragment is again 4 consecutive halves.
#pragma once

#include "common.cuh"

namespace ffn {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct MatRef {          // one weight matrix as the tile engine sees it
  const uint8_t *w;      // NVFP4 packed / ternary packed
  const uint8_t *s;      // NVFP4 block scales (unused for ternary)
};

template <int FMT, int NMAT, int R>
struct TileEngine {
  static constexpr int ROWS = 16 * R;
  static constexpr int CHUNK = FMT == FFN_B200_FMT_NVFP4 ? 128 : 256;  // columns per chunk
  // shared memory for the cross-warp reduction: [warp][mat][token][RLD]; the
  // row stride RLD = ROWS + 4 keeps both the fragment writes and the row-wise
  // reads free of bank conflicts.
  static constexpr int RLD = ROWS + 4;
  static constexpr int RED_FLOATS = kWarps * NMAT * kNTok * RLD;

  // Accumulate this warp's K-slice of the tile into acc.
  // rows: valid output rows of the matrices; row0: first row of the tile;
  // xhi/xlo: this thread's token row (token slot lane/4), used when has_tok.
  __device__ static void run(const MatRef (&m)[NMAT], int rows, int K, int row0, bool has_tok,
                             const __half *xhi, const __half *xlo, float (&acc)[NMAT][R][4]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[mi][i][q] = 0.f;

    // Row indices (clamped for loads; results of clamped rows are discarded).
    int ra[R], rb[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      ra[i] = min(row0 + 16 * i + g, rows - 1);
      rb[i] = min(row0 + 16 * i + g + 8, rows - 1);
    }
    const int nchunks = (K + CHUNK - 1) / CHUNK;

    if constexpr (FMT == FFN_B200_FMT_NVFP4) {
      const size_t wld = (size_t)K / 2, sld = (size_t)K / 16;
      for (int c = warp; c < nchunks; c += kWarps) {
        const int col0 = c * CHUNK + 32 * t;
        const bool valid = col0 < K;  // K % 32 == 0: a thread's 32 columns are all valid or not
        uint4 wa[NMAT][R], wb[NMAT][R];
        uint32_t sa[NMAT][R], sb[NMAT][R];
#pragma unroll
        for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
          for (int i = 0; i < R; ++i) {
            if (valid) {
              wa[mi][i] = ldg_stream(m[mi].w + ra[i] * wld + col0 / 2);
              wb[mi][i] = ldg_stream(m[mi].w + rb[i] * wld + col0 / 2);
              sa[mi][i] = __ldg(reinterpret_cast<const uint16_t *>(m[mi].s + ra[i] * sld + col0 / 16));
              sb[mi][i] = __ldg(reinterpret_cast<const uint16_t *>(m[mi].s + rb[i] * sld + col0 / 16));
            } else {
              wa[mi][i] = wb[mi][i] = make_uint4(0, 0, 0, 0);
              sa[mi][i] = sb[mi][i] = 0;
            }
          }
        uint32_t sfa[NMAT][R], sfb[NMAT][R];
#pragma unroll
        for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
          for (int i = 0; i < R; ++i) {
            sfa[mi][i] = e4m3x2_to_f16x2((uint16_t)sa[mi][i]);
            sfb[mi][i] = e4m3x2_to_f16x2((uint16_t)sb[mi][i]);
          }
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
          // word wd = bytes 4wd..4wd+3 = columns col0+8wd.. = k-steps 2wd, 2wd+1;
          // its activations are one 16-byte load each for hi and lo.
          uint32_t bh[4], bl[4];
          if (valid && has_tok) {
            const uint4 h = ldg_cached(xhi + col0 + 8 * wd);
            const uint4 l = ldg_cached(xlo + col0 + 8 * wd);
            bh[0] = h.x; bh[1] = h.y; bh[2] = h.z; bh[3] = h.w;
            bl[0] = l.x; bl[1] = l.y; bl[2] = l.z; bl[3] = l.w;
          } else {
            bh[0] = bh[1] = bh[2] = bh[3] = bl[0] = bl[1] = bl[2] = bl[3] = 0u;
          }
#pragma unroll
          for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
            for (int i = 0; i < R; ++i) {
              // group 0 (first 16 columns of the thread) for words 0, 1
              const uint32_t s_a = wd < 2 ? bcast_lo(sfa[mi][i]) : bcast_hi(sfa[mi][i]);
              const uint32_t s_b = wd < 2 ? bcast_lo(sfb[mi][i]) : bcast_hi(sfb[mi][i]);
              const uint32_t xa = wd == 0 ? wa[mi][i].x : wd == 1 ? wa[mi][i].y : wd == 2 ? wa[mi][i].z : wa[mi][i].w;
              const uint32_t xb = wd == 0 ? wb[mi][i].x : wd == 1 ? wb[mi][i].y : wd == 2 ? wb[mi][i].z : wb[mi][i].w;
              uint32_t da[4], db[4];
              e2m1x8_to_f16x2(xa, da);
              e2m1x8_to_f16x2(xb, db);
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t a0 = hmul2_u32(da[2 * h], s_a);
                const uint32_t a1 = hmul2_u32(db[2 * h], s_b);
                const uint32_t a2 = hmul2_u32(da[2 * h + 1], s_a);
                const uint32_t a3 = hmul2_u32(db[2 * h + 1], s_b);
                mma_f16(acc[mi][i], a0, a1, a2, a3, bh[2 * h], bh[2 * h + 1]);
                mma_f16(acc[mi][i], a0, a1, a2, a3, bl[2 * h], bl[2 * h + 1]);
              }
            }
        }
      }
    } else {
      const size_t wld = (size_t)K / 4;
      for (int c = warp; c < nchunks; c += kWarps) {
        const int col0 = c * CHUNK + 64 * t;
        const bool valid = col0 < K;  // K % 64 == 0
        uint4 wa[NMAT][R], wb[NMAT][R];
#pragma unroll
        for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
          for (int i = 0; i < R; ++i) {
            if (valid) {
              wa[mi][i] = ldg_stream(m[mi].w + ra[i] * wld + col0 / 4);
              wb[mi][i] = ldg_stream(m[mi].w + rb[i] * wld + col0 / 4);
            } else {
              // code 1 everywhere (0x55) decodes to zero
              wa[mi][i] = wb[mi][i] = make_uint4(0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u);
            }
          }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t bh[8], bl[8];
          if (valid && has_tok) {
#pragma unroll
            for (int v = 0; v < 2; ++v) {
              const uint4 h = ldg_cached(xhi + col0 + 16 * q + 8 * v);
              const uint4 l = ldg_cached(xlo + col0 + 16 * q + 8 * v);
              bh[4 * v] = h.x; bh[4 * v + 1] = h.y; bh[4 * v + 2] = h.z; bh[4 * v + 3] = h.w;
              bl[4 * v] = l.x; bl[4 * v + 1] = l.y; bl[4 * v + 2] = l.z; bl[4 * v + 3] = l.w;
            }
          } else {
#pragma unroll
            for (int v = 0; v < 8; ++v) bh[v] = bl[v] = 0u;
          }
#pragma unroll
          for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
            for (int i = 0; i < R; ++i) {
              const uint32_t xa = q == 0 ? wa[mi][i].x : q == 1 ? wa[mi][i].y : q == 2 ? wa[mi][i].z : wa[mi][i].w;
              const uint32_t xb = q == 0 ? wb[mi][i].x : q == 1 ? wb[mi][i].y : q == 2 ? wb[mi][i].z : wb[mi][i].w;
              tern_steps(acc[mi][i], xa, xb, bh, bl);
            }
        }
      }
    }
  }

  // Four MMA k-steps of one 16-column ternary word (rows g and g+8).
  __device__ static __forceinline__ void tern_steps(float (&d)[4], uint32_t xa, uint32_t xb,
                                                    const uint32_t (&bh)[8],
                                                    const uint32_t (&bl)[8]) {
#define FFN_TSTEP(S)                                                                  \
  {                                                                                   \
    const uint32_t a0 = tern_pair<2 * S>(xa), a1 = tern_pair<2 * S>(xb);              \
    const uint32_t a2 = tern_pair<2 * S + 1>(xa), a3 = tern_pair<2 * S + 1>(xb);      \
    mma_f16(d, a0, a1, a2, a3, bh[2 * S], bh[2 * S + 1]);                             \
    mma_f16(d, a0, a1, a2, a3, bl[2 * S], bl[2 * S + 1]);                             \
  }
    FFN_TSTEP(0) FFN_TSTEP(1) FFN_TSTEP(2) FFN_TSTEP(3)
#undef FFN_TSTEP
  }

  // Write this warp's partial sums to shared memory: red[warp][mat][tok][row].
  __device__ static void stash(float *red, const float (&acc)[NMAT][R][4]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
      for (int i = 0; i < R; ++i) {
        float *base = red + (warp * NMAT + mi) * kNTok * RLD;
        const int r0 = 16 * i + g, r1 = r0 + 8;
        base[(2 * t) * RLD + r0] = acc[mi][i][0];
        base[(2 * t + 1) * RLD + r0] = acc[mi][i][1];
        base[(2 * t) * RLD + r1] = acc[mi][i][2];
        base[(2 * t + 1) * RLD + r1] = acc[mi][i][3];
      }
  }

  // Sum of all warps' partials for (mat, row_in_tile, tok), fixed warp order.
  __device__ static __forceinline__ float total(const float *red, int mi, int r, int n) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[((w * NMAT + mi) * kNTok + n) * RLD + r];
    return s;
  }
};

}  // namespace ffn
