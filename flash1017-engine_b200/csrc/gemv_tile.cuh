// gemv_tile.cuh -- grouped low-token-count GEMM engine for NVFP4 and packed
// ternary weights on sm_100a: the per-warp building blocks.
//
// Work unit: a warp task = one slice of up to 8 tokens of one expert x one
// block of ROWS = 16*R output rows of NMAT matrices sharing those rows
// (gate+up: NMAT 2, R 1; one matrix: NMAT 1, R 2), over the whole reduction
// dimension K.  A warp runs its tasks independently of the other warps: no
// block barrier, no shared-memory reduction; a task's results sit in the
// warp's mma accumulators when its last K-chunk is done.
//
// Weight streaming: every warp owns a ring of STAGES shared-memory slots.  A
// "unit" is one K-chunk of one task (16 bytes of each of the task's rows per
// lane + the rows' block scales).  Units are copied with cp.async (16-byte .cg
// copies for weights, 4-byte copies for scales) STAGES-1 units ahead of the one
// being computed, across task boundaries, so the bytes in flight do not occupy
// registers.  Each lane reads back only the weight bytes it copied; scales are
// shared inside the warp.
//
// Decode into mma.sync m16n8k16 A fragments:
//   NVFP4   cvt.rn.f16x2.e2m1x2 gives the E2M1 values exactly; one HMUL2 by the
//           E4M3 block scale (also exact in f16: <= 6 significant bits, range
//           2^-10..2688) folds the block scale into A.  The per-tensor scale is
//           applied in f32 in the epilogue.
//   ternary the 2-bit code of each element is moved to bits 15:14 of an f16 and
//           inverted, giving exactly 2*v; the factor 1/2 and the row scale are
//           applied in the epilogue.
// Activations enter as two f16 terms (hi = f16(x), lo = f16(x - hi)) of a
// per-token power-of-two normalised row, so the products reproduce fp32 to
// about 2^-22 relative; accumulation is fp32.  A slice of up to 4 tokens puts
// the hi terms in MMA columns 0-3 and the lo terms in columns 4-7 (one MMA per
// k-step; the epilogue adds column n and n+4); larger slices use columns 0-7
// for tokens and two MMAs per k-step.
//
// Column <-> MMA-k mapping.  NVFP4: chunk c = 128 columns; lane t of a quad
// owns columns [c*128 + 32t, +32) = 16 bytes of each row = 8 MMA k-steps; step
// j uses bytes 2j (k = 2t, 2t+1) and 2j+1 (k = 2t+8, 2t+9), i.e. columns
// 4j..4j+3, and the B fragment is the 4 consecutive activation halves at those
// columns.  Ternary: chunk = 256 columns; lane t owns [c*256 + 64t, +64) =
// 16 bytes = four 16-column words; step s of word q uses code pairs 2s and
// 2s+1 (columns {2s, 2s+8} and {2s+1, 2s+9}); activations are stored in "pair
// order" (column i at 2i, column i+8 at 2i+1 inside each 16 block) so the B
// fragment is again 4 consecutive halves.
#pragma once

#include "common.cuh"

namespace ffn {

#ifndef FFN_WARPS
#define FFN_WARPS 4
#endif
constexpr int kWarps = FFN_WARPS;
constexpr int kThreads = kWarps * 32;

// ------------------------------------------------------------ cp.async
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src));
}
template <int N>
__device__ __forceinline__ void cp_async_n(void *dst, const void *src) {
  static_assert(N == 4 || N == 8 || N == 16, "cp.async copies 4, 8 or 16 bytes");
  if constexpr (N == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src));
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(smem_u32(dst)), "l"(src), "n"(N));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

struct MatRef {          // one weight matrix as the tile engine sees it
  const uint8_t *w;      // NVFP4 packed / ternary packed
  const uint8_t *s;      // NVFP4 block scales (unused for ternary)
};

template <int FMT, int NMAT, int R, int STAGES, int SUB = 1>
struct WarpEngine {
  static constexpr int ROWS = 16 * R;
  static constexpr int MT = NMAT * R;                                   // m-tiles per unit
  static constexpr bool F8 = FMT == FFN_B200_FMT_MXFP8;                // one byte per weight
  // columns per sub-chunk: a lane holds 16 bytes of each of its rows
  static constexpr int CHUNK = FMT == FFN_B200_FMT_NVFP4 ? 128 : F8 ? 64 : 256;
  static constexpr int SUB_W = MT * 2 * 32 * 16;                        // weight bytes per sub-chunk
  static constexpr int UNIT_W = SUB * SUB_W;
  // scale bytes per row per unit: NVFP4 E4M3 per 16 columns; ternary U8 block
  // scales per 64 columns (copied only for matrices that have them)
  // (MXFP8: one E8M0 scale per 32 x 32 block -- 2 * SUB bytes per m-tile and
  // unit, 16 bytes reserved per m-tile)
  static constexpr int SR = FMT == FFN_B200_FMT_NVFP4 ? 8 * SUB : 4 * SUB;
  static constexpr int UNIT_S = F8 ? MT * 16 : MT * 16 * SR;
  static constexpr int UNIT = UNIT_W + UNIT_S;                          // [SUB weight blocks][scales]
  static constexpr int RING = STAGES * UNIT;                            // per warp
  static constexpr size_t SMEM = (size_t)kWarps * RING;

  static __device__ __forceinline__ int nchunks(int K) { return (K + CHUNK * SUB - 1) / (CHUNK * SUB); }
  // scale bytes per matrix row
  static __host__ __device__ __forceinline__ int sld_of(int K) {
    return FMT == FFN_B200_FMT_NVFP4 ? K / 16 : F8 ? (K + 31) / 32 : K / 64;
  }

  // Issue the copies of unit c (columns [c*CHUNK*SUB, +CHUNK*SUB)) of the task
  // whose rows start at row0 into `slot`.  Weights: per sub-chunk and m-tile,
  // lane (g, t) copies 16 bytes of rows g and g+8; lanes whose 16-byte column
  // slice lies past K copy nothing (the compute step treats their weights as
  // zero).  NVFP4 scales: SR bytes of each of the unit's 16*MT rows, one
  // SR-byte copy per row when every scale row is SR-byte aligned (s_al),
  // otherwise 4-byte copies.
  // mx: an MXFP4 task on the NVFP4 instance (E8M0 scales per 32 columns:
  // SR / 2 bytes per row and unit, stored at the start of the row's SR slot)
  __device__ static void issue(uint8_t *slot, const MatRef (&m)[NMAT], int rows, int K, int row0, int c,
                               bool s_al, bool mx = false) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    constexpr int LB = FMT == FFN_B200_FMT_NVFP4 ? 32 : F8 ? 16 : 64;  // columns per lane per sub-chunk
    constexpr int EPB = FMT == FFN_B200_FMT_NVFP4 ? 2 : F8 ? 1 : 4;     // elements per byte
    const size_t wld = (size_t)K / EPB;
#pragma unroll
    for (int sb = 0; sb < SUB; ++sb) {
      const int col0 = (c * SUB + sb) * CHUNK + LB * t;
      if (col0 < K) {
        const size_t boff = (size_t)col0 / EPB;
#pragma unroll
        for (int mi = 0; mi < NMAT; ++mi)
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const int mt = mi * R + i;
            const int ra = min(row0 + 16 * i + g, rows - 1), rb = min(row0 + 16 * i + g + 8, rows - 1);
            uint8_t *d = slot + sb * SUB_W + mt * 1024 + lane * 16;
            cp_async16(d, m[mi].w + ra * wld + boff);
            cp_async16(d + 512, m[mi].w + rb * wld + boff);
          }
      }
    }
    if constexpr (F8) {
      // lane mt copies the 2 * SUB block scales of m-tile mt (row block
      // (first row) / 32, block columns [2 SUB c, +2 SUB)); K % 128 keeps the
      // 4-byte copies aligned and inside the scale row
      const int scols = sld_of(K);
      if (lane < MT && c * 2 * SUB < scols) {
        const int mi = lane / R, i = lane % R;
        const int rblk = min(row0 + 16 * i, rows - 1) / 32;
        static_assert(2 * SUB == 4, "one 4-byte copy per m-tile");
        cp_async4(slot + UNIT_W + lane * 16, m[mi].s + (size_t)rblk * scols + c * 2 * SUB);
      }
      return;
    }
    bool any_s = FMT == FFN_B200_FMT_NVFP4;
#pragma unroll
    for (int mi = 0; mi < NMAT; ++mi) any_s = any_s || m[mi].s != nullptr;
    if (any_s && mx) {
      constexpr int SRM = SR / 2;
      const int sld = K / 32;
      uint8_t *sbase = slot + UNIT_W;
      constexpr int NROW = MT * 16;
      if (s_al) {
#pragma unroll
        for (int j = 0; j < (NROW + 31) / 32; ++j) {
          const int rr = lane + 32 * j;
          if (rr < NROW && c * SRM < sld) {
            const int mt = rr >> 4, mi = mt / R, i = mt % R;
            const int sr = min(row0 + 16 * i + (rr & 15), rows - 1);
            cp_async_n<SRM>(sbase + rr * SR, m[mi].s + (size_t)sr * sld + c * SRM);
          }
        }
      } else {
        constexpr int PIECES = NROW * SRM / 4;
#pragma unroll
        for (int j = 0; j < (PIECES + 31) / 32; ++j) {
          const int p = lane + 32 * j;
          if (p < PIECES) {
            const int rr = p / (SRM / 4), q = p % (SRM / 4);
            const int mt = rr >> 4, mi = mt / R, i = mt % R;
            const int sr = min(row0 + 16 * i + (rr & 15), rows - 1);
            const int sc = c * SRM + 4 * q;
            if (sc < sld) cp_async4(sbase + rr * SR + 4 * q, m[mi].s + (size_t)sr * sld + sc);
          }
        }
      }
    } else if (any_s) {  // ternary: only the matrices that have block scales are copied
      const int sld = sld_of(K);
      uint8_t *sbase = slot + UNIT_W;
      constexpr int NROW = MT * 16;
      if (s_al) {
        // one SR-byte copy per row
#pragma unroll
        for (int j = 0; j < (NROW + 31) / 32; ++j) {
          const int rr = lane + 32 * j;
          if (rr < NROW && c * SR < sld) {
            const int mt = rr >> 4, mi = mt / R, i = mt % R;
            const int sr = min(row0 + 16 * i + (rr & 15), rows - 1);
            if (m[mi].s) cp_async_n<SR>(sbase + rr * SR, m[mi].s + (size_t)sr * sld + c * SR);
          }
        }
      } else {
        constexpr int PIECES = NROW * SR / 4;  // 4-byte pieces per unit
#pragma unroll
        for (int j = 0; j < (PIECES + 31) / 32; ++j) {
          const int p = lane + 32 * j;
          if (p < PIECES) {
            const int rr = p / (SR / 4), q = p % (SR / 4);
            const int mt = rr >> 4, mi = mt / R, i = mt % R;
            const int sr = min(row0 + 16 * i + (rr & 15), rows - 1);
            const int sc = c * SR + 4 * q;
            if (sc < sld && m[mi].s) cp_async4(sbase + rr * SR + 4 * q, m[mi].s + (size_t)sr * sld + sc);
          }
        }
      }
    }
  }

  template <bool PACKED>
  __device__ static __forceinline__ void compute(const uint8_t *slot, int K, int c, const __half *xa,
                                                 const __half *xb, float (&acc)[NMAT][R][4],
                                                 uint32_t bs_mask = 0, uint32_t mxinfo = 0) {
    // One copy of the (large) unrolled sub-chunk body, so the warps'
    // instruction fetches stay in cache (ternary gate/up 8 % and down 12 %
    // faster, NVFP4 down 3 %, than with the sub-chunks unrolled).
#pragma unroll 1
    for (int sb = 0; sb < SUB; ++sb) compute_sub<PACKED>(slot, sb, K, c * SUB + sb, xa, xb, acc, bs_mask, mxinfo);
  }

  // Accumulate one sub-chunk c from `slot` into acc.  xa/xb: this lane's
  // B-column source rows (packed: xa = a token's hi or lo halves, xb unused;
  // otherwise xa = hi, xb = lo), or xa == nullptr for an empty column.  The
  // unit's shared-memory weight words are read first; activation words are
  // read from global memory (L1-resident: the warps of a slice share them)
  // next to the k-steps that use them.
  template <bool PACKED>
  __device__ static void compute_sub(const uint8_t *unit, int sb, int K, int c, const __half *xa,
                                     const __half *xb, float (&acc)[NMAT][R][4], uint32_t bs_mask,
                                     uint32_t mxinfo) {
    const uint8_t *slot = unit + sb * SUB_W;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int col0 = c * CHUNK + (FMT == FFN_B200_FMT_NVFP4 ? 32 : F8 ? 16 : 64) * t;
    const bool valid = col0 < K;
    // activation words are loaded one 16-byte word at a time (hi and lo),
    // next to their use, which keeps the live registers at ~80 per thread
    const bool xv = valid && xa;
    auto xload = [&](const __half *src, int v) {
      return xv ? ldg_cached(src + col0 + 8 * v) : make_uint4(0u, 0u, 0u, 0u);
    };
    uint4 wq[MT][2];
    const uint4 zero = FMT == FFN_B200_FMT_NVFP4 ? make_uint4(0u, 0u, 0u, 0u)
                                                 : make_uint4(0x55555555u, 0x55555555u,
                                                              0x55555555u, 0x55555555u);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        wq[mt][h] = valid ? *reinterpret_cast<const uint4 *>(slot + mt * 1024 + h * 512 + lane * 16)
                          : zero;  // code 1 (ternary) / E2M1 0 (NVFP4) decode to zero
    if constexpr (F8) {
      // MXFP8: lane t's 16 columns lie in block column (4 sub-chunk + t) / 2;
      // rows g and g+8 share the m-tile's row block, so one scale per m-tile
      uint32_t sf[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int bias = (int)((mxinfo >> (8 * (mt / R))) & 0xFFu) - 128;
        sf[mt] = valid ? e8m0_f16x2(unit[UNIT_W + mt * 16 + 2 * sb + (t >> 1)], bias) : 0u;
      }
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        // activation word v = columns col0 + 8v .. +7 = k-steps 2v, 2v+1
        const uint4 xh = xload(xa, v);
        const uint4 xl = PACKED ? make_uint4(0u, 0u, 0u, 0u) : xload(xb, v);
        const uint32_t bh[4] = {xh.x, xh.y, xh.z, xh.w};
        const uint32_t bl[4] = {xl.x, xl.y, xl.z, xl.w};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = 2 * v + h;  // weight word j = columns col0 + 4j .. +3
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int mi = mt / R, i = mt % R;
            const uint32_t wa = j == 0 ? wq[mt][0].x : j == 1 ? wq[mt][0].y : j == 2 ? wq[mt][0].z : wq[mt][0].w;
            const uint32_t wb = j == 0 ? wq[mt][1].x : j == 1 ? wq[mt][1].y : j == 2 ? wq[mt][1].z : wq[mt][1].w;
            const uint32_t a0 = hmul2_u32(e4m3x2_to_f16x2((uint16_t)(wa & 0xFFFFu)), sf[mt]);
            const uint32_t a1 = hmul2_u32(e4m3x2_to_f16x2((uint16_t)(wb & 0xFFFFu)), sf[mt]);
            const uint32_t a2 = hmul2_u32(e4m3x2_to_f16x2((uint16_t)(wa >> 16)), sf[mt]);
            const uint32_t a3 = hmul2_u32(e4m3x2_to_f16x2((uint16_t)(wb >> 16)), sf[mt]);
            mma_f16(acc[mi][i], a0, a1, a2, a3, bh[2 * h], bh[2 * h + 1]);
            if (!PACKED) mma_f16(acc[mi][i], a0, a1, a2, a3, bl[2 * h], bl[2 * h + 1]);
          }
        }
      }
    } else if constexpr (FMT == FFN_B200_FMT_NVFP4) {
      uint32_t sfa[MT], sfb[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        // lanes past K read no scale bytes (they may be stale: an E4M3 NaN there
        // would turn the zero weights into NaN)
        if (mxinfo >> 31) {
          // MXFP4: the lane's 32 columns are one E8M0 block (block t of the
          // sub-chunk); both halves carry it, so the word's lo/hi broadcasts agree
          const uint8_t *sp = unit + UNIT_W + mt * 16 * SR + 4 * sb + t;
          const int bias = (int)((mxinfo >> (8 * (mt / R))) & 0xFFu) - 128;
          sfa[mt] = valid ? e8m0_f16x2(sp[g * SR], bias) : 0u;
          sfb[mt] = valid ? e8m0_f16x2(sp[(g + 8) * SR], bias) : 0u;
        } else {
          const uint8_t *sp = unit + UNIT_W + mt * 16 * SR + 8 * sb + 2 * t;
          sfa[mt] = valid ? e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t *>(sp + g * SR)) : 0u;
          sfb[mt] = valid ? e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t *>(sp + (g + 8) * SR)) : 0u;
        }
      }
      uint4 xhs[4], xls[4];
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
        xhs[wd] = xload(xa, wd);
        xls[wd] = PACKED ? make_uint4(0u, 0u, 0u, 0u) : xload(xb, wd);
      }
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
        const uint4 xh = xhs[wd];
        const uint4 xl = xls[wd];
        const uint32_t bh[4] = {xh.x, xh.y, xh.z, xh.w};
        const uint32_t bl[4] = {xl.x, xl.y, xl.z, xl.w};
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int mi = mt / R, i = mt % R;
          const uint32_t s_a = wd < 2 ? bcast_lo(sfa[mt]) : bcast_hi(sfa[mt]);
          const uint32_t s_b = wd < 2 ? bcast_lo(sfb[mt]) : bcast_hi(sfb[mt]);
          const uint32_t wa = wd == 0 ? wq[mt][0].x : wd == 1 ? wq[mt][0].y : wd == 2 ? wq[mt][0].z : wq[mt][0].w;
          const uint32_t wb = wd == 0 ? wq[mt][1].x : wd == 1 ? wq[mt][1].y : wd == 2 ? wq[mt][1].z : wq[mt][1].w;
          uint32_t da[4], db[4];
          e2m1x8_to_f16x2(wa, da);
          e2m1x8_to_f16x2(wb, db);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t a0 = hmul2_u32(da[2 * h], s_a);
            const uint32_t a1 = hmul2_u32(db[2 * h], s_b);
            const uint32_t a2 = hmul2_u32(da[2 * h + 1], s_a);
            const uint32_t a3 = hmul2_u32(db[2 * h + 1], s_b);
            mma_f16(acc[mi][i], a0, a1, a2, a3, bh[2 * h], bh[2 * h + 1]);
            if (!PACKED) mma_f16(acc[mi][i], a0, a1, a2, a3, bl[2 * h], bl[2 * h + 1]);
          }
        }
      }
    } else {
      // block scales: lane t's 64 columns of this sub-chunk are one block
      // (rows g and g+8 of every m-tile); 1 (f16 0x3C00) without block scales
      uint32_t sba[MT], sbb[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        sba[mt] = sbb[mt] = 0x3C003C00u;
        if ((bs_mask >> (mt / R)) & 1u) {
          const uint8_t *sp = unit + UNIT_W + mt * 16 * SR + 4 * sb + t;
          const __half ha = __ushort2half_rn(sp[g * SR]), hb = __ushort2half_rn(sp[(g + 8) * SR]);
          sba[mt] = (uint32_t)__half_as_ushort(ha) * 0x10001u;
          sbb[mt] = (uint32_t)__half_as_ushort(hb) * 0x10001u;
        }
      }
      // activation halves of ternary word q: 8 consecutive pair-order values
      // of the hi row (and of the lo row unless PACKED)
      auto txload = [&](int q, uint32_t(&bh)[8], uint32_t(&bl)[8]) {
        const uint4 h0 = xload(xa, 2 * q), h1 = xload(xa, 2 * q + 1);
        const uint4 l0 = PACKED ? make_uint4(0u, 0u, 0u, 0u) : xload(xb, 2 * q);
        const uint4 l1 = PACKED ? make_uint4(0u, 0u, 0u, 0u) : xload(xb, 2 * q + 1);
        bh[0] = h0.x; bh[1] = h0.y; bh[2] = h0.z; bh[3] = h0.w;
        bh[4] = h1.x; bh[5] = h1.y; bh[6] = h1.z; bh[7] = h1.w;
        bl[0] = l0.x; bl[1] = l0.y; bl[2] = l0.z; bl[3] = l0.w;
        bl[4] = l1.x; bl[5] = l1.y; bl[6] = l1.z; bl[7] = l1.w;
      };
      // One unrolled loop per case, chosen once per sub-chunk (warp-uniform):
      // no block scales, or block scales (a matrix without them multiplies
      // by 1.0, exact).  Choosing per m-tile inside the loop interleaves both
      // unrolled bodies in the instruction stream, and the warps then stall
      // on instruction fetch.
      if (bs_mask == 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t bh[8], bl[8];
          txload(q, bh, bl);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            tern_steps<PACKED>(acc[mt / R][mt % R], tern_word(wq[mt][0], q), tern_word(wq[mt][1], q), bh, bl);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t bh[8], bl[8];
          txload(q, bh, bl);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            tern_steps_scaled<PACKED>(acc[mt / R][mt % R], tern_word(wq[mt][0], q), tern_word(wq[mt][1], q),
                                      sba[mt], sbb[mt], bh, bl);
        }
      }
    }
  }

  __device__ static __forceinline__ uint32_t tern_word(const uint4 &w, int q) {
    return q == 0 ? w.x : q == 1 ? w.y : q == 2 ? w.z : w.w;
  }

  // Four MMA k-steps of one 16-column ternary word (rows g and g+8).
  template <bool PACKED>
  __device__ static __forceinline__ void tern_steps(float (&d)[4], uint32_t xa, uint32_t xb,
                                                    const uint32_t (&bh)[8],
                                                    const uint32_t (&bl)[8]) {
#define FFN_TSTEP(S)                                                                  \
  {                                                                                   \
    const uint32_t a0 = tern_pair<2 * S>(xa), a1 = tern_pair<2 * S>(xb);              \
    const uint32_t a2 = tern_pair<2 * S + 1>(xa), a3 = tern_pair<2 * S + 1>(xb);      \
    mma_f16(d, a0, a1, a2, a3, bh[2 * S], bh[2 * S + 1]);                             \
    if (!PACKED) mma_f16(d, a0, a1, a2, a3, bl[2 * S], bl[2 * S + 1]);                \
  }
    FFN_TSTEP(0) FFN_TSTEP(1) FFN_TSTEP(2) FFN_TSTEP(3)
#undef FFN_TSTEP
  }

  // The same with the rows' U8 block scales (f16x2 broadcasts sa: row g,
  // sb: row g+8) folded into A: 2 * L * scale <= 510 is exact in f16.
  template <bool PACKED>
  __device__ static __forceinline__ void tern_steps_scaled(float (&d)[4], uint32_t xa, uint32_t xb,
                                                           uint32_t sa, uint32_t sb,
                                                           const uint32_t (&bh)[8],
                                                           const uint32_t (&bl)[8]) {
#define FFN_TSTEP(S)                                                                  \
  {                                                                                   \
    const uint32_t a0 = hmul2_u32(tern_pair<2 * S>(xa), sa);                          \
    const uint32_t a1 = hmul2_u32(tern_pair<2 * S>(xb), sb);                          \
    const uint32_t a2 = hmul2_u32(tern_pair<2 * S + 1>(xa), sa);                      \
    const uint32_t a3 = hmul2_u32(tern_pair<2 * S + 1>(xb), sb);                      \
    mma_f16(d, a0, a1, a2, a3, bh[2 * S], bh[2 * S + 1]);                             \
    if (!PACKED) mma_f16(d, a0, a1, a2, a3, bl[2 * S], bl[2 * S + 1]);                \
  }
    FFN_TSTEP(0) FFN_TSTEP(1) FFN_TSTEP(2) FFN_TSTEP(3)
#undef FFN_TSTEP
  }
};

}  // namespace ffn
