// compress.cu -- the 106 GB format's compressor on the GPU: one NVFP4 matrix
// -> 1.58-bit ternary codes with U8 block-64 scales and per-row scales, plus
// the rank-16 Q8 core fitted to the quantisation residual.
//
// The reference runs this on the CPU (compress_nvfp4_matrix_to_158_jepa_q8,
// crates/flash-core/src/flash1017.rs:10377-10645, orthonormalize_cols_16
// :10342-10372) when it writes the 106 GB shards (:10700-10811).  Steps:
//   1. tern_b64_kernel, one CTA per row: dequantise (E2M1 x E4M3 x gs), per
//      64-column block the RMS, four candidate thresholds (0.42..0.78 x RMS),
//      the one maximising (w.t)^2 / |t| gives gamma and the codes; the row scale
//      is max gamma / 255, block scales round(gamma / row scale); the residual
//      R = W - code x block scale x row scale stays in the workspace;
//   2. randomised subspace iteration of rank 16 on R, two sweeps: p (cols x 16)
//      from the reference's splitmix-style generator, q = R p, z = R^T q, with
//      Gram-Schmidt (orthonormalize16_kernel) after each product as the
//      reference does;
//   3. q and z quantised per column to int8 with max|.| / 127 scales
//      (core_b = q, core_a = z^T).
// Every f32 operation is rounded separately (__fmul_rn / __fadd_rn, no FMA
// contraction) and every sum runs in the reference's order (the 64 values of a
// block, R p over the columns of a row, R^T q over the rows of a column, one thread
// per output element), so
// codes, scales and the residual are bit-exact.  The Gram-Schmidt dots and
// norms are f64 sums rounded to f32 as in the reference; here they are summed
// in a fixed tree order, which rounds to the same f32 value except in rare
// last-bit cases.
#include <algorithm>

#include "ffn_internal.h"

namespace ffn {
namespace {

constexpr int kTernThreads = 256;

// Column c of a row: E2M1 value x (E4M3 group scale x gs), flash1017.rs:10412-10416.
__device__ __forceinline__ float nvfp4_at(const uint8_t *wr, const uint8_t *sr, float gs, int c) {
  const uint32_t b = wr[c >> 1];
  const uint32_t nib = (c & 1) ? (b >> 4) : (b & 15u);
  return __fmul_rn(e2m1_to_f32(nib), __fmul_rn(e4m3_to_f32(sr[c >> 4]), gs));
}

__device__ __forceinline__ float lut3(uint32_t code) {  // [-1, 0, +1, 0]
  return code == 0u ? -1.0f : (code == 2u ? 1.0f : 0.0f);
}

// One CTA per row; thread t owns the 64-column blocks t, t + 256, ...
__global__ void __launch_bounds__(kTernThreads) tern_b64_kernel(int cols, const uint8_t *__restrict__ w,
                                                                const uint8_t *__restrict__ s, float gs,
                                                                uint8_t *packed, float *row_scales,
                                                                uint8_t *block_scales, float *res) {
  extern __shared__ float s_gamma[];  // [nblk]
  __shared__ float s_max[kTernThreads / 32];
  const int r = blockIdx.x, nblk = cols / 64, tid = threadIdx.x;
  const uint8_t *wr = w + (size_t)r * (cols / 2), *sr = s + (size_t)r * (cols / 16);
  uint8_t *pr = packed + (size_t)r * (cols / 4);
  float my_max = 0.0f;
  for (int blk = tid; blk < nblk; blk += kTernThreads) {
    float v[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = nvfp4_at(wr, sr, gs, blk * 64 + i);
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < 64; ++i) sq = __fadd_rn(sq, __fmul_rn(v[i], v[i]));
    const float rms = sqrtf(__fmul_rn(sq, 1.0f / 64.0f));
    uint32_t words[4] = {0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u};
    float gamma = 0.0f;
    if (!(rms <= 1e-12f)) {
      const float F[4] = {0.42f, 0.54f, 0.66f, 0.78f};
      float best_score = -1.0f, best_th = __fmul_rn(0.58f, rms);
#pragma unroll
      for (int f = 0; f < 4; ++f) {
        const float th = __fmul_rn(F[f], rms);
        float dot = 0.0f;
        uint32_t cnt = 0;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          if (v[i] > th) {
            dot = __fadd_rn(dot, v[i]);
            ++cnt;
          } else if (v[i] < -th) {
            dot = __fsub_rn(dot, v[i]);
            ++cnt;
          }
        }
        if (cnt > 0) {
          const float score = __fdiv_rn(__fmul_rn(dot, dot), (float)cnt);
          if (score > best_score) {
            best_score = score;
            gamma = __fdiv_rn(dot, (float)cnt);
            best_th = th;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t wd = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x = v[q * 16 + i];
          const uint32_t code = x > best_th ? 2u : (x < -best_th ? 0u : 1u);
          wd |= code << (2 * i);
        }
        words[q] = wd;
      }
      my_max = fmaxf(my_max, gamma);  // gamma >= 0
    }
    uint32_t *pw = reinterpret_cast<uint32_t *>(pr + (size_t)blk * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) pw[q] = words[q];
    s_gamma[blk] = gamma;
  }
  // max over the row's blocks (order-free), flash1017.rs:10470-10472
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) my_max = fmaxf(my_max, __shfl_xor_sync(0xffffffffu, my_max, o));
  if ((tid & 31) == 0) s_max[tid >> 5] = my_max;
  __syncthreads();
  float max_gamma = 0.0f;
#pragma unroll
  for (int i = 0; i < kTernThreads / 32; ++i) max_gamma = fmaxf(max_gamma, s_max[i]);
  const float row_sc = max_gamma > 1e-12f ? __fdiv_rn(max_gamma, 255.0f) : 0.0f;
  if (tid == 0) row_scales[r] = row_sc;
  float *rr = res + (size_t)r * cols;
  for (int blk = tid; blk < nblk; blk += kTernThreads) {
    uint8_t u8 = 0;
    if (row_sc > 0.0f) u8 = (uint8_t)fminf(fmaxf(roundf(__fdiv_rn(s_gamma[blk], row_sc)), 0.0f), 255.0f);
    block_scales[(size_t)r * nblk + blk] = u8;
    const float qg = __fmul_rn((float)u8, row_sc);
    const uint32_t *pw = reinterpret_cast<const uint32_t *>(pr + (size_t)blk * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t wd = pw[q];  // written by this thread above
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int c = blk * 64 + q * 16 + i;
        rr[c] = __fsub_rn(nvfp4_at(wr, sr, gs, c), __fmul_rn(lut3((wd >> (2 * i)) & 3u), qg));
      }
    }
  }
}

// p[c][k] = the reference generator's (16 c + k + 1)-th draw, flash1017.rs:10527-10537.
__global__ void rsi_init_kernel(int n, uint64_t seed, float *p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * 16) return;
  constexpr uint64_t kG = 0x9E3779B97F4A7C15ull;
  uint64_t x = (seed ^ kG) + (uint64_t)(i + 1) * kG;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x ^= x >> 31;
  p[i] = __fmul_rn((float)((int32_t)(x >> 40) - (1 << 23)), 1.0f / 8388608.0f);
}

// Block-wide f64 sum in a fixed order (lanes, then warps).
__device__ double block_sum(double v, double *s_red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) s_red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int i = 0; i < nw; ++i) t += s_red[i];
  return t;
}

// Gram-Schmidt on the 16 columns of m [n][16], flash1017.rs:10342-10372.
__global__ void __launch_bounds__(1024) orthonormalize16_kernel(float *m, int n) {
  __shared__ double s_red[32];
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int k = 0; k < 16; ++k) {
    for (int j = 0; j < k; ++j) {
      double part = 0.0;
      for (int r = tid; r < n; r += nt) part += (double)m[r * 16 + k] * (double)m[r * 16 + j];
      const float d = (float)block_sum(part, s_red);
      for (int r = tid; r < n; r += nt) m[r * 16 + k] = __fsub_rn(m[r * 16 + k], __fmul_rn(d, m[r * 16 + j]));
      __syncthreads();
    }
    double part = 0.0;
    for (int r = tid; r < n; r += nt) {
      const double v = (double)m[r * 16 + k];
      part += v * v;
    }
    const double norm_sq = block_sum(part, s_red);
    const float inv = norm_sq > 1e-24 ? (float)(1.0 / sqrt(norm_sq)) : 0.0f;
    for (int r = tid; r < n; r += nt) m[r * 16 + k] = __fmul_rn(m[r * 16 + k], inv);
    __syncthreads();
  }
}

// q[r][k] = sum over c (in order) of R[r][c] p[c][k]; one thread per (row, k),
// so each sum keeps the reference's order and 16x as many threads hide the
// load latency.
__global__ void __launch_bounds__(256) rsi_rp_kernel(int rows, int cols, const float *__restrict__ R,
                                                     const float *__restrict__ p, float *q) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long long)rows * 16) return;
  const int r = (int)(t >> 4), k = (int)(t & 15);
  const float4 *row = reinterpret_cast<const float4 *>(R + (size_t)r * cols);
  const float *pk = p + k;
  float acc = 0.0f;
#pragma unroll 4
  for (int c4 = 0; c4 < cols / 4; ++c4) {
    const float4 v4 = __ldg(row + c4);
    const float *pc = pk + (size_t)c4 * 64;
    acc = __fadd_rn(acc, __fmul_rn(v4.x, __ldg(pc)));
    acc = __fadd_rn(acc, __fmul_rn(v4.y, __ldg(pc + 16)));
    acc = __fadd_rn(acc, __fmul_rn(v4.z, __ldg(pc + 32)));
    acc = __fadd_rn(acc, __fmul_rn(v4.w, __ldg(pc + 48)));
  }
  q[(size_t)r * 16 + k] = acc;
}

// z[c][k] = sum over r (in order) of R[r][c] q[r][k]; one thread per (column, k).
__global__ void __launch_bounds__(256) rsi_rtq_kernel(int rows, int cols, const float *__restrict__ R,
                                                      const float *__restrict__ q, float *z) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long long)cols * 16) return;
  const int c = (int)(t >> 4), k = (int)(t & 15);
  const float *col = R + c;
  const float *qk = q + k;
  float acc = 0.0f;
#pragma unroll 8
  for (int r = 0; r < rows; ++r)
    acc = __fadd_rn(acc, __fmul_rn(__ldg(col + (size_t)r * cols), __ldg(qk + (size_t)r * 16)));
  z[(size_t)c * 16 + k] = acc;
}

// Column k of m [n][16] -> int8 with scale max|.| / 127 (flash1017.rs:10583-10628);
// out[i * istride + k * kstride].  One CTA per column.
__global__ void __launch_bounds__(1024) quant_q8_kernel(const float *m, int n, int8_t *out, size_t istride,
                                                        size_t kstride, float *scale) {
  __shared__ float s_red[32];
  const int k = blockIdx.x, tid = threadIdx.x;
  float mx = 0.0f;
  for (int i = tid; i < n; i += blockDim.x) mx = fmaxf(mx, fabsf(m[(size_t)i * 16 + k]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) s_red[tid >> 5] = mx;
  __syncthreads();
  mx = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, s_red[i]);
  const float sc = mx > 1e-12f ? __fdiv_rn(mx, 127.0f) : 0.0f;
  if (tid == 0) scale[k] = sc;
  const float inv = sc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
  for (int i = tid; i < n; i += blockDim.x) {
    float qv = 0.0f;
    if (sc > 0.0f) qv = fminf(fmaxf(roundf(__fmul_rn(m[(size_t)i * 16 + k], inv)), -127.0f), 127.0f);
    out[(size_t)i * istride + (size_t)k * kstride] = (int8_t)qv;
  }
}

struct CompressWs {
  float *res, *p, *q, *z;
};
CompressWs carve_compress(void *ws, size_t rows, size_t cols, size_t *bytes) {
  size_t off = 0;
  auto take = [&](size_t n) {
    const size_t at = off;
    off = (off + n * sizeof(float) + 255) & ~(size_t)255;
    return at;
  };
  const size_t o_res = take(rows * cols), o_p = take(cols * 16), o_q = take(rows * 16), o_z = take(cols * 16);
  *bytes = off;
  char *b = (char *)ws;
  return CompressWs{(float *)(b + o_res), (float *)(b + o_p), (float *)(b + o_q), (float *)(b + o_z)};
}

}  // namespace
}  // namespace ffn

using namespace ffn;

extern "C" {

size_t ffn_b200_compress_ws_bytes(size_t rows, size_t cols) {
  size_t bytes = 0;
  carve_compress(nullptr, rows, cols, &bytes);
  return bytes + 256;
}

int ffn_b200_compress_ternary_b64(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s, float gs,
                                  uint64_t seed, uint8_t *packed, float *row_scales, uint8_t *block_scales,
                                  int8_t *core_b, float *core_b_sc, int8_t *core_a, float *core_a_sc, void *ws,
                                  size_t ws_bytes, void *stream) {
  if (rows == 0 || cols == 0 || cols % 64)
    return fail(FFN_B200_EINVAL, "compress_ternary_b64: rows > 0 and cols a positive multiple of 64");
  if (rows > (1u << 24) || cols > (1u << 18))  // cols / 64 block gammas in shared memory (<= 16 KB)
    return fail(FFN_B200_EINVAL, "compress_ternary_b64: rows <= 2^24 and cols <= 2^18");
  if (!w || !s || !packed || !row_scales || !block_scales || !core_b || !core_b_sc || !core_a || !core_a_sc)
    return fail(FFN_B200_EINVAL, "compress_ternary_b64: null pointer");
  if (((uintptr_t)packed & 15) || (cols / 2) % 4)
    return fail(FFN_B200_EINVAL, "compress_ternary_b64: packed must be 16-byte aligned");
  if (!ws || ws_bytes < ffn_b200_compress_ws_bytes(rows, cols))
    return fail(FFN_B200_ENOSPC, "compress_ternary_b64: workspace too small (see ffn_b200_compress_ws_bytes)");
  size_t used = 0;
  char *base = (char *)(((uintptr_t)ws + 255) & ~(uintptr_t)255);
  CompressWs c = carve_compress(base, rows, cols, &used);
  cudaStream_t st = (cudaStream_t)stream;
  const int R = (int)rows, Cn = (int)cols, nblk = Cn / 64;
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "tern_b64_kernel",
             tern_b64_kernel<<<R, kTernThreads, (size_t)nblk * sizeof(float), st>>>(
                 Cn, w, s, gs, packed, row_scales, block_scales, c.res));
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "rsi_init_kernel",
             rsi_init_kernel<<<(Cn * 16 + 255) / 256, 256, 0, st>>>(Cn, seed, c.p));
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "orthonormalize16_kernel", orthonormalize16_kernel<<<1, 1024, 0, st>>>(c.p, Cn));
  float *p = c.p, *z = c.z;
  for (int sweep = 0; sweep < 2; ++sweep) {
    FFN_LAUNCH(FFN_B200_K_OTHER, st, "rsi_rp_kernel",
               rsi_rp_kernel<<<(R * 16 + 255) / 256, 256, 0, st>>>(R, Cn, c.res, p, c.q));
    FFN_LAUNCH(FFN_B200_K_OTHER, st, "orthonormalize16_kernel",
               orthonormalize16_kernel<<<1, 1024, 0, st>>>(c.q, R));
    FFN_LAUNCH(FFN_B200_K_OTHER, st, "rsi_rtq_kernel",
               rsi_rtq_kernel<<<(Cn * 16 + 255) / 256, 256, 0, st>>>(R, Cn, c.res, c.q, z));
    if (sweep == 0) {  // p <- z, orthonormalised; the old p buffer takes the next z
      std::swap(p, z);
      FFN_LAUNCH(FFN_B200_K_OTHER, st, "orthonormalize16_kernel",
                 orthonormalize16_kernel<<<1, 1024, 0, st>>>(p, Cn));
    }
  }
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "quant_q8_kernel",
             quant_q8_kernel<<<16, 1024, 0, st>>>(c.q, R, core_b, 16, 1, core_b_sc));
  FFN_LAUNCH(FFN_B200_K_OTHER, st, "quant_q8_kernel",
             quant_q8_kernel<<<16, 1024, 0, st>>>(z, Cn, core_a, 1, cols, core_a_sc));
  return 0;
}

}  // extern "C"
