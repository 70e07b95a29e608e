// common.cuh -- device helpers shared by the expert-FFN kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "ffn_b200.h"

namespace ffn {

// ---------------------------------------------------------------- status
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what);
void note_launch(uint64_t n = 1);

#define FFN_CUDA_TRY(expr)                                     \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return ::ffn::cuda_fail(_e, #expr); \
  } while (0)

// Event-pair timing of one launch (no-ops unless ffn_b200_profile_enable(1)).
void prof_begin(int kind, cudaStream_t st);
void prof_end(int kind, cudaStream_t st);

// Launch the kernel<<<...>>> expression given as the trailing arguments on
// stream `st`, timed under `kind`, and return the launch error if any.
#define FFN_LAUNCH(kind, st, name, ...)                             \
  do {                                                              \
    ::ffn::prof_begin(kind, st);                                    \
    __VA_ARGS__;                                                    \
    ::ffn::prof_end(kind, st);                                      \
    ::ffn::note_launch();                                           \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) return ::ffn::cuda_fail(_e, name);       \
  } while (0)

// Programmatic dependent launch.  The kernels of the MoE layer chain
// (xprep, router, top-k, grouping, the expert phases, combine) are launched
// with cudaLaunchAttributeProgrammaticStreamSerialization, so a kernel's CTAs
// may be scheduled while the previous kernel in the stream drains; each such
// kernel calls pdl_enter() before it reads anything an earlier kernel wrote.
// griddepcontrol.wait returns once the previous grid has completed and its
// memory is visible (immediately when the launch had no such dependency);
// launch_dependents then lets the next kernel be scheduled early in turn.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
bool pdl_allowed();  // false when FFN_B200_NO_PDL is set in the environment

template <typename... P, typename... A>
inline cudaError_t launch_pdl(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              A &&...args) {
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = pdl_allowed() ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...);
}

// FFN_LAUNCH for a kernel that calls pdl_enter(): kern (parenthesised if it
// has template arguments), grid, block, dynamic shared memory, then the
// kernel's arguments.
#define FFN_LAUNCH_PDL(kind, st, name, kern, grid, block, smem, ...)          \
  do {                                                                        \
    ::ffn::prof_begin(kind, st);                                              \
    cudaError_t _l = ::ffn::launch_pdl(kern, grid, block, smem, st, __VA_ARGS__); \
    ::ffn::prof_end(kind, st);                                                \
    ::ffn::note_launch();                                                     \
    cudaError_t _e = cudaGetLastError();                                      \
    if (_l != cudaSuccess) _e = _l;                                           \
    if (_e != cudaSuccess) return ::ffn::cuda_fail(_e, name);                 \
  } while (0)

constexpr int kTopKMax = 16;   // router top_k upper bound
constexpr int kNTok = 8;       // tokens per MMA column group (mma n = 8)

// One slice of tokens of one expert: pairs [offset, offset + count), count <= 8.
struct VExp {
  int32_t expert;
  int32_t offset;
  int32_t count;
  int32_t pad;
};

// ------------------------------------------------------------ decoders
// An E8M0 block scale 2^(e - 127) (flash1017.rs:1049-1057) divided by the
// matrix's power-of-two post-scale 2^bias, as an f16 pair: exact for
// -24 <= e - 127 - bias <= 15 (subnormal below -14), 0 further down, +inf
// above; e = 0xFF -> NaN.  Times an E2M1 value (0.5 .. 6, 2 significant bits)
// the product is exact in f16 while -23 <= e - 127 - bias <= 13.
__device__ __forceinline__ uint32_t e8m0_f16x2(uint32_t e, int bias) {
  const int k = (int)e - 127 - bias;
  uint32_t h;
  if (e == 0xFFu) h = 0x7E00u;
  else if (k > 15) h = 0x7C00u;
  else if (k >= -14) h = (uint32_t)(k + 15) << 10;
  else if (k >= -24) h = 1u << (k + 24);
  else h = 0u;
  return h * 0x10001u;
}

// Four E2M1 pairs of a 32-bit word (byte b: low nibble = even column) -> four
// f16x2 {even, odd}; exact.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

// Two E4M3 bytes (low byte = element 0) -> f16x2 (exact: every E4M3 value is an f16).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t two) {
  uint32_t out;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(two));
  return out;
}

// Reference decoders written as scalar functions (flash1017.rs:17-20, 1031-1045);
// used by the decode-check kernels.
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  uint32_t sign = (b & 0x80u) << 24;
  uint32_t em = b & 0x7Fu;
  if (em == 0x7Fu) return __int_as_float(0x7FC00000);
  if (em < 8u) return __int_as_float(sign | __float_as_uint((float)em * (1.0f / 512.0f)));
  return __int_as_float(sign | ((em + 960u) << 20));
}

__device__ __forceinline__ float e2m1_to_f32(uint32_t n) {
  // magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 in units of 0.5: 0,1,2,3,4,6,8,12
  const uint32_t m = n & 7u;
  const uint32_t halves = m < 4u ? m : (m == 4u ? 4u : (m == 5u ? 6u : (m == 6u ? 8u : 12u)));
  const float v = (float)halves * 0.5f;
  return (n & 8u) ? -v : v;
}

__device__ __forceinline__ float tern_to_f32(uint32_t code) {
  return code == 0u ? -1.0f : (code == 2u ? 1.0f : 0.0f);
}

// Ternary pair decode: word w holds 16 codes (element i at bits 2i..2i+1).
// Returns f16x2 {2*v(elem I), 2*v(elem I+8)}: bits 15:14 of each half are the
// inverted code bits, which gives 0xC000 (-2) for code 0, 0x4000 (+2) for code
// 2 and +-0 for codes 1 and 3.
template <int I>
__device__ __forceinline__ uint32_t tern_pair(uint32_t w) {
  return ~(w << (14 - 2 * I)) & 0xC000C000u;
}

// ---------------------------------------------------------- tensor cores
// D += A(16x16 f16, row) * B(16x8 f16, col), f32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}

// Broadcast the low / high half of an f16x2 into both halves.
__device__ __forceinline__ uint32_t bcast_lo(uint32_t v) { return __byte_perm(v, v, 0x1010); }
__device__ __forceinline__ uint32_t bcast_hi(uint32_t v) { return __byte_perm(v, v, 0x3232); }

// --------------------------------------------------------------- loads
__device__ __forceinline__ uint4 ldg_stream(const void *p) {  // weights: read once
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg_cached(const void *p) {  // activations: reused
  return __ldg(reinterpret_cast<const uint4 *>(p));
}

// x -> (hi, lo) f16 split: hi = f16(x), lo = f16(x - hi).
__device__ __forceinline__ void split_f16(float x, __half &hi, __half &lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

// Position of column c inside the "pair order" used for ternary consumers:
// within each 16-column block, column i (< 8) sits at 2i and column i+8 at 2i+1.
__device__ __forceinline__ int tern_pos(int c) {
  const int b = c & ~15, i = c & 15;
  return b + (i < 8 ? 2 * i : 2 * (i - 8) + 1);
}

__device__ __forceinline__ float pow2f(int e) {  // exact 2^e for |e| < 127
  return __int_as_float((uint32_t)(e + 127) << 23);
}

}  // namespace ffn
