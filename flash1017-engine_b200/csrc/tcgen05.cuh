// tcgen05.cuh -- sm_100a tensor-memory / mbarrier helpers used by the
// block-scaled FP4 kernels (fp4_gemm.cu).
//
// Conventions (PTX ISA, tcgen05 family):
//   * shared-memory matrix descriptors: start address >> 4 in bits 0-13,
//     leading-dimension byte offset >> 4 in 16-29, stride byte offset >> 4 in
//     32-45, bit 46 set (descriptor version of sm_100), layout type in 61-63
//     (0 = no swizzle, 2 = 128-byte swizzle);
//   * K-major tiles with 128-byte swizzle: rows of 128 bytes, 8-row groups of
//     1024 bytes, 16-byte piece c of row r stored at piece c ^ (r % 8); a
//     K-step of 64 FP4 values is 32 bytes, so the descriptor of step j starts
//     32 j bytes into the tile;
//   * block-scale factors: one 512-byte atom per 128 rows and K-step
//     (line m0 = 16 bytes = the 4 scales of rows m0, m0 + 32, m0 + 64, m0 + 96),
//     copied to TMEM with tcgen05.cp .32x128b.warpx4 (every 32-lane quarter
//     receives the 32 lines; the atom fills 4 columns).
// Every mbarrier wait is bounded: a wait that runs out sets *err and returns
// false, and the caller drains and leaves.
#pragma once

#include "common.cuh"

namespace ffn {
namespace tc {

constexpr long long kSpinLimit = 1LL << 22;  // try_wait polls per wait before giving up

__device__ __forceinline__ uint32_t sa(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// byte offset of 16-byte piece kc of row r in a 128-byte-swizzled K-major tile
__device__ __forceinline__ uint32_t sw128(int r, int kc) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((kc ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// a scale-factor atom: 32 rows of 16 bytes, contiguous (8-row core matrices 128 bytes apart)
__device__ __forceinline__ uint64_t desc_sf(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) |
         ((uint64_t)1 << 46);
}
// kind::mxf4nvf4 instruction descriptor: A and B E2M1 (format 1, bits 7-9 and
// 10-12), both K-major, N >> 3 in bits 17-22, UE4M3 scales (bit 23 = 0),
// M >> 4 in bits 24-28, dense K = 64.
__device__ __forceinline__ uint32_t idesc_nvf4(int M, int N) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void bar_init(uint64_t *b, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(count));
}
__device__ __forceinline__ void bar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
// Wait for the completion of the phase with parity `par`; false on time-out
// (or when another role already gave up and set *err).
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t par, int *err) {
  uint32_t ok = 0;
  for (long long it = 0; it < kSpinLimit; ++it) {
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(sa(b)), "r"(par) : "memory");
    if (ok) return true;
    if ((it & 1023) == 1023 && *(volatile int *)err) return false;
  }
  atomicExch(err, 1);
  return false;
}
// Wait for operations that always complete (this CTA's own MMAs): bounded,
// but not cut short by the error word.
__device__ __forceinline__ bool bar_wait_drain(uint64_t *b, uint32_t par) {
  uint32_t ok = 0;
  for (long long it = 0; it < 4 * kSpinLimit && !ok; ++it)
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(sa(b)), "r"(par) : "memory");
  return ok != 0;
}
// arrive (without a pending-count increment) on `b` once every cp.async this
// thread issued so far has landed
__device__ __forceinline__ void cp_async_arrive(uint64_t *b) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(sa(b)) : "memory");
}
// arrive on `b` and add `bytes` to the transaction count its phase waits for
__device__ __forceinline__ void bar_arrive_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}
// bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned) from
// this GPU's global memory into this CTA's shared memory, completing as
// transactions on `b`.  Plain (non-multicast) form only.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(sa(dst)), "l"(src), "r"(bytes), "r"(sa(b)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// arrive on `b` once every tcgen05 operation this thread issued so far has completed
__device__ __forceinline__ void commit(uint64_t *b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ void alloc(uint32_t *dst_smem, int cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(dst_smem)), "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void dealloc(uint32_t taddr, int cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols));
}
// D[128 x N] (+)= A . B^T with per-16 UE4M3 block scales of A (sfa) and B (sfb)
__device__ __forceinline__ void mma_nvf4(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t sfa,
                                         uint32_t sfb, uint32_t acc) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n"
               ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc), "r"(sfa), "r"(sfb));
}
// one scale-factor atom (shared memory) -> 4 TMEM columns of every lane quarter
__device__ __forceinline__ void cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc));
}
// 32 f32 columns of this thread's TMEM lane (complete after wait_ld)
__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                 "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                 "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                 "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
               : "r"(taddr) : "memory");
}
// 16 f32 columns of this thread's TMEM lane (complete after wait_ld)
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t *v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                 "=r"(v[15])
               : "r"(taddr) : "memory");
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace ffn
