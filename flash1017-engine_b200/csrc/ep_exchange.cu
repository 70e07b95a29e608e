// ep_exchange.cu -- the per-layer sum of the expert-parallel partial outputs
// over NVLink peer memory, one process per GPU.
//
// Every rank owns one block of experts and computes, for all tokens, the
// weighted sum of its own experts' outputs (its "partial").  The layer output is
// residual + sum over ranks of the partials, needed on every rank (the
// reference's decode MoE block, crates/flash-core/src/flash1017.rs:7521-7567,
// with the residual add of flash1017.rs:4900-4905).  One cooperative kernel per
// GPU (one CTA per SM) does it by pushing, never by polling a peer:
//
//   A. every CTA forms its share of this rank's partial rows -- from the part
//      buffer the MoE layer wrote, or (fused) straight from the layer's expert
//      outputs, combined per token as the combine kernel does -- and stores
//      each row into the inbox of the rank that owns the row's slice of tokens
//      (rank s owns rows [s R, (s+1) R), R = ceil(tokens / world)); then it adds
//      1 to every rank's arrival counter 1 (red.release.sys).
//   B. once counter 1 of this rank has reached world x grid x calls, every
//      sender's rows have landed in this rank's inbox: the CTAs sum the slice's
//      rows over the senders in rank order (deterministic), add the residual,
//      and store each result row into every rank's output slot; then they add 1
//      to every rank's counter 2.
//   C. once counter 2 has reached its target, the whole layer output sits in
//      this rank's slot; the CTAs copy it to `out`.
//
// NVLink traffic per rank and call: (N-1)/N of the partial rows out in A and
// (N-1)/N of the output rows out in B, all as plain 16-byte stores to peer
// memory (CUDA IPC mappings; no TMA of any form).  The counters only grow
// (each call adds world x grid), so no reset is needed; a rank can start call
// e+1 only after counter 2 of call e told it that every rank finished reading
// its inbox (B), so the inboxes need no double buffering; the output slots
// alternate by call parity, so the rows a peer writes for call e+1 never land
// on the slot this rank still reads as call e's input.  Every wait polls local
// memory only and gives up after a bounded time (kEpWaitNs): it sets the error
// word, the CTA writes NaN, and ffn_b200_ep_error reports it.
#include <cooperative_groups.h>

#include <algorithm>

#include "ffn_internal.h"

namespace ffn {
namespace {

constexpr int kEpMax = 8;
// A wait gives up after this long (ns of %globaltimer): well above any skew
// between ranks that reach the same call (a step's host work, a slow launch),
// short enough that a rank that never arrives ends the call.
constexpr unsigned long long kEpWaitNs = 5000000000ull;
constexpr int kEpThreads = 256;
constexpr int kEpChunk = 4 * kEpThreads;  // floats of a row per work unit

struct EpShared {  // header of every rank's shared allocation
  unsigned long long cnt1;  // arrivals of phase A
  unsigned long long pad1[15];
  unsigned long long cnt2;  // arrivals of phase B
  unsigned long long pad2[15];
  int err;
  int pad3[63];
};

struct PushArgs {
  int rank, world, n_tok, hidden, rows_per, chunks;
  unsigned long long target;      // counter value once every CTA of every rank arrived
  const float *part;              // the partial rows (unfused), or
  EpCombine comb;                 // the MoE layer's expert outputs (fused)
  int fused;
  float *inbox[kEpMax];           // every rank's inbox: [sender][rows_per][hidden]
  unsigned long long *flags[kEpMax];  // every rank's row flags: [sender][rows_per], = tag when sent
  const unsigned long long *flags_local;
  unsigned long long tag;         // this call's number (flags of earlier calls hold smaller ones)
  float *slot[kEpMax];            // every rank's output slot of this call
  unsigned long long *cnt1[kEpMax], *cnt2[kEpMax];
  const unsigned long long *cnt1_local, *cnt2_local;
  int *err;
  const float *residual;          // nullable
  float *out;
};

__device__ __forceinline__ void red_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Thread 0 polls the local counter until it reaches `target` (bounded in
// time); the CTA learns the outcome through shared memory.
__device__ bool wait_count(const unsigned long long *c, unsigned long long target, int *err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long t0 = global_ns();
    long long it = 0;
    while ((long long)(ld_acquire_sys(c) - target) < 0) {
      if ((++it & 255) == 0 && (global_ns() - t0 > kEpWaitNs || *(volatile int *)err)) { ok = 0; break; }
    }
    if (!ok) atomicExch(err, 1);
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

__device__ __forceinline__ float4 nan4() {
  const float q = __int_as_float(0x7FC00000);
  return make_float4(q, q, q, q);
}

// W = world size (compile time: every sender's load of a phase-B row issues at once).
template <int W>
__global__ void __launch_bounds__(kEpThreads) ep_push_kernel(const PushArgs a) {
  __shared__ float wk[kTopKMax];
  __shared__ int pk[kTopKMax];
  __shared__ int s_bad;
  const int H4 = a.hidden / 4;
  const bool moe_bad = a.fused && a.comb.err && *a.comb.err;
  // ---- A: this rank's partial rows into the owners' inboxes
  const int units_a = a.n_tok * a.chunks;
  for (int u = blockIdx.x; u < units_a; u += gridDim.x) {
    const int t = u / a.chunks, c4 = (u % a.chunks) * kEpThreads + threadIdx.x;
    if (a.fused) {
      __syncthreads();  // wk / pk of the previous unit are no longer read
      if (threadIdx.x == 0) s_bad = 0;
      __syncthreads();
      if (threadIdx.x < a.comb.top_k) {
        const int q = t * a.comb.top_k + threadIdx.x;
        const int e = a.comb.idx[q];
        if (e < 0 || e >= a.comb.n_exp) {  // no expert selected (every score NaN): no table read
          s_bad = 1;
          wk[threadIdx.x] = 0.f;
          pk[threadIdx.x] = -1;
        } else {
          float w = a.comb.wt[q];
          if (a.comb.experts[e].format == FFN_B200_FMT_TERNARY) w = w * a.comb.experts[e].proj_scale;
          const int pp = a.comb.inv[q];
          if (pp >= a.comb.y_rows) s_bad = 1;  // not a row of y: no read
          wk[threadIdx.x] = w;
          pk[threadIdx.x] = pp < a.comb.y_rows ? pp : -1;
        }
      }
      __syncthreads();
    }
    // a token none of whose experts is on this rank has a zero partial: it is
    // not sent (its flag stays old), and the owner adds zero in its place
    bool present = !a.fused || moe_bad || s_bad;
    if (!present)
      for (int k = 0; k < a.comb.top_k; ++k) present |= pk[k] >= 0;
    if (!present) continue;
    if (threadIdx.x == 0 && u % a.chunks == 0) {
      const int s = t / a.rows_per, j = t - s * a.rows_per;
      a.flags[s][a.rank * a.rows_per + j] = a.tag;
    }
    if (c4 < H4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (!a.fused) {
        acc = __ldcg(reinterpret_cast<const float4 *>(a.part + (size_t)t * a.hidden) + c4);
      } else if (moe_bad || s_bad) {
        acc = nan4();
      } else {
        // the combine kernel's arithmetic: acc += w_k * y_k over this rank's experts, in k order
        for (int k = 0; k < a.comb.top_k; ++k) {
          const int pp = pk[k];
          if (pp < 0) continue;
          const float4 y = __ldg(reinterpret_cast<const float4 *>(a.comb.y + (size_t)pp * a.comb.ld_y) + c4);
          acc.x = __fadd_rn(acc.x, __fmul_rn(wk[k], y.x));
          acc.y = __fadd_rn(acc.y, __fmul_rn(wk[k], y.y));
          acc.z = __fadd_rn(acc.z, __fmul_rn(wk[k], y.z));
          acc.w = __fadd_rn(acc.w, __fmul_rn(wk[k], y.w));
        }
      }
      const int s = t / a.rows_per, j = t - s * a.rows_per;
      float *dst = a.inbox[s] + ((size_t)a.rank * a.rows_per + j) * a.hidden;
      reinterpret_cast<float4 *>(dst)[c4] = acc;
    }
  }
  // the CTA's stores, then one system-scope fence and the releases (cumulative
  // over the stores the barrier ordered before them)
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x < W) red_release_sys(a.cnt1[threadIdx.x], 1ull);
  // ---- B: this rank's slice, summed over the senders, pushed to every rank
  const bool ok_a = wait_count(a.cnt1_local, a.target, a.err);
  const int r0 = a.rank * a.rows_per;
  const int nr = max(0, min(a.n_tok - r0, a.rows_per));
  const float *inbox = a.inbox[a.rank];
  for (int u = blockIdx.x; u < nr * a.chunks; u += gridDim.x) {
    const int j = u / a.chunks, c4 = (u % a.chunks) * kEpThreads + threadIdx.x;
    if (c4 >= H4) continue;
    const int t = r0 + j;
    float4 v[W];
#pragma unroll
    for (int src = 0; src < W; ++src)
      v[src] = __ldcg(a.flags_local + src * a.rows_per + j) == a.tag
                   ? __ldcg(reinterpret_cast<const float4 *>(inbox + ((size_t)src * a.rows_per + j) * a.hidden) + c4)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int src = 0; src < W; ++src) {
      acc.x = __fadd_rn(acc.x, v[src].x); acc.y = __fadd_rn(acc.y, v[src].y);
      acc.z = __fadd_rn(acc.z, v[src].z); acc.w = __fadd_rn(acc.w, v[src].w);
    }
    if (a.residual) {
      const float4 r = reinterpret_cast<const float4 *>(a.residual + (size_t)t * a.hidden)[c4];
      acc.x = __fadd_rn(r.x, acc.x); acc.y = __fadd_rn(r.y, acc.y);
      acc.z = __fadd_rn(r.z, acc.z); acc.w = __fadd_rn(r.w, acc.w);
    }
    if (!ok_a) acc = nan4();
#pragma unroll
    for (int dst = 0; dst < W; ++dst) reinterpret_cast<float4 *>(a.slot[dst] + (size_t)t * a.hidden)[c4] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x < W) red_release_sys(a.cnt2[threadIdx.x], 1ull);
  // ---- C: every slice has arrived in this rank's slot
  const bool ok = wait_count(a.cnt2_local, a.target, a.err) && ok_a;
  if (a.out) {
    const float *mine = a.slot[a.rank];
    const long long n4 = (long long)a.n_tok * H4;
    for (long long i = (long long)blockIdx.x * kEpThreads + threadIdx.x; i < n4;
         i += (long long)gridDim.x * kEpThreads)
      reinterpret_cast<float4 *>(a.out)[i] = ok ? __ldcg(reinterpret_cast<const float4 *>(mine) + i) : nan4();
  }
}

using ExchangeFn = void (*)(const PushArgs);
ExchangeFn exchange_kernel(int world) {
  switch (world) {
    case 1: return ep_push_kernel<1>;
    case 2: return ep_push_kernel<2>;
    case 3: return ep_push_kernel<3>;
    case 4: return ep_push_kernel<4>;
    case 5: return ep_push_kernel<5>;
    case 6: return ep_push_kernel<6>;
    case 7: return ep_push_kernel<7>;
    default: return ep_push_kernel<8>;
  }
}

}  // namespace
}  // namespace ffn

using namespace ffn;

struct ffn_b200_ep {
  int rank = 0, world = 1, device = 0;
  size_t max_tokens = 0, hidden = 0;
  size_t part_bytes = 0, inbox_bytes = 0;
  uint8_t *base = nullptr;              // own allocation: header | part | inbox | slot[2]
  uint8_t *peer[kEpMax] = {nullptr};    // every rank's allocation (own = base)
  unsigned long long epoch = 0;
  int grid = 0;
};

static size_t round256(size_t n) { return (n + 255) & ~(size_t)255; }
static size_t rows_max(size_t max_tokens, int world) { return (max_tokens + world - 1) / world; }
// the row flags sit after the inbox rows, inside the inbox area
static size_t flags_off(const ffn_b200_ep &ep) {
  return round256((size_t)ep.world * rows_max(ep.max_tokens, ep.world) * ep.hidden * sizeof(float));
}
static size_t ep_alloc_bytes(const ffn_b200_ep &ep) {
  return sizeof(EpShared) + ep.part_bytes + ep.inbox_bytes + 2 * ep.part_bytes;
}

namespace ffn {

// One exchange call: this rank's partial (the part buffer, or the MoE layer's
// expert outputs when comb != nullptr) summed over every rank, + residual, into out.
int ep_exchange(ffn_b200_ep *ep, size_t n_tok, const EpCombine *comb, const float *residual, float *out,
                cudaStream_t st) {
  if (!ep || !out) return fail(FFN_B200_EINVAL, "ep exchange: null argument");
  if (n_tok > ep->max_tokens) return fail(FFN_B200_EINVAL, "ep exchange: more tokens than ep_create's");
  for (int r = 0; r < ep->world; ++r)
    if (!ep->peer[r]) return fail(FFN_B200_EINVAL, "ep exchange: ep_connect has not opened every peer");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual)) & 15)
    return fail(FFN_B200_EINVAL, "ep exchange: out and residual must be 16-byte aligned");
  if (comb && (comb->ld_y % 4 || (reinterpret_cast<uintptr_t>(comb->y) & 15) || comb->top_k > kTopKMax))
    return fail(FFN_B200_EINVAL, "ep exchange: expert outputs must be 16-byte aligned rows");
  if (n_tok == 0) return 0;
  ++ep->epoch;
  PushArgs a{};
  a.rank = ep->rank;
  a.world = ep->world;
  a.n_tok = (int)n_tok;
  a.hidden = (int)ep->hidden;
  a.rows_per = (int)((n_tok + ep->world - 1) / ep->world);
  a.chunks = (int)((ep->hidden + kEpChunk - 1) / kEpChunk);
  a.target = ep->epoch * (unsigned long long)ep->world * (unsigned long long)ep->grid;
  a.part = reinterpret_cast<const float *>(ep->base + sizeof(EpShared));
  if (comb) {
    a.comb = *comb;
    a.fused = 1;
  }
  const size_t inbox_off = sizeof(EpShared) + ep->part_bytes;
  const size_t slot_off = inbox_off + ep->inbox_bytes + (ep->epoch & 1) * ep->part_bytes;
  a.tag = ep->epoch;
  for (int r = 0; r < ep->world; ++r) {
    EpShared *h = reinterpret_cast<EpShared *>(ep->peer[r]);
    a.inbox[r] = reinterpret_cast<float *>(ep->peer[r] + inbox_off);
    a.flags[r] = reinterpret_cast<unsigned long long *>(ep->peer[r] + inbox_off + flags_off(*ep));
    a.slot[r] = reinterpret_cast<float *>(ep->peer[r] + slot_off);
    a.cnt1[r] = &h->cnt1;
    a.cnt2[r] = &h->cnt2;
  }
  EpShared *mine = reinterpret_cast<EpShared *>(ep->base);
  a.flags_local = a.flags[ep->rank];
  a.cnt1_local = &mine->cnt1;
  a.cnt2_local = &mine->cnt2;
  a.err = &mine->err;
  a.residual = residual;
  a.out = out;
  void *args[] = {&a};
  prof_begin(FFN_B200_K_OTHER, st);
  cudaError_t e = cudaLaunchCooperativeKernel((const void *)exchange_kernel(ep->world), dim3(ep->grid),
                                              dim3(kEpThreads), args, 0, st);
  prof_end(FFN_B200_K_OTHER, st);
  note_launch();
  if (e != cudaSuccess) return cuda_fail(e, "ep exchange: cooperative launch");
  return 0;
}

}  // namespace ffn

extern "C" {

size_t ffn_b200_ep_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int ffn_b200_ep_create(int rank, int world, size_t max_tokens, size_t hidden, void *my_handle,
                       ffn_b200_ep **out) {
  if (!out || !my_handle) return fail(FFN_B200_EINVAL, "ep_create: null argument");
  *out = nullptr;
  if (world < 1 || world > kEpMax || rank < 0 || rank >= world)
    return fail(FFN_B200_EINVAL, "ep_create: world must be 1..8 and rank inside it");
  if (max_tokens == 0 || hidden == 0 || hidden % 4)
    return fail(FFN_B200_EINVAL, "ep_create: need max_tokens > 0 and hidden a multiple of 4");
  auto *ep = new ffn_b200_ep();
  ep->rank = rank;
  ep->world = world;
  ep->max_tokens = max_tokens;
  ep->hidden = hidden;
  ep->part_bytes = round256(max_tokens * hidden * sizeof(float));
  ep->inbox_bytes = round256((size_t)world * rows_max(max_tokens, world) * hidden * sizeof(float)) +
                    round256((size_t)world * rows_max(max_tokens, world) * sizeof(unsigned long long));
  cudaError_t e = cudaGetDevice(&ep->device);
  if (e == cudaSuccess) e = cudaMalloc(&ep->base, ep_alloc_bytes(*ep));
  if (e == cudaSuccess) e = cudaMemset(ep->base, 0, sizeof(EpShared));
  if (e == cudaSuccess)  // the row flags: 0 = no call has sent the row
    e = cudaMemset(ep->base + sizeof(EpShared) + ep->part_bytes + flags_off(*ep), 0,
                   ep->inbox_bytes - flags_off(*ep));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(my_handle), ep->base);
  int sms = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ep->device);
  int per_sm = 0;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, exchange_kernel(world), kEpThreads, 0);
  if (e == cudaSuccess && per_sm < 1) e = cudaErrorCooperativeLaunchTooLarge;
  if (e != cudaSuccess) {
    if (ep->base) cudaFree(ep->base);
    delete ep;
    return cuda_fail(e, "ep_create");
  }
  // one CTA per SM: every CTA of every rank must be resident at once (each
  // waits for the others' arrivals), and every rank uses the same count
  ep->grid = sms;
  ep->peer[rank] = ep->base;
  *out = ep;
  return 0;
}

int ffn_b200_ep_connect(ffn_b200_ep *ep, const void *all_handles) {
  if (!ep || !all_handles) return fail(FFN_B200_EINVAL, "ep_connect: null argument");
  const auto *h = reinterpret_cast<const cudaIpcMemHandle_t *>(all_handles);
  for (int r = 0; r < ep->world; ++r) {
    if (r == ep->rank || ep->peer[r]) continue;
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "ep_connect: cudaIpcOpenMemHandle");
    ep->peer[r] = reinterpret_cast<uint8_t *>(p);
  }
  return 0;
}

float *ffn_b200_ep_part(ffn_b200_ep *ep) {
  return ep ? reinterpret_cast<float *>(ep->base + sizeof(EpShared)) : nullptr;
}

int ffn_b200_ep_allreduce(ffn_b200_ep *ep, size_t n_tok, const float *residual, float *out,
                          void *stream) {
  return ffn::ep_exchange(ep, n_tok, nullptr, residual, out, (cudaStream_t)stream);
}

int ffn_b200_ep_error(ffn_b200_ep *ep, int *flag) {
  if (!ep || !flag) return fail(FFN_B200_EINVAL, "ep_error: null argument");
  FFN_CUDA_TRY(cudaMemcpy(flag, &reinterpret_cast<EpShared *>(ep->base)->err, sizeof(int),
                          cudaMemcpyDeviceToHost));
  return 0;
}

int ffn_b200_ep_destroy(ffn_b200_ep *ep) {
  if (!ep) return 0;
  for (int r = 0; r < ep->world; ++r)
    if (r != ep->rank && ep->peer[r]) cudaIpcCloseMemHandle(ep->peer[r]);
  if (ep->base) cudaFree(ep->base);
  delete ep;
  return 0;
}

}  // extern "C"
