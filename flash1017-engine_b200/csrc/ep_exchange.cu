// ep_exchange.cu -- the per-layer sum of the expert-parallel partial outputs
// over NVLink peer memory, one process per GPU.
//
// Every rank owns one block of experts and computes, for all tokens, the
// weighted sum of its own experts' outputs (its "part").  The layer output is
// residual + sum over ranks of the parts, needed on every rank (the reference's
// decode MoE block, crates/flash-core/src/flash1017.rs:7521-7567, with the
// residual add of flash1017.rs:4900-4905).  Instead of an NCCL all-reduce, one
// cooperative kernel per GPU does a two-shot exchange over peer memory:
//
//   1. signal "part ready" (epoch e) to every peer; wait for every peer's
//      signal (bounded);
//   2. rank r sums its slice of token rows [r T/N, (r+1) T/N) from all parts
//      in rank order (deterministic), adds the residual, and writes the rows to
//      its result buffer red[e % 2];
//   3. grid-wide sync, signal "slice ready"; wait for every peer's signal;
//   4. every rank copies all slices from the owners' result buffers into out.
//
// Bytes over NVLink per rank: (N-1)/N of the parts' rows in step 2 and (N-1)/N
// of the output in step 4.  Buffers live in one allocation per rank shared
// through CUDA IPC (cudaIpcGetMemHandle / cudaIpcOpenMemHandle; peers' memory
// is read with plain loads, no TMA and no multicast).  The result buffer is
// double-buffered by epoch: a rank can be at most one call ahead of a peer
// (step 1 of call e+1 waits for the peer to finish call e), so it never
// overwrites rows a peer is still reading.  Every wait gives up after a bounded
// number of polls, sets the error word and returns; the kernel then writes NaN
// over `out` so a failed exchange is visible.
#include <cooperative_groups.h>

#include <algorithm>

#include "ffn_internal.h"

namespace cg = cooperative_groups;

namespace ffn {
namespace {

constexpr int kEpMax = 8;
constexpr long long kEpSpin = 1LL << 22;  // flag polls per wait before giving up

struct EpShared {        // header of every rank's shared allocation
  uint32_t flags[2][kEpMax];  // [phase][source rank] = last epoch signalled
  int err;
  uint32_t pad[64 - 2 * kEpMax - 1];
};

struct EpArgs {
  int rank, world, n_tok, hidden;
  uint32_t epoch;
  const float *part[kEpMax];   // every rank's part (own entry local)
  float *red_local;            // own result buffer for this epoch
  const float *red[kEpMax];    // every rank's result buffer for this epoch
  uint32_t *flags_peer[kEpMax];// every rank's flags
  uint32_t *flags_local;
  int *err;
  const float *residual;       // nullable
  float *out;
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Block 0 tells every peer that this rank reached `phase` of call `epoch`;
// then every block waits until all peers did (epochs only grow, so >= works).
__device__ bool ep_barrier(const EpArgs &a, int phase) {
  __shared__ int s_ok;
  if (blockIdx.x == 0 && threadIdx.x < a.world)
    st_release_sys(a.flags_peer[threadIdx.x] + phase * kEpMax + a.rank, a.epoch);
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int src = 0; src < a.world && ok; ++src) {
      long long it = 0;
      while ((int32_t)(ld_acquire_sys(a.flags_local + phase * kEpMax + src) - a.epoch) < 0) {
        if (++it > kEpSpin || *(volatile int *)a.err) { ok = 0; break; }
      }
    }
    if (!ok) atomicExch(a.err, 1);
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// W = world size (compile time: every peer's load of a step issues at once).
template <int W>
__global__ void __launch_bounds__(256) ep_exchange_kernel(const EpArgs a) {
  cg::grid_group grid = cg::this_grid();
  const int H4 = a.hidden / 4;
  const int rows_per = (a.n_tok + W - 1) / W;
  const int r0 = min(a.n_tok, a.rank * rows_per), r1 = min(a.n_tok, r0 + rows_per);
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long nthr = (long long)gridDim.x * blockDim.x;
  bool ok = ep_barrier(a, 0);
  if (ok) {
    // step 2: own slice, summed over the ranks in rank order
    const long long n4 = (long long)(r1 - r0) * H4;
    for (long long i = tid; i < n4; i += nthr) {
      const size_t off = (size_t)r0 * a.hidden + (size_t)i * 4;
      float4 v[W];
#pragma unroll
      for (int src = 0; src < W; ++src) v[src] = __ldcg(reinterpret_cast<const float4 *>(a.part[src] + off));
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int src = 0; src < W; ++src) {
        acc.x = __fadd_rn(acc.x, v[src].x); acc.y = __fadd_rn(acc.y, v[src].y);
        acc.z = __fadd_rn(acc.z, v[src].z); acc.w = __fadd_rn(acc.w, v[src].w);
      }
      if (a.residual) {
        const float4 r = *reinterpret_cast<const float4 *>(a.residual + off);
        acc.x = __fadd_rn(r.x, acc.x); acc.y = __fadd_rn(r.y, acc.y);
        acc.z = __fadd_rn(r.z, acc.z); acc.w = __fadd_rn(r.w, acc.w);
      }
      *reinterpret_cast<float4 *>(a.red_local + off) = acc;
    }
  }
  __threadfence_system();
  grid.sync();
  ok = ok && !*(volatile int *)a.err && ep_barrier(a, 1);
  if (ok) {
    // step 4: every slice from its owner, four 16-byte loads in flight per thread
    const long long n4 = (long long)a.n_tok * H4;
    for (long long i0 = tid; i0 < n4; i0 += 4 * nthr) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long i = i0 + u * nthr;
        if (i < n4) {
          const int owner = min(W - 1, (int)(i / H4) / rows_per);
          v[u] = __ldcg(reinterpret_cast<const float4 *>(a.red[owner] + (size_t)i * 4));
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long i = i0 + u * nthr;
        if (i < n4) *reinterpret_cast<float4 *>(a.out + (size_t)i * 4) = v[u];
      }
    }
  } else {
    const long long n = (long long)a.n_tok * a.hidden;
    for (long long i = tid; i < n; i += nthr) a.out[i] = __int_as_float(0x7FC00000);
  }
}

using ExchangeFn = void (*)(const EpArgs);
ExchangeFn exchange_kernel(int world) {
  switch (world) {
    case 1: return ep_exchange_kernel<1>;
    case 2: return ep_exchange_kernel<2>;
    case 3: return ep_exchange_kernel<3>;
    case 4: return ep_exchange_kernel<4>;
    case 5: return ep_exchange_kernel<5>;
    case 6: return ep_exchange_kernel<6>;
    case 7: return ep_exchange_kernel<7>;
    default: return ep_exchange_kernel<8>;
  }
}

}  // namespace
}  // namespace ffn

using namespace ffn;

struct ffn_b200_ep {
  int rank = 0, world = 1, device = 0;
  size_t max_tokens = 0, hidden = 0;
  size_t part_bytes = 0;
  uint8_t *base = nullptr;              // own allocation: header | part | red[2]
  uint8_t *peer[kEpMax] = {nullptr};    // every rank's allocation (own = base)
  uint32_t epoch = 0;
  int grid = 0;
};

static size_t ep_alloc_bytes(size_t max_tokens, size_t hidden) {
  const size_t part = (max_tokens * hidden * sizeof(float) + 255) & ~(size_t)255;
  return sizeof(EpShared) + 3 * part;
}

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
  ep->part_bytes = (max_tokens * hidden * sizeof(float) + 255) & ~(size_t)255;
  cudaError_t e = cudaGetDevice(&ep->device);
  if (e == cudaSuccess) e = cudaMalloc(&ep->base, ep_alloc_bytes(max_tokens, hidden));
  if (e == cudaSuccess) e = cudaMemset(ep->base, 0, sizeof(EpShared));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(my_handle), ep->base);
  int sms = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ep->device);
  int per_sm = 0;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, exchange_kernel(world), 256, 0);
  if (e != cudaSuccess) {
    if (ep->base) cudaFree(ep->base);
    delete ep;
    return cuda_fail(e, "ep_create");
  }
  ep->grid = std::max(1, sms * std::min(per_sm, 2));  // co-resident (cooperative launch)
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
  if (!ep || !out) return fail(FFN_B200_EINVAL, "ep_allreduce: null argument");
  if (n_tok > ep->max_tokens) return fail(FFN_B200_EINVAL, "ep_allreduce: more tokens than ep_create's");
  for (int r = 0; r < ep->world; ++r)
    if (!ep->peer[r]) return fail(FFN_B200_EINVAL, "ep_allreduce: ep_connect has not opened every peer");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual)) & 15)
    return fail(FFN_B200_EINVAL, "ep_allreduce: out and residual must be 16-byte aligned");
  if (n_tok == 0) return 0;
  ++ep->epoch;
  EpArgs a{};
  a.rank = ep->rank;
  a.world = ep->world;
  a.n_tok = (int)n_tok;
  a.hidden = (int)ep->hidden;
  a.epoch = ep->epoch;
  const size_t red_off = sizeof(EpShared) + ep->part_bytes * (1 + (ep->epoch & 1));
  for (int r = 0; r < ep->world; ++r) {
    a.part[r] = reinterpret_cast<const float *>(ep->peer[r] + sizeof(EpShared));
    a.red[r] = reinterpret_cast<const float *>(ep->peer[r] + red_off);
    a.flags_peer[r] = reinterpret_cast<EpShared *>(ep->peer[r])->flags[0];
  }
  a.red_local = reinterpret_cast<float *>(ep->base + red_off);
  a.flags_local = reinterpret_cast<EpShared *>(ep->base)->flags[0];
  a.err = &reinterpret_cast<EpShared *>(ep->base)->err;
  a.residual = residual;
  a.out = out;
  void *args[] = {&a};
  cudaStream_t st = (cudaStream_t)stream;
  prof_begin(FFN_B200_K_OTHER, st);
  cudaError_t e = cudaLaunchCooperativeKernel((const void *)exchange_kernel(ep->world), dim3(ep->grid),
                                              dim3(256), args, 0, st);
  prof_end(FFN_B200_K_OTHER, st);
  note_launch();
  if (e != cudaSuccess) return cuda_fail(e, "ep_allreduce: cooperative launch");
  return 0;
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
