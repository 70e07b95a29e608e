// noalloc.cu -- an expert-forward entry point that allocates nothing.
//
// ffn_b200_expert_forward needs a scratch buffer from its caller.  Some callers
// cannot provide one and must not see this library call cudaMalloc: a host
// that loads the library as a plugin and owns the device-memory budget (the
// reference's plugin ABI has no scratch argument), code that runs while a CUDA
// stream is being captured (cudaMalloc is not a stream operation), and decode
// loops that cannot afford an allocation that may synchronise the device or
// fail in the middle of a step.  For them this file keeps the scratch in one
// file-scope __device__ array of kNoAllocScratchBytes; every GPU that loads the
// library holds that array until the process exits.
#include <mutex>

#include "ffn_internal.h"

namespace ffn {
namespace {

constexpr size_t kNoAllocScratchBytes = 1u << 20;  // 1 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device.  In host code
// the array's name is only a host-side stand-in; its device address comes
// from cudaGetSymbolAddress, called with that device current.
std::mutex g_mu;
void *g_addr[64] = {nullptr};

int scratch_address(void **out) {
  int dev = -1;
  FFN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FFN_B200_EUNSUP, "expert_forward_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "expert_forward_noalloc: cudaGetSymbolAddress");
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return 0;
}

}  // namespace
}  // namespace ffn

extern "C" int ffn_b200_expert_forward_noalloc(size_t inter, size_t hidden, size_t seq,
                                               const ffn_b200_expert *e, const float *x,
                                               float *out, float accum_weight, int accumulate,
                                               void *stream) {
  const size_t need = ffn_b200_expert_ws_bytes(inter, hidden, seq);
  if (need > ffn::kNoAllocScratchBytes)
    return ffn::fail(FFN_B200_EINVAL,
                     "expert_forward_noalloc: this shape needs " + std::to_string(need) +
                         " bytes of scratch, more than the fixed " +
                         std::to_string(ffn::kNoAllocScratchBytes) +
                         " (use ffn_b200_expert_forward with a caller buffer)");
  void *scratch = nullptr;
  int rc = ffn::scratch_address(&scratch);
  if (rc) return rc;
  // Every scratch byte this path reads is written earlier in the same call
  // (activation halves, exponents, core terms, SwiGLU output), so nothing has
  // to be cleared between calls.
  return ffn_b200_expert_forward(inter, hidden, seq, e, x, out, accum_weight, accumulate, scratch,
                                 ffn::kNoAllocScratchBytes, stream);
}
