// addon_abi.cu -- the reference's plugin ABI (include/merkaba_hw_addon.h) on B200.
//
// The Rust host (crates/flash-core/src/hardware_addon.rs, "HA") calls these
// functions with HOST pointers and reads `out` right after they return.  B200
// memory is discrete, so this layer
//   * keeps HBM copies of weight ranges: ranges registered through
//     gx10_rust_register_host_range are copied eagerly; any other weight
//     pointer (inside gx10_rust_register_shard_bounds ranges or not) is copied
//     the first time a kernel needs it, as exactly the bytes that call reads.
//     Weights are immutable for the process lifetime in the reference (mmap'd
//     read-only safetensors), which is what makes the cache valid.  The copies
//     are disjoint intervals (one predecessor search per lookup); when a budget
//     (ffn_b200_set_host_cache_budget) or the GPU's memory runs out, the least
//     recently used copies go first (first-use copies before registered
//     ranges) and are copied again when needed, so a model larger than HBM
//     (the reference registers only its hot experts, hardware_addon.rs:681-697,
//     flash1017.rs:5228-5239) keeps running on the GPU;
//   * stages x / out through device buffers on one internal stream;
//   * runs the same kernels as the device-resident ABI (ffn_b200.h).
// Calls are serialised by a mutex (the reference calls from one thread at a
// time, CLI:1833-1846).  There is no CPU compute path here: every result comes
// from a CUDA kernel, and failures are reported, not recomputed.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "ffn_internal.h"
#include "merkaba_hw_addon.h"

namespace ffn {
namespace {

struct DevBuf {
  void *p = nullptr;
  size_t n = 0;
  int ensure(size_t bytes) {
    if (bytes <= n) return 0;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    const size_t want = std::max<size_t>(bytes, 1 << 20);
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(staging)");
    n = want;
    return 0;
  }
};

// One HBM copy of host bytes [h, h + n).  The copies are disjoint (a new range
// that overlaps copies replaces them with one copy of the union), so the copy
// holding an address is its predecessor in the map.
struct Range {
  uintptr_t h;
  size_t n;
  char *d;
  uint64_t last_use;  // call number of the last call that resolved an address in it
  bool registered;    // through gx10_rust_register_host_range (evicted after first-use copies)
};

struct Ctx {
  std::mutex mu;
  bool init = false;
  int device = -1;
  cudaStream_t st = nullptr;
  cudaStream_t st2 = nullptr;  // side stream of queued runs (independent slice lists)
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  DevBuf x, out, ws, tmp;
  std::map<uintptr_t, Range> ranges;  // disjoint copies, by host start address
  size_t cached = 0;
  size_t budget = 0;       // bytes the copies may hold (0: as much as the GPU gives)
  uint64_t call_no = 0;    // entry-point calls so far (a call never evicts its own copies)
  std::vector<std::pair<uintptr_t, size_t>> shard_bounds;
  // pending accumulation of gx10_rust_*_mlp_accum / _mlp_batch
  float *pend_host = nullptr;
  size_t pend_n = 0;
  // Routed calls not yet run: accumulating *_mlp_accum calls (x rows in bx)
  // or *_mlp_batch calls (x rows in xall).  They run together as one routed
  // layer (ffn::routed_calls) when the host needs `out`.
  struct Call {
    ffn_b200_expert e;
    int32_t row0, m;
    int32_t dst[8];  // out rows
    float w[8];
  };
  std::vector<Call> queue;
  int q_src = 0;  // 1: bx, 2: xall
  size_t q_inter = 0, q_hidden = 0;
  int q_out_rows = 0;
  DevBuf bx;  // the queued *_mlp_accum calls' x rows
  // pinned host stages of the call tables, reused once their upload is done
  struct Stage {
    void *h = nullptr;
    size_t n = 0;
    cudaEvent_t ev = nullptr;
    bool used = false;
  };
  Stage stage[2];
  int stage_i = 0;
  // pinned host stages of the queued *_mlp_accum calls' x rows (one upload
  // per run); a call whose x equals the previous staged row reuses it
  Stage xstage[2];
  int xstage_i = 0;
  int q_xrows = 0;
  bool q_zero = false;  // the queue began with an overwriting call
  // batched-layer input x_all (ffn_b200_set_batch_input)
  const float *xall_host = nullptr;
  size_t xall_tok = 0, xall_hidden = 0;
  bool xall_dev_valid = false;
  DevBuf xall;
};

Ctx &ctx() {
  static Ctx *c = new Ctx();  // never destroyed: the vtable outlives static teardown
  return *c;
}

int ensure_init(Ctx &c) {
  ++c.call_no;
  if (c.init) {
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev == c.device) return 0;
    return fail(FFN_B200_EUNSUP, "reference ABI: called on a different device than the first call");
  }
  FFN_CUDA_TRY(cudaGetDevice(&c.device));
  FFN_CUDA_TRY(cudaStreamCreateWithFlags(&c.st, cudaStreamNonBlocking));
  FFN_CUDA_TRY(cudaStreamCreateWithFlags(&c.st2, cudaStreamNonBlocking));
  FFN_CUDA_TRY(cudaEventCreateWithFlags(&c.ev_fork, cudaEventDisableTiming));
  FFN_CUDA_TRY(cudaEventCreateWithFlags(&c.ev_join, cudaEventDisableTiming));
  c.init = true;
  return 0;
}

int run_queue(Ctx &c);

// Before a copy is freed: no queued or running work may still read it.
int quiesce(Ctx &c) {
  if (int rc = run_queue(c)) return rc;
  cudaError_t e = cudaStreamSynchronize(c.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c.st2);
  if (e != cudaSuccess) return cuda_fail(e, "weight cache: stream");
  return 0;
}

// Free the least recently used copy that the current call has not resolved
// and that does not overlap [lo, hi) (first-use copies before registered
// ranges); false when there is none.
bool evict_one(Ctx &c, uintptr_t lo, uintptr_t hi, bool &quiet, int &rc) {
  auto best = c.ranges.end();
  for (auto it = c.ranges.begin(); it != c.ranges.end(); ++it) {
    const Range &r = it->second;
    if (r.last_use == c.call_no || (r.h < hi && lo < r.h + r.n)) continue;
    if (best == c.ranges.end() || r.registered < best->second.registered ||
        (r.registered == best->second.registered && r.last_use < best->second.last_use))
      best = it;
  }
  if (best == c.ranges.end()) return false;
  if (!quiet) {
    if ((rc = quiesce(c))) return false;
    quiet = true;
  }
  cudaFree(best->second.d);
  c.cached -= best->second.n;
  c.ranges.erase(best);
  return true;
}

// Device address of host bytes [h, h+n): the copy containing them, or a new
// copy.  A new copy spans the union of [h, h+n) and every copy it overlaps
// (those are freed), so the copies stay disjoint and a lookup is one
// predecessor search.  When the budget or the GPU's memory runs out, least
// recently used copies are evicted (never one the current call resolved) and
// the bytes are copied again when a later call needs them.
int dev_ptr(Ctx &c, const void *hp, size_t n, const void **out, bool registered = false) {
  if (!hp) return fail(FFN_B200_EINVAL, "reference ABI: null weight pointer");
  const uintptr_t h = (uintptr_t)hp;
  auto it = c.ranges.upper_bound(h);
  if (it != c.ranges.begin()) {
    auto p = std::prev(it);
    if (h + n <= p->second.h + p->second.n) {
      p->second.last_use = c.call_no;
      p->second.registered = p->second.registered || registered;
      *out = p->second.d + (h - p->second.h);
      return 0;
    }
    if (h < p->second.h + p->second.n) it = p;  // overlaps from below
  }
  uintptr_t lo = h, hi = h + n;
  std::vector<uintptr_t> merged;
  for (auto q = it; q != c.ranges.end() && q->second.h < hi; ++q) {
    if (q->second.last_use == c.call_no)  // this call holds an address in it: it must not move
      return fail(FFN_B200_EUNSUP, "reference ABI: weight ranges of one call overlap");
    lo = std::min(lo, q->second.h);
    hi = std::max(hi, q->second.h + q->second.n);
    registered = registered || q->second.registered;
    merged.push_back(q->first);
  }
  size_t freed = 0;
  for (uintptr_t k : merged) freed += c.ranges[k].n;
  const size_t need = hi - lo;
  bool quiet = false;
  int rc = 0;
  while (c.budget && c.cached - freed + need > c.budget)
    if (!evict_one(c, lo, hi, quiet, rc)) {
      if (rc) return rc;
      break;  // nothing evictable: go over the budget rather than fail the call
    }
  char *d = nullptr;
  cudaError_t e;
  while ((e = cudaMalloc(&d, need)) == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    if (!evict_one(c, lo, hi, quiet, rc)) return rc ? rc : cuda_fail(e, "cudaMalloc(weight copy)");
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(weight copy)");
  e = cudaMemcpy(d, reinterpret_cast<const void *>(lo), need, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "cudaMemcpy(weight upload)");
  }
  if (!merged.empty()) {
    if (!quiet && (rc = quiesce(c))) {
      cudaFree(d);
      return rc;
    }
    for (uintptr_t k : merged) {
      cudaFree(c.ranges[k].d);
      c.cached -= c.ranges[k].n;
      c.ranges.erase(k);
    }
  }
  c.ranges[lo] = Range{lo, need, d, c.call_no, registered};
  c.cached += need;
  *out = d + (h - lo);
  return 0;
}

// Wait until the stage's last upload has been read, and give it `bytes`.
int stage_ready(Ctx::Stage &s, size_t bytes) {
  if (s.used) {
    cudaError_t e = cudaEventSynchronize(s.ev);
    if (e != cudaSuccess) return cuda_fail(e, "host stage wait");
    s.used = false;
  }
  if (!s.ev) FFN_CUDA_TRY(cudaEventCreateWithFlags(&s.ev, cudaEventDisableTiming));
  if (bytes > s.n) {
    if (s.h) cudaFreeHost(s.h);
    s.h = nullptr;
    s.n = 0;
    const size_t want = std::max<size_t>(bytes, 64 << 10);
    FFN_CUDA_TRY(cudaHostAlloc(&s.h, want, cudaHostAllocDefault));
    s.n = want;
  }
  return 0;
}

// The stage's upload has been issued on the stream.
void stage_issued(Ctx &c, Ctx::Stage &s) {
  if (cudaEventRecord(s.ev, c.st) == cudaSuccess) s.used = true;
}

void clear_queue(Ctx &c) {
  c.queue.clear();
  c.q_xrows = 0;
  c.q_zero = false;
}

// Run the queued routed calls (in call order) into c.out.
int run_queue(Ctx &c) {
  if (c.queue.empty()) return 0;
  const int n = (int)c.queue.size(), R = c.q_out_rows;
  std::vector<ffn_b200_expert> es(n);
  std::vector<int32_t> row0(n), m(n), tok_ptr((size_t)R + 1, 0), pair, cur;
  std::vector<float> wts;
  int P = 0;
  for (int k = 0; k < n; ++k) {
    const Ctx::Call &q = c.queue[k];
    es[k] = q.e;
    row0[k] = q.row0;
    m[k] = q.m;
    for (int j = 0; j < q.m; ++j) ++tok_ptr[q.dst[j] + 1];
    P += q.m;
  }
  for (int r = 0; r < R; ++r) tok_ptr[r + 1] += tok_ptr[r];
  // combine list per out row, entries in call order
  pair.resize(P);
  wts.resize(P);
  cur.assign(tok_ptr.begin(), tok_ptr.end() - 1);
  for (int k = 0, pos = 0; k < n; ++k)
    for (int j = 0; j < c.queue[k].m; ++j, ++pos) {
      const int e = cur[c.queue[k].dst[j]]++;
      pair[e] = pos;
      wts[e] = c.queue[k].w[j];
    }
  const bool from_bx = c.q_src == 1;
  const int xrows = c.q_xrows;
  // the queue began with an overwriting call: every out row starts from zero
  // (accumulate mode: the one row; batched layer: the shared expert's rows,
  // which are all of them)
  std::vector<uint8_t> zero((size_t)R, c.q_zero ? 1 : 0);
  clear_queue(c);
  if (from_bx) {
    // the staged x rows, one pinned upload
    Ctx::Stage &xs = c.xstage[c.xstage_i];
    cudaError_t er = cudaMemcpyAsync(c.bx.p, xs.h, (size_t)xrows * c.q_hidden * 4, cudaMemcpyHostToDevice, c.st);
    if (er != cudaSuccess) return cuda_fail(er, "x rows upload");
    stage_issued(c, xs);
    c.xstage_i ^= 1;
  }
  ffn::RoutedCalls q{};
  q.experts = es.data();
  q.row0 = row0.data();
  q.m = m.data();
  q.n = n;
  q.tok_ptr = tok_ptr.data();
  q.ent_pair = pair.data();
  q.ent_w = wts.data();
  q.out_rows = R;
  q.row_zero = zero.data();
  q.x = (const float *)(from_bx ? c.bx.p : c.xall.p);
  q.x_rows = from_bx ? xrows : (int)c.xall_tok;
  q.out = (float *)c.out.p;
  q.side = c.st2;
  q.fork = c.ev_fork;
  q.join = c.ev_join;
  int rc = c.ws.ensure(ffn::routed_calls_ws_bytes(c.q_inter, c.q_hidden, n, q.x_rows, R));
  Ctx::Stage &s = c.stage[c.stage_i];
  if (!rc) rc = stage_ready(s, ffn::routed_calls_stage_bytes(n, R));
  if (!rc) {
    rc = ffn::routed_calls(q, c.q_inter, c.q_hidden, s.h, c.ws.p, c.ws.n, c.st);
    stage_issued(c, s);
    c.stage_i ^= 1;
  }
  return rc;
}

// The host reads a fused call's `out` only after the call of the sequence that
// passes sync_now (flash1017.rs:7440-7512, 8193-8262).  A sequence it abandons
// (it breaks out of the loop and recomputes on its CPU path, dropping the
// buffer: flash1017.rs:7483-7486, 8228-8229) is never written back, because
// that memory may already be freed: the next call of any kind drops it.
void drop_pending(Ctx &c) {
  clear_queue(c);
  c.pend_host = nullptr;
  c.pend_n = 0;
}

// Run the queue and copy the result into the host's `out`: only while serving
// a sync_now call that passed that same pointer.
int deliver_pending(Ctx &c) {
  if (int rc = run_queue(c)) {
    c.pend_host = nullptr;
    c.pend_n = 0;
    return rc;
  }
  if (!c.pend_host) return 0;
  cudaError_t e = cudaMemcpyAsync(c.pend_host, c.out.p, c.pend_n * sizeof(float),
                                  cudaMemcpyDeviceToHost, c.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c.st);
  c.pend_host = nullptr;
  c.pend_n = 0;
  if (e != cudaSuccess) return cuda_fail(e, "pending out download");
  return 0;
}

void fill_nan(float *out, size_t n) {
  if (!out) return;
  const float q = std::nanf("");
  for (size_t i = 0; i < n; ++i) out[i] = q;
}

// Stage x, run `body(ctx, dx, dout)`, copy out back, synchronise.  void-returning
// ABI: on failure `out` is NaN-filled and the error is recorded.
template <class F>
void run_sync(size_t x_n, const float *x, size_t out_n, float *out, F body) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  int rc = ensure_init(c);
  drop_pending(c);
  if (!rc && (!x || !out)) rc = fail(FFN_B200_EINVAL, "reference ABI: null x/out");
  if (!rc) rc = c.x.ensure(x_n * sizeof(float));
  if (!rc) rc = c.out.ensure(out_n * sizeof(float));
  if (!rc) {
    cudaError_t e = cudaMemcpyAsync(c.x.p, x, x_n * sizeof(float), cudaMemcpyHostToDevice, c.st);
    if (e != cudaSuccess) rc = cuda_fail(e, "x upload");
  }
  if (!rc) rc = body(c, (const float *)c.x.p, (float *)c.out.p);
  if (!rc) {
    cudaError_t e = cudaMemcpyAsync(out, c.out.p, out_n * sizeof(float), cudaMemcpyDeviceToHost, c.st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.st);
    if (e != cudaSuccess) rc = cuda_fail(e, "out download");
  }
  if (rc) {
    std::fprintf(stderr, "[ffn_b200] %s\n", ffn_b200_last_error());
    fill_nan(out, out_n);
  }
}

// ------------------------------------------------------------- V1 dots
float dot_common(int mode, const void *a, size_t a_bytes, const void *aux, size_t aux_bytes,
                 const float *x, size_t x_n) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  float r = std::nanf("");
  int rc = ensure_init(c);
  drop_pending(c);
  if (!rc && (!a || !x)) rc = fail(FFN_B200_EINVAL, "dot: null pointer");
  if (!rc) rc = c.tmp.ensure(a_bytes + aux_bytes + x_n * 4 + 1024);
  if (!rc) {
    char *base = (char *)c.tmp.p;
    char *da = base, *daux = base + ((a_bytes + 255) & ~(size_t)255);
    char *dx = daux + ((aux_bytes + 255) & ~(size_t)255);
    float *dr = (float *)(dx + ((x_n * 4 + 255) & ~(size_t)255));
    cudaError_t e = cudaMemcpyAsync(da, a, a_bytes, cudaMemcpyHostToDevice, c.st);
    if (e == cudaSuccess && aux_bytes) e = cudaMemcpyAsync(daux, aux, aux_bytes, cudaMemcpyHostToDevice, c.st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dx, x, x_n * 4, cudaMemcpyHostToDevice, c.st);
    if (e != cudaSuccess) rc = cuda_fail(e, "dot upload");
    if (!rc) rc = launch_dot(mode, da, daux, (const float *)dx, x_n, dr, c.st);
    if (!rc) {
      e = cudaMemcpyAsync(&r, dr, 4, cudaMemcpyDeviceToHost, c.st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(c.st);
      if (e != cudaSuccess) rc = cuda_fail(e, "dot download");
    }
  }
  if (rc) std::fprintf(stderr, "[ffn_b200] %s\n", ffn_b200_last_error());
  return r;
}

float v1_dot_f32(const float *a, const float *b, size_t len) {
  return dot_common(0, a, len * 4, nullptr, 0, b, len);
}
float v1_dot_i8_f32(const int8_t *w, const float *x, size_t len) {
  return dot_common(1, w, len, nullptr, 0, x, len);
}
float v1_dot_q4_g32_f32(const uint8_t *nib, const uint16_t *sc, const float *x, size_t cols) {
  return dot_common(2, nib, cols / 2, sc, (cols / 32) * 2, x, cols);
}
float v1_dot_ternary_2bit_f32(const uint8_t *p, const float *x, size_t cols) {
  return dot_common(3, p, cols / 4, nullptr, 0, x, cols);
}

// ------------------------------------------------------------ V2/V3 matvecs
void v3_matbatch_bf16(size_t rows, size_t cols, size_t seq, const uint16_t *w, const float *xb,
                      float *ob) {
  run_sync(seq * cols, xb, seq * rows, ob, [&](Ctx &c, const float *dx, float *dout) {
    if (!w || rows == 0 || cols == 0) return fail(FFN_B200_EINVAL, "matbatch_bf16: bad arguments");
    const void *dw;
    int rc = dev_ptr(c, w, rows * cols * 2, &dw);
    if (rc) return rc;
    // exact sequential sum per row (flash1017.rs:2212-2226)
    return launch_exact_matvec(nullptr, (const uint16_t *)dw, dx, (int)seq, (int)rows, (int)cols,
                               dout, c.st);
  });
}
void v2_matvec_bf16(size_t rows, size_t cols, const uint16_t *w, const float *x, float *out) {
  v3_matbatch_bf16(rows, cols, 1, w, x, out);
}

void v3_matbatch_nvfp4(size_t rows, size_t cols, size_t seq, const uint8_t *w, const uint8_t *s,
                       float gs, const float *xb, float *ob) {
  run_sync(seq * cols, xb, seq * rows, ob, [&](Ctx &c, const float *dx, float *dout) {
    if (!w || !s || cols % 16) return fail(FFN_B200_EINVAL, "matbatch_nvfp4: bad arguments");
    ffn_b200_nvfp4_mat m{};
    const void *dw, *ds;
    int rc = dev_ptr(c, w, rows * cols / 2, &dw);
    if (!rc) rc = dev_ptr(c, s, rows * cols / 16, &ds);
    if (rc) return rc;
    m.w = (const uint8_t *)dw;
    m.s = (const uint8_t *)ds;
    m.gs = gs;
    if ((rc = c.ws.ensure(ffn_b200_matvec_ws_bytes(seq, cols)))) return rc;
    return ffn_b200_nvfp4_matvec(rows, cols, seq, &m, dx, dout, c.ws.p, c.ws.n, c.st);
  });
}
void v3_matvec_nvfp4(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s, float gs,
                     const float *x, float *out) {
  v3_matbatch_nvfp4(rows, cols, 1, w, s, gs, x, out);
}

void v3_matbatch_ternary(size_t rows, size_t cols, size_t seq, const uint8_t *p, const float *rs,
                         const float *xb, float *ob) {
  run_sync(seq * cols, xb, seq * rows, ob, [&](Ctx &c, const float *dx, float *dout) {
    if (!p || !rs || cols % 4) return fail(FFN_B200_EINVAL, "matbatch_ternary_158: bad arguments");
    ffn_b200_ternary_mat m{};
    const void *dp, *drs;
    int rc = dev_ptr(c, p, rows * cols / 4, &dp);
    if (!rc) rc = dev_ptr(c, rs, rows * 4, &drs);
    if (rc) return rc;
    m.p = (const uint8_t *)dp;
    m.rs = (const float *)drs;
    if ((rc = c.ws.ensure(ffn_b200_matvec_ws_bytes(seq, cols)))) return rc;
    return ffn_b200_ternary_matvec(rows, cols, seq, &m, dx, dout, c.ws.p, c.ws.n, c.st);
  });
}
void v3_matvec_ternary(size_t rows, size_t cols, const uint8_t *p, const float *rs,
                       const float *x, float *out) {
  v3_matbatch_ternary(rows, cols, 1, p, rs, x, out);
}

const char kId[] = "addon_b200_ffn";
const char kDesc[] =
    "B200 (sm_100a) quantized expert-FFN backend: NVFP4 + 1.58-bit ternary (+rank-16 Q8) "
    "tensor-core GEMV/GEMM, routed SwiGLU MoE";

// MXFP8 post-scale 2^B from the host scale bytes: the largest finite E8M0
// scale decodes to 2^7 (E4M3 448 x 2^7 < 65504, FFN_B200_FMT_MXFP8).
// Power-of-two post-scales gs = 2^B of E8M0 scale arrays, B = (largest finite
// scale byte) - top, so the largest block decodes to 2^(top - 127) in f16:
// top 134 for MXFP8 (E4M3 448 x 2^7 < 65504), 140 for MXFP4 (E2M1 6 x 2^13).
// Computed once per array: the host keeps a scale array's bytes unchanged
// while the process runs (the same assumption as the weight copies;
// ffn_b200_release_host_ranges drops both).
struct GsCache {
  std::mutex mu;
  std::map<std::pair<uintptr_t, size_t>, float> m;
};
GsCache &gs_cache() {
  static GsCache *g = new GsCache();
  return *g;
}

float mx_gs(const uint8_t *s, size_t n, int top) {
  GsCache &g = gs_cache();
  const std::pair<uintptr_t, size_t> key((uintptr_t)s, n * 256 + (size_t)top);
  {
    std::lock_guard<std::mutex> lk(g.mu);
    auto it = g.m.find(key);
    if (it != g.m.end()) return it->second;
  }
  int mx = -1;
  for (size_t q = 0; q < n; ++q)
    if (s[q] != 0xFF && s[q] > mx) mx = s[q];
  const float gs = std::ldexp(1.0f, mx < 0 ? 0 : mx - top);
  std::lock_guard<std::mutex> lk(g.mu);
  g.m[key] = gs;
  return gs;
}
float mxfp8_gs(const uint8_t *s, size_t n) { return mx_gs(s, n, 134); }
float mxfp4_gs(const uint8_t *s, size_t n) { return mx_gs(s, n, 140); }

void v3_matbatch_mxfp8(size_t rows, size_t cols, size_t seq, const uint8_t *w, const uint8_t *s,
                       const float *xb, float *ob) {
  run_sync(seq * cols, xb, seq * rows, ob, [&](Ctx &c, const float *dx, float *dout) {
    if (!w || !s || cols % 128) return fail(FFN_B200_EINVAL, "matbatch_mxfp8: bad arguments");
    const size_t sn = ((rows + 31) / 32) * (cols / 32);
    ffn_b200_nvfp4_mat m{};
    const void *dw, *ds;
    int rc = dev_ptr(c, w, rows * cols, &dw);
    if (!rc) rc = dev_ptr(c, s, sn, &ds);
    if (rc) return rc;
    m.w = (const uint8_t *)dw;
    m.s = (const uint8_t *)ds;
    m.gs = mxfp8_gs(s, sn);
    if ((rc = c.ws.ensure(ffn_b200_matvec_ws_bytes(seq, cols)))) return rc;
    return ffn_b200_mxfp8_matvec(rows, cols, seq, &m, dx, dout, c.ws.p, c.ws.n, c.st);
  });
}
void v3_matvec_mxfp8(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s, const float *x,
                     float *out) {
  v3_matbatch_mxfp8(rows, cols, 1, w, s, x, out);
}

HardwareAddonVTable make_vtable() {
  HardwareAddonVTable v;
  std::memset(&v, 0, sizeof(v));
  v.abi_version = MERKABA_HW_ABI_V3;
  v.addon_id_ptr = (const uint8_t *)kId;
  v.addon_id_len = sizeof(kId) - 1;
  v.addon_desc_ptr = (const uint8_t *)kDesc;
  v.addon_desc_len = sizeof(kDesc) - 1;
  v.dot_f32 = v1_dot_f32;
  v.dot_i8_f32 = v1_dot_i8_f32;
  v.dot_q4_g32_f32 = v1_dot_q4_g32_f32;
  v.dot_ternary_2bit_f32 = v1_dot_ternary_2bit_f32;
  v.matvec_bf16 = v2_matvec_bf16;
  v.matbatch_bf16 = v3_matbatch_bf16;
  v.matvec_nvfp4 = v3_matvec_nvfp4;
  v.matbatch_nvfp4 = v3_matbatch_nvfp4;
  v.matvec_ternary_158 = v3_matvec_ternary;
  v.matbatch_ternary_158 = v3_matbatch_ternary;
  v.matvec_mxfp8 = v3_matvec_mxfp8;
  v.matbatch_mxfp8 = v3_matbatch_mxfp8;
  return v;
}

// ---------------------------------------------------------- fused experts
int resolve_expert(Ctx &c, ffn_b200_expert &e, size_t inter, size_t hidden) {
  for (int i = 0; i < 3; ++i) {
    const size_t r = i == 2 ? hidden : inter, k = i == 2 ? inter : hidden;
    const void *a, *b;
    int rc;
    if (e.format == FFN_B200_FMT_MXFP8) {
      if ((rc = dev_ptr(c, e.nv[i].w, r * k, &a))) return rc;
      if ((rc = dev_ptr(c, e.nv[i].s, ((r + 31) / 32) * ((k + 31) / 32), &b))) return rc;
      e.nv[i].w = (const uint8_t *)a;
      e.nv[i].s = (const uint8_t *)b;
    } else if (e.format == FFN_B200_FMT_NVFP4 || e.format == FFN_B200_FMT_MXFP4) {
      if ((rc = dev_ptr(c, e.nv[i].w, r * k / 2, &a))) return rc;
      if ((rc = dev_ptr(c, e.nv[i].s, r * k / (e.format == FFN_B200_FMT_MXFP4 ? 32 : 16), &b))) return rc;
      e.nv[i].w = (const uint8_t *)a;
      e.nv[i].s = (const uint8_t *)b;
    } else {
      if ((rc = dev_ptr(c, e.tn[i].p, r * k / 4, &a))) return rc;
      if ((rc = dev_ptr(c, e.tn[i].rs, r * 4, &b))) return rc;
      e.tn[i].p = (const uint8_t *)a;
      e.tn[i].rs = (const float *)b;
    }
  }
  return 0;
}

// Queue one routed call (the caller holds the lock and has made c.out the
// call's target); the queue runs when it is full.
int enqueue(Ctx &c, const ffn_b200_expert &e, int src, size_t inter, size_t hidden, int out_rows,
            int32_t row0, int32_t m, const int32_t *dst, const float *w) {
  Ctx::Call q{};
  q.e = e;
  q.row0 = row0;
  q.m = m;
  for (int j = 0; j < m; ++j) {
    q.dst[j] = dst[j];
    q.w[j] = w[j];
  }
  c.queue.push_back(q);
  c.q_src = src;
  c.q_inter = inter;
  c.q_hidden = hidden;
  c.q_out_rows = out_rows;
  return c.queue.size() == (size_t)ffn::kCallsMax ? run_queue(c) : 0;
}

// Stage one call's x row in the queue's pinned x stage; `row` = its index.
int stage_x(Ctx &c, const float *x, size_t hidden, int32_t *row) {
  Ctx::Stage &xs = c.xstage[c.xstage_i];
  if (c.queue.empty()) {  // a new queue takes the next stage
    c.q_xrows = 0;
    if (int rc = stage_ready(xs, (size_t)ffn::kCallsMax * hidden * 4)) return rc;
  }
  float *rows = (float *)xs.h;
  const size_t nb = hidden * 4;
  if (c.q_xrows > 0 && std::memcmp(rows + (size_t)(c.q_xrows - 1) * hidden, x, nb) == 0) {
    *row = c.q_xrows - 1;  // the same x as the previous call (the reference's routed calls)
    return 0;
  }
  std::memcpy(rows + (size_t)c.q_xrows * hidden, x, nb);
  *row = c.q_xrows++;
  return 0;
}

// Shared by the *_mlp_accum entry points: x is one token, out [hidden].  Every
// call is queued, and the queue runs as one routed layer (calls in order) when
// the host needs `out`: sync_now, another target or dims, 64 calls, or another
// entry point.  An overwriting call (accumulate = false) starts a new queue
// whose output starts from zero; the reference's sequence per token (shared
// expert overwriting, then the routed experts accumulating, sync on the last,
// flash1017.rs:7401-7512) thus runs as one layer of 7 experts.
bool mlp_accum(const ffn_b200_expert &he, size_t inter, size_t hidden, const float *x, float *out,
               float w, bool accumulate, bool sync_now) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  int rc = ensure_init(c);
  if (!rc && (!x || !out)) rc = fail(FFN_B200_EINVAL, "mlp_accum: null x/out");
  // Another target, other dims, or an overwriting call (which replaces the
  // whole row) begin a new sequence: the unsynced one is dropped.
  if (c.pend_host && (c.pend_host != out || c.pend_n != hidden)) drop_pending(c);
  if (!c.queue.empty() && (c.q_src != 1 || c.q_inter != inter || c.q_hidden != hidden || !accumulate))
    drop_pending(c);
  if (!rc) rc = c.out.ensure(hidden * 4);
  if (!rc) rc = c.bx.ensure((size_t)ffn::kCallsMax * hidden * 4);
  ffn_b200_expert e = he;
  // shapes before any weight byte is read; the rest on the device copies
  if (!rc) rc = ffn::validate_expert_shape(e.format, inter, hidden, "mlp_accum");
  if (!rc) rc = resolve_expert(c, e, inter, hidden);
  if (!rc) rc = ffn::validate_expert(e, inter, hidden, "mlp_accum");
  if (!rc && accumulate && !c.pend_host) {
    // accumulate onto the host's current contents
    cudaError_t er = cudaMemcpyAsync(c.out.p, out, hidden * 4, cudaMemcpyHostToDevice, c.st);
    if (er != cudaSuccess) rc = cuda_fail(er, "out upload");
  }
  int32_t row = 0;
  const int32_t dst0 = 0;
  if (!rc) rc = stage_x(c, x, hidden, &row);
  if (!rc) {
    if (!accumulate) c.q_zero = true;  // the queue is empty here: this is its first call
    rc = enqueue(c, e, 1, inter, hidden, 1, row, 1, &dst0, &w);
  }
  if (!rc) {
    c.pend_host = out;
    c.pend_n = hidden;
    if (sync_now) rc = deliver_pending(c);
  }
  if (rc) {
    std::fprintf(stderr, "[ffn_b200] %s\n", ffn_b200_last_error());
    drop_pending(c);
    return false;
  }
  return true;
}

// Upload the host's x_all rows if they are not on the device yet.
int ensure_xall(Ctx &c) {
  if (c.xall_dev_valid) return 0;
  int rc = c.xall.ensure(c.xall_tok * c.xall_hidden * 4);
  if (rc) return rc;
  cudaError_t er = cudaMemcpyAsync(c.xall.p, c.xall_host, c.xall_tok * c.xall_hidden * 4,
                                   cudaMemcpyHostToDevice, c.st);
  if (er != cudaSuccess) return cuda_fail(er, "x_all upload");
  c.xall_dev_valid = true;
  return 0;
}

// Shared by the *_mlp_batch entry points (HA:441-479, call site
// flash1017.rs:8193-8262): expert(x_all rows x_off .. x_off + m - 1), row k
// added to out_batch row dst[k] with weight wscale * dw[k].  The calls are
// queued (one routed layer at sync_now).  wscale is the ternary proj_scale:
// the host passes unscaled weights here, and its CPU twin adds weight * sc
// (flash1017.rs:8317-8321).
bool mlp_batch(const ffn_b200_expert &he, float wscale, size_t inter, size_t hidden, size_t m,
               size_t x_off, const size_t *dst, const float *dw, size_t b_len, float *out,
               bool sync_now) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  int rc = ensure_init(c);
  if (!rc && (!dst || !dw || !out)) rc = fail(FFN_B200_EINVAL, "mlp_batch: null pointer");
  if (!rc && (!c.xall_host || c.xall_hidden != hidden || x_off + m > c.xall_tok))
    rc = fail(FFN_B200_EINVAL, "mlp_batch: x rows outside the x_all of the layer's mxfp8_mlp_batch call");
  if (!rc && (m == 0 || m > 8)) rc = fail(FFN_B200_EINVAL, "mlp_batch: 1..8 tokens per call");
  if (!rc && (b_len == 0 || b_len > 65535)) rc = fail(FFN_B200_EINVAL, "mlp_batch: b_len must be 1..65535");
  for (size_t k = 0; !rc && k < m; ++k)
    if (dst[k] >= b_len) rc = fail(FFN_B200_EINVAL, "mlp_batch: destination token out of range");
  if (c.pend_host && (c.pend_host != out || c.pend_n != b_len * hidden)) drop_pending(c);
  if (!c.queue.empty() && (c.q_src != 2 || c.q_inter != inter || c.q_hidden != hidden)) drop_pending(c);
  if (!rc) rc = c.out.ensure(b_len * hidden * 4);
  if (!rc) rc = ensure_xall(c);
  ffn_b200_expert e = he;
  if (!rc) rc = ffn::validate_expert_shape(e.format, inter, hidden, "mlp_batch");
  if (!rc) rc = resolve_expert(c, e, inter, hidden);
  if (!rc) rc = ffn::validate_expert(e, inter, hidden, "mlp_batch");
  if (!rc && e.format == FFN_B200_FMT_MXFP8) rc = fail(FFN_B200_EINVAL, "mlp_batch: MXFP8 expert");
  if (!rc && !c.pend_host) {
    cudaError_t er = cudaMemcpyAsync(c.out.p, out, b_len * hidden * 4, cudaMemcpyHostToDevice, c.st);
    if (er != cudaSuccess) rc = cuda_fail(er, "out_batch upload");
  }
  if (!rc) {
    int32_t d32[8];
    float w8[8];
    for (size_t k = 0; k < m; ++k) {
      d32[k] = (int32_t)dst[k];
      w8[k] = dw[k] * wscale;
    }
    rc = enqueue(c, e, 2, inter, hidden, (int)b_len, (int32_t)x_off, (int32_t)m, d32, w8);
  }
  if (!rc) {
    c.pend_host = out;
    c.pend_n = b_len * hidden;
    if (sync_now) rc = deliver_pending(c);
  }
  if (rc) {
    std::fprintf(stderr, "[ffn_b200] %s\n", ffn_b200_last_error());
    drop_pending(c);
    return false;
  }
  return true;
}

ffn_b200_expert nvfp4_expert(const uint8_t *w1, const uint8_t *s1, float g1, const uint8_t *w3,
                             const uint8_t *s3, float g3, const uint8_t *w2, const uint8_t *s2,
                             float g2) {
  ffn_b200_expert e{};
  e.format = FFN_B200_FMT_NVFP4;
  e.proj_scale = 1.0f;
  e.nv[0] = {w1, s1, g1, 0};
  e.nv[1] = {w3, s3, g3, 0};
  e.nv[2] = {w2, s2, g2, 0};
  return e;
}

ffn_b200_expert ternary_expert(const uint8_t *p1, const float *r1, const uint8_t *p3,
                               const float *r3, const uint8_t *p2, const float *r2, float sc) {
  ffn_b200_expert e{};
  e.format = FFN_B200_FMT_TERNARY;
  e.proj_scale = sc;
  e.tn[0].p = p1; e.tn[0].rs = r1;
  e.tn[1].p = p3; e.tn[1].rs = r3;
  e.tn[2].p = p2; e.tn[2].rs = r2;
  return e;
}

}  // namespace
}  // namespace ffn

using namespace ffn;

extern "C" {

const HardwareAddonVTable *merkaba_hardware_addon_v1(void) {
  static const HardwareAddonVTable vt = make_vtable();
  return &vt;
}

bool gx10_rust_nvfp4_mlp_accum(size_t inter_rows, size_t hidden_cols, const uint8_t *w1_fp4,
                               const uint8_t *w1_s, float w1_sc2, const uint8_t *w3_fp4,
                               const uint8_t *w3_s, float w3_sc2, const uint8_t *w2_fp4,
                               const uint8_t *w2_s, float w2_sc2, const float *x, float *out,
                               float accum_weight, bool accumulate, bool sync_now) {
  const ffn_b200_expert e =
      nvfp4_expert(w1_fp4, w1_s, w1_sc2, w3_fp4, w3_s, w3_sc2, w2_fp4, w2_s, w2_sc2);
  return mlp_accum(e, inter_rows, hidden_cols, x, out, accum_weight, accumulate, sync_now);
}

bool gx10_rust_mxfp4_mlp_accum(size_t inter_rows, size_t hidden_cols, const uint8_t *w1_fp4,
                               const uint8_t *w1_s, const uint8_t *w3_fp4, const uint8_t *w3_s,
                               const uint8_t *w2_fp4, const uint8_t *w2_s, const float *x, float *out,
                               float accum_weight, bool accumulate, bool sync_now) {
  ffn_b200_expert e{};
  e.format = FFN_B200_FMT_MXFP4;
  e.proj_scale = 1.0f;
  const uint8_t *w[3] = {w1_fp4, w3_fp4, w2_fp4}, *sc[3] = {w1_s, w3_s, w2_s};
  // the scale arrays are read only for shapes that pass (mlp_accum reports the error)
  const bool shape_ok = ffn::validate_expert_shape(e.format, inter_rows, hidden_cols, "mxfp4_mlp_accum") == 0;
  for (int i = 0; i < 3; ++i) {
    const size_t r = i == 2 ? hidden_cols : inter_rows, k = i == 2 ? inter_rows : hidden_cols;
    e.nv[i].w = w[i];
    e.nv[i].s = sc[i];
    // the reference's MXFP4 tensors have no global scale: gs is only the
    // power-of-two bias of the f16 decode
    e.nv[i].gs = sc[i] && shape_ok ? mxfp4_gs(sc[i], r * (k / 32)) : 1.0f;
  }
  return mlp_accum(e, inter_rows, hidden_cols, x, out, accum_weight, accumulate, sync_now);
}

bool gx10_rust_mxfp8_mlp_accum(size_t inter_rows, size_t hidden_cols, const uint8_t *w1_w,
                               const uint8_t *w1_s, const uint8_t *w3_w, const uint8_t *w3_s,
                               const uint8_t *w2_w, const uint8_t *w2_s, const float *x, float *out,
                               float accum_weight, bool accumulate, bool sync_now) {
  ffn_b200_expert e{};
  e.format = FFN_B200_FMT_MXFP8;
  e.proj_scale = 1.0f;
  const uint8_t *w[3] = {w1_w, w3_w, w2_w}, *sc[3] = {w1_s, w3_s, w2_s};
  // the scale arrays are read only for shapes that pass (mlp_accum reports the error)
  const bool shape_ok = ffn::validate_expert_shape(e.format, inter_rows, hidden_cols, "mxfp8_mlp_accum") == 0;
  for (int i = 0; i < 3; ++i) {
    const size_t r = i == 2 ? hidden_cols : inter_rows, k = i == 2 ? inter_rows : hidden_cols;
    e.nv[i].w = w[i];
    e.nv[i].s = sc[i];
    e.nv[i].gs = sc[i] && shape_ok ? mxfp8_gs(sc[i], ((r + 31) / 32) * ((k + 31) / 32)) : 1.0f;
  }
  return mlp_accum(e, inter_rows, hidden_cols, x, out, accum_weight, accumulate, sync_now);
}

bool gx10_rust_mxfp4_matvec(size_t rows, size_t cols, const uint8_t *packed_fp4,
                            const uint8_t *scales_e8m0, const float *x, float *out) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  int rc = ensure_init(c);
  drop_pending(c);  // an unsynced fused-expert sequence was abandoned
  if (!rc && (!packed_fp4 || !scales_e8m0 || !x || !out || cols % 128))
    rc = fail(FFN_B200_EINVAL, "mxfp4_matvec: bad arguments");
  const void *dw = nullptr, *ds = nullptr;
  if (!rc) rc = dev_ptr(c, packed_fp4, rows * cols / 2, &dw);
  if (!rc) rc = dev_ptr(c, scales_e8m0, rows * cols / 32, &ds);
  if (!rc) rc = c.x.ensure(cols * 4);
  if (!rc) rc = c.out.ensure(rows * 4);
  if (!rc) rc = c.ws.ensure(ffn_b200_matvec_ws_bytes(1, cols));
  if (!rc) {
    cudaError_t er = cudaMemcpyAsync(c.x.p, x, cols * 4, cudaMemcpyHostToDevice, c.st);
    if (er != cudaSuccess) rc = cuda_fail(er, "x upload");
  }
  if (!rc) {
    ffn_b200_nvfp4_mat m{};
    m.w = (const uint8_t *)dw;
    m.s = (const uint8_t *)ds;
    m.gs = mxfp4_gs(scales_e8m0, rows * (cols / 32));  // the f16 decode's power-of-two bias
    rc = ffn_b200_mxfp4_matvec(rows, cols, 1, &m, (const float *)c.x.p, (float *)c.out.p, c.ws.p, c.ws.n,
                               c.st);
  }
  if (!rc) {
    cudaError_t er = cudaMemcpyAsync(out, c.out.p, rows * 4, cudaMemcpyDeviceToHost, c.st);
    if (er == cudaSuccess) er = cudaStreamSynchronize(c.st);
    if (er != cudaSuccess) rc = cuda_fail(er, "out download");
  }
  if (rc) {
    std::fprintf(stderr, "[ffn_b200] %s\n", ffn_b200_last_error());
    return false;
  }
  return true;
}

bool gx10_rust_ternary_158_mlp_accum(size_t inter_rows, size_t hidden_cols, const uint8_t *w1_p,
                                     const float *w1_s, const uint8_t *w3_p, const float *w3_s,
                                     const uint8_t *w2_p, const float *w2_s, float proj_scale,
                                     const float *x, float *out, float accum_weight,
                                     bool accumulate, bool sync_now) {
  const ffn_b200_expert e = ternary_expert(w1_p, w1_s, w3_p, w3_s, w2_p, w2_s, proj_scale);
  return mlp_accum(e, inter_rows, hidden_cols, x, out, accum_weight, accumulate, sync_now);
}

bool gx10_rust_nvfp4_mlp_batch(size_t inter_rows, size_t hidden_cols, size_t seq_len,
                               const uint8_t *w1_fp4, const uint8_t *w1_s, float w1_sc2,
                               const uint8_t *w3_fp4, const uint8_t *w3_s, float w3_sc2,
                               const uint8_t *w2_fp4, const uint8_t *w2_s, float w2_sc2,
                               size_t x_tok_offset, const size_t *dst_tok_indices,
                               const float *dst_weights, size_t b_len, float *out_batch,
                               bool sync_now) {
  const ffn_b200_expert e =
      nvfp4_expert(w1_fp4, w1_s, w1_sc2, w3_fp4, w3_s, w3_sc2, w2_fp4, w2_s, w2_sc2);
  return mlp_batch(e, 1.0f, inter_rows, hidden_cols, seq_len, x_tok_offset, dst_tok_indices,
                   dst_weights, b_len, out_batch, sync_now);
}

bool gx10_rust_ternary_158_mlp_batch(size_t inter_rows, size_t hidden_cols, size_t seq_len,
                                     const uint8_t *w1_p, const float *w1_s, const uint8_t *w3_p,
                                     const float *w3_s, const uint8_t *w2_p, const float *w2_s,
                                     float proj_scale, size_t x_tok_offset,
                                     const size_t *dst_tok_indices, const float *dst_weights,
                                     size_t b_len, float *out_batch, bool sync_now) {
  const ffn_b200_expert e = ternary_expert(w1_p, w1_s, w3_p, w3_s, w2_p, w2_s, proj_scale);
  return mlp_batch(e, proj_scale, inter_rows, hidden_cols, seq_len, x_tok_offset, dst_tok_indices,
                   dst_weights, b_len, out_batch, sync_now);
}

bool gx10_rust_mxfp8_mlp_batch(size_t inter_rows, size_t hidden_cols, size_t seq_len,
                               const uint8_t *w1_w, const uint8_t *w1_s, const uint8_t *w3_w,
                               const uint8_t *w3_s, const uint8_t *w2_w, const uint8_t *w2_s,
                               const float *x_all, size_t x_total_tokens, float *out_batch,
                               bool sync_now) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  int rc = ensure_init(c);
  const size_t b_len = seq_len, H = hidden_cols, I = inter_rows;
  if (!rc && (seq_len >> 31))
    rc = fail(FFN_B200_EUNSUP,
              "mxfp8_mlp_batch: the NVFP4 q4-backbone shared expert (seq_len bit 31) is not supported");
  if (!rc && (!x_all || !out_batch)) rc = fail(FFN_B200_EINVAL, "mxfp8_mlp_batch: null x_all/out_batch");
  if (!rc && (b_len == 0 || b_len > 65535 || b_len > x_total_tokens || x_total_tokens > (1u << 20)))
    rc = fail(FFN_B200_EINVAL, "mxfp8_mlp_batch: need 1 <= seq_len <= min(x_total_tokens, 65535)");
  drop_pending(c);  // a new layer: an unsynced earlier one was abandoned
  if (!rc) {
    // x_all also holds the rows of this layer's routed *_mlp_batch calls
    c.xall_host = x_all;
    c.xall_tok = x_total_tokens;
    c.xall_hidden = H;
    c.xall_dev_valid = false;
    rc = ensure_xall(c);
  }
  ffn_b200_expert e{};
  e.format = FFN_B200_FMT_MXFP8;
  e.proj_scale = 1.0f;
  const uint8_t *w[3] = {w1_w, w3_w, w2_w}, *sc[3] = {w1_s, w3_s, w2_s};
  if (!rc) rc = ffn::validate_expert_shape(e.format, I, H, "mxfp8_mlp_batch");
  for (int i = 0; i < 3; ++i) {
    const size_t r = i == 2 ? H : I, k = i == 2 ? I : H;
    e.nv[i].w = w[i];
    e.nv[i].s = sc[i];
    e.nv[i].gs = sc[i] && !rc ? mxfp8_gs(sc[i], ((r + 31) / 32) * ((k + 31) / 32)) : 1.0f;
  }
  if (!rc) rc = resolve_expert(c, e, I, H);
  if (!rc) rc = ffn::validate_expert(e, I, H, "mxfp8_mlp_batch");
  if (!rc) rc = c.out.ensure(b_len * H * 4);
  if (!rc && b_len <= (size_t)kNTok) {
    // one slice: queued as the layer's first call (its rows start from
    // zero), so the layer's routed calls run with it as one routed layer
    int32_t dst[kNTok];
    float w1[kNTok];
    for (size_t t = 0; t < b_len; ++t) {
      dst[t] = (int32_t)t;
      w1[t] = 1.0f;
    }
    c.q_zero = true;
    rc = enqueue(c, e, 2, I, H, (int)b_len, 0, (int32_t)b_len, dst, w1);
  } else {
    if (!rc) rc = c.ws.ensure(ffn_b200_expert_ws_bytes(I, H, b_len));
    if (!rc)
      rc = ffn_b200_expert_forward(I, H, b_len, &e, (const float *)c.xall.p, (float *)c.out.p, 1.0f, 0,
                                   c.ws.p, c.ws.n, c.st);
  }
  if (!rc) {
    c.pend_host = out_batch;
    c.pend_n = b_len * H;
    if (sync_now) rc = deliver_pending(c);
  }
  if (rc) {
    std::fprintf(stderr, "[ffn_b200] %s\n", ffn_b200_last_error());
    drop_pending(c);
    return false;
  }
  return true;
}

void gx10_rust_register_host_range(const void *ptr, size_t bytes) {
  if (!ptr || !bytes) return;
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  const void *d;
  if (ensure_init(c) || dev_ptr(c, ptr, bytes, &d, true))
    std::fprintf(stderr, "[ffn_b200] register_host_range: %s\n", ffn_b200_last_error());
}

void gx10_rust_register_shard_bounds(const void *ptr, size_t bytes) {
  if (!ptr || !bytes) return;
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  // Shards are many GB; their tensors are copied on first use (dev_ptr).
  c.shard_bounds.emplace_back((uintptr_t)ptr, bytes);
}

int ffn_b200_set_batch_input(const float *x_all_host, size_t x_total_tokens, size_t hidden) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  // queued *_mlp_batch calls read the current device copy of x_all
  if (c.q_src == 2) {
    if (int rc = run_queue(c)) return rc;
  }
  c.xall_host = x_all_host;
  c.xall_tok = x_total_tokens;
  c.xall_hidden = hidden;
  c.xall_dev_valid = false;
  return 0;
}

int ffn_b200_release_host_ranges(void) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  // queued calls read the device copies freed here: an unsynced sequence is dropped
  drop_pending(c);
  int rc = 0;
  if (c.init) {
    const cudaError_t e = cudaStreamSynchronize(c.st);
    if (e != cudaSuccess) rc = cuda_fail(e, "release: stream");
  }
  for (auto &kv : c.ranges) cudaFree(kv.second.d);
  c.ranges.clear();
  c.cached = 0;
  {
    GsCache &g = gs_cache();
    std::lock_guard<std::mutex> lk2(g.mu);
    g.m.clear();
  }
  return rc;
}

int ffn_b200_set_host_cache_budget(size_t bytes) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  c.budget = bytes;
  if (!bytes || c.cached <= bytes) return 0;
  // over the new budget: evict now (least recently used first)
  bool quiet = false;
  int rc = 0;
  ++c.call_no;  // no copy belongs to a call in progress
  while (c.cached > c.budget && evict_one(c, 0, 0, quiet, rc)) {
  }
  return rc;
}

size_t ffn_b200_host_cache_bytes(void) {
  Ctx &c = ctx();
  std::lock_guard<std::mutex> lk(c.mu);
  return c.cached;
}

}  // extern "C"
