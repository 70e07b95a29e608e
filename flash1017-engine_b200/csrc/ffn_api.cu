// ffn_api.cu -- the device-resident extension ABI (include/ffn_b200.h).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ffn_internal.h"

namespace ffn {

// ------------------------------------------------------------------ status
static thread_local std::string t_last_error;
static std::atomic<uint64_t> g_launches{0};

void set_error(const std::string &msg) { t_last_error = msg; }
int fail(int code, const std::string &msg) {
  t_last_error = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char *what) {
  return fail(FFN_B200_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
void note_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
bool pdl_allowed() {
  static const bool on = [] {
    const char *v = std::getenv("FFN_B200_NO_PDL");
    return !(v && *v && *v != '0');
  }();
  return on;
}

// ------------------------------------------------------------- profiling
// A fixed pool of event pairs, created when profiling is enabled; launches
// beyond the pool are not timed (counted in `dropped`).
namespace {
struct Prof {
  std::mutex mu;
  bool on = false;
  uint32_t mask = ~0u;          // kinds timed while on
  std::vector<cudaEvent_t> ev;  // 2 per record
  std::vector<int> kind;        // per record
  size_t used = 0;              // records in use
  int open_kind = -1;
  double total_ms[FFN_B200_K_COUNT] = {0};
  uint64_t count[FFN_B200_K_COUNT] = {0};
  uint64_t dropped = 0;
};
Prof &prof() {
  static Prof *p = new Prof();
  return *p;
}
constexpr size_t kProfRecords = 16384;
}  // namespace

void prof_begin(int kind, cudaStream_t st) {
  Prof &p = prof();
  if (!p.on || !((p.mask >> kind) & 1u)) return;
  std::lock_guard<std::mutex> lk(p.mu);
  if (p.used >= p.kind.size()) { ++p.dropped; p.open_kind = -1; return; }
  cudaEventRecord(p.ev[2 * p.used], st);
  p.kind[p.used] = kind;
  p.open_kind = kind;
}

void prof_end(int kind, cudaStream_t st) {
  Prof &p = prof();
  if (!p.on || !((p.mask >> kind) & 1u)) return;
  std::lock_guard<std::mutex> lk(p.mu);
  if (p.open_kind != kind || p.used >= p.kind.size()) return;
  cudaEventRecord(p.ev[2 * p.used + 1], st);
  ++p.used;
  p.open_kind = -1;
}

// Folds the completed records into the totals (waits for the recorded events).
static int prof_collect(Prof &p) {
  for (size_t i = 0; i < p.used; ++i) {
    cudaError_t e = cudaEventSynchronize(p.ev[2 * i + 1]);
    if (e != cudaSuccess) return cuda_fail(e, "profile: cudaEventSynchronize");
    float ms = 0.f;
    e = cudaEventElapsedTime(&ms, p.ev[2 * i], p.ev[2 * i + 1]);
    if (e != cudaSuccess) return cuda_fail(e, "profile: cudaEventElapsedTime");
    const int k = p.kind[i] >= 0 && p.kind[i] < FFN_B200_K_COUNT ? p.kind[i] : FFN_B200_K_OTHER;
    p.total_ms[k] += ms;
    p.count[k] += 1;
  }
  p.used = 0;
  return 0;
}

int sm_count_of(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}


// ---------------------------------------------------------- workspace carving
// A bump allocator over the caller's buffer; with base == nullptr it only sizes.
struct Carve {
  char *base;
  size_t off = 0;
  explicit Carve(void *b) : base((char *)b) {}
  template <class T>
  T *take(size_t n) {
    off = (off + 255) & ~(size_t)255;
    T *p = base ? reinterpret_cast<T *>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

static bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

static int check_mat_shape(int fmt, size_t rows, size_t cols, const char *what) {
  if (rows == 0 || cols == 0)
    return fail(FFN_B200_EINVAL, std::string(what) + ": rows and cols must be positive");
  if (rows > (1u << 30) || cols > (1u << 24))
    return fail(FFN_B200_EINVAL, std::string(what) + ": shape too large");
  const size_t q = 64;  // a lane's 16-byte column slice, and 4-byte scale copies
  if (cols % q)
    return fail(FFN_B200_EUNSUP, std::string(what) + ": cols must be a multiple of " +
                                     std::to_string(q) + " for this format");
  return 0;
}

// The kernel family of a format: MXFP4 experts run on the NVFP4 instances
// (same packed nibbles; the kernels read the E8M0 block scales per task).
static int kfam(int fmt) {
  return fmt == FFN_B200_FMT_TERNARY || fmt == FFN_B200_FMT_MXFP8 ? fmt : FFN_B200_FMT_NVFP4;
}

// MXFP8: E4M3 [rows, cols], E8M0 [ceil(rows/32), cols/32]; 4-byte scale copies
// per 128 columns need cols % 128.
static int check_mxfp8(const ffn_b200_nvfp4_mat &m, size_t cols, const char *what) {
  if (cols % 128)
    return fail(FFN_B200_EUNSUP, std::string(what) + ": MXFP8 needs cols % 128 == 0");
  if (!m.w || !m.s) return fail(FFN_B200_EINVAL, std::string(what) + ": null MXFP8 pointer");
  if (!aligned(m.w, 16) || !aligned(m.s, 4))
    return fail(FFN_B200_EINVAL, std::string(what) + ": MXFP8 w must be 16-byte and s 4-byte aligned");
  int ex = 0;
  if (!(m.gs > 0.0f) || !std::isfinite(m.gs) || std::frexp(m.gs, &ex) != 0.5f)
    return fail(FFN_B200_EINVAL, std::string(what) + ": MXFP8 gs must be a power of two");
  return 0;
}

// MXFP4 rows of scales (cols/32 bytes) are copied in 4-byte pieces: cols % 128.
static int check_mxfp4(const ffn_b200_nvfp4_mat &m, size_t cols, const char *what) {
  if (cols % 128)
    return fail(FFN_B200_EUNSUP, std::string(what) + ": MXFP4 needs cols % 128 == 0");
  if (!m.w || !m.s) return fail(FFN_B200_EINVAL, std::string(what) + ": null MXFP4 pointer");
  if (!aligned(m.w, 16) || !aligned(m.s, 4))
    return fail(FFN_B200_EINVAL, std::string(what) + ": MXFP4 w must be 16-byte and s 4-byte aligned");
  int ex = 0;
  if (!(m.gs > 0.0f) || !std::isfinite(m.gs) || std::frexp(m.gs, &ex) != 0.5f)
    return fail(FFN_B200_EINVAL, std::string(what) + ": MXFP4 gs must be a power of two");
  return 0;
}

static int check_nvfp4(const ffn_b200_nvfp4_mat &m, const char *what) {
  if (!m.w || !m.s) return fail(FFN_B200_EINVAL, std::string(what) + ": null NVFP4 pointer");
  if (!aligned(m.w, 16) || !aligned(m.s, 4))
    return fail(FFN_B200_EINVAL, std::string(what) + ": NVFP4 w must be 16-byte and s 4-byte aligned");
  return 0;
}

static_assert(sizeof(ffn_b200_expert) == 264, "ffn_b200_expert is part of the extension ABI");

static int check_ternary(const ffn_b200_ternary_mat &m, const char *what) {
  if (!m.p || !m.rs) return fail(FFN_B200_EINVAL, std::string(what) + ": null ternary pointer");
  if (!aligned(m.p, 16) || !aligned(m.rs, 4))
    return fail(FFN_B200_EINVAL, std::string(what) + ": ternary p must be 16-byte and rs 4-byte aligned");
  if (m.core_a && (!m.core_b || !m.core_a_sc || !m.core_b_sc || !aligned(m.core_a, 16) ||
                   !aligned(m.core_b, 16)))
    return fail(FFN_B200_EINVAL, std::string(what) + ": incomplete or misaligned rank-16 core");
  if (m.bs && !aligned(m.bs, 4))
    return fail(FFN_B200_EINVAL, std::string(what) + ": ternary block scales must be 4-byte aligned");
  return 0;
}
// Block-scaled ternary rows are copied in 4-byte pieces of whole rows of scales.
static int check_ternary_bs(const ffn_b200_ternary_mat &m, size_t cols, const char *what) {
  if (m.bs && cols % 256)
    return fail(FFN_B200_EUNSUP, std::string(what) + ": block-scaled ternary needs cols % 256 == 0");
  return 0;
}

// Workspace of one dense activation block: x16 hi/lo + exponents + core z.
struct ActWs {
  __half *xh, *xl;
  int *xe;
  float *z;
};
static ActWs carve_act(Carve &c, size_t n_rows, size_t K) {
  ActWs w;
  w.xh = c.take<__half>(n_rows * K);
  w.xl = c.take<__half>(n_rows * K);
  w.xe = c.take<int>(n_rows);
  w.z = c.take<float>(n_rows * 3 * 16);
  return w;
}

// K-splits of a direct-mode phase launch (one expert or one matrix, few
// tokens): as many work items as one wave of resident warps holds (148 SMs x
// 12 warps on B200), at most one split per ring unit, partial sums within
// kSplitBytes.  A function of the shape only, so the workspace size does not
// depend on the device.
constexpr long long kSplitItems = 148 * 12;
constexpr size_t kSplitBytes = 512u << 10;
// partial sums of list-mode splits (MoE-layer and queued-call workspaces)
constexpr size_t kListSplitBytes = 2u << 20;

struct SplitPlan {
  int splits = 1, pt = 0;
  long long tasks = 0;
  size_t part_bytes = 0;  // partial sums (0 when splits == 1)
};

static SplitPlan plan_splits(int fmt, int phase, size_t rows, size_t K, size_t seq) {
  SplitPlan sp;
  const long long nv = (long long)((seq + kNTok - 1) / kNTok);
  sp.tasks = nv * (long long)((rows + rows_per_tile(phase) - 1) / rows_per_tile(phase));
  sp.pt = (int)std::min<size_t>(seq, kNTok);
  const long long nch = (long long)((K + chunk_cols(fmt) - 1) / chunk_cols(fmt));
  const size_t per = (size_t)sp.pt * rows_per_tile(phase) * (phase == 1 ? 2 : 1) * sizeof(float);
  long long s = std::min<long long>(kSplitItems / sp.tasks, nch);
  s = std::min<long long>(s, (long long)(kSplitBytes / ((size_t)sp.tasks * per)));
  sp.splits = (int)std::max<long long>(1, s);
  sp.part_bytes = sp.splits > 1 ? (size_t)sp.tasks * sp.splits * per : 0;
  return sp;
}

// Partial sums and arrival counters of up to two split launches.
struct SplitWs {
  float *part = nullptr;
  int *cnt = nullptr;  // [tasks of launch 0][tasks of launch 1]
};
static SplitWs carve_split(Carve &c, const SplitPlan &a, const SplitPlan &b) {
  SplitWs w;
  const size_t part = std::max(a.part_bytes, b.part_bytes);
  if (part) w.part = c.take<float>(part / sizeof(float));
  const size_t n = (a.splits > 1 ? a.tasks : 0) + (b.splits > 1 ? b.tasks : 0);
  if (n) w.cnt = c.take<int>(n);
  return w;
}
static int zero_counters(const SplitWs &w, const SplitPlan &a, const SplitPlan &b, cudaStream_t st) {
  const size_t n = (a.splits > 1 ? a.tasks : 0) + (b.splits > 1 ? b.tasks : 0);
  if (n) FFN_CUDA_TRY(cudaMemsetAsync(w.cnt, 0, n * sizeof(int), st));
  return 0;
}
static void apply_split(PhaseArgs &p, const SplitPlan &sp, const SplitWs &w, int *cnt) {
  p.splits = sp.splits;
  p.pt = sp.pt;
  p.part = sp.splits > 1 ? w.part : nullptr;
  p.cnt = sp.splits > 1 ? cnt : nullptr;
}

}  // namespace ffn

using namespace ffn;

extern "C" {

const char *ffn_b200_version(void) { return "ffn_b200 0.1 (sm_100a)"; }
const char *ffn_b200_last_error(void) { return t_last_error.c_str(); }
uint64_t ffn_b200_launch_count(void) { return g_launches.load(); }

int ffn_b200_set_device(int device) {
  FFN_CUDA_TRY(cudaSetDevice(device));
  return 0;
}

int ffn_b200_profile_enable(int enable) {
  Prof &p = prof();
  std::lock_guard<std::mutex> lk(p.mu);
  if (enable && p.ev.empty()) {
    p.ev.resize(2 * kProfRecords);
    for (auto &e : p.ev) FFN_CUDA_TRY(cudaEventCreate(&e));
    p.kind.assign(kProfRecords, -1);
  }
  if (enable) {  // a fresh window
    int rc = prof_collect(p);
    if (rc) return rc;
    for (int k = 0; k < FFN_B200_K_COUNT; ++k) { p.total_ms[k] = 0; p.count[k] = 0; }
    p.dropped = 0;
  }
  p.on = enable != 0;
  return 0;
}

int ffn_b200_profile_kinds(uint32_t mask) {
  Prof &p = prof();
  std::lock_guard<std::mutex> lk(p.mu);
  p.mask = mask;
  return 0;
}

int ffn_b200_profile_read(int kind, double *total_ms, uint64_t *launches) {
  if (kind < 0 || kind >= FFN_B200_K_COUNT) return fail(FFN_B200_EINVAL, "profile_read: bad kind");
  Prof &p = prof();
  std::lock_guard<std::mutex> lk(p.mu);
  int rc = prof_collect(p);
  if (rc) return rc;
  if (total_ms) *total_ms = p.total_ms[kind];
  if (launches) *launches = p.count[kind];
  return 0;
}

uint64_t ffn_b200_key(uint64_t parent, uint64_t v) {
  uint64_t z = parent + 0x9E3779B97F4A7C15ULL * (v + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

// ------------------------------------------------------------ single matrix
// (rows, format) enter through the split plan; the public size function keeps
// its (seq, cols) signature and sizes for the largest plan over rows/format.
static size_t matvec_ws(int fmt, size_t rows, size_t seq, size_t cols) {
  Carve c(nullptr);
  carve_act(c, seq, cols);
  const SplitPlan sp = plan_splits(fmt, 0, rows, cols, seq);
  carve_split(c, sp, SplitPlan{});
  return c.off + 256;
}

size_t ffn_b200_matvec_ws_bytes(size_t seq, size_t cols) {
  Carve c(nullptr);
  carve_act(c, seq, cols);
  // splits only when tasks * splits <= kSplitItems-ish; partials <= kSplitBytes,
  // counters <= kSplitItems
  c.take<float>(kSplitBytes / sizeof(float));
  c.take<int>(kSplitItems);
  return c.off + 256;
}

static int matvec_common(int fmt, size_t rows, size_t cols, size_t seq, const ffn_b200_expert &E,
                         const float *x, float *out, void *ws, size_t ws_bytes, void *stream) {
  if (seq == 0) return 0;
  if (!x || !out) return fail(FFN_B200_EINVAL, "matvec: null x/out");
  if (seq > (1u << 24)) return fail(FFN_B200_EINVAL, "matvec: seq too large");
  if (!ws || ws_bytes < matvec_ws(fmt, rows, seq, cols))
    return fail(FFN_B200_ENOSPC, "matvec: workspace too small (see ffn_b200_matvec_ws_bytes)");
  cudaStream_t st = (cudaStream_t)stream;
  Carve c(ws);
  ActWs a = carve_act(c, seq, cols);
  const SplitPlan sp = plan_splits(fmt, 0, rows, cols, seq);
  const SplitWs sw = carve_split(c, sp, SplitPlan{});
  const bool tern = fmt == FFN_B200_FMT_TERNARY;
  int rc = launch_xprep(x, (int)cols, (int)seq, (int)cols, tern ? nullptr : a.xh,
                        tern ? nullptr : a.xl, tern ? a.xh : nullptr, tern ? a.xl : nullptr,
                        (int)cols, a.xe, st);
  if (rc) return rc;
  if (tern && E.tn[0].core_a) {
    CoreZArgs z{};
    z.direct = E;
    z.n_tok_direct = (int)seq;
    z.K = (int)cols;
    z.mat0 = 0;
    z.nmat = 1;
    z.xf = x;
    z.ld_xf = (int)cols;
    z.z = a.z;
    if ((rc = launch_corez(z, (int)((seq + kNTok - 1) / kNTok), st))) return rc;
  }
  PhaseArgs p{};
  p.direct = E;
  p.n_tok_direct = (int)seq;
  p.rows = (int)rows;
  p.K = (int)cols;
  p.blocks = (int)((rows + rows_per_tile(0) - 1) / rows_per_tile(0));
  p.xh = a.xh;
  p.xl = a.xl;
  p.xe = a.xe;
  p.ld_x = (int)cols;
  p.z = a.z;
  p.y = out;
  p.ld_y = (int)rows;
  p.out_w = 1.0f;
  p.mat = 0;
  apply_split(p, sp, sw, sw.cnt);
  if ((rc = zero_counters(sw, sp, SplitPlan{}, st))) return rc;
  return launch_phase(fmt, 0, p, sp.tasks * sp.splits, st);
}

int ffn_b200_nvfp4_matvec(size_t rows, size_t cols, size_t seq, const ffn_b200_nvfp4_mat *m,
                          const float *x, float *out, void *ws, size_t ws_bytes, void *stream) {
  if (!m) return fail(FFN_B200_EINVAL, "nvfp4_matvec: null matrix");
  int rc = check_mat_shape(FFN_B200_FMT_NVFP4, rows, cols, "nvfp4_matvec");
  if (!rc) rc = check_nvfp4(*m, "nvfp4_matvec");
  if (rc) return rc;
  ffn_b200_expert E{};
  E.format = FFN_B200_FMT_NVFP4;
  E.proj_scale = 1.0f;
  E.nv[0] = *m;
  return matvec_common(FFN_B200_FMT_NVFP4, rows, cols, seq, E, x, out, ws, ws_bytes, stream);
}

int ffn_b200_ternary_matvec(size_t rows, size_t cols, size_t seq, const ffn_b200_ternary_mat *m,
                            const float *x, float *out, void *ws, size_t ws_bytes, void *stream) {
  if (!m) return fail(FFN_B200_EINVAL, "ternary_matvec: null matrix");
  int rc = check_mat_shape(FFN_B200_FMT_TERNARY, rows, cols, "ternary_matvec");
  if (!rc) rc = check_ternary(*m, "ternary_matvec");
  if (!rc) rc = check_ternary_bs(*m, cols, "ternary_matvec");
  if (rc) return rc;
  ffn_b200_expert E{};
  E.format = FFN_B200_FMT_TERNARY;
  E.proj_scale = 1.0f;
  E.tn[0] = *m;
  return matvec_common(FFN_B200_FMT_TERNARY, rows, cols, seq, E, x, out, ws, ws_bytes, stream);
}

int ffn_b200_mxfp4_matvec(size_t rows, size_t cols, size_t seq, const ffn_b200_nvfp4_mat *m,
                          const float *x, float *out, void *ws, size_t ws_bytes, void *stream) {
  if (!m) return fail(FFN_B200_EINVAL, "mxfp4_matvec: null matrix");
  int rc = check_mat_shape(FFN_B200_FMT_NVFP4, rows, cols, "mxfp4_matvec");
  if (!rc) rc = check_mxfp4(*m, cols, "mxfp4_matvec");
  if (rc) return rc;
  ffn_b200_expert E{};
  E.format = FFN_B200_FMT_MXFP4;
  E.proj_scale = 1.0f;
  E.nv[0] = *m;
  return matvec_common(FFN_B200_FMT_NVFP4, rows, cols, seq, E, x, out, ws, ws_bytes, stream);
}

int ffn_b200_mxfp8_matvec(size_t rows, size_t cols, size_t seq, const ffn_b200_nvfp4_mat *m,
                          const float *x, float *out, void *ws, size_t ws_bytes, void *stream) {
  if (!m) return fail(FFN_B200_EINVAL, "mxfp8_matvec: null matrix");
  int rc = check_mat_shape(FFN_B200_FMT_MXFP8, rows, cols, "mxfp8_matvec");
  if (!rc) rc = check_mxfp8(*m, cols, "mxfp8_matvec");
  if (rc) return rc;
  ffn_b200_expert E{};
  E.format = FFN_B200_FMT_MXFP8;
  E.proj_scale = 1.0f;
  E.nv[0] = *m;
  return matvec_common(FFN_B200_FMT_MXFP8, rows, cols, seq, E, x, out, ws, ws_bytes, stream);
}

// --------------------------------------------------------------- one expert
// Both formats plan the same way up to the unit width; size for the larger.
static void expert_plans(int fmt, size_t inter, size_t hidden, size_t seq, SplitPlan &s1, SplitPlan &s2) {
  s1 = plan_splits(fmt, 1, inter, hidden, seq);
  s2 = plan_splits(fmt, 2, hidden, inter, seq);
}
static void carve_expert(Carve &c, int fmt, size_t inter, size_t hidden, size_t seq, ActWs *a,
                         __half **hh, __half **hl, SplitWs *sw) {
  ActWs aw = carve_act(c, seq, hidden);
  __half *h0 = c.take<__half>(seq * inter), *h1 = c.take<__half>(seq * inter);
  SplitPlan s1, s2;
  expert_plans(fmt, inter, hidden, seq, s1, s2);
  SplitWs w = carve_split(c, s1, s2);
  if (a) *a = aw;
  if (hh) *hh = h0;
  if (hl) *hl = h1;
  if (sw) *sw = w;
}

size_t ffn_b200_expert_ws_bytes(size_t inter, size_t hidden, size_t seq) {
  size_t need = 0;
  for (int fmt : {FFN_B200_FMT_NVFP4, FFN_B200_FMT_TERNARY, FFN_B200_FMT_MXFP8}) {
    Carve c(nullptr);
    carve_expert(c, fmt, inter, hidden, seq, nullptr, nullptr, nullptr, nullptr);
    need = std::max(need, c.off + 256);
  }
  return std::max(need, expert_decode_ws_bytes(inter, seq) + 256);
}

static int check_expert(const ffn_b200_expert &e, size_t inter, size_t hidden, const char *what) {
  int rc;
  if (e.format != FFN_B200_FMT_NVFP4 && e.format != FFN_B200_FMT_TERNARY && e.format != FFN_B200_FMT_MXFP4 &&
      e.format != FFN_B200_FMT_MXFP8)
    return fail(FFN_B200_EINVAL, std::string(what) + ": unknown expert format");
  if ((rc = check_mat_shape(e.format, inter, hidden, what))) return rc;
  if ((rc = check_mat_shape(e.format, hidden, inter, what))) return rc;
  for (int i = 0; i < 3; ++i) {
    rc = e.format == FFN_B200_FMT_NVFP4   ? check_nvfp4(e.nv[i], what)
         : e.format == FFN_B200_FMT_MXFP4 ? check_mxfp4(e.nv[i], i == 2 ? inter : hidden, what)
         : e.format == FFN_B200_FMT_MXFP8 ? check_mxfp8(e.nv[i], i == 2 ? inter : hidden, what)
                                          : check_ternary(e.tn[i], what);
    if (!rc && e.format == FFN_B200_FMT_TERNARY) rc = check_ternary_bs(e.tn[i], i == 2 ? inter : hidden, what);
    if (rc) return rc;
  }
  return 0;
}

// The two-launch decode kernels for NVFP4 / MXFP4 experts over <= 8 tokens;
// FFN_B200_EXPERT_DECODE=0 in the environment keeps such calls on the GEMV
// phase kernels (read once per process).
static bool expert_decode_enabled() {
  static const bool on = [] {
    const char *v = getenv("FFN_B200_EXPERT_DECODE");
    return !(v && v[0] == '0');
  }();
  return on;
}

int ffn_b200_expert_forward(size_t inter, size_t hidden, size_t seq, const ffn_b200_expert *e,
                            const float *x, float *out, float accum_weight, int accumulate,
                            void *ws, size_t ws_bytes, void *stream) {
  if (!e) return fail(FFN_B200_EINVAL, "expert_forward: null expert");
  int rc = check_expert(*e, inter, hidden, "expert_forward");
  if (rc) return rc;
  if (seq == 0) return 0;
  if (!x || !out) return fail(FFN_B200_EINVAL, "expert_forward: null x/out");
  if (seq > (1u << 24)) return fail(FFN_B200_EINVAL, "expert_forward: seq too large");
  if (!ws || ws_bytes < ffn_b200_expert_ws_bytes(inter, hidden, seq))
    return fail(FFN_B200_ENOSPC, "expert_forward: workspace too small (see ffn_b200_expert_ws_bytes)");
  cudaStream_t st = (cudaStream_t)stream;
  if (expert_decode_enabled() && expert_decode_fits(*e, inter, hidden, seq) &&
      ws_bytes >= expert_decode_ws_bytes(inter, seq) && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 15) == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0)
    return launch_expert_decode(*e, inter, hidden, seq, x, out, accum_weight, accumulate, ws, st);
  const int fmt = kfam(e->format);  // kernel family
  const bool tern = fmt == FFN_B200_FMT_TERNARY;
  Carve c(ws);
  ActWs a;
  __half *hh, *hl;
  SplitWs sw;
  carve_expert(c, fmt, inter, hidden, seq, &a, &hh, &hl, &sw);
  SplitPlan s1, s2;
  expert_plans(fmt, inter, hidden, seq, s1, s2);
  if ((rc = zero_counters(sw, s1, s2, st))) return rc;
  const int nv = (int)((seq + kNTok - 1) / kNTok);
  if ((rc = launch_xprep(x, (int)hidden, (int)seq, (int)hidden, tern ? nullptr : a.xh,
                         tern ? nullptr : a.xl, tern ? a.xh : nullptr, tern ? a.xl : nullptr,
                         (int)hidden, a.xe, st)))
    return rc;
  const bool cores = tern && (e->tn[0].core_a || e->tn[1].core_a || e->tn[2].core_a);
  if (cores) {
    CoreZArgs z{};
    z.direct = *e;
    z.n_tok_direct = (int)seq;
    z.K = (int)hidden;
    z.mat0 = 0;
    z.nmat = 2;
    z.xf = x;
    z.ld_xf = (int)hidden;
    z.z = a.z;
    if ((rc = launch_corez(z, nv, st))) return rc;
  }
  PhaseArgs p{};
  p.direct = *e;
  p.n_tok_direct = (int)seq;
  p.rows = (int)inter;
  p.K = (int)hidden;
  p.blocks = (int)((inter + rows_per_tile(1) - 1) / rows_per_tile(1));
  p.xh = a.xh;
  p.xl = a.xl;
  p.xe = a.xe;
  p.ld_x = (int)hidden;
  p.z = a.z;
  p.hh = hh;
  p.hl = hl;
  p.ld_h = (int)inter;
  apply_split(p, s1, sw, sw.cnt);
  if ((rc = launch_phase(fmt, 1, p, s1.tasks * s1.splits, st))) return rc;
  if (cores) {
    CoreZArgs z{};
    z.direct = *e;
    z.n_tok_direct = (int)seq;
    z.K = (int)inter;
    z.mat0 = 2;
    z.nmat = 1;
    z.hh = hh;
    z.hl = hl;
    z.ld_h = (int)inter;
    z.z = a.z;
    if ((rc = launch_corez(z, nv, st))) return rc;
  }
  // h is written unscaled (|h| <= 100 by the clamps), so phase 2 takes no exponent.
  PhaseArgs q{};
  q.direct = *e;
  q.n_tok_direct = (int)seq;
  q.rows = (int)hidden;
  q.K = (int)inter;
  q.blocks = (int)((hidden + rows_per_tile(2) - 1) / rows_per_tile(2));
  q.xh = hh;
  q.xl = hl;
  q.xe = nullptr;
  q.ld_x = (int)inter;
  q.z = a.z;
  q.y = out;
  q.ld_y = (int)hidden;
  q.out_w = accum_weight;
  q.accumulate = accumulate ? 1 : 0;
  apply_split(q, s2, sw, sw.cnt ? sw.cnt + (s1.splits > 1 ? s1.tasks : 0) : nullptr);
  return launch_phase(fmt, 2, q, s2.tasks * s2.splits, st);
}

// ---------------------------------------------------------------- MoE layer
struct MoeWs {
  __half *xh, *xl, *th, *tl;
  float *xn;
  int *xe;
  float *logits;
  int32_t *idx, *inv, *pair_tok;
  float *wt;
  int *ints;
  VExp *vexp_nv, *vexp_tn;
  int *n_vexp;
  __half *hh, *hl;
  float *z, *y;
  uint8_t *chunk;  // grouped path: chunk list
  int *err;        // grouped path: timed-out wait flag
  float *part;     // GEMV path: K-split partial sums (kListSplitBytes)
  int *cnt;        // GEMV path: split arrival counters, kSplitItems per phase launch (4)
  // FP4 path: x and h as six NVFP4 terms, h in f32, the chunk list
  uint8_t *xq, *xs, *hq, *hs;
  int *xqe, *hqe;
  float *hf;
};

// The block-scaled FP4 path can run the layer: NVFP4 experts only, packed
// (stage images), shapes in whole 256-column stages and quantiser rows.
static bool fp4_path_ok(const ffn_b200_moe_desc &d) {
  return d.fp4_packed && d.has_nvfp4 && !d.has_ternary && !d.has_mxfp4 && d.hidden % 256 == 0 &&
         d.inter % 256 == 0 && d.hidden <= 16384 && d.inter <= 16384;
}

static MoeWs carve_moe(Carve &c, const ffn_b200_moe_desc &d, size_t T) {
  MoeWs w{};
  const size_t H = d.hidden, I = d.inter, E = d.n_experts, k = d.top_k, P = T * k;
  w.xh = c.take<__half>(T * H);  // natural order: NVFP4 experts and the tensor router
  w.xl = c.take<__half>(T * H);
  if (d.has_ternary) { w.th = c.take<__half>(T * H); w.tl = c.take<__half>(T * H); }
  w.xn = d.norm_w ? c.take<float>(T * H) : nullptr;
  w.xe = c.take<int>(T);
  w.logits = c.take<float>(4 * T * E);  // partial planes of the tensor router
  w.idx = c.take<int32_t>(P);
  w.wt = c.take<float>(P);
  w.inv = c.take<int32_t>(P);
  w.pair_tok = c.take<int32_t>(P);
  w.ints = c.take<int>(4 * E);
  w.vexp_nv = c.take<VExp>(P + E);
  w.vexp_tn = c.take<VExp>(P + E);
  w.n_vexp = c.take<int>(4);
  w.hh = c.take<__half>(P * I);
  w.hl = c.take<__half>(P * I);
  w.z = d.has_ternary ? c.take<float>(P * 3 * 16) : nullptr;
  w.y = c.take<float>(P * H);
  w.chunk = c.take<uint8_t>(gg_chunk_bytes((int)P, (int)E));
  w.err = c.take<int>(1);
  w.part = c.take<float>(kListSplitBytes / sizeof(float));
  w.cnt = c.take<int>(4 * (size_t)kSplitItems);
  if (fp4_path_ok(d)) {
    w.xq = c.take<uint8_t>(T * kFp4Terms * H / 2);
    w.xs = c.take<uint8_t>(T * kFp4Terms * H / 16);
    w.xqe = c.take<int>(T * kFp4Terms);
    w.hf = c.take<float>(P * I);
    w.hq = c.take<uint8_t>(P * kFp4Terms * I / 2);
    w.hs = c.take<uint8_t>(P * kFp4Terms * I / 16);
    w.hqe = c.take<int>(P * kFp4Terms);
  }
  return w;
}

size_t ffn_b200_moe_ws_bytes(const ffn_b200_moe_desc *d, size_t max_tokens) {
  if (!d) return 0;
  Carve c(nullptr);
  carve_moe(c, *d, max_tokens);
  return c.off + 256;
}

// K-splits of a list-mode phase launch over at most n_slices slices: the same
// rule as plan_splits (one wave of warps, at most one split per ring unit),
// partials within kListSplitBytes (a list launch has more row blocks than one
// expert's, so its partials need more room than kSplitBytes gives; only the
// MoE-layer and queued-call workspaces hold them).  pt = the largest slice.
static SplitPlan plan_list_splits(int fmt, int phase, size_t rows, size_t K, int n_slices, int pt) {
  SplitPlan sp;
  sp.tasks = (long long)n_slices * (long long)((rows + rows_per_tile(phase) - 1) / rows_per_tile(phase));
  sp.pt = pt;
  const long long nch = (long long)((K + chunk_cols(fmt) - 1) / chunk_cols(fmt));
  const size_t per = (size_t)pt * rows_per_tile(phase) * (phase == 1 ? 2 : 1) * sizeof(float);
  long long s = std::min<long long>(kSplitItems / sp.tasks, nch);
  s = std::min<long long>(s, (long long)(kListSplitBytes / ((size_t)sp.tasks * per)));
  sp.splits = (int)std::max<long long>(1, s);
  sp.part_bytes = sp.splits > 1 ? (size_t)sp.tasks * sp.splits * per : 0;
  return sp;
}
// The GEMV path's experts of a routed layer: per format, [rank-16 core z,]
// gate/up + SwiGLU -> h, [core z of h,] down -> y [pair][H] (unweighted).
// w.pair_tok / w.vexp_* / w.n_vexp come from launch_group.
static int moe_gemv_experts(const ffn_b200_moe_desc *d, MoeWs &w, int P, const float *xin,
                            cudaStream_t st) {
  const size_t H = d->hidden, I = d->inter;
  int rc;
  // Upper bound of slices per format (the device count is <= this).
  const int e_local = d->expert_end - d->expert_begin;
  const long long max_vexp = std::min<long long>((long long)P, (long long)P / kNTok + e_local);
  // K-splits from the slice bound: a few-token layer (single-token decode:
  // top_k slices) would otherwise leave most of the GPU idle; a layer with
  // many slices (config 4) plans one split, i.e. none.
  const int pt = (int)std::min<long long>(kNTok, (long long)P / (long long)d->top_k);
  SplitPlan plans[2][2];
  bool any_split = false;
  for (int f = 0; f < 2; ++f) {
    const int fmt = f == 0 ? FFN_B200_FMT_NVFP4 : FFN_B200_FMT_TERNARY;
    plans[f][0] = plan_list_splits(fmt, 1, I, H, (int)max_vexp, pt);
    plans[f][1] = plan_list_splits(fmt, 2, H, I, (int)max_vexp, pt);
    any_split = any_split || plans[f][0].splits > 1 || plans[f][1].splits > 1;
  }
  if (any_split) FFN_CUDA_TRY(cudaMemsetAsync(w.cnt, 0, 4 * (size_t)kSplitItems * sizeof(int), st));
  SplitWs sw;
  sw.part = w.part;
  for (int f = 0; f < 2; ++f) {
    const int fmt = f == 0 ? FFN_B200_FMT_NVFP4 : FFN_B200_FMT_TERNARY;
    if ((fmt == FFN_B200_FMT_NVFP4 && !d->has_nvfp4) || (fmt == FFN_B200_FMT_TERNARY && !d->has_ternary))
      continue;
    const VExp *vl = f == 0 ? w.vexp_nv : w.vexp_tn;
    const int *nvd = w.n_vexp + f;
    const bool tern = fmt == FFN_B200_FMT_TERNARY;
    if (tern) {
      CoreZArgs z{};
      z.experts = d->experts;
      z.vexp = vl;
      z.n_vexp_dev = nvd;
      z.K = (int)H;
      z.mat0 = 0;
      z.nmat = 2;
      z.xf = xin;
      z.ld_xf = (int)H;
      z.pair_tok = w.pair_tok;
      z.z = w.z;
      if ((rc = launch_corez(z, (int)max_vexp, st))) return rc;
    }
    PhaseArgs p{};
    p.experts = d->experts;
    p.vexp = vl;
    p.n_vexp_dev = nvd;
    p.rows = (int)I;
    p.K = (int)H;
    p.blocks = (int)((I + rows_per_tile(1) - 1) / rows_per_tile(1));
    p.xh = tern ? w.th : w.xh;
    p.xl = tern ? w.tl : w.xl;
    p.xe = w.xe;
    p.ld_x = (int)H;
    p.pair_tok = w.pair_tok;
    p.z = w.z;
    p.hh = w.hh;
    p.hl = w.hl;
    p.ld_h = (int)I;
    apply_split(p, plans[f][0], sw, w.cnt + (size_t)(2 * f) * kSplitItems);
    if ((rc = launch_phase(fmt, 1, p, max_vexp * p.blocks * plans[f][0].splits, st))) return rc;
    if (tern) {
      CoreZArgs z{};
      z.experts = d->experts;
      z.vexp = vl;
      z.n_vexp_dev = nvd;
      z.K = (int)I;
      z.mat0 = 2;
      z.nmat = 1;
      z.hh = w.hh;
      z.hl = w.hl;
      z.ld_h = (int)I;
      z.z = w.z;
      if ((rc = launch_corez(z, (int)max_vexp, st))) return rc;
    }
    PhaseArgs q{};
    q.experts = d->experts;
    q.vexp = vl;
    q.n_vexp_dev = nvd;
    q.rows = (int)H;
    q.K = (int)I;
    q.blocks = (int)((H + rows_per_tile(2) - 1) / rows_per_tile(2));
    q.xh = w.hh;
    q.xl = w.hl;
    q.xe = nullptr;
    q.ld_x = (int)I;
    q.z = w.z;
    q.y = w.y;
    q.ld_y = (int)H;
    apply_split(q, plans[f][1], sw, w.cnt + (size_t)(2 * f + 1) * kSplitItems);
    if ((rc = launch_phase(fmt, 2, q, max_vexp * q.blocks * plans[f][1].splits, st))) return rc;
  }
  return 0;
}

// ----------------------------------------------------- queued routed calls
static ffn_b200_moe_desc calls_desc(size_t inter, size_t hidden, int n, bool nv, bool tern, bool mx) {
  ffn_b200_moe_desc d{};
  d.hidden = hidden;
  d.inter = inter;
  d.n_experts = (size_t)n;
  d.top_k = 1;
  d.expert_begin = 0;
  d.expert_end = n;
  d.has_nvfp4 = nv ? 1 : 0;
  d.has_ternary = tern ? 1 : 0;
  d.has_mxfp4 = mx ? 1 : 0;
  d.path = FFN_B200_PATH_GEMV;
  return d;
}

}  // extern "C"

namespace {
// Slice lists of queued calls, one per engine instance: 0 NVFP4 and MXFP4,
// 1 ternary, 2 MXFP8.  Two phase launches per list, each with its own split
// arrival counters.
constexpr int kCallLists = 3;
constexpr int kCallLaunches = 2 * kCallLists;
int call_list(int format) {
  return format == FFN_B200_FMT_TERNARY ? 1 : format == FFN_B200_FMT_MXFP8 ? 2 : 0;
}
int list_format(int l) {
  return l == 0 ? FFN_B200_FMT_NVFP4 : l == 1 ? FFN_B200_FMT_TERNARY : FFN_B200_FMT_MXFP8;
}

// Byte offsets of the call tables, the same in the host stage and in the
// device copy (one upload; the split counters travel as zeros).
struct CallTables {
  size_t experts, pair_tok, vexp[kCallLists], n_vexp, cnt, tok_ptr, ent_pair, ent_w, row_zero, total;
};
CallTables call_tables(int n, int out_rows) {
  const size_t P = (size_t)n * kNTok;  // upper bound of the pairs
  CallTables t{};
  size_t o = 0;
  auto take = [&o](size_t bytes) {
    const size_t at = o;
    o = (o + bytes + 15) & ~(size_t)15;
    return at;
  };
  t.experts = take((size_t)n * sizeof(ffn_b200_expert));
  t.pair_tok = take(P * 4);
  for (int l = 0; l < kCallLists; ++l) t.vexp[l] = take((size_t)n * sizeof(VExp));  // one slice per call
  t.n_vexp = take(4 * sizeof(int));
  t.cnt = take((size_t)kCallLaunches * kSplitItems * sizeof(int));
  t.tok_ptr = take(((size_t)out_rows + 1) * 4);
  t.ent_pair = take(P * 4);
  t.ent_w = take(P * 4);
  t.row_zero = take((size_t)out_rows);
  t.total = o;
  return t;
}

}  // namespace

int ffn::validate_expert_shape(int format, size_t inter, size_t hidden, const char *what) {
  if (format != FFN_B200_FMT_NVFP4 && format != FFN_B200_FMT_TERNARY && format != FFN_B200_FMT_MXFP4 &&
      format != FFN_B200_FMT_MXFP8)
    return fail(FFN_B200_EINVAL, std::string(what) + ": unknown expert format");
  int rc;
  if ((rc = check_mat_shape(format, inter, hidden, what))) return rc;
  if ((rc = check_mat_shape(format, hidden, inter, what))) return rc;
  if ((format == FFN_B200_FMT_MXFP4 || format == FFN_B200_FMT_MXFP8) && (hidden % 128 || inter % 128))
    return fail(FFN_B200_EUNSUP, std::string(what) + ": MXFP4 / MXFP8 experts need hidden and inter % 128 == 0");
  return 0;
}

int ffn::validate_expert(const ffn_b200_expert &e, size_t inter, size_t hidden, const char *what) {
  return check_expert(e, inter, hidden, what);
}

size_t ffn::routed_calls_stage_bytes(int n, int out_rows) { return call_tables(n, out_rows).total; }

size_t ffn::routed_calls_ws_bytes(size_t inter, size_t hidden, int n, int x_rows, int out_rows) {
  const ffn_b200_moe_desc d = calls_desc(inter, hidden, n, true, true, true);
  const size_t rows = std::max<size_t>((size_t)x_rows, (size_t)n * kNTok);
  return ((call_tables(n, out_rows).total + 255) & ~(size_t)255) + ffn_b200_moe_ws_bytes(&d, rows) +
         2 * kListSplitBytes + 512;
}

int ffn::routed_calls(const RoutedCalls &q, size_t inter, size_t hidden, void *stage, void *ws,
                      size_t ws_bytes, cudaStream_t st) {
  const int n = q.n;
  if (n <= 0) return 0;
  if (n > kCallsMax) return fail(FFN_B200_EINVAL, "routed calls: too many calls");
  if (!q.experts || !q.row0 || !q.m || !q.tok_ptr || !q.ent_pair || !q.ent_w || !q.x || !q.out || !stage)
    return fail(FFN_B200_EINVAL, "routed calls: null pointer");
  if (q.out_rows <= 0 || q.x_rows <= 0) return fail(FFN_B200_EINVAL, "routed calls: no rows");
  int n_slices[kCallLists] = {0, 0, 0}, pt[kCallLists] = {0, 0, 0};
  bool mx = false;
  int P = 0, rc;
  for (int c = 0; c < n; ++c) {
    const ffn_b200_expert &e = q.experts[c];
    if ((rc = check_expert(e, inter, hidden, "routed calls"))) return rc;
    if (q.m[c] < 1 || q.m[c] > kNTok || q.row0[c] < 0 || q.row0[c] + q.m[c] > q.x_rows)
      return fail(FFN_B200_EINVAL, "routed calls: a call's x rows are out of range");
    const int l = call_list(e.format);
    ++n_slices[l];
    pt[l] = std::max(pt[l], (int)q.m[c]);
    mx = mx || e.format == FFN_B200_FMT_MXFP4;
    P += q.m[c];
  }
  if (q.tok_ptr[0] != 0 || q.tok_ptr[q.out_rows] != P)
    return fail(FFN_B200_EINVAL, "routed calls: the combine list must hold every pair once");
  for (int r = 0; r < q.out_rows; ++r)
    if (q.tok_ptr[r + 1] < q.tok_ptr[r]) return fail(FFN_B200_EINVAL, "routed calls: tok_ptr decreases");
  for (int e = 0; e < P; ++e)
    if (q.ent_pair[e] < 0 || q.ent_pair[e] >= P) return fail(FFN_B200_EINVAL, "routed calls: bad pair");
  if (ws_bytes < routed_calls_ws_bytes(inter, hidden, n, q.x_rows, q.out_rows))
    return fail(FFN_B200_ENOSPC, "routed calls: workspace too small");
  // host tables: slices (one per call, per list), pair -> x row, zeroed split
  // counters, the combine list
  const CallTables t = call_tables(n, q.out_rows);
  char *h = (char *)stage;
  std::memcpy(h + t.experts, q.experts, (size_t)n * sizeof(ffn_b200_expert));
  int32_t *pair_tok = (int32_t *)(h + t.pair_tok);
  int *nvx = (int *)(h + t.n_vexp);
  nvx[0] = nvx[1] = nvx[2] = nvx[3] = 0;
  for (int c = 0, pos = 0; c < n; ++c) {
    for (int j = 0; j < q.m[c]; ++j) pair_tok[pos + j] = q.row0[c] + j;
    const int l = call_list(q.experts[c].format);
    VExp &v = ((VExp *)(h + t.vexp[l]))[nvx[l]++];
    v.expert = c;
    v.offset = pos;
    v.count = q.m[c];
    v.pad = 0;
    pos += q.m[c];
  }
  std::memset(h + t.cnt, 0, (size_t)kCallLaunches * kSplitItems * sizeof(int));
  std::memcpy(h + t.tok_ptr, q.tok_ptr, ((size_t)q.out_rows + 1) * 4);
  std::memcpy(h + t.ent_pair, q.ent_pair, (size_t)P * 4);
  std::memcpy(h + t.ent_w, q.ent_w, (size_t)P * 4);
  if (q.row_zero) std::memcpy(h + t.row_zero, q.row_zero, (size_t)q.out_rows);
  else std::memset(h + t.row_zero, 0, (size_t)q.out_rows);
  char *dt = (char *)ws;
  FFN_CUDA_TRY(cudaMemcpyAsync(dt, h, t.total, cudaMemcpyHostToDevice, st));
  ffn_b200_moe_desc d = calls_desc(inter, hidden, n, n_slices[0] + n_slices[2] > 0, n_slices[1] > 0, mx);
  d.experts = (const ffn_b200_expert *)(dt + t.experts);
  Carve cv(dt + ((t.total + 255) & ~(size_t)255));
  MoeWs mw = carve_moe(cv, d, std::max<size_t>((size_t)q.x_rows, (size_t)P));
  float *part[2] = {cv.take<float>(kListSplitBytes / sizeof(float)),
                    cv.take<float>(kListSplitBytes / sizeof(float))};
  mw.pair_tok = (int32_t *)(dt + t.pair_tok);
  mw.n_vexp = (int *)(dt + t.n_vexp);
  int *cnt = (int *)(dt + t.cnt);
  const size_t H = hidden, I = inter;
  const bool natural = n_slices[0] + n_slices[2] > 0;  // NVFP4/MXFP4/MXFP8 read natural-order rows
  if ((rc = launch_xprep(q.x, (int)H, q.x_rows, (int)H, natural ? mw.xh : nullptr, natural ? mw.xl : nullptr,
                         mw.th, mw.tl, (int)H, mw.xe, st)))
    return rc;
  // one list: [core z], gate/up + SwiGLU -> h, [core z of h], down -> y [pair][H]
  auto run_list = [&](int l, cudaStream_t ls, float *lpart) -> int {
    int rc;
    const int fmt = list_format(l);
    const bool tern = fmt == FFN_B200_FMT_TERNARY;
    const VExp *vl = (const VExp *)(dt + t.vexp[l]);
    const int *nvd = mw.n_vexp + l;
    const SplitPlan s1 = plan_list_splits(fmt, 1, I, H, n_slices[l], pt[l]);
    const SplitPlan s2 = plan_list_splits(fmt, 2, H, I, n_slices[l], pt[l]);
    SplitWs sw;
    sw.part = lpart;
    if (tern) {
      CoreZArgs z{};
      z.experts = d.experts;
      z.vexp = vl;
      z.n_vexp_dev = nvd;
      z.K = (int)H;
      z.mat0 = 0;
      z.nmat = 2;
      z.xf = q.x;
      z.ld_xf = (int)H;
      z.pair_tok = mw.pair_tok;
      z.z = mw.z;
      if ((rc = launch_corez(z, n_slices[l], ls))) return rc;
    }
    PhaseArgs p{};
    p.experts = d.experts;
    p.vexp = vl;
    p.n_vexp_dev = nvd;
    p.rows = (int)I;
    p.K = (int)H;
    p.blocks = (int)((I + rows_per_tile(1) - 1) / rows_per_tile(1));
    p.xh = tern ? mw.th : mw.xh;
    p.xl = tern ? mw.tl : mw.xl;
    p.xe = mw.xe;
    p.ld_x = (int)H;
    p.pair_tok = mw.pair_tok;
    p.z = mw.z;
    p.hh = mw.hh;
    p.hl = mw.hl;
    p.ld_h = (int)I;
    apply_split(p, s1, sw, cnt + (size_t)(2 * l) * kSplitItems);
    if ((rc = launch_phase(fmt, 1, p, s1.tasks * s1.splits, ls))) return rc;
    if (tern) {
      CoreZArgs z{};
      z.experts = d.experts;
      z.vexp = vl;
      z.n_vexp_dev = nvd;
      z.K = (int)I;
      z.mat0 = 2;
      z.nmat = 1;
      z.hh = mw.hh;
      z.hl = mw.hl;
      z.ld_h = (int)I;
      z.z = mw.z;
      if ((rc = launch_corez(z, n_slices[l], ls))) return rc;
    }
    PhaseArgs r{};
    r.experts = d.experts;
    r.vexp = vl;
    r.n_vexp_dev = nvd;
    r.rows = (int)H;
    r.K = (int)I;
    r.blocks = (int)((H + rows_per_tile(2) - 1) / rows_per_tile(2));
    r.xh = mw.hh;
    r.xl = mw.hl;
    r.xe = nullptr;
    r.ld_x = (int)I;
    r.z = mw.z;
    r.y = mw.y;
    r.ld_y = (int)H;
    apply_split(r, s2, sw, cnt + (size_t)(2 * l + 1) * kSplitItems);
    return launch_phase(fmt, 2, r, s2.tasks * s2.splits, ls);
  };
  // The lists are independent until the combine (disjoint pairs): with a side
  // stream, the largest list (by weight bytes) runs on `st` and the others on
  // the side stream, forked after the activation prep and joined before the
  // combine.
  static const double kBytesPerWeight[kCallLists] = {0.5625, 0.25, 1.0};
  int main_l = -1, lists = 0;
  for (int l = 0; l < kCallLists; ++l)
    if (n_slices[l]) {
      ++lists;
      if (main_l < 0 || n_slices[l] * kBytesPerWeight[l] > n_slices[main_l] * kBytesPerWeight[main_l]) main_l = l;
    }
  const bool fork = q.side && q.fork && q.join && lists > 1;
  if (fork) {
    FFN_CUDA_TRY(cudaEventRecord(q.fork, st));
    FFN_CUDA_TRY(cudaStreamWaitEvent(q.side, q.fork, 0));
    rc = 0;
    for (int l = 0; l < kCallLists && !rc; ++l)
      if (n_slices[l] && l != main_l) rc = run_list(l, q.side, part[1]);
    if (!rc) rc = run_list(main_l, st, part[0]);
    // join even after a failed launch: later work on `st` reuses the workspace
    cudaError_t e = cudaEventRecord(q.join, q.side);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, q.join, 0);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail(e, "routed calls: side-stream join");
  } else {
    for (int l = 0; l < kCallLists; ++l)
      if (n_slices[l] && (rc = run_list(l, st, part[0]))) return rc;
  }
  return launch_rows_accum(mw.y, (const int32_t *)(dt + t.tok_ptr), (const int32_t *)(dt + t.ent_pair),
                           (const float *)(dt + t.ent_w), (const uint8_t *)(dt + t.row_zero), q.out_rows,
                           (int)H, q.out, st);
}

// Per token: out = residual + sum of w * y over the layer's routes (combine
// kernel), or, expert-parallel, over every rank's routes (exchange).
static int finish_layer(const ffn_b200_moe_desc *d, const MoeWs &w, int T, const float *residual, float *out,
                        const int *err, ffn_b200_ep *ep, cudaStream_t st) {
  const int H = (int)d->hidden, k = (int)d->top_k;
  const int E = (int)d->n_experts;
  if (!ep) return launch_combine(w.y, H, w.idx, w.wt, w.inv, T, k, d->experts, residual, out, H, st, err, E);
  EpCombine cb{w.y, H, w.idx, w.wt, w.inv, k, d->experts, err, E, T * k};
  return ep_exchange(ep, (size_t)T, &cb, residual, out, st);
}

// The MoE layer; with `ep`, this rank's partial goes through the expert-parallel
// exchange (combined per token inside it) instead of the combine kernel.
static int moe_layer_impl(const ffn_b200_moe_desc *d, size_t n_tok, const float *x, const float *residual,
                          float *out, int32_t *topk_idx, float *topk_w, void *ws, size_t ws_bytes,
                          void *stream, ffn_b200_ep *ep) {
  if (!d) return fail(FFN_B200_EINVAL, "moe_layer: null descriptor");
  const size_t H = d->hidden, I = d->inter, E = d->n_experts, k = d->top_k;
  if (!d->experts || !d->router_w) return fail(FFN_B200_EINVAL, "moe_layer: null experts/router");
  if (E == 0 || E > 4096) return fail(FFN_B200_EINVAL, "moe_layer: n_experts must be in 1..4096");
  if (k == 0 || k > (size_t)kTopKMax || k > E)
    return fail(FFN_B200_EINVAL, "moe_layer: top_k must be in 1..min(16, n_experts)");
  if (!d->has_nvfp4 && !d->has_ternary)
    return fail(FFN_B200_EINVAL, "moe_layer: has_nvfp4/has_ternary both zero");
  if (H % 64 || I % 64 || H == 0 || I == 0 || H > (1u << 20) || I > (1u << 20))
    return fail(FFN_B200_EUNSUP, "moe_layer: hidden and inter must be multiples of 64");
  if (d->expert_begin < 0 || d->expert_end > (int)E || d->expert_begin > d->expert_end)
    return fail(FFN_B200_EINVAL, "moe_layer: bad expert range");
  if (d->score_fn != FFN_B200_SCORE_REF_SQRTSOFTPLUS && d->score_fn != FFN_B200_SCORE_SIGMOID)
    return fail(FFN_B200_EINVAL, "moe_layer: unknown score_fn");
  if (d->router_mode != FFN_B200_ROUTER_EXACT && d->router_mode != FFN_B200_ROUTER_TENSOR)
    return fail(FFN_B200_EINVAL, "moe_layer: unknown router_mode");
  if (d->path != FFN_B200_PATH_AUTO && d->path != FFN_B200_PATH_GEMV && d->path != FFN_B200_PATH_GROUPED &&
      d->path != FFN_B200_PATH_FP4)
    return fail(FFN_B200_EINVAL, "moe_layer: unknown path");
  const bool fp4_ok = fp4_path_ok(*d);
  if (d->path == FFN_B200_PATH_FP4 && !fp4_ok)
    return fail(FFN_B200_EUNSUP,
                "moe_layer: the FP4 path needs NVFP4-only experts packed by ffn_b200_pack_nvfp4_expert "
                "(fp4_packed) and hidden, inter multiples of 256 up to 16384");
  const bool grouped_ok = !d->has_ternary && !d->has_mxfp4 && H % 256 == 0 && I % 256 == 0;
  if (d->path == FFN_B200_PATH_GROUPED && !grouped_ok)
    return fail(FFN_B200_EUNSUP,
                "moe_layer: the grouped path needs NVFP4-only experts and hidden, inter multiples "
                "of 256");
  if (n_tok == 0) return 0;
  if (!x || !out) return fail(FFN_B200_EINVAL, "moe_layer: null x/out");
  if (n_tok * k > (1u << 24)) return fail(FFN_B200_EINVAL, "moe_layer: too many tokens");
  if (!ws || ws_bytes < ffn_b200_moe_ws_bytes(d, n_tok))
    return fail(FFN_B200_ENOSPC, "moe_layer: workspace too small (see ffn_b200_moe_ws_bytes)");
  cudaStream_t st = (cudaStream_t)stream;
  Carve c(ws);
  MoeWs w = carve_moe(c, *d, n_tok);
  const int T = (int)n_tok, P = (int)(n_tok * k);
  int rc;
  const bool exact = d->router_mode == FFN_B200_ROUTER_EXACT;
  const float *xin = d->norm_w ? w.xn : x;  // what the router and the experts see
  const bool grouped =
      grouped_ok && (d->path == FFN_B200_PATH_GROUPED ||
                     (d->path == FFN_B200_PATH_AUTO && (size_t)P >= (size_t)FFN_B200_GROUPED_MIN_PAIRS * E));
  // (AUTO keeps the GEMV slices for an input row that is not 16-byte aligned)
  const bool fp4 = !grouped && fp4_ok &&
                   (d->path == FFN_B200_PATH_FP4 ||
                    (d->path == FFN_B200_PATH_AUTO && (reinterpret_cast<uintptr_t>(xin) & 15) == 0));
  const bool fused_q = fp4 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(d->norm_w)) & 15) == 0;
  if (fused_q) {
    // one pass: RMSNorm, the router's f16 split and the experts' six NVFP4
    // terms (xn reaches global memory only for the exact router)
    if ((rc = launch_xprep_q4(x, (int)H, T, (int)H, w.xh, w.xl, (int)H, w.xe, d->norm_w, d->norm_eps,
                              exact ? 1 : 0, exact && d->norm_w ? w.xn : nullptr, w.xq, w.xs, w.xqe, st)))
      return rc;
  } else if ((rc = launch_xprep(x, (int)H, T, (int)H, w.xh, w.xl, w.th, w.tl, (int)H, w.xe, st,
                                d->norm_w, d->norm_eps, exact ? 1 : 0, w.xn))) {
    return rc;
  }
  if ((rc = launch_router(d->router_w, d->router_bias, xin, w.xh, w.xl, w.xe, d->router_mode, T,
                          (int)E, (int)H, (int)k, d->score_fn, w.logits, w.idx, w.wt, st)))
    return rc;
  if ((rc = launch_group(w.idx, T, (int)k, (int)E, d->expert_begin, d->expert_end, d->experts,
                         w.ints, w.pair_tok, w.inv, w.vexp_nv, w.vexp_tn, w.n_vexp, st)))
    return rc;
  if (grouped) {
    GroupedArgs g{};
    g.experts = d->experts;
    g.e_begin = d->expert_begin;
    g.e_end = d->expert_end;
    g.n_pairs = P;
    g.hidden = (int)H;
    g.inter = (int)I;
    g.counts = w.ints;
    g.offsets = w.ints + E;
    g.pair_tok = w.pair_tok;
    g.xh = w.xh;
    g.ld_x = (int)H;
    g.xe = w.xe;
    g.h = w.hh;
    g.y = w.y;
    g.chunk_ws = w.chunk;
    g.err = w.err;
    if ((rc = launch_grouped_moe(g, st))) return rc;
    if ((rc = finish_layer(d, w, T, residual, out, w.err, ep, st))) return rc;
    if (topk_idx)
      FFN_CUDA_TRY(cudaMemcpyAsync(topk_idx, w.idx, P * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    if (topk_w)
      FFN_CUDA_TRY(cudaMemcpyAsync(topk_w, w.wt, P * sizeof(float), cudaMemcpyDeviceToDevice, st));
    return 0;
  }
  if (fp4) {
    Fp4Args g{};
    g.experts = d->experts;
    g.e_begin = d->expert_begin;
    g.e_end = d->expert_end;
    g.n_tok = T;
    g.n_pairs = P;
    g.hidden = (int)H;
    g.inter = (int)I;
    g.slices = w.vexp_nv;
    g.n_slices = w.n_vexp;
    g.pair_tok = w.pair_tok;
    g.x = fused_q ? nullptr : xin;  // nullptr: quantised above
    g.xq = w.xq;
    g.xs = w.xs;
    g.xqe = w.xqe;
    g.h = w.hf;
    g.hq = w.hq;
    g.hs = w.hs;
    g.hqe = w.hqe;
    g.y = w.y;
    g.err = w.err;
    if ((rc = launch_fp4_moe(g, st))) return rc;
  } else if ((rc = moe_gemv_experts(d, w, P, xin, st))) {
    return rc;
  }
  if ((rc = finish_layer(d, w, T, residual, out, fp4 ? w.err : nullptr, ep, st))) return rc;
  if (topk_idx)
    FFN_CUDA_TRY(cudaMemcpyAsync(topk_idx, w.idx, P * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  if (topk_w)
    FFN_CUDA_TRY(cudaMemcpyAsync(topk_w, w.wt, P * sizeof(float), cudaMemcpyDeviceToDevice, st));
  return 0;
}

extern "C" {

int ffn_b200_moe_layer(const ffn_b200_moe_desc *d, size_t n_tok, const float *x,
                       const float *residual, float *out, int32_t *topk_idx, float *topk_w,
                       void *ws, size_t ws_bytes, void *stream) {
  return moe_layer_impl(d, n_tok, x, residual, out, topk_idx, topk_w, ws, ws_bytes, stream, nullptr);
}

int ffn_b200_topk(size_t n_tok, size_t n_exp, size_t top_k, int32_t score_fn, const float *logits,
                  size_t n_part, const float *bias, int32_t *idx, float *wt, void *stream) {
  if (n_tok == 0) return 0;
  if (!logits || !idx || !wt) return fail(FFN_B200_EINVAL, "topk: null pointer");
  if (n_exp == 0 || n_exp > 4096 || top_k == 0 || top_k > (size_t)kTopKMax || top_k > n_exp)
    return fail(FFN_B200_EINVAL, "topk: n_exp must be in 1..4096 and top_k in 1..min(16, n_exp)");
  if (n_part == 0 || n_part > (size_t)kRouterPlanes) return fail(FFN_B200_EINVAL, "topk: n_part must be 1..3");
  if (n_tok > (1u << 24)) return fail(FFN_B200_EINVAL, "topk: too many tokens");
  if (score_fn != FFN_B200_SCORE_REF_SQRTSOFTPLUS && score_fn != FFN_B200_SCORE_SIGMOID)
    return fail(FFN_B200_EINVAL, "topk: unknown score_fn");
  return launch_topk(logits, (int)n_part, bias, (int)n_tok, (int)n_exp, (int)top_k, score_fn, idx, wt,
                     (cudaStream_t)stream);
}

int ffn_b200_ep_moe_layer(ffn_b200_ep *ep, const ffn_b200_moe_desc *d, size_t n_tok, const float *x,
                          const float *residual, float *out, int32_t *topk_idx, float *topk_w, void *ws,
                          size_t ws_bytes, void *stream) {
  if (!ep) return fail(FFN_B200_EINVAL, "ep_moe_layer: null exchange");
  return moe_layer_impl(d, n_tok, x, residual, out, topk_idx, topk_w, ws, ws_bytes, stream, ep);
}

// -------------------------------------------------------------- generators
int ffn_b200_gen_nvfp4(uint64_t key, size_t rows, size_t cols, uint8_t *w, uint8_t *s,
                       void *stream) {
  if (!w || !s || cols % 16) return fail(FFN_B200_EINVAL, "gen_nvfp4: bad arguments");
  if ((uintptr_t)w % 8) return fail(FFN_B200_EINVAL, "gen_nvfp4: w must be 8-byte aligned");
  return launch_gen_nvfp4(ffn_b200_key(key, 1), ffn_b200_key(key, 2), rows, cols, w, s,
                          (cudaStream_t)stream);
}
int ffn_b200_gen_ternary(uint64_t key, size_t rows, size_t cols, uint8_t *p, float *rs,
                         void *stream) {
  if (!p || !rs || cols % 4) return fail(FFN_B200_EINVAL, "gen_ternary: bad arguments");
  return launch_gen_ternary(ffn_b200_key(key, 3), ffn_b200_key(key, 4), rows, cols, p, rs,
                            (cudaStream_t)stream);
}
int ffn_b200_gen_core(uint64_t key, size_t rows, size_t cols, int8_t *a, float *a_sc, int8_t *b,
                      float *b_sc, void *stream) {
  if (!a || !a_sc || !b || !b_sc) return fail(FFN_B200_EINVAL, "gen_core: bad arguments");
  return launch_gen_core(ffn_b200_key(key, 5), ffn_b200_key(key, 6), ffn_b200_key(key, 7),
                         ffn_b200_key(key, 8), rows, cols, a, a_sc, b, b_sc, (cudaStream_t)stream);
}
int ffn_b200_gen_normal(uint64_t key, size_t n, float stdev, float *out, void *stream) {
  if (!out) return fail(FFN_B200_EINVAL, "gen_normal: null out");
  return launch_gen_normal(key, n, stdev, out, (cudaStream_t)stream);
}

int ffn_b200_dequant_nvfp4(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s,
                           float *out, void *stream) {
  if (!w || !s || !out || cols % 16) return fail(FFN_B200_EINVAL, "dequant_nvfp4: bad arguments");
  return launch_dequant_nvfp4(rows, cols, w, s, out, (cudaStream_t)stream);
}
int ffn_b200_dequant_ternary(size_t rows, size_t cols, const uint8_t *p, float *out,
                             void *stream) {
  if (!p || !out || cols % 4) return fail(FFN_B200_EINVAL, "dequant_ternary: bad arguments");
  return launch_dequant_ternary(rows, cols, p, out, (cudaStream_t)stream);
}

}  // extern "C"
