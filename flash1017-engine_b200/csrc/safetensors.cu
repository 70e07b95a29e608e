// safetensors.cu -- routed experts from a .safetensors shard straight into HBM.
//
// The reference maps each shard read-only and borrows tensor bytes from the
// mapping (Flash1017ShardInspector::open / get_tensor_data,
// crates/flash-core/src/flash1017.rs:108-235): an 8-byte little-endian header
// length, a JSON object {name: {dtype, shape, data_offsets: [start, end)}}
// (offsets relative to the end of the header, "__metadata__" skipped), then
// the payload.  Expert matrices are found by name (flash1017.rs:5219-5262):
//   NVFP4    <p>.weight [rows, cols/2] u8, <p>.weight_scale [rows, cols/16]
//            E4M3, <p>.weight_scale_2 f32 scalar (:2295-2309)
//   ternary  <p>.packed_ternary [rows, cols/4] u8, <p>.row_scales [rows] f32,
//            optional <p>.block_scales [rows, cols/64] u8 (:2495-2525) and the
//            rank-16 core <p>.core_b_q8 [rows, 16] i8, <p>.core_a_q8 [16, cols]
//            i8, <p>.core_b_scale / <p>.core_a_scale [16] f32 (:2415-2440)
// with <p> = <expert prefix>.w1 / .w3 / .w2 (gate, up, down).  Here the bytes
// go once into one caller-owned device buffer per expert and the expert
// descriptor points into it; nothing on the host is kept but the mapping.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "ffn_internal.h"

namespace {

struct StTensor {
  std::string dtype;
  std::vector<int64_t> shape;
  size_t start = 0, end = 0;  // payload-relative byte range
};

// A small JSON reader for the header: objects, arrays, strings (with
// escapes), numbers, true / false / null.  Only what a tensor entry needs is
// kept; other values are parsed and dropped.
struct Json {
  const char *p, *e;
  std::string err;
  bool fail(const char *m) {
    if (err.empty()) err = m;
    return false;
  }
  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool lit(const char *s) {
    const size_t n = std::strlen(s);
    if ((size_t)(e - p) < n || std::strncmp(p, s, n)) return fail("bad literal");
    p += n;
    return true;
  }
  bool str(std::string &out) {
    ws();
    if (p >= e || *p != '"') return fail("expected a string");
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= e) return fail("truncated escape");
        const char x = *p++;
        switch (x) {
          case '"': case '\\': case '/': out += x; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (e - p < 4) return fail("truncated \\u escape");
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p++;
              v <<= 4;
              if (h >= '0' && h <= '9') v |= h - '0';
              else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
              else return fail("bad \\u escape");
            }
            if (v < 0x80) out += (char)v;  // tensor names are ASCII; others kept as '?'
            else out += '?';
            break;
          }
          default: return fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (p >= e) return fail("unterminated string");
    ++p;
    return true;
  }
  bool num(double &v, bool &integral, int64_t &iv) {
    ws();
    const char *s = p;
    if (p < e && (*p == '-' || *p == '+')) ++p;
    while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+'))
      ++p;
    if (p == s) return fail("expected a number");
    const std::string t(s, p);
    integral = t.find_first_of(".eE") == std::string::npos;
    char *endp = nullptr;
    if (integral) {
      iv = std::strtoll(t.c_str(), &endp, 10);
      v = (double)iv;
    } else {
      v = std::strtod(t.c_str(), &endp);
      iv = (int64_t)v;
    }
    if (!endp || *endp) return fail("bad number");
    return true;
  }
  bool skip(int depth = 0) {  // any value
    if (depth > 64) return fail("nesting too deep");
    ws();
    if (p >= e) return fail("truncated value");
    if (*p == '{') {
      ++p;
      ws();
      if (p < e && *p == '}') { ++p; return true; }
      for (;;) {
        std::string k;
        if (!str(k)) return false;
        ws();
        if (p >= e || *p++ != ':') return fail("expected ':'");
        if (!skip(depth + 1)) return false;
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (*p == '[') {
      ++p;
      ws();
      if (p < e && *p == ']') { ++p; return true; }
      for (;;) {
        if (!skip(depth + 1)) return false;
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (*p == '"') { std::string s; return str(s); }
    if (*p == 't') return lit("true");
    if (*p == 'f') return lit("false");
    if (*p == 'n') return lit("null");
    double v; bool in; int64_t iv;
    return num(v, in, iv);
  }
  bool int_array(std::vector<int64_t> &out) {
    ws();
    if (p >= e || *p != '[') return fail("expected an array");
    ++p;
    out.clear();
    ws();
    if (p < e && *p == ']') { ++p; return true; }
    for (;;) {
      double v; bool in; int64_t iv;
      if (!num(v, in, iv)) return false;
      if (!in || iv < 0) return fail("expected a non-negative integer");
      out.push_back(iv);
      ws();
      if (p < e && *p == ',') { ++p; continue; }
      if (p < e && *p == ']') { ++p; return true; }
      return fail("expected ',' or ']'");
    }
  }
  bool tensor(StTensor &t) {  // {"dtype": ..., "shape": [...], "data_offsets": [a, b]}
    ws();
    if (p >= e || *p != '{') return fail("tensor entry is not an object");
    ++p;
    bool has_dt = false, has_sh = false, has_off = false;
    ws();
    if (p < e && *p == '}') return fail("empty tensor entry");
    for (;;) {
      std::string k;
      if (!str(k)) return false;
      ws();
      if (p >= e || *p++ != ':') return fail("expected ':'");
      if (k == "dtype") {
        if (!str(t.dtype)) return false;
        has_dt = true;
      } else if (k == "shape") {
        if (!int_array(t.shape)) return false;
        has_sh = true;
      } else if (k == "data_offsets") {
        std::vector<int64_t> o;
        if (!int_array(o)) return false;
        if (o.size() != 2 || o[0] > o[1]) return fail("bad data_offsets");
        t.start = (size_t)o[0];
        t.end = (size_t)o[1];
        has_off = true;
      } else if (!skip()) {
        return false;
      }
      ws();
      if (p < e && *p == ',') { ++p; continue; }
      if (p < e && *p == '}') { ++p; break; }
      return fail("expected ',' or '}'");
    }
    if (!has_dt || !has_sh || !has_off) return fail("tensor entry lacks dtype, shape or data_offsets");
    return true;
  }
};

size_t dtype_bytes(const std::string &d) {
  if (d == "U8" || d == "I8" || d == "F8_E4M3" || d == "F8_E5M2" || d == "F8_E8M0" || d == "BOOL") return 1;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  return 0;
}

}  // namespace

struct ffn_b200_st {
  int fd = -1;
  const uint8_t *map = nullptr;
  size_t size = 0, payload = 0;
  std::unordered_map<std::string, StTensor> tensors;
  std::vector<std::string> names;  // header order
};

namespace {

using ffn::fail;

int st_fail(ffn_b200_st *st, int code, const std::string &msg) {
  if (st) {
    if (st->map) munmap(const_cast<uint8_t *>(st->map), st->size);
    if (st->fd >= 0) close(st->fd);
    delete st;
  }
  return fail(code, msg);
}

// The tensor's bytes, checked against an expected dtype size and shape.
int get(const ffn_b200_st *st, const std::string &name, size_t elem, std::initializer_list<int64_t> shape,
        const uint8_t **data, size_t *nbytes) {
  auto it = st->tensors.find(name);
  if (it == st->tensors.end()) return fail(FFN_B200_EINVAL, "safetensors: no tensor '" + name + "'");
  const StTensor &t = it->second;
  const size_t eb = dtype_bytes(t.dtype);
  if (eb != elem) return fail(FFN_B200_EINVAL, "safetensors: '" + name + "' has dtype " + t.dtype);
  size_t n = 1;
  std::vector<int64_t> want(shape);
  if (!want.empty()) {
    // a scalar may be stored with shape [] or [1]
    const bool scalar_ok = want.size() == 1 && want[0] == 1 && t.shape.empty();
    if (!scalar_ok && t.shape != want) {
      std::string s = "safetensors: '" + name + "' has shape [";
      for (size_t i = 0; i < t.shape.size(); ++i) s += (i ? "," : "") + std::to_string(t.shape[i]);
      return fail(FFN_B200_EINVAL, s + "]");
    }
    for (int64_t d : want) n *= (size_t)d;
  }
  if (t.end - t.start != n * elem) return fail(FFN_B200_EINVAL, "safetensors: '" + name + "' byte length mismatch");
  *data = st->map + st->payload + t.start;
  *nbytes = n * elem;
  return 0;
}

bool has(const ffn_b200_st *st, const std::string &name) { return st->tensors.count(name) != 0; }

#define ST_TRY(expr)           \
  do {                         \
    const int st_rc_ = (expr); \
    if (st_rc_) return st_rc_; \
  } while (0)

// One matrix's tensors: (device offset, host bytes, length) triples.
struct Piece {
  const uint8_t *src;
  size_t n;
  size_t off;
};

struct ExpertPlan {
  int format = FFN_B200_FMT_NVFP4;
  size_t bytes = 0;
  std::vector<Piece> pieces;
  ffn_b200_expert e{};  // offsets (as pointers from 0) until relocated
};

int plan_expert(const ffn_b200_st *st, const std::string &prefix, size_t hidden, size_t inter, ExpertPlan &pl) {
  if (!hidden || !inter || hidden % 64 || inter % 64)
    return fail(FFN_B200_EINVAL, "safetensors: hidden and inter must be positive multiples of 64");
  const char *mname[3] = {".w1", ".w3", ".w2"};  // gate, up, down
  const size_t rows_of[3] = {inter, inter, hidden}, cols_of[3] = {hidden, hidden, inter};
  pl = ExpertPlan{};
  // NVFP4: .weight + .weight_scale (+ .weight_scale_2); MXFP4 (CachedMxfp4Mat,
  // flash1017.rs:2688-2699): .weight + .scale; else ternary
  pl.format = has(st, prefix + ".w1.weight")
                  ? (has(st, prefix + ".w1.weight_scale") ? FFN_B200_FMT_NVFP4 : FFN_B200_FMT_MXFP4)
                  : FFN_B200_FMT_TERNARY;
  // MXFP8 (CachedMxfp8Mat, the shared experts, flash1017.rs:1928-1939): .weight
  // + .scale with one byte per weight
  if (pl.format == FFN_B200_FMT_MXFP4) {
    const StTensor &w1 = st->tensors.at(prefix + ".w1.weight");
    if (w1.shape.size() == 2 && (size_t)w1.shape[1] == hidden) pl.format = FFN_B200_FMT_MXFP8;
  }
  if (pl.format == FFN_B200_FMT_TERNARY && !has(st, prefix + ".w1.packed_ternary"))
    return fail(FFN_B200_EINVAL, "safetensors: no expert '" + prefix + "' (neither .w1.weight nor .w1.packed_ternary)");
  auto add = [&](const uint8_t *src, size_t n) {
    const size_t off = pl.bytes;
    pl.pieces.push_back({src, n, off});
    pl.bytes = (pl.bytes + n + 255) & ~(size_t)255;
    return off;
  };
  pl.e.format = pl.format;
  pl.e.proj_scale = 1.0f;  // 1 for the 106 GB format (flash1017.rs:5105-5114); callers may override
  for (int i = 0; i < 3; ++i) {
    const std::string p = prefix + mname[i];
    const int64_t R = (int64_t)rows_of[i], Cc = (int64_t)cols_of[i];
    const uint8_t *d;
    size_t n;
    if (pl.format == FFN_B200_FMT_NVFP4) {
      ST_TRY(get(st, p + ".weight", 1, {R, Cc / 2}, &d, &n));
      pl.e.nv[i].w = (const uint8_t *)(uintptr_t)add(d, n);
      ST_TRY(get(st, p + ".weight_scale", 1, {R, Cc / 16}, &d, &n));
      pl.e.nv[i].s = (const uint8_t *)(uintptr_t)add(d, n);
      ST_TRY(get(st, p + ".weight_scale_2", 4, {1}, &d, &n));
      std::memcpy(&pl.e.nv[i].gs, d, 4);  // little-endian f32 (flash1017.rs:2299)
    } else if (pl.format == FFN_B200_FMT_MXFP8) {
      ST_TRY(get(st, p + ".weight", 1, {R, Cc}, &d, &n));
      pl.e.nv[i].w = (const uint8_t *)(uintptr_t)add(d, n);
      ST_TRY(get(st, p + ".scale", 1, {(R + 31) / 32, (Cc + 31) / 32}, &d, &n));
      pl.e.nv[i].s = (const uint8_t *)(uintptr_t)add(d, n);
      // gs = 2^B, B = largest finite scale byte - 134 (FFN_B200_FMT_MXFP8)
      int mx = -1;
      for (size_t q = 0; q < n; ++q)
        if (d[q] != 0xFF && d[q] > mx) mx = d[q];
      pl.e.nv[i].gs = std::ldexp(1.0f, mx < 0 ? 0 : mx - 134);
    } else if (pl.format == FFN_B200_FMT_MXFP4) {
      ST_TRY(get(st, p + ".weight", 1, {R, Cc / 2}, &d, &n));
      pl.e.nv[i].w = (const uint8_t *)(uintptr_t)add(d, n);
      ST_TRY(get(st, p + ".scale", 1, {R, Cc / 32}, &d, &n));
      pl.e.nv[i].s = (const uint8_t *)(uintptr_t)add(d, n);
      // gs = 2^B, B = largest finite block scale byte - 140: that block
      // decodes to 2^13 in f16 (FFN_B200_FMT_MXFP4)
      int mx = -1;
      for (size_t q = 0; q < n; ++q)
        if (d[q] != 0xFF && d[q] > mx) mx = d[q];
      pl.e.nv[i].gs = std::ldexp(1.0f, mx < 0 ? 0 : mx - 140);
    } else {
      ffn_b200_ternary_mat &m = pl.e.tn[i];
      ST_TRY(get(st, p + ".packed_ternary", 1, {R, Cc / 4}, &d, &n));
      m.p = (const uint8_t *)(uintptr_t)add(d, n);
      ST_TRY(get(st, p + ".row_scales", 4, {R}, &d, &n));
      m.rs = (const float *)(uintptr_t)add(d, n);
      if (has(st, p + ".block_scales")) {
        ST_TRY(get(st, p + ".block_scales", 1, {R, Cc / 64}, &d, &n));
        m.bs = (const uint8_t *)(uintptr_t)add(d, n);
      }
      const bool core = has(st, p + ".core_a_q8") || has(st, p + ".core_b_q8");
      if (core) {
        ST_TRY(get(st, p + ".core_b_q8", 1, {R, 16}, &d, &n));
        m.core_b = (const int8_t *)(uintptr_t)add(d, n);
        ST_TRY(get(st, p + ".core_a_q8", 1, {16, Cc}, &d, &n));
        m.core_a = (const int8_t *)(uintptr_t)add(d, n);
        ST_TRY(get(st, p + ".core_b_scale", 4, {16}, &d, &n));
        m.core_b_sc = (const float *)(uintptr_t)add(d, n);
        ST_TRY(get(st, p + ".core_a_scale", 4, {16}, &d, &n));
        m.core_a_sc = (const float *)(uintptr_t)add(d, n);
      }
    }
  }
  return 0;
}

template <typename T>
T *reloc(T *off, uint8_t *base) {
  return off ? reinterpret_cast<T *>(base + reinterpret_cast<uintptr_t>(off)) : nullptr;
}
// a zero offset is a real (first) piece for w / p, never absent
template <typename T>
T *reloc_first(T *off, uint8_t *base) {
  return reinterpret_cast<T *>(base + reinterpret_cast<uintptr_t>(off));
}

}  // namespace

extern "C" {

int ffn_b200_st_open(const char *path, ffn_b200_st **out) {
  if (!path || !out) return fail(FFN_B200_EINVAL, "st_open: null argument");
  *out = nullptr;
  ffn_b200_st *st = new ffn_b200_st();
  st->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (st->fd < 0) return st_fail(st, FFN_B200_EINVAL, std::string("st_open: cannot open ") + path);
  struct stat sb;
  if (fstat(st->fd, &sb) != 0) return st_fail(st, FFN_B200_EINVAL, "st_open: fstat failed");
  st->size = (size_t)sb.st_size;
  if (st->size < 8) return st_fail(st, FFN_B200_EINVAL, "st_open: file too small to be a safetensors archive");
  void *m = mmap(nullptr, st->size, PROT_READ, MAP_PRIVATE, st->fd, 0);
  if (m == MAP_FAILED) return st_fail(st, FFN_B200_EINVAL, "st_open: mmap failed");
  st->map = static_cast<const uint8_t *>(m);
  uint64_t hl = 0;
  for (int i = 7; i >= 0; --i) hl = (hl << 8) | st->map[i];  // little-endian header length
  if (hl > st->size - 8) return st_fail(st, FFN_B200_EINVAL, "st_open: file shorter than its header length");
  st->payload = 8 + (size_t)hl;
  Json j{reinterpret_cast<const char *>(st->map + 8), reinterpret_cast<const char *>(st->map + 8 + hl), {}};
  j.ws();
  if (j.p >= j.e || *j.p != '{') return st_fail(st, FFN_B200_EINVAL, "st_open: header is not a JSON object");
  ++j.p;
  j.ws();
  bool empty = j.p < j.e && *j.p == '}';
  if (empty) ++j.p;
  while (!empty) {
    std::string name;
    if (!j.str(name)) return st_fail(st, FFN_B200_EINVAL, "st_open: header: " + j.err);
    j.ws();
    if (j.p >= j.e || *j.p++ != ':') return st_fail(st, FFN_B200_EINVAL, "st_open: header: expected ':'");
    if (name == "__metadata__") {
      if (!j.skip()) return st_fail(st, FFN_B200_EINVAL, "st_open: header: " + j.err);
    } else {
      StTensor t;
      if (!j.tensor(t)) return st_fail(st, FFN_B200_EINVAL, "st_open: header: '" + name + "': " + j.err);
      if (t.end > st->size - st->payload)
        return st_fail(st, FFN_B200_EINVAL, "st_open: data offsets of '" + name + "' run past the end of the file");
      if (!st->tensors.emplace(name, t).second)
        return st_fail(st, FFN_B200_EINVAL, "st_open: tensor '" + name + "' listed twice");
      st->names.push_back(name);
    }
    j.ws();
    if (j.p < j.e && *j.p == ',') { ++j.p; continue; }
    if (j.p < j.e && *j.p == '}') { ++j.p; break; }
    return st_fail(st, FFN_B200_EINVAL, "st_open: header: expected ',' or '}'");
  }
  *out = st;
  return 0;
}

int ffn_b200_st_close(ffn_b200_st *st) {
  if (!st) return 0;
  if (st->map) munmap(const_cast<uint8_t *>(st->map), st->size);
  if (st->fd >= 0) close(st->fd);
  delete st;
  return 0;
}

size_t ffn_b200_st_count(const ffn_b200_st *st) { return st ? st->names.size() : 0; }

const char *ffn_b200_st_name(const ffn_b200_st *st, size_t i) {
  return st && i < st->names.size() ? st->names[i].c_str() : nullptr;
}

int ffn_b200_st_find(const ffn_b200_st *st, const char *name, const char **dtype, int64_t *shape,
                     int *ndim, const void **data, size_t *nbytes) {
  if (!st || !name) return fail(FFN_B200_EINVAL, "st_find: null argument");
  auto it = st->tensors.find(name);
  if (it == st->tensors.end()) return fail(FFN_B200_EINVAL, std::string("st_find: no tensor '") + name + "'");
  const StTensor &t = it->second;
  if (dtype) *dtype = t.dtype.c_str();
  if (ndim) *ndim = (int)t.shape.size();
  if (shape)
    for (size_t i = 0; i < t.shape.size() && i < 8; ++i) shape[i] = t.shape[i];
  if (data) *data = st->map + st->payload + t.start;
  if (nbytes) *nbytes = t.end - t.start;
  return 0;
}

int ffn_b200_st_expert_bytes(const ffn_b200_st *st, const char *prefix, size_t hidden, size_t inter,
                             int *format, size_t *bytes) {
  if (!st || !prefix) return fail(FFN_B200_EINVAL, "st_expert_bytes: null argument");
  ExpertPlan pl;
  const int rc = plan_expert(st, prefix, hidden, inter, pl);
  if (rc) return rc;
  if (format) *format = pl.format;
  if (bytes) *bytes = pl.bytes;
  return 0;
}

int ffn_b200_st_load_expert(const ffn_b200_st *st, const char *prefix, size_t hidden, size_t inter,
                            void *dev, size_t dev_bytes, void *stream, ffn_b200_expert *e) {
  if (!st || !prefix || !dev || !e) return fail(FFN_B200_EINVAL, "st_load_expert: null argument");
  if (reinterpret_cast<uintptr_t>(dev) & 255) return fail(FFN_B200_EINVAL, "st_load_expert: dev must be 256-byte aligned");
  ExpertPlan pl;
  int rc = plan_expert(st, prefix, hidden, inter, pl);
  if (rc) return rc;
  if (dev_bytes < pl.bytes) return fail(FFN_B200_ENOSPC, "st_load_expert: device buffer too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t *base = static_cast<uint8_t *>(dev);
  for (const Piece &pc : pl.pieces)
    FFN_CUDA_TRY(cudaMemcpyAsync(base + pc.off, pc.src, pc.n, cudaMemcpyHostToDevice, s));
  ffn_b200_expert out = pl.e;
  for (int i = 0; i < 3; ++i) {
    if (pl.format != FFN_B200_FMT_TERNARY) {
      out.nv[i].w = reloc_first(pl.e.nv[i].w, base);
      out.nv[i].s = reloc_first(pl.e.nv[i].s, base);
    } else {
      ffn_b200_ternary_mat &m = out.tn[i];
      const ffn_b200_ternary_mat &o = pl.e.tn[i];
      m.p = reloc_first(o.p, base);
      m.rs = reloc_first(o.rs, base);
      m.bs = reloc(o.bs, base);
      m.core_a = reloc(o.core_a, base);
      m.core_b = reloc(o.core_b, base);
      m.core_a_sc = reloc(o.core_a_sc, base);
      m.core_b_sc = reloc(o.core_b_sc, base);
    }
  }
  *e = out;
  return 0;
}

}  // extern "C"
