/*
 * ffn_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the quantized expert-FFN path of terox27/Flash1017-Engine
 * (Rust crate `flash-core`).  It is the parity checker for the CUDA library and
 * the CPU baseline timed by bench.py.  Nothing in the shipped library links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and the
 * `cpu_baseline` / `--impl reference` legs of bench.py use it.
 *
 * Every function restates one loop of the reference in the same loop order and
 * the same floating-point evaluation order.  Build with -ffp-contract=off: Rust
 * never fuses `a*b + c` unless `mul_add` is written, and the restated loops do
 * not use `mul_add`, so the restatement reproduces the Rust CPU path's rounding.
 * Transcendentals go through the platform libm (expf/logf/sqrtf), which is what
 * Rust's f32::exp/ln/sqrt call on Linux.
 *
 * Parity pinning: the reference cannot be executed here (no Rust toolchain, the
 * shipped binaries are aarch64 and closed).  The restatement is pinned by
 * known-answer vectors derived from the reference's own constant tables
 * (FP4_E2M1_LUT, f8_e4m3_to_f32), by an independent decoder
 * (torch.float8_e4m3fn) over all 256 E4M3 codes, by independent pure-Python
 * restatements evaluated on the reference's own test fixture, and by the
 * reference's own addon micro-benchmark test (hardware_addon.rs:1063-1244,
 * 1250-1294).  The summation-order restatement of the matvec loops is "parity
 * unpinned" against executed reference output.
 *
 * Reference paths below are relative to the reference project root:
 *   F  = crates/flash-core/src/flash1017.rs
 *   HA = crates/flash-core/src/hardware_addon.rs
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* Decoders                                                                   */
/* ------------------------------------------------------------------------- */

/* F:17-20  FP4_E2M1_LUT: nibble -> value; low nibble is the even column. */
static const float E2M1_LUT[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

/* F:2566 ternary LUT: code 0 -> -1, 1 -> 0, 2 -> +1, 3 -> 0. */
static const float TERN_LUT[4] = {-1.0f, 0.0f, 1.0f, 0.0f};

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* F:1031-1045 f8_e4m3_to_f32 (OCP E4M3, bias 7, 0x7F/0xFF -> NaN). */
ORC_API float orc_e4m3_to_f32(uint8_t b) {
    uint32_t sign = ((uint32_t)b & 0x80u) << 24;
    uint32_t em = (uint32_t)b & 0x7Fu;
    if (em == 0x7Fu) return NAN;
    if (em < 8u) {
        float sub = (float)em * (1.0f / 512.0f);
        return bits_f32(sign | f32_bits(sub));
    }
    return bits_f32(sign | ((em + 960u) << 20));
}

ORC_API float orc_e2m1_to_f32(uint8_t nibble) { return E2M1_LUT[nibble & 15u]; }

/* F:1049-1057 f8_e8m0_to_f32: 0xFF -> NaN, 0 -> 2^-127 (f32 bits 0x00400000),
 * else 2^(b - 127) (bits b << 23). */
ORC_API float orc_e8m0_to_f32(uint8_t b) {
    if (b == 0xFFu) return bits_f32(0x7FC00000u);
    if (b == 0u) return bits_f32(0x00400000u);
    return bits_f32((uint32_t)b << 23);
}

/* F:2717-2744 -- one row of CachedMxfp4Mat::matvec: E2M1 pairs, E8M0 scale
 * per 32 columns, no global scale. */
static float mxfp4_row(const uint8_t *w_row, const uint8_t *s_row, size_t cols, const float *x) {
    size_t scale_cols = cols / 32;
    float acc = 0.0f;
    for (size_t g = 0; g < scale_cols; ++g) {
        float sc = orc_e8m0_to_f32(s_row[g]);
        size_t b_off = g * 16, x_off = g * 32;
        float b_sum = 0.0f;
        for (size_t k = 0; k < 16; ++k) {
            uint8_t b = w_row[b_off + k];
            float w0 = E2M1_LUT[b & 0x0F];
            float w1 = E2M1_LUT[b >> 4];
            b_sum += w0 * x[x_off + k * 2] + w1 * x[x_off + k * 2 + 1];
        }
        acc += b_sum * sc;
    }
    return acc;
}

/* F:1960-1982 -- row r of CachedMxfp8Mat::matvec: E4M3 values [rows, cols],
 * E8M0 scales per 32 x 32 block ([ceil(rows/32)... ] row (r/32), column block c/32). */
static float mxfp8_row(const uint8_t *w, const uint8_t *s, size_t r, size_t cols, const float *x) {
    size_t scale_cols = (cols + 31) / 32;
    const uint8_t *w_row = w + r * cols;
    size_t sc_row_off = (r / 32) * scale_cols;
    float acc = 0.0f;
    for (size_t bc = 0; bc < scale_cols; ++bc) {
        float sc = orc_e8m0_to_f32(s[sc_row_off + bc]);
        size_t c_start = bc * 32, c_end = c_start + 32 < cols ? c_start + 32 : cols;
        float b_sum = 0.0f;
        for (size_t c = c_start; c < c_end; ++c) b_sum += orc_e4m3_to_f32(w_row[c]) * x[c];
        acc += b_sum * sc;
    }
    return acc;
}

/* ------------------------------------------------------------------------- */
/* NVFP4 matrix  (F:2282-2391, CachedNvfp4Mat)                                */
/* ------------------------------------------------------------------------- */

/* F:2331-2357 -- one row of CachedNvfp4Mat::matvec (CPU/Rayon branch). */
static float nvfp4_row(const uint8_t *w_row, const uint8_t *sc_row, size_t cols,
                       float g_sc2, const float *x) {
    size_t groups_per_row = cols / 16;
    float row_acc = 0.0f;
    for (size_t g = 0; g < groups_per_row; ++g) {
        float g_sc = orc_e4m3_to_f32(sc_row[g]);
        size_t b_base = g * 8, x_base = g * 16;
        float g_sum = 0.0f;
        for (size_t k = 0; k < 8; ++k) {
            uint8_t b = w_row[b_base + k];
            float v0 = E2M1_LUT[b & 0x0F];
            float v1 = E2M1_LUT[b >> 4];
            g_sum += v0 * x[x_base + k * 2] + v1 * x[x_base + k * 2 + 1];
        }
        row_acc += g_sum * g_sc;
    }
    return row_acc * g_sc2;
}

/* ------------------------------------------------------------------------- */
/* Ternary 1.58-bit matrix (F:2475-2672, CachedTernary158Mat)                 */
/* ------------------------------------------------------------------------- */

/* F:2602-2621 -- one row, no block scales; bytes 0x55 (four zeros) skipped. */
static float ternary_row(const uint8_t *row_b, size_t packed_cols, float sc,
                         const float *x) {
    float acc = 0.0f;
    for (size_t i = 0; i < packed_cols; ++i) {
        uint8_t b = row_b[i];
        if (b == 0x55) continue;
        size_t base = i * 4;
        acc += TERN_LUT[b & 3] * x[base] + TERN_LUT[(b >> 2) & 3] * x[base + 1] +
               TERN_LUT[(b >> 4) & 3] * x[base + 2] + TERN_LUT[(b >> 6) & 3] * x[base + 3];
    }
    return acc * sc;
}

/* F:2567-2601 -- one row with U8 per-64-column block scales. */
static float ternary_row_bs(const uint8_t *row_b, const uint8_t *bs_row, size_t cols,
                            float row_sc, const float *x) {
    size_t blocks_per_row = cols / 64;
    float row_acc = 0.0f;
    for (size_t blk = 0; blk < blocks_per_row; ++blk) {
        uint8_t u8_sc = bs_row[blk];
        if (u8_sc == 0) continue;
        size_t p_off = blk * 16;
        float b_acc = 0.0f;
        for (size_t k = 0; k < 16; ++k) {
            uint8_t b = row_b[p_off + k];
            if (b == 0x55) continue;
            size_t base = (p_off + k) * 4;
            b_acc += TERN_LUT[b & 3] * x[base] + TERN_LUT[(b >> 2) & 3] * x[base + 1] +
                     TERN_LUT[(b >> 4) & 3] * x[base + 2] +
                     TERN_LUT[(b >> 6) & 3] * x[base + 3];
        }
        row_acc += b_acc * (float)u8_sc;
    }
    return row_acc * row_sc;
}

/* ------------------------------------------------------------------------- */
/* Row-parallel driver (mirrors Rayon's par_chunks_exact(..).with_min_len(32)) */
/* Per-row results do not depend on the partitioning, so any thread count     */
/* gives bit-identical output.                                                */
/* ------------------------------------------------------------------------- */

typedef struct {
    int kind; /* 0 nvfp4, 1 ternary, 2 ternary+block scales, 3 mxfp4, 4 mxfp8 */
    size_t rows, cols;
    const uint8_t *w, *s;
    const float *rs;
    float gs;
    const float *x;
    float *out;
    size_t r0, r1;
} row_job;

static void run_rows(row_job *j) {
    for (size_t r = j->r0; r < j->r1; ++r) {
        if (j->kind == 0) {
            j->out[r] = nvfp4_row(j->w + r * (j->cols / 2), j->s + r * (j->cols / 16),
                                  j->cols, j->gs, j->x);
        } else if (j->kind == 1) {
            j->out[r] = ternary_row(j->w + r * (j->cols / 4), j->cols / 4, j->rs[r], j->x);
        } else if (j->kind == 3) {
            j->out[r] = mxfp4_row(j->w + r * (j->cols / 2), j->s + r * (j->cols / 32), j->cols, j->x);
        } else if (j->kind == 4) {
            j->out[r] = mxfp8_row(j->w, j->s, r, j->cols, j->x);
        } else {
            j->out[r] = ternary_row_bs(j->w + r * (j->cols / 4), j->s + r * (j->cols / 64),
                                       j->cols, j->rs[r], j->x);
        }
    }
}

static void *run_rows_thread(void *p) { run_rows((row_job *)p); return NULL; }

static int g_threads = 1;

ORC_API void orc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }
ORC_API int orc_get_threads(void) { return g_threads; }

static void par_rows(row_job base) {
    size_t nt = (size_t)g_threads;
    size_t min_len = 32;
    if (nt <= 1 || base.rows < 2 * min_len) {
        base.r0 = 0; base.r1 = base.rows;
        run_rows(&base);
        return;
    }
    size_t chunk = (base.rows + nt - 1) / nt;
    if (chunk < min_len) chunk = min_len;
    pthread_t th[256];
    int started[256];
    row_job jobs[256];
    size_t n = 0;
    for (size_t r0 = 0; r0 < base.rows && n < 256; r0 += chunk, ++n) {
        jobs[n] = base;
        jobs[n].r0 = r0;
        jobs[n].r1 = r0 + chunk < base.rows ? r0 + chunk : base.rows;
    }
    for (size_t i = 1; i < n; ++i) {
        started[i] = pthread_create(&th[i], NULL, run_rows_thread, &jobs[i]) == 0;
        if (!started[i]) run_rows(&jobs[i]);
    }
    run_rows(&jobs[0]);
    for (size_t i = 1; i < n; ++i)
        if (started[i]) pthread_join(th[i], NULL);
}

/* F:2314-2358 CachedNvfp4Mat::matvec (CPU branch). */
ORC_API void orc_nvfp4_matvec(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s,
                              float gs, const float *x, float *out) {
    row_job j = {0, rows, cols, w, s, NULL, gs, x, out, 0, 0};
    par_rows(j);
}

/* F:2700-2746 CachedMxfp4Mat::matvec (CPU branch): w [rows, cols/2], s E8M0 [rows, cols/32]. */
ORC_API void orc_mxfp4_matvec(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s,
                              const float *x, float *out) {
    row_job j = {3, rows, cols, w, s, NULL, 1.0f, x, out, 0, 0};
    par_rows(j);
}

/* F:1940-1984 CachedMxfp8Mat::matvec (CPU branch): w E4M3 [rows, cols], s E8M0
 * [ceil(rows/32), ceil(cols/32)]. */
ORC_API void orc_mxfp8_matvec(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s,
                              const float *x, float *out) {
    row_job j = {4, rows, cols, w, s, NULL, 1.0f, x, out, 0, 0};
    par_rows(j);
}

/* F:2361-2390 CachedNvfp4Mat::matbatch -> per-token matvec, [seq, rows]. */
ORC_API void orc_nvfp4_matbatch(size_t rows, size_t cols, size_t seq, const uint8_t *w,
                                const uint8_t *s, float gs, const float *xb, float *ob) {
    for (size_t t = 0; t < seq; ++t)
        orc_nvfp4_matvec(rows, cols, w, s, gs, xb + t * cols, ob + t * rows);
}

/* F:2396-2473 CachedRank16Q8Core::apply_add: y += scale * B (diag(a_sc b_sc) A x).
 * a: [rank, cols] i8, b: [rows, rank] i8, a_sc/b_sc: [rank] f32. */
ORC_API void orc_rank16_apply_add(size_t rows, size_t cols, size_t rank, const int8_t *a,
                                  const float *a_sc, const int8_t *b, const float *b_sc,
                                  const float *x, float *y, float scale) {
    if (rank == 0) return;
    float z[32] = {0};
    size_t r_lim = rank < 32 ? rank : 32;
    for (size_t r = 0; r < r_lim; ++r) {
        const int8_t *a_row = a + r * cols;
        float as = a_sc ? a_sc[r] : 1.0f, bs = b_sc ? b_sc[r] : 1.0f;
        float dot = 0.0f;
        for (size_t c = 0; c < cols; ++c) dot += (float)a_row[c] * x[c];
        z[r] = dot * as * bs * scale;
    }
    for (size_t row = 0; row < rows; ++row) {
        const int8_t *b_row = b + row * rank;
        float acc = 0.0f;
        for (size_t r = 0; r < r_lim; ++r) acc += (float)b_row[r] * z[r];
        y[row] += acc;
    }
}

/* Rank-16 core descriptor (the `.core_*` tensors of F:2417-2420). */
typedef struct {
    const int8_t *a;    /* [rank, cols] */
    const float *a_sc;  /* [rank] */
    const int8_t *b;    /* [rows, rank] */
    const float *b_sc;  /* [rank] */
    size_t rank;
} orc_core;

/* F:2538-2627 CachedTernary158Mat::matvec: ternary rows (+ optional U8 block
 * scales), then the rank-16 core if present. */
ORC_API void orc_ternary_matvec(size_t rows, size_t cols, const uint8_t *p, const float *rs,
                                const uint8_t *bs, const orc_core *core, const float *x,
                                float *out) {
    row_job j = {bs ? 2 : 1, rows, cols, p, bs, rs, 1.0f, x, out, 0, 0};
    par_rows(j);
    if (core && core->rank)
        orc_rank16_apply_add(rows, cols, core->rank, core->a, core->a_sc, core->b, core->b_sc,
                             x, out, 1.0f);
}

ORC_API void orc_ternary_matbatch(size_t rows, size_t cols, size_t seq, const uint8_t *p,
                                  const float *rs, const uint8_t *bs, const orc_core *core,
                                  const float *xb, float *ob) {
    for (size_t t = 0; t < seq; ++t)
        orc_ternary_matvec(rows, cols, p, rs, bs, core, xb + t * cols, ob + t * rows);
}

/* BF16 matvec (F:2212-2226, CachedBf16Mat CPU branch): sequential sum. */
ORC_API void orc_bf16_matvec(size_t rows, size_t cols, const uint16_t *w, const float *x,
                             float *out) {
    for (size_t r = 0; r < rows; ++r) {
        float sum = 0.0f;
        for (size_t c = 0; c < cols; ++c) sum += bits_f32((uint32_t)w[r * cols + c] << 16) * x[c];
        out[r] = sum;
    }
}

/* FP32 router matvec: the same loop as the BF16 one over f32 weights (the
 * synthetic configs specify an fp32 router; the reference's router is BF16). */
ORC_API void orc_f32_matvec(size_t rows, size_t cols, const float *w, const float *x,
                            float *out) {
    for (size_t r = 0; r < rows; ++r) {
        float sum = 0.0f;
        for (size_t c = 0; c < cols; ++c) sum += w[r * cols + c] * x[c];
        out[r] = sum;
    }
}

/* F:4880-4891 flash1017_rms_norm: out = x * (1/sqrt(sum(x^2)/n + eps)) * w. */
ORC_API void orc_rms_norm(size_t n, const float *x, const float *w, float eps, float *out) {
    float sum_sq = 0.0f;
    for (size_t i = 0; i < n; ++i) sum_sq += x[i] * x[i];
    float inv_rms = 1.0f / sqrtf(sum_sq / (float)n + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * inv_rms * w[i];
}

/* ------------------------------------------------------------------------- */
/* SwiGLU expert (F:7537-7547 NVFP4, F:7551-7561 ternary)                     */
/* ------------------------------------------------------------------------- */

static inline float rust_clamp(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

/* h_i = min(silu(g_i), 10) * clamp(u_i, -10, 10), silu(g) = g / (1 + e^-g). */
ORC_API void orc_swiglu(size_t n, const float *g, const float *u, float proj_scale,
                        int scaled, float *h) {
    for (size_t i = 0; i < n; ++i) {
        float gv = scaled ? g[i] * proj_scale : g[i];
        float silu = fminf(gv / (1.0f + expf(-gv)), 10.0f);
        float uv = scaled ? u[i] * proj_scale : u[i];
        h[i] = silu * rust_clamp(uv, -10.0f, 10.0f);
    }
}

/* F:4900-4905 flash1017_axpy_f32: dst[i] += scale * src[i]. */
ORC_API void orc_axpy(size_t n, float scale, const float *src, float *dst) {
    for (size_t i = 0; i < n; ++i) dst[i] += scale * src[i];
}

/* One NVFP4 SwiGLU expert, F:7529-7547: y = W2 (min(silu(W1 x),10) * clamp(W3 x)).
 * w[0..2] = (w1, w3, w2) packed, s[0..2] scales, gs[0..2] global scales. */
ORC_API void orc_nvfp4_expert(size_t inter, size_t hidden, const uint8_t *const *w,
                              const uint8_t *const *s, const float *gs, const float *x,
                              float *y, float *scratch /* 3*inter floats */) {
    float *g = scratch, *u = scratch + inter, *h = scratch + 2 * inter;
    orc_nvfp4_matvec(inter, hidden, w[0], s[0], gs[0], x, g);
    orc_nvfp4_matvec(inter, hidden, w[1], s[1], gs[1], x, u);
    orc_swiglu(inter, g, u, 1.0f, 0, h);
    orc_nvfp4_matvec(hidden, inter, w[2], s[2], gs[2], h, y);
}

/* One MXFP4 (F:9103-9158, MTP routed experts) or MXFP8 (F:9132-9142, shared
 * expert) SwiGLU expert: the NVFP4 expert's arithmetic on the other matvecs.
 * fmt 3 = MXFP4, 4 = MXFP8 (row_job kinds). */
ORC_API void orc_mx_expert(int fmt, size_t inter, size_t hidden, const uint8_t *const *w,
                           const uint8_t *const *s, const float *x, float *y, float *scratch) {
    float *g = scratch, *u = scratch + inter, *h = scratch + 2 * inter;
    void (*mv)(size_t, size_t, const uint8_t *, const uint8_t *, const float *, float *) =
        fmt == 3 ? orc_mxfp4_matvec : orc_mxfp8_matvec;
    mv(inter, hidden, w[0], s[0], x, g);
    mv(inter, hidden, w[1], s[1], x, u);
    orc_swiglu(inter, g, u, 1.0f, 0, h);
    mv(hidden, inter, w[2], s[2], h, y);
}

/* One ternary SwiGLU expert, F:7548-7561 (with the rank-16 cores applied inside
 * each matvec as F:2623-2625 does).  g, u are pre-multiplied by proj_scale. */
/* bs: NULL, or 3 pointers (each NULL or U8 block scales [rows, cols/64]) --
 * the 106 GB format writes block scales for every ternary matrix
 * (F:10783-10787), read by F:2567-2601. */
ORC_API void orc_ternary_expert(size_t inter, size_t hidden, const uint8_t *const *p,
                                const float *const *rs, const orc_core *cores /* 3 or NULL */,
                                const uint8_t *const *bs, float proj_scale, const float *x,
                                float *y, float *scratch) {
    float *g = scratch, *u = scratch + inter, *h = scratch + 2 * inter;
    orc_ternary_matvec(inter, hidden, p[0], rs[0], bs ? bs[0] : NULL, cores ? &cores[0] : NULL, x, g);
    orc_ternary_matvec(inter, hidden, p[1], rs[1], bs ? bs[1] : NULL, cores ? &cores[1] : NULL, x, u);
    orc_swiglu(inter, g, u, proj_scale, 1, h);
    orc_ternary_matvec(hidden, inter, p[2], rs[2], bs ? bs[2] : NULL, cores ? &cores[2] : NULL, h, y);
}

/* ------------------------------------------------------------------------- */
/* Router + top-k  (F:7277-7376; batched twin F:7987-8086)                    */
/* ------------------------------------------------------------------------- */

typedef struct { uint32_t e; float biased, score; } cand;

static int cand_desc(const void *pa, const void *pb) {
    const cand *a = (const cand *)pa, *b = (const cand *)pb;
    /* biased descending; the reference's unstable selection leaves ties in an
     * unspecified order -- the oracle breaks them by expert index ascending. */
    if (a->biased > b->biased) return -1;
    if (a->biased < b->biased) return 1;
    return a->e < b->e ? -1 : (a->e > b->e ? 1 : 0);
}

/* score_fn 0: reference sqrt(softplus(l)) + bias, weights score*1.5/sum (F:7280-7376).
 * score_fn 1: sigmoid(l) + bias, weights score/sum (renormalised).
 * logits [n_tok, n_exp] -> idx/wt/score [n_tok, top_k]. */
ORC_API void orc_route(size_t n_tok, size_t n_exp, size_t top_k, const float *logits,
                       const float *bias, int score_fn, int32_t *idx, float *wt,
                       float *score_out, float *biased_out) {
    cand *c = (cand *)malloc(n_exp * sizeof(cand));
    for (size_t t = 0; t < n_tok; ++t) {
        const float *lg = logits + t * n_exp;
        for (size_t e = 0; e < n_exp; ++e) {
            float l = lg[e], score;
            if (score_fn == 0) {
                float softplus = l > 20.0f ? l : (l < -20.0f ? expf(l) : logf(1.0f + expf(l)));
                score = sqrtf(fmaxf(softplus, 0.0f));
            } else {
                score = 1.0f / (1.0f + expf(-l));
            }
            c[e].e = (uint32_t)e;
            c[e].score = score;
            c[e].biased = score + (bias ? bias[e] : 0.0f);
        }
        qsort(c, n_exp, sizeof(cand), cand_desc);
        float sum = 0.0f;
        for (size_t k = 0; k < top_k; ++k) sum += c[k].score;
        float scale = score_fn == 0 ? (sum > 1e-12f ? 1.5f / sum : 0.0f)
                                    : (sum > 1e-12f ? 1.0f / sum : 0.0f);
        for (size_t k = 0; k < top_k; ++k) {
            idx[t * top_k + k] = (int32_t)c[k].e;
            wt[t * top_k + k] = c[k].score * scale;
            if (score_out) score_out[t * top_k + k] = c[k].score;
            if (biased_out) biased_out[t * top_k + k] = c[k].biased;
        }
    }
    free(c);
}

/* Decode MoE combine in the reference's order (F:7521-7566 fallback path, no
 * shared expert): out = 0; for each selected expert k: out += w_k * y_k.
 * y: [n_tok, top_k, hidden] expert outputs, wt: [n_tok, top_k]. */
ORC_API void orc_combine(size_t n_tok, size_t top_k, size_t hidden, const float *y,
                         const float *wt, float *out) {
    for (size_t t = 0; t < n_tok; ++t) {
        float *o = out + t * hidden;
        for (size_t i = 0; i < hidden; ++i) o[i] = 0.0f;
        for (size_t k = 0; k < top_k; ++k)
            orc_axpy(hidden, wt[t * top_k + k], y + (t * top_k + k) * hidden, o);
    }
}

/* ------------------------------------------------------------------------- */
/* Seeded synthetic generators.  Counter-based (SplitMix64 finaliser) so any  */
/* element can be generated independently; integer-only up to exactly rounded */
/* IEEE divisions/multiplications, so the device generator in the CUDA        */
/* library reproduces these bytes exactly.                                     */
/* ------------------------------------------------------------------------- */

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

ORC_API uint64_t orc_derive(uint64_t parent, uint64_t v) {
    return mix64(parent + 0x9E3779B97F4A7C15ULL * (v + 1));
}

static inline uint64_t rnd(uint64_t key, uint64_t i) {
    return mix64(key + 0x9E3779B97F4A7C15ULL * (i + 1));
}

/* N(0,1) by the Irwin-Hall sum of 12 16-bit uniforms: exact integer sum, one
 * exact scaling by 2^-16. */
static inline float normal_at(uint64_t key, uint64_t i) {
    int64_t s = 0;
    for (int d = 0; d < 3; ++d) {
        uint64_t r = rnd(key, 3 * i + (uint64_t)d);
        s += (int64_t)(r & 0xFFFF) + (int64_t)((r >> 16) & 0xFFFF) +
             (int64_t)((r >> 32) & 0xFFFF) + (int64_t)(r >> 48);
    }
    return (float)(s - 393210) * (1.0f / 65536.0f);
}

static inline float unit_at(uint64_t key, uint64_t i) { /* [0,1), 24 bits */
    return (float)(uint32_t)(rnd(key, i) >> 40) * (1.0f / 16777216.0f);
}

/* f32 -> OCP E4M3 with round-to-nearest-even and saturation to +-448. */
ORC_API uint8_t orc_f32_to_e4m3(float f) {
    uint32_t u = f32_bits(f);
    uint32_t sign = (u >> 24) & 0x80u;
    uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint8_t)(sign | 0x7Fu);         /* NaN */
    if (a >= 0x43E00000u) return (uint8_t)(sign | 0x7Eu);         /* >= 448: saturate */
    int e = (int)(a >> 23) - 127;
    if (e < -6) {                                                 /* subnormal: units of 2^-9 */
        /* value / 2^-9 rounded to nearest even; exact in double */
        double v = (double)bits_f32(a) * 512.0;
        double fl = floor(v);
        double rem = v - fl;
        uint32_t q = (uint32_t)fl;
        if (rem > 0.5 || (rem == 0.5 && (q & 1u))) q++;
        return (uint8_t)(sign | q); /* q == 8 rolls into the smallest normal */
    }
    uint32_t mant = a & 0x7FFFFFu;
    uint32_t keep = mant >> 20, rest = mant & 0xFFFFFu;
    uint32_t enc = ((uint32_t)(e + 7) << 3) | keep;
    if (rest > 0x80000u || (rest == 0x80000u && (keep & 1u))) enc++;
    if (enc > 0x7Eu) enc = 0x7Eu;
    return (uint8_t)(sign | enc);
}

/* |N(0,1)| stand-in for block scales: Irwin-Hall sum of the four 16-bit
 * uniforms of one 64-bit draw, centred and scaled to unit variance by one
 * exactly rounded multiplication. */
static inline float normal4_at(uint64_t key, uint64_t i) {
    uint64_t r = rnd(key, i);
    int64_t s = (int64_t)(r & 0xFFFF) + (int64_t)((r >> 16) & 0xFFFF) +
                (int64_t)((r >> 32) & 0xFFFF) + (int64_t)(r >> 48);
    return (float)(s - 131070) * (1.0f / 37837.227f);
}

/* NVFP4 matrix [rows, cols]: E2M1 codes uniform over all 16 values (one 64-bit
 * draw gives 8 packed bytes, little-endian), E4M3 scales RNE(|N(0,1)|/6). */
ORC_API void orc_gen_nvfp4(uint64_t key, size_t rows, size_t cols, uint8_t *w, uint8_t *s) {
    uint64_t kw = orc_derive(key, 1), ks = orc_derive(key, 2);
    size_t nb = rows * cols / 2, ns = rows * cols / 16;
    for (size_t i = 0; i < nb; ++i) w[i] = (uint8_t)(rnd(kw, i >> 3) >> (8 * (i & 7)));
    for (size_t i = 0; i < ns; ++i) s[i] = orc_f32_to_e4m3(fabsf(normal4_at(ks, i)) / 6.0f);
}

/* Ternary matrix [rows, cols]: codes P(-1,0,+1) = (.3,.4,.3), four per byte in
 * the layout of F:10484 (element 4j+i at bits 2i..2i+1); row scales U(.01,.05). */
ORC_API void orc_gen_ternary(uint64_t key, size_t rows, size_t cols, uint8_t *p, float *rs) {
    uint64_t kp = orc_derive(key, 3), kr = orc_derive(key, 4);
    size_t n = rows * cols;
    memset(p, 0, n / 4);
    for (size_t i = 0; i < n; ++i) {
        uint32_t u = (uint32_t)(rnd(kp, i) >> 32);
        uint32_t code = u < 1288490189u ? 0u : (u < 3006477107u ? 1u : 2u);
        p[i >> 2] |= (uint8_t)(code << ((i & 3) * 2));
    }
    for (size_t r = 0; r < rows; ++r) rs[r] = 0.01f + 0.04f * unit_at(kr, r);
}

/* Rank-16 core: int8 uniform in [-127,127], fp32 scales U(1e-4, 1e-3).
 * a = V^T [rank, cols], b = U [rows, rank]. */
ORC_API void orc_gen_core(uint64_t key, size_t rows, size_t cols, size_t rank, int8_t *a,
                          float *a_sc, int8_t *b, float *b_sc) {
    uint64_t ka = orc_derive(key, 5), kb = orc_derive(key, 6), kas = orc_derive(key, 7),
             kbs = orc_derive(key, 8);
    for (size_t i = 0; i < rank * cols; ++i) a[i] = (int8_t)((int)(rnd(ka, i) % 255u) - 127);
    for (size_t i = 0; i < rows * rank; ++i) b[i] = (int8_t)((int)(rnd(kb, i) % 255u) - 127);
    for (size_t r = 0; r < rank; ++r) {
        a_sc[r] = 0.0001f + 0.0009f * unit_at(kas, r);
        b_sc[r] = 0.0001f + 0.0009f * unit_at(kbs, r);
    }
}

/* f32 tensor of n elements ~ N(0,1) * stdev. */
ORC_API void orc_gen_normal(uint64_t key, size_t n, float stdev, float *out) {
    for (size_t i = 0; i < n; ++i) out[i] = normal_at(key, i) * stdev;
}

/* ------------------------------------------------------------------------- */
/* NVFP4 -> 1.58-bit block-64 ternary + rank-16 Q8 core compressor            */
/* (F:10342-10372 orthonormalize_cols_16, F:10377-10645                       */
/* compress_nvfp4_matrix_to_158_jepa_q8), loop for loop.  The writer of the   */
/* 106 GB format stores these outputs as .packed_ternary, .row_scales,        */
/* .block_scales and .core_* (F:10783-10811).                                 */
/* ------------------------------------------------------------------------- */
static void orc_orthonormalize16(float *m /* [n][16] */, size_t n) {
    if (n == 0) return;
    for (int k = 0; k < 16; ++k) {
        for (int j = 0; j < k; ++j) {
            double dot = 0.0;
            for (size_t r = 0; r < n; ++r) dot += (double)m[r * 16 + k] * (double)m[r * 16 + j];
            const float d = (float)dot;
            for (size_t r = 0; r < n; ++r) m[r * 16 + k] -= d * m[r * 16 + j];
        }
        double norm_sq = 0.0;
        for (size_t r = 0; r < n; ++r) {
            const double v = (double)m[r * 16 + k];
            norm_sq += v * v;
        }
        const float inv_norm = norm_sq > 1e-24 ? (float)(1.0 / sqrt(norm_sq)) : 0.0f;
        for (size_t r = 0; r < n; ++r) m[r * 16 + k] *= inv_norm;
    }
}

static float orc_clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* w [rows, cols/2] packed E2M1, s [rows, cols/16] E4M3, gs the per-tensor
 * scale; cols % 64 == 0.  Outputs: packed [rows, cols/4], row_scales [rows],
 * block_scales [rows, cols/64], core_b [rows, 16], core_b_sc [16], core_a
 * [16, cols], core_a_sc [16]; stats (or NULL) = orig_frob_sq, ternary_err_sq,
 * jepa_err_sq.  Returns 0, or -1 for a bad shape / allocation failure. */
ORC_API int orc_compress_ternary_b64(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s,
                                     float gs, uint64_t seed, uint8_t *packed, float *row_scales,
                                     uint8_t *block_scales, int8_t *core_b, float *core_b_sc,
                                     int8_t *core_a, float *core_a_sc, double *stats) {
    if (rows == 0 || cols == 0 || cols % 64) return -1;
    const size_t packed_cols = cols / 2, groups = cols / 16, pcols = (cols + 3) / 4, nblk = cols / 64;
    float *res = (float *)malloc(rows * cols * sizeof(float));
    float *gam = (float *)malloc(nblk * sizeof(float));
    float *p = (float *)malloc(cols * 16 * sizeof(float));
    float *q = (float *)malloc(rows * 16 * sizeof(float));
    float *z = (float *)malloc(cols * 16 * sizeof(float));
    if (!res || !gam || !p || !q || !z) {
        free(res); free(gam); free(p); free(q); free(z);
        return -1;
    }
    memset(packed, 0, rows * pcols);
    double orig = 0.0, terr = 0.0;
    static const float LUT[4] = {-1.0f, 0.0f, 1.0f, 0.0f};
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t *wr = w + r * packed_cols, *sr = s + r * groups;
        float *rr = res + r * cols;
        for (size_t g = 0; g < groups; ++g) {
            const float g_sc = orc_e4m3_to_f32(sr[g]) * gs;
            for (int k = 0; k < 8; ++k) {
                const uint8_t b = wr[g * 8 + k];
                const float w0 = E2M1_LUT[b & 0x0F] * g_sc, w1 = E2M1_LUT[b >> 4] * g_sc;
                rr[g * 16 + 2 * k] = w0;
                rr[g * 16 + 2 * k + 1] = w1;
                orig += (double)w0 * (double)w0 + (double)w1 * (double)w1;
            }
        }
        uint8_t *pr = packed + r * pcols;
        float max_gamma = 0.0f;
        for (size_t blk = 0; blk < nblk; ++blk) {
            const float *wb = rr + blk * 64;
            float sq = 0.0f;
            for (int i = 0; i < 64; ++i) sq += wb[i] * wb[i];
            const float rms = sqrtf(sq * (1.0f / 64.0f));
            if (rms <= 1e-12f) {
                gam[blk] = 0.0f;
                memset(pr + blk * 16, 0x55, 16);
                continue;
            }
            static const float F[4] = {0.42f, 0.54f, 0.66f, 0.78f};
            float best_score = -1.0f, best_gamma = 0.0f, best_th = 0.58f * rms;
            for (int f = 0; f < 4; ++f) {
                const float th = F[f] * rms;
                float dot = 0.0f;
                uint32_t cnt = 0;
                for (int i = 0; i < 64; ++i) {
                    if (wb[i] > th) { dot += wb[i]; ++cnt; }
                    else if (wb[i] < -th) { dot -= wb[i]; ++cnt; }
                }
                if (cnt > 0) {
                    const float score = (dot * dot) / (float)cnt;
                    if (score > best_score) {
                        best_score = score;
                        best_gamma = dot / (float)cnt;
                        best_th = th;
                    }
                }
            }
            gam[blk] = best_gamma;
            if (best_gamma > max_gamma) max_gamma = best_gamma;
            for (int i = 0; i < 64; ++i) {
                const uint8_t code = wb[i] > best_th ? 2 : (wb[i] < -best_th ? 0 : 1);
                pr[blk * 16 + (i >> 2)] |= (uint8_t)(code << ((i & 3) * 2));
            }
        }
        const float row_sc = max_gamma > 1e-12f ? max_gamma / 255.0f : 0.0f;
        row_scales[r] = row_sc;
        for (size_t blk = 0; blk < nblk; ++blk) {
            const uint8_t u8 = row_sc > 0.0f ? (uint8_t)orc_clampf(roundf(gam[blk] / row_sc), 0.0f, 255.0f) : 0;
            block_scales[r * nblk + blk] = u8;
            const float qg = (float)u8 * row_sc;
            float *rb = rr + blk * 64;
            for (int i = 0; i < 16; ++i) {
                const uint8_t pb = pr[blk * 16 + i];
                float v[4];
                for (int u = 0; u < 4; ++u) {
                    v[u] = rb[4 * i + u] - LUT[(pb >> (2 * u)) & 3] * qg;
                    rb[4 * i + u] = v[u];
                }
                /* one expression of four squares, as F:10514-10517 adds them */
                terr += (double)v[0] * (double)v[0] + (double)v[1] * (double)v[1] +
                        (double)v[2] * (double)v[2] + (double)v[3] * (double)v[3];
            }
        }
    }
    /* randomized subspace iteration, rank 16, two sweeps */
    uint64_t rng = seed ^ 0x9E3779B97F4A7C15ull;
    for (size_t c = 0; c < cols; ++c)
        for (int k = 0; k < 16; ++k) {
            rng += 0x9E3779B97F4A7C15ull;
            uint64_t x = rng;
            x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
            x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
            x ^= x >> 31;
            p[c * 16 + k] = (float)((int32_t)(x >> 40) - (1 << 23)) * (1.0f / (float)(1 << 23));
        }
    orc_orthonormalize16(p, cols);
    for (int sweep = 0; sweep < 2; ++sweep) {
        for (size_t r = 0; r < rows; ++r) {
            float acc[16] = {0};
            const float *rr = res + r * cols;
            for (size_t c = 0; c < cols; ++c)
                for (int k = 0; k < 16; ++k) acc[k] += rr[c] * p[c * 16 + k];
            memcpy(q + r * 16, acc, sizeof(acc));
        }
        orc_orthonormalize16(q, rows);
        memset(z, 0, cols * 16 * sizeof(float));
        for (size_t r = 0; r < rows; ++r) {
            const float *rr = res + r * cols;
            for (size_t c = 0; c < cols; ++c)
                for (int k = 0; k < 16; ++k) z[c * 16 + k] += rr[c] * q[r * 16 + k];
        }
        if (sweep == 0) {
            memcpy(p, z, cols * 16 * sizeof(float));
            orc_orthonormalize16(p, cols);
        }
    }
    double captured = 0.0;
    for (int k = 0; k < 16; ++k) {
        float max_u = 0.0f;
        for (size_t r = 0; r < rows; ++r)
            if (fabsf(q[r * 16 + k]) > max_u) max_u = fabsf(q[r * 16 + k]);
        const float b_sc = max_u > 1e-12f ? max_u / 127.0f : 0.0f;
        core_b_sc[k] = b_sc;
        for (size_t r = 0; r < rows; ++r) core_b[r * 16 + k] = 0;
        if (b_sc > 0.0f) {
            const float inv_b = 1.0f / b_sc;
            for (size_t r = 0; r < rows; ++r)
                core_b[r * 16 + k] = (int8_t)orc_clampf(roundf(q[r * 16 + k] * inv_b), -127.0f, 127.0f);
        }
        float max_z = 0.0f;
        double col_norm_sq = 0.0;
        for (size_t c = 0; c < cols; ++c) {
            const float zv = z[c * 16 + k];
            if (fabsf(zv) > max_z) max_z = fabsf(zv);
            col_norm_sq += (double)zv * (double)zv;
        }
        captured += col_norm_sq;
        const float a_sc = max_z > 1e-12f ? max_z / 127.0f : 0.0f;
        core_a_sc[k] = a_sc;
        for (size_t c = 0; c < cols; ++c) core_a[k * cols + c] = 0;
        if (a_sc > 0.0f) {
            const float inv_a = 1.0f / a_sc;
            for (size_t c = 0; c < cols; ++c)
                core_a[k * cols + c] = (int8_t)orc_clampf(roundf(z[c * 16 + k] * inv_a), -127.0f, 127.0f);
        }
    }
    if (stats) {
        stats[0] = orig;
        stats[1] = terr;
        stats[2] = terr - captured > 0.0 ? terr - captured : 0.0;
    }
    free(res); free(gam); free(p); free(q); free(z);
    return 0;
}
