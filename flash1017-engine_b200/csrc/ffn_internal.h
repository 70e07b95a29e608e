// ffn_internal.h -- declarations shared by the CUDA launchers and the C-ABI layers.
#pragma once

#include "common.cuh"

namespace ffn {

// Arguments of the grouped expert GEMV phases (see phase_kernel in ffn_kernels.cu).
struct PhaseArgs {
  const ffn_b200_expert *experts;  // device table (list mode)
  ffn_b200_expert direct;          // the expert of direct mode
  const VExp *vexp;                // list mode: slices; nullptr = direct mode
  const int *n_vexp_dev;           // list mode: number of slices
  int n_tok_direct;                // direct mode: tokens (slices of 8)
  int rows, K, blocks;             // output rows, reduction length, row blocks per slice
  // input activations (rows indexed by pair, or by pair_tok[pair] when set)
  const __half *xh, *xl;
  const int *xe;                   // per-row power-of-two exponent, or nullptr (0)
  int ld_x;
  const int *pair_tok;
  // rank-16 core terms z[pair][3][16] (ternary experts with cores)
  const float *z;
  // outputs
  __half *hh, *hl;  // phase 1: h [pair][rows]
  int ld_h;
  float *y;         // phase 2 list mode: y [pair][rows]; phase 0/2 direct: out [tok][rows]
  int ld_y;
  float out_w;      // direct mode epilogue weight
  int accumulate;   // direct mode: out += w*y (1) or out = w*y (0)
  int mat;          // phase 0: matrix index of `direct` used
  // K-splits (direct mode): each task's K-chunks are divided among `splits`
  // warps; they leave partial sums in part[task][split][NMAT][pt][ROWS] and
  // the last to arrive (cnt[task], zeroed before the launch) adds them up in
  // split order and runs the epilogue.  splits = 1: no partials.
  int splits = 1;
  int pt = 0;       // tokens per slice held in part (min(8, tokens))
  float *part;
  int *cnt;
};

// Tensor-core grouped MoE path (many tokens per expert; NVFP4 experts).
struct GroupedArgs {
  const ffn_b200_expert *experts;
  int e_begin, e_end;
  int n_pairs;
  int hidden, inter;
  const int *counts, *offsets;  // per expert, from the grouping kernel
  const int32_t *pair_tok;
  const __half *xh;             // f16 of x * 2^-xe, natural order [token][hidden]
  int ld_x;
  const int *xe;
  __half *h;                    // [pair][inter]
  float *y;                     // [pair][hidden]
  uint8_t *chunk_ws;            // gg_chunk_bytes(n_pairs, e_end - e_begin)
  int *err;                     // device int, nonzero after a timed-out wait
};
size_t gg_chunk_bytes(int n_pairs, int n_local);
int launch_grouped_moe(const GroupedArgs &g, cudaStream_t st);

// Block-scaled FP4 tensor-core MoE path (NVFP4 experts packed by
// ffn_b200_pack_nvfp4_expert, decode-sized chunks); activations as kFp4Terms
// NVFP4 terms.
constexpr int kFp4Terms = 6;
struct Fp4Args {
  const ffn_b200_expert *experts;
  int e_begin, e_end;
  int n_tok, n_pairs;
  int hidden, inter;
  const VExp *slices;           // the grouping kernel's NVFP4 slices (<= 8 pairs of one expert)
  const int *n_slices;          // their count (device)
  const int32_t *pair_tok;
  const float *x;               // [n_tok][hidden] f32, the layer input the experts see, or
                                // nullptr when xq/xs/xqe already hold its terms (launch_xprep_q4)
  uint8_t *xq, *xs;             // x as kFp4Terms NVFP4 terms: codes [tok][t][hidden/2], scales [tok][t][hidden/16]
  int *xqe;                     // [tok][t] exponents
  float *h;                     // [pair][inter] f32
  uint8_t *hq, *hs;             // h as kFp4Terms NVFP4 terms
  int *hqe;
  float *y;                     // [pair][hidden]
  int *err;                     // device int: 1 timed-out wait, 3 an expert without stage images
};
int launch_fp4_moe(const Fp4Args &g, cudaStream_t st);

// One NVFP4 / MXFP4 SwiGLU expert over 1..8 tokens in two launches
// (expert_decode.cu).  fits: the format, shapes, alignment and shared-memory
// budget the kernels take; ws holds h [seq][inter] f32 (16-byte aligned).
bool expert_decode_fits(const ffn_b200_expert &e, size_t inter, size_t hidden, size_t seq);
size_t expert_decode_ws_bytes(size_t inter, size_t seq);
int launch_expert_decode(const ffn_b200_expert &e, size_t inter, size_t hidden, size_t seq, const float *x,
                         float *out, float accum_weight, int accumulate, void *ws, cudaStream_t st);
// rows of f32 (K % 256 == 0, K <= 16384, 16-byte aligned rows) -> `terms` NVFP4 terms
int launch_q4(const float *x, int ld_x, int rows, int K, int terms, uint8_t *qc, uint8_t *qs, int *qe,
              cudaStream_t st);
// launch_xprep's natural-order output (RMSNorm, f16 hi/lo split, exponents;
// xn only when non-null) and launch_q4 of the normalised rows, in one kernel
int launch_xprep_q4(const float *x, int ld_x, int rows, int K, __half *nh, __half *nl, int ld_o, int *xe,
                    const float *norm_w, float norm_eps, int seq_norm, float *xn, uint8_t *qc,
                    uint8_t *qs, int *qe, cudaStream_t st);

// The MoE layer's per-pair expert outputs, combined per token inside the
// expert-parallel exchange (the fused form of launch_combine).
struct EpCombine {
  const float *y;             // [pair][ld_y] expert outputs (unweighted)
  int ld_y;
  const int32_t *idx;         // [tok][top_k] routed experts
  const float *wt;            // [tok][top_k] routing weights
  const int32_t *inv;         // [tok][top_k] pair row of each local route, -1 when not local
  int top_k;
  const ffn_b200_expert *experts;
  const int *err;             // upstream error word (nonzero: NaN partials), or nullptr
  int n_exp;                  // experts in the table (a route outside it: NaN partial)
  int y_rows;                 // rows of y (the layer's routed pairs)
};
// One exchange call over ep's ranks: out = residual + sum over ranks of each
// rank's partial (its part buffer, or its combined expert outputs).
int ep_exchange(ffn_b200_ep *ep, size_t n_tok, const EpCombine *comb, const float *residual, float *out,
                cudaStream_t st);

// Arguments of the rank-16 core z kernel.
struct CoreZArgs {
  const ffn_b200_expert *experts;
  ffn_b200_expert direct;
  const VExp *vexp;
  const int *n_vexp_dev;
  int n_tok_direct;
  int K;
  int mat0, nmat;            // matrices [mat0, mat0 + nmat)
  const float *xf;           // f32 input rows (gate/up cores), or nullptr
  int ld_xf;
  const int *pair_tok;
  const __half *hh, *hl;     // pair-order f16 input rows (down core)
  int ld_h;
  float *z;                  // [pair][3][16]
};

int rows_per_tile(int phase);
int chunk_cols(int fmt);  // K columns per ring unit

// A queue of routed expert calls run together as one routed layer.  Call c
// applies experts[c] (NVFP4, MXFP4, ternary or MXFP8) to the x rows row0[c] ..
// row0[c] + m[c] - 1 (1 <= m[c] <= kNTok); its m[c] output rows are the pairs
// pos0[c] .. pos0[c] + m[c] - 1, numbered in call order.  Output row r then
// receives, in list order, starting from 0 when row_zero[r] is set, else from
// out[r],
//   out[r] = fl(out[r] + fl(w[e] * y[pair[e]]))  for e in [tok_ptr[r], tok_ptr[r + 1]),
// which is the one-call-at-a-time arithmetic when the list is in call order
// (a first call that overwrites: row_zero).  All arrays here are HOST arrays;
// experts hold device weight pointers.
struct RoutedCalls {
  const ffn_b200_expert *experts;
  const int32_t *row0, *m;
  int n;
  const int32_t *tok_ptr;  // [out_rows + 1], tok_ptr[out_rows] = sum of m
  const int32_t *ent_pair;
  const float *ent_w;
  const uint8_t *row_zero;  // [out_rows] or nullptr (none)
  int out_rows;
  const float *x;  // device [x_rows][hidden]
  int x_rows;
  float *out;      // device [out_rows][hidden]
  // optional side stream and two events: independent slice lists run on it
  // concurrently with the largest one (forked and joined on the call's stream)
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
// Argument checks of the expert entry points: the shape rules alone (before
// any weight bytes are read from the caller's pointers), and the full check
// of a descriptor holding device pointers.
int validate_expert_shape(int format, size_t inter, size_t hidden, const char *what);
int validate_expert(const ffn_b200_expert &e, size_t inter, size_t hidden, const char *what);
constexpr int kCallsMax = 64;  // calls per routed_calls run
size_t routed_calls_ws_bytes(size_t inter, size_t hidden, int n, int x_rows, int out_rows);
size_t routed_calls_stage_bytes(int n, int out_rows);
// `stage`: routed_calls_stage_bytes of host memory for the call tables (pinned
// or pageable), which the caller leaves untouched until the stream has passed
// this point.
int routed_calls(const RoutedCalls &q, size_t inter, size_t hidden, void *stage, void *ws,
                 size_t ws_bytes, cudaStream_t st);
int launch_rows_accum(const float *y, const int32_t *tok_ptr, const int32_t *ent_pair,
                      const float *ent_w, const uint8_t *row_zero, int out_rows, int H, float *out,
                      cudaStream_t st);
int sm_count_of(int dev);  // multiprocessors of device `dev` (cached)
int launch_xprep(const float *x, int ld_x, int rows, int K, __half *nh, __half *nl, __half *th,
                 __half *tl, int ld_o, int *xe, cudaStream_t st, const float *norm_w = nullptr,
                 float norm_eps = 0.f, int seq_norm = 0, float *xn = nullptr);
int launch_phase(int fmt, int phase, const PhaseArgs &a, long long tasks, cudaStream_t st);
int launch_corez(const CoreZArgs &a, int max_vexp, cudaStream_t st);
int launch_exact_matvec(const float *w32, const uint16_t *w16, const float *x, int n_tok,
                        int rows, int H, float *out, cudaStream_t st);
int launch_router(const float *w, const float *bias, const float *x, const __half *xh,
                  const __half *xl, const int *xe, int mode, int n_tok, int n_exp, int H,
                  int top_k, int score_fn, float *logits /* 4 planes of n_tok x n_exp */,
                  int32_t *idx, float *wt,
                  cudaStream_t st);
// top_k per token from n_part partial logit planes [n_part][n_tok][n_exp] (added in plane order)
int launch_topk(const float *logits, int n_part, const float *bias, int n_tok, int n_exp, int top_k,
                int score_fn, int32_t *idx, float *wt, cudaStream_t st);
constexpr int kRouterPlanes = 3;  // partial logit planes the tensor router writes at most
int launch_group(const int32_t *idx, int n_tok, int top_k, int n_exp, int e_begin, int e_end,
                 const ffn_b200_expert *experts, int *ws_int, int32_t *pair_tok, int32_t *inv,
                 VExp *vexp_nv, VExp *vexp_tn, int *n_vexp, cudaStream_t st);
int launch_combine(const float *y, int ld_y, const int32_t *idx, const float *wt,
                   const int32_t *inv, int n_tok, int top_k, const ffn_b200_expert *experts,
                   const float *residual, float *out, int H, cudaStream_t st,
                   const int *err, int n_exp);
int launch_dot(int mode, const void *a, const void *aux, const float *x, size_t len, float *out,
               cudaStream_t st);
int launch_gen_nvfp4(uint64_t kw, uint64_t ks, size_t rows, size_t cols, uint8_t *w, uint8_t *s,
                     cudaStream_t st);
int launch_gen_ternary(uint64_t kp, uint64_t kr, size_t rows, size_t cols, uint8_t *p, float *rs,
                       cudaStream_t st);
int launch_gen_core(uint64_t ka, uint64_t kb, uint64_t kas, uint64_t kbs, size_t rows,
                    size_t cols, int8_t *a, float *a_sc, int8_t *b, float *b_sc, cudaStream_t st);
int launch_gen_normal(uint64_t key, size_t n, float stdev, float *out, cudaStream_t st);
int launch_dequant_nvfp4(size_t rows, size_t cols, const uint8_t *w, const uint8_t *s, float *out,
                         cudaStream_t st);
int launch_dequant_ternary(size_t rows, size_t cols, const uint8_t *p, float *out,
                           cudaStream_t st);

}  // namespace ffn
