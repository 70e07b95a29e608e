/*
 * ffn_b200.h -- B200 extension ABI of libffn_b200.so.
 *
 * The reference's plugin ABI (merkaba_hw_addon.h) passes host pointers and
 * synchronises on every call.  These entry points are the device-resident
 * fast path the same kernels run on: all tensor pointers are CUDA device
 * pointers on the current device, work is enqueued on `stream` (a
 * cudaStream_t, NULL = legacy default stream) and nothing synchronises.  A
 * Rust host that does not know these symbols keeps working through the
 * reference ABI.
 *
 * Every function returns 0 on success or a negative FFN_B200_E* code;
 * ffn_b200_last_error() returns the message of the last failure on the calling
 * thread.  No function here allocates device memory unless its comment says
 * so: scratch is the caller's `ws` buffer, sized by the matching *_ws_bytes.
 *
 * Weight layouts are the reference's on-disk layouts, byte for byte:
 *   NVFP4   w [rows, cols/2] E2M1 nibbles (low nibble = even column),
 *           s [rows, cols/16] E4M3 block scales, gs f32 per-tensor scale
 *           (flash1017.rs:2282-2391).
 *   ternary p [rows, cols/4] 2-bit codes (element 4j+i at bits 2i..2i+1 of
 *           byte j; 0->-1, 1->0, 2->+1, 3->0), rs [rows] f32 row scales;
 *           optional rank-16 Q8 core a [16, cols] i8 (= V^T), a_sc [16],
 *           b [rows, 16] i8 (= U), b_sc [16]  (flash1017.rs:2393-2672).
 * The FP4 path reads a derived copy of NVFP4 experts, its stage images
 * (ffn_b200_pack_nvfp4_expert), written from those layouts.
 */
#ifndef FFN_B200_H
#define FFN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifndef FFN_B200_EXPORT
#if defined(__GNUC__)
#define FFN_B200_EXPORT __attribute__((visibility("default")))
#else
#define FFN_B200_EXPORT
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FFN_B200_OK 0
#define FFN_B200_EINVAL (-1)   /* bad shape, pointer or alignment */
#define FFN_B200_ECUDA (-2)    /* CUDA runtime error */
#define FFN_B200_ENOSPC (-3)   /* workspace too small */
#define FFN_B200_ENCCL (-4)    /* NCCL error */
#define FFN_B200_EUNSUP (-5)   /* valid but unsupported configuration */

#define FFN_B200_FMT_NVFP4 0
#define FFN_B200_FMT_TERNARY 1
/* MXFP4 experts (the MTP routed experts, flash1017.rs:2674-2747) use the nv[]
 * descriptors: w E2M1 pairs [rows, cols/2], s E8M0 block scales [rows, cols/32]
 * (2^(s - 127), flash1017.rs:1049-1057), gs a power of two 2^B (1 for the
 * reference's tensors, which have no global scale).  The kernels decode each
 * block scale as 2^(s - 127 - B) in f16 and multiply the f32 sums by gs, so a
 * matrix is decoded exactly while every block obeys -23 <= s - 127 - B <= 13;
 * st_load_expert picks B from the largest block scale.  cols % 128 == 0. */
#define FFN_B200_FMT_MXFP4 2
/* MXFP8 matrices (the shared expert, CachedMxfp8Mat, flash1017.rs:1920-1984)
 * also use nv[]: w E4M3 [rows, cols], s E8M0 [ceil(rows/32), cols/32] (one
 * scale per 32 x 32 block), gs a power of two 2^B; decoded as E4M3 x
 * 2^(s - 127 - B) in f16, exact while -15 <= s - 127 - B <= 7 (the caller's B
 * from the largest scale: B = max(s) - 134).  cols % 128 == 0.  Dense experts
 * (expert_forward, gx10_rust_mxfp8_mlp_accum) and matvecs only: MoE tables
 * hold NVFP4, MXFP4 and ternary experts. */
#define FFN_B200_FMT_MXFP8 3

/* Router score functions.  REF: sqrt(softplus(l)) + bias, weights
 * score * 1.5 / sum (flash1017.rs:7280-7376).  SIGMOID: sigmoid(l) + bias,
 * weights score / sum (renormalised). */
#define FFN_B200_SCORE_REF_SQRTSOFTPLUS 0
#define FFN_B200_SCORE_SIGMOID 1

/* Router arithmetic.  EXACT sums each logit sequentially in column order
 * without FMA, the CPU loop's order, so logits are bit-identical to the
 * reference's; TENSOR uses split-f16 tensor-core products (about fp32
 * accurate, different summation order: selections can differ on near-ties). */
#define FFN_B200_ROUTER_EXACT 0
#define FFN_B200_ROUTER_TENSOR 1

typedef struct ffn_b200_nvfp4_mat {
    const uint8_t *w;  /* [rows, cols/2] */
    const uint8_t *s;  /* [rows, cols/16] */
    float gs;
    uint32_t reserved;
} ffn_b200_nvfp4_mat;

typedef struct ffn_b200_ternary_mat {
    const uint8_t *p;        /* [rows, cols/4] */
    const float *rs;         /* [rows] */
    const int8_t *core_a;    /* [16, cols] or NULL (no rank-16 core); 16-byte aligned */
    const float *core_a_sc;  /* [16] */
    const int8_t *core_b;    /* [rows, 16]; 16-byte aligned */
    const float *core_b_sc;  /* [16] */
    /* U8 block scales [rows, cols/64] (one per 64 columns, 4-byte aligned) or
     * NULL: row r = rs[r] * sum_b bs[r][b] * sum_{64 columns of b} L(code) x
     * (flash1017.rs:2567-2601, the `.block_scales` tensor the 106 GB
     * compressor writes, :10783-10787). */
    const uint8_t *bs;
} ffn_b200_ternary_mat;

/* One SwiGLU expert: matrix 0 = gate (w1), 1 = up (w3), 2 = down (w2). */
typedef struct ffn_b200_expert {
    int32_t format;     /* FFN_B200_FMT_* */
    float proj_scale;   /* ternary tier_b_proj_scale (flash1017.rs:7551-7561); 1 for NVFP4 */
    ffn_b200_nvfp4_mat nv[3];
    ffn_b200_ternary_mat tn[3];
    /* NVFP4 experts packed for the FP4 tensor-core path
     * (ffn_b200_pack_nvfp4_expert; DEVICE, 16-byte aligned), or NULL */
    const uint8_t *fp4_gu;  /* W1 and W3 stage images */
    const uint8_t *fp4_dn;  /* W2 stage images */
} ffn_b200_expert;

/* ---------------------------------------------------------------- library */
FFN_B200_EXPORT const char *ffn_b200_version(void);
FFN_B200_EXPORT const char *ffn_b200_last_error(void);
/* Number of kernels this library has launched in this process. */
FFN_B200_EXPORT uint64_t ffn_b200_launch_count(void);
/* Selects the device for later calls on this thread (cudaSetDevice). */
FFN_B200_EXPORT int ffn_b200_set_device(int device);

/* ------------------------------------------------------------ single matrices
 * out [seq, rows] = x [seq, cols] * W^T.  Same results as the reference's
 * CachedNvfp4Mat::matbatch / CachedTernary158Mat::matbatch (flash1017.rs:
 * 2361-2391, 2631-2668) within the parity tolerance.  ws: see *_ws_bytes.
 * cols must be a multiple of 64; NVFP4 w 16-byte and s 4-byte aligned,
 * ternary p 16-byte aligned. */
FFN_B200_EXPORT size_t ffn_b200_matvec_ws_bytes(size_t seq, size_t cols);
FFN_B200_EXPORT int ffn_b200_nvfp4_matvec(size_t rows, size_t cols, size_t seq,
                                          const ffn_b200_nvfp4_mat *m, const float *x,
                                          float *out, void *ws, size_t ws_bytes, void *stream);
/* MXFP4 rows (CachedMxfp4Mat::matvec, flash1017.rs:2700-2746): m->s holds the
 * E8M0 scales [rows, cols/32], m->gs a power of two (FFN_B200_FMT_MXFP4). */
FFN_B200_EXPORT int ffn_b200_mxfp4_matvec(size_t rows, size_t cols, size_t seq,
                                          const ffn_b200_nvfp4_mat *m, const float *x,
                                          float *out, void *ws, size_t ws_bytes, void *stream);
/* MXFP8 rows (CachedMxfp8Mat::matvec, flash1017.rs:1940-1984): m->w E4M3
 * [rows, cols], m->s E8M0 [ceil(rows/32), cols/32], m->gs a power of two
 * (FFN_B200_FMT_MXFP8). */
FFN_B200_EXPORT int ffn_b200_mxfp8_matvec(size_t rows, size_t cols, size_t seq,
                                          const ffn_b200_nvfp4_mat *m, const float *x,
                                          float *out, void *ws, size_t ws_bytes, void *stream);
/* Ternary rows, then y += B (diag(a_sc b_sc) A x) when m->core_a != NULL
 * (flash1017.rs:2538-2627, rank-16 core :2446-2472). */
FFN_B200_EXPORT int ffn_b200_ternary_matvec(size_t rows, size_t cols, size_t seq,
                                            const ffn_b200_ternary_mat *m, const float *x,
                                            float *out, void *ws, size_t ws_bytes,
                                            void *stream);

/* ------------------------------------------------------------- one expert
 * out[t] (=|+=) accum_weight * expert(x[t]) for t < seq, the fused expert of
 * gx10_rust_nvfp4_mlp_accum / gx10_rust_ternary_158_mlp_accum (HA:323-357)
 * plus the rank-16 cores the reference's fused path lacks (the reference
 * recomputes such experts on its CPU, flash1017.rs:7483-7486).  For ternary
 * experts the caller passes accum_weight = weight * proj_scale, as the
 * reference does.  `e` is a host struct holding device pointers.
 * NVFP4 and MXFP4 experts over 1..8 tokens and ternary experts over one token
 * (inter and hidden multiples of 512 whose 512-column chunks divide 16, up to
 * 8192; 16-byte aligned codes, scales, x, out and ws) run as two launches of
 * the decode kernels (a ternary expert with gate/up cores adds the cores'
 * z kernel first); their weights and scales are read before the wait on the
 * previous kernel in the stream, so they must not be written by a kernel the
 * caller queued just before that lets later work start early (programmatic
 * dependent launch).  FFN_B200_EXPERT_DECODE=0 in the environment (read once)
 * keeps every call on the GEMV kernels. */
FFN_B200_EXPORT size_t ffn_b200_expert_ws_bytes(size_t inter, size_t hidden, size_t seq);
FFN_B200_EXPORT int ffn_b200_expert_forward(size_t inter, size_t hidden, size_t seq,
                                            const ffn_b200_expert *e, const float *x,
                                            float *out, float accum_weight, int accumulate,
                                            void *ws, size_t ws_bytes, void *stream);

/* The same expert forward for callers that cannot allocate device memory or
 * hand over scratch: a plugin host that owns the memory budget, code running
 * during CUDA stream capture, decode loops that must not allocate.  This entry
 * point has no counterpart in the reference.  It uses a fixed 1 MiB scratch
 * array that the library keeps on every GPU that loads it until the process
 * exits, and calls no allocator.  Shapes that need more scratch than 1 MiB
 * (ffn_b200_expert_ws_bytes) are rejected with FFN_B200_EINVAL.  Before any
 * stream capture, make one call per device and per weight format the captured
 * code will use (NVFP4, MXFP4, ternary, MXFP8): the first call on a device looks
 * up the array's device address, and the first call of a format sets its
 * kernels' shared-memory attribute; neither may run under capture.  The
 * address is cached per device index for the process, so it assumes one CUDA
 * context per device (no cudaDeviceReset between calls).  All calls share the
 * one array: calls whose work overlaps on the GPU (different streams, or
 * different host threads) race on it and must be serialised by the caller. */
FFN_B200_EXPORT int ffn_b200_expert_forward_noalloc(size_t inter, size_t hidden, size_t seq,
                                                    const ffn_b200_expert *e, const float *x,
                                                    float *out, float accum_weight,
                                                    int accumulate, void *stream);

/* -------------------------------------------------------------- MoE layer
 * Routed SwiGLU MoE layer (flash1017.rs:7259-7567 decode, 7972-8326 batched):
 * router logits -> scores -> top_k -> per-expert token groups -> fused expert
 * GEMV/GEMM -> weighted combine in selection order.  Only experts in
 * [expert_begin, expert_end) are computed (expert parallelism); the others'
 * contributions are left out of `out`, so summing `out` over the ranks that
 * own disjoint ranges gives the full layer. */
typedef struct ffn_b200_moe_desc {
    size_t hidden, inter, n_experts, top_k;
    const ffn_b200_expert *experts;  /* DEVICE array [n_experts] */
    const float *router_w;           /* DEVICE [n_experts, hidden] f32 */
    const float *router_bias;        /* DEVICE [n_experts] or NULL */
    int32_t score_fn;                /* FFN_B200_SCORE_* */
    int32_t router_mode;             /* FFN_B200_ROUTER_* */
    int32_t expert_begin, expert_end;
    int32_t has_nvfp4, has_ternary;  /* which formats occur in experts[] (has_nvfp4: NVFP4 or MXFP4) */
    /* Optional RMSNorm of the layer input before routing and the experts, the
     * reference's ffn_norm (flash1017.rs:7637, 4880-4891): xn = x / sqrt(mean(x^2)
     * + norm_eps) * norm_w.  NULL: the experts see x itself. */
    const float *norm_w;             /* DEVICE [hidden] or NULL */
    float norm_eps;
    /* FFN_B200_PATH_*: AUTO (0), for a layer with only NVFP4 experts and
     * hidden, inter multiples of 256: the tensor-core grouped GEMM when the
     * routed pairs average >= FFN_B200_GROUPED_MIN_PAIRS per expert (prefill),
     * else the block-scaled FP4 path (decode; hidden, inter <= 16384); any
     * other layer takes the GEMV slices. */
    int32_t path;
    /* MXFP4 experts occur in experts[] (they count as has_nvfp4 too: same
     * kernel family; the grouped GEMM is NVFP4-only). */
    int32_t has_mxfp4;
    /* every expert in [expert_begin, expert_end) carries fp4_gu and fp4_dn
     * (the FP4 path needs them) */
    int32_t fp4_packed;
} ffn_b200_moe_desc;

#define FFN_B200_PATH_AUTO 0
#define FFN_B200_PATH_GEMV 1    /* slices of <= 8 tokens, f16 hi/lo activations (~fp32) */
#define FFN_B200_PATH_GROUPED 2 /* tcgen05 grouped GEMM, f16 activations (rel. err ~2e-4) */
/* tcgen05 kind::mxf4nvf4: the NVFP4 weights and their E4M3 block scales enter
 * the tensor core unchanged, from the stage images ffn_b200_pack_nvfp4_expert
 * writes (fp4_packed; scale bytes must be UE4M3: sign bit clear, not 0x7F),
 * activations as six NVFP4 residual terms (rel. err ~1e-5 per layer); chunks
 * of <= 8 tokens per expert.  AUTO takes it for NVFP4-only packed layers
 * below FFN_B200_GROUPED_MIN_PAIRS pairs per expert. */
#define FFN_B200_PATH_FP4 3
#define FFN_B200_GROUPED_MIN_PAIRS 48

/* The FP4 path's activation format (no reference counterpart: the reference
 * multiplies f32 activations).  Each row x of K values (K % 256 == 0, K <=
 * 16384; rows 16-byte aligned, ld_x % 4 == 0) becomes NVFP4 terms (four here),
 * x ~= sum_t 2^exps[t] * q_t: codes [rows][4][K/2] (E2M1 pairs, low nibble =
 * even column), scales [rows][4][K/16] (UE4M3 per 16 values), exps [rows][4].
 * Term t quantises what terms < t left: E_t = floor(log2 max|r_t|) - 8, block
 * scale = UE4M3 ceiling of max|r_t| 2^-E_t / 6, codes = E2M1 round-to-nearest-
 * even of r_t 2^-E_t / scale. */
FFN_B200_EXPORT int ffn_b200_quantize_nvfp4x4(size_t rows, size_t K, const float *x, size_t ld_x,
                                              uint8_t *codes, uint8_t *scales, int32_t *exps,
                                              void *stream);
/* The same with `terms` (1..8) terms: codes [rows][terms][K/2], scales
 * [rows][terms][K/16], exps [rows][terms].  The FP4 path uses six. */
FFN_B200_EXPORT int ffn_b200_quantize_nvfp4_terms(size_t rows, size_t K, size_t terms, const float *x,
                                                  size_t ld_x, uint8_t *codes, uint8_t *scales,
                                                  int32_t *exps, void *stream);

/* The FP4 path's weight format (no reference counterpart; the reference keeps
 * the row-major NVFP4 layout, which stays the input here).  A pipeline stage
 * of the FP4 kernels covers two 128-row blocks x 256 K values -- the W1 and W3
 * rows of an output block (gate/up), or the two halves of a 256-row W2 block
 * (down) -- and its image holds, in order: each block's codes as a K-major
 * 128-byte-swizzled tile (16 B piece c of row r at r/8*1024 + r%8*128 +
 * (c ^ r%8)*16; 16 KB per block), then each block's scale atoms (4 K-steps x
 * 512 B; line l = the 4 E4M3 scale bytes of rows l, l+32, l+64, l+96).  Images
 * follow in (row block, K step) order, 36,864 bytes each: gate/up
 * inter/128 x hidden/256 images, down hidden/256 x inter/256 -- the same bytes
 * as the reference layout.  which: 0 gate/up, 1 down; 0 when inter or hidden
 * is not a multiple of 256. */
FFN_B200_EXPORT size_t ffn_b200_fp4_pack_bytes(size_t inter, size_t hidden, int which);
/* Writes e's images (e: host struct, DEVICE pointers; w 16-byte, s 4-byte
 * aligned) into gu and/or dn (DEVICE, 16-byte aligned; either may be NULL).
 * Synchronises the stream.  FFN_B200_EINVAL when a scale byte is not UE4M3. */
FFN_B200_EXPORT int ffn_b200_pack_nvfp4_expert(size_t inter, size_t hidden, const ffn_b200_expert *e,
                                               uint8_t *gu, uint8_t *dn, void *stream);

/* The layer's top-k step on precomputed logits (flash1017.rs:7280-7376): per
 * token, logit = sum of the n_part (1..3) partial planes in plane order
 * (logits [n_part][n_tok][n_exp], DEVICE), score = score_fn(logit), biased =
 * score + bias (bias DEVICE [n_exp] or NULL); the top_k by biased score
 * (desc, lower expert index first on ties; NaN never selected; a round with no
 * candidate yields index 0x7fffffff, weight 0) in selection order, weights =
 * score * (1.5 for REF_SQRTSOFTPLUS, 1 for SIGMOID) / (sum of the selected
 * scores in selection order), 0 when that sum <= 1e-12.  idx, wt DEVICE
 * [n_tok][top_k]; top_k <= 16. */
FFN_B200_EXPORT int ffn_b200_topk(size_t n_tok, size_t n_exp, size_t top_k, int32_t score_fn,
                                  const float *logits, size_t n_part, const float *bias,
                                  int32_t *idx, float *wt, void *stream);

FFN_B200_EXPORT size_t ffn_b200_moe_ws_bytes(const ffn_b200_moe_desc *d, size_t max_tokens);
/* x [n_tok, hidden] f32; out [n_tok, hidden] = residual + moe(xn) when
 * residual != NULL, else moe(xn), with xn = x or its RMSNorm (norm_w); residual
 * may alias x or out.  topk_idx /
 * topk_w [n_tok, top_k] receive the routing when non-NULL. */
FFN_B200_EXPORT int ffn_b200_moe_layer(const ffn_b200_moe_desc *d, size_t n_tok,
                                       const float *x, const float *residual, float *out,
                                       int32_t *topk_idx, float *topk_w, void *ws,
                                       size_t ws_bytes, void *stream);

/* ----------------------------------------------- seeded synthetic weights
 * Counter-based generators (SplitMix64 finaliser + Irwin-Hall normals +
 * round-to-nearest-even E4M3), byte-identical to the CPU oracle's.  NVFP4 w
 * must be 8-byte aligned. */
FFN_B200_EXPORT uint64_t ffn_b200_key(uint64_t parent, uint64_t v);
FFN_B200_EXPORT int ffn_b200_gen_nvfp4(uint64_t key, size_t rows, size_t cols, uint8_t *w,
                                       uint8_t *s, void *stream);
FFN_B200_EXPORT int ffn_b200_gen_ternary(uint64_t key, size_t rows, size_t cols, uint8_t *p,
                                         float *rs, void *stream);
FFN_B200_EXPORT int ffn_b200_gen_core(uint64_t key, size_t rows, size_t cols, int8_t *a,
                                      float *a_sc, int8_t *b, float *b_sc, void *stream);
FFN_B200_EXPORT int ffn_b200_gen_normal(uint64_t key, size_t n, float stdev, float *out,
                                        void *stream);

/* --------------------------------------------------------- decode checks
 * The kernels' own weight decoders written out as f32: NVFP4 e2m1 * e4m3
 * (without the per-tensor scale) and ternary codes {-1,0,+1}. */
FFN_B200_EXPORT int ffn_b200_dequant_nvfp4(size_t rows, size_t cols, const uint8_t *w,
                                           const uint8_t *s, float *out, void *stream);
FFN_B200_EXPORT int ffn_b200_dequant_ternary(size_t rows, size_t cols, const uint8_t *p,
                                             float *out, void *stream);

/* ------------------------------------------------------ kernel timing
 * Measurement hooks.  While enabled, the library records a CUDA event pair
 * around every kernel it launches, on the stream the kernel is launched on,
 * and ffn_b200_profile_read() sums the device time per kernel kind (it
 * synchronises the recorded events).  Enabling creates the events; no work is
 * skipped or reordered.  Off by default. */
#define FFN_B200_K_XPREP 0
#define FFN_B200_K_ROUTER 1
#define FFN_B200_K_TOPK 2
#define FFN_B200_K_GROUP 3
#define FFN_B200_K_GATEUP_NVFP4 4
#define FFN_B200_K_DOWN_NVFP4 5
#define FFN_B200_K_GATEUP_TERNARY 6
#define FFN_B200_K_DOWN_TERNARY 7
#define FFN_B200_K_COREZ 8
#define FFN_B200_K_COMBINE 9
#define FFN_B200_K_MATVEC 10
#define FFN_B200_K_OTHER 11
#define FFN_B200_K_GEMM_GATEUP 12 /* grouped tensor-core path */
#define FFN_B200_K_GEMM_DOWN 13
#define FFN_B200_K_QUANT 14       /* activation rows -> six NVFP4 terms (FP4 path) */
#define FFN_B200_K_FP4_GATEUP 15  /* block-scaled FP4 tensor-core path */
#define FFN_B200_K_FP4_DOWN 16
#define FFN_B200_K_COUNT 17
FFN_B200_EXPORT int ffn_b200_profile_enable(int enable);
/* Which kinds get event pairs while enabled: bit k = FFN_B200_K_* k (default
 * all).  Timing fewer kinds puts fewer event records between the kernels. */
FFN_B200_EXPORT int ffn_b200_profile_kinds(uint32_t mask);
FFN_B200_EXPORT int ffn_b200_profile_read(int kind, double *total_ms, uint64_t *launches);

/* ----------------------------------------- expert-parallel exchange (NVLink)
 * No reference counterpart (the reference runs on one GB10).  One process per
 * GPU; rank r's MoE layer (expert range r) writes its partial output into
 * ffn_b200_ep_part(ep) with residual = NULL, then ffn_b200_ep_allreduce writes
 * out = residual + sum over ranks of the parts on every rank (or
 * ffn_b200_ep_moe_layer does both in one go).  One cooperative kernel per GPU:
 * each rank pushes its partial rows to the rank that owns their slice of tokens,
 * the owner sums the slice in rank order and pushes the result rows to every
 * rank, all by plain stores to peer memory with arrival counters (bounded
 * waits on local memory; on a timed-out wait it writes NaN over out and sets the
 * flag ffn_b200_ep_error reads).  Set-up: every rank calls ffn_b200_ep_create
 * (allocates its shared buffers and writes its IPC handle,
 * ffn_b200_ep_handle_bytes() bytes), the handles are exchanged out of band
 * (e.g. torch.distributed all_gather), then ffn_b200_ep_connect(ep, handles of
 * all ranks in rank order).  Every rank must make the same exchange calls in
 * the same order. */
typedef struct ffn_b200_ep ffn_b200_ep;
FFN_B200_EXPORT size_t ffn_b200_ep_handle_bytes(void);
FFN_B200_EXPORT int ffn_b200_ep_create(int rank, int world, size_t max_tokens, size_t hidden,
                                       void *my_handle, ffn_b200_ep **out);
FFN_B200_EXPORT int ffn_b200_ep_connect(ffn_b200_ep *ep, const void *all_handles);
FFN_B200_EXPORT float *ffn_b200_ep_part(ffn_b200_ep *ep);
FFN_B200_EXPORT int ffn_b200_ep_allreduce(ffn_b200_ep *ep, size_t n_tok, const float *residual,
                                          float *out, void *stream);
/* The MoE layer of this rank's experts (d->expert_begin .. d->expert_end) with
 * the exchange fused in: routing for all tokens, this rank's experts, then one
 * exchange kernel that combines this rank's routes per token and pushes them
 * through the exchange, so out = residual + the layer over every rank's
 * experts on every rank (no reference counterpart: the reference runs on one
 * GB10).  It counts as one ffn_b200_ep_allreduce call for the every-rank-the-
 * same-calls rule. */
FFN_B200_EXPORT int ffn_b200_ep_moe_layer(ffn_b200_ep *ep, const ffn_b200_moe_desc *d, size_t n_tok,
                                          const float *x, const float *residual, float *out,
                                          int32_t *topk_idx, float *topk_w, void *ws, size_t ws_bytes,
                                          void *stream);
FFN_B200_EXPORT int ffn_b200_ep_error(ffn_b200_ep *ep, int *flag);
FFN_B200_EXPORT int ffn_b200_ep_destroy(ffn_b200_ep *ep);

/* ------------------------------------------------ safetensors expert loader
 * Replaces the reference's shard mapping and tensor lookup
 * (Flash1017ShardInspector::open / get_tensor_data, flash1017.rs:108-235)
 * and its per-expert matrix constructors (CachedNvfp4Mat::from_shard
 * :2295-2309, CachedTernary158Mat::from_shard :2495-2525,
 * CachedRank16Q8Core::from_shard :2415-2440) for the routed experts of a
 * layer (names as flash1017.rs:5219-5262 builds them, e.g. prefix
 * "layers.3.ffn.experts.17"; matrices <prefix>.w1 gate, .w3 up, .w2 down).
 * The shard is mapped read-only; st_load_expert copies one expert's tensors
 * into a caller-owned device buffer (st_expert_bytes of it, 256-byte aligned)
 * on `stream` and fills *e with device pointers into it.  NVFP4 when
 * <prefix>.w1.weight and .weight_scale exist (weight u8 [rows, cols/2],
 * weight_scale [rows, cols/16], weight_scale_2 f32 scalar -> gs); MXFP4 when
 * .weight and .scale exist (CachedMxfp4Mat::from_shard :2688-2699; scale E8M0
 * [rows, cols/32]; gs = 2^(largest scale byte - 140)); MXFP8 when .weight
 * has one byte per weight (the shared experts, CachedMxfp8Mat :1928-1939;
 * scale [ceil(rows/32), cols/32]; gs = 2^(largest - 134)); else ternary
 * (packed_ternary [rows, cols/4], row_scales f32 [rows], optional
 * block_scales u8 [rows, cols/64], optional rank-16 core).  Shapes are checked
 * against inter x hidden; proj_scale is set to 1. */
typedef struct ffn_b200_st ffn_b200_st;
FFN_B200_EXPORT int ffn_b200_st_open(const char *path, ffn_b200_st **out);
FFN_B200_EXPORT int ffn_b200_st_close(ffn_b200_st *st);
FFN_B200_EXPORT size_t ffn_b200_st_count(const ffn_b200_st *st);
FFN_B200_EXPORT const char *ffn_b200_st_name(const ffn_b200_st *st, size_t i);
/* dtype string ("U8", "F32", "F8_E4M3", ...), shape (up to 8 dims), bytes in the
 * mapping; FFN_B200_EINVAL when the tensor is absent. */
FFN_B200_EXPORT int ffn_b200_st_find(const ffn_b200_st *st, const char *name, const char **dtype,
                                     int64_t *shape, int *ndim, const void **data, size_t *nbytes);
FFN_B200_EXPORT int ffn_b200_st_expert_bytes(const ffn_b200_st *st, const char *prefix, size_t hidden,
                                             size_t inter, int *format, size_t *bytes);
FFN_B200_EXPORT int ffn_b200_st_load_expert(const ffn_b200_st *st, const char *prefix, size_t hidden,
                                            size_t inter, void *dev, size_t dev_bytes, void *stream,
                                            ffn_b200_expert *e);

/* ------------------------------------------- 106 GB format compressor
 * compress_nvfp4_matrix_to_158_jepa_q8 (flash1017.rs:10377-10645, with
 * orthonormalize_cols_16 :10342-10372), which the reference runs on the CPU
 * when it writes the 106 GB shards (:10700-10811).  One NVFP4 matrix (w [rows,
 * cols/2] E2M1 pairs, s [rows, cols/16] E4M3, per-tensor scale gs; cols % 64
 * == 0) becomes ternary codes packed [rows, cols/4] (16-byte aligned), row
 * scales [rows], U8 block-64 scales [rows, cols/64], and the rank-16 Q8 core
 * core_b [rows, 16] / core_b_sc [16] / core_a [16, cols] / core_a_sc [16] of
 * the residual (seed: the reference's subspace-iteration seed).  The outputs
 * are exactly the tensors ffn_b200_ternary_mat reads.  Device pointers, caller
 * workspace, enqueued on `stream`.  The reference function also returns the
 * squared Frobenius norms of the matrix, of its ternary error and of the error
 * left after the core (its shard writer reports their ratio,
 * flash1017.rs:10747-10768); this entry point does not: a caller that wants
 * them decodes both forms (ffn_b200_dequant_nvfp4, ffn_b200_ternary_matvec on
 * unit vectors or the dequantised ternary) and sums the squares itself. */
FFN_B200_EXPORT size_t ffn_b200_compress_ws_bytes(size_t rows, size_t cols);
FFN_B200_EXPORT int ffn_b200_compress_ternary_b64(size_t rows, size_t cols, const uint8_t *w,
                                                  const uint8_t *s, float gs, uint64_t seed,
                                                  uint8_t *packed, float *row_scales,
                                                  uint8_t *block_scales, int8_t *core_b,
                                                  float *core_b_sc, int8_t *core_a, float *core_a_sc,
                                                  void *ws, size_t ws_bytes, void *stream);

/* -------------------------------------------- reference-ABI support hooks
 * Host-side x_all buffer for gx10_rust_*_mlp_batch, for hosts that do not make
 * the shared-expert call (gx10_rust_mxfp8_mlp_batch hands x_all over itself,
 * as the reference does, flash1017.rs:8170-8186).  The rows are read when the
 * first *_mlp_batch call needs them. */
FFN_B200_EXPORT int ffn_b200_set_batch_input(const float *x_all_host, size_t x_total_tokens,
                                             size_t hidden);
/* Drops every HBM weight copy made for host pointers. */
FFN_B200_EXPORT int ffn_b200_release_host_ranges(void);
/* Bytes of HBM currently held for host-pointer weight copies. */
FFN_B200_EXPORT size_t ffn_b200_host_cache_bytes(void);
/* HBM budget of those copies (no reference counterpart: GB10 memory is unified).
 * 0 (the default): as much as the GPU gives.  Past the budget, or when an
 * allocation fails, the least recently used copies are freed (first-use copies
 * before registered ranges, never one the current call uses) and copied again
 * when a later call needs them. */
FFN_B200_EXPORT int ffn_b200_set_host_cache_budget(size_t bytes);

#ifdef __cplusplus
}
#endif
#endif /* FFN_B200_H */
