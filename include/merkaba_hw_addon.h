/*
 * merkaba_hw_addon.h -- the reference's dot-kernel plugin ABI, as exported by
 * libffn_b200.so (the B200 backend for the quantized expert-FFN path).
 *
 * This is the C side of `#[repr(C)] HardwareAddonVTable` and the optional
 * `gx10_rust_*` symbols that the Rust host of terox27/Flash1017-Engine resolves
 * with dlopen/dlsym (crates/flash-core/src/hardware_addon.rs, "HA" below).
 * Field order, types and calling conventions follow HA exactly; the
 * static_asserts pin the LP64 layout the Rust side sees.
 *
 * Pointer contract (HA:79-120, 323-479; call sites in flash1017.rs): every
 * pointer is caller-owned HOST memory (mmap'd safetensors or Rust Vecs).  The
 * backend keeps an HBM copy of each weight range it has seen (registered via
 * gx10_rust_register_host_range, or copied on first use; weights are immutable
 * for the process lifetime in the reference) and stages x/out through device
 * buffers.  When a V1-V3 function returns, `out` holds the final values.  For
 * the *_mlp_* functions, `out` is final once a call with sync_now=true returns.
 *
 * Errors: V1-V3 functions return void (HA:143-174) and so cannot fail
 * visibly; on a bad argument or CUDA error they fill `out` with NaN and record
 * the message (ffn_b200_last_error() in ffn_b200.h).  The gx10_rust_*
 * functions return false, which makes the Rust host recompute on its CPU path
 * (flash1017.rs:7474-7519).
 */
#ifndef MERKABA_HW_ADDON_H
#define MERKABA_HW_ADDON_H

#include <stdbool.h>
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

/* HA:17-19 */
#define MERKABA_HW_ABI_V1 0x4D485701u
#define MERKABA_HW_ABI_V2 0x4D485702u
#define MERKABA_HW_ABI_V3 0x4D485703u

/* HA:21-28 */
typedef void (*merkaba_matvec_q4_g32_fn)(size_t rows, size_t cols, const uint8_t *packed_nibbles,
                                         const uint16_t *group_scales_bf16, const float *x,
                                         float *out);
/* HA:30-37 */
typedef void (*merkaba_matvec_q8_fn)(size_t rows, size_t cols, const int8_t *weights_i8,
                                     const float *row_scales, const float *x, float *out);
/* HA:39-45 */
typedef void (*merkaba_matvec_bf16_fn)(size_t rows, size_t cols, const uint16_t *weights_bf16,
                                       const float *x, float *out);
/* HA:47-55 */
typedef void (*merkaba_matbatch_q4_g32_fn)(size_t rows, size_t cols, size_t seq_len,
                                           const uint8_t *packed_nibbles,
                                           const uint16_t *group_scales_bf16,
                                           const float *x_batch, float *out_batch);
/* HA:57-65 */
typedef void (*merkaba_matbatch_q8_fn)(size_t rows, size_t cols, size_t seq_len,
                                       const int8_t *weights_i8, const float *row_scales,
                                       const float *x_batch, float *out_batch);
/* HA:67-75 */
typedef void (*merkaba_matbatch_bf16_fn)(size_t rows, size_t cols, size_t seq_len,
                                         const uint16_t *weights_bf16, const float *x_batch,
                                         float *out_batch);
/* HA:77-87  NVFP4: packed_fp4 [rows, cols/2] (low nibble = even column),
 * group_scales_fp8 [rows, cols/16] E4M3, per-tensor global_scale; cols unpacked. */
typedef void (*merkaba_matvec_nvfp4_fn)(size_t rows, size_t cols, const uint8_t *packed_fp4,
                                        const uint8_t *group_scales_fp8, float global_scale,
                                        const float *x, float *out);
/* HA:89-99  out_batch [seq_len, rows] = x_batch [seq_len, cols] * W^T */
typedef void (*merkaba_matbatch_nvfp4_fn)(size_t rows, size_t cols, size_t seq_len,
                                          const uint8_t *packed_fp4,
                                          const uint8_t *group_scales_fp8, float global_scale,
                                          const float *x_batch, float *out_batch);
/* HA:101-109  ternary: packed [rows, cols/4], code (b>>2i)&3: 0->-1, 1->0, 2->+1, 3->0 */
typedef void (*merkaba_matvec_ternary_158_fn)(size_t rows, size_t cols,
                                              const uint8_t *packed_ternary,
                                              const float *row_scales, const float *x,
                                              float *out);
/* HA:111-120 */
typedef void (*merkaba_matbatch_ternary_158_fn)(size_t rows, size_t cols, size_t seq_len,
                                                const uint8_t *packed_ternary,
                                                const float *row_scales, const float *x_batch,
                                                float *out_batch);
/* HA:122-130 */
typedef void (*merkaba_matvec_mxfp8_fn)(size_t rows, size_t cols, const uint8_t *weights_fp8,
                                        const uint8_t *block_scales_e8m0, const float *x,
                                        float *out);
/* HA:132-141 */
typedef void (*merkaba_matbatch_mxfp8_fn)(size_t rows, size_t cols, size_t seq_len,
                                          const uint8_t *weights_fp8,
                                          const uint8_t *block_scales_e8m0,
                                          const float *x_batch, float *out_batch);

/* HA:143-174  #[repr(C)] HardwareAddonVTable.  The V1 dot functions are
 * mandatory (non-Option) fields; the rest are Option<extern fn> (NULL = None). */
typedef struct HardwareAddonVTable {
    uint32_t abi_version;
    const uint8_t *addon_id_ptr;
    size_t addon_id_len;
    const uint8_t *addon_desc_ptr;
    size_t addon_desc_len;
    float (*dot_f32)(const float *a, const float *b, size_t len);
    float (*dot_i8_f32)(const int8_t *w_row, const float *x, size_t len);
    float (*dot_q4_g32_f32)(const uint8_t *row_nibbles, const uint16_t *row_scales_bf16,
                            const float *x, size_t cols);
    float (*dot_ternary_2bit_f32)(const uint8_t *row_packed, const float *x, size_t cols);
    /* ABI V2 */
    merkaba_matvec_q4_g32_fn matvec_q4_g32;
    merkaba_matvec_q8_fn matvec_q8;
    merkaba_matvec_bf16_fn matvec_bf16;
    merkaba_matbatch_q4_g32_fn matbatch_q4_g32;
    merkaba_matbatch_q8_fn matbatch_q8;
    /* ABI V3 */
    merkaba_matbatch_bf16_fn matbatch_bf16;
    merkaba_matvec_nvfp4_fn matvec_nvfp4;
    merkaba_matbatch_nvfp4_fn matbatch_nvfp4;
    merkaba_matvec_ternary_158_fn matvec_ternary_158;
    merkaba_matbatch_ternary_158_fn matbatch_ternary_158;
    merkaba_matvec_mxfp8_fn matvec_mxfp8;
    merkaba_matbatch_mxfp8_fn matbatch_mxfp8;
} HardwareAddonVTable;

#if defined(__cplusplus)
static_assert(sizeof(void *) == 8, "LP64 only");
static_assert(offsetof(HardwareAddonVTable, addon_id_ptr) == 8, "layout");
static_assert(offsetof(HardwareAddonVTable, dot_f32) == 40, "layout");
static_assert(offsetof(HardwareAddonVTable, matvec_q4_g32) == 72, "layout");
static_assert(offsetof(HardwareAddonVTable, matbatch_bf16) == 112, "layout");
static_assert(offsetof(HardwareAddonVTable, matbatch_mxfp8) == 160, "layout");
static_assert(sizeof(HardwareAddonVTable) == 168, "layout");
#endif

/* HA:839-849  entry point resolved by the loader; returns a vtable that stays
 * valid for the life of the process (it is kept in a static AtomicPtr, HA:910). */
FFN_B200_EXPORT const HardwareAddonVTable *merkaba_hardware_addon_v1(void);

/* HA:323-340 (call sites flash1017.rs:7407-7472, CPU twin :7537-7547):
 * out (=|+=) accum_weight * W2 (min(silu(W1 x), 10) * clamp(W3 x, -10, 10)).
 * w1/w3: [inter_rows, hidden_cols] NVFP4, w2: [hidden_cols, inter_rows] NVFP4.
 * accumulate=false overwrites out; sync_now=true makes out final on return. */
FFN_B200_EXPORT bool gx10_rust_nvfp4_mlp_accum(size_t inter_rows, size_t hidden_cols,
                                               const uint8_t *w1_fp4, const uint8_t *w1_s,
                                               float w1_sc2, const uint8_t *w3_fp4,
                                               const uint8_t *w3_s, float w3_sc2,
                                               const uint8_t *w2_fp4, const uint8_t *w2_s,
                                               float w2_sc2, const float *x, float *out,
                                               float accum_weight, bool accumulate,
                                               bool sync_now);

/* HA:307-320 (call sites flash1017.rs:7401-7405 and 9075-9091, CPU twin
 * :9132-9142): the shared expert, MXFP8 (E4M3 [rows, cols], E8M0 scales per
 * 32 x 32 block), same SwiGLU and accumulate / sync_now semantics as
 * gx10_rust_nvfp4_mlp_accum.  With it, nvfp4 and ternary present, the
 * reference takes its fused GPU MoE path (flash1017.rs:7401-7405). */
FFN_B200_EXPORT bool gx10_rust_mxfp8_mlp_accum(size_t inter_rows, size_t hidden_cols,
                                               const uint8_t *w1_w, const uint8_t *w1_s,
                                               const uint8_t *w3_w, const uint8_t *w3_s,
                                               const uint8_t *w2_w, const uint8_t *w2_s,
                                               const float *x, float *out, float accum_weight,
                                               bool accumulate, bool sync_now);

/* HA:359-373 (call site flash1017.rs:9103-9123, CPU twin :9145-9158): the MTP
 * layer's MXFP4 routed experts (E2M1 [rows, cols/2], E8M0 scales per 32
 * columns, no global scale), same SwiGLU and accumulate / sync_now semantics
 * as gx10_rust_nvfp4_mlp_accum. */
FFN_B200_EXPORT bool gx10_rust_mxfp4_mlp_accum(size_t inter_rows, size_t hidden_cols,
                                               const uint8_t *w1_fp4, const uint8_t *w1_s,
                                               const uint8_t *w3_fp4, const uint8_t *w3_s,
                                               const uint8_t *w2_fp4, const uint8_t *w2_s,
                                               const float *x, float *out, float accum_weight,
                                               bool accumulate, bool sync_now);
/* HA:298-305 (call sites flash1017.rs:940-956, 2704-2716): out [rows] =
 * MXFP4 W x, synchronous; false on error (the host then runs its CPU loop). */
FFN_B200_EXPORT bool gx10_rust_mxfp4_matvec(size_t rows, size_t cols, const uint8_t *packed_fp4,
                                            const uint8_t *scales_e8m0, const float *x, float *out);

/* HA:342-357 (call site flash1017.rs:7488-7504, CPU twin :7551-7561): gate/up
 * outputs are multiplied by proj_scale before the SwiGLU; the caller passes
 * accum_weight = weight * proj_scale. */
FFN_B200_EXPORT bool gx10_rust_ternary_158_mlp_accum(size_t inter_rows, size_t hidden_cols,
                                                     const uint8_t *w1_p, const float *w1_s,
                                                     const uint8_t *w3_p, const float *w3_s,
                                                     const uint8_t *w2_p, const float *w2_s,
                                                     float proj_scale, const float *x,
                                                     float *out, float accum_weight,
                                                     bool accumulate, bool sync_now);

/* HA:425-439 (call site flash1017.rs:8146-8186, CPU twin :8268-8277): the
 * batched layer's shared MXFP8 expert, out_batch[t] = expert(x_all[t]) for
 * t < seq_len (overwrite), and the hand-over of x_all [x_total_tokens,
 * hidden_cols], whose rows the layer's *_mlp_batch calls then read.  seq_len
 * with bit 31 set (the NVFP4 q4-backbone shared expert, flash1017.rs:8148-8158)
 * is not supported: false, and the host runs its CPU twin. */
FFN_B200_EXPORT bool gx10_rust_mxfp8_mlp_batch(size_t inter_rows, size_t hidden_cols,
                                               size_t seq_len, const uint8_t *w1_w,
                                               const uint8_t *w1_s, const uint8_t *w3_w,
                                               const uint8_t *w3_s, const uint8_t *w2_w,
                                               const uint8_t *w2_s, const float *x_all,
                                               size_t x_total_tokens, float *out_batch,
                                               bool sync_now);

/* HA:441-460 (call site flash1017.rs:8199-8223, CPU twin :8285-8303): one
 * expert over seq_len <= 8 tokens whose rows are x_all[x_tok_offset .. +seq_len]
 * of the batched layer's input; y_k is scatter-added as
 * out_batch[dst_tok_indices[k]] += dst_weights[k] * y_k.  out_batch is
 * [b_len, hidden_cols].  x_all comes from the layer's gx10_rust_mxfp8_mlp_batch
 * call (or ffn_b200_set_batch_input).  Calls are queued and run together as
 * one routed layer when the host needs out_batch (sync_now). */
FFN_B200_EXPORT bool gx10_rust_nvfp4_mlp_batch(size_t inter_rows, size_t hidden_cols,
                                               size_t seq_len, const uint8_t *w1_fp4,
                                               const uint8_t *w1_s, float w1_sc2,
                                               const uint8_t *w3_fp4, const uint8_t *w3_s,
                                               float w3_sc2, const uint8_t *w2_fp4,
                                               const uint8_t *w2_s, float w2_sc2,
                                               size_t x_tok_offset,
                                               const size_t *dst_tok_indices,
                                               const float *dst_weights, size_t b_len,
                                               float *out_batch, bool sync_now);

/* HA:462-479.  The weights added are dst_weights[k] * proj_scale, the
 * CPU twin's `weight * sc` (flash1017.rs:8317-8321). */
FFN_B200_EXPORT bool gx10_rust_ternary_158_mlp_batch(size_t inter_rows, size_t hidden_cols,
                                                     size_t seq_len, const uint8_t *w1_p,
                                                     const float *w1_s, const uint8_t *w3_p,
                                                     const float *w3_s, const uint8_t *w2_p,
                                                     const float *w2_s, float proj_scale,
                                                     size_t x_tok_offset,
                                                     const size_t *dst_tok_indices,
                                                     const float *dst_weights, size_t b_len,
                                                     float *out_batch, bool sync_now);

/* HA:494-495, 681-715: host-range registration hooks.  A range registered with
 * _register_host_range is copied into HBM once; later calls whose pointers fall
 * inside it read the HBM copy.  Shard bounds (many GB) are only recorded: the
 * tensors inside are copied the first time a call reads them. */
FFN_B200_EXPORT void gx10_rust_register_shard_bounds(const void *ptr, size_t bytes);
FFN_B200_EXPORT void gx10_rust_register_host_range(const void *ptr, size_t bytes);

#ifdef __cplusplus
}
#endif
#endif /* MERKABA_HW_ADDON_H */
