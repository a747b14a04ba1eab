// C ABI of libg4b200.so (declared in include/g4b200.h): contexts, argument validation and
// the op entry points. No computation happens here; every op launches the sm_100a kernels
// of g4_proj.cu / g4_attention.cu and there is no host or CPU fallback.
#include <cstring>
#include <mutex>

#include "g4_ctx.cuh"

using namespace g4::host;

namespace {

// Close the peers' mappings and free this rank's exchange buffer; back to a world of 1.
cudaError_t tp_release(g4_ctx* ctx) {
  cudaError_t first = cudaSuccess;
  for (void*& p : ctx->tp_peer) {
    if (p) {
      const cudaError_t e = cudaIpcCloseMemHandle(p);
      if (first == cudaSuccess) first = e;
      p = nullptr;
    }
  }
  if (ctx->tp_buf) {
    const cudaError_t e = cudaFree(ctx->tp_buf);
    if (first == cudaSuccess) first = e;
    ctx->tp_buf = nullptr;
  }
  ctx->tp_rank = 0;
  ctx->tp_world = 1;
  ctx->tp_ready = true;
  ctx->tp = g4::TpLink{0, 1, {}, nullptr, 0, ctx->tp_wait_ns};
  return first;
}

// The setup blob one rank hands to the others.
struct TpBlob {
  uint32_t magic, version;
  int32_t rank, world;
  unsigned char uuid[16];      // the rank's GPU
  cudaIpcMemHandle_t handle;   // its exchange buffer
  uint64_t bytes;              // the buffer's size
  uint32_t generation;         // the rank's count of setups (the group takes the largest)
};
static_assert(sizeof(TpBlob) <= G4_TP_BLOB_BYTES, "blob size");
constexpr uint32_t kTpMagic = 0x50543447u;  // "G4TP"
constexpr uint32_t kTpVersion = 2;
constexpr size_t kTpBufferBytes = g4::kTpExchangeWords * sizeof(unsigned long long) + 256;  // + epochs

}  // namespace

extern "C" {

const char* g4_status_string(g4_status s) {
  switch (s) {
    case G4_OK: return "ok";
    case G4_ERR_INVALID_ARGUMENT: return "invalid argument";
    case G4_ERR_MISALIGNED: return "misaligned pointer";
    case G4_ERR_CUDA: return "CUDA error";
    case G4_ERR_DEVICE: return "device-side error";
    case G4_ERR_UNSUPPORTED: return "unsupported size";
    default: return "unknown status";
  }
}

const char* g4_last_error(const g4_ctx* ctx) { return ctx ? ctx->last_error : "no context"; }

g4_status g4_ctx_create(int device, g4_ctx** out) {
  if (!out) return G4_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return G4_ERR_INVALID_ARGUMENT;
  g4_ctx* ctx = new g4_ctx();
  ctx->device = device;
  DeviceGuard guard(device);
  cudaError_t e = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  int major = 0, minor = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (e != cudaSuccess) {
    delete ctx;
    return G4_ERR_CUDA;
  }
  if (major != 10 || minor != 0 || !g4::proj_geometry_fits(ctx->sm_count)) {
    // the kernels are built for sm_100a only, and their launch geometry for its SM count
    delete ctx;
    return G4_ERR_UNSUPPORTED;
  }
  // scratch: error word + counters | split-K words | act | tile sums [| trace]
  const size_t off_counters = 256;
  const size_t off_partials = off_counters + g4::kCounterCount * sizeof(uint32_t);
  const size_t off_act = off_partials + g4::kPartialFloats * sizeof(float);
  const size_t off_ss = off_act + size_t(64) * g4::kL * sizeof(uint16_t);
  const size_t off_bh = off_ss + g4::kTileSsBytes;  // batched feed-forward: h | split-K words | unscale
  const size_t off_bw = off_bh + size_t(g4::kBatchMax) * g4::kH * sizeof(uint16_t);
  const size_t off_bu = off_bw + g4::batch_words_count(ctx->sm_count) * sizeof(unsigned long long);
  // term operands (1024-byte aligned: a TMA source) | their 2^-E
  const size_t off_bt = (off_bu + size_t(g4::kBatchMax) * sizeof(float) + 1023) / 1024 * 1024;
  const size_t off_be = off_bt + size_t(g4::kTermUnitsMax) * g4::kTermTokens * g4::kTerms * 256;
  const size_t off_trace = off_be + size_t(g4::kTermUnitsMax) * g4::kTermTokens * sizeof(float);
#ifdef G4_TRACE
  const size_t total = off_trace + size_t(65536 + 4096 * 32 * 8) * sizeof(uint64_t);
#else
  const size_t total = off_trace;
#endif
  e = cudaMalloc(&ctx->scratch, total);
  if (e == cudaSuccess) e = cudaMemset(ctx->scratch, 0, total);
  if (e == cudaSuccess) e = g4::prepare_proj_kernels();
  if (e == cudaSuccess) e = g4::prepare_attention_kernels();
  if (e == cudaSuccess) e = g4::prepare_batch_kernels();
  if (e == cudaSuccess) e = g4::prepare_batch_attn_kernels();
  if (e == cudaSuccess) e = g4::prepare_logits_batch_kernels();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (ctx->scratch) cudaFree(ctx->scratch);
    delete ctx;
    return G4_ERR_CUDA;
  }
  uint8_t* base = static_cast<uint8_t*>(ctx->scratch);
  ctx->scratch_bytes = total;
  ctx->sc.err = reinterpret_cast<uint32_t*>(base);
  ctx->sc.counters = reinterpret_cast<uint32_t*>(base + off_counters);
  ctx->sc.partials = reinterpret_cast<float*>(base + off_partials);
  ctx->sc.act = reinterpret_cast<uint16_t*>(base + off_act);
  ctx->act_bytes = off_ss - off_act;
  ctx->sc.tile_ss = reinterpret_cast<unsigned long long*>(base + off_ss);
  ctx->sc.batch_h = reinterpret_cast<uint16_t*>(base + off_bh);
  ctx->sc.batch_words = reinterpret_cast<unsigned long long*>(base + off_bw);
  ctx->sc.batch_unscale = reinterpret_cast<float*>(base + off_bu);
  ctx->sc.batch_terms = base + off_bt;
  ctx->sc.batch_texp = reinterpret_cast<float*>(base + off_be);
  ctx->batch_ok = g4::batch_geometry_fits(ctx->sm_count) && g4::batch_attn_geometry_fits(ctx->sm_count);
#ifdef G4_TRACE
  ctx->sc.trace = reinterpret_cast<uint64_t*>(base + off_trace);
#else
  ctx->sc.trace = nullptr;
#endif
  *out = ctx;
  return G4_OK;
}

g4_status g4_ctx_destroy(g4_ctx* ctx) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(ctx->device);
  cudaError_t e = tp_release(ctx);
  if (ctx->scratch) {
    const cudaError_t f = cudaFree(ctx->scratch);
    if (e == cudaSuccess) e = f;
  }
  delete ctx;
  return e == cudaSuccess ? G4_OK : G4_ERR_CUDA;
}

g4_status g4_ctx_set_overlap(g4_ctx* ctx, int enable) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  ctx->overlap = enable != 0;
  return G4_OK;
}

g4_status g4_ctx_check(g4_ctx* ctx, void* stream, uint32_t* flags) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(ctx->device);
  uint32_t word = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpy(&word, ctx->sc.err, sizeof word, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && word) e = cudaMemset(ctx->sc.err, 0, sizeof word);
  if (e == cudaSuccess && (word & (G4_DEVERR_WAIT_TIMEOUT | G4_DEVERR_PEER_TIMEOUT))) {
    // an abandoned launch can leave the epoch counters out of step: restart them, and clear the
    // epoch-tagged tile sums and split-K words so no old word matches a restarted epoch
    e = cudaMemset(ctx->sc.counters, 0, g4::kCounterCount * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(ctx->sc.tile_ss, 0, g4::kTileSsBytes);
    if (e == cudaSuccess) e = cudaMemset(ctx->sc.partials, 0, g4::kPartialFloats * sizeof(float));
  }
  // the ranks' exchange counters are out of step after a missed peer: refuse ops until the
  // caller sets the group up again
  if (word & G4_DEVERR_PEER_TIMEOUT) ctx->tp_ready = false;
  if (flags) *flags = word;
  if (e != cudaSuccess) return cuda_status(ctx, e, "g4_ctx_check");
  if (word) {
    snprintf(ctx->last_error, sizeof ctx->last_error, "device error bits 0x%x", word);
    return G4_ERR_DEVICE;
  }
  return G4_OK;
}

// m tokens (sequences) in one call: 1..64, and more than one only on a one-GPU context
static g4_status check_batch(g4_ctx* ctx, int32_t m) {
  if (m < 1 || m > g4::kBatchMax) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "m must be in [1, 64]");
  if (m > 1 && (ctx->tp_world != 1 || !ctx->batch_ok))
    return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "a batch of tokens runs on a one-GPU context only");
  return G4_OK;
}

static g4_status project_qkv(bool tiled, g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight, const uint8_t* k_weight,
                                 const uint8_t* v_weight, const uint16_t* q_weight_scale,
                                 const uint16_t* k_weight_scale, const uint16_t* v_weight_scale,
                                 const uint16_t* input_rms_weight, const uint16_t* q_rms_weight,
                                 const uint16_t* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                                 const uint16_t* cos, const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache,
                                 uint16_t* q_out, int32_t ring_len, int32_t rope_rows, void* stream, int32_t m = 1) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_batch(ctx, m);
  if (st != G4_OK) return st;
  st = check_ptrs(ctx, {{x, "x"},
                                  {q_weight, "q_weight"},
                                  {k_weight, "k_weight"},
                                  {v_weight, "v_weight"},
                                  {q_weight_scale, "q_weight_scale"},
                                  {k_weight_scale, "k_weight_scale"},
                                  {v_weight_scale, "v_weight_scale"},
                                  {input_rms_weight, "input_rms_weight"},
                                  {q_rms_weight, "q_rms_weight"},
                                  {k_rms_weight, "k_rms_weight"},
                                  {kv_offset, "kv_offset"},
                                  {rope_offset, "rope_offset"},
                                  {cos, "cos"},
                                  {sin, "sin"},
                                  {k_cache, "k_cache"},
                                  {v_cache, "v_cache"},
                                  {q_out, "q_out"}});
  if (st != G4_OK) return st;
  if (ring_len <= 0 || rope_rows <= 0)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be positive", ring_len <= 0 ? "ring_len" : "rope_rows");
  if (int64_t(rope_rows) * g4::kDs * 2 > INT32_MAX || int64_t(ring_len) * g4::kPs * 2 > INT32_MAX)
    return fail(ctx, G4_ERR_UNSUPPORTED, "%s: byte offsets would overflow i32", "ring_len/rope_rows");
  if ((st = check_tp(ctx)) != G4_OK) return st;
  DeviceGuard guard(ctx->device);
  g4::QkvArgs a{x,        q_weight,      k_weight,  v_weight, q_weight_scale, k_weight_scale, v_weight_scale,
                input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin,
                k_cache,  v_cache,       q_out,     ring_len, rope_rows, tiled};
  if (m > 1) return cuda_status(ctx, g4::launch_qkv_batch(a, m, env_of(ctx, stream)), "sliding_project_qkv_batch launch");
  return cuda_status(ctx, g4::launch_qkv(a, env_of(ctx, stream)), "sliding_project_qkv launch");
}

static g4_status sliding_attention(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                   const float* mask, uint16_t* out_hbm, int32_t ring_len, float scale,
                                   const int32_t* kv_offset, void* stream, int32_t m = 1) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_batch(ctx, m);
  if (st != G4_OK) return st;
  st = check_ptrs(ctx, {{q, "q"}, {k, "k"}, {v, "v"}, {mask, "mask"}, {out_hbm, "out_hbm"}});
  if (st != G4_OK) return st;
  if (ring_len <= 0 || ring_len % g4::attention_slot_multiple() != 0 || ring_len > g4::attention_max_ring())
    return fail(ctx, G4_ERR_UNSUPPORTED, "%s must be a positive multiple of 256, at most 8192", "ring_len");
  if (!(scale == scale)) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s is NaN", "scale");
  if ((st = check_tp(ctx)) != G4_OK) return st;
  DeviceGuard guard(ctx->device);
  g4::AttnArgs a{q, k, v, mask, out_hbm, ring_len, g4::kNs / ctx->tp_world, scale, kv_offset};
  a.batch = m;
  a.mask_stride = ring_len;
  return cuda_status(ctx, g4::launch_attention(a, env_of(ctx, stream)), "sliding_attention launch");
}

g4_status g4_sliding_attention(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                               const float* mask, uint16_t* out_hbm, int32_t ring_len, float scale, void* stream) {
  return sliding_attention(ctx, q, k, v, mask, out_hbm, ring_len, scale, nullptr, stream);
}

g4_status g4_sliding_attention_after_qkv(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                         const float* mask, uint16_t* out_hbm, int32_t ring_len, float scale,
                                         const int32_t* kv_offset, void* stream) {
  if (!kv_offset) return g4::host::fail(ctx, G4_ERR_INVALID_ARGUMENT, "null pointer: %s", "kv_offset");
  return sliding_attention(ctx, q, k, v, mask, out_hbm, ring_len, scale, kv_offset, stream);
}

static g4_status attention_output(bool tiled, g4_ctx* ctx, const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                      const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                      uint16_t* residual_hbm, void* stream, int32_t m = 1) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_batch(ctx, m);
  if (st != G4_OK) return st;
  st = check_ptrs(ctx, {{x, "x"},
                                  {post_attn_rms_weight, "post_attn_rms_weight"},
                                  {o_weight, "o_weight"},
                                  {o_weight_scale, "o_weight_scale"},
                                  {residual_hbm, "residual_hbm"}});
  if (st != G4_OK) return st;
  if ((st = check_tp(ctx)) != G4_OK) return st;
  DeviceGuard guard(ctx->device);
  g4::OArgs a{x, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, tiled};
  if (m > 1) return cuda_status(ctx, g4::launch_o_batch(a, m, env_of(ctx, stream)), "sliding_attention_output_batch launch");
  return cuda_status(ctx, g4::launch_o(a, env_of(ctx, stream)), "sliding_attention_output launch");
}

static g4_status decoder_feedforward(bool tiled, g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                 const uint8_t* up_weight_packed, const uint8_t* gate_weight_packed,
                                 const uint8_t* down_weight_packed, const uint8_t* up_weight_scale,
                                 const uint8_t* gate_weight_scale, const uint8_t* down_weight_scale,
                                 const float* up_global_scale, const float* gate_global_scale,
                                 const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                 const uint16_t* layer_scalar, void* stream, int32_t m = 1) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  if (m < 1 || m > g4::kBatchMax) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "m must be in [1, 64]");
  if (m > 1 && (ctx->tp_world != 1 || !ctx->batch_ok))
    return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "a batch of tokens runs on a one-GPU context only");
  g4_status st = check_ptrs(ctx, {{residual_hbm, "residual_hbm"},
                                  {pre_ff_rms_weight, "pre_ff_rms_weight"},
                                  {up_weight_packed, "up_weight_packed"},
                                  {gate_weight_packed, "gate_weight_packed"},
                                  {down_weight_packed, "down_weight_packed"},
                                  {up_weight_scale, "up_weight_scale"},
                                  {gate_weight_scale, "gate_weight_scale"},
                                  {down_weight_scale, "down_weight_scale"},
                                  {up_global_scale, "up_global_scale"},
                                  {gate_global_scale, "gate_global_scale"},
                                  {down_global_scale, "down_global_scale"},
                                  {post_ff_rms_weight, "post_ff_rms_weight"},
                                  {layer_scalar, "layer_scalar"}});
  if (st != G4_OK) return st;
  if ((st = check_tp(ctx)) != G4_OK) return st;
  DeviceGuard guard(ctx->device);
  g4::FfnArgs a{residual_hbm,      pre_ff_rms_weight, up_weight_packed, gate_weight_packed, down_weight_packed,
                up_weight_scale,   gate_weight_scale, down_weight_scale, up_global_scale,   gate_global_scale,
                down_global_scale, post_ff_rms_weight, layer_scalar, tiled};
  if (m > 1)
    return cuda_status(ctx, g4::launch_ffn_nvfp4_batch(a, m, env_of(ctx, stream)), "decoder_feedforward_batch launch");
  return cuda_status(ctx, g4::launch_ffn_nvfp4(a, env_of(ctx, stream)), "decoder_feedforward launch");
}


g4_status g4_sliding_project_qkv(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight, const uint8_t* k_weight,
                                 const uint8_t* v_weight, const uint16_t* q_weight_scale,
                                 const uint16_t* k_weight_scale, const uint16_t* v_weight_scale,
                                 const uint16_t* input_rms_weight, const uint16_t* q_rms_weight,
                                 const uint16_t* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                                 const uint16_t* cos, const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache,
                                 uint16_t* q_out, int32_t ring_len, int32_t rope_rows, void* stream) {
  return project_qkv(false, ctx, x, q_weight, k_weight, v_weight, q_weight_scale, k_weight_scale, v_weight_scale,
                     input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache,
                     q_out, ring_len, rope_rows, stream);
}

g4_status g4_sliding_project_qkv_tiled(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight,
                                       const uint8_t* k_weight, const uint8_t* v_weight,
                                       const uint16_t* q_weight_scale, const uint16_t* k_weight_scale,
                                       const uint16_t* v_weight_scale, const uint16_t* input_rms_weight,
                                       const uint16_t* q_rms_weight, const uint16_t* k_rms_weight,
                                       const int32_t* kv_offset, const int32_t* rope_offset, const uint16_t* cos,
                                       const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache, uint16_t* q_out,
                                       int32_t ring_len, int32_t rope_rows, void* stream) {
  return project_qkv(true, ctx, x, q_weight, k_weight, v_weight, q_weight_scale, k_weight_scale, v_weight_scale,
                     input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache,
                     q_out, ring_len, rope_rows, stream);
}

g4_status g4_sliding_attention_output(g4_ctx* ctx, const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                      const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                      uint16_t* residual_hbm, void* stream) {
  return attention_output(false, ctx, x, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, stream);
}

g4_status g4_sliding_attention_output_tiled(g4_ctx* ctx, const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                            const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                            uint16_t* residual_hbm, void* stream) {
  return attention_output(true, ctx, x, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, stream);
}

g4_status g4_sliding_project_qkv_batch(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight,
                                       const uint8_t* k_weight, const uint8_t* v_weight,
                                       const uint16_t* q_weight_scale, const uint16_t* k_weight_scale,
                                       const uint16_t* v_weight_scale, const uint16_t* input_rms_weight,
                                       const uint16_t* q_rms_weight, const uint16_t* k_rms_weight,
                                       const int32_t* kv_offset, const int32_t* rope_offset, const uint16_t* cos,
                                       const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache, uint16_t* q_out,
                                       int32_t ring_len, int32_t rope_rows, int32_t m, void* stream) {
  return project_qkv(false, ctx, x, q_weight, k_weight, v_weight, q_weight_scale, k_weight_scale, v_weight_scale,
                     input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache,
                     q_out, ring_len, rope_rows, stream, m);
}

g4_status g4_sliding_project_qkv_batch_tiled(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight,
                                             const uint8_t* k_weight, const uint8_t* v_weight,
                                             const uint16_t* q_weight_scale, const uint16_t* k_weight_scale,
                                             const uint16_t* v_weight_scale, const uint16_t* input_rms_weight,
                                             const uint16_t* q_rms_weight, const uint16_t* k_rms_weight,
                                             const int32_t* kv_offset, const int32_t* rope_offset,
                                             const uint16_t* cos, const uint16_t* sin, uint16_t* k_cache,
                                             uint16_t* v_cache, uint16_t* q_out, int32_t ring_len, int32_t rope_rows,
                                             int32_t m, void* stream) {
  return project_qkv(true, ctx, x, q_weight, k_weight, v_weight, q_weight_scale, k_weight_scale, v_weight_scale,
                     input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache,
                     q_out, ring_len, rope_rows, stream, m);
}

g4_status g4_sliding_attention_batch(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                     const float* mask, uint16_t* out_hbm, int32_t ring_len, float scale,
                                     const int32_t* kv_offset, int32_t m, void* stream) {
  return sliding_attention(ctx, q, k, v, mask, out_hbm, ring_len, scale, kv_offset, stream, m);
}

g4_status g4_sliding_attention_output_batch(g4_ctx* ctx, const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                            const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                            uint16_t* residual_hbm, int32_t m, void* stream) {
  return attention_output(false, ctx, x, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, stream, m);
}

g4_status g4_sliding_attention_output_batch_tiled(g4_ctx* ctx, const uint16_t* x,
                                                  const uint16_t* post_attn_rms_weight, const uint8_t* o_weight,
                                                  const uint16_t* o_weight_scale, uint16_t* residual_hbm, int32_t m,
                                                  void* stream) {
  return attention_output(true, ctx, x, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, stream, m);
}

g4_status g4_decoder_feedforward(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                 const uint8_t* up_weight_packed, const uint8_t* gate_weight_packed,
                                 const uint8_t* down_weight_packed, const uint8_t* up_weight_scale,
                                 const uint8_t* gate_weight_scale, const uint8_t* down_weight_scale,
                                 const float* up_global_scale, const float* gate_global_scale,
                                 const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                 const uint16_t* layer_scalar, void* stream) {
  return decoder_feedforward(false, ctx, residual_hbm, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
                             down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale,
                             up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar,
                             stream);
}

g4_status g4_decoder_feedforward_tiled(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                       const uint8_t* up_gate_weight_tiled, const uint8_t* down_weight_tiled,
                                       const uint8_t* up_gate_scale_tiled, const uint8_t* down_scale_tiled,
                                       const float* up_global_scale, const float* gate_global_scale,
                                       const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                       const uint16_t* layer_scalar, void* stream) {
  // the gate matrices are interleaved into the up buffers: pass them again where the row-major
  // path takes the gate pointers (validated, not read)
  return decoder_feedforward(true, ctx, residual_hbm, pre_ff_rms_weight, up_gate_weight_tiled, up_gate_weight_tiled,
                             down_weight_tiled, up_gate_scale_tiled, up_gate_scale_tiled, down_scale_tiled,
                             up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar,
                             stream);
}

g4_status g4_decoder_feedforward_batch(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                       const uint8_t* up_weight_packed, const uint8_t* gate_weight_packed,
                                       const uint8_t* down_weight_packed, const uint8_t* up_weight_scale,
                                       const uint8_t* gate_weight_scale, const uint8_t* down_weight_scale,
                                       const float* up_global_scale, const float* gate_global_scale,
                                       const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                       const uint16_t* layer_scalar, int32_t m, void* stream) {
  return decoder_feedforward(false, ctx, residual_hbm, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
                             down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale,
                             up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar,
                             stream, m);
}

g4_status g4_decoder_feedforward_batch_tiled(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                             const uint8_t* up_gate_weight_tiled, const uint8_t* down_weight_tiled,
                                             const uint8_t* up_gate_scale_tiled, const uint8_t* down_scale_tiled,
                                             const float* up_global_scale, const float* gate_global_scale,
                                             const float* down_global_scale, const uint16_t* post_ff_rms_weight,
                                             const uint16_t* layer_scalar, int32_t m, void* stream) {
  return decoder_feedforward(true, ctx, residual_hbm, pre_ff_rms_weight, up_gate_weight_tiled, up_gate_weight_tiled,
                             down_weight_tiled, up_gate_scale_tiled, up_gate_scale_tiled, down_scale_tiled,
                             up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar,
                             stream, m);
}

g4_status g4_embed_token(g4_ctx* ctx, const uint16_t* embedding_table, const int32_t* offset, uint16_t* out,
                         int32_t vocab_rows, void* stream) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_ptrs(ctx, {{embedding_table, "embedding_table"}, {offset, "offset"}, {out, "out"}});
  if (st != G4_OK) return st;
  if (vocab_rows <= 0 || vocab_rows > g4::kVocab)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be in [1, 262144]", "vocab_rows");
  DeviceGuard guard(ctx->device);
  return cuda_status(ctx, g4::launch_embed(embedding_table, offset, out, vocab_rows, env_of(ctx, stream)),
                     "embed_token launch");
}

g4_status g4_final_norm_and_logits(g4_ctx* ctx, const uint16_t* input, const uint16_t* rms_weight,
                                   const uint16_t* lm_head_weight, uint16_t* out, int32_t vocab_rows, void* stream) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_ptrs(ctx, {{input, "input"}, {rms_weight, "rms_weight"}, {lm_head_weight, "lm_head_weight"},
                                  {out, "out"}});
  if (st != G4_OK) return st;
  if (vocab_rows <= 0 || vocab_rows > g4::kVocab)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be in [1, 262144]", "vocab_rows");
  DeviceGuard guard(ctx->device);
  return cuda_status(ctx, g4::launch_logits(input, rms_weight, lm_head_weight, out, vocab_rows, env_of(ctx, stream)),
                     "final_norm_and_logits launch");
}

g4_status g4_final_norm_and_logits_batch(g4_ctx* ctx, const uint16_t* input, const uint16_t* rms_weight,
                                         const uint16_t* lm_head_weight, uint16_t* out, int32_t vocab_rows, int32_t m,
                                         void* stream) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  if (m < 1 || m > g4::kBatchMax) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "m must be in [1, 64]");
  g4_status st = check_ptrs(ctx, {{input, "input"}, {rms_weight, "rms_weight"}, {lm_head_weight, "lm_head_weight"},
                                  {out, "out"}});
  if (st != G4_OK) return st;
  if (vocab_rows <= 0 || vocab_rows > g4::kVocab)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be in [1, 262144]", "vocab_rows");
  DeviceGuard guard(ctx->device);
  const g4::LaunchEnv env = env_of(ctx, stream);
  const cudaError_t e = m > 1 ? g4::launch_logits_batch(input, rms_weight, lm_head_weight, out, vocab_rows, m, env)
                              : g4::launch_logits(input, rms_weight, lm_head_weight, out, vocab_rows, env);
  return cuda_status(ctx, e, "final_norm_and_logits_batch launch");
}

g4_status g4_full_project_qkv(g4_ctx* ctx, const uint16_t* x, const uint8_t* q_weight, const uint8_t* k_weight,
                              const uint16_t* q_weight_scale, const uint16_t* k_weight_scale,
                              const uint16_t* input_rms_weight, const uint16_t* q_rms_weight,
                              const uint16_t* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                              const uint16_t* cos, const uint16_t* sin, uint16_t* k_cache, uint16_t* v_cache,
                              uint16_t* q_out, int32_t rope_rows, void* stream) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_ptrs(ctx, {{x, "x"},
                                  {q_weight, "q_weight"},
                                  {k_weight, "k_weight"},
                                  {q_weight_scale, "q_weight_scale"},
                                  {k_weight_scale, "k_weight_scale"},
                                  {input_rms_weight, "input_rms_weight"},
                                  {q_rms_weight, "q_rms_weight"},
                                  {k_rms_weight, "k_rms_weight"},
                                  {kv_offset, "kv_offset"},
                                  {rope_offset, "rope_offset"},
                                  {cos, "cos"},
                                  {sin, "sin"},
                                  {k_cache, "k_cache"},
                                  {v_cache, "v_cache"},
                                  {q_out, "q_out"}});
  if (st != G4_OK) return st;
  if (rope_rows <= 0 || int64_t(rope_rows) * g4::kDf * 2 > INT32_MAX)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be positive (byte offsets within i32)", "rope_rows");
  if (ctx->tp_world != 1) return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "full_project_qkv runs on one GPU");
  DeviceGuard guard(ctx->device);
  const g4::FullQkvArgs a{x,           q_weight, k_weight, q_weight_scale, k_weight_scale, input_rms_weight,
                          q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache, q_out,
                          rope_rows,   false};
  return cuda_status(ctx, g4::launch_full_qkv(a, env_of(ctx, stream)), "full_project_qkv launch");
}

static g4_status full_attention(bool first, g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                const float* mask, float* running_max, float* running_sum, uint16_t* out_hbm,
                                void* stream) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_ptrs(ctx, {{q, "q"},
                                  {k, "k"},
                                  {v, "v"},
                                  {mask, "mask"},
                                  {running_max, "running_max"},
                                  {running_sum, "running_sum"},
                                  {out_hbm, "out_hbm"}});
  if (st != G4_OK) return st;
  if (ctx->tp_world != 1) return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "full attention runs on one GPU");
  DeviceGuard guard(ctx->device);
  const g4::FullAttnArgs a{q, k, v, mask, running_max, running_sum, out_hbm, first};
  return cuda_status(ctx, g4::launch_full_attention(a, env_of(ctx, stream)), "full attention page launch");
}

g4_status g4_full_attention_first_page(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                       const float* mask, float* running_max, float* running_sum, uint16_t* out_hbm,
                                       void* stream) {
  return full_attention(true, ctx, q, k, v, mask, running_max, running_sum, out_hbm, stream);
}

g4_status g4_full_attention_page(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                 const float* mask, float* running_max, float* running_sum, uint16_t* out_hbm,
                                 void* stream) {
  return full_attention(false, ctx, q, k, v, mask, running_max, running_sum, out_hbm, stream);
}

g4_status g4_full_attention_output(g4_ctx* ctx, const uint16_t* x, const float* running_sum,
                                   const uint16_t* post_attn_rms_weight, const uint8_t* o_weight,
                                   const uint16_t* o_weight_scale, uint16_t* residual_hbm, void* stream) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_ptrs(ctx, {{x, "x"},
                                  {running_sum, "running_sum"},
                                  {post_attn_rms_weight, "post_attn_rms_weight"},
                                  {o_weight, "o_weight"},
                                  {o_weight_scale, "o_weight_scale"},
                                  {residual_hbm, "residual_hbm"}});
  if (st != G4_OK) return st;
  if (ctx->tp_world != 1) return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "full_attention_output runs on one GPU");
  DeviceGuard guard(ctx->device);
  const g4::FullOArgs a{x, running_sum, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, false};
  return cuda_status(ctx, g4::launch_full_o(a, env_of(ctx, stream)), "full_attention_output launch");
}

static g4_status decoder_feedforward_fp8(bool tiled, g4_ctx* ctx, uint16_t* residual_hbm,
                                         const uint16_t* pre_ff_rms_weight, const uint8_t* up_weight,
                                         const uint8_t* gate_weight, const uint8_t* down_weight,
                                         const float* up_weight_scale, const float* gate_weight_scale,
                                         const float* down_weight_scale, const uint16_t* post_ff_rms_weight,
                                         const uint16_t* layer_scalar, void* stream, int32_t m = 1) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  if (m < 1 || m > g4::kBatchMax) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "m must be in [1, 64]");
  if (m > 1 && (ctx->tp_world != 1 || !ctx->batch_ok))
    return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "a batch of tokens runs on a one-GPU context only");
  g4_status st = check_ptrs(ctx, {{residual_hbm, "residual_hbm"},
                                  {pre_ff_rms_weight, "pre_ff_rms_weight"},
                                  {up_weight, "up_weight"},
                                  {gate_weight, "gate_weight"},
                                  {down_weight, "down_weight"},
                                  {up_weight_scale, "up_weight_scale"},
                                  {gate_weight_scale, "gate_weight_scale"},
                                  {down_weight_scale, "down_weight_scale"},
                                  {post_ff_rms_weight, "post_ff_rms_weight"},
                                  {layer_scalar, "layer_scalar"}});
  if (st != G4_OK) return st;
  if ((st = check_tp(ctx)) != G4_OK) return st;
  DeviceGuard guard(ctx->device);
  g4::Ffn8Args a{residual_hbm,      pre_ff_rms_weight, up_weight,          gate_weight,  down_weight, up_weight_scale,
                 gate_weight_scale, down_weight_scale, post_ff_rms_weight, layer_scalar, tiled};
  if (m > 1)
    return cuda_status(ctx, g4::launch_ffn_fp8_batch(a, m, env_of(ctx, stream)), "decoder_feedforward_fp8_batch launch");
  return cuda_status(ctx, g4::launch_ffn_fp8(a, env_of(ctx, stream)), "decoder_feedforward_fp8 launch");
}

g4_status g4_decoder_feedforward_fp8(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                     const uint8_t* up_weight, const uint8_t* gate_weight, const uint8_t* down_weight,
                                     const float* up_weight_scale, const float* gate_weight_scale,
                                     const float* down_weight_scale, const uint16_t* post_ff_rms_weight,
                                     const uint16_t* layer_scalar, void* stream) {
  return decoder_feedforward_fp8(false, ctx, residual_hbm, pre_ff_rms_weight, up_weight, gate_weight, down_weight,
                                 up_weight_scale, gate_weight_scale, down_weight_scale, post_ff_rms_weight,
                                 layer_scalar, stream);
}

g4_status g4_decoder_feedforward_fp8_tiled(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                           const uint8_t* up_gate_weight_tiled, const uint8_t* down_weight_tiled,
                                           const float* up_weight_scale, const float* gate_weight_scale,
                                           const float* down_weight_scale, const uint16_t* post_ff_rms_weight,
                                           const uint16_t* layer_scalar, void* stream) {
  // the gate rows are interleaved into the up buffer: it is passed again for the gate pointer
  // (validated, not read)
  return decoder_feedforward_fp8(true, ctx, residual_hbm, pre_ff_rms_weight, up_gate_weight_tiled,
                                 up_gate_weight_tiled, down_weight_tiled, up_weight_scale, gate_weight_scale,
                                 down_weight_scale, post_ff_rms_weight, layer_scalar, stream);
}

g4_status g4_decoder_feedforward_fp8_batch(g4_ctx* ctx, uint16_t* residual_hbm, const uint16_t* pre_ff_rms_weight,
                                           const uint8_t* up_weight, const uint8_t* gate_weight,
                                           const uint8_t* down_weight, const float* up_weight_scale,
                                           const float* gate_weight_scale, const float* down_weight_scale,
                                           const uint16_t* post_ff_rms_weight, const uint16_t* layer_scalar, int32_t m,
                                           void* stream) {
  return decoder_feedforward_fp8(false, ctx, residual_hbm, pre_ff_rms_weight, up_weight, gate_weight, down_weight,
                                 up_weight_scale, gate_weight_scale, down_weight_scale, post_ff_rms_weight,
                                 layer_scalar, stream, m);
}

g4_status g4_decoder_feedforward_fp8_batch_tiled(g4_ctx* ctx, uint16_t* residual_hbm,
                                                 const uint16_t* pre_ff_rms_weight,
                                                 const uint8_t* up_gate_weight_tiled, const uint8_t* down_weight_tiled,
                                                 const float* up_weight_scale, const float* gate_weight_scale,
                                                 const float* down_weight_scale, const uint16_t* post_ff_rms_weight,
                                                 const uint16_t* layer_scalar, int32_t m, void* stream) {
  return decoder_feedforward_fp8(true, ctx, residual_hbm, pre_ff_rms_weight, up_gate_weight_tiled,
                                 up_gate_weight_tiled, down_weight_tiled, up_weight_scale, gate_weight_scale,
                                 down_weight_scale, post_ff_rms_weight, layer_scalar, stream, m);
}

g4_status g4_tp_init(g4_ctx* ctx, int32_t rank, int32_t world, void* blob_out) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  if (!blob_out) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "null pointer: %s", "blob_out");
  if (!(world == 1 || world == 2 || world == 4 || world == 8) || rank < 0 || rank >= world)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s: world must be 1, 2, 4 or 8 and 0 <= rank < world", "g4_tp_init");
  DeviceGuard guard(ctx->device);
  cudaError_t e = tp_release(ctx);
  cudaDeviceProp prop;
  if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, ctx->device);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->tp_buf, kTpBufferBytes);
  if (e == cudaSuccess) e = cudaMemset(ctx->tp_buf, 0, kTpBufferBytes);
  // a rank's down slice is zero-padded to whole units: the padded activation entries must read 0
  if (e == cudaSuccess) e = cudaMemset(ctx->sc.act, 0, ctx->act_bytes);
  TpBlob b;
  std::memset(&b, 0, sizeof b);
  if (e == cudaSuccess && world > 1) e = cudaIpcGetMemHandle(&b.handle, ctx->tp_buf);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    tp_release(ctx);
    return cuda_status(ctx, e, "g4_tp_init");
  }
  b.magic = kTpMagic;
  b.version = kTpVersion;
  b.rank = rank;
  b.world = world;
  std::memcpy(b.uuid, prop.uuid.bytes, sizeof b.uuid);
  b.bytes = kTpBufferBytes;
  b.generation = ++ctx->tp_generation;
  std::memset(ctx->tp_blob, 0, sizeof ctx->tp_blob);
  std::memcpy(ctx->tp_blob, &b, sizeof b);
  std::memcpy(blob_out, ctx->tp_blob, G4_TP_BLOB_BYTES);
  ctx->tp_rank = rank;
  ctx->tp_world = world;
  ctx->tp = g4::TpLink{0, 1, {}, nullptr, 0, ctx->tp_wait_ns};
  ctx->tp_ready = world == 1;
  return G4_OK;
}

g4_status g4_tp_connect(g4_ctx* ctx, const void* blobs) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  if (!blobs) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "null pointer: %s", "blobs");
  if (!ctx->tp_buf) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s: call g4_tp_init first", "g4_tp_connect");
  const int world = ctx->tp_world, rank = ctx->tp_rank;
  const unsigned char* raw = static_cast<const unsigned char*>(blobs);
  TpBlob b[g4::kMaxTp];
  for (int s = 0; s < world; ++s) {
    std::memcpy(&b[s], raw + size_t(s) * G4_TP_BLOB_BYTES, sizeof(TpBlob));
    if (b[s].magic != kTpMagic || b[s].version != kTpVersion || b[s].rank != s || b[s].world != world ||
        b[s].bytes != kTpBufferBytes)
      return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s: blobs are not every rank's g4_tp_init output in rank order",
                  "g4_tp_connect");
  }
  if (std::memcmp(raw + size_t(rank) * G4_TP_BLOB_BYTES, ctx->tp_blob, G4_TP_BLOB_BYTES) != 0)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s: this rank's blob is not the one g4_tp_init returned",
                "g4_tp_connect");
  for (int s = 0; s < world; ++s)
    for (int t = s + 1; t < world; ++t)
      if (std::memcmp(b[s].uuid, b[t].uuid, sizeof b[s].uuid) == 0)
        return fail(ctx, G4_ERR_UNSUPPORTED, "%s: two ranks share one GPU (the exchange needs one GPU per rank)",
                    "g4_tp_connect");
  DeviceGuard guard(ctx->device);
  for (void*& p : ctx->tp_peer) {  // a second connect replaces the first
    if (p) cudaIpcCloseMemHandle(p);
    p = nullptr;
  }
  // every rank sees the same blobs, so every rank takes the same generation, larger than any
  // earlier setup of any member: words stored under an earlier setup never match this one's tags
  uint32_t gen = 0;
  for (int s = 0; s < world; ++s) gen = b[s].generation > gen ? b[s].generation : gen;
  ctx->tp_generation = gen;
  g4::TpLink link{rank, world, {}, nullptr, gen % 255u + 1u, ctx->tp_wait_ns};
  for (int s = 0; s < world; ++s) {
    if (s == rank) {
      link.slots[s] = static_cast<unsigned long long*>(ctx->tp_buf);
      continue;
    }
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, b[s].handle, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (void*& q : ctx->tp_peer) {
        if (q) cudaIpcCloseMemHandle(q);
        q = nullptr;
      }
      return cuda_status(ctx, e, "g4_tp_connect: opening a peer's exchange buffer");
    }
    ctx->tp_peer[s] = p;
    link.slots[s] = static_cast<unsigned long long*>(p);
  }
  link.epoch = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(ctx->tp_buf) +
                                           g4::kTpExchangeWords * sizeof(unsigned long long));
  ctx->tp = link;
  ctx->tp_ready = true;
  return G4_OK;
}

g4_status g4_tp_set_wait_limit(g4_ctx* ctx, uint64_t limit_ns) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  if (limit_ns < 1000000ull || limit_ns > 60000000000ull)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be in [1 ms, 60 s]", "limit_ns");
  ctx->tp_wait_ns = limit_ns;
  ctx->tp.wait_ns = limit_ns;
  return G4_OK;
}

g4_status g4_pack_tiles(g4_ctx* ctx, const uint8_t* src, const uint8_t* src2, uint8_t* dst, int32_t rows,
                        int32_t row_bytes, int32_t unit_bytes, int32_t tile_rows, void* stream) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_ptrs(ctx, {{src, "src"}, {dst, "dst"}});
  if (st != G4_OK) return st;
  if (src2 && !aligned16(src2)) return fail(ctx, G4_ERR_MISALIGNED, "pointer not 16-byte aligned: %s", "src2");
  if (rows <= 0 || row_bytes <= 0 || unit_bytes <= 0 || tile_rows <= 0 || unit_bytes % 16 != 0 ||
      row_bytes % unit_bytes != 0 || rows % tile_rows != 0)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s: need rows %% tile_rows == 0, row_bytes %% unit_bytes == 0, "
                "unit_bytes %% 16 == 0", "g4_pack_tiles");
  const uintptr_t n = uintptr_t(rows) * uintptr_t(row_bytes);
  const uintptr_t d0 = reinterpret_cast<uintptr_t>(dst), dn = n * (src2 ? 2 : 1);
  for (const uint8_t* sp : {src, src2}) {
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(sp);
    if (sp && s0 < d0 + dn && d0 < s0 + n)
      return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s: a source overlaps dst", "g4_pack_tiles");
  }
  DeviceGuard guard(ctx->device);
  return cuda_status(ctx, g4::launch_pack_tiles(src, src2, dst, rows, row_bytes, unit_bytes, tile_rows,
                                                static_cast<cudaStream_t>(stream)),
                     "g4_pack_tiles launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// g4_sliding_attention_output_noalloc: the O op on a fixed block of static device memory.

namespace {

// 512 KiB per device (the O op needs 510,208 bytes on a 148-SM B200). The entry point zeroes
// the whole block before every launch, so every call starts at epoch 1 with no stale word.
constexpr size_t kStaticScratchBytes = size_t(512) << 10;
constexpr int kStaticMaxDevices = 64;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

// Per device: the block's address (cudaGetSymbolAddress) and the SM count, looked up by the first
// call on that device. A __device__ symbol's address belongs to a CUDA context, so the entry
// also records the context it was looked up in and is redone when the calling thread's current
// context on that device is another one (a cudaDeviceReset, or a driver-API context).
struct StaticEntry {
  void* cu_ctx = nullptr;
  uint8_t* base = nullptr;
  int sms = 0;
};
StaticEntry g_static[kStaticMaxDevices];
std::mutex g_static_mutex;

typedef int (*CtxGetCurrentFn)(void**);  // cuCtxGetCurrent: CUresult (CUcontext*)
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

g4_status static_setup(int dev, uint8_t** base, int* sms) {
  // the calling thread's current context; with none yet, the runtime's first call on the
  // device (the symbol lookup) creates and binds the device's primary context
  void* cur = nullptr;
  CtxGetCurrentFn get = ctx_get_current();
  if (!get || get(&cur) != 0) return G4_ERR_CUDA;
  if (!cur) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || get(&cur) != 0 || !cur) return G4_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_static_mutex);
  StaticEntry& e = g_static[dev];
  if (e.base && e.cu_ctx == cur) {
    *base = e.base;
    *sms = e.sms;
    return G4_OK;
  }
  int major = 0, minor = 0, count = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return G4_ERR_CUDA;
  if (major != 10 || minor != 0 || !g4::proj_geometry_fits(count)) return G4_ERR_UNSUPPORTED;  // built for sm_100a only
  if (g4::prepare_proj_kernels() != cudaSuccess) return G4_ERR_CUDA;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return G4_ERR_CUDA;
  e.cu_ctx = cur;
  e.base = static_cast<uint8_t*>(p);
  e.sms = count;
  *base = e.base;
  *sms = count;
  return G4_OK;
}

}  // namespace

extern "C" {

g4_status g4_sliding_attention_output_noalloc(const uint16_t* x, const uint16_t* post_attn_rms_weight,
                                              const uint8_t* o_weight, const uint16_t* o_weight_scale,
                                              uint16_t* residual_hbm, void* stream) {
  g4_status st = check_ptrs(nullptr, {{x, "x"},
                                      {post_attn_rms_weight, "post_attn_rms_weight"},
                                      {o_weight, "o_weight"},
                                      {o_weight_scale, "o_weight_scale"},
                                      {residual_hbm, "residual_hbm"}});
  if (st != G4_OK) return st;
  const size_t need = g4::o_scratch_bytes();
  if (need > kStaticScratchBytes) return G4_ERR_UNSUPPORTED;  // this GPU needs more than the static block
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return G4_ERR_CUDA;
  if (dev < 0 || dev >= kStaticMaxDevices) return G4_ERR_UNSUPPORTED;
  uint8_t* base = nullptr;
  int sms = 0;
  if ((st = static_setup(dev, &base, &sms)) != G4_OK) return st;

  const size_t off_counters = g4::kScratchHeadBytes;
  const size_t off_ss = off_counters + size_t(g4::kCounterCount) * sizeof(uint32_t);
  const size_t off_partials = off_ss + g4::kTileSsBytes;
  g4::LaunchEnv env;
  env.device = dev;
  env.sm_count = sms;
  env.stream = static_cast<cudaStream_t>(stream);
  env.pdl = false;
  env.sc.err = reinterpret_cast<uint32_t*>(base);
  env.sc.counters = reinterpret_cast<uint32_t*>(base + off_counters);
  env.sc.partials = reinterpret_cast<float*>(base + off_partials);
  env.sc.act = nullptr;
  env.sc.tile_ss = reinterpret_cast<unsigned long long*>(base + off_ss);
  env.sc.trace = nullptr;
  env.maps = nullptr;
  // the error word, the epoch counters and every epoch-tagged word must be zero when the kernel
  // starts
  if (cudaMemsetAsync(base, 0, need, env.stream) != cudaSuccess) return G4_ERR_CUDA;
  const g4::OArgs a{x, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, false};
  return g4::launch_o_uncached(a, env) == cudaSuccess ? G4_OK : G4_ERR_CUDA;
}

#ifdef G4_TRACE
// Profiling builds only (not part of the public header): copy the phase timestamps out.
g4_status g4_trace_read(g4_ctx* ctx, uint64_t* host, int n) {
  if (!ctx || !host || n < 0 || n > 65536 + 4096 * 32 * 8) return G4_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(host, ctx->sc.trace, size_t(n) * sizeof(uint64_t), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(ctx->sc.trace, 0, size_t(65536 + 4096 * 32 * 8) * sizeof(uint64_t));
  return e == cudaSuccess ? G4_OK : G4_ERR_CUDA;
}
#endif

}  // extern "C"
