// Decode driver: one token through a whole model as one stream of launches (the reference host's
// Decode::run / run_layers, furiosa-opt-gemma4-12B/src/host/runtime.rs:340-451, with the position
// offsets it uploads once per token, runtime.rs:231-247).
//
// The host keeps the model as a table of layers. A step is:
//   decode_begin   from the device-resident {token, position} (one pair per sequence of a batch):
//                  every distinct ring's slot offset,
//                  the RoPE row offset, every ring's mask row (c <= min(position, ring - 1), the
//                  reference's mask_s rows, runtime.rs:159-160) and the token's scaled embedding
//   per layer      sliding_project_qkv, sliding_attention, sliding_attention_output and the NVFP4 or
//                  FP8 feed-forward, on the decoder's hidden / q / attention buffers
//   logits         final_norm_and_logits over this rank's lm_head rows
// Every kernel is launched with programmatic dependent launch (each waits on its predecessor
// before touching what that one writes), so the next kernel's weight copies start while the
// previous one drains; g4_decoder_capture records the whole step as one CUDA graph, so a token
// costs one graph launch and one 8-byte input update on the host.
//
// A decoder made for a batch of m sequences (g4_decoder_create_batch, m in 2..64, one GPU) runs
// the batched ops instead (g4_batch_attn.cu, g4_batch.cu): each layer's weights are read once for
// all m tokens, every sequence keeping its own ring in the layer's caches ([m][ring][Ns][Ds]) and
// its own position.
#include <algorithm>
#include <cstdlib>
#include <vector>

#include "g4_ctx.cuh"

using namespace g4::host;

namespace g4 {
namespace {

constexpr int kMaxRings = 4;           // distinct ring lengths one model may use
constexpr int kBeginThreads = 256;
constexpr int kBeginBlocks = 16;
// units of each FP8 up/gate CTA's run brought into L2 by a sliding layer's attention (hints)
constexpr int kDefaultL2Units = 12;

struct BeginArgs {
  const int32_t* input;  // [batch] {token, position}
  int32_t* rope_off;     // [batch] position * Ds * 2 (-1 when the position is outside the RoPE table)
  int32_t* kv_off;       // [kMaxRings][kv_stride] (position % ring) * Ns * Ds * 2, per sequence
  float* mask;           // [kMaxRings][batch][mask_stride]
  int batch, kv_stride;
  int rings[kMaxRings];
  int n_rings, mask_stride, rope_rows;
  const uint16_t* table;  // embedding table or null
  int vocab_rows;
  uint16_t* hidden;  // [batch][H]
};

__global__ void __launch_bounds__(kBeginThreads) decode_begin_kernel(BeginArgs a, Scratch sc) {
  pdl_wait_primary();  // the previous step's last kernels still read these buffers
  for (int b = blockIdx.x; b < a.batch; b += gridDim.x) {  // sequence b's offsets and embedding
    const int token = __ldcg(a.input + 2 * b), pos = __ldcg(a.input + 2 * b + 1);
    if (threadIdx.x == 0) a.rope_off[b] = pos >= 0 && pos < a.rope_rows ? pos * kDs * 2 : -1;
    if (threadIdx.x < a.n_rings)
      a.kv_off[threadIdx.x * a.kv_stride + b] = pos >= 0 ? (pos % a.rings[threadIdx.x]) * kPs * 2 : -1;
    if (a.table) {
      if (token >= 0 && token < a.vocab_rows)
        embed_row(a.table + size_t(token) * kH, a.hidden + size_t(b) * kH);
      else if (threadIdx.x == 0)
        atomicOr(sc.err, kErrTokenOffset);
    }
  }
  const int per_ring = a.batch * a.mask_stride, total = a.n_rings * per_ring;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int k = i / per_ring, b = (i / a.mask_stride) % a.batch, c = i % a.mask_stride;
    const int pos = __ldcg(a.input + 2 * b + 1);
    const int row = pos < a.rings[k] - 1 ? pos : a.rings[k] - 1;
    a.mask[i] = c <= row ? 1.0f : 0.0f;
  }
  pdl_launch_dependents();
}

}  // namespace
}  // namespace g4

struct g4_decoder {
  g4_ctx* ctx = nullptr;
  std::vector<g4_layer> layers;
  std::vector<int> ring_of;  // per layer: index into rings
  g4_model model{};
  int rings[g4::kMaxRings] = {};
  int n_rings = 0, mask_stride = 0;
  int batch = 1;   // sequences per step
  int kvs = 4;     // i32 spacing of the rings' kv offsets (16 bytes at batch 1)
  void* buf = nullptr;
  int32_t* input = nullptr;
  int32_t* rope_off = nullptr;
  int32_t* kv_off = nullptr;
  float* mask = nullptr;
  uint16_t *hidden = nullptr, *q = nullptr, *attn = nullptr, *logits = nullptr;
  // full-attention layers: q [Gf, Df], the attention output [Gf, Df], running max / sum [Gf]
  uint16_t *q_full = nullptr, *attn_full = nullptr;
  float *run_max = nullptr, *run_sum = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // units of every FP8 up/gate CTA's run that a sliding layer's attention brings into L2 (0: no
  // hints); G4_DECODER_L2_UNITS overrides the default at creation
  int l2_units = g4::kDefaultL2Units;
};

namespace {

g4_status check_layer(g4_ctx* ctx, const g4_layer& l) {
  if (l.kind != G4_LAYER_SLIDING && l.kind != G4_LAYER_FULL)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "layer.kind must be G4_LAYER_SLIDING or G4_LAYER_FULL");
  const bool full = l.kind == G4_LAYER_FULL;
  if (full && ctx->tp_world != 1) return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "full-attention layers run on one GPU");
  if (!full) {
    g4_status st = check_ptrs(ctx, {{l.v_weight, "layer.v_weight"}, {l.v_weight_scale, "layer.v_weight_scale"}});
    if (st != G4_OK) return st;
  }
  g4_status st = check_ptrs(ctx, {{l.input_rms_weight, "layer.input_rms_weight"},
                                  {l.q_weight, "layer.q_weight"},
                                  {l.k_weight, "layer.k_weight"},
                                  {l.q_weight_scale, "layer.q_weight_scale"},
                                  {l.k_weight_scale, "layer.k_weight_scale"},
                                  {l.q_rms_weight, "layer.q_rms_weight"},
                                  {l.k_rms_weight, "layer.k_rms_weight"},
                                  {l.k_cache, "layer.k_cache"},
                                  {l.v_cache, "layer.v_cache"},
                                  {l.post_attn_rms_weight, "layer.post_attn_rms_weight"},
                                  {l.o_weight, "layer.o_weight"},
                                  {l.o_weight_scale, "layer.o_weight_scale"},
                                  {l.pre_ff_rms_weight, "layer.pre_ff_rms_weight"},
                                  {l.post_ff_rms_weight, "layer.post_ff_rms_weight"},
                                  {l.layer_scalar, "layer.layer_scalar"},
                                  {l.up_weight, "layer.up_weight"},
                                  {l.down_weight, "layer.down_weight"},
                                  {l.up_scale, "layer.up_scale"},
                                  {l.down_scale, "layer.down_scale"}});
  if (st != G4_OK) return st;
  if (!l.tiled) {  // the row-major FFNs read the gate matrix separately
    if ((st = check_ptrs(ctx, {{l.gate_weight, "layer.gate_weight"}})) != G4_OK) return st;
  }
  if (!l.tiled || l.ffn == G4_FFN_FP8) {  // FP8 channel scales are never interleaved
    if ((st = check_ptrs(ctx, {{l.gate_scale, "layer.gate_scale"}})) != G4_OK) return st;
  }
  if (l.ffn == G4_FFN_NVFP4) {
    if ((st = check_ptrs(ctx, {{l.up_global_scale, "layer.up_global_scale"},
                               {l.gate_global_scale, "layer.gate_global_scale"},
                               {l.down_global_scale, "layer.down_global_scale"}})) != G4_OK)
      return st;
  } else if (l.ffn != G4_FFN_FP8) {
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "layer.ffn must be G4_FFN_NVFP4 or G4_FFN_FP8");
  }
  if (l.rope != G4_ROPE_LOCAL && l.rope != G4_ROPE_GLOBAL)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "layer.rope must be G4_ROPE_LOCAL or G4_ROPE_GLOBAL");
  if (full) {
    if (l.ring_len <= 0 || l.ring_len % g4::kTf != 0 || l.ring_len > 64 * g4::kTf)
      return fail(ctx, G4_ERR_UNSUPPORTED, "%s must be a positive multiple of 512, at most 32768", "layer.ring_len");
    if (l.rope != G4_ROPE_GLOBAL) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "a full layer uses G4_ROPE_GLOBAL");
  } else if (l.ring_len <= 0 || l.ring_len % g4::attention_slot_multiple() != 0 ||
             l.ring_len > g4::attention_max_ring()) {
    return fail(ctx, G4_ERR_UNSUPPORTED, "%s must be a positive multiple of 256, at most 8192", "layer.ring_len");
  }
  if (!(l.attn_scale == l.attn_scale)) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s is NaN", "layer.attn_scale");
  return G4_OK;
}

g4::Ffn8Args ffn8_args(const g4_decoder* d, const g4_layer& l) {
  const bool tiled = l.tiled != 0;
  return g4::Ffn8Args{d->hidden,
                      l.pre_ff_rms_weight,
                      l.up_weight,
                      tiled ? l.up_weight : l.gate_weight,
                      l.down_weight,
                      static_cast<const float*>(l.up_scale),
                      static_cast<const float*>(l.gate_scale),
                      static_cast<const float*>(l.down_scale),
                      l.post_ff_rms_weight,
                      l.layer_scalar,
                      tiled};
}

// Every kernel of one token on `stream`.
cudaError_t issue_step(g4_decoder* d, cudaStream_t stream) {
  g4_ctx* ctx = d->ctx;
  g4::LaunchEnv env = env_of(ctx, stream);
  env.pdl = true;  // every kernel of the step waits on its predecessor before using its output
  const g4_model& m = d->model;
  g4::BeginArgs b{};
  b.input = d->input;
  b.rope_off = d->rope_off;
  b.kv_off = d->kv_off;
  b.mask = d->mask;
  for (int k = 0; k < g4::kMaxRings; ++k) b.rings[k] = k < d->n_rings ? d->rings[k] : 1;
  b.n_rings = d->n_rings;
  b.mask_stride = d->mask_stride;
  b.batch = d->batch;
  b.kv_stride = d->kvs;
  b.rope_rows = m.rope_rows;
  b.table = m.embedding_table;
  b.vocab_rows = m.vocab_rows;
  b.hidden = d->hidden;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g4::kBeginBlocks);
    cfg.blockDim = dim3(g4::kBeginThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, g4::decode_begin_kernel, b, env.sc);
    if (e != cudaSuccess) return e;
  }
  const int heads = g4::kNs / ctx->tp_world;
  const int nb = d->batch;
  for (size_t i = 0; i < d->layers.size(); ++i) {
    const g4_layer& l = d->layers[i];
    const int r = d->ring_of[i];
    const bool global = l.rope == G4_ROPE_GLOBAL;
    const bool tiled = l.tiled != 0;
    cudaError_t e;
    if (l.kind == G4_LAYER_FULL) {
      // the reference host's full-layer launches (runtime.rs:462-541): QKV into the position's page,
      // every page up to it (later pages see the position and do nothing), then O
      const int32_t* pos = d->input + 1;
      g4::FullQkvArgs fq{d->hidden,        l.q_weight,       l.k_weight,     l.q_weight_scale, l.k_weight_scale,
                         l.input_rms_weight, l.q_rms_weight, l.k_rms_weight, nullptr,          nullptr,
                         m.cos_full,       m.sin_full,       l.k_cache,      l.v_cache,        d->q_full,
                         m.rope_rows,      tiled};
      fq.slots = l.ring_len;
      fq.position = pos;
      if ((e = g4::launch_full_qkv(fq, env)) != cudaSuccess) return e;
      for (int p = 0; p < l.ring_len / g4::kTf; ++p) {
        g4::FullAttnArgs fa{d->q_full, l.k_cache + size_t(p) * g4::kTf * g4::kDf, l.v_cache + size_t(p) * g4::kTf * g4::kDf,
                            nullptr,   d->run_max, d->run_sum, d->attn_full, p == 0};
        fa.page = p;
        fa.position = pos;
        if ((e = g4::launch_full_attention(fa, env)) != cudaSuccess) return e;
      }
      const g4::FullOArgs fo{d->attn_full, d->run_sum, l.post_attn_rms_weight, l.o_weight, l.o_weight_scale,
                             d->hidden,    tiled};
      if ((e = g4::launch_full_o(fo, env)) != cudaSuccess) return e;
    } else {
    const g4::QkvArgs qa{d->hidden,        l.q_weight,       l.k_weight,         l.v_weight,
                         l.q_weight_scale, l.k_weight_scale, l.v_weight_scale,   l.input_rms_weight,
                         l.q_rms_weight,   l.k_rms_weight,   d->kv_off + d->kvs * r,  d->rope_off,
                         global ? m.cos_global : m.cos_local,  global ? m.sin_global : m.sin_local,
                         l.k_cache,        l.v_cache,        d->q,               l.ring_len,
                         m.rope_rows,      tiled};
    if ((e = nb > 1 ? g4::launch_qkv_batch(qa, nb, env) : g4::launch_qkv(qa, env)) != cudaSuccess) return e;
    g4::AttnArgs aa{d->q,      l.k_cache, l.v_cache,    d->mask + size_t(r) * nb * d->mask_stride,
                    d->attn,   l.ring_len, heads,        l.attn_scale,
                    d->kv_off + d->kvs * r};  // the slots the QKV op above writes
    aa.batch = nb;
    aa.mask_stride = d->mask_stride;
    const g4::OArgs oa{d->attn, l.post_attn_rms_weight, l.o_weight, l.o_weight_scale, d->hidden, tiled};
    if (nb == 1 && d->l2_units > 0) {
      // attention moves few bytes: it brings O's weights and the first units of every FP8
      // up/gate CTA's run into L2 for the kernels that follow it
      aa.next[0] = g4::l2_hint_o(oa, g4::kL2HintAllUnits, env);
      if (l.ffn == G4_FFN_FP8) aa.next[1] = g4::l2_hint_ffn8_upgate(ffn8_args(d, l), d->l2_units, env);
    }
    if ((e = g4::launch_attention(aa, env)) != cudaSuccess) return e;
    if ((e = nb > 1 ? g4::launch_o_batch(oa, nb, env) : g4::launch_o(oa, env)) != cudaSuccess) return e;
    }
    if (l.ffn == G4_FFN_FP8) {
      const g4::Ffn8Args fa = ffn8_args(d, l);
      e = nb > 1 ? g4::launch_ffn_fp8_batch(fa, nb, env) : g4::launch_ffn_fp8(fa, env);
    } else {
      const g4::FfnArgs fa{d->hidden,
                           l.pre_ff_rms_weight,
                           l.up_weight,
                           tiled ? l.up_weight : l.gate_weight,
                           l.down_weight,
                           static_cast<const uint8_t*>(l.up_scale),
                           static_cast<const uint8_t*>(tiled ? l.up_scale : l.gate_scale),
                           static_cast<const uint8_t*>(l.down_scale),
                           l.up_global_scale,
                           l.gate_global_scale,
                           l.down_global_scale,
                           l.post_ff_rms_weight,
                           l.layer_scalar,
                           tiled};
      e = nb > 1 ? g4::launch_ffn_nvfp4_batch(fa, nb, env) : g4::launch_ffn_nvfp4(fa, env);
    }
    if (e != cudaSuccess) return e;
  }
  if (m.lm_head_weight) {
    if (nb > 1)
      return g4::launch_logits_batch(d->hidden, m.final_norm_weight, m.lm_head_weight, d->logits, m.lm_head_rows, nb,
                                     env);
    return g4::launch_logits(d->hidden, m.final_norm_weight, m.lm_head_weight, d->logits, m.lm_head_rows, env);
  }
  return cudaSuccess;
}

void release(g4_decoder* d) {
  if (d->exec) cudaGraphExecDestroy(d->exec);
  if (d->graph) cudaGraphDestroy(d->graph);
  if (d->buf) cudaFree(d->buf);
  d->exec = nullptr;
  d->graph = nullptr;
  d->buf = nullptr;
}

size_t align_up(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

extern "C" {

g4_status g4_decoder_create(g4_ctx* ctx, const g4_model* model, g4_decoder** out) {
  return g4_decoder_create_batch(ctx, model, 1, out);
}

g4_status g4_decoder_create_batch(g4_ctx* ctx, const g4_model* model, int32_t batch, g4_decoder** out) {
  if (!ctx) return G4_ERR_INVALID_ARGUMENT;
  if (!out || !model) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "null pointer: %s", out ? "model" : "out");
  *out = nullptr;
  if (batch < 1 || batch > g4::kBatchMax) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "batch must be in [1, 64]");
  if (batch > 1 && (ctx->tp_world != 1 || !ctx->batch_ok))
    return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "a batch of sequences runs on a one-GPU context only");
  const g4_model& m = *model;
  if (m.n_layers < 0 || (m.n_layers > 0 && !m.layers))
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "model.layers / n_layers");
  g4_status st = check_ptrs(ctx, {{m.cos_local, "model.cos_local"}, {m.sin_local, "model.sin_local"}});
  if (st != G4_OK) return st;
  if (m.rope_rows <= 0 || int64_t(m.rope_rows) * g4::kDs * 2 > INT32_MAX)
    return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be positive (and its byte offsets fit i32)", "model.rope_rows");
  if (m.embedding_table) {
    if ((st = check_ptrs(ctx, {{m.embedding_table, "model.embedding_table"}})) != G4_OK) return st;
    if (m.vocab_rows <= 0 || m.vocab_rows > g4::kVocab)
      return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be in [1, 262144]", "model.vocab_rows");
  }
  if (m.lm_head_weight) {
    if ((st = check_ptrs(ctx, {{m.lm_head_weight, "model.lm_head_weight"},
                               {m.final_norm_weight, "model.final_norm_weight"}})) != G4_OK)
      return st;
    if (m.lm_head_rows <= 0 || m.lm_head_rows > g4::kVocab)
      return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s must be in [1, 262144]", "model.lm_head_rows");
  }
  g4_decoder* d = new g4_decoder();
  d->ctx = ctx;
  d->layers.assign(m.layers, m.layers + m.n_layers);
  d->batch = batch;
  d->kvs = batch > 1 ? (batch + 3) / 4 * 4 : 4;
  if (const char* v = std::getenv("G4_DECODER_L2_UNITS")) d->l2_units = std::max(0, std::atoi(v));
  for (const g4_layer& l : d->layers) {
    if ((st = check_layer(ctx, l)) != G4_OK) {
      delete d;
      return st;
    }
    if (batch > 1 && l.kind == G4_LAYER_FULL) {
      delete d;
      return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "a batched decoder runs sliding-geometry layers only");
    }
    if (l.kind == G4_LAYER_FULL && (!m.cos_full || !m.sin_full)) {
      delete d;
      return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "a G4_LAYER_FULL layer needs model.cos_full / sin_full");
    }
    if (l.kind == G4_LAYER_SLIDING && l.rope == G4_ROPE_GLOBAL && (!m.cos_global || !m.sin_global)) {
      delete d;
      return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "a G4_ROPE_GLOBAL layer needs model.cos_global / sin_global");
    }
    if (l.kind == G4_LAYER_FULL) {  // its kernels derive the slot and the mask from the position
      d->ring_of.push_back(0);
      continue;
    }
    int r = 0;
    while (r < d->n_rings && d->rings[r] != l.ring_len) ++r;
    if (r == d->n_rings) {
      if (d->n_rings == g4::kMaxRings) {
        delete d;
        return fail(ctx, G4_ERR_UNSUPPORTED, "%s", "more than 4 distinct ring lengths in one model");
      }
      d->rings[d->n_rings++] = l.ring_len;
    }
    d->ring_of.push_back(r);
    d->mask_stride = l.ring_len > d->mask_stride ? l.ring_len : d->mask_stride;
  }
  if (m.cos_global && (st = check_ptrs(ctx, {{m.cos_global, "model.cos_global"}, {m.sin_global, "model.sin_global"}})) != G4_OK) {
    delete d;
    return st;
  }
  if (m.cos_full && (st = check_ptrs(ctx, {{m.cos_full, "model.cos_full"}, {m.sin_full, "model.sin_full"}})) != G4_OK) {
    delete d;
    return st;
  }
  d->model = m;
  d->model.layers = nullptr;  // the decoder's own copy is d->layers
  // device buffers: control words (inputs | rope offsets | kv offsets) | hidden | q | attention |
  // logits | masks, the per-sequence ones `batch` times
  const size_t nb = size_t(batch);
  const size_t off_rope = align_up(nb * 2 * sizeof(int32_t));
  const size_t off_kv = off_rope + align_up(nb * sizeof(int32_t));
  const size_t off_hidden = off_kv + align_up(size_t(g4::kMaxRings) * d->kvs * sizeof(int32_t));
  const size_t off_q = off_hidden + align_up(nb * g4::kH * 2);
  const size_t off_attn = off_q + align_up(nb * g4::kQs * 2);
  const size_t off_logits = off_attn + align_up(nb * g4::kQs * 2);
  const size_t off_mask = off_logits + align_up(nb * size_t(m.lm_head_weight ? m.lm_head_rows : 0) * 2);
  const size_t off_full = off_mask + align_up(size_t(d->n_rings) * nb * d->mask_stride * sizeof(float));
  const size_t total = off_full + 2 * align_up(size_t(g4::kQf) * 2) + 2 * align_up(g4::kGf * sizeof(float));
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaMalloc(&d->buf, total);
  if (e == cudaSuccess) e = cudaMemset(d->buf, 0, total);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    release(d);
    delete d;
    return cuda_status(ctx, e, "g4_decoder_create");
  }
  uint8_t* base = static_cast<uint8_t*>(d->buf);
  d->input = reinterpret_cast<int32_t*>(base);
  d->rope_off = reinterpret_cast<int32_t*>(base + off_rope);
  d->kv_off = reinterpret_cast<int32_t*>(base + off_kv);  // kvs i32 per ring
  d->hidden = reinterpret_cast<uint16_t*>(base + off_hidden);
  d->q = reinterpret_cast<uint16_t*>(base + off_q);
  d->attn = reinterpret_cast<uint16_t*>(base + off_attn);
  d->logits = m.lm_head_weight ? reinterpret_cast<uint16_t*>(base + off_logits) : nullptr;
  d->mask = reinterpret_cast<float*>(base + off_mask);
  d->q_full = reinterpret_cast<uint16_t*>(base + off_full);
  d->attn_full = reinterpret_cast<uint16_t*>(base + off_full + align_up(size_t(g4::kQf) * 2));
  d->run_max = reinterpret_cast<float*>(base + off_full + 2 * align_up(size_t(g4::kQf) * 2));
  d->run_sum = d->run_max + 256 / sizeof(float);
  *out = d;
  return G4_OK;
}

g4_status g4_decoder_destroy(g4_decoder* d) {
  if (!d) return G4_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(d->ctx->device);
  release(d);
  delete d;
  return G4_OK;
}

g4_status g4_decoder_buffers(g4_decoder* d, int32_t** input, uint16_t** hidden, uint16_t** logits) {
  if (!d) return G4_ERR_INVALID_ARGUMENT;
  if (input) *input = d->input;
  if (hidden) *hidden = d->hidden;
  if (logits) *logits = d->logits;
  return G4_OK;
}

g4_status g4_decoder_step(g4_decoder* d, void* stream) {
  if (!d) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_tp(d->ctx);
  if (st != G4_OK) return st;
  DeviceGuard guard(d->ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (d->exec) return cuda_status(d->ctx, cudaGraphLaunch(d->exec, s), "g4_decoder_step graph launch");
  return cuda_status(d->ctx, issue_step(d, s), "g4_decoder_step");
}

g4_status g4_decoder_capture(g4_decoder* d, void* stream) {
  if (!d) return G4_ERR_INVALID_ARGUMENT;
  g4_status st = check_tp(d->ctx);
  if (st != G4_OK) return st;
  if (!stream) return fail(d->ctx, G4_ERR_INVALID_ARGUMENT, "%s", "capture needs a stream other than the legacy default");
  DeviceGuard guard(d->ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (d->exec) cudaGraphExecDestroy(d->exec);
  if (d->graph) cudaGraphDestroy(d->graph);
  d->exec = nullptr;
  d->graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_status(d->ctx, e, "g4_decoder_capture: begin");
  const cudaError_t issued = issue_step(d, s);
  cudaGraph_t g = nullptr;
  e = cudaStreamEndCapture(s, &g);
  if (issued != cudaSuccess || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return cuda_status(d->ctx, issued != cudaSuccess ? issued : e, "g4_decoder_capture");
  }
  cudaGraphExec_t x = nullptr;
  e = cudaGraphInstantiate(&x, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    return cuda_status(d->ctx, e, "g4_decoder_capture: instantiate");
  }
  d->graph = g;
  d->exec = x;
  return G4_OK;
}

}  // extern "C"
