// Host-side launch interface of the decode-layer kernels (internal to the library).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <unordered_map>
#include <utility>

#include "g4_common.cuh"

namespace g4 {

struct QkvArgs {
  const uint16_t* x;
  const uint8_t* q_weight;
  const uint8_t* k_weight;
  const uint8_t* v_weight;
  const uint16_t* q_scale;
  const uint16_t* k_scale;
  const uint16_t* v_scale;
  const uint16_t* input_rms;
  const uint16_t* q_rms;
  const uint16_t* k_rms;
  const int32_t* kv_offset;
  const int32_t* rope_offset;
  const uint16_t* cos;
  const uint16_t* sin;
  uint16_t* k_cache;
  uint16_t* v_cache;
  uint16_t* q_out;
  int ring_len;
  int rope_rows;
  bool tiled;  // weights in the unit-tiled layout of g4_pack_tiles (else the reference row-major)
};

// Weights a later engine kernel streams first, requested into L2 by an earlier kernel of the
// decode step whose own HBM traffic is small (attention): the bytes then cross HBM while that
// kernel and the next one's prologue run, and the consumer's TMA loads hit L2. A hint only:
// nothing depends on it for correctness. The weights are unit-tiled (unit u at base + u
// unit_bytes); the consumer's CTA c runs units [c total / grid, (c + 1) total / grid), and the
// first `first_units` of every run are requested (runs' first units before their later ones).
struct L2Hint {
  const uint8_t* base = nullptr;
  uint32_t unit_bytes = 0;
  int total_units = 0;
  int consumer_grid = 0;
  int first_units = 0;
};
constexpr int kL2HintUnitsPerPrefetch = 2;  // units per bulk prefetch (64 KB of fp8 weights)
constexpr int kL2HintAllUnits = 1 << 20;    // first_units: every unit of every run

// This CTA's share (it is `cta` of `ctas` issuing CTAs) of the hints' bulk prefetches, one per
// thread; every thread of the CTA calls it.
__device__ __forceinline__ void issue_l2_hints(const L2Hint* hints, int nh, int cta, int ctas) {
  for (int h = 0; h < nh; ++h) {
    const L2Hint& hint = hints[h];
    if (!hint.base || hint.first_units <= 0 || hint.consumer_grid <= 0) continue;
    const int pieces = (hint.first_units + kL2HintUnitsPerPrefetch - 1) / kL2HintUnitsPerPrefetch;
    const int items = pieces * hint.consumer_grid;
    for (int k = cta + ctas * int(threadIdx.x); k < items; k += ctas * int(blockDim.x)) {
      const int piece = k / hint.consumer_grid, c = k % hint.consumer_grid;
      const int64_t t = hint.total_units, g = hint.consumer_grid;
      const int r0 = int(c * t / g), r1 = int((c + 1) * t / g);
      const int lim = r0 + hint.first_units < r1 ? r0 + hint.first_units : r1;
      const int u0 = r0 + piece * kL2HintUnitsPerPrefetch;
      const int u1 = u0 + kL2HintUnitsPerPrefetch < lim ? u0 + kL2HintUnitsPerPrefetch : lim;
      if (u1 > u0)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(hint.base + size_t(u0) * hint.unit_bytes),
                     "r"(uint32_t(u1 - u0) * hint.unit_bytes)
                     : "memory");
    }
  }
}

struct AttnArgs {
  const uint16_t* q;
  const uint16_t* k_cache;
  const uint16_t* v_cache;
  const float* mask;
  uint16_t* out;
  int ring_len;
  int heads;  // KV heads in the cache (8 / tensor-parallel degree)
  float scale;
  // the preceding QKV op's kv_offset (slot * Ns * Ds * 2), when the caller has it: every other
  // row of the cache is final, so the first pass's K and V rows are loaded before the wait on
  // that op and only the slot's rows after it (null: every row after the wait)
  const int32_t* kv_offset = nullptr;
  // a batch of sequences (g4_sliding_attention_batch): sequence b's query / output rows at
  // b heads Gs Ds, its ring at slots [b ring_len, (b + 1) ring_len) of the caches, its mask row at
  // b mask_stride and its kv_offset at kv_offset[b]
  int batch = 1;
  int mask_stride = 0;
  // the decode driver's hints for the O and feed-forward kernels that follow (issued before the
  // wait on the QKV op)
  L2Hint next[2];
};

struct OArgs {
  const uint16_t* x;
  const uint16_t* post_rms;
  const uint8_t* o_weight;
  const uint16_t* o_scale;
  uint16_t* residual;
  bool tiled;
};

struct FfnArgs {
  uint16_t* residual;
  const uint16_t* pre_rms;
  const uint8_t* up_packed;
  const uint8_t* gate_packed;
  const uint8_t* down_packed;
  const uint8_t* up_scale;
  const uint8_t* gate_scale;
  const uint8_t* down_scale;
  const float* up_global;
  const float* gate_global;
  const float* down_global;
  const uint16_t* post_rms;
  const uint16_t* layer_scalar;
  bool tiled;
};

// The global layer's fused QKV (FOG/src/ops.rs:78-116): one page [Tf, Df] of the K and V caches.
struct FullQkvArgs {
  const uint16_t* x;
  const uint8_t* q_weight;  // [Qf, H]
  const uint8_t* k_weight;  // [Df, H]
  const uint16_t* q_scale;
  const uint16_t* k_scale;
  const uint16_t* input_rms;
  const uint16_t* q_rms;    // [Df]
  const uint16_t* k_rms;
  const int32_t* kv_offset;  // byte offset of the slot in the page: (pos % Tf) * Df * 2
  const int32_t* rope_offset;  // pos * Df * 2
  const uint16_t* cos;       // [rope_rows, Df]
  const uint16_t* sin;
  uint16_t* k_cache;         // [Tf, Df]
  uint16_t* v_cache;
  uint16_t* q_out;           // [Gf, Df]
  int rope_rows;
  bool tiled;
  int slots = kTf;           // cache slots behind k_cache / v_cache (the op: one page)
  // the decode driver: the device-resident position, from which the kernel derives both offsets
  // ((pos % slots) * Df * 2 and pos * Df * 2) instead of reading kv_offset / rope_offset
  const int32_t* position = nullptr;
};

// One page of the global layer's attention (FOG/src/ops.rs:148-182) and its output projection
// (ops.rs:184-199).
struct FullAttnArgs {
  const uint16_t* q;     // [Gf, Df]
  const uint16_t* k;     // [Tf, Df]
  const uint16_t* v;
  const float* mask;     // [Tf]
  float* running_max;    // [Gf]
  float* running_sum;
  uint16_t* out;         // [Gf, Df]
  bool first;
  // the decode driver: the page's index and the device-resident position; a page past the
  // position does nothing, and the mask (null here) is slot <= position
  int page = 0;
  const int32_t* position = nullptr;
};
struct FullOArgs {
  const uint16_t* x;            // [Gf, Df]
  const float* running_sum;     // [Gf]
  const uint16_t* post_rms;
  const uint8_t* o_weight;      // [H, Qf]
  const uint16_t* o_scale;
  uint16_t* residual;
  bool tiled;
};

// The GeGLU feed-forward on FP8 e4m3 weights with f32 per-output-channel scales (BASELINE
// configs[0]; the reference's decoder_feedforward epilogue, FOG/src/ops.rs:201-239, around three
// scaled projections, FOG/scripts/generate_references.py:265-274).
struct Ffn8Args {
  uint16_t* residual;
  const uint16_t* pre_rms;
  const uint8_t* up_w;      // [L, H] (tiled: up and gate interleaved, g4_pack_tiles (128, 64))
  const uint8_t* gate_w;    // [L, H] (row-major only)
  const uint8_t* down_w;    // [H, L]
  const float* up_s;        // [L]
  const float* gate_s;      // [L]
  const float* down_s;      // [H]
  const uint16_t* post_rms;
  const uint16_t* layer_scalar;
  bool tiled;
};

// TMA tensor maps of the weight matrices, encoded on the host once per (pointer, shape) and
// kept by the context (encoding costs microseconds; a map is 128 bytes). A whole model's maps
// (ten or so per layer) stay cached: the table grows as needed.
class TmapCache {
 public:
  // Row-major uint8 matrix [rows, cols] (fp8 codes, e4m3 scales), box {box_cols, box_rows}.
  cudaError_t u8(const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows, bool swizzle128,
                 CUtensorMap* out);
  // Row-major bf16 (or, half = true, f16) matrix [rows, cols], box {box_cols, box_rows}, 128-byte
  // swizzle (box_cols = 64): rows past the end read as zeros.
  cudaError_t bf16(const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                   CUtensorMap* out, bool half = false);
  // KV ring cache [ring, heads, dim] bf16 as a 3-D tensor (dim, head, slot), box {dim, 1, box_slots}:
  // one load brings box_slots rows of one head.
  cudaError_t kv(const void* base, uint64_t ring, uint32_t heads, uint32_t dim, uint32_t box_slots, CUtensorMap* out);

 private:
  struct KeyHash {
    size_t operator()(const std::pair<const void*, uint64_t>& k) const {
      return std::hash<const void*>()(k.first) ^ (std::hash<uint64_t>()(k.second) * 0x9E3779B97F4A7C15ull);
    }
  };
  std::unordered_map<std::pair<const void*, uint64_t>, CUtensorMap, KeyHash> entries_;
  const CUtensorMap* find(const void* base, uint64_t key) const;
  void put(const void* base, uint64_t key, const CUtensorMap& map);
};

struct LaunchEnv {
  int device;
  int sm_count;
  cudaStream_t stream;
  bool pdl;  // launch with programmatic stream serialization
  Scratch sc;
  TmapCache* maps;
  TpLink tp{0, 1, {}, nullptr, 0, kWaitLimitNs};  // tensor-parallel rank (world 1: the whole layer on this GPU)
};

cudaError_t prepare_proj_kernels();       // one-time attributes (dynamic shared memory)
bool proj_geometry_fits(int sm_count);    // the launch geometry on this many SMs meets the kernels' limits
cudaError_t prepare_attention_kernels();  // one-time attributes (clusters)
cudaError_t launch_qkv(const QkvArgs& a, const LaunchEnv& env);
cudaError_t launch_attention(const AttnArgs& a, const LaunchEnv& env);
cudaError_t launch_o(const OArgs& a, const LaunchEnv& env);
cudaError_t launch_ffn_nvfp4(const FfnArgs& a, const LaunchEnv& env);
cudaError_t launch_ffn_fp8(const Ffn8Args& a, const LaunchEnv& env);
// L2 hints for the first `first_units` units of every CTA of a following O / FP8 up-gate kernel
// on this env (unit-tiled weights only: an empty hint otherwise).
L2Hint l2_hint_o(const OArgs& a, int first_units, const LaunchEnv& env);
L2Hint l2_hint_ffn8_upgate(const Ffn8Args& a, int first_units, const LaunchEnv& env);
// The NVFP4 feed-forward on m = 2..64 tokens (g4_batch.cu): residual [m][H]; one GPU.
cudaError_t prepare_batch_kernels();
bool batch_geometry_fits(int sm_count);
size_t batch_words_count(int sm_count);  // split-K words of the batched kernels
cudaError_t launch_ffn_nvfp4_batch(const FfnArgs& a, int m, const LaunchEnv& env);
cudaError_t launch_ffn_fp8_batch(const Ffn8Args& a, int m, const LaunchEnv& env);
// The attention block's projections on m = 2..64 tokens (g4_batch_attn.cu), one GPU. QKV: x, q_out
// [m][...], kv_offset / rope_offset [m], token i's ring at slots [i ring_len, (i + 1) ring_len) of
// the caches. O: x (the attention rows) and residual [m][...].
cudaError_t prepare_batch_attn_kernels();
bool batch_attn_geometry_fits(int sm_count);
cudaError_t launch_qkv_batch(const QkvArgs& a, int m, const LaunchEnv& env);
cudaError_t launch_o_batch(const OArgs& a, int m, const LaunchEnv& env);
// final_norm_and_logits on m = 2..64 tokens (g4_logits_batch.cu): input [m][H], out [m][rows].
cudaError_t prepare_logits_batch_kernels();
cudaError_t launch_logits_batch(const uint16_t* input, const uint16_t* gamma, const uint16_t* weight, uint16_t* out,
                                int rows, int m, const LaunchEnv& env);
cudaError_t launch_full_qkv(const FullQkvArgs& a, const LaunchEnv& env);
cudaError_t launch_full_attention(const FullAttnArgs& a, const LaunchEnv& env);
cudaError_t launch_full_o(const FullOArgs& a, const LaunchEnv& env);
// The vocabulary ends (g4_vocab.cu): the embedding-row gather and the final norm + lm_head.
cudaError_t launch_embed(const uint16_t* table, const int32_t* offset, uint16_t* out, int vocab_rows,
                         const LaunchEnv& env);
cudaError_t launch_logits(const uint16_t* input, const uint16_t* gamma, const uint16_t* weight, uint16_t* out,
                          int rows, const LaunchEnv& env);

// The O op without a context: scratch laid out as [error word | kScratchHeadBytes][epoch
// counters][tile sums][split-K words] at env.sc, o_scratch_bytes() in total; the tensor map is encoded on the
// stack (env.maps is not used). Row-major weights, one rank (env.tp.world == 1) only.
size_t o_scratch_bytes();
cudaError_t launch_o_uncached(const OArgs& a, const LaunchEnv& env);

// Unit-tiled weight layout: rows grouped into tiles of `tile_rows`, each row cut into units of
// `unit_bytes`; block (t, u) holds the unit-u bytes of tile t's rows of src and then (when src2
// is given) of src2, contiguously; blocks are tile-major. With n = 1 or 2 sources:
// dst[(((t * units + u) * n + which) * tile_rows + r) * unit_bytes + b]
//   = src_which[(t * tile_rows + r) * row_bytes + u * unit_bytes + b].
cudaError_t launch_pack_tiles(const uint8_t* src, const uint8_t* src2, uint8_t* dst, int rows, int row_bytes,
                              int unit_bytes, int tile_rows, cudaStream_t stream);

}  // namespace g4
