// The attention block of a decode step for a batch of M = 2..64 sequences on sm_100a: the reference
// ops sliding_project_qkv and sliding_attention_output (furiosa-opt-gemma4-12B/src/ops.rs:37-76,
// 130-146; oracle generate_references.py:321-334, 353-355) applied to each of M tokens, each token
// with its own ring cache and position, the FP8 weights streamed from HBM once for all M tokens on
// the token-batch engine (g4_batch.cuh).
//
//   batch_norm_kernel           h[m] = bf16(RMSNorm(x[m]) * gamma_in)                  (M CTAs)
//   qkv_batch_kernel            q | k | v projections' tile pieces, as split-K words     (one CTA per SM)
//   qkv_batch_finalize_kernel   per (head, token): the pieces added in CTA order, the row scale,
//                               the per-head RMSNorm, RoPE at the token's row, the q_out / ring
//                               slot store                                               (32 x M CTAs)
//   o_batch_kernel              the O projection's tile pieces                           (one CTA per SM)
//   batch_finalize_kernel       residual[m] = bf16(residual[m] + RMSNorm_post(O x[m]))   (M CTAs)
//
// Between the two, the attention itself runs per sequence (attention_kernel with one grid row per
// sequence, g4_attention.cu). The arithmetic per token is the single-token kernels' (g4_proj.cu):
// e4m3 codes are exact in f16 and bf16, so the tensor cores form every product exactly and only
// the f32 summation order differs from the reference's f32 contraction.
#include "g4_batch.cuh"

namespace g4 {
namespace {

constexpr int kQkvRows = kQs + 2 * kPs;             // q | k | v = 8192
constexpr int kQkvHeads = kQkvRows / kDs;               // 16 q + 8 k + 8 v heads
constexpr int kQkvUpt = kH / kUnitK;                    // 15 units per tile
constexpr int kQkvTiles = kQkvRows / kTileRows;         // 64
constexpr int kOUpt = kQs / kUnitK;                     // 16
constexpr int kOTiles = kH / kTileRows;                 // 30
constexpr int kQTiles = kQs / kTileRows, kKTiles = kPs / kTileRows;

// The three projection matrices (q, k, v: BatchMaps a, a2, s) of one unit: two K halves of 128
// rows x 128 e4m3 codes, row-major (two boxes) or unit-tiled (one 256-row box), as the
// single-token QKV kernel reads them.
template <int MPAD>
struct BatchQkvOp {
  using Shape = BatchShape<MPAD, true>;
  static constexpr int kUnitsPerTile = kQkvUpt;
  static constexpr int kTiles = kQkvTiles;
  static constexpr bool kF16 = true;  // f16 weights x the scaled f16 h
  const BatchMaps* maps;
  QkvArgs a;
  Scratch sc;
  int M;
  uint32_t tag = 0;
  int piece_no = 0;

  __device__ void load_a(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    const CUtensorMap* m = tile < kQTiles ? &maps->a : (tile < kQTiles + kKTiles ? &maps->a2 : &maps->s);
    const int t = tile < kQTiles ? tile : (tile < kQTiles + kKTiles ? tile - kQTiles : tile - kQTiles - kKTiles);
    if (a.tiled) {
      tma_load_2d(stage, m, 0, (t * kUnitsPerTile + kc) * 2 * kTileRows, bar, policy);
    } else {
      tma_load_2d(stage, m, kc * kUnitK, t * kTileRows, bar, policy);
      tma_load_2d(stage + 16384, m, kc * kUnitK + 128, t * kTileRows, bar, policy);
    }
  }
  __device__ void load_b(uint8_t* dst, int kc, uint64_t* bar, uint64_t policy) const {
#pragma unroll
    for (int q = 0; q < 4; ++q) tma_load_2d(dst + q * Shape::kBColBytes, &maps->b, kc * kUnitK + 64 * q, 0, bar, policy);
  }
  // units [u0, u1) of the fused q | k | v order into L2 (unit-tiled weights only)
  __device__ void prefetch_l2(int u0, int u1) const {
    if (!a.tiled) return;
    constexpr int kQU = kQTiles * kUnitsPerTile, kKU = kKTiles * kUnitsPerTile;
    constexpr uint32_t kB = Shape::kABytes;
    prefetch_units(a.q_weight, u0, u1 < kQU ? u1 : kQU, kB);
    prefetch_units(a.k_weight, (u0 > kQU ? u0 : kQU) - kQU, (u1 < kQU + kKU ? u1 : kQU + kKU) - kQU, kB);
    prefetch_units(a.v_weight, (u0 > kQU + kKU ? u0 : kQU + kKU) - kQU - kKU, u1 - kQU - kKU, kB);
  }
  __device__ void prologue() { tag = batch_tag(sc, kTagQkv); }
  __device__ void finish(BatchCtl&, uint8_t*, int, int row, uint32_t tsum, bool ok) {
    publish_piece<MPAD>(sc, tag, piece_no, M, row, tsum, ok);
  }
};

// The O projection [H, Qs] of the attention rows [M, Qs] (bf16 weights x the bf16 attention output).
template <int MPAD>
struct BatchOOp {
  using Shape = BatchShape<MPAD, true>;
  static constexpr int kUnitsPerTile = kOUpt;
  static constexpr int kTiles = kOTiles;
  static constexpr bool kF16 = false;
  const BatchMaps* maps;
  OArgs a;
  Scratch sc;
  int M;
  uint32_t tag = 0;
  int piece_no = 0;

  __device__ void load_a(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {
      tma_load_2d(stage, &maps->a, 0, (tile * kUnitsPerTile + kc) * 2 * kTileRows, bar, policy);
    } else {
      tma_load_2d(stage, &maps->a, kc * kUnitK, tile * kTileRows, bar, policy);
      tma_load_2d(stage + 16384, &maps->a, kc * kUnitK + 128, tile * kTileRows, bar, policy);
    }
  }
  __device__ void load_b(uint8_t* dst, int kc, uint64_t* bar, uint64_t policy) const {
#pragma unroll
    for (int q = 0; q < 4; ++q) tma_load_2d(dst + q * Shape::kBColBytes, &maps->b, kc * kUnitK + 64 * q, 0, bar, policy);
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (a.tiled) prefetch_units(a.o_weight, u0, u1, Shape::kABytes);
  }
  __device__ void prologue() { tag = batch_tag(sc, kTagO); }
  __device__ void finish(BatchCtl&, uint8_t*, int, int row, uint32_t tsum, bool ok) {
    publish_piece<MPAD>(sc, tag, piece_no, M, row, tsum, ok);
  }
};

template <int MPAD>
__global__ void __launch_bounds__(kBThreads, 1) qkv_batch_kernel(const __grid_constant__ BatchMaps maps, QkvArgs a,
                                                                 Scratch sc, int M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  BatchQkvOp<MPAD> op{&maps, a, sc, M};
  batch_run<BatchShape<MPAD, true>>(op, smem, sc);
}

template <int MPAD>
__global__ void __launch_bounds__(kBThreads, 1) o_batch_kernel(const __grid_constant__ BatchMaps maps, OArgs a,
                                                               Scratch sc, int M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  BatchOOp<MPAD> op{&maps, a, sc, M};
  batch_run<BatchShape<MPAD, true>>(op, smem, sc);
}

// The same projections on the term-operand engine (up to kTermTokens tokens; `maps.b` maps the
// call's term rows).
template <int MT>
__global__ void __launch_bounds__(kTThreads, 1) qkv_term_kernel(const __grid_constant__ BatchMaps maps, QkvArgs a,
                                                                Scratch sc, int M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  BatchQkvOp<kTermTokens> op{&maps, a, sc, M};
  batch_term_run<TermShape<MT>>(op, &maps.b, smem, sc);
}

template <int MT>
__global__ void __launch_bounds__(kTThreads, 1) o_term_kernel(const __grid_constant__ BatchMaps maps, OArgs a,
                                                              Scratch sc, int M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  BatchOOp<kTermTokens> op{&maps, a, sc, M};
  batch_term_run<TermShape<MT>>(op, &maps.b, smem, sc);
}

// Per (head, token), 256 threads (thread e: element e of the head, row e % 128 of tile
// 2 head + e / 128): the tile's pieces added in CTA order, times the token's 2^-k (exact), the
// row scale (scaled_projection: bf16((x @ codes.T) * scale), generate_references.py:265-274), the
// head's RMSNorm (q and k with their gamma, v without; gemma4.py:83-89), RoPE for q and k in the
// half-swap form with the low half of `sin` pre-negated by the caller (out[i] = bf16(bf16(n[i]
// cos[i]) + bf16(n[i ^ 128] sin'[i]))), then the store: q_out[m], or slot kv_offset[m] of token
// m's ring. A bad offset skips the token's stores and raises its bit in the error word, as the
// single-token op does.
__global__ void __launch_bounds__(kDs) qkv_batch_finalize_kernel(QkvArgs a, Scratch sc, int grid) {
  constexpr int64_t kTotal = int64_t(kQkvUpt) * kQkvTiles;
  __shared__ double red[kDs / 32];
  __shared__ float nrm[kDs];
  __shared__ __align__(16) uint16_t out[kDs];
  const int head = blockIdx.x, m = blockIdx.y, e = threadIdx.x;
  const int tile = 2 * head + e / kTileRows, row = e % kTileRows, r = head * kDs + e;
  const bool is_q = head < kQs / kDs, is_k = !is_q && head < (kQs + kPs) / kDs;
  // static operands and the token's offsets (written before the op's first kernel) before the wait
  const float scale = bf16_to_f32(is_q ? a.q_scale[r] : (is_k ? a.k_scale[r - kQs] : a.v_scale[r - kQs - kPs]));
  const float gamma = is_q ? bf16_to_f32(a.q_rms[e]) : (is_k ? bf16_to_f32(a.k_rms[e]) : 1.0f);
  const int kv = __ldg(a.kv_offset + m), rope = __ldg(a.rope_offset + m);
  const bool kv_ok = kv >= 0 && kv % (kPs * 2) == 0 && kv / (kPs * 2) < a.ring_len;
  const bool rope_ok = rope >= 0 && rope % (kDs * 2) == 0 && rope / (kDs * 2) < a.rope_rows;
  float cs = 0.f, sn = 0.f;
  if (rope_ok && (is_q || is_k)) {
    cs = bf16_to_f32(a.cos[size_t(rope / 2) + e]);
    sn = bf16_to_f32(a.sin[size_t(rope / 2) + e]);
  }
  const int first = cta_of_unit(int64_t(tile) * kQkvUpt, grid, kTotal);
  const int span = cta_of_unit(int64_t(tile) * kQkvUpt + kQkvUpt - 1, grid, kTotal) - first + 1;
  pdl_wait_primary();
  pdl_launch_dependents();
  const uint32_t tag = batch_tag(sc, kTagQkv);
  unsigned long long w[kMaxDownPieces];
#pragma unroll
  for (int k = 0; k < kMaxDownPieces; ++k) {  // every piece in flight at once
    w[k] = 0ull;
    const int c = first + k;
    if (k < span) {
      const int piece = run_first_tile(c, grid, kTotal, kQkvUpt) < tile ? 1 : 0;
      w[k] = __ldcg(sc.batch_words + ((size_t(c) * 2 + piece) * kBatchMax + m) * kTileRows + row);
    }
  }
  float acc = 0.f;  // the pieces in CTA order
#pragma unroll
  for (int k = 0; k < kMaxDownPieces; ++k) {
    if (k >= span) break;
    if (uint32_t(w[k] >> 32) != tag) {
      atomicOr(sc.err, kErrInternal);
      acc = __uint_as_float(0x7fc00000u);
    }
    acc += __uint_as_float(uint32_t(w[k]));
  }
  acc *= __ldcg(sc.batch_unscale + m);  // exact: 2^-k of the token's f16 activation
  const float y = bf16_round(acc * scale);
  const float inv = rms_inverse(block_sum_d(double(y) * double(y), red), kDs);
  if (!kv_ok || !rope_ok) {
    if (e == 0 && head == 0) atomicOr(sc.err, (kv_ok ? 0u : kErrKvOffset) | (rope_ok ? 0u : kErrRopeOffset));
    return;
  }
  const float sv = y * inv;
  const float n = (is_q || is_k) ? bf16_round(sv * gamma) : bf16_round(sv);
  nrm[e] = n;
  __syncthreads();
  out[e] = (is_q || is_k) ? f32_to_bf16(bf16_round(n * cs) + bf16_round(nrm[e ^ 128] * sn)) : f32_to_bf16(n);
  __syncthreads();
  if (e < kDs * 2 / 16) {  // 16-byte stores
    uint16_t* dst;
    const size_t ring0 = (size_t(m) * a.ring_len + size_t(kv / (kPs * 2))) * kPs;  // token m's slot
    if (is_q)
      dst = a.q_out + size_t(m) * kQs + head * kDs;
    else if (is_k)
      dst = a.k_cache + ring0 + (head - kQs / kDs) * kDs;
    else
      dst = a.v_cache + ring0 + (head - (kQs + kPs) / kDs) * kDs;
    reinterpret_cast<uint4*>(dst)[e] = reinterpret_cast<const uint4*>(out)[e];
  }
}

// A unit-tiled or row-major FP8 matrix of `rows` x `k` codes as the batched kernels read it: one
// 256-row box per unit (tiled), or 128 x 128 boxes.
cudaError_t fp8_map(const LaunchEnv& env, const void* w, bool tiled, int rows, int k, CUtensorMap* out) {
  return env.maps->u8(w, tiled ? 128 : uint64_t(k), tiled ? uint64_t(rows) * (k / 128) : uint64_t(rows), 128,
                      tiled ? 2 * kTileRows : kTileRows, true, out);
}

template <int MPAD>
cudaError_t launch_qkv_batch_t(const QkvArgs& a, int M, const LaunchEnv& env) {
  using Shape = BatchShape<MPAD, true>;
  BatchMaps mp{};
  cudaError_t e;
  if ((e = fp8_map(env, a.q_weight, a.tiled, kQs, kH, &mp.a))) return e;
  if ((e = fp8_map(env, a.k_weight, a.tiled, kPs, kH, &mp.a2))) return e;
  if ((e = fp8_map(env, a.v_weight, a.tiled, kPs, kH, &mp.s))) return e;
  if ((e = env.maps->bf16(env.sc.batch_h, kH, uint64_t(M), 64, MPAD, &mp.b, /*half=*/true))) return e;
  const int grid = env.sm_count;
  if ((e = launch_batch(batch_norm_kernel, M, 256, 0, env.pdl, env.stream, a.x, a.input_rms, env.sc))) return e;
  if ((e = launch_batch(qkv_batch_kernel<MPAD>, grid, kBThreads, Shape::kSmemBytes, true, env.stream, mp, a, env.sc,
                        M)))
    return e;
  return launch_batch(qkv_batch_finalize_kernel, dim3(kQkvHeads, M), kDs, 0, true, env.stream, a, env.sc, grid);
}

template <int MPAD>
cudaError_t launch_o_batch_t(const OArgs& a, int M, const LaunchEnv& env) {
  using Shape = BatchShape<MPAD, true>;
  BatchMaps mp{};
  cudaError_t e;
  if ((e = fp8_map(env, a.o_weight, a.tiled, kH, kQs, &mp.a))) return e;
  if ((e = env.maps->bf16(a.x, kQs, uint64_t(M), 64, MPAD, &mp.b))) return e;
  const int grid = env.sm_count;
  if ((e = launch_batch(o_batch_kernel<MPAD>, grid, kBThreads, Shape::kSmemBytes, env.pdl, env.stream, mp, a, env.sc,
                        M)))
    return e;
  const FinalizeArgs fa{a.residual, a.post_rms, nullptr, nullptr, nullptr, a.o_scale};
  return launch_batch(batch_finalize_kernel<kOUpt, kTagO>, M, kFinThreads, 0, true, env.stream, fa, env.sc, grid);
}

template <int MT>
cudaError_t launch_qkv_term_t(const QkvArgs& a, int M, const LaunchEnv& env) {
  BatchMaps mp{};
  cudaError_t e;
  if ((e = fp8_map(env, a.q_weight, a.tiled, kQs, kH, &mp.a))) return e;
  if ((e = fp8_map(env, a.k_weight, a.tiled, kPs, kH, &mp.a2))) return e;
  if ((e = fp8_map(env, a.v_weight, a.tiled, kPs, kH, &mp.s))) return e;
  if ((e = env.maps->u8(env.sc.batch_terms, 256, uint64_t(kQkvUpt) * MT * kTerms, 128, MT * kTerms, true, &mp.b)))
    return e;
  const int grid = env.sm_count;
  if ((e = launch_batch(batch_terms_kernel<true>, MT, 256, 0, env.pdl, env.stream, a.x, kH, a.input_rms, env.sc, M,
                        true)))
    return e;
  if ((e = launch_batch(qkv_term_kernel<MT>, grid, kTThreads, TermShape<MT>::kSmemBytes, true, env.stream, mp, a,
                        env.sc, M)))
    return e;
  return launch_batch(qkv_batch_finalize_kernel, dim3(kQkvHeads, M), kDs, 0, true, env.stream, a, env.sc, grid);
}

template <int MT>
cudaError_t launch_o_term_t(const OArgs& a, int M, const LaunchEnv& env) {
  BatchMaps mp{};
  cudaError_t e;
  if ((e = fp8_map(env, a.o_weight, a.tiled, kH, kQs, &mp.a))) return e;
  if ((e = env.maps->u8(env.sc.batch_terms, 256, uint64_t(kOUpt) * MT * kTerms, 128, MT * kTerms, true, &mp.b)))
    return e;
  const int grid = env.sm_count;
  if ((e = launch_batch(batch_terms_kernel<false>, MT, 256, 0, env.pdl, env.stream, a.x, kQs,
                        static_cast<const uint16_t*>(nullptr), env.sc, M, false)))
    return e;
  if ((e = launch_batch(o_term_kernel<MT>, grid, kTThreads, TermShape<MT>::kSmemBytes, true, env.stream, mp, a, env.sc,
                        M)))
    return e;
  const FinalizeArgs fa{a.residual, a.post_rms, nullptr, nullptr, nullptr, a.o_scale};
  return launch_batch(batch_finalize_kernel<kOUpt, kTagO>, M, kFinThreads, 0, true, env.stream, fa, env.sc, grid);
}

template <int MT>
cudaError_t prepare_term_t() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(qkv_term_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(TermShape<MT>::kSmemBytes))))
    return e;
  return cudaFuncSetAttribute(o_term_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(TermShape<MT>::kSmemBytes));
}

template <int MPAD>
cudaError_t prepare_t() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(qkv_batch_kernel<MPAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(BatchShape<MPAD, true>::kSmemBytes))))
    return e;
  return cudaFuncSetAttribute(o_batch_kernel<MPAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(BatchShape<MPAD, true>::kSmemBytes));
}

// A projection of `tiles` x `upt` units split over `grid` CTAs as batch_run splits it: every CTA's
// run within two tiles (its two piece slots) and every tile within kMaxDownPieces CTAs (the
// finalize kernels' loads).
bool split_fits(int grid, int upt, int tiles) {
  const int64_t total = int64_t(upt) * tiles;
  if (grid < 1 || grid > 1024 || total / grid + 1 > upt) return false;
  for (int t = 0; t < tiles; ++t)
    if (cta_of_unit(int64_t(t) * upt + upt - 1, grid, total) - cta_of_unit(int64_t(t) * upt, grid, total) + 1 >
        kMaxDownPieces)
      return false;
  return true;
}

}  // namespace

cudaError_t prepare_batch_attn_kernels() {
  cudaError_t e;
  if ((e = prepare_t<16>()) || (e = prepare_t<32>()) || (e = prepare_t<48>()) || (e = prepare_t<64>())) return e;
  if ((e = prepare_term_t<4>()) || (e = prepare_term_t<8>())) return e;
  return prepare_term_t<16>();
}

bool batch_attn_geometry_fits(int sm_count) {
  return split_fits(sm_count, kQkvUpt, kQkvTiles) && split_fits(sm_count, kOUpt, kOTiles);
}

cudaError_t launch_qkv_batch(const QkvArgs& a, int M, const LaunchEnv& env) {
  if (env.tp.world != 1) return cudaErrorNotSupported;  // the batched ops run on one GPU
  if (M < 2 || M > kBatchMax) return cudaErrorInvalidValue;
  if (M <= 4) return launch_qkv_term_t<4>(a, M, env);  // up to kTermTokens: the term-operand engine
  if (M <= 8) return launch_qkv_term_t<8>(a, M, env);
  if (M <= kTermTokens) return launch_qkv_term_t<16>(a, M, env);
  switch ((M + 15) / 16) {
    case 1: return launch_qkv_batch_t<16>(a, M, env);
    case 2: return launch_qkv_batch_t<32>(a, M, env);
    case 3: return launch_qkv_batch_t<48>(a, M, env);
    default: return launch_qkv_batch_t<64>(a, M, env);
  }
}

cudaError_t launch_o_batch(const OArgs& a, int M, const LaunchEnv& env) {
  if (env.tp.world != 1) return cudaErrorNotSupported;
  if (M < 2 || M > kBatchMax) return cudaErrorInvalidValue;
  if (M <= 4) return launch_o_term_t<4>(a, M, env);  // up to kTermTokens: the term-operand engine
  if (M <= 8) return launch_o_term_t<8>(a, M, env);
  if (M <= kTermTokens) return launch_o_term_t<16>(a, M, env);
  switch ((M + 15) / 16) {
    case 1: return launch_o_batch_t<16>(a, M, env);
    case 2: return launch_o_batch_t<32>(a, M, env);
    case 3: return launch_o_batch_t<48>(a, M, env);
    default: return launch_o_batch_t<64>(a, M, env);
  }
}

}  // namespace g4
