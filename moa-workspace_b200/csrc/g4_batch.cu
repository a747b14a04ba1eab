// The GeGLU feed-forward for a batch of M = 2..64 tokens on sm_100a, NVFP4 or FP8 weights: the
// reference op (furiosa-opt-gemma4-12B/src/ops.rs:201-239, oracle generate_references.py:265-274
// and 358-413) applied to each of M residual rows, with the weights streamed from HBM once for all
// M tokens, on the token-batch engine (g4_batch.cuh).
//
//   batch_norm_kernel        h[m] = bf16(RMSNorm(residual[m]) * gamma_pre)           (M CTAs)
//   ffn_batch_upgate_kernel  act[m] = bf16(bf16(gelu_tanh(gate[m])) * up[m])          (one CTA per SM)
//   ffn_batch_down_kernel    the down projection's tile pieces, as split-K words     (one CTA per SM)
//   batch_finalize_kernel    residual[m] = bf16(bf16(residual[m] + RMSNorm_post(down[m])) * lambda)
//
// The weights arrive in the M = 1 kernels' layouts (row-major, or unit-tiled by g4_pack_tiles).
// Up/gate: the CTA holding a tile's first unit adds the other CTAs' pieces and applies GeGLU to
// the tile's 64 up and 64 gate rows. Down: every piece is published and the finalize kernel adds
// them per token in CTA order.
#include "g4_batch.cuh"

namespace g4 {
namespace {

// The weights' format: NVFP4 (FfnArgs: packed codes, block scales, reciprocal global scales) or
// FP8 (Ffn8Args: e4m3 codes, f32 per-row scales).
template <bool FP8>
using BatchArgs = std::conditional_t<FP8, Ffn8Args, FfnArgs>;

template <int MPAD, bool FP8>
struct BatchUpGateOp {
  using Shape = BatchShape<MPAD, FP8>;
  static constexpr int kUnitsPerTile = kH / kUnitK;  // 15
  static constexpr int kTiles = kL / 64;             // 64 up + 64 gate rows per tile
  static constexpr bool kF16 = true;                 // f16 weights x the scaled f16 h
  const BatchMaps* maps;
  BatchArgs<FP8> a;
  Scratch sc;
  int M;
  float g_up = 0.f, g_gate = 0.f;
  uint32_t tag = 0;

  __device__ void load_a(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if constexpr (FP8) {  // [K half][64 up rows | 64 gate rows] x 128 codes
      if (a.tiled) {
        tma_load_2d(stage, &maps->a, 0, (tile * kUnitsPerTile + kc) * 2 * kTileRows, bar, policy);
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tma_load_2d(stage + h * 16384, &maps->a, kc * kUnitK + h * 128, tile * 64, bar, policy);
          tma_load_2d(stage + h * 16384 + 8192, &maps->a2, kc * kUnitK + h * 128, tile * 64, bar, policy);
        }
      }
    } else {
      uint8_t* scl = stage + Shape::kABytes;
      if (a.tiled) {
        tma_load_2d(stage, &maps->a, 0, (tile * kUnitsPerTile + kc) * kTileRows, bar, policy);
        bulk_g2s(scl, a.up_scale + size_t(tile * kUnitsPerTile + kc) * Shape::kScaleBytes, Shape::kScaleBytes, bar,
                 policy);
      } else {
        tma_load_2d(stage, &maps->a, kc * 128, tile * 64, bar, policy);
        tma_load_2d(stage + 8192, &maps->a2, kc * 128, tile * 64, bar, policy);
        tma_load_2d(scl, &maps->s, kc * 16, tile * 64, bar, policy);
        tma_load_2d(scl + 1024, &maps->s2, kc * 16, tile * 64, bar, policy);
      }
    }
  }
  __device__ void load_b(uint8_t* dst, int kc, uint64_t* bar, uint64_t policy) const {
#pragma unroll
    for (int q = 0; q < 4; ++q) tma_load_2d(dst + q * Shape::kBColBytes, &maps->b, kc * kUnitK + 64 * q, 0, bar, policy);
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (!a.tiled) return;
    if constexpr (FP8) {
      prefetch_units(a.up_w, u0, u1, Shape::kABytes);
    } else {
      prefetch_units(a.up_packed, u0, u1, Shape::kABytes);
      prefetch_units(a.up_scale, u0, u1, Shape::kScaleBytes);
    }
  }
  __device__ void prologue() {
    if constexpr (!FP8) {
      g_up = *a.up_global;
      g_gate = *a.gate_global;
    }
    tag = batch_tag(sc, kTagUpGate);
  }
  // The projection's bf16 value: NVFP4 GloballyScaled(nn.Linear), bf16(bf16(h @ W.T) * g)
  // (generate_references.py:358-372); FP8 scaled_projection, bf16((h @ codes.T) * s_row) (:265-274).
  __device__ float project(float dot, int tile, int row) const {
    if constexpr (FP8) {
      const float s = row < 64 ? __ldg(a.up_s + tile * 64 + row) : __ldg(a.gate_s + tile * 64 + row - 64);
      return bf16_round(dot * s);
    } else {
      return bf16_round(bf16_round(dot) * (row < 64 ? g_up : g_gate));
    }
  }
  // Then the down input bf16(bf16(gelu_tanh(gate)) * up) (gemma4.py:197), 16 tokens at a time: the
  // gate rows leave their bf16 values in shared memory, all 128 threads apply GeGLU's gelu to them,
  // and the up rows form the products.
  __device__ void finish(BatchCtl&, uint8_t* xbuf, int tile, int row, uint32_t tsum, bool ok) {
    const SplitPiece sp = split_begin<MPAD>(tile, kUnitsPerTile, int64_t(kUnitsPerTile) * kTiles, row, M, tsum, tag,
                                            sc.batch_words, ok, sc.err);
    if (sp.publish) return;  // CTA-uniform for the tile: no barrier is skipped by part of the warps
    uint16_t* gel = reinterpret_cast<uint16_t*>(xbuf);  // [16 tokens][64]
#pragma unroll 1
    for (int c = 0; c < MPAD && c < M; c += 16) {
      float a[16];
      split_chunk(sp, c, M, row, tsum, ok, a);
#pragma unroll
      for (int j = 0; j < 16; ++j) a[j] *= c + j < M ? __ldcg(sc.batch_unscale + c + j) : 1.f;  // exact: 2^-k
      if (row >= 64) {
#pragma unroll
        for (int j = 0; j < 16; ++j) gel[j * 64 + row - 64] = f32_to_bf16(project(a[j], tile, row));
      }
      named_bar(kBEpiBarrier, 128);
#pragma unroll
      for (int q = 0; q < 8; ++q) {  // 1024 gate values over 128 threads
        const int e = q * 128 + row;
        gel[e] = f32_to_bf16(gelu_tanh(bf16_to_f32(gel[e])));
      }
      named_bar(kBEpiBarrier, 128);
      if (row < 64) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c + j < M) {
            const float up = project(a[j], tile, row);
            sc.act[size_t(c + j) * kL + tile * 64 + row] = f32_to_bf16(bf16_to_f32(gel[j * 64 + row]) * up);
          }
      }
      named_bar(kBEpiBarrier, 128);  // the exchange buffer is free for the next chunk
    }
  }
};

template <int MPAD, bool FP8>
struct BatchDownOp {
  using Shape = BatchShape<MPAD, FP8>;
  static constexpr int kUnitsPerTile = kL / kUnitK;  // 60
  static constexpr int kTiles = kH / kTileRows;      // 30
  static constexpr bool kF16 = false;                // bf16 weights x the bf16 GeGLU activation
  const BatchMaps* maps;
  BatchArgs<FP8> a;
  Scratch sc;
  int M;
  uint32_t tag = 0;

  __device__ void load_a(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if constexpr (FP8) {  // two K halves of 128 rows x 128 codes
      if (a.tiled) {
        tma_load_2d(stage, &maps->a, 0, (tile * kUnitsPerTile + kc) * 2 * kTileRows, bar, policy);
      } else {
        tma_load_2d(stage, &maps->a, kc * kUnitK, tile * kTileRows, bar, policy);
        tma_load_2d(stage + 16384, &maps->a, kc * kUnitK + 128, tile * kTileRows, bar, policy);
      }
    } else {
      uint8_t* scl = stage + Shape::kABytes;
      if (a.tiled) {
        tma_load_2d(stage, &maps->a, 0, (tile * kUnitsPerTile + kc) * kTileRows, bar, policy);
        bulk_g2s(scl, a.down_scale + size_t(tile * kUnitsPerTile + kc) * Shape::kScaleBytes, Shape::kScaleBytes, bar,
                 policy);
      } else {
        tma_load_2d(stage, &maps->a, kc * 128, tile * kTileRows, bar, policy);
        tma_load_2d(scl, &maps->s, kc * 16, tile * kTileRows, bar, policy);
      }
    }
  }
  __device__ void load_b(uint8_t* dst, int kc, uint64_t* bar, uint64_t policy) const {
#pragma unroll
    for (int q = 0; q < 4; ++q) tma_load_2d(dst + q * Shape::kBColBytes, &maps->b, kc * kUnitK + 64 * q, 0, bar, policy);
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (!a.tiled) return;
    if constexpr (FP8) {
      prefetch_units(a.down_w, u0, u1, Shape::kABytes);
    } else {
      prefetch_units(a.down_packed, u0, u1, Shape::kABytes);
      prefetch_units(a.down_scale, u0, u1, Shape::kScaleBytes);
    }
  }
  __device__ void prologue() { tag = batch_tag(sc, kTagDown); }
  // Every piece (at most two per CTA: the end of one tile and the start of the next) goes out as
  // epoch-tagged words in the CTA's slot (its piece ordinal); batch_finalize_kernel adds them.
  __device__ void finish(BatchCtl&, uint8_t*, int, int row, uint32_t tsum, bool ok) {
    publish_piece<MPAD>(sc, tag, piece_no, M, row, tsum, ok);
  }
  int piece_no = 0;
};

template <int MPAD, bool FP8>
__global__ void __launch_bounds__(kBThreads, 1) ffn_batch_upgate_kernel(const __grid_constant__ BatchMaps maps,
                                                                        BatchArgs<FP8> a, Scratch sc, int M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  BatchUpGateOp<MPAD, FP8> op{&maps, a, sc, M};
  batch_run<BatchShape<MPAD, FP8>>(op, smem, sc);
}

template <int MPAD, bool FP8>
__global__ void __launch_bounds__(kBThreads, 1) ffn_batch_down_kernel(const __grid_constant__ BatchMaps maps,
                                                                      BatchArgs<FP8> a, Scratch sc, int M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  BatchDownOp<MPAD, FP8> op{&maps, a, sc, M};
  batch_run<BatchShape<MPAD, FP8>>(op, smem, sc);
}

// The same ops on the term-operand engine (FP8 weights, up to kTermTokens tokens): `maps.b` maps
// the call's term rows instead of the activation rows.
template <int MT>
__global__ void __launch_bounds__(kTThreads, 1) ffn_term_upgate_kernel(const __grid_constant__ BatchMaps maps,
                                                                       Ffn8Args a, Scratch sc, int M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  BatchUpGateOp<kTermTokens, true> op{&maps, a, sc, M};
  batch_term_run<TermShape<MT>>(op, &maps.b, smem, sc);
}

template <int MT>
__global__ void __launch_bounds__(kTThreads, 1) ffn_term_down_kernel(const __grid_constant__ BatchMaps maps,
                                                                     Ffn8Args a, Scratch sc, int M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  BatchDownOp<kTermTokens, true> op{&maps, a, sc, M};
  batch_term_run<TermShape<MT>>(op, &maps.b, smem, sc);
}

// The weight maps of each format (row-major: the reference layout; tiled: g4_pack_tiles).
cudaError_t batch_maps(const FfnArgs& a, const LaunchEnv& env, BatchMaps& ug, BatchMaps& dn) {
  cudaError_t e;
  if (a.tiled) {
    if ((e = env.maps->u8(a.up_packed, 128, uint64_t(kL) / 64 * (kH / kUnitK) * kTileRows, 128, kTileRows, true,
                          &ug.a)))
      return e;
    return env.maps->u8(a.down_packed, 128, uint64_t(kH) / kTileRows * (kL / kUnitK) * kTileRows, 128, kTileRows,
                        true, &dn.a);
  }
  if ((e = env.maps->u8(a.up_packed, kH / 2, kL, 128, 64, true, &ug.a))) return e;
  if ((e = env.maps->u8(a.gate_packed, kH / 2, kL, 128, 64, true, &ug.a2))) return e;
  if ((e = env.maps->u8(a.up_scale, kH / 16, kL, 16, 64, false, &ug.s))) return e;
  if ((e = env.maps->u8(a.gate_scale, kH / 16, kL, 16, 64, false, &ug.s2))) return e;
  if ((e = env.maps->u8(a.down_packed, kL / 2, kH, 128, kTileRows, true, &dn.a))) return e;
  return env.maps->u8(a.down_scale, kL / 16, kH, 16, kTileRows, false, &dn.s);
}
cudaError_t batch_maps(const Ffn8Args& a, const LaunchEnv& env, BatchMaps& ug, BatchMaps& dn) {
  cudaError_t e;
  if (a.tiled) {  // one 256-row box per unit (both K halves), as the M = 1 kernels read them
    if ((e = env.maps->u8(a.up_w, 128, uint64_t(2 * kL) * (kH / 128), 128, 2 * kTileRows, true, &ug.a))) return e;
    return env.maps->u8(a.down_w, 128, uint64_t(kH) * (kL / 128), 128, 2 * kTileRows, true, &dn.a);
  }
  if ((e = env.maps->u8(a.up_w, kH, kL, 128, 64, true, &ug.a))) return e;
  if ((e = env.maps->u8(a.gate_w, kH, kL, 128, 64, true, &ug.a2))) return e;
  return env.maps->u8(a.down_w, kL, kH, 128, kTileRows, true, &dn.a);
}

template <int MPAD, bool FP8>
cudaError_t launch_batch_t(const BatchArgs<FP8>& a, int M, const LaunchEnv& env) {
  using Shape = BatchShape<MPAD, FP8>;
  using UG = BatchUpGateOp<MPAD, FP8>;
  BatchMaps ug{}, dn{};
  cudaError_t e;
  if ((e = batch_maps(a, env, ug, dn))) return e;
  if ((e = env.maps->bf16(env.sc.batch_h, kH, uint64_t(M), 64, MPAD, &ug.b, /*half=*/true))) return e;
  if ((e = env.maps->bf16(env.sc.act, kL, uint64_t(M), 64, MPAD, &dn.b))) return e;
  const int gu = env.sm_count < UG::kUnitsPerTile * UG::kTiles ? env.sm_count : UG::kUnitsPerTile * UG::kTiles;
  const int gd = env.sm_count;
  Scratch su = env.sc, sd = env.sc;
#ifdef G4_TRACE
  if (su.trace) su.trace += 11 * 4096;  // profiling builds: stamp rows of their own
  if (sd.trace) sd.trace += 12 * 4096;
#endif
  if ((e = launch_batch(batch_norm_kernel, M, 256, 0, env.pdl, env.stream,
                        static_cast<const uint16_t*>(a.residual), a.pre_rms, env.sc)))
    return e;
  if ((e = launch_batch(ffn_batch_upgate_kernel<MPAD, FP8>, gu, kBThreads, Shape::kSmemBytes, true, env.stream, ug, a,
                        su, M)))
    return e;
  if ((e = launch_batch(ffn_batch_down_kernel<MPAD, FP8>, gd, kBThreads, Shape::kSmemBytes, true, env.stream, dn, a,
                        sd, M)))
    return e;
  FinalizeArgs fa{a.residual, a.post_rms, a.layer_scalar, nullptr, nullptr, nullptr};
  if constexpr (FP8) {
    fa.down_scale = a.down_s;
  } else {
    fa.down_global = a.down_global;
  }
  return launch_batch(batch_finalize_kernel<kL / kUnitK, kTagDown>, M, kFinThreads, 0, true, env.stream, fa, env.sc, gd);
}

// The FP8 feed-forward on the term-operand engine: the input's term rows (RMSNorm, counting the
// call), up/gate, the GeGLU activation's term rows, down, the per-token finalize.
template <int MT>
cudaError_t launch_term_t(const Ffn8Args& a, int M, const LaunchEnv& env) {
  using Shape = TermShape<MT>;
  BatchMaps ug{}, dn{};
  cudaError_t e;
  if ((e = batch_maps(a, env, ug, dn))) return e;
  constexpr int kUgUnits = kH / kUnitK, kDnUnits = kL / kUnitK;
  if ((e = env.maps->u8(env.sc.batch_terms, 256, uint64_t(kUgUnits) * MT * kTerms, 128, MT * kTerms, true, &ug.b)))
    return e;
  if ((e = env.maps->u8(env.sc.batch_terms, 256, uint64_t(kDnUnits) * MT * kTerms, 128, MT * kTerms, true, &dn.b)))
    return e;
  using UG = BatchUpGateOp<kTermTokens, true>;
  const int gu = env.sm_count < UG::kUnitsPerTile * UG::kTiles ? env.sm_count : UG::kUnitsPerTile * UG::kTiles;
  const int gd = env.sm_count;
  if ((e = launch_batch(batch_terms_kernel<true>, MT, 256, 0, env.pdl, env.stream,
                        static_cast<const uint16_t*>(a.residual), kH, a.pre_rms, env.sc, M, true)))
    return e;
  if ((e = launch_batch(ffn_term_upgate_kernel<MT>, gu, kTThreads, Shape::kSmemBytes, true, env.stream, ug, a,
                        env.sc, M)))
    return e;
  if ((e = launch_batch(batch_terms_kernel<false>, MT, 256, 0, true, env.stream,
                        static_cast<const uint16_t*>(env.sc.act), kL, static_cast<const uint16_t*>(nullptr), env.sc,
                        M, false)))
    return e;
  if ((e = launch_batch(ffn_term_down_kernel<MT>, gd, kTThreads, Shape::kSmemBytes, true, env.stream, dn, a, env.sc,
                        M)))
    return e;
  const FinalizeArgs fa{a.residual, a.post_rms, a.layer_scalar, nullptr, a.down_s, nullptr};
  return launch_batch(batch_finalize_kernel<kL / kUnitK, kTagDown>, M, kFinThreads, 0, true, env.stream, fa, env.sc,
                      gd);
}

template <int MT>
cudaError_t prepare_term_t() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(ffn_term_upgate_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(TermShape<MT>::kSmemBytes))))
    return e;
  return cudaFuncSetAttribute(ffn_term_down_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(TermShape<MT>::kSmemBytes));
}

template <int MPAD, bool FP8>
cudaError_t prepare_batch_t() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(ffn_batch_upgate_kernel<MPAD, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(BatchShape<MPAD, FP8>::kSmemBytes))))
    return e;
  return cudaFuncSetAttribute(ffn_batch_down_kernel<MPAD, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(BatchShape<MPAD, FP8>::kSmemBytes));
}

template <bool FP8>
cudaError_t launch_batch_any(const BatchArgs<FP8>& a, int M, const LaunchEnv& env) {
  if (env.tp.world != 1) return cudaErrorNotSupported;  // the batched feed-forward runs on one GPU
  if (M < 2 || M > kBatchMax) return cudaErrorInvalidValue;
  if constexpr (FP8) {  // up to kTermTokens tokens: the term-operand engine
    if (M <= 4) return launch_term_t<4>(a, M, env);
    if (M <= 8) return launch_term_t<8>(a, M, env);
    if (M <= kTermTokens) return launch_term_t<16>(a, M, env);
  }
  switch ((M + 15) / 16) {
    case 1: return launch_batch_t<16, FP8>(a, M, env);
    case 2: return launch_batch_t<32, FP8>(a, M, env);
    case 3: return launch_batch_t<48, FP8>(a, M, env);
    default: return launch_batch_t<64, FP8>(a, M, env);
  }
}

}  // namespace

cudaError_t prepare_batch_kernels() {
  cudaError_t e;
  if ((e = prepare_batch_t<16, false>()) || (e = prepare_batch_t<32, false>()) || (e = prepare_batch_t<48, false>()) ||
      (e = prepare_batch_t<64, false>()))
    return e;
  if ((e = prepare_batch_t<16, true>()) || (e = prepare_batch_t<32, true>()) || (e = prepare_batch_t<48, true>()))
    return e;
  if ((e = prepare_term_t<4>()) || (e = prepare_term_t<8>()) || (e = prepare_term_t<16>()))
    return e;
  return prepare_batch_t<64, true>();
}

bool batch_geometry_fits(int sm_count) {
  // a down CTA's run lies within two tiles (its two piece slots) and a down tile spans at most
  // kMaxDownPieces CTAs (the finalize kernel's loads); an up/gate tile at most kMaxCtasPerGroup
  constexpr int kDownUpt = kL / kUnitK, kDownTiles = kH / kTileRows, kUgUpt = kH / kUnitK, kUgTiles = kL / 64;
  const int grid = sm_count;
  if (grid > 1024) return false;  // the finalize kernel's table of down CTAs
  if (int64_t(kDownUpt) * kDownTiles / grid + 1 > kDownUpt) return false;
  for (int t = 0; t < kDownTiles; ++t)
    if (cta_of_unit(int64_t(t) * kDownUpt + kDownUpt - 1, grid, int64_t(kDownUpt) * kDownTiles) -
            cta_of_unit(int64_t(t) * kDownUpt, grid, int64_t(kDownUpt) * kDownTiles) + 1 > kMaxDownPieces)
      return false;
  const int gu = grid < kUgUpt * kUgTiles ? grid : kUgUpt * kUgTiles;
  for (int t = 0; t < kUgTiles; ++t)
    if (cta_of_unit(int64_t(t) * kUgUpt + kUgUpt - 1, gu, int64_t(kUgUpt) * kUgTiles) -
            cta_of_unit(int64_t(t) * kUgUpt, gu, int64_t(kUgUpt) * kUgTiles) > kMaxCtasPerGroup)
      return false;
  return true;
}

// split-K words of the batched kernels: two piece slots per CTA
size_t batch_words_count(int sm_count) { return size_t(sm_count) * 2 * kBatchMax * kTileRows; }

cudaError_t launch_ffn_nvfp4_batch(const FfnArgs& a, int M, const LaunchEnv& env) {
  return launch_batch_any<false>(a, M, env);
}

cudaError_t launch_ffn_fp8_batch(const Ffn8Args& a, int M, const LaunchEnv& env) {
  return launch_batch_any<true>(a, M, env);
}

}  // namespace g4
