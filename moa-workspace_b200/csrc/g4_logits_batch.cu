// final_norm_and_logits for a batch of M = 2..64 tokens on sm_100a (reference: furiosa-opt-gemma4-12B/
// src/ops.rs:241-298, lm_head contraction src/device/shared/lm_head.rs:13-80), the 2 GB lm_head
// streamed from HBM once for all M tokens:
//
//   logits_norm_kernel    h[m] = bf16(RMSNorm(x[m]) * gamma)                             (M CTAs)
//   logits_batch_kernel   out[m][v] = bf16(tanh(bf16(h[m] . W[v]) / 30) * 30)            (one CTA per SM)
//
// The table is bf16, so the contraction runs on the tensor cores as it is: tcgen05.mma kind::f16
// with bf16 A (128 table rows x 16 K, from shared memory) and B (the M tokens' h rows, N = MPAD),
// f32 accumulation in tensor memory. Each CTA owns a contiguous run of 128-row tiles; per tile the
// producer streams 30 K slices of 128 (32 KB of table rows + the h rows' slice, 128-byte swizzle)
// through a ring of stages, the issuer accumulates the tile's 240 MMAs into one of two TMEM
// accumulators, and four epilogue warps apply the device op's epilogue (its f32 division, tanh and
// product, one bf16 cast) while the next tile accumulates. Only the f32 summation order differs
// from the single-token kernel (g4_vocab.cu).
#include "g4_gemv.cuh"
#include "g4_ops.cuh"

namespace g4 {
namespace {

constexpr float kSoftcap = 30.0f;
constexpr int kLThreads = 192;  // warp 0 producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kLMaxStages = 6;
constexpr int kLHalfK = 128;                  // K elements per stage
constexpr int kLHalves = kH / kLHalfK;        // 30 per tile
constexpr int kLABytes = kTileRows * kLHalfK * 2;  // 32 KB: two 64-column boxes of 128 rows

template <int MPAD>
struct LogitsShape {
  static constexpr int kBBoxBytes = MPAD * 128;  // one 64-column box of the h rows
  static constexpr int kStageBytes = kLABytes + 2 * kBBoxBytes;
  static constexpr int kFit = (227 * 1024 - 2048) / kStageBytes;
  static constexpr int kStages = kFit < kLMaxStages ? kFit : kLMaxStages;
  static constexpr uint32_t kTmemCols = 2 * MPAD <= 32 ? 32 : (2 * MPAD <= 64 ? 64 : 128);
  static constexpr size_t kSmemBytes = size_t(kStages) * kStageBytes + 1024 + 1024;
  static_assert(kStages >= 3 && kStageBytes % 1024 == 0, "pipeline");
};

struct LogitsCtl {
  uint64_t full[kLMaxStages], empty[kLMaxStages], done[2], tempty[2], drain;
  uint32_t tmem_base;
  uint32_t abort;
};

__global__ void __launch_bounds__(256) logits_norm_kernel(const uint16_t* x, const uint16_t* gamma, uint16_t* h) {
  __shared__ double red[8];
  const int m = blockIdx.x;
  pdl_wait_primary();
  pdl_launch_dependents();
  const uint16_t* row = x + size_t(m) * kH;
  double ss = 0.0;
  for (int i = threadIdx.x; i < kH; i += blockDim.x) {
    const double v = bf16_to_f32(__ldcg(row + i));
    ss += v * v;
  }
  const float inv = rms_inverse(block_sum_d(ss, red), kH);
  for (int i = threadIdx.x; i < kH; i += blockDim.x)
    h[size_t(m) * kH + i] = f32_to_bf16((bf16_to_f32(__ldcg(row + i)) * inv) * bf16_to_f32(gamma[i]));
}

template <int MPAD>
__global__ void __launch_bounds__(kLThreads, 1) logits_batch_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                    const __grid_constant__ CUtensorMap hmap,
                                                                    uint16_t* out, int rows, int M, Scratch sc) {
  using Shape = LogitsShape<MPAD>;
  constexpr int S = Shape::kStages;
  constexpr uint32_t kIdesc = umma_idesc_bf16(kTileRows, MPAD);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  LogitsCtl& ctl = *reinterpret_cast<LogitsCtl*>(smem + size_t(S) * Shape::kStageBytes);
  auto stage = [&](int s) { return smem + size_t(s) * Shape::kStageBytes; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles = rows / kTileRows;
  const int t0 = int(int64_t(blockIdx.x) * tiles / gridDim.x), t1 = int(int64_t(blockIdx.x + 1) * tiles / gridDim.x);
  const int n = (t1 - t0) * kLHalves;  // stages of this CTA
  volatile uint32_t* abort = &ctl.abort;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&ctl.full[i], 1);
      mbar_init(&ctl.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl.done[i], 1);
      mbar_init(&ctl.tempty[i], 4);
    }
    mbar_init(&ctl.drain, 1);
    ctl.abort = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 1) tmem_alloc(&ctl.tmem_base, Shape::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ctl.tmem_base;
  const uint64_t policy = l2_evict_first_policy();
  const int prefetch = n < S ? n : S;
  auto load_a = [&](int i, int s) {
    const int tile = t0 + i / kLHalves, k0 = (i % kLHalves) * kLHalfK;
    tma_load_2d(stage(s), &wmap, k0, tile * kTileRows, &ctl.full[s], policy);
    tma_load_2d(stage(s) + kLABytes / 2, &wmap, k0 + 64, tile * kTileRows, &ctl.full[s], policy);
  };
  auto load_b = [&](int i, int s) {
    const int k0 = (i % kLHalves) * kLHalfK;
    tma_load_2d(stage(s) + kLABytes, &hmap, k0, 0, &ctl.full[s], 0ull);
    tma_load_2d(stage(s) + kLABytes + Shape::kBBoxBytes, &hmap, k0 + 64, 0, &ctl.full[s], 0ull);
  };
  // the first stages' table rows before the wait on the norm kernel, their h rows after it
  if (tid < prefetch) {
    mbar_arrive_expect_tx(&ctl.full[tid], uint32_t(Shape::kStageBytes));
    load_a(tid, tid);
  }
  __syncwarp();
  pdl_wait_primary();
  pdl_launch_dependents();
  if (tid < prefetch) load_b(tid, tid);
  __syncwarp();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = prefetch;
      for (int i = prefetch; i < n; ++i) {
        const int s = i % S;
        if (!mbar_wait_or_abort(&ctl.empty[s], uint32_t(((i - S) / S) & 1), abort, sc.err)) break;
        mbar_arrive_expect_tx(&ctl.full[s], uint32_t(Shape::kStageBytes));
        load_a(i, s);
        load_b(i, s);
        issued = i + 1;
      }
      for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i) {  // every copy landed before exit
        const uint64_t w0 = globaltimer_ns();
        while (!mbar_try_wait(&ctl.full[i % S], uint32_t((i / S) & 1)))
          if (globaltimer_ns() - w0 > kWaitLimitNs) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < n && ok; ++i) {
        const int s = i % S, tl = i / kLHalves, h = i % kLHalves, acc = tl & 1;
        if (h == 0 && tl >= 2) ok = mbar_wait_or_abort(&ctl.tempty[acc], uint32_t(((tl - 2) >> 1) & 1), abort, sc.err);
        if (ok) ok = mbar_wait_or_abort(&ctl.full[s], uint32_t((i / S) & 1), abort, sc.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tbase + uint32_t(acc * MPAD);
        const uint32_t a0 = smem_u32(stage(s)), b0 = a0 + kLABytes;
#pragma unroll
        for (int j = 0; j < kLHalfK / 16; ++j) {  // K = 16 each: box j / 4, 32 bytes a step
          const uint32_t cb = j / 4, kk = j % 4;
          umma_bf16(d, umma_desc_sw128(a0 + cb * uint32_t(kLABytes / 2) + kk * 32u),
                    umma_desc_sw128(b0 + cb * uint32_t(Shape::kBBoxBytes) + kk * 32u), kIdesc,
                    uint32_t(h > 0 || j > 0));
        }
        umma_commit(&ctl.empty[s]);
        if (h == kLHalves - 1) umma_commit(&ctl.done[acc]);
      }
      umma_commit(&ctl.drain);  // nothing of ours may still run when TMEM is released
      const uint64_t w0 = globaltimer_ns();
      while (!mbar_try_wait(&ctl.drain, 0))
        if (globaltimer_ns() - w0 > kWaitLimitNs) break;
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = warp & 3, row = quarter * 32 + lane;
    const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
    bool ok = true;
    for (int tl = 0; tl < t1 - t0; ++tl) {
      const int acc = tl & 1;
      if (ok) ok = mbar_wait_or_abort(&ctl.done[acc], uint32_t((tl >> 1) & 1), abort, sc.err);
      tc_fence_after();
      const size_t v = size_t(t0 + tl) * kTileRows + row;
#pragma unroll
      for (int c = 0; c < MPAD; c += 16) {
        if (c >= M) break;
        float a[16];
        if (ok) {
          tmem_ld16(tbase + lane_addr + uint32_t(acc * MPAD + c), a);
          tmem_ld_wait();
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (c + j >= M) break;
          const float logit = ok ? bf16_round(a[j]) : __uint_as_float(0x7fc00000u);
          out[size_t(c + j) * rows + v] = f32_to_bf16(tanhf(logit / kSoftcap) * kSoftcap);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl.tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, Shape::kTmemCols);
  }
}

template <int MPAD>
cudaError_t launch_t(const uint16_t* input, const uint16_t* gamma, const uint16_t* weight, uint16_t* out, int rows,
                     int M, const LaunchEnv& env) {
  CUtensorMap wmap, hmap;
  cudaError_t e;
  if ((e = env.maps->bf16(weight, kH, uint64_t(rows), 64, kTileRows, &wmap))) return e;
  if ((e = env.maps->bf16(env.sc.batch_h, kH, uint64_t(M), 64, MPAD, &hmap))) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M);
  cfg.blockDim = dim3(256);
  cfg.stream = env.stream;
  attr[0].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if ((e = cudaLaunchKernelEx(&cfg, logits_norm_kernel, input, gamma, env.sc.batch_h))) return e;
  const int tiles = rows / kTileRows;
  cfg.gridDim = dim3(tiles < env.sm_count ? tiles : env.sm_count);
  cfg.blockDim = dim3(kLThreads);
  cfg.dynamicSmemBytes = LogitsShape<MPAD>::kSmemBytes;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  return cudaLaunchKernelEx(&cfg, logits_batch_kernel<MPAD>, wmap, hmap, out, rows, M, env.sc);
}

template <int MPAD>
cudaError_t prepare_t() {
  return cudaFuncSetAttribute(logits_batch_kernel<MPAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(LogitsShape<MPAD>::kSmemBytes));
}

}  // namespace

cudaError_t prepare_logits_batch_kernels() {
  cudaError_t e;
  if ((e = prepare_t<16>()) || (e = prepare_t<32>()) || (e = prepare_t<48>())) return e;
  return prepare_t<64>();
}

cudaError_t launch_logits_batch(const uint16_t* input, const uint16_t* gamma, const uint16_t* weight, uint16_t* out,
                                int rows, int M, const LaunchEnv& env) {
  if (M < 2 || M > kBatchMax) return cudaErrorInvalidValue;
  if (rows <= 0 || rows % kTileRows != 0) {  // whole tiles only: token by token on the single-token kernel
    for (int m = 0; m < M; ++m) {
      cudaError_t e = launch_logits(input + size_t(m) * kH, gamma, weight, out + size_t(m) * rows, rows, env);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  switch ((M + 15) / 16) {
    case 1: return launch_t<16>(input, gamma, weight, out, rows, M, env);
    case 2: return launch_t<32>(input, gamma, weight, out, rows, M, env);
    case 3: return launch_t<48>(input, gamma, weight, out, rows, M, env);
    default: return launch_t<64>(input, gamma, weight, out, rows, M, env);
  }
}

}  // namespace g4
