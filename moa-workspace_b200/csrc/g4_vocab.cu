// The vocabulary ends of the decoder on sm_100a:
//   - embed_token            (reference: furiosa-opt-gemma4-12B/src/ops.rs:8-35)
//   - final_norm_and_logits  (ops.rs:241-298, lm_head contraction src/device/shared/lm_head.rs:13-80)
//
// embed_token: out = bf16(f32(table[row]) * EMBED_SCALE), the row addressed by a device-resident
// byte offset (token * H * 2), EMBED_SCALE = 61.967734 in f32 (src/lib.rs:23; the device op scales
// in f32 before its single bf16 cast).
//
// final_norm_and_logits: h = RMSNorm_gamma(input) (bf16, gemma4.py:83-89); logit = bf16(h . W[v])
// with an f32 contraction; out[v] = bf16(tanh(f32(logit) / 30) * 30) (the device op's f32
// division, tanh and product, one bf16 cast; LOGIT_SOFTCAP = 30, src/lib.rs:24).
//
// The contraction is a GEMV over bf16 rows (2 bytes per element, 2 FLOP each: far below the tensor
// cores' ridge point), bound by HBM: each warp streams whole rows with 16-byte loads of the read-only
// path, all of a row's loads in flight before the first use (lane l owns 16-byte chunks l, l + 32,
// ... of every row), the normalised activation read from shared memory as bf16.
#include "g4_ops.cuh"

namespace g4 {
namespace {

constexpr float kLogitSoftcap = 30.0f;
constexpr int kVocabThreads = 256;
constexpr int kChunksPerRow = kH * 2 / 16;             // 480 16-byte chunks per row
constexpr int kChunksPerLane = kChunksPerRow / 32;     // 15
static_assert(kChunksPerRow % 32 == 0, "whole chunks per lane");

__global__ void __launch_bounds__(kVocabThreads) embed_kernel(const uint16_t* __restrict__ table,
                                                              const int32_t* __restrict__ offset, uint16_t* out,
                                                              int vocab_rows, Scratch sc) {
  pdl_wait_primary();
  const int off = *offset;
  const bool ok = off >= 0 && off % (kH * 2) == 0 && off / (kH * 2) < vocab_rows;
  if (!ok) {
    if (threadIdx.x == 0) atomicOr(sc.err, kErrTokenOffset);
    return;
  }
  embed_row(table + size_t(off / (kH * 2)) * kH, out);
  pdl_launch_dependents();
}

// f32 products of 8 bf16 weights (a 16-byte chunk) with 8 bf16 activations (4 packed pairs),
// added to acc in element order.
__device__ __forceinline__ float dot8(const uint4& w, const uint32_t (&x)[4], float acc) {
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc = fmaf(__uint_as_float(ww[i] << 16), __uint_as_float(x[i] << 16), acc);
    acc = fmaf(__uint_as_float(ww[i] & 0xffff0000u), __uint_as_float(x[i] & 0xffff0000u), acc);
  }
  return acc;
}

__global__ void __launch_bounds__(kVocabThreads, 2) logits_kernel(const uint16_t* __restrict__ input,
                                                                  const uint16_t* __restrict__ gamma,
                                                                  const uint16_t* __restrict__ weight,
                                                                  uint16_t* out, int rows) {
  __shared__ double red[kVocabThreads / 32];
  __shared__ __align__(16) uint16_t h[kH];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = gridDim.x * (kVocabThreads / 32);
  const int gw = blockIdx.x * (kVocabThreads / 32) + warp;
  // this warp's contiguous run of rows; the first row's loads go out before the dependency wait
  const int r0 = int(int64_t(gw) * rows / warps), r1 = int(int64_t(gw + 1) * rows / warps);
  const uint4* wrow = reinterpret_cast<const uint4*>(weight);
  uint4 wv[kChunksPerLane];
  if (r0 < r1) {
#pragma unroll
    for (int i = 0; i < kChunksPerLane; ++i) wv[i] = __ldg(wrow + size_t(r0) * kChunksPerRow + lane + 32 * i);
  }
  pdl_wait_primary();
  pdl_launch_dependents();
  // RMSNorm of the input (every CTA: 7.5 KB from L2), the sum of squares exact in f64
  double ss = 0.0;
  for (int i = threadIdx.x; i < kH; i += kVocabThreads) {
    const double v = bf16_to_f32(__ldcg(input + i));
    ss += v * v;
  }
  const float inv = rms_inverse(block_sum_d(ss, red), kH);
  for (int i = threadIdx.x; i < kH; i += kVocabThreads)
    h[i] = f32_to_bf16((bf16_to_f32(__ldcg(input + i)) * inv) * bf16_to_f32(gamma[i]));
  __syncthreads();
  const uint4* hx = reinterpret_cast<const uint4*>(h);
  for (int r = r0; r < r1; ++r) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < kChunksPerLane; ++i) {
      const uint4 x = hx[lane + 32 * i];  // consecutive lanes, consecutive 16 bytes: no bank conflict
      const uint32_t xv[4] = {x.x, x.y, x.z, x.w};
      acc = dot8(wv[i], xv, acc);
    }
    if (r + 1 < r1) {  // the next row's loads in flight while this one is reduced
#pragma unroll
      for (int i = 0; i < kChunksPerLane; ++i) wv[i] = __ldg(wrow + size_t(r + 1) * kChunksPerRow + lane + 32 * i);
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      const float logit = bf16_round(acc);
      out[r] = f32_to_bf16(tanhf(logit / kLogitSoftcap) * kLogitSoftcap);
    }
  }
}

}  // namespace

cudaError_t launch_embed(const uint16_t* table, const int32_t* offset, uint16_t* out, int vocab_rows,
                         const LaunchEnv& env) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kVocabThreads);
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, embed_kernel, table, offset, out, vocab_rows, env.sc);
}

cudaError_t launch_logits(const uint16_t* input, const uint16_t* gamma, const uint16_t* weight, uint16_t* out,
                          int rows, const LaunchEnv& env) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * env.sm_count);  // two CTAs of 8 warps per SM
  cfg.blockDim = dim3(kVocabThreads);
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, logits_kernel, input, gamma, weight, out, rows);
}

}  // namespace g4
