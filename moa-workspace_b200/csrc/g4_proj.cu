// The projection ops of the sliding decoder layer on sm_100a:
//   - fused QKV   (reference: furiosa-opt-gemma4-12B/src/ops.rs:37-76)
//   - O + post-RMSNorm + residual (ops.rs:130-146)
//   - NVFP4 GeGLU feed-forward with the weighted residual epilogue (ops.rs:201-239)
// Each is one streaming pass over its weights (g4_stream.cuh) with the reference's
// normalisation / RoPE / GeGLU / residual steps fused into the prologue and epilogues. The
// rounding points are the reference oracle's (furiosa-opt-gemma4-12B/scripts/
// generate_references.py:265-274, 291-414): every op that torch runs on bf16 tensors is
// computed in f32 and rounded to bf16 once, at the same place.
#include "g4_ops.cuh"
#include "g4_stream.cuh"

namespace g4 {
namespace {

constexpr int kBatch = 256;  // K elements per unit

// (warps per CTA, units each warp keeps in flight) of each pass; one CTA per SM
constexpr int kQkvW = 12, kQkvS = 2;
constexpr int kOW = 12, kOS = 2;
constexpr int kUgW = 12, kUgS = 2;
constexpr int kDnW = 12, kDnS = 2;

template <WFmt F, int NMAT, int S, int W, int K>
constexpr size_t smem_bytes() {
  return engine_smem<NMAT>(W) + 2 * size_t(act_col_stride<kBatch>(K)) + 64 * 8;
}

struct SmemView {
  uint8_t* engine;
  uint8_t* cols;
  double* red;
};
template <WFmt F, int NMAT, int S, int W, int K>
__device__ SmemView carve(uint8_t* smem) {
  SmemView v;
  v.engine = smem;
  v.cols = smem + engine_smem<NMAT>(W);
  v.red = reinterpret_cast<double*>(v.cols + 2 * size_t(act_col_stride<kBatch>(K)));
  return v;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // F.gelu(approximate="tanh"): 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 * x^3)))
  const float cube = x * x * x;
  const float inner = 0.7978845608028654f * (x + 0.044715f * cube);
  return 0.5f * x * (1.0f + tanhf(inner));
}

// Last-CTA ticket: returns true in every thread of the CTA that finished last.
__device__ bool last_cta(uint32_t* counter) {
  __shared__ uint32_t is_last;
  __syncthreads();  // every thread's stores of this CTA precede the release below
  if (threadIdx.x == 0) {
    const uint32_t before = atomic_add_acq_rel_gpu(counter, 1u);
    is_last = (before == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();  // ... and the acquire precedes every thread's loads after it
  return is_last != 0;
}

// h = bf16((x * inv_rms(x)) * gamma) for a bf16 vector of K elements held as VPT vectors per
// thread (gemma4.py:83-89). Returns the f32 values of h in `vals`.
template <int K, int VPT>
__device__ void rms_norm_vec(const uint16_t* x, const uint16_t* gamma, float (&vals)[VPT][8], double* red) {
  float gv[VPT][8];
  load_bf16_vec<VPT>(x, K, vals, true);
  load_bf16_vec<VPT>(gamma, K, gv, false);
  double ss = 0.0;
#pragma unroll
  for (int v = 0; v < VPT; ++v)
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += double(vals[v][j]) * double(vals[v][j]);
  const float inv = rms_inverse(block_sum_d(ss, red), K);
#pragma unroll
  for (int v = 0; v < VPT; ++v)
#pragma unroll
    for (int j = 0; j < 8; ++j) vals[v][j] = bf16_round((vals[v][j] * inv) * gv[v][j]);
}

// residual <- bf16(residual + RMSNorm_gamma(y)) [then bf16(. * layer_scalar)], H elements, whole
// CTA, single pass (y is bf16 scratch written by other CTAs of this launch).
template <int THREADS>
__device__ void residual_epilogue(const uint16_t* y, const uint16_t* gamma, uint16_t* residual,
                                  const uint16_t* layer_scalar, double* red) {
  constexpr int VPT = (kH / 8 + THREADS - 1) / THREADS;
  float yv[VPT][8], gv[VPT][8], rv[VPT][8];
  load_bf16_vec<VPT>(y, kH, yv, true);
  load_bf16_vec<VPT>(gamma, kH, gv, false);
  load_bf16_vec<VPT>(residual, kH, rv, true);
  double ss = 0.0;
#pragma unroll
  for (int v = 0; v < VPT; ++v)
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += double(yv[v][j]) * double(yv[v][j]);
  const float inv = rms_inverse(block_sum_d(ss, red), kH);
  const float lam = layer_scalar ? bf16_to_f32(layer_scalar[0]) : 1.0f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int base = (threadIdx.x + v * blockDim.x) * 8;
    if (base < kH) {
      __align__(16) uint16_t out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float nrm = bf16_round((yv[v][j] * inv) * gv[v][j]);
        float r = bf16_round(rv[v][j] + nrm);
        if (layer_scalar) r = bf16_round(r * lam);
        out[j] = f32_to_bf16(r);
      }
      *reinterpret_cast<uint4*>(residual + base) = *reinterpret_cast<const uint4*>(out);
    }
  }
}

// ---------------------------------------------------------------------------------------
// QKV

__device__ void qkv_head_epilogue(const QkvArgs& a, const Scratch& sc, int head) {
  const int lane = threadIdx.x & 31;
  const int base = head * kDs;
  const uint4 raw = ld_cg_u4(sc.y + base + lane * 8);
  const uint16_t* yb = reinterpret_cast<const uint16_t*>(&raw);
  const bool is_q = head < kNs * kGs, is_k = !is_q && head < kNs * kGs + kNs;
  const uint16_t* gamma = is_q ? a.q_rms : (is_k ? a.k_rms : nullptr);
  uint4 graw = make_uint4(0, 0, 0, 0);
  if (gamma) graw = *reinterpret_cast<const uint4*>(gamma + lane * 8);
  const uint16_t* gb = reinterpret_cast<const uint16_t*>(&graw);
  const int kv = *a.kv_offset, rope = *a.rope_offset;
  const bool kv_ok = kv >= 0 && (kv % (kPs * 2)) == 0 && kv / (kPs * 2) < a.ring_len;
  const bool rope_ok = rope >= 0 && (rope % (kDs * 2)) == 0 && rope / (kDs * 2) < a.rope_rows;
  if (!kv_ok || !rope_ok) {
    if (lane == 0) atomicOr(sc.err, (kv_ok ? 0u : kErrKvOffset) | (rope_ok ? 0u : kErrRopeOffset));
    return;
  }
  const int slot = kv / (kPs * 2), row = rope / (kDs * 2);
  uint4 craw = make_uint4(0, 0, 0, 0), sraw = make_uint4(0, 0, 0, 0);
  if (is_q || is_k) {
    craw = *reinterpret_cast<const uint4*>(a.cos + size_t(row) * kDs + lane * 8);
    sraw = *reinterpret_cast<const uint4*>(a.sin + size_t(row) * kDs + lane * 8);
  }
  float y[8];
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    y[j] = bf16_to_f32(yb[j]);
    ss += double(y[j]) * double(y[j]);
  }
  ss = warp_sum_d(ss);
  const float inv = rms_inverse(ss, kDs);
  float nrm[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float s = y[j] * inv;
    nrm[j] = gamma ? bf16_round(s * bf16_to_f32(gb[j])) : bf16_round(s);
  }
  __align__(16) uint16_t outb[8];
  if (is_q || is_k) {
    // RoPE, half-swap form with the low half of `sin` pre-negated by the caller:
    // out[i] = bf16(bf16(n[i] cos[i]) + bf16(n[i ^ 128] sin'[i])). Element i ^ 128 lives in
    // lane ^ 16.
    const uint16_t* cb = reinterpret_cast<const uint16_t*>(&craw);
    const uint16_t* sb = reinterpret_cast<const uint16_t*>(&sraw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float partner = __shfl_xor_sync(0xffffffffu, nrm[j], 16);
      const float c = bf16_round(nrm[j] * bf16_to_f32(cb[j]));
      const float s = bf16_round(partner * bf16_to_f32(sb[j]));
      outb[j] = f32_to_bf16(c + s);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) outb[j] = f32_to_bf16(nrm[j]);
  }
  uint16_t* dst;
  if (is_q)
    dst = a.q_out + base + lane * 8;
  else if (is_k)
    dst = a.k_cache + size_t(slot) * kPs + (head - kNs * kGs) * kDs + lane * 8;
  else
    dst = a.v_cache + size_t(slot) * kPs + (head - kNs * kGs - kNs) * kDs + lane * 8;
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(outb);
}

__global__ void __launch_bounds__(kQkvW * 32, 1) qkv_kernel(QkvArgs a, Scratch sc) {
  constexpr WFmt F = WFmt::kFp8;
  constexpr int W = kQkvW, S = kQkvS;
  extern __shared__ __align__(1024) uint8_t smem[];
  const SmemView sm = carve<F, 1, S, W, kH>(smem);
  G4_STAMP(sc, 0);
  pdl_wait_primary();
  pdl_launch_dependents();
  G4_STAMP(sc, 1);

  // pre-attention RMSNorm -> exact f16 activation columns
  constexpr int VPT = (kH / 8 + W * 32 - 1) / (W * 32);
  float h[VPT][8];
  rms_norm_vec<kH, VPT>(a.x, a.input_rms, h, sm.red);
  const float unscale = build_act_columns<kBatch, VPT>(sm.cols, kH, h, reinterpret_cast<float*>(sm.red));
  __syncthreads();
  G4_STAMP(sc, 2);

  constexpr int kGroups = (kQs + 2 * kPs) / 16;
  auto rows_of = [&](int grp, int) -> const uint8_t* {
    const int r = grp * 16;
    if (r < kQs) return a.q_weight + size_t(r) * kH;
    if (r < kQs + kPs) return a.k_weight + size_t(r - kQs) * kH;
    return a.v_weight + size_t(r - kQs - kPs) * kH;
  };
  auto no_scales = [](int, int) -> const uint8_t* { return nullptr; };
  auto finalize = [&](int grp, const float (&tot)[1]) {
    const int lane = threadIdx.x & 31;
    if (lane < 16) {
      const int r = grp * 16 + lane;
      const uint16_t sb = r < kQs ? a.q_scale[r] : (r < kQs + kPs ? a.k_scale[r - kQs] : a.v_scale[r - kQs - kPs]);
      // scaled_projection: bf16((x @ codes.T) * scale) (generate_references.py:265-274)
      sc.y[r] = f32_to_bf16((tot[0] * unscale) * bf16_to_f32(sb));
    }
    __syncwarp();
    uint32_t head_done = 0;
    const int head = grp / (kDs / 16);
    if (lane == 0) {
      const uint32_t before = atomic_add_acq_rel_gpu(sc.counters + kHeadCounterBase + head, 1u);
      head_done = before == uint32_t(kDs / 16 - 1);
      if (head_done) sc.counters[kHeadCounterBase + head] = 0;
    }
    head_done = __shfl_sync(0xffffffffu, head_done, 0);
    if (head_done) qkv_head_epilogue(a, sc, head);
  };
  stream_gemv<F, 1, kBatch, S, W>(sm.engine, sm.cols, kH, kGroups, kH, 0, rows_of, no_scales, finalize, sc);
  G4_STAMP(sc, 3);
}

// ---------------------------------------------------------------------------------------
// O projection + post-attention RMSNorm + residual

__global__ void __launch_bounds__(kOW * 32, 1) o_kernel(OArgs a, Scratch sc) {
  constexpr WFmt F = WFmt::kFp8;
  constexpr int W = kOW, S = kOS;
  extern __shared__ __align__(1024) uint8_t smem[];
  const SmemView sm = carve<F, 1, S, W, kQs>(smem);
  G4_STAMP(sc, 0);
  pdl_wait_primary();
  pdl_launch_dependents();
  G4_STAMP(sc, 1);

  constexpr int VPT = (kQs / 8 + W * 32 - 1) / (W * 32);
  float xv[VPT][8];
  load_bf16_vec<VPT>(a.x, kQs, xv, true);
  const float unscale = build_act_columns<kBatch, VPT>(sm.cols, kQs, xv, reinterpret_cast<float*>(sm.red));
  __syncthreads();
  G4_STAMP(sc, 2);

  constexpr int kGroups = kH / 16;
  auto rows_of = [&](int grp, int) -> const uint8_t* { return a.o_weight + size_t(grp) * 16 * kQs; };
  auto no_scales = [](int, int) -> const uint8_t* { return nullptr; };
  auto finalize = [&](int grp, const float (&tot)[1]) {
    const int lane = threadIdx.x & 31;
    if (lane < 16) {
      const int r = grp * 16 + lane;
      sc.y[r] = f32_to_bf16((tot[0] * unscale) * bf16_to_f32(a.o_scale[r]));
    }
  };
  stream_gemv<F, 1, kBatch, S, W>(sm.engine, sm.cols, kQs, kGroups, kQs, 0, rows_of, no_scales, finalize, sc);
  G4_STAMP(sc, 3);

  if (last_cta(sc.counters + kCtaCounter)) {
    residual_epilogue<W * 32>(sc.y, a.post_rms, a.residual, nullptr, sm.red);
    if (threadIdx.x == 0) sc.counters[kCtaCounter] = 0;
  }
  G4_STAMP(sc, 4);
}

// ---------------------------------------------------------------------------------------
// NVFP4 feed-forward: up/gate + GeGLU, then down + post-RMSNorm + residual + layer scalar

__global__ void __launch_bounds__(kUgW * 32, 1) ffn_upgate_kernel(FfnArgs a, Scratch sc) {
  constexpr WFmt F = WFmt::kNvfp4;
  constexpr int W = kUgW, S = kUgS;
  extern __shared__ __align__(1024) uint8_t smem[];
  const SmemView sm = carve<F, 2, S, W, kH>(smem);
  G4_STAMP(sc, 0);
  pdl_wait_primary();
  pdl_launch_dependents();
  G4_STAMP(sc, 1);

  constexpr int VPT = (kH / 8 + W * 32 - 1) / (W * 32);
  float h[VPT][8];
  rms_norm_vec<kH, VPT>(a.residual, a.pre_rms, h, sm.red);
  const float unscale = build_act_columns<kBatch, VPT>(sm.cols, kH, h, reinterpret_cast<float*>(sm.red));
  __syncthreads();
  G4_STAMP(sc, 2);
  const float g_up = *a.up_global, g_gate = *a.gate_global;

  constexpr int kGroups = kL / 16;
  auto rows_of = [&](int grp, int m) -> const uint8_t* {
    return (m == 0 ? a.up_packed : a.gate_packed) + size_t(grp) * 16 * (kH / 2);
  };
  auto scales_of = [&](int grp, int m) -> const uint8_t* {
    return (m == 0 ? a.up_scale : a.gate_scale) + size_t(grp) * 16 * (kH / 16);
  };
  auto finalize = [&](int grp, const float (&tot)[2]) {
    const int lane = threadIdx.x & 31;
    if (lane < 16) {
      // GloballyScaled(nn.Linear): bf16(bf16(x @ W.T) * g)  (generate_references.py:358-372)
      const float up = bf16_round(bf16_round(tot[0] * unscale) * g_up);
      const float gate = bf16_round(bf16_round(tot[1] * unscale) * g_gate);
      // down_proj input: bf16(bf16(gelu_tanh(gate)) * up)  (gemma4.py:197)
      sc.act[grp * 16 + lane] = f32_to_bf16(bf16_round(gelu_tanh(gate)) * up);
    }
  };
  stream_gemv<F, 2, kBatch, S, W>(sm.engine, sm.cols, kH, kGroups, kH / 2, kH / 16, rows_of, scales_of, finalize,
                                  sc);
  G4_STAMP(sc, 3);
}

__global__ void __launch_bounds__(kDnW * 32, 1) ffn_down_kernel(FfnArgs a, Scratch sc) {
  constexpr WFmt F = WFmt::kNvfp4;
  constexpr int W = kDnW, S = kDnS;
  extern __shared__ __align__(1024) uint8_t smem[];
  const SmemView sm = carve<F, 1, S, W, kL>(smem);
  G4_STAMP(sc, 8);
  pdl_wait_primary();
  pdl_launch_dependents();
  G4_STAMP(sc, 9);

  constexpr int VPT = (kL / 8 + W * 32 - 1) / (W * 32);
  float av[VPT][8];
  load_bf16_vec<VPT>(sc.act, kL, av, true);
  const float unscale = build_act_columns<kBatch, VPT>(sm.cols, kL, av, reinterpret_cast<float*>(sm.red));
  __syncthreads();
  G4_STAMP(sc, 10);
  const float g_down = *a.down_global;

  constexpr int kGroups = kH / 16;
  auto rows_of = [&](int grp, int) -> const uint8_t* { return a.down_packed + size_t(grp) * 16 * (kL / 2); };
  auto scales_of = [&](int grp, int) -> const uint8_t* { return a.down_scale + size_t(grp) * 16 * (kL / 16); };
  auto finalize = [&](int grp, const float (&tot)[1]) {
    const int lane = threadIdx.x & 31;
    if (lane < 16) sc.y[grp * 16 + lane] = f32_to_bf16(bf16_round(tot[0] * unscale) * g_down);
  };
  stream_gemv<F, 1, kBatch, S, W>(sm.engine, sm.cols, kL, kGroups, kL / 2, kL / 16, rows_of, scales_of, finalize,
                                  sc);
  G4_STAMP(sc, 11);

  if (last_cta(sc.counters + kCtaCounter)) {
    residual_epilogue<W * 32>(sc.y, a.post_rms, a.residual, a.layer_scalar, sm.red);
    if (threadIdx.x == 0) sc.counters[kCtaCounter] = 0;
  }
  G4_STAMP(sc, 12);
}

// ---------------------------------------------------------------------------------------
// launch helpers

template <class... Args>
cudaError_t launch(void (*kernel)(Args...), int grid, int block, size_t smem, const LaunchEnv& env,
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

constexpr size_t kQkvSmem = smem_bytes<WFmt::kFp8, 1, kQkvS, kQkvW, kH>();
constexpr size_t kOSmem = smem_bytes<WFmt::kFp8, 1, kOS, kOW, kQs>();
constexpr size_t kUgSmem = smem_bytes<WFmt::kNvfp4, 2, kUgS, kUgW, kH>();
constexpr size_t kDnSmem = smem_bytes<WFmt::kNvfp4, 1, kDnS, kDnW, kL>();
static_assert(kQkvSmem <= 227 * 1024 && kOSmem <= 227 * 1024 && kUgSmem <= 227 * 1024 && kDnSmem <= 227 * 1024,
              "shared memory budget");

}  // namespace

cudaError_t prepare_proj_kernels() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kQkvSmem)))) return e;
  if ((e = cudaFuncSetAttribute(o_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kOSmem)))) return e;
  if ((e = cudaFuncSetAttribute(ffn_upgate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kUgSmem))))
    return e;
  if ((e = cudaFuncSetAttribute(ffn_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kDnSmem))))
    return e;
  return cudaSuccess;
}

cudaError_t launch_qkv(const QkvArgs& a, const LaunchEnv& env) {
  return launch(qkv_kernel, env.sm_count, kQkvW * 32, kQkvSmem, env, a, env.sc);
}

cudaError_t launch_o(const OArgs& a, const LaunchEnv& env) {
  return launch(o_kernel, env.sm_count, kOW * 32, kOSmem, env, a, env.sc);
}

cudaError_t launch_ffn_nvfp4(const FfnArgs& a, const LaunchEnv& env) {
  cudaError_t e = launch(ffn_upgate_kernel, env.sm_count, kUgW * 32, kUgSmem, env, a, env.sc);
  if (e != cudaSuccess) return e;
  LaunchEnv chained = env;
  chained.pdl = true;  // the down pass launches while the up/gate pass drains
  return launch(ffn_down_kernel, env.sm_count, kDnW * 32, kDnSmem, chained, a, env.sc);
}

}  // namespace g4
