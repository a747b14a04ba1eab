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

// ---------------------------------------------------------------------------------------
// Configuration (chunk K, warps per CTA, ring slots per warp)

constexpr int kQkvKc = 640, kQkvW = 8, kQkvS = 2;
constexpr int kOKc = 512, kOW = 8, kOS = 2;
constexpr int kUgKc = 256, kUgW = 8, kUgS = 4;
constexpr int kDnKc = 1024, kDnW = 8, kDnS = 2;

template <WFmt F, int NMAT, int KC, int W, int S>
constexpr size_t smem_bytes(int k_total) {
  return size_t(W) * S * SlotLayout<F, NMAT, KC>::kSlotBytes + 2 * size_t(act_col_stride(k_total)) +
         size_t(W) * S * 8 + 64 * 8;
}

struct SmemView {
  uint8_t* slots;
  uint8_t* cols;
  uint64_t* bars;
  double* red;
};

template <WFmt F, int NMAT, int KC, int W, int S>
__device__ SmemView carve(uint8_t* smem, int k_total) {
  SmemView v;
  v.slots = smem;
  v.cols = smem + size_t(W) * S * SlotLayout<F, NMAT, KC>::kSlotBytes;
  v.bars = reinterpret_cast<uint64_t*>(v.cols + 2 * size_t(act_col_stride(k_total)));
  v.red = reinterpret_cast<double*>(v.bars + W * S);
  return v;
}

__device__ __forceinline__ void init_warp_bars(uint64_t* bars, int s) {
  if ((threadIdx.x & 31) == 0)
    for (int i = 0; i < s; ++i) mbar_init(bars + i, 1);
  fence_mbar_init();
  __syncwarp();
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
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t before = atomicAdd(counter, 1u);
    is_last = (before == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (is_last) __threadfence();
  return is_last != 0;
}

// residual[i] <- bf16(residual[i] + RMSNorm(y)[i]) [ * layer_scalar ], over `n` elements, by
// the whole CTA (y is bf16 scratch written by other CTAs of this launch).
__device__ void residual_epilogue(const uint16_t* y, const uint16_t* gamma, uint16_t* residual, int n,
                                  const uint16_t* layer_scalar, double* red) {
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf16_to_f32(__ldcg(y + i));
    ss += double(v) * double(v);
  }
  ss = block_sum_d(ss, red);
  const float inv = rms_inverse(ss, n);
  const float lam = layer_scalar ? bf16_to_f32(layer_scalar[0]) : 1.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf16_to_f32(__ldcg(y + i));
    const float nrm = bf16_round((v * inv) * bf16_to_f32(gamma[i]));
    float r = bf16_round(bf16_to_f32(residual[i]) + nrm);
    if (layer_scalar) r = bf16_round(r * lam);
    residual[i] = f32_to_bf16(r);
  }
}

// ---------------------------------------------------------------------------------------
// QKV

__device__ void qkv_head_epilogue(const QkvArgs& a, const Scratch& sc, int head) {
  const int lane = threadIdx.x & 31;
  const int base = head * kDs;
  const uint4 raw = ld_cg_u4(sc.y + base + lane * 8);
  const uint16_t* yb = reinterpret_cast<const uint16_t*>(&raw);
  float y[8];
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    y[j] = bf16_to_f32(yb[j]);
    ss += double(y[j]) * double(y[j]);
  }
  ss = warp_sum_d(ss);
  const float inv = rms_inverse(ss, kDs);
  const bool is_q = head < kNs * kGs, is_k = !is_q && head < kNs * kGs + kNs;
  const uint16_t* gamma = is_q ? a.q_rms : (is_k ? a.k_rms : nullptr);
  float nrm[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float s = y[j] * inv;
    nrm[j] = gamma ? bf16_round(s * bf16_to_f32(gamma[lane * 8 + j])) : bf16_round(s);
  }
  const int kv = *a.kv_offset, rope = *a.rope_offset;
  const bool kv_ok = kv >= 0 && (kv % (kPs * 2)) == 0 && kv / (kPs * 2) < a.ring_len;
  const bool rope_ok = rope >= 0 && (rope % (kDs * 2)) == 0 && rope / (kDs * 2) < a.rope_rows;
  if (!kv_ok || !rope_ok) {
    if (lane == 0) atomicOr(sc.err, (kv_ok ? 0u : kErrKvOffset) | (rope_ok ? 0u : kErrRopeOffset));
    return;
  }
  const int slot = kv / (kPs * 2), row = rope / (kDs * 2);
  uint16_t outb[8];
  if (is_q || is_k) {
    // RoPE, half-swap form with the low half of `sin` pre-negated by the caller:
    // out[i] = bf16(bf16(n[i] cos[i]) + bf16(n[i ^ 128] sin'[i])). Element i ^ 128 lives in
    // lane ^ 16.
    const uint16_t* crow = a.cos + size_t(row) * kDs + lane * 8;
    const uint16_t* srow = a.sin + size_t(row) * kDs + lane * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float partner = __shfl_xor_sync(0xffffffffu, nrm[j], 16);
      const float c = bf16_round(nrm[j] * bf16_to_f32(crow[j]));
      const float s = bf16_round(partner * bf16_to_f32(srow[j]));
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
  extern __shared__ __align__(1024) uint8_t smem[];
  const SmemView sm = carve<F, 1, kQkvKc, kQkvW, kQkvS>(smem, kH);
  const int warp = threadIdx.x >> 5;
  uint8_t* my_slots = sm.slots + size_t(warp) * kQkvS * SlotLayout<F, 1, kQkvKc>::kSlotBytes;
  uint64_t* my_bars = sm.bars + warp * kQkvS;
  init_warp_bars(my_bars, kQkvS);

  constexpr int kGroups = (kQs + 2 * kPs) / 16;
  constexpr int kC = kH / kQkvKc;
  const int64_t nw = int64_t(gridDim.x) * kQkvW, wid = int64_t(blockIdx.x) * kQkvW + warp;
  auto rows_of = [&](int grp, int) -> const uint8_t* {
    const int r = grp * 16;
    if (r < kQs) return a.q_weight + size_t(r) * kH;
    if (r < kQs + kPs) return a.k_weight + size_t(r - kQs) * kH;
    return a.v_weight + size_t(r - kQs - kPs) * kH;
  };
  auto no_scales = [](int, int) -> const uint8_t* { return nullptr; };
  stream_prefill<F, 1, kQkvKc, kQkvS>(my_slots, my_bars, kH, wid, nw, kGroups, kH, 0, rows_of, no_scales);

  pdl_wait_primary();
  pdl_launch_dependents();

  // pre-attention RMSNorm (gemma4.py:83-89) -> exact f16 activation columns
  double ss = 0.0;
  for (int i = threadIdx.x; i < kH; i += blockDim.x) {
    const float v = bf16_to_f32(a.x[i]);
    ss += double(v) * double(v);
  }
  ss = block_sum_d(ss, sm.red);
  const float inv = rms_inverse(ss, kH);
  auto h_of = [&](int i) { return bf16_round((bf16_to_f32(a.x[i]) * inv) * bf16_to_f32(a.input_rms[i])); };
  const float unscale = build_act_columns(sm.cols, kH, h_of, reinterpret_cast<float*>(sm.red));
  __syncthreads();

  const int64_t total = int64_t(kGroups) * kC;
  auto flush = [&](int grp, int cstart, int nch, const float (&v)[1][2]) {
    if (!flush_piece<1>(sc.partials, sc.counters + grp, grp, kC, cstart, nch, v)) return;
    const int lane = threadIdx.x & 31;
    const float tot = gather_group<1>(sc.partials, grp, kC, 0, nw, total);
    if (lane < 16) {
      const int r = grp * 16 + lane;
      const uint16_t sb = r < kQs ? a.q_scale[r] : (r < kQs + kPs ? a.k_scale[r - kQs] : a.v_scale[r - kQs - kPs]);
      // scaled_projection: bf16((x @ codes.T) * scale) (generate_references.py:265-274)
      sc.y[r] = f32_to_bf16((tot * unscale) * bf16_to_f32(sb));
    }
    __threadfence();
    __syncwarp();
    uint32_t head_done = 0;
    if (lane == 0) {
      sc.counters[grp] = 0;
      const int head = grp / (kDs / 16);
      const uint32_t before = atomicAdd(sc.counters + kHeadCounterBase + head, 1u);
      head_done = before == uint32_t(kDs / 16 - 1);
      if (head_done) sc.counters[kHeadCounterBase + head] = 0;
    }
    head_done = __shfl_sync(0xffffffffu, head_done, 0);
    if (head_done) {
      __threadfence();
      qkv_head_epilogue(a, sc, grp / (kDs / 16));
    }
  };
  stream_gemv<F, 1, kQkvKc, kQkvS>(my_slots, my_bars, sm.cols, kH, wid, nw, kGroups, kH, 0, rows_of, no_scales,
                                    flush, sc.err, true);
}

// ---------------------------------------------------------------------------------------
// O projection + post-attention RMSNorm + residual

__global__ void __launch_bounds__(kOW * 32, 1) o_kernel(OArgs a, Scratch sc) {
  constexpr WFmt F = WFmt::kFp8;
  extern __shared__ __align__(1024) uint8_t smem[];
  const SmemView sm = carve<F, 1, kOKc, kOW, kOS>(smem, kQs);
  const int warp = threadIdx.x >> 5;
  uint8_t* my_slots = sm.slots + size_t(warp) * kOS * SlotLayout<F, 1, kOKc>::kSlotBytes;
  uint64_t* my_bars = sm.bars + warp * kOS;
  init_warp_bars(my_bars, kOS);

  constexpr int kGroups = kH / 16;
  constexpr int kC = kQs / kOKc;
  const int64_t nw = int64_t(gridDim.x) * kOW, wid = int64_t(blockIdx.x) * kOW + warp;
  auto rows_of = [&](int grp, int) -> const uint8_t* { return a.o_weight + size_t(grp) * 16 * kQs; };
  auto no_scales = [](int, int) -> const uint8_t* { return nullptr; };
  stream_prefill<F, 1, kOKc, kOS>(my_slots, my_bars, kQs, wid, nw, kGroups, kQs, 0, rows_of, no_scales);

  pdl_wait_primary();
  pdl_launch_dependents();

  auto h_of = [&](int i) { return bf16_to_f32(a.x[i]); };
  const float unscale = build_act_columns(sm.cols, kQs, h_of, reinterpret_cast<float*>(sm.red));
  __syncthreads();

  const int64_t total = int64_t(kGroups) * kC;
  auto flush = [&](int grp, int cstart, int nch, const float (&v)[1][2]) {
    if (!flush_piece<1>(sc.partials, sc.counters + grp, grp, kC, cstart, nch, v)) return;
    const int lane = threadIdx.x & 31;
    const float tot = gather_group<1>(sc.partials, grp, kC, 0, nw, total);
    if (lane < 16) {
      const int r = grp * 16 + lane;
      sc.y[r] = f32_to_bf16((tot * unscale) * bf16_to_f32(a.o_scale[r]));
    }
    __syncwarp();
    if (lane == 0) sc.counters[grp] = 0;
  };
  stream_gemv<F, 1, kOKc, kOS>(my_slots, my_bars, sm.cols, kQs, wid, nw, kGroups, kQs, 0, rows_of, no_scales, flush,
                                sc.err, true);

  if (last_cta(sc.counters + kCtaCounter)) {
    residual_epilogue(sc.y, a.post_rms, a.residual, kH, nullptr, sm.red);
    if (threadIdx.x == 0) sc.counters[kCtaCounter] = 0;
  }
}

// ---------------------------------------------------------------------------------------
// NVFP4 feed-forward: up/gate + GeGLU, then down + post-RMSNorm + residual + layer scalar

__global__ void __launch_bounds__(kUgW * 32, 1) ffn_upgate_kernel(FfnArgs a, Scratch sc) {
  constexpr WFmt F = WFmt::kNvfp4;
  extern __shared__ __align__(1024) uint8_t smem[];
  const SmemView sm = carve<F, 2, kUgKc, kUgW, kUgS>(smem, kH);
  const int warp = threadIdx.x >> 5;
  uint8_t* my_slots = sm.slots + size_t(warp) * kUgS * SlotLayout<F, 2, kUgKc>::kSlotBytes;
  uint64_t* my_bars = sm.bars + warp * kUgS;
  init_warp_bars(my_bars, kUgS);

  constexpr int kGroups = kL / 16;
  constexpr int kC = kH / kUgKc;
  const int64_t nw = int64_t(gridDim.x) * kUgW, wid = int64_t(blockIdx.x) * kUgW + warp;
  auto rows_of = [&](int grp, int m) -> const uint8_t* {
    return (m == 0 ? a.up_packed : a.gate_packed) + size_t(grp) * 16 * (kH / 2);
  };
  auto scales_of = [&](int grp, int m) -> const uint8_t* {
    return (m == 0 ? a.up_scale : a.gate_scale) + size_t(grp) * 16 * (kH / 16);
  };
  stream_prefill<F, 2, kUgKc, kUgS>(my_slots, my_bars, kH, wid, nw, kGroups, kH / 2, kH / 16, rows_of, scales_of);

  pdl_wait_primary();
  pdl_launch_dependents();

  // pre-feed-forward RMSNorm of the residual
  double ss = 0.0;
  for (int i = threadIdx.x; i < kH; i += blockDim.x) {
    const float v = bf16_to_f32(a.residual[i]);
    ss += double(v) * double(v);
  }
  ss = block_sum_d(ss, sm.red);
  const float inv = rms_inverse(ss, kH);
  auto h_of = [&](int i) { return bf16_round((bf16_to_f32(a.residual[i]) * inv) * bf16_to_f32(a.pre_rms[i])); };
  const float unscale = build_act_columns(sm.cols, kH, h_of, reinterpret_cast<float*>(sm.red));
  __syncthreads();
  const float g_up = *a.up_global, g_gate = *a.gate_global;

  const int64_t total = int64_t(kGroups) * kC;
  auto flush = [&](int grp, int cstart, int nch, const float (&v)[2][2]) {
    if (!flush_piece<2>(sc.partials, sc.counters + grp, grp, kC, cstart, nch, v)) return;
    const int lane = threadIdx.x & 31;
    const float tu = gather_group<2>(sc.partials, grp, kC, 0, nw, total);
    const float tg = gather_group<2>(sc.partials, grp, kC, 1, nw, total);
    if (lane < 16) {
      // GloballyScaled(nn.Linear): bf16(bf16(x @ W.T) * g)  (generate_references.py:358-372)
      const float up = bf16_round(bf16_round(tu * unscale) * g_up);
      const float gate = bf16_round(bf16_round(tg * unscale) * g_gate);
      // down_proj input: bf16(bf16(gelu_tanh(gate)) * up)  (gemma4.py:197)
      sc.act[grp * 16 + lane] = f32_to_bf16(bf16_round(gelu_tanh(gate)) * up);
    }
    __syncwarp();
    if (lane == 0) sc.counters[grp] = 0;
  };
  stream_gemv<F, 2, kUgKc, kUgS>(my_slots, my_bars, sm.cols, kH, wid, nw, kGroups, kH / 2, kH / 16, rows_of,
                                  scales_of, flush, sc.err, true);
}

__global__ void __launch_bounds__(kDnW * 32, 1) ffn_down_kernel(FfnArgs a, Scratch sc) {
  constexpr WFmt F = WFmt::kNvfp4;
  extern __shared__ __align__(1024) uint8_t smem[];
  const SmemView sm = carve<F, 1, kDnKc, kDnW, kDnS>(smem, kL);
  const int warp = threadIdx.x >> 5;
  uint8_t* my_slots = sm.slots + size_t(warp) * kDnS * SlotLayout<F, 1, kDnKc>::kSlotBytes;
  uint64_t* my_bars = sm.bars + warp * kDnS;
  init_warp_bars(my_bars, kDnS);

  constexpr int kGroups = kH / 16;
  constexpr int kC = kL / kDnKc;
  const int64_t nw = int64_t(gridDim.x) * kDnW, wid = int64_t(blockIdx.x) * kDnW + warp;
  auto rows_of = [&](int grp, int) -> const uint8_t* { return a.down_packed + size_t(grp) * 16 * (kL / 2); };
  auto scales_of = [&](int grp, int) -> const uint8_t* { return a.down_scale + size_t(grp) * 16 * (kL / 16); };
  stream_prefill<F, 1, kDnKc, kDnS>(my_slots, my_bars, kL, wid, nw, kGroups, kL / 2, kL / 16, rows_of, scales_of);

  pdl_wait_primary();
  pdl_launch_dependents();

  auto h_of = [&](int i) { return bf16_to_f32(__ldcg(sc.act + i)); };
  const float unscale = build_act_columns(sm.cols, kL, h_of, reinterpret_cast<float*>(sm.red));
  __syncthreads();
  const float g_down = *a.down_global;

  const int64_t total = int64_t(kGroups) * kC;
  auto flush = [&](int grp, int cstart, int nch, const float (&v)[1][2]) {
    if (!flush_piece<1>(sc.partials, sc.counters + grp, grp, kC, cstart, nch, v)) return;
    const int lane = threadIdx.x & 31;
    const float tot = gather_group<1>(sc.partials, grp, kC, 0, nw, total);
    if (lane < 16) sc.y[grp * 16 + lane] = f32_to_bf16(bf16_round(tot * unscale) * g_down);
    __syncwarp();
    if (lane == 0) sc.counters[grp] = 0;
  };
  stream_gemv<F, 1, kDnKc, kDnS>(my_slots, my_bars, sm.cols, kL, wid, nw, kGroups, kL / 2, kL / 16, rows_of,
                                  scales_of, flush, sc.err, true);

  if (last_cta(sc.counters + kCtaCounter)) {
    residual_epilogue(sc.y, a.post_rms, a.residual, kH, a.layer_scalar, sm.red);
    if (threadIdx.x == 0) sc.counters[kCtaCounter] = 0;
  }
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

constexpr size_t kQkvSmem = smem_bytes<WFmt::kFp8, 1, kQkvKc, kQkvW, kQkvS>(kH);
constexpr size_t kOSmem = smem_bytes<WFmt::kFp8, 1, kOKc, kOW, kOS>(kQs);
constexpr size_t kUgSmem = smem_bytes<WFmt::kNvfp4, 2, kUgKc, kUgW, kUgS>(kH);
constexpr size_t kDnSmem = smem_bytes<WFmt::kNvfp4, 1, kDnKc, kDnW, kDnS>(kL);
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
  chained.pdl = true;  // the down pass overlaps its weight prefetch with the up/gate tail
  return launch(ffn_down_kernel, env.sm_count, kDnW * 32, kDnSmem, chained, a, env.sc);
}

}  // namespace g4
