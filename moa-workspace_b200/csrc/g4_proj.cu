// The projection ops of the sliding decoder layer on sm_100a:
//   - fused QKV   (reference: furiosa-opt-gemma4-12B/src/ops.rs:37-76)
//   - O + post-RMSNorm + residual (ops.rs:130-146)
//   - NVFP4 GeGLU feed-forward with the weighted residual epilogue (ops.rs:201-239)
// Each is one tensor-core streaming pass over its weights (g4_gemv.cuh) with the reference's
// normalisation / RoPE / GeGLU / residual steps fused into the prologue and the epilogues. The
// rounding points are the reference oracle's (furiosa-opt-gemma4-12B/scripts/
// generate_references.py:265-274, 291-414): every op that torch runs on bf16 tensors is
// computed in f32 and rounded to bf16 once, at the same place.
#include <cudaTypedefs.h>

#include <utility>

#include "g4_gemv.cuh"
#include "g4_ops.cuh"

namespace g4 {
namespace {

// Pipeline shapes: <nvfp4, stages, K units per tile, tiles, B slots>. Units per tile = K / 256;
// B slots >= the largest number of distinct K units one CTA's run touches on a 148-SM grid
// (launchers grow the grid if a smaller GPU would need more).
using QkvShape = GemvShape<false, 6, kH / kUnitK, (kQs + 2 * kPs) / kTileRows, 8>;
using OShape = GemvShape<false, 6, kQs / kUnitK, kH / kTileRows, 4>;
using UpGateShape = GemvShape<true, 5, kH / kUnitK, kL / 64, 15>;  // tile = 64 up rows + 64 gate rows
using DownShape = GemvShape<true, 5, kL / kUnitK, kH / kTileRows, 13>;

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

// 1 / sqrt(mean(x^2) + eps) of a bf16 vector of K elements written by the preceding kernel
// (gemma4.py:83-89): squares summed exactly in f64, the mean narrowed to f32.
template <int K>
__device__ float rms_inverse_of(const uint16_t* x, double* red) {
  double ss = 0.0;
  for (int k = threadIdx.x * 8; k < K; k += blockDim.x * 8) {
    const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(x + k));
    const uint16_t* b = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const double f = bf16_to_f32(b[j]);
      ss += f * f;
    }
  }
  return rms_inverse(block_sum_d(ss, red), K);
}

// 16 bf16 elements from a vector another kernel wrote (L2-coherent loads).
__device__ __forceinline__ void load16_cg(const uint16_t* p, float (&v)[16]) {
  const uint4 a = __ldcg(reinterpret_cast<const uint4*>(p));
  const uint4 b = __ldcg(reinterpret_cast<const uint4*>(p + 8));
  const uint16_t* ha = reinterpret_cast<const uint16_t*>(&a);
  const uint16_t* hb = reinterpret_cast<const uint16_t*>(&b);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = bf16_to_f32(ha[j]);
    v[8 + j] = bf16_to_f32(hb[j]);
  }
}

// h = bf16((x * inv) * gamma) for 16 elements (the pre-norm of the QKV and FFN ops).
__device__ __forceinline__ void rms_scaled16(const uint16_t* x, const uint16_t* gamma, float inv, float (&v)[16]) {
  float g[16];
  load16_cg(x, v);
  const uint4 ga = *reinterpret_cast<const uint4*>(gamma);
  const uint4 gb = *reinterpret_cast<const uint4*>(gamma + 8);
  const uint16_t* ha = reinterpret_cast<const uint16_t*>(&ga);
  const uint16_t* hb = reinterpret_cast<const uint16_t*>(&gb);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    g[j] = bf16_to_f32(ha[j]);
    g[8 + j] = bf16_to_f32(hb[j]);
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = bf16_round((v[j] * inv) * g[j]);
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

// Per-head RMSNorm (+ RoPE for q and k) of one projected head and its store: q_out, or the
// addressed ring slot of the K / V cache. One warp, eight elements per lane.
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

struct QkvMaps {
  CUtensorMap q, k, v;
};

struct QkvOp {
  const QkvMaps* maps;
  QkvArgs a;
  Scratch sc;
  float inv = 0.f;
  uint32_t tx_bytes = QkvShape::kABytes;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    constexpr int kQTiles = kQs / kTileRows, kKTiles = kPs / kTileRows;
    const CUtensorMap* m = tile < kQTiles ? &maps->q : (tile < kQTiles + kKTiles ? &maps->k : &maps->v);
    const int row0 = (tile < kQTiles ? tile : (tile < kQTiles + kKTiles ? tile - kQTiles : tile - kQTiles - kKTiles)) *
                     kTileRows;
    tma_load_2d(stage, m, kc * kUnitK, row0, bar, policy);
    tma_load_2d(stage + 16384, m, kc * kUnitK + 128, row0, bar, policy);
  }
  __device__ void prologue(GemvCtl& ctl) { inv = rms_inverse_of<kH>(a.x, ctl.red_d); }
  __device__ void act16(int k0, float (&v)[16]) const { rms_scaled16(a.x + k0, a.input_rms + k0, inv, v); }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl& ctl) const {
    const int r = tile * kTileRows + row;
    const uint16_t sb = r < kQs ? a.q_scale[r] : (r < kQs + kPs ? a.k_scale[r - kQs] : a.v_scale[r - kQs - kPs]);
    // scaled_projection: bf16((x @ codes.T) * scale) (generate_references.py:265-274)
    sc.y[r] = f32_to_bf16(v * bf16_to_f32(sb));
    named_bar(kEpiBarrier, kEpiThreads);
    const int head = r / kDs;  // two tiles per head
    if (row == 0) {
      const uint32_t before = atomic_add_acq_rel_gpu(sc.counters + kHeadCounterBase + head, 1u);
      const bool done = before == uint32_t(kDs / kTileRows - 1);
      if (done) sc.counters[kHeadCounterBase + head] = 0;
      ctl.bcast2 = done ? 1u : 0u;
    }
    named_bar(kEpiBarrier, kEpiThreads);
    // the warp holding row 0 (it took the ticket) normalises, rotates and stores the head
    if (ctl.bcast2 && (threadIdx.x >> 5) == 4) qkv_head_epilogue(a, sc, head);
  }
};

__global__ void __launch_bounds__(kGemvThreads, 1) qkv_kernel(const __grid_constant__ QkvMaps maps, QkvArgs a,
                                                              Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  QkvOp op{&maps, a, sc};
  gemv_run<QkvShape>(op, smem, sc);
}

// ---------------------------------------------------------------------------------------
// O projection + post-attention RMSNorm + residual

struct OOp {
  const CUtensorMap* map;
  OArgs a;
  Scratch sc;
  uint32_t tx_bytes = OShape::kABytes;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    tma_load_2d(stage, map, kc * kUnitK, tile * kTileRows, bar, policy);
    tma_load_2d(stage + 16384, map, kc * kUnitK + 128, tile * kTileRows, bar, policy);
  }
  __device__ void prologue(GemvCtl&) {}
  __device__ void act16(int k0, float (&v)[16]) const { load16_cg(a.x + k0, v); }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl&) const {
    const int r = tile * kTileRows + row;
    sc.y[r] = f32_to_bf16(v * bf16_to_f32(a.o_scale[r]));
  }
};

__global__ void __launch_bounds__(kGemvThreads, 1) o_kernel(const __grid_constant__ CUtensorMap map, OArgs a,
                                                            Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ double red[8];
  OOp op{&map, a, sc};
  gemv_run<OShape>(op, smem, sc);
  if (last_cta(sc.counters + kCtaCounter)) {
    residual_epilogue<kGemvThreads>(sc.y, a.post_rms, a.residual, nullptr, red);
    if (threadIdx.x == 0) sc.counters[kCtaCounter] = 0;
  }
}

// ---------------------------------------------------------------------------------------
// NVFP4 feed-forward: up/gate + GeGLU, then down + post-RMSNorm + residual + layer scalar

struct UpGateMaps {
  CUtensorMap up, gate, up_s, gate_s;
};

struct UpGateOp {
  const UpGateMaps* maps;
  FfnArgs a;
  Scratch sc;
  float inv = 0.f, g_up = 0.f, g_gate = 0.f;
  uint32_t tx_bytes = 4 * 64 * 64 + 2 * 64 * 16;  // four 64-row e2m1 boxes + two scale boxes

  // stage: [K 0-127: up rows (8 KB) | gate rows (8 KB)] [K 128-255: same] [up scales | gate scales]
  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    const int row0 = tile * 64, x = kc * kUnitK;
    tma_load_2d(stage, &maps->up, x, row0, bar, policy);
    tma_load_2d(stage + 8192, &maps->gate, x, row0, bar, policy);
    tma_load_2d(stage + 16384, &maps->up, x + 128, row0, bar, policy);
    tma_load_2d(stage + 24576, &maps->gate, x + 128, row0, bar, policy);
    tma_load_2d(stage + UpGateShape::kABytes, &maps->up_s, kc * (kUnitK / 16), row0, bar, policy);
    tma_load_2d(stage + UpGateShape::kABytes + 1024, &maps->gate_s, kc * (kUnitK / 16), row0, bar, policy);
  }
  __device__ void prologue(GemvCtl& ctl) {
    inv = rms_inverse_of<kH>(a.residual, ctl.red_d);
    g_up = *a.up_global;
    g_gate = *a.gate_global;
  }
  __device__ void act16(int k0, float (&v)[16]) const { rms_scaled16(a.residual + k0, a.pre_rms + k0, inv, v); }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl& ctl) const {
    // GloballyScaled(nn.Linear): bf16(bf16(x @ W.T) * g)  (generate_references.py:358-372)
    const float val = bf16_round(bf16_round(v) * (row < 64 ? g_up : g_gate));
    if (row >= 64) ctl.xchg[row - 64] = val;
    named_bar(kEpiBarrier, kEpiThreads);
    // down_proj input: bf16(bf16(gelu_tanh(gate)) * up)  (gemma4.py:197)
    if (row < 64) sc.act[tile * 64 + row] = f32_to_bf16(bf16_round(gelu_tanh(ctl.xchg[row])) * val);
    named_bar(kEpiBarrier, kEpiThreads);
  }
};

__global__ void __launch_bounds__(kGemvThreads, 1) ffn_upgate_kernel(const __grid_constant__ UpGateMaps maps, FfnArgs a,
                                                                     Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  UpGateOp op{&maps, a, sc};
  gemv_run<UpGateShape>(op, smem, sc);
}

struct DownMaps {
  CUtensorMap w, s;
};

struct DownOp {
  const DownMaps* maps;
  FfnArgs a;
  Scratch sc;
  float g_down = 0.f;
  uint32_t tx_bytes = 2 * 128 * 64 + 128 * 16;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    const int row0 = tile * kTileRows, x = kc * kUnitK;
    tma_load_2d(stage, &maps->w, x, row0, bar, policy);
    tma_load_2d(stage + 16384, &maps->w, x + 128, row0, bar, policy);
    tma_load_2d(stage + DownShape::kABytes, &maps->s, kc * (kUnitK / 16), row0, bar, policy);
  }
  __device__ void prologue(GemvCtl&) { g_down = *a.down_global; }
  __device__ void act16(int k0, float (&v)[16]) const { load16_cg(sc.act + k0, v); }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl&) const {
    const int r = tile * kTileRows + row;
    sc.y[r] = f32_to_bf16(bf16_round(v) * g_down);
  }
};

__global__ void __launch_bounds__(kGemvThreads, 1) ffn_down_kernel(const __grid_constant__ DownMaps maps, FfnArgs a,
                                                                   Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ double red[8];
  DownOp op{&maps, a, sc};
  gemv_run<DownShape>(op, smem, sc);
  if (last_cta(sc.counters + kCtaCounter)) {
    residual_epilogue<kGemvThreads>(sc.y, a.post_rms, a.residual, a.layer_scalar, red);
    if (threadIdx.x == 0) sc.counters[kCtaCounter] = 0;
  }
}

// ---------------------------------------------------------------------------------------
// launch helpers

template <class... KArgs, class... Args>
cudaError_t launch(void (*kernel)(KArgs...), int grid, size_t smem, const LaunchEnv& env, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// One CTA per SM, unless a smaller GPU would give a CTA more K units than its B slots hold.
template <class Shape>
int grid_for(const LaunchEnv& env) {
  const int need = (Shape::kTotalUnits + Shape::kBSlots - 1) / Shape::kBSlots;
  return env.sm_count > need ? env.sm_count : need;
}

}  // namespace

cudaError_t prepare_proj_kernels() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(QkvShape::kSmemBytes))))
    return e;
  if ((e = cudaFuncSetAttribute(o_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(OShape::kSmemBytes))))
    return e;
  if ((e = cudaFuncSetAttribute(ffn_upgate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(UpGateShape::kSmemBytes))))
    return e;
  if ((e = cudaFuncSetAttribute(ffn_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(DownShape::kSmemBytes))))
    return e;
  return cudaSuccess;
}

cudaError_t launch_qkv(const QkvArgs& a, const LaunchEnv& env) {
  QkvMaps m;
  cudaError_t e;
  if ((e = env.maps->u8(a.q_weight, kH, kQs, 128, kTileRows, true, &m.q))) return e;
  if ((e = env.maps->u8(a.k_weight, kH, kPs, 128, kTileRows, true, &m.k))) return e;
  if ((e = env.maps->u8(a.v_weight, kH, kPs, 128, kTileRows, true, &m.v))) return e;
  return launch(qkv_kernel, grid_for<QkvShape>(env), QkvShape::kSmemBytes, env, m, a, env.sc);
}

cudaError_t launch_o(const OArgs& a, const LaunchEnv& env) {
  CUtensorMap m;
  cudaError_t e;
  if ((e = env.maps->u8(a.o_weight, kQs, kH, 128, kTileRows, true, &m))) return e;
  return launch(o_kernel, grid_for<OShape>(env), OShape::kSmemBytes, env, m, a, env.sc);
}

cudaError_t launch_ffn_nvfp4(const FfnArgs& a, const LaunchEnv& env) {
  UpGateMaps ug;
  DownMaps dn;
  cudaError_t e;
  if ((e = env.maps->fp4(a.up_packed, kH, kL, 64, &ug.up))) return e;
  if ((e = env.maps->fp4(a.gate_packed, kH, kL, 64, &ug.gate))) return e;
  if ((e = env.maps->u8(a.up_scale, kH / 16, kL, 16, 64, false, &ug.up_s))) return e;
  if ((e = env.maps->u8(a.gate_scale, kH / 16, kL, 16, 64, false, &ug.gate_s))) return e;
  if ((e = env.maps->fp4(a.down_packed, kL, kH, kTileRows, &dn.w))) return e;
  if ((e = env.maps->u8(a.down_scale, kL / 16, kH, 16, kTileRows, false, &dn.s))) return e;
  e = launch(ffn_upgate_kernel, grid_for<UpGateShape>(env), UpGateShape::kSmemBytes, env, ug, a, env.sc);
  if (e != cudaSuccess) return e;
  LaunchEnv chained = env;
  chained.pdl = true;  // the down pass prefetches its weights while the up/gate pass drains
  return launch(ffn_down_kernel, grid_for<DownShape>(env), DownShape::kSmemBytes, chained, dn, a, env.sc);
}

// ---------------------------------------------------------------------------------------
// tensor maps

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}
}  // namespace

const CUtensorMap* TmapCache::find(const void* base, uint64_t key) const {
  for (int i = 0; i < kEntries; ++i)
    if (entries_[i].base == base && entries_[i].key == key) return &entries_[i].map;
  return nullptr;
}

void TmapCache::put(const void* base, uint64_t key, const CUtensorMap& map) {
  entries_[next_].base = base;
  entries_[next_].key = key;
  entries_[next_].map = map;
  next_ = (next_ + 1) % kEntries;
}

cudaError_t TmapCache::u8(const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                          bool swizzle128, CUtensorMap* out) {
  const uint64_t key = (cols << 34) ^ (rows << 12) ^ (uint64_t(box_cols) << 4) ^ (uint64_t(box_rows) << 1) ^
                       (swizzle128 ? 1u : 0u) ^ (uint64_t(1) << 63);
  if (const CUtensorMap* m = find(base, key)) {
    *out = *m;
    return cudaSuccess;
  }
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {cols};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  put(base, key, *out);
  return cudaSuccess;
}

cudaError_t TmapCache::fp4(const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows, CUtensorMap* out) {
  const uint64_t key = (cols << 34) ^ (rows << 12) ^ (uint64_t(box_rows) << 1);
  if (const CUtensorMap* m = find(base, key)) {
    *out = *m;
    return cudaSuccess;
  }
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {cols / 2};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void*>(base), gdim, gstride, box,
                         estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  put(base, key, *out);
  return cudaSuccess;
}

}  // namespace g4
