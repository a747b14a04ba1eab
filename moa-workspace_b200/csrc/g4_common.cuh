// Shared device helpers for the Gemma-4 decode-layer kernels (sm_100a).
//
// Shapes follow the reference's axes (furiosa-opt-gemma4-12B/src/axes.rs:1-28):
// H = 3840 hidden, L = 15360 FFN, Ns = 8 KV heads, Gs = 2 query heads per KV head,
// Ds = 256 head dim, Qs = 4096, Ps = 2048, Ts = 1024 ring slots, E = 32768 RoPE rows.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace g4 {

constexpr int kH = 3840;
constexpr int kL = 15360;
constexpr int kNs = 8;
constexpr int kGs = 2;
constexpr int kDs = 256;
constexpr int kQs = kNs * kGs * kDs;  // 4096
constexpr int kPs = kNs * kDs;        // 2048
constexpr int kTs = 1024;
constexpr int kE = 32768;
constexpr int kVocab = 262144;  // W: embedding / lm_head rows
constexpr float kEps = 1e-6f;

// Tensor-parallel geometry (Megatron split over NTP ranks of one node): rank r owns KV heads
// [8r/NTP, 8(r+1)/NTP) with their query heads and ring-cache slice, the matching K columns of
// O, FFN rows [L r/NTP, L (r+1)/NTP) of up and gate and those K columns of down. The O and
// down outputs are the sum of the ranks' partials (one exchange per op). The down K slice is
// zero-padded to whole 256-element units (1920 -> 2048 at NTP = 8).
constexpr int kMaxTp = 8;
template <int NTP>
struct TpGeo {
  static_assert(NTP == 1 || NTP == 2 || NTP == 4 || NTP == 8, "tensor-parallel degree");
  static constexpr int kRanks = NTP;
  static constexpr int kKvHeads = kNs / NTP;
  static constexpr int kQRows = kQs / NTP;   // q projection rows (2 kKvHeads heads)
  static constexpr int kKvRows = kPs / NTP;  // k (and v) projection rows
  static constexpr int kFfnRows = kL / NTP;  // up / gate rows = down K
  static constexpr int kDownK = (kFfnRows + 255) / 256 * 256;
};

// Bits of the device-resident error word (`Scratch::err`). Kernels never trap: a bad
// device-side operand (an out-of-ring cache offset, a timed-out wait) sets a bit and the
// affected writes are skipped; the host reads the word back with g4_ctx_check().
enum : uint32_t {
  kErrKvOffset = 1u << 0,
  kErrRopeOffset = 1u << 1,
  kErrWaitTimeout = 1u << 2,
  kErrInternal = 1u << 3,  // a launch-geometry invariant did not hold (work was skipped)
  kErrNegativeScale = 1u << 4,  // an nvfp4 block scale has its sign bit set
  kErrPeerTimeout = 1u << 5,    // a tensor-parallel peer's partial did not arrive in time
  kErrTokenOffset = 1u << 6,    // an embedding-row offset outside the table or not row-aligned
};

// Global scratch owned by a context. The counters hold each op's call counts (per tile or
// head), which tag its split-K words and tile sums with the call's epoch; they only grow.
struct Scratch {
  uint32_t* err;       // error word
  uint32_t* counters;  // epoch counters (kCounterCount)
  float* partials;     // split-K words of each op (kSplitWords*; the region is sized in floats)
  uint16_t* act;       // bf16 GeGLU activation [M][L]
  unsigned long long* tile_ss;  // per output tile: sum of squares of its bf16 rows, as two words
                                // (epoch << 32 | low / high half of the f64), kTileSsCount tiles
  uint64_t* trace;     // per-CTA phase timestamps (profiling builds only; null otherwise)
  // the token-batched feed-forward (M > 1): its normalised input h [kBatchMax][H] (f16, scaled by a
  // power of two per token), those factors' inverses, and the split-K words [CTA][2 pieces]
  // [kBatchMax tokens][128 rows]
  uint16_t* batch_h;
  float* batch_unscale;  // [kBatchMax]: 2^-k of each token's f16 scaling of h
  unsigned long long* batch_words;
  // the term-operand path of FP8 weights at up to kTermTokens tokens: each token's activation as
  // exact e4m3 terms, [units][kTermTokens padded tokens][kTerms terms][256 bytes], and each
  // (unit, token)'s 2^-E
  uint8_t* batch_terms;
  float* batch_texp;
};
constexpr int kBatchMax = 64;  // tokens per batched feed-forward call
constexpr int kTermTokens = 16;   // the term-operand path's largest batch
constexpr int kTerms = 4;         // e4m3 terms per activation element (the term-operand path)
constexpr int kTermUnitsMax = 60;  // 256-element units of the longest activation (the FFN's 15360)
// the batched feed-forward's call count (tags its split-K words and tile sums)
constexpr int kBatchEpoch = 4080;
constexpr int kTileSsCount = 64;
// One region of tile sums per op (O, down), in words from `tile_ss`: the ops count their calls
// separately, so a word of one op must never be read by the other.
constexpr size_t kTileSsO = 0;
constexpr size_t kTileSsDown = size_t(kTileSsCount) * 2;
constexpr size_t kTileSsBytes = 2 * size_t(kTileSsCount) * 2 * sizeof(unsigned long long);

// Tensor-parallel exchange (one-shot all-reduce of the O / down partials over NVLink peer
// memory). Every rank owns one exchange buffer, mapped into every peer's address space:
//   words [op][parity][tile][source rank][row], 8 bytes = (tag << 32) | f32 bits,
// written by the source with one 64-bit store, so a reader that sees the call's tag sees the
// value too. The tag is (generation << 24) | (epoch & 0xFFFFFF). Each rank counts its calls per
// (op, tile) in `epoch` (local, never shared): the n-th call writes epoch n into parity n & 1. A
// source can be at most one call ahead of a reader per (op, tile): its next call's exchange needs
// the reader's contribution of this call, which the reader posts only after its previous kernels
// completed. The generation changes with every setup of the group (all ranks agree on it), so a
// word that a peer of an earlier setup stored late never matches a call of the new one.
constexpr int kTpOps = 2;      // 0: O projection, 1: FFN down
constexpr int kTpTiles = 30;   // H / 128 output tiles
constexpr size_t kTpExchangeWords = size_t(kTpOps) * 2 * kTpTiles * kMaxTp * 128;
struct TpLink {
  int rank, world;                                 // world 1: no exchange
  unsigned long long* slots[kMaxTp];               // rank s's exchange buffer (this process's mapping)
  uint32_t* epoch;                                 // [op][tile] calls so far (this rank's memory)
  uint32_t generation;                             // 1..255: this setup of the group
  uint64_t wait_ns;                                // limit of the wait for the peers' words
};
__host__ __device__ constexpr uint32_t tp_tag(uint32_t generation, uint32_t epoch) {
  return (generation << 24) | (epoch & 0xFFFFFFu);
}
constexpr size_t kScratchHeadBytes = 256;  // the error word, padded to the scratch alignment
constexpr int kCounterCount = 4096;
constexpr int kSplitEpochUpGate = 0;     // calls so far, per tile: up/gate (240 tiles), ...
constexpr int kTailEpochO = 3840;        // ... O and down (30 each; split-K and residual tail)
constexpr int kTailEpochDown = 3872;
constexpr int kHeadEpochBase = 3968;    // ... and QKV heads (32)
constexpr int kFullHeadEpochBase = 4000; // ... and the global layers' QKV heads (17)
constexpr size_t kPartialFloats = size_t(1) << 21;  // 8 MiB of split-K partials
// Split-K slots of each op: [tile][CTA of the tile][128 rows] epoch-tagged words (offsets in words
// from `partials`); one region per op, so a word of one op never reads as another op's.
constexpr size_t kSplitWordsO = 0;
constexpr size_t kSplitWordsDown = size_t(1) << 16;
constexpr size_t kSplitWordsQkv = size_t(1) << 17;
constexpr size_t kSplitWordsUpGate = size_t(1) << 18;
constexpr size_t kSplitWordsFullQkv = size_t(3) << 18;  // 68 tiles x 16 x 128 words, below 1 << 20
// Global (full-attention) layers: 16 query heads and one K = V head of 512 (the reference's Gf,
// Df, Qf = Gf * Df, Pf = Df) over pages of Tf = 512 slots.
constexpr int kGf = 16;
constexpr int kDf = 512;
constexpr int kQf = kGf * kDf;
constexpr int kTf = 512;

// ---------------------------------------------------------------------------------------
// bf16 / f16 / fp8 / fp4 conversions

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// Round-to-nearest-even f32 -> bf16 bits (inputs here are finite; NaN is kept quiet).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float bf16_round(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// f32 with the given unbiased exponent (exact power of two, normal range only).
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float(uint32_t(e + 127) << 23); }

// ---------------------------------------------------------------------------------------
// mbarrier + TMA bulk copy (global -> shared), no multicast.

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of a barrier phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for a barrier phase with a time limit. A copy that never lands (it cannot, for a
// valid address) would otherwise hang the SM; after the limit the wait gives up, raises
// kErrWaitTimeout and the caller abandons its remaining work.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(err, kErrWaitTimeout);
      return false;
    }
  }
  return true;
}

// L2 policy for weights that are read exactly once per call.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 1-D bulk copy: `bytes` (multiple of 16, both addresses 16-byte aligned) land in shared
// memory and complete `bytes` of transaction count on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue, and
// wait for the previous kernel's results before reading them.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_primary() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// System-scope 64-bit accesses for the tensor-parallel exchange words (peer memory over NVLink).
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The same at GPU scope (words other CTAs of this GPU write).
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// 16 bytes global (L2) -> shared memory without a register round trip; wait with cp_async_wait_all.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}

// Phase timestamps for profiling builds (-DG4_TRACE): thread 0 of each CTA records
// %globaltimer at numbered points of a kernel into trace[blockIdx.x * 16 + point].
#ifdef G4_TRACE
#define G4_STAMP(sc, point)                                                                     \
  do {                                                                                          \
    if ((sc).trace && threadIdx.x == 0) (sc).trace[blockIdx.x * 16 + (point)] = globaltimer_ns(); \
  } while (0)
// G4_STAMP_T records from whichever single thread calls it.
#define G4_STAMP_T(sc, point)                                                      \
  do {                                                                            \
    if ((sc).trace) (sc).trace[blockIdx.x * 16 + (point)] = globaltimer_ns();     \
  } while (0)
// Per-warp stamps go to trace[65536 + (blockIdx.x * 32 + warp) * 8 + point] (lane 0).
#define G4_STAMP_WARP(sc, point)                                                                         \
  do {                                                                                                   \
    if ((sc).trace && (threadIdx.x & 31) == 0)                                                           \
      (sc).trace[65536 + (blockIdx.x * 32 + (threadIdx.x >> 5)) * 8 + (point)] = globaltimer_ns();       \
  } while (0)
#else
#define G4_STAMP(sc, point) \
  do {                      \
  } while (0)
#define G4_STAMP_T(sc, point) \
  do {                        \
  } while (0)
#define G4_STAMP_WARP(sc, point) \
  do {                           \
  } while (0)
#endif

// ---------------------------------------------------------------------------------------
// The token embedding: out = bf16(f32(row) * EMBED_SCALE) for one row of the table, the threads
// of the calling block striding over its 16-byte chunks (the reference op: ops.rs:8-35; the scale
// is the device op's f32 constant, src/lib.rs:23).
constexpr float kEmbedScale = 61.967734f;
__device__ __forceinline__ void embed_row(const uint16_t* __restrict__ row, uint16_t* out) {
  for (int c = threadIdx.x; c < kH * 2 / 16; c += blockDim.x) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(row) + c);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = __uint_as_float(w[i] << 16) * kEmbedScale;
      const float hi = __uint_as_float(w[i] & 0xffff0000u) * kEmbedScale;
      o[i] = uint32_t(f32_to_bf16(lo)) | (uint32_t(f32_to_bf16(hi)) << 16);
    }
    reinterpret_cast<uint4*>(out)[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // F.gelu(approximate="tanh"): 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 * x^3)))
  const float cube = x * x * x;
  const float inner = 0.7978845608028654f * (x + 0.044715f * cube);
  return 0.5f * x * (1.0f + tanhf(inner));
}

// ---------------------------------------------------------------------------------------
// Reductions

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions; `red` needs blockDim.x / 32 doubles of shared memory.
__device__ __forceinline__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncwarp();
  __syncthreads();
  double t = 0.0;
  for (int i = 0; i < nw; ++i) t += red[i];  // fixed order: identical in every CTA
  return t;
}

// RMSNorm statistics exactly as the reference computes them (gemma4.py:83-89): the mean of
// squares of bf16 values, accumulated without loss in f64 and narrowed to f32, then
// 1/sqrt(ms + eps) with IEEE-rounded sqrt and divide.
__device__ __forceinline__ float rms_inverse(double sumsq, int n) {
  const float ms = static_cast<float>(sumsq / static_cast<double>(n));
  return 1.0f / sqrtf(ms + kEps);
}

// Global partial slots per split tile (a tile's K range spans at most this many CTAs).
constexpr int kMaxCtasPerGroup = 16;

}  // namespace g4
