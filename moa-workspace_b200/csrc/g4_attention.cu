// Sliding-window decode attention over the bf16 ring cache (reference op:
// furiosa-opt-gemma4-12B/src/ops.rs:118-128, device semantics src/device/sliding/attention.rs:7-199).
//
//   s[g,t] = bf16(scale * q[g] . k[t])                      (f32 contraction, bf16 scores)
//   m[g]   = max over ALL t of s[g,t]                       (masked slots included)
//   p[g,t] = min(exp(s[g,t] - m[g]), mask[t])               (0/1 mask row)
//   sum[g] = sum_t p[g,t] + 1e-6
//   out    = bf16( bf16(sum_t bf16(p[g,t]) v[t]) / sum[g] )
//
// One thread-block cluster of kChunks CTAs per KV head (64 CTAs for the 8 heads; a
// tensor-parallel rank holds 8 / n of them in its cache slice), each owning a contiguous run of
// ring slots. A CTA copies its K and V rows into shared memory with TMA boxes of 32 rows, each
// completing on its own barrier so that scoring starts as the first box lands, scores its slots
// for the head's two query heads and computes its score maximum. The rounding
// of p to bf16 depends on the maximum over the WHOLE ring, so the cluster exchanges maxima
// through distributed shared memory (a cluster barrier, then each CTA reads the others') before
// computing p. Each CTA then leaves its partial sum_t p and sum_t bf16(p) v in its shared memory;
// after a second cluster barrier CTA c adds the partials of head dimensions [32c, 32c + 32) over
// the cluster in chunk order, so the result does not depend on timing, and a third barrier keeps
// every CTA's shared memory alive until the others have read it.
#include "g4_ops.cuh"
#include "g4_tc.cuh"

namespace g4 {
namespace {

constexpr int kChunks = 8;                 // CTAs per KV head = the cluster size (portable)
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowBytes = kDs * 2;         // one head's row in one slot
constexpr int kSub = 128;                  // slots resident in shared memory per pass
constexpr int kBox = 32;                   // slots per TMA box, each with its own barrier
constexpr int kBoxes = kSub / kBox;
constexpr int kMaxRing = 8192;
constexpr int kMaxPer = kMaxRing / kChunks;
constexpr int kDimsPerCta = kDs / kChunks; // head dimensions each CTA combines

struct AttnSmem {
  uint8_t k[kSub * kRowBytes];
  uint8_t v[kSub * kRowBytes];
  float score[kMaxPer][kGs];  // scores, then bf16-rounded probabilities
  float red[kWarps][kGs];
  float cmax[kGs];            // this CTA's score maxima (read by the cluster)
  float po[kGs][kDs];         // this CTA's partial sum_t bf16(p) v (read by the cluster)
  float pz[kGs];              // and sum_t p
  __align__(16) uint16_t out[kGs * kDimsPerCta];
  uint64_t kbar[kBoxes], vbar[kBoxes];
};

struct KvMaps {
  CUtensorMap k, v;  // [ring][heads][dim] as (dim, head, slot), box {dim, 1, kBox}
};

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// A float of CTA `rank`'s shared memory at the address this CTA's copy of the object has.
__device__ __forceinline__ float ld_cluster_f32(const void* own, uint32_t rank) {
  uint32_t a;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(own)), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads, 1) attention_kernel(const __grid_constant__ KvMaps maps, AttnArgs a,
                                                                Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  AttnSmem& sm = *reinterpret_cast<AttnSmem*>(smem_raw);
  const int head = blockIdx.x / kChunks;
  const int chunk = int(cluster_ctarank());  // == blockIdx.x % kChunks
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = a.ring_len / kChunks;  // a multiple of 32, at most kMaxPer
  const int slot0 = chunk * per;
  const int passes = (per + kSub - 1) / kSub;
  volatile uint32_t abort_flag = 0;  // this CTA's own waits only
  G4_STAMP(sc, 0);
  if (tid < kBoxes) {
    mbar_init(&sm.kbar[tid], 1);
    mbar_init(&sm.vbar[tid], 1);
    fence_mbar_init();
  }
  // While the preceding QKV op finishes, bring this CTA's K and V rows into L2: it writes one
  // slot of them, but L2 is coherent, so the copies below (after the wait) still read its rows.
  for (int b = tid; b < 2 * (per / kBox); b += kThreads) {
    const int nb = per / kBox;
    tma_prefetch_l2_3d(b < nb ? &maps.k : &maps.v, 0, head, slot0 + (b < nb ? b : b - nb) * kBox);
  }
  __syncthreads();

  pdl_wait_primary();  // q and the cache rows come from the preceding QKV op
  pdl_launch_dependents();
  G4_STAMP(sc, 1);

  // rows [first, first + count) of a cache into a shared-memory buffer: box b (kBox rows) by
  // thread b, completing on its own barrier, so the rows can be used as their box lands
  const uint64_t policy = l2_evict_first_policy();  // each row is read once per step
  auto fetch = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* bars, int first, int count) {
    const int b = tid;
    if (b < count / kBox) {
      mbar_arrive_expect_tx(&bars[b], uint32_t(kBox) * kRowBytes);
      tma_load_3d(dst + b * kBox * kRowBytes, map, 0, head, slot0 + first + b * kBox, &bars[b], policy);
    }
  };
  fetch(&maps.k, sm.k, sm.kbar, 0, per < kSub ? per : kSub);
  if (passes == 1) fetch(&maps.v, sm.v, sm.vbar, 0, per);

  // phase 1: scores, kSub slots at a time. The 8 lanes 8i .. 8i + 7 of a warp score one slot,
  // so a warp scores 4 slots per step (one box of 32 slots per step of the 8 warps). Lane
  // `part` of a slot holds head dimensions c 64 + 8 part + j (c < 4, j < 8): for each c the 8
  // lanes read 128 contiguous bytes of the row.
  constexpr int kLanesPerSlot = 8, kSlotsPerStep = 32 / kLanesPerSlot;
  static_assert(kWarps * kSlotsPerStep == kBox, "one box per step of the CTA");
  const int sub = lane / kLanesPerSlot, part = lane % kLanesPerSlot;
  float qv[kGs][32];
#pragma unroll
  for (int g = 0; g < kGs; ++g) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(a.q + (head * kGs + g) * kDs + c * 64 + part * 8));
      const uint16_t* b = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) qv[g][c * 8 + j] = bf16_to_f32(b[j]);
    }
  }
  bool ok = true;
  for (int p = 0; p < passes; ++p) {
    const int first = p * kSub, rows = per - first < kSub ? per - first : kSub;
    if (p > 0) {
      __syncthreads();  // the previous pass is done with the K buffer
      fetch(&maps.k, sm.k, sm.kbar, first, rows);
    }
    for (int b = 0; b < rows / kBox; ++b) {
      if (ok) ok = mbar_wait_or_abort(&sm.kbar[b], uint32_t(p & 1), &abort_flag, sc.err);
      const int t = b * kBox + warp * kSlotsPerStep + sub;
      const uint8_t* row = sm.k + t * kRowBytes + part * 16;
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 kr = *reinterpret_cast<const uint4*>(row + c * 128);
        const uint16_t* kb = reinterpret_cast<const uint16_t*>(&kr);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float kf = bf16_to_f32(kb[j]);
          d0 = fmaf(qv[0][c * 8 + j], kf, d0);
          d1 = fmaf(qv[1][c * 8 + j], kf, d1);
        }
      }
#pragma unroll
      for (int o = kLanesPerSlot / 2; o; o >>= 1) {
        d0 += __shfl_xor_sync(0xffffffffu, d0, o);
        d1 += __shfl_xor_sync(0xffffffffu, d1, o);
      }
      if (part == 0) {
        sm.score[first + t][0] = bf16_round(a.scale * d0);
        sm.score[first + t][1] = bf16_round(a.scale * d1);
      }
    }
  }
  __syncthreads();
  G4_STAMP(sc, 2);

  // this CTA's maximum; then the head's maximum over the cluster (distributed shared memory)
  float m0 = -INFINITY, m1 = -INFINITY;
  for (int t = tid; t < per; t += kThreads) {
    m0 = fmaxf(m0, sm.score[t][0]);
    m1 = fmaxf(m1, sm.score[t][1]);
  }
  m0 = warp_max(m0);
  m1 = warp_max(m1);
  if (lane == 0) {
    sm.red[warp][0] = m0;
    sm.red[warp][1] = m1;
  }
  __syncthreads();
  if (tid < kGs) {
    float m = -INFINITY;
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, sm.red[w][tid]);
    sm.cmax[tid] = m;
  }
  cluster_sync();  // every CTA's maxima are in its shared memory
  float gm[kGs];
#pragma unroll
  for (int g = 0; g < kGs; ++g) {
    float pm[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) pm[c] = ld_cluster_f32(&sm.cmax[g], uint32_t(c));
    gm[g] = -INFINITY;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) gm[g] = fmaxf(gm[g], pm[c]);
  }
  G4_STAMP(sc, 3);

  // probabilities and this CTA's denominator (fixed summation order)
  float s0 = 0.f, s1 = 0.f;
  for (int t = tid; t < per; t += kThreads) {
    const float mk = a.mask[slot0 + t];
    const float p0 = fminf(expf(sm.score[t][0] - gm[0]), mk);
    const float p1 = fminf(expf(sm.score[t][1] - gm[1]), mk);
    s0 += p0;
    s1 += p1;
    sm.score[t][0] = bf16_round(p0);
    sm.score[t][1] = bf16_round(p1);
  }
  s0 = warp_sum(s0);
  s1 = warp_sum(s1);
  __syncthreads();  // every read of sm.red (the maxima) is done
  if (lane == 0) {
    sm.red[warp][0] = s0;
    sm.red[warp][1] = s1;
  }
  __syncthreads();
  G4_STAMP(sc, 4);

  // phase 2: o[g][d] = sum_t bf16(p[g][t]) v[t][d]; thread d owns dimension d of both heads
  float o0 = 0.f, o1 = 0.f;
  for (int p = 0; p < passes; ++p) {
    const int first = p * kSub, rows = per - first < kSub ? per - first : kSub;
    if (passes > 1) {
      __syncthreads();  // the previous pass is done with the V buffer
      fetch(&maps.v, sm.v, sm.vbar, first, rows);
    }
    for (int b = 0; b < rows / kBox; ++b) {
      if (ok) ok = mbar_wait_or_abort(&sm.vbar[b], uint32_t(p & 1), &abort_flag, sc.err);
#pragma unroll 8
      for (int t = b * kBox; t < (b + 1) * kBox; ++t) {
        const float vf = bf16_to_f32(reinterpret_cast<const uint16_t*>(sm.v + t * kRowBytes)[tid]);
        o0 = fmaf(sm.score[first + t][0], vf, o0);
        o1 = fmaf(sm.score[first + t][1], vf, o1);
      }
    }
  }
  sm.po[0][tid] = o0;
  sm.po[1][tid] = o1;
  if (tid < kGs) {
    float z = 0.f;
    for (int w = 0; w < kWarps; ++w) z += sm.red[w][tid];
    sm.pz[tid] = z;
  }
  cluster_sync();  // every CTA's partials are in its shared memory
  G4_STAMP(sc, 5);

  // CTA `chunk` combines dimensions [32 chunk, 32 chunk + 32) of both query heads, chunks in order
  if (tid < kGs * kDimsPerCta) {
    const int g = tid / kDimsPerCta, d = chunk * kDimsPerCta + tid % kDimsPerCta;
    float po[kChunks], pz[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {  // every load in flight at once
      po[c] = ld_cluster_f32(&sm.po[g][d], uint32_t(c));
      pz[c] = ld_cluster_f32(&sm.pz[g], uint32_t(c));
    }
    float o = 0.f, z = 0.f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      o += po[c];
      z += pz[c];
    }
    sm.out[tid] = f32_to_bf16(bf16_round(o) / (z + kEps));
  }
  cluster_sync();  // the others are done reading this CTA's partials (and sm.out is complete)
  if (tid < kGs * kDimsPerCta * 2 / 16) {  // 16-byte stores: 4 per query head
    const int g = tid / (kDimsPerCta * 2 / 16), q = tid % (kDimsPerCta * 2 / 16);
    reinterpret_cast<uint4*>(a.out + (head * kGs + g) * kDs + chunk * kDimsPerCta)[q] =
        reinterpret_cast<const uint4*>(sm.out + g * kDimsPerCta)[q];
  }
  G4_STAMP(sc, 6);
}

}  // namespace

cudaError_t prepare_attention_kernels() {
  return cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(AttnSmem)));
}

int attention_slot_multiple() { return kChunks * 32; }
int attention_max_ring() { return kMaxRing; }

cudaError_t launch_attention(const AttnArgs& a, const LaunchEnv& env) {
  KvMaps maps;
  cudaError_t e;
  if (a.heads < 1 || a.heads > kNs) return cudaErrorInvalidValue;
  if ((e = env.maps->kv(a.k_cache, uint64_t(a.ring_len), uint32_t(a.heads), kDs, uint32_t(kBox), &maps.k))) return e;
  if ((e = env.maps->kv(a.v_cache, uint64_t(a.ring_len), uint32_t(a.heads), kDs, uint32_t(kBox), &maps.v))) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.heads * kChunks);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(AttnSmem);
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // one cluster per KV head
  attr[1].val.clusterDim.x = kChunks;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  Scratch sc = env.sc;
#ifdef G4_TRACE
  if (sc.trace) sc.trace += 4096;  // profiling builds: separate stamp rows per kernel
#endif
  return cudaLaunchKernelEx(&cfg, attention_kernel, maps, a, sc);
}

}  // namespace g4
