// Sliding-window decode attention over the bf16 ring cache (reference op:
// furiosa-opt-gemma4-12B/src/ops.rs:118-128, device semantics src/device/sliding/attention.rs:7-199).
//
//   s[g,t] = bf16(scale * q[g] . k[t])                      (f32 contraction, bf16 scores)
//   m[g]   = max over ALL t of s[g,t]                       (masked slots included)
//   p[g,t] = min(exp(s[g,t] - m[g]), mask[t])               (0/1 mask row)
//   sum[g] = sum_t p[g,t] + 1e-6
//   out    = bf16( bf16(sum_t bf16(p[g,t]) v[t]) / sum[g] )
//
// One thread-block cluster of CL CTAs per KV head (CL = 16 where the GPU schedules clusters
// of 16, else 8); each CTA owns a contiguous run of ring slots. At entry every CTA starts
// copying its V rows into shared memory (cp.async, no registers held) and loads its K rows
// straight into registers, so the whole working set is requested in one round trip. The CTAs
// exchange their score maxima and output partials through distributed shared memory; rank 0
// adds the partials in rank order, so the result equals one pass over the ring and does not
// depend on timing.
#include <cooperative_groups.h>

#include "g4_ops.cuh"

namespace cg = cooperative_groups;

namespace g4 {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kRowBytes = kDs * 2;      // one head's row in one slot
constexpr int kVChunk = 256;            // V rows resident in shared memory at a time (128 KB)
constexpr int kKBatch = 16;             // K rows per warp held in registers at a time
constexpr int kMaxSlotsPerCta = 1024;   // scores kept for the whole run of a CTA

struct AttnSmem {
  uint8_t v[kVChunk * kRowBytes];
  float score[kMaxSlotsPerCta][kGs];  // scores, then bf16-rounded probabilities
  float opart[4][kGs][kDs];           // four slot residues, reduced before publishing
  float pub_max[kGs];
  float pub_sum[kGs];
  float red[kWarps][kGs];
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <int CL>
__global__ void __launch_bounds__(kThreads, 1) attention_kernel(AttnArgs a, Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  AttnSmem& sm = *reinterpret_cast<AttnSmem*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = int(cluster.block_rank());
  const int head = blockIdx.x / CL;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per_cta = a.ring_len / CL;      // <= kMaxSlotsPerCta, a multiple of kWarps
  const int per_warp = per_cta / kWarps;
  const int slot0 = rank * per_cta;
  G4_STAMP(sc, 0);

  pdl_wait_primary();  // q and the cache rows come from the preceding QKV op
  pdl_launch_dependents();
  G4_STAMP(sc, 1);

  // V rows [first, first + count) of this CTA -> shared memory, asynchronously (16 B per request)
  auto fetch_v = [&](int first, int count) {
    const int chunks = count * (kRowBytes / 16);
    for (int c = tid; c < chunks; c += kThreads) {
      const int r = c / (kRowBytes / 16), o = c % (kRowBytes / 16);
      cp_async16(sm.v + r * kRowBytes + o * 16,
                 reinterpret_cast<const uint8_t*>(a.v_cache + (size_t(slot0 + first + r) * kNs + head) * kDs) + o * 16);
    }
    cp_async_commit();
  };
  fetch_v(0, per_cta < kVChunk ? per_cta : kVChunk);

  // q rows of the two query heads of this KV head: lane holds dims 8*lane .. 8*lane+7
  float qv[kGs][8];
#pragma unroll
  for (int g = 0; g < kGs; ++g) {
    const uint4 raw = *reinterpret_cast<const uint4*>(a.q + (head * kGs + g) * kDs + lane * 8);
    const uint16_t* b = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) qv[g][j] = bf16_to_f32(b[j]);
  }

  // phase 1: this warp's K rows straight into registers (kKBatch at a time), then its scores
  const int wslot0 = warp * per_warp;
  for (int kb0 = 0; kb0 < per_warp; kb0 += kKBatch) {
    uint4 kr[kKBatch];
#pragma unroll
    for (int r = 0; r < kKBatch; ++r)
      if (kb0 + r < per_warp)
        kr[r] = __ldcs(reinterpret_cast<const uint4*>(a.k_cache + (size_t(slot0 + wslot0 + kb0 + r) * kNs + head) * kDs) +
                       lane);
#pragma unroll
    for (int r = 0; r < kKBatch; ++r) {
      if (kb0 + r < per_warp) {
        const uint16_t* kb = reinterpret_cast<const uint16_t*>(&kr[r]);
        float d0 = 0.f, d1 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float kf = bf16_to_f32(kb[j]);
          d0 = fmaf(qv[0][j], kf, d0);
          d1 = fmaf(qv[1][j], kf, d1);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          d0 += __shfl_xor_sync(0xffffffffu, d0, o);
          d1 += __shfl_xor_sync(0xffffffffu, d1, o);
        }
        if (lane == 0) {
          sm.score[wslot0 + kb0 + r][0] = bf16_round(a.scale * d0);
          sm.score[wslot0 + kb0 + r][1] = bf16_round(a.scale * d1);
        }
        __syncwarp();
      }
    }
  }
  __syncthreads();
  G4_STAMP(sc, 2);

  // global max over the whole ring (every CTA of the cluster)
  float m0 = -INFINITY, m1 = -INFINITY;
  for (int t = tid; t < per_cta; t += kThreads) {
    m0 = fmaxf(m0, sm.score[t][0]);
    m1 = fmaxf(m1, sm.score[t][1]);
  }
  m0 = warp_max(m0);
  m1 = warp_max(m1);
  if (lane == 0) {
    sm.red[warp][0] = m0;
    sm.red[warp][1] = m1;
  }
  __syncwarp();
  __syncthreads();
  if (tid == 0) {
    float a0 = -INFINITY, a1 = -INFINITY;
    for (int w = 0; w < kWarps; ++w) {
      a0 = fmaxf(a0, sm.red[w][0]);
      a1 = fmaxf(a1, sm.red[w][1]);
    }
    sm.pub_max[0] = a0;
    sm.pub_max[1] = a1;
  }
  __syncwarp();
  cluster.sync();
  float gm0 = -INFINITY, gm1 = -INFINITY;
  for (int r = 0; r < CL; ++r) {
    const float* pm = cluster.map_shared_rank(sm.pub_max, r);
    gm0 = fmaxf(gm0, pm[0]);
    gm1 = fmaxf(gm1, pm[1]);
  }
  G4_STAMP(sc, 3);

  // probabilities and the local denominator (fixed summation order)
  float s0 = 0.f, s1 = 0.f;
  for (int t = tid; t < per_cta; t += kThreads) {
    const float mk = a.mask[slot0 + t];
    const float p0 = fminf(expf(sm.score[t][0] - gm0), mk);
    const float p1 = fminf(expf(sm.score[t][1] - gm1), mk);
    s0 += p0;
    s1 += p1;
    sm.score[t][0] = bf16_round(p0);
    sm.score[t][1] = bf16_round(p1);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
  }
  __syncthreads();  // every read of sm.red (the maxima) is done
  if (lane == 0) {
    sm.red[warp][0] = s0;
    sm.red[warp][1] = s1;
  }
  __syncwarp();
  cp_async_wait_all();
  __syncthreads();
  if (tid == 0) {
    float a0 = 0.f, a1 = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      a0 += sm.red[w][0];
      a1 += sm.red[w][1];
    }
    sm.pub_sum[0] = a0;
    sm.pub_sum[1] = a1;
  }
  __syncwarp();
  G4_STAMP(sc, 4);

  // phase 2: o = sum_t bf16(p) v. Thread (res, pair) covers dims 2*pair, 2*pair+1 of both
  // query heads over the slots t = res (mod 4), one resident chunk of V rows at a time.
  {
    const int res = tid >> 7, pair = tid & 127;
    float o00 = 0.f, o01 = 0.f, o10 = 0.f, o11 = 0.f;
    for (int c0 = 0; c0 < per_cta; c0 += kVChunk) {
      const int rows = per_cta - c0 < kVChunk ? per_cta - c0 : kVChunk;
      if (c0 > 0) {  // later chunks of a long ring: refill the buffer
        __syncthreads();
        fetch_v(c0, rows);
        cp_async_wait_all();
        __syncthreads();
      }
      for (int t = res; t < rows; t += 4) {
        const uint32_t vv = *reinterpret_cast<const uint32_t*>(sm.v + t * kRowBytes + pair * 4);
        const float v0 = bf16_to_f32(uint16_t(vv & 0xffff)), v1 = bf16_to_f32(uint16_t(vv >> 16));
        const float w0 = sm.score[c0 + t][0], w1 = sm.score[c0 + t][1];
        o00 = fmaf(w0, v0, o00);
        o01 = fmaf(w0, v1, o01);
        o10 = fmaf(w1, v0, o10);
        o11 = fmaf(w1, v1, o11);
      }
    }
    sm.opart[res][0][2 * pair] = o00;
    sm.opart[res][0][2 * pair + 1] = o01;
    sm.opart[res][1][2 * pair] = o10;
    sm.opart[res][1][2 * pair + 1] = o11;
  }
  __syncthreads();
  {
    const int g = tid >> 8, d = tid & 255;
    sm.opart[0][g][d] = ((sm.opart[0][g][d] + sm.opart[1][g][d]) + sm.opart[2][g][d]) + sm.opart[3][g][d];
  }
  cluster.sync();
  G4_STAMP(sc, 5);

  if (rank == 0) {
    const int g = tid >> 8, d = tid & 255;
    float o = 0.f, z = 0.f;
    for (int r = 0; r < CL; ++r) {
      const float* op = cluster.map_shared_rank(&sm.opart[0][0][0], r);
      const float* ps = cluster.map_shared_rank(sm.pub_sum, r);
      o += op[g * kDs + d];
      z += ps[g];
    }
    z += kEps;
    a.out[(head * kGs + g) * kDs + d] = f32_to_bf16(bf16_round(o) / z);
  }
  cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
  G4_STAMP(sc, 6);
}

int g_cluster = 0;  // 16 or 8, decided once per process

}  // namespace

cudaError_t prepare_attention_kernels() {
  cudaError_t e = cudaFuncSetAttribute(attention_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(sizeof(AttnSmem)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_kernel<16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(AttnSmem)));
  if (e != cudaSuccess) return e;
  if (g_cluster == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kNs * 16);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sizeof(AttnSmem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 16;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    const cudaError_t q = cudaOccupancyMaxActiveClusters(&clusters, attention_kernel<16>, &cfg);
    // 16-CTA clusters only when all kNs of them fit on the GPU at once
    g_cluster = (q == cudaSuccess && clusters >= kNs) ? 16 : 8;
    if (q != cudaSuccess) (void)cudaGetLastError();
  }
  return cudaSuccess;
}

int attention_slot_multiple() { return (g_cluster ? g_cluster : 8) * kWarps; }
int attention_max_ring() { return 8 * kMaxSlotsPerCta; }

cudaError_t launch_attention(const AttnArgs& a, const LaunchEnv& env) {
  const int cl = g_cluster ? g_cluster : 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kNs * cl);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(AttnSmem);
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  Scratch sc = env.sc;
#ifdef G4_TRACE
  if (sc.trace) sc.trace += 4096;  // profiling builds: separate stamp rows per kernel
#endif
  return cl == 16 ? cudaLaunchKernelEx(&cfg, attention_kernel<16>, a, sc)
                  : cudaLaunchKernelEx(&cfg, attention_kernel<8>, a, sc);
}

}  // namespace g4
