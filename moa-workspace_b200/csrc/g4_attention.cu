// Sliding-window decode attention over the bf16 ring cache (reference op:
// furiosa-opt-gemma4-12B/src/ops.rs:118-128, device semantics src/device/sliding/attention.rs:7-199).
//
//   s[g,t] = bf16(scale * q[g] . k[t])                      (f32 contraction, bf16 scores)
//   m[g]   = max over ALL t of s[g,t]                       (masked slots included)
//   p[g,t] = min(exp(s[g,t] - m[g]), mask[t])               (0/1 mask row)
//   sum[g] = sum_t p[g,t] + 1e-6
//   out    = bf16( bf16(sum_t bf16(p[g,t]) v[t]) / sum[g] )
//
// One thread-block cluster of kClusterCtas CTAs per KV head; each CTA owns a contiguous
// run of ring slots, streams that run's K rows and then its V rows through a TMA bulk-copy
// ring, and the CTAs exchange their score maxima and output partials through distributed
// shared memory, so the result equals a single pass over the whole ring (partials are
// combined in rank order: deterministic).
#include <cooperative_groups.h>

#include "g4_ops.cuh"

namespace cg = cooperative_groups;

namespace g4 {
namespace {

constexpr int kClusterCtas = 8;
constexpr int kTile = 32;            // ring slots per bulk-copy tile
constexpr int kStages = 4;           // tiles in flight per CTA
constexpr int kThreads = 256;
constexpr int kRowBytes = kDs * 2;   // one head's row in one slot
constexpr int kTileBytes = kTile * kRowBytes;
constexpr int kMaxSlotsPerCta = 1024;

struct AttnSmem {
  uint8_t ring[kStages][kTileBytes];
  float score[kGs][kMaxSlotsPerCta];  // scores, then bf16-rounded probabilities
  float opart[kGs][kDs];
  float pub_max[kGs];
  float pub_sum[kGs];
  float red[kThreads / 32][kGs];
  uint64_t bars[kStages];
};

__global__ void __launch_bounds__(kThreads, 1) attention_kernel(AttnArgs a, Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  AttnSmem& sm = *reinterpret_cast<AttnSmem*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = int(cluster.block_rank());
  const int head = blockIdx.x / kClusterCtas;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per_cta = a.ring_len / kClusterCtas;
  const int n_tiles = per_cta / kTile;
  const int slot0 = rank * per_cta;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(&sm.bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();

  pdl_wait_primary();  // q and the cache rows come from the preceding QKV op
  pdl_launch_dependents();

  const uint64_t policy = l2_evict_first_policy();
  // tile i < n_tiles: K rows; n_tiles <= i < 2 n_tiles: V rows
  auto issue = [&](int i) {
    if (warp != 0) return;
    const uint16_t* cache = i < n_tiles ? a.k_cache : a.v_cache;
    const int first = slot0 + (i % n_tiles) * kTile;
    uint64_t* bar = &sm.bars[i % kStages];
    if (lane == 0) mbar_arrive_expect_tx(bar, kTileBytes);
    __syncwarp();
    const uint16_t* src = cache + (size_t(first + lane) * kNs + head) * kDs;
    bulk_g2s(sm.ring[i % kStages] + lane * kRowBytes, src, kRowBytes, bar, policy);
  };
  for (int i = 0; i < kStages && i < 2 * n_tiles; ++i) issue(i);

  // q rows of the two query heads of this KV head: lane holds dims 8*lane .. 8*lane+7
  float qv[kGs][8];
#pragma unroll
  for (int g = 0; g < kGs; ++g) {
    const uint4 raw = *reinterpret_cast<const uint4*>(a.q + (head * kGs + g) * kDs + lane * 8);
    const uint16_t* b = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) qv[g][j] = bf16_to_f32(b[j]);
  }

  bool ok = true;
  // phase 1: scores
  for (int i = 0; i < n_tiles; ++i) {
    ok = ok && mbar_wait(&sm.bars[i % kStages], uint32_t((i / kStages) & 1), sc.err);
    if (ok) {
      const uint8_t* tile = sm.ring[i % kStages];
#pragma unroll
      for (int r = 0; r < kTile / (kThreads / 32); ++r) {
        const int row = warp * (kTile / (kThreads / 32)) + r;
        const uint4 raw = *reinterpret_cast<const uint4*>(tile + row * kRowBytes + lane * 16);
        const uint16_t* kb = reinterpret_cast<const uint16_t*>(&raw);
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
          sm.score[0][i * kTile + row] = bf16_round(a.scale * d0);
          sm.score[1][i * kTile + row] = bf16_round(a.scale * d1);
        }
      }
    }
    __syncthreads();
    if (i + kStages < 2 * n_tiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(i + kStages);
    }
  }

  // global max over the whole ring (every CTA of the cluster)
  float m0 = -INFINITY, m1 = -INFINITY;
  for (int t = tid; t < per_cta; t += kThreads) {
    m0 = fmaxf(m0, sm.score[0][t]);
    m1 = fmaxf(m1, sm.score[1][t]);
  }
  m0 = warp_max(m0);
  m1 = warp_max(m1);
  if (lane == 0) {
    sm.red[warp][0] = m0;
    sm.red[warp][1] = m1;
  }
  __syncthreads();
  if (tid == 0) {
    float a0 = -INFINITY, a1 = -INFINITY;
    for (int w = 0; w < kThreads / 32; ++w) {
      a0 = fmaxf(a0, sm.red[w][0]);
      a1 = fmaxf(a1, sm.red[w][1]);
    }
    sm.pub_max[0] = a0;
    sm.pub_max[1] = a1;
  }
  cluster.sync();
  float gm0 = -INFINITY, gm1 = -INFINITY;
  for (int r = 0; r < kClusterCtas; ++r) {
    const float* pm = cluster.map_shared_rank(sm.pub_max, r);
    gm0 = fmaxf(gm0, pm[0]);
    gm1 = fmaxf(gm1, pm[1]);
  }

  // probabilities and the local denominator
  float s0 = 0.f, s1 = 0.f;
  for (int t = tid; t < per_cta; t += kThreads) {
    const float mk = a.mask[slot0 + t];
    const float p0 = fminf(expf(sm.score[0][t] - gm0), mk);
    const float p1 = fminf(expf(sm.score[1][t] - gm1), mk);
    s0 += p0;
    s1 += p1;
    sm.score[0][t] = bf16_round(p0);
    sm.score[1][t] = bf16_round(p1);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
  }
  __syncthreads();  // all reads of sm.red (max) are done
  if (lane == 0) {
    sm.red[warp][0] = s0;
    sm.red[warp][1] = s1;
  }
  __syncthreads();
  if (tid == 0) {
    float a0 = 0.f, a1 = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) {
      a0 += sm.red[w][0];
      a1 += sm.red[w][1];
    }
    sm.pub_sum[0] = a0;
    sm.pub_sum[1] = a1;
  }

  // phase 2: o = sum_t bf16(p) v, one output dim per thread
  float o0 = 0.f, o1 = 0.f;
  for (int i = n_tiles; i < 2 * n_tiles; ++i) {
    ok = ok && mbar_wait(&sm.bars[i % kStages], uint32_t((i / kStages) & 1), sc.err);
    if (ok) {
      const uint16_t* tile = reinterpret_cast<const uint16_t*>(sm.ring[i % kStages]);
      const int base = (i - n_tiles) * kTile;
#pragma unroll 8
      for (int r = 0; r < kTile; ++r) {
        const float vf = bf16_to_f32(tile[r * kDs + tid]);
        o0 = fmaf(sm.score[0][base + r], vf, o0);
        o1 = fmaf(sm.score[1][base + r], vf, o1);
      }
    }
    __syncthreads();
    if (i + kStages < 2 * n_tiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(i + kStages);
    }
  }
  sm.opart[0][tid] = o0;
  sm.opart[1][tid] = o1;
  cluster.sync();

  if (rank == 0) {
    float t0 = 0.f, t1 = 0.f, z0 = 0.f, z1 = 0.f;
    for (int r = 0; r < kClusterCtas; ++r) {
      const float* op = cluster.map_shared_rank(&sm.opart[0][0], r);
      const float* ps = cluster.map_shared_rank(sm.pub_sum, r);
      t0 += op[tid];
      t1 += op[kDs + tid];
      z0 += ps[0];
      z1 += ps[1];
    }
    z0 += kEps;
    z1 += kEps;
    if (ok) {
      a.out[(head * kGs + 0) * kDs + tid] = f32_to_bf16(bf16_round(t0) / z0);
      a.out[(head * kGs + 1) * kDs + tid] = f32_to_bf16(bf16_round(t1) / z1);
    }
  }
  cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
}

}  // namespace

cudaError_t prepare_attention_kernels() {
  return cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(AttnSmem)));
}

int attention_slot_multiple() { return kClusterCtas * kTile; }
int attention_max_ring() { return kClusterCtas * kMaxSlotsPerCta; }

cudaError_t launch_attention(const AttnArgs& a, const LaunchEnv& env) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kNs * kClusterCtas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(AttnSmem);
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, attention_kernel, a, env.sc);
}

}  // namespace g4
