// Sliding-window decode attention over the bf16 ring cache (reference op:
// furiosa-opt-gemma4-12B/src/ops.rs:118-128, device semantics src/device/sliding/attention.rs:7-199).
//
//   s[g,t] = bf16(scale * q[g] . k[t])                      (f32 contraction, bf16 scores)
//   m[g]   = max over ALL t of s[g,t]                       (masked slots included)
//   p[g,t] = min(exp(s[g,t] - m[g]), mask[t])               (0/1 mask row)
//   sum[g] = sum_t p[g,t] + 1e-6
//   out    = bf16( bf16(sum_t bf16(p[g,t]) v[t]) / sum[g] )
//
// kChunks CTAs per KV head (128 CTAs for the 8 heads; a tensor-parallel rank holds 8 / n of
// them in its cache slice), each owning a contiguous run of ring slots.
// A CTA copies its K and V rows into shared memory with TMA boxes of up to 128 rows,
// scores its slots for the head's two query heads, and publishes its score maximum. The rounding
// of p to bf16 depends on the maximum over the WHOLE ring, so the head's CTAs exchange maxima
// through global memory (a bounded wait on a per-head generation counter: the 128 CTAs are all
// resident, one per SM) before computing p. Each CTA then publishes its partial sum_t p and
// sum_t bf16(p) v; the last CTA of the head (ticket) adds the partials in chunk order, so the
// result does not depend on timing.
#include "g4_ops.cuh"
#include "g4_tc.cuh"

namespace g4 {
namespace {

constexpr int kChunks = 16;                // CTAs per KV head
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowBytes = kDs * 2;         // one head's row in one slot
constexpr int kSub = 128;                  // slots resident in shared memory per pass
constexpr int kMaxRing = 8192;
constexpr int kMaxPer = kMaxRing / kChunks;
constexpr int kAttnBarrier = 3900;         // counters: per-head max-exchange generations
constexpr int kAttnTicket = 3908;          // counters: per-head output tickets
constexpr size_t kAttnPartials = size_t(1) << 20;  // float offset into the partials scratch
constexpr int kPartFloats = 2 * kDs + 4;   // per (head, chunk): o[2][256], max[2], sum[2]

struct AttnSmem {
  uint8_t k[kSub * kRowBytes];
  uint8_t v[kSub * kRowBytes];
  float score[kMaxPer][kGs];  // scores, then bf16-rounded probabilities
  float red[kWarps][kGs];
  float gmax[kGs];
  __align__(16) uint16_t out[kGs * kDs];
  uint64_t kbar, vbar;
  uint32_t last;
};

struct KvMaps {
  CUtensorMap k, v;  // [ring][heads][dim] as (dim, head, slot), box {dim, 1, box_slots}
};

__global__ void __launch_bounds__(kThreads, 1) attention_kernel(const __grid_constant__ KvMaps maps, AttnArgs a,
                                                                int box_slots, Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  AttnSmem& sm = *reinterpret_cast<AttnSmem*>(smem_raw);
  const int head = blockIdx.x / kChunks, chunk = blockIdx.x % kChunks;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = a.ring_len / kChunks;  // a multiple of 16, at most kMaxPer
  const int slot0 = chunk * per;
  const int passes = (per + kSub - 1) / kSub;
  volatile uint32_t abort_flag = 0;  // this CTA's own waits only
  G4_STAMP(sc, 0);
  if (tid == 0) {
    mbar_init(&sm.kbar, 1);
    mbar_init(&sm.vbar, 1);
    fence_mbar_init();
  }
  // While the preceding QKV op finishes, bring this CTA's K and V rows into L2: it writes one
  // slot of them, but L2 is coherent, so the copies below (after the wait) still read its rows.
  for (int b = tid; b < 2 * (per / box_slots); b += kThreads) {
    const int nb = per / box_slots;
    tma_prefetch_l2_3d(b < nb ? &maps.k : &maps.v, 0, head, slot0 + (b < nb ? b : b - nb) * box_slots);
  }
  __syncthreads();

  pdl_wait_primary();  // q and the cache rows come from the preceding QKV op
  pdl_launch_dependents();
  G4_STAMP(sc, 1);

  // rows [first, first + count) of a cache into a shared-memory buffer, box_slots rows per TMA load
  const uint64_t policy = l2_evict_first_policy();  // each row is read once per step
  auto fetch = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* bar, int first, int count) {
    if (tid == 0) mbar_arrive_expect_tx(bar, uint32_t(count) * kRowBytes);
    for (int b = tid; b < count / box_slots; b += kThreads)
      tma_load_3d(dst + b * box_slots * kRowBytes, map, 0, head, slot0 + first + b * box_slots, bar, policy);
  };
  fetch(&maps.k, sm.k, &sm.kbar, 0, per < kSub ? per : kSub);
  if (passes == 1) fetch(&maps.v, sm.v, &sm.vbar, 0, per);

  // q rows of the two query heads: lane holds dims 8 lane .. 8 lane + 7
  float qv[kGs][8];
#pragma unroll
  for (int g = 0; g < kGs; ++g) {
    const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(a.q + (head * kGs + g) * kDs + lane * 8));
    const uint16_t* b = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) qv[g][j] = bf16_to_f32(b[j]);
  }

  // phase 1: scores of every slot of this CTA, kSub at a time; warp w scores slots w, w + 8, ...
  bool ok = true;
  for (int p = 0; p < passes; ++p) {
    const int first = p * kSub, rows = per - first < kSub ? per - first : kSub;
    if (p > 0) {
      __syncthreads();  // the previous pass is done with the K buffer
      fetch(&maps.k, sm.k, &sm.kbar, first, rows);
    }
    if (ok) ok = mbar_wait_or_abort(&sm.kbar, uint32_t(p & 1), &abort_flag, sc.err);
#pragma unroll 4
    for (int t = warp; t < rows; t += kWarps) {
      const uint4 kr = *reinterpret_cast<const uint4*>(sm.k + t * kRowBytes + lane * 16);
      const uint16_t* kb = reinterpret_cast<const uint16_t*>(&kr);
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
        sm.score[first + t][0] = bf16_round(a.scale * d0);
        sm.score[first + t][1] = bf16_round(a.scale * d1);
      }
    }
  }
  __syncthreads();
  G4_STAMP(sc, 2);

  // this CTA's maximum, published; then the head's maximum over all kChunks CTAs
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
  float* parts = sc.partials + kAttnPartials + size_t(head) * kChunks * kPartFloats;
  if (tid == 0) {
    float a0 = -INFINITY, a1 = -INFINITY;
    for (int w = 0; w < kWarps; ++w) {
      a0 = fmaxf(a0, sm.red[w][0]);
      a1 = fmaxf(a1, sm.red[w][1]);
    }
    parts[chunk * kPartFloats + 2 * kDs] = a0;
    parts[chunk * kPartFloats + 2 * kDs + 1] = a1;
    // generation barrier of the head's CTAs (the counter grows by kChunks per call)
    uint32_t* bar = sc.counters + kAttnBarrier + head;
    const uint32_t old = atomic_add_release_gpu(bar, 1u);
    const uint32_t target = old - old % kChunks + kChunks;
    const uint64_t t0 = globaltimer_ns();
    while (int32_t(ld_acquire_gpu(bar) - target) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(sc.err, kErrWaitTimeout);
        break;
      }
    }
  }
  __syncthreads();
  if (tid < kGs) {
    float m = -INFINITY;
    float pm[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) pm[c] = __ldcg(parts + c * kPartFloats + 2 * kDs + tid);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) m = fmaxf(m, pm[c]);
    sm.gmax[tid] = m;
  }
  __syncthreads();
  G4_STAMP(sc, 3);

  // probabilities and this CTA's denominator (fixed summation order)
  const float gm0 = sm.gmax[0], gm1 = sm.gmax[1];
  float s0 = 0.f, s1 = 0.f;
  for (int t = tid; t < per; t += kThreads) {
    const float mk = a.mask[slot0 + t];
    const float p0 = fminf(expf(sm.score[t][0] - gm0), mk);
    const float p1 = fminf(expf(sm.score[t][1] - gm1), mk);
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
      fetch(&maps.v, sm.v, &sm.vbar, first, rows);
    }
    if (ok) ok = mbar_wait_or_abort(&sm.vbar, uint32_t(p & 1), &abort_flag, sc.err);
    for (int t = 0; t < rows; ++t) {
      const float vf = bf16_to_f32(reinterpret_cast<const uint16_t*>(sm.v + t * kRowBytes)[tid]);
      o0 = fmaf(sm.score[first + t][0], vf, o0);
      o1 = fmaf(sm.score[first + t][1], vf, o1);
    }
  }
  parts[chunk * kPartFloats + tid] = o0;
  parts[chunk * kPartFloats + kDs + tid] = o1;
  if (tid < kGs) {
    float z = 0.f;
    for (int w = 0; w < kWarps; ++w) z += sm.red[w][tid];
    parts[chunk * kPartFloats + 2 * kDs + 2 + tid] = z;
  }
  __syncthreads();  // every partial of this CTA precedes the release below
  if (tid == 0) {
    uint32_t* ticket = sc.counters + kAttnTicket + head;
    const uint32_t before = atomic_add_acq_rel_gpu(ticket, 1u);
    sm.last = before == kChunks - 1 ? 1u : 0u;
    if (sm.last) *ticket = 0u;
  }
  __syncthreads();
  G4_STAMP(sc, 5);

  if (sm.last) {  // the head's last CTA: partials in chunk order
    float o[kGs] = {0.f, 0.f}, z[kGs] = {0.f, 0.f};
    float po[kChunks][kGs], pz[kChunks][kGs];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {  // every load in flight at once
      const float* pc = parts + c * kPartFloats;
      po[c][0] = __ldcg(pc + tid);
      po[c][1] = __ldcg(pc + kDs + tid);
      pz[c][0] = __ldcg(pc + 2 * kDs + 2);
      pz[c][1] = __ldcg(pc + 2 * kDs + 3);
    }
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      o[0] += po[c][0];
      o[1] += po[c][1];
      z[0] += pz[c][0];
      z[1] += pz[c][1];
    }
#pragma unroll
    for (int g = 0; g < kGs; ++g) sm.out[g * kDs + tid] = f32_to_bf16(bf16_round(o[g]) / (z[g] + kEps));
    __syncthreads();
    if (tid < kGs * kDs * 2 / 16)  // 16-byte stores
      reinterpret_cast<uint4*>(a.out + head * kGs * kDs)[tid] = reinterpret_cast<const uint4*>(sm.out)[tid];
  }
  G4_STAMP(sc, 6);
}

}  // namespace

cudaError_t prepare_attention_kernels() {
  return cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(AttnSmem)));
}

int attention_slot_multiple() { return kChunks * 16; }
int attention_max_ring() { return kMaxRing; }

cudaError_t launch_attention(const AttnArgs& a, const LaunchEnv& env) {
  // box: the largest of 128, 64, 32, 16 slots that divides a CTA's run (a multiple of 16)
  const int per = a.ring_len / kChunks;
  int box = kSub;
  while (per % box != 0) box /= 2;
  KvMaps maps;
  cudaError_t e;
  if (a.heads < 1 || a.heads > kNs) return cudaErrorInvalidValue;
  if ((e = env.maps->kv(a.k_cache, uint64_t(a.ring_len), uint32_t(a.heads), kDs, uint32_t(box), &maps.k))) return e;
  if ((e = env.maps->kv(a.v_cache, uint64_t(a.ring_len), uint32_t(a.heads), kDs, uint32_t(box), &maps.v))) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.heads * kChunks);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(AttnSmem);
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = env.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Scratch sc = env.sc;
#ifdef G4_TRACE
  if (sc.trace) sc.trace += 4096;  // profiling builds: separate stamp rows per kernel
#endif
  return cudaLaunchKernelEx(&cfg, attention_kernel, maps, a, box, sc);
}

}  // namespace g4
