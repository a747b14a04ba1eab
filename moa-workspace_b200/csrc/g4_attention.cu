// Sliding-window decode attention over the bf16 ring cache (reference op:
// furiosa-opt-gemma4-12B/src/ops.rs:118-128, device semantics src/device/sliding/attention.rs:7-199).
//
//   s[g,t] = bf16(scale * q[g] . k[t])                      (f32 contraction, bf16 scores)
//   m[g]   = max over ALL t of s[g,t]                       (masked slots included)
//   p[g,t] = min(exp(s[g,t] - m[g]), mask[t])               (0/1 mask row)
//   sum[g] = sum_t p[g,t] + 1e-6
//   out    = bf16( bf16(sum_t bf16(p[g,t]) v[t]) / sum[g] )
//
// One thread-block cluster of C CTAs per KV head (C = 16 for rings of 2048 to 4096 slots where
// the GPU can hold the clusters, and for 1024-slot rings too when at most half the heads are on
// the GPU; else the portable 8: 128 or 64 CTAs for the 8 heads; a tensor-parallel rank holds 8 / n
// of them in its cache slice), each owning a contiguous run of ring slots. A CTA copies its K and V
// rows into shared memory with TMA boxes of 32 rows, each completing on its own barrier so that
// scoring starts as the first box lands (the V rows of the first pass are requested with the K
// rows: they are not needed until the maximum is known), scores its slots for the head's two
// query heads and computes its score maximum. The rounding
// of p to bf16 depends on the maximum over the WHOLE ring, so the cluster exchanges maxima
// through distributed shared memory before computing p: each CTA stores its maxima into every
// CTA's shared memory, and after a cluster barrier reads them from its own. Each CTA then stores
// its partial sum_t p, and its partial sum_t bf16(p) v of head dimensions [c Ds / C, (c + 1) Ds / C),
// into CTA c; after a second cluster barrier CTA c adds the partials in chunk order, so the result
// does not depend on timing. No CTA reads another's shared memory, so none waits for the others
// before it exits (the first barrier's arrival, at the start, only makes sure every CTA runs
// before any stores into it).
#include "g4_ops.cuh"
#include "g4_tc.cuh"

namespace g4 {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowBytes = kDs * 2;         // one head's row in one slot
constexpr int kBox = 32;                   // slots per TMA box, each with its own barrier
constexpr int kMaxRing = 8192;
constexpr int kMinChunks = 8;              // the portable cluster size; 16 where it can be scheduled

// Batches of sequences: the cluster size and the slots per pass (several CTAs per SM, so one CTA's
// loads overlap another's scoring; a whole batch fills the GPU without long single-head rings).
#ifndef G4_ATTN_BATCH_C
#define G4_ATTN_BATCH_C 4
#endif
#ifndef G4_ATTN_BATCH_SUB
#define G4_ATTN_BATCH_SUB 64
#endif

// C CTAs per KV head (the cluster size); SUB slots resident in shared memory per pass. One
// sequence: C = 8 with passes of 128, or C = 16 with passes of 64 for rings of 2048 to 4096 slots
// (small enough that several CTAs share an SM, so eight 16-CTA clusters fit the GPU together).
template <int C, int SUB, int MAXRING = kMaxRing>
struct AttnSmem {
  static constexpr int kMaxPer = MAXRING / C;
  static constexpr int kDimsPerCta = kDs / C;  // head dimensions each CTA combines
  static constexpr int kSub = SUB;
  static constexpr int kBoxes = SUB / kBox;
  static_assert(SUB % kBox == 0 && kBoxes <= kThreads, "boxes per pass");
  // two pass buffers: the K passes, then the V passes, alternate between them, so a pass's rows
  // land while the previous pass is used
  uint8_t buf[2][kSub * kRowBytes];
  // per slot, the two query heads' bf16 scores, then their bf16-rounded probabilities (head 1 in
  // the high half): the values the reference rounds to bf16 anyway
  uint32_t score[kMaxPer];
  float red[kWarps][kGs];
  float po[kGs][kDs];         // this CTA's partial sum_t bf16(p) v (the value pass's two halves)
  // written by the cluster's CTAs (CTA c at index c) before a cluster barrier: their score maxima,
  // their partials of the head dimensions this CTA combines, and their sum_t p
  float in_max[C][kGs];
  float in_po[C][kGs][kDimsPerCta];
  float in_z[C][kGs];
  __align__(16) uint16_t out[kGs * kDimsPerCta];
  uint64_t bar[2][kBoxes];
};
using Attn8 = AttnSmem<8, 128>;
using Attn16 = AttnSmem<16, 64>;
constexpr int kBatchMaxRing = 4096;  // a batch's rings (longer ones take the single-sequence shape)
// Below kBatchWide sequences a batch's grid is too small to fill the GPU three CTAs per SM (the
// clusters pack onto fewer SMs): those launches ask for kBatchNarrowSmem of shared memory, so two
// CTAs share an SM (measured: batch 8 on 1024-slot rings 22.6 us three per SM, 19.9 two per SM).
constexpr int kBatchWide = 16;
constexpr size_t kBatchNarrowSmem = 100 * 1024;
using AttnBatch = AttnSmem<G4_ATTN_BATCH_C, G4_ATTN_BATCH_SUB, kBatchMaxRing>;

__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return uint32_t(f32_to_bf16(lo)) | (uint32_t(f32_to_bf16(hi)) << 16);
}

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
// The cluster barrier in two halves: a relaxed arrival, and the wait for every CTA's.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// Store a float into CTA `rank`'s shared memory at the address this CTA's copy of the object has.
__device__ __forceinline__ void st_cluster_f32(void* own, uint32_t rank, float v) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(own)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
// A float of CTA `rank`'s shared memory at the address this CTA's copy of the object has.
__device__ __forceinline__ float ld_cluster_f32(const void* own, uint32_t rank) {
  uint32_t a;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(own)), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}

// MINB: CTAs per SM the registers must allow (a batch runs three per SM).
template <int C, int SUB, int MINB = 2, int MAXRING = kMaxRing>
__global__ void __launch_bounds__(kThreads, MINB) attention_kernel(const __grid_constant__ KvMaps maps, AttnArgs a,
                                                                   Scratch sc) {
  using Sm = AttnSmem<C, SUB, MAXRING>;
  constexpr int kChunks = C;
  constexpr int kDimsPerCta = Sm::kDimsPerCta;
  constexpr int kBoxes = Sm::kBoxes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Sm& sm = *reinterpret_cast<Sm*>(smem_raw);
  const int head = blockIdx.x / kChunks;
  const int chunk = int(cluster_ctarank());  // == blockIdx.x % kChunks
  const int seq = blockIdx.y;                // the sequence of a batch (its own ring)
  const size_t qrow0 = size_t(seq) * a.heads * kGs * kDs;
  const float* mask = a.mask + size_t(seq) * a.mask_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kSub = Sm::kSub;
  const int per = a.ring_len / kChunks;  // a multiple of 32, at most kMaxPer
  const int slot0 = chunk * per;                  // in this sequence's ring
  const int gslot0 = seq * a.ring_len + slot0;  // in the batched caches
  const int passes = (per + kSub - 1) / kSub;
  volatile uint32_t abort_flag = 0;  // this CTA's own waits only
  G4_STAMP(sc, 0);
  if (tid < kBoxes) {
    mbar_init(&sm.bar[0][tid], 1);
    mbar_init(&sm.bar[1][tid], 1);
    fence_mbar_init();
  }
  // this CTA is running: the others may write into its shared memory once they have waited for
  // this arrival (before the first exchange)
  cluster_arrive_relaxed();
  // rows [first, first + count) of a cache into a shared-memory buffer: box b (kBox rows) by
  // thread b, completing on its own barrier, so the rows can be used as their box lands
  const uint64_t policy = l2_evict_first_policy();  // each row is read once per step
  auto fetch = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* bars, int first, int count) {
    const int b = tid;
    if (b < count / kBox) {
      mbar_arrive_expect_tx(&bars[b], uint32_t(kBox) * kRowBytes);
      tma_load_3d(dst + b * kBox * kRowBytes, map, 0, head, gslot0 + first + b * kBox, &bars[b], policy);
    }
  };
  // The loads as a sequence of jobs: job j < P is K pass j, job P + p is V pass p (P passes of
  // kSub slots, the last possibly shorter), job j into buffer j % 2. Jobs 0 and 1 are requested up
  // front, job j + 2 once job j is used. A box's barrier completes once per job that arms it: the
  // K passes' last job (P - 1) arms only `last_rows` of them.
  const int last_rows = per - (passes - 1) * kSub;
  auto job_rows = [&](int j) { return (j % passes) == passes - 1 ? last_rows : kSub; };
  auto issue = [&](int j) {
    if (j < 2 * passes) fetch(j < passes ? &maps.k : &maps.v, sm.buf[j % 2], sm.bar[j % 2], (j % passes) * kSub,
                              job_rows(j));
  };
  auto parity = [&](int j, int b) {
    const int skipped = j > passes - 1 && (passes - 1) % 2 == j % 2 && last_rows <= b * kBox ? 1 : 0;
    return uint32_t((j / 2 - skipped) & 1);
  };
  // The slot the preceding QKV op writes, when the caller says which (-1: any row may change).
  int cur = -1;
  if (a.kv_offset) {
    const int kv = __ldg(a.kv_offset + seq);  // written before the QKV op ran, not by it
    if (kv >= 0 && kv % (kPs * 2) == 0 && kv / (kPs * 2) < a.ring_len) cur = kv / (kPs * 2);
  }
  if (a.kv_offset) {
    // every row but the slot's is final: jobs 0 and 1 go straight into shared memory while the
    // QKV op finishes (the slot's rows are read again after the wait)
    __syncthreads();  // the barriers are initialised
    issue(0);
    issue(1);
  }
  // While the preceding QKV op finishes, bring this CTA's other K and V rows into L2 (L2 is
  // coherent, so copies made after the wait still see the slot that op writes).
  {
    const int first_rows = per < kSub ? per : kSub;
    const int nb = per / kBox, skip = a.kv_offset ? first_rows / kBox : 0;
    for (int b = skip + tid; b < nb; b += kThreads) {
      tma_prefetch_l2_3d(&maps.k, 0, head, gslot0 + b * kBox);
      tma_prefetch_l2_3d(&maps.v, 0, head, gslot0 + b * kBox);
    }
  }
  // and the weights the following O and feed-forward kernels stream first (the decode driver's
  // hints): this op moves few bytes, so HBM has time for them while it runs
  issue_l2_hints(a.next, 2, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
  __syncthreads();

  pdl_wait_primary();  // q and the cache rows come from the preceding QKV op
  pdl_launch_dependents();
  G4_STAMP(sc, 1);

  // phase 1: scores, kSub slots at a time. The 8 lanes 8i .. 8i + 7 of a warp score one slot,
  // so a warp scores 4 slots per step (one box of 32 slots per step of the 8 warps). Lane
  // `part` of a slot holds head dimensions c 64 + 8 part + j (c < 4, j < 8): for each c the 8
  // lanes read 128 contiguous bytes of the row.
  constexpr int kLanesPerSlot = 8, kSlotsPerStep = 32 / kLanesPerSlot;
  static_assert(kWarps * kSlotsPerStep == kBox, "one box per step of the CTA");
  const int sub = lane / kLanesPerSlot, part = lane % kLanesPerSlot;
  // This lane's 32 q elements of each head (loaded first: the slot's fresh rows below wait on
  // their boxes and on loads of their own), as f32 where the registers allow (one or two CTAs per
  // SM), else as bf16 pairs (element 2i low) converted at each use (the batch shape's three).
  constexpr bool kQf32 = MINB <= 2;
  uint32_t qv[kGs][16];
  float qf[kGs][kQf32 ? 32 : 1];
#pragma unroll
  for (int g = 0; g < kGs; ++g) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 raw =
          __ldcg(reinterpret_cast<const uint4*>(a.q + qrow0 + (head * kGs + g) * kDs + c * 64 + part * 8));
      qv[g][4 * c] = raw.x, qv[g][4 * c + 1] = raw.y, qv[g][4 * c + 2] = raw.z, qv[g][4 * c + 3] = raw.w;
    }
  }

  if (!a.kv_offset) {
    issue(0);
    issue(1);
  } else if (cur >= slot0) {
    // the slot's fresh rows over the early copies of jobs 0 and 1, once the boxes holding them
    // landed (both waits first, then both rows: threads 32 j .. 32 j + 31 copy job j's 32 x 16 bytes)
    int tj[2];
    bool okb = true, fixed = false;
    for (int j = 0; j < 2; ++j) {
      tj[j] = cur - slot0 - (j % passes) * kSub;
      if (j >= 2 * passes || tj[j] < 0 || tj[j] >= job_rows(j)) {
        tj[j] = -1;
        continue;
      }
      okb = mbar_wait_or_abort(&sm.bar[j % 2][tj[j] / kBox], 0u, &abort_flag, sc.err) && okb;
      fixed = true;
    }
    const int j = tid / (kRowBytes / 16), q16 = tid % (kRowBytes / 16);
    const int t = j == 0 ? tj[0] : tj[1];
    if (okb && j < 2 && t >= 0) {
      const uint16_t* src =
          (j < passes ? a.k_cache : a.v_cache) + (size_t(seq * a.ring_len + cur) * a.heads + head) * kDs;
      reinterpret_cast<uint4*>(sm.buf[j % 2] + t * kRowBytes)[q16] = __ldcg(reinterpret_cast<const uint4*>(src) + q16);
    }
    if (fixed) __syncthreads();  // the rows are in place before anyone reads them (CTA-uniform)
  }

  if constexpr (kQf32) {
#pragma unroll
    for (int g = 0; g < kGs; ++g)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        qf[g][2 * i] = lo_bf16(qv[g][i]);
        qf[g][2 * i + 1] = hi_bf16(qv[g][i]);
      }
  }
  auto q_at = [&](int g, int e) {  // element e (< 32) of this lane's share of query head g
    if constexpr (kQf32) return qf[g][e];
    else return e % 2 ? hi_bf16(qv[g][e / 2]) : lo_bf16(qv[g][e / 2]);
  };
  bool ok = true;
  for (int p = 0; p < passes; ++p) {  // job p
    const int first = p * kSub, rows = job_rows(p);
    for (int b = 0; b < rows / kBox; ++b) {
      if (ok) ok = mbar_wait_or_abort(&sm.bar[p % 2][b], parity(p, b), &abort_flag, sc.err);
      const int t = b * kBox + warp * kSlotsPerStep + sub;
      const uint8_t* row = sm.buf[p % 2] + t * kRowBytes + part * 16;
      // one accumulator per head and 64-dimension chunk (chains of 8), added pairwise after
      float dc[kGs][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 kr = *reinterpret_cast<const uint4*>(row + c * 128);
        const uint32_t kw[4] = {kr.x, kr.y, kr.z, kr.w};
        dc[0][c] = dc[1][c] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // elements 2i and 2i + 1 of the chunk, in element order
          const float k0 = lo_bf16(kw[i]), k1 = hi_bf16(kw[i]);
          dc[0][c] = fmaf(q_at(0, 8 * c + 2 * i), k0, dc[0][c]);
          dc[1][c] = fmaf(q_at(1, 8 * c + 2 * i), k0, dc[1][c]);
          dc[0][c] = fmaf(q_at(0, 8 * c + 2 * i + 1), k1, dc[0][c]);
          dc[1][c] = fmaf(q_at(1, 8 * c + 2 * i + 1), k1, dc[1][c]);
        }
      }
      float d0 = (dc[0][0] + dc[0][1]) + (dc[0][2] + dc[0][3]);
      float d1 = (dc[1][0] + dc[1][1]) + (dc[1][2] + dc[1][3]);
#pragma unroll
      for (int o = kLanesPerSlot / 2; o; o >>= 1) {
        d0 += __shfl_xor_sync(0xffffffffu, d0, o);
        d1 += __shfl_xor_sync(0xffffffffu, d1, o);
      }
      if (part == 0) sm.score[first + t] = pack_bf16(a.scale * d0, a.scale * d1);
    }
    __syncthreads();  // every thread is done with buffer p % 2 (and, the last pass, every score is in)
    issue(p + 2);     // the job after next into it
  }
  G4_STAMP(sc, 2);

  // this CTA's maximum; then the head's maximum over the cluster (distributed shared memory)
  float m0 = -INFINITY, m1 = -INFINITY;
  for (int t = tid; t < per; t += kThreads) {
    const uint32_t w = sm.score[t];
    m0 = fmaxf(m0, lo_bf16(w));
    m1 = fmaxf(m1, hi_bf16(w));
  }
  m0 = warp_max(m0);
  m1 = warp_max(m1);
  if (lane == 0) {
    sm.red[warp][0] = m0;
    sm.red[warp][1] = m1;
  }
  __syncthreads();
  cluster_wait();  // every CTA of the cluster is running
  if (tid < kGs * kChunks) {  // thread (g, c): this CTA's maximum of head g into CTA c
    const int g = tid / kChunks, c = tid % kChunks;
    float m = -INFINITY;
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, sm.red[w][g]);
    st_cluster_f32(&sm.in_max[chunk][g], uint32_t(c), m);
  }
  cluster_sync();  // every CTA's maxima are in every CTA's shared memory
  float gm[kGs];
#pragma unroll
  for (int g = 0; g < kGs; ++g) {
    gm[g] = -INFINITY;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) gm[g] = fmaxf(gm[g], sm.in_max[c][g]);
  }
  G4_STAMP(sc, 3);

  // probabilities and this CTA's denominator (fixed summation order)
  float s0 = 0.f, s1 = 0.f;
  for (int t = tid; t < per; t += kThreads) {
    const float mk = mask[slot0 + t];
    const uint32_t w = sm.score[t];
    const float p0 = fminf(expf(lo_bf16(w) - gm[0]), mk);
    const float p1 = fminf(expf(hi_bf16(w) - gm[1]), mk);
    s0 += p0;
    s1 += p1;
    sm.score[t] = pack_bf16(p0, p1);
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

  // phase 2: o[g][d] = sum_t bf16(p[g][t]) v[t][d]. Thread tid owns the dimension pair
  // (2 dp, 2 dp + 1), dp = tid % 128, of both heads over one half of every box's slots (slots
  // [16 h, 16 h + 16) of the box, h = tid / 128), in two accumulator sets (even and odd slots);
  // the sets, then the halves, are added in a fixed order.
  constexpr int kHalf = kBox / 2;
  static_assert(kThreads == kDs, "thread pairs cover the head's 128 dimension pairs twice");
  const int dp = tid % (kThreads / 2), half = tid / (kThreads / 2);
  float acc[2][kGs][2];
#pragma unroll
  for (int e = 0; e < 2; ++e)
#pragma unroll
    for (int g = 0; g < kGs; ++g) acc[e][g][0] = acc[e][g][1] = 0.f;
  for (int p = 0; p < passes; ++p) {  // job passes + p
    const int j = passes + p, first = p * kSub, rows = job_rows(j);
    const uint8_t* vb = sm.buf[j % 2];
    for (int b = 0; b < rows / kBox; ++b) {
      if (ok) ok = mbar_wait_or_abort(&sm.bar[j % 2][b], parity(j, b), &abort_flag, sc.err);
      const int t0 = b * kBox + half * kHalf;
#pragma unroll
      for (int k = 0; k < kHalf; ++k) {
        const uint32_t vw = reinterpret_cast<const uint32_t*>(vb + (t0 + k) * kRowBytes)[dp];
        const uint32_t w = sm.score[first + t0 + k];
        const float v0 = lo_bf16(vw), v1 = hi_bf16(vw), p0 = lo_bf16(w), p1 = hi_bf16(w);
        acc[k % 2][0][0] = fmaf(p0, v0, acc[k % 2][0][0]);
        acc[k % 2][0][1] = fmaf(p0, v1, acc[k % 2][0][1]);
        acc[k % 2][1][0] = fmaf(p1, v0, acc[k % 2][1][0]);
        acc[k % 2][1][1] = fmaf(p1, v1, acc[k % 2][1][1]);
      }
    }
    if (j + 2 < 2 * passes) {  // CTA-uniform
      __syncthreads();  // every thread is done with buffer j % 2
      issue(j + 2);
    }
  }
  if (half == 1) {
#pragma unroll
    for (int g = 0; g < kGs; ++g) {
      sm.po[g][2 * dp] = acc[0][g][0] + acc[1][g][0];
      sm.po[g][2 * dp + 1] = acc[0][g][1] + acc[1][g][1];
    }
  }
  __syncthreads();  // the second half's sums are in place
  if (half == 0) {  // this CTA's partial of dimensions 2 dp, 2 dp + 1 into the CTA that combines them
#pragma unroll
    for (int g = 0; g < kGs; ++g) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int d = 2 * dp + e;
        const float v = (acc[0][g][e] + acc[1][g][e]) + sm.po[g][d];
        st_cluster_f32(&sm.in_po[chunk][g][d % kDimsPerCta], uint32_t(d / kDimsPerCta), v);
      }
    }
  }
  if (tid >= kThreads - kGs * kChunks) {  // thread (g, c): this CTA's sum_t p of head g into CTA c
    const int i = tid - (kThreads - kGs * kChunks), g = i / kChunks, c = i % kChunks;
    float z = 0.f;
    for (int w = 0; w < kWarps; ++w) z += sm.red[w][g];
    st_cluster_f32(&sm.in_z[chunk][g], uint32_t(c), z);
  }
  cluster_sync();  // every partial is in the shared memory of the CTA that combines it
  G4_STAMP(sc, 5);

  // CTA `chunk` combines dimensions [32 chunk, 32 chunk + 32) of both query heads, chunks in order
  if (tid < kGs * kDimsPerCta) {
    const int g = tid / kDimsPerCta, dd = tid % kDimsPerCta;
    float o = 0.f, z = 0.f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      o += sm.in_po[c][g][dd];
      z += sm.in_z[c][g];
    }
    sm.out[tid] = f32_to_bf16(bf16_round(o) / (z + kEps));
  }
  __syncthreads();  // sm.out is complete (no CTA reads another's shared memory after the barrier)
  if (tid < kGs * kDimsPerCta * 2 / 16) {  // 16-byte stores: 4 per query head
    const int g = tid / (kDimsPerCta * 2 / 16), q = tid % (kDimsPerCta * 2 / 16);
    reinterpret_cast<uint4*>(a.out + qrow0 + (head * kGs + g) * kDs + chunk * kDimsPerCta)[q] =
        reinterpret_cast<const uint4*>(sm.out + g * kDimsPerCta)[q];
  }
  G4_STAMP(sc, 6);
}

// ---------------------------------------------------------------------------------------
// Global layers: one 512-slot page of the attention of 16 query heads over the single K = V head
// of 512 dims (FOG/src/ops.rs:148-182; device semantics FOG/src/device/full/attention.rs:205-339):
//   s = bf16(q . k) (f32 contraction); m = max over the page's slots (masked ones included), on a
//   later page max(m, running max); e = min(exp(s - m), mask); page sum = sum e + 1e-6; per group
//   of 32 rows g: P_g = bf16(sum_{t in g} bf16(e_t) v_t); values = bf16(sum_g P_g) (groups in order).
//   First page: out = values, running max / sum = m / page sum. Later pages, r = exp(old max - m):
//   running sum = old sum r + page sum, out = bf16(bf16(old out r) + values).
// One cluster of C CTAs per page, CTA c owning rows [c Tf / C, (c + 1) Tf / C) (whole 32-row
// groups). Its warps score (warp w: heads 2w, 2w + 1; lane l: dims [16 l, 16 l + 16), the 32
// slots' partial dots reduced across the lanes by a shuffle reduce-scatter so lane t ends with
// slot t's sums), the cluster exchanges the heads' maxima and then the group values through
// distributed shared memory, and CTA c adds dims [c Df / C, (c + 1) Df / C) of every head over
// the groups in order.

constexpr int kFullThreads = 256;
constexpr int kGroup = 32;

template <int C>
struct FullAttnSmem {
  static constexpr int kRows = kTf / C;
  static constexpr int kGroups = kRows / kGroup;
  __align__(16) uint16_t q[kGf][kDf];
  __align__(16) uint16_t k[kRows][kDf];
  __align__(16) uint16_t v[kRows][kDf];
  float s[kGf][kRows];               // scores, then bf16(e)
  float part[kGroups][kGf][kDf];     // this CTA's group values P_g (read by the cluster)
  float cmax[kGf], csum[kGf];        // this CTA's maxima and sums of e (read by the cluster)
  float gmax[kGf], old_max[kGf], old_sum[kGf];
};

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Lane L holds v[j] = its partial of slot j (j < 32); afterwards v[0] is slot L's sum over the
// warp's 32 lanes (a fixed butterfly order: the same in every call).
__device__ __forceinline__ float reduce_scatter32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = 16; h >= 1; h >>= 1) {
    const bool upper = (lane & h) != 0;
#pragma unroll
    for (int j = 0; j < h; ++j) {
      const float send = upper ? v[j] : v[j + h];
      const float keep = upper ? v[j + h] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, h);
    }
  }
  return v[0];
}

template <int C>
__global__ void __launch_bounds__(kFullThreads, 1) full_attention_kernel(FullAttnArgs a, Scratch sc) {
  using Sm = FullAttnSmem<C>;
  constexpr int kRows = Sm::kRows, kGroups = Sm::kGroups, kDims = kDf / C;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Sm& sm = *reinterpret_cast<Sm*>(smem_raw);
  const int c = int(cluster_ctarank());
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = c * kRows;
  const uint8_t* krow = reinterpret_cast<const uint8_t*>(a.k + size_t(r0) * kDf);
  const uint8_t* vrow = reinterpret_cast<const uint8_t*>(a.v + size_t(r0) * kDf);
  constexpr int kLines = kRows * kDf * 2 / 128;  // 128-byte lines of this CTA's K (and V) rows
  // while the preceding QKV op finishes: this CTA's rows into L2 (it writes one slot of the page;
  // L2 is coherent, so the copies after the wait still read it)
  for (int i = tid; i < 2 * kLines; i += kFullThreads)
    asm volatile("prefetch.global.L2 [%0];" ::"l"((i < kLines ? krow : vrow) + size_t(i % kLines) * 128) : "memory");
  pdl_wait_primary();
  pdl_launch_dependents();
  int pos = 0;
  if (a.position) {  // the decode driver: a page past the position does not exist yet
    pos = __ldcg(a.position);
    if (a.page * kTf > pos) return;  // (every CTA of the cluster sees the same position)
  }
  // q and K rows, then V rows, into shared memory (16-byte copies; V is waited for later)
  for (int i = tid; i < kGf * kDf / 8; i += kFullThreads) cp_async_16(&sm.q[0][0] + i * 8, a.q + i * 8);
  for (int i = tid; i < kRows * kDf / 8; i += kFullThreads) cp_async_16(&sm.k[0][0] + i * 8, a.k + size_t(r0) * kDf + i * 8);
  cp_async_commit();
  for (int i = tid; i < kRows * kDf / 8; i += kFullThreads) cp_async_16(&sm.v[0][0] + i * 8, a.v + size_t(r0) * kDf + i * 8);
  cp_async_commit();
  if (!a.first && tid < kGf) {
    sm.old_max[tid] = __ldcg(a.running_max + tid);
    sm.old_sum[tid] = __ldcg(a.running_sum + tid);
  }
  cp_async_wait_group<1>();
  __syncthreads();

  // scores: warp w takes heads 2w and 2w + 1; lane l dims [16 l, 16 l + 16)
  const int h0 = 2 * warp;
  float qa[16], qb[16];
  {
    const uint4* pa = reinterpret_cast<const uint4*>(&sm.q[h0][16 * lane]);
    const uint4* pb = reinterpret_cast<const uint4*>(&sm.q[h0 + 1][16 * lane]);
    const uint4 a0 = pa[0], a1 = pa[1], b0 = pb[0], b1 = pb[1];
    const uint32_t wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t wb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      qa[2 * i] = __uint_as_float(wa[i] << 16);
      qa[2 * i + 1] = __uint_as_float(wa[i] & 0xffff0000u);
      qb[2 * i] = __uint_as_float(wb[i] << 16);
      qb[2 * i + 1] = __uint_as_float(wb[i] & 0xffff0000u);
    }
  }
  float mya = -INFINITY, myb = -INFINITY;
#pragma unroll 1
  for (int blk = 0; blk < kRows / 32; ++blk) {
    float pa[32], pb[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      const uint4* pk = reinterpret_cast<const uint4*>(&sm.k[blk * 32 + t][16 * lane]);
      const uint4 k0 = pk[0], k1 = pk[1];
      const uint32_t wk[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float lo = __uint_as_float(wk[i] << 16), hi = __uint_as_float(wk[i] & 0xffff0000u);
        sa = fmaf(qa[2 * i], lo, sa);
        sa = fmaf(qa[2 * i + 1], hi, sa);
        sb = fmaf(qb[2 * i], lo, sb);
        sb = fmaf(qb[2 * i + 1], hi, sb);
      }
      pa[t] = sa;
      pb[t] = sb;
    }
    const float sa = bf16_round(reduce_scatter32(pa)), sb = bf16_round(reduce_scatter32(pb));
    sm.s[h0][blk * 32 + lane] = sa;
    sm.s[h0 + 1][blk * 32 + lane] = sb;
    mya = fmaxf(mya, sa);
    myb = fmaxf(myb, sb);
  }
  mya = warp_max(mya);
  myb = warp_max(myb);
  if (lane == 0) {
    sm.cmax[h0] = mya;
    sm.cmax[h0 + 1] = myb;
  }
  cluster_sync();  // every CTA's maxima are in its shared memory
  if (tid < kGf) {
    float pm[C];
#pragma unroll
    for (int j = 0; j < C; ++j) pm[j] = ld_cluster_f32(&sm.cmax[tid], uint32_t(j));
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < C; ++j) m = fmaxf(m, pm[j]);
    if (!a.first) m = fmaxf(m, sm.old_max[tid]);
    sm.gmax[tid] = m;
  }
  __syncthreads();
  // e = min(exp(s - m), mask), kept as bf16(e); the CTA's sum of e per head
  {
    float za = 0.f, zb = 0.f;
    for (int t = lane; t < kRows; t += 32) {
      const float mk = a.mask ? a.mask[r0 + t] : (a.page * kTf + r0 + t <= pos ? 1.0f : 0.0f);
      const float ea = fminf(expf(sm.s[h0][t] - sm.gmax[h0]), mk);
      const float eb = fminf(expf(sm.s[h0 + 1][t] - sm.gmax[h0 + 1]), mk);
      za += ea;
      zb += eb;
      sm.s[h0][t] = bf16_round(ea);
      sm.s[h0 + 1][t] = bf16_round(eb);
    }
    za = warp_sum(za);
    zb = warp_sum(zb);
    if (lane == 0) {
      sm.csum[h0] = za;
      sm.csum[h0 + 1] = zb;
    }
  }
  cp_async_wait_group<0>();
  __syncthreads();  // bf16(e) of every head and the V rows are in shared memory
  // group values: thread tid owns dims 2 tid, 2 tid + 1 of every head
#pragma unroll 1
  for (int g = 0; g < kGroups; ++g) {
    float acc[kGf][2];
#pragma unroll
    for (int h = 0; h < kGf; ++h) acc[h][0] = acc[h][1] = 0.f;
#pragma unroll 4
    for (int t = g * kGroup; t < (g + 1) * kGroup; ++t) {
      const uint32_t w2 = reinterpret_cast<const uint32_t*>(sm.v[t])[tid];
      const float v0 = __uint_as_float(w2 << 16), v1 = __uint_as_float(w2 & 0xffff0000u);
#pragma unroll
      for (int h = 0; h < kGf; ++h) {
        acc[h][0] = fmaf(sm.s[h][t], v0, acc[h][0]);
        acc[h][1] = fmaf(sm.s[h][t], v1, acc[h][1]);
      }
    }
#pragma unroll
    for (int h = 0; h < kGf; ++h) {
      sm.part[g][h][2 * tid] = bf16_round(acc[h][0]);
      sm.part[g][h][2 * tid + 1] = bf16_round(acc[h][1]);
    }
  }
  cluster_sync();  // every CTA's group values and sums are in its shared memory
  // CTA c combines dims [c kDims, (c + 1) kDims) of every head over the page's groups, in order
  for (int o = tid; o < kGf * kDims; o += kFullThreads) {
    const int h = o / kDims, d = c * kDims + o % kDims;
    float total = 0.f, z = 0.f;
#pragma unroll 1
    for (int j = 0; j < C; ++j) {
#pragma unroll
      for (int g = 0; g < kGroups; ++g) total += ld_cluster_f32(&sm.part[g][h][d], uint32_t(j));
      z += ld_cluster_f32(&sm.csum[h], uint32_t(j));
    }
    const float values = bf16_round(total), page_sum = z + kEps, m = sm.gmax[h];
    float outv, sum;
    if (a.first) {
      outv = values;
      sum = page_sum;
    } else {
      const float r = expf(sm.old_max[h] - m);
      outv = bf16_round(bf16_round(bf16_to_f32(__ldcg(a.out + h * kDf + d)) * r) + values);
      sum = sm.old_sum[h] * r + page_sum;
    }
    a.out[h * kDf + d] = f32_to_bf16(outv);
    if (c == 0 && d == 0) {  // one thread per head: the running statistics
      a.running_max[h] = m;
      a.running_sum[h] = sum;
    }
  }
  cluster_sync();  // the others are done reading this CTA's shared memory
}

template <int C>
cudaLaunchConfig_t full_attention_config(cudaStream_t stream, bool pdl, cudaLaunchAttribute (&attr)[2]) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C);
  cfg.blockDim = dim3(kFullThreads);
  cfg.dynamicSmemBytes = sizeof(FullAttnSmem<C>);
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cfg;
}

template <class Sm, int C>
cudaLaunchConfig_t attention_config(int heads, cudaStream_t stream, bool pdl, cudaLaunchAttribute (&attr)[2],
                                    int batch = 1, size_t smem = sizeof(Sm)) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(heads * C, batch);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // one cluster per KV head
  attr[1].val.clusterDim.x = C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cfg;
}

// Per device: whether 16-CTA clusters of the kernel fit the GPU a whole layer at a time (all 8
// heads' clusters resident together); otherwise every call uses the portable 8.
constexpr int kMaxDevices = 64;
int g_clusters16[kMaxDevices];  // 0 unknown, 1 yes, -1 no

}  // namespace

cudaError_t prepare_attention_kernels() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(attention_kernel<8, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(sizeof(Attn8)))))
    return e;
  if ((e = cudaFuncSetAttribute(attention_kernel<16, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(sizeof(Attn16)))))
    return e;
  if ((e = cudaFuncSetAttribute(attention_kernel<G4_ATTN_BATCH_C, G4_ATTN_BATCH_SUB, 3, kBatchMaxRing>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(sizeof(AttnBatch) > kBatchNarrowSmem ? sizeof(AttnBatch) : kBatchNarrowSmem))))
    return e;
  if (G4_ATTN_BATCH_C > 8 &&
      (e = cudaFuncSetAttribute(attention_kernel<G4_ATTN_BATCH_C, G4_ATTN_BATCH_SUB, 3, kBatchMaxRing>,
                                cudaFuncAttributeNonPortableClusterSizeAllowed, 1)))
    return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev))) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaSuccess;  // such a device keeps the portable size
  int fits = 0;
  if (cudaFuncSetAttribute(attention_kernel<16, 64>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
      cudaSuccess) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = attention_config<Attn16, 16>(kNs, nullptr, false, attr);
    if (cudaOccupancyMaxActiveClusters(&fits, attention_kernel<16, 64>, &cfg) != cudaSuccess) fits = 0;
  }
  cudaGetLastError();  // a refused query is not an error of this call
  g_clusters16[dev] = fits >= kNs ? 1 : -1;
  if ((e = cudaFuncSetAttribute(full_attention_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(sizeof(FullAttnSmem<8>)))))
    return e;
  if ((e = cudaFuncSetAttribute(full_attention_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(sizeof(FullAttnSmem<16>)))))
    return e;
  if (g_clusters16[dev] == 1 &&
      cudaFuncSetAttribute(full_attention_kernel<16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    cudaGetLastError();
    g_clusters16[dev] = -1;
  }
  return cudaSuccess;
}

cudaError_t launch_full_attention(const FullAttnArgs& a, const LaunchEnv& env) {
  if (env.tp.world != 1) return cudaErrorNotSupported;  // the global layers run on one GPU
  cudaLaunchAttribute attr[2];
  if (env.device >= 0 && env.device < kMaxDevices && g_clusters16[env.device] == 1) {
    const cudaLaunchConfig_t cfg = full_attention_config<16>(env.stream, env.pdl, attr);
    return cudaLaunchKernelEx(&cfg, full_attention_kernel<16>, a, env.sc);
  }
  const cudaLaunchConfig_t cfg = full_attention_config<8>(env.stream, env.pdl, attr);
  return cudaLaunchKernelEx(&cfg, full_attention_kernel<8>, a, env.sc);
}

int attention_slot_multiple() { return kMinChunks * 32; }
int attention_max_ring() { return kMaxRing; }

cudaError_t launch_attention(const AttnArgs& a, const LaunchEnv& env) {
  KvMaps maps;
  cudaError_t e;
  if (a.heads < 1 || a.heads > kNs || a.batch < 1 || a.batch > 65535) return cudaErrorInvalidValue;
  if (a.batch > 1 && a.mask_stride < a.ring_len) return cudaErrorInvalidValue;
  const uint64_t slots = uint64_t(a.ring_len) * uint64_t(a.batch);  // every sequence's ring, back to back
  if ((e = env.maps->kv(a.k_cache, slots, uint32_t(a.heads), kDs, uint32_t(kBox), &maps.k))) return e;
  if ((e = env.maps->kv(a.v_cache, slots, uint32_t(a.heads), kDs, uint32_t(kBox), &maps.v))) return e;
  Scratch sc = env.sc;
#ifdef G4_TRACE
  if (sc.trace) sc.trace += 4096;  // profiling builds: separate stamp rows per kernel
#endif
  cudaLaunchAttribute attr[2];
  if (a.batch > 1 && a.ring_len % (G4_ATTN_BATCH_C * kBox) == 0 && a.ring_len <= kBatchMaxRing) {
    const size_t smem = a.batch >= kBatchWide || sizeof(AttnBatch) > kBatchNarrowSmem ? sizeof(AttnBatch)
                                                                                       : kBatchNarrowSmem;
    const cudaLaunchConfig_t cfg =
        attention_config<AttnBatch, G4_ATTN_BATCH_C>(a.heads, env.stream, env.pdl, attr, a.batch, smem);
    return cudaLaunchKernelEx(&cfg, attention_kernel<G4_ATTN_BATCH_C, G4_ATTN_BATCH_SUB, 3, kBatchMaxRing>, maps, a,
                              sc);
  }
  // 16-CTA clusters for rings of 2 to 4 passes; for 1024-slot rings too when at most half the
  // heads are on this GPU (tensor parallelism), as the eight heads' 128 CTAs would leave the next
  // kernel too few SMs to start its weight copies on (measured slower at 8 heads)
  const bool few_heads = a.heads * a.batch <= kNs / 2;
  const bool c16 = env.device >= 0 && env.device < kMaxDevices && g_clusters16[env.device] == 1 &&
                   a.ring_len % (16 * kBox) == 0 && a.ring_len >= (few_heads ? 1024 : 2048) &&
                   a.ring_len <= 4 * 16 * Attn16::kSub;
  if (c16) {
    const cudaLaunchConfig_t cfg = attention_config<Attn16, 16>(a.heads, env.stream, env.pdl, attr, a.batch);
    return cudaLaunchKernelEx(&cfg, attention_kernel<16, 64>, maps, a, sc);
  }
  const cudaLaunchConfig_t cfg = attention_config<Attn8, 8>(a.heads, env.stream, env.pdl, attr, a.batch);
  return cudaLaunchKernelEx(&cfg, attention_kernel<8, 128>, maps, a, sc);
}

}  // namespace g4
