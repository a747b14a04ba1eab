// Weight-streaming GEMV engine on the Blackwell tensor cores (sm_100a), used by every
// projection of the decode layer.
//
// Unit of work: 128 weight rows x 256 K elements (one UMMA tile row-block). The flat list of
// tiles x K-units is split into one contiguous run per CTA (one CTA per SM), so every SM
// streams the same number of bytes. Roles inside a CTA (192 threads):
//   warp 0    TMA producer: 2-D tensor-map loads of the weight tiles (and NVFP4 block scales)
//             into an S-stage shared-memory ring. The first S units are requested before the
//             kernel waits on the preceding kernel (weights never depend on it).
//   warp 1    MMA issuer: tcgen05.mma kind::f8f6f4 (A = weight codes, e4m3 or e2m1; B = the
//             activation as exact e4m3 terms) into a ring of TMEM accumulator slots; one
//             tcgen05.commit per unit both frees the stage and hands the slot to the epilogue.
//   warps 2-5 epilogue: one thread per tile row; reads its TMEM lane, combines the terms (and
//             the NVFP4 block scales) in f32 and finalises or publishes the row.
// The activation is scaled by a power of two before the split, chosen per 16-element group
// for nvfp4 weights (one block) and per 256-element unit for fp8 weights, so a few huge
// activations never push small ones below the terms' range; the epilogue multiplies the
// group's / unit's partial dot by the inverse factor.
// B operand (N = 8 rows, K-major, 128-byte swizzle), per 256-element K unit:
//   fp8 weights   rows 0..7 = terms t_0..t_7 of every element; one accumulator per unit.
//   nvfp4 weights block-diagonal: within each 32-element MMA step, rows 0..3 hold the terms
//                 t_0..t_3 of the first 16-element block and rows 4..7 those of the second,
//                 so every MMA writes the per-block partial dots to its own 8 TMEM columns and
//                 the epilogue applies the e4m3 block scale per (row, block) in f32.
// Rows whose K range is split across CTAs are published to global memory and summed by the
// last CTA to finish the tile, in CTA order: the result never depends on timing.
#pragma once

#include "g4_tc.cuh"

namespace g4 {

constexpr int kGemvThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kUnitK = 256;
constexpr int kTileRows = 128;
constexpr int kUmmaN = 8;
constexpr int kMmaPerUnit = kUnitK / 32;
constexpr int kEpiBarrier = 1;  // named barrier id of the epilogue warps
constexpr int kMmaLookahead = 4;  // units whose readiness the MMA thread tests in one go

template <bool FP4, int STAGES, int UPT, int TILES, int BSLOTS, int L2AHEAD = 6>
struct GemvShape {
  static constexpr bool kFp4 = FP4;
  static constexpr int kStages = STAGES;
  static constexpr int kL2Ahead = L2AHEAD;  // units requested into L2 beyond the shared-memory ring
  static constexpr int kUnitsPerTile = UPT;
  static constexpr int kTiles = TILES;
  static constexpr int kBSlots = BSLOTS;  // distinct K units one CTA may touch
  static constexpr int kTotalUnits = UPT * TILES;
  static constexpr int kABytes = 2 * kTileRows * 128;                 // two 128-element K halves
  static constexpr int kScaleBytes = FP4 ? kTileRows * (kUnitK / 16) : 0;
  static constexpr int kStageBytes = kABytes;
  static constexpr int kTmemSlots = FP4 ? 8 : 16;
  static constexpr uint32_t kTmemCols = FP4 ? 512u : 128u;
  static constexpr int kSlotCols = FP4 ? kMmaPerUnit * kUmmaN : kUmmaN;
  static_assert(STAGES <= kTmemSlots, "a stage is released through its unit's TMEM-slot barrier");
  static constexpr uint32_t kIdesc = umma_idesc_f8f6f4(FP4 ? kFmtE2M1 : kFmtE4M3, kFmtE4M3, kTileRows, kUmmaN);
  static constexpr int kTerms = FP4 ? kUmmaN / 2 : kUmmaN;  // e4m3 terms per activation element
  // shared memory: stages | B slots | block-scale ring (nvfp4, one per TMEM slot) |
  //                term scales (2^-E per 16-element group) | control block
  static constexpr size_t kOffB = size_t(STAGES) * kStageBytes;
  static constexpr size_t kOffScl = kOffB + size_t(BSLOTS) * 2048;
  static constexpr size_t kOffExp = kOffScl + (FP4 ? size_t(kTmemSlots) * kScaleBytes : 0);
  static constexpr size_t kOffCtl = kOffExp + size_t(BSLOTS) * 16 * sizeof(float);
  static constexpr size_t kSmemBytes = kOffCtl + 1024 + 1024;  // control block + alignment slack
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct GemvCtl {
  uint64_t full[8], sfull[16], done[16], tempty[16], drain;
  uint32_t tmem_base;
  uint32_t abort;
  uint32_t bcast;
  uint32_t bcast2;
  uint32_t unit_max[16];  // per B slot: max |activation| bits (fp8 weights)
  float xchg[64];
  double red_d[8];
  float red_f[8];
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// The CTA (of `grid`) whose run contains unit u (runs are [c*total/grid, (c+1)*total/grid)).
__device__ __forceinline__ int cta_of_unit(int64_t u, int64_t grid, int64_t total) {
  return int(((u + 1) * grid + total - 1) / total - 1);
}

// Everything a CTA of the engine shares between its roles.
template <class Shape>
struct GemvCta {
  uint8_t* stages;
  uint8_t* bsm;
  GemvCtl* ctl;
  int u0, n;  // this CTA's run of units
  int c0;     // K unit of the run's first unit (B slot 0)
  int tid, warp, lane;

  __device__ uint8_t* stage(int s) const { return stages + size_t(s) * Shape::kStageBytes; }
  __device__ int bslot(int kc) const { return (kc - c0 + Shape::kUnitsPerTile) % Shape::kUnitsPerTile; }
};

// Sum of squares of 16 bf16 values (two uint4), exact in f64.
__device__ __forceinline__ double sum_squares_bf16x16(const uint4& a, const uint4& b) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const double lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xffff0000u);
    ss += lo * lo + hi * hi;
  }
  return ss;
}

// Engine driver. `op` supplies:
//   void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const  (TMA)
//   void load_scales(uint8_t* dst, int tile, int kc, uint64_t* bar, uint64_t policy) const (nvfp4)
//   void prefetch_l2(int u0, int u1) const      units [u0, u1) into L2 (may do nothing)
//   static bool kRms, int kRmsGroups   whether the activation is RMS-normalised over its
//                                      kRmsGroups * 16 elements (every group is then loaded)
//   void prologue(GemvCtl&)            scalar loads, after the wait on the preceding kernel
//   void load_group(int g, uint4 (&raw)[4]) const   issue the loads of 16-element group g
//                                      (bf16 input in raw[0..1], gamma in raw[2..3])
//   void finish_group(const uint4 (&raw)[4], float inv, float (&v)[16]) const   the activation
//   void finalize_tile(int tile, int row, float v, GemvCtl&) const   all 128 epilogue threads
//   uint32_t tx_bytes                  bytes one unit's weight tiles deliver (block scales: kScaleBytes)
template <class Shape, class Op>
__device__ void gemv_run(Op& op, uint8_t* smem_raw, const Scratch& sc) {
  constexpr int S = Shape::kStages, UPT = Shape::kUnitsPerTile, T = Shape::kTmemSlots;
  uint8_t* smem = align1024(smem_raw);
  GemvCta<Shape> c;
  c.stages = smem;
  c.bsm = smem + Shape::kOffB;
  c.ctl = reinterpret_cast<GemvCtl*>(smem + Shape::kOffCtl);
  GemvCtl& ctl = *c.ctl;
  c.tid = threadIdx.x;
  c.warp = c.tid >> 5;
  c.lane = c.tid & 31;
  const int64_t total = Shape::kTotalUnits, grid = gridDim.x;
  c.u0 = int(int64_t(blockIdx.x) * total / grid);
  c.n = int(int64_t(blockIdx.x + 1) * total / grid) - c.u0;
  c.c0 = c.u0 % UPT;
  const int nslots = c.n < UPT ? c.n : UPT;
  volatile uint32_t* abort = &ctl.abort;
  G4_STAMP(sc, 0);

  if (c.tid == 0) {
    for (int i = 0; i < S; ++i) mbar_init(&ctl.full[i], 1);
    for (int i = 0; i < T; ++i) {
      mbar_init(&ctl.sfull[i], 1);  // nvfp4: the unit's block scales have landed in the ring
      mbar_init(&ctl.done[i], 1);   // the unit's MMAs have completed (one commit per unit)
      mbar_init(&ctl.tempty[i], 4); // the epilogue is done with the TMEM slot (and scale slot)
    }
    mbar_init(&ctl.drain, 1);
    ctl.abort = 0;
    fence_mbar_init();
  }
  if (c.tid < 16) ctl.unit_max[c.tid] = 0u;
  __syncwarp();
  if (c.warp == 1) tmem_alloc(&ctl.tmem_base, Shape::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ctl.tmem_base;

  // weights first: they do not depend on the preceding kernel
  const uint64_t policy = l2_evict_first_policy();
  const int prefetch = c.n < S ? c.n : S;
  if (c.tid == 0) {
    for (int i = 0; i < prefetch; ++i) {  // i < S <= T: every stage and scale slot is free
      const int u = c.u0 + i;
      mbar_arrive_expect_tx(&ctl.full[i], op.tx_bytes);
      op.load_unit(c.stage(i), u / UPT, u % UPT, &ctl.full[i], policy);
      if constexpr (Shape::kFp4) {
        mbar_arrive_expect_tx(&ctl.sfull[i], Shape::kScaleBytes);
        op.load_scales(smem + Shape::kOffScl + size_t(i) * Shape::kScaleBytes, u / UPT, u % UPT, &ctl.sfull[i], policy);
      }
    }
    // the next units go to L2 only: the ring's loads then hit L2 instead of waiting on HBM
    op.prefetch_l2(c.u0 + prefetch, c.u0 + (prefetch + Shape::kL2Ahead < c.n ? prefetch + Shape::kL2Ahead : c.n));
  }
  __syncwarp();  // CTA barriers below need converged warps
  pdl_wait_primary();
  pdl_launch_dependents();
  G4_STAMP(sc, 1);

  // activation -> B operand (only the K units this CTA touches). Every global load of the
  // prologue is issued before any is used: one round trip while the weight tiles stream in.
  float* gexp = reinterpret_cast<float*>(smem + Shape::kOffExp);  // [slot][group] 2^-E
  {
    constexpr int MAXG = 2;  // 16-element groups per thread
    static_assert(!Op::kRms || Op::kRmsGroups <= MAXG * kGemvThreads, "RMS statistic: too many groups");
    static_assert(Shape::kBSlots * 16 <= MAXG * kGemvThreads, "B slots: too many groups");
    op.prologue(ctl);  // scalar loads only
    int grp[MAXG];
    bool have[MAXG];
    uint4 raw[MAXG][4];
#pragma unroll
    for (int q = 0; q < MAXG; ++q) {
      const int j = c.tid + q * kGemvThreads;
      if constexpr (Op::kRms) {  // the RMS statistic needs the whole vector
        grp[q] = j;
        have[q] = j < Op::kRmsGroups;
      } else {  // only the groups of this CTA's K units
        grp[q] = ((c.c0 + j / 16) % UPT) * 16 + j % 16;
        have[q] = j < nslots * 16;
      }
      if (have[q]) op.load_group(grp[q], raw[q]);
    }
    float inv = 0.f;
    G4_STAMP(sc, 9);
    if constexpr (Op::kRms) {
      double ss = 0.0;
#pragma unroll
      for (int q = 0; q < MAXG; ++q)
        if (have[q]) ss += sum_squares_bf16x16(raw[q][0], raw[q][1]);
      inv = rms_inverse(block_sum_d(ss, ctl.red_d), Op::kRmsGroups * 16);
    }
    // exponent E of a max |v| so that max |v| 2^E lies in [128, 256)
    auto exponent_of = [](float amax) {
      int e = 0;
      if (amax > 0.f) {
        e = 7 - (int((__float_as_uint(amax) >> 23) & 0xff) - 127);
        e = e > 120 ? 120 : (e < -120 ? -120 : e);
      }
      return e;
    };
    float v[MAXG][16], amax[MAXG];
    int slot[MAXG];
#pragma unroll
    for (int q = 0; q < MAXG; ++q) {
      slot[q] = c.bslot(grp[q] / 16);
      have[q] = have[q] && slot[q] < nslots;
      amax[q] = 0.f;
      if (have[q]) {
        op.finish_group(raw[q], inv, v[q]);
#pragma unroll
        for (int j = 0; j < 16; ++j) amax[q] = fmaxf(amax[q], fabsf(v[q][j]));
        if constexpr (!Shape::kFp4)  // one exponent per 256-element unit
          atomicMax(&ctl.unit_max[slot[q]], __float_as_uint(amax[q]));  // non-negative floats order as ints
      }
    }
    if constexpr (!Shape::kFp4) {
      __syncthreads();
#pragma unroll
      for (int q = 0; q < MAXG; ++q)
        if (have[q]) amax[q] = __uint_as_float(ctl.unit_max[slot[q]]);
    }
    const uint4 zero = make_uint4(0, 0, 0, 0);
    G4_STAMP(sc, 10);
#pragma unroll
    for (int q = 0; q < MAXG; ++q) {
      if (!have[q]) continue;
      const int e16 = (grp[q] % 16) * 16;
      const int e = exponent_of(amax[q]);
      const float up = pow2f(e);
      gexp[slot[q] * 16 + grp[q] % 16] = pow2f(-e);
#pragma unroll
      for (int j = 0; j < 16; ++j) v[q][j] *= up;
      uint4 tm[Shape::kTerms];
      split_terms16<Shape::kTerms>(v[q], tm);
      uint8_t* atom = c.bsm + size_t(slot[q]) * 2048 + (e16 / 128) * 1024;
      const uint32_t kb = e16 % 128;
      uint4 rows[8];
      if constexpr (Shape::kFp4) {
        const bool second = (e16 / 16) % 2;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          rows[j] = second ? zero : tm[j];
          rows[4 + j] = second ? tm[j] : zero;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) rows[j] = tm[j];
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) *reinterpret_cast<uint4*>(atom + sw128_offset(r, kb)) = rows[r];
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  G4_STAMP(sc, 2);

  if (c.warp == 0) {
    // ---------------------------------------------------------------- producer
    if (c.lane == 0) {
      int issued = prefetch;
      for (int i = prefetch; i < c.n; ++i) {
        const int s = i % S;
        // stage s is free once the MMAs of unit i - S have completed
        if (!mbar_wait_or_abort(&ctl.done[(i - S) % T], uint32_t(((i - S) / T) & 1), abort, sc.err)) break;
        const int u = c.u0 + i;
        mbar_arrive_expect_tx(&ctl.full[s], op.tx_bytes);
        op.load_unit(c.stage(s), u / UPT, u % UPT, &ctl.full[s], policy);
        if ((i - prefetch) % 2 == 0 && i + Shape::kL2Ahead < c.n)  // two units per bulk L2 prefetch
          op.prefetch_l2(u + Shape::kL2Ahead, c.u0 + (i + Shape::kL2Ahead + 2 < c.n ? i + Shape::kL2Ahead + 2 : c.n));
        if constexpr (Shape::kFp4) {  // scale slot t is free once the epilogue is done with unit i - T
          const int t = i % T;
          if (i >= T && !mbar_wait_or_abort(&ctl.tempty[t], uint32_t(((i / T) - 1) & 1), abort, sc.err)) break;
          mbar_arrive_expect_tx(&ctl.sfull[t], Shape::kScaleBytes);
          op.load_scales(smem + Shape::kOffScl + size_t(t) * Shape::kScaleBytes, u / UPT, u % UPT, &ctl.sfull[t], policy);
        }
        issued = i + 1;
#ifdef G4_TRACE
        if (sc.trace && blockIdx.x == 0 && i < 64) sc.trace[3000 + i] = globaltimer_ns();
#endif
      }
      // every requested tile has landed before the CTA may exit
      for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&ctl.full[i % S], uint32_t((i / S) & 1)))
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
      if constexpr (Shape::kFp4) {
        for (int i = issued - T > 0 ? issued - T : 0; i < issued; ++i) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&ctl.sfull[i % T], uint32_t((i / T) & 1)))
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        }
      }
    }
    __syncwarp();  // lanes 1..31 wait here for lane 0: the teardown barrier needs whole warps
  } else if (c.warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // One commit per unit both frees the stage's weight tiles and hands the TMEM slot to the
    // epilogue. Any shared-memory access of this thread (an mbarrier test included) waits for
    // the MMAs it has queued, so readiness is checked for several units at a time: one blocking
    // wait for the next unit, then non-blocking tests of the following ones.
    if (c.lane == 0) {
      int ready = 0;  // units [i, ready) have landed and have a free TMEM slot
      bool alive = true;
      for (int i = 0; i < c.n && alive; ++i) {
        const int s = i % S, t = i % T;
        if (i >= ready) {
          alive = mbar_wait_or_abort(&ctl.full[s], uint32_t((i / S) & 1), abort, sc.err) &&
                  (i < T || mbar_wait_or_abort(&ctl.tempty[t], uint32_t(((i / T) - 1) & 1), abort, sc.err));
          if (!alive) break;
          ready = i + 1;
          while (ready < c.n && ready < i + kMmaLookahead &&
                 mbar_test(&ctl.full[ready % S], uint32_t((ready / S) & 1)) &&
                 (ready < T || mbar_test(&ctl.tempty[ready % T], uint32_t(((ready / T) - 1) & 1))))
            ++ready;
          tc_fence_after();
        }
        if (i == 0) G4_STAMP_T(sc, 3);
#ifdef G4_TRACE
        if (sc.trace && blockIdx.x == 0 && i < 64) sc.trace[3064 + i] = globaltimer_ns();
#endif
        const int kc = (c.u0 + i) % UPT;
        const uint32_t a_base = smem_u32(c.stage(s));
        const uint32_t b_base = smem_u32(c.bsm) + uint32_t(c.bslot(kc)) * 2048u;
#pragma unroll
        for (int j = 0; j < kMmaPerUnit; ++j) {
          const uint32_t h = j / 4, kk = j % 4;
          const uint64_t ad = umma_desc_sw128(a_base + h * 16384u + kk * 32u);
          const uint64_t bd = umma_desc_sw128(b_base + h * 1024u + kk * 32u);
          const uint32_t col = Shape::kFp4 ? uint32_t(t * Shape::kSlotCols + j * kUmmaN) : uint32_t(t * kUmmaN);
          umma_f8f6f4(tbase + col, ad, bd, Shape::kIdesc, Shape::kFp4 ? 0u : uint32_t(j > 0));
        }
        umma_commit(&ctl.done[t]);
        if (i == c.n - 1) G4_STAMP_T(sc, 4);
#ifdef G4_TRACE
        if (sc.trace && blockIdx.x == 0 && i < 64) sc.trace[3128 + i] = globaltimer_ns();
#endif
      }
      // nothing of ours may still be running when TMEM is released
      umma_commit(&ctl.drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ctl.drain, 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    __syncwarp();  // lanes 1..31 wait here for lane 0: the teardown barrier needs whole warps
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = c.warp & 3;
    const int row = quarter * 32 + c.lane;
    const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
    float acc = 0.f;
    int in_piece = 0;
    bool ok = true;  // after a failed wait the loop keeps its shape (named barriers) but skips work
    for (int i = 0; i < c.n; ++i) {
      const int u = c.u0 + i, tile = u / UPT, kc = u % UPT, t = i % T;
      if (ok) ok = mbar_wait_or_abort(&ctl.done[t], uint32_t((i / T) & 1), abort, sc.err);
      if (row == 0 && i == 0) G4_STAMP_T(sc, 5);
      tc_fence_after();
      if (!ok) {
      } else if constexpr (!Shape::kFp4) {
        float d[8];
        tmem_ld8(tbase + lane_addr + uint32_t(t * kUmmaN), d);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (c.lane == 0) mbar_arrive(&ctl.tempty[t]);
        acc = fmaf(combine_terms<8>(d), gexp[c.bslot(kc) * 16], acc);
      } else {
        float d0[32], d1[32];
        tmem_ld32(tbase + lane_addr + uint32_t(t * Shape::kSlotCols), d0);
        tmem_ld32(tbase + lane_addr + uint32_t(t * Shape::kSlotCols + 32), d1);
        ok = mbar_wait_or_abort(&ctl.sfull[t], uint32_t((i / T) & 1), abort, sc.err);
        const uint4 sraw =
            *reinterpret_cast<const uint4*>(smem + Shape::kOffScl + size_t(t) * Shape::kScaleBytes + row * 16);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (c.lane == 0) mbar_arrive(&ctl.tempty[t]);
        // block b of the unit: MMA b / 2, columns 4 (b % 2) .. 4 (b % 2) + 3 of its 8
        const uint32_t sw[4] = {sraw.x, sraw.y, sraw.z, sraw.w};
        const float* ge = gexp + c.bslot(kc) * 16;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          const float2 sp = e4m3x2_to_f32x2(sw[b / 4] >> (16 * ((b / 2) % 2)));
          acc = fmaf((b % 2) ? sp.y : sp.x, combine_terms<4>(d0 + (b / 2) * 8 + (b % 2) * 4) * ge[b], acc);
        }
#pragma unroll
        for (int b = 8; b < 16; ++b) {
          const float2 sp = e4m3x2_to_f32x2(sw[b / 4] >> (16 * ((b / 2) % 2)));
          acc = fmaf((b % 2) ? sp.y : sp.x, combine_terms<4>(d1 + (b / 2 - 4) * 8 + (b % 2) * 4) * ge[b], acc);
        }
      }
      ++in_piece;
#ifdef G4_TRACE
      if (sc.trace && blockIdx.x == 0 && i < 64 && row == 0) sc.trace[3192 + i] = globaltimer_ns();
#endif
      if (kc == UPT - 1 || i == c.n - 1) {
        const float v = acc;
        if (in_piece == UPT) {
          op.finalize_tile(tile, row, v, ctl);
        } else {
          // the tile's K range is split across CTAs: publish, the last to arrive adds them up
          const int first = cta_of_unit(int64_t(tile) * UPT, grid, total);
          const int last = cta_of_unit(int64_t(tile) * UPT + UPT - 1, grid, total);
          float* part = sc.partials + size_t(tile) * kMaxCtasPerGroup * kTileRows;
          if (last - first >= kMaxCtasPerGroup) {  // cannot happen for the shapes launched here
            if (row == 0) atomicOr(sc.err, kErrInternal);
          } else {
            part[(blockIdx.x - first) * kTileRows + row] = v;
            named_bar(kEpiBarrier, kEpiThreads);
            if (row == 0) {
              const uint32_t before = atomic_add_acq_rel_gpu(sc.counters + tile, uint32_t(in_piece));
              const bool done = before + uint32_t(in_piece) == uint32_t(UPT);
              if (done) sc.counters[tile] = 0;
              ctl.bcast = done ? 1u : 0u;
            }
            __syncwarp();
            named_bar(kEpiBarrier, kEpiThreads);
            if (ctl.bcast) {
              float tot = 0.f;
              for (int cc = first; cc <= last; ++cc) tot += ld_cg_f32(part + (cc - first) * kTileRows + row);
              op.finalize_tile(tile, row, tot, ctl);
            }
          }
        }
        acc = 0.f;
        in_piece = 0;
      }
    }
    if (row == 0) G4_STAMP_T(sc, 6);
  }

  // teardown: every MMA has completed (drain) and every TMEM load has been waited for
  G4_STAMP_WARP(sc, 0);
  tc_fence_before();
  __syncthreads();
  G4_STAMP(sc, 7);
  G4_STAMP_WARP(sc, 1);
  if (c.warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, Shape::kTmemCols);
    G4_STAMP_WARP(sc, 2);
  }
  G4_STAMP_WARP(sc, 3);
}

}  // namespace g4
