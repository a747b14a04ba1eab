// Weight-streaming GEMV engine on the Blackwell tensor cores (sm_100a), used by every
// projection of the decode layer.
//
// Unit of work: 128 weight rows x 256 K elements (one UMMA tile row-block). The flat list of
// tiles x K-units is split into one contiguous run per CTA (one CTA per SM), so every SM
// streams the same number of bytes. Roles inside a CTA (224 threads):
//   warp 0    TMA producer: tensor-map loads of the weight tiles (and the nvfp4 block scales)
//             into an S-stage shared-memory ring. The ring is filled before the kernel
//             waits on the preceding kernel (weights never depend on it).
//   warp 1    MMA issuer (one thread). It never touches shared memory inside its loop: any
//             shared-memory access of the issuing thread waits for the MMAs it has queued.
//             Warp 6 (relay) waits on the unit's mbarriers and releases the issuer through a
//             named barrier that also carries an abort flag. One tcgen05.commit per unit
//             frees the stage.
//   warps 2-5 epilogue: one thread per tile row; reads its TMEM lane and finalises or
//             publishes the row. For nvfp4 weights they also move each unit's block scales
//             from shared memory into TMEM (tcgen05.st) ahead of the MMAs.
//
// fp8 weights: tcgen05.mma kind::f8f6f4 (A = e4m3 codes, K = 32 per instruction; B = the
//   activation as exact e4m3 terms, N = 8 rows: t_0..t_7). The activation is scaled by a power
//   of two per 256-element unit before the split, so each unit has its own TMEM accumulator;
//   the epilogue multiplies the unit's dot by the inverse factor and sums the units.
// nvfp4 weights: tcgen05.mma kind::mxf4nvf4 with 16-element ue4m3 block scales (A = packed e2m1
//   codes, K = 64 per instruction, its e4m3 block scales in TMEM; B = the activation as exact
//   e2m1 base-8 digits, N = 16 rows: two exponent classes x 8 digits, B block scale 1). All
//   units of a tile accumulate into one TMEM slot; the epilogue recombines the digits once per
//   tile. Block scales live in TMEM in the scale-factor layout of the MMA: the scales of MMA j
//   (blocks 4j..4j+3 of a row, 4 bytes) of row m sit in column 4j + m / 32, lane m % 32 of every
//   lane quarter; each MMA's 4 columns start on a multiple of 4.
// Rows whose K range is split across CTAs are published to global memory as epoch-tagged words
// and summed by the CTA holding the tile's first unit, in CTA order: the result never depends on
// timing.
#pragma once

#include "g4_tc.cuh"

namespace g4 {

constexpr int kGemvThreads = 224;
constexpr int kEpiThreads = 128;
constexpr int kRelayWarp = 6;
constexpr int kUnitK = 256;
constexpr int kTileRows = 128;
constexpr int kEpiBarrier = 1;    // named barrier of the epilogue warps
constexpr int kIssueBarrier = 2;  // named barrier of the MMA warp and the relay warp
constexpr int kIssueThreads = 64;
#ifndef G4_PREWAIT_UNITS
#define G4_PREWAIT_UNITS 12  // at most the ring
#endif

template <bool FP4, int STAGES, int UPT, int TILES, int BSLOTS, int L2AHEAD = 6>
struct GemvShape {
  static constexpr bool kFp4 = FP4;
  static constexpr int kStages = STAGES;
  static constexpr int kPreWait = G4_PREWAIT_UNITS < STAGES ? G4_PREWAIT_UNITS : STAGES;  // before the dependency wait
  static constexpr int kL2Ahead = L2AHEAD;  // units requested into L2 beyond the shared-memory ring
  static constexpr int kUnitsPerTile = UPT;
  static constexpr int kTiles = TILES;
  static constexpr int kBSlots = BSLOTS;  // distinct K units one CTA may touch
  static constexpr int kTotalUnits = UPT * TILES;
  static constexpr int kN = FP4 ? 16 : 8;  // B rows: digits / terms
  static constexpr int kABytes = FP4 ? kTileRows * 128 : 2 * kTileRows * 128;
  static constexpr int kScaleBytes = FP4 ? kTileRows * 16 : 0;  // [128 rows][16 blocks] e4m3
  static constexpr int kStageBytes = kABytes + kScaleBytes;
  static constexpr int kBSlotBytes = 2048;  // fp8: 8 rows x 256 B; nvfp4: 16 rows x 128 B
  // TMEM: fp8 - 16 accumulator slots of 8 columns (one per unit in flight).
  //       nvfp4 - 4 tile accumulators of 16 columns | B scales (4 columns) | A scales, 16
  //               columns per stage.
  static constexpr int kTmemSlots = FP4 ? STAGES : 16;
  static constexpr int kDSlots = 4;
  static constexpr uint32_t kColSfb = 64;
  static constexpr uint32_t kColSfa = 68;
  static constexpr uint32_t kTmemCols = FP4 ? 256u : 128u;
  static_assert(!FP4 || kColSfa + 16 * STAGES <= kTmemCols, "TMEM budget");
  static_assert(FP4 || STAGES <= kTmemSlots, "a stage is released through its unit's TMEM-slot barrier");
  static_assert(STAGES <= 12, "barrier arrays");
  static constexpr uint32_t kIdesc =
      FP4 ? umma_idesc_nvf4(kTileRows, kN) : umma_idesc_f8f6f4(kFmtE4M3, kFmtE4M3, kTileRows, kN);
  // shared memory: stages | B slots | nvfp4 activation (bf16, 256 per B slot) |
  //                fp8 unit scales 2^-E | control block
  static constexpr size_t kOffB = size_t(STAGES) * kStageBytes;
  static constexpr size_t kOffH = kOffB + size_t(BSLOTS) * kBSlotBytes;
  static constexpr size_t kOffExp = kOffH + (FP4 ? size_t(BSLOTS) * 512 : 0);
  static constexpr size_t kOffCtl = kOffExp + (FP4 ? 0 : size_t(BSLOTS) * 16 * sizeof(float));
  static constexpr size_t kCtlBytes = 2048;
  static constexpr size_t kSmemBytes = kOffCtl + kCtlBytes + 1024;  // control block + alignment slack
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct GemvCtl {
  uint64_t full[12], sready[12], done[16], tempty[16], dfull[4], dempty[4], drain;
  uint64_t bready[16];    // the B slot is built in shared memory (fp8: its terms and exponent)
  uint32_t tmem_base;
  uint32_t abort;
  int pmax;               // nvfp4: largest exponent of this CTA's activation
  uint32_t nonfinite;     // nvfp4: an activation of this CTA is Inf or NaN
  float xchg[64];
  __align__(16) uint16_t out16[kTileRows];  // a tile's bf16 results, stored to global 16 bytes at a time
  double red_d[8];
};
static_assert(sizeof(GemvCtl) <= 2048, "the control block's share of the engine's shared memory (kCtlBytes)");

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// The CTA (of `grid`) whose run contains unit u (runs are [c*total/grid, (c+1)*total/grid)).
__host__ __device__ __forceinline__ int cta_of_unit(int64_t u, int64_t grid, int64_t total) {
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

// Bring units [u0, u1) of a unit-tiled matrix (unit_bytes each) into L2 with one bulk prefetch.
__device__ __forceinline__ void prefetch_units(const uint8_t* base, int u0, int u1, uint32_t unit_bytes) {
  if (u1 > u0)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + size_t(u0) * unit_bytes),
                 "r"(uint32_t(u1 - u0) * unit_bytes)
                 : "memory");
}

// Loads of one 16-element group: bf16 input written by the preceding kernel (L2-coherent) and,
// for the normalised ops, its gamma.
__device__ __forceinline__ void load_group_cg(const uint16_t* x, int g, uint4 (&raw)[4]) {
  raw[0] = __ldcg(reinterpret_cast<const uint4*>(x + 16 * g));
  raw[1] = __ldcg(reinterpret_cast<const uint4*>(x + 16 * g + 8));
}
__device__ __forceinline__ void load_group_gamma(const uint16_t* gamma, int g, uint4 (&raw)[4]) {
  raw[2] = *reinterpret_cast<const uint4*>(gamma + 16 * g);
  raw[3] = *reinterpret_cast<const uint4*>(gamma + 16 * g + 8);
}

// The 16 bf16 values of two uint4 (element j in half j % 2 of word j / 2).
__device__ __forceinline__ void bf16x16_to_f32(const uint4& a, const uint4& b, float (&v)[16]) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// h = bf16((x * inv) * gamma) for one group (the RMSNorm of gemma4.py:83-89).
__device__ __forceinline__ void rms_apply16(const uint4 (&raw)[4], float inv, float (&v)[16]) {
  float g[16];
  bf16x16_to_f32(raw[0], raw[1], v);
  bf16x16_to_f32(raw[2], raw[3], g);
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = bf16_round((v[j] * inv) * g[j]);
}

// nvfp4 B operand: the digits of 8 consecutive activation elements (bf16 bits in `raw`) as
// 4-byte pieces of the 16 B rows. An element of exponent e >= pc - 14 is class 0 (rows 0-7,
// X = RN(v 2^(21 - pc)), exact); a smaller one is class 1 (rows 8-15, X = RN(v 2^(36 - pc)),
// exact for e >= pc - 29, else off by less than 2^(pc - 37)). |X| < 2^22 in both classes.
__device__ __forceinline__ void nvf4_digit_rows8(const uint4& raw, int pc, uint32_t (&rows)[16]) {
  const uint32_t h[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t w[8];
  uint32_t m0 = 0u;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float v = __uint_as_float(k % 2 ? (h[k / 2] & 0xffff0000u) : (h[k / 2] << 16));
    const bool cls0 = block_exponent(fabsf(v)) >= pc - 14;
    const int x = __float2int_rn(mul_pow2(v, cls0 ? 21 - pc : 36 - pc));
    w[k] = digit_codes8(uint32_t(x) + kDigitBias);
    m0 |= cls0 ? (0xFu << (4 * k)) : 0u;
  }
  transpose8_nibbles(w);  // w[i]: nibble k = code of digit i of element k
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    rows[i] = w[i] & m0;
    rows[8 + i] = w[i] & ~m0;
  }
}

// Poll the tagged words (epoch << 32 | f32 bits) at words[k * kTileRows], k < n, except k = own
// (whose value is `own_val`), until each carries `epoch`; return their sum in k order. A word
// that never arrives (bounded wait) raises kErrWaitTimeout and counts as NaN.
__device__ __forceinline__ float sum_tagged(const unsigned long long* words, int n, int own, float own_val,
                                            uint32_t epoch, uint32_t* err) {
  float pv[kMaxCtasPerGroup];
  uint32_t pending = 0u;
#pragma unroll
  for (int k = 0; k < kMaxCtasPerGroup; ++k) {
    pv[k] = k == own ? own_val : 0.f;
    if (k < n && k != own) pending |= 1u << k;
  }
  const uint64_t t0 = globaltimer_ns();
  while (pending) {
    unsigned long long w[kMaxCtasPerGroup];  // every pending word in flight at once, then the checks
#pragma unroll
    for (int k = 0; k < kMaxCtasPerGroup; ++k)
      if (pending & (1u << k)) w[k] = ld_relaxed_gpu_u64(words + k * kTileRows);
#pragma unroll
    for (int k = 0; k < kMaxCtasPerGroup; ++k) {
      if ((pending & (1u << k)) && uint32_t(w[k] >> 32) == epoch) {
        pv[k] = __uint_as_float(uint32_t(w[k]));
        pending &= ~(1u << k);
      }
    }
    if (pending && globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(err, kErrWaitTimeout);
#pragma unroll
      for (int k = 0; k < kMaxCtasPerGroup; ++k)
        if (pending & (1u << k)) pv[k] = __uint_as_float(0x7fc00000u);
      break;
    }
  }
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxCtasPerGroup; ++k)
    if (k < n) sum += pv[k];
  return sum;
}

// A finished piece of a tile (the units of it that this CTA ran), on the 128 epilogue threads.
// A whole tile is final. A tile whose K range is split across CTAs is finished by a fixed CTA,
// the one holding its first unit: that piece is the last of its run, so waiting there holds up
// nothing else. Every other CTA of the tile stores its partial rows into the tile's slots
// (op.split_words) as 64-bit words tagged with the call's epoch (op.epoch); the finishing CTA
// polls them and adds the pieces in CTA order, so the result never depends on timing, then
// records the call in the tile's epoch count (op.split_epochs). Ops that finish their pieces
// themselves (kOwnPieces) get them as they are.
template <class Shape, class Op>
__device__ void finish_piece(Op& op, GemvCtl& ctl, const Scratch& sc, int tile, int row, float val, int in_piece) {
  constexpr int UPT = Shape::kUnitsPerTile;
  const int64_t total = Shape::kTotalUnits, grid = gridDim.x;
  if constexpr (Op::kOwnPieces) {
    op.finish_piece(tile, row, val, in_piece, ctl);
  } else {
    if (in_piece != UPT) {
      const int first = cta_of_unit(int64_t(tile) * UPT, grid, total);
      const int span = cta_of_unit(int64_t(tile) * UPT + UPT - 1, grid, total) - first + 1;
      if (span > kMaxCtasPerGroup) {  // launchers keep every tile within the slots
        if (row == 0) atomicOr(sc.err, kErrInternal);
        return;
      }
      unsigned long long* words = op.split_words + size_t(tile) * kMaxCtasPerGroup * kTileRows + row;
      if (int(blockIdx.x) != first) {
        st_relaxed_gpu_u64(words + (blockIdx.x - first) * kTileRows,
                           (static_cast<unsigned long long>(op.epoch) << 32) | __float_as_uint(val));
        return;
      }
      val = sum_tagged(words, span, 0, val, op.epoch, sc.err);
    }
    if (row == 0) op.split_epochs[tile] = op.epoch;
    op.finalize_tile(tile, row, val, ctl);
  }
}

// Engine driver. `op` supplies:
//   void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const  (TMA)
//   void load_scales(uint8_t* dst, int tile, int kc, uint64_t* bar, uint64_t policy) const (nvfp4)
//   void prefetch_l2(int u0, int u1) const      units [u0, u1) into L2 (may do nothing)
//   static bool kRms, int kRmsGroups   whether the activation is RMS-normalised over its
//                                      kRmsGroups * 16 elements (every group is then loaded)
//   void prologue(GemvCtl&)            scalar loads, after the wait on the preceding kernel
//   void load_static(int g, uint4 (&raw)[4]) const  before the wait on the preceding kernel:
//                                      issue the loads of group g's static inputs (gamma in raw[2..3])
//   void load_group(int g, uint4 (&raw)[4]) const   issue the loads of 16-element group g of
//                                      the activation (bf16, raw[0..1])
//   void finish_group(const uint4 (&raw)[4], float inv, float (&v)[16]) const   the activation
//                                      (bf16-exact values)
//   void finalize_tile(int tile, int row, float v, GemvCtl&) const   all 128 epilogue threads
//   unsigned long long* split_words, uint32_t* split_epochs, uint32_t epoch   split tiles' slots,
//                                      per-tile call counts and this call's epoch (finish_piece)
//   static bool kOwnPieces             the op finishes every tile piece itself:
//   void finish_piece(int tile, int row, float v, int units, GemvCtl&) const
//   uint32_t tx_bytes                  bytes one unit delivers (codes and, nvfp4, block scales)
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
    for (int i = 0; i < S; ++i) {
      mbar_init(&ctl.full[i], 1);
      mbar_init(&ctl.sready[i], 4);  // nvfp4: the four epilogue warps put the unit's scales in TMEM
    }
    for (int i = 0; i < 16; ++i) {
      mbar_init(&ctl.done[i], 1);    // the unit's MMAs have completed (one commit per unit)
      mbar_init(&ctl.tempty[i], 4);  // fp8: the epilogue is done with the TMEM slot
    }
    for (int i = 0; i < Shape::kDSlots; ++i) {
      mbar_init(&ctl.dfull[i], 1);   // nvfp4: the tile accumulator is complete
      mbar_init(&ctl.dempty[i], 4);  // nvfp4: the epilogue has read it
    }
    mbar_init(&ctl.drain, 1);
    for (int i = 0; i < 16; ++i) mbar_init(&ctl.bready[i], 1);  // one arrival per built B slot
    ctl.abort = 0;
    ctl.pmax = -1000;
    ctl.nonfinite = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (c.warp == 1) tmem_alloc(&ctl.tmem_base, Shape::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ctl.tmem_base;

  // Weights do not depend on the preceding kernel: the first kPreWait units (the whole ring:
  // measured faster than holding part of it back) are requested before waiting on it; the L2
  // prefetch beyond the ring follows this CTA's activation loads.
  const uint64_t policy = l2_evict_first_policy();
  const int prefetch = c.n < S ? c.n : S;
  const int prewait = prefetch < Shape::kPreWait ? prefetch : Shape::kPreWait;
  // units [i0, i1) into their (free) stages, thread i0 + k of the CTA issuing unit i0 + k: each
  // TMA issue costs its thread tens of nanoseconds, so a single thread would stall the prologue.
  auto request = [&](int i0, int i1) {
    const int i = i0 + c.tid;
    if (i < i1) {
      const int u = c.u0 + i;
      mbar_arrive_expect_tx(&ctl.full[i], op.tx_bytes);
      op.load_unit(c.stage(i), u / UPT, u % UPT, &ctl.full[i], policy);
      if constexpr (Shape::kFp4) op.load_scales(c.stage(i) + Shape::kABytes, u / UPT, u % UPT, &ctl.full[i], policy);
    }
  };
  request(0, prewait);
  __syncwarp();  // CTA barriers below need converged warps

  // Epilogue warps (2-5): their lane quarter of TMEM, a flag that turns their later work into
  // no-ops after a failed wait (their loops keep their shape for the named barriers), and for
  // nvfp4 weights the copy of block scales of units [prep, lim) from the stages into TMEM, in
  // unit order. Row m's 16 scale bytes hold MMA j's 4 scales at bytes 4j..4j+3; this lane
  // writes rows lane + 32 g (g = 0..3) to columns 4j + g of its lane quarter.
  const uint32_t lane_addr = uint32_t((c.warp & 3) * 32) << 16;
  bool ok = true;
  int prep = 0;
  auto prepare = [&](int lim) {
    for (; prep < lim; ++prep) {
      const int s = prep % S;
      if (ok) ok = mbar_wait_or_abort(&ctl.full[s], uint32_t((prep / S) & 1), abort, sc.err);
      if (ok) {
        const uint8_t* scl = c.stage(s) + Shape::kABytes;
        uint32_t w[16];
        uint32_t sign = 0u;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint4 r = *reinterpret_cast<const uint4*>(scl + (c.lane + 32 * g) * 16);
          w[g] = r.x;
          w[4 + g] = r.y;
          w[8 + g] = r.z;
          w[12 + g] = r.w;
          sign |= r.x | r.y | r.z | r.w;
        }
        if (sign & 0x80808080u) atomicOr(sc.err, kErrNegativeScale);
        tmem_st16(tbase + lane_addr + Shape::kColSfa + uint32_t(s) * 16u, w);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (c.lane == 0) mbar_arrive(&ctl.sready[s]);
    }
  };
  if constexpr (Shape::kFp4) {
    // B block scales (1.0 for every block) and the first units' A scales into TMEM while the
    // preceding kernel finishes
    if (c.warp >= 2 && c.warp < 6) {
      const uint32_t one[4] = {0x38383838u, 0x38383838u, 0x38383838u, 0x38383838u};
      tmem_st4(tbase + lane_addr + Shape::kColSfb, one);
      tmem_st_wait();
      prepare(prewait < 2 ? prewait : 2);
    }
  }
  // activation -> B operand (only the K units this CTA touches). Every global load of the
  // prologue is issued before any is used; the normalisation weights (static) before the wait
  // on the preceding kernel, its output right after it.
  float* gexp = reinterpret_cast<float*>(smem + Shape::kOffExp);  // fp8: [slot][group] 2^-E
  uint16_t* hsm = reinterpret_cast<uint16_t*>(smem + Shape::kOffH);  // nvfp4: [slot][256] bf16
  constexpr int MAXG = 2;  // 16-element groups per thread
  static_assert(!Op::kRms || Op::kRmsGroups <= MAXG * kGemvThreads, "RMS statistic: too many groups");
  static_assert(Shape::kBSlots * 16 <= MAXG * kGemvThreads, "B slots: too many groups");
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
    if (have[q]) op.load_static(grp[q], raw[q]);
  }
  pdl_wait_primary();
  pdl_launch_dependents();
  G4_STAMP(sc, 1);
  {
    // the activation's loads go out first: the op's scalar prologue (offsets, then the copies that
    // depend on them) would otherwise hold them back by a round trip
#pragma unroll
    for (int q = 0; q < MAXG; ++q)
      if (have[q]) op.load_group(grp[q], raw[q]);
    op.prologue(ctl);  // scalar loads only
    // The rest of the ring (and the L2 prefetch beyond it) is requested once the issuing
    // thread's activation loads have landed: issued earlier, the weight data queued for this SM
    // delays the activation's return by microseconds.
    auto request_rest = [&]() {
      request(prewait, prefetch);
      // the next units go to L2 only: the ring's loads then hit L2 instead of waiting on HBM
      if (c.tid == kGemvThreads - 1)
        op.prefetch_l2(c.u0 + prefetch, c.u0 + (prefetch + Shape::kL2Ahead < c.n ? prefetch + Shape::kL2Ahead : c.n));
    };
    float inv = 0.f;
    G4_STAMP(sc, 9);
    if constexpr (Op::kRms) {
      double ss = 0.0;
#pragma unroll
      for (int q = 0; q < MAXG; ++q)
        if (have[q]) ss += sum_squares_bf16x16(raw[q][0], raw[q][1]);
      request_rest();
      G4_STAMP(sc, 12);
      inv = rms_inverse(block_sum_d(ss, ctl.red_d), Op::kRmsGroups * 16);
      G4_STAMP(sc, 13);
    }
    float v[MAXG][16];
    int slot[MAXG];
    uint32_t umax[MAXG];  // fp8: this group's max |v| bits
#pragma unroll
    for (int q = 0; q < MAXG; ++q) {
      slot[q] = c.bslot(grp[q] / 16);
      have[q] = have[q] && slot[q] < nslots;
      umax[q] = 0u;
      if (have[q]) {
        op.finish_group(raw[q], inv, v[q]);
        float amax = 0.f;
        bool nan = false;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          amax = fmaxf(amax, fabsf(v[q][j]));
          nan = nan || v[q][j] != v[q][j];
        }
        if constexpr (Shape::kFp4) {
          const int P = block_exponent(amax);
          if (P > 127 || nan) ctl.nonfinite = 1u;
          atomicMax(&ctl.pmax, P);
          uint32_t bits[8];  // the bf16 values (exact) for the digit pass
#pragma unroll
          for (int j = 0; j < 8; ++j)
            bits[j] = (__float_as_uint(v[q][2 * j]) >> 16) | (__float_as_uint(v[q][2 * j + 1]) & 0xffff0000u);
          uint4* dst = reinterpret_cast<uint4*>(hsm + slot[q] * 256 + (grp[q] % 16) * 16);
          dst[0] = make_uint4(bits[0], bits[1], bits[2], bits[3]);
          dst[1] = make_uint4(bits[4], bits[5], bits[6], bits[7]);
        } else {  // one exponent per 256-element unit; non-negative floats order as ints
          umax[q] = __float_as_uint(amax);
        }
      }
    }
    if constexpr (!Op::kRms) request_rest();
    if constexpr (Shape::kFp4) __syncthreads();  // the CTA's largest exponent (pmax) is complete
    G4_STAMP(sc, 10);
    G4_STAMP_WARP(sc, 4);
    if constexpr (Shape::kFp4) {
      // digit rows, one thread per 8 elements: a warp builds a whole slot (warp w slots w, w + 7,
      // ...) and arrives on its barrier, so the relay releases a unit as soon as its slot is built
      const int pc = ctl.pmax;
      for (int hb = c.tid; hb < nslots * 32; hb += kGemvThreads) {  // warp-uniform
        const int sl = hb / 32, e8 = hb % 32;  // elements 8 e8 .. 8 e8 + 7 of slot sl
        uint32_t rows[16];
        nvf4_digit_rows8(*reinterpret_cast<const uint4*>(hsm + sl * 256 + e8 * 8), pc, rows);
        uint8_t* bs = c.bsm + size_t(sl) * Shape::kBSlotBytes;
#pragma unroll
        for (int r = 0; r < 16; ++r) *reinterpret_cast<uint32_t*>(bs + sw128_offset(r, e8 * 4)) = rows[r];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the tensor cores read it
        __syncwarp();
        if (c.lane == 0) mbar_arrive(&ctl.bready[sl]);
      }
    } else {
      // exponent E of a max |v| so that max |v| 2^E lies in [128, 256)
      auto exponent_of = [](float a) {
        int e = 0;
        if (a > 0.f) {
          e = 7 - (int((__float_as_uint(a) >> 23) & 0xff) - 127);
          e = e > 120 ? 120 : (e < -120 ? -120 : e);
        }
        return e;
      };
      // Slot by slot, with no CTA-wide barrier: the 16 groups of a K unit are held by 16
      // consecutive threads (j = tid + 224 q and j / 16 name the unit), an aligned half-warp, so
      // the unit's largest |v| is a half-warp reduction; the half-warp then writes the unit's
      // terms and arrives on the slot's barrier, and the relay releases a unit as soon as its
      // slot is ready (the first MMAs start while later slots are still being built).
#pragma unroll
      for (int q = 0; q < MAXG; ++q) {
        uint32_t m = umax[q];
#pragma unroll
        for (int o = 8; o; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (have[q]) {
          const int e16 = (grp[q] % 16) * 16;
          const int e = exponent_of(__uint_as_float(m));
          const float up = pow2f(e);
          gexp[slot[q] * 16 + grp[q] % 16] = pow2f(-e);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[q][j] *= up;
          uint4 tm[8];
          split_terms16<8>(v[q], tm);
          uint8_t* atom = c.bsm + size_t(slot[q]) * Shape::kBSlotBytes + (e16 / 128) * 1024;
          const uint32_t kb = e16 % 128;
#pragma unroll
          for (int r = 0; r < 8; ++r) *reinterpret_cast<uint4*>(atom + sw128_offset(r, kb)) = tm[r];
          if (q == 0) G4_STAMP_WARP(sc, 5);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the tensor cores read it
          if (q == 0) G4_STAMP_WARP(sc, 6);
        }
        __syncwarp();
        if (have[q] && (c.lane & 15) == 0) mbar_arrive(&ctl.bready[slot[q]]);
      }
    }
    G4_STAMP(sc, 11);
    G4_STAMP_WARP(sc, 7);
  }
  G4_STAMP(sc, 2);

  if (c.warp == 0) {
    // ---------------------------------------------------------------- producer
    if (c.lane == 0) {
      int issued = prefetch;
      for (int i = prefetch; i < c.n; ++i) {
        const int s = i % S;
        // stage s is free once the MMAs of unit i - S have completed
        const int r = i - S;
        const bool free = Shape::kFp4 ? mbar_wait_or_abort(&ctl.done[s], uint32_t((r / S) & 1), abort, sc.err)
                                      : mbar_wait_or_abort(&ctl.done[r % T], uint32_t((r / T) & 1), abort, sc.err);
        if (!free) break;
        const int u = c.u0 + i;
        mbar_arrive_expect_tx(&ctl.full[s], op.tx_bytes);
        op.load_unit(c.stage(s), u / UPT, u % UPT, &ctl.full[s], policy);
        if constexpr (Shape::kFp4) op.load_scales(c.stage(s) + Shape::kABytes, u / UPT, u % UPT, &ctl.full[s], policy);
        if ((i - prefetch) % 2 == 0 && i + Shape::kL2Ahead < c.n)  // two units per bulk L2 prefetch
          op.prefetch_l2(u + Shape::kL2Ahead, c.u0 + (i + Shape::kL2Ahead + 2 < c.n ? i + Shape::kL2Ahead + 2 : c.n));
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
    }
    __syncwarp();  // lanes 1..31 wait here for lane 0: the teardown barrier needs whole warps
  } else if (c.warp == kRelayWarp) {
    // ---------------------------------------------------------------- relay
    // Unit i may be issued once it landed (fp8: and its TMEM slot is free; nvfp4: once its
    // scales are in TMEM and, for the first unit of a tile piece, its accumulator is free).
    // Both warps pass the issue barrier once per unit; a failed wait aborts both.
    int piece = -1;
    for (int i = 0; i < c.n; ++i) {
      bool bad = false;
      if (c.lane == 0) {
        const int s = i % S, kc = (c.u0 + i) % UPT;
        if constexpr (Shape::kFp4) {
          const bool first = i == 0 || kc == 0;
          if (first) ++piece;
          bad = !mbar_wait_or_abort(&ctl.sready[s], uint32_t((i / S) & 1), abort, sc.err) ||
                !mbar_wait_or_abort(&ctl.bready[c.bslot(kc)], 0u, abort, sc.err);
          if (!bad && first && piece >= Shape::kDSlots)
            bad = !mbar_wait_or_abort(&ctl.dempty[piece % Shape::kDSlots], uint32_t(((piece / Shape::kDSlots) - 1) & 1),
                                      abort, sc.err);
        } else {
          bad = !mbar_wait_or_abort(&ctl.full[s], uint32_t((i / S) & 1), abort, sc.err) ||
                (i >= T && !mbar_wait_or_abort(&ctl.tempty[i % T], uint32_t(((i / T) - 1) & 1), abort, sc.err)) ||
                !mbar_wait_or_abort(&ctl.bready[c.bslot(kc)], 0u, abort, sc.err);
        }
      }
#ifdef G4_TRACE
      if (sc.trace && blockIdx.x == 0 && i < 64 && c.lane == 0) sc.trace[3128 + i] = globaltimer_ns();  // unit ready
#endif
      __syncwarp();
      if (named_bar_or(kIssueBarrier, kIssueThreads, bad)) break;
      if (c.lane == 0 && i == 0) G4_STAMP_T(sc, 3);        // first unit released to the issuer
      if (c.lane == 0 && i == c.n - 1) G4_STAMP_T(sc, 4);  // last unit released
#ifdef G4_TRACE
      if (sc.trace && blockIdx.x == 0 && i < 64 && c.lane == 0) sc.trace[3064 + i] = globaltimer_ns();  // released
#endif
    }
  } else if (c.warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    int piece = -1;
    for (int i = 0; i < c.n; ++i) {
      if (named_bar_or(kIssueBarrier, kIssueThreads, false)) break;
      tc_fence_after();
      if (c.lane == 0) {  // (no trace stamps here: a global store of this thread waits for its MMAs)
        const int s = i % S, t = i % T, kc = (c.u0 + i) % UPT;
        const uint32_t a_base = smem_u32(c.stage(s));
        const uint32_t b_base = smem_u32(c.bsm) + uint32_t(c.bslot(kc)) * Shape::kBSlotBytes;
        if constexpr (Shape::kFp4) {
          const bool first = i == 0 || kc == 0;
          if (first) ++piece;
          const uint32_t d = tbase + uint32_t(piece % Shape::kDSlots) * 16u;
          const uint32_t sfa = tbase + Shape::kColSfa + uint32_t(s) * 16u;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            umma_nvf4(d, umma_desc_sw128(a_base + 32u * j), umma_desc_sw128(b_base + 32u * j), Shape::kIdesc,
                      sfa + 4 * j, tbase + Shape::kColSfb, uint32_t(!first || j > 0));
          umma_commit(&ctl.done[s]);
          if (i == c.n - 1 || kc == UPT - 1) umma_commit(&ctl.dfull[piece % Shape::kDSlots]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t h = j / 4, kk = j % 4;
            const uint64_t ad = umma_desc_sw128(a_base + h * 16384u + kk * 32u);
            const uint64_t bd = umma_desc_sw128(b_base + h * 1024u + kk * 32u);
            umma_f8f6f4(tbase + uint32_t(t * 8), ad, bd, Shape::kIdesc, uint32_t(j > 0));
          }
          umma_commit(&ctl.done[t]);
        }
      }
      __syncwarp();
    }
    // nothing of ours may still be running when TMEM is released
    if (c.lane == 0) {
      umma_commit(&ctl.drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ctl.drain, 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = c.warp & 3;
    const int row = quarter * 32 + c.lane;
    float acc = 0.f;
    int in_piece = 0, piece = -1;
    for (int i = 0; i < c.n; ++i) {
      const int u = c.u0 + i, tile = u / UPT, kc = u % UPT, t = i % T;
      const bool last = kc == UPT - 1 || i == c.n - 1;
      ++in_piece;
      if constexpr (Shape::kFp4) {
        if (i == 0 || kc == 0) ++piece;
        if (!last) continue;
        prepare(i + S < c.n ? i + S : c.n);  // keep the MMAs fed while this piece is finished
        const int ds = piece % Shape::kDSlots;
        if (ok) ok = mbar_wait_or_abort(&ctl.dfull[ds], uint32_t((piece / Shape::kDSlots) & 1), abort, sc.err);
        if (row == 0 && piece == 0) G4_STAMP_T(sc, 5);
        tc_fence_after();
        float d[16];
        if (ok) {
          tmem_ld16(tbase + lane_addr + uint32_t(ds * 16), d);
          tmem_ld_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (c.lane == 0) mbar_arrive(&ctl.dempty[ds]);
        if (ok) {
          const int pc = ctl.pmax;
          acc = mul_pow2(combine_digits8(d), pc - 20) + mul_pow2(combine_digits8(d + 8), pc - 35);
          if (ctl.nonfinite) acc = __uint_as_float(0x7fc00000u);
        }
      } else {
        if (ok) ok = mbar_wait_or_abort(&ctl.done[t], uint32_t((i / T) & 1), abort, sc.err);
        // (the slot's exponent below was written before its barrier, which the unit's release
        // passed; this test makes that order explicit for these threads)
        if (ok) ok = mbar_wait_or_abort(&ctl.bready[c.bslot(kc)], 0u, abort, sc.err);
        if (row == 0 && i == 0) G4_STAMP_T(sc, 5);
        tc_fence_after();
        if (ok) {
          float d[8];
          tmem_ld8(tbase + lane_addr + uint32_t(t * 8), d);
          tmem_ld_wait();
          acc = fmaf(combine_terms<8>(d), gexp[c.bslot(kc) * 16], acc);
        }
        tc_fence_before();
        __syncwarp();
        if (c.lane == 0) mbar_arrive(&ctl.tempty[t]);
        if (!last) continue;
      }
#ifdef G4_TRACE
      if (sc.trace && blockIdx.x == 0 && i < 64 && row == 0) sc.trace[3192 + i] = globaltimer_ns();
#endif
      finish_piece<Shape>(op, ctl, sc, tile, row, acc, in_piece);
      acc = 0.f;
      in_piece = 0;
    }
    if constexpr (Shape::kFp4) prepare(c.n);
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
