// The token-batch engine of sm_100a (a CTA per SM, 480 threads): one weight matrix streamed from
// HBM once for M = 2..64 tokens. tcgen05.mma kind::f16, M = 128 weight rows, N = MPAD (the tokens,
// zero-padded to a multiple of 16), K = 16 per instruction; A (the weights, dequantised by eight
// warps from e2m1 codes with e4m3 block scales or from e4m3 codes) in tensor memory, B (the
// tokens' activation rows, f16 or bf16) by TMA. Every code times its scale is exact in f16 and
// bf16, so every product is exact and the tensor cores' f32 sums are the only difference from a
// reference's f32 contraction of the dequantised weights.
//
// Users: the batched feed-forward (g4_batch.cu) and the batched QKV and O projections
// (g4_batch_attn.cu). An op supplies the unit grid, the weight / activation copies and the
// epilogue of a finished tile piece (`finish`); pieces of a tile that spans several CTAs go out as
// epoch-tagged split-K words (sc.batch_words, two piece slots per CTA) or are added by the tile's
// first CTA (split_begin / split_chunk).
#pragma once
#include <type_traits>

#include "g4_gemv.cuh"
#include "g4_ops.cuh"

namespace g4 {
namespace {

static_assert(kBatchEpoch < kCounterCount, "batch epoch counter inside the counter block");

constexpr int kBThreads = 480;  // 15 warps
constexpr int kWProducer = 0, kWIssuer = 1, kWRelay = 2, kWDq0 = 7, kDqWarps = 8;  // epilogue: warps 3-6
constexpr int kBIssueBarrier = 2;  // issuer + relay (64 threads)
constexpr int kBEpiBarrier = 1;    // the four epilogue warps
constexpr int kBMaxStages = 8;

struct BatchCtl {
  uint64_t full_a[kBMaxStages], full_b[kBMaxStages], empty[kBMaxStages];
  uint64_t hfull[3], hempty[3], done[8], tempty[8], drain;
  uint32_t tmem_base;
  uint32_t abort;
};

// Profiling builds: per-unit timestamps of CTA 0 at trace[3000 + 64 k + i] (k: 0 producer issued,
// 1 second half dequantised, 2 released to the issuer, 3 epilogue done, 4 / 6 first / second half's
// A slot free, 5 first half dequantised).
#ifdef G4_TRACE
#define G4_UNIT_STAMP(sc, k, i)                                                                           \
  do {                                                                                                \
    if ((sc).trace && blockIdx.x == 0 && (i) < 64) (sc).trace[3000 + 64 * (k) + (i)] = globaltimer_ns(); \
  } while (0)
#else
#define G4_UNIT_STAMP(sc, k, i) \
  do {                          \
  } while (0)
#endif

template <int MPAD, bool FP8 = false>
struct BatchShape {
  static constexpr int kMpad = MPAD;  // B rows: the tokens, zero-padded
  // a unit's weights: packed e2m1 codes (128 rows x 256 K) and their ue4m3 block scales, or fp8
  // codes as two K halves of 128 rows x 128 codes (per-row scales come with the epilogue)
  static constexpr int kABytes = FP8 ? 2 * kTileRows * 128 : kTileRows * 128;
  static constexpr int kScaleBytes = FP8 ? 0 : kTileRows * 16;
  static constexpr int kBColBytes = MPAD * 128;       // B: one 64-element K column block of MPAD rows
  static constexpr int kBBytes = 4 * kBColBytes;
  static constexpr int kStageBytes = kABytes + kScaleBytes + kBBytes;
  static constexpr size_t kXBytes = size_t(16) * 64 * 2;  // up/gate: bf16 gate, then gelu [16 tokens][64]
  static constexpr int kStagesFit = int((227 * 1024 - kXBytes - sizeof(BatchCtl) - 1024) / kStageBytes);
  static constexpr int kStages = kStagesFit < kBMaxStages ? kStagesFit : kBMaxStages;
  // TMEM (512 columns): kTSlots unit accumulators (one per unit in flight) of kChains x MPAD
  // columns, each row's running sum of its tile piece (MPAD columns), then the dequantised A
  // operand: a ring of kAHalves half units, 64 columns each (128 rows x 128 K 16-bit values, two
  // per column). A unit's 16 K steps go round-robin to kChains independent accumulators: MMAs
  // that accumulate into one D run back to back at the tensor cores' latency, independent ones
  // overlap (one chain of 16 held a unit to about 1 us). The same count for every MPAD keeps a
  // token's result independent of the batch it came in.
  static constexpr int kChains = 2;
  static constexpr int kTSlotsFit = (512 - 3 * 64 - MPAD) / (kChains * MPAD);
  static constexpr int kTSlots = kTSlotsFit < 8 ? kTSlotsFit : 8;
  static constexpr uint32_t kSlotCols = uint32_t(kChains) * MPAD;
  static constexpr uint32_t kColSum = uint32_t(kTSlots) * kSlotCols;
  static constexpr uint32_t kColA = (kColSum + MPAD + 31) / 32 * 32;
  static constexpr int kAHalves = 3;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr size_t kOffX = size_t(kStages) * kStageBytes;
  static constexpr size_t kOffCtl = kOffX + kXBytes;
  static constexpr size_t kSmemBytes = kOffCtl + sizeof(BatchCtl) + 1024;
  static_assert(kColA + kAHalves * 64 <= kTmemCols && kTSlots >= 2, "TMEM budget");
  static_assert(kStages >= 3, "pipeline depth");
  static_assert(MPAD % 16 == 0 && MPAD <= kBatchMax, "N of the MMA");
  static_assert(kStages <= kBMaxStages, "barrier arrays");
  static_assert(kStageBytes % 1024 == 0 && (kABytes + kScaleBytes) % 1024 == 0, "1024-byte swizzle atoms");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Eight e4m3 codes (element i in byte i) as eight f16 or, bf16 = true, bf16 (exact: every e4m3
// value is an f16 and a bf16 value).
__device__ __forceinline__ uint4 expand8_e4m3(uint32_t lo, uint32_t hi, bool bf16) {
  uint32_t h[4];
  asm("{\n .reg .b16 a, b, c, d;\n mov.b32 {a, b}, %4;\n mov.b32 {c, d}, %5;\n"
      " cvt.rn.f16x2.e4m3x2 %0, a;\n cvt.rn.f16x2.e4m3x2 %1, b;\n"
      " cvt.rn.f16x2.e4m3x2 %2, c;\n cvt.rn.f16x2.e4m3x2 %3, d;\n}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(lo), "r"(hi));
  if (bf16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
      const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
      h[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Eight packed e2m1 codes (element 2i in the low nibble of byte i) times their ue4m3 block scale,
// as eight bf16 (element j in half j % 2 of word j / 2). Exact: see the file comment.
__device__ __forceinline__ uint4 dequant8_bf16(uint32_t codes, uint32_t scale_byte) {
  uint32_t s2, h[4];
  asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}" : "=r"(s2) : "r"(scale_byte * 0x101u));
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(codes));
  const __half2 sc = *reinterpret_cast<const __half2*>(&s2);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 p = __hmul2(*reinterpret_cast<const __half2*>(&h[i]), sc);
    const float2 f = __half22float2(p);
    const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
    o[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// The same as eight f16 (exact too): the conversion and one multiply per pair.
__device__ __forceinline__ uint4 dequant8_f16(uint32_t codes, uint32_t scale_byte) {
  uint32_t s2, h[4];
  asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}" : "=r"(s2) : "r"(scale_byte * 0x101u));
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(codes));
  const __half2 sc = *reinterpret_cast<const __half2*>(&s2);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 p = __hmul2(*reinterpret_cast<const __half2*>(&h[i]), sc);
    o[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void st_release_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Split tiles. The tile piece of the CTA holding the tile's first unit gets the other pieces (later
// CTAs of the tile) added in CTA order; every other piece is published as epoch-tagged words, one
// per (token, row), in its CTA's slot. The publishing thread of a row stores its last token's word
// with release semantics after the others, so a reader that acquires that word with this call's
// tag sees the whole row: the finisher polls one word per piece (all pieces in flight at once),
// then reads the rest with independent loads. Tokens go 16 at a time from the row's running sum
// in TMEM (`tsum`, this thread's lane). Epilogue threads; `ok` false: nothing is read (NaN).
struct SplitPiece {
  unsigned long long* words;
  uint32_t tag;
  int first, later;  // the tile's first CTA; pieces after it
  bool publish;      // this CTA holds a later piece
};

template <int MPAD>
__device__ SplitPiece split_begin(int tile, int upt, int64_t total, int row, int M, uint32_t tsum, uint32_t tag,
                                  unsigned long long* words, bool& ok, uint32_t* err) {
  SplitPiece sp;
  const int64_t first_unit = int64_t(tile) * upt, grid = gridDim.x;
  sp.words = words;
  sp.tag = tag;
  sp.first = cta_of_unit(first_unit, grid, total);
  sp.later = cta_of_unit(first_unit + upt - 1, grid, total) - sp.first;
  sp.publish = sp.first != int(blockIdx.x);
  const unsigned long long tag_bits = static_cast<unsigned long long>(tag) << 32;
  if (sp.publish) {
    unsigned long long* w = words + size_t(blockIdx.x) * kBatchMax * kTileRows + row;
#pragma unroll
    for (int c = 0; c < MPAD; c += 16) {
      float a[16];
      if (ok) {
        tmem_ld16(tsum + uint32_t(c), a);
        tmem_ld_wait();
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const unsigned long long x = tag_bits | (ok ? __float_as_uint(a[j]) : 0x7fc00000u);
        if (c + j < M - 1) st_relaxed_gpu_u64(w + (c + j) * kTileRows, x);
        if (c + j == M - 1) st_release_gpu_u64(w + (c + j) * kTileRows, x);
      }
    }
    return sp;
  }
  constexpr int kPoll = 8;  // pieces whose last word is polled together
  const uint64_t t0 = globaltimer_ns();
  for (int g0 = 0; g0 < sp.later && ok; g0 += kPoll) {
    uint32_t pending = 0u;
#pragma unroll
    for (int k = 0; k < kPoll; ++k)
      if (g0 + k < sp.later) pending |= 1u << k;
    while (pending) {
      unsigned long long x[kPoll];  // every pending piece's last word in flight at once
#pragma unroll
      for (int k = 0; k < kPoll; ++k)
        if (pending & (1u << k))
          x[k] = ld_acquire_gpu_u64(words + (size_t(sp.first + 1 + g0 + k) * kBatchMax + (M - 1)) * kTileRows + row);
#pragma unroll
      for (int k = 0; k < kPoll; ++k)
        if ((pending & (1u << k)) && uint32_t(x[k] >> 32) == tag) pending &= ~(1u << k);
      if (pending && globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(err, kErrWaitTimeout);
        ok = false;
        break;
      }
    }
  }
  return sp;
}

// The finisher's sums of tokens [c, c + 16): its own piece from TMEM plus the later pieces in CTA order.
__device__ __forceinline__ void split_chunk(const SplitPiece& sp, int c, int M, int row, uint32_t tsum, bool ok,
                                            float (&a)[16]) {
  if (ok) {
    tmem_ld16(tsum + uint32_t(c), a);
    tmem_ld_wait();
  }
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (!ok) a[j] = __uint_as_float(0x7fc00000u);
  for (int k = 0; k < sp.later; ++k) {
    const unsigned long long* w = sp.words + (size_t(sp.first + 1 + k) * kBatchMax + c) * kTileRows + row;
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {  // independent loads, all in flight before the sums
      const unsigned long long x = (ok && c + j < M) ? __ldcg(w + j * kTileRows) : 0ull;
      v[j] = uint32_t(x >> 32) == sp.tag ? __uint_as_float(uint32_t(x)) : __uint_as_float(0x7fc00000u);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) a[j] += v[j];
  }
}

// A tile piece published whole: the CTA's piece `piece_no` (0 or 1: a CTA's run of units lies
// within two tiles, checked at set-up) goes out as epoch-tagged words, one per (token, row), in the
// CTA's slot; a per-token kernel adds a tile's pieces in CTA order. Epilogue threads (row = this
// thread's TMEM lane); `ok` false: NaN words.
template <int MPAD>
__device__ __forceinline__ void publish_piece(const Scratch& sc, uint32_t tag, int& piece_no, int M, int row,
                                              uint32_t tsum, bool ok) {
  unsigned long long* w =
      sc.batch_words + (size_t(blockIdx.x) * 2 + (piece_no < 2 ? piece_no : 1)) * kBatchMax * kTileRows + row;
  if (piece_no >= 2 && row == 0) atomicOr(sc.err, kErrInternal);
  ++piece_no;
  const unsigned long long tag_bits = static_cast<unsigned long long>(tag) << 32;
#pragma unroll
  for (int c = 0; c < MPAD; c += 16) {
    if (c >= M) break;
    float a[16];
    if (ok) {
      tmem_ld16(tsum + uint32_t(c), a);
      tmem_ld_wait();
    }
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c + j < M) w[size_t(c + j) * kTileRows] = tag_bits | (ok ? __float_as_uint(a[j]) : 0x7fc00000u);
  }
}

// The CTA of the batched grid that holds unit `unit` (contiguous runs, as batch_run splits them)
// and the tile its run starts in: a tile's pieces are CTAs cta_of_unit(first unit) ..
// cta_of_unit(last unit), and the piece of tile t in CTA c is its slot 1 when c's run began in an
// earlier tile.
__host__ __device__ __forceinline__ int run_first_tile(int cta, int64_t grid, int64_t total, int upt) {
  return int(int64_t(cta) * total / grid) / upt;
}

// Engine driver. `op` supplies:
//   static int kUnitsPerTile, kTiles                 the unit grid
//   void load_a(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const
//                                                    codes (kABytes) then scales (kScaleBytes)
//   void load_b(uint8_t* dst, int kc, uint64_t* bar, uint64_t policy) const    4 column blocks
//   void prefetch_l2(int u0, int u1) const
//   void prologue()                                  after the dependency wait (all threads)
//   void finish(BatchCtl&, uint8_t* xbuf, int tile, int row, uint32_t tsum, bool ok)
//                                                    the 128 epilogue threads, per tile piece (its sums:
//                                                    MPAD TMEM columns of this thread's lane at tsum)
template <class Shape, class Op>
__device__ void batch_run(Op& op, uint8_t* smem_raw, const Scratch& sc) {
  constexpr int S = Shape::kStages, MP = Shape::kMpad;
  constexpr int UPT = Op::kUnitsPerTile;
  uint8_t* smem = align1024(smem_raw);
  BatchCtl& ctl = *reinterpret_cast<BatchCtl*>(smem + Shape::kOffCtl);
  auto stage = [&](int s) { return smem + size_t(s) * Shape::kStageBytes; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t total = int64_t(UPT) * Op::kTiles, grid = gridDim.x;
  const int u0 = int(int64_t(blockIdx.x) * total / grid);
  const int n = int(int64_t(blockIdx.x + 1) * total / grid) - u0;
  volatile uint32_t* abort = &ctl.abort;
  constexpr uint32_t kATx = Shape::kABytes + Shape::kScaleBytes;
  constexpr uint32_t kIdesc = Op::kF16 ? umma_idesc_f16(kTileRows, MP) : umma_idesc_bf16(kTileRows, MP);

  G4_STAMP(sc, 0);
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&ctl.full_a[i], 1);
      mbar_init(&ctl.full_b[i], 1);
      mbar_init(&ctl.empty[i], 1);
    }
    for (int i = 0; i < Shape::kAHalves; ++i) {
      mbar_init(&ctl.hfull[i], kDqWarps);  // every dequantisation warp wrote its rows
      mbar_init(&ctl.hempty[i], 1);        // the half's MMAs completed
    }
    for (int i = 0; i < Shape::kTSlots; ++i) {
      mbar_init(&ctl.done[i], 1);    // the unit's MMAs completed
      mbar_init(&ctl.tempty[i], 4);  // the epilogue warps read the unit's accumulator
    }
    mbar_init(&ctl.drain, 1);
    ctl.abort = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == kWIssuer) tmem_alloc(&ctl.tmem_base, Shape::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ctl.tmem_base;
  const uint64_t policy = l2_evict_first_policy();
  const uint64_t policy_b = l2_evict_last_policy();  // every CTA reads the activation rows
  const int prefetch = n < S ? n : S;

  // the first units' weights before the wait on the preceding kernel (thread i: unit i), their
  // activation rows after it
  if (tid < prefetch) {
    const int u = u0 + tid;
    mbar_arrive_expect_tx(&ctl.full_a[tid], kATx);
    op.load_a(stage(tid), u / UPT, u % UPT, &ctl.full_a[tid], policy);
  }
  __syncwarp();
  pdl_wait_primary();
  pdl_launch_dependents();
  G4_STAMP(sc, 1);
  op.prologue();
  if (tid < prefetch) {
    mbar_arrive_expect_tx(&ctl.full_b[tid], Shape::kBBytes);
    op.load_b(stage(tid) + kATx, (u0 + tid) % UPT, &ctl.full_b[tid], policy_b);
  }
  if (tid == kBThreads - 1) op.prefetch_l2(u0 + prefetch, u0 + (prefetch + 6 < n ? prefetch + 6 : n));
  __syncwarp();

  if (warp == kWProducer) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = prefetch;
      for (int i = prefetch; i < n; ++i) {
        const int s = i % S, r = i - S;
        if (!mbar_wait_or_abort(&ctl.empty[s], uint32_t((r / S) & 1), abort, sc.err)) break;
        const int u = u0 + i;
        mbar_arrive_expect_tx(&ctl.full_a[s], kATx);
        op.load_a(stage(s), u / UPT, u % UPT, &ctl.full_a[s], policy);
        mbar_arrive_expect_tx(&ctl.full_b[s], Shape::kBBytes);
        op.load_b(stage(s) + kATx, u % UPT, &ctl.full_b[s], policy_b);
        G4_UNIT_STAMP(sc, 0, i);
        if ((i - prefetch) % 2 == 0 && i + 6 < n) op.prefetch_l2(u + 6, u0 + (i + 8 < n ? i + 8 : n));
        issued = i + 1;
      }
      // every requested copy has landed before the CTA may exit
      for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!(mbar_try_wait(&ctl.full_a[i % S], uint32_t((i / S) & 1)) &&
                 mbar_try_wait(&ctl.full_b[i % S], uint32_t((i / S) & 1))))
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
    }
    __syncwarp();
  } else if (warp >= kWDq0) {
    // ---------------------------------------------------------------- dequantisation
    // Warp w writes TMEM lane quarter w % 4: thread (row, sub), row = 32 (w % 4) + lane, expands K
    // elements [64 sub, 64 sub + 64) of each half unit (two 16-byte chunks of codes, four block
    // scales) into 32 TMEM columns of the half's slot in the A ring.
    const int quarter = warp & 3, r = quarter * 32 + lane, sub = (warp - kWDq0) >> 2;
    const uint32_t a_lane = tbase + (uint32_t(quarter * 32) << 16) + Shape::kColA + uint32_t(sub * 32);
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int s = i % S;
      if (ok) ok = mbar_wait_or_abort(&ctl.full_a[s], uint32_t((i / S) & 1), abort, sc.err);
      const uint8_t* a4 = stage(s);
      for (int h = 0; h < 2; ++h) {
        const int q = 2 * i + h, slot = q % Shape::kAHalves, use = q / Shape::kAHalves;
        if (ok && use > 0) ok = mbar_wait_or_abort(&ctl.hempty[slot], uint32_t((use - 1) & 1), abort, sc.err);
        tc_fence_after();  // the slot's previous MMAs (complete) before this thread's TMEM stores
        if (warp == kWDq0 && lane == 0) G4_UNIT_STAMP(sc, h == 0 ? 4 : 6, i);
        if (ok) {
          uint32_t o[32];
          if constexpr (Shape::kScaleBytes == 0) {
            // fp8: this half's row r holds 128 codes in eight 16-byte chunks; chunks 4 sub .. 4 sub + 3
            const uint8_t* row = a4 + h * (kTileRows * 128) + r * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 cq = *reinterpret_cast<const uint4*>(row + (((4 * sub + q) ^ (r & 7)) << 4));
              const uint4 lo = expand8_e4m3(cq.x, cq.y, !Op::kF16), hi = expand8_e4m3(cq.z, cq.w, !Op::kF16);
              o[8 * q] = lo.x, o[8 * q + 1] = lo.y, o[8 * q + 2] = lo.z, o[8 * q + 3] = lo.w;
              o[8 * q + 4] = hi.x, o[8 * q + 5] = hi.y, o[8 * q + 6] = hi.z, o[8 * q + 7] = hi.w;
            }
          } else {
            const int c0 = 4 * h + 2 * sub;  // code chunks c0, c0 + 1 (32 elements each)
            const uint4 q0 = *reinterpret_cast<const uint4*>(a4 + r * 128 + (((c0) ^ (r & 7)) << 4));
            const uint4 q1 = *reinterpret_cast<const uint4*>(a4 + r * 128 + (((c0 + 1) ^ (r & 7)) << 4));
            const uint32_t sw = *reinterpret_cast<const uint32_t*>(a4 + Shape::kABytes + r * 16 + 8 * h + 4 * sub);
            if (sw & 0x80808080u) atomicOr(sc.err, kErrNegativeScale);
            const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {  // elements 8j .. 8j + 7: block j / 2, columns 4j .. 4j + 3
              const uint4 v = Op::kF16 ? dequant8_f16(w[j], (sw >> (8 * (j / 2))) & 0xffu)
                                       : dequant8_bf16(w[j], (sw >> (8 * (j / 2))) & 0xffu);
              o[4 * j] = v.x;
              o[4 * j + 1] = v.y;
              o[4 * j + 2] = v.z;
              o[4 * j + 3] = v.w;
            }
          }
          tmem_st32(a_lane + uint32_t(slot * 64), o);
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl.hfull[slot]);
        if (warp == kWDq0 && lane == 0) G4_UNIT_STAMP(sc, h == 1 ? 1 : 5, i);
      }
    }
  } else if (warp == kWRelay) {
    // ---------------------------------------------------------------- relay
    // Each half of unit i may be issued once its bf16 rows are written (and, the first half,
    // once the unit's activation rows landed and its TMEM accumulator is free).
    bool stop = false;
    for (int i = 0; i < n && !stop; ++i) {
      const int s = i % S, t = i % Shape::kTSlots;
      for (int h = 0; h < 2; ++h) {
        const int q = 2 * i + h, slot = q % Shape::kAHalves;
        bool bad = false;
        if (lane == 0) {
          bad = !mbar_wait_or_abort(&ctl.hfull[slot], uint32_t((q / Shape::kAHalves) & 1), abort, sc.err);
          if (!bad && h == 0) bad = !mbar_wait_or_abort(&ctl.full_b[s], uint32_t((i / S) & 1), abort, sc.err);
          if (!bad && h == 0 && i >= Shape::kTSlots)
            bad = !mbar_wait_or_abort(&ctl.tempty[t], uint32_t(((i / Shape::kTSlots) - 1) & 1), abort, sc.err);
        }
        __syncwarp();
        if (named_bar_or(kBIssueBarrier, 64, bad)) {
          stop = true;
          break;
        }
        if (h == 0 && lane == 0) G4_UNIT_STAMP(sc, 2, i);
      }
    }
  } else if (warp == kWIssuer) {
    // ---------------------------------------------------------------- MMA issuer
    // Every unit has its own accumulator (16 MMAs, K = 256): the tensor cores' f32 sums stay
    // short and the epilogue adds the units with round-to-nearest, in unit order.
    bool stop = false;
    for (int i = 0; i < n && !stop; ++i) {
      const int s = i % S, t = i % Shape::kTSlots;
      for (int h = 0; h < 2; ++h) {
        if (named_bar_or(kBIssueBarrier, 64, false)) {
          stop = true;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const int slot = (2 * i + h) % Shape::kAHalves;
          const uint32_t d = tbase + uint32_t(t) * Shape::kSlotCols;
          const uint32_t a0 = tbase + Shape::kColA + uint32_t(slot * 64);
          const uint32_t b0 = smem_u32(stage(s) + kATx) + uint32_t(2 * h) * Shape::kBColBytes;
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // K = 16 each: A 8 TMEM columns; B column block j / 4, 32 bytes a step
            const uint32_t cb = j / 4, kk = j % 4;
            const int step = 8 * h + j, chain = step % Shape::kChains;
            umma_16bit_ta(d + uint32_t(chain * MP), a0 + uint32_t(8 * j),
                          umma_desc_sw128(b0 + cb * uint32_t(Shape::kBColBytes) + kk * 32u), kIdesc,
                          uint32_t(step >= Shape::kChains));
          }
          umma_commit(&ctl.hempty[slot]);
          if (h == 1) {
            umma_commit(&ctl.empty[s]);
            umma_commit(&ctl.done[t]);
          }
        }
        __syncwarp();
      }
    }
    if (lane == 0) {  // nothing of ours may still be running when TMEM is released
      umma_commit(&ctl.drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ctl.drain, 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 3-6)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
    uint8_t* xbuf = smem + Shape::kOffX;
    const uint32_t tsum = tbase + lane_addr + Shape::kColSum;
    bool ok = true;
    int in_piece = 0;
    for (int i = 0; i < n; ++i) {
      const int u = u0 + i, tile = u / UPT, kc = u % UPT, t = i % Shape::kTSlots;
      ++in_piece;
      if (ok) ok = mbar_wait_or_abort(&ctl.done[t], uint32_t((i / Shape::kTSlots) & 1), abort, sc.err);
      tc_fence_after();
      // running sum of the piece += this unit (its chains added in order), 16 tokens at a time (f32,
      // round to nearest)
#pragma unroll
      for (int c = 0; c < MP; c += 16) {
        float part[16], sum[16];
        if (ok) {
          const uint32_t slot = tbase + lane_addr + uint32_t(t) * Shape::kSlotCols + uint32_t(c);
          tmem_ld16(slot, part);
          if (in_piece > 1) tmem_ld16(tsum + uint32_t(c), sum);
          tmem_ld_wait();
#pragma unroll
          for (int ch = 1; ch < Shape::kChains; ++ch) {
            float more[16];
            tmem_ld16(slot + uint32_t(ch * MP), more);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) part[j] += more[j];
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) sum[j] = in_piece > 1 ? sum[j] + part[j] : part[j];
          uint32_t bits[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) bits[j] = __float_as_uint(sum[j]);
          tmem_st16(tsum + uint32_t(c), bits);
        }
      }
      if (ok) tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl.tempty[t]);
      if (row == 0) G4_UNIT_STAMP(sc, 3, i);
      if (!(kc == UPT - 1 || i == n - 1)) continue;
      op.finish(ctl, xbuf, tile, row, tsum, ok);
      if (row == 0) G4_STAMP_T(sc, 5);
      in_piece = 0;
    }
  }

  // teardown: every MMA has completed (drain) and every TMEM load has been waited for
  tc_fence_before();
  __syncthreads();
  G4_STAMP(sc, 6);
  if (warp == kWIssuer) {
    tc_fence_after();
    tmem_dealloc(tbase, Shape::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------
// The term-operand engine: FP8 weights at up to kTermTokens tokens.
//
// The weights go to the tensor cores as they are: tcgen05.mma kind::f8f6f4, A = 128 weight rows x
// 32 e4m3 codes from shared memory (K = 32 per instruction, 8 instructions per 256-element unit,
// no dequantisation), B = each token's activation as kTerms = 4 e4m3 terms: for every (unit,
// token) a power of two 2^E brings the unit's largest |h| into [128, 256), and h 2^E = sum_j
// t_j 16^-j with e4m3 terms t_j, each the round-to-nearest e4m3 of the remainder so far (the
// single-token FP8 kernels' split, split_terms16). A term carries 4 significant bits of its
// remainder and the remainder's last bit moves up 4 places per term, so a bf16 element x = h 2^E
// (8 significant bits) is represented exactly when |x| >= 2^-14, i.e. every element within about
// 2^-22 of the unit's largest (below that, the error is under 2^-21 of the scaled unit). The B
// rows are (token, term) pairs, N = 4 MT (MT: the tokens padded to 4, 8 or 16). The products are
// exact and the tensor cores sum them in f32; the epilogue adds each token's terms (smallest
// first) times 2^-E per unit, keeps the piece's running sums in registers and hands them to the
// op's epilogue in TMEM, as batch_run does, so the ops (their tile pieces, split-K words and
// finishing) are the same.
//
// The operand rows are built once per call by batch_terms_kernel into sc.batch_terms
// ([unit][token][term][256 bytes]) and reach shared memory by TMA per unit, from L2.

constexpr int kTThreads = 192;  // warp 0 producer, warp 1 MMA issuer, warps 2-5 epilogue

template <int MT>
struct TermShape {
  static constexpr int kMt = MT;
  static constexpr int kN = MT * kTerms;                // B rows: (token, term)
  static constexpr int kABytes = 2 * kTileRows * 128;   // two K halves of 128 rows x 128 codes
  static constexpr int kBHalfBytes = kN * 128;          // one K half of the B rows
  static constexpr int kStageBytes = kABytes + 2 * kBHalfBytes;
  static constexpr size_t kXBytes = size_t(16) * 64 * 2;  // the up/gate epilogue's exchange buffer
  static constexpr size_t kTexpBytes = size_t(kTermUnitsMax) * MT * sizeof(float);  // the call's 2^-E
  static constexpr int kStagesFit =
      int((227 * 1024 - kXBytes - kTexpBytes - sizeof(BatchCtl) - 1024) / kStageBytes);
  static constexpr int kStages = kStagesFit < kBMaxStages ? kStagesFit : kBMaxStages;
  static constexpr int kTSlotsFit = (512 - 16) / kN;    // unit accumulators (N columns each)
  static constexpr int kTSlots = kTSlotsFit < 4 ? kTSlotsFit : 4;
  static constexpr uint32_t kColSum = uint32_t(kTSlots) * kN;  // the piece's sums: 16 columns
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kIdesc = umma_idesc_f8f6f4(kFmtE4M3, kFmtE4M3, kTileRows, kN);
  static constexpr size_t kOffX = size_t(kStages) * kStageBytes;
  static constexpr size_t kOffTexp = kOffX + kXBytes;
  static constexpr size_t kOffCtl = kOffTexp + kTexpBytes;
  static constexpr size_t kSmemBytes = kOffCtl + sizeof(BatchCtl) + 1024;
  static_assert(MT >= 4 && MT <= kTermTokens && kN % 16 == 0, "N of the MMA");
  static_assert(kStages >= 3 && kTSlots >= 2 && kColSum + 16 <= kTmemCols, "pipeline and TMEM");
  static_assert(kStageBytes % 1024 == 0 && kBHalfBytes % 1024 == 0, "1024-byte swizzle atoms");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// The term operand of a token batch, one CTA per padded token (gridDim.x = MT; tokens >= M get
// zero terms). RMS = true: the rows are bf16(RMSNorm(src[m]) * gamma) over K = H (the QKV and
// feed-forward inputs), bump = true also counts the call (the split-K words' epoch) and sets the
// tokens' batch_unscale to 1 (the term sums are at true scale); RMS = false: src[m] itself (the
// GeGLU activation, the attention rows). 256 threads; thread t holds 16-element groups t + 256 q,
// so a unit's 16 groups sit in one half-warp and its largest |h| is a half-warp reduction.
template <bool RMS>
__global__ void __launch_bounds__(256) batch_terms_kernel(const uint16_t* src, int K, const uint16_t* gamma,
                                                          Scratch sc, int M, bool bump) {
  __shared__ double red[8];
  const int m = blockIdx.x, mt = gridDim.x, tid = threadIdx.x, groups = K / 16;
  const bool live = m < M;
  uint4 raw[4] = {};
  if (RMS && tid < groups) load_group_gamma(gamma, tid, raw);
  pdl_wait_primary();
  pdl_launch_dependents();
  if (bump && m == 0 && tid == 0) sc.counters[kBatchEpoch] = __ldcg(sc.counters + kBatchEpoch) + 1u;
  if (RMS && tid == 0 && m < kBatchMax) sc.batch_unscale[m] = 1.0f;
  float inv = 0.f;
  if constexpr (RMS) {  // K = H: one group per thread
    if (live && tid < groups) load_group_cg(src + size_t(m) * K, tid, raw);
    const double ss = live && tid < groups ? sum_squares_bf16x16(raw[0], raw[1]) : 0.0;
    inv = rms_inverse(block_sum_d(ss, red), K);
  }
  for (int q = 0; q * 256 < groups; ++q) {  // the same count in every thread (whole half-warps)
    const int g = tid + 256 * q;
    const bool have = g < groups;
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.f;
    if (have && live) {
      if constexpr (RMS) {
        rms_apply16(raw, inv, v);
      } else {
        uint4 r[4];
        load_group_cg(src + size_t(m) * K, g, r);
        bf16x16_to_f32(r[0], r[1], v);
      }
    }
    uint32_t mx = 0u;  // |v| as bits (a NaN compares above every finite value)
#pragma unroll
    for (int j = 0; j < 16; ++j) mx = max(mx, __float_as_uint(v[j]) & 0x7fffffffu);
#pragma unroll
    for (int o = 8; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (have) {
      int e = 0;  // 2^e brings the unit's largest |v| into [128, 256)
      if (mx) {
        e = 7 - (int((mx >> 23) & 0xff) - 127);
        e = e > 120 ? 120 : (e < -120 ? -120 : e);
      }
      const float up = pow2f(e);
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] *= up;
      uint4 tm[kTerms];
      split_terms16<kTerms>(v, tm);
      const int u = g / 16;
      uint8_t* rows = sc.batch_terms + (size_t(u) * mt + m) * kTerms * 256 + (g % 16) * 16;
#pragma unroll
      for (int j = 0; j < kTerms; ++j) *reinterpret_cast<uint4*>(rows + j * 256) = tm[j];
      if (g % 16 == 0) sc.batch_texp[u * mt + m] = live ? pow2f(-e) : 0.f;
    }
  }
}

// Engine driver (the op interface of batch_run; the op's load_b is not used: `terms` maps the
// call's term rows, [units x MT x kTerms rows, 256 bytes], box {128 bytes, N rows}).
template <class TShape, class Op>
__device__ void batch_term_run(Op& op, const CUtensorMap* terms, uint8_t* smem_raw, const Scratch& sc) {
  constexpr int S = TShape::kStages, T = TShape::kTSlots, N = TShape::kN, MT = TShape::kMt;
  constexpr int UPT = Op::kUnitsPerTile;
  uint8_t* smem = align1024(smem_raw);
  BatchCtl& ctl = *reinterpret_cast<BatchCtl*>(smem + TShape::kOffCtl);
  auto stage = [&](int s) { return smem + size_t(s) * TShape::kStageBytes; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t total = int64_t(UPT) * Op::kTiles, grid = gridDim.x;
  const int u0 = int(int64_t(blockIdx.x) * total / grid);
  const int n = int(int64_t(blockIdx.x + 1) * total / grid) - u0;
  volatile uint32_t* abort = &ctl.abort;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&ctl.full_a[i], 1);
      mbar_init(&ctl.empty[i], 1);
    }
    for (int i = 0; i < T; ++i) {
      mbar_init(&ctl.done[i], 1);    // the unit's MMAs completed
      mbar_init(&ctl.tempty[i], 4);  // the epilogue warps read the unit's accumulator
    }
    mbar_init(&ctl.drain, 1);
    ctl.abort = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 1) tmem_alloc(&ctl.tmem_base, TShape::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ctl.tmem_base;
  const uint64_t policy = l2_evict_first_policy();
  const uint64_t policy_b = l2_evict_last_policy();  // every CTA reads the term rows
  const int prefetch = n < S ? n : S;
  auto load_terms = [&](uint8_t* st, int kc, uint64_t* bar) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
      tma_load_2d(st + TShape::kABytes + h * TShape::kBHalfBytes, terms, h * 128, kc * N, bar, policy_b);
  };
  // the first units' weights before the wait on the preceding kernel, their term rows after it
  if (tid < prefetch) {
    const int u = u0 + tid;
    mbar_arrive_expect_tx(&ctl.full_a[tid], uint32_t(TShape::kStageBytes));
    op.load_a(stage(tid), u / UPT, u % UPT, &ctl.full_a[tid], policy);
  }
  __syncwarp();
  pdl_wait_primary();
  pdl_launch_dependents();
  op.prologue();
  if (tid < prefetch) load_terms(stage(tid), (u0 + tid) % UPT, &ctl.full_a[tid]);
  if (tid == kTThreads - 1) op.prefetch_l2(u0 + prefetch, u0 + (prefetch + 6 < n ? prefetch + 6 : n));
  __syncwarp();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = prefetch;
      for (int i = prefetch; i < n; ++i) {
        const int s = i % S, r = i - S;
        if (!mbar_wait_or_abort(&ctl.empty[s], uint32_t((r / S) & 1), abort, sc.err)) break;
        const int u = u0 + i;
        mbar_arrive_expect_tx(&ctl.full_a[s], uint32_t(TShape::kStageBytes));
        op.load_a(stage(s), u / UPT, u % UPT, &ctl.full_a[s], policy);
        load_terms(stage(s), u % UPT, &ctl.full_a[s]);
        if ((i - prefetch) % 2 == 0 && i + 6 < n) op.prefetch_l2(u + 6, u0 + (i + 8 < n ? i + 8 : n));
        issued = i + 1;
      }
      // every requested copy has landed before the CTA may exit
      for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&ctl.full_a[i % S], uint32_t((i / S) & 1)))
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      for (int i = 0; i < n; ++i) {
        const int s = i % S, t = i % T;
        bool ok = i < T || mbar_wait_or_abort(&ctl.tempty[t], uint32_t(((i / T) - 1) & 1), abort, sc.err);
        ok = ok && mbar_wait_or_abort(&ctl.full_a[s], uint32_t((i / S) & 1), abort, sc.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(stage(s)), b0 = a0 + uint32_t(TShape::kABytes);
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // K = 32 each: K half j / 4, 32 bytes a step
          const uint32_t h = j / 4, kk = j % 4;
          umma_f8f6f4(tbase + uint32_t(t * N), umma_desc_sw128(a0 + h * uint32_t(kTileRows * 128) + kk * 32u),
                      umma_desc_sw128(b0 + h * uint32_t(TShape::kBHalfBytes) + kk * 32u), TShape::kIdesc,
                      uint32_t(j > 0));
        }
        umma_commit(&ctl.empty[s]);
        umma_commit(&ctl.done[t]);
      }
      umma_commit(&ctl.drain);  // nothing of ours may still be running when TMEM is released
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ctl.drain, 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = warp & 3, row = quarter * 32 + lane;
    const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
    const uint32_t tsum = tbase + lane_addr + TShape::kColSum;
    uint8_t* xbuf = smem + TShape::kOffX;
    // the call's 2^-E of every (unit, token) into shared memory once (written before this kernel's wait)
    float* texp = reinterpret_cast<float*>(smem + TShape::kOffTexp);
    for (int k = tid - 64; k < UPT * MT; k += 128) texp[k] = __ldcg(sc.batch_texp + k);
    named_bar(kBEpiBarrier, 128);
    bool ok = true;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    for (int i = 0; i < n; ++i) {
      const int u = u0 + i, tile = u / UPT, kc = u % UPT, t = i % T;
      if (ok) ok = mbar_wait_or_abort(&ctl.done[t], uint32_t((i / T) & 1), abort, sc.err);
      tc_fence_after();
      float d[N];  // the unit's N columns of this row: every load in flight, one wait
      if (ok) {
#pragma unroll
        for (int c = 0; c < N; c += 16)
          tmem_ld16(tbase + lane_addr + uint32_t(t * N + c), *reinterpret_cast<float(*)[16]>(d + c));
        tmem_ld_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl.tempty[t]);  // the accumulator is free for the next unit
      if (ok) {
#pragma unroll
        for (int m = 0; m < MT; ++m)  // each token's terms, smallest first, times its 2^-E
          acc[m] = fmaf(combine_terms<kTerms>(d + kTerms * m), texp[kc * MT + m], acc[m]);
      }
      if (!(kc == UPT - 1 || i == n - 1)) continue;
      // the piece's sums (16 TMEM columns of this row) for the op's epilogue
      uint32_t bits[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) bits[m] = __float_as_uint(m < MT ? acc[m] : 0.f);
      if (ok) {
        tmem_st16(tsum, bits);
        tmem_st_wait();
      }
      op.finish(ctl, xbuf, tile, row, tsum, ok);
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    }
  }

  // teardown: every MMA has completed (drain) and every TMEM access has been waited for
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TShape::kTmemCols);
  }
}

// The epoch-tagged words of one batched kernel: the call count kept by batch_norm_kernel (bumped
// once per QKV and once per feed-forward call) and the kernel kind, so that words left by another
// kernel or an earlier call never match.
enum BatchKind : uint32_t { kTagUpGate = 0, kTagDown = 1, kTagQkv = 2, kTagO = 3 };
__device__ __forceinline__ uint32_t batch_tag(const Scratch& sc, BatchKind kind) {
  return (__ldcg(sc.counters + kBatchEpoch) << 2) | uint32_t(kind);
}

// ---------------------------------------------------------------------------------------
// The ops

// h[m] = bf16(RMSNorm(residual[m]) * gamma_pre): one CTA per token, 240 threads x 16 elements,
// stored as f16 times 2^k, k per token so that max |h| 2^k lies in [2^14, 2^15): every element of
// at least max |h| 2^-31 is exact in f16, and the up/gate sums are multiplied back by 2^-k
// (batch_unscale) before their bf16 rounding. Thread 0 of CTA 0 also counts the call (the epoch
// of the split-K words and tile sums).
__global__ void __launch_bounds__(256) batch_norm_kernel(const uint16_t* residual, const uint16_t* pre_rms,
                                                             Scratch sc) {
  __shared__ double red[8];
  __shared__ float wmax[8];
  const int m = blockIdx.x, g = threadIdx.x;
  const bool have = g < kH / 16;
  uint4 raw[4];
  if (have) load_group_gamma(pre_rms, g, raw);
  pdl_wait_primary();
  pdl_launch_dependents();
  if (m == 0 && g == 0) sc.counters[kBatchEpoch] = __ldcg(sc.counters + kBatchEpoch) + 1u;
  if (have) load_group_cg(residual + size_t(m) * kH, g, raw);
  const double ss = have ? sum_squares_bf16x16(raw[0], raw[1]) : 0.0;
  const float inv = rms_inverse(block_sum_d(ss, red), kH);
  float v[16];
  float amax = 0.f;
  if (have) {
    rms_apply16(raw, inv, v);
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));  // NaN-free here: a NaN max is caught below
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (v[j] != v[j]) amax = __uint_as_float(0x7f800000u);
  }
  amax = warp_max(amax);
  if ((g & 31) == 0) wmax[g >> 5] = amax;
  __syncthreads();
  amax = wmax[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, wmax[w]);
  int k = amax > 0.f ? 14 - block_exponent(amax) : 0;
  k = k > 120 ? 120 : (k < -120 ? -120 : k);
  if (g == 0) sc.batch_unscale[m] = pow2f(-k);
  if (have) {
    const float up = pow2f(k);
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __half2 h = __floats2half2_rn(v[2 * j] * up, v[2 * j + 1] * up);
      w[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    uint4* dst = reinterpret_cast<uint4*>(sc.batch_h + size_t(m) * kH + 16 * g);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

struct BatchMaps {
  CUtensorMap a, a2, s, s2;  // weights: up (or down) codes, gate codes, their block scales
  CUtensorMap b;             // activation rows [M, K] (up/gate: f16, down: bf16), box {64, MPAD}
};

// The pieces of a projection onto the hidden size (the feed-forward's down, UPT = 60 units per
// tile; the attention output's O, UPT = 16) added per token, then the residual epilogue of the
// reference ops (FOG/src/ops.rs:130-146 and 201-239): y = bf16(bf16(sum) g) or bf16(sum s_row),
// residual = bf16(residual + bf16(y inv gamma)), times the layer scalar where there is one
// (bf16), with inv the RMS statistic of the token's y. One CTA per token; every tile's pieces are
// added in CTA order, so the result does not depend on timing.
constexpr int kMaxDownPieces = 6;  // CTAs one tile may span (checked at set-up)
constexpr int kFinThreads = 768;  // 5 rows of H per thread: every load of a row in flight at once
// The epilogue's operands: one of down_global (NVFP4: the reciprocal global scale), down_scale
// (FP8 feed-forward: f32 per-row scales) and o_scale (O: bf16 per-row scales).
struct FinalizeArgs {
  uint16_t* residual;
  const uint16_t* post_rms;
  const uint16_t* layer_scalar;  // null: none (O)
  const float* down_global;
  const float* down_scale;
  const uint16_t* o_scale;
};
template <int UPT, BatchKind KIND>
__global__ void __launch_bounds__(kFinThreads) batch_finalize_kernel(FinalizeArgs a, Scratch sc, int down_grid) {
  constexpr int kUpt = UPT, kTiles = kH / kTileRows;
  constexpr int kTotal = kUpt * kTiles;
  constexpr int kMaxGrid = 1024;
  constexpr int kRows = kH / kFinThreads;
  static_assert(kH % kFinThreads == 0, "rows per thread");
  __shared__ double red[kFinThreads / 32];
  __shared__ int first_cta[kTiles], last_cta[kTiles];
  __shared__ uint8_t run_tile[kMaxGrid];  // the tile of each down CTA's first unit
  const int m = blockIdx.x;
  for (int t = threadIdx.x; t < kTiles; t += blockDim.x) {
    first_cta[t] = cta_of_unit(int64_t(t) * kUpt, down_grid, kTotal);
    last_cta[t] = cta_of_unit(int64_t(t) * kUpt + kUpt - 1, down_grid, kTotal);
  }
  for (int c = threadIdx.x; c < down_grid && c < kMaxGrid; c += blockDim.x)
    run_tile[c] = uint8_t(int(int64_t(c) * kTotal / down_grid) / kUpt);
  // the epilogue's static operands, then the residual rows (written by earlier kernels), before
  // the wait on the down kernel
  float gamma[kRows];
#pragma unroll
  for (int q = 0; q < kRows; ++q) gamma[q] = bf16_to_f32(a.post_rms[threadIdx.x + q * kFinThreads]);
  __syncthreads();
  pdl_wait_primary();
  pdl_launch_dependents();
  uint16_t* res = a.residual + size_t(m) * kH;
  uint16_t rbits[kRows];
#pragma unroll
  for (int q = 0; q < kRows; ++q) rbits[q] = __ldcg(res + threadIdx.x + q * kFinThreads);
  const uint32_t tag = batch_tag(sc, KIND);
  const float g = a.down_global ? *a.down_global : 1.0f;
  unsigned long long w[kRows][kMaxDownPieces];
#pragma unroll
  for (int q = 0; q < kRows; ++q) {  // every piece of every row in flight at once
    const int e = threadIdx.x + q * kFinThreads, t = e / kTileRows, r = e % kTileRows;
    const int first = first_cta[t], last = last_cta[t];
#pragma unroll
    for (int k = 0; k < kMaxDownPieces; ++k) {
      w[q][k] = 0ull;
      const int c = first + k;
      if (c <= last) {
        const int piece = run_tile[c] < t ? 1 : 0;  // tile t is CTA c's second piece when its run began earlier
        w[q][k] = __ldcg(sc.batch_words + ((size_t(c) * 2 + piece) * kBatchMax + m) * kTileRows + r);
      }
    }
  }
  float y[kRows];
  double ss = 0.0;
#pragma unroll
  for (int q = 0; q < kRows; ++q) {
    const int e = threadIdx.x + q * kFinThreads, t = e / kTileRows;
    const int n = last_cta[t] - first_cta[t] + 1;
    float sum = 0.f;  // the pieces in CTA order
#pragma unroll
    for (int k = 0; k < kMaxDownPieces; ++k) {
      if (k >= n) break;
      if (uint32_t(w[q][k] >> 32) != tag) {
        atomicOr(sc.err, kErrInternal);
        sum = __uint_as_float(0x7fc00000u);
      }
      sum += __uint_as_float(uint32_t(w[q][k]));
    }
    y[q] = a.down_scale ? bf16_round(sum * __ldg(a.down_scale + e))
                        : (a.o_scale ? bf16_round(sum * bf16_to_f32(__ldg(a.o_scale + e)))
                                     : bf16_round(bf16_round(sum) * g));
    ss += double(y[q]) * double(y[q]);
  }
  const float inv = rms_inverse(block_sum_d(ss, red), kH);
  const float lam = a.layer_scalar ? bf16_to_f32(a.layer_scalar[0]) : 1.0f;
#pragma unroll
  for (int q = 0; q < kRows; ++q) {
    const float nrm = bf16_round((y[q] * inv) * gamma[q]);
    float r = bf16_round(bf16_to_f32(rbits[q]) + nrm);
    if (a.layer_scalar) r = bf16_round(r * lam);
    res[threadIdx.x + q * kFinThreads] = f32_to_bf16(r);
  }
}


template <class... KArgs, class... Args>
cudaError_t launch_batch(void (*kernel)(KArgs...), dim3 grid, int threads, size_t smem, bool pdl, cudaStream_t stream,
                         Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace
}  // namespace g4
