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

#include <type_traits>
#include <utility>

#include "g4_gemv.cuh"
#include "g4_ops.cuh"

namespace g4 {
namespace {

// Pipeline shapes of one tensor-parallel rank (NTP ranks; 1 = the whole layer): <nvfp4, stages,
// K units per tile, tiles, B slots>. Units per tile = K / 256; B slots >= the largest number of
// distinct K units one CTA's run touches on a 148-SM grid (launchers grow the grid if a smaller
// GPU would need more).
template <int NTP>
struct Shapes {
  using Geo = TpGeo<NTP>;
  static constexpr int kOUnits = Geo::kQRows / kUnitK;
  static constexpr int kDownUnits = Geo::kDownK / kUnitK;
  using Qkv = GemvShape<false, 6, kH / kUnitK, (Geo::kQRows + 2 * Geo::kKvRows) / kTileRows, 8>;
  using O = GemvShape<false, 6, kOUnits, kH / kTileRows, (kOUnits < 4 ? kOUnits : 4)>;
  using UpGate = GemvShape<true, 10, kH / kUnitK, Geo::kFfnRows / 64, 15>;  // tile = 64 up rows + 64 gate rows
  using Down = GemvShape<true, 10, kDownUnits, kH / kTileRows, (kDownUnits < 13 ? kDownUnits : 13)>;
  // FP8 feed-forward: up/gate tiles of 64 up + 64 gate rows (K = H), down like O with K = L
  using UpGate8 = GemvShape<false, 6, kH / kUnitK, Geo::kFfnRows / 64, 15>;
  using Down8 = GemvShape<false, 5, kDownUnits, kH / kTileRows, (kDownUnits < 13 ? kDownUnits : 13)>;
};

// The global layers' projections (one GPU): q (16 heads x 512) and the single k head, then O with
// K = Qf = 8192.
using FullQkvShape = GemvShape<false, 6, kH / kUnitK, (kQf + kDf) / kTileRows, 8>;
using FullOShape = GemvShape<false, 6, kQf / kUnitK, kH / kTileRows, 8>;

// Unit-tiled weights (g4_pack_tiles): pipeline unit u of a matrix is one contiguous block,
// fetched by one TMA box: fp8, kUnitBox rows of 128 codes (both 128-element halves of its 128
// rows); nvfp4, 128 rows of 128 bytes (64 up + 64 gate rows, or 128 down rows, each the unit's
// 256 packed codes), its block scales one 2 KB block of the same 128 rows x 16 bytes.
constexpr int kUnitBox = 2 * kTileRows;


// ---------------------------------------------------------------------------------------
// Tensor parallelism: the one-shot all-reduce of a finished tile's partial rows (O and down).
// Called by the 128 epilogue threads of the CTA that finishes the tile; thread `row` stores its
// word (tag, value) into every peer's exchange buffer with one 64-bit system-scope store,
// waits (bounded) until every peer's word of this call is in its own buffer and adds the
// world's partials in rank order: every rank computes the same sum, bit for bit.
__device__ float tp_allreduce(const TpLink& tp, int op, int tile, int row, float v, uint32_t* err) {
  if (tp.world <= 1) return v;
  uint32_t* ep = tp.epoch + op * kTpTiles + tile;
  const uint32_t e = __ldcg(ep) + 1u;
  named_bar(kEpiBarrier, kEpiThreads);  // every thread has read the count before it moves on
  if (row == 0) *ep = e;
  const size_t base = ((size_t(op) * 2 + (e & 1u)) * kTpTiles + tile) * kMaxTp;
  const uint32_t tag = tp_tag(tp.generation, e);
  const unsigned long long word = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
#pragma unroll
  for (int s = 0; s < kMaxTp; ++s)
    if (s < tp.world && s != tp.rank) st_relaxed_sys_u64(tp.slots[s] + (base + tp.rank) * kTileRows + row, word);
  const unsigned long long* mine = tp.slots[tp.rank] + base * kTileRows + row;
  float pv[kMaxTp];
  uint32_t pending = 0u;
#pragma unroll
  for (int s = 0; s < kMaxTp; ++s) {
    pv[s] = s == tp.rank ? v : 0.f;
    if (s < tp.world && s != tp.rank) pending |= 1u << s;
  }
  const uint64_t t0 = globaltimer_ns();
  while (pending) {
    unsigned long long w[kMaxTp];  // every pending word in flight at once, then the checks
#pragma unroll
    for (int s = 0; s < kMaxTp; ++s)
      if (pending & (1u << s)) w[s] = ld_relaxed_sys_u64(mine + s * kTileRows);
#pragma unroll
    for (int s = 0; s < kMaxTp; ++s) {
      if ((pending & (1u << s)) && uint32_t(w[s] >> 32) == tag) {
        pv[s] = __uint_as_float(uint32_t(w[s]));
        pending &= ~(1u << s);
      }
    }
    if (pending && globaltimer_ns() - t0 > tp.wait_ns) {  // a peer never arrived: flag it, poison the row
      atomicOr(err, kErrPeerTimeout);
#pragma unroll
      for (int s = 0; s < kMaxTp; ++s)
        if (pending & (1u << s)) pv[s] = __uint_as_float(0x7fc00000u);
      break;
    }
  }
  float sum = 0.f;
#pragma unroll
  for (int s = 0; s < kMaxTp; ++s)
    if (s < tp.world) sum += pv[s];
  return sum;
}

// ---------------------------------------------------------------------------------------
// Post-RMSNorm + residual (O and FFN down): residual <- bf16(residual + RMSNorm_gamma(y)) [then
// bf16(. * layer_scalar)] over the H outputs. The statistic needs every output, so each CTA that
// finishes a tile keeps its 128 values of y in shared memory and publishes their sum of squares
// as two 64-bit words tagged with the call's epoch (epoch << 32 | half of the f64): a reader that
// sees this call's epoch in both words has the sum, with no flag or fence. Only those CTAs (at
// most one per tile) wait: they poll the 30 tiles' words, add the sums in a fixed order and update
// their own rows. Every other CTA leaves at once, so the next kernel's CTAs can take its SM and
// start their weight copies during the tail. The finishing CTAs are all resident (each is running
// when it publishes); the wait is bounded.
//
// The epoch is the number of calls so far. Each tile keeps its own count (in `epochs`), written
// only by the CTA that finishes the tile; every CTA reads the count of the first tile of its own
// run after the dependency wait, before it publishes anything, so that tile cannot have been
// finished yet in this call and every tile's count is the same.

constexpr int kMaxFinTiles = 4;  // tiles one CTA can finish (checked at set-up: check_geometry)

struct ResidualTail {
  float y[kMaxFinTiles][kTileRows];                     // the finished tiles' outputs (bf16 values)
  __align__(16) uint16_t gamma[kMaxFinTiles][kTileRows];  // their post-RMSNorm weights
  __align__(16) uint16_t res[kMaxFinTiles][kTileRows];    // and residual rows (copied asynchronously)
  int tile[kMaxFinTiles];
  int n;
  double red[4];
  double ss[kTileSsCount];
};

// The tile of this CTA's first unit (the engine's contiguous split of Shape's units).
template <class Shape>
__device__ __forceinline__ int first_tile() {
  return int(int64_t(blockIdx.x) * Shape::kTotalUnits / gridDim.x) / Shape::kUnitsPerTile;
}

// The epoch of this call for a CTA whose run starts in `first_tile` (all threads may call it).
__device__ __forceinline__ uint32_t tail_epoch(const uint32_t* epochs, int first_tile) {
  return __ldcg(epochs + first_tile) + 1u;
}

// Called by the 128 epilogue threads when a tile is final: record it and publish its sum of
// squares (f64, rows in order over the four warps) with the call's epoch.
__device__ void tail_record(ResidualTail& t, const uint16_t* gamma, const uint16_t* residual, unsigned long long* sums,
                            uint32_t* epochs, uint32_t epoch, int tile, int row, float y) {
  const int f = t.n;
  t.y[f][row] = y;
  if (row < 16) {  // 16 x 16 bytes each, in flight while the kernel goes on
    cp_async_16(&t.gamma[f][row * 8], gamma + tile * kTileRows + row * 8);
    cp_async_16(&t.res[f][row * 8], residual + tile * kTileRows + row * 8);
  }
  double ss = warp_sum_d(double(y) * double(y));
  if ((threadIdx.x & 31) == 0) t.red[row / 32] = ss;
  named_bar(kEpiBarrier, kEpiThreads);
  if (row == 0) {
    const double sum = ((t.red[0] + t.red[1]) + t.red[2]) + t.red[3];
    const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(sum));
    const unsigned long long tag = static_cast<unsigned long long>(epoch) << 32;
    st_relaxed_gpu_u64(sums + 2 * tile, tag | (bits & 0xffffffffull));
    st_relaxed_gpu_u64(sums + 2 * tile + 1, tag | (bits >> 32));
    epochs[tile] = epoch;
    t.tile[f] = tile;
    t.n = f + 1;
  }
  named_bar(kEpiBarrier, kEpiThreads);
}

// Whole CTA, after gemv_run: a CTA that finished tiles waits for every tile's sum of this call,
// then updates its recorded rows; the others return.
__device__ void tail_update(ResidualTail& t, uint16_t* residual, const Scratch& sc, const unsigned long long* sums,
                            uint32_t epoch, int tiles, const uint16_t* layer_scalar) {
  const float lam = layer_scalar ? bf16_to_f32(layer_scalar[0]) : 1.0f;
  cp_async_wait_all();
  __syncthreads();  // t.n is final
  if (t.n == 0) return;  // CTA-uniform: nothing of this CTA's waits on the statistic
  if (threadIdx.x < tiles) {  // thread i polls tile i's two words
    const unsigned long long* w = sums + 2 * threadIdx.x;
    unsigned long long lo = ld_relaxed_gpu_u64(w), hi = ld_relaxed_gpu_u64(w + 1);  // both in flight
    const uint64_t t0 = globaltimer_ns();
    while (uint32_t(lo >> 32) != epoch || uint32_t(hi >> 32) != epoch) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(sc.err, kErrWaitTimeout);
        break;
      }
      lo = ld_relaxed_gpu_u64(w);
      hi = ld_relaxed_gpu_u64(w + 1);
    }
    t.ss[threadIdx.x] = __longlong_as_double(static_cast<long long>((hi << 32) | (lo & 0xffffffffull)));
  }
  __syncthreads();
  G4_STAMP(sc, 12);
  double sum = 0.0;
  for (int i = 0; i < tiles; ++i) sum += t.ss[i];  // fixed order: identical in every CTA
  const float inv = rms_inverse(sum, kH);
  const int e = threadIdx.x - 64;  // the epilogue threads own the recorded rows
  if (e >= 0 && e < kEpiThreads) {
    for (int f = 0; f < t.n; ++f) {
      const float nrm = bf16_round((t.y[f][e] * inv) * bf16_to_f32(t.gamma[f][e]));
      float r = bf16_round(bf16_to_f32(t.res[f][e]) + nrm);
      if (layer_scalar) r = bf16_round(r * lam);
      t.res[f][e] = f32_to_bf16(r);  // in place, then whole 16-byte stores (the next kernel reads
    }                                // sectors written in 2-byte pieces slowly)
  }
  __syncthreads();
  if (threadIdx.x < 16 * t.n) {
    const int f = threadIdx.x / 16, q = threadIdx.x % 16;
    reinterpret_cast<uint4*>(residual + t.tile[f] * kTileRows)[q] = reinterpret_cast<const uint4*>(t.res[f])[q];
  }
  G4_STAMP(sc, 13);
}

// ---------------------------------------------------------------------------------------
// QKV

// Per-head RMSNorm (+ RoPE for q and k) and the store of one head (q_out, or the addressed ring
// slot of the K / V cache). A head is 256 projected rows = two tiles. The CTA holding the head's
// first unit finishes it at its last piece in the head; every other CTA that computes a piece of
// either tile publishes its partial row sums as epoch-tagged words, which the finishing CTA polls
// and adds in CTA order. Its 128 epilogue threads finish the head: thread e owns head elements e
// and e + 128, which are exactly the two elements RoPE's half swap pairs.

struct QkvStatic {  // per CTA, loaded while the weights stream in
  __align__(16) uint16_t cos[kDs];
  __align__(16) uint16_t sin[kDs];
  __align__(16) uint16_t qg[kDs];
  __align__(16) uint16_t kg[kDs];
  __align__(16) uint16_t out[kDs];
  double red[4];
  int slot, row;
  bool kv_ok, rope_ok;
};

struct QkvMaps {
  CUtensorMap q, k, v;
};

template <int NTP>
struct QkvOp {
  using QkvShape = typename Shapes<NTP>::Qkv;
  using Geo = TpGeo<NTP>;
  static constexpr int kQRows = Geo::kQRows, kKvRows = Geo::kKvRows;
  static constexpr int kQHeads = kQRows / kDs, kKvHeads = Geo::kKvHeads;
  const QkvMaps* maps;
  QkvArgs a;
  Scratch sc;
  uint32_t tx_bytes = QkvShape::kABytes;
  static constexpr bool kRms = true;
  static constexpr int kRmsGroups = kH / 16;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    constexpr int kQTiles = kQRows / kTileRows, kKTiles = kKvRows / kTileRows;
    const CUtensorMap* m = tile < kQTiles ? &maps->q : (tile < kQTiles + kKTiles ? &maps->k : &maps->v);
    const int t = tile < kQTiles ? tile : (tile < kQTiles + kKTiles ? tile - kQTiles : tile - kQTiles - kKTiles);
    if (a.tiled) {
      tma_load_2d(stage, m, 0, (t * QkvShape::kUnitsPerTile + kc) * kUnitBox, bar, policy);
    } else {  // row-major: (x = K offset, y = first row) per 128-element half
      tma_load_2d(stage, m, kc * kUnitK, t * kTileRows, bar, policy);
      tma_load_2d(stage + 16384, m, kc * kUnitK + 128, t * kTileRows, bar, policy);
    }
  }
  // units [u0, u1) of the fused q|k|v order into L2 (unit-tiled weights only)
  __device__ void prefetch_l2(int u0, int u1) const {
    if (!a.tiled) return;
    constexpr int kQU = kQRows / kTileRows * QkvShape::kUnitsPerTile;
    constexpr int kKU = kKvRows / kTileRows * QkvShape::kUnitsPerTile;
    constexpr uint32_t kB = QkvShape::kABytes;
    prefetch_units(a.q_weight, u0, u1 < kQU ? u1 : kQU, kB);
    prefetch_units(a.k_weight, (u0 > kQU ? u0 : kQU) - kQU, (u1 < kQU + kKU ? u1 : kQU + kKU) - kQU, kB);
    prefetch_units(a.v_weight, (u0 > kQU + kKU ? u0 : kQU + kKU) - kQU - kKU, u1 - kQU - kKU, kB);
  }
  static constexpr bool kOwnPieces = true;
  QkvStatic* st;
  uint32_t epoch = 0;  // this call's, for the heads' split-K words

  // the position offsets (device-resident, written before the call; byte offsets into the whole
  // layer's cache and table, the same on every tensor-parallel rank), then the RoPE row and the
  // per-head norm weights into shared memory, asynchronously (the epilogue threads wait for them)
  __device__ void prologue(GemvCtl&) {
    epoch = tail_epoch(sc.counters + kHeadEpochBase, first_tile<QkvShape>() / 2);
    const int kv = *a.kv_offset, rope = *a.rope_offset;
    const bool kv_ok = kv >= 0 && (kv % (kPs * 2)) == 0 && kv / (kPs * 2) < a.ring_len;
    const bool rope_ok = rope >= 0 && (rope % (kDs * 2)) == 0 && rope / (kDs * 2) < a.rope_rows;
    const int e = threadIdx.x - 64;
    if (e == 0) {
      st->kv_ok = kv_ok;
      st->rope_ok = rope_ok;
      st->slot = kv / (kPs * 2);
      st->row = rope / (kDs * 2);
    }
    if (e >= 0 && e < 32) {  // 32 x 16 bytes per 256-element row
      const int q = e;
      if (rope_ok) {
        const size_t row = size_t(rope / (kDs * 2)) * kDs;
        cp_async_16(st->cos + q * 8, a.cos + row + q * 8);
        cp_async_16(st->sin + q * 8, a.sin + row + q * 8);
      }
      cp_async_16(st->qg + q * 8, a.q_rms + q * 8);
      cp_async_16(st->kg + q * 8, a.k_rms + q * 8);
    }
  }

  // A head's pieces: the CTA holding the head's first unit finishes the head at its last piece
  // in the head (the last piece of its run); every other piece is published as epoch-tagged
  // words in the slots of its tile.
  __device__ void finish_piece(int tile, int row, float v, int, GemvCtl&) const {
    constexpr int UPT = QkvShape::kUnitsPerTile;
    const int64_t grid = gridDim.x, total = QkvShape::kTotalUnits;
    const int head = tile / 2;
    const int run_last = int(int64_t(blockIdx.x + 1) * total / grid) - 1;  // this CTA's last unit
    const int final_tile = run_last / UPT < 2 * head + 1 ? run_last / UPT : 2 * head + 1;
    if (int(blockIdx.x) == cta_of_unit(int64_t(2 * head) * UPT, grid, total) && tile == final_tile) {
      finish_head(head, row, tile, v);
      return;
    }
    const int first = cta_of_unit(int64_t(tile) * UPT, grid, total);
    st_relaxed_gpu_u64(words(tile) + (blockIdx.x - first) * kTileRows + row,
                       (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v));
  }

  __device__ unsigned long long* words(int tile) const {
    return reinterpret_cast<unsigned long long*>(sc.partials) + kSplitWordsQkv + size_t(tile) * kMaxCtasPerGroup * kTileRows;
  }

  // Thread e finishes elements e and e + 128 of the head: tile 2 head + t, row e. `own` is this
  // CTA's piece of tile `own_tile` (not published).
  __device__ void finish_head(int head, int e, int own_tile, float own) const {
    constexpr int UPT = QkvShape::kUnitsPerTile;
    const int64_t grid = gridDim.x, total = QkvShape::kTotalUnits;
    float y[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {  // element e + 128 t of the head = row e of tile 2 head + t
      const int tile = 2 * head + t;
      const int first = cta_of_unit(int64_t(tile) * UPT, grid, total);
      const int span = cta_of_unit(int64_t(tile) * UPT + UPT - 1, grid, total) - first + 1;
      const int r = tile * kTileRows + e;
      const uint16_t sb =
          r < kQRows ? a.q_scale[r] : (r < kQRows + kKvRows ? a.k_scale[r - kQRows] : a.v_scale[r - kQRows - kKvRows]);
      float acc = __uint_as_float(0x7fc00000u);
      if (span <= kMaxCtasPerGroup)
        acc = sum_tagged(words(tile) + e, span, tile == own_tile ? int(blockIdx.x) - first : -1, own, epoch, sc.err);
      else if (e == 0)
        atomicOr(sc.err, kErrInternal);
      // scaled_projection: bf16((x @ codes.T) * scale) (generate_references.py:265-274)
      y[t] = bf16_round(acc * bf16_to_f32(sb));
    }
    if (e == 0) sc.counters[kHeadEpochBase + head] = epoch;
    // RMSNorm over the head's 256 values (gemma4.py:83-89), the sum in a fixed order
    double ss = warp_sum_d(double(y[0]) * double(y[0]) + double(y[1]) * double(y[1]));
    cp_async_wait_all();
    if ((threadIdx.x & 31) == 0) st->red[e / 32] = ss;
    named_bar(kEpiBarrier, kEpiThreads);
    const float inv = rms_inverse(((st->red[0] + st->red[1]) + st->red[2]) + st->red[3], kDs);
    const bool is_q = head < kQHeads, is_k = !is_q && head < kQHeads + kKvHeads;
    if (!st->kv_ok || !st->rope_ok) {
      if (e == 0) atomicOr(sc.err, (st->kv_ok ? 0u : kErrKvOffset) | (st->rope_ok ? 0u : kErrRopeOffset));
      named_bar(kEpiBarrier, kEpiThreads);
      return;
    }
    const uint16_t* gamma = is_q ? st->qg : (is_k ? st->kg : nullptr);
    float nrm[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float sv = y[t] * inv;
      nrm[t] = gamma ? bf16_round(sv * bf16_to_f32(gamma[e + 128 * t])) : bf16_round(sv);
    }
    if (is_q || is_k) {
      // RoPE, half-swap form with the low half of `sin` pre-negated by the caller:
      // out[i] = bf16(bf16(n[i] cos[i]) + bf16(n[i ^ 128] sin'[i]))
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int i = e + 128 * t;
        const float c = bf16_round(nrm[t] * bf16_to_f32(st->cos[i]));
        const float sn = bf16_round(nrm[1 - t] * bf16_to_f32(st->sin[i]));
        st->out[i] = f32_to_bf16(c + sn);
      }
    } else {
      st->out[e] = f32_to_bf16(nrm[0]);
      st->out[e + 128] = f32_to_bf16(nrm[1]);
    }
    named_bar(kEpiBarrier, kEpiThreads);
    if (e < 32) {  // 16-byte stores
      uint16_t* dst;
      if (is_q)
        dst = a.q_out + head * kDs;
      else if (is_k)
        dst = a.k_cache + size_t(st->slot) * kKvRows + (head - kQHeads) * kDs;
      else
        dst = a.v_cache + size_t(st->slot) * kKvRows + (head - kQHeads - kKvHeads) * kDs;
      reinterpret_cast<uint4*>(dst)[e] = reinterpret_cast<const uint4*>(st->out)[e];
    }
    named_bar(kEpiBarrier, kEpiThreads);
  }

  __device__ void load_static(int g, uint4 (&raw)[4]) const { load_group_gamma(a.input_rms, g, raw); }
  __device__ void load_group(int g, uint4 (&raw)[4]) const { load_group_cg(a.x, g, raw); }
  __device__ void finish_group(const uint4 (&raw)[4], float inv, float (&v)[16]) const { rms_apply16(raw, inv, v); }
};

template <int NTP>
__global__ void __launch_bounds__(kGemvThreads, 1) qkv_kernel(const __grid_constant__ QkvMaps maps, QkvArgs a,
                                                              Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ QkvStatic st;
  QkvOp<NTP> op{&maps, a, sc};
  op.st = &st;
  gemv_run<typename Shapes<NTP>::Qkv>(op, smem, sc);
  cp_async_wait_all();  // a CTA that finished no head still has the prologue's copies in flight
}

// ---------------------------------------------------------------------------------------
// O projection + post-attention RMSNorm + residual

template <int NTP>
struct OOp {
  using OShape = typename Shapes<NTP>::O;
  const CUtensorMap* map;
  OArgs a;
  Scratch sc;
  uint32_t tx_bytes = OShape::kABytes;
  static constexpr bool kOwnPieces = false;
  static constexpr bool kRms = false;
  static constexpr int kRmsGroups = 0;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {
      tma_load_2d(stage, map, 0, (tile * OShape::kUnitsPerTile + kc) * kUnitBox, bar, policy);
    } else {
      tma_load_2d(stage, map, kc * kUnitK, tile * kTileRows, bar, policy);
      tma_load_2d(stage + 16384, map, kc * kUnitK + 128, tile * kTileRows, bar, policy);
    }
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (a.tiled) prefetch_units(a.o_weight, u0, u1, OShape::kABytes);
  }
  __device__ void prologue(GemvCtl&) { epoch = tail_epoch(sc.counters + kTailEpochO, first_tile<OShape>()); }
  __device__ void load_static(int, uint4 (&)[4]) const {}
  __device__ void load_group(int g, uint4 (&raw)[4]) const { load_group_cg(a.x, g, raw); }
  __device__ void finish_group(const uint4 (&raw)[4], float, float (&v)[16]) const {
    bf16x16_to_f32(raw[0], raw[1], v);
  }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl&) const {
    const int r = tile * kTileRows + row;
    const float sum = tp_allreduce(*tp, 0, tile, row, v, sc.err);  // the K slices of every rank
    tail_record(*tail, a.post_rms, a.residual, sc.tile_ss + kTileSsO, sc.counters + kTailEpochO, epoch, tile, row,
                bf16_round(sum * bf16_to_f32(a.o_scale[r])));
  }
  ResidualTail* tail;
  const TpLink* tp;
  uint32_t epoch = 0;  // this call's, for split tiles and the residual tail
  unsigned long long* split_words = reinterpret_cast<unsigned long long*>(sc.partials) + kSplitWordsO;
  uint32_t* split_epochs = sc.counters + kTailEpochO;
};

template <int NTP>
__global__ void __launch_bounds__(kGemvThreads, 1) o_kernel(const __grid_constant__ CUtensorMap map, OArgs a,
                                                            Scratch sc, const __grid_constant__ TpLink tp) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ ResidualTail tail;
  if (threadIdx.x == 0) tail.n = 0;  // ordered by the engine's first barrier
  OOp<NTP> op{&map, a, sc};
  op.tail = &tail;
  op.tp = &tp;
  gemv_run<typename Shapes<NTP>::O>(op, smem, sc);
  tail_update(tail, a.residual, sc, sc.tile_ss + kTileSsO, op.epoch, kH / kTileRows, nullptr);
  G4_STAMP(sc, 8);
}

// ---------------------------------------------------------------------------------------
// NVFP4 feed-forward: up/gate + GeGLU, then down + post-RMSNorm + residual + layer scalar

struct UpGateMaps {
  CUtensorMap up, gate, up_s, gate_s;
};

template <int NTP>
struct UpGateOp {
  using UpGateShape = typename Shapes<NTP>::UpGate;
  const UpGateMaps* maps;
  FfnArgs a;
  Scratch sc;
  float g_up = 0.f, g_gate = 0.f;
  uint32_t tx_bytes = UpGateShape::kABytes + UpGateShape::kScaleBytes;  // packed codes + block scales
  static constexpr bool kOwnPieces = false;
  static constexpr bool kRms = true;
  static constexpr int kRmsGroups = kH / 16;

  // stage: [64 up rows | 64 gate rows] x 128 bytes (the unit's 256 packed e2m1 codes per row)
  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {  // up and gate rows interleaved in one buffer: one box per unit
      tma_load_2d(stage, &maps->up, 0, (tile * UpGateShape::kUnitsPerTile + kc) * kTileRows, bar, policy);
    } else {
      tma_load_2d(stage, &maps->up, kc * 128, tile * 64, bar, policy);
      tma_load_2d(stage + 8192, &maps->gate, kc * 128, tile * 64, bar, policy);
    }
  }
  // block scales [64 up rows | 64 gate rows] x 16 bytes: unit-tiled - one 2 KB block, one bulk
  // copy; row-major - two boxes
  __device__ void load_scales(uint8_t* dst, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {
      bulk_g2s(dst, a.up_scale + size_t(tile * UpGateShape::kUnitsPerTile + kc) * UpGateShape::kScaleBytes,
               UpGateShape::kScaleBytes, bar, policy);
    } else {
      tma_load_2d(dst, &maps->up_s, kc * 16, tile * 64, bar, policy);
      tma_load_2d(dst + 1024, &maps->gate_s, kc * 16, tile * 64, bar, policy);
    }
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (!a.tiled) return;
    prefetch_units(a.up_packed, u0, u1, UpGateShape::kABytes);
    prefetch_units(a.up_scale, u0, u1, UpGateShape::kScaleBytes);
  }
  __device__ void prologue(GemvCtl&) {
    g_up = *a.up_global;
    g_gate = *a.gate_global;
    epoch = tail_epoch(split_epochs, first_tile<UpGateShape>());
  }
  uint32_t epoch = 0;  // this call's, for split tiles
  unsigned long long* split_words = reinterpret_cast<unsigned long long*>(sc.partials) + kSplitWordsUpGate;
  uint32_t* split_epochs = sc.counters + kSplitEpochUpGate;
  __device__ void load_static(int g, uint4 (&raw)[4]) const { load_group_gamma(a.pre_rms, g, raw); }
  __device__ void load_group(int g, uint4 (&raw)[4]) const { load_group_cg(a.residual, g, raw); }
  __device__ void finish_group(const uint4 (&raw)[4], float inv, float (&v)[16]) const { rms_apply16(raw, inv, v); }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl& ctl) const {
    // GloballyScaled(nn.Linear): bf16(bf16(x @ W.T) * g)  (generate_references.py:358-372)
    const float val = bf16_round(bf16_round(v) * (row < 64 ? g_up : g_gate));
    if (row >= 64) ctl.xchg[row - 64] = val;
    named_bar(kEpiBarrier, kEpiThreads);
    // down_proj input: bf16(bf16(gelu_tanh(gate)) * up)  (gemma4.py:197). Whole 16-byte
    // stores: a sector written in 2-byte pieces is slow for the next kernel to read.
    if (row < 64) ctl.out16[row] = f32_to_bf16(bf16_round(gelu_tanh(ctl.xchg[row])) * val);
    named_bar(kEpiBarrier, kEpiThreads);
    if (row < 8) reinterpret_cast<uint4*>(sc.act + tile * 64)[row] = reinterpret_cast<const uint4*>(ctl.out16)[row];
  }
};

template <int NTP>
__global__ void __launch_bounds__(kGemvThreads, 1) ffn_upgate_kernel(const __grid_constant__ UpGateMaps maps, FfnArgs a,
                                                                     Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  UpGateOp<NTP> op{&maps, a, sc};
  gemv_run<typename Shapes<NTP>::UpGate>(op, smem, sc);
  G4_STAMP(sc, 8);
}

struct DownMaps {
  CUtensorMap w, s;
};

template <int NTP>
struct DownOp {
  using DownShape = typename Shapes<NTP>::Down;
  const DownMaps* maps;
  FfnArgs a;
  Scratch sc;
  float g_down = 0.f;
  uint32_t tx_bytes = DownShape::kABytes + DownShape::kScaleBytes;
  static constexpr bool kOwnPieces = false;
  static constexpr bool kRms = false;
  static constexpr int kRmsGroups = 0;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {
      tma_load_2d(stage, &maps->w, 0, (tile * DownShape::kUnitsPerTile + kc) * kTileRows, bar, policy);
    } else {
      tma_load_2d(stage, &maps->w, kc * 128, tile * kTileRows, bar, policy);
    }
  }
  __device__ void load_scales(uint8_t* dst, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {
      bulk_g2s(dst, a.down_scale + size_t(tile * DownShape::kUnitsPerTile + kc) * DownShape::kScaleBytes,
               DownShape::kScaleBytes, bar, policy);
    } else {
      tma_load_2d(dst, &maps->s, kc * 16, tile * kTileRows, bar, policy);
    }
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (!a.tiled) return;
    prefetch_units(a.down_packed, u0, u1, DownShape::kABytes);
    prefetch_units(a.down_scale, u0, u1, DownShape::kScaleBytes);
  }
  __device__ void prologue(GemvCtl&) {
    g_down = *a.down_global;
    epoch = tail_epoch(sc.counters + kTailEpochDown, first_tile<DownShape>());
  }
  __device__ void load_static(int, uint4 (&)[4]) const {}
  __device__ void load_group(int g, uint4 (&raw)[4]) const { load_group_cg(sc.act, g, raw); }
  __device__ void finish_group(const uint4 (&raw)[4], float, float (&v)[16]) const {
    bf16x16_to_f32(raw[0], raw[1], v);
  }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl&) const {
    const float sum = tp_allreduce(*tp, 1, tile, row, v, sc.err);  // the K slices of every rank
    // GloballyScaled(nn.Linear): bf16(bf16(x @ W.T) * g)  (generate_references.py:358-413)
    tail_record(*tail, a.post_rms, a.residual, sc.tile_ss + kTileSsDown, sc.counters + kTailEpochDown, epoch, tile, row,
                bf16_round(bf16_round(sum) * g_down));
  }
  ResidualTail* tail;
  const TpLink* tp;
  uint32_t epoch = 0;  // this call's, for split tiles and the residual tail
  unsigned long long* split_words = reinterpret_cast<unsigned long long*>(sc.partials) + kSplitWordsDown;
  uint32_t* split_epochs = sc.counters + kTailEpochDown;
};

template <int NTP>
__global__ void __launch_bounds__(kGemvThreads, 1) ffn_down_kernel(const __grid_constant__ DownMaps maps, FfnArgs a,
                                                                   Scratch sc, const __grid_constant__ TpLink tp) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ ResidualTail tail;
  if (threadIdx.x == 0) tail.n = 0;  // ordered by the engine's first barrier
  DownOp<NTP> op{&maps, a, sc};
  op.tail = &tail;
  op.tp = &tp;
  gemv_run<typename Shapes<NTP>::Down>(op, smem, sc);
  tail_update(tail, a.residual, sc, sc.tile_ss + kTileSsDown, op.epoch, kH / kTileRows, a.layer_scalar);
  G4_STAMP(sc, 8);
}

// ---------------------------------------------------------------------------------------
// Global layer QKV (FOG/src/ops.rs:78-116): the q heads and the single K = V head are 512 rows =
// four tiles each. As in the sliding QKV, the CTA holding a head's first unit finishes the head at
// its last piece in it, adding the other CTAs' epoch-tagged partial rows in CTA order; thread e of
// its 128 epilogue threads owns head elements e + 128 t (t < 4), so the RoPE pairs (i, i ^ 256)
// are both its own (t and t ^ 2). The k head also yields v: the same raw projection normalised
// without a gamma (K = V, FOG/src/device/full/rmsnorm.rs:182-200).

struct FullQkvStatic {
  __align__(16) uint16_t cos[kDf];
  __align__(16) uint16_t sin[kDf];
  __align__(16) uint16_t qg[kDf];
  __align__(16) uint16_t kg[kDf];
  __align__(16) uint16_t out[kDf];
  __align__(16) uint16_t out_v[kDf];
  double red[4];
  int slot, row;
  bool kv_ok, rope_ok;
};

struct FullQkvMaps {
  CUtensorMap q, k;
};

struct FullQkvOp {
  using Shape = FullQkvShape;
  static constexpr int kQTiles = kQf / kTileRows;  // 64; tiles 64..67 are the k head
  static constexpr int kTilesPerHead = kDf / kTileRows;
  const FullQkvMaps* maps;
  FullQkvArgs a;
  Scratch sc;
  uint32_t tx_bytes = Shape::kABytes;
  static constexpr bool kRms = true;
  static constexpr int kRmsGroups = kH / 16;
  static constexpr bool kOwnPieces = true;
  FullQkvStatic* st;
  uint32_t epoch = 0;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    const CUtensorMap* m = tile < kQTiles ? &maps->q : &maps->k;
    const int t = tile < kQTiles ? tile : tile - kQTiles;
    if (a.tiled) {
      tma_load_2d(stage, m, 0, (t * Shape::kUnitsPerTile + kc) * kUnitBox, bar, policy);
    } else {
      tma_load_2d(stage, m, kc * kUnitK, t * kTileRows, bar, policy);
      tma_load_2d(stage + 16384, m, kc * kUnitK + 128, t * kTileRows, bar, policy);
    }
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (!a.tiled) return;
    constexpr int kQU = kQTiles * Shape::kUnitsPerTile;
    prefetch_units(a.q_weight, u0, u1 < kQU ? u1 : kQU, Shape::kABytes);
    prefetch_units(a.k_weight, (u0 > kQU ? u0 : kQU) - kQU, u1 - kQU, Shape::kABytes);
  }
  __device__ void prologue(GemvCtl&) {
    epoch = tail_epoch(sc.counters + kFullHeadEpochBase, first_tile<Shape>() / kTilesPerHead);
    int kv, rope;
    if (a.position) {
      const int pos = *a.position;
      kv = pos >= 0 ? (pos % a.slots) * kDf * 2 : -1;
      rope = pos >= 0 && pos < a.rope_rows ? pos * kDf * 2 : -1;
    } else {
      kv = *a.kv_offset;
      rope = *a.rope_offset;
    }
    const bool kv_ok = kv >= 0 && (kv % (kDf * 2)) == 0 && kv / (kDf * 2) < a.slots;
    const bool rope_ok = rope >= 0 && (rope % (kDf * 2)) == 0 && rope / (kDf * 2) < a.rope_rows;
    const int e = threadIdx.x - 64;
    if (e == 0) {
      st->kv_ok = kv_ok;
      st->rope_ok = rope_ok;
      st->slot = kv / (kDf * 2);
      st->row = rope / (kDf * 2);
    }
    if (e >= 0 && e < 64) {  // 64 x 16 bytes per 512-element row
      if (rope_ok) {
        const size_t row = size_t(rope / (kDf * 2)) * kDf;
        cp_async_16(st->cos + e * 8, a.cos + row + e * 8);
        cp_async_16(st->sin + e * 8, a.sin + row + e * 8);
      }
      cp_async_16(st->qg + e * 8, a.q_rms + e * 8);
      cp_async_16(st->kg + e * 8, a.k_rms + e * 8);
    }
  }

  __device__ unsigned long long* words(int tile) const {
    return reinterpret_cast<unsigned long long*>(sc.partials) + kSplitWordsFullQkv +
           size_t(tile) * kMaxCtasPerGroup * kTileRows;
  }

  __device__ void finish_piece(int tile, int row, float v, int, GemvCtl&) const {
    constexpr int UPT = Shape::kUnitsPerTile;
    const int64_t grid = gridDim.x, total = Shape::kTotalUnits;
    const int head = tile / kTilesPerHead;
    const int run_last = int(int64_t(blockIdx.x + 1) * total / grid) - 1;
    const int head_last = kTilesPerHead * head + kTilesPerHead - 1;
    const int final_tile = run_last / UPT < head_last ? run_last / UPT : head_last;
    if (int(blockIdx.x) == cta_of_unit(int64_t(kTilesPerHead * head) * UPT, grid, total) && tile == final_tile) {
      finish_head(head, row, tile, v);
      return;
    }
    const int first = cta_of_unit(int64_t(tile) * UPT, grid, total);
    st_relaxed_gpu_u64(words(tile) + (blockIdx.x - first) * kTileRows + row,
                       (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v));
  }

  __device__ void finish_head(int head, int e, int own_tile, float own) const {
    constexpr int UPT = Shape::kUnitsPerTile;
    const int64_t grid = gridDim.x, total = Shape::kTotalUnits;
    float y[kTilesPerHead];
#pragma unroll
    for (int t = 0; t < kTilesPerHead; ++t) {  // element e + 128 t of the head = row e of its tile t
      const int tile = kTilesPerHead * head + t;
      const int first = cta_of_unit(int64_t(tile) * UPT, grid, total);
      const int span = cta_of_unit(int64_t(tile) * UPT + UPT - 1, grid, total) - first + 1;
      const int r = tile * kTileRows + e;
      const uint16_t sb = r < kQf ? a.q_scale[r] : a.k_scale[r - kQf];
      float acc = __uint_as_float(0x7fc00000u);
      if (span <= kMaxCtasPerGroup)
        acc = sum_tagged(words(tile) + e, span, tile == own_tile ? int(blockIdx.x) - first : -1, own, epoch, sc.err);
      else if (e == 0)
        atomicOr(sc.err, kErrInternal);
      y[t] = bf16_round(acc * bf16_to_f32(sb));  // scaled_projection (generate_references.py:265-274)
    }
    if (e == 0) sc.counters[kFullHeadEpochBase + head] = epoch;
    double ss = 0.0;
#pragma unroll
    for (int t = 0; t < kTilesPerHead; ++t) ss += double(y[t]) * double(y[t]);
    ss = warp_sum_d(ss);
    cp_async_wait_all();
    if ((threadIdx.x & 31) == 0) st->red[e / 32] = ss;
    named_bar(kEpiBarrier, kEpiThreads);
    const float inv = rms_inverse(((st->red[0] + st->red[1]) + st->red[2]) + st->red[3], kDf);
    if (!st->kv_ok || !st->rope_ok) {
      if (e == 0) atomicOr(sc.err, (st->kv_ok ? 0u : kErrKvOffset) | (st->rope_ok ? 0u : kErrRopeOffset));
      named_bar(kEpiBarrier, kEpiThreads);
      return;
    }
    const bool is_k = head == kGf;
    const uint16_t* gamma = is_k ? st->kg : st->qg;
    float nrm[kTilesPerHead];
#pragma unroll
    for (int t = 0; t < kTilesPerHead; ++t) {
      const float sv = y[t] * inv;
      nrm[t] = bf16_round(sv * bf16_to_f32(gamma[e + 128 * t]));
      if (is_k) st->out_v[e + 128 * t] = f32_to_bf16(sv);  // v: no gamma, no rotation
    }
    // RoPE over 512: out[i] = bf16(bf16(n[i] cos[i]) + bf16(n[i ^ 256] sin'[i])), sin' with its
    // low half negated (the partial rotation lives in the table: cos 1, sin 0 where it does not turn)
#pragma unroll
    for (int t = 0; t < kTilesPerHead; ++t) {
      const int i = e + 128 * t;
      const float c = bf16_round(nrm[t] * bf16_to_f32(st->cos[i]));
      const float sn = bf16_round(nrm[t ^ 2] * bf16_to_f32(st->sin[i]));
      st->out[i] = f32_to_bf16(c + sn);
    }
    named_bar(kEpiBarrier, kEpiThreads);
    if (e < 64) {  // 16-byte stores
      if (is_k) {
        reinterpret_cast<uint4*>(a.k_cache + size_t(st->slot) * kDf)[e] = reinterpret_cast<const uint4*>(st->out)[e];
        reinterpret_cast<uint4*>(a.v_cache + size_t(st->slot) * kDf)[e] = reinterpret_cast<const uint4*>(st->out_v)[e];
      } else {
        reinterpret_cast<uint4*>(a.q_out + head * kDf)[e] = reinterpret_cast<const uint4*>(st->out)[e];
      }
    }
    named_bar(kEpiBarrier, kEpiThreads);
  }

  __device__ void load_static(int g, uint4 (&raw)[4]) const { load_group_gamma(a.input_rms, g, raw); }
  __device__ void load_group(int g, uint4 (&raw)[4]) const { load_group_cg(a.x, g, raw); }
  __device__ void finish_group(const uint4 (&raw)[4], float inv, float (&v)[16]) const { rms_apply16(raw, inv, v); }
};

__global__ void __launch_bounds__(kGemvThreads, 1) full_qkv_kernel(const __grid_constant__ FullQkvMaps maps,
                                                                   FullQkvArgs a, Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ FullQkvStatic st;
  FullQkvOp op{&maps, a, sc};
  op.st = &st;
  gemv_run<FullQkvShape>(op, smem, sc);
  cp_async_wait_all();
}

// Global layer O (FOG/src/ops.rs:184-199): the attention output divided by the softmax sum of its
// head, bf16 (FOG/src/device/full/attention.rs:341-364), then the O projection with K = Qf, the
// post-attention RMSNorm and the residual add: the sliding O's engine and tail (it shares their
// scratch regions and counters: one op at a time per context).
struct FullOOp {
  using Shape = FullOShape;
  const CUtensorMap* map;
  FullOArgs a;
  Scratch sc;
  uint32_t tx_bytes = Shape::kABytes;
  static constexpr bool kOwnPieces = false;
  static constexpr bool kRms = false;
  static constexpr int kRmsGroups = 0;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {
      tma_load_2d(stage, map, 0, (tile * Shape::kUnitsPerTile + kc) * kUnitBox, bar, policy);
    } else {
      tma_load_2d(stage, map, kc * kUnitK, tile * kTileRows, bar, policy);
      tma_load_2d(stage + 16384, map, kc * kUnitK + 128, tile * kTileRows, bar, policy);
    }
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (a.tiled) prefetch_units(a.o_weight, u0, u1, Shape::kABytes);
  }
  __device__ void prologue(GemvCtl&) { epoch = tail_epoch(sc.counters + kTailEpochO, first_tile<Shape>()); }
  __device__ void load_static(int, uint4 (&)[4]) const {}
  // the 16 elements of group g and the softmax sum of their head (raw[2].x)
  __device__ void load_group(int g, uint4 (&raw)[4]) const {
    load_group_cg(a.x, g, raw);
    raw[2].x = __float_as_uint(__ldcg(a.running_sum + g * 16 / kDf));
  }
  __device__ void finish_group(const uint4 (&raw)[4], float, float (&v)[16]) const {
    bf16x16_to_f32(raw[0], raw[1], v);
    const float sum = __uint_as_float(raw[2].x);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = bf16_round(v[j] / sum);
  }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl&) const {
    const int r = tile * kTileRows + row;
    tail_record(*tail, a.post_rms, a.residual, sc.tile_ss + kTileSsO, sc.counters + kTailEpochO, epoch, tile, row,
                bf16_round(v * bf16_to_f32(a.o_scale[r])));
  }
  ResidualTail* tail;
  uint32_t epoch = 0;
  unsigned long long* split_words = reinterpret_cast<unsigned long long*>(sc.partials) + kSplitWordsO;
  uint32_t* split_epochs = sc.counters + kTailEpochO;
};

__global__ void __launch_bounds__(kGemvThreads, 1) full_o_kernel(const __grid_constant__ CUtensorMap map, FullOArgs a,
                                                                 Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ ResidualTail tail;
  if (threadIdx.x == 0) tail.n = 0;  // ordered by the engine's first barrier
  FullOOp op{&map, a, sc};
  op.tail = &tail;
  gemv_run<FullOShape>(op, smem, sc);
  tail_update(tail, a.residual, sc, sc.tile_ss + kTileSsO, op.epoch, kH / kTileRows, nullptr);
}

// ---------------------------------------------------------------------------------------
// FP8 feed-forward (per-output-channel f32 scales): up/gate + GeGLU, then down + post-RMSNorm +
// residual + layer scalar. Each projection is the reference's scaled_projection,
// bf16((x @ codes.T) * scale) (generate_references.py:265-274); the epilogues are those of the
// NVFP4 op (ops.rs:201-239). The two kernels share the NVFP4 op's scratch regions and epoch
// counters (same tile counts), so a model may mix both formats on one context.

struct UpGate8Maps {
  CUtensorMap up, gate;
};

template <int NTP>
struct UpGate8Op {
  using Shape = typename Shapes<NTP>::UpGate8;
  const UpGate8Maps* maps;
  Ffn8Args a;
  Scratch sc;
  uint32_t tx_bytes = Shape::kABytes;
  static constexpr bool kOwnPieces = false;
  static constexpr bool kRms = true;
  static constexpr int kRmsGroups = kH / 16;

  // stage: [K half 0: 64 up rows | 64 gate rows][K half 1: same] x 128 codes
  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {  // up and gate interleaved per 128-element half: one 256-row box per unit
      tma_load_2d(stage, &maps->up, 0, (tile * Shape::kUnitsPerTile + kc) * kUnitBox, bar, policy);
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tma_load_2d(stage + h * 16384, &maps->up, kc * kUnitK + h * 128, tile * 64, bar, policy);
        tma_load_2d(stage + h * 16384 + 8192, &maps->gate, kc * kUnitK + h * 128, tile * 64, bar, policy);
      }
    }
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (a.tiled) prefetch_units(a.up_w, u0, u1, Shape::kABytes);
  }
  __device__ void prologue(GemvCtl&) { epoch = tail_epoch(split_epochs, first_tile<Shape>()); }
  uint32_t epoch = 0;
  unsigned long long* split_words = reinterpret_cast<unsigned long long*>(sc.partials) + kSplitWordsUpGate;
  uint32_t* split_epochs = sc.counters + kSplitEpochUpGate;
  __device__ void load_static(int g, uint4 (&raw)[4]) const { load_group_gamma(a.pre_rms, g, raw); }
  __device__ void load_group(int g, uint4 (&raw)[4]) const { load_group_cg(a.residual, g, raw); }
  __device__ void finish_group(const uint4 (&raw)[4], float inv, float (&v)[16]) const { rms_apply16(raw, inv, v); }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl& ctl) const {
    const float s = row < 64 ? __ldg(a.up_s + tile * 64 + row) : __ldg(a.gate_s + tile * 64 + row - 64);
    const float val = bf16_round(v * s);
    if (row >= 64) ctl.xchg[row - 64] = val;
    named_bar(kEpiBarrier, kEpiThreads);
    // down_proj input: bf16(bf16(gelu_tanh(gate)) * up)  (gemma4.py:197)
    if (row < 64) ctl.out16[row] = f32_to_bf16(bf16_round(gelu_tanh(ctl.xchg[row])) * val);
    named_bar(kEpiBarrier, kEpiThreads);
    if (row < 8) reinterpret_cast<uint4*>(sc.act + tile * 64)[row] = reinterpret_cast<const uint4*>(ctl.out16)[row];
  }
};

template <int NTP>
__global__ void __launch_bounds__(kGemvThreads, 1) ffn8_upgate_kernel(const __grid_constant__ UpGate8Maps maps,
                                                                      Ffn8Args a, Scratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  UpGate8Op<NTP> op{&maps, a, sc};
  gemv_run<typename Shapes<NTP>::UpGate8>(op, smem, sc);
}

template <int NTP>
struct Down8Op {
  using Shape = typename Shapes<NTP>::Down8;
  const CUtensorMap* map;
  Ffn8Args a;
  Scratch sc;
  uint32_t tx_bytes = Shape::kABytes;
  static constexpr bool kOwnPieces = false;
  static constexpr bool kRms = false;
  static constexpr int kRmsGroups = 0;

  __device__ void load_unit(uint8_t* stage, int tile, int kc, uint64_t* bar, uint64_t policy) const {
    if (a.tiled) {
      tma_load_2d(stage, map, 0, (tile * Shape::kUnitsPerTile + kc) * kUnitBox, bar, policy);
    } else {
      tma_load_2d(stage, map, kc * kUnitK, tile * kTileRows, bar, policy);
      tma_load_2d(stage + 16384, map, kc * kUnitK + 128, tile * kTileRows, bar, policy);
    }
  }
  __device__ void prefetch_l2(int u0, int u1) const {
    if (a.tiled) prefetch_units(a.down_w, u0, u1, Shape::kABytes);
  }
  __device__ void prologue(GemvCtl&) { epoch = tail_epoch(sc.counters + kTailEpochDown, first_tile<Shape>()); }
  __device__ void load_static(int, uint4 (&)[4]) const {}
  __device__ void load_group(int g, uint4 (&raw)[4]) const { load_group_cg(sc.act, g, raw); }
  __device__ void finish_group(const uint4 (&raw)[4], float, float (&v)[16]) const {
    bf16x16_to_f32(raw[0], raw[1], v);
  }
  __device__ void finalize_tile(int tile, int row, float v, GemvCtl&) const {
    const int r = tile * kTileRows + row;
    const float s = __ldg(a.down_s + r);
    const float sum = tp_allreduce(*tp, 1, tile, row, v, sc.err);  // the K slices of every rank
    tail_record(*tail, a.post_rms, a.residual, sc.tile_ss + kTileSsDown, sc.counters + kTailEpochDown, epoch, tile,
                row, bf16_round(sum * s));
  }
  ResidualTail* tail;
  const TpLink* tp;
  uint32_t epoch = 0;
  unsigned long long* split_words = reinterpret_cast<unsigned long long*>(sc.partials) + kSplitWordsDown;
  uint32_t* split_epochs = sc.counters + kTailEpochDown;
};

template <int NTP>
__global__ void __launch_bounds__(kGemvThreads, 1) ffn8_down_kernel(const __grid_constant__ CUtensorMap map,
                                                                    Ffn8Args a, Scratch sc,
                                                                    const __grid_constant__ TpLink tp) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ ResidualTail tail;
  if (threadIdx.x == 0) tail.n = 0;  // ordered by the engine's first barrier
  Down8Op<NTP> op{&map, a, sc};
  op.tail = &tail;
  op.tp = &tp;
  gemv_run<typename Shapes<NTP>::Down8>(op, smem, sc);
  tail_update(tail, a.residual, sc, sc.tile_ss + kTileSsDown, op.epoch, kH / kTileRows, a.layer_scalar);
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

// One CTA per SM (at most one per unit), unless a smaller GPU would give a CTA more distinct K
// units than its B slots hold (a run of n units touches min(n, units per tile) of them).
template <class Shape>
int grid_for(const LaunchEnv& env) {
  int grid = env.sm_count < Shape::kTotalUnits ? env.sm_count : Shape::kTotalUnits;
  if (Shape::kBSlots < Shape::kUnitsPerTile) {
    const int need = (Shape::kTotalUnits + Shape::kBSlots - 1) / Shape::kBSlots;
    grid = grid > need ? grid : need;
  }
  return grid;
}

// The kernels of one tensor-parallel degree, called as f(std::integral_constant<int, NTP>).
template <class F>
cudaError_t by_degree(int world, F&& f) {
  switch (world) {
    case 1: return f(std::integral_constant<int, 1>{});
    case 2: return f(std::integral_constant<int, 2>{});
    case 4: return f(std::integral_constant<int, 4>{});
    case 8: return f(std::integral_constant<int, 8>{});
    default: return cudaErrorInvalidValue;
  }
}

// The most tiles one CTA of a `grid`-CTA launch finishes: a tile is finished by the CTA holding
// its first unit (whole or split), so this counts the tiles whose first unit lies in one run.
template <class Shape>
int max_tiles_finished(int grid) {
  int best = 0, run = 0, prev = -1;
  for (int t = 0; t < Shape::kTiles; ++t) {
    const int c = cta_of_unit(int64_t(t) * Shape::kUnitsPerTile, grid, Shape::kTotalUnits);
    run = c == prev ? run + 1 : 1;
    prev = c;
    best = run > best ? run : best;
  }
  return best;
}

template <int NTP>
bool geometry_fits(int sm_count) {
  using S = Shapes<NTP>;
  LaunchEnv env{};
  env.sm_count = sm_count;
  // the residual tails keep at most kMaxFinTiles finished tiles of a CTA in shared memory, and a
  // split tile's pieces must fit its kMaxCtasPerGroup slots
  if (NTP == 1 && max_tiles_finished<FullOShape>(grid_for<FullOShape>(env)) > kMaxFinTiles) return false;
  return max_tiles_finished<typename S::O>(grid_for<typename S::O>(env)) <= kMaxFinTiles &&
         max_tiles_finished<typename S::Down>(grid_for<typename S::Down>(env)) <= kMaxFinTiles &&
         max_tiles_finished<typename S::Down8>(grid_for<typename S::Down8>(env)) <= kMaxFinTiles;
}

template <int NTP>
cudaError_t prepare_degree() {
  using S = Shapes<NTP>;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(qkv_kernel<NTP>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::Qkv::kSmemBytes))))
    return e;
  if ((e = cudaFuncSetAttribute(o_kernel<NTP>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::O::kSmemBytes))))
    return e;
  if ((e = cudaFuncSetAttribute(ffn_upgate_kernel<NTP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(S::UpGate::kSmemBytes))))
    return e;
  if ((e = cudaFuncSetAttribute(ffn_down_kernel<NTP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(S::Down::kSmemBytes))))
    return e;
  if ((e = cudaFuncSetAttribute(ffn8_upgate_kernel<NTP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(S::UpGate8::kSmemBytes))))
    return e;
  return cudaFuncSetAttribute(ffn8_down_kernel<NTP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(S::Down8::kSmemBytes));
}

template <int NTP>
cudaError_t launch_qkv_t(const QkvArgs& a, const LaunchEnv& env) {
  using Geo = TpGeo<NTP>;
  using Shape = typename Shapes<NTP>::Qkv;
  QkvMaps m;
  cudaError_t e;
  // unit-tiled: a matrix of R rows is [R * K / 128, 128] bytes, one 256-row box per unit
  const uint64_t cols = a.tiled ? 128 : kH, fq = a.tiled ? kH / 128 : 1;
  const uint32_t box = a.tiled ? kUnitBox : kTileRows;
  if ((e = env.maps->u8(a.q_weight, cols, Geo::kQRows * fq, 128, box, true, &m.q))) return e;
  if ((e = env.maps->u8(a.k_weight, cols, Geo::kKvRows * fq, 128, box, true, &m.k))) return e;
  if ((e = env.maps->u8(a.v_weight, cols, Geo::kKvRows * fq, 128, box, true, &m.v))) return e;
  return launch(qkv_kernel<NTP>, grid_for<Shape>(env), Shape::kSmemBytes, env, m, a, env.sc);  // stamps at 0
}

template <int NTP>
cudaError_t launch_o_t(const OArgs& a, const LaunchEnv& env) {
  constexpr int kK = TpGeo<NTP>::kQRows;  // this rank's K slice of O
  using Shape = typename Shapes<NTP>::O;
  CUtensorMap m;
  cudaError_t e;
  if ((e = env.maps->u8(a.o_weight, a.tiled ? 128 : kK, a.tiled ? uint64_t(kH) * (kK / 128) : kH, 128,
                        a.tiled ? kUnitBox : kTileRows, true, &m)))
    return e;
  Scratch sc = env.sc;
#ifdef G4_TRACE
  if (sc.trace) sc.trace += 2 * 4096;  // profiling builds: separate stamp rows per kernel
#endif
  return launch(o_kernel<NTP>, grid_for<Shape>(env), Shape::kSmemBytes, env, m, a, sc, env.tp);
}

template <int NTP>
cudaError_t launch_ffn_t(const FfnArgs& a, const LaunchEnv& env) {
  constexpr int kRows = TpGeo<NTP>::kFfnRows, kDownK = TpGeo<NTP>::kDownK;
  using UG = typename Shapes<NTP>::UpGate;
  using DN = typename Shapes<NTP>::Down;
  UpGateMaps ug;
  DownMaps dn;
  cudaError_t e;
  if (a.tiled) {
    // unit-tiled: up|gate codes interleaved, one 128-row x 128-byte box per unit; down codes
    // likewise. The block scales are read with bulk copies (no map). gate_packed / gate_scale
    // are not used (they live in the up buffers).
    ug.gate = ug.up;
    ug.gate_s = ug.up_s = ug.up;
    dn.s = dn.w;
    if ((e = env.maps->u8(a.up_packed, 128, uint64_t(kRows) / 64 * (kH / kUnitK) * kTileRows, 128, kTileRows, true,
                          &ug.up)))
      return e;
    if ((e = env.maps->u8(a.down_packed, 128, uint64_t(kH) / kTileRows * (kDownK / kUnitK) * kTileRows, 128,
                          kTileRows, true, &dn.w)))
      return e;
  } else {
    if ((e = env.maps->u8(a.up_packed, kH / 2, kRows, 128, 64, true, &ug.up))) return e;
    if ((e = env.maps->u8(a.gate_packed, kH / 2, kRows, 128, 64, true, &ug.gate))) return e;
    if ((e = env.maps->u8(a.up_scale, kH / 16, kRows, 16, 64, false, &ug.up_s))) return e;
    if ((e = env.maps->u8(a.gate_scale, kH / 16, kRows, 16, 64, false, &ug.gate_s))) return e;
    if ((e = env.maps->u8(a.down_packed, kDownK / 2, kH, 128, kTileRows, true, &dn.w))) return e;
    if ((e = env.maps->u8(a.down_scale, kDownK / 16, kH, 16, kTileRows, false, &dn.s))) return e;
  }
  Scratch sc = env.sc;
#ifdef G4_TRACE
  static int calls = 0;  // profiling builds: separate stamp rows per kernel, alternating per call
  const int row_base = 3 + 2 * (calls++ % 2);
  if (sc.trace) sc.trace += row_base * 4096;
#endif
  e = launch(ffn_upgate_kernel<NTP>, grid_for<UG>(env), UG::kSmemBytes, env, ug, a, sc);
  if (e != cudaSuccess) return e;
  LaunchEnv chained = env;
  chained.pdl = true;  // the down pass prefetches its weights while the up/gate pass drains
#ifdef G4_TRACE
  if (chained.sc.trace) chained.sc.trace += (row_base + 1) * 4096;  // profiling builds: separate stamp rows
#endif
  return launch(ffn_down_kernel<NTP>, grid_for<DN>(env), DN::kSmemBytes, chained, dn, a, chained.sc, env.tp);
}

template <int NTP>
cudaError_t launch_ffn8_t(const Ffn8Args& a, const LaunchEnv& env) {
  constexpr int kRows = TpGeo<NTP>::kFfnRows, kDownK = TpGeo<NTP>::kDownK;
  using UG = typename Shapes<NTP>::UpGate8;
  using DN = typename Shapes<NTP>::Down8;
  UpGate8Maps ug;
  CUtensorMap dn;
  cudaError_t e;
  if (a.tiled) {
    // up|gate interleaved per 128-element half of each tile's 64 + 64 rows: [2 kRows * H / 128, 128]
    // bytes, one 256-row box per unit; down unit-tiled like O
    ug.gate = ug.up;
    if ((e = env.maps->u8(a.up_w, 128, uint64_t(2 * kRows) * (kH / 128), 128, kUnitBox, true, &ug.up))) return e;
    if ((e = env.maps->u8(a.down_w, 128, uint64_t(kH) * (kDownK / 128), 128, kUnitBox, true, &dn))) return e;
  } else {
    if ((e = env.maps->u8(a.up_w, kH, kRows, 128, 64, true, &ug.up))) return e;
    if ((e = env.maps->u8(a.gate_w, kH, kRows, 128, 64, true, &ug.gate))) return e;
    if ((e = env.maps->u8(a.down_w, kDownK, kH, 128, kTileRows, true, &dn))) return e;
  }
  Scratch sc = env.sc;
#ifdef G4_TRACE
  if (sc.trace) sc.trace += 7 * 4096;  // profiling builds: separate stamp rows per kernel
#endif
  e = launch(ffn8_upgate_kernel<NTP>, grid_for<UG>(env), UG::kSmemBytes, env, ug, a, sc);
  if (e != cudaSuccess) return e;
  LaunchEnv chained = env;
  chained.pdl = true;  // the down pass prefetches its weights while the up/gate pass drains
#ifdef G4_TRACE
  if (sc.trace) sc.trace += 4096;
#endif
  return launch(ffn8_down_kernel<NTP>, grid_for<DN>(env), DN::kSmemBytes, chained, dn, a, sc, env.tp);
}

}  // namespace

bool proj_geometry_fits(int sm_count) {
  return geometry_fits<1>(sm_count) && geometry_fits<2>(sm_count) && geometry_fits<4>(sm_count) &&
         geometry_fits<8>(sm_count);
}

cudaError_t prepare_proj_kernels() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(full_qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(FullQkvShape::kSmemBytes))))
    return e;
  if ((e = cudaFuncSetAttribute(full_o_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(FullOShape::kSmemBytes))))
    return e;
  if ((e = prepare_degree<1>())) return e;
  if ((e = prepare_degree<2>())) return e;
  if ((e = prepare_degree<4>())) return e;
  return prepare_degree<8>();
}

cudaError_t launch_qkv(const QkvArgs& a, const LaunchEnv& env) {
  return by_degree(env.tp.world, [&](auto d) { return launch_qkv_t<decltype(d)::value>(a, env); });
}

cudaError_t launch_o(const OArgs& a, const LaunchEnv& env) {
  return by_degree(env.tp.world, [&](auto d) { return launch_o_t<decltype(d)::value>(a, env); });
}

cudaError_t launch_ffn_nvfp4(const FfnArgs& a, const LaunchEnv& env) {
  return by_degree(env.tp.world, [&](auto d) { return launch_ffn_t<decltype(d)::value>(a, env); });
}

cudaError_t launch_full_qkv(const FullQkvArgs& a, const LaunchEnv& env) {
  if (env.tp.world != 1) return cudaErrorNotSupported;  // the global layers run on one GPU
  FullQkvMaps m;
  cudaError_t e;
  const uint64_t cols = a.tiled ? 128 : kH, fq = a.tiled ? kH / 128 : 1;
  const uint32_t box = a.tiled ? kUnitBox : kTileRows;
  if ((e = env.maps->u8(a.q_weight, cols, uint64_t(kQf) * fq, 128, box, true, &m.q))) return e;
  if ((e = env.maps->u8(a.k_weight, cols, uint64_t(kDf) * fq, 128, box, true, &m.k))) return e;
  return launch(full_qkv_kernel, grid_for<FullQkvShape>(env), FullQkvShape::kSmemBytes, env, m, a, env.sc);
}

cudaError_t launch_full_o(const FullOArgs& a, const LaunchEnv& env) {
  if (env.tp.world != 1) return cudaErrorNotSupported;
  CUtensorMap m;
  cudaError_t e;
  if ((e = env.maps->u8(a.o_weight, a.tiled ? 128 : kQf, a.tiled ? uint64_t(kH) * (kQf / 128) : kH, 128,
                        a.tiled ? kUnitBox : kTileRows, true, &m)))
    return e;
  return launch(full_o_kernel, grid_for<FullOShape>(env), FullOShape::kSmemBytes, env, m, a, env.sc);
}

cudaError_t launch_ffn_fp8(const Ffn8Args& a, const LaunchEnv& env) {
  return by_degree(env.tp.world, [&](auto d) { return launch_ffn8_t<decltype(d)::value>(a, env); });
}

namespace {
template <class Shape>
L2Hint engine_hint(const uint8_t* w, int first_units, const LaunchEnv& env) {
  L2Hint h;
  h.base = w;
  h.unit_bytes = uint32_t(Shape::kABytes);
  h.total_units = Shape::kTotalUnits;
  h.consumer_grid = grid_for<Shape>(env);
  const int longest = (h.total_units + h.consumer_grid - 1) / h.consumer_grid;  // the longest run
  h.first_units = first_units < longest ? first_units : longest;
  return h;
}
template <template <int> class Pick>
L2Hint hint_by_degree(const uint8_t* w, int first_units, const LaunchEnv& env) {
  switch (env.tp.world) {
    case 1: return engine_hint<typename Pick<1>::type>(w, first_units, env);
    case 2: return engine_hint<typename Pick<2>::type>(w, first_units, env);
    case 4: return engine_hint<typename Pick<4>::type>(w, first_units, env);
    case 8: return engine_hint<typename Pick<8>::type>(w, first_units, env);
    default: return L2Hint{};
  }
}
template <int NTP>
struct PickO {
  using type = typename Shapes<NTP>::O;
};
template <int NTP>
struct PickUpGate8 {
  using type = typename Shapes<NTP>::UpGate8;
};
}  // namespace

L2Hint l2_hint_o(const OArgs& a, int first_units, const LaunchEnv& env) {
  return a.tiled ? hint_by_degree<PickO>(a.o_weight, first_units, env) : L2Hint{};
}

L2Hint l2_hint_ffn8_upgate(const Ffn8Args& a, int first_units, const LaunchEnv& env) {
  return a.tiled ? hint_by_degree<PickUpGate8>(a.up_w, first_units, env) : L2Hint{};
}

// ---------------------------------------------------------------------------------------
// unit-tiled weight layout

namespace {
// dst block (t, u) = [src rows of tile t, unit u] then, with src2, [src2 rows of tile t, unit u]
__global__ void pack_tiles_kernel(const uint8_t* __restrict__ src, const uint8_t* __restrict__ src2,
                                  uint8_t* __restrict__ dst, int rows, int row_bytes, int unit_bytes, int tile_rows) {
  // one thread per 16-byte chunk of the destination
  const int units = row_bytes / unit_bytes, chunks = unit_bytes / 16, nsrc = src2 ? 2 : 1;
  const int64_t total = int64_t(rows) * row_bytes / 16 * nsrc;
  for (int64_t q = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; q < total; q += int64_t(gridDim.x) * blockDim.x) {
    const int b = int(q % chunks) * 16;
    const int64_t row_in = q / chunks;  // ((blk * nsrc + which) * tile_rows + r)
    const int r = int(row_in % tile_rows);
    const int64_t bw = row_in / tile_rows;
    const int which = int(bw % nsrc);
    const int64_t blk = bw / nsrc;
    const int u = int(blk % units);
    const int64_t t = blk / units;
    const uint8_t* from = which ? src2 : src;
    *reinterpret_cast<uint4*>(dst + q * 16) =
        *reinterpret_cast<const uint4*>(from + (t * tile_rows + r) * int64_t(row_bytes) + int64_t(u) * unit_bytes + b);
  }
}
}  // namespace

cudaError_t launch_pack_tiles(const uint8_t* src, const uint8_t* src2, uint8_t* dst, int rows, int row_bytes,
                              int unit_bytes, int tile_rows, cudaStream_t stream) {
  const int64_t total = int64_t(rows) * row_bytes / 16 * (src2 ? 2 : 1);
  const int blocks = int((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  pack_tiles_kernel<<<blocks, 256, 0, stream>>>(src, src2, dst, rows, row_bytes, unit_bytes, tile_rows);
  return cudaGetLastError();
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
  const auto it = entries_.find({base, key});
  return it == entries_.end() ? nullptr : &it->second;
}

void TmapCache::put(const void* base, uint64_t key, const CUtensorMap& map) { entries_[{base, key}] = map; }

cudaError_t TmapCache::kv(const void* base, uint64_t ring, uint32_t heads, uint32_t dim, uint32_t box_slots,
                          CUtensorMap* out) {
  const uint64_t key = (ring << 32) ^ (uint64_t(heads) << 24) ^ (uint64_t(dim) << 12) ^ box_slots ^ (uint64_t(3) << 62);
  if (const CUtensorMap* m = find(base, key)) {
    *out = *m;
    return cudaSuccess;
  }
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t gdim[3] = {dim, heads, ring};
  const cuuint64_t gstride[2] = {uint64_t(dim) * 2, uint64_t(dim) * heads * 2};
  const cuuint32_t box[3] = {dim, 1, box_slots};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), gdim, gstride, box, estride,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  put(base, key, *out);
  return cudaSuccess;
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

cudaError_t TmapCache::bf16(const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                            CUtensorMap* out, bool half) {
  const uint64_t key = (cols << 34) ^ (rows << 12) ^ (uint64_t(box_cols) << 4) ^ (uint64_t(box_rows) << 1) ^
                       (uint64_t(1) << 62) ^ (uint64_t(half) << 61);
  if (const CUtensorMap* m = find(base, key)) {
    *out = *m;
    return cudaSuccess;
  }
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = enc(out, half ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                         const_cast<void*>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  put(base, key, *out);
  return cudaSuccess;
}

// ---------------------------------------------------------------------------------------
// O projection on scratch the caller provides, with nothing cached or allocated

size_t o_scratch_bytes() {
  return kScratchHeadBytes + size_t(kCounterCount) * sizeof(uint32_t) + kTileSsBytes +
         size_t(Shapes<1>::O::kTiles) * kMaxCtasPerGroup * kTileRows * sizeof(unsigned long long);
}

cudaError_t launch_o_uncached(const OArgs& a, const LaunchEnv& env) {
  if (a.tiled || env.tp.world != 1) return cudaErrorInvalidValue;  // one rank, row-major layout only
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap m;
  const cuuint64_t gdim[2] = {uint64_t(kQs), uint64_t(kH)};
  const cuuint64_t gstride[1] = {uint64_t(kQs)};
  const cuuint32_t box[2] = {128, uint32_t(kTileRows)};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.o_weight), gdim, gstride, box,
                         estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  using Shape = Shapes<1>::O;
  return launch(o_kernel<1>, grid_for<Shape>(env), Shape::kSmemBytes, env, m, a, env.sc, env.tp);
}

}  // namespace g4
