// Weight-streaming split-K GEMV engine shared by every projection of the decode layer.
//
// Unit of work: 16 consecutive weight rows x BATCH consecutive K elements. The flat sequence
// of G row groups x (K / BATCH) units is split evenly across every warp of the grid (contiguous
// runs, so a CTA covers a contiguous run too). Each warp streams its units through a private
// ring of S shared-memory slots with cp.async: every lane copies exactly the fragment bytes it
// will contract into lane-private, bank-conflict-free slots, so S-1 units stay in flight per
// warp without holding registers and no cross-lane synchronisation is needed. The codes are
// converted to exact f16 in registers and contracted on the tensor pipe with mma.m16n8k16
// (f32 accumulate) against the activation, held in shared memory as two exact f16 columns.
//
// K permutation: within a unit (BATCH elements of a row), lane t (of the 4 lanes sharing an
// MMA row pair) loads the 16-byte chunks at byte offsets 16t + 64v, so the four lanes read 64
// contiguous bytes of each row per load instruction (whole 32-byte sectors). k-step q takes 4
// consecutive elements of one of the lane's chunks, which the MMA sees as logical columns
// {2t, 2t+1, 2t+8, 2t+9}. The same permutation is applied to the activation fragment, so the
// contraction is exact in any order; an NVFP4 chunk (32 elements) holds two whole scale blocks.
//
// Reduction: a warp whose run covers a whole group finalises it directly. Partial pieces are
// parked in shared memory and summed per group in warp order once the CTA's warps are done;
// only groups that straddle two CTAs go through global memory (per-group ticket, CTA order).
// The result therefore never depends on timing.
#pragma once

#include "g4_common.cuh"

namespace g4 {

enum class WFmt { kFp8, kNvfp4 };

// ---------------------------------------------------------------------------------------
// Activation columns in shared memory

// f16 element e of a column sits at half index e + 8 * (e / 64): the pad spreads the four
// lanes of a row pair over distinct banks for both weight formats.
template <int BATCH>
__host__ __device__ constexpr int act_half_index(int e) {
  return e + 8 * (e / 64);
}
template <int BATCH>
__host__ __device__ constexpr int act_col_stride(int k) {
  // bytes per column, rounded so that column 1 sits two banks after column 0 (so column 1 is
  // 8-byte but not 16-byte aligned: every access to the columns is at most 8 bytes wide)
  int b = act_half_index<BATCH>(k) * 2;
  while (b % 128 != 8) b += 8;
  return b;
}

// Build the hi/lo f16 columns of a K-vector whose values this thread holds in `vals` (element
// index of vals[v][j] = (threadIdx.x + v * blockDim.x) * 8 + j). The vector is scaled by 2^e so
// that max|h| lands in [2^14, 2^15): hi = f16(h 2^e), lo = f16((h 2^e - hi) 2^24). Both are exact
// for every bf16 value within a 2^29 ratio of the maximum, so the tensor-op product reproduces
// the f32 dot product of the bf16 activation with the exact weights. Returns 2^-e.
template <int BATCH, int VPT>
__device__ float build_act_columns(uint8_t* cols, int k, const float (&vals)[VPT][8], float* red_f) {
  float amax = 0.f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int base = (threadIdx.x + v * blockDim.x) * 8;
    if (base < k) {
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(vals[v][j]));
    }
  }
  amax = block_max(amax, red_f);
  int e = 0;
  if (amax > 0.f) {
    const int ex = int((__float_as_uint(amax) >> 23) & 0xff) - 127;
    e = 14 - ex;
    e = e > 126 ? 126 : (e < -126 ? -126 : e);
  }
  const float up = pow2f(e);
  const int cs = act_col_stride<BATCH>(k);
  __half* hi = reinterpret_cast<__half*>(cols);
  __half* lo = reinterpret_cast<__half*>(cols + cs);
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int base = (threadIdx.x + v * blockDim.x) * 8;
    if (base < k) {
      __align__(16) __half h8[8], l8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float x = vals[v][j] * up;
        h8[j] = __float2half_rn(x);
        l8[j] = __float2half_rn((x - __half2float(h8[j])) * 16777216.0f);
      }
      // 8 consecutive elements never straddle a pad (the pad period is a multiple of 8). The lo
      // column is only 8-byte aligned (its stride keeps it two banks after hi): 8-byte stores.
      const int hidx = act_half_index<BATCH>(base);
      const uint2* h2 = reinterpret_cast<const uint2*>(h8);
      const uint2* l2 = reinterpret_cast<const uint2*>(l8);
      reinterpret_cast<uint2*>(hi + hidx)[0] = h2[0];
      reinterpret_cast<uint2*>(hi + hidx)[1] = h2[1];
      reinterpret_cast<uint2*>(lo + hidx)[0] = l2[0];
      reinterpret_cast<uint2*>(lo + hidx)[1] = l2[1];
    }
  }
  return pow2f(-e);
}

// Load a bf16 K-vector (16-byte aligned) as VPT 8-element vectors per thread, all loads in
// flight at once. Elements past k read as zero.
template <int VPT>
__device__ __forceinline__ void load_bf16_vec(const uint16_t* src, int k, float (&vals)[VPT][8], bool coherent) {
  uint4 raw[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int base = (threadIdx.x + v * blockDim.x) * 8;
    raw[v] = make_uint4(0, 0, 0, 0);
    if (base < k)
      raw[v] = coherent ? __ldcg(reinterpret_cast<const uint4*>(src + base)) : *reinterpret_cast<const uint4*>(src + base);
  }
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const uint16_t* b = reinterpret_cast<const uint16_t*>(&raw[v]);
#pragma unroll
    for (int j = 0; j < 8; ++j) vals[v][j] = bf16_to_f32(b[j]);
  }
}

// ---------------------------------------------------------------------------------------
// Engine geometry

template <WFmt F, int NMAT, int BATCH>
struct Unit {
  static constexpr bool kFp4 = (F == WFmt::kNvfp4);
  static constexpr int kLaneElems = BATCH / 4;                           // contiguous K elements per lane
  static constexpr int kLaneBytes = kFp4 ? kLaneElems / 2 : kLaneElems;  // code bytes per lane per row
  static constexpr int kVec = kLaneBytes / 16;                            // 16-byte loads per lane per row
  static constexpr int kSteps = BATCH / 16;                               // mma k-steps per unit
  static_assert(kLaneBytes % 16 == 0, "a lane run must be whole 16-byte loads");
  static_assert(BATCH == 256, "the k-step / scale bookkeeping below assumes 256-element units");
  uint4 code[NMAT][2][kVec];  // rows g and g+8 of each matrix
  uint32_t scale[NMAT][2];    // NVFP4: word 4t..4t+3 of the unit's 16 block scales, rows g and g+8
};

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

struct Parked {  // per warp: up to two partial pieces (its first and its last group)
  int grp[2];
  int units[2];
};

// shared memory the engine needs per CTA of W warps (parked pieces)
template <int NMAT>
__host__ __device__ constexpr size_t engine_smem(int warps) {
  return size_t(warps) * 2 * NMAT * 16 * 4 + size_t(warps) * sizeof(Parked);
}

// The warp whose run contains unit u.
__device__ __forceinline__ int64_t warp_of_unit(int64_t u, int64_t n_warps, int64_t total) {
  return ((u + 1) * n_warps + total - 1) / total - 1;
}

// Lanes 0..15 receive row `lane` from the MMA accumulator layout (rows g and g+8 at lane g*4).
__device__ __forceinline__ float rows_to_lanes(float v_g, float v_g8) {
  const int lane = threadIdx.x & 31;
  const float a = __shfl_sync(0xffffffffu, v_g, (lane & 7) * 4);
  const float b = __shfl_sync(0xffffffffu, v_g8, (lane & 7) * 4);
  return lane < 8 ? a : b;
}

// Global partial slots per straddling group (a group spans at most this many CTAs).
constexpr int kMaxCtasPerGroup = 8;

// The engine, run by every warp of every CTA (it synchronises the CTA once).
//   rows_of(grp, m)   -> first code byte of the group's row 0 in matrix m
//   scales_of(grp, m) -> first scale byte of the group's row 0 (NVFP4)
//   finalize(grp, tot[NMAT]) -> called exactly once per group in the grid by one whole warp;
//                              lanes 0..15 hold the f32 totals of rows 0..15 of each matrix.
// Each warp keeps the next PD units' fragments in flight in registers.
template <WFmt F, int NMAT, int BATCH, int PD, int W, class RowsFn, class ScalesFn, class FinalFn>
__device__ void stream_gemv(uint8_t* engine_mem, const uint8_t* act_cols, int k_total, int groups, int row_bytes,
                            int scale_row_bytes, RowsFn rows_of, ScalesFn scales_of, FinalFn finalize,
                            const Scratch& sc) {
  using U = Unit<F, NMAT, BATCH>;
  constexpr int D = PD + 1;  // register ring depth
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  const int per_group = k_total / BATCH;
  const int64_t total = int64_t(groups) * per_group;
  const int64_t n_warps = int64_t(gridDim.x) * W;
  const int64_t wid = int64_t(blockIdx.x) * W + warp;
  const int64_t u0 = split_begin(wid, n_warps, total);
  const int n = int(split_begin(wid + 1, n_warps, total) - u0);
  const int cs = act_col_stride<BATCH>(k_total);

  float* parked_v = reinterpret_cast<float*>(engine_mem);                     // [W][2][NMAT][16]
  Parked* parked = reinterpret_cast<Parked*>(parked_v + W * 2 * NMAT * 16);   // [W]
  if (lane == 0) parked[warp] = Parked{{-1, -1}, {0, 0}};

  auto load = [&](U& r, int i) {  // fragments of unit u0+i
    const int64_t u = u0 + i;
    const int grp = int(u / per_group), b = int(u % per_group);
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const uint8_t* ra = rows_of(grp, m) + size_t(g) * row_bytes + size_t(b) * (U::kVec * 64) + t * 16;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr)
#pragma unroll
        for (int v = 0; v < U::kVec; ++v) r.code[m][rr][v] = ldg_stream(ra + size_t(rr) * 8 * row_bytes + v * 64);
      if constexpr (U::kFp4) {
        const uint8_t* sa = scales_of(grp, m) + size_t(g) * scale_row_bytes + size_t(b) * (BATCH / 16) + t * 4;
        r.scale[m][0] = ldg_stream_u32(sa);
        r.scale[m][1] = ldg_stream_u32(sa + size_t(8) * scale_row_bytes);
      }
    }
  };

  float d[NMAT][4];
#pragma unroll
  for (int m = 0; m < NMAT; ++m) d[m][0] = d[m][1] = d[m][2] = d[m][3] = 0.f;
  int units_in_piece = 0, parked_count = 0;

  auto compute = [&](const U& cur, int i) {
    const int64_t u = u0 + i;
    const int grp = int(u / per_group), b = int(u % per_group);
    // activation fragment source: column (g & 1) of unit b
    const __half* bcol = reinterpret_cast<const __half*>(act_cols + (g & 1) * cs);
    const bool bact = g < 2;
    // NVFP4: gather this lane's four block scales (blocks 2t, 2t+1 of each 128-element half)
    // from the words that lanes t/2 and 2 + t/2 of the row pair loaded
    uint32_t lane_scale[NMAT][2];
    if constexpr (U::kFp4) {
      const int quad = lane & ~3;
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const uint32_t w0 = __shfl_sync(0xffffffffu, cur.scale[m][rr], quad + (t >> 1));
          const uint32_t w1 = __shfl_sync(0xffffffffu, cur.scale[m][rr], quad + 2 + (t >> 1));
          const uint32_t h0 = (t & 1) ? (w0 >> 16) : (w0 & 0xffff);
          const uint32_t h1 = (t & 1) ? (w1 >> 16) : (w1 & 0xffff);
          lane_scale[m][rr] = h0 | (h1 << 16);  // byte j = block of chunk j/2, half j%2
        }
    }
#pragma unroll
    for (int q = 0; q < U::kSteps; ++q) {
      // element offset of k-step q inside the unit (see the K permutation above)
      const int eoff = U::kFp4 ? (128 * (q / 8) + 32 * t + 4 * (q % 8)) : (64 * (q / 4) + 16 * t + 4 * (q % 4));
      uint2 bb = make_uint2(0, 0);
      if (bact) bb = *reinterpret_cast<const uint2*>(bcol + act_half_index<BATCH>(b * BATCH + eoff));
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        uint32_t a0, a1, a2, a3;
        if constexpr (!U::kFp4) {
          // fp8: k-step q uses word q % 4 of chunk q / 4
          const uint4 va = cur.code[m][0][q / 4], vb = cur.code[m][1][q / 4];
          const uint32_t wa = (q % 4 == 0) ? va.x : (q % 4 == 1) ? va.y : (q % 4 == 2) ? va.z : va.w;
          const uint32_t wb = (q % 4 == 0) ? vb.x : (q % 4 == 1) ? vb.y : (q % 4 == 2) ? vb.z : vb.w;
          a0 = cvt_e4m3x2_f16x2(uint16_t(wa & 0xffff));
          a1 = cvt_e4m3x2_f16x2(uint16_t(wb & 0xffff));
          a2 = cvt_e4m3x2_f16x2(uint16_t(wa >> 16));
          a3 = cvt_e4m3x2_f16x2(uint16_t(wb >> 16));
        } else {
          // nvfp4: k-step q uses bytes 2(q % 8), 2(q % 8) + 1 of chunk q / 8
          const uint4 va = cur.code[m][0][q / 8], vb = cur.code[m][1][q / 8];
          const int w = (q % 8) / 2;
          const uint32_t wa = (w == 0) ? va.x : (w == 1) ? va.y : (w == 2) ? va.z : va.w;
          const uint32_t wb = (w == 0) ? vb.x : (w == 1) ? vb.y : (w == 2) ? vb.z : vb.w;
          uint32_t fa0, fa1, fb0, fb1;
          cvt_e2m1x4_f16x2((q % 2 == 0) ? (wa & 0xffff) : (wa >> 16), fa0, fa1);
          cvt_e2m1x4_f16x2((q % 2 == 0) ? (wb & 0xffff) : (wb >> 16), fb0, fb1);
          // block scale of these elements: lane scale byte q / 4, exact as f16
          const int blk = q / 4;
          const uint16_t sab =
              uint16_t(((lane_scale[m][0] >> (8 * blk)) & 0xff) | (((lane_scale[m][1] >> (8 * blk)) & 0xff) << 8));
          const uint32_t sc2 = cvt_e4m3x2_f16x2(sab);
          const uint32_t sA = (sc2 & 0xffffu) * 0x10001u, sB = (sc2 >> 16) * 0x10001u;
          a0 = hmul2_u32(fa0, sA);
          a1 = hmul2_u32(fb0, sB);
          a2 = hmul2_u32(fa1, sA);
          a3 = hmul2_u32(fb1, sB);
        }
        mma_16816(d[m], a0, a1, a2, a3, bb.x, bb.y);
      }
    }
    ++units_in_piece;

    if (b == per_group - 1 || i == n - 1) {
      float tot[NMAT];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        tot[m] = rows_to_lanes(d[m][0] + d[m][1] * (1.0f / 16777216.0f), d[m][2] + d[m][3] * (1.0f / 16777216.0f));
        d[m][0] = d[m][1] = d[m][2] = d[m][3] = 0.f;
      }
      if (units_in_piece == per_group) {
        finalize(grp, tot);  // the whole group lies in this warp's run
      } else {
        // a partial piece: the first and/or the last group of the run (at most two)
        const int k = parked_count++;
        if (lane < 16)
#pragma unroll
          for (int m = 0; m < NMAT; ++m) parked_v[((warp * 2 + k) * NMAT + m) * 16 + lane] = tot[m];
        if (lane == 0) {
          parked[warp].grp[k] = grp;
          parked[warp].units[k] = units_in_piece;
        }
      }
      units_in_piece = 0;
    }
  };

  U buf[D];
#pragma unroll
  for (int j = 0; j < PD; ++j)
    if (j < n) load(buf[j], j);
  for (int i0 = 0; i0 < n; i0 += D) {
#pragma unroll
    for (int j = 0; j < D; ++j) {
      const int i = i0 + j;
      if (i < n) {
        if (i + PD < n) load(buf[(j + PD) % D], i + PD);
        compute(buf[j], i);
      }
    }
  }
  __syncthreads();
  G4_STAMP(sc, 13);

  // CTA-level reduction of the parked pieces, one group per warp, warps in order.
  const int64_t cu0 = split_begin(int64_t(blockIdx.x) * W, n_warps, total);
  const int64_t cu1 = split_begin(int64_t(blockIdx.x + 1) * W, n_warps, total);
  if (cu1 <= cu0) return;
  const int gfirst = int(cu0 / per_group), glast = int((cu1 - 1) / per_group);
  for (int grp = gfirst + warp; grp <= glast; grp += W) {
    float tot[NMAT];
    int units = 0;
#pragma unroll
    for (int m = 0; m < NMAT; ++m) tot[m] = 0.f;
    for (int w = 0; w < W; ++w)
      for (int k = 0; k < 2; ++k)
        if (parked[w].grp[k] == grp) {
          units += parked[w].units[k];
          if (lane < 16)
#pragma unroll
            for (int m = 0; m < NMAT; ++m) tot[m] += parked_v[((w * 2 + k) * NMAT + m) * 16 + lane];
        }
    if (units == 0) continue;  // finalised inside one warp
    const int64_t gu0 = int64_t(grp) * per_group, gu1 = gu0 + per_group;
    if (gu0 >= cu0 && gu1 <= cu1) {
      finalize(grp, tot);
      continue;
    }
    // the group straddles CTAs: publish this CTA's share, the last to arrive adds them up
    const int64_t cta_first = warp_of_unit(gu0, n_warps, total) / W;
    const int64_t cta_last = warp_of_unit(gu1 - 1, n_warps, total) / W;
    if (cta_last - cta_first >= kMaxCtasPerGroup) {  // cannot happen for the shapes launched here
      if (lane == 0) atomicOr(sc.err, kErrInternal);
      continue;
    }
    float* slot = sc.partials + (size_t(grp) * kMaxCtasPerGroup + size_t(blockIdx.x - cta_first)) * NMAT * 16;
    if (lane < 16)
#pragma unroll
      for (int m = 0; m < NMAT; ++m) slot[m * 16 + lane] = tot[m];
    __syncwarp();
    uint32_t done = 0;
    if (lane == 0) {
      const uint32_t before = atomic_add_acq_rel_gpu(sc.counters + grp, uint32_t(units));
      done = before + uint32_t(units) == uint32_t(per_group);
      if (done) sc.counters[grp] = 0;
    }
    done = __shfl_sync(0xffffffffu, done, 0);
    if (!done) continue;
#pragma unroll
    for (int m = 0; m < NMAT; ++m) tot[m] = 0.f;
    for (int64_t c = cta_first; c <= cta_last; ++c) {
      const int64_t cc0 = split_begin(c * W, n_warps, total), cc1 = split_begin((c + 1) * W, n_warps, total);
      if (cc1 <= cc0) continue;  // a CTA without units
      if (lane < 16)
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
          tot[m] += ld_cg_f32(sc.partials + (size_t(grp) * kMaxCtasPerGroup + size_t(c - cta_first)) * NMAT * 16 +
                              m * 16 + lane);
    }
    finalize(grp, tot);
  }
}

}  // namespace g4
