// Weight-streaming split-K GEMV engine shared by every projection of the decode layer.
//
// Work unit ("chunk"): 16 consecutive weight rows x KC consecutive K elements. The flat
// sequence of G row-groups x C chunks is split evenly across all warps of the grid; each
// warp streams its chunks through a private ring of S shared-memory slots filled by TMA
// bulk copies (one copy per row and per array, padded row stride so the fragment loads are
// bank-conflict free), converts the codes to exact f16 in registers and contracts them on
// the tensor pipe with mma.m16n8k16 (f32 accumulate) against the activation held in
// shared memory as two exact f16 columns (hi, lo). A warp flushes one partial row sum per
// group piece it covered; the warp that completes a group (ticket per group) adds the
// pieces in chunk order, so the result does not depend on timing.
#pragma once

#include "g4_common.cuh"

namespace g4 {

enum class WFmt { kFp8, kNvfp4 };

// Per-slot layout of one weight array family.
template <WFmt F, int NMAT, int KC>
struct SlotLayout {
  static_assert(KC % 64 == 0, "chunk must hold whole 64-element segments");
  static constexpr bool kFp4 = (F == WFmt::kNvfp4);
  static_assert(!kFp4 || KC % 256 == 0, "an NVFP4 chunk must carry whole 16-byte scale runs");
  static constexpr int kCodeBytes = kFp4 ? KC / 2 : KC;          // per row per matrix
  static constexpr int kScaleBytes = kFp4 ? KC / 16 : 0;         // per row per matrix
  static constexpr int kMatBytes = kCodeBytes + kScaleBytes;     // both multiples of 16
  static constexpr int kRawRow = NMAT * kMatBytes;
  // Row stride: 64 mod 128 for fp8 (16-byte fragment loads of two rows per quarter warp),
  // 32 or 96 mod 128 for fp4 (8-byte loads of four rows per half warp).
  static constexpr int pad_row(int raw) {
    int r = (raw + 15) / 16 * 16;
    while (kFp4 ? ((r % 128) != 32 && (r % 128) != 96) : ((r % 128) != 64)) r += 16;
    return r;
  }
  static constexpr int kRowBytes = pad_row(kRawRow);
  static constexpr int kSlotBytes = 16 * kRowBytes;
  static constexpr uint32_t kTxBytes = 16u * NMAT * kMatBytes;
  static constexpr int kSegs = KC / 64;
};

// Byte stride between the hi and lo activation columns in shared memory (k elements).
__host__ __device__ constexpr int act_col_stride(int k) { return k * 2 + 16; }

// Fill the two f16 activation columns from bf16 values h (per-element callback), scaled by
// 2^e so that max|h| lands in [2^14, 2^15): hi = f16(h 2^e), lo = f16((h 2^e - hi) 2^24).
// Both are exact for every bf16 value within a 2^29 ratio of the maximum, so the tensor-op
// product reproduces the f32 dot product of the bf16 activation with the exact weights.
// Returns 2^-e, the factor that undoes the scaling.
template <class HFn>
__device__ float build_act_columns(uint8_t* cols, int k, HFn h_of, float* red_f) {
  float amax = 0.f;
  for (int i = threadIdx.x; i < k; i += blockDim.x) amax = fmaxf(amax, fabsf(h_of(i)));
  amax = block_max(amax, red_f);
  int e = 0;
  if (amax > 0.f) {
    const int ex = int((__float_as_uint(amax) >> 23) & 0xff) - 127;
    e = 14 - ex;
    e = e > 126 ? 126 : (e < -126 ? -126 : e);
  }
  const float up = pow2f(e);
  const int cs = act_col_stride(k);
  __half* hi = reinterpret_cast<__half*>(cols);
  __half* lo = reinterpret_cast<__half*>(cols + cs);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const float v = h_of(i) * up;
    const __half vh = __float2half_rn(v);
    hi[i] = vh;
    lo[i] = __float2half_rn((v - __half2float(vh)) * 16777216.0f);
  }
  return pow2f(-e);
}

// One split-K GEMV pass over a warp's chunk range.
//   rows_of(group, mat)  -> pointer to the group's first row of matrix `mat` (codes)
//   scales_of(group,mat) -> pointer to the group's first row of scales (NVFP4 only)
//   flush(group, cstart, v) with v[mat*16 + row] the piece's f32 row sums (lanes 0..15 hold row=lane)
template <WFmt F, int NMAT, int KC, int S, class RowsFn, class ScalesFn, class FlushFn>
__device__ void stream_gemv(uint8_t* slots, uint64_t* bars, const uint8_t* act_cols, int k_total,
                            int64_t warp_id, int64_t n_warps, int groups, int row_bytes_global,
                            int scale_bytes_global, RowsFn rows_of, ScalesFn scales_of, FlushFn flush,
                            uint32_t* err, bool prefilled) {
  using Lay = SlotLayout<F, NMAT, KC>;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int C = k_total / KC;
  const int64_t total = int64_t(groups) * C;
  const int64_t q0 = split_begin(warp_id, n_warps, total);
  const int64_t q1 = split_begin(warp_id + 1, n_warps, total);
  const int nq = int(q1 - q0);
  const uint64_t policy = l2_evict_first_policy();
  const int cs = act_col_stride(k_total);

  auto issue = [&](int i) {  // chunk q0+i into slot i % S
    const int64_t q = q0 + i;
    const int grp = int(q / C), c = int(q % C);
    uint8_t* slot = slots + (i % S) * Lay::kSlotBytes;
    uint64_t* bar = bars + (i % S);
    if (lane == 0) mbar_arrive_expect_tx(bar, Lay::kTxBytes);
    __syncwarp();
    if (lane < 16) {
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        const uint8_t* src = rows_of(grp, m) + size_t(lane) * row_bytes_global + size_t(c) * Lay::kCodeBytes;
        bulk_g2s(slot + lane * Lay::kRowBytes + m * Lay::kMatBytes, src, Lay::kCodeBytes, bar, policy);
        if constexpr (Lay::kFp4) {
          const uint8_t* ssrc = scales_of(grp, m) + size_t(lane) * scale_bytes_global + size_t(c) * Lay::kScaleBytes;
          bulk_g2s(slot + lane * Lay::kRowBytes + m * Lay::kMatBytes + Lay::kCodeBytes, ssrc, Lay::kScaleBytes, bar,
                   policy);
        }
      }
    }
  };

  if (!prefilled) {
    for (int i = 0; i < S && i < nq; ++i) issue(i);
  }

  float d[NMAT][4];
#pragma unroll
  for (int m = 0; m < NMAT; ++m) d[m][0] = d[m][1] = d[m][2] = d[m][3] = 0.f;
  int cstart = nq > 0 ? int(q0 % C) : 0;

  for (int i = 0; i < nq; ++i) {
    const int64_t q = q0 + i;
    const int grp = int(q / C), c = int(q % C);
    if (!mbar_wait(bars + (i % S), uint32_t((i / S) & 1), err)) return;
    const uint8_t* slot = slots + (i % S) * Lay::kSlotBytes;
    const uint8_t* ra = slot + g * Lay::kRowBytes;
    const uint8_t* rb = slot + (g + 8) * Lay::kRowBytes;
    const uint8_t* bcol = act_cols + (g & 1) * cs + size_t(c) * KC * 2 + t * 32;
    const bool bact = g < 2;
#pragma unroll 2
    for (int s = 0; s < Lay::kSegs; ++s) {
      uint4 b01 = make_uint4(0, 0, 0, 0), b23 = make_uint4(0, 0, 0, 0);
      if (bact) {
        b01 = *reinterpret_cast<const uint4*>(bcol + s * 128);
        b23 = *reinterpret_cast<const uint4*>(bcol + s * 128 + 16);
      }
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        if constexpr (!Lay::kFp4) {
          const uint4 wa = *reinterpret_cast<const uint4*>(ra + m * Lay::kMatBytes + s * 64 + t * 16);
          const uint4 wb = *reinterpret_cast<const uint4*>(rb + m * Lay::kMatBytes + s * 64 + t * 16);
          const uint32_t wa_[4] = {wa.x, wa.y, wa.z, wa.w};
          const uint32_t wb_[4] = {wb.x, wb.y, wb.z, wb.w};
          const uint32_t bb[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            mma_16816(d[m], cvt_e4m3x2_f16x2(uint16_t(wa_[j] & 0xffff)), cvt_e4m3x2_f16x2(uint16_t(wb_[j] & 0xffff)),
                      cvt_e4m3x2_f16x2(uint16_t(wa_[j] >> 16)), cvt_e4m3x2_f16x2(uint16_t(wb_[j] >> 16)), bb[2 * j],
                      bb[2 * j + 1]);
          }
        } else {
          const uint8_t* ma = ra + m * Lay::kMatBytes;
          const uint8_t* mb = rb + m * Lay::kMatBytes;
          const uint2 ca = *reinterpret_cast<const uint2*>(ma + s * 32 + t * 8);
          const uint2 cb = *reinterpret_cast<const uint2*>(mb + s * 32 + t * 8);
          const uint16_t sab = uint16_t(ma[Lay::kCodeBytes + s * 4 + t]) | (uint16_t(mb[Lay::kCodeBytes + s * 4 + t]) << 8);
          const uint32_t sc = cvt_e4m3x2_f16x2(sab);
          const uint32_t sA = (sc & 0xffffu) * 0x10001u, sB = (sc >> 16) * 0x10001u;
          uint32_t fa[8], fb[8];
          cvt_e2m1x8_f16x2(ca.x, fa[0], fa[1], fa[2], fa[3]);
          cvt_e2m1x8_f16x2(ca.y, fa[4], fa[5], fa[6], fa[7]);
          cvt_e2m1x8_f16x2(cb.x, fb[0], fb[1], fb[2], fb[3]);
          cvt_e2m1x8_f16x2(cb.y, fb[4], fb[5], fb[6], fb[7]);
          const uint32_t bb[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            mma_16816(d[m], hmul2_u32(fa[2 * j], sA), hmul2_u32(fb[2 * j], sB), hmul2_u32(fa[2 * j + 1], sA),
                      hmul2_u32(fb[2 * j + 1], sB), bb[2 * j], bb[2 * j + 1]);
          }
        }
      }
    }

    const bool last_of_group = (c == C - 1) || (i == nq - 1);
    if (last_of_group) {
      // lanes (g, t=0) hold rows g and g+8: hi in columns 0, lo in column 1
      float v[NMAT][2];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        v[m][0] = d[m][0] + d[m][1] * (1.0f / 16777216.0f);
        v[m][1] = d[m][2] + d[m][3] * (1.0f / 16777216.0f);
        d[m][0] = d[m][1] = d[m][2] = d[m][3] = 0.f;
      }
      flush(grp, cstart, c - cstart + 1, v);
      cstart = 0;
    }
    __syncwarp();
    if (i + S < nq) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(i + S);
    }
  }
}

// Issue the first S chunks of a warp's range (lets a kernel start streaming weights before
// it waits for the previous kernel's activations).
template <WFmt F, int NMAT, int KC, int S, class RowsFn, class ScalesFn>
__device__ void stream_prefill(uint8_t* slots, uint64_t* bars, int k_total, int64_t warp_id, int64_t n_warps,
                               int groups, int row_bytes_global, int scale_bytes_global, RowsFn rows_of,
                               ScalesFn scales_of) {
  using Lay = SlotLayout<F, NMAT, KC>;
  const int lane = threadIdx.x & 31;
  const int C = k_total / KC;
  const int64_t total = int64_t(groups) * C;
  const int64_t q0 = split_begin(warp_id, n_warps, total);
  const int64_t q1 = split_begin(warp_id + 1, n_warps, total);
  const int nq = int(q1 - q0);
  const uint64_t policy = l2_evict_first_policy();
  for (int i = 0; i < S && i < nq; ++i) {
    const int64_t q = q0 + i;
    const int grp = int(q / C), c = int(q % C);
    uint8_t* slot = slots + i * Lay::kSlotBytes;
    uint64_t* bar = bars + i;
    if (lane == 0) mbar_arrive_expect_tx(bar, Lay::kTxBytes);
    __syncwarp();
    if (lane < 16) {
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        const uint8_t* src = rows_of(grp, m) + size_t(lane) * row_bytes_global + size_t(c) * Lay::kCodeBytes;
        bulk_g2s(slot + lane * Lay::kRowBytes + m * Lay::kMatBytes, src, Lay::kCodeBytes, bar, policy);
        if constexpr (Lay::kFp4) {
          const uint8_t* ssrc = scales_of(grp, m) + size_t(lane) * scale_bytes_global + size_t(c) * Lay::kScaleBytes;
          bulk_g2s(slot + lane * Lay::kRowBytes + m * Lay::kMatBytes + Lay::kCodeBytes, ssrc, Lay::kScaleBytes, bar,
                   policy);
        }
      }
    }
  }
}

// Sum the split-K pieces of one group in chunk order. Lanes 0..15 return row `lane` of
// matrix `mat`; pieces live at partials[((grp*C + cstart) * NMAT + mat) * 16 + row].
template <int NMAT>
__device__ float gather_group(const float* partials, int grp, int C, int mat, int64_t n_warps, int64_t total) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  if (lane < 16) {
    for (int c = 0; c < C; ++c) {
      const int64_t q = int64_t(grp) * C + c;
      if (c == 0 || is_range_start(q, n_warps, total))
        acc += ld_cg_f32(partials + ((size_t(grp) * C + c) * NMAT + mat) * 16 + lane);
    }
  }
  return acc;
}

// Store a piece, then take the group ticket. Returns true in every lane of the warp that
// completed the group (it must then run the group epilogue and reset the counter).
template <int NMAT>
__device__ bool flush_piece(float* partials, uint32_t* counter, int grp, int C, int cstart, int nchunks,
                            const float (&v)[NMAT][2]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (t == 0) {
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      float* p = partials + ((size_t(grp) * C + cstart) * NMAT + m) * 16;
      p[g] = v[m][0];
      p[g + 8] = v[m][1];
    }
  }
  __threadfence();  // every writer releases its piece before the ticket is taken
  __syncwarp();
  uint32_t done = 0;
  if (lane == 0) {
    const uint32_t before = atomicAdd(counter, uint32_t(nchunks));
    done = (before + uint32_t(nchunks) == uint32_t(C)) ? 1u : 0u;
  }
  done = __shfl_sync(0xffffffffu, done, 0);
  if (done) __threadfence();  // acquire side: the pieces of the other warps are visible
  return done != 0;
}

}  // namespace g4
