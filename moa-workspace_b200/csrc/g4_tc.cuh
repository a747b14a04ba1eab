// Blackwell (sm_100a) building blocks of the weight-streaming engine: TMA tensor-tile loads,
// mbarriers with bounded waits, tcgen05 (TMEM allocation, kind::f8f6f4 and block-scaled
// kind::mxf4nvf4 MMA, commit, TMEM loads and stores) and the shared-memory matrix descriptors.
// No TMA multicast is used anywhere.
#pragma once

#include <cuda.h>

#include "g4_common.cuh"

namespace g4 {

// ---------------------------------------------------------------------------------------
// mbarriers shared by several roles of a CTA. A wait gives up after kWaitLimitNs or when
// another role has already given up (`abort` in shared memory), so a stalled pipeline ends
// the kernel instead of hanging the SM.

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, volatile uint32_t* abort,
                                                   uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      *abort = 1u;
      atomicOr(err, kErrWaitTimeout);
      return false;
    }
  }
  return true;
}

// Named barrier among `count` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier among `count` threads that also ORs a predicate over them: true in every
// participant if any passed true. Whole warps only.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n bar.red.or.pred po, %2, %3, pi;\n selp.u32 %0, 1, 0, po;\n}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0u;
}

// ---------------------------------------------------------------------------------------
// TMA: 2-D tensor tile -> shared memory, completing its bytes on an mbarrier. The tensor map
// is a __grid_constant__ kernel parameter. x (innermost, in elements) is always a multiple of
// the 128-element box here, so it meets the 16-byte coordinate rule for every element type.

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// TMA: 3-D tensor box -> shared memory (same rules as the 2-D form).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// TMA: bring a 3-D tensor box into L2 only.
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

// TMA: bring a 2-D tensor tile into L2 only (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------
// TMEM

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 8 / 32 consecutive columns of f32 (this warp's lane quarter).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 lanes (this warp's quarter) x 16 consecutive columns from registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------------------
// UMMA descriptors

// K-major operand in the 128-byte swizzle layout: rows of 128 bytes (128 one-byte elements, or
// 128 e2m1 codes unpacked to a byte each by the 16U4_ALIGN16B tensor map), 8-row atoms of
// 1024 bytes stacked densely (stride 1024). `saddr` is the row-0 address of the K slice: the
// 1024-aligned atom base plus 32 bytes per 32-element K step.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = uint64_t((saddr & 0x3FFFFu) >> 4);  // start address
  d |= uint64_t(1) << 16;                           // leading offset (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;                   // stride between 8-row atoms
  d |= uint64_t(1) << 46;                           // descriptor version (sm_100)
  d |= uint64_t(2) << 61;                           // SWIZZLE_128B
  return d;
}

// Byte offset of (row, byte k) inside a 1024-aligned SW128 K-major region.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t kbyte) {
  return row * 128u + ((((kbyte >> 4) ^ (row & 7u))) << 4) + (kbyte & 15u);
}

enum : uint32_t { kFmtE4M3 = 0, kFmtE2M1 = 5 };

// Instruction descriptor of tcgen05.mma kind::f8f6f4: f32 accumulate, both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f8f6f4(uint32_t afmt, uint32_t bfmt, int m, int n) {
  return (1u << 4) | (afmt << 7) | (bfmt << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_f8f6f4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor of tcgen05.mma kind::mxf4nvf4 with 16-element block scales (ue4m3):
// A and B packed e2m1, f32 accumulate, both K-major, K = 64 per instruction.
__host__ __device__ constexpr uint32_t umma_idesc_nvf4(int m, int n) {
  return (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// D[tmem] (+)= (A . SFA)[smem] * (B . SFB)[smem]^T: every 16 K elements of a row of A (B) are
// multiplied by that row's ue4m3 scale, read from TMEM at tsfa (tsfb). Issued by one thread.
__device__ __forceinline__ void umma_nvf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// Instruction descriptor of tcgen05.mma kind::f16 with bf16 A and B: f32 accumulate, both K-major,
// K = 16 per instruction.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// The same with f16 A and B.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, 16-bit operands (bf16 or f16, as the descriptor says), issued
// by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with A in tensor memory: row m of A in TMEM lane m, two 16-bit K elements per column
// (the lower one in the low half), K = 16 per instruction = 8 columns from `tmem_a`.
__device__ __forceinline__ void umma_16bit_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------------------------------
// Exact e4m3 terms of a bf16 activation.
//
// For v = x * 2^E with |v| < 256 the terms t_0 = e4m3(v), t_j = e4m3(r_j) with r_0 = v,
// r_{j+1} = (r_j - t_j) * 16 (round to nearest even each time; every r_j is exact in f32 and
// never exceeds 256) satisfy v = sum_j t_j 16^-j - r_NT 16^-NT. Each term carries 4 significant
// bits, so a bf16 value (8 bits) is exact in two terms once it is in e4m3's normal range and
// every further term extends the exact range 16x downwards: NT terms keep all of v for
// |v| >= 2^(10 - 4 NT) and leave an absolute error below 2^(-10 - 4 (NT - 1)) otherwise. The
// tensor cores contract each term exactly against the weight codes, so sum_k w_k v_k is
// reproduced to f32 accuracy even when large values cancel and tiny ones decide the result.

// Two f32 -> two e4m3 codes (round to nearest even, saturating) in the low 16 bits (lo in the
// low byte). 16-bit values stay inside the asm blocks.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint32_t r;
  asm("{\n .reg .b16 t;\n cvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n cvt.u32.u16 %0, t;\n}" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// The two e4m3 codes in the low 16 bits of `two` (low byte first) as exact f32 values.
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t two) {
  uint32_t h;
  asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %1;\n cvt.rn.f16x2.e4m3x2 %0, lo;\n}" : "=r"(h) : "r"(two));
  const __half2 hv = __halves2half2(__ushort_as_half(uint16_t(h & 0xffffu)), __ushort_as_half(uint16_t(h >> 16)));
  return __half22float2(hv);
}

// Split 16 values (already scaled by 2^E) into NT 16-byte rows of e4m3 terms (element j in
// byte j of each row).
template <int NT>
__device__ __forceinline__ void split_terms16(const float (&v)[16], uint4 (&t)[NT]) {
  uint32_t w[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) w[j][0] = w[j][1] = w[j][2] = w[j][3] = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float ra = v[2 * i], rb = v[2 * i + 1];
    const int sh = 16 * (i % 2);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const uint32_t c = f32x2_to_e4m3x2(ra, rb);
      w[j][i / 2] |= c << sh;
      if (j + 1 < NT) {  // straight-line: once a remainder is zero its further terms are zero codes
        const float2 d = e4m3x2_to_f32x2(c);
        ra = (ra - d.x) * 16.0f;
        rb = (rb - d.y) * 16.0f;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) t[j] = make_uint4(w[j][0], w[j][1], w[j][2], w[j][3]);
}

// ---------------------------------------------------------------------------------------
// Exact e2m1 digits of a bf16 activation (nvfp4 weights, kind::mxf4nvf4).
//
// An integer |X| < 2^22 is written with eight balanced base-8 digits: Y = X + 4 (8^8 - 1) / 7
// is non-negative with base-8 digits e_i, and X = sum_i (e_i - 4) 8^i. Each digit d = e - 4 in
// [-4, 3] is the e2m1 value d / 2 exactly, and the e2m1 code of d / 2 is |d| with the sign in
// bit 3. The activation element v becomes X = RN(v 2^s) for a power of two chosen per exponent
// class (the engine's B operand); the digits of 8 elements are built as nibble vectors.

constexpr uint32_t kDigitBias = 0x924924u;  // 4 (8^8 - 1) / 7

// x * 2^e for e in [-252, 254], in two exact power-of-two steps.
__device__ __forceinline__ float mul_pow2(float x, int e) {
  const int e1 = e / 2;
  return (x * pow2f(e1)) * pow2f(e - e1);
}

// Exponent P with |v| < 2^(P+1) for the magnitude `amax`: at least -127 (subnormals and zero),
// 128 for Inf / NaN.
__device__ __forceinline__ int block_exponent(float amax) {
  const int f = int((__float_as_uint(amax) >> 23) & 0xffu);
  return f == 0 ? -127 : f - 127;
}

// The eight digit codes of Y = X + kDigitBias (< 2^24): nibble i holds the code of digit i.
__device__ __forceinline__ uint32_t digit_codes8(uint32_t y) {
  uint32_t e = (y & 0x000FFFu) | ((y & 0xFFF000u) << 4);  // 12-bit halves at bits 0 and 16
  e = (e & 0x003F003Fu) | ((e & 0x0FC00FC0u) << 2);       // 6-bit quarters at bits 0, 8, 16, 24
  e = (e & 0x07070707u) | ((e & 0x38383838u) << 1);       // digit e_i in nibble i
  const uint32_t m = ((e >> 2) & 0x11111111u) * 0xFu;     // nibbles with e >= 4 (d >= 0)
  return ((e ^ 0x44444444u) & m) | (((e ^ 0xFFFFFFFFu) - 0x33333333u) & ~m);  // d, or 8 | -d
}

// 8 x 8 nibble transpose: afterwards nibble k of w[i] is what nibble i of w[k] was.
__device__ __forceinline__ void transpose8_nibbles(uint32_t (&w)[8]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t a = w[k], b = w[k + 4];
    w[k] = (a & 0x0000FFFFu) | (b << 16);
    w[k + 4] = (a >> 16) | (b & 0xFFFF0000u);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int k = (q / 2) * 4 + q % 2;  // 0, 1, 4, 5
    const uint32_t a = w[k], b = w[k + 2];
    w[k] = (a & 0x00FF00FFu) | ((b << 8) & 0xFF00FF00u);
    w[k + 2] = ((a >> 8) & 0x00FF00FFu) | (b & 0xFF00FF00u);
  }
#pragma unroll
  for (int k = 0; k < 8; k += 2) {
    const uint32_t a = w[k], b = w[k + 1];
    w[k] = (a & 0x0F0F0F0Fu) | ((b << 4) & 0xF0F0F0F0u);
    w[k + 1] = ((a >> 4) & 0x0F0F0F0Fu) | (b & 0xF0F0F0F0u);
  }
}

// sum_i d[i] 8^i, most significant digit first.
__device__ __forceinline__ float combine_digits8(const float* d) {
  float acc = d[7];
#pragma unroll
  for (int i = 6; i >= 0; --i) acc = fmaf(acc, 8.0f, d[i]);
  return acc;
}

// sum_j d[j] 16^-j, smallest term first.
template <int NT>
__device__ __forceinline__ float combine_terms(const float* d) {
  float acc = d[NT - 1];
#pragma unroll
  for (int j = NT - 2; j >= 0; --j) acc = fmaf(acc, 0.0625f, d[j]);
  return acc;
}

}  // namespace g4
