// imma.cuh -- exact-product int8 tensor-core pieces of the Q4_K expert dots (sm_100a, mma.sync).
//
// A Q4_K dot runs as int8 MMAs over the raw 4-bit quants (A, 0..15) and a fixed-point image of
// the vector v (B):
//   * v is scaled by 2^k, k = 21 - floor(log2 max|v|) (digit_shift), and rounded to integers
//     |n| <= 2^22, split exactly into three signed base-256 digits n = 65536 d0 + 256 d1 + d2
//     (digits3: d1, d2 in [-128, 127], |d0| <= 64), each digit plane one B column;
//   * one m16n8k32 MMA covers one 32-element sub-block of 16 rows, so each result is the exact
//     integer sum(q * digit) of a sub-block; callers multiply it by the sub-block's 6-bit scale,
//     accumulate the super-block in int32 (|sum| < 2^31), convert once per super-block and
//     multiply by d; the min term -dmin * m * sum(n) uses the exact integer sums of n per
//     sub-block; the result is scaled back by 2^-k (digit_unscale).
// Against the real-valued dot the only roundings are v's (2^-23 of max|v|) and the final f32
// combine; every value is a deterministic function of the row and v.
//
// Fragment layout (PTX ISA, mma.m16n8k32 .s8): lane = 4 g + t holds A rows g and g + 8 at
// k = 4t..4t+3 (registers 0 / 1) and k = 16+4t..16+4t+3 (registers 2 / 3), B column g at the
// same k, and D rows g / g + 8 at columns 2t, 2t+1. The callers map k to the elements of a
// sub-block so that a lane's A bytes are 8 consecutive quant bytes of a row (8t..8t+7 of a
// 32-byte group): k = 4t + i is element 8t + i and k = 16 + 4t + i element 8t + 4 + i.
#pragma once

#include "common.cuh"

namespace b2 {

// D = A * B with a zero accumulator.
__device__ __forceinline__ void mma_s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                                       int (&d)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// k for a vector whose largest magnitude has the f32 bits `mbits` (|v| * 2^k < 2^22 for all v).
__device__ __forceinline__ int digit_shift(uint32_t mbits) {
  if (mbits == 0u || mbits >= 0x7F800000u) return 0;
  const int k = 21 - ((int)(mbits >> 23) - 127);
  return k > 126 ? 126 : k;
}

// 2^-k, or NaN when the vector holds an inf or a NaN (every dot over it is then NaN).
__device__ __forceinline__ float digit_unscale(uint32_t mbits, int k) {
  return mbits >= 0x7F800000u ? __int_as_float(0x7FC00000) : pow2i(-k);
}

// n = 65536 d0 + 256 d1 + d2 with d1, d2 in [-128, 127] (exact for |n| <= 2^22: |d0| <= 64).
// No intermediate overflows for any int n (garbage digits then only follow a NaN scale).
__device__ __forceinline__ void digits3(int n, int &d0, int &d1, int &d2) {
  d2 = n & 255;
  d2 -= (d2 & 128) << 1;
  const int r = (n >> 8) + ((n >> 7) & 1);
  d1 = r & 255;
  d1 -= (d1 & 128) << 1;
  d0 = (r >> 8) + ((r >> 7) & 1);
}

// The 6-bit scales (sc) and mins (mn) of a Q4_K super-block header h (h.y / h.z / h.w = scale
// bytes 0-3 / 4-7 / 8-11), byte-parallel get_scale_min_k4: byte i of lo is sub-block i, of hi
// sub-block 4 + i.
struct Q4kScales {
  uint32_t sc_lo, sc_hi, mn_lo, mn_hi;
};
__device__ __forceinline__ Q4kScales q4k_scale_words(const uint4 &h) {
  Q4kScales s;
  s.sc_lo = h.y & 0x3F3F3F3Fu;
  s.sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  s.mn_lo = h.z & 0x3F3F3F3Fu;
  s.mn_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  return s;
}

// Sub-block s (0..7) scale / min of a Q4kScales.
__device__ __forceinline__ int q4k_sc(const Q4kScales &s, int sb) {
  return (int)(((sb < 4 ? s.sc_lo : s.sc_hi) >> (8 * (sb & 3))) & 0xFFu);
}
__device__ __forceinline__ int q4k_mn(const Q4kScales &s, int sb) {
  return (int)(((sb < 4 ? s.mn_lo : s.mn_hi) >> (8 * (sb & 3))) & 0xFFu);
}

__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }

}  // namespace b2
