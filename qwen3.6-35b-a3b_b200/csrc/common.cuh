// common.cuh -- device helpers shared by every b200moe kernel (sm_100a).
//
// Q4_K super-block (144 B / 256 weights): {f16 d, f16 dmin, u8 scales[12], u8 qs[128]}.
// A "chunk" is one 16-byte slice of qs: chunk c (0..7) holds bytes 16c..16c+15, i.e. for
// g = c>>1 and l0 = 16*(c&1) the low nibbles of elements 64g+l0 .. 64g+l0+15 (sub-block 2g)
// and the high nibbles of elements 64g+32+l0 .. +15 (sub-block 2g+1)
// (element order: reference tools/gguf_reader.py:33-37).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b200moe.h"

namespace b2 {

constexpr int kH = 2048;   // hidden
constexpr int kE = 256;    // routed experts
constexpr int kK = 8;      // top-k
constexpr int kI = 512;    // expert / shared intermediate
constexpr int kQB = 144;   // Q4_K block bytes
constexpr int kRowUp = kH / 256 * kQB;    // 1152 B: one gate/up row (2048 weights)
constexpr int kRowDown = kI / 256 * kQB;  // 288 B: one down row (512 weights)

// ---------------------------------------------------------------- scalar conversions
__device__ __forceinline__ float bf16f(uint32_t b) { return __uint_as_float((b & 0xFFFFu) << 16); }

__device__ __forceinline__ uint16_t f2bf(float f) {  // RNE, canonical NaN
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float bf16r(float f) {  // f rounded to bf16 precision (RNE), as f32
  return __uint_as_float((uint32_t)f2bf(f) << 16);
}

__device__ __forceinline__ float f16f(uint32_t h) {  // exact widening
  return __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
}

__device__ __forceinline__ float pow2i(int n) { return __uint_as_float((uint32_t)(n + 127) << 23); }

// The library's own exp (identical operation sequence to oracle/c/oracle.c b2o_expf):
// Cody-Waite two-constant reduction x = n*ln2 + r, degree-7 Taylor polynomial in Horner
// form (J.-M. Muller, "Elementary Functions", ch. 11). IEEE basic ops only, so the host
// restatement reproduces it bit for bit; used where the router's result must be exact.
__device__ __forceinline__ float b2_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7F800000);
  if (x < -103.97208404541016f) return 0.0f;
  const float t = __fmul_rn(x, 1.44269502162933349609375f);
  const float n = rintf(t);
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.428606765330187045e-06f, r);
  float p = 1.984126984126984e-04f;
  p = __fmaf_rn(p, r, 1.388888888888889e-03f);
  p = __fmaf_rn(p, r, 8.333333333333333e-03f);
  p = __fmaf_rn(p, r, 4.166666666666667e-02f);
  p = __fmaf_rn(p, r, 1.666666666666667e-01f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = (int)n;
  if (ni > 127) return __fmul_rn(__fmul_rn(p, pow2i(127)), 2.0f);
  if (ni < -126) return __fmul_rn(__fmul_rn(p, pow2i(ni + 64)), pow2i(-64));
  return __fmul_rn(p, pow2i(ni));
}

__device__ __forceinline__ float silu_f(float z) { return __fdiv_rn(z, __fadd_rn(1.0f, expf(-z))); }

// ---------------------------------------------------------------- memory
// L2 policy for streamed weights: evict first, so the ~640 MB of Q4_K a decoded token reads
// does not push code, activations and the router rows out of the 126 MB L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Streaming 16-byte read-only load: no L1 allocation, L2 evict-first (weights are touched once).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p), "l"(l2_evict_first()));
  return r;
}

__device__ __forceinline__ float4 ldg_f4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// Bulk L2 prefetch of [p, p+bytes) (bytes a multiple of 16, p 16-byte aligned).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the previous grid's results / let the next one start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ float half_warp_sum(float v) {  // sums within lanes 0-15 / 16-31
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// ---------------------------------------------------------------- Q4_K chunk decoding
// x values a lane needs for one chunk: the 16 low-nibble positions and the 16 high-nibble
// positions, plus their sums (the min term of a sub-block is -dmin*m * sum(x)).
struct XChunk {
  float lo[16];
  float hi[16];
  float slo, shi;
};

// Position (within a 2048- or 512-long row) of the first low-nibble element of chunk c of
// block kb; the high run starts 32 elements later.
__device__ __forceinline__ int chunk_pos(int kb, int c) { return kb * 256 + 64 * (c >> 1) + 16 * (c & 1); }

// get_scale_min_k4 for the two sub-blocks of chunk c (2g and 2g+1), folded with d / dmin.
// hdr.x = d | dmin<<16, hdr.y/z/w = scale bytes 0-3 / 4-7 / 8-11. Byte-parallel: one word holds
// the four 6-bit scales (or mins) of sub-blocks 0-3 or 4-7 -- for j < 4, q[j] & 63 and
// q[j+4] & 63; for j >= 4, (q[j+4] & 15) | (q[j-4] >> 6) << 4 and (q[j+4] >> 4) | (q[j] >> 6) << 4
// -- so a chunk's two values are bytes 2(g&1) and 2(g&1)+1 of the word its half selects.
__device__ __forceinline__ void q4k_scales(const uint4 &h, int c, float &s0, float &m0, float &s1,
                                           float &m1) {
  const float d = f16f(h.x), dmin = f16f(h.x >> 16);
  const int g = c >> 1;
  const uint32_t sc = g < 2 ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
  const uint32_t mn = g < 2 ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
  const int sh = 16 * (g & 1);
  s0 = d * (float)((sc >> sh) & 0xFFu);
  m0 = dmin * (float)((mn >> sh) & 0xFFu);
  s1 = d * (float)((sc >> (sh + 8)) & 0xFFu);
  m1 = dmin * (float)((mn >> (sh + 8)) & 0xFFu);
}

// 4-bit value of byte b (0..3) of a nibble-masked word, as an exact float: 0x4B0000qq is
// 2^23 + q, so subtracting 2^23 leaves q. (Used where the result must be bit-exact.)
__device__ __forceinline__ float nib_f(uint32_t masked, int b) {
  return __uint_as_float(__byte_perm(masked, 0x4B000000u, 0x7540u | (uint32_t)b)) - 8388608.0f;
}

// 1 + q/16 for byte b of a prepared word whose bytes are 0x80 | (q << 3): one byte permute
// builds the float 0x3F8?0000 directly (mantissa bits 19..22 = q).
__device__ __forceinline__ float nib_1p(uint32_t prepared, int b) {
  return __uint_as_float(__byte_perm(prepared, 0x3F000000u, 0x7054u | ((uint32_t)b << 8)));
}

// sum over the chunk's 32 weights of w_i * x_i, with w = (d*sc)*q - dmin*m. The quants enter
// as f = 1 + q/16 (one byte permute each): sum(q x) = 16 (sum(f x) - sum(x)), so a run's
// contribution is 16*S*sum(f x) - (16*S + M) * sum(x). Each 16-element run is accumulated in
// two interleaved chains (words 0-1 and 2-3, added at the end) to halve the dependent latency.
__device__ __forceinline__ float q4k_chunk_dot(const uint4 &h, const uint4 &q, int c, const XChunk &x) {
  float s0, m0, s1, m1;
  q4k_scales(h, c, s0, m0, s1, m1);
  float al0 = 0.f, ah0 = 0.f, al1 = 0.f, ah1 = 0.f;
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t lo0 = ((w[i] << 3) & 0x78787878u) | 0x80808080u;
    const uint32_t hi0 = ((w[i] >> 1) & 0x78787878u) | 0x80808080u;
    const uint32_t lo1 = ((w[i + 2] << 3) & 0x78787878u) | 0x80808080u;
    const uint32_t hi1 = ((w[i + 2] >> 1) & 0x78787878u) | 0x80808080u;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      al0 = fmaf(nib_1p(lo0, b), x.lo[4 * i + b], al0);
      ah0 = fmaf(nib_1p(hi0, b), x.hi[4 * i + b], ah0);
      al1 = fmaf(nib_1p(lo1, b), x.lo[4 * (i + 2) + b], al1);
      ah1 = fmaf(nib_1p(hi1, b), x.hi[4 * (i + 2) + b], ah1);
    }
  }
  const float al = al0 + al1, ah = ah0 + ah1;
  const float S0 = 16.0f * s0, S1 = 16.0f * s1;
  return fmaf(S0, al, -(S0 + m0) * x.slo) + fmaf(S1, ah, -(S1 + m1) * x.shi);
}

// Load the x values of chunk (kb, c) from a dense f32 row.
__device__ __forceinline__ void load_xchunk(const float *row, int kb, int c, XChunk &x) {
  const int p = chunk_pos(kb, c);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 a = ldg_f4(row + p + 4 * i);
    const float4 b = ldg_f4(row + p + 32 + 4 * i);
    x.lo[4 * i] = a.x; x.lo[4 * i + 1] = a.y; x.lo[4 * i + 2] = a.z; x.lo[4 * i + 3] = a.w;
    x.hi[4 * i] = b.x; x.hi[4 * i + 1] = b.y; x.hi[4 * i + 2] = b.z; x.hi[4 * i + 3] = b.w;
  }
  float sl = 0.f, sh = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) { sl += x.lo[i]; sh += x.hi[i]; }
  x.slo = sl;
  x.shi = sh;
}

}  // namespace b2

// ---------------------------------------------------------------- host-side error plumbing
namespace b2host {
int set_error(int code, const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);
}  // namespace b2host

#define B2_CUDA(call)                                                   \
  do {                                                                  \
    cudaError_t e_ = (call);                                            \
    if (e_ != cudaSuccess) return b2host::cuda_status(e_, #call);       \
  } while (0)
