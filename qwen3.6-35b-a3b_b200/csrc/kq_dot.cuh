// kq_dot.cuh -- chunk dot products for the other block formats of the published Q4_K_M file
// (expert down Q5_K / Q6_K, shared expert Q8_0) on the decode kernels: straight from global
// memory in the gather-GEMV kernels (LdGlobal), from rows staged in shared memory in the
// persistent kernel (LdShared) -- the same arithmetic, so both paths give the same bits.
//
// Each function takes the same lane work as q4k_chunk_dot: chunk (kb, c) of a row, i.e. the 16
// elements chunk_pos(kb, c) + i ("lo") and the 16 elements 32 later ("hi"), with their x values
// in an XChunk, and returns sum_i w_i * x_i over those 32 elements in f32. The weights are the
// exact f32 values the dequantisers give (oracle/kquants.py); the sum is a plain f32 chain per
// run times the run's scale, the kernels' rounding, not a declared order.
//
// Layouts (tools/gguf_reader.py:238-333 in the reference; llama.cpp dequantize_row_*):
//   Q5_K 176 B / 256: f16 d | f16 dmin | 12 B scales+mins (Q4_K packing) | qh[32] | qs[128]
//        element e: j = e>>5, q = nibble (j&1) of qs[32(e>>6) + (e&31)] | bit j of qh[e&31] << 4
//        value (d*sc[j])*q - dmin*m[j]. Blocks 16-byte aligned (176 = 11 x 16).
//   Q6_K 210 B / 256: ql[128] | qh[64] | int8 sc[16] | f16 d
//        element e: G = e>>7, k = (e>>5)&3, l = e&31
//        q = (ql[64G + 32(k&1) + l] >> 4(k>>1)) & 15 | ((qh[32G + l] >> 2k) & 3) << 4
//        value (d*sc[e>>4])*(q - 32). Blocks only 2-byte aligned: 16-bit loads.
//   Q8_0  34 B / 32:  f16 d | int8 q[32]; value d*q. Blocks 2-byte aligned: 16-bit loads.
//   BF16  dense rows as the Hugging Face checkpoint stores them (2 B per weight, exact in f32):
//        the dense-expert layers speccheck/moe_ref.py takes; rows 16-byte aligned.
#pragma once

#include "common.cuh"

namespace b2 {

// Bytes of one row of `n` weights (n a multiple of 256) in GGML block type t (0 = Q4_K).
__host__ __device__ constexpr int64_t row_bytes(int t, int n) {
  return t == B200MOE_TYPE_BF16   ? (int64_t)n * 2
         : t == B200MOE_TYPE_Q5_K ? (int64_t)n / 256 * 176
         : t == B200MOE_TYPE_Q6_K ? (int64_t)n / 256 * 210
         : t == B200MOE_TYPE_Q8_0 ? (int64_t)n / 32 * 34
                                  : (int64_t)n / 256 * 144;
}

// The layer's block types with 0 read as Q4_K.
__host__ __device__ inline int layer_down_type(const b200moe_layer *L) {
  return L->down_type ? L->down_type : B200MOE_TYPE_Q4_K;
}
__host__ __device__ inline int layer_sh_type(const b200moe_layer *L) {
  return L->sh_type ? L->sh_type : B200MOE_TYPE_Q4_K;
}
__host__ __device__ inline int layer_gate_type(const b200moe_layer *L) {
  return L->gate_type ? L->gate_type : B200MOE_TYPE_Q4_K;
}
__host__ __device__ inline bool layer_all_q4k(const b200moe_layer *L) {
  return layer_gate_type(L) == B200MOE_TYPE_Q4_K && layer_down_type(L) == B200MOE_TYPE_Q4_K &&
         layer_sh_type(L) == B200MOE_TYPE_Q4_K;
}
// A dense layer: every expert and shared matrix in BF16 (the Hugging Face layout).
__host__ __device__ inline bool layer_dense(const b200moe_layer *L) {
  return layer_gate_type(L) == B200MOE_TYPE_BF16;
}

// Load policies: global memory (read-only, streamed: weights are read once per token) and
// shared memory (rows a kernel staged there). The arithmetic does not depend on the policy.
struct LdGlobal {
  static __device__ __forceinline__ uint4 v16(const uint8_t *p) { return ldg_stream(p); }
  static __device__ __forceinline__ uint32_t u16(const uint8_t *p) {
    return __ldg(reinterpret_cast<const unsigned short *>(p));
  }
  static __device__ __forceinline__ uint32_t u8(const uint8_t *p) { return __ldg(p); }
};
struct LdShared {
  static __device__ __forceinline__ uint4 v16(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
  static __device__ __forceinline__ uint32_t u16(const uint8_t *p) {
    return *reinterpret_cast<const unsigned short *>(p);
  }
  static __device__ __forceinline__ uint32_t u8(const uint8_t *p) { return *p; }
};

// 16 bytes from a 2-byte aligned address (eight 16-bit loads).
template <typename Ld>
__device__ __forceinline__ uint4 ld16_a2(const uint8_t *p) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = Ld::u16(p + 4 * i) | (Ld::u16(p + 4 * i + 2) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint32_t byte_of(const uint4 &v, int i) {  // byte i (0..15)
  const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
  return (w >> (8 * (i & 3))) & 0xFFu;
}

// Q5_K: block kb of the row at `row` (16-byte aligned).
template <typename Ld = LdGlobal>
__device__ __forceinline__ float q5k_chunk_dot(const uint8_t *row, int kb, int c, const XChunk &x) {
  const uint8_t *blk = row + (size_t)kb * 176;
  const uint4 h = Ld::v16(blk);
  const uint4 qh = Ld::v16(blk + 16 + 16 * (c & 1));
  const uint4 qs = Ld::v16(blk + 48 + 16 * c);
  float s0, m0, s1, m1;
  q4k_scales(h, c, s0, m0, s1, m1);  // sub-blocks 2g and 2g+1, g = c >> 1 (the Q4_K scale packing)
  const int j0 = 2 * (c >> 1);
  float al = 0.f, ah = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t b = byte_of(qs, i), hb = byte_of(qh, i);
    const uint32_t ql = (b & 15u) | (((hb >> j0) & 1u) << 4);
    const uint32_t qu = (b >> 4) | (((hb >> (j0 + 1)) & 1u) << 4);
    al = fmaf((float)ql, x.lo[i], al);
    ah = fmaf((float)qu, x.hi[i], ah);
  }
  return fmaf(s0, al, -m0 * x.slo) + fmaf(s1, ah, -m1 * x.shi);
}

// Q6_K: block kb of the row at `row` (2-byte aligned).
template <typename Ld = LdGlobal>
__device__ __forceinline__ float q6k_chunk_dot(const uint8_t *row, int kb, int c, const XChunk &x) {
  const uint8_t *blk = row + (size_t)kb * 210;
  const int g = c >> 1, G = g >> 1, l0 = 16 * (c & 1), sh = 4 * (g & 1);
  const uint4 qlo = ld16_a2<Ld>(blk + 64 * G + l0);       // k = 2(g&1): ql[64G + l], nibble g&1
  const uint4 qhi = ld16_a2<Ld>(blk + 64 * G + 32 + l0);  // k = 2(g&1)+1: ql[64G + 32 + l]
  const uint4 qh = ld16_a2<Ld>(blk + 128 + 32 * G + l0);  // bits 2k, 2k+1 of qh[32G + l]
  const float d = f16f(Ld::u16(blk + 208));
  const float s_lo = d * (float)(int8_t)Ld::u8(blk + 192 + 4 * g + (c & 1));  // sc[e >> 4], exact
  const float s_hi = d * (float)(int8_t)Ld::u8(blk + 192 + 4 * g + 2 + (c & 1));
  float al = 0.f, ah = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t hb = byte_of(qh, i);
    const int ql = (int)(((byte_of(qlo, i) >> sh) & 15u) | (((hb >> sh) & 3u) << 4)) - 32;
    const int qu = (int)(((byte_of(qhi, i) >> sh) & 15u) | (((hb >> (sh + 2)) & 3u) << 4)) - 32;
    al = fmaf((float)ql, x.lo[i], al);
    ah = fmaf((float)qu, x.hi[i], ah);
  }
  return fmaf(s_lo, al, s_hi * ah);
}

// Q8_0: the chunk's lo run is positions l0..l0+15 of block 8kb + 2g, its hi run the same
// positions of the next block (row 2-byte aligned).
template <typename Ld = LdGlobal>
__device__ __forceinline__ float q80_chunk_dot(const uint8_t *row, int kb, int c, const XChunk &x) {
  const int b0 = 8 * kb + 2 * (c >> 1), l0 = 16 * (c & 1);
  const uint8_t *p0 = row + (size_t)b0 * 34, *p1 = p0 + 34;
  const float d0 = f16f(Ld::u16(p0)), d1 = f16f(Ld::u16(p1));
  const uint4 q0 = ld16_a2<Ld>(p0 + 2 + l0), q1 = ld16_a2<Ld>(p1 + 2 + l0);
  float al = 0.f, ah = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    al = fmaf((float)(int8_t)byte_of(q0, i), x.lo[i], al);
    ah = fmaf((float)(int8_t)byte_of(q1, i), x.hi[i], ah);
  }
  return fmaf(d0, al, d1 * ah);
}

// BF16: the chunk's lo run is the 16 weights at chunk_pos(kb, c), its hi run the 16 weights 32
// later; each run is one 32-byte read (two 16-byte loads), a plain f32 FMA chain per run.
template <typename Ld = LdGlobal>
__device__ __forceinline__ float bf16_chunk_dot(const uint8_t *row, int kb, int c, const XChunk &x) {
  const uint8_t *p = row + (size_t)chunk_pos(kb, c) * 2;
  const uint4 l0 = Ld::v16(p), l1 = Ld::v16(p + 16), h0 = Ld::v16(p + 64), h1 = Ld::v16(p + 80);
  const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
  const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  float al = 0.f, ah = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    al = fmaf(bf16f(lw[i]), x.lo[2 * i], al);
    al = fmaf(bf16f(lw[i] >> 16), x.lo[2 * i + 1], al);
    ah = fmaf(bf16f(hw[i]), x.hi[2 * i], ah);
    ah = fmaf(bf16f(hw[i] >> 16), x.hi[2 * i + 1], ah);
  }
  return al + ah;
}

// Q4_K through a load policy (the same arithmetic as q4k_chunk_dot on registers).
template <typename Ld = LdGlobal>
__device__ __forceinline__ float q4k_row_chunk_dot(const uint8_t *row, int kb, int c, const XChunk &x) {
  const uint4 h = Ld::v16(row + (size_t)kb * kQB), q = Ld::v16(row + (size_t)kb * kQB + 16 + 16 * c);
  return q4k_chunk_dot(h, q, c, x);
}

// Chunk (kb, c) of a row in a block type known only at run time (warp-uniform).
template <typename Ld>
__device__ __forceinline__ float any_chunk_dot(int type, const uint8_t *row, int kb, int c, const XChunk &x) {
  if (type == B200MOE_TYPE_Q5_K) return q5k_chunk_dot<Ld>(row, kb, c, x);
  if (type == B200MOE_TYPE_Q6_K) return q6k_chunk_dot<Ld>(row, kb, c, x);
  if (type == B200MOE_TYPE_Q8_0) return q80_chunk_dot<Ld>(row, kb, c, x);
  if (type == B200MOE_TYPE_BF16) return bf16_chunk_dot<Ld>(row, kb, c, x);
  return q4k_row_chunk_dot<Ld>(row, kb, c, x);
}

// Chunk (kb, c) of a row stored in block type kT (B200MOE_TYPE_*), loads included.
template <int kT>
__device__ __forceinline__ float row_chunk_dot(const uint8_t *row, int kb, int c, const XChunk &x) {
  if constexpr (kT == B200MOE_TYPE_Q5_K) return q5k_chunk_dot(row, kb, c, x);
  else if constexpr (kT == B200MOE_TYPE_Q6_K) return q6k_chunk_dot(row, kb, c, x);
  else if constexpr (kT == B200MOE_TYPE_Q8_0) return q80_chunk_dot(row, kb, c, x);
  else if constexpr (kT == B200MOE_TYPE_BF16) return bf16_chunk_dot(row, kb, c, x);
  else return q4k_row_chunk_dot(row, kb, c, x);
}

}  // namespace b2
