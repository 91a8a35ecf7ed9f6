// kquant.cu -- Q5_K / Q6_K / Q8_0 block decoders: the other block formats of the published
// Q4_K_M file (expert down matrices Q5_K and Q6_K, the shared expert Q8_0), as stand-alone
// dequantisation into f32 or bf16 (b200moe_dequant).
//
// Layouts (llama.cpp dequantize_row_q5_K / q6_K / q8_0, as the reference transcribes them in
// tools/gguf_reader.py:238-333 and tools/gguf_fast_dequant.py:109-150):
//   Q8_0  34 B / 32:  f16 d | int8 q[32]                                  v = d * q
//   Q5_K 176 B / 256: f16 d | f16 dmin | 12 B scales+mins | qh[32] | qs[128]
//                     e: j = e>>5, q = (qs[32(e>>6) + (e&31)] >> 4(j&1)) & 15 | bit j of qh[e&31] << 4
//                     v = (d*sc[j])*q - dmin*m[j]
//   Q6_K 210 B / 256: ql[128] | qh[64] | int8 sc[16] | f16 d
//                     e: g = e>>7, k = (e>>5)&3, l = e&31
//                     q = (ql[64g + 32(k&1) + l] >> 4(k>>1)) & 15 | ((qh[32g + l] >> 2k) & 3) << 4
//                     v = (d*sc[e>>4])*(q - 32)
// Every product is exact in f32, so each value is the single rounding of the reference's f64
// expression (Q5_K: one fmaf; Q6_K and Q8_0: exact).
#include "common.cuh"

using namespace b2;

namespace {

template <bool kBF16>
__device__ __forceinline__ void store16(void *out, int64_t e0, const float (&v)[16]) {
  if (kBF16) {
    uint32_t p[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = (uint32_t)f2bf(v[2 * i]) | ((uint32_t)f2bf(v[2 * i + 1]) << 16);
    uint4 *o = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) + e0);
    o[0] = make_uint4(p[0], p[1], p[2], p[3]);
    o[1] = make_uint4(p[4], p[5], p[6], p[7]);
  } else {
    float4 *o = reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + e0);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

__device__ __forceinline__ float f16_at(const uint8_t *p) {
  return f16f((uint32_t)p[0] | ((uint32_t)p[1] << 8));
}

// One thread per 16 consecutive elements (16 threads per super-block, 2 per Q8_0 block).
template <bool kBF16>
__global__ void __launch_bounds__(256) k_q5k_dequant(const uint8_t *__restrict__ blocks, int64_t nblocks,
                                                     void *__restrict__ out) {
  for (int64_t tid = (int64_t)blockIdx.x * 256 + threadIdx.x; tid < nblocks * 16; tid += (int64_t)gridDim.x * 256) {
    const int64_t b = tid >> 4;
    const int part = (int)(tid & 15), j = part >> 1, h = part & 1;  // sub-block j, elements 16h..16h+15
    const uint8_t *blk = blocks + b * 176;
    const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
    float s0, m0, s1, m1;
    q4k_scales(hdr, 2 * (j >> 1), s0, m0, s1, m1);  // sub-blocks 2g, 2g+1 of group g = j >> 1
    const float s = (j & 1) ? s1 : s0, m = (j & 1) ? m1 : m0;
    const uint4 qh = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 16 * h));
    const uint4 qs = __ldg(reinterpret_cast<const uint4 *>(blk + 48 + 32 * (j >> 1) + 16 * h));
    const uint32_t wh[4] = {qh.x, qh.y, qh.z, qh.w}, wl[4] = {qs.x, qs.y, qs.z, qs.w};
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t lo = (wl[i >> 2] >> (8 * (i & 3) + 4 * (j & 1))) & 15u;
      const uint32_t hi = (wh[i >> 2] >> (8 * (i & 3) + j)) & 1u;
      v[i] = __fmaf_rn(s, (float)(lo | (hi << 4)), -m);
    }
    store16<kBF16>(out, b * 256 + 32 * j + 16 * h, v);
  }
}

template <bool kBF16>
__global__ void __launch_bounds__(256) k_q6k_dequant(const uint8_t *__restrict__ blocks, int64_t nblocks,
                                                     void *__restrict__ out) {
  for (int64_t tid = (int64_t)blockIdx.x * 256 + threadIdx.x; tid < nblocks * 16; tid += (int64_t)gridDim.x * 256) {
    const int64_t b = tid >> 4;
    const int e0 = (int)(tid & 15) * 16;  // elements e0 .. e0+15 (one scale)
    const int g = e0 >> 7, k = (e0 >> 5) & 3, l0 = e0 & 31;
    const uint8_t *blk = blocks + b * 210;  // 210-byte blocks: byte loads
    const float d = f16_at(blk + 208);
    const float s = d * (float)(int8_t)__ldg(blk + 192 + (e0 >> 4));  // exact
    const uint8_t *ql = blk + 64 * g + 32 * (k & 1) + l0, *qh = blk + 128 + 32 * g + l0;
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t lo = ((uint32_t)__ldg(ql + i) >> (4 * (k >> 1))) & 15u;
      const uint32_t hi = ((uint32_t)__ldg(qh + i) >> (2 * k)) & 3u;
      v[i] = s * (float)((int)(lo | (hi << 4)) - 32);  // exact
    }
    store16<kBF16>(out, b * 256 + e0, v);
  }
}

template <bool kBF16>
__global__ void __launch_bounds__(256) k_q80_dequant(const uint8_t *__restrict__ blocks, int64_t nblocks,
                                                     void *__restrict__ out) {
  for (int64_t tid = (int64_t)blockIdx.x * 256 + threadIdx.x; tid < nblocks * 2; tid += (int64_t)gridDim.x * 256) {
    const int64_t b = tid >> 1;
    const int h = (int)(tid & 1);
    const uint8_t *blk = blocks + b * 34;  // 34-byte blocks: byte loads
    const float d = f16_at(blk);
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = d * (float)(int8_t)__ldg(blk + 2 + 16 * h + i);  // exact
    store16<kBF16>(out, b * 32 + 16 * h, v);
  }
}

}  // namespace

extern "C" {

int b200moe_q4k_dequant(const void *blocks, int64_t nblocks, void *out, int out_dtype, void *stream);

int b200moe_dequant(const void *blocks, int type, int64_t nblocks, void *out, int out_dtype, void *stream) {
  if (type == B200MOE_TYPE_Q4_K) return b200moe_q4k_dequant(blocks, nblocks, out, out_dtype, stream);
  if (type != B200MOE_TYPE_Q5_K && type != B200MOE_TYPE_Q6_K && type != B200MOE_TYPE_Q8_0)
    return b2host::set_error(B200MOE_EINVAL, "dequant: GGML type %d is not Q4_K(12), Q5_K(13), Q6_K(14) or Q8_0(8)",
                             type);
  if (nblocks < 0) return b2host::set_error(B200MOE_EINVAL, "dequant: nblocks=%lld < 0", (long long)nblocks);
  if (nblocks == 0) return B200MOE_OK;
  if (!blocks || !out) return b2host::set_error(B200MOE_EINVAL, "dequant: NULL pointer");
  if (((uintptr_t)out & 15) || (type == B200MOE_TYPE_Q5_K && ((uintptr_t)blocks & 15)))
    return b2host::set_error(B200MOE_EINVAL, "dequant: out (and Q5_K blocks) must be 16-byte aligned");
  if (out_dtype != B200MOE_F32 && out_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "dequant: out_dtype %d is neither F32 nor BF16", out_dtype);
  const int64_t threads = nblocks * (type == B200MOE_TYPE_Q8_0 ? 2 : 16);
  int64_t grid = (threads + 255) / 256;
  if (grid > 148 * 64) grid = 148 * 64;
  cudaStream_t s = (cudaStream_t)stream;
  const uint8_t *b = (const uint8_t *)blocks;
  const bool bf = out_dtype == B200MOE_BF16;
  if (type == B200MOE_TYPE_Q5_K) {
    if (bf) k_q5k_dequant<true><<<(unsigned)grid, 256, 0, s>>>(b, nblocks, out);
    else k_q5k_dequant<false><<<(unsigned)grid, 256, 0, s>>>(b, nblocks, out);
  } else if (type == B200MOE_TYPE_Q6_K) {
    if (bf) k_q6k_dequant<true><<<(unsigned)grid, 256, 0, s>>>(b, nblocks, out);
    else k_q6k_dequant<false><<<(unsigned)grid, 256, 0, s>>>(b, nblocks, out);
  } else {
    if (bf) k_q80_dequant<true><<<(unsigned)grid, 256, 0, s>>>(b, nblocks, out);
    else k_q80_dequant<false><<<(unsigned)grid, 256, 0, s>>>(b, nblocks, out);
  }
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

}  // extern "C"
