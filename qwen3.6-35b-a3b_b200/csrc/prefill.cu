// prefill.cu -- the prefill / large-batch MoE path: token sort + Q4_K grouped GEMMs on tcgen05.
//
//   k_prep        warp per token: x (given, or RMSNorm of the residual) -> xn f32, x16 fp16,
//                 and the shared-expert gate sg = sigmoid(w_sg . x)
//   k_router_gemm R1 logits for all tokens on CUDA cores, in the declared order (32 chunks of
//                 64 sequential fmaf, chunk sums added left to right) -> bf16
//   k_route_tok   warp per token: R2..R5 -> ids, bf16 routing weights
//   k_count       per token: the slots whose expert is in the requested range, and their order
//   k_plan        one CTA: packed row offsets per expert (the shared expert is expert 256 with
//                 every token), near-equal chunks of at most 192 tokens, and the GEMM tile tables
//   k_fill        thread per assignment: a row in its expert's range (plist), and the
//                 assignment's row position (inv)
//   k_gather_x    the x16 rows in assignment-list order (the gate_up GEMM's B operand)
//   k_gemm<1>     gate_up: D[128 gate rows | 128 up rows][tokens] = W . x^T, s = silu(g)*u -> fp16
//   k_gemm<2>     down:    D[128 h rows][tokens] = W_d . s^T -> y[position][h] = o * w (routed)
//                 or o (shared): every tile writes contiguous rows
//   k_combine     out[t] = sum over the in-range slots in ascending expert id of y[inv] (+ sg * the
//                 shared row)
//
// Entry points: b200moe_moe_route (the first three kernels), b200moe_moe_experts (the rest,
// for pre-routed tokens and an expert range: the expert-parallel building block) and
// b200moe_moe_prefill (both, on one GPU).
//
// The grouped GEMMs put the dequantised weight rows in the M = 128 slot of the UMMA and the
// expert's tokens (<= 256, padded to a multiple of 16) in N, so a ragged expert wastes at most
// 15 token columns. Weights are Q4_K in HBM; producer warps dequantise each 128 x 64 K-slab to
// fp16 in shared memory (half2 math: exact integer quants, fp16 sub-block scale and min), token
// rows arrive by TMA; one thread issues tcgen05.mma into TMEM; four warps drain TMEM.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "kq_dot.cuh"
#include "route.cuh"
#include "tc.cuh"

using namespace b2;

namespace {

constexpr int kNE = kE + 1;     // 256 routed experts + the shared expert
constexpr int kChunk = 192;     // tokens per GEMM tile (at most)
constexpr float kSScale = 1.0f / 1024.0f;  // fp16 storage scale of s = silu(gate) * up
constexpr int kErrRange = 4;    // status bit: an fp16 operand (x or s) was out of range

struct PrefillWS {
  float *xn;
  __half *x16;
  uint16_t *logits;
  float *sg;
  int32_t *ids;
  uint16_t *wb;
  int32_t *order;
  int32_t *counts;   // [257]
  int32_t *offsets;  // [258]
  int32_t *plist;    // [9T]
  __half *x16p;      // [9T][2048] the gate_up GEMM's B rows: x16 rows in assignment-list order
  int4 *tiles1;
  int4 *tiles2;
  int32_t *ntiles;   // [2]
  __half *s16;       // [9T][512]
  float *y;          // [9T][2048] down outputs by row position (routed: times the routing weight)
  int32_t *inv;      // [8T] row position of assignment t * 8 + slot (in-range experts only)
  float *wrow;       // [9T] routing weight (bf16 value) by row position; 1 for the shared expert's rows
  int32_t *err;      // [1]
};

size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

size_t max_chunks(int T) { return (size_t)(9 * (size_t)T) / kChunk + kNE + 1; }

size_t prefill_ws_bytes(int T) {
  const size_t t = (size_t)T, mc = max_chunks(T);
  return al256(t * kH * 4) + al256(t * kH * 2) + al256(t * kE * 2) + al256(t * 4) + al256(t * kK * 4) +
         al256(t * kK * 2) + al256(t * kK * 4) + al256(kNE * 4) + al256((kNE + 1) * 4) + al256(9 * t * 4) +
         al256(9 * t * kH * 2) + al256(mc * 4 * 16) + al256(mc * 16 * 16) + al256(2 * 4) + al256(9 * t * kI * 2) +
         al256(9 * t * kH * 4) + al256(8 * t * 4) + al256(4) + al256(9 * t * 4);
}

PrefillWS carve_prefill(void *ws, int T) {
  const size_t t = (size_t)T, mc = max_chunks(T);
  char *p = (char *)ws;
  PrefillWS w;
  auto take = [&](size_t n) { char *r = p; p += al256(n); return r; };
  w.xn = (float *)take(t * kH * 4);
  w.x16 = (__half *)take(t * kH * 2);
  w.logits = (uint16_t *)take(t * kE * 2);
  w.sg = (float *)take(t * 4);
  w.ids = (int32_t *)take(t * kK * 4);
  w.wb = (uint16_t *)take(t * kK * 2);
  w.order = (int32_t *)take(t * kK * 4);
  w.counts = (int32_t *)take(kNE * 4);
  w.offsets = (int32_t *)take((kNE + 1) * 4);
  w.plist = (int32_t *)take(9 * t * 4);
  w.x16p = (__half *)take(9 * t * kH * 2);
  w.tiles1 = (int4 *)take(mc * 4 * 16);
  w.tiles2 = (int4 *)take(mc * 16 * 16);
  w.ntiles = (int32_t *)take(2 * 4);
  w.s16 = (__half *)take(9 * t * kI * 2);
  w.y = (float *)take(9 * t * kH * 4);
  w.inv = (int32_t *)take(8 * t * 4);
  w.err = (int32_t *)take(4);
  w.wrow = (float *)take(9 * t * 4);
  return w;
}

// ------------------------------------------------------------------------- k_prep
// Warp per token. The arithmetic is per lane over its 64-element chunk (the declared RMSNorm
// order; the shared-expert gate as the decode path computes it), but global memory is read and
// written in whole coalesced rows: the row is staged in shared memory as 32 segments of 64 at a
// 68-float pitch (conflict-free both ways).
constexpr int kPrepWarps = 4;
constexpr int kPrepPitch = 68;

__global__ void __launch_bounds__(32 * kPrepWarps) k_prep(const void *x, int x_dtype, const float *resid, float eps,
                                                          int T, const void *wsg, int wf32, const float *nw,
                                                          float *xn, __half *x16, float *sg, int32_t *err) {
  __shared__ __align__(16) float rows[kPrepWarps][32 * kPrepPitch];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int t = blockIdx.x * kPrepWarps + wp;
  if (t >= T) return;
  float *row = rows[wp];
  auto at = [](int e) { return (e >> 6) * kPrepPitch + (e & 63); };  // element -> staged position
  // coalesced load of the token's row into the staging row
  if (resid || x_dtype != B200MOE_BF16) {
    const float *src = resid ? resid + (size_t)t * kH : reinterpret_cast<const float *>(x) + (size_t)t * kH;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int e = 4 * (32 * i + lane);
      const float4 a = resid ? __ldcg(reinterpret_cast<const float4 *>(src + e))
                             : __ldg(reinterpret_cast<const float4 *>(src + e));
      *reinterpret_cast<float4 *>(row + at(e)) = a;
    }
  } else {
    const uint16_t *xb = reinterpret_cast<const uint16_t *>(x) + (size_t)t * kH;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = 8 * (32 * i + lane);
      const uint4 u = __ldg(reinterpret_cast<const uint4 *>(xb + e));
      *reinterpret_cast<float4 *>(row + at(e)) = make_float4(bf16f(u.x), bf16f(u.x >> 16), bf16f(u.y), bf16f(u.y >> 16));
      *reinterpret_cast<float4 *>(row + at(e + 4)) =
          make_float4(bf16f(u.z), bf16f(u.z >> 16), bf16f(u.w), bf16f(u.w >> 16));
    }
  }
  __syncwarp();
  float v[64];
  {
    const float *c = row + lane * kPrepPitch;  // this lane's chunk: elements 64 lane .. 64 lane + 63
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 a = *reinterpret_cast<const float4 *>(c + 4 * i);
      v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
    }
  }
  if (resid) {
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 64; ++i) ss = __fmaf_rn(v[i], v[i], ss);
    float tot = __shfl_sync(0xFFFFFFFFu, ss, 0);
#pragma unroll
    for (int c = 1; c < 32; ++c) tot = __fadd_rn(tot, __shfl_sync(0xFFFFFFFFu, ss, c));
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, 2048.0f), eps)));
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __fmul_rn(v[i], rs);
    if (nw) {  // Form A weight, a second rounding
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 w = __ldg(reinterpret_cast<const float4 *>(nw + 64 * lane + 4 * i));
        v[4 * i] = __fmul_rn(v[4 * i], w.x); v[4 * i + 1] = __fmul_rn(v[4 * i + 1], w.y);
        v[4 * i + 2] = __fmul_rn(v[4 * i + 2], w.z); v[4 * i + 3] = __fmul_rn(v[4 * i + 3], w.w);
      }
    }
    float *c = row + lane * kPrepPitch;  // the normalised chunk back into the staging row
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 16; ++i)
      *reinterpret_cast<float4 *>(c + 4 * i) = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
  bool range_bad = false;
#pragma unroll
  for (int i = 0; i < 64; ++i) range_bad |= !(fabsf(v[i]) <= 65504.0f);
  if (__any_sync(0xFFFFFFFFu, range_bad) && lane == 0) atomicOr(err, kErrRange);
  float z = 0.0f;
  if (wf32) {  // f32 gate weights
    const float *w = reinterpret_cast<const float *>(wsg) + 64 * lane;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 a = __ldg(reinterpret_cast<const float4 *>(w + 4 * i));
      z = fmaf(v[4 * i], a.x, z);
      z = fmaf(v[4 * i + 1], a.y, z);
      z = fmaf(v[4 * i + 2], a.z, z);
      z = fmaf(v[4 * i + 3], a.w, z);
    }
  } else {
    const uint16_t *w = reinterpret_cast<const uint16_t *>(wsg) + 64 * lane;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 u = __ldg(reinterpret_cast<const uint4 *>(w + 8 * i));
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        z = fmaf(v[8 * i + 2 * q], bf16f(uw[q]), z);
        z = fmaf(v[8 * i + 2 * q + 1], bf16f(uw[q] >> 16), z);
      }
    }
  }
  z = warp_sum(z);
  if (lane == 0) sg[t] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
  __syncwarp();
  // coalesced stores of the f32 row and its fp16 copy
  float *dst = xn + (size_t)t * kH;
  __half *d16 = x16 + (size_t)t * kH;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int e = 4 * (32 * i + lane);
    const float4 a = *reinterpret_cast<const float4 *>(row + at(e));
    *reinterpret_cast<float4 *>(dst + e) = a;
    const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t *>(&h0);
    pk.y = *reinterpret_cast<const uint32_t *>(&h1);
    *reinterpret_cast<uint2 *>(d16 + e) = pk;
  }
}

// ------------------------------------------------------------------------- k_router_gemm
// CTA: kTM tokens x 64 experts, 128 threads; thread (ty, tx) owns tokens ty + 8i (i < kTM / 8)
// and experts tx + 16j (j < 4): with kTM = 64, 32 outputs and 128 FMAs per 12 shared-memory
// loads. The token tile is chosen per call (router_tile) so the busiest SM has the fewest rows;
// every output is the same sequence of operations whatever the tile.
// The 32 K chunks stream through a kRgStages-deep cp.async ring (x rows as f32, router rows as
// stored: bf16 rows are widened in the inner loop, exactly), so a chunk's loads are issued
// kRgStages - 1 chunks ahead of its use: with small tiles (an expert-parallel rank's few hundred
// tokens) the chunk's arithmetic is shorter than an L2 round trip.
constexpr int kRgPitch = 68;   // x and f32 router rows: padded pitch (floats)
constexpr int kRgPitchB = 72;  // bf16 router rows: padded pitch (bf16; 144 B, 16-byte aligned)
template <bool kF32>
constexpr int rg_stages() { return kF32 ? 3 : 4; }
template <bool kF32, int kTM>
constexpr int rg_stage_bytes() { return kTM * kRgPitch * 4 + (kF32 ? 64 * kRgPitch * 4 : 64 * kRgPitchB * 2); }
template <bool kF32, int kTM>
constexpr size_t rg_smem() { return (size_t)rg_stages<kF32>() * rg_stage_bytes<kF32, kTM>(); }

template <bool kF32, int kTM>
__global__ void __launch_bounds__(128) k_router_gemm(const float *__restrict__ xn, int T,
                                                     const void *__restrict__ wg_, const float *bias,
                                                     uint16_t *logits) {
  constexpr int kTI = kTM / 8;  // tokens per thread
  constexpr int kS = rg_stages<kF32>();
  constexpr int kSB = rg_stage_bytes<kF32, kTM>();
  const uint16_t *wg = reinterpret_cast<const uint16_t *>(wg_);  // bf16 router
  const float *wgf = reinterpret_cast<const float *>(wg_);        // f32 router (kF32)
  extern __shared__ __align__(16) uint8_t rg_smem_raw[];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int t0 = blockIdx.x * kTM, e0 = blockIdx.y * 64;
  // stage st: x rows [kTM][kRgPitch] f32, then router rows [64][kRgPitch] f32 or [64][kRgPitchB] bf16
  auto xs_of = [&](int st) { return reinterpret_cast<float *>(rg_smem_raw + st * kSB); };
  auto ws_of = [&](int st) { return rg_smem_raw + st * kSB + kTM * kRgPitch * 4; };
  auto load = [&](int c) {  // chunk c into stage c % kS, as one cp.async group
    float *xd = xs_of(c % kS);
    uint8_t *wd = ws_of(c % kS);
#pragma unroll
    for (int q = 0; q < kTI; ++q) {  // kTM rows x 16 slots of 16 B (zero rows past T)
      const int idx = tid + 128 * q;
      const int row = idx >> 4, col = (idx & 15) * 4;
      const bool in = t0 + row < T;
      cp_async16(xd + row * kRgPitch + col, xn + (size_t)(in ? t0 + row : 0) * kH + 64 * c + col, in ? 16u : 0u);
    }
    if (kF32) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {  // 64 rows x 16 slots
        const int idx = tid + 128 * q;
        const int row = idx >> 4, col = (idx & 15) * 4;
        cp_async16(reinterpret_cast<float *>(wd) + row * kRgPitch + col, wgf + (size_t)(e0 + row) * kH + 64 * c + col, 16u);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // 64 rows x 8 slots
        const int idx = tid + 128 * q;
        const int row = idx >> 3, col = (idx & 7) * 8;
        cp_async16(reinterpret_cast<uint16_t *>(wd) + row * kRgPitchB + col, wg + (size_t)(e0 + row) * kH + 64 * c + col, 16u);
      }
    }
  };
#pragma unroll
  for (int c = 0; c < kS - 1; ++c) {
    load(c);
    cp_async_commit();
  }
  float tot[kTI][4];
  for (int c = 0; c < 32; ++c) {
    cp_async_wait_group<kS - 2>();  // chunk c has landed (this thread's copies) ...
    __syncthreads();                // ... and everyone's; stage (c - 1) % kS is free again
    if (c + kS - 1 < 32) load(c + kS - 1);
    cp_async_commit();              // (an empty group past the end keeps the count uniform)
    const float *xb = xs_of(c % kS);
    const uint8_t *wb = ws_of(c % kS);
    float acc[kTI][4];
#pragma unroll
    for (int i = 0; i < kTI; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
#pragma unroll 2
    for (int k = 0; k < 64; k += 4) {  // the chunk's 64 products of every output, in k order
      float4 xa[kTI], wa[4];
#pragma unroll
      for (int i = 0; i < kTI; ++i) xa[i] = *reinterpret_cast<const float4 *>(xb + (ty + 8 * i) * kRgPitch + k);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (kF32) {
          wa[j] = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(wb) + (tx + 16 * j) * kRgPitch + k);
        } else {  // four bf16 -> f32 (exact): element k in the low half
          const uint2 u = *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(wb) + (tx + 16 * j) * kRgPitchB + k);
          wa[j] = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                              __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
        }
      }
#pragma unroll
      for (int i = 0; i < kTI; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] = __fmaf_rn(xa[i].x, wa[j].x, acc[i][j]);
          acc[i][j] = __fmaf_rn(xa[i].y, wa[j].y, acc[i][j]);
          acc[i][j] = __fmaf_rn(xa[i].z, wa[j].z, acc[i][j]);
          acc[i][j] = __fmaf_rn(xa[i].w, wa[j].w, acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < kTI; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) tot[i][j] = (c == 0) ? acc[i][j] : __fadd_rn(tot[i][j], acc[i][j]);
  }
  cp_async_wait_all();
#pragma unroll
  for (int i = 0; i < kTI; ++i) {
    const int t = t0 + ty + 8 * i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx + 16 * j;
      float v = tot[i][j];
      if (bias) v = __fadd_rn(v, bias[e]);
      logits[(size_t)t * kE + e] = f2bf(v);
    }
  }
}

// ------------------------------------------------------------------------- k_router_rows
// R1 for up to a few hundred tokens: warp w of CTA (bx, by) owns kEW expert rows (bf16 router:
// 4 rows, 4 warps per CTA; f32: 1 row, 8 warps) and tokens 8 by .. 8 by + 7. Lane c holds chunk
// c of each of its rows (64 values per row) in registers and runs the chunk's 64 sequential fmaf
// for every (row, token) pair side by side (32 independent chains for bf16); lane (i, j) then
// adds the 32 chunk sums of row i, token j left to right. That is the declared order, so every
// logit equals k_router_gemm's bit for bit. The 8 x rows sit in shared memory with a 68-float
// pitch per chunk, so the 32 lanes' 16-byte loads spread over every bank; shared-memory reads
// bound the kernel, so each x load feeds the warp's kEW rows (measured route stage at 512
// tokens: 66 us with 2 rows x 8 warps, 63 with 4 x 4). With few tokens the tiled GEMM's 32
// chunks wait on L2 one after another (36 us for 8 tokens); here each router row is read once
// per 8 tokens, every lane's chunk in flight at once.
#ifndef B2_RR_ROWS
#define B2_RR_ROWS 4
#endif
#ifndef B2_RR_WARPS
#define B2_RR_WARPS 4
#endif
constexpr int kRrTok = 8;                                     // tokens per CTA
constexpr int kRrPitch = 68;                                  // floats per chunk row in shared memory
constexpr int kRrXBytes = kRrTok * 32 * kRrPitch * 4;         // 69,632
template <bool kF32>
constexpr int rr_rows_per_warp() { return kF32 ? 1 : B2_RR_ROWS; }
template <bool kF32>
constexpr int rr_warps() { return kF32 ? 8 : B2_RR_WARPS; }
template <bool kF32>
constexpr size_t rr_smem() { return (size_t)kRrXBytes + rr_warps<kF32>() * rr_rows_per_warp<kF32>() * kRrTok * 33 * 4; }

template <bool kF32>
__global__ void __launch_bounds__(256, 1) k_router_rows(const float *__restrict__ xn, int T, const void *__restrict__ wg_,
                                                     const float *bias, uint16_t *logits) {
  constexpr int kEW = rr_rows_per_warp<kF32>();
  constexpr int kNT = 32 * rr_warps<kF32>();
  extern __shared__ __align__(16) uint8_t rr_smem_raw[];
  float *xs = reinterpret_cast<float *>(rr_smem_raw);               // [8 tokens][32 chunks][kRrPitch]
  float *ps = reinterpret_cast<float *>(rr_smem_raw + kRrXBytes);   // [warps][kEW][8 tokens][33]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = (blockIdx.x * rr_warps<kF32>() + warp) * kEW, t0 = blockIdx.y * kRrTok;
#pragma unroll
  for (int q = 0; q < kRrTok * 32 * 16 / kNT; ++q) {  // 8 rows x 512 slots of 16 B (zero rows past T)
    const int idx = threadIdx.x + kNT * q;
    const int j = idx >> 9, c = (idx >> 4) & 31, k = (idx & 15) * 4;
    const bool in = t0 + j < T;
    cp_async16(xs + (j * 32 + c) * kRrPitch + k, xn + (size_t)(in ? t0 + j : 0) * kH + 64 * c + k, in ? 16u : 0u);
  }
  cp_async_commit();
  // this lane's chunk of each of the warp's router rows: bf16 pairs, or f32
  uint32_t w[kEW][kF32 ? 64 : 32];
#pragma unroll
  for (int i = 0; i < kEW; ++i) {
    const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(wg_) +
                                                       ((size_t)(e0 + i) * kH + 64 * lane) * (kF32 ? 4 : 2));
#pragma unroll
    for (int q = 0; q < (kF32 ? 16 : 8); ++q) {
      const uint4 v = __ldg(src + q);
      w[i][4 * q] = v.x; w[i][4 * q + 1] = v.y; w[i][4 * q + 2] = v.z; w[i][4 * q + 3] = v.w;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  float acc[kEW][kRrTok];
#pragma unroll
  for (int i = 0; i < kEW; ++i)
#pragma unroll
    for (int j = 0; j < kRrTok; ++j) acc[i][j] = 0.0f;
#pragma unroll
  for (int k = 0; k < 64; k += 4) {  // the chunk's 64 products, in k order
    float wv[kEW][4];
#pragma unroll
    for (int i = 0; i < kEW; ++i) {
      if (kF32) {
        wv[i][0] = __uint_as_float(w[i][k]); wv[i][1] = __uint_as_float(w[i][k + 1]);
        wv[i][2] = __uint_as_float(w[i][k + 2]); wv[i][3] = __uint_as_float(w[i][k + 3]);
      } else {  // bf16 -> f32 exactly; element k in the low half
        wv[i][0] = __uint_as_float(w[i][k / 2] << 16); wv[i][1] = __uint_as_float(w[i][k / 2] & 0xFFFF0000u);
        wv[i][2] = __uint_as_float(w[i][k / 2 + 1] << 16); wv[i][3] = __uint_as_float(w[i][k / 2 + 1] & 0xFFFF0000u);
      }
    }
#pragma unroll
    for (int j = 0; j < kRrTok; ++j) {
      const float4 x = *reinterpret_cast<const float4 *>(xs + (j * 32 + lane) * kRrPitch + k);
#pragma unroll
      for (int i = 0; i < kEW; ++i) {
        acc[i][j] = __fmaf_rn(x.x, wv[i][0], acc[i][j]);
        acc[i][j] = __fmaf_rn(x.y, wv[i][1], acc[i][j]);
        acc[i][j] = __fmaf_rn(x.z, wv[i][2], acc[i][j]);
        acc[i][j] = __fmaf_rn(x.w, wv[i][3], acc[i][j]);
      }
    }
  }
  float *pw = ps + warp * kEW * kRrTok * 33;
#pragma unroll
  for (int i = 0; i < kEW; ++i)
#pragma unroll
    for (int j = 0; j < kRrTok; ++j) pw[(i * kRrTok + j) * 33 + lane] = acc[i][j];
  __syncwarp();
  const int i = lane / kRrTok, j = lane % kRrTok;
  if (i < kEW && t0 + j < T) {
    const float *pr = pw + (i * kRrTok + j) * 33;
    float tot = pr[0];
#pragma unroll
    for (int c = 1; c < 32; ++c) tot = __fadd_rn(tot, pr[c]);
    if (bias) tot = __fadd_rn(tot, bias[e0 + i]);
    logits[(size_t)(t0 + j) * kE + e0 + i] = f2bf(tot);
  }
}

// ------------------------------------------------------------------------- k_route_tok
__global__ void __launch_bounds__(256) k_route_tok(const uint16_t *logits, int T, int32_t *ids, uint16_t *wb) {
  __shared__ Route rr[8];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + w;
  if (t >= T) return;
  route_warp(logits + (size_t)t * kE, &rr[w]);
  if (lane < kK) {
    ids[(size_t)t * kK + lane] = rr[w].ids[lane];
    wb[(size_t)t * kK + lane] = rr[w].wb[lane];
  }
}

// ------------------------------------------------------------------------- k_count
// Per token: count its slots whose expert lies in [e_lo, e_hi), and the combine order of its
// 8 slots (ascending expert id; ties cannot occur, top-8 ids are distinct). The counts go
// through a per-CTA histogram in shared memory: one global atomic per (CTA, expert) instead of
// one per slot on 256 hot addresses.
__global__ void __launch_bounds__(256) k_count(int T, const int32_t *ids, int e_lo, int e_hi, int32_t *counts,
                                               int32_t *order) {
  __shared__ int hist[kE];
  for (int i = threadIdx.x; i < kE; i += 256) hist[i] = 0;
  __syncthreads();
  const int t = blockIdx.x * 256 + threadIdx.x;
  if (t < T) {
    int id[kK];
#pragma unroll
    for (int k = 0; k < kK; ++k) id[k] = __ldg(ids + (size_t)t * kK + k);
#pragma unroll
    for (int k = 0; k < kK; ++k) {
      if (id[k] >= e_lo && id[k] < e_hi) atomicAdd(&hist[id[k]], 1);
      int rank = 0;
#pragma unroll
      for (int j = 0; j < kK; ++j) rank += (id[j] < id[k] || (id[j] == id[k] && j < k)) ? 1 : 0;
      order[(size_t)t * kK + rank] = k;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kE; i += 256)
    if (hist[i]) atomicAdd(counts + i, hist[i]);
}

// ------------------------------------------------------------------------- k_plan
// One CTA of 512 threads (thread e < 257 owns expert e; e = 256 is the shared expert).
// Row offsets follow expert order 0..256; the chunk (tile) order puts the shared expert's
// full-width chunks first, then experts 0..255, so the largest tiles are scheduled first.
__global__ void __launch_bounds__(512) k_plan(int n_shared, const int32_t *counts_in, int32_t *offsets,
                                              int4 *tiles1, int4 *tiles2, int32_t *ntiles) {
  __shared__ int sc[512], sn[512];
  const int e = threadIdx.x;
  const int cnt = e < kE ? counts_in[e] : (e == kE ? n_shared : 0);
  const int nch = (cnt + kChunk - 1) / kChunk;
  const int pos = e == kE ? 0 : (e < kE ? e + 1 : e);  // a permutation of 0..511
  sc[e] = cnt;
  sn[pos] = nch;
  __syncthreads();
  for (int o = 1; o < 512; o <<= 1) {  // inclusive Hillis-Steele scans
    const int a = e >= o ? sc[e - o] : 0, b = e >= o ? sn[e - o] : 0;
    __syncthreads();
    sc[e] += a;
    sn[e] += b;
    __syncthreads();
  }
  if (e < kNE) offsets[e] = sc[e] - cnt;
  if (e == kNE - 1) offsets[kNE] = sc[e];
  __shared__ int s_nch[kNE], s_cb[kNE], s_r0[kNE], s_cnt[kNE];
  if (e <= kE) {
    s_nch[e] = nch;
    s_cb[e] = sn[pos] - nch;
    s_r0[e] = sc[e] - cnt;
    s_cnt[e] = cnt;
  }
  __syncthreads();
  // The tile tables, a warp per expert: each of the expert's nch near-equal chunks (at most
  // kChunk rows) gives 4 gate_up tiles and 16 down tiles. (A thread per expert left the shared
  // expert's T / kChunk chunks to one thread.)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int ee = warp; ee <= kE; ee += 16) {
    const int nc = s_nch[ee], cb = s_cb[ee], r0 = s_r0[ee], cn = s_cnt[ee];
    for (int q = lane; q < nc * 20; q += 32) {
      const int c = q / 20, k = q % 20;
      const int a0 = (int)((long long)c * cn / nc), a1 = (int)((long long)(c + 1) * cn / nc);
      if (k < 4) tiles1[4 * (cb + c) + k] = make_int4(ee, r0 + a0, a1 - a0, k);
      else tiles2[16 * (cb + c) + k - 4] = make_int4(ee, r0 + a0, a1 - a0, k - 4);
    }
  }
  if (e == 0) {
    ntiles[0] = 4 * sn[511];
    ntiles[1] = 16 * sn[511];
  }
}

// ------------------------------------------------------------------------- k_fill
// One thread per assignment a = t * 8 + slot whose expert is in range: it takes a row of its
// expert's range (the count of that expert ends at zero), and
// records plist[row] = a, inv[a] = row and the row's routing weight wrow[row] (the bf16 value
// as f32; 1 for the shared expert's rows). The order of rows inside an expert changes no result:
// every GEMM column, and every token's combine, is computed on its own. Rows from
// offsets[kE] on are the shared expert's: tokens sh_lo .. sh_hi-1 in order.
__global__ void __launch_bounds__(1024) k_fill(int T, int sh_lo, int sh_hi, const int32_t *ids, const uint16_t *wb,
                                               int e_lo, int e_hi, const int32_t *offsets, int32_t *counts,
                                               int32_t *plist, int32_t *inv, float *wrow) {
  // The CTA's assignments of each expert take consecutive rows: a shared-memory count, then one
  // global atomic per (CTA, expert) reserves the range (counting the expert's count down to 0).
  __shared__ int hist[kE], base[kE];
  for (int i = threadIdx.x; i < kE; i += 1024) hist[i] = 0;
  __syncthreads();
  const int a = blockIdx.x * 1024 + threadIdx.x;
  int e = -1, li = 0;
  if (a < T * kK) {
    e = __ldg(ids + a);
    if (e >= e_lo && e < e_hi) li = atomicAdd(&hist[e], 1);
    else e = -1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kE; i += 1024)
    if (hist[i]) base[i] = atomicSub(counts + i, hist[i]) - hist[i];
  __syncthreads();
  if (e >= 0) {
    const int row = __ldg(offsets + e) + base[e] + li;
    plist[row] = a;
    inv[a] = row;
    wrow[row] = bf16f(__ldg(wb + a));
  }
  if (a < sh_hi - sh_lo) {
    const int row = __ldg(offsets + kE) + a;
    plist[row] = sh_lo + a;
    wrow[row] = 1.0f;
  }
}

// ------------------------------------------------------------------------- k_gather_x
// x16p[pos] = x16[token of assignment-list entry pos] (x16 rows `pitch` halves apart: kH, or the
// expert-parallel dispatch rows), one warp per row (4 KB), so the gate_up
// GEMM reads its B operand as contiguous 64-row TMA boxes. Rows from offsets[kE] on belong to
// the shared expert (entries are token ids); the others hold t * 8 + slot.
__global__ void __launch_bounds__(256) k_gather_x(int max_rows, const int32_t *offsets, const int32_t *plist,
                                                  const __half *x16, int64_t pitch, __half *x16p) {
  const int total = __ldg(offsets + kNE), sh0 = __ldg(offsets + kE);
  const int lane = threadIdx.x & 31;
  for (int pos = (blockIdx.x * 256 + threadIdx.x) >> 5; pos < total && pos < max_rows; pos += gridDim.x * 8) {
    const int pl = __ldg(plist + pos);
    const int t = pos >= sh0 ? pl : (pl >> 3);
    const uint4 *src = reinterpret_cast<const uint4 *>(x16 + (size_t)t * pitch);
    uint4 *dst = reinterpret_cast<uint4 *>(x16p + (size_t)pos * kH);
#pragma unroll
    for (int i = 0; i < kH / 8 / 32; ++i) dst[lane + 32 * i] = __ldg(src + lane + 32 * i);
  }
}

// ------------------------------------------------------------------------- grouped GEMM
// Block of 15 warps, each with one job:
//   warps 0-3    epilogue: TMEM lanes 32w..32w+31 -> s (gate_up) or y (down)
//   warps 4-11   dequant: raw Q4_K slab (shared memory) -> fp16 A operand of the K-slab in
//                TMEM (tcgen05.st), each thread one row: the whole slab (gate_up) or half of
//                its quant bytes (down)
//   warp 12      TMEM allocation; lane 0 issues tcgen05.mma (A from TMEM, B from shared
//                memory) and the commits
//   warp 13      raw producer (lane 0): per K-slab and 128-row weight tile, two TMA loads of
//                the Q4_K bytes -- the 16-byte block headers and the slab's 32 quant bytes of
//                all 128 rows -- through 3-D tensor maps (bytes, row, expert)
//   warp 14      B producer (lane 0): the tile's token rows -> B ring as 64-row TMA boxes,
//                128-byte swizzled, from the contiguous rows of x16p (gate_up: x in
//                assignment-list order) or s16 (down). (Gathering the x16 rows per K-slab -- TMA
//                gather4 per 4 rows, or 16-byte cp.async -- was tried: one SM sustains only
//                ~7-11 B/cycle of such small requests, a third of what the MMA consumes.)
// No load is multicast. One iteration = one K-slab of 64 of one tile; every role walks the
// same (tile, slab) sequence: tile = blockIdx.x + j * gridDim.x, slab = 0 .. kKS-1.
//
// The A operand lives in TMEM, not shared memory. Shared-memory bandwidth (128 B per cycle per
// SM) is what bounds this kernel: with A in shared memory a gate_up K-slab moved about 142 KB
// through it (MMA reads of A and B, the dequant's A writes and raw reads, the TMA writes) and
// the MMAs ran at half their rate; with A in TMEM it moves about 78 KB.
//
// Three rings, each with full/empty mbarriers:
//   A stages kAStages x kA x 32 TMEM columns   written by the dequant warps (8 arrivals);
//                                              emptied by the MMA commit
//   B ring   kBStages x 24 KB        TMA bytes (one arming arrival); emptied by the MMA commit
//   raw ring kRStages x kA x 6 KB    TMA bytes (one arming arrival); emptied by the 8 dequant
//                                    warps once their rows are dequantised
// TMEM (512 columns): a tile has at most kChunk = 192 tokens, so each 256-column half keeps
// 64 columns free for the A stages. The down GEMM double-buffers its accumulator (columns 0 and
// 256) so the epilogue of one tile overlaps the next tile's main loop; gate_up holds gate at 0
// and up at 256 for one tile.
//
// Epilogue writes go out as TMA tensor stores: a warp stages its 32 rows x 16 tokens in
// shared memory and lane 0 stores them as one 16-row box of s16 / y rows (a tile's rows are
// contiguous row positions). gate_up stages a whole tile (its single accumulator is released as
// soon as the last columns are in registers); down alternates two sets of four. A ragged last chunk
// is split into 8-, 4-, 2- and 1-row boxes, so no store reaches past the tile into another
// expert's rows. (Plain per-column 128-byte stores ran at ~6 B/cycle per SM: the epilogue, not
// the MMA, bounded the down GEMM.)
// 8 dequant warps: 16 were measured slower (0.80 vs 0.87 ms per 4096-token layer, with A in
// shared memory), their extra traffic and spinning waiters costing more than the latency they
// hide.
constexpr int kEpiWarps = 4, kDqWarps = 8;
constexpr int kDqThreads = 32 * kDqWarps;
constexpr int kMmaWarp = kEpiWarps + kDqWarps;
constexpr int kRawWarp = kMmaWarp + 1;
constexpr int kBWarp = kRawWarp + 1;
constexpr int kGemmThreads = 32 * (kBWarp + 1);
constexpr int kRawHdr = 128 * 16;               // per 128-row tile: the rows' block headers
constexpr int kRawTile = kRawHdr + 128 * 32;    // + the rows' 32 quant bytes of the slab

template <int kMode>
struct GemmCfg {
  static constexpr int kA = kMode == 1 ? 2 : 1;                // A tiles per stage (gate+up / down)
  static constexpr int kARows = 128 * kA;                       // weight rows per tile
  static constexpr int kTpr = kDqThreads / kARows;              // dequant threads per row (1 or 2)
  static constexpr int kNw = 8 / kTpr;                          // quant words (4 bytes) of a slab row per thread
  static constexpr int kKS = (kMode == 1 ? kH : kI) / 64;       // K-slabs of 64 per tile
  static constexpr int kAStages = kMode == 1 ? 2 : 4;           // A stages (in TMEM)
  static constexpr int kBStages = 3;
  static constexpr int kRStages = kMode == 1 ? 6 : 8;
  static constexpr int kBTile = kChunk * 128;                   // kChunk rows x 128 B
  static constexpr int kRawStage = kA * kRawTile;
  static constexpr int kNBuf = kMode == 1 ? 1 : 2;              // TMEM accumulator buffers
  static constexpr uint32_t kAccCols = kMode == 1 ? 512 : 256;  // column stride of the buffers
  static constexpr uint32_t kTmemCols = 512;
  // TMEM columns of A stage s, tile a (32 columns = one K-slab of 128 rows): the columns
  // kChunk..255 of each 256-column half, which the accumulators (N <= kChunk) leave free.
  // gate_up: accumulators gate 0.., up 256..; stages at 192 and 448 (64 columns each).
  // down: accumulator buffers 0.. and 256..; stages at 192, 224, 448, 480.
  __host__ __device__ static constexpr uint32_t a_col(int s, int a) {
    return kMode == 1 ? (uint32_t)(kChunk + 256 * s + 32 * a) : (uint32_t)(kChunk + 256 * (s >> 1) + 32 * (s & 1));
  }
  static constexpr int kG = kMode == 1 ? 2 : 4;                       // epilogue: 16-token chunks per group
  static constexpr int kStageChunks = kMode == 1 ? kChunk / 16 : 2 * kG;  // staged chunks per epilogue warp
  static constexpr int kStageBytes = 16 * 32 * (kMode == 1 ? 2 : 4);  // one warp's staged chunk
  static constexpr int kOffB = 0;                                     // 1024-aligned stages
  static constexpr int kOffRaw = kOffB + kBStages * kBTile;
  static constexpr int kOffMeta = kOffRaw + kRStages * kRawStage;     // epilogue routing weights
  static constexpr int kOffStage = kOffMeta + kEpiWarps * kChunk * 4;  // [4 warps][kStageChunks][16 x 32]
  static constexpr int kOffBar = kOffStage + kEpiWarps * kStageChunks * kStageBytes;
  static constexpr size_t kSmem = (size_t)kOffBar + 512 + 1024;       // + barriers, + alignment
  static_assert(kChunk + 64 <= 256 && a_col(kAStages - 1, kA - 1) + 32 <= kTmemCols, "TMEM columns");
  static_assert(kSmem <= 232448, "shared memory");
};

// Tensor maps of one launch (kernel parameter space; each 64-byte aligned).
struct GemmMaps {
  CUtensorMap hdr[2][2];  // [routed, shared][A tile: gate|down, up] -> block headers
  CUtensorMap qnt[2][2];  // same weights -> the 32 quant bytes of a slab
  CUtensorMap b;          // B rows (box 64 x 64, 128-byte swizzle): x16p (gate_up) or s16 (down)
  CUtensorMap st[5];      // epilogue stores into s16 (gate_up) or y (down): box 32 x 16, 8, 4, 2, 1
};

struct GemmParams {
  GemmMaps m;
  const int4 *tiles;
  const int32_t *ntiles;
  const float *wrow;
  __half *s16;
  float *y;
  int32_t *err;
};

// nw quant words of K-slab g of one Q4_K block row -> that row's TMEM lane, both halves. Byte j
// of the slab's 32 quant bytes holds element j (low nibble, sub-block 2g) and element 32+j (high
// nibble, sub-block 2g+1); element k of the slab sits in column k / 2 of the A stage (even k in
// the low half). `taddr` addresses the column of this thread's first low-nibble element pair;
// the high nibbles go 16 columns further. One byte permute feeds both halves: a low nibble ORed
// into the mantissa of 1024.0 reads as 1024+q, a high nibble (mantissa bits 4..7, unit 1/16 in
// [64, 128)) ORed into 64.0 reads as 64+q; either subtraction leaves q exactly, and
// x = fma(q, S, -M) in fp16.
template <int nw>
__device__ __forceinline__ void dequant_words(const uint4 &hd, const uint32_t (&qw)[nw], int g, uint32_t taddr) {
  float s0, m0, s1, m1;
  q4k_scales(hd, 2 * g, s0, m0, s1, m1);
  const __half2 S0 = __float2half2_rn(s0), M0 = __float2half2_rn(-m0);
  const __half2 S1 = __float2half2_rn(s1), M1 = __float2half2_rn(-m1);
  const __half2 k1024 = __float2half2_rn(1024.0f), k64 = __float2half2_rn(64.0f);
  uint32_t lo[2 * nw], hi[2 * nw];
#pragma unroll
  for (int i = 0; i < nw; ++i) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const uint32_t pr = __byte_perm(qw[i], 0u, p ? 0x4342u : 0x4140u);  // [b, 0, b', 0]
      const uint32_t ql = (pr & 0x000F000Fu) | 0x64006400u;
      const uint32_t qh = (pr & 0x00F000F0u) | 0x54005400u;
      const __half2 xl = __hfma2(__hsub2(*reinterpret_cast<const __half2 *>(&ql), k1024), S0, M0);
      const __half2 xh = __hfma2(__hsub2(*reinterpret_cast<const __half2 *>(&qh), k64), S1, M1);
      lo[2 * i + p] = *reinterpret_cast<const uint32_t *>(&xl);
      hi[2 * i + p] = *reinterpret_cast<const uint32_t *>(&xh);
    }
  }
#pragma unroll
  for (int j = 0; j < 2 * nw; j += 8) {
    tmem_st8(taddr + j, lo + j);
    tmem_st8(taddr + 16 + j, hi + j);
  }
}

template <int kMode>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm(const __grid_constant__ GemmParams P) {
  using C = GemmCfg<kMode>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *b_ring = smem + C::kOffB;
  uint8_t *raw_ring = smem + C::kOffRaw;
  float *col_w = (float *)(smem + C::kOffMeta);              // [4][kChunk] per epilogue warp
  uint64_t *a_full = (uint64_t *)(smem + C::kOffBar);
  uint64_t *a_empty = a_full + C::kAStages;
  uint64_t *b_full = a_empty + C::kAStages;
  uint64_t *b_empty = b_full + C::kBStages;
  uint64_t *r_full = b_empty + C::kBStages;     // [kRStages]
  uint64_t *r_empty = r_full + C::kRStages;     // [kRStages]
  uint64_t *acc_full = r_empty + C::kRStages;   // [kNBuf]
  uint64_t *acc_empty = acc_full + C::kNBuf;    // [kNBuf]
  uint64_t *drain = acc_empty + C::kNBuf;
  uint32_t *tmem_slot = (uint32_t *)(drain + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kAStages; ++s) {
      mbar_init(a_full + s, kDqWarps);  // one arrival per dequant warp
      mbar_init(a_empty + s, 1);
    }
    for (int s = 0; s < C::kBStages; ++s) {
      mbar_init(b_full + s, 1);  // the producer's arming arrival (+ the TMA bytes)
      mbar_init(b_empty + s, 1);
    }
    for (int s = 0; s < C::kRStages; ++s) {
      mbar_init(r_full + s, 1);
      mbar_init(r_empty + s, kDqWarps);
    }
    for (int b = 0; b < C::kNBuf; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = __ldg(P.ntiles + (kMode - 1));
  const int my_tiles = ntiles > (int)blockIdx.x ? (ntiles - (int)blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const uint32_t n_it = (uint32_t)my_tiles * C::kKS;
  bool ok = true;

  if (warp >= kEpiWarps && warp < kMmaWarp) {  // ----------------------------- dequant
    // Warp w may write only TMEM lanes 32 (w % 4) .. +31, so a warp's lanes are its tile rows:
    // thread (group wg, quarter wq, lane) has row 32 wq + lane; gate_up: group wg dequantises A
    // tile wg (the whole slab of its row); down: group wg takes quant words 4 wg .. 4 wg + 3.
    const int pt = threadIdx.x - 32 * kEpiWarps;
    const int wq = (pt >> 5) & 3, wg = pt >> 7;
    const int tl = kMode == 1 ? wg : 0, tr = 32 * wq + lane, w0 = kMode == 1 ? 0 : 4 * wg;
    const uint32_t tlane = tmem + ((uint32_t)(32 * wq) << 16) + 2 * w0;
    // The words of slab it+1 are read from the raw ring before slab it is dequantised, so the
    // shared-memory latency overlaps the arithmetic.
    uint4 hd = make_uint4(0u, 0u, 0u, 0u), hd_n = hd;
    uint32_t qw[C::kNw], qw_n[C::kNw];
    auto load = [&](uint32_t j, uint4 &h, uint32_t (&q)[C::kNw]) {
      const uint8_t *rt = raw_ring + (j % C::kRStages) * C::kRawStage + tl * kRawTile;
      h = *reinterpret_cast<const uint4 *>(rt + tr * 16);
      const uint4 *qp = reinterpret_cast<const uint4 *>(rt + kRawHdr + tr * 32 + 4 * w0);
#pragma unroll
      for (int i = 0; i < C::kNw / 4; ++i) {
        const uint4 v = qp[i];
        q[4 * i] = v.x; q[4 * i + 1] = v.y; q[4 * i + 2] = v.z; q[4 * i + 3] = v.w;
      }
      if constexpr (C::kNw == 2) {
        const uint2 v = *reinterpret_cast<const uint2 *>(qp);
        q[0] = v.x; q[C::kNw - 1] = v.y;
      }
    };
    // warp-uniform outcomes: a lane that timed out never leaves its warp behind in __syncwarp
    if (n_it > 0) {
      if (__all_sync(0xFFFFFFFFu, mbar_wait(r_full, 0))) load(0, hd, qw);
      else ok = false;
    }
    for (uint32_t it = 0; it < n_it && ok; ++it) {
      const int ks = it % C::kKS;
      const int s = it % C::kAStages, rs = it % C::kRStages;
      if (it + 1 < n_it) {
        const uint32_t jn = it + 1;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(r_full + jn % C::kRStages, (jn / C::kRStages) & 1))) { ok = false; break; }
        load(jn, hd_n, qw_n);
      }
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(a_empty + s, ((it / C::kAStages) & 1) ^ 1))) { ok = false; break; }
      tc_fence_after();  // the MMAs that read this stage have completed
      dequant_words<C::kNw>(hd, qw, ks & 3, tlane + C::a_col(s, tl));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(a_full + s);
        // The raw stage is released only now, after the dequant has CONSUMED the loaded words:
        // released right after the loads were issued, a load still in flight could read bytes
        // that the producer's next TMA load had already overwritten.
        mbar_arrive(r_empty + rs);
      }
      hd = hd_n;
#pragma unroll
      for (int i = 0; i < C::kNw; ++i) qw[i] = qw_n[i];
    }
  } else if (warp == kRawWarp) {  // ----------------------------------------- raw producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int ti = blockIdx.x; ti < ntiles && ok; ti += gridDim.x) {
        const int4 tl = __ldg(P.tiles + ti);
        const int sh = tl.x < kE ? 0 : 1, z = tl.x < kE ? tl.x : 0, y = tl.w * 128;
        for (int ks = 0; ks < C::kKS; ++ks, ++it) {
          const int rs = it % C::kRStages;
          if (!mbar_wait(r_empty + rs, ((it / C::kRStages) & 1) ^ 1)) { ok = false; break; }
          mbar_expect_tx(r_full + rs, C::kRawStage);
          const int xh = (ks >> 2) * kQB, xq = xh + 16 + 32 * (ks & 3);
#pragma unroll
          for (int a = 0; a < C::kA; ++a) {
            uint8_t *d = raw_ring + rs * C::kRawStage + a * kRawTile;
            tma_load_3d(d, &P.m.hdr[sh][a], xh, y, z, r_full + rs);
            tma_load_3d(d + kRawHdr, &P.m.qnt[sh][a], xq, y, z, r_full + rs);
          }
        }
      }
      // every issued load lands before the CTA can exit (their stages' last phases complete)
      for (uint32_t j = it > (uint32_t)C::kRStages ? it - C::kRStages : 0; j < it; ++j)
        if (!mbar_wait(r_full + j % C::kRStages, (j / C::kRStages) & 1)) ok = false;
    }
    __syncwarp();
  } else if (warp == kBWarp) {  // -------------------------------------------- B producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int ti = blockIdx.x; ti < ntiles && ok; ti += gridDim.x) {
        const int4 tl = __ldg(P.tiles + ti);
        const int nbox = (tl.z + 63) / 64;
        for (int ks = 0; ks < C::kKS; ++ks, ++it) {
          const int s = it % C::kBStages;
          if (!mbar_wait(b_empty + s, ((it / C::kBStages) & 1) ^ 1)) { ok = false; break; }
          mbar_expect_tx(b_full + s, (uint32_t)nbox * 64u * 128u);
          for (int g = 0; g < nbox; ++g)
            tma_load_2d(b_ring + s * C::kBTile + g * 64 * 128, &P.m.b, ks * 64, tl.y + 64 * g, b_full + s);
        }
      }
      // every issued load lands before the CTA can exit
      for (uint32_t j = it > (uint32_t)C::kBStages ? it - C::kBStages : 0; j < it; ++j)
        if (!mbar_wait(b_full + j % C::kBStages, (j / C::kBStages) & 1)) ok = false;
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {  // -------------------------------------------- MMA issue
    // The whole warp walks the loop and polls the barriers; one elected lane issues each slab's
    // MMAs as straight-line code from precomputed addresses, then the commits. (Issued by lane 0
    // of a diverged warp, with the descriptors built between the MMAs, the same MMAs took 4-8x
    // their tensor time on B200.)
    uint32_t it = 0, tcount = 0;
    const uint64_t bdesc0 = umma_desc_sw128(smem_u32(b_ring));
    for (int ti = blockIdx.x; ti < ntiles && ok; ti += gridDim.x, ++tcount) {
      const int4 tl = __ldg(P.tiles + ti);
      const uint32_t idesc = umma_idesc_f16((uint32_t)((tl.z + 15) & ~15));
      const uint32_t buf = tcount % C::kNBuf, use = tcount / C::kNBuf;
      if (use > 0 && !__all_sync(0xFFFFFFFFu, mbar_wait(acc_empty + buf, (use - 1) & 1))) { ok = false; break; }
      tc_fence_after();
      const uint32_t dacc = tmem + buf * C::kAccCols;
      for (int ks = 0; ks < C::kKS; ++ks, ++it) {
        const int sa = it % C::kAStages, sb = it % C::kBStages;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(a_full + sa, (it / C::kAStages) & 1))) { ok = false; break; }
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(b_full + sb, (it / C::kBStages) & 1))) { ok = false; break; }
        tc_fence_after();
        // B descriptors step by 32 bytes per K = 16 (address field in 16-byte units: +2)
        const uint64_t bd = bdesc0 + (uint64_t)((sb * C::kBTile) >> 4);
        const uint32_t at = tmem + C::a_col(sa, 0);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t acc = (ks | kk) != 0;
            umma_f16_ts(dacc, at + 8 * kk, bd + 2 * kk, idesc, acc);
            if (kMode == 1) umma_f16_ts(dacc + 256, at + 32 + 8 * kk, bd + 2 * kk, idesc, acc);
          }
          umma_commit(a_empty + sa);
          umma_commit(b_empty + sb);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (elect_one()) umma_commit(acc_full + buf);
      __syncwarp();
    }
    if (elect_one()) umma_commit(drain);  // every MMA this warp issued has completed before TMEM is released
    __syncwarp();
    if (!__all_sync(0xFFFFFFFFu, mbar_wait(drain, 0))) ok = false;
  } else {  // ---------------------------------------------------------- epilogue (warps 0-3)
    uint32_t tcount = 0, grp = 0;  // grp counts store groups across tiles: it picks the buffer set
    bool range_bad = false;
    uint8_t *stage = smem + C::kOffStage;
    for (int ti = blockIdx.x; ti < ntiles && ok; ti += gridDim.x, ++tcount) {
      const int4 tl = __ldg(P.tiles + ti);
      const int e = tl.x, r0 = tl.y, n = tl.z, wt = tl.w;
      const int npad = (n + 15) & ~15;
      const uint32_t buf = tcount % C::kNBuf, use = tcount / C::kNBuf;
      float *ww = col_w + warp * kChunk;
      if (kMode == 2) {
        // this warp's copy of the tile's output scales, loaded while the MMAs run: 2^10 (the s
        // storage scale undone) times the routing weight, or 2^10 alone for the shared expert.
        // Both factors are exact in f32, so one rounding of acc * scale equals the rounding of
        // (acc * 2^10) * weight.
        float wv[kChunk / 32];
#pragma unroll
        for (int j = 0; j < kChunk / 32; ++j)
          wv[j] = (e < kE && lane + 32 * j < n) ? __ldg(P.wrow + r0 + lane + 32 * j) * (1.0f / kSScale) : (1.0f / kSScale);
#pragma unroll
        for (int j = 0; j < kChunk / 32; ++j) ww[lane + 32 * j] = wv[j];
        __syncwarp();
      }
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(acc_full + buf, use & 1))) { ok = false; break; }
      tc_fence_after();
      if (kMode == 1) {  // the previous tile's stores have read this warp's staging area
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
      }
      const uint32_t lane_addr = tmem + buf * C::kAccCols + ((uint32_t)(32 * warp) << 16);
      const int col0 = wt * 128 + 32 * warp;  // this warp's first s16 column (gate_up) or y column (down)
      // Groups of kG 16-token chunks: every TMEM load of the group, one wait, then the group's
      // stores as one bulk group.
      for (int c0 = 0; c0 < npad; c0 += 16 * C::kG, ++grp) {
        const int nc = min(C::kG, (npad - c0) >> 4);  // chunks in this group (warp-uniform)
        float a[C::kG][16], u[kMode == 1 ? C::kG : 1][16];
#pragma unroll
        for (int g = 0; g < C::kG; ++g) {
          if (g < nc) {
            tmem_ld16(lane_addr + c0 + 16 * g, a[g]);
            if (kMode == 1) tmem_ld16(lane_addr + 256 + c0 + 16 * g, u[kMode == 1 ? g : 0]);
          }
        }
        tmem_wait_ld();
        if (c0 + 16 * C::kG >= npad) {  // every accumulator column of the tile is in registers: release TMEM
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty + buf);
        }
        // gate_up stages the whole tile (one buffer per chunk); down alternates two sets of kG
        // buffers, the bulk group that read one set two groups ago having finished reading.
        uint8_t *stg0 = stage + (warp * C::kStageChunks + (kMode == 1 ? (c0 >> 4) : (grp & 1) * C::kG)) * C::kStageBytes;
        if (kMode == 2) {
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
        }
#pragma unroll
        for (int g = 0; g < C::kG; ++g) {
          if (g < nc) {
            const int cg = c0 + 16 * g;
            uint8_t *stg = stg0 + g * C::kStageBytes;
            if (kMode == 1) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {  // silu(g) * u, stored as s * 2^-10 (exact scaling)
                const float x = a[g][i];
                const float v = __fdividef(x, 1.0f + __expf(-x)) * u[kMode == 1 ? g : 0][i] * kSScale;
                if (cg + i < n && !(fabsf(v) <= 65504.0f)) range_bad = true;
                reinterpret_cast<__half *>(stg)[i * 32 + lane] = __float2half_rn(v);
              }
            } else {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float4 w4 = *reinterpret_cast<const float4 *>(ww + cg + 4 * q);
                float *d = reinterpret_cast<float *>(stg) + 4 * q * 32 + lane;
                d[0] = __fmul_rn(a[g][4 * q], w4.x);
                d[32] = __fmul_rn(a[g][4 * q + 1], w4.y);
                d[64] = __fmul_rn(a[g][4 * q + 2], w4.z);
                d[96] = __fmul_rn(a[g][4 * q + 3], w4.w);
              }
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int g = 0; g < nc; ++g) {
            const int cg = c0 + 16 * g, m = min(16, n - cg);
            uint8_t *stg = stg0 + g * C::kStageBytes;
            if (m == 16) {
              tma_store_2d(&P.m.st[0], col0, r0 + cg, stg);
            } else {
              int q = 0;
#pragma unroll
              for (int p = 1; p < 5; ++p) {  // boxes of 8, 4, 2, 1 rows
                const int hgt = 16 >> p;
                if (m & hgt) {
                  tma_store_2d(&P.m.st[p], col0, r0 + cg + q, stg + q * 32 * (kMode == 1 ? 2 : 4));
                  q += hgt;
                }
              }
            }
          }
          bulk_commit_group();
        }
      }
      __syncwarp();  // this warp's metadata is read before the next tile overwrites it
    }
    if (lane == 0) bulk_wait_group_all();  // this warp's stores are complete before the CTA exits
    __syncwarp();
    if (range_bad) atomicOr(P.err, kErrRange);
  }
  if (!ok) atomicOr(P.err, kMode);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, C::kTmemCols);
}

// ------------------------------------------------------------------------- k_combine
// Expert-parallel return over peer memory: row r of the combine goes to rank r / rows, into its
// partial-row block of this rank (row (rank rows + r % rows) of that rank's ret buffer); rows
// without work are not sent.
constexpr int kMaxPeers = 8;
struct SegOut {
  float *base[kMaxPeers];
  int rows, rank, n;  // n = 0: plain output
};

// The CTA's stores into peer memory are performed at system scope before the kernel ends, so the
// flag that a later kernel on this stream stores (release, system scope) cannot overtake them:
// the barrier orders every thread's stores before thread 0's fence, which is cumulative over
// them. One fence per CTA; a fence in every thread cost one NVLink round trip per warp.
__device__ __forceinline__ void cta_fence_system() {
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
}

__global__ void __launch_bounds__(256) k_combine(int T, const float *y, const int32_t *inv, const int32_t *offsets,
                                                 const float *sg, int sh_lo, int sh_hi, const int32_t *ids,
                                                 const int32_t *order, int e_lo, int e_hi, float *out,
                                                 int accumulate, const SegOut seg) {
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;  // one float4 of one token
  const bool in = idx < (int64_t)T * (kH / 4);
  if (!in && !seg.n) return;
  const int t = in ? (int)(idx / (kH / 4)) : 0, h = in ? (int)(idx % (kH / 4)) * 4 : 0;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  bool work = in && sg && t >= sh_lo && t < sh_hi;
  if (in) {
#pragma unroll
    for (int i = 0; i < kK; ++i) {
      const int slot = __ldg(order + (size_t)t * kK + i);
      const int e = __ldg(ids + (size_t)t * kK + slot);
      if (e < e_lo || e >= e_hi) continue;
      work = true;
      const int pos = __ldg(inv + (size_t)t * kK + slot);
      const float4 v = __ldcs(reinterpret_cast<const float4 *>(y + (size_t)pos * kH + h));
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
  }
  float4 r = acc;
  if (in && sg && t >= sh_lo && t < sh_hi) {
    const float g = __ldg(sg + (t - sh_lo));
    const int pos = __ldg(offsets + kE) + (t - sh_lo);  // the shared expert's rows come last
    const float4 sh = __ldcs(reinterpret_cast<const float4 *>(y + (size_t)pos * kH + h));
    r = make_float4(__fadd_rn(acc.x, __fmul_rn(g, sh.x)), __fadd_rn(acc.y, __fmul_rn(g, sh.y)),
                    __fadd_rn(acc.z, __fmul_rn(g, sh.z)), __fadd_rn(acc.w, __fmul_rn(g, sh.w)));
  }
  if (seg.n) {  // every thread of the CTA reaches the closing fence
    if (work) {
      const int s = t / seg.rows;
      float *b = seg.base[0];
#pragma unroll
      for (int k = 1; k < kMaxPeers; ++k)
        if (k == s) b = seg.base[k];  // (a select, not an indexed copy of the parameter array)
      *reinterpret_cast<float4 *>(b + ((size_t)seg.rank * seg.rows + (t - s * seg.rows)) * kH + h) = r;
    }
    cta_fence_system();
    return;
  }
  float4 *dst = reinterpret_cast<float4 *>(out + (size_t)t * kH + h);
  if (accumulate) {
    const float4 o = *dst;
    r = make_float4(__fadd_rn(o.x, r.x), __fadd_rn(o.y, r.y), __fadd_rn(o.z, r.z), __fadd_rn(o.w, r.w));
  }
  *dst = r;
}

// ------------------------------------------------------------------------- expert parallelism
// Dispatch rows: one per (source token, destination rank) pair that has work there -- 2048 fp16
// x values, then the token's 8 expert ids (int32), its 8 bf16 routing weights and 16 bytes of
// padding (4160 B, 16-byte aligned). A source rank with T tokens fills a [world][T] grid of
// rows: destination d's rows 0 .. n_d - 1 are its tokens with a slot in d's expert range, in
// ascending token order (every token for d = rank, where the shared expert runs); rows from n_d
// on carry ids -1 and no work. pos[t][d] is token t's row at d (-1: none).
constexpr int kEpRowHalves = kH + 32;
constexpr int kEpIdsOff = kH * 2;          // byte offset of the ids in a row
constexpr int kEpWOff = kEpIdsOff + 32;    // byte offset of the weights
static_assert(kEpRowHalves * 2 == B200MOE_EP_ROW_BYTES, "dispatch row size");

// CTA d = destination: a block-wide scan over the tokens gives every row position; writes pos
// and the rows' ids / weights (the x values are copied by k_ep_copy).
// Flag words of the peer form: own_flags [world] receive every rank's epoch; peer_flags[d] is rank
// d's flag array (this rank writes element `rank` of it).
struct EpFlags {
  uint32_t *own_flags;
  uint32_t *peer_flags[kMaxPeers];
  const uint32_t *epoch;
};

// Where the rows for destination d go: block d of the local send buffer (an all-to-all moves it),
// or -- over peer memory -- straight into block `rank` of rank d's receive buffer.
struct EpDst {
  uint8_t *send;                   // local [world][T] rows, or NULL for the peer form
  uint8_t *peer_recv[kMaxPeers];   // peer form: each rank's receive buffer
  uint32_t *epoch;                 // peer form: this rank's step counter (bumped by block 0)
  __device__ uint8_t *block(int d, int rank, int T) const {
    if (send) return send + (size_t)d * T * B200MOE_EP_ROW_BYTES;
    uint8_t *b = peer_recv[0];
#pragma unroll
    for (int k = 1; k < kMaxPeers; ++k)
      if (k == d) b = peer_recv[k];  // a select: an indexed read would copy the array to local memory
    return b + (size_t)rank * T * B200MOE_EP_ROW_BYTES;
  }
};

__global__ void __launch_bounds__(1024) k_ep_plan(int T, const int32_t *ids, const uint16_t *wb, int rank, int world,
                                                  const EpDst dst, int32_t *pos) {
  __shared__ int wsum[32];
  const int d = blockIdx.x, per = kE / world, lo = d * per, hi = lo + per;
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  if (d == 0 && threadIdx.x == 0 && dst.epoch) *dst.epoch += 1u;  // this step's signal value
  uint8_t *seg = dst.block(d, rank, T);
  int carry = 0;
  for (int base = 0; base < T; base += 1024) {
    const int t = base + threadIdx.x;
    bool f = false;
    int4 i0 = make_int4(-1, -1, -1, -1), i1 = i0;
    if (t < T) {
      i0 = __ldg(reinterpret_cast<const int4 *>(ids + (size_t)t * kK));
      i1 = __ldg(reinterpret_cast<const int4 *>(ids + (size_t)t * kK) + 1);
      const int id[8] = {i0.x, i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w};
      f = d == rank;
#pragma unroll
      for (int k = 0; k < kK; ++k) f |= id[k] >= lo && id[k] < hi;
    }
    const unsigned b = __ballot_sync(0xFFFFFFFFu, f);
    if (lane == 0) wsum[wp] = __popc(b);
    __syncthreads();
    if (wp == 0) {  // inclusive scan of the 32 warp counts
      int v = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (lane >= o) v += u;
      }
      wsum[lane] = v;
    }
    __syncthreads();
    const int p = carry + (wp ? wsum[wp - 1] : 0) + __popc(b & ((1u << lane) - 1u));
    if (t < T) {
      pos[(size_t)t * world + d] = f ? p : -1;
      if (f) {
        uint8_t *row = seg + (size_t)p * B200MOE_EP_ROW_BYTES;
        reinterpret_cast<int4 *>(row + kEpIdsOff)[0] = i0;
        reinterpret_cast<int4 *>(row + kEpIdsOff)[1] = i1;
        *reinterpret_cast<uint4 *>(row + kEpWOff) = __ldg(reinterpret_cast<const uint4 *>(wb + (size_t)t * kK));
      }
    }
    carry += wsum[31];
    __syncthreads();  // wsum is rewritten by the next round
  }
  const int4 none = make_int4(-1, -1, -1, -1);
  for (int p = carry + threadIdx.x; p < T; p += 1024) {  // rows without work
    uint8_t *row = seg + (size_t)p * B200MOE_EP_ROW_BYTES;
    reinterpret_cast<int4 *>(row + kEpIdsOff)[0] = none;
    reinterpret_cast<int4 *>(row + kEpIdsOff)[1] = none;
  }
  if (!dst.send) cta_fence_system();  // peer stores complete before the dispatch signal
}

// CTA t: token t's 4 KB of x16 into its row at every destination that takes it.
__global__ void __launch_bounds__(256) k_ep_copy(int T, const __half *x16, int rank, int world, const int32_t *pos,
                                                 const EpDst dst) {
  const int t = blockIdx.x;
  const uint4 v = __ldg(reinterpret_cast<const uint4 *>(x16 + (size_t)t * kH) + threadIdx.x);
  for (int d = 0; d < world; ++d) {
    const int p = __ldg(pos + (size_t)t * world + d);
    if (p >= 0) reinterpret_cast<uint4 *>(dst.block(d, rank, T) + (size_t)p * B200MOE_EP_ROW_BYTES)[threadIdx.x] = v;
  }
  if (!dst.send) cta_fence_system();
}

// Peer signalling: lane d stores this step's epoch into rank d's flag word for this rank
// (release at system scope, after the kernels that wrote into rank d's memory), and the wait
// polls this rank's own flag words until every peer's epoch has arrived -- bounded: after
// ~1 s it sets status bit 8 and returns, so a rank that is gone cannot hang this one.
constexpr int kErrPeer = 8;

__global__ void __launch_bounds__(32) k_ep_signal(int world, int rank, const EpFlags f) {
  const int d = threadIdx.x;
  if (d >= world) return;
  const uint32_t e = *f.epoch;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f.peer_flags[d] + rank), "r"(e) : "memory");
}

__global__ void __launch_bounds__(32) k_ep_wait(int world, const EpFlags f, int32_t *status) {
  const int s = threadIdx.x;
  if (s >= world) return;
  const uint32_t e = *f.epoch;
  const long long t0 = clock64();
  for (;;) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f.own_flags + s) : "memory");
    if ((int32_t)(v - e) >= 0) break;
    if (clock64() - t0 > kWaitBudgetCycles) {
      atomicOr(status, kErrPeer);
      break;
    }
  }
}

// Receiver: the ids and weights of the R gathered rows into contiguous arrays.
__global__ void __launch_bounds__(256) k_ep_unpack(int R, const uint8_t *rows, int32_t *ids, uint16_t *wb) {
  const int r = blockIdx.x * 256 + threadIdx.x;
  if (r >= R) return;
  const uint8_t *row = rows + (size_t)r * B200MOE_EP_ROW_BYTES;
  reinterpret_cast<int4 *>(ids + (size_t)r * kK)[0] = reinterpret_cast<const int4 *>(row + kEpIdsOff)[0];
  reinterpret_cast<int4 *>(ids + (size_t)r * kK)[1] = reinterpret_cast<const int4 *>(row + kEpIdsOff)[1];
  *reinterpret_cast<uint4 *>(wb + (size_t)r * kK) = *reinterpret_cast<const uint4 *>(row + kEpWOff);
}

// Source: out[t] (+)= sum over destinations d = 0, 1, ... (ascending expert ranges) of the partial
// row ret[d][pos[t][d]]; one thread per float4.
__global__ void __launch_bounds__(256) k_ep_sum(int T, int world, const float *ret, const int32_t *pos, float *out,
                                                int accumulate) {
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (idx >= (int64_t)T * (kH / 4)) return;
  const int t = (int)(idx / (kH / 4)), h = (int)(idx % (kH / 4)) * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int d = 0; d < world; ++d) {
    const int p = __ldg(pos + (size_t)t * world + d);
    if (p < 0) continue;
    const float4 v = __ldcs(reinterpret_cast<const float4 *>(ret + ((size_t)d * T + p) * kH + h));
    acc = make_float4(__fadd_rn(acc.x, v.x), __fadd_rn(acc.y, v.y), __fadd_rn(acc.z, v.z), __fadd_rn(acc.w, v.w));
  }
  float4 *dst = reinterpret_cast<float4 *>(out + (size_t)t * kH + h);
  if (accumulate) {
    const float4 o = *dst;
    acc = make_float4(__fadd_rn(o.x, acc.x), __fadd_rn(o.y, acc.y), __fadd_rn(o.z, acc.z), __fadd_rn(o.w, acc.w));
  }
  *dst = acc;
}

bool a16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

int g_num_sms = 0;

template <bool kF32>
cudaError_t router_gemm_attrs();

int ensure_gemm_attrs() {
  static int done = 0;
  if (done) return B200MOE_OK;
  B2_CUDA(cudaFuncSetAttribute(k_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GemmCfg<1>::kSmem));
  B2_CUDA(cudaFuncSetAttribute(k_gemm<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GemmCfg<2>::kSmem));
  B2_CUDA(router_gemm_attrs<false>());
  B2_CUDA(router_gemm_attrs<true>());
  B2_CUDA(cudaFuncSetAttribute(k_router_rows<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rr_smem<false>()));
  B2_CUDA(cudaFuncSetAttribute(k_router_rows<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rr_smem<true>()));
  int dev = 0;
  B2_CUDA(cudaGetDevice(&dev));
  B2_CUDA(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  done = 1;
  return B200MOE_OK;
}

constexpr int kMaxTPrefill = 1 << 16;

// ---------------------------------------------------------------- tensor maps
// Encoded maps are cached by their full description (a layer's weights and a workspace are
// reused call after call), so steady-state calls encode nothing.
struct MapKey {
  const void *base;
  int dtype, swz;
  uint64_t d0, d1, d2, s1, s2;
  uint32_t b0, b1;
  bool operator==(const MapKey &o) const {
    return base == o.base && dtype == o.dtype && swz == o.swz && d0 == o.d0 && d1 == o.d1 && d2 == o.d2 &&
           s1 == o.s1 && s2 == o.s2 && b0 == o.b0 && b1 == o.b1;
  }
};

// The driver's encoder, found at run time through the runtime API, so the library itself does
// not depend on libcuda (it loads on a machine without a driver; calls then fail cleanly).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_map(const MapKey &k, CUtensorMap *out) {
  static std::mutex mu;
  static MapKey keys[128];
  static CUtensorMap maps[128];
  static int n = 0, next = 0;
  static EncodeTiledFn encode = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    B2_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn)
      return b2host::set_error(B200MOE_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    encode = (EncodeTiledFn)fn;
  }
  for (int i = 0; i < n; ++i)
    if (keys[i] == k) {
      *out = maps[i];
      return B200MOE_OK;
    }
  const cuuint64_t dims[3] = {k.d0, k.d1, k.d2};
  const cuuint64_t strides[2] = {k.s1, k.s2};
  const cuuint32_t box[3] = {k.b0, k.b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const int rank = k.d2 > 0 ? 3 : 2;
  const CUresult r = encode(
      out,
      k.dtype == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                   : (k.dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8),
      (cuuint32_t)rank,
      const_cast<void *>(k.base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      k.swz ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return b2host::set_error(B200MOE_EINVAL, "tensor map encode failed (%d) for %p, dims %llu x %llu x %llu", (int)r,
                             k.base, (unsigned long long)k.d0, (unsigned long long)k.d1, (unsigned long long)k.d2);
  keys[next] = k;
  maps[next] = *out;
  next = (next + 1) % 128;
  if (n < 128) ++n;
  return B200MOE_OK;
}

// Header and quant maps of one Q4_K weight matrix [experts][rows][row_bytes] (3-D, bytes).
int weight_maps(const void *base, int row_bytes, int rows, int experts, int64_t expert_stride, CUtensorMap *hdr,
                CUtensorMap *qnt) {
  if (((uintptr_t)base & 15) || (expert_stride & 15))
    return b2host::set_error(B200MOE_EINVAL, "prefill: weight base %p / expert stride %lld not 16-byte aligned", base,
                             (long long)expert_stride);
  MapKey k{base, 0, 0, (uint64_t)row_bytes, (uint64_t)rows, (uint64_t)experts, (uint64_t)row_bytes,
           (uint64_t)(experts > 1 ? expert_stride : (int64_t)rows * row_bytes), 16, 128};
  int rc = encode_map(k, hdr);
  if (rc) return rc;
  k.b0 = 32;
  return encode_map(k, qnt);
}

// All maps of one GEMM launch: kMode 1 (gate_up: the four weight matrices, B = the 9Ts rows of
// x16p, stores into s16) or 2 (down: the two weight matrices, B = the 9Ts rows of s16, stores
// into y).
int gemm_maps(int mode, const b200moe_layer *L, const __half *x16p, const __half *s16, const float *y, int Ts,
              GemmMaps &m) {
  int rc;
  if (mode == 1) {
    if ((rc = weight_maps(L->gate, kRowUp, kI, kE, L->gate_up_expert_stride, &m.hdr[0][0], &m.qnt[0][0]))) return rc;
    if ((rc = weight_maps(L->up, kRowUp, kI, kE, L->gate_up_expert_stride, &m.hdr[0][1], &m.qnt[0][1]))) return rc;
    if ((rc = weight_maps(L->sh_gate, kRowUp, kI, 1, 0, &m.hdr[1][0], &m.qnt[1][0]))) return rc;
    if ((rc = weight_maps(L->sh_up, kRowUp, kI, 1, 0, &m.hdr[1][1], &m.qnt[1][1]))) return rc;
    const MapKey kb{x16p, 1, 1, (uint64_t)kH, (uint64_t)9 * Ts, 0, (uint64_t)kH * 2, 0, 64, 64};
    if ((rc = encode_map(kb, &m.b))) return rc;
    for (int p = 0; p < 5; ++p) {
      const MapKey ks{s16, 1, 0, (uint64_t)kI, (uint64_t)9 * Ts, 0, (uint64_t)kI * 2, 0, 32, (uint32_t)(16 >> p)};
      if ((rc = encode_map(ks, &m.st[p]))) return rc;
    }
    return B200MOE_OK;
  }
  if ((rc = weight_maps(L->down, kRowDown, kH, kE, L->down_expert_stride, &m.hdr[0][0], &m.qnt[0][0]))) return rc;
  if ((rc = weight_maps(L->sh_down, kRowDown, kH, 1, 0, &m.hdr[1][0], &m.qnt[1][0]))) return rc;
  m.hdr[0][1] = m.hdr[0][0];
  m.qnt[0][1] = m.qnt[0][0];
  m.hdr[1][1] = m.hdr[1][0];
  m.qnt[1][1] = m.qnt[1][0];
  const MapKey kb{s16, 1, 1, (uint64_t)kI, (uint64_t)9 * Ts, 0, (uint64_t)kI * 2, 0, 64, 64};
  if ((rc = encode_map(kb, &m.b))) return rc;
  for (int p = 0; p < 5; ++p) {
    const MapKey ky{y, 2, 0, (uint64_t)kH, (uint64_t)9 * Ts, 0, (uint64_t)kH * 4, 0, 32, (uint32_t)(16 >> p)};
    if ((rc = encode_map(ky, &m.st[p]))) return rc;
  }
  return B200MOE_OK;
}

// experts: the call runs the grouped GEMMs, which take Q4_K expert and shared rows only.
int check_prefill_layer(const b200moe_layer *L, const char *who, bool experts = true) {
  if (!L || !L->gate || !L->up || !L->down || !L->sh_gate || !L->sh_up || !L->sh_down || !L->router_w ||
      !L->sh_gate_w)
    return b2host::set_error(B200MOE_EINVAL, "%s: layer is NULL or has a NULL weight pointer", who);
  if (experts && !layer_all_q4k(L))
    return b2host::set_error(B200MOE_EINVAL,
                             "%s: the grouped GEMMs take Q4_K expert and shared rows; this layer has down type %d, "
                             "shared type %d (run it through b200moe_moe_decode)",
                             who, layer_down_type(L), layer_sh_type(L));
  return B200MOE_OK;
}

// The router GEMM's token tile kTM (8 .. 64 in steps of 8): the one whose busiest SM has the
// fewest token rows to multiply -- ceil(CTAs / SMs) CTAs of kTM rows -- and of those the
// largest (more FMAs per shared-memory load). 4096 tokens on 148 SMs: kTM = 56, 296 CTAs, two
// per SM (64 would give 256 CTAs: 108 SMs with two, 40 with one).
template <bool kF32, int kTM>
void router_gemm_launch(const float *xn, int T, const void *wg, const float *bias, uint16_t *logits,
                        cudaStream_t s) {
  k_router_gemm<kF32, kTM><<<dim3((T + kTM - 1) / kTM, kE / 64), 128, rg_smem<kF32, kTM>(), s>>>(xn, T, wg, bias, logits);
}

template <bool kF32, int kTM>
cudaError_t router_gemm_attr() {
  return cudaFuncSetAttribute((const void *)k_router_gemm<kF32, kTM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)rg_smem<kF32, kTM>());
}

template <bool kF32>
cudaError_t router_gemm_attrs() {
  const cudaError_t e[8] = {router_gemm_attr<kF32, 8>(),  router_gemm_attr<kF32, 16>(), router_gemm_attr<kF32, 24>(),
                            router_gemm_attr<kF32, 32>(), router_gemm_attr<kF32, 40>(), router_gemm_attr<kF32, 48>(),
                            router_gemm_attr<kF32, 56>(), router_gemm_attr<kF32, 64>()};
  for (cudaError_t x : e)
    if (x != cudaSuccess) return x;
  return cudaSuccess;
}

int router_tile(int T, int sms) {
  int best = 8;
  long long best_cost = -1;
  for (int tm = 8; tm <= 64; tm += 8) {
    const long long ctas = (long long)((T + tm - 1) / tm) * (kE / 64);
    const long long cost = (ctas + sms - 1) / sms * tm;
    if (best_cost < 0 || cost <= best_cost) {
      best = tm;
      best_cost = cost;
    }
  }
  return best;
}

template <bool kF32>
cudaError_t launch_router_gemm_t(const float *xn, int T, const void *wg, const float *bias, uint16_t *logits,
                                 cudaStream_t s) {
  switch (router_tile(T, g_num_sms > 0 ? g_num_sms : 148)) {
    case 8: router_gemm_launch<kF32, 8>(xn, T, wg, bias, logits, s); break;
    case 16: router_gemm_launch<kF32, 16>(xn, T, wg, bias, logits, s); break;
    case 24: router_gemm_launch<kF32, 24>(xn, T, wg, bias, logits, s); break;
    case 32: router_gemm_launch<kF32, 32>(xn, T, wg, bias, logits, s); break;
    case 40: router_gemm_launch<kF32, 40>(xn, T, wg, bias, logits, s); break;
    case 48: router_gemm_launch<kF32, 48>(xn, T, wg, bias, logits, s); break;
    case 56: router_gemm_launch<kF32, 56>(xn, T, wg, bias, logits, s); break;
    default: router_gemm_launch<kF32, 64>(xn, T, wg, bias, logits, s); break;
  }
  return cudaGetLastError();
}

// Up to kRouterRowsMaxT tokens take the row kernel, more the tiled GEMM (both give the same
// bits). Measured route stage, row kernel / tiled GEMM: 34 / 61 us at 8 tokens, 47 / 63 at 256,
// 63 / 67 at 512, 89 / 78 at 1024.
#ifndef B2_ROUTER_ROWS_MAX_T
#define B2_ROUTER_ROWS_MAX_T 576
#endif
constexpr int kRouterRowsMaxT = B2_ROUTER_ROWS_MAX_T;

cudaError_t launch_router_gemm(bool f32, const float *xn, int T, const void *wg, const float *bias, uint16_t *logits,
                               cudaStream_t s) {
  if (T <= kRouterRowsMaxT) {
    const unsigned ty = (unsigned)((T + kRrTok - 1) / kRrTok);
    if (f32)
      k_router_rows<true><<<dim3(kE / (rr_warps<true>() * rr_rows_per_warp<true>()), ty), 32 * rr_warps<true>(),
                            rr_smem<true>(), s>>>(xn, T, wg, bias, logits);
    else
      k_router_rows<false><<<dim3(kE / (rr_warps<false>() * rr_rows_per_warp<false>()), ty), 32 * rr_warps<false>(),
                             rr_smem<false>(), s>>>(xn, T, wg, bias, logits);
    return cudaGetLastError();
  }
  return f32 ? launch_router_gemm_t<true>(xn, T, wg, bias, logits, s)
             : launch_router_gemm_t<false>(xn, T, wg, bias, logits, s);
}

// Route stage: x (or rmsnorm(resid)) -> x16, ids, wb, sg (each to the given pointer).
int route_stage(const void *x, int x_dtype, const float *resid, float eps, int T, const b200moe_layer *L,
                __half *x16, int32_t *ids, uint16_t *wb, float *sg, const PrefillWS &w, cudaStream_t s) {
  int rc = ensure_gemm_attrs();  // (also the router GEMM's shared-memory size)
  if (rc) return rc;
  B2_CUDA(cudaMemsetAsync(w.err, 0, 4, s));
  k_prep<<<(T + kPrepWarps - 1) / kPrepWarps, 32 * kPrepWarps, 0, s>>>(x, x_dtype, resid, eps, T, L->sh_gate_w,
                                                                   L->router_f32, resid ? L->norm_w : nullptr,
                                                                   w.xn, x16, sg, w.err);
  B2_CUDA(cudaGetLastError());
  B2_CUDA(launch_router_gemm(L->router_f32 != 0, w.xn, T, L->router_w, L->logit_bias, w.logits, s));
  k_route_tok<<<(T + 7) / 8, 256, 0, s>>>(w.logits, T, ids, wb);
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

// Expert stage: grouped GEMMs for the slots whose expert is in [e_lo, e_hi) (+ the shared
// expert when sg != NULL), then the combine into out (accumulate: out += result).
int experts_stage(const __half *x16, int T, const int32_t *ids, const uint16_t *wb, int e_lo, int e_hi,
                  const float *sg, int sh_lo, int sh_hi, const b200moe_layer *L, float *out, int accumulate,
                  const PrefillWS &w, cudaStream_t s, int64_t x16_pitch = kH, const SegOut *seg = nullptr) {
  int rc = ensure_gemm_attrs();
  if (rc) return rc;
  B2_CUDA(cudaMemsetAsync(w.counts, 0, kNE * 4, s));
  k_count<<<(T + 255) / 256, 256, 0, s>>>(T, ids, e_lo, e_hi, w.counts, w.order);
  B2_CUDA(cudaGetLastError());
  if (!sg) sh_lo = sh_hi = 0;
  k_plan<<<1, 512, 0, s>>>(sh_hi - sh_lo, w.counts, w.offsets, w.tiles1, w.tiles2, w.ntiles);
  B2_CUDA(cudaGetLastError());
  k_fill<<<(unsigned)(((int64_t)T * kK + 1023) / 1024), 1024, 0, s>>>(T, sh_lo, sh_hi, ids, wb, e_lo, e_hi, w.offsets,
                                                                   w.counts, w.plist, w.inv, w.wrow);
  B2_CUDA(cudaGetLastError());
  GemmParams g;
  k_gather_x<<<4 * g_num_sms, 256, 0, s>>>(9 * T, w.offsets, w.plist, x16, x16_pitch, w.x16p);
  B2_CUDA(cudaGetLastError());
  rc = gemm_maps(1, L, w.x16p, w.s16, w.y, T, g.m);
  if (rc) return rc;
  g.tiles = w.tiles1;
  g.ntiles = w.ntiles;
  g.wrow = w.wrow;
  g.s16 = w.s16;
  g.y = w.y;
  g.err = w.err;
  k_gemm<1><<<g_num_sms, kGemmThreads, GemmCfg<1>::kSmem, s>>>(g);
  B2_CUDA(cudaGetLastError());
  rc = gemm_maps(2, L, w.x16p, w.s16, w.y, T, g.m);
  if (rc) return rc;
  g.tiles = w.tiles2;
  k_gemm<2><<<g_num_sms, kGemmThreads, GemmCfg<2>::kSmem, s>>>(g);
  B2_CUDA(cudaGetLastError());
  const int64_t nthreads = (int64_t)T * (kH / 4);
  k_combine<<<(unsigned)((nthreads + 255) / 256), 256, 0, s>>>(T, w.y, w.inv, w.offsets, sg, sh_lo, sh_hi, ids,
                                                               w.order, e_lo, e_hi, out, accumulate,
                                                               seg ? *seg : SegOut{});
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

}  // namespace

extern "C" {

size_t b200moe_prefill_workspace_size(int T) {
  return (T <= 0 || T > kMaxTPrefill) ? 0 : prefill_ws_bytes(T);
}

int b200moe_moe_prefill(const void *x, int x_dtype, float *resid, float eps, int T, const b200moe_layer *L,
                        float *out, int32_t *ids_out, void *ws, size_t ws_bytes, void *stream) {
  if (T <= 0 || T > kMaxTPrefill)
    return b2host::set_error(B200MOE_EINVAL, "moe_prefill: T=%d outside [1, %d]", T, kMaxTPrefill);
  if ((!x && !resid) || (!out && !resid) || !ws)
    return b2host::set_error(B200MOE_EINVAL, "moe_prefill: need (x and out) or resid, and ws");
  if (!resid && x_dtype != B200MOE_F32 && x_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "moe_prefill: x_dtype %d is neither F32 nor BF16", x_dtype);
  if ((x && !a16(x)) || (out && !a16(out)) || (resid && !a16(resid)) || !a16(ws))
    return b2host::set_error(B200MOE_EINVAL, "moe_prefill: pointers must be 16-byte aligned");
  if (ws_bytes < prefill_ws_bytes(T))
    return b2host::set_error(B200MOE_ESIZE, "moe_prefill: workspace %zu B < required %zu B", ws_bytes,
                             prefill_ws_bytes(T));
  int rc = check_prefill_layer(L, "moe_prefill");
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const PrefillWS w = carve_prefill(ws, T);
  rc = route_stage(x, x_dtype, resid, eps, T, L, w.x16, w.ids, w.wb, w.sg, w, s);
  if (rc) return rc;
  if (ids_out) B2_CUDA(cudaMemcpyAsync(ids_out, w.ids, (size_t)T * kK * 4, cudaMemcpyDeviceToDevice, s));
  return experts_stage(w.x16, T, w.ids, w.wb, 0, kE, w.sg, 0, T, L, resid ? resid : out, resid ? 1 : 0, w, s);
}

int b200moe_moe_route(const void *x, int x_dtype, float *resid, float eps, int T, const b200moe_layer *L,
                      void *x16_out, int32_t *ids_out, uint16_t *w_out, float *sg_out, void *ws, size_t ws_bytes,
                      void *stream) {
  if (T <= 0 || T > kMaxTPrefill)
    return b2host::set_error(B200MOE_EINVAL, "moe_route: T=%d outside [1, %d]", T, kMaxTPrefill);
  if ((!x && !resid) || !x16_out || !ids_out || !w_out || !sg_out || !ws)
    return b2host::set_error(B200MOE_EINVAL, "moe_route: x or resid, all four outputs and ws are required");
  if (!resid && x_dtype != B200MOE_F32 && x_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "moe_route: x_dtype %d is neither F32 nor BF16", x_dtype);
  if ((x && !a16(x)) || (resid && !a16(resid)) || !a16(x16_out) || !a16(ws))
    return b2host::set_error(B200MOE_EINVAL, "moe_route: pointers must be 16-byte aligned");
  if (ws_bytes < prefill_ws_bytes(T))
    return b2host::set_error(B200MOE_ESIZE, "moe_route: workspace %zu B < required %zu B", ws_bytes,
                             prefill_ws_bytes(T));
  int rc = check_prefill_layer(L, "moe_route", false);
  if (rc) return rc;
  return route_stage(x, x_dtype, resid, eps, T, L, (__half *)x16_out, ids_out, w_out, sg_out, carve_prefill(ws, T),
                     (cudaStream_t)stream);
}

int b200moe_moe_experts(const void *x16, int T, const int32_t *ids, const uint16_t *w_bf16, int e_lo, int e_hi,
                        const float *sg, int sh_lo, int sh_hi, const b200moe_layer *L, float *out, int accumulate,
                        void *ws, size_t ws_bytes, void *stream) {
  if (T <= 0 || T > kMaxTPrefill)
    return b2host::set_error(B200MOE_EINVAL, "moe_experts: T=%d outside [1, %d]", T, kMaxTPrefill);
  if (!x16 || !ids || !w_bf16 || !out || !ws)
    return b2host::set_error(B200MOE_EINVAL, "moe_experts: x16, ids, w_bf16, out and ws are required");
  if (e_lo < 0 || e_hi > kE || e_lo > e_hi)
    return b2host::set_error(B200MOE_EINVAL, "moe_experts: expert range [%d, %d) not within [0, 256)", e_lo, e_hi);
  if (sg && (sh_lo < 0 || sh_hi > T || sh_lo > sh_hi))
    return b2host::set_error(B200MOE_EINVAL, "moe_experts: shared rows [%d, %d) not within [0, %d)", sh_lo, sh_hi, T);
  if (!a16(x16) || !a16(out) || !a16(ws))
    return b2host::set_error(B200MOE_EINVAL, "moe_experts: pointers must be 16-byte aligned");
  if (ws_bytes < prefill_ws_bytes(T))
    return b2host::set_error(B200MOE_ESIZE, "moe_experts: workspace %zu B < required %zu B", ws_bytes,
                             prefill_ws_bytes(T));
  int rc = check_prefill_layer(L, "moe_experts");
  if (rc) return rc;
  const PrefillWS w = carve_prefill(ws, T);
  B2_CUDA(cudaMemsetAsync(w.err, 0, 4, (cudaStream_t)stream));
  return experts_stage((const __half *)x16, T, ids, w_bf16, e_lo, e_hi, sg, sh_lo, sh_hi, L, out, accumulate, w,
                       (cudaStream_t)stream);
}

int b200moe_prefill_status(const void *ws, int T, int *status, void *stream) {
  if (!ws || !status || T <= 0 || T > kMaxTPrefill) return b2host::set_error(B200MOE_EINVAL, "prefill_status: bad args");
  PrefillWS w = carve_prefill(const_cast<void *>(ws), T);
  B2_CUDA(cudaMemcpyAsync(status, w.err, 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  B2_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  return B200MOE_OK;
}

int b200moe_ep_pack(const void *x16, const int32_t *ids, const uint16_t *w_bf16, int T, int rank, int world,
                    void *send_rows, int32_t *pos, void *stream) {
  if (T <= 0 || T > kMaxTPrefill) return b2host::set_error(B200MOE_EINVAL, "ep_pack: T=%d outside [1, %d]", T, kMaxTPrefill);
  if (world < 1 || world > kE || kE % world || rank < 0 || rank >= world)
    return b2host::set_error(B200MOE_EINVAL, "ep_pack: rank %d / world %d (world must divide 256)", rank, world);
  if (!x16 || !ids || !w_bf16 || !send_rows || !pos)
    return b2host::set_error(B200MOE_EINVAL, "ep_pack: x16, ids, w_bf16, send_rows and pos are required");
  if (!a16(x16) || !a16(ids) || !a16(w_bf16) || !a16(send_rows))
    return b2host::set_error(B200MOE_EINVAL, "ep_pack: pointers must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  EpDst dst = {};
  dst.send = (uint8_t *)send_rows;
  k_ep_plan<<<world, 1024, 0, s>>>(T, ids, w_bf16, rank, world, dst, pos);
  B2_CUDA(cudaGetLastError());
  k_ep_copy<<<T, 256, 0, s>>>(T, (const __half *)x16, rank, world, pos, dst);
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

int b200moe_ep_experts(const void *recv_rows, int T, int rank, int world, const float *sg, const b200moe_layer *L,
                       float *partial, void *ws, size_t ws_bytes, void *stream) {
  if (world < 1 || world > kE || kE % world || rank < 0 || rank >= world)
    return b2host::set_error(B200MOE_EINVAL, "ep_experts: rank %d / world %d (world must divide 256)", rank, world);
  const int64_t R = (int64_t)world * T;
  if (T <= 0 || R > kMaxTPrefill)
    return b2host::set_error(B200MOE_EINVAL, "ep_experts: world x T = %lld outside [1, %d]", (long long)R, kMaxTPrefill);
  if (!recv_rows || !sg || !partial || !ws)
    return b2host::set_error(B200MOE_EINVAL, "ep_experts: recv_rows, sg, partial and ws are required");
  if (!a16(recv_rows) || !a16(partial) || !a16(ws))
    return b2host::set_error(B200MOE_EINVAL, "ep_experts: pointers must be 16-byte aligned");
  if (ws_bytes < prefill_ws_bytes((int)R))
    return b2host::set_error(B200MOE_ESIZE, "ep_experts: workspace %zu B < required %zu B (world x T rows)", ws_bytes,
                             prefill_ws_bytes((int)R));
  int rc = check_prefill_layer(L, "ep_experts");
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const PrefillWS w = carve_prefill(ws, (int)R);
  B2_CUDA(cudaMemsetAsync(w.err, 0, 4, s));
  k_ep_unpack<<<(unsigned)((R + 255) / 256), 256, 0, s>>>((int)R, (const uint8_t *)recv_rows, w.ids, w.wb);
  B2_CUDA(cudaGetLastError());
  const int per = kE / world;
  return experts_stage((const __half *)recv_rows, (int)R, w.ids, w.wb, rank * per, (rank + 1) * per, sg, rank * T,
                       rank * T + T, L, partial, 0, w, s, kEpRowHalves);
}

int b200moe_ep_combine(const float *ret, const int32_t *pos, int T, int world, float *out, int accumulate,
                       void *stream) {
  if (T <= 0 || T > kMaxTPrefill || world < 1 || world > kE)
    return b2host::set_error(B200MOE_EINVAL, "ep_combine: T=%d / world=%d out of range", T, world);
  if (!ret || !pos || !out) return b2host::set_error(B200MOE_EINVAL, "ep_combine: ret, pos and out are required");
  if (!a16(ret) || !a16(out)) return b2host::set_error(B200MOE_EINVAL, "ep_combine: pointers must be 16-byte aligned");
  const int64_t n = (int64_t)T * (kH / 4);
  k_ep_sum<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(T, world, ret, pos, out, accumulate);
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

}  // extern "C"

// ---- expert parallelism over peer memory (b200moe_ep_peers)
namespace {
int check_peers(const b200moe_ep_peers *P, const char *who) {
  if (!P) return b2host::set_error(B200MOE_EINVAL, "%s: NULL peers", who);
  if (P->world < 2 || P->world > kMaxPeers || kE % P->world || P->rank < 0 || P->rank >= P->world)
    return b2host::set_error(B200MOE_EINVAL, "%s: rank %d / world %d (peer form: 2..%d ranks dividing 256)", who,
                             P->rank, P->world, kMaxPeers);
  for (int d = 0; d < P->world; ++d)
    if (!P->recv[d] || !P->ret[d] || !P->flag_dispatch[d] || !P->flag_return[d] || !a16(P->recv[d]) ||
        !a16(P->ret[d]))
      return b2host::set_error(B200MOE_EINVAL, "%s: rank %d's buffers are NULL or unaligned", who, d);
  if (!P->epoch || !P->status) return b2host::set_error(B200MOE_EINVAL, "%s: epoch and status are required", who);
  return B200MOE_OK;
}

EpFlags flags_of(const b200moe_ep_peers *P, bool dispatch) {
  EpFlags f = {};
  f.own_flags = dispatch ? P->flag_dispatch[P->rank] : P->flag_return[P->rank];
  for (int d = 0; d < P->world; ++d) f.peer_flags[d] = dispatch ? P->flag_dispatch[d] : P->flag_return[d];
  f.epoch = P->epoch;
  return f;
}
}  // namespace

extern "C" {

int b200moe_ep_dispatch_p2p(const void *x16, const int32_t *ids, const uint16_t *w_bf16, int T,
                            const b200moe_ep_peers *peers, int32_t *pos, void *stream) {
  int rc = check_peers(peers, "ep_dispatch_p2p");
  if (rc) return rc;
  if (T <= 0 || (int64_t)T * peers->world > kMaxTPrefill)
    return b2host::set_error(B200MOE_EINVAL, "ep_dispatch_p2p: T=%d out of range", T);
  if (!x16 || !ids || !w_bf16 || !pos || !a16(x16) || !a16(ids) || !a16(w_bf16))
    return b2host::set_error(B200MOE_EINVAL, "ep_dispatch_p2p: x16, ids, w_bf16 (16-byte aligned) and pos are required");
  cudaStream_t s = (cudaStream_t)stream;
  EpDst dst = {};
  for (int d = 0; d < peers->world; ++d) dst.peer_recv[d] = (uint8_t *)peers->recv[d];
  dst.epoch = peers->epoch;
  k_ep_plan<<<peers->world, 1024, 0, s>>>(T, ids, w_bf16, peers->rank, peers->world, dst, pos);
  B2_CUDA(cudaGetLastError());
  k_ep_copy<<<T, 256, 0, s>>>(T, (const __half *)x16, peers->rank, peers->world, pos, dst);
  B2_CUDA(cudaGetLastError());
  k_ep_signal<<<1, 32, 0, s>>>(peers->world, peers->rank, flags_of(peers, true));
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

int b200moe_ep_experts_p2p(int T, const float *sg, const b200moe_layer *L, const b200moe_ep_peers *peers, void *ws,
                           size_t ws_bytes, void *stream) {
  int rc = check_peers(peers, "ep_experts_p2p");
  if (rc) return rc;
  const int world = peers->world, rank = peers->rank;
  const int64_t R = (int64_t)world * T;
  if (T <= 0 || R > kMaxTPrefill) return b2host::set_error(B200MOE_EINVAL, "ep_experts_p2p: T=%d out of range", T);
  if (!sg || !ws || !a16(ws)) return b2host::set_error(B200MOE_EINVAL, "ep_experts_p2p: sg and ws are required");
  if (ws_bytes < prefill_ws_bytes((int)R))
    return b2host::set_error(B200MOE_ESIZE, "ep_experts_p2p: workspace %zu B < required %zu B", ws_bytes,
                             prefill_ws_bytes((int)R));
  rc = check_prefill_layer(L, "ep_experts_p2p");
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const PrefillWS w = carve_prefill(ws, (int)R);
  B2_CUDA(cudaMemsetAsync(w.err, 0, 4, s));
  k_ep_wait<<<1, 32, 0, s>>>(world, flags_of(peers, true), peers->status);  // every source's rows are in
  B2_CUDA(cudaGetLastError());
  const uint8_t *recv = (const uint8_t *)peers->recv[rank];
  k_ep_unpack<<<(unsigned)((R + 255) / 256), 256, 0, s>>>((int)R, recv, w.ids, w.wb);
  B2_CUDA(cudaGetLastError());
  SegOut seg = {};
  for (int d = 0; d < world; ++d) seg.base[d] = peers->ret[d];
  seg.rows = T;
  seg.rank = rank;
  seg.n = world;
  const int per = kE / world;
  rc = experts_stage((const __half *)recv, (int)R, w.ids, w.wb, rank * per, (rank + 1) * per, sg, rank * T,
                     rank * T + T, L, nullptr, 0, w, s, kEpRowHalves, &seg);
  if (rc) return rc;
  k_ep_signal<<<1, 32, 0, s>>>(world, rank, flags_of(peers, false));
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

int b200moe_ep_combine_p2p(int T, const int32_t *pos, const b200moe_ep_peers *peers, float *out, int accumulate,
                           void *stream) {
  int rc = check_peers(peers, "ep_combine_p2p");
  if (rc) return rc;
  if (T <= 0 || T > kMaxTPrefill || !pos || !out || !a16(out))
    return b2host::set_error(B200MOE_EINVAL, "ep_combine_p2p: T=%d, pos and a 16-byte aligned out are required", T);
  cudaStream_t s = (cudaStream_t)stream;
  k_ep_wait<<<1, 32, 0, s>>>(peers->world, flags_of(peers, false), peers->status);  // every partial row is in
  B2_CUDA(cudaGetLastError());
  const int64_t n = (int64_t)T * (kH / 4);
  k_ep_sum<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(T, peers->world, peers->ret[peers->rank], pos, out,
                                                       accumulate);
  B2_CUDA(cudaGetLastError());
  return B200MOE_OK;
}

}  // extern "C"
