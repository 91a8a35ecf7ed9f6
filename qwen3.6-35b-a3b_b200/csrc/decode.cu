// decode.cu -- the gather-GEMV MoE decode path and the router.
//
// Per layer, three kernels chained with programmatic dependent launch (PDL):
//   K1 k_router  : one warp per expert logit (R1). Each warp holds its router row in
//                  registers (loaded before waiting on the previous grid) and its lane's
//                  64-element slice of x (given, or RMSNorm of the residual, computed
//                  redundantly per warp so no CTA barrier is needed). One extra warp computes
//                  the shared-expert gate sigmoid(w_sg . x).
//   K2 k_gateup  : the 8 routed experts + the shared expert (slot 8): streams Q4_K gate/up
//                  row pairs -> s = silu(g) * u. Routed CTAs derive R2..R5 from the logits
//                  with one warp (redundantly per CTA: cheaper than any cross-CTA hand-off);
//                  shared-expert CTAs load their first rows before the dependency resolves.
//   K3 k_down    : derives the route in its prologue (the logits are two grids back) and
//                  loads its down rows into registers while K2 still runs; then
//                  o_e[h] = W_d[e][h].s_e
//                  for the 9 experts and the combine: ascending expert id, product and sum
//                  rounded separately, + gate * shared (engine/m3_forward.py:452-475).
// Q4_K is dequantised in registers straight from 16-byte streaming loads; every weight byte
// is read once per token. K2 / K3 are templates on the layer's block types: Q5_K / Q6_K down
// and a Q8_0 shared expert (the published Q4_K_M file) go through kq_dot.cuh's chunk dots,
// loaded after the dependency resolves.
// Which kernels run (run_layer): 2..16 tokens of a Q4_K layer take K1 (which then also writes
// each token's x as int8 digit planes) and the grouped kernels of grouped.cu, which read each
// distinct expert's rows once for all its tokens; other layers, the stage dumps and the
// no-allocation entry point (whose static scratch has no room for the grouped buffers) take
// K1 -> K2 -> K3. A single token takes the persistent kernel (persist.cu) when it is resident.
#include <mutex>

#include "common.cuh"
#include "grouped.cuh"
#include "imma.cuh"
#include "kq_dot.cuh"
#include "mega.cuh"
#include "route.cuh"

using namespace b2;

namespace {

// ------------------------------------------------------------------------- K1
constexpr int kK1Ctas = kE / 4 + 1;  // 64 router CTAs of 4 warps + 1 shared-gate CTA (one row)
// K1's grid: one row of kK1Ctas CTAs per token up to 16 rows (the rows split the tokens)
inline dim3 k1_grid(int T) { return dim3((unsigned)kK1Ctas, (unsigned)(T < 16 ? T : 16)); }

struct K1Params {
  const void *x;
  int x_dtype;
  const float *resid;  // non-NULL: x = rmsnorm(resid) (* nw)
  const float *nw;     // RMSNorm weight (resid mode) or NULL
  float eps;
  int T;
  const void *wg;        // router weights, bf16 or f32 (wf32)
  const float *bias;
  const void *wsg;       // NULL: router only
  int wf32;              // 1: wg / wsg are f32
  float *xw;             // [T][2048] f32 copy of x for K2 (or NULL)
  uint8_t *xd;           // [T][b2grp::kXBlk] x as digit planes for the grouped path (or NULL)
  uint16_t *logits;      // [T][256]
  float *sg;             // [T]
  uint32_t *status;      // decode status word to clear (the call's first router launch), or NULL
  int bf16_stages;       // 1: the shared gate as speccheck/moe_ref.py's "ref" form rounds it
};

// R1's declared order for one value: lane L holds chunk L's sequential sum; the 32 chunk
// sums are added left to right. Every lane returns the same bits. The partials go through the
// warp's 32-float shared-memory scratch (one store, eight vector loads, 31 dependent adds on
// lane 0) instead of 31 dependent shuffles.
__device__ __forceinline__ float chunk_total(float acc, float *scr) {
  const int lane = threadIdx.x & 31;
  scr[lane] = acc;
  __syncwarp();
  float tot = 0.0f;
  if (lane == 0) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 q = reinterpret_cast<const float4 *>(scr)[i];
      v[4 * i] = q.x; v[4 * i + 1] = q.y; v[4 * i + 2] = q.z; v[4 * i + 3] = q.w;
    }
    tot = v[0];
#pragma unroll
    for (int c = 1; c < 32; ++c) tot = __fadd_rn(tot, v[c]);
  }
  tot = __shfl_sync(0xFFFFFFFFu, tot, 0);
  __syncwarp();
  return tot;
}

// Lane L's 64 elements [64L, 64L+64) of token t's MoE input x, in registers.
__device__ __forceinline__ void load_x_slice(const K1Params &P, int t, int lane, float (&v)[64], float *scr) {
  if (P.resid) {
    const float *r = P.resid + (size_t)t * kH + 64 * lane;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 a = __ldcg(reinterpret_cast<const float4 *>(r + 4 * i));
      v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 64; ++i) ss = __fmaf_rn(v[i], v[i], ss);
    const float tot = chunk_total(ss, scr);
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, 2048.0f), P.eps)));
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __fmul_rn(v[i], rs);
    if (P.nw) {  // Form A weight, a second rounding
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 w = __ldg(reinterpret_cast<const float4 *>(P.nw + 64 * lane + 4 * i));
        v[4 * i] = __fmul_rn(v[4 * i], w.x); v[4 * i + 1] = __fmul_rn(v[4 * i + 1], w.y);
        v[4 * i + 2] = __fmul_rn(v[4 * i + 2], w.z); v[4 * i + 3] = __fmul_rn(v[4 * i + 3], w.w);
      }
    }
  } else if (P.x_dtype == B200MOE_BF16) {
    const uint16_t *xb = reinterpret_cast<const uint16_t *>(P.x) + (size_t)t * kH + 64 * lane;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 u = __ldcg(reinterpret_cast<const uint4 *>(xb + 8 * i));
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[8 * i + 2 * q] = bf16f(uw[q]);
        v[8 * i + 2 * q + 1] = bf16f(uw[q] >> 16);
      }
    }
  } else {
    const float *xf = reinterpret_cast<const float *>(P.x) + (size_t)t * kH + 64 * lane;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 a = __ldcg(reinterpret_cast<const float4 *>(xf + 4 * i));
      v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
    }
  }
}

// One token's x (lane L holds elements 64L..64L+63) as the grouped path's digit block
// (grouped.cuh): three int8 planes of the integer image n = rint(x 2^k), the per-sub-block sums
// of n (lane L: sub-blocks 2L, 2L+1) and 2^-k (imma.cuh).
__device__ __forceinline__ void write_digits(const float (&v)[64], uint8_t *blk, int lane) {
  uint32_t mx = 0;
#pragma unroll
  for (int i = 0; i < 64; ++i) mx = max(mx, __float_as_uint(v[i]) & 0x7FFFFFFFu);
  mx = __reduce_max_sync(0xFFFFFFFFu, mx);
  const int k = digit_shift(mx);
  const float up = pow2i(k);
  int sum[2] = {0, 0};
#pragma unroll
  for (int c = 0; c < 4; ++c) {  // 16 elements per store
    uint32_t pk[3][4] = {};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int n = __float2int_rn(__fmul_rn(v[16 * c + i], up));
      int d[3];
      digits3(n, d[0], d[1], d[2]);
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) pk[pl][i >> 2] |= ((uint32_t)d[pl] & 0xFFu) << (8 * (i & 3));
      sum[c >> 1] += n;
    }
#pragma unroll
    for (int pl = 0; pl < 3; ++pl)
      *reinterpret_cast<uint4 *>(blk + pl * b2grp::kXPlane + 64 * lane + 16 * c) =
          make_uint4(pk[pl][0], pk[pl][1], pk[pl][2], pk[pl][3]);
  }
  float *sx = reinterpret_cast<float *>(blk + 3 * b2grp::kXPlane);
  sx[2 * lane] = (float)sum[0];
  sx[2 * lane + 1] = (float)sum[1];
  if (lane == 0) *reinterpret_cast<float *>(blk + b2grp::kXUnOff) = digit_unscale(mx, k);
}

// kF32: router weights stored as f32 (held as 64 floats per lane) instead of bf16 (32 words).
template <bool kF32>
__global__ void __launch_bounds__(128) k_router(K1Params P) {
  __shared__ __align__(16) float scr_all[4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float *scr = scr_all[warp];
  const bool gate_cta = blockIdx.x == kK1Ctas - 1;
  if (gate_cta && (warp != 0 || !P.wsg)) return;
  const int e = 4 * blockIdx.x + warp;
  // This warp's weight slice (router row e, or w_sg) as f32 values, independent of the previous
  // grid (bf16 widens exactly).
  float wv[64];
  if (kF32) {
    const float *src = gate_cta ? (const float *)P.wsg : (const float *)P.wg + (size_t)e * kH;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint4 u = ldg_stream(src + 64 * lane + 4 * i);
      wv[4 * i] = __uint_as_float(u.x); wv[4 * i + 1] = __uint_as_float(u.y);
      wv[4 * i + 2] = __uint_as_float(u.z); wv[4 * i + 3] = __uint_as_float(u.w);
    }
  } else {
    const uint16_t *src = gate_cta ? (const uint16_t *)P.wsg : (const uint16_t *)P.wg + (size_t)e * kH;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 u = ldg_stream(src + 64 * lane + 8 * i);
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        wv[8 * i + 2 * q] = bf16f(w4[q]);
        wv[8 * i + 2 * q + 1] = bf16f(w4[q] >> 16);
      }
    }
  }
  const float bias = (!gate_cta && P.bias) ? P.bias[e] : 0.0f;
  pdl_wait();
  pdl_trigger();
  if (P.status && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *P.status = 0u;  // no bounded waits here
  // CTA row y takes tokens y, y + gridDim.y, ... (each token's arithmetic is the same in any row)
  for (int t = blockIdx.y; t < P.T; t += gridDim.y) {
    float v[64];
    load_x_slice(P, t, lane, v, scr);
    if (blockIdx.x == 0 && warp == 0 && P.xw) {
      float *g = P.xw + (size_t)t * kH + 64 * lane;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        *reinterpret_cast<float4 *>(g + 4 * i) = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    if (blockIdx.x == 0 && warp == 0 && P.xd) write_digits(v, P.xd + (size_t)t * b2grp::kXBlk, lane);
    float acc = 0.0f;
    if (gate_cta) {  // shared-expert gate: any summation order (tolerance-checked)
#pragma unroll
      for (int i = 0; i < 64; ++i) acc = fmaf(v[i], wv[i], acc);
      float z = warp_sum(acc);
      if (P.bf16_stages) z = bf16r(z);  // F.linear in bf16, then sigmoid rounded to bf16
      const float g = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
      if (lane == 0) P.sg[t] = P.bf16_stages ? bf16r(g) : g;
      continue;
    }
#pragma unroll
    for (int i = 0; i < 64; ++i) acc = __fmaf_rn(v[i], wv[i], acc);  // R1: sequential over the lane's 64
    float tot = chunk_total(acc, scr);
    if (P.bias) tot = __fadd_rn(tot, bias);
    if (lane == 0) P.logits[(size_t)t * kE + e] = f2bf(tot);
  }
}

// Router entry point tail: R2..R5 for token blockIdx.x from the published logits.
__global__ void __launch_bounds__(32) k_route_tail(const uint16_t *logits, int32_t *ids, float *wf, uint16_t *wb) {
  __shared__ Route rr;
  const int t = blockIdx.x;
  pdl_wait();
  route_warp(logits + (size_t)t * kE, &rr);
  if (threadIdx.x < kK) {
    const int r = threadIdx.x;
    if (ids) ids[(size_t)t * kK + r] = rr.ids[r];
    if (wf) wf[(size_t)t * kK + r] = rr.wf[r];
    if (wb) wb[(size_t)t * kK + r] = rr.wb[r];
  }
}

// ------------------------------------------------------------------------- K2
constexpr int kK2RowsPerWarp = 4;
constexpr int kK2Warps = 4;
constexpr int kK2RowsPerCta = kK2RowsPerWarp * kK2Warps;        // 16 row-pairs
constexpr int kK2CtasPerSlot = kI / kK2RowsPerCta;              // 32
constexpr int kK2CtasPerToken = (kK + 1) * kK2CtasPerSlot;       // 288: 8 routed + shared

struct K2Params {
  const uint8_t *gate;
  const uint8_t *up;
  int64_t stride;
  const uint8_t *sh_gate;
  const uint8_t *sh_up;
  const uint16_t *logits;
  const float *xw;
  float *s;
  int bf16_stages;  // dense layers: round gate, up, silu(gate) and s to bf16 (moe_ref "ref" form)
};

// The 8 loads (gate/up x two chunks x {header, quants}) of one row-pair for this lane.
__device__ __forceinline__ void load_rowpair(const uint8_t *rg, const uint8_t *ru, int kb0, int cc, uint4 (&hq)[8]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int kb = kb0 + 4 * h;
    hq[4 * h + 0] = ldg_stream(rg + kb * kQB);
    hq[4 * h + 1] = ldg_stream(rg + kb * kQB + 16 + 16 * cc);
    hq[4 * h + 2] = ldg_stream(ru + kb * kQB);
    hq[4 * h + 3] = ldg_stream(ru + kb * kQB + 16 + 16 * cc);
  }
}

// kShQ8: the shared expert's gate / up rows are Q8_0 (2176 B), dotted chunk by chunk.
template <bool kShQ8>
__global__ void __launch_bounds__(128) k_gateup(K2Params P) {
  __shared__ Route rr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x / kK2CtasPerToken, r = blockIdx.x % kK2CtasPerToken;
  const int k = r / kK2CtasPerSlot;
  const int jbase = (r % kK2CtasPerSlot) * kK2RowsPerCta + warp * kK2RowsPerWarp;
  const int kb0 = lane >> 3, cc = lane & 7;
  if (kShQ8 && k == kK) {  // the whole CTA is in the shared slot
    pdl_wait();
    pdl_trigger();
    XChunk X0, X1;
    load_xchunk(P.xw + (size_t)t * kH, kb0, cc, X0);
    load_xchunk(P.xw + (size_t)t * kH, kb0 + 4, cc, X1);
    constexpr int64_t kRow = row_bytes(B200MOE_TYPE_Q8_0, kH);
    float *sdst = P.s + ((size_t)t * 9 + kK) * kI + jbase;
#pragma unroll 1
    for (int jj = 0; jj < kK2RowsPerWarp; ++jj) {
      const uint8_t *rg = P.sh_gate + (size_t)(jbase + jj) * kRow, *ru = P.sh_up + (size_t)(jbase + jj) * kRow;
      float g = q80_chunk_dot(rg, kb0, cc, X0) + q80_chunk_dot(rg, kb0 + 4, cc, X1);
      float u = q80_chunk_dot(ru, kb0, cc, X0) + q80_chunk_dot(ru, kb0 + 4, cc, X1);
      g = warp_sum(g);
      u = warp_sum(u);
      if (lane == 0) sdst[jj] = __fmul_rn(silu_f(g), u);
    }
    return;
  }
  const uint8_t *gb, *ub;
  uint4 cur[8];
  if (k == kK) {  // shared expert: static rows, load before the dependency resolves
    gb = P.sh_gate;
    ub = P.sh_up;
    load_rowpair(gb + (size_t)jbase * kRowUp, ub + (size_t)jbase * kRowUp, kb0, cc, cur);
  }
  pdl_wait();
  pdl_trigger();
  if (k < kK) {  // routed: R2..R5 from the logits (one warp), then this CTA's expert
    if (warp == 0) route_warp(P.logits + (size_t)t * kE, &rr);
    __syncthreads();
    const int e = rr.ids[k];
    gb = P.gate + (size_t)e * P.stride;
    ub = P.up + (size_t)e * P.stride;
    load_rowpair(gb + (size_t)jbase * kRowUp, ub + (size_t)jbase * kRowUp, kb0, cc, cur);
  }
  XChunk X0, X1;
  load_xchunk(P.xw + (size_t)t * kH, kb0, cc, X0);
  load_xchunk(P.xw + (size_t)t * kH, kb0 + 4, cc, X1);
  float *sdst = P.s + ((size_t)t * 9 + k) * kI + jbase;
#pragma unroll 1
  for (int jj = 0; jj < kK2RowsPerWarp; ++jj) {
    uint4 nxt[8];
    if (jj + 1 < kK2RowsPerWarp)
      load_rowpair(gb + (size_t)(jbase + jj + 1) * kRowUp, ub + (size_t)(jbase + jj + 1) * kRowUp, kb0, cc, nxt);
    float g = q4k_chunk_dot(cur[0], cur[1], cc, X0) + q4k_chunk_dot(cur[4], cur[5], cc, X1);
    float u = q4k_chunk_dot(cur[2], cur[3], cc, X0) + q4k_chunk_dot(cur[6], cur[7], cc, X1);
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) sdst[jj] = __fmul_rn(silu_f(g), u);
#pragma unroll
    for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
  }
}

// Dense (BF16) gate/up rows -- a layer as the Hugging Face checkpoint stores it (fused
// gate_up [E][1024][2048]: gate = rows 0..511 of an expert, up = rows 512..1023). Same grid and
// lane split as k_gateup; rows are read straight from global memory (each lane's two chunks are
// 128 B per row). With bf16_stages the values round where speccheck/moe_ref.py's "ref" form
// rounds them: F.linear outputs (gate, up), F.silu's output and the product.
__global__ void __launch_bounds__(128) k_gateup_dense(K2Params P) {
  __shared__ Route rr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x / kK2CtasPerToken, r = blockIdx.x % kK2CtasPerToken;
  const int k = r / kK2CtasPerSlot;
  const int jbase = (r % kK2CtasPerSlot) * kK2RowsPerCta + warp * kK2RowsPerWarp;
  const int kb0 = lane >> 3, cc = lane & 7;
  constexpr int64_t kRow = row_bytes(B200MOE_TYPE_BF16, kH);
  pdl_wait();
  pdl_trigger();
  const uint8_t *gb = P.sh_gate, *ub = P.sh_up;
  if (k < kK) {  // routed: R2..R5 from the logits (one warp), then this CTA's expert
    if (warp == 0) route_warp(P.logits + (size_t)t * kE, &rr);
    __syncthreads();
    const int e = rr.ids[k];
    gb = P.gate + (size_t)e * P.stride;
    ub = P.up + (size_t)e * P.stride;
  }
  XChunk X0, X1;
  load_xchunk(P.xw + (size_t)t * kH, kb0, cc, X0);
  load_xchunk(P.xw + (size_t)t * kH, kb0 + 4, cc, X1);
  float *sdst = P.s + ((size_t)t * 9 + k) * kI + jbase;
#pragma unroll 1
  for (int jj = 0; jj < kK2RowsPerWarp; ++jj) {
    const uint8_t *rg = gb + (size_t)(jbase + jj) * kRow, *ru = ub + (size_t)(jbase + jj) * kRow;
    float g = bf16_chunk_dot(rg, kb0, cc, X0) + bf16_chunk_dot(rg, kb0 + 4, cc, X1);
    float u = bf16_chunk_dot(ru, kb0, cc, X0) + bf16_chunk_dot(ru, kb0 + 4, cc, X1);
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) {
      if (P.bf16_stages) {
        g = bf16r(g);
        u = bf16r(u);
        sdst[jj] = bf16r(__fmul_rn(bf16r(silu_f(g)), u));
      } else {
        sdst[jj] = __fmul_rn(silu_f(g), u);
      }
    }
  }
}

// ------------------------------------------------------------------------- K3
constexpr int kK3Rows = 8;                       // h rows per CTA
constexpr int kK3CtasPerToken = kH / kK3Rows;    // 256

struct K3Params {
  const uint8_t *down;
  int64_t stride;
  const uint8_t *sh_down;
  const uint16_t *logits;
  const float *s;
  const float *sg;
  float *out;
  int accumulate;  // 1: out += result (the residual stream)
  int32_t *ids_out;
  uint16_t *w_out;
  int bf16_stages;     // dense layers: moe_ref's "ref" form -- expert outputs, every weighted
                       // product, the running routed sum, the gated shared output and the block
                       // output each rounded to bf16 (the sum in ascending expert id)
  float *raw_out;      // [T][8][2048] each slot's expert output before weighting (top-k order), or NULL
  float *routed_out;   // [T][2048] the routed sum, or NULL
  float *shraw_out;    // [T][2048] the shared expert's output before its gate, or NULL
};

// kDn: block type of the routed down rows (Q4_K / Q5_K / Q6_K); kSh: of the shared down rows
// (Q4_K / Q8_0). Q4_K rows are loaded into registers before the dependency resolves, the
// others read after it.
template <int kDn, int kSh>
__global__ void __launch_bounds__(288) k_down(K3Params P) {
  __shared__ Route rr;
  __shared__ float o[9][kK3Rows];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x / kK3CtasPerToken, h0 = (blockIdx.x % kK3CtasPerToken) * kK3Rows;
  // The logits were written by K1 (two grids back), so they are complete before K2 lets this
  // grid start: route now and load this CTA's down rows while K2 still runs.
  if (warp == 0) route_warp(P.logits + (size_t)t * kE, &rr);
  __syncthreads();
  const int half = lane >> 4, kb = (lane >> 3) & 1, cc = lane & 7;
  const bool routed = warp < kK;
  const uint8_t *base = routed ? P.down + (size_t)rr.ids[warp] * P.stride : P.sh_down;
  const bool q4 = routed ? kDn == B200MOE_TYPE_Q4_K : kSh == B200MOE_TYPE_Q4_K;
  uint4 hq[kK3Rows / 2][2];
  if (q4) {
#pragma unroll
    for (int it = 0; it < kK3Rows / 2; ++it) {
      const uint8_t *p = base + (size_t)(h0 + 2 * it + half) * kRowDown + kb * kQB;
      hq[it][0] = ldg_stream(p);
      hq[it][1] = ldg_stream(p + 16 + 16 * cc);
    }
  }
  pdl_wait();
  pdl_trigger();
  XChunk X;
  load_xchunk(P.s + ((size_t)t * 9 + warp) * kI, kb, cc, X);
#pragma unroll
  for (int it = 0; it < kK3Rows / 2; ++it) {
    const int h = h0 + 2 * it + half;
    float v;
    if (q4) v = q4k_chunk_dot(hq[it][0], hq[it][1], cc, X);
    else if (routed) v = row_chunk_dot<kDn>(base + (size_t)h * row_bytes(kDn, kI), kb, cc, X);
    else v = row_chunk_dot<kSh>(base + (size_t)h * row_bytes(kSh, kI), kb, cc, X);
    v = half_warp_sum(v);
    if ((lane & 15) == 0) o[warp][2 * it + half] = v;
  }
  __syncthreads();
  if (threadIdx.x < kK3Rows) {
    const int hh = threadIdx.x;
    float acc = 0.0f, res, shraw = o[8][hh];
    if (P.bf16_stages) {
      shraw = bf16r(shraw);
#pragma unroll
      for (int i = 0; i < kK; ++i) {
        const int slot = rr.order[i];
        acc = bf16r(__fadd_rn(acc, bf16r(__fmul_rn(bf16r(o[slot][hh]), bf16f(rr.wb[slot])))));
      }
      res = bf16r(__fadd_rn(acc, bf16r(__fmul_rn(__ldcg(P.sg + t), shraw))));
    } else {
#pragma unroll
      for (int i = 0; i < kK; ++i) {
        const int slot = rr.order[i];
        acc = __fadd_rn(acc, __fmul_rn(o[slot][hh], bf16f(rr.wb[slot])));
      }
      res = __fadd_rn(acc, __fmul_rn(__ldcg(P.sg + t), shraw));
    }
    float *dst = P.out + (size_t)t * kH + h0 + hh;
    *dst = P.accumulate ? __fadd_rn(*dst, res) : res;
    if (P.routed_out) P.routed_out[(size_t)t * kH + h0 + hh] = acc;
    if (P.shraw_out) P.shraw_out[(size_t)t * kH + h0 + hh] = shraw;
    if (P.raw_out) {
#pragma unroll
      for (int slot = 0; slot < kK; ++slot)
        P.raw_out[((size_t)t * kK + slot) * kH + h0 + hh] = P.bf16_stages ? bf16r(o[slot][hh]) : o[slot][hh];
    }
  }
  if (h0 == 0 && threadIdx.x < kK) {
    if (P.ids_out) P.ids_out[(size_t)t * kK + threadIdx.x] = rr.ids[threadIdx.x];
    if (P.w_out) P.w_out[(size_t)t * kK + threadIdx.x] = rr.wb[threadIdx.x];
  }
}

// ------------------------------------------------------------------------- host side
template <typename Kern, typename... Args>
cudaError_t launch(Kern k, dim3 grid, unsigned block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

constexpr size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

struct DecodeWS {
  float *xw;
  uint16_t *logits;
  float *s;
  float *sg;
  void *xchg;  // cross-CTA exchange area of the persistent single-token kernel
  // the grouped small-batch path (NULL when the workspace has no room for it)
  uint8_t *xd;
  void *plan;
  float *o;
};

// The three-kernel path's workspace (also the no-allocation entry point's static scratch).
constexpr size_t decode_ws_base(int T) {
  return align256((size_t)T * kH * 4) + align256((size_t)T * kE * 2) + align256((size_t)T * 9 * kI * 4) +
         align256((size_t)T * 4) + align256(b2mega::kScratchBytes);
}

constexpr bool grouped_t(int T) { return T >= 2 && T <= b2grp::kMaxT; }

// The grouped path's buffers, after the base layout: x digit blocks, the plan, the unweighted
// expert outputs. Above kMaxT tokens (no grouped path) the size keeps the kMaxT figure, so the
// workspace size never shrinks as T grows: a workspace sized for T tokens serves every smaller T.
constexpr size_t grouped_ws_extra(int T) {
  return T < 2 ? 0
               : align256((size_t)(T < b2grp::kMaxT ? T : b2grp::kMaxT) * b2grp::kXBlk) +
                     align256(b2grp::kPlanBytes) +
                     align256((size_t)(T < b2grp::kMaxT ? T : b2grp::kMaxT) * (kK + 1) * kH * 4);
}

constexpr size_t decode_ws_bytes(int T) { return decode_ws_base(T) + grouped_ws_extra(T); }

DecodeWS carve(void *ws, int T, bool grouped = true) {
  char *p = (char *)ws;
  DecodeWS w;
  w.xw = (float *)p;
  p += align256((size_t)T * kH * 4);
  w.logits = (uint16_t *)p;
  p += align256((size_t)T * kE * 2);
  w.s = (float *)p;
  p += align256((size_t)T * 9 * kI * 4);
  w.sg = (float *)p;
  p += align256((size_t)T * 4);
  w.xchg = p;
  p += align256(b2mega::kScratchBytes);
  w.xd = nullptr;
  w.plan = nullptr;
  w.o = nullptr;
  if (grouped && grouped_t(T)) {
    w.xd = (uint8_t *)p;
    p += align256((size_t)T * b2grp::kXBlk);
    w.plan = p;
    p += align256(b2grp::kPlanBytes);
    w.o = (float *)p;
  }
  return w;
}

bool al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// The decode status word of a carved workspace: inside the persistent kernel's exchange area,
// which that kernel clears before each launch; the three-kernel path's first router launch
// clears it too, so it always describes the last call made on the workspace.
uint32_t *status_word(const DecodeWS &w) {
  return reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(w.xchg) + b2mega::kStatusOffset);
}

int read_status(const DecodeWS &w, int *status, cudaStream_t s, const char *who) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, status_word(w), 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return b2host::cuda_status(e, who);
  *status = (int)v;
  return B200MOE_OK;
}

int check_layer(const b200moe_layer *L, const char *who) {
  if (!L) return b2host::set_error(B200MOE_EINVAL, "%s: NULL layer", who);
  if (!L->gate || !L->up || !L->down || !L->sh_gate || !L->sh_up || !L->sh_down || !L->router_w || !L->sh_gate_w)
    return b2host::set_error(B200MOE_EINVAL, "%s: layer has a NULL weight pointer", who);
  if (!al16(L->gate) || !al16(L->up) || !al16(L->down) || !al16(L->sh_gate) || !al16(L->sh_up) ||
      !al16(L->sh_down) || !al16(L->router_w) || !al16(L->sh_gate_w))
    return b2host::set_error(B200MOE_EINVAL, "%s: weight pointers must be 16-byte aligned", who);
  const int dt = layer_down_type(L), st = layer_sh_type(L), gt = layer_gate_type(L);
  if (gt == B200MOE_TYPE_BF16) {  // dense: every matrix BF16 as the checkpoint stores it
    if (dt != B200MOE_TYPE_BF16 || st != B200MOE_TYPE_BF16)
      return b2host::set_error(B200MOE_EINVAL, "%s: a dense (BF16) layer needs down_type and sh_type BF16(30), got %d / %d",
                               who, L->down_type, L->sh_type);
    if (L->gate_up_expert_stride < (int64_t)kI * row_bytes(B200MOE_TYPE_BF16, kH) || (L->gate_up_expert_stride & 15) ||
        L->down_expert_stride < (int64_t)kH * row_bytes(B200MOE_TYPE_BF16, kI) || (L->down_expert_stride & 15))
      return b2host::set_error(B200MOE_EINVAL, "%s: dense layer strides %lld / %lld too small or unaligned", who,
                               (long long)L->gate_up_expert_stride, (long long)L->down_expert_stride);
    return B200MOE_OK;
  }
  if (gt != B200MOE_TYPE_Q4_K)
    return b2host::set_error(B200MOE_EINVAL, "%s: gate_type %d is not Q4_K(12) or BF16(30)", who, L->gate_type);
  if (dt != B200MOE_TYPE_Q4_K && dt != B200MOE_TYPE_Q5_K && dt != B200MOE_TYPE_Q6_K)
    return b2host::set_error(B200MOE_EINVAL, "%s: down_type %d is not Q4_K(12), Q5_K(13) or Q6_K(14)", who,
                             L->down_type);
  if (st != B200MOE_TYPE_Q4_K && st != B200MOE_TYPE_Q8_0)
    return b2host::set_error(B200MOE_EINVAL, "%s: sh_type %d is not Q4_K(12) or Q8_0(8)", who, L->sh_type);
  if (L->gate_up_expert_stride < (int64_t)kI * kRowUp || (L->gate_up_expert_stride & 15))
    return b2host::set_error(B200MOE_EINVAL, "%s: gate_up_expert_stride %lld invalid", who,
                             (long long)L->gate_up_expert_stride);
  if (L->down_expert_stride < (int64_t)kH * row_bytes(dt, kI) || (L->down_expert_stride & 15))
    return b2host::set_error(B200MOE_EINVAL, "%s: down_expert_stride %lld invalid for down_type %d (at least %lld)",
                             who, (long long)L->down_expert_stride, dt, (long long)(kH * row_bytes(dt, kI)));
  return B200MOE_OK;
}

// K3 for the layer's (down, shared) block types.
cudaError_t launch_down(const b200moe_layer *L, unsigned grid, cudaStream_t s, const K3Params &p);

K1Params k1_params(const void *x, int x_dtype, const float *resid, float eps, int T, const b200moe_layer *L,
                   const DecodeWS &w) {
  K1Params p = {};
  p.x = x;
  p.x_dtype = x_dtype;
  p.resid = resid;
  p.eps = eps;
  p.T = T;
  p.wg = L->router_w;
  p.bias = L->logit_bias;
  p.wsg = L->sh_gate_w;
  p.wf32 = L->router_f32 ? 1 : 0;
  p.nw = resid ? L->norm_w : nullptr;
  p.xw = w.xw;
  p.logits = w.logits;
  p.sg = w.sg;
  return p;
}

// Stage outputs and the arithmetic form of b200moe_moe_decode_stages (NULL: plain decode).
struct Stages {
  int bf16;
  float *raw, *routed, *shraw;
};

// One layer: K1 -> K2 -> K3 on stream s. x given (resid == NULL) or rmsnorm(resid).
// `first`: K1 is the first launch of this API call -- its stream predecessor may be any
// operation (a memcpy node in a captured graph), so it is launched without the PDL attribute.
int run_layer(const void *x, int x_dtype, float *resid, float eps, int T, const b200moe_layer *L, float *out,
              int32_t *ids_out, uint16_t *w_out, const DecodeWS &w, cudaStream_t s, bool first,
              const Stages *st = nullptr) {
  // 2..16 tokens of a Q4_K layer: the grouped path (every distinct expert's rows read once)
  const bool grouped = !st && w.xd && grouped_t(T) && layer_all_q4k(L);
  K1Params p1 = k1_params(x, x_dtype, resid, eps, T, L, w);
  if (first) p1.status = status_word(w);
  p1.bf16_stages = st ? st->bf16 : 0;
  if (grouped) {
    p1.xw = nullptr;
    p1.xd = w.xd;
  }
  if (p1.wf32) B2_CUDA(launch(k_router<true>, k1_grid(T), 128, 0, s, !first, p1));
  else B2_CUDA(launch(k_router<false>, k1_grid(T), 128, 0, s, !first, p1));
  if (grouped) {
    b2grp::Args ga = {};
    ga.T = T;
    ga.layer = L;
    ga.logits = w.logits;
    ga.xd = w.xd;
    ga.sg = w.sg;
    ga.plan = w.plan;
    ga.s = w.s;
    ga.o = w.o;
    ga.out = resid ? resid : out;
    ga.accumulate = resid ? 1 : 0;
    ga.ids_out = ids_out;
    ga.w_out = w_out;
    return b2grp::run(ga, s);
  }
  K2Params p2;
  p2.gate = (const uint8_t *)L->gate;
  p2.up = (const uint8_t *)L->up;
  p2.stride = L->gate_up_expert_stride;
  p2.sh_gate = (const uint8_t *)L->sh_gate;
  p2.sh_up = (const uint8_t *)L->sh_up;
  p2.logits = w.logits;
  p2.xw = w.xw;
  p2.s = w.s;
  p2.bf16_stages = st ? st->bf16 : 0;
  if (layer_dense(L))
    B2_CUDA(launch(k_gateup_dense, (unsigned)(T * kK2CtasPerToken), 32 * kK2Warps, 0, s, true, p2));
  else if (layer_sh_type(L) == B200MOE_TYPE_Q8_0)
    B2_CUDA(launch(k_gateup<true>, (unsigned)(T * kK2CtasPerToken), 32 * kK2Warps, 0, s, true, p2));
  else
    B2_CUDA(launch(k_gateup<false>, (unsigned)(T * kK2CtasPerToken), 32 * kK2Warps, 0, s, true, p2));
  K3Params p3;
  p3.down = (const uint8_t *)L->down;
  p3.stride = L->down_expert_stride;
  p3.sh_down = (const uint8_t *)L->sh_down;
  p3.logits = w.logits;
  p3.s = w.s;
  p3.sg = w.sg;
  p3.out = resid ? resid : out;
  p3.accumulate = resid ? 1 : 0;
  p3.ids_out = ids_out;
  p3.w_out = w_out;
  p3.bf16_stages = st ? st->bf16 : 0;
  p3.raw_out = st ? st->raw : nullptr;
  p3.routed_out = st ? st->routed : nullptr;
  p3.shraw_out = st ? st->shraw : nullptr;
  B2_CUDA(launch_down(L, (unsigned)(T * kK3CtasPerToken), s, p3));
  return B200MOE_OK;
}

cudaError_t launch_down(const b200moe_layer *L, unsigned grid, cudaStream_t s, const K3Params &p) {
  constexpr int Q4 = B200MOE_TYPE_Q4_K, Q5 = B200MOE_TYPE_Q5_K, Q6 = B200MOE_TYPE_Q6_K, Q8 = B200MOE_TYPE_Q8_0;
  const int dt = layer_down_type(L);
  if (layer_dense(L)) return launch(k_down<B200MOE_TYPE_BF16, B200MOE_TYPE_BF16>, grid, 288, 0, s, true, p);
  if (layer_sh_type(L) == Q8) {
    if (dt == Q5) return launch(k_down<Q5, Q8>, grid, 288, 0, s, true, p);
    if (dt == Q6) return launch(k_down<Q6, Q8>, grid, 288, 0, s, true, p);
    return launch(k_down<Q4, Q8>, grid, 288, 0, s, true, p);
  }
  if (dt == Q5) return launch(k_down<Q5, Q4>, grid, 288, 0, s, true, p);
  if (dt == Q6) return launch(k_down<Q6, Q4>, grid, 288, 0, s, true, p);
  return launch(k_down<Q4, Q4>, grid, 288, 0, s, true, p);
}

constexpr int kMaxT = 1 << 16;

// One token through n_layers layers with the persistent kernel (persist.cu): x mode (one
// layer, out = block(x)) when resid is NULL, else resid mode. Same routing as run_layer; the
// Q4_K expert dots run on the tensor cores there (agreeing with run_layer's to ~1e-6 relative).
int run_persistent(const void *x, int x_dtype, float *resid, float eps, int n_layers, const b200moe_layer *layers,
                   float *out, int32_t *ids_out, uint16_t *w_out, const DecodeWS &w, cudaStream_t s) {
  b2mega::Args a = {};
  a.n_layers = n_layers;
  a.eps = eps;
  a.x = x;
  a.x_dtype = x_dtype;
  a.resid = resid;
  a.out = out;
  a.ids_out = ids_out;
  a.w_out = w_out;
  a.scratch = w.xchg;
  a.layers = layers;
  return b2mega::launch(a, s);
}

// ------------------------------------------------------------------------- no-allocation entry
// Scratch for b200moe_moe_decode_noalloc: a fixed, file-scope device array sized for
// B200MOE_NOALLOC_MAX_T tokens (about 505 KB; every GPU that loads this library holds it
// until the process exits). Host code may not use the array's name as a device address, so
// its address is looked up once per device with cudaGetSymbolAddress and cached.
constexpr int kNoAllocMaxT = B200MOE_NOALLOC_MAX_T;
__device__ __align__(256) unsigned char g_noalloc_scratch[decode_ws_base(kNoAllocMaxT)];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[128] = {};

int noalloc_scratch(void **out) {
  int dev = 0;
  B2_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 128) return b2host::set_error(B200MOE_EINVAL, "moe_decode_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // current device
    if (e != cudaSuccess) return b2host::cuda_status(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return B200MOE_OK;
}

}  // namespace

extern "C" {

size_t b200moe_router_workspace_size(int T) { return (T <= 0 || T > kMaxT) ? 0 : decode_ws_bytes(T); }

int b200moe_router(const void *x, int x_dtype, int T, const void *router_w, int router_dtype, const float *logit_bias,
                   uint16_t *logits, int32_t *ids, float *w_f32, uint16_t *w_bf16, void *ws, size_t ws_bytes,
                   void *stream) {
  if (T <= 0 || T > kMaxT) return b2host::set_error(B200MOE_EINVAL, "router: T=%d outside [1, %d]", T, kMaxT);
  if (!x || !router_w || !ws) return b2host::set_error(B200MOE_EINVAL, "router: x, router_w and ws are required");
  if (x_dtype != B200MOE_F32 && x_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "router: x_dtype %d is neither F32 nor BF16", x_dtype);
  if (router_dtype != B200MOE_F32 && router_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "router: router_dtype %d is neither F32 nor BF16", router_dtype);
  if (!al16(x) || !al16(router_w) || !al16(ws) || (logits && !al16(logits)))
    return b2host::set_error(B200MOE_EINVAL, "router: pointers must be 16-byte aligned");
  if (ws_bytes < decode_ws_bytes(T))
    return b2host::set_error(B200MOE_ESIZE, "router: workspace %zu B < required %zu B", ws_bytes, decode_ws_bytes(T));
  cudaStream_t s = (cudaStream_t)stream;
  DecodeWS w = carve(ws, T);
  if (logits) w.logits = logits;
  b200moe_layer L = {};
  L.router_w = router_w;
  L.logit_bias = logit_bias;
  L.router_f32 = router_dtype == B200MOE_F32;
  K1Params p1 = k1_params(x, x_dtype, nullptr, 0.f, T, &L, w);
  p1.wsg = nullptr;
  p1.xw = nullptr;
  if (p1.wf32) B2_CUDA(launch(k_router<true>, k1_grid(T), 128, 0, s, false, p1));
  else B2_CUDA(launch(k_router<false>, k1_grid(T), 128, 0, s, false, p1));
  B2_CUDA(launch(k_route_tail, (unsigned)T, 32, 0, s, true, (const uint16_t *)w.logits, ids, w_f32, w_bf16));
  return B200MOE_OK;
}

size_t b200moe_decode_workspace_size(int T) { return (T <= 0 || T > kMaxT) ? 0 : decode_ws_bytes(T); }

int b200moe_moe_decode(const void *x, int x_dtype, int T, const b200moe_layer *layer, float *out, int32_t *ids_out,
                       uint16_t *w_out, void *ws, size_t ws_bytes, void *stream) {
  if (T <= 0 || T > kMaxT) return b2host::set_error(B200MOE_EINVAL, "moe_decode: T=%d outside [1, %d]", T, kMaxT);
  if (!x || !out || !ws) return b2host::set_error(B200MOE_EINVAL, "moe_decode: x, out and ws are required");
  if (x_dtype != B200MOE_F32 && x_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "moe_decode: x_dtype %d is neither F32 nor BF16", x_dtype);
  if (!al16(x) || !al16(out) || !al16(ws)) return b2host::set_error(B200MOE_EINVAL, "moe_decode: pointers must be 16-byte aligned");
  if (ws_bytes < decode_ws_bytes(T))
    return b2host::set_error(B200MOE_ESIZE, "moe_decode: workspace %zu B < required %zu B", ws_bytes, decode_ws_bytes(T));
  int rc = check_layer(layer, "moe_decode");
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const DecodeWS w = carve(ws, T);
  if (T == 1 && !layer_dense(layer) && b2mega::usable(!layer_all_q4k(layer)))
    return run_persistent(x, x_dtype, nullptr, 0.f, 1, layer, out, ids_out, w_out, w, s);
  return run_layer(x, x_dtype, nullptr, 0.f, T, layer, out, ids_out, w_out, w, s, true);
}

int b200moe_moe_decode_noalloc(const void *x, int x_dtype, int T, const b200moe_layer *layer, float *out,
                               int32_t *ids_out, uint16_t *w_out, void *stream) {
  if (T <= 0 || T > kNoAllocMaxT)
    return b2host::set_error(B200MOE_ESIZE,
                             "moe_decode_noalloc: T=%d outside [1, %d]; the built-in scratch holds at most %d tokens "
                             "(use b200moe_moe_decode with a caller workspace for more)",
                             T, kNoAllocMaxT, kNoAllocMaxT);
  if (!x || !out) return b2host::set_error(B200MOE_EINVAL, "moe_decode_noalloc: x and out are required");
  if (x_dtype != B200MOE_F32 && x_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "moe_decode_noalloc: x_dtype %d is neither F32 nor BF16", x_dtype);
  if (!al16(x) || !al16(out)) return b2host::set_error(B200MOE_EINVAL, "moe_decode_noalloc: pointers must be 16-byte aligned");
  int rc = check_layer(layer, "moe_decode_noalloc");
  if (rc) return rc;
  void *scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  if (T == 1 && !layer_dense(layer) && b2mega::usable(!layer_all_q4k(layer)))
    return run_persistent(x, x_dtype, nullptr, 0.f, 1, layer, out, ids_out, w_out, carve(scratch, T, false),
                          (cudaStream_t)stream);
  return run_layer(x, x_dtype, nullptr, 0.f, T, layer, out, ids_out, w_out, carve(scratch, T, false),
                   (cudaStream_t)stream, true);
}

int b200moe_decode_persistent_formats(int *formats) {
  if (!formats) return b2host::set_error(B200MOE_EINVAL, "decode_persistent_formats: NULL pointer");
  *formats = b2mega::usable(true) ? 1 : 0;
  return B200MOE_OK;
}

int b200moe_decode_persistent_info(int *ctas, int *cluster) {
  const int C = b2mega::cluster_ctas();
  if (ctas) *ctas = C ? b2mega::kCtas : 0;
  if (cluster) *cluster = C;
  return B200MOE_OK;
}

int b200moe_moe_decode_stages(const void *x, int x_dtype, int T, const b200moe_layer *layer,
                              const b200moe_stages *st, float *out, int32_t *ids_out, uint16_t *w_out, void *ws,
                              size_t ws_bytes, void *stream) {
  if (T <= 0 || T > kMaxT) return b2host::set_error(B200MOE_EINVAL, "moe_decode_stages: T=%d outside [1, %d]", T, kMaxT);
  if (!x || !out || !ws || !st) return b2host::set_error(B200MOE_EINVAL, "moe_decode_stages: x, st, out and ws are required");
  if (x_dtype != B200MOE_F32 && x_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "moe_decode_stages: x_dtype %d is neither F32 nor BF16", x_dtype);
  if (!al16(x) || !al16(out) || !al16(ws)) return b2host::set_error(B200MOE_EINVAL, "moe_decode_stages: pointers must be 16-byte aligned");
  if (ws_bytes < decode_ws_bytes(T))
    return b2host::set_error(B200MOE_ESIZE, "moe_decode_stages: workspace %zu B < required %zu B", ws_bytes, decode_ws_bytes(T));
  int rc = check_layer(layer, "moe_decode_stages");
  if (rc) return rc;
  if (st->bf16_stages && (!layer_dense(layer) || x_dtype != B200MOE_BF16))
    return b2host::set_error(B200MOE_EINVAL, "moe_decode_stages: bf16 stages (moe_ref's \"ref\" form) need a dense "
                             "BF16 layer and bf16 x");
  cudaStream_t s = (cudaStream_t)stream;
  const DecodeWS w = carve(ws, T);
  const Stages sv = {st->bf16_stages ? 1 : 0, st->expert_raw, st->routed_sum, st->shared_raw};
  rc = run_layer(x, x_dtype, nullptr, 0.f, T, layer, out, ids_out, w_out, w, s, true, &sv);
  if (rc) return rc;
  if (st->router_logits)
    B2_CUDA(cudaMemcpyAsync(st->router_logits, w.logits, (size_t)T * kE * 2, cudaMemcpyDeviceToDevice, s));
  if (st->shared_gate) B2_CUDA(cudaMemcpyAsync(st->shared_gate, w.sg, (size_t)T * 4, cudaMemcpyDeviceToDevice, s));
  return B200MOE_OK;
}

int b200moe_decode_status(const void *ws, int T, int *status, void *stream) {
  if (!ws || !status || T <= 0 || T > kMaxT)
    return b2host::set_error(B200MOE_EINVAL, "decode_status: ws and status required, T=%d outside [1, %d]", T, kMaxT);
  return read_status(carve(const_cast<void *>(ws), T), status, (cudaStream_t)stream, "decode_status");
}

int b200moe_decode_noalloc_status(int T, int *status, void *stream) {
  if (!status || T <= 0 || T > kNoAllocMaxT)
    return b2host::set_error(B200MOE_EINVAL, "decode_noalloc_status: status required, T=%d outside [1, %d]", T,
                             kNoAllocMaxT);
  void *scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return read_status(carve(scratch, T, false), status, (cudaStream_t)stream, "decode_noalloc_status");
}

int b200moe_debug_decode_faults(long long wait_budget_cycles, int withhold_cta) {
  if (wait_budget_cycles < 0 || withhold_cta < -1 || withhold_cta >= b2mega::kCtas)
    return b2host::set_error(B200MOE_EINVAL, "debug_decode_faults: budget %lld < 0 or CTA %d outside [-1, %d)",
                             wait_budget_cycles, withhold_cta, b2mega::kCtas);
  b2mega::set_fault_hook(wait_budget_cycles, withhold_cta);
  return B200MOE_OK;
}

size_t b200moe_stack_workspace_size(int T, int n_layers) {
  return (T <= 0 || T > kMaxT || n_layers <= 0) ? 0 : decode_ws_bytes(T);
}

int b200moe_stack_decode(float *resid, int T, const b200moe_layer *layers, int n_layers, float eps, int32_t *ids_out,
                         void *ws, size_t ws_bytes, void *stream) {
  if (T <= 0 || T > kMaxT) return b2host::set_error(B200MOE_EINVAL, "stack_decode: T=%d outside [1, %d]", T, kMaxT);
  if (!resid || !layers || !ws || n_layers <= 0)
    return b2host::set_error(B200MOE_EINVAL, "stack_decode: resid, layers, ws required and n_layers > 0");
  if (!al16(resid) || !al16(ws)) return b2host::set_error(B200MOE_EINVAL, "stack_decode: pointers must be 16-byte aligned");
  if (ws_bytes < decode_ws_bytes(T))
    return b2host::set_error(B200MOE_ESIZE, "stack_decode: workspace %zu B < required %zu B", ws_bytes, decode_ws_bytes(T));
  bool q4 = true;  // every layer Q4_K throughout (else the persistent kernel's format variant)
  bool dense = false;  // some layer dense (BF16): the three-kernel path
  for (int l = 0; l < n_layers; ++l) {
    int rc = check_layer(&layers[l], "stack_decode");
    if (rc) return rc;
    q4 = q4 && layer_all_q4k(&layers[l]);
    dense = dense || layer_dense(&layers[l]);
  }
  cudaStream_t s = (cudaStream_t)stream;
  const DecodeWS w = carve(ws, T);
  if (T == 1 && !dense && b2mega::usable(!q4))
    return run_persistent(nullptr, B200MOE_F32, resid, eps, n_layers, layers, nullptr, ids_out, nullptr, w, s);
  for (int l = 0; l < n_layers; ++l) {
    int rc = run_layer(nullptr, B200MOE_F32, resid, eps, T, &layers[l], nullptr,
                       ids_out ? ids_out + (size_t)l * T * kK : nullptr, nullptr, w, s, l == 0);
    if (rc) return rc;
  }
  return B200MOE_OK;
}

}  // extern "C"
