// decode.cu -- the gather-GEMV MoE decode path and the router.
//
// Per layer, three kernels chained with programmatic dependent launch (PDL):
//   K1 k_router_shared : x (given, or RMSNorm of the residual) -> router logits R1 (bf16),
//                        the shared expert's gate/up rows -> s_shared = silu(g)*u, and the
//                        shared-expert gate sigmoid(w_sg.x). Before waiting on the previous
//                        grid it bulk-prefetches its static weight rows into L2.
//   K2 k_routed_gateup : every CTA re-derives R2..R5 (softmax, top-8, renorm, bf16 cast) from
//                        the logits with one warp, then streams its slice of the 8 selected
//                        experts' Q4_K gate/up rows -> s = silu(g)*u.
//   K3 k_down_combine  : re-derives the routing in its prologue, bulk-prefetches its down rows
//                        into L2 while K2 still runs, then computes o_e[h] = W_d[e][h].s_e for
//                        the 8 routed experts + shared, and the combine: ascending expert id,
//                        product and sum rounded separately, + sigmoid gate * shared
//                        (reference engine/m3_forward.py:452-475).
// Q4_K is dequantised in registers straight from 16-byte streaming loads; every weight byte
// is read once per token.
#include <mutex>

#include "common.cuh"

using namespace b2;

namespace {

// ------------------------------------------------------------------------- routing (R2..R5)
struct Route {
  int ids[kK];
  float wf[kK];
  uint16_t wb[kK];
  int order[kK];  // slots sorted by ascending expert id (the combine order)
};

// One warp. R2: m = max logit, e_l = b2_expf(l - m), S = per-lane sequential sums of
// e_{8L..8L+7} then an xor butterfly (16,8,4,2,1), p_l = e_l / S. R3: top-8 by
// (p desc, index asc). R4: s8 = sequential sum in rank order, w = p / s8. R5: bf16 RNE.
// Identical operation order to oracle/c/oracle.c b2o_router.
__device__ void route_warp(const uint16_t *logits_t, Route *rr) {
  const int lane = threadIdx.x & 31;
  const uint4 raw = *reinterpret_cast<const uint4 *>(logits_t + 8 * lane);
  const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf16f(rw[i]);
    v[2 * i + 1] = bf16f(rw[i] >> 16);
  }
  float m = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) m = fmaxf(m, v[i]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  float e[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = b2_expf(__fsub_rn(v[i], m));
  float s = e[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) s = __fadd_rn(s, e[i]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, o));
  float p[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = __fdiv_rn(e[i], s);
  uint32_t taken = 0;
  int ids[kK];
  float pk[kK];
#pragma unroll
  for (int r = 0; r < kK; ++r) {
    uint32_t best = 0;
    int bi = -1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = __float_as_uint(p[i]);
      if (!((taken >> i) & 1u) && (bi < 0 || b > best)) {
        best = b;
        bi = i;
      }
    }
    const uint32_t key = bi >= 0 ? best : 0u;
    const uint32_t mx = __reduce_max_sync(0xFFFFFFFFu, key);
    const uint32_t my = (bi >= 0 && key == mx) ? (uint32_t)(8 * lane + bi) : 0xFFFFu;
    const uint32_t win = __reduce_min_sync(0xFFFFFFFFu, my);
    if (win >= (uint32_t)(8 * lane) && win < (uint32_t)(8 * lane + 8)) taken |= 1u << (win - 8 * lane);
    ids[r] = (int)win;
    pk[r] = __uint_as_float(mx);
  }
  if (lane == 0) {
    float s8 = 0.0f;
#pragma unroll
    for (int r = 0; r < kK; ++r) s8 = __fadd_rn(s8, pk[r]);
#pragma unroll
    for (int r = 0; r < kK; ++r) {
      const float w = (s8 == 0.0f) ? 0.0f : __fdiv_rn(pk[r], s8);
      rr->ids[r] = ids[r];
      rr->wf[r] = w;
      rr->wb[r] = f2bf(w);
      rr->order[r] = r;
    }
    for (int a = 1; a < kK; ++a) {  // stable insertion sort of slots by expert id
      const int cur = rr->order[a];
      int b = a - 1;
      while (b >= 0 && rr->ids[rr->order[b]] > rr->ids[cur]) {
        rr->order[b + 1] = rr->order[b];
        --b;
      }
      rr->order[b + 1] = cur;
    }
  }
  __syncwarp();
}

// ------------------------------------------------------------------------- K1
constexpr int kXPad = 68;  // padded 64-float segment: conflict-free 16-byte smem reads
constexpr int kTB = 8;     // tokens staged per pass
constexpr int kK1Grid = 128;

struct K1Params {
  const void *x;
  int x_dtype;
  const float *resid;  // non-NULL: x = rmsnorm(resid)
  float eps;
  int T;
  const uint16_t *wg;
  const float *bias;
  const uint8_t *sh_gate;
  const uint8_t *sh_up;
  const uint16_t *wsg;
  float *xw;          // [T][2048] f32 copy of x for K2 (or NULL)
  uint16_t *logits;   // [T][256]
  float *s;           // [T][9][512] (slot 8 = shared) or NULL for router-only
  float *sg;          // [T]
};

__device__ __forceinline__ void load_xchunk_smem(const float *xt, int kb, int c, XChunk &x) {
  const int p = chunk_pos(kb, c);
  const float *seg = xt + (p >> 6) * kXPad + (p & 63);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 a = *reinterpret_cast<const float4 *>(seg + 4 * i);
    const float4 b = *reinterpret_cast<const float4 *>(seg + 32 + 4 * i);
    x.lo[4 * i] = a.x; x.lo[4 * i + 1] = a.y; x.lo[4 * i + 2] = a.z; x.lo[4 * i + 3] = a.w;
    x.hi[4 * i] = b.x; x.hi[4 * i + 1] = b.y; x.hi[4 * i + 2] = b.z; x.hi[4 * i + 3] = b.w;
  }
  float sl = 0.f, sh = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) { sl += x.lo[i]; sh += x.hi[i]; }
  x.slo = sl;
  x.shi = sh;
}

// R1's declared order for one value: lane L holds chunk L's sequential sum; the 32 chunk
// sums are added left to right. Every lane returns the same bits.
__device__ __forceinline__ float chunk_total(float acc) {
  float tot = __shfl_sync(0xFFFFFFFFu, acc, 0);
#pragma unroll
  for (int c = 1; c < 32; ++c) tot = __fadd_rn(tot, __shfl_sync(0xFFFFFFFFu, acc, c));
  return tot;
}

__global__ void __launch_bounds__(256) k_router_shared(K1Params P) {
  extern __shared__ float xs[];  // [kTB][32][kXPad]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, cta = blockIdx.x;
  const bool shared = P.s != nullptr;
  if (threadIdx.x == 0) {  // static weights: prefetch before the previous grid finishes
    prefetch_l2(P.wg + (size_t)2 * cta * kH, 2 * kH * 2);
    if (shared) {
      prefetch_l2(P.sh_gate + (size_t)4 * cta * kRowUp, 4 * kRowUp);
      prefetch_l2(P.sh_up + (size_t)4 * cta * kRowUp, 4 * kRowUp);
    }
  }
  // Register-resident weights of this warp's role (one array, reused by role):
  //   warps 0,1       : router row 2*cta+warp, elements 64L..64L+63 (32 words of bf16 pairs)
  //   warps 2..5      : shared gate/up row j = 4*cta+warp-2: {hdr, qs} x {gate, up} x {kb0, kb0+4}
  //   warp 6 of CTA 0 : w_sg elements 64L..64L+63
  uint32_t wr[32];
  const int kb0 = lane >> 3, cc = lane & 7;
  const int j = 4 * cta + warp - 2;
  const bool role_dot = warp < 2 || (warp == 6 && cta == 0 && shared);
  const bool role_shared = warp >= 2 && warp < 6 && shared;
  if (role_dot) {
    const uint16_t *src = warp < 2 ? P.wg + (size_t)(2 * cta + warp) * kH : P.wsg;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 u = ldg_stream(src + 64 * lane + 8 * i);
      wr[4 * i] = u.x; wr[4 * i + 1] = u.y; wr[4 * i + 2] = u.z; wr[4 * i + 3] = u.w;
    }
  } else if (role_shared) {
    const uint8_t *rg = P.sh_gate + (size_t)j * kRowUp, *ru = P.sh_up + (size_t)j * kRowUp;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int kb = kb0 + 4 * h;
      const uint4 q0 = ldg_stream(rg + kb * kQB), q1 = ldg_stream(rg + kb * kQB + 16 + 16 * cc);
      const uint4 q2 = ldg_stream(ru + kb * kQB), q3 = ldg_stream(ru + kb * kQB + 16 + 16 * cc);
      const uint4 qq[4] = {q0, q1, q2, q3};
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        wr[16 * h + 4 * n] = qq[n].x; wr[16 * h + 4 * n + 1] = qq[n].y;
        wr[16 * h + 4 * n + 2] = qq[n].z; wr[16 * h + 4 * n + 3] = qq[n].w;
      }
    }
  }
  pdl_wait();
  pdl_trigger();
  for (int t0 = 0; t0 < P.T; t0 += kTB) {
    const int nb = min(kTB, P.T - t0);
    if (warp < nb) {  // stage token t0+warp: lane L owns elements 64L .. 64L+63
      const int t = t0 + warp;
      float *dst = xs + (warp * 32 + lane) * kXPad;
      float *gdst = (cta == 0 && P.xw) ? P.xw + (size_t)t * kH + 64 * lane : nullptr;
      if (P.resid) {
        const float *r = P.resid + (size_t)t * kH + 64 * lane;
        float ss = 0.0f;
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const float4 a = ldg_f4(r + 4 * i);
          ss = __fmaf_rn(a.x, a.x, ss);
          ss = __fmaf_rn(a.y, a.y, ss);
          ss = __fmaf_rn(a.z, a.z, ss);
          ss = __fmaf_rn(a.w, a.w, ss);
        }
        const float tot = chunk_total(ss);
        const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, 2048.0f), P.eps)));
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const float4 a = ldg_f4(r + 4 * i);
          const float4 v = make_float4(__fmul_rn(a.x, rs), __fmul_rn(a.y, rs), __fmul_rn(a.z, rs), __fmul_rn(a.w, rs));
          *reinterpret_cast<float4 *>(dst + 4 * i) = v;
          if (gdst) *reinterpret_cast<float4 *>(gdst + 4 * i) = v;
        }
      } else if (P.x_dtype == B200MOE_BF16) {
        const uint16_t *xb = reinterpret_cast<const uint16_t *>(P.x) + (size_t)t * kH + 64 * lane;
#pragma unroll 2
        for (int i = 0; i < 8; ++i) {
          const uint4 u = *reinterpret_cast<const uint4 *>(xb + 8 * i);
          const float4 v0 = make_float4(bf16f(u.x), bf16f(u.x >> 16), bf16f(u.y), bf16f(u.y >> 16));
          const float4 v1 = make_float4(bf16f(u.z), bf16f(u.z >> 16), bf16f(u.w), bf16f(u.w >> 16));
          *reinterpret_cast<float4 *>(dst + 8 * i) = v0;
          *reinterpret_cast<float4 *>(dst + 8 * i + 4) = v1;
          if (gdst) {
            *reinterpret_cast<float4 *>(gdst + 8 * i) = v0;
            *reinterpret_cast<float4 *>(gdst + 8 * i + 4) = v1;
          }
        }
      } else {
        const float *xf = reinterpret_cast<const float *>(P.x) + (size_t)t * kH + 64 * lane;
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const float4 v = ldg_f4(xf + 4 * i);
          *reinterpret_cast<float4 *>(dst + 4 * i) = v;
          if (gdst) *reinterpret_cast<float4 *>(gdst + 4 * i) = v;
        }
      }
    }
    __syncthreads();
    if (warp < 2) {  // R1 for expert e, declared 32x64 chunk order
      const int e = 2 * cta + warp;
      const float bias = P.bias ? P.bias[e] : 0.0f;
      for (int tt = 0; tt < nb; ++tt) {
        const float *xt = xs + (tt * 32 + lane) * kXPad;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 a = *reinterpret_cast<const float4 *>(xt + 4 * i);
          acc = __fmaf_rn(a.x, bf16f(wr[2 * i]), acc);
          acc = __fmaf_rn(a.y, bf16f(wr[2 * i] >> 16), acc);
          acc = __fmaf_rn(a.z, bf16f(wr[2 * i + 1]), acc);
          acc = __fmaf_rn(a.w, bf16f(wr[2 * i + 1] >> 16), acc);
        }
        float tot = chunk_total(acc);
        if (P.bias) tot = __fadd_rn(tot, bias);
        if (lane == 0) P.logits[(size_t)(t0 + tt) * kE + e] = f2bf(tot);
      }
    } else if (role_shared) {  // shared expert gate/up row j
      for (int tt = 0; tt < nb; ++tt) {
        const float *xt = xs + tt * 32 * kXPad;
        float g = 0.f, u = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          XChunk X;
          load_xchunk_smem(xt, kb0 + 4 * h, cc, X);
          const uint4 g0 = make_uint4(wr[16 * h], wr[16 * h + 1], wr[16 * h + 2], wr[16 * h + 3]);
          const uint4 g1 = make_uint4(wr[16 * h + 4], wr[16 * h + 5], wr[16 * h + 6], wr[16 * h + 7]);
          const uint4 u0 = make_uint4(wr[16 * h + 8], wr[16 * h + 9], wr[16 * h + 10], wr[16 * h + 11]);
          const uint4 u1 = make_uint4(wr[16 * h + 12], wr[16 * h + 13], wr[16 * h + 14], wr[16 * h + 15]);
          g += q4k_chunk_dot(g0, g1, cc, X);
          u += q4k_chunk_dot(u0, u1, cc, X);
        }
        g = warp_sum(g);
        u = warp_sum(u);
        if (lane == 0) P.s[((size_t)(t0 + tt) * 9 + 8) * kI + j] = __fmul_rn(silu_f(g), u);
      }
    } else if (role_dot) {  // warp 6 of CTA 0: shared expert gate sigmoid(w_sg . x)
      for (int tt = 0; tt < nb; ++tt) {
        const float *xt = xs + (tt * 32 + lane) * kXPad;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 a = *reinterpret_cast<const float4 *>(xt + 4 * i);
          acc = fmaf(a.x, bf16f(wr[2 * i]), acc);
          acc = fmaf(a.y, bf16f(wr[2 * i] >> 16), acc);
          acc = fmaf(a.z, bf16f(wr[2 * i + 1]), acc);
          acc = fmaf(a.w, bf16f(wr[2 * i + 1] >> 16), acc);
        }
        const float z = warp_sum(acc);
        if (lane == 0) P.sg[t0 + tt] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------- router-only tail
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
constexpr int kK2RowsPerCta = kK2RowsPerWarp * kK2Warps;  // 16 row-pairs
constexpr int kK2CtasPerToken = kK * kI / kK2RowsPerCta;  // 256

struct K2Params {
  int T;
  const uint8_t *gate;
  const uint8_t *up;
  int64_t stride;
  const uint16_t *logits;
  const float *xw;
  float *s;
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

__global__ void __launch_bounds__(128) k_routed_gateup(K2Params P) {
  __shared__ Route rr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x / kK2CtasPerToken, r = blockIdx.x % kK2CtasPerToken;
  const int k = r / (kI / kK2RowsPerCta);
  const int jbase = (r % (kI / kK2RowsPerCta)) * kK2RowsPerCta + warp * kK2RowsPerWarp;
  pdl_wait();
  pdl_trigger();
  if (warp == 0) route_warp(P.logits + (size_t)t * kE, &rr);
  const int kb0 = lane >> 3, cc = lane & 7;
  XChunk X0, X1;
  load_xchunk(P.xw + (size_t)t * kH, kb0, cc, X0);
  load_xchunk(P.xw + (size_t)t * kH, kb0 + 4, cc, X1);
  __syncthreads();
  const int e = rr.ids[k];
  const uint8_t *gb = P.gate + (size_t)e * P.stride, *ub = P.up + (size_t)e * P.stride;
  uint4 cur[8], nxt[8];
  load_rowpair(gb + (size_t)jbase * kRowUp, ub + (size_t)jbase * kRowUp, kb0, cc, cur);
#pragma unroll
  for (int jj = 0; jj < kK2RowsPerWarp; ++jj) {
    if (jj + 1 < kK2RowsPerWarp)
      load_rowpair(gb + (size_t)(jbase + jj + 1) * kRowUp, ub + (size_t)(jbase + jj + 1) * kRowUp, kb0, cc, nxt);
    float g = q4k_chunk_dot(cur[0], cur[1], cc, X0) + q4k_chunk_dot(cur[4], cur[5], cc, X1);
    float u = q4k_chunk_dot(cur[2], cur[3], cc, X0) + q4k_chunk_dot(cur[6], cur[7], cc, X1);
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) P.s[((size_t)t * 9 + k) * kI + jbase + jj] = __fmul_rn(silu_f(g), u);
    if (jj + 1 < kK2RowsPerWarp) {
#pragma unroll
      for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
    }
  }
}

// ------------------------------------------------------------------------- K3
constexpr int kK3Rows = 8;                       // h rows per CTA
constexpr int kK3CtasPerToken = kH / kK3Rows;    // 256

struct K3Params {
  int T;
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
};

__global__ void __launch_bounds__(288) k_down_combine(K3Params P) {
  __shared__ Route rr;
  __shared__ float o[9][kK3Rows];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x / kK3CtasPerToken, h0 = (blockIdx.x % kK3CtasPerToken) * kK3Rows;
  // The logits were written two grids back (K1), so they are visible before this grid's
  // own dependency (K2) resolves: route now and prefetch this CTA's down rows into L2.
  if (warp == 0) route_warp(P.logits + (size_t)t * kE, &rr);
  __syncthreads();
  if (warp == 1 && lane < 9) {
    const uint8_t *b = lane < 8 ? P.down + (size_t)rr.ids[lane] * P.stride : P.sh_down;
    prefetch_l2(b + (size_t)h0 * kRowDown, kK3Rows * kRowDown);
  }
  const int half = lane >> 4, kb = (lane >> 3) & 1, cc = lane & 7;
  const uint8_t *base = warp < 8 ? P.down + (size_t)rr.ids[warp] * P.stride : P.sh_down;
  uint4 hq[kK3Rows / 2][2];
#pragma unroll
  for (int it = 0; it < kK3Rows / 2; ++it) {
    const uint8_t *p = base + (size_t)(h0 + 2 * it + half) * kRowDown + kb * kQB;
    hq[it][0] = ldg_stream(p);
    hq[it][1] = ldg_stream(p + 16 + 16 * cc);
  }
  pdl_wait();
  pdl_trigger();
  XChunk X;
  load_xchunk(P.s + ((size_t)t * 9 + warp) * kI, kb, cc, X);
#pragma unroll
  for (int it = 0; it < kK3Rows / 2; ++it) {
    const float v = half_warp_sum(q4k_chunk_dot(hq[it][0], hq[it][1], cc, X));
    if ((lane & 15) == 0) o[warp][2 * it + half] = v;
  }
  __syncthreads();
  if (threadIdx.x < kK3Rows) {
    const int hh = threadIdx.x;
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kK; ++i) {
      const int slot = rr.order[i];
      acc = __fadd_rn(acc, __fmul_rn(o[slot][hh], bf16f(rr.wb[slot])));
    }
    const float res = __fadd_rn(acc, __fmul_rn(P.sg[t], o[8][hh]));
    float *dst = P.out + (size_t)t * kH + h0 + hh;
    *dst = P.accumulate ? __fadd_rn(*dst, res) : res;
  }
  if (h0 == 0 && threadIdx.x < kK) {
    if (P.ids_out) P.ids_out[(size_t)t * kK + threadIdx.x] = rr.ids[threadIdx.x];
    if (P.w_out) P.w_out[(size_t)t * kK + threadIdx.x] = rr.wb[threadIdx.x];
  }
}

// ------------------------------------------------------------------------- host side
template <typename Kern, typename... Args>
cudaError_t launch(Kern k, unsigned grid, unsigned block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
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

size_t k1_smem(int T) { return (size_t)min(T, kTB) * 32 * kXPad * sizeof(float); }

int ensure_attrs() {
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(k_router_shared, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)(kTB * 32 * kXPad * sizeof(float)));
  });
  if (err != cudaSuccess) return b2host::cuda_status(err, "cudaFuncSetAttribute(k_router_shared)");
  return B200MOE_OK;
}

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

struct DecodeWS {
  float *xw;
  uint16_t *logits;
  float *s;
  float *sg;
};

size_t decode_ws_bytes(int T) {
  return align256((size_t)T * kH * 4) + align256((size_t)T * kE * 2) + align256((size_t)T * 9 * kI * 4) +
         align256((size_t)T * 4);
}

DecodeWS carve(void *ws, int T) {
  char *p = (char *)ws;
  DecodeWS w;
  w.xw = (float *)p;
  p += align256((size_t)T * kH * 4);
  w.logits = (uint16_t *)p;
  p += align256((size_t)T * kE * 2);
  w.s = (float *)p;
  p += align256((size_t)T * 9 * kI * 4);
  w.sg = (float *)p;
  return w;
}

bool al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

int check_layer(const b200moe_layer *L, const char *who) {
  if (!L) return b2host::set_error(B200MOE_EINVAL, "%s: NULL layer", who);
  if (!L->gate || !L->up || !L->down || !L->sh_gate || !L->sh_up || !L->sh_down || !L->router_w || !L->sh_gate_w)
    return b2host::set_error(B200MOE_EINVAL, "%s: layer has a NULL weight pointer", who);
  if (!al16(L->gate) || !al16(L->up) || !al16(L->down) || !al16(L->sh_gate) || !al16(L->sh_up) ||
      !al16(L->sh_down) || !al16(L->router_w) || !al16(L->sh_gate_w))
    return b2host::set_error(B200MOE_EINVAL, "%s: weight pointers must be 16-byte aligned", who);
  if (L->gate_up_expert_stride < (int64_t)kI * kRowUp || (L->gate_up_expert_stride & 15))
    return b2host::set_error(B200MOE_EINVAL, "%s: gate_up_expert_stride %lld invalid", who,
                             (long long)L->gate_up_expert_stride);
  if (L->down_expert_stride < (int64_t)kH * kRowDown || (L->down_expert_stride & 15))
    return b2host::set_error(B200MOE_EINVAL, "%s: down_expert_stride %lld invalid", who,
                             (long long)L->down_expert_stride);
  return B200MOE_OK;
}

// One layer: K1 -> K2 -> K3 on stream s. x given (resid == NULL) or rmsnorm(resid).
// `first`: K1 is the first launch of this API call -- its stream predecessor may be any
// operation (a memcpy node in a captured graph), so it is launched without the PDL attribute.
int run_layer(const void *x, int x_dtype, float *resid, float eps, int T, const b200moe_layer *L, float *out,
              int32_t *ids_out, uint16_t *w_out, const DecodeWS &w, cudaStream_t s, bool first) {
  K1Params p1;
  p1.x = x;
  p1.x_dtype = x_dtype;
  p1.resid = resid;
  p1.eps = eps;
  p1.T = T;
  p1.wg = L->router_w;
  p1.bias = L->logit_bias;
  p1.sh_gate = (const uint8_t *)L->sh_gate;
  p1.sh_up = (const uint8_t *)L->sh_up;
  p1.wsg = L->sh_gate_w;
  p1.xw = w.xw;
  p1.logits = w.logits;
  p1.s = w.s;
  p1.sg = w.sg;
  B2_CUDA(launch(k_router_shared, kK1Grid, 256, k1_smem(T), s, !first, p1));
  K2Params p2;
  p2.T = T;
  p2.gate = (const uint8_t *)L->gate;
  p2.up = (const uint8_t *)L->up;
  p2.stride = L->gate_up_expert_stride;
  p2.logits = w.logits;
  p2.xw = w.xw;
  p2.s = w.s;
  B2_CUDA(launch(k_routed_gateup, (unsigned)(T * kK2CtasPerToken), 32 * kK2Warps, 0, s, true, p2));
  K3Params p3;
  p3.T = T;
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
  B2_CUDA(launch(k_down_combine, (unsigned)(T * kK3CtasPerToken), 288, 0, s, true, p3));
  return B200MOE_OK;
}

constexpr int kMaxT = 1 << 16;

}  // namespace

extern "C" {

int b200moe_router(const void *x, int x_dtype, int T, const uint16_t *router_w, const float *logit_bias,
                   uint16_t *logits, int32_t *ids, float *w_f32, uint16_t *w_bf16, void *stream) {
  if (T <= 0 || T > kMaxT) return b2host::set_error(B200MOE_EINVAL, "router: T=%d outside [1, %d]", T, kMaxT);
  if (!x || !router_w || !logits) return b2host::set_error(B200MOE_EINVAL, "router: x, router_w and logits are required");
  if (x_dtype != B200MOE_F32 && x_dtype != B200MOE_BF16)
    return b2host::set_error(B200MOE_EINVAL, "router: x_dtype %d is neither F32 nor BF16", x_dtype);
  if (!al16(x) || !al16(router_w) || !al16(logits))
    return b2host::set_error(B200MOE_EINVAL, "router: pointers must be 16-byte aligned");
  int rc = ensure_attrs();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  K1Params p1 = {};
  p1.x = x;
  p1.x_dtype = x_dtype;
  p1.T = T;
  p1.wg = router_w;
  p1.bias = logit_bias;
  p1.logits = logits;
  B2_CUDA(launch(k_router_shared, kK1Grid, 256, k1_smem(T), s, false, p1));
  B2_CUDA(launch(k_route_tail, (unsigned)T, 32, 0, s, true, (const uint16_t *)logits, ids, w_f32, w_bf16));
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
  rc = ensure_attrs();
  if (rc) return rc;
  return run_layer(x, x_dtype, nullptr, 0.f, T, layer, out, ids_out, w_out, carve(ws, T), (cudaStream_t)stream, true);
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
  for (int l = 0; l < n_layers; ++l) {
    int rc = check_layer(&layers[l], "stack_decode");
    if (rc) return rc;
  }
  int rc = ensure_attrs();
  if (rc) return rc;
  const DecodeWS w = carve(ws, T);
  for (int l = 0; l < n_layers; ++l) {
    rc = run_layer(nullptr, B200MOE_F32, resid, eps, T, &layers[l], nullptr,
                   ids_out ? ids_out + (size_t)l * T * kK : nullptr, nullptr, w, (cudaStream_t)stream, l == 0);
    if (rc) return rc;
  }
  return B200MOE_OK;
}

}  // extern "C"
