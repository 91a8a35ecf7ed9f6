// grouped.cu -- small-batch MoE decode (2..16 tokens): every distinct expert's rows read ONCE
// per layer and applied to all of its tokens on the tensor cores.
//
// The per-token gather-GEMV kernels re-read an expert's rows for every token that routes to it
// (the reference's own loop reads each hit expert once for all its tokens,
// engine/m3_forward.py:447-465). Here, after the router K1 (decode.cu, which also writes each
// token's x as three int8 digit planes), one layer is:
//   k_plan      one CTA: R2..R5 for every token (route.cuh, the declared rule), the distinct
//               experts in ascending id, and per expert its (token, slot) list in token order;
//   k_gu_grp    CTA = (expert, 32 row pairs): the CTA stages the digit planes of the expert's
//               tokens in shared memory; a warp takes 8 gate rows (MMA rows 0..7) and the 8
//               matching up rows (rows 8..15), streams them from HBM into registers once and,
//               per 32-element sub-block, runs one int8 m16n8k32 MMA per token pair (token A's
//               three digit planes in columns 0..2, token B's in 4..6; imma.cuh) ->
//               s = silu(gate) * up per (token, slot);
//   k_dn_grp    CTA = (expert, 64 down rows): the expert's tokens' s turned into digit planes in
//               shared memory, the same MMA scheme over the 512-long down rows -> the expert
//               outputs per (token, slot), unweighted;
//   k_comb_grp  per token: the slots in ascending expert id, product and sum rounded separately,
//               + sigmoid gate * shared (engine/m3_forward.py:452,464-475), as the other paths.
// The shared expert is expert "0" of both grouped kernels (every token, slot 8); its CTAs are
// always active. Grids are sized for 8T distinct experts; CTAs past the plan's count exit at once.
// Every column of a token pair is reduced by the same two lanes in the same order, so a token's
// values do not depend on its partner or position: a call with two copies of a token gives them
// the same bits. The Q4_K dots carry the exact-product arithmetic of imma.cuh.
#include "common.cuh"
#include "grouped.cuh"
#include "imma.cuh"
#include "route.cuh"

using namespace b2;

namespace b2grp {
namespace {

constexpr int kMaxPairs = kMaxT / 2;
constexpr int kMaxU = kK * kMaxT;      // distinct routed experts at most
constexpr int kGuCtasPerExpert = kI / 8;    // one 8-pair tile per CTA (a K quarter per warp)
constexpr int kDnCtasPerExpert = kH / 64;   // 4 warps x 16 down rows
constexpr uint32_t kNib = 0x0F0F0F0Fu;

struct Plan {
  int n_u;                          // distinct routed experts
  int pad_[3];
  int e[kMaxU];                     // their ids, ascending
  int cnt[kMaxU];                   // tokens per expert
  int off[kMaxU];                   // first entry in tk
  uint16_t tk[kMaxU];               // (token << 4) | slot, expert-major, tokens ascending
  Route rt[kMaxT];                  // per token: ids, weights, combine order
};

static_assert(sizeof(Plan) <= kPlanBytes, "the plan fits its workspace slot");

__device__ __forceinline__ uint2 ldg64(const uint8_t *p) {
  uint2 r;
  asm("ld.global.nc.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;" : "=r"(r.x), "=r"(r.y) : "l"(p), "l"(l2_evict_first()));
  return r;
}

// ------------------------------------------------------------------------- plan
__global__ void __launch_bounds__(512) k_plan(const uint16_t *logits, int T, Plan *P) {
  __shared__ Route rr[kMaxT];
  __shared__ int cnt_s[kE / 32], off_s[kE / 32];
  const int tid = threadIdx.x, warp = tid >> 5;
  pdl_wait();
  pdl_trigger();
  if (warp < T) route_warp(logits + (size_t)warp * kE, &rr[warp]);
  __syncthreads();
  // thread e < 256: expert e's token count, then (block-wide exclusive scans in ascending e) its
  // index among the hit experts and its first entry
  int c = 0;
  if (tid < kE) {
    for (int t = 0; t < T; ++t)
#pragma unroll
      for (int k = 0; k < kK; ++k) c += rr[t].ids[k] == tid;
  }
  const int lane = tid & 31;
  int hu = c ? 1 : 0, ho = c;  // inclusive warp scans of (hit, count)
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xFFFFFFFFu, hu, o), b = __shfl_up_sync(0xFFFFFFFFu, ho, o);
    if (lane >= o) {
      hu += a;
      ho += b;
    }
  }
  if (tid < kE && lane == 31) {
    cnt_s[warp] = hu;  // warp totals (reusing the first 16 slots)
    off_s[warp] = ho;
  }
  __syncthreads();
  int bu = 0, bo = 0;
  for (int w = 0; w < warp && w < kE / 32; ++w) {
    bu += cnt_s[w];
    bo += off_s[w];
  }
  const int u = bu + hu - (c ? 1 : 0), o0 = bo + ho - c;
  if (tid == kE - 1) P->n_u = u + (c ? 1 : 0);
  if (tid < kE && c) {
    P->e[u] = tid;
    P->cnt[u] = c;
    P->off[u] = o0;
    int o = o0;
    for (int t = 0; t < T; ++t)
#pragma unroll
      for (int k = 0; k < kK; ++k)
        if (rr[t].ids[k] == tid) P->tk[o++] = (uint16_t)(t << 4 | k);
  }
  if (tid < T) P->rt[tid] = rr[tid];
}

// The expert of grouped-kernel index ue (0: shared, u + 1: routed u): token count, entry offset
// and whether the CTA has work. Plan fields come from a grid two launches back (complete).
__device__ __forceinline__ bool expert_of(const Plan *pl, int ue, int T, int &cnt, int &off, int &e) {
  if (ue == 0) {
    cnt = T;
    off = 0;
    e = -1;
    return true;
  }
  // all four loads in flight at once (index ue - 1 < 8T is inside the arrays either way)
  const int n_u = __ldcg(&pl->n_u);
  e = __ldcg(&pl->e[ue - 1]);
  cnt = __ldcg(&pl->cnt[ue - 1]);
  off = __ldcg(&pl->off[ue - 1]);
  return ue - 1 < n_u;
}

__device__ __forceinline__ int entry_of(const Plan *pl, int ue, int off, int i) {
  return ue == 0 ? (i << 4 | kK) : (int)__ldcg(&pl->tk[off + i]);
}

// One warp's rows of one super-block, in registers: the headers of rows ra (MMA rows 0..7 =
// lane group g) and rb (rows 8..15) and this lane's 8 quant bytes of each 32-byte group.
struct RowRegs {
  uint4 ha, hb;
  uint2 wa[4], wb[4];
};

__device__ __forceinline__ void load_rows(RowRegs &r, const uint8_t *ra, const uint8_t *rb) {
  const int t = threadIdx.x & 3;
  r.ha = ldg_stream(ra);
  r.hb = ldg_stream(rb);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    r.wa[j] = ldg64(ra + 16 + 32 * j + 8 * t);
    r.wb[j] = ldg64(rb + 16 + 32 * j + 8 * t);
  }
}

// One warp, 16 Q4_K rows over kNsb super-blocks already loaded (rr), against the digit blocks
// dg[i] (i < cnt; block pitch `blk`, plane pitch `pp`, per-sub-block sums at 3 pp, all in the
// super-blocks' own coordinates). fa / fb[p]: this lane's partial sums for token
// 2p + (lane % 4 >= 2) of the pair (rows ra / rb), to be completed by the xor-1 lane.
template <int kNsb>
__device__ __forceinline__ void group_rows(const RowRegs (&rr)[kNsb], const uint8_t *dg, int blk, int pp, int cnt,
                                           float (&fa)[kMaxPairs], float (&fb)[kMaxPairs]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int np = (cnt + 1) >> 1;
  const float flo = (t & 1) ? 1.0f : 65536.0f, fhi = (t & 1) ? 0.0f : 256.0f;
  const int bplane = g & 3, bsel = g >> 2, tsel = t >> 1;
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) fa[p] = fb[p] = 0.0f;
#pragma unroll
  for (int b = 0; b < kNsb; ++b) {
    const uint4 ca = rr[b].ha, cb = rr[b].hb;
    uint32_t al[4][4], ah[4][4];  // [group][A register]: low / high nibbles
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint2 wa = rr[b].wa[j], wb = rr[b].wb[j];
      al[j][0] = wa.x & kNib; al[j][1] = wb.x & kNib; al[j][2] = wa.y & kNib; al[j][3] = wb.y & kNib;
      ah[j][0] = (wa.x >> 4) & kNib; ah[j][1] = (wb.x >> 4) & kNib;
      ah[j][2] = (wa.y >> 4) & kNib; ah[j][3] = (wb.y >> 4) & kNib;
    }
    const Q4kScales sa = q4k_scale_words(ca), sb = q4k_scale_words(cb);
    const float da = f16f(ca.x), db = f16f(cb.x), dma = f16f(ca.x >> 16), dmb = f16f(cb.x >> 16);
#pragma unroll
    for (int p = 0; p < kMaxPairs; ++p) {
      if (p >= np) break;  // warp-uniform
      const int ib = 2 * p + bsel;  // the token whose digit plane this lane supplies as B
      const bool bval = bplane < 3 && ib < cnt;
      const uint8_t *xb = dg + (size_t)(bval ? ib : 0) * blk + bplane * pp + 256 * b + 8 * t;
      int ia0 = 0, ia1 = 0, ib0 = 0, ib1 = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint2 x0 = make_uint2(0u, 0u), x1 = make_uint2(0u, 0u);
        if (bval) {
          x0 = lds64(xb + 64 * j);
          x1 = lds64(xb + 64 * j + 32);
        }
        int d[4], e[4];
        mma_s8(al[j][0], al[j][1], al[j][2], al[j][3], x0.x, x0.y, d);
        mma_s8(ah[j][0], ah[j][1], ah[j][2], ah[j][3], x1.x, x1.y, e);
        const int sa0 = q4k_sc(sa, 2 * j), sa1 = q4k_sc(sa, 2 * j + 1);
        const int sb0 = q4k_sc(sb, 2 * j), sb1 = q4k_sc(sb, 2 * j + 1);
        ia0 += sa0 * d[0] + sa1 * e[0];
        ia1 += sa0 * d[1] + sa1 * e[1];
        ib0 += sb0 * d[2] + sb1 * e[2];
        ib1 += sb0 * d[3] + sb1 * e[3];
      }
      fa[p] = fmaf(da, fmaf(fhi, (float)ia1, flo * (float)ia0), fa[p]);
      fb[p] = fmaf(db, fmaf(fhi, (float)ib1, flo * (float)ib0), fb[p]);
      const int it = 2 * p + tsel;  // this lane's token: the min term over sub-blocks t&1, +2, +4, +6
      if (it < cnt) {
        const float *sx = reinterpret_cast<const float *>(dg + (size_t)it * blk + 3 * pp) + 8 * b;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int sbk = (t & 1) + 2 * q;
          const float n = sx[sbk];
          fa[p] = fmaf(-(dma * (float)q4k_mn(sa, sbk)), n, fa[p]);
          fb[p] = fmaf(-(dmb * (float)q4k_mn(sb, sbk)), n, fb[p]);
        }
      }
    }
  }
}

// ------------------------------------------------------------------------- gate / up
struct GuParams {
  const uint8_t *gate, *up;
  int64_t stride;
  const uint8_t *sh_gate, *sh_up;
  const Plan *plan;
  const uint8_t *xd;  // [T][kXBlk] token digit blocks (K1)
  float *s;           // [T][9][512]
  int T;
};

// CTA = one 8-pair tile of one expert (gate rows on MMA rows 0..7, the matching up rows on
// 8..15); warp w takes K quarter w (super-blocks 2w, 2w+1), so each warp issues all its row loads
// at once. Shared memory: per warp, its K quarter of each token's digit block (kSBlk layout);
// once every warp is done with them, the per-warp part sums [cnt][4][16] in their place.
__global__ void __launch_bounds__(128, 4) k_gu_grp(GuParams P) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int ue = blockIdx.x / kGuCtasPerExpert, tile = blockIdx.x % kGuCtasPerExpert;
  const size_t row_off = (size_t)(8 * tile + g) * kRowUp + 2 * warp * kQB;
  RowRegs rr[2];
  if (ue == 0) {  // the shared expert's rows do not depend on the plan: requested before it is ready
    load_rows(rr[0], P.sh_gate + row_off, P.sh_up + row_off);
    load_rows(rr[1], P.sh_gate + row_off + kQB, P.sh_up + row_off + kQB);
  }
  pdl_wait();
  pdl_trigger();
  int cnt, off, e;
  if (!expert_of(P.plan, ue, P.T, cnt, off, e)) return;
  if (ue != 0) {
    const uint8_t *ra = P.gate + (size_t)e * P.stride + row_off, *rb = P.up + (size_t)e * P.stride + row_off;
    load_rows(rr[0], ra, rb);
    load_rows(rr[1], ra + kQB, rb + kQB);
  }
  // this warp's K quarter of each token's digits: 512 bytes of each plane, 16 sums, 2^-k
  uint8_t *wsm = sm + (size_t)warp * cnt * kSBlk;
  // lane i holds entry i (one load for all tokens); two tokens' loads in flight per step
  const int my_en = lane < cnt ? entry_of(P.plan, ue, off, lane) : 0;
#pragma unroll 2
  for (int i = 0; i < cnt; ++i) {
    const uint8_t *src = P.xd + (size_t)(__shfl_sync(0xFFFFFFFFu, my_en, i) >> 4) * kXBlk;
    uint8_t *dst = wsm + (size_t)i * kSBlk;
    uint4 pv[3], sv = make_uint4(0u, 0u, 0u, 0u);
    float uv = 0.0f;
#pragma unroll
    for (int pl = 0; pl < 3; ++pl)
      pv[pl] = __ldcg(reinterpret_cast<const uint4 *>(src + pl * kXPlane + 512 * warp + 16 * lane));
    if (lane < 4) sv = __ldcg(reinterpret_cast<const uint4 *>(src + 3 * kXPlane + 64 * warp + 16 * lane));
    if (lane == 4) uv = __ldcg(reinterpret_cast<const float *>(src + kXUnOff));
#pragma unroll
    for (int pl = 0; pl < 3; ++pl) *reinterpret_cast<uint4 *>(dst + pl * kSPlane + 16 * lane) = pv[pl];
    if (lane < 4) *reinterpret_cast<uint4 *>(dst + 3 * kSPlane + 16 * lane) = sv;
    if (lane == 4) *reinterpret_cast<float *>(dst + kSUnOff) = uv;
  }
  __syncwarp();
  float fa[kMaxPairs], fb[kMaxPairs];
  group_rows<2>(rr, wsm, kSBlk, kSPlane, cnt, fa, fb);
  __syncthreads();  // every warp's digits are consumed: the part sums take their place
  float *part = reinterpret_cast<float *>(sm);  // [cnt][4 warps][16 rows]
  const int np = (cnt + 1) >> 1;
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) {
    if (p >= np) break;
    const float va = fa[p] + __shfl_xor_sync(0xFFFFFFFFu, fa[p], 1);
    const float vb = fb[p] + __shfl_xor_sync(0xFFFFFFFFu, fb[p], 1);
    const int it = 2 * p + (t >> 1);
    if (!(t & 1) && it < cnt) {
      part[(it * 4 + warp) * 16 + g] = va;
      part[(it * 4 + warp) * 16 + g + 8] = vb;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < cnt * 8; idx += blockDim.x) {  // (token, pair): quarters added in order
    const int it = idx >> 3, pr = idx & 7;
    const float *q = part + it * 64;
    const float gs = __fadd_rn(__fadd_rn(__fadd_rn(q[pr], q[16 + pr]), q[32 + pr]), q[48 + pr]);
    const float us = __fadd_rn(__fadd_rn(__fadd_rn(q[8 + pr], q[24 + pr]), q[40 + pr]), q[56 + pr]);
    const int en = entry_of(P.plan, ue, off, it);
    const float un = __ldcg(reinterpret_cast<const float *>(P.xd + (size_t)(en >> 4) * kXBlk + kXUnOff));
    P.s[((size_t)(en >> 4) * (kK + 1) + (en & 15)) * kI + 8 * tile + pr] =
        __fmul_rn(silu_f(__fmul_rn(gs, un)), __fmul_rn(us, un));
  }
}

// ------------------------------------------------------------------------- down
struct DnParams {
  const uint8_t *down;
  int64_t stride;
  const uint8_t *sh_down;
  const Plan *plan;
  const float *s;  // [T][9][512]
  float *o;        // [T][9][2048] expert outputs before weighting
  int T;
};

__global__ void __launch_bounds__(128, 4) k_dn_grp(DnParams P) {
  extern __shared__ __align__(16) uint8_t sm[];  // [cnt][kSBlk]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int ue = blockIdx.x / kDnCtasPerExpert;
  const int h0 = (blockIdx.x % kDnCtasPerExpert) * 64 + 16 * warp;
  int cnt, off, e;
  // the plan is two grids back: complete once the previous grid lets this one start, so the
  // CTA's rows are requested before the s it needs are ready
  const bool live = expert_of(P.plan, ue, P.T, cnt, off, e);
  RowRegs rr[2];
  if (live) {
    const uint8_t *base = e < 0 ? P.sh_down : P.down + (size_t)e * P.stride;
    const uint8_t *ra = base + (size_t)(h0 + g) * kRowDown, *rb = base + (size_t)(h0 + g + 8) * kRowDown;
    load_rows(rr[0], ra, rb);
    load_rows(rr[1], ra + kQB, rb + kQB);
  }
  pdl_wait();
  pdl_trigger();
  if (!live) return;
  // the expert's tokens' s -> digit planes: warp w takes tokens w, w + 4, ...; lane L elements 16L..16L+15
  for (int i = warp; i < cnt; i += 4) {
    const int en = entry_of(P.plan, ue, off, i);
    const float *sv = P.s + ((size_t)(en >> 4) * (kK + 1) + (en & 15)) * kI + 16 * lane;
    float v[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 f = __ldcg(reinterpret_cast<const float4 *>(sv) + q);
      v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
    }
    uint32_t mx = 0;
#pragma unroll
    for (int q = 0; q < 16; ++q) mx = max(mx, __float_as_uint(v[q]) & 0x7FFFFFFFu);
    mx = __reduce_max_sync(0xFFFFFFFFu, mx);
    const int ks = digit_shift(mx);
    const float ups = pow2i(ks);
    uint32_t pk[3][4] = {};
    int tot = 0;
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int n = __float2int_rn(__fmul_rn(v[q], ups));
      int d[3];
      digits3(n, d[0], d[1], d[2]);
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) pk[pl][q >> 2] |= ((uint32_t)d[pl] & 0xFFu) << (8 * (q & 3));
      tot += n;
    }
    uint8_t *blk = sm + (size_t)i * kSBlk;
#pragma unroll
    for (int pl = 0; pl < 3; ++pl)
      *reinterpret_cast<uint4 *>(blk + pl * kSPlane + 16 * lane) = make_uint4(pk[pl][0], pk[pl][1], pk[pl][2], pk[pl][3]);
    tot += __shfl_xor_sync(0xFFFFFFFFu, tot, 1);  // lanes 2i, 2i+1: sub-block i
    if (!(lane & 1)) reinterpret_cast<float *>(blk + 3 * kSPlane)[lane >> 1] = (float)tot;
    if (lane == 0) *reinterpret_cast<float *>(blk + kSUnOff) = digit_unscale(mx, ks);
  }
  __syncthreads();
  float fa[kMaxPairs], fb[kMaxPairs];
  group_rows<kI / 256>(rr, sm, kSBlk, kSPlane, cnt, fa, fb);
  const int np = (cnt + 1) >> 1;
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) {
    if (p >= np) break;
    const float va = fa[p] + __shfl_xor_sync(0xFFFFFFFFu, fa[p], 1);
    const float vb = fb[p] + __shfl_xor_sync(0xFFFFFFFFu, fb[p], 1);
    const int it = 2 * p + (t >> 1);
    if (!(t & 1) && it < cnt) {
      const int en = entry_of(P.plan, ue, off, it);
      const float un = *reinterpret_cast<const float *>(sm + (size_t)it * kSBlk + kSUnOff);
      float *dst = P.o + ((size_t)(en >> 4) * (kK + 1) + (en & 15)) * kH + h0 + g;
      dst[0] = __fmul_rn(va, un);
      dst[8] = __fmul_rn(vb, un);
    }
  }
}

// ------------------------------------------------------------------------- combine
struct CombParams {
  const Plan *plan;
  const float *o;   // [T][9][2048]
  const float *sg;  // [T]
  float *out;       // [T][2048]
  int accumulate;   // 1: out += result (the residual stream)
  int32_t *ids_out;
  uint16_t *w_out;
};

__global__ void __launch_bounds__(256) k_comb_grp(CombParams P) {
  const int t = blockIdx.x >> 3, h = (blockIdx.x & 7) * 256 + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const Route *r = &P.plan->rt[t];
  const float *ot = P.o + (size_t)t * (kK + 1) * kH + h;
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < kK; ++i) {
    const int slot = __ldcg(&r->order[i]);
    acc = __fadd_rn(acc, __fmul_rn(__ldcg(ot + (size_t)slot * kH), bf16f(__ldcg(&r->wb[slot]))));
  }
  const float res = __fadd_rn(acc, __fmul_rn(__ldcg(P.sg + t), __ldcg(ot + (size_t)kK * kH)));
  float *dst = P.out + (size_t)t * kH + h;
  *dst = P.accumulate ? __fadd_rn(*dst, res) : res;
  if ((blockIdx.x & 7) == 0 && threadIdx.x < kK) {
    if (P.ids_out) P.ids_out[(size_t)t * kK + threadIdx.x] = __ldcg(&r->ids[threadIdx.x]);
    if (P.w_out) P.w_out[(size_t)t * kK + threadIdx.x] = __ldcg(&r->wb[threadIdx.x]);
  }
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern k, unsigned grid, unsigned block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

bool g_attr_done[128] = {};

// k_gu_grp's shared memory for up to T tokens per expert: 4 warps' digit quarters + part sums
constexpr size_t gu_smem(int T) { return (size_t)T * 4 * kSBlk; }
static_assert(4 * kSBlk >= 4 * 16 * 4, "the part sums fit the digit region");

}  // namespace

int run(const Args &a, cudaStream_t s) {
  if (a.T < 2 || a.T > kMaxT) return b2host::set_error(B200MOE_EINVAL, "grouped decode: T=%d outside [2, %d]", a.T, kMaxT);
  int dev = 0;
  B2_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 128 && !g_attr_done[dev]) {
    B2_CUDA(cudaFuncSetAttribute(k_gu_grp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gu_smem(kMaxT)));
    g_attr_done[dev] = true;
  }
  const b200moe_layer *L = a.layer;
  Plan *plan = reinterpret_cast<Plan *>(a.plan);
  B2_CUDA(launch_pdl(k_plan, 1u, 512u, 0, s, (const uint16_t *)a.logits, a.T, plan));
  const unsigned experts = (unsigned)(1 + kK * a.T);
  GuParams pg;
  pg.gate = (const uint8_t *)L->gate;
  pg.up = (const uint8_t *)L->up;
  pg.stride = L->gate_up_expert_stride;
  pg.sh_gate = (const uint8_t *)L->sh_gate;
  pg.sh_up = (const uint8_t *)L->sh_up;
  pg.plan = plan;
  pg.xd = a.xd;
  pg.s = a.s;
  pg.T = a.T;
  B2_CUDA(launch_pdl(k_gu_grp, experts * kGuCtasPerExpert, 128u, gu_smem(a.T), s, pg));
  DnParams pd;
  pd.down = (const uint8_t *)L->down;
  pd.stride = L->down_expert_stride;
  pd.sh_down = (const uint8_t *)L->sh_down;
  pd.plan = plan;
  pd.s = a.s;
  pd.o = a.o;
  pd.T = a.T;
  B2_CUDA(launch_pdl(k_dn_grp, experts * kDnCtasPerExpert, 128u, (size_t)a.T * kSBlk, s, pd));
  CombParams pc;
  pc.plan = plan;
  pc.o = a.o;
  pc.sg = a.sg;
  pc.out = a.out;
  pc.accumulate = a.accumulate;
  pc.ids_out = a.ids_out;
  pc.w_out = a.w_out;
  B2_CUDA(launch_pdl(k_comb_grp, (unsigned)(a.T * 8), 256u, 0, s, pc));
  return B200MOE_OK;
}

}  // namespace b2grp
