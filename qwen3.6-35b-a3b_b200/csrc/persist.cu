// persist.cu -- single-token MoE decode as ONE persistent kernel over a whole layer stack.
//
// Grid: one CTA per SM (cooperative launch, so every CTA is resident), 288 threads (9 warps).
// Every value one CTA hands to the others travels as a single 64-bit word
// (phase tag << 32 | value bits) written with one relaxed store: a reader polls the words it
// needs until each carries the expected tag, so no fence, no flag and no second round trip
// sits between producer and consumer. Tags are 3l + p + 1 (layer l, phase p); the exchange
// area is cleared before every launch. Every poll and mbarrier wait is bounded (~1 s); a CTA
// that gives up raises the abort word, which ends every other CTA's polls.
//
// Each CTA keeps the whole residual in shared memory and applies every layer's 2048 deltas
// itself, so all CTAs hold identical residuals. Per layer l:
//   R  poll the 2048 deltas of layer l-1; resid += delta; rs = 1/sqrt(mean(resid^2) + eps)
//      (declared chunk order); this CTA's router rows (c and c + n of the 257 = 256 logits +
//      the shared-expert gate, staged in shared memory one layer ahead) -> tagged logits.
//   S  one warp polls the 256 logits and selects the top 8 (R3); the CTA then issues all
//      bulk copies of its routed rows of this layer at once -- gate/up row pairs [q0, q0+nq)
//      of the flattened (slot, j) space in 4 chunks with one mbarrier each, and down rows
//      [h0, h0+nh) of the 8 experts -- and the warp finishes R2, R4, R5 meanwhile.
//   G  s[k][j] = silu(gate . x) * (up . x) for the CTA's shared-expert row pairs (prefetched
//      one layer ahead) and routed row pairs, chunk by chunk as they land -> tagged s.
//   D  poll the 9 x 512 s; o[k][h] = down_k[h] . s_k for the 9 experts and the CTA's h rows;
//      combine in ascending expert id + sg * shared -> tagged deltas (last layer: the final
//      residual rows, or out in single-layer mode).
// Shared-memory vectors use a padded layout (64-float segments at a 68-float pitch) so the
// per-lane sequential reads of the declared orders and the Q4_K chunk gathers are free of
// bank conflicts.
//
// The arithmetic of every value (RMSNorm, R1 logits in the declared chunk order, R2..R5,
// per-lane Q4_K chunk dots, warp sums, SiLU, combine order, residual add) is the same sequence
// of operations as the three-kernel path in decode.cu, so both paths give identical bits.
#include "common.cuh"
#include "mega.cuh"
#include "route.cuh"
#include "tc.cuh"

using namespace b2;

namespace {

constexpr int kThreads = 288;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxLayers = 64;             // layers per launch (kernel parameter space)
constexpr int kRouterUnits = kE / 2 + 1;   // 128 logit pairs + the shared-expert gate
constexpr int kMinCtas = kRouterUnits;     // one router unit per CTA
constexpr int kRowPair = 2 * kRowUp;       // 2304 B: gate row + up row
constexpr int kRouterRowBytes = kH * 2;    // 4096 B of bf16
constexpr int kGuChunks = 4;               // routed gate/up arrival chunks (one mbarrier each)
constexpr int kGuChunk = 8;                // row pairs per chunk (capq <= 32)
constexpr int kPadSeg = 68;                // padded pitch of a 64-float segment
constexpr int kResPad = kH / 64 * kPadSeg;   // 2176 floats
constexpr int kSPad = kI / 64 * kPadSeg;     // 544 floats per expert slot

// exchange area slots (see mega.cuh): per CTA c, line-aligned, written by c only
//   logits: word 0 = logits 2c | 2c+1 << 16 (c < 128) or the shared-expert gate (c = 128)
//   s:      its routed s values (flattened (slot, j) order from q0), then its shared ones
//   deltas: its residual deltas h0 .. h0+nh-1
constexpr int kSlotLogits = 16, kSlotS = 32, kSlotDelta = 16;  // 64-bit words

__host__ __device__ inline int split_at(int total, int n, int c) { return (int)(((long long)total * c) / n); }
__host__ __device__ inline int pad(int i) { return (i >> 6) * kPadSeg + (i & 63); }

struct Geo {
  int q0, nq;  // routed gate/up row pairs: flattened (slot, j) indices [q0, q0 + nq)
  int j0, nj;  // shared-expert gate/up row pairs [j0, j0 + nj)
  int h0, nh;  // down rows [h0, h0 + nh)
  int nrt;     // router rows of unit c: 2 (logits 2c, 2c+1), 1 (c == 128: gate), 0
};

__host__ __device__ inline Geo geo(int c, int n) {
  Geo g;
  g.q0 = split_at(kK * kI, n, c);
  g.nq = split_at(kK * kI, n, c + 1) - g.q0;
  g.j0 = split_at(kI, n, c);
  g.nj = split_at(kI, n, c + 1) - g.j0;
  g.h0 = split_at(kH, n, c);
  g.nh = split_at(kH, n, c + 1) - g.h0;
  g.nrt = c < kE / 2 ? 2 : (c == kE / 2 ? 1 : 0);
  return g;
}

struct MegaParams {
  int n_layers;
  float eps;
  const void *x;
  int x_dtype;
  float *resid;
  float *out;
  int32_t *ids_out;
  uint16_t *w_out;
  uint8_t *xchg;         // exchange area (mega.cuh layout)
  int capq, capj, caph;  // per-CTA maxima of nq, nj, nh for this grid
  int off_s, off_rt, off_gu, off_dn, off_o, off_rr, off_tab, off_bar;
  b200moe_layer L[kMaxLayers];
};

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_tagged(uint64_t *p, uint32_t tag, uint32_t bits) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((uint64_t)tag << 32) | bits) : "memory");
}

// Bounded mbarrier wait that suspends the thread (hint: 20 us) instead of spinning, so idle
// warps leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kWaitBudgetCycles) return false;
  }
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Global -> shared bulk copy (no multicast), completion counted in bytes on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_normal() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void ld_relaxed_v2u64(const uint64_t *p, uint64_t &a, uint64_t &b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Gather the tagged words of every CTA's slot (slot pitch `pitch` words, cnt(c) words used) into
// the CTA, in two stages: (1) thread t < n polls word 0 of slot t until it carries `tag` -- one
// cheap load per writer while the writers are still busy; (2) after a barrier every thread reads
// its share of all slots' words (64-bit pairs, coalesced) and re-polls only words whose tag is
// not there yet. sink(c, i, bits) receives word i of slot c. Returns false (CTA-uniform) on abort
// or after the wait budget.
template <int kPitch, int kMaxPer, typename Cnt, typename Sink>
__device__ __forceinline__ bool gather_slots(const uint64_t *base, int n, uint32_t tag, const uint32_t *abort_word,
                                             Cnt cnt, Sink sink) {
  const long long t0 = clock64();
  bool fail = false;
  if ((int)threadIdx.x < n) {
    const uint64_t *w0 = base + (size_t)threadIdx.x * kPitch;
    for (int it = 1; (uint32_t)(ld_relaxed_u64(w0) >> 32) != tag; ++it) {
      if ((it & 15) == 0 && (ld_relaxed_u32(abort_word) != 0u || clock64() - t0 > kWaitBudgetCycles)) {
        fail = true;
        break;
      }
    }
  }
  if (__syncthreads_or(fail)) return false;
  constexpr int kPairs = kPitch / 2;
  uint32_t pending = 0;  // two bits per pair
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int pr = threadIdx.x + k * kThreads;
    if (pr < n * kPairs) {
      const int i = 2 * (pr % kPairs), m = cnt(pr / kPairs);
      pending |= ((i < m ? 1u : 0u) | (i + 1 < m ? 2u : 0u)) << (2 * k);
    }
  }
  for (int it = 1; pending && !fail; ++it) {
#pragma unroll
    for (int k = 0; k < kMaxPer; ++k) {
      const uint32_t want = (pending >> (2 * k)) & 3u;
      if (!want) continue;
      const int pr = threadIdx.x + k * kThreads;
      uint64_t a, b;
      ld_relaxed_v2u64(base + 2 * (size_t)pr, a, b);
      const int c = pr / kPairs, i = 2 * (pr % kPairs);
      if ((want & 1u) && (uint32_t)(a >> 32) == tag) {
        sink(c, i, (uint32_t)a);
        pending &= ~(1u << (2 * k));
      }
      if ((want & 2u) && (uint32_t)(b >> 32) == tag) {
        sink(c, i + 1, (uint32_t)b);
        pending &= ~(2u << (2 * k));
      }
    }
    if (pending && (it & 15) == 0 && (ld_relaxed_u32(abort_word) != 0u || clock64() - t0 > kWaitBudgetCycles))
      fail = true;
  }
  return !__syncthreads_or(fail);
}

// x values of chunk (kb, c) from a padded row, each scaled by rs (1.0f: unscaled).
__device__ __forceinline__ void xchunk_pad(const float *row, float rs, int kb, int c, XChunk &x) {
  const int p = (4 * kb + (c >> 1)) * kPadSeg + 16 * (c & 1);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 a = *reinterpret_cast<const float4 *>(row + p + 4 * i);
    const float4 b = *reinterpret_cast<const float4 *>(row + p + 32 + 4 * i);
    x.lo[4 * i] = __fmul_rn(a.x, rs); x.lo[4 * i + 1] = __fmul_rn(a.y, rs);
    x.lo[4 * i + 2] = __fmul_rn(a.z, rs); x.lo[4 * i + 3] = __fmul_rn(a.w, rs);
    x.hi[4 * i] = __fmul_rn(b.x, rs); x.hi[4 * i + 1] = __fmul_rn(b.y, rs);
    x.hi[4 * i + 2] = __fmul_rn(b.z, rs); x.hi[4 * i + 3] = __fmul_rn(b.w, rs);
  }
  float sl = 0.f, sh = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) { sl += x.lo[i]; sh += x.hi[i]; }
  x.slo = sl;
  x.shi = sh;
}

__device__ __forceinline__ float chunk_total32(float acc) {
  float tot = __shfl_sync(0xFFFFFFFFu, acc, 0);
#pragma unroll
  for (int c = 1; c < 32; ++c) tot = __fadd_rn(tot, __shfl_sync(0xFFFFFFFFu, acc, c));
  return tot;
}

enum { kBarRt0 = 0, kBarRt1, kBarGu0, kBarDn = kBarGu0 + kGuChunks, kBarShGu, kBarShDn, kNumBars };

__global__ void __launch_bounds__(kThreads, 1) k_mega(const __grid_constant__ MegaParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  float *res_s = reinterpret_cast<float *>(smem);                 // [kResPad] residual (or x)
  float *s_s = reinterpret_cast<float *>(smem + P.off_s);         // [9][kSPad]
  uint8_t *rt = smem + P.off_rt;   // [2 layers][2 rows][4096]
  uint8_t *gu_g = smem + P.off_gu;                            // [capq routed + capj shared] gate rows
  uint8_t *gu_u = gu_g + (size_t)(P.capq + P.capj) * kRowUp;  // the matching up rows
  uint8_t *dn = smem + P.off_dn;   // [9][caph] down rows
  float *o_s = reinterpret_cast<float *>(smem + P.off_o);  // [9][caph]
  Route *rr = reinterpret_cast<Route *>(smem + P.off_rr);
  uint2 *lg16 = reinterpret_cast<uint2 *>(smem + P.off_rr + 128);  // [64] the 256 bf16 logits
  Geo *tab = reinterpret_cast<Geo *>(smem + P.off_tab);              // [n] every CTA's work ranges
  uint16_t *lgp = reinterpret_cast<uint16_t *>(lg16 + 64);           // [2] this CTA's logit pair
  float *s_out = reinterpret_cast<float *>(lg16 + 66);               // [32] this CTA's s values
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + P.off_bar);
  float *misc = reinterpret_cast<float *>(bar + kNumBars);  // [1] sg

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, n = gridDim.x;
  const Geo G = geo(c, n);
  uint32_t *abort_word = reinterpret_cast<uint32_t *>(P.xchg);  // [1]: status for the host
  uint64_t *tl = reinterpret_cast<uint64_t *>(P.xchg + b2mega::kXLogits);
  uint64_t *ts = reinterpret_cast<uint64_t *>(P.xchg + b2mega::kXS);
  uint64_t *td = reinterpret_cast<uint64_t *>(P.xchg + b2mega::kXDelta);
  const uint64_t pol_first = l2_evict_first(), pol_normal = l2_evict_normal();

  uint32_t armed = 0;  // thread 0: barriers with a phase in flight
  uint32_t ph[kNumBars];
#pragma unroll
  for (int b = 0; b < kNumBars; ++b) ph[b] = 0;

  auto issue_router_rows = [&](int l) {  // thread 0: layer l's router rows -> rt[l & 1], one copy
    uint64_t *b = bar + kBarRt0 + (l & 1);
    mbar_expect_tx(b, (uint32_t)G.nrt * kRouterRowBytes);
    if (G.nrt > 0) {
      const void *src = G.nrt == 2 ? (const void *)((const uint16_t *)P.L[l].router_w + (size_t)(2 * c) * kH)
                                   : P.L[l].sh_gate_w;
      bulk_g2s(rt + (l & 1) * 2 * kRouterRowBytes, src, (uint32_t)G.nrt * kRouterRowBytes, b, pol_normal);
    }
    armed |= 1u << (kBarRt0 + (l & 1));
  };
  auto issue_shared_gu = [&](int l) {  // thread 0: layer l's shared-expert gate/up rows, 2 copies
    mbar_expect_tx(bar + kBarShGu, (uint32_t)G.nj * kRowPair);
    if (G.nj > 0) {
      const size_t off = (size_t)G.j0 * kRowUp;
      bulk_g2s(gu_g + (size_t)P.capq * kRowUp, (const uint8_t *)P.L[l].sh_gate + off, G.nj * kRowUp, bar + kBarShGu,
               pol_normal);
      bulk_g2s(gu_u + (size_t)P.capq * kRowUp, (const uint8_t *)P.L[l].sh_up + off, G.nj * kRowUp, bar + kBarShGu,
               pol_normal);
    }
    armed |= 1u << kBarShGu;
  };
  auto issue_shared_dn = [&](int l) {  // thread 0: layer l's shared-expert down rows (slot 8), 1 copy
    mbar_expect_tx(bar + kBarShDn, (uint32_t)G.nh * kRowDown);
    if (G.nh > 0)
      bulk_g2s(dn + (size_t)8 * P.caph * kRowDown, (const uint8_t *)P.L[l].sh_down + (size_t)G.h0 * kRowDown,
               G.nh * kRowDown, bar + kBarShDn, pol_normal);
    armed |= 1u << kBarShDn;
  };
  // bounded wait on barrier b's pending phase; flips this thread's parity only on success
  auto wait_bar = [&](int b) -> bool {
    const bool ok = mbar_wait_sleep(bar + b, ph[b]);
    if (ok) {
      ph[b] ^= 1u;
      if (tid == 0) armed &= ~(1u << b);
    }
    return ok;
  };

  if (tid == 0) {
    for (int b = 0; b < kNumBars; ++b) mbar_init(bar + b, 1);
    mbar_fence_init();
  }
  // layer 0's input: the residual (resid mode) or x, into the padded vector
  if (P.resid) {
    for (int i = tid; i < kH / 4; i += kThreads)
      *reinterpret_cast<float4 *>(res_s + pad(4 * i)) = __ldcg(reinterpret_cast<const float4 *>(P.resid) + i);
  } else if (P.x_dtype == B200MOE_BF16) {
    const uint16_t *xb = reinterpret_cast<const uint16_t *>(P.x);
    for (int i = tid; i < kH; i += kThreads) res_s[pad(i)] = bf16f(__ldcg(xb + i));
  } else {
    const float *xf = reinterpret_cast<const float *>(P.x);
    for (int i = tid; i < kH; i += kThreads) res_s[pad(i)] = __ldcg(xf + i);
  }
  for (int i = tid; i < n; i += kThreads) tab[i] = geo(i, n);
  __syncthreads();
  if (tid == 0) {
    issue_router_rows(0);
    issue_shared_gu(0);
    issue_shared_dn(0);
  }

  bool fail = false, aborted = false;
  const int kb0 = lane >> 3, cc = lane & 7;  // gate/up lane mapping (blocks kb0, kb0 + 4; chunk cc)
  for (int l = 0; l < P.n_layers; ++l) {
    const b200moe_layer &Lp = P.L[l];
    const uint32_t ep = 3u * (uint32_t)l;
    const bool last = l + 1 == P.n_layers;
    // ---------------------------------------------------------------- phase R
    if (l > 0) {  // resid += the previous layer's deltas (every CTA applies all of them)
      if (!gather_slots<kSlotDelta, (b2mega::kMaxCtas * kSlotDelta / 2 + kThreads - 1) / kThreads>(
              td, n, ep, abort_word, [&](int src) { return tab[src].nh; },
              [&](int src, int i, uint32_t v) {
                float *r = res_s + pad(tab[src].h0 + i);
                *r = __fadd_rn(*r, __uint_as_float(v));
              })) {
        aborted = true;
        break;
      }
    }
    if (tid == 0 && !last) issue_router_rows(l + 1);
    float rs = 1.0f;  // every warp derives the RMSNorm scale itself (identical bits, no barrier)
    if (P.resid) {    // sum of squares in the declared chunk order
      const float *v = res_s + lane * kPadSeg;
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 a = *reinterpret_cast<const float4 *>(v + 4 * i);
        ss = __fmaf_rn(a.x, a.x, ss);
        ss = __fmaf_rn(a.y, a.y, ss);
        ss = __fmaf_rn(a.z, a.z, ss);
        ss = __fmaf_rn(a.w, a.w, ss);
      }
      const float tot = chunk_total32(ss);
      rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, 2048.0f), P.eps)));
    }
    fail = !__all_sync(0xFFFFFFFFu, wait_bar(kBarRt0 + (l & 1)));  // every thread consumes the phase
    if (warp < G.nrt && !fail) {
      {
        const uint4 *rp = reinterpret_cast<const uint4 *>(rt + ((l & 1) * 2 + warp) * kRouterRowBytes) + 8 * lane;
        const float *xv = res_s + lane * kPadSeg;
        float acc = 0.0f;
        if (G.nrt == 2) {  // R1 for logit 2c + warp: sequential fmaf over the lane's 64 elements
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 u = rp[i];
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
            const float4 x0 = *reinterpret_cast<const float4 *>(xv + 8 * i);
            const float4 x1 = *reinterpret_cast<const float4 *>(xv + 8 * i + 4);
            const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              acc = __fmaf_rn(__fmul_rn(xs[2 * q], rs), bf16f(w[q]), acc);
              acc = __fmaf_rn(__fmul_rn(xs[2 * q + 1], rs), bf16f(w[q] >> 16), acc);
            }
          }
          float tot = chunk_total32(acc);
          if (Lp.logit_bias) tot = __fadd_rn(tot, Lp.logit_bias[2 * c + warp]);
          if (lane == 0) lgp[warp] = f2bf(tot);
        } else {  // shared-expert gate: sigmoid(w_sg . x), the decode path's arithmetic
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 u = rp[i];
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
            const float4 x0 = *reinterpret_cast<const float4 *>(xv + 8 * i);
            const float4 x1 = *reinterpret_cast<const float4 *>(xv + 8 * i + 4);
            const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              acc = fmaf(__fmul_rn(xs[2 * q], rs), bf16f(w[q]), acc);
              acc = fmaf(__fmul_rn(xs[2 * q + 1], rs), bf16f(w[q] >> 16), acc);
            }
          }
          const float z = warp_sum(acc);
          if (lane == 0)
            st_tagged(tl + (size_t)c * kSlotLogits, ep + 1, __float_as_uint(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)))));
        }
      }
    }
    if (__syncthreads_or(fail)) { aborted = true; break; }
    if (tid == 0 && G.nrt == 2)
      st_tagged(tl + (size_t)c * kSlotLogits, ep + 1, (uint32_t)lgp[0] | ((uint32_t)lgp[1] << 16));
    // ---------------------------------------------------------------- phase S
    uint32_t rw[4] = {0, 0, 0, 0}, mine = 0;
    if (warp == 0) {  // lane L polls word 0 of the logit slots of CTAs L, L+32, ..., (<= 128)
      const long long t0 = clock64();
      uint32_t got = 0, want = 0;
#pragma unroll
      for (int m = 0; m < 5; ++m)
        if (lane + 32 * m <= kE / 2) want |= 1u << m;
      for (int it = 1; got != want && !fail; ++it) {
#pragma unroll
        for (int m = 0; m < 5; ++m) {
          if (!(want & ~got & (1u << m))) continue;
          const int src = lane + 32 * m;
          const uint64_t w = ld_relaxed_u64(tl + (size_t)src * kSlotLogits);
          if ((uint32_t)(w >> 32) == ep + 1) {
            if (src < kE / 2) reinterpret_cast<uint32_t *>(lg16)[src] = (uint32_t)w;  // logits 2src, 2src+1
            else misc[1] = __uint_as_float((uint32_t)w);                             // the shared-expert gate
            got |= 1u << m;
          }
        }
        if (got != want && (it & 15) == 0 &&
            (ld_relaxed_u32(abort_word) != 0u || clock64() - t0 > kWaitBudgetCycles))
          fail = true;
      }
      __syncwarp();
      {  // lane L: logits 8L .. 8L+7 for the route
        const uint4 v = reinterpret_cast<const uint4 *>(lg16)[lane];
        rw[0] = v.x; rw[1] = v.y; rw[2] = v.z; rw[3] = v.w;
      }
      fail = !__all_sync(0xFFFFFFFFu, !fail);
      if (!fail) {
        mine = route_select(rw);
        const int my_sel = 255 - (int)(mine & 0xFFu);
        if (lane == 0) {
#pragma unroll
          for (int g = 0; g < kGuChunks; ++g) {
            const int cnt = min(kGuChunk, max(0, G.nq - g * kGuChunk));
            mbar_expect_tx(bar + kBarGu0 + g, (uint32_t)cnt * kRowPair);
          }
          mbar_expect_tx(bar + kBarDn, (uint32_t)(kK * G.nh * kRowDown));
          armed |= (((1u << kGuChunks) - 1u) << kBarGu0) | (1u << kBarDn);
        }
        __syncwarp();
        // Routed bulk copies, one per lane, each a contiguous row range:
        //   lanes 0..15: chunk g = lane >> 2, piece (lane >> 1) & 1 (the part of the chunk in its
        //                first / second expert slot), matrix lane & 1 (gate / up);
        //   lanes 16..23: down rows [h0, h0 + nh) of slot lane - 16.
        int a0 = 0, b0 = 0, slot = 0;  // gate/up lanes: chunk rows [a0, b0) of one expert slot
        if (lane < 16) {
          const int g = lane >> 2, piece = (lane >> 1) & 1;
          const int r0 = g * kGuChunk, r1 = min(G.nq, r0 + kGuChunk);
          a0 = r0;
          b0 = r1;
          if (r0 < r1) {
            const int split = ((G.q0 + r0) / kI + 1) * kI - G.q0;  // first row of the next slot
            if (piece == 0) b0 = min(r1, split);
            else a0 = max(r0, split);
          }
          slot = a0 < b0 ? (G.q0 + a0) / kI : 0;
        } else {
          slot = (lane - 16) & 7;
        }
        const int e = __shfl_sync(0xFFFFFFFFu, my_sel, slot);
        const uint8_t *src = nullptr;
        uint8_t *dst = nullptr;
        uint32_t bytes = 0;
        uint64_t *cb = bar + kBarDn;
        if (lane < 16) {
          if (a0 < b0) {
            const int which = lane & 1, j = (G.q0 + a0) % kI;
            src = (const uint8_t *)(which ? Lp.up : Lp.gate) + (size_t)e * Lp.gate_up_expert_stride + (size_t)j * kRowUp;
            dst = (which ? gu_u : gu_g) + (size_t)a0 * kRowUp;
            bytes = (uint32_t)(b0 - a0) * kRowUp;
            cb = bar + kBarGu0 + (lane >> 2);
          }
        } else if (lane < 24 && G.nh > 0) {
          src = (const uint8_t *)Lp.down + (size_t)e * Lp.down_expert_stride + (size_t)G.h0 * kRowDown;
          dst = dn + (size_t)slot * P.caph * kRowDown;
          bytes = (uint32_t)G.nh * kRowDown;
        }
        if (bytes) bulk_g2s(dst, src, bytes, cb, pol_first);
        route_finish(rw, mine, rr);  // R2, R4, R5 while the rows stream in
        if (c == 0 && lane < kK) {
          if (P.ids_out) P.ids_out[(size_t)l * kK + lane] = rr->ids[lane];
          if (P.w_out) P.w_out[(size_t)l * kK + lane] = rr->wb[lane];
        }
      }
    }
    // ---------------------------------------------------------------- phase G
    {  // warps 1..8 (warp 0 routes above); shared pairs first: their rows are already resident
      const int total = G.nj + G.nq;
      uint32_t have = 0;  // bit 0: shared, bit 1 + g: routed chunk g
      if (warp > 0) {
        XChunk X0, X1;
        xchunk_pad(res_s, rs, kb0, cc, X0);
        xchunk_pad(res_s, rs, kb0 + 4, cc, X1);
        for (int idx = warp - 1; idx < total && !fail; idx += kWarps - 1) {
          const bool shared = idx < G.nj;
          const int rp = idx - G.nj;
          const int need = shared ? 0 : 1 + rp / kGuChunk;
          if (!(have & (1u << need))) {  // warp-uniform outcome: the warp reduces together below
            fail = !__all_sync(0xFFFFFFFFu, wait_bar(shared ? kBarShGu : kBarGu0 + need - 1));
            have |= 1u << need;
            if (fail) break;
          }
          const int row = shared ? P.capq + idx : rp;
          const uint8_t *gp = gu_g + (size_t)row * kRowUp, *up = gu_u + (size_t)row * kRowUp;
          int k, j;
          if (shared) {
            k = kK;
            j = G.j0 + idx;
          } else {
            const int qq = G.q0 + rp;
            k = qq / kI;
            j = qq % kI;
          }
          uint4 hq[8];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int kb = kb0 + 4 * h;
            hq[4 * h + 0] = *reinterpret_cast<const uint4 *>(gp + kb * kQB);
            hq[4 * h + 1] = *reinterpret_cast<const uint4 *>(gp + kb * kQB + 16 + 16 * cc);
            hq[4 * h + 2] = *reinterpret_cast<const uint4 *>(up + kb * kQB);
            hq[4 * h + 3] = *reinterpret_cast<const uint4 *>(up + kb * kQB + 16 + 16 * cc);
          }
          float g = q4k_chunk_dot(hq[0], hq[1], cc, X0) + q4k_chunk_dot(hq[4], hq[5], cc, X1);
          float u = q4k_chunk_dot(hq[2], hq[3], cc, X0) + q4k_chunk_dot(hq[6], hq[7], cc, X1);
          g = warp_sum(g);
          u = warp_sum(u);
          if (lane == 0) s_out[shared ? G.nq + idx : rp] = __fmul_rn(silu_f(g), u);
        }
      }
      // every thread consumes every phase of this layer (thread 0 tracks them for the drain)
      if (!fail && !(have & 1u)) fail = !wait_bar(kBarShGu);
      for (int g = 0; g < kGuChunks && !fail; ++g)
        if (!(have & (2u << g))) fail = !wait_bar(kBarGu0 + g);
    }
    if (__syncthreads_or(fail)) { aborted = true; break; }
    if (warp == 0 && lane < G.nq + G.nj)  // this CTA's s values, one coalesced 256-byte store
      st_tagged(ts + (size_t)c * kSlotS + lane, ep + 2, __float_as_uint(s_out[lane]));
    if (tid == 0 && !last) issue_shared_gu(l + 1);  // this layer's shared gate/up reads are done
    // ---------------------------------------------------------------- phase D
    if (!gather_slots<kSlotS, (b2mega::kMaxCtas * kSlotS / 2 + kThreads - 1) / kThreads>(
            ts, n, ep + 2, abort_word, [&](int src) { return tab[src].nq + tab[src].nj; },
            [&](int src, int w, uint32_t v) {
              const Geo &g2 = tab[src];
              int k, j;
              if (w < g2.nq) {
                const int qq = g2.q0 + w;
                k = qq / kI;
                j = qq % kI;
              } else {
                k = kK;
                j = g2.j0 + (w - g2.nq);
              }
              s_s[k * kSPad + pad(j)] = __uint_as_float(v);
            })) {
      aborted = true;
      break;
    }
    if (!fail) fail = !wait_bar(kBarDn);
    if (!fail) fail = !wait_bar(kBarShDn);
    if (__syncthreads_or(fail)) { aborted = true; break; }
    {
      const int slot = warp;  // 9 warps: routed slots 0..7, shared expert 8
      const int half = lane >> 4, kb = (lane >> 3) & 1;
      XChunk X;
      xchunk_pad(s_s + slot * kSPad, 1.0f, kb, cc, X);
      for (int it = 0; 2 * it < G.nh; ++it) {
        const int hh = 2 * it + half;
        const int hr = hh < G.nh ? hh : G.nh - 1;  // odd count: the spare half-warp repeats a row
        const uint8_t *p = dn + (size_t)(slot * P.caph + hr) * kRowDown + kb * kQB;
        const uint4 h4 = *reinterpret_cast<const uint4 *>(p);
        const uint4 q4 = *reinterpret_cast<const uint4 *>(p + 16 + 16 * cc);
        const float v = half_warp_sum(q4k_chunk_dot(h4, q4, cc, X));
        if ((lane & 15) == 0 && hh < G.nh) o_s[slot * P.caph + hh] = v;
      }
    }
    __syncthreads();
    if (tid < G.nh) {
      float acc = 0.0f;
#pragma unroll
      for (int i = 0; i < kK; ++i) {
        const int slot = rr->order[i];
        acc = __fadd_rn(acc, __fmul_rn(o_s[slot * P.caph + tid], bf16f(rr->wb[slot])));
      }
      const float res = __fadd_rn(acc, __fmul_rn(misc[1], o_s[8 * P.caph + tid]));
      const int h = G.h0 + tid;
      if (!last) {
        st_tagged(td + (size_t)c * kSlotDelta + tid, ep + 3, __float_as_uint(res));
      } else if (P.resid) {
        __stcg(P.resid + h, __fadd_rn(res_s[pad(h)], res));
      } else {
        __stcg(P.out + h, res);
      }
    }
    __syncthreads();  // this layer's down rows are consumed
    if (tid == 0 && !last) issue_shared_dn(l + 1);
  }
  if (aborted && tid == 0) {
    atomicExch(abort_word, 1u);      // ends every other CTA's polls
    atomicExch(abort_word + 1, 1u);  // status for the host
    // every armed phase completes on its own (its copies were issued together with it):
    // let them land before this CTA's shared memory is released
    for (int b = 0; b < kNumBars; ++b)
      if (armed & (1u << b)) mbar_wait(bar + b, ph[b]);
  }
}

// ---------------------------------------------------------------- host side
struct DevInfo {
  bool init = false, ok = false;
  int n = 0;
  size_t smem = 0;
  MegaParams layout;  // offsets and capacities only
};

DevInfo g_dev[64];

size_t al16(size_t v) { return (v + 15) & ~(size_t)15; }

bool prepare(int dev, DevInfo &d) {
  if (d.init) return d.ok;
  d.init = true;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
  int coop = 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop) return false;
  const int n = sms < b2mega::kMaxCtas ? sms : b2mega::kMaxCtas;
  if (n < kMinCtas) return false;
  MegaParams &p = d.layout;
  p.capq = (kK * kI + n - 1) / n;
  p.capj = (kI + n - 1) / n;
  p.caph = (kH + n - 1) / n;
  if (p.capq > kGuChunks * kGuChunk) return false;
  size_t off = (size_t)kResPad * 4;                  // residual / x, padded
  p.off_s = (int)off; off += (size_t)(kK + 1) * kSPad * 4;
  p.off_rt = (int)off; off += 4 * (size_t)kRouterRowBytes;
  p.off_gu = (int)off; off += (size_t)(p.capq + p.capj) * kRowPair;
  p.off_dn = (int)off; off += (size_t)(kK + 1) * p.caph * kRowDown;
  p.off_o = (int)off; off += al16((size_t)(kK + 1) * p.caph * 4);
  p.off_rr = (int)off; off += 128 + 64 * 8 + 16 + 128;  // Route, the 256 logits, the CTA's pair, its s
  p.off_tab = (int)off; off += al16(sizeof(Geo) * (size_t)n);
  if (p.capq + p.capj > kSlotS || p.caph > kSlotDelta) return false;
  p.off_bar = (int)off; off += kNumBars * 8 + 16;
  d.smem = off;
  int maxsm = 0;
  if (cudaDeviceGetAttribute(&maxsm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return false;
  if ((size_t)maxsm < d.smem) return false;
  if (cudaFuncSetAttribute(k_mega, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)d.smem) != cudaSuccess) return false;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_mega, kThreads, d.smem) != cudaSuccess || per_sm < 1)
    return false;
  d.n = n;
  d.ok = true;
  return true;
}

}  // namespace

namespace b2mega {

bool usable() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  return prepare(dev, g_dev[dev]);
}

int launch(const Args &a, cudaStream_t stream) {
  int dev = 0;
  B2_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !prepare(dev, g_dev[dev]))
    return b2host::set_error(B200MOE_EINVAL, "persistent decode: device %d cannot host one resident CTA per SM", dev);
  const DevInfo &d = g_dev[dev];
  MegaParams p = d.layout;
  p.eps = a.eps;
  p.x = a.x;
  p.x_dtype = a.x_dtype;
  p.resid = a.resid;
  p.out = a.out;
  p.xchg = reinterpret_cast<uint8_t *>(a.scratch);
  for (int l0 = 0; l0 < a.n_layers; l0 += kMaxLayers) {
    const int nl = a.n_layers - l0 < kMaxLayers ? a.n_layers - l0 : kMaxLayers;
    p.n_layers = nl;
    p.ids_out = a.ids_out ? a.ids_out + (size_t)l0 * kK : nullptr;
    p.w_out = a.w_out ? a.w_out + (size_t)l0 * kK : nullptr;
    for (int l = 0; l < nl; ++l) p.L[l] = a.layers[l0 + l];
    B2_CUDA(cudaMemsetAsync(a.scratch, 0, kScratchClear, stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)d.n);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = d.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B2_CUDA(cudaLaunchKernelEx(&cfg, k_mega, p));
  }
  return B200MOE_OK;
}

}  // namespace b2mega
