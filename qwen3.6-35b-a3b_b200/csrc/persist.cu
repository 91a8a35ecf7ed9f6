// persist.cu -- single-token MoE decode as ONE persistent kernel over a whole layer stack.
//
// Grid: 128 CTAs of 384 threads (12 warps), one per SM, launched in thread-block clusters of
// C CTAs (C = 8, 4 or 2: the largest whose clusters all fit at once; C = 1 falls back to a
// cooperative launch). CTA c owns fixed, aligned slices of the layer's work:
//   * router: logits 2c, 2c+1 (every CTA also computes the shared-expert gate itself);
//   * gate/up: routed row pairs q = 32c .. 32c+31 of the flattened (slot, j) space -- all in
//     expert slot c / 16 -- and shared-expert row pairs j = 4c .. 4c+3;
//   * down: rows h = 16c .. 16c+15 of all 9 experts, and their combine.
// Per layer l, three phases and three all-to-all exchanges:
//   R  resid += the 2048 deltas of layer l-1 (every CTA keeps the whole residual in shared
//      memory and applies every delta itself, so all CTAs hold identical residuals);
//      rs = 1/sqrt(mean(resid^2) + eps) in the declared chunk order (each warp derives it);
//      the CTA's two router rows and the gate row (staged in shared memory one layer ahead)
//      -> published logit pair.                                                   exchange 1
//   S  top 8 (R3); the CTA issues the bulk copies of its routed rows of this layer at once --
//      its 32 gate and 32 up rows in 8 chunks (one mbarrier each), then its 16 down rows of
//      each of the 8 experts -- then finishes R2, R4, R5.
//   G  s = silu(gate . x) * (up . x) for its 4 shared-expert pairs (prefetched one layer
//      ahead) and 32 routed pairs, chunk by chunk as they land -> published s.  exchange 2
//   D  o[k][h] = down_k[h] . s_k for the 9 experts and its 16 h rows; combine in ascending
//      expert id + sg * shared -> published deltas (last layer: the final residual rows, or
//      out in single-layer mode).                                                 exchange 3
//
// Exchange mechanics (no fences on the critical path):
//   * publish: each value is one 64-bit word (phase tag << 32 | value bits) in the writer's own
//     line-aligned slot, written with one relaxed store (single-copy atomic: the tag vouches
//     for the value);
//   * gather: the cluster reads every writer's slot from L2 ONCE. Cluster rank r owns the
//     writers [r 128/C, (r+1) 128/C), whose values form one contiguous slice of each gathered
//     array (logit pairs, routed s, shared s, deltas). It polls the owned slots (re-reading only
//     words whose tag has not arrived) straight into that slice of its own shared memory, then
//     copies the
//     slice to the same offset in each of the C-1 peers with one shared-to-shared bulk copy,
//     completing bytes on the peer's exchange mbarrier. Each exchange mbarrier is armed with
//     the bytes the peers will send before any peer can send them; a bounded wait on it ends
//     the gather. Nothing is unpacked. A slice is overwritten (next layer) only after every
//     peer has received it: a peer's next contribution to any exchange implies it.
// Every poll and mbarrier wait is bounded (~1 s); a CTA that gives up raises the abort word,
// which ends every other CTA's polls. Every CTA ends with a cluster barrier, so no CTA exits
// while a peer may still write into its shared memory.
//
// The residual uses a padded layout (64-float segments at a 68-float pitch) so the per-lane
// sequential reads of the declared orders and the Q4_K chunk gathers are free of bank
// conflicts.
//
// RMSNorm, R1 logits in the declared chunk order, R2..R5, SiLU, the combine order and the
// residual add are the same sequence of operations as the three-kernel path in decode.cu (routing
// ids and weights bit-identical for the same residual). The Q4_K expert dots of modes 0 / 1 run
// on the tensor cores (q4k_mma_rows: int8 MMAs over the raw quants and an exact three-digit
// fixed-point image of x / s, 2^-23 of the vector's largest magnitude), so their values agree
// with the three-kernel path's f32 dots to ~1e-7 relative rather than bit for bit. Layers in the
// published file's other block formats (Q5_K / Q6_K down, Q8_0 shared) run in the kMode = 2
// instantiation with kq_dot.cuh's chunk dots over the staged rows, bit-identical to the
// gather-GEMV kernels.
#include <atomic>

#include "common.cuh"
#include "imma.cuh"
#include "kq_dot.cuh"
#include "mega.cuh"
#include "route.cuh"
#include "tc.cuh"

using namespace b2;

namespace {

constexpr int kThreads = 384;  // 12 warps: 3 per SM sub-partition (168 registers each)
constexpr int kWarps = kThreads / 32;
constexpr int kMaxLayers = 64;           // layers per launch (kernel parameter space)
constexpr int kN = b2mega::kCtas;        // 128 CTAs
constexpr int kQ = kK * kI / kN;         // 32 routed row pairs per CTA
constexpr int kJ = kI / kN;              // 4 shared row pairs per CTA
constexpr int kHr = kH / kN;             // 16 down rows per CTA
constexpr int kRowPair = 2 * kRowUp;     // 2304 B: gate row + up row
constexpr int kRtRows = 3;               // per layer: the CTA's 2 router rows + the gate row
constexpr int kGuChunks = 8;             // routed gate/up arrival chunks (one mbarrier each)
constexpr int kGuChunk = kQ / kGuChunks; // 4 row pairs per chunk
constexpr int kPadSeg = 68;              // padded pitch of a 64-float segment
constexpr int kResPad = kH / 64 * kPadSeg;  // 2176 floats
// Modes 0 / 1 (tensor-core dots): the three int8 digit planes of x and of each expert's s, each
// plane 32 bytes longer than its vector so the three planes a fragment load reads start on
// different banks; the per-K-part row sums (phase G: [36 pairs][gate, up][4 parts], phase D:
// [9 slots][4 parts][16 rows], f32, one region).
constexpr int kDigPitchX = kH + 32;
constexpr int kDigPitchS = kI + 32;
constexpr int kPartBytes = (kK + 1) * 4 * kHr * 4;
static_assert((kQ + kJ) * 2 * 4 * 4 <= kPartBytes, "phase G part sums fit the region");

// exchange slots (64-bit words, see mega.cuh): per CTA c, line-aligned, written by c only
using b2mega::kSlotLogits;  // word 0: logits 2c | 2c+1 << 16
using b2mega::kSlotS;       // words 0..31: routed s (q = 32c + i), 32..35: shared s (j = 4c + i - 32)
using b2mega::kSlotDelta;   // words 0..15: deltas h = 16c + i
static_assert(kQ == 32 && kJ == 4 && kHr == 16, "the fixed 128-CTA partition");
static_assert(kSlotS >= kQ + kJ && kSlotDelta >= kHr, "exchange slots");

__host__ __device__ inline int pad(int i) { return (i >> 6) * kPadSeg + (i & 63); }

struct MegaParams {
  int n_layers;
  float eps;
  const void *x;
  int x_dtype;
  float *resid;
  float *out;
  int32_t *ids_out;
  uint16_t *w_out;
  uint8_t *xchg;  // exchange area (mega.cuh layout)
  long long budget;  // clock cycles a poll or mbarrier wait may take before the CTA gives up
  int withhold;      // test hook: this CTA (>= 0) never publishes its layer-0 logit pair
  b200moe_layer L[kMaxLayers];
};

// dynamic shared memory layout (bytes). Three instantiations of the kernel (kMode):
//   0  bf16 router rows, no RMSNorm weight, Q4_K throughout: 4 KB router slots, none of the
//      branches below;
//   1  f32 router rows or an RMSNorm weight (kGen): 8 KB router slots;
//   2  kGen plus layers in the published file's other block formats (down Q5_K / Q6_K, shared
//      expert Q8_0; per layer at run time): the down slots sized for Q6_K rows, a separate
//      region for the shared gate / up rows at the Q8_0 width, and single-buffered router rows
//      (layer l+1's are issued once layer l's router has read them) to stay within 227 KB.
constexpr int kOffRes = 0;                                   // [kResPad] f32 residual (or x)
constexpr int kOffS = kOffRes + kResPad * 4;                 // [4096] f32 routed s, flat (slot, j)
constexpr int kOffSsh = kOffS + kK * kI * 4;                 // [512] f32 shared-expert s
constexpr int kOffDl = kOffSsh + kI * 4;                     // [2048] f32 gathered deltas
constexpr int kOffLg = kOffDl + kH * 4;                      // [128] u32 gathered logit pairs
constexpr int kOffRt = kOffLg + kN * 4;                      // [kRouterBufs][3 rows][slot] router rows
//
// Modes 0 / 1 run the Q4_K dots on the tensor cores (see q4k_mma_rows) and stage the gate / up
// rows so that the eight rows one fragment load touches sit at four different offsets modulo
// 128 bytes (two rows per offset: two shared-memory wavefronts per 256-byte warp load, the
// minimum): routed chunk g at g * kChunkPitch (4 rows + 32 bytes, so chunks 2t and 2t+1 differ
// by 32 bytes), the up array 64 bytes off the gate array. Mode 2 keeps the dense layout.
template <int kMode>
struct Lay {
  static constexpr bool kFmt = kMode == 2;
  static constexpr bool kTc = !kFmt;
  static constexpr int kRouterSlot = kMode >= 1 ? kH * 4 : kH * 2;       // bytes per router row slot
  static constexpr int kRouterBufs = kFmt ? 1 : 2;
  static constexpr int kOffGu = kOffRt + kRouterBufs * kRtRows * kRouterSlot;  // gate rows, then up rows
  static constexpr int kChunkPitch = kGuChunk * kRowUp + (kTc ? 32 : 0);       // routed chunk g at g * pitch
  static constexpr int kShOff = kGuChunks * kChunkPitch;                       // the 4 shared rows (dense)
  static constexpr int kGuArr = kShOff + kJ * kRowUp;                          // one array: gate or up
  static constexpr int kUpOff = kGuArr + (kTc ? 64 : 0);                       // up array, from the gate array
  static constexpr int kGuBytes = kUpOff + kGuArr;
  static constexpr int kShRow = (int)row_bytes(B200MOE_TYPE_Q8_0, kH);   // mode 2: shared gate / up row slot
  static constexpr int kOffShGu = kOffGu + kGuBytes;                     // mode 2: [4] gate rows, then [4] up rows
  static constexpr int kOffDn = kOffShGu + (kFmt ? 2 * kJ * kShRow : 0);  // [8] routed down slots of 16 rows
  static constexpr int kDnSlot = kHr * (kFmt ? (int)row_bytes(B200MOE_TYPE_Q6_K, kI) : kRowDown);
  static constexpr int kOffDnSh = kOffDn + kK * kDnSlot;                  // the shared expert's 16 down rows
  static constexpr int kOffO = kOffDnSh + kHr * (kFmt ? (int)row_bytes(B200MOE_TYPE_Q8_0, kI) : kRowDown);
  static constexpr int kOffRr = kOffO + (kK + 1) * kHr * 4;               // Route
  static constexpr int kOffMisc = kOffRr + 128;                           // [3] router row results, [36] s out
  static constexpr int kOffScr = kOffMisc + 256;                          // [12][32] f32 per-warp scratch
  static constexpr int kOffBar = kOffScr + 12 * 32 * 4;                   // mbarriers
  static constexpr int kOffPart = kOffBar + 256;                          // modes 0 / 1: per-K-part row sums
  static constexpr int kSmem = kOffPart + (kTc ? kPartBytes : 0);
};
static_assert(Lay<0>::kOffDnSh == Lay<0>::kOffDn + 8 * kHr * kRowDown && Lay<1>::kOffO == Lay<1>::kOffDnSh + kHr * kRowDown,
              "modes 0 / 1: the [9][16] down rows of one array");
static_assert(Lay<2>::kSmem <= 232448 && Lay<1>::kSmem <= 232448, "227 KB of shared memory per CTA");
static_assert(Lay<2>::kOffShGu % 128 == 0 && Lay<2>::kOffDn % 128 == 0 && Lay<2>::kOffDnSh % 128 == 0,
              "bulk-copy destinations");
static_assert(Lay<2>::kGuBytes == (kQ + kJ) * kRowPair && Lay<2>::kChunkPitch == kGuChunk * kRowUp,
              "mode 2: the dense gate / up staging");
static_assert(Lay<0>::kOffGu % 128 == 0 && Lay<1>::kOffGu % 128 == 0 && Lay<0>::kChunkPitch % 128 == 32 &&
                  Lay<0>::kUpOff % 128 == 64 && Lay<0>::kShOff % 128 == 0 && Lay<0>::kOffDn % 16 == 0 &&
                  Lay<1>::kOffDn % 16 == 0,
              "modes 0 / 1: the skewed gate / up staging (bank offsets 0 / 32 / 64 / 96)");
// Modes 0 / 1: the digit planes of the tensor-core dots. x (2048) lives in the router-row buffer
// the layer has finished with, s (9 x 512) in the routed gate-row area phase G has finished with.
static_assert(3 * kDigPitchX + kH / 32 * 4 <= kRtRows * kH * 2, "x digits fit one router-row buffer");
static_assert(9 * 3 * kDigPitchS + 9 * (kI / 32) * 4 <= Lay<0>::kShOff, "s digits fit the routed gate rows");

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Two tagged words (each 64-bit element is single-copy atomic on its own).
__device__ __forceinline__ void ld_relaxed_v2u64(const uint64_t *p, uint64_t &a, uint64_t &b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ void st_tagged(uint64_t *p, uint32_t tag, uint32_t bits) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((uint64_t)tag << 32) | bits) : "memory");
}

// Bounded mbarrier wait (try_wait without a suspend-time hint: a waiter resumes as soon as the
// phase completes). kCluster: acquire at cluster scope (the phase is completed by peers' bulk
// copies).
template <bool kCluster>
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, long long budget) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    if (kCluster) {
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(smem_u32(bar)), "r"(parity)
          : "memory");
    } else {
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(smem_u32(bar)), "r"(parity)
          : "memory");
    }
    if (ok) return true;
    if (clock64() - t0 > budget) return false;
  }
}

// Global -> shared bulk copy (no multicast), completion counted in bytes on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Shared-to-shared bulk copy into a peer CTA (cluster addresses), completing bytes on the peer's
// mbarrier.
__device__ __forceinline__ void bulk_s2s(uint32_t rdst, uint32_t src, uint32_t bytes, uint32_t rbar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   rdst),
               "r"(src), "r"(bytes), "r"(rbar)
               : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_normal() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Address of this CTA's shared-memory location `saddr` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Named barrier 1 over warps 1..11 (warp 0 routes meanwhile).
__device__ __forceinline__ void bar_sync_g() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads - 32) : "memory"); }

// ---------------------------------------------------------------- tensor-core Q4_K dots (modes 0 / 1)
// The expert dots of modes 0 / 1 run as exact-product int8 MMAs (imma.cuh: raw quants as A, a
// three-digit fixed-point image of x or s as B columns 0..2, per-sub-block integer results scaled
// by the 6-bit scales, the min term from exact per-sub-block sums of the image).

// One warp: the dots of 16 Q4_K rows with v over super-blocks [b0, b1) and, within each, the
// 32-byte quant groups [j0, j1) (sub-blocks 2j0 .. 2j1-1). Fragment row g = lane / 4 reads row
// ra, fragment row g + 8 row rb. dig: digit plane 0 (planes at pitch dpitch, element order);
// sx: per-sub-block sums of n (f32, element order / 32). Lane t = lane % 4 of group g supplies
// quant bytes 8t..8t+7 of each group (low nibbles: sub-block 2j, high: 2j+1), so MMA index
// k = 4t + i is element 32 s + 8t + i and k = 16 + 4t + i element 32 s + 8t + 4 + i of sub-block
// s; the B fragment of lane (g < 3, t) is digit plane g at those elements, one 8-byte load.
// Returns the sums for ra and rb (in units of v * 2^k), the same in all four lanes of the group.
__device__ __forceinline__ void q4k_mma_rows(const uint8_t *ra, const uint8_t *rb, const int8_t *dig, int dpitch,
                                             const float *sx, int b0, int b1, int j0, int j1, float &acc_a,
                                             float &acc_b) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint8_t *dp = reinterpret_cast<const uint8_t *>(dig) + (g < 3 ? g : 0) * dpitch + 8 * t;
  // lane t holds D columns 2t, 2t+1: digit planes 0 (x 65536) and 1 (x 256) in lane 0, plane 2 in
  // lane 1 (its second column, and lanes 2 and 3, are zero columns)
  const float flo = t == 0 ? 65536.0f : (t == 1 ? 1.0f : 0.0f), fhi = t == 0 ? 256.0f : 0.0f;
  constexpr uint32_t kNib = 0x0F0F0F0Fu;
  float fa = 0.0f, fb = 0.0f;
  for (int b = b0; b < b1; ++b) {
    const uint4 ha = *reinterpret_cast<const uint4 *>(ra + kQB * b);
    const uint4 hb = *reinterpret_cast<const uint4 *>(rb + kQB * b);
    // get_scale_min_k4, byte-parallel: byte i of the lo word is sub-block i, of the hi word 4 + i
    const uint32_t sa_lo = ha.y & 0x3F3F3F3Fu, sa_hi = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
    const uint32_t sb_lo = hb.y & 0x3F3F3F3Fu, sb_hi = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
    int ia0 = 0, ia1 = 0, ib0 = 0, ib1 = 0;
#pragma unroll 2
    for (int j = j0; j < j1; ++j) {
      const uint2 wa = lds64(ra + kQB * b + 16 + 32 * j + 8 * t);
      const uint2 wb = lds64(rb + kQB * b + 16 + 32 * j + 8 * t);
      uint2 x0 = make_uint2(0u, 0u), x1 = make_uint2(0u, 0u);
      if (g < 3) {
        x0 = lds64(dp + 256 * b + 64 * j);
        x1 = lds64(dp + 256 * b + 64 * j + 32);
      }
      int d[4], e[4];
      mma_s8(wa.x & kNib, wb.x & kNib, wa.y & kNib, wb.y & kNib, x0.x, x0.y, d);
      mma_s8((wa.x >> 4) & kNib, (wb.x >> 4) & kNib, (wa.y >> 4) & kNib, (wb.y >> 4) & kNib, x1.x, x1.y, e);
      const int sh = 16 * (j & 1);  // sub-blocks 2j, 2j+1: bytes 2(j&1), 2(j&1)+1 of the lo / hi word
      const uint32_t swa = j < 2 ? sa_lo : sa_hi, swb = j < 2 ? sb_lo : sb_hi;
      const int sca0 = (int)((swa >> sh) & 0xFFu), sca1 = (int)((swa >> (sh + 8)) & 0xFFu);
      const int scb0 = (int)((swb >> sh) & 0xFFu), scb1 = (int)((swb >> (sh + 8)) & 0xFFu);
      ia0 += sca0 * d[0] + sca1 * e[0];
      ia1 += sca0 * d[1] + sca1 * e[1];
      ib0 += scb0 * d[2] + scb1 * e[2];
      ib1 += scb0 * d[3] + scb1 * e[3];
    }
    const float da = f16f(ha.x), db = f16f(hb.x);
    fa = fmaf(da, fmaf(fhi, (float)ia1, flo * (float)ia0), fa);
    fb = fmaf(db, fmaf(fhi, (float)ib1, flo * (float)ib0), fb);
    // the min term: lane t takes sub-blocks 2j0 + t, 2j0 + t + 4 (those below 2j1) of both rows
    const uint32_t ma_lo = ha.z & 0x3F3F3F3Fu, ma_hi = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
    const uint32_t mb_lo = hb.z & 0x3F3F3F3Fu, mb_hi = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
    const float dma = f16f(ha.x >> 16), dmb = f16f(hb.x >> 16);
    for (int s = 2 * j0 + t; s < 2 * j1; s += 4) {
      const int sh = 8 * (s & 3);
      const float ma = (float)(((s < 4 ? ma_lo : ma_hi) >> sh) & 0xFFu);
      const float mb = (float)(((s < 4 ? mb_lo : mb_hi) >> sh) & 0xFFu);
      const float n = sx[8 * b + s];
      fa = fmaf(-(dma * ma), n, fa);
      fb = fmaf(-(dmb * mb), n, fb);
    }
  }
  fa += __shfl_xor_sync(0xFFFFFFFFu, fa, 1);
  fb += __shfl_xor_sync(0xFFFFFFFFu, fb, 1);
  fa += __shfl_xor_sync(0xFFFFFFFFu, fa, 2);
  fb += __shfl_xor_sync(0xFFFFFFFFu, fb, 2);
  acc_a = fa;
  acc_b = fb;
}

// x values of chunk (kb, c) from the padded residual, each scaled by rs (and, kGen only, by the
// RMSNorm weight nw, a second rounding, when given).
template <bool kGen>
__device__ __forceinline__ void xchunk_pad(const float *row, float rs, const float *nw, int kb, int c, XChunk &x) {
  const int p = (4 * kb + (c >> 1)) * kPadSeg + 16 * (c & 1);
  const int e = (4 * kb + (c >> 1)) * 64 + 16 * (c & 1);  // element index of the run's start
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 a = *reinterpret_cast<const float4 *>(row + p + 4 * i);
    const float4 b = *reinterpret_cast<const float4 *>(row + p + 32 + 4 * i);
    x.lo[4 * i] = __fmul_rn(a.x, rs); x.lo[4 * i + 1] = __fmul_rn(a.y, rs);
    x.lo[4 * i + 2] = __fmul_rn(a.z, rs); x.lo[4 * i + 3] = __fmul_rn(a.w, rs);
    x.hi[4 * i] = __fmul_rn(b.x, rs); x.hi[4 * i + 1] = __fmul_rn(b.y, rs);
    x.hi[4 * i + 2] = __fmul_rn(b.z, rs); x.hi[4 * i + 3] = __fmul_rn(b.w, rs);
    if (kGen && nw) {
      const float4 wa = __ldg(reinterpret_cast<const float4 *>(nw + e + 4 * i));
      const float4 wb = __ldg(reinterpret_cast<const float4 *>(nw + e + 32 + 4 * i));
      x.lo[4 * i] = __fmul_rn(x.lo[4 * i], wa.x); x.lo[4 * i + 1] = __fmul_rn(x.lo[4 * i + 1], wa.y);
      x.lo[4 * i + 2] = __fmul_rn(x.lo[4 * i + 2], wa.z); x.lo[4 * i + 3] = __fmul_rn(x.lo[4 * i + 3], wa.w);
      x.hi[4 * i] = __fmul_rn(x.hi[4 * i], wb.x); x.hi[4 * i + 1] = __fmul_rn(x.hi[4 * i + 1], wb.y);
      x.hi[4 * i + 2] = __fmul_rn(x.hi[4 * i + 2], wb.z); x.hi[4 * i + 3] = __fmul_rn(x.hi[4 * i + 3], wb.w);
    }
  }
  float sl = 0.f, sh = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) { sl += x.lo[i]; sh += x.hi[i]; }
  x.slo = sl;
  x.shi = sh;
}

// The declared R1 / RMSNorm order: the 32 lanes' partials added left to right. They go through
// a 32-float shared-memory scratch of the warp (one store, eight vector loads) instead of 31
// dependent shuffles; the result is broadcast to every lane.
__device__ __forceinline__ float chunk_total32(float acc, float *scratch) {
  const int lane = threadIdx.x & 31;
  scratch[lane] = acc;
  __syncwarp();
  float tot = 0.0f;
  if (lane == 0) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 q = reinterpret_cast<const float4 *>(scratch)[i];
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

// One router row staged in shared memory (bf16, or f32 when wf32): R1 in the declared order
// (bf16 logit bits) or, for the shared-expert gate, sigmoid(w_sg . x) with the decode path's
// arithmetic (f32 bits). Lane 0 holds the result. The !kGen form takes bf16 rows and no weight
// (wf32 and nw ignored) and scales x inside the dot product: the same roundings in the same order.
template <bool kGen>
__device__ __forceinline__ uint32_t router_row(const uint8_t *row, bool wf32, const float *res, float rs,
                                               const float *nw, int lane, bool gate, float bias, float *scratch) {
  const float *xv = res + lane * kPadSeg;
  float acc = 0.0f;
  if constexpr (!kGen) {
    const uint4 *rp = reinterpret_cast<const uint4 *>(row) + 8 * lane;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 u = rp[i];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      const float4 x0 = *reinterpret_cast<const float4 *>(xv + 8 * i);
      const float4 x1 = *reinterpret_cast<const float4 *>(xv + 8 * i + 4);
      const float x8[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc = __fmaf_rn(__fmul_rn(x8[2 * q], rs), bf16f(w[q]), acc);
        acc = __fmaf_rn(__fmul_rn(x8[2 * q + 1], rs), bf16f(w[q] >> 16), acc);
      }
    }
  } else {
    // the lane's 64 inputs: resid * rs (* nw), in element order
    float xs[64];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 x = *reinterpret_cast<const float4 *>(xv + 4 * i);
      xs[4 * i] = __fmul_rn(x.x, rs); xs[4 * i + 1] = __fmul_rn(x.y, rs);
      xs[4 * i + 2] = __fmul_rn(x.z, rs); xs[4 * i + 3] = __fmul_rn(x.w, rs);
    }
    if (nw) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 w = __ldg(reinterpret_cast<const float4 *>(nw + 64 * lane + 4 * i));
        xs[4 * i] = __fmul_rn(xs[4 * i], w.x); xs[4 * i + 1] = __fmul_rn(xs[4 * i + 1], w.y);
        xs[4 * i + 2] = __fmul_rn(xs[4 * i + 2], w.z); xs[4 * i + 3] = __fmul_rn(xs[4 * i + 3], w.w);
      }
    }
    if (wf32) {
      const float4 *rp = reinterpret_cast<const float4 *>(row) + 16 * lane;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 w = rp[i];
        acc = __fmaf_rn(xs[4 * i], w.x, acc);
        acc = __fmaf_rn(xs[4 * i + 1], w.y, acc);
        acc = __fmaf_rn(xs[4 * i + 2], w.z, acc);
        acc = __fmaf_rn(xs[4 * i + 3], w.w, acc);
      }
    } else {
      const uint4 *rp = reinterpret_cast<const uint4 *>(row) + 8 * lane;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 u = rp[i];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc = __fmaf_rn(xs[8 * i + 2 * q], bf16f(w[q]), acc);
          acc = __fmaf_rn(xs[8 * i + 2 * q + 1], bf16f(w[q] >> 16), acc);
        }
      }
    }
  }
  if (gate) {
    const float z = warp_sum(acc);
    return __float_as_uint(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z))));
  }
  const float tot = __fadd_rn(chunk_total32(acc, scratch), bias);
  return f2bf(tot);
}

enum {
  kBarRt0 = 0, kBarRt1, kBarGu0, kBarDn = kBarGu0 + kGuChunks, kBarShGu, kBarShDn,
  kBarXLg, kBarXS, kBarXDl,  // exchange barriers: bytes from the cluster peers
  kNumBars
};

// ---------------------------------------------------------------- the gather
// One exchange (see the file comment). This rank owns writers [w0, w0 + 128/C); every writer has
// kCnt used words in its slot (pitch kPitch). put(w, i, bits) stores word i of writer w into
// this CTA's gathered arrays; `slices` (nsl of them: shared-memory address, bytes) are this
// rank's contiguous slices, sent to every peer. Returns false (CTA-uniform) on abort or after
// the wait budget.
struct Slice {
  uint32_t addr, bytes;
};

template <int kPitch, int kCnt, typename Put>
__device__ __forceinline__ bool gather(const uint64_t *base, uint32_t tag, const uint32_t *abort_word, int C, int r,
                                       uint64_t *xbar, uint32_t parity, const Slice *slices, int nsl, long long budget,
                                       Put put) {
  const long long t0 = clock64();
  const int per = kN / C, w0 = r * per;
  bool fail = false;
  constexpr int kPairs = (kCnt + 1) / 2;                            // used pairs per writer
  constexpr int kMaxPer = (kN * kPairs + kThreads - 1) / kThreads;  // the C = 1 bound
  uint32_t pending = 0;  // two bits per pair
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int pr = threadIdx.x + k * kThreads;
    if (pr < per * kPairs) {
      const int i = 2 * (pr % kPairs);
      pending |= ((i < kCnt ? 1u : 0u) | (i + 1 < kCnt ? 2u : 0u)) << (2 * k);
    }
  }
  for (int it = 1; pending && !fail; ++it) {  // the owned slots -> this rank's slices (re-poll the rest)
#pragma unroll
    for (int k = 0; k < kMaxPer; ++k) {
      const uint32_t want = (pending >> (2 * k)) & 3u;
      if (!want) continue;
      const int pr = threadIdx.x + k * kThreads;
      const int w = w0 + pr / kPairs, i = 2 * (pr % kPairs);
      uint64_t a, b;
      ld_relaxed_v2u64(base + (size_t)w * kPitch + i, a, b);
      if ((want & 1u) && (uint32_t)(a >> 32) == tag) {
        put(w, i, (uint32_t)a);
        pending &= ~(1u << (2 * k));
      }
      if ((want & 2u) && (uint32_t)(b >> 32) == tag) {
        put(w, i + 1, (uint32_t)b);
        pending &= ~(2u << (2 * k));
      }
    }
    if (pending && (it & 15) == 0 && (ld_relaxed_u32(abort_word) != 0u || clock64() - t0 > budget))
      fail = true;
  }
  fence_proxy_async_smem();  // the slices are read by the bulk copies below (async proxy)
  if (__syncthreads_or(fail)) return false;
  if (threadIdx.x == 0) {
    const uint32_t lbar = smem_u32(xbar);
    for (int q = 1; q < C; ++q) {
      const uint32_t peer = (uint32_t)((r + q) % C);
      for (int s = 0; s < nsl; ++s)
        bulk_s2s(mapa(slices[s].addr, peer), slices[s].addr, slices[s].bytes, mapa(lbar, peer));
    }
  }
  // the peers' slices: bytes completed on this CTA's exchange barrier
  fail = !mbar_wait_bounded<true>(xbar, parity, budget);
  return !__syncthreads_or(fail);
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1) k_mega(const __grid_constant__ MegaParams P) {
  using SL = Lay<kMode>;
  constexpr bool kGen = kMode >= 1, kFmt = kMode == 2;
  extern __shared__ __align__(128) uint8_t smem[];
  float *res_s = reinterpret_cast<float *>(smem + kOffRes);
  float *s_s = reinterpret_cast<float *>(smem + kOffS);
  float *ssh_s = reinterpret_cast<float *>(smem + kOffSsh);
  float *dl_s = reinterpret_cast<float *>(smem + kOffDl);
  uint32_t *lg_s = reinterpret_cast<uint32_t *>(smem + kOffLg);
  uint8_t *rt = smem + kOffRt;
  uint8_t *gu_g = smem + SL::kOffGu;                  // [32 routed + 4 shared] gate rows
  uint8_t *gu_u = gu_g + SL::kUpOff;                  // the matching up rows
  uint8_t *dn = smem + SL::kOffDn;                    // [8][16] routed down rows
  uint8_t *dn_sh = smem + SL::kOffDnSh;               // the shared expert's 16 down rows
  uint8_t *shg = smem + SL::kOffShGu, *shu = shg + kJ * SL::kShRow;  // mode 2: shared gate / up rows
  float *o_s = reinterpret_cast<float *>(smem + SL::kOffO);
  Route *rr = reinterpret_cast<Route *>(smem + SL::kOffRr);
  uint32_t *row_out = reinterpret_cast<uint32_t *>(smem + SL::kOffMisc);  // [3] router row results
  float *s_out = reinterpret_cast<float *>(smem + SL::kOffMisc + 16);      // [36] this CTA's s values
  float *warp_scr = reinterpret_cast<float *>(smem + SL::kOffScr);
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + SL::kOffBar);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  const int C = (int)cluster_size(), r = (int)cluster_rank();
  const int slot_c = c / (kI / kQ), j_c = (c * kQ) % kI;  // this CTA's routed expert slot, first row
  uint32_t *abort_word = reinterpret_cast<uint32_t *>(P.xchg);  // [1]: status for the host
  uint64_t *tl = reinterpret_cast<uint64_t *>(P.xchg + b2mega::kXLogits);
  uint64_t *ts = reinterpret_cast<uint64_t *>(P.xchg + b2mega::kXS);
  uint64_t *td = reinterpret_cast<uint64_t *>(P.xchg + b2mega::kXDelta);
  const uint64_t pol_first = l2_evict_first(), pol_normal = l2_evict_normal();

  uint32_t armed = 0;  // thread 0: copy barriers with a phase in flight
  uint32_t ph[kNumBars];
#pragma unroll
  for (int b = 0; b < kNumBars; ++b) ph[b] = 0;

  // the router-row buffer of layer l (mode 2: one buffer)
  auto rt_buf = [&](int l) -> int { return kFmt ? 0 : (l & 1); };
  // layer l's block types (modes 0 / 1: Q4_K)
  auto down_t = [&](int l) -> int { return kFmt ? layer_down_type(&P.L[l]) : B200MOE_TYPE_Q4_K; };
  auto sh_t = [&](int l) -> int { return kFmt ? layer_sh_type(&P.L[l]) : B200MOE_TYPE_Q4_K; };
  auto issue_router_rows = [&](int l) {  // thread 0: layer l's 2 router rows + gate row -> its buffer
    uint64_t *b = bar + kBarRt0 + rt_buf(l);
    // bytes of one row as stored; the rows sit at that pitch, the CTA's two router rows one copy
    const uint32_t rb = (kGen && P.L[l].router_f32) ? kH * 4 : kH * 2;
    mbar_expect_tx(b, kRtRows * rb);
    uint8_t *d = rt + (size_t)rt_buf(l) * kRtRows * SL::kRouterSlot;
    bulk_g2s(d, (const uint8_t *)P.L[l].router_w + (size_t)(2 * c) * rb, 2 * rb, b, pol_normal);
    bulk_g2s(d + 2 * rb, P.L[l].sh_gate_w, rb, b, pol_normal);
    armed |= 1u << (kBarRt0 + rt_buf(l));
  };
  auto issue_shared_gu = [&](int l) {  // thread 0: layer l's shared-expert gate/up rows, 2 copies
    if constexpr (kFmt) {
      const uint32_t rg = (uint32_t)row_bytes(sh_t(l), kH);
      mbar_expect_tx(bar + kBarShGu, 2 * kJ * rg);
      const size_t off = (size_t)(kJ * c) * rg;
      bulk_g2s(shg, (const uint8_t *)P.L[l].sh_gate + off, kJ * rg, bar + kBarShGu, pol_normal);
      bulk_g2s(shu, (const uint8_t *)P.L[l].sh_up + off, kJ * rg, bar + kBarShGu, pol_normal);
    } else {
      mbar_expect_tx(bar + kBarShGu, kJ * kRowPair);
      const size_t off = (size_t)(kJ * c) * kRowUp;
      bulk_g2s(gu_g + SL::kShOff, (const uint8_t *)P.L[l].sh_gate + off, kJ * kRowUp, bar + kBarShGu, pol_normal);
      bulk_g2s(gu_u + SL::kShOff, (const uint8_t *)P.L[l].sh_up + off, kJ * kRowUp, bar + kBarShGu, pol_normal);
    }
    armed |= 1u << kBarShGu;
  };
  auto issue_shared_dn = [&](int l) {  // thread 0: layer l's shared-expert down rows (slot 8), 1 copy
    const uint32_t rd = (uint32_t)row_bytes(sh_t(l), kI);
    mbar_expect_tx(bar + kBarShDn, kHr * rd);
    bulk_g2s(dn_sh, (const uint8_t *)P.L[l].sh_down + (size_t)(kHr * c) * rd, kHr * rd, bar + kBarShDn,
             pol_normal);
    armed |= 1u << kBarShDn;
  };
  // bounded wait on copy barrier b's pending phase; flips this thread's parity only on success
  auto wait_bar = [&](int b) -> bool {
    const bool ok = mbar_wait_bounded<false>(bar + b, ph[b], P.budget);
    if (ok) {
      ph[b] ^= 1u;
      if (tid == 0) armed &= ~(1u << b);
    }
    return ok;
  };

  // this rank's slices of the gathered arrays (owned writers [r 128/C, (r+1) 128/C))
  const int per = kN / C, w0 = r * per;
  const Slice sl_lg[1] = {{smem_u32(lg_s + w0), (uint32_t)(per * 4)}};
  const Slice sl_s[2] = {{smem_u32(s_s + w0 * kQ), (uint32_t)(per * kQ * 4)},
                         {smem_u32(ssh_s + w0 * kJ), (uint32_t)(per * kJ * 4)}};
  const Slice sl_dl[1] = {{smem_u32(dl_s + w0 * kHr), (uint32_t)(per * kHr * 4)}};
  // every exchange brings (C - 1) peer slices
  const uint32_t rx_lg = (uint32_t)(C - 1) * per * 4, rx_s = (uint32_t)(C - 1) * per * (kQ + kJ) * 4,
                 rx_dl = (uint32_t)(C - 1) * per * kHr * 4;

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
  __syncthreads();
  if (tid == 0) {
    // the first phase of each exchange barrier (the deltas are first consumed by layer 1)
    mbar_expect_tx(bar + kBarXLg, rx_lg);
    mbar_expect_tx(bar + kBarXS, rx_s);
    if (P.n_layers > 1) mbar_expect_tx(bar + kBarXDl, rx_dl);
    issue_router_rows(0);
    issue_shared_gu(0);
    issue_shared_dn(0);
  }
  // every peer's barriers are initialised and armed before anyone can send into them
  cluster_sync_all();

  bool fail = false, aborted = false;
  const int kb0 = lane >> 3, cc = lane & 7;  // gate/up lane mapping (blocks kb0, kb0 + 4; chunk cc)
  for (int l = 0; l < P.n_layers; ++l) {
    const b200moe_layer &Lp = P.L[l];
    const uint32_t ep = 3u * (uint32_t)l;
    const bool last = l + 1 == P.n_layers;
    // ---------------------------------------------------------------- phase R
    if (l > 0) {  // resid += the previous layer's deltas (every CTA applies all of them)
      if (!gather<kSlotDelta, kHr>(td, ep, abort_word, C, r, bar + kBarXDl, ph[kBarXDl], sl_dl, 1, P.budget,
                                   [&](int w, int i, uint32_t v) { dl_s[w * kHr + i] = __uint_as_float(v); })) {
        aborted = true;
        break;
      }
      ph[kBarXDl] ^= 1u;
      if (tid == 0 && !last) mbar_expect_tx(bar + kBarXDl, rx_dl);  // the next layer's deltas
      for (int h = tid; h < kH; h += kThreads) {
        float *rp = res_s + pad(h);
        *rp = __fadd_rn(*rp, dl_s[h]);
      }
      __syncthreads();
    }
    if (!kFmt && tid == 0 && !last) issue_router_rows(l + 1);
    __syncwarp();
    // Every warp derives the RMSNorm scale itself (identical bits, no barrier): the router warps
    // now, the others at the start of phase G, where they would wait for rows anyway (so they do
    // not compete for shared memory with the router on the critical path).
    auto rms_scale = [&]() -> float {
      if (!P.resid) return 1.0f;
      const float *v = res_s + lane * kPadSeg;  // sum of squares in the declared chunk order
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 a = *reinterpret_cast<const float4 *>(v + 4 * i);
        ss = __fmaf_rn(a.x, a.x, ss);
        ss = __fmaf_rn(a.y, a.y, ss);
        ss = __fmaf_rn(a.z, a.z, ss);
        ss = __fmaf_rn(a.w, a.w, ss);
      }
      const float tot = chunk_total32(ss, warp_scr + 32 * warp);
      return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, 2048.0f), P.eps)));
    };
    float rs = warp < kRtRows ? rms_scale() : 1.0f;
    fail = !__all_sync(0xFFFFFFFFu, wait_bar(kBarRt0 + rt_buf(l)));  // every thread consumes the phase
    if (!fail && warp < kRtRows) {  // warps 0, 1: logits 2c, 2c+1; warp 2: the gate
      const bool gate = warp == 2;
      const float bias = (!gate && Lp.logit_bias) ? Lp.logit_bias[2 * c + warp] : 0.0f;
      const bool wf32 = kGen && Lp.router_f32 != 0;
      const uint32_t v = router_row<kGen>(rt + (size_t)rt_buf(l) * kRtRows * SL::kRouterSlot +
                                              (size_t)warp * (wf32 ? kH * 4 : kH * 2),
                                          wf32, res_s, rs, P.resid ? Lp.norm_w : nullptr, lane, gate, bias,
                                          warp_scr + 32 * warp);
      if (lane == 0) row_out[warp] = v;
    }
    if (__syncthreads_or(fail)) { aborted = true; break; }
    if (tid == 0 && !(l == 0 && c == P.withhold))
      st_tagged(tl + (size_t)c * kSlotLogits, ep + 1, row_out[0] | (row_out[1] << 16));
    if (kFmt && tid == 0 && !last) issue_router_rows(l + 1);  // the one buffer is read (barrier above)
    // ---------------------------------------------------------------- phase S
    if (!gather<kSlotLogits, 1>(tl, ep + 1, abort_word, C, r, bar + kBarXLg, ph[kBarXLg], sl_lg, 1, P.budget,
                                [&](int w, int, uint32_t v) { lg_s[w] = v; })) {
      aborted = true;
      break;
    }
    ph[kBarXLg] ^= 1u;
    if (tid == 0 && !last) mbar_expect_tx(bar + kBarXLg, rx_lg);  // the next layer's logits
    int e_dn = 0;     // warp 0, lanes 16..23: the expert of slot lane - 16 (its down rows)
    if (warp == 0) {  // lane L: logits 8L .. 8L+7
      const uint4 v = reinterpret_cast<const uint4 *>(lg_s)[lane];
      uint32_t rw[4] = {v.x, v.y, v.z, v.w};
      const uint32_t mine = route_select(rw);
      const int my_sel = 255 - (int)(mine & 0xFFu);
      if (lane == 0) {
#pragma unroll
        for (int g = 0; g < kGuChunks; ++g) mbar_expect_tx(bar + kBarGu0 + g, kGuChunk * kRowPair);
        armed |= ((1u << kGuChunks) - 1u) << kBarGu0;
        if constexpr (kFmt) {
          mbar_expect_tx(bar + kBarDn, kK * kHr * (uint32_t)row_bytes(down_t(l), kI));
          armed |= 1u << kBarDn;
        }
      }
      __syncwarp();
      // Routed bulk copies, one per lane, in the order they are consumed: lanes 0..15 -> chunk
      // lane >> 1 of the gate (even) or up (odd) rows of this CTA's expert; lanes 16..23 -> the
      // 16 down rows of slot lane - 16 (not needed before the s exchange). Modes 0 / 1 request
      // the down rows at the start of phase G instead, once the last gate / up chunk has landed,
      // so they do not share HBM with the gate / up stream (measured 0.642 -> 0.638 ms per
      // 40-layer token; mode 2, whose CUDA-core gate / up is the bound, keeps them here).
      const int k = lane < 2 * kGuChunks ? slot_c : (lane - 2 * kGuChunks) & 7;
      const int e = __shfl_sync(0xFFFFFFFFu, my_sel, k);
      e_dn = e;
      if (lane < 2 * kGuChunks) {
        const int g = lane >> 1, which = lane & 1;
        const uint8_t *src = (const uint8_t *)(which ? Lp.up : Lp.gate) + (size_t)e * Lp.gate_up_expert_stride +
                             (size_t)(j_c + g * kGuChunk) * kRowUp;
        bulk_g2s((which ? gu_u : gu_g) + g * SL::kChunkPitch, src, kGuChunk * kRowUp, bar + kBarGu0 + g,
                 pol_first);
      }
      if constexpr (kFmt) {  // mode 2: the down rows right behind the gate / up rows
        __syncwarp();
        if (lane >= 2 * kGuChunks && lane < 2 * kGuChunks + kK) {
          const uint32_t rd = (uint32_t)row_bytes(down_t(l), kI);  // down row bytes at the layer's format
          const uint8_t *src = (const uint8_t *)Lp.down + (size_t)e * Lp.down_expert_stride + (size_t)(kHr * c) * rd;
          bulk_g2s(dn + (size_t)k * kHr * rd, src, kHr * rd, bar + kBarDn, pol_first);
        }
      }
      __syncwarp();
      route_finish(rw, mine, rr);  // R2, R4, R5 while the rows stream in
      if (c == 0 && lane < kK) {
        if (P.ids_out) P.ids_out[(size_t)l * kK + lane] = rr->ids[lane];
        if (P.w_out) P.w_out[(size_t)l * kK + lane] = rr->wb[lane];
      }
    }
    // ---------------------------------------------------------------- phase G
    {  // warps 1..11 (warp 0 routes above). Mode 2: two adjacent row pairs per iteration, in
       // arrival order (items 0..3 the shared pairs, items 4..35 the routed pairs in chunk order;
       // warp w takes items 2(w-1), 2(w-1)+1, then the same 22 items later). Modes 0 / 1: the x
       // digits, then tensor-core tiles of 8 row pairs (routed pairs 8T..8T+7 = chunks 2T, 2T+1,
       // split in K quarters: warps 1..8 take T = 0 / 1 then T = 2 / 3) and the shared tile
       // (K halves: warps 9, 10); per-part row sums go to shared memory.
      uint32_t have = 0;  // bit 0: shared, bit 1 + g: routed chunk g
      // wait (warp-uniform) for the copy barriers in `need` this thread has not consumed yet
      auto need_bits = [&](uint32_t need) {
        for (int bit = 0; bit < 1 + kGuChunks && !fail; ++bit) {
          if (!(need & ~have & (1u << bit))) continue;
          fail = !__all_sync(0xFFFFFFFFu, wait_bar(bit == 0 ? kBarShGu : kBarGu0 + bit - 1));
          have |= 1u << bit;
        }
      };
      if (!kFmt && warp == 0) {  // modes 0 / 1: the routed down rows, once the last gate / up chunk has landed
        __syncwarp();
        need_bits(1u << kGuChunks);
        if (!fail) {
          const uint32_t rd = (uint32_t)row_bytes(down_t(l), kI);  // down row bytes (kRowDown for Q4_K)
          if (lane == 0) {
            mbar_expect_tx(bar + kBarDn, kK * kHr * rd);
            armed |= 1u << kBarDn;
          }
          __syncwarp();
          if (lane >= 2 * kGuChunks && lane < 2 * kGuChunks + kK) {
            const int k = lane - 2 * kGuChunks;
            const uint8_t *src = (const uint8_t *)Lp.down + (size_t)e_dn * Lp.down_expert_stride + (size_t)(kHr * c) * rd;
            bulk_g2s(dn + (size_t)k * kHr * rd, src, kHr * rd, bar + kBarDn, pol_first);
          }
          __syncwarp();
        }
      }
      if (warp > 0) {
        __syncwarp();
        if (warp >= kRtRows) rs = rms_scale();
        if constexpr (kFmt) {
          XChunk X0, X1;
          const float *nw = P.resid ? Lp.norm_w : nullptr;
          xchunk_pad<kGen>(res_s, rs, nw, kb0, cc, X0);
          xchunk_pad<kGen>(res_s, rs, nw, kb0 + 4, cc, X1);
          constexpr int kStep = 2 * (kWarps - 1);
          for (int ia = 2 * (warp - 1); ia < kJ + kQ && !fail; ia += kStep) {
            const int ib = ia + 1;  // the second pair of this iteration (if any)
            const bool two = ib < kJ + kQ;
            uint32_t need = 1u << (ia < kJ ? 0 : 1 + (ia - kJ) / kGuChunk);
            if (two) need |= 1u << (ib < kJ ? 0 : 1 + (ib - kJ) / kGuChunk);
            for (int bit = 0; bit < 1 + kGuChunks; ++bit) {  // warp-uniform outcomes
              if (!(need & ~have & (1u << bit))) continue;
              fail = !__all_sync(0xFFFFFFFFu, wait_bar(bit == 0 ? kBarShGu : kBarGu0 + bit - 1));
              have |= 1u << bit;
              if (fail) break;
            }
            if (fail) break;
            const uint8_t *rowp[2];
  #pragma unroll
            for (int p = 0; p < 2; ++p) {
              const int idx = p ? ib : ia;
              const int row = !two && p ? kQ : (idx < kJ ? kQ + idx : idx - kJ);  // a spare read when !two
              rowp[p] = gu_g + (size_t)row * kRowUp;
            }
            float g[2], u[2];
            if (kFmt && ia < kJ) {  // mode 2: shared pairs ia, ia + 1 (kJ is even: never mixed with routed)
              const int st = sh_t(l);
              const size_t rg = (size_t)row_bytes(st, kH);  // rows staged at their own pitch
  #pragma unroll
              for (int p = 0; p < 2; ++p) {
                const uint8_t *rgp = shg + (size_t)(ia + p) * rg, *rup = shu + (size_t)(ia + p) * rg;
                g[p] = any_chunk_dot<LdShared>(st, rgp, kb0, cc, X0) + any_chunk_dot<LdShared>(st, rgp, kb0 + 4, cc, X1);
                u[p] = any_chunk_dot<LdShared>(st, rup, kb0, cc, X0) + any_chunk_dot<LdShared>(st, rup, kb0 + 4, cc, X1);
              }
            } else {
  #pragma unroll
            for (int m = 0; m < 2; ++m) {  // gate rows of both pairs, then their up rows
              uint4 hq[2][4];
  #pragma unroll
              for (int p = 0; p < 2; ++p) {
                const uint8_t *rp = rowp[p] + m * (size_t)(kQ + kJ) * kRowUp;
                hq[p][0] = *reinterpret_cast<const uint4 *>(rp + kb0 * kQB);
                hq[p][1] = *reinterpret_cast<const uint4 *>(rp + kb0 * kQB + 16 + 16 * cc);
                hq[p][2] = *reinterpret_cast<const uint4 *>(rp + (kb0 + 4) * kQB);
                hq[p][3] = *reinterpret_cast<const uint4 *>(rp + (kb0 + 4) * kQB + 16 + 16 * cc);
              }
  #pragma unroll
              for (int p = 0; p < 2; ++p) {
                const float v = q4k_chunk_dot(hq[p][0], hq[p][1], cc, X0) + q4k_chunk_dot(hq[p][2], hq[p][3], cc, X1);
                if (m == 0) g[p] = v;
                else u[p] = v;
              }
            }
            }
  #pragma unroll
            for (int p = 0; p < 2; ++p) {
              g[p] = warp_sum(g[p]);
              u[p] = warp_sum(u[p]);
            }
            if (lane == 0) {
              s_out[ia < kJ ? kQ + ia : ia - kJ] = __fmul_rn(silu_f(g[0]), u[0]);
              if (two) s_out[ib < kJ ? kQ + ib : ib - kJ] = __fmul_rn(silu_f(g[1]), u[1]);
            }
          }
        } else {
          // x = resid * rs (* nw): warp w - 1 takes sub-blocks w - 1, w + 10, ... (lane = element)
          int8_t *digx = reinterpret_cast<int8_t *>(rt + (size_t)rt_buf(l) * kRtRows * SL::kRouterSlot);
          float *sxx = reinterpret_cast<float *>(digx + 3 * kDigPitchX);
          uint32_t *xmax = reinterpret_cast<uint32_t *>(smem + SL::kOffMisc + 160);
          float *partg = reinterpret_cast<float *>(smem + SL::kOffPart);  // [36 pairs][gate, up][4 parts]
          const float *nw = P.resid ? Lp.norm_w : nullptr;
          const int wv = warp - 1;
          constexpr int kSubs = kH / 32, kPer = (kSubs + kWarps - 2) / (kWarps - 1);
          float xv[kPer];
          uint32_t mx = 0;
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int sb = wv + (kWarps - 1) * i;
            float v = 0.0f;
            if (sb < kSubs) {
              const int e = 32 * sb + lane;
              v = __fmul_rn(res_s[pad(e)], rs);
              if (kGen && nw) v = __fmul_rn(v, __ldg(nw + e));
            }
            xv[i] = v;
            mx = max(mx, __float_as_uint(v) & 0x7FFFFFFFu);
          }
          mx = __reduce_max_sync(0xFFFFFFFFu, mx);
          if (lane == 0) xmax[wv] = mx;
          bar_sync_g();
          uint32_t M = 0;
#pragma unroll
          for (int i = 0; i < kWarps - 1; ++i) M = max(M, xmax[i]);
          const int kx = digit_shift(M);
          const float upx = pow2i(kx);
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int sb = wv + (kWarps - 1) * i;
            if (sb < kSubs) {  // warp-uniform
              const int n = __float2int_rn(__fmul_rn(xv[i], upx));
              int d0, d1, d2;
              digits3(n, d0, d1, d2);
              const int e = 32 * sb + lane;
              digx[e] = (int8_t)d0;
              digx[kDigPitchX + e] = (int8_t)d1;
              digx[2 * kDigPitchX + e] = (int8_t)d2;
              const int tot = __reduce_add_sync(0xFFFFFFFFu, n);
              if (lane == 0) sxx[sb] = (float)tot;
            }
          }
          fence_proxy_async_smem();  // a bulk copy refills this buffer two layers on
          bar_sync_g();
          const float unx = digit_unscale(M, kx);
          const int lg = lane >> 2, lt = lane & 3;
          if (warp <= 8) {
            // fragment row g: chunk 2T + (g & 1), gate (g >> 1 even) or up, pair-in-chunk g >> 2;
            // row g + 8: the same chunk and kind, pair-in-chunk 2 + (g >> 2)
            const int cp = lg & 1, kind = (lg >> 1) & 1, pic = lg >> 2, q = (warp - 1) & 3;
            for (int it = 0; it < 2 && !fail; ++it) {
              const int T = 2 * it + ((warp - 1) >> 2), chunk = 2 * T + cp;
              need_bits(3u << (1 + 2 * T));
              if (fail) break;
              const uint8_t *ra = (kind ? gu_u : gu_g) + chunk * SL::kChunkPitch + pic * kRowUp;
              float va, vb;
              q4k_mma_rows(ra, ra + 2 * kRowUp, digx, kDigPitchX, sxx, 2 * q, 2 * q + 2, 0, 4, va, vb);
              if (lt == 0) {
                const int pa = kGuChunk * chunk + pic;
                partg[(pa * 2 + kind) * 4 + q] = __fmul_rn(va, unx);
                partg[((pa + 2) * 2 + kind) * 4 + q] = __fmul_rn(vb, unx);
              }
            }
          } else if (warp <= 10) {
            // the shared tile: fragment row g = pair g >> 1 (& 3), gate / up by g & 1; rows g + 8 repeat it
            need_bits(1u);
            if (!fail) {
              const int kind = lg & 1, p = (lg >> 1) & 3, h = warp - 9;
              const uint8_t *ra = (kind ? gu_u : gu_g) + SL::kShOff + p * kRowUp;
              float va, vb;
              q4k_mma_rows(ra, ra, digx, kDigPitchX, sxx, 4 * h, 4 * h + 4, 0, 4, va, vb);
              if (lt == 0) partg[((kQ + p) * 2 + kind) * 4 + h] = __fmul_rn(va, unx);
            }
          }
        }
      }
      // every thread consumes every phase of this layer (thread 0 tracks them for the drain)
      if (!fail && !(have & 1u)) fail = !wait_bar(kBarShGu);
      for (int g = 0; g < kGuChunks && !fail; ++g)
        if (!(have & (2u << g))) fail = !wait_bar(kBarGu0 + g);
    }
    if (__syncthreads_or(fail)) { aborted = true; break; }
    if (tid < kQ + kJ) {  // this CTA's s values: one coalesced store
      float sv;
      if constexpr (kFmt) {
        sv = s_out[tid];
      } else {  // pair tid: its gate and up rows' part sums, added in part order
        const float *pp = reinterpret_cast<const float *>(smem + SL::kOffPart) + tid * 8;
        float gs, us;
        if (tid < kQ) {
          gs = __fadd_rn(__fadd_rn(__fadd_rn(pp[0], pp[1]), pp[2]), pp[3]);
          us = __fadd_rn(__fadd_rn(__fadd_rn(pp[4], pp[5]), pp[6]), pp[7]);
        } else {
          gs = __fadd_rn(pp[0], pp[1]);
          us = __fadd_rn(pp[4], pp[5]);
        }
        sv = __fmul_rn(silu_f(gs), us);
      }
      st_tagged(ts + (size_t)c * kSlotS + tid, ep + 2, __float_as_uint(sv));
    }
    if (tid == 0 && !last) issue_shared_gu(l + 1);  // this layer's shared gate/up reads are done
    // ---------------------------------------------------------------- phase D
    if (!gather<kSlotS, kQ + kJ>(ts, ep + 2, abort_word, C, r, bar + kBarXS, ph[kBarXS], sl_s, 2, P.budget,
                                 [&](int w, int i, uint32_t v) {
                                   if (i < kQ) s_s[w * kQ + i] = __uint_as_float(v);
                                   else ssh_s[w * kJ + i - kQ] = __uint_as_float(v);
                                 })) {
      aborted = true;
      break;
    }
    ph[kBarXS] ^= 1u;
    if (tid == 0 && !last) mbar_expect_tx(bar + kBarXS, rx_s);  // the next layer's s
    fail = !wait_bar(kBarDn);
    fail = !wait_bar(kBarShDn) || fail;
    if (__syncthreads_or(fail)) { aborted = true; break; }
    float *partd = reinterpret_cast<float *>(smem + SL::kOffPart);  // modes 0 / 1: [9 slots][4 parts][16 rows]
    if constexpr (!kFmt) {
      // Tensor-core down: warp w < 9 turns expert w's s into digits (lane L: elements 16L..16L+15)
      // in the routed gate-row area, then 36 items (slot, K quarter) of 16 rows, three per warp.
      // Reconverge the warp first (thread 0's solo branches can leave warp 0 split).
      __syncwarp();
      int8_t *digs = reinterpret_cast<int8_t *>(gu_g);                           // [9][3 planes][kDigPitchS]
      float *sxs = reinterpret_cast<float *>(gu_g + (kK + 1) * 3 * kDigPitchS);  // [9][16]
      float *sinv = reinterpret_cast<float *>(smem + SL::kOffMisc + 208);       // [9]
      if (warp < kK + 1) {
        const float *sv = (warp < kK ? s_s + warp * kI : ssh_s) + 16 * lane;
        float v[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 f = *reinterpret_cast<const float4 *>(sv + 4 * i);
          v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        uint32_t mx = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) mx = max(mx, __float_as_uint(v[i]) & 0x7FFFFFFFu);
        mx = __reduce_max_sync(0xFFFFFFFFu, mx);
        const int ks = digit_shift(mx);
        const float ups = pow2i(ks);
        uint32_t pk[3][4] = {};
        int tot = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int n = __float2int_rn(__fmul_rn(v[i], ups));
          int d[3];
          digits3(n, d[0], d[1], d[2]);
#pragma unroll
          for (int pl = 0; pl < 3; ++pl) pk[pl][i >> 2] |= ((uint32_t)d[pl] & 0xFFu) << (8 * (i & 3));
          tot += n;
        }
        int8_t *dst = digs + warp * 3 * kDigPitchS + 16 * lane;
#pragma unroll
        for (int pl = 0; pl < 3; ++pl)
          *reinterpret_cast<uint4 *>(dst + pl * kDigPitchS) = make_uint4(pk[pl][0], pk[pl][1], pk[pl][2], pk[pl][3]);
        tot += __shfl_xor_sync(0xFFFFFFFFu, tot, 1);  // lanes 2i, 2i+1: sub-block i
        if (!(lane & 1)) sxs[warp * (kI / 32) + (lane >> 1)] = (float)tot;
        if (lane == 0) sinv[warp] = digit_unscale(mx, ks);
        fence_proxy_async_smem();  // the next layer's bulk copies land in this area
      }
      __syncthreads();
      const int lg = lane >> 2, lt = lane & 3;
#pragma unroll 1
      for (int it = 0; it < 3; ++it) {
        const int item = warp + kWarps * it;  // 0..35
        const int slot = item >> 2, q = item & 3, sb = q >> 1, j0 = 2 * (q & 1);
        const uint8_t *base = slot < kK ? dn + (size_t)slot * kHr * kRowDown : dn_sh;
        float va, vb;
        q4k_mma_rows(base + lg * kRowDown, base + (lg + 8) * kRowDown, digs + slot * 3 * kDigPitchS, kDigPitchS,
                     sxs + slot * (kI / 32), sb, sb + 1, j0, j0 + 2, va, vb);
        if (lt == 0) {
          const float un = sinv[slot];
          partd[(slot * 4 + q) * kHr + lg] = __fmul_rn(va, un);
          partd[(slot * 4 + q) * kHr + lg + 8] = __fmul_rn(vb, un);
        }
      }
    } else
      {
        // All 12 warps: warp w < 9 takes rows 0..11 of slot w (routed slots 0..7, the shared expert
        // 8), warp 9 + i rows 12..15 of slots 3i, 3i + 1, 3i + 2 -- four rows per iteration (two per
        // half-warp, in flight together), three iterations per warp, so each SM sub-partition runs
        // the same number of row dots (with one warp per slot, three of them ran a third more).
        // Each row's dot is the same sequence of operations whichever warp runs it.
        // Reconverge the warp first: thread 0's solo branches (copy issue, barrier arming) can
        // leave warp 0 split, and a split warp runs this loop once per part.
        __syncwarp();
        const int half = lane >> 4, kb = (lane >> 3) & 1;
        XChunk X;
        if (warp < 9) load_xchunk(warp < kK ? s_s + warp * kI : ssh_s, kb, cc, X);
  #pragma unroll 1
        for (int it = 0; it < 3; ++it) {
          const int slot = warp < 9 ? warp : 3 * (warp - 9) + it;
          const int rbase = warp < 9 ? 4 * it : 12;
          if (warp >= 9) load_xchunk(slot < kK ? s_s + slot * kI : ssh_s, kb, cc, X);
          float v[2];
  #pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int hh = rbase + 2 * p + half;
            if constexpr (kFmt) {  // the layer's row formats, staged at their own pitch
              const int t = slot < kK ? down_t(l) : sh_t(l);
              const size_t rb = (size_t)row_bytes(t, kI);
              const uint8_t *row = (slot < kK ? dn + (size_t)slot * kHr * rb : dn_sh) + (size_t)hh * rb;
              v[p] = any_chunk_dot<LdShared>(t, row, kb, cc, X);
            } else {
              const uint8_t *pp = dn + (size_t)(slot * kHr + hh) * kRowDown + kb * kQB;
              const uint4 h4 = *reinterpret_cast<const uint4 *>(pp);
              const uint4 q4 = *reinterpret_cast<const uint4 *>(pp + 16 + 16 * cc);
              v[p] = q4k_chunk_dot(h4, q4, cc, X);
            }
          }
  #pragma unroll
          for (int p = 0; p < 2; ++p) {
            v[p] = half_warp_sum(v[p]);
            if ((lane & 15) == 0) o_s[slot * kHr + rbase + 2 * p + half] = v[p];
          }
        }
      }
    __syncthreads();
    if (tid < kHr) {
      // expert `slot`'s output row tid (modes 0 / 1: its four K-part sums, added in part order)
      auto o_at = [&](int slot) -> float {
        if constexpr (kFmt) {
          return o_s[slot * kHr + tid];
        } else {
          const float *pp = partd + slot * 4 * kHr + tid;
          return __fadd_rn(__fadd_rn(__fadd_rn(pp[0], pp[kHr]), pp[2 * kHr]), pp[3 * kHr]);
        }
      };
      float acc = 0.0f;
#pragma unroll
      for (int i = 0; i < kK; ++i) {
        const int slot = rr->order[i];
        acc = __fadd_rn(acc, __fmul_rn(o_at(slot), bf16f(rr->wb[slot])));
      }
      const float sg = __uint_as_float(row_out[2]);
      const float res = __fadd_rn(acc, __fmul_rn(sg, o_at(kK)));
      const int h = kHr * c + tid;
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
    // every armed copy phase completes on its own (its copies were issued together with it):
    // let them land before this CTA's shared memory is released
    for (int b = 0; b < kBarXLg; ++b)
      if (armed & (1u << b)) mbar_wait(bar + b, ph[b]);
  }
  // no CTA leaves while a cluster peer may still deliver into its shared memory
  __syncthreads();
  cluster_sync_all();
}

// ---------------------------------------------------------------- host side
struct DevInfo {
  bool init = false, ok = false, fmt_ok = false;  // fmt_ok: mode 2 is resident with the same C
  int C = 1;
};

DevInfo g_dev[64];

// Whether all kN CTAs of k_mega<kMode> are resident at once with clusters of C (C = 1: one CTA
// per SM, the cooperative launch's condition).
template <int kMode>
bool resident(int C) {
  if (C == 1) {
    int per_sm = 0;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_mega<kMode>, kThreads, Lay<kMode>::kSmem) ==
               cudaSuccess &&
           per_sm >= 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kN);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Lay<kMode>::kSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, k_mega<kMode>, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return clusters * C >= kN;
}

template <int kMode>
bool set_smem(int maxsm) {
  return maxsm >= Lay<kMode>::kSmem &&
         cudaFuncSetAttribute(k_mega<kMode>, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay<kMode>::kSmem) ==
             cudaSuccess;
}

bool prepare(int dev, DevInfo &d) {
  if (d.init) return d.ok;
  d.init = true;
  int sms = 0, maxsm = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < kN) return false;
  if (cudaDeviceGetAttribute(&maxsm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return false;
  if (!set_smem<0>(maxsm) || !set_smem<1>(maxsm)) return false;
  // the largest cluster size whose 128 / C clusters are all resident at once (mode 1 has the
  // larger footprint of modes 0 and 1), else a cooperative launch
  int C = 0;
  for (int c : {8, 4, 2})
    if (resident<1>(c)) {
      C = c;
      break;
    }
  if (!C) {
    int coop = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop ||
        !resident<1>(1))
      return false;
    C = 1;
  }
  d.C = C;
  d.ok = true;
  d.fmt_ok = set_smem<2>(maxsm) && resident<2>(C);
  (void)cudaGetLastError();
  return true;
}

}  // namespace

namespace b2mega {

// The failure-path test hook (b200moe_debug_decode_faults): a shorter wait budget and a CTA that
// withholds its first logit pair. Process-wide; read at every launch.
std::atomic<long long> g_hook_budget{0};
std::atomic<int> g_hook_withhold{-1};

void set_fault_hook(long long budget_cycles, int withhold_cta) {
  g_hook_budget.store(budget_cycles > 0 ? budget_cycles : 0);
  g_hook_withhold.store(withhold_cta >= 0 && withhold_cta < kCtas ? withhold_cta : -1);
}

bool usable(bool formats) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  return prepare(dev, g_dev[dev]) && (!formats || g_dev[dev].fmt_ok);
}

int cluster_ctas() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !prepare(dev, g_dev[dev])) return 0;
  return g_dev[dev].C;
}

int launch(const Args &a, cudaStream_t stream) {
  int dev = 0;
  B2_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !prepare(dev, g_dev[dev]))
    return b2host::set_error(B200MOE_EINVAL, "persistent decode: device %d cannot host %d resident CTAs", dev, kN);
  const DevInfo &d = g_dev[dev];
  MegaParams p;
  p.eps = a.eps;
  p.x = a.x;
  p.x_dtype = a.x_dtype;
  p.resid = a.resid;
  p.out = a.out;
  p.xchg = reinterpret_cast<uint8_t *>(a.scratch);
  const long long hb = g_hook_budget.load();
  p.budget = hb > 0 ? hb : kWaitBudgetCycles;
  p.withhold = g_hook_withhold.load();
  for (int l0 = 0; l0 < a.n_layers; l0 += kMaxLayers) {
    const int nl = a.n_layers - l0 < kMaxLayers ? a.n_layers - l0 : kMaxLayers;
    p.n_layers = nl;
    p.ids_out = a.ids_out ? a.ids_out + (size_t)l0 * kK : nullptr;
    p.w_out = a.w_out ? a.w_out + (size_t)l0 * kK : nullptr;
    int mode = 0;  // 1: f32 router rows or an applied RMSNorm weight; 2: a layer not Q4_K throughout
    for (int l = 0; l < nl; ++l) {
      p.L[l] = a.layers[l0 + l];
      if (layer_dense(&p.L[l]))
        return b2host::set_error(B200MOE_EINVAL, "persistent decode: layer %d is dense (BF16)", l0 + l);
      if (!layer_all_q4k(&p.L[l])) mode = 2;
      else if (mode == 0 && (p.L[l].router_f32 != 0 || (a.resid && p.L[l].norm_w))) mode = 1;
    }
    if (mode == 2 && !d.fmt_ok)
      return b2host::set_error(B200MOE_EINVAL, "persistent decode: device %d cannot host the block-format variant",
                               dev);
    B2_CUDA(cudaMemsetAsync(a.scratch, 0, kScratchClear, stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kN);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = mode == 2 ? Lay<2>::kSmem : mode == 1 ? Lay<1>::kSmem : Lay<0>::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (d.C > 1) {  // clusters: every cluster co-scheduled; all 128 / C clusters fit at once
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = (unsigned)d.C;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
    } else {        // one CTA per SM, all resident
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (mode == 2) B2_CUDA(cudaLaunchKernelEx(&cfg, k_mega<2>, p));
    else if (mode == 1) B2_CUDA(cudaLaunchKernelEx(&cfg, k_mega<1>, p));
    else B2_CUDA(cudaLaunchKernelEx(&cfg, k_mega<0>, p));
  }
  return B200MOE_OK;
}

}  // namespace b2mega
