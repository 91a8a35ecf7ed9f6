// route.cuh -- R2..R5 of the router for one token with one warp (shared by decode and prefill).
//
// Declared rule (mirrored operation for operation by oracle/c/oracle.c b2o_router):
//   R2  m = max logit; e_l = b2_expf(logit_l - m); S = per-lane sequential sums of
//       e_{8L..8L+7} (lane L = 0..31), then an xor butterfly 16, 8, 4, 2, 1
//   R3  top-8 by (bf16 logit descending, expert index ascending). The softmax is monotone in
//       the logit, so this is the reference's top-k over probabilities with its unspecified
//       tie order fixed to "lower index first" (the reference kernel's strict-> rule,
//       prototype/moe_router/moe_router_kernels.h:289-321).
//   R4  p_k = e_k / S for the 8 selected; s8 = sequential sum of p in rank order; w_k = p_k / s8
//   R5  w_bf16 = RNE(w_k) (cast before any multiply, specification/11-moe-block.md:39-60)
// Selection uses a 24-bit key (order-preserving bf16 bits << 8 | (255 - index)): one
// redux.max per rank, no division before the 8 winners are known.
#pragma once

#include "common.cuh"

namespace b2 {

struct Route {
  int ids[kK];
  float wf[kK];
  uint16_t wb[kK];
  int order[kK];  // slots sorted by ascending expert id (the combine order)
};

// Order-preserving 16-bit image of a bf16 (-0 folded onto +0).
__device__ __forceinline__ uint32_t bf16_mono(uint32_t b) {
  b &= 0xFFFFu;
  if (b == 0x8000u) b = 0u;
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

__device__ __forceinline__ void route_warp(const uint16_t *logits_t, Route *rr) {
  const int lane = threadIdx.x & 31;
  const uint4 raw = __ldcg(reinterpret_cast<const uint4 *>(logits_t + 8 * lane));
  const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
  float v[8];
  uint32_t key[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf16f(rw[i]);
    v[2 * i + 1] = bf16f(rw[i] >> 16);
    key[2 * i] = (bf16_mono(rw[i]) << 8) | (uint32_t)(255 - (8 * lane + 2 * i));
    key[2 * i + 1] = (bf16_mono(rw[i] >> 16) << 8) | (uint32_t)(255 - (8 * lane + 2 * i + 1));
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
  // R3: eight rounds of warp max over the lanes' current best keys
  uint32_t best = key[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) best = max(best, key[i]);
  int my_id = 0;      // lane r (< 8) ends holding rank r's expert id ...
  float my_e = 0.0f;  // ... and its exp value
#pragma unroll
  for (int r = 0; r < kK; ++r) {
    const uint32_t w = __reduce_max_sync(0xFFFFFFFFu, best);
    const int id = 255 - (int)(w & 0xFFu);
    float ew = 0.0f;
    if ((id >> 3) == lane) {  // owner: retire the key (keys are unique and never 0)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (key[i] == w) {
          ew = e[i];
          key[i] = 0u;
        }
      }
      best = key[0];
#pragma unroll
      for (int i = 1; i < 8; ++i) best = max(best, key[i]);
    }
    const float ewin = __shfl_sync(0xFFFFFFFFu, ew, id >> 3);
    if (lane == r) {
      my_id = id;
      my_e = ewin;
    }
  }
  // R4/R5 in lanes 0..7 (lane k holds rank k)
  const float pk = __fdiv_rn(my_e, s);
  float s8 = 0.0f;
#pragma unroll
  for (int r = 0; r < kK; ++r) s8 = __fadd_rn(s8, __shfl_sync(0xFFFFFFFFu, pk, r));
  const float wk = (s8 == 0.0f) ? 0.0f : __fdiv_rn(pk, s8);
  int rank = 0;
#pragma unroll
  for (int r = 0; r < kK; ++r) {
    const int other = __shfl_sync(0xFFFFFFFFu, my_id, r);
    rank += (other < my_id) ? 1 : 0;
  }
  if (lane < kK) {
    rr->ids[lane] = my_id;
    rr->wf[lane] = wk;
    rr->wb[lane] = f2bf(wk);
    rr->order[rank] = lane;
  }
  __syncwarp();
}


// ---------------------------------------------------------------- split form (persistent decode)
// The same R2..R5 as route_warp, in two steps so a caller can act on the winners' ids before
// the weights exist. Lane L passes logits 8L..8L+7 as four bf16 pairs.
//   route_select: R3 -> lane r (< 8) gets rank r's key (id = 255 - (key & 0xFF)).
//   route_finish: R2, R4, R5 and the combine order; every value equals route_warp's (the
//                 winner's exp is recomputed from its bf16 logit, an identical input).
__device__ __forceinline__ void key_cas(uint32_t &a, uint32_t &b) {  // a >= b afterwards
  const uint32_t hi = max(a, b), lo = min(a, b);
  a = hi;
  b = lo;
}

__device__ __forceinline__ uint32_t route_select(const uint32_t (&rw)[4]) {
  const int lane = threadIdx.x & 31;
  uint32_t k[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    k[2 * i] = (bf16_mono(rw[i]) << 8) | (uint32_t)(255 - (8 * lane + 2 * i));
    k[2 * i + 1] = (bf16_mono(rw[i] >> 16) << 8) | (uint32_t)(255 - (8 * lane + 2 * i + 1));
  }
  // the lane's 8 keys in descending order (19-comparator network); keys are unique
  key_cas(k[0], k[2]); key_cas(k[1], k[3]); key_cas(k[4], k[6]); key_cas(k[5], k[7]);
  key_cas(k[0], k[4]); key_cas(k[1], k[5]); key_cas(k[2], k[6]); key_cas(k[3], k[7]);
  key_cas(k[0], k[1]); key_cas(k[2], k[3]); key_cas(k[4], k[5]); key_cas(k[6], k[7]);
  key_cas(k[2], k[4]); key_cas(k[3], k[5]);
  key_cas(k[1], k[4]); key_cas(k[3], k[6]);
  key_cas(k[1], k[2]); key_cas(k[3], k[4]); key_cas(k[5], k[6]);
  uint32_t mine = 0;
#pragma unroll
  for (int r = 0; r < kK; ++r) {
    const uint32_t w = __reduce_max_sync(0xFFFFFFFFu, k[0]);
    if (k[0] == w) {  // the owner retires its best key
#pragma unroll
      for (int i = 0; i < 7; ++i) k[i] = k[i + 1];
      k[7] = 0u;
    }
    if (lane == r) mine = w;
  }
  return mine;
}

// bf16 bits back from bf16_mono (the folded -0 comes back as +0: same value).
__device__ __forceinline__ uint32_t bf16_unmono(uint32_t m) { return (m & 0x8000u) ? (m & 0x7FFFu) : (~m & 0xFFFFu); }

__device__ __forceinline__ void route_finish(const uint32_t (&rw)[4], uint32_t mine, Route *rr) {
  const int lane = threadIdx.x & 31;
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
  float s = b2_expf(__fsub_rn(v[0], m));
#pragma unroll
  for (int i = 1; i < 8; ++i) s = __fadd_rn(s, b2_expf(__fsub_rn(v[i], m)));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, o));
  const int my_id = 255 - (int)(mine & 0xFFu);
  const float my_e = b2_expf(__fsub_rn(bf16f(bf16_unmono(mine >> 8)), m));
  const float pk = __fdiv_rn(my_e, s);
  float s8 = 0.0f;
#pragma unroll
  for (int r = 0; r < kK; ++r) s8 = __fadd_rn(s8, __shfl_sync(0xFFFFFFFFu, pk, r));
  const float wk = (s8 == 0.0f) ? 0.0f : __fdiv_rn(pk, s8);
  int rank = 0;
#pragma unroll
  for (int r = 0; r < kK; ++r) {
    const int other = __shfl_sync(0xFFFFFFFFu, my_id, r);
    rank += (other < my_id) ? 1 : 0;
  }
  if (lane < kK) {
    rr->ids[lane] = my_id;
    rr->wf[lane] = wk;
    rr->wb[lane] = f2bf(wk);
    rr->order[rank] = lane;
  }
  __syncwarp();
}

}  // namespace b2
