// grouped.cuh -- host interface of the small-batch grouped decode (grouped.cu) and the layout
// of the per-token digit blocks the router writes for it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "b200moe.h"

namespace b2grp {

constexpr int kMaxT = 16;  // tokens per call on the grouped path

// One token's MoE input x as the tensor-core dots take it (imma.cuh), written by the router K1:
// three int8 digit planes of 2048 (+32 padding, so the planes start on different banks), the
// 64 per-sub-block sums of the integer image (f32, exact), then 2^-k (f32).
constexpr int kXPlane = 2048 + 32;
constexpr int kXUnOff = 3 * kXPlane + 64 * 4;
constexpr int kXBlk = kXUnOff + 16;
// The same for one (token, expert) s vector of 512 (built in shared memory by k_dn_grp).
constexpr int kSPlane = 512 + 32;
constexpr int kSUnOff = 3 * kSPlane + 16 * 4;
constexpr int kSBlk = kSUnOff + 16;
static_assert(kXBlk % 16 == 0 && kSBlk % 16 == 0, "16-byte block pitch");

constexpr size_t kPlanBytes = 4096;  // the routing plan (grouped.cu Plan)

struct Args {
  int T;                          // 2 .. kMaxT
  const b200moe_layer *layer;     // Q4_K throughout
  const uint16_t *logits;         // [T][256] bf16 (K1)
  const uint8_t *xd;              // [T][kXBlk] (K1)
  const float *sg;                // [T] shared-expert gate (K1)
  void *plan;                     // kPlanBytes
  float *s;                       // [T][9][512]
  float *o;                       // [T][9][2048]
  float *out;                     // [T][2048]
  int accumulate;                 // 1: out += block output (the residual stream)
  int32_t *ids_out;               // [T][8] or NULL
  uint16_t *w_out;                // [T][8] or NULL
};

// Enqueue k_plan, k_gu_grp, k_dn_grp, k_comb_grp on `stream` (each with programmatic dependent
// launch after the router K1). Returns a B200MOE_* code.
int run(const Args &a, cudaStream_t stream);

}  // namespace b2grp
