// mega.cuh -- host interface of the persistent single-token decode kernel (persist.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "b200moe.h"

namespace b2mega {

constexpr int kCtas = 128;  // the persistent grid: 128 CTAs, one per SM
// Cross-CTA exchange area. Every value one CTA hands to the others travels as one 64-bit word
// (phase tag << 32 | value bits, single-copy atomic), in per-CTA line-aligned slots -- no two
// CTAs ever store into the same 128-byte line:
//   [0, 128)                 abort word, status word
//   logits [c][16] u64       CTA c's logit pair
//   s      [c][48] u64       CTA c's activations s (32 routed, 4 shared)
//   deltas [c][16] u64       CTA c's residual deltas
// Everything is cleared before each launch (tags are launch-local).
constexpr int kSlotLogits = 16, kSlotS = 48, kSlotDelta = 16;  // 64-bit words per CTA
constexpr size_t kXLogits = 128;
constexpr size_t kXS = kXLogits + (size_t)kCtas * kSlotLogits * 8;
constexpr size_t kXDelta = kXS + (size_t)kCtas * kSlotS * 8;
constexpr size_t kScratchBytes = kXDelta + (size_t)kCtas * kSlotDelta * 8;
constexpr size_t kScratchClear = kScratchBytes;

struct Args {
  int n_layers;
  float eps;
  const void *x;      // x mode (resid == NULL, one layer): the block input, one token
  int x_dtype;
  float *resid;       // resid mode: x_l = rmsnorm(resid), resid += block_l(x_l)
  float *out;         // x mode: out = block(x)
  int32_t *ids_out;   // [n_layers][8] or NULL
  uint16_t *w_out;    // [n_layers][8] bf16 routing weights or NULL
  void *scratch;      // kScratchBytes, 16-byte aligned; cleared by launch() on the stream
  const b200moe_layer *layers;  // host array of n_layers
};

// 1 if the current device can run the persistent kernel (128 CTAs resident at once); with
// `formats`, also its variant for layers in other block formats (Q5_K / Q6_K down, Q8_0 shared).
bool usable(bool formats = false);

// Cluster size the launches use on the current device (1: cooperative launch; 0: unusable).
int cluster_ctas();

// Test hook for the failure path: every later launch uses `budget_cycles` (> 0; else the default
// ~1 s) as its wait budget, and CTA `withhold_cta` (>= 0; else none) never publishes its first
// logit pair, so the other CTAs' gathers run out of budget and the kernel ends with its status set.
void set_fault_hook(long long budget_cycles, int withhold_cta);

// Status word (u32) in the exchange area: bit 1 = a bounded wait ran out (the launch's outputs
// are incomplete). Cleared with the exchange area before each launch.
constexpr size_t kStatusOffset = 4;

// Enqueue the flag reset and the persistent kernel(s) on `stream`. Returns a B200MOE_* code.
int launch(const Args &a, cudaStream_t stream);

}  // namespace b2mega
