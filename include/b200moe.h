/* b200moe.h -- C ABI of the B200 (sm_100a) Qwen3.6-35B-A3B MoE block.
 *
 * Plain pointers, sizes and an opaque `void *stream` (a cudaStream_t; NULL = legacy default
 * stream). Every entry point returns B200MOE_OK (0) or an error code and never throws; the
 * message of the last failure on the calling thread is b200moe_last_error(). No entry point
 * allocates device memory: scratch comes from a caller-provided workspace whose size the
 * matching *_workspace_size() query returns. All device pointers must be 16-byte aligned.
 *
 * Geometry (checkpoints/Qwen3.6-35B-A3B.config.json:17,69,73,74,93 in the reference):
 * hidden H = 2048, 256 routed experts, top-8, expert and shared intermediate I = 512.
 *
 * Weight layout in HBM (GGUF order, expert axis slowest, engine/README.md:185-190):
 *   Q4_K super-block: 144 B per 256 weights {f16 d, f16 dmin, u8 scales[12], u8 qs[128]}
 *   routed gate / up : [256 experts][512 rows][8 blocks]   (row = 2048 weights, 1152 B)
 *   routed down      : [256 experts][2048 rows][2 blocks]  (row = 512 weights, 288 B)
 *   shared gate / up : [512][8] blocks,  shared down: [2048][2] blocks
 *   router W_g       : [256][2048] bf16,  shared-expert gate w_sg: [2048] bf16
 * The published Q4_K_M file mixes block formats per tensor (down Q5_K, or Q6_K at three
 * layers; the shared expert Q8_0): b200moe_layer.down_type / sh_type say which, rows keep the
 * GGUF order with the format's own row bytes (down row: Q4_K 288, Q5_K 352, Q6_K 420 B;
 * Q8_0 shared gate/up row 2176 B, down row 544 B).
 */
#ifndef B200MOE_H
#define B200MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200MOE_ABI_VERSION 4
#define B200MOE_HIDDEN 2048
#define B200MOE_EXPERTS 256
#define B200MOE_TOPK 8
#define B200MOE_INTER 512
#define B200MOE_Q4K_BLOCK_BYTES 144

enum { B200MOE_OK = 0, B200MOE_EINVAL = 1, B200MOE_ECUDA = 2, B200MOE_ESIZE = 3 };
enum { B200MOE_F32 = 0, B200MOE_BF16 = 1 };

/* GGML block type ids (as stored in GGUF tensor infos): b200moe_dequant's `type`, and
 * b200moe_layer.down_type / sh_type. */
enum { B200MOE_TYPE_Q8_0 = 8, B200MOE_TYPE_Q4_K = 12, B200MOE_TYPE_Q5_K = 13, B200MOE_TYPE_Q6_K = 14,
       B200MOE_TYPE_BF16 = 30 };

/* One MoE layer's device-resident weights. `gate_up_expert_stride` is the byte distance
 * between consecutive experts inside `gate` and `up`: 589,824 for the two separate GGUF
 * tensors ffn_gate_exps / ffn_up_exps, 1,179,648 for one fused HF-style [E, 2I, H] stack
 * (then up = gate + 589,824). `down_expert_stride` is 589,824 for ffn_down_exps. */
typedef struct b200moe_layer {
    const void *gate;
    const void *up;
    int64_t gate_up_expert_stride;
    const void *down;
    int64_t down_expert_stride;
    const void *sh_gate;
    const void *sh_up;
    const void *sh_down;
    const void *router_w;    /* [256][2048] router weights, bf16 or f32 (router_f32) */
    const void *sh_gate_w;   /* [2048] shared-expert gate weights, same type */
    const float *logit_bias; /* [256] f32 added to R1's f32 dot before the bf16 cast, or NULL */
    int32_t router_f32;      /* 0: router_w / sh_gate_w are bf16; 1: f32 (the published file's
                                F32 ffn_gate_inp / ffn_gate_inp_shexp, used exactly) */
    const float *norm_w;     /* [2048] f32 post-attention RMSNorm weight as stored (Form A: the
                                GGUF post_attention_norm holds 1 + w), applied where the library
                                normalises the residual itself (resid / stack modes):
                                x = (resid * rs) * norm_w, two roundings; NULL: weight 1 */
    int32_t down_type;       /* block type of `down`: 0 or B200MOE_TYPE_Q4_K, B200MOE_TYPE_Q5_K,
                                B200MOE_TYPE_Q6_K. down_expert_stride >= 2048 rows x row bytes */
    int32_t sh_type;         /* block type of sh_gate / sh_up / sh_down: 0 or B200MOE_TYPE_Q4_K,
                                B200MOE_TYPE_Q8_0. A layer with any type other than Q4_K runs on
                                the decode paths only (the single-token persistent kernel's
                                format variant, or the gather-GEMV kernels): the grouped GEMMs
                                (moe_prefill, moe_experts) take Q4_K and refuse such a layer
                                (B200MOE_EINVAL) */
    int32_t gate_type;       /* block type of `gate` / `up`: 0 or B200MOE_TYPE_Q4_K, or
                                B200MOE_TYPE_BF16 for a dense layer as the Hugging Face checkpoint
                                stores it -- then down_type and sh_type are B200MOE_TYPE_BF16 too:
                                gate_up [256][1024][2048] (gate = rows 0..511 of each expert, up =
                                rows 512..1023, gate_up_expert_stride 4 MiB), down [256][2048][512]
                                (stride 2 MiB), shared gate / up [512][2048], shared down
                                [2048][512]. A dense layer runs on the gather-GEMV decode kernels
                                at every token count (speccheck/moe_ref.py's weights) */
} b200moe_layer;

/* ABI version (B200MOE_ABI_VERSION) and the last error message on this thread. */
int b200moe_abi_version(void);
const char *b200moe_last_error(void);

/* Q4_K -> f32 (out_dtype B200MOE_F32) or bf16 (B200MOE_BF16, RNE of the f32 value) for
 * `nblocks` consecutive super-blocks, elements in stored order.
 * Replaces tools/gguf_fast_dequant.py:87 dequant_np (Q4_K branch :109-125) and
 * tools/gguf_reader.py:178 dequant -> _deq_q4_k :248-267; bit-exact against both. */
int b200moe_q4k_dequant(const void *blocks, int64_t nblocks, void *out, int out_dtype,
                        void *stream);

/* Q4_K, Q5_K, Q6_K or Q8_0 (`type`, GGML id) -> f32 or bf16 for `nblocks` consecutive blocks,
 * elements in stored order; `out` 16-byte aligned (and Q5_K `blocks`). The published Q4_K_M
 * file stores most expert down matrices as Q5_K, three as Q6_K and the shared expert as Q8_0.
 * Replaces tools/gguf_reader.py:178 dequant (_deq_q8_0 :238, _deq_q5_k :271, _deq_q6_k :299)
 * and tools/gguf_fast_dequant.py:87 dequant_np (:109-150); bit-exact against both. */
int b200moe_dequant(const void *blocks, int type, int64_t nblocks, void *out, int out_dtype,
                    void *stream);

/* Seeded synthetic Q4_K blocks [block0, block0+nblocks) of stream `stream_id` (the
 * benchmark's weight generator; the same bytes as oracle/q4k.py synth_blocks). No
 * counterpart in the reference, which reads a GGUF file instead. */
int b200moe_synth_q4k(uint64_t seed, uint32_t stream_id, int64_t block0, int64_t nblocks,
                      void *out, void *stream);

/* Workspace bytes for b200moe_router with T tokens. */
size_t b200moe_router_workspace_size(int T);

/* Router R1..R5 for T tokens: x [T][2048] (f32 or bf16), W_g [256][2048] bf16 (router_dtype
 * B200MOE_BF16) or f32 (B200MOE_F32), optional f32 logit bias [256]. Outputs (each may be NULL): logits [T][256] bf16, ids [T][8] int32 in
 * top-k rank order, w_f32 [T][8] renormalised weights, w_bf16 [T][8] their R5 bf16 cast.
 * Replaces engine/m3_forward.py:443-446 and engine/block_forward.py:614 moe_router.
 * Deterministic declared order (R1 32x64 chunked fmaf, softmax with the library's own exp,
 * top-8 by (p desc, index asc)); bit-exact against oracle/c/oracle.c b2o_router. */
int b200moe_router(const void *x, int x_dtype, int T, const void *router_w, int router_dtype,
                   const float *logit_bias, uint16_t *logits, int32_t *ids, float *w_f32,
                   uint16_t *w_bf16, void *ws, size_t ws_bytes, void *stream);

/* Workspace bytes for b200moe_moe_decode with T tokens (0 for T outside [1, 65536]). The size
 * never shrinks as T grows, so a workspace sized for T tokens serves every smaller T. */
size_t b200moe_decode_workspace_size(int T);

/* One MoE layer over T tokens (the decode paths): out [T][2048] f32 =
 * routed (8 experts, weights R5-cast, summed in ascending expert id) + sigmoid(w_sg.x) *
 * shared expert. ids_out [T][8] / w_out [T][8] bf16 may be NULL. T = 1 runs the persistent
 * kernel; 2..16 tokens of a Q4_K layer the grouped kernels (each distinct expert's rows read
 * once for all its tokens, exact-product int8 tensor-core dots); otherwise the per-token
 * gather-GEMV kernels.
 * Replaces engine/m3_forward.py:430 moe_block (and the MoE stages of
 * engine/block_forward.py:670 moe_block). */
int b200moe_moe_decode(const void *x, int x_dtype, int T, const b200moe_layer *layer,
                       float *out, int32_t *ids_out, uint16_t *w_out, void *ws,
                       size_t ws_bytes, void *stream);

/* Stage outputs of b200moe_moe_decode_stages; every pointer may be NULL. */
typedef struct b200moe_stages {
    int32_t bf16_stages;      /* 1 (dense BF16 layer and bf16 x only): round where
                                 speccheck/moe_ref.py's "ref" form rounds -- the F.linear outputs
                                 (router logits, gate, up, expert and shared outputs, shared gate
                                 pre-sigmoid), silu, the SwiGLU product, each weighted product, the
                                 running routed sum (ascending expert id), the gated shared output
                                 and the block output; 0: f32 throughout, as b200moe_moe_decode */
    uint16_t *router_logits;  /* [T][256] bf16 */
    float *expert_raw;        /* [T][8][2048] each slot's expert output before weighting, top-k order */
    float *routed_sum;        /* [T][2048] */
    float *shared_raw;        /* [T][2048] the shared expert's output before its gate */
    float *shared_gate;       /* [T] sigmoid(w_sg . x) */
} b200moe_stages;

/* b200moe_moe_decode on the gather-GEMV kernels with the block's stage tensors written out, for
 * stage-level parity gates. Replaces speccheck/moe_ref.py:499 moe_block (its stage dictionary:
 * router_logits, expert_raw, routed_sum, shared_raw, shared_gate_prob, shared_out, combined_out)
 * on dense BF16 weights, and the stage keys of engine/block_forward.py:670 moe_block. */
int b200moe_moe_decode_stages(const void *x, int x_dtype, int T, const b200moe_layer *layer,
                              const b200moe_stages *st, float *out, int32_t *ids_out, uint16_t *w_out,
                              void *ws, size_t ws_bytes, void *stream);

/* Largest token count b200moe_moe_decode_noalloc accepts. */
#define B200MOE_NOALLOC_MAX_T 16

/* b200moe_moe_decode without a caller workspace, for callers that cannot allocate device
 * memory at the point of the call: a plugin inside a host framework that hands it only
 * input/output buffers, code running while a CUDA graph is being captured (allocation is
 * not allowed there), or an FFI caller with no device allocator of its own. No counterpart
 * in the reference, whose CPU path allocates freely.
 * Scratch lives in a fixed static device array inside the library, sized for at most
 * B200MOE_NOALLOC_MAX_T (16) tokens; larger T is refused with B200MOE_ESIZE. The array is
 * resident on every GPU that loads the library for the life of the process. The first call
 * on each device looks up the array's device address (cudaGetSymbolAddress), so make that
 * first call before any stream capture. All calls on a device share the one array: calls
 * that can overlap on the GPU (different streams without ordering) race on it and must be
 * serialised by the caller. Whatever must start at zero is cleared by each call itself.
 * The looked-up address is cached per device ordinal for the life of the process and does not
 * survive cudaDeviceReset (or any re-creation of the device's primary context): do not call
 * this entry point after such a reset. b200moe_decode_noalloc_status reads its status word.
 * For 2..16 tokens it runs the per-token gather-GEMV kernels (the grouped kernels' buffers are
 * not part of the static array), whose outputs agree with b200moe_moe_decode's within the decode
 * parity bar (same routing ids and weights); one token runs the same persistent kernel.
 * Allocates nothing (no cudaMalloc / cudaFree, no allocating library routine). */
int b200moe_moe_decode_noalloc(const void *x, int x_dtype, int T, const b200moe_layer *layer,
                               float *out, int32_t *ids_out, uint16_t *w_out, void *stream);

/* Decode status of the last b200moe_moe_decode / b200moe_stack_decode call made with
 * workspace `ws` and T tokens (b200moe_decode_noalloc_status: of the last
 * b200moe_moe_decode_noalloc call with T tokens), copied to *status; synchronises `stream`.
 * 0 = complete. Bit 1 = a bounded wait of the single-token persistent kernel ran out (a
 * cross-CTA exchange or a weight copy did not complete within its ~1 s budget, e.g. when other
 * work kept some of its CTAs from being resident): that call's outputs are incomplete and must
 * not be used; the three-kernel path (T >= 2) has no such waits and always leaves 0.
 * The reference refuses such a state loudly (engine/m3_forward.py:165-170 Refused); this is the
 * device path's stream-ordered equivalent, like b200moe_prefill_status. */
int b200moe_decode_status(const void *ws, int T, int *status, void *stream);
int b200moe_decode_noalloc_status(int T, int *status, void *stream);

/* Test hook for the persistent decode kernel's failure path (no counterpart in the reference).
 * Every later persistent launch in this process uses a wait budget of `wait_budget_cycles`
 * clock cycles (0 = the default, ~1 s), and CTA `withhold_cta` (0..127; -1 = none) never
 * publishes its first logit pair, so every other CTA's gather runs out of budget: the kernel
 * then ends on every CTA with status bit 1 set and the device context intact. Reset with (0, -1). */
int b200moe_debug_decode_faults(long long wait_budget_cycles, int withhold_cta);

/* Which single-token decode path this device runs. At T = 1, b200moe_moe_decode,
 * b200moe_moe_decode_noalloc and b200moe_stack_decode run one persistent kernel per call
 * (ctas CTAs, one per SM, launched in thread-block clusters of `cluster` CTAs; cluster 1 =
 * a cooperative launch) when the device can keep all of them resident, else the
 * three-kernel-per-layer path (ctas = cluster = 0). Both give the same routing ids and weights;
 * for Q4_K layers the persistent kernel runs the expert dots as exact-product int8 tensor-core
 * MMAs over a 24-bit fixed-point image of x and s, so its outputs agree with the three-kernel
 * path's f32 dots to ~1e-6 relative rather than bit for bit (layers in the other block formats:
 * bit for bit). Every call is deterministic. Introspection only; no counterpart in the
 * reference. Call with the device current. */
int b200moe_decode_persistent_info(int *ctas, int *cluster);

/* *formats = 1 when the persistent kernel also runs single-token layers in the other block
 * formats (Q5_K / Q6_K down, Q8_0 shared: its larger-footprint variant is resident with the
 * same cluster size), else 0 (such layers then take the three-kernel path). Introspection only. */
int b200moe_decode_persistent_formats(int *formats);

/* Workspace bytes for b200moe_stack_decode. */
size_t b200moe_stack_workspace_size(int T, int n_layers);

/* The config-4 MoE sub-stack: for l in 0..n_layers-1:
 *   resid <- resid + moe_block_l(rmsnorm(resid; eps, weight 1))
 * in place on resid [T][2048] f32 (engine/m3_forward.py:731-737 with the mixer sublayers
 * taken out, rmsnorm_a :303-307). `layers` is a HOST array of n_layers descriptors.
 * ids_out [n_layers][T][8] may be NULL. */
int b200moe_stack_decode(float *resid, int T, const b200moe_layer *layers, int n_layers,
                         float eps, int32_t *ids_out, void *ws, size_t ws_bytes, void *stream);

/* Workspace bytes for b200moe_moe_prefill with T tokens. */
size_t b200moe_prefill_workspace_size(int T);

/* One MoE layer over many tokens (the prefill / large-batch path; replaces
 * engine/m3_forward.py:430 moe_block for T tokens): router R1..R5 (same declared order as
 * b200moe_router, so the ids are bit-identical), per-expert token lists in ascending
 * (token, slot) order, Q4_K grouped GEMMs on tcgen05 tensor cores (weights dequantised to
 * fp16 in shared memory, fp16 activations, f32 accumulation in TMEM), and the weighted
 * combine in ascending expert id plus the gated shared expert.
 * If `resid` is non-NULL: x = rmsnorm(resid; eps, weight 1) and resid += block output
 * (x, x_dtype and out are ignored). Otherwise out [T][2048] f32 = block(x).
 * ids_out [T][8] may be NULL. Asynchronous; a pipeline wait that timed out leaves a non-zero
 * status word that b200moe_prefill_status reads back. */
int b200moe_moe_prefill(const void *x, int x_dtype, float *resid, float eps, int T,
                        const b200moe_layer *layer, float *out, int32_t *ids_out, void *ws,
                        size_t ws_bytes, void *stream);

/* The route stage of b200moe_moe_prefill on its own (used by expert parallelism, where a rank
 * routes its own tokens and then ships them to the ranks owning the chosen experts): x (or
 * rmsnorm(resid)) -> x16_out [T][2048] fp16 activations, ids_out [T][8], w_out [T][8] bf16
 * routing weights, sg_out [T] shared-expert gate sigmoid(w_sg.x). Same declared router as
 * b200moe_router. Workspace: b200moe_prefill_workspace_size(T).
 * Replaces engine/m3_forward.py:436-446 (router and shared gate). */
int b200moe_moe_route(const void *x, int x_dtype, float *resid, float eps, int T,
                      const b200moe_layer *layer, void *x16_out, int32_t *ids_out,
                      uint16_t *w_out, float *sg_out, void *ws, size_t ws_bytes, void *stream);

/* The expert stage of b200moe_moe_prefill for pre-routed tokens: for each token, the slots
 * whose expert id lies in [e_lo, e_hi) go through the Q4_K grouped GEMMs (tcgen05), and
 * out[t] (+)= sum over those slots in ascending expert id of w * expert(x) -- plus, for rows
 * t in [sh_lo, sh_hi) when sg is non-NULL, sg[t - sh_lo] * shared_expert(x[t]) (its tiles
 * share the GEMM launches with the routed ones). Slots outside the range are skipped, so a
 * rank of an expert-parallel group passes its own expert range over every gathered token and
 * the shared-expert rows of its own tokens. accumulate != 0 adds into out.
 * Replaces engine/m3_forward.py:447-475 (grouping, expert loop, combine). */
int b200moe_moe_experts(const void *x16, int T, const int32_t *ids, const uint16_t *w_bf16,
                        int e_lo, int e_hi, const float *sg, int sh_lo, int sh_hi,
                        const b200moe_layer *layer, float *out, int accumulate, void *ws,
                        size_t ws_bytes, void *stream);

/* ---- Expert parallelism (one process per GPU; the caller moves the buffers between ranks,
 * e.g. with two equal-split all-to-alls). The reference runs every expert in one process
 * (engine/m3_forward.py:447-475: group the (token, slot) pairs by expert, run each hit expert,
 * combine in ascending expert id); these three calls split that loop across `world` ranks that
 * each own the experts [rank 256/world, (rank+1) 256/world) and T tokens of their own.
 *
 * Dispatch row (B200MOE_EP_ROW_BYTES): 2048 fp16 x values, the token's 8 expert ids (int32),
 * its 8 bf16 routing weights, 16 bytes of padding. */
#define B200MOE_EP_ROW_BYTES 4160

/* Source side, after b200moe_moe_route: fills send_rows [world][T] dispatch rows -- block d holds,
 * in ascending token order, the tokens with at least one slot in d's expert range (every token
 * for d = rank: the shared expert runs there), then rows with ids -1 -- and pos [T][world], the
 * row of token t in block d or -1. Exchange block d with rank d (equal splits of
 * T x B200MOE_EP_ROW_BYTES bytes). */
int b200moe_ep_pack(const void *x16, const int32_t *ids, const uint16_t *w_bf16, int T, int rank, int world,
                    void *send_rows, int32_t *pos, void *stream);

/* Receiver side: recv_rows [world][T] dispatch rows (block s from rank s) -> partial [world][T]
 * [2048] f32: per row, its slots in this rank's expert range through the Q4_K grouped GEMMs,
 * summed in ascending expert id, plus sg[t] * shared_expert(x) on the own block (rows
 * rank T .. rank T + T - 1 = this rank's tokens, sg [T] from b200moe_moe_route); 0 for rows
 * without work. Send block s back to rank s. Workspace: b200moe_prefill_workspace_size(world T).
 * Asynchronous; b200moe_prefill_status(ws, world T, ...) reads its status word. */
int b200moe_ep_experts(const void *recv_rows, int T, int rank, int world, const float *sg,
                       const b200moe_layer *layer, float *partial, void *ws, size_t ws_bytes,
                       void *stream);

/* Source side: out[t] (+= when accumulate) the sum over d = 0 .. world-1 (ascending expert
 * ranges) of ret[d][pos[t][d]] for pos >= 0, where ret [world][T][2048] f32 holds the partial
 * rows sent back by every rank. */
int b200moe_ep_combine(const float *ret, const int32_t *pos, int T, int world, float *out, int accumulate,
                       void *stream);

/* ---- The same three stages over peer memory (NVLink), for up to 8 ranks of one node: the pack
 * writes the dispatch rows straight into each destination's receive buffer and the expert
 * stage's combine writes each partial row straight into its source's return buffer, so only
 * rows that carry work cross NVLink (no padded all-to-all). Each hand-off ends with a
 * release-store of this step's epoch into the receiver's flag word for the sender; the next
 * stage polls its own flag words with acquire loads, bounded (~1 s: status bit 8, then it
 * proceeds). Buffers are shared once with CUDA IPC (b200moe_ipc_*): plain device memory, no
 * multicast object, no library kernel ever reads a peer pointer.
 *
 * Per rank r (identical layouts on every rank): recv [world][T] dispatch rows, ret [world][T]
 * [2048] f32, flag_dispatch [world] and flag_return [world] u32 (zeroed once at set-up), epoch
 * u32 (zeroed once; bumped by each dispatch), status i32. `recv[d]` etc. are rank d's buffers
 * as mapped in this process (this rank's own at index rank). */
typedef struct b200moe_ep_peers {
    int32_t world, rank;
    void *recv[8];
    float *ret[8];
    uint32_t *flag_dispatch[8];
    uint32_t *flag_return[8];
    uint32_t *epoch;
    int32_t *status;
} b200moe_ep_peers;

/* b200moe_ep_pack into the peers' receive buffers, then the dispatch signal. pos [T][world]. */
int b200moe_ep_dispatch_p2p(const void *x16, const int32_t *ids, const uint16_t *w_bf16, int T,
                            const b200moe_ep_peers *peers, int32_t *pos, void *stream);
/* Wait for every source's rows, b200moe_ep_experts on this rank's receive buffer with each
 * partial row stored into its source's return buffer (rows without work are not sent), then the
 * return signal. Workspace: b200moe_prefill_workspace_size(world T). */
int b200moe_ep_experts_p2p(int T, const float *sg, const b200moe_layer *layer, const b200moe_ep_peers *peers,
                           void *ws, size_t ws_bytes, void *stream);
/* Wait for every partial row, then b200moe_ep_combine over this rank's return buffer. */
int b200moe_ep_combine_p2p(int T, const int32_t *pos, const b200moe_ep_peers *peers, float *out, int accumulate,
                           void *stream);

/* CUDA IPC for the buffers above (no counterpart in the reference, which runs on one device):
 * the handle (B200MOE_IPC_HANDLE_BYTES) and offset of the allocation that holds `dptr`; map a
 * peer's handle into this process (*dptr = its base + offset); unmap. */
#define B200MOE_IPC_HANDLE_BYTES 64
int b200moe_ipc_handle(const void *dptr, void *handle, int64_t *offset);
int b200moe_ipc_open(const void *handle, int64_t offset, void **dptr);
int b200moe_ipc_close(void *dptr, int64_t offset);

/* Copy the prefill workspace's device status word to *status (synchronises `stream`). Bits:
 * 1 / 2 = a gate_up / down GEMM pipeline wait exceeded its ~1 s budget; 4 = an fp16 tensor-core
 * operand was out of range (|x| or |silu(gate)*up| * 2^-10 above 65504). 0 = ok. */
int b200moe_prefill_status(const void *ws, int T, int *status, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B200MOE_H */
