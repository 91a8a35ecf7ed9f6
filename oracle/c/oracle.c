/* oracle.c -- plain-C restatement of the bit-exact parts of the MoE block hot path.
 *
 * TEST INFRASTRUCTURE ONLY: compiled by oracle/build.py (gcc -O2 -ffp-contract=off
 * -fno-fast-math) into oracle/_build/liboracle.so and called from tests/ through ctypes.
 * The product never links it.
 *
 * What is restated, and from where (reference paths are relative to its project root):
 *   b2o_q4k_dequant   tools/gguf_reader.py:248-267 (_deq_q4_k), get_scale_min_k4 at :165-176.
 *                     f32 route: d*sc, *q and dmin*m are exact in f32, so the one rounding at the
 *                     subtraction equals the reference's f64-then-f32 rounding
 *                     (prototype/q4k_dequant/q4k_dequant_kernels.h:43-60 argues the same).
 *   b2o_router        R1..R5 of engine/m3_forward.py:443-446 and engine/block_forward.py:631-635
 *   (b2o_router_f32w  the same with f32 router weights),
 *                     under the DECLARED deterministic order that the CUDA router also follows:
 *                       R1  logit[e] = bf16_rne( (((c_0 + c_1) + c_2) + ... + c_31) [+ bias[e]] )
 *                           c_j = fmaf-chain over k = 64j .. 64j+63 ascending, starting at 0.0f
 *                       R2  m = max logit; e_l = b2o_expf(logit_l - m);
 *                           S: s_L = sequential sum of e_{8L..8L+7} (L = 0..31), then an xor
 *                           butterfly s_L += s_{L^o} for o = 16, 8, 4, 2, 1; p_l = e_l / S
 *                       R3  top-8 by (bf16 logit descending, expert index ascending); the
 *                           softmax is monotone in the logit, so this is the reference's top-k
 *                           over probabilities with its unspecified tie order fixed to the
 *                           reference kernel's strict-> rule (moe_router_kernels.h:289-321)
 *                       R4  s8 = sequential sum of the 8 p in rank order; w_k = p_k / s8
 *                       R5  w_bf16 = bf16_rne(w_k)  (cast BEFORE any multiply,
 *                           specification/11-moe-block.md:39-60)
 *   b2o_expf          own exp: Cody-Waite two-constant range reduction x = n*ln2 + r and a
 *                     degree-7 Taylor polynomial in Horner form (J.-M. Muller, "Elementary
 *                     Functions", ch. 11). Only IEEE basic operations, so the CUDA copy in
 *                     qwen3.6-35b-a3b_b200/csrc/common.cuh is bit-identical to this one.
 *   b2o_rmsnorm       engine/m3_forward.py:303-307 (rmsnorm_a, weight 1), declared order:
 *                     ss = the R1 chunk order applied to x.x (32 chunks of 64 sequential fmaf,
 *                     chunk sums added left to right); r = 1/sqrtf(ss/2048 + eps); y = x*r.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define H 2048
#define E 256
#define TOPK 8

static float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t ex = (h >> 10) & 0x1F, man = h & 0x3FF;
    uint32_t u;
    if (ex == 0) {
        float v = (float)man * 5.9604644775390625e-8f; /* 2^-24, exact */
        return sign ? -v : v;
    } else if (ex == 31) {
        u = sign | 0x7F800000u | (man << 13);
    } else {
        u = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static float pow2i(int n) { /* 2^n for -126 <= n <= 127 */
    uint32_t u = (uint32_t)(n + 127) << 23;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float b2o_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541016f) return 0.0f;
    float t = x * 1.44269502162933349609375f;
    float n = rintf(t);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.428606765330187045e-06f, r);
    float p = 1.984126984126984e-04f;
    p = fmaf(p, r, 1.388888888888889e-03f);
    p = fmaf(p, r, 8.333333333333333e-03f);
    p = fmaf(p, r, 4.166666666666667e-02f);
    p = fmaf(p, r, 1.666666666666667e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) return (p * pow2i(127)) * 2.0f;
    if (ni < -126) return (p * pow2i(ni + 64)) * pow2i(-64);
    return p * pow2i(ni);
}

void b2o_q4k_dequant(const uint8_t *blk, int64_t nb, float *out) {
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *p = blk + b * 144;
        const float d = f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
        const float dmin = f16_to_f32((uint16_t)(p[2] | (p[3] << 8)));
        const uint8_t *q = p + 4;
        for (int j = 0; j < 8; ++j) {
            uint32_t sc, m;
            if (j < 4) {
                sc = q[j] & 63u;
                m = q[j + 4] & 63u;
            } else {
                sc = (q[j + 4] & 0xFu) | ((q[j - 4] >> 6) << 4);
                m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
            }
            const float scale = d * (float)sc;
            const float mins = dmin * (float)m;
            for (int l = 0; l < 32; ++l) {
                const uint8_t byte = p[16 + 32 * (j >> 1) + l];
                const uint32_t qv = (j & 1) ? (byte >> 4) : (byte & 15u);
                out[b * 256 + 32 * j + l] = fmaf(scale, (float)qv, -mins);
            }
        }
    }
}

/* R1 for one (token, expert): the declared 32-chunk order, weights as f32 values (a bf16 router
 * widens exactly, so both router widths share this arithmetic). */
static float logit_f32(const float *x, const float *w) {
    float tot = 0.0f;
    for (int c = 0; c < 32; ++c) {
        float acc = 0.0f;
        for (int i = 0; i < 64; ++i) {
            const int k = 64 * c + i;
            acc = fmaf(x[k], w[k], acc);
        }
        tot = (c == 0) ? acc : tot + acc;
    }
    return tot;
}

float b2o_dot_chunked(const float *x, const uint16_t *w) {
    float wf[H];
    for (int k = 0; k < H; ++k) wf[k] = bf16_to_f32(w[k]);
    return logit_f32(x, wf);
}

/* The router with f32 router weights (the published file stores ffn_gate_inp as F32). */
void b2o_router_f32w(const float *x, int T, const float *wg, const float *bias, uint16_t *logits_out,
                     float *probs_out, int32_t *ids, float *w_f32, uint16_t *w_bf16);

void b2o_router(const float *x, int T, const uint16_t *wg, const float *bias, uint16_t *logits_out,
                float *probs_out, int32_t *ids, float *w_f32, uint16_t *w_bf16) {
    static float wf[(int64_t)E * H];
    for (int64_t k = 0; k < (int64_t)E * H; ++k) wf[k] = bf16_to_f32(wg[k]);
    b2o_router_f32w(x, T, wf, bias, logits_out, probs_out, ids, w_f32, w_bf16);
}

void b2o_router_f32w(const float *x, int T, const float *wg, const float *bias, uint16_t *logits_out,
                     float *probs_out, int32_t *ids, float *w_f32, uint16_t *w_bf16) {
    for (int t = 0; t < T; ++t) {
        const float *xt = x + (int64_t)t * H;
        float lg[E], ev[E], pr[E];
        for (int e = 0; e < E; ++e) {
            float v = logit_f32(xt, wg + (int64_t)e * H);
            if (bias) v = v + bias[e];
            uint16_t b = f32_to_bf16(v);
            if (logits_out) logits_out[(int64_t)t * E + e] = b;
            lg[e] = bf16_to_f32(b);
        }
        float m = lg[0];
        for (int e = 1; e < E; ++e)
            if (lg[e] > m) m = lg[e];
        for (int e = 0; e < E; ++e) ev[e] = b2o_expf(lg[e] - m);
        float s[32], s2[32];
        for (int L = 0; L < 32; ++L) {
            float a = ev[8 * L];
            for (int i = 1; i < 8; ++i) a = a + ev[8 * L + i];
            s[L] = a;
        }
        for (int o = 16; o >= 1; o >>= 1) {
            for (int L = 0; L < 32; ++L) s2[L] = s[L] + s[L ^ o];
            memcpy(s, s2, sizeof(s));
        }
        const float S = s[0];
        for (int e = 0; e < E; ++e) pr[e] = ev[e] / S;
        if (probs_out) memcpy(probs_out + (int64_t)t * E, pr, sizeof(pr));
        int used[E];
        memset(used, 0, sizeof(used));
        int sel[TOPK];
        for (int k = 0; k < TOPK; ++k) {
            int best = -1;
            float bv = 0.0f;
            for (int e = 0; e < E; ++e) {
                if (used[e]) continue;
                if (best < 0 || lg[e] > bv) { /* strict >: an exact tie keeps the lower index */
                    best = e;
                    bv = lg[e];
                }
            }
            used[best] = 1;
            sel[k] = best;
        }
        float s8 = 0.0f;
        for (int k = 0; k < TOPK; ++k) s8 = s8 + pr[sel[k]];
        for (int k = 0; k < TOPK; ++k) {
            const float w = (s8 == 0.0f) ? 0.0f : pr[sel[k]] / s8;
            ids[(int64_t)t * TOPK + k] = sel[k];
            if (w_f32) w_f32[(int64_t)t * TOPK + k] = w;
            if (w_bf16) w_bf16[(int64_t)t * TOPK + k] = f32_to_bf16(w);
        }
    }
}

void b2o_rmsnorm(const float *x, int T, float eps, float *y) {
    for (int t = 0; t < T; ++t) {
        const float *xt = x + (int64_t)t * H;
        float ss = 0.0f;
        for (int c = 0; c < 32; ++c) {
            float acc = 0.0f;
            for (int i = 0; i < 64; ++i) acc = fmaf(xt[64 * c + i], xt[64 * c + i], acc);
            ss = (c == 0) ? acc : ss + acc;
        }
        const float r = 1.0f / sqrtf(ss / (float)H + eps);
        for (int k = 0; k < H; ++k) y[(int64_t)t * H + k] = xt[k] * r;
    }
}
