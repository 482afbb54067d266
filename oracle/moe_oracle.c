/*
 * CPU oracle for the DeepSeek-V2 MoE block -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg
 * may load this library, and only as the checker or the timed CPU baseline. The product
 * path (libuocr_moe.so) never links or calls it.
 *
 * Every function states, in fp32, an operation order that a CUDA kernel of this build
 * reproduces bit for bit, so GPU results are compared bitwise against it:
 *
 *   oracle_exp_f32        the softmax's exponential (Cody-Waite range reduction by ln 2 with a
 *                         two-constant split, then a degree-7 Taylor polynomial of e^r in
 *                         Horner form, then an exact scale by 2^n). The GPU uses the same
 *                         steps (csrc/common.cuh: uocr_exp), not CUDA's expf.
 *   oracle_router_logit   one router logit: the hidden dim cut in 8 equal segments, each an
 *                         fma chain in ascending k from +0, the 8 segment sums added in
 *                         ascending order. Follows MoEGate.__call__ (decoder.py:509-514,
 *                         logits = x @ Wg^T in fp32); the segment order is this build's.
 *   oracle_route_fp32     MoEGate + routing semantics (decoder.py:500-514,
 *                         model_config.py:52-63,135-150): optional per-expert bias added to the
 *                         logits (benchmark input only), softmax over all experts, greedy
 *                         top-k by (prob desc, index asc), no renormalisation, no scaling.
 *                         The softmax sum is the warp-butterfly order: s_l = e_l + e_{l+32},
 *                         then s_l += s_{l^16}, ^8, ^4, ^2, ^1.
 *   oracle_int8_qmv       moe_int8_qmv's exact order (kernels/moe_int8.mojo:114-148;
 *                         tests/test_kernels_int8.py:173-197): per group
 *                         gsum = fma(q, x, gsum) in ascending k, then acc = fma(scale, gsum, acc).
 *
 * Compile with -ffp-contract=off: every fused multiply-add here is an explicit fmaf.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float f32_from_bits(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ln 2 split for the range reduction: LN2_HI is ln 2 truncated to 16 significant bits
 * (0x3F317200 = 0.693145751953125), LN2_LO = fp32(ln 2 - LN2_HI). Derived from
 * ln 2 = 0.693147180559945309..., nothing else. */
#define UOCR_LN2_HI 0.693145751953125f
#define UOCR_LN2_LO 1.428606765330187e-06f
#define UOCR_LOG2E 1.44269504088896341f
/* below this argument the softmax term is defined as exactly 0 (keeps 2^n normal) */
#define UOCR_EXP_LO (-80.0f)

float oracle_exp_f32(float x) {
    if (!(x >= UOCR_EXP_LO)) return 0.0f; /* also maps NaN to 0 */
    float t = x * UOCR_LOG2E;
    float n = rintf(t);
    float r = fmaf(-n, UOCR_LN2_HI, x);
    r = fmaf(-n, UOCR_LN2_LO, r);
    /* Taylor coefficients 1/k!, k = 7..0, each rounded once from the exact rational */
    float p = (float)(1.0 / 5040.0);
    p = fmaf(p, r, (float)(1.0 / 720.0));
    p = fmaf(p, r, (float)(1.0 / 120.0));
    p = fmaf(p, r, (float)(1.0 / 24.0));
    p = fmaf(p, r, (float)(1.0 / 6.0));
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    float scale = f32_from_bits((uint32_t)(ni + 127) << 23);
    return p * scale;
}

/* One logit: 8 segments of H/8, fma chain per segment from +0, segments summed in order. */
float oracle_router_logit(const float* x, const uint16_t* wrow, int H) {
    int L = H / 8;
    float total = 0.0f;
    for (int s = 0; s < 8; ++s) {
        float acc = 0.0f;
        for (int k = s * L; k < (s + 1) * L; ++k) acc = fmaf(bf16_to_f32(wrow[k]), x[k], acc);
        total = (s == 0) ? acc : total + acc;
    }
    return total;
}

/* Softmax + greedy top-k for one token's E <= 64 logits (already biased). */
static void route_one(const float* logits, int E, int topk, int32_t* ids, float* wts, float* probs_out) {
    float m = logits[0];
    for (int j = 1; j < E; ++j) m = logits[j] > m ? logits[j] : m;
    float e[64];
    for (int j = 0; j < 64; ++j) e[j] = (j < E) ? oracle_exp_f32(logits[j] - m) : 0.0f;
    float s[32];
    for (int l = 0; l < 32; ++l) s[l] = e[l] + e[l + 32];
    for (int off = 16; off >= 1; off >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = s[l] + s[l ^ off];
        memcpy(s, t, sizeof s);
    }
    float sum = s[0];
    float p[64];
    for (int j = 0; j < E; ++j) p[j] = e[j] / sum;
    if (probs_out)
        for (int j = 0; j < E; ++j) probs_out[j] = p[j];
    unsigned long long taken = 0ull;
    for (int r = 0; r < topk; ++r) {
        int best = -1;
        for (int j = 0; j < E; ++j) {
            if (taken >> j & 1ull) continue;
            if (best < 0 || p[j] > p[best]) best = j; /* strict >: the lower index wins a tie */
        }
        taken |= 1ull << best;
        ids[r] = best;
        wts[r] = p[best];
    }
}

/* x [T,H] fp32, wg [E,H] bf16 bits, bias [E] or NULL -> ids [T,topk], wts [T,topk],
 * logits_out [T,E] (biased) and probs_out [T,E] optional. E <= 64, H % 8 == 0. */
int oracle_route_fp32(const float* x, int T, int H, const uint16_t* wg, const float* bias, int E, int topk,
                      int32_t* ids, float* wts, float* logits_out, float* probs_out) {
    if (E < 1 || E > 64 || topk < 1 || topk > E || H % 8) return 1;
    float logits[64];
    for (int t = 0; t < T; ++t) {
        for (int j = 0; j < E; ++j) {
            float l = oracle_router_logit(x + (size_t)t * H, wg + (size_t)j * H, H);
            if (bias) l = l + bias[j];
            logits[j] = l;
            if (logits_out) logits_out[(size_t)t * E + j] = l;
        }
        route_one(logits, E, topk, ids + (size_t)t * topk, wts + (size_t)t * topk,
                  probs_out ? probs_out + (size_t)t * E : 0);
    }
    return 0;
}

static inline int clamp_expert(int32_t e, int E) { return e < 0 ? 0 : (e >= E ? E - 1 : e); }

/* moe_int8_qmv's bits: x [k,K], ids [k], w [E,N,K] int8, scales [E,N,G] -> out [k,N]. */
int oracle_int8_qmv(const float* x, int k, int K, const int32_t* ids, const int8_t* w, const float* scales,
                    int E, int N, int groups, float* out) {
    if (groups < 1 || K % groups) return 1;
    int gsize = K / groups;
    for (int s = 0; s < k; ++s) {
        int e = clamp_expert(ids[s], E);
        const float* xs = x + (size_t)s * K;
        for (int n = 0; n < N; ++n) {
            const int8_t* wr = w + ((size_t)e * N + n) * K;
            const float* sr = scales + ((size_t)e * N + n) * groups;
            float acc = 0.0f;
            for (int g = 0; g < groups; ++g) {
                float gsum = 0.0f;
                for (int kk = g * gsize; kk < (g + 1) * gsize; ++kk) gsum = fmaf((float)wr[kk], xs[kk], gsum);
                acc = fmaf(sr[g], gsum, acc);
            }
            out[(size_t)s * N + n] = acc;
        }
    }
    return 0;
}

/* A plain fp32 elementwise exp over n values (for the accuracy test of oracle_exp_f32). */
void oracle_exp_many(const float* x, float* y, long n) {
    for (long i = 0; i < n; ++i) y[i] = oracle_exp_f32(x[i]);
}
