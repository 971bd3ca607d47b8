/*
 * tsg_oracle.c -- CPU restatement of Tsugumi's MoE feed-forward block.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in tsugumi_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * path never links, loads or calls it.
 *
 * The reference is Swift + Metal (he-be/tsugumi) and cannot run in this
 * environment (no Swift toolchain, no Metal).  This is a from-scratch C
 * restatement of the reference's CPU reference and host-side algorithms.
 * Each function names the reference file:line it follows (paths relative to
 * the reference project root).
 *
 * Formats (the build's target format; where the reference differs it is said):
 *   - expert weights: int4 symmetric, w = s * (q - 8), q in [0, 15] stored as
 *     nibbles, low nibble = even element, group of 32 along K, fp16 scales.
 *     The reference stores bf16 scales (Quantization.swift:86-99, :166-208).
 *   - activations: bf16 in, results in fp32.
 *   - router: fp32 W [E, D].
 *
 * Arithmetic: every dot product accumulates in double ("fp32-accumulated
 * reference"), elementwise maths in double, results rounded to float.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OK 0
/* Error codes mirror PrefillMoEGroupingError
 * (Sources/Tsugumi/Kernels/Prefill/MoE/PrefillMoEGrouping.swift:52-88). */
#define ORC_ERR_INVALID_QUERY_COUNT 1
#define ORC_ERR_INVALID_TOPK 2
#define ORC_ERR_INVALID_NUM_EXPERTS 3
#define ORC_ERR_INVALID_TILE_EXPERT_COUNT 4
#define ORC_ERR_PAIR_COUNT_MISMATCH 5
#define ORC_ERR_TOKEN_OUT_OF_RANGE 6
#define ORC_ERR_RANK_OUT_OF_RANGE 7
#define ORC_ERR_EXPERT_OUT_OF_RANGE 8
#define ORC_ERR_DUPLICATE_TOKEN_RANK 9
#define ORC_ERR_SORT_KEY_COUNT_MISMATCH 10
#define ORC_ERR_ALLOC 11

/* ------------------------------------------------------------------------ */
/* PRNG: SplitMix64 + SeedTree                                               */
/* ------------------------------------------------------------------------ */

/* Sources/TsugumiValidation/Support/PRNG/SplitMix64.swift:10-16 */
uint64_t orc_splitmix64_next(uint64_t *state) {
    *state += 0x9E3779B97F4A7C15ull;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* SplitMix64.swift:19-22: uniform in [lo, hi) with 24 bits. */
float orc_splitmix64_uniform(uint64_t *state, float lo, float hi) {
    float u = (float)(orc_splitmix64_next(state) >> 40) / (float)(1u << 24);
    return lo + (hi - lo) * u;
}

/* Sources/TsugumiValidation/Support/PRNG/SeedTree.swift:11-18: FNV-1a of the
 * label xor the root gives the child stream's seed. */
uint64_t orc_seedtree_key(uint64_t root, const char *label) {
    uint64_t h = 0xCBF29CE484222325ull;
    for (const unsigned char *p = (const unsigned char *)label; *p; ++p) {
        h ^= (uint64_t)(*p);
        h *= 0x100000001B3ull;
    }
    return root ^ h;
}

/* ------------------------------------------------------------------------ */
/* 16-bit float helpers                                                      */
/* ------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Quantization.swift:63-69: bf16 bits with round-half-to-even. */
uint16_t orc_bf16_bits(float x) {
    uint32_t bits = f2u(x);
    uint32_t lsb = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7FFFu + lsb) >> 16);
}

/* Quantization.swift:71-74 */
float orc_bf16_to_f32(uint16_t b) { return u2f(((uint32_t)b) << 16); }

/* IEEE binary16 -> binary32 (exact). */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        /* subnormal: man * 2^-24 */
        float v = (float)man * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7F800000u | (man << 13));
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* binary32 -> binary16, round to nearest even, saturating to inf. */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) { /* inf or nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
    if (ax < 0x38800000u) { /* below fp16 min normal: subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to 0 */
        /* value = m * 2^(e-150); in fp16 subnormal units of 2^-24 that is
         * m >> (126 - e), with 126 - e in [14, 24] here. */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t sh = 126u - e;
        uint32_t r = m >> sh;
        uint32_t rem = m & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t r = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

/* ------------------------------------------------------------------------ */
/* int4 symmetric weight format                                              */
/* ------------------------------------------------------------------------ */

/* Restates Quantization.quantizeInt4Symmetric (Quantization.swift:166-208):
 * scale = max(-wmin/8, wmax/7, FLT_MIN) rounded to the scale format, then
 * q = clamp(round(w / scale) + 8, 0, 15).  This build's scale format is fp16
 * (the reference rounds to bf16). */
void orc_quantize_int4_sym(const float *row, int n, int group, uint8_t *packed,
                           uint16_t *scales_f16) {
    int ngroups = n / group;
    memset(packed, 0, (size_t)n / 2);
    for (int g = 0; g < ngroups; ++g) {
        float wmin = INFINITY, wmax = -INFINITY;
        for (int k = 0; k < group; ++k) {
            float w = row[g * group + k];
            if (w < wmin) wmin = w;
            if (w > wmax) wmax = w;
        }
        float s = fmaxf(fmaxf(-wmin / 8.0f, wmax / 7.0f), 1.17549435e-38f);
        uint16_t sb = orc_f32_to_f16(s);
        if ((sb & 0x7FFFu) == 0) sb = 0x0001u; /* keep the scale non-zero */
        scales_f16[g] = sb;
        float scale = orc_f16_to_f32(sb);
        float inv = scale == 0.0f ? 0.0f : 1.0f / scale;
        for (int k = 0; k < group; ++k) {
            float t = row[g * group + k] * inv;
            /* Swift's rounded() rounds half away from zero. */
            int q = (int)(t >= 0.0f ? floorf(t + 0.5f) : ceilf(t - 0.5f)) + 8;
            if (q < 0) q = 0;
            if (q > 15) q = 15;
            int byte = g * (group / 2) + k / 2;
            if ((k & 1) == 0) packed[byte] = (uint8_t)((packed[byte] & 0xF0u) | (uint8_t)q);
            else packed[byte] = (uint8_t)((packed[byte] & 0x0Fu) | (uint8_t)(q << 4));
        }
    }
}

/* Restates Quantization.dequantizeInt4Affine (Quantization.swift:210-227) for
 * the sym scheme, where bias == -8 * scale exactly (Quantization.swift:45-52). */
void orc_dequant_int4_sym_row(const uint8_t *packed, const uint16_t *scales_f16,
                              int n, int group, float *out) {
    int ngroups = n / group;
    for (int g = 0; g < ngroups; ++g) {
        float scale = orc_f16_to_f32(scales_f16[g]);
        float bias = -8.0f * scale;
        for (int k = 0; k < group; ++k) {
            uint8_t b = packed[g * (group / 2) + k / 2];
            int nib = (k & 1) == 0 ? (b & 0x0F) : (b >> 4);
            out[g * group + k] = (float)nib * scale + bias;
        }
    }
}

/* Restates DequantInt4GemvRef.apply
 * (Sources/TsugumiValidation/Support/Reference/Quant/DequantInt4Gemv.swift:12-44):
 * dequantise each row, then dot with x.  Accumulates in double. */
static void gemv_int4_sym(const uint8_t *codes, const uint16_t *scales, int m, int n,
                          int group, const double *x, double *y, float *rowbuf) {
    for (int r = 0; r < m; ++r) {
        orc_dequant_int4_sym_row(codes + (size_t)r * (n / 2),
                                 scales + (size_t)r * (n / group), n, group, rowbuf);
        double acc = 0.0;
        for (int k = 0; k < n; ++k) acc += (double)rowbuf[k] * x[k];
        y[r] = acc;
    }
}

/* ------------------------------------------------------------------------ */
/* Activations                                                               */
/* ------------------------------------------------------------------------ */

/* MoeRef.geluTanh (Sources/TsugumiValidation/Support/Reference/MoE/Moe.swift:16-29):
 * 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))). */
double orc_gelu_tanh(double x) {
    const double c = 0.7978845608028654;
    const double k = 0.044715;
    return 0.5 * x * (1.0 + tanh(c * (x + k * x * x * x)));
}

/* moe.metal:114-118 (FC_MOE_ACT_SILU arm): x / (1 + e^-x). */
double orc_silu(double x) { return x / (1.0 + exp(-x)); }

/* Scripts/qwen35/reference_forward.py:53-54 and qwen.metal:423-460. */
double orc_sigmoid(double x) { return 1.0 / (1.0 + exp(-x)); }

static inline double act_fn(int act, double g) {
    return act == 1 ? orc_silu(g) : orc_gelu_tanh(g);
}

/* ------------------------------------------------------------------------ */
/* Layer description                                                         */
/* ------------------------------------------------------------------------ */

/* Byte offsets of one expert's sub-tensors inside its blob; mirrors
 * MoEExpertOffsets (Sources/Tsugumi/Kernels/MoE/MoE.swift:4-29).  The bias
 * offsets are carried for layout compatibility and never read (sym). */
typedef struct {
    uint32_t gate_w_off, gate_s_off, gate_b_off;
    uint32_t up_w_off, up_s_off, up_b_off;
    uint32_t down_w_off, down_s_off, down_b_off;
} orc_expert_offsets;

typedef struct {
    int d, f, num_experts, top_k, group;
    int act; /* 0 = gelu_pytorch_tanh (Gemma), 1 = SiLU (Qwen) */
    const uint8_t *experts;      /* E blobs, expert_stride bytes apart */
    uint64_t expert_stride;
    orc_expert_offsets off;
    const float *router_w;         /* [E, D] */
    const float *effective_scale;  /* [D] or NULL (= 1) */
    const float *per_expert_scale; /* [E] or NULL (= 1) */
    const float *logit_bias;       /* [E] or NULL (= 0) */
    int router_norm;               /* 1: no-scale RMSNorm of the input */
    float norm_eps;
    /* optional shared expert */
    const uint8_t *shared;
    int shared_f;
    orc_expert_offsets shared_off;
    const float *shared_gate_w;    /* [D] or NULL: no sigmoid gate */
} orc_layer;

/* One expert FFN, MoeRef.runFFN (Moe.swift:33-56): gate GEMV, up GEMV,
 * act(gate) * up, down GEMV.  All in double. */
static void expert_ffn(const orc_layer *L, const uint8_t *blob, const orc_expert_offsets *o,
                       int f, const double *x, double *out, double *g, double *u,
                       double *a, float *rowbuf) {
    const int d = L->d, G = L->group;
    gemv_int4_sym(blob + o->gate_w_off, (const uint16_t *)(blob + o->gate_s_off), f, d, G, x, g,
                  rowbuf);
    gemv_int4_sym(blob + o->up_w_off, (const uint16_t *)(blob + o->up_s_off), f, d, G, x, u,
                  rowbuf);
    for (int i = 0; i < f; ++i) a[i] = act_fn(L->act, g[i]) * u[i];
    gemv_int4_sym(blob + o->down_w_off, (const uint16_t *)(blob + o->down_s_off), d, f, G, a, out,
                  rowbuf);
}

/* ------------------------------------------------------------------------ */
/* Router                                                                    */
/* ------------------------------------------------------------------------ */

/* rmsnorm_no_scale (Sources/Tsugumi/Metal/Primitives/rmsnorm.metal:154-175):
 * 1 / sqrt(mean(x^2) + eps). */
double orc_inv_rms(const float *x, int d, float eps) {
    double s = 0.0;
    for (int i = 0; i < d; ++i) s += (double)x[i] * (double)x[i];
    return 1.0 / sqrt(s / (double)d + (double)eps);
}

/* Router logit for one row, router_gemv_gemma4_bf16_body (moe.metal:187-213):
 * logit[e] = sum_i W[e,i] * x_i * eff_scale_i, plus the optional per-expert
 * logit bias this build adds for the skewed configurations. */
static void router_logits_row(const orc_layer *L, const double *xr, double *logits) {
    for (int e = 0; e < L->num_experts; ++e) {
        const float *w = L->router_w + (size_t)e * L->d;
        double acc = 0.0;
        for (int i = 0; i < L->d; ++i) {
            double xi = xr[i] * (L->effective_scale ? (double)L->effective_scale[i] : 1.0);
            acc += (double)w[i] * xi;
        }
        if (L->logit_bias) acc += (double)L->logit_bias[e];
        logits[e] = acc;
    }
}

/* Top-K selection with the kernel's tie rule and renormalised softmax
 * weights.  Follows router_topk_select_k8_body (moe.metal:281-329),
 * prefill_router_emit_topk (prefill.metal:555-606), the host twin
 * QwenForwardRunner.rankLogits (QwenForwardRunner.swift:1517-1541) and the
 * test reference RouterTopKTests.reference
 * (Tests/Tsugumi/Core/Kernels/MoE/RouterTopKTests.swift:270-295):
 * insertion into a K-slot list, a score wins a slot when strictly greater,
 * or equal with a lower expert index; w_k = exp(s_k - s_0) / sum_j exp(s_j -
 * s_0) * per_expert_scale[e_k].  Returns the K-th / (K+1)-th logit gap. */
double orc_topk_select(const double *logits, int num_experts, int k,
                       const float *per_expert_scale, uint32_t *out_idx, float *out_w) {
    int idx[256];
    double score[256];
    for (int i = 0; i <= k && i < 256; ++i) { idx[i] = 0; score[i] = -INFINITY; }
    int slots = k + 1 <= num_experts ? k + 1 : k; /* keep one extra to measure the gap */
    for (int e = 0; e < num_experts; ++e) {
        double s = logits[e];
        if (s <= score[slots - 1] && !(s == score[slots - 1] && e < idx[slots - 1])) continue;
        int pos = slots;
        for (int i = 0; i < slots; ++i) {
            if (s > score[i] || (s == score[i] && e < idx[i])) { pos = i; break; }
        }
        if (pos >= slots) continue;
        for (int i = slots - 1; i > pos; --i) { idx[i] = idx[i - 1]; score[i] = score[i - 1]; }
        idx[pos] = e;
        score[pos] = s;
    }
    double mx = score[0], sum = 0.0, ex[256];
    for (int i = 0; i < k; ++i) { ex[i] = exp(score[i] - mx); sum += ex[i]; }
    for (int i = 0; i < k; ++i) {
        out_idx[i] = (uint32_t)idx[i];
        double gain = per_expert_scale ? (double)per_expert_scale[idx[i]] : 1.0;
        out_w[i] = (float)(ex[i] / sum * gain);
    }
    return slots > k ? score[k - 1] - score[k] : INFINITY;
}

/* Router over T rows: optional no-scale RMSNorm, logits, top-K.  Writes ids
 * [T, K], weights [T, K], the boundary gap per row [T] (optional) and the
 * fp32 logits [T, E] (optional). */
void orc_router(const orc_layer *L, const uint16_t *x_bf16, int T, uint32_t *ids, float *w,
                double *gap, float *logits_out) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int t = 0; t < T; ++t) {
        const int d = L->d;
        float *xf = (float *)malloc(sizeof(float) * d);
        double *xr = (double *)malloc(sizeof(double) * d);
        double *lg = (double *)malloc(sizeof(double) * L->num_experts);
        for (int i = 0; i < d; ++i) xf[i] = orc_bf16_to_f32(x_bf16[(size_t)t * d + i]);
        double inv = L->router_norm ? orc_inv_rms(xf, d, L->norm_eps) : 1.0;
        for (int i = 0; i < d; ++i) xr[i] = (double)xf[i] * inv;
        router_logits_row(L, xr, lg);
        double g = orc_topk_select(lg, L->num_experts, L->top_k, L->per_expert_scale,
                                   ids + (size_t)t * L->top_k, w + (size_t)t * L->top_k);
        if (gap) gap[t] = g;
        if (logits_out)
            for (int e = 0; e < L->num_experts; ++e)
                logits_out[(size_t)t * L->num_experts + e] = (float)lg[e];
        free(xf); free(xr); free(lg);
    }
}

/* ------------------------------------------------------------------------ */
/* The whole block                                                           */
/* ------------------------------------------------------------------------ */

/* MoE block for T rows.  The routed part follows MoeRef.applyStreamedRouted
 * (Moe.swift:90-121): y = residual + sum over slots, in slot order, of
 * w_slot * FFN_e(x).  With a shared expert the residual is the shared
 * branch, sigmoid(w_s . x) * FFN_shared(x), as in
 * QwenForwardRunner.encodeSharedExpert / encodeRoutedExperts
 * (QwenForwardRunner.swift:1548-1612) and ReferenceModel._moe
 * (Scripts/qwen35/reference_forward.py:300-334).
 *
 * The expert input is x scaled by the row's inverse RMS when router_norm is
 * set (the router input is normalised, rmsnorm.metal:154-175), else x.
 * If ids/w are given (ids_in != NULL) they replace the router's choice, which
 * lets a test feed the GPU's routing into the expert maths. */
void orc_moe_block(const orc_layer *L, const uint16_t *x_bf16, int T, const uint32_t *ids_in,
                   const float *w_in, float *y, uint32_t *ids_out, float *w_out) {
    const int d = L->d, K = L->top_k;
    const int U = K + (L->shared ? 1 : 0); /* units per token: K routed slots (+ shared) */
    const int CH = 64;                      /* tokens per chunk */
    const int fmax = L->f > L->shared_f ? L->f : L->shared_f;
    double *xe = (double *)malloc(sizeof(double) * (size_t)CH * d);
    double *outs = (double *)malloc(sizeof(double) * (size_t)CH * U * d);
    double *gates = (double *)malloc(sizeof(double) * CH);
    uint32_t *ids = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)CH * K);
    float *ws = (float *)malloc(sizeof(float) * (size_t)CH * K);
    for (int t0 = 0; t0 < T; t0 += CH) {
        const int nt = T - t0 < CH ? T - t0 : CH;
        /* 1. per token: normalised input, routing, shared-gate logit */
#pragma omp parallel for schedule(dynamic, 1)
        for (int i = 0; i < nt; ++i) {
            const int t = t0 + i;
            float *xf = (float *)malloc(sizeof(float) * d);
            double *lg = (double *)malloc(sizeof(double) * L->num_experts);
            for (int k = 0; k < d; ++k) xf[k] = orc_bf16_to_f32(x_bf16[(size_t)t * d + k]);
            double inv = L->router_norm ? orc_inv_rms(xf, d, L->norm_eps) : 1.0;
            double *xi = xe + (size_t)i * d;
            for (int k = 0; k < d; ++k) xi[k] = (double)xf[k] * inv;
            if (ids_in) {
                for (int r = 0; r < K; ++r) {
                    ids[i * K + r] = ids_in[(size_t)t * K + r];
                    ws[i * K + r] = w_in[(size_t)t * K + r];
                }
            } else {
                router_logits_row(L, xi, lg);
                orc_topk_select(lg, L->num_experts, K, L->per_expert_scale, ids + i * K, ws + i * K);
            }
            gates[i] = 1.0;
            if (L->shared && L->shared_gate_w) {
                double s = 0.0;
                for (int k = 0; k < d; ++k) s += (double)L->shared_gate_w[k] * xi[k];
                gates[i] = orc_sigmoid(s);
            }
            free(xf);
            free(lg);
        }
        /* 2. every (token, slot) expert FFN, MoeRef.runFFN (Moe.swift:33-56) */
#pragma omp parallel for schedule(dynamic, 1)
        for (int uu = 0; uu < nt * U; ++uu) {
            const int i = uu / U, slot = uu % U;
            double *g = (double *)malloc(sizeof(double) * fmax);
            double *u = (double *)malloc(sizeof(double) * fmax);
            double *a = (double *)malloc(sizeof(double) * fmax);
            float *rowbuf = (float *)malloc(sizeof(float) * (d > fmax ? d : fmax));
            double *o = outs + (size_t)uu * d;
            if (slot < K) {
                const uint8_t *blob = L->experts + (size_t)ids[i * K + slot] * L->expert_stride;
                expert_ffn(L, blob, &L->off, L->f, xe + (size_t)i * d, o, g, u, a, rowbuf);
            } else {
                expert_ffn(L, L->shared, &L->shared_off, L->shared_f, xe + (size_t)i * d, o, g, u,
                           a, rowbuf);
            }
            free(g); free(u); free(a); free(rowbuf);
        }
        /* 3. combine in slot order, MoeRef.applyStreamedRouted (Moe.swift:90-121),
         * starting from the gated shared branch (QwenForwardRunner.swift:1583-1612) */
#pragma omp parallel for schedule(static)
        for (int i = 0; i < nt; ++i) {
            const int t = t0 + i;
            for (int k = 0; k < d; ++k) {
                double acc = 0.0;
                if (L->shared) acc = gates[i] * outs[((size_t)i * U + K) * d + k];
                for (int r = 0; r < K; ++r)
                    acc += (double)ws[i * K + r] * outs[((size_t)i * U + r) * d + k];
                y[(size_t)t * d + k] = (float)acc;
            }
            if (ids_out) for (int r = 0; r < K; ++r) ids_out[(size_t)t * K + r] = ids[i * K + r];
            if (w_out) for (int r = 0; r < K; ++r) w_out[(size_t)t * K + r] = ws[i * K + r];
        }
    }
    free(xe); free(outs); free(gates); free(ids); free(ws);
}

/* Shared expert alone, SharedExpertInt4.encode (SharedExpertInt4.swift:30-94)
 * plus the Qwen sigmoid gate (qwen.metal:423-460).  y [T, D]. */
void orc_shared_expert(const orc_layer *L, const uint16_t *x_bf16, int T, float *y) {
    const int d = L->d;
#pragma omp parallel for schedule(dynamic, 1)
    for (int t = 0; t < T; ++t) {
        int f = L->shared_f;
        float *xf = (float *)malloc(sizeof(float) * d);
        double *xe = (double *)malloc(sizeof(double) * d);
        double *out = (double *)malloc(sizeof(double) * d);
        double *g = (double *)malloc(sizeof(double) * f);
        double *u = (double *)malloc(sizeof(double) * f);
        double *a = (double *)malloc(sizeof(double) * f);
        float *rowbuf = (float *)malloc(sizeof(float) * (d > f ? d : f));
        for (int i = 0; i < d; ++i) xf[i] = orc_bf16_to_f32(x_bf16[(size_t)t * d + i]);
        double inv = L->router_norm ? orc_inv_rms(xf, d, L->norm_eps) : 1.0;
        for (int i = 0; i < d; ++i) xe[i] = (double)xf[i] * inv;
        expert_ffn(L, L->shared, &L->shared_off, f, xe, out, g, u, a, rowbuf);
        double gate = 1.0;
        if (L->shared_gate_w) {
            double s = 0.0;
            for (int i = 0; i < d; ++i) s += (double)L->shared_gate_w[i] * xe[i];
            gate = orc_sigmoid(s);
        }
        for (int i = 0; i < d; ++i) y[(size_t)t * d + i] = (float)(gate * out[i]);
        free(xf); free(xe); free(out); free(g); free(u); free(a); free(rowbuf);
    }
}

/* ------------------------------------------------------------------------ */
/* Permutation, planner and combine                                          */
/* ------------------------------------------------------------------------ */

/* PrefillTokenExpertPair (Sources/Tsugumi/Kernels/Prefill/MoE/PrefillRouter.swift:4-28):
 * 16 bytes, fields at 0/4/8/12. */
typedef struct {
    uint32_t token, expert, rank, weight_bits;
} orc_pair;

typedef struct { uint32_t expert, pair_start, pair_count; } orc_group;
typedef struct { uint32_t group_start, group_count, pair_start, pair_count; } orc_tile;

/* PrefillRouter.makeTokenExpertPairs (PrefillRouter.swift:238-258):
 * token-major pairs, weight carried as fp16 bits. */
void orc_make_pairs(const uint32_t *ids, const uint16_t *w_f16, int T, int K, orc_pair *out) {
    for (int t = 0; t < T; ++t)
        for (int r = 0; r < K; ++r) {
            int i = t * K + r;
            out[i].token = (uint32_t)t;
            out[i].expert = ids[i];
            out[i].rank = (uint32_t)r;
            out[i].weight_bits = w_f16 ? (uint32_t)w_f16[i] : 0u;
        }
}

static const uint64_t *g_sort_keys;
static int pair_cmp(const void *pa, const void *pb) {
    const orc_pair *a = (const orc_pair *)pa, *b = (const orc_pair *)pb;
    if (g_sort_keys) {
        uint64_t ka = g_sort_keys[a->expert], kb = g_sort_keys[b->expert];
        if (ka != kb) return ka < kb ? -1 : 1;
    }
    if (a->expert != b->expert) return a->expert < b->expert ? -1 : 1;
    if (a->token != b->token) return a->token < b->token ? -1 : 1;
    if (a->rank != b->rank) return a->rank < b->rank ? -1 : 1;
    return 0;
}

/* PrefillMoEGrouping.groupTokenExpertPairs (PrefillMoEGrouping.swift:91-201):
 * validate, sort by (sortKey, expert, token, rank), per-expert offsets
 * (UINT32_MAX when empty) and counts, groups, tiles of <= tileExpertCount
 * groups with the optional forced cut after group tile_break (pass -1 for
 * none).  out_error_value receives the offending value of a failed check.
 * Returns ORC_OK or one of the ORC_ERR_* codes. */
int orc_group_pairs(const orc_pair *pairs, int n_pairs, int query_count, int top_k,
                    int num_experts, int tile_expert_count, const uint64_t *sort_keys,
                    int n_sort_keys, int tile_break, orc_pair *sorted, uint32_t *offsets,
                    uint32_t *counts, orc_group *groups, int *n_groups, orc_tile *tiles,
                    int *n_tiles, uint32_t *out_error_value) {
    if (query_count < 0) { *out_error_value = (uint32_t)query_count; return ORC_ERR_INVALID_QUERY_COUNT; }
    if (top_k <= 0) { *out_error_value = (uint32_t)top_k; return ORC_ERR_INVALID_TOPK; }
    if (num_experts <= 0) { *out_error_value = (uint32_t)num_experts; return ORC_ERR_INVALID_NUM_EXPERTS; }
    if (tile_expert_count < 1 || tile_expert_count > 16) {
        *out_error_value = (uint32_t)tile_expert_count;
        return ORC_ERR_INVALID_TILE_EXPERT_COUNT;
    }
    if (sort_keys && n_sort_keys != num_experts) {
        *out_error_value = (uint32_t)n_sort_keys;
        return ORC_ERR_SORT_KEY_COUNT_MISMATCH;
    }
    if (n_pairs != query_count * top_k) { *out_error_value = (uint32_t)n_pairs; return ORC_ERR_PAIR_COUNT_MISMATCH; }
    uint8_t *seen = (uint8_t *)calloc((size_t)(query_count > 0 ? query_count : 1) * top_k, 1);
    if (!seen) return ORC_ERR_ALLOC;
    for (int i = 0; i < n_pairs; ++i) {
        const orc_pair *p = &pairs[i];
        if (p->token >= (uint32_t)query_count) { free(seen); *out_error_value = p->token; return ORC_ERR_TOKEN_OUT_OF_RANGE; }
        if (p->rank >= (uint32_t)top_k) { free(seen); *out_error_value = p->rank; return ORC_ERR_RANK_OUT_OF_RANGE; }
        if (p->expert >= (uint32_t)num_experts) { free(seen); *out_error_value = p->expert; return ORC_ERR_EXPERT_OUT_OF_RANGE; }
        size_t key = (size_t)p->token * top_k + p->rank;
        if (seen[key]) { free(seen); *out_error_value = p->token; return ORC_ERR_DUPLICATE_TOKEN_RANK; }
        seen[key] = 1;
    }
    free(seen);
    memcpy(sorted, pairs, sizeof(orc_pair) * (size_t)n_pairs);
    g_sort_keys = sort_keys;
    qsort(sorted, (size_t)n_pairs, sizeof(orc_pair), pair_cmp);
    g_sort_keys = NULL;
    for (int e = 0; e < num_experts; ++e) { offsets[e] = 0xFFFFFFFFu; counts[e] = 0; }
    int ng = 0;
    int i = 0;
    while (i < n_pairs) {
        uint32_t e = sorted[i].expert;
        int start = i;
        while (i < n_pairs && sorted[i].expert == e) ++i;
        offsets[e] = (uint32_t)start;
        counts[e] = (uint32_t)(i - start);
        groups[ng].expert = e;
        groups[ng].pair_start = (uint32_t)start;
        groups[ng].pair_count = (uint32_t)(i - start);
        ++ng;
    }
    *n_groups = ng;
    int nt = 0, gs = 0;
    while (gs < ng) {
        int ge = gs + tile_expert_count < ng ? gs + tile_expert_count : ng;
        if (tile_break >= 0 && gs < tile_break && ge > tile_break) ge = tile_break;
        tiles[nt].group_start = (uint32_t)gs;
        tiles[nt].group_count = (uint32_t)(ge - gs);
        tiles[nt].pair_start = groups[gs].pair_start;
        tiles[nt].pair_count = groups[ge - 1].pair_start + groups[ge - 1].pair_count - groups[gs].pair_start;
        ++nt;
        gs = ge;
    }
    *n_tiles = nt;
    return ORC_OK;
}

/* PrefillRoutedGEMMBlock (PrefillGroupedRoutedMoE.swift:20-25). */
typedef struct { uint32_t local_slot, pair_start, row_count, local_row; } orc_block;

/* PrefillRoutedGEMMPlanner.plan (PrefillGroupedRoutedMoE.swift:42-83): cut
 * groups into batches of <= tile_rows-row blocks; a batch never splits a
 * group that fits an empty batch; an over-budget group is cut on whole
 * blocks.  Writes blocks in order and, per batch, its row count and its
 * [first block, block count).  Returns the number of batches. */
int orc_plan_routed_gemm(const orc_group *groups, int n_groups, int max_rows_per_batch,
                         int tile_rows, orc_block *blocks, int *n_blocks, int *batch_rows,
                         int *batch_first_block, int *batch_block_count) {
    int budget = (max_rows_per_batch / tile_rows) * tile_rows;
    if (budget < tile_rows) budget = tile_rows;
    int nb = 0, nbatch = 0, rows = 0, first = 0;
#define ORC_FLUSH()                                        \
    do {                                                   \
        if (rows > 0) {                                    \
            batch_rows[nbatch] = rows;                     \
            batch_first_block[nbatch] = first;             \
            batch_block_count[nbatch] = nb - first;        \
            ++nbatch;                                      \
            first = nb;                                    \
            rows = 0;                                      \
        }                                                  \
    } while (0)
    for (int slot = 0; slot < n_groups; ++slot) {
        int taken = 0, count = (int)groups[slot].pair_count;
        while (taken < count) {
            if (rows == budget) ORC_FLUSH();
            if (rows > 0 && rows + (count - taken) > budget) ORC_FLUSH();
            int take = count - taken < budget - rows ? count - taken : budget - rows;
            int done = 0;
            while (done < take) {
                int rc = take - done < tile_rows ? take - done : tile_rows;
                blocks[nb].local_slot = (uint32_t)slot;
                blocks[nb].pair_start = groups[slot].pair_start + (uint32_t)(taken + done);
                blocks[nb].row_count = (uint32_t)rc;
                blocks[nb].local_row = (uint32_t)(rows + done);
                ++nb;
                done += rc;
            }
            rows += take;
            taken += take;
        }
    }
    ORC_FLUSH();
#undef ORC_FLUSH
    *n_blocks = nb;
    return nbatch;
}

/* prefill_moe_reduce_token_major (Sources/Tsugumi/Metal/Prefill/prefill.metal:796-817):
 * h2[t,d] = sum over r ascending of fma(w[t,r], partial[(t*K+r)*D + d]). */
void orc_reduce_token_major(const float *partials, const float *w, int T, int K, int D,
                            float *h2) {
#pragma omp parallel for
    for (int t = 0; t < T; ++t)
        for (int d = 0; d < D; ++d) {
            double acc = 0.0;
            for (int r = 0; r < K; ++r)
                acc += (double)w[t * K + r] * (double)partials[((size_t)t * K + r) * D + d];
            h2[(size_t)t * D + d] = (float)acc;
        }
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
