/*
 * qf_oracle.c -- CPU restatement of the QwenFieldfare MoE-block hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see qf_oracle.h): the checker for libqf_moe.so,
 * never linked into it.  Every function names the reference lines it follows
 * (paths inside tanishqpatil/qwen-fieldfare).  Compile with -ffp-contract=off.
 */
#include "qf_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* 16-bit floats                                                       */
/* ------------------------------------------------------------------ */
float qfo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int sh = -1;
            do {
                m <<= 1;
                sh++;
            } while (!(m & 0x400u));
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(112 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t qfo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (ax < 0x38800000u) { /* below 2^-14: fp16 subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign;
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t sh = 126u - e;
        uint32_t q = m >> sh;
        uint32_t rem = m & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t r = ax - 0x38000000u;
    r += 0xFFFu + ((r >> 13) & 1u);
    if (r >= 0x0F800000u) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | (r >> 13));
}

float qfo_bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t qfo_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

/* Threads used by the row loops when the block runs fewer tokens than threads
 * (the row loops then parallelise instead of the token loop). */
static int g_inner_threads = 1;

static inline float cvt16(uint16_t h, int bf16) {
    return bf16 ? qfo_bf16_to_f32(h) : qfo_f16_to_f32(h);
}
static inline uint16_t round16(float f, int bf16) {
    return bf16 ? qfo_f32_to_bf16(f) : qfo_f32_to_f16(f);
}

/* ------------------------------------------------------------------ */
/* Seeded synthetic data: SplitMix64 streams keyed by (seed, layer,    */
/* tensor tag, index).  Normal draws are Irwin-Hall(12) so that every  */
/* step is exact integer or single IEEE fp32 operations (the CUDA      */
/* generator in the product reproduces the same bytes).                */
/* ------------------------------------------------------------------ */
#define QF_GAMMA 0x9E3779B97F4A7C15ull
enum {
    TAG_GATE_W = 1,
    TAG_GATE_S = 2,
    TAG_UP_W = 3,
    TAG_UP_S = 4,
    TAG_DOWN_W = 5,
    TAG_DOWN_S = 6,
    TAG_ROUTER_W = 7,
    TAG_ROUTER_S = 8,
    TAG_COEF_W = 9,
    TAG_COEF_S = 10,
    TAG_HIDDEN = 11
};

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t qfo_stream_key(uint64_t seed, uint32_t layer, uint32_t tag, uint32_t index) {
    uint64_t k = mix64(seed + QF_GAMMA);
    k = mix64(k ^ (((uint64_t)layer + 1ull) * QF_GAMMA));
    k = mix64(k ^ (((uint64_t)tag << 32) | (uint64_t)index));
    return k;
}

uint64_t qfo_draw(uint64_t key, uint64_t i) { return mix64(key + (i + 1ull) * QF_GAMMA); }

/* Irwin-Hall(12) standard-normal stand-in from draws 3g..3g+2 (exact in fp32) */
static float irwin_hall(uint64_t key, uint64_t g) {
    int32_t s = 0;
    for (int d = 0; d < 3; d++) {
        uint64_t r = qfo_draw(key, 3ull * g + (uint64_t)d);
        for (int j = 0; j < 4; j++) s += (int32_t)((r >> (16 * j)) & 0xFFFFu);
    }
    return (float)(s - 393210) * (1.0f / 65536.0f);
}

/* scale ~ |N(0,0.01)| + 1e-3, as separately rounded fp32 ops, times `mult` */
static float synth_scale(uint64_t key, uint64_t g, float mult) {
    float z = irwin_hall(key, g);
    float a = fabsf(z);
    float m = a * 0.01f;
    float v = m + 0.001f;
    return v * mult;
}

static void synth_codes(uint64_t key, uint8_t *dst, size_t nbytes) {
    for (size_t j = 0; j < nbytes; j += 8) {
        uint64_t r = qfo_draw(key, j >> 3);
        for (size_t b = 0; b < 8 && j + b < nbytes; b++) dst[j + b] = (uint8_t)(r >> (8 * b));
    }
}

static void synth_scales(uint64_t key, uint16_t *s, uint16_t *b, size_t ngroups, float mult,
                         float bias_mult, int bf16) {
    for (size_t g = 0; g < ngroups; g++) {
        uint16_t sb = round16(synth_scale(key, g, mult), bf16);
        s[g] = sb;
        b[g] = round16(bias_mult * cvt16(sb, bf16), bf16);
    }
}

void qfo_synth_expert_record(uint64_t seed, uint32_t layer, uint32_t expert, int scale_bf16,
                             uint8_t *rec) {
    static const uint32_t wtag[3] = {TAG_GATE_W, TAG_UP_W, TAG_DOWN_W};
    static const uint32_t stag[3] = {TAG_GATE_S, TAG_UP_S, TAG_DOWN_S};
    static const uint32_t woff[3] = {QFO_OFF_GATE_W, QFO_OFF_UP_W, QFO_OFF_DOWN_W};
    static const uint32_t soff[3] = {QFO_OFF_GATE_S, QFO_OFF_UP_S, QFO_OFF_DOWN_S};
    static const uint32_t boff[3] = {QFO_OFF_GATE_B, QFO_OFF_UP_B, QFO_OFF_DOWN_B};
    for (int p = 0; p < 3; p++) {
        synth_codes(qfo_stream_key(seed, layer, wtag[p], expert), rec + woff[p], 524288);
        synth_scales(qfo_stream_key(seed, layer, stag[p], expert), (uint16_t *)(rec + soff[p]),
                     (uint16_t *)(rec + boff[p]), 16384, 1.0f, -8.0f, scale_bf16);
    }
}

void qfo_synth_router(uint64_t seed, uint32_t layer, int scale_bf16, uint8_t *w, uint16_t *s,
                      uint16_t *b) {
    synth_codes(qfo_stream_key(seed, layer, TAG_ROUTER_W, 0), w, 256u * 2048u);
    synth_scales(qfo_stream_key(seed, layer, TAG_ROUTER_S, 0), s, b, 256u * 32u, 0.0625f,
                 -128.0f, scale_bf16);
}

void qfo_synth_coef(uint64_t seed, uint32_t layer, int scale_bf16, uint8_t *w, uint16_t *s,
                    uint16_t *b) {
    synth_codes(qfo_stream_key(seed, layer, TAG_COEF_W, 0), w, 2048u);
    synth_scales(qfo_stream_key(seed, layer, TAG_COEF_S, 0), s, b, 32u, 0.0625f, -128.0f,
                 scale_bf16);
}

void qfo_synth_hidden(uint64_t seed, uint64_t tok0, int T, uint16_t *x) {
    float z[QFO_HIDDEN];
    for (int t = 0; t < T; t++) {
        uint64_t key = qfo_stream_key(seed, 0, TAG_HIDDEN, (uint32_t)(tok0 + (uint64_t)t));
        double ss = 0.0;
        for (int i = 0; i < QFO_HIDDEN; i++) {
            z[i] = irwin_hall(key, (uint64_t)i);
            ss += (double)z[i] * (double)z[i];
        }
        double inv = 1.0 / sqrt(ss / QFO_HIDDEN + 1e-6);
        for (int i = 0; i < QFO_HIDDEN; i++)
            x[(size_t)t * QFO_HIDDEN + i] = qfo_f32_to_f16((float)((double)z[i] * inv));
    }
}

/* ------------------------------------------------------------------ */
/* Reference-order matvec primitives                                   */
/* ------------------------------------------------------------------ */

/* simd_sum over 32 lanes as an xor butterfly (16, 8, 4, 2, 1) */
static float butterfly32(float *v) {
    float t[32];
    for (int m = 16; m >= 1; m >>= 1) {
        for (int l = 0; l < 32; l++) t[l] = v[l] + v[l ^ m];
        memcpy(v, t, sizeof(t));
    }
    return v[0];
}

/* deltanet.metal:1838-1895 qwen_q4_row_simd_f32 (factored: fma(s,dot), fma(b,sum)) */
float qfo_q4_row(const uint8_t *w_row, const uint16_t *s_row, const uint16_t *b_row,
                 const float *vec, int cols, int bf16) {
    float lane_acc[32];
    const int groups = cols / 64;
    const int full_blocks = groups / 4;
    for (int lane = 0; lane < 32; lane++) {
        float acc = 0.0f;
        for (int blk = 0; blk < full_blocks; blk++) {
            const int byte_base = blk * 128 + lane * 4;
            const uint32_t w4 = (uint32_t)w_row[byte_base] | ((uint32_t)w_row[byte_base + 1] << 8) |
                                ((uint32_t)w_row[byte_base + 2] << 16) |
                                ((uint32_t)w_row[byte_base + 3] << 24);
            const int g = blk * 4 + (lane >> 3);
            const float scale = cvt16(s_row[g], bf16);
            const float bias = cvt16(b_row[g], bf16);
            const int elem = byte_base * 2;
            const float *e = vec + elem;
            float dot = 0.0f;
            for (int j = 0; j < 4; j++) {
                const uint32_t byte = (w4 >> (8 * j)) & 0xFFu;
                dot = fmaf((float)(byte & 0x0Fu), e[2 * j], dot);
                dot = fmaf((float)(byte >> 4), e[2 * j + 1], dot);
            }
            float sum = e[0];
            for (int j = 1; j < 8; j++) sum = sum + e[j];
            acc = fmaf(scale, dot, acc);
            acc = fmaf(bias, sum, acc);
        }
        for (int g = full_blocks * 4; g < groups; g++) {
            const uint8_t packed = w_row[g * 32 + lane];
            const float x0 = vec[g * 64 + lane * 2];
            const float x1 = vec[g * 64 + lane * 2 + 1];
            const float dot = fmaf((float)(packed & 0x0Fu), x0, (float)(packed >> 4) * x1);
            acc = fmaf(cvt16(s_row[g], bf16), dot, acc);
            acc = fmaf(cvt16(b_row[g], bf16), x0 + x1, acc);
        }
        lane_acc[lane] = acc;
    }
    return butterfly32(lane_acc);
}

/* deltanet.metal:2229-2260 qwen_q8_row_simd_f32 (cols fixed at 2048) */
float qfo_q8_row(const uint8_t *w_row, const uint16_t *s_row, const uint16_t *b_row,
                 const float *vec, int bf16) {
    float lane_acc[32];
    for (int lane = 0; lane < 32; lane++) {
        float acc = 0.0f;
        for (int blk = 0; blk < 8; blk++) {
            const int byte_base = blk * 256 + lane * 8;
            const int g = blk * 4 + (lane >> 3);
            const float scale = cvt16(s_row[g], bf16);
            const float bias = cvt16(b_row[g], bf16);
            float dot = 0.0f;
            float sum = 0.0f;
            for (int i = 0; i < 8; i++) {
                const float x = vec[byte_base + i];
                dot = fmaf((float)w_row[byte_base + i], x, dot);
                sum = sum + x;
            }
            acc = fmaf(scale, dot, acc);
            acc = fmaf(bias, sum, acc);
        }
        lane_acc[lane] = acc;
    }
    return butterfly32(lane_acc);
}

/* deltanet.metal:1897-1919 qwen_gemv_q4_affine_simd_f32: one 32-lane row per
 * SIMD group, rows independent (the LM head at cols = 2048) */
void qfo_lm_head(const uint8_t *w, const uint16_t *s, const uint16_t *b, int rows, const float *x,
                 int scale_bf16, float *out) {
#ifdef _OPENMP
#pragma omp parallel for if (!omp_in_parallel()) schedule(static)
#endif
    for (int r = 0; r < rows; r++)
        out[r] = qfo_q4_row(w + (size_t)r * 1024, s + (size_t)r * 32, b + (size_t)r * 32, x, 2048, scale_bf16);
}

/* deltanet.metal:18-53 qwen_rmsnorm_f32 dispatched with 64 threads: thread i
 * sums v*v over i, i+64, ... (fma chain); simd_sum per 32-lane group (xor
 * butterfly); the two partials add (simd_sum of [p0, p1, 0, ...]); rsqrt
 * restated as a correctly rounded 1/sqrt; out = (in * inv) * w, to fp16 */
void qfo_post_norm_to_f16(const float *in, const float *w, int T, float eps, uint16_t *x_out) {
    for (int t = 0; t < T; t++) {
        const float *v = in + (size_t)t * 2048;
        float lanes[64];
        for (int i = 0; i < 64; i++) {
            float acc = 0.0f;
            for (int j = i; j < 2048; j += 64) acc = fmaf(v[j], v[j], acc);
            lanes[i] = acc;
        }
        const float p0 = butterfly32(lanes), p1 = butterfly32(lanes + 32);
        const float s = p0 + p1;
        const float inv = 1.0f / sqrtf(s / 2048.0f + eps);
        for (int i = 0; i < 2048; i++) x_out[(size_t)t * 2048 + i] = qfo_f32_to_f16((v[i] * inv) * w[i]);
    }
}

/* deltanet.metal:2262-2281 qwen_router_q8_logits_simd_f32 */
void qfo_router_logits(const qfo_layer *L, const float *x, float *logits) {
#ifdef _OPENMP
#pragma omp parallel for if (!omp_in_parallel() && g_inner_threads > 1) num_threads(g_inner_threads) schedule(static)
#endif
    for (int r = 0; r < QFO_EXPERTS; r++)
        logits[r] = qfo_q8_row(L->router_w + (size_t)r * 2048, L->router_s + (size_t)r * 32,
                               L->router_b + (size_t)r * 32, x, L->scale_bf16);
}

/* deltanet.metal:2283-2329 qwen_router_top8_logits_f32 (k generalised; bias is the
 * harness-only logit bias added before selection) */
void qfo_topk(const float *logits, const float *bias, int n, int k, int32_t *idx, float *w) {
    float vals[1024];
    int32_t top_idx[64];
    float top_val[64];
    for (int i = 0; i < n; i++) vals[i] = bias ? logits[i] + bias[i] : logits[i];
    for (int j = 0; j < k; j++) {
        top_idx[j] = 0;
        top_val[j] = -INFINITY;
    }
    for (int i = 0; i < n; i++) {
        const float value = vals[i];
        if (value > top_val[k - 1]) {
            top_val[k - 1] = value;
            top_idx[k - 1] = i;
            for (int j = k - 2; j >= 0; --j) {
                if (top_val[j + 1] <= top_val[j]) break;
                float sv = top_val[j];
                top_val[j] = top_val[j + 1];
                top_val[j + 1] = sv;
                int32_t si = top_idx[j];
                top_idx[j] = top_idx[j + 1];
                top_idx[j + 1] = si;
            }
        }
    }
    const float max_value = top_val[0];
    float den = 0.0f;
    for (int i = 0; i < n; i++) den += expf(vals[i] - max_value);
    float top_sum = 0.0f;
    float prob[64];
    for (int j = 0; j < k; j++) {
        prob[j] = expf(top_val[j] - max_value) / den;
        top_sum += prob[j];
    }
    for (int j = 0; j < k; j++) {
        idx[j] = top_idx[j];
        w[j] = prob[j] / top_sum;
    }
}

/* deltanet.metal:863-902 qwen_gemv_q8_affine with rows=1 (thread-per-row naive form;
 * the Metal fast-math build contracts q*scale+bias and acc+=w*v, restated as fmaf) */
float qfo_coef(const qfo_layer *L, const float *x) {
    float acc = 0.0f;
    for (int g = 0; g < 32; g++) {
        const float scale = cvt16(L->coef_s[g], L->scale_bf16);
        const float bias = cvt16(L->coef_b[g], L->scale_bf16);
        for (int i = 0; i < 64; i++) {
            const float wq = fmaf((float)L->coef_w[g * 64 + i], scale, bias);
            acc = fmaf(wq, x[g * 64 + i], acc);
        }
    }
    return acc;
}

static inline float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }


/* deltanet.metal:1985-2048 + :2050-2076 / :2155-2179: act = SiLU(G x) * (U x) */
void qfo_gate_up(const uint8_t *rec, int bf16, const float *x, float *act) {
    const uint8_t *gw = rec + QFO_OFF_GATE_W;
    const uint16_t *gs = (const uint16_t *)(rec + QFO_OFF_GATE_S);
    const uint16_t *gb = (const uint16_t *)(rec + QFO_OFF_GATE_B);
    const uint8_t *uw = rec + QFO_OFF_UP_W;
    const uint16_t *us = (const uint16_t *)(rec + QFO_OFF_UP_S);
    const uint16_t *ub = (const uint16_t *)(rec + QFO_OFF_UP_B);
#ifdef _OPENMP
#pragma omp parallel for if (!omp_in_parallel() && g_inner_threads > 1) num_threads(g_inner_threads) schedule(static)
#endif
    for (int r = 0; r < QFO_INTER; r++) {
        const float g = qfo_q4_row(gw + (size_t)r * 1024, gs + r * 32, gb + r * 32, x, 2048, bf16);
        const float u = qfo_q4_row(uw + (size_t)r * 1024, us + r * 32, ub + r * 32, x, 2048, bf16);
        act[r] = silu_mul(g, u);
    }
}

/* deltanet.metal:2099-2122 / :2181-2211 row dots of the down projection (K = 512) */
void qfo_down(const uint8_t *rec, int bf16, const float *act, float *y) {
    const uint8_t *dw = rec + QFO_OFF_DOWN_W;
    const uint16_t *ds = (const uint16_t *)(rec + QFO_OFF_DOWN_S);
    const uint16_t *db = (const uint16_t *)(rec + QFO_OFF_DOWN_B);
#ifdef _OPENMP
#pragma omp parallel for if (!omp_in_parallel() && g_inner_threads > 1) num_threads(g_inner_threads) schedule(static)
#endif
    for (int r = 0; r < QFO_HIDDEN; r++)
        y[r] = qfo_q4_row(dw + (size_t)r * 256, ds + r * 8, db + r * 8, act, 512, bf16);
}

/* One token through the block, in the production streaming order
 * (QwenQ4ActiveExpertStreamingRunner.swift:1169-1381). */
/* qwen_combine_cached_moe_subsets_f32 (deltanet.metal:2213-2227) with the
 * shared down's gate (:2118-2120): out = (residual + sigmoid(c) * y_sh) +
 * sum_k w_k y_k, the routed products summed in router order. */
void qfo_combine(const float *y, const float *w, const float *sh_y, float c, const float *res,
                 float *out) {
    const float coeff = 1.0f / (1.0f + expf(-c));
    for (int r = 0; r < QFO_HIDDEN; r++) {
        const float shared = sh_y[r] * coeff;
        float routed = y[r] * w[0];
        for (int k = 1; k < QFO_TOPK; k++) routed = routed + y[(size_t)k * QFO_HIDDEN + r] * w[k];
        const float base = res ? res[r] : 0.0f;
        out[r] = (base + shared) + routed;
    }
}

static void block_token(const qfo_layer *L, const uint16_t *x16, const float *res,
                        const float *bias, const int32_t *idx_in, const float *w_in, float *out,
                        int32_t *idx_out, float *w_out, float *logits_out, float *coef_out) {
    float x[QFO_HIDDEN];
    float logits[QFO_EXPERTS];
    int32_t idx[QFO_TOPK];
    float w[QFO_TOPK];
    float sh_act[QFO_INTER], act[QFO_TOPK][QFO_INTER];
    float sh_y[QFO_HIDDEN], y[QFO_TOPK][QFO_HIDDEN];
    for (int i = 0; i < QFO_HIDDEN; i++) x[i] = qfo_f16_to_f32(x16[i]);
    if (idx_in) {
        memcpy(idx, idx_in, sizeof(idx));
        memcpy(w, w_in, sizeof(w));
        if (logits_out) {
            qfo_router_logits(L, x, logits);
            memcpy(logits_out, logits, sizeof(logits));
        }
    } else {
        qfo_router_logits(L, x, logits);
        qfo_topk(logits, bias, QFO_EXPERTS, QFO_TOPK, idx, w);
        if (logits_out) memcpy(logits_out, logits, sizeof(logits));
    }
    const float c = qfo_coef(L, x);
    qfo_gate_up(L->shared_record, L->scale_bf16, x, sh_act);
    qfo_down(L->shared_record, L->scale_bf16, sh_act, sh_y);
    for (int k = 0; k < QFO_TOPK; k++) {
        const uint8_t *rec = L->expert_records[idx[k]];
        qfo_gate_up(rec, L->scale_bf16, x, act[k]);
        qfo_down(rec, L->scale_bf16, act[k], y[k]);
    }
    qfo_combine(&y[0][0], w, sh_y, c, res, out);
    if (idx_out) memcpy(idx_out, idx, sizeof(idx));
    if (w_out) memcpy(w_out, w, sizeof(w));
    if (coef_out) *coef_out = c;
}

void qfo_block(const qfo_layer *L, int T, const uint16_t *x, const float *residual,
               const float *bias, const int32_t *idx_in, const float *w_in, float *out,
               int32_t *idx_out, float *w_out, float *logits_out, float *coef_out, int threads) {
#ifdef _OPENMP
    int nt = threads > 0 ? threads : omp_get_max_threads();
    int outer = T < nt ? T : nt;
    g_inner_threads = T < nt ? nt : 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(outer)
#endif
    for (int t = 0; t < T; t++) {
        const size_t o = (size_t)t * QFO_HIDDEN;
        block_token(L, x + o, residual ? residual + o : NULL, bias,
                    idx_in ? idx_in + (size_t)t * QFO_TOPK : NULL,
                    w_in ? w_in + (size_t)t * QFO_TOPK : NULL, out + o,
                    idx_out ? idx_out + (size_t)t * QFO_TOPK : NULL,
                    w_out ? w_out + (size_t)t * QFO_TOPK : NULL,
                    logits_out ? logits_out + (size_t)t * QFO_EXPERTS : NULL,
                    coef_out ? coef_out + t : NULL);
    }
    (void)threads;
}

/* RMSNorm of the stack transition (deltanet.metal:18-53 qwen_rmsnorm_f32, unit
 * weight): the reference sums v*v with an fma chain per thread and simd_sum,
 * whose order Metal leaves open; the order fixed here (and used by the CUDA
 * kernels) is 128 tiles of 16 consecutive elements, an fma chain inside each
 * tile, tiles summed in order.  inv = 1/sqrt(mean + eps) is the correctly
 * rounded form of the reference's rsqrt; out = fp16(in * inv). */
void qfo_rmsnorm_to_f16(const float *in, int T, float eps, uint16_t *x_out) {
    for (int t = 0; t < T; t++) {
        const float *v = in + (size_t)t * QFO_HIDDEN;
        float total = 0.0f;
        for (int c = 0; c < QFO_HIDDEN / 16; c++) {
            float acc = 0.0f;
            for (int j = 0; j < 16; j++) acc = fmaf(v[c * 16 + j], v[c * 16 + j], acc);
            total = total + acc;
        }
        const float mean_sq = total / (float)QFO_HIDDEN;
        const float inv = 1.0f / sqrtf(mean_sq + eps);
        for (int i = 0; i < QFO_HIDDEN; i++)
            x_out[(size_t)t * QFO_HIDDEN + i] = qfo_f32_to_f16(v[i] * inv);
    }
}

/* Stable counting sort of the (token, k) pairs by expert: the dispatch plan the
 * build adds in front of the grouped expert GEMM (no reference counterpart). */
void qfo_dispatch_plan(const int32_t *idx, int T, int k, int E, int32_t *counts,
                       int32_t *offsets, int32_t *perm) {
    memset(counts, 0, sizeof(int32_t) * (size_t)E);
    const int n = T * k;
    for (int i = 0; i < n; i++) counts[idx[i]]++;
    offsets[0] = 0;
    for (int e = 0; e < E; e++) offsets[e + 1] = offsets[e] + counts[e];
    int32_t *cursor = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
    memcpy(cursor, offsets, sizeof(int32_t) * (size_t)E);
    for (int i = 0; i < n; i++) perm[cursor[idx[i]]++] = i;
    free(cursor);
}

/* ------------------------------------------------------------------ */
/* Expert-slot cache: Q4BoundedExpertCache.swift (exact port)          */
/* ------------------------------------------------------------------ */
static const int kLayerWeights[40] = {86, 82, 78, 72, 64, 58, 54, 48, 35, 42, 58, 59, 45, 48,
                                      38, 43, 45, 41, 42, 38, 34, 37, 53, 55, 43, 45, 38, 41,
                                      46, 41, 43, 40, 48, 54, 55, 42, 45, 47, 51, 66};

struct qfo_cache {
    int capacity, prob_capacity, prot_capacity, layer_count;
    int key_layers, key_experts;
    int *range_start, *range_count;
    int32_t *key_to_slot; /* [key_layers*key_experts] */
    int32_t *slot_key;    /* [capacity] */
    uint64_t *access_time;
    uint8_t *prob, *prot;
    uint8_t *prefetched; /* per key */
    uint64_t *lock_gen;
    uint64_t gen;
    uint64_t tick;
    int64_t total_requests, hits, misses, evictions, bytes_fetched, prefetches, useful, wasted;
};

qfo_cache *qfo_cache_create(int capacity, double ratio, int requested_layers, int key_layers,
                            int key_experts) {
    qfo_cache *c = (qfo_cache *)calloc(1, sizeof(qfo_cache));
    c->capacity = capacity;
    c->key_layers = key_layers;
    c->key_experts = key_experts;
    int req = requested_layers < 1 ? 1 : requested_layers;
    c->layer_count = capacity >= req * 8 ? req : 1;
    c->range_start = (int *)calloc((size_t)c->layer_count, sizeof(int));
    c->range_count = (int *)calloc((size_t)c->layer_count, sizeof(int));
    if (c->layer_count == 40) {
        const int base = 8;
        const int remaining = capacity - 40 * base;
        int excess[40], counts[40], order[40];
        int64_t total = 0;
        for (int i = 0; i < 40; i++) {
            excess[i] = kLayerWeights[i] - base;
            total += excess[i];
        }
        int sum = 0;
        for (int i = 0; i < 40; i++) {
            counts[i] = base + (int)(((int64_t)remaining * excess[i]) / total);
            sum += counts[i];
            order[i] = i;
        }
        /* remainder order: descending (remaining*excess) % total; Swift's sort is not
         * stable, ties are broken here by lower layer index */
        for (int i = 1; i < 40; i++) {
            int v = order[i], j = i - 1;
            int64_t rv = ((int64_t)remaining * excess[v]) % total;
            while (j >= 0 && (((int64_t)remaining * excess[order[j]]) % total) < rv) {
                order[j + 1] = order[j];
                j--;
            }
            order[j + 1] = v;
        }
        int left = capacity - sum, ri = 0;
        while (left > 0) {
            counts[order[ri]]++;
            left--;
            ri++;
        }
        int start = 0;
        for (int i = 0; i < 40; i++) {
            c->range_start[i] = start;
            c->range_count[i] = counts[i];
            start += counts[i];
        }
    } else if (c->layer_count > 1) {
        int start = 0;
        for (int l = 0; l < c->layer_count; l++) {
            int cnt = capacity / c->layer_count + (l < capacity % c->layer_count ? 1 : 0);
            c->range_start[l] = start;
            c->range_count[l] = cnt;
            start += cnt;
        }
    } else {
        c->range_start[0] = 0;
        c->range_count[0] = capacity;
    }
    int pc = (int)((double)capacity * ratio);
    c->prob_capacity = pc > 16 ? pc : 16;
    c->prot_capacity = capacity - c->prob_capacity;
    size_t nk = (size_t)key_layers * (size_t)key_experts;
    c->key_to_slot = (int32_t *)malloc(nk * sizeof(int32_t));
    c->prefetched = (uint8_t *)calloc(nk, 1);
    c->slot_key = (int32_t *)malloc((size_t)capacity * sizeof(int32_t));
    c->access_time = (uint64_t *)calloc((size_t)capacity, sizeof(uint64_t));
    c->prob = (uint8_t *)calloc((size_t)capacity, 1);
    c->prot = (uint8_t *)calloc((size_t)capacity, 1);
    c->lock_gen = (uint64_t *)calloc((size_t)capacity, sizeof(uint64_t));
    qfo_cache_clear(c);
    return c;
}

void qfo_cache_destroy(qfo_cache *c) {
    if (!c) return;
    free(c->range_start);
    free(c->range_count);
    free(c->key_to_slot);
    free(c->prefetched);
    free(c->slot_key);
    free(c->access_time);
    free(c->prob);
    free(c->prot);
    free(c->lock_gen);
    free(c);
}

void qfo_cache_clear(qfo_cache *c) {
    size_t nk = (size_t)c->key_layers * (size_t)c->key_experts;
    for (size_t i = 0; i < nk; i++) c->key_to_slot[i] = -1;
    memset(c->prefetched, 0, nk);
    for (int s = 0; s < c->capacity; s++) c->slot_key[s] = -1;
    memset(c->access_time, 0, sizeof(uint64_t) * (size_t)c->capacity);
    memset(c->prob, 0, (size_t)c->capacity);
    memset(c->prot, 0, (size_t)c->capacity);
    c->tick = 0;
}

void qfo_cache_reset_metrics(qfo_cache *c) {
    c->total_requests = c->hits = c->misses = c->evictions = 0;
    c->bytes_fetched = c->prefetches = c->useful = c->wasted = 0;
}

static void layer_range(const qfo_cache *c, int layer, int *lo, int *hi) {
    int l = layer < 0 ? 0 : (layer > c->layer_count - 1 ? c->layer_count - 1 : layer);
    *lo = c->range_start[l];
    *hi = c->range_start[l] + c->range_count[l];
}

int qfo_cache_acquire(qfo_cache *c, int layer, const uint32_t *experts, int n, uint32_t *slots,
                      uint32_t *miss_pos, int *n_miss, uint32_t *fetch_expert,
                      uint32_t *fetch_slot, int *n_fetch) {
    int lo, hi;
    layer_range(c, layer, &lo, &hi);
    const int cnt = hi - lo;
    int lpc = (int)((double)cnt * (double)c->prot_capacity / (double)c->capacity);
    if (lpc < 8) lpc = 8;
    c->tick++;
    const uint64_t tick = c->tick;
    c->gen++;
    const uint64_t gen = c->gen;
    const int n8 = n < 8 ? n : 8;
    uint32_t missing[8];
    int nfetch = 0;
    for (int p = 0; p < n8; p++) {
        const uint32_t e = experts[p];
        const int32_t key = layer * c->key_experts + (int32_t)e;
        c->total_requests++;
        if (c->prefetched[key]) {
            c->useful++;
            c->prefetched[key] = 0;
        }
        int32_t slot = c->key_to_slot[key];
        if (slot >= 0) {
            c->hits++;
            c->access_time[slot] = tick;
            c->lock_gen[slot] = gen;
            slots[p] = (uint32_t)slot;
            if (c->prob[slot]) {
                c->prob[slot] = 0;
                c->prot[slot] = 1;
                int prot_in_layer = 0;
                for (int s = lo; s < hi; s++) prot_in_layer += c->prot[s];
                if (prot_in_layer > lpc) {
                    uint64_t min_t = UINT64_MAX;
                    int cand = -1;
                    for (int s = lo; s < hi; s++) {
                        if (c->prot[s] && c->lock_gen[s] != gen) {
                            if (c->access_time[s] < min_t) {
                                min_t = c->access_time[s];
                                cand = s;
                            }
                        }
                    }
                    if (cand != -1) {
                        c->prot[cand] = 0;
                        c->prob[cand] = 1;
                    }
                }
            }
        } else {
            c->misses++;
            int victim = -1;
            for (int s = lo; s < hi; s++)
                if (c->slot_key[s] < 0 && c->lock_gen[s] != gen) {
                    victim = s;
                    break;
                }
            if (victim == -1) {
                uint64_t min_t = UINT64_MAX;
                for (int s = lo; s < hi; s++)
                    if (c->prob[s] && c->lock_gen[s] != gen && c->access_time[s] < min_t) {
                        min_t = c->access_time[s];
                        victim = s;
                    }
            }
            if (victim == -1) {
                uint64_t min_t = UINT64_MAX;
                for (int s = lo; s < hi; s++)
                    if (c->prot[s] && c->lock_gen[s] != gen && c->access_time[s] < min_t) {
                        min_t = c->access_time[s];
                        victim = s;
                    }
            }
            if (victim == -1) {
                for (int s = lo; s < hi; s++)
                    if (c->lock_gen[s] != gen) {
                        victim = s;
                        break;
                    }
            }
            if (victim == -1) victim = 0;
            const int32_t old = c->slot_key[victim];
            if (old >= 0) {
                if (c->prefetched[old]) {
                    c->wasted++;
                    c->prefetched[old] = 0;
                }
                c->key_to_slot[old] = -1;
                c->prob[victim] = 0;
                c->prot[victim] = 0;
                c->evictions++;
            }
            if (fetch_expert) fetch_expert[nfetch] = e;
            if (fetch_slot) fetch_slot[nfetch] = (uint32_t)victim;
            missing[nfetch] = e;
            nfetch++;
            c->bytes_fetched += (int64_t)QFO_RECORD_BYTES;
            c->key_to_slot[key] = victim;
            c->slot_key[victim] = key;
            c->access_time[victim] = tick;
            c->prob[victim] = 1;
            c->lock_gen[victim] = gen;
            slots[p] = (uint32_t)victim;
        }
    }
    /* acquireSlotsParallel: positions whose expert is in the set of missing experts */
    int nm = 0;
    for (int p = 0; p < n8; p++) {
        int is_miss = 0;
        for (int j = 0; j < nfetch; j++)
            if (missing[j] == experts[p]) is_miss = 1;
        if (is_miss) miss_pos[nm++] = (uint32_t)p;
    }
    *n_miss = nm;
    if (n_fetch) *n_fetch = nfetch;
    return n8;
}

void qfo_cache_prefetch(qfo_cache *c, int layer, const uint32_t *cands, int n) {
    int lo, hi;
    layer_range(c, layer, &lo, &hi);
    int any_free = 0;
    for (int s = lo; s < hi; s++)
        if (c->slot_key[s] < 0) any_free = 1;
    if (!any_free) return;
    const uint64_t tick = c->tick;
    for (int i = 0; i < n; i++) {
        const int32_t key = layer * c->key_experts + (int32_t)cands[i];
        if (c->key_to_slot[key] >= 0) continue;
        int free_slot = -1;
        for (int s = lo; s < hi; s++)
            if (c->slot_key[s] < 0) {
                free_slot = s;
                break;
            }
        if (free_slot == -1) break;
        c->bytes_fetched += (int64_t)QFO_RECORD_BYTES;
        c->key_to_slot[key] = free_slot;
        c->slot_key[free_slot] = key;
        c->access_time[free_slot] = tick;
        c->prob[free_slot] = 1;
        c->prefetched[key] = 1;
        c->prefetches++;
    }
}

void qfo_cache_metrics(const qfo_cache *c, int64_t out[11]) {
    int64_t occ = 0, pr = 0, pt = 0;
    for (int s = 0; s < c->capacity; s++) {
        occ += c->slot_key[s] >= 0;
        pr += c->prob[s];
        pt += c->prot[s];
    }
    out[0] = c->capacity;
    out[1] = occ;
    out[2] = pr;
    out[3] = pt;
    out[4] = c->hits;
    out[5] = c->misses;
    out[6] = c->evictions;
    out[7] = c->bytes_fetched;
    out[8] = c->prefetches;
    out[9] = c->useful;
    out[10] = c->wasted;
}

int qfo_cache_layer_count(const qfo_cache *c) { return c->layer_count; }
int qfo_cache_probationary_capacity(const qfo_cache *c) { return c->prob_capacity; }
void qfo_cache_layer_capacities(const qfo_cache *c, int32_t *out) {
    for (int l = 0; l < c->layer_count; l++) out[l] = c->range_count[l];
}

/* Sources/QwenFieldfareBench/main.swift:400-482 simulateSegmentedLRU */
int64_t qfo_slru_replay(const uint16_t *trace, int64_t n, int capacity) {
    const int prot_cap = (capacity * 3) / 4 > 8 ? (capacity * 3) / 4 : 8;
    int32_t key_to_slot[65536];
    for (int i = 0; i < 65536; i++) key_to_slot[i] = -1;
    int32_t *slot_key = (int32_t *)malloc(sizeof(int32_t) * (size_t)capacity);
    int64_t *atime = (int64_t *)calloc((size_t)capacity, sizeof(int64_t));
    uint8_t *prob = (uint8_t *)calloc((size_t)capacity, 1);
    uint8_t *prot = (uint8_t *)calloc((size_t)capacity, 1);
    int64_t *lock = (int64_t *)calloc((size_t)capacity, sizeof(int64_t));
    for (int s = 0; s < capacity; s++) slot_key[s] = -1;
    int64_t tick = 0, misses = 0;
    int prot_count = 0;
    for (int64_t g0 = 0; g0 < n; g0 += 8) {
        tick++;
        const int64_t g1 = g0 + 8 < n ? g0 + 8 : n;
        for (int64_t i = g0; i < g1; i++) {
            const uint16_t e = trace[i];
            int32_t slot = key_to_slot[e];
            if (slot >= 0) {
                atime[slot] = tick;
                lock[slot] = tick;
                if (prob[slot]) {
                    prob[slot] = 0;
                    prot[slot] = 1;
                    prot_count++;
                    if (prot_count > prot_cap) {
                        int cand = -1;
                        int64_t oldest = INT64_MAX;
                        for (int s = 0; s < capacity; s++)
                            if (prot[s] && lock[s] != tick && atime[s] < oldest) {
                                oldest = atime[s];
                                cand = s;
                            }
                        if (cand >= 0) {
                            prot[cand] = 0;
                            prot_count--;
                            prob[cand] = 1;
                        }
                    }
                }
                continue;
            }
            misses++;
            int victim = -1;
            for (int s = 0; s < capacity; s++)
                if (slot_key[s] < 0 && lock[s] != tick) {
                    victim = s;
                    break;
                }
            if (victim < 0) {
                int64_t oldest = INT64_MAX;
                for (int s = 0; s < capacity; s++)
                    if (prob[s] && lock[s] != tick && atime[s] < oldest) {
                        oldest = atime[s];
                        victim = s;
                    }
            }
            if (victim < 0) {
                int64_t oldest = INT64_MAX;
                for (int s = 0; s < capacity; s++)
                    if (prot[s] && lock[s] != tick && atime[s] < oldest) {
                        oldest = atime[s];
                        victim = s;
                    }
            }
            if (victim < 0) {
                victim = 0;
                for (int s = 0; s < capacity; s++)
                    if (lock[s] != tick) {
                        victim = s;
                        break;
                    }
            }
            if (slot_key[victim] >= 0) {
                key_to_slot[slot_key[victim]] = -1;
                prob[victim] = 0;
                if (prot[victim]) prot_count--;
                prot[victim] = 0;
            }
            key_to_slot[e] = victim;
            slot_key[victim] = e;
            atime[victim] = tick;
            prob[victim] = 1;
            lock[victim] = tick;
        }
    }
    free(slot_key);
    free(atime);
    free(prob);
    free(prot);
    free(lock);
    return misses;
}
