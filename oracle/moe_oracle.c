/*
 * CPU oracle for the quantized MoE-layer forward of moe-lab.
 *
 * TEST INFRASTRUCTURE ONLY. This file is a plain-C restatement of the reference's algorithm for the hot
 * path; it is the checker for the CUDA kernels in moelab_b200/csrc and the CPU baseline ("port") timed by
 * bench.py. Nothing in the product path links or calls it.
 *
 * Reference citations are paths inside Tigerly1/moe-lab:
 *   moelab/problem.py            contract, fp64 reference           (:3-10, :67-85)
 *   moelab/torch_backend.py      fp32 reference on dequant weights  (:57-67)
 *   moelab/router.py             fused router tail semantics        (:1-12, :15-66, :71-80)
 *   moelab/e2e.py                router family rules                (:56-63, :136-140, :171-176)
 *   moelab/variants/mlx/metal_q4_moe.py        int4 affine g64 state (:32-39)
 *   moelab/variants/mlx/metal_mxfp4_moe.py     MXFP4 state + decode  (:1-12, :33-41, :448-455)
 *   moelab/variants/mlx/metal_mxfp4_gptoss.py  gpt-oss epilogue      (:35-43, :110-126)
 *
 * The quantizers restate the published algorithms of mlx==0.32.4 (`mx.quantize(w, 64, 4)` affine and
 * `mode="mxfp4"`, OCP MX v1.0), which are third-party code absent from the reference tree; no reference test
 * pins their output values, so quantizer parity with MLX is unpinned. They are the definition the GPU
 * quantizer must reproduce bit for bit.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off so every fmaf below is the only fused operation).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- bf16 helpers */
static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) { /* round to nearest even, NaN kept quiet */
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

uint16_t orc_f32_to_bf16(float f) { return f32_to_bf16(f); }

/* ---------------------------------------------------------------- int4 affine, group 64
 * mx.quantize(w, group_size=64, bits=4) as called at metal_q4_moe.py:35 / gather_qmm_q4.py:13:
 * per group of 64 inputs, the extreme of larger magnitude ("edge") is made exactly representable,
 * scale = (max - min) / 15 (sign chosen so codes are >= 0), q = clamp(rint((w - bias) / scale), 0, 15).
 * Packed layout (metal_q4_decode_v4.py:57-63): uint32 [rows][K/8], element 8j+i at bits 4i of word j.
 * Scales and biases are stored as bf16 [rows][K/64]. */
void orc_q4_quantize(const uint16_t *w, int64_t rows, int64_t K, uint32_t *qw, uint16_t *scales, uint16_t *biases) {
    const int gs = 64;
    const float n_bins = 15.0f, eps = 1e-7f;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t g = 0; g < K / gs; ++g) {
            const uint16_t *src = w + r * K + g * gs;
            float wmax = -INFINITY, wmin = INFINITY;
            for (int i = 0; i < gs; ++i) {
                float v = bf16_to_f32(src[i]);
                wmax = v > wmax ? v : wmax;
                wmin = v < wmin ? v : wmin;
            }
            int mask = fabsf(wmin) > fabsf(wmax);
            float scale = (wmax - wmin) / n_bins;
            scale = scale > eps ? scale : eps;
            scale = mask ? scale : -scale;
            float edge = mask ? wmin : wmax;
            float q0 = rintf(edge / scale);
            float bias = 0.0f;
            if (q0 != 0.0f) {
                scale = edge / q0;
                bias = edge;
            }
            uint32_t *dst = qw + r * (K / 8) + g * (gs / 8);
            for (int j = 0; j < gs / 8; ++j) dst[j] = 0;
            for (int i = 0; i < gs; ++i) {
                float q = rintf((bf16_to_f32(src[i]) - bias) / scale);
                q = q < 0.0f ? 0.0f : (q > n_bins ? n_bins : q);
                dst[i / 8] |= ((uint32_t)q & 0xfu) << (4 * (i % 8));
            }
            scales[r * (K / gs) + g] = f32_to_bf16(scale);
            biases[r * (K / gs) + g] = f32_to_bf16(bias);
        }
    }
}

/* mx.dequantize as the fp32 value the kernels multiply: w = fmaf(scale, q, bias) with bf16 scale/bias
 * (metal_q4_moe.py:38-39). */
void orc_q4_dequant(const uint32_t *qw, const uint16_t *scales, const uint16_t *biases, int64_t rows, int64_t K,
                    float *out) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < K; ++k) {
            uint32_t q = (qw[r * (K / 8) + k / 8] >> (4 * (k % 8))) & 0xfu;
            float s = bf16_to_f32(scales[r * (K / 64) + k / 64]);
            float b = bf16_to_f32(biases[r * (K / 64) + k / 64]);
            out[r * K + k] = fmaf(s, (float)q, b);
        }
}

/* ---------------------------------------------------------------- MXFP4 (e2m1 values, e8m0 scale per 32)
 * mx.quantize(w, mode="mxfp4") (metal_mxfp4_moe.py:448-455), restated after OCP MX v1.0: shared exponent
 * floor(log2(amax)) - 2 (emax of e2m1), elements v / 2^exp rounded to the nearest e2m1 value (ties to
 * even mantissa), saturating at +-6. Code bits: sign 3, exponent 1-2, mantissa 0 (metal_mxfp4_moe.py:33-37).
 * Packed like int4: uint32 [rows][K/8] (element 8j+i at bits 4i), scales uint8 [rows][K/32]. */
static const float E2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

static uint32_t e2m1_round(float v) {
    uint32_t sign = v < 0.0f || (v == 0.0f && signbit(v)) ? 8u : 0u;
    float a = fabsf(v);
    uint32_t c;
    if (!(a == a)) c = 7; /* NaN: saturate (never produced by finite weights) */
    else if (a <= 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7;
    return sign | c;
}

void orc_mxfp4_quantize(const uint16_t *w, int64_t rows, int64_t K, uint32_t *qw, uint8_t *scales) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t g = 0; g < K / 32; ++g) {
            const uint16_t *src = w + r * K + g * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) {
                float a = fabsf(bf16_to_f32(src[i]));
                amax = a > amax ? a : amax;
            }
            int e;
            if (amax == 0.0f) e = -127;
            else {
                int ex;
                frexpf(amax, &ex); /* amax = m * 2^ex, m in [0.5, 1) -> floor(log2 amax) = ex - 1 */
                e = ex - 1 - 2;
            }
            if (e < -127) e = -127;
            if (e > 127) e = 127;
            uint8_t byte = (uint8_t)(e + 127);
            float inv = ldexpf(1.0f, -e);
            uint32_t *dst = qw + r * (K / 8) + g * 4;
            for (int j = 0; j < 4; ++j) dst[j] = 0;
            for (int i = 0; i < 32; ++i) {
                uint32_t c = e2m1_round(bf16_to_f32(src[i]) * inv);
                dst[i / 8] |= c << (4 * (i % 8));
            }
            scales[r * (K / 32) + g] = byte;
        }
}

/* value = e2m1(code) * 2^(byte - 127), exact in fp32 for every byte 0..254 (metal_mxfp4_moe.py:38-41). */
void orc_mxfp4_dequant(const uint32_t *qw, const uint8_t *scales, int64_t rows, int64_t K, float *out) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < K; ++k) {
            uint32_t c = (qw[r * (K / 8) + k / 8] >> (4 * (k % 8))) & 0xfu;
            float v = E2M1[c & 7u];
            if (c & 8u) v = -v;
            out[r * K + k] = ldexpf(v, (int)scales[r * (K / 32) + k / 32] - 127);
        }
}

/* ---------------------------------------------------------------- router
 * logits[t][e] = x[t] . Wg[e] (+ bias[e]) in fp32, in the fixed order the CUDA router uses: lane l of a
 * 32-lane group accumulates the 8-element chunks c = l, l+32, ... in increasing order with fmaf, then the
 * 32 partials are combined by a xor butterfly (offsets 16, 8, 4, 2, 1). Reproducing that order makes the
 * GPU logits - and so the top-k ids - bit-exact. The gate is a bf16 Linear (e2e.py:56, :171). */
void orc_router_logits(const uint16_t *x, const uint16_t *wg, const uint16_t *bias, int64_t T, int64_t E,
                       int64_t d, float *logits) {
    const int64_t nch = d / 8;
    for (int64_t t = 0; t < T; ++t)
        for (int64_t e = 0; e < E; ++e) {
            float p[32], q[32];
            for (int l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (int64_t c = l; c < nch; c += 32)
                    for (int j = 0; j < 8; ++j)
                        acc = fmaf(bf16_to_f32(x[t * d + c * 8 + j]), bf16_to_f32(wg[e * d + c * 8 + j]), acc);
                p[l] = acc;
            }
            for (int off = 16; off >= 1; off >>= 1) {
                for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ off];
                memcpy(p, q, sizeof p);
            }
            float v = p[0];
            if (bias) v = v + bf16_to_f32(bias[e]);
            logits[t * E + e] = v;
        }
}

/* Top-k with router.py semantics (:15-66): NaN counts as -inf, the largest value wins and ties go to the
 * lowest expert id; with fewer than k values above -inf the remaining slots take the lowest unused ids with
 * weight 0. norm=1: softmax over the k selected logits (Qwen3 norm_topk_prob, gpt-oss softmax over top-k,
 * e2e.py:58-63, :171-176). norm=0: full-softmax probabilities of the selected experts (DeepSeek-V2 greedy,
 * e2e.py:136-140). Weights are multiplied by `scale` (routed_scaling_factor). */
void orc_topk(const float *logits, int64_t T, int64_t E, int k, int norm, float scale, int32_t *idx, float *wts) {
    float *v = (float *)malloc(sizeof(float) * E);
    float topv[64];
    int32_t topi[64];
    for (int64_t t = 0; t < T; ++t) {
        float m0 = -INFINITY;
        for (int64_t e = 0; e < E; ++e) {
            float l = logits[t * E + e];
            v[e] = (l != l) ? -INFINITY : l;
            m0 = v[e] > m0 ? v[e] : m0;
        }
        double den = 0.0;
        if (!norm)
            for (int64_t e = 0; e < E; ++e) den += v[e] == -INFINITY ? 0.0 : exp((double)v[e] - (double)m0);
        for (int r = 0; r < k; ++r) {
            float b = -INFINITY;
            int64_t bi = -1;
            for (int64_t e = 0; e < E; ++e)
                if (v[e] > b) { b = v[e]; bi = e; }
            if (bi < 0) { /* no value above -inf left: lowest unused id, weight 0 */
                int32_t sel = 0;
                for (int used = 1; used;) {
                    used = 0;
                    for (int q = 0; q < r; ++q) used |= topi[q] == sel;
                    if (used) ++sel;
                }
                topi[r] = sel;
                topv[r] = -INFINITY;
            } else {
                topi[r] = (int32_t)bi;
                topv[r] = b;
                v[bi] = -INFINITY;
            }
        }
        double s = 0.0;
        double off = norm ? (double)topv[0] : (double)m0;
        if (norm) for (int r = 0; r < k; ++r) s += exp((double)topv[r] - off);
        else s = den;
        for (int r = 0; r < k; ++r) {
            idx[t * k + r] = topi[r];
            wts[t * k + r] = (float)(exp((double)topv[r] - off) / s) * scale;
        }
    }
    free(v);
}

/* ---------------------------------------------------------------- MoE forward on dequantized weights
 * y[t] = sum_j wts[t,j] * (Wd_e act(Wg_e x_t + bg_e, Wu_e x_t + bu_e) + bd_e), e = idx[t,j]
 * (problem.py:3-10, :67-85; torch_backend.py:57-67; gpt-oss biases and clamp: metal_mxfp4_gptoss.py:110-126).
 * Accumulates in double (the fp64 truth of problem.reference). act: 0 SiLU-GLU, 1 tanh-GELU GLU (Gemma-4,
 * metal_q4_decode_v4.py:36-40), 2 gpt-oss clamped SwiGLU (alpha 1.702, limit 7, up + 1).
 * Weights are fp32 [E][f][d] (gate, up) and [E][d][f] (down); x fp32 [T][d]; optional biases fp32
 * (NULL = none). Out-of-range ids contribute nothing. h_round: round h to bf16 like the kernels do. */
static double act_fn(int act, double g, double u) {
    if (act == 1) return 0.5 * g * (1.0 + tanh(0.7978845608028654 * (g + 0.044715 * g * g * g))) * u;
    if (act == 2) {
        g = g < 7.0 ? g : 7.0;
        u = u < -7.0 ? -7.0 : (u > 7.0 ? 7.0 : u);
        return g / (1.0 + exp(-1.702 * g)) * (u + 1.0);
    }
    return g / (1.0 + exp(-g)) * u;
}

void orc_moe_forward(const float *x, const float *wg, const float *wu, const float *wd, const float *bg,
                     const float *bu, const float *bd, const int32_t *idx, const float *wts, int64_t T, int64_t d,
                     int64_t f, int64_t E, int k, int act, int h_round, float *y) {
    double *h = (double *)malloc(sizeof(double) * f);
    double *acc = (double *)malloc(sizeof(double) * d);
    for (int64_t t = 0; t < T; ++t) {
        for (int64_t i = 0; i < d; ++i) acc[i] = 0.0;
        for (int j = 0; j < k; ++j) {
            int32_t e = idx[t * k + j];
            if (e < 0 || e >= E) continue;
            const float *xr = x + t * d;
            for (int64_t r = 0; r < f; ++r) {
                const float *gr = wg + ((int64_t)e * f + r) * d, *ur = wu + ((int64_t)e * f + r) * d;
                double g = 0.0, u = 0.0;
                for (int64_t c = 0; c < d; ++c) {
                    g += (double)gr[c] * xr[c];
                    u += (double)ur[c] * xr[c];
                }
                if (bg) g += bg[(int64_t)e * f + r];
                if (bu) u += bu[(int64_t)e * f + r];
                double hv = act_fn(act, g, u);
                if (h_round) hv = bf16_to_f32(f32_to_bf16((float)hv));
                h[r] = hv;
            }
            double w = wts[t * k + j];
            for (int64_t r = 0; r < d; ++r) {
                const float *dr = wd + ((int64_t)e * d + r) * f;
                double o = 0.0;
                for (int64_t c = 0; c < f; ++c) o += (double)dr[c] * h[c];
                if (bd) o += bd[(int64_t)e * d + r];
                acc[r] += w * o;
            }
        }
        for (int64_t i = 0; i < d; ++i) y[t * d + i] = (float)acc[i];
    }
    free(h);
    free(acc);
}
