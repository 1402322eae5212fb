/*
 * sllm_oracle.c -- TEST INFRASTRUCTURE ONLY: the CPU restatement of
 * saphira-llm's I2_S decode path that the CUDA backend is checked against.
 * See sllm_oracle.h for the rules this file follows. The product never links
 * it.
 *
 * Floating-point rules (the whole point of this file):
 *   - compiled with -ffp-contract=off, so a*b+c is two roundings unless
 *     fmaf() is written, exactly where the reference fuses;
 *   - the reference's x86-64-v3 SIMD reductions are restated lane by lane
 *     (RMSNorm 4 f64 lanes, softmax 8-wide blocks with an f64 pair sum,
 *     lm_head 4 x 8 f32 FMA accumulators and its reduction tree);
 *   - libm (expf, cosf, sinf, powf, roundf, sqrtf) is called where the
 *     reference calls it, with run-time arguments, so nothing is folded at
 *     compile time to a different value.
 */
#define _POSIX_C_SOURCE 200809L

#include "sllm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define QK 128

static int g_threads = 0;

void orc_set_threads(int n) {
    g_threads = n;
#ifdef _OPENMP
    if (n > 0) { omp_set_num_threads(n); }
#endif
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------ */
/* I2_S                                                                */
/* ------------------------------------------------------------------ */

/* src/i2s_gemm.c:45-83. amax has no floor; roundf is half-away-from-zero.
 * The reference converts with a plain (int) cast, which on x86-64 turns a
 * NaN or out-of-range product (an infinite input times scale 0, or any input
 * times a scale that overflowed to inf for a tiny amax) into INT_MIN, clamped
 * to -128; that case is spelled out here so it does not depend on the cast. */
void orc_i2s_quant_act(const float * x, size_t n, int8_t * q, orc_act * act) {
    float amax = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        const float a = fabsf(x[i]);
        if (a > amax) { amax = a; }
    }
    const float s = (amax > 0.0f) ? 127.0f / amax : 0.0f;
    int32_t sum = 0;
    for (size_t i = 0; i < n; ++i) {
        const float p = x[i] * s;
        int v = !(fabsf(p) < 2147483648.0f) ? -128 : (int) roundf(p);
        if (v > 127) { v = 127; }
        if (v < -128) { v = -128; }
        q[i] = (int8_t) v;
        sum += v;
    }
    act->scale = s;
    act->sum = sum;
}

/* src/i2s_gemm.c:89-112 (the scalar oracle): element 32*field + lane of each
 * 128-element block sits in byte `lane` at shift 6 - 2*field. */
int32_t orc_i2s_dot(const uint8_t * w, const int8_t * q, size_t n) {
    if (w == NULL || q == NULL || n < QK) { return 0; }   /* src/i2s_gemm.c:246-249 */
    int32_t acc = 0;
    for (size_t b = 0; b < n / QK; ++b) {
        const uint8_t * blk = w + b * 32;
        const int8_t * qb = q + b * QK;
        for (int lane = 0; lane < 32; ++lane) {
            for (int f = 0; f < 4; ++f) {
                const int code = (blk[lane] >> (6 - 2 * f)) & 3;
                acc += code * (int32_t) qb[32 * f + lane];
            }
        }
    }
    return acc;
}

/* src/i2s_gemm.c:260-269; rows are independent, so threading is exact. */
void orc_i2s_gemv(const uint8_t * w, size_t n_rows, size_t n,
                  const int8_t * q, int32_t * rows_out) {
    if (w == NULL || q == NULL || rows_out == NULL) { return; }
    const size_t rb = n / 4;
    #pragma omp parallel for schedule(static) if (n_rows >= 256)
    for (long r = 0; r < (long) n_rows; ++r) {
        rows_out[r] = orc_i2s_dot(w + (size_t) r * rb, q, n);
    }
}

/* src/i2s_gemm.c:271-290: one division per column, then subtract and multiply. */
float orc_i2s_epilogue(int32_t dot, int32_t act_sum, float act_scale, float w_scale) {
    const float post = w_scale / act_scale;
    return (float) (dot - act_sum) * post;
}

/* src/quant.c:102-106: the f32 scale sits right after the n/4 packed bytes. */
float orc_i2s_scale(const uint8_t * packed, size_t n_elements) {
    float s;
    memcpy(&s, packed + n_elements / 4, 4);
    return s;
}

/* src/quant.c:77-100: byte (k/128)*32 + k%32, field (k%128)/32 at 6-2*field. */
uint8_t orc_i2s_code(const uint8_t * packed, size_t k) {
    const uint8_t byte = packed[(k / QK) * 32 + (k % 32)];
    return (uint8_t) ((byte >> (6 - 2 * ((k % QK) / 32))) & 3);
}

/* src/i2s_convert.c:31-35 */
size_t orc_i2s_packed_size(size_t n_elements) { return n_elements / 4 + 32; }

/* Packing of ready-made codes into the interleaved layout of
 * src/i2s_convert.c:168-176 (tail zeroed, scale written at n/4). */
int orc_i2s_pack_codes(const uint8_t * codes, size_t n, float scale, uint8_t * dst) {
    if (dst == NULL || (codes == NULL && n > 0) || n % 4 != 0) { return 1; }
    memset(dst, 0, orc_i2s_packed_size(n));
    for (size_t i = 0; i < n; ++i) {
        dst[(i / QK) * 32 + (i % 32)] |= (uint8_t) ((codes[i] & 3) << (6 - 2 * ((i % QK) / 32)));
    }
    memcpy(dst + n / 4, &scale, 4);
    return 0;
}

/* src/i2s_convert.c:101-104 + 107-178 with SLLM_I2S_RULE_GGUF_PY: the code is
 * decided by a strict +-0.5 threshold on w * (1/scale) in double. */
int orc_i2s_quantize_scaled_py(const float * src, size_t n, float scale, uint8_t * dst) {
    if (dst == NULL || (src == NULL && n > 0)) { return 1; }
    if (n % 4 != 0) { return 2; }
    uint8_t * codes = (uint8_t *) malloc(n > 0 ? n : 1);
    if (codes == NULL) { return 1; }
    const double inv = 1.0 / (double) scale;
    for (size_t i = 0; i < n; ++i) {
        const double t = (double) src[i] * inv;
        codes[i] = (t > 0.5) ? 2 : (t < -0.5) ? 0 : 1;
    }
    const int rc = orc_i2s_pack_codes(codes, n, scale, dst);
    free(codes);
    return rc;
}

void orc_i2s_gemv_f32(const uint8_t * w, size_t n_rows, size_t n,
                      const float * x, float * y, int32_t * dots) {
    int8_t * q = (int8_t *) malloc(n);
    int32_t * d = dots ? dots : (int32_t *) malloc(n_rows * sizeof(int32_t));
    if (q == NULL || d == NULL) { free(q); if (!dots) { free(d); } return; }
    orc_act act;
    orc_i2s_quant_act(x, n, q, &act);
    orc_i2s_gemv(w, n_rows, n, q, d);
    const float post = orc_i2s_scale(w, n_rows * n) / act.scale;
    for (size_t r = 0; r < n_rows; ++r) { y[r] = (float) (d[r] - act.sum) * post; }
    free(q);
    if (!dots) { free(d); }
}

/* ------------------------------------------------------------------ */
/* f16                                                                 */
/* ------------------------------------------------------------------ */

/* src/quant.c:24-52: the exact conversion (the lm_head's F16C path
 * converts exactly too, src/ops.c:124-125). */
float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    if (e == 0x1fu) { return u2f(sign | 0x7f800000u | (m << 13)); }
    if (e != 0) { return u2f(sign | ((e + 112u) << 23) | (m << 13)); }
    /* zero or subnormal: m * 2^-24, exact in f32 */
    const float mag = (float) m * 0x1p-24f;
    return (h & 0x8000u) ? -mag : mag;
}

/* src/forward.c:239-263, the conversion the embedding lookup uses. It
 * normalises a subnormal with one less in the exponent than src/quant.c, so a
 * subnormal f16 comes out at HALF its value. Parity needs the same. */
float orc_fp16_to_fp32_embd(uint16_t h) {
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    if (e == 0 && m != 0) {
        const float mag = (float) m * 0x1p-25f;
        return (h & 0x8000u) ? -mag : mag;
    }
    return orc_fp16_to_fp32(h);
}

/* ------------------------------------------------------------------ */
/* RMSNorm, expf, softmax, SiLU, RoPE                                   */
/* ------------------------------------------------------------------ */

/* src/ops.c:254-322 in its x86 order: four f64 lanes; for each 8-block, lane
 * k adds the f32 square of element k, then of element k+4; the lanes are
 * summed 0..3; a tail (n % 8) adds f64 squares; then mean narrows to f32,
 * scale = 1/sqrtf(mean + eps), dst = (scale * x) * w. */
void orc_rms_norm(float * dst, const float * x, const float * w, size_t n, float eps) {
    double lane[4] = { 0.0, 0.0, 0.0, 0.0 };
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        for (int k = 0; k < 4; ++k) {
            const float s = x[i + k] * x[i + k];
            lane[k] = lane[k] + (double) s;
        }
        for (int k = 0; k < 4; ++k) {
            const float s = x[i + 4 + k] * x[i + 4 + k];
            lane[k] = lane[k] + (double) s;
        }
    }
    double ss = 0.0;
    for (int k = 0; k < 4; ++k) { ss += lane[k]; }
    for (; i < n; ++i) { ss += (double) x[i] * (double) x[i]; }
    const float mean = (float) (ss / (double) n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (size_t j = 0; j < n; ++j) { dst[j] = scale * x[j]; }
    if (w != NULL) {
        for (size_t j = 0; j < n; ++j) { dst[j] = dst[j] * w[j]; }
    }
}

/* One lane of ggml_v_expf as src/ops.c:342-379 computes it: a range
 * reduction by rounding x*log2(e) with the 1.5*2^23 shift, a two-part
 * ln2 correction, a degree-5 polynomial in FMAs and an exponent rebuild,
 * with the |n| > 126 and |n| > 192 special scalings. The vector form's
 * early return (no lane special) gives each lane the same value as the
 * general form, so one lane can be restated on its own. */
float orc_v_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = fmaf(x, 0x1.715476p+0f, r);
    const float nn = z - r;
    const float b = fmaf(-nn, 0x1.7f7d1cp-20f, fmaf(-nn, 0x1.62e4p-1f, x));
    const uint32_t e = f2u(z) << 23;
    const float k = u2f(e + f2u(1.0f));
    const int c = fabsf(nn) > 126.0f;
    const float u = b * b;
    const float j = fmaf(fmaf(fmaf(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u,
                              fmaf(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                         u, 0x1.ffffecp-1f * b);
    if (!c) { return fmaf(k, j, k); }
    const uint32_t g = (nn <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = u2f(g + 0x7f000000u);
    const float s2 = u2f(e - g);
    if (fabsf(nn) > 192.0f) { return s1 * s1; }
    return fmaf(s2, j, s2) * s1;
}

/* src/ops.c:386-422: 8-blocks take the polynomial exp and add
 * ((t0+t1)+t2)+t3 with t_k = (double)v_k + (double)v_{k+4}; the tail takes
 * libm expf; inv = (float)(1/sum) in double; every value is scaled by inv. */
void orc_softmax(float * x, size_t n) {
    if (n == 0) { return; }
    float mx = x[0];
    for (size_t i = 1; i < n; ++i) { if (x[i] > mx) { mx = x[i]; } }
    double sum = 0.0;
    size_t i = 0;
    for (; i + 7 < n; i += 8) {
        float v[8];
        for (int k = 0; k < 8; ++k) { v[k] = orc_v_expf(x[i + k] - mx); x[i + k] = v[k]; }
        double t[4];
        for (int k = 0; k < 4; ++k) { t[k] = (double) v[k] + (double) v[k + 4]; }
        sum += t[0] + t[1] + t[2] + t[3];
    }
    for (; i < n; ++i) {
        const float e = expf(x[i] - mx);
        x[i] = e;
        sum += (double) e;
    }
    const float inv = (float) (1.0 / sum);
    for (size_t j = 0; j < n; ++j) { x[j] *= inv; }
}

/* src/ops.c:428-461: v / (1 + expf_poly(0 - v)) in 8-blocks, libm tail. */
void orc_silu(float * x, size_t n) {
    size_t i = 0;
    for (; i + 7 < n; i += 8) {
        for (int k = 0; k < 8; ++k) {
            const float v = x[i + k];
            x[i + k] = v / (1.0f + orc_v_expf(0.0f - v));
        }
    }
    for (; i < n; ++i) { x[i] = x[i] / (1.0f + expf(-x[i])); }
}

/* src/ops.c:467-551, NEOX pairing (k, k + n_rot/2), freq_scale 1: the angle
 * starts at (float)pos and is multiplied by powf(theta, -2/n_rot) once per
 * pair, cos/sin are libm's, and the rotation is two products and a sum each. */
void orc_rope_neox(float * x, size_t n_rot, int32_t pos, float theta) {
    if (n_rot < 2) { return; }
    if (n_rot % 2 != 0) { n_rot -= 1; }
    const size_t half = n_rot / 2;
    const float theta_scale = powf(theta, -2.0f / (float) n_rot);
    float th = (float) pos;
    for (size_t k = 0; k < half; ++k) {
        const float f = 1.0f * th;
        const float c = cosf(f);
        const float s = sinf(f);
        th *= theta_scale;
        const float xa = x[k];
        const float xb = x[k + half];
        x[k] = xa * c - xb * s;
        x[k + half] = xa * s + xb * c;
    }
}

/* src/ops.c:106-154 in its x86 order: accumulator (j, l) takes, by FMA, every
 * element d with d % 32 == 8*j + l of the 32-aligned head, in order; then
 * acc0 += acc2, acc1 += acc3, acc0 += acc1 (per lane), t_l = acc0[l] +
 * acc0[l+4], head = (t0 + t1) + (t2 + t3); the tail adds products in order. */
float orc_dot_f16(const uint16_t * row, const float * x, size_t n) {
    if (row == NULL || x == NULL) { return 0.0f; }
    float acc[4][8];
    memset(acc, 0, sizeof acc);
    size_t d = 0;
    if (n >= 32) {
        const size_t np = n & ~(size_t) 31;
        for (; d < np; d += 32) {
            for (int j = 0; j < 4; ++j) {
                for (int l = 0; l < 8; ++l) {
                    const size_t e = d + (size_t) (8 * j + l);
                    acc[j][l] = fmaf(orc_fp16_to_fp32(row[e]), x[e], acc[j][l]);
                }
            }
        }
    }
    for (int l = 0; l < 8; ++l) { acc[0][l] = acc[0][l] + acc[2][l]; acc[1][l] = acc[1][l] + acc[3][l]; }
    for (int l = 0; l < 8; ++l) { acc[0][l] = acc[0][l] + acc[1][l]; }
    float t[4];
    for (int l = 0; l < 4; ++l) { t[l] = acc[0][l] + acc[0][l + 4]; }
    float r = (t[0] + t[1]) + (t[2] + t[3]);
    for (; d < n; ++d) { r += orc_fp16_to_fp32(row[d]) * x[d]; }
    return r;
}

/* src/forward.c:876-883: first index of the maximum (strict >). */
int32_t orc_argmax(const float * logits, int32_t n) {
    int32_t best = 0;
    float bv = logits[0];
    for (int32_t i = 1; i < n; ++i) { if (logits[i] > bv) { bv = logits[i]; best = i; } }
    return best;
}

/* ------------------------------------------------------------------ */
/* the decode chain                                                    */
/* ------------------------------------------------------------------ */

struct orc_ctx {
    int32_t n_ctx, n_past, n_layer, kv_dim, n_embd, n_ff, n_vocab;
    int     kv_f16;       /* this project's fp16-KV variant: cache values rounded to half */
    float * k_cache;      /* [layer][head_kv][pos][head_dim] (src/forward.c:81-83) */
    float * v_cache;
    float * last_logits;
    int     have_logits;
    /* one column of scratch */
    float * x, * xn, * ffn_inp, * q, * k, * v, * attn, * proj, * g, * u, * h, * scores;
    int8_t * qa;
    int32_t * dots;
};

int orc_ctx_new(const sllm_cuda_model_desc * m, int32_t n_ctx, orc_ctx ** out) {
    if (m == NULL || out == NULL || n_ctx <= 0) { return SLLM_CUDA_ERR_ARG; }
    *out = NULL;
    orc_ctx * c = (orc_ctx *) calloc(1, sizeof *c);
    if (c == NULL) { return SLLM_CUDA_ERR_NOMEM; }
    const int32_t hd = m->n_embd / m->n_head;
    c->n_ctx = n_ctx;
    c->n_layer = m->n_layer;
    c->kv_dim = hd * m->n_head_kv;
    c->n_embd = m->n_embd;
    c->n_ff = m->n_ff;
    c->n_vocab = m->n_vocab;
    const size_t kv = (size_t) m->n_layer * (size_t) c->kv_dim * (size_t) n_ctx;
    const size_t big = (size_t) (m->n_embd > m->n_ff ? m->n_embd : m->n_ff);
    c->k_cache = (float *) calloc(kv, sizeof(float));
    c->v_cache = (float *) calloc(kv, sizeof(float));
    c->last_logits = (float *) calloc((size_t) m->n_vocab, sizeof(float));
    const size_t E = (size_t) m->n_embd, F = (size_t) m->n_ff;
    c->x = (float *) malloc(E * 4); c->xn = (float *) malloc(E * 4);
    c->ffn_inp = (float *) malloc(E * 4); c->q = (float *) malloc(E * 4);
    c->k = (float *) malloc((size_t) c->kv_dim * 4); c->v = (float *) malloc((size_t) c->kv_dim * 4);
    c->attn = (float *) malloc(E * 4); c->proj = (float *) malloc(E * 4);
    c->g = (float *) malloc(F * 4); c->u = (float *) malloc(F * 4); c->h = (float *) malloc(F * 4);
    c->scores = (float *) malloc((size_t) n_ctx * 4);
    c->qa = (int8_t *) malloc(big);
    c->dots = (int32_t *) malloc(big * 4);
    if (!c->k_cache || !c->v_cache || !c->last_logits || !c->x || !c->xn || !c->ffn_inp ||
        !c->q || !c->k || !c->v || !c->attn || !c->proj || !c->g || !c->u || !c->h ||
        !c->scores || !c->qa || !c->dots) {
        orc_ctx_free(c);
        return SLLM_CUDA_ERR_NOMEM;
    }
    *out = c;
    return SLLM_CUDA_OK;
}

void orc_ctx_free(orc_ctx * c) {
    if (c == NULL) { return; }
    free(c->k_cache); free(c->v_cache); free(c->last_logits);
    free(c->x); free(c->xn); free(c->ffn_inp); free(c->q); free(c->k); free(c->v);
    free(c->attn); free(c->proj); free(c->g); free(c->u); free(c->h); free(c->scores);
    free(c->qa); free(c->dots);
    free(c);
}

/*
 * Not in the reference: the fp16 KV option of the CUDA backend, restated so
 * that it can be checked bit for bit. Every value stored into the cache is
 * rounded to the nearest IEEE half (ties to even) and widened back exactly;
 * everything else is the reference's order. float -> half by the standard
 * round-to-nearest-even rules (overflow to infinity from 65520 up, gradual
 * underflow to the half subnormals).
 */
static uint16_t orc_fp32_to_fp16_rne(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {     /* infinity or NaN */
        return (uint16_t) (sign | 0x7c00u | (ax > 0x7f800000u ? (0x200u | ((ax >> 13) & 0x3ffu)) : 0u));
    }
    if (ax >= 0x477ff000u) { return (uint16_t) (sign | 0x7c00u); }   /* >= 65520 */
    if (ax >= 0x38800000u) {     /* a normal half: rebias, keep 10 mantissa bits */
        const uint32_t v = ax - 0x38000000u;
        uint32_t h = v >> 13;
        const uint32_t rem = v & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) { h += 1u; }
        return (uint16_t) (sign | h);
    }
    const uint32_t e = ax >> 23;
    if (e < 102u) { return (uint16_t) sign; }          /* below 2^-25: zero */
    const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;                    /* 14 .. 24 */
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t mid = 1u << (shift - 1u);
    if (rem > mid || (rem == mid && (h & 1u))) { h += 1u; }
    return (uint16_t) (sign | h);
}

static float orc_kv_round(const orc_ctx * c, float v) {
    return c->kv_f16 ? orc_fp16_to_fp32(orc_fp32_to_fp16_rne(v)) : v;
}

void orc_ctx_set_kv_f16(orc_ctx * c, int on) { if (c != NULL) { c->kv_f16 = on ? 1 : 0; } }

uint16_t orc_fp32_to_fp16(float f) { return orc_fp32_to_fp16_rne(f); }

/* src/forward.c:530-562: clear the live prefix of every layer, rewind. */
void orc_ctx_reset(orc_ctx * c) {
    if (c == NULL) { return; }
    if (c->n_past > 0) {
        const size_t live = (size_t) c->n_layer * (size_t) c->kv_dim * (size_t) c->n_ctx;
        memset(c->k_cache, 0, live * sizeof(float));
        memset(c->v_cache, 0, live * sizeof(float));
    }
    c->n_past = 0;
    c->have_logits = 0;
}

int32_t orc_ctx_n_past(const orc_ctx * c) { return c ? c->n_past : 0; }

const float * orc_ctx_last_logits(const orc_ctx * c) {
    return (c != NULL && c->have_logits) ? c->last_logits : NULL;
}

/* One projection: quantise `src` (n wide), GEMV, epilogue -- the three steps
 * src/forward.c:650-655 runs for every I2_S tensor. */
static void project(orc_ctx * c, const uint8_t * w, size_t rows, size_t n,
                    const float * src, float * dst, const orc_act * have_act) {
    orc_act act;
    if (have_act == NULL) { orc_i2s_quant_act(src, n, c->qa, &act); }
    else { act = *have_act; }
    orc_i2s_gemv(w, rows, n, c->qa, c->dots);
    const float post = orc_i2s_scale(w, rows * n) / act.scale;
    for (size_t r = 0; r < rows; ++r) { dst[r] = (float) (c->dots[r] - act.sum) * post; }
}

/* One token at absolute position pos, every layer, logits out: the body of
 * src/forward.c:621-827 for one column. */
static void forward_one(const sllm_cuda_model_desc * m, orc_ctx * c,
                        int32_t token, int32_t pos, float * logits) {
    const size_t E = (size_t) m->n_embd, F = (size_t) m->n_ff, G = (size_t) c->kv_dim;
    const int32_t hd = m->n_embd / m->n_head;
    const int32_t grp = m->n_head / m->n_head_kv;
    const float attn_scale = 1.0f / sqrtf((float) hd);
    const size_t kv_layer = G * (size_t) c->n_ctx;

    for (size_t d = 0; d < E; ++d) {                       /* forward.c:621-626 */
        c->x[d] = orc_fp16_to_fp32_embd(m->tok_embd[(size_t) token * E + d]);
    }
    for (int32_t il = 0; il < m->n_layer; ++il) {
        const sllm_cuda_layer_desc * L = &m->layers[il];
        orc_act act;
        orc_rms_norm(c->xn, c->x, L->attn_norm, E, m->f_rms_eps);   /* :631-636 */
        orc_i2s_quant_act(c->xn, E, c->qa, &act);                    /* :650-666 */
        project(c, L->wq, E, E, NULL, c->q, &act);
        project(c, L->wk, G, E, NULL, c->k, &act);
        project(c, L->wv, G, E, NULL, c->v, &act);
        for (int32_t h = 0; h < m->n_head; ++h) {                    /* :668-681 */
            orc_rope_neox(c->q + (size_t) h * hd, (size_t) m->n_rot, pos, m->rope_freq_base);
        }
        for (int32_t h = 0; h < m->n_head_kv; ++h) {
            orc_rope_neox(c->k + (size_t) h * hd, (size_t) m->n_rot, pos, m->rope_freq_base);
        }
        float * kb = c->k_cache + (size_t) il * kv_layer;             /* :683-696 */
        float * vb = c->v_cache + (size_t) il * kv_layer;
        for (int32_t h = 0; h < m->n_head_kv; ++h) {
            float * kd = kb + ((size_t) h * c->n_ctx + pos) * hd;
            float * vd = vb + ((size_t) h * c->n_ctx + pos) * hd;
            for (int32_t d = 0; d < hd; ++d) {
                kd[d] = orc_kv_round(c, c->k[(size_t) h * hd + d]);
                vd[d] = orc_kv_round(c, c->v[(size_t) h * hd + d]);
            }
        }
        const int32_t npast = pos + 1;                                /* :698-726 */
        for (int32_t h = 0; h < m->n_head; ++h) {
            const int32_t kvh = h / grp;
            const float * qh = c->q + (size_t) h * hd;
            const float * kc = kb + (size_t) kvh * c->n_ctx * hd;
            const float * vc = vb + (size_t) kvh * c->n_ctx * hd;
            for (int32_t s = 0; s < npast; ++s) {
                float acc = 0.0f;
                for (int32_t d = 0; d < hd; ++d) { acc += qh[d] * kc[(size_t) s * hd + d]; }
                c->scores[s] = acc * attn_scale;
            }
            orc_softmax(c->scores, (size_t) npast);
            float * oh = c->attn + (size_t) h * hd;
            for (int32_t d = 0; d < hd; ++d) { oh[d] = 0.0f; }
            for (int32_t s = 0; s < npast; ++s) {
                const float wgt = c->scores[s];
                for (int32_t d = 0; d < hd; ++d) { oh[d] += wgt * vc[(size_t) s * hd + d]; }
            }
        }
        orc_rms_norm(c->xn, c->attn, L->attn_sub_norm, E, m->f_rms_eps);  /* :728-742 */
        project(c, L->wo, E, E, c->xn, c->proj, NULL);
        for (size_t d = 0; d < E; ++d) { c->ffn_inp[d] = c->proj[d] + c->x[d]; }  /* :744-750 */
        orc_rms_norm(c->xn, c->ffn_inp, L->ffn_norm, E, m->f_rms_eps);   /* :756-779 */
        orc_i2s_quant_act(c->xn, E, c->qa, &act);
        project(c, L->ffn_gate, F, E, NULL, c->g, &act);
        project(c, L->ffn_up, F, E, NULL, c->u, &act);
        orc_silu(c->g, F);
        for (size_t r = 0; r < F; ++r) { c->h[r] = c->g[r] * c->u[r]; }
        orc_rms_norm(c->h, c->h, L->ffn_sub_norm, F, m->f_rms_eps);      /* :781-793 */
        project(c, L->ffn_down, E, F, c->h, c->proj, NULL);
        for (size_t d = 0; d < E; ++d) { c->x[d] = c->proj[d] + c->ffn_inp[d]; }  /* :795-801 */
    }
    orc_rms_norm(c->xn, c->x, m->output_norm, E, m->f_rms_eps);          /* :804-809 */
    #pragma omp parallel for schedule(static)
    for (long v = 0; v < (long) m->n_vocab; ++v) {                        /* :818-827 */
        logits[v] = orc_dot_f16(m->tok_embd + (size_t) v * E, c->xn, E);
    }
}

/* src/forward.c:589-609 argument rules, then one column at a time. */
int orc_forward_chunk(const sllm_cuda_model_desc * m, orc_ctx * c,
                      const int32_t * tokens, int32_t n, int32_t base,
                      float * logits_out) {
    if (m == NULL || c == NULL || tokens == NULL || logits_out == NULL) { return SLLM_CUDA_ERR_ARG; }
    if (n < 1 || n > 256) { return SLLM_CUDA_ERR_ARG; }
    if (base < c->n_past || base + n > c->n_ctx) { return SLLM_CUDA_ERR_ARG; }
    for (int32_t t = 0; t < n; ++t) {
        if (tokens[t] < 0 || tokens[t] >= m->n_vocab) { return SLLM_CUDA_ERR_ARG; }
    }
    c->n_past = base + n;
    for (int32_t t = 0; t < n; ++t) {
        forward_one(m, c, tokens[t], base + t, logits_out + (size_t) t * m->n_vocab);
    }
    memcpy(c->last_logits, logits_out + (size_t) (n - 1) * m->n_vocab, (size_t) m->n_vocab * 4);
    c->have_logits = 1;
    return SLLM_CUDA_OK;
}

/* src/forward.c:885-938, including the BOS fallback and the continuation
 * from the last logits when there is no prompt. */
int orc_generate_greedy(const sllm_cuda_model_desc * m, orc_ctx * c,
                        const int32_t * prompt, int32_t n_prompt,
                        int32_t n_new, int32_t * out) {
    if (m == NULL || c == NULL || out == NULL || n_prompt < 0 || n_new < 0) { return SLLM_CUDA_ERR_ARG; }
    if (n_prompt + n_new + c->n_past > c->n_ctx) { return SLLM_CUDA_ERR_TOO_LARGE; }
    float * logits = (float *) malloc((size_t) m->n_vocab * 4);
    if (logits == NULL) { return SLLM_CUDA_ERR_NOMEM; }
    const int32_t base = c->n_past;
    int32_t next = 128000;
    int rc = SLLM_CUDA_OK;
    if (n_prompt == 0 && base > 0) {
        next = orc_argmax(c->last_logits, m->n_vocab);
        for (int32_t i = 0; i < n_new; ++i) {
            out[i] = next;
            rc = orc_forward_chunk(m, c, &next, 1, base + i, logits);
            if (rc != SLLM_CUDA_OK) { free(logits); return rc; }
            next = orc_argmax(logits, m->n_vocab);
        }
        free(logits);
        return SLLM_CUDA_OK;
    }
    for (int32_t i = 0; i < n_prompt; ++i) {
        rc = orc_forward_chunk(m, c, &prompt[i], 1, base + i, logits);
        if (rc != SLLM_CUDA_OK) { free(logits); return rc; }
    }
    if (n_prompt > 0) { next = orc_argmax(logits, m->n_vocab); }
    for (int32_t i = 0; i < n_new; ++i) {
        out[i] = next;
        rc = orc_forward_chunk(m, c, &next, 1, base + n_prompt + i, logits);
        if (rc != SLLM_CUDA_OK) { free(logits); return rc; }
        next = orc_argmax(logits, m->n_vocab);
    }
    free(logits);
    return SLLM_CUDA_OK;
}

void orc_layer_chain(const sllm_cuda_model_desc * m, int32_t layer,
                     float * x, float * scratch) {
    const size_t E = (size_t) m->n_embd, F = (size_t) m->n_ff;
    const size_t G = (size_t) (m->n_embd / m->n_head) * (size_t) m->n_head_kv;
    const sllm_cuda_layer_desc * L = &m->layers[layer];
    float * xn = scratch, * q = xn + E, * k = q + E, * v = k + G, * proj = v + G;
    float * fi = proj + E, * g = fi + E, * u = g + F, * h = u + F;
    int8_t * qa = (int8_t *) malloc(F > E ? F : E);
    int32_t * dots = (int32_t *) malloc((F > E ? F : E) * 4);
    if (qa == NULL || dots == NULL) { free(qa); free(dots); return; }
    orc_act act;
    #define PROJ(W, ROWS, N, DST) do { \
        orc_i2s_gemv((W), (ROWS), (N), qa, dots); \
        const float post_ = orc_i2s_scale((W), (ROWS) * (N)) / act.scale; \
        for (size_t r_ = 0; r_ < (ROWS); ++r_) { (DST)[r_] = (float) (dots[r_] - act.sum) * post_; } \
    } while (0)
    orc_rms_norm(xn, x, L->attn_norm, E, m->f_rms_eps);
    orc_i2s_quant_act(xn, E, qa, &act);
    PROJ(L->wq, E, E, q);
    PROJ(L->wk, G, E, k);
    PROJ(L->wv, G, E, v);
    orc_rms_norm(xn, q, L->attn_sub_norm, E, m->f_rms_eps);
    orc_i2s_quant_act(xn, E, qa, &act);
    PROJ(L->wo, E, E, proj);
    for (size_t d = 0; d < E; ++d) { fi[d] = proj[d] + x[d]; }
    orc_rms_norm(xn, fi, L->ffn_norm, E, m->f_rms_eps);
    orc_i2s_quant_act(xn, E, qa, &act);
    PROJ(L->ffn_gate, F, E, g);
    PROJ(L->ffn_up, F, E, u);
    orc_silu(g, F);
    for (size_t r = 0; r < F; ++r) { h[r] = g[r] * u[r]; }
    orc_rms_norm(h, h, L->ffn_sub_norm, F, m->f_rms_eps);
    orc_i2s_quant_act(h, F, qa, &act);
    PROJ(L->ffn_down, E, F, proj);
    for (size_t d = 0; d < E; ++d) { x[d] = proj[d] + fi[d]; }
    #undef PROJ
    free(qa);
    free(dots);
}
