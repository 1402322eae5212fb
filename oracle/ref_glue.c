/*
 * ref_glue.c -- TEST INFRASTRUCTURE ONLY. A thin C layer that drives the
 * reference saphira-llm library, compiled from its own unmodified sources
 * into oracle/_ref/libsllm_ref.so by oracle/Makefile, through its public API.
 * Tests use it to pin the restatement in sllm_oracle.c; bench.py uses it as
 * the timed CPU baseline. Nothing here computes anything itself: every
 * arithmetic step is a call into the reference.
 */
#define _POSIX_C_SOURCE 200809L

#include <saphira_llm/forward.h>
#include <saphira_llm/gguf.h>
#include <saphira_llm/i2s_gemm.h>
#include <saphira_llm/isa.h>
#include <saphira_llm/ops.h>
#include <saphira_llm/quant.h>
#include <saphira_llm/thread.h>

#include "../include/sllm_cuda.h"

#include <stdlib.h>
#include <string.h>

typedef struct refg_model {
    sllm_gguf   g;
    sllm_model * m;
    sllm_ctx   * c;
    sllm_pool  * pool;
} refg_model;

/* A pool of n threads (1 = the caller only), sllm_pool_create (thread.h:75). */
void * refg_pool_create(int n_threads) {
    sllm_pool_config cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.n_threads = n_threads;
    return sllm_pool_create(&cfg);
}

void refg_pool_destroy(void * pool) { sllm_pool_destroy((sllm_pool *) pool); }

int refg_pool_threads(void * pool) { return sllm_pool_threads((const sllm_pool *) pool); }

/* The ISA the reference's ternary kernel selected (isa.h ladder). */
int refg_select_auto(void) {
    sllm_i2s_select_auto();
    return (int) sllm_i2s_dot_isa();
}

/* Open a GGUF image held in memory (it must outlive the handle), load the
 * model, make a context of n_ctx positions and a pool of n_threads. */
int refg_model_open(const void * data, size_t size, int32_t n_ctx, int n_threads,
                    void ** out, char * err, size_t err_len) {
    refg_model * h = (refg_model *) calloc(1, sizeof *h);
    if (h == NULL) { return SLLM_ERR_NOMEM; }
    sllm_status st = sllm_gguf_open_memory(data, size, &h->g, err, err_len);
    if (st != SLLM_OK) { free(h); return st; }
    st = sllm_model_load(&h->g, &h->m);
    if (st != SLLM_OK) { sllm_gguf_close(&h->g); free(h); return st; }
    st = sllm_ctx_new(h->m, n_ctx, &h->c);
    if (st != SLLM_OK) { sllm_model_free(h->m); sllm_gguf_close(&h->g); free(h); return st; }
    h->pool = (sllm_pool *) refg_pool_create(n_threads);
    sllm_ctx_set_pool(h->c, h->pool);
    *out = h;
    return SLLM_OK;
}

void refg_model_close(void * vh) {
    refg_model * h = (refg_model *) vh;
    if (h == NULL) { return; }
    sllm_ctx_free(h->c);
    sllm_pool_destroy(h->pool);
    sllm_model_free(h->m);
    sllm_gguf_close(&h->g);
    free(h);
}

void refg_ctx_reset(void * vh) { sllm_ctx_reset(((refg_model *) vh)->c); }

int refg_forward_chunk(void * vh, const int32_t * tokens, int32_t n, int32_t base, float * logits) {
    refg_model * h = (refg_model *) vh;
    return sllm_forward_chunk(h->m, h->c, tokens, n, base, logits);
}

int refg_generate_greedy(void * vh, const int32_t * prompt, int32_t n_prompt,
                         int32_t n_new, int32_t * out) {
    refg_model * h = (refg_model *) vh;
    return sllm_generate_greedy(h->m, h->c, prompt, n_prompt, n_new, out);
}

int refg_last_logits(void * vh, float * out, int32_t n_vocab) {
    const float * l = sllm_ctx_last_logits(((refg_model *) vh)->c);
    if (l == NULL) { return SLLM_ERR_ARG; }
    memcpy(out, l, (size_t) n_vocab * sizeof(float));
    return SLLM_OK;
}

/* ------------------------------------------------------------------ */
/* kernel level, pooled the way src/forward.c:175-205 pools a GEMV      */
/* ------------------------------------------------------------------ */

typedef struct {
    const uint8_t * w;
    size_t row_bytes, n;
    const int8_t * q;
    int32_t * out;
} refg_gemv_job;

static void refg_gemv_rows(void * vctx, size_t begin, size_t end) {
    const refg_gemv_job * j = (const refg_gemv_job *) vctx;
    sllm_i2s_gemv(j->w + begin * j->row_bytes, end - begin, j->n, j->q, j->out + begin);
}

/* The same distribution rule as src/forward.c:175-205 (grain 64, distribute
 * only when every worker gets 512 rows). */
void refg_gemv_pooled(void * pool, const uint8_t * w, size_t n_rows, size_t n,
                      const int8_t * q, int32_t * out) {
    sllm_pool * p = (sllm_pool *) pool;
    const int t = p ? sllm_pool_threads(p) : 1;
    if (t < 2 || n_rows < (size_t) 512 * (size_t) t || n_rows < 128) {
        sllm_i2s_gemv(w, n_rows, n, q, out);
        return;
    }
    const refg_gemv_job j = { w, n / 4, n, q, out };
    sllm_parallel_rows(p, refg_gemv_rows, (void *) &j, n_rows, 64);
}

/* One projection with the reference kernels: quant, pooled GEMV, epilogue. */
static void refg_project(void * pool, const uint8_t * w, size_t rows, size_t n,
                         const int8_t * q, const sllm_i2s_act * act, int32_t * dots, float * dst) {
    refg_gemv_pooled(pool, w, rows, n, q, dots);
    const float ws = sllm_i2s_scale(w, rows * n);
    for (size_t r = 0; r < rows; ++r) { dst[r] = sllm_i2s_epilogue(dots[r], act->sum, act->scale, ws); }
}

/*
 * The benchmark's layer GEMV chain (see orc_layer_chain in sllm_oracle.h for
 * its definition) run entirely with reference calls: sllm_rms_norm,
 * sllm_i2s_quant_act, pooled sllm_i2s_gemv, sllm_i2s_epilogue,
 * sllm_silu_inplace and sllm_add.
 * `scratch` holds 4*n_embd + 2*n_embd_gqa + 3*n_ff floats; `qbuf` max(n_embd,
 * n_ff) bytes; `dots` max(n_embd, n_ff) int32.
 */
void refg_layer_chain(void * pool, const sllm_cuda_model_desc * m, int32_t layer,
                      float * x, float * scratch, int8_t * qbuf, int32_t * dots) {
    const size_t E = (size_t) m->n_embd, F = (size_t) m->n_ff;
    const size_t G = (size_t) (m->n_embd / m->n_head) * (size_t) m->n_head_kv;
    const sllm_cuda_layer_desc * L = &m->layers[layer];
    float * xn = scratch, * q = xn + E, * k = q + E, * v = k + G, * proj = v + G;
    float * fi = proj + E, * g = fi + E, * u = g + F, * h = u + F;
    sllm_i2s_act act;
    sllm_rms_norm(xn, x, L->attn_norm, E, m->f_rms_eps);
    sllm_i2s_quant_act(xn, E, qbuf, &act);
    refg_project(pool, L->wq, E, E, qbuf, &act, dots, q);
    refg_project(pool, L->wk, G, E, qbuf, &act, dots, k);
    refg_project(pool, L->wv, G, E, qbuf, &act, dots, v);
    sllm_rms_norm(xn, q, L->attn_sub_norm, E, m->f_rms_eps);
    sllm_i2s_quant_act(xn, E, qbuf, &act);
    refg_project(pool, L->wo, E, E, qbuf, &act, dots, proj);
    sllm_add(fi, proj, x, E);
    sllm_rms_norm(xn, fi, L->ffn_norm, E, m->f_rms_eps);
    sllm_i2s_quant_act(xn, E, qbuf, &act);
    refg_project(pool, L->ffn_gate, F, E, qbuf, &act, dots, g);
    refg_project(pool, L->ffn_up, F, E, qbuf, &act, dots, u);
    sllm_silu_inplace(g, F);
    sllm_mul(h, g, u, F);
    sllm_rms_norm(h, h, L->ffn_sub_norm, F, m->f_rms_eps);
    sllm_i2s_quant_act(h, F, qbuf, &act);
    refg_project(pool, L->ffn_down, E, F, qbuf, &act, dots, proj);
    sllm_add(x, proj, fi, E);
}

/* ------------------------------------------------------------------ */
/* the tied F16 head, pooled the way src/forward.c:215-233,818-827     */
/* pools it: rows of sllm_dot_f16_f32 over the pool's workers          */
/* ------------------------------------------------------------------ */

typedef struct {
    const uint16_t * embd;
    const float * x;
    size_t n_embd;
    float * out;
} refg_head_job;

static void refg_head_rows(void * vctx, size_t begin, size_t end) {
    const refg_head_job * j = (const refg_head_job *) vctx;
    for (size_t v = begin; v < end; ++v) {
        j->out[v] = sllm_dot_f16_f32(j->embd + v * j->n_embd, j->x, j->n_embd);
    }
}

void refg_lm_head_pooled(void * pool, const uint16_t * embd, size_t n_rows, size_t n_embd,
                         const float * x, float * out) {
    sllm_pool * p = (sllm_pool *) pool;
    const refg_head_job j = { embd, x, n_embd, out };
    if (p == NULL || sllm_pool_threads(p) < 2) {
        refg_head_rows((void *) &j, 0, n_rows);
        return;
    }
    sllm_parallel_rows(p, refg_head_rows, (void *) &j, n_rows, 64);
}
