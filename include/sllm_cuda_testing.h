/*
 * sllm_cuda_testing.h -- test hooks of libsllm_cuda.so. Not part of the
 * product interface: no reference call site corresponds to these, and a
 * production caller never needs them.
 */
#ifndef SLLM_CUDA_TESTING_H
#define SLLM_CUDA_TESTING_H

#include "sllm_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Force every certified double-precision sum (RMSNorm mean, softmax
 * normaliser) to take its reference-order fallback, so tests can show that
 * the fallback gives the same bits as the fast path. Read when a kernel is
 * launched, and baked into a context's decode graph when the graph is first
 * captured (its first forward), so set it before creating the context.
 */
SLLM_CUDA_API void sllm_cuda_test_set_force_fallback(int on);

/* How many times a fallback ran in this process (or -1 without a device). */
SLLM_CUDA_API int sllm_cuda_test_fallback_count(void);

/*
 * The device error word of the prefill GEMM kernels (0: no bounded wait gave
 * up since the last call of this function, which clears it). Synchronises
 * the device; -1 without a device.
 */
SLLM_CUDA_API int sllm_cuda_test_gemm_error(void);
/* The prefill GEMM's form: 0 by size (at most 16 tokens: weight rows as the
 * MMA's M operand, tokens as N = 16), 1 the 128-token tiles, 2 the skinny
 * form only. */
SLLM_CUDA_API void sllm_cuda_test_gemm_form(int form);
/* sllm_cuda_i2s_gemm over columns of a wider activation matrix: row t of the
 * k contracted bytes starts at q + t * lda (lda >= k, a multiple of 16). */
SLLM_CUDA_API int sllm_cuda_test_gemm_strided(const uint8_t * w, int32_t n_rows, int32_t k, int32_t m,
                                              const int8_t * q, int32_t lda, const sllm_cuda_act * acts,
                                              int32_t * dots, float * y, void * stream);

/*
 * Greedy decode over the N contexts of ranks 0..N-1 of one tensor-parallel
 * model, all on one device and in one process, with the exchanges done by
 * device copies instead of NCCL: the same phases, the same bits, testable on
 * a single GPU. out receives the tokens (every rank's are the same).
 */
/* 1 when the context runs its layer GEMVs on the persistent engine, 0 when
 * on the per-GEMV kernels (widths the engine is not compiled for) */
SLLM_CUDA_API int sllm_cuda_test_tp_uses_engine(const sllm_cuda_tp_ctx * c);

/* the number of layers that run as one fused engine program (Q/K/V,
 * attention, O, gate/up behind grid barriers): n_layer on one rank with the
 * engine, 0 otherwise */
SLLM_CUDA_API int sllm_cuda_test_tp_fused_layers(const sllm_cuda_tp_ctx * c);

/* 1 when the context's step runs the fused peer exchange: per layer one
 * program that stores its results into every rank's memory and waits on
 * flags inside its stages, instead of separate exchange kernels */
SLLM_CUDA_API int sllm_cuda_test_tp_fused_exchange(const sllm_cuda_tp_ctx * c);

/* how the context exchanges between ranks: 0 none (one rank), 1 NCCL
 * collectives, 2 the one-shot peer-memory exchange */
SLLM_CUDA_API int sllm_cuda_test_tp_exchange_kind(const sllm_cuda_tp_ctx * c);

SLLM_CUDA_API int sllm_cuda_test_tp_generate_group(sllm_cuda_tp_ctx ** cs, int32_t n,
                                     const int32_t * prompt, int32_t n_prompt,
                                     int32_t n_new, int32_t * out);

/*
 * How many kernels this library has put on streams in this process: each
 * launch of one of its CUDA graphs adds the graph's kernel nodes, each direct
 * kernel launch adds one. Kernels enqueued while the caller is capturing a
 * stream count when enqueued, not when the caller's graph runs.
 */
SLLM_CUDA_API long long sllm_cuda_test_kernel_launches(void);

/*
 * Device time (ms) of the decode steps of the last forward / generate call on
 * a context: two events recorded on the context's stream around the step
 * launches, so the host round trips before and after are excluded. -1 when
 * nothing has run yet.
 */
SLLM_CUDA_API float sllm_cuda_test_ctx_last_run_ms(const sllm_cuda_ctx * c);
SLLM_CUDA_API float sllm_cuda_test_tp_ctx_last_run_ms(const sllm_cuda_tp_ctx * c);

/*
 * Failure injection without a GPU fault. sllm_cuda_test_fail_next: the next
 * `count` device allocations of a model or context (what = 1) or the next
 * `count` communicator set-ups (what = 2) fail as if refused (NOMEM, COMM).
 * sllm_cuda_test_engine_faults on `device`: every bounded wait of the
 * persistent engine gives up after wait_ms (<= 0: the default 2 s), and CTA
 * skip_arrival_cta (-1: none) leaves out its first grid-barrier arrival, so
 * the other CTAs' barrier waits run out; the call that ran reports
 * SLLM_CUDA_ERR_TIMEOUT and the context stays usable. Read by every launch.
 */
SLLM_CUDA_API void sllm_cuda_test_fail_next(int what, int count);
SLLM_CUDA_API int sllm_cuda_test_engine_faults(int device, int skip_arrival_cta, double wait_ms);

/* The device error word of a GEMV batch's launch: SLLM_CUDA_OK, or
 * SLLM_CUDA_ERR_TIMEOUT when a bounded wait gave up; -1 before its first run. */
SLLM_CUDA_API int sllm_cuda_test_gemv_batch_error(sllm_cuda_gemv_batch * b);

/*
 * The persistent engine's split of each stage's rows over `grid` CTAs, the
 * host computation every engine program is built with (no device is used).
 * Op i has rows[i] rows of K[i] elements, epilogue epi[i] (0 dots, 1 f32,
 * 2 residual, 3 gate/up pair, 4 attention heads) and input group group[i];
 * stage s runs ops [stage_first[s], stage_first[s + 1]). `out` receives
 * n_stages * (grid + 1) cursors as (op, row) pairs: CTA c of stage s runs
 * the rows from cursor c up to cursor c + 1. Returns SLLM_CUDA_ERR_ARG for
 * inconsistent arguments.
 */
/*
 * The tensor-parallel shard of rank `rank` of `n_ranks`, as
 * sllm_cuda_tp_model_upload computes it (host code, no device is used):
 * out[0..7] = query heads, kv heads, n_embd columns (of O), n_ff rows (of
 * gate/up) and columns (of down), down chunks, columns per chunk, first
 * vocabulary row, vocabulary rows. Returns the upload's error for a
 * geometry it refuses.
 */
SLLM_CUDA_API int sllm_cuda_test_tp_plan(int32_t n_layer, int32_t E, int32_t F, int32_t H, int32_t Hkv,
                           int32_t V, int32_t n_ranks, int32_t rank, int32_t * out);

/*
 * Where sllm_cuda_layer_projections cuts a call of n_layers layers into two
 * engine launches (the first piece's outputs are copied back while the
 * second computes): the first layer of the second piece, or 0 when the call
 * runs as one launch (fewer than 16 layers, or widths the engine is not
 * compiled for). -1 for nonsensical widths.
 */
SLLM_CUDA_API int sllm_cuda_test_projection_split(int32_t n_embd, int32_t n_ff, int32_t n_embd_gqa,
                                    int32_t n_layers);

SLLM_CUDA_API int sllm_cuda_test_engine_split(const int32_t * rows, const int32_t * K, const int32_t * epi,
                                const int32_t * group, int32_t n_ops, const int32_t * stage_first,
                                int32_t n_stages, int32_t grid, int32_t * out);

/* device time of the last sllm_cuda_tp_batch_generate_greedy's steps (ms) */
SLLM_CUDA_API float sllm_cuda_test_tp_batch_last_run_ms(const sllm_cuda_tp_batch * b);
/* N batches of the N shards of one model on one device, the exchanges by
 * device copies (as sllm_cuda_test_tp_generate_group) */
SLLM_CUDA_API int sllm_cuda_test_tp_batch_generate_group(sllm_cuda_tp_batch ** bs, int32_t n,
                                                         const int32_t * prompts, int32_t n_prompt,
                                                         int32_t n_new, int32_t * out);

#ifdef __cplusplus
}
#endif

#endif /* SLLM_CUDA_TESTING_H */
