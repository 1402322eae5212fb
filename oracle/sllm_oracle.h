/*
 * sllm_oracle.h -- TEST INFRASTRUCTURE ONLY. A CPU restatement of
 * saphira-llm's I2_S decode path, used as the parity checker for the CUDA
 * backend. Nothing in the product (libsllm_cuda.so) links, loads or calls
 * this code; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg do.
 *
 * Every function restates, in this project's own code, the arithmetic of the
 * reference function it cites (path:line in the saphira-llm tree), in the
 * reference's exact floating-point order: where the reference's x86-64-v3
 * build vectorises a reduction, the restatement spells out the same lane
 * structure in scalar code. Build with -ffp-contract=off (oracle/Makefile),
 * as the reference is (Makefile:34).
 *
 * Parity is pinned two ways, both in tests/: against the reference compiled
 * from its own sources (oracle/_ref/libsllm_ref.so, built by oracle/Makefile)
 * on seeded inputs, and against the reference's own golden vectors and
 * known-answer tests (tests/golden/).
 */
#ifndef SLLM_ORACLE_H
#define SLLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/sllm_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_act {
    float   scale;
    int32_t sum;
} orc_act;

/* I2_S format and kernels (src/i2s_gemm.c, src/quant.c, src/i2s_convert.c) */
void     orc_i2s_quant_act(const float * x, size_t n, int8_t * q, orc_act * act);
int32_t  orc_i2s_dot(const uint8_t * w, const int8_t * q, size_t n);
void     orc_i2s_gemv(const uint8_t * w, size_t n_rows, size_t n,
                      const int8_t * q, int32_t * rows_out);
float    orc_i2s_epilogue(int32_t dot, int32_t act_sum, float act_scale, float w_scale);
float    orc_i2s_scale(const uint8_t * packed, size_t n_elements);
uint8_t  orc_i2s_code(const uint8_t * packed, size_t k);
size_t   orc_i2s_packed_size(size_t n_elements);
int      orc_i2s_pack_codes(const uint8_t * codes, size_t n, float scale, uint8_t * dst);
int      orc_i2s_quantize_scaled_py(const float * src, size_t n, float scale, uint8_t * dst);
/* quant + GEMV + epilogue, as src/forward.c:651-655 runs one projection */
void     orc_i2s_gemv_f32(const uint8_t * w, size_t n_rows, size_t n,
                          const float * x, float * y, int32_t * dots);

/* vector ops (src/ops.c, src/forward.c) */
float    orc_fp16_to_fp32(uint16_t h);
float    orc_fp16_to_fp32_embd(uint16_t h);
void     orc_rms_norm(float * dst, const float * x, const float * w, size_t n, float eps);
float    orc_v_expf(float x);
void     orc_softmax(float * x, size_t n);
void     orc_silu(float * x, size_t n);
void     orc_rope_neox(float * x, size_t n_rot, int32_t pos, float theta);
float    orc_dot_f16(const uint16_t * row, const float * x, size_t n);
int32_t  orc_argmax(const float * logits, int32_t n);

/* the decode chain (src/forward.c:466-938) on a model description */
typedef struct orc_ctx orc_ctx;
int      orc_ctx_new(const sllm_cuda_model_desc * m, int32_t n_ctx, orc_ctx ** out);
void     orc_ctx_free(orc_ctx * c);
void     orc_ctx_reset(orc_ctx * c);
int32_t  orc_ctx_n_past(const orc_ctx * c);
/* this project's fp16-KV variant (not the reference): round cached values to half */
void     orc_ctx_set_kv_f16(orc_ctx * c, int on);
uint16_t orc_fp32_to_fp16(float f);
const float * orc_ctx_last_logits(const orc_ctx * c);
int      orc_forward_chunk(const sllm_cuda_model_desc * m, orc_ctx * c,
                           const int32_t * tokens, int32_t n, int32_t base,
                           float * logits_out);
int      orc_generate_greedy(const sllm_cuda_model_desc * m, orc_ctx * c,
                             const int32_t * prompt, int32_t n_prompt,
                             int32_t n_new, int32_t * out);

/*
 * The projection chain of one layer without attention, the workload the
 * benchmark calls "layer GEMV chain": norm -> quant -> Q,K,V; Q stands in for
 * the attention output -> sub-norm -> O -> +x; ffn norm -> gate, up ->
 * silu(gate)*up -> ffn sub-norm -> down -> +residual. Every op in it is the
 * decode layer's own (src/forward.c:631-801). `x` is updated in place.
 * `scratch` must hold 4*n_embd + 2*n_embd_gqa + 3*n_ff floats.
 */
void     orc_layer_chain(const sllm_cuda_model_desc * m, int32_t layer,
                         float * x, float * scratch);

/* number of OpenMP threads the row loops use (results never depend on it) */
void     orc_set_threads(int n);

#ifdef __cplusplus
}
#endif

#endif /* SLLM_ORACLE_H */
