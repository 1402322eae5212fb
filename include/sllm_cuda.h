/*
 * sllm_cuda.h -- the C ABI of the B200 (sm_100a) backend for saphira-llm's
 * I2_S ternary decode path.
 *
 * Everything here is plain C: pointers, sizes and int status codes. No CUDA,
 * torch or C++ type crosses this boundary, so saphira-llm's C11 host code can
 * include this header and link libsllm_cuda.so directly. A stream is passed as
 * `void *` (a cudaStream_t value; NULL means the legacy default stream).
 *
 * Each entry point names the reference interface it replaces, as
 * path:line inside the saphira-llm source tree.
 *
 * Conventions, held by every function below:
 *   - Status codes are numerically identical to saphira-llm's sllm_status
 *     (include/saphira_llm/status.h:26-56), so a caller can return them
 *     unchanged. Three new negative codes (-60, -61, -62) name device-side
 *     failures.
 *   - The kernel-level functions take DEVICE pointers and are asynchronous on
 *     the given stream. The model-level functions take HOST pointers and
 *     return when their results are on the host.
 *   - Once this backend is selected there is no CPU fallback. A missing or
 *     unsuitable device is reported as SLLM_CUDA_ERR_UNSUPPORTED, never
 *     silently computed on the host.
 */
#ifndef SLLM_CUDA_H
#define SLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#  define SLLM_CUDA_API __attribute__((visibility("default")))
#else
#  define SLLM_CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ */
/* status codes                                                        */
/* ------------------------------------------------------------------ */

#define SLLM_CUDA_OK               0    /* SLLM_OK                  */
#define SLLM_CUDA_ERR_ARG         (-1)  /* SLLM_ERR_ARG             */
#define SLLM_CUDA_ERR_NOMEM       (-2)  /* SLLM_ERR_NOMEM: host or device allocation failed */
#define SLLM_CUDA_ERR_IO          (-3)  /* SLLM_ERR_IO              */
#define SLLM_CUDA_ERR_UNSUPPORTED (-4)  /* SLLM_ERR_UNSUPPORTED: no sm_100 device, or a shape this backend does not run */
#define SLLM_CUDA_ERR_TRUNCATED   (-12) /* SLLM_ERR_GGUF_TRUNCATED: a state file ends early */
#define SLLM_CUDA_ERR_KV_TYPE     (-32) /* SLLM_ERR_KV_TYPE: not a state file, or another version */
#define SLLM_CUDA_ERR_TENSOR_SHAPE (-34) /* SLLM_ERR_TENSOR_SHAPE: a state file of another geometry */
#define SLLM_CUDA_ERR_TOO_LARGE   (-36) /* SLLM_ERR_TOO_LARGE       */
#define SLLM_CUDA_ERR_DEVICE      (-60) /* a CUDA runtime call or kernel launch failed */
#define SLLM_CUDA_ERR_TIMEOUT     (-61) /* a bounded device-side wait ran out; the context stays usable */
#define SLLM_CUDA_ERR_COMM        (-62) /* a collective between devices failed */

/* Stable, human-readable name for a status. Never NULL. */
SLLM_CUDA_API const char * sllm_cuda_status_string(int status);

/* The message recorded with the most recent failure on this thread, or "". */
SLLM_CUDA_API const char * sllm_cuda_last_error(void);

/*
 * Capability probe for the dispatch row (src/dispatch.c:133
 * sllm_dispatch_resolve, src/i2s_gemm.c:315 sllm_i2s_select_auto).
 * Reports the device count and the compute capability of device 0.
 * Returns SLLM_CUDA_ERR_UNSUPPORTED when no device of compute capability
 * 10.x is visible. Any output pointer may be NULL.
 */
SLLM_CUDA_API int sllm_cuda_probe(int * n_devices, int * cc_major, int * cc_minor);

/* ------------------------------------------------------------------ */
/* kernel level: device pointers, asynchronous on `stream`             */
/* ------------------------------------------------------------------ */

/* Layout-identical to sllm_i2s_act (include/saphira_llm/i2s_gemm.h:37-40). */
typedef struct sllm_cuda_act {
    float   scale;   /* 127 / amax, or 0 for an all-zero row */
    int32_t sum;     /* sum of the quantised values          */
} sllm_cuda_act;

/*
 * Per-token int8 absmax quantisation of one row of `n` floats.
 * Replaces sllm_i2s_quant_act (include/saphira_llm/i2s_gemm.h:57,
 * src/i2s_gemm.c:45-83) with identical results: amax without a floor,
 * scale = 127/amax (IEEE division), q = clamp(roundf(x*scale)), sum of q.
 * `act_out` is one device struct. n must be >= 1 and <= 65536.
 */
SLLM_CUDA_API int sllm_cuda_i2s_quant_act(const float * x, size_t n, int8_t * q_out,
                            sllm_cuda_act * act_out, void * stream);

/*
 * Raw I2_S GEMV: rows_out[r] = sum over k of code(w, r, k) * q[k], the
 * 2-bit code (0, 1 or 2) times the int8 activation, in int32.
 * Replaces sllm_i2s_gemv (include/saphira_llm/i2s_gemm.h:81,
 * src/i2s_gemm.c:260-269) bit for bit. `w` is the packed tensor as stored in
 * the GGUF (rows of n/4 bytes, I2_S interleaved layout). Unlike the reference,
 * which silently returns 0 for n < 128, this returns SLLM_CUDA_ERR_ARG for
 * n % 128 != 0 (the loader refuses such tensors anyway, src/forward.c:306-316).
 * n above 8192 is refused with SLLM_CUDA_ERR_UNSUPPORTED (the 2B-4T model's
 * widths are 2560 and 6912; the tensor-parallel path splits wider
 * contractions into chunks of at most 8192).
 */
SLLM_CUDA_API int sllm_cuda_i2s_gemv(const uint8_t * w, size_t n_rows, size_t n,
                       const int8_t * q, int32_t * rows_out, void * stream);

/*
 * Fused float GEMV: quantise x (as sllm_cuda_i2s_quant_act), run the raw GEMV
 * and apply the epilogue y[r] = (float)(dot[r] - act.sum) * (w_scale / act.scale),
 * where w_scale is the f32 stored after the packed weights
 * (src/quant.c:102-106). This is the sequence src/forward.c:651-655 runs for
 * every projection, and the epilogue grouping is sllm_i2s_epilogue's
 * (src/i2s_gemm.c:271-290). `dots` (nullable) receives the raw int32 dots.
 */
SLLM_CUDA_API int sllm_cuda_i2s_gemv_f32(const uint8_t * w, size_t n_rows, size_t n,
                           const float * x, float * y, int32_t * dots,
                           void * stream);

/*
 * A batch of `count` (<= 256) independent float GEMVs of one shape, each as
 * sllm_cuda_i2s_gemv_f32 computes it, run as one persistent launch: GEMV i
 * reads the packed tensor w[i] (device, 16-byte aligned, scale tail after the
 * codes), input x + i * x_stride (x_stride 0: every GEMV shares x, as Q, K and
 * V share one quantised activation in src/forward.c:651-666) and writes
 * y + i * n_rows. It replaces a host loop of sllm_i2s_quant_act +
 * sllm_i2s_gemv + epilogue over tensors (src/i2s_gemm.c:45-83, :260-290;
 * bench/kernel_bench.c:62-130 times such loops). n_rows % 4 == 0. The first
 * run with given x, x_stride and y builds the launch's tables (device
 * allocation); later runs with the same buffers only launch. Results are
 * bit-identical to sllm_cuda_i2s_gemv_f32 on each tensor.
 */
typedef struct sllm_cuda_gemv_batch sllm_cuda_gemv_batch;
SLLM_CUDA_API int sllm_cuda_gemv_batch_new(const uint8_t * const * w, size_t count, size_t n_rows,
                                           size_t n, int device, sllm_cuda_gemv_batch ** out);
SLLM_CUDA_API int sllm_cuda_gemv_batch_run(sllm_cuda_gemv_batch * b, const float * x, size_t x_stride,
                                           float * y, void * stream);
SLLM_CUDA_API void sllm_cuda_gemv_batch_free(sllm_cuda_gemv_batch * b);

/* ------------------------------------------------------------------ */
/* multi-token (prefill) kernels: device pointers                      */
/* ------------------------------------------------------------------ */

/*
 * Per-token activation quantisation of a row-major [m][n] batch: row t of q
 * and acts[t] are sllm_i2s_quant_act of row t of x
 * (include/saphira_llm/i2s_gemm.h:59, src/i2s_gemm.c:45-83), the per-token
 * quantisation the prefill runs before each projection (src/forward.c:756-764).
 */
SLLM_CUDA_API int sllm_cuda_i2s_quant_act_rows(const float * x, size_t m, size_t n,
                                 int8_t * q, sllm_cuda_act * acts, void * stream);

/*
 * Prefill GEMM on the tensor cores: for every token t < m and row r <
 * n_rows, dots[t][r] = sum over k of code(w, r, k) * q[t][k] (int32), which is
 * sllm_i2s_gemv of token t (src/i2s_gemm.c:260-269) bit for bit, and
 * y[t][r] = (float)(dots[t][r] - acts[t].sum) * (w_scale / acts[t].scale),
 * the per-token epilogue of src/forward.c:653-655. The reference has no GEMM:
 * its prefill runs the GEMV once per token; this computes all of them in one
 * int8 contraction. q is row-major [m][n]; dots and y are row-major
 * [m][n_rows] and either may be NULL (not both). n % 128 == 0, n <= 65536;
 * w and q 16-byte aligned. Asynchronous on `stream`.
 */
SLLM_CUDA_API int sllm_cuda_i2s_gemm(const uint8_t * w, size_t n_rows, size_t n, size_t m,
                       const int8_t * q, const sllm_cuda_act * acts,
                       int32_t * dots, float * y, void * stream);

/*
 * The gate/up pair of the prefill FFN in one pass: h[t][r] =
 * silu(gate[t][r]) * up[t][r], each projection with the epilogue above and
 * SiLU as sllm_silu_inplace computes it (src/forward.c:756-779,
 * src/ops.c:428-461). w_gate and w_up have the same shape.
 */
SLLM_CUDA_API int sllm_cuda_i2s_gemm_silu(const uint8_t * w_gate, const uint8_t * w_up, size_t n_rows,
                            size_t n, size_t m, const int8_t * q,
                            const sllm_cuda_act * acts, float * h, void * stream);

/* ------------------------------------------------------------------ */
/* model level: host pointers                                          */
/* ------------------------------------------------------------------ */

/*
 * One bitnet-b1.58 layer as the reference loader records it
 * (src/forward.c:47-54, filled at src/forward.c:391-444). The I2_S pointers
 * address packed tensors INCLUDING their scale tail (rows * cols / 4 bytes of
 * codes, then the f32 scale and 28 pad bytes). All pointers are host memory
 * and are only read during sllm_cuda_model_upload.
 */
typedef struct sllm_cuda_layer_desc {
    const uint8_t * wq;        /* n_embd     x n_embd  */
    const uint8_t * wk;        /* n_embd_gqa x n_embd  */
    const uint8_t * wv;        /* n_embd_gqa x n_embd  */
    const uint8_t * wo;        /* n_embd     x n_embd  */
    const uint8_t * ffn_gate;  /* n_ff       x n_embd  */
    const uint8_t * ffn_up;    /* n_ff       x n_embd  */
    const uint8_t * ffn_down;  /* n_embd     x n_ff    */
    const float   * attn_norm;      /* n_embd */
    const float   * attn_sub_norm;  /* n_embd */
    const float   * ffn_norm;       /* n_embd */
    const float   * ffn_sub_norm;   /* n_ff   */
} sllm_cuda_layer_desc;

/*
 * The model hyperparameters and tensors (src/forward.c:56-76; metadata keys
 * read at src/forward.c:348-366). `tok_embd` is the F16 [n_vocab][n_embd]
 * embedding that is also the tied output head.
 */
typedef struct sllm_cuda_model_desc {
    int32_t n_layer;
    int32_t n_embd;
    int32_t n_ff;
    int32_t n_head;
    int32_t n_head_kv;
    int32_t n_vocab;
    int32_t n_rot;
    int32_t n_ctx_train;
    float   f_rms_eps;
    float   rope_freq_base;
    const uint16_t * tok_embd;     /* F16 bits, n_vocab * n_embd */
    const float    * output_norm;  /* n_embd */
    const sllm_cuda_layer_desc * layers;  /* n_layer entries */
} sllm_cuda_model_desc;

typedef struct sllm_cuda_model sllm_cuda_model;
typedef struct sllm_cuda_ctx   sllm_cuda_ctx;

/*
 * Copy a model to device `device` once; the device copy is immutable and may
 * be shared by several contexts. Validates the same shape rules as
 * sllm_model_load (src/forward.c:368-444): returns SLLM_CUDA_ERR_ARG for a
 * NULL desc or tensor, SLLM_CUDA_ERR_UNSUPPORTED for widths this backend does
 * not run (n_embd or n_ff not a multiple of 128 or above 8192, a head dim
 * n_embd / n_head other than 128, n_rot other than the head dim,
 * n_head % n_head_kv != 0), SLLM_CUDA_ERR_NOMEM when device memory runs out.
 * Pairs with sllm_model_load / sllm_model_free (include/saphira_llm/forward.h:32-33).
 */
SLLM_CUDA_API int  sllm_cuda_model_upload(const sllm_cuda_model_desc * desc, int device,
                            sllm_cuda_model ** out);
SLLM_CUDA_API void sllm_cuda_model_free(sllm_cuda_model * m);

/*
 * A context owns the device-resident KV cache (fp32, [layer][head_kv][pos][dim],
 * src/forward.c:81-83) and the scratch of one sequence.
 * Replaces sllm_ctx_new / sllm_ctx_free / sllm_ctx_reset
 * (include/saphira_llm/forward.h:44-48, src/forward.c:466-562).
 */
SLLM_CUDA_API int  sllm_cuda_ctx_new(const sllm_cuda_model * m, int32_t n_ctx,
                       sllm_cuda_ctx ** out);

/*
 * The same with a choice of KV cache type. SLLM_CUDA_KV_F32 is the
 * reference's cache and sllm_cuda_ctx_new's. SLLM_CUDA_KV_F16 is an option the
 * reference does not have: every cached K and V value is stored rounded to
 * the nearest half (ties to even) and read back exactly, halving the cache.
 * Everything else is computed as in the fp32 context, so the logits differ
 * from the reference's only through that rounding; the benchmark reports how
 * many greedy tokens still agree. State files stay SLKV v1 with f32 values
 * (export widens exactly, import rounds).
 */
#define SLLM_CUDA_KV_F32 0
#define SLLM_CUDA_KV_F16 1
SLLM_CUDA_API int  sllm_cuda_ctx_new_kv(const sllm_cuda_model * m, int32_t n_ctx, int32_t kv_type,
                                        sllm_cuda_ctx ** out);
SLLM_CUDA_API void sllm_cuda_ctx_free(sllm_cuda_ctx * c);
SLLM_CUDA_API void sllm_cuda_ctx_reset(sllm_cuda_ctx * c);

/* Tokens consumed so far (the reference's n_past). */
SLLM_CUDA_API int32_t sllm_cuda_ctx_n_past(const sllm_cuda_ctx * c);

/*
 * Run `n` tokens at absolute positions [base, base+n) and write n * n_vocab
 * logits to `logits_out` (host, may be NULL when only `argmax_out` is wanted).
 * `argmax_out` (host, nullable) receives the argmax of each position's logits
 * (lowest index on ties, src/forward.c:876-883). Argument rules and status
 * codes follow sllm_forward_chunk (include/saphira_llm/forward.h:107-109,
 * src/forward.c:589-609): n in [1, 256], base >= n_past, base + n <= n_ctx,
 * tokens in [0, n_vocab).
 */
SLLM_CUDA_API int sllm_cuda_forward_chunk(const sllm_cuda_model * m, sllm_cuda_ctx * c,
                            const int32_t * tokens, int32_t n, int32_t base,
                            float * logits_out, int32_t * argmax_out);

/*
 * Greedy generation, replacing sllm_generate_greedy
 * (include/saphira_llm/forward.h:136-138, src/forward.c:885-938), including
 * its BOS fallback (128000) and its continuation from the last logits when
 * n_prompt == 0. The whole loop runs on the device: one token id crosses back
 * per generated token only at the end, in `out` (n_new ids).
 */
SLLM_CUDA_API int sllm_cuda_generate_greedy(const sllm_cuda_model * m, sllm_cuda_ctx * c,
                              const int32_t * prompt, int32_t n_prompt,
                              int32_t n_new, int32_t * out);

/*
 * The projection chain of layers [layer_begin, layer_begin + n_layers) without
 * attention -- the workload the benchmark measures as "one layer's seven I2_S
 * GEMVs with RMSNorm between them": attn_norm -> quant -> Q, K, V; Q stands in
 * for the attention output -> attn_sub_norm -> quant -> O -> + x; ffn_norm ->
 * quant -> gate, up -> silu(gate) * up -> ffn_sub_norm -> quant -> down ->
 * + residual. Every step is the decode layer's own (src/forward.c:631-801),
 * with the same rounding. `x_in` / `x_out` are host arrays of n_embd floats
 * (they may alias). Uses the context's scratch and stream; it does not touch
 * the KV cache or n_past.
 */
SLLM_CUDA_API int sllm_cuda_layer_chain(const sllm_cuda_model * m, sllm_cuda_ctx * c,
                          int32_t layer_begin, int32_t n_layers,
                          const float * x_in, float * x_out);

/*
 * The same chain on a device vector `x` (n_embd floats, 16-byte aligned,
 * updated in place), asynchronous on `stream`. It uses the context's scratch
 * buffers, so it must not overlap other work on the same context.
 */
SLLM_CUDA_API int sllm_cuda_layer_chain_device(const sllm_cuda_model * m, sllm_cuda_ctx * c,
                                 int32_t layer_begin, int32_t n_layers,
                                 float * x, void * stream);

/*
 * The seven projections of layers [layer_begin, layer_begin + n_layers), each
 * on its OWN input vector -- the benchmark's configuration 1 taken literally
 * ("each uses an f32 N(0,1) activation ... with RMSNorm between them"). For
 * every layer, GEMV p normalises input p with the norm its projection uses in
 * the decode layer (Q, K, V: attn_norm; O: attn_sub_norm; gate, up: ffn_norm;
 * down: ffn_sub_norm), quantises it per token and writes f32 outputs; nothing
 * feeds one projection into another, so consecutive GEMVs overlap on the
 * device.
 *   x: 6 * n_embd + n_ff floats, inputs of Q, K, V, O, gate, up (n_embd each)
 *      and down (n_ff), shared by every layer;
 *   y: n_layers blocks of 3 * n_embd + 2 * n_embd_gqa + 2 * n_ff floats:
 *      Q (n_embd), K, V (n_embd_gqa), O (n_embd), gate, up (n_ff), down (n_embd).
 * sllm_cuda_layer_projections_sizes returns the input length and stores the
 * per-layer output length. The _device form takes 16-byte aligned device
 * vectors and is asynchronous on `stream`. The host form returns when y is on
 * the host; from 16 layers up it runs them as two launches and copies the
 * first launch's outputs back on a second stream of the context while the
 * second computes (any host memory; pinned copies faster).
 */
SLLM_CUDA_API size_t sllm_cuda_layer_projections_sizes(const sllm_cuda_model * m,
                                                       size_t * y_floats_per_layer);
SLLM_CUDA_API int sllm_cuda_layer_projections(const sllm_cuda_model * m, sllm_cuda_ctx * c,
                                              int32_t layer_begin, int32_t n_layers,
                                              const float * x_host, float * y_host);
SLLM_CUDA_API int sllm_cuda_layer_projections_device(const sllm_cuda_model * m, sllm_cuda_ctx * c,
                                                     int32_t layer_begin, int32_t n_layers,
                                                     const float * x, float * y, void * stream);

/*
 * sllm_cuda_layer_chain_device without any allocation. This entry point has
 * no counterpart in the reference: it serves callers that cannot call
 * cudaMalloc -- hosts whose own allocator already holds the device's memory
 * (a late cudaMalloc fails or fragments it), loops that cannot take
 * cudaMalloc's implicit device synchronisation -- and that hold a model but
 * no context. Same results as sllm_cuda_layer_chain_device, bit for bit. It
 * calls no cudaMalloc, cudaFree or allocating library routine.
 *
 * Its scratch (2*n_embd + 2*n_embd_gqa + n_ff floats) is a fixed 128 KB
 * device array inside the library (32768 floats), held by every device that
 * loads the library until the process exits; a larger model is refused with
 * SLLM_CUDA_ERR_TOO_LARGE. The first call on a device looks up the array's
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture. Every call on a device shares the one array, so calls that can
 * overlap on the GPU (different streams, or different threads) race: order
 * them on one stream. `x` is a device vector of n_embd floats, 16-byte
 * aligned, updated in place; asynchronous on `stream`.
 */
SLLM_CUDA_API int sllm_cuda_layer_chain_device_noalloc(const sllm_cuda_model * m,
                                                       int32_t layer_begin, int32_t n_layers,
                                                       float * x, void * stream);

/*
 * The KV cache of a context in the reference's host layout: k_out / v_out are
 * n_layer * n_head_kv * n_ctx * 128 floats each, [layer][kv head][pos][dim]
 * (src/forward.c:81-83, the layout sllm_ctx_new allocates at
 * src/forward.c:480-487). Export writes the rows of positions below n_past
 * and leaves the others untouched. Import replaces the device cache with the
 * given rows below n_past, clears every row at or above it, and sets n_past
 * and the last position's logits (n_vocab floats; NULL only when n_past is
 * 0), so that a generation without a prompt continues from them, as after
 * sllm_state_load (src/forward.c:1034-1123).
 */
SLLM_CUDA_API int sllm_cuda_ctx_kv_export(const sllm_cuda_ctx * c, float * k_out, float * v_out);
SLLM_CUDA_API int sllm_cuda_ctx_kv_import(sllm_cuda_ctx * c, const float * k_in, const float * v_in,
                                          int32_t n_past, const float * last_logits);

/*
 * Save / restore a context's state in the reference's own file format, SLKV
 * version 1 (src/forward.c:963-1123): files written here load into a CPU
 * context of the same model and back, and continue identically. Replaces
 * sllm_state_save / sllm_state_load (include/saphira_llm/forward.h:155-156),
 * with the same refusals: SLLM_CUDA_ERR_KV_TYPE for a file that is not SLKV
 * v1, SLLM_CUDA_ERR_TENSOR_SHAPE for another model or context depth,
 * SLLM_CUDA_ERR_TRUNCATED for a short file, SLLM_CUDA_ERR_IO when the file
 * cannot be opened or written.
 */
SLLM_CUDA_API int sllm_cuda_state_save(const sllm_cuda_model * m, const sllm_cuda_ctx * c, const char * path);
SLLM_CUDA_API int sllm_cuda_state_load(const sllm_cuda_model * m, sllm_cuda_ctx * c, const char * path);

/* Bytes of weights one decode step streams: every I2_S tensor with its scale
 * tail, every norm, and the F16 embedding / output head. */
SLLM_CUDA_API size_t sllm_cuda_model_weight_bytes(const sllm_cuda_model * m);

/*
 * Copy the most recent position's logits (n_vocab floats) to host memory.
 * Replaces sllm_ctx_last_logits (include/saphira_llm/forward.h:77).
 * Returns SLLM_CUDA_ERR_ARG if nothing has been forwarded yet.
 */
SLLM_CUDA_API int sllm_cuda_ctx_last_logits(const sllm_cuda_ctx * c, float * host_out);

/* ------------------------------------------------------------------ */
/* tensor-parallel decode across the GPUs of one node                  */
/* ------------------------------------------------------------------ */
/*
 * The reference decodes on one host (src/forward.c:589-835); these entry
 * points shard the same forward pass over N GPUs, one process (rank) per
 * GPU: Q/K/V and gate/up split by rows (heads, FFN rows), O and down by
 * contraction columns with an int32 all-reduce of the partial dots (exact in
 * any order), the tied f16 head by vocabulary rows. Every rank calls every
 * entry point with the same arguments (SPMD); the results equal the
 * single-GPU path's, bit for bit. NCCL carries the exchanges.
 */
#define SLLM_CUDA_TP_ID_BYTES 128

typedef struct sllm_cuda_tp_comm sllm_cuda_tp_comm;
typedef struct sllm_cuda_tp_model sllm_cuda_tp_model;
typedef struct sllm_cuda_tp_ctx sllm_cuda_tp_ctx;

/* the group's identity: rank 0 creates it and hands the bytes to the others */
SLLM_CUDA_API int sllm_cuda_tp_unique_id(uint8_t * id_out);
SLLM_CUDA_API int sllm_cuda_tp_comm_init(const uint8_t * id, int32_t n_ranks, int32_t rank,
                           int32_t device, sllm_cuda_tp_comm ** out);
SLLM_CUDA_API void sllm_cuda_tp_comm_free(sllm_cuda_tp_comm * c);

/*
 * Rank `rank`'s shard of a model given as host tensors (the same description
 * as sllm_cuda_model_upload). n_head, n_head_kv, n_embd / n_ranks and
 * n_ff / n_ranks must divide evenly (multiples of 128 for the widths); head
 * dim 128, n_embd <= 8192, n_ff <= 28672.
 */
SLLM_CUDA_API int sllm_cuda_tp_model_upload(const sllm_cuda_model_desc * d, int32_t n_ranks,
                              int32_t rank, int32_t device, sllm_cuda_tp_model ** out);

/*
 * A seeded synthetic model generated on the device, shard by shard (the
 * benchmark's configs[4]: 80 layers, 8192 / 28672, 64 / 8 heads, vocab
 * 128256): ternary codes i.i.d. over {-1, 0, 1} from a counter-based hash of
 * (seed, layer, tensor, row, column), per-tensor scales in [0.01, 0.1), norm
 * weights ~N(1, 0.02), the f16 table ~N(0, 0.02). Every shard is a slice of
 * the same model for every rank count.
 */
typedef struct sllm_cuda_tp_synth_desc {
    int32_t  n_layer, n_embd, n_ff, n_head, n_head_kv, n_vocab;
    float    f_rms_eps, rope_freq_base;
    uint64_t seed;
} sllm_cuda_tp_synth_desc;

SLLM_CUDA_API int sllm_cuda_tp_model_synth(const sllm_cuda_tp_synth_desc * d, int32_t n_ranks,
                             int32_t rank, int32_t device, sllm_cuda_tp_model ** out);
SLLM_CUDA_API void sllm_cuda_tp_model_free(sllm_cuda_tp_model * m);
SLLM_CUDA_API size_t sllm_cuda_tp_model_bytes(const sllm_cuda_tp_model * m);
/* this shard's vocabulary rows [*v0, *v0 + *n) */
SLLM_CUDA_API int sllm_cuda_tp_vocab_range(const sllm_cuda_tp_model * m, int32_t * v0, int32_t * n);

/*
 * a decode context over one shard. sllm_cuda_tp_generate_greedy needs comm
 * whenever the model has more than one rank; a context without one serves a
 * single rank, or a one-process test group.
 */
SLLM_CUDA_API int sllm_cuda_tp_ctx_new(const sllm_cuda_tp_model * m, sllm_cuda_tp_comm * comm,
                         int32_t n_ctx, sllm_cuda_tp_ctx ** out);
SLLM_CUDA_API void sllm_cuda_tp_ctx_free(sllm_cuda_tp_ctx * c);
SLLM_CUDA_API int sllm_cuda_tp_ctx_reset(sllm_cuda_tp_ctx * c);

/*
 * sllm_generate_greedy (src/forward.c:885-938) over the shards: argument
 * rules, BOS fallback and outputs as sllm_cuda_generate_greedy. A step whose
 * exchanges make no progress for 120 s aborts the communicator and returns
 * SLLM_CUDA_ERR_TIMEOUT. The exchanges are NCCL collectives, or, with the
 * environment variable SLLM_CUDA_TP_EXCHANGE=p2p at context creation, one-shot
 * kernels that store into the peers' memory over NVLink (CUDA IPC) and wait
 * on epoch flags (bounded).
 */
SLLM_CUDA_API int sllm_cuda_tp_generate_greedy(sllm_cuda_tp_ctx * c, const int32_t * prompt,
                                 int32_t n_prompt, int32_t n_new, int32_t * out);
/* the last step's logits of this shard's vocabulary rows */
SLLM_CUDA_API int sllm_cuda_tp_last_logits(const sllm_cuda_tp_ctx * c, float * host_out);

/*
 * Batch decode over one shard: n_seq <= 16 sequences, each with its own KV
 * cache of n_ctx positions, stepped together. The reference serves a batch
 * as one context per sequence (src/forward.c:78-84, :466-562); here each
 * layer GEMV of a step is one GEMM over the n_seq tokens on the tensor cores
 * (every weight byte read once per step), and each sequence's tokens and
 * logits equal, bit for bit, those of sllm_cuda_tp_generate_greedy on its own
 * context. E <= 8192 and F <= 32768 (a multiple of 32). Needs comm as a
 * context does.
 */
typedef struct sllm_cuda_tp_batch sllm_cuda_tp_batch;
SLLM_CUDA_API int sllm_cuda_tp_batch_new(const sllm_cuda_tp_model * m, sllm_cuda_tp_comm * comm,
                                         int32_t n_seq, int32_t n_ctx, sllm_cuda_tp_batch ** out);
SLLM_CUDA_API void sllm_cuda_tp_batch_free(sllm_cuda_tp_batch * b);
SLLM_CUDA_API int sllm_cuda_tp_batch_reset(sllm_cuda_tp_batch * b);
/*
 * sllm_generate_greedy (src/forward.c:885-938) for every sequence at once:
 * prompts is row-major [n_seq][n_prompt] (the same length for every
 * sequence; n_prompt may be 0 only to continue after an earlier call), out
 * receives row-major [n_seq][n_new]. Failures as sllm_cuda_tp_generate_greedy.
 */
SLLM_CUDA_API int sllm_cuda_tp_batch_generate_greedy(sllm_cuda_tp_batch * b, const int32_t * prompts,
                                                     int32_t n_prompt, int32_t n_new, int32_t * out);
/* sequence seq's last-step logits of this shard's vocabulary rows */
SLLM_CUDA_API int sllm_cuda_tp_batch_last_logits(const sllm_cuda_tp_batch * b, int32_t seq, float * host_out);

#ifdef __cplusplus
}
#endif

#endif /* SLLM_CUDA_H */
