// decode.cuh -- parameters of the decode-step kernels (decode.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace sllm {

struct AttnParams {
    const float* q;          // [n_head * 128] projected, before RoPE
    const float* k;          // [n_head_kv * 128]
    const float* v;          // [n_head_kv * 128]
    float* k_cache;          // this layer: [n_head_kv][128][n_ctx] (K stored transposed); __half when kv_f16
    float* v_cache;          // this layer: [n_head_kv][n_ctx][128]; __half when kv_f16
    const float* rope_cos;   // [n_ctx][64]
    const float* rope_sin;   // [n_ctx][64]
    const int32_t* pos_ptr;  // absolute position of the query (device)
    float* out;              // [n_head * 128]
    int n_ctx;
    int group;               // query heads per kv head
    float attn_scale;        // 1.0f / sqrtf(128.0f)
    int* fallback_count;     // nullable
    int force_fallback;
    int kv_f16;              // kAttnKvF16: the cache holds f16 (the fp16 KV option), else f32 (the
                             // reference's); | kAttnKvStored: this position's k, v are already stored
};
constexpr int kAttnKvF16 = 1;
constexpr int kAttnKvStored = 2;

struct LmParams {
    const float* x;          // residual stream [E]
    const float* norm_w;     // output_norm [E]
    float eps;
    const uint16_t* embd;    // tied head, f16 [V][E]
    int E, V;
    float* logits;           // [V]
    float* part_v;           // [grid] per-CTA best value
    int* part_i;             // [grid] per-CTA best index
    int* counter;            // zero between launches
    int* argmax_out;         // [1]
    int32_t* pos_ptr;        // advanced by one at the end of the step
    int32_t* tok_seq;        // token of each position; greedy writes pos + 1
    const int32_t* prompt_end;
    int32_t* argmax_hist;    // nullable: argmax of each position
    int n_ctx;
    int* fallback_count;
    int force_fallback;
    // tensor-parallel vocabulary slice (nullable): rows are global rows
    // row_base .. row_base + V - 1; the last CTA writes {best value bits,
    // best global row, isnan(logits[0])} here and leaves the argmax across
    // slices, the greedy feedback and the position advance to the caller
    int32_t* tp_out;
    int row_base;
};

// The head of a batch of B sequences' residual streams x [B][E]: every
// token's logits and per-slice best as LmParams's tensor-parallel form.
struct LmBatchParams {
    const float* x;          // [B][E]
    const float* norm_w;
    float eps;
    const uint16_t* embd;    // f16 [V][E]: the slice's first row
    int E, V, B;
    float* logits;           // [B][V]
    float* part_v;           // [B][lm_head_batch_ctas]
    int* part_i;
    int* counter;            // zero between launches
    int32_t* out;            // [B][3]: {best value bits, best global row, isnan(logits[b][0])}
    int row_base;
    int* fallback_count;
    int force_fallback;
};

// reset_word (nullable): a word the kernel zeroes, the decode step's engine
// barrier, so that the step graph needs no memset node before the engine
cudaError_t launch_embed(const uint16_t* tok_embd, const int32_t* tok_seq, const int32_t* pos_ptr, int E, int V,
                         float* x, cudaStream_t st, unsigned* reset_word = nullptr);
int attention_max_ctx();
cudaError_t prepare_decode_kernels();
cudaError_t launch_attention(const AttnParams& p, int n_head, cudaStream_t st);
// The multi-token (chunk) forms, n tokens at positions pos[0..n): the f16
// embedding rows of tok_seq[base..base+n) into x [n][E]; RoPE + store of every
// token's K and V (p.q/k/v/out are the chunk's row-major [n][...] buffers);
// then attention for every (head, token) with the cache already holding the
// chunk (src/forward.c:684-726 per column).
cudaError_t launch_embed_rows(const uint16_t* tok_embd, const int32_t* tok_seq, int n, int E, int V, float* x,
                              cudaStream_t st);
// seq_stride: bytes from token t's caches to token t+1's (0: one sequence,
// the chunk's; a batch of sequences each with its own cache otherwise)
cudaError_t launch_chunk_kv_store(const AttnParams& p, const int32_t* pos, int n, int n_head_kv, int E, int G,
                                  cudaStream_t st, size_t seq_stride = 0);
cudaError_t launch_attention_chunk(const AttnParams& p, const int32_t* pos, int n, int n_head, int E, int G,
                                   cudaStream_t st, size_t seq_stride = 0);
// out[i] = a[i] + b[i] (the residual adds, src/forward.c:745-750, 796-801)
cudaError_t launch_add(const float* a, const float* b, float* out, size_t n, cudaStream_t st);
int lm_head_grid(int num_sms);
cudaError_t launch_lm_head(const LmParams& p, int grid, cudaStream_t st);
// CTAs per token group of the batch head (the per-token partials' length)
int lm_head_batch_ctas(int B, int num_sms);
cudaError_t launch_lm_head_batch(const LmBatchParams& p, int num_sms, cudaStream_t st);

}  // namespace sllm
