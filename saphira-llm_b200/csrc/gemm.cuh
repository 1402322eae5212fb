// gemm.cuh -- the multi-token I2_S GEMM on the tcgen05 tensor cores (i2s_gemm.cu).
//
// For every token m of a batch and every weight row r:
//   dots[m][r] = sum_k code[r][k] * q[m][k]            (int32, exact)
//   y[m][r]    = (float)(dots[m][r] - act[m].sum) * (ws / act[m].scale)
// which is, token by token, sllm_i2s_gemv + the forward pass's epilogue
// (src/i2s_gemm.c:260-269, src/forward.c:653-655). The gate/up form fuses
// h = silu(gate) * up (src/forward.c:756-779).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/sllm_cuda.h"

namespace sllm {

struct GemmArgs {
    const uint8_t* w;            // [n_rows][K/4] I2_S codes, scale tail after them
    const uint8_t* w2;           // gate/up: the up tensor (same shape), else null
    const int8_t* q;             // [m][K] int8 activations, row-major
    const sllm_cuda_act* acts;   // [m]
    int32_t* dots;               // [m][n_rows] or null (single tensor only)
    float* y;                    // [m][n_rows] or null; gate/up: h
    int m, n_rows, K;
    int lda;                     // bytes from one token's q row to the next (0: K); a multiple of 16
};

// 0 when the shapes are supported (K % 128 == 0, 16-byte aligned rows and
// pointers); a negative sllm status and a message otherwise
int gemm_check(const GemmArgs& a, const char** why);
cudaError_t launch_i2s_gemm(const GemmArgs& a, int* error, cudaStream_t st);
// the same results for at most 16 tokens (a.m <= 16), weight rows as the
// MMA's M operand and the tokens as its N = 16 operand
cudaError_t launch_i2s_gemm_skinny(const GemmArgs& a, int* error, cudaStream_t st);

// One tensor of a multi-tensor skinny launch: rows of w (and of w2, the up
// tensor of a gate/up pair: then y receives h = silu(gate) * up and every
// segment is a pair), contracted with activation columns [kx, kx + K) of q.
struct SkinnySeg {
    const uint8_t* w;
    const uint8_t* w2;
    int n_rows;
    int kx;                      // a multiple of 16
    int32_t* dots;               // [m][n_rows] or null
    float* y;                    // [m][n_rows] or null
};
// up to four segments sharing q (row stride lda bytes, 0: K), K and the
// token count m <= 16
cudaError_t launch_i2s_gemm_skinny_segs(const SkinnySeg* segs, int nseg, const int8_t* q, int lda, int m, int K,
                                        const sllm_cuda_act* acts, int* error, cudaStream_t st);
// test hook: 0 picks the form by size (skinny for m <= 16), 1 forces the
// 128-token tiles, 2 the skinny form
void gemm_set_form(int form);

}  // namespace sllm
