// gemv.cuh -- parameters of the fused I2_S GEMV (i2s_gemv.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/sllm_cuda.h"

namespace sllm {

enum GemvPrologue { PRO_Q8 = 0, PRO_QUANT = 1, PRO_NORM = 2 };
enum GemvEpilogue { EPI_DOTS = 0, EPI_F32 = 1, EPI_RESID = 2, EPI_SILU = 3 };

// One weight tensor of a launch. Up to three tensors that share the input
// activation (Q, K, V) run as one launch; EPI_SILU pairs row r of seg[0]
// (gate) with row r of seg[1] (up).
struct GemvSeg {
    const uint8_t* w;     // packed I2_S rows, scale tail after rows*K/4 bytes
    int rows;
    float* y;             // f32 outputs (nullable)
    int32_t* dots;        // raw int32 dots (nullable)
};

struct GemvParams {
    int K;                        // contracted width, multiple of 128, <= gemv_max_k()
    int nseg;
    GemvSeg seg[3];
    const float* x;               // PRO_QUANT / PRO_NORM input (K floats, 16-byte aligned)
    const float* norm_w;          // PRO_NORM weight (K floats, 16-byte aligned)
    float eps;
    const int8_t* q_in;           // PRO_Q8 input (K bytes, 16-byte aligned)
    const sllm_cuda_act* act_in;
    const float* resid;           // EPI_RESID: y = proj + resid
    float* h_out;                 // EPI_SILU: h = silu(gate) * up
    int8_t* q_out;                // nullable: the quantised activation (CTA 0 writes it)
    sllm_cuda_act* act_out;       // nullable
    int* fallback_count;          // nullable: counts reference-order RMSNorm sums
    int force_fallback;           // test hook: always take the reference-order sum
    double inv_k;                 // 1.0 / K, set by launch_gemv
};

// How a launch relates to the kernel before it in the stream:
//   GEMV_PLAIN        an ordinary launch
//   GEMV_DEPENDENT    programmatic dependent launch; the input vector is the
//                     previous kernel's output (waits before reading it)
//   GEMV_INDEPENDENT  programmatic dependent launch over an input nothing in
//                     flight writes (waits only before exiting)
enum GemvMode { GEMV_PLAIN = 0, GEMV_DEPENDENT = 1, GEMV_INDEPENDENT = 2 };

int gemv_max_k();
cudaError_t launch_gemv(const GemvParams& p, int pro, int epi, int num_sms, cudaStream_t st,
                        int mode = GEMV_PLAIN);
cudaError_t launch_quant_act(const float* x, int n, int8_t* q, sllm_cuda_act* act, cudaStream_t st);
// RMSNorm (certified, as the GEMV prologue) + quantisation of each row of a
// row-major [rows][K] batch; K % 128 == 0, K <= gemv_max_k()
cudaError_t launch_norm_quant_rows(const float* x, const float* w, int K, float eps, int rows, int8_t* q,
                                   sllm_cuda_act* acts, int* fb, int force, cudaStream_t st);
// rows independent vectors of a row-major [rows][n] batch, one block each
cudaError_t launch_quant_act_rows(const float* x, int rows, int n, int8_t* q, sllm_cuda_act* acts, cudaStream_t st);

}  // namespace sllm
