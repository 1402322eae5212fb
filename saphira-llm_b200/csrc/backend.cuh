// backend.cuh -- internals of backend.cu shared with tp.cu (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <vector>

#include "engine.cuh"

namespace sllm {

// record a failure for sllm_cuda_last_error and return `status`
int fail(int status, const char* fmt, ...);
// a CUDA error as an sllm status (NOMEM for allocation failures, else DEVICE)
int cuda_fail(cudaError_t e, const char* what);
int num_sms_of(int dev);
bool aligned16(const void* p);
// the reference's RoPE angle recurrence on the host libm, [n_ctx][n_rot / 2]
void rope_table(int n_ctx, int n_rot, float base, std::vector<float>& cs, std::vector<float>& sn);
// the per-process certified-sum fallback counter and the test switch
int* fallback_counter();
int force_fallback_flag();
// the per-device error word of the prefill GEMM's bounded waits
int* gemm_error_word();
// CUDA graphs whose kernel nodes are counted for sllm_cuda_test_kernel_launches
cudaError_t instantiate(cudaGraphExec_t* exec, cudaGraph_t g);
cudaError_t graph_launch(cudaGraphExec_t exec, cudaStream_t st);
void graph_exec_destroy(cudaGraphExec_t exec);
void count_launches(long long n);
// cudaMalloc for the model and context allocations, with the test hook that
// makes the next n of them fail (sllm_cuda_test_fail_next)
cudaError_t dev_malloc(void** p, size_t bytes);
// the test hook for communicator set-up: true when this one must fail
bool fail_next_comm_init();
// split every stage's rows over `grid` CTAs by weight bytes (engine programs)
std::vector<EngCursor> engine_starts(const std::vector<EngOp>& ops, const std::vector<int>& stage_first, int grid);

}  // namespace sllm

#define CK(call, what)                                              \
    do {                                                            \
        cudaError_t e_ = (call);                                    \
        if (e_ != cudaSuccess) return ::sllm::cuda_fail(e_, (what)); \
    } while (0)
