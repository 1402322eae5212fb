// tp.cu -- tensor-parallel decode across the GPUs of one node.
//
// Megatron-style shards of every layer, one process (or, for tests, one
// context) per rank r of N:
//   Q/K/V   rows of this rank's heads (H/N query heads, Hkv/N kv heads)
//   O       every row, columns [r E/N, (r+1) E/N) of the contraction
//   gate/up rows [r F/N, (r+1) F/N)
//   down    every row, columns [r F/N, (r+1) F/N), stored as C chunks of at
//           most 8192 columns each (a K range of an I2_S row is itself an
//           I2_S row, so every chunk is an ordinary packed tensor)
//   head    vocabulary rows [r V/N, (r+1) V/N) of the tied f16 table
// Per layer and token (src/forward.c:628-801 with the exchange points):
//   1. attn_norm + GEMV of the local Q/K/V rows, RoPE, KV append, attention
//      over the local heads                          -> all-gather (f32)
//   2. attn_sub_norm + quantisation of the whole attention output (every
//      rank, identical), partial int32 dots of O over the local columns
//                                                    -> all-reduce (int32 sum)
//   3. epilogue + residual, ffn_norm + GEMV of the local gate/up rows with
//      silu(gate) * up                               -> all-gather (f32)
//   4. ffn_sub_norm + quantisation of all of h, partial int32 dots of down
//                                                    -> all-reduce (int32 sum)
//   5. epilogue + residual
// The head: output_norm + the local vocabulary rows, the slice's argmax
// -> all-gather, then the first maximum over slices (src/forward.c:876-883).
//
// Exactness: the exchanged dots are integers, so their sum is the same in
// any order; every float operation happens identically on every rank or on
// the rank that owns the value, in the single-GPU kernels' order. So TP = N
// gives the bits of TP = 1, which gives the reference's.
//
// The exchanges are NCCL collectives on the context's stream, captured with
// the step's kernels into one CUDA graph. For tests on one GPU, a group of N
// contexts without a communicator runs the same phases and exchanges through
// device copies (sllm_cuda_test_tp_generate_group).

#include <chrono>
#include <dlfcn.h>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <type_traits>
#include <vector>

#include <nccl.h>
#include <cooperative_groups.h>

#include "backend.cuh"
#include "upload.cuh"
#include "common.cuh"
#include "decode.cuh"
#include "engine.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "../../include/sllm_cuda.h"
#include "../../include/sllm_cuda_testing.h"

using namespace sllm;

namespace {

// NCCL, resolved at the first tensor-parallel call: the process's own
// libnccl.so.2 when one is loaded already (a host that also runs a framework
// with its own NCCL keeps a single copy), else the system's. Nothing links
// against it, so the library loads where NCCL is absent.
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*comm_abort)(ncclComm_t);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    const char* (*error_string)(ncclResult_t);
};

const NcclApi* nccl() {
    static NcclApi api;
    static int state = 0;      // 0 untried, 1 loaded, -1 unavailable
    if (state != 0) return state > 0 ? &api : nullptr;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) { state = -1; return nullptr; }
    bool ok = true;
    auto sym = [&](auto& fn, const char* name) {
        fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
        ok = ok && fn != nullptr;
    };
    sym(api.get_unique_id, "ncclGetUniqueId");
    sym(api.comm_init_rank, "ncclCommInitRank");
    sym(api.comm_destroy, "ncclCommDestroy");
    sym(api.comm_abort, "ncclCommAbort");
    sym(api.all_gather, "ncclAllGather");
    sym(api.all_reduce, "ncclAllReduce");
    sym(api.error_string, "ncclGetErrorString");
    state = ok ? 1 : -1;
    return ok ? &api : nullptr;
}

const char* nccl_err(ncclResult_t r) { return nccl() ? nccl()->error_string(r) : "NCCL unavailable"; }

constexpr int kHeadDim = 128;
constexpr int kMaxChunkK = 8192;
constexpr int kNqThreads = 1024;
constexpr int kNqKpt = 7;                 // float4 per thread: K <= 28672
constexpr int kMaxRanks = 8;

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t gtimer_d() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}


// RMSNorm (certified mean, src/ops.c:254-322) + per-token int8 quantisation
// (src/i2s_gemm.c:45-83) of one vector, q in natural order, one CTA.
__global__ void __launch_bounds__(kNqThreads)
tp_norm_quant_kernel(const float* __restrict__ x, const float* __restrict__ w, int K, float eps, double inv_k,
                     int8_t* __restrict__ q, sllm_cuda_act* act, int* fb, int force) {
    __shared__ double dred[32];
    __shared__ float fred[32];
    __shared__ int ired[32];
    __shared__ float s_bcast;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // as the cluster form
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int K4 = K >> 2;
    float4 xv[kNqKpt];
    #pragma unroll
    for (int j = 0; j < kNqKpt; ++j) {
        const int i = tid + j * kNqThreads;
        xv[j] = i < K4 ? reinterpret_cast<const float4*>(x)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    #pragma unroll
    for (int j = 0; j < kNqKpt; ++j) {
        s0 = __dadd_rn(s0, (double)__fmul_rn(xv[j].x, xv[j].x));
        s1 = __dadd_rn(s1, (double)__fmul_rn(xv[j].y, xv[j].y));
        s2 = __dadd_rn(s2, (double)__fmul_rn(xv[j].z, xv[j].z));
        s3 = __dadd_rn(s3, (double)__fmul_rn(xv[j].w, xv[j].w));
    }
    double ss = warp_sum_d(__dadd_rn(__dadd_rn(s0, s1), __dadd_rn(s2, s3)));
    if (lane == 0) dred[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        double S = 0.0;
        for (int i = 0; i < kNqThreads / 32; ++i) S = __dadd_rn(S, dred[i]);
        float mean;
        if (!certify_mean_mul(S, K, inv_k, &mean) || force) {
            mean = __double2float_rn(__ddiv_rn(rms_ss_reference_order(x, K), (double)K));
            if (fb != nullptr) atomicAdd(fb, 1);
        }
        s_bcast = rms_scale(mean, eps);
    }
    __syncthreads();
    const float sc = s_bcast;
    float amax = 0.0f;
    #pragma unroll
    for (int j = 0; j < kNqKpt; ++j) {
        const int i = tid + j * kNqThreads;
        // the norm weight is read here, not held across the reduction (registers)
        const float4 wv = i < K4 ? __ldg(reinterpret_cast<const float4*>(w) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        xv[j].x = __fmul_rn(__fmul_rn(sc, xv[j].x), wv.x);
        xv[j].y = __fmul_rn(__fmul_rn(sc, xv[j].y), wv.y);
        xv[j].z = __fmul_rn(__fmul_rn(sc, xv[j].z), wv.z);
        xv[j].w = __fmul_rn(__fmul_rn(sc, xv[j].w), wv.w);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(xv[j].x), fabsf(xv[j].y)), fmaxf(fabsf(xv[j].z), fabsf(xv[j].w))));
    }
    amax = warp_max(amax);
    __syncthreads();
    if (lane == 0) fred[warp] = amax;
    __syncthreads();
    if (tid == 0) {
        float m = 0.0f;
        for (int i = 0; i < kNqThreads / 32; ++i) m = fmaxf(m, fred[i]);
        s_bcast = quant_scale(m);
    }
    __syncthreads();
    const float s = s_bcast;
    int sum = 0;
    #pragma unroll
    for (int j = 0; j < kNqKpt; ++j) {
        const int i = tid + j * kNqThreads;
        if (i < K4) {
            const int a = quant_one(xv[j].x, s), b = quant_one(xv[j].y, s);
            const int c = quant_one(xv[j].z, s), d = quant_one(xv[j].w, s);
            sum += (a + b) + (c + d);
            reinterpret_cast<uint32_t*>(q)[i] = (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) |
                                                ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
        }
    }
    sum = __reduce_add_sync(0xffffffffu, sum);
    if (lane == 0) ired[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        int total = 0;
        for (int i = 0; i < kNqThreads / 32; ++i) total += ired[i];
        act->scale = s;
        act->sum = total;
    }
}

// The same RMSNorm + quantisation on a cluster of eight CTAs: each CTA holds
// one eighth of the vector (one float4 per thread, K % 32 == 0, K <= 32768),
// and the three reductions (the f64 sum of squares, the absmax, the code sum)
// pass per-CTA partials through distributed shared memory behind cluster
// barriers. The results are the single CTA's: the sum is certified for any
// order, max and the integer sum do not depend on it. Every CTA runs the same
// straight-line code, so each one reaches every cluster barrier.
constexpr int kNqCluster = 8;

// A kernel's wait for an exchange every rank published (the fused peer
// exchange): flag[kind][r] of this rank's region reaching steps * n_layer +
// layer + 1 for every rank r, bounded; flags == nullptr: no wait.
struct XWait {
    const uint32_t* flags;     // this rank's flags of the kind: [kMaxRanks]
    const uint32_t* steps;
    int n_peer, n_layer, layer;
    int* error;                // set when the wait gave up
};
constexpr uint64_t kXWaitNs = 10000000000ull;     // 10 s: a peer may still be launching

__device__ __forceinline__ void xwait_block(const XWait& w) {
    if (w.flags == nullptr) return;
    if (threadIdx.x == 0) {
        const uint32_t val = *(volatile const uint32_t*)w.steps * (uint32_t)w.n_layer + (uint32_t)w.layer + 1u;
        const uint64_t t0 = gtimer_d();
        for (int q = 0; q < w.n_peer; ++q) {
            uint32_t f;
            while (true) {
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(w.flags + q) : "memory");
                if (f >= val) break;
                if (gtimer_d() - t0 > kXWaitNs || *(volatile const int*)w.error != 0) {
                    atomicExch(w.error, ENG_TIMEOUT_PEER);
                    q = w.n_peer;
                    break;
                }
                __nanosleep(64);
            }
        }
    }
    __syncthreads();
}

__global__ void __cluster_dims__(kNqCluster, 1, 1) __launch_bounds__(kNqThreads)
tp_norm_quant_cluster_kernel(const float* __restrict__ x, const float* __restrict__ w, int K, float eps,
                             double inv_k, int8_t* __restrict__ q, sllm_cuda_act* act, int* fb, int force,
                             XWait xw) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    __shared__ double dred[32];
    __shared__ float fred[32];
    __shared__ int ired[32];
    __shared__ double c_ss;          // this CTA's partials, read by the whole cluster
    __shared__ float c_amax;
    __shared__ int c_sum;
    __shared__ float s_bcast;
    const int rank = (int)cl.block_rank();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // several clusters: one row each of a row-major [rows][K] batch
    {
        const int row = blockIdx.x / kNqCluster;
        x += (size_t)row * K;
        q += (size_t)row * K;
        act += row;
    }
    // programmatic dependent launch: the next launch (the down program, whose
    // consumers wait for this one) may be scheduled now, and x comes from the
    // previous launch
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    xwait_block(xw);     // x gathered from every rank's stores (the fused peer exchange)
    const int per = (K >> 2) / kNqCluster;                 // float4 per CTA
    const int i = rank * per + tid;
    const bool live = tid < per;
    float4 xv = live ? reinterpret_cast<const float4*>(x)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    double ss = __dadd_rn(__dadd_rn((double)__fmul_rn(xv.x, xv.x), (double)__fmul_rn(xv.y, xv.y)),
                          __dadd_rn((double)__fmul_rn(xv.z, xv.z), (double)__fmul_rn(xv.w, xv.w)));
    ss = warp_sum_d(ss);
    if (lane == 0) dred[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        double S = 0.0;
        for (int k = 0; k < kNqThreads / 32; ++k) S = __dadd_rn(S, dred[k]);
        c_ss = S;
    }
    cl.sync();
    if (tid == 0) {
        double S = 0.0;
        for (int r = 0; r < kNqCluster; ++r) S = __dadd_rn(S, *cl.map_shared_rank(&c_ss, r));
        float mean;
        if (!certify_mean_mul(S, K, inv_k, &mean) || force) {
            // every CTA re-sums in the reference's order and gets the same mean
            mean = __double2float_rn(__ddiv_rn(rms_ss_reference_order(x, K), (double)K));
            if (fb != nullptr && rank == 0) atomicAdd(fb, 1);
        }
        s_bcast = rms_scale(mean, eps);
    }
    __syncthreads();
    const float sc = s_bcast;
    const float4 wv = live ? __ldg(reinterpret_cast<const float4*>(w) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    xv.x = __fmul_rn(__fmul_rn(sc, xv.x), wv.x);
    xv.y = __fmul_rn(__fmul_rn(sc, xv.y), wv.y);
    xv.z = __fmul_rn(__fmul_rn(sc, xv.z), wv.z);
    xv.w = __fmul_rn(__fmul_rn(sc, xv.w), wv.w);
    float amax = fmaxf(fmaxf(fabsf(xv.x), fabsf(xv.y)), fmaxf(fabsf(xv.z), fabsf(xv.w)));
    amax = warp_max(amax);
    if (lane == 0) fred[warp] = amax;
    __syncthreads();
    if (tid == 0) {
        float m = 0.0f;
        for (int k = 0; k < kNqThreads / 32; ++k) m = fmaxf(m, fred[k]);
        c_amax = m;
    }
    cl.sync();
    if (tid == 0) {
        float m = 0.0f;
        for (int r = 0; r < kNqCluster; ++r) m = fmaxf(m, *cl.map_shared_rank(&c_amax, r));
        s_bcast = quant_scale(m);
    }
    __syncthreads();
    const float s = s_bcast;
    int sum = 0;
    if (live) {
        const int a = quant_one(xv.x, s), b = quant_one(xv.y, s);
        const int c = quant_one(xv.z, s), d = quant_one(xv.w, s);
        sum = (a + b) + (c + d);
        reinterpret_cast<uint32_t*>(q)[i] = (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) |
                                            ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
    }
    sum = __reduce_add_sync(0xffffffffu, sum);
    if (lane == 0) ired[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        int t = 0;
        for (int k = 0; k < kNqThreads / 32; ++k) t += ired[k];
        c_sum = t;
    }
    cl.sync();
    if (rank == 0 && tid == 0) {
        int total = 0;
        for (int r = 0; r < kNqCluster; ++r) total += *cl.map_shared_rank(&c_sum, r);
        act->scale = s;
        act->sum = total;
    }
    cl.sync();      // no CTA leaves while rank 0 may still read its shared memory
}

// The batch form of the whole-row norm + quantisation, one cluster per row
// of a [rows][K] batch (the h rows before down) after an all-gather, reading
// the row straight from the gather's rank-major layout
// x[b][j] = g[(j / c) B c + b c + j % c] while also writing the whole row to
// out, so the unshard copy is not a launch of its own. The reference-order
// fallback reads the row back from out after a cluster barrier (every CTA's
// slice written). (Folding the O and down epilogues in as well measured
// slower at 8192-wide rows than the separate epilogue and one-CTA norm.)
enum RowSrcMode { RS_GATHER = 2 };

struct RowSrc {
    const float* g;                 // RS_GATHER: [N][rows][c]
    int c;
    int rows;
    float* out;                     // RS_GATHER: [rows][K]
};

template <int MODE>
__global__ void __cluster_dims__(kNqCluster, 1, 1) __launch_bounds__(kNqThreads)
tp_rows_norm_quant_kernel(const RowSrc src, const float* __restrict__ w, int K, float eps, double inv_k,
                          int8_t* __restrict__ q, sllm_cuda_act* act, int* fb, int force) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    __shared__ double dred[32];
    __shared__ float fred[32];
    __shared__ int ired[32];
    __shared__ double c_ss;
    __shared__ float c_amax;
    __shared__ int c_sum;
    __shared__ float s_bcast;
    const int rank = (int)cl.block_rank();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row = blockIdx.x / kNqCluster;
    q += (size_t)row * K;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int per = (K >> 2) / kNqCluster;                 // float4 per CTA
    const int i = rank * per + tid;
    const bool live = tid < per;
    float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* xrow = src.out + (size_t)row * K;
    if (live) {
        // element j = 4 i of the row lies in rank j / c's slice (c % 4 == 0)
        const int j = 4 * i, r = j / src.c, jj = j - r * src.c;
        xv = *reinterpret_cast<const float4*>(src.g + ((size_t)r * src.rows + row) * src.c + jj);
        *reinterpret_cast<float4*>(src.out + (size_t)row * K + j) = xv;
    }
    double ss = __dadd_rn(__dadd_rn((double)__fmul_rn(xv.x, xv.x), (double)__fmul_rn(xv.y, xv.y)),
                          __dadd_rn((double)__fmul_rn(xv.z, xv.z), (double)__fmul_rn(xv.w, xv.w)));
    ss = warp_sum_d(ss);
    if (lane == 0) dred[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        double S = 0.0;
        for (int k = 0; k < kNqThreads / 32; ++k) S = __dadd_rn(S, dred[k]);
        c_ss = S;
    }
    cl.sync();      // also: every CTA's slice of out is written
    if (tid == 0) {
        double S = 0.0;
        for (int r = 0; r < kNqCluster; ++r) S = __dadd_rn(S, *cl.map_shared_rank(&c_ss, r));
        float mean;
        if (!certify_mean_mul(S, K, inv_k, &mean) || force) {
            mean = __double2float_rn(__ddiv_rn(rms_ss_reference_order(xrow, K), (double)K));
            if (fb != nullptr && rank == 0) atomicAdd(fb, 1);
        }
        s_bcast = rms_scale(mean, eps);
    }
    __syncthreads();
    const float sc = s_bcast;
    const float4 wv = live ? __ldg(reinterpret_cast<const float4*>(w) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    xv.x = __fmul_rn(__fmul_rn(sc, xv.x), wv.x);
    xv.y = __fmul_rn(__fmul_rn(sc, xv.y), wv.y);
    xv.z = __fmul_rn(__fmul_rn(sc, xv.z), wv.z);
    xv.w = __fmul_rn(__fmul_rn(sc, xv.w), wv.w);
    float amax = fmaxf(fmaxf(fabsf(xv.x), fabsf(xv.y)), fmaxf(fabsf(xv.z), fabsf(xv.w)));
    amax = warp_max(amax);
    if (lane == 0) fred[warp] = amax;
    __syncthreads();
    if (tid == 0) {
        float m = 0.0f;
        for (int k = 0; k < kNqThreads / 32; ++k) m = fmaxf(m, fred[k]);
        c_amax = m;
    }
    cl.sync();
    if (tid == 0) {
        float m = 0.0f;
        for (int r = 0; r < kNqCluster; ++r) m = fmaxf(m, *cl.map_shared_rank(&c_amax, r));
        s_bcast = quant_scale(m);
    }
    __syncthreads();
    const float s = s_bcast;
    int sum = 0;
    if (live) {
        const int a = quant_one(xv.x, s), b = quant_one(xv.y, s);
        const int c = quant_one(xv.z, s), d = quant_one(xv.w, s);
        sum = (a + b) + (c + d);
        reinterpret_cast<uint32_t*>(q)[i] = (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) |
                                            ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
    }
    sum = __reduce_add_sync(0xffffffffu, sum);
    if (lane == 0) ired[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        int t = 0;
        for (int k = 0; k < kNqThreads / 32; ++k) t += ired[k];
        c_sum = t;
    }
    cl.sync();
    if (rank == 0 && tid == 0) {
        int total = 0;
        for (int r = 0; r < kNqCluster; ++r) total += *cl.map_shared_rank(&c_sum, r);
        act[row].scale = s;
        act[row].sum = total;
    }
    cl.sync();      // no CTA leaves while rank 0 may still read its shared memory
}

// y[r] = (float)(sum over chunks of dots - act.sum) * (ws / act.scale) + resid[r]
// (src/forward.c:739-750, 790-801)
__global__ void tp_epilogue_kernel(const int32_t* __restrict__ dots, int n_chunks, int rows, const sllm_cuda_act* act,
                                   const float* __restrict__ ws, const float* __restrict__ resid, float* __restrict__ y) {
    asm volatile("griddepcontrol.wait;" ::: "memory");      // the dots come from the previous launch
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    int d = 0;
    for (int c = 0; c < n_chunks; ++c) d += dots[(size_t)c * rows + r];
    const sllm_cuda_act a = *act;
    const float post = __fdiv_rn(*ws, a.scale);
    y[r] = __fadd_rn(__fmul_rn(__int2float_rn(d - a.sum), post), resid[r]);
}

// The same epilogue over every rank's slots of a contraction split over ranks
// and column chunks, once the exchange that filled them is complete
// (the fused peer exchange; the step's last down projection).
__global__ void tp_xreduce_kernel(XWait xw, const int32_t* __restrict__ slots, int n_slots, int rows,
                                  const sllm_cuda_act* act, const float* __restrict__ ws,
                                  const float* __restrict__ resid, float* __restrict__ y) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    xwait_block(xw);
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    int d = 0;
    for (int c = 0; c < n_slots; ++c) d += __ldcg(slots + (size_t)c * rows + r);
    const sllm_cuda_act a = *act;
    const float post = __fdiv_rn(*ws, a.scale);
    y[r] = __fadd_rn(__fmul_rn(__int2float_rn(d - a.sum), post), resid[r]);
}

// first maximum over the slices' bests, in rank (= row) order, then the
// greedy feedback and position advance of the step (as lm_head_kernel)
__device__ __forceinline__ bool tp_better(float v, int i, float bv, int bi) {
    if (isnan(v)) return false;
    if (isnan(bv)) return true;
    return v > bv || (v == bv && i < bi);
}

__global__ void tp_finalize_kernel(const int32_t* trip_all, int n_ranks, int32_t* pos_ptr, int32_t* tok_seq,
                                   const int32_t* prompt_end, int32_t* argmax_out, int32_t* hist, int n_ctx,
                                   uint32_t* steps) {
    float bv = NAN;
    int bi = 0x7fffffff;
    for (int r = 0; r < n_ranks; ++r) {
        const float v = __int_as_float(trip_all[3 * r]);
        const int i = trip_all[3 * r + 1];
        if (i != 0x7fffffff && tp_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    int next = bi;
    if (bi == 0x7fffffff || trip_all[2] != 0) next = 0;   // rank 0 holds row 0
    *argmax_out = next;
    const int pos = *pos_ptr;
    if (pos + 1 >= *prompt_end && pos + 1 < n_ctx) tok_seq[pos + 1] = next;
    if (hist != nullptr) hist[pos] = next;
    *pos_ptr = pos + 1;
    if (steps != nullptr) *steps += 1u;      // the fused exchange's flag values move on
}

// element-wise int32 sum of up to kMaxRanks buffers into each of them (the
// all-reduce of a one-process group)
struct SumArgs {
    int32_t* buf[kMaxRanks];
    int n;
    size_t count;
};
__global__ void tp_group_sum_kernel(const __grid_constant__ SumArgs a) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < a.count; i += (size_t)gridDim.x * blockDim.x) {
        int s = 0;
        for (int r = 0; r < a.n; ++r) s += a.buf[r][i];
        for (int r = 0; r < a.n; ++r) a.buf[r][i] = s;
    }
}

// --- the one-shot peer exchange ----------------------------------------------
// One CTA per rank and exchange: store this rank's `count` words into slot
// `rank` of the destination area in every rank's region (plain stores over
// NVLink to the peers' mapped regions), publish them (system fence, then a
// release store of the exchange's epoch into flag[rank] of every region),
// wait until every rank's flag in this region reaches the epoch (acquire,
// bounded by the global timer), then read the area through L2: a gather
// copies the N slots to `dst`, a reduction sums them (int32, exact in any
// order) into `dst`.
constexpr uint64_t kXchgWaitNs = 10000000000ull;     // 10 s: a peer may still be setting up

struct XParams {
    char* peer[kMaxRanks];      // every rank's region; peer[rank] is this rank's
    const uint32_t* src;
    uint32_t* dst;
    size_t off;                 // the destination area's offset in every region
    size_t off_flags;
    uint32_t count;             // words per rank
    int n, rank;
    int reduce;                 // 0: gather (dst = [N][count]), 1: int32 sum (dst = [count])
    uint32_t* epoch;            // this rank's exchange counter (device)
    int* error;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(1024) tp_exchange_kernel(const __grid_constant__ XParams x) {
    __shared__ int s_ok;
    const int tid = threadIdx.x;
    const uint32_t epoch = *x.epoch + 1;
    // 16-byte stores (count is a multiple of 4 for every exchange but the
    // 3-word argmax triple, which goes word by word)
    const uint32_t n4 = (x.count % 4 == 0) ? x.count / 4 : 0;
    for (int p = 0; p < x.n; ++p) {
        uint32_t* d = reinterpret_cast<uint32_t*>(x.peer[p] + x.off) + (size_t)x.rank * x.count;
        if (n4 > 0) {
            const uint4* s4 = reinterpret_cast<const uint4*>(x.src);
            uint4* d4 = reinterpret_cast<uint4*>(d);
            for (uint32_t i = tid; i < n4; i += blockDim.x) d4[i] = s4[i];
        } else {
            for (uint32_t i = tid; i < x.count; i += blockDim.x) d[i] = x.src[i];
        }
    }
    // the barrier orders every thread's stores before the flag stores; a
    // release store at system scope is cumulative over them
    __syncthreads();
    if (tid < x.n) st_release_sys(reinterpret_cast<uint32_t*>(x.peer[tid] + x.off_flags) + x.rank, epoch);
    if (tid == 0) s_ok = 1;
    __syncthreads();
    if (tid < x.n) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(x.peer[x.rank] + x.off_flags) + tid;
        const uint64_t t0 = gtimer_d();
        while (ld_acquire_sys(f) < epoch) {
            if (gtimer_d() - t0 > kXchgWaitNs) {
                s_ok = 0;
                atomicExch(x.error, 1);
                break;
            }
        }
    }
    __syncthreads();
    if (!s_ok) return;
    const uint32_t* area = reinterpret_cast<const uint32_t*>(x.peer[x.rank] + x.off);
    if (x.reduce) {
        for (uint32_t i = tid; i < x.count; i += blockDim.x) {
            int sum = 0;
            for (int r = 0; r < x.n; ++r) sum += (int)__ldcg(area + (size_t)r * x.count + i);
            x.dst[i] = (uint32_t)sum;
        }
    } else {
        for (uint32_t i = tid; i < x.n * x.count; i += blockDim.x) x.dst[i] = __ldcg(area + i);
    }
    if (tid == 0) *x.epoch = epoch;
}

// --- seeded synthetic weights, generated on the device -----------------------
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__host__ __device__ __forceinline__ uint64_t tensor_key(uint64_t seed, int layer, int tensor) {
    return splitmix64(seed ^ splitmix64(((uint64_t)(layer + 1) << 8) | (uint64_t)tensor));
}

// ternary code {0, 1, 2} (= t + 1) of element (row, col) of a tensor, each
// value with probability 1/3 up to 2^-32
__device__ __forceinline__ uint32_t synth_code(uint64_t key, int row, int col) {
    const uint64_t h = splitmix64(key + (((uint64_t)row << 20) | (uint64_t)col));
    return (uint32_t)(((h >> 32) * 3ull) >> 32);
}

__host__ __device__ __forceinline__ float synth_scale(uint64_t key) {
    return 0.01f + 0.09f * (float)(splitmix64(key ^ 0x5CA1Eull) >> 40) * (1.0f / 16777216.0f);
}

// rows [row0, row0 + rows) and columns [col0, col0 + cols) of a ternary
// tensor, packed as I2_S (element 32f + l of a 128-block in byte l at shift
// 6 - 2f), scale tail after the rows
__global__ void tp_gen_i2s_kernel(uint8_t* out, uint64_t key, int row0, int rows, int col0, int cols) {
    const size_t rb = (size_t)cols / 4, total = (size_t)rows * rb;
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < total; b += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(b / rb);
        const int j = (int)(b % rb);
        const int blk = j >> 5, l = j & 31;
        uint32_t byte = 0;
        #pragma unroll
        for (int f = 0; f < 4; ++f)
            byte |= synth_code(key, row0 + r, col0 + blk * 128 + 32 * f + l) << (6 - 2 * f);
        out[b] = (uint8_t)byte;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        float* tail = reinterpret_cast<float*>(out + total);
        tail[0] = synth_scale(key);
        for (int i = 1; i < 8; ++i) tail[i] = 0.0f;
    }
}

__device__ __forceinline__ float synth_normal(uint64_t key, int i) {
    const uint64_t h = splitmix64(key + (uint64_t)i);
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)((h >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.283185307f * u2);
}

__global__ void tp_gen_norm_kernel(float* out, uint64_t key, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = 1.0f + 0.02f * synth_normal(key, i);
}

__global__ void tp_gen_embd_kernel(uint16_t* out, uint64_t key, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __half_as_ushort(__float2half_rn(0.02f * synth_normal(key, (int)(i & 0x7fffffff)) ));
}

// ---------------------------------------------------------------------------
// host structures
// ---------------------------------------------------------------------------
struct TpLayer {
    const uint8_t *wq, *wk, *wv, *wo, *gate, *up;
    std::vector<const uint8_t*> down;       // chunks of down_k columns
    const float *attn_norm, *attn_sub_norm, *ffn_norm, *ffn_sub_norm;
};

int down_chunks(int f_loc) {
    int c = (f_loc + kMaxChunkK - 1) / kMaxChunkK;
    while (f_loc % (c * 128) != 0) ++c;
    return c;
}

size_t i2s_bytes(int rows, int cols) { return (size_t)rows * (size_t)cols / 4 + 32; }
size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

}  // namespace

struct sllm_cuda_tp_model {
    int device = 0, n_ranks = 1, rank = 0;
    int n_layer = 0, E = 0, F = 0, H = 0, Hkv = 0, V = 0;
    int hq = 0, hk = 0, e_loc = 0, f_loc = 0, down_c = 1, down_k = 0, v0 = 0, v_loc = 0;
    float eps = 1e-5f, rope_base = 500000.0f;
    uint8_t* blob = nullptr;
    size_t blob_bytes = 0;
    std::vector<TpLayer> layers;
    const uint16_t* tok_embd = nullptr;     // [V][E], every rank
    const float* output_norm = nullptr;
};

struct sllm_cuda_tp_comm {
    ncclComm_t comm = nullptr;
    int n_ranks = 1, rank = 0, device = 0;
};

struct sllm_cuda_tp_ctx {
    const sllm_cuda_tp_model* m = nullptr;
    sllm_cuda_tp_comm* comm = nullptr;
    int n_ctx = 0, n_past = 0, lm_grid = 0;
    bool have_logits = false;
    cudaStream_t stream = nullptr;
    float *k_cache = nullptr, *v_cache = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    float *x = nullptr, *ffn_inp = nullptr, *q = nullptr, *k = nullptr, *v = nullptr;
    float *attn_loc = nullptr, *attn_full = nullptr, *h_loc = nullptr, *h_full = nullptr, *logits = nullptr;
    int8_t *qa = nullptr, *qh = nullptr;
    sllm_cuda_act *act_a = nullptr, *act_h = nullptr;
    int32_t *dots_o = nullptr, *dots_d = nullptr;
    float* part_v = nullptr;
    int* part_i = nullptr;
    int* counter = nullptr;
    int32_t *trip = nullptr, *trip_all = nullptr, *argmax = nullptr, *pos = nullptr, *prompt_end = nullptr;
    int32_t *tok_seq = nullptr, *hist = nullptr;
    int32_t* pinned = nullptr;
    cudaGraphExec_t step = nullptr;
    std::vector<void*> allocs;
    // the layer GEMVs on the persistent engine: [layer][phase] programs
    // (Q/K/V, O partial dots, gate/up, down partial dots); empty when the
    // model's widths have no compiled engine instance (per-GEMV kernels then)
    struct Prog {
        EngParams p;
        int wa, wb;
    };
    std::vector<Prog> progs;
    // one rank: per layer one four-stage program (Q/K/V, attention, O +
    // residual, gate/up) behind grid barriers, in place of phases 0-2, their
    // two norm/quantise and epilogue kernels and the local copies; each has
    // its own barrier word, all zeroed once per step
    std::vector<Prog> fused;
    unsigned* fused_barriers = nullptr;
    int grid = 0;
    int* eng_error = nullptr;
    unsigned* eng_barrier = nullptr;
    // the one-shot peer exchange (n_ranks > 1): a receive region on this
    // device that every rank stores into, the peers' regions mapped here
    bool p2p = false;
    char* region = nullptr;
    char* peer[kMaxRanks] = {};
    size_t off_flags = 0, off_attn = 0, off_h = 0, off_dots_o = 0, off_dots_d = 0, off_trip = 0;
    uint32_t* epoch = nullptr;
    int* x_error = nullptr;
    // the fused peer exchange (more than one rank over peer memory, widths
    // with an exchanging engine instance): per layer one program A (the
    // reduce of the previous layer's down, Q/K/V, attention, O's partial
    // dots, their reduce, gate/up) and one program D (down's partial dots),
    // with the norm/quantisation of h between them; every exchange is stores
    // into every rank's region plus flags, inside those launches
    std::vector<Prog> xa, xd;
    unsigned* x_barriers = nullptr;   // one grid barrier word per A program
    unsigned* x_done = nullptr;       // end-of-kernel arrival counter of the A and D programs
    uint32_t* x_steps = nullptr;      // steps completed: the flag values
    size_t off_xflags = 0;            // flags [kind][kMaxRanks] in every region
    // recorded on `stream` around the step launches of the last generate call
    cudaEvent_t run_ev[2] = {};
};

namespace {

// ---------------------------------------------------------------------------
// model construction
// ---------------------------------------------------------------------------
int check_geometry(int n_layer, int E, int F, int H, int Hkv, int V, int n_ranks, int rank) {
    if (n_layer < 1 || E < 128 || F < 128 || H < 1 || Hkv < 1 || V < 1 || n_ranks < 1 || n_ranks > kMaxRanks ||
        rank < 0 || rank >= n_ranks)
        return fail(SLLM_CUDA_ERR_ARG, "tp: bad model geometry or rank");
    if (E != H * kHeadDim || H % Hkv != 0) return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp: head dim must be 128");
    if (H % n_ranks != 0 || Hkv % n_ranks != 0)
        return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp: %d ranks do not divide %d q / %d kv heads", n_ranks, H, Hkv);
    if ((E / n_ranks) % 128 != 0 || (F / n_ranks) % 128 != 0)
        return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp: E/N and F/N must be multiples of 128");
    if (E > kMaxChunkK) return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp: n_embd above %d", kMaxChunkK);
    if (F > kNqThreads * kNqKpt * 4) return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp: n_ff above %d", kNqThreads * kNqKpt * 4);
    return SLLM_CUDA_OK;
}

void fill_geometry(sllm_cuda_tp_model* m, int n_layer, int E, int F, int H, int Hkv, int V, int n_ranks, int rank) {
    m->n_layer = n_layer; m->E = E; m->F = F; m->H = H; m->Hkv = Hkv; m->V = V;
    m->n_ranks = n_ranks; m->rank = rank;
    m->hq = H / n_ranks; m->hk = Hkv / n_ranks;
    m->e_loc = E / n_ranks; m->f_loc = F / n_ranks;
    m->down_c = down_chunks(m->f_loc);
    m->down_k = m->f_loc / m->down_c;
    const int vs = (V + n_ranks - 1) / n_ranks;
    m->v0 = rank * vs < V ? rank * vs : V;
    m->v_loc = (m->v0 + vs < V ? m->v0 + vs : V) - m->v0;
}

// device byte offsets of every tensor of the shard, in one blob
struct Layout {
    std::vector<size_t> off;
    size_t total = 0;
    size_t add(size_t bytes) {
        off.push_back(total);
        total += align256(bytes);
        return off.back();
    }
};

// order per layer: wq, wk, wv, wo, gate, up, down[C], 4 norms; then embd, output_norm
Layout shard_layout(const sllm_cuda_tp_model* m) {
    Layout L;
    const int D = kHeadDim;
    for (int l = 0; l < m->n_layer; ++l) {
        L.add(i2s_bytes(m->hq * D, m->E));
        L.add(i2s_bytes(m->hk * D, m->E));
        L.add(i2s_bytes(m->hk * D, m->E));
        L.add(i2s_bytes(m->E, m->e_loc));
        L.add(i2s_bytes(m->f_loc, m->E));
        L.add(i2s_bytes(m->f_loc, m->E));
        for (int c = 0; c < m->down_c; ++c) L.add(i2s_bytes(m->E, m->down_k));
        L.add((size_t)m->E * 4);
        L.add((size_t)m->E * 4);
        L.add((size_t)m->E * 4);
        L.add((size_t)m->F * 4);
    }
    L.add((size_t)m->V * m->E * 2);
    L.add((size_t)m->E * 4);
    return L;
}

void bind_pointers(sllm_cuda_tp_model* m, const Layout& L) {
    size_t i = 0;
    auto P = [&](void) { return m->blob + L.off[i++]; };
    m->layers.resize(m->n_layer);
    for (int l = 0; l < m->n_layer; ++l) {
        TpLayer& t = m->layers[l];
        t.wq = P(); t.wk = P(); t.wv = P(); t.wo = P(); t.gate = P(); t.up = P();
        t.down.resize(m->down_c);
        for (int c = 0; c < m->down_c; ++c) t.down[c] = P();
        t.attn_norm = reinterpret_cast<const float*>(P());
        t.attn_sub_norm = reinterpret_cast<const float*>(P());
        t.ffn_norm = reinterpret_cast<const float*>(P());
        t.ffn_sub_norm = reinterpret_cast<const float*>(P());
    }
    m->tok_embd = reinterpret_cast<const uint16_t*>(P());
    m->output_norm = reinterpret_cast<const float*>(P());
}

// host tensor rows [r0, r0 + rows) x columns [c0, c0 + cols) of an I2_S
// tensor of `ncols` columns, with its scale tail, into a packed buffer
void slice_i2s(const uint8_t* src, int src_rows, int ncols, int r0, int rows, int c0, int cols, std::vector<uint8_t>& out) {
    const size_t srb = (size_t)ncols / 4, drb = (size_t)cols / 4;
    out.assign(i2s_bytes(rows, cols), 0);
    for (int r = 0; r < rows; ++r) memcpy(out.data() + (size_t)r * drb, src + (size_t)(r0 + r) * srb + c0 / 4, drb);
    memcpy(out.data() + (size_t)rows * drb, src + (size_t)src_rows * srb, 4);
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" int sllm_cuda_tp_unique_id(uint8_t* id_out) {
    if (id_out == nullptr) return fail(SLLM_CUDA_ERR_ARG, "tp_unique_id: null");
    if (nccl() == nullptr) return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp_unique_id: libnccl.so.2 not found");
    ncclUniqueId id;
    if (nccl()->get_unique_id(&id) != ncclSuccess) return fail(SLLM_CUDA_ERR_COMM, "ncclGetUniqueId failed");
    static_assert(sizeof(id) == SLLM_CUDA_TP_ID_BYTES, "NCCL unique id size");
    memcpy(id_out, &id, sizeof(id));
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_tp_comm_init(const uint8_t* id, int32_t n_ranks, int32_t rank, int32_t device,
                                      sllm_cuda_tp_comm** out) {
    if (id == nullptr || out == nullptr || n_ranks < 1 || n_ranks > kMaxRanks || rank < 0 || rank >= n_ranks)
        return fail(SLLM_CUDA_ERR_ARG, "tp_comm_init: bad arguments");
    *out = nullptr;
    if (nccl() == nullptr) return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp_comm_init: libnccl.so.2 not found");
    if (fail_next_comm_init()) return fail(SLLM_CUDA_ERR_COMM, "ncclCommInitRank: refused (injected by a test)");
    CK(cudaSetDevice(device), "cudaSetDevice");
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    auto* c = new sllm_cuda_tp_comm();
    c->n_ranks = n_ranks; c->rank = rank; c->device = device;
    const ncclResult_t r = nccl()->comm_init_rank(&c->comm, n_ranks, uid, rank);
    if (r != ncclSuccess) {
        delete c;
        return fail(SLLM_CUDA_ERR_COMM, "ncclCommInitRank: %s", nccl_err(r));
    }
    *out = c;
    return SLLM_CUDA_OK;
}

extern "C" void sllm_cuda_tp_comm_free(sllm_cuda_tp_comm* c) {
    if (c == nullptr) return;
    cudaSetDevice(c->device);
    if (c->comm != nullptr && nccl() != nullptr) nccl()->comm_destroy(c->comm);
    delete c;
}

extern "C" int sllm_cuda_test_tp_plan(int32_t n_layer, int32_t E, int32_t F, int32_t H, int32_t Hkv, int32_t V,
                                      int32_t n_ranks, int32_t rank, int32_t* out) {
    if (out == nullptr) return fail(SLLM_CUDA_ERR_ARG, "tp_plan: null output");
    const int rc = check_geometry(n_layer, E, F, H, Hkv, V, n_ranks, rank);
    if (rc != SLLM_CUDA_OK) return rc;
    sllm_cuda_tp_model m;
    fill_geometry(&m, n_layer, E, F, H, Hkv, V, n_ranks, rank);
    const int32_t v[8] = {m.hq, m.hk, m.e_loc, m.f_loc, m.down_c, m.down_k, m.v0, m.v_loc};
    std::memcpy(out, v, sizeof v);
    return SLLM_CUDA_OK;
}

static int tp_model_alloc(sllm_cuda_tp_model* m, int device) {
    m->device = device;
    const Layout L = shard_layout(m);
    m->blob_bytes = L.total;
    CK(cudaSetDevice(device), "cudaSetDevice");
    CK(dev_malloc((void**)&m->blob, L.total), "tp model blob");
    bind_pointers(m, L);
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_tp_model_upload(const sllm_cuda_model_desc* d, int32_t n_ranks, int32_t rank, int32_t device,
                                         sllm_cuda_tp_model** out) {
    if (d == nullptr || out == nullptr || d->layers == nullptr || d->tok_embd == nullptr || d->output_norm == nullptr)
        return fail(SLLM_CUDA_ERR_ARG, "tp_model_upload: bad arguments");
    *out = nullptr;
    int rc = check_geometry(d->n_layer, d->n_embd, d->n_ff, d->n_head, d->n_head_kv, d->n_vocab, n_ranks, rank);
    if (rc != SLLM_CUDA_OK) return rc;
    if (d->n_rot != kHeadDim) return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp_model_upload: n_rot must be 128");
    auto* m = new sllm_cuda_tp_model();
    fill_geometry(m, d->n_layer, d->n_embd, d->n_ff, d->n_head, d->n_head_kv, d->n_vocab, n_ranks, rank);
    m->eps = d->f_rms_eps;
    m->rope_base = d->rope_freq_base;
    rc = tp_model_alloc(m, device);
    if (rc != SLLM_CUDA_OK) { delete m; return rc; }
    const int E = m->E, F = m->F, D = kHeadDim, G = m->Hkv * D;
    std::vector<uint8_t> buf;
    Uploader up(device);     // pinned, double-buffered staging
    // the slices are re-packed in buf, which the next slice reuses
    auto put = [&](const void* dst, const void* src, size_t n) {
        return up.put(const_cast<void*>(dst), src, n, src == buf.data());
    };
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < m->n_layer && e == cudaSuccess; ++l) {
        const sllm_cuda_layer_desc& h = d->layers[l];
        const TpLayer& t = m->layers[l];
        slice_i2s(h.wq, E, E, rank * m->hq * D, m->hq * D, 0, E, buf); e = put(t.wq, buf.data(), buf.size());
        slice_i2s(h.wk, G, E, rank * m->hk * D, m->hk * D, 0, E, buf); if (!e) e = put(t.wk, buf.data(), buf.size());
        slice_i2s(h.wv, G, E, rank * m->hk * D, m->hk * D, 0, E, buf); if (!e) e = put(t.wv, buf.data(), buf.size());
        slice_i2s(h.wo, E, E, 0, E, rank * m->e_loc, m->e_loc, buf); if (!e) e = put(t.wo, buf.data(), buf.size());
        slice_i2s(h.ffn_gate, F, E, rank * m->f_loc, m->f_loc, 0, E, buf); if (!e) e = put(t.gate, buf.data(), buf.size());
        slice_i2s(h.ffn_up, F, E, rank * m->f_loc, m->f_loc, 0, E, buf); if (!e) e = put(t.up, buf.data(), buf.size());
        for (int c = 0; c < m->down_c && !e; ++c) {
            slice_i2s(h.ffn_down, E, F, 0, E, rank * m->f_loc + c * m->down_k, m->down_k, buf);
            e = put(t.down[c], buf.data(), buf.size());
        }
        if (!e) e = put(t.attn_norm, h.attn_norm, (size_t)E * 4);
        if (!e) e = put(t.attn_sub_norm, h.attn_sub_norm, (size_t)E * 4);
        if (!e) e = put(t.ffn_norm, h.ffn_norm, (size_t)E * 4);
        if (!e) e = put(t.ffn_sub_norm, h.ffn_sub_norm, (size_t)F * 4);
    }
    if (!e) e = put(m->tok_embd, d->tok_embd, (size_t)m->V * E * 2);
    if (!e) e = put(m->output_norm, d->output_norm, (size_t)E * 4);
    if (!e) e = up.finish();
    if (e != cudaSuccess) {
        cudaFree(m->blob);
        delete m;
        return cuda_fail(e, "tp_model_upload");
    }
    *out = m;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_tp_model_synth(const sllm_cuda_tp_synth_desc* d, int32_t n_ranks, int32_t rank,
                                        int32_t device, sllm_cuda_tp_model** out) {
    if (d == nullptr || out == nullptr) return fail(SLLM_CUDA_ERR_ARG, "tp_model_synth: bad arguments");
    *out = nullptr;
    int rc = check_geometry(d->n_layer, d->n_embd, d->n_ff, d->n_head, d->n_head_kv, d->n_vocab, n_ranks, rank);
    if (rc != SLLM_CUDA_OK) return rc;
    auto* m = new sllm_cuda_tp_model();
    fill_geometry(m, d->n_layer, d->n_embd, d->n_ff, d->n_head, d->n_head_kv, d->n_vocab, n_ranks, rank);
    m->eps = d->f_rms_eps;
    m->rope_base = d->rope_freq_base;
    rc = tp_model_alloc(m, device);
    if (rc != SLLM_CUDA_OK) { delete m; return rc; }
    const int E = m->E, D = kHeadDim, grid = 4 * num_sms_of(device), blk = 256;
    const uint64_t seed = d->seed;
    for (int l = 0; l < m->n_layer; ++l) {
        const TpLayer& t = m->layers[l];
        auto gen = [&](const uint8_t* dst, int tensor, int r0, int rows, int c0, int cols) {
            tp_gen_i2s_kernel<<<grid, blk>>>(const_cast<uint8_t*>(dst), tensor_key(seed, l, tensor), r0, rows, c0, cols);
        };
        gen(t.wq, 0, rank * m->hq * D, m->hq * D, 0, E);
        gen(t.wk, 1, rank * m->hk * D, m->hk * D, 0, E);
        gen(t.wv, 2, rank * m->hk * D, m->hk * D, 0, E);
        gen(t.wo, 3, 0, E, rank * m->e_loc, m->e_loc);
        gen(t.gate, 4, rank * m->f_loc, m->f_loc, 0, E);
        gen(t.up, 5, rank * m->f_loc, m->f_loc, 0, E);
        for (int c = 0; c < m->down_c; ++c) gen(t.down[c], 6, 0, E, rank * m->f_loc + c * m->down_k, m->down_k);
        tp_gen_norm_kernel<<<grid, blk>>>(const_cast<float*>(t.attn_norm), tensor_key(seed, l, 8), E);
        tp_gen_norm_kernel<<<grid, blk>>>(const_cast<float*>(t.attn_sub_norm), tensor_key(seed, l, 9), E);
        tp_gen_norm_kernel<<<grid, blk>>>(const_cast<float*>(t.ffn_norm), tensor_key(seed, l, 10), E);
        tp_gen_norm_kernel<<<grid, blk>>>(const_cast<float*>(t.ffn_sub_norm), tensor_key(seed, l, 11), m->F);
    }
    tp_gen_embd_kernel<<<grid, blk>>>(const_cast<uint16_t*>(m->tok_embd), tensor_key(seed, -1, 12), (size_t)m->V * E);
    tp_gen_norm_kernel<<<grid, blk>>>(const_cast<float*>(m->output_norm), tensor_key(seed, -1, 13), E);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        cudaFree(m->blob);
        delete m;
        return cuda_fail(e, "tp_model_synth");
    }
    *out = m;
    return SLLM_CUDA_OK;
}

extern "C" void sllm_cuda_tp_model_free(sllm_cuda_tp_model* m) {
    if (m == nullptr) return;
    cudaSetDevice(m->device);
    cudaFree(m->blob);
    delete m;
}

extern "C" size_t sllm_cuda_tp_model_bytes(const sllm_cuda_tp_model* m) { return m ? m->blob_bytes : 0; }

// ---------------------------------------------------------------------------
// context and the decode step
// ---------------------------------------------------------------------------
namespace {

template <class T>
cudaError_t ctx_alloc(sllm_cuda_tp_ctx* c, T** p, size_t count) {
    void* v = nullptr;
    const cudaError_t e = dev_malloc(&v, align256(count * sizeof(T)));
    if (e == cudaSuccess) {
        c->allocs.push_back(v);
        *p = static_cast<T*>(v);
    }
    return e;
}

// The exchange after a phase: NCCL on the context's stream, or, for a
// one-process group, device copies across the group's contexts.
enum Xchg { X_ATTN = 0, X_DOTS_O, X_H, X_DOTS_D, X_ARGMAX };

void xchg_counts(const sllm_cuda_tp_model* m, int which, size_t* count, bool* gather) {
    switch (which) {
        case X_ATTN: *count = (size_t)m->hq * kHeadDim; *gather = true; break;
        case X_DOTS_O: *count = (size_t)m->E; *gather = false; break;
        case X_H: *count = (size_t)m->f_loc; *gather = true; break;
        case X_DOTS_D: *count = (size_t)m->E * m->down_c; *gather = false; break;
        default: *count = 3; *gather = true; break;
    }
}

void xchg_buffers(sllm_cuda_tp_ctx* c, int which, void** src, void** dst) {
    switch (which) {
        case X_ATTN: *src = c->attn_loc; *dst = c->attn_full; break;
        case X_DOTS_O: *src = c->dots_o; *dst = c->dots_o; break;
        case X_H: *src = c->h_loc; *dst = c->h_full; break;
        case X_DOTS_D: *src = c->dots_d; *dst = c->dots_d; break;
        default: *src = c->trip; *dst = c->trip_all; break;
    }
}

cudaError_t xchg_nccl(sllm_cuda_tp_ctx* c, int which, cudaStream_t st, ncclResult_t* nr) {
    size_t count;
    bool gather;
    void *src, *dst;
    xchg_counts(c->m, which, &count, &gather);
    xchg_buffers(c, which, &src, &dst);
    if (c->m->n_ranks == 1) {
        // the fused programs write the attention output and h where the
        // gathers would copy them to
        if (!c->fused.empty() && (which == X_ATTN || which == X_H)) return cudaSuccess;
        if (gather && src != dst) return cudaMemcpyAsync(dst, src, count * 4, cudaMemcpyDeviceToDevice, st);
        return cudaSuccess;
    }
    if (c->p2p) {
        XParams x{};
        for (int r = 0; r < c->m->n_ranks; ++r) x.peer[r] = c->peer[r];
        x.src = static_cast<const uint32_t*>(src);
        x.dst = static_cast<uint32_t*>(dst);
        x.off = which == X_ATTN ? c->off_attn : which == X_DOTS_O ? c->off_dots_o : which == X_H ? c->off_h
                : which == X_DOTS_D ? c->off_dots_d : c->off_trip;
        x.off_flags = c->off_flags;
        x.count = (uint32_t)count;
        x.n = c->m->n_ranks;
        x.rank = c->m->rank;
        x.reduce = gather ? 0 : 1;
        x.epoch = c->epoch;
        x.error = c->x_error;
        tp_exchange_kernel<<<1, 1024, 0, st>>>(x);
        return cudaGetLastError();
    }
    if (gather) {
        *nr = nccl()->all_gather(src, dst, count, which == X_ARGMAX ? ncclInt32 : ncclFloat32, c->comm->comm, st);
    } else {
        *nr = nccl()->all_reduce(src, dst, count, ncclInt32, ncclSum, c->comm->comm, st);
    }
    return *nr == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t xchg_group(sllm_cuda_tp_ctx** cs, int n, int which, cudaStream_t st) {
    size_t count;
    bool gather;
    xchg_counts(cs[0]->m, which, &count, &gather);
    if (gather) {
        for (int r = 0; r < n; ++r) {
            void *dst, *unused;
            xchg_buffers(cs[r], which, &unused, &dst);
            for (int s = 0; s < n; ++s) {
                void *src, *unused2;
                xchg_buffers(cs[s], which, &src, &unused2);
                const cudaError_t e = cudaMemcpyAsync(static_cast<char*>(dst) + (size_t)s * count * 4, src, count * 4,
                                                      cudaMemcpyDeviceToDevice, st);
                if (e != cudaSuccess) return e;
            }
        }
        return cudaSuccess;
    }
    SumArgs a{};
    a.n = n;
    a.count = count;
    for (int r = 0; r < n; ++r) {
        void *src, *dst;
        xchg_buffers(cs[r], which, &src, &dst);
        a.buf[r] = static_cast<int32_t*>(dst);
    }
    tp_group_sum_kernel<<<64, 256, 0, st>>>(a);
    count_launches(1);
    return cudaGetLastError();
}

// phases of the step: 0 = embedding; per layer l: 1 + 4l + {0: Q/K/V +
// attention, 1: O dots, 2: residual + gate/up, 3: down dots}; then the
// residual of the last layer + the head; then the finalize. The exchange
// after each phase is given by phase_xchg (-1: none).
int n_phases(const sllm_cuda_tp_model* m) { return 1 + 4 * m->n_layer + 2; }

int phase_xchg(const sllm_cuda_tp_model* m, int ph) {
    if (ph == 0 || ph == n_phases(m) - 1) return -1;
    if (ph == n_phases(m) - 2) return X_ARGMAX;
    return (ph - 1) % 4;     // X_ATTN, X_DOTS_O, X_H, X_DOTS_D in order
}

// a launch with programmatic stream serialisation: it may be scheduled while
// the previous kernel runs; the kernel waits for it (griddepcontrol.wait)
// before its first global access
cudaLaunchConfig_t pdl_config(int grid, int block, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = st;
    return cfg;
}

cudaLaunchAttribute pdl_attribute() {
    cudaLaunchAttribute a = {};
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

cudaError_t launch_count(cudaError_t e, int n) {
    if (e == cudaSuccess) count_launches(n);
    return e;
}

// RMSNorm + quantisation of a whole vector: the eight-CTA cluster when the
// length allows it (a multiple of 32, at most 32768), else one CTA
cudaError_t launch_norm_quant(const float* x, const float* w, int K, float eps, int8_t* q, sllm_cuda_act* act,
                              int* fb, int force, cudaStream_t st, const XWait& xw = XWait{}, int rows = 1) {
    const double inv_k = 1.0 / (double)K;
    const bool cluster = K % (4 * kNqCluster) == 0 && K <= 4 * kNqCluster * kNqThreads;
    if (rows > 1 && !cluster) return cudaErrorInvalidValue;      // several rows: the cluster form only
    cudaLaunchConfig_t cfg = pdl_config(cluster ? kNqCluster * rows : 1, kNqThreads, st);
    cudaLaunchAttribute attr = pdl_attribute();
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cluster)
        return cudaLaunchKernelEx(&cfg, tp_norm_quant_cluster_kernel, x, w, K, eps, inv_k, q, act, fb, force, xw);
    return cudaLaunchKernelEx(&cfg, tp_norm_quant_kernel, x, w, K, eps, inv_k, q, act, fb, force);
}

// a layer GEMV phase: the context's engine program when it has one, else the
// per-GEMV kernel with parameters p
cudaError_t gemv_or_engine(sllm_cuda_tp_ctx* c, int l, int phase, const GemvParams& p, int pro, int epi, int sms,
                           cudaStream_t st) {
    if (!c->progs.empty()) {
        const sllm_cuda_tp_ctx::Prog& pr = c->progs[(size_t)l * 4 + phase];
        return launch_engine(pr.p, c->grid, st, pr.wa, pr.wb);
    }
    return launch_gemv(p, pro, epi, sms, st);
}

cudaError_t enqueue_phase(sllm_cuda_tp_ctx* c, int ph, cudaStream_t st, bool counted) {
    const sllm_cuda_tp_model* m = c->m;
    const int E = m->E, D = kHeadDim, sms = num_sms_of(m->device);
    int* fb = fallback_counter();
    const int force = force_fallback_flag();
    const int cnt = counted ? 1 : 0;
    auto epi = [&](const int32_t* dots, int chunks, const sllm_cuda_act* act, const uint8_t* w, int rows, int cols,
                   const float* resid, float* y) {
        const float* ws = reinterpret_cast<const float*>(w + (size_t)rows * cols / 4);
        cudaLaunchConfig_t cfg = pdl_config((rows + 255) / 256, 256, st);
        cudaLaunchAttribute attr = pdl_attribute();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        return launch_count(cudaLaunchKernelEx(&cfg, tp_epilogue_kernel, dots, chunks, rows, act, ws, resid, y), cnt);
    };
    if (ph == 0) {
        cudaError_t e = launch_count(launch_embed(m->tok_embd, c->tok_seq, c->pos, E, m->V, c->x, st), cnt);
        if (e == cudaSuccess && !c->fused.empty())
            e = cudaMemsetAsync(c->fused_barriers, 0, sizeof(unsigned) * c->fused.size(), st);
        return e;
    }
    if (ph == n_phases(m) - 1) {
        tp_finalize_kernel<<<1, 1, 0, st>>>(c->trip_all, m->n_ranks, c->pos, c->tok_seq, c->prompt_end, c->argmax,
                                            c->hist, c->n_ctx,
                                            c->x_steps);
        return launch_count(cudaGetLastError(), cnt);
    }
    if (ph == n_phases(m) - 2) {
        const TpLayer& t = m->layers[m->n_layer - 1];
        cudaError_t e = epi(c->dots_d, m->down_c, c->act_h, t.down[0], E, m->down_k, c->ffn_inp, c->x);
        if (e != cudaSuccess) return e;
        LmParams lp{};
        lp.x = c->x; lp.norm_w = m->output_norm; lp.eps = m->eps;
        lp.embd = m->tok_embd + (size_t)m->v0 * E;
        lp.E = E; lp.V = m->v_loc; lp.logits = c->logits;
        lp.part_v = c->part_v; lp.part_i = c->part_i; lp.counter = c->counter; lp.argmax_out = c->argmax;
        lp.pos_ptr = c->pos; lp.tok_seq = c->tok_seq; lp.prompt_end = c->prompt_end; lp.argmax_hist = nullptr;
        lp.n_ctx = c->n_ctx; lp.fallback_count = fb; lp.force_fallback = force;
        lp.tp_out = c->trip; lp.row_base = m->v0;
        return launch_count(launch_lm_head(lp, c->lm_grid, st), cnt);
    }
    const int l = (ph - 1) / 4, sub = (ph - 1) % 4;
    const TpLayer& t = m->layers[l];
    GemvParams p{};
    p.eps = m->eps;
    p.fallback_count = fb;
    p.force_fallback = force;
    if (sub == 0) {
        if (l > 0) {
            // the residual of the previous layer's down projection
            const TpLayer& tp = m->layers[l - 1];
            cudaError_t e = epi(c->dots_d, m->down_c, c->act_h, tp.down[0], E, m->down_k, c->ffn_inp, c->x);
            if (e != cudaSuccess) return e;
        }
        if (!c->fused.empty()) {
            const sllm_cuda_tp_ctx::Prog& pr = c->fused[(size_t)l];
            return launch_count(launch_engine(pr.p, c->grid, st, pr.wa, pr.wb), cnt);
        }
        // attn_norm -> local Q, K, V (src/forward.c:631-666)
        p.K = E; p.nseg = 3;
        p.seg[0] = GemvSeg{t.wq, m->hq * D, c->q, nullptr};
        p.seg[1] = GemvSeg{t.wk, m->hk * D, c->k, nullptr};
        p.seg[2] = GemvSeg{t.wv, m->hk * D, c->v, nullptr};
        p.x = c->x; p.norm_w = t.attn_norm;
        cudaError_t e = launch_count(gemv_or_engine(c, l, 0, p, PRO_NORM, EPI_F32, sms, st), cnt);
        if (e != cudaSuccess) return e;
        const size_t kv_layer = (size_t)m->hk * D * (size_t)c->n_ctx;
        AttnParams ap{};
        ap.q = c->q; ap.k = c->k; ap.v = c->v;
        ap.k_cache = c->k_cache + (size_t)l * kv_layer;
        ap.v_cache = c->v_cache + (size_t)l * kv_layer;
        ap.rope_cos = c->rope_cos; ap.rope_sin = c->rope_sin;
        ap.pos_ptr = c->pos; ap.out = c->attn_loc; ap.n_ctx = c->n_ctx;
        ap.group = m->hq / m->hk;
        ap.attn_scale = 1.0f / sqrtf((float)D);
        ap.fallback_count = fb; ap.force_fallback = force;
        return launch_count(launch_attention(ap, m->hq, st), cnt);
    }
    if (!c->fused.empty() && (sub == 1 || sub == 2)) return cudaSuccess;   // inside the layer's program
    if (sub == 1) {
        // attn_sub_norm + quantisation of the whole attention output, then
        // this rank's columns of O (src/forward.c:728-741)
        cudaError_t e = launch_count(
            launch_norm_quant(c->attn_full, t.attn_sub_norm, E, m->eps, c->qa, c->act_a, fb, force, st), cnt);
        if (e != cudaSuccess) return e;
        p.K = m->e_loc; p.nseg = 1;
        p.seg[0] = GemvSeg{t.wo, E, nullptr, c->dots_o};
        p.q_in = c->qa + (size_t)m->rank * m->e_loc;
        p.act_in = c->act_a;
        return launch_count(gemv_or_engine(c, l, 1, p, PRO_Q8, EPI_DOTS, sms, st), cnt);
    }
    if (sub == 2) {
        // O epilogue + residual, then ffn_norm -> local gate, up -> h (src/forward.c:742-779)
        cudaError_t e = epi(c->dots_o, 1, c->act_a, t.wo, E, m->e_loc, c->x, c->ffn_inp);
        if (e != cudaSuccess) return e;
        p.K = E; p.nseg = 2;
        p.seg[0] = GemvSeg{t.gate, m->f_loc, nullptr, nullptr};
        p.seg[1] = GemvSeg{t.up, m->f_loc, nullptr, nullptr};
        p.x = c->ffn_inp; p.norm_w = t.ffn_norm; p.h_out = c->h_loc;
        return launch_count(gemv_or_engine(c, l, 2, p, PRO_NORM, EPI_SILU, sms, st), cnt);
    }
    // ffn_sub_norm + quantisation of all of h, then this rank's columns of
    // down, chunk by chunk (src/forward.c:781-792)
    cudaError_t e =
        launch_count(launch_norm_quant(c->h_full, t.ffn_sub_norm, m->F, m->eps, c->qh, c->act_h, fb, force, st), cnt);
    if (e == cudaSuccess && !c->progs.empty()) return launch_count(gemv_or_engine(c, l, 3, p, 0, 0, sms, st), cnt);
    for (int ch = 0; ch < m->down_c && e == cudaSuccess; ++ch) {
        GemvParams d = p;
        d.K = m->down_k; d.nseg = 1;
        d.seg[0] = GemvSeg{t.down[ch], E, nullptr, c->dots_d + (size_t)ch * E};
        d.q_in = c->qh + (size_t)m->rank * m->f_loc + (size_t)ch * m->down_k;
        d.act_in = c->act_h;
        e = launch_count(launch_gemv(d, PRO_Q8, EPI_DOTS, sms, st), cnt);
    }
    return e;
}

// The receive region of the peer exchange and the peers' mappings (CUDA IPC
// handles swapped with one NCCL all-gather), when SLLM_CUDA_TP_EXCHANGE=p2p
// asks for it; every rank uses it only when all ranks set it up (NCCL
// min-reduce of the outcome), else NCCL carries the exchanges (the default:
// on two B200s NCCL's collectives measured slightly faster than this).
int setup_peer_exchange(sllm_cuda_tp_ctx* c) {
    const sllm_cuda_tp_model* m = c->m;
    const int N = m->n_ranks;
    if (N < 2 || c->comm == nullptr || c->comm->comm == nullptr) return SLLM_CUDA_OK;
    const char* env = getenv("SLLM_CUDA_TP_EXCHANGE");
    if (env == nullptr || strcmp(env, "p2p") != 0) return SLLM_CUDA_OK;
    const size_t E = m->E;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    c->off_flags = take(4 * kMaxRanks);
    c->off_attn = take(4 * E);
    c->off_h = take(4 * (size_t)m->F);
    c->off_dots_o = take(4 * E * N);
    c->off_dots_d = take(4 * E * m->down_c * N);
    c->off_trip = take(4 * 3 * (size_t)N);
    c->off_xflags = take(4 * 4 * (size_t)kMaxRanks);
    int ok = 1;
    cudaIpcMemHandle_t mine{};
    if (cudaMalloc(&c->region, off) != cudaSuccess) { c->region = nullptr; ok = 0; }
    if (ok && cudaMemset(c->region, 0, off) != cudaSuccess) ok = 0;
    if (ok && cudaIpcGetMemHandle(&mine, c->region) != cudaSuccess) ok = 0;
    char* dev = nullptr;
    CK(cudaMalloc(&dev, sizeof(cudaIpcMemHandle_t) * (N + 1) + 16), "exchange set-up");
    std::vector<cudaIpcMemHandle_t> all(N);
    int* okd = reinterpret_cast<int*>(dev + sizeof(cudaIpcMemHandle_t) * (N + 1));
    cudaError_t e = cudaMemcpy(dev, &mine, sizeof(mine), cudaMemcpyHostToDevice);
    ncclResult_t nr = ncclSuccess;
    if (e == cudaSuccess)
        nr = nccl()->all_gather(dev, dev + sizeof(mine), sizeof(mine), ncclInt8, c->comm->comm, c->stream);
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess && nr == ncclSuccess)
        e = cudaMemcpy(all.data(), dev + sizeof(mine), sizeof(mine) * N, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess || nr != ncclSuccess) ok = 0;
    for (int r = 0; r < N && ok; ++r) {
        if (r == m->rank) { c->peer[r] = c->region; continue; }
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) { ok = 0; break; }
        c->peer[r] = static_cast<char*>(ptr);
    }
    cudaGetLastError();
    // every rank must take the same path
    int agreed = 0;
    e = cudaMemcpy(okd, &ok, 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) nr = nccl()->all_reduce(okd, okd, 1, ncclInt32, ncclMin, c->comm->comm, c->stream);
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaMemcpy(&agreed, okd, 4, cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (e != cudaSuccess) return cuda_fail(e, "exchange set-up");
    if (nr != ncclSuccess) return fail(SLLM_CUDA_ERR_COMM, "exchange set-up: %s", nccl_err(nr));
    if (agreed == 1) {
        CK(ctx_alloc(c, &c->epoch, 1), "exchange counter");
        CK(ctx_alloc(c, &c->x_error, 1), "exchange error word");
        CK(cudaMemset(c->epoch, 0, 4), "exchange counter");
        CK(cudaMemset(c->x_error, 0, 4), "exchange error word");
        c->p2p = true;
    }
    return SLLM_CUDA_OK;
}

float read_scale(const uint8_t* w, int rows, int cols) {
    float v = 0.0f;
    cudaMemcpy(&v, w + (size_t)rows * cols / 4, 4, cudaMemcpyDeviceToHost);
    return v;
}

int wpl_of(int K) { return engine_wpl(K); }

// One single-stage engine program per layer and GEMV phase, tables in device
// memory owned by the context. Returns OK and leaves c->progs empty when the
// widths are not compiled in.
// One rank: each layer's Q/K/V, attention, O and gate/up as one engine
// program of four stages (src/forward.c:628-779), as the single-GPU decode
// step runs them: the attention output and h go straight to the buffers the
// rest of the step reads, O's epilogue adds the residual into ffn_inp. The
// down projection (n_ff = 28672 is quantised by its own kernel) keeps its
// phase. Results are identical: the same GEMV, attention and epilogue
// arithmetic, in the same order.
int build_fused_programs(sllm_cuda_tp_ctx* c, int wa, int wb) {
    const sllm_cuda_tp_model* m = c->m;
    const int D = kHeadDim, E = m->E;
    int* fb = fallback_counter();
    CK(ctx_alloc(c, &c->fused_barriers, (size_t)m->n_layer), "fused program barriers");
    const size_t kv_layer = (size_t)m->hk * D * (size_t)c->n_ctx;
    for (int l = 0; l < m->n_layer; ++l) {
        const TpLayer& t = m->layers[l];
        std::vector<EngGroup> groups;
        std::vector<EngOp> ops;
        std::vector<int> stage_first;
        auto op = [&](const uint8_t* w, const uint8_t* w2, float* y, const float* resid, float* h, int rows, int K,
                      int epi, int group) {
            EngOp o{};
            o.w = w; o.w2 = w2; o.y = y; o.resid = resid; o.h = h; o.rows = rows; o.K = K; o.epi = epi; o.group = group;
            o.chunk_rows = epi == kEpiAttention ? 1 : engine_chunk_rows(K, epi);
            o.ws = w != nullptr ? read_scale(w, rows, K) : 0.0f;
            o.ws2 = w2 != nullptr ? read_scale(w2, rows, K) : 0.0f;
            ops.push_back(o);
        };
        auto group = [&](const float* x, const float* norm_w) {
            EngGroup g{}; g.x = x; g.norm_w = norm_w; g.K = E; g.pro = PRO_NORM;
            groups.push_back(g);
            return (int)groups.size() - 1;
        };
        stage_first.push_back((int)ops.size());         // attn_norm -> Q, K, V
        int g = group(c->x, t.attn_norm);
        op(t.wq, nullptr, c->q, nullptr, nullptr, m->hq * D, E, EPI_F32, g);
        op(t.wk, nullptr, c->k, nullptr, nullptr, m->hk * D, E, EPI_F32, g);
        op(t.wv, nullptr, c->v, nullptr, nullptr, m->hk * D, E, EPI_F32, g);
        stage_first.push_back((int)ops.size());         // attention, one head per row
        op(nullptr, nullptr, c->attn_full, nullptr, nullptr, m->hq, c->n_ctx, kEpiAttention, 0);
        stage_first.push_back((int)ops.size());         // attn_sub_norm -> O, + x into ffn_inp
        g = group(c->attn_full, t.attn_sub_norm);
        op(t.wo, nullptr, c->ffn_inp, c->x, nullptr, E, E, EPI_RESID, g);
        stage_first.push_back((int)ops.size());         // ffn_norm -> gate, up -> h
        g = group(c->ffn_inp, t.ffn_norm);
        op(t.gate, t.up, nullptr, nullptr, c->h_full, m->f_loc, E, EPI_SILU, g);
        stage_first.push_back((int)ops.size());
        AttnParams ap{};
        ap.q = c->q; ap.k = c->k; ap.v = c->v;
        ap.k_cache = c->k_cache + (size_t)l * kv_layer;
        ap.v_cache = c->v_cache + (size_t)l * kv_layer;
        ap.rope_cos = c->rope_cos; ap.rope_sin = c->rope_sin;
        ap.pos_ptr = c->pos; ap.out = c->attn_full; ap.n_ctx = c->n_ctx;
        ap.group = m->hq / m->hk;
        ap.attn_scale = 1.0f / sqrtf((float)D);
        ap.fallback_count = fb; ap.force_fallback = force_fallback_flag();
        const int n_stages = (int)stage_first.size() - 1;
        if (engine_smem_bytes((int)groups.size(), (int)ops.size(), n_stages, 1) == 0) {
            c->fused.clear();       // does not fit: the per-phase programs stay in use
            return SLLM_CUDA_OK;
        }
        const std::vector<EngCursor> st = engine_starts(ops, stage_first, c->grid);
        EngGroup* dg = nullptr;
        EngOp* dop = nullptr;
        EngCursor* ds = nullptr;
        AttnParams* da = nullptr;
        CK(ctx_alloc(c, &dg, groups.size()), "fused program groups");
        CK(ctx_alloc(c, &dop, ops.size()), "fused program ops");
        CK(ctx_alloc(c, &ds, st.size()), "fused program cursors");
        CK(ctx_alloc(c, &da, 1), "fused program attention");
        CK(cudaMemcpy(dg, groups.data(), groups.size() * sizeof(EngGroup), cudaMemcpyHostToDevice), "tables");
        CK(cudaMemcpy(dop, ops.data(), ops.size() * sizeof(EngOp), cudaMemcpyHostToDevice), "tables");
        CK(cudaMemcpy(ds, st.data(), st.size() * sizeof(EngCursor), cudaMemcpyHostToDevice), "tables");
        CK(cudaMemcpy(da, &ap, sizeof(AttnParams), cudaMemcpyHostToDevice), "tables");
        sllm_cuda_tp_ctx::Prog pr{};
        pr.p.groups = dg; pr.p.ops = dop; pr.p.starts = ds; pr.p.attn = da; pr.p.n_attn = 1;
        pr.p.n_groups = (int)groups.size(); pr.p.n_ops = (int)ops.size(); pr.p.n_stages = n_stages;
        pr.p.barrier = c->fused_barriers + l; pr.p.error = c->eng_error; pr.p.eps = m->eps;
        pr.p.fallback_count = fb; pr.p.force_fallback = force_fallback_flag();
        pr.wa = wa;
        pr.wb = wb;
        c->fused.push_back(pr);
    }
    return SLLM_CUDA_OK;
}

int build_engine_programs(sllm_cuda_tp_ctx* c) {
    const sllm_cuda_tp_model* m = c->m;
    // each phase's program needs a compiled (WA, WB) pair with WA = the n_embd
    // width (Q/K/V, the gate/up pair) and its own width as WA or WB
    const int wa = wpl_of(m->E), wo = wpl_of(m->e_loc), wd = wpl_of(m->down_k);
    auto partner = [&](int w) {
        if (w != wa) return engine_supports(wa, w) ? w : -1;
        for (int cand = 1; cand <= 16; ++cand)
            if (engine_supports(wa, cand)) return cand;
        return -1;
    };
    const int wb_main = partner(wa), wb_o = partner(wo), wb_d = partner(wd);
    if (m->E > kMaxChunkK || wb_main < 0 || wb_o < 0 || wb_d < 0) return SLLM_CUDA_OK;
    CK(prepare_engine(), "engine attributes");
    c->grid = engine_grid(m->device);
    CK(ctx_alloc(c, &c->eng_error, 1), "engine error word");
    CK(ctx_alloc(c, &c->eng_barrier, 4), "engine barrier");
    CK(cudaMemset(c->eng_error, 0, 4), "engine error word");
    CK(cudaMemset(c->eng_barrier, 0, 16), "engine barrier");
    const int D = kHeadDim, E = m->E;
    int* fb = fallback_counter();
    for (int l = 0; l < m->n_layer; ++l) {
        const TpLayer& t = m->layers[l];
        for (int ph = 0; ph < 4; ++ph) {
            std::vector<EngGroup> groups;
            std::vector<EngOp> ops;
            auto op = [&](const uint8_t* w, const uint8_t* w2, float* y, float* h, int rows, int K, int epi, int group) {
                EngOp o{};
                o.w = w; o.w2 = w2; o.y = y; o.h = h; o.rows = rows; o.K = K; o.epi = epi; o.group = group;
                o.chunk_rows = engine_chunk_rows(K, epi);
                o.ws = read_scale(w, rows, K);
                o.ws2 = w2 != nullptr ? read_scale(w2, rows, K) : 0.0f;
                ops.push_back(o);
            };
            if (ph == 0) {          // attn_norm -> local Q, K, V
                EngGroup g{}; g.x = c->x; g.norm_w = t.attn_norm; g.K = E; g.pro = PRO_NORM;
                groups.push_back(g);
                op(t.wq, nullptr, c->q, nullptr, m->hq * D, E, EPI_F32, 0);
                op(t.wk, nullptr, c->k, nullptr, m->hk * D, E, EPI_F32, 0);
                op(t.wv, nullptr, c->v, nullptr, m->hk * D, E, EPI_F32, 0);
            } else if (ph == 1) {   // this rank's columns of O: partial int32 dots
                EngGroup g{}; g.q8 = c->qa + (size_t)m->rank * m->e_loc; g.act8 = c->act_a; g.K = m->e_loc; g.pro = PRO_Q8;
                groups.push_back(g);
                op(t.wo, nullptr, reinterpret_cast<float*>(c->dots_o), nullptr, E, m->e_loc, EPI_DOTS, 0);
            } else if (ph == 2) {   // ffn_norm -> local gate, up -> h
                EngGroup g{}; g.x = c->ffn_inp; g.norm_w = t.ffn_norm; g.K = E; g.pro = PRO_NORM;
                groups.push_back(g);
                op(t.gate, t.up, nullptr, c->h_loc, m->f_loc, E, EPI_SILU, 0);
            } else {                // this rank's columns of down, chunk by chunk
                for (int ch = 0; ch < m->down_c; ++ch) {
                    EngGroup g{};
                    g.q8 = c->qh + (size_t)m->rank * m->f_loc + (size_t)ch * m->down_k;
                    g.act8 = c->act_h; g.K = m->down_k; g.pro = PRO_Q8;
                    groups.push_back(g);
                    op(t.down[ch], nullptr, reinterpret_cast<float*>(c->dots_d + (size_t)ch * E), nullptr, E,
                       m->down_k, EPI_DOTS, ch);
                }
            }
            const std::vector<int> stage_first{0, (int)ops.size()};
            const std::vector<EngCursor> st = engine_starts(ops, stage_first, c->grid);
            if (engine_smem_bytes((int)groups.size(), (int)ops.size(), 1) == 0)
                return fail(SLLM_CUDA_ERR_TOO_LARGE, "tp engine program does not fit in shared memory");
            EngGroup* dg = nullptr;
            EngOp* dop = nullptr;
            EngCursor* ds = nullptr;
            CK(ctx_alloc(c, &dg, groups.size()), "tp engine groups");
            CK(ctx_alloc(c, &dop, ops.size()), "tp engine ops");
            CK(ctx_alloc(c, &ds, st.size()), "tp engine cursors");
            CK(cudaMemcpy(dg, groups.data(), groups.size() * sizeof(EngGroup), cudaMemcpyHostToDevice), "tables");
            CK(cudaMemcpy(dop, ops.data(), ops.size() * sizeof(EngOp), cudaMemcpyHostToDevice), "tables");
            CK(cudaMemcpy(ds, st.data(), st.size() * sizeof(EngCursor), cudaMemcpyHostToDevice), "tables");
            sllm_cuda_tp_ctx::Prog pr{};
            pr.p.groups = dg; pr.p.ops = dop; pr.p.starts = ds;
            pr.p.n_groups = (int)groups.size(); pr.p.n_ops = (int)ops.size(); pr.p.n_stages = 1;
            pr.p.barrier = c->eng_barrier; pr.p.error = c->eng_error; pr.p.eps = m->eps;
            pr.p.fallback_count = fb; pr.p.force_fallback = force_fallback_flag();
            pr.wa = wa;
            pr.wb = ph == 1 ? wb_o : ph == 3 ? wb_d : wb_main;
            c->progs.push_back(pr);
        }
    }
    if (m->n_ranks == 1 && c->n_ctx <= kEngAttnMaxCtx) {
        const int rc = build_fused_programs(c, wa, wb_main);
        if (rc != SLLM_CUDA_OK) return rc;
    }
    return SLLM_CUDA_OK;
}

// Exchange kinds of the fused peer exchange (one of each per layer).
enum XKind { XK_ATTN = 0, XK_DOTS_O = 1, XK_H = 2, XK_DOTS_D = 3 };

// The fused peer exchange's programs (see sllm_cuda_tp_ctx::xa). Built when
// the peer exchange is set up and the widths have an exchanging instance;
// otherwise the per-phase programs and exchange kernels stay in use.
int build_xch_programs(sllm_cuda_tp_ctx* c) {
    const sllm_cuda_tp_model* m = c->m;
    const int N = m->n_ranks, E = m->E, D = kHeadDim, C = m->down_c;
    if (!c->p2p || c->progs.empty() || N > kEngMaxPeers || c->n_ctx > kEngAttnMaxCtx) return SLLM_CUDA_OK;
    const int wa = wpl_of(E), wo = wpl_of(m->e_loc), wd = wpl_of(m->down_k);
    if (!engine_supports_xch(wa, wo) || !engine_supports_xch(wa, wd) || m->F % (4 * 8) != 0 ||
        m->F > 4 * 8 * kNqThreads || m->e_loc % 128 != 0)
        return SLLM_CUDA_OK;
    int* fb = fallback_counter();
    CK(ctx_alloc(c, &c->x_barriers, (size_t)m->n_layer), "exchange program barriers");
    CK(ctx_alloc(c, &c->x_done, 1), "exchange program counter");
    CK(ctx_alloc(c, &c->x_steps, 1), "exchange step counter");
    CK(cudaMemset(c->x_done, 0, 4), "exchange program counter");
    CK(cudaMemset(c->x_steps, 0, 4), "exchange step counter");
    char* region = c->region;
    float* attn_full = reinterpret_cast<float*>(region + c->off_attn);
    float* h_full = reinterpret_cast<float*>(region + c->off_h);
    int32_t* dots_o = reinterpret_cast<int32_t*>(region + c->off_dots_o);   // [N][E]
    int32_t* dots_d = reinterpret_cast<int32_t*>(region + c->off_dots_d);   // [N][C][E]
    EngX xb{};
    for (int q = 0; q < N; ++q) xb.peer[q] = c->peer[q];
    xb.flag_off = (uint32_t)c->off_xflags;
    xb.steps = c->x_steps;
    xb.done = c->x_done;
    xb.n_peer = N;
    xb.rank = m->rank;
    xb.n_layer = m->n_layer;
    const size_t kv_layer = (size_t)m->hk * D * (size_t)c->n_ctx;
    auto upload = [&](const std::vector<EngGroup>& groups, const std::vector<EngOp>& ops,
                      const std::vector<int>& stage_first, const AttnParams* ap, EngParams& p) -> int {
        const std::vector<EngCursor> st = engine_starts(ops, stage_first, c->grid);
        const int n_stages = (int)stage_first.size() - 1;
        if (engine_smem_bytes((int)groups.size(), (int)ops.size(), n_stages, ap ? 1 : 0) == 0)
            return fail(SLLM_CUDA_ERR_TOO_LARGE, "tp exchange program does not fit in shared memory");
        EngGroup* dg = nullptr;
        EngOp* dop = nullptr;
        EngCursor* ds = nullptr;
        AttnParams* da = nullptr;
        CK(ctx_alloc(c, &dg, groups.size()), "exchange program groups");
        CK(ctx_alloc(c, &dop, ops.size()), "exchange program ops");
        CK(ctx_alloc(c, &ds, st.size()), "exchange program cursors");
        CK(cudaMemcpy(dg, groups.data(), groups.size() * sizeof(EngGroup), cudaMemcpyHostToDevice), "tables");
        CK(cudaMemcpy(dop, ops.data(), ops.size() * sizeof(EngOp), cudaMemcpyHostToDevice), "tables");
        CK(cudaMemcpy(ds, st.data(), st.size() * sizeof(EngCursor), cudaMemcpyHostToDevice), "tables");
        if (ap != nullptr) {
            CK(ctx_alloc(c, &da, 1), "exchange program attention");
            CK(cudaMemcpy(da, ap, sizeof(AttnParams), cudaMemcpyHostToDevice), "tables");
        }
        p.groups = dg; p.ops = dop; p.starts = ds; p.attn = da; p.n_attn = ap ? 1 : 0;
        p.n_groups = (int)groups.size(); p.n_ops = (int)ops.size(); p.n_stages = n_stages;
        p.error = c->eng_error; p.eps = m->eps; p.fallback_count = fb; p.force_fallback = force_fallback_flag();
        p.xch = 1;
        return SLLM_CUDA_OK;
    };
    for (int l = 0; l < m->n_layer; ++l) {
        const TpLayer& t = m->layers[l];
        std::vector<EngGroup> groups;
        std::vector<EngOp> ops;
        std::vector<int> stage_first;
        EngX x = xb;
        x.layer = l;
        x.end_kind = XK_H;
        auto op = [&](const uint8_t* w, const uint8_t* w2, float* y, const float* resid, float* h, int rows, int K,
                      int epi, int group, int k0x) {
            EngOp o{};
            o.w = w; o.w2 = w2; o.y = y; o.resid = resid; o.h = h; o.rows = rows; o.K = K; o.epi = epi;
            o.group = group; o.k0x = k0x;
            o.chunk_rows = epi == kEpiAttention ? 1 : epi == kEpiReduce ? rows : engine_chunk_rows(K, epi);
            o.ws = (w != nullptr && epi != kEpiReduce) ? read_scale(w, rows, K) : 0.0f;
            o.ws2 = (w2 != nullptr && epi != kEpiReduce) ? read_scale(w2, rows, K) : 0.0f;
            ops.push_back(o);
        };
        auto group = [&](const float* xv, const float* norm_w, sllm_cuda_act* act_out) {
            EngGroup g{}; g.x = xv; g.norm_w = norm_w; g.K = E; g.pro = PRO_NORM; g.act8 = act_out;
            groups.push_back(g);
            return (int)groups.size() - 1;
        };
        int si = 0;
        if (l > 0) {
            // the previous layer's down: x = its reduce + ffn_inp, once every
            // rank's partial dots have arrived (published by its program D)
            const TpLayer& tp = m->layers[l - 1];
            stage_first.push_back((int)ops.size());
            op(reinterpret_cast<const uint8_t*>(dots_d), reinterpret_cast<const uint8_t*>(c->act_h), c->x,
               c->ffn_inp, nullptr, E, N * C, kEpiReduce, 0, 0);
            ops.back().ws = read_scale(tp.down[0], E, m->down_k);
            x.xs[si++] = (int8_t)((XK_DOTS_D + 1) | kXsPrev);     // published by layer l - 1's program D
        }
        // attn_norm -> local Q, K, V (src/forward.c:631-666)
        stage_first.push_back((int)ops.size());
        int g = group(c->x, t.attn_norm, nullptr);
        op(t.wq, nullptr, c->q, nullptr, nullptr, m->hq * D, E, EPI_F32, g, 0);
        op(t.wk, nullptr, c->k, nullptr, nullptr, m->hk * D, E, EPI_F32, g, 0);
        op(t.wv, nullptr, c->v, nullptr, nullptr, m->hk * D, E, EPI_F32, g, 0);
        x.xs[si++] = 0;
        // attention over the local heads; the outputs into this rank's slice
        // of the whole attention vector in every region
        float* attn_slice = attn_full + (size_t)m->rank * m->hq * D;
        stage_first.push_back((int)ops.size());
        op(nullptr, nullptr, attn_slice, nullptr, nullptr, m->hq, c->n_ctx, kEpiAttention, 0, kOpScatter);
        x.xs[si++] = kXsFence;
        // attn_sub_norm + quantisation of the whole vector, this rank's
        // columns of O: partial dots into slot `rank` of every region
        stage_first.push_back((int)ops.size());
        g = group(attn_full, t.attn_sub_norm, c->act_a);
        op(t.wo, nullptr, reinterpret_cast<float*>(dots_o + (size_t)m->rank * E), nullptr, nullptr, E, m->e_loc,
           EPI_DOTS, g, (m->rank * m->e_loc) | kOpScatter);
        x.xs[si++] = (int8_t)((XK_ATTN + 1) | kXsSignal | kXsFence);
        // O's epilogue + residual (src/forward.c:739-750) from every rank's dots
        stage_first.push_back((int)ops.size());
        op(reinterpret_cast<const uint8_t*>(dots_o), reinterpret_cast<const uint8_t*>(c->act_a), c->ffn_inp, c->x,
           nullptr, E, N, kEpiReduce, 0, 0);
        ops.back().ws = read_scale(t.wo, E, m->e_loc);
        x.xs[si++] = (int8_t)((XK_DOTS_O + 1) | kXsSignal);
        // ffn_norm -> local gate, up -> h, into this rank's slice of h in
        // every region (src/forward.c:752-779)
        stage_first.push_back((int)ops.size());
        g = group(c->ffn_inp, t.ffn_norm, nullptr);
        op(t.gate, t.up, nullptr, nullptr, h_full + (size_t)m->rank * m->f_loc, m->f_loc, E, EPI_SILU, g, kOpScatter);
        x.xs[si++] = kXsFence;
        stage_first.push_back((int)ops.size());
        AttnParams ap{};
        ap.q = c->q; ap.k = c->k; ap.v = c->v;
        ap.k_cache = c->k_cache + (size_t)l * kv_layer;
        ap.v_cache = c->v_cache + (size_t)l * kv_layer;
        ap.rope_cos = c->rope_cos; ap.rope_sin = c->rope_sin;
        ap.pos_ptr = c->pos; ap.out = attn_slice; ap.n_ctx = c->n_ctx;
        ap.group = m->hq / m->hk;
        ap.attn_scale = 1.0f / sqrtf((float)D);
        ap.fallback_count = fb; ap.force_fallback = force_fallback_flag();
        sllm_cuda_tp_ctx::Prog pa{};
        int rc = upload(groups, ops, stage_first, &ap, pa.p);
        if (rc != SLLM_CUDA_OK) return rc;
        pa.p.barrier = c->x_barriers + l;
        pa.p.x = x;
        pa.wa = wa;
        pa.wb = wo;
        c->xa.push_back(pa);

        // program D: this rank's columns of down (pre-quantised h slices),
        // partial dots into slot [rank][chunk] of every region
        std::vector<EngGroup> dgs;
        std::vector<EngOp> dops;
        for (int ch = 0; ch < C; ++ch) {
            EngGroup dg{};
            dg.q8 = c->qh + (size_t)m->rank * m->f_loc + (size_t)ch * m->down_k;
            dg.act8 = c->act_h; dg.K = m->down_k; dg.pro = PRO_Q8;
            dgs.push_back(dg);
            EngOp o{};
            o.w = t.down[ch];
            o.y = reinterpret_cast<float*>(dots_d + ((size_t)m->rank * C + ch) * E);
            o.rows = E; o.K = m->down_k; o.epi = EPI_DOTS; o.group = ch; o.k0x = kOpScatter;
            o.chunk_rows = engine_chunk_rows(m->down_k, EPI_DOTS);
            o.ws = read_scale(t.down[ch], E, m->down_k);
            dops.push_back(o);
        }
        sllm_cuda_tp_ctx::Prog pd{};
        rc = upload(dgs, dops, std::vector<int>{0, (int)dops.size()}, nullptr, pd.p);
        if (rc != SLLM_CUDA_OK) return rc;
        pd.p.barrier = c->eng_barrier;
        EngX xd = xb;
        xd.layer = l;
        xd.end_kind = XK_DOTS_D;
        pd.p.x = xd;
        pd.wa = wa;
        pd.wb = wd;
        c->xd.push_back(pd);
    }
    return SLLM_CUDA_OK;
}

// The step of the fused peer exchange: embedding; per layer program A (a
// cooperative launch), the norm/quantisation of h once every rank's slice
// has arrived, program D; the last layer's down reduce; the head and the
// argmax exchange; the finalize (which advances the flag values).
cudaError_t enqueue_xstep(sllm_cuda_tp_ctx* c, cudaStream_t st) {
    const sllm_cuda_tp_model* m = c->m;
    const int N = m->n_ranks, E = m->E, C = m->down_c;
    int* fb = fallback_counter();
    const int force = force_fallback_flag();
    cudaError_t e = launch_embed(m->tok_embd, c->tok_seq, c->pos, E, m->V, c->x, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->x_barriers, 0, sizeof(unsigned) * m->n_layer, st);
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(c->region + c->off_xflags);
    for (int l = 0; l < m->n_layer && e == cudaSuccess; ++l) {
        e = launch_engine(c->xa[l].p, c->grid, st, c->xa[l].wa, c->xa[l].wb);
        XWait xw{flags + XK_H * kMaxRanks, c->x_steps, N, m->n_layer, l, c->eng_error};
        if (e == cudaSuccess)
            e = launch_norm_quant(reinterpret_cast<const float*>(c->region + c->off_h), m->layers[l].ffn_sub_norm,
                                  m->F, m->eps, c->qh, c->act_h, fb, force, st, xw);
        if (e == cudaSuccess) e = launch_engine(c->xd[l].p, c->grid, st, c->xd[l].wa, c->xd[l].wb);
    }
    if (e != cudaSuccess) return e;
    const TpLayer& t = m->layers[m->n_layer - 1];
    {
        XWait xw{flags + XK_DOTS_D * kMaxRanks, c->x_steps, N, m->n_layer, m->n_layer - 1, c->eng_error};
        cudaLaunchConfig_t cfg = pdl_config((E + 255) / 256, 256, st);
        cudaLaunchAttribute attr = pdl_attribute();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        const float* ws = reinterpret_cast<const float*>(t.down[0] + (size_t)E * m->down_k / 4);
        e = cudaLaunchKernelEx(&cfg, tp_xreduce_kernel, xw,
                               reinterpret_cast<const int32_t*>(c->region + c->off_dots_d), N * C, E,
                               (const sllm_cuda_act*)c->act_h, ws, (const float*)c->ffn_inp, c->x);
    }
    if (e != cudaSuccess) return e;
    LmParams lp{};
    lp.x = c->x; lp.norm_w = m->output_norm; lp.eps = m->eps;
    lp.embd = m->tok_embd + (size_t)m->v0 * E;
    lp.E = E; lp.V = m->v_loc; lp.logits = c->logits;
    lp.part_v = c->part_v; lp.part_i = c->part_i; lp.counter = c->counter; lp.argmax_out = c->argmax;
    lp.pos_ptr = c->pos; lp.tok_seq = c->tok_seq; lp.prompt_end = c->prompt_end; lp.argmax_hist = nullptr;
    lp.n_ctx = c->n_ctx; lp.fallback_count = fb; lp.force_fallback = force;
    lp.tp_out = c->trip; lp.row_base = m->v0;
    e = launch_lm_head(lp, c->lm_grid, st);
    ncclResult_t nr = ncclSuccess;
    if (e == cudaSuccess) e = xchg_nccl(c, X_ARGMAX, st, &nr);
    if (e == cudaSuccess) {
        tp_finalize_kernel<<<1, 1, 0, st>>>(c->trip_all, N, c->pos, c->tok_seq, c->prompt_end, c->argmax, c->hist,
                                            c->n_ctx, c->x_steps);
        e = cudaGetLastError();
    }
    return e;
}

int ensure_tp_graph(sllm_cuda_tp_ctx* c) {
    if (c->step != nullptr) return SLLM_CUDA_OK;
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    cudaError_t e = cudaSuccess;
    ncclResult_t nr = ncclSuccess;
    if (!c->xa.empty()) {
        e = enqueue_xstep(c, c->stream);
    } else {
        for (int ph = 0; ph < n_phases(c->m) && e == cudaSuccess; ++ph) {
            e = enqueue_phase(c, ph, c->stream, false);
            const int x = phase_xchg(c->m, ph);
            if (e == cudaSuccess && x >= 0) e = xchg_nccl(c, x, c->stream, &nr);
        }
    }
    const cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
    if (nr != ncclSuccess) { if (g) cudaGraphDestroy(g); return fail(SLLM_CUDA_ERR_COMM, "tp step: %s", nccl_err(nr)); }
    if (e != cudaSuccess) { if (g) cudaGraphDestroy(g); return cuda_fail(e, "capture tp step"); }
    if (e2 != cudaSuccess) return cuda_fail(e2, "end capture");
    e = instantiate(&c->step, g);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { c->step = nullptr; return cuda_fail(e, "instantiate tp step"); }
    return SLLM_CUDA_OK;
}

// wait for the stream, bounded: a rank whose peers stopped answering aborts
// its communicator instead of waiting for good
int tp_sync(sllm_cuda_tp_ctx* c, double seconds) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t e = cudaStreamQuery(c->stream);
        if (e == cudaSuccess) return SLLM_CUDA_OK;
        if (e != cudaErrorNotReady) return cuda_fail(e, "tp step");
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > seconds) {
            if (c->comm != nullptr && c->comm->comm != nullptr) {
                nccl()->comm_abort(c->comm->comm);
                c->comm->comm = nullptr;
            }
            return fail(SLLM_CUDA_ERR_TIMEOUT, "tp step: no progress in %.0f s (communicator aborted)", seconds);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int tp_validate(const sllm_cuda_tp_ctx* c, const int32_t* prompt, int32_t n_prompt, int32_t n_new, int32_t* out) {
    if (c == nullptr || out == nullptr || n_prompt < 0 || n_new < 0 || (n_prompt > 0 && prompt == nullptr))
        return fail(SLLM_CUDA_ERR_ARG, "tp_generate_greedy: bad arguments");
    if ((int64_t)n_prompt + n_new + c->n_past > c->n_ctx)
        return fail(SLLM_CUDA_ERR_TOO_LARGE, "tp_generate_greedy: %d + %d tokens after %d exceed n_ctx %d", n_prompt,
                    n_new, c->n_past, c->n_ctx);
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= c->m->V) return fail(SLLM_CUDA_ERR_ARG, "tp_generate_greedy: token %d out of range", prompt[i]);
    if (n_prompt == 0 && c->n_past == 0 && n_new > 0 && 128000 >= c->m->V)
        return fail(SLLM_CUDA_ERR_ARG, "tp_generate_greedy: BOS 128000 outside the vocabulary");
    return SLLM_CUDA_OK;
}

// the prompt (or BOS, src/forward.c:909) and the step's position registers
int tp_seed(sllm_cuda_tp_ctx* c, const int32_t* prompt, int32_t n_prompt) {
    const int base = c->n_past;
    if (n_prompt == 0 && base == 0) {
        c->pinned[2] = 128000;
        CK(cudaMemcpyAsync(c->tok_seq, &c->pinned[2], 4, cudaMemcpyHostToDevice, c->stream), "bos");
    } else if (n_prompt > 0) {
        CK(cudaMemcpyAsync(c->tok_seq + base, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, c->stream), "prompt");
    }
    c->pinned[0] = base;
    c->pinned[1] = base + n_prompt;
    CK(cudaMemcpyAsync(c->pos, &c->pinned[0], 4, cudaMemcpyHostToDevice, c->stream), "set pos");
    CK(cudaMemcpyAsync(c->prompt_end, &c->pinned[1], 4, cudaMemcpyHostToDevice, c->stream), "set prompt end");
    return SLLM_CUDA_OK;
}

}  // namespace

extern "C" int sllm_cuda_tp_ctx_new(const sllm_cuda_tp_model* m, sllm_cuda_tp_comm* comm, int32_t n_ctx,
                                    sllm_cuda_tp_ctx** out) {
    if (m == nullptr || out == nullptr || n_ctx < 1 || n_ctx > attention_max_ctx())
        return fail(SLLM_CUDA_ERR_ARG, "tp_ctx_new: bad arguments");
    *out = nullptr;
    if (comm != nullptr && (comm->n_ranks != m->n_ranks || comm->rank != m->rank || comm->device != m->device))
        return fail(SLLM_CUDA_ERR_ARG, "tp_ctx_new: the communicator's rank does not match the shard's");
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    CK(prepare_decode_kernels(), "decode kernel attributes");
    if (fallback_counter() == nullptr) return fail(SLLM_CUDA_ERR_NOMEM, "tp_ctx_new: diagnostics counter");
    auto* c = new sllm_cuda_tp_ctx();
    c->m = m;
    c->comm = comm;
    c->n_ctx = n_ctx;
    c->lm_grid = lm_head_grid(num_sms_of(m->device));
    const int D = kHeadDim, E = m->E;
    const size_t kv = (size_t)m->n_layer * m->hk * D * n_ctx;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (!e) e = ctx_alloc(c, &c->k_cache, kv);
    if (!e) e = ctx_alloc(c, &c->v_cache, kv);
    if (!e) e = ctx_alloc(c, &c->rope_cos, (size_t)n_ctx * D / 2);
    if (!e) e = ctx_alloc(c, &c->rope_sin, (size_t)n_ctx * D / 2);
    if (!e) e = ctx_alloc(c, &c->x, E);
    if (!e) e = ctx_alloc(c, &c->ffn_inp, E);
    if (!e) e = ctx_alloc(c, &c->q, (size_t)m->hq * D);
    if (!e) e = ctx_alloc(c, &c->k, (size_t)m->hk * D);
    if (!e) e = ctx_alloc(c, &c->v, (size_t)m->hk * D);
    if (!e) e = ctx_alloc(c, &c->attn_loc, (size_t)m->hq * D);
    if (!e) e = ctx_alloc(c, &c->attn_full, E);
    if (!e) e = ctx_alloc(c, &c->h_loc, (size_t)m->f_loc);
    if (!e) e = ctx_alloc(c, &c->h_full, (size_t)m->F);
    if (!e) e = ctx_alloc(c, &c->logits, (size_t)(m->v_loc > 0 ? m->v_loc : 1));
    if (!e) e = ctx_alloc(c, &c->qa, E);
    if (!e) e = ctx_alloc(c, &c->qh, (size_t)m->F);
    if (!e) e = ctx_alloc(c, &c->act_a, 1);
    if (!e) e = ctx_alloc(c, &c->act_h, 1);
    if (!e) e = ctx_alloc(c, &c->dots_o, E);
    if (!e) e = ctx_alloc(c, &c->dots_d, (size_t)E * m->down_c);
    if (!e) e = ctx_alloc(c, &c->part_v, c->lm_grid);
    if (!e) e = ctx_alloc(c, &c->part_i, c->lm_grid);
    if (!e) e = ctx_alloc(c, &c->counter, 1);
    if (!e) e = ctx_alloc(c, &c->trip, 3);
    if (!e) e = ctx_alloc(c, &c->trip_all, (size_t)3 * m->n_ranks);
    if (!e) e = ctx_alloc(c, &c->argmax, 1);
    if (!e) e = ctx_alloc(c, &c->pos, 1);
    if (!e) e = ctx_alloc(c, &c->prompt_end, 1);
    if (!e) e = ctx_alloc(c, &c->tok_seq, (size_t)n_ctx);
    if (!e) e = ctx_alloc(c, &c->hist, (size_t)n_ctx);
    if (!e) e = cudaMallocHost(&c->pinned, 16);
    if (!e) e = cudaEventCreate(&c->run_ev[0]);
    if (!e) e = cudaEventCreate(&c->run_ev[1]);
    if (!e) e = cudaMemset(c->counter, 0, 4);
    if (!e) e = cudaMemset(c->tok_seq, 0, (size_t)n_ctx * 4);
    if (!e) {
        std::vector<float> cs, sn;
        rope_table(n_ctx, D, m->rope_base, cs, sn);
        e = cudaMemcpy(c->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
        if (!e) e = cudaMemcpy(c->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        sllm_cuda_tp_ctx_free(c);
        return cuda_fail(e, "tp_ctx_new");
    }
    int rc = build_engine_programs(c);
    if (rc == SLLM_CUDA_OK) rc = setup_peer_exchange(c);
    if (rc == SLLM_CUDA_OK) rc = build_xch_programs(c);
    if (rc != SLLM_CUDA_OK) {
        sllm_cuda_tp_ctx_free(c);
        return rc;
    }
    *out = c;
    return SLLM_CUDA_OK;
}

extern "C" void sllm_cuda_tp_ctx_free(sllm_cuda_tp_ctx* c) {
    if (c == nullptr) return;
    cudaSetDevice(c->m->device);
    graph_exec_destroy(c->step);
    if (c->stream) cudaStreamDestroy(c->stream);
    for (int r = 0; r < kMaxRanks; ++r)
        if (c->peer[r] != nullptr && c->peer[r] != c->region) cudaIpcCloseMemHandle(c->peer[r]);
    if (c->region != nullptr) cudaFree(c->region);
    for (void* p : c->allocs) cudaFree(p);
    if (c->pinned) cudaFreeHost(c->pinned);
    for (cudaEvent_t ev : c->run_ev)
        if (ev) cudaEventDestroy(ev);
    delete c;
}

extern "C" int sllm_cuda_tp_generate_greedy(sllm_cuda_tp_ctx* c, const int32_t* prompt, int32_t n_prompt,
                                            int32_t n_new, int32_t* out) {
    int rc = tp_validate(c, prompt, n_prompt, n_new, out);
    if (rc != SLLM_CUDA_OK) return rc;
    if (n_prompt == 0 && c->n_past == 0 && n_new == 0) return SLLM_CUDA_OK;
    CK(cudaSetDevice(c->m->device), "cudaSetDevice");
    if (c->m->n_ranks > 1 && (c->comm == nullptr || c->comm->comm == nullptr))
        return fail(SLLM_CUDA_ERR_COMM, "tp_generate_greedy: no communicator");
    rc = ensure_tp_graph(c);
    if (rc != SLLM_CUDA_OK) return rc;
    const int base = c->n_past;
    rc = tp_seed(c, prompt, n_prompt);
    if (rc != SLLM_CUDA_OK) return rc;
    const int steps = n_prompt + n_new;
    CK(cudaEventRecord(c->run_ev[0], c->stream), "run timer");
    for (int s = 0; s < steps; ++s) CK(graph_launch(c->step, c->stream), "tp step");
    CK(cudaEventRecord(c->run_ev[1], c->stream), "run timer");
    if (n_new > 0)
        CK(cudaMemcpyAsync(out, c->tok_seq + base + n_prompt, (size_t)n_new * 4, cudaMemcpyDeviceToHost, c->stream), "ids");
    rc = tp_sync(c, 120.0);
    if (rc != SLLM_CUDA_OK) return rc;
    if (c->x_error != nullptr) {
        int err = 0;
        CK(cudaMemcpy(&err, c->x_error, 4, cudaMemcpyDeviceToHost), "exchange error word");
        if (err != 0) {
            cudaMemset(c->x_error, 0, 4);
            return fail(SLLM_CUDA_ERR_TIMEOUT, "tp step: a peer's exchange flag did not arrive in time");
        }
    }
    if (c->eng_error != nullptr) {
        int err = 0;
        CK(cudaMemcpy(&err, c->eng_error, 4, cudaMemcpyDeviceToHost), "engine error word");
        if (err != 0) {
            cudaMemset(c->eng_error, 0, 4);
            return fail(SLLM_CUDA_ERR_TIMEOUT, "tp step: an engine wait gave up (code %d)", err);
        }
    }
    c->n_past = base + steps;
    c->have_logits = steps > 0;
    return SLLM_CUDA_OK;
}

extern "C" float sllm_cuda_test_tp_ctx_last_run_ms(const sllm_cuda_tp_ctx* c) {
    float ms = -1.0f;
    if (c == nullptr || cudaSetDevice(c->m->device) != cudaSuccess) return -1.0f;
    if (cudaEventElapsedTime(&ms, c->run_ev[0], c->run_ev[1]) != cudaSuccess) {
        cudaGetLastError();
        return -1.0f;
    }
    return ms;
}

extern "C" int sllm_cuda_test_tp_fused_exchange(const sllm_cuda_tp_ctx* c) { return c != nullptr && !c->xa.empty(); }

extern "C" int sllm_cuda_tp_ctx_reset(sllm_cuda_tp_ctx* c) {
    if (c == nullptr) return fail(SLLM_CUDA_ERR_ARG, "tp_ctx_reset: null");
    c->n_past = 0;
    c->have_logits = false;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_tp_vocab_range(const sllm_cuda_tp_model* m, int32_t* v0, int32_t* n) {
    if (m == nullptr || v0 == nullptr || n == nullptr) return fail(SLLM_CUDA_ERR_ARG, "tp_vocab_range: null");
    *v0 = m->v0;
    *n = m->v_loc;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_tp_last_logits(const sllm_cuda_tp_ctx* c, float* host_out) {
    if (c == nullptr || host_out == nullptr || !c->have_logits)
        return fail(SLLM_CUDA_ERR_ARG, "tp_last_logits: nothing forwarded");
    CK(cudaSetDevice(c->m->device), "cudaSetDevice");
    CK(cudaMemcpy(host_out, c->logits, (size_t)c->m->v_loc * 4, cudaMemcpyDeviceToHost), "tp last logits");
    return SLLM_CUDA_OK;
}

// one process, one device, N contexts of the N shards: the same phases, the
// exchanges by device copies (tests of the sharding on a single GPU)
extern "C" int sllm_cuda_test_tp_generate_group(sllm_cuda_tp_ctx** cs, int32_t n, const int32_t* prompt,
                                                int32_t n_prompt, int32_t n_new, int32_t* out) {
    if (cs == nullptr || n < 1 || n > kMaxRanks) return fail(SLLM_CUDA_ERR_ARG, "tp group: bad arguments");
    for (int r = 0; r < n; ++r) {
        if (cs[r] == nullptr || cs[r]->m->n_ranks != n || cs[r]->m->rank != r || cs[r]->m->device != cs[0]->m->device ||
            cs[r]->n_past != cs[0]->n_past || cs[r]->n_ctx != cs[0]->n_ctx)
            return fail(SLLM_CUDA_ERR_ARG, "tp group: contexts do not form ranks 0..%d of one model on one device", n - 1);
        int rc = tp_validate(cs[r], prompt, n_prompt, n_new, out);
        if (rc != SLLM_CUDA_OK) return rc;
    }
    if (n_prompt == 0 && cs[0]->n_past == 0 && n_new == 0) return SLLM_CUDA_OK;
    CK(cudaSetDevice(cs[0]->m->device), "cudaSetDevice");
    cudaStream_t st = cs[0]->stream;
    // every context's registers are set on the group's stream
    for (int r = 0; r < n; ++r) {
        cudaStream_t own = cs[r]->stream;
        cs[r]->stream = st;
        const int rc = tp_seed(cs[r], prompt, n_prompt);
        cs[r]->stream = own;
        if (rc != SLLM_CUDA_OK) return rc;
    }
    const int base = cs[0]->n_past, steps = n_prompt + n_new;
    for (int s = 0; s < steps; ++s) {
        for (int ph = 0; ph < n_phases(cs[0]->m); ++ph) {
            for (int r = 0; r < n; ++r) CK(enqueue_phase(cs[r], ph, st, true), "tp group phase");
            const int x = phase_xchg(cs[0]->m, ph);
            if (x >= 0) CK(xchg_group(cs, n, x, st), "tp group exchange");
        }
    }
    if (n_new > 0)
        CK(cudaMemcpyAsync(out, cs[0]->tok_seq + base + n_prompt, (size_t)n_new * 4, cudaMemcpyDeviceToHost, st), "ids");
    CK(cudaStreamSynchronize(st), "tp group sync");
    for (int r = 0; r < n; ++r) {
        cs[r]->n_past = base + steps;
        cs[r]->have_logits = steps > 0;
    }
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_test_tp_uses_engine(const sllm_cuda_tp_ctx* c) {
    return c != nullptr && !c->progs.empty() ? 1 : 0;
}

extern "C" int sllm_cuda_test_tp_fused_layers(const sllm_cuda_tp_ctx* c) {
    return c != nullptr ? (int)c->fused.size() : 0;
}

extern "C" int sllm_cuda_test_tp_exchange_kind(const sllm_cuda_tp_ctx* c) {
    if (c == nullptr || c->m->n_ranks < 2) return 0;
    return c->p2p ? 2 : 1;
}

// ---------------------------------------------------------------------------
// Batch decode: B <= 16 sequences, one KV cache each, stepped together. A
// step is the single-sequence step with every GEMV of the layer turned into
// one GEMM over the B tokens (the skinny tcgen05 form: each weight byte is
// read once per step for all sequences), the attention per (head, sequence)
// over that sequence's cache and position, and the exchanges carrying B rows.
// Each sequence's tokens and logits are, bit for bit, those of its own batch-1
// run: the int32 dots are exact in any grouping and every float operation is
// the single-token kernels', token by token. The reference runs one sequence
// per context (src/forward.c:78-84, :466-562); a batch of B is B of those.
// ---------------------------------------------------------------------------
namespace {

__global__ void tp_embed_batch_kernel(const uint16_t* __restrict__ tok_embd, const int32_t* __restrict__ tok_seq,
                                      const int32_t* __restrict__ pos, int n_ctx, int E, int V, float* __restrict__ x) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int b = blockIdx.x;
    int tok = tok_seq[(size_t)b * n_ctx + pos[b]];
    if ((unsigned)tok >= (unsigned)V) tok = 0;
    const uint16_t* row = tok_embd + (size_t)tok * (size_t)E;
    float* xr = x + (size_t)b * E;
    for (int d = threadIdx.x; d < E; d += blockDim.x) xr[d] = f16_embd(row[d]);
}

// [N][B][c] (rank-major, as an all-gather leaves it) -> [B][N c]
__global__ void tp_unshard_kernel(const float* __restrict__ src, float* __restrict__ dst, int N, int B, int c) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t total = (size_t)N * B * c;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int j = (int)(i % c);
        const size_t rb = i / c;
        const int b = (int)(rb % B), r = (int)(rb / B);
        dst[((size_t)b * N + r) * c + j] = src[i];
    }
}

// tp_epilogue_kernel for B rows: dots [C][B][rows], act [B], resid and y [B][rows]
__global__ void tp_epilogue_rows_kernel(const int32_t* __restrict__ dots, int n_chunks, int B, int rows,
                                        const sllm_cuda_act* act, const float* __restrict__ ws,
                                        const float* __restrict__ resid, float* __restrict__ y) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int r = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
    if (r >= rows) return;
    const size_t o = (size_t)b * rows + r;
    int d = 0;
    for (int c = 0; c < n_chunks; ++c) d += dots[(size_t)c * B * rows + o];
    const sllm_cuda_act a = act[b];
    const float post = __fdiv_rn(*ws, a.scale);
    y[o] = __fadd_rn(__fmul_rn(__int2float_rn(d - a.sum), post), resid[o]);
}

// tp_finalize_kernel per sequence: trip_all [N][B][3]
__global__ void tp_finalize_batch_kernel(const int32_t* trip_all, int n_ranks, int B, int32_t* pos, int32_t* tok_seq,
                                         const int32_t* prompt_end, int32_t* argmax_out, int n_ctx) {
    const int b = threadIdx.x;
    if (b >= B) return;
    float bv = NAN;
    int bi = 0x7fffffff;
    for (int r = 0; r < n_ranks; ++r) {
        const int32_t* t = trip_all + ((size_t)r * B + b) * 3;
        const float v = __int_as_float(t[0]);
        if (t[1] != 0x7fffffff && tp_better(v, t[1], bv, bi)) { bv = v; bi = t[1]; }
    }
    int next = bi;
    if (bi == 0x7fffffff || trip_all[(size_t)b * 3 + 2] != 0) next = 0;   // rank 0 holds row 0
    argmax_out[b] = next;
    const int p = pos[b];
    if (p + 1 >= prompt_end[b] && p + 1 < n_ctx) tok_seq[(size_t)b * n_ctx + p + 1] = next;
    pos[b] = p + 1;
}

constexpr int kMaxBatch = 16;

}  // namespace

struct sllm_cuda_tp_batch {
    const sllm_cuda_tp_model* m = nullptr;
    sllm_cuda_tp_comm* comm = nullptr;
    int B = 0, n_ctx = 0, n_past = 0, head_ctas = 0;
    bool have_logits = false;
    cudaStream_t stream = nullptr;
    float *k_cache = nullptr, *v_cache = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    float *x = nullptr, *ffn_inp = nullptr, *q = nullptr, *k = nullptr, *v = nullptr;
    float *attn_loc = nullptr, *attn_full = nullptr, *h_loc = nullptr, *h_full = nullptr, *gather = nullptr;
    float* logits = nullptr;
    int8_t *qa = nullptr, *qh = nullptr;
    sllm_cuda_act *act_a = nullptr, *act_h = nullptr;
    int32_t *dots_o = nullptr, *dots_d = nullptr;
    float* part_v = nullptr;
    int* part_i = nullptr;
    int* counter = nullptr;
    int32_t *trip = nullptr, *trip_all = nullptr, *argmax = nullptr, *pos = nullptr, *prompt_end = nullptr;
    int32_t* tok_seq = nullptr;
    int32_t* pinned = nullptr;
    cudaGraphExec_t step = nullptr;
    std::vector<void*> allocs;
    cudaEvent_t run_ev[2] = {};
};

namespace {

template <class T>
cudaError_t batch_alloc(sllm_cuda_tp_batch* b, T** p, size_t count) {
    void* v = nullptr;
    const cudaError_t e = dev_malloc(&v, align256(count * sizeof(T)));
    if (e == cudaSuccess) {
        b->allocs.push_back(v);
        *p = static_cast<T*>(v);
    }
    return e;
}

// the exchanges of a batch step (X_ATTN, X_DOTS_O, X_H, X_DOTS_D, X_ARGMAX):
// element counts per rank, and whether they are gathered (else summed)
void bxchg_counts(const sllm_cuda_tp_batch* b, int which, size_t* count, bool* gather) {
    const sllm_cuda_tp_model* m = b->m;
    const size_t B = (size_t)b->B;
    switch (which) {
        case X_ATTN: *count = B * m->hq * kHeadDim; *gather = true; break;
        case X_DOTS_O: *count = B * m->E; *gather = false; break;
        case X_H: *count = B * m->f_loc; *gather = true; break;
        case X_DOTS_D: *count = B * m->E * m->down_c; *gather = false; break;
        default: *count = B * 3; *gather = true; break;
    }
}

void bxchg_buffers(sllm_cuda_tp_batch* b, int which, void** src, void** dst) {
    switch (which) {
        case X_ATTN: *src = b->attn_loc; *dst = b->gather; break;
        case X_DOTS_O: *src = b->dots_o; *dst = b->dots_o; break;
        case X_H: *src = b->h_loc; *dst = b->gather; break;
        case X_DOTS_D: *src = b->dots_d; *dst = b->dots_d; break;
        default: *src = b->trip; *dst = b->trip_all; break;
    }
}

cudaError_t bxchg_nccl(sllm_cuda_tp_batch* b, int which, cudaStream_t st, ncclResult_t* nr) {
    if (b->m->n_ranks == 1) return cudaSuccess;       // one rank: the buffers alias
    size_t count;
    bool gather;
    void *src, *dst;
    bxchg_counts(b, which, &count, &gather);
    bxchg_buffers(b, which, &src, &dst);
    if (gather)
        *nr = nccl()->all_gather(src, dst, count, which == X_ARGMAX ? ncclInt32 : ncclFloat32, b->comm->comm, st);
    else
        *nr = nccl()->all_reduce(src, dst, count, ncclInt32, ncclSum, b->comm->comm, st);
    return *nr == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t bxchg_group(sllm_cuda_tp_batch** bs, int n, int which, cudaStream_t st) {
    if (n == 1) return cudaSuccess;
    size_t count;
    bool gather;
    bxchg_counts(bs[0], which, &count, &gather);
    if (gather) {
        for (int r = 0; r < n; ++r) {
            void *dst, *unused;
            bxchg_buffers(bs[r], which, &unused, &dst);
            for (int s = 0; s < n; ++s) {
                void *src, *unused2;
                bxchg_buffers(bs[s], which, &src, &unused2);
                const cudaError_t e = cudaMemcpyAsync(static_cast<char*>(dst) + (size_t)s * count * 4, src, count * 4,
                                                      cudaMemcpyDeviceToDevice, st);
                if (e != cudaSuccess) return e;
            }
        }
        return cudaSuccess;
    }
    SumArgs a{};
    a.n = n;
    a.count = count;
    for (int r = 0; r < n; ++r) {
        void *src, *dst;
        bxchg_buffers(bs[r], which, &src, &dst);
        a.buf[r] = static_cast<int32_t*>(dst);
    }
    tp_group_sum_kernel<<<64, 256, 0, st>>>(a);
    count_launches(1);
    return cudaGetLastError();
}

template <class K, class... Args>
cudaError_t launch_pdl_k(K kernel, dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr = pdl_attribute();
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

cudaError_t bgemm(const uint8_t* w, const uint8_t* w2, int rows, int K, const int8_t* q, int lda,
                  const sllm_cuda_act* acts, int B, int32_t* dots, float* y, cudaStream_t st) {
    GemmArgs a{};
    a.w = w; a.w2 = w2; a.q = q; a.acts = acts; a.dots = dots; a.y = y;
    a.m = B; a.n_rows = rows; a.K = K; a.lda = lda;
    const char* why = nullptr;
    if (gemm_check(a, &why) != SLLM_CUDA_OK) return cudaErrorInvalidValue;
    return launch_i2s_gemm_skinny(a, gemm_error_word(), st);
}

template <int MODE>
cudaError_t launch_rows_norm_quant(const RowSrc& src, const float* w, int K, float eps, int8_t* q, sllm_cuda_act* act,
                                   int* fb, int force, cudaStream_t st) {
    if (K % (4 * kNqCluster) != 0 || K > 4 * kNqCluster * kNqThreads || src.rows < 1) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = pdl_config(kNqCluster * src.rows, kNqThreads, st);
    cudaLaunchAttribute attr = pdl_attribute();
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tp_rows_norm_quant_kernel<MODE>, src, w, K, eps, 1.0 / (double)K, q, act, fb,
                              force);
}

// phases as the single-sequence step's (n_phases, phase_xchg), B rows each
cudaError_t enqueue_bphase(sllm_cuda_tp_batch* b, int ph, cudaStream_t st) {
    const sllm_cuda_tp_model* m = b->m;
    const int E = m->E, D = kHeadDim, B = b->B, N = m->n_ranks;
    int* fb = fallback_counter();
    const int force = force_fallback_flag();
    auto epi = [&](const int32_t* dots, int chunks, const sllm_cuda_act* act, const uint8_t* w, int rows, int cols,
                   const float* resid, float* y) {
        const float* ws = reinterpret_cast<const float*>(w + (size_t)rows * cols / 4);
        return launch_pdl_k(tp_epilogue_rows_kernel, dim3((rows + 255) / 256, B), dim3(256), st, dots, chunks, B, rows,
                            act, ws, resid, y);
    };
    if (ph == 0) return launch_pdl_k(tp_embed_batch_kernel, dim3(B), dim3(256), st, m->tok_embd,
                                     (const int32_t*)b->tok_seq, (const int32_t*)b->pos, b->n_ctx, E, m->V, b->x);
    if (ph == n_phases(m) - 1) {
        tp_finalize_batch_kernel<<<1, kMaxBatch * 2, 0, st>>>(b->trip_all, N, B, b->pos, b->tok_seq, b->prompt_end,
                                                              b->argmax, b->n_ctx);
        return cudaGetLastError();
    }
    if (ph == n_phases(m) - 2) {
        const TpLayer& t = m->layers[m->n_layer - 1];
        cudaError_t e = epi(b->dots_d, m->down_c, b->act_h, t.down[0], E, m->down_k, b->ffn_inp, b->x);
        if (e != cudaSuccess) return e;
        LmBatchParams lp{};
        lp.x = b->x; lp.norm_w = m->output_norm; lp.eps = m->eps;
        lp.embd = m->tok_embd + (size_t)m->v0 * E;
        lp.E = E; lp.V = m->v_loc; lp.B = B; lp.logits = b->logits;
        lp.part_v = b->part_v; lp.part_i = b->part_i; lp.counter = b->counter; lp.out = b->trip;
        lp.row_base = m->v0; lp.fallback_count = fb; lp.force_fallback = force;
        return launch_lm_head_batch(lp, num_sms_of(m->device), st);
    }
    const int l = (ph - 1) / 4, sub = (ph - 1) % 4;
    const TpLayer& t = m->layers[l];
    cudaError_t e = cudaSuccess;
    RowSrc rs{};
    rs.rows = B;
    if (sub == 0) {
        if (l > 0) {
            const TpLayer& tp = m->layers[l - 1];
            e = epi(b->dots_d, m->down_c, b->act_h, tp.down[0], E, m->down_k, b->ffn_inp, b->x);
            if (e != cudaSuccess) return e;
        }
        // attn_norm -> local Q, K, V for every sequence (src/forward.c:631-666)
        e = launch_norm_quant_rows(b->x, t.attn_norm, E, m->eps, B, b->qa, b->act_a, fb, force, st);
        if (e == cudaSuccess) {
            const SkinnySeg segs[3] = {{t.wq, nullptr, m->hq * D, 0, nullptr, b->q},
                                       {t.wk, nullptr, m->hk * D, 0, nullptr, b->k},
                                       {t.wv, nullptr, m->hk * D, 0, nullptr, b->v}};
            e = launch_i2s_gemm_skinny_segs(segs, 3, b->qa, 0, B, E, b->act_a, gemm_error_word(), st);
        }
        if (e != cudaSuccess) return e;
        const size_t kv_layer = (size_t)m->hk * D * (size_t)b->n_ctx;
        AttnParams ap{};
        ap.q = b->q; ap.k = b->k; ap.v = b->v;
        ap.k_cache = b->k_cache + (size_t)l * kv_layer;
        ap.v_cache = b->v_cache + (size_t)l * kv_layer;
        ap.rope_cos = b->rope_cos; ap.rope_sin = b->rope_sin;
        ap.out = b->attn_loc; ap.n_ctx = b->n_ctx;
        ap.group = m->hq / m->hk;
        ap.attn_scale = 1.0f / sqrtf((float)D);
        ap.fallback_count = fb; ap.force_fallback = force;
        const size_t seq_stride = (size_t)m->n_layer * kv_layer * sizeof(float);
        e = launch_chunk_kv_store(ap, b->pos, B, m->hk, m->hq * D, m->hk * D, st, seq_stride);
        if (e == cudaSuccess) e = launch_attention_chunk(ap, b->pos, B, m->hq, m->hq * D, m->hk * D, st, seq_stride);
        return e;
    }
    if (sub == 1) {
        // attn_sub_norm + quantisation of every whole attention output, then
        // this rank's columns of O (src/forward.c:728-741)
        if (N > 1)
            e = launch_pdl_k(tp_unshard_kernel, dim3(148), dim3(256), st, (const float*)b->gather, b->attn_full, N, B,
                             m->hq * D);
        if (e == cudaSuccess)
            e = launch_norm_quant_rows(b->attn_full, t.attn_sub_norm, E, m->eps, B, b->qa, b->act_a, fb, force, st);
        if (e == cudaSuccess)
            e = bgemm(t.wo, nullptr, E, m->e_loc, b->qa + (size_t)m->rank * m->e_loc, E, b->act_a, B, b->dots_o,
                      nullptr, st);
        return e;
    }
    if (sub == 2) {
        // O epilogue + residual, ffn_norm -> local gate, up -> h (src/forward.c:742-779)
        e = epi(b->dots_o, 1, b->act_a, t.wo, E, m->e_loc, b->x, b->ffn_inp);
        if (e == cudaSuccess)
            e = launch_norm_quant_rows(b->ffn_inp, t.ffn_norm, E, m->eps, B, b->qa, b->act_a, fb, force, st);
        if (e == cudaSuccess) e = bgemm(t.gate, t.up, m->f_loc, E, b->qa, 0, b->act_a, B, nullptr, b->h_loc, st);
        return e;
    }
    // ffn_sub_norm + quantisation of all of h, this rank's columns of down,
    // chunk by chunk (src/forward.c:781-792)
    if (N > 1) {
        rs.g = b->gather; rs.c = m->f_loc; rs.out = b->h_full;
        e = launch_rows_norm_quant<RS_GATHER>(rs, t.ffn_sub_norm, m->F, m->eps, b->qh, b->act_h, fb, force, st);
    } else {
        e = launch_norm_quant(b->h_full, t.ffn_sub_norm, m->F, m->eps, b->qh, b->act_h, fb, force, st, XWait{}, B);
    }
    if (e == cudaSuccess) {
        // the column chunks of down as the segments of one launch
        SkinnySeg segs[4];
        for (int ch = 0; ch < m->down_c; ++ch)
            segs[ch] = SkinnySeg{t.down[ch], nullptr, E, m->rank * m->f_loc + ch * m->down_k,
                                 b->dots_d + (size_t)ch * B * E, nullptr};
        e = launch_i2s_gemm_skinny_segs(segs, m->down_c, b->qh, m->F, B, m->down_k, b->act_h, gemm_error_word(), st);
    }
    return e;
}

int ensure_batch_graph(sllm_cuda_tp_batch* b) {
    if (b->step != nullptr) return SLLM_CUDA_OK;
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    cudaError_t e = cudaSuccess;
    ncclResult_t nr = ncclSuccess;
    for (int ph = 0; ph < n_phases(b->m) && e == cudaSuccess; ++ph) {
        e = enqueue_bphase(b, ph, b->stream);
        const int x = phase_xchg(b->m, ph);
        if (e == cudaSuccess && x >= 0) e = bxchg_nccl(b, x, b->stream, &nr);
    }
    const cudaError_t e2 = cudaStreamEndCapture(b->stream, &g);
    if (nr != ncclSuccess) { if (g) cudaGraphDestroy(g); return fail(SLLM_CUDA_ERR_COMM, "batch step: %s", nccl_err(nr)); }
    if (e != cudaSuccess) { if (g) cudaGraphDestroy(g); return cuda_fail(e, "capture batch step"); }
    if (e2 != cudaSuccess) return cuda_fail(e2, "end capture");
    e = instantiate(&b->step, g);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { b->step = nullptr; return cuda_fail(e, "instantiate batch step"); }
    return SLLM_CUDA_OK;
}

int batch_validate(const sllm_cuda_tp_batch* b, const int32_t* prompts, int32_t n_prompt, int32_t n_new,
                   const int32_t* out) {
    if (b == nullptr || (out == nullptr && n_new > 0) || n_prompt < 0 || n_new < 0 ||
        (n_prompt > 0 && prompts == nullptr))
        return fail(SLLM_CUDA_ERR_ARG, "tp_batch_generate: bad arguments");
    if (n_prompt == 0 && b->n_past == 0 && n_new > 0)
        return fail(SLLM_CUDA_ERR_ARG, "tp_batch_generate: the first call needs a prompt for every sequence");
    if ((int64_t)n_prompt + n_new + b->n_past > b->n_ctx)
        return fail(SLLM_CUDA_ERR_TOO_LARGE, "tp_batch_generate: %d + %d tokens after %d exceed n_ctx %d", n_prompt,
                    n_new, b->n_past, b->n_ctx);
    for (int64_t i = 0; i < (int64_t)n_prompt * b->B; ++i)
        if (prompts[i] < 0 || prompts[i] >= b->m->V)
            return fail(SLLM_CUDA_ERR_ARG, "tp_batch_generate: token %d out of range", prompts[i]);
    return SLLM_CUDA_OK;
}

int batch_seed(sllm_cuda_tp_batch* b, const int32_t* prompts, int32_t n_prompt, cudaStream_t st) {
    const int base = b->n_past;
    if (n_prompt > 0)
        CK(cudaMemcpy2DAsync(b->tok_seq + base, (size_t)b->n_ctx * 4, prompts, (size_t)n_prompt * 4,
                             (size_t)n_prompt * 4, (size_t)b->B, cudaMemcpyHostToDevice, st),
           "prompts");
    for (int i = 0; i < b->B; ++i) {
        b->pinned[i] = base;
        b->pinned[kMaxBatch + i] = base + n_prompt;
    }
    CK(cudaMemcpyAsync(b->pos, b->pinned, (size_t)b->B * 4, cudaMemcpyHostToDevice, st), "positions");
    CK(cudaMemcpyAsync(b->prompt_end, b->pinned + kMaxBatch, (size_t)b->B * 4, cudaMemcpyHostToDevice, st),
       "prompt ends");
    return SLLM_CUDA_OK;
}

int batch_sync(sllm_cuda_tp_batch* b, double seconds) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t e = cudaStreamQuery(b->stream);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(e, "batch step");
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > seconds) {
            if (b->comm != nullptr && b->comm->comm != nullptr) {
                nccl()->comm_abort(b->comm->comm);
                b->comm->comm = nullptr;
            }
            return fail(SLLM_CUDA_ERR_TIMEOUT, "batch step: no progress in %.0f s (communicator aborted)", seconds);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    return SLLM_CUDA_OK;
}

int batch_gemm_status() {
    int* w = gemm_error_word();
    int v = 0;
    if (w != nullptr && cudaMemcpy(&v, w, 4, cudaMemcpyDeviceToHost) == cudaSuccess && v != 0) {
        cudaMemset(w, 0, 4);
        return fail(SLLM_CUDA_ERR_TIMEOUT, "batch step: a GEMM wait gave up (code %d)", v);
    }
    return SLLM_CUDA_OK;
}

}  // namespace

extern "C" int sllm_cuda_tp_batch_new(const sllm_cuda_tp_model* m, sllm_cuda_tp_comm* comm, int32_t n_seq,
                                      int32_t n_ctx, sllm_cuda_tp_batch** out) {
    if (m == nullptr || out == nullptr || n_seq < 1 || n_seq > kMaxBatch || n_ctx < 1 || n_ctx > attention_max_ctx())
        return fail(SLLM_CUDA_ERR_ARG, "tp_batch_new: bad arguments (n_seq %d, n_ctx %d)", n_seq, n_ctx);
    *out = nullptr;
    if (comm != nullptr && (comm->n_ranks != m->n_ranks || comm->rank != m->rank || comm->device != m->device))
        return fail(SLLM_CUDA_ERR_ARG, "tp_batch_new: the communicator's rank does not match the shard's");
    if (m->E > 8192 || m->E % 128 != 0 || m->F % 32 != 0 || m->F > 32768 || m->down_c > 4)
        return fail(SLLM_CUDA_ERR_UNSUPPORTED, "tp_batch_new: widths %d / %d", m->E, m->F);
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    CK(prepare_decode_kernels(), "decode kernel attributes");
    if (fallback_counter() == nullptr || gemm_error_word() == nullptr)
        return fail(SLLM_CUDA_ERR_NOMEM, "tp_batch_new: diagnostics words");
    auto* b = new sllm_cuda_tp_batch();
    b->m = m;
    b->comm = comm;
    b->B = n_seq;
    b->n_ctx = n_ctx;
    b->head_ctas = lm_head_batch_ctas(n_seq, num_sms_of(m->device));
    const int D = kHeadDim, E = m->E, N = m->n_ranks;
    const size_t B = (size_t)n_seq;
    const size_t kv = B * m->n_layer * m->hk * D * n_ctx;
    cudaError_t e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
    if (!e) e = batch_alloc(b, &b->k_cache, kv);
    if (!e) e = batch_alloc(b, &b->v_cache, kv);
    if (!e) e = batch_alloc(b, &b->rope_cos, (size_t)n_ctx * D / 2);
    if (!e) e = batch_alloc(b, &b->rope_sin, (size_t)n_ctx * D / 2);
    if (!e) e = batch_alloc(b, &b->x, B * E);
    if (!e) e = batch_alloc(b, &b->ffn_inp, B * E);
    if (!e) e = batch_alloc(b, &b->q, B * m->hq * D);
    if (!e) e = batch_alloc(b, &b->k, B * m->hk * D);
    if (!e) e = batch_alloc(b, &b->v, B * m->hk * D);
    if (!e) e = batch_alloc(b, &b->attn_loc, B * m->hq * D);
    if (!e) e = batch_alloc(b, &b->h_loc, B * m->f_loc);
    if (N > 1) {
        if (!e) e = batch_alloc(b, &b->attn_full, B * E);
        if (!e) e = batch_alloc(b, &b->h_full, B * m->F);
        if (!e) e = batch_alloc(b, &b->gather, (size_t)N * B * std::max(m->hq * D, m->f_loc));
        if (!e) e = batch_alloc(b, &b->trip_all, (size_t)N * B * 3);
    }
    if (!e) e = batch_alloc(b, &b->logits, B * (size_t)(m->v_loc > 0 ? m->v_loc : 1));
    if (!e) e = batch_alloc(b, &b->qa, B * E);
    if (!e) e = batch_alloc(b, &b->qh, B * m->F);
    if (!e) e = batch_alloc(b, &b->act_a, B);
    if (!e) e = batch_alloc(b, &b->act_h, B);
    if (!e) e = batch_alloc(b, &b->dots_o, B * E);
    if (!e) e = batch_alloc(b, &b->dots_d, B * E * m->down_c);
    if (!e) e = batch_alloc(b, &b->part_v, B * b->head_ctas);
    if (!e) e = batch_alloc(b, &b->part_i, B * b->head_ctas);
    if (!e) e = batch_alloc(b, &b->counter, 1);
    if (!e) e = batch_alloc(b, &b->trip, B * 3);
    if (!e) e = batch_alloc(b, &b->argmax, B);
    if (!e) e = batch_alloc(b, &b->pos, B);
    if (!e) e = batch_alloc(b, &b->prompt_end, B);
    if (!e) e = batch_alloc(b, &b->tok_seq, B * n_ctx);
    if (!e) e = cudaMallocHost(&b->pinned, 2 * kMaxBatch * sizeof(int32_t));
    if (!e) e = cudaEventCreate(&b->run_ev[0]);
    if (!e) e = cudaEventCreate(&b->run_ev[1]);
    if (!e) e = cudaMemset(b->counter, 0, 4);
    if (!e) e = cudaMemset(b->tok_seq, 0, B * n_ctx * 4);
    if (!e && N == 1) {
        // one rank: nothing is gathered, the local buffers are the whole ones
        b->attn_full = b->attn_loc;
        b->h_full = b->h_loc;
        b->trip_all = b->trip;
    }
    if (!e) {
        std::vector<float> cs, sn;
        rope_table(n_ctx, D, m->rope_base, cs, sn);
        e = cudaMemcpy(b->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
        if (!e) e = cudaMemcpy(b->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        sllm_cuda_tp_batch_free(b);
        return cuda_fail(e, "tp_batch_new");
    }
    *out = b;
    return SLLM_CUDA_OK;
}

extern "C" void sllm_cuda_tp_batch_free(sllm_cuda_tp_batch* b) {
    if (b == nullptr) return;
    cudaSetDevice(b->m->device);
    graph_exec_destroy(b->step);
    if (b->stream) cudaStreamDestroy(b->stream);
    for (void* p : b->allocs) cudaFree(p);
    if (b->pinned) cudaFreeHost(b->pinned);
    for (cudaEvent_t ev : b->run_ev)
        if (ev) cudaEventDestroy(ev);
    delete b;
}

extern "C" int sllm_cuda_tp_batch_reset(sllm_cuda_tp_batch* b) {
    if (b == nullptr) return fail(SLLM_CUDA_ERR_ARG, "tp_batch_reset: null");
    b->n_past = 0;
    b->have_logits = false;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_tp_batch_generate_greedy(sllm_cuda_tp_batch* b, const int32_t* prompts, int32_t n_prompt,
                                                  int32_t n_new, int32_t* out) {
    int rc = batch_validate(b, prompts, n_prompt, n_new, out);
    if (rc != SLLM_CUDA_OK) return rc;
    if (n_prompt == 0 && n_new == 0) return SLLM_CUDA_OK;
    CK(cudaSetDevice(b->m->device), "cudaSetDevice");
    if (b->m->n_ranks > 1 && (b->comm == nullptr || b->comm->comm == nullptr))
        return fail(SLLM_CUDA_ERR_COMM, "tp_batch_generate: no communicator");
    rc = ensure_batch_graph(b);
    if (rc != SLLM_CUDA_OK) return rc;
    const int base = b->n_past;
    rc = batch_seed(b, prompts, n_prompt, b->stream);
    if (rc != SLLM_CUDA_OK) return rc;
    const int steps = n_prompt + n_new;
    CK(cudaEventRecord(b->run_ev[0], b->stream), "run timer");
    for (int s = 0; s < steps; ++s) CK(graph_launch(b->step, b->stream), "batch step");
    CK(cudaEventRecord(b->run_ev[1], b->stream), "run timer");
    if (n_new > 0)
        CK(cudaMemcpy2DAsync(out, (size_t)n_new * 4, b->tok_seq + base + n_prompt, (size_t)b->n_ctx * 4,
                             (size_t)n_new * 4, (size_t)b->B, cudaMemcpyDeviceToHost, b->stream),
           "ids");
    rc = batch_sync(b, 120.0);
    if (rc != SLLM_CUDA_OK) return rc;
    rc = batch_gemm_status();
    if (rc != SLLM_CUDA_OK) return rc;
    b->n_past = base + steps;
    b->have_logits = true;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_tp_batch_last_logits(const sllm_cuda_tp_batch* b, int32_t seq, float* host_out) {
    if (b == nullptr || host_out == nullptr || seq < 0 || seq >= b->B)
        return fail(SLLM_CUDA_ERR_ARG, "tp_batch_last_logits: bad arguments");
    if (!b->have_logits) return fail(SLLM_CUDA_ERR_ARG, "tp_batch_last_logits: nothing forwarded");
    CK(cudaSetDevice(b->m->device), "cudaSetDevice");
    CK(cudaMemcpy(host_out, b->logits + (size_t)seq * b->m->v_loc, (size_t)b->m->v_loc * 4, cudaMemcpyDeviceToHost),
       "logits");
    return SLLM_CUDA_OK;
}

extern "C" float sllm_cuda_test_tp_batch_last_run_ms(const sllm_cuda_tp_batch* b) {
    float ms = -1.0f;
    if (b == nullptr || cudaEventElapsedTime(&ms, b->run_ev[0], b->run_ev[1]) != cudaSuccess) return -1.0f;
    return ms;
}

extern "C" int sllm_cuda_test_tp_batch_generate_group(sllm_cuda_tp_batch** bs, int32_t n, const int32_t* prompts,
                                                      int32_t n_prompt, int32_t n_new, int32_t* out) {
    if (bs == nullptr || n < 1 || n > kMaxRanks) return fail(SLLM_CUDA_ERR_ARG, "tp batch group: bad arguments");
    for (int r = 0; r < n; ++r) {
        if (bs[r] == nullptr || bs[r]->m->n_ranks != n || bs[r]->m->rank != r ||
            bs[r]->m->device != bs[0]->m->device || bs[r]->n_past != bs[0]->n_past || bs[r]->n_ctx != bs[0]->n_ctx ||
            bs[r]->B != bs[0]->B)
            return fail(SLLM_CUDA_ERR_ARG, "tp batch group: not ranks 0..%d of one model and batch on one device", n - 1);
        const int rc = batch_validate(bs[r], prompts, n_prompt, n_new, out);
        if (rc != SLLM_CUDA_OK) return rc;
    }
    if (n_prompt == 0 && n_new == 0) return SLLM_CUDA_OK;
    CK(cudaSetDevice(bs[0]->m->device), "cudaSetDevice");
    cudaStream_t st = bs[0]->stream;
    for (int r = 0; r < n; ++r) {
        const int rc = batch_seed(bs[r], prompts, n_prompt, st);
        if (rc != SLLM_CUDA_OK) return rc;
    }
    const int base = bs[0]->n_past, steps = n_prompt + n_new;
    for (int s = 0; s < steps; ++s) {
        for (int ph = 0; ph < n_phases(bs[0]->m); ++ph) {
            for (int r = 0; r < n; ++r) CK(enqueue_bphase(bs[r], ph, st), "tp batch group phase");
            const int x = phase_xchg(bs[0]->m, ph);
            if (x >= 0) CK(bxchg_group(bs, n, x, st), "tp batch group exchange");
        }
    }
    if (n_new > 0)
        CK(cudaMemcpy2DAsync(out, (size_t)n_new * 4, bs[0]->tok_seq + base + n_prompt, (size_t)bs[0]->n_ctx * 4,
                             (size_t)n_new * 4, (size_t)bs[0]->B, cudaMemcpyDeviceToHost, st),
           "ids");
    CK(cudaStreamSynchronize(st), "tp batch group sync");
    const int rc = batch_gemm_status();
    if (rc != SLLM_CUDA_OK) return rc;
    for (int r = 0; r < n; ++r) {
        bs[r]->n_past = base + steps;
        bs[r]->have_logits = true;
    }
    return SLLM_CUDA_OK;
}
