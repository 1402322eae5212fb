// decode.cu -- the non-GEMV kernels of one bitnet-b1.58 decode step on
// sm_100a: embedding lookup, RoPE + KV store + attention, and the tied F16
// lm_head fused with the greedy argmax and the step's position update.
//
// Every floating-point reduction here reproduces saphira-llm's CPU order
// exactly (src/forward.c:621-835, src/ops.c:106-154, 386-422, 467-551):
// attention dot products and the P.V sums are sequential per output in the
// reference's index order; the softmax f64 sum is computed in parallel and
// certified (with a reference-order fallback); the lm_head keeps the
// reference's 32 FMA chains per row and its reduction tree.

#include "common.cuh"
#include "decode.cuh"
#include "libm_expf.h"
#include <algorithm>

#include "attn.cuh"

namespace sllm {

__device__ __forceinline__ void pdl_trigger_d() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_d() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... Args, typename Kern>
static cudaError_t launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// ---------------------------------------------------------------------------
// embedding: x = f16_to_f32(tok_embd[token]) (src/forward.c:621-626)
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const uint16_t* __restrict__ tok_embd, const int32_t* __restrict__ tok_seq,
                             const int32_t* __restrict__ pos_ptr, int E, int V, float* __restrict__ x,
                             unsigned* reset_word) {
    if (reset_word != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *reset_word = 0u;
    int tok = tok_seq[*pos_ptr];
    // the host validates every token it writes and the argmax is in range;
    // this only keeps a corrupted id from reading outside the table
    if ((unsigned)tok >= (unsigned)V) tok = 0;
    const uint16_t* row = tok_embd + (size_t)tok * (size_t)E;
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < E; d += gridDim.x * blockDim.x)
        x[d] = f16_embd(row[d]);
}

// the embeddings of n tokens, one CTA per token
__global__ void embed_rows_kernel(const uint16_t* __restrict__ tok_embd, const int32_t* __restrict__ tok_seq, int E,
                                  int V, float* __restrict__ x) {
    pdl_wait_d();
    int tok = tok_seq[blockIdx.x];
    if ((unsigned)tok >= (unsigned)V) tok = 0;
    const uint16_t* row = tok_embd + (size_t)tok * (size_t)E;
    float* xr = x + (size_t)blockIdx.x * E;
    for (int d = threadIdx.x; d < E; d += blockDim.x) xr[d] = f16_embd(row[d]);
}

// RoPE NEOX on the k of every token of a chunk and the store of k and v at
// its position, exactly as attention_head does for one position (the same
// products and sums, the same rounding of an f16 cache); one CTA of 128
// threads per (token, kv head)
__global__ void chunk_kv_store_kernel(const AttnParams p, const int32_t* __restrict__ pos_arr, int E, int G,
                                      size_t seq_stride) {
    pdl_wait_d();
    const int t = blockIdx.x, kvh = blockIdx.y, i = threadIdx.x;
    const int pos = pos_arr[t];
    const int nctx = p.n_ctx;
    const float* kr = p.k + (size_t)t * G + kvh * kHeadDim;
    const float* vr = p.v + (size_t)t * G + kvh * kHeadDim;
    const bool f16 = (p.kv_f16 & kAttnKvF16) != 0;
    const size_t elt = f16 ? 2 : 4;
    // token t's sequence: the same cache for a chunk, its own for a batch
    char* kT = reinterpret_cast<char*>(p.k_cache) + (size_t)t * seq_stride + (size_t)kvh * kHeadDim * nctx * elt;
    char* vC = reinterpret_cast<char*>(p.v_cache) + (size_t)t * seq_stride + (size_t)kvh * nctx * kHeadDim * elt;
    float k;
    if (i < kHeadDim / 2) {
        const float c = p.rope_cos[(size_t)pos * (kHeadDim / 2) + i], s = p.rope_sin[(size_t)pos * (kHeadDim / 2) + i];
        k = __fsub_rn(__fmul_rn(kr[i], c), __fmul_rn(kr[i + 64], s));
    } else {
        const int j = i - 64;
        const float c = p.rope_cos[(size_t)pos * (kHeadDim / 2) + j], s = p.rope_sin[(size_t)pos * (kHeadDim / 2) + j];
        k = __fadd_rn(__fmul_rn(kr[j], s), __fmul_rn(kr[j + 64], c));
    }
    const float v = vr[i];
    if (f16) {
        reinterpret_cast<__half*>(kT)[(size_t)i * nctx + pos] = __float2half_rn(k);
        reinterpret_cast<__half*>(vC)[(size_t)pos * kHeadDim + i] = __float2half_rn(v);
    } else {
        reinterpret_cast<float*>(kT)[(size_t)i * nctx + pos] = k;
        reinterpret_cast<float*>(vC)[(size_t)pos * kHeadDim + i] = v;
    }
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                           size_t n) {
    pdl_wait_d();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

// ---------------------------------------------------------------------------
// attention for one query position, one CTA per query head
// ---------------------------------------------------------------------------
constexpr int kAttnThreads = 256;

struct CtaSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

__global__ void __launch_bounds__(kAttnThreads)
attention_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float sc[];          // n_ctx scores
    __shared__ float qs[kHeadDim], kcur[kHeadDim];
    __shared__ float fred[32];
    __shared__ double dred[32];
    pdl_trigger_d();
    pdl_wait_d();                 // q, k, v come from the previous kernel
    attention_head<kAttnThreads>(p, blockIdx.x, threadIdx.x, sc, qs, kcur, fred, dred, CtaSync());
}

// every (head, token) of a chunk whose K and V are already in the cache;
// two CTAs per SM (128 registers): a batch step launches 1024 of them
__global__ void __launch_bounds__(kAttnThreads, 2)
attention_chunk_kernel(const __grid_constant__ AttnParams p, const int32_t* __restrict__ pos_arr, int E, int G,
                       size_t seq_stride) {
    extern __shared__ __align__(16) float sc[];
    __shared__ float qs[kHeadDim], kcur[kHeadDim];
    __shared__ float fred[32];
    __shared__ double dred[32];
    // token t's parameters, once per CTA in shared memory (a per-thread copy
    // would sit in local memory: the head body takes them by reference)
    __shared__ AttnParams pt;
    pdl_wait_d();
    const int t = blockIdx.y;
    if (threadIdx.x == 0) {
        pt = p;
        pt.q = p.q + (size_t)t * E;
        pt.k = p.k + (size_t)t * G;
        pt.v = p.v + (size_t)t * G;
        pt.out = p.out + (size_t)t * E;
        pt.pos_ptr = pos_arr + t;
        pt.kv_f16 = p.kv_f16 | kAttnKvStored;
        pt.k_cache = reinterpret_cast<float*>(reinterpret_cast<char*>(p.k_cache) + (size_t)t * seq_stride);
        pt.v_cache = reinterpret_cast<float*>(reinterpret_cast<char*>(p.v_cache) + (size_t)t * seq_stride);
    }
    __syncthreads();
    attention_head<kAttnThreads>(pt, blockIdx.x, threadIdx.x, sc, qs, kcur, fred, dred, CtaSync());
}

// ---------------------------------------------------------------------------
// lm_head + argmax
//
// Four lanes per vocabulary row, eight rows per warp; lane j of a row owns the
// reference's accumulators acc[j][0..7] and reads 16 bytes per step, so a warp
// instruction covers 64 contiguous bytes of each of eight rows. After E/32
// FMA steps the reference's tree (src/ops.c:135-143) runs as two shuffle
// rounds (acc0+=acc2, acc1+=acc3; acc0+=acc1), then t_l = acc0[l] + acc0[l+4]
// and (t0+t1) + (t2+t3) in the row's first lane. A persistent grid of two
// CTAs per SM; the last CTA to finish reduces the per-CTA argmax partials.
// ---------------------------------------------------------------------------
constexpr int kLmThreads = 512;
constexpr int kLmWarps = kLmThreads / 32;

struct Best { float v; int i; };

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    if (isnan(v)) return false;
    if (isnan(bv)) return true;
    return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(kLmThreads)
lm_head_kernel(const LmParams p) {
    extern __shared__ __align__(16) float xs[];                 // E floats: rms_norm(x) * w
    __shared__ double dred[32];
    __shared__ float s_scale;
    __shared__ float bv_s[kLmWarps];
    __shared__ int bi_s[kLmWarps];
    __shared__ int s_last;
    const int E = p.E, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait_d();                 // x comes from the last layer (a no-op in an ordinary launch)

    // output_norm (src/forward.c:805-809), f32, certified mean
    double ss = 0.0;
    for (int i = tid; i < E; i += kLmThreads) {
        const float v = p.x[i];
        xs[i] = v;
        ss = __dadd_rn(ss, (double)__fmul_rn(v, v));
    }
    ss = warp_sum_d(ss);
    if (lane == 0) dred[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        double S = 0.0;
        for (int i = 0; i < kLmWarps; ++i) S = __dadd_rn(S, dred[i]);
        float mean;
        if (!certify_mean_mul(S, E, 1.0 / (double)E, &mean) || p.force_fallback) {
            mean = __double2float_rn(__ddiv_rn(rms_ss_reference_order(xs, E), (double)E));
            if (p.fallback_count != nullptr && blockIdx.x == 0) atomicAdd(p.fallback_count, 1);
        }
        s_scale = rms_scale(mean, p.eps);
    }
    __syncthreads();
    const float sc = s_scale;
    for (int i = tid; i < E; i += kLmThreads) xs[i] = __fmul_rn(__fmul_rn(sc, xs[i]), p.norm_w[i]);
    __syncthreads();

    // Four lanes per vocabulary row, eight rows per warp. Lane j of a row
    // owns the reference's accumulators acc[j][0..7] (src/ops.c:120-130):
    // at step m it loads the 16 bytes of elements 32m + 8j .. 32m + 8j + 7 and
    // runs one FMA chain per element slot, in the reference's order.
    const int sub = lane >> 2, j4 = lane & 3;
    const int nsteps = E >> 5;
    const int ngroups = (p.V + 7) >> 3;
    float bv = NAN;
    int bi = 0x7fffffff;
    constexpr int U = 8;
    for (int grp = blockIdx.x * kLmWarps + warp; grp < ngroups; grp += gridDim.x * kLmWarps) {
        const int row = 8 * grp + sub;
        const bool valid = row < p.V;
        const uint8_t* wrow = reinterpret_cast<const uint8_t*>(p.embd + (size_t)(valid ? row : 0) * (size_t)E) + 16 * j4;
        float a[8];
        #pragma unroll
        for (int l = 0; l < 8; ++l) a[l] = 0.0f;
        for (int m0 = 0; m0 < nsteps; m0 += U) {
            uint4 wv[U];
            #pragma unroll
            for (int u = 0; u < U; ++u) wv[u] = (m0 + u < nsteps) ? ld_stream_u128(wrow + 64 * (m0 + u)) : make_uint4(0, 0, 0, 0);
            #pragma unroll
            for (int u = 0; u < U; ++u) {
                if (m0 + u < nsteps) {
                    const float4* xv = reinterpret_cast<const float4*>(xs + 32 * (m0 + u) + 8 * j4);
                    const float4 x0 = xv[0], x1 = xv[1];
                    const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv[u].x));
                    const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv[u].y));
                    const float2 w45 = __half22float2(*reinterpret_cast<const __half2*>(&wv[u].z));
                    const float2 w67 = __half22float2(*reinterpret_cast<const __half2*>(&wv[u].w));
                    a[0] = __fmaf_rn(w01.x, x0.x, a[0]);
                    a[1] = __fmaf_rn(w01.y, x0.y, a[1]);
                    a[2] = __fmaf_rn(w23.x, x0.z, a[2]);
                    a[3] = __fmaf_rn(w23.y, x0.w, a[3]);
                    a[4] = __fmaf_rn(w45.x, x1.x, a[4]);
                    a[5] = __fmaf_rn(w45.y, x1.y, a[5]);
                    a[6] = __fmaf_rn(w67.x, x1.z, a[6]);
                    a[7] = __fmaf_rn(w67.y, x1.w, a[7]);
                }
            }
        }
        // the reference's tree (src/ops.c:135-143): acc0 += acc2, acc1 += acc3
        // (lanes j4 = 0, 1 add lanes 2, 3), then acc0 += acc1, then
        // t_l = acc0[l] + acc0[l + 4] and (t0 + t1) + (t2 + t3)
        #pragma unroll
        for (int l = 0; l < 8; ++l) a[l] = __fadd_rn(a[l], __shfl_down_sync(0xffffffffu, a[l], 2));
        #pragma unroll
        for (int l = 0; l < 8; ++l) a[l] = __fadd_rn(a[l], __shfl_down_sync(0xffffffffu, a[l], 1));
        const float t0 = __fadd_rn(a[0], a[4]), t1 = __fadd_rn(a[1], a[5]);
        const float t2 = __fadd_rn(a[2], a[6]), t3 = __fadd_rn(a[3], a[7]);
        const float logit = __fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3));
        if (j4 == 0 && valid) {
            p.logits[row] = logit;
            if (better(logit, row, bv, bi)) { bv = logit; bi = row; }
        }
    }
    // argmax: warp, CTA, then the last CTA over all CTAs
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { bv_s[warp] = bv; bi_s[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kLmWarps; ++w) if (better(bv_s[w], bi_s[w], bv, bi)) { bv = bv_s[w]; bi = bi_s[w]; }
        p.part_v[blockIdx.x] = bv;
        p.part_i[blockIdx.x] = bi;
        __threadfence();
        const int done = atomicAdd(p.counter, 1);
        s_last = (done == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    // the last CTA: every thread takes a stride of the per-CTA partials, then
    // a warp and a CTA reduction (the order of candidates is irrelevant: ties
    // resolve to the lowest index)
    __threadfence();
    bv = NAN;
    bi = 0x7fffffff;
    for (int b = tid; b < (int)gridDim.x; b += kLmThreads) {
        const float v = __ldcg(&p.part_v[b]);
        const int i = __ldcg(&p.part_i[b]);
        if (better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    __syncthreads();              // bv_s / bi_s reused
    if (lane == 0) { bv_s[warp] = bv; bi_s[warp] = bi; }
    __syncthreads();
    if (tid != 0) return;
    for (int w = 1; w < kLmWarps; ++w) if (better(bv_s[w], bi_s[w], bv, bi)) { bv = bv_s[w]; bi = bi_s[w]; }
    if (p.tp_out != nullptr) {
        p.tp_out[0] = __float_as_int(bv);
        p.tp_out[1] = bi == 0x7fffffff ? 0x7fffffff : bi + p.row_base;
        p.tp_out[2] = isnan(*(volatile const float*)&p.logits[0]) ? 1 : 0;
        *p.counter = 0;
        return;
    }
    // first index of the maximum with '>' (src/forward.c:876-883): a NaN at
    // index 0 wins outright, a NaN elsewhere never does
    int next = bi;
    if (bi == 0x7fffffff || isnan(*(volatile const float*)&p.logits[0])) next = 0;
    *p.counter = 0;
    *p.argmax_out = next;
    // greedy feedback and the position advance of the step
    const int pos = *p.pos_ptr;
    if (pos + 1 >= *p.prompt_end && pos + 1 < p.n_ctx) p.tok_seq[pos + 1] = next;
    if (p.argmax_hist != nullptr) p.argmax_hist[pos] = next;
    *p.pos_ptr = pos + 1;
}

// ---------------------------------------------------------------------------
// lm_head of a batch of sequences: CTA (g, c) takes tokens [g T, g T + T) and
// the row groups c, c + G, ... of the slice, so the T-token groups of one row
// range run side by side and share its table reads in L2. Each token's
// output_norm and each row's four-lane FMA chains and tree are lm_head_kernel's,
// token by token; the last CTA reduces every token's per-CTA bests and writes
// {best value bits, best global row, isnan(logits[b][0])} per token (the
// slice's candidate; the argmax across slices and the feedback are the
// caller's, as for a tensor-parallel slice above).
// ---------------------------------------------------------------------------
constexpr int kLmbTokens = 4;
constexpr int kLmbRows = 2;         // R: groups of eight rows a warp takes per iteration

// the weight ring of lm_head_batch_kernel: D steps x R rows x one 16-byte slot
// per thread, behind the T x E floats of normalised activations
__host__ __device__ constexpr size_t lm_head_batch_smem(int E, int D) {
    return (size_t)kLmbTokens * (size_t)E * sizeof(float) + (size_t)D * kLmbRows * kLmThreads * 16u;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// D: depth of the weight ring. Each thread copies its own 16-byte pieces of
// the table into its own slots (cp.async) and reads them back after its own
// wait, so no other thread is involved; D - 1 steps of copies stay in flight
// per thread without holding registers (a register prefetch of one step left
// the kernel waiting on the table's latency).
template <int D>
__global__ void __launch_bounds__(kLmThreads)
lm_head_batch_kernel(const LmBatchParams p) {
    constexpr int T = kLmbTokens;
    extern __shared__ __align__(16) float xs[];                 // T x E floats, then the weight ring
    __shared__ double dred[32];
    __shared__ float s_scale;
    __shared__ float bv_s[T][kLmWarps];
    __shared__ int bi_s[T][kLmWarps];
    __shared__ int s_last;
    const int E = p.E, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.x * T, nt = min(T, p.B - t0);
    const int ncta = gridDim.y, cta = blockIdx.y;
    pdl_wait_d();
    for (int t = 0; t < T; ++t) {
        float* xt = xs + (size_t)t * E;
        if (t >= nt) {
            for (int i = tid; i < E; i += kLmThreads) xt[i] = 0.0f;
            continue;
        }
        const float* xg = p.x + (size_t)(t0 + t) * E;
        double ss = 0.0;
        for (int i = tid; i < E; i += kLmThreads) {
            const float v = xg[i];
            xt[i] = v;
            ss = __dadd_rn(ss, (double)__fmul_rn(v, v));
        }
        ss = warp_sum_d(ss);
        if (lane == 0) dred[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            double S = 0.0;
            for (int i = 0; i < kLmWarps; ++i) S = __dadd_rn(S, dred[i]);
            float mean;
            if (!certify_mean_mul(S, E, 1.0 / (double)E, &mean) || p.force_fallback) {
                mean = __double2float_rn(__ddiv_rn(rms_ss_reference_order(xt, E), (double)E));
                if (p.fallback_count != nullptr && cta == 0) atomicAdd(p.fallback_count, 1);
            }
            s_scale = rms_scale(mean, p.eps);
        }
        __syncthreads();
        const float sc = s_scale;
        for (int i = tid; i < E; i += kLmThreads) xt[i] = __fmul_rn(__fmul_rn(sc, xt[i]), p.norm_w[i]);
        __syncthreads();
    }

    const int sub = lane >> 2, j4 = lane & 3;
    const int nsteps = E >> 5;
    // R groups of eight rows per warp iteration: each lane's x loads serve R rows
    constexpr int R = kLmbRows;
    uint4* ring = reinterpret_cast<uint4*>(xs + (size_t)T * E) + tid;   // slot (d, r): ring[(d R + r) kLmThreads]
    const int ngroups = (p.V + 8 * R - 1) / (8 * R);
    float bv[T];
    int bi[T];
    #pragma unroll
    for (int t = 0; t < T; ++t) { bv[t] = NAN; bi[t] = 0x7fffffff; }
    for (int grp = cta * kLmWarps + warp; grp < ngroups; grp += ncta * kLmWarps) {
        int rows[R];
        bool valid[R];
        const uint8_t* wrow[R];
        #pragma unroll
        for (int r = 0; r < R; ++r) {
            rows[r] = 8 * (R * grp + r) + sub;
            valid[r] = rows[r] < p.V;
            wrow[r] = reinterpret_cast<const uint8_t*>(p.embd + (size_t)(valid[r] ? rows[r] : 0) * (size_t)E) + 16 * j4;
        }
        float a[R][T][8];
        #pragma unroll
        for (int r = 0; r < R; ++r)
            #pragma unroll
            for (int t = 0; t < T; ++t)
                #pragma unroll
                for (int l = 0; l < 8; ++l) a[r][t][l] = 0.0f;
        // steps 0 .. D-2 in flight; one commit group per step (empty past the row's end)
        #pragma unroll
        for (int m = 0; m < D - 1; ++m) {
            if (m < nsteps) {
                #pragma unroll
                for (int r = 0; r < R; ++r) cp_async16(ring + (m * R + r) * kLmThreads, wrow[r] + 64 * m);
            }
            cp_async_commit();
        }
        for (int m0 = 0; m0 < nsteps; ++m0) {
            // the slot of step m0 + D - 1 last held step m0 - 1, whose reads
            // this thread finished before its FMAs of the previous iteration
            const int mf = m0 + D - 1;
            if (mf < nsteps) {
                const int sf = mf % D;
                #pragma unroll
                for (int r = 0; r < R; ++r) cp_async16(ring + (sf * R + r) * kLmThreads, wrow[r] + 64 * mf);
            }
            cp_async_commit();
            cp_async_wait<D - 1>();         // step m0's group is complete
            const int sc = m0 % D;
            float w[R][8];
            #pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint4 wv = ring[(sc * R + r) * kLmThreads];
                const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
                const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
                const float2 w45 = __half22float2(*reinterpret_cast<const __half2*>(&wv.z));
                const float2 w67 = __half22float2(*reinterpret_cast<const __half2*>(&wv.w));
                w[r][0] = w01.x; w[r][1] = w01.y; w[r][2] = w23.x; w[r][3] = w23.y;
                w[r][4] = w45.x; w[r][5] = w45.y; w[r][6] = w67.x; w[r][7] = w67.y;
            }
            #pragma unroll
            for (int t = 0; t < T; ++t) {
                const float4* xv = reinterpret_cast<const float4*>(xs + (size_t)t * E + 32 * m0 + 8 * j4);
                const float4 x0 = xv[0], x1 = xv[1];
                const float xx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                #pragma unroll
                for (int r = 0; r < R; ++r)
                    #pragma unroll
                    for (int l = 0; l < 8; ++l) a[r][t][l] = __fmaf_rn(w[r][l], xx[l], a[r][t][l]);
            }
        }
        #pragma unroll
        for (int r = 0; r < R; ++r) {
            #pragma unroll
            for (int t = 0; t < T; ++t) {
                // the reference's tree (src/ops.c:135-143), as lm_head_kernel
                #pragma unroll
                for (int l = 0; l < 8; ++l) a[r][t][l] = __fadd_rn(a[r][t][l], __shfl_down_sync(0xffffffffu, a[r][t][l], 2));
                #pragma unroll
                for (int l = 0; l < 8; ++l) a[r][t][l] = __fadd_rn(a[r][t][l], __shfl_down_sync(0xffffffffu, a[r][t][l], 1));
                const float q0 = __fadd_rn(a[r][t][0], a[r][t][4]), q1 = __fadd_rn(a[r][t][1], a[r][t][5]);
                const float q2 = __fadd_rn(a[r][t][2], a[r][t][6]), q3 = __fadd_rn(a[r][t][3], a[r][t][7]);
                const float logit = __fadd_rn(__fadd_rn(q0, q1), __fadd_rn(q2, q3));
                if (j4 == 0 && valid[r] && t < nt) {
                    p.logits[(size_t)(t0 + t) * p.V + rows[r]] = logit;
                    if (better(logit, rows[r], bv[t], bi[t])) { bv[t] = logit; bi[t] = rows[r]; }
                }
            }
        }
    }
    #pragma unroll
    for (int t = 0; t < T; ++t) {
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv[t], o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi[t], o);
            if (better(ov, oi, bv[t], bi[t])) { bv[t] = ov; bi[t] = oi; }
        }
        if (lane == 0) { bv_s[t][warp] = bv[t]; bi_s[t][warp] = bi[t]; }
    }
    __syncthreads();
    if (tid == 0) {
        for (int t = 0; t < nt; ++t) {
            float v = bv_s[t][0];
            int i = bi_s[t][0];
            for (int w = 1; w < kLmWarps; ++w) if (better(bv_s[t][w], bi_s[t][w], v, i)) { v = bv_s[t][w]; i = bi_s[t][w]; }
            p.part_v[(size_t)(t0 + t) * ncta + cta] = v;
            p.part_i[(size_t)(t0 + t) * ncta + cta] = i;
        }
        __threadfence();
        const int done = atomicAdd(p.counter, 1);
        s_last = (done == (int)(gridDim.x * gridDim.y) - 1);
    }
    __syncthreads();
    if (!s_last) return;
    // the last CTA: each token's per-CTA partials, one warp per token
    __threadfence();
    for (int b = warp; b < p.B; b += kLmWarps) {
        float v = NAN;
        int i = 0x7fffffff;
        for (int c = lane; c < ncta; c += 32) {
            const float cv = __ldcg(&p.part_v[(size_t)b * ncta + c]);
            const int ci = __ldcg(&p.part_i[(size_t)b * ncta + c]);
            if (better(cv, ci, v, i)) { v = cv; i = ci; }
        }
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            if (better(ov, oi, v, i)) { v = ov; i = oi; }
        }
        if (lane == 0) {
            p.out[3 * b] = __float_as_int(v);
            p.out[3 * b + 1] = i == 0x7fffffff ? 0x7fffffff : i + p.row_base;
            p.out[3 * b + 2] = isnan(__ldcg(&p.logits[(size_t)b * p.V])) ? 1 : 0;
        }
    }
    __syncthreads();
    if (tid == 0) *p.counter = 0;
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
cudaError_t launch_embed(const uint16_t* tok_embd, const int32_t* tok_seq, const int32_t* pos_ptr, int E, int V,
                         float* x, cudaStream_t st, unsigned* reset_word) {
    embed_kernel<<<(E + 255) / 256, 256, 0, st>>>(tok_embd, tok_seq, pos_ptr, E, V, x, reset_word);
    return cudaGetLastError();
}

int attention_max_ctx() { return 48 * 1024; }

cudaError_t prepare_decode_kernels() {
    // called outside any stream capture, before the first launch
    cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attention_max_ctx() * (int)sizeof(float));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(lm_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                65536 * (int)sizeof(float) / 2);
}

cudaError_t launch_attention(const AttnParams& p, int n_head, cudaStream_t st) {
    const size_t smem = (size_t)p.n_ctx * sizeof(float);
    return launch_pdl(attention_kernel, dim3(n_head), dim3(kAttnThreads), smem, st, true, p);
}

cudaError_t launch_embed_rows(const uint16_t* tok_embd, const int32_t* tok_seq, int n, int E, int V, float* x,
                              cudaStream_t st) {
    return launch_pdl(embed_rows_kernel, dim3(n), dim3(256), 0, st, true, tok_embd, tok_seq, E, V, x);
}

cudaError_t launch_chunk_kv_store(const AttnParams& p, const int32_t* pos, int n, int n_head_kv, int E, int G,
                                  cudaStream_t st, size_t seq_stride) {
    return launch_pdl(chunk_kv_store_kernel, dim3(n, n_head_kv), dim3(kHeadDim), 0, st, true, p, pos, E, G,
                      seq_stride);
}

cudaError_t launch_attention_chunk(const AttnParams& p, const int32_t* pos, int n, int n_head, int E, int G,
                                   cudaStream_t st, size_t seq_stride) {
    const size_t smem = (size_t)p.n_ctx * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(attention_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attention_max_ctx() * (int)sizeof(float));
    if (e != cudaSuccess) return e;
    return launch_pdl(attention_chunk_kernel, dim3(n_head, n), dim3(kAttnThreads), smem, st, true, p, pos, E, G,
                      seq_stride);
}

cudaError_t launch_add(const float* a, const float* b, float* out, size_t n, cudaStream_t st) {
    const int grid = (int)std::min<size_t>((n + 255) / 256, 1184);
    return launch_pdl(add_kernel, dim3(grid), dim3(256), 0, st, true, a, b, out, n);
}

int lm_head_grid(int num_sms) { return 2 * num_sms; }

cudaError_t launch_lm_head_batch(const LmBatchParams& p, int num_sms, cudaStream_t st) {
    if (p.B < 1 || p.E < 32 || p.E % 32 != 0) return cudaErrorInvalidValue;
    const int groups = (p.B + kLmbTokens - 1) / kLmbTokens;
    const dim3 grid(groups, lm_head_batch_ctas(p.B, num_sms));
    // six steps in flight per thread where they fit beside the activations
    // (n_embd up to 8192), else two
    constexpr size_t kMax = 227u * 1024u - 1024u;
    size_t smem = lm_head_batch_smem(p.E, 6);
    if (smem <= kMax) {
        cudaError_t e = cudaFuncSetAttribute(lm_head_batch_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        return launch_pdl(lm_head_batch_kernel<6>, grid, dim3(kLmThreads), smem, st, false, p);
    }
    smem = lm_head_batch_smem(p.E, 2);
    if (smem > kMax) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(lm_head_batch_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(lm_head_batch_kernel<2>, grid, dim3(kLmThreads), smem, st, false, p);
}

int lm_head_batch_ctas(int B, int num_sms) {
    const int groups = (B + kLmbTokens - 1) / kLmbTokens;
    return std::max(1, num_sms / groups);
}

// An ordinary launch, not a programmatic dependent one: measured in the decode
// step, the head's CTAs launched early behind the layer program streamed the
// table at half the bandwidth for the whole kernel (238 us against 112 us per
// token at 2B-4T), for a gain of a few microseconds of launch latency.
cudaError_t launch_lm_head(const LmParams& p, int grid, cudaStream_t st) {
    const size_t smem = (size_t)p.E * sizeof(float);
    return launch_pdl(lm_head_kernel, dim3(grid), dim3(kLmThreads), smem, st, false, p);
}

}  // namespace sllm
