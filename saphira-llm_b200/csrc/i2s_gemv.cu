// i2s_gemv.cu -- batch-1 I2_S ternary GEMV for sm_100a, with the decode
// layer's prologues (int8 quantisation, certified RMSNorm) and epilogues
// (per-tensor scale, residual add, SiLU gating) fused around it.
//
// Replaces saphira-llm's sllm_i2s_quant_act / sllm_i2s_gemv / the inlined
// epilogue (src/i2s_gemm.c:45-290, src/forward.c:631-801).
//
// Mapping. The packed weight rows are consumed in the GGUF's own I2_S layout
// (rows of K/4 bytes). A warp owns U rows at a time; lane l owns 32-bit word
// l + 32 i (i < WPL) of every row, so each warp load instruction reads 128
// contiguous bytes of one row and a lane's word positions are the same for
// every row it visits. That lets each lane keep the int8 activations those
// words pair with (4 per word) in registers for the whole kernel, so the only
// memory traffic per weight byte is the weight byte. The int32 dot of a row
// is one warp REDUX; integer sums are exact in any order, so the result is
// bit-identical to the reference's scalar oracle (src/i2s_gemm.c:89-112).
//
// Latency. A GEMV of one layer moves 0.4-9 MB, a few microseconds at HBM
// speed, so the fixed costs decide the achieved bandwidth:
//   - the first weight words of every warp are requested before anything
//     else, so DRAM latency overlaps the whole prologue;
//   - the prologue keeps x and the norm weight in registers and needs three
//     CTA barriers, each followed by a shuffle reduction of the 16 warp
//     partials (no serial loops, no double division);
//   - programmatic dependent launch: every CTA releases the next kernel in
//     the stream at its start, so the next GEMV's CTAs become resident and
//     start their own weight loads while this one finishes. A dependent
//     kernel (the decode chain) waits for its predecessor with
//     griddepcontrol.wait before reading its input vector; an independent one
//     (separate inputs) waits only before it exits, which keeps completion in
//     stream order.

#include "common.cuh"
#include "gemv.cuh"

namespace sllm {

constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Cross-warp reductions: warp w has left its partial in red[w]; after a
// barrier every warp reduces the 16 partials with shuffles, so every thread
// holds the result without a serial loop.
__device__ __forceinline__ float cta_max(float v, float* red) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = red[threadIdx.x & (kGemvWarps - 1)];
    for (int o = kGemvWarps / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int cta_sum_i(int v, int* red) {
    v = __reduce_add_sync(0xffffffffu, v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = red[threadIdx.x & (kGemvWarps - 1)];
    for (int o = kGemvWarps / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double cta_sum_d(double v, double* red) {
    v = warp_sum_d(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = red[threadIdx.x & (kGemvWarps - 1)];
    for (int o = kGemvWarps / 2; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

struct ProSmem {
    double dred[kGemvWarps];
    float fred[kGemvWarps];
    int ired[kGemvWarps];
    float fallback_mean;
};

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
}

// ---------------------------------------------------------------------------
// Prologue: int8 activations into qs[K]; returns {scale, sum}, in every thread.
//   PRO_Q8    copy a ready row (the raw GEMV API)
//   PRO_QUANT quantise x (src/i2s_gemm.c:45-83)
//   PRO_NORM  RMSNorm x with norm_w (src/ops.c:254-322), then quantise
// KPT float4 of x per thread (K <= 8192 = 512 threads x 4 float4).
// xs is K floats of scratch, touched only by the reference-order fallback.
// ---------------------------------------------------------------------------
template <int PRO, int KPT, bool DEP>
__device__ __forceinline__ sllm_cuda_act gemv_prologue(const GemvParams& p, int8_t* qs, float* xs, ProSmem& ps) {
    const int K = p.K, tid = threadIdx.x, K4 = K >> 2;
    sllm_cuda_act act;
    if (PRO == PRO_Q8) {
        if (DEP) pdl_wait();
        const int4* src = reinterpret_cast<const int4*>(p.q_in);
        int4* dst = reinterpret_cast<int4*>(qs);
        for (int i = tid; i < K / 16; i += kGemvThreads) dst[i] = src[i];
        act = *p.act_in;
        __syncthreads();
        return act;
    }
    float4 w[KPT], x[KPT];
    if (PRO == PRO_NORM) {
        const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
        #pragma unroll
        for (int j = 0; j < KPT; ++j) {
            const int i = tid + j * kGemvThreads;
            w[j] = i < K4 ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    if (DEP) pdl_wait();
    const float4* x4 = reinterpret_cast<const float4*>(p.x);
    #pragma unroll
    for (int j = 0; j < KPT; ++j) {
        const int i = tid + j * kGemvThreads;
        x[j] = i < K4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (PRO == PRO_NORM) {
        double ss = 0.0;
        #pragma unroll
        for (int j = 0; j < KPT; ++j) {
            ss = __dadd_rn(ss, (double)__fmul_rn(x[j].x, x[j].x));
            ss = __dadd_rn(ss, (double)__fmul_rn(x[j].y, x[j].y));
            ss = __dadd_rn(ss, (double)__fmul_rn(x[j].z, x[j].z));
            ss = __dadd_rn(ss, (double)__fmul_rn(x[j].w, x[j].w));
        }
        const double S = cta_sum_d(ss, ps.dred);
        float mean;
        const bool ok = certify_mean_mul(S, K, p.inv_k, &mean) && !p.force_fallback;   // uniform in the CTA
        if (!ok) {
            #pragma unroll
            for (int j = 0; j < KPT; ++j) {
                const int i = tid + j * kGemvThreads;
                if (i < K4) reinterpret_cast<float4*>(xs)[i] = x[j];
            }
            __syncthreads();
            if (tid == 0) {
                ps.fallback_mean = __double2float_rn(__ddiv_rn(rms_ss_reference_order(xs, K), (double)K));
                if (p.fallback_count != nullptr && blockIdx.x == 0) atomicAdd(p.fallback_count, 1);
            }
            __syncthreads();
            mean = ps.fallback_mean;
        }
        const float sc = rms_scale(mean, p.eps);
        #pragma unroll
        for (int j = 0; j < KPT; ++j) {
            x[j].x = __fmul_rn(__fmul_rn(sc, x[j].x), w[j].x);
            x[j].y = __fmul_rn(__fmul_rn(sc, x[j].y), w[j].y);
            x[j].z = __fmul_rn(__fmul_rn(sc, x[j].z), w[j].z);
            x[j].w = __fmul_rn(__fmul_rn(sc, x[j].w), w[j].w);
        }
    }
    // amax: NaN never raises it (src/i2s_gemm.c:64-69 compares a > amax)
    float amax = 0.0f;
    #pragma unroll
    for (int j = 0; j < KPT; ++j)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x[j].x), fabsf(x[j].y)), fmaxf(fabsf(x[j].z), fabsf(x[j].w))));
    amax = cta_max(amax, ps.fred);
    const float s = quant_scale(amax);
    int sum = 0;
    #pragma unroll
    for (int j = 0; j < KPT; ++j) {
        const int i = tid + j * kGemvThreads;
        if (i < K4) {
            const int a = quant_one(x[j].x, s), b = quant_one(x[j].y, s);
            const int c = quant_one(x[j].z, s), d = quant_one(x[j].w, s);
            sum += a + b + c + d;
            reinterpret_cast<uint32_t*>(qs)[i] = pack4(a, b, c, d);
        }
    }
    sum = cta_sum_i(sum, ps.ired);     // its barrier also publishes qs
    act.scale = s;
    act.sum = sum;
    return act;
}

// ---------------------------------------------------------------------------
// the GEMV
// ---------------------------------------------------------------------------
template <int WPL, int U, int PRO, int EPI, bool DEP>
__global__ void __launch_bounds__(kGemvThreads)
i2s_gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ ProSmem ps;
    constexpr int KPT = (WPL + 3) / 4;
    const int K = p.K;
    const int W = K >> 4;                      // 32-bit words per row
    int8_t* qs = reinterpret_cast<int8_t*>(smem);
    float* xs = reinterpret_cast<float*>(smem + K);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    pdl_trigger();

    constexpr bool pair = (EPI == EPI_SILU);
    const int rows0 = p.seg[0].rows;
    const int rows1 = p.nseg > 1 ? p.seg[1].rows : 0;
    const int total = pair ? rows0 : rows0 + rows1 + (p.nseg > 2 ? p.seg[2].rows : 0);
    constexpr int R = pair ? 2 * U : U;        // rows a task touches
    const int ntasks = (total + U - 1) / U;
    const int stride = gridDim.x * kGemvWarps;
    int task = blockIdx.x * kGemvWarps + warp;

    // row j of a task -> (segment, local row); -1 when past the end
    auto locate = [&](int t, int j, int& s, int& r) {
        if (pair) {
            s = j < U ? 0 : 1;
            r = t * U + (j < U ? j : j - U);
            if (r >= rows0) { s = -1; }
            return;
        }
        int g = t * U + j;
        if (g >= total) { s = -1; r = 0; return; }
        if (g < rows0) { s = 0; r = g; return; }
        g -= rows0;
        if (g < rows1) { s = 1; r = g; return; }
        s = 2; r = g - rows1;
    };

    uint32_t wr[R][WPL];
    auto load_task = [&](int t) {
        #pragma unroll
        for (int j = 0; j < R; ++j) {
            int s, r;
            locate(t, j, s, r);
            const uint8_t* base = s >= 0 ? p.seg[s].w + (size_t)r * (size_t)(K >> 2) : nullptr;
            #pragma unroll
            for (int i = 0; i < WPL; ++i) {
                const int wi = lane + 32 * i;
                wr[j][i] = (s >= 0 && wi < W) ? ld_stream_u32(base + 4 * wi) : 0u;
            }
        }
    };

    if (task < ntasks) load_task(task);

    // the per-tensor scales follow the packed codes (src/quant.c:102-106);
    // the raw-dot API never reads them (its caller need not pass a tail)
    float ws[3] = {0.f, 0.f, 0.f};
    if (EPI != EPI_DOTS) {
        #pragma unroll
        for (int s = 0; s < 3; ++s)
            if (s < p.nseg)
                ws[s] = *reinterpret_cast<const float*>(p.seg[s].w + (size_t)p.seg[s].rows * (size_t)(K >> 2));
    }

    const sllm_cuda_act act = gemv_prologue<PRO, KPT, DEP>(p, qs, xs, ps);
    float post[3];
    #pragma unroll
    for (int s = 0; s < 3; ++s) post[s] = __fdiv_rn(ws[s], act.scale);
    if (blockIdx.x == 0 && p.q_out != nullptr) {
        for (int i = threadIdx.x; i < K / 16; i += kGemvThreads)
            reinterpret_cast<int4*>(p.q_out)[i] = reinterpret_cast<const int4*>(qs)[i];
        if (threadIdx.x == 0 && p.act_out != nullptr) *p.act_out = act;
    }

    // the int8 activations this lane's words pair with
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qs);
    int aq[WPL][4];
    #pragma unroll
    for (int i = 0; i < WPL; ++i) {
        const int wi = lane + 32 * i;
        #pragma unroll
        for (int f = 0; f < 4; ++f)
            aq[i][f] = wi < W ? (int)q32[(wi >> 3) * 32 + 8 * f + (wi & 7)] : 0;
    }
    const int asum = act.sum;

    while (task < ntasks) {
        int dot[R];
        #pragma unroll
        for (int j = 0; j < R; ++j) {
            int acc = 0;
            #pragma unroll
            for (int i = 0; i < WPL; ++i) acc = i2s_dot_word(wr[j][i], aq[i][0], aq[i][1], aq[i][2], aq[i][3], acc);
            dot[j] = acc;
        }
        const int cur = task;
        task += stride;
        if (task < ntasks) load_task(task);       // next rows in flight during the epilogue
        #pragma unroll
        for (int j = 0; j < R; ++j) dot[j] = __reduce_add_sync(0xffffffffu, dot[j]);

        if (lane < U) {
            int s, r;
            locate(cur, lane, s, r);
            int d0 = dot[0], d1 = pair ? dot[U] : 0;
            #pragma unroll
            for (int j = 1; j < U; ++j)
                if (lane == j) { d0 = dot[j]; if (pair) d1 = dot[U + j]; }
            if (s >= 0) {
                if (EPI == EPI_SILU) {
                    // row r of gate (seg 0) and of up (seg 1): h = silu(g) * u
                    // (src/forward.c:765-778, src/ops.c:452-456)
                    const float g = __fmul_rn(__int2float_rn(d0 - asum), post[0]);
                    const float u = __fmul_rn(__int2float_rn(d1 - asum), post[1]);
                    if (p.seg[0].y) p.seg[0].y[r] = g;
                    if (p.seg[1].y) p.seg[1].y[r] = u;
                    if (p.seg[0].dots) p.seg[0].dots[r] = d0;
                    if (p.seg[1].dots) p.seg[1].dots[r] = d1;
                    p.h_out[r] = __fmul_rn(silu_block(g), u);
                } else {
                    const float ps_ = s == 0 ? post[0] : (s == 1 ? post[1] : post[2]);
                    const GemvSeg& sg = p.seg[s];
                    if (sg.dots) sg.dots[r] = d0;
                    if (EPI != EPI_DOTS && sg.y) {
                        float v = __fmul_rn(__int2float_rn(d0 - asum), ps_);
                        if (EPI == EPI_RESID) v = __fadd_rn(v, p.resid[r]);
                        sg.y[r] = v;
                    }
                }
            }
        }
    }
    if (!DEP) pdl_wait();   // complete in stream order
}

// RMSNorm + quantisation of every row of a row-major [rows][K] batch, one CTA
// per row: the per-column prologue of a multi-token chunk (src/forward.c:
// 631-666, 728-741, 752-764, 781-792, column by column), with the GEMV
// prologue's arithmetic; q in natural order for the GEMM.
template <int KPT>
__global__ void __launch_bounds__(kGemvThreads)
norm_quant_rows_kernel(const GemvParams p, int8_t* q, sllm_cuda_act* acts) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ ProSmem ps;
    const int K = p.K;
    // launched with programmatic stream serialisation: the next launch (a
    // GEMM, which waits for this one after its set-up) may be scheduled now,
    // and x may come from the previous launch
    pdl_trigger();
    pdl_wait();
    int8_t* qs = reinterpret_cast<int8_t*>(smem);
    float* xs = reinterpret_cast<float*>(smem + K);
    GemvParams pr = p;
    pr.x = p.x + (size_t)blockIdx.x * K;
    const sllm_cuda_act act = gemv_prologue<PRO_NORM, KPT, true>(pr, qs, xs, ps);
    int4* dst = reinterpret_cast<int4*>(q + (size_t)blockIdx.x * K);
    for (int i = threadIdx.x; i < K / 16; i += kGemvThreads) dst[i] = reinterpret_cast<const int4*>(qs)[i];
    if (threadIdx.x == 0) acts[blockIdx.x] = act;
}

// standalone quantisation (sllm_cuda_i2s_quant_act): one CTA
__global__ void __launch_bounds__(kGemvThreads)
quant_act_kernel(const float* x, int n, int8_t* q, sllm_cuda_act* act) {
    __shared__ float fred[kGemvWarps];
    __shared__ int ired[kGemvWarps];
    const int tid = threadIdx.x;
    // block b quantises row b of a row-major [rows][n] batch (one row per token)
    x += (size_t)blockIdx.x * n;
    q += (size_t)blockIdx.x * n;
    act += blockIdx.x;
    float amax = 0.0f;
    for (int i = tid; i < n; i += kGemvThreads) amax = fmaxf(amax, fabsf(x[i]));
    amax = cta_max(amax, fred);
    const float s = quant_scale(amax);
    int sum = 0;
    for (int i = tid; i < n; i += kGemvThreads) {
        const int v = quant_one(x[i], s);
        q[i] = (int8_t)v;
        sum += v;
    }
    sum = cta_sum_i(sum, ired);
    if (tid == 0) { act->scale = s; act->sum = sum; }
}

// The same quantisation for whole rows of n % 4 == 0 elements (n <= 8192) on
// 16-byte aligned rows: 256 threads, each row read once as float4 into
// registers, the int8 codes stored four to a word. Identical results: the
// same amax (order-free), scale, rounding and sum (exact).
constexpr int kQrThreads = 256;

template <int VPT>
__global__ void __launch_bounds__(kQrThreads)
quant_rows_vec_kernel(const float* x, int n, int8_t* q, sllm_cuda_act* act) {
    __shared__ float fred[kQrThreads / 32];
    __shared__ int ired[kQrThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n4 = n >> 2;
    // launched with programmatic stream serialisation: the next launch (a
    // GEMM, which waits for this one after its set-up) may be scheduled now,
    // and x may come from the previous launch
    pdl_trigger();
    pdl_wait();
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)blockIdx.x * n);
    uint32_t* qr = reinterpret_cast<uint32_t*>(q + (size_t)blockIdx.x * n);
    float4 v[VPT];
    #pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int i = tid + j * kQrThreads;
        v[j] = i < n4 ? __ldg(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float amax = 0.0f;
    #pragma unroll
    for (int j = 0; j < VPT; ++j)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
    amax = warp_max(amax);
    if (lane == 0) fred[warp] = amax;
    __syncthreads();
    amax = fred[lane & (kQrThreads / 32 - 1)];
    #pragma unroll
    for (int o = kQrThreads / 64; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = quant_scale(amax);
    int sum = 0;
    #pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int i = tid + j * kQrThreads;
        if (i < n4) {
            const int a = quant_one(v[j].x, sc), b = quant_one(v[j].y, sc);
            const int c = quant_one(v[j].z, sc), d = quant_one(v[j].w, sc);
            sum += a + b + c + d;
            qr[i] = (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) |
                    ((uint32_t)d << 24);
        }
    }
    sum = __reduce_add_sync(0xffffffffu, sum);
    if (lane == 0) ired[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        int t = 0;
        #pragma unroll
        for (int w = 0; w < kQrThreads / 32; ++w) t += ired[w];
        act[blockIdx.x].scale = sc;
        act[blockIdx.x].sum = t;
    }
}

// ---------------------------------------------------------------------------
// host-side dispatch over the compile-time shapes
// ---------------------------------------------------------------------------
template <int WPL, int U, int PRO, int EPI, bool DEP>
static cudaError_t launch_one(const GemvParams& p, int grid, cudaStream_t st, bool pdl) {
    // K <= 8192: at most 40 KB of dynamic shared memory, inside the default
    // 48 KB, so no attribute call is needed (launches may be graph-captured)
    const size_t smem = (size_t)p.K * 5;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, i2s_gemv_kernel<WPL, U, PRO, EPI, DEP>, p);
}

template <int U, int PRO, int EPI, bool DEP>
static cudaError_t launch_wpl(const GemvParams& p, int wpl, int grid, cudaStream_t st, bool pdl) {
    switch (wpl) {
#define SLLM_WPL_CASE(n) case n: return launch_one<n, U, PRO, EPI, DEP>(p, grid, st, pdl);
        SLLM_WPL_CASE(1) SLLM_WPL_CASE(2) SLLM_WPL_CASE(3) SLLM_WPL_CASE(4)
        SLLM_WPL_CASE(5) SLLM_WPL_CASE(6) SLLM_WPL_CASE(7) SLLM_WPL_CASE(8)
        SLLM_WPL_CASE(9) SLLM_WPL_CASE(10) SLLM_WPL_CASE(11) SLLM_WPL_CASE(12)
        SLLM_WPL_CASE(13) SLLM_WPL_CASE(14) SLLM_WPL_CASE(15) SLLM_WPL_CASE(16)
#undef SLLM_WPL_CASE
        default: return cudaErrorInvalidValue;
    }
}

int gemv_max_k() { return 16 * 32 * 16; }   // WPL 16: 8192

cudaError_t launch_gemv(const GemvParams& p_in, int pro, int epi, int num_sms, cudaStream_t st, int mode) {
    GemvParams p = p_in;
    p.inv_k = 1.0 / (double)p.K;
    const int W = p.K / 16;
    const int wpl = (W + 31) / 32;
    if (p.K % kQK != 0 || wpl < 1 || wpl > 16) return cudaErrorInvalidValue;
    constexpr int U = 2;
    int total = p.seg[0].rows;
    if (epi != EPI_SILU) for (int s = 1; s < p.nseg; ++s) total += p.seg[s].rows;
    const int ntasks = (total + U - 1) / U;
    int grid = (ntasks + kGemvWarps - 1) / kGemvWarps;
    const int cap = 2 * num_sms;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    const bool pdl = mode != GEMV_PLAIN;
    if (mode == GEMV_INDEPENDENT) {
        if (pro == PRO_NORM && epi == EPI_F32) return launch_wpl<U, PRO_NORM, EPI_F32, false>(p, wpl, grid, st, pdl);
        return cudaErrorInvalidValue;
    }
    // plain launches and dependent (decode-chain) launches share the DEP form:
    // without the launch attribute griddepcontrol.wait returns at once
    if (pro == PRO_Q8 && epi == EPI_DOTS) return launch_wpl<U, PRO_Q8, EPI_DOTS, true>(p, wpl, grid, st, pdl);
    if (pro == PRO_QUANT && epi == EPI_F32) return launch_wpl<U, PRO_QUANT, EPI_F32, true>(p, wpl, grid, st, pdl);
    if (pro == PRO_NORM && epi == EPI_F32) return launch_wpl<U, PRO_NORM, EPI_F32, true>(p, wpl, grid, st, pdl);
    if (pro == PRO_NORM && epi == EPI_RESID) return launch_wpl<U, PRO_NORM, EPI_RESID, true>(p, wpl, grid, st, pdl);
    if (pro == PRO_NORM && epi == EPI_SILU) return launch_wpl<U, PRO_NORM, EPI_SILU, true>(p, wpl, grid, st, pdl);
    return cudaErrorInvalidValue;
}

cudaError_t launch_norm_quant_rows(const float* x, const float* w, int K, float eps, int rows, int8_t* q,
                                   sllm_cuda_act* acts, int* fb, int force, cudaStream_t st) {
    if (K % kQK != 0 || K > gemv_max_k() || rows < 1) return cudaErrorInvalidValue;
    GemvParams p{};
    p.K = K;
    p.x = x;
    p.norm_w = w;
    p.eps = eps;
    p.inv_k = 1.0 / (double)K;
    p.fallback_count = fb;
    p.force_fallback = force;
    const int kpt = (K / 4 + kGemvThreads - 1) / kGemvThreads;    // 1..4
    const size_t smem = (size_t)K * 5;                              // qs, then the fallback's floats
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (kpt) {
        case 1: return cudaLaunchKernelEx(&cfg, norm_quant_rows_kernel<1>, p, q, acts);
        case 2: return cudaLaunchKernelEx(&cfg, norm_quant_rows_kernel<2>, p, q, acts);
        case 3: return cudaLaunchKernelEx(&cfg, norm_quant_rows_kernel<3>, p, q, acts);
        default: return cudaLaunchKernelEx(&cfg, norm_quant_rows_kernel<4>, p, q, acts);
    }
}

cudaError_t launch_quant_act(const float* x, int n, int8_t* q, sllm_cuda_act* act, cudaStream_t st) {
    quant_act_kernel<<<1, kGemvThreads, 0, st>>>(x, n, q, act);
    return cudaGetLastError();
}

cudaError_t launch_quant_act_rows(const float* x, int rows, int n, int8_t* q, sllm_cuda_act* acts, cudaStream_t st) {
    const bool vec = n % 4 == 0 && n <= 8192 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(q) & 3u) == 0;
    if (vec) {
        const int vpt = (n / 4 + kQrThreads - 1) / kQrThreads;     // 1..8
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(rows);
        cfg.blockDim = dim3(kQrThreads);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        switch (vpt) {
#define SLLM_QR_CASE(k) case k: return cudaLaunchKernelEx(&cfg, quant_rows_vec_kernel<k>, x, n, q, acts);
            SLLM_QR_CASE(1) SLLM_QR_CASE(2) SLLM_QR_CASE(3) SLLM_QR_CASE(4)
            SLLM_QR_CASE(5) SLLM_QR_CASE(6) SLLM_QR_CASE(7) SLLM_QR_CASE(8)
#undef SLLM_QR_CASE
            default: quant_act_kernel<<<rows, kGemvThreads, 0, st>>>(x, n, q, acts); break;
        }
        return cudaGetLastError();
    }
    quant_act_kernel<<<rows, kGemvThreads, 0, st>>>(x, n, q, acts);
    return cudaGetLastError();
}

}  // namespace sllm
