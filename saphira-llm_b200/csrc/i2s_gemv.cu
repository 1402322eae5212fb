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
// The weight loads of a warp's first rows are issued before the prologue, so
// the DRAM latency of the first bytes overlaps the activation quantisation.

#include "common.cuh"
#include "gemv.cuh"

namespace sllm {

constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;

// ---------------------------------------------------------------------------
// block reductions
// ---------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < NT / 32; ++i) r = fmaxf(r, red[i]);
    return r;
}

template <int NT>
__device__ __forceinline__ int block_sum_i(int v, int* red) {
    v = __reduce_add_sync(0xffffffffu, v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    int r = 0;
    for (int i = 0; i < NT / 32; ++i) r += red[i];
    return r;
}

template <int NT>
__device__ __forceinline__ double block_sum_d(double v, double* red) {
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    double r = 0.0;
    for (int i = 0; i < NT / 32; ++i) r = __dadd_rn(r, red[i]);
    return r;
}

struct ProSmem {
    double dred[32];
    float fred[32];
    int ired[32];
    float post[3];
    float rms_scale;
    sllm_cuda_act act;
};

// ---------------------------------------------------------------------------
// Prologue: leave int8 activations in qs[K] and {scale, sum} in ps.act.
//   PRO_Q8    copy a ready row (the raw GEMV API)
//   PRO_QUANT quantise x (src/i2s_gemm.c:45-83)
//   PRO_NORM  RMSNorm x with norm_w (src/ops.c:254-322), then quantise
// ys is K floats of scratch for PRO_QUANT/PRO_NORM.
// ---------------------------------------------------------------------------
template <int PRO, int NT>
__device__ void gemv_prologue(const GemvParams& p, int8_t* qs, float* ys, ProSmem& ps) {
    const int K = p.K, tid = threadIdx.x;
    if (PRO == PRO_Q8) {
        const int4* src = reinterpret_cast<const int4*>(p.q_in);
        int4* dst = reinterpret_cast<int4*>(qs);
        for (int i = tid; i < K / 16; i += NT) dst[i] = src[i];
        if (tid == 0) ps.act = *p.act_in;
        __syncthreads();
        return;
    }
    const float4* x4 = reinterpret_cast<const float4*>(p.x);
    float4* y4 = reinterpret_cast<float4*>(ys);
    if (PRO == PRO_NORM) {
        double ss = 0.0;
        for (int i = tid; i < K / 4; i += NT) {
            const float4 v = x4[i];
            y4[i] = v;
            ss = __dadd_rn(ss, (double)__fmul_rn(v.x, v.x));
            ss = __dadd_rn(ss, (double)__fmul_rn(v.y, v.y));
            ss = __dadd_rn(ss, (double)__fmul_rn(v.z, v.z));
            ss = __dadd_rn(ss, (double)__fmul_rn(v.w, v.w));
        }
        const double S = block_sum_d<NT>(ss, ps.dred);
        if (tid == 0) {
            float mean;
            const bool ok = certify_mean(S, K, &mean) && !p.force_fallback;
            if (!ok) {
                mean = __double2float_rn(__ddiv_rn(rms_ss_reference_order(ys, K), (double)K));
                if (p.fallback_count != nullptr && blockIdx.x == 0) atomicAdd(p.fallback_count, 1);
            }
            ps.rms_scale = rms_scale(mean, p.eps);
        }
        __syncthreads();
        const float sc = ps.rms_scale;
        const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
        float amax = 0.0f;
        for (int i = tid; i < K / 4; i += NT) {
            float4 v = y4[i];
            const float4 w = w4[i];
            v.x = __fmul_rn(__fmul_rn(sc, v.x), w.x);
            v.y = __fmul_rn(__fmul_rn(sc, v.y), w.y);
            v.z = __fmul_rn(__fmul_rn(sc, v.z), w.z);
            v.w = __fmul_rn(__fmul_rn(sc, v.w), w.w);
            y4[i] = v;
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        amax = block_max<NT>(amax, ps.fred);
        const float s = quant_scale(amax);
        int sum = 0;
        for (int i = tid; i < K / 4; i += NT) {
            const float4 v = y4[i];
            const int a = quant_one(v.x, s), b = quant_one(v.y, s), c = quant_one(v.z, s), d = quant_one(v.w, s);
            sum += a + b + c + d;
            reinterpret_cast<uint32_t*>(qs)[i] =
                (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
        }
        sum = block_sum_i<NT>(sum, ps.ired);
        if (tid == 0) { ps.act.scale = s; ps.act.sum = sum; }
        __syncthreads();
        return;
    }
    // PRO_QUANT
    float amax = 0.0f;
    for (int i = tid; i < K / 4; i += NT) {
        const float4 v = x4[i];
        y4[i] = v;
        // NaN never raises amax (src/i2s_gemm.c:64-69 compares a > amax).
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    amax = block_max<NT>(amax, ps.fred);
    const float s = quant_scale(amax);
    int sum = 0;
    for (int i = tid; i < K / 4; i += NT) {
        const float4 v = y4[i];
        const int a = quant_one(v.x, s), b = quant_one(v.y, s), c = quant_one(v.z, s), d = quant_one(v.w, s);
        sum += a + b + c + d;
        reinterpret_cast<uint32_t*>(qs)[i] =
            (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
    }
    sum = block_sum_i<NT>(sum, ps.ired);
    if (tid == 0) { ps.act.scale = s; ps.act.sum = sum; }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// the GEMV
// ---------------------------------------------------------------------------
template <int WPL, int U, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads)
i2s_gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ ProSmem ps;
    const int K = p.K;
    const int W = K >> 4;                      // 32-bit words per row
    int8_t* qs = reinterpret_cast<int8_t*>(smem);
    float* ys = reinterpret_cast<float*>(smem + K);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    const bool pair = (EPI == EPI_SILU);
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

    gemv_prologue<PRO, kGemvThreads>(p, qs, ys, ps);

    if (EPI != EPI_DOTS && threadIdx.x < p.nseg) {
        // (the raw-dot API never reads the scale tail: its caller need not pass one)
        const GemvSeg& sg = p.seg[threadIdx.x];
        // the per-tensor scale follows the packed codes (src/quant.c:102-106)
        const float ws = *reinterpret_cast<const float*>(sg.w + (size_t)sg.rows * (size_t)(K >> 2));
        ps.post[threadIdx.x] = __fdiv_rn(ws, ps.act.scale);
    }
    if (blockIdx.x == 0 && p.q_out != nullptr) {
        for (int i = threadIdx.x; i < K / 16; i += kGemvThreads)
            reinterpret_cast<int4*>(p.q_out)[i] = reinterpret_cast<const int4*>(qs)[i];
        if (threadIdx.x == 0 && p.act_out != nullptr) *p.act_out = ps.act;
    }
    __syncthreads();

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
    const int asum = ps.act.sum;

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

        if (EPI == EPI_SILU) {
            // row r of gate (seg 0) and of up (seg 1): h = silu(g) * u
            // (src/forward.c:765-778, src/ops.c:452-456)
            if (lane < U) {
                int s, r;
                locate(cur, lane, s, r);
                int d0 = dot[0], d1 = dot[U];
                #pragma unroll
                for (int j = 1; j < U; ++j) if (lane == j) { d0 = dot[j]; d1 = dot[U + j]; }
                if (s >= 0) {
                    const float g = __fmul_rn(__int2float_rn(d0 - asum), ps.post[0]);
                    const float u = __fmul_rn(__int2float_rn(d1 - asum), ps.post[1]);
                    if (p.seg[0].y) p.seg[0].y[r] = g;
                    if (p.seg[1].y) p.seg[1].y[r] = u;
                    if (p.seg[0].dots) p.seg[0].dots[r] = d0;
                    if (p.seg[1].dots) p.seg[1].dots[r] = d1;
                    p.h_out[r] = __fmul_rn(silu_block(g), u);
                }
            }
        } else {
            if (lane < U) {
                int s, r;
                locate(cur, lane, s, r);
                int d = dot[0];
                #pragma unroll
                for (int j = 1; j < U; ++j) if (lane == j) d = dot[j];
                if (s >= 0) {
                    const GemvSeg& sg = p.seg[s];
                    if (sg.dots) sg.dots[r] = d;
                    if (EPI != EPI_DOTS && sg.y) {
                        float v = __fmul_rn(__int2float_rn(d - asum), ps.post[s]);
                        if (EPI == EPI_RESID) v = __fadd_rn(v, p.resid[r]);
                        sg.y[r] = v;
                    }
                }
            }
        }
    }
}

// standalone quantisation (sllm_cuda_i2s_quant_act): one CTA
__global__ void __launch_bounds__(kGemvThreads)
quant_act_kernel(const float* x, int n, int8_t* q, sllm_cuda_act* act) {
    __shared__ float fred[32];
    __shared__ int ired[32];
    const int tid = threadIdx.x;
    float amax = 0.0f;
    for (int i = tid; i < n; i += kGemvThreads) amax = fmaxf(amax, fabsf(x[i]));
    amax = block_max<kGemvThreads>(amax, fred);
    const float s = quant_scale(amax);
    int sum = 0;
    for (int i = tid; i < n; i += kGemvThreads) {
        const int v = quant_one(x[i], s);
        q[i] = (int8_t)v;
        sum += v;
    }
    sum = block_sum_i<kGemvThreads>(sum, ired);
    if (tid == 0) { act->scale = s; act->sum = sum; }
}

// ---------------------------------------------------------------------------
// host-side dispatch over the compile-time shapes
// ---------------------------------------------------------------------------
template <int WPL, int U, int PRO, int EPI>
static cudaError_t launch_one(const GemvParams& p, int grid, cudaStream_t st) {
    // K <= 8192: at most 40 KB of dynamic shared memory, inside the default
    // 48 KB, so no attribute call is needed (launches may be graph-captured)
    const size_t smem = (size_t)p.K + (PRO == PRO_Q8 ? 0 : (size_t)p.K * 4);
    i2s_gemv_kernel<WPL, U, PRO, EPI><<<grid, kGemvThreads, smem, st>>>(p);
    return cudaGetLastError();
}

template <int U, int PRO, int EPI>
static cudaError_t launch_wpl(const GemvParams& p, int wpl, int grid, cudaStream_t st) {
    switch (wpl) {
#define SLLM_WPL_CASE(n) case n: return launch_one<n, U, PRO, EPI>(p, grid, st);
        SLLM_WPL_CASE(1) SLLM_WPL_CASE(2) SLLM_WPL_CASE(3) SLLM_WPL_CASE(4)
        SLLM_WPL_CASE(5) SLLM_WPL_CASE(6) SLLM_WPL_CASE(7) SLLM_WPL_CASE(8)
        SLLM_WPL_CASE(9) SLLM_WPL_CASE(10) SLLM_WPL_CASE(11) SLLM_WPL_CASE(12)
        SLLM_WPL_CASE(13) SLLM_WPL_CASE(14) SLLM_WPL_CASE(15) SLLM_WPL_CASE(16)
#undef SLLM_WPL_CASE
        default: return cudaErrorInvalidValue;
    }
}

int gemv_max_k() { return 16 * 32 * 16; }   // WPL 16: 8192

cudaError_t launch_gemv(const GemvParams& p, int pro, int epi, int num_sms, cudaStream_t st) {
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
    if (pro == PRO_Q8 && epi == EPI_DOTS) return launch_wpl<U, PRO_Q8, EPI_DOTS>(p, wpl, grid, st);
    if (pro == PRO_QUANT && epi == EPI_F32) return launch_wpl<U, PRO_QUANT, EPI_F32>(p, wpl, grid, st);
    if (pro == PRO_NORM && epi == EPI_F32) return launch_wpl<U, PRO_NORM, EPI_F32>(p, wpl, grid, st);
    if (pro == PRO_NORM && epi == EPI_RESID) return launch_wpl<U, PRO_NORM, EPI_RESID>(p, wpl, grid, st);
    if (pro == PRO_NORM && epi == EPI_SILU) return launch_wpl<U, PRO_NORM, EPI_SILU>(p, wpl, grid, st);
    return cudaErrorInvalidValue;
}

cudaError_t launch_quant_act(const float* x, int n, int8_t* q, sllm_cuda_act* act, cudaStream_t st) {
    quant_act_kernel<<<1, kGemvThreads, 0, st>>>(x, n, q, act);
    return cudaGetLastError();
}

}  // namespace sllm
