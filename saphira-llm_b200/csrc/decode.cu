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
                             const int32_t* __restrict__ pos_ptr, int E, int V, float* __restrict__ x) {
    int tok = tok_seq[*pos_ptr];
    // the host validates every token it writes and the argmax is in range;
    // this only keeps a corrupted id from reading outside the table
    if ((unsigned)tok >= (unsigned)V) tok = 0;
    const uint16_t* row = tok_embd + (size_t)tok * (size_t)E;
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < E; d += gridDim.x * blockDim.x)
        x[d] = f16_embd(row[d]);
}

// ---------------------------------------------------------------------------
// attention for one query position, one CTA per query head
// ---------------------------------------------------------------------------
constexpr int kAttnThreads = 256;
constexpr int kHeadDim = 128;

__global__ void __launch_bounds__(kAttnThreads)
attention_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float sc[];          // n_ctx scores
    __shared__ float qs[kHeadDim], kcur[kHeadDim];
    __shared__ float fred[32];
    __shared__ double dred[32];
    __shared__ float s_inv;
    const int h = blockIdx.x, t = threadIdx.x;
    const int kvh = h / p.group;
    pdl_trigger_d();
    pdl_wait_d();                 // q, k, v come from the previous kernel
    const int pos = *p.pos_ptr;
    const int npast = pos + 1;
    const int nctx = p.n_ctx;
    const float* cs = p.rope_cos + (size_t)pos * (kHeadDim / 2);
    const float* sn = p.rope_sin + (size_t)pos * (kHeadDim / 2);

    // RoPE NEOX on q and on this head's k: pairs (i, i+64), angle table from
    // the host (src/ops.c:529-549): x' = (xa*c - xb*s, xa*s + xb*c)
    if (t < kHeadDim / 2) {
        const float c = cs[t], s = sn[t];
        const float qa = p.q[h * kHeadDim + t], qb = p.q[h * kHeadDim + t + 64];
        qs[t] = __fsub_rn(__fmul_rn(qa, c), __fmul_rn(qb, s));
        qs[t + 64] = __fadd_rn(__fmul_rn(qa, s), __fmul_rn(qb, c));
    } else if (t < kHeadDim) {
        const int i = t - 64;
        const float c = cs[i], s = sn[i];
        const float ka = p.k[kvh * kHeadDim + i], kb = p.k[kvh * kHeadDim + i + 64];
        kcur[i] = __fsub_rn(__fmul_rn(ka, c), __fmul_rn(kb, s));
        kcur[i + 64] = __fadd_rn(__fmul_rn(ka, s), __fmul_rn(kb, c));
    }
    __syncthreads();

    float* kT = p.k_cache + (size_t)kvh * kHeadDim * nctx;   // [d][pos]
    float* vC = p.v_cache + (size_t)kvh * nctx * kHeadDim;   // [pos][d]
    // the first query head of the group stores this position's K and V
    // (src/forward.c:683-696); every CTA uses kcur / v directly for pos
    if (h % p.group == 0 && t < kHeadDim) {
        kT[(size_t)t * nctx + pos] = kcur[t];
        vC[(size_t)pos * kHeadDim + t] = p.v[kvh * kHeadDim + t];
    }

    // scores: sequential f32 dot over d, then * 1/sqrt(hd) (src/forward.c:710-715)
    for (int s = t; s < npast; s += kAttnThreads) {
        float acc = 0.0f;
        if (s == pos) {
            #pragma unroll 8
            for (int d = 0; d < kHeadDim; ++d) acc = __fadd_rn(acc, __fmul_rn(qs[d], kcur[d]));
        } else {
            const float* col = kT + s;
            #pragma unroll 16
            for (int d = 0; d < kHeadDim; ++d) acc = __fadd_rn(acc, __fmul_rn(qs[d], col[(size_t)d * nctx]));
        }
        sc[s] = __fmul_rn(acc, p.attn_scale);
    }
    __syncthreads();

    // softmax (src/ops.c:386-422)
    float mx = -INFINITY;
    for (int s = t; s < npast; s += kAttnThreads) mx = fmaxf(mx, sc[s]);
    mx = warp_max(mx);
    if ((t & 31) == 0) fred[t >> 5] = mx;
    __syncthreads();
    mx = fred[0];
    for (int i = 1; i < kAttnThreads / 32; ++i) mx = fmaxf(mx, fred[i]);
    // the reference's max is the first-seen maximum with '>' ; with no NaN
    // it is the same value (a NaN score propagates identically below).
    const int nblk = npast & ~7;
    double part = 0.0;
    for (int s = t; s < npast; s += kAttnThreads) {
        const float d = __fsub_rn(sc[s], mx);
        const float e = (s < nblk) ? v_expf(d) : sllm_libm_expf(d);
        sc[s] = e;
        part = __dadd_rn(part, (double)e);
    }
    part = warp_sum_d(part);
    __syncthreads();
    if ((t & 31) == 0) dred[t >> 5] = part;
    __syncthreads();
    if (t == 0) {
        double S = 0.0;
        for (int i = 0; i < kAttnThreads / 32; ++i) S = __dadd_rn(S, dred[i]);
        // certified: any order of these npast non-negative terms lies within
        // (npast + 64) * 2^-52 relative of the reference's; 1/x is monotone.
        const double e = (double)(npast + 64) * 0x1p-52;
        const float ia = __double2float_rn(__ddiv_rn(1.0, __dmul_ru(S, 1.0 + e)));
        const float ib = __double2float_rn(__ddiv_rn(1.0, __dmul_rd(S, 1.0 - e)));
        float inv = ia;
        if (f2u(ia) != f2u(ib) || p.force_fallback) {
            // reference order: per 8-block ((t0+t1)+t2)+t3 with
            // t_k = e_k + e_{k+4}; the tail one at a time
            double sum = 0.0;
            int i = 0;
            for (; i + 7 < npast; i += 8) {
                const double t0 = __dadd_rn((double)sc[i + 0], (double)sc[i + 4]);
                const double t1 = __dadd_rn((double)sc[i + 1], (double)sc[i + 5]);
                const double t2 = __dadd_rn((double)sc[i + 2], (double)sc[i + 6]);
                const double t3 = __dadd_rn((double)sc[i + 3], (double)sc[i + 7]);
                sum = __dadd_rn(sum, __dadd_rn(__dadd_rn(__dadd_rn(t0, t1), t2), t3));
            }
            for (; i < npast; ++i) sum = __dadd_rn(sum, (double)sc[i]);
            inv = __double2float_rn(__ddiv_rn(1.0, sum));
            if (p.fallback_count != nullptr) atomicAdd(p.fallback_count, 1);
        }
        s_inv = inv;
    }
    __syncthreads();
    const float inv = s_inv;
    for (int s = t; s < npast; s += kAttnThreads) sc[s] = __fmul_rn(sc[s], inv);
    __syncthreads();

    // o[d] = sum over s of w_s * v[s][d], sequential in s (src/forward.c:718-724)
    if (t < kHeadDim) {
        float o = 0.0f;
        const float vcur = p.v[kvh * kHeadDim + t];
        int s = 0;
        for (; s + 8 <= pos; s += 8) {
            float vv[8];
            #pragma unroll
            for (int j = 0; j < 8; ++j) vv[j] = vC[(size_t)(s + j) * kHeadDim + t];
            #pragma unroll
            for (int j = 0; j < 8; ++j) o = __fadd_rn(o, __fmul_rn(sc[s + j], vv[j]));
        }
        for (; s < pos; ++s) o = __fadd_rn(o, __fmul_rn(sc[s], vC[(size_t)s * kHeadDim + t]));
        o = __fadd_rn(o, __fmul_rn(sc[pos], vcur));
        p.out[h * kHeadDim + t] = o;
    }
}

// ---------------------------------------------------------------------------
// lm_head + argmax
//
// Half a warp per vocabulary row; lane c (0..15) owns the reference's
// accumulators 2c and 2c+1 (acc[j][l] with 8j + l = 2c, 2c+1), so every step
// reads one half2 per lane: 64 contiguous bytes per row, two rows per warp
// instruction. After E/32 FMA steps the reference's tree (src/ops.c:135-143)
// runs as shuffles: acc0+=acc2, acc1+=acc3; acc0+=acc1; t_l = acc0[l] +
// acc0[l+4]; (t0+t1) + (t2+t3).
// ---------------------------------------------------------------------------
constexpr int kLmThreads = 512;
constexpr int kLmWarps = kLmThreads / 32;
constexpr int kLmUnroll = 16;

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
    pdl_wait_d();                 // x comes from the last layer

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

    const int half = lane >> 4, c = lane & 15;
    const int nsteps = E >> 5;
    const int npairs = (p.V + 1) >> 1;
    float bv = NAN;
    int bi = 0x7fffffff;
    for (int pr = blockIdx.x * kLmWarps + warp; pr < npairs; pr += gridDim.x * kLmWarps) {
        const int row = 2 * pr + half;
        const bool valid = row < p.V;
        const uint32_t* wrow = reinterpret_cast<const uint32_t*>(p.embd + (size_t)(valid ? row : 0) * (size_t)E);
        float a0 = 0.0f, a1 = 0.0f;
        for (int m0 = 0; m0 < nsteps; m0 += kLmUnroll) {
            uint32_t wv[kLmUnroll];
            #pragma unroll
            for (int j = 0; j < kLmUnroll; ++j)
                wv[j] = (m0 + j < nsteps) ? ld_stream_u32(wrow + 16 * (m0 + j) + c) : 0u;
            #pragma unroll
            for (int j = 0; j < kLmUnroll; ++j) {
                if (m0 + j < nsteps) {
                    const float2 wf = __half22float2(*reinterpret_cast<const __half2*>(&wv[j]));
                    const float2 xf = *reinterpret_cast<const float2*>(xs + 32 * (m0 + j) + 2 * c);
                    a0 = __fmaf_rn(wf.x, xf.x, a0);
                    a1 = __fmaf_rn(wf.y, xf.y, a1);
                }
            }
        }
        // tree, within each 16-lane half
        a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 8));
        a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 8));
        a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 4));
        a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 4));
        a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 2));
        a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 2));
        // lane c=0 holds t0, t1; lane c=1 holds t2, t3
        const float pairsum = __fadd_rn(a0, a1);
        const float other = __shfl_down_sync(0xffffffffu, pairsum, 1);
        const float logit = __fadd_rn(pairsum, other);
        if (c == 0 && valid) {
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
    if (!s_last || tid != 0) return;
    __threadfence();
    for (int b = 0; b < (int)gridDim.x; ++b) {
        const float v = *(volatile float*)&p.part_v[b];
        const int i = *(volatile int*)&p.part_i[b];
        if (better(v, i, bv, bi)) { bv = v; bi = i; }
    }
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
// launchers
// ---------------------------------------------------------------------------
cudaError_t launch_embed(const uint16_t* tok_embd, const int32_t* tok_seq, const int32_t* pos_ptr, int E, int V,
                         float* x, cudaStream_t st) {
    embed_kernel<<<(E + 255) / 256, 256, 0, st>>>(tok_embd, tok_seq, pos_ptr, E, V, x);
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

int lm_head_grid(int num_sms) { return 2 * num_sms; }

cudaError_t launch_lm_head(const LmParams& p, int grid, cudaStream_t st) {
    const size_t smem = (size_t)p.E * sizeof(float);
    return launch_pdl(lm_head_kernel, dim3(grid), dim3(kLmThreads), smem, st, true, p);
}

}  // namespace sllm
