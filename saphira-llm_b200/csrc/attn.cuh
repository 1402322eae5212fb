// attn.cuh -- one query head of decode attention (src/forward.c:698-726),
// shared by the standalone attention kernel (decode.cu, 256 threads) and the
// persistent engine's attention stage (engine.cu, its 480 consumer threads).
//
// RoPE NEOX on q and k from the host angle table, the K/V append of this
// position (by the first query head of each kv group), scores as sequential
// f32 dots scaled by 1/sqrt(128), the softmax with a certified f64 sum (any
// thread count: the interval covers every summation order, and the rare
// ambiguous case re-sums in the reference's 8-block order), then P.V
// sequential in s. NT threads; `sync` is the barrier of those NT threads.
// Shared scratch: sc[n_ctx], qs[128], kcur[128], fred and dred with a slot
// per warp.
//
// Every sum keeps the reference's order, so the time is latency: the chains
// of dependent adds and the L2 round trips that feed them. The last 128
// threads run P.V, one per dimension, with 64 V rows in flight: four batches
// of 16 in registers, each refilled with the rows 64 further on as soon as it
// has been added. The normalisation is folded into P.V: the weight
// fl(e_s * inv) is formed as the reference stores it, then multiplied by v.
// Two barriers separate scores, exponentials and P.V; every thread forms the
// certified reciprocal itself.
#pragma once

#include <type_traits>
#include <cuda_fp16.h>

#include "common.cuh"
#include "decode.cuh"
#include "libm_expf.h"

namespace sllm {

constexpr int kHeadDim = 128;

// The cache's element type. The reference keeps K and V in fp32
// (src/forward.c:486-487), which is the default and bit-exact. The fp16 option
// stores each value rounded to the nearest half (ties to even) and reads it
// back exactly; the current position's k and v are rounded the same way, as if
// stored and read back, so every use sees the cached value.
// A cache is addressed by element index; f16 selects the element type (one
// body for both, so the kernels that inline it keep one copy).
template <class T>
struct KvRef {
    T* base;
    __device__ __forceinline__ float ld(size_t i) const;
    __device__ __forceinline__ void st(size_t i, float v) const;
    __device__ __forceinline__ float round(float v) const;
};
template <> __device__ __forceinline__ float KvRef<float>::ld(size_t i) const { return base[i]; }
template <> __device__ __forceinline__ void KvRef<float>::st(size_t i, float v) const { base[i] = v; }
template <> __device__ __forceinline__ float KvRef<float>::round(float v) const { return v; }
template <> __device__ __forceinline__ float KvRef<__half>::ld(size_t i) const { return __half2float(base[i]); }
template <> __device__ __forceinline__ void KvRef<__half>::st(size_t i, float v) const { base[i] = __float2half_rn(v); }
template <> __device__ __forceinline__ float KvRef<__half>::round(float v) const {
    return __half2float(__float2half_rn(v));
}

template <int NT, class KV, class Sync>
__device__ __forceinline__ void attention_head_t(const AttnParams& p, int h, int t, float* sc, float* qs, float* kcur,
                                                 float* fred, double* dred, Sync sync) {
    static_assert(NT % 32 == 0 && NT >= 2 * kHeadDim, "two 128-thread teams at least");
    const int kvh = h / p.group;
    const int pos = *(volatile const int32_t*)p.pos_ptr;
    const int npast = pos + 1;
    const int nctx = p.n_ctx;
    const float* cs = p.rope_cos + (size_t)pos * (kHeadDim / 2);
    const float* sn = p.rope_sin + (size_t)pos * (kHeadDim / 2);
    const KvRef<KV> kT{reinterpret_cast<KV*>(p.k_cache) + (size_t)kvh * kHeadDim * nctx};   // [d][pos]
    const KvRef<KV> vC{reinterpret_cast<KV*>(p.v_cache) + (size_t)kvh * nctx * kHeadDim};   // [pos][d]
    const int pv_d = t - (NT - kHeadDim);                   // this thread's P.V dimension, < 0: none


    // RoPE NEOX on q and on this head's k: pairs (i, i+64), angle table from
    // the host (src/ops.c:529-549): x' = (xa*c - xb*s, xa*s + xb*c)
    if (t < kHeadDim / 2) {
        const float c = cs[t], s = sn[t];
        // through L2: inside the engine another CTA wrote q, k, v in this launch
        const float qa = __ldcg(p.q + h * kHeadDim + t), qb = __ldcg(p.q + h * kHeadDim + t + 64);
        qs[t] = __fsub_rn(__fmul_rn(qa, c), __fmul_rn(qb, s));
        qs[t + 64] = __fadd_rn(__fmul_rn(qa, s), __fmul_rn(qb, c));
    } else if (t < kHeadDim) {
        const int i = t - 64;
        const float c = cs[i], s = sn[i];
        const float ka = __ldcg(p.k + kvh * kHeadDim + i), kb = __ldcg(p.k + kvh * kHeadDim + i + 64);
        kcur[i] = kT.round(__fsub_rn(__fmul_rn(ka, c), __fmul_rn(kb, s)));
        kcur[i + 64] = kT.round(__fadd_rn(__fmul_rn(ka, s), __fmul_rn(kb, c)));
    }
    sync();

    // the first query head of the group stores this position's K and V
    // (src/forward.c:683-696); every head uses kcur / v directly for pos
    if (h % p.group == 0 && t < kHeadDim && (p.kv_f16 & kAttnKvStored) == 0) {
        kT.st((size_t)t * nctx + pos, kcur[t]);
        vC.st((size_t)pos * kHeadDim + t, __ldcg(p.v + kvh * kHeadDim + t));
    }

    // scores: sequential f32 dot over d, then * 1/sqrt(hd) (src/forward.c:710-715)
    float mx = -INFINITY;
    if (t < pos) {
        float acc = 0.0f;
        #pragma unroll
        for (int d0 = 0; d0 < kHeadDim; d0 += 32) {
            float kv[32];
            #pragma unroll
            for (int j = 0; j < 32; ++j) kv[j] = kT.ld((size_t)(d0 + j) * nctx + t);
            #pragma unroll
            for (int j = 0; j < 32; ++j) acc = __fadd_rn(acc, __fmul_rn(qs[d0 + j], kv[j]));
        }
        sc[t] = __fmul_rn(acc, p.attn_scale);
        mx = fmaxf(mx, sc[t]);
    } else if (t == pos) {
        float acc = 0.0f;
        #pragma unroll 8
        for (int d = 0; d < kHeadDim; ++d) acc = __fadd_rn(acc, __fmul_rn(qs[d], kcur[d]));
        sc[t] = __fmul_rn(acc, p.attn_scale);
        mx = fmaxf(mx, sc[t]);
    }
    // keys beyond the first NT (contexts longer than the thread count)
    for (int s = t + NT; s < npast; s += NT) {
        float acc = 0.0f;
        if (s == pos) {
            #pragma unroll 8
            for (int d = 0; d < kHeadDim; ++d) acc = __fadd_rn(acc, __fmul_rn(qs[d], kcur[d]));
        } else {
            #pragma unroll
            for (int d0 = 0; d0 < kHeadDim; d0 += 32) {
                float kv[32];
                #pragma unroll
                for (int j = 0; j < 32; ++j) kv[j] = kT.ld((size_t)(d0 + j) * nctx + s);
                #pragma unroll
                for (int j = 0; j < 32; ++j) acc = __fadd_rn(acc, __fmul_rn(qs[d0 + j], kv[j]));
            }
        }
        sc[s] = __fmul_rn(acc, p.attn_scale);
        mx = fmaxf(mx, sc[s]);
    }
    mx = warp_max(mx);
    if ((t & 31) == 0) fred[t >> 5] = mx;
    sync();

    // softmax (src/ops.c:386-422). The reference's max is the first-seen
    // maximum with '>'; with no NaN it is the same value (a NaN score
    // propagates identically below). Each thread exponentiates its own keys.
    mx = warp_max((t & 31) < NT / 32 ? fred[t & 31] : -INFINITY);
    const int nblk = npast & ~7;
    double part = 0.0;
    for (int s = t; s < npast; s += NT) {
        const float d = __fsub_rn(sc[s], mx);
        const float e = (s < nblk) ? v_expf(d) : sllm_libm_expf(d);
        sc[s] = e;
        part = __dadd_rn(part, (double)e);
    }
    part = warp_sum_d(part);
    if ((t & 31) == 0) dred[t >> 5] = part;
    sync();
    // every thread forms the same certified reciprocal: any order of these
    // npast non-negative terms lies within (npast + 64) * 2^-52 relative of
    // the reference's sum, and 1/x is monotone
    const double S = warp_sum_d((t & 31) < NT / 32 ? dred[t & 31] : 0.0);
    const double eb = (double)(npast + 64) * 0x1p-52;
    const float ia = __double2float_rn(__ddiv_rn(1.0, __dmul_ru(S, 1.0 + eb)));
    const float ib = __double2float_rn(__ddiv_rn(1.0, __dmul_rd(S, 1.0 - eb)));
    float inv = ia;
    if (f2u(ia) != f2u(ib) || p.force_fallback) {
        // reference order: per 8-block ((t0+t1)+t2)+t3 with t_k = e_k + e_{k+4};
        // the tail one at a time
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
        if (t == 0 && p.fallback_count != nullptr) atomicAdd(p.fallback_count, 1);
    }

    // o[d] = sum over s of w_s * v[s][d], sequential in s, with
    // w_s = fl(e_s * inv) (src/ops.c:418-421, src/forward.c:718-724).
    // r holds rows s .. s+RB-1 as batches of 16; while whole blocks of RB
    // rows follow, each batch is refilled with the rows RB further on as soon
    // as it has been added (no bounds predicates in that loop). Then the rows
    // left in r, and the last ones in batches of 16. RB = 64 for the fp32
    // cache; 32 for the f16 one, whose engine instance has fewer registers
    // to spare.
    if (pv_d >= 0) {
        constexpr int RB = std::is_same<KV, float>::value ? 64 : 32;
        const float vcur = vC.round(__ldcg(p.v + kvh * kHeadDim + pv_d));
        const int last = pos > 0 ? pos - 1 : 0;     // loads past the last stored row read that row
        float r[RB];
        float o = 0.0f;
        int s = 0;
        if (pos > 0) {
            #pragma unroll
            for (int j = 0; j < RB; ++j) r[j] = vC.ld((size_t)min(j, last) * kHeadDim + pv_d);
            #pragma unroll 1
            for (; s + RB < pos; s += RB) {
                // rows s .. s+RB-1 are all stored; refill with the next block
                #pragma unroll
                for (int b = 0; b < RB / 16; ++b) {
                    #pragma unroll
                    for (int j = 0; j < 16; ++j)
                        o = __fadd_rn(o, __fmul_rn(__fmul_rn(sc[s + 16 * b + j], inv), r[16 * b + j]));
                    #pragma unroll
                    for (int j = 0; j < 16; ++j)
                        r[16 * b + j] = vC.ld((size_t)min(s + RB + 16 * b + j, last) * kHeadDim + pv_d);
                }
            }
            // the last block: rows s .. pos-1
            const int rem = pos - s;
            #pragma unroll
            for (int b = 0; b < RB / 16; ++b) {
                if (16 * b < rem) {
                    #pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (16 * b + j < rem) o = __fadd_rn(o, __fmul_rn(__fmul_rn(sc[s + 16 * b + j], inv), r[16 * b + j]));
                }
            }
        }
        o = __fadd_rn(o, __fmul_rn(__fmul_rn(sc[pos], inv), vcur));
        p.out[h * kHeadDim + pv_d] = o;
    }
}

// The fp16 cache out of line: a kernel that inlines the fp32 head keeps its
// registers, and the fp16 head costs one call per head.
template <int NT, class Sync>
__device__ __noinline__ void attention_head_f16(const AttnParams& p, int h, int t, float* sc, float* qs, float* kcur,
                                                float* fred, double* dred, Sync sync) {
    attention_head_t<NT, __half>(p, h, t, sc, qs, kcur, fred, dred, sync);
}

template <int NT, class Sync>
__device__ __forceinline__ void attention_head(const AttnParams& p, int h, int t, float* sc, float* qs, float* kcur,
                                               float* fred, double* dred, Sync sync) {
    if (p.kv_f16 & kAttnKvF16)
        attention_head_f16<NT>(p, h, t, sc, qs, kcur, fred, dred, sync);
    else
        attention_head_t<NT, float>(p, h, t, sc, qs, kcur, fred, dred, sync);
}

}  // namespace sllm
