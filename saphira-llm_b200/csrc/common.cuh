// common.cuh -- device helpers shared by the sm_100a kernels.
//
// Floating-point contract: every kernel is compiled with -fmad=false and
// without fast-math (saphira-llm_b200/Makefile), so a*b+c is two IEEE
// roundings unless __fmaf_rn is written, and '/' and sqrtf are IEEE-exact.
// That is the reference's contract (-ffp-contract=off, its Makefile:34), and
// it is what makes bit-exact parity with its CPU path possible.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "../../include/sllm_cuda.h"

namespace sllm {

constexpr int kQK = 128;            // I2_S block: 128 elements in 32 bytes
constexpr int kMaxK = 65536;        // largest contracted width any kernel takes

// ---------------------------------------------------------------------------
// bit casts and loads
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// Weights are read exactly once per token: stream them past L1.
__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ld_stream_u128(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// ---------------------------------------------------------------------------
// I2_S unpack: one 32-bit word of a 32-byte block holds byte lanes j..j+3;
// field f of each byte (shift 6-2f) is element 32f + lane. Masking one field
// out of the word gives four consecutive codes that pair with the four
// consecutive int8 activations at 32f + j .. 32f + j + 3 -- one __dp4a.
// (src/quant.c:77-100, src/i2s_gemm.c:89-112 of saphira-llm.)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int i2s_dot_word(uint32_t w, int a0, int a1, int a2, int a3, int acc) {
    acc = __dp4a((int)((w >> 6) & 0x03030303u), a0, acc);
    acc = __dp4a((int)((w >> 4) & 0x03030303u), a1, acc);
    acc = __dp4a((int)((w >> 2) & 0x03030303u), a2, acc);
    acc = __dp4a((int)(w & 0x03030303u), a3, acc);
    return acc;
}

// ---------------------------------------------------------------------------
// activation quantisation, one element (src/i2s_gemm.c:74-81): roundf is
// half-away-from-zero; the reference's (int) cast turns a NaN or infinite
// product (an infinite input, or a scale that overflowed for a tiny amax) into
// INT_MIN on x86-64, which the clamp makes -128.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int quant_one(float x, float s) {
    const float p = __fmul_rn(x, s);
    if (!(fabsf(p) < 2147483648.0f)) return -128;
    float r = roundf(p);
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    return __float2int_rz(r);
}

// scale = amax > 0 ? 127/amax : 0 (src/i2s_gemm.c:70)
__device__ __forceinline__ float quant_scale(float amax) {
    return amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
}

// ---------------------------------------------------------------------------
// warp / block reductions (order-free ones only: max, integer sum)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// Certified rounding of the RMSNorm mean.
//
// The reference sums f32 squares into four f64 lanes in a fixed order and
// narrows (float)(ss / n) (src/ops.c:259-305). Any summation order of the same
// n non-negative f64 terms lands within (depth) * 2^-53 relative of the exact
// sum, and both orders here have depth below n + 64. So with the parallel sum
// S, the reference's ss lies in [S(1-e), S(1+e)] for e = (n + 64) * 2^-52, and
// because x -> (float)(x / n) is monotone, if both ends narrow to the same
// float that float IS the reference's mean. Otherwise the caller recomputes
// the sum in the reference's exact order (rare: about 1e-5 of calls).
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool certify_mean(double S, int n, float* mean) {
    const double e = (double)(n + 64) * 0x1p-52;
    const double lo = __dmul_rd(S, 1.0 - e);
    const double hi = __dmul_ru(S, 1.0 + e);
    const float mlo = __double2float_rn(__ddiv_rn(lo, (double)n));
    const float mhi = __double2float_rn(__ddiv_rn(hi, (double)n));
    *mean = mlo;
    return f2u(mlo) == f2u(mhi);
}

// The same certificate without a double division: a = S * (1/n) carries two
// more roundings, so the interval is widened by 8 * 2^-53 on top of the
// summation bound; RN(ss/n) lies in [a(1-E), a(1+E)] and narrows uniquely
// when both ends do.
__device__ __forceinline__ bool certify_mean_mul(double S, int n, double inv_n, float* mean) {
    const double E = (double)(n + 72) * 0x1p-52;
    const double a = __dmul_rn(S, inv_n);
    const float mlo = __double2float_rn(__dmul_rd(a, 1.0 - E));
    const float mhi = __double2float_rn(__dmul_ru(a, 1.0 + E));
    *mean = mlo;
    return f2u(mlo) == f2u(mhi);
}

// The reference's own order for n % 8 == 0 (src/ops.c:262-286): lane k adds
// (double)(x[8b+k]^2) then (double)(x[8b+4+k]^2) for b ascending; the lanes
// are summed 0..3. Only the fallback path runs this.
__device__ __forceinline__ double rms_ss_reference_order(const float* x, int n) {
    double l0 = 0.0, l1 = 0.0, l2 = 0.0, l3 = 0.0;
    for (int b = 0; b < n; b += 8) {
        l0 = __dadd_rn(l0, (double)__fmul_rn(x[b + 0], x[b + 0]));
        l1 = __dadd_rn(l1, (double)__fmul_rn(x[b + 1], x[b + 1]));
        l2 = __dadd_rn(l2, (double)__fmul_rn(x[b + 2], x[b + 2]));
        l3 = __dadd_rn(l3, (double)__fmul_rn(x[b + 3], x[b + 3]));
        l0 = __dadd_rn(l0, (double)__fmul_rn(x[b + 4], x[b + 4]));
        l1 = __dadd_rn(l1, (double)__fmul_rn(x[b + 5], x[b + 5]));
        l2 = __dadd_rn(l2, (double)__fmul_rn(x[b + 6], x[b + 6]));
        l3 = __dadd_rn(l3, (double)__fmul_rn(x[b + 7], x[b + 7]));
    }
    double ss = 0.0;
    ss = __dadd_rn(ss, l0);
    ss = __dadd_rn(ss, l1);
    ss = __dadd_rn(ss, l2);
    ss = __dadd_rn(ss, l3);
    return ss;
}

// scale = 1.0f / sqrtf(mean + eps) (src/ops.c:305-306)
__device__ __forceinline__ float rms_scale(float mean, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// ---------------------------------------------------------------------------
// ggml_v_expf, one lane (src/ops.c:342-379 of saphira-llm): the reference's
// polynomial exp, with the same FMAs in the same places.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float v_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = __fmaf_rn(x, 0x1.715476p+0f, r);
    const float nn = __fsub_rn(z, r);
    const float b = __fmaf_rn(-nn, 0x1.7f7d1cp-20f, __fmaf_rn(-nn, 0x1.62e4p-1f, x));
    const uint32_t e = f2u(z) << 23;
    const float k = u2f(e + 0x3f800000u);
    const bool c = fabsf(nn) > 126.0f;
    const float u = __fmul_rn(b, b);
    const float j = __fmaf_rn(__fmaf_rn(__fmaf_rn(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u,
                                        __fmaf_rn(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                              u, __fmul_rn(0x1.ffffecp-1f, b));
    if (!c) return __fmaf_rn(k, j, k);
    const uint32_t g = (nn <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = u2f(g + 0x7f000000u);
    const float s2 = u2f(e - g);
    if (fabsf(nn) > 192.0f) return __fmul_rn(s1, s1);
    return __fmul_rn(__fmaf_rn(s2, j, s2), s1);
}

// silu of one element of an 8-block (src/ops.c:452-456): v / (1 + exp(0 - v))
__device__ __forceinline__ float silu_block(float v) {
    return __fdiv_rn(v, __fadd_rn(1.0f, v_expf(__fsub_rn(0.0f, v))));
}

// f16 bits to f32 as src/forward.c:239-263 does for the embedding lookup:
// a subnormal half comes out at half its value there, reproduced.
__device__ __forceinline__ float f16_embd(uint16_t h) {
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0 && m != 0) {
        const float mag = __fmul_rn((float)m, 0x1p-25f);
        return (h & 0x8000u) ? -mag : mag;
    }
    return __half2float(__ushort_as_half(h));
}

}  // namespace sllm
