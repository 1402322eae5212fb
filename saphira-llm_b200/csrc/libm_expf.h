/*
 * libm_expf.h -- the host C library's expf, restated so that device code can
 * reproduce it bit for bit.
 *
 * saphira-llm's softmax computes the n % 8 tail with libm expf
 * (src/ops.c:413-417), so a bit-exact device softmax needs the host libm's
 * exact results. glibc (2.27 and later, like musl) implements expf with the
 * published algorithm of ARM's optimized-routines library (Szabolcs Nagy,
 * 2017): with N = 32,
 *
 *     z  = x * (N / ln 2)                    in double
 *     k  = round(z) via the 1.5 * 2^52 shift trick,  r = z - k
 *     s  = 2^(k/N), from a table of 2^(i/N) (i = k mod N) with k/N folded
 *          into the exponent bits
 *     p  = 1 + r*C2 + r^2*(C1 + r*C0)        (C: a degree-3 fit of 2^(r/N))
 *     expf(x) = (float)(p * s)
 *
 * with r and the polynomial evaluated by fused multiply-adds, as the x86-64
 * FMA build that glibc selects on any x86-64-v3 CPU evaluates them (r as
 * fma(x, N/ln2, -k), which is what makes the last two of 2^32 inputs agree). The table below
 * is the correctly rounded double of 2^(i/32) minus i << 47, computed for this
 * file with 60-digit decimal arithmetic. tests/test_libm_expf.py checks this
 * function against the host's expf over every float, so a host libm that
 * disagrees is caught before any device result depends on it.
 *
 * Plain C99 and CUDA at once: the CPU test compiles this header with gcc, the
 * attention kernel includes it as device code.
 */
#ifndef SLLM_LIBM_EXPF_H
#define SLLM_LIBM_EXPF_H

#include <stdint.h>

#ifdef __CUDACC__
#  define SLLM_EXPF_FN __device__ __forceinline__
#  define SLLM_EXPF_TABLE __device__ __constant__
#  ifdef __CUDA_ARCH__
#    define SLLM_FMA_D(a, b, c) __fma_rn((a), (b), (c))
#    define SLLM_D2U(d) ((uint64_t) __double_as_longlong(d))
#    define SLLM_U2D(u) __longlong_as_double((long long) (u))
#    define SLLM_F2U(f) __float_as_uint(f)
#    define SLLM_U2F(u) __uint_as_float(u)
#  endif
#else
#  include <math.h>
#  include <string.h>
#  define SLLM_EXPF_FN static inline
#  define SLLM_EXPF_TABLE static const
#endif

#ifndef SLLM_FMA_D
#  define SLLM_FMA_D(a, b, c) fma((a), (b), (c))
static inline uint64_t sllm_d2u_(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }
static inline double sllm_u2d_(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static inline uint32_t sllm_f2u_(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float sllm_u2f_(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
#  define SLLM_D2U(d) sllm_d2u_(d)
#  define SLLM_U2D(u) sllm_u2d_(u)
#  define SLLM_F2U(f) sllm_f2u_(f)
#  define SLLM_U2F(u) sllm_u2f_(u)
#endif

SLLM_EXPF_TABLE uint64_t sllm_exp2f_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

SLLM_EXPF_FN float sllm_libm_expf(float x) {
    const uint32_t ux = SLLM_F2U(x);
    const uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {                       /* |x| >= 88, or inf / nan */
        if (ux == 0xff800000u) return 0.0f;       /* -inf */
        if (abstop >= 0x7f8u) return x + x;       /* +inf or nan */
        if (x > 0x1.62e42ep6f) return SLLM_U2F(0x7f800000u);   /* overflow: +inf */
        if (x < -0x1.9fe368p6f) return 0.0f;                    /* underflow: +0 */
    }
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = (double) x;
    const double z = inv_ln2_n * xd;
    double kd = z + shift;
    const uint64_t ki = SLLM_D2U(kd);
    kd -= shift;
    /* the FMA build contracts r = z - kd into one fused operation */
    const double r = SLLM_FMA_D(inv_ln2_n, xd, -kd);
    const uint64_t t = sllm_exp2f_tab[ki % 32] + (ki << 47);
    const double s = SLLM_U2D(t);
    const double zz = SLLM_FMA_D(c0, r, c1);
    const double r2 = r * r;
    double y = SLLM_FMA_D(c2, r, 1.0);
    y = SLLM_FMA_D(zz, r2, y);
    y = y * s;
    return (float) y;
}

#endif /* SLLM_LIBM_EXPF_H */
