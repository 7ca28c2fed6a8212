/*
 * lal_expf.h -- the sampler's exp, bit-identical to glibc's expf on every
 * non-positive float.
 *
 * The reference weighs each top-k candidate with libm expf
 * (runtime/lal_sampling.h:112,120; tools/server/qwen7b_server.c:283,290) and
 * sums the weights sequentially in float.  To reproduce those sums bit for bit
 * on the GPU, the device evaluates exp in double precision with a fixed
 * sequence of IEEE operations (identical on host and device: explicit fma,
 * no contraction), rounds once to float, and then consults a table of the
 * inputs on which glibc's float result differs from that rounding.  The table
 * is produced at build time by gen_expf_fixups.c, which calls the host's
 * glibc expf on all 2^31 non-positive floats; the table therefore encodes
 * glibc's observable outputs only.
 *
 * Method: Cody & Waite argument reduction x = k*ln2 + r with the two-part ln2
 * split published with fdlibm, a degree-13 Taylor polynomial for exp(r) on
 * |r| <= ln2/2 in Horner form (truncation error < 4e-18 relative), and an
 * exact scaling by 2^k built from the exponent bits.
 *
 * Inputs the sampler can produce are (l - max_l) / T with T > 0 and
 * l <= max_l, i.e. x <= 0 (or NaN); positive inputs are computed without
 * table fix-ups.
 */
#ifndef LAL_EXPF_H
#define LAL_EXPF_H

#include <stdint.h>

#if defined(__CUDACC__)
#define LAL_HD __host__ __device__ __forceinline__
#else
#define LAL_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define LAL_FMA(a, b, c) __fma_rn((a), (b), (c))
#define LAL_MUL(a, b) __dmul_rn((a), (b))
#define LAL_RINT(a) rint(a)
#else
#include <math.h>
#define LAL_FMA(a, b, c) fma((a), (b), (c))
#define LAL_MUL(a, b) ((a) * (b))
#define LAL_RINT(a) rint(a)
#endif

LAL_HD double lal_exp_core(double x) {
    const double inv_ln2 = 1.4426950408889634074;       /* 1/ln 2 */
    const double ln2_hi = 6.93147180369123816490e-01;   /* fdlibm ln2_hi */
    const double ln2_lo = 1.90821492927058770002e-10;   /* fdlibm ln2_lo */
    double k = LAL_RINT(LAL_MUL(x, inv_ln2));
    double r = LAL_FMA(-k, ln2_hi, x);
    r = LAL_FMA(-k, ln2_lo, r);
    /* sum_{n=0}^{13} r^n / n!, Horner */
    double p = 1.0 / 6227020800.0;                      /* 1/13! */
    p = LAL_FMA(p, r, 1.0 / 479001600.0);               /* 1/12! */
    p = LAL_FMA(p, r, 1.0 / 39916800.0);
    p = LAL_FMA(p, r, 1.0 / 3628800.0);
    p = LAL_FMA(p, r, 1.0 / 362880.0);
    p = LAL_FMA(p, r, 1.0 / 40320.0);
    p = LAL_FMA(p, r, 1.0 / 5040.0);
    p = LAL_FMA(p, r, 1.0 / 720.0);
    p = LAL_FMA(p, r, 1.0 / 120.0);
    p = LAL_FMA(p, r, 1.0 / 24.0);
    p = LAL_FMA(p, r, 1.0 / 6.0);
    p = LAL_FMA(p, r, 0.5);
    p = LAL_FMA(p, r, 1.0);
    p = LAL_FMA(p, r, 1.0);
    int64_t ki = (int64_t)k;
    uint64_t bits = (uint64_t)(ki + 1023) << 52;         /* 2^k, k in [-151, 128] */
    double s;
#if defined(__CUDA_ARCH__)
    s = __longlong_as_double((long long)bits);
#else
    union { uint64_t u; double d; } cv; cv.u = bits; s = cv.d;
#endif
    return LAL_MUL(p, s);
}

/* exp rounded once to float; 0 below -110 and for -inf, NaN passes through. */
LAL_HD float lal_expf_rounded(float x) {
    if (x != x) return x;
    if (x < -110.0f) return 0.0f;
    if (x > 88.8f) return (float)(1.0e300 * 1.0e300);   /* +inf, as expf overflows */
    return (float)lal_exp_core((double)x);
}

LAL_HD uint32_t lal_f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    union { float f; uint32_t u; } cv; cv.f = f; return cv.u;
#endif
}
LAL_HD float lal_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    union { uint32_t u; float f; } cv; cv.u = u; return cv.f;
#endif
}

/* glibc-exact expf: the rounded value, corrected from the sorted fix-up table
 * (tab_x: input bit patterns ascending, tab_y: glibc's result bits). */
LAL_HD float lal_expf_glibc(float x, const uint32_t *tab_x, const uint32_t *tab_y, int n) {
    float y = lal_expf_rounded(x);
    if (!(x <= 0.0f) || n <= 0) return y;
    uint32_t xb = lal_f2u(x);
    int lo = 0, hi = n - 1;
    while (lo <= hi) {
        int mid = (lo + hi) >> 1;
        uint32_t v = tab_x[mid];
        if (v == xb) return lal_u2f(tab_y[mid]);
        if (v < xb) lo = mid + 1; else hi = mid - 1;
    }
    return y;
}

#endif /* LAL_EXPF_H */
