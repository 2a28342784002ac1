/*
 * dw_expf.h -- the exponential used by the SiLU epilogue of the fused INT8
 * convolution, shared by the CUDA kernels and by any host code that needs the
 * identical value.
 *
 * Why a shared definition: the reference computes SiLU as x * (1 / (1 + exp(-x)))
 * with Rust's f32::exp (crates/dragonwing-cpu/src/ops.rs:1865-1870, used by the
 * Mul(x, Sigmoid(x)) pattern that fusion.rs:126-190 collapses into SiLU), which
 * on Linux is the platform libm expf.  CUDA's expf and a libm expf may differ by
 * one unit in the last place, which can flip the final int8 rounding.  This file
 * defines one exp that both the device and the host evaluate identically, and
 * that is correctly rounded except in cases within 2^-52 relative of a float
 * rounding midpoint (so it agrees with a correctly rounded libm expf).
 *
 * Method (published):
 *   1. Cody & Waite range reduction (W. J. Cody, W. Waite, "Software Manual for
 *      the Elementary Functions", 1980): x = k*ln2 + r, k = rint(x/ln2), with ln2
 *      split into a 32-significant-bit high part and a low part (the split used
 *      by Sun's fdlibm e_exp.c), so k*ln2_hi is exact for |k| < 2^21.
 *   2. exp(r), |r| <= ln2/2, by its Taylor series sum_{n<=13} r^n/n! in Horner
 *      form; the truncation error r^14/14! < 4e-18 relative.
 *   3. Scale by 2^k (built from exponent bits; exact in double) and round once
 *      to float (IEEE round-to-nearest-even; handles overflow and subnormals).
 * Every double operation is a separately rounded IEEE multiply or add: the
 * device path uses the __dmul_rn/__dadd_rn intrinsics (never contracted into
 * FMA) and host code must be compiled with -ffp-contract=off.
 */
#ifndef DW_EXPF_H
#define DW_EXPF_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define DW_EXPF_QUAL __host__ __device__ static inline
#else
#define DW_EXPF_QUAL static inline
#endif

#if defined(__CUDA_ARCH__)
#define DW_DMUL(a, b) __dmul_rn((a), (b))
#define DW_DADD(a, b) __dadd_rn((a), (b))
#define DW_DSUB(a, b) __dsub_rn((a), (b))
#define DW_RINT(a) rint(a)
#else
#include <math.h>
#define DW_DMUL(a, b) ((a) * (b))
#define DW_DADD(a, b) ((a) + (b))
#define DW_DSUB(a, b) ((a) - (b))
#define DW_RINT(a) rint(a)
#endif

DW_EXPF_QUAL float dw_expf(float x) {
    if (x != x) return x;                       /* NaN propagates */
    if (x > 100.0f) return (float)(1e300 * 1e300); /* +inf (exp overflows above ~88.72) */
    if (x < -110.0f) return 0.0f;               /* exp(x) < 2^-150: rounds to +0 */
    const double kLog2e = 0x1.71547652b82fep+0; /* 1/ln2 */
    const double kLn2Hi = 0x1.62e42fee00000p-1; /* ln2 high part, 32 significant bits */
    const double kLn2Lo = 0x1.a39ef35793c76p-33; /* ln2 - kLn2Hi */
    /* 1/n! for n = 0..13, each correctly rounded to double. */
    const double c0 = 0x1.0000000000000p+0, c1 = 0x1.0000000000000p+0;
    const double c2 = 0x1.0000000000000p-1, c3 = 0x1.5555555555555p-3;
    const double c4 = 0x1.5555555555555p-5, c5 = 0x1.1111111111111p-7;
    const double c6 = 0x1.6c16c16c16c17p-10, c7 = 0x1.a01a01a01a01ap-13;
    const double c8 = 0x1.a01a01a01a01ap-16, c9 = 0x1.71de3a556c734p-19;
    const double c10 = 0x1.27e4fb7789f5cp-22, c11 = 0x1.ae64567f544e4p-26;
    const double c12 = 0x1.1eed8eff8d898p-29, c13 = 0x1.6124613a86d09p-33;

    const double xd = (double)x;
    const double kd = DW_RINT(DW_DMUL(xd, kLog2e));
    const double r = DW_DSUB(DW_DSUB(xd, DW_DMUL(kd, kLn2Hi)), DW_DMUL(kd, kLn2Lo));
    double p = c13;
    p = DW_DADD(DW_DMUL(p, r), c12);
    p = DW_DADD(DW_DMUL(p, r), c11);
    p = DW_DADD(DW_DMUL(p, r), c10);
    p = DW_DADD(DW_DMUL(p, r), c9);
    p = DW_DADD(DW_DMUL(p, r), c8);
    p = DW_DADD(DW_DMUL(p, r), c7);
    p = DW_DADD(DW_DMUL(p, r), c6);
    p = DW_DADD(DW_DMUL(p, r), c5);
    p = DW_DADD(DW_DMUL(p, r), c4);
    p = DW_DADD(DW_DMUL(p, r), c3);
    p = DW_DADD(DW_DMUL(p, r), c2);
    p = DW_DADD(DW_DMUL(p, r), c1);
    p = DW_DADD(DW_DMUL(p, r), c0);
    const int k = (int)kd;                      /* |k| <= 159 here */
    const uint64_t bits = (uint64_t)(int64_t)(k + 1023) << 52;
    double two_k;
    memcpy(&two_k, &bits, sizeof two_k);
    return (float)DW_DMUL(p, two_k);
}

/* SiLU of the contract: y * (1 / (1 + exp(-y))), each float op rounded to
 * nearest (ops.rs:1865-1870 for the sigmoid, fusion.rs:126-190 for x*sigmoid). */
DW_EXPF_QUAL float dw_silu_f32(float y) {
#if defined(__CUDA_ARCH__)
    const float e = dw_expf(-y);
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return __fmul_rn(y, sig);
#else
    const float e = dw_expf(-y);
    const float sig = 1.0f / (1.0f + e);
    return y * sig;
#endif
}

#endif /* DW_EXPF_H */
