/*
 * loom_select_math.h -- the arithmetic that decides a sampled token.
 *
 * The sampling chain's decision stage (softmax over the top-k survivors, the top-p cutoff and the
 * inverse-CDF draw) runs in double precision, and its result must be identical bit for bit on the
 * host and on the GPU. Two things make that possible:
 *
 *   1. every operation below is an IEEE-754 basic operation (add, sub, mul, div, fused multiply-add)
 *      in round-to-nearest, written so that no compiler may contract or reassociate it (the device
 *      build spells each one as an explicit `__*_rn` intrinsic; the host build is compiled with
 *      `-ffp-contract=off`);
 *   2. the exponential is this file's own `loom_exp_d`, not a library `exp`, so both sides evaluate
 *      the same formula.
 *
 * loom_exp_d: exp(x) for double x, from the textbook method.
 *   - Argument reduction (Cody & Waite, "Software Manual for the Elementary Functions", 1980):
 *     n = nearest integer to x / ln 2, r = (x - n*L1) - n*L2, where L1 + L2 = ln 2 and L1 has only
 *     42 significant bits so that n*L1 is exact for |n| < 2^11. Then |r| <= ln(2)/2.
 *   - exp(r) by its Taylor series sum_{k=0}^{13} r^k / k!, evaluated in Horner form with fused
 *     multiply-adds. The first omitted term is below 2^-54 of the result for |r| <= ln(2)/2.
 *   - The result is scaled by 2^n through the exponent field, in two exact steps when it is
 *     subnormal so that only the final multiply rounds.
 *   The constants were derived here from ln 2 and 1/k! (computed in 80-digit decimal arithmetic and
 *   rounded to double); none is taken from any vendor math library.
 *
 * Plain C (C99) and CUDA C++ both compile this header.
 */
#ifndef LOOM_SELECT_MATH_H
#define LOOM_SELECT_MATH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define LOOM_HD __host__ __device__ __forceinline__
#else
#include <math.h>
#include <string.h>
#define LOOM_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define LOOM_DADD(a, b) __dadd_rn((a), (b))
#define LOOM_DSUB(a, b) __dsub_rn((a), (b))
#define LOOM_DMUL(a, b) __dmul_rn((a), (b))
#define LOOM_DDIV(a, b) __ddiv_rn((a), (b))
#define LOOM_DFMA(a, b, c) __fma_rn((a), (b), (c))
#else
#define LOOM_DADD(a, b) ((a) + (b))
#define LOOM_DSUB(a, b) ((a) - (b))
#define LOOM_DMUL(a, b) ((a) * (b))
#define LOOM_DDIV(a, b) ((a) / (b))
#define LOOM_DFMA(a, b, c) fma((a), (b), (c))
#endif

LOOM_HD double loom_bits_to_double(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double d;
    memcpy(&d, &u, sizeof d);
    return d;
#endif
}

/* 2^e for an integer e in [-1022, 1023], built in the exponent field (exact). */
LOOM_HD double loom_pow2_d(int e) {
    return loom_bits_to_double((uint64_t)(int64_t)(e + 1023) << 52);
}

LOOM_HD double loom_exp_d(double x) {
    /* log2(e), and ln 2 split as L1 (42 significant bits) + L2. */
    const double kLog2e = 0x1.71547652b82fep+0;
    const double kL1 = 0x1.62e42fefa3800p-1;
    const double kL2 = 0x1.ef35793c76730p-45;
    /* 1.5 * 2^52: adding then subtracting it rounds a |t| < 2^51 to the nearest integer (ties even). */
    const double kRound = 0x1.8p52;
    if (x != x) return x;                   /* NaN */
    if (x > 709.8) return loom_bits_to_double(0x7ff0000000000000ull); /* overflow to +inf */
    if (x < -745.2) return 0.0;             /* below half the smallest subnormal */
    const double t = LOOM_DMUL(x, kLog2e);
    const double nd = LOOM_DSUB(LOOM_DADD(t, kRound), kRound);
    const double r = LOOM_DFMA(-nd, kL2, LOOM_DFMA(-nd, kL1, x));
    double p = 0x1.6124613a86d09p-33;       /* 1/13! */
    p = LOOM_DFMA(p, r, 0x1.1eed8eff8d898p-29); /* 1/12! */
    p = LOOM_DFMA(p, r, 0x1.ae64567f544e4p-26); /* 1/11! */
    p = LOOM_DFMA(p, r, 0x1.27e4fb7789f5cp-22); /* 1/10! */
    p = LOOM_DFMA(p, r, 0x1.71de3a556c734p-19); /* 1/9! */
    p = LOOM_DFMA(p, r, 0x1.a01a01a01a01ap-16); /* 1/8! */
    p = LOOM_DFMA(p, r, 0x1.a01a01a01a01ap-13); /* 1/7! */
    p = LOOM_DFMA(p, r, 0x1.6c16c16c16c17p-10); /* 1/6! */
    p = LOOM_DFMA(p, r, 0x1.1111111111111p-7);  /* 1/5! */
    p = LOOM_DFMA(p, r, 0x1.5555555555555p-5);  /* 1/4! */
    p = LOOM_DFMA(p, r, 0x1.5555555555555p-3);  /* 1/3! */
    p = LOOM_DFMA(p, r, 0.5);                   /* 1/2! */
    p = LOOM_DFMA(p, r, 1.0);
    p = LOOM_DFMA(p, r, 1.0);
    const int n = (int)nd;
    if (n > 1023) return LOOM_DMUL(LOOM_DMUL(p, loom_pow2_d(1023)), loom_pow2_d(n - 1023));
    if (n >= -1022) return LOOM_DMUL(p, loom_pow2_d(n));
    /* subnormal result: the first scaling is exact, the second rounds once */
    return LOOM_DMUL(LOOM_DMUL(p, loom_pow2_d(n + 600)), loom_pow2_d(-600));
}

/*
 * The ordering key of the sampling chain: a larger key ranks first.
 * Values order as floats do, -0 and +0 share one key, and NaN ranks below -inf.
 */
LOOM_HD uint32_t loom_order_key(float y) {
    if (y != y) return 0u;
#if defined(__CUDA_ARCH__)
    uint32_t u = (uint32_t)__float_as_uint(y);
#else
    uint32_t u;
    memcpy(&u, &y, sizeof u);
#endif
    if ((u & 0x7fffffffu) == 0u) u = 0u; /* -0 -> +0 */
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* Full key of a (value, id) pair: value descending, then id ascending. Larger ranks first. */
LOOM_HD uint64_t loom_rank_key(float y, int32_t id) {
    return ((uint64_t)loom_order_key(y) << 32) | (uint64_t)(0xffffffffu - (uint32_t)id);
}

/*
 * Weight of survivor i in the survivor softmax: exp(y_i - m) in double, with m the top survivor's
 * value. NaN survivors (and every survivor when m itself is NaN) weigh 0; a survivor equal to m
 * weighs exactly 1, which also covers m = +-inf.
 */
LOOM_HD double loom_survivor_weight(float y, float m) {
    if (y != y || m != m) return 0.0;
    if (y == m) return 1.0;
    return loom_exp_d(LOOM_DSUB((double)y, (double)m));
}

#endif /* LOOM_SELECT_MATH_H */
