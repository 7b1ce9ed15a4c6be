/*
 * i4d_expf_impl.h -- the library's binary32 exp, shared by host and device.
 *
 * Table-driven method of P. T. P. Tang (ACM TOMS 15(2), 1989) evaluated in
 * binary64: k = rint(x * 64/ln2), r = x - k*ln2/64 (two-constant reduction
 * with fused multiply-adds), exp(r) - 1 by its Taylor series to degree 6,
 * result 2^(k>>6) * T[k&63] * (1 + q) rounded once to binary32.  Its relative
 * error before the final rounding is about 2^-52, so it is correctly rounded
 * except on a handful of inputs.  The host C library's expf (which the
 * reference emulator calls, software_sim/llama2_decoder_sw_emulator.cpp:719)
 * is not correctly rounded everywhere; gen_expf_table.c compares the two on
 * every binary32 input and records each input where they differ, and the
 * device applies that table (see i4d_expf.cuh).
 *
 * The same operation sequence runs on host and device (only IEEE mul, fma,
 * rint and conversions), so both produce identical bits.  Define
 * I4D_EXPF_DEVICE before including for the CUDA form.
 *
 * Where the table can matter: a function whose error is below 0.502 ulp (the
 * C library's stated bound) returns the correctly rounded value unless the
 * exact result lies within 0.002 ulp of a rounding midpoint.  The core's
 * binary64 value locates that midpoint; i4d_expf_near_tie flags results
 * within 1/128 ulp of one (and zero, subnormal or overflowing results), and
 * only those consult the table.  gen_expf_table.c checks, on every input,
 * that each recorded difference is flagged.
 */
#ifndef I4D_EXPF_IMPL_H
#define I4D_EXPF_IMPL_H

#include "gen/expf_consts.h"

#ifdef I4D_EXPF_DEVICE
#define I4D_EXPF_QUAL __device__ __forceinline__
#define I4D_FMA(a, b, c) __fma_rn((a), (b), (c))
#define I4D_DMUL(a, b) __dmul_rn((a), (b))
#define I4D_RINT(a) rint(a)
#define I4D_D2F(a) __double2float_rn(a)
#define I4D_D_AS_U64(d) ((unsigned long long)__double_as_longlong(d))
#define I4D_U64_AS_D(u) __longlong_as_double((long long)(u))
#define I4D_F_AS_U32(f) __float_as_uint(f)
#define I4D_U32_AS_F(u) __uint_as_float(u)
#else
#include <math.h>
#include <string.h>
#define I4D_EXPF_QUAL static inline
#define I4D_FMA(a, b, c) fma((a), (b), (c))
#define I4D_DMUL(a, b) ((a) * (b))
#define I4D_RINT(a) rint(a)
#define I4D_D2F(a) ((float)(a))
static inline double i4d_u64_as_d(unsigned long long u) { double d; memcpy(&d, &u, 8); return d; }
#define I4D_U64_AS_D(u) i4d_u64_as_d(u)
static inline unsigned i4d_f_as_u32(float f) { unsigned u; memcpy(&u, &f, 4); return u; }
static inline float i4d_u32_as_f(unsigned u) { float f; memcpy(&f, &u, 4); return f; }
#define I4D_F_AS_U32(f) i4d_f_as_u32(f)
#define I4D_U32_AS_F(u) i4d_u32_as_f(u)
#endif

/* Nonzero when the binary64 value yd, rounded to the binary32 f, lies within
 * 1/128 of f's spacing from a rounding midpoint, or when f is zero,
 * subnormal, the largest finite value or infinite.  Every operation is exact:
 * yd - f and the spacings are differences of nearby values. */
I4D_EXPF_QUAL int i4d_expf_near_tie(double yd, float f) {
    const unsigned u = I4D_F_AS_U32(f);
    if (u < 0x00800000u || u >= 0x7f7fffffu) return 1;
    const double fd = (double)f;
    const double r = yd - fd;
    const double up = (double)I4D_U32_AS_F(u + 1u) - fd;
    const double dn = fd - (double)I4D_U32_AS_F(u - 1u);
    const double sp = r >= 0.0 ? up : dn;
    const double dist = 0.5 * sp - (r >= 0.0 ? r : -r);
    return dist < sp * (1.0 / 128.0);
}

/* expf(x) by the method above; *near_tie as i4d_expf_near_tie (0 for NaN,
 * x > 100 and x < -110, whose results every implementation shares). */
I4D_EXPF_QUAL float i4d_expf_core2(float x, const double* table, int* near_tie) {
    *near_tie = 0;
    if (x != x) return x;
    if (x > 100.0f) return __builtin_inff();
    if (x < -110.0f) return 0.0f;
    const double xd = (double)x;
    const double kd = I4D_RINT(I4D_DMUL(xd, I4D_EXPF_INV_LN2_64));
    const int k = (int)kd;
    double r = I4D_FMA(-kd, I4D_EXPF_LN2_64_HI, xd);
    r = I4D_FMA(-kd, I4D_EXPF_LN2_64_LO, r);
    double p = I4D_FMA(I4D_EXPF_C6, r, I4D_EXPF_C5);
    p = I4D_FMA(p, r, I4D_EXPF_C4);
    p = I4D_FMA(p, r, I4D_EXPF_C3);
    p = I4D_FMA(p, r, I4D_EXPF_C2);
    const double q = I4D_FMA(I4D_DMUL(r, r), p, r);
    const double t = table[k & 63];
    const double y = I4D_FMA(t, q, t);
    const int m = k >> 6;
    const double two_m = I4D_U64_AS_D((unsigned long long)(m + 1023) << 52);
    const double yd = I4D_DMUL(y, two_m);
    const float f = I4D_D2F(yd);
    *near_tie = i4d_expf_near_tie(yd, f);
    return f;
}

I4D_EXPF_QUAL float i4d_expf_core(float x, const double* table) {
    int near_tie;
    return i4d_expf_core2(x, table, &near_tie);
}

#endif
