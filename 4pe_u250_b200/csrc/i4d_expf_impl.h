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
#endif

I4D_EXPF_QUAL float i4d_expf_core(float x, const double* table) {
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
    return I4D_D2F(I4D_DMUL(y, two_m));
}

#endif
