// i4d_expf.cuh -- device binary32 exp that reproduces the host C library.
//
// i4d_expf_core (i4d_expf_impl.h) is evaluated in binary64; inputs on which
// the host C library's expf returns different bits were measured at build
// time (gen_expf_table.c) and are looked up here in an open-addressing hash
// table of (input bits, result bits) pairs built at context creation.
#pragma once

#define I4D_EXPF_DEVICE
#include "i4d_expf_impl.h"

#include <cstdint>

namespace i4d {

__device__ const double g_expf_table[64] = I4D_EXPF_TABLE_INIT;

// Exceptions table: a two-choice bucketed hash.  Bucket b is 8 words (one
// 32-byte sector): 4 keys (float bits of x, 0xffffffff = empty) then their
// 4 expf values.  A key sits in bucket h1 or h2, so a lookup is two
// independent sector loads, never a probe chain.
struct ExpfFix {
    const uint32_t* buckets;  // [mask + 1][8]
    uint32_t mask;
};

constexpr uint32_t kExpfSeed2 = 0x5bd1e995u;

__host__ __device__ __forceinline__ uint32_t expf_hash(uint32_t k) {
    k ^= k >> 16;
    k *= 0x7feb352du;
    k ^= k >> 15;
    k *= 0x846ca68bu;
    k ^= k >> 16;
    return k;
}

// The table value of x if it holds one, else y (a near-midpoint input).
__device__ __noinline__ float expf_table_fix(float x, float y, const ExpfFix& fx) {
    const uint32_t key = __float_as_uint(x);
    const uint4* B = reinterpret_cast<const uint4*>(fx.buckets);
    const uint32_t b1 = expf_hash(key) & fx.mask, b2 = expf_hash(key ^ kExpfSeed2) & fx.mask;
    const uint4 k1 = __ldg(B + 2 * b1), v1 = __ldg(B + 2 * b1 + 1);
    const uint4 k2 = __ldg(B + 2 * b2), v2 = __ldg(B + 2 * b2 + 1);
    uint32_t r = __float_as_uint(y);
    r = k1.x == key ? v1.x : r;
    r = k1.y == key ? v1.y : r;
    r = k1.z == key ? v1.z : r;
    r = k1.w == key ? v1.w : r;
    r = k2.x == key ? v2.x : r;
    r = k2.y == key ? v2.y : r;
    r = k2.z == key ? v2.z : r;
    r = k2.w == key ? v2.w : r;
    return __uint_as_float(r);
}

// The host C library's expf: the core, corrected from the table only where
// the core's result is near a rounding midpoint.  `table` is g_expf_table or
// a copy of it in shared memory (kernels whose L1 is mostly carved out for
// shared memory would otherwise fetch it from L2).
__device__ __forceinline__ float expf_libc(float x, const ExpfFix& fx, const double* table = g_expf_table) {
    int near_tie;
    const float y = i4d_expf_core2(x, table, &near_tie);
    return near_tie ? expf_table_fix(x, y, fx) : y;
}

// SwiGLU of one element (emulator:716-722): (g * (1 / (1 + e))) * u with
// e = expf(-g).
__device__ __forceinline__ float swiglu_e(float g, float u, float e) {
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return __fmul_rn(__fmul_rn(g, sig), u);
}
__device__ __forceinline__ float swiglu1(float g, float u, const ExpfFix& fx, const double* table = g_expf_table) {
    return swiglu_e(g, u, expf_libc(-g, fx, table));
}

}  // namespace i4d
