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

__device__ __forceinline__ float expf_libc(float x, const ExpfFix& fx) {
    const uint32_t key = __float_as_uint(x);
    const uint4* B = reinterpret_cast<const uint4*>(fx.buckets);
    const uint32_t b1 = expf_hash(key) & fx.mask, b2 = expf_hash(key ^ kExpfSeed2) & fx.mask;
    const uint4 k1 = __ldg(B + 2 * b1), v1 = __ldg(B + 2 * b1 + 1);
    const uint4 k2 = __ldg(B + 2 * b2), v2 = __ldg(B + 2 * b2 + 1);
    uint32_t y = __float_as_uint(i4d_expf_core(x, g_expf_table));
    y = k1.x == key ? v1.x : y;
    y = k1.y == key ? v1.y : y;
    y = k1.z == key ? v1.z : y;
    y = k1.w == key ? v1.w : y;
    y = k2.x == key ? v2.x : y;
    y = k2.y == key ? v2.y : y;
    y = k2.z == key ? v2.z : y;
    y = k2.w == key ? v2.w : y;
    return __uint_as_float(y);
}

// Key words of a bucket, kept in L2 across tokens (the table is small and hot).
__device__ __forceinline__ uint4 expf_bucket_keys(const ExpfFix& fx, uint32_t b, uint64_t pol) {
    uint4 k;
    asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(k.x), "=r"(k.y), "=r"(k.z), "=r"(k.w)
                 : "l"(fx.buckets + 8ull * b), "l"(pol));
    return k;
}

__device__ __forceinline__ int expf_match(uint4 k, uint32_t key) {
    return k.x == key ? 0 : k.y == key ? 1 : k.z == key ? 2 : k.w == key ? 3 : -1;
}

// SwiGLU of N elements with every table load issued before any is needed:
// the same results as N calls of swiglu1.
template <int N>
__device__ __forceinline__ void swiglu_n(const float (&g)[N], const float (&u)[N], float (&out)[N], const ExpfFix& fx) {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    uint4 ka[N], kb[N];
    uint32_t ba[N], bb[N];
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const uint32_t key = __float_as_uint(-g[i]);
        ba[i] = expf_hash(key) & fx.mask;
        bb[i] = expf_hash(key ^ kExpfSeed2) & fx.mask;
        ka[i] = expf_bucket_keys(fx, ba[i], pol);
        kb[i] = expf_bucket_keys(fx, bb[i], pol);
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float x = -g[i];
        const uint32_t key = __float_as_uint(x);
        float e = i4d_expf_core(x, g_expf_table);
        const int ma = expf_match(ka[i], key), mb = expf_match(kb[i], key);
        if (ma >= 0) e = __uint_as_float(__ldg(fx.buckets + 8ull * ba[i] + 4 + ma));
        else if (mb >= 0) e = __uint_as_float(__ldg(fx.buckets + 8ull * bb[i] + 4 + mb));
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
        out[i] = __fmul_rn(__fmul_rn(g[i], sig), u[i]);
    }
}

// SwiGLU of one element (emulator:716-722): (g * (1 / (1 + expf(-g)))) * u.
__device__ __forceinline__ float swiglu1(float g, float u, const ExpfFix& fx) {
    const float e = expf_libc(-g, fx);
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

}  // namespace i4d
