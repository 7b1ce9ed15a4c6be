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

struct ExpfFix {
    const uint32_t* slots;  // [2 * (mask + 1)]: key, value; key 0xffffffff = empty
    uint32_t mask;
    int max_probe;
};

__host__ __device__ __forceinline__ uint32_t expf_hash(uint32_t k) {
    k ^= k >> 16;
    k *= 0x7feb352du;
    k ^= k >> 15;
    k *= 0x846ca68bu;
    k ^= k >> 16;
    return k;
}

__device__ __forceinline__ float expf_libc(float x, const ExpfFix& fx) {
    const float y = i4d_expf_core(x, g_expf_table);
    const uint32_t key = __float_as_uint(x);
    uint32_t s = expf_hash(key) & fx.mask;
    for (int p = 0; p < fx.max_probe; ++p) {
        const uint2 e = __ldg(reinterpret_cast<const uint2*>(fx.slots) + s);
        if (e.x == key) return __uint_as_float(e.y);
        if (e.x == 0xffffffffu) break;
        s = (s + 1) & fx.mask;
    }
    return y;
}

// SwiGLU of one element (emulator:716-722): (g * (1 / (1 + expf(-g)))) * u.
__device__ __forceinline__ float swiglu1(float g, float u, const ExpfFix& fx) {
    const float e = expf_libc(-g, fx);
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

}  // namespace i4d
