// i4d_attention.cuh -- RoPE + INT8-KV online-softmax attention (SwiftKV).
//
// Replaces int4_swiftkv_attention_pe0..3 (swiftkv_attention.cpp:2759-2884):
// per head, the Q/K/V rows are finished from the QKV bank partials,
// converted to Q15.17, rotated with the RoPE LUT row of `position`, the
// current K/V are quantised into the 320-byte HLS record, and the cache is
// scanned with the reference's fixed-point online softmax.  The result is
// quantised to INT14 + E8M0 for the O projection.  All arithmetic is integer
// or single-rounding FP32 and bit-exact with emulator:602-714.
//
// Parallel form of the sequential recurrence: scores are exact integers and
// computed for all tokens at once; the running maximum before each token is
// a prefix maximum, so every softmax coefficient c_t is computed in
// parallel; only the normaliser and the per-dimension state chains run
// serially over tokens.
#pragma once

#include "i4d_device.cuh"

namespace i4d {

struct AttnArgs {
    const float* partials;   // QKV stage partials [4][12288], or null
    const int32_t* direct;   // Q15.17 q,k,v before RoPE [3][4096], or null
    const int* pos_ptr;      // decode position (device memory)
    const int32_t* rope_cos; // [4096][64] Q1.17
    const int32_t* rope_sin;
    const uint32_t* exp2_q30; // 33-entry LUT
    int log2e_q21;
    int32_t score_scale;      // float_to_q17(1/sqrt(128))
    uint8_t* kv;              // [4][layers][8][stride][320]
    int layers, stride, layer;
    int16_t* out_q;
    uint8_t* out_e;
    unsigned* err;
};

constexpr int kAttnThreads = 128;
constexpr int kMaxCtx = 4096;

// Fixed-point exp of a non-positive Q15.17 value (emulator:575-595,
// swiftkv_attention.cpp:199-260).
__device__ __forceinline__ uint32_t exp_negative_q17(int32_t x, const uint32_t* lut, int log2e_q21) {
    if (x >= 0) return 1u << 17;
    if (x <= -(32 << 17)) return 0;
    long long l2 = rshift_even(static_cast<long long>(x) * log2e_q21, 21);
    l2 = wrap_bits(l2, 24);
    const int ex = static_cast<int>(l2 >> 17);
    const int32_t fr = static_cast<int32_t>(l2 - (static_cast<long long>(ex) << 17));
    const unsigned idx = static_cast<unsigned>(fr) >> 12;
    const unsigned rem = static_cast<unsigned>(fr) & 0xfffu;
    const uint32_t base = lut[idx];
    const uint32_t delta = lut[idx + 1] - base;
    const uint32_t interp =
        base + static_cast<uint32_t>((static_cast<unsigned long long>(delta) * rem + (1u << 11)) >> 12);
    const int sh = 13 - ex;
    unsigned long long out = 0;
    if (sh <= 0) out = static_cast<unsigned long long>(interp) << (-sh);
    else if (sh < 32) out = (static_cast<unsigned long long>(interp) + (1ull << (sh - 1))) >> sh;
    return static_cast<uint32_t>(out) & ((1u << 18) - 1u);
}

// KV group shift: max(0, msb(max |v|) - 6) (swiftkv_attention.cpp:358-389).
__device__ __forceinline__ uint32_t kv_shift_of(uint32_t maxmag) {
    if (maxmag == 0) return 0;
    const int msb = 31 - __clz(maxmag);
    return msb > 6 ? static_cast<uint32_t>(msb - 6) : 0u;
}

// INT8 quantiser with round-half-up magnitude (swiftkv_attention.cpp:391-414).
__device__ __forceinline__ int kv_quant(int32_t raw, uint32_t shift) {
    const long long w = raw;
    unsigned long long mag = static_cast<unsigned long long>(w < 0 ? -w : w);
    if (shift) mag += 1ull << (shift - 1);
    mag >>= shift;
    if (mag > 127) mag = 127;
    return w < 0 ? -static_cast<int>(mag) : static_cast<int>(mag);
}

__device__ __forceinline__ uint8_t* kv_record(const AttnArgs& a, int head, int token) {
    const int bank = head / kLocalHeads, lh = head % kLocalHeads;
    const size_t rec = ((static_cast<size_t>(bank) * a.layers + a.layer) * kLocalHeads + lh) *
                           static_cast<size_t>(a.stride) + static_cast<size_t>(token);
    return a.kv + rec * 320;
}

__global__ void __launch_bounds__(kAttnThreads) k_attention(const AttnArgs a) {
    __shared__ int32_t s_q[kHeadDim], s_k[kHeadDim];
    __shared__ int8_t s_k8[kHeadDim], s_v8[kHeadDim];
    __shared__ uint32_t s_shift[8];
    __shared__ uint32_t s_lut[33];
    __shared__ int32_t s_score[kMaxCtx];
    __shared__ uint32_t s_coef[kMaxCtx];
    __shared__ int32_t s_cmax[kAttnThreads];
    __shared__ uint32_t s_norm;

    const int h = blockIdx.x, d = threadIdx.x, lane = d & 31, warp = d >> 5;
    if (d < 33) s_lut[d] = a.exp2_q30[d];
    pdl_trigger();
    pdl_wait();
    const int pos = *a.pos_ptr;
    if (pos < 0 || pos >= a.stride) {
        if (d == 0) atomicOr(a.err, kErrArg);
        return;
    }

    // Q/K/V rows of this head (finalizer pair tree + float_to_q17).
    int32_t qv, kv, vv;
    const int row = h * kHeadDim + d;
    if (a.direct) {
        qv = a.direct[row];
        kv = a.direct[kDim + row];
        vv = a.direct[2 * kDim + row];
    } else {
        qv = float_to_q17(combine4(a.partials, 3 * kDim, row));
        kv = float_to_q17(combine4(a.partials, 3 * kDim, kDim + row));
        vv = float_to_q17(combine4(a.partials, 3 * kDim, 2 * kDim + row));
    }
    s_q[d] = qv;
    s_k[d] = kv;
    __syncthreads();
    // Adjacent-pair RoPE (emulator:526-541).
    {
        const int pr = d >> 1;
        const long long c = a.rope_cos[pos * 64 + pr], sn = a.rope_sin[pos * 64 + pr];
        const long long qa = s_q[2 * pr], qb = s_q[2 * pr + 1];
        const long long ka = s_k[2 * pr], kb = s_k[2 * pr + 1];
        qv = (d & 1) ? sat32((qa * sn + qb * c) >> 17) : sat32((qa * c - qb * sn) >> 17);
        kv = (d & 1) ? sat32((ka * sn + kb * c) >> 17) : sat32((ka * c - kb * sn) >> 17);
    }
    __syncthreads();
    s_q[d] = qv;

    // Current token's KV record: warp = 32-value group.
    {
        const uint32_t kmag = static_cast<uint32_t>(kv < 0 ? -static_cast<long long>(kv) : kv);
        const uint32_t vmag = static_cast<uint32_t>(vv < 0 ? -static_cast<long long>(vv) : vv);
        const uint32_t ks = kv_shift_of(__reduce_max_sync(0xffffffffu, kmag));
        const uint32_t vs = kv_shift_of(__reduce_max_sync(0xffffffffu, vmag));
        const int k8 = kv_quant(kv, ks), v8 = kv_quant(vv, vs);
        s_k8[d] = static_cast<int8_t>(k8);
        s_v8[d] = static_cast<int8_t>(v8);
        if (lane == 0) {
            s_shift[warp] = ks;
            s_shift[4 + warp] = vs;
        }
        uint8_t* rec = kv_record(a, h, pos);
        rec[64 + d] = static_cast<uint8_t>(k8);
        rec[192 + d] = static_cast<uint8_t>(v8);
        __syncthreads();
        if (d < 8) {
            unsigned long long meta = 0;
            if (d == 0) {
                for (int g = 0; g < 4; ++g) {
                    meta |= static_cast<unsigned long long>(s_shift[g]) << (5 * g);
                    meta |= static_cast<unsigned long long>(s_shift[4 + g]) << (20 + 5 * g);
                }
            }
            reinterpret_cast<unsigned long long*>(rec)[d] = meta;
        }
    }

    // Scores for every token (emulator:633-655).
    {
        long long qe[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) qe[i] = s_q[4 * lane + i];
        const int grp = lane >> 3;
        for (int t = warp; t <= pos; t += 4) {
            uint32_t kw;
            uint32_t sh;
            if (t == pos) {
                kw = *reinterpret_cast<const uint32_t*>(s_k8 + 4 * lane);
                sh = s_shift[grp];
            } else {
                const uint8_t* rec = kv_record(a, h, t);
                kw = *reinterpret_cast<const uint32_t*>(rec + 64 + 4 * lane);
                const unsigned long long meta = *reinterpret_cast<const unsigned long long*>(rec);
                sh = static_cast<uint32_t>((meta >> (5 * grp)) & 31u);
            }
            long long part = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) part += qe[i] * static_cast<long long>(static_cast<int8_t>(kw >> (8 * i)));
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            long long hv = wrap_bits(sh >= 10 ? static_cast<long long>(static_cast<unsigned long long>(part) << (sh - 10))
                                              : (part >> (10 - sh)), 44);
            if (lane & 3) hv = 0;
            hv += __shfl_xor_sync(0xffffffffu, hv, 4);
            hv += __shfl_xor_sync(0xffffffffu, hv, 8);
            hv += __shfl_xor_sync(0xffffffffu, hv, 16);
            const long long dot = wrap_bits(hv, 44);
            if (lane == 0) s_score[t] = sat32(rshift_even(dot * a.score_scale, 24));
        }
    }
    __syncthreads();

    // Coefficients from the prefix maximum (emulator:656-672).
    const int n = pos + 1;
    const int cs = (n + kAttnThreads - 1) / kAttnThreads;
    const int t0 = d * cs, t1 = min(n, t0 + cs);
    {
        int32_t m = INT32_MIN;
        for (int t = t0; t < t1; ++t) m = max(m, s_score[t]);
        s_cmax[d] = m;
    }
    __syncthreads();
    {
        int32_t run = INT32_MIN;  // max of all tokens before t0
        for (int i = 0; i < d; ++i) run = max(run, s_cmax[i]);
        for (int t = t0; t < t1; ++t) {
            const int32_t sc = s_score[t];
            uint32_t cf;
            if (t == 0) {
                cf = 1u << 17;
            } else if (sc <= run) {
                cf = exp_negative_q17(sat32(static_cast<long long>(sc) - run), s_lut, a.log2e_q21);
            } else {
                cf = exp_negative_q17(sat32(static_cast<long long>(run) - sc), s_lut, a.log2e_q21) | 0x80000000u;
            }
            s_coef[t] = cf;
            run = max(run, sc);
        }
    }
    __syncthreads();

    // Normaliser chain (thread 0) and state chain (one dimension per thread).
    if (d == 0) {
        uint32_t z = 1u << 17;
        const uint32_t m30 = (1u << 30) - 1u;
        for (int t = 1; t < n; ++t) {
            const uint32_t cf = s_coef[t];
            const uint32_t c = cf & 0x7fffffffu;
            if (cf >> 31) z = ((static_cast<uint32_t>(rshift_even(static_cast<long long>(z) * c, 17)) & m30) + (1u << 17)) & m30;
            else z = (z + c) & m30;
        }
        s_norm = z;
    }
    const int grp = d >> 5;
    int32_t st = 0;
    for (int t = 0; t < n; ++t) {
        int32_t val;
        if (t == pos) {
            val = static_cast<int32_t>(s_v8[d]) << s_shift[4 + grp];
        } else {
            const uint8_t* rec = kv_record(a, h, t);
            const unsigned long long meta = *reinterpret_cast<const unsigned long long*>(rec);
            val = static_cast<int32_t>(static_cast<int8_t>(rec[192 + d])) << ((meta >> (20 + 5 * grp)) & 31u);
        }
        const uint32_t cf = s_coef[t];
        const uint32_t c = cf & 0x7fffffffu;
        if (t == 0) st = val;
        else if (cf >> 31) st = sat32(static_cast<long long>(mulq17(st, c)) + val);
        else st = sat32(static_cast<long long>(st) + mulq17(val, c));
    }
    __syncthreads();

    // Normalise and quantise the head output (emulator:686-711).
    const uint32_t z = s_norm;
    const uint32_t inv = z == 0 ? 0u : static_cast<uint32_t>(((1ull << 34) + (z >> 1)) / z);
    const int32_t o = mulq17(st, inv);
    const int32_t mag = o == INT32_MIN ? INT32_MAX : abs(o);
    const int32_t mx = __reduce_max_sync(0xffffffffu, mag);
    const float maxf = __fmul_rn(__int2float_rn(mx), 1.0f / 131072.0f);
    int maxe = -127;
    if (maxf != 0.0f) frexpf(maxf, &maxe);
    const float inv_scale = maxf == 0.0f ? 0.0f : pow2f(13 - maxe);
    float r = __fmul_rn(__fmul_rn(__int2float_rn(o), 1.0f / 131072.0f), inv_scale);
    r = __fadd_rn(r, r >= 0.0f ? 0.5f : -0.5f);
    r = fmaxf(-8191.0f, fminf(8191.0f, r));
    a.out_q[row] = static_cast<int16_t>(__float2int_rz(r));
    if (lane == 0) a.out_e[h * 4 + warp] = maxf == 0.0f ? 0 : static_cast<uint8_t>(maxe + 127);
}

}  // namespace i4d
