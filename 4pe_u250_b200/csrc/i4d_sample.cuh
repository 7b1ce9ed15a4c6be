// i4d_sample.cuh -- the token sampler on the device (one CTA).
//
// Two reference samplers, selected by mode:
//   SAMPLE_HOST (0): the hardware host's Sampler (decode_host.cpp:724-868):
//     repeat penalty on finite logits, temperature 0 -> argmax with NaN
//     skipped, p_i = expf((v_i - max_finite) / T) (non-finite -> 0), serial
//     FP32 sum, p_i /= sum, coin from xorshift64*, multinomial (T > 0 and
//     top_p outside (0, 1)) or top-p with `nucleus >= top_p`.
//   SAMPLE_EMULATOR (1): the emulator's (llama2.c) sampler (emulator:1411-1569):
//     penalty on every logit, temperature 0 -> first strict maximum from
//     index 0, v_i /= T first, p_i = expf(v_i - max), top-p with
//     `cumulative > top_p`.
// Sums and walks that the references run serially (the softmax sum, the
// multinomial and nucleus walks) run serially here too, on one thread over
// shared memory: FP32 addition is not associative.  Everything else is
// parallel: the repeat penalty, the per-slice maxima (k_sample_prep) and the
// expf of every value (k_sample_exp) run over kSampleSlices CTAs first.  Top-p candidates (p >= (1 - top_p) / (n - 1)) are ordered by a
// stable LSD radix sort on the probability bits, so equal probabilities keep
// index order (both references use an unstable library sort there).
#pragma once

#include "i4d_device.cuh"
#include "i4d_expf.cuh"

namespace i4d {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kSampleMaxVocab = 32256;
constexpr int kSampleMaxHistory = 16384;
constexpr int kSampleSlices = 32;    // CTAs of the parallel passes, 1000 values each for 32000
enum SampleMode : int { SAMPLE_HOST = 0, SAMPLE_EMULATOR = 1 };
// Results below zero: the host sampler's exceptions.
constexpr int kSampleAllNan = -1;      // every logit NaN (argmax)
constexpr int kSampleNoFinite = -2;    // no finite logit
constexpr int kSampleBadSum = -3;      // probability sum not positive and finite

struct SampleArgs {
    const float* logits;      // [n]
    int n;                    // vocabulary (<= kSampleMaxVocab)
    const int* history;       // [n_history] token ids (any values; out-of-range ids are ignored)
    int n_history;
    float temperature, top_p, penalty;
    int mode;
    unsigned long long* state;  // xorshift64* state, advanced when a coin is drawn
    ExpfFix expf;
    float* v;                 // scratch [n]: penalised (and, emulator, temperature-divided) values, then expf
    float* slice_max;         // scratch [kSampleSlices]
    uint32_t* keys;           // scratch [2][kSampleMaxVocab]
    uint32_t* idx;            // scratch [2][kSampleMaxVocab]
    int* out;                 // token, or a negative code above
};

__host__ __device__ inline size_t sample_smem_bytes() {
    return static_cast<size_t>(kSampleMaxVocab) * 4 + kSampleWarps * 256 * 4;
}

__device__ __forceinline__ float sample_coin(unsigned long long* st) {
    unsigned long long s = *st;
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    *st = s;
    const uint32_t u = static_cast<uint32_t>((s * 0x2545F4914F6CDD1DULL) >> 32);
    return __fdiv_rn(static_cast<float>(u >> 8), 16777216.0f);
}

// Key of an argmax candidate: larger wins, equal values favour the smaller
// index, -0 counts as +0, NaN never wins (key 0).
__device__ __forceinline__ unsigned long long sample_key(float v, int i) {
    if (v != v) return 0ull;
    unsigned b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | (0xffffffffu - static_cast<unsigned>(i));
}

template <typename T, typename Op>
__device__ __forceinline__ T sample_block_reduce(T v, T* scratch, Op op) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    v = scratch[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// First index of the maximum of p[0, n) (NaN skipped); -1 if every value is NaN.
__device__ __forceinline__ int sample_argmax(const float* p, int n, unsigned long long* scratch) {
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += kSampleThreads) {
        const unsigned long long k = sample_key(p[i], i);
        best = k > best ? k : best;
    }
    best = sample_block_reduce(best, scratch, [](unsigned long long x, unsigned long long y) { return x > y ? x : y; });
    return best == 0ull ? -1 : static_cast<int>(0xffffffffu - static_cast<uint32_t>(best & 0xffffffffu));
}

// Serial FP32 sum of v[0, m), in order, from +0.0f.  Batches of 32 values
// are loaded before their chain of adds, so the loop runs at the add latency.
__device__ __forceinline__ float sample_serial_sum(const float* v, int m) {
    float s = 0.0f;
    int i = 0;
    for (; i + 32 <= m; i += 32) {
        float x[32];
#pragma unroll
        for (int k = 0; k < 32; k += 4) *reinterpret_cast<float4*>(x + k) = *reinterpret_cast<const float4*>(v + i + k);
#pragma unroll
        for (int k = 0; k < 32; ++k) s = __fadd_rn(s, x[k]);
    }
    for (; i < m; ++i) s = __fadd_rn(s, v[i]);
    return s;
}

// Serial running sums c_i = fl(c_{i-1} + v_i) (c_{-1} = +0.0f) written over
// v, up to the first i where stop(c_i) holds; returns that i, or m.  Batches
// of 32 are summed first and then checked element by element (a NaN makes
// every later sum NaN, so the end of a batch alone cannot tell).  v must be
// 16-byte aligned.
template <typename Stop>
__device__ __forceinline__ int sample_serial_prefix(float* v, int m, Stop stop) {
    float c = 0.0f;
    int i = 0;
    for (; i + 32 <= m; i += 32) {
        float x[32];
#pragma unroll
        for (int k = 0; k < 32; k += 4) *reinterpret_cast<float4*>(x + k) = *reinterpret_cast<const float4*>(v + i + k);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            c = __fadd_rn(c, x[k]);
            x[k] = c;
        }
#pragma unroll
        for (int k = 0; k < 32; k += 4) *reinterpret_cast<float4*>(v + i + k) = *reinterpret_cast<const float4*>(x + k);
        bool any = false;
#pragma unroll
        for (int k = 0; k < 32; ++k) any |= stop(x[k]);
        if (any) {
            for (int k = 0; k < 32; ++k)
                if (stop(x[k])) return i + k;
        }
    }
    for (; i < m; ++i) {
        c = __fadd_rn(c, v[i]);
        v[i] = c;
        if (stop(c)) return i;
    }
    return m;
}

__device__ __forceinline__ int sample_slice_len(int n) { return (n + kSampleSlices - 1) / kSampleSlices; }

// Pass 1 (kSampleSlices CTAs, one value per thread): the repeat penalty, once
// per distinct token (a token belongs to one slice, whose CTA marks it from
// the whole history), the emulator's division by the temperature, and the
// slice's maximum (host: finite values; emulator: non-NaN values).
__global__ void __launch_bounds__(kSampleThreads) k_sample_prep(const __grid_constant__ SampleArgs a) {
    __shared__ uint32_t marks[kSampleThreads / 32];
    __shared__ float red[32];
    const int tid = threadIdx.x;
    const int len = sample_slice_len(a.n), i0 = blockIdx.x * len, i1 = min(a.n, i0 + len);
    const bool host = a.mode == SAMPLE_HOST;
    if (tid < kSampleThreads / 32) marks[tid] = 0u;
    __syncthreads();
    if (a.penalty != 1.0f)
        for (int h = tid; h < a.n_history; h += kSampleThreads) {
            const int t = a.history[h];
            if (t >= i0 && t < i1) atomicOr(&marks[(t - i0) >> 5], 1u << ((t - i0) & 31));
        }
    __syncthreads();
    const int i = i0 + tid;
    float mx = -INFINITY;
    if (i < i1) {
        float v = a.logits[i];
        if ((marks[tid >> 5] >> (tid & 31)) & 1u)
            if (!host || isfinite(v)) v = v < 0.0f ? __fmul_rn(v, a.penalty) : __fdiv_rn(v, a.penalty);
        if (!host && a.temperature != 0.0f) v = __fdiv_rn(v, a.temperature);
        a.v[i] = v;
        if (host ? isfinite(v) : v == v) mx = v;
    }
    mx = sample_block_reduce(mx, red, [](float x, float y) { return fmaxf(x, y); });
    if (tid == 0) a.slice_max[blockIdx.x] = mx;
}

// The softmax maximum of the slice maxima (the emulator's stays NaN when its
// scan starts from a NaN at index 0).
__device__ __forceinline__ float sample_max(const SampleArgs& a) {
    float mx = -INFINITY;
    for (int s = 0; s < kSampleSlices; ++s) mx = fmaxf(mx, a.slice_max[s]);
    if (a.mode != SAMPLE_HOST && a.v[0] != a.v[0]) mx = a.v[0];
    return mx;
}

// Pass 2 (temperature > 0): the softmax numerators, expf as the C library.
__global__ void __launch_bounds__(kSampleThreads) k_sample_exp(const __grid_constant__ SampleArgs a) {
    const int len = sample_slice_len(a.n), i = blockIdx.x * len + threadIdx.x;
    if (threadIdx.x >= len || i >= a.n) return;
    const float mx = sample_max(a);
    const float v = a.v[i];
    if (a.mode == SAMPLE_HOST) a.v[i] = isfinite(v) ? expf_libc(__fdiv_rn(__fsub_rn(v, mx), a.temperature), a.expf) : 0.0f;
    else a.v[i] = expf_libc(__fsub_rn(v, mx), a.expf);
}

__global__ void __launch_bounds__(kSampleThreads, 1) k_sample(const __grid_constant__ SampleArgs a) {
    extern __shared__ __align__(16) uint8_t sample_smem[];
    float* p = reinterpret_cast<float*>(sample_smem);
    uint32_t* hist = reinterpret_cast<uint32_t*>(p + kSampleMaxVocab);  // [warp][256] radix counts
    __shared__ unsigned long long red64[32];
    __shared__ float redf[32];
    __shared__ int s_m;
    __shared__ float s_coin;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = a.n;
    const bool host = a.mode == SAMPLE_HOST;
    const float T = a.temperature;

    // The values of pass 1 (temperature 0) or the numerators of pass 2.
    for (int i = tid; i < n; i += kSampleThreads) p[i] = a.v[i];
    __syncthreads();
    if (T == 0.0f) {
        int r = sample_argmax(p, n, red64);
        if (!host && p[0] != p[0]) r = 0;  // the emulator's scan starts from a NaN at 0 and never leaves it
        if (tid == 0) *a.out = r < 0 ? kSampleAllNan : r;
        return;
    }
    if (host && !isfinite(sample_max(a))) {
        if (tid == 0) *a.out = kSampleNoFinite;
        return;
    }
    if (tid == 0) redf[0] = sample_serial_sum(p, n);  // the serial sum of both references
    __syncthreads();
    const float sum = redf[0];
    if (host && (!(sum > 0.0f) || !isfinite(sum))) {
        if (tid == 0) *a.out = kSampleBadSum;
        return;
    }
    for (int i = tid; i < n; i += kSampleThreads) p[i] = __fdiv_rn(p[i], sum);
    if (tid == 0) {
        unsigned long long st = *a.state;
        s_coin = sample_coin(&st);
        *a.state = st;
    }
    __syncthreads();
    const float coin = s_coin;
    const float top_p = a.top_p;
    if (top_p <= 0.0f || top_p >= 1.0f) {
        if (tid == 0) {  // multinomial walk: the first running sum above the coin
            const int r = sample_serial_prefix(p, n, [coin](float c) { return coin < c; });
            *a.out = r < n ? r : n - 1;
        }
        return;
    }
    // Top-p: candidates in index order (each thread compacts a contiguous range).
    const float cutoff = __fdiv_rn(__fsub_rn(1.0f, top_p), static_cast<float>(n - 1));
    const int per = (n + kSampleThreads - 1) / kSampleThreads;
    const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
    int cnt = 0;
    for (int i = i0; i < i1; ++i) cnt += p[i] >= cutoff;
    // Block exclusive scan of the counts.
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    __shared__ int wsum[32];
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = wsum[lane], wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        wsum[lane] = wi - w;
        if (lane == 31) s_m = wi;
    }
    __syncthreads();
    {
        int pos = wsum[warp] + incl - cnt;
        for (int i = i0; i < i1; ++i)
            if (p[i] >= cutoff) {
                a.keys[pos] = ~__float_as_uint(p[i]);  // p >= 0: descending probability
                a.idx[pos] = static_cast<uint32_t>(i);
                ++pos;
            }
    }
    __syncthreads();
    const int m = s_m;
    if (m == 0) {
        const int r = sample_argmax(p, n, red64);
        if (tid == 0) *a.out = r < 0 ? kSampleAllNan : r;
        return;
    }
    // Stable LSD radix sort, 4 passes of 8 bits; warp w owns a contiguous
    // segment and scatters it in order, so equal keys keep index order.
    const int seg = (m + kSampleWarps - 1) / kSampleWarps;
    const int sb = min(m, warp * seg), se = min(m, sb + seg);
    const unsigned FULL = 0xffffffffu;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 8 * pass;
        const uint32_t* ks = a.keys + (pass & 1) * kSampleMaxVocab;
        const uint32_t* is = a.idx + (pass & 1) * kSampleMaxVocab;
        uint32_t* kd = a.keys + ((pass + 1) & 1) * kSampleMaxVocab;
        uint32_t* id = a.idx + ((pass + 1) & 1) * kSampleMaxVocab;
        for (int e = tid; e < kSampleWarps * 256; e += kSampleThreads) hist[e] = 0u;
        __syncthreads();
        for (int i = sb + lane; i < se; i += 32) atomicAdd(&hist[warp * 256 + ((ks[i] >> shift) & 255u)], 1u);
        __syncthreads();
        // Exclusive scan in (digit, warp) order: thread t holds entries 8t..8t+7.
        {
            uint32_t v[8], loc = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int e = tid * 8 + k, d = e / kSampleWarps, w = e % kSampleWarps;
                v[k] = hist[w * 256 + d];
                loc += v[k];
            }
            uint32_t inc = loc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(FULL, inc, o);
                if (lane >= o) inc += y;
            }
            __shared__ uint32_t wtot[32];
            if (lane == 31) wtot[warp] = inc;
            __syncthreads();
            if (warp == 0) {
                const uint32_t w0 = wtot[lane];
                uint32_t wi = w0;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(FULL, wi, o);
                    if (lane >= o) wi += y;
                }
                wtot[lane] = wi - w0;
            }
            __syncthreads();
            uint32_t run = wtot[warp] + inc - loc;
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int e = tid * 8 + k, d = e / kSampleWarps, w = e % kSampleWarps;
                hist[w * 256 + d] = run;
                run += v[k];
            }
        }
        __syncthreads();
        for (int base = sb; base < se; base += 32) {
            const int i = base + lane;
            const bool valid = i < se;
            const uint32_t k = valid ? ks[i] : 0u;
            const uint32_t d = (k >> shift) & 255u;
            const unsigned peers = __match_any_sync(FULL, valid ? d : 256u + lane);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            if (valid) {
                const uint32_t at = hist[warp * 256 + d] + rank;
                kd[at] = k;
                id[at] = is[i];
            }
            __syncwarp();
            if (valid && lane == __ffs(peers) - 1) hist[warp * 256 + d] += __popc(peers);
            __syncwarp();
        }
        __syncthreads();
    }
    // Nucleus and the walk inside it: the sorted probabilities to shared
    // memory (p is free now), running sums in place, serially.
    for (int i = tid; i < m; i += kSampleThreads) p[i] = __uint_as_float(~a.keys[i]);  // four passes end in buffer 0
    __syncthreads();
    if (tid == 0) {
        int last;
        if (host) last = sample_serial_prefix(p, m, [top_p](float c) { return c >= top_p; });
        else last = sample_serial_prefix(p, m, [top_p](float c) { return c > top_p; });
        if (last > m - 1) last = m - 1;  // no break: the sum of every candidate
        const float cum = p[last];
        const float target = __fmul_rn(coin, cum);
        // First i <= last with target < c_i (the running sums do not decrease).
        int lo = 0, hi = last + 1;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (target < p[mid]) hi = mid;
            else lo = mid + 1;
        }
        *a.out = static_cast<int>(a.idx[lo <= last ? lo : last]);
    }
}

}  // namespace i4d
