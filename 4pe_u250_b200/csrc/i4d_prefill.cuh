// i4d_prefill.cuh -- prompt batches: up to kPrefillMax tokens per pass over
// the weights.
//
// The reference runs a prompt one token at a time through the whole decoder
// (decode_host.cpp:1570-1580, run_one_token at :1340), so every prompt token
// streams all 3.46 GB of weights.  Here the GEMV stages of a layer take a
// batch of T prompt tokens: each weight chunk is streamed into shared memory
// once and every consumer warp applies it to its own token.  Per (token, row)
// the arithmetic is the decode path's unchanged (exact G32 int32 dots on the
// split activations, contrib = fl(float(dot) * fl(ws * as)), the FP32 chain
// in local-group order from +0.0f, emulator:216-264), so each token's
// partials, residual and KV record are bit-identical to decoding it alone.
// Attention runs per (head, token) in two launches (i4d_attention.cuh phase
// 1 writes all T records, phase 2 attends), which is the decode order: token
// t reads records 0..t.
#pragma once

#include "i4d_device.cuh"
#include "i4d_expf.cuh"
#include "i4d_linear.cuh"

namespace i4d {

constexpr int kPrefillMax = 16;                      // tokens per batch = consumer warps
constexpr int kBatchThreads = 32 * (1 + kPrefillMax);
constexpr int kBatchSlots = 24;                      // chunk ring slots
constexpr int kPfTok = 11264;                        // activation columns per token (DOWN input)

struct BatchArgs {
    const uint8_t* w;       // unit 0 of bank 0 of the stage (GEMV layout)
    size_t bank_stride;     // bytes from one bank's unit 0 to the next bank's
    int cpb;                // CTAs per bank; gridDim.x == 4 * cpb
    int units;              // units per bank
    int chunks;             // chunks per unit
    int T;                  // tokens in the batch, 1..kPrefillMax
    const int16_t* act_q;   // [T][kPfTok]; bank b at b * act_bank_stride
    const uint8_t* act_e;   // [T][kPfTok / 32]
    int act_bank_stride;
    float* partials;        // [T][4][units * 32]
    unsigned* err;
};

__host__ __device__ inline size_t batch_smem_bytes(int chunks, int T) {
    return static_cast<size_t>(kBatchSlots) * kChunkBytes + 2 * kBatchSlots * 8 +
           static_cast<size_t>(T) * chunks * 8 * 72;
}

// One CTA per SM: a producer thread streams the CTA's units chunk by chunk;
// consumer warp t (token t) reads every chunk, lane = row, and chains the
// unit's 8 x chunks group contributions in order in a register.
__global__ void __launch_bounds__(kBatchThreads, 1) k_linear_batch(const __grid_constant__ BatchArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int groups = a.chunks * 8;
    uint8_t* ring = smem_raw;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + static_cast<size_t>(kBatchSlots) * kChunkBytes);
    uint64_t* empty = full + kBatchSlots;
    uint8_t* act_base = reinterpret_cast<uint8_t*>(empty + kBatchSlots);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bank = blockIdx.x / a.cpb, c = blockIdx.x % a.cpb;
    const int u0 = static_cast<int>((static_cast<long long>(c) * a.units) / a.cpb);
    const int u1 = static_cast<int>((static_cast<long long>(c + 1) * a.units) / a.cpb);
    const int nchunks = (u1 - u0) * a.chunks;
    const int nt = a.T < kPrefillMax ? a.T : kPrefillMax;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kBatchSlots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], nt);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            const uint8_t* src = a.w + static_cast<size_t>(bank) * a.bank_stride +
                                 static_cast<size_t>(u0) * a.chunks * kChunkBytes;
            int slot = 0;
            uint32_t phase = 0;
            for (int i = 0; i < nchunks; ++i) {
                if (i >= kBatchSlots) mbar_wait(&empty[slot], phase ^ 1u, a.err, kErrWaitEmpty);
                mbar_arrive_expect_tx(&full[slot], kChunkBytes);
                bulk_g2s(ring + static_cast<size_t>(slot) * kChunkBytes, src + static_cast<size_t>(i) * kChunkBytes,
                         kChunkBytes, &full[slot]);
                if (++slot == kBatchSlots) {
                    slot = 0;
                    phase ^= 1u;
                }
            }
        }
        return;
    }
    const int t = warp - 1;
    if (t >= nt) return;

    // This token's split activations (layout of put_act, per token).
    int8_t* hi = reinterpret_cast<int8_t*>(act_base + static_cast<size_t>(t) * groups * 72);
    uint8_t* lo = reinterpret_cast<uint8_t*>(hi + groups * 32);
    int* corr = reinterpret_cast<int*>(lo + groups * 32);
    float* ascale = reinterpret_cast<float*>(corr + groups);
    {
        const size_t base = static_cast<size_t>(t) * kPfTok + static_cast<size_t>(bank) * a.act_bank_stride;
        const int16_t* q = a.act_q + base;
        const uint8_t* e = a.act_e + base / 32;
        for (int lg = 0; lg < groups; ++lg) {
            const int v = q[lg * 32 + lane];
            hi[lg * 32 + lane] = static_cast<int8_t>(v >> 7);
            lo[lg * 32 + lane] = static_cast<uint8_t>(v & 127);
            const int lo16 = __reduce_add_sync(0xffffffffu, lane < 16 ? v : 0);
            if (lane == 0) {
                corr[lg] = 8 * lo16;
                ascale[lg] = e8m0_scale(e[lg]);
            }
        }
    }
    __syncwarp();

    const int rows_total = a.units * 32;
    float* out = a.partials + (static_cast<size_t>(t) * 4 + bank) * rows_total + lane;
    float acc = 0.0f;
    int j = 0, u = u0, slot = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nchunks; ++i) {
        mbar_wait(&full[slot], phase, a.err, kErrWaitFull);
        const uint8_t* ch = ring + static_cast<size_t>(slot) * kChunkBytes;
        uint4 wv[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) wv[g] = *reinterpret_cast<const uint4*>(ch + chunk_piece(lane, g));
        const int16_t raw0 = reinterpret_cast<const int16_t*>(ch)[lane * 2];
        const int16_t raw1 = reinterpret_cast<const int16_t*>(ch)[lane * 2 + 1];
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == kBatchSlots) {
            slot = 0;
            phase ^= 1u;
        }
        const float ws0 = __fmul_rn(static_cast<float>(raw0), 1.0f / 32768.0f);
        const float ws1 = __fmul_rn(static_cast<float>(raw1), 1.0f / 32768.0f);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const int lg = j * 8 + g;
            const int dot = group_dot(wv[g], hi + lg * 32, lo + lg * 32, corr[lg]);
            acc = __fadd_rn(acc, __fmul_rn(static_cast<float>(dot), __fmul_rn(g < 4 ? ws0 : ws1, ascale[lg])));
        }
        if (++j == a.chunks) {
            out[static_cast<size_t>(u) * 32] = acc;
            acc = 0.0f;
            j = 0;
            ++u;
        }
    }
}

// Per-token prologue of a norm (one CTA of 1024 threads per token): the
// optional residual update r += (p0+p1)+(p2+p3) from a stage's partials, the
// RMS reciprocal of r (rms_recip_warp: the reference's 8 serial slots per
// bank, emulator:427-447) and, when gamma is set, q = quantize(fl(fl(r * inv)
// * gamma)) in G32 groups (emulator:448-453).
struct PfNormArgs {
    float* resid;            // [T][4096]
    const float* partials;   // [T][4][rows], or null (no residual update)
    int rows;                // rows of the partials' stage
    const float* gamma;      // [4096], or null (no quantisation)
    float* recip;            // [T]
    int16_t* q;              // [T][kPfTok]
    uint8_t* e;              // [T][kPfTok / 32]
};

__global__ void __launch_bounds__(1024) k_pf_norm(const __grid_constant__ PfNormArgs a) {
    const int t = blockIdx.x, i = threadIdx.x;
    float* r = a.resid + static_cast<size_t>(t) * kDim;
    float x[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int col = i + k * 1024;
        x[k] = r[col];
        if (a.partials) {
            x[k] = __fadd_rn(x[k], combine4(a.partials + static_cast<size_t>(t) * 4 * a.rows, a.rows, col));
            r[col] = x[k];
        }
    }
    __shared__ float inv_s;
    __syncthreads();
    if (i < 32) {
        const float inv = rms_recip_warp(r);
        if (i == 0) {
            inv_s = inv;
            a.recip[t] = inv;
        }
    }
    __syncthreads();
    if (!a.gamma) return;
    const float inv = inv_s;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int col = i + k * 1024;
        uint32_t e8;
        const int q = quantize_g32_lane(__fmul_rn(__fmul_rn(x[k], inv), a.gamma[col]), &e8);
        a.q[static_cast<size_t>(t) * kPfTok + col] = static_cast<int16_t>(q);
        if ((col & 31) == 0) a.e[static_cast<size_t>(t) * (kPfTok / 32) + (col >> 5)] = static_cast<uint8_t>(e8);
    }
}

// SwiGLU of the GATE/UP partials then the G32 quantiser, per token (as
// linear_finalize's EPI_SWIGLU; emulator:716-722, 769-770).  Grid (stripes, T).
__global__ void __launch_bounds__(32) k_pf_swiglu(const float* partials, int units, ExpfFix fx, int16_t* q,
                                                   uint8_t* e) {
    const int stripe = blockIdx.x, t = blockIdx.y, lane = threadIdx.x;
    const int rows = units * 32, stripes = units / 2;
    const float* P = partials + static_cast<size_t>(t) * 4 * rows;
    const float g = combine4(P, rows, stripe * 32 + lane);
    const float u = combine4(P, rows, (stripes + stripe) * 32 + lane);
    uint32_t e8;
    const int v = quantize_g32_lane(swiglu1(g, u, fx), &e8);
    q[static_cast<size_t>(t) * kPfTok + stripe * 32 + lane] = static_cast<int16_t>(v);
    if (lane == 0) e[static_cast<size_t>(t) * (kPfTok / 32) + stripe] = static_cast<uint8_t>(e8);
}

// Prompt embeddings: resid[t] = emb[ids[t]] (ids checked on the host).
__global__ void __launch_bounds__(1024) k_pf_embed(const float* emb, const int* ids, float* resid) {
    const int t = blockIdx.x;
    const float4* src = reinterpret_cast<const float4*>(emb + static_cast<size_t>(ids[t]) * kDim);
    reinterpret_cast<float4*>(resid + static_cast<size_t>(t) * kDim)[threadIdx.x] = src[threadIdx.x];
}

}  // namespace i4d
