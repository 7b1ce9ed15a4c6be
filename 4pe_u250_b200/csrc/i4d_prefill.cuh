// i4d_prefill.cuh -- prompt batches: up to kPrefillMax tokens per pass over
// the weights.
//
// The reference runs a prompt one token at a time through the whole decoder
// (decode_host.cpp:1570-1580, run_one_token at :1340), so every prompt token
// streams all 3.46 GB of weights.  Here the GEMV stages of a layer take a
// batch of T prompt tokens: each weight chunk is streamed into shared memory
// once and applied to all T tokens with int8 tensor-core MMAs.  Per (token, row)
// the arithmetic is the decode path's unchanged (exact G32 int32 dots on the
// split activations, contrib = fl(float(dot) * fl(ws * as)), the FP32 chain
// in local-group order from +0.0f, emulator:216-264), so each token's
// partials, residual and KV record are bit-identical to decoding it alone.
// Attention runs per (head, token) in two launches (k_pf_kv writes all T
// records, then k_attention phase 2 attends), which is the decode order:
// token t reads records 0..t.  Every kernel of a batch is launched with
// programmatic dependent launch: it waits for its predecessor before reading
// any of its outputs, and the GEMV producer streams weights before that.
#pragma once

#include "i4d_device.cuh"
#include "i4d_expf.cuh"
#include "i4d_linear.cuh"
#include "i4d_sample.cuh"
#include "i4d_token.cuh"

namespace i4d {

constexpr int kPrefillMax = 32;                      // tokens per batch (four MMA token tiles)
constexpr int kBatchWarps = 16;                      // MMA warps: units in flight x 2 row tiles x token tiles
constexpr int kBatchThreads = 32 * (1 + kBatchWarps);
constexpr int kBatchSlots = 24;                      // most chunk ring slots
constexpr int kBatchSmemMax = 232448;                // dynamic shared memory of one CTA (227 KB)
constexpr int kPfTok = 11264;                        // activation columns per token (DOWN input)

struct BatchArgs {
    const uint8_t* w;       // unit 0 of bank 0 of the stage (GEMV layout)
    size_t bank_stride;     // bytes from one bank's unit 0 to the next bank's
    int cpb;                // CTAs per bank; gridDim.x == 4 * cpb
    int units;              // units per bank
    int chunks;             // chunks per unit
    int T;                  // tokens in the batch, 1..kPrefillMax
    int ns;                 // ring slots (batch_slots), 2..kBatchSlots
    const int16_t* act_q;   // [T][kPfTok]; bank b at b * act_bank_stride
    const uint8_t* act_e;   // [T][kPfTok / 32]
    int act_bank_stride;
    float* partials;        // [T][4][units * 32]
    unsigned* err;
};

// Per-token activation block in shared memory: ah [groups][32] (int8),
// al [groups][32] (0..127), the group scales [groups] (FP32) and 16 bytes of
// padding.  The stride, groups * 17 + 4 words, is 4 x an odd number, so the 8
// tokens that one MMA B fragment reads start in 8 distinct 4-bank groups.
__host__ __device__ constexpr int batch_tok_stride(int groups) { return groups * 68 + 16; }

// Token tiles of 8 in use for T tokens, and the units a CTA works on at a
// time: 4 (two token tiles or fewer) or 2 (four token tiles).
__host__ __device__ constexpr int batch_tiles(int T) { return (T + 7) >> 3; }
__host__ __device__ constexpr int batch_units(int T) { return batch_tiles(T) <= 2 ? 4 : 2; }

__host__ __device__ inline size_t batch_fixed_bytes(int chunks, int T) {
    return 2 * kBatchSlots * 8 + align16(kBatchSlots * 4) +
           static_cast<size_t>(8 * batch_tiles(T)) * batch_tok_stride(chunks * 8);
}

// Ring slots that fit beside the activations (DOWN at 32 tokens: 9).
__host__ __device__ inline int batch_slots(int chunks, int T) {
    const long long n = (kBatchSmemMax - static_cast<long long>(batch_fixed_bytes(chunks, T))) / kChunkBytes;
    return static_cast<int>(n < kBatchSlots ? n : kBatchSlots);
}

__host__ __device__ inline size_t batch_smem_bytes(int chunks, int T, int ns) {
    return static_cast<size_t>(ns) * kChunkBytes + batch_fixed_bytes(chunks, T);
}

// Four INT4 weights of one packed word as int8 MMA operands, both scaled by
// 16: the low nibbles hold w + 8 (offset binary) and the high nibbles w
// (two's complement), so 16w is (x << 4) ^ 0x80 and (x & 0xF0) per byte.
__device__ __forceinline__ uint32_t w16_lo(uint32_t x) { return ((x << 4) & 0xF0F0F0F0u) ^ 0x80808080u; }
__device__ __forceinline__ uint32_t w16_hi(uint32_t x) { return x & 0xF0F0F0F0u; }

// D = A (16 x 32 int8, row-major) x B (32 x 8 int8), int32.
__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// One CTA per SM.  A producer thread streams the CTA's units in rounds of
// batch_units(T), chunk j of every unit of the round before chunk j + 1, into
// a ring.  Warp (s, rt, tt) takes unit s of each round, rows 16 rt .. 16 rt +
// 15 of it and tokens 8 tt .. 8 tt + 7: per chunk and G32 group two int8
// MMAs (the activation's high and low parts, a = 128 ah + al) give the exact
// int32 dot of every (row, token), and each (row, token) chains its group
// contributions in order in a register, as the decode path.
__global__ void __launch_bounds__(kBatchThreads, 1) k_linear_batch(const __grid_constant__ BatchArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int groups = a.chunks * 8;
    const int tstride = batch_tok_stride(groups);
    const int ns = a.ns;
    uint8_t* ring = smem_raw;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + static_cast<size_t>(ns) * kChunkBytes);
    uint64_t* empty = full + kBatchSlots;
    int* issued = reinterpret_cast<int*>(empty + kBatchSlots);
    uint8_t* act = reinterpret_cast<uint8_t*>(issued) + align16(kBatchSlots * 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bank = blockIdx.x / a.cpb, c = blockIdx.x % a.cpb;
    const int u0 = static_cast<int>((static_cast<long long>(c) * a.units) / a.cpb);
    const int u1 = static_cast<int>((static_cast<long long>(c + 1) * a.units) / a.cpb);
    const int nunits = u1 - u0;
    const int T = a.T < kPrefillMax ? a.T : kPrefillMax;
    const int ntt = batch_tiles(T);   // token tiles in use
    const int upr = batch_units(T);   // units per round
    const int wpu = kBatchWarps / upr;  // warps per unit: 2 row tiles x (wpu / 2) token tiles

    if (threadIdx.x == 0) {
        for (int i = 0; i < ns; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 2 * ntt);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < ns) issued[threadIdx.x] = -1;
    __syncthreads();
    pdl_trigger();

    if (warp == 0) {  // weights never depend on earlier kernels: no wait
        if (lane == 0) {
            const uint8_t* src = a.w + static_cast<size_t>(bank) * a.bank_stride +
                                 static_cast<size_t>(u0) * a.chunks * kChunkBytes;
            int idx = 0, slot = 0;
            uint32_t phase = 0;
            for (int rb = 0; rb < nunits; rb += upr) {
                const int nu = min(upr, nunits - rb);
                for (int j = 0; j < a.chunks; ++j)
                    for (int su = 0; su < nu; ++su, ++idx) {
                        if (idx >= ns) mbar_wait(&empty[slot], phase ^ 1u, a.err, kErrWaitEmpty);
                        publish_issued(&issued[slot], idx);
                        mbar_arrive_expect_tx(&full[slot], kChunkBytes);
                        bulk_g2s(ring + static_cast<size_t>(slot) * kChunkBytes,
                                 src + (static_cast<size_t>(rb + su) * a.chunks + j) * kChunkBytes, kChunkBytes,
                                 &full[slot]);
                        if (++slot == ns) {
                            slot = 0;
                            phase ^= 1u;
                        }
                    }
            }
        }
        return;
    }

    // Activations of tokens 0 .. 8 ntt - 1 (zero past T): 8 values per
    // thread and step, split into ah / al bytes; then the group scales.
    const int cw = warp - 1, ct = threadIdx.x - 32;
    pdl_wait();
    {
        const int per_tok = groups * 4;  // 8-value pieces per token
        for (int i = ct; i < 8 * ntt * per_tok; i += 32 * kBatchWarps) {
            const int n = i / per_tok, col = (i - n * per_tok) * 8;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (n < T)
                v = *reinterpret_cast<const uint4*>(a.act_q + static_cast<size_t>(n) * kPfTok +
                                                    static_cast<size_t>(bank) * a.act_bank_stride + col);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            uint32_t hv[2] = {0u, 0u}, lv[2] = {0u, 0u};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int q = static_cast<int16_t>((w[k >> 1] >> (16 * (k & 1))) & 0xffffu);
                hv[k >> 2] |= (static_cast<uint32_t>(q >> 7) & 0xffu) << (8 * (k & 3));
                lv[k >> 2] |= static_cast<uint32_t>(q & 127) << (8 * (k & 3));
            }
            uint8_t* tb = act + static_cast<size_t>(n) * tstride;
            *reinterpret_cast<uint2*>(tb + col) = make_uint2(hv[0], hv[1]);
            *reinterpret_cast<uint2*>(tb + groups * 32 + col) = make_uint2(lv[0], lv[1]);
        }
        for (int i = ct; i < 8 * ntt * groups; i += 32 * kBatchWarps) {
            const int n = i / groups, lg = i - n * groups;
            float* asc = reinterpret_cast<float*>(act + static_cast<size_t>(n) * tstride + groups * 64);
            asc[lg] = n < T ? e8m0_scale(a.act_e[(static_cast<size_t>(n) * kPfTok +
                                                  static_cast<size_t>(bank) * a.act_bank_stride) / 32 + lg])
                            : 0.0f;
        }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(32 * kBatchWarps) : "memory");
    const int su = cw / wpu, rt = cw & 1, tt = (cw % wpu) >> 1;
    if (tt >= ntt) return;

    const int gid = lane >> 2, tig = lane & 3;
    const int r0 = rt * 16 + gid, r1 = r0 + 8;           // rows of c0/c1 and c2/c3
    const int n0 = tt * 8 + 2 * tig;                      // tokens of c0/c2 and c1/c3
    const uint8_t* tb = act + static_cast<size_t>(tt * 8 + gid) * tstride;  // B operand: token tt*8 + gid
    const uint8_t* bh = tb + 4 * tig;
    const uint8_t* bl = tb + groups * 32 + 4 * tig;
    const float* as0 = reinterpret_cast<const float*>(act + static_cast<size_t>(n0) * tstride + groups * 64);
    const float* as1 = reinterpret_cast<const float*>(act + static_cast<size_t>(n0 + 1) * tstride + groups * 64);
    const int rows_total = a.units * 32;
    const size_t tok_stride = static_cast<size_t>(4) * rows_total;
    float* out = a.partials + static_cast<size_t>(bank) * rows_total;
    // chunk_piece(r, g) for the two rows (r & 7 == gid; r >> 3 == 2 rt, 2 rt + 1)
    const int p0 = kChunkScaleBytes + ((gid * 4 + 2 * rt) * 8) * 16 + 4 * tig;
    const int p1 = p0 + 8 * 16;

    for (int rb = 0; rb + su < nunits; rb += upr) {
        const int nu = min(upr, nunits - rb);
        float c00 = 0.0f, c01 = 0.0f, c10 = 0.0f, c11 = 0.0f;  // [row r0/r1][token n0/n0+1]
        for (int j = 0; j < a.chunks; ++j) {
            const int idx = rb * a.chunks + j * nu + su;
            const int slot = idx % ns;
            wait_issued(&issued[slot], idx, a.err);
            mbar_wait(&full[slot], static_cast<uint32_t>((idx / ns) & 1), a.err, kErrWaitFull);
            const uint8_t* ch = ring + static_cast<size_t>(slot) * kChunkBytes;
            uint32_t w0[8], w1[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                w0[g] = *reinterpret_cast<const uint32_t*>(ch + p0 + ((g ^ gid) << 4));
                w1[g] = *reinterpret_cast<const uint32_t*>(ch + p1 + ((g ^ gid) << 4));
            }
            const int16_t* sc = reinterpret_cast<const int16_t*>(ch);
            const float ws00 = __fmul_rn(static_cast<float>(sc[r0 * 2]), 1.0f / 32768.0f);
            const float ws01 = __fmul_rn(static_cast<float>(sc[r0 * 2 + 1]), 1.0f / 32768.0f);
            const float ws10 = __fmul_rn(static_cast<float>(sc[r1 * 2]), 1.0f / 32768.0f);
            const float ws11 = __fmul_rn(static_cast<float>(sc[r1 * 2 + 1]), 1.0f / 32768.0f);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const int lg = j * 8 + g;
                const uint32_t a0 = w16_lo(w0[g]), a1 = w16_lo(w1[g]), a2 = w16_hi(w0[g]), a3 = w16_hi(w1[g]);
                const uint32_t h0 = *reinterpret_cast<const uint32_t*>(bh + lg * 32);
                const uint32_t h1 = *reinterpret_cast<const uint32_t*>(bh + lg * 32 + 16);
                const uint32_t l0 = *reinterpret_cast<const uint32_t*>(bl + lg * 32);
                const uint32_t l1 = *reinterpret_cast<const uint32_t*>(bl + lg * 32 + 16);
                int dh[4], dl[4];
                mma_s8(dh, a0, a1, a2, a3, h0, h1);
                mma_s8(dl, a0, a1, a2, a3, l0, l1);
                // 16 * dot = 16 * (128 * sum(w ah) + sum(w al)); exact in int32
                const int d0 = (dh[0] * 128 + dl[0]) >> 4, d1 = (dh[1] * 128 + dl[1]) >> 4;
                const int d2 = (dh[2] * 128 + dl[2]) >> 4, d3 = (dh[3] * 128 + dl[3]) >> 4;
                const float s0 = as0[lg], s1 = as1[lg];
                const float wa = g < 4 ? ws00 : ws01, wb = g < 4 ? ws10 : ws11;
                c00 = __fadd_rn(c00, __fmul_rn(static_cast<float>(d0), __fmul_rn(wa, s0)));
                c01 = __fadd_rn(c01, __fmul_rn(static_cast<float>(d1), __fmul_rn(wa, s1)));
                c10 = __fadd_rn(c10, __fmul_rn(static_cast<float>(d2), __fmul_rn(wb, s0)));
                c11 = __fadd_rn(c11, __fmul_rn(static_cast<float>(d3), __fmul_rn(wb, s1)));
            }
        }
        const size_t row0 = static_cast<size_t>(u0 + rb + su) * 32 + r0;
        if (n0 < T) {
            out[n0 * tok_stride + row0] = c00;
            out[n0 * tok_stride + row0 + 8] = c10;
        }
        if (n0 + 1 < T) {
            out[(n0 + 1) * tok_stride + row0] = c01;
            out[(n0 + 1) * tok_stride + row0 + 8] = c11;
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
    pdl_trigger();
    pdl_wait();
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
    // RMS as rms_recip_warp, one bank per warp: lane s < 8 of warp b sums
    // slot s of bank b (8 lanes, 8 distinct shared-memory banks).
    __shared__ float xs[kDim];
    __shared__ float bank_total[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) xs[i + k * 1024] = x[k];
    __syncthreads();
    const int w = i >> 5, lane = i & 31;
    if (w < 4 && lane < 8) {
        const float* base = xs + w * 1024 + lane;
        float acc = 0.0f;
#pragma unroll 32
        for (int k = 0; k < 128; ++k) {
            const float v = base[k * 8];
            acc = __fadd_rn(acc, __fmul_rn(v, v));
        }
        float total = 0.0f;
        for (int sl = 0; sl < 8; ++sl) total = __fadd_rn(total, __shfl_sync(0xffu, acc, sl));
        if (lane == 0) bank_total[w] = total;
    }
    __syncthreads();
    const float sum = __fadd_rn(__fadd_rn(bank_total[0], bank_total[1]), __fadd_rn(bank_total[2], bank_total[3]));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(sum, 1.0f / 4096.0f), 1.0e-5f)));
    if (i == 0) a.recip[t] = inv;
    if (!a.gamma) return;
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
// linear_finalize's EPI_SWIGLU; emulator:716-722, 769-770).  Grid (stripes /
// 8, T), one warp per stripe.
__global__ void __launch_bounds__(256) k_pf_swiglu(const float* partials, int units, ExpfFix fx, int16_t* q,
                                                    uint8_t* e) {
    pdl_trigger();
    pdl_wait();
    const int stripe = blockIdx.x * 8 + (threadIdx.x >> 5), t = blockIdx.y, lane = threadIdx.x & 31;
    const int rows = units * 32, stripes = units / 2;
    const float* P = partials + static_cast<size_t>(t) * 4 * rows;
    const float g = combine4(P, rows, stripe * 32 + lane);
    const float u = combine4(P, rows, (stripes + stripe) * 32 + lane);
    uint32_t e8;
    const int v = quantize_g32_lane(swiglu1(g, u, fx), &e8);
    q[static_cast<size_t>(t) * kPfTok + stripe * 32 + lane] = static_cast<int16_t>(v);
    if (lane == 0) e[static_cast<size_t>(t) * (kPfTok / 32) + stripe] = static_cast<uint8_t>(e8);
}

// Perplexity terms of every token of a batch (emulator calculate_perplexity,
// :1902-1926), from the LM-head partials [T][4][32256]:
//   k_pf_logits  logits l_i = (p0+p1)+(p2+p3), i < 32000; max_l as the serial
//                scan `if (l[i] > max_l)` from l[0] finds it (the value of the
//                first maximum, NaN skipped; NaN when l[0] is NaN); the
//                target's logit.  One CTA per token.
//   k_pf_exp     expf(l_i - max_l) in place (glibc-equal expf).
//   k_pf_sum     the serial FP32 sum from +0.0f in index order.
// The host finishes each term as the emulator: (double)(max_l +
// logf(sum_exp)) and -(logit - that) in double.
struct PfNllArgs {
    const float* partials;  // [T][4][kPVocab]
    float* lg;              // [T][kVocab]: logits, then the expf terms
    const int* target;      // [T]
    float* terms;           // [T][4]: max_l, sum_exp, target logit, 0
    ExpfFix expf;
};

__global__ void __launch_bounds__(1024) k_pf_logits(const __grid_constant__ PfNllArgs a) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    const float* P = a.partials + static_cast<size_t>(t) * 4 * kPVocab;
    float* lg = a.lg + static_cast<size_t>(t) * kVocab;
    const int tgt = a.target[t];
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < kVocab; i += 1024) {
        const float v = combine4(P, kPVocab, i);
        lg[i] = v;
        const unsigned long long k = argmax_key(v, i);
        best = k > best ? k : best;
        if (i == tgt) a.terms[t * 4 + 2] = v;
    }
    __shared__ unsigned long long w[32];
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) w[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        const unsigned long long k = warp_max_u64(w[threadIdx.x]);
        if (threadIdx.x == 0) {
            const float l0 = lg[0];
            a.terms[t * 4] = (l0 != l0 || k == 0ull) ? l0 : lg[0xffffffffu - static_cast<uint32_t>(k & 0xffffffffu)];
            a.terms[t * 4 + 3] = 0.0f;
        }
    }
}

__global__ void __launch_bounds__(1024) k_pf_exp(const __grid_constant__ PfNllArgs a) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y, i = blockIdx.x * 1024 + threadIdx.x;
    if (i >= kVocab) return;
    float* lg = a.lg + static_cast<size_t>(t) * kVocab;
    lg[i] = expf_libc(__fsub_rn(lg[i], a.terms[t * 4]), a.expf);
}

__global__ void __launch_bounds__(32) k_pf_sum(const __grid_constant__ PfNllArgs a) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    if (threadIdx.x == 0) a.terms[t * 4 + 1] = sample_serial_sum(a.lg + static_cast<size_t>(t) * kVocab, kVocab);
}

// Prompt embeddings: resid[t] = emb[ids[t]] (ids checked on the host).
__global__ void __launch_bounds__(1024) k_pf_embed(const float* emb, const int* ids, float* resid) {
    const int t = blockIdx.x;
    const float4* src = reinterpret_cast<const float4*>(emb + static_cast<size_t>(ids[t]) * kDim);
    reinterpret_cast<float4*>(resid + static_cast<size_t>(t) * kDim)[threadIdx.x] = src[threadIdx.x];
}

}  // namespace i4d
