// i4d_linear.cuh -- fused dequant-GEMV stage kernel and the weight re-tiling.
//
// Replaces int4_linear_controller's reader / scale emitter / accumulator /
// pair reducers (int4_linear_controller.cpp:253-951, 1339-1439).
//
// GEMV layout in HBM (written once at load by k_relayout from the unchanged
// bank image): a "unit" is 32 output rows x one bank's local columns; it is
// stored as chunks of 32 rows x 256 columns, 4224 bytes each:
//   [  0,128): Q1.15 scales, int16 at (row*2 + g128)*2
//   [128,4224): 256 pieces of 16 bytes, one per (row, group), placed by
//               chunk_piece (row-block major, group XOR-swizzled); a piece
//               holds the 32 INT4 weights of its row and group: uint32 word
//               j, byte b holds column 4j+b in the low nibble as offset
//               binary (w+8) and column 16+4j+b in the high nibble as two's
//               complement.
// The units of one stage and bank are contiguous, so every CTA streams one
// contiguous range with 1-D bulk copies.
//
// Arithmetic (bit-exact with emulator:216-264): per row and bank the G32
// dot products are exact integers (dp4a on split activations a = 128*ah + al),
// contrib = fl(float(dot) * fl(ws * as)), and the FP32 chain adds the
// contributions in local-group order.  Rows are then combined as
// (p0+p1)+(p2+p3) by whichever CTA completes a stripe last.
#pragma once

#include "i4d_device.cuh"
#include "i4d_expf.cuh"

namespace i4d {

enum InKind : int { IN_ACT = 0, IN_RMS = 1 };
enum EpiKind : int { EPI_PARTIAL = 0, EPI_STORE = 1, EPI_RESID = 2, EPI_SWIGLU = 3 };

struct LinearArgs {
    const uint8_t* w;      // unit 0 of bank 0 of this launch (GEMV layout)
    size_t bank_stride;    // bytes from one bank's unit 0 to the next bank's
    int nbanks;            // 1..4
    int cpb;               // CTAs per bank; gridDim.x == nbanks * cpb
    int units;             // units per bank
    int chunks;            // chunks per unit: local columns / 256
    int ns;                // ring slots
    int nu;                // contribution slots (units in flight per CTA)
    // input activation of this bank: IN_ACT reads act_q/act_e at
    // bank*act_bank_stride; IN_RMS normalises resid with gamma and *recip.
    int in_kind;
    const int16_t* act_q;
    const uint8_t* act_e;
    int act_bank_stride;
    const float* resid;
    const float* gamma;
    const float* recip;
    int hls_zero;          // 1: chains start at the first contribution
    float* partials;       // [bank][units*32]
    int epi;
    float* out;            // EPI_STORE: y; EPI_RESID: residual (updated in place)
    float* recip_out;      // EPI_RESID: RMS reciprocal of the updated residual
    int16_t* q_out;        // EPI_SWIGLU
    uint8_t* e_out;
    unsigned* counters;
    ExpfFix expf;
    unsigned* err;
};

constexpr int kFinMax = 64;   // stripes one CTA may finalise (<= units per CTA)

struct LinearSmem {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    int8_t* act_hi;     // [groups][32]
    uint8_t* act_lo;    // [groups][32]
    int* corr;          // [groups]: 8 * sum of the group's first 16 values
    float* act_scale;   // [groups]
    float* contrib;     // [nu][groups*32]
    int* unit_cnt;      // [nu]: chunks of the unit done
    int* slot_ok;       // [nu]: first unit index allowed to use the slot
    int* fin;           // [kFinMax + 2]: count, level-2 flag, stripe list
    int* issued;        // [ns]: chunk index last issued into each ring slot
};

__host__ __device__ constexpr size_t align16(size_t b) { return (b + 15) & ~static_cast<size_t>(15); }

__host__ __device__ inline size_t linear_smem_bytes(int ns, int chunks, int nu) {
    const size_t groups = static_cast<size_t>(chunks) * 8;
    size_t b = static_cast<size_t>(ns) * kChunkBytes;
    b += align16(2 * static_cast<size_t>(ns) * 8);
    b += align16(groups * 64) + align16(groups * 8);
    b += static_cast<size_t>(nu) * groups * 32 * 4;
    b += align16(2 * static_cast<size_t>(nu) * 4) + align16((kFinMax + 2) * 4);
    b += align16(static_cast<size_t>(ns) * 4);
    return b;
}

__device__ __forceinline__ LinearSmem carve(uint8_t* base, int ns, int chunks, int nu) {
    LinearSmem s;
    const size_t groups = static_cast<size_t>(chunks) * 8;
    uint8_t* p = base;
    s.ring = p;
    p += static_cast<size_t>(ns) * kChunkBytes;
    s.full = reinterpret_cast<uint64_t*>(p);
    s.empty = s.full + ns;
    p += align16(2 * static_cast<size_t>(ns) * 8);
    s.act_hi = reinterpret_cast<int8_t*>(p);
    s.act_lo = reinterpret_cast<uint8_t*>(p + groups * 32);
    p += align16(groups * 64);
    s.corr = reinterpret_cast<int*>(p);
    s.act_scale = reinterpret_cast<float*>(p + groups * 4);
    p += align16(groups * 8);
    s.contrib = reinterpret_cast<float*>(p);
    p += static_cast<size_t>(nu) * groups * 32 * 4;
    s.unit_cnt = reinterpret_cast<int*>(p);
    s.slot_ok = s.unit_cnt + nu;
    p += align16(2 * static_cast<size_t>(nu) * 4);
    s.fin = reinterpret_cast<int*>(p);
    p += align16((kFinMax + 2) * 4);
    s.issued = reinterpret_cast<int*>(p);
    return s;
}

// Stores one lane's INT14 activation (value q of local group lg, column
// `lane`) in split form, plus the group's scale and offset correction.
__device__ __forceinline__ void put_act(const LinearSmem& s, int lg, int lane, int q, uint32_t e8m0) {
    s.act_hi[lg * 32 + lane] = static_cast<int8_t>(q >> 7);
    s.act_lo[lg * 32 + lane] = static_cast<uint8_t>(q & 127);
    int lo16 = lane < 16 ? q : 0;
    lo16 = __reduce_add_sync(0xffffffffu, lo16);
    if (lane == 0) {
        s.corr[lg] = 8 * lo16;
        s.act_scale[lg] = e8m0_scale(e8m0);
    }
}

// Byte offset inside a chunk of the 16 weight bytes of (row, group).  Row
// r = 8*rb + k is stored k-major and the group index is XOR-swizzled by k,
// so that a warp reading one group of 32 rows (lane = row) and a warp
// reading 8 groups x 4 row blocks (lane = group + 8*rb, one k per load) both
// touch every shared-memory bank once per 8-lane phase.
__host__ __device__ constexpr int chunk_piece(int row, int g) {
    return kChunkScaleBytes + (((row & 7) * 4 + (row >> 3)) * 8 + (g ^ (row & 7))) * 16;
}

// Exact G32 dot of one (row, group): weights w (16 bytes), split activations
// held in registers (h0/l0: columns 0..15, h1/l1: columns 16..31).
__device__ __forceinline__ int group_dot_r(uint4 w, uint4 h0, uint4 h1, uint4 l0, uint4 l1, int corr) {
    int Lh = 0, Ll = 0, Hh = 0, Hl = 0;
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    const uint32_t h0v[4] = {h0.x, h0.y, h0.z, h0.w};
    const uint32_t h1v[4] = {h1.x, h1.y, h1.z, h1.w};
    const uint32_t l0v[4] = {l0.x, l0.y, l0.z, l0.w};
    const uint32_t l1v[4] = {l1.x, l1.y, l1.z, l1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t u = wv[j] & 0x0F0F0F0Fu;  // (w + 8) of columns 4j..4j+3
        const uint32_t h = wv[j] & 0xF0F0F0F0u;  // 16 * w of columns 16+4j..
        Lh = dp4a_us(u, h0v[j], Lh);
        Ll = dp4a_uu(u, l0v[j], Ll);
        Hh = dp4a_ss(h, h1v[j], Hh);
        Hl = dp4a_su(h, l1v[j], Hl);
    }
    return ((Lh + (Hh >> 4)) << 7) + Ll + (Hl >> 4) - corr;
}

// The same with the activations read from shared memory.
__device__ __forceinline__ int group_dot(uint4 w, const int8_t* hi, const uint8_t* lo, int corr) {
    return group_dot_r(w, *reinterpret_cast<const uint4*>(hi), *reinterpret_cast<const uint4*>(hi + 16),
                       *reinterpret_cast<const uint4*>(lo), *reinterpret_cast<const uint4*>(lo + 16), corr);
}

// Builds this bank's split activations in shared memory (consumer warps).
__device__ __forceinline__ void linear_prologue(const LinearArgs& a, const LinearSmem& s, int bank, int cw,
                                                int lane, int groups) {
    constexpr int kMaxPer = (kMaxLocalGroups + kConsumerWarps - 1) / kConsumerWarps;  // 11
    float v[kMaxPer];
    int qv[kMaxPer];
    uint32_t ev[kMaxPer];
    if (a.in_kind == IN_RMS) {
        const float r = *a.recip;
        float x[kMaxPer], g[kMaxPer];
#pragma unroll
        for (int k = 0; k < kMaxPer; ++k) {
            const int lg = cw + k * kConsumerWarps;
            if (lg < groups) {
                const int col = bank * groups * 32 + lg * 32 + lane;
                x[k] = a.resid[col];
                g[k] = a.gamma[col];
            }
        }
#pragma unroll
        for (int k = 0; k < kMaxPer; ++k) v[k] = __fmul_rn(__fmul_rn(x[k], r), g[k]);
#pragma unroll
        for (int k = 0; k < kMaxPer; ++k) {
            const int lg = cw + k * kConsumerWarps;
            if (lg < groups) qv[k] = quantize_g32_lane(v[k], &ev[k]);
        }
    } else {
        const size_t base = static_cast<size_t>(bank) * a.act_bank_stride;
#pragma unroll
        for (int k = 0; k < kMaxPer; ++k) {
            const int lg = cw + k * kConsumerWarps;
            if (lg < groups) {
                qv[k] = a.act_q[base + lg * 32 + lane];
                ev[k] = a.act_e[base / 32 + lg];
            }
        }
    }
#pragma unroll
    for (int k = 0; k < kMaxPer; ++k) {
        const int lg = cw + k * kConsumerWarps;
        if (lg < groups) put_act(s, lg, lane, qv[k], ev[k]);
    }
}

// Finalises one stripe once all its bank partials are in (one warp).
__device__ __noinline__ void linear_finalize(const LinearArgs& a, int stripe, int* level2_last) {
    const int lane = threadIdx.x & 31;
    const int rows_total = a.units * 32;
    const float* P = a.partials;
    if (a.epi == EPI_STORE) {
        const int row = stripe * 32 + lane;
        a.out[row] = a.nbanks == 4 ? combine4(P, rows_total, row) : __ldcg(P + row);
        return;
    }
    if (a.epi == EPI_SWIGLU) {
        const int stripes = a.units / 2;
        const int gr = stripe * 32 + lane, ur = (stripes + stripe) * 32 + lane;
        const float g = combine4(P, rows_total, gr);
        const float u = combine4(P, rows_total, ur);
        uint32_t e8;
        const int q = quantize_g32_lane(swiglu1(g, u, a.expf), &e8);
        a.q_out[stripe * 32 + lane] = static_cast<int16_t>(q);
        if (lane == 0) a.e_out[stripe] = static_cast<uint8_t>(e8);
        return;
    }
    // EPI_RESID: residual += y; the last stripe overall triggers the RMS.
    const int row = stripe * 32 + lane;
    a.out[row] = __fadd_rn(__ldcg(a.out + row), combine4(P, rows_total, row));
    __threadfence();
    __syncwarp();
    unsigned old = 0;
    if (lane == 0) old = atomicAdd(&a.counters[kCounterLevel2], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + 1 == static_cast<unsigned>(a.units)) {
        if (lane == 0) {
            a.counters[kCounterLevel2] = 0;
            *level2_last = 1;
        }
    }
}

__global__ void __launch_bounds__(kLinearThreads, 2) k_linear(const __grid_constant__ LinearArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int groups = a.chunks * 8;
    LinearSmem s = carve(smem_raw, a.ns, a.chunks, a.nu);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bank = blockIdx.x / a.cpb, c = blockIdx.x % a.cpb;
    const int u0 = static_cast<int>((static_cast<long long>(c) * a.units) / a.cpb);
    const int u1 = static_cast<int>((static_cast<long long>(c + 1) * a.units) / a.cpb);
    const int nchunks = (u1 - u0) * a.chunks;

    if (threadIdx.x == 0) {
        for (int i = 0; i < a.ns; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < a.nu) {
        s.unit_cnt[threadIdx.x] = 0;
        s.slot_ok[threadIdx.x] = threadIdx.x;
    }
    if (threadIdx.x < 2) s.fin[threadIdx.x] = 0;
    for (int i = threadIdx.x; i < a.ns; i += blockDim.x) s.issued[i] = -1;
    __syncthreads();
    pdl_trigger();

    if (warp == 0) {
        // Producer: weights never depend on the previous kernel, so streaming
        // starts before griddepcontrol.wait.
        if (lane == 0) {
            const uint8_t* src = a.w + static_cast<size_t>(bank) * a.bank_stride +
                                 static_cast<size_t>(u0) * a.chunks * kChunkBytes;
            int slot = 0;
            uint32_t phase = 0;
            for (int i = 0; i < nchunks; ++i) {
                if (i >= a.ns) mbar_wait(&s.empty[slot], phase ^ 1u, a.err, kErrWaitEmpty);
                publish_issued(&s.issued[slot], i);
                mbar_arrive_expect_tx(&s.full[slot], kChunkBytes);
                bulk_g2s(s.ring + static_cast<size_t>(slot) * kChunkBytes,
                         src + static_cast<size_t>(i) * kChunkBytes, kChunkBytes, &s.full[slot]);
                if (++slot == a.ns) { slot = 0; phase ^= 1u; }
            }
        }
        return;
    }

    // Consumers: warp cw takes chunks cw, cw+8, ... whole (8 groups x 32 rows).
    const int cw = warp - 1;
    pdl_wait();
    linear_prologue(a, s, bank, cw, lane, groups);
    consumer_bar();

    const int rows_total = a.units * 32;
    for (int i = cw; i < nchunks; i += kConsumerWarps) {
        const int slot = i % a.ns;
        wait_issued(&s.issued[slot], i, a.err);
        mbar_wait(&s.full[slot], static_cast<uint32_t>((i / a.ns) & 1), a.err, kErrWaitFull);
        const uint8_t* ch = s.ring + static_cast<size_t>(slot) * kChunkBytes;
        uint4 wv[8];
#pragma unroll
        for (int g = 0; g < 8; ++g)
            wv[g] = *reinterpret_cast<const uint4*>(ch + chunk_piece(lane, g));
        const int16_t raw0 = reinterpret_cast<const int16_t*>(ch)[lane * 2];
        const int16_t raw1 = reinterpret_cast<const int16_t*>(ch)[lane * 2 + 1];
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[slot]);

        const int uidx = i / a.chunks, j = i - uidx * a.chunks;
        const int us = uidx % a.nu;
        // Contribution slot `us` is free once unit uidx - nu has been chained.
        if (*reinterpret_cast<volatile int*>(&s.slot_ok[us]) < uidx) {
            uint32_t spins = 0;
            while (*reinterpret_cast<volatile int*>(&s.slot_ok[us]) < uidx) {
                __nanosleep(64);
                if (++spins > (1u << 24)) { atomicOr(a.err, kErrWaitFull); break; }
            }
        }
        float* cb = s.contrib + static_cast<size_t>(us) * groups * 32;
        const float ws0 = __fmul_rn(static_cast<float>(raw0), 1.0f / 32768.0f);
        const float ws1 = __fmul_rn(static_cast<float>(raw1), 1.0f / 32768.0f);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const int lg = j * 8 + g;
            const int dot = group_dot(wv[g], s.act_hi + lg * 32, s.act_lo + lg * 32, s.corr[lg]);
            cb[lg * 32 + lane] = __fmul_rn(static_cast<float>(dot), __fmul_rn(g < 4 ? ws0 : ws1, s.act_scale[lg]));
        }
        __syncwarp();
        __threadfence_block();
        int old = 0;
        if (lane == 0) old = atomicAdd(&s.unit_cnt[us], 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == a.chunks - 1) {
            // Last chunk of the unit: FP32 chain in local-group order.
            __threadfence_block();
            float acc = cb[lane];
            if (!a.hls_zero) acc = __fadd_rn(0.0f, acc);
            for (int lg = 1; lg < groups; ++lg) acc = __fadd_rn(acc, cb[lg * 32 + lane]);
            a.partials[static_cast<size_t>(bank) * rows_total + static_cast<size_t>(u0 + uidx) * 32 + lane] = acc;
            __syncwarp();
            __threadfence_block();
            if (lane == 0) {
                s.unit_cnt[us] = 0;
                *reinterpret_cast<volatile int*>(&s.slot_ok[us]) = uidx + a.nu;
            }
        }
    }
    if (a.epi == EPI_PARTIAL) return;

    // End of this CTA's stage: one counter add per stripe it touched; the CTA
    // that completes a stripe (all banks) finalises it.
    __threadfence();
    consumer_bar();
    const int stripes = a.epi == EPI_SWIGLU ? a.units / 2 : a.units;
    const unsigned need = static_cast<unsigned>(a.epi == EPI_SWIGLU ? 2 * a.nbanks : a.nbanks);
    if (cw == 0) {
        for (int b = u0; b < u1; b += 32) {
            const int u = b + lane;
            if (u < u1) {
                const int stripe = u % stripes;
                const unsigned old = atomicAdd(&a.counters[stripe], 1u);
                if (old + 1 == need) {
                    a.counters[stripe] = 0;
                    const int k = atomicAdd(&s.fin[0], 1);
                    if (k < kFinMax) s.fin[2 + k] = stripe;
                    else atomicOr(a.err, kErrArg);
                }
            }
        }
        __threadfence();
    }
    consumer_bar();
    const int nfin = min(s.fin[0], kFinMax);
    for (int k = cw; k < nfin; k += kConsumerWarps) linear_finalize(a, s.fin[2 + k], &s.fin[1]);
    if (a.epi != EPI_RESID) return;
    consumer_bar();
    if (s.fin[1] == 0) return;
    // Last stripe of the whole residual: RMS reciprocal for the next norm.
    __threadfence();
    float* xs = reinterpret_cast<float*>(s.ring);
    const int t = threadIdx.x - 32;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        reinterpret_cast<float4*>(xs)[t + k * 256] =
            __ldcg(reinterpret_cast<const float4*>(a.out) + t + k * 256);
    consumer_bar();
    if (cw == 0) {
        const float r = rms_recip_warp(xs);
        if (lane == 0) *a.recip_out = r;
    }
}

// ------------------------------------------------------------- re-tiling

struct RelayoutArgs {
    const uint8_t* src;    // the bank's superblock stream of one matrix
    uint8_t* dst;          // this bank's unit 0 of the stage in the GEMV layout
    int unit_offset;       // first unit of this matrix inside the stage
    int lit;               // local input tiles (chunks per unit)
};

// One block per (stripe, chunk); thread = (group g, row).  Reads the
// reference tile words (autoround_pack_llama2_u250.py:114-189,
// emulator:840-888) and writes the GEMV layout above.
__global__ void __launch_bounds__(256) k_relayout(const RelayoutArgs a) {
    const int stripe = blockIdx.x / a.lit, j = blockIdx.x % a.lit;
    const int g = threadIdx.x >> 5, row = threadIdx.x & 31;
    const int ot = stripe >> 2, sub = stripe & 3;
    const int t = ot * a.lit + j;
    const uint8_t* blk = a.src + static_cast<size_t>(t / 16) * 4224 * 64;
    const int tib = t % 16;
    const int trow = sub * 32 + row;
    uint8_t* chunk = a.dst + (static_cast<size_t>(a.unit_offset + stripe) * a.lit + j) * kChunkBytes;
    if (threadIdx.x < 64) {
        const int r = threadIdx.x >> 1, g128 = threadIdx.x & 1;
        const int tr = sub * 32 + r;
        const int16_t v = *reinterpret_cast<const int16_t*>(blk + (tib * 8 + tr / 16) * 64 + (2 * (tr % 16) + g128) * 2);
        reinterpret_cast<int16_t*>(chunk)[r * 2 + g128] = v;
    }
    const uint8_t* word = blk + 128 * 64 + (static_cast<size_t>(tib) * 256 + g * 32 + trow / 4) * 64;
    const int r4 = trow & 3;
    int wv[32];
#pragma unroll
    for (int l = 0; l < 32; ++l) {
        const uint8_t byte = word[2 * l + (r4 >> 1)];
        const int nib = (r4 & 1) ? (byte & 15) : (byte >> 4);
        wv[l] = nib >= 8 ? nib - 16 : nib;
    }
    uint32_t out[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        uint32_t v = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t lo = static_cast<uint32_t>(wv[4 * jj + b] + 8) & 15u;
            const uint32_t hi = static_cast<uint32_t>(wv[16 + 4 * jj + b]) & 15u;
            v |= (lo | (hi << 4)) << (8 * b);
        }
        out[jj] = v;
    }
    *reinterpret_cast<uint4*>(chunk + chunk_piece(row, g)) = make_uint4(out[0], out[1], out[2], out[3]);
}

}  // namespace i4d
