// i4d_attn_item.cuh -- one (head, 32-dimension part) item of the SwiftKV
// attention step (swiftkv_attention_4pe, emulator:602-714; the HLS scan of
// swiftkv_attention.cpp:1882-2032), shared by the persistent token kernel and
// the standalone attention kernel.  18 warps (576 threads) work on an item.
//
// The current token: q/k/v of the head (from the QKV bank partials or given
// directly), Q15.17, adjacent-pair RoPE, the KV shift quantiser and the
// 320-byte record (part 0 writes it to the cache).  Then the cache is
// scanned in tiles of kTile records, double-buffered by bulk copies:
//  * scores: exact integer dot products (16 warps x 4 tokens, 8 lanes each);
//  * one warp: running maximum before each token (a prefix maximum carried
//    across tiles), the softmax coefficients c_t, the tokens where the
//    maximum grows ("events"), the tile's sum of c_t over the other tokens
//    and a bound on the magnitudes of their state terms;
//  * state terms mulq17(v_t, c_t) per (token, dimension) in 32-bit form, and
//    per dimension the tile's sum over the non-event tokens.
// Warp 0 (lane = dimension) then applies the tile, one tile behind the
// workers: a tile with no event whose bound shows that no step of the
// saturating chain can saturate adds its sum in one step (integer addition
// is associative; the normaliser adds modulo 2^30); any other tile runs the
// reference's token-order recurrence over the tile's precomputed terms.
// Either way the state is bit-exact with the sequential scan.
#pragma once

#include "i4d_attention.cuh"

namespace i4d {

constexpr int kItemWarps = 18;
constexpr int kItemThreads = 32 * kItemWarps;
constexpr int kAttnParts = 4;              // 32-dimension parts per head
constexpr int kAttnItems = kHeads * kAttnParts;

struct TileInfo {
    unsigned long long ev;     // nonzero: the tile holds an event (or token 0)
    unsigned long long zsum;   // sum of c_t over the tile's non-event tokens
    unsigned long long bound;  // sum of the bounds on |term| over the same tokens
    unsigned long long pad;
};

struct AttnItemSmem {
    uint8_t* tile[2];     // kTile records each
    uint8_t* cur;         // current token's record
    int32_t* score;       // [kTile]
    uint32_t* coef;       // [2][kTile]: c | event << 31, by tile parity
    int32_t* tbuf;        // [2][kTile][32]: state terms of this part (v_t itself at events)
    int32_t* psum;        // [2][32]: per dimension, the tile's sum of the non-event terms
    TileInfo* tinfo;      // [2]
    uint32_t* lut;        // [33] exp2 table
    int32_t* qrot;        // [128]
    unsigned long long* meta;  // current record's shift word
    int* misc;            // [16]
};

constexpr size_t kAttnItemBytes = 2 * kTile * 320 + 320 + kTile * 4 + 2 * kTile * 4 + 2 * kTile * 32 * 4 + 2 * 32 * 4 +
                                  2 * sizeof(TileInfo) + 144 + 128 * 4 + 16 + 16 * 4;

__device__ __forceinline__ AttnItemSmem attn_item_carve(uint8_t* p) {
    AttnItemSmem s;
    s.tile[0] = p;
    s.tile[1] = p + kTile * 320;
    p += 2 * kTile * 320;
    s.cur = p;
    p += 320;
    s.score = reinterpret_cast<int32_t*>(p);
    p += kTile * 4;
    s.coef = reinterpret_cast<uint32_t*>(p);
    p += 2 * kTile * 4;
    s.tbuf = reinterpret_cast<int32_t*>(p);
    p += 2 * kTile * 32 * 4;
    s.psum = reinterpret_cast<int32_t*>(p);
    p += 2 * 32 * 4;
    s.tinfo = reinterpret_cast<TileInfo*>(p);
    p += 2 * sizeof(TileInfo);
    s.lut = reinterpret_cast<uint32_t*>(p);
    p += 144;
    s.qrot = reinterpret_cast<int32_t*>(p);
    p += 128 * 4;
    s.meta = reinterpret_cast<unsigned long long*>(p);
    p += 16;
    s.misc = reinterpret_cast<int*>(p);
    return s;
}

// Barriers of the item: all 18 warps, and the 16 worker warps (2..17).
__device__ __forceinline__ void item_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kItemThreads) : "memory"); }
__device__ __forceinline__ void item_wbar() { asm volatile("bar.sync 2, %0;" ::"n"(kItemThreads - 64) : "memory"); }

// mulq17(v8 << shift, c) for a cached value v8 (|v8| <= 127) and a softmax
// coefficient c <= 2^17 (emulator:597-600 on the value of emulator:677).
// For shift <= 24, p = v8 * c fits in 25 bits and v8 << shift in 32, so the
// product's round-half-even shift by 17 is p << (shift - 17) or
// rhe(p, 17 - shift) in 32-bit arithmetic (checked equal on every v8,
// shift <= 24 and c <= 2^17).  Larger shifts (only from saturated values)
// take the 64-bit form on the wrapped value, as the reference computes it.
__device__ __forceinline__ int32_t term_q17(int v8, uint32_t shift, uint32_t c) {
    if (shift > 24) return mulq17(static_cast<int32_t>(static_cast<uint32_t>(v8) << shift), c);
    const int32_t p = v8 * static_cast<int32_t>(c);
    if (shift >= 17) return static_cast<int32_t>(static_cast<uint32_t>(p) << (shift - 17));
    const uint32_t s = 17 - shift;
    return (p + ((1 << (s - 1)) - 1) + ((p >> s) & 1)) >> s;
}

// Upper bound on |term_q17(v8, shift, c)| over every |v8| <= 127.
__device__ __forceinline__ unsigned long long term_bound(uint32_t shift, uint32_t c) {
    if (shift > 24) return 1ull << 40;
    return ((static_cast<unsigned long long>(127u * c) << shift) >> 17) + 1ull;
}

// Bounded mbarrier wait of an item; `fail(code)` records a timeout, and a
// nonzero *abort_word (may be null) ends the wait early.
template <class Fail>
__device__ __forceinline__ bool item_mbar_wait(uint64_t* bar, uint32_t parity, const unsigned* abort_word,
                                               Fail fail) {
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15) == 0 && abort_word && *reinterpret_cast<const volatile unsigned*>(abort_word)) return false;
        if (it > (1u << 22)) {
            fail(kErrWaitFull | kErrWaitTile);
            return false;
        }
        if (it >= 256) __nanosleep(64);
    }
}

// One attention item: head h, dimensions [32 part, 32 part + 32), thread
// `tid` of 576.  `wait_input()` runs on thread 0 after the first tile's
// copy is issued (the token kernel waits there for the QKV stage).  Warp 0
// ends with the item's 32 outputs stored (a.out_q, a.out_e); the caller
// publishes them.
template <class WaitInput, class Fail>
__device__ __forceinline__ void attn_item(const AttnArgs& a, const AttnItemSmem& S, uint64_t* abar, int h, int part,
                                          int tid, const unsigned* abort_word, WaitInput wait_input, Fail fail) {
    const unsigned FULL = 0xffffffffu;
    const uint32_t M30 = (1u << 30) - 1u;
    const int warp = tid >> 5, lane = tid & 31;
    int* misc = S.misc;
    const int pos = *a.pos_ptr;
    const int n = pos + 1;
    const int ntiles = (n + kTile - 1) / kTile;
    const uint8_t* head_base = kv_record(a, h, 0);
    if (tid == 0) {
        mbar_init(&abar[0], 1);
        mbar_init(&abar[1], 1);
        mbar_fence_init();
        misc[0] = INT32_MIN;  // running maximum of the tiles scanned so far
        *S.meta = 0ull;
    }
    if (tid < 33) S.lut[tid] = a.exp2_q30[tid];
    if (tid < 16) reinterpret_cast<uint32_t*>(S.cur)[tid] = 0u;  // record word 0
    // RoPE factors of this position: independent of the projections.
    long long rope_c = 0, rope_s = 0;
    if (tid < 128) {
        rope_c = a.rope_cos[pos * 64 + (tid >> 1)];
        rope_s = a.rope_sin[pos * 64 + (tid >> 1)];
    }
    item_bar();
    if (tid == 0) {
        // Cached records of earlier tokens are final: stream the first tile
        // while the projections are still being produced.
        const int cnt = min(kTile, n);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&abar[0], cnt * 320);
        bulk_g2s(S.tile[0], head_base, cnt * 320, &abar[0]);
        wait_input();
    }
    item_bar();

    // ---- current token: thread = dimension d of the head (warps 0-3) ----
    uint8_t* grec = kv_record(a, h, pos);
    if (tid < 128) {
        const int d = tid, row = h * kHeadDim + d;
        int32_t qv, kv, vv;
        if (a.direct) {
            qv = a.direct[row];
            kv = a.direct[kDim + row];
            vv = a.direct[2 * kDim + row];
        } else {
            qv = float_to_q17(combine4(a.partials, 3 * kDim, row));
            kv = float_to_q17(combine4(a.partials, 3 * kDim, kDim + row));
            vv = float_to_q17(combine4(a.partials, 3 * kDim, 2 * kDim + row));
        }
        // Adjacent-pair RoPE (emulator:526-541): pair (2i, 2i+1) is the lane pair (d, d^1).
        const int32_t qo = __shfl_xor_sync(FULL, qv, 1), ko = __shfl_xor_sync(FULL, kv, 1);
        const long long qa = (d & 1) ? qo : qv, qb = (d & 1) ? qv : qo;
        const long long ka = (d & 1) ? ko : kv, kb = (d & 1) ? kv : ko;
        const int32_t qr = (d & 1) ? sat32((qa * rope_s + qb * rope_c) >> 17) : sat32((qa * rope_c - qb * rope_s) >> 17);
        const int32_t kr = (d & 1) ? sat32((ka * rope_s + kb * rope_c) >> 17) : sat32((ka * rope_c - kb * rope_s) >> 17);
        S.qrot[d] = qr;
        // KV shift quantiser per 32-value group (warp), emulator:543-564.
        const uint32_t kmag = static_cast<uint32_t>(kr < 0 ? -static_cast<long long>(kr) : kr);
        const uint32_t vmag = static_cast<uint32_t>(vv < 0 ? -static_cast<long long>(vv) : vv);
        const uint32_t ks = kv_shift_of(__reduce_max_sync(FULL, kmag));
        const uint32_t vs = kv_shift_of(__reduce_max_sync(FULL, vmag));
        const uint8_t k8 = static_cast<uint8_t>(kv_quant(kr, ks)), v8 = static_cast<uint8_t>(kv_quant(vv, vs));
        S.cur[64 + d] = k8;
        S.cur[192 + d] = v8;
        if (part == 0) {
            grec[64 + d] = k8;
            grec[192 + d] = v8;
        }
        if (lane == 0)
            atomicOr(S.meta, (static_cast<unsigned long long>(ks) << (5 * warp)) |
                                 (static_cast<unsigned long long>(vs) << (20 + 5 * warp)));
    }
    item_bar();
    if (tid < 8) {
        const unsigned long long m = tid == 0 ? *S.meta : 0ull;
        reinterpret_cast<unsigned long long*>(S.cur)[tid] = m;
        if (part == 0) reinterpret_cast<unsigned long long*>(grec)[tid] = m;
    }
    // q of this lane's 16-value half-group, split into 16-bit halves for dp2a.
    const int hg = lane & 7;
    uint32_t qh2[8], ql2[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int32_t x0 = S.qrot[hg * 16 + 2 * i], x1 = S.qrot[hg * 16 + 2 * i + 1];
        qh2[i] = (static_cast<uint32_t>(x0 >> 16) & 0xffffu) | (static_cast<uint32_t>(x1 >> 16) << 16);
        ql2[i] = (static_cast<uint32_t>(x0) & 0xffffu) | (static_cast<uint32_t>(x1) << 16);
    }
    item_bar();

    const int dl = lane;                     // dimension inside this part
    const int dim = part * 32 + dl;
    const uint32_t vbit = 20 + 5 * part;     // this part's V shift field in a record's word 0
    int32_t st = 0;                          // warp 0: the state of dimension `dim`
    uint32_t z = 1u << 17;                   // warp 0: the normaliser (every lane)
    const int wtid = tid - 64, wcw = warp - 2;
    for (int k = 0; k <= ntiles; ++k) {
        if (warp >= 2) {
            if (k < ntiles) {
                const int T0 = k * kTile, cnt = min(kTile, n - T0), p = k & 1;
                uint8_t* buf = S.tile[p];
                uint32_t* coef = S.coef + p * kTile;
                int32_t* tbuf = S.tbuf + p * kTile * 32;
                int32_t* psum = S.psum + p * 32;
                if (wtid == 0 && k + 1 < ntiles) {  // buffer p ^ 1 was last read in iteration k - 1
                    fence_proxy_async_smem();
                    const int c2 = min(kTile, n - T0 - kTile);
                    mbar_arrive_expect_tx(&abar[p ^ 1], c2 * 320);
                    bulk_g2s(S.tile[p ^ 1], head_base + static_cast<size_t>(T0 + kTile) * 320, c2 * 320,
                             &abar[p ^ 1]);
                }
                if (wtid < 32) psum[wtid] = 0;
                item_mbar_wait(&abar[p], static_cast<uint32_t>((k >> 1) & 1), abort_word, fail);
                if (pos < T0 + cnt) {  // the tile holds the current token: use the fresh record
                    if (wtid < 80)
                        reinterpret_cast<uint32_t*>(buf + (pos - T0) * 320)[wtid] =
                            reinterpret_cast<const uint32_t*>(S.cur)[wtid];
                    item_wbar();
                }
                {   // scores (emulator:633-655): 16 warps x 4 tokens, 8 lanes per token
                    const int tl = wcw * 4 + (lane >> 3);
                    long long hv = 0;
                    if (tl < cnt) {
                        const uint8_t* rec = buf + tl * 320;
                        const uint4 kw = *reinterpret_cast<const uint4*>(rec + 64 + hg * 16);
                        const unsigned long long meta = *reinterpret_cast<const unsigned long long*>(rec);
                        const uint32_t sh = static_cast<uint32_t>((meta >> (5 * (hg >> 1))) & 31u);
                        int sh16 = 0, sl16 = 0;
                        sh16 = dp2a_lo_ss(qh2[0], kw.x, sh16);
                        sh16 = dp2a_hi_ss(qh2[1], kw.x, sh16);
                        sh16 = dp2a_lo_ss(qh2[2], kw.y, sh16);
                        sh16 = dp2a_hi_ss(qh2[3], kw.y, sh16);
                        sh16 = dp2a_lo_ss(qh2[4], kw.z, sh16);
                        sh16 = dp2a_hi_ss(qh2[5], kw.z, sh16);
                        sh16 = dp2a_lo_ss(qh2[6], kw.w, sh16);
                        sh16 = dp2a_hi_ss(qh2[7], kw.w, sh16);
                        sl16 = dp2a_lo_us(ql2[0], kw.x, sl16);
                        sl16 = dp2a_hi_us(ql2[1], kw.x, sl16);
                        sl16 = dp2a_lo_us(ql2[2], kw.y, sl16);
                        sl16 = dp2a_hi_us(ql2[3], kw.y, sl16);
                        sl16 = dp2a_lo_us(ql2[4], kw.z, sl16);
                        sl16 = dp2a_hi_us(ql2[5], kw.z, sl16);
                        sl16 = dp2a_lo_us(ql2[6], kw.w, sl16);
                        sl16 = dp2a_hi_us(ql2[7], kw.w, sl16);
                        const long long half = static_cast<long long>(sh16) * 65536 + sl16;
                        hv = wrap_bits(sh >= 10 ? static_cast<long long>(static_cast<unsigned long long>(half) << (sh - 10))
                                                : (half >> (10 - sh)), 44);
                    }
                    hv += __shfl_xor_sync(FULL, hv, 1);
                    hv += __shfl_xor_sync(FULL, hv, 2);
                    hv += __shfl_xor_sync(FULL, hv, 4);
                    if ((lane & 7) == 0 && tl < cnt) S.score[tl] = sat32(rshift_even(wrap_bits(hv, 44) * a.score_scale, 24));
                }
                item_wbar();
                if (wcw == 0) {
                    // Coefficients from the running maximum before each token
                    // (emulator:656-672): lane l takes tokens 2l and 2l + 1.
                    const int32_t carry = misc[0];
                    const int t0 = 2 * lane;
                    const int32_t s0 = t0 < cnt ? S.score[t0] : INT32_MIN;
                    const int32_t s1 = t0 + 1 < cnt ? S.score[t0 + 1] : INT32_MIN;
                    int32_t mx = max(s0, s1);
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int32_t y = __shfl_up_sync(FULL, mx, o);
                        if (lane >= o) mx = max(mx, y);
                    }
                    int32_t ex = __shfl_up_sync(FULL, mx, 1);
                    if (lane == 0) ex = INT32_MIN;
                    const int32_t prev0 = max(carry, ex);
                    const int32_t prev1 = max(prev0, s0);
                    bool any_ev = false;
                    uint32_t zs = 0;
                    unsigned long long bs = 0;
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int tl = t0 + j;
                        if (tl < cnt) {
                            const int32_t sc = j ? s1 : s0, prev = j ? prev1 : prev0;
                            uint32_t c;
                            bool ev;
                            if (T0 + tl == 0) {
                                c = 1u << 17;
                                ev = true;
                            } else if (sc <= prev) {
                                c = exp_negative_q17(sat32(static_cast<long long>(sc) - prev), S.lut, a.log2e_q21);
                                ev = false;
                            } else {
                                c = exp_negative_q17(sat32(static_cast<long long>(prev) - sc), S.lut, a.log2e_q21);
                                ev = true;
                            }
                            coef[tl] = c | (ev ? 0x80000000u : 0u);
                            if (ev) {
                                any_ev = true;
                            } else {
                                const unsigned long long meta =
                                    *reinterpret_cast<const unsigned long long*>(buf + tl * 320);
                                zs += c;
                                bs += term_bound(static_cast<uint32_t>((meta >> vbit) & 31u), c);
                            }
                        }
                    }
                    const unsigned evb = __ballot_sync(FULL, any_ev);
                    zs = __reduce_add_sync(FULL, zs);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) bs += __shfl_xor_sync(FULL, bs, o);
                    if (lane == 31) misc[0] = max(carry, mx);
                    if (lane == 0) {
                        S.tinfo[p].ev = evb;
                        S.tinfo[p].zsum = zs;
                        S.tinfo[p].bound = bs;
                    }
                }
                item_wbar();
                {   // state terms: warp = 4 tokens, lane = dimension
                    int32_t ps = 0;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int tl = wcw * 4 + i;
                        if (tl < cnt) {
                            const uint8_t* rec = buf + tl * 320;
                            const unsigned long long meta = *reinterpret_cast<const unsigned long long*>(rec);
                            const uint32_t sh = static_cast<uint32_t>((meta >> vbit) & 31u);
                            const int v8 = static_cast<int8_t>(rec[192 + dim]);
                            const uint32_t cf = coef[tl];
                            int32_t term;
                            if (cf >> 31) {
                                term = static_cast<int32_t>(static_cast<uint32_t>(v8) << sh);  // v itself
                            } else {
                                term = term_q17(v8, sh, cf);
                                ps += term;
                            }
                            tbuf[tl * 32 + dl] = term;
                        }
                    }
                    atomicAdd(&psum[dl], ps);
                }
            }
        } else if (warp == 0 && k >= 1) {  // tile k - 1 onto the state, in token order
            const int kp = k - 1, p = kp & 1, T0 = kp * kTile, cnt = min(kTile, n - T0);
            const TileInfo ti = S.tinfo[p];
            const long long mag = st < 0 ? -static_cast<long long>(st) : st;
            if (ti.ev == 0 && static_cast<unsigned long long>(mag) + ti.bound <= static_cast<unsigned long long>(INT32_MAX)) {
                st += S.psum[p * 32 + dl];  // no step of the chain can saturate: the sum is exact
                z = (z + static_cast<uint32_t>(ti.zsum)) & M30;
            } else {
                const uint32_t* coef = S.coef + p * kTile;
                const int32_t* tbuf = S.tbuf + p * kTile * 32;
                for (int tl = 0; tl < cnt; ++tl) {
                    const uint32_t cf = coef[tl];
                    const uint32_t cc = cf & 0x7fffffffu;
                    const int32_t tv = tbuf[tl * 32 + dl];
                    if (T0 + tl == 0) {
                        st = tv;
                        z = 1u << 17;
                    } else if (cf >> 31) {  // new maximum: rescale, then add v (emulator:674-685)
                        st = add_sat32(mulq17_w(st, cc), tv);
                        z = ((static_cast<uint32_t>(mulq17_w(static_cast<int32_t>(z), cc)) & M30) + (1u << 17)) & M30;
                    } else {
                        st = add_sat32(st, tv);
                        z = (z + cc) & M30;
                    }
                }
            }
        }
        item_bar();
    }
    if (warp == 0) {  // normalise and quantise this part's 32-value group (emulator:686-711)
        const uint32_t inv = z == 0 ? 0u : static_cast<uint32_t>(((1ull << 34) + (z >> 1)) / z);
        const int32_t o = mulq17(st, inv);
        const int32_t mag = o == INT32_MIN ? INT32_MAX : abs(o);
        const int32_t mx = __reduce_max_sync(FULL, mag);
        const float maxf = __fmul_rn(__int2float_rn(mx), 1.0f / 131072.0f);
        int maxe = -127;
        if (maxf != 0.0f) frexpf(maxf, &maxe);
        const float inv_scale = maxf == 0.0f ? 0.0f : pow2f(13 - maxe);
        float r = __fmul_rn(__fmul_rn(__int2float_rn(o), 1.0f / 131072.0f), inv_scale);
        r = __fadd_rn(r, r >= 0.0f ? 0.5f : -0.5f);
        r = fmaxf(-8191.0f, fminf(8191.0f, r));
        a.out_q[h * kHeadDim + dim] = static_cast<int16_t>(__float2int_rz(r));
        if (lane == 0) a.out_e[h * 4 + part] = maxf == 0.0f ? 0 : static_cast<uint8_t>(maxe + 127);
    }
}

// Standalone attention step of one layer: one CTA per (head, part) item,
// 128 CTAs of 576 threads.  Position from a.pos_ptr; q/k/v from a.direct or
// the QKV partials.
__global__ void __launch_bounds__(kItemThreads, 1) k_attn_items(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(128) uint8_t item_smem[];
    uint64_t* abar = reinterpret_cast<uint64_t*>(item_smem);
    const AttnItemSmem S = attn_item_carve(item_smem + 128);
    const int item = blockIdx.x, h = item / kAttnParts, part = item % kAttnParts;
    const int pos = *a.pos_ptr;
    if (pos < 0 || pos >= a.stride) {
        if (threadIdx.x == 0) atomicOr(a.err, kErrArg);
        return;
    }
    attn_item(a, S, abar, h, part, static_cast<int>(threadIdx.x), nullptr, [] {},
              [&](unsigned code) { atomicOr(a.err, code); });
}

__host__ __device__ constexpr size_t attn_items_smem_bytes() { return 128 + kAttnItemBytes; }

}  // namespace i4d
