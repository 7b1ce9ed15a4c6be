// i4d_attn_item.cuh -- one (head, 32-dimension part) item of the SwiftKV
// attention step (swiftkv_attention_4pe, emulator:602-714; the HLS scan of
// swiftkv_attention.cpp:1882-2032), shared by the persistent token kernel and
// the standalone attention kernel.  18 warps (576 threads) work on an item.
//
// The current token: q/k/v of the head (from the QKV bank partials or given
// directly), Q15.17, adjacent-pair RoPE, the KV shift quantiser and the
// 320-byte record (part 0 writes it to the cache).  Then the cache is
// scanned in tiles of kTile records, double-buffered by bulk copies; per
// tile the 16 worker warps compute
//  * scores: exact integer dot products (16 warps x 4 tokens, 8 lanes each);
//  * coefficients (two warps, one token per lane): the running maximum before
//    each token is a prefix maximum carried across tiles, so every softmax
//    coefficient c_t is known at once, with the tokens where the maximum
//    grows ("events", and token 0), the tile's sum of c_t over its other
//    tokens and a bound on the magnitudes of their state terms;
//  * state terms mulq17(v_t, c_t) per (token, dimension) in 32-bit form (v_t
//    itself at events).
// Warp 0 (lane = dimension) then applies the tile, one tile behind the
// workers.  When the tile's bound shows that no step of the reference's
// saturating chain can saturate, the runs of non-event tokens are added as
// plain sums (integer addition is associative; the normaliser adds modulo
// 2^30) and only the events (rescale, then add v) are applied one by one;
// otherwise the reference's token-order recurrence runs over the
// precomputed terms.  Either way the state is bit-exact with the sequential
// scan.
#pragma once

#include "i4d_attention.cuh"

namespace i4d {

constexpr int kItemWarps = 18;
constexpr int kItemThreads = 32 * kItemWarps;
constexpr int kAttnParts = 4;              // 32-dimension parts per head
constexpr int kAttnItems = kHeads * kAttnParts;

constexpr int kTileBytes = kTile * 320;

struct TileInfo {
    unsigned evm[4];            // bit t of word w: token 32w + t of the window is an event (token 0 included)
    unsigned long long bound;   // bound on sum |term_t| + sum |v_e| over the window (>= 2^40: unbounded)
    unsigned zsum;              // sum of c_t over the window's non-event tokens
    unsigned runs;              // nonzero: each run's sums are in place (the workers' run pass ran)
    unsigned nev;               // events in the window (set by the run pass)
    unsigned pad[3];
};

struct AttnItemSmem {
    // Two tile buffers of kTile records, adjacent: buffer b at tiles + b * kTileBytes.
    // (A pointer array indexed by the runtime parity would put the whole
    // carve in local memory.)
    uint8_t* tiles;
    uint8_t* cur;         // current token's record
    int32_t* score;       // [2 * kTile]: a single window scores up to 128 tokens
    uint32_t* coef;       // [2][kTile]: c | event << 31, by tile parity
    int32_t* tbuf;        // [2][kTile][32]: state terms of this part (v_t itself at events)
    TileInfo* tinfo;      // [2]
    uint32_t* zseg;       // [kZseg]: per run of non-event tokens (in token order), the sum of its c_t
    uint32_t* lut;        // [33] exp2 table
    int32_t* qrot;        // [128]
    unsigned long long* meta;  // current record's shift word
    int* misc;            // [16]
};

constexpr int kZseg = 2 * kTile + 4;       // runs of a window: one more than its events (by parity: 2 x (kTile + 2))
constexpr size_t kAttnItemBytes = 2 * kTile * 320 + 320 + 2 * kTile * 4 + 2 * kTile * 4 + 2 * kTile * 32 * 4 +
                                  2 * sizeof(TileInfo) + kZseg * 4 + 144 + 128 * 4 + 16 + 16 * 4;

__device__ __forceinline__ AttnItemSmem attn_item_carve(uint8_t* p) {
    AttnItemSmem s;
    s.tiles = p;
    p += 2 * kTile * 320;
    s.cur = p;
    p += 320;
    s.score = reinterpret_cast<int32_t*>(p);
    p += 2 * kTile * 4;
    s.coef = reinterpret_cast<uint32_t*>(p);
    p += 2 * kTile * 4;
    s.tbuf = reinterpret_cast<int32_t*>(p);
    p += 2 * kTile * 32 * 4;
    s.tinfo = reinterpret_cast<TileInfo*>(p);
    p += 2 * sizeof(TileInfo);
    s.zseg = reinterpret_cast<uint32_t*>(p);
    p += kZseg * 4;
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

// Upper bound on |term_q17(v8, shift, c)| over every int8 v8, and on |v8 <<
// shift| (an event's value, c = 2^17), at most 2^25 each; anything larger
// reads as 2^40 (no bound).
__device__ __forceinline__ uint32_t term_bound(uint32_t shift, uint32_t c) {
    if (shift > 24) return 1u << 31;
    const unsigned long long b = ((static_cast<unsigned long long>(128u * c) << shift) >> 17) + 1ull;
    return b > (1ull << 25) ? (1u << 31) : static_cast<uint32_t>(b);
}

// Bounded mbarrier wait of an item; `fail(code)` records a timeout, and a
// nonzero *abort_word (may be null) ends the wait early.
template <class Fail>
__device__ __forceinline__ bool item_mbar_wait(uint64_t* bar, uint32_t parity, const unsigned* abort_word,
                                               Fail fail) {
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u && abort_word && *reinterpret_cast<const volatile unsigned*>(abort_word)) return false;
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
// `mark(k)` runs on thread 0 at the item's internal milestones (k = 0: the
// current token done; 1 + i: tile loop iteration i done, i < 3; 4: all tiles
// applied; 5: outputs stored).
template <class WaitInput, class Fail, class Mark>
__device__ __forceinline__ void attn_item(const AttnArgs a, const AttnItemSmem S, uint64_t* abar, int h, int part,
                                          int tid, const unsigned* abort_word, WaitInput wait_input, Fail fail,
                                          Mark mark) {
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
        misc[2] = INT32_MIN;  // running maximum before tile k: misc[2 + (k & 1)]
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
    // A context of up to 2 * kTile tokens is one window over both (adjacent)
    // tile buffers, scanned in one pass; a longer one goes tile by tile.
    const bool one = n <= 2 * kTile;
    if (tid == 0) {
        // Cached records of earlier tokens are final: stream the first tile
        // (both, for a single window) while the projections are still being
        // produced.
        const int cnt = min(kTile, n);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&abar[0], cnt * 320);
        bulk_g2s(S.tiles, head_base, cnt * 320, &abar[0]);
        if (one && n > kTile) {
            mbar_arrive_expect_tx(&abar[1], (n - kTile) * 320);
            bulk_g2s(S.tiles + kTileBytes, head_base + static_cast<size_t>(kTile) * 320, (n - kTile) * 320, &abar[1]);
        }
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
    // q split into 16-bit halves for dp2a, per 16-value half-group hg and
    // pair i: qs[8 hg + i] (high halves) and qs[64 + 8 hg + i] (low halves),
    // in place of qrot.  It stays in shared memory: held in registers
    // through the scan it would be demoted to local memory, whose lines the
    // token kernel's small L1 does not keep.
    const int hg = lane & 7;
    {
        uint32_t qh = 0, ql = 0;
        if (tid < 64) {
            const int32_t x0 = S.qrot[2 * tid], x1 = S.qrot[2 * tid + 1];
            qh = (static_cast<uint32_t>(x0 >> 16) & 0xffffu) | (static_cast<uint32_t>(x1 >> 16) << 16);
            ql = (static_cast<uint32_t>(x0) & 0xffffu) | (static_cast<uint32_t>(x1) << 16);
        }
        item_bar();
        if (tid < 64) {
            reinterpret_cast<uint32_t*>(S.qrot)[tid] = qh;
            reinterpret_cast<uint32_t*>(S.qrot)[64 + tid] = ql;
        }
    }
    item_bar();
    if (tid == 0) mark(0);

    const int dl = lane;                     // dimension inside this part
    const int dim = part * 32 + dl;
    const uint32_t vbit = 20 + 5 * part;     // this part's V shift field in a record's word 0
    int32_t st = 0;                          // warp 0: the state of dimension `dim`
    uint32_t z = 1u << 17;                   // warp 0: the normaliser (every lane)
    const int wtid = tid - 64, wcw = warp - 2;
    const int nwin = one ? 1 : ntiles;       // windows: W tokens each
    const int W = one ? 2 * kTile : kTile;
    static_assert(kTile == 64, "a window's event masks are 32-token words, at most four");
    // Window k onto the state (warp 0, lane = dimension), in token order.
    auto apply = [&](int k) {
        const int p = one ? 0 : k & 1, T0 = k * W, cnt = min(W, n - T0);
        const TileInfo& ti = S.tinfo[p];
        const uint32_t* coef = S.coef + p * kTile;
        const int32_t* tbuf = S.tbuf + p * kTile * 32 + dl;
        const uint32_t* zseg = S.zseg + (one ? 0 : p * (kTile + 2));
        const long long mag = st < 0 ? -static_cast<long long>(st) : st;
        if (one && ti.runs) {
            // A single window starts from the empty state, so its bound alone
            // decides (the run pass ran only if it holds): the chain over
            // the compact arrays the run pass left in the record buffers.
            const int32_t* RS = reinterpret_cast<const int32_t*>(S.tiles) + dl;
            const int32_t* EV = RS + (2 * kTile + 1) * 32;
            const uint32_t* EC = reinterpret_cast<const uint32_t*>(EV - dl + 2 * kTile * 32);
            const int nev = static_cast<int>(ti.nev);
            // Event 0 is token 0, which resets the state (run 0 is empty).
            st = EV[0];
            z = 1u << 17;
            int32_t rs = RS[32], ev = EV[32];
            uint32_t c = EC[1], zr = zseg[1];
            for (int i = 1; i < nev; ++i) {
                const int j = i + 1 < nev ? i + 1 : i;  // operands of the next event, loaded ahead
                const int32_t rs2 = RS[j * 32], ev2 = EV[j * 32];
                const uint32_t c2 = EC[j], zr2 = zseg[j];
                st = mulq17_w(st + rs, c) + ev;
                z = ((static_cast<uint32_t>(mulq17_w(static_cast<int32_t>((z + zr) & M30), c)) & M30) + (1u << 17)) & M30;
                rs = rs2;
                ev = ev2;
                c = c2;
                zr = zr2;
            }
            st += RS[nev * 32];
            z = (z + zseg[nev]) & M30;
        } else if (ti.bound <= static_cast<unsigned long long>(INT32_MAX) &&
                   static_cast<unsigned long long>(mag) + ti.bound <= static_cast<unsigned long long>(INT32_MAX)) {
            // A 64-token tile of a longer context: |state| stays below |st| +
            // bound <= 2^31 - 1 at every step, so no step saturates; each run
            // of non-event tokens is summed here from the terms (eight
            // independent accumulators; integer addition is associative), and
            // only the events are applied one by one.  This runs one tile
            // behind the workers, in parallel with their next tile.
            unsigned long long m = static_cast<unsigned long long>(ti.evm[0]) |
                                   (static_cast<unsigned long long>(ti.evm[1]) << 32);
            int t = 0;
            for (;;) {
                const int e = m ? __ffsll(static_cast<long long>(m)) - 1 : cnt;
                int32_t s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0, s5 = 0, s6 = 0, s7 = 0;
                uint32_t z0 = 0, z1 = 0;
                for (; t + 8 <= e; t += 8) {
                    s0 += tbuf[t * 32];
                    s1 += tbuf[(t + 1) * 32];
                    s2 += tbuf[(t + 2) * 32];
                    s3 += tbuf[(t + 3) * 32];
                    s4 += tbuf[(t + 4) * 32];
                    s5 += tbuf[(t + 5) * 32];
                    s6 += tbuf[(t + 6) * 32];
                    s7 += tbuf[(t + 7) * 32];
                    z0 += (coef[t] + coef[t + 1]) + (coef[t + 2] + coef[t + 3]);
                    z1 += (coef[t + 4] + coef[t + 5]) + (coef[t + 6] + coef[t + 7]);
                }
                for (; t < e; ++t) {
                    s0 += tbuf[t * 32];
                    z0 += coef[t];
                }
                st += ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7));
                z = (z + z0 + z1) & M30;
                if (e >= cnt) break;
                const uint32_t c = coef[e] & 0x7fffffffu;
                const int32_t v = tbuf[e * 32];
                if (T0 + e == 0) {
                    st = v;
                    z = 1u << 17;
                } else {  // new maximum: rescale, then add v (emulator:674-685)
                    st = mulq17_w(st, c) + v;
                    z = ((static_cast<uint32_t>(mulq17_w(static_cast<int32_t>(z), c)) & M30) + (1u << 17)) & M30;
                }
                t = e + 1;
                m &= m - 1ull;
            }
        } else {
            // The reference's recurrence (emulator:656-685), saturating at
            // every step, with each term recomputed from the cached record
            // (the window's buffers may already hold later records).
            for (int tl = 0; tl < cnt; ++tl) {
                const uint32_t cf = coef[tl];
                const uint32_t cc = cf & 0x7fffffffu;
                const uint8_t* rec = T0 + tl == pos ? S.cur : kv_record(a, h, T0 + tl);
                const unsigned long long meta = *reinterpret_cast<const volatile unsigned long long*>(rec);
                const uint32_t sh = static_cast<uint32_t>((meta >> vbit) & 31u);
                const int v8 = static_cast<int8_t>(*reinterpret_cast<const volatile uint8_t*>(rec + 192 + dim));
                const int32_t vfull = static_cast<int32_t>(static_cast<uint32_t>(v8) << sh);
                if (cf >> 31) {
                    if (T0 + tl == 0) {
                        st = vfull;
                        z = 1u << 17;
                    } else {  // new maximum: rescale, then add v (emulator:674-685)
                        st = add_sat32(mulq17_w(st, cc), vfull);
                        z = ((static_cast<uint32_t>(mulq17_w(static_cast<int32_t>(z), cc)) & M30) + (1u << 17)) & M30;
                    }
                } else {
                    st = add_sat32(st, term_q17(v8, sh, cc));
                    z = (z + cc) & M30;
                }
            }
        }
    };
    for (int k = 0; k <= nwin; ++k) {
        if (warp >= 2) {
            if (k < nwin) {
                const int T0 = k * W, cnt = min(W, n - T0), p = one ? 0 : k & 1;
                const int rounds = (cnt + 63) >> 6;  // 64-token rounds of the worker warps
                uint8_t* buf = S.tiles + p * kTileBytes;
                uint32_t* coef = S.coef + p * kTile;
                int32_t* tbuf = S.tbuf + p * kTile * 32;
                TileInfo& ti = S.tinfo[p];
                if (!one && wtid == 0 && k + 1 < ntiles) {  // buffer p ^ 1 was last read in iteration k - 1
                    fence_proxy_async_smem();
                    const int c2 = min(kTile, n - T0 - kTile);
                    mbar_arrive_expect_tx(&abar[p ^ 1], c2 * 320);
                    bulk_g2s(S.tiles + (p ^ 1) * kTileBytes, head_base + static_cast<size_t>(T0 + kTile) * 320, c2 * 320,
                             &abar[p ^ 1]);
                }
                if (wtid == 0) {  // this parity's summary was last read by warp 0 in iteration k - 1
                    ti.zsum = 0u;
                    ti.bound = 0ull;
                }
                if (wtid < 4) ti.evm[wtid] = 0u;  // words past the window's last token stay empty
                item_mbar_wait(&abar[p], static_cast<uint32_t>((k >> 1) & 1), abort_word, fail);
                if (one && cnt > kTile) item_mbar_wait(&abar[1], 0u, abort_word, fail);
                if (pos < T0 + cnt) {  // the window holds the current token: use the fresh record
                    if (wtid < 80)
                        reinterpret_cast<uint32_t*>(buf + (pos - T0) * 320)[wtid] =
                            reinterpret_cast<const uint32_t*>(S.cur)[wtid];
                    item_wbar();
                }
                {   // scores (emulator:633-655): 16 warps x 4 tokens per round, 8 lanes per token
                    const uint32_t* qs = reinterpret_cast<const uint32_t*>(S.qrot);
                    const uint4 qa = *reinterpret_cast<const uint4*>(qs + 8 * hg);
                    const uint4 qb = *reinterpret_cast<const uint4*>(qs + 8 * hg + 4);
                    const uint4 la = *reinterpret_cast<const uint4*>(qs + 64 + 8 * hg);
                    const uint4 lb = *reinterpret_cast<const uint4*>(qs + 64 + 8 * hg + 4);
                    const uint32_t qh2[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    const uint32_t ql2[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
                    long long hv[2] = {0, 0};
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const int tl = r * 64 + wcw * 4 + (lane >> 3);
                        if (r < rounds && tl < cnt) {
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
                            hv[r] = wrap_bits(sh >= 10 ? static_cast<long long>(static_cast<unsigned long long>(half) << (sh - 10))
                                                       : (half >> (10 - sh)), 44);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        hv[r] += __shfl_xor_sync(FULL, hv[r], 1);
                        hv[r] += __shfl_xor_sync(FULL, hv[r], 2);
                        hv[r] += __shfl_xor_sync(FULL, hv[r], 4);
                        const int tl = r * 64 + wcw * 4 + (lane >> 3);
                        if ((lane & 7) == 0 && r < rounds && tl < cnt)
                            S.score[tl] = sat32(rshift_even(wrap_bits(hv[r], 44) * a.score_scale, 24));
                    }
                }
                item_wbar();
                if (wcw * 32 < cnt) {
                    // Coefficients (emulator:656-672), lane = token wcw * 32 + lane:
                    // the running maximum before it is the largest of the
                    // carry, the window's earlier 32-token words and the
                    // prefix of its own word.
                    const int tl = wcw * 32 + lane;
                    int32_t carry = misc[2 + p];
                    for (int j = 0; j < wcw; ++j) carry = max(carry, __reduce_max_sync(FULL, S.score[j * 32 + lane]));
                    const int32_t sc = tl < cnt ? S.score[tl] : INT32_MIN;
                    int32_t pm = sc;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int32_t y = __shfl_up_sync(FULL, pm, o);
                        if (lane >= o) pm = max(pm, y);
                    }
                    int32_t ex = __shfl_up_sync(FULL, pm, 1);
                    if (lane == 0) ex = INT32_MIN;
                    const int32_t prev = max(carry, ex);
                    const bool ev = tl < cnt && (T0 + tl == 0 || sc > prev);
                    const unsigned evm = __ballot_sync(FULL, ev);
                    if (lane == 0) ti.evm[wcw] = evm;
                    if (lane == 31 && (wcw + 1) * 32 >= cnt) misc[2 + (p ^ 1)] = max(carry, pm);  // the next window's carry
                    uint32_t c = 0, zs = 0, bs = 0;
                    if (tl < cnt) {
                        if (T0 + tl == 0) c = 1u << 17;
                        else if (!ev) c = exp_negative_q17(sat32(static_cast<long long>(sc) - prev), S.lut, a.log2e_q21);
                        else c = exp_negative_q17(sat32(static_cast<long long>(prev) - sc), S.lut, a.log2e_q21);
                        coef[tl] = c | (ev ? 0x80000000u : 0u);
                        const uint32_t vsh = static_cast<uint32_t>(
                            (*reinterpret_cast<const unsigned long long*>(buf + tl * 320) >> vbit) & 31u);
                        zs = ev ? 0u : c;
                        bs = term_bound(vsh, ev ? (1u << 17) : c);
                    }
                    zs = __reduce_add_sync(FULL, zs);
                    const bool big = __any_sync(FULL, bs > (1u << 25));
                    bs = __reduce_add_sync(FULL, big ? 0u : bs);  // at most 32 * 2^25
                    if (lane == 0) {
                        atomicAdd(&ti.zsum, zs);
                        atomicAdd(&ti.bound, big ? (1ull << 40) : static_cast<unsigned long long>(bs));
                    }
                }
                item_wbar();
                for (int r = 0; r < rounds; ++r) {  // state terms: warp = 4 tokens per round, lane = dimension
                    unsigned long long mt[4];
                    int v8[4];
                    uint32_t cf[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {  // operands first, then the arithmetic
                        const int tl = min(r * 64 + wcw * 4 + i, cnt - 1);
                        const uint8_t* rec = buf + tl * 320;
                        mt[i] = *reinterpret_cast<const unsigned long long*>(rec);
                        v8[i] = static_cast<int8_t>(rec[192 + dim]);
                        cf[i] = coef[tl];
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int tl = r * 64 + wcw * 4 + i;
                        const uint32_t sh = static_cast<uint32_t>((mt[i] >> vbit) & 31u);
                        const int32_t t = (cf[i] >> 31) ? static_cast<int32_t>(static_cast<uint32_t>(v8[i]) << sh)  // v itself
                                                        : term_q17(v8[i], sh, cf[i]);
                        if (tl < cnt) tbuf[tl * 32 + dl] = t;
                    }
                }
                // Run pass: warp w sums runs w, w + 16, ... of non-event
                // tokens (run r ends before event r, the last run at the
                // window's end) per dimension into the run's last term slot,
                // and their c_t into zseg[r].  It is done only when the
                // window's bound allows the summed form at all; warp 0 still
                // checks it against its state before using the sums.
                // (Tiles of a longer context go without: warp 0 sums their
                // runs from the terms, one tile behind.)
                if (one) {
                item_wbar();
                const bool runs = ti.bound <= static_cast<unsigned long long>(INT32_MAX);
                if (runs) {
                    const unsigned e0 = ti.evm[0], e1 = ti.evm[1], e2 = ti.evm[2], e3 = ti.evm[3];
                    const int n0 = __popc(e0), n1 = __popc(e1), n2 = __popc(e2), n3 = __popc(e3);
                    const int nev = n0 + n1 + n2 + n3;
                    // Position of event r (0-based, in token order); nev -> cnt.
                    auto ev_pos = [&](int r) -> int {
                        if (r < 0) return -1;
                        if (r >= nev) return cnt;
                        if (r < n0) return __fns(e0, 0, r + 1);
                        r -= n0;
                        if (r < n1) return 32 + __fns(e1, 0, r + 1);
                        r -= n1;
                        if (r < n2) return 64 + __fns(e2, 0, r + 1);
                        return 96 + __fns(e3, 0, r - n2 + 1);
                    };
                    uint32_t* zseg = S.zseg + (one ? 0 : p * (kTile + 2));
                    // A single window has no further copies, so its record
                    // buffers are free now: the runs and events go there as
                    // compact arrays in event order (RS[r][32], EV[i][32],
                    // EC[i]) for warp 0's chain.
                    int32_t* RS = reinterpret_cast<int32_t*>(S.tiles);
                    int32_t* EV = RS + (2 * kTile + 1) * 32;
                    uint32_t* EC = reinterpret_cast<uint32_t*>(EV + 2 * kTile * 32);
                    if (one)
                        for (int i = wcw; i < nev; i += 16) {
                            const int e = ev_pos(i);
                            EV[i * 32 + dl] = tbuf[e * 32 + dl];
                            if (lane == 0) EC[i] = coef[e] & 0x7fffffffu;
                        }
                    for (int r = wcw; r <= nev; r += 16) {
                        const int t0 = ev_pos(r - 1) + 1, t1 = ev_pos(r);
                        int32_t s0 = 0, s1 = 0;
                        uint32_t zs = 0;
                        int t = t0;
                        for (; t + 2 <= t1; t += 2) {
                            s0 += tbuf[t * 32 + dl];
                            s1 += tbuf[(t + 1) * 32 + dl];
                            zs += coef[t] + coef[t + 1];
                        }
                        if (t < t1) {
                            s0 += tbuf[t * 32 + dl];
                            zs += coef[t];
                        }
                        if (one) RS[r * 32 + dl] = s0 + s1;
                        else if (t1 > t0) tbuf[(t1 - 1) * 32 + dl] = s0 + s1;
                        if (lane == 0) zseg[r] = zs;
                    }
                    if (wtid == 0) ti.nev = static_cast<unsigned>(nev);
                }
                if (wtid == 0) ti.runs = runs ? 1u : 0u;
                }  // single window
            }
        } else if (warp == 0 && k >= 1) {
            apply(k - 1);  // window k - 1, one window behind the workers
        }
        item_bar();
        if (tid == 0 && k < 3) mark(1 + k);
    }
    if (tid == 0) mark(4);
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
        if (tid == 0) mark(5);
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
              [&](unsigned code) { atomicOr(a.err, code); }, [](int) {});
}

__host__ __device__ constexpr size_t attn_items_smem_bytes() { return 128 + kAttnItemBytes; }

}  // namespace i4d
