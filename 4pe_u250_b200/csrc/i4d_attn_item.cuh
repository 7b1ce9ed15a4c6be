// i4d_attn_item.cuh -- one (head, 32-dimension part) item of the SwiftKV
// attention step (swiftkv_attention_4pe, emulator:602-714; the HLS scan of
// swiftkv_attention.cpp:1882-2032), shared by the persistent token kernel and
// the standalone attention kernel.  18 warps (576 threads) work on an item.
//
// The current token: q/k/v of the head (from the QKV bank partials or given
// directly), Q15.17, adjacent-pair RoPE, the KV shift quantiser and the
// 320-byte record (part 0 writes it to the cache).  Then the cache is
// scanned in windows of kWin records, read straight from global memory (the
// head's records are requested into L2 when the item starts); per window the
// 16 worker warps compute
//  * scores: exact integer dot products (8 lanes per token, 4 rounds of 4
//    tokens per warp), keeping this part's V bytes and V shift per token;
//  * coefficients (one warp per 32 tokens, one token per lane): the running
//    maximum before each token is a prefix maximum carried across windows,
//    so every softmax coefficient c_t is known at once, with the tokens where
//    the maximum grows ("events", and token 0);
//  * run sums (lane = dimension, 16 consecutive tokens per warp): the state
//    terms mulq17(v_t, c_t) of each run of non-event tokens and their c_t,
//    summed per run (integer addition is associative; the normaliser adds
//    modulo 2^30) -- each warp sums its part of every run it touches, and a
//    run that spans warps is completed by walking back over their partial
//    sums -- v_t at each event, and per dimension the sum of the magnitudes
//    of all of them.
// Warp 0 (lane = dimension) then applies the window.  A rescale never grows
// the state's magnitude, so while |state| plus that magnitude sum stays
// within int32, no step of the reference's saturating chain can saturate:
// the runs then add as whole sums and only the events (rescale, then add v)
// are applied one by one.  Otherwise (or with more than kMaxEv events) the
// reference's token-order recurrence runs over the window's coefficients and
// V bytes.  Either way the state is bit-exact with the sequential scan.
#pragma once

#include "i4d_attention.cuh"

namespace i4d {

constexpr int kItemWarps = 18;
constexpr int kItemThreads = 32 * kItemWarps;
constexpr int kAttnParts = 4;              // 32-dimension parts per head
constexpr int kAttnItems = kHeads * kAttnParts;

constexpr int kWin = 256;                  // tokens per window (16 worker warps x 4 rounds x 4 tokens)
constexpr int kMaxEv = 96;                 // events a window applies as a chain (more: token by token)
constexpr int kRunWarps = 16;              // worker warps of the run pass, 16 tokens each

// Per-window summary of the run pass.  Worker warp w covers tokens
// [16 w, 16 w + 16): pre[w] is the sum of its values before its first event
// (all of them when it holds none), post[w] the sum after its last event;
// the runs between two of its events go straight to the run sums.
struct WinInfo {
    unsigned evm[kWin / 32];         // bit t of word w: token 32w + t of the window is an event (token 0 included)
    int32_t pre[kRunWarps][32];
    int32_t post[kRunWarps][32];
    uint32_t mag[kRunWarps][32];     // per warp and dimension: sum of |value|, clamped to 2^31
    uint32_t zpre[kRunWarps], zpost[kRunWarps];
    uint32_t pad[4];
};
static_assert(sizeof(WinInfo) % 16 == 0, "the carve keeps 16-byte alignment after the window summary");

struct AttnItemSmem {
    uint8_t* cur;         // current token's record (320 B)
    int32_t* score;       // [kWin]
    uint32_t* coef;       // [kWin]: c | event << 31
    int8_t* vbuf;         // [kWin][32]: this part's V bytes
    uint8_t* vsh;         // [kWin]: this part's V shift
    int32_t* rs;          // [kMaxEv + 1][32]: run sums per dimension (run r ends before event r)
    int32_t* ev;          // [kMaxEv][32]: v << shift at each event
    uint32_t* ec;         // [kMaxEv]: each event's coefficient
    uint32_t* zs;         // [kMaxEv + 1]: each run's sum of c_t (mod 2^32)
    WinInfo* info;
    uint32_t* lut;        // [33] exp2 table
    int32_t* qrot;        // [128]
    int* misc;            // [16]
};

constexpr size_t kZsBytes = ((kMaxEv + 1) * 4 + 15) / 16 * 16;
constexpr size_t kAttnItemBytes = 320 + kWin * 4 + kWin * 4 + kWin * 32 + kWin + (kMaxEv + 1) * 128 +
                                  kMaxEv * 128 + kMaxEv * 4 + kZsBytes + sizeof(WinInfo) + 144 + 128 * 4 + 16 * 4;
// Offsets of the carve's 16-byte accessed arrays (the carve starts 16-byte
// aligned): coef (four-word loads), vbuf (cp.async and 16-byte stores), vsh
// (16-byte loads), the window summary (64-bit atomics) and qrot (16-byte loads).
constexpr size_t kOffCoef = 320 + kWin * 4;
constexpr size_t kOffVbuf = kOffCoef + kWin * 4;
constexpr size_t kOffVsh = kOffVbuf + kWin * 32;
constexpr size_t kOffInfo = kOffVsh + kWin + (kMaxEv + 1) * 128 + kMaxEv * 128 + kMaxEv * 4 + kZsBytes;
constexpr size_t kOffQrot = kOffInfo + sizeof(WinInfo) + 144;
static_assert(kOffCoef % 16 == 0 && kOffVbuf % 16 == 0 && kOffVsh % 16 == 0 && kOffInfo % 16 == 0 &&
                  kOffQrot % 16 == 0,
              "16-byte alignment of the attention item's vector-accessed arrays");
static_assert(kOffQrot + 128 * 4 + 16 * 4 == kAttnItemBytes, "the carve and its size agree");

__device__ __forceinline__ AttnItemSmem attn_item_carve(uint8_t* p) {
    AttnItemSmem s;
    s.cur = p;
    p += 320;
    s.score = reinterpret_cast<int32_t*>(p);
    p += kWin * 4;
    s.coef = reinterpret_cast<uint32_t*>(p);
    p += kWin * 4;
    s.vbuf = reinterpret_cast<int8_t*>(p);
    p += kWin * 32;
    s.vsh = p;
    p += kWin;
    s.rs = reinterpret_cast<int32_t*>(p);
    p += (kMaxEv + 1) * 128;
    s.ev = reinterpret_cast<int32_t*>(p);
    p += kMaxEv * 128;
    s.ec = reinterpret_cast<uint32_t*>(p);
    p += kMaxEv * 4;
    s.zs = reinterpret_cast<uint32_t*>(p);
    p += kZsBytes;
    s.info = reinterpret_cast<WinInfo*>(p);
    p += sizeof(WinInfo);
    s.lut = reinterpret_cast<uint32_t*>(p);
    p += 144;
    s.qrot = reinterpret_cast<int32_t*>(p);
    p += 128 * 4;
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

// One attention item: head h, dimensions [32 part, 32 part + 32), thread
// `tid` of 576.  `wait_input()` runs on thread 0 after the head's records
// are requested into L2 (the token kernel waits there for the QKV stage).
// Warp 0 ends with the item's 32 outputs stored (a.out_q, a.out_e); the
// caller publishes them.
// `mark(k)` runs on thread 0 at the item's internal milestones (k = 0: the
// current token done; 1 + i: window i done, i < 3; 4: all windows applied;
// 5: outputs stored).
template <class WaitInput, class Mark>
__device__ __forceinline__ void attn_item(const AttnArgs a, const AttnItemSmem S, int h, int part, int tid,
                                          WaitInput wait_input, Mark mark) {
    const unsigned FULL = 0xffffffffu;
    const uint32_t M30 = (1u << 30) - 1u;
    const int warp = tid >> 5, lane = tid & 31;
    int* misc = S.misc;
    const int pos = *a.pos_ptr;
    const int n = pos + 1;
    const int nwin = (n + kWin - 1) / kWin;
    const uint8_t* head_base = kv_record(a, h, 0);
    if (tid == 0) misc[2] = INT32_MIN;  // running maximum before window k: misc[2 + (k & 1)]
    if (tid < 33) S.lut[tid] = a.exp2_q30[tid];
    if (tid < 16) reinterpret_cast<uint32_t*>(S.cur)[tid] = 0u;  // record bytes 0..63: shift word (ORed in below), padding
    // RoPE factors of this position: independent of the projections.
    long long rope_c = 0, rope_s = 0;
    if (tid < 128) {
        rope_c = a.rope_cos[pos * 64 + (tid >> 1)];
        rope_s = a.rope_sin[pos * 64 + (tid >> 1)];
    }
    item_bar();
    if (tid == 0) {
        // Cached records of earlier tokens are final: pull the head's records
        // into L2 while the projections are still being produced, in pieces
        // of 64 records, the four parts of the head taking every fourth.
        for (int t = 64 * part; t < pos; t += 64 * kAttnParts)
            bulk_prefetch_l2(head_base + static_cast<size_t>(t) * 320, min(64, pos - t) * 320);
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
        // q split into 16-bit halves for dp2a, per pair i = d / 2: qs[i] the
        // high halves, qs[64 + i] the low halves (per 16-value half-group hg:
        // qs[8 hg ..]).  It stays in shared memory: held in registers
        // through the scan it would be demoted to local memory, whose lines
        // the token kernel's small L1 does not keep.
        const int32_t qn = __shfl_xor_sync(FULL, qr, 1);
        if (!(d & 1)) {
            reinterpret_cast<uint32_t*>(S.qrot)[d >> 1] =
                (static_cast<uint32_t>(qr >> 16) & 0xffffu) | (static_cast<uint32_t>(qn >> 16) << 16);
            reinterpret_cast<uint32_t*>(S.qrot)[64 + (d >> 1)] =
                (static_cast<uint32_t>(qr) & 0xffffu) | (static_cast<uint32_t>(qn) << 16);
        }
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
        // The record's shift word (word 0, zeroed above): this group's fields.
        if (lane == 0)
            atomicOr(reinterpret_cast<unsigned long long*>(S.cur),
                     (static_cast<unsigned long long>(ks) << (5 * warp)) |
                         (static_cast<unsigned long long>(vs) << (20 + 5 * warp)));
    }
    item_bar();
    if (part == 0 && tid < 8)  // bytes 0..63 of the record: the shift word, then zeros
        reinterpret_cast<unsigned long long*>(grec)[tid] = reinterpret_cast<const unsigned long long*>(S.cur)[tid];
    const int hg = lane & 7;
    if (tid == 0) mark(0);

    const int dl = lane;                     // dimension inside this part
    const int dim = part * 32 + dl;
    const uint32_t vbit = 20 + 5 * part;     // this part's V shift field in a record's word 0
    int32_t st = 0;                          // warp 0: the state of dimension `dim`
    uint32_t z = 1u << 17;                   // warp 0: the normaliser (every lane)
    const int wcw = warp - 2;
    WinInfo& wi = *S.info;
    for (int k = 0; k < nwin; ++k) {
        const int T0 = k * kWin, cnt = min(kWin, n - T0);
        if (warp >= 2) {
            // ---- scores (emulator:633-655): token r * 64 + 4 wcw + lane / 8,
            // lane & 7 = 16-value half-group hg of K (and of V) ----
            if (tid - 64 < kWin / 32) wi.evm[tid - 64] = 0u;  // words past the window's last token stay empty
            const int rounds = (cnt + 63) >> 6;
            // Every load of the window first: K and the shift word into
            // registers through the read-only path (records before the
            // current token are final), this part's V bytes straight into
            // shared memory (cp.async), the current token from its record in
            // shared memory.
            uint4 kw[4];
            unsigned long long mt[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int tl = r * 64 + wcw * 4 + (lane >> 3);
                kw[r] = make_uint4(0u, 0u, 0u, 0u);
                mt[r] = 0ull;
                if (r < rounds && tl < cnt && T0 + tl != pos) {
                    const uint8_t* rec = kv_record(a, h, T0 + tl);
                    kw[r] = __ldg(reinterpret_cast<const uint4*>(rec + 64 + hg * 16));
                    mt[r] = __ldg(reinterpret_cast<const unsigned long long*>(rec));
                    if ((hg >> 1) == part) cp_async16(S.vbuf + tl * 32 + (hg & 1) * 16, rec + 192 + hg * 16);
                }
            }
            cp_async_commit();
            if (pos >= T0 && pos - T0 < rounds * 64) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int tl = r * 64 + wcw * 4 + (lane >> 3);
                    if (r < rounds && T0 + tl == pos) {
                        kw[r] = *reinterpret_cast<const uint4*>(S.cur + 64 + hg * 16);
                        mt[r] = *reinterpret_cast<const unsigned long long*>(S.cur);
                        if ((hg >> 1) == part)
                            *reinterpret_cast<uint4*>(S.vbuf + tl * 32 + (hg & 1) * 16) =
                                *reinterpret_cast<const uint4*>(S.cur + 192 + hg * 16);
                    }
                }
            }
            const uint32_t* qs = reinterpret_cast<const uint32_t*>(S.qrot);
            const uint4 qa = *reinterpret_cast<const uint4*>(qs + 8 * hg);
            const uint4 qb = *reinterpret_cast<const uint4*>(qs + 8 * hg + 4);
            const uint4 la = *reinterpret_cast<const uint4*>(qs + 64 + 8 * hg);
            const uint4 lb = *reinterpret_cast<const uint4*>(qs + 64 + 8 * hg + 4);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int tl = r * 64 + wcw * 4 + (lane >> 3);
                long long hv = 0;
                if (r < rounds && tl < cnt) {
                    const uint32_t sh = static_cast<uint32_t>((mt[r] >> (5 * (hg >> 1))) & 31u);
                    int sh16 = 0, sl16 = 0;
                    sh16 = dp2a_lo_ss(qa.x, kw[r].x, sh16);
                    sh16 = dp2a_hi_ss(qa.y, kw[r].x, sh16);
                    sh16 = dp2a_lo_ss(qa.z, kw[r].y, sh16);
                    sh16 = dp2a_hi_ss(qa.w, kw[r].y, sh16);
                    sh16 = dp2a_lo_ss(qb.x, kw[r].z, sh16);
                    sh16 = dp2a_hi_ss(qb.y, kw[r].z, sh16);
                    sh16 = dp2a_lo_ss(qb.z, kw[r].w, sh16);
                    sh16 = dp2a_hi_ss(qb.w, kw[r].w, sh16);
                    sl16 = dp2a_lo_us(la.x, kw[r].x, sl16);
                    sl16 = dp2a_hi_us(la.y, kw[r].x, sl16);
                    sl16 = dp2a_lo_us(la.z, kw[r].y, sl16);
                    sl16 = dp2a_hi_us(la.w, kw[r].y, sl16);
                    sl16 = dp2a_lo_us(lb.x, kw[r].z, sl16);
                    sl16 = dp2a_hi_us(lb.y, kw[r].z, sl16);
                    sl16 = dp2a_lo_us(lb.z, kw[r].w, sl16);
                    sl16 = dp2a_hi_us(lb.w, kw[r].w, sl16);
                    const long long half = static_cast<long long>(sh16) * 65536 + sl16;
                    hv = wrap_bits(sh >= 10 ? static_cast<long long>(static_cast<unsigned long long>(half) << (sh - 10))
                                            : (half >> (10 - sh)), 44);
                    if (hg == 2 * part) S.vsh[tl] = static_cast<uint8_t>((mt[r] >> vbit) & 31u);
                }
                hv += __shfl_xor_sync(FULL, hv, 1);
                hv += __shfl_xor_sync(FULL, hv, 2);
                hv += __shfl_xor_sync(FULL, hv, 4);
                if (hg == 0 && r < rounds && tl < cnt)
                    S.score[tl] = sat32(rshift_even(wrap_bits(hv, 44) * a.score_scale, 24));
            }
            cp_async_wait_all();
            item_wbar();
            if (wcw * 32 < cnt) {
                // ---- coefficients (emulator:656-672), lane = token wcw * 32 +
                // lane: the running maximum before it is the largest of the
                // carry, the window's earlier 32-token words and the prefix of
                // its own word ----
                const int tl = wcw * 32 + lane;
                const int p = k & 1;
                int32_t earlier[kWin / 32 - 1];
#pragma unroll
                for (int j = 0; j < kWin / 32 - 1; ++j) earlier[j] = j < wcw ? S.score[j * 32 + lane] : INT32_MIN;
                int32_t carry = misc[2 + p];
#pragma unroll
                for (int j = 0; j < kWin / 32 - 1; ++j)
                    if (j < wcw) carry = max(carry, __reduce_max_sync(FULL, earlier[j]));
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
                if (lane == 0) wi.evm[wcw] = evm;
                if (lane == 31 && (wcw + 1) * 32 >= cnt) misc[2 + (p ^ 1)] = max(carry, pm);  // the next window's carry
                if (tl < cnt) {
                    uint32_t c;
                    if (T0 + tl == 0) c = 1u << 17;
                    else if (!ev) c = exp_negative_q17(sat32(static_cast<long long>(sc) - prev), S.lut, a.log2e_q21);
                    else c = exp_negative_q17(sat32(static_cast<long long>(prev) - sc), S.lut, a.log2e_q21);
                    S.coef[tl] = c | (ev ? 0x80000000u : 0u);
                }
            }
            item_wbar();
            // ---- runs: tokens [16 wcw, 16 wcw + 16), lane = dimension ----
            int nev = 0, before = 0;
            uint32_t wmask = 0u;  // bit u: worker warp u's tokens hold an event
            const int t0 = wcw * 16;
#pragma unroll
            for (int j = 0; j < kWin / 32; ++j) {
                const unsigned m = wi.evm[j];
                nev += __popc(m);
                if (j < (t0 >> 5)) before += __popc(m);
                wmask |= ((m & 0xffffu) ? 1u : 0u) << (2 * j);
                wmask |= ((m >> 16) ? 1u : 0u) << (2 * j + 1);
            }
            const unsigned mine = (wi.evm[t0 >> 5] >> (t0 & 31)) & 0xffffu;  // this warp's events
            before += __popc(wi.evm[t0 >> 5] & ((1u << (t0 & 31)) - 1u));
            if (nev <= kMaxEv) {
                // The warp's 16 coefficients and shifts as four and one
                // 16-byte shared loads (entries past the window are stale
                // and masked below), its dimension's V bytes one by one.
                int8_t v8[16];
                uint32_t cf[16], sh[16];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 c4 = *reinterpret_cast<const uint4*>(S.coef + t0 + 4 * q);
                    cf[4 * q] = c4.x;
                    cf[4 * q + 1] = c4.y;
                    cf[4 * q + 2] = c4.z;
                    cf[4 * q + 3] = c4.w;
                }
                const uint4 s4 = *reinterpret_cast<const uint4*>(S.vsh + t0);
                const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) sh[i] = (sw[i >> 2] >> (8 * (i & 3))) & 0xffu;
#pragma unroll
                for (int i = 0; i < 16; ++i) v8[i] = S.vbuf[min(t0 + i, cnt - 1) * 32 + dl];
                // Each token's value: v = v8 << shift itself at an event,
                // else the state term mulq17(v, c) (emulator:674-685, on the
                // value of emulator:677); tokens past the window add 0.  The
                // magnitude sum saturates at 2^31 (each |value| taken below
                // 2^31, so two never overflow 32 bits).
                int32_t x[16];
                uint32_t mag = 0u, zsum = 0u;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int32_t vfull = static_cast<int32_t>(static_cast<uint32_t>(v8[i]) << sh[i]);
                    const bool in = t0 + i < cnt;
                    x[i] = !in ? 0 : (cf[i] >> 31) ? vfull : mulq17_w(vfull, cf[i]);
                    const uint32_t ux = static_cast<uint32_t>(x[i]);
                    const uint32_t ax = min(x[i] < 0 ? 0u - ux : ux, 0x7fffffffu);
                    mag = min(mag + ax, 1u << 31);
                    zsum += (in && !(cf[i] >> 31)) ? cf[i] : 0u;
                }
                wi.mag[wcw][dl] = mag;
                if (mine == 0u) {  // one part of one run: a plain sum
                    int32_t acc = 0;
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc += x[i];
                    wi.pre[wcw][dl] = acc;
                    if (lane == 0) wi.zpre[wcw] = zsum;
                } else {
                    // In token order: the part before the first event, each
                    // run between two of this warp's events (complete here:
                    // stored), the part after the last one.
                    int r = before;
                    int32_t acc = 0;
                    uint32_t zacc = 0;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        if ((mine >> i) & 1u) {  // event r ends run r
                            if (r == before) {
                                wi.pre[wcw][dl] = acc;
                                if (lane == 0) wi.zpre[wcw] = zacc;
                            } else {
                                S.rs[r * 32 + dl] = acc;
                                if (lane == 0) S.zs[r] = zacc;
                            }
                            S.ev[r * 32 + dl] = x[i];
                            if (lane == 0) S.ec[r] = cf[i] & 0x7fffffffu;
                            ++r;
                            acc = 0;
                            zacc = 0;
                        } else if (t0 + i < cnt) {
                            acc += x[i];
                            zacc += cf[i];
                        }
                    }
                    wi.post[wcw][dl] = acc;
                    if (lane == 0) wi.zpost[wcw] = zacc;
                }
            }
            item_wbar();
            // A run that crosses warps: the warp holding its closing event
            // (run `before`, closed by this warp's first event), or the last
            // warp for the window's final run, adds the partial sums of the
            // warps back to where the run opened -- after the last event of
            // an earlier warp (its post part), or at the window start.  The
            // opening warp comes from the event mask, the sums are
            // independent loads.
            if (nev <= kMaxEv) {
#pragma unroll 1
                for (int pass = 0; pass < 2; ++pass) {
                    if (pass == 0 && mine == 0u) continue;
                    if (pass == 1 && wcw != kRunWarps - 1) break;
                    const bool own_post = pass == 1 && mine != 0u;  // the final run opened in this warp
                    int32_t tot = own_post ? wi.post[wcw][dl] : wi.pre[wcw][dl];
                    uint32_t zt = own_post ? wi.zpost[wcw] : wi.zpre[wcw];
                    if (!own_post) {
                        const uint32_t m = wmask & ((1u << wcw) - 1u);
                        const int open = m ? 31 - __clz(m) : -1;  // warp whose post part opens the run
                        if (open >= 0) {
                            tot += wi.post[open][dl];
                            zt += wi.zpost[open];
                        }
#pragma unroll
                        for (int u = 0; u < kRunWarps - 1; ++u) {
                            const bool take = u > open && u < wcw;
                            const int32_t pv = wi.pre[u][dl];
                            const uint32_t zv = wi.zpre[u];
                            tot += take ? pv : 0;
                            zt += take ? zv : 0u;
                        }
                    }
                    const int run = pass == 0 ? before : nev;
                    S.rs[run * 32 + dl] = tot;
                    if (lane == 0) S.zs[run] = zt;
                }
            }
        }
        item_bar();
        if (warp == 0) {
            // ---- the window onto the state (lane = dimension), in token order ----
            int nev = 0;
#pragma unroll
            for (int j = 0; j < kWin / 32; ++j) nev += __popc(wi.evm[j]);
            unsigned long long mag = st < 0 ? -static_cast<long long>(st) : st;
#pragma unroll
            for (int w = 0; w < kRunWarps; ++w) mag += wi.mag[w][dl];
            const bool fits = mag <= static_cast<unsigned long long>(INT32_MAX);
            if (nev <= kMaxEv && __all_sync(FULL, fits)) {
                // |state| stays within |st| + the window's magnitude sum <=
                // 2^31 - 1 at every step: runs add as sums, events one by one.
                st += S.rs[dl];
                z = (z + S.zs[0]) & M30;
                int32_t ev = nev > 0 ? S.ev[dl] : 0, rs = nev > 0 ? S.rs[32 + dl] : 0;
                uint32_t c = nev > 0 ? S.ec[0] : 0u, zr = nev > 0 ? S.zs[1] : 0u;
                for (int i = 0; i < nev; ++i) {
                    const int j = i + 1 < nev ? i + 1 : i;  // operands of the next event, loaded ahead
                    const int32_t ev2 = S.ev[j * 32 + dl], rs2 = S.rs[(j + 1) * 32 + dl];
                    const uint32_t c2 = S.ec[j], zr2 = S.zs[j + 1];
                    if (k == 0 && i == 0) {  // token 0 starts the state (emulator:674-685)
                        st = ev;
                        z = 1u << 17;
                    } else {  // new maximum: rescale, then add v
                        st = mulq17_w(st, c) + ev;
                        z = ((static_cast<uint32_t>(mulq17_w(static_cast<int32_t>(z), c)) & M30) + (1u << 17)) & M30;
                    }
                    st += rs;
                    z = (z + zr) & M30;
                    ev = ev2;
                    rs = rs2;
                    c = c2;
                    zr = zr2;
                }
            } else {
                // The reference's recurrence (emulator:656-685), saturating at
                // every step, over the window's coefficients and V bytes.
                for (int tl = 0; tl < cnt; ++tl) {
                    const uint32_t cf = S.coef[tl];
                    const uint32_t cc = cf & 0x7fffffffu;
                    const uint32_t sh = S.vsh[tl];
                    const int v8 = S.vbuf[tl * 32 + dl];
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
    const AttnItemSmem S = attn_item_carve(item_smem);
    const int item = blockIdx.x, h = item / kAttnParts, part = item % kAttnParts;
    const int pos = *a.pos_ptr;
    if (pos < 0 || pos >= a.stride) {
        if (threadIdx.x == 0) atomicOr(a.err, kErrArg);
        return;
    }
    attn_item(a, S, h, part, static_cast<int>(threadIdx.x), [] {}, [](int) {});
}

__host__ __device__ constexpr size_t attn_items_smem_bytes() { return kAttnItemBytes; }

}  // namespace i4d
