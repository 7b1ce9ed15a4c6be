// i4d_token.cuh -- the whole decode step as one persistent kernel.
//
// Replaces the 4-CU control plane and the per-PE token schedule of the
// reference (int4_decoder_multikernel.cpp:70-424, int4_decoder_controller.cpp
// :138-234): one cooperative launch per token, one CTA per SM.  In every CTA
// a producer warp streams the CTA's share of ALL the token's weights (each
// GEMV stage's unit range of the CTA's bank, layer after layer, then the LM
// head) through a shared-memory ring with 1-D bulk copies; it never waits on
// activations, so HBM keeps streaming across the dependency points.  Sixteen
// consumer warps run the stages in order:
//   QKV GEMV -> attention (128 items: head x 32-dim part) -> O GEMV
//   (+ residual, RMS) -> GATE/UP GEMV (+ SwiGLU) -> DOWN GEMV (+ residual,
//   RMS) ... -> LM head,
// waiting between stages on readiness counters in global memory.  The
// arithmetic is the per-stage kernels' (i4d_linear.cuh, i4d_attention.cuh),
// bit-exact with the reference emulator.
//
// All CTAs are co-resident (cooperative launch), so the counter waits always
// end; each wait is still bounded: on timeout it raises the error word and an
// abort flag that makes every other wait return at once, so the kernel always
// terminates.
#pragma once

#include "i4d_attention.cuh"
#include "i4d_attn_item.cuh"
#include "i4d_device.cuh"
#include "i4d_expf.cuh"
#include "i4d_linear.cuh"

namespace i4d {

constexpr int kTokWarps = 18;                // consumer warps (GEMV units, attention item)
constexpr int kTokThreads = 32 * (1 + kTokWarps);
constexpr int kTokRing = 40;               // ring capacity in chunks of kChunkBytes
constexpr int kTokCpc = 4;                 // chunks per bulk copy (16,896 B: streams near the HBM peak)
constexpr int kTokSlots = kTokRing / kTokCpc;  // ring slots, one copy each
constexpr int kTokSlotBytes = kTokCpc * kChunkBytes;
constexpr int kTokUnion = 60160;           // GEMV activations + transpose tiles, or attention scratch
// Activation record of one local G32 group (80 B): hi int8[32], lo
// uint8[32], correction int32, scale float, 8 pad bytes.  The 80-byte stride
// puts the 8 groups a warp reads at once on distinct shared-memory banks.
constexpr int kActRec = 80;
constexpr int kTokActBytes = kMaxLocalGroups * kActRec;  // 7,040
constexpr int kTileFloats = 8 * 36;                      // one warp's transpose tile
constexpr int kTokTileBytes = kTokWarps * 2 * kTileFloats * 4;
constexpr int kTokQaccBytes = 4 * 32 * 4;                 // running row sums of each quad's unit
static_assert(kTokActBytes + kTokTileBytes + kTokQaccBytes + 16 <= kTokUnion, "union region");
static_assert(kAttnItemBytes <= kTokUnion, "attention item scratch exceeds the union region");
static_assert(kTokWarps == kItemWarps, "the attention item runs on the token kernel's consumer warps");

// Global synchronisation words.  They only grow, token after token; the
// epoch word (tokens completed) sets each token's targets.  The host clears
// them, with the epoch, after a failed step.
// Stage ordinals: QKV, O, GATE/UP, DOWN of layer l are 4l .. 4l+3, the LM
// head 4L.
constexpr int kSyncAbort = 0;
constexpr int kSyncExit = 1;
constexpr int kSyncStage = 2;                   // + ordinal: CTAs whose partials of that stage are stored
constexpr int kSyncAtt = kSyncStage + 4 * 32 + 1;  // + layer: attention items finished
constexpr int kSyncEpoch = kSyncAtt + 32;
constexpr int kSyncLocal = kSyncEpoch + 1;      // + ordinal: this rank's CTAs arrived (bank-sharded groups)
constexpr int kSyncWords = kSyncLocal + 4 * 32 + 1;
constexpr int kPartialBuf = 4 * 32256;          // floats of one partial buffer [4 banks][rows]

enum TokStage : int { TS_QKV = 0, TS_O, TS_GU, TS_DOWN, TS_LOGITS };

struct TokenArgs {
    const uint8_t* w;          // GEMV layout
    size_t layer_bytes;        // bytes of one layer's four stages (all banks)
    size_t stage_off[5];       // offset of each stage inside its layer (LOGITS: absolute)
    size_t bank_bytes[5];      // one bank's region of each stage
    int layers;
    int cpb;                   // CTAs per bank held (gridDim.x == nbanks * cpb)
    int bank0, nbanks;         // banks held: [bank0, bank0 + nbanks) (all four without sharding)
    int world;                 // ranks of the bank-sharded group (1 without sharding)
    float* peer_partials[4];   // every rank's partial buffers, as mapped here ([rank]; own at [rank])
    unsigned* peer_sync[4];    // every rank's synchronisation words, as mapped here
    const unsigned* epoch;     // tokens completed by this context (counter targets are epoch based)
    // Greedy steps (emb != null): the input is row *token_in of emb, and the
    // kernel leaves the first index of the maximum logit (NaN skipped) in
    // *argmax as argmax_key(value, index).
    const float* emb;
    const int* token_in;
    unsigned long long* argmax;
    float* resid;              // [2][4096]: after residual update n, buffer n & 1 (0: token input and output)
    const float* gamma;        // [65][4096]
    float* partials;           // [2][4][32256]: stage ordinal k writes buffer k & 1
    int16_t* ao_q;             // attention output
    uint8_t* ao_e;
    float* logits;
    unsigned* sync;            // [kSyncWords]
    AttnArgs attn;             // position, RoPE, KV, LUT, coefficient scratch
    ExpfFix expf;
    unsigned* err;
    unsigned long long* trace;  // optional [gridDim.x][kTraceSlots] cycle sums, or null
    unsigned long long* timeline;  // optional [gridDim.x][kTlEvents] global-timer stamps of layer tl_layer
    int tl_layer;
};

// Cycle-sum categories of the optional trace (per CTA, summed over a token).
enum TraceSlot : int {
    TR_WAIT = 0,      // + stage (QKV, O, GATE/UP, DOWN, LM head): waiting for the stage's input
    TR_PROLOGUE = 5,  // + stage: building the stage's activations
    TR_CHUNKS = 10,   // + stage: chunk loop up to the CTA barrier
    TR_ATTN_WAIT = 15,  // attention item: waiting for the QKV partials
    TR_ATTN,          // attention item: everything else
    TR_RING_FULL,     // producer: blocked on a full ring
    TR_TOTAL,         // consumer: whole kernel
    TR_ARRIVE,        // + stage: thread 0's release fence and counter arrival after the stage
    TR_W_DATA = TR_ARRIVE + 5,        // + 4 * stage, per consumer warp (summed over warps): waiting for ring data
    TR_W_SLOT,        // + 4 * stage, per warp: waiting for the quad's row chains
    TR_W_COMPUTE,     // + 4 * stage, per warp: chunk arithmetic
    TR_W_CHAIN,       // + 4 * stage, per warp: adding to the row chains and storing them
    kTraceSlots = TR_W_DATA + 20
};

// Timeline events (per CTA, one layer): stage s (QKV, O, GATE/UP, DOWN, LM
// head) at 4s + {0 begin, 1 input ready, 2 chunk loop start, 3 arrival};
// attention 20 start, 21 QKV ready, 22 end; 23 producer's first copy of the
// layer; 24 + s: copies of stage s already landed when its chunk loop
// starts (a count, not a time); 29 + s: copies of stage s; 34 + 8w + k:
// consumer warp w in the QKV stage: k < 6 time of its k-th unit grab, 6 loop
// exit, 7 number of grabs; 162 + q: GATE/UP stage, time the producer issued
// copy q of the stage (q < 24); 186 + q: time the first compute warp found
// copy q landed; 210 + k: attention item milestone k (attn_item's mark).
constexpr int kTlEvents = 34 + 8 * 16 + 48 + 8;

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Stage-level stamps are cheap (a few stores per stage) and compiled into
// both instantiations; per-chunk counters and per-warp stamps only into the
// traced one.
template <bool TR>
__device__ __forceinline__ void tl_mark(const TokenArgs& a, int layer, int event) {
    if (a.timeline && layer == a.tl_layer) a.timeline[blockIdx.x * kTlEvents + event] = global_ns();
}

template <bool TR>
__device__ __forceinline__ void trace_add(const TokenArgs& a, int slot, long long cycles) {
    if constexpr (TR)
        if (a.trace) a.trace[blockIdx.x * kTraceSlots + slot] += static_cast<unsigned long long>(cycles);
}

__host__ __device__ constexpr int stage_units(int st) {
    return st == TS_QKV ? 384 : st == TS_O ? 128 : st == TS_GU ? 704 : st == TS_DOWN ? 128 : 1008;
}
__host__ __device__ constexpr int stage_chunks(int st) { return st == TS_DOWN ? 11 : 4; }

struct TokSmem {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    uint8_t* uni;        // union region
    int* flag;           // [4] misc
    int* issued;         // [kTokSlots]: copy sequence number last issued into each slot
    double* expf_tab;    // [64]: the expf core's 2^(j/64) table
};

__host__ __device__ constexpr size_t tok_smem_bytes() {
    return static_cast<size_t>(kTokRing) * kChunkBytes + 2 * kTokSlots * 8 + kTokUnion + 16 +
           align16(kTokSlots * 4) + 64 * 8;
}
// One CTA per SM: the carve must fit the 227 KB a block may opt into, and the
// union region (GEMV activations, attention scratch) must start 16-byte aligned.
static_assert(tok_smem_bytes() <= 227 * 1024, "token kernel shared memory exceeds the per-block maximum");
static_assert((static_cast<size_t>(kTokRing) * kChunkBytes + 2 * kTokSlots * 8) % 16 == 0,
              "union region alignment");

__device__ __forceinline__ TokSmem tok_carve(uint8_t* p) {
    TokSmem s;
    s.ring = p;
    p += static_cast<size_t>(kTokRing) * kChunkBytes;
    s.full = reinterpret_cast<uint64_t*>(p);
    s.empty = s.full + kTokSlots;
    p += 2 * kTokSlots * 8;
    s.uni = p;
    p += kTokUnion;
    s.flag = reinterpret_cast<int*>(p);
    p += 16;
    s.issued = reinterpret_cast<int*>(p);
    p += align16(kTokSlots * 4);
    s.expf_tab = reinterpret_cast<double*>(p);
    return s;
}

__device__ __forceinline__ void tok_bar() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kTokWarps) : "memory"); }

__device__ __forceinline__ bool aborted(const TokenArgs& a) {
    return *reinterpret_cast<volatile unsigned*>(&a.sync[kSyncAbort]) != 0;
}

__device__ __forceinline__ void raise_abort(const TokenArgs& a, unsigned code) {
    atomicOr(a.err, code);
    atomicExch(&a.sync[kSyncAbort], 1u);
    // The other ranks of a sharded group leave their waits too.
    for (int p = 0; p < a.world; ++p)
        if (a.peer_sync[p] != a.sync) atomicExch(&a.peer_sync[p][kSyncAbort], 1u);
}

// Spins (bounded) until the counter *word has reached target; false on
// abort or timeout.  Counters only grow (mod 2^32), so the comparison is
// taken on the signed difference.  The poll is an acquire load (paired with
// the release reductions of the arrivals); a relaxed poll followed by a
// full fence was measured about 10 us per token slower.  Every spin loop of
// the kernel reads the abort word only once per 256 polls, never on the
// first miss: it is another global round trip in the poll's path.
__device__ bool wait_counter(const TokenArgs& a, const unsigned* word, unsigned target) {
    for (uint32_t it = 0;; ++it) {
        const unsigned v = a.world > 1 ? ld_acquire_sys(word) : ld_acquire_gpu(word);
        if (static_cast<int>(v - target) >= 0) return true;
        if ((it & 255u) == 255u && aborted(a)) return false;
        if (it > (1u << 24)) {
            raise_abort(a, kErrWaitFull | kErrWaitCounter);
            return false;
        }
        if (it >= 256) __nanosleep(it < 1024 ? 32 : 256);
    }
}

// mbarrier wait that also gives up when the token was aborted.
__device__ __forceinline__ bool tok_mbar_wait(const TokenArgs& a, uint64_t* bar, uint32_t parity, unsigned code) {
    if (mbar_try_wait(bar, parity)) return true;
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u && aborted(a)) return false;
        if (it > (1u << 22)) {
            raise_abort(a, code);
            return false;
        }
        if (it >= 256) __nanosleep(64);
    }
}

// ------------------------------------------------------------ GEMV stages

struct StageDesc {
    int st;               // TokStage
    int layer;
    int u0, u1;           // this CTA's units in its bank
    int bank;
    int cbase;            // global copy sequence number of the stage's first copy
    unsigned tgt_stage;   // stage counter value once every CTA (one rank) or every rank (sharded) arrived
    unsigned tgt_local;   // sharded: local counter value once every CTA of this rank arrived
    unsigned tgt_att;     // attention counter value once this rank's items finished (this token)
};

__device__ __forceinline__ int stage_ordinal(int st, int layer) { return st == TS_LOGITS ? 4 * layer : 4 * layer + st; }

__device__ __forceinline__ float* stage_partials(const TokenArgs& a, int ordinal) {
    return a.partials + static_cast<size_t>(ordinal & 1) * kPartialBuf;
}

// Input of an RMS-normalised stage (norm index n: 2l before QKV of layer l,
// 2l+1 before GATE/UP, 2L before the LM head, whose gamma is row 64 whatever
// L is), built by every CTA from the
// bank partials of the stage that just ended:
//   residual_n = residual_{n-1} + ((p0+p1)+(p2+p3))   (emulator:764, 772)
//   r = RMS reciprocal of residual_n                  (emulator:427-453)
//   x = fl(fl(residual_n * r) * gamma_n) -> G32 quantizer, this bank's columns.
// Every CTA computes the same residual; CTA 0 stores it for the next update.
// All loads (gammas, residual_{n-1}, the four partials) are issued as one
// batch after the stage wait; loading before the wait was measured slower.
// Stores one lane's INT14 activation (value q of local group lg, column
// `lane`) in split form (q = 128 * hi + lo, lo in [0, 128)), plus the group's
// offset correction (8 * the sum of its first 16 values, for the offset-binary
// low nibbles) and scale.
__device__ __forceinline__ void put_act_rec(uint8_t* acts, int lg, int lane, int q, uint32_t e8m0) {
    uint8_t* r = acts + lg * kActRec;
    reinterpret_cast<int8_t*>(r)[lane] = static_cast<int8_t>(q >> 7);
    r[32 + lane] = static_cast<uint8_t>(q & 127);
    int lo16 = lane < 16 ? q : 0;
    lo16 = __reduce_add_sync(0xffffffffu, lo16);
    if (lane == 0) *reinterpret_cast<int2*>(r + 64) = make_int2(8 * lo16, __float_as_int(e8m0_scale(e8m0)));
}

template <int G>
__device__ __forceinline__ void tok_input_rms(const TokenArgs& a, const TokSmem& s, uint8_t* acts, int bank,
                                              int norm, int prev_ordinal, float* xs, int cw, int lane) {
    constexpr int kPer = (G + kTokWarps - 1) / kTokWarps;
    constexpr int kQ = kDim / 4;                                      // float4 per vector
    constexpr int kRmsQ = (kQ + 32 * kTokWarps - 1) / (32 * kTokWarps);  // float4 per thread
    const int tid = cw * 32 + lane;
    const int gamma_row = norm == 2 * a.layers ? kGammaFinal : norm;
    float g[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int lg = cw + k * kTokWarps;
        g[k] = lg < G ? a.gamma[static_cast<size_t>(gamma_row) * kDim + bank * G * 32 + lg * 32 + lane] : 0.0f;
    }
    // Greedy steps take the token's input from the embedding table (CTA 0
    // stores it as the residual input, read again by the first update).
    const bool embed = norm == 0 && a.emb != nullptr;
    const float4* rin = reinterpret_cast<const float4*>(
        embed ? a.emb + static_cast<size_t>(*reinterpret_cast<const volatile int*>(a.token_in)) * kDim
              : a.resid + (norm == 0 ? 0 : ((norm - 1) & 1) * kDim));
    float4 xin[kRmsQ];
#pragma unroll
    for (int k = 0; k < kRmsQ; ++k) {
        const int i = tid + k * 32 * kTokWarps;
        xin[k] = i < kQ ? __ldcg(rin + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float4* rout = reinterpret_cast<float4*>(a.resid + (norm & 1) * kDim);
    const float4* P = reinterpret_cast<const float4*>(stage_partials(a, prev_ordinal));
#pragma unroll
    for (int k = 0; k < kRmsQ; ++k) {
        const int i = tid + k * 32 * kTokWarps;
        if (i >= kQ) break;
        float4 x = xin[k];
        if (norm > 0) {
            const float4 p0 = __ldcg(P + i), p1 = __ldcg(P + kQ + i);
            const float4 p2 = __ldcg(P + 2 * kQ + i), p3 = __ldcg(P + 3 * kQ + i);
            x.x = __fadd_rn(x.x, __fadd_rn(__fadd_rn(p0.x, p1.x), __fadd_rn(p2.x, p3.x)));
            x.y = __fadd_rn(x.y, __fadd_rn(__fadd_rn(p0.y, p1.y), __fadd_rn(p2.y, p3.y)));
            x.z = __fadd_rn(x.z, __fadd_rn(__fadd_rn(p0.z, p1.z), __fadd_rn(p2.z, p3.z)));
            x.w = __fadd_rn(x.w, __fadd_rn(__fadd_rn(p0.w, p1.w), __fadd_rn(p2.w, p3.w)));
            if (blockIdx.x == 0) __stcg(rout + i, x);
        } else if (embed && blockIdx.x == 0) {
            __stcg(rout + i, x);
        }
        reinterpret_cast<float4*>(xs)[i] = x;
    }
    tok_bar();
    // RMS reciprocal in the reference's order (emulator:427-447): warp b sums
    // bank b, lane s its slot s (elements b*1024 + s + 8i, i = 0..127, in
    // order), then the bank total is ((0 + s0) + s1) ... + s7.  One bank per
    // warp keeps the eight lanes' loads on distinct shared-memory banks (a
    // single warp over all four banks met a 4-way conflict on every load).
    float* bank_total = xs + kDim;
    if (cw < 4 && lane < 8) {
        const float* base = xs + cw * 1024 + lane;
        float acc = 0.0f;
#pragma unroll 32
        for (int i = 0; i < 128; ++i) {
            const float v = base[i * 8];
            acc = __fadd_rn(acc, __fmul_rn(v, v));
        }
        float total = 0.0f;
#pragma unroll
        for (int sl = 0; sl < 8; ++sl) total = __fadd_rn(total, __shfl_sync(0xffu, acc, sl));
        if (lane == 0) bank_total[cw] = total;
    }
    tok_bar();
    const float sum = __fadd_rn(__fadd_rn(bank_total[0], bank_total[1]), __fadd_rn(bank_total[2], bank_total[3]));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(sum, 1.0f / 4096.0f), 1.0e-5f)));
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int lg = cw + k * kTokWarps;
        if (lg < G) {
            uint32_t e8;
            const float v = __fmul_rn(__fmul_rn(xs[bank * G * 32 + lg * 32 + lane], r), g[k]);
            const int q = quantize_g32_lane(v, &e8);
            put_act_rec(acts, lg, lane, q, e8);
        }
    }
}

// Input of DOWN: SwiGLU of this bank's 2816 FFN columns from the GATE/UP
// partials (gate rows [0, 11264), up rows [11264, 22528)), then the G32
// quantizer (emulator:716-722, 769-770).
__device__ __forceinline__ void tok_input_swiglu(const TokenArgs& a, const TokSmem& s, uint8_t* acts, int bank,
                                                 int layer, int cw, int lane) {
    constexpr int G = 88;
    constexpr int kPer = (G + kTokWarps - 1) / kTokWarps;
    constexpr int kRows = 22528;
    const float* P = stage_partials(a, stage_ordinal(TS_GU, layer));
    float gv[kPer], uv[kPer], sw[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int lg = min(cw + k * kTokWarps, G - 1);  // warps with 5 groups repeat their last one
        const int f = bank * G * 32 + lg * 32 + lane;
        gv[k] = combine4(P, kRows, f);
        uv[k] = combine4(P, kRows, kFfn + f);
    }
    // expf(-g) of every value first; the rare near-midpoint results then take
    // the exception table, one lookup per lane at a time, so that a warp pays
    // one table round trip for its first flagged values (taken value by value,
    // every flagged k cost a warp one more trip).
    float e[kPer];
    int nt[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) e[k] = i4d_expf_core2(-gv[k], s.expf_tab, &nt[k]);
    int pending = 0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) pending |= nt[k] << k;
    while (__any_sync(0xffffffffu, pending != 0)) {
        const int k0 = pending ? __ffs(pending) - 1 : -1;
        float xf = 0.0f, yf = 0.0f;
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            if (k == k0) {
                xf = -gv[k];
                yf = e[k];
            }
        if (k0 >= 0) {
            const float fixed = expf_table_fix(xf, yf, a.expf);
#pragma unroll
            for (int k = 0; k < kPer; ++k)
                if (k == k0) e[k] = fixed;
            pending &= pending - 1;
        }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) sw[k] = swiglu_e(gv[k], uv[k], e[k]);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int lg = cw + k * kTokWarps;
        if (lg < G) {
            uint32_t e8;
            const int q = quantize_g32_lane(sw[k], &e8);
            put_act_rec(acts, lg, lane, q, e8);
        }
    }
}

// Input of O: the attention output of this bank's 8 heads.
__device__ __forceinline__ void tok_input_attention(const TokenArgs& a, uint8_t* acts, int bank, int cw, int lane) {
    constexpr int G = 32;
    constexpr int kPer = (G + kTokWarps - 1) / kTokWarps;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int lg = cw + k * kTokWarps;
        if (lg >= G) break;
        const int q = __ldcg(a.ao_q + bank * 1024 + lg * 32 + lane);
        const uint32_t e8 = __ldcg(a.ao_e + bank * 32 + lg);
        put_act_rec(acts, lg, lane, q, e8);
    }
}

// Waits until copy `cp` is issued into `slot` and has landed.
__device__ __forceinline__ void tok_wait_copy(const TokenArgs& a, const TokSmem& s, int cp, int slot) {
    for (uint32_t it = 0; *reinterpret_cast<volatile int*>(&s.issued[slot]) != cp; ++it) {
        if ((it & 255u) == 255u && aborted(a)) break;
        if (it > (1u << 24)) {
            raise_abort(a, kErrWaitFull | kErrWaitCopy);
            break;
        }
        if (it >= 256) __nanosleep(32);
    }
    tok_mbar_wait(a, &s.full[slot], static_cast<uint32_t>((cp / kTokSlots) & 1), kErrWaitFull | kErrWaitCopy);
}

struct WarpTimes {
    long long data = 0, comp = 0, chain_wait = 0, chain = 0;
};

// Chain hand-off words of a quad (shared memory): acquire / release at CTA scope.
__device__ __forceinline__ int ld_acquire_cta_s(const int* p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta_s(int* p, int v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

constexpr int kQuads = 4;                 // GEMV warps: kQuads x 4 (warps 16, 17 take no units)

// Unit loop of a GEMV stage.  A unit is 32 output rows x this bank's local
// columns (C chunks of 256 columns).  Quad q (warps 4q .. 4q+3) takes units
// q, q + 4, ... of the CTA's range; over the quad's stream of chunks
// s = 0, 1, ... (unit s / C, chunk s % C), warp j takes s = j, j + 4, ...,
// so the four chunks of a ring copy are worked on at once and a slot is held
// for about one chunk's time.
//
// Per chunk, lane (g = lane % 8, rb = lane / 8) computes the exact G32 dots
// of group g for rows 8rb .. 8rb+7 and their contributions
// fl(float(dot) * fl(ws * as)); an 8 x 8 transpose through the warp's
// shared-memory tile gives lane (g, rb) row 8rb+g's contributions of the
// chunk's 8 groups in column order.  The row's serial FP32 chain over the
// bank's groups (emulator:216-264) then passes through the quad in chunk
// order: the warp of chunk s waits until the quad's chain word reads s,
// adds its 8 values to the running sums of the unit's 32 rows (or starts
// them from +0.0f at chunk 0), and stores them back -- or, at the unit's
// last chunk, stores the bank partials -- before releasing s + 1.  Only the
// 8 additions wait; the dots of the next chunk do not.
template <int C, bool TR>
__device__ __forceinline__ void tok_units(const TokenArgs& a, const TokSmem& s, const StageDesc& d,
                                          const uint8_t* acts, float* tile, float* qacc, int* qflag,
                                          float* partials, int cw, int lane, WarpTimes& wt) {
    const int quad = cw >> 2, j = cw & 3;
    const int g = lane & 7, rb = lane >> 3, g128 = g >> 2;
    const int row = 8 * rb + g;  // the row this lane chains
    const int nunits = d.u1 - d.u0;
    const int nchunks = nunits * C;
    const int nq = nunits > quad ? (nunits - quad + kQuads - 1) / kQuads : 0;  // this quad's units
    const int rows_total = stage_units(d.st) * 32;
    const int ord = stage_ordinal(d.st, d.layer);
    const bool tr = TR && a.trace != nullptr;
    int par = 0;
    // With 4 chunks per unit a warp always takes chunk j: its group's
    // activations stay in registers for the whole stage.
    uint4 h0, h1, l0, l1;
    int2 cs;
    auto load_acts = [&](int c) {
        const uint8_t* ar = acts + (c * 8 + g) * kActRec;
        h0 = *reinterpret_cast<const uint4*>(ar);
        h1 = *reinterpret_cast<const uint4*>(ar + 16);
        l0 = *reinterpret_cast<const uint4*>(ar + 32);
        l1 = *reinterpret_cast<const uint4*>(ar + 48);
        cs = *reinterpret_cast<const int2*>(ar + 64);
    };
    if (C == 4) load_acts(j);
#pragma unroll 1
    for (int sq = j; sq < nq * C; sq += 4) {
        const long long c0 = tr ? clock64() : 0;
        const int us = sq / C, c = sq - us * C;
        const int k = quad + kQuads * us;  // unit index in the CTA's range
        const int i = k * C + c;           // chunk index in the CTA's stage stream
        const int cp = d.cbase + i / kTokCpc;
        const int slot = cp % kTokSlots;
        if (C != 4) load_acts(c);
        tok_wait_copy(a, s, cp, slot);
        const long long c1 = tr ? clock64() : 0;
        const uint8_t* ch = s.ring + static_cast<size_t>(slot) * kTokSlotBytes + (i % kTokCpc) * kChunkBytes;
        uint4 wv[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) wv[q] = *reinterpret_cast<const uint4*>(ch + chunk_piece(rb * 8 + q, g));
        // Scales of rows 8rb .. 8rb+7: int16 at (row * 2 + g128) * 2.
        const uint4 sa = *reinterpret_cast<const uint4*>(ch + rb * 32);
        const uint4 sb = *reinterpret_cast<const uint4*>(ch + rb * 32 + 16);
        __syncwarp();
        if (lane == 0) {
            // The empty barrier counts kTokCpc chunk releases; the last chunk
            // of a short final copy also releases the chunks the copy lacks.
            uint32_t rel = 1;
            if (i == nchunks - 1 && nchunks % kTokCpc != 0) rel = kTokCpc - nchunks % kTokCpc + 1;
            mbar_arrive_cnt(&s.empty[slot], rel);
        }
        const float as = __int_as_float(cs.y);
        const uint32_t sw[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
        float cv[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int16_t raw = static_cast<int16_t>(g128 ? (sw[q] >> 16) : (sw[q] & 0xffffu));
            const float ws = __fmul_rn(static_cast<float>(raw), 1.0f / 32768.0f);
            const int dot = group_dot_r(wv[q], h0, h1, l0, l1, cs.x);
            cv[q] = __fmul_rn(static_cast<float>(dot), __fmul_rn(ws, as));
        }
        // Transpose: tile[group][row] with a 36-float group stride (both the
        // 16-byte stores and the column reads hit every bank once per phase).
        float* T = tile + par * kTileFloats;
        *reinterpret_cast<float4*>(T + 36 * g + 8 * rb) = make_float4(cv[0], cv[1], cv[2], cv[3]);
        *reinterpret_cast<float4*>(T + 36 * g + 8 * rb + 4) = make_float4(cv[4], cv[5], cv[6], cv[7]);
        __syncwarp();
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = T[36 * q + row];
        par ^= 1;  // the other tile: its reads finished before this chunk's __syncwarp
        const long long c2 = tr ? clock64() : 0;
        // The chain: wait for chunk sq - 1 of the quad's stream.
        for (uint32_t it = 0; ld_acquire_cta_s(qflag) != sq; ++it) {
            if ((it & 255u) == 255u && aborted(a)) break;
            if (it > (1u << 24)) {
                raise_abort(a, kErrWaitFull | kErrWaitUnit);
                break;
            }
            if (it >= 64) __nanosleep(32);
        }
        const long long c3 = tr ? clock64() : 0;
        float acc = c == 0 ? 0.0f : qacc[row];
#pragma unroll
        for (int q = 0; q < 8; ++q) acc = __fadd_rn(acc, t[q]);
        if (c == C - 1) {
            const size_t off = static_cast<size_t>(d.bank) * rows_total + static_cast<size_t>(d.u0 + k) * 32 + row;
            partials[off] = acc;
            // Bank sharding: every rank receives every bank's partials.
            for (int p = 0; p < a.world; ++p)
                if (a.peer_partials[p] != a.partials) a.peer_partials[p][(ord & 1) * kPartialBuf + off] = acc;
        } else {
            qacc[row] = acc;
        }
        __syncwarp();
        if (lane == 0) st_release_cta_s(qflag, sq + 1);
        if (tr) {
            wt.data += c1 - c0;
            wt.comp += c2 - c1;
            wt.chain_wait += c3 - c2;
            wt.chain += clock64() - c3;
        }
    }
}

// The stage, attention and LM-head functions are inlined into k_token on
// purpose.  Out of line, they receive the shared-memory carve and the stage
// descriptor through references to the caller's stack: the carve's pointers
// are then generic (not provably shared), and every inline-asm memory clobber
// (mbarrier operations, fences) reloads them from local memory, which misses
// the 28 KB of L1 left beside 225 KB of shared memory.  That cost about
// 500 cycles per shared-memory step of the chunk loop; inlined, the token
// step runs about 1.4x faster.
template <int C, bool TR>
__device__ __forceinline__ void tok_gemv_stage(const TokenArgs& a, const TokSmem& s, const StageDesc& d, int cw,
                                            int lane) {
    constexpr int G = C * 8;
    static_assert(G * kActRec <= kTokActBytes, "activation records");
    uint8_t* acts = s.uni;
    float* tiles = reinterpret_cast<float*>(s.uni + kTokActBytes);
    float* qacc = reinterpret_cast<float*>(s.uni + kTokActBytes + kTokTileBytes);
    int* qflag = reinterpret_cast<int*>(s.uni + kTokActBytes + kTokTileBytes + kTokQaccBytes);
    const int tid = cw * 32 + lane;
    const int ord = stage_ordinal(d.st, d.layer);
    const int tl_layer = d.st == TS_LOGITS ? a.tl_layer : d.layer;  // the LM head is recorded with any layer
    tl_mark<TR>(a, tl_layer, 4 * d.st);
    const long long t_begin = clock64();

    // Input readiness: the previous stage's partials from every CTA, or the
    // attention items of this layer.
    if (tid == 0) {
        if (d.st == TS_O) wait_counter(a, &a.sync[kSyncAtt + d.layer], d.tgt_att);
        else if (ord > 0) wait_counter(a, &a.sync[kSyncStage + ord - 1], d.tgt_stage);
    }
    if (tid < kQuads) qflag[tid] = 0;  // chunks chained by each quad in this stage
    tok_bar();
    const long long t_ready = clock64();
    if (tid == 0) tl_mark<TR>(a, tl_layer, 4 * d.st + 1);
    if (d.st == TS_O) {
        tok_input_attention(a, acts, d.bank, cw, lane);
    } else if (d.st == TS_DOWN) {
        tok_input_swiglu(a, s, acts, d.bank, d.layer, cw, lane);
    } else {
        const int norm = d.st == TS_QKV ? 2 * d.layer : d.st == TS_GU ? 2 * d.layer + 1 : 2 * d.layer;
        if constexpr (G == 32) tok_input_rms<32>(a, s, acts, d.bank, norm, ord - 1, tiles, cw, lane);
    }
    tok_bar();
    const long long t_loop = clock64();
    if (tid == 0) {
        tl_mark<TR>(a, tl_layer, 4 * d.st + 2);
        if (TR && a.timeline && tl_layer == a.tl_layer) {
            const int ncp = ((d.u1 - d.u0) * C + kTokCpc - 1) / kTokCpc;
            int landed = 0;
            for (int q = 0; q < ncp; ++q) {
                const int cp = d.cbase + q, sl = cp % kTokSlots;
                if (*reinterpret_cast<volatile int*>(&s.issued[sl]) == cp &&
                    mbar_test_wait(&s.full[sl], static_cast<uint32_t>((cp / kTokSlots) & 1)))
                    ++landed;
            }
            a.timeline[blockIdx.x * kTlEvents + 24 + d.st] = static_cast<unsigned long long>(landed);
            a.timeline[blockIdx.x * kTlEvents + 29 + d.st] = static_cast<unsigned long long>(ncp);
        }
    }

    float* partials = stage_partials(a, ord);
    const bool tr = TR && a.trace != nullptr;
    WarpTimes wt;
    if (cw < 4 * kQuads)
        tok_units<C, TR>(a, s, d, acts, tiles + cw * 2 * kTileFloats, qacc + (cw >> 2) * 32, qflag + (cw >> 2),
                         partials, cw, lane, wt);
    // Release: the CTA barrier orders every warp's partial stores before
    // thread 0's release arrival (the grid-sync pattern).
    tok_bar();
    const long long t_epi = clock64();
    if (tid == 0) {
        tl_mark<TR>(a, tl_layer, 4 * d.st + 3);
        // Arrive with a release reduction.  One rank: on the stage counter.
        // Bank-sharded: on this rank's local counter at system scope (which
        // also covers the partials this CTA stored in peer memory); the
        // rank's last CTA, having acquired every local arrival, then makes
        // the rank's single arrival on every rank's stage counter -- G remote
        // reductions per stage instead of one per CTA and rank.
        if (a.world > 1) {
            const unsigned old = atom_add_acq_rel_sys(&a.sync[kSyncLocal + ord], 1u);
            if (old + 1u == d.tgt_local)
                for (int p = 0; p < a.world; ++p) red_release_sys(&a.peer_sync[p][kSyncStage + ord], 1u);
        } else {
            red_release_gpu(&a.sync[kSyncStage + ord], 1u);
        }
        trace_add<TR>(a, TR_ARRIVE + d.st, clock64() - t_epi);
        trace_add<TR>(a, TR_WAIT + d.st, t_ready - t_begin);
        trace_add<TR>(a, TR_PROLOGUE + d.st, t_loop - t_ready);
        trace_add<TR>(a, TR_CHUNKS + d.st, t_epi - t_loop);
    }
    // Per-warp sums after the arrival, so the release does not wait for them.
    if (tr && lane == 0) {
        unsigned long long* t = a.trace + blockIdx.x * kTraceSlots;
        atomicAdd(t + TR_W_DATA + 4 * d.st, static_cast<unsigned long long>(wt.data));
        atomicAdd(t + TR_W_COMPUTE + 4 * d.st, static_cast<unsigned long long>(wt.comp));
        atomicAdd(t + TR_W_SLOT + 4 * d.st, static_cast<unsigned long long>(wt.chain_wait));
        atomicAdd(t + TR_W_CHAIN + 4 * d.st, static_cast<unsigned long long>(wt.chain));
    }
}
// Key of a logit for the greedy argmax: larger keys win; equal values favour
// the smaller index (the first maximum, as emulator:1428-1438 and
// decode_host.cpp:703-717 scan); -0.0 counts as +0.0; NaN never wins (key 0).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    if (v != v) return 0ull;
    unsigned b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | (0xffffffffu - static_cast<unsigned>(idx));
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long y = __shfl_xor_sync(0xffffffffu, k, o);
        k = y > k ? y : k;
    }
    return k;
}

// First index of the maximum of x[0, n) (NaN skipped; -1 encoded as key 0):
// the argmax of the greedy step, as an op-level test hook.  One block.
__global__ void __launch_bounds__(1024) k_argmax(const float* x, int n, unsigned long long* out) {
    __shared__ unsigned long long w[32];
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = argmax_key(x[i], i);
        best = k > best ? k : best;
    }
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) w[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        unsigned long long v = threadIdx.x < (blockDim.x >> 5) ? w[threadIdx.x] : 0ull;
        v = warp_max_u64(v);
        if (threadIdx.x == 0) *out = v;
    }
}

// Logits: every CTA combines a slice of the LM-head rows once all partials
// are stored ((p0+p1)+(p2+p3), emulator sharded_gemv_4pe).
__device__ __forceinline__ void tok_logits(const TokenArgs& a, unsigned tgt_stage, int cw, int lane) {
    const int tid = cw * 32 + lane;
    const int ord = stage_ordinal(TS_LOGITS, a.layers);
    if (tid == 0) wait_counter(a, &a.sync[kSyncStage + ord], tgt_stage);
    tok_bar();
    const float* P = stage_partials(a, ord);
    const int r0 = static_cast<int>((static_cast<long long>(blockIdx.x) * kPVocab) / gridDim.x);
    const int r1 = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * kPVocab) / gridDim.x);
    unsigned long long best = 0ull;
    for (int r = r0 + tid; r < r1; r += 32 * kTokWarps) {
        const float v = combine4(P, kPVocab, r);
        a.logits[r] = v;
        if (r < kVocab) {
            const unsigned long long k = argmax_key(v, r);
            best = k > best ? k : best;
        }
    }
    if (a.emb) {  // greedy step: the CTA's best, then one atomic per warp
        best = warp_max_u64(best);
        if (lane == 0 && best != 0ull) atomicMax(a.argmax, best);
    }
}

// ------------------------------------------------------------ attention item

// Attention of one (head, 32-dimension part) item after the QKV stage
// (i4d_attn_item.cuh); thread 0 then publishes the item's outputs to the O
// stage with a release arrival on the layer's attention counter.
template <bool TR>
__device__ __forceinline__ void tok_attention(const TokenArgs& ta, const TokSmem& s, int layer, int item, int cw,
                                              int lane, unsigned tgt_qkv) {
    AttnArgs a = ta.attn;
    a.layer = layer;
    a.partials = stage_partials(ta, stage_ordinal(TS_QKV, layer));
    a.out_q = ta.ao_q;
    a.out_e = ta.ao_e;
    const int tid = cw * 32 + lane;
    const AttnItemSmem S = attn_item_carve(s.uni);
    const long long t_a0 = clock64();
    long long t_a1 = t_a0;
    if (tid == 0) tl_mark<TR>(ta, layer, 20);
    attn_item(a, S, item / kAttnParts, item % kAttnParts, tid,
              [&] {
                  wait_counter(ta, &ta.sync[kSyncStage + stage_ordinal(TS_QKV, layer)], tgt_qkv);
                  t_a1 = clock64();
                  tl_mark<TR>(ta, layer, 21);
              },
              [&](int k) { tl_mark<TR>(ta, layer, 210 + k); });
    __syncwarp();
    if (tid == 0) {
        red_release_gpu(&ta.sync[kSyncAtt + layer], 1u);
        trace_add<TR>(ta, TR_ATTN_WAIT, t_a1 - t_a0);
        trace_add<TR>(ta, TR_ATTN, clock64() - t_a1);
        tl_mark<TR>(ta, layer, 22);
    }
}

// ---------------------------------------------------------------- kernel

// This CTA's units [u0, u1) of a stage in its bank.
__device__ __forceinline__ void stage_urange(const TokenArgs& a, int c, int st, int* u0, int* u1) {
    const int U = stage_units(st);
    *u0 = static_cast<int>((static_cast<long long>(c) * U) / a.cpb);
    *u1 = static_cast<int>((static_cast<long long>(c + 1) * U) / a.cpb);
}

// Position in the CTA's sequence of weight copies: layer, stage, first chunk
// of the copy, chunks in the stage and the stage's source bytes.
struct CopyCursor {
    int l, st, i, n;
    const uint8_t* src;
};

__device__ __forceinline__ void cursor_stage(const TokenArgs& a, int bank, int c, CopyCursor& k) {
    int u0, u1;
    stage_urange(a, c, k.st, &u0, &u1);
    const int C = stage_chunks(k.st);
    k.i = 0;
    k.n = (u1 - u0) * C;
    k.src = a.w + (k.st == TS_LOGITS ? a.stage_off[TS_LOGITS] : k.l * a.layer_bytes + a.stage_off[k.st]) +
            static_cast<size_t>(bank) * a.bank_bytes[k.st] + static_cast<size_t>(u0) * C * kChunkBytes;
}

__device__ __forceinline__ bool cursor_valid(const TokenArgs& a, const CopyCursor& k) { return k.l <= a.layers; }

__device__ __forceinline__ void cursor_begin(const TokenArgs& a, int bank, int c, CopyCursor& k) {
    k.l = 0;
    k.st = a.layers == 0 ? TS_LOGITS : TS_QKV;
    cursor_stage(a, bank, c, k);
}

__device__ __forceinline__ void cursor_advance(const TokenArgs& a, int bank, int c, CopyCursor& k) {
    k.i += kTokCpc;
    while (k.l <= a.layers && k.i >= k.n) {
        if (k.st == TS_LOGITS) {
            k.l = a.layers + 1;
            return;
        }
        if (k.st == TS_DOWN) {
            ++k.l;
            k.st = k.l == a.layers ? TS_LOGITS : TS_QKV;
        } else {
            ++k.st;
        }
        cursor_stage(a, bank, c, k);
    }
}

template <bool TR>
__global__ void __launch_bounds__(kTokThreads, 1) k_token(const __grid_constant__ TokenArgs a) {
    extern __shared__ __align__(128) uint8_t tok_smem_raw[];
    TokSmem s = tok_carve(tok_smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lbank = blockIdx.x / a.cpb, c = blockIdx.x % a.cpb;  // bank index among the banks held
    auto urange = [&](int st, int* u0, int* u1) {
        const int U = stage_units(st);
        *u0 = static_cast<int>((static_cast<long long>(c) * U) / a.cpb);
        *u1 = static_cast<int>((static_cast<long long>(c + 1) * U) / a.cpb);
    };
    if (threadIdx.x == 0) {
        for (int i = 0; i < kTokSlots; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kTokCpc);
            s.issued[i] = -1;
        }
        mbar_fence_init();
    }
    if (threadIdx.x < 64) s.expf_tab[threadIdx.x] = g_expf_table[threadIdx.x];
    __syncthreads();

    if (warp == 0) {
        // Producer: this CTA's chunks of every stage, in consumption order.
        if (lane == 0) {
            int slot = 0, issued = 0;
            uint32_t phase = 0;
            CopyCursor cur;
            // Weights are read once per token: evict them first, so the
            // partials, residual and counters of the stage handoffs stay in L2.
            const uint64_t pol_first = l2_policy_evict_first();
            cursor_begin(a, lbank, c, cur);

            while (cursor_valid(a, cur)) {
                const int cnt = min(kTokCpc, cur.n - cur.i);
                if (issued >= kTokSlots) {
                    const long long t0 = TR && a.trace ? clock64() : 0;
                    if (!tok_mbar_wait(a, &s.empty[slot], phase ^ 1u, kErrWaitEmpty)) break;
                    if (TR && a.trace) trace_add<TR>(a, TR_RING_FULL, clock64() - t0);
                }
                if (cur.i == 0 && cur.st == TS_QKV) tl_mark<TR>(a, cur.l, 23);
                if (TR && a.timeline && cur.st == TS_GU && cur.l == a.tl_layer && cur.i / kTokCpc < 24)
                    a.timeline[blockIdx.x * kTlEvents + 162 + cur.i / kTokCpc] = global_ns();
                publish_issued(&s.issued[slot], issued);
                mbar_arrive_expect_tx(&s.full[slot], cnt * kChunkBytes);
                bulk_g2s_hint(s.ring + static_cast<size_t>(slot) * kTokSlotBytes,
                              cur.src + static_cast<size_t>(cur.i) * kChunkBytes, cnt * kChunkBytes, &s.full[slot],
                              pol_first);
                ++issued;
                if (++slot == kTokSlots) {
                    slot = 0;
                    phase ^= 1u;
                }
                cursor_advance(a, lbank, c, cur);
            }
            // Never leave with copies in flight: wait for the last ones to land.
            for (int k = 0; k < kTokSlots && k < issued; ++k) {
                const int g = issued - 1 - k;
                const int sl = g % kTokSlots;
                for (uint32_t it = 0; !mbar_try_wait(&s.full[sl], static_cast<uint32_t>((g / kTokSlots) & 1)); ++it) {
                    if (it > (1u << 22)) {
                        atomicOr(a.err, kErrWaitFull | kErrWaitDrain);
                        break;
                    }
                    __nanosleep(64);
                }
            }
        }
        return;
    }

    const int cw = warp - 1;
    const int tid = cw * 32 + lane;
    const long long t_kernel = clock64();
    if (a.emb && blockIdx.x == 0 && tid == 0) *a.argmax = 0ull;  // read by the host after the step
    StageDesc d;
    d.bank = a.bank0 + lbank;
    // Counter targets of this token: counters only grow -- a stage counter by
    // grid arrivals per token (one rank) or by world rank arrivals (sharded,
    // with the local counter growing by grid), the attention counter by this
    // rank's items per layer.
    const unsigned epoch = *reinterpret_cast<const volatile unsigned*>(a.epoch);
    const int att_items = kAttnItems / a.world;
    d.tgt_stage = (epoch + 1u) * (a.world > 1 ? static_cast<unsigned>(a.world) : gridDim.x);
    d.tgt_local = (epoch + 1u) * gridDim.x;
    d.tgt_att = (epoch + 1u) * static_cast<unsigned>(att_items);
    d.cbase = 0;
    for (int l = 0; l <= a.layers; ++l) {
        for (int st = TS_QKV; st <= TS_DOWN; ++st) {
            const int stage = l == a.layers ? TS_LOGITS : st;
            if (l == a.layers && st != TS_QKV) break;
            d.st = stage;
            d.layer = l;
            urange(stage, &d.u0, &d.u1);
            if (stage == TS_DOWN) tok_gemv_stage<11, TR>(a, s, d, cw, lane);
            else tok_gemv_stage<4, TR>(a, s, d, cw, lane);
            d.cbase += ((d.u1 - d.u0) * stage_chunks(stage) + kTokCpc - 1) / kTokCpc;
            if (stage == TS_QKV && l < a.layers) {
                if (blockIdx.x < att_items)
                    tok_attention<TR>(a, s, l, a.bank0 * kLocalHeads * kAttnParts + blockIdx.x, cw, lane, d.tgt_stage);
                tok_bar();
            }
        }
    }
    tok_logits(a, d.tgt_stage, cw, lane);
    // The last CTA to finish advances the epoch: the counters are never
    // cleared (a faster rank may already be arriving for the next token), the
    // next token's targets are one token's arrivals higher.
    tok_bar();
    if (tid == 0) {
        trace_add<TR>(a, TR_TOTAL, clock64() - t_kernel);
        __threadfence();
        const unsigned old = atomicAdd(&a.sync[kSyncExit], 1u);
        if (old + 1 == (epoch + 1u) * gridDim.x) {
            __threadfence();
            atomicAdd(const_cast<unsigned*>(a.epoch), 1u);
        }
    }
}

}  // namespace i4d
