// i4d_device.cuh -- device helpers shared by the decode kernels (sm_100a).
//
// Every floating-point operation that the reference rounds separately is
// written with an explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn,
// __fdiv_rn, __fsqrt_rn) and the library is compiled with -fmad=false, so no
// multiply-add is ever contracted (the emulator forces the same with volatile
// temporaries, software_sim/llama2_decoder_sw_emulator.cpp:154-162).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace i4d {

constexpr int kDim = 4096;
constexpr int kFfn = 11264;
constexpr int kPVocab = 32256;
constexpr int kVocab = 32000;
constexpr int kHeads = 32;
constexpr int kHeadDim = 128;
constexpr int kLocalHeads = 8;
constexpr int kGammaFinal = 64;      // row of the final norm's gamma in the [65][4096] table
constexpr int kChunkBytes = 4224;     // 32 rows x 256 columns: 128 B scales + 4096 B weights
constexpr int kChunkScaleBytes = 128;
constexpr int kConsumerWarps = 8;
constexpr int kLinearThreads = 32 * (1 + kConsumerWarps);
constexpr int kMaxLocalGroups = 88;   // DOWN: 2816 local columns
constexpr int kCounterSlots = 4096;
constexpr int kCounterLevel2 = 4095;

// Device error word bits.
constexpr unsigned kErrWaitFull = 1u;
constexpr unsigned kErrWaitEmpty = 2u;
constexpr unsigned kErrArg = 4u;
// Which bounded wait gave up (token kernel): stage counter, ring copy,
// contribution slot, unit completion, attention tile, producer drain.
constexpr unsigned kErrWaitCounter = 8u;
constexpr unsigned kErrWaitCopy = 16u;
constexpr unsigned kErrWaitSlot = 32u;
constexpr unsigned kErrWaitUnit = 64u;
constexpr unsigned kErrWaitTile = 128u;
constexpr unsigned kErrWaitDrain = 256u;

// ------------------------------------------------------------------ PTX

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of a phase's completion.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: after ~2^22 polls (well over a second) it records `code` in
// the error word and returns false; the caller carries on so that no other
// warp is left waiting at a barrier.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (i > 32) __nanosleep(256);
    }
    atomicOr(err, code);
    return false;
}

// 1-D bulk copy global -> shared, completing on an mbarrier (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of global memory into L2 (no destination and no completion
// to wait for); address and size multiples of 16 bytes.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 16-byte asynchronous copy global -> shared (no registers on the way);
// both addresses 16-byte aligned.  Completion: cp_async_commit, then
// cp_async_wait_all in the issuing thread, then a barrier for the others.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// L2 policy for data read once (weights): evict before anything else.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Release/acquire counter operations of the grid hand-offs.  A release
// reduction after a CTA barrier orders every thread's earlier stores of the
// CTA before the counter update (the barrier makes them causally precede it).
__device__ __forceinline__ void red_release_gpu(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel_sys(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.sys.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Ring-slot handshake.  Before issuing chunk c into a slot the producer
// records c in issued[slot]; the consumer of chunk c waits for that record
// before its parity wait on the slot's full barrier.  Parity alone cannot
// tell apart phases that are two apart: without the record, a consumer of
// chunk c + NS could pass while chunk c is still landing and free the slot
// early, letting a second copy into a slot that still has one in flight.
__device__ __forceinline__ void publish_issued(int* issued, int c) {
    *reinterpret_cast<volatile int*>(issued) = c;
}

__device__ __forceinline__ bool wait_issued(const int* issued, int c, unsigned* err) {
    for (uint32_t it = 0; *reinterpret_cast<const volatile int*>(issued) != c; ++it) {
        if (it > (1u << 24)) {
            atomicOr(err, kErrWaitFull);
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// dp4a with explicit byte signedness: d = c + sum_i a_i * b_i.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// ------------------------------------------------------------ exact math

// 2^n as a binary32 for -149 <= n <= 127 (exact, subnormals included).
__device__ __forceinline__ float pow2f(int n) {
    if (n >= -126) return __uint_as_float(static_cast<uint32_t>(n + 127) << 23);
    return __uint_as_float(1u << (n + 149));
}

// Activation scale of an E8M0 byte: 2^(byte - 127 - 13).
__device__ __forceinline__ float e8m0_scale(uint32_t e) { return pow2f(static_cast<int>(e) - 140); }

__device__ __forceinline__ int32_t sat32(long long v) {
    return v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : static_cast<int32_t>(v));
}

// Round-half-even arithmetic right shift (emulator:507-517), branch-free:
// floor((v + 2^(sh-1) - 1 + bit_sh(v)) / 2^sh) rounds to nearest with ties to
// the even quotient for either sign (bit_sh(v) is the parity of floor(v/2^sh)).
// Every caller has |v| <= (2^31-1)(2^32-1), so the addition cannot overflow.
__device__ __forceinline__ long long rshift_even(long long v, unsigned sh) {
    if (sh == 0) return v;
    return (v + ((1ll << (sh - 1)) - 1) + ((v >> sh) & 1)) >> sh;
}

// Low `bits` bits, sign-extended (emulator:519-524).
__device__ __forceinline__ long long wrap_bits(long long v, unsigned bits) {
    const unsigned long long mask = (1ull << bits) - 1ull;
    unsigned long long raw = static_cast<unsigned long long>(v) & mask;
    if (raw & (1ull << (bits - 1))) raw |= ~mask;
    return static_cast<long long>(raw);
}

// Q15.17 conversion, round half to even, saturating (emulator:481-505).
__device__ __forceinline__ int32_t float_to_q17(float value) {
    const uint32_t bits = __float_as_uint(value);
    const bool neg = (bits >> 31) != 0;
    const uint32_t e = (bits >> 23) & 0xffu;
    const uint32_t frac = bits & 0x7fffffu;
    if (e < 109) return 0;
    if (e >= 141) return neg ? INT32_MIN : INT32_MAX;
    const uint32_t sig = (1u << 23) | frac;
    unsigned long long mag;
    if (e >= 133) {
        mag = static_cast<unsigned long long>(sig) << (e - 133);
    } else {
        const unsigned sh = 133 - e;
        uint32_t q = sig >> sh;
        const uint32_t rem = sig & ((1u << sh) - 1u);
        const uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        mag = q;
    }
    if (!neg) return mag > 0x7fffffffull ? INT32_MAX : static_cast<int32_t>(mag);
    return mag >= (1ull << 31) ? INT32_MIN : -static_cast<int32_t>(mag);
}

// Q17 multiply with round-half-even and 32-bit wrap (emulator:597-600).
__device__ __forceinline__ int32_t mulq17(int32_t a, uint32_t b) {
    return static_cast<int32_t>(
        wrap_bits(rshift_even(static_cast<long long>(a) * static_cast<long long>(b), 17), 32));
}

// mulq17 for b < 2^31 in 32-bit steps: one wide multiply, a funnel shift for
// floor(p / 2^17) mod 2^32, and the round-half-even increment from the 17
// dropped bits and the quotient's parity.  Equal to mulq17 (checked on 2e8
// random and edge operands); shorter on a serial chain.
__device__ __forceinline__ int32_t mulq17_w(int32_t a, uint32_t b) {
    const long long p = static_cast<long long>(a) * static_cast<int32_t>(b);
    const uint32_t lo = static_cast<uint32_t>(p), hi = static_cast<uint32_t>(static_cast<unsigned long long>(p) >> 32);
    const uint32_t q = __funnelshift_r(lo, hi, 17);
    const uint32_t r = lo & 0x1FFFFu;
    const uint32_t inc = static_cast<uint32_t>(r > 0x10000u) | (static_cast<uint32_t>(r == 0x10000u) & q);
    return static_cast<int32_t>(q + (inc & 1u));
}

// sat32(x + y) of two int32 values.
__device__ __forceinline__ int32_t add_sat32(int32_t x, int32_t y) {
    int32_t d;
    asm("add.sat.s32 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(y));
    return d;
}

// One lane's share of the G32 E8M0/INT14 quantizer (emulator:167-210,
// int4_decoder_blocks.cpp:22-73); all 32 lanes of the warp hold one group.
// Returns the INT14 value; *e8m0 receives max_exp + 127.
__device__ __forceinline__ int quantize_g32_lane(float v, uint32_t* e8m0) {
    int ex = -255;
    int mraw = 0;
    if (v != 0.0f) {
        const float m = frexpf(v, &ex);
        // m * 8192 is exact in binary32 (a power-of-two scaling of a float),
        // so the single-precision floor equals the emulator's double one.
        mraw = static_cast<int>(floorf(__fmul_rn(m, 8192.0f)));
    }
    int maxe = __reduce_max_sync(0xffffffffu, ex);
    if (maxe < -127) maxe = -127;
    *e8m0 = static_cast<uint32_t>(maxe + 127);
    int q = 0;
    if (ex != -255) {
        const int dif = maxe - ex;
        q = dif >= 31 ? (mraw < 0 ? -1 : 0) : (mraw >> dif);
    }
    return q > 8191 ? 8191 : (q < -8191 ? -8191 : q);
}

// Pair tree of the four bank partials: (p0 + p1) + (p2 + p3)
// (int4_linear_finalize_pair_schedule, int4_linear_controller.cpp:1384-1439).
// Partials come from other CTAs of the same or the previous kernel, so they
// are read at L2 (ld.global.cg), never from a possibly stale L1 line.
__device__ __forceinline__ float combine4(const float* partials, int stride, int row) {
    const float s01 = __fadd_rn(__ldcg(partials + row), __ldcg(partials + stride + row));
    const float s23 = __fadd_rn(__ldcg(partials + 2 * stride + row), __ldcg(partials + 3 * stride + row));
    return __fadd_rn(s01, s23);
}

// RMS reciprocal of a 4096 residual with the reference's exact summation
// order (emulator:427-447): 8 cyclic slots per 1024-column bank, slots
// summed serially, then (p0+p1)+(p2+p3); r = 1/sqrt(total/4096 + 1e-5).
// Executed by one full warp: lane = bank*8 + slot.  Returns r in every lane.
__device__ __forceinline__ float rms_recip_warp(const float* x) {
    const int lane = threadIdx.x & 31;
    const int bank = lane >> 3, slot = lane & 7;
    const float* base = x + bank * 1024 + slot;
    float acc = 0.0f;
#pragma unroll 16
    for (int i = 0; i < 128; ++i) {
        const float v = base[i * 8];
        acc = __fadd_rn(acc, __fmul_rn(v, v));
    }
    // total of bank = ((((0 + s0) + s1) + s2) ... + s7)
    float total = 0.0f;
#pragma unroll
    for (int s = 0; s < 8; ++s) total = __fadd_rn(total, __shfl_sync(0xffffffffu, acc, bank * 8 + s));
    const float t0 = __shfl_sync(0xffffffffu, total, 0);
    const float t1 = __shfl_sync(0xffffffffu, total, 8);
    const float t2 = __shfl_sync(0xffffffffu, total, 16);
    const float t3 = __shfl_sync(0xffffffffu, total, 24);
    const float sum = __fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3));
    const float mean_eps = __fadd_rn(__fmul_rn(sum, 1.0f / 4096.0f), 1.0e-5f);
    return __fdiv_rn(1.0f, __fsqrt_rn(mean_eps));
}

}  // namespace i4d
