// i4d_pack.cuh -- the bank-image producer on the device: AutoRound W4G128
// matrices (and the FP32 LM head) into the reference's superblock layout.
//
// Restates scripts/autoround_pack_llama2_u250.py:
//   read_ar_matrix (:413-424): offset-binary nibbles, column 2i in the low
//     nibble, w = nibble - 8; scales Q1.15 = clip(round_half_even(s * 32768)).
//   permute_qk_rows (:101-113): Q/K rows from split-half to adjacent-pair RoPE
//     order: destination row 2j of a head is source row j, row 2j+1 is 64+j.
//   pack_matrix_to_super_blocks (:115-188): 16 tiles per superblock; 128
//     scale words (tile t, word w, slot s: row 16w + 4(s/8) + (s%8)/2, group
//     s%2) then 4096 weight words (tile t, group g, row block rb: 32 lanes x
//     2 bytes, byte0 = r0<<4 | r1, byte1 = r2<<4 | r3, r = 4rb..4rb+3).
//   pack_logits_into_banks (:268-307), max-abs RTN path: per 128 columns
//     s = max(max|x|, 1e-8) / 7, w = clip(round(x / (s + 1e-12)), -8, 7).
// Every destination word is computed from the source directly (no staging):
// one thread per 64-byte word, four 16-byte stores.
#pragma once

#include <cstdint>

namespace i4d {

constexpr int kPackThreads = 256;
constexpr int kPackWordsPerBlock = 128 + 4096;

struct PackArgs {
    const uint8_t* nib;    // AutoRound nibbles [Mv][Kv/2], or null
    const int8_t* w8;      // int8 weights [Mv][Kv] (the quantised head), or null
    const float* scales;   // FP32 group-128 scales [Mv][Kv/128]
    int Mv, Kv;            // the source's (valid) rows and columns
    int lit;               // local input tiles per bank (padded columns / 1024)
    int blocks;            // superblocks per bank
    int permute_qk;        // Q/K: adjacent-pair RoPE row order
    uint8_t* dst[4];       // the matrix's superblock region in each bank image
};

__device__ __forceinline__ int pack_src_row(const PackArgs& a, int r) {
    if (!a.permute_qk) return r;
    const int h = r >> 7, d = r & 127;
    return (h << 7) + ((d & 1) ? 64 + (d >> 1) : (d >> 1));
}

// Q1.15 of a source scale, 0 outside the source (the padded rows / groups).
__device__ __forceinline__ int16_t pack_scale(const PackArgs& a, int r, int g128) {
    if (r >= a.Mv || g128 >= a.Kv / 128) return 0;
    const float s = a.scales[static_cast<size_t>(pack_src_row(a, r)) * (a.Kv / 128) + g128];
    int q = __float2int_rn(__fmul_rn(s, 32768.0f));
    q = q < -32768 ? -32768 : (q > 32767 ? 32767 : q);
    return static_cast<int16_t>(q);
}

// 4-bit two's complement (w & 0x0F) of a source weight, 0 outside the source.
__device__ __forceinline__ uint32_t pack_q4(const PackArgs& a, int r, int c) {
    if (r >= a.Mv || c >= a.Kv) return 0u;
    const size_t row = static_cast<size_t>(pack_src_row(a, r));
    if (a.nib) {
        const uint32_t b = a.nib[row * (a.Kv / 2) + (c >> 1)];
        return ((c & 1) ? (b >> 4) : (b & 15u)) ^ 8u;  // (nibble - 8) & 0x0F
    }
    return static_cast<uint32_t>(a.w8[row * a.Kv + c]) & 15u;
}

__global__ void __launch_bounds__(kPackThreads) k_pack_matrix(const __grid_constant__ PackArgs a) {
    const long long gid = static_cast<long long>(blockIdx.x) * kPackThreads + threadIdx.x;
    const long long per_bank = static_cast<long long>(a.blocks) * kPackWordsPerBlock;
    if (gid >= 4 * per_bank) return;
    const int pe = static_cast<int>(gid / per_bank);
    const int word = static_cast<int>(gid % per_bank);
    const int b = word / kPackWordsPerBlock, wb = word % kPackWordsPerBlock;
    uint32_t out[16];
    if (wb < 128) {  // scale word: tile t, word w
        const int t = wb >> 3, w = wb & 7;
        const int mt = b * 16 + t, out_tile = mt / a.lit, lct = mt % a.lit;
        const int row_start = out_tile * 128, g128_start = (pe * a.lit + lct) * 2;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            uint32_t v = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int sl = 2 * k + h;
                const int r = (w * 4 + sl / 8) * 4 + (sl % 8) / 2;
                v |= static_cast<uint32_t>(static_cast<uint16_t>(pack_scale(a, row_start + r, g128_start + (sl & 1))))
                     << (16 * h);
            }
            out[k] = v;
        }
    } else {  // weight word: tile t, group g, row block rb
        const int ww = wb - 128;
        const int t = ww >> 8, g = (ww >> 5) & 7, rb = ww & 31;
        const int mt = b * 16 + t, out_tile = mt / a.lit, lct = mt % a.lit;
        const int r0 = out_tile * 128 + 4 * rb, c0 = (pe * a.lit + lct) * 256 + g * 32;
#pragma unroll
        for (int k = 0; k < 16; ++k) {  // lanes 2k, 2k+1: bytes 4k .. 4k+3
            uint32_t v = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int c = c0 + 2 * k + h;
                const uint32_t b0 = (pack_q4(a, r0, c) << 4) | pack_q4(a, r0 + 1, c);
                const uint32_t b1 = (pack_q4(a, r0 + 2, c) << 4) | pack_q4(a, r0 + 3, c);
                v |= (b0 | (b1 << 8)) << (16 * h);
            }
            out[k] = v;
        }
    }
    uint4* d = reinterpret_cast<uint4*>(a.dst[pe] + static_cast<size_t>(word) * 64);
#pragma unroll
    for (int k = 0; k < 4; ++k) d[k] = make_uint4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
}

// The LM head's max-abs RTN quantiser: one warp per (row, 128 columns) of the
// padded [rows][4096] head (rows >= Mv are zero).
struct HeadQuantArgs {
    const float* head;  // [Mv][4096]
    int Mv, rows;
    int8_t* w8;         // [rows][4096]
    float* scales;      // [rows][32]
};

__global__ void __launch_bounds__(kPackThreads) k_quant_head(const __grid_constant__ HeadQuantArgs a) {
    const long long gw = (static_cast<long long>(blockIdx.x) * kPackThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= static_cast<long long>(a.rows) * 32) return;
    const int r = static_cast<int>(gw >> 5), g = static_cast<int>(gw & 31);
    float x[4];
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        x[k] = r < a.Mv ? a.head[static_cast<size_t>(r) * 4096 + g * 128 + lane * 4 + k] : 0.0f;
        m = fmaxf(m, fabsf(x[k]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = __fdiv_rn(fmaxf(m, 1e-8f), 7.0f);
    const float den = __fadd_rn(s, 1e-12f);
    char4 q;
    int v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float y = rintf(__fdiv_rn(x[k], den));
        v[k] = static_cast<int>(fminf(7.0f, fmaxf(-8.0f, y)));
    }
    q.x = static_cast<signed char>(v[0]);
    q.y = static_cast<signed char>(v[1]);
    q.z = static_cast<signed char>(v[2]);
    q.w = static_cast<signed char>(v[3]);
    *reinterpret_cast<char4*>(a.w8 + static_cast<size_t>(r) * 4096 + g * 128 + lane * 4) = q;
    if (lane == 0) a.scales[static_cast<size_t>(r) * 32 + g] = s;
}

}  // namespace i4d
