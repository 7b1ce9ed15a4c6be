/*
 * i4d_oracle.c -- CPU restatement of the reference decode arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker, never the product).
 * Built with -O2 -ffp-contract=off and without -ffast-math so that every
 * float operation rounds exactly once, as the reference emulator forces with
 * volatile temporaries (software_sim/llama2_decoder_sw_emulator.cpp:154-162).
 */
#include "i4d_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- geometry */

/* emulator:786-797 and autoround_pack_llama2_u250.py:59-80 */
int i4o_mode_rows(int mode) {
    if (mode <= I4O_O || mode == I4O_DOWN) return I4O_DIM;
    if (mode == I4O_GATE || mode == I4O_UP) return I4O_PHIDDEN;
    return I4O_PVOCAB;
}

int i4o_mode_cols(int mode) { return mode == I4O_DOWN ? I4O_PHIDDEN : I4O_DIM; }

int i4o_mode_local_in_tiles(int mode) { return i4o_mode_cols(mode) / (I4O_BANKS * 256); }

int i4o_mode_out_tiles(int mode) { return i4o_mode_rows(mode) / 128; }

int i4o_mode_data_words(int mode) {
    const int tiles = i4o_mode_out_tiles(mode) * i4o_mode_local_in_tiles(mode);
    return tiles / 16 * I4O_SUPERBLOCK_WORDS;
}

/* emulator:786-797, int4_model_layout.hpp:120-136 (data base word 4160). */
uint64_t i4o_matrix_word_offset(int layer, int mode) {
    uint64_t stride = 0;
    for (int m = 0; m < 7; ++m) stride += (uint64_t)i4o_mode_data_words(m);
    if (mode == I4O_LOGITS) return I4O_NORM_WORDS + 32ULL * stride;
    uint64_t off = I4O_NORM_WORDS + (uint64_t)layer * stride;
    for (int m = 0; m < mode; ++m) off += (uint64_t)i4o_mode_data_words(m);
    return off;
}

/* autoround_pack_llama2_u250.py:95-99, int4_model_layout.hpp:205-213 */
uint64_t i4o_norm_word_offset(int layer, int which) {
    if (which == 2) return 32ULL * 128ULL;
    return (uint64_t)layer * 128ULL + (which == 1 ? 64ULL : 0ULL);
}

static inline float fmul(float a, float b) { volatile float r = a * b; return r; }
static inline float fadd(float a, float b) { volatile float r = a + b; return r; }

/* -------------------------------------------------------------- quantizer */

/* emulator:167-210.  frexp, floor(m*8192), arithmetic shift to the group
 * maximum exponent, clamp to +-8191.  E8M0 byte = max_exp + 127. */
void i4o_quantize_g32(const float* x, int n, int16_t* q, uint8_t* e8m0) {
    for (int g = 0; g < n / I4O_GROUP; ++g) {
        const float* in = x + g * I4O_GROUP;
        int exps[I4O_GROUP];
        int32_t mraw[I4O_GROUP];
        int maxe = -255;
        for (int i = 0; i < I4O_GROUP; ++i) {
            if (in[i] != 0.0f) {
                const float m = frexpf(in[i], &exps[i]);
                mraw[i] = (int32_t)floor((double)m * 8192.0);
                if (exps[i] > maxe) maxe = exps[i];
            } else {
                mraw[i] = 0;
                exps[i] = -255;
            }
        }
        if (maxe < -127) maxe = -127;
        e8m0[g] = (uint8_t)(maxe + 127);
        for (int i = 0; i < I4O_GROUP; ++i) {
            int v;
            if (exps[i] == -255) {
                v = 0;
            } else {
                const int dif = maxe - exps[i];
                v = dif >= 31 ? (mraw[i] < 0 ? -1 : 0) : (mraw[i] >> dif);
            }
            if (v > 8191) v = 8191;
            if (v < -8191) v = -8191;
            q[g * I4O_GROUP + i] = (int16_t)v;
        }
    }
}

/* ---------------------------------------------------------------- RMSNorm */

/* emulator:427-453 (== int4_local_sumsq + int4_rms_pair01_schedule +
 * int4_local_rms_normalize_quantize, int4_decoder_blocks.cpp:77-227). */
void i4o_rmsnorm_quantize(const float* x, const float* gamma, int16_t* q,
                          uint8_t* e8m0, float* recip) {
    float part[I4O_BANKS];
    for (int p = 0; p < I4O_BANKS; ++p) {
        float slots[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int i = 0; i < 1024; ++i) {
            const float v = x[p * 1024 + i];
            slots[i & 7] = fadd(slots[i & 7], fmul(v, v));
        }
        float total = 0.0f;
        for (int s = 0; s < 8; ++s) total = fadd(total, slots[s]);
        part[p] = total;
    }
    const float total = fadd(fadd(part[0], part[1]), fadd(part[2], part[3]));
    const float mean_eps = fadd(fmul(total, 1.0f / 4096.0f), 1.0e-5f);
    volatile float root = sqrtf(mean_eps);
    volatile float r = 1.0f / root;
    if (recip) *recip = r;
    float* norm = (float*)malloc(sizeof(float) * I4O_DIM);
    for (int i = 0; i < I4O_DIM; ++i) norm[i] = fmul(fmul(x[i], r), gamma[i]);
    i4o_quantize_g32(norm, I4O_DIM, q, e8m0);
    free(norm);
}

/* ------------------------------------------------------------------ Q15.17 */

/* emulator:481-505: float -> Q15.17, round half to even, saturate. */
int32_t i4o_float_to_q17(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    const int neg = (bits >> 31) != 0;
    const uint32_t e = (bits >> 23) & 0xffu;
    const uint32_t frac = bits & 0x7fffffu;
    if (e == 0 || e < 109) return 0;
    if (e >= 141) return neg ? INT32_MIN : INT32_MAX;
    const uint32_t sig = (1u << 23) | frac;
    uint64_t mag;
    if (e >= 133) {
        mag = (uint64_t)sig << (e - 133);
    } else {
        const unsigned sh = 133 - e;
        uint32_t quo = sig >> sh;
        const uint32_t rem = sig & ((1u << sh) - 1u);
        const uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (quo & 1u))) ++quo;
        mag = quo;
    }
    if (!neg) return mag > (uint64_t)INT32_MAX ? INT32_MAX : (int32_t)mag;
    return mag >= (1ULL << 31) ? INT32_MIN : -(int32_t)mag;
}

static inline int32_t sat32(int64_t v) {
    if (v > INT32_MAX) return INT32_MAX;
    if (v < INT32_MIN) return INT32_MIN;
    return (int32_t)v;
}

/* emulator:507-517: round half to even on a signed right shift. */
static inline int64_t rshift_even(int64_t v, unsigned sh) {
    if (sh == 0) return v;
    const int neg = v < 0;
    const uint64_t mag = neg ? (uint64_t)(-(v + 1)) + 1u : (uint64_t)v;
    uint64_t quo = mag >> sh;
    const uint64_t rem = mag & ((1ULL << sh) - 1u);
    const uint64_t half = 1ULL << (sh - 1);
    if (rem > half || (rem == half && (quo & 1u))) ++quo;
    return neg ? -(int64_t)quo : (int64_t)quo;
}

/* emulator:519-524: keep the low `bits` bits, sign-extended. */
static inline int64_t wrap_bits(int64_t v, unsigned bits) {
    const uint64_t mask = (1ULL << bits) - 1u;
    uint64_t raw = (uint64_t)v & mask;
    if (raw & (1ULL << (bits - 1))) raw |= ~mask;
    return (int64_t)raw;
}

/* -------------------------------------------------------------------- RoPE */

/* emulator:937-968 / generate_rope_lut.py:20-41: position p, pair i lives in
 * 608-bit word p*4 + i/16 (two 64-byte DDR words), lane i%16 at bit 38*lane:
 * 19-bit cosine then 19-bit sine, signed Q1.17. */
void i4o_decode_rope_lut(const uint8_t* lut, int32_t* cosv, int32_t* sinv) {
    for (int pos = 0; pos < I4O_MAX_SEQ; ++pos) {
        for (int grp = 0; grp < 4; ++grp) {
            const uint8_t* base = lut + ((size_t)pos * 4 + grp) * 128;
            for (int lane = 0; lane < 16; ++lane) {
                uint32_t fields[2];
                for (int f = 0; f < 2; ++f) {
                    const int bit0 = lane * 38 + f * 19;
                    uint32_t v = 0;
                    for (int b = 0; b < 19; ++b) {
                        const int s = bit0 + b;
                        v |= (uint32_t)((base[s >> 3] >> (s & 7)) & 1u) << b;
                    }
                    fields[f] = v;
                }
                const int pair = grp * 16 + lane;
                for (int f = 0; f < 2; ++f) {
                    const uint32_t raw = fields[f];
                    const int32_t sv = (raw & (1u << 18)) ? (int32_t)(raw | 0xfff80000u) : (int32_t)raw;
                    if (f == 0) cosv[(size_t)pos * 64 + pair] = sv;
                    else sinv[(size_t)pos * 64 + pair] = sv;
                }
            }
        }
    }
}

/* emulator:526-541: adjacent pairs (2i, 2i+1) of every head. */
void i4o_rope_q17(int32_t* vec, const int32_t* c, const int32_t* s) {
    for (int h = 0; h < I4O_HEADS; ++h) {
        int32_t* hv = vec + h * I4O_HEAD_DIM;
        for (int pr = 0; pr < 64; ++pr) {
            const int64_t a = hv[2 * pr], b = hv[2 * pr + 1];
            hv[2 * pr] = sat32((a * c[pr] - b * s[pr]) >> 17);
            hv[2 * pr + 1] = sat32((a * s[pr] + b * c[pr]) >> 17);
        }
    }
}

/* -------------------------------------------------------------- INT8 KV */

/* emulator:543-553 (== swiftkv_kv_power2_shift, swiftkv_attention.cpp:358-389):
 * shift = max(0, msb(max |v|) - 6). */
uint8_t i4o_kv_shift(const int32_t* v32) {
    uint32_t mx = 0;
    for (int i = 0; i < I4O_GROUP; ++i) {
        const int64_t v = v32[i];
        const uint32_t mag = (uint32_t)(v < 0 ? -v : v);
        if (mag > mx) mx = mag;
    }
    if (mx == 0) return 0;
    int msb = 31;
    while (msb > 0 && ((mx >> msb) & 1u) == 0) --msb;
    return (uint8_t)(msb > 6 ? msb - 6 : 0);
}

/* emulator:555-564 (== swiftkv_quantize_kv_raw, swiftkv_attention.cpp:391-414). */
int8_t i4o_kv_quant(int32_t raw, uint8_t shift) {
    const int64_t w = raw;
    uint64_t mag = (uint64_t)(w < 0 ? -w : w);
    if (shift) mag += 1ULL << (shift - 1);
    mag >>= shift;
    if (mag > 127) mag = 127;
    return (int8_t)(w < 0 ? -(int)mag : (int)mag);
}

/* Record layout (swiftkv_attention.cpp:517-581, swiftkv_attention.hpp:21-36):
 * word 0 bits [5g,5g+5) = K shift of group g, bits [20+5g, 25+5g) = V shift;
 * words 1-2 = K int8[0..127]; words 3-4 = V int8[0..127]. */
void i4o_kv_write_record(uint8_t* rec, const int32_t* k, const int32_t* v) {
    memset(rec, 0, I4O_KV_RECORD_BYTES);
    uint64_t meta = 0;
    for (int g = 0; g < 4; ++g) {
        const uint8_t ks = i4o_kv_shift(k + g * 32);
        const uint8_t vs = i4o_kv_shift(v + g * 32);
        meta |= (uint64_t)ks << (5 * g);
        meta |= (uint64_t)vs << (20 + 5 * g);
        for (int l = 0; l < 32; ++l) {
            rec[64 + g * 32 + l] = (uint8_t)i4o_kv_quant(k[g * 32 + l], ks);
            rec[192 + g * 32 + l] = (uint8_t)i4o_kv_quant(v[g * 32 + l], vs);
        }
    }
    for (int b = 0; b < 5; ++b) rec[b] = (uint8_t)(meta >> (8 * b));
}

static inline unsigned rec_k_shift(const uint8_t* rec, int g) {
    uint64_t meta = 0;
    for (int b = 0; b < 5; ++b) meta |= (uint64_t)rec[b] << (8 * b);
    return (unsigned)((meta >> (5 * g)) & 31u);
}

static inline unsigned rec_v_shift(const uint8_t* rec, int g) {
    uint64_t meta = 0;
    for (int b = 0; b < 5; ++b) meta |= (uint64_t)rec[b] << (8 * b);
    return (unsigned)((meta >> (20 + 5 * g)) & 31u);
}

/* ------------------------------------------------------ online softmax exp */

static uint32_t g_exp2_q30[33];
static int g_exp2_ready = 0;

/* The reference table (emulator:566-573, swiftkv_attention.cpp:185-195) holds
 * round(2^(30 + i/32)) for i = 0..32; it is computed here. */
static void exp2_table_init(void) {
    if (g_exp2_ready) return;
    for (int i = 0; i <= 32; ++i)
        g_exp2_q30[i] = (uint32_t)llroundl(exp2l(30.0L + (long double)i / 32.0L));
    g_exp2_ready = 1;
}

/* emulator:575-595 (== swiftkv_exp_negative, swiftkv_attention.cpp:199-260):
 * exp(x) for Q15.17 x <= 0 via log2(e) in Q21, 5-bit LUT, linear
 * interpolation over the 12 remaining fraction bits, result Q1.17 wrap18. */
uint32_t i4o_exp_negative_q17(int32_t x) {
    exp2_table_init();
    if (x >= 0) return 1u << 17;
    if (x <= -(32 << 17)) return 0;
    const int32_t log2e_q21 = (int32_t)nearbyint(1.4426950408889634 * (double)(1 << 21));
    int64_t l2 = rshift_even((int64_t)x * log2e_q21, 21);
    l2 = wrap_bits(l2, 24);
    const int ex = (int)(l2 >> 17);
    const int32_t fr = (int32_t)(l2 - ((int64_t)ex << 17));
    const unsigned idx = (unsigned)fr >> 12;
    const unsigned rem = (unsigned)fr & 0xfffu;
    const uint32_t base = g_exp2_q30[idx];
    const uint32_t delta = g_exp2_q30[idx + 1] - base;
    const uint32_t interp = base + (uint32_t)(((uint64_t)delta * rem + (1u << 11)) >> 12);
    const int sh = 13 - ex;
    uint64_t out = 0;
    if (sh <= 0) out = (uint64_t)interp << (-sh);
    else if (sh < 32) out = ((uint64_t)interp + (1ULL << (sh - 1))) >> sh;
    return (uint32_t)out & ((1u << 18) - 1u);
}

/* emulator:597-600 */
static inline int32_t mulq17(int32_t a, uint32_t b) {
    return (int32_t)wrap_bits(rshift_even((int64_t)a * (int64_t)b, 17), 32);
}

/* ---------------------------------------------------------------- attention */

static uint8_t* kv_record(uint8_t* kv, int layers, int stride, int bank,
                          int layer, int lh, int token) {
    const size_t rec = ((((size_t)bank * layers + layer) * I4O_LOCAL_HEADS + lh) *
                        (size_t)stride + (size_t)token);
    return kv + rec * I4O_KV_RECORD_BYTES;
}

/* emulator:602-714 for one head (bank p, local head lh). */
static void attention_head(uint8_t* kv, int layers, int stride, int layer,
                           int pos, int gh, const int32_t* qh,
                           const int32_t* kh, const int32_t* vh,
                           int16_t* out_q, uint8_t* out_e8m0) {
    const int p = gh / I4O_LOCAL_HEADS, lh = gh % I4O_LOCAL_HEADS;
    const int32_t score_scale = i4o_float_to_q17(0.08838834764831845f);
    i4o_kv_write_record(kv_record(kv, layers, stride, p, layer, lh, pos), kh, vh);

    int32_t running_max = 0;
    uint32_t norm = 0;
    int32_t state[I4O_HEAD_DIM];
    memset(state, 0, sizeof(state));
    for (int t = 0; t <= pos; ++t) {
        const uint8_t* rec = kv_record(kv, layers, stride, p, layer, lh, t);
        const int8_t* k8 = (const int8_t*)(rec + 64);
        const int8_t* v8 = (const int8_t*)(rec + 192);
        int64_t dot = 0;
        for (int g = 0; g < 4; ++g) {
            int64_t halves[2];
            const int sh = (int)rec_k_shift(rec, g);
            for (int hf = 0; hf < 2; ++hf) {
                int64_t sum = 0;
                for (int l = 0; l < 16; ++l) {
                    const int idx = g * 32 + hf * 16 + l;
                    sum += (int64_t)qh[idx] * k8[idx];
                }
                halves[hf] = wrap_bits(sh >= 10 ? (int64_t)((uint64_t)sum << (sh - 10))
                                                : (sum >> (10 - sh)), 44);
            }
            const int64_t gd = wrap_bits(halves[0] + halves[1], 44);
            dot = g == 0 ? gd : wrap_bits(dot + gd, 44);
        }
        const int32_t score = sat32(rshift_even(dot * score_scale, 24));
        uint32_t coef = 1u << 17;
        int rescale = 0;
        if (t == 0) {
            running_max = score;
            norm = 1u << 17;
        } else if (score <= running_max) {
            coef = i4o_exp_negative_q17(sat32((int64_t)score - running_max));
            norm = (norm + coef) & ((1u << 30) - 1u);
        } else {
            coef = i4o_exp_negative_q17(sat32((int64_t)running_max - score));
            norm = (uint32_t)rshift_even((int64_t)norm * coef, 17) & ((1u << 30) - 1u);
            norm = (norm + (1u << 17)) & ((1u << 30) - 1u);
            running_max = score;
            rescale = 1;
        }
        for (int d = 0; d < I4O_HEAD_DIM; ++d) {
            const int32_t val = (int32_t)v8[d] << rec_v_shift(rec, d / 32);
            if (t == 0) state[d] = val;
            else if (rescale) state[d] = sat32((int64_t)mulq17(state[d], coef) + val);
            else state[d] = sat32((int64_t)state[d] + mulq17(val, coef));
        }
    }
    const uint32_t inv = norm == 0 ? 0u
        : (uint32_t)(((1ULL << 34) + (norm >> 1)) / norm);
    int32_t nrm[I4O_HEAD_DIM];
    for (int d = 0; d < I4O_HEAD_DIM; ++d) nrm[d] = mulq17(state[d], inv);
    for (int g = 0; g < 4; ++g) {
        int32_t mx = 0;
        for (int l = 0; l < 32; ++l) {
            const int32_t v = nrm[g * 32 + l];
            const int32_t mag = v == INT32_MIN ? INT32_MAX : abs(v);
            if (mag > mx) mx = mag;
        }
        const float maxf = (float)mx * (1.0f / 131072.0f);
        int maxe = -127;
        if (maxf != 0.0f) frexpf(maxf, &maxe);
        const float inv_scale = maxf == 0.0f ? 0.0f : ldexpf(1.0f, 13 - maxe);
        const int gg = gh * 4 + g;
        /* The E8M0 form of the emulator's float scale 2^(maxe-13) is maxe+127;
         * a zero scale maps to byte 0 (swiftkv_attention.cpp:2670-2676). */
        out_e8m0[gg] = maxf == 0.0f ? 0 : (uint8_t)(maxe + 127);
        for (int l = 0; l < 32; ++l) {
            const float val = (float)nrm[g * 32 + l] * (1.0f / 131072.0f);
            float r = fmul(val, inv_scale);
            r += r >= 0.0f ? 0.5f : -0.5f;
            if (r > 8191.0f) r = 8191.0f;
            if (r < -8191.0f) r = -8191.0f;
            out_q[gg * 32 + l] = (int16_t)r;
        }
    }
}

void i4o_attention(uint8_t* kv, int layers, int stride, int layer, int pos,
                   const int32_t* q, const int32_t* k, const int32_t* v,
                   int16_t* out_q, uint8_t* out_e8m0) {
    exp2_table_init();
#pragma omp parallel for schedule(static)
    for (int gh = 0; gh < I4O_HEADS; ++gh)
        attention_head(kv, layers, stride, layer, pos, gh,
                       q + gh * I4O_HEAD_DIM, k + gh * I4O_HEAD_DIM,
                       v + gh * I4O_HEAD_DIM, out_q, out_e8m0);
}

/* ------------------------------------------------------------------ linear */

/* One bank's partial sums, restating emulator:216-264 over the packed
 * superblock stream (reader emulator:799-892; writer
 * autoround_pack_llama2_u250.py:114-189):
 *   tile t = out_tile*local_in_tiles + in_tile, superblock t/16,
 *   scale word w of tile: rows 16w..16w+15, int16 s = 2*(row%16) + g128,
 *   weight word g*32 + rb: lanes l (column g*32+l) as bytes 2l, 2l+1 =
 *   (row0<<4 | row1), (row2<<4 | row3) of rows 4rb..4rb+3.
 * For every row the FP32 chain runs over the local G32 groups in order:
 * acc = fl(acc + fl(float(dot) * fl(ws * as))). */
void i4o_linear_bank(const uint8_t* sb, int out_tiles, int lit,
                     const int16_t* aq, const uint8_t* ae, int hls_start,
                     float* partial) {
    const int groups = lit * 8;
    float* as = (float*)malloc(sizeof(float) * (size_t)groups);
    for (int g = 0; g < groups; ++g) as[g] = ldexpf(1.0f, (int)ae[g] - 140);
#pragma omp parallel for schedule(static)
    for (int ot = 0; ot < out_tiles; ++ot) {
        float acc[128];
        for (int it = 0; it < lit; ++it) {
            const int t = ot * lit + it;
            const uint8_t* blk = sb + (size_t)(t / 16) * I4O_SUPERBLOCK_WORDS * 64;
            const uint8_t* scl = blk + (size_t)(t % 16) * 8 * 64;
            const uint8_t* wts = blk + 128 * 64 + (size_t)(t % 16) * 256 * 64;
            for (int g = 0; g < 8; ++g) {
                const int lg = it * 8 + g;
                const int16_t* a = aq + lg * 32;
                for (int rb = 0; rb < 32; ++rb) {
                    const uint8_t* word = wts + (size_t)(g * 32 + rb) * 64;
                    int32_t dot[4] = {0, 0, 0, 0};
                    for (int l = 0; l < 32; ++l) {
                        const uint8_t b0 = word[2 * l], b1 = word[2 * l + 1];
                        const int n[4] = {b0 >> 4, b0 & 15, b1 >> 4, b1 & 15};
                        for (int r = 0; r < 4; ++r) {
                            const int w = n[r] >= 8 ? n[r] - 16 : n[r];
                            dot[r] += w * (int32_t)a[l];
                        }
                    }
                    for (int r = 0; r < 4; ++r) {
                        const int row = rb * 4 + r;
                        int16_t raw;
                        memcpy(&raw, scl + (size_t)(row / 16) * 64 + (size_t)(((row % 16) * 2 + g / 4) * 2), 2);
                        const float ws = (float)raw * (1.0f / 32768.0f);
                        const float contrib = fmul((float)dot[r], fmul(ws, as[lg]));
                        if (lg == 0) acc[row] = hls_start ? contrib : fadd(0.0f, contrib);
                        else acc[row] = fadd(acc[row], contrib);
                    }
                }
            }
        }
        memcpy(partial + (size_t)ot * 128, acc, sizeof(acc));
    }
    free(as);
}

void i4o_gemv(const uint8_t* const banks[4], int layer, int mode,
              const int16_t* aq, const uint8_t* ae, float* y, float* partials) {
    const int rows = i4o_mode_rows(mode);
    const int lit = i4o_mode_local_in_tiles(mode);
    const int local = lit * 256;
    float* part = (float*)malloc(sizeof(float) * (size_t)rows * 4);
    const uint64_t off = i4o_matrix_word_offset(layer, mode) * 64ULL;
    for (int p = 0; p < 4; ++p)
        i4o_linear_bank(banks[p] + off, i4o_mode_out_tiles(mode), lit,
                        aq + p * local, ae + p * local / 32, 0,
                        part + (size_t)p * rows);
    for (int r = 0; r < rows; ++r)
        y[r] = fadd(fadd(part[r], part[rows + r]),
                    fadd(part[2 * rows + r], part[3 * rows + r]));
    if (partials) memcpy(partials, part, sizeof(float) * (size_t)rows * 4);
    free(part);
}

/* ------------------------------------------------------------------ SwiGLU */

/* emulator:716-722: (g * (1 / (1 + expf(-g)))) * u with the C library expf. */
void i4o_swiglu(const float* gate, const float* up, int n, float* out) {
    for (int i = 0; i < n; ++i) {
        const float g = gate[i];
        volatile float e = expf(-g);
        volatile float den = 1.0f + e;
        volatile float sig = 1.0f / den;
        out[i] = fmul(fmul(g, sig), up[i]);
    }
}

/* ----------------------------------------------------------------- forward */

/* emulator:970-990: 1024 FP32 per bank at the norm word offset. */
void i4o_read_gamma(const uint8_t* const banks[4], int layer, int which,
                    float* gamma) {
    const uint64_t off = i4o_norm_word_offset(layer, which) * 64ULL;
    for (int p = 0; p < 4; ++p) memcpy(gamma + p * 1024, banks[p] + off, 4096);
}

/* emulator:727-783 */
void i4o_forward(const uint8_t* const banks[4], const int32_t* rope_cos,
                 const int32_t* rope_sin, uint8_t* kv, int layers, int stride,
                 int pos, float* residual, float* logits) {
    float* gamma = (float*)malloc(sizeof(float) * I4O_DIM);
    float* qf = (float*)malloc(sizeof(float) * I4O_DIM * 3);
    float* kf = qf + I4O_DIM;
    float* vf = kf + I4O_DIM;
    int32_t* q = (int32_t*)malloc(sizeof(int32_t) * I4O_DIM * 3);
    int32_t* k = q + I4O_DIM;
    int32_t* v = k + I4O_DIM;
    float* proj = (float*)malloc(sizeof(float) * I4O_DIM);
    float* gate = (float*)malloc(sizeof(float) * I4O_PHIDDEN * 3);
    float* up = gate + I4O_PHIDDEN;
    float* sw = up + I4O_PHIDDEN;
    int16_t* aq = (int16_t*)malloc(sizeof(int16_t) * I4O_PHIDDEN);
    uint8_t* ae = (uint8_t*)malloc(I4O_PHIDDEN / 32);
    const int32_t* c = rope_cos + (size_t)pos * 64;
    const int32_t* s = rope_sin + (size_t)pos * 64;
    for (int l = 0; l < layers; ++l) {
        i4o_read_gamma(banks, l, 0, gamma);
        i4o_rmsnorm_quantize(residual, gamma, aq, ae, NULL);
        i4o_gemv(banks, l, I4O_Q, aq, ae, qf, NULL);
        i4o_gemv(banks, l, I4O_K, aq, ae, kf, NULL);
        i4o_gemv(banks, l, I4O_V, aq, ae, vf, NULL);
        for (int i = 0; i < I4O_DIM; ++i) {
            q[i] = i4o_float_to_q17(qf[i]);
            k[i] = i4o_float_to_q17(kf[i]);
            v[i] = i4o_float_to_q17(vf[i]);
        }
        i4o_rope_q17(q, c, s);
        i4o_rope_q17(k, c, s);
        i4o_attention(kv, layers, stride, l, pos, q, k, v, aq, ae);
        i4o_gemv(banks, l, I4O_O, aq, ae, proj, NULL);
        for (int i = 0; i < I4O_DIM; ++i) residual[i] = fadd(residual[i], proj[i]);
        i4o_read_gamma(banks, l, 1, gamma);
        i4o_rmsnorm_quantize(residual, gamma, aq, ae, NULL);
        i4o_gemv(banks, l, I4O_GATE, aq, ae, gate, NULL);
        i4o_gemv(banks, l, I4O_UP, aq, ae, up, NULL);
        i4o_swiglu(gate, up, I4O_PHIDDEN, sw);
        i4o_quantize_g32(sw, I4O_PHIDDEN, aq, ae);
        i4o_gemv(banks, l, I4O_DOWN, aq, ae, proj, NULL);
        for (int i = 0; i < I4O_DIM; ++i) residual[i] = fadd(residual[i], proj[i]);
    }
    i4o_read_gamma(banks, 0, 2, gamma);
    i4o_rmsnorm_quantize(residual, gamma, aq, ae, NULL);
    i4o_gemv(banks, 0, I4O_LOGITS, aq, ae, logits, NULL);
    free(gamma); free(qf); free(q); free(proj); free(gate); free(aq); free(ae);
}

int i4o_argmax(const float* logits, int n) {
    int best = 0;
    float bv = logits[0];
    for (int i = 1; i < n; ++i)
        if (logits[i] > bv) { best = i; bv = logits[i]; }
    return best;
}

/* ---- perplexity term (emulator:1902-1926) ---- */

double i4o_nll(const float* logits, int n, int target, float* max_out, float* sum_out) {
    float max_l = logits[0];
    for (int i = 1; i < n; ++i)
        if (logits[i] > max_l) max_l = logits[i];
    float sum_exp = 0.0f;
    for (int i = 0; i < n; ++i) sum_exp += expf(logits[i] - max_l);
    const float lse_f = max_l + logf(sum_exp);
    const double log_sum_exp = (double)lse_f;
    const double log_prob = (double)logits[target] - log_sum_exp;
    if (max_out) *max_out = max_l;
    if (sum_out) *sum_out = sum_exp;
    return -log_prob;
}

/* ---- sampler (decode_host.cpp:724-868, emulator:1411-1569) ---- */

/* decode_host.cpp:703-717: first strict maximum, NaN skipped; -1 if none. */
static int sample_argmax_host(const float* p, int n) {
    int best = -1;
    for (int i = 0; i < n; ++i) {
        if (isnan(p[i])) continue;
        if (best < 0 || p[i] > p[best]) best = i;
    }
    return best;
}

/* Both references: xorshift64* (decode_host.cpp:806-816, emulator:1509-1518). */
static float sample_coin(uint64_t* st) {
    *st ^= *st >> 12;
    *st ^= *st << 25;
    *st ^= *st >> 27;
    const uint32_t u = (uint32_t)((*st * 0x2545F4914F6CDD1DULL) >> 32);
    return (float)(u >> 8) / 16777216.0f;
}

typedef struct {
    float p;
    int i;
} SampleCand;

static int cand_desc(const void* a, const void* b) {
    const SampleCand* x = (const SampleCand*)a;
    const SampleCand* y = (const SampleCand*)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

int i4o_sample(int mode, const float* logits, int n, const int32_t* history, int n_history,
               float temperature, float top_p, float repeat_penalty, uint64_t* rng_state) {
    const int host = mode == 0;
    if (host && temperature == 0.0f && repeat_penalty == 1.0f) return sample_argmax_host(logits, n);
    float* p = (float*)malloc(sizeof(float) * (size_t)n);
    unsigned char* pen = (unsigned char*)calloc((size_t)n, 1);
    memcpy(p, logits, sizeof(float) * (size_t)n);
    int result = -3;
    if (repeat_penalty != 1.0f) {
        for (int h = 0; h < n_history; ++h) {
            const int t = history[h];
            if (t < 0 || t >= n || pen[t]) continue;
            if (!host || isfinite(p[t])) p[t] = p[t] < 0.0f ? p[t] * repeat_penalty : p[t] / repeat_penalty;
            pen[t] = 1;
        }
    }
    if (temperature == 0.0f) {
        result = host ? sample_argmax_host(p, n) : i4o_argmax(p, n);
        goto done;
    }
    float mx;
    if (host) {
        mx = -INFINITY;
        for (int i = 0; i < n; ++i)
            if (isfinite(p[i]) && p[i] > mx) mx = p[i];
        if (!isfinite(mx)) {
            result = -2;
            goto done;
        }
    } else {
        for (int i = 0; i < n; ++i) p[i] /= temperature;
        mx = p[0];
        for (int i = 1; i < n; ++i)
            if (p[i] > mx) mx = p[i];
    }
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        if (host) p[i] = isfinite(p[i]) ? expf((p[i] - mx) / temperature) : 0.0f;
        else p[i] = expf(p[i] - mx);
        sum += p[i];
    }
    if (host && (!(sum > 0.0f) || !isfinite(sum))) {
        result = -3;
        goto done;
    }
    for (int i = 0; i < n; ++i) p[i] /= sum;
    const float coin = sample_coin(rng_state);
    if (top_p <= 0.0f || top_p >= 1.0f) {
        float cdf = 0.0f;
        result = n - 1;
        for (int i = 0; i < n; ++i) {
            cdf += p[i];
            if (coin < cdf) {
                result = i;
                break;
            }
        }
        goto done;
    }
    {
        const float cutoff = (1.0f - top_p) / (float)(n - 1);
        SampleCand* c = (SampleCand*)malloc(sizeof(SampleCand) * (size_t)n);
        int m = 0;
        for (int i = 0; i < n; ++i)
            if (p[i] >= cutoff) {
                c[m].p = p[i];
                c[m].i = i;
                ++m;
            }
        if (m == 0) {
            result = sample_argmax_host(p, n);
            free(c);
            goto done;
        }
        qsort(c, (size_t)m, sizeof(SampleCand), cand_desc);
        float cum = 0.0f;
        int last;
        if (host) {
            for (last = 0; last < m; ++last) {
                cum += c[last].p;
                if (cum >= top_p) break;
            }
            if (last > m - 1) last = m - 1;
        } else {
            last = m - 1;
            for (int i = 0; i < m; ++i) {
                cum += c[i].p;
                if (cum > top_p) {
                    last = i;
                    break;
                }
            }
        }
        const float target = coin * cum;
        float cdf = 0.0f;
        result = c[last].i;
        for (int i = 0; i <= last; ++i) {
            cdf += c[i].p;
            if (target < cdf) {
                result = c[i].i;
                break;
            }
        }
        free(c);
    }
done:
    free(p);
    free(pen);
    return result;
}

void i4o_float_to_q17_array(const float* x, int n, int32_t* out) {
    for (int i = 0; i < n; ++i) out[i] = i4o_float_to_q17(x[i]);
}

void i4o_expf_array(const float* x, float* y, size_t n) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) y[i] = expf(x[i]);
}
