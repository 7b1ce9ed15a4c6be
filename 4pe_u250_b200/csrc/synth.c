/*
 * synth.c -- seeded synthetic model images in the reference's on-disk format.
 *
 * The reference decodes real AutoRound checkpoints that are not available
 * here, so every test and benchmark uses seeded random weights written in
 * the exact bank format that scripts/autoround_pack_llama2_u250.py:114-189
 * produces (W4G128 superblocks: 128 Q1.15 scale words then 4096 weight
 * words, norm words first).  Both the CUDA path and the CPU oracle consume
 * the same images.
 *
 * Random streams are a counter hash (splitmix64 finaliser) of
 * (seed, stream, index), so any element can be regenerated independently and
 * the fill parallelises without changing the result.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define DIM 4096
#define HIDDEN 11008
#define PHIDDEN 11264
#define VOCAB 32000
#define PVOCAB 32256
#define SB_WORDS 4224
#define NORM_WORDS 4160

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static inline uint64_t hash3(uint64_t seed, uint64_t stream, uint64_t idx) {
    return mix64(mix64(seed * 0xD1B54A32D192ED03ULL ^ mix64(stream)) + idx);
}

static inline double unit_double(uint64_t h) { return (double)(h >> 11) * (1.0 / 9007199254740992.0); }

/* ---- geometry (autoround_pack_llama2_u250.py:59-99) ---- */
static int rows_of(int mode) { return (mode <= 3 || mode == 6) ? DIM : (mode <= 5 ? PHIDDEN : PVOCAB); }
static int cols_of(int mode) { return mode == 6 ? PHIDDEN : DIM; }
static int valid_rows(int mode) { return (mode == 4 || mode == 5) ? HIDDEN : (mode == 7 ? VOCAB : DIM); }
static int valid_cols(int mode) { return mode == 6 ? HIDDEN : DIM; }
static int data_words(int mode) { return rows_of(mode) / 128 * (cols_of(mode) / 1024) / 16 * SB_WORDS; }

uint64_t i4s_matrix_byte_offset(int layer, int mode) {
    uint64_t stride = 0;
    for (int m = 0; m < 7; ++m) stride += (uint64_t)data_words(m);
    uint64_t off = NORM_WORDS;
    if (mode == 7) off += 32ULL * stride;
    else {
        off += (uint64_t)layer * stride;
        for (int m = 0; m < mode; ++m) off += (uint64_t)data_words(m);
    }
    return off * 64ULL;
}

/* ---- element generators ---- */

/* INT4 weight uniform in [-8, 7]; zero in the padded rows/columns, as the
 * reference packer pads (autoround_pack_llama2_u250.py:477-485, 279-283). */
int i4s_weight(uint64_t seed, int layer, int mode, int row, int col) {
    if (row >= valid_rows(mode) || col >= valid_cols(mode)) return 0;
    const uint64_t idx = ((uint64_t)row * (uint64_t)cols_of(mode) + (uint64_t)col);
    const uint64_t h = hash3(seed, 1 + (uint64_t)layer * 8 + (uint64_t)mode, idx >> 4);
    return (int)((h >> ((idx & 15) * 4)) & 15) - 8;
}

/* Per (row, 128-column group) scale uniform in [0.002, 0.02], stored Q1.15
 * as round(s * 32768) (read_ar_matrix, autoround_pack_llama2_u250.py:413-424). */
int i4s_scale(uint64_t seed, int layer, int mode, int row, int g128) {
    if (row >= valid_rows(mode) || g128 * 128 >= valid_cols(mode)) return 0;
    const uint64_t idx = (uint64_t)row * (uint64_t)(cols_of(mode) / 128) + (uint64_t)g128;
    const double s = 0.002 + 0.018 * unit_double(hash3(seed, 1000 + (uint64_t)layer * 8 + (uint64_t)mode, idx));
    return (int)nearbyint(s * 32768.0);
}

/* Box-Muller normal sample; element i of stream `stream`. */
static double normal_at(uint64_t seed, uint64_t stream, uint64_t i) {
    const uint64_t h = hash3(seed, stream, i);
    const double u1 = ((double)(h >> 40) + 0.5) * (1.0 / 16777216.0);
    const double u2 = (double)(h & 0xFFFFFFULL) * (1.0 / 16777216.0);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

void i4s_fill_normal(float* out, uint64_t n, float mean, float std, uint64_t seed, uint64_t stream) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        out[i] = (float)(mean + std * normal_at(seed, stream, (uint64_t)i));
}

/* RMSNorm gamma ~ N(1, 0.05); which = 0 attention, 1 FFN, 2 final. */
void i4s_gamma(float* out, uint64_t seed, int layer, int which) {
    for (int i = 0; i < DIM; ++i)
        out[i] = (float)(1.0 + 0.05 * normal_at(seed, 5000 + (uint64_t)layer * 3 + (uint64_t)which, (uint64_t)i));
}

/* ---- packing (autoround_pack_llama2_u250.py:114-189) ----
 * tile t of this bank's matrix: out_tile = t / lit, local column tile t % lit,
 * global columns (bank*lit + t%lit)*256 + [0,256).  Superblock t/16 holds the
 * 8 scale words of its 16 tiles first (word w: rows 16w.., int16 slot
 * 2*(row%16)+g128), then 256 weight words per tile (word g*32+rb: column
 * lane l in bytes 2l, 2l+1 = (r0<<4)|r1, (r2<<4)|r3 of rows 4rb..4rb+3). */
static void pack_tile(uint8_t* dst, int t, int lit, const int8_t* tw /*128x256*/,
                      const int16_t* ts /*128x2*/) {
    uint8_t* blk = dst + (size_t)(t / 16) * SB_WORDS * 64;
    uint8_t* scl = blk + (size_t)(t % 16) * 8 * 64;
    uint8_t* wts = blk + 128 * 64 + (size_t)(t % 16) * 256 * 64;
    for (int w = 0; w < 8; ++w)
        for (int s = 0; s < 32; ++s) {
            const int row = 16 * w + s / 2;
            const int16_t v = ts[row * 2 + (s & 1)];
            memcpy(scl + w * 64 + s * 2, &v, 2);
        }
    for (int g = 0; g < 8; ++g)
        for (int rb = 0; rb < 32; ++rb) {
            uint8_t* word = wts + (size_t)(g * 32 + rb) * 64;
            for (int l = 0; l < 32; ++l) {
                const int c = g * 32 + l;
                const uint8_t n0 = (uint8_t)(tw[(4 * rb + 0) * 256 + c] & 15);
                const uint8_t n1 = (uint8_t)(tw[(4 * rb + 1) * 256 + c] & 15);
                const uint8_t n2 = (uint8_t)(tw[(4 * rb + 2) * 256 + c] & 15);
                const uint8_t n3 = (uint8_t)(tw[(4 * rb + 3) * 256 + c] & 15);
                word[2 * l] = (uint8_t)((n0 << 4) | n1);
                word[2 * l + 1] = (uint8_t)((n2 << 4) | n3);
            }
        }
}

/* Pack dense arrays w[M][K] (int8 in [-8,7]) and s[M][K/128] (Q1.15) for one
 * bank; M and K are the padded sizes.  Mirrors pack_matrix_to_super_blocks. */
void i4s_pack_arrays(const int8_t* w, const int16_t* s, int M, int K, int bank,
                     int out_tiles, int lit, uint8_t* dst) {
    /* Only whole superblocks are written, as block_count = tiles // 16 in the
     * reference packer (autoround_pack_llama2_u250.py:119-120). */
    const int tiles = out_tiles * lit / 16 * 16;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tiles; ++t) {
        int8_t tw[128 * 256];
        int16_t ts[256];
        const int r0 = (t / lit) * 128, c0 = (bank * lit + t % lit) * 256;
        for (int r = 0; r < 128; ++r) {
            for (int c = 0; c < 256; ++c)
                tw[r * 256 + c] = (r0 + r < M && c0 + c < K) ? w[(size_t)(r0 + r) * K + c0 + c] : 0;
            for (int g = 0; g < 2; ++g)
                ts[r * 2 + g] = (r0 + r < M && c0 / 128 + g < K / 128) ? s[(size_t)(r0 + r) * (K / 128) + c0 / 128 + g] : 0;
        }
        pack_tile(dst, t, lit, tw, ts);
    }
}

/* Write one synthetic matrix (layer, mode) into all four bank images. */
void i4s_fill_matrix(uint8_t* const banks[4], int layer, int mode, uint64_t seed) {
    const int lit = cols_of(mode) / 1024, out_tiles = rows_of(mode) / 128;
    const uint64_t off = i4s_matrix_byte_offset(layer, mode);
    for (int p = 0; p < 4; ++p) {
        uint8_t* dst = banks[p] + off;
#pragma omp parallel for schedule(static)
        for (int t = 0; t < out_tiles * lit; ++t) {
            int8_t tw[128 * 256];
            int16_t ts[256];
            const int r0 = (t / lit) * 128, c0 = (p * lit + t % lit) * 256;
            for (int r = 0; r < 128; ++r) {
                for (int c = 0; c < 256; ++c) tw[r * 256 + c] = (int8_t)i4s_weight(seed, layer, mode, r0 + r, c0 + c);
                for (int g = 0; g < 2; ++g) ts[r * 2 + g] = (int16_t)i4s_scale(seed, layer, mode, r0 + r, c0 / 128 + g);
            }
            pack_tile(dst, t, lit, tw, ts);
        }
    }
}

/* Norm region: layer l attention gamma at word l*128, FFN at l*128+64, final
 * at 4096; bank p holds columns [1024p, 1024p+1024) (py:460-472, 496-503). */
void i4s_fill_norms(uint8_t* const banks[4], int layers, uint64_t seed) {
    float g[DIM];
    for (int l = 0; l <= layers; ++l)
        for (int which = 0; which < 3; ++which) {
            if ((l == layers) != (which == 2)) continue;
            i4s_gamma(g, seed, which == 2 ? 0 : l, which);
            const uint64_t word = which == 2 ? 4096ULL : (uint64_t)l * 128ULL + (which == 1 ? 64ULL : 0ULL);
            for (int p = 0; p < 4; ++p) memcpy(banks[p] + word * 64ULL, g + p * 1024, 4096);
        }
}

/* Layers [0, layers) plus the LM head and the norm words. */
void i4s_fill_model(uint8_t* const banks[4], int layers, uint64_t seed) {
    i4s_fill_norms(banks, layers, seed);
    for (int l = 0; l < layers; ++l)
        for (int m = 0; m < 7; ++m) i4s_fill_matrix(banks, l, m, seed);
    i4s_fill_matrix(banks, 0, 7, seed);
}
