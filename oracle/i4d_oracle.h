/*
 * i4d_oracle.h -- CPU restatement of the reference per-token decode arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * may load it, and only to check or time the reference algorithm; the product
 * library (libi4d) never links or calls it.
 *
 * Every function restates one reference function; the citation is
 * path:line inside the reference project (dungnx3112/4PE_U250).
 * Parity of this restatement is pinned by
 *   - rope_lut.bin (the only committed binary fixture of the reference),
 *   - the bit-exact FP32 partial-sum known-answer test of
 *     testbench/tb_linear_hardened_rtl.cpp:19-104,
 *   - the attention + KV FNV-1a hashes of
 *     _rtl_check/linear_4pe_reduction_cosim/tb_attention_pe0_kv_rtl.cpp:109-110,
 *   - and by running the reference emulator itself (oracle/_ref) on the same
 *     inputs.
 */
#ifndef I4D_ORACLE_H
#define I4D_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Geometry: software_sim/llama2_decoder_sw_emulator.cpp:27-54,
 * kernel_HLS/int4_types.hpp:33-56, kernel_HLS/int4_model_layout.hpp:151-173. */
#define I4O_DIM 4096
#define I4O_HIDDEN 11008
#define I4O_PHIDDEN 11264
#define I4O_VOCAB 32000
#define I4O_PVOCAB 32256
#define I4O_HEADS 32
#define I4O_HEAD_DIM 128
#define I4O_BANKS 4
#define I4O_LOCAL_HEADS 8
#define I4O_GROUP 32
#define I4O_MAX_SEQ 4096
#define I4O_LAYERS 32
#define I4O_WORD_BYTES 64
#define I4O_NORM_WORDS 4160
#define I4O_BANK_WORDS 13516736ULL
#define I4O_BANK_BYTES (I4O_BANK_WORDS * 64ULL)
#define I4O_SUPERBLOCK_WORDS 4224
#define I4O_KV_RECORD_BYTES 320
#define I4O_ROPE_BYTES 2097152

/* Linear modes: kernel_HLS/int4_types.hpp:152-177. */
enum { I4O_Q = 0, I4O_K, I4O_V, I4O_O, I4O_GATE, I4O_UP, I4O_DOWN, I4O_LOGITS };

/* Per-mode geometry (rows, cols, local input tiles, output tiles, data words,
 * word offset of the matrix inside the bank image).
 * emulator:786-797, autoround_pack_llama2_u250.py:59-99. */
int i4o_mode_rows(int mode);
int i4o_mode_cols(int mode);
int i4o_mode_local_in_tiles(int mode);
int i4o_mode_out_tiles(int mode);
int i4o_mode_data_words(int mode);
uint64_t i4o_matrix_word_offset(int layer, int mode);
uint64_t i4o_norm_word_offset(int layer, int which /* 0 attn, 1 ffn, 2 final */);

/* emulator:167-210 (== int4_decoder_blocks.cpp:22-73).  q[n], e8m0[n/32]
 * where the E8M0 byte is max_exp+127 and the scale is 2^(byte-140). */
void i4o_quantize_g32(const float* x, int n, int16_t* q, uint8_t* e8m0);

/* emulator:427-453: 8 cyclic slots per 1024-column bank, pair tree, then
 * normalize * gamma and quantize.  Also returns the reciprocal when recip!=0. */
void i4o_rmsnorm_quantize(const float* x, const float* gamma, int16_t* q,
                          uint8_t* e8m0, float* recip);

/* One bank's linear stage over its superblock stream: emulator:216-264 with
 * the unpacking of emulator:799-892.  act_q / act_e8m0 are the bank-local
 * activations (local_in_tiles*256 values).  hls_zero_start != 0 starts the
 * per-row chain from the first contribution (int4_linear_controller.cpp
 * :763-812, tb_linear_hardened_rtl.cpp:97), otherwise from +0.0f as the
 * emulator does. */
void i4o_linear_bank(const uint8_t* superblocks, int out_tiles,
                     int local_in_tiles, const int16_t* act_q,
                     const uint8_t* act_e8m0, int hls_zero_start,
                     float* partial);

/* Full 4-bank GEMV: per-bank partials then (p0+p1)+(p2+p3).  banks[p] points
 * at the whole bank image.  emulator:216-264. */
void i4o_gemv(const uint8_t* const banks[4], int layer, int mode,
              const int16_t* act_q, const uint8_t* act_e8m0, float* y,
              float* partials /* optional [4][rows] */);

/* emulator:481-505 (== int4_linear_controller.cpp:38-80). */
int32_t i4o_float_to_q17(float value);

/* Decode rope_lut.bin into cos/sin [4096][64] Q1.17 (emulator:937-968). */
void i4o_decode_rope_lut(const uint8_t* lut, int32_t* cosv, int32_t* sinv);

/* Adjacent-pair RoPE on a 4096-vector at one position (emulator:526-541). */
void i4o_rope_q17(int32_t* vec, const int32_t* cos_pos, const int32_t* sin_pos);

/* KV group shift and INT8 quantizer (emulator:543-564). */
uint8_t i4o_kv_shift(const int32_t* values32);
int8_t i4o_kv_quant(int32_t raw, uint8_t shift);

/* exp LUT of the online softmax (emulator:575-595).  The 33-entry Q30 table is
 * round(2^(30+i/32)), computed here rather than transcribed. */
uint32_t i4o_exp_negative_q17(int32_t x);

/* Write one HLS KV record (swiftkv_attention.cpp:427-582) for a 128-vector. */
void i4o_kv_write_record(uint8_t* record, const int32_t* k, const int32_t* v);

/* SwiftKV attention over all 32 heads: emulator:602-714.  q and k are already
 * rotated.  kv is the HLS record store [bank][layer][local_head][token] with
 * `stride` token slots per (layer, head) and `layers` layers per bank.  The
 * current token's record is written before the scan, as the reference does. */
void i4o_attention(uint8_t* kv, int layers, int stride, int layer, int pos,
                   const int32_t* q, const int32_t* k, const int32_t* v,
                   int16_t* out_q, uint8_t* out_e8m0);

/* SwiGLU with the host C library's expf (emulator:716-722). */
void i4o_swiglu(const float* gate, const float* up, int n, float* out);

/* Gamma extraction from the bank norm region (emulator:970-990). */
void i4o_read_gamma(const uint8_t* const banks[4], int layer, int which,
                    float* gamma);

/* The token schedule (emulator:727-783).  residual is in/out (in = the
 * embedding row).  logits receives all 32256 padded rows. */
void i4o_forward(const uint8_t* const banks[4], const int32_t* rope_cos,
                 const int32_t* rope_sin, uint8_t* kv, int layers, int stride,
                 int pos, float* residual, float* logits);

/* Array helpers for the Python test harness. */
void i4o_float_to_q17_array(const float* x, int n, int32_t* out);
void i4o_expf_array(const float* x, float* y, size_t n); /* host C library expf */

/* emulator:1428-1438: index of the first strict maximum over n. */
int i4o_argmax(const float* logits, int n);

/* Negative log-likelihood of `target` as the emulator's perplexity loop
 * computes it (emulator:1902-1926): max_l = serial maximum from logits[0]
 * (strictly greater replaces), sum_exp = serial FP32 sum of expf(l - max_l)
 * from 0.0f, log_sum_exp = (double)(max_l + logf(sum_exp)) (float
 * arithmetic, then widened), nll = -((double)logits[target] - log_sum_exp).
 * max_out / sum_out (may be NULL) receive max_l and sum_exp. */
double i4o_nll(const float* logits, int n, int target, float* max_out, float* sum_out);

/* One sampler draw over logits[0, n), the state advanced in place.
 * mode 0: decode_host.cpp:724-868 (the hardware host's Sampler); mode 1:
 * emulator:1411-1569 (llama2.c's).  Top-p candidates are ordered by
 * probability, descending, equal probabilities by index (both references
 * leave that order to an unstable library sort).  Returns the token, or
 * -1 (every logit NaN), -2 (no finite logit), -3 (invalid probability sum):
 * the host's exceptions. */
int i4o_sample(int mode, const float* logits, int n, const int32_t* history, int n_history,
               float temperature, float top_p, float repeat_penalty, uint64_t* rng_state);

#ifdef __cplusplus
}
#endif
#endif
