/*
 * i4d.h -- C ABI of the B200-native INT4 Llama-2-7B batch-1 decode path.
 *
 * Drop-in for the per-token decode of the 4PE_U250 design: it consumes the
 * reference's unchanged model images (model_bank{0..3}.bin, rope_lut.bin,
 * embeddings.bin) and keeps its launch contract (scalar position in, logits
 * shards out).  Plain C: pointers and sizes only, integer status codes, no
 * exceptions cross this boundary.
 *
 * A context is not thread-safe; every call on it is serialised on the
 * context's CUDA stream and returns once its host buffers may be reused.
 * Reference interfaces replaced are cited as path:line inside the reference
 * project.
 */
#ifndef I4D_H
#define I4D_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int i4d_status;
#define I4D_OK 0
#define I4D_ERR_ARG 1     /* bad argument: range, null pointer, mode */
#define I4D_ERR_SIZE 2    /* buffer size differs from the format's size */
#define I4D_ERR_CUDA 3    /* a CUDA call failed (message in i4d_last_error) */
#define I4D_ERR_TIMEOUT 4 /* a bounded device-side wait gave up */
#define I4D_ERR_STATE 5   /* call out of order (e.g. decode before loading) */
#define I4D_ERR_NOMEM 6   /* device or pinned host allocation failed */

/* Geometry of the reference model (int4_types.hpp:33-56,
 * int4_model_layout.hpp:151-173, decode_host.cpp:63-119). */
#define I4D_DIM 4096
#define I4D_FFN 11264          /* 11008 padded to 44 x 256 */
#define I4D_VOCAB 32000
#define I4D_PADDED_VOCAB 32256 /* 4 logits shards of 8064 */
#define I4D_BANKS 4
#define I4D_LAYERS 32
#define I4D_MAX_POSITIONS 4096
#define I4D_BANK_BYTES 865071104ULL        /* dense image, 13,516,736 words */
#define I4D_LEGACY_BANK_BYTES 891277312ULL /* rejected, as decode_host does */
#define I4D_ROPE_BYTES 2097152ULL
#define I4D_KV_RECORD_BYTES 320            /* metadata, K0, K1, V0, V1 words */

/* Linear modes (int4_types.hpp:152-177). */
#define I4D_MODE_Q 0
#define I4D_MODE_K 1
#define I4D_MODE_V 2
#define I4D_MODE_O 3
#define I4D_MODE_GATE 4
#define I4D_MODE_UP 5
#define I4D_MODE_DOWN 6
#define I4D_MODE_LOGITS 7

/* Context flags. */
#define I4D_FLAG_NO_GRAPH 1u /* launch the token schedule eagerly */
#define I4D_FLAG_NO_PDL 2u   /* no programmatic dependent launch (staged path) */
#define I4D_FLAG_STAGED 4u   /* one kernel per stage instead of the persistent token kernel */

typedef struct i4d_ctx i4d_ctx;

typedef struct i4d_config {
    int device;       /* CUDA device ordinal */
    int num_layers;   /* decoder layers run per token, 1..32 (emulator g_num_layers) */
    int kv_capacity;  /* token slots per (layer, head), 1..4096; 0 = 4096 as the HLS */
    unsigned flags;   /* I4D_FLAG_* */
} i4d_config;

/* Creates a context on cfg->device and allocates its device memory (weights,
 * KV cache, workspace).  Replaces decode_host.cpp:1161-1294 (device open,
 * buffer allocation, KV zeroing). */
i4d_status i4d_create(const i4d_config* cfg, i4d_ctx** out);
void i4d_destroy(i4d_ctx* ctx);
/* Message of the last failing call on ctx (never NULL). */
const char* i4d_last_error(const i4d_ctx* ctx);

/* ---- Bank sharding across GPUs (one process per GPU) ----
 * The reference's four processing elements each hold one bank image and
 * exchange bank partials through its pair reducers and finalizer
 * (int4_linear_controller.cpp:1339-1439, int4_decoder_multikernel.hpp:11-65).
 * Here `world` contexts (2 or 4, one per GPU) split the banks: rank r holds
 * banks [r*4/world, (r+1)*4/world) and runs attention for their heads with
 * their KV records; the token kernel stores every bank partial into every
 * rank's memory over NVLink and counts arrivals in every rank's counters, so
 * each rank ends the step with the full residual and all logits, bit-exact
 * with a single context.  All ranks must decode the same positions and
 * inputs, step by step.
 *
 * i4d_create_shard: as i4d_create, for rank `rank` of `world` (world 1 is
 * i4d_create).  Only the banks it holds may be loaded.
 * i4d_shard_export: writes this context's handle (I4D_SHARD_HANDLE_BYTES,
 * opaque) for the other ranks.
 * i4d_shard_attach: takes all ranks' handles in rank order (world *
 * I4D_SHARD_HANDLE_BYTES bytes) and maps the peers; decoding needs it.
 * The per-kernel measurement hooks, i4d_gemv and i4d_attention are not
 * available on a shard (I4D_ERR_STATE). */
#define I4D_SHARD_HANDLE_BYTES 64
i4d_status i4d_create_shard(const i4d_config* cfg, int rank, int world, i4d_ctx** out);
i4d_status i4d_shard_export(i4d_ctx* ctx, void* handle, size_t n);
i4d_status i4d_shard_attach(i4d_ctx* ctx, const void* handles, size_t n);

/* Loads one unchanged bank image, from host or device memory (n must be
 * I4D_BANK_BYTES; the legacy
 * 891,277,312-byte layout is rejected with I4D_ERR_SIZE as
 * decode_host.cpp:1218-1227 detects it).  The image is re-tiled on the device
 * into the GEMV layout; gammas are extracted from its norm words.
 * Replaces load_bo_from_file(modelN, ...) decode_host.cpp:1261-1268. */
i4d_status i4d_load_bank(i4d_ctx* ctx, int bank, const void* bytes, size_t n);

/* Loads rope_lut.bin (n must be I4D_ROPE_BYTES).  Replaces
 * load_bo_from_file(ropeN, ...) decode_host.cpp:1282-1289. */
i4d_status i4d_load_rope(i4d_ctx* ctx, const void* bytes, size_t n);

/* Loads embeddings.bin (n_floats must be 32000*4096) into device memory.
 * Replaces load_embeddings, decode_host.cpp:1296. */
i4d_status i4d_load_embeddings(i4d_ctx* ctx, const float* emb, size_t n_floats);

/* One decode step: the reference launch contract of
 * int4_decoder_pe{0..3}_kernel (int4_decoder_multikernel.hpp:11-65) as driven
 * by run_one_token (decode_host.cpp:1340-1556).  residual_in is the
 * embedding row (the four 1024-float residual shards concatenated,
 * decode_host.cpp:666-676); logits_out receives the 32256 padded logits
 * (four 8064-float shards concatenated, decode_host.cpp:690-701);
 * residual_out (may be NULL) the final residual.  position must be below the
 * KV capacity; every position < `position` must already hold this
 * sequence's KV records. */
i4d_status i4d_decode_token(i4d_ctx* ctx, uint32_t position, const float* residual_in,
                            float* logits_out, float* residual_out);

/* Greedy step on the device (the embedding lookup and the argmax of
 * decode_host.cpp:666-676 and 703-717 moved onto the GPU): the input is row token_id of the embeddings loaded by i4d_load_embeddings, and
 * next_id receives the first index of the maximum of logits[0, 32000), NaN
 * skipped (-1 if every logit is NaN), as argmax_logits.  logits_out (may be
 * NULL) receives the 32256 padded logits.  Per step only the position and id
 * go to the device and the id back. */
i4d_status i4d_decode_greedy(i4d_ctx* ctx, uint32_t position, int32_t token_id, int32_t* next_id,
                             float* logits_out);

/* Prompt prefill in batches.  The reference feeds a prompt through
 * run_one_token one position at a time (decode_host.cpp:1570-1580),
 * streaming every weight once per token; here
 * up to 32 prompt tokens share each pass over the weights.  The result is
 * bit-identical to n calls of i4d_decode_token at positions position0 ..
 * position0 + n - 1: the same KV records of every token, and logits_out (may
 * be NULL) receives the last token's 32256 padded logits.  residuals_in:
 * n x 4096 FP32 embedding rows (host).  Needs a context holding all four
 * banks (not a shard); position0 + n must not exceed the KV capacity.  After
 * an error status the records of the prompt's positions are unspecified;
 * records before position0 are untouched. */
i4d_status i4d_prefill(i4d_ctx* ctx, uint32_t position0, const float* residuals_in, uint32_t n,
                       float* logits_out);

/* i4d_prefill from token ids (host, n ids in [0, 32000)) with the embeddings
 * of i4d_load_embeddings; next_id (may be NULL) receives the greedy next
 * token of the last position, as i4d_decode_greedy. */
i4d_status i4d_prefill_tokens(i4d_ctx* ctx, uint32_t position0, const int32_t* token_ids, uint32_t n,
                              int32_t* next_id, float* logits_out);

/* Perplexity terms of one evaluation chunk (the chunk loop body of
 * calculate_perplexity, emulator:1857-1927): token_ids[0..n),
 * 2 <= n, n - 1 <= KV capacity; positions 0 .. n-2 run as prompt batches
 * from position 0 (the chunk's cache restart), and nll_out[p] (n - 1
 * doubles) receives -(logits[ids[p+1]] - (double)(max_l + logf(sum_exp)))
 * with max_l the first maximum of the 32000 logits and sum_exp the serial
 * FP32 sum of expf(logit - max_l), in the emulator's types and order.  The
 * caller sums nll_out over chunks as the emulator does (total_nll / count,
 * exp of that).  Overwrites the context's KV records from position 0. */
i4d_status i4d_eval_nll(i4d_ctx* ctx, const int32_t* token_ids, uint32_t n, double* nll_out);

/* Bank-image producer on the device (scripts/autoround_pack_llama2_u250.py).
 * bank_images_dev: four device buffers of I4D_BANK_BYTES, the images being
 * built (i4d_load_bank accepts them as they are).
 * i4d_pack_autoround_matrix writes projection `mode` (0..6: Q, K, V, O, GATE,
 * UP, DOWN) of `layer` into all four images at the reference's offsets, from
 * the AutoRound export's raw data: nibbles_dev = uint8 [rows][cols/2] (column
 * 2i in the low nibble, offset binary) and scales_dev = FP32 [rows][cols/128]
 * for the unpadded shape (GATE/UP 11008 x 4096, DOWN 4096 x 11008, others
 * 4096 x 4096).  It unpacks as read_ar_matrix (:413-424), permutes Q/K rows
 * as permute_qk_rows (:101-113), pads, and lays out superblocks as
 * pack_matrix_to_super_blocks (:115-188).  Norm words are plain FP32 copies
 * the caller writes.  i4d_pack_fp32_head quantises an FP32 LM head
 * (32000 x 4096, device) with the max-abs RTN of pack_logits_into_banks
 * (:268-307) and packs it; it allocates 137 MB of scratch for the call.
 * Both return when the images are written.  Scales outside Q1.15 saturate as
 * the reference's clip; NaN inputs are not supported. */
i4d_status i4d_pack_autoround_matrix(i4d_ctx* ctx, int layer, int mode, const uint8_t* nibbles_dev,
                                     const float* scales_dev, uint8_t* const bank_images_dev[4]);
i4d_status i4d_pack_fp32_head(i4d_ctx* ctx, const float* head_dev, uint8_t* const bank_images_dev[4]);

/* Token sampler (temperature, top-p, repeat penalty) on the device.
 * Replaces the host's Sampler (decode_host.cpp:724-868, mode
 * I4D_SAMPLER_HOST) and also reproduces the emulator's llama2.c sampler
 * (emulator:1411-1569, mode I4D_SAMPLER_EMULATOR).  Temperature 0 is greedy.
 * A top_p outside (0, 1) samples the whole softmax (multinomial). Only
 * rng_state changes between draws: each draw that flips a coin advances it,
 * as the reference's member state does. */
#define I4D_SAMPLER_HOST 0
#define I4D_SAMPLER_EMULATOR 1
typedef struct i4d_sampler {
    float temperature;
    float top_p;
    float repeat_penalty; /* 1: off; applied once per distinct token of the history */
    int32_t mode;         /* I4D_SAMPLER_HOST or I4D_SAMPLER_EMULATOR */
    uint64_t rng_state;   /* xorshift64* state */
} i4d_sampler;

/* Fills *s as the reference's constructors do (the host sampler replaces a
 * zero seed by 1, decode_host.cpp:731; the emulator keeps it). */
void i4d_sampler_init(i4d_sampler* s, float temperature, float top_p, float repeat_penalty, uint64_t seed,
                      int32_t mode);

/* One draw over logits_dev[0, 32000) (a device pointer, e.g. the logits of
 * i4d_decode_token_async); history (host, n_history <= 16384 ids; ids outside
 * the vocabulary are ignored) feeds the repeat penalty.  Writes the token and
 * advances s->rng_state.  The host sampler's exceptions (all logits NaN, none
 * finite, invalid probability sum) return I4D_ERR_ARG.  Top-p candidates with
 * exactly equal probabilities are taken in index order, where the references'
 * unstable library sorts leave the order unspecified.  One CTA; the serial
 * sums and walks of the references stay serial (FP32 addition is not
 * associative). */
i4d_status i4d_sample(i4d_ctx* ctx, const float* logits_dev, const int32_t* history, uint32_t n_history,
                      i4d_sampler* s, int32_t* token_out);

/* i4d_decode_greedy with the sampler in place of the argmax: one decode step
 * from token_id at position, then one draw (as i4d_sample) over its logits,
 * all on the device; per step only the position, the id and the history go to
 * the device and the id and state back (no logits).  Needs i4d_load_embeddings. */
i4d_status i4d_decode_sample(i4d_ctx* ctx, uint32_t position, int32_t token_id, const int32_t* history,
                             uint32_t n_history, i4d_sampler* s, int32_t* next_id);

/* Device-resident form of i4d_decode_token for pipelines that keep their
 * data on the GPU: residual_in_dev / logits_out_dev are device pointers
 * (4096 / 32256 floats).  The step is only enqueued on the context stream;
 * i4d_sync waits for it and reports device-side errors.  No reference
 * counterpart (the XRT host always stages through host memory). */
i4d_status i4d_decode_token_async(i4d_ctx* ctx, uint32_t position, const float* residual_in_dev,
                                  float* logits_out_dev);

/* The context's CUDA stream (a cudaStream_t), for callers that record their
 * own events around i4d_decode_token_async.  No reference counterpart. */
void* i4d_stream(i4d_ctx* ctx);

/* Measurement hook: runs one step eagerly with a CUDA event pair around every
 * kernel and returns the device time per kernel class in kernel_ms[8] and the
 * launch counts in launches[8]: 0 QKV GEMV, 1 attention, 2 O GEMV,
 * 3 GATE/UP GEMV, 4 DOWN GEMV, 5 LOGITS GEMV, 6 RMS (staged path),
 * 7 persistent token kernel.  No reference
 * counterpart (decode_host's verbose timing, decode_host.cpp:1539-1553, is
 * host-side only). */
i4d_status i4d_profile_token(i4d_ctx* ctx, uint32_t position, const float* residual_in_dev,
                             float* kernel_ms, uint32_t* launches);

/* Measurement hook for the persistent token kernel: runs one step with
 * per-CTA cycle counters and returns the CTA-averaged microseconds (at the
 * device's nominal clock) of: 0..4 waiting for the input of the QKV, O,
 * GATE/UP, DOWN and LM-head stages, 5..9 building their activations,
 * 10..14 their chunk loops, 15 attention waits for QKV, 16 attention work,
 * 17 producer blocked on a full ring, 18 whole kernel, 19..23 thread 0's
 * release fence and counter arrival after each stage, and per consumer warp
 * (averaged over warps) for each stage s: 24+4s waiting for ring data,
 * 25+4s waiting for a contribution slot, 26+4s chunk arithmetic, 27+4s row
 * chains.  n_out >= 44.  No reference counterpart. */
i4d_status i4d_token_breakdown(i4d_ctx* ctx, uint32_t position, const float* residual_in_dev, float* us_out,
                               int n_out);

/* Measurement hook for the persistent token kernel: runs one step (with
 * detail != 0 the instrumented kernel, which also records per-warp stamps)
 * and returns, per CTA, global-timer stamps (ns) of 24 events of `layer`: for
 * the QKV, O, GATE/UP, DOWN and LM-head stages s, 4s+0 begin, 4s+1 input
 * ready, 4s+2 chunk loop start, 4s+3 arrival; 20..22 attention start, QKV
 * ready, end (CTAs with an attention item); 23 the producer's first copy of
 * the layer; then counts, not times: 24+s copies of stage s already landed
 * when its chunk loop starts, 29+s copies of stage s; 34+8w+k for consumer
 * warp w in the QKV stage: k < 6 the time of its k-th unit grab, 6 its loop
 * exit, 7 its number of grabs; 162+q / 186+q (q < 24) the times copy q of
 * the GATE/UP stage was issued by the producer / found landed by a compute
 * warp.  out holds max_ctas x 210 values; *n_ctas receives the grid size.
 * No reference counterpart. */
i4d_status i4d_token_timeline(i4d_ctx* ctx, uint32_t position, const float* residual_in_dev, int layer,
                              int detail, uint64_t* out, int max_ctas, int* n_ctas);

/* Clears the KV cache (decode_host.cpp:1291-1294 zero_bo). */
i4d_status i4d_kv_reset(i4d_ctx* ctx);
/* Reads / writes one 320-byte KV record in the HLS layout
 * (swiftkv_attention.hpp:21-36): bank, layer, local head 0..7, token. */
i4d_status i4d_kv_read(i4d_ctx* ctx, int bank, int layer, int local_head, int token, void* record);
i4d_status i4d_kv_write(i4d_ctx* ctx, int bank, int layer, int local_head, int token, const void* record);
/* Writes the records of tokens [token0, token0 + n) of one (bank, layer,
 * local head) from n x 320 contiguous host bytes, in one copy: restoring a
 * saved cache, or a synthetic context for the attention measurements.  The
 * HLS host fills the cache through its KV buffer object the same way
 * (decode_host.cpp:1291-1294). */
i4d_status i4d_kv_write_tokens(i4d_ctx* ctx, int bank, int layer, int local_head, int token0, int n,
                               const void* records);
/* Waits for all work on the context. */
i4d_status i4d_sync(i4d_ctx* ctx);

/* ---- Op-level entry points (the per-stage services of the reference) ---- */

/* One bank's linear stage over a raw superblock stream (n_bytes =
 * out_tiles*local_in_tiles/16 superblocks): FP32 partials of every output
 * row, chained over the bank's G32 groups in order.  Replaces
 * int4_linear_local_stage_peN (int4_linear_controller.hpp:50-62).
 * act_q: local_in_tiles*256 INT14 values; act_e8m0: one E8M0 byte per G32
 * group (scale 2^(byte-140)).  hls_zero_start != 0 starts each row chain
 * from its first contribution as the HLS does; 0 starts from +0.0f as the
 * software emulator does (they differ only in the sign of an all-zero sum). */
i4d_status i4d_linear_bank(i4d_ctx* ctx, const void* superblocks, size_t n_bytes,
                           int local_in_tiles, int out_tiles, const int16_t* act_q,
                           const uint8_t* act_e8m0, int hls_zero_start, float* partial_out);

/* i4d_linear_bank without any allocation, for callers that must not allocate
 * once they are running: a serving loop whose device memory is reserved up
 * front, or one that shares the GPU with other streams (cudaFree waits for
 * the whole device, so a per-call free stalls them).  No counterpart in the
 * reference.  Same arithmetic and result as i4d_linear_bank, but every buffer
 * is a device pointer (superblocks_dev and act_q_dev 2-byte aligned,
 * partial_out_dev 4-byte aligned) and the re-tiled weights go to a fixed
 * 5,947,392-byte static device array (22 superblocks: any bank slice of a
 * decoder-layer matrix); a larger stream, such as the LM head's, is rejected
 * with I4D_ERR_SIZE.  The array's device error word is cleared at the start
 * of each call; nothing else needs to start at zero.  The first call on a
 * device looks up the array's address (cudaGetSymbolAddress), so make that
 * first call before any stream capture.  The call is synchronous: it reads
 * the caller's device buffers on the context's stream without waiting for
 * any other stream, so superblocks_dev, act_q_dev and act_e8m0_dev must be
 * fully written before the call (e.g. synchronise the stream that wrote
 * them), and it returns once its own work has finished.  The array is
 * shared by every context of a
 * device: calls that overlap on one device, from any thread or context,
 * race on it and must be serialised by the caller. */
i4d_status i4d_linear_bank_noalloc(i4d_ctx* ctx, const void* superblocks_dev, size_t n_bytes,
                                   int local_in_tiles, int out_tiles, const int16_t* act_q_dev,
                                   const uint8_t* act_e8m0_dev, int hls_zero_start,
                                   float* partial_out_dev);

/* Full 4-bank GEMV of a loaded matrix: y = (p0+p1)+(p2+p3) (pair reducers and
 * finalizer, int4_linear_controller.hpp:64-93; emulator sharded_gemv_4pe).
 * partials_out ([4][rows], may be NULL) receives the per-bank partials. */
i4d_status i4d_gemv(i4d_ctx* ctx, int layer, int mode, const int16_t* act_q,
                    const uint8_t* act_e8m0, float* y_out, float* partials_out);

/* G32 E8M0/INT14 activation quantizer (int4_decoder_blocks.cpp:22-73); n % 32 == 0. */
i4d_status i4d_quantize_g32(i4d_ctx* ctx, const float* x, int n, int16_t* q, uint8_t* e8m0);

/* RMSNorm + quantize of a 4096 residual (int4_local_sumsq, pair schedule and
 * int4_local_rms_normalize_quantize, int4_decoder_blocks.hpp:77-125). */
i4d_status i4d_rms_quant(i4d_ctx* ctx, const float* x, const float* gamma, int16_t* q,
                         uint8_t* e8m0);

/* SwiftKV attention of one layer at `position` (int4_swiftkv_attention_pe0..3,
 * swiftkv_attention.hpp:167-209): q, k, v are the Q15.17 projections before
 * RoPE (4096 each); RoPE, the KV record write and the scan run on the device.
 * Output: INT14[4096] + E8M0[128] for the O projection. */
i4d_status i4d_attention(i4d_ctx* ctx, int layer, uint32_t position, const int32_t* q,
                         const int32_t* k, const int32_t* v, int16_t* out_q, uint8_t* out_e8m0);

/* SwiGLU + quantize over 11264 rows (int4_local_swiglu_quantize,
 * int4_decoder_blocks.cpp:487-521). */
i4d_status i4d_swiglu_quant(i4d_ctx* ctx, const float* gate, const float* up, int16_t* q,
                            uint8_t* e8m0);

/* The device argmax of i4d_decode_greedy over a host buffer of n <= 32256
 * values (test hook). */
i4d_status i4d_argmax(i4d_ctx* ctx, const float* logits, size_t n, int32_t* index);

/* The device expf used by SwiGLU, element-wise (test hook: its results must
 * equal the host C library's expf, which the reference emulator calls). */
i4d_status i4d_expf(i4d_ctx* ctx, const float* x, float* y, size_t n);

/* Build target of the loaded device code and the GPU it runs on, queried at
 * run time: *binary_version = the token kernel's binary architecture (100
 * for an sm_100a build), *device_cc = the device's compute capability as
 * 10 * major + minor.  No counterpart in the reference (an FPGA build checks
 * its xclbin at load, decode_host.cpp:1189). */
i4d_status i4d_device_arch(int device, int* binary_version, int* device_cc);

/* Measurement hooks of the op-level kernels, on the context's stream, timed
 * with CUDA events (no counterpart in the reference; the FPGA design reports
 * only per-token latency, docs/thesis/main.tex:410-414).
 * i4d_profile_gemv: `reps` back-to-back GEMVs of `mode`, layer r mod
 * num_layers for the r-th (a different matrix each time, so a model of more
 * than 126 MB of such matrices streams each from HBM), fixed activations;
 * *ms_per_gemv = elapsed / reps.  The GEMV of sharded_gemv_4pe,
 * emulator:216-264.
 * i4d_profile_attention: the attention step of one layer at `position` over
 * the records in the KV cache (swiftkv_attention_4pe, emulator:602-714).
 * With fill > 0 it first runs the step at every position below `position`
 * with q/k/v row p % fill of qkv_dev ([fill][3][4096] Q15.17, device), so
 * the cache holds records of those rows; then times `reps` steps at
 * `position` with row 0. */
i4d_status i4d_profile_gemv(i4d_ctx* ctx, int mode, int reps, float* ms_per_gemv);
i4d_status i4d_profile_attention(i4d_ctx* ctx, int layer, uint32_t position, const int32_t* qkv_dev, int fill,
                                 int reps, float* ms_per_step);

#ifdef __cplusplus
}
#endif
#endif
