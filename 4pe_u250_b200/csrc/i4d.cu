// i4d.cu -- host runtime and C ABI of libi4d (see include/i4d.h).
//
// One context = one GPU, one CUDA stream.  The token schedule of
// int4_decoder_controller.cpp:138-234 (RMS -> QKV -> attention -> O+residual
// -> RMS -> GATE/UP -> SwiGLU -> DOWN+residual, 32 layers, final RMS ->
// LOGITS) is 5 kernels per layer plus 2, launched with programmatic dependent
// launch so every GEMV kernel streams its weights while the previous kernel
// finishes, and captured once as a CUDA graph whose position lives in device
// memory.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "i4d.h"
#include "i4d_attention.cuh"
#include "i4d_blocks.cuh"
#include "i4d_linear.cuh"
#include "i4d_token.cuh"
#include "i4d_sample.cuh"
#include "i4d_pack.cuh"
#include "i4d_prefill.cuh"

extern "C" {
extern const unsigned int i4d_expf_fix_count;
extern const unsigned int i4d_expf_fix[];
extern const char i4d_expf_fix_libc[];
}

using namespace i4d;

namespace {

// Stage kinds of the GEMV layout.
enum Stage { ST_QKV = 0, ST_O, ST_GU, ST_DOWN, ST_LOGITS, ST_COUNT };
constexpr int kStageUnits[ST_COUNT] = {384, 128, 704, 128, 1008};
constexpr int kStageChunks[ST_COUNT] = {4, 4, 4, 11, 4};
constexpr size_t kSmemBudget = 115712;  // two CTAs per SM

size_t stage_bank_bytes(int st) {
    return static_cast<size_t>(kStageUnits[st]) * kStageChunks[st] * kChunkBytes;
}

// Reference geometry (emulator:786-797, autoround_pack_llama2_u250.py:59-99).
int mode_rows(int m) { return (m <= 3 || m == 6) ? 4096 : (m <= 5 ? 11264 : 32256); }
int mode_lit(int m) { return m == 6 ? 11 : 4; }
uint64_t mode_words(int m) { return static_cast<uint64_t>(mode_rows(m) / 128) * mode_lit(m) / 16 * 4224; }
uint64_t matrix_word_offset(int layer, int m) {
    uint64_t stride = 0;
    for (int i = 0; i < 7; ++i) stride += mode_words(i);
    uint64_t off = 4160;
    if (m == 7) return off + 32ull * stride;
    off += static_cast<uint64_t>(layer) * stride;
    for (int i = 0; i < m; ++i) off += mode_words(i);
    return off;
}
int mode_stage(int m) { return m <= 2 ? ST_QKV : (m == 3 ? ST_O : (m <= 5 ? ST_GU : (m == 6 ? ST_DOWN : ST_LOGITS))); }
int mode_unit_offset(int m) { return m <= 2 ? m * 128 : (m == 5 ? 352 : 0); }

int32_t host_float_to_q17(float value) {
    uint32_t bits;
    std::memcpy(&bits, &value, 4);
    const bool neg = (bits >> 31) != 0;
    const uint32_t e = (bits >> 23) & 0xffu;
    if (e < 109) return 0;
    if (e >= 141) return neg ? INT32_MIN : INT32_MAX;
    const uint32_t sig = (1u << 23) | (bits & 0x7fffffu);
    uint64_t mag;
    if (e >= 133) {
        mag = static_cast<uint64_t>(sig) << (e - 133);
    } else {
        const unsigned sh = 133 - e;
        uint32_t q = sig >> sh;
        const uint32_t rem = sig & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        mag = q;
    }
    if (!neg) return mag > 0x7fffffffull ? INT32_MAX : static_cast<int32_t>(mag);
    return mag >= (1ull << 31) ? INT32_MIN : -static_cast<int32_t>(mag);
}

}  // namespace

struct i4d_ctx {
    int device = 0, layers = 32, stride = 4096, num_sms = 148, cpb = 37;
    // Bank sharding: this context holds banks [bank0, bank0 + nbanks) of a
    // group of `world` contexts, one per GPU (world 1: all four banks).
    int rank = 0, world = 1, nbanks = 4, bank0 = 0;
    bool attached = false;                   // peers mapped (world > 1)
    void* d_shared = nullptr;                // partials + synchronisation words, exported to peers
    float* peer_partials[4] = {};
    unsigned* peer_sync[4] = {};
    void* peer_base[4] = {};                 // opened IPC mappings
    unsigned flags = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    // weights (GEMV layout), norms, tables
    uint8_t* d_w = nullptr;
    size_t w_bytes = 0;
    float* d_gamma = nullptr;  // [65][4096]: attn l at 2l, ffn l at 2l+1, final at 64
    int32_t* d_rope_cos = nullptr;
    int32_t* d_rope_sin = nullptr;
    uint32_t* d_exp2 = nullptr;
    uint32_t* d_expf_slots = nullptr;
    ExpfFix expf{};
    int log2e_q21 = 0;
    int32_t score_scale = 0;
    uint8_t* d_kv = nullptr;
    size_t kv_bytes = 0;
    float* d_emb = nullptr;
    // workspace
    float* d_resid = nullptr;
    float* d_recip = nullptr;
    float* d_partials = nullptr;
    int16_t* d_ao_q = nullptr;
    uint8_t* d_ao_e = nullptr;
    int16_t* d_ad_q = nullptr;
    uint8_t* d_ad_e = nullptr;
    float* d_logits = nullptr;
    unsigned* d_counters = nullptr;
    unsigned* d_err = nullptr;
    int* d_pos = nullptr;
    int* d_tok = nullptr;                    // greedy: input token id
    unsigned long long* d_argmax = nullptr;  // greedy: argmax key of the step's logits
    uint32_t* d_attn_coef = nullptr;  // [128][stride] attention coefficients
    unsigned* d_sync = nullptr;       // persistent-kernel synchronisation words
    float* d_recips = nullptr;        // [65] RMS reciprocal of every norm of a token
    float* d_scratch = nullptr;  // op-level staging, 3 x 32256 floats
    // pinned staging for the decode contract
    float* h_resid_in = nullptr;
    float* h_resid_out = nullptr;
    float* h_logits = nullptr;
    int* h_pos = nullptr;
    int* h_tok = nullptr;
    unsigned long long* h_argmax = nullptr;
    // Sampler: history, radix-sort scratch, state and result words.
    int* d_sample_hist = nullptr;
    uint32_t* d_sample_keys = nullptr;
    uint32_t* d_sample_idx = nullptr;
    unsigned long long* d_sample_state = nullptr;
    int* d_sample_out = nullptr;
    float* d_sample_v = nullptr;
    float* d_sample_smax = nullptr;
    unsigned long long* h_sample_state = nullptr;
    int* h_sample_out = nullptr;
    unsigned* h_err = nullptr;
    // Prompt batches (i4d_prefill): per-token residuals, RMS reciprocals,
    // quantised activations, stage partials, rotated q, attention
    // coefficients and positions of up to kPrefillMax tokens.
    float* d_pf_resid = nullptr;
    float* d_pf_recip = nullptr;
    int16_t* d_pf_q = nullptr;
    uint8_t* d_pf_e = nullptr;
    float* d_pf_part = nullptr;
    int32_t* d_pf_qrot = nullptr;
    uint32_t* d_pf_coef = nullptr;
    int* d_pf_pos = nullptr;
    int* d_pf_ids = nullptr;
    int* d_pf_tgt = nullptr;      // perplexity: target id of every token of the batch
    float* d_pf_lg = nullptr;     // perplexity: [16][32000] logits / expf terms
    float* d_pf_terms = nullptr;  // perplexity: [16][4] max, sum, target logit
    float* h_pf_terms = nullptr;
    float* h_pf_resid = nullptr;
    int* h_pf_pos = nullptr;
    int* h_pf_ids = nullptr;
    bool bank_loaded[4] = {false, false, false, false};
    bool rope_loaded = false;
    cudaGraphExec_t graph = nullptr;       // H2D + token kernels + D2H
    cudaGraphExec_t graph_dev = nullptr;   // token kernels only
    cudaGraphExec_t graph_greedy = nullptr;  // token id in, next token id out
    // profiling: when set, enqueue_token brackets every kernel with events
    cudaEvent_t prof_ev[2 * 256] = {};
    int prof_class[256] = {};
    int prof_n = 0;
    bool profiling = false;
    unsigned long long* d_trace = nullptr;  // optional token-kernel trace
    unsigned long long* d_timeline = nullptr;  // optional token-kernel timeline
    int tl_layer = -1;
    bool tl_detail = false;
};

namespace {

i4d_status fail(i4d_ctx* c, i4d_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (c) c->err = buf;
    return st;
}

#define CK(call)                                                                        \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            return fail(c, I4D_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

size_t stage_offset(const i4d_ctx* c, int layer, int st) {
    size_t per_layer = 0;
    for (int s = 0; s < ST_LOGITS; ++s) per_layer += c->nbanks * stage_bank_bytes(s);
    if (st == ST_LOGITS) return static_cast<size_t>(c->layers) * per_layer;
    size_t off = static_cast<size_t>(layer) * per_layer;
    for (int s = 0; s < st; ++s) off += c->nbanks * stage_bank_bytes(s);
    return off;
}

// Units in flight per CTA (FP32 contribution buffers): about 24 KB of them.
int contrib_slots(int chunks) {
    const int per_unit = chunks * 8 * 32 * 4;
    const int nu = 24576 / per_unit;
    return nu < 2 ? 2 : nu;
}

int ring_slots(int chunks) {
    const size_t fixed = linear_smem_bytes(0, chunks, contrib_slots(chunks));
    return static_cast<int>((kSmemBudget - fixed - 16) / (kChunkBytes + 16 + 4));
}

template <typename Kern, typename... Args>
cudaError_t launch(i4d_ctx* c, bool pdl, Kern kern, dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    if (pdl && !(c->flags & I4D_FLAG_NO_PDL)) {
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    return e;
}

LinearArgs base_linear(i4d_ctx* c, int layer, int st) {
    LinearArgs a = {};
    a.w = c->d_w + stage_offset(c, layer, st);
    a.bank_stride = stage_bank_bytes(st);
    a.nbanks = 4;
    a.cpb = c->cpb;
    a.units = kStageUnits[st];
    a.chunks = kStageChunks[st];
    a.ns = ring_slots(a.chunks);
    a.nu = contrib_slots(a.chunks);
    a.partials = c->d_partials;
    a.counters = c->d_counters;
    a.expf = c->expf;
    a.err = c->d_err;
    return a;
}

cudaError_t run_linear(i4d_ctx* c, const LinearArgs& a, bool pdl) {
    const size_t smem = linear_smem_bytes(a.ns, a.chunks, a.nu);
    return launch(c, pdl, k_linear, dim3(a.nbanks * a.cpb), dim3(kLinearThreads), smem, a);
}

AttnArgs base_attn(i4d_ctx* c, int layer) {
    AttnArgs a = {};
    a.partials = c->d_partials;
    a.pos_ptr = c->d_pos;
    a.rope_cos = c->d_rope_cos;
    a.rope_sin = c->d_rope_sin;
    a.exp2_q30 = c->d_exp2;
    a.log2e_q21 = c->log2e_q21;
    a.score_scale = c->score_scale;
    a.kv = c->d_kv;
    a.bank0 = c->bank0;
    a.layers = c->layers;
    a.stride = c->stride;
    a.layer = layer;
    a.coef_scratch = c->d_attn_coef;
    a.out_q = c->d_ao_q;
    a.out_e = c->d_ao_e;
    a.err = c->d_err;
    return a;
}

enum KernelClass { KC_QKV = 0, KC_ATTN, KC_O, KC_GU, KC_DOWN, KC_LOGITS, KC_RMS, KC_TOKEN, KC_COUNT };

cudaError_t prof_begin(i4d_ctx* c, int cls) {
    if (!c->profiling || c->prof_n >= 256) return cudaSuccess;
    c->prof_class[c->prof_n] = cls;
    return cudaEventRecord(c->prof_ev[2 * c->prof_n], c->stream);
}

cudaError_t prof_end(i4d_ctx* c) {
    if (!c->profiling || c->prof_n >= 256) return cudaSuccess;
    return cudaEventRecord(c->prof_ev[2 * c->prof_n++ + 1], c->stream);
}

#define TIMED(cls, call)        \
    do {                        \
        CK(prof_begin(c, cls)); \
        CK(call);               \
        CK(prof_end(c));        \
    } while (0)

TokenArgs token_args(i4d_ctx* c) {
    TokenArgs t = {};
    t.w = c->d_w;
    t.layer_bytes = stage_offset(c, 1, ST_QKV);
    for (int st = 0; st < ST_COUNT; ++st) {
        t.stage_off[st] = st == ST_LOGITS ? stage_offset(c, 0, ST_LOGITS) : stage_offset(c, 0, st);
        t.bank_bytes[st] = stage_bank_bytes(st);
    }
    t.layers = c->layers;
    t.cpb = c->cpb;
    t.bank0 = c->bank0;
    t.nbanks = c->nbanks;
    t.world = c->world;
    for (int p = 0; p < 4; ++p) {
        t.peer_partials[p] = c->peer_partials[p];
        t.peer_sync[p] = c->peer_sync[p];
    }
    t.epoch = c->d_sync + kSyncEpoch;
    t.emb = nullptr;
    t.token_in = nullptr;
    t.argmax = nullptr;
    t.resid = c->d_resid;
    t.gamma = c->d_gamma;
    t.partials = c->d_partials;
    t.ao_q = c->d_ao_q;
    t.ao_e = c->d_ao_e;
    t.logits = c->d_logits;
    t.sync = c->d_sync;
    t.attn = base_attn(c, 0);
    t.expf = c->expf;
    t.err = c->d_err;
    t.trace = c->d_trace;
    t.timeline = c->d_timeline;
    t.tl_layer = c->tl_layer;
    return t;
}

// One token as a single cooperative launch of the persistent kernel.
// After a failed step: the error word, counters and epoch back to zero.
// Ordered on the context's stream and waited for: a plain cudaMemset runs on
// the legacy stream, which does not order with the non-blocking context
// stream, so it could land inside the next step.
cudaError_t reset_sync(i4d_ctx* c) {
    cudaError_t e = cudaMemsetAsync(c->d_err, 0, sizeof(unsigned), c->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->d_sync, 0, kSyncWords * sizeof(unsigned), c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    return e;
}

cudaError_t launch_token_with(i4d_ctx* c, const TokenArgs& t) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c->nbanks * c->cpb);
    cfg.blockDim = dim3(kTokThreads);
    cfg.dynamicSmemBytes = tok_smem_bytes();
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // The measurement hooks run the instantiation with cycle counters and stamps.
    if (c->d_trace || (c->d_timeline && c->tl_detail)) return cudaLaunchKernelEx(&cfg, k_token<true>, t);
    return cudaLaunchKernelEx(&cfg, k_token<false>, t);
}

cudaError_t launch_token(i4d_ctx* c) { return launch_token_with(c, token_args(c)); }

// Greedy step: H2D position + token id, the token kernel with the embedding
// lookup and argmax, D2H argmax key + error word.
i4d_status enqueue_greedy(i4d_ctx* c) {
    CK(cudaMemcpyAsync(c->d_pos, c->h_pos, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_tok, c->h_tok, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    TokenArgs t = token_args(c);
    t.emb = c->d_emb;
    t.token_in = c->d_tok;
    t.argmax = c->d_argmax;
    CK(launch_token_with(c, t));
    CK(cudaMemcpyAsync(c->h_argmax, c->d_argmax, sizeof(unsigned long long), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream));
    return I4D_OK;
}

// The kernels of one token (position and residual already in device memory).
i4d_status enqueue_token(i4d_ctx* c) {
    if (!(c->flags & I4D_FLAG_STAGED)) {
        TIMED(KC_TOKEN, launch_token(c));
        return I4D_OK;
    }
    TIMED(KC_RMS, launch(c, false, k_rms_recip, dim3(1), dim3(32), 0, (const float*)c->d_resid, c->d_recip));
    for (int l = 0; l < c->layers; ++l) {
        LinearArgs q = base_linear(c, l, ST_QKV);
        q.in_kind = IN_RMS;
        q.resid = c->d_resid;
        q.gamma = c->d_gamma + static_cast<size_t>(2 * l) * kDim;
        q.recip = c->d_recip;
        q.epi = EPI_PARTIAL;
        TIMED(KC_QKV, run_linear(c, q, true));

        TIMED(KC_ATTN, launch(c, true, k_attention, dim3(kHeads), dim3(kAttnThreads), attn_smem_bytes(), base_attn(c, l)));

        LinearArgs o = base_linear(c, l, ST_O);
        o.in_kind = IN_ACT;
        o.act_q = c->d_ao_q;
        o.act_e = c->d_ao_e;
        o.act_bank_stride = 1024;
        o.epi = EPI_RESID;
        o.out = c->d_resid;
        o.recip_out = c->d_recip;
        TIMED(KC_O, run_linear(c, o, true));

        LinearArgs gu = base_linear(c, l, ST_GU);
        gu.in_kind = IN_RMS;
        gu.resid = c->d_resid;
        gu.gamma = c->d_gamma + static_cast<size_t>(2 * l + 1) * kDim;
        gu.recip = c->d_recip;
        gu.epi = EPI_SWIGLU;
        gu.q_out = c->d_ad_q;
        gu.e_out = c->d_ad_e;
        TIMED(KC_GU, run_linear(c, gu, true));

        LinearArgs dn = base_linear(c, l, ST_DOWN);
        dn.in_kind = IN_ACT;
        dn.act_q = c->d_ad_q;
        dn.act_e = c->d_ad_e;
        dn.act_bank_stride = 2816;
        dn.epi = EPI_RESID;
        dn.out = c->d_resid;
        dn.recip_out = c->d_recip;
        TIMED(KC_DOWN, run_linear(c, dn, true));
    }
    LinearArgs lg = base_linear(c, 0, ST_LOGITS);
    lg.in_kind = IN_RMS;
    lg.resid = c->d_resid;
    lg.gamma = c->d_gamma + static_cast<size_t>(64) * kDim;
    lg.recip = c->d_recip;
    lg.epi = EPI_STORE;
    lg.out = c->d_logits;
    TIMED(KC_LOGITS, run_linear(c, lg, true));
    return I4D_OK;
}

i4d_status enqueue_decode(i4d_ctx* c) {
    CK(cudaMemcpyAsync(c->d_resid, c->h_resid_in, kDim * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_pos, c->h_pos, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    const i4d_status st = enqueue_token(c);
    if (st != I4D_OK) return st;
    CK(cudaMemcpyAsync(c->h_logits, c->d_logits, kPVocab * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(c->h_resid_out, c->d_resid, kDim * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream));
    return I4D_OK;
}

i4d_status finish(i4d_ctx* c) {
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
    unsigned e = 0;
    CK(cudaMemcpy(&e, c->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost));
    if (e) {
        CK(reset_sync(c));
        if (e & kErrArg) return fail(c, I4D_ERR_ARG, "device rejected an argument (error word 0x%x)", e);
        return fail(c, I4D_ERR_TIMEOUT, "a bounded device wait gave up (error word 0x%x)", e);
    }
    return I4D_OK;
}

// One GEMV stage of a prompt batch (act: the batch's [T][kPfTok] activations).
cudaError_t run_batch(i4d_ctx* c, int layer, int st, int T, int act_bank_stride) {
    BatchArgs b = {};
    b.w = c->d_w + stage_offset(c, layer, st);
    b.bank_stride = stage_bank_bytes(st);
    b.cpb = c->cpb;
    b.units = kStageUnits[st];
    b.chunks = kStageChunks[st];
    b.T = T;
    b.act_q = c->d_pf_q;
    b.act_e = c->d_pf_e;
    b.act_bank_stride = act_bank_stride;
    b.partials = c->d_pf_part;
    b.err = c->d_err;
    b.ns = batch_slots(b.chunks, T);
    if (b.ns < 2) return cudaErrorInvalidValue;
    return launch(c, true, k_linear_batch, dim3(4 * c->cpb), dim3(kBatchThreads),
                  batch_smem_bytes(b.chunks, T, b.ns), b);
}

cudaError_t run_pf_norm(i4d_ctx* c, int T, int partial_stage, const float* gamma) {
    PfNormArgs n = {};
    n.resid = c->d_pf_resid;
    n.partials = partial_stage < 0 ? nullptr : c->d_pf_part;
    n.rows = partial_stage < 0 ? 0 : kStageUnits[partial_stage] * 32;
    n.gamma = gamma;
    n.recip = c->d_pf_recip;
    n.q = c->d_pf_q;
    n.e = c->d_pf_e;
    return launch(c, true, k_pf_norm, dim3(T), dim3(1024), 0, n);
}

// The layers of one prompt batch of T tokens (residuals in d_pf_resid,
// positions in d_pf_pos), in the decode order of every token: norm, QKV,
// attention (records of all T tokens, then the T queries), O + residual,
// norm, GATE/UP, SwiGLU, DOWN + residual.  With `last`, the final norm and
// the LM head of the batch's last token follow (logits in d_logits); with
// `nll`, the final norm and LM head of every token and its perplexity terms
// (targets in d_pf_tgt, terms in d_pf_terms).
i4d_status enqueue_prefill(i4d_ctx* c, int T, bool last, bool nll) {
    for (int l = 0; l < c->layers; ++l) {
        CK(run_pf_norm(c, T, l == 0 ? -1 : ST_DOWN, c->d_gamma + static_cast<size_t>(2 * l) * kDim));
        CK(run_batch(c, l, ST_QKV, T, 1024));
        AttnArgs at = base_attn(c, l);
        at.partials = c->d_pf_part;
        at.part_tok_stride = static_cast<size_t>(4) * kStageUnits[ST_QKV] * 32;
        at.pos_ptr = c->d_pf_pos;
        at.q_rot = c->d_pf_qrot;
        at.coef_scratch = c->d_pf_coef;
        at.out_q = c->d_pf_q;
        at.out_e = c->d_pf_e;
        at.out_tok_stride = kPfTok;
        CK(launch(c, true, k_pf_kv, dim3(kHeads, T), dim3(128), 0, at));
        at.phase = 2;
        CK(launch(c, true, k_attention, dim3(kHeads, T), dim3(kAttnThreads), attn_smem_bytes(), at));
        CK(run_batch(c, l, ST_O, T, 1024));
        CK(run_pf_norm(c, T, ST_O, c->d_gamma + static_cast<size_t>(2 * l + 1) * kDim));
        CK(run_batch(c, l, ST_GU, T, 1024));
        CK(launch(c, true, k_pf_swiglu, dim3(kStageUnits[ST_GU] / 16, T), dim3(256), 0, (const float*)c->d_pf_part,
                  static_cast<int>(kStageUnits[ST_GU]), c->expf, c->d_pf_q, c->d_pf_e));
        CK(run_batch(c, l, ST_DOWN, T, 2816));
    }
    if (nll) {
        CK(run_pf_norm(c, T, ST_DOWN, c->d_gamma + static_cast<size_t>(64) * kDim));
        CK(run_batch(c, 0, ST_LOGITS, T, 1024));
        PfNllArgs na = {};
        na.partials = c->d_pf_part;
        na.lg = c->d_pf_lg;
        na.target = c->d_pf_tgt;
        na.terms = c->d_pf_terms;
        na.expf = c->expf;
        CK(launch(c, true, k_pf_logits, dim3(T), dim3(1024), 0, na));
        CK(launch(c, true, k_pf_exp, dim3((kVocab + 1023) / 1024, T), dim3(1024), 0, na));
        CK(launch(c, true, k_pf_sum, dim3(T), dim3(32), 0, na));
        return I4D_OK;
    }
    CK(run_pf_norm(c, T, ST_DOWN, nullptr));
    if (!last) return I4D_OK;
    CK(cudaMemcpyAsync(c->d_resid, c->d_pf_resid + static_cast<size_t>(T - 1) * kDim, kDim * sizeof(float),
                       cudaMemcpyDeviceToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_recip, c->d_pf_recip + (T - 1), sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    LinearArgs lg = base_linear(c, 0, ST_LOGITS);
    lg.in_kind = IN_RMS;
    lg.resid = c->d_resid;
    lg.gamma = c->d_gamma + static_cast<size_t>(64) * kDim;
    lg.recip = c->d_recip;
    lg.epi = EPI_STORE;
    lg.out = c->d_logits;
    CK(run_linear(c, lg, false));
    return I4D_OK;
}

bool all_loaded(const i4d_ctx* c) {
    for (int b = c->bank0; b < c->bank0 + c->nbanks; ++b)
        if (!c->bank_loaded[b]) return false;
    return c->rope_loaded && (c->world == 1 || c->attached);
}

}  // namespace

// ===================================================================== C ABI

extern "C" {

const char* i4d_last_error(const i4d_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

void i4d_destroy(i4d_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->graph) cudaGraphExecDestroy(c->graph);
    if (c->graph_dev) cudaGraphExecDestroy(c->graph_dev);
    if (c->graph_greedy) cudaGraphExecDestroy(c->graph_greedy);
    for (cudaEvent_t ev : c->prof_ev)
        if (ev) cudaEventDestroy(ev);
    for (void* p : c->peer_base)
        if (p) cudaIpcCloseMemHandle(p);
    void* dev[] = {c->d_w, c->d_gamma, c->d_rope_cos, c->d_rope_sin, c->d_exp2, c->d_expf_slots, c->d_kv,
                   c->d_emb, c->d_resid, c->d_recip, c->d_shared, c->d_ao_q, c->d_ao_e, c->d_ad_q,
                   c->d_ad_e, c->d_logits, c->d_counters, c->d_err, c->d_pos, c->d_scratch, c->d_attn_coef, c->d_recips, c->d_trace,
                   c->d_tok, c->d_argmax, c->d_sample_hist, c->d_sample_keys, c->d_sample_idx,
                   c->d_sample_state, c->d_sample_out, c->d_sample_v, c->d_sample_smax, c->d_pf_resid,
                   c->d_pf_recip, c->d_pf_q, c->d_pf_e, c->d_pf_part, c->d_pf_qrot, c->d_pf_coef, c->d_pf_pos,
                   c->d_pf_ids, c->d_pf_tgt, c->d_pf_lg, c->d_pf_terms};
    for (void* p : dev)
        if (p) cudaFree(p);
    void* host[] = {c->h_resid_in, c->h_resid_out, c->h_logits, c->h_pos, c->h_err, c->h_tok, c->h_argmax,
                    c->h_sample_state, c->h_sample_out, c->h_pf_resid, c->h_pf_pos, c->h_pf_ids, c->h_pf_terms};
    for (void* p : host)
        if (p) cudaFreeHost(p);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

static i4d_status create_impl(const i4d_config* cfg, int rank, int world, i4d_ctx** out) {
    if (!cfg || !out || (world != 1 && world != 2 && world != 4) || rank < 0 || rank >= world) return I4D_ERR_ARG;
    *out = nullptr;
    i4d_ctx* c = new i4d_ctx();
    c->rank = rank;
    c->world = world;
    c->nbanks = 4 / world;
    c->bank0 = rank * c->nbanks;
    c->device = cfg->device;
    c->layers = cfg->num_layers;
    c->stride = cfg->kv_capacity == 0 ? 4096 : cfg->kv_capacity;
    c->flags = cfg->flags;
    if (c->layers < 1 || c->layers > 32 || c->stride < 1 || c->stride > 4096) {
        i4d_destroy(c);
        return I4D_ERR_ARG;
    }
    auto bail = [&](i4d_status st) {
        // keep the message readable by the caller through a temporary context
        fprintf(stderr, "i4d_create: %s\n", c->err.c_str());
        i4d_destroy(c);
        return st;
    };
#define CKC(call)                                                                              \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess) {                                                               \
            fail(c, e_ == cudaErrorMemoryAllocation ? I4D_ERR_NOMEM : I4D_ERR_CUDA, "%s: %s", #call, \
                 cudaGetErrorString(e_));                                                      \
            return bail(e_ == cudaErrorMemoryAllocation ? I4D_ERR_NOMEM : I4D_ERR_CUDA);       \
        }                                                                                      \
    } while (0)
    CKC(cudaSetDevice(c->device));
    CKC(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, c->device));
    c->cpb = c->num_sms / c->nbanks > 0 ? c->num_sms / c->nbanks : 1;
    CKC(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    CKC(cudaFuncSetAttribute(k_linear, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBudget)));
    CKC(cudaFuncSetAttribute(k_attn_items, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(attn_items_smem_bytes())));
    CKC(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(attn_smem_bytes())));
    CKC(cudaFuncSetAttribute(k_linear_batch, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kBatchSmemMax));
    CKC(cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sample_smem_bytes())));
    CKC(cudaFuncSetAttribute(k_token<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(tok_smem_bytes())));
    CKC(cudaFuncSetAttribute(k_token<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(tok_smem_bytes())));
    {
        int per_sm = 0, per_sm_tr = 0;
        CKC(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_token<false>, kTokThreads, tok_smem_bytes()));
        CKC(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_tr, k_token<true>, kTokThreads, tok_smem_bytes()));
        if (per_sm < 1 || per_sm_tr < 1 || c->nbanks * c->cpb > c->num_sms) c->flags |= I4D_FLAG_STAGED;
        if (world > 1 && (c->flags & I4D_FLAG_STAGED)) {
            fail(c, I4D_ERR_STATE, "bank sharding needs the persistent token kernel");
            return bail(I4D_ERR_STATE);
        }
    }

    c->w_bytes = stage_offset(c, 0, ST_LOGITS) + c->nbanks * stage_bank_bytes(ST_LOGITS);
    CKC(cudaMalloc(&c->d_w, c->w_bytes));
    CKC(cudaMalloc(&c->d_gamma, 65ull * kDim * sizeof(float)));
    CKC(cudaMalloc(&c->d_rope_cos, 4096ull * 64 * sizeof(int32_t)));
    CKC(cudaMalloc(&c->d_rope_sin, 4096ull * 64 * sizeof(int32_t)));
    c->kv_bytes = static_cast<size_t>(c->nbanks) * c->layers * kLocalHeads * static_cast<size_t>(c->stride) * 320;
    CKC(cudaMalloc(&c->d_kv, c->kv_bytes));
    CKC(cudaMemset(c->d_kv, 0, c->kv_bytes));
    CKC(cudaMalloc(&c->d_resid, 2 * kDim * sizeof(float)));  // two buffers for the token kernel
    CKC(cudaMalloc(&c->d_recip, 16));
    // Partials (two buffers for the token kernel) and the synchronisation words
    // share one allocation, which the ranks of a sharded group map.
    const size_t partial_bytes = 2ull * kPartialBuf * sizeof(float);
    CKC(cudaMalloc(&c->d_shared, partial_bytes + kSyncWords * sizeof(unsigned)));
    c->d_partials = static_cast<float*>(c->d_shared);
    c->d_sync = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(c->d_shared) + partial_bytes);
    c->peer_partials[rank] = c->d_partials;
    c->peer_sync[rank] = c->d_sync;
    CKC(cudaMalloc(&c->d_ao_q, kDim * sizeof(int16_t)));
    CKC(cudaMalloc(&c->d_ao_e, kDim / 32));
    CKC(cudaMalloc(&c->d_ad_q, kFfn * sizeof(int16_t)));
    CKC(cudaMalloc(&c->d_ad_e, kFfn / 32));
    CKC(cudaMalloc(&c->d_logits, kPVocab * sizeof(float)));
    CKC(cudaMalloc(&c->d_counters, kCounterSlots * sizeof(unsigned)));
    CKC(cudaMemset(c->d_counters, 0, kCounterSlots * sizeof(unsigned)));
    CKC(cudaMalloc(&c->d_err, sizeof(unsigned)));
    CKC(cudaMemset(c->d_err, 0, sizeof(unsigned)));
    CKC(cudaMalloc(&c->d_pos, sizeof(int)));
    CKC(cudaMalloc(&c->d_tok, sizeof(int)));
    CKC(cudaMalloc(&c->d_argmax, sizeof(unsigned long long)));
    CKC(cudaMalloc(&c->d_attn_coef, 128ull * c->stride * sizeof(uint32_t)));
    CKC(cudaMemset(c->d_sync, 0, kSyncWords * sizeof(unsigned)));
    CKC(cudaMalloc(&c->d_recips, 80 * sizeof(float)));
    CKC(cudaMalloc(&c->d_scratch, 3ull * kPVocab * sizeof(float)));
    CKC(cudaMallocHost(&c->h_resid_in, kDim * sizeof(float)));
    CKC(cudaMallocHost(&c->h_resid_out, kDim * sizeof(float)));
    CKC(cudaMallocHost(&c->h_logits, kPVocab * sizeof(float)));
    CKC(cudaMallocHost(&c->h_pos, sizeof(int)));
    CKC(cudaMallocHost(&c->h_tok, sizeof(int)));
    CKC(cudaMallocHost(&c->h_argmax, sizeof(unsigned long long)));
    CKC(cudaMalloc(&c->d_sample_hist, kSampleMaxHistory * sizeof(int)));
    CKC(cudaMalloc(&c->d_sample_keys, 2ull * kSampleMaxVocab * sizeof(uint32_t)));
    CKC(cudaMalloc(&c->d_sample_idx, 2ull * kSampleMaxVocab * sizeof(uint32_t)));
    CKC(cudaMalloc(&c->d_sample_state, sizeof(unsigned long long)));
    CKC(cudaMalloc(&c->d_sample_out, sizeof(int)));
    CKC(cudaMalloc(&c->d_sample_v, kSampleMaxVocab * sizeof(float)));
    CKC(cudaMalloc(&c->d_sample_smax, kSampleSlices * sizeof(float)));
    CKC(cudaMallocHost(&c->h_sample_state, sizeof(unsigned long long)));
    CKC(cudaMallocHost(&c->h_sample_out, sizeof(int)));
    CKC(cudaMallocHost(&c->h_err, sizeof(unsigned)));
    CKC(cudaMalloc(&c->d_pf_resid, static_cast<size_t>(kPrefillMax) * kDim * sizeof(float)));
    CKC(cudaMalloc(&c->d_pf_recip, kPrefillMax * sizeof(float)));
    CKC(cudaMalloc(&c->d_pf_q, static_cast<size_t>(kPrefillMax) * kPfTok * sizeof(int16_t)));
    CKC(cudaMalloc(&c->d_pf_e, static_cast<size_t>(kPrefillMax) * kPfTok / 32));
    CKC(cudaMalloc(&c->d_pf_part, static_cast<size_t>(kPrefillMax) * 4 * kPVocab * sizeof(float)));
    CKC(cudaMalloc(&c->d_pf_qrot, static_cast<size_t>(kPrefillMax) * kDim * sizeof(int32_t)));
    CKC(cudaMalloc(&c->d_pf_coef, static_cast<size_t>(kPrefillMax) * kHeads * c->stride * sizeof(uint32_t)));
    CKC(cudaMalloc(&c->d_pf_pos, kPrefillMax * sizeof(int)));
    CKC(cudaMalloc(&c->d_pf_ids, kPrefillMax * sizeof(int)));
    CKC(cudaMallocHost(&c->h_pf_resid, static_cast<size_t>(kPrefillMax) * kDim * sizeof(float)));
    CKC(cudaMallocHost(&c->h_pf_pos, kPrefillMax * sizeof(int)));
    CKC(cudaMallocHost(&c->h_pf_ids, 2 * kPrefillMax * sizeof(int)));
    CKC(cudaMalloc(&c->d_pf_tgt, kPrefillMax * sizeof(int)));
    CKC(cudaMalloc(&c->d_pf_lg, static_cast<size_t>(kPrefillMax) * kVocab * sizeof(float)));
    CKC(cudaMalloc(&c->d_pf_terms, kPrefillMax * 4 * sizeof(float)));
    CKC(cudaMallocHost(&c->h_pf_terms, kPrefillMax * 4 * sizeof(float)));

    // exp2 LUT of the online softmax: round(2^(30 + i/32)), and log2(e) in
    // Q21 (emulator:566-579 define the same quantities).
    uint32_t lut[33];
    for (int i = 0; i <= 32; ++i) lut[i] = static_cast<uint32_t>(llroundl(exp2l(30.0L + i / 32.0L)));
    CKC(cudaMalloc(&c->d_exp2, sizeof(lut)));
    CKC(cudaMemcpyAsync(c->d_exp2, lut, sizeof(lut), cudaMemcpyHostToDevice, c->stream));
    c->log2e_q21 = static_cast<int>(std::nearbyint(1.4426950408889634 * static_cast<double>(1 << 21)));
    c->score_scale = host_float_to_q17(0.08838834764831845f);

    // Two-choice bucketed hash of the measured expf exceptions (layout in
    // i4d_expf.cuh); grows until every key has a bucket with room.
    std::vector<uint32_t> buckets;
    uint32_t nb = 1;
    while (nb < i4d_expf_fix_count / 2 + 1) nb <<= 1;
    for (;; nb <<= 1) {
        buckets.assign(8ull * nb, 0xffffffffu);
        std::vector<uint8_t> fill(nb, 0);
        bool ok = true;
        for (uint32_t i = 0; i < i4d_expf_fix_count && ok; ++i) {
            const uint32_t key = i4d_expf_fix[2 * i], val = i4d_expf_fix[2 * i + 1];
            const uint32_t b1 = expf_hash(key) & (nb - 1), b2 = expf_hash(key ^ kExpfSeed2) & (nb - 1);
            const uint32_t b = fill[b2] < fill[b1] ? b2 : b1;
            if (fill[b] == 4) {
                ok = false;
                break;
            }
            buckets[8ull * b + fill[b]] = key;
            buckets[8ull * b + 4 + fill[b]] = val;
            ++fill[b];
        }
        if (ok) break;
        if (nb >= (1u << 24)) {
            fail(c, I4D_ERR_STATE, "expf exception table does not fit");
            return bail(I4D_ERR_STATE);
        }
    }
    CKC(cudaMalloc(&c->d_expf_slots, buckets.size() * sizeof(uint32_t)));
    CKC(cudaMemcpyAsync(c->d_expf_slots, buckets.data(), buckets.size() * sizeof(uint32_t), cudaMemcpyHostToDevice,
                        c->stream));
    c->expf.buckets = c->d_expf_slots;
    c->expf.mask = nb - 1;
    // The initialising cudaMemset calls above run on the legacy stream, which
    // does not order with the context's non-blocking stream.
    CKC(cudaDeviceSynchronize());
#undef CKC
    *out = c;
    return I4D_OK;
}

i4d_status i4d_create(const i4d_config* cfg, i4d_ctx** out) { return create_impl(cfg, 0, 1, out); }

i4d_status i4d_create_shard(const i4d_config* cfg, int rank, int world, i4d_ctx** out) {
    return create_impl(cfg, rank, world, out);
}

i4d_status i4d_shard_export(i4d_ctx* c, void* handle, size_t n) {
    if (!c || !handle || n < I4D_SHARD_HANDLE_BYTES) return c ? fail(c, I4D_ERR_ARG, "bad handle buffer") : I4D_ERR_ARG;
    static_assert(sizeof(cudaIpcMemHandle_t) <= I4D_SHARD_HANDLE_BYTES, "IPC handle size");
    CK(cudaSetDevice(c->device));
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, c->d_shared));
    std::memset(handle, 0, I4D_SHARD_HANDLE_BYTES);
    std::memcpy(handle, &h, sizeof(h));
    return I4D_OK;
}

i4d_status i4d_shard_attach(i4d_ctx* c, const void* handles, size_t n) {
    if (!c || !handles) return c ? fail(c, I4D_ERR_ARG, "null handles") : I4D_ERR_ARG;
    if (n != static_cast<size_t>(c->world) * I4D_SHARD_HANDLE_BYTES)
        return fail(c, I4D_ERR_SIZE, "expected %d handles of %d bytes", c->world, I4D_SHARD_HANDLE_BYTES);
    if (c->attached) return fail(c, I4D_ERR_STATE, "peers already attached");
    CK(cudaSetDevice(c->device));
    const size_t partial_bytes = 2ull * kPartialBuf * sizeof(float);
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(p) * I4D_SHARD_HANDLE_BYTES, sizeof(h));
        void* ptr = nullptr;
        CK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        c->peer_base[p] = ptr;
        c->peer_partials[p] = static_cast<float*>(ptr);
        c->peer_sync[p] = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ptr) + partial_bytes);
    }
    if (c->graph) {
        cudaGraphExecDestroy(c->graph);
        c->graph = nullptr;
    }
    if (c->graph_dev) {
        cudaGraphExecDestroy(c->graph_dev);
        c->graph_dev = nullptr;
    }
    if (c->graph_greedy) {
        cudaGraphExecDestroy(c->graph_greedy);
        c->graph_greedy = nullptr;
    }
    c->attached = true;
    return I4D_OK;
}

i4d_status i4d_load_bank(i4d_ctx* c, int bank, const void* bytes, size_t n) {
    if (!c || !bytes || bank < 0 || bank > 3) return c ? fail(c, I4D_ERR_ARG, "bad bank or pointer") : I4D_ERR_ARG;
    if (n == I4D_LEGACY_BANK_BYTES)
        return fail(c, I4D_ERR_SIZE, "legacy 891,277,312-byte bank layout is not supported; repack dense");
    if (n != I4D_BANK_BYTES) return fail(c, I4D_ERR_SIZE, "bank image has %zu bytes; expected 865071104", n);
    if (bank < c->bank0 || bank >= c->bank0 + c->nbanks)
        return fail(c, I4D_ERR_ARG, "bank %d is not held by this shard (banks %d..%d)", bank, c->bank0,
                    c->bank0 + c->nbanks - 1);
    CK(cudaSetDevice(c->device));
    if (c->graph) {
        cudaGraphExecDestroy(c->graph);
        c->graph = nullptr;
    }
    if (c->graph_dev) {
        cudaGraphExecDestroy(c->graph_dev);
        c->graph_dev = nullptr;
    }
    if (c->graph_greedy) {
        cudaGraphExecDestroy(c->graph_greedy);
        c->graph_greedy = nullptr;
    }
    uint8_t* stage = nullptr;
    CK(cudaMalloc(&stage, n));
    // Stream-ordered: a plain cudaMemcpy from pageable memory may return
    // before its DMA lands, and the context stream does not wait for it.
    // The image may be in host or device memory (a bank packed on the GPU).
    cudaError_t e = cudaMemcpyAsync(stage, bytes, n, cudaMemcpyDefault, c->stream);
    for (int l = 0; e == cudaSuccess && l <= c->layers; ++l) {
        for (int m = 0; m < 8; ++m) {
            if ((l == c->layers) != (m == 7)) continue;
            const int st = mode_stage(m);
            RelayoutArgs r;
            r.src = stage + matrix_word_offset(l, m) * 64;
            r.dst = c->d_w + stage_offset(c, l, st) + static_cast<size_t>(bank - c->bank0) * stage_bank_bytes(st);
            r.unit_offset = mode_unit_offset(m);
            r.lit = mode_lit(m);
            k_relayout<<<mode_rows(m) / 32 * r.lit, 256, 0, c->stream>>>(r);
            e = cudaGetLastError();
            if (e != cudaSuccess) break;
        }
    }
    // Gammas: attention at word l*128, FFN at l*128+64, final at 4096.
    for (int l = 0; e == cudaSuccess && l < 32; ++l)
        for (int which = 0; which < 2 && e == cudaSuccess; ++which)
            e = cudaMemcpyAsync(c->d_gamma + static_cast<size_t>(2 * l + which) * kDim + bank * 1024,
                                stage + (static_cast<size_t>(l) * 128 + which * 64) * 64, 4096,
                                cudaMemcpyDeviceToDevice, c->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(c->d_gamma + 64ull * kDim + bank * 1024, stage + 4096ull * 64, 4096,
                            cudaMemcpyDeviceToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(stage);
    if (e != cudaSuccess) return fail(c, I4D_ERR_CUDA, "bank load: %s", cudaGetErrorString(e));
    c->bank_loaded[bank] = true;
    return I4D_OK;
}

i4d_status i4d_load_rope(i4d_ctx* c, const void* bytes, size_t n) {
    if (!c || !bytes) return c ? fail(c, I4D_ERR_ARG, "null rope pointer") : I4D_ERR_ARG;
    if (n != I4D_ROPE_BYTES) return fail(c, I4D_ERR_SIZE, "rope LUT has %zu bytes; expected 2097152", n);
    // Position p, pair i: 608-bit word p*4 + i/16 as two 64-byte words, lane
    // i%16 at bit 38*lane, 19-bit cosine then sine, Q1.17 (generate_rope_lut.py:20-41).
    const uint8_t* lut = static_cast<const uint8_t*>(bytes);
    std::vector<int32_t> cs(4096 * 64), sn(4096 * 64);
    for (int pos = 0; pos < 4096; ++pos)
        for (int pair = 0; pair < 64; ++pair) {
            const uint8_t* base = lut + (static_cast<size_t>(pos) * 4 + pair / 16) * 128;
            const int lane = pair % 16;
            for (int f = 0; f < 2; ++f) {
                uint32_t v = 0;
                for (int b = 0; b < 19; ++b) {
                    const int bit = lane * 38 + f * 19 + b;
                    v |= static_cast<uint32_t>((base[bit >> 3] >> (bit & 7)) & 1u) << b;
                }
                const int32_t sv = (v & (1u << 18)) ? static_cast<int32_t>(v | 0xfff80000u) : static_cast<int32_t>(v);
                (f == 0 ? cs : sn)[static_cast<size_t>(pos) * 64 + pair] = sv;
            }
        }
    CK(cudaSetDevice(c->device));
    CK(cudaMemcpyAsync(c->d_rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, c->stream));
    c->rope_loaded = true;
    return I4D_OK;
}

i4d_status i4d_load_embeddings(i4d_ctx* c, const float* emb, size_t n_floats) {
    if (!c || !emb) return c ? fail(c, I4D_ERR_ARG, "null embeddings") : I4D_ERR_ARG;
    if (n_floats != 32000ull * kDim) return fail(c, I4D_ERR_SIZE, "embeddings have %zu floats; expected 131072000", n_floats);
    CK(cudaSetDevice(c->device));
    if (!c->d_emb) CK(cudaMalloc(&c->d_emb, n_floats * sizeof(float)));
    CK(cudaMemcpyAsync(c->d_emb, emb, n_floats * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    return I4D_OK;
}

i4d_status i4d_decode_greedy(i4d_ctx* c, uint32_t position, int32_t token_id, int32_t* next_id, float* logits_out) {
    if (!c || !next_id) return c ? fail(c, I4D_ERR_ARG, "null next_id") : I4D_ERR_ARG;
    if (!all_loaded(c) || !c->d_emb)
        return fail(c, I4D_ERR_STATE, "banks, rope LUT and embeddings must be loaded before greedy decoding");
    if (c->flags & I4D_FLAG_STAGED) return fail(c, I4D_ERR_STATE, "greedy decoding needs the persistent token kernel");
    if (position >= static_cast<uint32_t>(c->stride))
        return fail(c, I4D_ERR_ARG, "position %u out of range (KV capacity %d)", position, c->stride);
    if (token_id < 0 || token_id >= kVocab) return fail(c, I4D_ERR_ARG, "token id %d out of range", token_id);
    CK(cudaSetDevice(c->device));
    *c->h_pos = static_cast<int>(position);
    *c->h_tok = token_id;
    *c->h_err = 0;
    if (c->flags & I4D_FLAG_NO_GRAPH) {
        const i4d_status st = enqueue_greedy(c);
        if (st != I4D_OK) return st;
    } else {
        if (!c->graph_greedy) {
            cudaGraph_t g = nullptr;
            CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
            const i4d_status st = enqueue_greedy(c);
            cudaError_t e = cudaStreamEndCapture(c->stream, &g);
            if (st != I4D_OK) {
                if (g) cudaGraphDestroy(g);
                return st;
            }
            if (e != cudaSuccess) return fail(c, I4D_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
            e = cudaGraphInstantiate(&c->graph_greedy, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) {
                c->graph_greedy = nullptr;
                return fail(c, I4D_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
            }
        }
        CK(cudaGraphLaunch(c->graph_greedy, c->stream));
    }
    CK(cudaStreamSynchronize(c->stream));
    if (*c->h_err) {
        const unsigned e = *c->h_err;
        CK(reset_sync(c));
        return fail(c, (e & kErrArg) ? I4D_ERR_ARG : I4D_ERR_TIMEOUT, "device error word 0x%x", e);
    }
    const unsigned long long k = *c->h_argmax;
    *next_id = k == 0ull ? -1 : static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(k & 0xffffffffu));
    if (logits_out) CK(cudaMemcpy(logits_out, c->d_logits, kPVocab * sizeof(float), cudaMemcpyDeviceToHost));
    return I4D_OK;
}

static i4d_status launch_pack(i4d_ctx* c, const PackArgs& a) {
    const long long threads = 4ll * a.blocks * kPackWordsPerBlock;
    k_pack_matrix<<<static_cast<unsigned>((threads + kPackThreads - 1) / kPackThreads), kPackThreads, 0, c->stream>>>(a);
    CK(cudaGetLastError());
    return I4D_OK;
}

static bool images_ok(uint8_t* const images[4]) {
    for (int p = 0; p < 4; ++p)
        if (!images[p]) return false;
    return true;
}

i4d_status i4d_pack_autoround_matrix(i4d_ctx* c, int layer, int mode, const uint8_t* nibbles_dev,
                                     const float* scales_dev, uint8_t* const bank_images_dev[4]) {
    if (!c || !nibbles_dev || !scales_dev || !bank_images_dev || !images_ok(bank_images_dev))
        return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (mode < 0 || mode > 6) return fail(c, I4D_ERR_ARG, "mode %d is not an AutoRound projection (0..6)", mode);
    if (layer < 0 || layer >= 32) return fail(c, I4D_ERR_ARG, "layer %d out of range", layer);
    CK(cudaSetDevice(c->device));
    PackArgs a = {};
    a.nib = nibbles_dev;
    a.scales = scales_dev;
    a.Mv = (mode == 4 || mode == 5) ? 11008 : 4096;
    a.Kv = mode == 6 ? 11008 : 4096;
    a.lit = mode_lit(mode);
    a.blocks = static_cast<int>(mode_words(mode) / kPackWordsPerBlock);
    a.permute_qk = mode <= 1;
    const uint64_t off = matrix_word_offset(layer, mode) * 64;
    for (int p = 0; p < 4; ++p) a.dst[p] = bank_images_dev[p] + off;
    const i4d_status st = launch_pack(c, a);
    if (st != I4D_OK) return st;
    CK(cudaStreamSynchronize(c->stream));
    return I4D_OK;
}

i4d_status i4d_pack_fp32_head(i4d_ctx* c, const float* head_dev, uint8_t* const bank_images_dev[4]) {
    if (!c || !head_dev || !bank_images_dev || !images_ok(bank_images_dev))
        return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    CK(cudaSetDevice(c->device));
    int8_t* w8 = nullptr;
    float* sc = nullptr;
    if (cudaMalloc(&w8, static_cast<size_t>(kPVocab) * 4096) != cudaSuccess ||
        cudaMalloc(&sc, static_cast<size_t>(kPVocab) * 32 * sizeof(float)) != cudaSuccess) {
        cudaFree(w8);
        return fail(c, I4D_ERR_NOMEM, "no device memory for the quantised head (137 MB)");
    }
    HeadQuantArgs q = {head_dev, kVocab, kPVocab, w8, sc};
    const long long threads = static_cast<long long>(kPVocab) * 32 * 32;
    k_quant_head<<<static_cast<unsigned>(threads / kPackThreads), kPackThreads, 0, c->stream>>>(q);
    cudaError_t e = cudaGetLastError();
    PackArgs a = {};
    a.w8 = w8;
    a.scales = sc;
    a.Mv = kPVocab;  // the padded rows are zero already
    a.Kv = 4096;
    a.lit = mode_lit(7);
    a.blocks = static_cast<int>(mode_words(7) / kPackWordsPerBlock);
    const uint64_t off = matrix_word_offset(0, 7) * 64;
    for (int p = 0; p < 4; ++p) a.dst[p] = bank_images_dev[p] + off;
    i4d_status st = e == cudaSuccess ? launch_pack(c, a) : I4D_ERR_CUDA;
    if (e == cudaSuccess && st == I4D_OK) e = cudaStreamSynchronize(c->stream);
    cudaFree(w8);
    cudaFree(sc);
    if (e != cudaSuccess) return fail(c, I4D_ERR_CUDA, "head packing: %s", cudaGetErrorString(e));
    return st;
}

void i4d_sampler_init(i4d_sampler* s, float temperature, float top_p, float repeat_penalty, uint64_t seed,
                      int32_t mode) {
    if (!s) return;
    s->temperature = temperature;
    s->top_p = top_p;
    s->repeat_penalty = repeat_penalty;
    s->mode = mode;
    // The host sampler never starts from a zero state (decode_host.cpp:731);
    // the emulator takes the seed as it is (emulator:1499).
    s->rng_state = (mode == I4D_SAMPLER_HOST && seed == 0) ? 1 : seed;
}

static i4d_status check_sampler(i4d_ctx* c, const int32_t* history, uint32_t n_history, const i4d_sampler* s) {
    if (!s) return fail(c, I4D_ERR_ARG, "null sampler");
    if (s->mode != I4D_SAMPLER_HOST && s->mode != I4D_SAMPLER_EMULATOR)
        return fail(c, I4D_ERR_ARG, "sampler mode %d unknown", s->mode);
    if (!(s->temperature >= 0.0f) || !(s->repeat_penalty > 0.0f) || s->top_p != s->top_p)
        return fail(c, I4D_ERR_ARG, "sampler parameters out of range (temperature %g, top_p %g, penalty %g)",
                    s->temperature, s->top_p, s->repeat_penalty);
    if (n_history > static_cast<uint32_t>(kSampleMaxHistory))
        return fail(c, I4D_ERR_SIZE, "history of %u tokens exceeds %d", n_history, kSampleMaxHistory);
    if (n_history && !history) return fail(c, I4D_ERR_ARG, "null history");
    return I4D_OK;
}

// Enqueues one draw over logits_dev[0, 32000) on the context stream.
static i4d_status enqueue_sample(i4d_ctx* c, const float* logits_dev, const int32_t* history, uint32_t n_history,
                                 const i4d_sampler* s) {
    if (n_history)
        CK(cudaMemcpyAsync(c->d_sample_hist, history, n_history * sizeof(int32_t), cudaMemcpyHostToDevice, c->stream));
    *c->h_sample_state = s->rng_state;
    CK(cudaMemcpyAsync(c->d_sample_state, c->h_sample_state, sizeof(unsigned long long), cudaMemcpyHostToDevice,
                       c->stream));
    SampleArgs a = {};
    a.logits = logits_dev;
    a.n = kVocab;
    a.history = c->d_sample_hist;
    a.n_history = static_cast<int>(n_history);
    a.temperature = s->temperature;
    a.top_p = s->top_p;
    a.penalty = s->repeat_penalty;
    a.mode = s->mode;
    a.state = c->d_sample_state;
    a.expf = c->expf;
    a.keys = c->d_sample_keys;
    a.idx = c->d_sample_idx;
    a.out = c->d_sample_out;
    a.v = c->d_sample_v;
    a.slice_max = c->d_sample_smax;
    k_sample_prep<<<kSampleSlices, kSampleThreads, 0, c->stream>>>(a);
    if (s->temperature != 0.0f) k_sample_exp<<<kSampleSlices, kSampleThreads, 0, c->stream>>>(a);
    k_sample<<<1, kSampleThreads, sample_smem_bytes(), c->stream>>>(a);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(c->h_sample_out, c->d_sample_out, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(c->h_sample_state, c->d_sample_state, sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                       c->stream));
    return I4D_OK;
}

// After the stream has finished: the token and the advanced state, or the
// host sampler's exceptions as errors.
static i4d_status finish_sample(i4d_ctx* c, i4d_sampler* s, int32_t* token_out) {
    const int r = *c->h_sample_out;
    if (r == kSampleAllNan) return fail(c, I4D_ERR_ARG, "all valid-vocabulary logits are NaN");
    if (r == kSampleNoFinite) return fail(c, I4D_ERR_ARG, "all valid-vocabulary logits are non-finite");
    if (r == kSampleBadSum) return fail(c, I4D_ERR_ARG, "invalid probability sum during sampling");
    s->rng_state = *c->h_sample_state;
    *token_out = r;
    return I4D_OK;
}

i4d_status i4d_sample(i4d_ctx* c, const float* logits_dev, const int32_t* history, uint32_t n_history,
                      i4d_sampler* s, int32_t* token_out) {
    if (!c || !logits_dev || !token_out) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    const i4d_status chk = check_sampler(c, history, n_history, s);
    if (chk != I4D_OK) return chk;
    CK(cudaSetDevice(c->device));
    const i4d_status st = enqueue_sample(c, logits_dev, history, n_history, s);
    if (st != I4D_OK) return st;
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
    return finish_sample(c, s, token_out);
}

i4d_status i4d_decode_sample(i4d_ctx* c, uint32_t position, int32_t token_id, const int32_t* history,
                             uint32_t n_history, i4d_sampler* s, int32_t* next_id) {
    if (!c || !next_id) return c ? fail(c, I4D_ERR_ARG, "null next_id") : I4D_ERR_ARG;
    if (!all_loaded(c) || !c->d_emb)
        return fail(c, I4D_ERR_STATE, "banks, rope LUT and embeddings must be loaded before sampled decoding");
    if (c->flags & I4D_FLAG_STAGED) return fail(c, I4D_ERR_STATE, "sampled decoding needs the persistent token kernel");
    if (position >= static_cast<uint32_t>(c->stride))
        return fail(c, I4D_ERR_ARG, "position %u out of range (KV capacity %d)", position, c->stride);
    if (token_id < 0 || token_id >= kVocab) return fail(c, I4D_ERR_ARG, "token id %d out of range", token_id);
    const i4d_status chk = check_sampler(c, history, n_history, s);
    if (chk != I4D_OK) return chk;
    CK(cudaSetDevice(c->device));
    *c->h_pos = static_cast<int>(position);
    *c->h_tok = token_id;
    *c->h_err = 0;
    i4d_status st = enqueue_greedy(c);
    if (st == I4D_OK) st = enqueue_sample(c, c->d_logits, history, n_history, s);
    if (st != I4D_OK) return st;
    CK(cudaStreamSynchronize(c->stream));
    if (*c->h_err) {
        const unsigned e = *c->h_err;
        CK(reset_sync(c));
        return fail(c, (e & kErrArg) ? I4D_ERR_ARG : I4D_ERR_TIMEOUT, "device error word 0x%x", e);
    }
    return finish_sample(c, s, next_id);
}

i4d_status i4d_decode_token(i4d_ctx* c, uint32_t position, const float* residual_in, float* logits_out,
                            float* residual_out) {
    if (!c || !residual_in || !logits_out) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (!all_loaded(c)) return fail(c, I4D_ERR_STATE, "banks and rope LUT must be loaded before decoding");
    if (position >= static_cast<uint32_t>(c->stride))
        return fail(c, I4D_ERR_ARG, "position %u out of range (KV capacity %d)", position, c->stride);
    CK(cudaSetDevice(c->device));
    std::memcpy(c->h_resid_in, residual_in, kDim * sizeof(float));
    *c->h_pos = static_cast<int>(position);
    *c->h_err = 0;
    if (c->flags & I4D_FLAG_NO_GRAPH) {
        const i4d_status st = enqueue_decode(c);
        if (st != I4D_OK) return st;
    } else {
        if (!c->graph) {
            cudaGraph_t g = nullptr;
            CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
            const i4d_status st = enqueue_decode(c);
            cudaError_t e = cudaStreamEndCapture(c->stream, &g);
            if (st != I4D_OK) {
                if (g) cudaGraphDestroy(g);
                return st;
            }
            if (e != cudaSuccess) return fail(c, I4D_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
            e = cudaGraphInstantiate(&c->graph, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) {
                c->graph = nullptr;
                return fail(c, I4D_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
            }
        }
        CK(cudaGraphLaunch(c->graph, c->stream));
    }
    CK(cudaStreamSynchronize(c->stream));
    if (*c->h_err) {
        const unsigned e = *c->h_err;
        CK(reset_sync(c));
        return fail(c, (e & kErrArg) ? I4D_ERR_ARG : I4D_ERR_TIMEOUT, "device error word 0x%x", e);
    }
    std::memcpy(logits_out, c->h_logits, kPVocab * sizeof(float));
    if (residual_out) std::memcpy(residual_out, c->h_resid_out, kDim * sizeof(float));
    return I4D_OK;
}

// Prompt of n tokens in batches of kPrefillMax; ids (device embeddings) or
// residuals (host) give each token's input.
static i4d_status prefill_impl(i4d_ctx* c, uint32_t position0, const float* residuals, const int32_t* ids,
                               uint32_t n, int32_t* next_id, float* logits_out, const int32_t* targets = nullptr,
                               double* nll_out = nullptr) {
    if (!all_loaded(c)) return fail(c, I4D_ERR_STATE, "banks and rope LUT must be loaded before a prefill");
    if (c->world != 1) return fail(c, I4D_ERR_STATE, "prefill needs all four banks in one context");
    if (ids && !c->d_emb) return fail(c, I4D_ERR_STATE, "embeddings must be loaded before a token prefill");
    if (n == 0) return fail(c, I4D_ERR_ARG, "empty prompt");
    if (position0 >= static_cast<uint32_t>(c->stride) || n > static_cast<uint32_t>(c->stride) - position0)
        return fail(c, I4D_ERR_ARG, "positions %u..%u out of range (KV capacity %d)", position0,
                    position0 + n - 1, c->stride);
    if (ids)
        for (uint32_t i = 0; i < n; ++i)
            if (ids[i] < 0 || ids[i] >= kVocab) return fail(c, I4D_ERR_ARG, "token id %d out of range", ids[i]);
    CK(cudaSetDevice(c->device));
    for (uint32_t b = 0; b < n; b += kPrefillMax) {
        const int T = static_cast<int>(n - b < static_cast<uint32_t>(kPrefillMax) ? n - b : kPrefillMax);
        const bool last = b + T == n;
        for (int t = 0; t < T; ++t) c->h_pf_pos[t] = static_cast<int>(position0 + b + t);
        CK(cudaMemcpyAsync(c->d_pf_pos, c->h_pf_pos, T * sizeof(int), cudaMemcpyHostToDevice, c->stream));
        if (ids) {
            std::memcpy(c->h_pf_ids, ids + b, T * sizeof(int));
            CK(cudaMemcpyAsync(c->d_pf_ids, c->h_pf_ids, T * sizeof(int), cudaMemcpyHostToDevice, c->stream));
            k_pf_embed<<<T, kDim / 4, 0, c->stream>>>(c->d_emb, c->d_pf_ids, c->d_pf_resid);
            CK(cudaGetLastError());
        } else {
            std::memcpy(c->h_pf_resid, residuals + static_cast<size_t>(b) * kDim, static_cast<size_t>(T) * kDim * sizeof(float));
            CK(cudaMemcpyAsync(c->d_pf_resid, c->h_pf_resid, static_cast<size_t>(T) * kDim * sizeof(float),
                               cudaMemcpyHostToDevice, c->stream));
        }
        if (targets) {  // staged in the second half of h_pf_ids
            std::memcpy(c->h_pf_ids + kPrefillMax, targets + b, T * sizeof(int));
            CK(cudaMemcpyAsync(c->d_pf_tgt, c->h_pf_ids + kPrefillMax, T * sizeof(int), cudaMemcpyHostToDevice,
                               c->stream));
        }
        const i4d_status st = enqueue_prefill(c, T, last && !targets, targets != nullptr);
        if (st != I4D_OK) return st;
        if (targets)
            CK(cudaMemcpyAsync(c->h_pf_terms, c->d_pf_terms, T * 4 * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
        if (last && next_id) {
            k_argmax<<<1, 1024, 0, c->stream>>>(c->d_logits, kVocab, c->d_argmax);
            CK(cudaGetLastError());
        }
        // The pinned staging is reused by the next batch.
        const i4d_status fs = finish(c);
        if (fs != I4D_OK) return fs;
        for (int t = 0; nll_out && t < T; ++t) {  // emulator:1922-1926, in its types
            const float* tm = c->h_pf_terms + 4 * t;
            const double log_sum_exp = tm[0] + std::log(tm[1]);
            const double log_prob = tm[2] - log_sum_exp;
            nll_out[b + t] = -log_prob;
        }
    }
    if (next_id) {
        unsigned long long k = 0;
        CK(cudaMemcpy(&k, c->d_argmax, sizeof(k), cudaMemcpyDeviceToHost));
        *next_id = k == 0ull ? -1 : static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(k & 0xffffffffu));
    }
    if (logits_out) CK(cudaMemcpy(logits_out, c->d_logits, kPVocab * sizeof(float), cudaMemcpyDeviceToHost));
    return I4D_OK;
}

i4d_status i4d_prefill(i4d_ctx* c, uint32_t position0, const float* residuals_in, uint32_t n, float* logits_out) {
    if (!c || !residuals_in) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    return prefill_impl(c, position0, residuals_in, nullptr, n, nullptr, logits_out);
}

i4d_status i4d_prefill_tokens(i4d_ctx* c, uint32_t position0, const int32_t* token_ids, uint32_t n,
                              int32_t* next_id, float* logits_out) {
    if (!c || !token_ids) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    return prefill_impl(c, position0, nullptr, token_ids, n, next_id, logits_out);
}

i4d_status i4d_eval_nll(i4d_ctx* c, const int32_t* token_ids, uint32_t n, double* nll_out) {
    if (!c || !token_ids || !nll_out) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (n < 2) return fail(c, I4D_ERR_ARG, "perplexity needs at least 2 tokens");
    for (uint32_t i = 0; i < n; ++i)
        if (token_ids[i] < 0 || token_ids[i] >= kVocab)
            return fail(c, I4D_ERR_ARG, "token id %d out of range", token_ids[i]);
    return prefill_impl(c, 0, nullptr, token_ids, n - 1, nullptr, nullptr, token_ids + 1, nll_out);
}

i4d_status i4d_kv_reset(i4d_ctx* c) {
    if (!c) return I4D_ERR_ARG;
    CK(cudaSetDevice(c->device));
    CK(cudaMemsetAsync(c->d_kv, 0, c->kv_bytes, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return I4D_OK;
}

static i4d_status kv_addr(i4d_ctx* c, int bank, int layer, int lh, int token, size_t* off) {
    if (bank < c->bank0 || bank >= c->bank0 + c->nbanks || layer < 0 || layer >= c->layers || lh < 0 || lh > 7 ||
        token < 0 || token >= c->stride)
        return fail(c, I4D_ERR_ARG, "KV record index out of range (or bank not held by this shard)");
    *off = ((((static_cast<size_t>(bank - c->bank0) * c->layers + layer) * kLocalHeads + lh) * c->stride) + token) * 320;
    return I4D_OK;
}

i4d_status i4d_kv_read(i4d_ctx* c, int bank, int layer, int lh, int token, void* record) {
    if (!c || !record) return c ? fail(c, I4D_ERR_ARG, "null record") : I4D_ERR_ARG;
    size_t off;
    const i4d_status st = kv_addr(c, bank, layer, lh, token, &off);
    if (st != I4D_OK) return st;
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(record, c->d_kv + off, 320, cudaMemcpyDeviceToHost));
    return I4D_OK;
}

i4d_status i4d_kv_write(i4d_ctx* c, int bank, int layer, int lh, int token, const void* record) {
    if (!c || !record) return c ? fail(c, I4D_ERR_ARG, "null record") : I4D_ERR_ARG;
    size_t off;
    const i4d_status st = kv_addr(c, bank, layer, lh, token, &off);
    if (st != I4D_OK) return st;
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpyAsync(c->d_kv + off, record, 320, cudaMemcpyHostToDevice, c->stream));
    return I4D_OK;
}

i4d_status i4d_kv_write_tokens(i4d_ctx* c, int bank, int layer, int lh, int token0, int n, const void* records) {
    if (!c || !records || n <= 0) return c ? fail(c, I4D_ERR_ARG, "bad records") : I4D_ERR_ARG;
    size_t off, last;
    i4d_status st = kv_addr(c, bank, layer, lh, token0, &off);
    if (st == I4D_OK) st = kv_addr(c, bank, layer, lh, token0 + n - 1, &last);
    if (st != I4D_OK) return st;
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(c->d_kv + off, records, static_cast<size_t>(n) * 320, cudaMemcpyHostToDevice));
    return I4D_OK;
}

i4d_status i4d_sync(i4d_ctx* c) {
    if (!c) return I4D_ERR_ARG;
    CK(cudaSetDevice(c->device));
    return finish(c);
}

void* i4d_stream(i4d_ctx* c) { return c ? static_cast<void*>(c->stream) : nullptr; }

static i4d_status capture(i4d_ctx* c, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const i4d_status st = enqueue_token(c);
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (st != I4D_OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (e != cudaSuccess) return fail(c, I4D_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        *out = nullptr;
        return fail(c, I4D_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    }
    return I4D_OK;
}

i4d_status i4d_decode_token_async(i4d_ctx* c, uint32_t position, const float* residual_in_dev,
                                  float* logits_out_dev) {
    if (!c || !residual_in_dev || !logits_out_dev) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (!all_loaded(c)) return fail(c, I4D_ERR_STATE, "banks and rope LUT must be loaded before decoding");
    if (position >= static_cast<uint32_t>(c->stride))
        return fail(c, I4D_ERR_ARG, "position %u out of range (KV capacity %d)", position, c->stride);
    CK(cudaSetDevice(c->device));
    k_set_pos<<<1, 1, 0, c->stream>>>(c->d_pos, static_cast<int>(position));
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(c->d_resid, residual_in_dev, kDim * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    if (c->flags & I4D_FLAG_NO_GRAPH) {
        const i4d_status st = enqueue_token(c);
        if (st != I4D_OK) return st;
    } else {
        if (!c->graph_dev) {
            const i4d_status st = capture(c, &c->graph_dev);
            if (st != I4D_OK) return st;
        }
        CK(cudaGraphLaunch(c->graph_dev, c->stream));
    }
    CK(cudaMemcpyAsync(logits_out_dev, c->d_logits, kPVocab * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    return I4D_OK;
}

i4d_status i4d_profile_token(i4d_ctx* c, uint32_t position, const float* residual_in_dev, float* kernel_ms,
                             uint32_t* launches) {
    if (c && c->world > 1) return fail(c, I4D_ERR_STATE, "not available on a bank shard");
    if (!c || !residual_in_dev || !kernel_ms || !launches) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (!all_loaded(c)) return fail(c, I4D_ERR_STATE, "banks and rope LUT must be loaded before decoding");
    if (position >= static_cast<uint32_t>(c->stride)) return fail(c, I4D_ERR_ARG, "position out of range");
    CK(cudaSetDevice(c->device));
    for (cudaEvent_t& ev : c->prof_ev)
        if (!ev) CK(cudaEventCreate(&ev));
    k_set_pos<<<1, 1, 0, c->stream>>>(c->d_pos, static_cast<int>(position));
    CK(cudaMemcpyAsync(c->d_resid, residual_in_dev, kDim * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    c->profiling = true;
    c->prof_n = 0;
    const i4d_status st = enqueue_token(c);
    c->profiling = false;
    if (st != I4D_OK) return st;
    const i4d_status st2 = finish(c);
    if (st2 != I4D_OK) return st2;
    for (int k = 0; k < KC_COUNT; ++k) {
        kernel_ms[k] = 0.0f;
        launches[k] = 0;
    }
    for (int i = 0; i < c->prof_n; ++i) {
        float ms = 0.0f;
        CK(cudaEventElapsedTime(&ms, c->prof_ev[2 * i], c->prof_ev[2 * i + 1]));
        kernel_ms[c->prof_class[i]] += ms;
        launches[c->prof_class[i]] += 1;
    }
    return I4D_OK;
}

}  // extern "C"

// ------------------------------------------------------ op-level entry points

namespace {
struct DevBuf {
    void* p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};
}  // namespace

#define DEVBUF(name, bytes) \
    DevBuf name;            \
    CK(cudaMalloc(&name.p, (bytes)))

namespace {

// ---- Scratch of i4d_linear_bank_noalloc ----
// A fixed device array replaces the per-call allocations of i4d_linear_bank:
// bytes [0, 4) are the call's device error word (cleared at the start of
// every call), the re-tiled weights start at byte 256.  22 superblocks
// (5,947,392 B) hold one bank's slice of the largest decoder-layer matrix
// (GATE, UP or DOWN; Q, K, V and O need 8); the LM head (63) does not fit.
constexpr size_t kNoAllocHeader = 256;
constexpr size_t kNoAllocMaxBytes = 22ull * 4224 * 64;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocHeader + kNoAllocMaxBytes];

constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[kNoAllocDevices];  // device address of the array, per device ordinal

// Once per device, with that device current: the array's device address.
i4d_status noalloc_scratch(i4d_ctx* c, uint8_t** out) {
    if (c->device < 0 || c->device >= kNoAllocDevices)
        return fail(c, I4D_ERR_ARG, "device ordinal %d out of range for the static scratch", c->device);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[c->device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(c, I4D_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch) failed: %s", cudaGetErrorString(e));
        g_noalloc_ptr[c->device] = static_cast<uint8_t*>(p);
    }
    *out = g_noalloc_ptr[c->device];
    return I4D_OK;
}

}  // namespace

extern "C" {

i4d_status i4d_linear_bank(i4d_ctx* c, const void* superblocks, size_t n_bytes, int lit, int out_tiles,
                           const int16_t* act_q, const uint8_t* act_e8m0, int hls_zero_start, float* partial_out) {
    if (!c || !superblocks || !act_q || !act_e8m0 || !partial_out) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (lit < 1 || lit > 11 || out_tiles < 1 || out_tiles > 1008 || (out_tiles * lit) % 16 != 0)
        return fail(c, I4D_ERR_ARG, "unsupported linear geometry: %d local input tiles, %d output tiles", lit, out_tiles);
    const size_t need = static_cast<size_t>(out_tiles) * lit / 16 * 4224 * 64;
    if (n_bytes != need) return fail(c, I4D_ERR_SIZE, "superblock stream has %zu bytes; expected %zu", n_bytes, need);
    CK(cudaSetDevice(c->device));
    DEVBUF(src, n_bytes);
    DEVBUF(gem, n_bytes);
    DEVBUF(aq, lit * 256 * sizeof(int16_t));
    DEVBUF(ae, lit * 8);
    CK(cudaMemcpyAsync(src.p, superblocks, n_bytes, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(aq.p, act_q, lit * 256 * sizeof(int16_t), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(ae.p, act_e8m0, lit * 8, cudaMemcpyHostToDevice, c->stream));
    RelayoutArgs r;
    r.src = src.as<uint8_t>();
    r.dst = gem.as<uint8_t>();
    r.unit_offset = 0;
    r.lit = lit;
    k_relayout<<<out_tiles * 4 * lit, 256, 0, c->stream>>>(r);
    CK(cudaGetLastError());
    LinearArgs a = {};
    a.w = gem.as<uint8_t>();
    a.bank_stride = 0;
    a.nbanks = 1;
    a.units = out_tiles * 4;
    a.cpb = a.units < c->num_sms ? a.units : c->num_sms;
    a.chunks = lit;
    a.ns = ring_slots(lit);
    a.nu = contrib_slots(lit);
    a.in_kind = IN_ACT;
    a.act_q = aq.as<int16_t>();
    a.act_e = ae.as<uint8_t>();
    a.act_bank_stride = 0;
    a.hls_zero = hls_zero_start ? 1 : 0;
    a.partials = c->d_partials;
    a.epi = EPI_PARTIAL;
    a.counters = c->d_counters;
    a.expf = c->expf;
    a.err = c->d_err;
    CK(run_linear(c, a, false));
    const i4d_status st = finish(c);
    if (st != I4D_OK) return st;
    CK(cudaMemcpy(partial_out, c->d_partials, static_cast<size_t>(out_tiles) * 128 * sizeof(float), cudaMemcpyDeviceToHost));
    return I4D_OK;
}

i4d_status i4d_linear_bank_noalloc(i4d_ctx* c, const void* superblocks_dev, size_t n_bytes, int lit, int out_tiles,
                                   const int16_t* act_q_dev, const uint8_t* act_e8m0_dev, int hls_zero_start,
                                   float* partial_out_dev) {
    if (!c) return I4D_ERR_ARG;
    if (!superblocks_dev || !act_q_dev || !act_e8m0_dev || !partial_out_dev) return fail(c, I4D_ERR_ARG, "null buffer");
    if ((reinterpret_cast<uintptr_t>(superblocks_dev) | reinterpret_cast<uintptr_t>(act_q_dev)) & 1 ||
        reinterpret_cast<uintptr_t>(partial_out_dev) & 3)
        return fail(c, I4D_ERR_ARG, "misaligned device buffer (superblocks and act_q need 2 bytes, partial_out 4)");
    if (lit < 1 || lit > 11 || out_tiles < 1 || out_tiles > 1008 || (out_tiles * lit) % 16 != 0)
        return fail(c, I4D_ERR_ARG, "unsupported linear geometry: %d local input tiles, %d output tiles", lit, out_tiles);
    const size_t need = static_cast<size_t>(out_tiles) * lit / 16 * 4224 * 64;
    if (n_bytes != need) return fail(c, I4D_ERR_SIZE, "superblock stream has %zu bytes; expected %zu", n_bytes, need);
    if (n_bytes > kNoAllocMaxBytes)
        return fail(c, I4D_ERR_SIZE,
                    "superblock stream of %zu bytes exceeds the %zu-byte static scratch of "
                    "i4d_linear_bank_noalloc (22 superblocks); use i4d_linear_bank",
                    n_bytes, kNoAllocMaxBytes);
    CK(cudaSetDevice(c->device));
    uint8_t* scratch = nullptr;
    const i4d_status st = noalloc_scratch(c, &scratch);
    if (st != I4D_OK) return st;
    unsigned* err = reinterpret_cast<unsigned*>(scratch);
    uint8_t* tiles = scratch + kNoAllocHeader;
    CK(cudaMemsetAsync(err, 0, sizeof(unsigned), c->stream));
    RelayoutArgs r;
    r.src = static_cast<const uint8_t*>(superblocks_dev);
    r.dst = tiles;
    r.unit_offset = 0;
    r.lit = lit;
    k_relayout<<<out_tiles * 4 * lit, 256, 0, c->stream>>>(r);
    CK(cudaGetLastError());
    LinearArgs a = {};
    a.w = tiles;
    a.bank_stride = 0;
    a.nbanks = 1;
    a.units = out_tiles * 4;
    a.cpb = a.units < c->num_sms ? a.units : c->num_sms;
    a.chunks = lit;
    a.ns = ring_slots(lit);
    a.nu = contrib_slots(lit);
    a.in_kind = IN_ACT;
    a.act_q = act_q_dev;
    a.act_e = act_e8m0_dev;
    a.act_bank_stride = 0;
    a.hls_zero = hls_zero_start ? 1 : 0;
    a.partials = partial_out_dev;
    a.epi = EPI_PARTIAL;
    a.counters = nullptr;  // the partial epilogue uses no stripe counters
    a.expf = c->expf;
    a.err = err;
    CK(run_linear(c, a, false));
    unsigned e = 0;
    CK(cudaMemcpyAsync(&e, err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (e & kErrArg) return fail(c, I4D_ERR_ARG, "device rejected an argument (error word 0x%x)", e);
    if (e) return fail(c, I4D_ERR_TIMEOUT, "a bounded device wait gave up (error word 0x%x)", e);
    return I4D_OK;
}

i4d_status i4d_gemv(i4d_ctx* c, int layer, int mode, const int16_t* act_q, const uint8_t* act_e8m0, float* y_out,
                    float* partials_out) {
    if (c && c->world > 1) return fail(c, I4D_ERR_STATE, "not available on a bank shard");
    if (!c || !act_q || !act_e8m0 || !y_out) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (mode < 0 || mode > 7 || (mode < 7 && (layer < 0 || layer >= c->layers)))
        return fail(c, I4D_ERR_ARG, "bad layer %d / mode %d", layer, mode);
    if (!c->bank_loaded[0] || !c->bank_loaded[1] || !c->bank_loaded[2] || !c->bank_loaded[3])
        return fail(c, I4D_ERR_STATE, "all four banks must be loaded");
    CK(cudaSetDevice(c->device));
    const int rows = mode_rows(mode), cols = mode == 6 ? kFfn : kDim;
    const int st = mode_stage(mode);
    DEVBUF(aq, cols * sizeof(int16_t));
    DEVBUF(ae, cols / 32);
    DEVBUF(y, rows * sizeof(float));
    CK(cudaMemcpyAsync(aq.p, act_q, cols * sizeof(int16_t), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(ae.p, act_e8m0, cols / 32, cudaMemcpyHostToDevice, c->stream));
    LinearArgs a = base_linear(c, mode == 7 ? 0 : layer, st);
    a.w += static_cast<size_t>(mode_unit_offset(mode)) * a.chunks * kChunkBytes;
    a.units = rows / 32;
    a.in_kind = IN_ACT;
    a.act_q = aq.as<int16_t>();
    a.act_e = ae.as<uint8_t>();
    a.act_bank_stride = cols / 4;
    a.epi = EPI_STORE;
    a.out = y.as<float>();
    CK(run_linear(c, a, false));
    const i4d_status s2 = finish(c);
    if (s2 != I4D_OK) return s2;
    CK(cudaMemcpy(y_out, y.p, rows * sizeof(float), cudaMemcpyDeviceToHost));
    if (partials_out)
        CK(cudaMemcpy(partials_out, c->d_partials, 4ull * rows * sizeof(float), cudaMemcpyDeviceToHost));
    return I4D_OK;
}

i4d_status i4d_quantize_g32(i4d_ctx* c, const float* x, int n, int16_t* q, uint8_t* e8m0) {
    if (!c || !x || !q || !e8m0 || n <= 0 || n % 32) return c ? fail(c, I4D_ERR_ARG, "bad quantize arguments") : I4D_ERR_ARG;
    CK(cudaSetDevice(c->device));
    DEVBUF(dx, n * sizeof(float));
    DEVBUF(dq, n * sizeof(int16_t));
    DEVBUF(de, n / 32);
    CK(cudaMemcpyAsync(dx.p, x, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    k_quant_g32<<<(n + 127) / 128, 128, 0, c->stream>>>(dx.as<float>(), n, dq.as<int16_t>(), de.as<uint8_t>());
    CK(cudaGetLastError());
    const i4d_status st = finish(c);
    if (st != I4D_OK) return st;
    CK(cudaMemcpy(q, dq.p, n * sizeof(int16_t), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(e8m0, de.p, n / 32, cudaMemcpyDeviceToHost));
    return I4D_OK;
}

i4d_status i4d_rms_quant(i4d_ctx* c, const float* x, const float* gamma, int16_t* q, uint8_t* e8m0) {
    if (!c || !x || !gamma || !q || !e8m0) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    CK(cudaSetDevice(c->device));
    DEVBUF(dx, kDim * sizeof(float));
    DEVBUF(dg, kDim * sizeof(float));
    DEVBUF(dr, 16);
    DEVBUF(dq, kDim * sizeof(int16_t));
    DEVBUF(de, kDim / 32);
    CK(cudaMemcpyAsync(dx.p, x, kDim * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(dg.p, gamma, kDim * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    k_rms_recip<<<1, 32, 0, c->stream>>>(dx.as<float>(), dr.as<float>());
    k_norm_quant<<<kDim / 128, 128, 0, c->stream>>>(dx.as<float>(), dg.as<float>(), dr.as<float>(), dq.as<int16_t>(),
                                                    de.as<uint8_t>());
    CK(cudaGetLastError());
    const i4d_status st = finish(c);
    if (st != I4D_OK) return st;
    CK(cudaMemcpy(q, dq.p, kDim * sizeof(int16_t), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(e8m0, de.p, kDim / 32, cudaMemcpyDeviceToHost));
    return I4D_OK;
}

i4d_status i4d_attention(i4d_ctx* c, int layer, uint32_t position, const int32_t* q, const int32_t* k,
                         const int32_t* v, int16_t* out_q, uint8_t* out_e8m0) {
    if (c && c->world > 1) return fail(c, I4D_ERR_STATE, "not available on a bank shard");
    if (!c || !q || !k || !v || !out_q || !out_e8m0) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (!c->rope_loaded) return fail(c, I4D_ERR_STATE, "rope LUT not loaded");
    if (layer < 0 || layer >= c->layers || position >= static_cast<uint32_t>(c->stride))
        return fail(c, I4D_ERR_ARG, "layer %d / position %u out of range", layer, position);
    CK(cudaSetDevice(c->device));
    DEVBUF(dqkv, 3ull * kDim * sizeof(int32_t));
    DEVBUF(dq, kDim * sizeof(int16_t));
    DEVBUF(de, kDim / 32);
    CK(cudaMemcpyAsync(dqkv.as<int32_t>(), q, kDim * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(dqkv.as<int32_t>() + kDim, k, kDim * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(dqkv.as<int32_t>() + 2 * kDim, v, kDim * 4, cudaMemcpyHostToDevice, c->stream));
    const int p = static_cast<int>(position);
    CK(cudaMemcpyAsync(c->d_pos, &p, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    AttnArgs a = base_attn(c, layer);
    a.partials = nullptr;
    a.direct = dqkv.as<int32_t>();
    a.out_q = dq.as<int16_t>();
    a.out_e = de.as<uint8_t>();
    k_attn_items<<<kAttnItems, kItemThreads, attn_items_smem_bytes(), c->stream>>>(a);
    CK(cudaGetLastError());
    const i4d_status st = finish(c);
    if (st != I4D_OK) return st;
    CK(cudaMemcpy(out_q, dq.p, kDim * sizeof(int16_t), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(out_e8m0, de.p, kDim / 32, cudaMemcpyDeviceToHost));
    return I4D_OK;
}

i4d_status i4d_swiglu_quant(i4d_ctx* c, const float* gate, const float* up, int16_t* q, uint8_t* e8m0) {
    if (!c || !gate || !up || !q || !e8m0) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    CK(cudaSetDevice(c->device));
    DEVBUF(dg, kFfn * sizeof(float));
    DEVBUF(du, kFfn * sizeof(float));
    DEVBUF(dq, kFfn * sizeof(int16_t));
    DEVBUF(de, kFfn / 32);
    CK(cudaMemcpyAsync(dg.p, gate, kFfn * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(du.p, up, kFfn * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    k_swiglu_quant<<<kFfn / 128, 128, 0, c->stream>>>(dg.as<float>(), du.as<float>(), kFfn, c->expf, dq.as<int16_t>(),
                                                      de.as<uint8_t>());
    CK(cudaGetLastError());
    const i4d_status st = finish(c);
    if (st != I4D_OK) return st;
    CK(cudaMemcpy(q, dq.p, kFfn * sizeof(int16_t), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(e8m0, de.p, kFfn / 32, cudaMemcpyDeviceToHost));
    return I4D_OK;
}

i4d_status i4d_argmax(i4d_ctx* c, const float* logits, size_t n, int32_t* index) {
    if (!c || !logits || !index || n == 0 || n > static_cast<size_t>(kPVocab))
        return c ? fail(c, I4D_ERR_ARG, "bad arguments") : I4D_ERR_ARG;
    CK(cudaSetDevice(c->device));
    DEVBUF(x, n * sizeof(float));
    DEVBUF(k, sizeof(unsigned long long));
    CK(cudaMemcpyAsync(x.p, logits, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    k_argmax<<<1, 1024, 0, c->stream>>>(x.as<float>(), static_cast<int>(n), k.as<unsigned long long>());
    CK(cudaGetLastError());
    unsigned long long key = 0;
    CK(cudaMemcpyAsync(&key, k.p, sizeof(key), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    *index = key == 0ull ? -1 : static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffu));
    return I4D_OK;
}

i4d_status i4d_device_arch(int device, int* binary_version, int* device_cc) {
    if (!binary_version || !device_cc) return I4D_ERR_ARG;
    if (cudaSetDevice(device) != cudaSuccess) return I4D_ERR_CUDA;
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, k_token<false>) != cudaSuccess) return I4D_ERR_CUDA;
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess)
        return I4D_ERR_CUDA;
    *binary_version = fa.binaryVersion;
    *device_cc = major * 10 + minor;
    return I4D_OK;
}

i4d_status i4d_expf(i4d_ctx* c, const float* x, float* y, size_t n) {
    if (!c || !x || !y) return c ? fail(c, I4D_ERR_ARG, "null buffer") : I4D_ERR_ARG;
    if (n == 0) return I4D_OK;
    CK(cudaSetDevice(c->device));
    DEVBUF(dx, n * sizeof(float));
    DEVBUF(dy, n * sizeof(float));
    CK(cudaMemcpyAsync(dx.p, x, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    k_expf<<<static_cast<unsigned>((n + 255) / 256), 256, 0, c->stream>>>(dx.as<float>(), dy.as<float>(), n, c->expf);
    CK(cudaGetLastError());
    const i4d_status st = finish(c);
    if (st != I4D_OK) return st;
    CK(cudaMemcpy(y, dy.p, n * sizeof(float), cudaMemcpyDeviceToHost));
    return I4D_OK;
}

}  // extern "C"

extern "C" i4d_status i4d_token_breakdown(i4d_ctx* c, uint32_t position, const float* residual_in_dev,
                                          float* us_out, int n_out) {
    if (c && c->world > 1) return fail(c, I4D_ERR_STATE, "not available on a bank shard");
    if (!c || !residual_in_dev || !us_out || n_out < kTraceSlots) return c ? fail(c, I4D_ERR_ARG, "bad arguments") : I4D_ERR_ARG;
    if (c->flags & I4D_FLAG_STAGED) return fail(c, I4D_ERR_STATE, "breakdown needs the persistent token kernel");
    if (!all_loaded(c)) return fail(c, I4D_ERR_STATE, "banks and rope LUT must be loaded before decoding");
    if (position >= static_cast<uint32_t>(c->stride)) return fail(c, I4D_ERR_ARG, "position out of range");
    CK(cudaSetDevice(c->device));
    const size_t slots = static_cast<size_t>(4 * c->cpb) * kTraceSlots;
    if (!c->d_trace) CK(cudaMalloc(&c->d_trace, slots * sizeof(unsigned long long)));
    CK(cudaMemsetAsync(c->d_trace, 0, slots * sizeof(unsigned long long), c->stream));
    k_set_pos<<<1, 1, 0, c->stream>>>(c->d_pos, static_cast<int>(position));
    CK(cudaMemcpyAsync(c->d_resid, residual_in_dev, kDim * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    CK(launch_token(c));
    const i4d_status st = finish(c);
    std::vector<unsigned long long> h(slots);
    CK(cudaMemcpy(h.data(), c->d_trace, slots * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    CK(cudaFree(c->d_trace));
    c->d_trace = nullptr;
    if (st != I4D_OK) return st;
    int khz = 0;
    CK(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, c->device));
    for (int k = 0; k < kTraceSlots; ++k) {
        double sum = 0.0;
        for (int b = 0; b < 4 * c->cpb; ++b) sum += static_cast<double>(h[static_cast<size_t>(b) * kTraceSlots + k]);
        const double per = k >= TR_W_DATA ? 4.0 * c->cpb * 4 * kQuads : 4.0 * c->cpb;  // warp slots: per GEMV warp
        us_out[k] = static_cast<float>(sum / per / (khz * 1e-3));
    }
    return I4D_OK;
}

extern "C" i4d_status i4d_token_timeline(i4d_ctx* c, uint32_t position, const float* residual_in_dev, int layer,
                                         int detail, uint64_t* out, int max_ctas, int* n_ctas) {
    if (c && c->world > 1) return fail(c, I4D_ERR_STATE, "not available on a bank shard");
    if (!c || !residual_in_dev || !out || !n_ctas) return c ? fail(c, I4D_ERR_ARG, "bad arguments") : I4D_ERR_ARG;
    if (c->flags & I4D_FLAG_STAGED) return fail(c, I4D_ERR_STATE, "timeline needs the persistent token kernel");
    if (!all_loaded(c)) return fail(c, I4D_ERR_STATE, "banks and rope LUT must be loaded before decoding");
    if (position >= static_cast<uint32_t>(c->stride)) return fail(c, I4D_ERR_ARG, "position out of range");
    if (layer < 0 || layer >= c->layers) return fail(c, I4D_ERR_ARG, "layer out of range");
    const int grid = 4 * c->cpb;
    *n_ctas = grid;
    if (max_ctas < grid) return fail(c, I4D_ERR_SIZE, "timeline needs room for %d CTAs", grid);
    CK(cudaSetDevice(c->device));
    const size_t n = static_cast<size_t>(grid) * kTlEvents;
    CK(cudaMalloc(&c->d_timeline, n * sizeof(unsigned long long)));
    c->tl_layer = layer;
    c->tl_detail = detail != 0;
    cudaError_t e = cudaMemsetAsync(c->d_timeline, 0, n * sizeof(unsigned long long), c->stream);
    if (e == cudaSuccess) {
        k_set_pos<<<1, 1, 0, c->stream>>>(c->d_pos, static_cast<int>(position));
        e = cudaMemcpyAsync(c->d_resid, residual_in_dev, kDim * sizeof(float), cudaMemcpyDeviceToDevice, c->stream);
    }
    if (e == cudaSuccess) e = launch_token(c);
    const i4d_status st = e == cudaSuccess ? finish(c) : fail(c, I4D_ERR_CUDA, "%s", cudaGetErrorString(e));
    // The stamps are returned even when a bounded wait gave up: they show how
    // far each CTA got.
    if (st == I4D_OK || st == I4D_ERR_TIMEOUT)
        e = cudaMemcpy(out, c->d_timeline, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(c->d_timeline);
    c->d_timeline = nullptr;
    c->tl_layer = -1;
    c->tl_detail = false;
    if (st != I4D_OK) return st;
    if (e != cudaSuccess) return fail(c, I4D_ERR_CUDA, "%s", cudaGetErrorString(e));
    return I4D_OK;
}

// ------------------------------------------------------ op-level measurement

extern "C" i4d_status i4d_profile_gemv(i4d_ctx* c, int mode, int reps, float* ms_per_gemv) {
    if (c && c->world > 1) return fail(c, I4D_ERR_STATE, "not available on a bank shard");
    if (!c || !ms_per_gemv || reps <= 0 || mode < 0 || mode > 7) return c ? fail(c, I4D_ERR_ARG, "bad arguments") : I4D_ERR_ARG;
    if (!c->bank_loaded[0] || !c->bank_loaded[1] || !c->bank_loaded[2] || !c->bank_loaded[3])
        return fail(c, I4D_ERR_STATE, "all four banks must be loaded");
    CK(cudaSetDevice(c->device));
    for (cudaEvent_t& ev : c->prof_ev)
        if (!ev) CK(cudaEventCreate(&ev));
    const int rows = mode_rows(mode), cols = mode == 6 ? kFfn : kDim;
    const int st = mode_stage(mode);
    DEVBUF(aq, cols * sizeof(int16_t));
    DEVBUF(ae, cols / 32);
    DEVBUF(y, rows * sizeof(float));
    // The arithmetic does not depend on the values: a fixed activation.
    CK(cudaMemsetAsync(aq.p, 0x15, cols * sizeof(int16_t), c->stream));
    CK(cudaMemsetAsync(ae.p, 127, cols / 32, c->stream));
    auto one = [&](int r) {
        const int layer = mode == 7 ? 0 : r % c->layers;  // a different matrix each launch
        LinearArgs a = base_linear(c, layer, st);
        a.w += static_cast<size_t>(mode_unit_offset(mode)) * a.chunks * kChunkBytes;
        a.units = rows / 32;
        a.in_kind = IN_ACT;
        a.act_q = aq.as<int16_t>();
        a.act_e = ae.as<uint8_t>();
        a.act_bank_stride = cols / 4;
        a.epi = EPI_STORE;
        a.out = y.as<float>();
        return run_linear(c, a, true);
    };
    for (int r = 0; r < 3; ++r) CK(one(r));  // warm-up
    CK(cudaEventRecord(c->prof_ev[0], c->stream));
    for (int r = 0; r < reps; ++r) CK(one(r));
    CK(cudaEventRecord(c->prof_ev[1], c->stream));
    const i4d_status s = finish(c);
    if (s != I4D_OK) return s;
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, c->prof_ev[0], c->prof_ev[1]));
    *ms_per_gemv = ms / reps;
    return I4D_OK;
}

// Attention of one layer at `position` over the records already in the KV
// cache.  fill > 0: first writes the records of positions [0, position) by
// running the attention step at each of them with q/k/v row (p % fill) of
// qkv_dev ([fill][3][4096] Q15.17); then times `reps` steps at `position`
// (each rewrites that position's record) with row 0.
extern "C" i4d_status i4d_profile_attention(i4d_ctx* c, int layer, uint32_t position, const int32_t* qkv_dev,
                                            int fill, int reps, float* ms_per_step) {
    if (c && c->world > 1) return fail(c, I4D_ERR_STATE, "not available on a bank shard");
    if (!c || !qkv_dev || !ms_per_step || reps <= 0 || fill < 0) return c ? fail(c, I4D_ERR_ARG, "bad arguments") : I4D_ERR_ARG;
    if (!c->rope_loaded) return fail(c, I4D_ERR_STATE, "rope LUT not loaded");
    if (layer < 0 || layer >= c->layers || position >= static_cast<uint32_t>(c->stride))
        return fail(c, I4D_ERR_ARG, "layer %d / position %u out of range", layer, position);
    CK(cudaSetDevice(c->device));
    for (cudaEvent_t& ev : c->prof_ev)
        if (!ev) CK(cudaEventCreate(&ev));
    AttnArgs a = base_attn(c, layer);
    a.partials = nullptr;
    auto step = [&](int p, int row) {
        k_set_pos<<<1, 1, 0, c->stream>>>(c->d_pos, p);
        a.direct = qkv_dev + static_cast<size_t>(row) * 3 * kDim;
        k_attn_items<<<kAttnItems, kItemThreads, attn_items_smem_bytes(), c->stream>>>(a);
        return cudaGetLastError();
    };
    if (fill > 0)
        for (uint32_t p = 0; p < position; ++p) CK(step(static_cast<int>(p), static_cast<int>(p % fill)));
    CK(step(static_cast<int>(position), 0));  // warm-up
    CK(cudaEventRecord(c->prof_ev[0], c->stream));
    for (int r = 0; r < reps; ++r) CK(step(static_cast<int>(position), 0));
    CK(cudaEventRecord(c->prof_ev[1], c->stream));
    const i4d_status s = finish(c);
    if (s != I4D_OK) return s;
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, c->prof_ev[0], c->prof_ev[1]));
    *ms_per_step = ms / reps;
    return I4D_OK;
}
