// ref_emulator_harness.cpp -- exposes the UNMODIFIED reference emulator as a
// shared library for parity tests and the CPU baseline.
//
// TEST INFRASTRUCTURE ONLY.  The reference source is compiled from where it
// lies (REF_ROOT/software_sim/llama2_decoder_sw_emulator.cpp) by
// oracle/Makefile; nothing of it is copied into this repository.  Its main()
// is renamed so the static functions (forward, sharded_gemv_4pe,
// rmsnorm_quantize_hls, swiftkv_attention_4pe, ...) can be driven directly,
// bypassing generate(), which needs tokenizer.bin and stops at EOS
// (emulator:1608-1682).
#define main ref_emulator_main
#include "llama2_decoder_sw_emulator.cpp"
#undef main

#include <memory>

namespace {
TransformerModel g_model;
std::vector<KVCachePE> g_kv;
bool g_loaded = false;

void alloc_kv() {
    g_kv.assign(NUM_PES, KVCachePE());
    for (int p = 0; p < NUM_PES; ++p) {
        const size_t records = static_cast<size_t>(g_num_layers) * LOCAL_HEADS * g_cache_seq_len;
        g_kv[p].k_cache.assign(records * HEAD_DIM, 0);
        g_kv[p].k_shift.assign(records * (HEAD_DIM / 32), 0);
        g_kv[p].v_cache.assign(records * HEAD_DIM, 0);
        g_kv[p].v_shift.assign(records * (HEAD_DIM / 32), 0);
    }
}

QuantizedActivation make_act(const int16_t* q, const uint8_t* e8m0, int n) {
    QuantizedActivation a;
    a.q.assign(q, q + n);
    a.scale.resize(n / GROUP_SIZE);
    for (int g = 0; g < n / GROUP_SIZE; ++g) a.scale[g] = std::ldexp(1.0f, int(e8m0[g]) - 140);
    return a;
}

void act_out(const QuantizedActivation& a, int16_t* q, uint8_t* e8m0) {
    std::copy(a.q.begin(), a.q.end(), q);
    for (size_t g = 0; g < a.scale.size(); ++g) {
        int e = 0;
        if (a.scale[g] == 0.0f) { e8m0[g] = 0; continue; }
        std::frexp(a.scale[g], &e);           // scale = 2^(e-1)
        e8m0[g] = static_cast<uint8_t>(e - 1 + 140);
    }
}

const QuantizedMatrix& matrix(int layer, int mode) {
    if (mode == 7) return g_model.w_logits;
    const DecoderLayer& L = g_model.layers.at(layer);
    switch (mode) {
        case 0: return L.w_q; case 1: return L.w_k; case 2: return L.w_v;
        case 3: return L.w_o; case 4: return L.w_gate; case 5: return L.w_up;
        default: return L.w_down;
    }
}
}  // namespace

extern "C" {

// Load model_bank{0..3}.bin, embeddings.bin and rope_lut.bin from `dir`
// (emulator:894-1005) for `layers` layers and a KV stride of `stride` tokens.
int ref_load(const char* dir, int layers, int stride) {
    g_num_layers = layers;
    g_cache_seq_len = stride;
    g_model = TransformerModel();
    if (!load_real_model(g_model, dir, layers)) return -1;
    alloc_kv();
    g_loaded = true;
    return 0;
}

void ref_kv_reset(void) { alloc_kv(); }

int ref_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// emulator:727-783; logits receives the first 32000 rows.
void ref_forward(int token, int pos, float* logits, float* residual_out) {
    std::vector<float> residual(DIM), out;
    forward(g_model, g_kv.data(), token, pos, residual, out);
    std::copy(out.begin(), out.end(), logits);
    if (residual_out) std::copy(residual.begin(), residual.end(), residual_out);
}

void ref_quantize_g32(const float* x, int n, int16_t* q, uint8_t* e8m0) {
    QuantizedActivation a;
    quantize_activation_g32(x, n, a);
    act_out(a, q, e8m0);
}

void ref_rmsnorm_quantize(const float* x, const float* gamma, int16_t* q, uint8_t* e8m0) {
    QuantizedActivation a;
    rmsnorm_quantize_hls(x, gamma, a);
    act_out(a, q, e8m0);
}

void ref_gemv(int layer, int mode, const int16_t* q, const uint8_t* e8m0, float* y) {
    const QuantizedMatrix& m = matrix(layer, mode);
    QuantizedActivation a = make_act(q, e8m0, m.cols);
    std::vector<float> out;
    sharded_gemv_4pe(m, a, out);
    std::copy(out.begin(), out.end(), y);
}

int32_t ref_float_to_q17(float v) { return float_to_q17(v); }

void ref_rope_q17(int32_t* vec, int pos) { apply_rope_q17(vec, pos); }

void ref_attention(const int32_t* q, const int32_t* k, const int32_t* v, int layer, int pos,
                   int16_t* out_q, uint8_t* out_e8m0) {
    QuantizedActivation a;
    swiftkv_attention_4pe(q, k, v, g_kv.data(), layer, pos, a);
    act_out(a, out_q, out_e8m0);
}

void ref_swiglu(const float* gate, const float* up, int n, float* out) { swiglu(gate, up, n, out); }

// One cached (bank, layer, local head, token) entry in the emulator's own
// split arrays (emulator:81-86, 617-631).
void ref_kv_get(int bank, int layer, int lh, int token, int8_t* k8, uint8_t* kshift,
                int8_t* v8, uint8_t* vshift) {
    const KVCachePE& pe = g_kv.at(bank);
    const size_t rec = (static_cast<size_t>(layer) * LOCAL_HEADS + lh) * g_cache_seq_len + token;
    std::copy(pe.k_cache.begin() + rec * HEAD_DIM, pe.k_cache.begin() + (rec + 1) * HEAD_DIM, k8);
    std::copy(pe.v_cache.begin() + rec * HEAD_DIM, pe.v_cache.begin() + (rec + 1) * HEAD_DIM, v8);
    std::copy(pe.k_shift.begin() + rec * 4, pe.k_shift.begin() + rec * 4 + 4, kshift);
    std::copy(pe.v_shift.begin() + rec * 4, pe.v_shift.begin() + rec * 4 + 4, vshift);
}

// Writes one cached entry (the inverse of ref_kv_get): lets a test start the
// emulator at a position whose earlier records it did not compute.
void ref_kv_set(int bank, int layer, int lh, int token, const int8_t* k8, const uint8_t* kshift,
                const int8_t* v8, const uint8_t* vshift) {
    KVCachePE& pe = g_kv.at(bank);
    const size_t rec = (static_cast<size_t>(layer) * LOCAL_HEADS + lh) * g_cache_seq_len + token;
    std::copy(k8, k8 + HEAD_DIM, pe.k_cache.begin() + rec * HEAD_DIM);
    std::copy(v8, v8 + HEAD_DIM, pe.v_cache.begin() + rec * HEAD_DIM);
    std::copy(kshift, kshift + 4, pe.k_shift.begin() + rec * 4);
    std::copy(vshift, vshift + 4, pe.v_shift.begin() + rec * 4);
}

int ref_argmax(const float* logits, int n) { return sample_argmax(const_cast<float*>(logits), n); }

// The emulator's sampler (emulator:1411-1569): one draw with the given state,
// which is advanced in place.  `logits` is modified (penalty, softmax) as the
// emulator does; pass a copy.
int ref_sample(float* logits, int n, const int32_t* history, int n_history, float temperature, float topp,
               float repeat_penalty, unsigned long long* rng_state) {
    Sampler s;
    build_sampler(&s, n, temperature, topp, repeat_penalty, *rng_state);
    const std::vector<int> h(history, history + n_history);
    const int t = sample(&s, logits, h);
    *rng_state = s.rng_state;
    free_sampler(&s);
    return t;
}

// The emulator's perplexity loop (calculate_perplexity, emulator:1775-1958)
// over a pre-tokenized int32 file whose name ends in .bin (no tokenizer is
// read on that path); the report goes to stdout.
void ref_perplexity(const char* token_file, int max_tokens) {
    calculate_perplexity(g_model, nullptr, token_file, max_tokens);
    std::cout.flush();
}

}  // extern "C"
