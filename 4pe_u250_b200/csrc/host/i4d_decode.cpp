// i4d_decode -- C++ host replacing the XRT decode_host for the decode path.
//
// Loads model_bank{0..3}.bin, rope_lut.bin and embeddings.bin exactly as
// decode_host does (host/decode_host.cpp:1236-1296, same size checks), then
// runs the per-token contract through libi4d: residual = embedding row in,
// 32256 padded logits out (decode_host.cpp:1340-1556).  The prompt runs one
// token per step as in the reference (decode_host.cpp:1570-1580), or with
// --prefill as one i4d_prefill call (batches of 16 prompt tokens, the same KV
// records and last logits); generation is greedy (argmax of the first 32000
// logits, NaN skipped, decode_host.cpp:703-717).  The tokenizer and
// stochastic sampler are outside this path: prompts are token ids.
//
//   i4d_decode --banks DIR [--rope FILE] [--embeddings FILE] --prompt-ids 1,2,3
//              [--max-tokens N] [--layers L] [--kv-capacity S] [--device D]
//              [--dump-logits DIR] [--no-eos] [--prefill] [--verbose]
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "i4d.h"

namespace {

struct Config {
    std::string banks_dir, rope, embeddings, dump_logits;
    std::vector<int> prompt;
    int max_tokens = 128, layers = 32, kv_capacity = 4096, device = 0;
    bool stop_on_eos = true, verbose = false, prefill = false;
};

std::vector<char> read_file(const std::string& path, size_t expect) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw std::runtime_error("cannot open " + path);
    const size_t n = static_cast<size_t>(f.tellg());
    if (expect && n != expect)
        throw std::runtime_error(path + " has " + std::to_string(n) + " bytes; expected " + std::to_string(expect));
    std::vector<char> buf(n);
    f.seekg(0);
    f.read(buf.data(), static_cast<std::streamsize>(n));
    return buf;
}

void check(i4d_ctx* ctx, i4d_status st, const char* what) {
    if (st != I4D_OK)
        throw std::runtime_error(std::string(what) + ": status " + std::to_string(st) + ": " + i4d_last_error(ctx));
}

int argmax_logits(const float* logits) {
    int best = -1;
    for (int i = 0; i < I4D_VOCAB; ++i) {
        if (std::isnan(logits[i])) continue;
        if (best < 0 || logits[i] > logits[best]) best = i;
    }
    if (best < 0) throw std::runtime_error("all valid-vocabulary logits are NaN");
    return best;
}

Config parse(int argc, char** argv) {
    Config c;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto next = [&]() -> std::string {
            if (i + 1 >= argc) throw std::runtime_error("missing value for " + a);
            return argv[++i];
        };
        if (a == "--banks") c.banks_dir = next();
        else if (a == "--rope") c.rope = next();
        else if (a == "--embeddings") c.embeddings = next();
        else if (a == "--dump-logits") c.dump_logits = next();
        else if (a == "--max-tokens") c.max_tokens = std::stoi(next());
        else if (a == "--layers") c.layers = std::stoi(next());
        else if (a == "--kv-capacity") c.kv_capacity = std::stoi(next());
        else if (a == "--device") c.device = std::stoi(next());
        else if (a == "--no-eos") c.stop_on_eos = false;
        else if (a == "--verbose") c.verbose = true;
        else if (a == "--prefill") c.prefill = true;
        else if (a == "--prompt-ids") {
            std::stringstream ss(next());
            std::string tok;
            while (std::getline(ss, tok, ',')) c.prompt.push_back(std::stoi(tok));
        } else throw std::runtime_error("unknown argument " + a);
    }
    if (c.banks_dir.empty() || c.prompt.empty()) throw std::runtime_error("--banks and --prompt-ids are required");
    if (c.rope.empty()) c.rope = c.banks_dir + "/rope_lut.bin";
    if (c.embeddings.empty()) c.embeddings = c.banks_dir + "/embeddings.bin";
    return c;
}

}  // namespace

int main(int argc, char** argv) {
    i4d_ctx* ctx = nullptr;
    try {
        const Config cfg = parse(argc, argv);
        i4d_config ic{cfg.device, cfg.layers, cfg.kv_capacity, 0u};
        if (i4d_create(&ic, &ctx) != I4D_OK) throw std::runtime_error("i4d_create failed");
        for (int p = 0; p < I4D_BANKS; ++p) {
            const auto img = read_file(cfg.banks_dir + "/model_bank" + std::to_string(p) + ".bin", 0);
            check(ctx, i4d_load_bank(ctx, p, img.data(), img.size()), "load bank");
        }
        const auto rope = read_file(cfg.rope, I4D_ROPE_BYTES);
        check(ctx, i4d_load_rope(ctx, rope.data(), rope.size()), "load rope");
        const auto embb = read_file(cfg.embeddings, static_cast<size_t>(I4D_VOCAB) * I4D_DIM * 4);
        const float* emb = reinterpret_cast<const float*>(embb.data());

        std::vector<float> logits(I4D_PADDED_VOCAB);
        std::vector<int> generated;
        double total_ms = 0.0;
        int pos = 0, next = -1;
        auto step = [&](int token) {
            if (token < 0 || token >= I4D_VOCAB) throw std::runtime_error("token id out of range");
            const auto t0 = std::chrono::steady_clock::now();
            check(ctx, i4d_decode_token(ctx, static_cast<uint32_t>(pos), emb + static_cast<size_t>(token) * I4D_DIM,
                                        logits.data(), nullptr),
                  "decode");
            total_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            if (!cfg.dump_logits.empty()) {
                char name[64];
                std::snprintf(name, sizeof(name), "/logits_pos%04d_token%05d.bin", pos, token);
                std::ofstream(cfg.dump_logits + name, std::ios::binary)
                    .write(reinterpret_cast<const char*>(logits.data()), I4D_PADDED_VOCAB * 4);
            }
            ++pos;
            next = argmax_logits(logits.data());
        };
        if (cfg.prefill) {  // the whole prompt in batches; logits of its last token
            std::vector<float> rows(cfg.prompt.size() * I4D_DIM);
            for (size_t i = 0; i < cfg.prompt.size(); ++i) {
                const int token = cfg.prompt[i];
                if (token < 0 || token >= I4D_VOCAB) throw std::runtime_error("token id out of range");
                std::memcpy(rows.data() + i * I4D_DIM, emb + static_cast<size_t>(token) * I4D_DIM, I4D_DIM * 4);
            }
            const auto t0 = std::chrono::steady_clock::now();
            check(ctx, i4d_prefill(ctx, 0, rows.data(), static_cast<uint32_t>(cfg.prompt.size()), logits.data()),
                  "prefill");
            total_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            pos = static_cast<int>(cfg.prompt.size());
            next = argmax_logits(logits.data());
        } else {
            for (int t : cfg.prompt) step(t);
        }
        while (static_cast<int>(generated.size()) < cfg.max_tokens && pos < cfg.kv_capacity) {
            if (cfg.stop_on_eos && (next == 1 || next == 2)) break;
            generated.push_back(next);
            if (static_cast<int>(generated.size()) >= cfg.max_tokens || pos >= cfg.kv_capacity) break;
            step(next);
        }
        std::printf("[Generated token IDs]");
        for (int t : generated) std::printf(" %d", t);
        std::printf("\n[Stats] steps=%d total_ms=%.3f ms_per_step=%.3f\n", pos, total_ms, total_ms / pos);
        i4d_destroy(ctx);
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ERROR: %s\n", e.what());
        if (ctx) i4d_destroy(ctx);
        return 1;
    }
}
