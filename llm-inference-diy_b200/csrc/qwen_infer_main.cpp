// qwen_infer_main.cpp — drop-in replacement for the reference engine
// executable (framework_src/qwen_infer.cu:743-822), speaking the same
// stdin/stdout protocol that web_chat/app.py:202-278 and test_engine.py
// consume:
//   argv[1]                 path of the QWDF .bin
//   stdout                  free-form start-up lines, then a line with [ENGINE_READY]
//   stdin "reset"           -> [RESET_DONE]
//   stdin "exit" / ""       -> exit 0
//   stdin "<id> <id> ..."   -> [GENERATION_START], one id per line (stop ids
//                              151645/151643 are not printed), [GENERATION_END]
// and one verb the reference does not have (continuous batching of many turns):
//   stdin "batch", then one request per line ("<id> <id> ..."), then "end"
//                           -> [BATCH_START] <n>, then "<r> <id>" for every token
//                              request r (0-based, input order) generates, as the
//                              tokens are produced (requests interleave), "[DONE] <r>"
//                              when r ends (stop id, token limit, or a rejected
//                              prompt), and [BATCH_END].  Each request gets what a
//                              turn of its own would print; up to LLMDIY_MAX_BATCH
//                              (default 16) decode together, the rest wait for a slot.
// Every turn restarts at position 0 (qwen_infer.cu:789).  stdout is
// unbuffered.  Environment knobs for benchmarking only (defaults keep the
// reference behaviour): LLMDIY_MAX_NEW_TOKENS (default 512),
// LLMDIY_IGNORE_EOS=1 (do not stop at the stop ids).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <iostream>
#include <string>
#include <vector>

#include "batch_sched.h"
#include "llmdiy_batch.h"
#include "llmdiy_engine.h"

namespace {

void print_token(int token, void*) { std::cout << token << std::endl; }

bool parse_ids(const std::string& line, std::vector<int>& out, std::string& bad) {
    // qwen_infer.cu:770-784 splits on ' ' and converts with stoi; malformed
    // ids are reported instead of terminating the process.
    std::string cur;
    auto flush = [&]() -> bool {
        if (cur.empty()) return true;
        char* end = nullptr;
        long v = std::strtol(cur.c_str(), &end, 10);
        if (*end != '\0' || v < -2147483647L || v > 2147483647L) { bad = cur; return false; }
        out.push_back((int)v);
        cur.clear();
        return true;
    };
    for (char c : line) {
        if (c == ' ') {
            if (!flush()) return false;
        } else if (c != '\r') {
            cur += c;
        }
    }
    return flush();
}

int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return v && *v ? std::atoi(v) : dflt;
}

// The "batch" verb: requests until "end" (or end of input), run with continuous batching.
void serve_batch(llmdiy_engine* engine, llmdiy_batch*& batch, const llmdiy_config& c, int max_new, bool stop_on_eos) {
    std::vector<std::vector<int>> reqs;
    std::string line;
    while (std::getline(std::cin, line)) {
        if (!line.empty() && line.back() == '\r') line.pop_back();
        if (line == "end") break;
        std::vector<int> p;
        std::string bad;
        if (!parse_ids(line, p, bad)) {
            std::cerr << "[ERROR] request " << reqs.size() << ": invalid token id '" << bad << "'" << std::endl;
            p.clear();  // rejected below (empty prompt)
        }
        reqs.push_back(std::move(p));
    }
    const int slots = std::max(1, std::min(env_int("LLMDIY_MAX_BATCH", 16), 64));
    const int max_len = std::max(2, std::min((int)c.max_seqlen, env_int("LLMDIY_BATCH_MAX_LEN", 4096)));
    std::cout << "[BATCH_START] " << reqs.size() << std::endl;
    if (!batch) {
        const int rc = llmdiy_batch_create(engine, slots, max_len, &batch);
        if (rc) {
            std::cerr << "[ERROR] batch create failed (code " << rc << ")" << std::endl;
            for (size_t r = 0; r < reqs.size(); ++r) std::cout << "[DONE] " << r << std::endl;
            std::cout << "[BATCH_END]" << std::endl;
            batch = nullptr;
            return;
        }
    }
    llmdiy::SchedConfig sc{slots, max_len, max_new, stop_on_eos, (int)c.vocab_size};
    std::vector<char> finished(reqs.size(), 0);
    const int rc = llmdiy::run_continuous_batch(
        sc, reqs, [&](int s, const int* t, int n) { return llmdiy_batch_prefill(batch, s, t, n); },
        [&](int B, const int* t, const int* p, int* out) {
            return llmdiy_batch_decode(batch, B, t, p, 1, out, nullptr);
        },
        [&](int r, int t) { std::cout << r << " " << t << "\n"; },
        [&](int r, int why) {
            if (why == llmdiy::DONE_REJECTED)
                std::cerr << "[ERROR] request " << r << " rejected (empty, bad id or too long)" << std::endl;
            finished[(size_t)r] = 1;
            std::cout << "[DONE] " << r << std::endl;
        });
    if (rc) {
        std::cerr << "[ERROR] batched generation: " << llmdiy_batch_last_error(batch) << " (code " << rc << ")"
                  << std::endl;
        for (size_t r = 0; r < reqs.size(); ++r)
            if (!finished[r]) std::cout << "[DONE] " << r << std::endl;
    }
    std::cout << "[BATCH_END]" << std::endl;
}

}  // namespace

int main(int argc, char* argv[]) {
    std::cout << std::unitbuf;
    std::string model_path = "../model_weights/qwen_1.8b.bin";
    if (argc > 1) model_path = argv[1];
    const char* mx = std::getenv("LLMDIY_MAX_NEW_TOKENS");
    const int max_new_tokens = mx ? std::atoi(mx) : 512;
    const char* ie = std::getenv("LLMDIY_IGNORE_EOS");
    const bool stop_on_eos = !(ie && ie[0] == '1');

    llmdiy_engine* engine = nullptr;
    llmdiy_batch* batch = nullptr;  // created by the first "batch" request
    int rc = llmdiy_engine_create(model_path.c_str(), 0, &engine);
    if (rc) {
        std::cerr << "Error: cannot load model weights file " << model_path << " (code " << rc << ")" << std::endl;
        return 1;
    }
    llmdiy_config c;
    llmdiy_engine_get_config(engine, &c);
    std::cout << "\n=== Weight Config Loaded Successfully ===" << std::endl;
    std::cout << "  Vocab size:        " << c.vocab_size << std::endl;
    std::cout << "  Hidden size:       " << c.hidden_size << std::endl;
    std::cout << "  Layers count:      " << c.num_layers << std::endl;
    std::cout << "  Heads count:       " << c.num_heads << std::endl;
    std::cout << "  FFN Intermediate:  " << c.intermediate_size << std::endl;
    std::cout << "  Max seqlen:        " << c.max_seqlen << std::endl;
    std::cout << "\n[ENGINE_READY] B200 Qwen-1.8B Inference Engine is fully ready." << std::endl;

    while (true) {
        std::string line;
        if (!std::getline(std::cin, line)) break;
        if (!line.empty() && line.back() == '\r') line.pop_back();
        if (line.empty() || line == "exit") break;
        if (line == "batch") {
            serve_batch(engine, batch, c, max_new_tokens, stop_on_eos);
            continue;
        }
        if (line == "reset") {
            rc = llmdiy_engine_reset(engine);
            if (rc) std::cerr << "[ERROR] reset: " << llmdiy_engine_last_error(engine) << std::endl;
            std::cout << "[RESET_DONE]" << std::endl;
            continue;
        }
        std::vector<int> prompt;
        std::string bad;
        if (!parse_ids(line, prompt, bad)) {
            std::cerr << "[ERROR] invalid token id '" << bad << "'" << std::endl;
            std::cout << "[GENERATION_START]" << std::endl;
            std::cout << "[GENERATION_END]" << std::endl;
            continue;
        }
        if (prompt.empty()) continue;
        std::cout << "[GENERATION_START]" << std::endl;
        int n_out = 0;
        rc = llmdiy_engine_generate_stream(engine, prompt.data(), (int)prompt.size(), max_new_tokens,
                                           stop_on_eos ? 1 : 0, print_token, nullptr, &n_out);
        if (rc) std::cerr << "[ERROR] generation: " << llmdiy_engine_last_error(engine) << std::endl;
        std::cout << "[GENERATION_END]" << std::endl;
    }
    if (batch) llmdiy_batch_destroy(batch);
    llmdiy_engine_destroy(engine);
    return 0;
}
