// device_decode_main.cpp — greedy decode of a QuickLM checkpoint with the
// whole forward on the GPU (qlm_model_*: activations stay in HBM, one token id
// crosses to the host per step). Same driver loop and output line as
// decode_main.cpp (prefill of prompt[:-1], then forward + greedy choice,
// src/main.cpp:590-690), so the two are compared token for token.
//
//   device_decode_main MODEL_DIR PROMPT_IDS_FILE N_NEW [DEVICE]
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <vector>

#include "qlm_b200.h"

int main(int argc, char** argv) {
    if (argc < 4) {
        std::fprintf(stderr, "usage: %s MODEL_DIR PROMPT_IDS_FILE N_NEW [DEVICE]\n", argv[0]);
        return 2;
    }
    const int n_new = std::atoi(argv[3]);
    const int device = argc > 4 ? std::atoi(argv[4]) : 0;
    std::vector<int> prompt;
    {
        std::ifstream f(argv[2]);
        int id;
        while (f >> id) prompt.push_back(id);
    }
    if (prompt.size() < 2 || n_new < 1) {
        std::fprintf(stderr, "need at least 2 prompt ids and 1 new token\n");
        return 2;
    }
    const int max_seq = 2048;  // DecoderModel::load(dir, 2048, ...) in decode_main.cpp
    auto t_load0 = std::chrono::steady_clock::now();
    qlm_model* m = nullptr;
    if (qlm_model_load(argv[1], device, max_seq, &m) != QLM_OK) {
        std::fprintf(stderr, "model load failed: %s\n", qlm_last_error());
        return 1;
    }
    auto t_load1 = std::chrono::steady_clock::now();
    int pos = 0, next = 0;
    auto t0 = std::chrono::steady_clock::now();
    for (size_t i = 0; i + 1 < prompt.size(); ++i) {
        if (qlm_model_decode(m, prompt[i], pos++, &next, nullptr) != QLM_OK) {
            std::fprintf(stderr, "prefill step failed: %s\n", qlm_last_error());
            return 1;
        }
    }
    auto t1 = std::chrono::steady_clock::now();
    std::vector<int> out;
    next = prompt.back();
    const char* dump = std::getenv("QLM_DUMP_LOGITS");  // first decode step's logits, raw float32
    int vocab = 0;
    qlm_model_info(m, &vocab, nullptr, nullptr, nullptr, nullptr);
    std::vector<float> first(dump && *dump ? (size_t)vocab : 0);
    for (int i = 0; i < n_new; ++i) {
        int tok = 0;
        if (qlm_model_decode(m, next, pos++, &tok, i == 0 && !first.empty() ? first.data() : nullptr) != QLM_OK) {
            std::fprintf(stderr, "decode step failed: %s\n", qlm_last_error());
            return 1;
        }
        next = tok;
        out.push_back(tok);
    }
    auto t2 = std::chrono::steady_clock::now();
    if (!first.empty()) {
        if (FILE* f = std::fopen(dump, "wb")) {
            std::fwrite(first.data(), sizeof(float), first.size(), f);
            std::fclose(f);
        }
    }
    const double load_s = std::chrono::duration<double>(t_load1 - t_load0).count();
    const double prefill_s = std::chrono::duration<double>(t1 - t0).count();
    const double decode_s = std::chrono::duration<double>(t2 - t1).count();
    std::printf("{\"tokens\": [");
    for (size_t i = 0; i < out.size(); ++i) std::printf("%s%d", i ? ", " : "", out[i]);
    std::printf("], \"prompt_len\": %zu, \"load_s\": %.3f, \"prefill_s\": %.4f, \"decode_s\": %.4f, "
                "\"decode_tok_s\": %.3f, \"threads\": 0}\n",
                prompt.size(), load_s, prefill_s, decode_s, n_new / decode_s);
    if (std::getenv("QUICKLM_PROF")) {  // as src/main.cpp:706-709, device time of the linear calls
        double ms = 0.0;
        int64_t calls = 0;
        if (qlm_prof_matmul_ms(&ms, &calls) == QLM_OK)
            std::fprintf(stderr, "[prof] cumulative matmul (device): %g ms over %lld calls\n", ms, (long long)calls);
    }
    qlm_model_free(m);
    return 0;
}
