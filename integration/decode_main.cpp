// decode_main.cpp — model-only greedy decode through QuickLM's DecoderModel.
//
// Mirrors the CLI's turn loop without tokenizer, chat template or speculative
// decoding (src/main.cpp:590-674): the prompt minus its last token is
// prefilled with forward_batch, the last token starts the decode, and each
// step is forward + greedy sample(logits, 0, 0). Linked either against the
// unmodified reference (the CPU oracle) or with integration/qlm_dropin.cpp
// (int8 matmuls on the B200); both print the same JSON line.
//
//   decode_main MODEL_DIR PROMPT_IDS_FILE N_NEW THREADS [PRECISION]
//
// PROMPT_IDS_FILE: whitespace-separated token ids. With QUICKLM_PROF set, the
// cumulative matmul time is printed to stderr as the reference CLI does.
#include "math_ops.hpp"
#include "model.hpp"
#ifdef QLM_DROPIN
#include "qlm_b200.h"
#endif

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

int main(int argc, char** argv) {
    if (argc < 5) {
        std::fprintf(stderr, "usage: %s MODEL_DIR PROMPT_IDS_FILE N_NEW THREADS [PRECISION]\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    const int n_new = std::atoi(argv[3]);
    const int threads = std::atoi(argv[4]);
    const std::string precision = argc > 5 ? argv[5] : "int8";
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
    try {
        math::init_thread_pool(threads > 0 ? threads : 1);
        // The engine prints progress on stdout; keep stdout for the result line.
        std::streambuf* saved = std::cout.rdbuf(std::cerr.rdbuf());
        auto t_load0 = std::chrono::steady_clock::now();
        DecoderModel model;
        if (!model.load(dir, 2048, precision)) {
            std::cout.rdbuf(saved);
            std::fprintf(stderr, "model load failed\n");
            return 1;
        }
        auto t_load1 = std::chrono::steady_clock::now();
        const int vocab = model.get_config().vocab_size;
        Context ctx;
        std::vector<int> prefill(prompt.begin(), prompt.end() - 1);
        ctx.pos = 0;
        Tensor prefill_logits({(int)prefill.size(), vocab});
        auto t0 = std::chrono::steady_clock::now();
        model.forward_batch(prefill, prefill_logits, ctx);
        auto t1 = std::chrono::steady_clock::now();
        int pos = (int)prefill.size();
        Tensor logits({vocab});
        std::vector<int> out;
        int next = prompt.back();
        const char* dump = std::getenv("QLM_DUMP_LOGITS");  // first decode step's logits, raw float32
        for (int i = 0; i < n_new; ++i) {
            ctx.pos = pos++;
            model.forward(next, logits, ctx);
            if (i == 0 && dump && *dump) {
                if (FILE* f = std::fopen(dump, "wb")) {
                    std::fwrite(logits.data, sizeof(float), (size_t)vocab, f);
                    std::fclose(f);
                }
            }
            next = model.sample(logits, 0.0f, 0);
            out.push_back(next);
        }
        auto t2 = std::chrono::steady_clock::now();
        std::cout.rdbuf(saved);
        const double load_s = std::chrono::duration<double>(t_load1 - t_load0).count();
        const double prefill_s = std::chrono::duration<double>(t1 - t0).count();
        const double decode_s = std::chrono::duration<double>(t2 - t1).count();
        std::printf("{\"tokens\": [");
        for (size_t i = 0; i < out.size(); ++i) std::printf("%s%d", i ? ", " : "", out[i]);
        std::printf("], \"prompt_len\": %zu, \"load_s\": %.3f, \"prefill_s\": %.4f, \"decode_s\": %.4f, "
                    "\"decode_tok_s\": %.3f, \"threads\": %d}\n",
                    prompt.size(), load_s, prefill_s, decode_s, n_new / decode_s, threads);
        if (std::getenv("QUICKLM_PROF")) {  // as src/main.cpp:706-709
            std::fprintf(stderr, "[prof] cumulative matmul: %g ms\n", math::get_matmul_ms());
#ifdef QLM_DROPIN
            // The line above counts the matmuls left on the CPU; the int8 ones ran on the device.
            double ms = 0.0;
            int64_t calls = 0;
            if (qlm_prof_matmul_ms(&ms, &calls) == QLM_OK)
                std::fprintf(stderr, "[prof] cumulative int8 matmul (device): %g ms over %lld calls\n", ms,
                             (long long)calls);
#endif
        }
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
}
