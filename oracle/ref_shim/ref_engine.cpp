// ref_engine.cpp -- greedy generation with the reference's own model and engine.
//
// TEST INFRASTRUCTURE ONLY.  Links the reference's QwenModel, InferenceEngine,
// SafeTensorsFile and CpuBackend (compiled from its sources by
// oracle/Makefile target `engine`) and prints the token ids that
// InferenceEngine::generate (src/engine/inference_engine.cpp:26-67, greedy
// pick 84-95) produces, so the device decoder can be checked token for token.
//
//   ref_engine <model.safetensors> <config.json> <prompt.txt> <max_new> [threads]
//
// prompt.txt holds whitespace-separated token ids.  The end-of-sequence id is
// disabled (-1) so exactly max_new tokens are produced.
#include <chrono>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "mruntime/cpu_backend.h"
#include "mruntime/inference_engine.h"
#include "mruntime/qwen_model.h"
#include "mruntime/safetensors.h"

int main(int argc, char** argv) {
    if (argc < 5) {
        std::cerr << "usage: ref_engine model.safetensors config.json prompt.txt max_new [threads]\n";
        return 2;
    }
    try {
        std::ifstream cf(argv[2]);
        std::stringstream cs;
        cs << cf.rdbuf();
        mruntime::QwenConfig config = mruntime::QwenConfig::from_json(cs.str());
        std::ifstream pf(argv[3]);
        std::vector<int> prompt;
        for (int id; pf >> id;) prompt.push_back(id);
        const size_t max_new = std::stoul(argv[4]);
        const size_t threads = argc > 5 ? std::stoul(argv[5]) : 0;

        auto t0 = std::chrono::steady_clock::now();
        auto file = mruntime::SafeTensorsFile::open(argv[1]);
        mruntime::QwenModel model(config);
        model.load_weights(*file);
        auto t1 = std::chrono::steady_clock::now();
        mruntime::CpuBackend backend(threads);
        mruntime::InferenceEngine engine(model, backend);
        mruntime::GenerationConfig gen;
        gen.max_new_tokens = max_new;
        gen.greedy = true;
        gen.eos_token_id = -1;
        std::vector<int> out = engine.generate(prompt, gen);
        auto t2 = std::chrono::steady_clock::now();
        std::cout << "LOAD_SECONDS " << std::chrono::duration<double>(t1 - t0).count() << "\n";
        std::cout << "GENERATE_SECONDS " << std::chrono::duration<double>(t2 - t1).count() << "\n";
        std::cout << "THREADS " << (threads ? threads : 0) << "\n";
        std::cout << "TOKENS";
        for (size_t i = prompt.size(); i < out.size(); ++i) std::cout << " " << out[i];
        std::cout << "\n";
    } catch (const std::exception& e) {
        std::cerr << "error: " << e.what() << "\n";
        return 1;
    }
    return 0;
}
