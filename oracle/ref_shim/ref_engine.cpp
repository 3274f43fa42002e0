// ref_engine.cpp -- greedy generation with the reference's own model and engine.
//
// TEST INFRASTRUCTURE ONLY.  Links the reference's QwenModel, InferenceEngine
// and SafeTensorsFile (compiled from its sources) and prints the token ids
// that InferenceEngine::generate (src/engine/inference_engine.cpp:26-67,
// greedy pick 84-95) produces, plus the top-2 margin of every logits row a
// greedy pick was made from (logit_margins.h).
//
// Two builds of this one file:
//   * oracle/Makefile target `engine` -> oracle/_ref/ref_engine: the
//     reference's CpuBackend, the golden-token run;
//   * tests/cpp/Makefile target `engine_cuda` (-DREF_ENGINE_CUDA) ->
//     tests/cpp/_build/ref_engine_cuda: the same model and engine with this
//     repository's CudaBackend in CpuBackend's place, the drop-in check.
//
//   ref_engine <model.safetensors> <config.json> <prompt.txt> <max_new> [threads] [--profile]
//
// prompt.txt holds whitespace-separated token ids.  The end-of-sequence id is
// disabled (-1) so exactly max_new tokens are produced.  --profile wraps the
// backend in the reference's ProfilingBackend decorator
// (include/mruntime/profiling_backend.h:388-403) and prints its per-op calls.
#include <chrono>
#include <cstring>
#include <fstream>
#include <iostream>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "logit_margins.h"
#include "mruntime/inference_engine.h"
#include "mruntime/profiling_backend.h"
#include "mruntime/qwen_model.h"
#include "mruntime/safetensors.h"
#ifdef REF_ENGINE_CUDA
#include "cuda_backend.h"
#else
#include "mruntime/cpu_backend.h"
#endif

int main(int argc, char** argv) {
    std::vector<std::string> args;
    bool profile = false;
    for (int i = 1; i < argc; ++i) {
        if (std::strcmp(argv[i], "--profile") == 0)
            profile = true;
        else
            args.emplace_back(argv[i]);
    }
    if (args.size() < 4) {
        std::cerr << "usage: ref_engine model.safetensors config.json prompt.txt max_new [threads] [--profile]\n";
        return 2;
    }
    try {
        std::ifstream cf(args[1]);
        std::stringstream cs;
        cs << cf.rdbuf();
        mruntime::QwenConfig config = mruntime::QwenConfig::from_json(cs.str());
        std::ifstream pf(args[2]);
        std::vector<int> prompt;
        for (int id; pf >> id;) prompt.push_back(id);
        const size_t max_new = std::stoul(args[3]);
        const size_t threads = args.size() > 4 ? std::stoul(args[4]) : 0;

        auto t0 = std::chrono::steady_clock::now();
        auto file = mruntime::SafeTensorsFile::open(args[0]);
        mruntime::QwenModel model(config);
        model.load_weights(*file);
        auto t1 = std::chrono::steady_clock::now();
#ifdef REF_ENGINE_CUDA
        (void)threads;
        mruntime_b200::CudaBackend backend(0);
        const char* backend_name = "CudaBackend";
#else
        mruntime::CpuBackend backend(threads);
        const char* backend_name = "CpuBackend";
#endif
        std::unique_ptr<mruntime::ProfilingBackend> prof;
        mruntime::Backend* inner = &backend;
        if (profile) {
            prof = std::make_unique<mruntime::ProfilingBackend>(backend);
            inner = prof.get();
        }
        ref_shim::LogitMargins margins(*inner, config.vocab_size);
        mruntime::InferenceEngine engine(model, margins);
        mruntime::GenerationConfig gen;
        gen.max_new_tokens = max_new;
        gen.greedy = true;
        gen.eos_token_id = -1;
        std::vector<int> out = engine.generate(prompt, gen);
        auto t2 = std::chrono::steady_clock::now();
        std::cout << "BACKEND " << backend_name << (profile ? "+ProfilingBackend" : "") << "\n";
        std::cout << "LOAD_SECONDS " << std::chrono::duration<double>(t1 - t0).count() << "\n";
        std::cout << "GENERATE_SECONDS " << std::chrono::duration<double>(t2 - t1).count() << "\n";
        std::cout << "THREADS " << threads << "\n";
        std::cout << "TOKENS";
        for (size_t i = prompt.size(); i < out.size(); ++i) std::cout << " " << out[i];
        std::cout << "\n";
        // The pick of new token j comes from forward prompt.size() - 1 + j.
        const auto& picks = margins.picks();
        std::cout << "MARGINS";
        for (size_t j = 0; j + prompt.size() - 1 < picks.size() && j < out.size() - prompt.size(); ++j) {
            const auto& p = picks[prompt.size() - 1 + j];
            std::cout << " " << (p.top1 - p.top2);
        }
        std::cout << "\n";
        // Runner-up index and top logit of the same picks.
        std::cout << "RUNNERS_UP";
        for (size_t j = 0; j + prompt.size() - 1 < picks.size() && j < out.size() - prompt.size(); ++j)
            std::cout << " " << picks[prompt.size() - 1 + j].second_index;
        std::cout << "\n";
        std::cout << "TOP1";
        for (size_t j = 0; j + prompt.size() - 1 < picks.size() && j < out.size() - prompt.size(); ++j)
            std::cout << " " << picks[prompt.size() - 1 + j].top1;
        std::cout << "\n";
        if (prof) {
            for (int op = 0; op < static_cast<int>(mruntime::BackendOp::Count); ++op) {
                const auto s = prof->profiler().snapshot(static_cast<mruntime::BackendOp>(op));
                std::cout << "PROFILE " << mruntime::backend_op_name(static_cast<mruntime::BackendOp>(op)) << " "
                          << s.calls << " " << s.total_ns << "\n";
            }
        }
    } catch (const std::exception& e) {
        std::cerr << "error: " << e.what() << "\n";
        return 1;
    }
    return 0;
}
