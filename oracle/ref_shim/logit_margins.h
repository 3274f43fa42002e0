// logit_margins.h -- a pass-through mruntime::Backend that records, for every
// lm_head contraction, the greedy pick of the last row and its top-2 margin.
//
// TEST INFRASTRUCTURE ONLY.  InferenceEngine::generate
// (src/engine/inference_engine.cpp:26-67) hides its logits; the model produces
// them with one Backend::gemm whose output's last dimension is the vocabulary
// (src/models/qwen/qwen_model.cpp:372-374).  Wrapping the engine's backend in
// this decorator sees that output after the inner backend wrote it (the
// reference's calls are synchronous, so the host tensor is complete on
// return) and keeps, per call, the index the reference's greedy rule would
// pick (first maximum under strict `>`, inference_engine.cpp:84-95), its value
// and the runner-up's value and index.  The margin top1 - top2 says how close
// each greedy decision was.
#pragma once

#include <cstddef>
#include <limits>
#include <vector>

#include "mruntime/backend.h"
#include "mruntime/dtype.h"
#include "mruntime/tensor.h"

namespace ref_shim {

struct Pick {
    int index = -1;
    int second_index = -1;  // the runner-up: first index holding top2 (other than `index`)
    float top1 = 0.0f;
    float top2 = 0.0f;
};

class LogitMargins : public mruntime::Backend {
public:
    LogitMargins(mruntime::Backend& inner, size_t vocab) : inner_(inner), vocab_(vocab) {}

    const std::vector<Pick>& picks() const { return picks_; }

    void gemm(const mruntime::Tensor& A, const mruntime::Tensor& B, mruntime::Tensor& C, float alpha, float beta,
              bool trans_a, bool trans_b) override {
        inner_.gemm(A, B, C, alpha, beta, trans_a, trans_b);
        if (C.ndim() >= 2 && C.dim(C.ndim() - 1) == vocab_) record(C);
    }
    void flash_attention(const mruntime::Tensor& Q, const mruntime::Tensor& K, const mruntime::Tensor& V,
                         mruntime::Tensor& output, float scale, bool causal) override {
        inner_.flash_attention(Q, K, V, output, scale, causal);
    }
    void rmsnorm(const mruntime::Tensor& input, const mruntime::Tensor& weight, mruntime::Tensor& output,
                 float eps) override {
        inner_.rmsnorm(input, weight, output, eps);
    }
    void rope(mruntime::Tensor& Q, mruntime::Tensor& K, size_t position_offset, float theta) override {
        inner_.rope(Q, K, position_offset, theta);
    }
    void silu(const mruntime::Tensor& input, mruntime::Tensor& output) override { inner_.silu(input, output); }
    void elementwise_mul(const mruntime::Tensor& a, const mruntime::Tensor& b, mruntime::Tensor& output) override {
        inner_.elementwise_mul(a, b, output);
    }
    void add(const mruntime::Tensor& a, const mruntime::Tensor& b, mruntime::Tensor& output) override {
        inner_.add(a, b, output);
    }
    void softmax(const mruntime::Tensor& input, mruntime::Tensor& output, int dim) override {
        inner_.softmax(input, output, dim);
    }
    void embedding_lookup(const mruntime::Tensor& weight, const std::vector<int>& token_ids,
                          mruntime::Tensor& output) override {
        inner_.embedding_lookup(weight, token_ids, output);
    }

private:
    void record(const mruntime::Tensor& C) {
        const size_t rows = C.numel() / vocab_;
        const size_t base = (rows - 1) * vocab_;
        Pick p;
        float best = -std::numeric_limits<float>::infinity();
        float second = -std::numeric_limits<float>::infinity();
        for (size_t i = 0; i < vocab_; ++i) {
            const float v = mruntime::load_scalar_as_fp32(C.data(), C.dtype(), base + i);
            if (v > best) {
                second = best;
                p.second_index = p.index;
                best = v;
                p.index = static_cast<int>(i);
            } else if (v > second) {
                second = v;
                p.second_index = static_cast<int>(i);
            }
        }
        if (p.index < 0) p.index = 0;  // all -inf/NaN: the reference's rule keeps index 0
        p.top1 = best;
        p.top2 = second;
        picks_.push_back(p);
    }

    mruntime::Backend& inner_;
    size_t vocab_;
    std::vector<Pick> picks_;
};

}  // namespace ref_shim
