// ref_capi.cpp -- C entry points over the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile together with the
// reference's src/core/{cpu_backend,tensor,kai_gemm}.cpp (read in place, not
// copied) into oracle/_ref/libmrt_ref.so.  Tests use it to pin the oracle
// restatement and to produce golden vectors; bench.py uses it as the timed
// CPU baseline.  Each function wraps one reference call without changing its
// arithmetic.
#include <cstddef>
#include <cstdint>
#include <limits>
#include <vector>

#include "mruntime/cpu_backend.h"
#include "mruntime/dtype.h"
#include "mruntime/tensor.h"

using mruntime::CpuBackend;
using mruntime::DType;
using mruntime::Shape;
using mruntime::Tensor;

namespace {
DType to_dtype(int d) {
    return d == 1 ? DType::BF16 : (d == 2 ? DType::FP32 : DType::FP16);
}
}  // namespace

extern "C" {

// CpuBackend(threads) (include/mruntime/cpu_backend.h:10-11); 0 = all cores.
void* refb_create(size_t threads) {
    return threads == 0 ? new CpuBackend() : new CpuBackend(threads);
}

void refb_destroy(void* b) { delete static_cast<CpuBackend*>(b); }

// CpuBackend::gemm (src/core/cpu_backend.cpp:72-169) on tensors that view the
// caller's buffers (Tensor::from_buffer, src/core/tensor.cpp:20-26).
// A is [a_rows, a_cols], B is [b_rows, b_cols], C is [c_rows, c_cols].
int refb_gemm(void* backend, const void* A, int a_dtype, size_t a_rows, size_t a_cols,
              const void* B, int b_dtype, size_t b_rows, size_t b_cols, void* C, int c_dtype,
              size_t c_rows, size_t c_cols, float alpha, float beta, int trans_a, int trans_b) {
    const size_t M = trans_a ? a_cols : a_rows;
    const size_t K = trans_a ? a_rows : a_cols;
    const size_t N = trans_b ? b_rows : b_cols;
    if ((trans_b ? b_cols : b_rows) != K || c_rows != M || c_cols != N) return -1;
    Tensor ta = Tensor::from_buffer(const_cast<void*>(A), Shape({a_rows, a_cols}), to_dtype(a_dtype));
    Tensor tb = Tensor::from_buffer(const_cast<void*>(B), Shape({b_rows, b_cols}), to_dtype(b_dtype));
    Tensor tc = Tensor::from_buffer(C, Shape({c_rows, c_cols}), to_dtype(c_dtype));
    static_cast<CpuBackend*>(backend)->gemm(ta, tb, tc, alpha, beta, trans_a != 0, trans_b != 0);
    return 0;
}

// CpuBackend::add (src/core/cpu_backend.cpp:430-455): out = a + b element-wise
// over n FP16 values -- the residual adds of src/models/qwen/qwen_model.cpp:316, 324.
void refb_add(void* backend, const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n) {
    Tensor ta = Tensor::from_buffer(const_cast<uint16_t*>(a), Shape({n}), DType::FP16);
    Tensor tb = Tensor::from_buffer(const_cast<uint16_t*>(b), Shape({n}), DType::FP16);
    Tensor to = Tensor::from_buffer(out, Shape({n}), DType::FP16);
    static_cast<CpuBackend*>(backend)->add(ta, tb, to);
}

// Reference converters (include/mruntime/dtype.h:39-167), element-wise.
void refb_f32_to_f16_n(const float* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = mruntime::float_to_fp16_bits(src[i]);
}
void refb_f16_to_f32_n(const uint16_t* src, float* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = mruntime::fp16_bits_to_float(src[i]);
}
void refb_f32_to_bf16_n(const float* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = mruntime::float_to_bf16(src[i]);
}
void refb_bf16_to_f32_n(const uint16_t* src, float* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = mruntime::bf16_to_float(src[i]);
}

// The q/k/v bias add of src/models/qwen/qwen_model.cpp:130-155 is a lambda
// inside QwenAttention::forward, so it cannot be called from outside; this is
// the same loop written over the reference's own load/store helpers
// (include/mruntime/dtype.h:169-194), with the same operand order.
void refb_add_bias(void* out, int out_dtype, const void* bias, int bias_dtype, size_t rows,
                   size_t n) {
    const DType od = to_dtype(out_dtype);
    const DType bd = to_dtype(bias_dtype);
    for (size_t r = 0; r < rows; ++r)
        for (size_t i = 0; i < n; ++i) {
            float v = mruntime::load_scalar_as_fp32(out, od, r * n + i);
            v += mruntime::load_scalar_as_fp32(bias, bd, i);
            mruntime::store_scalar_from_fp32(out, od, r * n + i, v);
        }
}

// Greedy selection of InferenceEngine::sample (src/engine/inference_engine.cpp:84-95),
// which is private; same loop over the reference's load helper.
int64_t refb_argmax(const void* logits, int dtype, size_t n) {
    const DType d = to_dtype(dtype);
    float best = -std::numeric_limits<float>::infinity();
    size_t best_idx = 0;
    for (size_t i = 0; i < n; ++i) {
        const float v = mruntime::load_scalar_as_fp32(logits, d, i);
        if (v > best) {
            best = v;
            best_idx = i;
        }
    }
    return static_cast<int64_t>(best_idx);
}

}  // extern "C"
