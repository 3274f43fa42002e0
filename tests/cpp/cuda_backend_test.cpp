// cuda_backend_test.cpp -- CudaBackend as a drop-in mruntime::Backend.
//
// Written like the reference's own test/backend_test.cpp (one function per
// op, "PASSED" lines), but every result is compared with the reference's
// CpuBackend (compiled from its sources into oracle/_ref) on the same seeded
// inputs: bit-exact where the device path keeps the reference's arithmetic
// (general gemm, SiLU, mul, add, RoPE, embedding), within FP16 rounding of an
// FP32 sum otherwise.  The reference's ProfilingBackend decorator is wrapped
// around CudaBackend unchanged.  Needs a B200; run by tests/test_cuda_backend_gpu.py.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <iostream>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "cuda_backend.h"
#include "mruntime/cpu_backend.h"
#include "mruntime/profiling_backend.h"
#include "mruntime/tensor.h"

using namespace mruntime;
using mruntime_b200::CudaBackend;
using mruntime_b200::DeviceTensor;

namespace {

int g_failures = 0;

#define CHECK(cond, msg)                                                          \
    do {                                                                          \
        if (!(cond)) {                                                            \
            std::cerr << "CHECK FAILED " << __FILE__ << ":" << __LINE__ << ": " << msg << "\n"; \
            ++g_failures;                                                         \
        }                                                                         \
    } while (0)

Tensor random_tensor(Shape shape, DType dt, float stddev, uint32_t seed) {
    Tensor t = Tensor::empty(std::move(shape), dt);
    std::mt19937 gen(seed);
    std::normal_distribution<float> nd(0.0f, stddev);
    for (size_t i = 0; i < t.numel(); ++i) store_scalar_from_fp32(t.data(), dt, i, nd(gen));
    return t;
}

Tensor clone(const Tensor& t) {
    Tensor c = Tensor::empty(Shape(t.shape().dims()), t.dtype());
    std::memcpy(c.data(), t.data(), t.nbytes());
    return c;
}

size_t count_diff(const Tensor& a, const Tensor& b) {
    size_t d = 0;
    const uint8_t* x = static_cast<const uint8_t*>(a.data());
    const uint8_t* y = static_cast<const uint8_t*>(b.data());
    const size_t es = dtype_size(a.dtype());
    for (size_t i = 0; i < a.numel(); ++i) d += std::memcmp(x + i * es, y + i * es, es) != 0;
    return d;
}

// Largest |a - b| in units of the FP16 spacing at |b| (at least one subnormal step).
double max_ulp_fp16(const Tensor& a, const Tensor& b) {
    double worst = 0.0;
    for (size_t i = 0; i < a.numel(); ++i) {
        const double x = load_scalar_as_fp32(a.data(), a.dtype(), i);
        const double y = load_scalar_as_fp32(b.data(), b.dtype(), i);
        const double spacing = std::max(std::ldexp(1.0, std::ilogb(std::max(std::fabs(y), 6.1e-5)) - 10), 5.96e-8);
        worst = std::max(worst, std::fabs(x - y) / spacing);
    }
    return worst;
}

// Elements of Y (device) and R (reference) for Y = X * W^T may differ by the
// FP16 rounding of two different FP32 sums: one FP16 spacing at |R| plus
// 4 sqrt(K) 2^-24 sum_k |x w| (FP32 summation in any order).  Returns the
// number of elements outside that bound.
size_t outside_fp32_sum_bound(const Tensor& X, const Tensor& W, const Tensor& Y, const Tensor& R) {
    const size_t K = X.dim(X.ndim() - 1), M = X.numel() / K, N = W.dim(0);
    size_t bad = 0;
    for (size_t m = 0; m < M; ++m)
        for (size_t n = 0; n < N; ++n) {
            double absdot = 0.0;
            for (size_t k = 0; k < K; ++k)
                absdot += std::fabs(static_cast<double>(load_scalar_as_fp32(X.data(), X.dtype(), m * K + k)) *
                                    load_scalar_as_fp32(W.data(), W.dtype(), n * K + k));
            const double y = load_scalar_as_fp32(Y.data(), Y.dtype(), m * N + n);
            const double r = load_scalar_as_fp32(R.data(), R.dtype(), m * N + n);
            const double spacing = std::max(std::ldexp(1.0, std::ilogb(std::max(std::fabs(r), 6.1e-5)) - 10), 5.96e-8);
            if (std::fabs(y - r) > spacing + 4.0 * std::sqrt(static_cast<double>(K)) * std::ldexp(1.0, -24) * absdot)
                ++bad;
        }
    return bad;
}

void test_gemm_known_answer(CudaBackend& backend) {
    // reference test/backend_test.cpp:11-29
    Tensor A = Tensor::zeros(Shape({2, 3}), DType::FP16);
    Tensor B = Tensor::zeros(Shape({3, 4}), DType::FP16);
    Tensor C = Tensor::zeros(Shape({2, 4}), DType::FP16);
    for (int i = 0; i < 6; ++i) A.data_ptr<uint16_t>()[i] = float_to_fp16_bits(static_cast<float>(i + 1));
    for (int i = 0; i < 12; ++i) B.data_ptr<uint16_t>()[i] = float_to_fp16_bits(static_cast<float>(i + 1));
    backend.gemm(A, B, C);
    const uint16_t* c = C.data_ptr<uint16_t>();
    CHECK(std::abs(fp16_bits_to_float(c[0]) - 38.0f) < 0.05f, "C[0,0]");
    CHECK(std::abs(fp16_bits_to_float(c[1]) - 44.0f) < 0.05f, "C[0,1]");
    CpuBackend cpu(4);
    Tensor R = Tensor::zeros(Shape({2, 4}), DType::FP16);
    cpu.gemm(A, B, R);
    CHECK(count_diff(C, R) == 0, "known-answer gemm differs from CpuBackend");
    std::cout << "test_gemm_known_answer PASSED\n";
}

void test_gemm_general_patterns(CudaBackend& backend) {
    CpuBackend cpu(4);
    // trans_a, alpha, beta, FP32 and BF16 operands: the general device kernel
    // keeps the reference's k-order FP32 sum, so results are bit-exact.
    Tensor A = random_tensor(Shape({13, 7}), DType::FP16, 1.0f, 1);
    Tensor B = random_tensor(Shape({13, 9}), DType::BF16, 0.1f, 2);
    Tensor C0 = random_tensor(Shape({7, 9}), DType::FP32, 1.0f, 3);
    Tensor C = clone(C0), R = clone(C0);
    backend.gemm(A, B, C, 0.5f, 0.25f, true, false);
    cpu.gemm(A, B, R, 0.5f, 0.25f, true, false);
    CHECK(count_diff(C, R) == 0, "trans_a/alpha/beta gemm differs from CpuBackend");
    Tensor A3 = random_tensor(Shape({1, 5, 12}), DType::FP16, 1.0f, 4);  // 3-D A, flattened rows
    Tensor W = random_tensor(Shape({6, 12}), DType::FP16, 0.1f, 5);
    Tensor C3 = Tensor::zeros(Shape({1, 5, 6}), DType::FP16), R3 = Tensor::zeros(Shape({1, 5, 6}), DType::FP16);
    backend.gemm(A3, W, C3, 1.0f, 0.0f, false, true);
    cpu.gemm(A3, W, R3, 1.0f, 0.0f, false, true);
    CHECK(count_diff(C3, R3) == 0, "K=12 model-layout gemm (general path) differs");
    bool threw = false;
    try {
        Tensor bad = Tensor::zeros(Shape({5, 6}), DType::FP16);
        backend.gemm(A3, W, bad, 1.0f, 0.0f, true, true);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    CHECK(threw, "shape mismatch must throw std::invalid_argument");
    std::cout << "test_gemm_general_patterns PASSED\n";
}

void test_gemm_model_layout(CudaBackend& backend) {
    CpuBackend cpu(0);
    for (size_t M : {1, 7, 16, 33, 300}) {
        Tensor X = random_tensor(Shape({1, M, 896}), DType::FP16, 1.0f, 10 + M);
        Tensor W = random_tensor(Shape({640, 896}), DType::BF16, 0.02f, 20 + M);
        Tensor Y = Tensor::empty(Shape({1, M, 640}), DType::FP16);
        Tensor R = Tensor::empty(Shape({1, M, 640}), DType::FP16);
        backend.gemm(X, W, Y, 1.0f, 0.0f, false, true);  // host tensors, weight uploaded on first use
        cpu.gemm(X, W, R, 1.0f, 0.0f, false, true);
        const size_t bad = outside_fp32_sum_bound(X, W, Y, R);
        const double frac = 1.0 - static_cast<double>(count_diff(Y, R)) / Y.numel();
        CHECK(bad == 0, "M=" << M << ": " << bad << " outputs outside the FP32-sum bound (max ulp "
                               << max_ulp_fp16(Y, R) << ")");
        CHECK(frac > 0.9, "M=" << M << " identical fraction " << frac);
        // device-resident operands with an explicit weight handle give the same bits
        Tensor Wd = backend.upload_weight(W);
        DeviceTensor Xd = DeviceTensor::from_host(X);
        DeviceTensor Yd(Shape({1, M, 640}), DType::FP16);
        backend.gemm(Xd.tensor(), Wd, Yd.tensor(), 1.0f, 0.0f, false, true);
        Tensor Y2 = Tensor::empty(Shape({1, M, 640}), DType::FP16);
        Yd.copy_to_host(Y2);
        CHECK(count_diff(Y, Y2) == 0, "device-resident call differs from host call, M=" << M);
    }
    std::cout << "test_gemm_model_layout PASSED\n";
}

void test_gemm_bias(CudaBackend& backend) {
    CpuBackend cpu(0);
    Tensor X = random_tensor(Shape({1, 9, 896}), DType::FP16, 1.0f, 31);
    Tensor W = random_tensor(Shape({128, 896}), DType::BF16, 0.02f, 32);
    Tensor b = random_tensor(Shape({128}), DType::FP16, 0.02f, 33);
    Tensor Wd = backend.upload_weight(W);
    backend.attach_bias(Wd, b);
    Tensor Y = Tensor::empty(Shape({1, 9, 128}), DType::FP16);
    backend.gemm_bias(X, Wd, Y);
    Tensor Y0 = Tensor::empty(Shape({1, 9, 128}), DType::FP16);
    backend.gemm(X, Wd, Y0, 1.0f, 0.0f, false, true);
    // qwen_model.cpp:143-150 applied to the unbiased device output
    for (size_t r = 0; r < 9; ++r)
        for (size_t i = 0; i < 128; ++i) {
            float v = load_scalar_as_fp32(Y0.data(), DType::FP16, r * 128 + i);
            v += load_scalar_as_fp32(b.data(), DType::FP16, i);
            store_scalar_from_fp32(Y0.data(), DType::FP16, r * 128 + i, v);
        }
    CHECK(count_diff(Y, Y0) == 0, "bias epilogue differs from the reference's add_bias step");
    std::cout << "test_gemm_bias PASSED\n";
}

void test_elementwise_ops(CudaBackend& backend) {
    CpuBackend cpu(0);
    Tensor a = random_tensor(Shape({1, 3, 4864}), DType::FP16, 3.0f, 41);
    Tensor b = random_tensor(Shape({1, 3, 4864}), DType::FP16, 3.0f, 42);
    Tensor o = Tensor::empty(a.shape(), DType::FP16), r = Tensor::empty(a.shape(), DType::FP16);
    backend.silu(a, o);
    cpu.silu(a, r);
    CHECK(count_diff(o, r) == 0, "silu differs");
    backend.elementwise_mul(a, b, o);
    cpu.elementwise_mul(a, b, r);
    CHECK(count_diff(o, r) == 0, "mul differs");
    backend.add(a, b, o);
    cpu.add(a, b, r);
    CHECK(count_diff(o, r) == 0, "add differs");
    Tensor w = random_tensor(Shape({4864}), DType::FP16, 1.0f, 43);
    backend.rmsnorm(a, w, o, 1e-6f);
    cpu.rmsnorm(a, w, r, 1e-6f);
    CHECK(max_ulp_fp16(o, r) <= 1.0, "rmsnorm more than 1 ulp off");
    Tensor s = random_tensor(Shape({4, 37}), DType::FP16, 2.0f, 44);
    Tensor so = Tensor::empty(s.shape(), DType::FP16), sr = Tensor::empty(s.shape(), DType::FP16);
    backend.softmax(s, so, -1);
    cpu.softmax(s, sr, -1);
    CHECK(max_ulp_fp16(so, sr) <= 2.0, "softmax more than 2 ulp off");
    std::cout << "test_elementwise_ops PASSED\n";
}

void test_rope_embedding_attention(CudaBackend& backend) {
    CpuBackend cpu(0);
    Tensor q = random_tensor(Shape({1, 5, 4, 64}), DType::FP16, 1.0f, 51);
    Tensor k = random_tensor(Shape({1, 5, 2, 64}), DType::FP16, 1.0f, 52);
    Tensor q2 = clone(q), k2 = clone(k);
    backend.rope(q, k, 17, 1000000.0f);
    cpu.rope(q2, k2, 17, 1000000.0f);
    CHECK(count_diff(q, q2) == 0 && count_diff(k, k2) == 0, "rope differs");
    Tensor table = random_tensor(Shape({50, 64}), DType::BF16, 0.5f, 53);
    std::vector<int> ids = {3, 0, 49, 3};
    Tensor e = Tensor::empty(Shape({1, 4, 64}), DType::FP16), er = Tensor::empty(Shape({1, 4, 64}), DType::FP16);
    backend.embedding_lookup(table, ids, e);
    cpu.embedding_lookup(table, ids, er);
    CHECK(count_diff(e, er) == 0, "embedding differs");
    bool threw = false;
    try {
        Tensor one = Tensor::empty(Shape({1, 1, 64}), DType::FP16);
        backend.embedding_lookup(table, {50}, one);
    } catch (const std::out_of_range&) {
        threw = true;
    }
    CHECK(threw, "out-of-range token id must throw std::out_of_range");
    Tensor Q = random_tensor(Shape({1, 2, 3, 64}), DType::FP16, 1.0f, 54);
    Tensor K = random_tensor(Shape({1, 2, 11, 64}), DType::FP16, 1.0f, 55);
    Tensor V = random_tensor(Shape({1, 2, 11, 64}), DType::FP16, 1.0f, 56);
    Tensor O = Tensor::empty(Shape({1, 2, 3, 64}), DType::FP16), OR = Tensor::empty(Shape({1, 2, 3, 64}), DType::FP16);
    backend.flash_attention(Q, K, V, O, 0.125f, true);
    cpu.flash_attention(Q, K, V, OR, 0.125f, true);
    CHECK(max_ulp_fp16(O, OR) <= 2.0, "attention more than 2 ulp off");
    std::cout << "test_rope_embedding_attention PASSED\n";
}

void test_profiling_decorator(CudaBackend& backend) {
    // reference test/profiling_backend_test.cpp:11-42 with CudaBackend inside
    ProfilingBackend::Options opts;
    opts.enabled = true;
    opts.trace_enabled = true;
    ProfilingBackend prof(backend, opts);
    Tensor A = Tensor::zeros(Shape({2, 3}), DType::FP16);
    Tensor B = Tensor::zeros(Shape({3, 4}), DType::FP16);
    Tensor C = Tensor::zeros(Shape({2, 4}), DType::FP16);
    for (int i = 0; i < 6; ++i) A.data_ptr<uint16_t>()[i] = float_to_fp16_bits(static_cast<float>(i + 1));
    for (int i = 0; i < 12; ++i) B.data_ptr<uint16_t>()[i] = float_to_fp16_bits(static_cast<float>(i + 1));
    prof.gemm(A, B, C);
    CHECK(std::abs(fp16_bits_to_float(C.data_ptr<uint16_t>()[0]) - 38.0f) < 0.05f, "C[0,0] through the decorator");
    const auto snap = prof.profiler().snapshot(BackendOp::Gemm);
    CHECK(snap.calls == 1 && snap.total_ns > 0, "decorator stats");
    CHECK(prof.trace_writer().event_count() == 1, "decorator trace");
    std::cout << "test_profiling_decorator PASSED\n";
}

}  // namespace

int main() {
    try {
        CudaBackend backend(0);
        const int64_t launches0 = backend.kernel_launches();
        test_gemm_known_answer(backend);
        test_gemm_general_patterns(backend);
        test_gemm_model_layout(backend);
        test_gemm_bias(backend);
        test_elementwise_ops(backend);
        test_rope_embedding_attention(backend);
        test_profiling_decorator(backend);
        std::cout << "kernel launches: " << backend.kernel_launches() - launches0 << "\n";
    } catch (const std::exception& e) {
        std::cerr << "exception: " << e.what() << "\n";
        return 2;
    }
    if (g_failures != 0) {
        std::cerr << g_failures << " check(s) failed\n";
        return 1;
    }
    std::cout << "\nAll CudaBackend tests passed!\n";
    return 0;
}
