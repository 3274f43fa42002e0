// cuda_backend.cpp -- mruntime::Backend on a B200, over the C ABI (mrt_b200.h).
#include "cuda_backend.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

using mruntime::DType;
using mruntime::Shape;
using mruntime::Tensor;

namespace mruntime_b200 {
namespace {

int to_mrt(DType d) {
    switch (d) {
        case DType::FP16: return MRT_FP16;
        case DType::BF16: return MRT_BF16;
        case DType::FP32: return MRT_FP32;
    }
    throw std::invalid_argument("unknown dtype");
}

void throw_on(int rc, const char* what) {
    if (rc == MRT_OK) return;
    std::string msg = std::string(what) + ": " + mrt_last_error_string();
    if (rc == MRT_ERR_SHAPE || rc == MRT_ERR_DTYPE || rc == MRT_ERR_INVALID_ARG) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

bool on_device(const void* p) {
    int kind = MRT_PTR_HOST;
    if (p == nullptr) return false;
    throw_on(mrt_pointer_kind(p, &kind), "mrt_pointer_kind");
    return kind != MRT_PTR_HOST;
}

// Rows of a 2-D or 3-D contiguous tensor viewed as a matrix (the reference
// flattens a 3-D A to dim0*dim1 rows, cpu_backend.cpp:87).
size_t rows_of(const Tensor& t) { return t.ndim() == 2 ? t.dim(0) : t.dim(0) * t.dim(1); }

}  // namespace

// ------------------------------------------------------------------ DeviceTensor

DeviceTensor::DeviceTensor(Shape shape, DType dtype) {
    void* p = nullptr;
    const size_t bytes = shape.numel() * mruntime::dtype_size(dtype);
    throw_on(mrt_device_alloc(bytes, &p), "mrt_device_alloc");
    storage_ = std::shared_ptr<void>(p, [](void* q) { mrt_device_free(q); });
    view_ = Tensor::from_buffer(p, std::move(shape), dtype, false);
}

DeviceTensor DeviceTensor::from_host(const Tensor& host) {
    if (!host.is_contiguous()) throw std::invalid_argument("DeviceTensor::from_host needs a contiguous tensor");
    DeviceTensor d(Shape(host.shape().dims()), host.dtype());
    d.copy_from_host(host);
    return d;
}

void DeviceTensor::copy_from_host(const Tensor& host) {
    if (host.nbytes() != nbytes()) throw std::invalid_argument("size mismatch");
    throw_on(mrt_memcpy(storage_.get(), host.data(), nbytes(), nullptr), "mrt_memcpy");
}

void DeviceTensor::copy_to_host(Tensor& host) const {
    if (host.nbytes() != nbytes()) throw std::invalid_argument("size mismatch");
    throw_on(mrt_memcpy(host.data(), storage_.get(), nbytes(), nullptr), "mrt_memcpy");
}

// ------------------------------------------------------------------ CudaBackend

CudaBackend::CudaBackend(int device) : device_(device) { throw_on(mrt_init(device), "mrt_init"); }

CudaBackend::~CudaBackend() {
    mrt_sync(stream_);
    for (auto& kv : uploaded_) mrt_weight_free(kv.second);
    for (auto& kv : implicit_) mrt_weight_free(kv.second.w);
    for (auto& kv : tables_) mrt_device_free(kv.second.data);
    for (auto& s : scratch_) mrt_device_free(s.first);
}

int64_t CudaBackend::kernel_launches() const {
    int64_t n = 0;
    mrt_launch_count(&n);
    return n;
}

void CudaBackend::check(int rc, const char* what) const { throw_on(rc, what); }

void CudaBackend::sync() { check(mrt_sync(stream_), "mrt_sync"); }

void* CudaBackend::scratch(int slot, size_t bytes) {
    if (scratch_.size() <= static_cast<size_t>(slot)) scratch_.resize(slot + 1, {nullptr, 0});
    auto& s = scratch_[slot];
    if (s.second < bytes) {
        if (s.first) {
            sync();
            mrt_device_free(s.first);
            s = {nullptr, 0};
        }
        void* p = nullptr;
        check(mrt_device_alloc(bytes, &p), "allocating staging memory");
        s = {p, bytes};
    }
    return s.first;
}

CudaBackend::Staged CudaBackend::stage_in(const Tensor& t, int slot) {
    if (t.numel() == 0) return {};
    if (on_device(t.data())) return {const_cast<void*>(t.data()), false};
    void* d = scratch(slot, t.nbytes());
    check(mrt_memcpy(d, t.data(), t.nbytes(), stream_), "copying an operand to the device");
    return {d, true};
}

CudaBackend::Staged CudaBackend::stage_out(const Tensor& t, int slot, bool need_contents) {
    if (t.numel() == 0) return {};
    if (on_device(t.data())) return {const_cast<void*>(t.data()), false};
    void* d = scratch(slot, t.nbytes());
    if (need_contents) check(mrt_memcpy(d, t.data(), t.nbytes(), stream_), "copying an output to the device");
    return {d, true};
}

void CudaBackend::finish_out(const Staged& s, Tensor& t) {
    if (s.staged) check(mrt_memcpy(t.data(), s.ptr, t.nbytes(), stream_), "copying a result to the host");
    sync();
}

Tensor CudaBackend::upload_weight(const Tensor& weight) {
    if (weight.ndim() != 2 || !weight.is_contiguous())
        throw std::invalid_argument("upload_weight: need a contiguous [N, K] tensor");
    const int64_t N = static_cast<int64_t>(weight.dim(0)), K = static_cast<int64_t>(weight.dim(1));
    mrt_weight w = nullptr;
    check(mrt_weight_upload(weight.data(), to_mrt(weight.dtype()), on_device(weight.data()) ? 1 : 0, N, K, nullptr,
                            0, 0, K, stream_, &w),
          "mrt_weight_upload");
    void* data = nullptr;
    check(mrt_weight_data(w, &data, nullptr), "mrt_weight_data");
    uploaded_[data] = w;
    // A handle: the data is in the library's (tiled) layout, so the view is
    // meant for gemm/gemm_bias/attach_bias only.
    return Tensor::from_buffer(data, Shape({weight.dim(0), weight.dim(1)}), DType::FP16, false);
}

void CudaBackend::attach_bias(const Tensor& uploaded_weight, const Tensor& bias) {
    auto it = uploaded_.find(uploaded_weight.data());
    if (it == uploaded_.end()) throw std::invalid_argument("attach_bias: weight was not returned by upload_weight");
    if (bias.numel() != uploaded_weight.dim(0)) throw std::invalid_argument("attach_bias: bias length != N");
    check(mrt_weight_attach_bias(it->second, bias.data(), to_mrt(bias.dtype()), on_device(bias.data()) ? 1 : 0,
                                 stream_),
          "mrt_weight_attach_bias");
}

// FNV-1a over 64 elements spread evenly across a host tensor (0 for device
// tensors, whose contents are not inspected).
uint64_t CudaBackend::fingerprint(const Tensor& t) {
    if (on_device(t.data()) || t.numel() == 0) return 0;
    const size_t es = mruntime::dtype_size(t.dtype());
    const uint8_t* p = static_cast<const uint8_t*>(t.data());
    uint64_t h = 1469598103934665603ull;
    const size_t n = t.numel();
    for (size_t i = 0; i < 64; ++i) {
        const size_t idx = (n * i) / 64 + (i * 7919u) % std::max<size_t>(1, n / 64);
        for (size_t b = 0; b < es; ++b) {
            h ^= p[std::min(idx, n - 1) * es + b];
            h *= 1099511628211ull;
        }
    }
    return h;
}

const void* CudaBackend::device_table(const Tensor& t) {
    if (on_device(t.data())) return t.data();
    const auto key = std::make_tuple(static_cast<const void*>(t.data()), t.dim(0), t.dim(1), to_mrt(t.dtype()));
    const uint64_t fp = fingerprint(t);
    auto it = tables_.find(key);
    if (it != tables_.end()) {
        if (it->second.fingerprint == fp) return it->second.data;
        sync();
        mrt_device_free(it->second.data);
        tables_.erase(it);
    }
    void* d = nullptr;
    check(mrt_device_alloc(t.nbytes(), &d), "allocating an embedding table");
    check(mrt_memcpy(d, t.data(), t.nbytes(), stream_), "uploading an embedding table");
    tables_[key] = Table{d, fp};
    return d;
}

mrt_weight CudaBackend::weight_for(const Tensor& B, size_t N, size_t K) {
    auto up = uploaded_.find(B.data());
    if (up != uploaded_.end()) return up->second;
    const auto key = std::make_tuple(static_cast<const void*>(B.data()), N, K, to_mrt(B.dtype()));
    const uint64_t fp = fingerprint(B);
    auto it = implicit_.find(key);
    if (it != implicit_.end()) {
        if (it->second.fingerprint == fp) return it->second.w;
        sync();
        mrt_weight_free(it->second.w);  // the address now holds a different tensor
        implicit_.erase(it);
    }
    mrt_weight w = nullptr;
    const bool dev = on_device(B.data());
    if (dev && B.dtype() == DType::FP16) {
        check(mrt_weight_view(B.data(), static_cast<int64_t>(N), static_cast<int64_t>(K), &w), "mrt_weight_view");
    } else {
        check(mrt_weight_upload(B.data(), to_mrt(B.dtype()), dev ? 1 : 0, static_cast<int64_t>(N),
                                static_cast<int64_t>(K), nullptr, 0, 0, static_cast<int64_t>(K), stream_, &w),
              "mrt_weight_upload");
    }
    implicit_[key] = Implicit{w, fp};
    return w;
}

// Backend::gemm (reference include/mruntime/backend.h:13-21).  Shape rules and
// the fast-path condition follow CpuBackend::gemm (src/core/cpu_backend.cpp:81-106);
// shape errors throw std::invalid_argument where the reference asserts.
void CudaBackend::gemm(const Tensor& A, const Tensor& B, Tensor& C, float alpha, float beta, bool trans_a,
                       bool trans_b) {
    if (!A.is_contiguous() || !B.is_contiguous() || !C.is_contiguous())
        throw std::invalid_argument("gemm: operands must be contiguous");
    if ((A.ndim() != 2 && A.ndim() != 3) || B.ndim() != 2 || (C.ndim() != 2 && C.ndim() != 3))
        throw std::invalid_argument("gemm: A and C must be 2-D or 3-D, B 2-D");
    const size_t a_rows0 = rows_of(A), a_cols0 = A.dim(A.ndim() - 1);
    const size_t b_rows0 = B.dim(0), b_cols0 = B.dim(1);
    const size_t M = trans_a ? a_cols0 : a_rows0;
    const size_t K = trans_a ? a_rows0 : a_cols0;
    const size_t N = trans_b ? b_rows0 : b_cols0;
    if ((trans_b ? b_cols0 : b_rows0) != K) throw std::invalid_argument("gemm: inner dimensions differ");
    if (rows_of(C) != M || C.dim(C.ndim() - 1) != N) throw std::invalid_argument("gemm: C has the wrong shape");
    if (M == 0 || N == 0) return;  // cpu_backend.cpp:124-126

    const bool model_call = !trans_a && trans_b && alpha == 1.0f && beta == 0.0f && A.dtype() == DType::FP16 &&
                            C.dtype() == DType::FP16 && (B.dtype() == DType::FP16 || B.dtype() == DType::BF16);
    if (model_call && K > 0) {
        mrt_weight w = weight_for(B, N, K);
        Staged a = stage_in(A, 0);
        Staged c = stage_out(C, 1, false);
        check(mrt_gemm(w, a.ptr, static_cast<int64_t>(K), c.ptr, static_cast<int64_t>(N), static_cast<int64_t>(M), 0,
                       stream_),
              "mrt_gemm");
        finish_out(c, C);
        return;
    }
    Staged a = stage_in(A, 0);
    Staged b = stage_in(B, 2);
    Staged c = stage_out(C, 1, beta != 0.0f);
    check(mrt_gemm_general(a.ptr, to_mrt(A.dtype()), static_cast<int64_t>(a_rows0), static_cast<int64_t>(a_cols0),
                           b.ptr, to_mrt(B.dtype()), static_cast<int64_t>(b_rows0), static_cast<int64_t>(b_cols0), c.ptr,
                           to_mrt(C.dtype()), alpha, beta, trans_a ? 1 : 0, trans_b ? 1 : 0, stream_),
          "mrt_gemm_general");
    finish_out(c, C);
}

void CudaBackend::gemm_bias(const Tensor& A, const Tensor& uploaded_weight, Tensor& C) {
    auto it = uploaded_.find(uploaded_weight.data());
    if (it == uploaded_.end()) throw std::invalid_argument("gemm_bias: weight was not returned by upload_weight");
    const size_t M = rows_of(A), K = A.dim(A.ndim() - 1), N = uploaded_weight.dim(0);
    if (uploaded_weight.dim(1) != K || rows_of(C) != M || C.dim(C.ndim() - 1) != N)
        throw std::invalid_argument("gemm_bias: shape mismatch");
    if (A.dtype() != DType::FP16 || C.dtype() != DType::FP16) throw std::invalid_argument("gemm_bias: FP16 A and C");
    Staged a = stage_in(A, 0);
    Staged c = stage_out(C, 1, false);
    check(mrt_gemm(it->second, a.ptr, static_cast<int64_t>(K), c.ptr, static_cast<int64_t>(N), static_cast<int64_t>(M),
                   MRT_GEMM_BIAS, stream_),
          "mrt_gemm");
    finish_out(c, C);
}

// cpu_backend.cpp:171-290
void CudaBackend::flash_attention(const Tensor& Q, const Tensor& K, const Tensor& V, Tensor& output, float scale,
                                  bool causal) {
    if (Q.ndim() != 4 || K.ndim() != 4 || V.ndim() != 4 || output.ndim() != 4)
        throw std::invalid_argument("flash_attention: 4-D tensors expected");
    const int64_t b = Q.dim(0), h = Q.dim(1), q_len = Q.dim(2), d = Q.dim(3), kv = K.dim(2), vd = V.dim(3);
    if (K.dim(0) != Q.dim(0) || K.dim(1) != Q.dim(1) || V.dim(0) != Q.dim(0) || V.dim(1) != Q.dim(1) ||
        K.dim(3) != Q.dim(3) || V.dim(2) != K.dim(2) || output.dim(0) != Q.dim(0) || output.dim(1) != Q.dim(1) ||
        output.dim(2) != Q.dim(2) || output.dim(3) != V.dim(3))
        throw std::invalid_argument("flash_attention: shape mismatch");
    // Strided views are passed as-is when on the device; host views are
    // staged with the extent their strides span.
    auto span = [](const Tensor& t) {
        size_t last = 0;
        for (size_t i = 0; i < 4; ++i) last += (t.dim(i) - 1) * t.stride(i);
        return (last + 1) * mruntime::dtype_size(t.dtype());
    };
    auto in = [&](const Tensor& t, int slot) -> void* {
        if (on_device(t.data())) return const_cast<void*>(t.data());
        void* p = scratch(slot, span(t));
        check(mrt_memcpy(p, t.data(), span(t), stream_), "copying an attention operand");
        return p;
    };
    void* q = in(Q, 0);
    void* k = in(K, 2);
    void* v = in(V, 3);
    const bool out_dev = on_device(output.data());
    void* o = out_dev ? output.data() : scratch(1, span(output));
    if (!out_dev) check(mrt_memcpy(o, output.data(), span(output), stream_), "copying the attention output");
    int64_t qs[4], ks[4], vs[4], os[4];
    for (int i = 0; i < 4; ++i) {
        qs[i] = Q.stride(i); ks[i] = K.stride(i); vs[i] = V.stride(i); os[i] = output.stride(i);
    }
    check(mrt_attention(q, to_mrt(Q.dtype()), qs, k, to_mrt(K.dtype()), ks, v, to_mrt(V.dtype()), vs, o,
                        to_mrt(output.dtype()), os, b, h, q_len, kv, d, vd, scale, causal ? 1 : 0, stream_),
          "mrt_attention");
    if (!out_dev) check(mrt_memcpy(output.data(), o, span(output), stream_), "copying the attention result");
    sync();
}

// cpu_backend.cpp:292-330
void CudaBackend::rmsnorm(const Tensor& input, const Tensor& weight, Tensor& output, float eps) {
    if (!input.is_contiguous() || !weight.is_contiguous() || !output.is_contiguous())
        throw std::invalid_argument("rmsnorm: contiguous tensors expected");
    const size_t hidden = input.dim(input.ndim() - 1);
    Staged i = stage_in(input, 0);
    Staged w = stage_in(weight, 2);
    Staged o = stage_out(output, 1, false);
    check(mrt_rmsnorm(i.ptr, to_mrt(input.dtype()), w.ptr, to_mrt(weight.dtype()), o.ptr, to_mrt(output.dtype()),
                      static_cast<int64_t>(input.numel() / hidden), static_cast<int64_t>(hidden), eps, stream_),
          "mrt_rmsnorm");
    finish_out(o, output);
}

// cpu_backend.cpp:332-379: Q and K are [batch, seq, heads, head_dim], rotated in place.
void CudaBackend::rope(Tensor& Q, Tensor& K, size_t position_offset, float theta) {
    for (Tensor* t : {&Q, &K}) {
        if (t->ndim() != 4 || !t->is_contiguous()) throw std::invalid_argument("rope: contiguous 4-D tensors expected");
        Staged s = stage_out(*t, 1, true);
        check(mrt_rope(s.ptr, to_mrt(t->dtype()), t->dim(0), t->dim(1), t->dim(2), t->dim(3),
                       static_cast<int64_t>(position_offset), theta, stream_),
              "mrt_rope");
        finish_out(s, *t);
    }
}

void CudaBackend::silu(const Tensor& input, Tensor& output) {
    if (input.numel() != output.numel()) throw std::invalid_argument("silu: size mismatch");
    Staged i = stage_in(input, 0);
    Staged o = stage_out(output, 1, false);
    check(mrt_silu(i.ptr, to_mrt(input.dtype()), o.ptr, to_mrt(output.dtype()), static_cast<int64_t>(input.numel()),
                   stream_),
          "mrt_silu");
    finish_out(o, output);
}

void CudaBackend::elementwise_mul(const Tensor& a, const Tensor& b, Tensor& output) {
    if (a.numel() != b.numel() || a.numel() != output.numel()) throw std::invalid_argument("mul: size mismatch");
    Staged x = stage_in(a, 0);
    Staged y = stage_in(b, 2);
    Staged o = stage_out(output, 1, false);
    check(mrt_mul(x.ptr, to_mrt(a.dtype()), y.ptr, to_mrt(b.dtype()), o.ptr, to_mrt(output.dtype()),
                  static_cast<int64_t>(a.numel()), stream_),
          "mrt_mul");
    finish_out(o, output);
}

void CudaBackend::add(const Tensor& a, const Tensor& b, Tensor& output) {
    if (a.numel() != b.numel() || a.numel() != output.numel()) throw std::invalid_argument("add: size mismatch");
    Staged x = stage_in(a, 0);
    Staged y = stage_in(b, 2);
    Staged o = stage_out(output, 1, false);
    check(mrt_add(x.ptr, to_mrt(a.dtype()), y.ptr, to_mrt(b.dtype()), o.ptr, to_mrt(output.dtype()),
                  static_cast<int64_t>(a.numel()), stream_),
          "mrt_add");
    finish_out(o, output);
}

// cpu_backend.cpp:457-515
void CudaBackend::softmax(const Tensor& input, Tensor& output, int dim) {
    if (input.numel() != output.numel()) throw std::invalid_argument("softmax: size mismatch");
    if (dim < 0) dim += static_cast<int>(input.ndim());
    if (dim < 0 || static_cast<size_t>(dim) >= input.ndim()) throw std::invalid_argument("softmax: bad dim");
    int64_t outer = 1, inner = 1;
    for (int i = 0; i < dim; ++i) outer *= input.dim(i);
    for (size_t i = dim + 1; i < input.ndim(); ++i) inner *= input.dim(i);
    Staged i = stage_in(input, 0);
    Staged o = stage_out(output, 1, false);
    check(mrt_softmax(i.ptr, to_mrt(input.dtype()), o.ptr, to_mrt(output.dtype()), outer,
                      static_cast<int64_t>(input.dim(dim)), inner, stream_),
          "mrt_softmax");
    finish_out(o, output);
}

// cpu_backend.cpp:517-569 (an out-of-range id throws std::out_of_range, as there)
void CudaBackend::embedding_lookup(const Tensor& weight, const std::vector<int>& token_ids, Tensor& output) {
    if (weight.ndim() != 2 || output.ndim() != 3 || output.dim(0) != 1 || output.dim(1) != token_ids.size() ||
        output.dim(2) != weight.dim(1))
        throw std::invalid_argument("embedding_lookup: shape mismatch");
    for (int id : token_ids)
        if (id < 0 || static_cast<size_t>(id) >= weight.dim(0))
            throw std::out_of_range("embedding_lookup: token_id out of range");
    if (token_ids.empty()) return;
    // The table can be large: use it in place when it is on the device,
    // otherwise keep one row-major device copy per host table.
    const void* w = device_table(weight);
    const int wdt = to_mrt(weight.dtype());
    std::vector<int32_t> ids(token_ids.begin(), token_ids.end());
    Staged o = stage_out(output, 1, false);
    check(mrt_embedding(w, wdt, static_cast<int64_t>(weight.dim(0)), static_cast<int64_t>(weight.dim(1)), ids.data(),
                        static_cast<int64_t>(ids.size()), o.ptr, to_mrt(output.dtype()), stream_),
          "mrt_embedding");
    finish_out(o, output);
}

}  // namespace mruntime_b200
