// cuda_backend.h -- mruntime::Backend on a B200.
//
// CudaBackend implements the reference's abstract Backend
// (include/mruntime/backend.h:9-74, included from the reference tree, not
// copied) so QwenModel / InferenceEngine take it wherever they take
// CpuBackend.  Its gemm runs the sm_100a kernels through the C ABI in
// mrt_b200.h; every other call is a thin host-side layer over that ABI.
//
// Tensors may live in host memory (the reference's own Tensor storage) or in
// device memory (DeviceTensor below, or any Tensor::from_buffer over a device
// pointer); host operands are staged through device buffers inside the call.
// Calls are synchronous, as the reference's are: outputs are valid on return.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <tuple>
#include <vector>

#include "mrt_b200.h"
#include "mruntime/backend.h"
#include "mruntime/tensor.h"

namespace mruntime_b200 {

// Device storage with a mruntime::Tensor view of it (the device counterpart
// of Tensor::empty, reference src/core/tensor.cpp:8-12).
class DeviceTensor {
public:
    DeviceTensor() = default;
    DeviceTensor(mruntime::Shape shape, mruntime::DType dtype);
    static DeviceTensor from_host(const mruntime::Tensor& host);

    mruntime::Tensor& tensor() { return view_; }
    const mruntime::Tensor& tensor() const { return view_; }
    void* data() const { return storage_.get(); }
    size_t nbytes() const { return view_.nbytes(); }
    void copy_from_host(const mruntime::Tensor& host);
    void copy_to_host(mruntime::Tensor& host) const;

private:
    std::shared_ptr<void> storage_;
    mruntime::Tensor view_;
};

class CudaBackend : public mruntime::Backend {
public:
    explicit CudaBackend(int device = 0);
    ~CudaBackend() override;
    CudaBackend(const CudaBackend&) = delete;
    CudaBackend& operator=(const CudaBackend&) = delete;

    // Upload a projection weight [N, K] (FP16/BF16/FP32, host or device) once
    // and return a Tensor view of the device FP16 copy; gemm() recognises the
    // view and streams it directly.  This replaces the reference's packed-RHS
    // cache keyed by raw pointer (src/core/cpu_backend.cpp:24-30) with an
    // explicit handle.
    mruntime::Tensor upload_weight(const mruntime::Tensor& weight);

    // Upload a bias for a weight returned by upload_weight; gemm_bias() then
    // applies it with the reference's q/k/v rounding (qwen_model.cpp:130-155).
    void attach_bias(const mruntime::Tensor& uploaded_weight, const mruntime::Tensor& bias);
    void gemm_bias(const mruntime::Tensor& A, const mruntime::Tensor& uploaded_weight, mruntime::Tensor& C);

    // Stream the backend issues work on (default: the legacy stream).
    void set_stream(void* stream) { stream_ = stream; }
    void* stream() const { return stream_; }
    int device() const { return device_; }
    // Number of kernels launched by the library so far (diagnostics).
    int64_t kernel_launches() const;

    void gemm(const mruntime::Tensor& A, const mruntime::Tensor& B, mruntime::Tensor& C, float alpha = 1.0f,
              float beta = 0.0f, bool trans_a = false, bool trans_b = false) override;

    void flash_attention(const mruntime::Tensor& Q, const mruntime::Tensor& K, const mruntime::Tensor& V,
                         mruntime::Tensor& output, float scale, bool causal = true) override;
    void rmsnorm(const mruntime::Tensor& input, const mruntime::Tensor& weight, mruntime::Tensor& output,
                 float eps = 1e-6f) override;
    void rope(mruntime::Tensor& Q, mruntime::Tensor& K, size_t position_offset, float theta = 10000.0f) override;
    void silu(const mruntime::Tensor& input, mruntime::Tensor& output) override;
    void elementwise_mul(const mruntime::Tensor& a, const mruntime::Tensor& b, mruntime::Tensor& output) override;
    void add(const mruntime::Tensor& a, const mruntime::Tensor& b, mruntime::Tensor& output) override;
    void softmax(const mruntime::Tensor& input, mruntime::Tensor& output, int dim = -1) override;
    void embedding_lookup(const mruntime::Tensor& weight, const std::vector<int>& token_ids,
                          mruntime::Tensor& output) override;

private:
    // A device view of an operand: its own pointer when it already lives on
    // the device, else a staging copy.
    struct Staged {
        void* ptr = nullptr;
        bool staged = false;
    };
    Staged stage_in(const mruntime::Tensor& t, int slot);
    Staged stage_out(const mruntime::Tensor& t, int slot, bool need_contents);
    void finish_out(const Staged& s, mruntime::Tensor& t);
    void* scratch(int slot, size_t bytes);
    mrt_weight weight_for(const mruntime::Tensor& B, size_t N, size_t K);
    void check(int rc, const char* what) const;
    void sync();

    int device_ = 0;
    void* stream_ = nullptr;
    // Uploaded weights by device data pointer.
    std::map<const void*, mrt_weight> uploaded_;
    // Weights first seen in gemm() (host or unregistered device memory), by
    // (pointer, rows, cols, dtype) -- the reference's own cache key -- plus a
    // fingerprint of sampled host elements, so a freed host weight whose
    // address is reused by a different tensor is uploaded again instead of
    // hitting the stale entry (the hazard of cpu_backend.cpp:24-30).
    struct Implicit {
        mrt_weight w = nullptr;
        uint64_t fingerprint = 0;
    };
    std::map<std::tuple<const void*, size_t, size_t, int>, Implicit> implicit_;
    static uint64_t fingerprint(const mruntime::Tensor& t);
    // Row-major device copies of host embedding tables (same key and check).
    struct Table {
        void* data = nullptr;
        uint64_t fingerprint = 0;
    };
    std::map<std::tuple<const void*, size_t, size_t, int>, Table> tables_;
    const void* device_table(const mruntime::Tensor& t);
    std::vector<std::pair<void*, size_t>> scratch_;
};

}  // namespace mruntime_b200
