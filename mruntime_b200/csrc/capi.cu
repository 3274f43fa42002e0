// capi.cu -- C ABI of the linear-layer path (declared in include/mrt_b200.h):
// device contexts, weight upload, GEMM planning and dispatch, argmax.
// Tensor-parallel entry points live in tp.cu.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ctx.h"
#include "kernels.h"

namespace mrt {

namespace {
thread_local std::string g_last_error;
std::mutex g_ctx_mu;
DevCtx* g_ctx[64] = {};
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

static std::atomic<int64_t> g_launches{0};
void note_launches(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int set_error(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    return set_error(MRT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                                       cudaGetErrorString(e) + ")");
}

void clear_error() { g_last_error.clear(); }

EncodeTiledFn encode_tiled_fn() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    return g_encode;
}

static DevCtx* create_ctx(int device) {
    DevCtx* c = new DevCtx();
    c->device = device;
    cudaError_t e = cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) {
        delete c;
        cuda_error(e, "cudaDeviceGetAttribute");
        return nullptr;
    }
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (major != 10) {
        delete c;
        set_error(MRT_ERR_UNSUPPORTED, "mruntime_b200 kernels are built for sm_100a (B200); device " +
                                           std::to_string(device) + " has compute capability major " +
                                           std::to_string(major));
        return nullptr;
    }
    e = cudaMalloc(&c->d_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        delete c;
        cuda_error(e, "allocating the device error flag");
        return nullptr;
    }
    return c;
}

DevCtx* current_ctx() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cuda_error(e, "cudaGetDevice");
        return nullptr;
    }
    if (dev < 0 || dev >= 64) {
        set_error(MRT_ERR_INVALID_ARG, "device index out of range");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    if (g_ctx[dev] == nullptr) g_ctx[dev] = create_ctx(dev);
    return g_ctx[dev];
}

int ensure_buffer(void** buf, size_t* cur, size_t bytes, const char* what) {
    if (*cur >= bytes) return MRT_OK;
    size_t want = std::max(bytes, *cur * 2);
    want = (want + 0xFFFFF) & ~size_t(0xFFFFF);  // 1 MiB granules
    if (*buf != nullptr) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_error(e, "synchronising before growing a buffer");
        cudaFree(*buf);
        *buf = nullptr;
        *cur = 0;
    }
    cudaError_t e = cudaMalloc(buf, want);
    if (e != cudaSuccess) {
        *buf = nullptr;
        return cuda_error(e, what);
    }
    *cur = want;
    return MRT_OK;
}

int make_tmap_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                  int box_rows) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (enc == nullptr) return set_error(MRT_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 2) % 16 != 0)
        return set_error(MRT_ERR_INVALID_ARG, "TMA operand must be 16-byte aligned with a 16-byte-multiple row pitch");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
    const cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1u, 1u};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(MRT_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r)));
    return MRT_OK;
}

int make_tmap_f16_rows64(CUtensorMap* map, const void* base, int64_t rows, int box_rows) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (enc == nullptr) return set_error(MRT_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return set_error(MRT_ERR_INVALID_ARG, "TMA operand must be 16-byte aligned");
    const cuuint64_t dims[2] = {64u, static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {128u};
    const cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1u, 1u};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(MRT_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r)));
    return MRT_OK;
}

}  // namespace mrt

using namespace mrt;

// ====================================================================== runtime

extern "C" int mrt_version(void) { return 100; }

extern "C" const char* mrt_last_error_string(void) { return g_last_error.c_str(); }

extern "C" int mrt_init(int device) {
    clear_error();
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    return current_ctx() ? MRT_OK : MRT_ERR_CUDA;
}

extern "C" int mrt_device_sm_count(int* out) {
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    if (out) *out = c->sms;
    return MRT_OK;
}

extern "C" int mrt_launch_count(int64_t* out) {
    if (out == nullptr) return set_error(MRT_ERR_INVALID_ARG, "out is NULL");
    *out = g_launches.load(std::memory_order_relaxed);
    return MRT_OK;
}

extern "C" int mrt_sync(void* stream) {
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    // the host-buffer copies queued by mrt_gemm_host_async
    if (e == cudaSuccess && c->io_out != nullptr) e = cudaStreamSynchronize(c->io_out);
    if (e == cudaSuccess && c->io_in != nullptr) e = cudaStreamSynchronize(c->io_in);
    if (e != cudaSuccess) return cuda_error(e, "cudaStreamSynchronize");
    int flag = 0;
    e = cudaMemcpy(&flag, c->d_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_error(e, "reading the device error flag");
    if (flag != 0) {
        cudaMemset(c->d_err, 0, sizeof(int));
        // A kernel that gave up may have left K-split tile counters counted.
        if (c->counters != nullptr) cudaMemset(c->counters, 0, c->counters_bytes);
        if (flag == 6)  // kErrBadToken: the decoder's embedding met an id outside the vocabulary
            return set_error(MRT_ERR_INVALID_ARG, "embedding_lookup: token_id out of range (device error code 6)");
        static const char* what[] = {"", "TMA producer", "MMA issuer", "epilogue", "clean-up", "wait self-test",
                                     "embedding", "peer all-reduce"};
        return set_error(MRT_ERR_TIMEOUT, std::string("a kernel wait timed out in the ") +
                                              (flag > 0 && flag < 8 ? what[flag] : "kernel") +
                                              " (device error code " + std::to_string(flag) + ")");
    }
    return MRT_OK;
}

extern "C" int mrt_selftest_wait_timeout(int limit_ms, void* stream) {
    clear_error();
    if (limit_ms < 1 || limit_ms > 10000) return set_error(MRT_ERR_INVALID_ARG, "limit_ms must be in [1, 10000]");
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    cudaError_t e = launch_wait_selftest(c->d_err, static_cast<uint64_t>(limit_ms) * 1000000ull,
                                         static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "self-test launch");
}

extern "C" int mrt_reserve_workspace(size_t bytes) {
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    return ensure_buffer(&c->ws, &c->ws_bytes, bytes, "allocating the scratch buffer");
}

// ====================================================================== weights

static size_t dtype_bytes(int dt) { return dt == MRT_FP32 ? 4 : 2; }

extern "C" int mrt_weight_upload(const void* src, int src_dtype, int src_on_device, int64_t N, int64_t K,
                                 const int64_t* row_ranges, int64_t n_ranges, int64_t k_begin,
                                 int64_t k_end, void* stream, mrt_weight* out) {
    clear_error();
    if (out == nullptr) return set_error(MRT_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (src == nullptr || N <= 0 || K <= 0) return set_error(MRT_ERR_INVALID_ARG, "empty or NULL weight");
    if (src_dtype != MRT_FP16 && src_dtype != MRT_BF16 && src_dtype != MRT_FP32)
        return set_error(MRT_ERR_DTYPE, "weight dtype must be FP16, BF16 or FP32");
    if (k_begin < 0 || k_end > K || k_begin >= k_end)
        return set_error(MRT_ERR_SHAPE, "column range must satisfy 0 <= k_begin < k_end <= K");
    std::vector<int64_t> ranges;
    if (row_ranges == nullptr || n_ranges == 0) {
        ranges = {0, N};
    } else {
        if (n_ranges < 0 || n_ranges > 64) return set_error(MRT_ERR_INVALID_ARG, "n_ranges must be in [0, 64]");
        ranges.assign(row_ranges, row_ranges + 2 * n_ranges);
    }
    int64_t n_keep = 0;
    for (size_t i = 0; i < ranges.size(); i += 2) {
        if (ranges[i] < 0 || ranges[i + 1] > N || ranges[i] >= ranges[i + 1])
            return set_error(MRT_ERR_SHAPE, "row range outside [0, N) or empty");
        n_keep += ranges[i + 1] - ranges[i];
    }
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t k_keep = k_end - k_begin;
    const size_t es = dtype_bytes(src_dtype);

    mrt_weight_s* w = new mrt_weight_s();
    w->device = c->device;
    w->n = n_keep;
    w->k = k_keep;
    w->src_n = N;
    w->n_ranges = static_cast<int64_t>(ranges.size() / 2);
    w->ranges = new int64_t[ranges.size()];
    std::copy(ranges.begin(), ranges.end(), w->ranges);
    // Weights the tensor-core kernels can stream (K a multiple of 8) are stored
    // pre-swizzled in 128 x 64 tiles; others stay row-major for the general kernel.
    w->tiled = (k_keep % 8) == 0;
    w->k_tiles = (k_keep + 63) / 64;
    w->n_pad = w->tiled ? (n_keep + 255) / 256 * 256 : n_keep;
    const size_t elems = w->tiled ? static_cast<size_t>(w->n_pad) * w->k_tiles * 64 : static_cast<size_t>(n_keep * k_keep);
    cudaError_t e = cudaMalloc(&w->data, elems * 2);
    if (e == cudaSuccess && w->tiled) e = cudaMemsetAsync(w->data, 0, elems * 2, s);
    if (e != cudaSuccess) {
        if (w->data) cudaFree(w->data);
        delete[] w->ranges;
        delete w;
        return cuda_error(e, "allocating weight storage");
    }
    void* stage = nullptr;
    int64_t row_off = 0;
    int rc = MRT_OK;
    for (size_t i = 0; i < ranges.size() && rc == MRT_OK; i += 2) {
        const int64_t rows = ranges[i + 1] - ranges[i];
        const char* s0 = static_cast<const char*>(src) + (ranges[i] * K + k_begin) * es;
        uint16_t* d0 = w->data + row_off * k_keep;
        if (w->tiled) {
            const void* dsrc = s0;
            int64_t dld = K;
            if (!src_on_device) {
                // Stage the native-dtype rows on the device first.
                if (stage != nullptr) {
                    cudaStreamSynchronize(s);
                    cudaFree(stage);
                    stage = nullptr;
                }
                e = cudaMalloc(&stage, static_cast<size_t>(rows * k_keep) * es);
                if (e == cudaSuccess)
                    e = cudaMemcpy2DAsync(stage, k_keep * es, s0, K * es, k_keep * es, rows, cudaMemcpyHostToDevice, s);
                dsrc = stage;
                dld = k_keep;
            }
            if (e == cudaSuccess)
                e = launch_convert_rows_to_tiled(dsrc, src_dtype, dld, rows, k_keep, w->data, row_off, w->k_tiles, s);
            if (e != cudaSuccess) rc = cuda_error(e, "uploading the weight into the tiled layout");
        } else if (src_dtype == MRT_FP16) {
            e = cudaMemcpy2DAsync(d0, k_keep * 2, s0, K * 2, k_keep * 2, rows,
                                  src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) rc = cuda_error(e, "copying the weight");
        } else if (src_on_device) {
            e = launch_convert_2d_to_f16(s0, src_dtype, K, rows, k_keep, d0, s);
            if (e != cudaSuccess) rc = cuda_error(e, "converting the weight to FP16");
        } else {
            // Stage the native-dtype rows on the device, then round once to FP16.
            if (stage != nullptr) {
                cudaStreamSynchronize(s);
                cudaFree(stage);
                stage = nullptr;
            }
            e = cudaMalloc(&stage, static_cast<size_t>(rows * k_keep) * es);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(stage, k_keep * es, s0, K * es, k_keep * es, rows, cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess) e = launch_convert_2d_to_f16(stage, src_dtype, k_keep, rows, k_keep, d0, s);
            if (e != cudaSuccess) rc = cuda_error(e, "staging and converting the weight");
        }
        row_off += rows;
    }
    e = cudaStreamSynchronize(s);
    if (stage != nullptr) cudaFree(stage);
    if (rc == MRT_OK && e != cudaSuccess) rc = cuda_error(e, "finishing the weight upload");
    if (rc != MRT_OK) {
        cudaFree(w->data);
        delete[] w->ranges;
        delete w;
        return rc;
    }
    *out = w;
    return MRT_OK;
}

extern "C" int mrt_weight_attach_bias(mrt_weight w, const void* src, int src_dtype, int src_on_device,
                                      void* stream) {
    clear_error();
    if (w == nullptr || src == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL weight or bias");
    if (src_dtype != MRT_FP16 && src_dtype != MRT_BF16 && src_dtype != MRT_FP32)
        return set_error(MRT_ERR_DTYPE, "bias dtype must be FP16, BF16 or FP32");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t es = dtype_bytes(src_dtype);
    if (w->bias == nullptr) {
        cudaError_t e = cudaMalloc(&w->bias, static_cast<size_t>(w->n) * 2);
        if (e != cudaSuccess) {
            w->bias = nullptr;
            return cuda_error(e, "allocating bias storage");
        }
    }
    void* stage = nullptr;
    cudaError_t e = cudaMalloc(&stage, static_cast<size_t>(w->src_n) * es);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(stage, src, static_cast<size_t>(w->src_n) * es,
                            src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s);
    int64_t off = 0;
    for (int64_t i = 0; i < w->n_ranges && e == cudaSuccess; ++i) {
        const int64_t b = w->ranges[2 * i], rows = w->ranges[2 * i + 1] - b;
        e = launch_convert(static_cast<const char*>(stage) + b * es, src_dtype, w->bias + off, MRT_FP16, rows, s);
        off += rows;
    }
    cudaError_t e2 = cudaStreamSynchronize(s);
    if (stage) cudaFree(stage);
    if (e != cudaSuccess) return cuda_error(e, "uploading the bias");
    if (e2 != cudaSuccess) return cuda_error(e2, "finishing the bias upload");
    return MRT_OK;
}

extern "C" int mrt_weight_view(const void* w_dev_f16, int64_t N, int64_t K, mrt_weight* out) {
    clear_error();
    if (out == nullptr || w_dev_f16 == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    if (N <= 0 || K <= 0) return set_error(MRT_ERR_SHAPE, "empty weight");
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    mrt_weight_s* w = new mrt_weight_s();
    w->device = c->device;
    w->n = N;
    w->k = K;
    w->src_n = N;
    w->data = static_cast<uint16_t*>(const_cast<void*>(w_dev_f16));
    w->owns_data = false;
    w->n_ranges = 1;
    w->ranges = new int64_t[2]{0, N};
    *out = w;
    return MRT_OK;
}

extern "C" int mrt_device_alloc(size_t bytes, void** out) {
    clear_error();
    if (out == nullptr) return set_error(MRT_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (!current_ctx()) return MRT_ERR_CUDA;
    if (bytes == 0) return MRT_OK;
    cudaError_t e = cudaMalloc(out, bytes);
    if (e != cudaSuccess) {
        *out = nullptr;
        return cuda_error(e, "cudaMalloc");
    }
    return MRT_OK;
}

extern "C" int mrt_device_free(void* p) {
    if (p == nullptr) return MRT_OK;
    cudaError_t e = cudaFree(p);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "cudaFree");
}

extern "C" int mrt_memcpy(void* dst, const void* src, size_t bytes, void* stream) {
    clear_error();
    if (bytes == 0) return MRT_OK;
    if (dst == nullptr || src == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyAsync");
    cudaPointerAttributes ad{}, as{};
    const bool pageable = cudaPointerGetAttributes(&ad, dst) != cudaSuccess || ad.type == cudaMemoryTypeUnregistered ||
                          cudaPointerGetAttributes(&as, src) != cudaSuccess || as.type == cudaMemoryTypeUnregistered;
    cudaGetLastError();  // clear a failed attribute query
    if (pageable) {
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_error(e, "waiting for a pageable copy");
    }
    return MRT_OK;
}

extern "C" int mrt_pointer_kind(const void* p, int* kind) {
    clear_error();
    if (kind == nullptr) return set_error(MRT_ERR_INVALID_ARG, "kind is NULL");
    cudaPointerAttributes a{};
    cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *kind = MRT_PTR_HOST;
        return MRT_OK;
    }
    *kind = a.type == cudaMemoryTypeDevice ? MRT_PTR_DEVICE
                                           : (a.type == cudaMemoryTypeManaged ? MRT_PTR_MANAGED : MRT_PTR_HOST);
    return MRT_OK;
}

extern "C" int mrt_weight_free(mrt_weight w) {
    if (w == nullptr) return MRT_OK;
    if (w->owns_data) cudaFree(w->data);
    if (w->bias) cudaFree(w->bias);
    delete[] w->ranges;
    delete w;
    return MRT_OK;
}

extern "C" int mrt_weight_shape(mrt_weight w, int64_t* n, int64_t* k) {
    if (w == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL weight");
    if (n) *n = w->n;
    if (k) *k = w->k;
    return MRT_OK;
}

extern "C" int mrt_weight_data(mrt_weight w, void** dev_ptr, int* tiled) {
    if (w == nullptr || dev_ptr == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    *dev_ptr = w->data;
    if (tiled) *tiled = w->tiled ? 1 : 0;
    return MRT_OK;
}

extern "C" int mrt_weight_read(mrt_weight w, void* dst_dev, int64_t ld, void* stream) {
    clear_error();
    if (w == nullptr || dst_dev == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    if (ld < w->k) return set_error(MRT_ERR_SHAPE, "ld must be >= K");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = w->tiled ? launch_untile(w->data, w->n, w->k, w->k_tiles, static_cast<uint16_t*>(dst_dev), ld, s)
                             : cudaMemcpy2DAsync(dst_dev, ld * 2, w->data, w->k * 2, w->k * 2, w->n,
                                                 cudaMemcpyDeviceToDevice, s);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "reading the weight");
}

// ====================================================================== GEMM

namespace mrt {

// Tile plan for the tcgen05 kernel.  A work unit of BN columns and kb
// 64-wide k-blocks on one SM costs the larger of its MMA time (one 128x128x64
// block-step is ~0.22 us at the sustained clock) and its operand streaming
// time (the SM's share of HBM bandwidth for W, L2 for X).  Units run round
// robin over the persistent CTAs.  Three shapes are compared per tile width:
// every tile over the whole K; whole waves over the whole K plus the last
// partial wave split along K; every tile split along K (the same formula with
// no whole wave).  Split slices pay for writing and re-reading FP32 partials.
struct TcPlan {
    int bn = 256, grid = 1, full = 0, splits = 1, kb_per = 0;
    bool pair = false;  // SM-pair kernel (cta_group::2), 256-row tiles
};

// SM pairs for normal-mode plans: chosen by cost; MRT_GEMM_PAIR=0 never
// uses them, MRT_GEMM_PAIR=1 always when the shape allows, over the whole K
// (read per plan).
static int pair_mode() {
    const char* v = std::getenv("MRT_GEMM_PAIR");
    if (v == nullptr) return -1;
    return std::strcmp(v, "0") == 0 ? 0 : (std::strcmp(v, "1") == 0 ? 1 : -1);
}

// MRT_GEMM_PAIR_SPLITS=s (2..16, read per plan): SM-pair plans cut the last
// partial wave's tiles into s K-slices whatever the cost (for tests).
static int pair_splits_forced() {
    const char* v = std::getenv("MRT_GEMM_PAIR_SPLITS");
    if (v == nullptr) return 0;
    const int n = std::atoi(v);
    return n >= 2 && n <= 16 ? n : 0;
}

static double unit_us(int bn, int64_t kb, int64_t active, int sms, int64_t x_rows) {
    const double compute = (bn / 128.0) * (static_cast<double>(kb) + 2.0) * 0.22;
    // One SM streams at most ~50 GB/s (its ring of TMA loads in flight over
    // the memory latency); together they share ~6.5 TB/s of HBM.
    const double hbm_share = std::min(50e9, 6.5e12 / static_cast<double>(std::max<int64_t>(1, std::min<int64_t>(active, sms))));
    const double w_bytes = static_cast<double>(bn) * 128.0 * kb;
    const double x_bytes = static_cast<double>(x_rows) * 128.0 * kb;
    const double mem = (w_bytes / hbm_share + x_bytes / (2.0 * hbm_share)) * 1e6;
    return std::max(compute, mem);
}

// K-slices of swap-mode tiles are summed inside thread-block clusters for more
// than 8 tokens (measured on the 7B decode step: at 9-16 tokens the cluster
// finish is 1-6 % faster per step, at 8 and fewer 5 % slower than the
// global-memory finish, which reads so little there that one pass suffices).
static bool cluster_tokens(int64_t M) { return M > 8; }

// Plan for few tokens (M <= 64), swap mode: the weight is the 128-row MMA
// operand, so a tile is 128 weight rows x all tokens and the work is streaming
// W.  Swap-mode CTAs use ~108 KB of shared memory, so two fit on an SM and
// plans may launch up to 2 x SMs CTAs.  Candidates: every tile over the whole
// K (one or two CTAs per SM) and, when whole tiles cannot fill two CTAs per
// SM, every tile split along K (K-slices summed through global memory, or
// inside thread-block clusters for 32/64-token tiles).  (Whole waves with a
// split last wave, the normal mode's third shape, never won here: with two
// CTAs per SM the last wave is already short.)  Their times come from a
// linear model of the busiest CTA's streamed bytes, the call's total bytes,
// the transposed epilogue stores, the units per CTA and the K-split finish,
// least-squares fitted to graph-replayed chains of calls on B200 (the
// Qwen2.5-7B projections, the 4864x896 GEMV and the 151936x896 lm_head at 1..64
// tokens over every split count and grid; the pick is within ~2.5 % of the
// fastest measured plan on average).  Units never exceed kSegMinKb k-blocks,
// so the tensor cores' accumulation stays as accurate as the reference's loop.
static TcPlan plan_swap(int64_t M, int64_t N, int64_t K, int sms) {
    const int bn = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    const int64_t tiles = (N + 127) / 128;
    const int64_t num_kb = (K + 63) / 64;
    const bool long_k = num_kb > kSegMinKb;
    const double tokp = static_cast<double>((std::min<int64_t>(M, bn) + 3) / 4 * 4);  // tokens, whole float4 groups
    const double kb_bytes = 128.0 * 64.0 * 2.0 + 0.5 * bn * 64.0 * 2.0;  // W tile + half the X tile per k-block
    const double total = static_cast<double>(tiles) * num_kb * kb_bytes;
    const int64_t max_grid = 2LL * sms;
    auto ceil_div = [](int64_t a, int64_t b) { return (a + b - 1) / b; };
    // Predicted us: `cta_kb` k-blocks streamed by the busiest CTA, `upc` units
    // it runs, `st_tiles` whole-K tiles whose outputs it stores itself, and
    // the finish of `split_tiles` tiles cut into `splits` slices.
    auto cost = [&](int64_t grid, int64_t cta_kb, int64_t upc, int64_t st_tiles, int64_t split_tiles, int64_t splits,
                    bool cluster) {
        double t = 3.388 + 8.595 * tokp * st_tiles / 64.0 + 12.935 * cta_kb * kb_bytes / 1e6 + 68.437 * total / 1e9 +
                   0.421 * upc;
        if (split_tiles > 0 && !cluster)
            t += 0.287 + 2.013 * tokp * splits / 64.0 + 0.472 * split_tiles * splits * tokp * 512.0 / 1e6;
        if (split_tiles > 0 && cluster)
            t += 1.933 + 0.378 * splits * tokp / 64.0 +
                 1.04 * static_cast<double>(std::max<int64_t>(0, grid - sms)) / sms * splits;
        return t;
    };
    TcPlan best{bn, 1, static_cast<int>(tiles), 1, 0};
    double best_cost = 1e300;
    auto consider = [&](double c, const TcPlan& p) {
        if (c < best_cost - 1e-9) {
            best_cost = c;
            best = p;
        }
    };
    if (!long_k) {
        // every tile over the whole K, one or two CTAs per SM
        for (int64_t cap : {static_cast<int64_t>(sms), max_grid}) {
            const int64_t grid = std::min(tiles, cap);
            const int64_t upc = ceil_div(tiles, grid);
            consider(cost(grid, upc * num_kb, upc, upc, 0, 1, false),
                     TcPlan{bn, static_cast<int>(grid), static_cast<int>(tiles), 1, 0});
        }
    }
    // every tile split along K, when whole tiles cannot fill two CTAs per SM
    if (long_k || tiles < max_grid) {
        for (int64_t s = 2; s <= 32 && s <= num_kb; ++s) {
            const int64_t kb_per = ceil_div(num_kb, s);
            const int64_t splits = ceil_div(num_kb, kb_per);
            if (splits < 2 || kb_per > kSegMinKb) continue;
            const int64_t units = tiles * splits;
            for (int64_t cap : {static_cast<int64_t>(sms), max_grid}) {
                const int64_t grid = std::min(units, cap);
                const int64_t upc = ceil_div(units, grid);
                const bool cluster = cluster_tokens(M) && splits <= 8 && grid == units;
                consider(cost(grid, upc * kb_per, upc, 0, tiles, splits, cluster),
                         TcPlan{bn, static_cast<int>(grid), 0, static_cast<int>(splits), static_cast<int>(kb_per)});
            }
        }
    }
    if (best_cost > 1e299) {
        // K beyond 32 x kSegMinKb k-blocks: the most slices the finish sums
        const int64_t kb_per = std::max<int64_t>(1, ceil_div(num_kb, 32));
        const int64_t splits = ceil_div(num_kb, kb_per);
        best = TcPlan{bn, static_cast<int>(std::min(tiles * splits, max_grid)), 0, static_cast<int>(splits),
                      static_cast<int>(kb_per)};
    }
    return best;
}

static TcPlan plan_tc(int64_t M, int64_t N, int64_t K, int sms, bool tiled = true) {
    const int64_t num_m = (M + 127) / 128;
    const int64_t num_kb = (K + 63) / 64;
    const int64_t x_rows = std::min<int64_t>(M, 128);
    TcPlan best;
    double best_cost = 1e300;
    const int pm = pair_mode();
    if (tiled && pm != 0 && M >= 256 && sms >= 2) {
        // SM pairs (tcgen05 cta_group::2): 256 x 256 tiles on sms / 2 pairs.
        // Each CTA computes a 128 x 256 tile per k-block as in the one-SM
        // kernel but loads a third less; measured 6-9 % faster per tile at
        // M >= 512 (7B gate+up, q|k|v), so its units cost 0.92 of the one-SM
        // kernel's.
        const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
        const int64_t all_pairs = sms / 2;
        const int64_t pairs = std::min<int64_t>(tiles, all_pairs);
        best = TcPlan{256, static_cast<int>(2 * pairs), static_cast<int>(tiles), 1, 0, true};
        if (pm == 1) return best;
        // Tiles [0, full) over the whole K, the other tiles cut into s
        // K-slices; returns the busiest pair's k-blocks in slices, each slice
        // counted with `unit_kb` extra k-blocks (its partial tile's store,
        // pipeline refill and share of the reduction).
        auto split_plan = [&](int64_t full, int64_t s, double unit_kb, TcPlan* out) -> double {
            const int64_t kb_per = (num_kb + s - 1) / s;
            const int64_t splits = (num_kb + kb_per - 1) / kb_per;
            if (splits < 2) return 1e300;
            const int64_t units = (tiles - full) * splits;
            *out = TcPlan{256, static_cast<int>(2 * std::min(full + units, all_pairs)), static_cast<int>(full),
                          static_cast<int>(splits), static_cast<int>(kb_per), true};
            return static_cast<double>((units + all_pairs - 1) / all_pairs) * (static_cast<double>(kb_per) + unit_kb);
        };
        const int64_t full = (tiles / all_pairs) * all_pairs;
        if (const int forced = pair_splits_forced()) {
            TcPlan p;
            if (tiles > full && forced <= num_kb && split_plan(full, forced, 0.0, &p) < 1e299) best = p;
            return best;
        }
        // K-split slices pay off only for long K (measured on the 7B down
        // projection, K = 18944, against whole-K pairs: M = 2048 (1.5 waves)
        // 3 % faster with the last half wave in 5 slices, M = 4096 9 % with
        // its two leftover tiles in 16, M = 256 / 512 (14 / 28 tiles) 2.4x /
        // 1.8x with every tile in 5, 7-8 % faster than the one-SM kernel
        // there; at K = 3584 (7B o, M = 2048) slices were 25 % slower).
        // Below a full wave the slices keep every pair busy, at more
        // than half a wave whole tiles do (M = 1024: 56 tiles).  The per-slice
        // overhead (12 k-blocks) is fitted to those measurements.
        if (num_kb >= 256 && (tiles >= all_pairs || 2 * tiles <= all_pairs)) {
            const int64_t f = tiles >= all_pairs ? full : 0;
            const double unit_kb = 12.0;
            // the whole-K alternative: its last partial wave runs num_kb
            double best_kb = tiles > f ? static_cast<double>(num_kb) : 1e300;
            for (int64_t s = 2; tiles > f && s <= 16 && s <= num_kb; ++s) {
                TcPlan p;
                const double kb = split_plan(f, s, unit_kb, &p);
                if (kb < best_kb - 1e-9) {
                    best_kb = kb;
                    best = p;
                }
            }
            return best;
        }
        // With at least half a wave of pair tiles, and a last wave at least
        // half full (or four waves and more), the pairs win outright
        // (measured at 1.5 waves against the one-SM kernel's K-split tails,
        // e.g. 7B o and down at M = 2048; at 0.57 waves, M = 768 o, 7 %
        // faster); otherwise they compete on cost (a 1.03-wave gate|up of
        // the 0.5B layer at M = 512 ran 25.6 us on pairs, 20.9 us on one-SM
        // 128-column tiles).
        const int64_t rem = tiles % all_pairs;
        const bool fills = rem == 0 || 2 * rem >= all_pairs || tiles >= 4 * all_pairs;
        if ((2 * tiles >= all_pairs && fills) || num_kb >= 256) return best;
        const int64_t waves = (tiles + pairs - 1) / pairs;
        best_cost = 0.92 * static_cast<double>(waves) * unit_us(256, num_kb, 2 * pairs, sms, x_rows);
    }
    for (int bn : {256, 128, 64}) {
        // One 128-row m-tile (decode batches of 65..128 tokens): 256-column
        // tiles measured slower than 128-column ones on every 7B projection
        // and the 0.5B lm_head at M = 128 (gate+up 53.2 vs 50.5 us, lm_head
        // 63.6 vs 57.4, down 35.6 vs 34.8), so they are not considered.
        if (num_m == 1 && bn == 256) continue;
        const int64_t tiles = num_m * ((N + bn - 1) / bn);
        // every tile over the whole K
        {
            const int64_t waves = (tiles + sms - 1) / sms;
            const double cost = waves * unit_us(bn, num_kb, tiles, sms, x_rows);
            if (cost < best_cost - 1e-9) {
                best_cost = cost;
                best = TcPlan{bn, static_cast<int>(std::min<int64_t>(tiles, sms)), static_cast<int>(tiles), 1, 0};
            }
        }
        // whole waves over K, tail tiles split (no whole wave = every tile split)
        const int64_t full = (tiles / sms) * sms;
        const int64_t n_tail = tiles - full;
        if (n_tail == 0) continue;
        for (int64_t s = 2; s <= 16 && s <= num_kb; ++s) {
            const int64_t kb_per = (num_kb + s - 1) / s;
            const int64_t splits = (num_kb + kb_per - 1) / kb_per;  // no empty slice
            if (splits < 2) continue;
            const int64_t tail_units = n_tail * splits;
            double cost = static_cast<double>(full / sms) * unit_us(bn, num_kb, sms, sms, x_rows);
            cost += static_cast<double>((tail_units + sms - 1) / sms) * unit_us(bn, kb_per, tail_units, sms, x_rows);
            const double partial_bytes = static_cast<double>(n_tail) * 128.0 * bn * 4.0 * (splits + 1.0);
            cost += partial_bytes / 6.0e12 * 1e6 + 3.0;
            if (cost < best_cost - 1e-9) {
                best_cost = cost;
                const int64_t units = full + tail_units;
                best = TcPlan{bn, static_cast<int>(std::min<int64_t>(units, sms)), static_cast<int>(full),
                              static_cast<int>(splits), static_cast<int>(kb_per)};
            }
        }
    }
    return best;
}

// Swap-mode plans of more than 8 tokens whose every tile is split into 2..8
// K-slices, one slice per CTA (the grid is the slices, up to two CTAs per
// SM), sum the slices inside thread-block clusters (distributed shared
// memory) instead of through global memory, where the finish re-reads the
// tokens' FP32 columns of every slice; with 8 tokens or fewer that read is one
// short pass and the global finish is the faster one (cluster_tokens).
// MRT_GEMM_CLUSTER=0 (read once) keeps the global-memory finish everywhere.
// The SIMT GEMV (gemv.cu) on a tiled weight: by default for one token and
// weights of at most kGemvMaxBytes.  Measured on B200 in graph-chained calls
// with the weights cold in L2: 4864x896 (8.7 MB) 4.17 us against 5.44 for the
// swap-mode tcgen05 kernel, the Qwen2.5-0.5B projections 17.0 against 22.9 us
// per layer, the 7B projections sharded eight ways 25.0 against 26.9 us; but
// the weights of 30 MB and more stream faster through the tcgen05 ring (7B
// gate+up 41.6 against 51.8 us), and from two tokens on the activation loads
// per weight load cost more than the tensor cores' set-up.  MRT_GEMV=1 takes
// it for every call of 1..4 tokens it can run, MRT_GEMV=0 never (read per
// call).
constexpr double kGemvMaxBytes = 20e6;

static bool use_gemv(int64_t M, int64_t N, int64_t K) {
    if (M < 1 || M > 4) return false;
    const char* v = std::getenv("MRT_GEMV");
    if (v != nullptr && std::strcmp(v, "1") == 0) return true;
    if (v != nullptr && std::strcmp(v, "0") == 0) return false;
    return M == 1 && 2.0 * static_cast<double>(N) * static_cast<double>(K) <= kGemvMaxBytes;
}

// Row quads per GEMV CTA: the most (whole K per warp) that still gives at
// least two CTAs per SM, else one quad whose eight warps split K.
// MRT_GEMV_RQ=1|2|4|8 forces it (read per call).
static int gemv_row_quads(int64_t N, int sms) {
    if (const char* v = std::getenv("MRT_GEMV_RQ")) {
        const int f = std::atoi(v);
        if (f == 1 || f == 2 || f == 4 || f == 8) return f;
    }
    const int64_t quads = (N + 3) / 4;
    int rq = 8;
    while (rq > 1 && (quads + rq - 1) / rq < 2LL * sms) rq /= 2;
    return rq;
}

static bool use_cluster(bool swap, const TcPlan& p, int64_t tiles, int64_t M) {
    static const bool enabled = [] {
        const char* v = std::getenv("MRT_GEMM_CLUSTER");
        return v == nullptr || std::strcmp(v, "0") != 0;
    }();
    return enabled && swap && cluster_tokens(M) && p.full == 0 && p.splits >= 2 && p.splits <= 8 &&
           static_cast<int64_t>(p.grid) == tiles * p.splits && tc_cluster_ok(p.bn, p.splits);
}

// The weight's TMA map whose box is exactly the kernel's W tile (bn rows).
static const CUtensorMap* weight_tmap(mrt_weight w, int bn) {
    const int slot = bn == 64 ? 0 : (bn == 128 ? 1 : (bn == 256 ? 2 : -1));
    if (slot < 0) {
        set_error(MRT_ERR_INVALID_ARG, "no tensor map for tile width " + std::to_string(bn));
        return nullptr;
    }
    if (!w->tmap_ok[slot]) {
        if (make_tmap_f16(&w->tmap[slot], w->data, w->n, w->k, w->k, bn) != MRT_OK) return nullptr;
        w->tmap_ok[slot] = true;
    }
    return &w->tmap[slot];
}

// Optional epilogue extras of one GEMM call.
struct GemmEpi {
    const uint16_t* residual = nullptr;  // y = fp16(residual + fp16(acc)), row stride ldr
    int64_t ldr = 0;
    float* am_val = nullptr;             // greedy-pick partials (swap mode; see TcGemmArgs)
    int64_t* am_idx = nullptr;
};

// Shared body of mrt_gemm / mrt_gemm_f32 / mrt_gemm_residual and the fused
// lm_head.  With greedy-pick partials requested, launches nothing and sets
// *fused = false when the call cannot produce them (the caller falls back).
static int gemm_dispatch(mrt_weight w, const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M,
                         bool out_f32, bool use_bias, cudaStream_t s, const uint16_t* swiglu_lut = nullptr,
                         bool* fused = nullptr, const GemmEpi& epi = GemmEpi{}) {
    if (fused) *fused = false;
    if (w == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL weight");
    if (M < 0) return set_error(MRT_ERR_SHAPE, "M must be >= 0");
    if (M == 0) return MRT_OK;
    if (x == nullptr || (y == nullptr && epi.am_val == nullptr)) return set_error(MRT_ERR_INVALID_ARG, "NULL x or y");
    if (ldx < w->k || (y != nullptr && ldy < (swiglu_lut ? w->n / 2 : w->n)))
        return set_error(MRT_ERR_SHAPE, "ldx must be >= K and ldy >= N");
    if (epi.residual != nullptr && (out_f32 || swiglu_lut != nullptr || epi.ldr < w->n))
        return set_error(MRT_ERR_SHAPE, "the residual epilogue needs an FP16 output and ldr >= N");
    if (use_bias && w->bias == nullptr) return set_error(MRT_ERR_INVALID_ARG, "MRT_GEMM_BIAS without an attached bias");
    if (M > (1LL << 31) - 1 || w->n > (1LL << 31) - 1 || w->k > (1LL << 31) - 1)
        return set_error(MRT_ERR_SHAPE, "dimensions must fit in 31 bits");
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    if (c->device != w->device) return set_error(MRT_ERR_INVALID_ARG, "weight lives on another device");
    const uint16_t* bias = use_bias ? w->bias : nullptr;

    const bool fast = (w->k % 8 == 0) && (ldx % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    cudaError_t e;
    if (swiglu_lut != nullptr && (!fast || (w->n & 1) != 0)) return MRT_OK;  // not fused: the caller falls back
    if (epi.am_val != nullptr && (!fast || M > 64 || out_f32 || swiglu_lut != nullptr)) return MRT_OK;  // not fused
    if (!fast) {
        GeneralGemmArgs g{};
        g.a = x; g.a_dtype = MRT_FP16; g.a_cols0 = ldx;
        g.b = w->data; g.b_dtype = MRT_FP16; g.b_cols0 = w->k;
        g.c = y; g.c_dtype = out_f32 ? MRT_FP32 : MRT_FP16; g.ldc = ldy;
        g.M = M; g.N = w->n; g.K = w->k; g.alpha = 1.0f; g.beta = 0.0f;
        g.trans_a = 0; g.trans_b = 1; g.bias = bias;
        g.b_k_tiles = w->tiled ? w->k_tiles : 0;
        g.residual = epi.residual; g.ldr = epi.ldr;
        e = launch_general_gemm(g, s);
        return e == cudaSuccess ? MRT_OK : cuda_error(e, "general gemm launch");
    }
    if (w->tiled && epi.am_val == nullptr && use_gemv(M, w->n, w->k) &&
        (swiglu_lut == nullptr || ((w->n & 1) == 0 && !out_f32 && bias == nullptr))) {
        GemvArgs g{};
        g.w = w->data; g.k_tiles = w->k_tiles;
        g.x = static_cast<const uint16_t*>(x); g.ldx = ldx;
        g.y = y; g.ldy = ldy; g.out_f32 = out_f32 ? 1 : 0; g.bias = bias;
        g.residual = epi.residual; g.ldr = epi.ldr;
        g.M = static_cast<int>(M); g.N = static_cast<int>(w->n); g.K = static_cast<int>(w->k);
        g.swiglu_lut = swiglu_lut;
        g.rq = gemv_row_quads(w->n, c->sms);
        e = launch_gemv_tiled(g, s);
        if (e != cudaSuccess) return cuda_error(e, "gemv launch");
        if (fused) *fused = swiglu_lut != nullptr;
        return MRT_OK;
    }
    const bool swap = M <= 64;
    const TcPlan p = swap ? plan_swap(M, w->n, w->k, c->sms) : plan_tc(M, w->n, w->k, c->sms, w->tiled);
    if (p.pair && epi.am_val == nullptr) {
        CUtensorMap tx;
        int rc = make_tmap_f16(&tx, x, M, w->k, ldx, 128);
        if (rc != MRT_OK) return rc;
        if (!w->tmap_rows_ok) {
            rc = make_tmap_f16_rows64(&w->tmap_rows, w->data, w->n_pad * w->k_tiles, 128);
            if (rc != MRT_OK) return rc;
            w->tmap_rows_ok = true;
        }
        TcGemmArgs a{};
        a.M = static_cast<int>(M); a.N = static_cast<int>(w->n); a.K = static_cast<int>(w->k);
        a.pair = 1;
        a.w_tiled = w->data; a.w_k_tiles = w->k_tiles; a.w_prefetch = 1;
        a.bn = p.bn; a.grid = p.grid; a.full_tiles = p.full; a.tail_splits = p.splits; a.kb_per = p.kb_per;
        a.y = y; a.ldy = ldy; a.out_f32 = out_f32 ? 1 : 0; a.bias = bias; a.err_flag = c->d_err;
        a.residual = epi.residual; a.ldr = epi.ldr;
        a.seg_kb = kSegKb;
        const int64_t n_tail = tc_gemm_tiles(a) - p.full;
        if (swiglu_lut != nullptr && n_tail > 0) return MRT_OK;  // K-split plan: not fused
        a.swiglu_lut = swiglu_lut;
        if (n_tail > 0) {
            const size_t need = static_cast<size_t>(n_tail) * p.splits * 256 * p.bn * sizeof(float);
            rc = ensure_buffer(&c->ws, &c->ws_bytes, need, "allocating split-K scratch");
            if (rc != MRT_OK) return rc;
            a.partials = static_cast<float*>(c->ws);
        }
        e = launch_tc_pair(a, tx, w->tmap_rows, s);
        if (e != cudaSuccess) return cuda_error(e, "tcgen05 pair gemm launch");
        if (n_tail > 0) {
            e = launch_reduce_tail(a, s);
            if (e != cudaSuccess) return cuda_error(e, "split-K reduction launch");
        }
        if (fused) *fused = swiglu_lut != nullptr;
        return MRT_OK;
    }
    if (swiglu_lut != nullptr) {
        const int64_t tiles = swap ? (w->n + 127) / 128 : ((M + 127) / 128) * ((w->n + p.bn - 1) / p.bn);
        if (p.full != tiles) return MRT_OK;  // K-split plan: not fused
    }
    // X's box is 128 rows in normal mode and bn rows in swap mode; a row-major
    // W needs a tensor map with the other box, a tiled W is copied linearly.
    CUtensorMap tx;
    int rc = make_tmap_f16(&tx, x, M, w->k, ldx, swap ? p.bn : 128);
    if (rc != MRT_OK) return rc;
    const CUtensorMap* tw = &tx;
    if (!w->tiled) {
        tw = weight_tmap(w, swap ? 128 : p.bn);
        if (tw == nullptr) return MRT_ERR_CUDA;
    }
    TcGemmArgs a{};
    a.M = static_cast<int>(M); a.N = static_cast<int>(w->n); a.K = static_cast<int>(w->k);
    a.swap = swap ? 1 : 0;
    a.w_tiled = w->tiled ? w->data : nullptr;
    a.w_k_tiles = w->k_tiles;
    a.w_prefetch = w->tiled ? 1 : 0;  // uploads finish before returning; views are never tiled
    a.bn = p.bn; a.grid = p.grid; a.full_tiles = p.full; a.tail_splits = p.splits; a.kb_per = p.kb_per;
    a.y = y; a.ldy = ldy; a.out_f32 = out_f32 ? 1 : 0; a.bias = bias; a.err_flag = c->d_err;
    a.swiglu_lut = swiglu_lut;
    a.residual = epi.residual; a.ldr = epi.ldr;
    a.am_val = epi.am_val; a.am_idx = epi.am_idx;
    a.am_chunks = static_cast<int>(4 * ((w->n + 127) / 128));
    a.seg_kb = kSegKb;
    const int64_t tiles = tc_gemm_tiles(a);
    const int64_t n_tail = tiles - p.full;
    if (use_cluster(swap, p, tiles, M) && epi.am_val == nullptr) a.cluster_k = p.splits;
    if (n_tail > 0 && a.cluster_k == 0) {
        const size_t need = static_cast<size_t>(n_tail) * p.splits * 128 * p.bn * sizeof(float);
        rc = ensure_buffer(&c->ws, &c->ws_bytes, need, "allocating split-K scratch");
        if (rc != MRT_OK) return rc;
        a.partials = static_cast<float*>(c->ws);
        const size_t counters = static_cast<size_t>(n_tail) * 4 * sizeof(int);
        if (swap && c->counters_bytes < counters) {
            void* p_cnt = c->counters;
            rc = ensure_buffer(&p_cnt, &c->counters_bytes, counters, "allocating split-K counters");
            if (rc != MRT_OK) return rc;
            c->counters = static_cast<int*>(p_cnt);
            e = cudaMemset(c->counters, 0, c->counters_bytes);  // kernels keep them zero afterwards
            if (e != cudaSuccess) return cuda_error(e, "clearing split-K counters");
        }
        a.tile_counters = swap ? c->counters : nullptr;
    }
    e = launch_tc_gemm(a, tx, *tw, s);
    if (e != cudaSuccess) return cuda_error(e, "tcgen05 gemm launch");
    if (fused) *fused = swiglu_lut != nullptr || epi.am_val != nullptr;
    if (n_tail > 0 && !swap) {
        e = launch_reduce_tail(a, s);
        if (e != cudaSuccess) return cuda_error(e, "split-K reduction launch");
    }
    return MRT_OK;
}

int gemm_swiglu(mrt_weight w, const void* x, int64_t ldx, void* act, int64_t ld_act, int64_t M,
                const uint16_t* lut, cudaStream_t s, bool* fused) {
    if (lut == nullptr || fused == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL SiLU table or flag");
    return gemm_dispatch(w, x, ldx, act, ld_act, M, false, false, s, lut, fused);
}

}  // namespace mrt

extern "C" int mrt_gemm_plan(int64_t M, int64_t N, int64_t K, int sms, int* kernel, int* bn, int* full_tiles,
                             int* tail_splits, int* kb_per, int* grid) {
    clear_error();
    if (M <= 0 || N <= 0 || K <= 0) return set_error(MRT_ERR_SHAPE, "M, N and K must be positive");
    if (sms <= 0) {
        DevCtx* c = current_ctx();
        if (!c) return MRT_ERR_CUDA;
        sms = c->sms;
    }
    if (use_gemv(M, N, K)) {
        const int rq = gemv_row_quads(N, sms);
        if (kernel) *kernel = 5;
        if (bn) *bn = 0;
        if (full_tiles) *full_tiles = 0;
        if (tail_splits) *tail_splits = 1;
        if (kb_per) *kb_per = static_cast<int>((K + 63) / 64);
        if (grid) *grid = static_cast<int>(((N + 3) / 4 + rq - 1) / rq);
        return MRT_OK;
    }
    const bool swap = M <= 64;
    const TcPlan p = swap ? plan_swap(M, N, K, sms) : plan_tc(M, N, K, sms);
    const int64_t tiles = swap ? ((N + 127) / 128) : 0;
    if (kernel) *kernel = swap ? (use_cluster(true, p, tiles, M) ? 3 : 2) : (p.pair ? 4 : 1);
    if (bn) *bn = p.bn;
    if (full_tiles) *full_tiles = p.full;
    if (tail_splits) *tail_splits = p.splits;
    if (kb_per) *kb_per = p.kb_per;
    if (grid) *grid = p.grid;
    return MRT_OK;
}

extern "C" int mrt_gemm(mrt_weight w, const void* x_dev, int64_t ldx, void* y_dev, int64_t ldy, int64_t M,
                        unsigned flags, void* stream) {
    clear_error();
    return gemm_dispatch(w, x_dev, ldx, y_dev, ldy, M, false, (flags & MRT_GEMM_BIAS) != 0,
                         static_cast<cudaStream_t>(stream));
}

extern "C" int mrt_gemm_swiglu(mrt_weight w, const void* x_dev, int64_t ldx, void* act_dev, int64_t ld_act,
                               int64_t M, void* stream) {
    clear_error();
    if (w == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL weight");
    if (w->n % 2 != 0) return set_error(MRT_ERR_SHAPE, "an interleaved gate|up weight has an even row count");
    if (M < 0) return set_error(MRT_ERR_SHAPE, "M must be >= 0");
    if (M == 0) return MRT_OK;
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    const uint16_t* lut = silu_lut_for_device(c->device);
    if (lut == nullptr) return set_error(MRT_ERR_CUDA, "building the SiLU table failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    bool fused = false;
    int rc = gemm_swiglu(w, x_dev, ldx, act_dev, ld_act, M, lut, s, &fused);
    if (rc != MRT_OK || fused) return rc;
    // The plan splits K: the interleaved product into scratch, then the pairs.
    const size_t bytes = static_cast<size_t>(M) * static_cast<size_t>(w->n) * 2;
    if ((rc = ensure_buffer(&c->gu, &c->gu_bytes, bytes, "allocating gate|up scratch")) != MRT_OK) return rc;
    if ((rc = gemm_dispatch(w, x_dev, ldx, c->gu, w->n, M, false, false, s)) != MRT_OK) return rc;
    const cudaError_t e = launch_swiglu_pairs(static_cast<const uint16_t*>(c->gu), w->n, w->n / 2, M, lut,
                                              static_cast<uint16_t*>(act_dev), ld_act, s);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "swiglu launch");
}

extern "C" int mrt_gemm_f32(mrt_weight w, const void* x_dev, int64_t ldx, float* y_dev, int64_t ldy,
                            int64_t M, void* stream) {
    clear_error();
    return gemm_dispatch(w, x_dev, ldx, y_dev, ldy, M, true, false, static_cast<cudaStream_t>(stream));
}

namespace mrt {

// True when the host pointer is page-locked (cudaHostAlloc / cudaHostRegister),
// so DMA can read or write it directly and copies can overlap.
static bool host_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

static int io_pipeline_init(DevCtx* c) {
    if (c->io_in != nullptr) return MRT_OK;
    cudaError_t e = cudaStreamCreateWithFlags(&c->io_in, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->io_out, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->io_start, cudaEventDisableTiming);
    for (int i = 0; i < DevCtx::kIoChunks && e == cudaSuccess; ++i) {
        e = cudaEventCreateWithFlags(&c->io_h2d[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->io_mm[i], cudaEventDisableTiming);
    }
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "creating the host-copy streams");
}

// Rows per chunk of the host-buffer pipeline: whole 128-row tiles, chunks of
// at least ~2 MB of copies each, at most kIoChunks chunks; 0 = one piece.
static int64_t io_chunk_rows(int64_t M, int64_t N, int64_t K) {
    if (M < 256) return 0;
    const int64_t row_bytes = 2 * (N + K);
    int64_t rows = std::max<int64_t>(128, ((2 << 20) / row_bytes + 127) / 128 * 128);
    rows = std::max(rows, (M + DevCtx::kIoChunks - 1) / DevCtx::kIoChunks);
    rows = std::max<int64_t>(rows, (M / 8 + 127) / 128 * 128);  // about 8 chunks for large M
    rows = (rows + 127) / 128 * 128;
    return rows >= M ? 0 : rows;
}

}  // namespace mrt

extern "C" int mrt_gemm_host(mrt_weight w, const void* x_host, void* y_host, int64_t M, unsigned flags,
                             void* stream) {
    clear_error();
    if (w == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL weight");
    if (M < 0) return set_error(MRT_ERR_SHAPE, "M must be >= 0");
    if (M == 0) return MRT_OK;
    if (x_host == nullptr || y_host == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL x or y");
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool bias = (flags & MRT_GEMM_BIAS) != 0;
    const size_t xb = static_cast<size_t>(M * w->k) * 2, yb = static_cast<size_t>(M * w->n) * 2;
    int rc = ensure_buffer(&c->io_x, &c->io_x_bytes, xb, "allocating input staging");
    if (rc == MRT_OK) rc = ensure_buffer(&c->io_y, &c->io_y_bytes, yb, "allocating output staging");
    if (rc != MRT_OK) return rc;
    const int64_t chunk = io_chunk_rows(M, w->n, w->k);
    cudaError_t e;
    if (chunk == 0 || !host_pinned(x_host) || !host_pinned(y_host)) {
        // One piece (small M, or pageable memory, which the driver stages
        // through its own buffers and cannot overlap): copy in, multiply,
        // copy out, wait.
        e = cudaMemcpyAsync(c->io_x, x_host, xb, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cuda_error(e, "copying x to the device");
        rc = gemm_dispatch(w, c->io_x, w->k, c->io_y, w->n, M, false, bias, s);
        if (rc != MRT_OK) return rc;
        e = cudaMemcpyAsync(y_host, c->io_y, yb, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return cuda_error(e, "copying y to the host");
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_error(e, "waiting for the host-buffer gemm");
        return MRT_OK;
    }
    // Pinned buffers: rows in chunks through three streams, so chunk i+1's
    // host-to-device copy, chunk i's product and chunk i-1's device-to-host
    // copy run at the same time (PCIe carries both directions at once).  Each
    // chunk is its own GEMM over its rows, so its plan -- and with it the
    // order of a K-split sum -- may differ from a one-piece call's: results
    // meet the same error bars, and a given M and buffer kind always takes
    // the same chunks, so repeated calls give identical bits.
    if ((rc = io_pipeline_init(c)) != MRT_OK) return rc;
    const int64_t n_chunks = (M + chunk - 1) / chunk;
    // The staging buffers may still be read or written by work the caller
    // queued on s earlier: the side streams start after it.
    if ((e = cudaEventRecord(c->io_start, s)) != cudaSuccess) return cuda_error(e, "recording the start");
    if ((e = cudaStreamWaitEvent(c->io_in, c->io_start, 0)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(c->io_out, c->io_start, 0)) != cudaSuccess)
        return cuda_error(e, "ordering the copy streams");
    const char* x8 = static_cast<const char*>(x_host);
    char* y8 = static_cast<char*>(y_host);
    uint16_t* dx = static_cast<uint16_t*>(c->io_x);
    uint16_t* dy = static_cast<uint16_t*>(c->io_y);
    for (int64_t i = 0; i < n_chunks; ++i) {
        const int slot = static_cast<int>(i % DevCtx::kIoChunks);
        const int64_t r0 = i * chunk, rows = std::min(chunk, M - r0);
        const size_t xo = static_cast<size_t>(r0 * w->k), yo = static_cast<size_t>(r0 * w->n);
        e = cudaMemcpyAsync(dx + xo, x8 + xo * 2, static_cast<size_t>(rows * w->k) * 2, cudaMemcpyHostToDevice,
                            c->io_in);
        if (e == cudaSuccess) e = cudaEventRecord(c->io_h2d[slot], c->io_in);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, c->io_h2d[slot], 0);
        if (e != cudaSuccess) return cuda_error(e, "queueing a chunk's copy to the device");
        rc = gemm_dispatch(w, dx + xo, w->k, dy + yo, w->n, rows, false, bias, s);
        if (rc != MRT_OK) return rc;
        e = cudaEventRecord(c->io_mm[slot], s);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->io_out, c->io_mm[slot], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(y8 + yo * 2, dy + yo, static_cast<size_t>(rows * w->n) * 2, cudaMemcpyDeviceToHost,
                                c->io_out);
        if (e != cudaSuccess) return cuda_error(e, "queueing a chunk's copy to the host");
    }
    e = cudaStreamSynchronize(c->io_out);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_error(e, "waiting for the host-buffer gemm");
    return MRT_OK;
}

extern "C" int mrt_gemm_host_async(mrt_weight w, const void* x_host, void* y_host, int64_t M, unsigned flags,
                                   void* stream) {
    clear_error();
    if (w == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL weight");
    if (M < 0) return set_error(MRT_ERR_SHAPE, "M must be >= 0");
    if (M == 0) return MRT_OK;
    if (x_host == nullptr || y_host == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL x or y");
    if (!host_pinned(x_host) || !host_pinned(y_host))
        return set_error(MRT_ERR_INVALID_ARG, "mrt_gemm_host_async needs page-locked (pinned) host buffers");
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    int rc = io_pipeline_init(c);
    if (rc != MRT_OK) return rc;
    cudaError_t e = cudaSuccess;
    for (int k = 0; k < DevCtx::kAsyncSets && e == cudaSuccess; ++k)
        if (c->a_free[k] == nullptr) e = cudaEventCreateWithFlags(&c->a_free[k], cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_error(e, "creating the staging events");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool bias = (flags & MRT_GEMM_BIAS) != 0;
    const int set = c->a_next;
    c->a_next = (set + 1) % DevCtx::kAsyncSets;
    const size_t xb = static_cast<size_t>(M * w->k) * 2, yb = static_cast<size_t>(M * w->n) * 2;
    if (c->ax_bytes[set] < xb || c->ay_bytes[set] < yb) {
        // Growing a set waits for its last user (ensure_buffer synchronises).
        rc = ensure_buffer(&c->ax[set], &c->ax_bytes[set], xb, "allocating input staging");
        if (rc == MRT_OK) rc = ensure_buffer(&c->ay[set], &c->ay_bytes[set], yb, "allocating output staging");
        if (rc != MRT_OK) return rc;
    }
    // This set's previous call is done with it (its last copy to the host);
    // the other sets' calls may still be copying in either direction.
    if ((e = cudaStreamWaitEvent(c->io_in, c->a_free[set], 0)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(s, c->a_free[set], 0)) != cudaSuccess)
        return cuda_error(e, "ordering the staging set");
    int64_t chunk = io_chunk_rows(M, w->n, w->k);
    if (chunk == 0) chunk = M;
    const int64_t n_chunks = (M + chunk - 1) / chunk;
    const char* x8 = static_cast<const char*>(x_host);
    char* y8 = static_cast<char*>(y_host);
    uint16_t* dx = static_cast<uint16_t*>(c->ax[set]);
    uint16_t* dy = static_cast<uint16_t*>(c->ay[set]);
    for (int64_t i = 0; i < n_chunks; ++i) {
        const int slot = static_cast<int>(i % DevCtx::kIoChunks);
        const int64_t r0 = i * chunk, rows = std::min(chunk, M - r0);
        const size_t xo = static_cast<size_t>(r0 * w->k), yo = static_cast<size_t>(r0 * w->n);
        e = cudaMemcpyAsync(dx + xo, x8 + xo * 2, static_cast<size_t>(rows * w->k) * 2, cudaMemcpyHostToDevice,
                            c->io_in);
        if (e == cudaSuccess) e = cudaEventRecord(c->io_h2d[slot], c->io_in);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, c->io_h2d[slot], 0);
        if (e != cudaSuccess) return cuda_error(e, "queueing a chunk's copy to the device");
        rc = gemm_dispatch(w, dx + xo, w->k, dy + yo, w->n, rows, false, bias, s);
        if (rc != MRT_OK) return rc;
        e = cudaEventRecord(c->io_mm[slot], s);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->io_out, c->io_mm[slot], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(y8 + yo * 2, dy + yo, static_cast<size_t>(rows * w->n) * 2, cudaMemcpyDeviceToHost,
                                c->io_out);
        if (e != cudaSuccess) return cuda_error(e, "queueing a chunk's copy to the host");
    }
    e = cudaEventRecord(c->a_free[set], c->io_out);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "recording the staging set's release");
}

extern "C" int mrt_gemm_general(const void* a_dev, int a_dtype, int64_t a_rows, int64_t a_cols,
                                const void* b_dev, int b_dtype, int64_t b_rows, int64_t b_cols, void* c_dev,
                                int c_dtype, float alpha, float beta, int trans_a, int trans_b, void* stream) {
    clear_error();
    for (int dt : {a_dtype, b_dtype, c_dtype})
        if (dt != MRT_FP16 && dt != MRT_BF16 && dt != MRT_FP32)
            return set_error(MRT_ERR_DTYPE, "dtypes must be FP16, BF16 or FP32");
    if (a_rows < 0 || a_cols < 0 || b_rows < 0 || b_cols < 0) return set_error(MRT_ERR_SHAPE, "negative dimension");
    const int64_t M = trans_a ? a_cols : a_rows;
    const int64_t K = trans_a ? a_rows : a_cols;
    const int64_t N = trans_b ? b_rows : b_cols;
    if ((trans_b ? b_cols : b_rows) != K)
        return set_error(MRT_ERR_SHAPE, "inner dimensions of A and B differ");
    if (M == 0 || N == 0) return MRT_OK;  // cpu_backend.cpp:124-126
    if (!current_ctx()) return MRT_ERR_CUDA;
    GeneralGemmArgs g{};
    g.a = a_dev; g.a_dtype = a_dtype; g.a_cols0 = a_cols;
    g.b = b_dev; g.b_dtype = b_dtype; g.b_cols0 = b_cols;
    g.c = c_dev; g.c_dtype = c_dtype; g.ldc = N;
    g.M = M; g.N = N; g.K = K; g.alpha = alpha; g.beta = beta;
    g.trans_a = trans_a ? 1 : 0; g.trans_b = trans_b ? 1 : 0; g.bias = nullptr;
    cudaError_t e = launch_general_gemm(g, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "general gemm launch");
}

// ====================================================================== logits

extern "C" int mrt_argmax_f16(const void* logits_dev, int64_t M, int64_t V, int64_t ld, int64_t index_base,
                              int64_t* idx_dev, float* val_dev, void* stream) {
    clear_error();
    if (M < 0 || V < 0 || ld < V) return set_error(MRT_ERR_SHAPE, "need M >= 0, V >= 0, ld >= V");
    if (M == 0) return MRT_OK;
    if (V == 0) return set_error(MRT_ERR_SHAPE, "argmax over an empty row");
    if (M > 65535) return set_error(MRT_ERR_SHAPE, "at most 65535 rows per call");
    if (logits_dev == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL logits");
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    int rc = ensure_buffer(&c->ws, &c->ws_bytes, argmax_scratch_bytes(M, V), "allocating argmax scratch");
    if (rc != MRT_OK) return rc;
    cudaError_t e = launch_argmax(static_cast<const uint16_t*>(logits_dev), M, V, ld, index_base, idx_dev,
                                  val_dev, c->ws, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "argmax launch");
}

extern "C" int mrt_lm_head_argmax(mrt_weight w, const void* x_dev, int64_t ldx, int64_t M, void* logits_dev,
                                  int64_t index_base, int64_t* idx_dev, float* val_dev, void* stream) {
    clear_error();
    if (w == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL weight");
    if (M < 0) return set_error(MRT_ERR_SHAPE, "M must be >= 0");
    if (M == 0) return MRT_OK;
    if (M > 65535) return set_error(MRT_ERR_SHAPE, "at most 65535 rows per call");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    // Decode (M <= 64): the GEMM's epilogue leaves the best (value, index) of
    // every 32 vocabulary rows per token, so the logits need not be written
    // (logits_dev may be NULL) nor read back; one small kernel picks the row's
    // best of those partials.
    if (M <= 64) {
        const int64_t chunks = 4 * ((w->n + 127) / 128);
        const size_t bytes = static_cast<size_t>(M * chunks) * (sizeof(float) + sizeof(int64_t));
        int rc = ensure_buffer(&c->am, &c->am_bytes, bytes, "allocating greedy-pick partials");
        if (rc != MRT_OK) return rc;
        GemmEpi epi;
        epi.am_idx = static_cast<int64_t*>(c->am);
        epi.am_val = reinterpret_cast<float*>(epi.am_idx + M * chunks);
        bool fused = false;
        rc = gemm_dispatch(w, x_dev, ldx, logits_dev, w->n, M, false, false, s, nullptr, &fused, epi);
        if (rc != MRT_OK) return rc;
        if (fused) {
            const cudaError_t e = launch_argmax_final(epi.am_val, epi.am_idx, M, chunks, index_base, idx_dev, val_dev, s);
            return e == cudaSuccess ? MRT_OK : cuda_error(e, "greedy pick launch");
        }
    }
    if (logits_dev == nullptr) {
        // the unfused path needs the logits: keep them in per-device scratch
        int rc = ensure_buffer(&c->gu, &c->gu_bytes, static_cast<size_t>(M * w->n) * 2, "allocating logits scratch");
        if (rc != MRT_OK) return rc;
        logits_dev = c->gu;
    }
    int rc = mrt_gemm(w, x_dev, ldx, logits_dev, w->n, M, 0, stream);
    if (rc != MRT_OK) return rc;
    return mrt_argmax_f16(logits_dev, M, w->n, w->n, index_base, idx_dev, val_dev, stream);
}

extern "C" int mrt_gemm_residual(mrt_weight w, const void* x_dev, int64_t ldx, const void* res_dev, int64_t ldr,
                                 void* y_dev, int64_t ldy, int64_t M, unsigned flags, void* stream) {
    clear_error();
    if (res_dev == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL residual");
    GemmEpi epi;
    epi.residual = static_cast<const uint16_t*>(res_dev);
    epi.ldr = ldr;
    return gemm_dispatch(w, x_dev, ldx, y_dev, ldy, M, false, (flags & MRT_GEMM_BIAS) != 0,
                         static_cast<cudaStream_t>(stream), nullptr, nullptr, epi);
}

extern "C" int mrt_convert(const void* src_dev, int src_dtype, void* dst_dev, int dst_dtype, int64_t n,
                           void* stream) {
    clear_error();
    for (int dt : {src_dtype, dst_dtype})
        if (dt != MRT_FP16 && dt != MRT_BF16 && dt != MRT_FP32)
            return set_error(MRT_ERR_DTYPE, "dtypes must be FP16, BF16 or FP32");
    if (n < 0) return set_error(MRT_ERR_SHAPE, "n must be >= 0");
    if (n == 0) return MRT_OK;
    if (!current_ctx()) return MRT_ERR_CUDA;
    cudaError_t e = launch_convert(src_dev, src_dtype, dst_dev, dst_dtype, n, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "convert launch");
}
