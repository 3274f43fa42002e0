// noalloc.cu -- greedy argmax with no device allocation (mrt_argmax_f16_noalloc).
//
// Runs the same two argmax kernels as mrt_argmax_f16, but their (value,
// index) partials go to a fixed array compiled into this library rather than
// to the per-device context's growable scratch.  The entry point touches no
// context (creating one allocates), calls no cudaMalloc / cudaFree and no
// library routine that allocates.  Callers that cannot allocate: hosts that
// capture their decode step into a CUDA graph, and runtimes that own all
// device memory through their own arenas.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "ctx.h"
#include "kernels.h"

namespace mrt {
namespace {

// 8192 (index, value) pairs: 8 bytes of index + 4 of value each, plus the
// 64 bytes of slack argmax_scratch_bytes() accounts for.
constexpr size_t kNoAllocPairs = 8192;
constexpr size_t kNoAllocBytes = kNoAllocPairs * (sizeof(int64_t) + sizeof(float)) + 64;

// One copy per device that loads this library, kept until the process exits.
// Host code must not take this name's address: on the host it is only a
// stand-in; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_argmax_scratch[kNoAllocBytes];

std::mutex g_addr_mu;
void* g_addr[64] = {};

// Device address of g_argmax_scratch on the current device, looked up with
// that device current.  Outside stream capture the lookup runs on every call
// (after the first it only reads the loaded module's symbol table and
// allocates nothing), so a context torn down by cudaDeviceReset and created
// again gets the new address; during capture the address of the last lookup
// on this device is used, which is why the first call must come before any
// capture.
int scratch_address(int device, cudaStream_t stream, void** out) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
        cudaGetLastError();
        cs = cudaStreamCaptureStatusActive;  // unknown: do not touch the module
    }
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (cs == cudaStreamCaptureStatusNone || g_addr[device] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress of the static argmax buffer");
        g_addr[device] = p;
    }
    *out = g_addr[device];
    return MRT_OK;
}

}  // namespace
}  // namespace mrt

using namespace mrt;

extern "C" int mrt_argmax_f16_noalloc(const void* logits_dev, int64_t M, int64_t V, int64_t ld,
                                      int64_t index_base, int64_t* idx_dev, float* val_dev, void* stream) {
    clear_error();
    if (M < 0 || V < 0 || ld < V) return set_error(MRT_ERR_SHAPE, "need M >= 0, V >= 0, ld >= V");
    if (M == 0) return MRT_OK;
    if (V == 0) return set_error(MRT_ERR_SHAPE, "argmax over an empty row");
    if (M > 65535) return set_error(MRT_ERR_SHAPE, "at most 65535 rows per call");
    if (logits_dev == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL logits");
    const size_t need = argmax_scratch_bytes(M, V);
    if (need > kNoAllocBytes)
        return set_error(MRT_ERR_SHAPE, "mrt_argmax_f16_noalloc: " + std::to_string(M) + " rows of " + std::to_string(V) +
                                            " logits need " + std::to_string(need) + " bytes of scratch; the static buffer holds " +
                                            std::to_string(kNoAllocBytes) + " (M * ceil(V / 8192) <= 8192)");
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (device < 0 || device >= 64) return set_error(MRT_ERR_INVALID_ARG, "device index out of range");
    void* scratch = nullptr;
    int rc = scratch_address(device, static_cast<cudaStream_t>(stream), &scratch);
    if (rc != MRT_OK) return rc;
    e = launch_argmax(static_cast<const uint16_t*>(logits_dev), M, V, ld, index_base, idx_dev, val_dev, scratch,
                      static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "argmax launch");
}
