// ctx.h -- per-device context and error helpers shared by the C-ABI sources.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "mrt_b200.h"

namespace mrt {

// One per device, created by mrt_init (or lazily by the first call).
struct DevCtx {
    int device = -1;
    int sms = 0;
    int* d_err = nullptr;   // device-side error flag written by bounded waits
    void* ws = nullptr;     // scratch: split-K partials, argmax partials
    size_t ws_bytes = 0;
    int* counters = nullptr;  // K-split tile counters, all zero between calls
    size_t counters_bytes = 0;
    void* io_x = nullptr;   // staging for host-buffer calls
    size_t io_x_bytes = 0;
    void* io_y = nullptr;
    size_t io_y_bytes = 0;
    void* gu = nullptr;     // interleaved gate|up product of an unfused mrt_gemm_swiglu
    size_t gu_bytes = 0;
    void* am = nullptr;     // greedy-pick partials of a fused lm_head (mrt_lm_head_argmax)
    size_t am_bytes = 0;
    // Host-buffer pipeline (mrt_gemm_host): a copy-in and a copy-out stream
    // beside the caller's, and events that hand each row chunk from one to
    // the next (created on first use).
    static constexpr int kIoChunks = 16;
    cudaStream_t io_in = nullptr;
    cudaStream_t io_out = nullptr;
    cudaEvent_t io_start = nullptr;
    cudaEvent_t io_h2d[kIoChunks] = {};
    cudaEvent_t io_mm[kIoChunks] = {};
    // mrt_gemm_host_async: kAsyncSets staging sets used in turn, each free
    // again once the event recorded after its last copy to the host has
    // completed (four: a step of four projections never waits for its own
    // earlier calls' copies to the host before copying its inputs in).
    static constexpr int kAsyncSets = 4;
    void* ax[kAsyncSets] = {};
    size_t ax_bytes[kAsyncSets] = {};
    void* ay[kAsyncSets] = {};
    size_t ay_bytes[kAsyncSets] = {};
    cudaEvent_t a_free[kAsyncSets] = {};
    int a_next = 0;
};

// Record an error for mrt_last_error_string() and return its code.
int set_error(int code, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);
void clear_error();

// Context of the current device (creating it on first use); nullptr after
// set_error on failure.
DevCtx* current_ctx();

// Grow a device buffer to at least `bytes` (synchronises the device before
// freeing a smaller one, so in-flight kernels never see it vanish).
int ensure_buffer(void** buf, size_t* cur, size_t bytes, const char* what);

// cuTensorMapEncodeTiled, resolved through the runtime so the library loads
// on machines without a driver.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// 2-D FP16 tensor map over a row-major [rows, cols] matrix with row stride
// `ld` elements, box = 64 columns x box_rows rows, 128-byte swizzle, zero fill.
int make_tmap_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                  int box_rows);
// The same over rows of exactly 64 FP16 with no swizzle (box 64 x box_rows).
int make_tmap_f16_rows64(CUtensorMap* map, const void* base, int64_t rows, int box_rows);

// Rank and world size of a tensor-parallel handle (tp.cu).
int tp_rank_world(mrt_tp tp, int* rank, int* world);
// Every rank's `bytes` host bytes, gathered in rank order into out[world * bytes]
// (synchronous; every rank of tp must call it).
int tp_allgather_host(mrt_tp tp, const void* in, void* out, size_t bytes);

// mrt_gemm with the SwiGLU epilogue for a weight whose rows interleave gate
// and up (row 2j = gate j, row 2j + 1 = up j): act[m][j] = fp16(lut[fp16(g)] *
// fp16(u)), act of w->n / 2 columns with row stride ld_act.  Runs only when
// the plan computes every tile over the whole K (*fused = true); otherwise
// launches nothing and sets *fused = false.
int gemm_swiglu(mrt_weight w, const void* x, int64_t ldx, void* act, int64_t ld_act, int64_t M,
                const uint16_t* lut, cudaStream_t s, bool* fused);
// The FP16 SiLU table of a device (ops.cu; nullptr if it cannot be built).
const uint16_t* silu_lut_for_device(int device);
// act[m][i] = fp16(lut[gu[m][2i]] * gu[m][2i+1]) for i < I (ops.cu).
cudaError_t launch_swiglu_pairs(const uint16_t* gu, int64_t ld_gu, int64_t I, int64_t M, const uint16_t* lut,
                                uint16_t* act, int64_t ld_act, cudaStream_t s);

// Number of decoder layers of a decoder handle (decoder.cu).
int64_t decoder_layer_count(mrt_decoder d);

}  // namespace mrt

// Opaque handle types of the public header.
struct mrt_weight_s {
    int device = -1;
    int64_t n = 0;  // rows kept
    int64_t k = 0;  // columns kept
    // FP16 data.  Row-major [n, k] when !tiled; when tiled, 128 x 64 tiles
    // [n_pad / 128][k_tiles][128][64], each stored in the byte order the
    // tensor cores read with 128-byte swizzling (16-byte chunk c of row r at
    // chunk position c ^ (r % 8)), padded with zeros to n_pad rows (a multiple
    // of 256) and k_tiles * 64 columns, so one linear bulk copy fills a
    // shared-memory ring stage.
    uint16_t* data = nullptr;
    bool owns_data = true;     // false for mrt_weight_view
    bool tiled = false;
    int64_t n_pad = 0;
    int64_t k_tiles = 0;
    uint16_t* bias = nullptr;  // FP16 [n] or nullptr
    int64_t src_n = 0;         // rows of the full source weight
    int64_t* ranges = nullptr; // row ranges kept (pairs)
    int64_t n_ranges = 0;
    // TMA maps of the weight, one per tile width (box rows 64, 128, 256); a
    // map's box must equal the kernel's W tile or the copy overruns the ring.
    CUtensorMap tmap[3];
    bool tmap_ok[3] = {false, false, false};
    // Tiled weights: the tiles as rows of 64 FP16 ([n_pad / 128 * k_tiles * 128]
    // rows, 64 x 128 box, no swizzle), for the SM-pair kernel's copies.
    CUtensorMap tmap_rows;
    bool tmap_rows_ok = false;
};
