// elementwise.cu -- HBM-bound helper kernels of the linear-layer path:
//   * dtype conversion with the reference's rounding (weight upload: the
//     BF16 -> FP16 step of src/core/cpu_backend.cpp:48-55, done once on the
//     device instead of on the host per packed weight);
//   * FP32 -> FP16 rounding after a row-parallel all-reduce;
//   * greedy argmax over FP16 logits (src/engine/inference_engine.cpp:84-95),
//     in two passes: per-chunk (value, index) partials in scratch memory, then
//     one block per row combines them.
// All grids are sized in multiples of the SM count or by the data; loads and
// stores are 16-byte vectors where alignment allows.
#include "common.cuh"
#include "kernels.h"

namespace mrt {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float load_as_f32(const void* p, int dt, int64_t i) {
    if (dt == 2) return static_cast<const float*>(p)[i];
    const uint16_t v = static_cast<const uint16_t*>(p)[i];
    return dt == 1 ? bf16_bits_to_f32(v) : f16_bits_to_f32(v);
}

__device__ __forceinline__ void store_from_f32(void* p, int dt, int64_t i, float v) {
    if (dt == 2) {
        static_cast<float*>(p)[i] = v;
    } else if (dt == 1) {
        static_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
    } else {
        static_cast<uint16_t*>(p)[i] = f32_to_f16_bits(v);
    }
}

__global__ void convert_kernel(const void* src, int sdt, void* dst, int ddt, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        if (sdt == ddt && sdt != 2) {
            static_cast<uint16_t*>(dst)[i] = static_cast<const uint16_t*>(src)[i];
        } else {
            store_from_f32(dst, ddt, i, load_as_f32(src, sdt, i));
        }
    }
}

__global__ void convert_2d_kernel(const void* src, int sdt, int64_t ld, int64_t rows, int64_t cols,
                                  uint16_t* dst) {
    const int64_t total = rows * cols;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols;
        const int64_t c = i - r * cols;
        const int64_t si = r * ld + c;
        dst[i] = (sdt == 0) ? static_cast<const uint16_t*>(src)[si]
                            : f32_to_f16_bits(load_as_f32(src, sdt, si));
    }
}

// Weight upload into the tiled layout: rows [row0, row0 + rows) of the
// destination from a [rows, cols] source (row stride ld) of dtype sdt, rounded
// to FP16 with the reference's converter.  Padding was zeroed beforehand.
__global__ void convert_rows_to_tiled_kernel(const void* src, int sdt, int64_t ld, int64_t rows, int64_t cols,
                                             uint16_t* dst, int64_t row0, int64_t k_tiles) {
    const int64_t total = rows * cols;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols;
        const int64_t c = i - r * cols;
        const int64_t si = r * ld + c;
        const uint16_t v = (sdt == 0) ? static_cast<const uint16_t*>(src)[si]
                                      : f32_to_f16_bits(load_as_f32(src, sdt, si));
        dst[tiled_offset(row0 + r, c, k_tiles)] = v;
    }
}

// Row-major [n, k] copy (row stride ld) of a tiled weight.
__global__ void untile_kernel(const uint16_t* src, int64_t n, int64_t k, int64_t k_tiles, uint16_t* dst, int64_t ld) {
    const int64_t total = n * k;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / k;
        const int64_t c = i - r * k;
        dst[r * ld + c] = src[tiled_offset(r, c, k_tiles)];
    }
}

// Finish the K-split tail tiles of a normal-mode tensor-core GEMM plan (the
// swap mode finishes its small tiles inside the GEMM kernel): partials are
// [tail_splits][n_tail][tile_m][bn] FP32 (tile_m = 128, or 256 for SM-pair
// plans); slices are added in index order, so results are deterministic.  The
// whole GPU shares the work, which matters for wide tiles (a 128 x 256 tile
// is 128 KB per slice).
__global__ void reduce_tail_kernel(const TcGemmArgs a, int num_m, int n_tail, int tile_m) {
    // Launched while the GEMM still runs; its partials are read after it.
    griddep_launch_dependents();
    griddep_wait();
    const int bn = a.bn;
    const int64_t per_tile = static_cast<int64_t>(tile_m) * bn;
    const int64_t total4 = static_cast<int64_t>(n_tail) * per_tile / 4;
    for (int64_t e4 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e4 < total4;
         e4 += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = e4 * 4;
        const int64_t ti = e / per_tile;
        const int64_t rem = e - ti * per_tile;
        const int64_t r = rem / bn, c = rem - r * bn;
        const int64_t t = a.full_tiles + ti;
        const int64_t row = (t % num_m) * tile_m + r;
        const int64_t col = (t / num_m) * bn + c;
        if (row >= a.M || col >= a.N) continue;
        float4 s = *reinterpret_cast<const float4*>(a.partials + e);
        for (int sp = 1; sp < a.tail_splits; ++sp) {
            const float4 p =
                *reinterpret_cast<const float4*>(a.partials + (sp * static_cast<int64_t>(n_tail) + ti) * per_tile + rem);
            s.x += p.x;
            s.y += p.y;
            s.z += p.z;
            s.w += p.w;
        }
        const float v[4] = {s.x, s.y, s.z, s.w};
        for (int j = 0; j < 4 && col + j < a.N; ++j) {
            if (a.out_f32) {
                static_cast<float*>(a.y)[row * a.ldy + col + j] = v[j];
            } else {
                static_cast<uint16_t*>(a.y)[row * a.ldy + col + j] =
                    add_residual(round_out(v[j], a.bias, col + j), a.residual, row * a.ldr + col + j);
            }
        }
    }
}

__global__ void f32_to_f16_kernel(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = f32_to_f16_bits(src[i]);
}

// ---------------------------------------------------------------- argmax

using Best = ArgBest;

__device__ __forceinline__ Best better(Best a, Best b) { return arg_better(a, b); }

__device__ __forceinline__ Best block_best(Best b) {
    __shared__ float sv[kThreads / 32];
    __shared__ int64_t si[kThreads / 32];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        Best o;
        o.v = __shfl_down_sync(0xFFFFFFFFu, b.v, off);
        o.i = __shfl_down_sync(0xFFFFFFFFu, b.i, off);
        b = better(b, o);
    }
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[warp] = b.v;
        si[warp] = b.i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kThreads / 32; ++w) b = better(b, Best{sv[w], si[w]});
    }
    return b;  // valid in thread 0
}

constexpr int64_t kArgmaxChunk = 8192;  // logits per block in the first pass

// Pass 1: block (c, m) scans logits[m, c*chunk, (c+1)*chunk).
__global__ void argmax_partial_kernel(const uint16_t* logits, int64_t V, int64_t ld, float* pv,
                                      int64_t* pi, int64_t nchunks) {
    const int64_t m = blockIdx.y;
    const int64_t c = blockIdx.x;
    const uint16_t* row = logits + m * ld;
    const int64_t lo = c * kArgmaxChunk;
    const int64_t hi = min(V, lo + kArgmaxChunk);
    Best b{-INFINITY, INT64_MAX};
    const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0) && (lo % 8 == 0);
    if (vec) {
        for (int64_t base = lo + threadIdx.x * 8; base < hi; base += kThreads * 8) {
            if (base + 8 <= hi) {
                const uint4 q = __ldg(reinterpret_cast<const uint4*>(row + base));
                const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    b = better(b, Best{nan_to_ninf(f16_bits_to_f32(static_cast<uint16_t>(w[j] & 0xFFFFu))),
                                       base + 2 * j});
                    b = better(b, Best{nan_to_ninf(f16_bits_to_f32(static_cast<uint16_t>(w[j] >> 16))),
                                       base + 2 * j + 1});
                }
            } else {
                for (int64_t i = base; i < hi; ++i)
                    b = better(b, Best{nan_to_ninf(f16_bits_to_f32(row[i])), i});
            }
        }
    } else {
        for (int64_t i = lo + threadIdx.x; i < hi; i += kThreads)
            b = better(b, Best{nan_to_ninf(f16_bits_to_f32(row[i])), i});
    }
    b = block_best(b);
    if (threadIdx.x == 0) {
        pv[m * nchunks + c] = b.v;
        pi[m * nchunks + c] = b.i;
    }
}

// Pass 2: one block per row over its chunk partials.
__global__ void argmax_final_kernel(const float* pv, const int64_t* pi, int64_t nchunks,
                                    int64_t index_base, int64_t* idx, float* val) {
    const int64_t m = blockIdx.x;
    Best b{-INFINITY, INT64_MAX};
    for (int64_t c = threadIdx.x; c < nchunks; c += kThreads)
        b = better(b, Best{pv[m * nchunks + c], pi[m * nchunks + c]});
    b = block_best(b);
    if (threadIdx.x == 0) {
        if (idx) idx[m] = b.i + index_base;
        if (val) val[m] = b.v;
    }
}

// Combine per-rank partials gathered as [world, M] (indices already global).
__global__ void argmax_combine_kernel(const float* vals, const int64_t* idxs, int world, int64_t M,
                                      int64_t* out) {
    const int64_t m = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (m >= M) return;
    Best b{vals[m], idxs[m]};
    for (int r = 1; r < world; ++r) b = better(b, Best{vals[r * M + m], idxs[r * M + m]});
    out[m] = b.i;
}

// One thread waits on an mbarrier that never completes a phase (count 1, no
// arrival) with the GEMM kernels' wait routine and a short limit.
__global__ void wait_selftest_kernel(int* flag, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, flag, kErrSelfTest, limit_ns);
}

unsigned grid_for(int64_t n) {
    int64_t blocks = (n + kThreads - 1) / kThreads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    return static_cast<unsigned>(blocks < 1 ? 1 : blocks);
}

}  // namespace

cudaError_t launch_convert(const void* src, int sdt, void* dst, int ddt, int64_t n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    convert_kernel<<<grid_for(n), kThreads, 0, s>>>(src, sdt, dst, ddt, n);
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_convert_2d_to_f16(const void* src, int sdt, int64_t ld, int64_t rows,
                                     int64_t cols, uint16_t* dst, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    convert_2d_kernel<<<grid_for(rows * cols), kThreads, 0, s>>>(src, sdt, ld, rows, cols, dst);
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_convert_rows_to_tiled(const void* src, int sdt, int64_t ld, int64_t rows, int64_t cols,
                                         uint16_t* dst, int64_t row0, int64_t k_tiles, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    convert_rows_to_tiled_kernel<<<grid_for(rows * cols), kThreads, 0, s>>>(src, sdt, ld, rows, cols, dst, row0, k_tiles);
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_untile(const uint16_t* src, int64_t n, int64_t k, int64_t k_tiles, uint16_t* dst, int64_t ld,
                          cudaStream_t s) {
    if (n <= 0 || k <= 0) return cudaSuccess;
    untile_kernel<<<grid_for(n * k), kThreads, 0, s>>>(src, n, k, k_tiles, dst, ld);
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_reduce_tail(const TcGemmArgs& a, cudaStream_t s) {
    if (a.swap) return cudaErrorInvalidValue;  // swap mode finishes its tail tiles in the GEMM kernel
    const int tile_m = a.pair ? 256 : 128;
    const int num_m = (a.M + tile_m - 1) / tile_m;
    const int n_tail = tc_gemm_tiles(a) - a.full_tiles;
    if (n_tail <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid_for(static_cast<int64_t>(n_tail) * tile_m * a.bn / 4));
    cfg.blockDim = dim3(kThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, reduce_tail_kernel, a, num_m, n_tail, tile_m);
    if (e != cudaSuccess) return e;
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_wait_selftest(int* flag, uint64_t limit_ns, cudaStream_t s) {
    wait_selftest_kernel<<<1, 32, 0, s>>>(flag, limit_ns);
    note_launches(1);
    return cudaGetLastError();
}


cudaError_t launch_f32_to_f16(const float* src, uint16_t* dst, int64_t n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    f32_to_f16_kernel<<<grid_for(n), kThreads, 0, s>>>(src, dst, n);
    note_launches(1);
    return cudaGetLastError();
}

size_t argmax_scratch_bytes(int64_t M, int64_t V) {
    const int64_t nchunks = (V + kArgmaxChunk - 1) / kArgmaxChunk;
    return static_cast<size_t>(M * nchunks) * (sizeof(float) + sizeof(int64_t)) + 64;
}

cudaError_t launch_argmax(const uint16_t* logits, int64_t M, int64_t V, int64_t ld,
                          int64_t index_base, int64_t* idx, float* val, void* scratch,
                          cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (V <= 0) return cudaErrorInvalidValue;
    const int64_t nchunks = (V + kArgmaxChunk - 1) / kArgmaxChunk;
    int64_t* pi = static_cast<int64_t*>(scratch);
    float* pv = reinterpret_cast<float*>(pi + M * nchunks);
    dim3 grid(static_cast<unsigned>(nchunks), static_cast<unsigned>(M));
    argmax_partial_kernel<<<grid, kThreads, 0, s>>>(logits, V, ld, pv, pi, nchunks);
    note_launches(1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    argmax_final_kernel<<<static_cast<unsigned>(M), kThreads, 0, s>>>(pv, pi, nchunks, index_base, idx, val);
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_argmax_final(const float* pv, const int64_t* pi, int64_t M, int64_t nchunks,
                                int64_t index_base, int64_t* idx, float* val, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (nchunks <= 0) return cudaErrorInvalidValue;
    argmax_final_kernel<<<static_cast<unsigned>(M), kThreads, 0, s>>>(pv, pi, nchunks, index_base, idx, val);
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_argmax_combine(const float* vals, const int64_t* idxs, int world, int64_t M,
                                  int64_t* idx_out, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    argmax_combine_kernel<<<static_cast<unsigned>((M + 127) / 128), 128, 0, s>>>(vals, idxs, world, M, idx_out);
    note_launches(1);
    return cudaGetLastError();
}

}  // namespace mrt
