// tp.cu -- tensor-parallel shard map and NCCL collectives over NVLink.
//
// Column-parallel layers (q/k/v, gate/up, lm_head) split W's rows across
// ranks and need no exchange; row-parallel layers (o_proj, down) split K and
// all-reduce FP32 partials, rounding once to FP16 afterwards; the sharded
// lm_head all-gathers one (value, index) pair per row.  The reference has no
// parallelism beyond its CPU thread pool (src/core/cpu_backend.cpp:139-168).
//
// NCCL is resolved with dlopen at mrt_tp_init: the copy already loaded in the
// process (PyTorch's) is preferred, so one process never mixes two NCCL
// builds, and the library still loads where NCCL is absent.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "kernels.h"

namespace mrt {
namespace {

struct Nccl {
    bool loaded = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

Nccl g_nccl;

int load_nccl() {
    if (g_nccl.loaded) return MRT_OK;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) {
        const char* env = getenv("MRT_NCCL_LIBRARY");
        h = dlopen(env && *env ? env : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }
    if (h == nullptr) return set_error(MRT_ERR_NCCL, std::string("cannot load NCCL: ") + dlerror());
#define MRT_SYM(field, name)                                                       \
    g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name));       \
    if (g_nccl.field == nullptr) return set_error(MRT_ERR_NCCL, "NCCL symbol missing: " name);
    MRT_SYM(GetUniqueId, "ncclGetUniqueId")
    MRT_SYM(CommInitRank, "ncclCommInitRank")
    MRT_SYM(CommDestroy, "ncclCommDestroy")
    MRT_SYM(AllReduce, "ncclAllReduce")
    MRT_SYM(AllGather, "ncclAllGather")
    MRT_SYM(GetErrorString, "ncclGetErrorString")
#undef MRT_SYM
    g_nccl.loaded = true;
    return MRT_OK;
}

int nccl_error(ncclResult_t r, const char* what) {
    return set_error(MRT_ERR_NCCL, std::string(what) + ": " +
                                       (g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "NCCL error"));
}

}  // namespace
}  // namespace mrt

namespace mrt {
namespace {
constexpr int kP2PMaxRanks = 8;
constexpr size_t kP2PFlagBytes = 4096;  // two rows of kP2PMaxRanks 64-bit flags, padded
}  // namespace
}  // namespace mrt

struct mrt_tp_s {
    ncclComm_t comm = nullptr;
    int rank = 0;
    int world = 1;
    int device = -1;
    void* buf = nullptr;  // gather space
    size_t buf_bytes = 0;
    // Peer exchange (mrt_tp_p2p_init): this rank's region -- flags, an FP32
    // partial area of p2p_cap elements, an FP16 output area of p2p_cap --
    // exported by CUDA IPC; every rank's region as this rank maps it; and the
    // device counter of exchanges made so far.
    char* p2p_region = nullptr;
    char* p2p_peer[mrt::kP2PMaxRanks] = {};
    int64_t p2p_cap = 0;
    size_t p2p_part_off = 0, p2p_out_off = 0;
    unsigned long long* p2p_epoch = nullptr;
};

using namespace mrt;

namespace mrt {
int tp_rank_world(mrt_tp tp, int* rank, int* world) {
    if (tp == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL tensor-parallel handle");
    *rank = tp->rank;
    *world = tp->world;
    return MRT_OK;
}

int tp_allgather_host(mrt_tp tp, const void* in, void* out, size_t bytes) {
    if (tp == nullptr || in == nullptr || out == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    void* dev = nullptr;
    cudaError_t e = cudaMalloc(&dev, bytes * (tp->world + 1));
    if (e != cudaSuccess) return cuda_error(e, "allocating the exchange buffer");
    char* mine = static_cast<char*>(dev) + bytes * tp->world;
    e = cudaMemcpy(mine, in, bytes, cudaMemcpyHostToDevice);
    int rc = MRT_OK;
    if (e != cudaSuccess) {
        rc = cuda_error(e, "staging the exchange buffer");
    } else {
        ncclResult_t r = g_nccl.AllGather(mine, dev, bytes, ncclUint8, tp->comm, nullptr);
        if (r != ncclSuccess) {
            rc = nccl_error(r, "ncclAllGather of exchange records");
        } else {
            e = cudaMemcpy(out, dev, bytes * tp->world, cudaMemcpyDeviceToHost);  // waits for the gather
            if (e != cudaSuccess) rc = cuda_error(e, "reading the exchange records");
        }
    }
    cudaFree(dev);
    return rc;
}
}  // namespace mrt

extern "C" int mrt_shard_rows(const int64_t* part_rows, int64_t n_parts, int world, int rank,
                              int64_t* ranges_out) {
    clear_error();
    if (part_rows == nullptr || ranges_out == nullptr || n_parts <= 0)
        return set_error(MRT_ERR_INVALID_ARG, "need part sizes and an output array");
    if (world <= 0 || rank < 0 || rank >= world) return set_error(MRT_ERR_INVALID_ARG, "bad rank/world");
    int64_t off = 0;
    for (int64_t p = 0; p < n_parts; ++p) {
        const int64_t rows = part_rows[p];
        if (rows < world) return set_error(MRT_ERR_SHAPE, "a part has fewer rows than ranks");
        ranges_out[2 * p] = off + rows * rank / world;
        ranges_out[2 * p + 1] = off + rows * (rank + 1) / world;
        off += rows;
    }
    return MRT_OK;
}

extern "C" int mrt_shard_cols(int64_t K, int world, int rank, int64_t* k_begin, int64_t* k_end) {
    clear_error();
    if (world <= 0 || rank < 0 || rank >= world) return set_error(MRT_ERR_INVALID_ARG, "bad rank/world");
    if (K < world) return set_error(MRT_ERR_SHAPE, "K smaller than the number of ranks");
    // Slices stay multiples of 8 columns where K allows, so every shard keeps
    // the 16-byte rows the fast kernels stream.
    const int64_t unit = (K % (8LL * world) == 0) ? 8 : 1;
    const int64_t units = K / unit;
    if (k_begin) *k_begin = unit * (units * rank / world);
    if (k_end) *k_end = unit * (units * (rank + 1) / world);
    return MRT_OK;
}

extern "C" int mrt_tp_unique_id(void* id_out, size_t len) {
    clear_error();
    if (id_out == nullptr || len < sizeof(ncclUniqueId)) return set_error(MRT_ERR_INVALID_ARG, "id buffer too small");
    int rc = load_nccl();
    if (rc != MRT_OK) return rc;
    ncclUniqueId id;
    ncclResult_t r = g_nccl.GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_error(r, "ncclGetUniqueId");
    std::memcpy(id_out, &id, sizeof(id));
    return MRT_OK;
}

extern "C" int mrt_tp_init(int rank, int world, const void* id, size_t len, mrt_tp* out) {
    clear_error();
    if (out == nullptr || id == nullptr || len < sizeof(ncclUniqueId)) return set_error(MRT_ERR_INVALID_ARG, "bad arguments");
    if (world <= 0 || rank < 0 || rank >= world) return set_error(MRT_ERR_INVALID_ARG, "bad rank/world");
    *out = nullptr;
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    int rc = load_nccl();
    if (rc != MRT_OK) return rc;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    mrt_tp_s* tp = new mrt_tp_s();
    tp->rank = rank;
    tp->world = world;
    tp->device = c->device;
    ncclResult_t r = g_nccl.CommInitRank(&tp->comm, world, uid, rank);
    if (r != ncclSuccess) {
        delete tp;
        return nccl_error(r, "ncclCommInitRank");
    }
    *out = tp;
    return MRT_OK;
}

static void p2p_release(mrt_tp tp) {
    for (int q = 0; q < mrt::kP2PMaxRanks; ++q) {
        if (q != tp->rank && tp->p2p_peer[q] != nullptr) cudaIpcCloseMemHandle(tp->p2p_peer[q]);
        tp->p2p_peer[q] = nullptr;
    }
    if (tp->p2p_region) cudaFree(tp->p2p_region);
    if (tp->p2p_epoch) cudaFree(tp->p2p_epoch);
    tp->p2p_region = nullptr;
    tp->p2p_epoch = nullptr;
    tp->p2p_cap = 0;
}

extern "C" int mrt_tp_destroy(mrt_tp tp) {
    if (tp == nullptr) return MRT_OK;
    if (tp->p2p_region != nullptr) {
        // Every rank stops reading its peers' regions before any region goes.
        cudaDeviceSynchronize();
        int one = 1;
        std::vector<int> all(static_cast<size_t>(tp->world));
        tp_allgather_host(tp, &one, all.data(), sizeof(int));
        p2p_release(tp);
    }
    if (tp->comm) g_nccl.CommDestroy(tp->comm);
    if (tp->buf) cudaFree(tp->buf);
    delete tp;
    return MRT_OK;
}

extern "C" int mrt_tp_allreduce_f32_to_f16(mrt_tp tp, float* partial_dev, void* out_dev, int64_t count,
                                           void* stream) {
    clear_error();
    if (tp == nullptr || partial_dev == nullptr || out_dev == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    if (count < 0) return set_error(MRT_ERR_SHAPE, "count must be >= 0");
    if (count == 0) return MRT_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (tp->world > 1) {
        ncclResult_t r = g_nccl.AllReduce(partial_dev, partial_dev, static_cast<size_t>(count), ncclFloat32, ncclSum,
                                          tp->comm, s);
        if (r != ncclSuccess) return nccl_error(r, "ncclAllReduce");
    }
    cudaError_t e = launch_f32_to_f16(partial_dev, static_cast<uint16_t*>(out_dev), count, s);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "rounding the all-reduced sum");
}

extern "C" int mrt_tp_allgather_cols_f16(mrt_tp tp, const void* local_dev, int64_t M, int64_t n_local,
                                         void* out_dev, void* stream) {
    clear_error();
    if (tp == nullptr || local_dev == nullptr || out_dev == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    if (M < 0 || n_local < 0) return set_error(MRT_ERR_SHAPE, "negative size");
    if (M == 0 || n_local == 0) return MRT_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t block = static_cast<size_t>(M * n_local);
    if (M == 1) {
        ncclResult_t r = g_nccl.AllGather(local_dev, out_dev, block, ncclFloat16, tp->comm, s);
        return r == ncclSuccess ? MRT_OK : nccl_error(r, "ncclAllGather");
    }
    int rc = ensure_buffer(&tp->buf, &tp->buf_bytes, block * 2 * tp->world, "allocating the gather buffer");
    if (rc != MRT_OK) return rc;
    ncclResult_t r = g_nccl.AllGather(local_dev, tp->buf, block, ncclFloat16, tp->comm, s);
    if (r != ncclSuccess) return nccl_error(r, "ncclAllGather");
    for (int q = 0; q < tp->world; ++q) {
        cudaError_t e = cudaMemcpy2DAsync(static_cast<char*>(out_dev) + q * n_local * 2, tp->world * n_local * 2,
                                          static_cast<char*>(tp->buf) + q * block * 2, n_local * 2, n_local * 2, M,
                                          cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_error(e, "assembling gathered columns");
    }
    return MRT_OK;
}

extern "C" int mrt_tp_argmax(mrt_tp tp, const float* val_dev, const int64_t* idx_dev, int64_t M,
                             int64_t* idx_out_dev, void* stream) {
    clear_error();
    if (tp == nullptr || val_dev == nullptr || idx_dev == nullptr || idx_out_dev == nullptr)
        return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    if (M < 0) return set_error(MRT_ERR_SHAPE, "M must be >= 0");
    if (M == 0) return MRT_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t need = static_cast<size_t>(M) * tp->world * (sizeof(float) + sizeof(int64_t));
    int rc = ensure_buffer(&tp->buf, &tp->buf_bytes, need, "allocating the gather buffer");
    if (rc != MRT_OK) return rc;
    int64_t* gi = static_cast<int64_t*>(tp->buf);
    float* gv = reinterpret_cast<float*>(gi + M * tp->world);
    ncclResult_t r = g_nccl.AllGather(idx_dev, gi, static_cast<size_t>(M), ncclInt64, tp->comm, s);
    if (r == ncclSuccess) r = g_nccl.AllGather(val_dev, gv, static_cast<size_t>(M), ncclFloat32, tp->comm, s);
    if (r != ncclSuccess) return nccl_error(r, "ncclAllGather of argmax pairs");
    cudaError_t e = launch_argmax_combine(gv, gi, tp->world, M, idx_out_dev, s);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "argmax combine launch");
}

// ====================================================================== peer exchange
//
// Row-parallel outputs (o_proj, down_proj split along K) summed over NVLink
// by this library's own kernels instead of NCCL.  Every rank's GEMM writes its
// FP32 partial [count] into its exported region; then
//   kernel 1  publishes "my partial is complete" (epoch e, system-scope
//             release store into every peer's flag row 0), waits (bounded)
//             for every peer's, and reduces this rank's 1/world slice: the
//             world partials read over NVLink and added in rank order (the
//             same order for every element, so every rank's result is
//             bit-identical), rounded once to FP16 and stored into every
//             rank's output area (peer stores) -- reduce-scatter and
//             all-gather in one pass, 4 B read + 2 B written per element per
//             peer instead of an FP32 all-reduce's 8 B;
//   kernel 2  publishes "my stores into your output are complete" (flag row
//             1), waits (bounded) for every peer's, and advances the epoch.
// After kernel 2 every peer has finished reading this rank's partial area, so
// the next GEMM may overwrite it; a rank writes a peer's output area only after
// that peer published its next partial, which it does after consuming the
// previous output (stream order).  Waits give up after 2 s with kErrPeerWait
// (mrt_sync reports MRT_ERR_TIMEOUT); no load uses TMA or cluster broadcast.

namespace mrt {
namespace {

struct P2PArgs {
    const float* part[kP2PMaxRanks];
    uint16_t* out[kP2PMaxRanks];
    unsigned long long* flags[kP2PMaxRanks];
    unsigned long long* epoch;
    int64_t count;
    int rank, world;
    int* err;
};

// Threads 0 .. world-1 of the block: thread q != rank releases `epoch` into
// peer q's flag row `row` (slot = this rank) when `publish`, then waits for
// peer q's flag in this rank's row.  Returns the mask of ranks that arrived.
__device__ __forceinline__ unsigned p2p_meet(const P2PArgs& a, int row, unsigned long long epoch, bool publish) {
    __shared__ unsigned arrived;
    if (threadIdx.x == 0) arrived = 1u << a.rank;
    __syncthreads();
    const int q = static_cast<int>(threadIdx.x);
    if (q < a.world && q != a.rank) {
        if (publish) st_release_sys(a.flags[q] + row * kP2PMaxRanks + a.rank, epoch);
        const unsigned long long t0 = global_ns();
        while (true) {
            if (ld_acquire_sys(a.flags[a.rank] + row * kP2PMaxRanks + q) >= epoch) {
                atomicOr(&arrived, 1u << q);
                break;
            }
            if (global_ns() - t0 > kWaitLimitNs) {
                raise_error(a.err, kErrPeerWait);
                break;
            }
        }
    }
    __syncthreads();
    return arrived;
}

__global__ void __launch_bounds__(256) p2p_reduce_kernel(const P2PArgs a) {
    const unsigned long long epoch = *a.epoch + 1ull;
    const unsigned all = (a.world >= 32 ? 0xFFFFFFFFu : ((1u << a.world) - 1u));
    if (p2p_meet(a, 0, epoch, blockIdx.x == 0) != all) return;  // a peer is missing: error raised
    // This rank's slice (whole octets of elements), walked 256 elements per
    // warp and step: lane i reads float4 i and 32 + i of the step from every
    // rank -- each instruction one contiguous 512-byte run, four whole lines
    // per request over NVLink -- and writes the rounded halves back as two
    // 8-byte pieces per rank (256-byte runs).
    const int64_t groups = a.count / 8;
    const int64_t g0 = groups * a.rank / a.world, g1 = groups * (a.rank + 1) / a.world;
    const int64_t f_begin = g0 * 2, f_end = g1 * 2;  // float4 indices
    const int lane = static_cast<int>(threadIdx.x) & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t base = f_begin + warp0 * 64; base < f_end; base += nwarps * 64) {
        const int64_t fa = base + lane, fb = base + 32 + lane;
        const bool ha = fa < f_end, hb = fb < f_end;
        float4 va[kP2PMaxRanks], vb[kP2PMaxRanks];
#pragma unroll
        for (int q = 0; q < kP2PMaxRanks; ++q)
            if (q < a.world) {
                const float4* src = reinterpret_cast<const float4*>(a.part[q]);
                if (ha) va[q] = __ldcg(src + fa);
                if (hb) vb[q] = __ldcg(src + fb);
            }
        float ta[4] = {va[0].x, va[0].y, va[0].z, va[0].w};
        float tb[4] = {vb[0].x, vb[0].y, vb[0].z, vb[0].w};
#pragma unroll
        for (int q = 1; q < kP2PMaxRanks; ++q)
            if (q < a.world) {
                const float ua[4] = {va[q].x, va[q].y, va[q].z, va[q].w};
                const float ub[4] = {vb[q].x, vb[q].y, vb[q].z, vb[q].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    ta[e] = __fadd_rn(ta[e], ua[e]);
                    tb[e] = __fadd_rn(tb[e], ub[e]);
                }
            }
        const uint2 ha2 = make_uint2(
            static_cast<uint32_t>(f32_to_f16_bits(ta[0])) | (static_cast<uint32_t>(f32_to_f16_bits(ta[1])) << 16),
            static_cast<uint32_t>(f32_to_f16_bits(ta[2])) | (static_cast<uint32_t>(f32_to_f16_bits(ta[3])) << 16));
        const uint2 hb2 = make_uint2(
            static_cast<uint32_t>(f32_to_f16_bits(tb[0])) | (static_cast<uint32_t>(f32_to_f16_bits(tb[1])) << 16),
            static_cast<uint32_t>(f32_to_f16_bits(tb[2])) | (static_cast<uint32_t>(f32_to_f16_bits(tb[3])) << 16));
#pragma unroll
        for (int q = 0; q < kP2PMaxRanks; ++q)
            if (q < a.world) {
                uint2* dst = reinterpret_cast<uint2*>(a.out[q]);
                if (ha) dst[fa] = ha2;
                if (hb) dst[fb] = hb2;
            }
    }
    // the last count % 8 elements: the last rank's first thread
    if (a.rank == a.world - 1 && blockIdx.x == 0 && threadIdx.x == 0) {
        for (int64_t i = groups * 8; i < a.count; ++i) {
            float s = a.part[0][i];
            for (int q = 1; q < a.world; ++q) s = __fadd_rn(s, a.part[q][i]);
            const uint16_t h = f32_to_f16_bits(s);
            for (int q = 0; q < a.world; ++q) a.out[q][i] = h;
        }
    }
}

__global__ void p2p_done_kernel(const P2PArgs a) {
    const unsigned long long epoch = *a.epoch + 1ull;
    __threadfence_system();  // this rank's output stores (previous kernel) before the release
    p2p_meet(a, 1, epoch, true);
    if (threadIdx.x == 0) *a.epoch = epoch;
}

}  // namespace
}  // namespace mrt

extern "C" int mrt_tp_p2p_init(mrt_tp tp, int64_t max_count) {
    clear_error();
    if (tp == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL tensor-parallel handle");
    if (max_count <= 0) return set_error(MRT_ERR_SHAPE, "max_count must be > 0");
    if (tp->world > kP2PMaxRanks) return set_error(MRT_ERR_INVALID_ARG, "the peer exchange serves at most 8 ranks");
    if (tp->p2p_region != nullptr && tp->p2p_cap >= max_count) return MRT_OK;
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    if (tp->p2p_region != nullptr) {
        cudaDeviceSynchronize();
        int one = 1;
        std::vector<int> all(static_cast<size_t>(tp->world));
        int rc = tp_allgather_host(tp, &one, all.data(), sizeof(int));
        if (rc != MRT_OK) return rc;
        p2p_release(tp);
    }
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t part_off = kP2PFlagBytes;
    const size_t out_off = part_off + up(static_cast<size_t>(max_count) * 4);
    const size_t bytes = out_off + up(static_cast<size_t>(max_count) * 2);
    cudaError_t e = cudaMalloc(&tp->p2p_region, bytes);
    if (e != cudaSuccess) {
        tp->p2p_region = nullptr;
        return cuda_error(e, "allocating the peer exchange region");
    }
    e = cudaMalloc(&tp->p2p_epoch, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(tp->p2p_region, 0, kP2PFlagBytes);
    if (e == cudaSuccess) e = cudaMemset(tp->p2p_epoch, 0, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        p2p_release(tp);
        return cuda_error(e, "preparing the peer exchange region");
    }
    struct Rec {
        cudaIpcMemHandle_t h;
        int ok;
        int pad[15];
    } rec{};
    rec.ok = cudaIpcGetMemHandle(&rec.h, tp->p2p_region) == cudaSuccess ? 1 : 0;
    cudaGetLastError();
    std::vector<Rec> recs(static_cast<size_t>(tp->world));
    int rc = tp_allgather_host(tp, &rec, recs.data(), sizeof(Rec));
    if (rc != MRT_OK) {
        p2p_release(tp);
        return rc;
    }
    bool ok = true;
    for (const Rec& r : recs) ok = ok && r.ok;
    for (int q = 0; q < tp->world && ok; ++q) {
        if (q == tp->rank) {
            tp->p2p_peer[q] = tp->p2p_region;
            continue;
        }
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, recs[static_cast<size_t>(q)].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
        } else {
            tp->p2p_peer[q] = static_cast<char*>(p);
        }
    }
    // Every rank must have mapped every peer before any of them uses the path.
    int mine = ok ? 1 : 0;
    std::vector<int> oks(static_cast<size_t>(tp->world));
    rc = tp_allgather_host(tp, &mine, oks.data(), sizeof(int));
    if (rc != MRT_OK) {
        p2p_release(tp);
        return rc;
    }
    for (int v : oks) ok = ok && v;
    if (!ok) {
        p2p_release(tp);
        return set_error(MRT_ERR_CUDA, "peer memory cannot be mapped between these ranks (CUDA IPC)");
    }
    tp->p2p_cap = max_count;
    tp->p2p_part_off = part_off;
    tp->p2p_out_off = out_off;
    return MRT_OK;
}

extern "C" int mrt_tp_p2p_buffers(mrt_tp tp, float** partial_dev, void** out_dev) {
    clear_error();
    if (tp == nullptr || tp->p2p_region == nullptr) return set_error(MRT_ERR_INVALID_ARG, "peer exchange not initialised");
    if (partial_dev) *partial_dev = reinterpret_cast<float*>(tp->p2p_region + tp->p2p_part_off);
    if (out_dev) *out_dev = tp->p2p_region + tp->p2p_out_off;
    return MRT_OK;
}

extern "C" int mrt_tp_p2p_allreduce_f32_to_f16(mrt_tp tp, int64_t count, void* out_dev, int64_t ld_out,
                                               int64_t row_len, void* stream) {
    clear_error();
    if (tp == nullptr || tp->p2p_region == nullptr) return set_error(MRT_ERR_INVALID_ARG, "peer exchange not initialised");
    if (count < 0 || count > tp->p2p_cap) return set_error(MRT_ERR_SHAPE, "count exceeds the exchange region");
    if (count == 0) return MRT_OK;
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    P2PArgs a{};
    for (int q = 0; q < tp->world; ++q) {
        a.part[q] = reinterpret_cast<const float*>(tp->p2p_peer[q] + tp->p2p_part_off);
        a.out[q] = reinterpret_cast<uint16_t*>(tp->p2p_peer[q] + tp->p2p_out_off);
        a.flags[q] = reinterpret_cast<unsigned long long*>(tp->p2p_peer[q]);
    }
    a.epoch = tp->p2p_epoch;
    a.count = count;
    a.rank = tp->rank;
    a.world = tp->world;
    a.err = c->d_err;
    const int64_t per_rank = (count / 8 + tp->world - 1) / tp->world;
    int64_t blocks = (per_rank + 255) / 256;
    blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, static_cast<int64_t>(c->sms) * 8));
    p2p_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "peer reduce launch");
    p2p_done_kernel<<<1, 32, 0, s>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "peer exchange completion launch");
    note_launches(2);
    void* region_out = tp->p2p_region + tp->p2p_out_off;
    if (out_dev != nullptr && out_dev != region_out) {
        // The summed rows into the caller's buffer (rows of row_len, stride ld_out).
        if (row_len <= 0 || count % row_len != 0 || ld_out < row_len)
            return set_error(MRT_ERR_SHAPE, "count must be a whole number of rows of row_len <= ld_out");
        e = cudaMemcpy2DAsync(out_dev, static_cast<size_t>(ld_out) * 2, region_out, static_cast<size_t>(row_len) * 2,
                              static_cast<size_t>(row_len) * 2, static_cast<size_t>(count / row_len),
                              cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_error(e, "copying the summed rows out");
    }
    return MRT_OK;
}

extern "C" int mrt_tp_gemm_rowpar(mrt_tp tp, mrt_weight w, const void* x_dev, int64_t ldx, int64_t M, void* y_dev,
                                  int64_t ldy, void* stream) {
    clear_error();
    if (tp == nullptr || tp->p2p_region == nullptr) return set_error(MRT_ERR_INVALID_ARG, "peer exchange not initialised");
    int64_t n = 0, k = 0;
    int rc = mrt_weight_shape(w, &n, &k);
    if (rc != MRT_OK) return rc;
    if (M < 0) return set_error(MRT_ERR_SHAPE, "M must be >= 0");
    if (M == 0) return MRT_OK;
    if (M * n > tp->p2p_cap) return set_error(MRT_ERR_SHAPE, "M x N exceeds the exchange region");
    if (y_dev != nullptr && ldy < n) return set_error(MRT_ERR_SHAPE, "ldy must be >= N");
    // The whole FP32 partial into this rank's area, then the exchange.
    float* part = reinterpret_cast<float*>(tp->p2p_region + tp->p2p_part_off);
    rc = mrt_gemm_f32(w, x_dev, ldx, part, n, M, stream);
    if (rc != MRT_OK) return rc;
    return mrt_tp_p2p_allreduce_f32_to_f16(tp, M * n, y_dev, ldy, n, stream);
}
