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

#include <cstring>
#include <string>

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

struct mrt_tp_s {
    ncclComm_t comm = nullptr;
    int rank = 0;
    int world = 1;
    int device = -1;
    void* buf = nullptr;  // gather space
    size_t buf_bytes = 0;
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

extern "C" int mrt_tp_destroy(mrt_tp tp) {
    if (tp == nullptr) return MRT_OK;
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
