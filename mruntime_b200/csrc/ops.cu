// ops.cu -- the non-GEMM Backend operations on the device (support for running
// a whole model with device-resident tensors).  Each kernel restates one
// CpuBackend op of the reference (src/core/cpu_backend.cpp:171-569); the
// arithmetic keeps the reference's operand order and separately rounded FP32
// operations (__fmul_rn / __fadd_rn / __fdiv_rn / __fsqrt_rn never fuse).
// Transcendentals that a GPU library would round differently from glibc are
// taken from host-built tables instead: SiLU on FP16 (all 65536 inputs) and
// RoPE's cos/sin (the reference's own float expressions).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "kernels.h"

namespace mrt {
namespace {

constexpr int kT = 256;

__device__ __forceinline__ float ld(const void* p, int dt, int64_t i) {
    if (dt == 2) return static_cast<const float*>(p)[i];
    const uint16_t v = static_cast<const uint16_t*>(p)[i];
    return dt == 1 ? bf16_bits_to_f32(v) : f16_bits_to_f32(v);
}

__device__ __forceinline__ void st(void* p, int dt, int64_t i, float v) {
    if (dt == 2) {
        static_cast<float*>(p)[i] = v;
    } else if (dt == 1) {
        static_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
    } else {
        static_cast<uint16_t*>(p)[i] = f32_to_f16_bits(v);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

unsigned blocks_for(int64_t n) {
    int64_t b = (n + kT - 1) / kT;
    if (b > 148 * 32) b = 148 * 32;
    return static_cast<unsigned>(b < 1 ? 1 : b);
}

// cpu_backend.cpp:292-330.  One block per token row.
__global__ void rmsnorm_kernel(const void* in, int idt, const void* w, int wdt, void* out, int odt, int64_t hidden,
                               float eps) {
    __shared__ float part[kT / 32];
    const int64_t row = blockIdx.x;
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < hidden; i += kT) {
        const float v = ld(in, idt, row * hidden + i);
        s = __fadd_rn(s, __fmul_rn(v, v));
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    float total = 0.0f;
    for (int wi = 0; wi < kT / 32; ++wi) total = __fadd_rn(total, part[wi]);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(hidden)), eps));
    const float inv = __fdiv_rn(1.0f, rms);
    for (int64_t i = threadIdx.x; i < hidden; i += kT) {
        const float x = ld(in, idt, row * hidden + i);
        st(out, odt, row * hidden + i, __fmul_rn(__fmul_rn(x, inv), ld(w, wdt, i)));
    }
}

// cpu_backend.cpp:332-379 with host-built cos/sin [seq][half].
__global__ void rope_kernel(void* x, int dt, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                            const float* cs, const float* sn) {
    const int64_t half = head_dim / 2;
    const int64_t total = batch * seq * heads * half;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * kT) {
        const int64_t i = e % half;
        const int64_t bh = e / half;  // (b*seq + s)*heads + h
        const int64_t s = (bh / heads) % seq;
        const int64_t base = bh * head_dim;
        const float c = cs[s * half + i], sv = sn[s * half + i];
        const float x0 = ld(x, dt, base + i);
        const float x1 = ld(x, dt, base + i + half);
        st(x, dt, base + i, __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sv)));
        st(x, dt, base + i + half, __fadd_rn(__fmul_rn(x0, sv), __fmul_rn(x1, c)));
    }
}

__global__ void silu_lut_kernel(const uint16_t* in, uint16_t* out, int64_t n, const uint16_t* lut) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * kT)
        out[i] = lut[in[i]];
}

__global__ void silu_kernel(const void* in, int idt, void* out, int odt, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * kT) {
        const float x = ld(in, idt, i);
        st(out, odt, i, __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))));
    }
}

// cpu_backend.cpp:403-455: op 0 = multiply, 1 = add.
__global__ void binary_kernel(const void* a, int adt, const void* b, int bdt, void* out, int odt, int64_t n, int op) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * kT) {
        const float x = ld(a, adt, i), y = ld(b, bdt, i);
        st(out, odt, i, op == 0 ? __fmul_rn(x, y) : __fadd_rn(x, y));
    }
}

// cpu_backend.cpp:457-515.  One warp per (outer, inner) row.
__global__ void softmax_kernel(const void* in, int idt, void* out, int odt, int64_t outer, int64_t dim, int64_t inner) {
    const int64_t row = (blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= outer * inner) return;
    const int64_t o = row / inner, in_i = row % inner;
    auto idx = [&](int64_t d) { return (o * dim + d) * inner + in_i; };
    float mx = -INFINITY;
    for (int64_t d = lane; d < dim; d += 32) mx = fmaxf(mx, ld(in, idt, idx(d)));
    mx = warp_max(mx);
    float s = 0.0f;
    for (int64_t d = lane; d < dim; d += 32) s = __fadd_rn(s, expf(__fsub_rn(ld(in, idt, idx(d)), mx)));
    s = warp_sum(s);
    for (int64_t d = lane; d < dim; d += 32) st(out, odt, idx(d), __fdiv_rn(expf(__fsub_rn(ld(in, idt, idx(d)), mx)), s));
}

// cpu_backend.cpp:517-569.
__global__ void embedding_kernel(const void* w, int wdt, int64_t hidden, const int32_t* ids, int64_t n, void* out,
                                 int odt) {
    const int64_t total = n * hidden;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x; e < total; e += static_cast<int64_t>(gridDim.x) * kT) {
        const int64_t t = e / hidden, i = e % hidden;
        const int64_t src = static_cast<int64_t>(ids[t]) * hidden + i;
        if (wdt == odt && wdt != 2) {
            static_cast<uint16_t*>(out)[e] = static_cast<const uint16_t*>(w)[src];
        } else {
            st(out, odt, e, ld(w, wdt, src));
        }
    }
}

struct AttnArgs {
    const void* q;
    const void* k;
    const void* v;
    void* o;
    int qdt, kdt, vdt, odt;
    int64_t qs[4], ks[4], vs[4], os[4];
    int64_t batch, heads, q_len, kv_len, qk_dim, v_dim;
    float scale;
    int causal;
};

constexpr int kMaxVDimPerLane = 8;  // v_dim <= 256

// cpu_backend.cpp:171-290.  One warp per (batch, head, query).  Two passes over
// the keys like the reference (max first, then exp-sum and weighted V sum in
// key order); the q.k dot is a warp tree sum.
__global__ void attention_kernel(const AttnArgs a) {
    const int64_t task = (blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (task >= a.batch * a.heads * a.q_len) return;
    const int64_t qi = task % a.q_len;
    const int64_t h = (task / a.q_len) % a.heads;
    const int64_t b = task / (a.q_len * a.heads);
    const int64_t base_pos = a.kv_len >= a.q_len ? a.kv_len - a.q_len : 0;
    int64_t max_k = a.kv_len - 1;
    if (a.causal && a.kv_len >= a.q_len) {
        max_k = base_pos + qi;
        if (max_k >= a.kv_len) max_k = a.kv_len - 1;
    }
    const int64_t qb = b * a.qs[0] + h * a.qs[1] + qi * a.qs[2];
    const int64_t kb = b * a.ks[0] + h * a.ks[1];
    const int64_t vb = b * a.vs[0] + h * a.vs[1];
    auto score = [&](int64_t ki) {
        float d = 0.0f;
        for (int64_t x = lane; x < a.qk_dim; x += 32)
            d = __fadd_rn(d, __fmul_rn(ld(a.q, a.qdt, qb + x * a.qs[3]), ld(a.k, a.kdt, kb + ki * a.ks[2] + x * a.ks[3])));
        return __fmul_rn(warp_sum(d), a.scale);
    };
    float mx = -INFINITY;
    for (int64_t ki = 0; ki <= max_k; ++ki) mx = fmaxf(mx, score(ki));
    float acc[kMaxVDimPerLane];
#pragma unroll
    for (int j = 0; j < kMaxVDimPerLane; ++j) acc[j] = 0.0f;
    float sum = 0.0f;
    for (int64_t ki = 0; ki <= max_k; ++ki) {
        const float e = expf(__fsub_rn(score(ki), mx));
        sum = __fadd_rn(sum, e);
#pragma unroll
        for (int j = 0; j < kMaxVDimPerLane; ++j) {
            const int64_t d = lane + 32 * j;
            if (d < a.v_dim) acc[j] = __fadd_rn(acc[j], __fmul_rn(e, ld(a.v, a.vdt, vb + ki * a.vs[2] + d * a.vs[3])));
        }
    }
    const float inv = __fdiv_rn(1.0f, sum);
    const int64_t ob = b * a.os[0] + h * a.os[1] + qi * a.os[2];
#pragma unroll
    for (int j = 0; j < kMaxVDimPerLane; ++j) {
        const int64_t d = lane + 32 * j;
        if (d < a.v_dim) st(a.o, a.odt, ob + d * a.os[3], __fmul_rn(acc[j], inv));
    }
}

// ---------------------------------------------------------------- host tables

std::mutex g_lut_mu;
uint16_t* g_silu_lut[64] = {};

// x / (1 + exp(-x)) for every FP16 input, with the reference's float
// expression (cpu_backend.cpp:397) on the host, rounded by the reference's
// converter rule.
uint16_t host_f32_to_f16(float f);

const uint16_t* silu_lut(int device) {
    std::lock_guard<std::mutex> lk(g_lut_mu);
    if (g_silu_lut[device] != nullptr) return g_silu_lut[device];
    std::vector<uint16_t> lut(65536);
    for (uint32_t h = 0; h < 65536; ++h) {
        __half_raw r;
        r.x = static_cast<unsigned short>(h);
        float x = __half2float(__half(r));
        if (x != x) x = std::numeric_limits<float>::quiet_NaN();  // the reference widens every NaN to +qNaN
        const float y = x / (1.0f + std::exp(-x));
        lut[h] = host_f32_to_f16(y);
    }
    uint16_t* d = nullptr;
    if (cudaMalloc(&d, 65536 * 2) != cudaSuccess) return nullptr;
    if (cudaMemcpy(d, lut.data(), 65536 * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(d);
        return nullptr;
    }
    g_silu_lut[device] = d;
    return d;
}

// Host restatement of the reference's FP32 -> FP16 rounding
// (include/mruntime/dtype.h:39-119), used only to build tables.
uint16_t host_f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint16_t sign = static_cast<uint16_t>((x >> 16) & 0x8000u);
    const uint32_t e = (x >> 23) & 0xFFu, m = x & 0x7FFFFFu;
    if (e == 0xFFu) {
        if (m == 0) return static_cast<uint16_t>(sign | 0x7C00u);
        uint32_t p = m >> 13;
        if ((p & 0x3FFu) == 0) p = 1;
        return static_cast<uint16_t>(sign | 0x7C00u | p);
    }
    if (e == 0) return sign;
    const int32_t he = static_cast<int32_t>(e) - 112;
    if (he >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
    if (he < -10) return sign;
    const uint32_t sig = m | 0x800000u;
    const int shift = he > 0 ? 13 : 14 - he;
    uint32_t q = sig >> shift;
    const uint32_t rem = sig & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    if (he > 0) return static_cast<uint16_t>(sign | ((static_cast<uint32_t>(he - 1) << 10) + q));
    return static_cast<uint16_t>(sign | q);
}

bool valid_dt(int dt) { return dt == MRT_FP16 || dt == MRT_BF16 || dt == MRT_FP32; }

int launch_status(const char* what) {
    cudaError_t e = cudaGetLastError();
    note_launches(1);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, what);
}

}  // namespace

// The FP16 SiLU table of `device` (built on first use), for fused kernels.
const uint16_t* silu_lut_for_device(int device) { return silu_lut(device); }

namespace {

// act[m][i] = fp16(silu(gate) * up) from an interleaved gate|up product
// (gate i at column 2i, up i at 2i + 1 of row m; qwen_model.cpp:278-285).
__global__ void swiglu_pairs_kernel(const uint16_t* gu, int64_t ld_gu, int64_t I, int64_t M, const uint16_t* lut,
                                    uint16_t* act, int64_t ld_act) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t total = M * I;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(kT) + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * kT) {
        const int64_t m = e / I, i = e % I;
        const uint16_t g = gu[m * ld_gu + 2 * i], u = gu[m * ld_gu + 2 * i + 1];
        act[m * ld_act + i] = f32_to_f16_bits(__fmul_rn(f16_bits_to_f32(lut[g]), f16_bits_to_f32(u)));
    }
}

}  // namespace

cudaError_t launch_swiglu_pairs(const uint16_t* gu, int64_t ld_gu, int64_t I, int64_t M, const uint16_t* lut,
                                uint16_t* act, int64_t ld_act, cudaStream_t s) {
    const int64_t blocks = std::min<int64_t>((M * I + kT - 1) / kT, 148 * 16);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks < 1 ? 1 : blocks));
    cfg.blockDim = dim3(kT);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, swiglu_pairs_kernel, gu, ld_gu, I, M, lut, act, ld_act);
    if (e == cudaSuccess) note_launches(1);
    return e;
}

}  // namespace mrt

using namespace mrt;

extern "C" int mrt_rmsnorm(const void* in, int idt, const void* w, int wdt, void* out, int odt, int64_t rows,
                           int64_t hidden, float eps, void* stream) {
    clear_error();
    if (!valid_dt(idt) || !valid_dt(wdt) || !valid_dt(odt)) return set_error(MRT_ERR_DTYPE, "bad dtype");
    if (rows < 0 || hidden <= 0) return set_error(MRT_ERR_SHAPE, "bad shape");
    if (rows == 0) return MRT_OK;
    if (!current_ctx()) return MRT_ERR_CUDA;
    rmsnorm_kernel<<<static_cast<unsigned>(rows), kT, 0, static_cast<cudaStream_t>(stream)>>>(in, idt, w, wdt, out, odt,
                                                                                             hidden, eps);
    return launch_status("rmsnorm launch");
}

extern "C" int mrt_rope(void* x, int dt, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                        int64_t position_offset, float theta, void* stream) {
    clear_error();
    if (!valid_dt(dt)) return set_error(MRT_ERR_DTYPE, "bad dtype");
    if (batch < 0 || seq < 0 || heads < 0 || head_dim < 2) return set_error(MRT_ERR_SHAPE, "bad shape");
    if (batch * seq * heads == 0) return MRT_OK;
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    const int64_t half = head_dim / 2;
    std::vector<float> tab(static_cast<size_t>(2 * seq * half));
    for (int64_t s = 0; s < seq; ++s)
        for (int64_t i = 0; i < half; ++i) {
            // cpu_backend.cpp:363-366, same float expressions
            const float freq = 1.0f / std::pow(theta, static_cast<float>(2 * i) / static_cast<float>(head_dim));
            const float angle = static_cast<float>(static_cast<size_t>(position_offset + s)) * freq;
            tab[s * half + i] = std::cos(angle);
            tab[seq * half + s * half + i] = std::sin(angle);
        }
    const size_t bytes = tab.size() * sizeof(float);
    int rc = ensure_buffer(&c->io_x, &c->io_x_bytes, bytes, "allocating RoPE tables");
    if (rc != MRT_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(c->io_x, tab.data(), bytes, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);  // the table is pageable host memory
    if (e != cudaSuccess) return cuda_error(e, "uploading RoPE tables");
    const float* cs = static_cast<const float*>(c->io_x);
    rope_kernel<<<blocks_for(batch * seq * heads * half), kT, 0, st>>>(x, dt, batch, seq, heads, head_dim, cs,
                                                                       cs + seq * half);
    return launch_status("rope launch");
}

extern "C" int mrt_silu(const void* in, int idt, void* out, int odt, int64_t n, void* stream) {
    clear_error();
    if (!valid_dt(idt) || !valid_dt(odt)) return set_error(MRT_ERR_DTYPE, "bad dtype");
    if (n < 0) return set_error(MRT_ERR_SHAPE, "n < 0");
    if (n == 0) return MRT_OK;
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (idt == MRT_FP16 && odt == MRT_FP16) {
        const uint16_t* lut = silu_lut(c->device);
        if (lut == nullptr) return set_error(MRT_ERR_CUDA, "building the SiLU table failed");
        silu_lut_kernel<<<blocks_for(n), kT, 0, st>>>(static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out), n, lut);
    } else {
        silu_kernel<<<blocks_for(n), kT, 0, st>>>(in, idt, out, odt, n);
    }
    return launch_status("silu launch");
}

static int binary(const void* a, int adt, const void* b, int bdt, void* out, int odt, int64_t n, int op, void* stream) {
    clear_error();
    if (!valid_dt(adt) || !valid_dt(bdt) || !valid_dt(odt)) return set_error(MRT_ERR_DTYPE, "bad dtype");
    if (n < 0) return set_error(MRT_ERR_SHAPE, "n < 0");
    if (n == 0) return MRT_OK;
    if (!current_ctx()) return MRT_ERR_CUDA;
    binary_kernel<<<blocks_for(n), kT, 0, static_cast<cudaStream_t>(stream)>>>(a, adt, b, bdt, out, odt, n, op);
    return launch_status(op == 0 ? "mul launch" : "add launch");
}

extern "C" int mrt_mul(const void* a, int adt, const void* b, int bdt, void* out, int odt, int64_t n, void* stream) {
    return binary(a, adt, b, bdt, out, odt, n, 0, stream);
}

extern "C" int mrt_add(const void* a, int adt, const void* b, int bdt, void* out, int odt, int64_t n, void* stream) {
    return binary(a, adt, b, bdt, out, odt, n, 1, stream);
}

extern "C" int mrt_softmax(const void* in, int idt, void* out, int odt, int64_t outer, int64_t dim, int64_t inner,
                           void* stream) {
    clear_error();
    if (!valid_dt(idt) || !valid_dt(odt)) return set_error(MRT_ERR_DTYPE, "bad dtype");
    if (outer < 0 || dim <= 0 || inner <= 0) return set_error(MRT_ERR_SHAPE, "bad shape");
    if (outer == 0) return MRT_OK;
    if (!current_ctx()) return MRT_ERR_CUDA;
    const int64_t threads = outer * inner * 32;
    softmax_kernel<<<static_cast<unsigned>((threads + kT - 1) / kT), kT, 0, static_cast<cudaStream_t>(stream)>>>(
        in, idt, out, odt, outer, dim, inner);
    return launch_status("softmax launch");
}

extern "C" int mrt_embedding(const void* w, int wdt, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t n,
                             void* out, int odt, void* stream) {
    clear_error();
    if (!valid_dt(wdt) || !valid_dt(odt)) return set_error(MRT_ERR_DTYPE, "bad dtype");
    if (vocab <= 0 || hidden <= 0 || n < 0) return set_error(MRT_ERR_SHAPE, "bad shape");
    if (n == 0) return MRT_OK;
    if (ids == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL token ids");
    for (int64_t t = 0; t < n; ++t)
        if (ids[t] < 0 || ids[t] >= vocab) return set_error(MRT_ERR_INVALID_ARG, "embedding_lookup: token_id out of range");
    DevCtx* c = current_ctx();
    if (!c) return MRT_ERR_CUDA;
    int rc = ensure_buffer(&c->io_x, &c->io_x_bytes, static_cast<size_t>(n) * 4, "allocating token ids");
    if (rc != MRT_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(c->io_x, ids, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_error(e, "uploading token ids");
    embedding_kernel<<<blocks_for(n * hidden), kT, 0, st>>>(w, wdt, hidden, static_cast<const int32_t*>(c->io_x), n,
                                                            out, odt);
    return launch_status("embedding launch");
}

extern "C" int mrt_attention(const void* q, int qdt, const int64_t* qs, const void* k, int kdt, const int64_t* ks,
                             const void* v, int vdt, const int64_t* vs, void* out, int odt, const int64_t* os,
                             int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int64_t qk_dim,
                             int64_t v_dim, float scale, int causal, void* stream) {
    clear_error();
    if (!valid_dt(qdt) || !valid_dt(kdt) || !valid_dt(vdt) || !valid_dt(odt)) return set_error(MRT_ERR_DTYPE, "bad dtype");
    if (!qs || !ks || !vs || !os) return set_error(MRT_ERR_INVALID_ARG, "NULL strides");
    if (batch < 0 || heads < 0 || q_len < 0 || kv_len <= 0 || qk_dim <= 0 || v_dim <= 0)
        return set_error(MRT_ERR_SHAPE, "bad shape");
    if (v_dim > 32 * kMaxVDimPerLane) return set_error(MRT_ERR_UNSUPPORTED, "v head size above 256");
    if (batch * heads * q_len == 0) return MRT_OK;
    if (!current_ctx()) return MRT_ERR_CUDA;
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.o = out;
    a.qdt = qdt; a.kdt = kdt; a.vdt = vdt; a.odt = odt;
    for (int i = 0; i < 4; ++i) {
        a.qs[i] = qs[i]; a.ks[i] = ks[i]; a.vs[i] = vs[i]; a.os[i] = os[i];
    }
    a.batch = batch; a.heads = heads; a.q_len = q_len; a.kv_len = kv_len;
    a.qk_dim = qk_dim; a.v_dim = v_dim; a.scale = scale; a.causal = causal;
    const int64_t threads = batch * heads * q_len * 32;
    attention_kernel<<<static_cast<unsigned>((threads + kT - 1) / kT), kT, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return launch_status("attention launch");
}
