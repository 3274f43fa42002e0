// decoder.cu -- device-resident greedy generation for Qwen2-architecture
// decoders: the reference's QwenModel::forward (src/models/qwen/qwen_model.cpp:
// 104-376) driven by InferenceEngine::generate's greedy path
// (src/engine/inference_engine.cpp:26-95), with every tensor resident in HBM.
//
// Layout in HBM:
//   weights    per layer: q|k|v rows fused into one tiled weight with the
//              three biases attached (FP16, the reference's double rounding),
//              o, gate|up fused, down; lm_head tiled; the embedding table as a
//              row-major FP16 copy; RMSNorm gains in their source dtype.
//   KV cache   K and V [layer][kv_head][max_seq][head_dim] FP16 -- the
//              reference's KVCache layout (qwen_model.cpp:37-52).
//   activations [S, width] FP16 rows, reused across layers.
//   state      {position, step, current token} on the device, so one
//              captured decode step (a CUDA graph) replays for every token
//              without a host round trip; generated ids go to a device array.
//
// Per layer: add+RMSNorm (the previous layer's residual), q|k|v GEMM with
// bias, RoPE + KV append, attention, o GEMM, add+RMSNorm, gate|up GEMM,
// SiLU*up, down GEMM; then the final add+RMSNorm, lm_head on the last row and
// the greedy pick.  Every small kernel first lets the next launch start
// (griddepcontrol.launch_dependents) and then waits (griddepcontrol.wait) for
// the kernel before it before touching memory, so launches are hidden and each
// GEMM's weight stream begins while the small kernels before it run.
//
// Rounding points are the reference's: every op reads FP16 and writes FP16,
// computing in FP32 with its operand order (no fused multiply-adds).  The
// reductions (RMSNorm's sum of squares, attention) are summed in a
// different order than the reference's sequential loops, so results agree
// within FP32 rounding, not bit for bit.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "decode_step.h"
#include "kernels.h"

namespace mrt {

const uint16_t* silu_lut_for_device(int device);

namespace {

constexpr int kNT = 256;

struct DecState {
    int32_t pos;    // position of the first row of the current forward
    int32_t step;   // generated tokens so far
    int32_t token;  // last generated token
    int32_t pad;
};

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
    if (e == cudaSuccess) note_launches(1);
    return e;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < kNT / 32; ++w) t = __fadd_rn(t, red[w]);
    return t;
}

constexpr int kNormVec = 8;  // 16-byte vectors per thread: hidden <= 256 * 8 * 8 = 16384
constexpr int64_t kPreloadRows = 148;  // row launches up to one wave preload their RMSNorm gains

__device__ __forceinline__ uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ void unpack8(const uint4& v, float (&x)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        x[2 * e] = f16_bits_to_f32(static_cast<uint16_t>(w[e] & 0xFFFFu));
        x[2 * e + 1] = f16_bits_to_f32(static_cast<uint16_t>(w[e] >> 16));
    }
}

__device__ __forceinline__ uint32_t pack2(uint16_t lo, uint16_t hi) {
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// Eight RMSNorm gains starting at element i, in their dtype.
__device__ __forceinline__ void gains8(const void* w, int wdt, int64_t i, float (&g)[8]) {
    if (wdt == MRT_FP32) {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(w) + i);
        const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(w) + i + 4);
        g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w; g[4] = b.x; g[5] = b.y; g[6] = b.z; g[7] = b.w;
        return;
    }
    const uint4 v = ld16(static_cast<const uint16_t*>(w) + i);
    const uint32_t q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint16_t lo = static_cast<uint16_t>(q[e] & 0xFFFFu), hi = static_cast<uint16_t>(q[e] >> 16);
        g[2 * e] = wdt == MRT_BF16 ? bf16_bits_to_f32(lo) : f16_bits_to_f32(lo);
        g[2 * e + 1] = wdt == MRT_BF16 ? bf16_bits_to_f32(hi) : f16_bits_to_f32(hi);
    }
}

// RMSNorm of one row whose FP16-rounded values this thread holds as
// x[j][e] = element (threadIdx.x + j * kNT) * 8 + e (cpu_backend.cpp:292-330):
// rms = sqrt(sum(x^2) / n + eps); out = fp16((x * (1 / rms)) * w).
// This thread's RMSNorm gains (the vectors norm_vecs writes), loaded before
// the programmatic wait by kernels of at most one wave of rows (decode): the
// gains are never written after the decoder is loaded, so their latency
// overlaps the previous kernel.  Larger launches (prefill) load them after
// the reduction instead and keep the registers (two blocks per SM).
__device__ __forceinline__ void load_gains(const void* w, int wdt, int nv, float (&g)[kNormVec][8]) {
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int v = static_cast<int>(threadIdx.x) + j * kNT;
        if (v < nv) gains8(w, wdt, static_cast<int64_t>(v) * 8, g[j]);
    }
}

template <bool kPre>
__device__ __forceinline__ void norm_vecs(const float (&x)[kNormVec][8], int nv, int64_t H,
                                          const float (&g)[kNormVec][8], const void* w, int wdt, float eps,
                                          uint16_t* __restrict__ out, float* red) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kNormVec; ++j)
        if (static_cast<int>(threadIdx.x) + j * kNT < nv)
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(x[j][e], x[j][e]));
    const float total = block_sum(ss, red);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), eps));
    const float inv = __fdiv_rn(1.0f, rms);
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int v = static_cast<int>(threadIdx.x) + j * kNT;
        if (v >= nv) continue;
        float gl[8];
        if constexpr (kPre) {
#pragma unroll
            for (int e = 0; e < 8; ++e) gl[e] = g[j][e];
        } else {
            gains8(w, wdt, static_cast<int64_t>(v) * 8, gl);
        }
        uint16_t h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = f32_to_f16_bits(__fmul_rn(__fmul_rn(x[j][e], inv), gl[e]));
        *reinterpret_cast<uint4*>(out + static_cast<int64_t>(v) * 8) =
            make_uint4(pack2(h[0], h[1]), pack2(h[2], h[3]), pack2(h[4], h[5]), pack2(h[6], h[7]));
    }
}

// Row s: hidden = table[id] (qwen_model.cpp:59-64), normed = RMSNorm(hidden).
// ids == nullptr: the id is the state's current token.  Rows are 16-byte
// vectors; every load of a thread is issued before any is used.
template <bool kPre>
__global__ void __launch_bounds__(kNT) embed_norm_kernel(const uint16_t* __restrict__ table, int64_t vocab, int64_t H,
                                                         const int32_t* ids, const DecState* st,
                                                         uint16_t* __restrict__ hidden, const void* __restrict__ w,
                                                         int wdt, float eps, uint16_t* __restrict__ normed, int* err) {
    griddep_launch_dependents();
    float g[kNormVec][8];
    if constexpr (kPre) load_gains(w, wdt, static_cast<int>(H / 8), g);
    griddep_wait();
    __shared__ float red[kNT / 32];
    const int64_t s = blockIdx.x;
    int64_t id = ids != nullptr ? ids[s] : st->token;
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) raise_error(err, kErrBadToken);
        id = 0;
    }
    const int nv = static_cast<int>(H / 8);
    uint4 v[kNormVec];
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int i = static_cast<int>(threadIdx.x) + j * kNT;
        if (i < nv) v[j] = ld16(table + id * H + static_cast<int64_t>(i) * 8);
    }
    float x[kNormVec][8];
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int i = static_cast<int>(threadIdx.x) + j * kNT;
        if (i >= nv) continue;
        *reinterpret_cast<uint4*>(hidden + s * H + static_cast<int64_t>(i) * 8) = v[j];
        unpack8(v[j], x[j]);
    }
    norm_vecs<kPre>(x, nv, H, g, w, wdt, eps, normed + s * H, red);
}

// Row s: out = fp16(a + b) (cpu_backend.cpp:403-455), normed = RMSNorm(out).
template <bool kPre>
__global__ void __launch_bounds__(kNT) add_norm_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                                                       uint16_t* __restrict__ out, int64_t H, const void* __restrict__ w,
                                                       int wdt, float eps, uint16_t* __restrict__ normed) {
    griddep_launch_dependents();
    float g[kNormVec][8];
    if constexpr (kPre) load_gains(w, wdt, static_cast<int>(H / 8), g);
    griddep_wait();
    __shared__ float red[kNT / 32];
    const int64_t s = blockIdx.x;
    const int nv = static_cast<int>(H / 8);
    uint4 va[kNormVec], vb[kNormVec];
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int i = static_cast<int>(threadIdx.x) + j * kNT;
        if (i < nv) {
            va[j] = ld16(a + s * H + static_cast<int64_t>(i) * 8);
            vb[j] = ld16(b + s * H + static_cast<int64_t>(i) * 8);
        }
    }
    float x[kNormVec][8];
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int i = static_cast<int>(threadIdx.x) + j * kNT;
        if (i >= nv) continue;
        float fa[8], fb[8];
        unpack8(va[j], fa);
        unpack8(vb[j], fb);
        uint16_t h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            h[e] = f32_to_f16_bits(__fadd_rn(fa[e], fb[e]));
            x[j][e] = f16_bits_to_f32(h[e]);
        }
        *reinterpret_cast<uint4*>(out + s * H + static_cast<int64_t>(i) * 8) =
            make_uint4(pack2(h[0], h[1]), pack2(h[2], h[3]), pack2(h[4], h[5]), pack2(h[6], h[7]));
    }
    norm_vecs<kPre>(x, nv, H, g, w, wdt, eps, normed + s * H, red);
}

// RoPE on the q and k heads of S rows (cpu_backend.cpp:332-379, cos/sin from
// a host table built with the reference's expressions) and the KV-cache append
// (qwen_model.cpp:162-205): q is rotated in place, the rotated k and the v row
// go to cache position pos + s.  One thread per rotation pair.
__global__ void rope_append_kernel(uint16_t* qkv, int64_t ldq, int64_t S, int heads, int kv_heads, int D,
                                   const float* cos_t, const float* sin_t, uint16_t* kc, uint16_t* vc,
                                   int64_t max_seq, const DecState* st) {
    griddep_launch_dependents();
    griddep_wait();
    const int half = D / 2;
    const int64_t per_row = static_cast<int64_t>(heads + kv_heads) * half;
    const int64_t total = S * per_row;
    const int64_t pos0 = st->pos;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(kNT) + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * kNT) {
        const int64_t s = e / per_row;
        const int64_t r = e % per_row;
        const int hh = static_cast<int>(r / half);
        const int i = static_cast<int>(r % half);
        const int64_t pos = pos0 + s;
        if (pos >= max_seq) continue;  // the host checks lengths; never write past the cache
        const float c = cos_t[pos * half + i], sn = sin_t[pos * half + i];
        uint16_t* x = qkv + s * ldq + static_cast<int64_t>(hh) * D;
        const float x0 = f16_bits_to_f32(x[i]);
        const float x1 = f16_bits_to_f32(x[i + half]);
        const uint16_t y0 = f32_to_f16_bits(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
        const uint16_t y1 = f32_to_f16_bits(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
        if (hh < heads) {
            x[i] = y0;
            x[i + half] = y1;
        } else {
            const int g = hh - heads;
            const int64_t slot = (static_cast<int64_t>(g) * max_seq + pos) * D;
            kc[slot + i] = y0;
            kc[slot + i + half] = y1;
            const uint16_t* v = qkv + s * ldq + static_cast<int64_t>(heads + kv_heads + g) * D;
            vc[slot + i] = v[i];
            vc[slot + i + half] = v[i + half];
        }
    }
}

constexpr int kAttnWarps = 4;
constexpr int kKeysPerWarp = 8;
constexpr int kSplitKeys = kAttnWarps * kKeysPerWarp;  // keys per split block

// PER FP16 elements (PER = head_dim / 32) of one row, lane-contiguous.
template <int PER>
__device__ __forceinline__ void load_per(const uint16_t* p, float (&x)[PER]) {
    if constexpr (PER == 2) {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
        x[0] = f16_bits_to_f32(static_cast<uint16_t>(v & 0xFFFFu));
        x[1] = f16_bits_to_f32(static_cast<uint16_t>(v >> 16));
    } else if constexpr (PER == 4) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        const uint32_t w[2] = {v.x, v.y};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            x[2 * e] = f16_bits_to_f32(static_cast<uint16_t>(w[e] & 0xFFFFu));
            x[2 * e + 1] = f16_bits_to_f32(static_cast<uint16_t>(w[e] >> 16));
        }
    } else if constexpr (PER == 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            x[2 * e] = f16_bits_to_f32(static_cast<uint16_t>(w[e] & 0xFFFFu));
            x[2 * e + 1] = f16_bits_to_f32(static_cast<uint16_t>(w[e] >> 16));
        }
    } else {
#pragma unroll
        for (int e = 0; e < PER; ++e) x[e] = f16_bits_to_f32(p[e]);
    }
}

// RoPE of one head held lane-contiguously (lane l: elements l*PER .. +PER-1):
// element i < D/2 pairs with i + D/2, which lane l ^ 16 holds.  Same
// arithmetic and rounding as rope_append_kernel; `bits` gets the FP16 result,
// `x` its value.
template <int PER>
__device__ __forceinline__ void rope_lane_f16(float (&x)[PER], uint16_t (&bits)[PER], int lane, const float* cos_row,
                                              const float* sin_row) {
    const int i0 = (lane & 15) * PER;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const float other = __shfl_xor_sync(0xFFFFFFFFu, x[e], 16);
        const float c = cos_row[i0 + e], sn = sin_row[i0 + e];
        if (lane < 16)
            bits[e] = f32_to_f16_bits(__fsub_rn(__fmul_rn(x[e], c), __fmul_rn(other, sn)));
        else
            bits[e] = f32_to_f16_bits(__fadd_rn(__fmul_rn(other, sn), __fmul_rn(x[e], c)));
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) x[e] = f16_bits_to_f32(bits[e]);
}

constexpr int kMergeChunk = 128;  // splits merged per pass (one per thread)
constexpr int kMergeBatch = 32;   // up to this many splits are merged from one batch of loads

// Decode attention for one query row (cpu_backend.cpp:171-290 with q_len = 1)
// with the step's RoPE and KV-cache append folded in (qwen_model.cpp:162-205).
// Block (h, split) covers keys [32 split, 32 split + 32) of local kv head g:
// it rotates its raw query head from the q|k|v projection in registers; the
// current position's key and value come straight from the projection (the key
// rotated the same way), and the first local query head of each kv head
// writes them to the cache at that position -- no block of this launch reads
// that slot from the cache.  Each warp loads its <= 8 keys' K and V rows at
// once, scores them (q.k as a warp tree sum, times scale) and keeps (max, sum
// of exp, sum of exp * v).  The block merges its warps and writes the split's
// partial to `part`; the last split block of the head to arrive merges every
// split in split order (per-split weights exp(m_s - M) computed once) and
// writes out = fp16(acc * (1 / sum)).  kv_len = state position + 1.
template <int PER>
__global__ void __launch_bounds__(kAttnWarps * 32)
    attn_decode_kernel(const uint16_t* __restrict__ qkv, int nh, int nkv, uint16_t* __restrict__ kc,
                       uint16_t* __restrict__ vc, uint16_t* __restrict__ out, int group, int h0, int g0,
                       int64_t max_seq, float scale, const DecState* st, float* part, int* counters,
                       const float* __restrict__ cos_t, const float* __restrict__ sin_t) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr int D = PER * 32;
    __shared__ float sm_m[kAttnWarps], sm_l[kAttnWarps];
    __shared__ float sm_acc[kAttnWarps][D];
    __shared__ float sm_w[kMergeChunk], sm_ls[kMergeChunk], sm_red[kAttnWarps];
    __shared__ int sm_last;
    // Local query head h is global head h0 + h; its kv head, local index g.
    const int h = blockIdx.x, sp = blockIdx.y, nsplit = gridDim.y;
    const int g = (h0 + h) / group - g0;
    const bool writer = h == 0 || (h0 + h - 1) / group - g0 != g;  // first local head of kv head g
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t pos = st->pos;
    int64_t kv_len = pos + 1;
    if (kv_len > max_seq) kv_len = max_seq;
    const float* cos_row = cos_t + pos * (D / 2);
    const float* sin_row = sin_t + pos * (D / 2);
    const int64_t kw = static_cast<int64_t>(sp) * kSplitKeys + warp * kKeysPerWarp;
    const int nk = kv_len - kw <= 0 ? 0 : (kv_len - kw >= kKeysPerWarp ? kKeysPerWarp : static_cast<int>(kv_len - kw));
    const int icur = pos < max_seq && pos >= kw && pos < kw + nk ? static_cast<int>(pos - kw) : -1;  // warp-uniform
    // The cached keys and values first: they depend on nothing in this
    // launch, so their latency overlaps the query's load and rotation.
    const uint16_t* kb = kc + (static_cast<int64_t>(g) * max_seq + kw) * D + lane * PER;
    const uint16_t* vb = vc + (static_cast<int64_t>(g) * max_seq + kw) * D + lane * PER;
    float kx[kKeysPerWarp][PER], vx[kKeysPerWarp][PER];
#pragma unroll
    for (int i = 0; i < kKeysPerWarp; ++i)
        if (i < nk && i != icur) {
            load_per<PER>(kb + i * D, kx[i]);
            load_per<PER>(vb + i * D, vx[i]);
        }
    float qv[PER];
    uint16_t qb[PER];
    load_per<PER>(qkv + static_cast<int64_t>(h) * D + lane * PER, qv);
    rope_lane_f16<PER>(qv, qb, lane, cos_row, sin_row);
    if (icur >= 0) {
        const uint16_t* kr = qkv + static_cast<int64_t>(nh + g) * D + lane * PER;
        const uint16_t* vr = qkv + static_cast<int64_t>(nh + nkv + g) * D + lane * PER;
        float kcur[PER], vcur[PER];
        uint16_t kbits[PER];
        load_per<PER>(kr, kcur);
        load_per<PER>(vr, vcur);
        rope_lane_f16<PER>(kcur, kbits, lane, cos_row, sin_row);
#pragma unroll
        for (int i = 0; i < kKeysPerWarp; ++i)
            if (i == icur) {
#pragma unroll
                for (int e = 0; e < PER; ++e) {
                    kx[i][e] = kcur[e];
                    vx[i][e] = vcur[e];
                }
            }
        if (writer) {
            const int64_t slot = (static_cast<int64_t>(g) * max_seq + pos) * D + lane * PER;
#pragma unroll
            for (int e = 0; e < PER; ++e) {
                kc[slot + e] = kbits[e];
                vc[slot + e] = vr[e];
            }
        }
    }
    float sc[kKeysPerWarp];
#pragma unroll
    for (int i = 0; i < kKeysPerWarp; ++i) {
        float d = 0.0f;
#pragma unroll
        for (int e = 0; e < PER; ++e) d = __fadd_rn(d, __fmul_rn(qv[e], i < nk ? kx[i][e] : 0.0f));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d = __fadd_rn(d, __shfl_xor_sync(0xFFFFFFFFu, d, o));
        sc[i] = i < nk ? __fmul_rn(d, scale) : -INFINITY;
    }
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kKeysPerWarp; ++i) m = fmaxf(m, sc[i]);
    float l = 0.0f, acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.0f;
    if (nk > 0) {
#pragma unroll
        for (int i = 0; i < kKeysPerWarp; ++i)
            if (i < nk) {
                const float p = expf(__fsub_rn(sc[i], m));
                l = __fadd_rn(l, p);
#pragma unroll
                for (int e = 0; e < PER; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(p, vx[i][e]));
            }
    }
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) sm_acc[warp][lane * PER + e] = acc[e];
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w]);
    float* dst = part + (static_cast<int64_t>(h) * nsplit + sp) * (D + 2);
    if (threadIdx.x == 0) {
        float L = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w)
            if (sm_m[w] != -INFINITY) L = __fadd_rn(L, __fmul_rn(sm_l[w], expf(__fsub_rn(sm_m[w], M))));
        dst[0] = M;
        dst[1] = L;
    }
    for (int d = threadIdx.x; d < D; d += kAttnWarps * 32) {
        float A = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w)
            if (sm_m[w] != -INFINITY) A = __fadd_rn(A, __fmul_rn(sm_acc[w][d], expf(__fsub_rn(sm_m[w], M))));
        dst[2 + d] = A;
    }
    // Count this split in: the block's partial writes are ordered before
    // thread 0's acquire-release atomic by the barrier; the last split's
    // acquire (shared by the barrier after it) makes every split visible.
    __syncthreads();
    if (threadIdx.x == 0) {
        int prev;
        asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(prev) : "l"(counters + h) : "memory");
        sm_last = prev == nsplit - 1;
        if (sm_last) counters[h] = 0;
    }
    __syncthreads();
    if (!sm_last) return;
    const float* ph = part + static_cast<int64_t>(h) * nsplit * (D + 2);
    const int used = static_cast<int>((kv_len + kSplitKeys - 1) / kSplitKeys);  // splits holding keys
    constexpr int kJ = (D + kAttnWarps * 32 - 1) / (kAttnWarps * 32);  // output elements per thread
    if (used <= kMergeBatch) {
        // Up to 1024 keys: one batch of loads -- every thread's columns of
        // every split, and split s's maximum and sum of exp by thread s --
        // before the maximum is reduced; then the same arithmetic in the same
        // order as the chunked merge below, with no further global loads.
        float av[kJ][kMergeBatch];
#pragma unroll
        for (int s2 = 0; s2 < kMergeBatch; ++s2)
            if (s2 < used)
#pragma unroll
                for (int j = 0; j < kJ; ++j) {
                    const int d = threadIdx.x + j * kAttnWarps * 32;
                    if (d < D) av[j][s2] = __ldcg(ph + s2 * (D + 2) + 2 + d);
                }
        float my_m = -INFINITY, my_l = 0.0f;
        if (static_cast<int>(threadIdx.x) < used) {
            my_m = __ldcg(ph + threadIdx.x * (D + 2));
            my_l = __ldcg(ph + threadIdx.x * (D + 2) + 1);
        }
        float mb = my_m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, o));
        if (lane == 0) sm_red[warp] = mb;
        __syncthreads();
        float MMb = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) MMb = fmaxf(MMb, sm_red[w]);
        if (static_cast<int>(threadIdx.x) < used) {
            sm_w[threadIdx.x] = expf(__fsub_rn(my_m, MMb));
            sm_ls[threadIdx.x] = my_l;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float LLb = 0.0f;
            for (int s2 = 0; s2 < used; ++s2) LLb = __fadd_rn(LLb, __fmul_rn(sm_ls[s2], sm_w[s2]));
            sm_red[0] = __fdiv_rn(1.0f, LLb);  // every warp read its maximum above
        }
        float Ab[kJ];
#pragma unroll
        for (int j = 0; j < kJ; ++j) {
            Ab[j] = 0.0f;
#pragma unroll
            for (int s2 = 0; s2 < kMergeBatch; ++s2)
                if (s2 < used) Ab[j] = __fadd_rn(Ab[j], __fmul_rn(av[j][s2], sm_w[s2]));
        }
        __syncthreads();
        const float invb = sm_red[0];
#pragma unroll
        for (int j = 0; j < kJ; ++j) {
            const int d = threadIdx.x + j * kAttnWarps * 32;
            if (d < D) out[static_cast<int64_t>(h) * D + d] = f32_to_f16_bits(__fmul_rn(Ab[j], invb));
        }
        return;
    }
    // M = max over the splits' maxima (order-free).
    float mx = -INFINITY;
    for (int s2 = threadIdx.x; s2 < used; s2 += kAttnWarps * 32) mx = fmaxf(mx, __ldcg(ph + s2 * (D + 2)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (lane == 0) sm_red[warp] = mx;
    __syncthreads();
    float MM = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) MM = fmaxf(MM, sm_red[w]);
    // LL and every output element summed in split order, chunk by chunk, with
    // each split's weight exp(m_s - MM) computed once.
    float LL = 0.0f;
    float A[(D + kAttnWarps * 32 - 1) / (kAttnWarps * 32)];
#pragma unroll
    for (int j = 0; j < (D + kAttnWarps * 32 - 1) / (kAttnWarps * 32); ++j) A[j] = 0.0f;
    for (int c0 = 0; c0 < used; c0 += kMergeChunk) {
        const int cn = used - c0 < kMergeChunk ? used - c0 : kMergeChunk;
        __syncthreads();  // the previous chunk's weights are no longer read
        if (threadIdx.x < cn) {
            const float* q2 = ph + static_cast<int64_t>(c0 + threadIdx.x) * (D + 2);
            sm_w[threadIdx.x] = expf(__fsub_rn(__ldcg(q2), MM));
            sm_ls[threadIdx.x] = __ldcg(q2 + 1);
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int s2 = 0; s2 < cn; ++s2) LL = __fadd_rn(LL, __fmul_rn(sm_ls[s2], sm_w[s2]));
#pragma unroll
        for (int j = 0; j < (D + kAttnWarps * 32 - 1) / (kAttnWarps * 32); ++j) {
            const int d = threadIdx.x + j * kAttnWarps * 32;
            if (d >= D) break;
            const float* col = ph + static_cast<int64_t>(c0) * (D + 2) + 2 + d;
            int s2 = 0;
            for (; s2 + 8 <= cn; s2 += 8) {
                float v8[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v8[u] = __ldcg(col + (s2 + u) * (D + 2));
#pragma unroll
                for (int u = 0; u < 8; ++u) A[j] = __fadd_rn(A[j], __fmul_rn(v8[u], sm_w[s2 + u]));
            }
            for (; s2 < cn; ++s2) A[j] = __fadd_rn(A[j], __fmul_rn(__ldcg(col + s2 * (D + 2)), sm_w[s2]));
        }
    }
    if (threadIdx.x == 0) sm_red[0] = __fdiv_rn(1.0f, LL);
    __syncthreads();
    const float inv = sm_red[0];
#pragma unroll
    for (int j = 0; j < (D + kAttnWarps * 32 - 1) / (kAttnWarps * 32); ++j) {
        const int d = threadIdx.x + j * kAttnWarps * 32;
        if (d < D) out[static_cast<int64_t>(h) * D + d] = f32_to_f16_bits(__fmul_rn(A[j], inv));
    }
}

template <int PER>
cudaError_t launch_attn_decode(dim3 grid, cudaStream_t s, const uint16_t* qkv, int nh, int nkv, uint16_t* kc,
                               uint16_t* vc, uint16_t* out, int group, int h0, int g0, int64_t max_seq, float scale,
                               const DecState* st, float* part, int* counters, const float* cos_t,
                               const float* sin_t) {
    return launch_pdl(attn_decode_kernel<PER>, grid, dim3(kAttnWarps * 32), 0, s, qkv, nh, nkv, kc, vc, out, group, h0,
                      g0, max_seq, scale, st, part, counters, cos_t, sin_t);
}

// Decode attention with the step's RoPE and KV append (see attn_decode_kernel).
cudaError_t attn_decode(int D, dim3 grid, cudaStream_t s, const uint16_t* qkv, int nh, int nkv, uint16_t* kc,
                        uint16_t* vc, uint16_t* out, int group, int h0, int g0, int64_t max_seq, float scale,
                        const DecState* st, float* part, int* counters, const float* cos_t, const float* sin_t) {
#define MRT_ATTN_CASE(P)                                                                                      \
    case P:                                                                                                   \
        return launch_attn_decode<P>(grid, s, qkv, nh, nkv, kc, vc, out, group, h0, g0, max_seq, scale, st, \
                                     part, counters, cos_t, sin_t);
    switch (D / 32) {
        MRT_ATTN_CASE(1)
        MRT_ATTN_CASE(2)
        MRT_ATTN_CASE(3)
        MRT_ATTN_CASE(4)
        MRT_ATTN_CASE(5)
        MRT_ATTN_CASE(6)
        MRT_ATTN_CASE(7)
        MRT_ATTN_CASE(8)
        default: return cudaErrorInvalidValue;
    }
#undef MRT_ATTN_CASE
}

constexpr int kPfTile = 64;    // queries per block and keys per step
constexpr int kPfThreads = 256; // 16 query groups x 16 key (or dimension) groups

// Causal prefill attention (cpu_backend.cpp:171-290 for q_len = S rows that
// follow pos0 cached positions): block (h, tile) holds 64 queries of head h in
// shared memory and walks key tiles of 64 from kv head h / group; thread
// (tq, tk) scores queries 4 tq..+3 against keys 4 tk..+3, keeps the running
// max and sum of exp for its rows (the 16 threads of a row share them through
// shuffles) and accumulates dimensions tk * DPT..+DPT of the output.  Query q
// sees keys <= pos0 + q.  out row s = fp16(acc * (1 / sum)) at [s, h, :].
template <int DPT>
__global__ void __launch_bounds__(kPfThreads)
    attn_prefill_kernel(const uint16_t* __restrict__ qkv, int64_t ldq, int64_t S, int64_t pos0,
                        const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc, int64_t max_seq,
                        uint16_t* __restrict__ out, int64_t ldo, int group, int h0, int g0, float scale) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr int D = DPT * 16;
    constexpr int LD = D + 1;
    extern __shared__ float pf_smem[];
    float* Qs = pf_smem;                    // [64][LD]
    float* Ks = Qs + kPfTile * LD;          // [64][LD]
    float* Vs = Ks + kPfTile * LD;          // [64][LD]
    float* Ps = Vs + kPfTile * LD;          // [64][65]
    const int h = blockIdx.x, g = (h0 + h) / group - g0;  // local query head, local kv head
    const int64_t q0 = static_cast<int64_t>(blockIdx.y) * kPfTile;
    const int tid = threadIdx.x, tq = tid >> 4, tk = tid & 15;
    for (int e = tid; e < kPfTile * D; e += kPfThreads) {
        const int r = e / D, c = e % D;
        const int64_t s = q0 + r;
        Qs[r * LD + c] = s < S ? f16_bits_to_f32(qkv[s * ldq + static_cast<int64_t>(h) * D + c]) : 0.0f;
    }
    float m[4], l[4], o[4][DPT];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < DPT; ++j) o[i][j] = 0.0f;
    }
    const int64_t q_last = (q0 + kPfTile < S ? q0 + kPfTile : S) - 1;
    const int64_t k_end = pos0 + q_last + 1;  // keys this tile can see
    const uint16_t* kb = kc + static_cast<int64_t>(g) * max_seq * D;
    const uint16_t* vb = vc + static_cast<int64_t>(g) * max_seq * D;
    for (int64_t k0 = 0; k0 < k_end; k0 += kPfTile) {
        __syncthreads();  // the previous tile's K, V and P are consumed
        for (int e = tid; e < kPfTile * D; e += kPfThreads) {
            const int r = e / D, c = e % D;
            const int64_t kk = k0 + r;
            const bool in = kk < k_end;
            Ks[r * LD + c] = in ? f16_bits_to_f32(kb[kk * D + c]) : 0.0f;
            Vs[r * LD + c] = in ? f16_bits_to_f32(vb[kk * D + c]) : 0.0f;
        }
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.0f;
        for (int d = 0; d < D; ++d) {
            float qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = Qs[(tq * 4 + i) * LD + d];
#pragma unroll
            for (int j = 0; j < 4; ++j) kv[j] = Ks[(tk * 4 + j) * LD + d];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) sc[i][j] = __fadd_rn(sc[i][j], __fmul_rn(qv[i], kv[j]));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t qpos = pos0 + q0 + tq * 4 + i;
            float rmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t kk = k0 + tk * 4 + j;
                sc[i][j] = (kk <= qpos && kk < k_end) ? __fmul_rn(sc[i][j], scale) : -INFINITY;
                rmax = fmaxf(rmax, sc[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xFFFFFFFFu, rmax, off));
            const float m_new = fmaxf(m[i], rmax);
            // Rows past S (or with no visible key in this tile yet) stay at -inf.
            const float corr = m_new == -INFINITY ? 1.0f : expf(__fsub_rn(m[i], m_new));
            float psum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p = sc[i][j] == -INFINITY ? 0.0f : expf(__fsub_rn(sc[i][j], m_new));
                Ps[(tq * 4 + i) * (kPfTile + 1) + tk * 4 + j] = p;
                psum = __fadd_rn(psum, p);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) psum = __fadd_rn(psum, __shfl_xor_sync(0xFFFFFFFFu, psum, off));
            l[i] = __fadd_rn(__fmul_rn(l[i], corr), psum);
#pragma unroll
            for (int j = 0; j < DPT; ++j) o[i][j] = __fmul_rn(o[i][j], corr);
            m[i] = m_new;
        }
        __syncthreads();
        for (int k = 0; k < kPfTile; ++k) {
            float vv[DPT];
#pragma unroll
            for (int j = 0; j < DPT; ++j) vv[j] = Vs[k * LD + tk * DPT + j];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float p = Ps[(tq * 4 + i) * (kPfTile + 1) + k];
#pragma unroll
                for (int j = 0; j < DPT; ++j) o[i][j] = __fadd_rn(o[i][j], __fmul_rn(p, vv[j]));
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t s = q0 + tq * 4 + i;
        if (s >= S) continue;
        const float inv = __fdiv_rn(1.0f, l[i]);
#pragma unroll
        for (int j = 0; j < DPT; ++j)
            out[s * ldo + static_cast<int64_t>(h) * D + tk * DPT + j] = f32_to_f16_bits(__fmul_rn(o[i][j], inv));
    }
}

size_t prefill_smem(int D) { return static_cast<size_t>(3 * kPfTile * (D + 1) + kPfTile * (kPfTile + 1)) * 4; }

template <int DPT>
cudaError_t launch_attn_prefill_t(int heads, int64_t S, cudaStream_t s, const uint16_t* qkv, int64_t ldq, int64_t pos0,
                                  const uint16_t* kc, const uint16_t* vc, int64_t max_seq, uint16_t* out, int64_t ldo,
                                  int group, int h0, int g0, float scale) {
    const size_t smem = prefill_smem(DPT * 16);
    static bool set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel<DPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        set[dev] = true;
    }
    const dim3 grid(static_cast<unsigned>(heads), static_cast<unsigned>((S + kPfTile - 1) / kPfTile));
    return launch_pdl(attn_prefill_kernel<DPT>, grid, dim3(kPfThreads), smem, s, qkv, ldq, S, pos0, kc, vc, max_seq,
                      out, ldo, group, h0, g0, scale);
}

cudaError_t attn_prefill(int D, int heads, int64_t S, cudaStream_t s, const uint16_t* qkv, int64_t ldq, int64_t pos0,
                         const uint16_t* kc, const uint16_t* vc, int64_t max_seq, uint16_t* out, int64_t ldo, int group,
                         int h0, int g0, float scale) {
    switch (D) {
        case 32: return launch_attn_prefill_t<2>(heads, S, s, qkv, ldq, pos0, kc, vc, max_seq, out, ldo, group, h0, g0, scale);
        case 64: return launch_attn_prefill_t<4>(heads, S, s, qkv, ldq, pos0, kc, vc, max_seq, out, ldo, group, h0, g0, scale);
        case 96: return launch_attn_prefill_t<6>(heads, S, s, qkv, ldq, pos0, kc, vc, max_seq, out, ldo, group, h0, g0, scale);
        case 128: return launch_attn_prefill_t<8>(heads, S, s, qkv, ldq, pos0, kc, vc, max_seq, out, ldo, group, h0, g0, scale);
        case 160: return launch_attn_prefill_t<10>(heads, S, s, qkv, ldq, pos0, kc, vc, max_seq, out, ldo, group, h0, g0, scale);
        case 192: return launch_attn_prefill_t<12>(heads, S, s, qkv, ldq, pos0, kc, vc, max_seq, out, ldo, group, h0, g0, scale);
        case 224: return launch_attn_prefill_t<14>(heads, S, s, qkv, ldq, pos0, kc, vc, max_seq, out, ldo, group, h0, g0, scale);
        case 256: return launch_attn_prefill_t<16>(heads, S, s, qkv, ldq, pos0, kc, vc, max_seq, out, ldo, group, h0, g0, scale);
        default: return cudaErrorInvalidValue;
    }
}

constexpr int kMaxRanks = 8;

// Where every rank's exchange region is, as this rank sees it (own region
// included): the FP32 partial buffer of one call site and the flag array
// (one 64-bit slot per source rank).
struct PeerArgs {
    const float* buf[kMaxRanks];
    unsigned long long* flags[kMaxRanks];
    int rank, world;
};

// Row-parallel output finished across GPUs, fused with the residual add and
// RMSNorm that consume it (qwen_model.cpp:321-332).  Every rank's GEMM left
// its FP32 partial rows in its own exchange buffer.  Block 0 publishes this
// rank's epoch to every peer (system-scope release stores, one thread per
// peer); each block waits (bounded, 2 s, one polling thread per peer) for
// every peer's epoch, then reads all W partials of its row
// over NVLink and sums them in rank order -- the same order on every rank, so
// every rank holds bit-identical rows -- rounds once to FP16 (the projection's
// output), and continues as add_norm_kernel: out = fp16(a + p), normed =
// RMSNorm(out).  Rows row0 .. row0 + gridDim.x - 1.  The epoch of call c of a
// forward is *epoch_base + c + 1; epoch_base advances by the calls per forward.
// A peer that never arrives leaves its partial out and raises kErrPeerWait.
template <bool kPre>
__global__ void __launch_bounds__(kNT)
    ar_add_norm_kernel(const PeerArgs pa, int64_t row0, const uint16_t* __restrict__ a, uint16_t* __restrict__ out,
                       int64_t H, const void* __restrict__ w, int wdt, float eps, uint16_t* __restrict__ normed,
                       const unsigned long long* epoch_base, int call, int* err) {
    griddep_launch_dependents();
    float g[kNormVec][8];
    if constexpr (kPre) load_gains(w, wdt, static_cast<int>(H / 8), g);
    griddep_wait();
    __shared__ float red[kNT / 32];
    __shared__ unsigned arrived;  // bit q: rank q's partial may be read
    const unsigned long long epoch = *epoch_base + static_cast<unsigned long long>(call) + 1ull;
    if (threadIdx.x == 0) arrived = 1u << pa.rank;
    __syncthreads();
    // Thread q talks to peer q, so the world's publishes and polls overlap
    // instead of queueing behind one thread's system-scope fences.
    const int q = static_cast<int>(threadIdx.x);
    if (q < pa.world && q != pa.rank) {
        // This rank's partial (written by the previous kernel) is released
        // to peer q with the epoch.
        if (blockIdx.x == 0) st_release_sys(pa.flags[q] + pa.rank, epoch);
        const unsigned long long t0 = global_ns();
        while (true) {
            if (ld_acquire_sys(pa.flags[pa.rank] + q) >= epoch) {
                atomicOr(&arrived, 1u << q);
                break;
            }
            if (global_ns() - t0 > kWaitLimitNs) {
                raise_error(err, kErrPeerWait);
                break;
            }
        }
    }
    __syncthreads();
    const unsigned got = arrived;
    const int64_t row = row0 + blockIdx.x;
    const int nv = static_cast<int>(H / 8);
    float x[kNormVec][8];
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int i = static_cast<int>(threadIdx.x) + j * kNT;
        if (i >= nv) continue;
        const int64_t e0 = row * H + static_cast<int64_t>(i) * 8;
        float4 p0[kMaxRanks], p1[kMaxRanks];
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
            if (q < pa.world && (got >> q & 1u)) {
                p0[q] = __ldcg(reinterpret_cast<const float4*>(pa.buf[q] + e0));
                p1[q] = __ldcg(reinterpret_cast<const float4*>(pa.buf[q] + e0 + 4));
            }
        float acc[8];
        bool first = true;
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q) {
            if (!(q < pa.world && (got >> q & 1u))) continue;
            const float v[8] = {p0[q].x, p0[q].y, p0[q].z, p0[q].w, p1[q].x, p1[q].y, p1[q].z, p1[q].w};
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = first ? v[e] : __fadd_rn(acc[e], v[e]);
            first = false;
        }
        const uint4 va = ld16(a + e0);
        float fa[8];
        unpack8(va, fa);
        uint16_t h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float pv = f16_bits_to_f32(f32_to_f16_bits(acc[e]));  // the projection's FP16 output
            h[e] = f32_to_f16_bits(__fadd_rn(fa[e], pv));
            x[j][e] = f16_bits_to_f32(h[e]);
        }
        *reinterpret_cast<uint4*>(out + e0) =
            make_uint4(pack2(h[0], h[1]), pack2(h[2], h[3]), pack2(h[4], h[5]), pack2(h[6], h[7]));
    }
    norm_vecs<kPre>(x, nv, H, g, w, wdt, eps, normed + row * H, red);
}

// After the greedy pick of a forward over `rows` tokens: record the token and
// move the state to the next position.
// The cross-GPU all-reduce epoch base (when there is one) advances by the
// number of all-reduce calls a forward makes.
__global__ void advance_kernel(const int64_t* idx, DecState* st, int32_t* tokens, int64_t max_tokens, int rows,
                               unsigned long long* epoch_base, int calls) {
    griddep_launch_dependents();
    griddep_wait();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int32_t t = static_cast<int32_t>(idx[0]);
    if (st->step < max_tokens) tokens[st->step] = t;
    st->step += 1;
    st->token = t;
    st->pos += rows;
    if (epoch_base != nullptr) *epoch_base += static_cast<unsigned long long>(calls);
}

}  // namespace
}  // namespace mrt

using namespace mrt;

namespace {

struct DecLayer {
    mrt_weight qkv = nullptr, o = nullptr, gateup = nullptr, down = nullptr;
    void* ln1 = nullptr;
    int ln1_dt = MRT_FP16;
    void* ln2 = nullptr;
    int ln2_dt = MRT_FP16;
    bool qkv_bias = false;
    // FP16 staging of the fused weights until every part has arrived.
    uint16_t* st_qkv = nullptr;
    uint32_t qkv_have = 0;  // bit 0 q, 1 k, 2 v
    uint16_t* st_bias = nullptr;
    uint32_t bias_have = 0;
    uint16_t* st_gu = nullptr;
    uint32_t gu_have = 0;  // bit 0 gate, 1 up
};

}  // namespace

struct mrt_decoder_s {
    int device = 0;
    mrt_decoder_config cfg{};
    int64_t H = 0, D = 0, heads = 0, kvh = 0, I = 0, V = 0, L = 0, max_seq = 0;
    // Tensor parallelism (world 1 without a handle): this rank's query heads
    // [h0, h0 + nh), kv heads [g0, g0 + nkv), intermediate columns [i0, i1) and
    // vocabulary rows [v0, v1); n_qkv = local q|k|v rows.
    mrt_tp tp = nullptr;
    int rank = 0, world = 1;
    int64_t h0 = 0, nh = 0, g0 = 0, nkv = 0, i0 = 0, i1 = 0, v0 = 0, v1 = 0, n_qkv = 0;
    std::vector<DecLayer> layers;
    uint16_t* embed = nullptr;  // [V, H] FP16 row-major
    mrt_weight lm_head = nullptr;
    void* norm = nullptr;
    int norm_dt = MRT_FP16;
    bool ready = false;
    // activations and state (allocated by finalize)
    uint16_t *x = nullptr, *r = nullptr, *p = nullptr, *normed = nullptr, *qkv = nullptr, *attn = nullptr,
             *act = nullptr, *logits = nullptr, *kc = nullptr, *vc = nullptr;
    float *cos_t = nullptr, *sin_t = nullptr, *part = nullptr, *am_val = nullptr;
    int* counters = nullptr;
    int64_t* am_idx = nullptr;
    void* am_scratch = nullptr;
    DecState* state = nullptr;
    int32_t* tokens = nullptr;
    int64_t tokens_cap = 0;
    int32_t* ids = nullptr;
    int64_t ids_cap = 0;
    float* partial = nullptr;   // FP32 row-parallel partials [max_seq, H] (world > 1, NCCL path)
    int64_t* am_gidx = nullptr; // the greedy pick across vocabulary shards
    // Peer all-reduce (world > 1): this rank's exchange region (flags, then
    // one FP32 partial buffer per row-parallel call site), the peers' regions
    // mapped through CUDA IPC, and the device epoch counter.
    bool p2p = false;
    void* xreg = nullptr;
    void* peer_reg[kMaxRanks] = {};
    PeerArgs pa[2] = {};
    unsigned long long* ar_epoch = nullptr;
    // Persistent decode step (one launch per token) when the shapes allow it.
    bool fused_step = false;
    int step_grid = 0;
    StepArgs step{};
    StepLayer* step_layers = nullptr;
    int nsplit = 1;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
};

namespace {

int dec_alloc(mrt_decoder d, void** p, size_t bytes, const char* what) {
    cudaError_t e = cudaMalloc(p, bytes < 16 ? 16 : bytes);
    if (e != cudaSuccess) return cuda_error(e, what);
    d->allocs.push_back(*p);
    return MRT_OK;
}

void dec_release(mrt_decoder d, void* p) {
    if (p == nullptr) return;
    for (auto& a : d->allocs)
        if (a == p) a = nullptr;
    cudaFree(p);
}

size_t es_of(int dt) { return dt == MRT_FP32 ? 4 : 2; }

// n elements of a host or device source of dtype dt into FP16 device memory,
// rounded once by the reference's converter rule.
int to_f16(const void* src, int dt, bool on_dev, int64_t n, uint16_t* dst, cudaStream_t s) {
    if (dt == MRT_FP16) {
        cudaError_t e = cudaMemcpyAsync(dst, src, static_cast<size_t>(n) * 2,
                                        on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        return e == cudaSuccess ? MRT_OK : cuda_error(e, "copying a decoder tensor");
    }
    const void* dsrc = src;
    void* tmp = nullptr;
    if (!on_dev) {
        cudaError_t e = cudaMalloc(&tmp, static_cast<size_t>(n) * es_of(dt));
        if (e == cudaSuccess) e = cudaMemcpy(tmp, src, static_cast<size_t>(n) * es_of(dt), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            if (tmp) cudaFree(tmp);
            return cuda_error(e, "staging a decoder tensor");
        }
        dsrc = tmp;
    }
    int rc = mrt_convert(dsrc, dt, dst, MRT_FP16, n, s);
    cudaError_t e = cudaStreamSynchronize(s);
    if (tmp) cudaFree(tmp);
    if (rc != MRT_OK) return rc;
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "converting a decoder tensor");
}

// A copy of a small tensor in its own dtype (RMSNorm gains).
int to_native(mrt_decoder d, const void* src, int dt, bool on_dev, int64_t n, void** out) {
    int rc = dec_alloc(d, out, static_cast<size_t>(n) * es_of(dt), "allocating a norm weight");
    if (rc != MRT_OK) return rc;
    cudaError_t e = cudaMemcpy(*out, src, static_cast<size_t>(n) * es_of(dt),
                               on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "copying a norm weight");
}

int upload_f16(const uint16_t* dev, int64_t N, int64_t K, cudaStream_t s, mrt_weight* w) {
    return mrt_weight_upload(dev, MRT_FP16, 1, N, K, nullptr, 0, 0, K, s, w);
}

bool parse_layer(const std::string& name, int64_t* layer, std::string* suffix) {
    const std::string pre = "model.layers.";
    if (name.compare(0, pre.size(), pre) != 0) return false;
    size_t i = pre.size(), j = i;
    while (j < name.size() && name[j] >= '0' && name[j] <= '9') ++j;
    if (j == i || j >= name.size() || name[j] != '.') return false;
    *layer = std::stoll(name.substr(i, j - i));
    *suffix = name.substr(j + 1);
    return true;
}

}  // namespace

namespace {

// Query heads [h0, h0 + nh) and kv heads [g0, g0 + nkv) of `rank`: whole kv
// groups per rank when world divides the kv heads, else every kv head is
// replicated on world / kv_heads ranks that split its query heads.
bool head_split(int64_t heads, int64_t kvh, int world, int rank, int64_t* h0, int64_t* nh, int64_t* g0, int64_t* nkv) {
    const int64_t group = heads / kvh;
    if (world <= kvh) {
        if (kvh % world != 0) return false;
        *nkv = kvh / world;
        *g0 = rank * *nkv;
        *h0 = *g0 * group;
        *nh = *nkv * group;
        return true;
    }
    if (world % kvh != 0) return false;
    const int64_t R = world / kvh;  // ranks per kv head
    if (group < R) return false;
    const int64_t g = rank / R, j = rank % R;
    const int64_t a = group * j / R, b = group * (j + 1) / R;
    *g0 = g;
    *nkv = 1;
    *h0 = g * group + a;
    *nh = b - a;
    return true;
}

int dec_create(const mrt_decoder_config* cfg, mrt_tp tp, mrt_decoder* out) {
    clear_error();
    if (out == nullptr || cfg == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL config or out");
    *out = nullptr;
    const mrt_decoder_config& c = *cfg;
    if (c.vocab_size <= 0 || c.hidden_size <= 0 || c.num_layers <= 0 || c.num_attention_heads <= 0 ||
        c.num_kv_heads <= 0 || c.intermediate_size <= 0 || c.max_seq_len <= 0)
        return set_error(MRT_ERR_SHAPE, "decoder sizes must be positive");
    if (c.hidden_size % c.num_attention_heads != 0 || c.num_attention_heads % c.num_kv_heads != 0)
        return set_error(MRT_ERR_SHAPE, "hidden_size must split into heads and heads into kv groups");
    const int64_t D = c.hidden_size / c.num_attention_heads;
    if (D % 32 != 0 || D > 256) return set_error(MRT_ERR_UNSUPPORTED, "head_dim must be a multiple of 32, at most 256");
    if (c.hidden_size % 8 != 0 || c.intermediate_size % 8 != 0)
        return set_error(MRT_ERR_UNSUPPORTED, "hidden and intermediate sizes must be multiples of 8");
    if (c.hidden_size > 16384) return set_error(MRT_ERR_UNSUPPORTED, "hidden_size above 16384");
    if (c.max_seq_len > (int64_t{1} << 30)) return set_error(MRT_ERR_SHAPE, "max_seq_len too large");
    DevCtx* ctx = current_ctx();
    if (!ctx) return MRT_ERR_CUDA;
    mrt_decoder d = new mrt_decoder_s();
    d->device = ctx->device;
    d->cfg = c;
    d->H = c.hidden_size;
    d->D = D;
    d->heads = c.num_attention_heads;
    d->kvh = c.num_kv_heads;
    d->I = c.intermediate_size;
    d->V = c.vocab_size;
    d->L = c.num_layers;
    d->max_seq = c.max_seq_len;
    d->tp = tp;
    if (tp != nullptr) {
        int rc = tp_rank_world(tp, &d->rank, &d->world);
        if (rc != MRT_OK) {
            delete d;
            return rc;
        }
    }
    if (!head_split(d->heads, d->kvh, d->world, d->rank, &d->h0, &d->nh, &d->g0, &d->nkv)) {
        delete d;
        return set_error(MRT_ERR_UNSUPPORTED, "the attention heads do not split over " + std::to_string(d->world) +
                                                  " ranks (need world | kv_heads, or kv_heads | world <= heads)");
    }
    if (d->world > 1) {
        int rc = mrt_shard_cols(d->I, d->world, d->rank, &d->i0, &d->i1);
        if (rc != MRT_OK || (d->i1 - d->i0) % 8 != 0) {
            delete d;
            return rc != MRT_OK ? rc : set_error(MRT_ERR_UNSUPPORTED, "intermediate_size must split into multiples of 8");
        }
        d->v0 = d->V * d->rank / d->world;
        d->v1 = d->V * (d->rank + 1) / d->world;
    } else {
        d->i0 = 0;
        d->i1 = d->I;
        d->v0 = 0;
        d->v1 = d->V;
    }
    d->n_qkv = (d->nh + 2 * d->nkv) * D;
    d->layers.resize(static_cast<size_t>(d->L));
    cudaError_t e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete d;
        return cuda_error(e, "creating the decoder stream");
    }
    *out = d;
    return MRT_OK;
}

}  // namespace

namespace mrt {
int64_t decoder_layer_count(mrt_decoder d) { return d ? d->L : 0; }
}  // namespace mrt

extern "C" int mrt_decoder_create(const mrt_decoder_config* cfg, mrt_decoder* out) {
    return dec_create(cfg, nullptr, out);
}

extern "C" int mrt_decoder_create_tp(const mrt_decoder_config* cfg, mrt_tp tp, mrt_decoder* out) {
    if (tp == nullptr) {
        clear_error();
        return set_error(MRT_ERR_INVALID_ARG, "NULL tensor-parallel handle");
    }
    return dec_create(cfg, tp, out);
}

extern "C" int mrt_decoder_load(mrt_decoder d, const char* name_c, const void* src, int dt, int on_dev, int64_t rows,
                                int64_t cols) {
    clear_error();
    if (d == nullptr || name_c == nullptr || src == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    if (dt != MRT_FP16 && dt != MRT_BF16 && dt != MRT_FP32) return set_error(MRT_ERR_DTYPE, "dtype must be FP16, BF16 or FP32");
    if (d->ready) return set_error(MRT_ERR_INVALID_ARG, "the decoder has already run; load every tensor first");
    const std::string name(name_c);
    cudaStream_t s = d->stream;
    if (on_dev) {
        // The decoder's stream does not order after the caller's streams: let
        // every write of the source finish first (loading is one-time set-up).
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_error(e, "waiting for the source tensor");
    }
    const int64_t H = d->H, D = d->D, kv = d->kvh * D, I = d->I;
    auto shape = [&](int64_t r, int64_t k) -> int {
        if (rows != r || cols != k)
            return set_error(MRT_ERR_SHAPE, name + ": expected " + std::to_string(r) + " x " + std::to_string(k) + ", got " +
                                                std::to_string(rows) + " x " + std::to_string(cols));
        return MRT_OK;
    };
    int rc;
    if (name == "model.embed_tokens.weight") {
        if ((rc = shape(d->V, H)) != MRT_OK) return rc;
        if (d->embed == nullptr &&
            (rc = dec_alloc(d, reinterpret_cast<void**>(&d->embed), static_cast<size_t>(d->V * H) * 2, "allocating the embedding")) != MRT_OK)
            return rc;
        return to_f16(src, dt, on_dev != 0, d->V * H, d->embed, s);
    }
    if (name == "lm_head.weight") {
        if ((rc = shape(d->V, H)) != MRT_OK) return rc;
        if (d->lm_head) mrt_weight_free(d->lm_head);
        d->lm_head = nullptr;
        const int64_t vr[2] = {d->v0, d->v1};  // this rank's vocabulary rows
        return mrt_weight_upload(src, dt, on_dev, d->V, H, vr, 1, 0, H, s, &d->lm_head);
    }
    if (name == "model.norm.weight") {
        if ((rc = shape(H, 1)) != MRT_OK) return rc;
        dec_release(d, d->norm);
        d->norm_dt = dt;
        return to_native(d, src, dt, on_dev != 0, H, &d->norm);
    }
    int64_t li = -1;
    std::string suf;
    if (!parse_layer(name, &li, &suf) || li < 0 || li >= d->L)
        return set_error(MRT_ERR_INVALID_ARG, "unknown decoder tensor '" + name + "'");
    DecLayer& ly = d->layers[static_cast<size_t>(li)];
    if (suf == "input_layernorm.weight" || suf == "post_attention_layernorm.weight") {
        if ((rc = shape(H, 1)) != MRT_OK) return rc;
        const bool first = suf[0] == 'i';
        void*& p = first ? ly.ln1 : ly.ln2;
        dec_release(d, p);
        p = nullptr;
        (first ? ly.ln1_dt : ly.ln2_dt) = dt;
        return to_native(d, src, dt, on_dev != 0, H, &p);
    }
    if (suf == "self_attn.o_proj.weight" || suf == "mlp.down_proj.weight") {
        const bool o = suf[0] == 's';
        if ((rc = o ? shape(H, H) : shape(H, I)) != MRT_OK) return rc;
        mrt_weight& w = o ? ly.o : ly.down;
        if (w) mrt_weight_free(w);
        w = nullptr;
        // Row-parallel: this rank's input columns (its heads' attention
        // outputs for o, its intermediate columns for down).
        const int64_t k0 = o ? d->h0 * D : d->i0, k1 = o ? (d->h0 + d->nh) * D : d->i1;
        return mrt_weight_upload(src, dt, on_dev, H, o ? H : I, nullptr, 0, k0, k1, s, &w);
    }
    // q|k|v rows [0, H), [H, H + kv), [H + kv, H + 2 kv) of one weight.
    static const char* qkv_w[3] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight"};
    static const char* qkv_b[3] = {"self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias"};
    // Full part rows, this rank's first row within the part, its row count
    // and where those rows go in the local fused weight.
    const int64_t len[3] = {H, kv, kv};
    const int64_t first[3] = {d->h0 * D, d->g0 * D, d->g0 * D};
    const int64_t take[3] = {d->nh * D, d->nkv * D, d->nkv * D};
    const int64_t off[3] = {0, d->nh * D, (d->nh + d->nkv) * D};
    const char* csrc = static_cast<const char*>(src);
    for (int part = 0; part < 3; ++part) {
        if (suf == qkv_w[part]) {
            if ((rc = shape(len[part], H)) != MRT_OK) return rc;
            if (ly.qkv != nullptr) return set_error(MRT_ERR_INVALID_ARG, name + ": the fused q|k|v weight is already built");
            if (ly.st_qkv == nullptr &&
                (rc = dec_alloc(d, reinterpret_cast<void**>(&ly.st_qkv), static_cast<size_t>(d->n_qkv * H) * 2, "staging q|k|v")) != MRT_OK)
                return rc;
            if ((rc = to_f16(csrc + first[part] * H * static_cast<int64_t>(es_of(dt)), dt, on_dev != 0, take[part] * H,
                             ly.st_qkv + off[part] * H, s)) != MRT_OK)
                return rc;
            ly.qkv_have |= 1u << part;
            if (ly.qkv_have == 7u) {
                rc = upload_f16(ly.st_qkv, d->n_qkv, H, s, &ly.qkv);
                dec_release(d, ly.st_qkv);
                ly.st_qkv = nullptr;
                return rc;
            }
            return MRT_OK;
        }
        if (suf == qkv_b[part]) {
            if ((rc = shape(len[part], 1)) != MRT_OK) return rc;
            if (ly.st_bias == nullptr &&
                (rc = dec_alloc(d, reinterpret_cast<void**>(&ly.st_bias), static_cast<size_t>(d->n_qkv) * 2, "staging q|k|v biases")) != MRT_OK)
                return rc;
            // The reference converts biases to FP16 at load (qwen_model.cpp:93-101).
            if ((rc = to_f16(csrc + first[part] * static_cast<int64_t>(es_of(dt)), dt, on_dev != 0, take[part],
                             ly.st_bias + off[part], s)) != MRT_OK)
                return rc;
            ly.bias_have |= 1u << part;
            return MRT_OK;
        }
    }
    if (suf == "mlp.gate_proj.weight" || suf == "mlp.up_proj.weight") {
        const int part = suf[4] == 'g' ? 0 : 1;
        if ((rc = shape(I, H)) != MRT_OK) return rc;
        if (ly.gateup != nullptr) return set_error(MRT_ERR_INVALID_ARG, name + ": the fused gate|up weight is already built");
        const int64_t il = d->i1 - d->i0;  // this rank's intermediate rows
        if (ly.st_gu == nullptr &&
            (rc = dec_alloc(d, reinterpret_cast<void**>(&ly.st_gu), static_cast<size_t>(2 * il * H) * 2, "staging gate|up")) != MRT_OK)
            return rc;
        if ((rc = to_f16(static_cast<const char*>(src) + d->i0 * H * static_cast<int64_t>(es_of(dt)), dt, on_dev != 0, il * H,
                         ly.st_gu + part * il * H, s)) != MRT_OK)
            return rc;
        ly.gu_have |= 1u << part;
        if (ly.gu_have == 3u) {
            // Interleave the rows (row 2j = gate j, row 2j + 1 = up j) so
            // that each pair lands in one GEMM tile and the SwiGLU epilogue
            // sees both halves of it.
            uint16_t* inter = nullptr;
            if ((rc = dec_alloc(d, reinterpret_cast<void**>(&inter), static_cast<size_t>(2 * il * H) * 2,
                                "interleaving gate|up")) != MRT_OK)
                return rc;
            const size_t row = static_cast<size_t>(H) * 2;
            cudaError_t e = cudaMemcpy2DAsync(inter, 2 * row, ly.st_gu, row, row, static_cast<size_t>(il),
                                              cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(inter + H, 2 * row, ly.st_gu + il * H, row, row, static_cast<size_t>(il),
                                      cudaMemcpyDeviceToDevice, s);
            rc = e == cudaSuccess ? upload_f16(inter, 2 * il, H, s, &ly.gateup) : cuda_error(e, "interleaving gate|up");
            dec_release(d, inter);
            dec_release(d, ly.st_gu);
            ly.st_gu = nullptr;
            return rc;
        }
        return MRT_OK;
    }
    return set_error(MRT_ERR_INVALID_ARG, "unknown decoder tensor '" + name + "'");
}

namespace {

#define DEC_TRY(x)                   \
    do {                             \
        int rc_ = (x);               \
        if (rc_ != MRT_OK) return rc_; \
    } while (0)
#define DEC_CU(x, what)                                   \
    do {                                                  \
        cudaError_t e_ = (x);                             \
        if (e_ != cudaSuccess) return cuda_error(e_, what); \
    } while (0)

constexpr size_t kFlagBytes = 256;  // kMaxRanks 64-bit flags, padded

// Exchange regions for the peer all-reduce: every rank exports its region by
// CUDA IPC, the handles travel over the NCCL communicator, and each rank maps
// its peers' regions.  Any failure leaves p2p off (the NCCL path is used).
int dec_setup_p2p(mrt_decoder d) {
    // Each buffer holds a prefill's FP32 partial rows and, for the persistent
    // decode step, one [SMs][2][128] block of split-GEMV partials.
    const size_t buf_bytes = std::max(static_cast<size_t>(d->max_seq * d->H) * 4,
                                      static_cast<size_t>(current_ctx()->sms) * 256 * 4);
    const size_t region = kFlagBytes + 2 * buf_bytes;
    int rc = dec_alloc(d, &d->xreg, region, "the all-reduce exchange region");
    if (rc != MRT_OK) return rc;
    rc = dec_alloc(d, reinterpret_cast<void**>(&d->ar_epoch), 8, "the all-reduce epoch");
    if (rc != MRT_OK) return rc;
    cudaError_t e = cudaMemset(d->xreg, 0, kFlagBytes);
    if (e == cudaSuccess) e = cudaMemset(d->ar_epoch, 0, 8);
    if (e != cudaSuccess) return cuda_error(e, "clearing the exchange flags");
    cudaIpcMemHandle_t mine{};
    e = cudaIpcGetMemHandle(&mine, d->xreg);
    int ok = e == cudaSuccess ? 1 : 0;
    struct Rec {
        cudaIpcMemHandle_t h;
        int ok;
        int pad[15];
    } rec{mine, ok, {}};
    std::vector<Rec> all(static_cast<size_t>(d->world));
    rc = tp_allgather_host(d->tp, &rec, all.data(), sizeof(Rec));
    if (rc != MRT_OK) return rc;
    bool every = true;
    for (const Rec& r : all) every = every && r.ok;
    if (every) {
        for (int q = 0; q < d->world && every; ++q) {
            if (q == d->rank) {
                d->peer_reg[q] = d->xreg;
                continue;
            }
            e = cudaIpcOpenMemHandle(&d->peer_reg[q], all[static_cast<size_t>(q)].h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                d->peer_reg[q] = nullptr;
                every = false;
                cudaGetLastError();
            }
        }
    }
    // Every rank must agree before using the peer path.
    int mine_ok = every ? 1 : 0;
    std::vector<int> oks(static_cast<size_t>(d->world));
    rc = tp_allgather_host(d->tp, &mine_ok, oks.data(), sizeof(int));
    if (rc != MRT_OK) return rc;
    for (int v : oks) every = every && v;
    if (!every) {
        for (int q = 0; q < d->world; ++q)
            if (q != d->rank && d->peer_reg[q]) cudaIpcCloseMemHandle(d->peer_reg[q]);
        for (auto& r : d->peer_reg) r = nullptr;
        return MRT_OK;
    }
    for (int par = 0; par < 2; ++par) {
        d->pa[par].rank = d->rank;
        d->pa[par].world = d->world;
        for (int q = 0; q < d->world; ++q) {
            char* base = static_cast<char*>(d->peer_reg[q]);
            d->pa[par].buf[q] = reinterpret_cast<const float*>(base + kFlagBytes + par * buf_bytes);
            d->pa[par].flags[q] = reinterpret_cast<unsigned long long*>(base);
        }
    }
    d->p2p = true;
    return MRT_OK;
}

// The persistent decode-step kernel's tables and scratch.  It covers tiled
// weights, head_dim 64 / 128 / 256, at most 256 intermediate rows per CTA,
// and tensor parallelism over mapped peers; other decoders keep the per-op
// step.
int dec_setup_step(mrt_decoder d) {
    // Opt-in while the per-op step is faster on the 7B shape:
    // MRT_DECODE_STEP=persistent selects the persistent kernel.
    const char* sel = std::getenv("MRT_DECODE_STEP");
    if (sel == nullptr || std::string(sel) != "persistent") return MRT_OK;
    if (d->world > 1 && !d->p2p) return MRT_OK;
    const int grid = decode_step_grid();
    if (grid <= 0) return MRT_OK;
    const int64_t D = d->D, il = d->i1 - d->i0;
    if (!(D == 64 || D == 128 || D == 256) || d->H % 8 != 0 || d->H > 16384) return MRT_OK;
    if ((il + grid - 1) / grid > 256 || (d->nh * D) % 8 != 0 || il % 8 != 0) return MRT_OK;
    // The split down GEMV: at most one 128-row tile per CTA, so a CTA's unit
    // range spans at most two tiles.
    if ((d->H + 127) / 128 > grid) return MRT_OK;
    for (auto& ly : d->layers)
        for (mrt_weight w : {ly.qkv, ly.o, ly.gateup, ly.down})
            if (!w->tiled) return MRT_OK;
    if (!d->lm_head->tiled) return MRT_OK;
    const int64_t att_split = std::max<int64_t>(1, grid / d->nh);
    std::vector<StepLayer> hl(static_cast<size_t>(d->L));
    const int64_t kv_layer = d->nkv * d->max_seq * D;
    for (int64_t l = 0; l < d->L; ++l) {
        const DecLayer& ly = d->layers[static_cast<size_t>(l)];
        StepLayer& t = hl[static_cast<size_t>(l)];
        t.qkv = ly.qkv->data;
        t.bias = ly.qkv_bias ? ly.qkv->bias : nullptr;
        t.o = ly.o->data;
        t.gu = ly.gateup->data;
        t.down = ly.down->data;
        t.ln1 = ly.ln1;
        t.ln2 = ly.ln2;
        t.ln1_dt = ly.ln1_dt;
        t.ln2_dt = ly.ln2_dt;
        t.kc = d->kc + l * kv_layer;
        t.vc = d->vc + l * kv_layer;
    }
    int rc;
    StepArgs& a = d->step;
    auto buf = [&](void** p, size_t bytes, const char* w) { return dec_alloc(d, p, bytes, w); };
    if ((rc = buf(reinterpret_cast<void**>(&d->step_layers), hl.size() * sizeof(StepLayer), "decode-step tables")) ||
        (rc = buf(reinterpret_cast<void**>(&a.x), static_cast<size_t>(d->H) * 2, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.r1), static_cast<size_t>(d->H) * 2, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.qkv_out), static_cast<size_t>(d->n_qkv) * 2, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.attn), static_cast<size_t>(d->nh * D) * 2, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.yo), static_cast<size_t>(d->H) * 2, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.act), static_cast<size_t>(il) * 2, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.yd), static_cast<size_t>(d->H) * 2, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.att_part), static_cast<size_t>(d->nh * att_split * (D + 2)) * 4, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.att_cnt), static_cast<size_t>(d->nh) * 4, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.cand_val), static_cast<size_t>(grid) * 4, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.cand_idx), static_cast<size_t>(grid) * 8, "decode-step scratch")) ||
        (rc = buf(reinterpret_cast<void**>(&a.bar), 256, "decode-step barrier")))
        return rc;
    cudaError_t e = cudaMemcpy(d->step_layers, hl.data(), hl.size() * sizeof(StepLayer), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(a.att_cnt, 0, static_cast<size_t>(d->nh) * 4);
    if (e != cudaSuccess) return cuda_error(e, "initialising the decode step");
    a.layers = d->step_layers;
    a.L = static_cast<int>(d->L);
    a.H = d->H;
    a.D = D;
    a.nh = d->nh;
    a.nkv = d->nkv;
    a.group = d->heads / d->kvh;
    a.h0 = d->h0;
    a.g0 = d->g0;
    a.I = il;
    a.V = d->v1 - d->v0;
    a.max_seq = d->max_seq;
    a.n_qkv = d->n_qkv;
    a.embed = d->embed;
    a.vocab = d->V;
    a.norm = d->norm;
    a.norm_dt = d->norm_dt;
    a.lm = d->lm_head->data;
    a.eps = d->cfg.rms_norm_eps;
    a.scale = 1.0f / std::sqrt(static_cast<float>(D));  // qwen_model.cpp:220
    a.cos_t = d->cos_t;
    a.sin_t = d->sin_t;
    a.silu_lut = silu_lut_for_device(d->device);
    a.att_split = static_cast<int>(att_split);
    a.st = reinterpret_cast<StepState*>(d->state);
    a.err = current_ctx()->d_err;
    a.rank = d->rank;
    a.world = d->world;
    a.v0 = d->v0;
    if (d->world > 1) {
        for (int q = 0; q < d->world; ++q) {
            a.peer_buf[0][q] = d->pa[0].buf[q];
            a.peer_buf[1][q] = d->pa[1].buf[q];
            a.peer_flags[q] = d->pa[0].flags[q];
            a.peer_cand[q] = reinterpret_cast<float*>(static_cast<char*>(d->peer_reg[q]) + 128);
        }
        a.epoch = d->ar_epoch;
        a.part_down = const_cast<float*>(d->pa[1].buf[d->rank]);
    } else if ((rc = buf(reinterpret_cast<void**>(&a.part_down), static_cast<size_t>(grid) * 256 * 4, "decode-step partials"))) {
        return rc;
    }
    d->step_grid = grid;
    d->fused_step = true;
    return MRT_OK;
}

// One decode step as a single persistent launch (the barrier counter is
// cleared first; both are stream-ordered, so the pair can be captured).
int dec_step_fused(mrt_decoder d) {
    d->step.tokens = d->tokens;
    d->step.tokens_cap = d->tokens_cap;
    DEC_CU(cudaMemsetAsync(d->step.bar, 0, 256, d->stream), "clearing the step barrier");
    const cudaError_t e = launch_decode_step(d->step, d->step_grid, d->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(MRT_ERR_CUDA, std::string("decode-step launch: ") + cudaGetErrorString(e) + "; " + decode_step_diag());
    }
    return MRT_OK;
}

// Checks every tensor is present, ties lm_head to the embedding when absent,
// and allocates the KV cache, activations, RoPE tables and scratch.
int dec_finalize(mrt_decoder d) {
    if (d->ready) return MRT_OK;
    if (d->embed == nullptr) return set_error(MRT_ERR_INVALID_ARG, "model.embed_tokens.weight was not loaded");
    if (d->norm == nullptr) return set_error(MRT_ERR_INVALID_ARG, "model.norm.weight was not loaded");
    for (int64_t l = 0; l < d->L; ++l) {
        DecLayer& ly = d->layers[static_cast<size_t>(l)];
        const std::string p = "model.layers." + std::to_string(l) + ".";
        if (!ly.ln1 || !ly.ln2) return set_error(MRT_ERR_INVALID_ARG, p + "*_layernorm.weight missing");
        if (!ly.qkv) return set_error(MRT_ERR_INVALID_ARG, p + "self_attn.{q,k,v}_proj.weight missing");
        if (!ly.o || !ly.down) return set_error(MRT_ERR_INVALID_ARG, p + "o_proj / down_proj weight missing");
        if (!ly.gateup) return set_error(MRT_ERR_INVALID_ARG, p + "mlp.{gate,up}_proj.weight missing");
        if (ly.bias_have != 0 && ly.bias_have != 7u)
            return set_error(MRT_ERR_INVALID_ARG, p + "self_attn: only some of the q/k/v biases were loaded");
        if (ly.bias_have == 7u && !ly.qkv_bias) {
            int rc = mrt_weight_attach_bias(ly.qkv, ly.st_bias, MRT_FP16, 1, d->stream);
            if (rc != MRT_OK) return rc;
            ly.qkv_bias = true;
            dec_release(d, ly.st_bias);
            ly.st_bias = nullptr;
        }
    }
    if (d->lm_head == nullptr) {
        // Tied embeddings (qwen_model.cpp:346-352): this rank's vocabulary rows.
        const int64_t vr[2] = {d->v0, d->v1};
        int rc = mrt_weight_upload(d->embed, MRT_FP16, 1, d->V, d->H, vr, 1, 0, d->H, d->stream, &d->lm_head);
        if (rc != MRT_OK) return rc;
    }
    const int64_t S = d->max_seq, H = d->H, D = d->D;
    int rc;
    auto act = [&](uint16_t** p, int64_t elems, const char* w) {
        return dec_alloc(d, reinterpret_cast<void**>(p), static_cast<size_t>(elems) * 2, w);
    };
    if ((rc = act(&d->x, S * H, "activations")) || (rc = act(&d->r, S * H, "activations")) ||
        (rc = act(&d->p, S * H, "activations")) || (rc = act(&d->normed, S * H, "activations")) ||
        (rc = act(&d->qkv, S * d->n_qkv, "activations")) || (rc = act(&d->attn, S * d->nh * D, "activations")) ||
        (rc = act(&d->act, S * (d->i1 - d->i0), "activations")) ||
        (rc = act(&d->logits, d->v1 - d->v0, "logits")) || (rc = act(&d->kc, d->L * d->nkv * S * D, "the KV cache")) ||
        (rc = act(&d->vc, d->L * d->nkv * S * D, "the KV cache")))
        return rc;
    if (d->world > 1 &&
        (rc = dec_alloc(d, reinterpret_cast<void**>(&d->partial), static_cast<size_t>(S * H) * 4, "row-parallel partials")))
        return rc;
    if (d->world > 1 && d->world <= kMaxRanks && (rc = dec_setup_p2p(d)) != MRT_OK) return rc;
    // RoPE tables with the reference's float expressions (cpu_backend.cpp:363-366).
    const int64_t half = D / 2;
    std::vector<float> cs(static_cast<size_t>(S * half)), sn(static_cast<size_t>(S * half));
    const float theta = d->cfg.rope_theta;
    for (int64_t pos = 0; pos < S; ++pos)
        for (int64_t i = 0; i < half; ++i) {
            const float freq = 1.0f / std::pow(theta, static_cast<float>(2 * i) / static_cast<float>(D));
            const float angle = static_cast<float>(static_cast<size_t>(pos)) * freq;
            cs[static_cast<size_t>(pos * half + i)] = std::cos(angle);
            sn[static_cast<size_t>(pos * half + i)] = std::sin(angle);
        }
    if ((rc = dec_alloc(d, reinterpret_cast<void**>(&d->cos_t), cs.size() * 4, "RoPE tables")) ||
        (rc = dec_alloc(d, reinterpret_cast<void**>(&d->sin_t), sn.size() * 4, "RoPE tables")))
        return rc;
    cudaError_t e = cudaMemcpy(d->cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(d->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_error(e, "uploading RoPE tables");
    // Decode attention: one block per 32 cached positions per query head.
    const int64_t ns = (S + kSplitKeys - 1) / kSplitKeys;
    if (ns > 65535) return set_error(MRT_ERR_UNSUPPORTED, "max_seq_len above 2097120");
    d->nsplit = static_cast<int>(ns);
    if ((rc = dec_alloc(d, reinterpret_cast<void**>(&d->part), static_cast<size_t>(d->nh * d->nsplit * (D + 2)) * 4, "attention scratch")) ||
        (rc = dec_alloc(d, reinterpret_cast<void**>(&d->counters), static_cast<size_t>(d->nh) * 4, "attention counters")) ||
        (rc = dec_alloc(d, reinterpret_cast<void**>(&d->am_idx), 8, "argmax output")) ||
        (rc = dec_alloc(d, reinterpret_cast<void**>(&d->am_gidx), 8, "argmax output")) ||
        (rc = dec_alloc(d, reinterpret_cast<void**>(&d->am_val), 4, "argmax output")) ||
        (rc = dec_alloc(d, &d->am_scratch, argmax_scratch_bytes(1, d->v1 - d->v0), "argmax scratch")) ||
        (rc = dec_alloc(d, reinterpret_cast<void**>(&d->state), sizeof(DecState), "decoder state")))
        return rc;
    e = cudaMemset(d->counters, 0, static_cast<size_t>(d->nh) * 4);
    if (e == cudaSuccess) e = cudaMemset(d->kc, 0, static_cast<size_t>(d->L * d->nkv * S * D) * 2);
    if (e == cudaSuccess) e = cudaMemset(d->vc, 0, static_cast<size_t>(d->L * d->nkv * S * D) * 2);
    if (e != cudaSuccess) return cuda_error(e, "clearing decoder buffers");
    if (silu_lut_for_device(d->device) == nullptr) return set_error(MRT_ERR_CUDA, "building the SiLU table failed");
    if ((rc = dec_setup_step(d)) != MRT_OK) return rc;
    d->ready = true;
    return MRT_OK;
}


// One forward over S rows starting at the state's position: prefill
// (ids = the prompt on the device, pos0 its host-known start) or one decode
// step (ids == nullptr: the state's token), ending with the greedy pick of
// the last row and the state update.
int dec_forward(mrt_decoder d, int64_t S, const int32_t* ids, int64_t pos0, bool decode) {
    cudaStream_t s = d->stream;
    DevCtx* ctx = current_ctx();
    if (!ctx) return MRT_ERR_CUDA;
    const int64_t H = d->H, D = d->D, nq = d->n_qkv, group = d->heads / d->kvh;
    const int64_t il = d->i1 - d->i0, nh = d->nh, ad = d->nh * D;  // local widths
    const size_t row_smem = 0;
    const float eps = d->cfg.rms_norm_eps;
    const float scale = 1.0f / std::sqrt(static_cast<float>(D));  // qwen_model.cpp:220
    const int64_t kv_layer = d->nkv * d->max_seq * D;
    // Row-parallel output: FP32 partials, summed across ranks, rounded once.
    // With the peer path the partial stays in this rank's exchange buffer of
    // the call site (0 = o, 1 = down) and the next add+norm kernel finishes it.
    auto row_parallel = [&](mrt_weight w, const uint16_t* x, int64_t ldx, int site) -> int {
        if (d->world == 1) return mrt_gemm(w, x, ldx, d->p, H, S, 0, s);
        if (d->p2p) return mrt_gemm_f32(w, x, ldx, const_cast<float*>(d->pa[site].buf[d->rank]), H, S, s);
        int rc = mrt_gemm_f32(w, x, ldx, d->partial, H, S, s);
        if (rc != MRT_OK) return rc;
        return mrt_tp_allreduce_f32_to_f16(d->tp, d->partial, d->p, S * H, s);
    };
    // out = fp16(a + the row-parallel output of `site`), normed = RMSNorm(out).
    auto add_norm = [&](const uint16_t* a, uint16_t* out, const void* gw, int gdt, int site, int call, int64_t row0,
                        int64_t rows) -> cudaError_t {
        const bool pre = rows <= kPreloadRows;
        if (d->p2p)
            return launch_pdl(pre ? ar_add_norm_kernel<true> : ar_add_norm_kernel<false>, dim3(static_cast<unsigned>(rows)),
                              dim3(kNT), 0, s, d->pa[site], row0, a, out, H, gw, gdt, eps, d->normed, d->ar_epoch, call,
                              ctx->d_err);
        return launch_pdl(pre ? add_norm_kernel<true> : add_norm_kernel<false>, dim3(static_cast<unsigned>(rows)),
                          dim3(kNT), row_smem, s, a + row0 * H, d->p + row0 * H, out + row0 * H, H, gw, gdt, eps,
                          d->normed + row0 * H);
    };
    const int calls = static_cast<int>(2 * d->L);
    auto grid_for = [](int64_t n) {
        int64_t b = (n + kNT - 1) / kNT;
        return static_cast<unsigned>(b < 1 ? 1 : (b > 148 * 16 ? 148 * 16 : b));
    };
    for (int64_t l = 0; l < d->L; ++l) {
        DecLayer& ly = d->layers[static_cast<size_t>(l)];
        if (l == 0) {
            DEC_CU(launch_pdl(S <= kPreloadRows ? embed_norm_kernel<true> : embed_norm_kernel<false>,
                              dim3(static_cast<unsigned>(S)), dim3(kNT), row_smem, s, d->embed, d->V, H, ids, d->state,
                              d->x, ly.ln1, ly.ln1_dt, eps, d->normed, ctx->d_err),
                   "embedding launch");
        } else {
            DEC_CU(add_norm(d->r, d->x, ly.ln1, ly.ln1_dt, 1, static_cast<int>(2 * (l - 1) + 1), 0, S), "add+rmsnorm launch");
        }
        DEC_TRY(mrt_gemm(ly.qkv, d->normed, H, d->qkv, nq, S, ly.qkv_bias ? MRT_GEMM_BIAS : 0, s));
        uint16_t* kc = d->kc + l * kv_layer;
        uint16_t* vc = d->vc + l * kv_layer;
        if (decode) {
            // RoPE and the KV append run inside the attention launch.
            DEC_CU(attn_decode(static_cast<int>(D), dim3(static_cast<unsigned>(nh), static_cast<unsigned>(d->nsplit)), s,
                               d->qkv, static_cast<int>(nh), static_cast<int>(d->nkv), kc, vc, d->attn,
                               static_cast<int>(group), static_cast<int>(d->h0), static_cast<int>(d->g0), d->max_seq,
                               scale, d->state, d->part, d->counters, d->cos_t, d->sin_t),
                   "attention launch");
        } else {
            DEC_CU(launch_pdl(rope_append_kernel, dim3(grid_for(S * (nh + d->nkv) * (D / 2))), dim3(kNT), 0, s, d->qkv,
                              nq, S, static_cast<int>(nh), static_cast<int>(d->nkv), static_cast<int>(D), d->cos_t,
                              d->sin_t, kc, vc, d->max_seq, d->state),
                   "rope launch");
            // Query head h over kv head h / group (qwen_model.cpp:212-245).
            DEC_CU(attn_prefill(static_cast<int>(D), static_cast<int>(nh), S, s, d->qkv, nq, pos0, kc, vc, d->max_seq,
                                d->attn, ad, static_cast<int>(group), static_cast<int>(d->h0), static_cast<int>(d->g0),
                                scale),
                   "prefill attention launch");
        }
        DEC_TRY(row_parallel(ly.o, d->attn, ad, 0));
        DEC_CU(add_norm(d->x, d->r, ly.ln2, ly.ln2_dt, 0, static_cast<int>(2 * l), 0, S), "add+rmsnorm launch");
        // gate|up with SiLU(gate) * up (in the GEMM's epilogue when its plan
        // keeps whole tiles).
        DEC_TRY(mrt_gemm_swiglu(ly.gateup, d->normed, H, d->act, il, S, s));
        DEC_TRY(row_parallel(ly.down, d->act, il, 1));
    }
    // Final residual and norm of the last row, lm_head, greedy pick.
    const int64_t last = (S - 1) * H;
    DEC_CU(add_norm(d->r, d->x, d->norm, d->norm_dt, 1, calls - 1, S - 1, 1), "final norm launch");
    const int64_t vl = d->v1 - d->v0;
    // The GEMM's epilogue reduces every 32 vocabulary rows to their best
    // (value, index); one small kernel picks among those.
    (void)vl;
    DEC_TRY(mrt_lm_head_argmax(d->lm_head, d->normed + last, H, 1, d->logits, d->v0, d->am_idx, d->am_val, s));
    const int64_t* pick = d->am_idx;
    if (d->world > 1) {
        // Vocabulary shards: the first maximum over every rank's (value, index).
        DEC_TRY(mrt_tp_argmax(d->tp, d->am_val, d->am_idx, 1, d->am_gidx, s));
        pick = d->am_gidx;
    }
    DEC_CU(launch_pdl(advance_kernel, dim3(1), dim3(32), 0, s, pick, d->state, d->tokens, d->tokens_cap,
                      static_cast<int>(S), d->p2p ? d->ar_epoch : nullptr, calls),
           "advance launch");
    return MRT_OK;
}

}  // namespace

extern "C" int mrt_decoder_generate(mrt_decoder d, const int32_t* prompt, int64_t n_prompt, int64_t max_new,
                                    int32_t eos, int32_t* out_tokens, int64_t* n_out, mrt_decoder_stats* stats,
                                    void* user_stream) {
    clear_error();
    if (d == nullptr || prompt == nullptr || out_tokens == nullptr || n_out == nullptr)
        return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    *n_out = 0;
    if (stats) *stats = mrt_decoder_stats{0.0f, 0.0f, 0.0f, 0};
    if (n_prompt < 1 || max_new < 0) return set_error(MRT_ERR_SHAPE, "need n_prompt >= 1 and max_new >= 0");
    if (max_new == 0) return MRT_OK;
    if (n_prompt + max_new - 1 > d->max_seq)
        return set_error(MRT_ERR_SHAPE, "n_prompt + max_new - 1 exceeds max_seq_len");
    if (n_prompt > 65535) return set_error(MRT_ERR_SHAPE, "at most 65535 prompt tokens per call");
    for (int64_t i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= d->V)
            return set_error(MRT_ERR_INVALID_ARG, "embedding_lookup: token_id out of range");
    DevCtx* ctx = current_ctx();
    if (!ctx) return MRT_ERR_CUDA;
    DEC_TRY(dec_finalize(d));
    cudaStream_t s = d->stream;
    if (d->ids_cap < n_prompt) {
        dec_release(d, d->ids);
        d->ids = nullptr;
        DEC_TRY(dec_alloc(d, reinterpret_cast<void**>(&d->ids), static_cast<size_t>(n_prompt) * 4, "prompt ids"));
        d->ids_cap = n_prompt;
    }
    if (d->tokens_cap < max_new) {
        dec_release(d, d->tokens);
        d->tokens = nullptr;
        DEC_TRY(dec_alloc(d, reinterpret_cast<void**>(&d->tokens), static_cast<size_t>(max_new) * 4, "generated ids"));
        d->tokens_cap = max_new;
    }
    // Order after the caller's work, then start from position 0.
    cudaEvent_t ev[5] = {};
    for (auto& e : ev) DEC_CU(cudaEventCreate(&e), "creating events");
    struct Cleanup {
        cudaEvent_t* ev;
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        ~Cleanup() {
            if (exec) cudaGraphExecDestroy(exec);
            if (graph) cudaGraphDestroy(graph);
            for (int i = 0; i < 5; ++i)
                if (ev[i]) cudaEventDestroy(ev[i]);
        }
    } cleanup{ev};
    DEC_CU(cudaEventRecord(ev[0], static_cast<cudaStream_t>(user_stream)), "recording an event");
    DEC_CU(cudaStreamWaitEvent(s, ev[0], 0), "ordering after the caller's stream");
    const DecState st0{0, 0, 0, 0};
    DEC_CU(cudaMemcpyAsync(d->state, &st0, sizeof(st0), cudaMemcpyHostToDevice, s), "resetting the decoder state");
    DEC_CU(cudaMemcpyAsync(d->ids, prompt, static_cast<size_t>(n_prompt) * 4, cudaMemcpyHostToDevice, s), "uploading the prompt");
    DEC_CU(cudaStreamSynchronize(s), "uploading the prompt");  // prompt and st0 are pageable host memory
    // The reference prefills one token at a time (inference_engine.cpp:42-48);
    // every op is row-independent under the causal mask, so one batched
    // forward gives the same rows.
    DEC_CU(cudaEventRecord(ev[0], s), "recording an event");
    DEC_TRY(dec_forward(d, n_prompt, d->ids, 0, false));
    DEC_CU(cudaEventRecord(ev[1], s), "recording an event");
    int64_t replays = 0;
    auto step = [&]() { return d->fused_step ? dec_step_fused(d) : dec_forward(d, 1, nullptr, 0, true); };
    if (max_new >= 2) {
        DEC_TRY(step());  // eager: sizes every scratch buffer
        DEC_CU(cudaEventRecord(ev[2], s), "recording an event");
        replays = max_new - 2;
        if (replays > 0) {
            DEC_CU(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "beginning the decode-step capture");
            const int rc = step();
            const cudaError_t ec = cudaStreamEndCapture(s, &cleanup.graph);
            if (rc != MRT_OK) return rc;
            DEC_CU(ec, "capturing the decode step");
            DEC_CU(cudaGraphInstantiate(&cleanup.exec, cleanup.graph, 0), "instantiating the decode step");
            DEC_CU(cudaEventRecord(ev[3], s), "recording an event");
            for (int64_t i = 0; i < replays; ++i) DEC_CU(cudaGraphLaunch(cleanup.exec, s), "replaying the decode step");
            DEC_CU(cudaEventRecord(ev[4], s), "recording an event");
        }
    }
    DEC_TRY(mrt_sync(s));
    std::vector<int32_t> toks(static_cast<size_t>(max_new));
    DEC_CU(cudaMemcpy(toks.data(), d->tokens, static_cast<size_t>(max_new) * 4, cudaMemcpyDeviceToHost), "reading tokens");
    int64_t n = 0;
    for (; n < max_new; ++n) {
        out_tokens[n] = toks[static_cast<size_t>(n)];
        if (eos >= 0 && toks[static_cast<size_t>(n)] == eos) {
            ++n;
            break;
        }
    }
    *n_out = n;
    if (stats) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ev[0], ev[1]);
        stats->prefill_ms = ms;
        if (max_new >= 2) {
            cudaEventElapsedTime(&ms, ev[1], ev[2]);
            stats->first_step_ms = ms;
        }
        if (replays > 0) {
            cudaEventElapsedTime(&ms, ev[3], ev[4]);
            stats->decode_ms = ms;
            stats->decode_steps = replays;
        }
    }
    return MRT_OK;
}

extern "C" void mrt_decoder_free(mrt_decoder d) {
    if (d == nullptr) return;
    cudaStreamSynchronize(d->stream);
    if (d->p2p) {
        for (int q = 0; q < d->world; ++q)
            if (q != d->rank && d->peer_reg[q]) cudaIpcCloseMemHandle(d->peer_reg[q]);
        // No rank frees its exchange region while a peer still maps it.
        int one = 1;
        std::vector<int> all(static_cast<size_t>(d->world));
        tp_allgather_host(d->tp, &one, all.data(), sizeof(int));
    }
    for (auto& ly : d->layers)
        for (mrt_weight w : {ly.qkv, ly.o, ly.gateup, ly.down})
            if (w) mrt_weight_free(w);
    if (d->lm_head) mrt_weight_free(d->lm_head);
    for (void* p : d->allocs)
        if (p) cudaFree(p);
    cudaStreamDestroy(d->stream);
    delete d;
}
