// gemv.cu -- y = x * W^T for 1..4 tokens straight from the tiled weight layout:
// the decode-side GEMV of the linear-layer path (the reference's
// Backend::gemm at M = 1, src/core/cpu_backend.cpp:72-169, called by
// src/models/qwen/qwen_model.cpp:126-128, 256, 278-279, 288 once per token).
//
// Why a SIMT kernel beside the swap-mode tcgen05 kernel: with one token the
// MMA does 1/16 useful work and the tcgen05 set-up (TMEM allocation, mbarrier
// ring, pipeline fill, TMEM read-back, K-split finish) costs a few
// microseconds per call whatever the weight size, which is most of an 8.7 MB
// GEMV.  Here every lane issues its 16-byte weight loads before the
// programmatic wait on the previous kernel, so the weight stream overlaps the
// previous kernel's tail, and the products are summed with warp shuffles.
//
// Work split.  A warp covers four consecutive weight rows: in one 16-byte
// load per lane it reads those rows' 128-byte runs of one 128 x 64 tile
// (4 x 128 B contiguous, whole L2 lines), lane l taking row l / 8 and stored
// chunk l % 8, which holds k-chunk (l % 8) ^ (row % 8) of the tile (the
// tensor cores' 128-byte swizzle the upload applied).  A CTA of eight warps
// holds `rq` row quads (1, 2, 4 or 8); the 8 / rq warps of a quad split the
// tile columns (K) into contiguous slices.  Sums: each lane accumulates its
// chunks in FP32 in K order, the eight lanes of a row combine by a fixed
// shuffle tree, and the K-slices of a row are added in slice order through
// shared memory -- deterministic, no scratch memory, no atomics.
#include "common.cuh"
#include "kernels.h"

namespace mrt {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvBatch = 8;        // 16-byte weight loads in flight per lane
constexpr int kTileElems = 128 * 64;  // one tiled weight block

// Weight load: read once per call, so it bypasses L1 and is evicted first
// from L2.
__device__ __forceinline__ uint4 ld_weight_v4(const uint16_t* p, uint64_t pol) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

// acc += dot(eight FP16 weights, eight FP16 activations), in k order.
__device__ __forceinline__ float dot8(float acc, const float (&w)[8], uint4 xv) {
    const float2 x0 = h2_to_f2(xv.x), x1 = h2_to_f2(xv.y), x2 = h2_to_f2(xv.z), x3 = h2_to_f2(xv.w);
    acc = fmaf(w[0], x0.x, acc);
    acc = fmaf(w[1], x0.y, acc);
    acc = fmaf(w[2], x1.x, acc);
    acc = fmaf(w[3], x1.y, acc);
    acc = fmaf(w[4], x2.x, acc);
    acc = fmaf(w[5], x2.y, acc);
    acc = fmaf(w[6], x3.x, acc);
    acc = fmaf(w[7], x3.y, acc);
    return acc;
}

template <int MT>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_tiled_kernel(GemvArgs a) {
    __shared__ float red[kGemvWarps][32][MT];  // [K-slice][row of the CTA][token]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = kGemvWarps / a.rq;  // K-slices per row quad
    const int quad_local = warp / ks, slice = warp - quad_local * ks;
    const int row_local = quad_local * 4 + (lane >> 3);
    const int64_t n = static_cast<int64_t>(blockIdx.x) * a.rq * 4 + row_local;  // < N rounded up to 32 <= n_pad
    const int r = static_cast<int>(n & 127);
    const int pos = lane & 7;
    const int c = pos ^ (r & 7);  // k-chunk held by stored chunk `pos` of row r
    const int k_tiles = static_cast<int>(a.k_tiles);
    const int per = (k_tiles + ks - 1) / ks;
    const int kt0 = min(k_tiles, slice * per), kt1 = min(k_tiles, kt0 + per);
    const uint16_t* wp = a.w + (n >> 7) * a.k_tiles * kTileElems + r * 64 + pos * 8;
    const uint64_t pol = l2_policy_evict_first();

    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;

    // The weights never change between calls: start streaming them before
    // waiting for the kernel that produced x (and may still read y).
    uint4 wv[kGemvBatch];
#pragma unroll
    for (int u = 0; u < kGemvBatch; ++u)
        if (kt0 + u < kt1) wv[u] = ld_weight_v4(wp + static_cast<int64_t>(kt0 + u) * kTileElems, pol);
    griddep_wait();
    griddep_launch_dependents();

    for (int kb = kt0; kb < kt1; kb += kGemvBatch) {
        if (kb != kt0) {
#pragma unroll
            for (int u = 0; u < kGemvBatch; ++u)
                if (kb + u < kt1) wv[u] = ld_weight_v4(wp + static_cast<int64_t>(kb + u) * kTileElems, pol);
        }
#pragma unroll
        for (int u = 0; u < kGemvBatch; ++u) {
            const int k = (kb + u) * 64 + c * 8;
            if (kb + u < kt1 && k < a.K) {  // tile columns past K are zero padding; x ends at K
                float w[8];
                const float2 w0 = h2_to_f2(wv[u].x), w1 = h2_to_f2(wv[u].y), w2 = h2_to_f2(wv[u].z),
                             w3 = h2_to_f2(wv[u].w);
                w[0] = w0.x; w[1] = w0.y; w[2] = w1.x; w[3] = w1.y;
                w[4] = w2.x; w[5] = w2.y; w[6] = w3.x; w[7] = w3.y;
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < a.M)
                        acc[m] = dot8(acc[m], w, __ldg(reinterpret_cast<const uint4*>(a.x + m * a.ldx + k)));
            }
        }
    }

    // The eight lanes of a row: fixed shuffle tree.
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 4);
        acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 2);
        acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 1);
    }
    if (pos == 0) {
#pragma unroll
        for (int m = 0; m < MT; ++m) red[slice][row_local][m] = acc[m];
    }
    __syncthreads();

    // K-slices of a row in slice order (slices past the last k-tile hold nothing).
    const int used = (k_tiles + per - 1) / per;
    const int t = threadIdx.x;
    if (t < a.rq * 4 * MT) {
        const int row = t / MT, m = t - row * MT;
        const int64_t nn = static_cast<int64_t>(blockIdx.x) * a.rq * 4 + row;
        if (m < a.M && nn < a.N) {
            auto row_sum = [&](int rl) {
                float s = red[0][rl][m];
                for (int sl = 1; sl < used; ++sl) s += red[sl][rl][m];
                return s;
            };
            const float s = row_sum(row);
            if (a.swiglu_lut != nullptr) {
                // Interleaved gate|up rows (2j = gate j, 2j + 1 = up j, both in
                // this CTA): gate and up rounded to FP16, SiLU from the FP16
                // table, the product rounded (qwen_model.cpp:278-285), as the
                // tcgen05 kernel's SwiGLU epilogue does.
                if ((nn & 1) == 0) {
                    const uint16_t g = f32_to_f16_bits(s);
                    const uint16_t u = f32_to_f16_bits(row_sum(row + 1));
                    static_cast<uint16_t*>(a.y)[m * a.ldy + (nn >> 1)] = f32_to_f16_bits(
                        __fmul_rn(f16_bits_to_f32(a.swiglu_lut[g]), f16_bits_to_f32(u)));
                }
            } else if (a.out_f32) {
                static_cast<float*>(a.y)[m * a.ldy + nn] = s;
            } else {
                uint16_t h = round_out(s, a.bias, nn);
                h = add_residual(h, a.residual, m * a.ldr + nn);
                static_cast<uint16_t*>(a.y)[m * a.ldy + nn] = h;
            }
        }
    }
}

}  // namespace

cudaError_t launch_gemv_tiled(const GemvArgs& a, cudaStream_t s) {
    if (a.M < 1 || a.M > 4 || (a.rq != 1 && a.rq != 2 && a.rq != 4 && a.rq != 8) || a.N < 1 || a.k_tiles < 1)
        return cudaErrorInvalidValue;
    const int64_t quads = (static_cast<int64_t>(a.N) + 3) / 4;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>((quads + a.rq - 1) / a.rq));
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (a.M == 1)
        e = cudaLaunchKernelEx(&cfg, gemv_tiled_kernel<1>, a);
    else if (a.M == 2)
        e = cudaLaunchKernelEx(&cfg, gemv_tiled_kernel<2>, a);
    else
        e = cudaLaunchKernelEx(&cfg, gemv_tiled_kernel<4>, a);
    if (e != cudaSuccess) return e;
    note_launches(1);
    return cudaGetLastError();
}

}  // namespace mrt
