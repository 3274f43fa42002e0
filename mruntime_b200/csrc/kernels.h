// kernels.h -- host-side launchers of the sm_100a kernels (internal to the
// library; the public surface is include/mrt_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mrt {

// Count one kernel launch (read through mrt_launch_count).
void note_launches(int n);


// Y = X * W^T on the tcgen05 tensor cores.  The MMA's 128-row operand ("A")
// is X (normal mode) or W (swap mode, for few tokens: the weight rows fill the
// 128 TMEM lanes and the tokens are the MMA's N = bn); the bn-row operand
// ("B") is the other one.  tmap_a: box 64 x 128, tmap_b: box 64 x bn, both
// K-major with 128-byte swizzle.  Tiles are 128 A-rows x bn B-rows, numbered
// A-fastest.  Tiles [0, full_tiles) run over the whole K and store the output
// directly; each remaining ("tail") tile runs as tail_splits K-slices of
// kb_per 64-wide k-blocks that store FP32 partials, tile-major, into
// `partials` ([tail_splits][n_tail][128][bn]).  Swap mode: the last slice to
// finish a 32-row quadrant of a tail tile sums the slices and stores it
// (tile_counters); normal mode: launch_reduce_tail does it on the whole GPU.
struct TcGemmArgs {
    int M, N, K;     // tokens, weight rows, reduction length (in both modes)
    int swap;        // 1: A = W, B = X
    int bn;          // B rows per tile: 64/128/256 (normal), 16/32/64 (swap)
    int grid;        // persistent CTAs
    int full_tiles;  // tiles computed over the whole K
    int tail_splits; // K-slices per tail tile (>= 1)
    int kb_per;      // k-blocks per tail slice
    void* y;         // FP16 or FP32 output [M, ldy]
    int64_t ldy;
    int out_f32;
    const uint16_t* bias;
    float* partials;
    // One counter per (tail tile, 32-row quadrant), zero between calls: every
    // epilogue warp of a K-slice adds one after storing its partial rows; the
    // warp that brings it to tail_splits sums the slices in slice order,
    // stores the output and resets the counter.
    int* tile_counters;
    int* err_flag;
    // Weight in the tiled layout (nullptr: the weight's tensor map is used).
    const uint16_t* w_tiled;
    int64_t w_k_tiles;
    // Every launch carries a programmatic edge to the previous kernel in the
    // stream, whose completion the kernel awaits (griddepcontrol.wait) before
    // it reads activations or writes anything.  1: the first ring pass of
    // tiled weight tiles may be fetched before that wait (the weights must
    // not be written by the kernel being overlapped).
    int w_prefetch;
    // Swap mode, every tile split into cluster_k (2..8) K-slices and one slice
    // per CTA: the slices of a tile run as one thread-block cluster and are
    // summed through distributed shared memory (partials and tile_counters
    // unused).  0: slices are summed through global memory.
    int cluster_k;
    // Non-null: SwiGLU epilogue for a weight whose rows interleave gate and
    // up (row 2j = gate j, row 2j + 1 = up j): y[m][j] = fp16(lut[fp16(g)] *
    // fp16(u)) with y of N / 2 columns.  Plans without a K-split only; no
    // bias, FP16 output.
    const uint16_t* swiglu_lut;
    // Non-null: residual add after the output rounding, y[m][n] =
    // fp16(res[m][n] + fp16(acc (+ bias))) with res of row stride ldr (the
    // reference's add op after o_proj and down_proj).  FP16 output only; y may
    // be res itself (each element is read, then written, by one thread).
    const uint16_t* residual;
    int64_t ldr;
    // Non-null (swap mode, FP16 output, no cluster finish): greedy-pick
    // partials.  For every token m and every 32 weight rows (chunk c = row / 32)
    // the epilogue writes the best (value, index) of those rows' FP16 outputs
    // under the reference's rule to am_val / am_idx[m * am_chunks + c];
    // am_chunks = 4 * ceil(N / 128).  y may then be null (no logits stored).
    float* am_val;
    int64_t* am_idx;
    int am_chunks;
    // Segmented variant only: k-blocks per accumulator segment (kSegKb).
    int seg_kb;
    // 1: SM-pair plan (launch_tc_pair): tiles of 256 X rows, partials
    // [tail_splits][n_tail][256][bn].
    int pair;
};

// Whether a swap-mode launch of tile width bn may use clusters of k CTAs on
// the current device (checked once per device, width and k).
bool tc_cluster_ok(int bn, int k);
cudaError_t launch_tc_gemm(const TcGemmArgs& a, const CUtensorMap& tmap_x, const CUtensorMap& tmap_w,
                           cudaStream_t s);
// Output tiles of a plan (128 A rows x bn B rows each; 256 A rows for pairs).
int tc_gemm_tiles(const TcGemmArgs& a);
// Units longer than this many 64-wide k-blocks accumulate in segments (normal
// mode: the segmented kernel variant; swap-mode plans keep every unit at or
// below it).
constexpr int kSegMinKb = 64;
// k-blocks per accumulator segment of the segmented variant: at K = 18944 the
// error against FP64 is then within 0.02 % of 16-block segments' (which match
// the reference's own), for ~3 % of the kernel's time instead of ~11 %.
constexpr int kSegKb = 64;
// Whether a normal-mode launch uses the segmented-accumulation variant.
bool tc_gemm_segmented(const TcGemmArgs& a);
// Normal mode on SM pairs (tcgen05 cta_group::2, a.pair = 1): tiles of 256
// X rows x bn (256) W rows, numbered m-fastest, a.grid = 2 x pairs (even).
// Tiles [0, full_tiles) run over the whole K; each remaining tile runs as
// tail_splits K-slices whose FP32 partials launch_reduce_tail sums, as in the
// one-SM kernel.  tmap_w_rows views the tiled weight as
// [n_pad * k_tiles * 128] rows of 64 FP16 with a 64 x 128 box and no swizzle
// (one tile per box).
cudaError_t launch_tc_pair(const TcGemmArgs& a, const CUtensorMap& tmap_x, const CUtensorMap& tmap_w_rows,
                           cudaStream_t s);
// Normal mode only: sum the K-slices of every tail tile in slice order on
// the whole GPU, round (+bias) or keep FP32, and store.
cudaError_t launch_reduce_tail(const TcGemmArgs& a, cudaStream_t s);

// y = x * W^T for 1..4 tokens on the tiled weight layout (gemv.cu): SIMT
// 16-byte weight loads, FP32 sums, no scratch memory.  x: M rows of K FP16
// (16-byte aligned, ldx a multiple of 8); y: FP16 (bias, residual or SwiGLU
// as in the tcgen05 kernel's epilogue) or FP32.  rq: row quads per CTA (1, 2, 4, 8).
struct GemvArgs {
    const uint16_t* w;  // tiled weight [n_pad / 128][k_tiles][128][64]
    int64_t k_tiles;
    const uint16_t* x;
    int64_t ldx;
    void* y;
    int64_t ldy;
    int out_f32;
    const uint16_t* bias;      // FP16, N entries, or null
    const uint16_t* residual;  // y = fp16(residual + fp16(acc)), or null
    int64_t ldr;
    const uint16_t* swiglu_lut;  // SwiGLU on interleaved gate|up rows (N even, FP16 out, no bias), or null
    int M, N, K;
    int rq;
};
cudaError_t launch_gemv_tiled(const GemvArgs& a, cudaStream_t s);


// Element-wise conversions with the reference's rounding.
cudaError_t launch_convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n,
                           cudaStream_t s);
// Gather rows/columns of a [rows, cols] source of dtype src_dtype into a
// dense FP16 [rows, k1-k0] destination (weight upload of a shard).
cudaError_t launch_convert_2d_to_f16(const void* src, int src_dtype, int64_t src_ld, int64_t rows,
                                     int64_t cols, uint16_t* dst, cudaStream_t s);

// Tiled weight layout (see mrt_weight_s and tiled_offset in common.cuh).
cudaError_t launch_convert_rows_to_tiled(const void* src, int src_dtype, int64_t src_ld, int64_t rows,
                                         int64_t cols, uint16_t* dst, int64_t row0, int64_t k_tiles,
                                         cudaStream_t s);
cudaError_t launch_untile(const uint16_t* src, int64_t n, int64_t k, int64_t k_tiles, uint16_t* dst,
                          int64_t ld, cudaStream_t s);

// Row argmax in two passes through `scratch` (see argmax_scratch_bytes).
size_t argmax_scratch_bytes(int64_t M, int64_t V);
cudaError_t launch_argmax(const uint16_t* logits, int64_t M, int64_t V, int64_t ld,
                          int64_t index_base, int64_t* idx, float* val, void* scratch,
                          cudaStream_t s);
// Second pass alone: best of pv / pi[m * nchunks + c] per row m.
cudaError_t launch_argmax_final(const float* pv, const int64_t* pi, int64_t M, int64_t nchunks,
                                int64_t index_base, int64_t* idx, float* val, cudaStream_t s);
// Combine per-rank (value, index) pairs gathered as [world, M].
cudaError_t launch_argmax_combine(const float* vals, const int64_t* idxs, int world, int64_t M,
                                  int64_t* idx_out, cudaStream_t s);

// A single wait on a barrier that never completes, bounded by limit_ns.
cudaError_t launch_wait_selftest(int* flag, uint64_t limit_ns, cudaStream_t s);

// FP32 -> FP16 rounding of an all-reduced buffer.
cudaError_t launch_f32_to_f16(const float* src, uint16_t* dst, int64_t n, cudaStream_t s);

// General strided GEMM covering the whole Backend::gemm contract.
struct GeneralGemmArgs {
    const void* a;
    int a_dtype;
    int64_t a_cols0;
    const void* b;
    int b_dtype;
    int64_t b_cols0;
    void* c;
    int c_dtype;
    int64_t ldc;  // row stride of C (N for a dense C)
    int64_t M, N, K;
    float alpha, beta;
    int trans_a, trans_b;
    const uint16_t* bias;  // FP16 [N] added after rounding (FP16 C only) or nullptr
    int64_t b_k_tiles;     // > 0: B is an FP16 weight [N, K] in the tiled layout (trans_b)
    const uint16_t* residual;  // FP16 C only: c = fp16(residual + fp16(...)) (row stride ldr), or nullptr
    int64_t ldr;
};
cudaError_t launch_general_gemm(const GeneralGemmArgs& a, cudaStream_t s);

}  // namespace mrt
