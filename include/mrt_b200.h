/*
 * mrt_b200.h -- C ABI of the B200 linear-layer path for mruntime.
 *
 * This is the boundary a host runtime binds (ctypes, cgo, JNI, or the C++
 * CudaBackend in mruntime_b200/csrc/cuda_backend.h).  It replaces the body of
 * mruntime::Backend::gemm (reference include/mruntime/backend.h:13-21) and the
 * pieces around it that the reference runs on the host: the weight load and
 * repack step, the q/k/v bias add, and the greedy argmax over logits.
 *
 * Conventions
 *   - Every entry point returns an int status (MRT_OK == 0).  On failure
 *     mrt_last_error_string() describes the error of the calling thread.
 *   - Pointers named *_dev are device pointers on the current device; *_host
 *     are host pointers (pinned memory makes the copies asynchronous).
 *   - 16-bit data travel as raw bit patterns (IEEE binary16 or bfloat16).
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).  Calls
 *     are asynchronous on that stream unless documented otherwise; one
 *     context's scratch buffers are shared, so calls that use scratch must be
 *     issued on one stream at a time per device.
 *   - Weights are W[N, K] row-major (Hugging Face layout) and every GEMM
 *     computes Y[M, N] = X[M, K] * W^T, i.e. the reference's call pattern
 *     gemm(A, B, C, 1, 0, trans_a=false, trans_b=true)
 *     (reference src/models/qwen/qwen_model.cpp:126-128, 256, 278-279, 288, 374).
 *   - Accumulation is FP32 and outputs are rounded once to FP16 with
 *     round-to-nearest-even, as float_to_fp16_bits does
 *     (reference include/mruntime/dtype.h:39-119).
 */
#ifndef MRT_B200_H
#define MRT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MRT_OK 0
#define MRT_ERR_INVALID_ARG 1
#define MRT_ERR_SHAPE 2
#define MRT_ERR_DTYPE 3
#define MRT_ERR_CUDA 4
#define MRT_ERR_NCCL 5
#define MRT_ERR_TIMEOUT 6
#define MRT_ERR_UNSUPPORTED 7
#define MRT_ERR_NOT_INITIALIZED 8

/* Element types, numbered as mruntime::DType (reference include/mruntime/dtype.h:12-16). */
#define MRT_FP16 0
#define MRT_BF16 1
#define MRT_FP32 2

/* mrt_gemm flags. */
#define MRT_GEMM_BIAS 1u /* add the weight's attached bias after rounding, see mrt_weight_attach_bias */

typedef struct mrt_weight_s* mrt_weight;
typedef struct mrt_tp_s* mrt_tp;

/* ---------------------------------------------------------------- runtime */

/* Library version (major*10000 + minor*100 + patch). */
int mrt_version(void);

/* Make `device` current for this thread and create its context (scratch
 * buffers, device error flag, TMA encoder).  Idempotent.  Replaces the
 * construction of CpuBackend (reference include/mruntime/cpu_backend.h:10-11). */
int mrt_init(int device);

/* Text of the last error raised on this thread ("" if none). */
const char* mrt_last_error_string(void);

/* Wait for all work on `stream` (and for the host copies that
 * mrt_gemm_host_async queued on the library's copy streams), then read and
 * clear the device-side error flag that bounded waits inside the kernels set
 * when they give up.  Returns MRT_ERR_TIMEOUT if a kernel reported a
 * timed-out wait. */
int mrt_sync(void* stream);

/* Grow the context's scratch buffer to at least `bytes` now (call before
 * capturing a CUDA graph that contains split-K or argmax launches). */
int mrt_reserve_workspace(size_t bytes);

/* Number of streaming multiprocessors of the current device. */
int mrt_device_sm_count(int* out);

/* Kernels this library has launched in this process so far (all devices). */
int mrt_launch_count(int64_t* out);

/* Self-test of the kernels' bounded waits: launches one block that waits on
 * an mbarrier no thread ever arrives at, with the same wait routine the GEMM
 * kernels use but a limit of `limit_ms` milliseconds.  The wait gives up,
 * records its error code and the kernel returns; the call then reports
 * MRT_ERR_TIMEOUT through mrt_sync and leaves the context usable.  No
 * counterpart in the reference (it has no device code). */
int mrt_selftest_wait_timeout(int limit_ms, void* stream);

/* ---------------------------------------------------------------- device storage */

/* Device-resident tensor storage: the device counterpart of Tensor::empty's
 * host heap allocation (reference src/core/tensor.cpp:8-12).  Blocks are at
 * least 256-byte aligned. */
int mrt_device_alloc(size_t bytes, void** out);
int mrt_device_free(void* p);

/* Copy `bytes` between any two of host / device memory (direction inferred
 * from the pointers), ordered on `stream`; waits for completion when either
 * side is pageable host memory. */
int mrt_memcpy(void* dst, const void* src, size_t bytes, void* stream);

/* Where a pointer lives: 0 = host (pageable or pinned), 1 = device memory,
 * 2 = managed memory. */
#define MRT_PTR_HOST 0
#define MRT_PTR_DEVICE 1
#define MRT_PTR_MANAGED 2
int mrt_pointer_kind(const void* p, int* kind);

/* ---------------------------------------------------------------- weights */

/*
 * Upload a weight (or a tensor-parallel shard of it) once and convert it to
 * the FP16 K-major layout the kernels stream.  Replaces the reference's
 * SafeTensorsFile::load_tensor_copy of a projection weight
 * (src/loader/safetensors.cpp:166-172) together with the packed-RHS cache of
 * CpuBackend::get_or_create_packed_rhs_fp16 (src/core/cpu_backend.cpp:24-70):
 * BF16 and FP32 sources are rounded to FP16 with the same converter the
 * reference's packing step uses (cpu_backend.cpp:48-63), once, on the device.
 *
 *   src        full weight W[N, K] of dtype src_dtype (host or device memory)
 *   row_ranges NULL for all rows, else n_ranges pairs [begin, end) of rows of
 *              W kept, in order (column-parallel shard of a fused weight takes
 *              one range per part)
 *   k_begin/k_end  columns of W kept ([0, K) for the whole row; a row-parallel
 *              shard keeps a slice)
 * The handle is the cache key (not the source address), so a freed and
 * reused host buffer cannot hit a stale entry.
 */
int mrt_weight_upload(const void* src, int src_dtype, int src_on_device, int64_t N, int64_t K,
                      const int64_t* row_ranges, int64_t n_ranges, int64_t k_begin, int64_t k_end,
                      void* stream, mrt_weight* out);

/* Attach a bias vector b[N] (full length of the original weight; the
 * handle's row ranges pick the shard).  It is stored in FP16 after the
 * reference's load-time conversion (src/models/qwen/qwen_model.cpp:93-101). */
int mrt_weight_attach_bias(mrt_weight w, const void* src, int src_dtype, int src_on_device,
                           void* stream);

/* Borrow an FP16 weight W[N, K] that already lives in device memory, without
 * copying (the caller keeps it alive until mrt_weight_free of the view). */
int mrt_weight_view(const void* w_dev_f16, int64_t N, int64_t K, mrt_weight* out);

int mrt_weight_free(mrt_weight w);

/* Rows (N) and columns (K) of the uploaded shard. */
int mrt_weight_shape(mrt_weight w, int64_t* n, int64_t* k);

/* The weight's FP16 device storage in the library's layout: row-major [N, K]
 * for views and for K not a multiple of 8; otherwise 128 x 64 tiles
 * ([N_pad/128][ceil(K/64)][128][64], N_pad a multiple of 256, zero padding)
 * stored in the order the tensor cores read them with 128-byte swizzling
 * (16-byte chunk c of row r at chunk position c ^ (r % 8)), so each tile is
 * one contiguous bulk copy.  *tiled (may be NULL) tells which. */
int mrt_weight_data(mrt_weight w, void** dev_ptr, int* tiled);

/* Copy the weight as row-major FP16 [N, K] (row stride ld) to dst_dev. */
int mrt_weight_read(mrt_weight w, void* dst_dev, int64_t ld, void* stream);

/* ---------------------------------------------------------------- GEMM */

/*
 * y_dev[M, N] (row stride ldy, FP16) = fp16(x_dev[M, K] (row stride ldx, FP16) * W^T).
 * With MRT_GEMM_BIAS the attached bias is added as the reference's q/k/v
 * bias step does it: fp16(fp32(fp16(acc)) + fp32(bias))
 * (src/models/qwen/qwen_model.cpp:130-155).
 * Both regimes run the tcgen05 tensor-core kernel: M <= 64 (decode) with the
 * weight as the 128-row MMA operand streamed from HBM, larger M with X.  One
 * token on a tiled weight of at most 20 MB runs a SIMT GEMV instead (no
 * scratch memory; MRT_GEMV=0/1 never/always for 1..4 tokens).  Replaces Backend::gemm (include/mruntime/backend.h:13-21)
 * as implemented by CpuBackend::gemm (src/core/cpu_backend.cpp:72-169).
 */
int mrt_gemm(mrt_weight w, const void* x_dev, int64_t ldx, void* y_dev, int64_t ldy, int64_t M,
             unsigned flags, void* stream);

/* The kernel mrt_gemm would run for an M x N x K product on a device with
 * `sms` multiprocessors (0 = the current device): kernel 1 = tcgen05 with X
 * as the 128-row MMA operand (M > 64), 2 = tcgen05 in swap mode with the
 * weight as the 128-row operand and the tokens as N (M <= 64), 3 = swap mode
 * whose K-slices (every tile split, 2..8 slices, one per CTA) are summed
 * inside thread-block clusters on the current device, 4 = kernel 1 on SM
 * pairs, 5 = the SIMT GEMV (one token, a tiled weight of at most 20 MB;
 * bn 0, no tiles, kb_per = the k-blocks of K, grid = its CTAs); then the
 * tile's bn, the number of tiles run over the whole K, the K-slices of each
 * remaining tile, k-blocks per slice and the persistent grid.  Host-only. */
int mrt_gemm_plan(int64_t M, int64_t N, int64_t K, int sms, int* kernel, int* bn, int* full_tiles,
                  int* tail_splits, int* kb_per, int* grid);

/* Gate|up projection with SwiGLU: w's rows interleave the gate and up
 * projections (row 2j = gate row j, row 2j + 1 = up row j, N = 2 I rows) and
 * act_dev[m][j] = fp16(silu(fp16(x.gate_j)) * fp16(x.up_j)), act of I columns
 * with row stride ld_act >= I -- the reference's gate GEMM, up GEMM, FP16
 * SiLU and multiply (qwen_model.cpp:278-285) in one call.  Plans that keep
 * whole tiles do it in the GEMM's epilogue; K-split plans store the product
 * in per-device scratch and run one more kernel. */
int mrt_gemm_swiglu(mrt_weight w, const void* x_dev, int64_t ldx, void* act_dev, int64_t ld_act, int64_t M,
                    void* stream);

/* Same product without the final rounding: y_dev is FP32.  Used for the
 * partial sums of a row-parallel (K-split) shard before the all-reduce. */
int mrt_gemm_f32(mrt_weight w, const void* x_dev, int64_t ldx, float* y_dev, int64_t ldy,
                 int64_t M, void* stream);

/* mrt_gemm followed by the residual add the reference applies to the o and
 * down projections' outputs (src/models/qwen/qwen_model.cpp:316 and 324, the
 * add op of src/core/cpu_backend.cpp:430-455), in the GEMM's epilogue:
 * y[m][n] = fp16(res[m][n] + fp16(x.W_n (+ bias))), res_dev FP16 [M, N] with
 * row stride ldr >= N.  y_dev may be res_dev (in place).  flags as mrt_gemm. */
int mrt_gemm_residual(mrt_weight w, const void* x_dev, int64_t ldx, const void* res_dev, int64_t ldr,
                      void* y_dev, int64_t ldy, int64_t M, unsigned flags, void* stream);

/* mrt_gemm on host buffers, the reference's own calling convention (its
 * Tensors live in host memory): copies x_host to the device, runs the
 * product, copies y back and waits.  x is [M, K] and y [M, N], both dense. */
int mrt_gemm_host(mrt_weight w, const void* x_host, void* y_host, int64_t M, unsigned flags,
                  void* stream);

/* mrt_gemm_host without waiting, for hosts that queue several products on
 * host buffers: both buffers must be page-locked (cudaHostAlloc /
 * cudaHostRegister) and stay valid, x unmodified and y unread, until
 * mrt_sync(stream) returns.  Rows travel in chunks on the library's copy
 * streams as in mrt_gemm_host; consecutive calls use four device staging
 * sets in turn, so earlier calls' copies to the host overlap later calls'
 * copies to the device and their products (PCIe carries both directions at
 * once: queue calls with large outputs before calls with large inputs).
 * Every call of a thread must use one stream. */
int mrt_gemm_host_async(mrt_weight w, const void* x_host, void* y_host, int64_t M, unsigned flags,
                        void* stream);

/*
 * The full Backend::gemm contract (include/mruntime/backend.h:13-21) for call
 * patterns the model never issues: any of FP16/BF16/FP32 for A, B and C,
 * trans_a/trans_b, alpha and beta, unaligned shapes.  A is [a_rows, a_cols],
 * B is [b_rows, b_cols], C is [M, N] dense.  Each output is one FP32 sum in
 * k order followed by *alpha, +beta*C and the reference's rounding, like the
 * scalar path of src/core/cpu_backend.cpp:139-168.  Device pointers only.
 */
int mrt_gemm_general(const void* a_dev, int a_dtype, int64_t a_rows, int64_t a_cols,
                     const void* b_dev, int b_dtype, int64_t b_rows, int64_t b_cols, void* c_dev,
                     int c_dtype, float alpha, float beta, int trans_a, int trans_b, void* stream);

/* ---------------------------------------------------------------- logits */

/*
 * Greedy argmax of each of M rows of FP16 logits (row stride ld): the first
 * index holding the largest value, NaN never chosen, an all -inf/NaN row
 * gives 0 -- the selection of InferenceEngine::sample
 * (src/engine/inference_engine.cpp:84-95).  Writes the winning index plus
 * index_base (int64) and its value (FP32) per row; either output may be NULL.
 */
int mrt_argmax_f16(const void* logits_dev, int64_t M, int64_t V, int64_t ld, int64_t index_base,
                   int64_t* idx_dev, float* val_dev, void* stream);

/*
 * mrt_argmax_f16 for callers that must not allocate device memory: the same
 * kernels and results, but the per-chunk partials live in a fixed buffer
 * compiled into the library (96 KiB per device, held by every GPU that loads
 * the library until the process exits) instead of the context's growable
 * scratch, and the call never reaches cudaMalloc or cudaFree.  Who needs it:
 * a host that captures its whole decode step in a CUDA graph (an allocation,
 * or the device-wide synchronisation a cudaFree implies, cannot happen inside
 * the capture), and serving runtimes that reserve all device memory for their
 * own arenas up front.  Limit: M * ceil(V / 8192) <= 8192 (e.g. up to 431
 * rows of a 152064-entry vocabulary); larger calls fail with MRT_ERR_SHAPE.
 * The first call on a device resolves the buffer's device address (module
 * set-up inside the CUDA driver), so make it once before any stream capture.
 * Outside capture every call looks the address up again (no allocation), so
 * the entry point keeps working after cudaDeviceReset recreates the context;
 * inside a capture it uses the address of the last call on that device.
 * All calls share the buffer, so calls that overlap on the GPU (different
 * streams, or the same stream from several threads without ordering) race;
 * every slot a call reads was written earlier in the same call, so nothing
 * needs clearing between calls.  No counterpart in the reference.
 */
int mrt_argmax_f16_noalloc(const void* logits_dev, int64_t M, int64_t V, int64_t ld, int64_t index_base,
                           int64_t* idx_dev, float* val_dev, void* stream);

/* lm_head and greedy pick in one call: logits_dev[M, N] = x * W^T (FP16),
 * then the greedy pick of every row (src/models/qwen/qwen_model.cpp:374
 * followed by src/engine/inference_engine.cpp:84-95).  index_base offsets the
 * indices of a vocabulary shard.  For M <= 64 the GEMM's epilogue reduces each
 * 32 vocabulary rows to their best (value, index) per token and one small
 * kernel picks among those, so logits_dev may be NULL (the logits are then
 * never written); larger M, or a NULL logits_dev there, computes the logits
 * (in per-device scratch when NULL) and runs mrt_argmax_f16's two passes. */
int mrt_lm_head_argmax(mrt_weight w, const void* x_dev, int64_t ldx, int64_t M, void* logits_dev,
                       int64_t index_base, int64_t* idx_dev, float* val_dev, void* stream);

/* ---------------------------------------------------------------- conversions */

/* Element-wise conversions on the device with the reference's rounding
 * (include/mruntime/dtype.h:39-194): src_dtype -> dst_dtype, n elements. */
int mrt_convert(const void* src_dev, int src_dtype, void* dst_dev, int dst_dtype, int64_t n,
                void* stream);

/* ---------------------------------------------------------------- support ops */

/*
 * The other Backend operations (reference include/mruntime/backend.h:23-73),
 * on device pointers, so a model can run with every tensor on the device.
 * They restate src/core/cpu_backend.cpp:171-569.  Rounding: element-wise
 * results are computed in FP32 and stored with the reference's converters;
 * SiLU on FP16 uses a 65536-entry table built on the host with the
 * reference's own float expression (x / (1 + exp(-x)), glibc exp), and RoPE's
 * cos/sin are built on the host with the reference's expressions
 * (cpu_backend.cpp:363-366), so both match the reference bit for bit.
 * Reductions (RMSNorm's sum of squares, softmax and attention sums) use
 * parallel FP32 trees; their results agree with the reference within FP32
 * rounding.
 */
int mrt_rmsnorm(const void* in_dev, int in_dtype, const void* w_dev, int w_dtype, void* out_dev,
                int out_dtype, int64_t rows, int64_t hidden, float eps, void* stream);
int mrt_rope(void* x_dev, int dtype, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
             int64_t position_offset, float theta, void* stream);
int mrt_silu(const void* in_dev, int in_dtype, void* out_dev, int out_dtype, int64_t n, void* stream);
int mrt_mul(const void* a_dev, int a_dtype, const void* b_dev, int b_dtype, void* out_dev, int out_dtype,
            int64_t n, void* stream);
int mrt_add(const void* a_dev, int a_dtype, const void* b_dev, int b_dtype, void* out_dev, int out_dtype,
            int64_t n, void* stream);
int mrt_softmax(const void* in_dev, int in_dtype, void* out_dev, int out_dtype, int64_t outer, int64_t dim,
                int64_t inner, void* stream);
/* token_ids in host memory; each is checked against vocab (std::out_of_range in
 * the reference, cpu_backend.cpp:533-537, MRT_ERR_INVALID_ARG here). */
int mrt_embedding(const void* w_dev, int w_dtype, int64_t vocab, int64_t hidden, const int32_t* token_ids,
                  int64_t n, void* out_dev, int out_dtype, void* stream);
/* Q [batch, heads, q_len, qk_dim], K [batch, heads, kv_len, qk_dim],
 * V [batch, heads, kv_len, v_dim], out [batch, heads, q_len, v_dim], each with
 * its own element strides (4 per tensor).  Causal masking keeps key positions
 * <= kv_len - q_len + query index (cpu_backend.cpp:233-247). */
int mrt_attention(const void* q_dev, int q_dtype, const int64_t* q_strides, const void* k_dev, int k_dtype,
                  const int64_t* k_strides, const void* v_dev, int v_dtype, const int64_t* v_strides,
                  void* out_dev, int out_dtype, const int64_t* out_strides, int64_t batch, int64_t heads,
                  int64_t q_len, int64_t kv_len, int64_t qk_dim, int64_t v_dim, float scale, int causal,
                  void* stream);

/* ---------------------------------------------------------------- tensor parallel */

/*
 * Shard map.  Column-parallel weights (q/k/v, gate/up, lm_head) keep rows:
 * for a weight made of n_parts stacked parts (e.g. q,k,v or gate,up) rank r
 * keeps, from every part p of size part_rows[p], the rows
 * [off_p + r*part_rows[p]/world, off_p + (r+1)*part_rows[p]/world), so every
 * rank holds matching columns of each part.  Writes 2*n_parts int64 into
 * ranges_out.  Row-parallel weights (o_proj, down) keep the column slice
 * returned by mrt_shard_cols.  The reference has no parallelism beyond its
 * thread pool (src/core/cpu_backend.cpp:139-168); this is new.
 */
int mrt_shard_rows(const int64_t* part_rows, int64_t n_parts, int world, int rank,
                   int64_t* ranges_out);
int mrt_shard_cols(int64_t K, int world, int rank, int64_t* k_begin, int64_t* k_end);

/* NCCL unique id for a new tensor-parallel group (written to id_out, len >= 128). */
int mrt_tp_unique_id(void* id_out, size_t len);

/* Join a group of `world` ranks (one process per GPU) with the id rank 0 made.
 * Blocks until every rank has joined.  Uses the NCCL already loaded in the
 * process when there is one. */
int mrt_tp_init(int rank, int world, const void* id, size_t len, mrt_tp* out);
int mrt_tp_destroy(mrt_tp tp);

/* Row-parallel output: sum the FP32 partials of all ranks in place, then
 * round once to FP16 into out_dev (count elements; out may alias nothing). */
int mrt_tp_allreduce_f32_to_f16(mrt_tp tp, float* partial_dev, void* out_dev, int64_t count,
                                void* stream);

/* Column-parallel gather: every rank's FP16 [M, n_local] block is assembled
 * into out_dev[M, world*n_local] in rank order. */
int mrt_tp_allgather_cols_f16(mrt_tp tp, const void* local_dev, int64_t M, int64_t n_local,
                              void* out_dev, void* stream);

/* Row-parallel outputs summed over NVLink by this library's kernels (no
 * NCCL): the exchange the reference's o_proj and down_proj outputs need once
 * those projections are split along K (src/models/qwen/qwen_model.cpp:256, 288).
 * mrt_tp_p2p_init (collective, every rank) allocates and exports by CUDA IPC a
 * region of max_count FP32 partials + max_count FP16 outputs per rank and maps
 * the peers' regions; it fails with MRT_ERR_CUDA when peer memory cannot be
 * mapped (then use mrt_tp_allreduce_f32_to_f16).  mrt_tp_p2p_buffers returns
 * this rank's partial and output areas.
 * mrt_tp_p2p_allreduce_f32_to_f16 (collective, same order on every rank):
 * every rank's count partials (written to its partial area by the work
 * before it on the stream) are summed in rank order, rounded once to FP16 and
 * left in every rank's output area, identical on all ranks; when out_dev is
 * given (not the output area) the result is also copied there as rows of
 * row_len with stride ld_out.  Waits are bounded (2 s; mrt_sync then reports
 * MRT_ERR_TIMEOUT).  The output area stays valid until the next exchange.
 * mrt_tp_gemm_rowpar: mrt_gemm_f32 of this rank's K-shard into the partial
 * area, then the exchange into y_dev [M, N] (row stride ldy). */
int mrt_tp_p2p_init(mrt_tp tp, int64_t max_count);
int mrt_tp_p2p_buffers(mrt_tp tp, float** partial_dev, void** out_dev);
int mrt_tp_p2p_allreduce_f32_to_f16(mrt_tp tp, int64_t count, void* out_dev, int64_t ld_out, int64_t row_len,
                                    void* stream);
int mrt_tp_gemm_rowpar(mrt_tp tp, mrt_weight w, const void* x_dev, int64_t ldx, int64_t M, void* y_dev,
                       int64_t ldy, void* stream);

/* Vocabulary-sharded greedy pick: combine each rank's per-row (value, global
 * index) into the global first maximum; idx_out_dev[M] is the same on every
 * rank. */
int mrt_tp_argmax(mrt_tp tp, const float* val_dev, const int64_t* idx_dev, int64_t M,
                  int64_t* idx_out_dev, void* stream);

/* ------------------------------------------------------------ decoder
 * Device-resident greedy generation for Qwen2-architecture decoders: the
 * reference's QwenModel (src/models/qwen/qwen_model.cpp, forward 104-376) run
 * by InferenceEngine::generate with greedy selection
 * (src/engine/inference_engine.cpp:26-95).  Weights, KV cache and activations
 * live in HBM; each decode step after the first is one CUDA-graph replay.
 * Replaces constructing QwenModel + InferenceEngine over a Backend.
 */
typedef struct mrt_decoder_config {
    int64_t vocab_size;         /* QwenConfig fields (include/mruntime/qwen_model.h) */
    int64_t hidden_size;
    int64_t num_layers;
    int64_t num_attention_heads;
    int64_t num_kv_heads;
    int64_t intermediate_size;
    int64_t max_seq_len;        /* KV-cache capacity: prompt + generated tokens */
    float rms_norm_eps;
    float rope_theta;
} mrt_decoder_config;

typedef struct mrt_decoder_s* mrt_decoder;

typedef struct mrt_decoder_stats {
    float prefill_ms;       /* batched prompt forward + first greedy pick */
    float first_step_ms;    /* the first decode step (run eagerly, sizes scratch) */
    float decode_ms;        /* the remaining decode steps (graph replays) */
    int64_t decode_steps;   /* number of steps in decode_ms */
} mrt_decoder_stats;

int mrt_decoder_create(const mrt_decoder_config* cfg, mrt_decoder* out);

/* The same decoder, tensor-parallel over the ranks of `tp` (one process per
 * GPU, every rank loads the full tensors and keeps its shard): q|k|v and
 * gate|up column-parallel, o and down row-parallel (FP32 partials all-reduced
 * and rounded once), lm_head sharded by vocabulary with the greedy pick
 * combined across ranks, embedding and norms replicated.  Ranks own whole kv
 * groups when world divides num_kv_heads; otherwise each kv head is kept on
 * world / num_kv_heads ranks that split its query heads.  Every rank must
 * make the same calls with the same prompt; all return the same tokens. */
int mrt_decoder_create_tp(const mrt_decoder_config* cfg, mrt_tp tp, mrt_decoder* out);

/* One checkpoint tensor by its Hugging Face / reference name
 * (qwen_model.cpp:54-101, 336-353): "model.embed_tokens.weight",
 * "model.layers.<i>.{input_layernorm,post_attention_layernorm}.weight",
 * "model.layers.<i>.self_attn.{q,k,v,o}_proj.weight",
 * "model.layers.<i>.self_attn.{q,k,v}_proj.bias",
 * "model.layers.<i>.mlp.{gate,up,down}_proj.weight", "model.norm.weight",
 * "lm_head.weight" (optional: tied to the embedding when absent).  rows x cols
 * is the tensor's shape (cols = 1 for vectors); dtype FP16/BF16/FP32; src in
 * host or device memory (a device source is read after the whole device
 * synchronises, so any stream may have produced it).  Unknown names are
 * MRT_ERR_INVALID_ARG. */
int mrt_decoder_load(mrt_decoder d, const char* name, const void* src, int src_dtype, int src_on_device,
                     int64_t rows, int64_t cols);

/* Greedy generation: prompt[n_prompt] (host) -> out_tokens[max_new] (host),
 * stopping after eos_token_id (< 0: never); *n_out = tokens written.  Needs
 * n_prompt + max_new - 1 <= max_seq_len.  Synchronous, like the reference;
 * stream (may be NULL) is waited on first.  stats may be NULL. */
int mrt_decoder_generate(mrt_decoder d, const int32_t* prompt, int64_t n_prompt, int64_t max_new,
                         int32_t eos_token_id, int32_t* out_tokens, int64_t* n_out,
                         mrt_decoder_stats* stats, void* stream);

/* Releases the decoder.  For a tensor-parallel decoder this is collective:
 * every rank calls it (ranks unmap each other's exchange buffers first). */
void mrt_decoder_free(mrt_decoder d);

/* ---------------------------------------------------------------- checkpoints */

/*
 * Safetensors checkpoints read straight into device memory.  Replaces the
 * reference's SafeTensorsFile (include/mruntime/safetensors.h:19-53,
 * src/loader/safetensors.cpp:71-172): the file is mmap'ed and its JSON header
 * parsed with the same rules (8-byte little-endian header length,
 * "__metadata__" skipped, dtypes F16 / BF16 / F32, any other dtype an error),
 * plus checks the reference leaves out (data offsets inside the file, byte
 * count equal to dtype x shape).  Tensor bytes travel from the mapping to HBM
 * through two pinned 16 MiB staging buffers, the host copy of one chunk
 * overlapping the DMA of the previous one, instead of load_tensor_copy's
 * host memcpy (safetensors.cpp:166-172).
 */
typedef struct mrt_safetensors_s* mrt_safetensors;

/* Open and index a checkpoint (SafeTensorsFile::open, safetensors.cpp:71-131).
 * Host-only: needs no device. */
int mrt_safetensors_open(const char* path, mrt_safetensors* out);
int mrt_safetensors_close(mrt_safetensors f);

/* Tensor count, and the i-th name in sorted order (tensor_names(),
 * safetensors.cpp:148-155); the name stays valid until close.  Host-only. */
int mrt_safetensors_count(mrt_safetensors f, int64_t* n);
int mrt_safetensors_name(mrt_safetensors f, int64_t i, const char** name);

/* dtype (MRT_FP16/BF16/FP32), rank, shape (up to 8 entries written) and byte
 * size of a tensor (tensor_info, safetensors.cpp:144-146); an unknown name is
 * MRT_ERR_INVALID_ARG (the reference throws std::out_of_range).  Host-only. */
int mrt_safetensors_info(mrt_safetensors f, const char* name, int* dtype, int* ndim, int64_t* shape,
                         uint64_t* nbytes);

/* The tensor's raw bytes into dst (host or device memory, at least its byte
 * size): the device path stages through pinned memory and waits before
 * returning (load_tensor_copy, safetensors.cpp:166-172, with the copy landing
 * in HBM). */
int mrt_safetensors_read(mrt_safetensors f, const char* name, void* dst, uint64_t dst_bytes, void* stream);

/* mrt_weight_upload of a 2-D checkpoint tensor (with the same shard
 * arguments), its bytes taken from the file through pinned staging: the
 * weight is converted and tiled on the device, once. */
int mrt_safetensors_upload_weight(mrt_safetensors f, const char* name, const int64_t* row_ranges, int64_t n_ranges,
                                  int64_t k0, int64_t k1, void* stream, mrt_weight* out);

/* Every tensor of the checkpoint the decoder takes (QwenModel::load_weights,
 * src/models/qwen/qwen_model.cpp:336-353: other tensors are ignored, as
 * there) through mrt_decoder_load with a device source; *n_loaded (may be
 * NULL) counts them.  A tensor-parallel decoder keeps its shard of each. */
int mrt_decoder_load_safetensors(mrt_decoder d, mrt_safetensors f, int64_t* n_loaded);

#ifdef __cplusplus
}
#endif
#endif /* MRT_B200_H */
