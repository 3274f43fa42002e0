// decode_step.h -- the persistent decode-step kernel: one launch runs a whole
// greedy decode step (every layer, lm_head and the pick) of a Qwen2-shaped
// decoder for one token.  Used by decoder.cu for every decode step after the
// prompt; the prompt itself goes through the per-op kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mrt {

// One layer's tensors (device pointers).  Weights are in the tiled layout
// (mrt_weight_s with tiled = true): [n_pad/128][k_tiles][128][64] FP16 tiles.
struct StepLayer {
    const uint16_t* qkv;    // q|k|v rows (local heads), K = hidden
    const uint16_t* bias;   // FP16 q|k|v bias or nullptr
    const uint16_t* o;      // [hidden, local heads * head_dim]
    const uint16_t* gu;     // gate and up rows interleaved: row 2j = gate j, 2j + 1 = up j (local I), K = hidden
    const uint16_t* down;   // [hidden, local I]
    const void* ln1;        // RMSNorm gains before attention
    const void* ln2;        // RMSNorm gains before the MLP
    int ln1_dt, ln2_dt;
    uint16_t* kc;           // K cache of this layer: [local kv heads][max_seq][head_dim]
    uint16_t* vc;
};

struct StepState {          // same layout as the decoder's device state
    int32_t pos, step, token, pad;
};

struct StepArgs {
    const StepLayer* layers;
    int L;
    int64_t H, D, nh, nkv, group, h0, g0, I, V, max_seq, n_qkv;
    const uint16_t* embed;      // [vocab, hidden] FP16 row-major
    int64_t vocab;
    const void* norm;           // final RMSNorm gains
    int norm_dt;
    const uint16_t* lm;         // tiled lm_head [V, hidden]
    float eps, scale;
    const float* cos_t;         // RoPE tables [max_seq][head_dim / 2]
    const float* sin_t;
    const uint16_t* silu_lut;   // FP16 SiLU table (65536 entries)
    // global scratch (device)
    uint16_t* x;                // residual stream [hidden]
    uint16_t* r1;               // residual after attention [hidden]
    uint16_t* qkv_out;          // [n_qkv]
    uint16_t* attn;             // [local heads * head_dim]
    uint16_t* yo;               // o projection output [hidden]
    uint16_t* act;              // SiLU(gate) * up [local I]
    uint16_t* yd;               // down projection output [hidden]
    float* part_down;           // down's split partials [grid][2][128] (own exchange buffer under TP)
    float* att_part;            // [local heads][att_split][head_dim + 2]
    int* att_cnt;               // [local heads], zero between steps
    int att_split;
    float* cand_val;            // [grid] per-CTA best logit
    int64_t* cand_idx;
    unsigned* bar;              // grid barrier: [0] arrivals; zeroed before each launch
    StepState* st;
    int32_t* tokens;
    int64_t tokens_cap;
    int* err;
    // Tensor parallelism (world > 1): o and down are row-parallel.  Each rank
    // writes its FP32 partial row to its own exchange buffer (site 0 = o,
    // 1 = down) and the ranks' rows are summed in rank order; the greedy pick
    // combines every rank's (value, global index) candidate.  Epoch of call c
    // of a step = *epoch + c + 1; CTA 0 advances *epoch by 2 L + 1 per step.
    int rank, world;
    int64_t v0;                               // first vocabulary row of this rank
    const float* peer_buf[2][8];              // every rank's partial buffers (own included)
    unsigned long long* peer_flags[8];        // every rank's flag array, indexed by source rank
    float* peer_cand[8];                      // every rank's candidate slot: value, then the index (int64)
    unsigned long long* epoch;
};

// Shared memory the kernel needs for a given operand width (elements).
size_t decode_step_smem(int64_t max_operand);
// Cooperative launch on `grid` CTAs (one per SM); `a.bar` must be zero.
cudaError_t launch_decode_step(const StepArgs& a, int grid, cudaStream_t s);
int decode_step_grid();  // CTAs per launch on the current device (0: unsupported)
const char* decode_step_diag();  // why the last launch was refused ("" if it was not)

}  // namespace mrt
