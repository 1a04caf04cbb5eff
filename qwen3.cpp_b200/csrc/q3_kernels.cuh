// Layer-wise kernels of the B200 Qwen3 forward pass (any config shape). The fused
// whole-step decode kernel for the Qwen3-0.6B shape lives in q3_decode_fused.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3_common.cuh"

namespace q3 {

// GEMV epilogues.
enum GemvEpi : int {
    kEpiStore = 0,     // out[r] = W[r] . xin
    kEpiResidual = 1,  // out[r] += W[r] . xin            (x += proj, src/inference.cpp:847-849)
    kEpiSiluMul = 2,   // out[r] = silu(W[r].xin) * (Wb[r].xin)   (src/inference.cpp:1009-1011)
};

// out = epilogue(W . xin) with xin = RmsNorm(x, norm_w) when norm_w != nullptr, else x.
// W is [n, k] bf16 row-major. argmax_part (nullable, kEpiStore only) receives one
// (value, index) pair per block for a following greedy reduction. lin2 (nullable, kEpiSiluMul
// only) receives the raw Wb . xin values.
void launch_gemv(int epi, const uint16_t* W, const uint16_t* Wb, const float* x,
                 const uint16_t* norm_w, float eps, float* out, float* lin2, int n, int k,
                 float2* argmax_part, int grid_override, cudaStream_t s);
int gemv_grid(int n);  // blocks launch_gemv uses for n rows (argmax partial count)

// Embedding row -> fp32 hidden state (src/inference.cpp:601-603). Token read from sp.
void launch_embed(const StepParams* sp, const uint16_t* embed, float* x, int dim,
                  cudaStream_t s);

// Per-head QK-RMSNorm + RoPE of q and k (src/inference.cpp:800-810), bf16 K/V write at kv_pos
// (:812-815) and the attention-sink re-rotation (:817-827). q is updated in place inside qkv.
struct QkvArgs {
    float* qkv;                // [n_heads*hd | n_kv*hd (k) | n_kv*hd (v)]
    const uint16_t* q_norm;    // [hd]
    const uint16_t* k_norm;    // [hd]
    const float2* rope;        // [table_len][rotary_dim/2] (cos, sin)
    int rope_len;
    uint16_t* k_cache;         // paged [pages][n_kv][16][hd]
    uint16_t* v_cache;
    const int32_t* page_table; // logical page -> physical page
    const StepParams* sp;
    int n_heads, n_kv, hd, rotary_dim;
    float eps;
};
void launch_qk_rope_kv(const QkvArgs& a, cudaStream_t s);

// Split-K decode attention over a KV cache (paged, or the reference's strided layout), GQA:
// each block serves the n_heads/n_kv query heads of one KV head over one chunk of positions and
// writes (max, sum, unnormalised output) partials; attn_combine merges them
// (FastAttn + Softmax, src/inference.cpp:1017-1058, :925-946).
struct AttnArgs {
    const float* q;            // [n_heads*hd]
    const uint16_t* k;         // paged pools, or strided base (reference layout)
    const uint16_t* v;
    const int32_t* page_table; // nullptr: strided layout with row stride n_kv*hd
    const StepParams* sp;      // kv_len source (nullable: use kv_len_const)
    int kv_len_const;
    int n_heads, n_kv, hd;
    int row_stride;            // strided layout: elements between consecutive positions
    int n_splits;
    float* part_o;             // [n_heads][n_splits][hd]
    float2* part_ml;           // [n_heads][n_splits] (max, sum)
    float* out;                // [n_heads*hd]
};
void launch_attention(const AttnArgs& a, cudaStream_t s);
int attn_splits_for(int max_kv_len);

// Greedy argmax over per-block partials (lowest index wins ties, src/inference.cpp:703-709),
// and the device-side advance of a decode loop: token = argmax, pos += 1, positions recomputed.
void launch_argmax_final(const float2* part, int n_part, int32_t* out_index, StepParams* sp,
                         int32_t* token_log, int ctx, const int32_t* forced_next,
                         cudaStream_t s);

// Single-block argmax over a full vector (the free q3_greedy entry point).
void launch_argmax_full(const float* x, int n, int32_t* out, cudaStream_t s);

// Free-function kernels.
void launch_rmsnorm(float* out, const float* x, const uint16_t* w, float eps, int n,
                    cudaStream_t s);
void launch_softmax(float* out, const float* x, int n, cudaStream_t s);
struct RopeRow {
    float c[256];
    float s[256];
};
void launch_rope_row(float* x, int d, int head_dim, int rotary_dim, const RopeRow& row,
                     cudaStream_t s);

}  // namespace q3
