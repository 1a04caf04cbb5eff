// Whole-step fused decode for the Qwen3-0.6B shape (dim 1024, 16 Q / 8 KV heads of 128,
// MLP 3072): one persistent cooperative kernel per call runs every layer, the final norm, the
// tied lm_head and the greedy argmax for n_steps tokens.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3_common.cuh"
#include "q3_model.cuh"

namespace q3 {

struct FusedArgs {
    const LayerWeights* layers;  // device array [n_layers]
    const uint16_t* embed;       // [vocab, 1024] (also the tied classifier)
    const uint16_t* lm_head;     // classifier rows (== embed when tied)
    const uint16_t* final_norm;  // [1024]
    uint16_t* k_cache;           // paged pools, layer l at + l * layer_elems
    uint16_t* v_cache;
    size_t layer_elems;
    const int32_t* page_table;
    const float2* rope;          // [rope_len][64]
    int rope_len;
    float* x;                    // [1024] residual stream
    float* qkv;                  // [4096]
    float* h;                    // [3072]
    float* part_o;               // [16][s_max][128]
    float2* part_ml;             // [16][s_max]
    float2* am_part;             // [grid] per-CTA (value, index) of the lm_head rows
    float* logits;               // [vocab]
    float* taps;                 // nullable: [(n_layers+1), 1024]
    StepParams* sp;
    int32_t* token_log;
    const int32_t* forced;       // nullable: teacher-forced tokens
    unsigned* bar;               // grid arrival counter, zero at launch
    unsigned* err;               // error word: 1 = a bounded wait gave up
    int n_layers, vocab, ctx, n_steps, s_max;
    float eps;
    long long spin_cycles;       // bound of every wait, in SM clock cycles
    int barrier_offset;          // 0; a test sets 1 so that a grid wait can never complete
};

// Whether the fused kernel serves this config, and its launch geometry on `device`.
bool fused_supported(const q3_config& c);
int fused_grid(int device);
size_t fused_smem_bytes();
void launch_decode_fused(const FusedArgs& a, int grid, cudaStream_t s);

}  // namespace q3
