// Whole-step fused decode for the Qwen3-0.6B shape (dim 1024, 16 Q / 8 KV heads of 128,
// MLP 3072): one persistent cooperative kernel per call runs every layer, the final norm, the
// tied lm_head and the greedy argmax for n_steps tokens.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3_common.cuh"
#include "q3_model.cuh"

namespace q3 {

constexpr int kFusedMaxRanks = 8;

// FusedLayer (the per-layer weight copies the kernel streams) is declared in q3_model.cuh.

struct FusedArgs {
    const FusedLayer* layers;    // device array [n_layers]
    const uint16_t* embed;       // [vocab, 1024] (original layout, for the embedding gather)
    const uint16_t* lm_head;     // classifier rows, swizzled copy
    const uint16_t* final_norm;  // [1024]
    uint16_t* k_cache;           // paged pools [page][8][16][128], layer l at + l * layer_elems
    uint16_t* v_cache;
    size_t layer_elems;
    const int32_t* page_table;
    const float2* rope;          // [rope_len][64] (cos, sin)
    int rope_len;
    float* ybuf;                 // [2][n_layers][copies][1024] down-projection accumulators (by
                                 // step parity), fused_ybuf_floats(); the first step's parity
                                 // zero at launch (each step zeroes the other parity, which
                                 // the next step - of this launch or the next - uses)
    int parity0;                 // accumulator parity of the first step
    unsigned long long* qkvt;    // [4096] q|k|v, tagged (value bits | tag << 32)
    unsigned long long* opart;   // [8][1024] o_proj partial of each KV-head group, tagged
    unsigned epoch;              // tag base of this launch (differs from the previous launch)
    float* part_o;               // [16][s_max][128]  (long-context attention)
    float2* part_ml;             // [16][s_max]
    float2* am_part;             // [grid] per-CTA (value, index) of the lm_head rows
    float* logits;               // [vocab]
    float* taps;                 // nullable: [(n_layers+1), 1024]
    StepParams* sp;              // device step parameters: read at launch unless sp_from_args,
                                 // advanced past the last step at the end
    StepParams sp_init;          // the first step's parameters when sp_from_args
    int sp_from_args;    int32_t* token_log;
    const int32_t* forced;       // nullable: teacher-forced tokens
    unsigned* bar;               // grid arrival counter: zero at launch; CTA 0 sets it back to
                                 // zero once every arrival of the launch has been made
    unsigned* err;               // error word: 1 = a bounded wait gave up
    int n_layers, vocab, ctx, n_steps, s_max;
    float eps;
    long long spin_cycles;       // bound of every wait, in SM clock cycles
    int barrier_offset;          // 0; a test sets 1 so that a grid wait can never complete
    int l2_ahead;                // layers of weights the producer prefetches into L2 ahead of its
                                 // ring copies (0: none)
    unsigned long long* prof;    // nullable: per (phase, CTA) globaltimer stamps [k][G][8]
    unsigned long long* dbg;     // nullable: first failed self-check (builds with Q3_FUSED_CHECKS)

    // Tensor parallelism (one kernel per GPU, `world` ranks). This rank runs KV-head groups
    // [kv0, kv0 + nkv) (layers[].wqkv then holds only their [wq;wk;wv] rows: q rows of the 2 nkv
    // query heads, k rows, v rows), MLP indices [rank hl, rank hl + hl) (layers[].w1 / w3 / w2t
    // point at them) and lm_head rows [v0, v0 + vocab). One rank: nkv 8, kv0 0, hl 3072, v0 0.
    int nkv, kv0, hl, v0;
    int world, rank;
    // xchg: exchange the down-projection sums and the greedy argmax between ranks through the
    // tagged words below (set for world > 1; at world 1 it routes them through this rank's own
    // buffers). sys: the exchanged words cross GPUs (system-scope accesses).
    int xchg, sys;
    unsigned long long* opart_dst[kFusedMaxRanks];  // every rank's opart (this rank's = opart)
    unsigned long long* yx;                          // [2][kFusedMaxRanks][1024] per-rank sums
    unsigned long long* yx_dst[kFusedMaxRanks];
    unsigned long long* amx;                         // [kFusedMaxRanks][2] (value, index) words
    unsigned long long* amx_dst[kFusedMaxRanks];
    // nullable: the last step's greedy token also goes here (pinned host memory of a one-step
    // ForwardToken + Greedy call, whose logits pointer is pinned host memory too).
    int32_t* token_out;
    // nullable: CTA 0 copies the error word here at the end of a launch that ran to completion
    // (the caller presets it to a non-zero value, so an aborted launch leaves it non-zero).
    unsigned* err_out;
};

// Tagged words of the tensor-parallel exchange region (opart [8][1024], yx, amx), in u64 words.
constexpr size_t kFusedXchgWords = 8 * 1024 + 2 * kFusedMaxRanks * 1024 + 2 * kFusedMaxRanks;

// Whether the fused kernel serves this config, and its launch geometry on `device`.
bool fused_supported(const q3_config& c);
int fused_grid(int device);
size_t fused_smem_bytes();
// Layers of weights prefetched into L2 ahead of the ring copies.
int fused_l2_ahead();
// Floats of FusedArgs::ybuf for n_layers.
size_t fused_ybuf_floats(int n_layers);
void launch_decode_fused(const FusedArgs& a, int grid, cudaStream_t s);
// Phases of one decode step at kv_len (3 per layer up to 128 positions, else 4; + lm_head).
int fused_phases_per_step(int n_layers, int kv_len);
// Re-layout kernels: wop / w2t, and the row-parity swizzle of every matrix the fused kernel
// multiplies with tensor-core MMAs (in odd rows the two 64-byte halves of each 128-byte block are
// swapped, which makes the MMA operand loads from shared memory bank-conflict free).
void launch_permute_wo(const uint16_t* wo, uint16_t* wop, cudaStream_t s);
void launch_transpose_w2(const uint16_t* w2, uint16_t* w2t, cudaStream_t s);
void launch_swizzle_rows(const uint16_t* src, uint16_t* dst, size_t rows, int K, cudaStream_t s);

}  // namespace q3
