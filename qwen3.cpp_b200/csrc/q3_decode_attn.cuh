// Decode attention over the paged KV cache on the CUDA cores: the reference's FastAttn + Softmax
// (src/inference.cpp:1017-1058, :925-946) for the one new position of every sequence of a batch,
// or for the local KV heads of a tensor-parallel rank. The work is split over the cached pages
// (flash-decoding), so that every SM streams pages at once; the last split of a (sequence, KV
// head) to finish merges the partial results.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace q3 {

struct DecodeAttnArgs {
    const float* q;            // fp32 query rows (QK-normed, rotated): local KV head g's query heads
                               // 2g, 2g+1 at q + row * q_stride + 2g * 128
    int q_stride;
    const uint16_t* k_cache;   // one layer: [page][n_kv_cache][16][128] bf16
    const uint16_t* v_cache;
    const int32_t* page_table; // row b reads page_table + b * pages_per_seq
    int pages_per_seq;
    const int32_t* dec_pos;    // [rows] position of the new token; positions [0, pos] are cached
    int rows, n_kv;            // local KV heads per row
    int kv_head0, n_kv_cache;  // local KV head g is cache head kv_head0 + g of n_kv_cache
    int pages_per_split, max_splits;
    float* part_o;             // [rows * n_kv][max_splits][2][128]
    float2* part_ml;           // [rows * n_kv][max_splits][2] (max, sum)
    unsigned* counter;         // [rows * n_kv], zero; reset by the merging split
    uint16_t* out;             // nullable: bf16 attention output, heads 2g, 2g+1 at
                               // out + row * out_stride + 2g * 128
    uint16_t* out_lo;          // nullable: bf16(o - out), the low part of a split activation
    float* out_f32;            // nullable: the fp32 output, same layout
    int out_stride;
};

// Pages per split for `rows` x `n_kv` (sequence, KV head) pairs of at most max_pages pages each:
// enough splits for several blocks per SM.
int decode_attn_pages_per_split(int rows, int n_kv, int max_pages, int num_sms);
void launch_decode_attention(const DecodeAttnArgs& a, cudaStream_t s);

}  // namespace q3
