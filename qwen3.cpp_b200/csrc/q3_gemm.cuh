// Batched-token (prefill) contractions on the sm_100a tensor cores: C[M, N] = A[M, K] . B[N, K]^T
// with A the bf16 activations of M tokens and B a bf16 weight matrix in the reference's row-major
// [out, in] layout (both K-major), fp32 accumulation in TMEM, and the epilogue of the op that
// follows the projection fused in.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace q3 {

enum GemmEpilogue : int {
    kEpiStoreF32 = 0,  // out[m, n] = acc (fp32)
    kEpiAddF32 = 1,    // out[m, n] += acc (fp32 residual stream: x += proj)
    kEpiSwiGLU = 2,    // B rows = 128 of w1 then the same 128 of w3 per tile; out bf16 [M, N/2]:
                       // h = silu(w1 . x) * (w3 . x)
    kEpiStoreBF16 = 3, // out[m, n] = bf16(acc)
    kEpiQkvRope = 4,   // [wq;wk;wv] rows: per 128-column head QK-RMSNorm + RoPE of q and k, then q
                       // rows to GemmArgs::qkv.q_out (bf16) and k, v rows into the paged cache
};

// Destinations of the kEpiQkvRope epilogue (src/inference.cpp:800-815 for every row m, the token
// at position pos0 + m).
struct QkvEpilogue {
    uint16_t* q_out = nullptr;           // [M, n_heads * 128] bf16
    uint16_t* k_cache = nullptr;         // this layer's paged pools [page][n_kv][16][128] bf16
    uint16_t* v_cache = nullptr;
    const int32_t* page_table = nullptr; // page of positions [16p, 16p + 16)
    const float2* rope = nullptr;        // [pos][64] (cos, sin)
    const uint16_t* q_norm = nullptr;    // [128]
    const uint16_t* k_norm = nullptr;    // [128]
    int pos0 = 0, n_heads = 0, n_kv = 0;
    float eps = 0.0f;
    int q_f16 = 0;                       // q rows as fp16 instead of bf16
    // Nullable: fp16 copies of the K/V rows written to the cache (the same bf16-rounded values,
    // same paged layout), the operands of the fp16 prefill attention.
    uint16_t* k_stage = nullptr;
    uint16_t* v_stage = nullptr;
    // Rows of several sequences (nullable): row m is the token at position tok_pos[m], whose K/V
    // go to cache row tok_row[m] = physical page * 16 + position % 16 (page_table and pos0 are
    // then unused).
    const int32_t* tok_pos = nullptr;
    const int32_t* tok_row = nullptr;
};

// A 2-D K-major bf16 matrix [rows, cols] (cols contiguous) as a TMA tensor map with 128-byte
// swizzling and a box of 64 columns x box_rows rows. base must be 16-byte aligned and cols a
// multiple of 8.
void make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                    uint32_t box_rows);

// The paged KV cache of every layer, [pages][n_kv][16][128] bf16, as a 4-D TMA map
// {128, 16, n_kv, pages} with a box of 64 x 16 x 1 x 8 (eight consecutive pages of one KV head, one
// 64-column panel) and 128-byte swizzling.
void make_tmap_kv_pages(CUtensorMap* map, const void* base, uint64_t n_kv, uint64_t pages);

// As make_tmap_bf16 for a sub-matrix: rows are row_stride elements apart (a column slice of a
// wider matrix); base and row_stride * 2 bytes must be 16-byte aligned.
void make_tmap_bf16_strided(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                            uint64_t row_stride, uint32_t box_rows);

// The output [rows, cols] of a contraction (fp32, or bf16 when bf16) as a TMA map for the
// epilogue's stores: boxes of 128 bytes x 32 rows with 128-byte swizzling. cols * element size
// must be a multiple of 128 bytes.
void make_tmap_out(CUtensorMap* map, void* base, uint64_t rows, uint64_t cols, bool bf16);

struct GemmArgs {
    int M = 0, N = 0, K = 0;  // N: output columns of the tile space (2 x hidden for SwiGLU)
    unsigned* err = nullptr;  // set non-zero when a bounded wait gives up
    long long budget = 4000000000LL;  // cycles per wait
    int ksplit = 1;           // K slices (residual add only; chosen by launch_gemm)
    int bn = 0;               // tile width override (128 or 256; 0: gemm_tile_n)
    int max_ksplit = 4;       // residual add: split K up to this many slices ...
    int min_slice_kblocks = 8;  // ... of at least this many 64-wide k-blocks
    QkvEpilogue qkv;            // kEpiQkvRope only
    bool dependent = false;     // programmatic dependent launch (see launch_dep)
    // A and B are fp16 (else bf16); the SwiGLU epilogue then writes fp16 as well.
    int f16 = 0;
};

// Opts every contraction kernel into its shared memory on the current device (launch_gemm does it
// on first use; call this before capturing launches into a CUDA graph).
void prepare_gemm_kernels();

// Tile N width used for an epilogue and output width (128 or 256).
int gemm_tile_n(int epi, int N);
// Enqueues the contraction. `a` maps A [M, K] with 128-row boxes; `b` maps B [N, K] with
// box_rows = gemm_tile_n(...) (SwiGLU: `b` = w1 and `b2` = w3, each [N/2, K] with 128-row boxes);
// `out` (make_tmap_out) maps the output: fp32 [M, N] (store or residual add) or bf16 ([M, N/2]
// for SwiGLU, [M, N] for kEpiStoreBF16). K must be a multiple of 64, N a multiple of the tile
// width. Grid: one persistent CTA per SM at most. Returns cudaSuccess or the launch error.
// a_lo (optional; store, residual-add and QKV epilogues): the A operand is a + a_lo, two parts
// (bf16, or fp16 with GemmArgs::f16) of fp32 activations (same shape and boxes as a), multiplied
// into the same accumulator.
cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap* b2,
                        const CUtensorMap& out, const GemmArgs& args, int epi, int num_sms,
                        cudaStream_t stream, const CUtensorMap* a_lo = nullptr);

}  // namespace q3
