// Batched prefill of a prompt chunk (the reference prefills one token at a time through
// ForwardToken, src/inference.cpp:669-671): every projection is a tensor-core contraction over all
// tokens of the chunk (q3_gemm.cuh), attention is causal flash attention over the paged KV cache.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "q3_common.cuh"
#include "q3_model.cuh"

namespace q3 {

// Row-wise RmsNorm (src/inference.cpp:887-923) of fp32 rows into bf16 MMA operands (fp16 with
// f16); with ids non-null, the fp32 rows are first gathered from the embedding (:601-603) into x.
// out_lo (nullable) receives y - out(y), so that out + out_lo carries 16 (fp16: 22) significant
// bits. dependent: programmatic dependent launch (launch_dep).
void launch_rmsnorm_rows_bf16(const int32_t* ids, const uint16_t* embed, float* x,
                              const uint16_t* w, float eps, uint16_t* out, int rows, int dim,
                              cudaStream_t s, uint16_t* out_lo = nullptr, bool dependent = false,
                              bool f16 = false);

// Per-token, per-head QK-RMSNorm + RoPE (src/inference.cpp:800-810) and bf16 K/V write into the
// paged cache at kv_pos = pos (:812-815) for tokens at positions pos0 .. pos0+rows-1, all below
// the context length (no ring wrap). q is written as bf16 [rows, n_heads*128].
struct PrefillQkvArgs {
    float* qkv;                // [rows, (n_heads + 2*n_kv) * 128] fp32
    const uint16_t* q_norm;
    const uint16_t* k_norm;
    const float2* rope;        // [len][64] (cos, sin)
    uint16_t* q_out;           // nullable: [rows, n_heads*128] bf16
    uint16_t* k_cache;
    uint16_t* v_cache;
    const int32_t* page_table;
    int rows, pos0, n_heads, n_kv;
    float eps;
    // Decode of independent sequences: row b is at position dec_pos[b] and uses the page table
    // page_table + b * pages_per_seq (null: row i is at pos0 + i of one sequence).
    const int32_t* dec_pos = nullptr;
    int pages_per_seq = 0;
    // Tensor-parallel shard: the n_kv local KV heads are heads kv_head0.. of a cache laid out
    // for n_kv_cache heads (0: n_kv).
    int kv_head0 = 0, n_kv_cache = 0;
    int clear_input = 0;  // zero qkv after reading it (for reduce-add producers of the next step)
    float* q_out_f32 = nullptr;  // nullable: the fp32 q rows as well [rows, n_heads*128]
};
void launch_prefill_qkv(const PrefillQkvArgs& a, cudaStream_t s);

// Causal attention of `rows` query tokens (positions pos0..) over KV positions [0, pos] of the
// paged cache (FastAttn + Softmax, src/inference.cpp:1017-1058, :925-946, for every prompt token
// at once) on the tcgen05 tensor cores (q3_prefill_attn.cu); head_dim 128, two query heads per KV
// head, out bf16 [rows, n_heads*128]. q maps the bf16 q rows
// [rows, n_heads*128] with 64 x 64 boxes; k and v map each whole paged cache (every layer) as
// [n_layers * n_pages * n_kv * 16, 128] with 64 x 16 boxes, k4 and v4 as 4-D page maps
// (make_tmap_kv_pages over n_layers * n_pages pages).
struct PrefillAttnTcArgs {
    const int32_t* page_table;
    uint16_t* out;             // [rows, n_heads*128] bf16
    unsigned* err;             // set non-zero when a bounded wait gives up
    long long budget = 4000000000LL;
    int rows, pos0, n_kv, n_pages, layer;
    int pages_per_seq = 0;       // length of page_table (0: n_pages)
    uint16_t* out_lo = nullptr;  // optional: attention output - bf16(output)
    // q, K, V and the probabilities are fp16 (k and v then map fp16 copies of the cache), the
    // output is fp16 (out_lo unused).
    int f16 = 0;
    // Several sequences at once (nullable): n_work query blocks {first q/out row, rows (<= 64),
    // position of the first row, offset of the sequence's page table in page_table}, longest
    // first; rows and pos0 are then unused.
    const int4* work = nullptr;
    int n_work = 0;
};
void launch_prefill_attention_tc(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                 const CUtensorMap& k4, const CUtensorMap& v4,
                                 const PrefillAttnTcArgs& a, cudaStream_t s);

// A paged KV cache as the prefill sees it: every layer's pages back to back from k_base /
// v_base ([n_layers][n_pages][n_kv][16][128] bf16), the page table of the sequence being
// prefilled, and the RoPE table.
struct KvView {
    uint16_t* k_base = nullptr;
    uint16_t* v_base = nullptr;
    int n_pages = 0;                     // pages per layer
    const int32_t* page_table = nullptr; // logical -> physical page of this sequence
    const float2* rope = nullptr;        // [rope_len][64] (cos, sin)
    int rope_len = 0;
    int table_len = 0;                   // entries of page_table (0: n_pages)
};
KvView engine_view(Engine& e);

// fp16 copies of the five matrices of every layer ([wq;wk;wv], wo, w1, w3, w2: each bf16 value
// is an fp16 value in the range the weights take, and smaller ones round to the fp16 subnormal
// grid), in one arena; the norm pointers are those of `layers`.
void make_f16_layers(const q3_config& c, const std::vector<LayerWeights>& layers,
                     DeviceBuffer& arena, std::vector<LayerWeights>& out, cudaStream_t s);

// Driver of a batched prefill over the layers of a Model.
class Prefill {
public:
    static constexpr int kMaxChunk = 4096;  // tokens per pass; longer prompts run in chunks

    // The shapes the batched path handles (head_dim 128 with full rotary width, 2 query heads
    // per KV head, widths that tile by the contraction kernel); others prefill token by token.
    static bool supported(const q3_config& c);

    Prefill(const q3_config& c, int device);
    ~Prefill() = default;

    // Runs every layer for tokens ids_dev[0..n) at positions pos0..pos0+n-1 (pos0 + n <= ctx),
    // writing each layer's K/V rows into the engine's cache, and leaves the hidden state of the
    // last token in x_last (fp32 [dim]). taps (nullable) receive the last token's hidden state
    // before the first layer and after every layer ([(n_layers+1) * dim]).
    // layers16: the same layers with the five matrices ([wq;wk;wv], wo, w1, w3, w2) as fp16
    // copies (the norms as in `layers`); required in the fp16 precision.
    void run(const int32_t* ids_dev, int n, int pos0, const uint16_t* embed,
             const std::vector<LayerWeights>& layers, const KvView& kv, float* x_last,
             float* taps, cudaStream_t s, const std::vector<LayerWeights>* layers16 = nullptr);

    // Operand precision of the contractions and the attention. kPrecisionF16 (the default):
    // fp16 weights (exact copies of the bf16 values) and fp16 activations, the [wq;wk;wv] input
    // as an fp16 hi + lo pair (two MMAs), the attention on fp16 copies of the cache rows (the
    // same bf16 values); fp32 accumulation throughout. kPrecisionBF16: bf16 activations (one bf16
    // rounding per operand: 8 significant bits against fp16's 11).
    enum Precision : int { kPrecisionBF16 = 0, kPrecisionF16 = 1 };
    void set_precision(int p) { precision_ = p; }
    int precision() const { return precision_; }
    // The prompts of several new sequences in one pass per chunk of at most kMaxChunk tokens
    // (each sequence whole inside one chunk, so each prompt is at most kMaxChunk tokens): the
    // contractions run over the tokens of every sequence of the chunk together (M = their sum),
    // the QKV epilogue writes each token's K/V into its own sequence's pages, and the attention
    // takes a list of (sequence, 64-token query block) items. Sequence i has the tokens
    // ids_dev[offset[i] .. offset[i] + len[i]) at positions 0 .. len[i] - 1 and the page table
    // kv.page_table + table_off[i] (table_host: the same table on the host, for the cache rows).
    // x_last (device, [n_seqs, dim]) receives each sequence's last hidden state.
    void run_varlen(const int32_t* ids_dev, const std::vector<int>& offset,
                    const std::vector<int>& len, const std::vector<int>& table_off,
                    const int32_t* table_host, const uint16_t* embed,
                    const std::vector<LayerWeights>& layers, const KvView& kv, float* x_last,
                    cudaStream_t s, const std::vector<LayerWeights>* layers16 = nullptr);
    // Non-zero when a contraction's bounded wait gave up in the last run.
    unsigned read_error(cudaStream_t s);
    // Attention kernel: tcgen05 (default) or the mma.sync flash-attention kernel.

    // TMA maps of the paged caches (2-D rows and 4-D page boxes) for a view, over the cache
    // itself (bf16 precision) or over its fp16 copy (allocated here on first use); cached.
    void ensure_kv_maps(const KvView& kv, int n_layers);
    const CUtensorMap& kmap() const { return kmap_; }
    const CUtensorMap& vmap() const { return vmap_; }
    const CUtensorMap& kmap4() const { return kmap4_; }
    const CUtensorMap& vmap4() const { return vmap4_; }
    unsigned* err() const { return static_cast<unsigned*>(err_.ptr); }
    int num_sms() const { return num_sms_; }

private:
    // Rows of one pass: one sequence at positions p0.. (tok_pos null), or the tokens of several
    // (per-token positions and cache rows, the attention's work items).
    struct PassRows {
        int p0 = 0;
        const int32_t* tok_pos = nullptr;
        const int32_t* tok_row = nullptr;
        const int4* work = nullptr;
        int n_work = 0;
    };
    // Every layer over S rows (the chunk's token ids at `ids`); taps (nullable) as run's.
    void layer_pass(const int32_t* ids, int S, const PassRows& pr, const uint16_t* embed,
                    const std::vector<LayerWeights>& layers, const KvView& kv, float* taps,
                    cudaStream_t s);
    void prepare(const std::vector<LayerWeights>& layers, const KvView& kv,
                 const std::vector<LayerWeights>* layers16, int rows);
    void ensure_rows(int rows);
    void ensure_weight_maps(const std::vector<LayerWeights>& layers);
    size_t layer_elems(const KvView& kv) const;

    q3_config cfg_;
    int device_ = 0;
    int num_sms_ = 148;
    int cap_rows_ = 0;
    int precision_ = kPrecisionF16;
    DeviceBuffer x_, xn_, xn_lo_, q_, o_, h_, err_;
    // fp16 copies of the K/V rows of the cache this driver serves ([n_layers] x the view's
    // layout), the operands of the fp16 attention.
    DeviceBuffer k16_, v16_;
    bool kv_maps_f16_ = false;
    // Varlen pass: per-token positions and cache rows, attention work items (device), staging.
    DeviceBuffer tok_pos_, tok_row_, work_;
    PinnedBuffer pinned_varlen_;
    struct LayerMaps {
        CUtensorMap wqkv, wo, w1, w3, w2;
    };
    std::vector<LayerMaps> wmaps_;
    const uint16_t* wmaps_key_ = nullptr;
    CUtensorMap kmap_, vmap_, kmap4_, vmap4_;
    const uint16_t* kv_key_ = nullptr;
    int kv_pages_ = 0;
};

}  // namespace q3
