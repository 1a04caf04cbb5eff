// Batched decode of independent sequences on one GPU (the data-parallel serving configuration):
// the reference's ForwardToken + Greedy (src/inference.cpp:592-637, :703-709) for every sequence
// of a batch at once. Each decode step streams the weights once for all sequences (tensor-core
// contractions with M = number of sequences) and reads every sequence's own KV pages.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <vector>

#include "q3_model.cuh"
#include "q3_prefill.cuh"

namespace q3 {

class Batch {
public:
    // Room for max_seqs sequences of at most max_tokens positions each (prompt + generated),
    // in a paged KV pool of 16-token pages; each sequence owns a contiguous range of pages.
    Batch(Model& model, int max_seqs, int max_tokens);
    ~Batch();
    Batch(const Batch&) = delete;
    Batch& operator=(const Batch&) = delete;

    // Adds a sequence and prefills its prompt (batched on the tensor cores) into its pages.
    // Returns the slot; *next_token (nullable) receives the greedy token after the prompt,
    // last_logits (nullable, host) its logits.
    int add(const int32_t* ids_host, int n, int32_t* next_token, float* last_logits);
    // Adds n_seqs sequences at once: prompt i is lens[i] tokens of ids_host (the prompts back to
    // back). Prompts of up to 4096 tokens are prefilled together (one tensor-core pass over all
    // their tokens per 4096-token chunk, Prefill::run_varlen), longer ones one by one. Returns the
    // slot of the first; next_tokens[n_seqs] (nullable) and last_logits[n_seqs][vocab] (nullable,
    // host) as add's.
    int add_many(const int32_t* ids_host, const int* lens, int n_seqs, int32_t* next_tokens,
                 float* last_logits);
    int size() const { return static_cast<int>(len_.size()); }
    cudaStream_t stream() const { return s_; }
    int length(int slot) const { return len_.at(slot); }

    // n_steps greedy steps for every sequence: each feeds its current token at its next
    // position; tokens_host[n_steps][size()] (nullable) receives the generated tokens.
    void decode(int n_steps, int32_t* tokens_host);
    // Teacher-forced steps: feeds tokens_host[step][size()], writes the greedy argmax of each to
    // argmax_host[step][size()] and (nullable) all logits to logits_host[step][size()][vocab].
    void decode_forced(const int32_t* tokens_host, int n_steps, int32_t* argmax_host,
                       float* logits_host);
    // Row `pos` of sequence `slot`'s layer-`layer` K and V (reference KVCache layout).
    void kv_row(int slot, int layer, int pos, uint16_t* k_host, uint16_t* v_host);

private:
    void ensure_step_buffers();
    void enqueue_step(bool forced, int n_forced);
    void enqueue_small_layers();
    // Decode steps of at most 16 sequences (of 1024-multiple widths) run their weight products as
    // CUDA-core GEMVs over fp32 rows instead of tensor-core contractions.
    bool small_path() const;
    void run(int n_steps, const int32_t* forced_host, int32_t* log_host, float* logits_host);

    Model& m_;
    q3_config cfg_;
    int max_seqs_, max_tokens_, pps_;  // pages per sequence
    int pool_pages_;                   // pages per layer in the pool
    cudaStream_t s_ = nullptr;
    std::unique_ptr<Prefill> prefill_;
    DeviceBuffer k_, v_, table_, rope_, pos_, tok_, step_, forced_, log_, err_;
    DeviceBuffer x_, xn_, qkv_, o_, gu_, h_, logits_, x_last_, ids_, xn_lo_, o_lo_, h_lo_;
    DeviceBuffer q32_, attn_part_o_, attn_part_ml_, attn_counter_, o32_, h32_, am_part_, am_counter_;
    int attn_pps_ = 8, attn_splits_ = 1;
    int rope_len_ = 0;
    int cap_rows_ = 0;  // rows the step buffers and maps were built for
    int log_cap_ = 0;
    std::vector<int32_t> table_host_;  // the page table (slot s owns pages [s*pps, (s+1)*pps))
    std::vector<int> len_;             // positions filled per sequence
    std::vector<int32_t> next_;        // token each sequence feeds next
    PinnedBuffer pinned_;
    // TMA maps for the decode step (rebuilt when the number of sequences changes).
    CUtensorMap a_xn_, a_o_, a_h_, a_xn_lo_, a_o_lo_, a_h_lo_, o_qkv_, o_x_, o_gu_,
        o_logits_;
    struct LayerMaps {
        CUtensorMap wqkv, wo, w13, w2;
    };
    std::vector<LayerMaps> wmaps_;
    CUtensorMap lm_;
    cudaGraphExec_t graph_ = nullptr;
    int graph_rows_ = -1;
    bool graph_forced_ = false;
};

}  // namespace q3
