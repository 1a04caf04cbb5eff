// Tensor-parallel single-sequence decode over the GPUs of one node (one process per GPU).
//
// Rank r of N holds, for every layer, the query heads [r*16/N, (r+1)*16/N) and KV heads
// [r*8/N, (r+1)*8/N) (QKV projection rows, attention, o_proj columns), the MLP rows/columns
// [r*H/N, (r+1)*H/N) (gate/up rows, down columns), and a 128-row-aligned slice of the tied
// lm_head; the residual stream x is replicated. After o_proj and after down_proj every rank holds
// a partial sum of x's update: an all-reduce over NVLink peer memory (each rank pushes its 4 KB
// partial into every peer's buffer, then raises a flag there) adds them in rank order, so x stays
// bit-identical on every rank. The greedy argmax is all-reduced the same way over the vocabulary
// slices (lowest index on ties). Two ways to run the steps:
//   fused (default where the model has the fused decode kernel): one persistent kernel per GPU
//     runs up to 256 steps; the o_proj partials of each rank's KV-head groups go straight into
//     every rank's buffer as tagged words from the kernel's o_proj epilogue, and the ranks'
//     down-projection sums and greedy candidates travel the same way, polled in rank order by
//     the next phase (no separate all-reduce launch, no flag round trip).
//   graph: one captured CUDA graph per step: CUDA-core GEMVs on the local weight slices (fp32
//     activations, RmsNorm fused as their prologue), the paged decode attention of the local KV
//     heads, and the two all-reduce kernels.
//   graph + NCCL (a comparison arm): the same graph with ncclAllReduce (and an all-gather of the
//     greedy candidates) captured in place of this library's all-reduce kernels.
// The reference has no counterpart (it runs on one CPU).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <vector>

#include "q3_decode_fused.cuh"
#include "q3_model.cuh"

namespace q3 {

constexpr int kTpMaxRanks = 8;

class TpDecoder {
public:
    // model: this rank's full model (its prompt prefill fills the KV cache of every head; the
    // decoder then only touches the local heads). The model must outlive the decoder.
    TpDecoder(Model& model, int rank, int world);
    ~TpDecoder();
    TpDecoder(const TpDecoder&) = delete;
    TpDecoder& operator=(const TpDecoder&) = delete;

    // CUDA IPC handle (64 bytes) of this rank's exchange buffer.
    void ipc_handle(void* out) const;
    // Maps every peer's exchange buffer (handles of all ranks, rank order, 64 bytes each).
    void connect(const void* handles);

    // n_steps greedy steps from token `first` at position pos0 (positions below pos0 are in the
    // KV cache); tokens_host[n_steps] receives the generated tokens (identical on every rank).
    // forced_host (nullable): teacher forcing, token i fed at step i; argmax to tokens_host.
    void decode(int32_t first, int pos0, int n_steps, const int32_t* forced_host,
                int32_t* tokens_host);
    cudaStream_t stream() const { return s_; }
    // solo_allreduce: at world 1, send the o_proj / down_proj partials through the all-reduce
    // kernel (this rank as its only member) instead of adding them into x directly.
    // wait_cycles: budget (SM clock cycles) of each bounded flag wait.
    void configure(bool solo_allreduce, long long wait_cycles);
    // After a timeout (decode threw DeviceTimeout and refuses further steps): zero the
    // invocation counter, error word and exchange buffer. Every rank resets before any decodes.
    void reset();
    // Step path (Q3_TP_FUSED, Q3_TP_GRAPH, Q3_TP_GRAPH_NCCL); every rank of a group picks alike.
    void set_path(int path);
    int path() const;
    bool fused() const { return fused_; }
    // NCCL communicator of the graph + NCCL path: one rank makes the unique id (128 bytes), every
    // rank connects with it.
    static void nccl_unique_id(void* out);
    void nccl_connect(const void* id);
    bool fused_available() const { return f_grid_ > 0; }

private:
    void enqueue_step(bool forced);
    void setup_fused();
    void launch_fused(int n_steps, bool forced);
    void run_graph(bool forced, int n_steps);

    Model& m_;
    q3_config cfg_;
    int rank_, world_;
    int hq_, hkv_, hl_;     // local query heads, KV heads, MLP rows
    int v0_, vn_;           // local vocabulary rows [v0, v0 + vn)
    cudaStream_t s_ = nullptr;
    DeviceBuffer shard_;    // this rank's weight slices (ShardLayer per layer)
    struct ShardLayer {
        const uint16_t* wqkv;  // [(hq + 2 hkv) * 128][1024]: local rows of wq; wk; wv
        const uint16_t* w1;    // [hl][1024]
        const uint16_t* w3;    // [hl][1024]
        const uint16_t* wo;    // [1024][hq * 128]: wo[:, local attention columns]
        const uint16_t* w2;    // [1024][hl]: w2[:, local MLP columns]
    };
    std::vector<ShardLayer> layers_;
    DeviceBuffer x_, qkv_, q32_, o32_, part_, h32_, logits_, scratch_;
    DeviceBuffer pos_, tok_, step_, forced_, log_, err_, counter_, part_o_, part_ml_, attn_counter_;
    DeviceBuffer xbuf_;     // exchange buffer (IPC-exported): data, argmax slots, flags
    std::vector<void*> peer_mapped_;
    std::vector<uint8_t> self_peer_;  // peers given this rank's own handle
    bool connected_ = false;
    bool failed_ = false;
    bool solo_allreduce_ = false;
    long long wait_cycles_ = 4000000000LL;  // ~2 s at the B200 boost clock
    int log_cap_ = 0;
    int attn_pps_ = 8, attn_splits_ = 1;  // decode attention: pages per split, splits
    int sms_ = 0;
    cudaGraphExec_t graph_ = nullptr;
    bool graph_forced_ = false;
    const float2* graph_rope_ = nullptr;
    // Fused path: local [wq;wk;wv] rows of the fused kernel's weight copies, per-layer pointers,
    // and the kernel's own state (down-projection accumulators, tagged q|k|v, attention split
    // partials, per-CTA argmax, arrival counter, step parameters).
    bool fused_ = false;
    bool use_nccl_ = false;
    void* nccl_comm_ = nullptr;  // ncclComm_t
    DeviceBuffer am_nccl_;       // [1 + world] (value, index): this rank's, then the gathered
    int f_grid_ = 0, f_smax_ = 0, f_parity_ = 0;
    unsigned f_epoch_ = 0;
    DeviceBuffer f_wqkv_, f_layers_, f_y_, f_qkvt_, f_part_o_, f_part_ml_, f_am_, f_sync_, f_sp_;
};

}  // namespace q3
