// Host-side classes of the B200 Qwen3 library (behind the C ABI of include/q3_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <array>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "q3_b200.h"
#include "q3_common.cuh"

namespace q3 {

void validate_config(const q3_config& c);
void validate_kernel_limits(const q3_config& c);

// Per-layer weights as the fused kernel streams them: copies made at load time so that every
// CTA's share of a phase is one contiguous byte range, with the row-parity swizzle on the matrices
// multiplied by MMAs (wqkv, wop, w1, w3 and the lm_head copy):
//   wop[g][r][j] = wo[r][256*g + j]   (o_proj split by KV-head group: [8][1024][256])
//   w2t[i][r]    = w2[r][i]           (down_proj split by MLP index: [3072][1024])
struct FusedLayer {
    const uint16_t* wqkv;       // [4096][1024]: wq; wk; wv rows (swizzled)
    const uint16_t* wop;        // [8][1024][256] (swizzled)
    const uint16_t* w1;         // [3072][1024] (swizzled)
    const uint16_t* w3;         // [3072][1024] (swizzled)
    const uint16_t* w2t;        // [3072][1024]
    const uint16_t* attn_norm;  // [1024]
    const uint16_t* q_norm;     // [128]
    const uint16_t* k_norm;     // [128]
    const uint16_t* mlp_norm;   // [1024]
};

// A parsed, memory-mapped Qwen3.bin (the layout of the reference's convert.py:2-20).
class ModelFile {
public:
    struct Tensor {
        std::string name;
        uint32_t dtype = 0;
        std::vector<uint64_t> shape;
        size_t offset = 0;
        size_t byte_size = 0;
    };
    explicit ModelFile(const std::string& path);
    ~ModelFile();
    ModelFile(const ModelFile&) = delete;
    ModelFile& operator=(const ModelFile&) = delete;

    const q3_config& config() const { return config_; }
    const Tensor& tensor(const std::string& name) const;
    size_t tensor_count() const { return tensors_.size(); }
    const uint8_t* data() const { return data_; }
    // Metadata strings of the header ("arch", "dtype", "act_type").
    const std::string& metadata(const std::string& key) const;
    // Name of record i in file order.
    const std::string& tensor_name(size_t i) const { return names_.at(i); }

private:
    std::string path_;
    int fd_ = -1;
    const uint8_t* data_ = nullptr;
    size_t size_ = 0;
    q3_config config_{};
    std::string arch_, dtype_, act_;
    std::unordered_map<std::string, Tensor> tensors_;
    std::vector<std::string> names_;  // record order
};

struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer();
    void alloc(size_t n);
    void reset();
};

struct PinnedBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    PinnedBuffer() = default;
    PinnedBuffer(const PinnedBuffer&) = delete;
    PinnedBuffer& operator=(const PinnedBuffer&) = delete;
    ~PinnedBuffer();
    void ensure(size_t n);
};

// Device pointers of one decoder layer inside a weight arena.
struct LayerWeights {
    const uint16_t* attn_norm = nullptr;
    const uint16_t* q_norm = nullptr;
    const uint16_t* k_norm = nullptr;
    const uint16_t* wqkv = nullptr;  // [wq; wk; wv] rows, [q_dim + 2*kv_dim, dim]
    const uint16_t* wo = nullptr;
    const uint16_t* mlp_norm = nullptr;
    const uint16_t* w1 = nullptr;
    const uint16_t* w3 = nullptr;
    const uint16_t* w2 = nullptr;
};

std::vector<float2> rope_table_host(float theta, int rotary_dim, int len);

// Activations, KV cache (paged, 16-token pages) and per-step graphs for n_layers layers of one
// sequence. The kernels of one decoder layer are enqueued by enqueue_layer.
class Engine {
public:
    Engine(const q3_config& cfg, int n_layers, int device, int kv_slots);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    cudaStream_t stream() const { return stream_; }
    StepParams* step_params() const { return static_cast<StepParams*>(sp_.ptr); }
    float* x() const { return static_cast<float*>(x_.ptr); }
    float* qkv() const { return static_cast<float*>(qkv_.ptr); }
    float* h() const { return static_cast<float*>(h_.ptr); }
    size_t layer_elems() const { return static_cast<size_t>(n_pages_) * page_elems_; }
    float* taps() const { return static_cast<float*>(taps_.ptr); }
    uint16_t* k_layer(int l) const;
    uint16_t* v_layer(int l) const;
    const int32_t* page_table() const { return static_cast<const int32_t*>(page_table_.ptr); }
    const float2* rope() const { return static_cast<const float2*>(rope_.ptr); }
    int rope_len() const { return rope_len_; }
    int n_pages() const { return n_pages_; }
    int n_splits() const { return n_splits_; }

    void ensure_rope(int needed_len);
    void reset_cache();
    void enqueue_layer(int l, const LayerWeights& w);
    void write_step(const StepParams& p);
    StepParams read_step();
    void read_kv_row(int l, int slot, uint16_t* k, uint16_t* v);
    void read_cache(int l, uint16_t* k, uint16_t* v, int rows);
    void write_cache(int l, const uint16_t* k, const uint16_t* v, int rows);
    cudaGraphExec_t graph(int key, const std::function<void()>& enqueue);
    void drop_graphs();

private:
    q3_config cfg_;
    int n_layers_;
    int device_;
    int kv_slots_;
    int q_dim_ = 0, kv_dim_ = 0, n_pages_ = 0, n_splits_ = 1;
    size_t page_elems_ = 0;
    cudaStream_t stream_ = nullptr;
    DeviceBuffer k_cache_, v_cache_, page_table_, sp_, x_, qkv_, att_, h_, part_o_, part_ml_,
        taps_, rope_;
    int rope_len_ = 0;
    PinnedBuffer pinned_sp_;
    std::map<int, cudaGraphExec_t> graphs_;
};

class Prefill;

// class Qwen3 of the reference (include/inference.h:227-264) on one GPU.
class Model {
public:
    Model(const std::string& path, int ctx, int device);
    ~Model();

    const q3_config& config() const { return cfg_; }
    int device() const { return device_; }
    int tensor_count() const { return tensor_count_; }
    const ModelFile& file() const { return file_; }
    cudaStream_t stream() const { return engine_->stream(); }
    Engine& engine() { return *engine_; }
    const LayerWeights& layer(int l) const { return layers_[l]; }
    const uint16_t* embed() const { return embed_; }
    const uint16_t* output() const { return output_; }
    const uint16_t* final_norm() const { return final_norm_; }
    float* logits() const { return static_cast<float*>(logits_.ptr); }

    void reset();
    // err_after_logits: logits_host has room for one more word, which receives the fused
    // kernel's error word in the same copy.
    // next_host (nullable): the step's greedy token (Sampler::Greedy of the logits).
    void forward_token(int32_t token, int pos, float* hidden_host, float* logits_host,
                       bool err_after_logits = false, int32_t* next_host = nullptr);
    // ForwardToken returning the logits in a model-owned pinned host buffer, valid until the
    // next call (the reference returns a reference to its logits vector); next (nullable)
    // receives their greedy token, computed on the device.
    const float* forward_token_ref(int32_t token, int pos, int32_t* next = nullptr);
    void decode_loop(const int32_t* forced_host, int n, int32_t first_token, int pos0,
                     int32_t* out_tokens_host, float* last_logits_host, float* all_logits_host);
    // Prompt prefill. Batched (tensor-core contractions over all tokens) when the shape allows
    // it, the batched path is selected and the prompt fits below the context; token by token
    // otherwise. hidden_host (nullable) receives the last token's hidden state before the
    // first layer and after every layer ([(n_layers+1) * dim]).
    void prefill(const int32_t* ids, int n, int pos0, float* last_logits, int32_t* next,
                 float* hidden_host = nullptr);
    bool batched_prefill_enabled() const { return use_batched_prefill_; }
    void set_batched_prefill(bool on) { use_batched_prefill_ = on; }
    // Operand precision of the batched prefill (Prefill::Precision; fp16 by default).
    int prefill_precision() const { return prefill_precision_; }
    void set_prefill_precision(int p);
    // The layers with fp16 copies of their five matrices (made on first use), the operands of
    // the fp16 batched prefill of this model and of its batches.
    const std::vector<LayerWeights>& layers_f16();
    bool batched_prefill_ok(int n, int pos0) const;
    void generate(const int32_t* prompt, int n_prompt, size_t max_new, bool stop_on_eos,
                  int32_t* out, size_t* n_out, q3_generation_stats* stats);
    void kv_row(int layer, int kv_pos, uint16_t* k, uint16_t* v);

    // Decode path: the fused whole-step kernel when the config is the Qwen3-0.6B shape and the
    // device can hold one CTA per SM, else the layer-wise kernels (both on the GPU).
    bool fused_available() const { return fused_grid_ > 0; }
    bool fused_enabled() const { return use_fused_ && fused_grid_ > 0; }
    void set_fused(bool on) { use_fused_ = on; }
    int fused_grid() const { return fused_grid_; }
    // The fused kernel's weight copies (host copy of its per-layer pointers) and lm_head copy.
    const std::vector<FusedLayer>& fused_layers_host() const { return fused_host_layers_; }
    const uint16_t* fused_lm() const { return fused_lm_; }
    // Runs one fused launch whose grid-wide waits can never complete, with a short bound, and
    // reports whether the kernel returned with its timeout status set (failure-path test).
    bool fused_timeout_selftest();
    // One fused decode step with per-(phase, CTA) globaltimer stamps [phases][grid][4].
    void fused_profile(int32_t token, int pos, uint64_t* stamps, size_t cap, int* n_phases,
                       int* grid);

private:
    void check_token_pos(int32_t token, int pos) const;
    StepParams start_params(int32_t token, int pos, int n_forced) const;
    void ensure_logs(int n);
    void enqueue_step(bool forced, bool taps);
    // sp_init (fused path, n == 1): the step's parameters go to the kernel as an argument and
    // the device copy is not written first.
    void run_steps(int n, bool forced, bool taps, float* logits_log_dev,
                   const StepParams* sp_init = nullptr);
    void prefill_batched(const int32_t* ids, int n, int pos0, float* last_logits, int32_t* next,
                         float* hidden_host);
    void launch_fused(int n_steps, bool forced, bool taps, long long spin_cycles, int offset,
                      unsigned long long* prof = nullptr, const StepParams* sp_init = nullptr);
    void clear_fused_error();
    void check_fused_error();
    // Zeroes the arrival counter, the error word and both accumulator parities (after a launch
    // that gave up, whose state is then undefined).
    void reset_fused_state();
    unsigned* fused_err_word() const;  // the word after the logits in logits_

    ModelFile file_;
    q3_config cfg_{};
    int device_ = 0;
    int tensor_count_ = 0;
    DeviceBuffer arena_;
    const uint16_t* embed_ = nullptr;
    const uint16_t* output_ = nullptr;
    const uint16_t* final_norm_ = nullptr;
    std::vector<LayerWeights> layers_;
    std::unique_ptr<Engine> engine_;
    DeviceBuffer logits_, argmax_part_, argmax_out_, token_log_, forced_;
    int log_cap_ = 0;
    PinnedBuffer pinned_io_;
    PinnedBuffer pinned_logits_, pinned_err_;
    // Fused decode state.
    int fused_grid_ = 0;
    int fused_s_max_ = 0;
    const uint16_t* fused_lm_ = nullptr;
    bool use_fused_ = true;
    bool use_batched_prefill_ = true;
    std::unique_ptr<Prefill> prefill_;
    DeviceBuffer prefill_ids_;
    int prefill_precision_ = 1;  // Prefill::kPrecisionF16
    DeviceBuffer f16_arena_;
    std::vector<LayerWeights> layers16_;
    DeviceBuffer fused_layers_, fused_part_o_, fused_part_ml_, fused_am_, fused_sync_, fused_wperm_,
        fused_y_, fused_tagged_, fused_dbg_;
    std::vector<FusedLayer> fused_host_layers_;
    // One-step ForwardToken + Greedy on the fused path: the launch writes its logits and token
    // straight into pinned host memory (device addresses of it), no copy afterwards.
    float* fused_logits_out_ = nullptr;
    int32_t* fused_token_out_ = nullptr;
    unsigned* fused_err_out_ = nullptr;
    unsigned fused_epoch_ = 0;  // tag base of the last fused launch (1..4095)
    int fused_parity_ = 0;      // accumulator parity of the next launch's first step
};

// class Block of the reference (include/inference.h:178-202) on one GPU.
class Block {
public:
    Block(const q3_config& cfg, const uint16_t* const* w, const size_t* counts, int device);
    ~Block();
    void forward(float* x_host, int pos, int num_sink, int kv_pos, int kv_len);
    Engine& engine() { return *engine_; }
    const q3_config& config() const { return cfg_; }

private:
    q3_config cfg_{};
    DeviceBuffer arena_;
    LayerWeights lw_;
    std::unique_ptr<Engine> engine_;
};

}  // namespace q3
