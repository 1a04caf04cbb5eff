// inference_b200.h - the C++ surface of asriva32/Qwen3.cpp's include/inference.h, backed by the
// B200 library (include/q3_b200.h). Same class and function names, argument meanings and
// exception types (std::runtime_error / std::invalid_argument / std::out_of_range), in namespace
// q3b200, so a reference user switches by changing the include and the namespace:
//
//   #include "inference.h"        ->  #include "inference_b200.h"
//   Qwen3 model(path, ctx);       ->  q3b200::Qwen3 model(path, ctx);
//
// Differences: the tokenizer stays with the caller (Generate takes token IDs; the reference
// encodes text with tokenizers-cpp, src/inference.cpp:647-658, and GenerationResult has no
// text); State is accepted and ignored (the device workspace belongs to the model or block);
// Block::GetCache returns a snapshot read back from the device; the free kernels take host
// pointers like the reference's and run on the current GPU. Requires C++23 (std::bfloat16_t),
// like the reference. Link with -lq3b200_cxx -lq3b200.
#ifndef INFERENCE_B200_H
#define INFERENCE_B200_H

#include <concepts>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <span>
#include <stdexcept>
#include <stdfloat>
#include <string>
#include <unordered_map>
#include <vector>

#include "q3_b200.h"

namespace q3b200 {

// TensorDType and TensorInfo (include/inference.h:23-36): the record codes of convert.py.
enum class TensorDType : std::uint32_t { Float32 = 1, BFloat16 = 3, UInt8 = 4, Int32 = 5 };

struct TensorInfo {
    std::string name;
    TensorDType dtype = TensorDType::BFloat16;
    std::vector<size_t> shape;
    size_t data_offset = 0;
    size_t byte_size = 0;
};

template <typename T>
concept SupportedTensorElement = std::same_as<T, float> || std::same_as<T, std::int32_t> ||
                                 std::same_as<T, std::uint8_t> || std::same_as<T, std::bfloat16_t>;

// Tensor<T> (include/inference.h:52-63): a host copy of one record.
template <SupportedTensorElement T>
struct Tensor {
    TensorInfo info;
    std::vector<T> data;
    const T* ptr() const { return data.data(); }
    T* ptr() { return data.data(); }
};

// Config (include/inference.h:66-90).
class Config {
public:
    std::string arch, dtype, act_type;
    std::int32_t dim = 0, hidden_dim = 0, head_dim = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0;
    std::int32_t vocab_size = 0, max_seq_len = 0, bos_token_id = 0, eos_token_id = 0,
                 rotary_dim = 0;
    float rope_theta = 0.0f, norm_eps = 0.0f;
    bool tie_word_embeddings = false, attention_bias = false, qk_norm = false;
};

// State (include/inference.h:92-138): the reference's per-call scratch. The GPU path keeps its
// scratch on the device, so this carries nothing; it exists so calls keep their shape.
struct State {
    State() = default;
    explicit State(const std::shared_ptr<Config>&) {}
};

// KVCache (include/inference.h:140-161), in the reference layout.
struct KVCache {
    std::vector<std::bfloat16_t> k_;  // (seq_len, n_kv_heads * head_dim)
    std::vector<std::bfloat16_t> v_;
    int seq_len = 0, n_kv_heads = 0, head_dim = 0;
};

// BlockWeights (include/inference.h:163-176).
struct BlockWeights {
    using bf16 = std::bfloat16_t;
    std::vector<bf16> attn_norm, q_norm, k_norm, wq, wk, wv, wo, mlp_norm, w1, w2, w3;
};

// Block (include/inference.h:178-202) on one GPU.
class Block {
public:
    Block(const std::shared_ptr<Config>& config, BlockWeights weights, int device = 0);
    ~Block();
    Block(const Block&) = delete;
    Block& operator=(const Block&) = delete;
    Block(Block&& other) noexcept;
    Block& operator=(Block&& other) noexcept;

    // Block::forward (src/inference.cpp:766-866), in place on the host vector x.
    void forward(float* x, int pos, int num_sink, int kv_pos, int kv_len);
    void forward(float* x, int pos, int num_sink, int kv_pos, int kv_len, State&) {
        forward(x, pos, num_sink, kv_pos, kv_len);
    }
    // Block::ResetCache (src/inference.cpp:732-735).
    void ResetCache();
    // Block::GetCache: a snapshot of the device cache, max_seq_len rows.
    KVCache GetCache() const;
    // Writes the device cache from the reference layout.
    void SetCache(const KVCache& cache);
    Config* GetConfig() { return config_.get(); }

private:
    std::shared_ptr<Config> config_;
    q3_block* handle_ = nullptr;
};

class Sampler {
public:
    // Sampler::Greedy (src/inference.cpp:703-709): first index of the maximum, computed on the
    // GPU; an empty span throws std::invalid_argument.
    static std::int32_t Greedy(std::span<const float> logits);
};

// GenerationStats / GenerationResult (include/inference.h:209-225).
struct GenerationStats {
    size_t prompt_tokens = 0;
    size_t generated_tokens = 0;
    double prefill_seconds = 0.0;
    double decode_seconds = 0.0;
    bool stopped_on_eos = false;
    bool reached_token_limit = false;
    double PrefillTokensPerSecond() const;
    double DecodeTokensPerSecond() const;
};

struct GenerationResult {
    std::vector<std::int32_t> tokens;
    GenerationStats stats;
};

// Qwen3 (include/inference.h:227-264) on one GPU.
class Qwen3 {
public:
    Qwen3(const std::string& path, int context_length = 512, int device = 0);
    ~Qwen3();
    Qwen3(const Qwen3&) = delete;
    Qwen3& operator=(const Qwen3&) = delete;

    void ResetInference();
    // ForwardToken (src/inference.cpp:592-637); the returned logits stay valid until the next
    // call on this model.
    const std::vector<float>& ForwardToken(std::int32_t token, int pos);
    const std::vector<float>& ForwardToken(std::int32_t token, int pos, State&) {
        return ForwardToken(token, pos);
    }
    // Generate (src/inference.cpp:639-700) on token IDs: an empty prompt becomes [bos]; greedy
    // tokens until max_generated_tokens or, with stop_on_eos, the EOS id. Without on_tokens the
    // decode loop runs on the device; with it, one step per token so that on_tokens sees the
    // tokens generated so far after each one, as in the reference.
    GenerationResult Generate(std::span<const std::int32_t> prompt_tokens,
                              size_t max_generated_tokens = 512, bool stop_on_eos = true,
                              const std::function<void(std::span<const std::int32_t>)>&
                                  on_tokens = {});

    template <SupportedTensorElement T>
    Tensor<T> LoadTensor(const std::string& name) const;

    const Config* GetConfig() const { return config_.get(); }
    const std::unordered_map<std::string, TensorInfo>& GetTensorIndex() const { return tensors_; }
    // Row kv_pos of layer `layer`'s KV cache (a debug tap with no reference counterpart).
    void KvRow(int layer, int kv_pos, std::vector<std::bfloat16_t>& k,
               std::vector<std::bfloat16_t>& v) const;
    q3_model* handle() const { return handle_; }

private:
    std::vector<std::uint8_t> LoadTensorBytes(const std::string& name, TensorDType expected,
                                              TensorInfo& info) const;

    q3_model* handle_ = nullptr;
    std::shared_ptr<Config> config_;
    std::unordered_map<std::string, TensorInfo> tensors_;
    std::vector<float> logits_;
};

template <typename T>
constexpr TensorDType ExpectedDType() {
    if constexpr (std::same_as<T, std::bfloat16_t>) return TensorDType::BFloat16;
    else if constexpr (std::same_as<T, float>) return TensorDType::Float32;
    else if constexpr (std::same_as<T, std::int32_t>) return TensorDType::Int32;
    else return TensorDType::UInt8;
}

template <SupportedTensorElement T>
Tensor<T> Qwen3::LoadTensor(const std::string& name) const {
    Tensor<T> t;
    const std::vector<std::uint8_t> bytes = LoadTensorBytes(name, ExpectedDType<T>(), t.info);
    t.data.resize(bytes.size() / sizeof(T));
    if (!bytes.empty()) std::memcpy(t.data.data(), bytes.data(), t.data.size() * sizeof(T));
    return t;
}

// Free kernels of include/inference.h:308-315 on host pointers, run on the current GPU.
void RmsNorm(float* out, const float* x, const std::bfloat16_t* weights, float eps, int n);
void Softmax(float* out, const float* x, int n);
// Silu (src/inference.cpp:948-950) is a scalar host function, as in the reference.
float Silu(float x);
void MatMul(float* out, const float* x, const std::bfloat16_t* y, int n, int m);
void ApplyRotaryEmb(float* out, int d, int head_dim, int pos, float theta, int rotary_dim);
void FeedForwardNetwork(float* out, float* lin1, float* lin2, const float* x,
                        const std::bfloat16_t* w1, const std::bfloat16_t* w2,
                        const std::bfloat16_t* w3, int hidden_dim, int dim);
// FastAttn for one query head; k/v point at the head's first element of a
// [kv_len, n_kv_heads*head_dim] cache. atth is accepted and left unwritten: the GPU kernel keeps
// its split-K partials in device scratch.
void FastAttn(float* out, float* atth, const float* q, const std::bfloat16_t* k,
              const std::bfloat16_t* v, int head_dim, int n_kv_heads, int kv_len);
// Attn (src/inference.cpp:1060-1090), the scalar form of the same attention: same GPU kernel.
void Attn(float* out, float* atth, const float* q, const std::bfloat16_t* k,
          const std::bfloat16_t* v, int head_dim, int n_kv_heads, int kv_len);

}  // namespace q3b200

#endif  // INFERENCE_B200_H
