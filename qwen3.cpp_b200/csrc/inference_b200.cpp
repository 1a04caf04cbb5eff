// inference_b200.cpp - the reference's C++ classes (include/inference_b200.h) over the C ABI of
// libq3b200.so. Every status code becomes the exception type the reference throws; the free
// kernels stage host buffers through device memory and run the library's CUDA kernels.
#include "inference_b200.h"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <bit>
#include <chrono>
#include <cmath>
#include <string>
#include <utility>

namespace q3b200 {
namespace {

void check(q3_status s) {
    if (s == Q3_OK) return;
    const std::string msg = q3_last_error();
    if (s == Q3_ERR_OUT_OF_RANGE) throw std::out_of_range(msg);
    if (s == Q3_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

static_assert(sizeof(std::bfloat16_t) == sizeof(std::uint16_t));

const std::uint16_t* bits(const std::bfloat16_t* p) {
    return reinterpret_cast<const std::uint16_t*>(p);
}

// A device buffer of the current GPU, for the free kernels' host-pointer interface.
class DeviceBytes {
public:
    explicit DeviceBytes(size_t n) : n_(n) {
        if (n_) check_cuda(cudaMalloc(&p_, n_), "cudaMalloc");
    }
    ~DeviceBytes() {
        if (p_) cudaFree(p_);
    }
    DeviceBytes(const DeviceBytes&) = delete;
    DeviceBytes& operator=(const DeviceBytes&) = delete;
    DeviceBytes(DeviceBytes&& o) noexcept
        : p_(std::exchange(o.p_, nullptr)), n_(std::exchange(o.n_, 0)) {}
    DeviceBytes& operator=(DeviceBytes&&) = delete;
    template <typename T>
    T* as() const { return static_cast<T*>(p_); }
    void upload(const void* src, size_t n) {
        if (n) check_cuda(cudaMemcpy(p_, src, n, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
    }
    void download(void* dst, size_t n) const {
        if (n) check_cuda(cudaMemcpy(dst, p_, n, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
    }

private:
    void* p_ = nullptr;
    size_t n_ = 0;
};

template <typename T>
DeviceBytes upload(const T* src, size_t count) {
    DeviceBytes d(count * sizeof(T));
    d.upload(src, count * sizeof(T));
    return d;
}

void finish() { check_cuda(cudaDeviceSynchronize(), "kernel"); }

q3_config to_c(const Config& c) {
    q3_config o{};
    o.dim = c.dim;
    o.hidden_dim = c.hidden_dim;
    o.head_dim = c.head_dim;
    o.n_layers = c.n_layers;
    o.n_heads = c.n_heads;
    o.n_kv_heads = c.n_kv_heads;
    o.vocab_size = c.vocab_size;
    o.max_seq_len = c.max_seq_len;
    o.bos_token_id = c.bos_token_id;
    o.eos_token_id = c.eos_token_id;
    o.rotary_dim = c.rotary_dim;
    o.rope_theta = c.rope_theta;
    o.norm_eps = c.norm_eps;
    o.tie_word_embeddings = c.tie_word_embeddings;
    o.attention_bias = c.attention_bias;
    o.qk_norm = c.qk_norm;
    return o;
}

std::string model_string(const q3_model* m, const char* key) {
    size_t len = 0;
    check(q3_model_metadata(m, key, nullptr, 0, &len));
    std::string s(len + 1, '\0');
    check(q3_model_metadata(m, key, s.data(), s.size(), nullptr));
    s.resize(len);
    return s;
}

}  // namespace

// ------------------------------------------------------------------ Block

Block::Block(const std::shared_ptr<Config>& config, BlockWeights weights, int device)
    : config_(config) {
    if (!config_) throw std::invalid_argument("Block config must not be null");
    const q3_config c = to_c(*config_);
    const std::vector<std::bfloat16_t>* order[11] = {
        &weights.attn_norm, &weights.q_norm, &weights.k_norm, &weights.wq,
        &weights.wk,        &weights.wv,     &weights.wo,     &weights.mlp_norm,
        &weights.w1,        &weights.w2,     &weights.w3};
    const std::uint16_t* ptrs[11];
    size_t counts[11];
    for (int i = 0; i < 11; ++i) {
        ptrs[i] = bits(order[i]->data());
        counts[i] = order[i]->size();
    }
    check(q3_block_create(&c, ptrs, counts, device, &handle_));
}

Block::~Block() {
    if (handle_) q3_block_free(handle_);
}

Block::Block(Block&& other) noexcept
    : config_(std::move(other.config_)), handle_(std::exchange(other.handle_, nullptr)) {}

Block& Block::operator=(Block&& other) noexcept {
    if (this != &other) {
        if (handle_) q3_block_free(handle_);
        config_ = std::move(other.config_);
        handle_ = std::exchange(other.handle_, nullptr);
    }
    return *this;
}

void Block::forward(float* x, int pos, int num_sink, int kv_pos, int kv_len) {
    check(q3_block_forward(handle_, x, pos, num_sink, kv_pos, kv_len));
}

void Block::ResetCache() { check(q3_block_reset_cache(handle_)); }

KVCache Block::GetCache() const {
    KVCache c;
    c.seq_len = config_->max_seq_len;
    c.n_kv_heads = config_->n_kv_heads;
    c.head_dim = config_->head_dim;
    const size_t n = static_cast<size_t>(c.seq_len) * c.n_kv_heads * c.head_dim;
    c.k_.resize(n);
    c.v_.resize(n);
    check(q3_block_get_cache(handle_, reinterpret_cast<std::uint16_t*>(c.k_.data()),
                             reinterpret_cast<std::uint16_t*>(c.v_.data())));
    return c;
}

void Block::SetCache(const KVCache& cache) {
    const size_t n = static_cast<size_t>(config_->max_seq_len) * config_->n_kv_heads *
                     config_->head_dim;
    if (cache.k_.size() != n || cache.v_.size() != n) {
        throw std::invalid_argument("KV cache size does not match the block config");
    }
    check(q3_block_set_cache(handle_, bits(cache.k_.data()), bits(cache.v_.data())));
}

// ------------------------------------------------------------------ Sampler / stats

std::int32_t Sampler::Greedy(std::span<const float> logits) {
    if (logits.empty()) throw std::invalid_argument("Cannot sample empty logits");
    if (logits.size() > static_cast<size_t>(INT32_MAX)) {
        throw std::invalid_argument("logits span too large");
    }
    DeviceBytes d = upload(logits.data(), logits.size());
    DeviceBytes idx(sizeof(std::int32_t));
    check(q3_greedy(d.as<float>(), static_cast<int>(logits.size()), idx.as<std::int32_t>(),
                    nullptr));
    std::int32_t out = 0;
    idx.download(&out, sizeof(out));
    return out;
}

double GenerationStats::PrefillTokensPerSecond() const {
    return prefill_seconds > 0.0 ? prompt_tokens / prefill_seconds : 0.0;
}

double GenerationStats::DecodeTokensPerSecond() const {
    return decode_seconds > 0.0 ? generated_tokens / decode_seconds : 0.0;
}

// ------------------------------------------------------------------ Qwen3

Qwen3::Qwen3(const std::string& path, int context_length, int device) {
    check(q3_model_load(path.c_str(), context_length, device, &handle_));
    try {
        q3_config c{};
        check(q3_model_config(handle_, &c));
        config_ = std::make_shared<Config>();
        Config& o = *config_;
        o.arch = model_string(handle_, "arch");
        o.dtype = model_string(handle_, "dtype");
        o.act_type = model_string(handle_, "act_type");
        o.dim = c.dim;
        o.hidden_dim = c.hidden_dim;
        o.head_dim = c.head_dim;
        o.n_layers = c.n_layers;
        o.n_heads = c.n_heads;
        o.n_kv_heads = c.n_kv_heads;
        o.vocab_size = c.vocab_size;
        o.max_seq_len = c.max_seq_len;
        o.bos_token_id = c.bos_token_id;
        o.eos_token_id = c.eos_token_id;
        o.rotary_dim = c.rotary_dim;
        o.rope_theta = c.rope_theta;
        o.norm_eps = c.norm_eps;
        o.tie_word_embeddings = c.tie_word_embeddings != 0;
        o.attention_bias = c.attention_bias != 0;
        o.qk_norm = c.qk_norm != 0;
        int count = 0;
        check(q3_model_tensor_count(handle_, &count));
        for (int i = 0; i < count; ++i) {
            size_t len = 0;
            check(q3_model_tensor_name(handle_, i, nullptr, 0, &len));
            std::string name(len + 1, '\0');
            check(q3_model_tensor_name(handle_, i, name.data(), name.size(), nullptr));
            name.resize(len);
            q3_tensor_info ti{};
            check(q3_model_tensor_info(handle_, name.c_str(), &ti));
            TensorInfo info;
            info.name = name;
            info.dtype = static_cast<TensorDType>(ti.dtype);
            info.shape.assign(ti.shape, ti.shape + ti.rank);
            info.data_offset = ti.data_offset;
            info.byte_size = ti.byte_size;
            tensors_.emplace(name, std::move(info));
        }
        logits_.resize(static_cast<size_t>(o.vocab_size));
    } catch (...) {
        q3_model_free(handle_);
        handle_ = nullptr;
        throw;
    }
}

Qwen3::~Qwen3() {
    if (handle_) q3_model_free(handle_);
}

void Qwen3::ResetInference() { check(q3_reset(handle_)); }

const std::vector<float>& Qwen3::ForwardToken(std::int32_t token, int pos) {
    check(q3_forward_token(handle_, token, pos, logits_.data()));
    return logits_;
}

GenerationResult Qwen3::Generate(std::span<const std::int32_t> prompt_tokens,
                                 size_t max_generated_tokens, bool stop_on_eos,
                                 const std::function<void(std::span<const std::int32_t>)>&
                                     on_tokens) {
    std::vector<std::int32_t> prompt(prompt_tokens.begin(), prompt_tokens.end());
    if (prompt.empty()) prompt.push_back(config_->bos_token_id);
    if (prompt.size() > static_cast<size_t>(INT32_MAX)) {
        throw std::invalid_argument("prompt too long");
    }
    GenerationResult result;
    if (!on_tokens) {
        result.tokens.resize(max_generated_tokens);
        size_t n_out = 0;
        q3_generation_stats st{};
        check(q3_generate(handle_, prompt.data(), static_cast<int>(prompt.size()),
                          max_generated_tokens, stop_on_eos ? 1 : 0, result.tokens.data(), &n_out,
                          &st));
        result.tokens.resize(n_out);
        result.stats.prompt_tokens = st.prompt_tokens;
        result.stats.generated_tokens = st.generated_tokens;
        result.stats.prefill_seconds = st.prefill_seconds;
        result.stats.decode_seconds = st.decode_seconds;
        result.stats.stopped_on_eos = st.stopped_on_eos != 0;
        result.stats.reached_token_limit = st.reached_token_limit != 0;
        return result;
    }
    // The reference's loop (src/inference.cpp:669-699), one device step per generated token.
    using clock = std::chrono::steady_clock;
    result.stats.prompt_tokens = prompt.size();
    const auto t0 = clock::now();
    std::int32_t token = 0;
    check(q3_prefill(handle_, prompt.data(), static_cast<int>(prompt.size()), 0, nullptr,
                     &token));
    int pos = static_cast<int>(prompt.size());
    const auto t1 = clock::now();
    result.stats.prefill_seconds = std::chrono::duration<double>(t1 - t0).count();
    while (result.tokens.size() < max_generated_tokens) {
        if (stop_on_eos && token == config_->eos_token_id) {
            result.stats.stopped_on_eos = true;
            break;
        }
        result.tokens.push_back(token);
        on_tokens(result.tokens);
        std::int32_t next = 0;
        check(q3_decode_greedy(handle_, token, pos++, 1, &next, nullptr));
        token = next;
    }
    const auto t2 = clock::now();
    result.stats.generated_tokens = result.tokens.size();
    result.stats.reached_token_limit =
        !result.stats.stopped_on_eos && result.tokens.size() == max_generated_tokens;
    result.stats.decode_seconds = std::chrono::duration<double>(t2 - t1).count();
    return result;
}

std::vector<std::uint8_t> Qwen3::LoadTensorBytes(const std::string& name, TensorDType expected,
                                                 TensorInfo& info) const {
    const auto it = tensors_.find(name);
    if (it == tensors_.end()) throw std::runtime_error("Tensor not found: " + name);
    info = it->second;
    std::vector<std::uint8_t> bytes(info.byte_size);
    check(q3_model_load_tensor(handle_, name.c_str(), static_cast<std::uint32_t>(expected),
                               bytes.data(), bytes.size()));
    return bytes;
}

void Qwen3::KvRow(int layer, int kv_pos, std::vector<std::bfloat16_t>& k,
                  std::vector<std::bfloat16_t>& v) const {
    const size_t n = static_cast<size_t>(config_->n_kv_heads) * config_->head_dim;
    k.resize(n);
    v.resize(n);
    check(q3_kv_row(handle_, layer, kv_pos, reinterpret_cast<std::uint16_t*>(k.data()),
                    reinterpret_cast<std::uint16_t*>(v.data())));
}

// ------------------------------------------------------------------ free kernels

void RmsNorm(float* out, const float* x, const std::bfloat16_t* weights, float eps, int n) {
    if (n < 0) throw std::invalid_argument("negative size");
    DeviceBytes dx = upload(x, n);
    DeviceBytes dw = upload(weights, n);
    check(q3_rmsnorm(dx.as<float>(), dx.as<float>(), dw.as<std::uint16_t>(), eps, n, nullptr));
    finish();
    dx.download(out, sizeof(float) * n);
}

void Softmax(float* out, const float* x, int n) {
    if (n < 0) throw std::invalid_argument("negative size");
    DeviceBytes dx = upload(x, n);
    check(q3_softmax(dx.as<float>(), dx.as<float>(), n, nullptr));
    finish();
    dx.download(out, sizeof(float) * n);
}

float Silu(float x) { return x / (1.0f + std::exp(-x)); }

void MatMul(float* out, const float* x, const std::bfloat16_t* y, int n, int m) {
    if (n < 0 || m < 0) throw std::invalid_argument("negative size");
    DeviceBytes dx = upload(x, m);
    DeviceBytes dw = upload(y, static_cast<size_t>(n) * m);
    DeviceBytes dout(sizeof(float) * n);
    check(q3_matmul(dout.as<float>(), dx.as<float>(), dw.as<std::uint16_t>(), n, m, nullptr));
    finish();
    dout.download(out, sizeof(float) * n);
}

void ApplyRotaryEmb(float* out, int d, int head_dim, int pos, float theta, int rotary_dim) {
    if (d < 0) throw std::invalid_argument("negative size");
    DeviceBytes dx = upload(out, d);
    check(q3_rope(dx.as<float>(), d, head_dim, pos, theta, rotary_dim, nullptr));
    finish();
    dx.download(out, sizeof(float) * d);
}

void FeedForwardNetwork(float* out, float* lin1, float* lin2, const float* x,
                        const std::bfloat16_t* w1, const std::bfloat16_t* w2,
                        const std::bfloat16_t* w3, int hidden_dim, int dim) {
    if (hidden_dim < 0 || dim < 0) throw std::invalid_argument("negative size");
    const size_t wn = static_cast<size_t>(hidden_dim) * dim;
    DeviceBytes dx = upload(x, dim);
    DeviceBytes d1 = upload(w1, wn), d2 = upload(w2, wn), d3 = upload(w3, wn);
    DeviceBytes l1(sizeof(float) * hidden_dim), l2(sizeof(float) * hidden_dim);
    DeviceBytes dout(sizeof(float) * dim);
    check(q3_ffn(dout.as<float>(), l1.as<float>(), l2.as<float>(), dx.as<float>(),
                 d1.as<std::uint16_t>(), d2.as<std::uint16_t>(), d3.as<std::uint16_t>(),
                 hidden_dim, dim, nullptr));
    finish();
    dout.download(out, sizeof(float) * dim);
    l1.download(lin1, sizeof(float) * hidden_dim);
    l2.download(lin2, sizeof(float) * hidden_dim);
}

void FastAttn(float* out, float* /*atth*/, const float* q, const std::bfloat16_t* k,
              const std::bfloat16_t* v, int head_dim, int n_kv_heads, int kv_len) {
    if (head_dim <= 0 || n_kv_heads <= 0 || kv_len <= 0) {
        throw std::invalid_argument("attention sizes must be positive");
    }
    const size_t stride = static_cast<size_t>(n_kv_heads) * head_dim;
    const size_t span = (static_cast<size_t>(kv_len) - 1) * stride + head_dim;
    DeviceBytes dq = upload(q, head_dim);
    DeviceBytes dk = upload(k, span), dv = upload(v, span);
    DeviceBytes dout(sizeof(float) * head_dim);
    DeviceBytes ws(q3_attn_workspace_size(head_dim, kv_len));
    check(q3_attn(dout.as<float>(), ws.as<void>(), dq.as<float>(), dk.as<std::uint16_t>(),
                  dv.as<std::uint16_t>(), head_dim, n_kv_heads, kv_len, nullptr));
    finish();
    dout.download(out, sizeof(float) * head_dim);
}

void Attn(float* out, float* atth, const float* q, const std::bfloat16_t* k,
          const std::bfloat16_t* v, int head_dim, int n_kv_heads, int kv_len) {
    FastAttn(out, atth, q, k, v, head_dim, n_kv_heads, kv_len);
}

}  // namespace q3b200
