// Test infrastructure only (the oracle): a C-ABI driver around the UNMODIFIED reference
// engine (src/inference.cpp + include/inference.h of asriva32/Qwen3.cpp), compiled from the
// reference sources by oracle/Makefile into oracle/_ref/libq3ref.so. Tests, the smoke check
// and the CPU-baseline leg of bench.py load it through ctypes; nothing in the product links it.
//
// The reference CLI cannot run on a weights-only random-init file (src/main.cpp:111-112
// needs tokenizer tables) and Qwen3::Generate needs a tokenizer (src/inference.cpp:655), so
// this driver is ID-driven:
//   * q3ref_forward_token   -> Qwen3::ForwardToken (src/inference.cpp:592-637), stock path.
//   * q3ref_forward_layers  -> the same steps as ForwardToken (:601-635) built from the
//     reference's public pieces (Qwen3::LoadTensor, Block, RmsNorm, MatMul) so that the
//     hidden state after every layer and the per-layer KV caches can be read back.
//   * q3ref_generate_ids    -> the prefill and greedy loops of Qwen3::Generate (:663-697)
//     with `--benchmark N` semantics (EOS ignored), timed with the same steady_clock marks.
//   * q3ref_block_*         -> Block(config, weights) / Block::forward / ResetCache / GetCache.
//   * q3ref_<op>            -> the free functions of include/inference.h:308-315 and
//     Sampler::Greedy (include/inference.h:204-207).
#include "inference.h"

#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

thread_local std::string g_last_error;

enum : int { kOk = 0, kRuntime = 1, kInvalidArgument = 2, kOutOfRange = 3, kOther = 4 };

template <typename F>
int Guard(F&& fn) {
    try {
        fn();
        return kOk;
    } catch (const std::out_of_range& e) {
        g_last_error = e.what();
        return kOutOfRange;
    } catch (const std::invalid_argument& e) {
        g_last_error = e.what();
        return kInvalidArgument;
    } catch (const std::runtime_error& e) {
        g_last_error = e.what();
        return kRuntime;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return kOther;
    }
}

std::vector<std::bfloat16_t> ToBf16Vector(const std::uint16_t* p, std::size_t n) {
    std::vector<std::bfloat16_t> v(n);
    if (n) std::memcpy(v.data(), p, n * sizeof(std::uint16_t));
    return v;
}

struct RefModel {
    std::unique_ptr<Qwen3> model;
    std::shared_ptr<Config> cfg;
    std::unique_ptr<State> state;
    // Per-layer path (built on first use).
    std::vector<Block> blocks;
    std::vector<std::bfloat16_t> embed;
    std::vector<std::bfloat16_t> final_norm;
    std::vector<float> hidden;
    std::vector<float> normed;
    std::vector<float> logits;

    void EnsureBlocks() {
        if (!blocks.empty()) return;
        using bf16 = std::bfloat16_t;
        embed = model->LoadTensor<bf16>("model.embed.weight").data;
        final_norm = model->LoadTensor<bf16>("model.norm.weight").data;
        blocks.reserve(cfg->n_layers);
        for (int layer = 0; layer < cfg->n_layers; ++layer) {
            const std::string p = "model.layers." + std::to_string(layer);
            BlockWeights w;
            w.attn_norm = model->LoadTensor<bf16>(p + ".attn.norm.weight").data;
            w.q_norm = model->LoadTensor<bf16>(p + ".attn.q_norm.weight").data;
            w.k_norm = model->LoadTensor<bf16>(p + ".attn.k_norm.weight").data;
            w.wq = model->LoadTensor<bf16>(p + ".attn.wq.weight").data;
            w.wk = model->LoadTensor<bf16>(p + ".attn.wk.weight").data;
            w.wv = model->LoadTensor<bf16>(p + ".attn.wv.weight").data;
            w.wo = model->LoadTensor<bf16>(p + ".attn.wo.weight").data;
            w.mlp_norm = model->LoadTensor<bf16>(p + ".mlp.norm.weight").data;
            w.w1 = model->LoadTensor<bf16>(p + ".mlp.w1.weight").data;
            w.w2 = model->LoadTensor<bf16>(p + ".mlp.w2.weight").data;
            w.w3 = model->LoadTensor<bf16>(p + ".mlp.w3.weight").data;
            blocks.emplace_back(cfg, std::move(w));
        }
        hidden.assign(cfg->dim, 0.0f);
        normed.assign(cfg->dim, 0.0f);
        logits.assign(cfg->vocab_size, 0.0f);
    }
};

struct RefBlock {
    std::shared_ptr<Config> cfg;
    std::unique_ptr<Block> block;
    std::unique_ptr<State> state;
};

}  // namespace

extern "C" {

const char* q3ref_last_error() { return g_last_error.c_str(); }

// ---------------------------------------------------------------- whole model

int q3ref_load(const char* path, int ctx, void** out) {
    return Guard([&] {
        auto m = std::make_unique<RefModel>();
        m->model = std::make_unique<Qwen3>(std::string(path), ctx);
        m->cfg = std::make_shared<Config>(*m->model->GetConfig());
        m->state = std::make_unique<State>(m->cfg);
        *out = m.release();
    });
}

void q3ref_free(void* h) { delete static_cast<RefModel*>(h); }

// ints: dim hidden_dim head_dim n_layers n_heads n_kv_heads vocab_size max_seq_len
//       bos eos rotary_dim tie qk_norm attention_bias ; floats: rope_theta norm_eps
int q3ref_config(void* h, int* ints, float* floats) {
    return Guard([&] {
        const Config& c = *static_cast<RefModel*>(h)->model->GetConfig();
        const int v[] = {c.dim, c.hidden_dim, c.head_dim, c.n_layers, c.n_heads, c.n_kv_heads,
                         c.vocab_size, c.max_seq_len, c.bos_token_id, c.eos_token_id,
                         c.rotary_dim, c.tie_word_embeddings, c.qk_norm, c.attention_bias};
        std::memcpy(ints, v, sizeof(v));
        floats[0] = c.rope_theta;
        floats[1] = c.norm_eps;
    });
}

int q3ref_tensor_count(void* h) {
    return static_cast<int>(static_cast<RefModel*>(h)->model->GetTensorIndex().size());
}

int q3ref_reset(void* h) {
    return Guard([&] {
        auto* m = static_cast<RefModel*>(h);
        m->model->ResetInference();
        for (Block& b : m->blocks) b.ResetCache();
    });
}

// Stock path: Qwen3::ForwardToken.
int q3ref_forward_token(void* h, int token, int pos, float* logits) {
    return Guard([&] {
        auto* m = static_cast<RefModel*>(h);
        const std::vector<float>& out = m->model->ForwardToken(token, pos, *m->state);
        if (logits) std::memcpy(logits, out.data(), out.size() * sizeof(float));
    });
}

// Per-layer path: the steps of Qwen3::ForwardToken (src/inference.cpp:594-635), with the
// hidden state after the embedding and after each layer written to hidden[(L+1)*dim].
int q3ref_forward_layers(void* h, int token, int pos, float* hidden_out, float* logits_out) {
    return Guard([&] {
        auto* m = static_cast<RefModel*>(h);
        m->EnsureBlocks();
        const Config& c = *m->cfg;
        if (token < 0 || token >= c.vocab_size) {
            throw std::out_of_range("Token id is outside the vocabulary");
        }
        if (pos < 0) {
            throw std::out_of_range("Token position must not be negative");
        }
        const auto* row = m->embed.data() + static_cast<size_t>(token) * c.dim;
        for (int i = 0; i < c.dim; ++i) m->hidden[i] = static_cast<float>(row[i]);
        constexpr int kAttentionSinks = 4;
        const int ctx = c.max_seq_len;
        const int num_sink = pos >= ctx ? std::min(kAttentionSinks, ctx - 1) : 0;
        const int kv_pos = pos < ctx ? pos : num_sink + (pos - num_sink) % (ctx - num_sink);
        const int kv_len = std::min(pos + 1, ctx);
        if (hidden_out) std::memcpy(hidden_out, m->hidden.data(), c.dim * sizeof(float));
        for (int l = 0; l < c.n_layers; ++l) {
            m->blocks[l].forward(m->hidden.data(), pos, num_sink, kv_pos, kv_len, *m->state);
            if (hidden_out) {
                std::memcpy(hidden_out + static_cast<size_t>(l + 1) * c.dim, m->hidden.data(),
                            c.dim * sizeof(float));
            }
        }
        RmsNorm(m->normed.data(), m->hidden.data(), m->final_norm.data(), c.norm_eps, c.dim);
        MatMul(m->logits.data(), m->normed.data(), m->embed.data(), c.vocab_size, c.dim);
        if (logits_out) {
            std::memcpy(logits_out, m->logits.data(), m->logits.size() * sizeof(float));
        }
    });
}

// KV-cache row kv_pos of one layer, from the per-layer path's blocks.
int q3ref_kv_row(void* h, int layer, int kv_pos, std::uint16_t* k, std::uint16_t* v) {
    return Guard([&] {
        auto* m = static_cast<RefModel*>(h);
        m->EnsureBlocks();
        const KVCache& cache = m->blocks.at(layer).GetCache();
        const int kv_dim = cache.n_kv_heads * cache.head_dim;
        if (kv_pos < 0 || kv_pos >= cache.seq_len) throw std::out_of_range("kv_pos");
        std::memcpy(k, cache.k_.data() + static_cast<size_t>(kv_pos) * kv_dim, kv_dim * 2);
        std::memcpy(v, cache.v_.data() + static_cast<size_t>(kv_pos) * kv_dim, kv_dim * 2);
    });
}

// The prefill and greedy decode loops of Qwen3::Generate (src/inference.cpp:663-697) on token
// IDs, with `--benchmark N` semantics (src/main.cpp:78): exactly `steps` tokens, EOS ignored.
int q3ref_generate_ids(void* h, const int* prompt, int n_prompt, int steps, int* out_tokens,
                       double* prefill_s, double* decode_s) {
    return Guard([&] {
        auto* m = static_cast<RefModel*>(h);
        int pos = 0;
        const std::vector<float>* logits = nullptr;
        const auto t0 = std::chrono::steady_clock::now();
        State state(m->cfg);
        for (int i = 0; i < n_prompt; ++i) logits = &m->model->ForwardToken(prompt[i], pos++, state);
        const auto t1 = std::chrono::steady_clock::now();
        const auto t2 = std::chrono::steady_clock::now();
        for (int i = 0; i < steps; ++i) {
            const auto token = Sampler::Greedy(*logits);
            out_tokens[i] = token;
            logits = &m->model->ForwardToken(token, pos++, state);
        }
        const auto t3 = std::chrono::steady_clock::now();
        *prefill_s = std::chrono::duration<double>(t1 - t0).count();
        *decode_s = std::chrono::duration<double>(t3 - t2).count();
    });
}

// ---------------------------------------------------------------- single block

// ints: dim hidden_dim head_dim n_heads n_kv_heads max_seq_len rotary_dim; floats: theta eps
// w: attn_norm q_norm k_norm wq wk wv wo mlp_norm w1 w2 w3 (bf16 bits)
int q3ref_block_create(const int* ints, const float* floats, const std::uint16_t* const* w,
                       void** out) {
    return Guard([&] {
        auto b = std::make_unique<RefBlock>();
        b->cfg = std::make_shared<Config>();
        Config& c = *b->cfg;
        c.dim = ints[0];
        c.hidden_dim = ints[1];
        c.head_dim = ints[2];
        c.n_heads = ints[3];
        c.n_kv_heads = ints[4];
        c.max_seq_len = ints[5];
        c.rotary_dim = ints[6];
        c.rope_theta = floats[0];
        c.norm_eps = floats[1];
        const size_t d = c.dim, hd = c.head_dim, hid = c.hidden_dim;
        const size_t qd = static_cast<size_t>(c.n_heads) * hd;
        const size_t kvd = static_cast<size_t>(c.n_kv_heads) * hd;
        BlockWeights bw;
        bw.attn_norm = ToBf16Vector(w[0], d);
        bw.q_norm = ToBf16Vector(w[1], hd);
        bw.k_norm = ToBf16Vector(w[2], hd);
        bw.wq = ToBf16Vector(w[3], qd * d);
        bw.wk = ToBf16Vector(w[4], kvd * d);
        bw.wv = ToBf16Vector(w[5], kvd * d);
        bw.wo = ToBf16Vector(w[6], d * qd);
        bw.mlp_norm = ToBf16Vector(w[7], d);
        bw.w1 = ToBf16Vector(w[8], hid * d);
        bw.w2 = ToBf16Vector(w[9], d * hid);
        bw.w3 = ToBf16Vector(w[10], hid * d);
        b->block = std::make_unique<Block>(b->cfg, std::move(bw));
        b->state = std::make_unique<State>(b->cfg);
        *out = b.release();
    });
}

void q3ref_block_free(void* h) { delete static_cast<RefBlock*>(h); }

int q3ref_block_forward(void* h, float* x, int pos, int num_sink, int kv_pos, int kv_len) {
    return Guard([&] {
        auto* b = static_cast<RefBlock*>(h);
        b->block->forward(x, pos, num_sink, kv_pos, kv_len, *b->state);
    });
}

int q3ref_block_reset(void* h) {
    return Guard([&] { static_cast<RefBlock*>(h)->block->ResetCache(); });
}

// The cache is a private member with only a const getter (include/inference.h:193-195); the
// block test fills it through a const_cast, as the reference offers no setter.
int q3ref_block_set_cache(void* h, const std::uint16_t* k, const std::uint16_t* v) {
    return Guard([&] {
        auto& cache = const_cast<KVCache&>(static_cast<RefBlock*>(h)->block->GetCache());
        std::memcpy(cache.k_.data(), k, cache.k_.size() * 2);
        std::memcpy(cache.v_.data(), v, cache.v_.size() * 2);
    });
}

int q3ref_block_get_cache(void* h, std::uint16_t* k, std::uint16_t* v) {
    return Guard([&] {
        const auto& cache = static_cast<RefBlock*>(h)->block->GetCache();
        std::memcpy(k, cache.k_.data(), cache.k_.size() * 2);
        std::memcpy(v, cache.v_.data(), cache.v_.size() * 2);
    });
}

// ---------------------------------------------------------------- free functions

void q3ref_rmsnorm(float* out, const float* x, const std::uint16_t* w, float eps, int n) {
    RmsNorm(out, x, reinterpret_cast<const std::bfloat16_t*>(w), eps, n);
}

void q3ref_softmax(float* out, const float* x, int n) { Softmax(out, x, n); }

float q3ref_silu(float x) { return Silu(x); }

void q3ref_matmul(float* out, const float* x, const std::uint16_t* w, int n, int m) {
    MatMul(out, x, reinterpret_cast<const std::bfloat16_t*>(w), n, m);
}

void q3ref_rope(float* out, int d, int head_dim, int pos, float theta, int rotary_dim) {
    ApplyRotaryEmb(out, d, head_dim, pos, theta, rotary_dim);
}

void q3ref_ffn(float* out, float* lin1, float* lin2, const float* x, const std::uint16_t* w1,
               const std::uint16_t* w2, const std::uint16_t* w3, int hidden_dim, int dim) {
    FeedForwardNetwork(out, lin1, lin2, x, reinterpret_cast<const std::bfloat16_t*>(w1),
                       reinterpret_cast<const std::bfloat16_t*>(w2),
                       reinterpret_cast<const std::bfloat16_t*>(w3), hidden_dim, dim);
}

void q3ref_fastattn(float* out, float* atth, const float* q, const std::uint16_t* k,
                    const std::uint16_t* v, int head_dim, int n_kv_heads, int kv_len) {
    FastAttn(out, atth, q, reinterpret_cast<const std::bfloat16_t*>(k),
             reinterpret_cast<const std::bfloat16_t*>(v), head_dim, n_kv_heads, kv_len);
}

int q3ref_greedy(const float* logits, int n, int* out) {
    return Guard([&] { *out = Sampler::Greedy(std::span<const float>(logits, n)); });
}

}  // extern "C"
