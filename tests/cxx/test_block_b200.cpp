// The checks of the reference's tst/test_block.cpp (lines 90-192) through the C++ surface of
// include/inference_b200.h on the GPU: rotary embedding, greedy sampling, softmax stability,
// a block whose query heads outnumber the model width, GQA value sharing, the normalised key in
// the cache, ResetCache, and the out_of_range rejection of a write into the sink region.
// Exit status 0 and "block tests passed" on success.
#include "inference_b200.h"

#include <algorithm>
#include <cmath>
#include <iostream>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

using namespace q3b200;

namespace {

void Expect(bool ok, const std::string& what) {
    if (!ok) throw std::runtime_error(what);
}

// |actual - expected| <= 1e-5 (tst/test_block.cpp:19-25).
void ExpectNear(float actual, float expected, const std::string& what) {
    if (!(std::fabs(actual - expected) <= 1e-5f)) {
        throw std::runtime_error(what + ": expected " + std::to_string(expected) + ", got " +
                                 std::to_string(actual));
    }
}

using bf16 = std::bfloat16_t;

float RoundBf16(float v) { return static_cast<float>(static_cast<bf16>(v)); }

std::vector<bf16> Filled(size_t n, float v) { return std::vector<bf16>(n, static_cast<bf16>(v)); }

std::vector<bf16> FromFloats(std::initializer_list<float> vals) {
    std::vector<bf16> out;
    for (float v : vals) out.push_back(static_cast<bf16>(v));
    return out;
}

std::shared_ptr<Config> SmallConfig(int dim, int hidden_dim, int max_seq_len) {
    auto c = std::make_shared<Config>();
    c->dim = dim;
    c->hidden_dim = hidden_dim;
    c->head_dim = 2;
    c->n_heads = 2;
    c->n_kv_heads = 1;
    c->max_seq_len = max_seq_len;
    c->rotary_dim = 2;
    c->rope_theta = 10000.0f;
    c->norm_eps = 1e-5f;
    return c;
}

// dim 4: wk picks x[0..1], wv picks x[2..3], wo is the identity, the MLP is zero.
BlockWeights GqaWeights() {
    BlockWeights w;
    w.attn_norm = Filled(4, 1.0f);
    w.q_norm = Filled(2, 1.0f);
    w.k_norm = Filled(2, 1.0f);
    w.wq = Filled(16, 0.0f);
    w.wk = FromFloats({1, 0, 0, 0, 0, 1, 0, 0});
    w.wv = FromFloats({0, 0, 1, 0, 0, 0, 0, 1});
    w.wo = Filled(16, 0.0f);
    for (int i = 0; i < 4; ++i) w.wo[i * 4 + i] = static_cast<bf16>(1.0f);
    w.mlp_norm = Filled(4, 1.0f);
    w.w1 = Filled(8, 0.0f);
    w.w2 = Filled(8, 0.0f);
    w.w3 = Filled(8, 0.0f);
    return w;
}

// dim 2 with 2 query heads of head_dim 2: q_dim (4) is wider than the model (2).
BlockWeights ExpandedQueryWeights() {
    BlockWeights w;
    w.attn_norm = Filled(2, 1.0f);
    w.q_norm = Filled(2, 1.0f);
    w.k_norm = Filled(2, 1.0f);
    w.wq = Filled(8, 0.0f);
    w.wk = Filled(4, 0.0f);
    w.wv = Filled(4, 0.0f);
    w.wo = Filled(8, 0.0f);
    w.mlp_norm = Filled(2, 1.0f);
    w.w1 = Filled(4, 0.0f);
    w.w2 = Filled(4, 0.0f);
    w.w3 = Filled(4, 0.0f);
    return w;
}

}  // namespace

int main() {
    try {
        float rot[] = {1.0f, 2.0f, 3.0f, 4.0f};
        ApplyRotaryEmb(rot, 4, 4, 1, 10000.0f, 4);
        ExpectNear(rot[0], std::cos(1.0f) - 3.0f * std::sin(1.0f), "rotary first half 0");
        ExpectNear(rot[2], 3.0f * std::cos(1.0f) + std::sin(1.0f), "rotary second half 0");
        ExpectNear(rot[1], 2.0f * std::cos(0.01f) - 4.0f * std::sin(0.01f), "rotary first half 1");
        ExpectNear(rot[3], 4.0f * std::cos(0.01f) + 2.0f * std::sin(0.01f), "rotary second half 1");

        const std::vector<float> logits = {-2.0f, 0.5f, 0.25f};
        Expect(Sampler::Greedy(logits) == 1, "greedy sampler chose the wrong token");
        bool empty_rejected = false;
        try {
            Sampler::Greedy(std::span<const float>{});
        } catch (const std::invalid_argument&) {
            empty_rejected = true;
        }
        Expect(empty_rejected, "greedy sampler accepted empty logits");

        float sm[] = {-10000.0f, -10001.0f, -10002.0f};
        Softmax(sm, sm, 3);
        const float total = 1.0f + std::exp(-1.0f) + std::exp(-2.0f);
        ExpectNear(sm[0], 1.0f / total, "softmax large-negative value 0");
        ExpectNear(sm[1], std::exp(-1.0f) / total, "softmax large-negative value 1");
        ExpectNear(sm[2], std::exp(-2.0f) / total, "softmax large-negative value 2");

        auto expanded = SmallConfig(2, 2, 2);
        Block expanded_block(expanded, ExpandedQueryWeights());
        float ex[] = {1.0f, -1.0f};
        State state(expanded);
        expanded_block.forward(ex, 0, 0, 0, 1, state);
        ExpectNear(ex[0], 1.0f, "expanded-query residual 0");
        ExpectNear(ex[1], -1.0f, "expanded-query residual 1");

        auto config = SmallConfig(4, 2, 4);
        Block block(config, GqaWeights());
        float x[] = {1.0f, 2.0f, 3.0f, 4.0f};
        const float rms = std::sqrt(7.5f + config->norm_eps);
        block.forward(x, 0, 0, 0, 1);
        // Both query heads read the one KV head: the same value lands in both halves.
        const float v0 = RoundBf16(3.0f / rms);
        const float v1 = RoundBf16(4.0f / rms);
        ExpectNear(x[0], 1.0f + v0, "first attention residual");
        ExpectNear(x[1], 2.0f + v1, "second attention residual");
        ExpectNear(x[2], 3.0f + v0, "GQA first value");
        ExpectNear(x[3], 4.0f + v1, "GQA second value");

        KVCache cache = block.GetCache();
        const float key_rms = std::sqrt(
            ((1.0f / rms) * (1.0f / rms) + (2.0f / rms) * (2.0f / rms)) / 2.0f + config->norm_eps);
        ExpectNear(static_cast<float>(cache.k_[0]), RoundBf16((1.0f / rms) / key_rms),
                   "cached normalized key 0");
        ExpectNear(static_cast<float>(cache.k_[1]), RoundBf16((2.0f / rms) / key_rms),
                   "cached normalized key 1");
        ExpectNear(static_cast<float>(cache.v_[0]), v0, "cached value 0");
        ExpectNear(static_cast<float>(cache.v_[1]), v1, "cached value 1");

        block.ResetCache();
        cache = block.GetCache();
        const auto zero = [](bf16 b) { return static_cast<float>(b) == 0.0f; };
        Expect(std::all_of(cache.k_.begin(), cache.k_.end(), zero), "ResetCache left keys");
        Expect(std::all_of(cache.v_.begin(), cache.v_.end(), zero), "ResetCache left values");

        // SetCache round trip (the reference's test writes the cache through GetCache).
        for (size_t i = 0; i < cache.k_.size(); ++i) {
            cache.k_[i] = static_cast<bf16>(0.25f * static_cast<float>(i));
            cache.v_[i] = static_cast<bf16>(-0.5f * static_cast<float>(i));
        }
        block.SetCache(cache);
        const KVCache back = block.GetCache();
        for (size_t i = 0; i < cache.k_.size(); ++i) {
            Expect(static_cast<float>(back.k_[i]) == static_cast<float>(cache.k_[i]) &&
                       static_cast<float>(back.v_[i]) == static_cast<float>(cache.v_[i]),
                   "SetCache/GetCache round trip");
        }

        bool rejected = false;
        try {
            block.forward(x, 4, 1, 0, 4, state);
        } catch (const std::out_of_range&) {
            rejected = true;
        }
        Expect(rejected, "Block accepted a write into the sink region");

        bool bad_weights = false;
        try {
            BlockWeights w = GqaWeights();
            w.wo.pop_back();
            Block b(config, std::move(w));
        } catch (const std::invalid_argument&) {
            bad_weights = true;
        }
        Expect(bad_weights, "Block accepted a wrongly sized weight");

        std::cout << "block tests passed\n";
    } catch (const std::exception& e) {
        std::cerr << "block test failed: " << e.what() << '\n';
        return 1;
    }
    return 0;
}
