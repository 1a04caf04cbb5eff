// The checks of the reference's tst/test_loader.cpp (config, tensor index, LoadTensor) through
// include/inference_b200.h, on a Qwen3-0.6B-shaped Qwen3.bin written without tokenizer records
// (so 310 records rather than the 313 of a converted checkpoint), plus the Qwen3 calls a user
// makes: ForwardToken, Generate with and without the per-token callback, ResetInference.
// Usage: test_loader_b200 <Qwen3.bin>. Exit status 0 and "loader tests passed" on success.
#include "inference_b200.h"

#include <algorithm>
#include <cmath>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

using namespace q3b200;

namespace {

void Expect(bool ok, const std::string& what) {
    if (!ok) throw std::runtime_error(what);
}

const TensorInfo& Find(const Qwen3& model, const std::string& name) {
    const auto& index = model.GetTensorIndex();
    const auto it = index.find(name);
    if (it == index.end()) throw std::runtime_error("missing tensor: " + name);
    return it->second;
}

}  // namespace

int main(int argc, char** argv) {
    const std::string path = argc > 1 ? argv[1] : "Qwen3.bin";
    try {
        Qwen3 model(path, 256);
        Expect(model.GetConfig() != nullptr, "missing model config");
        const Config& c = *model.GetConfig();
        Expect(c.arch == "Qwen3ForCausalLM", "unexpected architecture");
        Expect(c.dtype == "bf16", "unexpected dtype");
        Expect(c.dim == 1024 && c.hidden_dim == 3072 && c.head_dim == 128, "unexpected widths");
        Expect(c.n_layers == 28 && c.n_heads == 16 && c.n_kv_heads == 8, "unexpected layout");
        Expect(c.vocab_size == 151936, "unexpected vocab size");
        Expect(c.max_seq_len == 256, "context length not applied");
        Expect(c.bos_token_id >= 0 && c.eos_token_id >= 0, "invalid special token ids");
        Expect(c.tie_word_embeddings && c.qk_norm, "expected tied embeddings and q/k norm");
        Expect(model.GetTensorIndex().size() == 310, "unexpected tensor record count");

        const TensorInfo& embed = Find(model, "model.embed.weight");
        Expect(embed.dtype == TensorDType::BFloat16, "embedding dtype should be bf16");
        Expect(embed.shape.size() == 2 && embed.shape[0] == 151936u && embed.shape[1] == 1024u,
               "embedding shape mismatch");
        Expect(embed.byte_size == 311164928u, "embedding byte size mismatch");
        Expect(embed.data_offset > 0, "embedding data offset should be positive");

        const TensorInfo& qn = Find(model, "model.layers.0.attn.q_norm.weight");
        Expect(qn.dtype == TensorDType::BFloat16 && qn.shape.size() == 1 && qn.shape[0] == 128u,
               "q_norm record mismatch");
        const Tensor<std::bfloat16_t> qt = model.LoadTensor<std::bfloat16_t>(qn.name);
        Expect(qt.data.size() * sizeof(std::bfloat16_t) == qn.byte_size, "q_norm payload size");
        Expect(qt.ptr() != nullptr && qt.data.size() == 128u, "q_norm bf16 view");

        bool mismatch = false;
        try {
            (void)model.LoadTensor<float>(qn.name);
        } catch (const std::runtime_error&) {
            mismatch = true;
        }
        Expect(mismatch, "LoadTensor accepted the wrong element type");
        bool missing = false;
        try {
            (void)model.LoadTensor<std::bfloat16_t>("no.such.tensor");
        } catch (const std::runtime_error&) {
            missing = true;
        }
        Expect(missing, "LoadTensor accepted an unknown name");

        // ForwardToken and the range check on token ids.
        State state;
        const std::vector<float>& logits = model.ForwardToken(17, 0, state);
        Expect(logits.size() == 151936u, "logits size");
        Expect(std::all_of(logits.begin(), logits.end(), [](float v) { return v == v; }),
               "logits contain NaN");
        bool range = false;
        try {
            model.ForwardToken(151936, 1);
        } catch (const std::out_of_range&) {
            range = true;
        }
        Expect(range, "ForwardToken accepted an out-of-range token id");

        // Generate: device loop and per-token callback loop give the same greedy tokens.
        const std::vector<std::int32_t> prompt = {9707, 11, 1879, 0, 42, 151643, 7, 3};
        model.ResetInference();
        const GenerationResult a = model.Generate(prompt, 12, false);
        model.ResetInference();
        size_t calls = 0;
        const GenerationResult b = model.Generate(prompt, 12, false,
                                                  [&](std::span<const std::int32_t> toks) {
                                                      ++calls;
                                                      Expect(toks.size() == calls,
                                                             "callback span size");
                                                  });
        Expect(a.tokens.size() == 12 && b.tokens.size() == 12, "Generate token counts");
        // The two paths agree token for token, or first part at a near tie: the down-projection
        // sums use fp32 atomics whose order varies from run to run, so where two logits are
        // closer than twice the logit tolerance either token is a correct greedy choice.
        size_t first = 0;
        while (first < a.tokens.size() && a.tokens[first] == b.tokens[first]) ++first;
        if (first < a.tokens.size()) {
            model.ResetInference();
            int pos = 0;
            const std::vector<float>* lg = nullptr;
            for (const std::int32_t t : prompt) lg = &model.ForwardToken(t, pos++, state);
            for (size_t i = 0; i < first; ++i) lg = &model.ForwardToken(a.tokens[i], pos++, state);
            const float gap = std::fabs((*lg)[a.tokens[first]] - (*lg)[b.tokens[first]]);
            Expect(gap <= 0.1f, "Generate paths disagree at token " + std::to_string(first) +
                                    " by a logit gap of " + std::to_string(gap));
        }
        Expect(calls == 12, "callback count");
        Expect(a.stats.prompt_tokens == prompt.size() && a.stats.generated_tokens == 12,
               "generation stats");
        Expect(a.stats.reached_token_limit && !a.stats.stopped_on_eos, "generation flags");
        Expect(a.stats.DecodeTokensPerSecond() > 0.0, "decode rate");

        // An empty prompt becomes [bos] (src/inference.cpp:656-658).
        model.ResetInference();
        const GenerationResult e = model.Generate(std::span<const std::int32_t>{}, 2, false);
        Expect(e.stats.prompt_tokens == 1 && e.tokens.size() == 2, "empty prompt handling");

        std::cout << "loader tests passed\n";
    } catch (const std::exception& err) {
        std::cerr << "loader test failed: " << err.what() << '\n';
        return 1;
    }
    return 0;
}
