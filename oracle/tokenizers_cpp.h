// Test infrastructure only: a stand-in for the mlc-ai/tokenizers-cpp header so that the
// reference engine (src/inference.cpp) compiles without its Rust tokenizer backend.
//
// The reference includes <tokenizers_cpp.h> (src/inference.cpp:3) and uses exactly five
// members of tokenizers::Tokenizer: FromBlobJSON (src/inference.cpp:374), GetVocabSize
// (:398), IdToToken (:413), Encode (:433) and Decode (:440). The dependency is an
// un-vendored git submodule (.gitmodules:1-3) and needs cargo, which is not installed.
// None of it is on the forward path: the oracle drives the engine with token IDs.
//
// FromBlobJSON returns null, so a Qwen3.bin with an embedded tokenizer.json makes the
// reference constructor throw "Failed to initialize tokenizer backend"
// (src/inference.cpp:375-377). Weight files written for parity tests carry no tokenizer
// records, so the constructor never reaches that branch.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace tokenizers {

class Tokenizer {
public:
    virtual ~Tokenizer() = default;

    static std::unique_ptr<Tokenizer> FromBlobJSON(const std::string&) { return nullptr; }

    std::vector<std::int32_t> Encode(const std::string&) { return {}; }
    std::string Decode(const std::vector<std::int32_t>&) { return {}; }
    std::size_t GetVocabSize() { return 0; }
    std::string IdToToken(std::int32_t) { return {}; }
};

}  // namespace tokenizers
