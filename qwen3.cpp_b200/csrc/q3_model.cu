// Host side of the B200 Qwen3 library: Qwen3.bin loader, HBM arena, KV cache, per-step CUDA
// graphs, and the C ABI of include/q3_b200.h.
//
// The loader restates the reference's (asriva32/Qwen3.cpp src/inference.cpp:17-263, :445-581)
// checks and error kinds; the forward orchestration restates Qwen3::ForwardToken (:592-637) and
// Block::forward (:766-866) as a fixed sequence of kernel launches captured once into a CUDA
// graph and replayed for every token, with the per-step scalars in device memory.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <limits>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "q3_common.cuh"
#include "q3_decode_fused.cuh"
#include "q3_kernels.cuh"
#include "q3_model.cuh"
#include "q3_prefill.cuh"
#include "q3_batch.cuh"
#include "q3_tp.cuh"

namespace q3 {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

// ------------------------------------------------------------------ Qwen3.bin parsing

namespace {

constexpr char kMagic[8] = {'Q', 'W', 'E', 'N', '3', 'C', 'P', '\0'};
constexpr uint32_t kVersion = 1;

enum DType : uint32_t { kF32 = 1, kBF16 = 3, kU8 = 4, kI32 = 5 };

size_t dtype_size(uint32_t d) {
    switch (d) {
        case kF32: return 4;
        case kBF16: return 2;
        case kU8: return 1;
        case kI32: return 4;
    }
    throw std::runtime_error("Unknown tensor dtype");
}

struct Reader {
    const uint8_t* p;
    size_t size;
    size_t off = 0;
    template <typename T>
    T pod() {
        if (off + sizeof(T) > size) throw std::runtime_error("Unexpected end of Qwen3.bin");
        T v;
        std::memcpy(&v, p + off, sizeof(T));
        off += sizeof(T);
        return v;
    }
    std::string str(uint64_t n) {
        if (off + n > size) throw std::runtime_error("Unexpected end of Qwen3.bin while reading string");
        std::string s(reinterpret_cast<const char*>(p + off), n);
        off += n;
        return s;
    }
};

// JsonValue (src/inference.cpp:97-124): the naive `"key":` lookup of the reference.
std::string json_value(const std::string& js, const std::string& key) {
    const std::string qk = "\"" + key + "\":";
    const size_t kp = js.find(qk);
    if (kp == std::string::npos) throw std::runtime_error("Missing metadata key: " + key);
    size_t p = kp + qk.size();
    while (p < js.size() && js[p] == ' ') ++p;
    if (p >= js.size()) throw std::runtime_error("Malformed metadata value for: " + key);
    if (js[p] == '"') {
        const size_t e = js.find('"', p + 1);
        if (e == std::string::npos) {
            throw std::runtime_error("Unterminated string metadata value for: " + key);
        }
        return js.substr(p + 1, e - p - 1);
    }
    const size_t e = js.find_first_of(",}", p);
    if (e == std::string::npos) throw std::runtime_error("Unterminated metadata value for: " + key);
    return js.substr(p, e - p);
}

bool json_bool(const std::string& js, const std::string& key) {
    const std::string v = json_value(js, key);
    if (v == "true") return true;
    if (v == "false") return false;
    throw std::runtime_error("Metadata value is not bool for: " + key);
}

}  // namespace

// ValidateConfig (src/inference.cpp:145-157).
void validate_config(const q3_config& c) {
    if (c.dim <= 0 || c.hidden_dim <= 0 || c.head_dim <= 0 || c.n_heads <= 0 ||
        c.n_kv_heads <= 0 || c.max_seq_len <= 0) {
        throw std::invalid_argument("Block config dimensions must be positive");
    }
    if (c.n_heads % c.n_kv_heads != 0) {
        throw std::invalid_argument("Attention head count must be divisible by KV head count");
    }
    if (c.rotary_dim < 0 || c.rotary_dim > c.head_dim || c.rotary_dim % 2 != 0) {
        throw std::invalid_argument("rotary_dim must be even and no larger than head_dim");
    }
}

// Limits of the CUDA kernels beyond the reference's own checks.
void validate_kernel_limits(const q3_config& c) {
    if (c.head_dim > 256) throw std::invalid_argument("head_dim above 256 is not supported");
    if (c.n_heads / c.n_kv_heads > 8) {
        throw std::invalid_argument("more than 8 query heads per KV head is not supported");
    }
}

ModelFile::ModelFile(const std::string& path) : path_(path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("Failed to open model file: " + path);
    struct stat st {};
    if (fstat(fd_, &st) != 0) throw std::runtime_error("Failed to open model file: " + path);
    size_ = static_cast<size_t>(st.st_size);
    if (size_ > 0) {
        void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (m == MAP_FAILED) throw std::runtime_error("Failed to map model file: " + path);
        data_ = static_cast<const uint8_t*>(m);
    }
    Reader r{data_, size_};
    if (size_ < 8 || std::memcmp(data_, kMagic, 8) != 0) {
        throw std::runtime_error("Invalid Qwen3 model file magic");
    }
    r.off = 8;
    if (r.pod<uint32_t>() != kVersion) throw std::runtime_error("Unsupported Qwen3 model file version");
    const auto meta_size = r.pod<uint64_t>();
    const std::string js = r.str(meta_size);
    // ParseConfig (src/inference.cpp:159-182).
    arch_ = json_value(js, "arch");
    dtype_ = json_value(js, "dtype");
    act_ = json_value(js, "act_type");
    q3_config& c = config_;
    c.dim = std::stoi(json_value(js, "dim"));
    c.hidden_dim = std::stoi(json_value(js, "hidden_dim"));
    c.head_dim = std::stoi(json_value(js, "head_dim"));
    c.n_layers = std::stoi(json_value(js, "n_layers"));
    c.n_heads = std::stoi(json_value(js, "n_heads"));
    c.n_kv_heads = std::stoi(json_value(js, "n_kv_heads"));
    c.vocab_size = std::stoi(json_value(js, "vocab_size"));
    c.max_seq_len = std::stoi(json_value(js, "max_seq_len"));
    c.bos_token_id = std::stoi(json_value(js, "bos_token_id"));
    c.eos_token_id = std::stoi(json_value(js, "eos_token_id"));
    c.rotary_dim = std::stoi(json_value(js, "rotary_dim"));
    c.rope_theta = std::stof(json_value(js, "rope_theta"));
    c.norm_eps = std::stof(json_value(js, "norm_eps"));
    c.tie_word_embeddings = json_bool(js, "tie_word_embeddings");
    c.attention_bias = json_bool(js, "attention_bias");
    c.qk_norm = json_bool(js, "qk_norm");
    validate_config(c);
    if (dtype_ != "bf16") throw std::runtime_error("Only bf16 Qwen3.bin files are supported");

    const auto count = r.pod<uint64_t>();
    for (uint64_t i = 0; i < count; ++i) {
        Tensor t;
        const auto nlen = r.pod<uint32_t>();
        t.name = r.str(nlen);
        t.dtype = r.pod<uint32_t>();
        const auto ndim = r.pod<uint32_t>();
        for (uint32_t d = 0; d < ndim; ++d) t.shape.push_back(r.pod<uint64_t>());
        t.byte_size = r.pod<uint64_t>();
        t.offset = r.off;
        // ValidateTensorByteSize (:85-95) and ValidateSupportedTensorType (:211-232).
        size_t n = 1;
        for (auto d : t.shape) {
            if (d != 0 && n > std::numeric_limits<size_t>::max() / d) {
                throw std::runtime_error("Tensor shape element count overflow");
            }
            n *= d;
        }
        if (n * dtype_size(t.dtype) != t.byte_size) {
            throw std::runtime_error("Tensor byte size mismatch for " + t.name);
        }
        const bool tok = t.name == "tokenizer.json" || t.name == "tokenizer.tokens" ||
                         t.name == "tokenizer.offsets";
        if (tok) {
            const bool ok = (t.name != "tokenizer.offsets" && t.dtype == kU8) ||
                            (t.name == "tokenizer.offsets" && t.dtype == kI32);
            if (!ok) throw std::runtime_error("Unsupported tokenizer tensor dtype for " + t.name);
        } else if (t.dtype != kBF16) {
            throw std::runtime_error("Only bf16 model tensors are supported: " + t.name);
        }
        if (t.offset + t.byte_size > size_) {
            throw std::runtime_error("Unexpected end of Qwen3.bin while skipping tensor payload");
        }
        if (!tensors_.emplace(t.name, t).second) {
            throw std::runtime_error("Duplicate tensor record: " + t.name);
        }
        names_.push_back(t.name);
        r.off += t.byte_size;
    }
}

ModelFile::~ModelFile() {
    if (data_) munmap(const_cast<uint8_t*>(data_), size_);
    if (fd_ >= 0) ::close(fd_);
}

const ModelFile::Tensor& ModelFile::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw std::runtime_error("Tensor not found: " + name);
    return it->second;
}

const std::string& ModelFile::metadata(const std::string& key) const {
    if (key == "arch") return arch_;
    if (key == "dtype") return dtype_;
    if (key == "act_type") return act_;
    throw std::invalid_argument("Unknown metadata key: " + key);
}

// ------------------------------------------------------------------ device buffers

DeviceBuffer::~DeviceBuffer() { reset(); }
void DeviceBuffer::reset() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
}
void DeviceBuffer::alloc(size_t n) {
    reset();
    if (n == 0) return;
    Q3_CUDA(cudaMalloc(&ptr, n));
    bytes = n;
}

PinnedBuffer::~PinnedBuffer() {
    if (ptr) cudaFreeHost(ptr);
}
void PinnedBuffer::ensure(size_t n) {
    if (n <= bytes) return;
    if (ptr) cudaFreeHost(ptr);
    ptr = nullptr;
    Q3_CUDA(cudaMallocHost(&ptr, n));
    bytes = n;
}

// ------------------------------------------------------------------ RoPE table

// cos/sin of RoPE evaluated on the host with the reference's fp32 expressions
// (src/inference.cpp:979-982), for positions [0, len).
std::vector<float2> rope_table_host(float theta, int rotary_dim, int len) {
    const int half = rotary_dim / 2;
    std::vector<float2> t(static_cast<size_t>(len) * (half > 0 ? half : 0));
    std::vector<float> freq(half);
    for (int i = 0; i < half; ++i) {
        freq[i] = 1.0f / powf(theta, 2.0f * i / rotary_dim);
    }
    for (int p = 0; p < len; ++p) {
        for (int i = 0; i < half; ++i) {
            const float angle = p * freq[i];
            t[static_cast<size_t>(p) * half + i] = make_float2(cosf(angle), sinf(angle));
        }
    }
    return t;
}

// ------------------------------------------------------------------ layer engine

Engine::Engine(const q3_config& cfg, int n_layers, int device, int kv_slots)
    : cfg_(cfg), n_layers_(n_layers), device_(device), kv_slots_(kv_slots) {
    Q3_CUDA(cudaSetDevice(device_));
    Q3_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    const int hd = cfg.head_dim, nq = cfg.n_heads, nk = cfg.n_kv_heads;
    q_dim_ = nq * hd;
    kv_dim_ = nk * hd;
    n_pages_ = (kv_slots_ + kPageTokens - 1) / kPageTokens;
    n_splits_ = attn_splits_for(kv_slots_);
    page_elems_ = static_cast<size_t>(nk) * kPageTokens * hd;
    const size_t layer_kv = static_cast<size_t>(n_pages_) * page_elems_;
    k_cache_.alloc(layer_kv * n_layers * 2);
    v_cache_.alloc(layer_kv * n_layers * 2);
    std::vector<int32_t> table(n_pages_);
    for (int i = 0; i < n_pages_; ++i) table[i] = i;
    page_table_.alloc(table.size() * 4);
    Q3_CUDA(cudaMemcpy(page_table_.ptr, table.data(), table.size() * 4, cudaMemcpyHostToDevice));

    sp_.alloc(sizeof(StepParams));
    x_.alloc(cfg.dim * 4);
    qkv_.alloc((q_dim_ + 2 * kv_dim_) * 4);
    att_.alloc(q_dim_ * 4);
    h_.alloc(static_cast<size_t>(cfg.hidden_dim) * 4);
    part_o_.alloc(static_cast<size_t>(nq) * n_splits_ * hd * 4);
    part_ml_.alloc(static_cast<size_t>(nq) * n_splits_ * sizeof(float2));
    taps_.alloc(static_cast<size_t>(n_layers + 1) * cfg.dim * 4);
    pinned_sp_.ensure(sizeof(StepParams));
    ensure_rope(kv_slots_ + 1);
    reset_cache();
}

Engine::~Engine() {
    cudaSetDevice(device_);
    for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second);
    if (stream_) cudaStreamDestroy(stream_);
}

void Engine::drop_graphs() {
    for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second);
    graphs_.clear();
}

void Engine::ensure_rope(int needed_len) {
    if (needed_len <= rope_len_) return;
    int len = rope_len_ > 0 ? rope_len_ : 1;
    while (len < needed_len) len *= 2;
    const auto t = rope_table_host(cfg_.rope_theta, cfg_.rotary_dim, len);
    Q3_CUDA(cudaStreamSynchronize(stream_));
    rope_.alloc(std::max<size_t>(t.size(), 1) * sizeof(float2));
    if (!t.empty()) {
        Q3_CUDA(cudaMemcpy(rope_.ptr, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice));
    }
    rope_len_ = len;
    drop_graphs();  // graphs hold the table pointer
}

void Engine::reset_cache() {
    Q3_CUDA(cudaMemsetAsync(k_cache_.ptr, 0, k_cache_.bytes, stream_));
    Q3_CUDA(cudaMemsetAsync(v_cache_.ptr, 0, v_cache_.bytes, stream_));
    Q3_CUDA(cudaStreamSynchronize(stream_));
}

uint16_t* Engine::k_layer(int l) const {
    return static_cast<uint16_t*>(k_cache_.ptr) + static_cast<size_t>(l) * n_pages_ * page_elems_;
}
uint16_t* Engine::v_layer(int l) const {
    return static_cast<uint16_t*>(v_cache_.ptr) + static_cast<size_t>(l) * n_pages_ * page_elems_;
}

// Block::forward (src/inference.cpp:795-865) for layer l on the engine's x_.
void Engine::enqueue_layer(int l, const LayerWeights& w) {
    const q3_config& c = cfg_;
    cudaStream_t s = stream_;
    float* x = static_cast<float*>(x_.ptr);
    float* qkv = static_cast<float*>(qkv_.ptr);
    float* att = static_cast<float*>(att_.ptr);
    float* h = static_cast<float*>(h_.ptr);
    const StepParams* sp = static_cast<const StepParams*>(sp_.ptr);
    // RmsNorm + q/k/v MatMuls (:795-798) as one GEMV over the stacked [wq; wk; wv] rows.
    launch_gemv(kEpiStore, w.wqkv, nullptr, x, w.attn_norm, c.norm_eps, qkv, nullptr,
                q_dim_ + 2 * kv_dim_, c.dim, nullptr, 0, s);
    QkvArgs qa{};
    qa.qkv = qkv;
    qa.q_norm = w.q_norm;
    qa.k_norm = w.k_norm;
    qa.rope = static_cast<const float2*>(rope_.ptr);
    qa.rope_len = rope_len_;
    qa.k_cache = k_layer(l);
    qa.v_cache = v_layer(l);
    qa.page_table = static_cast<const int32_t*>(page_table_.ptr);
    qa.sp = sp;
    qa.n_heads = c.n_heads;
    qa.n_kv = c.n_kv_heads;
    qa.hd = c.head_dim;
    qa.rotary_dim = c.rotary_dim;
    qa.eps = c.norm_eps;
    launch_qk_rope_kv(qa, s);
    AttnArgs aa{};
    aa.q = qkv;
    aa.k = k_layer(l);
    aa.v = v_layer(l);
    aa.page_table = static_cast<const int32_t*>(page_table_.ptr);
    aa.sp = sp;
    aa.n_heads = c.n_heads;
    aa.n_kv = c.n_kv_heads;
    aa.hd = c.head_dim;
    aa.row_stride = kv_dim_;
    aa.n_splits = n_splits_;
    aa.part_o = static_cast<float*>(part_o_.ptr);
    aa.part_ml = static_cast<float2*>(part_ml_.ptr);
    aa.out = att;
    launch_attention(aa, s);
    // o_proj + residual (:846-849).
    launch_gemv(kEpiResidual, w.wo, nullptr, att, nullptr, 0.0f, x, nullptr, c.dim, q_dim_,
                nullptr, 0, s);
    // RmsNorm + gate/up + SiLU*up (:851, :1005-1011), then down + residual (:1013, :863-865).
    launch_gemv(kEpiSiluMul, w.w1, w.w3, x, w.mlp_norm, c.norm_eps, h, nullptr, c.hidden_dim,
                c.dim, nullptr, 0, s);
    launch_gemv(kEpiResidual, w.w2, nullptr, h, nullptr, 0.0f, x, nullptr, c.dim, c.hidden_dim,
                nullptr, 0, s);
}

void Engine::write_step(const StepParams& p) {
    // One pinned staging slot: wait for the previous copy out of it before overwriting.
    Q3_CUDA(cudaStreamSynchronize(stream_));
    std::memcpy(pinned_sp_.ptr, &p, sizeof(p));
    Q3_CUDA(cudaMemcpyAsync(sp_.ptr, pinned_sp_.ptr, sizeof(p), cudaMemcpyHostToDevice, stream_));
}

StepParams Engine::read_step() {
    Q3_CUDA(cudaMemcpyAsync(pinned_sp_.ptr, sp_.ptr, sizeof(StepParams), cudaMemcpyDeviceToHost,
                            stream_));
    Q3_CUDA(cudaStreamSynchronize(stream_));
    StepParams p;
    std::memcpy(&p, pinned_sp_.ptr, sizeof(p));
    return p;
}

// Reference layout <-> paged layout of one layer's cache (host side, for debug taps and tests).
void Engine::read_kv_row(int l, int slot, uint16_t* k, uint16_t* v) {
    const int hd = cfg_.head_dim, nk = cfg_.n_kv_heads;
    const int page = slot / kPageTokens, off = slot % kPageTokens;  // identity page table
    for (int g = 0; g < nk; ++g) {
        const size_t e = (static_cast<size_t>(page) * nk + g) * kPageTokens * hd +
                         static_cast<size_t>(off) * hd;
        Q3_CUDA(cudaMemcpyAsync(k + g * hd, k_layer(l) + e, hd * 2, cudaMemcpyDeviceToHost, stream_));
        Q3_CUDA(cudaMemcpyAsync(v + g * hd, v_layer(l) + e, hd * 2, cudaMemcpyDeviceToHost, stream_));
    }
    Q3_CUDA(cudaStreamSynchronize(stream_));
}

void Engine::read_cache(int l, uint16_t* k, uint16_t* v, int rows) {
    const int hd = cfg_.head_dim, nk = cfg_.n_kv_heads;
    const size_t n = static_cast<size_t>(n_pages_) * page_elems_;
    std::vector<uint16_t> kp(n), vp(n);
    Q3_CUDA(cudaMemcpyAsync(kp.data(), k_layer(l), n * 2, cudaMemcpyDeviceToHost, stream_));
    Q3_CUDA(cudaMemcpyAsync(vp.data(), v_layer(l), n * 2, cudaMemcpyDeviceToHost, stream_));
    Q3_CUDA(cudaStreamSynchronize(stream_));
    for (int t = 0; t < rows; ++t) {
        for (int g = 0; g < nk; ++g) {
            const size_t e = ((static_cast<size_t>(t / kPageTokens) * nk + g) * kPageTokens +
                              t % kPageTokens) * hd;
            std::memcpy(k + (static_cast<size_t>(t) * nk + g) * hd, kp.data() + e, hd * 2);
            std::memcpy(v + (static_cast<size_t>(t) * nk + g) * hd, vp.data() + e, hd * 2);
        }
    }
}

void Engine::write_cache(int l, const uint16_t* k, const uint16_t* v, int rows) {
    const int hd = cfg_.head_dim, nk = cfg_.n_kv_heads;
    const size_t n = static_cast<size_t>(n_pages_) * page_elems_;
    std::vector<uint16_t> kp(n, 0), vp(n, 0);
    for (int t = 0; t < rows; ++t) {
        for (int g = 0; g < nk; ++g) {
            const size_t e = ((static_cast<size_t>(t / kPageTokens) * nk + g) * kPageTokens +
                              t % kPageTokens) * hd;
            std::memcpy(kp.data() + e, k + (static_cast<size_t>(t) * nk + g) * hd, hd * 2);
            std::memcpy(vp.data() + e, v + (static_cast<size_t>(t) * nk + g) * hd, hd * 2);
        }
    }
    Q3_CUDA(cudaMemcpyAsync(k_layer(l), kp.data(), n * 2, cudaMemcpyHostToDevice, stream_));
    Q3_CUDA(cudaMemcpyAsync(v_layer(l), vp.data(), n * 2, cudaMemcpyHostToDevice, stream_));
    Q3_CUDA(cudaStreamSynchronize(stream_));
}

cudaGraphExec_t Engine::graph(int key, const std::function<void()>& enqueue) {
    auto it = graphs_.find(key);
    if (it != graphs_.end()) return it->second;
    cudaGraph_t g = nullptr;
    Q3_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeRelaxed));
    try {
        enqueue();
    } catch (...) {
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    Q3_CUDA(cudaStreamEndCapture(stream_, &g));
    cudaGraphExec_t ge = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    Q3_CUDA(e);
    graphs_[key] = ge;
    return ge;
}

// ------------------------------------------------------------------ model

namespace {

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

Model::Model(const std::string& path, int ctx, int device) : file_(path) {
    cfg_ = file_.config();
    // InitializeInference (src/inference.cpp:529-581).
    if (ctx <= 0 || ctx > cfg_.max_seq_len) {
        throw std::invalid_argument("Context length is outside the model's supported range");
    }
    cfg_.max_seq_len = ctx;
    validate_kernel_limits(cfg_);
    Q3_CUDA(cudaSetDevice(device));
    device_ = device;

    const q3_config& c = cfg_;
    const size_t D = c.dim, H = c.hidden_dim, V = c.vocab_size, hd = c.head_dim;
    const size_t qd = static_cast<size_t>(c.n_heads) * hd, kvd = static_cast<size_t>(c.n_kv_heads) * hd;
    const auto& embed = file_.tensor("model.embed.weight");
    const auto& norm = file_.tensor("model.norm.weight");
    const ModelFile::Tensor* output = c.tie_word_embeddings ? nullptr : &file_.tensor("model.output.weight");
    if (embed.byte_size != V * D * 2 || norm.byte_size != D * 2 ||
        (output && output->byte_size != V * D * 2)) {
        throw std::runtime_error("Invalid embedding, final norm, or output tensor shape");
    }
    // Arena layout: embed | output? | final_norm | per layer: attn_norm q_norm k_norm
    // [wq;wk;wv] wo mlp_norm [w1;w3] w2 - every block 256-byte aligned, wq/wk/wv and w1/w3 back
    // to back.
    struct Piece {
        const ModelFile::Tensor* t;
        size_t expect;
        size_t off;
    };
    std::vector<Piece> pieces;
    size_t off = 0;
    auto place = [&](const ModelFile::Tensor& t, size_t expect_elems, bool pad = true) {
        pieces.push_back({&t, expect_elems, off});
        off += expect_elems * 2;
        if (pad) off = align256(off);
        return pieces.back().off;
    };
    const size_t embed_off = place(embed, V * D);
    const size_t output_off = output ? place(*output, V * D) : embed_off;
    const size_t norm_off = place(norm, D);
    std::vector<std::array<size_t, 10>> loffs(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        const auto& t_an = file_.tensor(p + "attn.norm.weight");
        const auto& t_qn = file_.tensor(p + "attn.q_norm.weight");
        const auto& t_kn = file_.tensor(p + "attn.k_norm.weight");
        const auto& t_wq = file_.tensor(p + "attn.wq.weight");
        const auto& t_wk = file_.tensor(p + "attn.wk.weight");
        const auto& t_wv = file_.tensor(p + "attn.wv.weight");
        const auto& t_wo = file_.tensor(p + "attn.wo.weight");
        const auto& t_mn = file_.tensor(p + "mlp.norm.weight");
        const auto& t_w1 = file_.tensor(p + "mlp.w1.weight");
        const auto& t_w2 = file_.tensor(p + "mlp.w2.weight");
        const auto& t_w3 = file_.tensor(p + "mlp.w3.weight");
        // Block::ValidateWeights (src/inference.cpp:737-764).
        auto require = [](const ModelFile::Tensor& t, size_t expected, const char* name) {
            if (t.byte_size / 2 != expected) {
                throw std::invalid_argument(std::string("Invalid ") + name + " size: expected " +
                                            std::to_string(expected) + ", got " +
                                            std::to_string(t.byte_size / 2));
            }
        };
        require(t_an, D, "attn_norm");
        require(t_qn, hd, "q_norm");
        require(t_kn, hd, "k_norm");
        require(t_wq, qd * D, "wq");
        require(t_wk, kvd * D, "wk");
        require(t_wv, kvd * D, "wv");
        require(t_wo, D * qd, "wo");
        require(t_mn, D, "mlp_norm");
        require(t_w1, H * D, "w1");
        require(t_w2, D * H, "w2");
        require(t_w3, H * D, "w3");
        auto& lo = loffs[l];
        lo[0] = place(t_an, D);
        lo[1] = place(t_qn, hd);
        lo[2] = place(t_kn, hd);
        lo[3] = place(t_wq, qd * D, false);
        place(t_wk, kvd * D, false);
        place(t_wv, kvd * D);
        lo[4] = place(t_wo, D * qd);
        lo[5] = place(t_mn, D);
        lo[6] = place(t_w1, H * D, false);  // w1 and w3 back to back: one [2H, D] operand
        lo[7] = place(t_w3, H * D);
        lo[8] = place(t_w2, D * H);
    }
    arena_.alloc(off);
    // Upload through two pinned staging buffers so file reads overlap the copies.
    {
        const size_t kChunk = 64u << 20;
        PinnedBuffer stage[2];
        stage[0].ensure(kChunk);
        stage[1].ensure(kChunk);
        cudaEvent_t done[2];
        Q3_CUDA(cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming));
        Q3_CUDA(cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming));
        cudaStream_t s;
        Q3_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        int which = 0;
        bool used[2] = {false, false};
        for (const Piece& p : pieces) {
            const uint8_t* src = file_.data() + p.t->offset;
            uint8_t* dst = static_cast<uint8_t*>(arena_.ptr) + p.off;
            size_t left = p.t->byte_size;
            while (left > 0) {
                const size_t n = std::min(left, kChunk);
                if (used[which]) Q3_CUDA(cudaEventSynchronize(done[which]));
                std::memcpy(stage[which].ptr, src, n);
                Q3_CUDA(cudaMemcpyAsync(dst, stage[which].ptr, n, cudaMemcpyHostToDevice, s));
                Q3_CUDA(cudaEventRecord(done[which], s));
                used[which] = true;
                which ^= 1;
                src += n;
                dst += n;
                left -= n;
            }
        }
        Q3_CUDA(cudaStreamSynchronize(s));
        cudaEventDestroy(done[0]);
        cudaEventDestroy(done[1]);
        cudaStreamDestroy(s);
    }
    const uint16_t* base = static_cast<const uint16_t*>(arena_.ptr);
    embed_ = base + embed_off / 2;
    output_ = base + output_off / 2;
    final_norm_ = base + norm_off / 2;
    layers_.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        auto& lo = loffs[l];
        LayerWeights& w = layers_[l];
        w.attn_norm = base + lo[0] / 2;
        w.q_norm = base + lo[1] / 2;
        w.k_norm = base + lo[2] / 2;
        w.wqkv = base + lo[3] / 2;
        w.wo = base + lo[4] / 2;
        w.mlp_norm = base + lo[5] / 2;
        w.w1 = base + lo[6] / 2;
        w.w3 = base + lo[7] / 2;
        w.w2 = base + lo[8] / 2;
    }
    tensor_count_ = static_cast<int>(file_.tensor_count());

    engine_ = std::make_unique<Engine>(cfg_, c.n_layers, device_, ctx);
    // The fused kernel's error word sits right after the logits, so that one copy brings back
    // both (q3_forward_token_ref).
    logits_.alloc(V * 4 + 64);
    Q3_CUDA(cudaMemset(logits_.ptr, 0, logits_.bytes));
    argmax_part_.alloc(static_cast<size_t>(gemv_grid(c.vocab_size)) * sizeof(float2));
    argmax_out_.alloc(16);
    ensure_logs(1024);

    if (fused_supported(cfg_)) {
        fused_grid_ = q3::fused_grid(device_);
        if (fused_grid_ >= 8) {
            fused_s_max_ = fused_grid_ / c.n_kv_heads;
            // The fused kernel's weight copies, per layer: [wq;wk;wv], wo split by KV-head group,
            // w1 and w3 (row-parity swizzled), and w2 transposed; plus the swizzled lm_head.
            const size_t qkv_elems = (qd + 2 * kvd) * D;
            const size_t wo_elems = D * qd;
            const size_t w13_elems = H * D;
            const size_t w2_elems = D * H;
            const size_t per_layer = qkv_elems + wo_elems + 2 * w13_elems + w2_elems;
            fused_wperm_.alloc((per_layer * c.n_layers + V * D) * 2);
            DeviceBuffer tmp;
            tmp.alloc(wo_elems * 2);
            cudaStream_t ls = engine_->stream();
            std::vector<FusedLayer> fl(c.n_layers);
            uint16_t* wp = static_cast<uint16_t*>(fused_wperm_.ptr);
            for (int l = 0; l < c.n_layers; ++l) {
                const LayerWeights& w = layers_[l];
                uint16_t* qkv = wp + per_layer * l;
                uint16_t* wop = qkv + qkv_elems;
                uint16_t* w1 = wop + wo_elems;
                uint16_t* w3 = w1 + w13_elems;
                uint16_t* w2t = w3 + w13_elems;
                launch_swizzle_rows(w.wqkv, qkv, qd + 2 * kvd, static_cast<int>(D), ls);
                launch_permute_wo(w.wo, static_cast<uint16_t*>(tmp.ptr), ls);
                launch_swizzle_rows(static_cast<uint16_t*>(tmp.ptr), wop, c.n_kv_heads * D,
                                    static_cast<int>(wo_elems / (c.n_kv_heads * D)), ls);
                launch_swizzle_rows(w.w1, w1, H, static_cast<int>(D), ls);
                launch_swizzle_rows(w.w3, w3, H, static_cast<int>(D), ls);
                launch_transpose_w2(w.w2, w2t, ls);
                fl[l] = FusedLayer{qkv, wop, w1, w3, w2t, w.attn_norm, w.q_norm, w.k_norm,
                                   w.mlp_norm};
                Q3_CUDA(cudaStreamSynchronize(ls));  // tmp is reused by the next layer
            }
            fused_lm_ = wp + per_layer * c.n_layers;
            launch_swizzle_rows(output_, const_cast<uint16_t*>(fused_lm_), V, static_cast<int>(D), ls);
            Q3_CUDA(cudaStreamSynchronize(ls));
            fused_host_layers_ = fl;
            fused_layers_.alloc(fl.size() * sizeof(FusedLayer));
            Q3_CUDA(cudaMemcpy(fused_layers_.ptr, fl.data(), fl.size() * sizeof(FusedLayer),
                               cudaMemcpyHostToDevice));
            fused_y_.alloc(fused_ybuf_floats(c.n_layers) * 4);
            Q3_CUDA(cudaMemset(fused_y_.ptr, 0, fused_y_.bytes));
            // Tagged q|k|v [4096] and o_proj partials [8][1024]; zero tags never match a launch's.
            fused_tagged_.alloc((static_cast<size_t>(c.n_heads + 2 * c.n_kv_heads) * c.head_dim +
                                 static_cast<size_t>(c.n_kv_heads) * D) * 8);
            Q3_CUDA(cudaMemset(fused_tagged_.ptr, 0, fused_tagged_.bytes));
            fused_part_o_.alloc(static_cast<size_t>(c.n_heads) * fused_s_max_ * c.head_dim * 4);
            fused_part_ml_.alloc(static_cast<size_t>(c.n_heads) * fused_s_max_ * sizeof(float2));
            fused_am_.alloc(static_cast<size_t>(fused_grid_) * sizeof(float2));
            fused_sync_.alloc(256);  // [0] arrival counter
            Q3_CUDA(cudaMemset(fused_sync_.ptr, 0, 256));
            if (getenv("Q3_FUSED_CHECKS")) {
                // Record buffer of the self-checking build (compiled with -DQ3_FUSED_CHECKS).
                fused_dbg_.alloc(8 * sizeof(unsigned long long));
                Q3_CUDA(cudaMemset(fused_dbg_.ptr, 0, fused_dbg_.bytes));
            }
        } else {
            fused_grid_ = 0;
        }
    }
}

void Model::fused_profile(int32_t token, int pos, uint64_t* stamps, size_t cap, int* n_phases,
                          int* grid) {
    if (!fused_available()) throw std::runtime_error("fused decode path is not available");
    check_token_pos(token, pos);
    int ns = 0, kp = 0, kl = 0;
    step_positions(pos, cfg_.max_seq_len, &ns, &kp, &kl);
    const int phases = fused_phases_per_step(cfg_.n_layers, kl) + 1;
    const size_t n = static_cast<size_t>(phases) * fused_grid_ * 8;
    *n_phases = phases;
    *grid = fused_grid_;
    if (cap < n) throw std::invalid_argument("stamp buffer too small");
    Engine& e = *engine_;
    e.ensure_rope(pos + 2);
    e.write_step(start_params(token, pos, 0));
    DeviceBuffer prof;
    prof.alloc(n * 8);
    Q3_CUDA(cudaMemsetAsync(prof.ptr, 0, n * 8, e.stream()));
    clear_fused_error();
    launch_fused(1, false, false, 4000000000LL, 0, static_cast<unsigned long long*>(prof.ptr));
    check_fused_error();
    Q3_CUDA(cudaMemcpyAsync(stamps, prof.ptr, n * 8, cudaMemcpyDeviceToHost, e.stream()));
    Q3_CUDA(cudaStreamSynchronize(e.stream()));
}

void Model::launch_fused(int n_steps, bool forced, bool taps, long long spin_cycles, int offset,
                         unsigned long long* prof, const StepParams* sp_init) {
    Engine& e = *engine_;
    FusedArgs a{};
    a.prof = prof;
    a.dbg = static_cast<unsigned long long*>(fused_dbg_.ptr);
    a.layers = static_cast<const FusedLayer*>(fused_layers_.ptr);
    a.embed = embed_;
    a.lm_head = fused_lm_;
    a.final_norm = final_norm_;
    a.k_cache = e.k_layer(0);
    a.v_cache = e.v_layer(0);
    a.layer_elems = e.layer_elems();
    a.page_table = e.page_table();
    a.rope = e.rope();
    a.rope_len = e.rope_len();
    a.ybuf = static_cast<float*>(fused_y_.ptr);
    // The first step's accumulators were zeroed by the previous launch's last step (or at
    // allocation / after a launch that gave up).
    a.parity0 = fused_parity_;
    fused_parity_ = (fused_parity_ + n_steps) & 1;
    a.qkvt = static_cast<unsigned long long*>(fused_tagged_.ptr);
    a.opart = a.qkvt + static_cast<size_t>(cfg_.n_heads + 2 * cfg_.n_kv_heads) * cfg_.head_dim;
    fused_epoch_ = (fused_epoch_ + 1) & 0xFFFu;
    if (fused_epoch_ == 0) fused_epoch_ = 1;
    a.epoch = fused_epoch_;
    a.part_o = static_cast<float*>(fused_part_o_.ptr);
    a.part_ml = static_cast<float2*>(fused_part_ml_.ptr);
    a.am_part = static_cast<float2*>(fused_am_.ptr);
    a.logits = fused_logits_out_ ? fused_logits_out_ : static_cast<float*>(logits_.ptr);
    a.token_out = fused_token_out_;
    a.err_out = fused_err_out_;
    a.taps = taps ? e.taps() : nullptr;
    a.sp = e.step_params();
    if (sp_init) {
        a.sp_init = *sp_init;
        a.sp_from_args = 1;
    }
    a.token_log = static_cast<int32_t*>(token_log_.ptr);
    a.forced = forced ? static_cast<const int32_t*>(forced_.ptr) : nullptr;
    a.bar = static_cast<unsigned*>(fused_sync_.ptr);
    a.err = fused_err_word();
    a.n_layers = cfg_.n_layers;
    a.vocab = cfg_.vocab_size;
    a.ctx = cfg_.max_seq_len;
    a.n_steps = n_steps;
    a.s_max = fused_s_max_;
    a.eps = cfg_.norm_eps;
    a.spin_cycles = spin_cycles;
    a.barrier_offset = offset;
    a.l2_ahead = fused_l2_ahead();
    // One rank: every KV group, MLP index and lm_head row; o_proj partials into its own buffer.
    a.nkv = cfg_.n_kv_heads;
    a.kv0 = 0;
    a.hl = cfg_.hidden_dim;
    a.v0 = 0;
    a.world = 1;
    a.rank = 0;
    a.opart_dst[0] = a.opart;
    // The arrival counter is zero here: set at allocation, back to zero at the end of every
    // launch that completed (CTA 0), and by reset_fused_state after one that gave up.
    launch_decode_fused(a, fused_grid_, e.stream());
}

void Model::reset_fused_state() {
    cudaStream_t s = engine_->stream();
    Q3_CUDA(cudaStreamSynchronize(s));
    Q3_CUDA(cudaMemsetAsync(fused_sync_.ptr, 0, fused_sync_.bytes, s));
    Q3_CUDA(cudaMemsetAsync(fused_err_word(), 0, sizeof(unsigned), s));
    Q3_CUDA(cudaMemsetAsync(fused_y_.ptr, 0, fused_y_.bytes, s));
    Q3_CUDA(cudaStreamSynchronize(s));
    fused_parity_ = 0;
}

// The error word is zero unless a launch gave up, and check_fused_error zeroes the state again
// when it reports one; only the self-check record (checking builds) is cleared per call.
void Model::clear_fused_error() {
    if (!fused_enabled()) return;
    if (fused_dbg_.ptr) {
        Q3_CUDA(cudaMemsetAsync(fused_dbg_.ptr, 0, fused_dbg_.bytes, engine_->stream()));
    }
}

void Model::check_fused_error() {
    if (!fused_enabled()) return;
    unsigned err = 0;
    unsigned long long dbg[8] = {};
    Q3_CUDA(cudaMemcpyAsync(&err, fused_err_word(), sizeof(unsigned),
                            cudaMemcpyDeviceToHost, engine_->stream()));
    if (fused_dbg_.ptr) {
        Q3_CUDA(cudaMemcpyAsync(dbg, fused_dbg_.ptr, sizeof(dbg), cudaMemcpyDeviceToHost,
                                engine_->stream()));
    }
    Q3_CUDA(cudaStreamSynchronize(engine_->stream()));
    if (dbg[0] || err) reset_fused_state();
    if (dbg[0]) {
        throw std::runtime_error(
            "fused decode kernel self-check " + std::to_string(dbg[0]) + " failed in CTA " +
            std::to_string(dbg[1]) + " thread " + std::to_string(dbg[2]) + " values " +
            std::to_string(static_cast<long long>(dbg[3])) + " " +
            std::to_string(static_cast<long long>(dbg[4])) + " " +
            std::to_string(static_cast<long long>(dbg[5])));
    }
    if (err) {
        throw DeviceTimeout("fused decode kernel: a bounded device-side wait gave up");
    }
}

bool Model::fused_timeout_selftest() {
    if (!fused_available()) throw std::runtime_error("fused decode path is not available");
    Engine& e = *engine_;
    e.ensure_rope(2);
    e.write_step(start_params(0, 0, 0));
    // ~10 ms bound; barrier target one above what the grid can reach.
    launch_fused(1, false, false, 20000000LL, 1);
    unsigned err = 0;
    Q3_CUDA(cudaMemcpyAsync(&err, fused_err_word(), sizeof(unsigned),
                            cudaMemcpyDeviceToHost, e.stream()));
    Q3_CUDA(cudaStreamSynchronize(e.stream()));
    reset_fused_state();  // the launch gave up: counter, error word and accumulators undefined
    return err != 0;
}

Model::~Model() {
    engine_.reset();
}

void Model::ensure_logs(int n) {
    if (n <= log_cap_) return;
    int cap = log_cap_ > 0 ? log_cap_ : 1024;
    while (cap < n + 1) cap *= 2;
    token_log_.alloc(static_cast<size_t>(cap) * 4);
    forced_.alloc(static_cast<size_t>(cap) * 4);
    log_cap_ = cap;
    engine_->drop_graphs();
}

// The whole step: embedding, every layer, final norm, tied lm_head, greedy argmax and the
// device-side advance (ForwardToken, src/inference.cpp:592-637, plus Greedy :703-709).
void Model::enqueue_step(bool forced, bool taps) {
    const q3_config& c = cfg_;
    Engine& e = *engine_;
    cudaStream_t s = e.stream();
    StepParams* sp = e.step_params();
    float* x = e.x();
    launch_embed(sp, embed_, x, c.dim, s);
    if (taps) Q3_CUDA(cudaMemcpyAsync(e.taps(), x, c.dim * 4, cudaMemcpyDeviceToDevice, s));
    for (int l = 0; l < c.n_layers; ++l) {
        e.enqueue_layer(l, layers_[l]);
        if (taps) {
            Q3_CUDA(cudaMemcpyAsync(e.taps() + static_cast<size_t>(l + 1) * c.dim, x, c.dim * 4,
                                    cudaMemcpyDeviceToDevice, s));
        }
    }
    const int grid = gemv_grid(c.vocab_size);
    launch_gemv(kEpiStore, output_, nullptr, x, final_norm_, c.norm_eps,
                static_cast<float*>(logits_.ptr), nullptr, c.vocab_size, c.dim,
                static_cast<float2*>(argmax_part_.ptr), grid, s);
    launch_argmax_final(static_cast<const float2*>(argmax_part_.ptr), grid,
                        static_cast<int32_t*>(argmax_out_.ptr), sp,
                        static_cast<int32_t*>(token_log_.ptr), c.max_seq_len,
                        forced ? static_cast<const int32_t*>(forced_.ptr) : nullptr, s);
}

void Model::run_steps(int n, bool forced, bool taps, float* logits_log_dev,
                      const StepParams* sp_init) {
    Engine& e = *engine_;
    if (fused_enabled()) {
        constexpr long long kSpinCycles = 4000000000LL;  // ~2 s at the B200 boost clock
        if (sp_init) {
            launch_fused(1, forced, taps, kSpinCycles, 0, nullptr, sp_init);
        } else if (logits_log_dev || taps) {
            for (int i = 0; i < n; ++i) {
                launch_fused(1, forced, taps, kSpinCycles, 0);
                if (logits_log_dev) {
                    Q3_CUDA(cudaMemcpyAsync(logits_log_dev + static_cast<size_t>(i) * cfg_.vocab_size,
                                            logits_.ptr, static_cast<size_t>(cfg_.vocab_size) * 4,
                                            cudaMemcpyDeviceToDevice, e.stream()));
                }
            }
        } else {
            constexpr int kMaxStepsPerLaunch = 256;
            for (int done = 0; done < n; done += kMaxStepsPerLaunch) {
                launch_fused(std::min(kMaxStepsPerLaunch, n - done), forced, false, kSpinCycles, 0);
            }
        }
        return;
    }
    const int key = (forced ? 1 : 0) | (taps ? 2 : 0);
    cudaGraphExec_t g = e.graph(key, [&] { enqueue_step(forced, taps); });
    for (int i = 0; i < n; ++i) {
        Q3_CUDA(cudaGraphLaunch(g, e.stream()));
        if (logits_log_dev) {
            Q3_CUDA(cudaMemcpyAsync(logits_log_dev + static_cast<size_t>(i) * cfg_.vocab_size,
                                    logits_.ptr, static_cast<size_t>(cfg_.vocab_size) * 4,
                                    cudaMemcpyDeviceToDevice, e.stream()));
        }
    }
}

StepParams Model::start_params(int32_t token, int pos, int n_forced) const {
    StepParams p{};
    p.token = token;
    p.pos = pos;
    step_positions(pos, cfg_.max_seq_len, &p.num_sink, &p.kv_pos, &p.kv_len);
    p.step = 0;
    p.n_forced = n_forced;
    return p;
}

void Model::check_token_pos(int32_t token, int pos) const {
    // Range checks of ForwardToken (src/inference.cpp:594-599).
    if (token < 0 || token >= cfg_.vocab_size) {
        throw std::out_of_range("Token id is outside the vocabulary");
    }
    if (pos < 0) throw std::out_of_range("Token position must not be negative");
}

unsigned* Model::fused_err_word() const {
    return reinterpret_cast<unsigned*>(static_cast<char*>(logits_.ptr) +
                                       static_cast<size_t>(cfg_.vocab_size) * 4);
}

void Model::forward_token(int32_t token, int pos, float* hidden_host, float* logits_host,
                          bool err_after_logits, int32_t* next_host) {
    check_token_pos(token, pos);
    Engine& e = *engine_;
    e.ensure_rope(pos + 2);
    const StepParams sp = start_params(token, pos, 0);
    clear_fused_error();
    if (fused_enabled()) {
        // The step's parameters travel with the launch (no staging copy, no synchronisation).
        run_steps(1, false, hidden_host != nullptr, nullptr, &sp);
    } else {
        e.write_step(sp);
        run_steps(1, false, hidden_host != nullptr, nullptr);
    }
    cudaStream_t s = e.stream();
    // The error word comes back with the outputs: one synchronisation per call; with
    // err_after_logits it is the word after the logits in logits_host (one copy for both).
    pinned_err_.ensure(sizeof(unsigned));
    unsigned* err_host = static_cast<unsigned*>(pinned_err_.ptr);
    *err_host = 0u;
    if (err_after_logits) {
        err_host = reinterpret_cast<unsigned*>(logits_host + cfg_.vocab_size);
    } else if (fused_enabled()) {
        Q3_CUDA(cudaMemcpyAsync(err_host, fused_err_word(), sizeof(unsigned),
                                cudaMemcpyDeviceToHost, s));
    }
    if (hidden_host) {
        Q3_CUDA(cudaMemcpyAsync(hidden_host, e.taps(),
                                static_cast<size_t>(cfg_.n_layers + 1) * cfg_.dim * 4,
                                cudaMemcpyDeviceToHost, s));
    }
    if (logits_host) {
        Q3_CUDA(cudaMemcpyAsync(logits_host, logits_.ptr,
                                static_cast<size_t>(cfg_.vocab_size) * 4 +
                                    (err_after_logits ? sizeof(unsigned) : 0),
                                cudaMemcpyDeviceToHost, s));
    }
    if (next_host) {
        // The step's greedy token (both decode paths log it at index 0 of a one-step call).
        Q3_CUDA(cudaMemcpyAsync(next_host, token_log_.ptr, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    }
    Q3_CUDA(cudaStreamSynchronize(s));
    if (*err_host != 0u) check_fused_error();  // throws
}

const float* Model::forward_token_ref(int32_t token, int pos, int32_t* next) {
    // [logits][error word][greedy token]
    pinned_logits_.ensure(static_cast<size_t>(cfg_.vocab_size) * 4 + 2 * sizeof(unsigned));
    float* buf = static_cast<float*>(pinned_logits_.ptr);
    unsigned* err_host = reinterpret_cast<unsigned*>(buf + cfg_.vocab_size);
    int32_t* tok = reinterpret_cast<int32_t*>(buf + cfg_.vocab_size + 1);
    if (!fused_enabled()) {
        forward_token(token, pos, nullptr, buf, true, next ? tok : nullptr);
        if (next) *next = *tok;
        return buf;
    }
    // Fused path: the kernel's lm_head phase writes the logits into this pinned buffer (over the
    // host link while the phase runs) and CTA 0 the greedy token; only the error word is copied.
    check_token_pos(token, pos);
    Engine& e = *engine_;
    e.ensure_rope(pos + 2);
    const StepParams sp = start_params(token, pos, 0);
    clear_fused_error();
    void* dev_buf = nullptr;
    Q3_CUDA(cudaHostGetDevicePointer(&dev_buf, buf, 0));
    float* dev_logits = static_cast<float*>(dev_buf);
    // The kernel's CTA 0 overwrites the preset error slot when the launch runs to completion.
    *err_host = ~0u;
    fused_logits_out_ = dev_logits;
    fused_token_out_ = reinterpret_cast<int32_t*>(dev_logits + cfg_.vocab_size + 1);
    fused_err_out_ = reinterpret_cast<unsigned*>(dev_logits + cfg_.vocab_size);
    try {
        run_steps(1, false, false, nullptr, &sp);
    } catch (...) {
        fused_logits_out_ = nullptr;
        fused_token_out_ = nullptr;
        fused_err_out_ = nullptr;
        throw;
    }
    fused_logits_out_ = nullptr;
    fused_token_out_ = nullptr;
    fused_err_out_ = nullptr;
    Q3_CUDA(cudaStreamSynchronize(e.stream()));
    if (*err_host != 0u) {
        check_fused_error();  // throws when the device error word is set
        throw std::runtime_error("fused decode: the launch did not run to completion");
    }
    if (next) *next = *tok;
    return buf;
}

void Model::decode_loop(const int32_t* forced_host, int n, int32_t first_token, int pos0,
                        int32_t* out_tokens_host, float* last_logits_host,
                        float* all_logits_host) {
    if (n <= 0) return;
    if (forced_host) {
        for (int i = 0; i < n; ++i) check_token_pos(forced_host[i], pos0 + i);
    } else {
        check_token_pos(first_token, pos0);
    }
    if (pos0 > std::numeric_limits<int>::max() - n) {
        throw std::out_of_range("Token position must not be negative");
    }
    Engine& e = *engine_;
    ensure_logs(n);
    e.ensure_rope(pos0 + n + 1);
    cudaStream_t s = e.stream();
    if (forced_host) {
        Q3_CUDA(cudaStreamSynchronize(s));
        pinned_io_.ensure(static_cast<size_t>(n) * 4);
        std::memcpy(pinned_io_.ptr, forced_host, static_cast<size_t>(n) * 4);
        Q3_CUDA(cudaMemcpyAsync(forced_.ptr, pinned_io_.ptr, static_cast<size_t>(n) * 4,
                                cudaMemcpyHostToDevice, s));
    }
    e.write_step(start_params(forced_host ? forced_host[0] : first_token, pos0,
                              forced_host ? n : 0));
    DeviceBuffer all;
    if (all_logits_host) all.alloc(static_cast<size_t>(n) * cfg_.vocab_size * 4);
    clear_fused_error();
    run_steps(n, forced_host != nullptr, false, static_cast<float*>(all.ptr));
    check_fused_error();
    if (out_tokens_host) {
        Q3_CUDA(cudaMemcpyAsync(out_tokens_host, token_log_.ptr, static_cast<size_t>(n) * 4,
                                cudaMemcpyDeviceToHost, s));
    }
    if (last_logits_host) {
        Q3_CUDA(cudaMemcpyAsync(last_logits_host, logits_.ptr,
                                static_cast<size_t>(cfg_.vocab_size) * 4, cudaMemcpyDeviceToHost, s));
    }
    if (all_logits_host) {
        Q3_CUDA(cudaMemcpyAsync(all_logits_host, all.ptr, all.bytes, cudaMemcpyDeviceToHost, s));
    }
    Q3_CUDA(cudaStreamSynchronize(s));
}

void Model::set_prefill_precision(int p) {
    if (p != Prefill::kPrecisionBF16 && p != Prefill::kPrecisionF16) {
        throw std::invalid_argument("unknown prefill precision");
    }
    prefill_precision_ = p;
}

const std::vector<LayerWeights>& Model::layers_f16() {
    if (layers16_.empty()) {
        cudaStream_t s = engine_->stream();
        make_f16_layers(cfg_, layers_, f16_arena_, layers16_, s);
        Q3_CUDA(cudaStreamSynchronize(s));
    }
    return layers16_;
}

bool Model::batched_prefill_ok(int n, int pos0) const {
    return use_batched_prefill_ && Prefill::supported(cfg_) && n > 0 && pos0 >= 0 &&
           pos0 <= cfg_.max_seq_len - n;
}

void Model::prefill(const int32_t* ids, int n, int pos0, float* last_logits, int32_t* next,
                    float* hidden_host) {
    if (n <= 0) throw std::invalid_argument("Prefill needs at least one token");
    if (!ids) throw std::invalid_argument("null argument");
    if (batched_prefill_ok(n, pos0)) {
        prefill_batched(ids, n, pos0, last_logits, next, hidden_host);
        return;
    }
    // Token by token: the reference's loop (src/inference.cpp:669-671) driven on the device;
    // the last token runs alone when its per-layer hidden states are wanted.
    const int bulk = hidden_host ? n - 1 : n;
    std::vector<int32_t> argmax(n);
    if (bulk > 0) decode_loop(ids, bulk, 0, pos0, argmax.data(), last_logits, nullptr);
    if (hidden_host) {
        forward_token(ids[n - 1], pos0 + n - 1, hidden_host, nullptr);
        std::vector<float> lg(cfg_.vocab_size);
        Q3_CUDA(cudaMemcpy(lg.data(), logits_.ptr, lg.size() * 4, cudaMemcpyDeviceToHost));
        if (last_logits) std::memcpy(last_logits, lg.data(), lg.size() * 4);
        argmax[n - 1] = static_cast<int32_t>(std::max_element(lg.begin(), lg.end()) - lg.begin());
    }
    if (next) *next = argmax[n - 1];
}

void Model::prefill_batched(const int32_t* ids, int n, int pos0, float* last_logits,
                            int32_t* next, float* hidden_host) {
    for (int i = 0; i < n; ++i) check_token_pos(ids[i], pos0 + i);
    Engine& e = *engine_;
    cudaStream_t s = e.stream();
    e.ensure_rope(pos0 + n + 1);
    if (!prefill_) prefill_ = std::make_unique<Prefill>(cfg_, device_);
    prefill_->set_precision(prefill_precision_);
    const std::vector<LayerWeights>* l16 =
        prefill_precision_ == Prefill::kPrecisionF16 ? &layers_f16() : nullptr;
    if (prefill_ids_.bytes < static_cast<size_t>(n) * 4) {
        Q3_CUDA(cudaStreamSynchronize(s));
        prefill_ids_.alloc(static_cast<size_t>(n) * 4);
    }
    Q3_CUDA(cudaStreamSynchronize(s));
    pinned_io_.ensure(static_cast<size_t>(n) * 4);
    std::memcpy(pinned_io_.ptr, ids, static_cast<size_t>(n) * 4);
    Q3_CUDA(cudaMemcpyAsync(prefill_ids_.ptr, pinned_io_.ptr, static_cast<size_t>(n) * 4,
                            cudaMemcpyHostToDevice, s));
    prefill_->run(static_cast<const int32_t*>(prefill_ids_.ptr), n, pos0, embed_, layers_,
                  engine_view(e), e.x(), hidden_host ? e.taps() : nullptr, s, l16);
    // Final RmsNorm + tied lm_head of the last token (src/inference.cpp:619-635) and Greedy.
    const q3_config& c = cfg_;
    // Greedy over the GEMV's per-block (max, index) partials (two-level, lowest index on ties).
    launch_gemv(kEpiStore, output_, nullptr, e.x(), final_norm_, c.norm_eps,
                static_cast<float*>(logits_.ptr), nullptr, c.vocab_size, c.dim,
                static_cast<float2*>(argmax_part_.ptr), gemv_grid(c.vocab_size), s);
    launch_argmax_final(static_cast<const float2*>(argmax_part_.ptr), gemv_grid(c.vocab_size),
                        static_cast<int32_t*>(argmax_out_.ptr), nullptr, nullptr, 0, nullptr, s);
    int32_t am = 0;
    Q3_CUDA(cudaMemcpyAsync(&am, argmax_out_.ptr, 4, cudaMemcpyDeviceToHost, s));
    if (last_logits) {
        Q3_CUDA(cudaMemcpyAsync(last_logits, logits_.ptr, static_cast<size_t>(c.vocab_size) * 4,
                                cudaMemcpyDeviceToHost, s));
    }
    if (hidden_host) {
        Q3_CUDA(cudaMemcpyAsync(hidden_host, e.taps(),
                                static_cast<size_t>(c.n_layers + 1) * c.dim * 4,
                                cudaMemcpyDeviceToHost, s));
    }
    Q3_CUDA(cudaStreamSynchronize(s));
    const unsigned err = prefill_->read_error(s);
    if (err) {
        throw DeviceTimeout("batched prefill: a tensor-core pipeline wait gave up (code " +
                            std::to_string(err) + ")");
    }
    if (next) *next = am;
}

// Qwen3::Generate on token IDs (src/inference.cpp:639-700). The reference feeds every generated
// token through ForwardToken, including the last one, so max_new tokens cost max_new forwards.
// Without stop_on_eos the decode loop runs on the device in one go; with it, in chunks that are
// scanned for EOS on the host (steps past EOS only touch KV rows that a later call rewrites
// before reading, since each step writes its own row before attending).
void Model::generate(const int32_t* prompt, int n_prompt, size_t max_new, bool stop_on_eos,
                     int32_t* out, size_t* n_out, q3_generation_stats* stats) {
    std::vector<int32_t> ids(prompt, prompt + n_prompt);
    if (ids.empty()) ids.push_back(cfg_.bos_token_id);
    if (max_new > static_cast<size_t>(std::numeric_limits<int>::max() - ids.size())) {
        throw std::invalid_argument("max_new_tokens is too large");
    }
    q3_generation_stats st{};
    st.prompt_tokens = ids.size();
    using clock = std::chrono::steady_clock;
    const auto t0 = clock::now();
    int32_t next = 0;
    prefill(ids.data(), static_cast<int>(ids.size()), 0, nullptr, &next);
    const auto t1 = clock::now();
    size_t produced = 0;
    int pos = static_cast<int>(ids.size());
    const size_t chunk = stop_on_eos ? 16 : (max_new > 0 ? max_new : 1);
    std::vector<int32_t> log;
    while (produced < max_new) {
        if (stop_on_eos && next == cfg_.eos_token_id) {
            st.stopped_on_eos = 1;
            break;
        }
        const int n = static_cast<int>(std::min(chunk, max_new - produced));
        log.assign(n, 0);
        decode_loop(nullptr, n, next, pos, log.data(), nullptr, nullptr);
        // Tokens of this chunk: next, then log[0..n-2]; log[n-1] is the next chunk's first.
        bool eos = false;
        for (int i = 0; i < n; ++i) {
            const int32_t t = i == 0 ? next : log[i - 1];
            if (stop_on_eos && t == cfg_.eos_token_id) {
                eos = true;
                break;
            }
            out[produced++] = t;
        }
        if (eos) {
            st.stopped_on_eos = 1;
            break;
        }
        next = log[n - 1];
        pos += n;
    }
    const auto t2 = clock::now();
    st.generated_tokens = produced;
    st.reached_token_limit = !st.stopped_on_eos && produced == max_new;
    st.prefill_seconds = std::chrono::duration<double>(t1 - t0).count();
    st.decode_seconds = std::chrono::duration<double>(t2 - t1).count();
    if (n_out) *n_out = produced;
    if (stats) *stats = st;
}

void Model::reset() {
    engine_->reset_cache();
}

void Model::kv_row(int layer, int kv_pos, uint16_t* k, uint16_t* v) {
    if (layer < 0 || layer >= cfg_.n_layers || kv_pos < 0 || kv_pos >= cfg_.max_seq_len) {
        throw std::out_of_range("KV row is outside the cache");
    }
    engine_->read_kv_row(layer, kv_pos, k, v);
}

// ------------------------------------------------------------------ block

Block::Block(const q3_config& cfg, const uint16_t* const* w, const size_t* counts, int device)
    : cfg_(cfg) {
    validate_config(cfg_);
    validate_kernel_limits(cfg_);
    const size_t D = cfg.dim, H = cfg.hidden_dim, hd = cfg.head_dim;
    const size_t qd = static_cast<size_t>(cfg.n_heads) * hd, kvd = static_cast<size_t>(cfg.n_kv_heads) * hd;
    const size_t sizes[11] = {D, hd, hd, qd * D, kvd * D, kvd * D, D * qd, D, H * D, D * H, H * D};
    const char* names[11] = {"attn_norm", "q_norm", "k_norm", "wq", "wk", "wv",
                             "wo", "mlp_norm", "w1", "w2", "w3"};
    if (counts) {
        for (int i = 0; i < 11; ++i) {
            if (counts[i] != sizes[i]) {
                throw std::invalid_argument(std::string("Invalid ") + names[i] +
                                            " size: expected " + std::to_string(sizes[i]) +
                                            ", got " + std::to_string(counts[i]));
            }
        }
    }
    for (int i = 0; i < 11; ++i) {
        if (!w[i] && sizes[i]) throw std::invalid_argument("Block weight pointer must not be null");
    }
    Q3_CUDA(cudaSetDevice(device));
    // Same arena order as a model layer: norms | [wq;wk;wv] | wo | mlp_norm | w1 | w3 | w2.
    const int order[11] = {0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 9};
    size_t offs[11];
    size_t off = 0;
    for (int j = 0; j < 11; ++j) {
        const int i = order[j];
        offs[i] = off;
        off += sizes[i] * 2;
        const bool stack = (i == 3 || i == 4);  // keep wq|wk|wv contiguous
        if (!stack) off = align256(off);
    }
    arena_.alloc(off);
    for (int i = 0; i < 11; ++i) {
        Q3_CUDA(cudaMemcpy(static_cast<uint8_t*>(arena_.ptr) + offs[i], w[i], sizes[i] * 2,
                           cudaMemcpyHostToDevice));
    }
    const uint16_t* base = static_cast<const uint16_t*>(arena_.ptr);
    lw_.attn_norm = base + offs[0] / 2;
    lw_.q_norm = base + offs[1] / 2;
    lw_.k_norm = base + offs[2] / 2;
    lw_.wqkv = base + offs[3] / 2;
    lw_.wo = base + offs[6] / 2;
    lw_.mlp_norm = base + offs[7] / 2;
    lw_.w1 = base + offs[8] / 2;
    lw_.w2 = base + offs[9] / 2;
    lw_.w3 = base + offs[10] / 2;
    engine_ = std::make_unique<Engine>(cfg_, 1, device, cfg.max_seq_len);
}

Block::~Block() { engine_.reset(); }

void Block::forward(float* x_host, int pos, int num_sink, int kv_pos, int kv_len) {
    if (!x_host) throw std::invalid_argument("Block input must not be null");
    const q3_config& c = cfg_;
    // Range checks of Block::forward (src/inference.cpp:786-790).
    if (pos < 0 || kv_len <= 0 || kv_len > c.max_seq_len || kv_pos < 0 || kv_pos >= kv_len ||
        num_sink < 0 || num_sink > kv_len || num_sink >= c.max_seq_len || kv_pos < num_sink) {
        throw std::out_of_range("Invalid position or KV-cache range");
    }
    Engine& e = *engine_;
    e.ensure_rope(pos + 2);
    StepParams p{};
    p.pos = pos;
    p.num_sink = num_sink;
    p.kv_pos = kv_pos;
    p.kv_len = kv_len;
    e.write_step(p);
    cudaStream_t s = e.stream();
    Q3_CUDA(cudaMemcpyAsync(e.x(), x_host, c.dim * 4, cudaMemcpyHostToDevice, s));
    e.enqueue_layer(0, lw_);
    Q3_CUDA(cudaMemcpyAsync(x_host, e.x(), c.dim * 4, cudaMemcpyDeviceToHost, s));
    Q3_CUDA(cudaStreamSynchronize(s));
}

}  // namespace q3

// ==================================================================== C ABI

using q3::guard;

struct q3_model {
    std::unique_ptr<q3::Model> m;
};
struct q3_batch {
    std::unique_ptr<q3::Batch> b;
};

struct q3_tp {
    std::unique_ptr<q3::TpDecoder> t;
};

struct q3_block {
    std::unique_ptr<q3::Block> b;
};

extern "C" {

const char* q3_last_error(void) { return q3::g_last_error.c_str(); }
const char* q3_version(void) { return "q3_b200 0.1 (sm_100a)"; }

q3_status q3_model_load(const char* path, int context_length, int device, q3_model** out) {
    return guard([&] {
        if (!path || !out) throw std::invalid_argument("null argument");
        auto h = std::make_unique<q3_model>();
        h->m = std::make_unique<q3::Model>(path, context_length, device);
        *out = h.release();
    });
}

void q3_model_free(q3_model* model) { delete model; }

q3_status q3_model_config(const q3_model* model, q3_config* out) {
    return guard([&] {
        if (!model || !out) throw std::invalid_argument("null argument");
        *out = model->m->config();
    });
}

q3_status q3_model_tensor_count(const q3_model* model, int* out) {
    return guard([&] {
        if (!model || !out) throw std::invalid_argument("null argument");
        *out = model->m->tensor_count();
    });
}

q3_status q3_model_metadata(const q3_model* model, const char* key, char* buf, size_t capacity,
                            size_t* length) {
    return guard([&] {
        if (!model || !key) throw std::invalid_argument("null argument");
        const std::string& v = model->m->file().metadata(key);
        if (length) *length = v.size();
        if (buf) {
            if (capacity <= v.size()) throw std::invalid_argument("metadata buffer too small");
            std::memcpy(buf, v.c_str(), v.size() + 1);
        }
    });
}

q3_status q3_model_tensor_name(const q3_model* model, int index, char* buf, size_t capacity,
                               size_t* length) {
    return guard([&] {
        if (!model) throw std::invalid_argument("null argument");
        if (index < 0 || static_cast<size_t>(index) >= model->m->file().tensor_count()) {
            throw std::out_of_range("tensor index out of range");
        }
        const std::string& v = model->m->file().tensor_name(static_cast<size_t>(index));
        if (length) *length = v.size();
        if (buf) {
            if (capacity <= v.size()) throw std::invalid_argument("name buffer too small");
            std::memcpy(buf, v.c_str(), v.size() + 1);
        }
    });
}

q3_status q3_model_tensor_info(const q3_model* model, const char* name, q3_tensor_info* out) {
    return guard([&] {
        if (!model || !name || !out) throw std::invalid_argument("null argument");
        const auto& t = model->m->file().tensor(name);
        if (t.shape.size() > 8) throw std::runtime_error("Tensor rank above 8: " + t.name);
        *out = q3_tensor_info{};
        out->dtype = t.dtype;
        out->rank = static_cast<uint32_t>(t.shape.size());
        for (size_t i = 0; i < t.shape.size(); ++i) out->shape[i] = t.shape[i];
        out->data_offset = t.offset;
        out->byte_size = t.byte_size;
    });
}

q3_status q3_model_load_tensor(const q3_model* model, const char* name, uint32_t expected_dtype,
                               void* host, size_t capacity) {
    return guard([&] {
        if (!model || !name) throw std::invalid_argument("null argument");
        const auto& t = model->m->file().tensor(name);
        // LoadTensorBytes (src/inference.cpp:307-317).
        if (t.dtype != expected_dtype) throw std::runtime_error("Tensor dtype mismatch: " + t.name);
        if (t.byte_size > 0) {
            if (!host || capacity < t.byte_size) {
                throw std::invalid_argument("tensor buffer too small: " + t.name);
            }
            std::memcpy(host, model->m->file().data() + t.offset, t.byte_size);
        }
    });
}

q3_status q3_reset(q3_model* model) {
    return guard([&] {
        if (!model) throw std::invalid_argument("null argument");
        model->m->reset();
    });
}

q3_status q3_forward_token(q3_model* model, int32_t token, int pos, float* logits_host) {
    return guard([&] {
        if (!model) throw std::invalid_argument("null argument");
        model->m->forward_token(token, pos, nullptr, logits_host);
    });
}

q3_status q3_forward_token_ref(q3_model* model, int32_t token, int pos, const float** logits) {
    return guard([&] {
        if (!model || !logits) throw std::invalid_argument("null argument");
        *logits = model->m->forward_token_ref(token, pos);
    });
}

q3_status q3_forward_token_greedy(q3_model* model, int32_t token, int pos, const float** logits,
                                  int32_t* next_token) {
    return guard([&] {
        if (!model || !logits || !next_token) throw std::invalid_argument("null argument");
        *logits = model->m->forward_token_ref(token, pos, next_token);
    });
}

q3_status q3_forward_token_layers(q3_model* model, int32_t token, int pos, float* hidden_host,
                                  float* logits_host) {
    return guard([&] {
        if (!model) throw std::invalid_argument("null argument");
        model->m->forward_token(token, pos, hidden_host, logits_host);
    });
}

q3_status q3_kv_row(q3_model* model, int layer, int kv_pos, uint16_t* k_host, uint16_t* v_host) {
    return guard([&] {
        if (!model || !k_host || !v_host) throw std::invalid_argument("null argument");
        model->m->kv_row(layer, kv_pos, k_host, v_host);
    });
}

q3_status q3_prefill(q3_model* model, const int32_t* ids_host, int n, int pos0,
                     float* last_logits_host, int32_t* next_token_host) {
    return guard([&] {
        if (!model || !ids_host) throw std::invalid_argument("null argument");
        model->m->prefill(ids_host, n, pos0, last_logits_host, next_token_host);
    });
}

q3_status q3_prefill_layers(q3_model* model, const int32_t* ids_host, int n, int pos0,
                            float* hidden_host, float* last_logits_host, int32_t* next_token_host) {
    return guard([&] {
        if (!model || !ids_host) throw std::invalid_argument("null argument");
        model->m->prefill(ids_host, n, pos0, last_logits_host, next_token_host, hidden_host);
    });
}

q3_status q3_model_set_prefill_path(q3_model* model, int path) {
    return guard([&] {
        if (!model) throw std::invalid_argument("null argument");
        if (path != Q3_PREFILL_TOKENWISE && path != Q3_PREFILL_BATCHED) {
            throw std::invalid_argument("unknown prefill path");
        }
        model->m->set_batched_prefill(path == Q3_PREFILL_BATCHED);
    });
}

q3_status q3_model_prefill_path(const q3_model* model, int* path) {
    return guard([&] {
        if (!model || !path) throw std::invalid_argument("null argument");
        *path = model->m->batched_prefill_enabled() && q3::Prefill::supported(model->m->config())
                    ? Q3_PREFILL_BATCHED
                    : Q3_PREFILL_TOKENWISE;
    });
}

q3_status q3_model_set_prefill_precision(q3_model* model, int precision) {
    return guard([&] {
        if (!model) throw std::invalid_argument("null argument");
        if (precision != Q3_PREFILL_BF16 && precision != Q3_PREFILL_F16) {
            throw std::invalid_argument("unknown prefill precision");
        }
        model->m->set_prefill_precision(precision == Q3_PREFILL_F16 ? q3::Prefill::kPrecisionF16
                                                                    : q3::Prefill::kPrecisionBF16);
    });
}

q3_status q3_model_prefill_precision(const q3_model* model, int* precision) {
    return guard([&] {
        if (!model || !precision) throw std::invalid_argument("null argument");
        *precision = model->m->prefill_precision() == q3::Prefill::kPrecisionF16 ? Q3_PREFILL_F16
                                                                                 : Q3_PREFILL_BF16;
    });
}

q3_status q3_decode_greedy(q3_model* model, int32_t first_token, int pos0, int n_steps,
                           int32_t* tokens_host, float* last_logits_host) {
    return guard([&] {
        if (!model) throw std::invalid_argument("null argument");
        if (n_steps < 0) throw std::invalid_argument("n_steps must not be negative");
        model->m->decode_loop(nullptr, n_steps, first_token, pos0, tokens_host, last_logits_host,
                              nullptr);
    });
}

q3_status q3_decode_forced(q3_model* model, const int32_t* tokens_host, int n, int pos0,
                           int32_t* argmax_host, float* logits_host) {
    return guard([&] {
        if (!model || (!tokens_host && n > 0)) throw std::invalid_argument("null argument");
        model->m->decode_loop(tokens_host, n, 0, pos0, argmax_host, nullptr, logits_host);
    });
}

q3_status q3_generate(q3_model* model, const int32_t* prompt_host, int n_prompt,
                      size_t max_new_tokens, int stop_on_eos, int32_t* out_tokens_host,
                      size_t* n_out, q3_generation_stats* stats) {
    return guard([&] {
        if (!model || (n_prompt > 0 && !prompt_host) || (max_new_tokens > 0 && !out_tokens_host)) {
            throw std::invalid_argument("null argument");
        }
        if (n_prompt < 0) throw std::invalid_argument("n_prompt must not be negative");
        model->m->generate(prompt_host, n_prompt, max_new_tokens, stop_on_eos != 0,
                           out_tokens_host, n_out, stats);
    });
}

q3_status q3_model_stream(q3_model* model, void** stream) {
    return guard([&] {
        if (!model || !stream) throw std::invalid_argument("null argument");
        *stream = model->m->stream();
    });
}

q3_status q3_model_set_decode_path(q3_model* model, int path) {
    return guard([&] {
        if (!model) throw std::invalid_argument("null argument");
        if (path != Q3_PATH_LAYERWISE && path != Q3_PATH_FUSED) {
            throw std::invalid_argument("unknown decode path");
        }
        if (path == Q3_PATH_FUSED && !model->m->fused_available()) {
            throw std::invalid_argument("the fused decode kernel does not serve this model");
        }
        model->m->set_fused(path == Q3_PATH_FUSED);
    });
}

q3_status q3_model_decode_path(const q3_model* model, int* path) {
    return guard([&] {
        if (!model || !path) throw std::invalid_argument("null argument");
        *path = model->m->fused_enabled() ? Q3_PATH_FUSED : Q3_PATH_LAYERWISE;
    });
}

q3_status q3_model_fused_profile(q3_model* model, int32_t token, int pos, uint64_t* stamps_host,
                                 size_t capacity, int* n_phases, int* grid) {
    return guard([&] {
        if (!model || !stamps_host || !n_phases || !grid) throw std::invalid_argument("null argument");
        model->m->fused_profile(token, pos, stamps_host, capacity, n_phases, grid);
    });
}

q3_status q3_model_fused_timeout_selftest(q3_model* model, int* timed_out) {
    return guard([&] {
        if (!model || !timed_out) throw std::invalid_argument("null argument");
        *timed_out = model->m->fused_timeout_selftest() ? 1 : 0;
    });
}

q3_status q3_batch_create(q3_model* model, int max_seqs, int max_tokens, q3_batch** out) {
    return guard([&] {
        if (!model || !out) throw std::invalid_argument("null argument");
        auto h = std::make_unique<q3_batch>();
        h->b = std::make_unique<q3::Batch>(*model->m, max_seqs, max_tokens);
        *out = h.release();
    });
}

void q3_batch_free(q3_batch* batch) { delete batch; }

q3_status q3_batch_add(q3_batch* batch, const int32_t* ids_host, int n, int* slot,
                       int32_t* next_token_host, float* last_logits_host) {
    return guard([&] {
        if (!batch) throw std::invalid_argument("null argument");
        const int s = batch->b->add(ids_host, n, next_token_host, last_logits_host);
        if (slot) *slot = s;
    });
}

q3_status q3_batch_add_many(q3_batch* batch, const int32_t* ids_host, const int* lens_host,
                            int n_seqs, int* first_slot, int32_t* next_tokens_host,
                            float* last_logits_host) {
    return guard([&] {
        if (!batch || !ids_host || !lens_host) throw std::invalid_argument("null argument");
        const int s = batch->b->add_many(ids_host, lens_host, n_seqs, next_tokens_host,
                                         last_logits_host);
        if (first_slot) *first_slot = s;
    });
}

q3_status q3_batch_size(const q3_batch* batch, int* n_seqs) {
    return guard([&] {
        if (!batch || !n_seqs) throw std::invalid_argument("null argument");
        *n_seqs = batch->b->size();
    });
}

q3_status q3_batch_stream(q3_batch* batch, void** stream) {
    return guard([&] {
        if (!batch || !stream) throw std::invalid_argument("null argument");
        *stream = batch->b->stream();
    });
}

q3_status q3_batch_decode(q3_batch* batch, int n_steps, int32_t* tokens_host) {
    return guard([&] {
        if (!batch) throw std::invalid_argument("null argument");
        batch->b->decode(n_steps, tokens_host);
    });
}

q3_status q3_batch_decode_forced(q3_batch* batch, const int32_t* tokens_host, int n_steps,
                                 int32_t* argmax_host, float* logits_host) {
    return guard([&] {
        if (!batch) throw std::invalid_argument("null argument");
        batch->b->decode_forced(tokens_host, n_steps, argmax_host, logits_host);
    });
}

q3_status q3_batch_kv_row(q3_batch* batch, int slot, int layer, int pos, uint16_t* k_host,
                          uint16_t* v_host) {
    return guard([&] {
        if (!batch) throw std::invalid_argument("null argument");
        batch->b->kv_row(slot, layer, pos, k_host, v_host);
    });
}

q3_status q3_tp_create(q3_model* model, int rank, int world, q3_tp** out) {
    return guard([&] {
        if (!model || !out) throw std::invalid_argument("null argument");
        auto h = std::make_unique<q3_tp>();
        h->t = std::make_unique<q3::TpDecoder>(*model->m, rank, world);
        *out = h.release();
    });
}

void q3_tp_free(q3_tp* tp) { delete tp; }

q3_status q3_tp_ipc_handle(q3_tp* tp, void* handle_host) {
    return guard([&] {
        if (!tp || !handle_host) throw std::invalid_argument("null argument");
        tp->t->ipc_handle(handle_host);
    });
}

q3_status q3_tp_connect(q3_tp* tp, const void* handles_host) {
    return guard([&] {
        if (!tp || !handles_host) throw std::invalid_argument("null argument");
        tp->t->connect(handles_host);
    });
}

q3_status q3_tp_stream(q3_tp* tp, void** stream) {
    return guard([&] {
        if (!tp || !stream) throw std::invalid_argument("null argument");
        *stream = tp->t->stream();
    });
}

q3_status q3_tp_decode(q3_tp* tp, int32_t first_token, int pos0, int n_steps,
                       int32_t* tokens_host) {
    return guard([&] {
        if (!tp) throw std::invalid_argument("null argument");
        tp->t->decode(first_token, pos0, n_steps, nullptr, tokens_host);
    });
}

q3_status q3_tp_decode_forced(q3_tp* tp, const int32_t* tokens_host, int n, int pos0,
                              int32_t* argmax_host) {
    return guard([&] {
        if (!tp || !tokens_host) throw std::invalid_argument("null argument");
        tp->t->decode(0, pos0, n, tokens_host, argmax_host);
    });
}

q3_status q3_tp_configure(q3_tp* tp, int solo_allreduce, long long wait_cycles) {
    return guard([&] {
        if (!tp) throw std::invalid_argument("null argument");
        tp->t->configure(solo_allreduce != 0, wait_cycles);
    });
}

q3_status q3_tp_reset(q3_tp* tp) {
    return guard([&] {
        if (!tp) throw std::invalid_argument("null argument");
        tp->t->reset();
    });
}

q3_status q3_tp_set_path(q3_tp* tp, int path) {
    return guard([&] {
        if (!tp) throw std::invalid_argument("null argument");
        tp->t->set_path(path);
    });
}

q3_status q3_tp_path(q3_tp* tp, int* path) {
    return guard([&] {
        if (!tp || !path) throw std::invalid_argument("null argument");
        *path = tp->t->path();
    });
}

q3_status q3_tp_nccl_unique_id(void* id_host) {
    return guard([&] {
        if (!id_host) throw std::invalid_argument("null argument");
        q3::TpDecoder::nccl_unique_id(id_host);
    });
}

q3_status q3_tp_nccl_connect(q3_tp* tp, const void* id_host) {
    return guard([&] {
        if (!tp || !id_host) throw std::invalid_argument("null argument");
        tp->t->nccl_connect(id_host);
    });
}

q3_status q3_block_create(const q3_config* cfg, const uint16_t* const* weights_host,
                          const size_t* counts, int device, q3_block** out) {
    return guard([&] {
        if (!cfg || !weights_host || !out) throw std::invalid_argument("null argument");
        auto h = std::make_unique<q3_block>();
        h->b = std::make_unique<q3::Block>(*cfg, weights_host, counts, device);
        *out = h.release();
    });
}

void q3_block_free(q3_block* block) { delete block; }

q3_status q3_block_forward(q3_block* block, float* x_host, int pos, int num_sink, int kv_pos,
                           int kv_len) {
    return guard([&] {
        if (!block) throw std::invalid_argument("null argument");
        block->b->forward(x_host, pos, num_sink, kv_pos, kv_len);
    });
}

q3_status q3_block_reset_cache(q3_block* block) {
    return guard([&] {
        if (!block) throw std::invalid_argument("null argument");
        block->b->engine().reset_cache();
    });
}

q3_status q3_block_get_cache(q3_block* block, uint16_t* k_host, uint16_t* v_host) {
    return guard([&] {
        if (!block || !k_host || !v_host) throw std::invalid_argument("null argument");
        block->b->engine().read_cache(0, k_host, v_host, block->b->config().max_seq_len);
    });
}

q3_status q3_block_set_cache(q3_block* block, const uint16_t* k_host, const uint16_t* v_host) {
    return guard([&] {
        if (!block || !k_host || !v_host) throw std::invalid_argument("null argument");
        block->b->engine().write_cache(0, k_host, v_host, block->b->config().max_seq_len);
    });
}

// ------------------------------------------------------------------ free kernels

q3_status q3_rmsnorm(float* out, const float* x, const uint16_t* w, float eps, int n,
                     void* stream) {
    return guard([&] {
        if (!out || !x || !w || n <= 0) throw std::invalid_argument("invalid RmsNorm arguments");
        q3::launch_rmsnorm(out, x, w, eps, n, static_cast<cudaStream_t>(stream));
    });
}

q3_status q3_softmax(float* out, const float* x, int n, void* stream) {
    return guard([&] {
        if (!out || !x || n <= 0) throw std::invalid_argument("invalid Softmax arguments");
        q3::launch_softmax(out, x, n, static_cast<cudaStream_t>(stream));
    });
}

q3_status q3_matmul(float* out, const float* x, const uint16_t* w, int n, int m, void* stream) {
    return guard([&] {
        if (!out || !x || !w || n <= 0 || m <= 0) throw std::invalid_argument("invalid MatMul arguments");
        q3::launch_gemv(q3::kEpiStore, w, nullptr, x, nullptr, 0.0f, out, nullptr, n, m, nullptr,
                        0, static_cast<cudaStream_t>(stream));
    });
}

q3_status q3_rope(float* x, int d, int head_dim, int pos, float theta, int rotary_dim,
                  void* stream) {
    return guard([&] {
        if (!x || d <= 0 || head_dim <= 0 || d % head_dim != 0 || rotary_dim < 0 ||
            rotary_dim % 2 != 0 || rotary_dim > head_dim || rotary_dim > 512) {
            throw std::invalid_argument("invalid ApplyRotaryEmb arguments");
        }
        q3::RopeRow row{};
        const int half = rotary_dim / 2;
        for (int i = 0; i < half; ++i) {
            const float freq = 1.0f / powf(theta, 2.0f * i / rotary_dim);
            const float angle = pos * freq;
            row.c[i] = cosf(angle);
            row.s[i] = sinf(angle);
        }
        q3::launch_rope_row(x, d, head_dim, rotary_dim, row, static_cast<cudaStream_t>(stream));
    });
}

q3_status q3_ffn(float* out, float* lin1, float* lin2, const float* x, const uint16_t* w1,
                 const uint16_t* w2, const uint16_t* w3, int hidden_dim, int dim, void* stream) {
    return guard([&] {
        if (!out || !lin1 || !x || !w1 || !w2 || !w3 || hidden_dim <= 0 || dim <= 0) {
            throw std::invalid_argument("invalid FeedForwardNetwork arguments");
        }
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        q3::launch_gemv(q3::kEpiSiluMul, w1, w3, x, nullptr, 0.0f, lin1, lin2, hidden_dim, dim,
                        nullptr, 0, s);
        q3::launch_gemv(q3::kEpiStore, w2, nullptr, lin1, nullptr, 0.0f, out, nullptr, dim,
                        hidden_dim, nullptr, 0, s);
    });
}

size_t q3_attn_workspace_size(int head_dim, int kv_len) {
    if (head_dim <= 0 || kv_len <= 0) return 0;
    const size_t S = static_cast<size_t>(q3::attn_splits_for(kv_len));
    return S * head_dim * 4 + 256 + S * sizeof(float2);
}

q3_status q3_attn(float* out, void* workspace, const float* q, const uint16_t* k,
                  const uint16_t* v, int head_dim, int n_kv_heads, int kv_len, void* stream) {
    return guard([&] {
        if (!out || !workspace || !q || !k || !v || head_dim <= 0 || head_dim > 256 ||
            n_kv_heads <= 0 || kv_len <= 0) {
            throw std::invalid_argument("invalid FastAttn arguments");
        }
        const int S = q3::attn_splits_for(kv_len);
        q3::AttnArgs a{};
        a.q = q;
        a.k = k;
        a.v = v;
        a.page_table = nullptr;
        a.sp = nullptr;
        a.kv_len_const = kv_len;
        a.n_heads = 1;
        a.n_kv = 1;
        a.hd = head_dim;
        a.row_stride = n_kv_heads * head_dim;
        a.n_splits = S;
        a.part_o = static_cast<float*>(workspace);
        const size_t o_bytes = (static_cast<size_t>(S) * head_dim * 4 + 255) & ~size_t(255);
        a.part_ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) + o_bytes);
        a.out = out;
        q3::launch_attention(a, static_cast<cudaStream_t>(stream));
    });
}

q3_status q3_greedy(const float* logits, int n, int32_t* out_index, void* stream) {
    return guard([&] {
        if (n <= 0) throw std::invalid_argument("Cannot sample empty logits");
        if (!logits || !out_index) throw std::invalid_argument("null argument");
        q3::launch_argmax_full(logits, n, out_index, static_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
