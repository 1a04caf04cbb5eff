// Batched decode of independent sequences (see q3_batch.cuh).
//
// One decode step for B sequences, all on the GPU and captured as one CUDA graph:
//   embedding rows of the B current tokens + RmsNorm -> bf16 operand
//   per layer: [wq;wk;wv] contraction (M = B, split K, reduce-added into a zeroed buffer),
//              per-row QK-norm + RoPE + K/V write at each sequence's own position and pages,
//              tcgen05 attention per (sequence, KV head) over that sequence's pages,
//              x += wo . attn, RmsNorm, [w1;w3] contraction, SiLU(gate) * up, x += w2 . h
//   final RmsNorm, tied lm_head contraction for all B rows, per-row argmax (lowest index on
//   ties), and the device-side advance: token = argmax (or the forced token), position + 1.
#include <cuda_bf16.h>
#include <float.h>

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

#include "q3_batch.cuh"
#include "q3_decode_attn.cuh"
#include "q3_gemm.cuh"
#include "q3_kernels.cuh"

namespace q3 {

namespace {

constexpr int HD = 128;

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// h[r][i] = silu(gu[r][i]) * gu[r][H + i] (src/inference.cpp:948-950, :1009-1011) as a bf16
// hi + lo pair.
__global__ void swiglu_rows_kernel(const float* __restrict__ gu, uint16_t* __restrict__ h,
                                   uint16_t* __restrict__ h_lo, int rows, int H) {
    pdl_wait();
    pdl_trigger();
    const size_t n = static_cast<size_t>(rows) * H / 4;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = (i * 4) / H, c = (i * 4) % H;
        const float4 g = *reinterpret_cast<const float4*>(gu + r * 2 * H + c);
        const float4 u = *reinterpret_cast<const float4*>(gu + r * 2 * H + H + c);
        const float a = g.x / (1.0f + expf(-g.x)) * u.x, b = g.y / (1.0f + expf(-g.y)) * u.y;
        const float cc = g.z / (1.0f + expf(-g.z)) * u.z, d = g.w / (1.0f + expf(-g.w)) * u.w;
        const uint2 hi = make_uint2(pack2(a, b), pack2(cc, d));
        *reinterpret_cast<uint2*>(h + r * H + c) = hi;
        *reinterpret_cast<uint2*>(h_lo + r * H + c) =
            make_uint2(pack2(a - __uint_as_float(hi.x << 16), b - __uint_as_float(hi.x & 0xffff0000u)),
                       pack2(cc - __uint_as_float(hi.y << 16), d - __uint_as_float(hi.y & 0xffff0000u)));
    }
}

// Row b: greedy argmax of logits[b] (lowest index wins ties, src/inference.cpp:703-709), logged
// at log[step][b]; the sequence then feeds the argmax (or the forced token of the next step) at
// position + 1. state = {step, n_forced}.
__global__ void __launch_bounds__(1024) batch_argmax_kernel(const float* __restrict__ logits,
                                                            int rows, int V, int32_t* tok,
                                                            int32_t* pos, int32_t* log,
                                                            const int32_t* state,
                                                            const int32_t* forced) {
    pdl_wait();
    pdl_trigger();
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int b = blockIdx.x;
    const float* row = logits + static_cast<size_t>(b) * V;
    float best = -INFINITY;
    int idx = INT_MAX;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = row[i];
        if (v > best || (v == best && i < idx)) {
            best = v;
            idx = i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) {
            best = ov;
            idx = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        bv[threadIdx.x >> 5] = best;
        bi[threadIdx.x >> 5] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x) / 32; ++w) {
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
                best = bv[w];
                idx = bi[w];
            }
        }
        const int step = state[0], n_forced = state[1];
        log[static_cast<size_t>(step) * rows + b] = idx;
        tok[b] = (forced && step + 1 < n_forced) ? forced[static_cast<size_t>(step + 1) * rows + b]
                                                 : idx;
        pos[b] += 1;
    }
}

__global__ void advance_step_kernel(int32_t* state) {
    pdl_wait();
    pdl_trigger();
    state[0] += 1;
}

}  // namespace

Batch::Batch(Model& model, int max_seqs, int max_tokens)
    : m_(model), cfg_(model.config()), max_seqs_(max_seqs), max_tokens_(max_tokens) {
    const q3_config& c = cfg_;
    if (!Prefill::supported(c)) {
        throw std::invalid_argument("batched decode needs the Qwen3 attention shape (head_dim 128, 2 query heads per KV head)");
    }
    if (max_seqs <= 0 || max_tokens <= 0) throw std::invalid_argument("batch sizes must be positive");
    Q3_CUDA(cudaSetDevice(model.device()));
    Q3_CUDA(cudaStreamCreateWithFlags(&s_, cudaStreamNonBlocking));
    pps_ = (max_tokens + kPageTokens - 1) / kPageTokens;
    pool_pages_ = max_seqs * pps_;
    const size_t layer_elems = static_cast<size_t>(pool_pages_) * c.n_kv_heads * kPageTokens * HD;
    k_.alloc(layer_elems * c.n_layers * 2);
    v_.alloc(layer_elems * c.n_layers * 2);
    Q3_CUDA(cudaMemsetAsync(k_.ptr, 0, k_.bytes, s_));
    Q3_CUDA(cudaMemsetAsync(v_.ptr, 0, v_.bytes, s_));
    std::vector<int32_t> table(static_cast<size_t>(pool_pages_));
    for (int i = 0; i < pool_pages_; ++i) table[i] = i;  // slot s owns pages [s*pps, (s+1)*pps)
    table_.alloc(table.size() * 4);
    Q3_CUDA(cudaMemcpy(table_.ptr, table.data(), table.size() * 4, cudaMemcpyHostToDevice));
    table_host_ = table;
    rope_len_ = max_tokens + 1;
    const auto rt = rope_table_host(c.rope_theta, c.rotary_dim, rope_len_);
    rope_.alloc(rt.size() * sizeof(float2));
    Q3_CUDA(cudaMemcpy(rope_.ptr, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice));
    pos_.alloc(static_cast<size_t>(max_seqs) * 4);
    tok_.alloc(static_cast<size_t>(max_seqs) * 4);
    step_.alloc(2 * 4);
    err_.alloc(4);
    Q3_CUDA(cudaMemsetAsync(err_.ptr, 0, 4, s_));
    x_last_.alloc(static_cast<size_t>(c.dim) * 4);
    prefill_ = std::make_unique<Prefill>(c, model.device());
    prepare_gemm_kernels();  // no attribute setup may happen inside a graph capture
    // Contraction operands of every layer with 128-row boxes (tile width 128: many CTAs for the
    // few rows of a decode step). w1 and w3 sit back to back in the arena: one [2H, D] operand.
    const int qkv = (c.n_heads + 2 * c.n_kv_heads) * HD, qd = c.n_heads * HD;
    wmaps_.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& w = model.layer(l);
        if (w.w3 != w.w1 + static_cast<size_t>(c.hidden_dim) * c.dim) {
            throw std::runtime_error("w1 and w3 are not adjacent in the weight arena");
        }
        make_tmap_bf16(&wmaps_[l].wqkv, w.wqkv, qkv, c.dim, 128);
        make_tmap_bf16(&wmaps_[l].wo, w.wo, c.dim, qd, 128);
        make_tmap_bf16(&wmaps_[l].w13, w.w1, 2 * static_cast<uint64_t>(c.hidden_dim), c.dim, 128);
        make_tmap_bf16(&wmaps_[l].w2, w.w2, c.dim, c.hidden_dim, 128);
    }
    make_tmap_bf16(&lm_, model.output(), c.vocab_size, c.dim, 128);
    Q3_CUDA(cudaStreamSynchronize(s_));
}

Batch::~Batch() {
    if (graph_) cudaGraphExecDestroy(graph_);
    if (s_) cudaStreamDestroy(s_);
}

int Batch::add(const int32_t* ids, int n, int32_t* next_token, float* last_logits) {
    const q3_config& c = cfg_;
    if (!ids || n <= 0) throw std::invalid_argument("a sequence needs at least one prompt token");
    if (size() >= max_seqs_) throw std::out_of_range("the batch is full");
    if (n > max_tokens_) throw std::out_of_range("prompt longer than the batch's sequence capacity");
    for (int i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= c.vocab_size) throw std::out_of_range("Token id is outside the vocabulary");
    }
    const int slot = size();
    if (ids_.bytes < static_cast<size_t>(n) * 4) ids_.alloc(static_cast<size_t>(n) * 4);
    Q3_CUDA(cudaMemcpyAsync(ids_.ptr, ids, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, s_));
    KvView kv;
    kv.k_base = static_cast<uint16_t*>(k_.ptr);
    kv.v_base = static_cast<uint16_t*>(v_.ptr);
    kv.n_pages = pool_pages_;
    kv.page_table = static_cast<const int32_t*>(table_.ptr) + static_cast<size_t>(slot) * pps_;
    kv.rope = static_cast<const float2*>(rope_.ptr);
    kv.rope_len = rope_len_;
    kv.table_len = pps_;
    float* xl = static_cast<float*>(x_last_.ptr);
    std::vector<LayerWeights> layers(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) layers[l] = m_.layer(l);
    // The prompt's slot range is checked against the slot's pages, not the model's context.
    prefill_->set_precision(m_.prefill_precision());
    const std::vector<LayerWeights>* l16 =
        m_.prefill_precision() == Prefill::kPrecisionF16 ? &m_.layers_f16() : nullptr;
    prefill_->run(static_cast<const int32_t*>(ids_.ptr), n, 0, m_.embed(), layers, kv, xl,
                  nullptr, s_, l16);
    DeviceBuffer lg, am, part;
    lg.alloc(static_cast<size_t>(c.vocab_size) * 4);
    am.alloc(4);
    part.alloc(static_cast<size_t>(gemv_grid(c.vocab_size)) * sizeof(float2));
    launch_gemv(kEpiStore, m_.output(), nullptr, xl, m_.final_norm(), c.norm_eps,
                static_cast<float*>(lg.ptr), nullptr, c.vocab_size, c.dim,
                static_cast<float2*>(part.ptr), gemv_grid(c.vocab_size), s_);
    launch_argmax_final(static_cast<const float2*>(part.ptr), gemv_grid(c.vocab_size),
                        static_cast<int32_t*>(am.ptr), nullptr, nullptr, 0, nullptr, s_);
    int32_t nt = 0;
    Q3_CUDA(cudaMemcpyAsync(&nt, am.ptr, 4, cudaMemcpyDeviceToHost, s_));
    if (last_logits) {
        Q3_CUDA(cudaMemcpyAsync(last_logits, lg.ptr, lg.bytes, cudaMemcpyDeviceToHost, s_));
    }
    Q3_CUDA(cudaStreamSynchronize(s_));
    if (const unsigned e = prefill_->read_error(s_)) {
        throw DeviceTimeout("batched prefill: a tensor-core pipeline wait gave up (code " +
                            std::to_string(e) + ")");
    }
    len_.push_back(n);
    next_.push_back(nt);
    if (next_token) *next_token = nt;
    return slot;
}

int Batch::add_many(const int32_t* ids, const int* lens, int n_seqs, int32_t* next_tokens,
                    float* last_logits) {
    const q3_config& c = cfg_;
    if (!ids || !lens || n_seqs <= 0) throw std::invalid_argument("add_many needs sequences");
    if (size() + n_seqs > max_seqs_) throw std::out_of_range("the batch is full");
    std::vector<int> off(n_seqs), len(n_seqs), toff(n_seqs);
    size_t total = 0;
    for (int i = 0; i < n_seqs; ++i) {
        if (lens[i] <= 0) throw std::invalid_argument("a sequence needs at least one prompt token");
        if (lens[i] > max_tokens_) {
            throw std::out_of_range("prompt longer than the batch's sequence capacity");
        }
        off[i] = static_cast<int>(total);
        len[i] = lens[i];
        toff[i] = (size() + i) * pps_;
        total += lens[i];
    }
    for (size_t i = 0; i < total; ++i) {
        if (ids[i] < 0 || ids[i] >= c.vocab_size) {
            throw std::out_of_range("Token id is outside the vocabulary");
        }
    }
    const int slot0 = size();
    if (ids_.bytes < total * 4) {
        Q3_CUDA(cudaStreamSynchronize(s_));
        ids_.alloc(total * 4);
    }
    Q3_CUDA(cudaMemcpyAsync(ids_.ptr, ids, total * 4, cudaMemcpyHostToDevice, s_));
    KvView kv;
    kv.k_base = static_cast<uint16_t*>(k_.ptr);
    kv.v_base = static_cast<uint16_t*>(v_.ptr);
    kv.n_pages = pool_pages_;
    kv.page_table = static_cast<const int32_t*>(table_.ptr);
    kv.rope = static_cast<const float2*>(rope_.ptr);
    kv.rope_len = rope_len_;
    kv.table_len = pps_;
    std::vector<LayerWeights> layers(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) layers[l] = m_.layer(l);
    prefill_->set_precision(m_.prefill_precision());
    const std::vector<LayerWeights>* l16 =
        m_.prefill_precision() == Prefill::kPrecisionF16 ? &m_.layers_f16() : nullptr;
    DeviceBuffer xl;
    xl.alloc(static_cast<size_t>(n_seqs) * c.dim * 4);
    float* XL = static_cast<float*>(xl.ptr);
    // Prompts that fit one chunk go through the varlen pass, in runs of consecutive ones; their
    // last hidden states land in XL at their own index.
    std::vector<int> vo, vl, vt, vi;
    auto flush = [&] {
        if (vo.empty()) return;
        DeviceBuffer xs;
        xs.alloc(vo.size() * c.dim * 4);
        prefill_->run_varlen(static_cast<const int32_t*>(ids_.ptr), vo, vl, vt, table_host_.data(),
                             m_.embed(), layers, kv, static_cast<float*>(xs.ptr), s_, l16);
        for (size_t j = 0; j < vi.size(); ++j) {
            Q3_CUDA(cudaMemcpyAsync(XL + static_cast<size_t>(vi[j]) * c.dim,
                                    static_cast<float*>(xs.ptr) + j * c.dim, c.dim * 4,
                                    cudaMemcpyDeviceToDevice, s_));
        }
        Q3_CUDA(cudaStreamSynchronize(s_));
        vo.clear();
        vl.clear();
        vt.clear();
        vi.clear();
    };
    for (int i = 0; i < n_seqs; ++i) {
        if (len[i] <= Prefill::kMaxChunk) {
            vo.push_back(off[i]);
            vl.push_back(len[i]);
            vt.push_back(toff[i]);
            vi.push_back(i);
            continue;
        }
        flush();
        KvView one = kv;
        one.page_table = static_cast<const int32_t*>(table_.ptr) + toff[i];
        prefill_->run(static_cast<const int32_t*>(ids_.ptr) + off[i], len[i], 0, m_.embed(),
                      layers, one, XL + static_cast<size_t>(i) * c.dim, nullptr, s_, l16);
    }
    flush();
    // Final RmsNorm + tied lm_head and Greedy of each prompt's last token (src/inference.cpp:
    // 619-635, :703-709).
    DeviceBuffer lg, am, part;
    lg.alloc(static_cast<size_t>(c.vocab_size) * 4);
    am.alloc(static_cast<size_t>(n_seqs) * 4);
    part.alloc(static_cast<size_t>(gemv_grid(c.vocab_size)) * sizeof(float2));
    for (int i = 0; i < n_seqs; ++i) {
        launch_gemv(kEpiStore, m_.output(), nullptr, XL + static_cast<size_t>(i) * c.dim,
                    m_.final_norm(), c.norm_eps, static_cast<float*>(lg.ptr), nullptr,
                    c.vocab_size, c.dim, static_cast<float2*>(part.ptr),
                    gemv_grid(c.vocab_size), s_);
        launch_argmax_final(static_cast<const float2*>(part.ptr), gemv_grid(c.vocab_size),
                            static_cast<int32_t*>(am.ptr) + i, nullptr, nullptr, 0, nullptr, s_);
        if (last_logits) {
            Q3_CUDA(cudaMemcpyAsync(last_logits + static_cast<size_t>(i) * c.vocab_size, lg.ptr,
                                    lg.bytes, cudaMemcpyDeviceToHost, s_));
        }
    }
    std::vector<int32_t> nt(n_seqs);
    Q3_CUDA(cudaMemcpyAsync(nt.data(), am.ptr, static_cast<size_t>(n_seqs) * 4,
                            cudaMemcpyDeviceToHost, s_));
    Q3_CUDA(cudaStreamSynchronize(s_));
    if (const unsigned e = prefill_->read_error(s_)) {
        throw DeviceTimeout("batched prefill: a tensor-core pipeline wait gave up (code " +
                            std::to_string(e) + ")");
    }
    for (int i = 0; i < n_seqs; ++i) {
        len_.push_back(len[i]);
        next_.push_back(nt[i]);
        if (next_tokens) next_tokens[i] = nt[i];
    }
    return slot0;
}

void Batch::ensure_step_buffers() {
    const int B = size();
    if (B == cap_rows_) return;
    const q3_config& c = cfg_;
    const int qkv = (c.n_heads + 2 * c.n_kv_heads) * HD, qd = c.n_heads * HD, H = c.hidden_dim;
    x_.alloc(static_cast<size_t>(B) * c.dim * 4);
    xn_.alloc(static_cast<size_t>(B) * c.dim * 2);
    xn_lo_.alloc(static_cast<size_t>(B) * c.dim * 2);
    o_lo_.alloc(static_cast<size_t>(B) * qd * 2);
    h_lo_.alloc(static_cast<size_t>(B) * H * 2);
    qkv_.alloc(static_cast<size_t>(B) * qkv * 4);
    o_.alloc(static_cast<size_t>(B) * qd * 2);
    gu_.alloc(static_cast<size_t>(B) * 2 * H * 4);
    h_.alloc(static_cast<size_t>(B) * H * 2);
    logits_.alloc(static_cast<size_t>(B) * c.vocab_size * 4);
    make_tmap_bf16(&a_xn_, xn_.ptr, B, c.dim, 128);
    make_tmap_bf16(&a_o_, o_.ptr, B, qd, 128);
    make_tmap_bf16(&a_h_, h_.ptr, B, H, 128);
    make_tmap_bf16(&a_xn_lo_, xn_lo_.ptr, B, c.dim, 128);
    make_tmap_bf16(&a_o_lo_, o_lo_.ptr, B, qd, 128);
    make_tmap_bf16(&a_h_lo_, h_lo_.ptr, B, H, 128);
    make_tmap_out(&o_qkv_, qkv_.ptr, B, qkv, false);
    make_tmap_out(&o_x_, x_.ptr, B, c.dim, false);
    make_tmap_out(&o_gu_, gu_.ptr, B, 2 * static_cast<uint64_t>(H), false);
    make_tmap_out(&o_logits_, logits_.ptr, B, c.vocab_size, false);
    // Decode attention on the CUDA cores: fp32 q rows, split partials and merge counters.
    q32_.alloc(static_cast<size_t>(B) * qd * 4);
    attn_pps_ = decode_attn_pages_per_split(B, c.n_kv_heads, pps_, prefill_->num_sms());
    attn_splits_ = (pps_ + attn_pps_ - 1) / attn_pps_;
    const size_t pairs = static_cast<size_t>(B) * c.n_kv_heads;
    attn_part_o_.alloc(pairs * attn_splits_ * 2 * HD * 4);
    attn_part_ml_.alloc(pairs * attn_splits_ * 2 * sizeof(float2));
    attn_counter_.alloc(pairs * sizeof(unsigned));
    Q3_CUDA(cudaMemset(attn_counter_.ptr, 0, attn_counter_.bytes));
    cap_rows_ = B;
    if (graph_) {
        cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
}

void Batch::enqueue_step(bool forced, int n_forced) {
    const q3_config& c = cfg_;
    const int B = size();
    const int qkv = (c.n_heads + 2 * c.n_kv_heads) * HD, qd = c.n_heads * HD, H = c.hidden_dim;
    const int sms = prefill_->num_sms();
    unsigned* err = static_cast<unsigned*>(err_.ptr);
    float* X = static_cast<float*>(x_.ptr);
    uint16_t* Xn = static_cast<uint16_t*>(xn_.ptr);
    const size_t layer_elems = static_cast<size_t>(pool_pages_) * c.n_kv_heads * kPageTokens * HD;
    // Every contraction takes its activations as a bf16 hi + lo pair (fp32-like operands: the
    // extra MMA is free while the step streams weights from HBM).
    auto gemm = [&](const CUtensorMap& a, const CUtensorMap& a_lo, const CUtensorMap& b,
                    const CUtensorMap& out, int N, int K, int epi) {
        GemmArgs g;
        g.M = B;
        g.N = N;
        g.K = K;
        g.err = err;
        g.bn = 128;
        g.max_ksplit = 16;
        g.min_slice_kblocks = 2;
        g.dependent = true;
        Q3_CUDA(launch_gemm(a, b, nullptr, out, g, epi, sms, s_, &a_lo));
    };
    uint16_t* Xn_lo = static_cast<uint16_t*>(xn_lo_.ptr);
    launch_rmsnorm_rows_bf16(static_cast<const int32_t*>(tok_.ptr), m_.embed(), X,
                             m_.layer(0).attn_norm, c.norm_eps, Xn, B, c.dim, s_, Xn_lo);
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& w = m_.layer(l);
        const LayerMaps& wm = wmaps_[l];
        Q3_CUDA(cudaMemsetAsync(qkv_.ptr, 0, qkv_.bytes, s_));
        gemm(a_xn_, a_xn_lo_, wm.wqkv, o_qkv_, qkv, c.dim, kEpiAddF32);
        PrefillQkvArgs qa{};
        qa.qkv = static_cast<float*>(qkv_.ptr);
        qa.q_norm = w.q_norm;
        qa.k_norm = w.k_norm;
        qa.rope = static_cast<const float2*>(rope_.ptr);
        qa.k_cache = static_cast<uint16_t*>(k_.ptr) + layer_elems * l;
        qa.v_cache = static_cast<uint16_t*>(v_.ptr) + layer_elems * l;
        qa.page_table = static_cast<const int32_t*>(table_.ptr);
        qa.rows = B;
        qa.pos0 = 0;
        qa.n_heads = c.n_heads;
        qa.n_kv = c.n_kv_heads;
        qa.eps = c.norm_eps;
        qa.dec_pos = static_cast<const int32_t*>(pos_.ptr);
        qa.pages_per_seq = pps_;
        qa.q_out_f32 = static_cast<float*>(q32_.ptr);
        launch_prefill_qkv(qa, s_);
        {
            DecodeAttnArgs da{};
            da.q = static_cast<const float*>(q32_.ptr);
            da.q_stride = qd;
            da.k_cache = static_cast<const uint16_t*>(k_.ptr) + layer_elems * l;
            da.v_cache = static_cast<const uint16_t*>(v_.ptr) + layer_elems * l;
            da.page_table = static_cast<const int32_t*>(table_.ptr);
            da.pages_per_seq = pps_;
            da.dec_pos = static_cast<const int32_t*>(pos_.ptr);
            da.rows = B;
            da.n_kv = c.n_kv_heads;
            da.kv_head0 = 0;
            da.n_kv_cache = c.n_kv_heads;
            da.pages_per_split = attn_pps_;
            da.max_splits = attn_splits_;
            da.part_o = static_cast<float*>(attn_part_o_.ptr);
            da.part_ml = static_cast<float2*>(attn_part_ml_.ptr);
            da.counter = static_cast<unsigned*>(attn_counter_.ptr);
            da.out = static_cast<uint16_t*>(o_.ptr);
            da.out_lo = static_cast<uint16_t*>(o_lo_.ptr);
            da.out_stride = qd;
            launch_decode_attention(da, s_);
        }
        gemm(a_o_, a_o_lo_, wm.wo, o_x_, c.dim, qd, kEpiAddF32);
        launch_rmsnorm_rows_bf16(nullptr, nullptr, X, w.mlp_norm, c.norm_eps, Xn, B, c.dim, s_,
                                 Xn_lo);
        Q3_CUDA(cudaMemsetAsync(gu_.ptr, 0, gu_.bytes, s_));
        gemm(a_xn_, a_xn_lo_, wm.w13, o_gu_, 2 * H, c.dim, kEpiAddF32);
        const size_t quads = static_cast<size_t>(B) * H / 4;
        launch_dep(false, swiglu_rows_kernel,
                   dim3(static_cast<unsigned>(std::min<size_t>((quads + 255) / 256, 4096))), dim3(256),
                   0, s_, static_cast<const float*>(gu_.ptr), static_cast<uint16_t*>(h_.ptr),
                   static_cast<uint16_t*>(h_lo_.ptr), B, H);
        Q3_CUDA(cudaGetLastError());
        gemm(a_h_, a_h_lo_, wm.w2, o_x_, c.dim, H, kEpiAddF32);
        const uint16_t* next_norm = l + 1 < c.n_layers ? m_.layer(l + 1).attn_norm : m_.final_norm();
        launch_rmsnorm_rows_bf16(nullptr, nullptr, X, next_norm, c.norm_eps, Xn, B, c.dim, s_,
                                 Xn_lo);
    }
    // Tied lm_head for every row, argmax and the advance.
    gemm(a_xn_, a_xn_lo_, lm_, o_logits_, c.vocab_size, c.dim, kEpiStoreF32);
    launch_dep(false, batch_argmax_kernel, dim3(B), dim3(1024), 0, s_,
               static_cast<const float*>(logits_.ptr), B, c.vocab_size,
               static_cast<int32_t*>(tok_.ptr), static_cast<int32_t*>(pos_.ptr),
               static_cast<int32_t*>(log_.ptr), static_cast<const int32_t*>(step_.ptr),
               forced ? static_cast<const int32_t*>(forced_.ptr) : nullptr);
    Q3_CUDA(cudaGetLastError());
    launch_dep(false, advance_step_kernel, dim3(1), dim3(1), 0, s_, static_cast<int32_t*>(step_.ptr));
    Q3_CUDA(cudaGetLastError());
    (void)n_forced;
}

void Batch::run(int n_steps, const int32_t* forced_host, int32_t* log_host, float* logits_host) {
    const int B = size();
    if (B == 0) throw std::invalid_argument("the batch has no sequences");
    if (n_steps <= 0) return;
    for (int b = 0; b < B; ++b) {
        if (len_[b] + n_steps > max_tokens_) {
            throw std::out_of_range("decode past the batch's sequence capacity");
        }
    }
    if (forced_host) {
        for (size_t i = 0; i < static_cast<size_t>(n_steps) * B; ++i) {
            if (forced_host[i] < 0 || forced_host[i] >= cfg_.vocab_size) {
                throw std::out_of_range("Token id is outside the vocabulary");
            }
        }
    }
    ensure_step_buffers();
    const size_t log_elems = static_cast<size_t>(n_steps) * B;
    if (static_cast<size_t>(log_cap_) < log_elems) {
        log_.alloc(log_elems * 4);
        forced_.alloc(log_elems * 4);
        log_cap_ = static_cast<int>(log_elems);
        if (graph_) {
            cudaGraphExecDestroy(graph_);
            graph_ = nullptr;
        }
    }
    // Per-sequence state: position of the token fed next and the token itself.
    std::vector<int32_t> pos(B), tok(B);
    for (int b = 0; b < B; ++b) {
        pos[b] = len_[b];
        tok[b] = forced_host ? forced_host[b] : next_[b];
    }
    const int32_t state[2] = {0, forced_host ? n_steps : 0};
    Q3_CUDA(cudaMemcpyAsync(pos_.ptr, pos.data(), B * 4, cudaMemcpyHostToDevice, s_));
    Q3_CUDA(cudaMemcpyAsync(tok_.ptr, tok.data(), B * 4, cudaMemcpyHostToDevice, s_));
    Q3_CUDA(cudaMemcpyAsync(step_.ptr, state, sizeof(state), cudaMemcpyHostToDevice, s_));
    if (forced_host) {
        Q3_CUDA(cudaMemcpyAsync(forced_.ptr, forced_host, log_elems * 4, cudaMemcpyHostToDevice, s_));
    }
    const bool forced = forced_host != nullptr;
    if (logits_host) {
        // Logits of every step go to the host: plain launches, one step at a time.
        for (int i = 0; i < n_steps; ++i) {
            enqueue_step(forced, n_steps);
            Q3_CUDA(cudaMemcpyAsync(logits_host + static_cast<size_t>(i) * B * cfg_.vocab_size,
                                    logits_.ptr, static_cast<size_t>(B) * cfg_.vocab_size * 4,
                                    cudaMemcpyDeviceToHost, s_));
        }
    } else {
        if (!graph_ || graph_rows_ != B || graph_forced_ != forced) {
            if (graph_) cudaGraphExecDestroy(graph_);
            graph_ = nullptr;
            // Device constants the kernels read (tensor maps of the KV pool) are set up first.
            KvView kv;
            kv.k_base = static_cast<uint16_t*>(k_.ptr);
            kv.v_base = static_cast<uint16_t*>(v_.ptr);
            kv.n_pages = pool_pages_;
            prefill_->ensure_kv_maps(kv, cfg_.n_layers);
            cudaGraph_t g = nullptr;
            Q3_CUDA(cudaStreamBeginCapture(s_, cudaStreamCaptureModeThreadLocal));
            try {
                enqueue_step(forced, n_steps);
            } catch (...) {
                cudaStreamEndCapture(s_, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            Q3_CUDA(cudaStreamEndCapture(s_, &g));
            const cudaError_t ie = cudaGraphInstantiate(&graph_, g, 0);
            cudaGraphDestroy(g);
            Q3_CUDA(ie);
            graph_rows_ = B;
            graph_forced_ = forced;
        }
        for (int i = 0; i < n_steps; ++i) Q3_CUDA(cudaGraphLaunch(graph_, s_));
    }
    std::vector<int32_t> log(log_elems);
    Q3_CUDA(cudaMemcpyAsync(log.data(), log_.ptr, log_elems * 4, cudaMemcpyDeviceToHost, s_));
    Q3_CUDA(cudaStreamSynchronize(s_));
    unsigned e = 0;
    Q3_CUDA(cudaMemcpy(&e, err_.ptr, 4, cudaMemcpyDeviceToHost));
    if (e) {
        Q3_CUDA(cudaMemset(err_.ptr, 0, 4));
        throw DeviceTimeout("batched decode: a tensor-core pipeline wait gave up (code " +
                            std::to_string(e) + ")");
    }
    for (int b = 0; b < B; ++b) {
        len_[b] += n_steps;
        next_[b] = log[static_cast<size_t>(n_steps - 1) * B + b];
    }
    if (log_host) std::memcpy(log_host, log.data(), log_elems * 4);
}

void Batch::decode(int n_steps, int32_t* tokens_host) { run(n_steps, nullptr, tokens_host, nullptr); }

void Batch::decode_forced(const int32_t* tokens_host, int n_steps, int32_t* argmax_host,
                          float* logits_host) {
    if (!tokens_host) throw std::invalid_argument("null argument");
    run(n_steps, tokens_host, argmax_host, logits_host);
}

void Batch::kv_row(int slot, int layer, int pos, uint16_t* k_host, uint16_t* v_host) {
    const q3_config& c = cfg_;
    if (slot < 0 || slot >= size() || layer < 0 || layer >= c.n_layers || pos < 0 ||
        pos >= len_[slot]) {
        throw std::out_of_range("KV row outside the sequence");
    }
    const size_t layer_elems = static_cast<size_t>(pool_pages_) * c.n_kv_heads * kPageTokens * HD;
    const int page = slot * pps_ + pos / kPageTokens;
    Q3_CUDA(cudaStreamSynchronize(s_));
    for (int g = 0; g < c.n_kv_heads; ++g) {
        const size_t off = layer_elems * layer +
                           ((static_cast<size_t>(page) * c.n_kv_heads + g) * kPageTokens +
                            pos % kPageTokens) * HD;
        if (k_host) {
            Q3_CUDA(cudaMemcpy(k_host + g * HD, static_cast<uint16_t*>(k_.ptr) + off, HD * 2,
                               cudaMemcpyDeviceToHost));
        }
        if (v_host) {
            Q3_CUDA(cudaMemcpy(v_host + g * HD, static_cast<uint16_t*>(v_.ptr) + off, HD * 2,
                               cudaMemcpyDeviceToHost));
        }
    }
}

}  // namespace q3
