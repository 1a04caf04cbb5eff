// Tensor-parallel single-sequence decode (see q3_tp.cuh).
//
// One decode step per rank, captured as one CUDA graph; every contraction takes its activations
// as bf16 hi + lo pairs (as in batched decode) and consumers clear their fp32 inputs for the next
// step's reduce-adds, so no memsets run inside the step:
//   embedding row + RmsNorm
//   per layer: local [wq;wk;wv] rows -> local q/k/v; QK-norm + RoPE + K/V write of the local KV
//              heads; attention over the local heads (split over KV positions, then merged);
//              o_proj over the local columns -> partial; all-reduce + RmsNorm;
//              local [w1;w3] rows -> SiLU(gate) * up; down_proj over the local columns ->
//              partial; all-reduce + RmsNorm of the next layer (or the final norm)
//   lm_head over the local vocabulary rows, argmax all-reduce, device-side advance.
//
// All-reduce over peer memory. Exchange buffer of every rank (CUDA IPC, mapped by every peer):
//   data  [2 parities][8 sources][dim] fp32, argmax [2][8] (value, index), flags [8] u32.
// Invocation c (a per-rank counter, identical on all ranks since every rank runs the same step):
// rank r stores its partial into data[c&1][r] of every peer, fences (system scope), then stores
// flag[r] = c into every peer (release); it waits (bounded) until its own flag[s] >= c for every
// source s (acquire) and sums data[c&1][0..N-1] in rank order. Parity buffers are safe: a peer
// can only write parity c&1 again at invocation c+2, after it has seen this rank's flag c+1,
// which this rank raises after it consumed invocation c.
#include <cuda_bf16.h>
#include <float.h>

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

#include "q3_gemm.cuh"
#include "q3_kernels.cuh"
#include "q3_prefill.cuh"
#include "q3_tp.cuh"
#include "q3_decode_attn.cuh"

namespace q3 {

namespace {

constexpr int HD = 128;
constexpr int kDim = 1024;          // residual width the exchange buffer is sized for
constexpr size_t kDataBytes = 2ull * kTpMaxRanks * kDim * 4;
constexpr size_t kAmOff = kDataBytes;
constexpr size_t kFlagOff = kAmOff + 2ull * kTpMaxRanks * sizeof(float2);
constexpr size_t kXbufBytes = kFlagOff + 256;

struct TpPeers {
    uint8_t* buf[kTpMaxRanks];  // exchange buffers of every rank (this rank's own included)
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Waits (bounded) until every source's flag in this rank's buffer reached seq. Threads
// [0, world) poll one source each. Returns false on timeout.
__device__ bool wait_flags(const uint8_t* own, int world, unsigned seq, long long budget) {
    bool ok = true;
    if (static_cast<int>(threadIdx.x) < world) {
        const unsigned* f = reinterpret_cast<const unsigned*>(own + kFlagOff) + threadIdx.x;
        const long long t0 = clock64();
        while (ld_acquire_sys(f) < seq) {
            if (clock64() - t0 > budget) {
                ok = false;
                break;
            }
        }
    }
    return __syncthreads_and(ok) != 0;
}

__device__ void raise_flags(const TpPeers& P, int world, int rank, unsigned seq) {
    if (static_cast<int>(threadIdx.x) < world) {
        st_release_sys(reinterpret_cast<unsigned*>(P.buf[threadIdx.x] + kFlagOff) + rank, seq);
    }
}

// x += sum over ranks of part (rank order), then xn/xn_lo = RmsNorm(x) * w as a bf16 hi + lo pair
// (src/inference.cpp:905-921); part is cleared for the next step's reduce-adds. One block.
__global__ void __launch_bounds__(256) tp_allreduce_norm_kernel(
    TpPeers P, float* part, float* x, int rank, int world, unsigned* counter, unsigned* err,
    long long budget, const uint16_t* w, float eps, uint16_t* xn, uint16_t* xn_lo) {
    __shared__ float red[8];
    __shared__ unsigned s_seq;
    const int tid = threadIdx.x;
    if (tid == 0) s_seq = *counter + 1;
    __syncthreads();
    const unsigned seq = s_seq;
    const size_t par = seq & 1;
    const int i = tid * 4;  // kDim / 256 = 4 elements per thread
    const float4 mine = *reinterpret_cast<const float4*>(part + i);
    for (int p = 0; p < world; ++p) {
        float* dst = reinterpret_cast<float*>(P.buf[p]) + (par * kTpMaxRanks + rank) * kDim;
        *reinterpret_cast<float4*>(dst + i) = mine;
    }
    *reinterpret_cast<float4*>(part + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    __threadfence_system();
    __syncthreads();
    raise_flags(P, world, rank, seq);
    if (!wait_flags(P.buf[rank], world, seq, budget)) {
        if (tid == 0) atomicCAS(err, 0u, 21u);
        return;
    }
    // Peer-written data: L2-coherent loads (a line cached in L1 two invocations ago is stale).
    const float* own = reinterpret_cast<const float*>(P.buf[rank]) + par * kTpMaxRanks * kDim;
    float4 sum = __ldcg(reinterpret_cast<const float4*>(own + i));
    for (int s = 1; s < world; ++s) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(own + s * kDim + i));
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
    }
    float4 xv = *reinterpret_cast<float4*>(x + i);
    xv.x += sum.x;
    xv.y += sum.y;
    xv.z += sum.z;
    xv.w += sum.w;
    *reinterpret_cast<float4*>(x + i) = xv;
    float ss = xv.x * xv.x;
    ss = fmaf(xv.y, xv.y, ss);
    ss = fmaf(xv.z, xv.z, ss);
    ss = fmaf(xv.w, xv.w, ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(kDim) + eps);
    const uint2 wb = *reinterpret_cast<const uint2*>(w + i);
    const float y0 = (xv.x * inv) * bf16_lo(wb.x), y1 = (xv.y * inv) * bf16_hi(wb.x);
    const float y2 = (xv.z * inv) * bf16_lo(wb.y), y3 = (xv.w * inv) * bf16_hi(wb.y);
    const uint2 hi = make_uint2(pack2(y0, y1), pack2(y2, y3));
    *reinterpret_cast<uint2*>(xn + i) = hi;
    *reinterpret_cast<uint2*>(xn_lo + i) =
        make_uint2(pack2(y0 - bf16_lo(hi.x), y1 - bf16_hi(hi.x)), pack2(y2 - bf16_lo(hi.y), y3 - bf16_hi(hi.y)));
    if (tid == 0) *counter = seq;
}

// Greedy argmax over this rank's vocabulary rows, all-reduced (lowest index wins ties,
// src/inference.cpp:703-709); then log[step] = token, the next token (argmax or forced),
// position + 1, step + 1. state = {step, n_forced}. One block of 1024 threads.
__global__ void __launch_bounds__(1024) tp_argmax_kernel(
    TpPeers P, const float* logits, int vn, int v0, int rank, int world, unsigned* counter,
    unsigned* err, long long budget, int32_t* tok, int32_t* pos, int32_t* log, int32_t* state,
    const int32_t* forced) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    __shared__ unsigned s_seq;
    const int tid = threadIdx.x;
    if (tid == 0) s_seq = *counter + 1;
    float best = -INFINITY;
    int idx = INT_MAX;
    for (int i = tid; i < vn; i += blockDim.x) {
        const float v = logits[i];
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
    if ((tid & 31) == 0) {
        bv[tid >> 5] = best;
        bi[tid >> 5] = idx;
    }
    __syncthreads();
    const unsigned seq = s_seq;
    const size_t par = seq & 1;
    if (tid == 0) {
        for (int w = 1; w < 32; ++w) {
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
                best = bv[w];
                idx = bi[w];
            }
        }
        const float2 mine = make_float2(best, __int_as_float(idx + v0));
        for (int p = 0; p < world; ++p) {
            reinterpret_cast<float2*>(P.buf[p] + kAmOff)[par * kTpMaxRanks + rank] = mine;
        }
        __threadfence_system();
    }
    __syncthreads();
    raise_flags(P, world, rank, seq);
    if (!wait_flags(P.buf[rank], world, seq, budget)) {
        if (tid == 0) atomicCAS(err, 0u, 22u);
        return;
    }
    if (tid == 0) {
        const float2* am = reinterpret_cast<const float2*>(P.buf[rank] + kAmOff) + par * kTpMaxRanks;
        const float2 a0 = __ldcg(am);
        float b = a0.x;
        int bi0 = __float_as_int(a0.y);
        for (int s = 1; s < world; ++s) {
            const float2 as = __ldcg(am + s);
            const int si = __float_as_int(as.y);
            if (as.x > b || (as.x == b && si < bi0)) {
                b = as.x;
                bi0 = si;
            }
        }
        const int step = state[0];
        log[step] = bi0;
        tok[0] = (forced && step + 1 < state[1]) ? forced[step + 1] : bi0;
        pos[0] += 1;
        state[0] = step + 1;
        *counter = seq;
    }
}

// h = silu(gu[:H]) * gu[H:] as bf16 hi + lo; gu is cleared for the next step's reduce-add.
__global__ void tp_swiglu_kernel(float* gu, uint16_t* h, uint16_t* h_lo, int H) {
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) * 2; i < H; i += gridDim.x * blockDim.x * 2) {
        const float g0 = gu[i], g1 = gu[i + 1], u0 = gu[H + i], u1 = gu[H + i + 1];
        gu[i] = gu[i + 1] = gu[H + i] = gu[H + i + 1] = 0.0f;
        const float a = g0 / (1.0f + expf(-g0)) * u0, b = g1 / (1.0f + expf(-g1)) * u1;
        const uint32_t hi = pack2(a, b);
        *reinterpret_cast<uint32_t*>(h + i) = hi;
        *reinterpret_cast<uint32_t*>(h_lo + i) =
            pack2(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xffff0000u));
    }
}

}  // namespace

TpDecoder::TpDecoder(Model& model, int rank, int world)
    : m_(model), cfg_(model.config()), rank_(rank), world_(world) {
    const q3_config& c = cfg_;
    if (world < 1 || world > kTpMaxRanks || rank < 0 || rank >= world) {
        throw std::invalid_argument("tensor parallelism: rank/world out of range");
    }
    if (!Prefill::supported(c) || c.dim != kDim || c.n_kv_heads % world != 0 ||
        c.hidden_dim % (128 * world) != 0 || c.vocab_size % 128 != 0) {
        throw std::invalid_argument("tensor parallelism needs the Qwen3-0.6B shape and a world "
                                    "size dividing the KV heads");
    }
    Q3_CUDA(cudaSetDevice(model.device()));
    Q3_CUDA(cudaStreamCreateWithFlags(&s_, cudaStreamNonBlocking));
    hkv_ = c.n_kv_heads / world;
    hq_ = c.n_heads / world;
    hl_ = c.hidden_dim / world;
    const int vtiles = c.vocab_size / 128, per = (vtiles + world - 1) / world;
    v0_ = std::min(vtiles, rank * per) * 128;
    vn_ = (std::min(vtiles, (rank + 1) * per) * 128) - v0_;
    if (vn_ <= 0) throw std::invalid_argument("vocabulary too small for this many ranks");
    const size_t D = c.dim, qd = static_cast<size_t>(c.n_heads) * HD;
    const size_t kvd = static_cast<size_t>(c.n_kv_heads) * HD;
    const size_t qkv_l = static_cast<size_t>(hq_ + 2 * hkv_) * HD;
    const size_t shard_layer = (qkv_l + 2 * static_cast<size_t>(hl_)) * D;
    shard_.alloc(shard_layer * c.n_layers * 2);
    wmaps_.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& w = model.layer(l);
        uint16_t* sq = static_cast<uint16_t*>(shard_.ptr) + shard_layer * l;
        uint16_t* s13 = sq + qkv_l * D;
        // [wq;wk;wv] rows of the local heads, then [w1;w3] rows of the local MLP slice.
        const uint16_t* wq = w.wqkv;
        const uint16_t* wk = w.wqkv + qd * D;
        const uint16_t* wv = wk + kvd * D;
        Q3_CUDA(cudaMemcpyAsync(sq, wq + static_cast<size_t>(rank) * hq_ * HD * D,
                                static_cast<size_t>(hq_) * HD * D * 2, cudaMemcpyDeviceToDevice, s_));
        Q3_CUDA(cudaMemcpyAsync(sq + static_cast<size_t>(hq_) * HD * D,
                                wk + static_cast<size_t>(rank) * hkv_ * HD * D,
                                static_cast<size_t>(hkv_) * HD * D * 2, cudaMemcpyDeviceToDevice, s_));
        Q3_CUDA(cudaMemcpyAsync(sq + static_cast<size_t>(hq_ + hkv_) * HD * D,
                                wv + static_cast<size_t>(rank) * hkv_ * HD * D,
                                static_cast<size_t>(hkv_) * HD * D * 2, cudaMemcpyDeviceToDevice, s_));
        Q3_CUDA(cudaMemcpyAsync(s13, w.w1 + static_cast<size_t>(rank) * hl_ * D,
                                static_cast<size_t>(hl_) * D * 2, cudaMemcpyDeviceToDevice, s_));
        Q3_CUDA(cudaMemcpyAsync(s13 + static_cast<size_t>(hl_) * D,
                                w.w3 + static_cast<size_t>(rank) * hl_ * D,
                                static_cast<size_t>(hl_) * D * 2, cudaMemcpyDeviceToDevice, s_));
        make_tmap_bf16(&wmaps_[l].wqkv, sq, qkv_l, D, 128);
        make_tmap_bf16(&wmaps_[l].w13, s13, 2 * static_cast<uint64_t>(hl_), D, 128);
        // Column slices read in place: wo[:, local q columns], w2[:, local MLP columns].
        make_tmap_bf16_strided(&wmaps_[l].wo, w.wo + static_cast<size_t>(rank) * hq_ * HD, D,
                               static_cast<uint64_t>(hq_) * HD, qd, 128);
        make_tmap_bf16_strided(&wmaps_[l].w2, w.w2 + static_cast<size_t>(rank) * hl_, D, hl_,
                               c.hidden_dim, 128);
    }
    make_tmap_bf16(&lm_, model.output() + static_cast<size_t>(v0_) * D, vn_, D, 128);

    x_.alloc(D * 4);
    xn_.alloc(D * 2);
    xn_lo_.alloc(D * 2);
    qkv_.alloc(qkv_l * 4);
    q32_.alloc(static_cast<size_t>(hq_) * HD * 4);
    o_.alloc(static_cast<size_t>(hq_) * HD * 2);
    o_lo_.alloc(static_cast<size_t>(hq_) * HD * 2);
    part_.alloc(D * 4);
    gu_.alloc(2 * static_cast<size_t>(hl_) * 4);
    h_.alloc(static_cast<size_t>(hl_) * 2);
    h_lo_.alloc(static_cast<size_t>(hl_) * 2);
    logits_.alloc(static_cast<size_t>(vn_) * 4);
    pos_.alloc(4);
    tok_.alloc(4);
    step_.alloc(8);
    err_.alloc(4);
    counter_.alloc(4);
    xbuf_.alloc(kXbufBytes);
    for (DeviceBuffer* b : {&qkv_, &part_, &gu_, &err_, &counter_, &xbuf_}) {
        Q3_CUDA(cudaMemsetAsync(b->ptr, 0, b->bytes, s_));
    }
    make_tmap_bf16(&a_xn_, xn_.ptr, 1, D, 128);
    make_tmap_bf16(&a_xn_lo_, xn_lo_.ptr, 1, D, 128);
    make_tmap_bf16(&a_o_, o_.ptr, 1, static_cast<uint64_t>(hq_) * HD, 128);
    make_tmap_bf16(&a_o_lo_, o_lo_.ptr, 1, static_cast<uint64_t>(hq_) * HD, 128);
    make_tmap_bf16(&a_h_, h_.ptr, 1, hl_, 128);
    make_tmap_bf16(&a_h_lo_, h_lo_.ptr, 1, hl_, 128);
    make_tmap_out(&o_qkv_, qkv_.ptr, 1, qkv_l, false);
    make_tmap_out(&o_part_, part_.ptr, 1, D, false);
    make_tmap_out(&o_gu_, gu_.ptr, 1, 2 * static_cast<uint64_t>(hl_), false);
    make_tmap_out(&o_logits_, logits_.ptr, 1, vn_, false);
    // Decode attention split over the cached pages of the local KV heads.
    Q3_CUDA(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, model.device()));
    const int max_pages = model.engine().n_pages();
    attn_pps_ = decode_attn_pages_per_split(1, hkv_, max_pages, sms_);
    attn_splits_ = (max_pages + attn_pps_ - 1) / attn_pps_;
    part_o_.alloc(static_cast<size_t>(hkv_) * attn_splits_ * 2 * HD * 4);
    part_ml_.alloc(static_cast<size_t>(hkv_) * attn_splits_ * 2 * sizeof(float2));
    attn_counter_.alloc(static_cast<size_t>(hkv_) * sizeof(unsigned));
    Q3_CUDA(cudaMemsetAsync(attn_counter_.ptr, 0, attn_counter_.bytes, s_));
    prepare_gemm_kernels();
    Q3_CUDA(cudaStreamSynchronize(s_));
}

TpDecoder::~TpDecoder() {
    if (graph_) cudaGraphExecDestroy(graph_);
    for (void* p : peer_mapped_) {
        if (p) cudaIpcCloseMemHandle(p);
    }
    if (s_) cudaStreamDestroy(s_);
}

void TpDecoder::ipc_handle(void* out) const {
    cudaIpcMemHandle_t h;
    Q3_CUDA(cudaIpcGetMemHandle(&h, xbuf_.ptr));
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(out, &h, sizeof(h));
}

void TpDecoder::connect(const void* handles) {
    if (connected_) throw std::runtime_error("tensor parallelism: already connected");
    peer_mapped_.assign(world_, nullptr);
    const auto* hs = static_cast<const uint8_t*>(handles);
    for (int p = 0; p < world_; ++p) {
        if (p == rank_) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + 64 * p, 64);
        void* ptr = nullptr;
        Q3_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        peer_mapped_[p] = ptr;
    }
    connected_ = true;
}

void TpDecoder::enqueue_step(bool forced) {
    const q3_config& c = cfg_;
    const int qkv_l = (hq_ + 2 * hkv_) * HD;
    const int sms = sms_;
    unsigned* err = static_cast<unsigned*>(err_.ptr);
    unsigned* counter = static_cast<unsigned*>(counter_.ptr);
    TpPeers P{};
    for (int p = 0; p < world_; ++p) {
        P.buf[p] = static_cast<uint8_t*>(p == rank_ ? xbuf_.ptr : peer_mapped_[p]);
    }
    constexpr long long kBudget = 4000000000LL;
    auto gemm = [&](const CUtensorMap& a, const CUtensorMap& a_lo, const CUtensorMap& b,
                    const CUtensorMap& out, int N, int K, int epi) {
        GemmArgs g;
        g.M = 1;
        g.N = N;
        g.K = K;
        g.err = err;
        g.bn = 128;
        g.max_ksplit = 16;
        g.min_slice_kblocks = 2;
        Q3_CUDA(launch_gemm(a, b, nullptr, out, g, epi, sms, s_, &a_lo));
    };
    float* X = static_cast<float*>(x_.ptr);
    uint16_t* Xn = static_cast<uint16_t*>(xn_.ptr);
    uint16_t* Xn_lo = static_cast<uint16_t*>(xn_lo_.ptr);
    Engine& e = m_.engine();
    launch_rmsnorm_rows_bf16(static_cast<const int32_t*>(tok_.ptr), m_.embed(), X,
                             m_.layer(0).attn_norm, c.norm_eps, Xn, 1, c.dim, s_, Xn_lo);
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& w = m_.layer(l);
        const LayerMaps& wm = wmaps_[l];
        gemm(a_xn_, a_xn_lo_, wm.wqkv, o_qkv_, qkv_l, c.dim, kEpiAddF32);
        PrefillQkvArgs qa{};
        qa.qkv = static_cast<float*>(qkv_.ptr);
        qa.q_norm = w.q_norm;
        qa.k_norm = w.k_norm;
        qa.rope = e.rope();
        qa.q_out_f32 = static_cast<float*>(q32_.ptr);
        qa.k_cache = e.k_layer(l);
        qa.v_cache = e.v_layer(l);
        qa.page_table = e.page_table();
        qa.rows = 1;
        qa.n_heads = hq_;
        qa.n_kv = hkv_;
        qa.eps = c.norm_eps;
        qa.dec_pos = static_cast<const int32_t*>(pos_.ptr);
        qa.pages_per_seq = e.n_pages();
        qa.kv_head0 = rank_ * hkv_;
        qa.n_kv_cache = c.n_kv_heads;
        qa.clear_input = 1;
        launch_prefill_qkv(qa, s_);
        DecodeAttnArgs da{};
        da.q = static_cast<const float*>(q32_.ptr);
        da.q_stride = hq_ * HD;
        da.k_cache = e.k_layer(l);
        da.v_cache = e.v_layer(l);
        da.page_table = e.page_table();
        da.pages_per_seq = e.n_pages();
        da.dec_pos = static_cast<const int32_t*>(pos_.ptr);
        da.rows = 1;
        da.n_kv = hkv_;
        da.kv_head0 = rank_ * hkv_;
        da.n_kv_cache = c.n_kv_heads;
        da.pages_per_split = attn_pps_;
        da.max_splits = attn_splits_;
        da.part_o = static_cast<float*>(part_o_.ptr);
        da.part_ml = static_cast<float2*>(part_ml_.ptr);
        da.counter = static_cast<unsigned*>(attn_counter_.ptr);
        da.out = static_cast<uint16_t*>(o_.ptr);
        da.out_lo = static_cast<uint16_t*>(o_lo_.ptr);
        da.out_stride = hq_ * HD;
        launch_decode_attention(da, s_);
        gemm(a_o_, a_o_lo_, wm.wo, o_part_, c.dim, hq_ * HD, kEpiAddF32);
        tp_allreduce_norm_kernel<<<1, 256, 0, s_>>>(P, static_cast<float*>(part_.ptr), X, rank_,
                                                    world_, counter, err, kBudget, w.mlp_norm,
                                                    c.norm_eps, Xn, Xn_lo);
        Q3_CUDA(cudaGetLastError());
        gemm(a_xn_, a_xn_lo_, wm.w13, o_gu_, 2 * hl_, c.dim, kEpiAddF32);
        tp_swiglu_kernel<<<std::max(1, hl_ / 256), 128, 0, s_>>>(
            static_cast<float*>(gu_.ptr), static_cast<uint16_t*>(h_.ptr),
            static_cast<uint16_t*>(h_lo_.ptr), hl_);
        Q3_CUDA(cudaGetLastError());
        gemm(a_h_, a_h_lo_, wm.w2, o_part_, c.dim, hl_, kEpiAddF32);
        const uint16_t* next_norm = l + 1 < c.n_layers ? m_.layer(l + 1).attn_norm : m_.final_norm();
        tp_allreduce_norm_kernel<<<1, 256, 0, s_>>>(P, static_cast<float*>(part_.ptr), X, rank_,
                                                    world_, counter, err, kBudget, next_norm,
                                                    c.norm_eps, Xn, Xn_lo);
        Q3_CUDA(cudaGetLastError());
    }
    gemm(a_xn_, a_xn_lo_, lm_, o_logits_, vn_, c.dim, kEpiStoreF32);
    tp_argmax_kernel<<<1, 1024, 0, s_>>>(
        P, static_cast<const float*>(logits_.ptr), vn_, v0_, rank_, world_, counter, err, kBudget,
        static_cast<int32_t*>(tok_.ptr), static_cast<int32_t*>(pos_.ptr),
        static_cast<int32_t*>(log_.ptr), static_cast<int32_t*>(step_.ptr),
        forced ? static_cast<const int32_t*>(forced_.ptr) : nullptr);
    Q3_CUDA(cudaGetLastError());
}

void TpDecoder::decode(int32_t first, int pos0, int n_steps, const int32_t* forced_host,
                       int32_t* tokens_host) {
    const q3_config& c = cfg_;
    if (!connected_ && world_ > 1) throw std::runtime_error("tensor parallelism: not connected");
    if (world_ == 1 && !connected_) {
        peer_mapped_.assign(1, nullptr);
        connected_ = true;
    }
    if (n_steps <= 0) return;
    if (pos0 < 0 || pos0 + n_steps > c.max_seq_len) {
        throw std::out_of_range("tensor-parallel decode stays below the context length");
    }
    const int32_t t0 = forced_host ? forced_host[0] : first;
    if (t0 < 0 || t0 >= c.vocab_size) throw std::out_of_range("Token id is outside the vocabulary");
    if (forced_host) {
        for (int i = 0; i < n_steps; ++i) {
            if (forced_host[i] < 0 || forced_host[i] >= c.vocab_size) {
                throw std::out_of_range("Token id is outside the vocabulary");
            }
        }
    }
    if (log_cap_ < n_steps) {
        log_.alloc(static_cast<size_t>(n_steps) * 4);
        forced_.alloc(static_cast<size_t>(n_steps) * 4);
        log_cap_ = n_steps;
        if (graph_) {
            cudaGraphExecDestroy(graph_);
            graph_ = nullptr;
        }
    }
    m_.engine().ensure_rope(pos0 + n_steps + 1);
    Q3_CUDA(cudaStreamSynchronize(m_.engine().stream()));
    const int32_t state[2] = {0, forced_host ? n_steps : 0};
    Q3_CUDA(cudaMemcpyAsync(pos_.ptr, &pos0, 4, cudaMemcpyHostToDevice, s_));
    Q3_CUDA(cudaMemcpyAsync(tok_.ptr, &t0, 4, cudaMemcpyHostToDevice, s_));
    Q3_CUDA(cudaMemcpyAsync(step_.ptr, state, sizeof(state), cudaMemcpyHostToDevice, s_));
    if (forced_host) {
        Q3_CUDA(cudaMemcpyAsync(forced_.ptr, forced_host, static_cast<size_t>(n_steps) * 4,
                                cudaMemcpyHostToDevice, s_));
    }
    const bool forced = forced_host != nullptr;
    if (graph_rope_ != m_.engine().rope()) {  // the graph holds the RoPE table's address
        if (graph_) cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
    if (!graph_ || graph_forced_ != forced) {
        if (graph_) cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
        cudaGraph_t g = nullptr;
        Q3_CUDA(cudaStreamBeginCapture(s_, cudaStreamCaptureModeThreadLocal));
        try {
            enqueue_step(forced);
        } catch (...) {
            cudaStreamEndCapture(s_, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        Q3_CUDA(cudaStreamEndCapture(s_, &g));
        const cudaError_t ie = cudaGraphInstantiate(&graph_, g, 0);
        cudaGraphDestroy(g);
        Q3_CUDA(ie);
        graph_forced_ = forced;
        graph_rope_ = m_.engine().rope();
    }
    for (int i = 0; i < n_steps; ++i) Q3_CUDA(cudaGraphLaunch(graph_, s_));
    if (tokens_host) {
        Q3_CUDA(cudaMemcpyAsync(tokens_host, log_.ptr, static_cast<size_t>(n_steps) * 4,
                                cudaMemcpyDeviceToHost, s_));
    }
    Q3_CUDA(cudaStreamSynchronize(s_));
    unsigned e = 0;
    Q3_CUDA(cudaMemcpy(&e, err_.ptr, 4, cudaMemcpyDeviceToHost));
    if (e) {
        Q3_CUDA(cudaMemset(err_.ptr, 0, 4));
        throw DeviceTimeout("tensor-parallel decode: a bounded wait gave up (code " +
                            std::to_string(e) + ")");
    }
}

}  // namespace q3
