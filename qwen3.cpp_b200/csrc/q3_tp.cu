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
#include <dlfcn.h>
#include <float.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

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
// Fused path: tagged words of the fused kernel's exchange (o_proj partials [8][1024], per-rank
// down-projection sums [2][8][1024], greedy candidates [8][2]).
constexpr size_t kFxOff = (kFlagOff + 256 + 255) / 256 * 256;
constexpr size_t kFxOpart = 0, kFxYx = 8 * 1024, kFxAmx = kFxYx + 2ull * kFusedMaxRanks * 1024;
constexpr size_t kXbufBytes = kFxOff + kFusedXchgWords * 8;
static_assert(kTpMaxRanks == kFusedMaxRanks, "one rank limit");

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

// Waits (bounded) until every source's flag in this rank's buffer reached seq. Threads
// [0, world) poll one source each; a poller also gives up as soon as another kernel of this
// rank has reported an error (so that one timeout does not make every later all-reduce of the
// step wait out its own budget). Returns false on timeout or error.
__device__ bool wait_flags(const uint8_t* own, int world, unsigned seq, long long budget,
                           const unsigned* err) {
    bool ok = true;
    if (static_cast<int>(threadIdx.x) < world) {
        const unsigned* f = reinterpret_cast<const unsigned*>(own + kFlagOff) + threadIdx.x;
        const long long t0 = clock64();
        for (unsigned it = 0; ld_acquire_sys(f) < seq; ++it) {
            if ((it & 63) == 63 && (*reinterpret_cast<const volatile unsigned*>(err) != 0u ||
                                    clock64() - t0 > budget)) {
                ok = false;
                break;
            }
        }
    }
    return __syncthreads_and(ok) != 0;
}

// True when an earlier kernel of this rank reported an error: the kernel then returns without
// touching the exchange buffers (its peers see no flag from it and give up in their turn).
__device__ __forceinline__ bool failed_before(const unsigned* err) {
    return *reinterpret_cast<const volatile unsigned*>(err) != 0u;
}

__device__ void raise_flags(const TpPeers& P, int world, int rank, unsigned seq) {
    if (static_cast<int>(threadIdx.x) < world) {
        st_release_sys(reinterpret_cast<unsigned*>(P.buf[threadIdx.x] + kFlagOff) + rank, seq);
    }
}

// x += sum over ranks of part, in rank order, so that x stays bit-identical on every rank (the
// residual adds x += proj of src/inference.cpp:847-849, 863-865). One block of 256 threads.
__global__ void __launch_bounds__(256) tp_allreduce_kernel(TpPeers P, const float* part, float* x,
                                                           int rank, int world, unsigned* counter,
                                                           unsigned* err, long long budget) {
    __shared__ unsigned s_seq;
    pdl_wait();
    pdl_trigger();
    if (failed_before(err)) return;
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
    // The flag stores are releases at system scope, ordered after every thread's data stores by
    // the barrier (release is cumulative).
    __syncthreads();
    raise_flags(P, world, rank, seq);
    if (!wait_flags(P.buf[rank], world, seq, budget, err)) {
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
    if (tid == 0) *counter = seq;
}

// NCCL comparison path: x += the all-reduced partial (one block of 256 threads).
__global__ void __launch_bounds__(256) tp_add_kernel(float* x, const float* sum) {
    pdl_wait();
    pdl_trigger();
    const int i = threadIdx.x * 4;
    float4 xv = *reinterpret_cast<float4*>(x + i);
    const float4 v = *reinterpret_cast<const float4*>(sum + i);
    xv.x += v.x;
    xv.y += v.y;
    xv.z += v.z;
    xv.w += v.w;
    *reinterpret_cast<float4*>(x + i) = xv;
}

// Block argmax of logits[0, vn) (lowest index on ties); valid in thread 0.
__device__ void block_argmax(const float* logits, int vn, float& best_out, int& idx_out) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int tid = threadIdx.x;
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
    if (tid == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) {
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
                best = bv[w];
                idx = bi[w];
            }
        }
    }
    best_out = best;
    idx_out = idx;
}

// NCCL comparison path, first half of the greedy step: this rank's (value, global index).
__global__ void __launch_bounds__(1024) tp_argmax_local_kernel(const float* logits, int vn, int v0,
                                                                float2* out) {
    pdl_wait();
    pdl_trigger();
    float b;
    int i;
    block_argmax(logits, vn, b, i);
    if (threadIdx.x == 0) *out = make_float2(b, __int_as_float(i + v0));
}

// Second half, after the all-gather of every rank's pair: the greedy token (lowest index on
// ties), then log[step] = token, the next token (argmax or forced), position + 1, step + 1.
__global__ void tp_argmax_final_kernel(const float2* am, int world, int32_t* tok, int32_t* pos,
                                       int32_t* log, int32_t* state, const int32_t* forced) {
    pdl_wait();
    pdl_trigger();
    float b = am[0].x;
    int bi0 = __float_as_int(am[0].y);
    for (int s = 1; s < world; ++s) {
        const int si = __float_as_int(am[s].y);
        if (am[s].x > b || (am[s].x == b && si < bi0)) {
            b = am[s].x;
            bi0 = si;
        }
    }
    const int step = state[0];
    log[step] = bi0;
    tok[0] = (forced && step + 1 < state[1]) ? forced[step + 1] : bi0;
    pos[0] += 1;
    state[0] = step + 1;
}

// NCCL entry points, resolved at run time from the process's libnccl.so.2 (the copy PyTorch
// loaded, else the system one), so that the library needs NCCL only when this path is used.
struct NcclApi {
    decltype(&ncclGetUniqueId) get_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

const NcclApi& nccl() {
    static const NcclApi api = [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
        if (!h) throw std::runtime_error("tensor parallelism: NCCL (libnccl.so.2) is not available");
        NcclApi a;
        auto sym = [&](const char* name) {
            void* f = dlsym(h, name);
            if (!f) throw std::runtime_error(std::string("tensor parallelism: NCCL lacks ") + name);
            return f;
        };
        a.get_id = reinterpret_cast<decltype(a.get_id)>(sym("ncclGetUniqueId"));
        a.init_rank = reinterpret_cast<decltype(a.init_rank)>(sym("ncclCommInitRank"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(sym("ncclAllReduce"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(sym("ncclAllGather"));
        a.destroy = reinterpret_cast<decltype(a.destroy)>(sym("ncclCommDestroy"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(sym("ncclGetErrorString"));
        return a;
    }();
    return api;
}

void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) {
        throw std::runtime_error(std::string("tensor parallelism: ") + what + ": " +
                                 nccl().error_string(r));
    }
}

// Greedy argmax over this rank's vocabulary rows, all-reduced (lowest index wins ties,
// src/inference.cpp:703-709); then log[step] = token, the next token (argmax or forced),
// position + 1, step + 1. state = {step, n_forced}. One block of 1024 threads.
__global__ void __launch_bounds__(1024) tp_argmax_kernel(
    TpPeers P, const float* logits, int vn, int v0, int rank, int world, unsigned* counter,
    unsigned* err, long long budget, int32_t* tok, int32_t* pos, int32_t* log, int32_t* state,
    const int32_t* forced) {
    pdl_wait();
    pdl_trigger();
    if (failed_before(err)) return;
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
    }
    __syncthreads();  // the flag releases below are ordered after thread 0's stores
    raise_flags(P, world, rank, seq);
    if (!wait_flags(P.buf[rank], world, seq, budget, err)) {
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
    const size_t qc = static_cast<size_t>(hq_) * HD;  // local attention-output columns
    // Per layer, contiguous: [wq;wk;wv] rows of the local heads, [w1;w3] rows of the local MLP
    // slice, and the column slices wo[:, local q columns], w2[:, local MLP columns].
    const size_t shard_layer = (qkv_l + 2 * static_cast<size_t>(hl_)) * D + D * qc + D * hl_;
    shard_.alloc(shard_layer * c.n_layers * 2);
    layers_.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& w = model.layer(l);
        uint16_t* sq = static_cast<uint16_t*>(shard_.ptr) + shard_layer * l;
        uint16_t* s13 = sq + qkv_l * D;
        uint16_t* so = s13 + 2 * static_cast<size_t>(hl_) * D;
        uint16_t* s2 = so + D * qc;
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
        Q3_CUDA(cudaMemcpy2DAsync(so, qc * 2, w.wo + static_cast<size_t>(rank) * qc, qd * 2,
                                  qc * 2, D, cudaMemcpyDeviceToDevice, s_));
        Q3_CUDA(cudaMemcpy2DAsync(s2, static_cast<size_t>(hl_) * 2,
                                  w.w2 + static_cast<size_t>(rank) * hl_,
                                  static_cast<size_t>(c.hidden_dim) * 2,
                                  static_cast<size_t>(hl_) * 2, D, cudaMemcpyDeviceToDevice, s_));
        layers_[l] = ShardLayer{sq, s13, s13 + static_cast<size_t>(hl_) * D, so, s2};
    }

    x_.alloc(D * 4);
    qkv_.alloc(qkv_l * 4);
    q32_.alloc(qc * 4);
    o32_.alloc(qc * 4);
    part_.alloc(D * 4);
    h32_.alloc(static_cast<size_t>(hl_) * 4);
    scratch_.alloc(D * 2);
    logits_.alloc(static_cast<size_t>(vn_) * 4);
    pos_.alloc(4);
    tok_.alloc(4);
    step_.alloc(8);
    err_.alloc(4);
    counter_.alloc(4);
    xbuf_.alloc(kXbufBytes);
    for (DeviceBuffer* b : {&err_, &counter_, &xbuf_}) {
        Q3_CUDA(cudaMemsetAsync(b->ptr, 0, b->bytes, s_));
    }
    // Decode attention split over the cached pages of the local KV heads.
    Q3_CUDA(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, model.device()));
    const int max_pages = model.engine().n_pages();
    attn_pps_ = decode_attn_pages_per_split(1, hkv_, max_pages, sms_);
    attn_splits_ = (max_pages + attn_pps_ - 1) / attn_pps_;
    part_o_.alloc(static_cast<size_t>(hkv_) * attn_splits_ * 2 * HD * 4);
    part_ml_.alloc(static_cast<size_t>(hkv_) * attn_splits_ * 2 * sizeof(float2));
    attn_counter_.alloc(static_cast<size_t>(hkv_) * sizeof(unsigned));
    Q3_CUDA(cudaMemsetAsync(attn_counter_.ptr, 0, attn_counter_.bytes, s_));
    if (model.fused_available() && model.fused_grid() / hkv_ >= 1 &&
        hl_ <= 64 * model.fused_grid()) {
        setup_fused();
        fused_ = true;
    }
    Q3_CUDA(cudaStreamSynchronize(s_));
}

void TpDecoder::setup_fused() {
    const q3_config& c = cfg_;
    const size_t D = c.dim, qd = static_cast<size_t>(c.n_heads) * HD;
    const size_t kvd = static_cast<size_t>(c.n_kv_heads) * HD;
    const size_t qkv_l = static_cast<size_t>(hq_ + 2 * hkv_) * HD;
    f_grid_ = m_.fused_grid();
    f_smax_ = f_grid_ / hkv_;
    // Per layer: the local q, k and v rows of the fused kernel's swizzled [wq;wk;wv] copy (row
    // offsets are even, so every row keeps its parity swizzle), and pointers into its wop (by
    // global KV group), w1 / w3 / w2t (this rank's MLP indices) copies.
    const std::vector<FusedLayer>& fl = m_.fused_layers_host();
    f_wqkv_.alloc(qkv_l * D * 2 * c.n_layers);
    std::vector<FusedLayer> ll(c.n_layers);
    const size_t mlp0 = static_cast<size_t>(rank_) * hl_ * D;
    for (int l = 0; l < c.n_layers; ++l) {
        uint16_t* dst = static_cast<uint16_t*>(f_wqkv_.ptr) + qkv_l * D * l;
        const uint16_t* src = fl[l].wqkv;
        const size_t q0 = static_cast<size_t>(rank_) * hq_ * HD, k0 = static_cast<size_t>(rank_) * hkv_ * HD;
        Q3_CUDA(cudaMemcpyAsync(dst, src + q0 * D, static_cast<size_t>(hq_) * HD * D * 2,
                                cudaMemcpyDeviceToDevice, s_));
        Q3_CUDA(cudaMemcpyAsync(dst + static_cast<size_t>(hq_) * HD * D, src + (qd + k0) * D,
                                static_cast<size_t>(hkv_) * HD * D * 2, cudaMemcpyDeviceToDevice, s_));
        Q3_CUDA(cudaMemcpyAsync(dst + static_cast<size_t>(hq_ + hkv_) * HD * D,
                                src + (qd + kvd + k0) * D, static_cast<size_t>(hkv_) * HD * D * 2,
                                cudaMemcpyDeviceToDevice, s_));
        ll[l] = fl[l];
        ll[l].wqkv = dst;
        ll[l].w1 = fl[l].w1 + mlp0;
        ll[l].w3 = fl[l].w3 + mlp0;
        ll[l].w2t = fl[l].w2t + mlp0;
    }
    f_layers_.alloc(ll.size() * sizeof(FusedLayer));
    Q3_CUDA(cudaMemcpyAsync(f_layers_.ptr, ll.data(), f_layers_.bytes, cudaMemcpyHostToDevice, s_));
    f_y_.alloc(fused_ybuf_floats(c.n_layers) * 4);
    f_qkvt_.alloc(qkv_l * 8);
    f_part_o_.alloc(static_cast<size_t>(hq_) * f_smax_ * HD * 4);
    f_part_ml_.alloc(static_cast<size_t>(hq_) * f_smax_ * sizeof(float2));
    f_am_.alloc(static_cast<size_t>(f_grid_) * sizeof(float2));
    f_sync_.alloc(256);
    f_sp_.alloc(sizeof(StepParams));
    for (DeviceBuffer* b : {&f_y_, &f_qkvt_, &f_sync_}) {
        Q3_CUDA(cudaMemsetAsync(b->ptr, 0, b->bytes, s_));
    }
    Q3_CUDA(cudaStreamSynchronize(s_));  // the host copy of the layer pointers goes out of scope
}

void TpDecoder::set_path(int path) {
    if (path == Q3_TP_FUSED && !fused_available()) {
        throw std::invalid_argument("tensor parallelism: the fused decode kernel is not available");
    }
    if (path == Q3_TP_GRAPH_NCCL && !nccl_comm_) {
        throw std::invalid_argument("tensor parallelism: connect NCCL first (q3_tp_nccl_connect)");
    }
    if (path != Q3_TP_FUSED && path != Q3_TP_GRAPH && path != Q3_TP_GRAPH_NCCL) {
        throw std::invalid_argument("unknown tensor-parallel path");
    }
    const bool nccl_on = path == Q3_TP_GRAPH_NCCL;
    if (nccl_on != use_nccl_ && graph_) {  // the captured step holds the collective calls
        cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
    fused_ = path == Q3_TP_FUSED;
    use_nccl_ = nccl_on;
}

int TpDecoder::path() const {
    return fused_ ? Q3_TP_FUSED : (use_nccl_ ? Q3_TP_GRAPH_NCCL : Q3_TP_GRAPH);
}

void TpDecoder::nccl_unique_id(void* out) {
    ncclUniqueId id;
    nccl_check(nccl().get_id(&id), "ncclGetUniqueId");
    std::memcpy(out, &id, sizeof(id));
}

void TpDecoder::nccl_connect(const void* id) {
    if (nccl_comm_) throw std::runtime_error("tensor parallelism: NCCL already connected");
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    Q3_CUDA(cudaSetDevice(m_.device()));
    ncclComm_t comm = nullptr;
    nccl_check(nccl().init_rank(&comm, world_, uid, rank_), "ncclCommInitRank");
    nccl_comm_ = comm;
    am_nccl_.alloc(static_cast<size_t>(1 + world_) * sizeof(float2));
}

void TpDecoder::launch_fused(int n_steps, bool forced) {
    const q3_config& c = cfg_;
    Engine& e = m_.engine();
    FusedArgs a{};
    a.layers = static_cast<const FusedLayer*>(f_layers_.ptr);
    a.embed = m_.embed();
    a.lm_head = m_.fused_lm() + static_cast<size_t>(v0_) * c.dim;
    a.final_norm = m_.final_norm();
    a.k_cache = e.k_layer(0);
    a.v_cache = e.v_layer(0);
    a.layer_elems = e.layer_elems();
    a.page_table = e.page_table();
    a.rope = e.rope();
    a.rope_len = e.rope_len();
    a.ybuf = static_cast<float*>(f_y_.ptr);
    a.parity0 = f_parity_;
    f_parity_ = (f_parity_ + n_steps) & 1;
    a.qkvt = static_cast<unsigned long long*>(f_qkvt_.ptr);
    f_epoch_ = (f_epoch_ + 1) & 0xFFFu;
    if (f_epoch_ == 0) f_epoch_ = 1;
    a.epoch = f_epoch_;
    a.part_o = static_cast<float*>(f_part_o_.ptr);
    a.part_ml = static_cast<float2*>(f_part_ml_.ptr);
    a.am_part = static_cast<float2*>(f_am_.ptr);
    a.logits = static_cast<float*>(logits_.ptr);
    a.taps = nullptr;
    a.sp = static_cast<StepParams*>(f_sp_.ptr);
    a.token_log = static_cast<int32_t*>(log_.ptr);
    a.forced = forced ? static_cast<const int32_t*>(forced_.ptr) : nullptr;
    a.bar = static_cast<unsigned*>(f_sync_.ptr);
    a.err = static_cast<unsigned*>(err_.ptr);
    a.n_layers = c.n_layers;
    a.vocab = vn_;
    a.ctx = c.max_seq_len;
    a.n_steps = n_steps;
    a.s_max = f_smax_;
    a.eps = c.norm_eps;
    a.spin_cycles = wait_cycles_;
    a.l2_ahead = fused_l2_ahead();
    a.nkv = hkv_;
    a.kv0 = rank_ * hkv_;
    a.hl = hl_;
    a.v0 = v0_;
    a.world = world_;
    a.rank = rank_;
    a.xchg = (world_ > 1 || solo_allreduce_) ? 1 : 0;
    a.sys = world_ > 1 ? 1 : 0;
    auto* own = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(xbuf_.ptr) + kFxOff);
    a.opart = own + kFxOpart;
    a.yx = own + kFxYx;
    a.amx = own + kFxAmx;
    for (int p = 0; p < world_; ++p) {
        const bool mine = p == rank_ || (p < static_cast<int>(self_peer_.size()) && self_peer_[p]);
        auto* base = mine ? own
                          : reinterpret_cast<unsigned long long*>(
                                static_cast<uint8_t*>(peer_mapped_[p]) + kFxOff);
        a.opart_dst[p] = base + kFxOpart;
        a.yx_dst[p] = base + kFxYx;
        a.amx_dst[p] = base + kFxAmx;
    }
    launch_decode_fused(a, f_grid_, s_);
}

TpDecoder::~TpDecoder() {
    if (graph_) cudaGraphExecDestroy(graph_);  // before the communicator its NCCL calls use
    if (nccl_comm_) nccl().destroy(static_cast<ncclComm_t>(nccl_comm_));
    for (void* p : peer_mapped_) {
        if (p) cudaIpcCloseMemHandle(p);
    }
    if (s_) cudaStreamDestroy(s_);
}

void TpDecoder::configure(bool solo_allreduce, long long wait_cycles) {
    if (wait_cycles <= 0) throw std::invalid_argument("tensor parallelism: wait budget must be > 0");
    solo_allreduce_ = solo_allreduce;
    wait_cycles_ = wait_cycles;
    if (graph_) cudaGraphExecDestroy(graph_);  // the captured step holds both
    graph_ = nullptr;
}

void TpDecoder::reset() {
    // Invocation counter, error word, exchange data and flags back to zero: every rank resets
    // (and the ranks meet on the host) before any of them decodes again.
    Q3_CUDA(cudaStreamSynchronize(s_));
    for (DeviceBuffer* b : {&err_, &counter_, &xbuf_, &f_y_, &f_qkvt_, &f_sync_}) {
        if (b->ptr) Q3_CUDA(cudaMemsetAsync(b->ptr, 0, b->bytes, s_));
    }
    Q3_CUDA(cudaStreamSynchronize(s_));
    f_epoch_ = 0;
    f_parity_ = 0;
    failed_ = false;
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
    self_peer_.assign(world_, 0);
    uint8_t own[64];
    ipc_handle(own);
    const auto* hs = static_cast<const uint8_t*>(handles);
    for (int p = 0; p < world_; ++p) {
        if (p == rank_) continue;
        if (std::memcmp(hs + 64 * p, own, 64) == 0) {
            // This rank's own buffer given as a peer's (a process cannot open its own IPC
            // handle): used as is. Nothing raises that peer's flag, so every all-reduce of such
            // a decoder ends in the bounded wait's timeout - the form the timeout test uses.
            self_peer_[p] = 1;
            continue;
        }
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
    const int qkv_l = (hq_ + 2 * hkv_) * HD, qc = hq_ * HD;
    unsigned* err = static_cast<unsigned*>(err_.ptr);
    unsigned* counter = static_cast<unsigned*>(counter_.ptr);
    TpPeers P{};
    for (int p = 0; p < world_; ++p) {
        const bool own = p == rank_ || (p < static_cast<int>(self_peer_.size()) && self_peer_[p]);
        P.buf[p] = static_cast<uint8_t*>(own ? xbuf_.ptr : peer_mapped_[p]);
    }
    const long long kBudget = wait_cycles_;
    float* X = static_cast<float*>(x_.ptr);
    float* qkv = static_cast<float*>(qkv_.ptr);
    float* part = static_cast<float*>(part_.ptr);
    Engine& e = m_.engine();
    // One rank: the projections add straight into x, unless configured to route them through
    // the all-reduce kernel with this rank as its only member. Several: each writes its partial,
    // and the all-reduce adds the ranks' partials in rank order.
    const bool solo = world_ == 1 && !solo_allreduce_ && !use_nccl_;
    const int proj_epi = solo ? kEpiResidual : kEpiStore;
    float* proj_out = solo ? X : part;
    auto allreduce = [&]() {
        if (solo) return;
        if (use_nccl_) {
            // Comparison arm: NCCL sums the partials in place, then x += sum.
            nccl_check(nccl().all_reduce(part, part, c.dim, ncclFloat32, ncclSum,
                                         static_cast<ncclComm_t>(nccl_comm_), s_),
                       "ncclAllReduce");
            launch_dep(false, tp_add_kernel, dim3(1), dim3(256), 0, s_, X,
                       static_cast<const float*>(part));
        } else {
            launch_dep(false, tp_allreduce_kernel, dim3(1), dim3(256), 0, s_, P,
                       static_cast<const float*>(part), X, rank_, world_, counter, err, kBudget);
        }
        Q3_CUDA(cudaGetLastError());
    };
    // x = embedding row of the step's token (the bf16 normalised copy is not used).
    launch_rmsnorm_rows_bf16(static_cast<const int32_t*>(tok_.ptr), m_.embed(), X,
                             m_.layer(0).attn_norm, c.norm_eps,
                             static_cast<uint16_t*>(scratch_.ptr), 1, c.dim, s_);
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& w = m_.layer(l);
        const ShardLayer& sl = layers_[l];
        // q|k|v of the local heads = [wq;wk;wv]_local . RmsNorm(x) (src/inference.cpp:795-798).
        launch_gemv(kEpiStore, sl.wqkv, nullptr, X, w.attn_norm, c.norm_eps, qkv, nullptr, qkv_l,
                    c.dim, nullptr, 0, s_);
        PrefillQkvArgs qa{};
        qa.qkv = qkv;
        qa.q_norm = w.q_norm;
        qa.k_norm = w.k_norm;
        qa.rope = e.rope();
        qa.q_out = nullptr;
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
        launch_prefill_qkv(qa, s_);
        DecodeAttnArgs da{};
        da.q = static_cast<const float*>(q32_.ptr);
        da.q_stride = qc;
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
        da.out_f32 = static_cast<float*>(o32_.ptr);
        da.out_stride = qc;
        launch_decode_attention(da, s_);
        // x += wo[:, local] . attn_local summed over ranks (:846-849).
        launch_gemv(proj_epi, sl.wo, nullptr, static_cast<const float*>(o32_.ptr), nullptr, 0.0f,
                    proj_out, nullptr, c.dim, qc, nullptr, 0, s_);
        allreduce();
        // h = silu(w1 . xn) * (w3 . xn) on the local MLP slice, x += w2[:, local] . h (:851-865).
        launch_gemv(kEpiSiluMul, sl.w1, sl.w3, X, w.mlp_norm, c.norm_eps,
                    static_cast<float*>(h32_.ptr), nullptr, hl_, c.dim, nullptr, 0, s_);
        launch_gemv(proj_epi, sl.w2, nullptr, static_cast<const float*>(h32_.ptr), nullptr, 0.0f,
                    proj_out, nullptr, c.dim, hl_, nullptr, 0, s_);
        allreduce();
    }
    // Final RmsNorm + this rank's slice of the tied lm_head, then the all-reduced argmax.
    launch_gemv(kEpiStore, m_.output() + static_cast<size_t>(v0_) * c.dim, nullptr, X,
                m_.final_norm(), c.norm_eps, static_cast<float*>(logits_.ptr), nullptr, vn_, c.dim,
                nullptr, 0, s_);
    if (use_nccl_) {
        float2* am = static_cast<float2*>(am_nccl_.ptr);
        launch_dep(false, tp_argmax_local_kernel, dim3(1), dim3(1024), 0, s_,
                   static_cast<const float*>(logits_.ptr), vn_, v0_, am);
        nccl_check(nccl().all_gather(am, am + 1, 2, ncclFloat32,
                                     static_cast<ncclComm_t>(nccl_comm_), s_),
                   "ncclAllGather");
        launch_dep(false, tp_argmax_final_kernel, dim3(1), dim3(1), 0, s_,
                   static_cast<const float2*>(am + 1), world_, static_cast<int32_t*>(tok_.ptr),
                   static_cast<int32_t*>(pos_.ptr), static_cast<int32_t*>(log_.ptr),
                   static_cast<int32_t*>(step_.ptr),
                   forced ? static_cast<const int32_t*>(forced_.ptr) : nullptr);
    } else {
        launch_dep(false, tp_argmax_kernel, dim3(1), dim3(1024), 0, s_, P,
                   static_cast<const float*>(logits_.ptr), vn_, v0_, rank_, world_, counter, err,
                   kBudget, static_cast<int32_t*>(tok_.ptr), static_cast<int32_t*>(pos_.ptr),
                   static_cast<int32_t*>(log_.ptr), static_cast<int32_t*>(step_.ptr),
                   forced ? static_cast<const int32_t*>(forced_.ptr) : nullptr);
    }
    Q3_CUDA(cudaGetLastError());
}

void TpDecoder::decode(int32_t first, int pos0, int n_steps, const int32_t* forced_host,
                       int32_t* tokens_host) {
    const q3_config& c = cfg_;
    if (failed_) {
        throw std::runtime_error("tensor-parallel decode: an earlier step timed out; every rank "
                                 "must reset the decoder before decoding again");
    }
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
    if (fused_) {
        StepParams sp{};
        sp.token = t0;
        sp.pos = pos0;
        step_positions(pos0, c.max_seq_len, &sp.num_sink, &sp.kv_pos, &sp.kv_len);
        sp.step = 0;
        sp.n_forced = forced ? n_steps : 0;
        Q3_CUDA(cudaMemcpyAsync(f_sp_.ptr, &sp, sizeof(sp), cudaMemcpyHostToDevice, s_));
        constexpr int kMaxStepsPerLaunch = 256;
        for (int done = 0; done < n_steps; done += kMaxStepsPerLaunch) {
            launch_fused(std::min(kMaxStepsPerLaunch, n_steps - done), forced);
        }
    } else {
        run_graph(forced, n_steps);
    }
    if (tokens_host) {
        Q3_CUDA(cudaMemcpyAsync(tokens_host, log_.ptr, static_cast<size_t>(n_steps) * 4,
                                cudaMemcpyDeviceToHost, s_));
    }
    Q3_CUDA(cudaStreamSynchronize(s_));
    unsigned e = 0;
    Q3_CUDA(cudaMemcpy(&e, err_.ptr, 4, cudaMemcpyDeviceToHost));
    if (e) {
        // The ranks' invocation counters (graph) or the kernel's arrival counter and exchange
        // words (fused) may now disagree: refuse further steps until reset.
        failed_ = true;
        throw DeviceTimeout("tensor-parallel decode: a bounded wait gave up (code " +
                            std::to_string(e) + ")");
    }
}

void TpDecoder::run_graph(bool forced, int n_steps) {
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
}

}  // namespace q3
