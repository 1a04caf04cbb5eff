// Batched decode of independent sequences (see q3_batch.cuh).
//
// One decode step for B sequences, all on the GPU and captured as one CUDA graph:
//   embedding rows of the B current tokens + RmsNorm -> bf16 operand
//   per layer: [wq;wk;wv] contraction (M = B, split K, reduce-added into a zeroed buffer),
//              per-row QK-norm + RoPE + K/V write at each sequence's own position and pages,
//              decode attention per (sequence, KV head) over that sequence's pages (CUDA cores),
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
// hi + lo pair; gu is zeroed behind the reads for the next step's split-K reduce-add.
__global__ void swiglu_rows_kernel(float* __restrict__ gu, uint16_t* __restrict__ h,
                                   uint16_t* __restrict__ h_lo, int rows, int H) {
    pdl_wait();
    pdl_trigger();
    const size_t n = static_cast<size_t>(rows) * H / 4;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = (i * 4) / H, c = (i * 4) % H;
        const float4 g = *reinterpret_cast<const float4*>(gu + r * 2 * H + c);
        const float4 u = *reinterpret_cast<const float4*>(gu + r * 2 * H + H + c);
        *reinterpret_cast<float4*>(gu + r * 2 * H + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(gu + r * 2 * H + H + c) = make_float4(0.f, 0.f, 0.f, 0.f);
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
// position + 1. state = {step, n_forced}. Block (b, s) takes slice s of the row's kArgmaxSlices
// and leaves its best (value, index) in part[b][s]; the last block of the row to finish (counter[b],
// reset by it) reduces the slices in order.
constexpr int kArgmaxSlices = 32;
constexpr int kArgmaxThreads = 256;

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(kArgmaxThreads)
    batch_argmax_kernel(const float* __restrict__ logits, int rows, int V, int32_t* tok,
                        int32_t* pos, int32_t* log, const int32_t* state, const int32_t* forced,
                        float2* part, unsigned* counter) {
    pdl_wait();
    pdl_trigger();
    __shared__ float bv[kArgmaxThreads / 32];
    __shared__ int bi[kArgmaxThreads / 32];
    __shared__ int last;
    const int b = blockIdx.x, sl = blockIdx.y;
    const int per = (V + kArgmaxSlices - 1) / kArgmaxSlices;
    const int i0 = sl * per, i1 = min(V, i0 + per);
    const float* row = logits + static_cast<size_t>(b) * V;
    float best = -INFINITY;
    int idx = INT_MAX;
    for (int i = i0 + threadIdx.x; i < i1; i += kArgmaxThreads) {
        const float v = row[i];
        if (arg_better(v, i, best, idx)) {
            best = v;
            idx = i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (arg_better(ov, oi, best, idx)) {
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
        for (int w = 1; w < kArgmaxThreads / 32; ++w) {
            if (arg_better(bv[w], bi[w], best, idx)) {
                best = bv[w];
                idx = bi[w];
            }
        }
        part[b * kArgmaxSlices + sl] = make_float2(best, __int_as_float(idx));
        __threadfence();
        last = atomicAdd(counter + b, 1u) == kArgmaxSlices - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    best = -INFINITY;
    idx = INT_MAX;
    for (int k = 0; k < kArgmaxSlices; ++k) {
        const float2 p = __ldcg(part + b * kArgmaxSlices + k);
        const int pi = __float_as_int(p.y);
        if (arg_better(p.x, pi, best, idx)) {
            best = p.x;
            idx = pi;
        }
    }
    counter[b] = 0u;
    const int step = state[0], n_forced = state[1];
    log[static_cast<size_t>(step) * rows + b] = idx;
    tok[b] = (forced && step + 1 < n_forced) ? forced[static_cast<size_t>(step + 1) * rows + b]
                                             : idx;
    pos[b] += 1;
}

__global__ void advance_step_kernel(int32_t* state) {
    pdl_wait();
    pdl_trigger();
    state[0] += 1;
}

// ------------------------------------------------------------------ small-batch GEMV

// Batches of at most kSmallRows sequences run their weight products on the CUDA cores: at a few
// rows a tensor-core tile is mostly padding and its launch and pipeline latency dominate, while
// a GEMV over M activation rows streams each weight once and does M fp32 FMAs with it (the
// reference's MatMul, src/inference.cpp:952-966, for every sequence: fp32 activations, bf16
// weights, fp32 accumulation).
//
// out[m][n] (+)= sum_k W[n][k] * xs[m][k] for m < M rows of x (row stride ldx). Block: 4 warps,
// one task of GR rows of W at a time, warp w taking the k-quarter [w K/4, (w+1) K/4); lane l the
// 16-byte units l + 32 j of that quarter. NORM: xs = RmsNorm(x) with weights nw (:887-923).
// SWIGLU: rows 0..GR/2-1 of a task come from W (w1), GR/2..GR-1 from Wb (w3) at the same output
// indices, out = silu(gate) * up (:1009-1011). RESID: out += (the residual adds :847-849,
// :863-865).
constexpr int kSmallRows = 16;
constexpr int kGvWarps = 4;
constexpr int kGvVals = 64;  // accumulators per lane: GR rows x MR activation rows

template <int MR, bool NORM, bool SWIGLU, bool RESID>
__global__ void __launch_bounds__(kGvWarps * 32)
    gemv_rows_kernel(const uint16_t* __restrict__ W, const uint16_t* __restrict__ Wb,
                     const float* __restrict__ x, int ldx, const uint16_t* __restrict__ nw,
                     float eps, float* __restrict__ out, int ldo, int M, int N, int K) {
    constexpr int GR = kGvVals / MR;               // weight rows per task
    constexpr int NOUT = SWIGLU ? GR / 2 : GR;     // outputs per task
    extern __shared__ float4 gv_smem[];
    float* xs = reinterpret_cast<float*>(gv_smem);               // [MR][K]
    float* red = xs + static_cast<size_t>(MR) * K;               // [kGvWarps][kGvVals]
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kq = K / kGvWarps;            // this warp's k-quarter
    const int k0 = warp * kq;
    const int ntask = (N + NOUT - 1) / NOUT;
    const int nc = kq / 256;                // 16-byte column steps of a task per lane
    // The weights of step (task, column step) i + 1 are loaded while step i is multiplied.
    auto load_w = [&](int task, int ci, uint4 (&w)[GR]) {
        const int n0 = task * NOUT, c = k0 + ci * 256 + lane * 8;
#pragma unroll
        for (int r = 0; r < GR; ++r) {
            const int rr = SWIGLU ? (r % NOUT) : r;
            const int n = min(n0 + rr, N - 1);  // rows past N repeat the last (not stored)
            const uint16_t* base = (SWIGLU && r >= NOUT) ? Wb : W;
            w[r] = ldg_stream(base + static_cast<size_t>(n) * K + c);
        }
    };
    uint4 wn[GR];
    // The first weights are on their way from HBM while the activations are staged.
    if (static_cast<int>(blockIdx.x) < ntask) load_w(blockIdx.x, 0, wn);
    // Stage the activation rows with asynchronous 16-byte copies, all in flight at once (zero
    // rows past M).
    for (int m = 0; m < MR; ++m) {
        for (int i = tid * 4; i < K; i += kGvWarps * 128) {
            float* dst = xs + static_cast<size_t>(m) * K + i;
            if (m < M) {
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                                 static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                             "l"(x + static_cast<size_t>(m) * ldx + i)
                             : "memory");
            } else {
                *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (NORM) {
        // Row m by warp m % kGvWarps: (x * (1 / rms)) * w, rms = sqrtf(ss / K + eps).
        for (int m = warp; m < M; m += kGvWarps) {
            float* xr = xs + static_cast<size_t>(m) * K;
            float ss = 0.0f;
            for (int i = lane * 4; i < K; i += 128) {
                const float4 v = *reinterpret_cast<const float4*>(xr + i);
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
            }
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
            for (int i = lane * 4; i < K; i += 128) {
                const float4 v = *reinterpret_cast<const float4*>(xr + i);
                const uint2 wb = *reinterpret_cast<const uint2*>(nw + i);
                *reinterpret_cast<float4*>(xr + i) =
                    make_float4((v.x * inv) * bf16_lo(wb.x), (v.y * inv) * bf16_hi(wb.x),
                                (v.z * inv) * bf16_lo(wb.y), (v.w * inv) * bf16_hi(wb.y));
            }
        }
        __syncthreads();
    }
    for (int task = blockIdx.x; task < ntask; task += gridDim.x) {
        const int n0 = task * NOUT;
        float acc[kGvVals];
#pragma unroll
        for (int i = 0; i < kGvVals; ++i) acc[i] = 0.0f;
        for (int ci = 0; ci < nc; ++ci) {
            uint4 w[GR];
#pragma unroll
            for (int r = 0; r < GR; ++r) w[r] = wn[r];
            if (ci + 1 < nc) {
                load_w(task, ci + 1, wn);
            } else if (task + static_cast<int>(gridDim.x) < ntask) {
                load_w(task + gridDim.x, 0, wn);
            }
            const int c = k0 + ci * 256 + lane * 8;
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                const float4 a = *reinterpret_cast<const float4*>(xs + static_cast<size_t>(m) * K + c);
                const float4 b = *reinterpret_cast<const float4*>(xs + static_cast<size_t>(m) * K + c + 4);
#pragma unroll
                for (int r = 0; r < GR; ++r) acc[r * MR + m] = dot8(w[r], a, b, acc[r * MR + m]);
            }
        }
        // Transposing butterfly: after the xor 16 .. 1 rounds lane l holds the lane sums of
        // entries 2l and 2l + 1 (entry r * MR + m).
#pragma unroll
        for (int half = kGvVals / 2, off = 16; off >= 1; half >>= 1, off >>= 1) {
            const bool up = lane & off;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const float send = up ? acc[i] : acc[i + half];
                const float keep = up ? acc[i + half] : acc[i];
                acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
        *reinterpret_cast<float2*>(red + warp * kGvVals + 2 * lane) = make_float2(acc[0], acc[1]);
        __syncthreads();
        if (warp == 0) {
            float2 v = *reinterpret_cast<const float2*>(red + 2 * lane);
#pragma unroll
            for (int w2 = 1; w2 < kGvWarps; ++w2) {
                const float2 u = *reinterpret_cast<const float2*>(red + w2 * kGvVals + 2 * lane);
                v.x += u.x;
                v.y += u.y;
            }
            const float vv[2] = {v.x, v.y};
            float up[2] = {0.0f, 0.0f};
            if (SWIGLU) {
                // The up entries (rows NOUT..GR-1) sit NOUT * MR entries = 16 lanes further on.
                up[0] = __shfl_down_sync(0xffffffffu, v.x, NOUT * MR / 2);
                up[1] = __shfl_down_sync(0xffffffffu, v.y, NOUT * MR / 2);
            }
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int idx = 2 * lane + e, r = idx / MR, m = idx % MR;
                const int n = n0 + r;
                if (r >= NOUT || m >= M || n >= N) continue;
                float* o = out + static_cast<size_t>(m) * ldo + n;
                if (SWIGLU) {
                    const float g = vv[e];
                    *o = g / (1.0f + expf(-g)) * up[e];
                } else if (RESID) {
                    *o += vv[e];
                } else {
                    *o = vv[e];
                }
            }
        }
        __syncthreads();
    }
}

template <int MR, bool NORM, bool SWIGLU, bool RESID>
void gemv_rows_t(const uint16_t* W, const uint16_t* Wb, const float* x, int ldx, const uint16_t* nw,
                 float eps, float* out, int ldo, int M, int N, int K, int num_sms, cudaStream_t s) {
    auto fn = gemv_rows_kernel<MR, NORM, SWIGLU, RESID>;
    const size_t smem = (static_cast<size_t>(MR) * K + kGvWarps * kGvVals) * sizeof(float);
    static bool configured[64] = {};
    int dev = 0;
    Q3_CUDA(cudaGetDevice(&dev));
    if (!configured[dev & 63]) {
        Q3_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        configured[dev & 63] = true;
    }
    constexpr int NOUT = SWIGLU ? kGvVals / MR / 2 : kGvVals / MR;
    const int ntask = (N + NOUT - 1) / NOUT;
    // As many blocks as fit on the SMs at once (registers and shared memory), each streaming
    // several tasks.
    int per_sm = 1;
    Q3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kGvWarps * 32, smem));
    const int grid = std::min(ntask, num_sms * std::max(per_sm, 1));
    launch_dep(false, fn, dim3(grid), dim3(kGvWarps * 32), smem, s, W, Wb, x, ldx, nw, eps, out, ldo,
               M, N, K);
    Q3_CUDA(cudaGetLastError());
}

// out (+)= W . x (see gemv_rows_kernel) for M <= kSmallRows rows; K a multiple of 1024.
template <bool NORM, bool SWIGLU, bool RESID>
void gemv_rows(const uint16_t* W, const uint16_t* Wb, const float* x, int ldx, const uint16_t* nw,
               float eps, float* out, int ldo, int M, int N, int K, int num_sms, cudaStream_t s) {
    if (M <= 0 || M > kSmallRows || K % (kGvWarps * 256) != 0) {
        throw std::invalid_argument("small-batch GEMV: 1..16 rows, K a multiple of 1024");
    }
    if (M <= 8) {
        gemv_rows_t<8, NORM, SWIGLU, RESID>(W, Wb, x, ldx, nw, eps, out, ldo, M, N, K, num_sms, s);
    } else {
        gemv_rows_t<16, NORM, SWIGLU, RESID>(W, Wb, x, ldx, nw, eps, out, ldo, M, N, K, num_sms, s);
    }
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
    am_part_.alloc(static_cast<size_t>(B) * kArgmaxSlices * sizeof(float2));
    am_counter_.alloc(static_cast<size_t>(B) * sizeof(unsigned));
    Q3_CUDA(cudaMemset(am_counter_.ptr, 0, am_counter_.bytes));
    if (small_path()) {
        // The small-batch GEMV path's fp32 operands: attention output and SwiGLU output.
        o32_.alloc(static_cast<size_t>(B) * qd * 4);
        h32_.alloc(static_cast<size_t>(B) * H * 4);
    }
    // The split-K contractions reduce-add into qkv and gu; their readers (the QK-norm/RoPE kernel,
    // the SwiGLU kernel) zero them behind their reads, so they start and end every step at zero.
    Q3_CUDA(cudaMemset(qkv_.ptr, 0, qkv_.bytes));
    Q3_CUDA(cudaMemset(gu_.ptr, 0, gu_.bytes));
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
    if (small_path()) {
        enqueue_small_layers();
    } else {
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& w = m_.layer(l);
        const LayerMaps& wm = wmaps_[l];
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
        qa.clear_input = 1;
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
        gemm(a_xn_, a_xn_lo_, wm.w13, o_gu_, 2 * H, c.dim, kEpiAddF32);
        const size_t quads = static_cast<size_t>(B) * H / 4;
        launch_dep(false, swiglu_rows_kernel,
                   dim3(static_cast<unsigned>(std::min<size_t>((quads + 255) / 256, 4096))), dim3(256),
                   0, s_, static_cast<float*>(gu_.ptr), static_cast<uint16_t*>(h_.ptr),
                   static_cast<uint16_t*>(h_lo_.ptr), B, H);
        Q3_CUDA(cudaGetLastError());
        gemm(a_h_, a_h_lo_, wm.w2, o_x_, c.dim, H, kEpiAddF32);
        const uint16_t* next_norm = l + 1 < c.n_layers ? m_.layer(l + 1).attn_norm : m_.final_norm();
        launch_rmsnorm_rows_bf16(nullptr, nullptr, X, next_norm, c.norm_eps, Xn, B, c.dim, s_,
                                 Xn_lo);
    }
    }
    // Tied lm_head for every row, argmax and the advance.
    if (small_path()) {
        // The lm_head stays a tensor-core contraction (151,936 rows: streaming-bound either way).
        launch_rmsnorm_rows_bf16(nullptr, nullptr, X, m_.final_norm(), c.norm_eps, Xn, B, c.dim, s_,
                                 Xn_lo);
    }
    gemm(a_xn_, a_xn_lo_, lm_, o_logits_, c.vocab_size, c.dim, kEpiStoreF32);
    launch_dep(false, batch_argmax_kernel, dim3(B, kArgmaxSlices), dim3(kArgmaxThreads), 0, s_,
               static_cast<const float*>(logits_.ptr), B, c.vocab_size,
               static_cast<int32_t*>(tok_.ptr), static_cast<int32_t*>(pos_.ptr),
               static_cast<int32_t*>(log_.ptr), static_cast<const int32_t*>(step_.ptr),
               forced ? static_cast<const int32_t*>(forced_.ptr) : nullptr,
               static_cast<float2*>(am_part_.ptr), static_cast<unsigned*>(am_counter_.ptr));
    Q3_CUDA(cudaGetLastError());
    launch_dep(false, advance_step_kernel, dim3(1), dim3(1), 0, s_, static_cast<int32_t*>(step_.ptr));
    Q3_CUDA(cudaGetLastError());
    (void)n_forced;
}

bool Batch::small_path() const {
    const q3_config& c = cfg_;
    const int qd = c.n_heads * HD;
    return size() <= kSmallRows && c.dim % 1024 == 0 && qd % 1024 == 0 && c.hidden_dim % 1024 == 0;
}

// Layers of a decode step of at most kSmallRows sequences: the weight products as CUDA-core GEMVs
// over the batch's fp32 rows (RmsNorm fused into the QKV and gate/up products, SwiGLU into the
// gate/up epilogue, the residual adds into the o_proj and down epilogues), six launches a layer.
void Batch::enqueue_small_layers() {
    const q3_config& c = cfg_;
    const int B = size();
    const int qkv = (c.n_heads + 2 * c.n_kv_heads) * HD, qd = c.n_heads * HD, H = c.hidden_dim;
    const int sms = prefill_->num_sms();
    float* X = static_cast<float*>(x_.ptr);
    float* Q = static_cast<float*>(qkv_.ptr);
    float* O = static_cast<float*>(o32_.ptr);
    float* Hh = static_cast<float*>(h32_.ptr);
    const size_t layer_elems = static_cast<size_t>(pool_pages_) * c.n_kv_heads * kPageTokens * HD;
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& w = m_.layer(l);
        gemv_rows<true, false, false>(w.wqkv, nullptr, X, c.dim, w.attn_norm, c.norm_eps, Q, qkv, B,
                                      qkv, c.dim, sms, s_);
        PrefillQkvArgs qa{};
        qa.qkv = Q;
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
        qa.clear_input = 1;
        launch_prefill_qkv(qa, s_);
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
        da.out_f32 = O;
        da.out_stride = qd;
        launch_decode_attention(da, s_);
        gemv_rows<false, false, true>(w.wo, nullptr, O, qd, nullptr, 0.0f, X, c.dim, B, c.dim, qd,
                                      sms, s_);
        gemv_rows<true, true, false>(w.w1, w.w3, X, c.dim, w.mlp_norm, c.norm_eps, Hh, H, B, H,
                                     c.dim, sms, s_);
        gemv_rows<false, false, true>(w.w2, nullptr, Hh, H, nullptr, 0.0f, X, c.dim, B, c.dim, H,
                                      sms, s_);
    }
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
        // A contraction that gave up may have left partial sums behind.
        Q3_CUDA(cudaMemset(qkv_.ptr, 0, qkv_.bytes));
        Q3_CUDA(cudaMemset(gu_.ptr, 0, gu_.bytes));
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
