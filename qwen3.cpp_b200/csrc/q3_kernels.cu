// Layer-wise CUDA kernels of the B200 Qwen3 forward pass, generic over the config shape.
//
// Every kernel restates one step of the reference CPU forward (asriva32/Qwen3.cpp,
// src/inference.cpp) with fp32 activations, bf16 weights and fp32 accumulation:
//   gemv            MatMul (:952-966) with RmsNorm (:887-923) fused into the prologue and the
//                   residual add (:847-849, :863-865) or SiLU*up (:1009-1011) in the epilogue
//   qk_rope_kv      per-head QK-RMSNorm, RoPE, bf16 KV write, sink re-rotation (:800-827)
//   attention       FastAttn + Softmax (:1017-1058, :925-946) as split-K flash-decoding
//   argmax          Sampler::Greedy (:703-709), lowest index wins ties
#include <cuda_runtime.h>
#include <float.h>
#include <limits.h>

#include "q3_kernels.cuh"

namespace q3 {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvMaxGrid = 148 * 8;

__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    if (warp == 0) {
        t = lane < nw ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? red[lane] : -FLT_MAX;
        t = warp_max(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

// (value, index) ordering of Sampler::Greedy: larger value wins, then the lower index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// ------------------------------------------------------------------ GEMV

template <int EPI, bool NORM, bool VEC, bool ARGMAX>
__global__ void __launch_bounds__(kGemvThreads)
gemv_kernel(const uint16_t* __restrict__ W, const uint16_t* __restrict__ Wb,
            const float* __restrict__ x, const uint16_t* __restrict__ nw, float eps,
            float* out, float* lin2, int n, int k, float2* argmax_part) {
    extern __shared__ float4 smem4[];
    pdl_wait();
    pdl_trigger();
    float* xs = reinterpret_cast<float*>(smem4);
    __shared__ float red[32];
    __shared__ float2 best_s[kGemvWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    for (int i = tid; i < k; i += kGemvThreads) xs[i] = x[i];
    __syncthreads();
    if (NORM) {
        float ss = 0.0f;
        for (int i = tid; i < k; i += kGemvThreads) ss = fmaf(xs[i], xs[i], ss);
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(k) + eps);
        for (int i = tid; i < k; i += kGemvThreads) xs[i] = (xs[i] * inv) * bf16_to_f32(nw[i]);
        __syncthreads();
    }

    float best = -FLT_MAX;
    int best_i = INT_MAX;
    for (int r = blockIdx.x * kGemvWarps + warp; r < n; r += gridDim.x * kGemvWarps) {
        const uint16_t* wr = W + static_cast<size_t>(r) * k;
        const uint16_t* wbr = EPI == kEpiSiluMul ? Wb + static_cast<size_t>(r) * k : nullptr;
        float acc = 0.0f, accb = 0.0f;
        if (VEC) {
#pragma unroll 4
            for (int c = lane * 8; c < k; c += 256) {
                const uint4 w = ldg_stream(wr + c);
                uint4 wb;
                if (EPI == kEpiSiluMul) wb = ldg_stream(wbr + c);
                const float4 a = *reinterpret_cast<const float4*>(xs + c);
                const float4 b = *reinterpret_cast<const float4*>(xs + c + 4);
                acc = dot8(w, a, b, acc);
                if (EPI == kEpiSiluMul) accb = dot8(wb, a, b, accb);
            }
        } else {
            for (int c = lane; c < k; c += 32) {
                acc = fmaf(bf16_to_f32(wr[c]), xs[c], acc);
                if (EPI == kEpiSiluMul) accb = fmaf(bf16_to_f32(wbr[c]), xs[c], accb);
            }
        }
        acc = warp_sum(acc);
        if (EPI == kEpiSiluMul) accb = warp_sum(accb);
        if (lane == 0) {
            if (EPI == kEpiStore) out[r] = acc;
            if (EPI == kEpiResidual) out[r] += acc;
            if (EPI == kEpiSiluMul) {
                out[r] = silu(acc) * accb;
                if (lin2) lin2[r] = accb;
            }
        }
        if (ARGMAX && better(acc, r, best, best_i)) {
            best = acc;
            best_i = r;
        }
    }
    if (ARGMAX) {
        if (lane == 0) best_s[warp] = make_float2(best, __int_as_float(best_i));
        __syncthreads();
        if (tid == 0) {
            float bv = best_s[0].x;
            int bi = __float_as_int(best_s[0].y);
            for (int w = 1; w < kGemvWarps; ++w) {
                const float v = best_s[w].x;
                const int i = __float_as_int(best_s[w].y);
                if (better(v, i, bv, bi)) {
                    bv = v;
                    bi = i;
                }
            }
            argmax_part[blockIdx.x] = make_float2(bv, __int_as_float(bi));
        }
    }
}

template <int EPI, bool NORM, bool VEC, bool ARGMAX>
void gemv_launch_t(const uint16_t* W, const uint16_t* Wb, const float* x, const uint16_t* nw,
                   float eps, float* out, float* lin2, int n, int k, float2* part, int grid,
                   cudaStream_t s) {
    auto fn = gemv_kernel<EPI, NORM, VEC, ARGMAX>;
    const size_t smem = static_cast<size_t>(k) * sizeof(float);
    static bool configured[64] = {};
    int dev = 0;
    Q3_CUDA(cudaGetDevice(&dev));
    if (!configured[dev & 63]) {
        Q3_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        configured[dev & 63] = true;
    }
    launch_dep(false, fn, dim3(grid), dim3(kGemvThreads), smem, s, W, Wb, x, nw, eps, out, lin2, n, k, part);
    Q3_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------ embedding

__global__ void embed_kernel(const StepParams* sp, const uint16_t* __restrict__ embed, float* x,
                             int dim) {
    const size_t row = static_cast<size_t>(sp->token) * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
        x[i] = bf16_to_f32(embed[row + i]);
    }
}

// ------------------------------------------------------------------ QK-norm + RoPE + KV write

__device__ __forceinline__ size_t paged_index(const int32_t* table, int t, int g, int n_kv,
                                              int hd) {
    const int page = table[t / kPageTokens];
    return ((static_cast<size_t>(page) * n_kv + g) * kPageTokens + (t % kPageTokens)) *
           static_cast<size_t>(hd);
}

__device__ void rope_in_smem(float* buf, const float2* row, int half) {
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float2 cs = row[i];
        const float a = buf[i], b = buf[i + half];
        buf[i] = a * cs.x - b * cs.y;
        buf[i + half] = b * cs.x + a * cs.y;
    }
    __syncthreads();
}

__global__ void qk_rope_kv_kernel(QkvArgs a) {
    __shared__ float buf[512];
    __shared__ float red[32];
    const int b = blockIdx.x, tid = threadIdx.x, hd = a.hd, half = a.rotary_dim / 2;
    const int nq = a.n_heads, nk = a.n_kv;
    const StepParams sp = *a.sp;
    if (b < nq + nk) {
        const bool isq = b < nq;
        float* x = a.qkv + (isq ? b * hd : nq * hd + (b - nq) * hd);
        const uint16_t* w = isq ? a.q_norm : a.k_norm;
        float ss = 0.0f;
        for (int i = tid; i < hd; i += blockDim.x) {
            const float v = x[i];
            buf[i] = v;
            ss = fmaf(v, v, ss);
        }
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(hd) + a.eps);
        for (int i = tid; i < hd; i += blockDim.x) buf[i] = (buf[i] * inv) * bf16_to_f32(w[i]);
        __syncthreads();
        const int p = min(sp.pos, a.rope_len - 1);
        rope_in_smem(buf, a.rope + static_cast<size_t>(p) * half, half);
        if (isq) {
            for (int i = tid; i < hd; i += blockDim.x) x[i] = buf[i];
        } else {
            uint16_t* dst = a.k_cache + paged_index(a.page_table, sp.kv_pos, b - nq, nk, hd);
            for (int i = tid; i < hd; i += blockDim.x) dst[i] = f32_to_bf16(buf[i]);
        }
    } else if (b < nq + 2 * nk) {
        const int g = b - nq - nk;
        const float* x = a.qkv + (nq + nk + g) * hd;
        uint16_t* dst = a.v_cache + paged_index(a.page_table, sp.kv_pos, g, nk, hd);
        for (int i = tid; i < hd; i += blockDim.x) dst[i] = f32_to_bf16(x[i]);
    } else {
        // Sink re-rotation: K[s] = bf16(rope(float(K[s]), pos=1)) for s < num_sink.
        const int idx = b - nq - 2 * nk, s = idx / nk, g = idx % nk;
        if (s >= sp.num_sink) return;
        uint16_t* row = a.k_cache + paged_index(a.page_table, s, g, nk, hd);
        for (int i = tid; i < hd; i += blockDim.x) buf[i] = bf16_to_f32(row[i]);
        __syncthreads();
        rope_in_smem(buf, a.rope + static_cast<size_t>(1) * half, half);
        for (int i = tid; i < hd; i += blockDim.x) row[i] = f32_to_bf16(buf[i]);
    }
}

// ------------------------------------------------------------------ attention

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxGroup = 8;   // query heads per KV head
constexpr int kMaxPerLane = 8; // head_dim <= 256

template <bool PAGED>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnArgs a) {
    __shared__ float qs[kMaxGroup * 256];
    __shared__ float wm[kAttnWarps][kMaxGroup];
    __shared__ float wl[kAttnWarps][kMaxGroup];
    __shared__ float wo[kAttnWarps][kMaxGroup * 256];
    const int g = blockIdx.x, split = blockIdx.y, tid = threadIdx.x, lane = tid & 31,
              warp = tid >> 5;
    const int hd = a.hd, G = a.n_heads / a.n_kv, nj = (hd + 31) / 32;
    const int kv_len = a.sp ? a.sp->kv_len : a.kv_len_const;
    const int chunk = (kv_len + a.n_splits - 1) / a.n_splits;
    const int t0 = split * chunk, t1 = min(kv_len, t0 + chunk);
    const float sq = sqrtf(static_cast<float>(hd));

    for (int i = tid; i < G * hd; i += kAttnThreads) qs[i] = a.q[(g * G) * hd + i];
    __syncthreads();

    float m[kMaxGroup], l[kMaxGroup], o[kMaxGroup][kMaxPerLane];
#pragma unroll
    for (int gi = 0; gi < kMaxGroup; ++gi) {
        m[gi] = -FLT_MAX;
        l[gi] = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) o[gi][j] = 0.0f;
    }
    const size_t stride = static_cast<size_t>(a.row_stride);
    for (int t = t0 + warp; t < t1; t += kAttnWarps) {
        const size_t base = PAGED ? paged_index(a.page_table, t, g, a.n_kv, hd)
                                  : static_cast<size_t>(t) * stride + static_cast<size_t>(g) * hd;
        float kv[kMaxPerLane];
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int d = lane + 32 * j;
            kv[j] = (j < nj && d < hd) ? bf16_to_f32(a.k[base + d]) : 0.0f;
        }
        float vv[kMaxPerLane];
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int d = lane + 32 * j;
            vv[j] = (j < nj && d < hd) ? bf16_to_f32(a.v[base + d]) : 0.0f;
        }
#pragma unroll
        for (int gi = 0; gi < kMaxGroup; ++gi) {
            if (gi >= G) break;
            float dot = 0.0f;
#pragma unroll
            for (int j = 0; j < kMaxPerLane; ++j) {
                const int d = lane + 32 * j;
                if (j < nj && d < hd) dot = fmaf(kv[j], qs[gi * hd + d], dot);
            }
            const float s = warp_sum(dot) / sq;
            const float mn = fmaxf(m[gi], s);
            const float alpha = expf(m[gi] - mn);
            const float p = expf(s - mn);
            l[gi] = l[gi] * alpha + p;
#pragma unroll
            for (int j = 0; j < kMaxPerLane; ++j) o[gi][j] = o[gi][j] * alpha + p * vv[j];
            m[gi] = mn;
        }
    }
    // Merge the warps of this block.
    for (int gi = 0; gi < G; ++gi) {
        if (lane == 0) {
            wm[warp][gi] = m[gi];
            wl[warp][gi] = l[gi];
        }
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int d = lane + 32 * j;
            if (j < nj && d < hd) wo[warp][gi * hd + d] = o[gi][j];
        }
    }
    __syncthreads();
    for (int idx = tid; idx < G * hd; idx += kAttnThreads) {
        const int gi = idx / hd, d = idx % hd;
        float M = -FLT_MAX;
        for (int w = 0; w < kAttnWarps; ++w)
            if (wl[w][gi] > 0.0f) M = fmaxf(M, wm[w][gi]);
        float L = 0.0f, acc = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) {
            if (wl[w][gi] > 0.0f) {
                const float sc = expf(wm[w][gi] - M);
                L += wl[w][gi] * sc;
                acc += wo[w][gi * hd + d] * sc;
            }
        }
        const int head = g * G + gi;
        const size_t pi = static_cast<size_t>(head) * a.n_splits + split;
        a.part_o[pi * hd + d] = acc;
        if (d == 0) a.part_ml[pi] = make_float2(M, L);
    }
}

__global__ void attention_combine_kernel(AttnArgs a) {
    const int head = blockIdx.x, hd = a.hd, S = a.n_splits;
    const float2* ml = a.part_ml + static_cast<size_t>(head) * S;
    float M = -FLT_MAX;
    for (int s = 0; s < S; ++s)
        if (ml[s].y > 0.0f) M = fmaxf(M, ml[s].x);
    float L = 0.0f;
    for (int s = 0; s < S; ++s)
        if (ml[s].y > 0.0f) L += ml[s].y * expf(ml[s].x - M);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < S; ++s) {
            if (ml[s].y > 0.0f) {
                acc += a.part_o[(static_cast<size_t>(head) * S + s) * hd + d] * expf(ml[s].x - M);
            }
        }
        a.out[head * hd + d] = acc / L;
    }
}

// ------------------------------------------------------------------ argmax / step advance

__global__ void argmax_final_kernel(const float2* part, int n_part, int32_t* out_index,
                                    StepParams* sp, int32_t* token_log, int ctx,
                                    const int32_t* forced_next) {
    __shared__ float bv_s[32];
    __shared__ int bi_s[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int i = tid; i < n_part; i += blockDim.x) {
        const float v = part[i].x;
        const int j = __float_as_int(part[i].y);
        if (better(v, j, bv, bi)) {
            bv = v;
            bi = j;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o);
        const int j = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(v, j, bv, bi)) {
            bv = v;
            bi = j;
        }
    }
    if (lane == 0) {
        bv_s[warp] = bv;
        bi_s[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (blockDim.x >> 5); ++w) {
            if (better(bv_s[w], bi_s[w], bv, bi)) {
                bv = bv_s[w];
                bi = bi_s[w];
            }
        }
        if (bi == INT_MAX) bi = 0;  // all NaN: std::max_element would return the first
        if (out_index) *out_index = bi;
        if (sp) {
            StepParams p = *sp;
            if (token_log) token_log[p.step] = bi;
            p.token = (forced_next && p.step + 1 < p.n_forced) ? forced_next[p.step + 1] : bi;
            p.step += 1;
            p.pos += 1;
            step_positions(p.pos, ctx, &p.num_sink, &p.kv_pos, &p.kv_len);
            *sp = p;
        }
    }
}

__global__ void argmax_full_kernel(const float* x, int n, int32_t* out) {
    __shared__ float bv_s[32];
    __shared__ int bi_s[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int i = tid; i < n; i += blockDim.x) {
        if (better(x[i], i, bv, bi)) {
            bv = x[i];
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o);
        const int j = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(v, j, bv, bi)) {
            bv = v;
            bi = j;
        }
    }
    if (lane == 0) {
        bv_s[warp] = bv;
        bi_s[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (blockDim.x >> 5); ++w) {
            if (better(bv_s[w], bi_s[w], bv, bi)) {
                bv = bv_s[w];
                bi = bi_s[w];
            }
        }
        *out = bi == INT_MAX ? 0 : bi;
    }
}

// ------------------------------------------------------------------ free-function kernels

__global__ void rmsnorm_kernel(float* out, const float* x, const uint16_t* w, float eps, int n) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = (x[i] * inv) * bf16_to_f32(w[i]);
}

__global__ void softmax_kernel(float* out, const float* x, int n) {
    __shared__ float red[32];
    float mx = -FLT_MAX;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, x[i]);
    mx = block_max(mx, red);
    float sum = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(x[i] - mx);
        out[i] = e;
        sum += e;
    }
    sum = block_sum(sum, red);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] /= sum;
}

__global__ void rope_row_kernel(float* x, int d, int head_dim, int rotary_dim, RopeRow row) {
    const int half = rotary_dim / 2, heads = d / head_dim;
    for (int idx = threadIdx.x; idx < heads * half; idx += blockDim.x) {
        const int h = idx / half, i = idx % half;
        float* p = x + h * head_dim;
        const float a = p[i], b = p[i + half], c = row.c[i], s = row.s[i];
        p[i] = a * c - b * s;
        p[i + half] = b * c + a * s;
    }
}

}  // namespace

// ------------------------------------------------------------------ launchers

int gemv_grid(int n) {
    const int g = (n + kGemvWarps - 1) / kGemvWarps;
    return g < kGemvMaxGrid ? g : kGemvMaxGrid;
}

void launch_gemv(int epi, const uint16_t* W, const uint16_t* Wb, const float* x,
                 const uint16_t* norm_w, float eps, float* out, float* lin2, int n, int k,
                 float2* argmax_part, int grid_override, cudaStream_t s) {
    if (n <= 0 || k <= 0) return;
    if (static_cast<size_t>(k) * sizeof(float) > 200 * 1024) {
        throw std::invalid_argument("MatMul inner dimension too large for one block's input");
    }
    const int grid = grid_override > 0 ? grid_override : gemv_grid(n);
    const bool vec = (k % 8 == 0) && (reinterpret_cast<uintptr_t>(W) % 16 == 0) &&
                     (Wb == nullptr || reinterpret_cast<uintptr_t>(Wb) % 16 == 0);
    const bool norm = norm_w != nullptr;
    const bool am = argmax_part != nullptr;
#define Q3_GEMV(E, N, V, A) \
    gemv_launch_t<E, N, V, A>(W, Wb, x, norm_w, eps, out, lin2, n, k, argmax_part, grid, s)
    if (epi == kEpiStore) {
        if (am) {
            if (norm) { vec ? Q3_GEMV(kEpiStore, true, true, true) : Q3_GEMV(kEpiStore, true, false, true); }
            else { vec ? Q3_GEMV(kEpiStore, false, true, true) : Q3_GEMV(kEpiStore, false, false, true); }
        } else {
            if (norm) { vec ? Q3_GEMV(kEpiStore, true, true, false) : Q3_GEMV(kEpiStore, true, false, false); }
            else { vec ? Q3_GEMV(kEpiStore, false, true, false) : Q3_GEMV(kEpiStore, false, false, false); }
        }
    } else if (epi == kEpiResidual) {
        if (norm) { vec ? Q3_GEMV(kEpiResidual, true, true, false) : Q3_GEMV(kEpiResidual, true, false, false); }
        else { vec ? Q3_GEMV(kEpiResidual, false, true, false) : Q3_GEMV(kEpiResidual, false, false, false); }
    } else {
        if (norm) { vec ? Q3_GEMV(kEpiSiluMul, true, true, false) : Q3_GEMV(kEpiSiluMul, true, false, false); }
        else { vec ? Q3_GEMV(kEpiSiluMul, false, true, false) : Q3_GEMV(kEpiSiluMul, false, false, false); }
    }
#undef Q3_GEMV
}

void launch_embed(const StepParams* sp, const uint16_t* embed, float* x, int dim,
                  cudaStream_t s) {
    embed_kernel<<<(dim + 255) / 256, 256, 0, s>>>(sp, embed, x, dim);
    Q3_CUDA(cudaGetLastError());
}

void launch_qk_rope_kv(const QkvArgs& a, cudaStream_t s) {
    const int blocks = a.n_heads + 2 * a.n_kv + 4 * a.n_kv;
    qk_rope_kv_kernel<<<blocks, 128, 0, s>>>(a);
    Q3_CUDA(cudaGetLastError());
}

int attn_splits_for(int max_kv_len) {
    int s = (max_kv_len + 255) / 256;
    return s < 1 ? 1 : (s > 64 ? 64 : s);
}

void launch_attention(const AttnArgs& a, cudaStream_t s) {
    dim3 grid(a.n_kv, a.n_splits);
    if (a.page_table) {
        attention_kernel<true><<<grid, kAttnThreads, 0, s>>>(a);
    } else {
        attention_kernel<false><<<grid, kAttnThreads, 0, s>>>(a);
    }
    Q3_CUDA(cudaGetLastError());
    attention_combine_kernel<<<a.n_heads, 128, 0, s>>>(a);
    Q3_CUDA(cudaGetLastError());
}

void launch_argmax_final(const float2* part, int n_part, int32_t* out_index, StepParams* sp,
                         int32_t* token_log, int ctx, const int32_t* forced_next,
                         cudaStream_t s) {
    argmax_final_kernel<<<1, 512, 0, s>>>(part, n_part, out_index, sp, token_log, ctx,
                                          forced_next);
    Q3_CUDA(cudaGetLastError());
}

void launch_argmax_full(const float* x, int n, int32_t* out, cudaStream_t s) {
    argmax_full_kernel<<<1, 1024, 0, s>>>(x, n, out);
    Q3_CUDA(cudaGetLastError());
}

void launch_rmsnorm(float* out, const float* x, const uint16_t* w, float eps, int n,
                    cudaStream_t s) {
    rmsnorm_kernel<<<1, 1024, 0, s>>>(out, x, w, eps, n);
    Q3_CUDA(cudaGetLastError());
}

void launch_softmax(float* out, const float* x, int n, cudaStream_t s) {
    softmax_kernel<<<1, 1024, 0, s>>>(out, x, n);
    Q3_CUDA(cudaGetLastError());
}

void launch_rope_row(float* x, int d, int head_dim, int rotary_dim, const RopeRow& row,
                     cudaStream_t s) {
    rope_row_kernel<<<1, 256, 0, s>>>(x, d, head_dim, rotary_dim, row);
    Q3_CUDA(cudaGetLastError());
}

}  // namespace q3
