// Batched prefill (see q3_prefill.cuh): row RmsNorm into bf16 operands, per-head QK-norm + RoPE
// with the paged K/V write, causal flash attention over the paged cache, and the driver that
// chains them with the tensor-core contractions of q3_gemm.cu.
#include <cuda_bf16.h>
#include <float.h>

#include <algorithm>
#include <stdexcept>

#include "q3_gemm.cuh"
#include "q3_prefill.cuh"

namespace q3 {

namespace {

constexpr int HD = 128;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t pack2_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // low half = a
    return *reinterpret_cast<const uint32_t*>(&h);
}

// ------------------------------------------------------------------ row RmsNorm -> bf16

constexpr int kNormWarps = 8;  // rows per block, one warp per row

// Elements i..i+3 of the normalised row as bf16 (or fp16) at out, their low parts at out_lo.
__device__ __forceinline__ void norm_emit4(uint16_t* orow, uint16_t* lorow, int i, float4 v,
                                           float inv, const uint16_t* w, int f16) {
    const uint2 wb = *reinterpret_cast<const uint2*>(w + i);
    const float y0 = (v.x * inv) * bf16_lo(wb.x), y1 = (v.y * inv) * bf16_hi(wb.x);
    const float y2 = (v.z * inv) * bf16_lo(wb.y), y3 = (v.w * inv) * bf16_hi(wb.y);
    if (f16) {
        const uint2 hi = make_uint2(pack2_f16(y0, y1), pack2_f16(y2, y3));
        *reinterpret_cast<uint2*>(orow + i) = hi;
        if (lorow) {  // y - f16(y): the hi + lo pair carries 22 significant bits
            *reinterpret_cast<uint2*>(lorow + i) =
                make_uint2(pack2_f16(y0 - f16_lo(hi.x), y1 - f16_hi(hi.x)),
                           pack2_f16(y2 - f16_lo(hi.y), y3 - f16_hi(hi.y)));
        }
        return;
    }
    const uint2 hi = make_uint2(pack2_bf16(y0, y1), pack2_bf16(y2, y3));
    *reinterpret_cast<uint2*>(orow + i) = hi;
    if (lorow) {  // y - bf16(y): the hi + lo pair carries 16 significant bits
        *reinterpret_cast<uint2*>(lorow + i) =
            make_uint2(pack2_bf16(y0 - bf16_lo(hi.x), y1 - bf16_hi(hi.x)),
                       pack2_bf16(y2 - bf16_lo(hi.y), y3 - bf16_hi(hi.y)));
    }
}

// One warp per row: x (from the embedding rows of ids when given) -> RmsNorm (src/inference.cpp:
// 905-921: (x * (1 / rms)) * w, rms = sqrtf(ss / n + eps)) -> bf16 / fp16 (+ low parts). DIM > 0:
// the row width as a constant, the row held in registers between the sum of squares and the
// output (one read of x); DIM = 0: any width (a multiple of 256), x read twice. Both sum the
// squares in the same order, so they give the same bits.
template <int DIM>
__global__ void __launch_bounds__(kNormWarps * 32)
    rmsnorm_rows_kernel(const int32_t* __restrict__ ids, const uint16_t* __restrict__ embed,
                        float* __restrict__ x, const uint16_t* __restrict__ w, float eps,
                        uint16_t* __restrict__ out, uint16_t* __restrict__ out_lo, int rows,
                        int dim, int f16) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    if (DIM > 0) dim = DIM;
    float* xr = x + static_cast<size_t>(row) * dim;
    uint16_t* orow = out + static_cast<size_t>(row) * dim;
    uint16_t* lorow = out_lo ? out_lo + static_cast<size_t>(row) * dim : nullptr;
    if (DIM > 0) {
        constexpr int NV = DIM > 0 ? DIM / 128 : 1;  // float4 per lane
        float4 v[NV];
        if (ids) {
            const uint16_t* er = embed + static_cast<size_t>(ids[row]) * dim;
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                const int i = lane * 4 + 128 * j;
                const uint2 e = *reinterpret_cast<const uint2*>(er + i);
                v[j] = make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
                *reinterpret_cast<float4*>(xr + i) = v[j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < NV; ++j) v[j] = *reinterpret_cast<const float4*>(xr + lane * 4 + 128 * j);
        }
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            ss = fmaf(v[j].x, v[j].x, ss);
            ss = fmaf(v[j].y, v[j].y, ss);
            ss = fmaf(v[j].z, v[j].z, ss);
            ss = fmaf(v[j].w, v[j].w, ss);
        }
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
#pragma unroll
        for (int j = 0; j < NV; ++j) norm_emit4(orow, lorow, lane * 4 + 128 * j, v[j], inv, w, f16);
        return;
    }
    if (ids) {
        const uint16_t* er = embed + static_cast<size_t>(ids[row]) * dim;
        for (int i = lane * 8; i < dim; i += 256) {
            const uint4 e = *reinterpret_cast<const uint4*>(er + i);
            *reinterpret_cast<float4*>(xr + i) = make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
            *reinterpret_cast<float4*>(xr + i + 4) = make_float4(bf16_lo(e.z), bf16_hi(e.z), bf16_lo(e.w), bf16_hi(e.w));
        }
        __syncwarp();
    }
    float ss = 0.0f;
    for (int i = lane * 4; i < dim; i += 128) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
    for (int i = lane * 4; i < dim; i += 128) {
        norm_emit4(orow, lorow, i, *reinterpret_cast<const float4*>(xr + i), inv, w, f16);
    }
}

// ------------------------------------------------------------------ QK-norm + RoPE + KV write

// One warp per (token, head); lane l holds elements 4l..4l+3 of the 128-wide head, so the RoPE
// partner of element e (e + 64 or e - 64) sits in lane l ^ 16.
__global__ void __launch_bounds__(256) prefill_qkv_kernel(PrefillQkvArgs a) {
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x;
    const int head = blockIdx.y * 8 + warp;
    const int nq = a.n_heads, nk = a.n_kv, nkc = a.n_kv_cache ? a.n_kv_cache : a.n_kv;
    if (head >= nq + 2 * nk) return;
    const int pos = a.dec_pos ? a.dec_pos[row] : a.pos0 + row;
    const int32_t* table = a.dec_pos ? a.page_table + static_cast<size_t>(row) * a.pages_per_seq
                                     : a.page_table;
    float* src = a.qkv + static_cast<size_t>(row) * (nq + 2 * nk) * HD + head * HD;
    float4 v = reinterpret_cast<const float4*>(src)[lane];
    if (a.clear_input) reinterpret_cast<float4*>(src)[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int e = lane * 4;
    uint16_t* dst;
    if (head < nq + nk) {
        const bool isq = head < nq;
        const uint16_t* w = isq ? a.q_norm : a.k_norm;
        float ss = v.x * v.x;
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(HD) + a.eps);
        const uint2 wb = *reinterpret_cast<const uint2*>(w + e);
        v.x = (v.x * inv) * bf16_lo(wb.x);
        v.y = (v.y * inv) * bf16_hi(wb.x);
        v.z = (v.z * inv) * bf16_lo(wb.y);
        v.w = (v.w * inv) * bf16_hi(wb.y);
        // ApplyRotaryEmb (src/inference.cpp:968-991): (a, b) = (x_i, x_{i+64}) ->
        // (a cos - b sin, b cos + a sin).
        const float4 p = make_float4(__shfl_xor_sync(0xffffffffu, v.x, 16),
                                     __shfl_xor_sync(0xffffffffu, v.y, 16),
                                     __shfl_xor_sync(0xffffffffu, v.z, 16),
                                     __shfl_xor_sync(0xffffffffu, v.w, 16));
        const float2* cs = a.rope + static_cast<size_t>(pos) * (HD / 2) + (e & 63);
        const float4 c01 = *reinterpret_cast<const float4*>(cs);
        const float4 c23 = *reinterpret_cast<const float4*>(cs + 2);
        if (lane < 16) {
            v.x = v.x * c01.x - p.x * c01.y;
            v.y = v.y * c01.z - p.y * c01.w;
            v.z = v.z * c23.x - p.z * c23.y;
            v.w = v.w * c23.z - p.w * c23.w;
        } else {
            v.x = v.x * c01.x + p.x * c01.y;
            v.y = v.y * c01.z + p.y * c01.w;
            v.z = v.z * c23.x + p.z * c23.y;
            v.w = v.w * c23.z + p.w * c23.w;
        }
        if (isq) {
            if (a.q_out_f32) {
                reinterpret_cast<float4*>(a.q_out_f32 + static_cast<size_t>(row) * nq * HD +
                                          head * HD)[lane] = v;
            }
            if (!a.q_out) return;
            dst = a.q_out + static_cast<size_t>(row) * nq * HD + head * HD;
        } else {
            const int g = a.kv_head0 + head - nq;
            dst = a.k_cache +
                  ((static_cast<size_t>(table[pos / kPageTokens]) * nkc + g) * kPageTokens +
                   pos % kPageTokens) * HD;
        }
    } else {
        const int g = a.kv_head0 + head - nq - nk;
        dst = a.v_cache +
              ((static_cast<size_t>(table[pos / kPageTokens]) * nkc + g) * kPageTokens +
               pos % kPageTokens) * HD;
    }
    reinterpret_cast<uint2*>(dst)[lane] = make_uint2(pack2_bf16(v.x, v.y), pack2_bf16(v.z, v.w));
}

// bf16 -> fp16 (same values in range), 8 elements per thread.
__global__ void bf16_to_f16_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                   size_t n8) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint4 v = reinterpret_cast<const uint4*>(src)[i];
        reinterpret_cast<uint4*>(dst)[i] =
            make_uint4(bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z),
                       bf16x2_to_f16x2(v.w));
    }
}

// fp16 copies of the cache rows of logical pages [0, pages) of one sequence, every layer (the
// rows a prefill at a later position attends to but did not write itself). Block (page, layer).
__global__ void kv_to_f16_kernel(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                                 uint16_t* __restrict__ k16, uint16_t* __restrict__ v16,
                                 const int32_t* __restrict__ table, size_t layer_elems,
                                 int page_elems) {
    const size_t base = static_cast<size_t>(blockIdx.y) * layer_elems +
                        static_cast<size_t>(__ldg(table + blockIdx.x)) * page_elems;
    for (int i = threadIdx.x; i < page_elems / 8; i += blockDim.x) {
        const size_t e = base / 8 + i;
        const uint4 kv = reinterpret_cast<const uint4*>(k)[e];
        const uint4 vv = reinterpret_cast<const uint4*>(v)[e];
        reinterpret_cast<uint4*>(k16)[e] = make_uint4(bf16x2_to_f16x2(kv.x), bf16x2_to_f16x2(kv.y),
                                                      bf16x2_to_f16x2(kv.z), bf16x2_to_f16x2(kv.w));
        reinterpret_cast<uint4*>(v16)[e] = make_uint4(bf16x2_to_f16x2(vv.x), bf16x2_to_f16x2(vv.y),
                                                      bf16x2_to_f16x2(vv.z), bf16x2_to_f16x2(vv.w));
    }
}

int device_sms(int device) {
    int n = 0;
    Q3_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
    return n;
}

}  // namespace

void launch_rmsnorm_rows_bf16(const int32_t* ids, const uint16_t* embed, float* x,
                              const uint16_t* w, float eps, uint16_t* out, int rows, int dim,
                              cudaStream_t s, uint16_t* out_lo, bool dependent, bool f16) {
    if (rows <= 0) return;
    if (dim % 256 != 0) throw std::invalid_argument("row RmsNorm needs a width that is a multiple of 256");
    launch_dep(dependent, dim == 1024 ? rmsnorm_rows_kernel<1024> : rmsnorm_rows_kernel<0>,
               dim3((rows + kNormWarps - 1) / kNormWarps), dim3(kNormWarps * 32), 0, s, ids, embed,
               x, w, eps, out, out_lo, rows, dim, static_cast<int>(f16));
    Q3_CUDA(cudaGetLastError());
}

void launch_prefill_qkv(const PrefillQkvArgs& a, cudaStream_t s) {
    if (a.rows <= 0) return;
    const dim3 grid(a.rows, (a.n_heads + 2 * a.n_kv + 7) / 8);
    launch_dep(false, prefill_qkv_kernel, grid, dim3(256), 0, s, a);
    Q3_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------ driver

bool Prefill::supported(const q3_config& c) {
    return c.head_dim == HD && c.rotary_dim == HD && c.n_kv_heads > 0 &&
           c.n_heads == 2 * c.n_kv_heads && c.dim % 256 == 0 && c.hidden_dim % 128 == 0 &&
           (c.n_heads * HD) % 64 == 0 && ((c.n_heads + 2 * c.n_kv_heads) * HD) % 128 == 0 &&
           c.dim % 128 == 0;
}

Prefill::Prefill(const q3_config& c, int device) : cfg_(c), device_(device) {
    num_sms_ = device_sms(device);
    err_.alloc(sizeof(unsigned));
    Q3_CUDA(cudaMemset(err_.ptr, 0, sizeof(unsigned)));
}

void make_f16_layers(const q3_config& c, const std::vector<LayerWeights>& layers,
                     DeviceBuffer& arena, std::vector<LayerWeights>& out, cudaStream_t s) {
    const size_t D = c.dim, H = c.hidden_dim;
    const size_t qkv = static_cast<size_t>(c.n_heads + 2 * c.n_kv_heads) * HD;
    const size_t qd = static_cast<size_t>(c.n_heads) * HD;
    const size_t per = qkv * D + D * qd + 2 * H * D + D * H;  // elements of one layer
    arena.alloc(per * layers.size() * 2);
    out = layers;
    auto conv = [&](const uint16_t* src, uint16_t* dst, size_t n) {
        if (n % 8 != 0) throw std::invalid_argument("fp16 copy: size not a multiple of 8");
        bf16_to_f16_kernel<<<1024, 256, 0, s>>>(src, dst, n / 8);
        Q3_CUDA(cudaGetLastError());
    };
    for (size_t l = 0; l < layers.size(); ++l) {
        const LayerWeights& w = layers[l];
        uint16_t* p = static_cast<uint16_t*>(arena.ptr) + per * l;
        uint16_t* wqkv = p;
        uint16_t* wo = wqkv + qkv * D;
        uint16_t* w1 = wo + D * qd;
        uint16_t* w3 = w1 + H * D;
        uint16_t* w2 = w3 + H * D;
        conv(w.wqkv, wqkv, qkv * D);
        conv(w.wo, wo, D * qd);
        conv(w.w1, w1, H * D);
        conv(w.w3, w3, H * D);
        conv(w.w2, w2, D * H);
        out[l].wqkv = wqkv;
        out[l].wo = wo;
        out[l].w1 = w1;
        out[l].w3 = w3;
        out[l].w2 = w2;
    }
}

void Prefill::ensure_rows(int rows) {
    if (rows <= cap_rows_) return;
    const int cap = (rows + 127) / 128 * 128;
    const q3_config& c = cfg_;
    const size_t qd = static_cast<size_t>(c.n_heads) * HD;
    x_.alloc(static_cast<size_t>(cap) * c.dim * 4);
    xn_.alloc(static_cast<size_t>(cap) * c.dim * 2);
    xn_lo_.alloc(static_cast<size_t>(cap) * c.dim * 2);
    q_.alloc(static_cast<size_t>(cap) * qd * 2);
    o_.alloc(static_cast<size_t>(cap) * qd * 2);
    h_.alloc(static_cast<size_t>(cap) * c.hidden_dim * 2);
    cap_rows_ = cap;
}

void Prefill::ensure_weight_maps(const std::vector<LayerWeights>& layers) {
    if (!layers.empty() && wmaps_key_ == layers[0].wqkv && wmaps_.size() == layers.size()) return;
    const q3_config& c = cfg_;
    const int qd = c.n_heads * HD;
    const int qkv = (c.n_heads + 2 * c.n_kv_heads) * HD;
    wmaps_.resize(layers.size());
    for (size_t l = 0; l < layers.size(); ++l) {
        const LayerWeights& w = layers[l];
        make_tmap_bf16(&wmaps_[l].wqkv, w.wqkv, qkv, c.dim, gemm_tile_n(kEpiStoreF32, qkv));
        make_tmap_bf16(&wmaps_[l].wo, w.wo, c.dim, qd, gemm_tile_n(kEpiAddF32, c.dim));
        make_tmap_bf16(&wmaps_[l].w1, w.w1, c.hidden_dim, c.dim, 128);
        make_tmap_bf16(&wmaps_[l].w3, w.w3, c.hidden_dim, c.dim, 128);
        make_tmap_bf16(&wmaps_[l].w2, w.w2, c.dim, c.hidden_dim, gemm_tile_n(kEpiAddF32, c.dim));
    }
    wmaps_key_ = layers.empty() ? nullptr : layers[0].wqkv;
}

size_t Prefill::layer_elems(const KvView& kv) const {
    return static_cast<size_t>(kv.n_pages) * cfg_.n_kv_heads * kPageTokens * HD;
}

void Prefill::ensure_kv_maps(const KvView& kv, int L) {
    const bool f16 = precision_ == kPrecisionF16;
    if (kv_key_ == kv.k_base && kv_pages_ == kv.n_pages && kv_maps_f16_ == f16) return;
    const q3_config& c = cfg_;
    const uint64_t kv_rows = static_cast<uint64_t>(L) * kv.n_pages * c.n_kv_heads * kPageTokens;
    const void* kb = kv.k_base;
    const void* vb = kv.v_base;
    if (f16) {
        const size_t bytes = kv_rows * HD * 2;
        if (k16_.bytes != bytes || kv_key_ != kv.k_base) {
            k16_.alloc(bytes);
            v16_.alloc(bytes);
        }
        kb = k16_.ptr;
        vb = v16_.ptr;
    }
    make_tmap_bf16(&kmap_, kb, kv_rows, HD, kPageTokens);
    make_tmap_bf16(&vmap_, vb, kv_rows, HD, kPageTokens);
    // The 4-D page maps serve tiles of 8 pages inside one layer; with fewer pages per layer the
    // kernel never takes that path and the 2-D maps stand in.
    if (kv.n_pages >= 8) {
        const uint64_t pages = static_cast<uint64_t>(L) * kv.n_pages;
        make_tmap_kv_pages(&kmap4_, kb, c.n_kv_heads, pages);
        make_tmap_kv_pages(&vmap4_, vb, c.n_kv_heads, pages);
    } else {
        kmap4_ = kmap_;
        vmap4_ = vmap_;
    }
    kv_key_ = kv.k_base;
    kv_pages_ = kv.n_pages;
    kv_maps_f16_ = f16;
}

unsigned Prefill::read_error(cudaStream_t s) {
    unsigned v = 0;
    Q3_CUDA(cudaMemcpyAsync(&v, err_.ptr, sizeof(v), cudaMemcpyDeviceToHost, s));
    Q3_CUDA(cudaStreamSynchronize(s));
    if (v) Q3_CUDA(cudaMemsetAsync(err_.ptr, 0, sizeof(unsigned), s));
    return v;
}

KvView engine_view(Engine& e) {
    KvView v;
    v.k_base = e.k_layer(0);
    v.v_base = e.v_layer(0);
    v.n_pages = e.n_pages();
    v.page_table = e.page_table();
    v.rope = e.rope();
    v.rope_len = e.rope_len();
    return v;
}

void Prefill::layer_pass(const int32_t* ids, int S, const PassRows& pr, const uint16_t* embed,
                         const std::vector<LayerWeights>& layers, const KvView& kv, float* taps,
                         cudaStream_t s) {
    const q3_config& c = cfg_;
    const int qd = c.n_heads * HD;
    const int qkv = (c.n_heads + 2 * c.n_kv_heads) * HD;
    const int L = static_cast<int>(layers.size());
    const int table_len = kv.table_len ? kv.table_len : kv.n_pages;
    const bool f16 = precision_ == kPrecisionF16;
    float* X = static_cast<float*>(x_.ptr);
    uint16_t* Xn = static_cast<uint16_t*>(xn_.ptr);
    uint16_t* XnLo = f16 ? static_cast<uint16_t*>(xn_lo_.ptr) : nullptr;
    unsigned* err = static_cast<unsigned*>(err_.ptr);
    uint16_t* k16 = f16 ? static_cast<uint16_t*>(k16_.ptr) : nullptr;
    uint16_t* v16 = f16 ? static_cast<uint16_t*>(v16_.ptr) : nullptr;
    CUtensorMap m_xn, m_xn_lo, m_o, m_h, m_q;
    make_tmap_bf16(&m_q, q_.ptr, S, qd, 64);
    make_tmap_bf16(&m_xn, xn_.ptr, S, c.dim, 128);
    make_tmap_bf16(&m_xn_lo, xn_lo_.ptr, S, c.dim, 128);
    make_tmap_bf16(&m_o, o_.ptr, S, qd, 128);
    make_tmap_bf16(&m_h, h_.ptr, S, c.hidden_dim, 128);
    CUtensorMap o_x, o_h;  // contraction outputs
    make_tmap_out(&o_x, X, S, c.dim, false);
    make_tmap_out(&o_h, h_.ptr, S, c.hidden_dim, true);
    auto tap = [&](int slot) {
        if (taps) {
            Q3_CUDA(cudaMemcpyAsync(taps + static_cast<size_t>(slot) * c.dim,
                                    X + static_cast<size_t>(S - 1) * c.dim, c.dim * 4,
                                    cudaMemcpyDeviceToDevice, s));
        }
    };
    launch_rmsnorm_rows_bf16(ids, embed, X, layers[0].attn_norm, c.norm_eps, Xn, S, c.dim, s, XnLo,
                             true, f16);
    tap(0);
    for (int l = 0; l < L; ++l) {
        const LayerWeights& w = layers[l];
        const LayerMaps& wm = wmaps_[l];
        GemmArgs g;
        g.err = err;
        g.dependent = true;  // the prefill's kernels launch as programmatic dependents
        g.f16 = f16 ? 1 : 0;
        g.M = S;
        // [wq; wk; wv] . xn (src/inference.cpp:795-798) with the QK-RMSNorm, RoPE and the paged
        // K/V write (:800-815) in the epilogue: q rows to q_.
        g.N = qkv;
        g.K = c.dim;
        g.qkv.q_out = static_cast<uint16_t*>(q_.ptr);
        g.qkv.k_cache = kv.k_base + layer_elems(kv) * l;
        g.qkv.v_cache = kv.v_base + layer_elems(kv) * l;
        g.qkv.page_table = kv.page_table;
        g.qkv.rope = kv.rope;
        g.qkv.q_norm = w.q_norm;
        g.qkv.k_norm = w.k_norm;
        g.qkv.pos0 = pr.p0;
        g.qkv.tok_pos = pr.tok_pos;
        g.qkv.tok_row = pr.tok_row;
        g.qkv.n_heads = c.n_heads;
        g.qkv.n_kv = c.n_kv_heads;
        g.qkv.eps = c.norm_eps;
        if (f16) {
            // fp16 q for the attention, fp16 copies of the K/V rows it reads; the RmsNorm'd
            // input as an fp16 hi + lo pair (the one input where the error of a single fp16
            // rounding still shows in the hidden states).
            g.qkv.q_f16 = 1;
            g.qkv.k_stage = k16 + layer_elems(kv) * l;
            g.qkv.v_stage = v16 + layer_elems(kv) * l;
            Q3_CUDA(launch_gemm(m_xn, wm.wqkv, nullptr, m_xn, g, kEpiQkvRope, num_sms_, s,
                                &m_xn_lo));
        } else {
            Q3_CUDA(launch_gemm(m_xn, wm.wqkv, nullptr, m_xn, g, kEpiQkvRope, num_sms_, s));
        }
        g.qkv = QkvEpilogue{};
        PrefillAttnTcArgs ta{};
        ta.page_table = kv.page_table;
        ta.out = static_cast<uint16_t*>(o_.ptr);
        ta.err = err;
        ta.rows = S;
        ta.pos0 = pr.p0;
        ta.n_kv = c.n_kv_heads;
        ta.n_pages = kv.n_pages;
        ta.pages_per_seq = table_len;
        ta.layer = l;
        ta.f16 = f16 ? 1 : 0;
        ta.work = pr.work;
        ta.n_work = pr.n_work;
        launch_prefill_attention_tc(m_q, kmap_, vmap_, kmap4_, vmap4_, ta, s);
        // x += wo . attn (:846-849).
        g.N = c.dim;
        g.K = qd;
        Q3_CUDA(launch_gemm(m_o, wm.wo, nullptr, o_x, g, kEpiAddF32, num_sms_, s));
        launch_rmsnorm_rows_bf16(nullptr, nullptr, X, w.mlp_norm, c.norm_eps, Xn, S, c.dim, s,
                                 nullptr, true, f16);
        // h = silu(w1 . xn) * (w3 . xn) (:851, :1005-1011).
        g.N = 2 * c.hidden_dim;
        g.K = c.dim;
        Q3_CUDA(launch_gemm(m_xn, wm.w1, &wm.w3, o_h, g, kEpiSwiGLU, num_sms_, s));
        // x += w2 . h (:1013, :863-865).
        g.N = c.dim;
        g.K = c.hidden_dim;
        Q3_CUDA(launch_gemm(m_h, wm.w2, nullptr, o_x, g, kEpiAddF32, num_sms_, s));
        if (l + 1 < L) {
            launch_rmsnorm_rows_bf16(nullptr, nullptr, X, layers[l + 1].attn_norm, c.norm_eps, Xn,
                                     S, c.dim, s, XnLo, true, f16);
        }
        tap(l + 1);
    }
}

void Prefill::prepare(const std::vector<LayerWeights>& layers, const KvView& kv,
                      const std::vector<LayerWeights>* layers16, int rows) {
    const bool f16 = precision_ == kPrecisionF16;
    if (f16 && (!layers16 || layers16->size() != layers.size())) {
        throw std::invalid_argument("fp16 prefill needs the fp16 weight copies");
    }
    ensure_rows(rows);
    ensure_weight_maps(f16 ? *layers16 : layers);
    ensure_kv_maps(kv, static_cast<int>(layers.size()));
}

void Prefill::run(const int32_t* ids_dev, int n, int pos0, const uint16_t* embed,
                  const std::vector<LayerWeights>& layers, const KvView& kv, float* x_last,
                  float* taps, cudaStream_t s, const std::vector<LayerWeights>* layers16) {
    const q3_config& c = cfg_;
    if (n <= 0) return;
    const int table_len = kv.table_len ? kv.table_len : kv.n_pages;
    if (pos0 < 0 || pos0 + n > table_len * kPageTokens) {
        throw std::out_of_range("batched prefill past the context length");
    }
    if (kv.rope_len < pos0 + n) throw std::runtime_error("RoPE table shorter than the prompt");
    const int L = static_cast<int>(layers.size());
    prepare(layers, kv, layers16, std::min(n, kMaxChunk));
    if (precision_ == kPrecisionF16 && pos0 > 0) {
        // Cache rows before this prompt (earlier prompts, decoded tokens): their fp16 copies.
        const int pages = (pos0 + kPageTokens - 1) / kPageTokens;
        const int page_elems = c.n_kv_heads * kPageTokens * HD;
        kv_to_f16_kernel<<<dim3(pages, L), 256, 0, s>>>(
            kv.k_base, kv.v_base, static_cast<uint16_t*>(k16_.ptr),
            static_cast<uint16_t*>(v16_.ptr), kv.page_table, layer_elems(kv), page_elems);
        Q3_CUDA(cudaGetLastError());
    }
    const float* X = static_cast<const float*>(x_.ptr);
    for (int c0 = 0; c0 < n; c0 += kMaxChunk) {
        const int S = std::min(kMaxChunk, n - c0);
        const bool last = c0 + S == n;
        PassRows pr;
        pr.p0 = pos0 + c0;
        layer_pass(ids_dev + c0, S, pr, embed, layers, kv, last ? taps : nullptr, s);
        if (last) {
            Q3_CUDA(cudaMemcpyAsync(x_last, X + static_cast<size_t>(S - 1) * c.dim, c.dim * 4,
                                    cudaMemcpyDeviceToDevice, s));
        }
    }
}

void Prefill::run_varlen(const int32_t* ids_dev, const std::vector<int>& offset,
                         const std::vector<int>& len, const std::vector<int>& table_off,
                         const int32_t* table_host, const uint16_t* embed,
                         const std::vector<LayerWeights>& layers, const KvView& kv,
                         float* x_last, cudaStream_t s,
                         const std::vector<LayerWeights>* layers16) {
    const q3_config& c = cfg_;
    const int n_seqs = static_cast<int>(len.size());
    if (n_seqs == 0) return;
    if (offset.size() != len.size() || table_off.size() != len.size() || !table_host) {
        throw std::invalid_argument("varlen prefill: one offset, length and table per sequence");
    }
    const int table_len = kv.table_len ? kv.table_len : kv.n_pages;
    int max_len = 0;
    for (int i = 0; i < n_seqs; ++i) {
        if (len[i] <= 0 || len[i] > kMaxChunk) {
            throw std::out_of_range("varlen prefill: every prompt 1 .. 4096 tokens");
        }
        if (len[i] > table_len * kPageTokens) {
            throw std::out_of_range("batched prefill past the context length");
        }
        max_len = std::max(max_len, len[i]);
    }
    if (kv.rope_len < max_len) throw std::runtime_error("RoPE table shorter than the prompt");
    prepare(layers, kv, layers16, kMaxChunk);
    // Query blocks of one chunk: at most one partial block per sequence beyond the full ones.
    constexpr int kMaxWork = kMaxChunk / 64 + kMaxChunk;
    if (tok_pos_.bytes == 0) {
        tok_pos_.alloc(static_cast<size_t>(kMaxChunk) * 4);
        tok_row_.alloc(static_cast<size_t>(kMaxChunk) * 4);
        work_.alloc(static_cast<size_t>(kMaxWork) * sizeof(int4));
    }
    pinned_varlen_.ensure(static_cast<size_t>(kMaxChunk) * 8 + kMaxWork * sizeof(int4));
    int32_t* h_pos = static_cast<int32_t*>(pinned_varlen_.ptr);
    int32_t* h_row = h_pos + kMaxChunk;
    int4* h_work = reinterpret_cast<int4*>(h_row + kMaxChunk);
    const float* X = static_cast<const float*>(x_.ptr);

    for (int first = 0; first < n_seqs;) {
        // Sequences [first, last): contiguous in ids, together at most one chunk of tokens.
        int last = first, S = 0;
        while (last < n_seqs && S + len[last] <= kMaxChunk &&
               (last == first || offset[last] == offset[last - 1] + len[last - 1])) {
            S += len[last];
            ++last;
        }
        // The pinned staging is reused chunk after chunk: the previous chunk's copies are done.
        Q3_CUDA(cudaStreamSynchronize(s));
        std::vector<int4> items;
        int row = 0;
        for (int i = first; i < last; ++i) {
            const int32_t* tab = table_host + table_off[i];
            for (int p = 0; p < len[i]; ++p) {
                h_pos[row + p] = p;
                h_row[row + p] = tab[p / kPageTokens] * kPageTokens + p % kPageTokens;
            }
            for (int b = 0; b < len[i]; b += 64) {
                items.push_back(make_int4(row + b, std::min(64, len[i] - b), b, table_off[i]));
            }
            row += len[i];
        }
        // Blocks with the most KV positions first (the longest work starts first).
        std::stable_sort(items.begin(), items.end(), [](const int4& a, const int4& b) {
            return a.z + a.y > b.z + b.y;
        });
        if (static_cast<int>(items.size()) > kMaxWork) {
            throw std::runtime_error("varlen prefill: too many query blocks");
        }
        std::copy(items.begin(), items.end(), h_work);
        Q3_CUDA(cudaMemcpyAsync(tok_pos_.ptr, h_pos, static_cast<size_t>(S) * 4,
                                cudaMemcpyHostToDevice, s));
        Q3_CUDA(cudaMemcpyAsync(tok_row_.ptr, h_row, static_cast<size_t>(S) * 4,
                                cudaMemcpyHostToDevice, s));
        Q3_CUDA(cudaMemcpyAsync(work_.ptr, h_work, items.size() * sizeof(int4),
                                cudaMemcpyHostToDevice, s));
        PassRows pr;
        pr.tok_pos = static_cast<const int32_t*>(tok_pos_.ptr);
        pr.tok_row = static_cast<const int32_t*>(tok_row_.ptr);
        pr.work = static_cast<const int4*>(work_.ptr);
        pr.n_work = static_cast<int>(items.size());
        layer_pass(ids_dev + offset[first], S, pr, embed, layers, kv, nullptr, s);
        int r0 = 0;
        for (int i = first; i < last; ++i) {
            r0 += len[i];
            Q3_CUDA(cudaMemcpyAsync(x_last + static_cast<size_t>(i) * c.dim,
                                    X + static_cast<size_t>(r0 - 1) * c.dim, c.dim * 4,
                                    cudaMemcpyDeviceToDevice, s));
        }
        first = last;
    }
}

}  // namespace q3
