// Decode attention over the paged KV cache (see q3_decode_attn.cuh).
//
// Block (sequence b, local KV head g, split s) of 4 warps takes the pages [s*P, (s+1)*P) of b's
// cached positions; warp w takes every 4th of them. Per 16-position page (4 KB of K, 4 KB of V for
// head g) a lane holds 8 dimensions (one 16-byte unit) of 8 of the 16 rows - rows of its parity
// hb = lane / 16 - and computes, for both query heads of the group, the partial dot products of
// those rows; a transposing butterfly over the 16 lanes of each half leaves one score per lane
// (head dl / 8, row 2 (dl % 8) + hb), the page's softmax statistics are warp reductions, and the
// lane then accumulates p * V for its rows and dimensions. The online-softmax states of the warps
// and then of the splits are merged as in flash-decoding; the arithmetic per score follows the
// reference: q . k / sqrtf(128), exp(s - max) (src/inference.cpp:1029-1057, :925-946).
#include <float.h>

#include <algorithm>
#include <stdexcept>

#include "q3_common.cuh"
#include "q3_decode_attn.cuh"

namespace q3 {

namespace {

constexpr int HD = 128;
constexpr int DA_WARPS = 4;
constexpr int DA_THREADS = DA_WARPS * 32;
constexpr int kMaxSplits = 64;  // splits per (sequence, KV head): the merge holds them in smem

__device__ __forceinline__ void unpack8(const uint4 w, float f[8]) {
    f[0] = bf16_lo(w.x);
    f[1] = bf16_hi(w.x);
    f[2] = bf16_lo(w.y);
    f[3] = bf16_hi(w.y);
    f[4] = bf16_lo(w.z);
    f[5] = bf16_hi(w.z);
    f[6] = bf16_lo(w.w);
    f[7] = bf16_hi(w.w);
}

// Writes o (already divided by the softmax sum) at element off of the outputs.
__device__ __forceinline__ void put_out(const DecodeAttnArgs& a, size_t off, float o) {
    if (a.out_f32) a.out_f32[off] = o;
    if (a.out) {
        const uint16_t hi = f32_to_bf16(o);
        a.out[off] = hi;
        if (a.out_lo) a.out_lo[off] = f32_to_bf16(o - bf16_to_f32(hi));
    }
}

__global__ void __launch_bounds__(DA_THREADS) decode_attn_kernel(const DecodeAttnArgs a) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) float s_o[DA_WARPS][2][HD];  // written as float4
    __shared__ float2 s_ml[DA_WARPS][2];
    __shared__ int s_last;
    __shared__ float2 s_pml[2 * kMaxSplits];  // merge: (max, sum) per (split, head)
    __shared__ float s_sc[2 * kMaxSplits];    // merge: scale of each (split, head)
    __shared__ float s_ML[2][2];              // merge: (max, sum) per head
    __shared__ float4 s_half[2][2][HD / 4];   // merge: the two split halves' sums

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = static_cast<int>(blockIdx.x) % a.max_splits;
    const int rg = static_cast<int>(blockIdx.x) / a.max_splits;  // row * n_kv + g
    const int g = rg % a.n_kv, row = rg / a.n_kv;
    const int kv_len = a.dec_pos[row] + 1;
    const int n_pages = (kv_len + kPageTokens - 1) / kPageTokens;
    const int nsplit = (n_pages + a.pages_per_split - 1) / a.pages_per_split;
    if (split >= nsplit) return;
    const int pg0 = split * a.pages_per_split;
    const int pg1 = min(n_pages, pg0 + a.pages_per_split);
    const int32_t* table = a.page_table + static_cast<size_t>(row) * a.pages_per_seq;
    const int gc = a.kv_head0 + g;
    const int hb = lane >> 4, dl = lane & 15;
    const float sq = sqrtf(static_cast<float>(HD));

    // This lane's 8 dimensions of both query heads.
    const float* qp = a.q + static_cast<size_t>(row) * a.q_stride + 2 * g * HD + 8 * dl;
    float q0[8], q1[8];
    {
        const float4 x0 = *reinterpret_cast<const float4*>(qp);
        const float4 x1 = *reinterpret_cast<const float4*>(qp + 4);
        const float4 y0 = *reinterpret_cast<const float4*>(qp + HD);
        const float4 y1 = *reinterpret_cast<const float4*>(qp + HD + 4);
        q0[0] = x0.x; q0[1] = x0.y; q0[2] = x0.z; q0[3] = x0.w;
        q0[4] = x1.x; q0[5] = x1.y; q0[6] = x1.z; q0[7] = x1.w;
        q1[0] = y0.x; q1[1] = y0.y; q1[2] = y0.z; q1[3] = y0.w;
        q1[4] = y1.x; q1[5] = y1.y; q1[6] = y1.z; q1[7] = y1.w;
    }

    float m[2] = {-FLT_MAX, -FLT_MAX}, l[2] = {0.0f, 0.0f};
    float o[2][8];
#pragma unroll
    for (int d = 0; d < 8; ++d) o[0][d] = o[1][d] = 0.0f;

    for (int pg = pg0 + warp; pg < pg1; pg += DA_WARPS) {
        const size_t base =
            (static_cast<size_t>(__ldg(table + pg)) * a.n_kv_cache + gc) * kPageTokens * HD;
        const uint4* kp = reinterpret_cast<const uint4*>(a.k_cache + base);
        const uint4* vp = reinterpret_cast<const uint4*>(a.v_cache + base);
        const int t0 = pg * kPageTokens;
        uint4 kr[8], vr[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool valid = t0 + 2 * i + hb < kv_len;
            kr[i] = valid ? ldg_stream(kp + (2 * i + hb) * (HD / 8) + dl) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool valid = t0 + 2 * i + hb < kv_len;
            vr[i] = valid ? ldg_stream(vp + (2 * i + hb) * (HD / 8) + dl) : make_uint4(0, 0, 0, 0);
        }
        // Partial scores sv[h * 8 + i] of row 2i + hb over this lane's 8 dimensions.
        float sv[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float kf[8];
            unpack8(kr[i], kf);
            float d0 = kf[0] * q0[0], d1 = kf[0] * q1[0];
#pragma unroll
            for (int d = 1; d < 8; ++d) {
                d0 = fmaf(kf[d], q0[d], d0);
                d1 = fmaf(kf[d], q1[d], d1);
            }
            sv[i] = d0;
            sv[8 + i] = d1;
        }
        // Transposing butterfly over the 16 lanes of this half: lane dl ends with the full sum of
        // entry dl (head dl >> 3, row 2 (dl & 7) + hb).
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool up = dl & 8;
            const float send = up ? sv[i] : sv[8 + i];
            const float keep = up ? sv[8 + i] : sv[i];
            sv[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const bool up = dl & 4;
            const float send = up ? sv[i] : sv[4 + i];
            const float keep = up ? sv[4 + i] : sv[i];
            sv[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const bool up = dl & 2;
            const float send = up ? sv[i] : sv[2 + i];
            const float keep = up ? sv[2 + i] : sv[i];
            sv[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
        float dot;
        {
            const bool up = dl & 1;
            const float send = up ? sv[0] : sv[1];
            const float keep = up ? sv[1] : sv[0];
            dot = keep + __shfl_xor_sync(0xffffffffu, send, 1);
        }
        const int my_h = dl >> 3;
        const bool my_valid = t0 + 2 * (dl & 7) + hb < kv_len;
        const float s = my_valid ? dot / sq : -FLT_MAX;
        // Page maximum of this lane's head: the 16 lanes with the same bit 3.
        float mx = s;
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mx_other = __shfl_xor_sync(0xffffffffu, mx, 8);
        const float mx0 = my_h ? mx_other : mx, mx1 = my_h ? mx : mx_other;
        const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
        const float p = my_valid ? expf(s - (my_h ? mn1 : mn0)) : 0.0f;
        float ps = p;
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        ps += __shfl_xor_sync(0xffffffffu, ps, 16);
        const float ps_other = __shfl_xor_sync(0xffffffffu, ps, 8);
        const float ps0 = my_h ? ps_other : ps, ps1 = my_h ? ps : ps_other;
        const float al0 = expf(m[0] - mn0), al1 = expf(m[1] - mn1);
        l[0] = l[0] * al0 + ps0;
        l[1] = l[1] * al1 + ps1;
        m[0] = mn0;
        m[1] = mn1;
#pragma unroll
        for (int d = 0; d < 8; ++d) {
            o[0][d] *= al0;
            o[1][d] *= al1;
        }
        // o[h] += p(h, row 2i + hb) * V[row] over this lane's rows.
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float p0 = __shfl_sync(0xffffffffu, p, hb * 16 + i);
            const float p1 = __shfl_sync(0xffffffffu, p, hb * 16 + 8 + i);
            float vf[8];
            unpack8(vr[i], vf);
#pragma unroll
            for (int d = 0; d < 8; ++d) {
                o[0][d] = fmaf(p0, vf[d], o[0][d]);
                o[1][d] = fmaf(p1, vf[d], o[1][d]);
            }
        }
    }
    // The two row parities of the warp hold the same dimensions.
#pragma unroll
    for (int d = 0; d < 8; ++d) {
        o[0][d] += __shfl_xor_sync(0xffffffffu, o[0][d], 16);
        o[1][d] += __shfl_xor_sync(0xffffffffu, o[1][d], 16);
    }
    if (hb == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            *reinterpret_cast<float4*>(&s_o[warp][h][8 * dl]) =
                make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
            *reinterpret_cast<float4*>(&s_o[warp][h][8 * dl + 4]) =
                make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
        }
    }
    if (lane == 0) {
        s_ml[warp][0] = make_float2(m[0], l[0]);
        s_ml[warp][1] = make_float2(m[1], l[1]);
    }
    __syncthreads();

    // Merge the warps: thread t holds (head t / 64, dimensions 2 (t % 64), +1).
    const int h = tid >> 6, d2 = 2 * (tid & 63);
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < DA_WARPS; ++w)
        if (s_ml[w][h].y > 0.0f) M = fmaxf(M, s_ml[w][h].x);
    float L = 0.0f, oa = 0.0f, ob = 0.0f;
#pragma unroll
    for (int w = 0; w < DA_WARPS; ++w) {
        const float2 ml = s_ml[w][h];
        if (ml.y > 0.0f) {
            const float sc = expf(ml.x - M);
            L += ml.y * sc;
            oa += s_o[w][h][d2] * sc;
            ob += s_o[w][h][d2 + 1] * sc;
        }
    }
    const size_t out_off = static_cast<size_t>(row) * a.out_stride + (2 * g + h) * HD + d2;
    if (nsplit == 1) {
        put_out(a, out_off, oa / L);
        put_out(a, out_off + 1, ob / L);
        return;
    }
    const size_t pi = (static_cast<size_t>(rg) * a.max_splits + split) * 2 + h;
    *reinterpret_cast<float2*>(a.part_o + pi * HD + d2) = make_float2(oa, ob);
    if ((tid & 63) == 0) a.part_ml[pi] = make_float2(M, L);

    // The last split of (row, g) to finish merges all of them.
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(a.counter + rg, 1u);
        s_last = prev == static_cast<unsigned>(nsplit - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Merge the splits: their (max, sum) pairs through shared memory, then each thread sums one
    // head's 4 dimensions over every other split.
    const size_t pb = static_cast<size_t>(rg) * a.max_splits * 2;
    if (tid < 2 * nsplit) s_pml[tid] = __ldcg(a.part_ml + pb + tid);
    __syncthreads();
    if (tid < 2) {
        float MM = -FLT_MAX;
        for (int sp = 0; sp < nsplit; ++sp) {
            const float2 ml = s_pml[2 * sp + tid];
            if (ml.y > 0.0f) MM = fmaxf(MM, ml.x);
        }
        float LL = 0.0f;
        for (int sp = 0; sp < nsplit; ++sp) {
            const float2 ml = s_pml[2 * sp + tid];
            if (ml.y > 0.0f) LL += ml.y * expf(ml.x - MM);
        }
        s_ML[tid][0] = MM;
        s_ML[tid][1] = LL;
    }
    __syncthreads();
    if (tid < 2 * nsplit) {
        const float2 ml = s_pml[tid];
        s_sc[tid] = ml.y > 0.0f ? expf(ml.x - s_ML[tid & 1][0]) : 0.0f;
    }
    __syncthreads();
    {
        const int half = tid >> 6, hh = (tid >> 5) & 1, quad = tid & 31;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 4
        for (int sp = half; sp < nsplit; sp += 2) {
            const float sc = s_sc[2 * sp + hh];
            const float4 v = __ldcg(reinterpret_cast<const float4*>(
                a.part_o + (pb + 2 * sp + hh) * HD) + quad);
            acc.x = fmaf(v.x, sc, acc.x);
            acc.y = fmaf(v.y, sc, acc.y);
            acc.z = fmaf(v.z, sc, acc.z);
            acc.w = fmaf(v.w, sc, acc.w);
        }
        s_half[half][hh][quad] = acc;
    }
    __syncthreads();
    if (tid < 64) {
        const int hh = tid >> 5, quad = tid & 31;
        const float4 u = s_half[0][hh][quad], v = s_half[1][hh][quad];
        const float inv = 1.0f / s_ML[hh][1];
        const size_t off = static_cast<size_t>(row) * a.out_stride + (2 * g + hh) * HD + 4 * quad;
        put_out(a, off, (u.x + v.x) * inv);
        put_out(a, off + 1, (u.y + v.y) * inv);
        put_out(a, off + 2, (u.z + v.z) * inv);
        put_out(a, off + 3, (u.w + v.w) * inv);
    }
    if (tid == 0) a.counter[rg] = 0u;
}

}  // namespace

int decode_attn_pages_per_split(int rows, int n_kv, int max_pages, int num_sms) {
    // Short splits (8 pages and up) and up to ~32 blocks per SM when every pair is at its longest:
    // the blocks of short sequences end early and the scheduler fills the SMs with the rest. At
    // most kMaxSplits splits per pair (the merge holds them in shared memory).
    const long long pairs = static_cast<long long>(rows) * n_kv;
    const long long target = 32LL * num_sms;
    int pps = 8;
    while ((pps < 64 && pairs * ((max_pages + pps - 1) / pps) > target) ||
           (max_pages + pps - 1) / pps > kMaxSplits) {
        pps *= 2;
    }
    return pps;
}

void launch_decode_attention(const DecodeAttnArgs& a, cudaStream_t s) {
    if (a.rows <= 0) return;
    if (a.max_splits < 1 || a.max_splits > kMaxSplits || a.pages_per_split < 1) {
        throw std::invalid_argument("decode attention: 1..64 splits of at least one page");
    }
    const dim3 grid(static_cast<unsigned>(a.rows * a.n_kv * a.max_splits));
    launch_dep(false, decode_attn_kernel, grid, dim3(DA_THREADS), 0, s, a);
    Q3_CUDA(cudaGetLastError());
}

}  // namespace q3
