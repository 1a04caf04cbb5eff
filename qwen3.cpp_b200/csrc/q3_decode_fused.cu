// Fused whole-step decode for the Qwen3-0.6B shape on B200 (sm_100a).
//
// One persistent cooperative launch (one CTA per SM) runs n_steps greedy decode steps. Each step
// is the reference's ForwardToken (asriva32/Qwen3.cpp src/inference.cpp:592-637) + Greedy
// (:703-709): 28 x Block::forward (:766-866), final RmsNorm, tied lm_head, argmax.
//
// Dataflow. Decode at batch 1 streams 1.19 GB of bf16 weights per token, so the kernel is built
// around one continuous weight stream per SM: a producer warp walks the fixed sequence of weight
// row-chunks this CTA owns for the whole call (layer by layer: [wq;wk;wv], wo, w1|w3 pairs, w2,
// then lm_head rows) and copies them with TMA bulk copies (cp.async.bulk, no multicast) into a
// 32-slot shared-memory ring guarded by full/empty mbarriers. It never waits for activations, so
// the stream runs ahead across the grid-wide dependencies. Eight consumer warps wait for the
// activation vector of each phase (a monotonic arrival counter in global memory, acquire/release),
// stage it in shared memory (with the RMSNorm fused in), and dot it with the weight rows as they
// land. Phases per layer:
//   A  x -> RmsNorm -> qkv = [wq;wk;wv] . xn                     (:795-798)
//   B  per (KV head, split): QK-RMSNorm + RoPE of q/k, bf16 K/V write at kv_pos, attention-sink
//      re-rotation, split-K attention over the paged KV cache     (:800-844)
//   C  combine splits; x += wo . attn                              (:846-849)
//   D  x -> RmsNorm -> h = silu(w1 . xn) * (w3 . xn)               (:851, :1005-1011)
//   E  x += w2 . h                                                 (:1013, :863-865)
// then the final RmsNorm + lm_head with a per-CTA argmax; the next step (or the host) reduces the
// per-CTA (value, index) pairs, lowest index winning ties.
//
// Every wait is bounded (clock64): on timeout the kernel sets *err, stops issuing copies, waits
// for the copies already issued and returns; the host reports Q3_ERR_DEVICE_TIMEOUT.
#include <cuda_runtime.h>
#include <float.h>
#include <limits.h>

#include "q3_decode_fused.cuh"

namespace q3 {

namespace {

constexpr int D = 1024, H = 3072, NQ = 16, NKV = 8, HD = 128;
constexpr int QD = NQ * HD, KVD = NKV * HD, QKV_ROWS = QD + 2 * KVD;
constexpr int NCW = 8;                 // consumer warps
constexpr int NCT = NCW * 32;          // consumer threads
constexpr int NT = NCT + 32;           // + one producer warp
constexpr int NS = 32;                 // ring slots
constexpr int SLOT = 6144;             // bytes per slot
constexpr int ATT_TOK = 24;            // KV positions staged per attention sub-chunk

enum Mode : int { kStore = 0, kResid = 1, kPair = 2, kLogits = 3 };

struct __align__(128) Smem {
    uint8_t ring[NS][SLOT];
    float4 xs4[H / 4];        // staged activation, permuted per 8-element vector (see stage_*)
    float xres[D];            // residual-stream copy for the o/down epilogues
    float qk[3][HD];          // normalised + rotated q heads (2) and k head of a KV group
    float2 mlw[NCW][2];       // per-warp attention (max, sum)
    float red[NCW];
    float2 best[NCW];
    uint64_t full[NS];
    uint64_t empty[NS];
    int abort_flag;
    int token;
    int go;
};

// ------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// 1-D TMA bulk copy global -> this CTA's shared memory, completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void bar_consumers() {
    asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// ------------------------------------------------------------------ bounded waits

__device__ bool mbar_wait(uint64_t* b, uint32_t parity, const FusedArgs& a, volatile int* abort) {
    if (mbar_try_wait(b, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(b, parity)) return true;
        if ((it & 31) == 31) {
            if (*abort) return false;
            if (clock64() - t0 > a.spin_cycles) {
                *abort = 1;
                atomicOr(a.err, 1u);
                return false;
            }
        }
    }
}

// Consumer thread 0: wait until `target` CTAs have arrived on the grid counter.
__device__ bool grid_wait(const FusedArgs& a, unsigned target, volatile int* abort) {
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        if (ld_acquire(a.bar) >= target) return true;
        if (*reinterpret_cast<volatile unsigned*>(a.err) != 0u) {
            *abort = 1;
            return false;
        }
        if (clock64() - t0 > a.spin_cycles) {
            *abort = 1;
            atomicOr(a.err, 1u);
            return false;
        }
        if (it > 16) __nanosleep(32);
    }
}

// ------------------------------------------------------------------ work partition

struct Span {
    int r0, n;
};
__device__ __forceinline__ Span part(int rows, int G, int c) {
    const int r0 = static_cast<int>((static_cast<long long>(rows) * c) / G);
    const int r1 = static_cast<int>((static_cast<long long>(rows) * (c + 1)) / G);
    return {r0, r1 - r0};
}
template <int K, int MODE>
struct Chunking {
    // Rows (or gate/up pairs) per ring slot.
    static constexpr int RPC = MODE == kPair ? SLOT / (2 * K * 2) : SLOT / (K * 2);
    static_assert(RPC >= 1, "slot too small");
};

__device__ __forceinline__ size_t paged(const int32_t* table, int t, int g) {
    const int page = __ldg(table + t / kPageTokens);
    return ((static_cast<size_t>(page) * NKV + g) * kPageTokens + (t % kPageTokens)) * HD;
}

// ------------------------------------------------------------------ producer

struct Producer {
    Smem& sm;
    const FusedArgs& a;
    uint64_t pol;
    uint32_t q = 0;

    __device__ bool issue(const void* s1, uint32_t b1, const void* s2, uint32_t b2, int off2) {
        const int slot = q % NS;
        if (q >= NS && !mbar_wait(&sm.empty[slot], ((q / NS) - 1) & 1, a, &sm.abort_flag)) {
            return false;
        }
        mbar_arrive_expect_tx(&sm.full[slot], b1 + b2);
        bulk_g2s(sm.ring[slot], s1, b1, &sm.full[slot], pol);
        if (b2) bulk_g2s(sm.ring[slot] + off2, s2, b2, &sm.full[slot], pol);
        ++q;
        return true;
    }

    template <int K, int MODE>
    __device__ bool rows(const uint16_t* w, const uint16_t* w2, Span sp) {
        constexpr int RPC = Chunking<K, MODE>::RPC;
        for (int rb = sp.r0; rb < sp.r0 + sp.n; rb += RPC) {
            const int rn = min(RPC, sp.r0 + sp.n - rb);
            const uint32_t bytes = static_cast<uint32_t>(rn) * K * 2;
            const size_t off = static_cast<size_t>(rb) * K;
            if (!issue(w + off, bytes, MODE == kPair ? w2 + off : nullptr,
                       MODE == kPair ? bytes : 0u, RPC * K * 2)) {
                return false;
            }
        }
        return true;
    }

    __device__ void run(int G, int c) {
        pol = evict_first_policy();
        bool ok = true;
        for (int st = 0; ok && st < a.n_steps; ++st) {
            for (int l = 0; ok && l < a.n_layers; ++l) {
                const LayerWeights w = a.layers[l];
                ok = ok && rows<D, kStore>(w.wqkv, nullptr, part(QKV_ROWS, G, c));
                ok = ok && rows<QD, kResid>(w.wo, nullptr, part(D, G, c));
                ok = ok && rows<D, kPair>(w.w1, w.w3, part(H, G, c));
                ok = ok && rows<H, kResid>(w.w2, nullptr, part(D, G, c));
            }
            ok = ok && rows<D, kLogits>(a.lm_head, nullptr, part(a.vocab, G, c));
        }
        // Wait for every copy still in flight before the CTA may exit.
        const uint32_t first = q > NS ? q - NS : 0;
        for (uint32_t k = first; k < q; ++k) {
            const int slot = k % NS;
            const long long t0 = clock64();
            while (!mbar_try_wait(&sm.full[slot], (k / NS) & 1)) {
                if (clock64() - t0 > a.spin_cycles) break;
            }
        }
    }
};

// ------------------------------------------------------------------ consumer helpers

__device__ __forceinline__ float consumer_sum(float v, Smem& sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) sm.red[warp] = v;
    bar_consumers();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) t += sm.red[w];
    bar_consumers();
    return t;
}

// Stage a 1024-vector for a K=1024 GEMV: xres = x, xs = RmsNorm(x, nw) (src/inference.cpp:887-923)
// in the permuted layout xs4[v] = x[8v..8v+3], xs4[128+v] = x[8v+4..8v+7].
__device__ void stage_norm(Smem& sm, float4 xv, const uint16_t* nw, float eps) {
    const int t = threadIdx.x;
    reinterpret_cast<float4*>(sm.xres)[t] = xv;
    const float ss = consumer_sum(xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w, sm);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
    const uint2 wv = __ldg(reinterpret_cast<const uint2*>(nw) + t);
    float4 y;
    y.x = (xv.x * inv) * bf16_lo(wv.x);
    y.y = (xv.y * inv) * bf16_hi(wv.x);
    y.z = (xv.z * inv) * bf16_lo(wv.y);
    y.w = (xv.w * inv) * bf16_hi(wv.y);
    sm.xs4[(t & 1) * (D / 8) + (t >> 1)] = y;
    bar_consumers();
}

__device__ __forceinline__ float4 load_x_global(const FusedArgs& a) {
    return __ldcg(reinterpret_cast<const float4*>(a.x) + threadIdx.x);
}

__device__ __forceinline__ float4 load_embed(const FusedArgs& a, int token) {
    const uint2 e = __ldg(reinterpret_cast<const uint2*>(a.embed + static_cast<size_t>(token) * D) +
                          threadIdx.x);
    return make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
}

// Dot the rows of this CTA's chunks of one task with the staged activation. After an abort the
// remaining chunks are skipped (each wait then fails at once), but the warp still returns to the
// caller so that every consumer thread reaches the same barriers.
template <int K, int MODE>
__device__ void consume(Smem& sm, const FusedArgs& a, uint32_t& q, Span sp, float* out,
                        float& best_v, int& best_i) {
    constexpr int RPC = Chunking<K, MODE>::RPC;
    constexpr int NV = K / 8;  // 16-byte vectors per row
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nch = (sp.n + RPC - 1) / RPC;
    for (int ci = 0; ci < nch; ++ci) {
        const uint32_t qq = q + ci;
        if (static_cast<int>(qq % NCW) != warp) continue;
        const int slot = qq % NS;
        const uint32_t parity = (qq / NS) & 1;
        // Lane 0 does the bounded wait; the verdict is made warp-uniform before any shuffle.
        int ok = lane == 0 ? static_cast<int>(mbar_wait(&sm.full[slot], parity, a, &sm.abort_flag)) : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) continue;
        // Every lane observes the completed phase (the copy's bytes are then visible to it); the
        // phase cannot advance again before this warp releases the slot, so this returns at once.
        while (!mbar_try_wait(&sm.full[slot], parity)) {
        }
        const uint8_t* base = sm.ring[slot];
        const int rb = sp.r0 + ci * RPC;
        const int rn = min(RPC, sp.r0 + sp.n - rb);
        for (int j = 0; j < rn; ++j) {
            const uint4* wrow = reinterpret_cast<const uint4*>(base + j * K * 2);
            const uint4* urow = reinterpret_cast<const uint4*>(base + (RPC + j) * K * 2);
            float acc = 0.0f, acc2 = 0.0f;
#pragma unroll
            for (int v = lane; v < NV; v += 32) {
                const uint4 w = wrow[v];
                const float4 xa = sm.xs4[v];
                const float4 xb = sm.xs4[NV + v];
                acc = dot8(w, xa, xb, acc);
                if (MODE == kPair) acc2 = dot8(urow[v], xa, xb, acc2);
            }
            acc = warp_sum(acc);
            if (MODE == kPair) acc2 = warp_sum(acc2);
            const int r = rb + j;
            if (lane == 0) {
                if (MODE == kStore || MODE == kLogits) out[r] = acc;
                if (MODE == kResid) out[r] = sm.xres[r] + acc;
                if (MODE == kPair) out[r] = silu(acc) * acc2;
            }
            if (MODE == kLogits && better(acc, r, best_v, best_i)) {
                best_v = acc;
                best_i = r;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
    q += nch;
}

// RoPE on a 128-vector spread over a warp, 4 elements per lane: lanes 0-15 hold the first half,
// lanes 16-31 the second; pairs (i, i+64) sit 16 lanes apart (src/inference.cpp:976-990).
__device__ __forceinline__ void rope_warp(float y[4], const float2* row) {
    const int lane = threadIdx.x & 31;
    const bool first = lane < 16;
    const int i0 = (lane & 15) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float p = __shfl_xor_sync(0xffffffffu, y[j], 16);
        const float2 cs = __ldg(row + i0 + j);
        y[j] = first ? (y[j] * cs.x - p * cs.y) : (y[j] * cs.x + p * cs.y);
    }
}

__device__ __forceinline__ uint2 pack_bf16x4(const float y[4]) {
    return make_uint2(static_cast<uint32_t>(f32_to_bf16(y[0])) |
                          (static_cast<uint32_t>(f32_to_bf16(y[1])) << 16),
                      static_cast<uint32_t>(f32_to_bf16(y[2])) |
                          (static_cast<uint32_t>(f32_to_bf16(y[3])) << 16));
}

struct StepPos {
    int pos, num_sink, kv_pos, kv_len, splits;
};

// Phase B for one (KV head, split) item of this CTA.
__device__ void attention_item(Smem& sm, const FusedArgs& a, const LayerWeights& w, int l,
                               const StepPos& p, int item) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = p.splits;
    const int g = item % NKV, s = item / NKV;
    const int chunk = (p.kv_len + S - 1) / S;
    const int t0 = s * chunk, t1 = min(p.kv_len, t0 + chunk);
    const bool own = p.kv_pos >= t0 && p.kv_pos < t1;
    uint16_t* kc = a.k_cache + static_cast<size_t>(l) * a.layer_elems;
    uint16_t* vc = a.v_cache + static_cast<size_t>(l) * a.layer_elems;
    const int rp = min(p.pos, a.rope_len - 1);

    if (warp < 3) {
        // QK-RMSNorm (src/inference.cpp:800-807) + RoPE (:809-810) of q heads 2g, 2g+1 and k head g.
        const float* src = warp < 2 ? a.qkv + (2 * g + warp) * HD : a.qkv + QD + g * HD;
        const float4 e = __ldcg(reinterpret_cast<const float4*>(src) + lane);
        const float ss = warp_sum(e.x * e.x + e.y * e.y + e.z * e.z + e.w * e.w);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(HD) + a.eps);
        const uint2 wv = __ldg(reinterpret_cast<const uint2*>(warp < 2 ? w.q_norm : w.k_norm) + lane);
        float y[4] = {(e.x * inv) * bf16_lo(wv.x), (e.y * inv) * bf16_hi(wv.x),
                      (e.z * inv) * bf16_lo(wv.y), (e.w * inv) * bf16_hi(wv.y)};
        rope_warp(y, a.rope + static_cast<size_t>(rp) * (HD / 2));
        reinterpret_cast<float4*>(sm.qk[warp])[lane] = make_float4(y[0], y[1], y[2], y[3]);
        if (warp == 2 && own) {
            // bf16 K write at kv_pos (:812-815).
            reinterpret_cast<uint2*>(kc + paged(a.page_table, p.kv_pos, g))[lane] = pack_bf16x4(y);
        }
    } else if (warp == 3) {
        if (own) {
            const float4 e = __ldcg(reinterpret_cast<const float4*>(a.qkv + QD + KVD + g * HD) + lane);
            const float y[4] = {e.x, e.y, e.z, e.w};
            reinterpret_cast<uint2*>(vc + paged(a.page_table, p.kv_pos, g))[lane] = pack_bf16x4(y);
        }
    } else if (s == 0 && warp - 4 < p.num_sink) {
        // Attention-sink re-rotation once the ring buffer has wrapped (:817-827).
        uint2* row = reinterpret_cast<uint2*>(kc + paged(a.page_table, warp - 4, g));
        const uint2 v = __ldcg(row + lane);
        float y[4] = {bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y)};
        rope_warp(y, a.rope + static_cast<size_t>(1) * (HD / 2));
        row[lane] = pack_bf16x4(y);
    }
    bar_consumers();

    // Split-K attention over positions [t0, t1) for the two query heads of KV head g
    // (FastAttn + Softmax, :1017-1058, :925-946), online softmax per warp.
    const float4 q0 = reinterpret_cast<const float4*>(sm.qk[0])[lane];
    const float4 q1 = reinterpret_cast<const float4*>(sm.qk[1])[lane];
    const float sq = sqrtf(static_cast<float>(HD));
    float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.0f, l1 = 0.0f;
    float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
    uint4* stage = reinterpret_cast<uint4*>(sm.xs4);  // [ATT_TOK][K 16 | V 16] uint4
    for (int tb = t0; tb < t1; tb += ATT_TOK) {
        const int n = min(ATT_TOK, t1 - tb);
        for (int idx = tid; idx < n * 32; idx += NCT) {
            const int tok = idx >> 5, kind = (idx >> 4) & 1, vec = idx & 15;
            const uint16_t* src = (kind ? vc : kc) + paged(a.page_table, tb + tok, g);
            stage[idx] = __ldcg(reinterpret_cast<const uint4*>(src) + vec);
        }
        bar_consumers();
        for (int tok = warp; tok < n; tok += NCW) {
            const uint2 kk = reinterpret_cast<const uint2*>(stage + tok * 32)[lane];
            const uint2 vv = reinterpret_cast<const uint2*>(stage + tok * 32 + 16)[lane];
            const float k4[4] = {bf16_lo(kk.x), bf16_hi(kk.x), bf16_lo(kk.y), bf16_hi(kk.y)};
            const float v4[4] = {bf16_lo(vv.x), bf16_hi(vv.x), bf16_lo(vv.y), bf16_hi(vv.y)};
            float d0 = k4[0] * q0.x;
            d0 = fmaf(k4[1], q0.y, d0);
            d0 = fmaf(k4[2], q0.z, d0);
            d0 = fmaf(k4[3], q0.w, d0);
            float d1 = k4[0] * q1.x;
            d1 = fmaf(k4[1], q1.y, d1);
            d1 = fmaf(k4[2], q1.z, d1);
            d1 = fmaf(k4[3], q1.w, d1);
            const float s0 = warp_sum(d0) / sq, s1 = warp_sum(d1) / sq;
            const float n0 = fmaxf(m0, s0), n1 = fmaxf(m1, s1);
            const float a0 = expf(m0 - n0), a1 = expf(m1 - n1);
            const float p0 = expf(s0 - n0), p1 = expf(s1 - n1);
            l0 = l0 * a0 + p0;
            l1 = l1 * a1 + p1;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                o0[j] = o0[j] * a0 + p0 * v4[j];
                o1[j] = o1[j] * a1 + p1 * v4[j];
            }
            m0 = n0;
            m1 = n1;
        }
        bar_consumers();
    }
    // Merge the warps and write this split's partial (max, sum, unnormalised output).
    float* mb = reinterpret_cast<float*>(sm.xs4);  // [NCW][2][HD]
    reinterpret_cast<float4*>(mb + (warp * 2 + 0) * HD)[lane] = make_float4(o0[0], o0[1], o0[2], o0[3]);
    reinterpret_cast<float4*>(mb + (warp * 2 + 1) * HD)[lane] = make_float4(o1[0], o1[1], o1[2], o1[3]);
    if (lane == 0) {
        sm.mlw[warp][0] = make_float2(m0, l0);
        sm.mlw[warp][1] = make_float2(m1, l1);
    }
    bar_consumers();
    {
        const int hq = tid >> 7, d = tid & (HD - 1);
        float M = -FLT_MAX;
#pragma unroll
        for (int w2 = 0; w2 < NCW; ++w2)
            if (sm.mlw[w2][hq].y > 0.0f) M = fmaxf(M, sm.mlw[w2][hq].x);
        float L = 0.0f, acc = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < NCW; ++w2) {
            const float2 ml = sm.mlw[w2][hq];
            if (ml.y > 0.0f) {
                const float sc = expf(ml.x - M);
                L += ml.y * sc;
                acc += mb[(w2 * 2 + hq) * HD + d] * sc;
            }
        }
        const size_t pi = static_cast<size_t>(2 * g + hq) * a.s_max + s;
        a.part_o[pi * HD + d] = acc;
        if (d == 0) a.part_ml[pi] = make_float2(M, L);
    }
}

// Phase C prologue: merge the split partials of all 16 heads into the staged attention output
// (permuted layout for K = 2048).
__device__ void stage_attention(Smem& sm, const FusedArgs& a, int S) {
    const int t = threadIdx.x;
    const int head = t >> 4, d0 = (t & 15) * 8;
    float M = -FLT_MAX;
    for (int s = 0; s < S; ++s) {
        const float2 ml = __ldcg(a.part_ml + head * a.s_max + s);
        if (ml.y > 0.0f) M = fmaxf(M, ml.x);
    }
    float L = 0.0f;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < S; ++s) {
        const size_t pi = static_cast<size_t>(head) * a.s_max + s;
        const float2 ml = __ldcg(a.part_ml + pi);
        if (ml.y > 0.0f) {
            const float sc = expf(ml.x - M);
            L += ml.y * sc;
            const float4 u = __ldcg(reinterpret_cast<const float4*>(a.part_o + pi * HD + d0));
            const float4 v = __ldcg(reinterpret_cast<const float4*>(a.part_o + pi * HD + d0 + 4));
            acc[0] += u.x * sc; acc[1] += u.y * sc; acc[2] += u.z * sc; acc[3] += u.w * sc;
            acc[4] += v.x * sc; acc[5] += v.y * sc; acc[6] += v.z * sc; acc[7] += v.w * sc;
        }
    }
    const int vidx = (head * HD + d0) / 8;
    sm.xs4[vidx] = make_float4(acc[0] / L, acc[1] / L, acc[2] / L, acc[3] / L);
    sm.xs4[QD / 8 + vidx] = make_float4(acc[4] / L, acc[5] / L, acc[6] / L, acc[7] / L);
    bar_consumers();
}

// Phase E prologue: stage h (K = 3072) in the permuted layout.
__device__ void stage_h(Smem& sm, const FusedArgs& a) {
    const int t = threadIdx.x;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int f = t + k * NCT;  // float4 index: elements 4f..4f+3
        sm.xs4[(f & 1) * (H / 8) + (f >> 1)] = __ldcg(reinterpret_cast<const float4*>(a.h) + f);
    }
    bar_consumers();
}

// Greedy argmax over the per-CTA partials (consumer warp 0), lowest index on ties.
__device__ int reduce_argmax(const FusedArgs& a, int G) {
    const int lane = threadIdx.x & 31;
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int i = lane; i < G; i += 32) {
        const float2 p = __ldcg(a.am_part + i);
        const int j = __float_as_int(p.y);
        if (better(p.x, j, bv, bi)) {
            bv = p.x;
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
    return bi == INT_MAX ? 0 : bi;
}

__global__ void __launch_bounds__(NT, 1) decode_fused_kernel(const FusedArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;

    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        sm.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == NCW) {
        if (lane == 0) {
            Producer pr{sm, a};
            pr.run(G, c);
        }
        return;
    }

    // ---------------- consumers
    const StepParams sp0 = *a.sp;
    unsigned k = 0;  // global phase index
    uint32_t q = 0;  // ring chunk index
    float dummy_v = 0.0f;
    int dummy_i = 0;
    volatile int* abort = &sm.abort_flag;

    // Phase entry: thread 0 waits for the previous phase grid-wide and publishes one verdict
    // that every consumer thread reads after the same barrier (so all leave together on abort).
    auto begin = [&](unsigned kk) -> bool {
        if (tid == 0) {
            const bool ok = kk == 0 || grid_wait(a, G * kk + a.barrier_offset, abort);
            sm.go = ok && *abort == 0;
        }
        bar_consumers();
        return sm.go != 0;
    };
    auto end = [&]() {
        bar_consumers();
        if (tid == 0) {
            __threadfence();
            atomicAdd(a.bar, 1u);
        }
    };

    for (int st = 0; st < a.n_steps; ++st) {
        StepPos p;
        p.pos = sp0.pos + st;
        step_positions(p.pos, a.ctx, &p.num_sink, &p.kv_pos, &p.kv_len);
        p.splits = min(max((p.kv_len + ATT_TOK - 1) / ATT_TOK, 1), a.s_max);
        for (int l = 0; l < a.n_layers; ++l) {
            const LayerWeights w = a.layers[l];
            // ---- A: x -> RmsNorm -> [wq;wk;wv]
            if (!begin(k++)) return;
            float4 xv;
            if (l == 0) {
                if (warp == 0) {
                    int tok = sp0.token;
                    if (st > 0) {
                        const int best = reduce_argmax(a, G);
                        const int idx = sp0.step + st;
                        tok = (a.forced && idx < sp0.n_forced) ? __ldg(a.forced + idx) : best;
                        if (c == 0 && lane == 0) a.token_log[idx - 1] = best;
                    }
                    if (lane == 0) sm.token = tok;
                }
                bar_consumers();
                xv = load_embed(a, sm.token);
            } else {
                xv = load_x_global(a);
            }
            if (a.taps && c == 0) reinterpret_cast<float4*>(a.taps + static_cast<size_t>(l) * D)[tid] = xv;
            stage_norm(sm, xv, w.attn_norm, a.eps);
            consume<D, kStore>(sm, a, q, part(QKV_ROWS, G, c), a.qkv, dummy_v, dummy_i);
            end();
            // ---- B: QK-norm, RoPE, KV write, attention partials
            if (!begin(k++)) return;
            if (c < NKV * p.splits) attention_item(sm, a, w, l, p, c);
            end();
            // ---- C: combine, x += wo . attn
            if (!begin(k++)) return;
            stage_attention(sm, a, p.splits);
            consume<QD, kResid>(sm, a, q, part(D, G, c), a.x, dummy_v, dummy_i);
            end();
            // ---- D: x -> RmsNorm -> silu(w1 .) * (w3 .)
            if (!begin(k++)) return;
            stage_norm(sm, load_x_global(a), w.mlp_norm, a.eps);
            consume<D, kPair>(sm, a, q, part(H, G, c), a.h, dummy_v, dummy_i);
            end();
            // ---- E: x += w2 . h
            if (!begin(k++)) return;
            stage_h(sm, a);
            consume<H, kResid>(sm, a, q, part(D, G, c), a.x, dummy_v, dummy_i);
            end();
        }
        // ---- final RmsNorm + lm_head + per-CTA argmax
        if (!begin(k++)) return;
        const float4 xv = load_x_global(a);
        if (a.taps && c == 0) {
            reinterpret_cast<float4*>(a.taps + static_cast<size_t>(a.n_layers) * D)[tid] = xv;
        }
        stage_norm(sm, xv, a.final_norm, a.eps);
        float bv = -FLT_MAX;
        int bi = INT_MAX;
        consume<D, kLogits>(sm, a, q, part(a.vocab, G, c), a.logits, bv, bi);
        if (lane == 0) sm.best[warp] = make_float2(bv, __int_as_float(bi));
        bar_consumers();
        if (tid == 0) {
            for (int w2 = 1; w2 < NCW; ++w2) {
                const float v = sm.best[w2].x;
                const int i = __float_as_int(sm.best[w2].y);
                if (better(v, i, bv, bi)) {
                    bv = v;
                    bi = i;
                }
            }
            a.am_part[c] = make_float2(bv, __int_as_float(bi));
        }
        end();
    }

    // Final greedy token and the device-side advance of the step parameters (CTA 0).
    if (c == 0) {
        if (!begin(k)) return;
        if (warp == 0) {
            const int best = reduce_argmax(a, G);
            if (lane == 0) {
                const int idx = sp0.step + a.n_steps;
                a.token_log[idx - 1] = best;
                StepParams np = sp0;
                np.token = (a.forced && idx < sp0.n_forced) ? a.forced[idx] : best;
                np.step = idx;
                np.pos = sp0.pos + a.n_steps;
                step_positions(np.pos, a.ctx, &np.num_sink, &np.kv_pos, &np.kv_len);
                *a.sp = np;
            }
        }
    }
}

}  // namespace

bool fused_supported(const q3_config& c) {
    return c.dim == D && c.hidden_dim == H && c.head_dim == HD && c.n_heads == NQ &&
           c.n_kv_heads == NKV && c.rotary_dim == HD;
}

size_t fused_smem_bytes() { return sizeof(Smem); }

int fused_grid(int device) {
    int sms = 0;
    Q3_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    Q3_CUDA(cudaFuncSetAttribute(decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(Smem))));
    int per_sm = 0;
    Q3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_fused_kernel, NT,
                                                          sizeof(Smem)));
    if (per_sm < 1) return 0;
    return sms;
}

void launch_decode_fused(const FusedArgs& a, int grid, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = sizeof(Smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q3_CUDA(cudaLaunchKernelEx(&cfg, decode_fused_kernel, a));
}

}  // namespace q3
