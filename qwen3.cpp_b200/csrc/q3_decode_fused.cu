// Fused whole-step decode for the Qwen3-0.6B shape on B200 (sm_100a).
//
// One persistent cooperative launch (one CTA per SM) runs n_steps greedy decode steps. Each step
// is the reference's ForwardToken (asriva32/Qwen3.cpp src/inference.cpp:592-637) + Greedy
// (:703-709): 28 x Block::forward (:766-866), final RmsNorm, tied lm_head, argmax.
//
// Dataflow. Decode at batch 1 streams 1.19 GB of bf16 weights per token. Each SM runs one
// continuous stream: a producer warp walks the fixed sequence of byte ranges this CTA owns for the
// whole call and copies them with 1-D TMA bulk copies (cp.async.bulk into this CTA only) into an 8-slot
// shared-memory ring guarded by full/empty mbarriers. It runs ahead across the grid-wide
// dependencies (it only waits for a free slot, and - for KV pages - for the step that wrote
// them). Eight consumer warps wait for each phase's input (a monotonic arrival counter in global
// memory, release/acquire), stage it in shared memory with the RMSNorm fused in, and dot it with
// the rows as they land. Three grid-wide phases per layer (four past 128 cached positions):
//   A   x = Xprev + Y[l-1] (or the embedding row); qkv = [wq;wk;wv] . RmsNorm(x)
//       (src/inference.cpp:795-798)
//   BC  CTA (g, p) of KV head g: QK-RMSNorm + RoPE (:800-810), bf16 K/V write at kv_pos
//       (:812-815), attention over the KV pages streamed through the ring with the sink rows
//       re-rotated on the fly (:817-844), then rows p of wo[:, 256g:256g+256] . attn_g, the
//       group-g partial of the o_proj (:846-849)
//   (past 128 positions: B = split-K attention partials read through L2, C = combine + the same
//    o_proj partial)
//   DE  Xcur = x + sum_g partial_g (x += proj, :849), h_i = silu(w1_i . xn) * (w3_i . xn) for this
//       CTA's MLP indices i, then Y[l] += sum_i h_i * w2[:, i] (split-K down_proj, :851,
//       :1005-1015, :863-865); the attention-sink rows are written back rotated (:817-827)
// then the final RmsNorm + lm_head with a per-CTA argmax; every CTA reduces the (value, index)
// pairs itself (lowest index wins ties) for the next step's embedding row.
//
// Hand-offs. Only DE (and B, past 128 positions) and the lm_head end with a grid-wide arrival
// counter. A -> BC and BC -> DE hand their outputs over as tagged 64-bit words (fp32 bits | the
// (launch, step, layer) tag), each written once and polled by its readers until the tag matches:
// one L2 round trip instead of a release, a counter and a reload. Every thread keeps its four
// elements of the residual stream in registers from phase to phase.
//
// The down_proj split-K sums use fp32 atomics, so the order of those fp32 additions varies from
// run to run; the o_proj partials are summed in group order.
//
// Every wait is bounded (clock64): on timeout the kernel sets *err, stops issuing copies, waits
// for the copies already issued and returns; the host reports Q3_ERR_DEVICE_TIMEOUT.
#include <cuda_runtime.h>
#include <float.h>
#include <limits.h>
#include <stdlib.h>

#include <algorithm>

#include "q3_decode_fused.cuh"

namespace q3 {

namespace {

constexpr int D = 1024, H = 3072, NQ = 16, NKV = 8, HD = 128;
constexpr int QD = NQ * HD, KVD = NKV * HD;
constexpr int GRP = 2 * HD;            // attention output of one KV-head group (2 query heads)
constexpr int NCW = 8;                 // consumer warps
constexpr int NCT = NCW * 32;          // consumer threads
constexpr int NT = NCT + 32;           // + one producer warp
constexpr int NS = 8;                  // ring slots
constexpr int kProducerSleepNs = 256;  // back-off of the producer while the ring is full
// Copies of each layer's down-projection accumulator: CTA c adds into copy c % kYRep, which cuts
// the number of fp32 atomics per address kYRep-fold; phase A sums the copies (measured: 4 copies
// 0.6% faster than 8, 16 copies 1.5% slower).
constexpr int kYRep = 4;
constexpr int SLOT = 16384;            // bytes per slot
// Chunk q lives in slot q % NS and, in warp-owned tasks, is consumed by warp q % NCW; shared
// chunks (KV pages, w2t rows) are read by every consumer warp. A slot is free again after NCW
// arrivals: the owner warp arrives with count NCW, each warp once for a shared chunk. With NS a
// multiple of NCW every use of a slot inside a warp-owned task belongs to the same warp, every
// warp consumes its chunks in order, and every shared section starts after a consumer barrier, so
// no warp can wait on use n of a slot before use n-1 was filled (a parity wait for use n would
// then be satisfied by the completion of use n-2).
static_assert(NS % 8 == 0, "ring slots must be a multiple of the consumer warps");
// Rows per ring chunk: one 8-row dot group (fma_rows8) per chunk.
constexpr int RPC_ROW = 8;             // 1024-element rows ([wq;wk;wv], lm_head, w2t)
constexpr int RPC_GRP = 8;             // 256-element rows (wo split by KV-head group)
constexpr int RPC_PAIR = 4;            // w1 | w3 row pairs (4 + 4 rows)
constexpr int T_SHORT = 128;           // KV positions up to which attention runs from the ring
constexpr int ATT_TOK = 24;            // at least this many positions per attention split
constexpr int PAGE_BYTES = kPageTokens * HD * 2;

enum Mode : int { kTag = 0, kPair = 2, kLogits = 3, kTagX = 4 };

// The kernel is instantiated twice: TP = false for one rank without the exchange (every shard
// size a compile-time constant: all 8 KV groups, all 3072 MLP indices), TP = true for the
// tensor-parallel shards of FusedArgs (nkv, kv0, hl, the exchange words).
template <bool TP>
struct Shard {
    __device__ static int nkv(const FusedArgs& a) { return TP ? a.nkv : NKV; }
    __device__ static int kv0(const FusedArgs& a) { return TP ? a.kv0 : 0; }
    __device__ static int hl(const FusedArgs& a) { return TP ? a.hl : H; }
    __device__ static bool xchg(const FusedArgs& a) { return TP && a.xchg != 0; }
};

struct __align__(128) Smem {
    uint8_t ring[NS][SLOT];
    float4 xa[D / 8];         // staged fp32 activation of a GEMV: elements 8u..8u+3 in xa[u],
    float4 xb[D / 8];         // 8u+4..8u+7 in xb[u] (a warp's 32 consecutive units, no conflicts)
    float4 xs4[H / 4];        // attention staging and merge buffers
    float qk[4][HD];          // q head 2g, q head 2g+1, k and v at kv_pos (bf16-rounded)
    float hbuf[64];           // h of this CTA's MLP indices
    float2 mlw[NCW][2];       // per-warp attention (max, sum)
    float red[NCW];
    float2 best[NCW];
    uint64_t full[NS];
    uint64_t empty[NS];
    unsigned long long wait_cycles;  // instrumentation only
    unsigned long long gt0;          // instrumentation: globaltimer and clock64 at the start
    long long clk0;
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
__device__ __forceinline__ void mbar_arrive_n(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(n)
                 : "memory");
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
// Non-blocking probe (try_wait may suspend the thread for a while before it reports failure).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
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
__device__ __forceinline__ uint64_t evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
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
// L2 prefetch of a 16-byte aligned range (no completion, no shared memory).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    const uint8_t* b = static_cast<const uint8_t*>(src);
    constexpr uint32_t kPiece = 16384;
    for (uint32_t o = 0; o < bytes; o += kPiece) {
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b + o),
                     "r"(min(kPiece, bytes - o))
                     : "memory");
    }
}
// Fire-and-forget fp32 additions in L2 (no value returned, the thread does not wait).
__device__ __forceinline__ void red_add4(float* p, float4 v) {
    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x),
                 "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
// Tagged hand-off words: fp32 bits in the low half, the producing (launch, step, layer) tag in the
// high half, written and read as single 64-bit accesses (a reader that sees the tag sees the
// value written with it).
__device__ __forceinline__ void st_tagged(unsigned long long* p, float v, unsigned tag) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void ld_tagged2(const unsigned long long* p, unsigned long long& w0,
                                           unsigned long long& w1) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];"
                 : "=l"(w0), "=l"(w1)
                 : "l"(p)
                 : "memory");
}
// Tensor-parallel exchange: words written by other GPUs (or read by them) are accessed at system
// scope; `sys` is uniform over the launch.
__device__ __forceinline__ void ld_tagged2x(const unsigned long long* p, unsigned long long& w0,
                                            unsigned long long& w1, bool sys) {
    if (sys) {
        asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];"
                     : "=l"(w0), "=l"(w1)
                     : "l"(p)
                     : "memory");
    } else {
        ld_tagged2(p, w0, w1);
    }
}
__device__ __forceinline__ void st_tagged_x(unsigned long long* p, float v, unsigned tag, bool sys) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    if (sys) {
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
    } else {
        asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
    }
}
// Four tagged words (32-byte aligned) as two 16-byte stores.
__device__ __forceinline__ void st_tagged4_x(unsigned long long* p, float4 v, unsigned tag, bool sys) {
    const unsigned long long t = static_cast<unsigned long long>(tag) << 32;
    const unsigned long long w0 = t | __float_as_uint(v.x), w1 = t | __float_as_uint(v.y);
    const unsigned long long w2 = t | __float_as_uint(v.z), w3 = t | __float_as_uint(v.w);
    if (sys) {
        asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
        asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p + 2), "l"(w2), "l"(w3) : "memory");
    } else {
        asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
        asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(p + 2), "l"(w2), "l"(w3) : "memory");
    }
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void bar_consumers() {
    asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
}
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// ------------------------------------------------------------------ self-checks
//
// Builds with Q3_FUSED_CHECKS validate every shared-memory offset, bulk-copy range and epilogue
// index of the kernel, and record the first failed check (or the site of a wait that gave up)
// in a.dbg: [0] code, [1] CTA, [2] thread, [3..5] values; a failed access is skipped.

#ifdef Q3_FUSED_CHECKS
__device__ __noinline__ void dbg_report(const FusedArgs& a, unsigned long long code, long long v0,
                                        long long v1, long long v2) {
    if (a.dbg && atomicCAS(a.dbg, 0ull, code) == 0ull) {
        a.dbg[1] = blockIdx.x;
        a.dbg[2] = threadIdx.x;
        a.dbg[3] = static_cast<unsigned long long>(v0);
        a.dbg[4] = static_cast<unsigned long long>(v1);
        a.dbg[5] = static_cast<unsigned long long>(v2);
        __threadfence();
    }
}
#define Q3_CHECK(cond, code, v0, v1, v2)                  \
    (((cond)) ? true                                      \
              : (dbg_report(a, (code), (long long)(v0),   \
                            (long long)(v1), (long long)(v2)), \
                 false))
#else
#define Q3_CHECK(cond, code, v0, v1, v2) true
#endif

// ------------------------------------------------------------------ bounded waits

// sleep_ns > 0: back off between probes (a waiting thread then takes almost no issue slots from
// the warps that share its scheduler).
__device__ bool mbar_wait(uint64_t* b, uint32_t parity, const FusedArgs& a, volatile int* abort,
                          int site = 0, long long info = 0, int sleep_ns = 0) {
    if (mbar_try_wait(b, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(b, parity)) return true;
        if (sleep_ns > 0) __nanosleep(sleep_ns);
        if ((it & 31) == 31) {
            if (*abort) return false;
            if (clock64() - t0 > a.spin_cycles) {
                *abort = 1;
                atomicOr(a.err, 1u);
                Q3_CHECK(false, 1000 + site, info, parity, 0);
                return false;
            }
        }
    }
}

// Tag of the hand-offs of layer l in step st of this launch.
__device__ __forceinline__ unsigned step_tag(const FusedArgs& a, int st, int l) {
    return ((a.epoch & 0xFFFu) << 20) | (static_cast<unsigned>(st * a.n_layers + l) & 0xFFFFFu);
}

// Bounded wait until the four tagged words at p (32-byte aligned) carry `tag`; their values.
__device__ float4 poll4(const FusedArgs& a, const unsigned long long* p, unsigned tag,
                        volatile int* abort, int site, bool sys = false) {
    unsigned long long w0, w1, w2, w3;
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        ld_tagged2x(p, w0, w1, sys);
        ld_tagged2x(p + 2, w2, w3, sys);
        if (static_cast<unsigned>(w0 >> 32) == tag && static_cast<unsigned>(w1 >> 32) == tag &&
            static_cast<unsigned>(w2 >> 32) == tag && static_cast<unsigned>(w3 >> 32) == tag) {
            break;
        }
        if ((it & 15) == 15) {
            if (*abort || *reinterpret_cast<volatile unsigned*>(a.err) != 0u) {
                *abort = 1;
                break;
            }
            if (clock64() - t0 > a.spin_cycles) {
                *abort = 1;
                atomicOr(a.err, 1u);
                Q3_CHECK(false, 3000 + site, tag, static_cast<long long>(w0 >> 32), 0);
                break;
            }
        }
    }
    return make_float4(__uint_as_float(static_cast<unsigned>(w0)),
                       __uint_as_float(static_cast<unsigned>(w1)),
                       __uint_as_float(static_cast<unsigned>(w2)),
                       __uint_as_float(static_cast<unsigned>(w3)));
}

// Wait until `target` CTA arrivals are visible on the grid counter.
__device__ bool grid_wait(const FusedArgs& a, unsigned target, volatile int* abort, int site = 0) {
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        const unsigned seen = ld_acquire(a.bar);
        if (seen >= target) return true;
        if ((it & 15) == 15) {
            if (*reinterpret_cast<volatile unsigned*>(a.err) != 0u || *abort) {
                *abort = 1;
                return false;
            }
            if (clock64() - t0 > a.spin_cycles) {
                *abort = 1;
                atomicOr(a.err, 1u);
                Q3_CHECK(false, 2000 + site, target, seen, 0);
                return false;
            }
            if (it > 4096) __nanosleep(64);
        }
    }
}

// Warp-level wait on a ring slot: lane 0 does the bounded wait, the verdict is made warp-uniform,
// then every lane observes the completed phase (so the copied bytes are visible to it; the phase
// cannot advance again before the slot is released, so that second wait returns at once).
__device__ __forceinline__ bool warp_wait_full(Smem& sm, int slot, uint32_t parity,
                                               const FusedArgs& a) {
    const int lane = threadIdx.x & 31;
    int ok = 0;
    if (!Q3_CHECK(slot >= 0 && slot < NS, 20, slot, parity, 0)) return false;
    // Fast path: the chunk has landed (the usual case, the ring runs ahead): every lane's own
    // non-blocking probe observes the completed phase.
    if (__all_sync(0xffffffffu, mbar_test_wait(&sm.full[slot], parity))) return true;
    if (lane == 0) {
        if (a.prof && !mbar_test_wait(&sm.full[slot], parity)) {
            // Instrumentation: time this warp spends waiting for ring data.
            const long long t0 = clock64();
            ok = static_cast<int>(mbar_wait(&sm.full[slot], parity, a, &sm.abort_flag, 1, slot));
            atomicAdd(&sm.wait_cycles, static_cast<unsigned long long>(clock64() - t0));
        } else {
            ok = static_cast<int>(mbar_wait(&sm.full[slot], parity, a, &sm.abort_flag, 1, slot));
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return false;
    // Bounded as well: the phase already completed for lane 0 and cannot advance again before
    // this warp releases the slot.
    bool seen = false;
    for (int spin = 0; spin < (1 << 20); ++spin) {
        if (mbar_try_wait(&sm.full[slot], parity)) {
            seen = true;
            break;
        }
    }
    if (!seen) Q3_CHECK(false, 21, slot, parity, 0);
    return __all_sync(0xffffffffu, seen);
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
// As part, in whole row pairs (rows even): every share starts on an even row, so the lm_head
// epilogue writes its logits as aligned 8-byte pairs (fewer, fuller transactions, which matters
// when the logits go straight to pinned host memory).
__device__ __forceinline__ Span part2(int rows, int G, int c) {
    const Span s = part(rows / 2, G, c);
    return {2 * s.r0, 2 * s.n};
}

static_assert(RPC_ROW * D * 2 <= SLOT && RPC_GRP * GRP * 2 <= SLOT &&
                  2 * RPC_PAIR * D * 2 <= SLOT && 4 * kPageTokens * HD * 2 <= SLOT,
              "ring slot too small");

__device__ __forceinline__ size_t page_elem(const int32_t* table, int page, int g) {
    return (static_cast<size_t>(__ldg(table + page)) * NKV + g) * kPageTokens * HD;
}
__device__ __forceinline__ size_t paged(const int32_t* table, int t, int g) {
    return page_elem(table, t / kPageTokens, g) + static_cast<size_t>(t % kPageTokens) * HD;
}

struct StepPos {
    int pos, num_sink, kv_pos, kv_len, splits;
    bool shrt;
};

__device__ __forceinline__ StepPos step_pos(const FusedArgs& a, const StepParams& sp0, int st) {
    StepPos p;
    p.pos = sp0.pos + st;
    step_positions(p.pos, a.ctx, &p.num_sink, &p.kv_pos, &p.kv_len);
    p.shrt = p.kv_len <= T_SHORT;
    p.splits = min(max((p.kv_len + ATT_TOK - 1) / ATT_TOK, 1), a.s_max);
    return p;
}

// Past T_SHORT positions: the positions [t0, t1) of this rank's KV group g (local index) that
// CTA c attends to (split c / nkv of group c % nkv; t0 >= t1 for a split past kv_len), `on` for
// the CTAs that take part. Its KV pages are [j0, j1) (none for an empty split).
struct SplitRange {
    bool on;
    int g, s, t0, t1, j0, j1;
};
__device__ __forceinline__ SplitRange split_range(const StepPos& p, int c, int nkv) {
    SplitRange r;
    r.on = !p.shrt && c < nkv * p.splits;
    r.g = c % nkv;
    r.s = c / nkv;
    const int chunk = (p.kv_len + p.splits - 1) / p.splits;
    r.t0 = min(r.s * chunk, p.kv_len);
    r.t1 = min(p.kv_len, r.t0 + chunk);
    r.j0 = r.t0 / kPageTokens;
    r.j1 = r.t1 > r.t0 ? (r.t1 + kPageTokens - 1) / kPageTokens : r.j0;
    return r;
}
__device__ __forceinline__ int chunks_of_i(int n, int per) { return (n + per - 1) / per; }

// Grid arrivals of one step: after every DE (and every B past 128 positions) and the lm_head.
__device__ __forceinline__ int barriers_of(const FusedArgs& a, bool shrt) {
    return a.n_layers * (shrt ? 1 : 2) + 1;
}

// ------------------------------------------------------------------ producer

// L2 prefetch of unit u of a CTA's copy sequence (u < n_layers: this CTA's weight rows of layer
// u; u == n_layers: the first rows of its lm_head slice), so that the ring copies of that unit hit
// L2 while the HBM stream keeps running through the grid-wide waits in between. Out of line (run
// once per unit): it stays out of the producer loop's instruction working set.
// Takes its inputs by value: a reference to the kernel parameters would make every access a
// generic-address load (measured: 1% slower decode steps).
__device__ __noinline__ void prefetch_unit(const FusedLayer* layers, int n_layers,
                                           const uint16_t* lm_head, int vocab, int nkv, int kv0,
                                           int hl, int u, int G, int c) {
    const int P = G / nkv;
    const int g = kv0 + c % nkv, p = c / nkv;
    if (u < n_layers) {
        const FusedLayer w = layers[u];
        Span sp = part(nkv * 4 * HD, G, c);
        prefetch_l2(w.wqkv + static_cast<size_t>(sp.r0) * D, sp.n * D * 2);
        if (c < nkv * P) {
            sp = part(D, P, p);
            prefetch_l2(w.wop + static_cast<size_t>(g) * D * GRP + static_cast<size_t>(sp.r0) * GRP,
                        sp.n * GRP * 2);
        }
        sp = part(hl, G, c);
        prefetch_l2(w.w1 + static_cast<size_t>(sp.r0) * D, sp.n * D * 2);
        prefetch_l2(w.w3 + static_cast<size_t>(sp.r0) * D, sp.n * D * 2);
        prefetch_l2(w.w2t + static_cast<size_t>(sp.r0) * D, sp.n * D * 2);
    } else {
        const Span sp = part2(vocab, G, c);
        prefetch_l2(lm_head + static_cast<size_t>(sp.r0) * D, min(sp.n, 96) * D * 2);
    }
}


template <bool TP>
struct Producer {
    Smem& sm;
    const FusedArgs& a;
    uint64_t pol_w, pol_kv;
    uint32_t q = 0;

    unsigned long long blocked = 0;  // instrumentation: cycles spent waiting for a free slot

    __device__ bool issue(const void* s1, uint32_t b1, const void* s2, uint32_t b2, int off2,
                          uint64_t pol) {
        const int slot = q % NS;
        if (!Q3_CHECK(b1 % 16 == 0 && b2 % 16 == 0 && b1 > 0 && b1 <= SLOT &&
                          (b2 == 0 || (off2 % 16 == 0 && off2 >= static_cast<int>(b1) &&
                                       off2 + b2 <= SLOT)),
                      30, b1, b2, off2) ||
            !Q3_CHECK((reinterpret_cast<uintptr_t>(s1) & 15) == 0 &&
                          (reinterpret_cast<uintptr_t>(s2) & 15) == 0,
                      31, reinterpret_cast<uintptr_t>(s1), reinterpret_cast<uintptr_t>(s2), q)) {
            return false;
        }
        if (!take_slot(slot)) return false;
        mbar_arrive_expect_tx(&sm.full[slot], b1 + b2);
        bulk_g2s(sm.ring[slot], s1, b1, &sm.full[slot], pol);
        if (b2) bulk_g2s(sm.ring[slot] + off2, s2, b2, &sm.full[slot], pol);
        ++q;
        return true;
    }

    // Bounded wait until ring slot `slot` (chunk q) is free: its previous use (chunk q - NS) was
    // released by every consumer warp.
    __device__ bool take_slot(int slot) {
        if (q < NS) return true;
        const uint32_t par = ((q / NS) - 1) & 1;
        if (a.prof && !mbar_test_wait(&sm.empty[slot], par)) {
            const long long t0 = clock64();
            const bool ok = mbar_wait(&sm.empty[slot], par, a, &sm.abort_flag, 2, q, kProducerSleepNs);
            blocked += clock64() - t0;
            return ok;
        }
        return mbar_wait(&sm.empty[slot], par, a, &sm.abort_flag, 2, q, kProducerSleepNs);
    }

    // One chunk of two KV pages: K and V of page e0 at [0, 2 PAGE_BYTES), of page e1 after them.
    __device__ bool issue_page_pair(const uint16_t* kc, const uint16_t* vc, size_t e0, size_t e1) {
        const int slot = q % NS;
        if (!Q3_CHECK(((reinterpret_cast<uintptr_t>(kc + e0) | reinterpret_cast<uintptr_t>(vc + e0) |
                        reinterpret_cast<uintptr_t>(kc + e1) | reinterpret_cast<uintptr_t>(vc + e1)) &
                       15) == 0,
                      32, e0, e1, q)) {
            return false;
        }
        if (!take_slot(slot)) return false;
        mbar_arrive_expect_tx(&sm.full[slot], 4 * PAGE_BYTES);
        bulk_g2s(sm.ring[slot], kc + e0, PAGE_BYTES, &sm.full[slot], pol_kv);
        bulk_g2s(sm.ring[slot] + PAGE_BYTES, vc + e0, PAGE_BYTES, &sm.full[slot], pol_kv);
        bulk_g2s(sm.ring[slot] + 2 * PAGE_BYTES, kc + e1, PAGE_BYTES, &sm.full[slot], pol_kv);
        bulk_g2s(sm.ring[slot] + 3 * PAGE_BYTES, vc + e1, PAGE_BYTES, &sm.full[slot], pol_kv);
        ++q;
        return true;
    }

    template <int ROW_BYTES, int RPC>
    __device__ bool rows(const void* base, Span sp) {
        const uint8_t* b = static_cast<const uint8_t*>(base);
        for (int rb = sp.r0; rb < sp.r0 + sp.n; rb += RPC) {
            const int rn = min(RPC, sp.r0 + sp.n - rb);
            if (!issue(b + static_cast<size_t>(rb) * ROW_BYTES, rn * ROW_BYTES, nullptr, 0u, 0,
                       pol_w)) {
                return false;
            }
        }
        return true;
    }

    __device__ bool pairs(const uint16_t* w1, const uint16_t* w3, Span sp) {
        constexpr int RPC = RPC_PAIR;
        for (int rb = sp.r0; rb < sp.r0 + sp.n; rb += RPC) {
            const int rn = min(RPC, sp.r0 + sp.n - rb);
            const size_t off = static_cast<size_t>(rb) * D;
            if (!issue(w1 + off, rn * D * 2, w3 + off, rn * D * 2, RPC * D * 2, pol_w)) {
                return false;
            }
        }
        return true;
    }

    // K and V pages [j0, j1) of KV head g, layer l: one chunk per page.
    __device__ bool kv_pages(int l, int g, int j0, int j1) {
        const uint16_t* kc = a.k_cache + static_cast<size_t>(l) * a.layer_elems;
        const uint16_t* vc = a.v_cache + static_cast<size_t>(l) * a.layer_elems;
        for (int j = j0; j < j1; ++j) {
            const size_t e = page_elem(a.page_table, j, g);
            if (!issue(kc + e, PAGE_BYTES, vc + e, PAGE_BYTES, PAGE_BYTES, pol_kv)) return false;
        }
        return true;
    }

    // K and V pages [j0, j1) of KV head g, layer l, two pages per chunk (a last odd page alone),
    // for the split attention past T_SHORT positions.
    __device__ bool kv_page_pairs(int l, int g, int j0, int j1) {
        const uint16_t* kc = a.k_cache + static_cast<size_t>(l) * a.layer_elems;
        const uint16_t* vc = a.v_cache + static_cast<size_t>(l) * a.layer_elems;
        for (int j = j0; j < j1; j += 2) {
            const size_t e0 = page_elem(a.page_table, j, g);
            const bool ok = j + 1 < j1
                                ? issue_page_pair(kc, vc, e0, page_elem(a.page_table, j + 1, g))
                                : issue(kc + e0, PAGE_BYTES, vc + e0, PAGE_BYTES, PAGE_BYTES, pol_kv);
            if (!ok) return false;
        }
        return true;
    }

    // Prefetches unit k of the whole call (units n_layers + 1 per step) if it exists.
    __device__ void prefetch_ahead(int k, int G, int c) {
        const int per = a.n_layers + 1;
        if (a.l2_ahead > 0 && k < a.n_steps * per) {
            prefetch_unit(a.layers, a.n_layers, a.lm_head, a.vocab, Shard<TP>::nkv(a),
                          Shard<TP>::kv0(a), Shard<TP>::hl(a), k % per, G, c);
        }
    }

    __device__ void run(int G, int c) {
        pol_w = evict_first_policy();
        pol_kv = evict_last_policy();
        const StepParams sp0 = a.sp_from_args ? a.sp_init : *a.sp;
        const int nkv = Shard<TP>::nkv(a), kv0 = Shard<TP>::kv0(a), hl = Shard<TP>::hl(a);
        const int P = G / nkv;
        const bool in_grp = c < nkv * P;
        const int g = kv0 + c % nkv, p = c / nkv;  // KV group (global index) of BC
        const int per = a.n_layers + 1;
        bool ok = true;
        unsigned base = 0, prev_base = 0;
        bool prev_short = true;
        for (int k = 1; k < a.l2_ahead; ++k) prefetch_ahead(k, G, c);
        for (int st = 0; ok && st < a.n_steps; ++st) {
            const StepPos sp = step_pos(a, sp0, st);
            for (int l = 0; ok && l < a.n_layers; ++l) {
                const FusedLayer w = a.layers[l];
                prefetch_ahead(st * per + l + a.l2_ahead, G, c);
                ok = ok && rows<D * 2, RPC_ROW>(w.wqkv, part(nkv * 4 * HD, G, c));
                // KV pages this CTA's attention reads: all of head g's (short contexts) or those
                // of its split (long ones).
                const SplitRange sr = split_range(sp, c, nkv);
                if (ok && (sp.shrt ? in_grp : sr.on)) {
                    // KV pages of this layer were last written (row kv_pos, sink rows) by the
                    // previous step's phases up to DE(l): wait until every CTA is past them.
                    if (st > 0) {
                        const unsigned de = prev_base + (prev_short ? l : 2 * l + 1);
                        ok = grid_wait(a, G * (de + 1) + a.barrier_offset, &sm.abort_flag, 3);
                    }
                    ok = ok && (sp.shrt ? kv_pages(l, g, 0, chunks_of_i(sp.kv_len, kPageTokens))
                                        : kv_page_pairs(l, kv0 + sr.g, sr.j0, sr.j1));
                }
                if (in_grp) {
                    ok = ok && rows<GRP * 2, RPC_GRP>(w.wop + static_cast<size_t>(g) * D * GRP,
                                                      part(D, P, p));
                }
                ok = ok && pairs(w.w1, w.w3, part(hl, G, c));
                ok = ok && rows<D * 2, RPC_ROW>(w.w2t, part(hl, G, c));
            }
            prefetch_ahead(st * per + a.n_layers + a.l2_ahead, G, c);
            ok = ok && rows<D * 2, RPC_ROW>(a.lm_head, part2(a.vocab, G, c));
            prev_base = base;
            prev_short = sp.shrt;
            base += barriers_of(a, sp.shrt);
        }
        // This CTA's rows of the first layer into L2 for the next launch (a decode loop of
        // one-step calls would otherwise start every step on a cold stream).
        if (ok && a.l2_ahead > 0) {
            prefetch_unit(a.layers, a.n_layers, a.lm_head, a.vocab, nkv, kv0, hl, 0, G, c);
        }
        if (a.prof) a.prof[static_cast<size_t>(c) * 8 + 4] = blocked;
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

__device__ __forceinline__ uint8_t* smem_raw_ptr() {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    return smem_raw;
}

//

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

// The staged activation x of a GEMV is kept in fp32 (sm.xa / sm.xb) and multiplied against the
// bf16 weights on the CUDA cores with fp32 accumulation, as the reference's MatMul does.
__device__ __forceinline__ void xs_put(Smem& sm, int e, float val) {
    float* half = reinterpret_cast<float*>((e & 4) ? sm.xb : sm.xa);
    half[(e >> 3) * 4 + (e & 3)] = val;
}

// Stage xs = RmsNorm(x) (src/inference.cpp:887-923) for a K=1024 GEMV; thread t holds x[4t..4t+3]
// and its norm weights wv.
__device__ __forceinline__ void stage_norm(Smem& sm, float4 xv, uint2 wv, float eps) {
    const int t = threadIdx.x;
    const float ss = consumer_sum(xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w, sm);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
    ((t & 1) ? sm.xb : sm.xa)[t >> 1] =
        make_float4((xv.x * inv) * bf16_lo(wv.x), (xv.y * inv) * bf16_hi(wv.x),
                    (xv.z * inv) * bf16_lo(wv.y), (xv.w * inv) * bf16_hi(wv.y));
    bar_consumers();
}

// Dot products of 8 weight rows (a ring chunk, row-major, K bf16 per row, rows swizzled by row
// parity: in odd rows the two 64-byte halves of every 128-byte block are swapped) with the staged
// fp32 activation. Lane l takes the 16-byte units u = l + 32 j (j < K / 256) of every row and
// holds the matching activation elements 8u..8u+7 in registers; a transposing butterfly over the
// eight row sums leaves row q in lanes 4q..4q+3. Result: lanes 0-3 hold rows 2t and 2t+1
// (t = lane) in .x, .y. Out of line: every phase that dots K-element rows runs the same copy of
// this code, which keeps the kernel's instruction working set small.
template <int K>
__device__ __noinline__ float2 fma_rows8(int slot, int row0) {
    static_assert(8 * K * 2 <= SLOT, "eight rows per ring chunk");
    constexpr int U = K / 256;
    const Smem& sm = *reinterpret_cast<const Smem*>(smem_raw_ptr());
    const uint8_t* rows = sm.ring[slot];
    const int lane = threadIdx.x & 31;
    float xr[U][8];
#pragma unroll
    for (int j = 0; j < U; ++j) {
        const float4 p = sm.xa[lane + 32 * j];
        const float4 q = sm.xb[lane + 32 * j];
        xr[j][0] = p.x; xr[j][1] = p.y; xr[j][2] = p.z; xr[j][3] = p.w;
        xr[j][4] = q.x; xr[j][5] = q.y; xr[j][6] = q.z; xr[j][7] = q.w;
    }
    float s[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const uint8_t* rp = rows + r * K * 2;
        const int sw = ((row0 + r) & 1) << 2;
        // Even elements accumulate in .x, odd ones in .y: one packed fp32x2 FMA per weight pair.
        float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int u = (lane + 32 * j) ^ sw;
            const uint4 w = *reinterpret_cast<const uint4*>(rp + (u << 4));
            acc = ffma2(make_float2(bf16_lo(w.x), bf16_hi(w.x)), make_float2(xr[j][0], xr[j][1]), acc);
            acc = ffma2(make_float2(bf16_lo(w.y), bf16_hi(w.y)), make_float2(xr[j][2], xr[j][3]), acc);
            acc = ffma2(make_float2(bf16_lo(w.z), bf16_hi(w.z)), make_float2(xr[j][4], xr[j][5]), acc);
            acc = ffma2(make_float2(bf16_lo(w.w), bf16_hi(w.w)), make_float2(xr[j][6], xr[j][7]), acc);
        }
        s[r] = acc.x + acc.y;
    }
    // Butterfly: after xor 16 / 8 / 4 each lane keeps one row, q = lane >> 2, then xor 2 / 1.
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float t4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = b4 ? s[i] : s[i + 4];
        const float keep = b4 ? s[i + 4] : s[i];
        t4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float t2[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b3 ? t4[i] : t4[i + 2];
        const float keep = b3 ? t4[i + 2] : t4[i];
        t2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float v = (b2 ? t2[1] : t2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? t2[0] : t2[1], 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    const int t = lane & 3;
    return make_float2(__shfl_sync(0xffffffffu, v, 8 * t), __shfl_sync(0xffffffffu, v, 8 * t + 4));
}

// As fma_rows8 for 4 rows; returns the row sums with row q in lanes 8q..8q+7.
template <int K>
__device__ __forceinline__ float fma_rows4(const Smem& sm, const uint8_t* rows, int row0) {
    constexpr int U = K / 256;
    const int lane = threadIdx.x & 31;
    float xr[U][8];
#pragma unroll
    for (int j = 0; j < U; ++j) {
        const float4 p = sm.xa[lane + 32 * j];
        const float4 q = sm.xb[lane + 32 * j];
        xr[j][0] = p.x; xr[j][1] = p.y; xr[j][2] = p.z; xr[j][3] = p.w;
        xr[j][4] = q.x; xr[j][5] = q.y; xr[j][6] = q.z; xr[j][7] = q.w;
    }
    float s[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const uint8_t* rp = rows + r * K * 2;
        const int sw = ((row0 + r) & 1) << 2;
        float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const uint4 w = *reinterpret_cast<const uint4*>(rp + (((lane + 32 * j) ^ sw) << 4));
            acc = ffma2(make_float2(bf16_lo(w.x), bf16_hi(w.x)), make_float2(xr[j][0], xr[j][1]), acc);
            acc = ffma2(make_float2(bf16_lo(w.y), bf16_hi(w.y)), make_float2(xr[j][2], xr[j][3]), acc);
            acc = ffma2(make_float2(bf16_lo(w.z), bf16_hi(w.z)), make_float2(xr[j][4], xr[j][5]), acc);
            acc = ffma2(make_float2(bf16_lo(w.w), bf16_hi(w.w)), make_float2(xr[j][6], xr[j][7]), acc);
        }
        s[r] = acc.x + acc.y;
    }
    const bool b4 = lane & 16, b3 = lane & 8;
    float t2[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b4 ? s[i] : s[i + 2];
        const float keep = b4 ? s[i + 2] : s[i];
        t2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float v = (b3 ? t2[1] : t2[0]) + __shfl_xor_sync(0xffffffffu, b3 ? t2[0] : t2[1], 8);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v;
}

__device__ __forceinline__ uint2 load_norm(const uint16_t* nw) {
    return __ldg(reinterpret_cast<const uint2*>(nw) + threadIdx.x);
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// Dot the rows of this CTA's warp-owned chunks of one task (chunks q0.. of `rpc` rows of K
// elements) with the staged activation, epilogue by `mode`: kTag writes row r as a tagged word to
// outt[r], kTagX to a.opart_dst[d][xoff + r] of every rank d, kPair h to out[], kLogits the logits
// to out[] and leaves each warp's best (value, index) in sm.best. After an abort the remaining chunks are skipped (each wait then fails at once) but
// the warp still returns, so every consumer thread reaches the same barriers.
template <int K, int rpc, int mode>
__device__ __forceinline__ void consume_rows(Smem& sm, const FusedArgs& a, uint32_t q0, int r0,
                                             int n, float* out, int out_n,
                                             unsigned long long* outt = nullptr,
                                             unsigned tag = 0, size_t xoff = 0) {
    static_assert(mode == kPair ? rpc == 4 : rpc == 8, "one 8-row dot group per chunk");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, t = lane & 3;
    const int nch = (n + rpc - 1) / rpc;
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int ci = (warp - static_cast<int>(q0 % NCW) + NCW) % NCW; ci < nch; ci += NCW) {
        const uint32_t qq = q0 + ci;
        const int slot = qq % NS;
        if (!warp_wait_full(sm, slot, (qq / NS) & 1, a)) continue;
        const int rb = r0 + ci * rpc;
        const int rn = min(rpc, r0 + n - rb);
        const float2 yv = fma_rows8<K>(slot, rb);
        const float y0 = yv.x, y1 = yv.y;
        __syncwarp();
        if (lane == 0) mbar_arrive_n(&sm.empty[slot], NCW);  // a warp-owned chunk
        if (mode == kPair) {
            // Rows 0-3 of the group are w1 rows rb..rb+3 (lanes 0-1), rows 4-7 the w3 rows
            // (lanes 2-3): h = silu(gate) * up (src/inference.cpp:1009-1011).
            const float u0 = __shfl_down_sync(0xffffffffu, y0, 2);
            const float u1 = __shfl_down_sync(0xffffffffu, y1, 2);
            if (lane < 2) {
                const int i = 2 * t;
                if (i < rn && Q3_CHECK(rb - r0 + i < out_n, 50, rb, r0, i)) {
                    out[rb - r0 + i] = silu(y0) * u0;
                }
                if (i + 1 < rn && Q3_CHECK(rb - r0 + i + 1 < out_n, 51, rb, r0, i)) {
                    out[rb - r0 + i + 1] = silu(y1) * u1;
                }
            }
        } else if (lane < 4) {
            const int i = 2 * t;
            const float yy[2] = {y0, y1};
            if (mode == kLogits && i + 1 < rn && ((rb + i) & 1) == 0 &&
                Q3_CHECK(rb + i >= 0 && rb + i + 1 < out_n, 53, rb, i, out_n)) {
                // Rows rb + i, rb + i + 1 as one aligned pair (every lm_head share starts even).
                *reinterpret_cast<float2*>(out + rb + i) = make_float2(y0, y1);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if (better(yy[j], rb + i + j, bv, bi)) {
                        bv = yy[j];
                        bi = rb + i + j;
                    }
                }
                continue;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                if (i + j >= rn) break;
                const int r = rb + i + j;
                if (!Q3_CHECK(r >= 0 && r < out_n, 52, r, out_n, mode)) break;
                if (mode == kLogits) out[r] = yy[j];
                if (mode == kTag) st_tagged(outt + r, yy[j], tag);
                if (mode == kTagX) {
                    for (int d = 0; d < a.world; ++d) st_tagged_x(a.opart_dst[d] + xoff + r, yy[j], tag, a.sys);
                }
                if (mode == kLogits && better(yy[j], r, bv, bi)) {
                    bv = yy[j];
                    bi = r;
                }
            }
        }
    }
    if (mode == kLogits) {
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            const float v = __shfl_xor_sync(0xffffffffu, bv, o);
            const int j = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(v, j, bv, bi)) {
                bv = v;
                bi = j;
            }
        }
        if (lane == 0) sm.best[warp] = make_float2(bv, __int_as_float(bi));
    }
}

__device__ __forceinline__ uint32_t chunks_of(int n, int rpc) {
    return static_cast<uint32_t>((n + rpc - 1) / rpc);
}

// RoPE on a 128-vector spread over a warp, 4 elements per lane: lanes 0-15 hold the first half,
// lanes 16-31 the second; pairs (i, i+64) sit 16 lanes apart (src/inference.cpp:976-990).
__device__ __forceinline__ void rope_warp(float y[4], const float2 cs[4]) {
    const bool first = (threadIdx.x & 31) < 16;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float p = __shfl_xor_sync(0xffffffffu, y[j], 16);
        y[j] = first ? (y[j] * cs[j].x - p * cs[j].y) : (y[j] * cs[j].x + p * cs[j].y);
    }
}

__device__ __forceinline__ void load_rope(float2 cs[4], const FusedArgs& a, int pos) {
    const int rp = min(pos, a.rope_len - 1);
    const float2* row = a.rope + static_cast<size_t>(rp) * (HD / 2) + ((threadIdx.x & 31) & 15) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) cs[j] = __ldg(row + j);
}

__device__ __forceinline__ uint2 pack_bf16x4(const float y[4]) {
    return make_uint2(static_cast<uint32_t>(f32_to_bf16(y[0])) |
                          (static_cast<uint32_t>(f32_to_bf16(y[1])) << 16),
                      static_cast<uint32_t>(f32_to_bf16(y[2])) |
                          (static_cast<uint32_t>(f32_to_bf16(y[3])) << 16));
}
__device__ __forceinline__ void unpack_bf16x4(uint2 v, float y[4]) {
    y[0] = bf16_lo(v.x);
    y[1] = bf16_hi(v.x);
    y[2] = bf16_lo(v.y);
    y[3] = bf16_hi(v.y);
}

// Phase A with at most NCW / 2 chunks of 8 rows: two warps per chunk, four rows each, so that
// every consumer warp takes part; rows go out as tagged words to outt[row].
__device__ __forceinline__ void consume_rows_halves(Smem& sm, const FusedArgs& a, uint32_t q0,
                                                    int r0, int n, unsigned long long* outt,
                                                    unsigned tag) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nch = (n + RPC_ROW - 1) / RPC_ROW;
    const int ci = warp >> 1, half = warp & 1;
    if (ci >= nch) return;
    const uint32_t qq = q0 + ci;
    const int slot = qq % NS;
    if (!warp_wait_full(sm, slot, (qq / NS) & 1, a)) return;
    const int rb = r0 + ci * RPC_ROW + 4 * half;  // first row of this warp's half
    const float v = fma_rows4<D>(sm, sm.ring[slot] + half * 4 * D * 2, rb);
    __syncwarp();
    if (lane == 0) mbar_arrive_n(&sm.empty[slot], NCW / 2);  // two warps release the chunk
    const float y = __shfl_sync(0xffffffffu, v, 8 * (lane & 3));
    if (lane < 4 && rb + lane < r0 + n) st_tagged(outt + rb + lane, y, tag);
}

// Static inputs of the attention prologue, loaded before the phase's grid wait.
struct HeadPre {
    uint2 nw;        // q_norm (warps 0-1) or k_norm (warp 2) for this lane
    float2 cs[4];    // RoPE at pos
    float2 cs1[4];   // RoPE at position 1 (sink re-rotation)
};

__device__ __forceinline__ void head_preload(HeadPre& hp, const FusedArgs& a, const FusedLayer& w,
                                             int pos) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    hp.nw = __ldg(reinterpret_cast<const uint2*>(warp < 2 ? w.q_norm : w.k_norm) + lane);
    load_rope(hp.cs, a, pos);
    load_rope(hp.cs1, a, 1);
}

// QK-RMSNorm (src/inference.cpp:800-807) + RoPE (:809-810) of q heads 2g, 2g+1 and k head g into
// sm.qk[0..2]; v head g into sm.qk[3]; k and v rounded to bf16 as the cache stores them (:812-815)
// and, when `writer`, written to the cache at kv_pos. g: global KV head; gl: its index among this
// rank's groups (the rows of a.qkvt: q of the 2 nkv local query heads, then k, then v). Ends with
// a consumer barrier.
__device__ __forceinline__ void prep_heads(Smem& sm, const FusedArgs& a, const HeadPre& hp, int l,
                                        int nkv, int gl, int g, int kv_pos, bool writer,
                                        unsigned tag) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qd = nkv * 2 * HD, kvd = nkv * HD;
    if (warp < 3) {
        const unsigned long long* src = warp < 2 ? a.qkvt + (2 * gl + warp) * HD : a.qkvt + qd + gl * HD;
        const float4 e = poll4(a, src + 4 * lane, tag, &sm.abort_flag, 1);
        const float ss = warp_sum(e.x * e.x + e.y * e.y + e.z * e.z + e.w * e.w);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(HD) + a.eps);
        float y[4] = {(e.x * inv) * bf16_lo(hp.nw.x), (e.y * inv) * bf16_hi(hp.nw.x),
                      (e.z * inv) * bf16_lo(hp.nw.y), (e.w * inv) * bf16_hi(hp.nw.y)};
        rope_warp(y, hp.cs);
        if (warp == 2) {
            const uint2 kb = pack_bf16x4(y);
            unpack_bf16x4(kb, y);
            if (writer) {
                uint16_t* kc = a.k_cache + static_cast<size_t>(l) * a.layer_elems;
                reinterpret_cast<uint2*>(kc + paged(a.page_table, kv_pos, g))[lane] = kb;
            }
        }
        reinterpret_cast<float4*>(sm.qk[warp])[lane] = make_float4(y[0], y[1], y[2], y[3]);
    } else if (warp == 3) {
        const float4 e = poll4(a, a.qkvt + qd + kvd + gl * HD + 4 * lane, tag, &sm.abort_flag, 2);
        float y[4] = {e.x, e.y, e.z, e.w};
        const uint2 vb = pack_bf16x4(y);
        unpack_bf16x4(vb, y);
        if (writer) {
            uint16_t* vc = a.v_cache + static_cast<size_t>(l) * a.layer_elems;
            reinterpret_cast<uint2*>(vc + paged(a.page_table, kv_pos, g))[lane] = vb;
        }
        reinterpret_cast<float4*>(sm.qk[3])[lane] = make_float4(y[0], y[1], y[2], y[3]);
    }
    bar_consumers();
}

// Online-softmax state of one warp for the two query heads of a KV group.
struct AttnAcc {
    float m0, m1, l0, l1;
    float o0[4], o1[4];
};

__device__ __forceinline__ void acc_init(AttnAcc& s) {
    s.m0 = s.m1 = -FLT_MAX;
    s.l0 = s.l1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) s.o0[j] = s.o1[j] = 0.0f;
}

// Two cached positions a, b (b only when has_b) in one online-softmax update: the four dot
// products and their warp reductions are independent, and the running state is rescaled once.
__device__ __forceinline__ void acc_add2(AttnAcc& s, const float ka[4], const float va[4],
                                         const float kb[4], const float vb[4], bool has_b,
                                         float4 q0, float4 q1) {
    const float sq = 11.313708498984761f;  // sqrtf(128), the reference's sqrtf(head_dim)
    float da0 = ka[0] * q0.x, da1 = ka[0] * q1.x, db0 = kb[0] * q0.x, db1 = kb[0] * q1.x;
    da0 = fmaf(ka[1], q0.y, da0);
    da1 = fmaf(ka[1], q1.y, da1);
    db0 = fmaf(kb[1], q0.y, db0);
    db1 = fmaf(kb[1], q1.y, db1);
    da0 = fmaf(ka[2], q0.z, da0);
    da1 = fmaf(ka[2], q1.z, da1);
    db0 = fmaf(kb[2], q0.z, db0);
    db1 = fmaf(kb[2], q1.z, db1);
    da0 = fmaf(ka[3], q0.w, da0);
    da1 = fmaf(ka[3], q1.w, da1);
    db0 = fmaf(kb[3], q0.w, db0);
    db1 = fmaf(kb[3], q1.w, db1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        da0 += __shfl_xor_sync(0xffffffffu, da0, o);
        da1 += __shfl_xor_sync(0xffffffffu, da1, o);
        db0 += __shfl_xor_sync(0xffffffffu, db0, o);
        db1 += __shfl_xor_sync(0xffffffffu, db1, o);
    }
    const float sa0 = da0 / sq, sa1 = da1 / sq;
    const float sb0 = has_b ? db0 / sq : -FLT_MAX, sb1 = has_b ? db1 / sq : -FLT_MAX;
    const float n0 = fmaxf(s.m0, fmaxf(sa0, sb0)), n1 = fmaxf(s.m1, fmaxf(sa1, sb1));
    const float a0 = expf(s.m0 - n0), a1 = expf(s.m1 - n1);
    const float pa0 = expf(sa0 - n0), pa1 = expf(sa1 - n1);
    const float pb0 = has_b ? expf(sb0 - n0) : 0.0f, pb1 = has_b ? expf(sb1 - n1) : 0.0f;
    s.l0 = (s.l0 * a0 + pa0) + pb0;
    s.l1 = (s.l1 * a1 + pa1) + pb1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        s.o0[j] = (s.o0[j] * a0 + pa0 * va[j]) + pb0 * vb[j];
        s.o1[j] = (s.o1[j] * a1 + pa1 * va[j]) + pb1 * vb[j];
    }
    s.m0 = n0;
    s.m1 = n1;
}

// Key/value of cached position t for this lane: the in-register current row at kv_pos, and the
// attention-sink rows rotated by RoPE(position 1) and re-rounded (the reference rotates them in
// the cache before attending, :817-827; the rotated rows are written back in phase DE).
__device__ __forceinline__ void kv_lane(Smem& sm, const HeadPre& hp, int t, int kv_pos,
                                        int num_sink, uint2 kk, uint2 vv, float k4[4],
                                        float v4[4]) {
    const int lane = threadIdx.x & 31;
    if (t == kv_pos) {
        const float4 kc = reinterpret_cast<const float4*>(sm.qk[2])[lane];
        const float4 vc = reinterpret_cast<const float4*>(sm.qk[3])[lane];
        k4[0] = kc.x; k4[1] = kc.y; k4[2] = kc.z; k4[3] = kc.w;
        v4[0] = vc.x; v4[1] = vc.y; v4[2] = vc.z; v4[3] = vc.w;
        return;
    }
    unpack_bf16x4(kk, k4);
    unpack_bf16x4(vv, v4);
    if (t < num_sink) {
        rope_warp(k4, hp.cs1);
        unpack_bf16x4(pack_bf16x4(k4), k4);
    }
}

// Merge the 8 warps' online-softmax states: into the staged attention output of the group
// (K = 256 layout) or, for a split of a long context, into the partial buffers.
__device__ __forceinline__ void merge_warps(Smem& sm, const FusedArgs& a, const AttnAcc& acc, int g,
                                         int split, bool to_partials) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    bar_consumers();  // staging buffers alias the merge buffer
    float* mb = reinterpret_cast<float*>(sm.xs4) + 2 * GRP;  // [NCW][2][HD] after the output
    reinterpret_cast<float4*>(mb + (warp * 2 + 0) * HD)[lane] =
        make_float4(acc.o0[0], acc.o0[1], acc.o0[2], acc.o0[3]);
    reinterpret_cast<float4*>(mb + (warp * 2 + 1) * HD)[lane] =
        make_float4(acc.o1[0], acc.o1[1], acc.o1[2], acc.o1[3]);
    if (lane == 0) {
        sm.mlw[warp][0] = make_float2(acc.m0, acc.l0);
        sm.mlw[warp][1] = make_float2(acc.m1, acc.l1);
    }
    bar_consumers();
    const int hq = tid >> 7, d = tid & (HD - 1);
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < NCW; ++w)
        if (sm.mlw[w][hq].y > 0.0f) M = fmaxf(M, sm.mlw[w][hq].x);
    float L = 0.0f, o = 0.0f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) {
        const float2 ml = sm.mlw[w][hq];
        if (ml.y > 0.0f) {
            const float sc = expf(ml.x - M);
            L += ml.y * sc;
            o += mb[(w * 2 + hq) * HD + d] * sc;
        }
    }
    if (to_partials) {
        const size_t pi = static_cast<size_t>(2 * g + hq) * a.s_max + split;
        a.part_o[pi * HD + d] = o;
        if (d == 0) a.part_ml[pi] = make_float2(M, L);
    } else {
        xs_put(sm, tid, o / L);
    }
    bar_consumers();
}

// Phase BC attention (<= 128 cached positions): all positions of KV head g from the KV pages the
// producer streamed into the ring (shared chunks, released by every warp after each page).
__device__ __forceinline__ void attention_short(Smem& sm, const FusedArgs& a, const HeadPre& hp,
                                                int kv_len, int kv_pos, int num_sink, int g,
                                                uint32_t q0) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float4 q0v = reinterpret_cast<const float4*>(sm.qk[0])[lane];
    const float4 q1v = reinterpret_cast<const float4*>(sm.qk[1])[lane];
    AttnAcc acc;
    acc_init(acc);
    const int np = (kv_len + kPageTokens - 1) / kPageTokens;
    for (int j = 0; j < np; ++j) {
        const uint32_t qq = q0 + j;
        const int slot = qq % NS;
        if (warp_wait_full(sm, slot, (qq / NS) & 1, a)) {
            static_assert(kPageTokens == 2 * NCW, "two positions of a page per warp");
            const uint8_t* page = sm.ring[slot];
            const int ta = j * kPageTokens + warp, tb = ta + NCW;
            if (ta < kv_len) {
                const uint2 ka = reinterpret_cast<const uint2*>(page + warp * HD * 2)[lane];
                const uint2 va = reinterpret_cast<const uint2*>(page + PAGE_BYTES + warp * HD * 2)[lane];
                const int ub = tb < kv_len ? warp + NCW : warp;
                const uint2 kb = reinterpret_cast<const uint2*>(page + ub * HD * 2)[lane];
                const uint2 vb = reinterpret_cast<const uint2*>(page + PAGE_BYTES + ub * HD * 2)[lane];
                float k4[4], v4[4], k4b[4], v4b[4];
                kv_lane(sm, hp, ta, kv_pos, num_sink, ka, va, k4, v4);
                kv_lane(sm, hp, tb < kv_len ? tb : ta, kv_pos, num_sink, kb, vb, k4b, v4b);
                acc_add2(acc, k4, v4, k4b, v4b, tb < kv_len, q0v, q1v);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);  // one of NCW releases of a shared chunk
    }
    merge_warps(sm, a, acc, g, 0, false);
}

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

// One ring page of split attention (one warp): rows 2i + hb (hb = lane / 16) of page j, the lane's
// 8 dimensions 8 dl .. 8 dl + 7 (dl = lane % 16), for both query heads; positions outside
// [t0, t1) are masked. The row at kv_pos comes from sm.qk (this step's row, which the page copy
// may predate); attention-sink rows are rotated by RoPE(position 1) and re-rounded on the fly
// (src/inference.cpp:817-827). Updates the warp's online-softmax state (m, l warp-uniform; o per
// lane over its rows of parity hb).
__device__ __forceinline__ void split_page(const Smem& sm, const FusedArgs& a, const uint8_t* page,
                                        int j, int t0, int t1, int kv_pos, int num_sink,
                                        const float (&q0)[8], const float (&q1)[8], float (&m)[2],
                                        float (&l)[2], float (&o)[2][8]) {
    const int lane = threadIdx.x & 31;
    const int hb = lane >> 4, dl = lane & 15;
    const int tp = j * kPageTokens;
    float sv[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = 2 * i + hb, t = tp + r;
        float kf[8];
        unpack8(*reinterpret_cast<const uint4*>(page + (r * HD + 8 * dl) * 2), kf);
        if (t == kv_pos) {
            const float4* kc = reinterpret_cast<const float4*>(sm.qk[2] + 8 * dl);
            const float4 k0 = kc[0], k1 = kc[1];
            kf[0] = k0.x; kf[1] = k0.y; kf[2] = k0.z; kf[3] = k0.w;
            kf[4] = k1.x; kf[5] = k1.y; kf[6] = k1.z; kf[7] = k1.w;
        }
        // Sink rows (page 0 of a wrapped cache): pairs (d, d + 64) sit in lanes dl, dl ^ 8.
        if (tp < num_sink) {
            const bool sink = t < num_sink && t != kv_pos;
            const float2* cs = a.rope + HD / 2 + 8 * (dl & 7);  // RoPE at position 1
            const bool first = dl < 8;
#pragma unroll
            for (int d = 0; d < 8; ++d) {
                const float pr = __shfl_xor_sync(0xffffffffu, kf[d], 8);
                const float2 c = __ldg(cs + d);
                const float y = first ? (kf[d] * c.x - pr * c.y) : (kf[d] * c.x + pr * c.y);
                if (sink) kf[d] = bf16_to_f32(f32_to_bf16(y));
            }
        }
        float d0 = kf[0] * q0[0], d1 = kf[0] * q1[0];
#pragma unroll
        for (int d = 1; d < 8; ++d) {
            d0 = fmaf(kf[d], q0[d], d0);
            d1 = fmaf(kf[d], q1[d], d1);
        }
        sv[i] = d0;
        sv[8 + i] = d1;
    }
    // Transposing butterfly over the 16 lanes of each half: lane dl ends with the full score of
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
    const float sq = 11.313708498984761f;  // sqrtf(128), the reference's sqrtf(head_dim)
    const int my_h = dl >> 3, my_t = tp + 2 * (dl & 7) + hb;
    const bool my_valid = my_t >= t0 && my_t < t1;
    const float sc = my_valid ? dot / sq : -FLT_MAX;
    float mx = sc;
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float mx_other = __shfl_xor_sync(0xffffffffu, mx, 8);
    const float mx0 = my_h ? mx_other : mx, mx1 = my_h ? mx : mx_other;
    const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
    const float p = my_valid ? expf(sc - (my_h ? mn1 : mn0)) : 0.0f;
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
    // o[h] += p(h, row 2i + hb) * V[row] over this lane's rows (V re-read from the page).
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = 2 * i + hb;
        const float p0 = __shfl_sync(0xffffffffu, p, hb * 16 + i);
        const float p1 = __shfl_sync(0xffffffffu, p, hb * 16 + 8 + i);
        float vf[8];
        if (tp + r == kv_pos) {
            const float4* vc = reinterpret_cast<const float4*>(sm.qk[3] + 8 * dl);
            const float4 v0 = vc[0], v1 = vc[1];
            vf[0] = v0.x; vf[1] = v0.y; vf[2] = v0.z; vf[3] = v0.w;
            vf[4] = v1.x; vf[5] = v1.y; vf[6] = v1.z; vf[7] = v1.w;
        } else {
            unpack8(*reinterpret_cast<const uint4*>(page + PAGE_BYTES + (r * HD + 8 * dl) * 2), vf);
        }
#pragma unroll
        for (int d = 0; d < 8; ++d) {
            o[0][d] = fmaf(p0, vf[d], o[0][d]);
            o[1][d] = fmaf(p1, vf[d], o[1][d]);
        }
    }
}

// Phase B attention (> 128 cached positions): split `split` of KV head g, positions [t0, t1),
// from its KV pages [t0 / 16, ceil(t1 / 16)) in the ring (shared chunks: every warp waits for and
// releases each); warp w attends over every NCW-th page; the warps' states are merged into the
// split's (max, sum, unnormalised output) partials.
// Out of line (its register allocation stays apart from the rest of the kernel's); the shared
// memory is re-derived from the kernel's extern array so that its accesses stay shared-space ones.
__device__ __noinline__ void attention_split(const FusedArgs& a, int t0, int t1, int kv_pos,
                                             int num_sink, int g, int split, uint32_t q0) {
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw_ptr());
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int dl = lane & 15;
    float q0r[8], q1r[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) {
        q0r[d] = sm.qk[0][8 * dl + d];
        q1r[d] = sm.qk[1][8 * dl + d];
    }
    float m[2] = {-FLT_MAX, -FLT_MAX}, l[2] = {0.0f, 0.0f};
    float o[2][8];
#pragma unroll
    for (int d = 0; d < 8; ++d) o[0][d] = o[1][d] = 0.0f;
    // Pages [j0, j1) arrive two per chunk; page j0 + i belongs to warp i % NCW, so a warp's pages
    // sit in every fourth chunk and alternate between two ring slots: the next one lands while
    // the warp works on the current one.
    const int j0 = t0 / kPageTokens, j1 = t1 > t0 ? (t1 + kPageTokens - 1) / kPageTokens : j0;
    const int np = j1 - j0;
    for (int ci = 0; 2 * ci < np; ++ci) {
        const uint32_t qq = q0 + ci;
        const int slot = qq % NS;
        const int h = (warp - 2 * ci) & (NCW - 1);  // this warp's page in the chunk when h < 2
        if (warp_wait_full(sm, slot, (qq / NS) & 1, a) && h < 2 && 2 * ci + h < np) {
            split_page(sm, a, sm.ring[slot] + h * 2 * PAGE_BYTES, j0 + 2 * ci + h, t0, t1, kv_pos,
                       num_sink, q0r, q1r, m, l, o);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);  // one of NCW releases of a shared chunk
    }
    // The two row-parity halves hold partial sums over different rows: add them, then hand lane
    // k the dimensions 4k .. 4k + 3 (merge_warps' layout).
    AttnAcc acc;
    acc.m0 = m[0];
    acc.m1 = m[1];
    acc.l0 = l[0];
    acc.l1 = l[1];
#pragma unroll
    for (int d = 0; d < 8; ++d) {
        o[0][d] += __shfl_xor_sync(0xffffffffu, o[0][d], 16);
        o[1][d] += __shfl_xor_sync(0xffffffffu, o[1][d], 16);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float a0 = __shfl_sync(0xffffffffu, o[0][k], lane >> 1);
        const float b0 = __shfl_sync(0xffffffffu, o[0][4 + k], lane >> 1);
        const float a1 = __shfl_sync(0xffffffffu, o[1][k], lane >> 1);
        const float b1 = __shfl_sync(0xffffffffu, o[1][4 + k], lane >> 1);
        acc.o0[k] = (lane & 1) ? b0 : a0;
        acc.o1[k] = (lane & 1) ? b1 : a1;
    }
    merge_warps(sm, a, acc, g, split, true);
}

// Phase C prologue (> 128 positions): combine the split partials of heads 2g, 2g+1.
__device__ __forceinline__ void combine_group(Smem& sm, const FusedArgs& a, int S, int g) {
    const int t = threadIdx.x;
    const int head = 2 * g + (t >> 7), d = t & (HD - 1);
    float M = -FLT_MAX;
    for (int s = 0; s < S; ++s) {
        const float2 ml = __ldcg(a.part_ml + head * a.s_max + s);
        if (ml.y > 0.0f) M = fmaxf(M, ml.x);
    }
    float L = 0.0f, o = 0.0f;
    for (int s = 0; s < S; ++s) {
        const size_t pi = static_cast<size_t>(head) * a.s_max + s;
        const float2 ml = __ldcg(a.part_ml + pi);
        if (ml.y > 0.0f) {
            const float sc = expf(ml.x - M);
            L += ml.y * sc;
            o += __ldcg(a.part_o + pi * HD + d) * sc;
        }
    }
    xs_put(sm, t, o / L);
    bar_consumers();
}

// Phase C prologue of the tensor-parallel instance, whose ranks hold one to four KV groups and so
// 37 to 148 splits per group (up to 18 in the one-rank instance, which keeps the loop above).
__device__ __noinline__ void combine_group_wide(Smem& sm, const FusedArgs& a, int S, int g) {
    // Phase C: the flash-decoding merge of the S splits of KV group g (both query heads): each
    // split's (max, sum) pair staged in shared memory with one load per thread, the heads' maxima
    // and every split's scale computed once, then warp w sums the scaled o-partials of splits
    // w, w + NCW, ... (lane l: dimensions 4l .. 4l + 3 of both heads, the loads independent) and
    // the warps' sums meet in shared memory. Empty splits (sum 0) take no part.
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float2* mls = reinterpret_cast<float2*>(sm.xs4);             // [2][S]: (max, sum) -> (scale, -)
    float* ows = reinterpret_cast<float*>(sm.xs4) + 4 * a.s_max;  // [NCW][2][HD] warp sums
    for (int i = t; i < 2 * S; i += NCT) {
        const int hq = i / S, sp = i - hq * S;
        mls[i] = __ldcg(a.part_ml + static_cast<size_t>(2 * g + hq) * a.s_max + sp);
    }
    bar_consumers();
    if (warp < 2) {
        float2* m2 = mls + warp * S;
        float M = -FLT_MAX;
        for (int sp = lane; sp < S; sp += 32) {
            const float2 ml = m2[sp];
            if (ml.y > 0.0f) M = fmaxf(M, ml.x);
        }
        M = warp_max(M);
        float L = 0.0f;
        for (int sp = lane; sp < S; sp += 32) {
            const float2 ml = m2[sp];
            const float sc = ml.y > 0.0f ? expf(ml.x - M) : 0.0f;
            L += ml.y * sc;
            m2[sp].x = ml.y > 0.0f ? sc : -1.0f;  // -1: an empty split
        }
        L = warp_sum(L);
        if (lane == 0) sm.red[warp] = L;
    }
    bar_consumers();
    float4 o0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), o1 = o0;
    const float4* p0 = reinterpret_cast<const float4*>(a.part_o + static_cast<size_t>(2 * g) * a.s_max * HD) + lane;
    const float4* p1 = reinterpret_cast<const float4*>(a.part_o + static_cast<size_t>(2 * g + 1) * a.s_max * HD) + lane;
#pragma unroll 4
    for (int sp = warp; sp < S; sp += NCW) {
        const float sc0 = mls[sp].x, sc1 = mls[S + sp].x;
        const float4 u = __ldcg(p0 + static_cast<size_t>(sp) * (HD / 4));
        const float4 v = __ldcg(p1 + static_cast<size_t>(sp) * (HD / 4));
        if (sc0 >= 0.0f) {
            o0.x = fmaf(u.x, sc0, o0.x); o0.y = fmaf(u.y, sc0, o0.y);
            o0.z = fmaf(u.z, sc0, o0.z); o0.w = fmaf(u.w, sc0, o0.w);
        }
        if (sc1 >= 0.0f) {
            o1.x = fmaf(v.x, sc1, o1.x); o1.y = fmaf(v.y, sc1, o1.y);
            o1.z = fmaf(v.z, sc1, o1.z); o1.w = fmaf(v.w, sc1, o1.w);
        }
    }
    reinterpret_cast<float4*>(ows + (warp * 2 + 0) * HD)[lane] = o0;
    reinterpret_cast<float4*>(ows + (warp * 2 + 1) * HD)[lane] = o1;
    bar_consumers();
    const int hq = t >> 7, d = t & (HD - 1);
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) o += ows[(w * 2 + hq) * HD + d];
    xs_put(sm, t, o / sm.red[hq]);
    bar_consumers();
}

// Phase DE tail: sum_i h_i * w2t[i] over this CTA's MLP indices (shared chunks: warp w owns
// output columns [128w, 128w+128), 4 per lane); returns this lane's 4 sums (columns
// 128 warp + 4 lane ..), which the caller adds into Y[l] with one float4 atomic.
__device__ __forceinline__ float4 down_splitk(Smem& sm, const FusedArgs& a, uint32_t q0, int n) {
    constexpr int RPC = RPC_ROW;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nch = (n + RPC - 1) / RPC;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int ci = 0; ci < nch; ++ci) {
        const uint32_t qq = q0 + ci;
        const int slot = qq % NS;
        if (warp_wait_full(sm, slot, (qq / NS) & 1, a)) {
            const int rn = min(RPC, n - ci * RPC);
            // Unrolled with a predicate, so that the 16 shared-memory loads issue back to back.
            float hv[RPC];
            uint2 wv[RPC];
#pragma unroll
            for (int j = 0; j < RPC; ++j) {
                const bool in = j < rn && Q3_CHECK(ci * RPC + j < 64, 60, ci, j, n);
                hv[j] = in ? sm.hbuf[ci * RPC + j] : 0.0f;
                wv[j] = in ? reinterpret_cast<const uint2*>(sm.ring[slot] + j * D * 2 + warp * 256)[lane]
                           : make_uint2(0u, 0u);
            }
#pragma unroll
            for (int j = 0; j < RPC; ++j) {
                acc[0] = fmaf(hv[j], bf16_lo(wv[j].x), acc[0]);
                acc[1] = fmaf(hv[j], bf16_hi(wv[j].x), acc[1]);
                acc[2] = fmaf(hv[j], bf16_lo(wv[j].y), acc[2]);
                acc[3] = fmaf(hv[j], bf16_hi(wv[j].y), acc[3]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);  // one of NCW releases of a shared chunk
    }
    return make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// Write back the attention-sink rows of KV head g rotated by RoPE(position 1) (:817-827); every
// reader of this step applied the same rotation on the fly.
__device__ __forceinline__ void sink_writeback(const FusedArgs& a, const HeadPre& hp, int l, int g,
                                            int num_sink) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp >= num_sink) return;
    uint16_t* kcache = a.k_cache + static_cast<size_t>(l) * a.layer_elems;
    uint2* row = reinterpret_cast<uint2*>(kcache + paged(a.page_table, warp, g));
    float y[4];
    unpack_bf16x4(__ldcg(row + lane), y);
    rope_warp(y, hp.cs1);
    row[lane] = pack_bf16x4(y);
}

// Greedy argmax over the per-CTA partials (one warp), lowest index on ties: (value, index bits),
// the index local to this rank's lm_head rows (INT_MAX when there are none).
__device__ __forceinline__ float2 reduce_argmax(const FusedArgs& a, int G) {
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
    return make_float2(bv, __int_as_float(bi));
}

// Bounded wait until the two tagged words at p (16-byte aligned) carry `tag`.
__device__ bool poll2(const FusedArgs& a, const unsigned long long* p, unsigned tag,
                      volatile int* abort, unsigned long long& w0, unsigned long long& w1) {
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        ld_tagged2x(p, w0, w1, a.sys != 0);
        if (static_cast<unsigned>(w0 >> 32) == tag && static_cast<unsigned>(w1 >> 32) == tag) {
            return true;
        }
        if ((it & 15) == 15) {
            if (*abort || *reinterpret_cast<volatile unsigned*>(a.err) != 0u) {
                *abort = 1;
                return false;
            }
            if (clock64() - t0 > a.spin_cycles) {
                *abort = 1;
                atomicOr(a.err, 1u);
                Q3_CHECK(false, 3006, tag, static_cast<long long>(w0 >> 32), 0);
                return false;
            }
        }
    }
}

// The greedy token of step st over every rank's lm_head rows (one warp per CTA): CTA 0 sends
// this rank's best (value, global index) to every rank as two tagged words; lane r waits for
// rank r's pair and the warp keeps the best (lowest index on ties, src/inference.cpp:703-709).
// One rank without the exchange: the local best.
__device__ __noinline__ int greedy_token(Smem& sm, const FusedArgs& a, int G, int st, int c) {
    const int lane = threadIdx.x & 31;
    const float2 lb = reduce_argmax(a, G);
    int bi = __float_as_int(lb.y);
    if (!a.xchg) return bi == INT_MAX ? 0 : bi;  // one rank of the TP instance, no exchange
    const unsigned tag = step_tag(a, st, 0);
    if (c == 0 && lane == 0) {
        const unsigned gi = bi == INT_MAX ? 0x7fffffffu : static_cast<unsigned>(bi + a.v0);
        for (int d = 0; d < a.world; ++d) {
            unsigned long long* p = a.amx_dst[d] + 2 * a.rank;
            st_tagged_x(p, lb.x, tag, a.sys != 0);
            st_tagged_x(p + 1, __uint_as_float(gi), tag, a.sys != 0);
        }
    }
    float bv = -FLT_MAX;
    bi = INT_MAX;
    if (lane < a.world) {
        unsigned long long w0, w1;
        if (poll2(a, a.amx + 2 * lane, tag, &sm.abort_flag, w0, w1)) {
            bv = __uint_as_float(static_cast<unsigned>(w0));
            bi = static_cast<int>(static_cast<unsigned>(w1));
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

__device__ __noinline__ void stamp_write(unsigned long long* slot) {
    // Nanoseconds on the globaltimer scale, interpolated with the SM cycle counter (at the
    // 1965 MHz maximum clock) for a resolution finer than the globaltimer's update interval.
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw_ptr());
    const long long dc = clock64() - sm.clk0;
    *slot = sm.gt0 + static_cast<unsigned long long>(dc * 1000 / 1965);
}

__device__ __forceinline__ void stamp(const FusedArgs& a, unsigned kk, int G, int c, int which) {
    if (a.prof && threadIdx.x == 0) stamp_write(a.prof + (static_cast<size_t>(kk) * G + c) * 8 + which);
}

// Phase entry: with nb > 0 thread 0 waits until every CTA has made nb arrivals; in any case one
// verdict (no abort so far) is published to all consumer threads after the same barrier, so
// that all leave together on abort.
__device__ __forceinline__ bool phase_begin(Smem& sm, const FusedArgs& a, unsigned k, unsigned nb,
                                            int G, int c) {
    stamp(a, k, G, c, 0);
    if (threadIdx.x == 0) {
        const bool ok = nb == 0 || grid_wait(a, G * nb + a.barrier_offset, &sm.abort_flag, 4);
        sm.go = ok && sm.abort_flag == 0;
    }
    bar_consumers();
    stamp(a, k, G, c, 1);
    return sm.go != 0;
}

// Phase exit: all consumer threads are done with phase k; with `arrive` thread 0 adds this CTA's
// arrival on the grid counter (release).
__device__ __forceinline__ void phase_end(Smem& sm, const FusedArgs& a, unsigned k, bool arrive,
                                          int G, int c) {
    stamp(a, k, G, c, 6);
    bar_consumers();
    stamp(a, k, G, c, 7);
    if (threadIdx.x == 0) {
        if (arrive) red_release_add(a.bar, 1u);
        if (a.prof) {
            // Summed ring-wait cycles of all consumer warps in this phase.
            a.prof[(static_cast<size_t>(k) * G + c) * 8 + 5] = sm.wait_cycles;
            sm.wait_cycles = 0;
        }
    }
}

// This thread's four elements of a layer's down-projection output: the sum of its kYRep copies.
__device__ __forceinline__ float4 sum_y(const float* y) {
    float4 v[kYRep];
#pragma unroll
    for (int r = 0; r < kYRep; ++r) v[r] = __ldcg(reinterpret_cast<const float4*>(y + r * D) + threadIdx.x);
    float4 t = v[0];
#pragma unroll
    for (int r = 1; r < kYRep; ++r) t = add4(t, v[r]);
    return t;
}

// Tensor parallelism: x's down-projection update of layer lp (step st) summed over the ranks in
// rank order (the same sum on every rank): CTA 0 sends this rank's sum (the kYRep copies at y) to
// every rank as tagged words; every thread then waits for its four elements from each rank. The
// words alternate between two buffers from one exchange to the next: a rank writes a buffer again
// two exchanges later, after every rank's CTAs have read it (each rank's next exchange follows
// its DE grid barrier, which every CTA reaches after phase A).
__device__ __noinline__ float4 y_exchange(Smem& sm, const FusedArgs& a, const float* y, int st, int lp, int c) {
    const int x = st * a.n_layers + lp;
    const unsigned tag = step_tag(a, st, lp);
    const size_t base = static_cast<size_t>(x & 1) * kFusedMaxRanks * D + 4 * threadIdx.x;
    if (c == 0) {
        const float4 v = sum_y(y);
        for (int d = 0; d < a.world; ++d) {
            st_tagged4_x(a.yx_dst[d] + base + static_cast<size_t>(a.rank) * D, v, tag, a.sys != 0);
        }
    }
    float4 t = poll4(a, a.yx + base, tag, &sm.abort_flag, 5, a.sys != 0);
    for (int r = 1; r < a.world; ++r) {
        t = add4(t, poll4(a, a.yx + base + static_cast<size_t>(r) * D, tag, &sm.abort_flag, 5,
                          a.sys != 0));
    }
    return t;
}

// x = Xcur + Y[lp]: this rank's accumulators, or the ranks' sums through the exchange.
template <bool TP>
__device__ __forceinline__ float4 x_after(Smem& sm, const FusedArgs& a, float4 xcur, const float* yb,
                                          int st, int lp, int c) {
    const float* y = yb + static_cast<size_t>(lp) * kYRep * D;
    return add4(xcur, Shard<TP>::xchg(a) ? y_exchange(sm, a, y, st, lp, c) : sum_y(y));
}

// Greedy token of step st: this rank's best (TP = false), else over every rank.
template <bool TP>
__device__ __forceinline__ int step_token(Smem& sm, const FusedArgs& a, int G, int st, int c) {
    if (TP) return greedy_token(sm, a, G, st, c);
    const int bi = __float_as_int(reduce_argmax(a, G).y);
    return bi == INT_MAX ? 0 : bi;
}

// Phase A input: the embedding row of the step's token (layer 0; the token is the greedy argmax of
// the previous step, or the teacher-forced one) or x = Xcur + Y[l-1], with Xcur this thread's four
// elements of the residual stream after the previous layer's o_proj (kept in registers) and yb the
// step's down-projection accumulators; writes (CTA 0) the debug tap. Returns this thread's
// four elements of x.
template <bool TP>
__device__ __forceinline__ float4 phase_a_input(Smem& sm, const FusedArgs& a, const StepParams& sp0,
                                             int st, int l, float4 xcur, const float* yb, int G,
                                             int c) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float4 xv;
    if (l == 0) {
        if (warp == 0) {
            int tok = sp0.token;
            if (st > 0) {
                const int best = step_token<TP>(sm, a, G, st - 1, c);
                const int idx = sp0.step + st;
                tok = (a.forced && idx < sp0.n_forced) ? __ldg(a.forced + idx) : best;
                if (c == 0 && lane == 0) a.token_log[idx - 1] = best;
            }
            if (lane == 0) sm.token = tok;
        }
        bar_consumers();
        const uint2 e = __ldg(reinterpret_cast<const uint2*>(
                                  a.embed + static_cast<size_t>(sm.token) * D) + tid);
        xv = make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
        // Zero this CTA's share of the other step parity's down-projection accumulators: their
        // last readers arrived at the previous step's lm_head barrier, their next writers (next
        // step) come after this step's.
        float* yz = a.ybuf + static_cast<size_t>((a.parity0 + st + 1) & 1) * a.n_layers * kYRep * D;
        const Span ys = part(a.n_layers * kYRep * D, G, c);
        for (int i = tid; i < ys.n; i += NCT) yz[ys.r0 + i] = 0.0f;
    } else {
        xv = x_after<TP>(sm, a, xcur, yb, st, l - 1, c);
    }
    if (a.taps && c == 0) reinterpret_cast<float4*>(a.taps + static_cast<size_t>(l) * D)[tid] = xv;
    return xv;
}

// Xcur = x + sum_g partial_g over the eight KV-head groups (in group order), this thread's four
// elements, from the tagged o_proj partials of phase BC / C.
// The first probes of all eight groups are issued together (one L2 round trip when the partials
// have landed); only groups not yet written are then polled, one after another.
template <bool SYS>
__device__ __forceinline__ float4 gather_oproj(Smem& sm, const FusedArgs& a, float4 xv,
                                               unsigned tag) {
    unsigned long long w[NKV][4];
#pragma unroll
    for (int gg = 0; gg < NKV; ++gg) {
        const unsigned long long* p = a.opart + static_cast<size_t>(gg) * D + 4 * threadIdx.x;
        ld_tagged2x(p, w[gg][0], w[gg][1], SYS);
        ld_tagged2x(p + 2, w[gg][2], w[gg][3], SYS);
    }
    float4 proj = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int gg = 0; gg < NKV; ++gg) {
        const bool ready = static_cast<unsigned>(w[gg][0] >> 32) == tag &&
                           static_cast<unsigned>(w[gg][1] >> 32) == tag &&
                           static_cast<unsigned>(w[gg][2] >> 32) == tag &&
                           static_cast<unsigned>(w[gg][3] >> 32) == tag;
        const float4 p =
            ready ? make_float4(__uint_as_float(static_cast<unsigned>(w[gg][0])),
                                __uint_as_float(static_cast<unsigned>(w[gg][1])),
                                __uint_as_float(static_cast<unsigned>(w[gg][2])),
                                __uint_as_float(static_cast<unsigned>(w[gg][3])))
                  : poll4(a, a.opart + static_cast<size_t>(gg) * D + 4 * threadIdx.x, tag,
                          &sm.abort_flag, 3, SYS);
        proj = add4(proj, p);
    }
    return add4(xv, proj);
}

template <bool TP>
__global__ void __launch_bounds__(NT, 1) decode_fused_kernel(const __grid_constant__ FusedArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;

    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], NCW);  // every consumer warp releases each chunk
        }
        sm.abort_flag = 0;
        sm.wait_cycles = 0;
        sm.gt0 = globaltimer();
        sm.clk0 = clock64();
        if (a.prof) {
            // Instrumentation: pair the cycle counter with the moment the globaltimer ticks, so
            // that the stamps of different SMs share one time base to within a loop iteration
            // rather than to within the timer's update interval. Bounded: gives up after 2^16
            // reads and keeps the first pairing.
            for (int it = 0; it < (1 << 16); ++it) {
                const unsigned long long t = globaltimer();
                const long long cnow = clock64();
                if (t != sm.gt0) {
                    sm.gt0 = t;
                    sm.clk0 = cnow;
                    break;
                }
            }
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == NCW) {
        if (lane == 0) {
            Producer<TP> pr{sm, a};
            pr.run(G, c);
        }
        return;
    }

    // ---------------- consumers
    const StepParams sp0 = a.sp_from_args ? a.sp_init : *a.sp;
    const int nkv = Shard<TP>::nkv(a), kv0 = Shard<TP>::kv0(a), hl = Shard<TP>::hl(a);
    const int P = G / nkv;
    const bool in_grp = c < nkv * P;
    const int gl = c % nkv, g = kv0 + gl, gp = c / nkv;  // BC: KV group (local, global)
    unsigned k = 0;   // global phase index (profiling stamps)
    unsigned nb = 0;  // grid arrivals every CTA has made so far
    uint32_t q = 0;   // ring chunk index
    float4 xcur = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // Xcur, this thread's 4 elements

    for (int st = 0; st < a.n_steps; ++st) {
        const StepPos p = step_pos(a, sp0, st);
        float* yb = a.ybuf + static_cast<size_t>((a.parity0 + st) & 1) * a.n_layers * kYRep * D;
        for (int l = 0; l < a.n_layers; ++l) {
            const FusedLayer w = a.layers[l];
            const unsigned tag = step_tag(a, st, l);
            // ---- A: x = Xcur + Y[l-1], RmsNorm -> [wq;wk;wv] (tagged)
            float4 xv;
            {
                const uint2 nw = load_norm(w.attn_norm);
                if (!phase_begin(sm, a, k, nb, G, c)) return;
                xv = phase_a_input<TP>(sm, a, sp0, st, l, xcur, yb, G, c);
                stage_norm(sm, xv, nw, a.eps);
                stamp(a, k, G, c, 3);
                const int qkv_rows = nkv * 4 * HD;
                const Span s = part(qkv_rows, G, c);
                if (chunks_of(s.n, RPC_ROW) * 2 <= NCW) {
                    consume_rows_halves(sm, a, q, s.r0, s.n, a.qkvt, tag);
                } else {
                    consume_rows<D, RPC_ROW, kTag>(sm, a, q, s.r0, s.n, nullptr, qkv_rows, a.qkvt, tag);
                }
                q += chunks_of(s.n, RPC_ROW);
                stamp(a, k, G, c, 4);
                phase_end(sm, a, k++, false, G, c);
            }
            HeadPre hp;
            head_preload(hp, a, w, p.pos);
            const Span os = part(D, P, gp);
            const size_t opart_g = static_cast<size_t>(g) * D;  // group g's partial in every opart
            if (p.shrt) {
                // ---- BC: attention of KV head g from the ring, o_proj partial of group g
                if (!phase_begin(sm, a, k, 0, G, c)) return;
                if (in_grp) {
                    prep_heads(sm, a, hp, l, nkv, gl, g, p.kv_pos, gp == 0, tag);
                    stamp(a, k, G, c, 2);
                    attention_short(sm, a, hp, p.kv_len, p.kv_pos, p.num_sink, gl, q);
                    q += chunks_of(p.kv_len, kPageTokens);
                    stamp(a, k, G, c, 3);
                    consume_rows<GRP, RPC_GRP, TP ? kTagX : kTag>(sm, a, q, os.r0, os.n, nullptr, D,
                                                                  a.opart + opart_g, tag, opart_g);
                    q += chunks_of(os.n, RPC_GRP);
                    stamp(a, k, G, c, 4);
                }
                phase_end(sm, a, k++, false, G, c);
            } else {
                // ---- B: split-K attention partials
                if (!phase_begin(sm, a, k, 0, G, c)) return;
                const SplitRange sr = split_range(p, c, nkv);
                if (sr.on) {
                    const bool own = p.kv_pos >= sr.t0 && p.kv_pos < sr.t1;
                    prep_heads(sm, a, hp, l, nkv, sr.g, kv0 + sr.g, p.kv_pos, own, tag);
                    attention_split(a, sr.t0, sr.t1, p.kv_pos, p.num_sink, sr.g, sr.s, q);
                    q += static_cast<uint32_t>(chunks_of_i(sr.j1 - sr.j0, 2));
                }
                phase_end(sm, a, k++, true, G, c);
                ++nb;
                // ---- C: combine + o_proj partial of group g
                if (!phase_begin(sm, a, k, nb, G, c)) return;
                if (in_grp) {
                    if (TP) {
                        combine_group_wide(sm, a, p.splits, gl);
                    } else {
                        combine_group(sm, a, p.splits, gl);
                    }
                    consume_rows<GRP, RPC_GRP, TP ? kTagX : kTag>(sm, a, q, os.r0, os.n, nullptr, D,
                                                                  a.opart + opart_g, tag, opart_g);
                    q += chunks_of(os.n, RPC_GRP);
                }
                phase_end(sm, a, k++, false, G, c);
            }
            // ---- DE: Xcur = x + o_proj, RmsNorm -> silu(w1 .) * (w3 .) -> split-K down into Y[l]
            {
                const uint2 mw = load_norm(w.mlp_norm);
                if (!phase_begin(sm, a, k, 0, G, c)) return;
                xcur = (TP && a.sys) ? gather_oproj<true>(sm, a, xv, tag)
                                     : gather_oproj<false>(sm, a, xv, tag);
                stage_norm(sm, xcur, mw, a.eps);
                stamp(a, k, G, c, 2);
                const Span hs = part(hl, G, c);
                consume_rows<D, RPC_PAIR, kPair>(sm, a, q, hs.r0, hs.n, sm.hbuf, 64);
                q += chunks_of(hs.n, RPC_PAIR);
                bar_consumers();
                stamp(a, k, G, c, 3);
                const float4 yd = down_splitk(sm, a, q, hs.n);
                q += chunks_of(hs.n, RPC_ROW);
                stamp(a, k, G, c, 4);
                red_add4(yb + (static_cast<size_t>(l) * kYRep + c % kYRep) * D + 4 * tid, yd);
                if (c < nkv && p.num_sink > 0) sink_writeback(a, hp, l, kv0 + c, p.num_sink);
                phase_end(sm, a, k++, true, G, c);
                ++nb;
            }
        }
        // ---- final RmsNorm + lm_head + per-CTA argmax
        const uint2 fw = load_norm(a.final_norm);
        if (!phase_begin(sm, a, k, nb, G, c)) return;
        const float4 xv = x_after<TP>(sm, a, xcur, yb, st, a.n_layers - 1, c);
        if (a.taps && c == 0) {
            reinterpret_cast<float4*>(a.taps + static_cast<size_t>(a.n_layers) * D)[tid] = xv;
        }
        stage_norm(sm, xv, fw, a.eps);
        const Span vs = part2(a.vocab, G, c);
        consume_rows<D, RPC_ROW, kLogits>(sm, a, q, vs.r0, vs.n, a.logits, a.vocab);
        q += chunks_of(vs.n, RPC_ROW);
        bar_consumers();
        if (tid == 0) {
            float bv = sm.best[0].x;
            int bi = __float_as_int(sm.best[0].y);
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
        phase_end(sm, a, k++, true, G, c);
        ++nb;
    }

    // Final greedy token and the device-side advance of the step parameters (CTA 0).
    if (c == 0) {
        if (!phase_begin(sm, a, k, nb, G, c)) return;
        if (warp == 0) {
            const int best = step_token<TP>(sm, a, G, a.n_steps - 1, c);
            if (lane == 0) {
                const int idx = sp0.step + a.n_steps;
                a.token_log[idx - 1] = best;
                if (a.token_out) *a.token_out = best;
                if (a.err_out) *a.err_out = *reinterpret_cast<volatile unsigned*>(a.err);
                StepParams np = sp0;
                np.token = (a.forced && idx < sp0.n_forced) ? a.forced[idx] : best;
                np.step = idx;
                np.pos = sp0.pos + a.n_steps;
                step_positions(np.pos, a.ctx, &np.num_sink, &np.kv_pos, &np.kv_len);
                *a.sp = np;
            }
        }
        // Every CTA has made its last arrival and waits on the counter no more (each producer
        // passed its last grid wait before its consumers could finish): the counter starts the
        // next launch at zero.
        if (tid == 0) *a.bar = 0u;
    }
}

// ------------------------------------------------------------------ weight re-layout

__global__ void permute_wo_kernel(const uint16_t* __restrict__ wo, uint16_t* __restrict__ wop) {
    // wop[g][r][j] = wo[r][256 g + j]; one thread per 8-element vector.
    const size_t n = static_cast<size_t>(D) * QD / 8;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t e = i * 8;
        const int r = static_cast<int>(e / QD), col = static_cast<int>(e % QD);
        const int gg = col / GRP, j = col % GRP;
        const uint4 v = *reinterpret_cast<const uint4*>(wo + e);
        *reinterpret_cast<uint4*>(wop + (static_cast<size_t>(gg) * D + r) * GRP + j) = v;
    }
}

__global__ void swizzle_rows_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                    size_t rows, int K) {
    // Odd rows: swap the two 64-byte halves of every 128-byte block (the layout fma_rows8 reads).
    const size_t units = static_cast<size_t>(K) / 8;
    const size_t n = rows * units;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = i / units, u = i % units;
        const size_t du = u ^ ((r & 1) << 2);
        reinterpret_cast<uint4*>(dst)[r * units + du] = reinterpret_cast<const uint4*>(src)[i];
    }
}

__global__ void transpose_w2_kernel(const uint16_t* __restrict__ w2, uint16_t* __restrict__ w2t) {
    // w2t[i][r] = w2[r][i] for w2 [1024][3072], through 32x32 shared tiles.
    __shared__ uint16_t tile[32][33];
    const int i0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int y = threadIdx.y; y < 32; y += blockDim.y)
        tile[y][threadIdx.x] = w2[static_cast<size_t>(r0 + y) * H + i0 + threadIdx.x];
    __syncthreads();
    for (int y = threadIdx.y; y < 32; y += blockDim.y)
        w2t[static_cast<size_t>(i0 + y) * D + r0 + threadIdx.x] = tile[threadIdx.x][y];
}

}  // namespace

bool fused_supported(const q3_config& c) {
    return c.dim == D && c.hidden_dim == H && c.head_dim == HD && c.n_heads == NQ &&
           c.n_kv_heads == NKV && c.rotary_dim == HD;
}

size_t fused_smem_bytes() { return sizeof(Smem); }

size_t fused_ybuf_floats(int n_layers) { return 2ull * n_layers * kYRep * D; }

int fused_l2_ahead() {
    // Layers of L2 run-ahead; Q3_FUSED_L2_AHEAD overrides (0 turns the prefetch off).
    static const int v = [] {
        const char* e = getenv("Q3_FUSED_L2_AHEAD");
        const int n = e ? atoi(e) : 1;
        return n < 0 ? 0 : (n > 3 ? 3 : n);
    }();
    return v;
}

int fused_phases_per_step(int n_layers, int kv_len) {
    return n_layers * (kv_len <= T_SHORT ? 3 : 4) + 1;
}

int fused_grid(int device) {
    int sms = 0;
    Q3_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    int per_sm = 1;
    for (auto kern : {decode_fused_kernel<false>, decode_fused_kernel<true>}) {
        Q3_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(sizeof(Smem))));
        int n = 0;
        Q3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, NT, sizeof(Smem)));
        per_sm = std::min(per_sm, n);
    }
    if (per_sm < 1) return 0;
    // Every CTA must own at most 64 MLP indices (the h buffer) and the grid must cover 8 groups.
    if (sms < 48) return 0;
    return sms;
}

void launch_decode_fused(const FusedArgs& a, int grid, cudaStream_t s) {
    // combine_group stages 2 x s_max (max, sum) pairs and NCW x 2 x HD warp sums in sm.xs4.
    static_assert(sizeof(Smem::xs4) >= 16 * 256 + NCW * 2 * HD * 4, "combine staging");
    if (a.s_max < 1 || a.s_max > 256) {
        throw std::invalid_argument("fused decode: 1..256 attention splits per KV group");
    }
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
    // The tensor-parallel instance for several ranks or a routed exchange; else the one-rank one.
    if (a.world > 1 || a.xchg) {
        Q3_CUDA(cudaLaunchKernelEx(&cfg, decode_fused_kernel<true>, a));
    } else {
        Q3_CUDA(cudaLaunchKernelEx(&cfg, decode_fused_kernel<false>, a));
    }
}

void launch_permute_wo(const uint16_t* wo, uint16_t* wop, cudaStream_t s) {
    permute_wo_kernel<<<1024, 256, 0, s>>>(wo, wop);
    Q3_CUDA(cudaGetLastError());
}

void launch_swizzle_rows(const uint16_t* src, uint16_t* dst, size_t rows, int K, cudaStream_t s) {
    if (K % 64 != 0) throw std::invalid_argument("row swizzle needs K % 64 == 0");
    swizzle_rows_kernel<<<2048, 256, 0, s>>>(src, dst, rows, K);
    Q3_CUDA(cudaGetLastError());
}

void launch_transpose_w2(const uint16_t* w2, uint16_t* w2t, cudaStream_t s) {
    transpose_w2_kernel<<<dim3(H / 32, D / 32), dim3(32, 8), 0, s>>>(w2, w2t);
    Q3_CUDA(cudaGetLastError());
}

}  // namespace q3
