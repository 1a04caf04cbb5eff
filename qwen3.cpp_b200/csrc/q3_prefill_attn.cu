// Causal prefill attention on tcgen05 tensor cores (sm_100a): FastAttn + Softmax
// (src/inference.cpp:1017-1058, :925-946) for every prompt token of a chunk at once.
//
// One CTA per (64-token query block, KV head g); a 1-D grid ordered longest query block first
// across all KV heads. The two query heads 2g and 2g+1 share the KV head, so their 64 rows each
// are stacked into one 128-row operand Q (rows 0-63 head 2g, rows 64-127 head 2g+1) and every K/V
// tile is read once for both. KV tiles are 128 positions (8 pages of 16), loaded by TMA from the
// paged cache: one 4-D box per 64-column panel when the 8 pages are physically consecutive, else
// one 2-D box per page. K runs one tile ahead of V in separate two-stage rings. Per tile j:
//   MMA warp      S_j = Q . K_j^T into TMEM buffer j%2 (M=128, N=128, K=128 dims)
//   softmax warps two threads per row r (64 keys each): masked partial row max exchanged with the
//                 partner thread, P_j = exp2(S_j*scale - m_j) written to shared memory as bf16 in
//                 the MMA's operand layout, partial row sums
//   MMA warp      O_j = P_j . V_j into TMEM buffer 2 + j%2 (V read as an MN-major operand)
//   softmax warps acc = acc * exp2(m_{j-1} - m_j) + O_j in registers (64 fp32 per thread)
// S_{j+1} runs on the tensor cores while the softmax warps work on S_j, and O_j while they work
// on S_{j+1}. Warp roles: 0 TMA producer, 1 MMA issuer, 2-9 softmax (warp w reads TMEM lanes
// 32*(w%4).. and column half (w-2)/4).
// Every wait is bounded; a wait that gives up sets *err and the CTA drains and returns.
#include <cuda_bf16.h>

#include <stdexcept>

#include "q3_prefill.cuh"
#include "q3_sm100.cuh"

namespace q3 {

namespace {

using namespace sm100;

constexpr int HD = 128;
constexpr int ROWS = 128;                 // 64 tokens x 2 query heads
constexpr int TOK = 64;
constexpr int KEYS = 128;                 // KV positions per tile
constexpr int PANEL = ROWS * 128;         // bytes of a 64-column panel of 128 rows
constexpr int Q_OFF = 0;                  // Q: 2 panels
constexpr int KV_OFF = 2 * PANEL;         // 2 stages x (K: 2 panels, V: 2 panels)
constexpr int KV_STAGE = 4 * PANEL;
constexpr int P_OFF = KV_OFF + 2 * KV_STAGE;  // 2 buffers x 2 panels
constexpr int P_BUF = 2 * PANEL;
constexpr int RED_OFF = P_OFF + 2 * P_BUF;    // 229,376: row-max exchange [2][2][128] floats
constexpr int BAR_OFF = RED_OFF + 2 * 2 * ROWS * 4;
constexpr int SMEM = BAR_OFF + 320;  // 34 barriers + slot + flag           // 231,680 (base 1024-aligned, checked)
constexpr int NSOFT = 8;                      // softmax warps
constexpr int NTHREADS = 64 + NSOFT * 32;
constexpr uint32_t TMEM_COLS = 512;       // S0, S1, O0, O1: 128 fp32 columns each

// 4-D tiled TMA load (x innermost), completing on an mbarrier.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            int w, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}


__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// MN-major operand descriptor with 128-byte swizzling: 64-element rows of 128 B along N, 8-row
// groups along K at 1024 B, further 64-element panels along N at `panel_bytes`.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t panel_bytes) {
    uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
    d |= static_cast<uint64_t>((panel_bytes >> 4) & 0x3FFF) << 16;  // leading: next N panel
    d |= static_cast<uint64_t>(1024 >> 4) << 32;                     // stride: next 8 K rows
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// 2^x with the MUFU instruction (relative error ~2^-22; the probabilities are rounded to bf16).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 64 consecutive fp32 TMEM columns of this thread's lane: two loads, one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]),
          "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]),
          "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
          "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]),
          "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]),
          "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr), "r"(taddr + 32u)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void fail(volatile int* abort, unsigned* err, unsigned code) {
    *abort = 1;
    if (err) atomicCAS(err, 0u, code);
}

// acc = acc * exp2(m_acc - m_i) + O_i for this thread's 64 columns of O_i (TMEM buffer
// 2 + i%2); m_acc = m_i.
__device__ __forceinline__ bool fold_o(float (&acc)[HD / 2], float& m_acc, int i, float m_i,
                                       uint32_t tmem_lane_half, uint64_t* o_full,
                                       uint64_t* o_empty, int lane, long long budget,
                                       volatile int* abort) {
    if (!mbar_wait_warp(&o_full[i & 1], (i >> 1) & 1, budget, abort)) return false;
    tc_fence_after();
    const float f = ex2(m_acc - m_i);
    const uint32_t ob = tmem_lane_half + static_cast<uint32_t>(256 + (i & 1) * 128);
    float o[64];
    tmem_ld64(ob, o);
    const float2 f2 = make_float2(f, f);
#pragma unroll
    for (int k = 0; k < 64; k += 2) {
        const float2 r2 = ffma2(make_float2(acc[k], acc[k + 1]), f2, make_float2(o[k], o[k + 1]));
        acc[k] = r2.x;
        acc[k + 1] = r2.y;
    }
    m_acc = m_i;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&o_empty[i & 1]);
    return true;
}

// The two threads of row r (one per column half) publish a value and read the other's, through
// shared memory and mx_bar[t & 1] (use number t >> 1 of it). NaN when the wait gave up.
__device__ __forceinline__ float exchange_row(float* red, uint64_t* mx_bar, int t, int half, int r,
                                              float v, long long budget, volatile int* abort) {
    uint64_t* b = &mx_bar[(t & 1) * 4 + (r >> 5)];
    red[((t & 1) * 2 + half) * ROWS + r] = v;
    mbar_arrive(b);
    if (!mbar_wait_warp(b, (t >> 1) & 1, budget, abort)) return __int_as_float(0x7fc00000);
    return red[((t & 1) * 2 + (half ^ 1)) * ROWS + r];
}

__global__ void __launch_bounds__(NTHREADS, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tq,
                           const __grid_constant__ CUtensorMap tk,
                           const __grid_constant__ CUtensorMap tv,
                           const __grid_constant__ CUtensorMap tk4,
                           const __grid_constant__ CUtensorMap tv4, const PrefillAttnTcArgs a) {
    extern __shared__ __align__(1024) uint8_t sm[];
    pdl_wait();
    pdl_trigger();
    // The swizzled operand panels need a 1024-byte aligned base; nothing is touched otherwise.
    if ((smem_u32(sm) & 1023) != 0) {
        if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0u, 10u);
        return;
    }
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BAR_OFF);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;   // [2] K tiles
    uint64_t* kv_empty = bars + 3;  // [2] K tiles
    uint64_t* v_full = bars + 19;   // [2]
    uint64_t* v_empty = bars + 21;  // [2]
    uint64_t* s_full = bars + 5;    // [2]
    uint64_t* s_empty = bars + 7;   // [2]
    uint64_t* p_full = bars + 9;    // [2]
    uint64_t* o_full = bars + 11;   // [2]
    uint64_t* o_empty = bars + 13;  // [2]
    uint64_t* done = bars + 15;
    uint64_t* mx_bar = bars + 24;   // [2 parities][4 row quadrants]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 32);
    float* red = reinterpret_cast<float*>(sm + RED_OFF);  // [tile parity][half][row]
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // 1-D grid, longest query blocks first across every KV head, so that the block scheduler
    // starts the longest work first and the short blocks fill the tail.
    const int g = static_cast<int>(blockIdx.x) % a.n_kv;
    // This CTA's query block: rows tok0 .. tok0 + nrows - 1 of the q / out buffers, the tokens at
    // positions pos_first .. pos_first + nrows - 1 of the sequence whose page table is `table`.
    int tok0, nrows, pos_first;
    const int32_t* table;
    if (a.work) {
        // Several sequences (work items ordered longest first by the host).
        const int4 it = a.work[blockIdx.x / a.n_kv];
        tok0 = it.x;
        nrows = it.y;
        pos_first = it.z;
        table = a.page_table + it.w;
    } else {
        const int n_qb = gridDim.x / a.n_kv;
        const int qb = n_qb - 1 - static_cast<int>(blockIdx.x) / a.n_kv;
        tok0 = qb * TOK;
        nrows = min(a.rows - tok0, TOK);
        pos_first = a.pos0 + tok0;
        table = a.page_table;
    }
    const int kv_end = pos_first + nrows;
    const int table_len = a.pages_per_seq ? a.pages_per_seq : a.n_pages;
    const int ntiles = (kv_end + KEYS - 1) / KEYS;
    const int valid_pages = (kv_end + kPageTokens - 1) / kPageTokens;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], NSOFT);
            mbar_init(&p_full[i], NSOFT);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_empty[i], NSOFT);
            for (int qd = 0; qd < 4; ++qd) mbar_init(&mx_bar[i * 4 + qd], 64);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        mbar_init(done, 1);
        *abort = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        tma_prefetch_map(&tq);
        tma_prefetch_map(&tk);
        tma_prefetch_map(&tv);
        tma_prefetch_map(&tk4);
        tma_prefetch_map(&tv4);
        tmem_alloc(tmem_slot, TMEM_COLS);
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------------ TMA producer
            uint32_t issued = 0, issued_parity = 0;  // bit 0: q, bits 1-2: kv stages
            mbar_arrive_expect_tx(q_full, 2 * PANEL);
            for (int hs = 0; hs < 2; ++hs) {
                for (int p = 0; p < 2; ++p) {
                    tma_load_2d(sm + Q_OFF + p * PANEL + hs * (PANEL / 2), &tq,
                                (2 * g + hs) * HD + p * 64, tok0, q_full);
                }
            }
            issued |= 1u;
            uint32_t vissued = 0, vissued_parity = 0;
            // Page rows of a tile's 8 pages (the last tile's pages past the table repeat its last
            // valid page; such a tile takes the per-page path).
            constexpr int PPT = KEYS / kPageTokens;
            auto load_rows = [&](int j, int (&r)[PPT]) {
                const int lp0 = j * PPT;
                const bool all_in = lp0 + PPT <= table_len;
#pragma unroll
                for (int pg = 0; pg < PPT; ++pg) {
                    r[pg] = __ldg(table + (all_in ? lp0 + pg : min(lp0 + pg, valid_pages - 1)));
                }
            };
            // The page rows of tile step + 1 are loaded while the waits of step run (they were a
            // dependent global round trip in front of every copy).
            int rows_k[PPT] = {}, rows_v[PPT] = {}, rows_n[PPT] = {};
            if (ntiles > 0) load_rows(0, rows_k);
            // Loads run K one tile ahead of V: K_{j+1} waits only for S_{j-1}, V_j for PV_{j-2},
            // so the score MMAs never wait behind the slower P.V chain.
            for (int step = 0; step <= ntiles && !*abort; ++step) {
                if (step + 1 < ntiles) load_rows(step + 1, rows_n);
                for (int kind = 0; kind < 2 && !*abort; ++kind) {
                    const int j = kind ? step - 1 : step;   // kind 0: K_step, kind 1: V_{step-1}
                    if (j < 0 || j >= ntiles) continue;
                    const int st = j & 1;
                    const uint32_t ph = (j >> 1) & 1;
                    uint8_t* dst = sm + KV_OFF + st * KV_STAGE + kind * 2 * PANEL;
                    uint64_t* emp = kind ? &v_empty[st] : &kv_empty[st];
                    uint64_t* ful = kind ? &v_full[st] : &kv_full[st];
                    int rows8[PPT];
#pragma unroll
                    for (int pg = 0; pg < PPT; ++pg) rows8[pg] = kind ? rows_v[pg] : rows_k[pg];
                    const bool all_in = j * PPT + PPT <= table_len;
                    bool contiguous = all_in;
#pragma unroll
                    for (int pg = 1; pg < KEYS / kPageTokens; ++pg) {
                        contiguous &= rows8[pg] == rows8[0] + pg;
                    }
                    const int page4 = a.layer * a.n_pages + rows8[0];
                    if (!mbar_wait(emp, ph ^ 1, a.budget, abort)) {
                        fail(abort, a.err, 11);
                        break;
                    }
                    mbar_arrive_expect_tx(ful, 2 * PANEL);
                    if (contiguous) {
#pragma unroll
                        for (int p = 0; p < 2; ++p) {
                            tma_load_4d(dst + p * PANEL, kind ? &tv4 : &tk4, p * 64, 0, g, page4, ful);
                        }
                    } else {
#pragma unroll
                        for (int pg = 0; pg < KEYS / kPageTokens; ++pg) {
                            const int row =
                                ((a.layer * a.n_pages + rows8[pg]) * a.n_kv + g) * kPageTokens;
#pragma unroll
                            for (int p = 0; p < 2; ++p) {
                                tma_load_2d(dst + p * PANEL + pg * (kPageTokens * 128),
                                            kind ? &tv : &tk, p * 64, row, ful);
                            }
                        }
                    }
                    if (kind) {
                        vissued |= 1u << st;
                        vissued_parity = (vissued_parity & ~(1u << st)) | (ph << st);
                    } else {
                        issued |= 2u << st;
                        issued_parity = (issued_parity & ~(2u << st)) | (ph << (st + 1));
                    }
                }
#pragma unroll
                for (int pg = 0; pg < PPT; ++pg) {
                    rows_v[pg] = rows_k[pg];
                    rows_k[pg] = rows_n[pg];
                }
            }
            for (int st = 0; st < 2; ++st) {
                if (!(vissued & (1u << st))) continue;
                const long long t1 = clock64();
                while (!mbar_try_wait(&v_full[st], (vissued_parity >> st) & 1)) {
                    if (clock64() - t1 > a.budget) { fail(abort, a.err, 12); break; }
                }
            }
            // Drain: every issued load has landed before the CTA exits.
            const long long t0 = clock64();
            while (!mbar_try_wait(q_full, 0)) {
                if (clock64() - t0 > a.budget) {
                    fail(abort, a.err, 12);
                    break;
                }
            }
            for (int st = 0; st < 2; ++st) {
                if (!(issued & (2u << st))) continue;
                const long long t1 = clock64();
                while (!mbar_try_wait(&kv_full[st], (issued_parity >> (st + 1)) & 1)) {
                    if (clock64() - t1 > a.budget) {
                        fail(abort, a.err, 12);
                        break;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            const uint32_t idesc_s = a.f16 ? idesc_f16_f32(ROWS, KEYS) : idesc_bf16_f32(ROWS, KEYS);
            const uint32_t idesc_pv =
                (a.f16 ? idesc_f16_f32(ROWS, HD) : idesc_bf16_f32(ROWS, HD)) | (1u << 16);  // B MN-major
            const uint32_t q_addr = smem_u32(sm + Q_OFF);
            bool ok = mbar_wait(q_full, 0, a.budget, abort);
            if (!ok) fail(abort, a.err, 13);
            for (int j = 0; ok && j <= ntiles && !*abort; ++j) {
                if (j < ntiles) {
                    const int st = j & 1;
                    if (!mbar_wait(&kv_full[st], (j >> 1) & 1, a.budget, abort) ||
                        !mbar_wait(&s_empty[j & 1], ((j >> 1) & 1) ^ 1, a.budget, abort)) {
                        fail(abort, a.err, 14);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t k_addr = smem_u32(sm + KV_OFF + st * KV_STAGE);
                    const uint32_t d = tmem + static_cast<uint32_t>((j & 1) * 128);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint64_t ad = desc_k_sw128(q_addr + (kk >> 2) * PANEL) + 2 * (kk & 3);
                        const uint64_t bd = desc_k_sw128(k_addr + (kk >> 2) * PANEL) + 2 * (kk & 3);
                        mma_bf16(d, ad, bd, idesc_s, kk > 0);
                    }
                    mma_commit(&s_full[j & 1]);
                    mma_commit(&kv_empty[st]);
                }
                if (j >= 1) {
                    const int i = j - 1, st = i & 1;
                    if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, a.budget, abort) ||
                        !mbar_wait(&v_full[st], (i >> 1) & 1, a.budget, abort) ||
                        !mbar_wait(&o_empty[i & 1], ((i >> 1) & 1) ^ 1, a.budget, abort)) {
                        fail(abort, a.err, 15);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t p_addr = smem_u32(sm + P_OFF + (i & 1) * P_BUF);
                    const uint32_t v_addr = smem_u32(sm + KV_OFF + st * KV_STAGE + 2 * PANEL);
                    const uint32_t d = tmem + static_cast<uint32_t>(256 + (i & 1) * 128);
#pragma unroll
                    for (int kk = 0; kk < KEYS / 16; ++kk) {
                        const uint64_t ad = desc_k_sw128(p_addr + (kk >> 2) * PANEL) + 2 * (kk & 3);
                        const uint64_t bd = desc_mn_sw128(v_addr + kk * 16 * 128, PANEL);
                        mma_bf16(d, ad, bd, idesc_pv, kk > 0);
                    }
                    mma_commit(&o_full[i & 1]);
                    mma_commit(&v_empty[st]);
                }
            }
            mma_commit(done);
            const long long t0 = clock64();
            while (!mbar_try_wait(done, 0)) {
                if (clock64() - t0 > a.budget) {
                    fail(abort, a.err, 16);
                    break;
                }
            }
        }
    } else {
        // ---------------------------------------------------------------- softmax warps
        const int lg = warp & 3;
        const int half = (warp - 2) >> 2;                // key half of S, column half of O
        const int r = lg * 32 + lane;                    // row of the 128-row tile
        const int qpos = pos_first + min(r & (TOK - 1), nrows - 1);
        const uint32_t lane_half = tmem + (static_cast<uint32_t>(lg * 32) << 16) +
                                   static_cast<uint32_t>(half * 64);
        const float scale = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
        float acc[HD / 2];
#pragma unroll
        for (int i = 0; i < HD / 2; ++i) acc[i] = 0.0f;
        float m_run = -1e30f, l = 0.0f, m_acc = -1e30f, m_prev = -1e30f;
        bool ok = true;

        for (int t = 0; t < ntiles && !*abort; ++t) {
            if (!mbar_wait_warp(&s_full[t & 1], (t >> 1) & 1, a.budget, abort)) {
                fail(abort, a.err, 17);
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t srow = tmem + (static_cast<uint32_t>(lg * 32) << 16) +
                                  static_cast<uint32_t>((t & 1) * 128);
            const uint32_t sb = srow + static_cast<uint32_t>(half * 64);
            const int tile_key0 = t * KEYS;
            const int key0 = tile_key0 + half * 64;
            // Row max over all 128 keys of the tile (both halves read the whole row from TMEM, so
            // they agree on it without exchanging). Scores are scaled after the max (scale > 0).
            const bool full_tile = tile_key0 + KEYS - 1 <= qpos;  // no masked key in this tile
            float sv[64];
            tmem_ld64(sb, sv);
            // Max as 8 independent chains and a tree (short dependent latency).
            float mx8[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) mx8[j] = -1e30f;
            if (full_tile) {
#pragma unroll
                for (int k = 0; k < 64; ++k) mx8[k & 7] = fmaxf(mx8[k & 7], sv[k]);
            } else {
#pragma unroll
                for (int k = 0; k < 64; ++k) {
                    if (key0 + k <= qpos) mx8[k & 7] = fmaxf(mx8[k & 7], sv[k]);
                }
            }
            float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            const float other = exchange_row(red, mx_bar, t, half, r, mx, a.budget, abort);
            if (other != other) {
                fail(abort, a.err, 19);
                ok = false;
                break;
            }
            mx = fmaxf(mx, other);
            const float m_new = fmaxf(m_run, mx * scale);
            float sum = 0.0f;
            uint8_t* prow = sm + P_OFF + (t & 1) * P_BUF + half * PANEL + r * 128;
            const float2 sc2 = make_float2(scale, scale), nm2 = make_float2(-m_new, -m_new);
#pragma unroll
            for (int k = 0; k < 64; k += 2) {
                const float2 x = ffma2(make_float2(sv[k], sv[k + 1]), sc2, nm2);
                sv[k] = ex2(x.x);
                sv[k + 1] = ex2(x.y);
            }
            if (!full_tile) {
#pragma unroll
                for (int k = 0; k < 64; ++k) sv[k] = key0 + k <= qpos ? sv[k] : 0.0f;
            }
            float2 s4[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                            make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll
            for (int k = 0; k < 64; k += 2) s4[(k >> 1) & 3] = fadd2(s4[(k >> 1) & 3], make_float2(sv[k], sv[k + 1]));
            const float2 s2 = fadd2(fadd2(s4[0], s4[1]), fadd2(s4[2], s4[3]));
            sum = s2.x + s2.y;
            if (a.f16) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int chunk = q ^ (r & 7);
                    *reinterpret_cast<uint4*>(prow + chunk * 16) =
                        make_uint4(pack2_f16(sv[8 * q], sv[8 * q + 1]),
                                   pack2_f16(sv[8 * q + 2], sv[8 * q + 3]),
                                   pack2_f16(sv[8 * q + 4], sv[8 * q + 5]),
                                   pack2_f16(sv[8 * q + 6], sv[8 * q + 7]));
                }
            } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int chunk = q ^ (r & 7);
                    *reinterpret_cast<uint4*>(prow + chunk * 16) =
                        make_uint4(pack_bf16x2(sv[8 * q], sv[8 * q + 1]),
                                   pack_bf16x2(sv[8 * q + 2], sv[8 * q + 3]),
                                   pack_bf16x2(sv[8 * q + 4], sv[8 * q + 5]),
                                   pack_bf16x2(sv[8 * q + 6], sv[8 * q + 7]));
                }
            }
            tc_fence_before();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&s_empty[t & 1]);
                mbar_arrive(&p_full[t & 1]);
            }
            l = l * ex2(m_run - m_new) + sum;
            m_run = m_new;
            if (t >= 1 && !fold_o(acc, m_acc, t - 1, m_prev, lane_half, o_full, o_empty, lane,
                                   a.budget, abort)) {
                fail(abort, a.err, 18);
                ok = false;
                break;
            }
            m_prev = m_new;
        }
        if (ok && !*abort && ntiles > 0 &&
            !fold_o(acc, m_acc, ntiles - 1, m_prev, lane_half, o_full, o_empty, lane, a.budget,
                    abort)) {
            fail(abort, a.err, 18);
            ok = false;
        }
        if (ok && !*abort) {
            // Row sum = the two halves' partial sums (both relative to the same running max).
            // The exchange barriers were used once per tile; this is use number ntiles.
            const float l_other = exchange_row(red, mx_bar, ntiles, half, r, l, a.budget, abort);
            if (l_other != l_other) {
                fail(abort, a.err, 19);
            } else {
                const int token = tok0 + (r & (TOK - 1));
                if ((r & (TOK - 1)) < nrows) {
                    const float inv = 1.0f / (l + l_other);
                    const size_t off = static_cast<size_t>(token) * (2 * a.n_kv) * HD +
                                       (2 * g + (r >> 6)) * HD + half * 64;
                    uint4* dst = reinterpret_cast<uint4*>(a.out + off);
#pragma unroll
                    for (int i = 0; i < HD / 16; ++i) {
                        float y[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) y[k] = acc[8 * i + k] * inv;
                        if (a.f16) {
                            dst[i] = make_uint4(pack2_f16(y[0], y[1]), pack2_f16(y[2], y[3]),
                                                pack2_f16(y[4], y[5]), pack2_f16(y[6], y[7]));
                            continue;
                        }
                        const uint4 hi = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                                                    pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
                        dst[i] = hi;
                        if (a.out_lo) {
                            const uint32_t h4[4] = {hi.x, hi.y, hi.z, hi.w};
                            uint32_t l4[4];
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                l4[k] = pack_bf16x2(y[2 * k] - __uint_as_float(h4[k] << 16),
                                                    y[2 * k + 1] - __uint_as_float(h4[k] & 0xffff0000u));
                            }
                            reinterpret_cast<uint4*>(a.out_lo + off)[i] = make_uint4(l4[0], l4[1], l4[2], l4[3]);
                        }
                    }
                }
            }
        }
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

void launch_prefill_attention_tc(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                 const CUtensorMap& k4, const CUtensorMap& v4,
                                 const PrefillAttnTcArgs& a, cudaStream_t s) {
    if (a.rows <= 0) return;
    static bool configured[64] = {};
    int dev = 0;
    Q3_CUDA(cudaGetDevice(&dev));
    if (!configured[dev & 63]) {
        Q3_CUDA(cudaFuncSetAttribute(prefill_attn_tc_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        configured[dev & 63] = true;
    }
    const dim3 grid((a.work ? a.n_work : (a.rows + TOK - 1) / TOK) * a.n_kv);
    launch_dep(true, prefill_attn_tc_kernel, grid, dim3(NTHREADS), SMEM, s, q, k, v, k4, v4, a);
    Q3_CUDA(cudaGetLastError());
}

}  // namespace q3
