// Prefill contractions on tcgen05 tensor cores (sm_100a).
//
// Persistent, warp-specialised kernel, one CTA per SM (192 threads):
//   warp 0      TMA producer: for every (tile, k-block) of this CTA, waits for a free stage and
//               loads the 128 x 64 A box and the BN x 64 B box (128-byte swizzle) into it.
//   warp 1      MMA issuer (one thread): per k-block four tcgen05.mma (M=128, N=BN, K=16) into
//               one of two TMEM accumulators; tcgen05.commit frees the stage when the MMAs that
//               read it are done, and signals the epilogue after the tile's last k-block.
//   warps 2-5   epilogue: warp w reads TMEM lanes 32*(w%4).. (one output row per thread), 32
//               fp32 columns per tcgen05.ld, applies the fused op, writes its 32-row block into
//               a double-buffered 128-byte-swizzled shared-memory tile and one lane hands it to
//               a TMA store (or a TMA reduce-add for the residual stream), so the global writes
//               run asynchronously as full lines. Two TMEM accumulators let the epilogue of one
//               tile overlap the MMAs of the next.
// Every mbarrier wait is bounded; a wait that gives up sets args.err and the CTA drains its
// outstanding TMA loads and MMAs before freeing TMEM and returning.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "q3_b200.h"
#include "q3_common.cuh"
#include "q3_gemm.cuh"
#include "q3_sm100.cuh"

namespace q3 {

namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int NTHREADS = 192;

// SPLIT: the A operand comes as two bf16 parts (hi and lo, a = hi + lo) that both multiply the same
// B tile into the accumulator - fp32-like activations at twice the MMA work, for the
// weight-streaming small-M contractions of batched decode.
template <int BN, bool SPLIT = false>
struct GemmCfg {
    static constexpr int A_PART = BM * BK * 2;
    static constexpr int A_BYTES = (SPLIT ? 2 : 1) * A_PART;
    static constexpr int STAGES = (196608 / (A_BYTES + BN * BK * 2)) > 6 ? 6 : (196608 / (A_BYTES + BN * BK * 2));
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int STG_BYTES = 4 * 2 * 4096;  // per epilogue warp: 2 x (32 rows x 128 B)
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STG_BYTES + 1024 + 256;
};

// TMA store / reduce-add of a shared-memory box to global memory (asynchronous, bulk group).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x,
                                                  int y) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], "
        "[%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // RNE, like static_cast<bfloat16_t>
    return *reinterpret_cast<const uint32_t*>(&h);
}


__device__ __forceinline__ void fail(volatile int* abort, unsigned* err, unsigned code) {
    *abort = 1;
    if (err) atomicCAS(err, 0u, code);
}

template <int BN, int EPI, bool SPLIT = false>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                const __grid_constant__ CUtensorMap tb2, const __grid_constant__ CUtensorMap tout,
                const __grid_constant__ CUtensorMap ta_lo, const GemmArgs args) {
    using C = GemmCfg<BN, SPLIT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* stg_all = smem + C::STAGES * C::STAGE_BYTES;  // epilogue staging, 1024-aligned
    uint64_t* full = reinterpret_cast<uint64_t*>(stg_all + C::STG_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (args.M + BM - 1) / BM;
    const int num_n = args.N / BN;
    // Residual-add contractions may split K: every slice reduce-adds its partial sum.
    const int ksplit = EPI == kEpiAddF32 ? args.ksplit : 1;
    const int tiles = num_m * num_n * ksplit;
    const int kblocks = args.K / BK / ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);
        }
        mbar_init(done, 1);
        *abort = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        tma_prefetch_map(&ta);
        tma_prefetch_map(&tb);
        if (EPI == kEpiSwiGLU) tma_prefetch_map(&tb2);
        if (SPLIT) tma_prefetch_map(&ta_lo);
        tma_prefetch_map(&tout);
        tmem_alloc(tmem_slot, C::TMEM_COLS);
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Set-up above touches no global data; the previous kernel's outputs are read below.
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------------------- producer
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_parity = 0;
            for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
                const int tmn = t % (num_m * num_n), ks = t / (num_m * num_n);
                const int tm = tmn % num_m, tn = tmn / num_m;
                for (int kbi = 0; kbi < kblocks; ++kbi) {
                    const int kb = ks * kblocks + kbi;
                    if (!mbar_wait(&empty[stage], phase ^ 1, args.budget, abort)) {
                        fail(abort, args.err, 1);
                        break;
                    }
                    uint8_t* sa = smem + stage * C::STAGE_BYTES;
                    uint8_t* sb = sa + C::A_BYTES;
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(sa, &ta, kb * BK, tm * BM, &full[stage]);
                    if (SPLIT) tma_load_2d(sa + C::A_PART, &ta_lo, kb * BK, tm * BM, &full[stage]);
                    if (EPI == kEpiSwiGLU) {
                        tma_load_2d(sb, &tb, kb * BK, tn * (BN / 2), &full[stage]);
                        tma_load_2d(sb + C::B_BYTES / 2, &tb2, kb * BK, tn * (BN / 2), &full[stage]);
                    } else {
                        tma_load_2d(sb, &tb, kb * BK, tn * BN, &full[stage]);
                    }
                    issued_mask |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Drain: every load issued into shared memory has landed before the CTA exits.
            for (int s = 0; s < C::STAGES; ++s) {
                if (issued_mask & (1u << s)) {
                    const long long t0 = clock64();
                    while (!mbar_try_wait(&full[s], (issued_parity >> s) & 1)) {
                        if (clock64() - t0 > args.budget) {
                            fail(abort, args.err, 2);
                            break;
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------------------- MMA issuer
            const uint32_t idesc = args.f16 ? idesc_f16_f32(BM, BN) : idesc_bf16_f32(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok && !*abort; t += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.budget, abort)) {
                    fail(abort, args.err, 3);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
                for (int kbi = 0; kbi < kblocks; ++kbi) {
                    if (!mbar_wait(&full[stage], phase, args.budget, abort)) {
                        fail(abort, args.err, 4);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
                    const uint64_t adesc = desc_k_sw128(sa);
                    const uint64_t bdesc = desc_k_sw128(sa + C::A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        mma_bf16(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kbi | k) != 0);
                        if (SPLIT) {
                            mma_bf16(d, adesc + (C::A_PART >> 4) + 2 * k, bdesc + 2 * k, idesc, 1);
                        }
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                mma_commit(&tfull[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            // Drain: all MMAs issued by this thread complete before TMEM is freed.
            mma_commit(done);
            const long long t0 = clock64();
            while (!mbar_try_wait(done, 0)) {
                if (clock64() - t0 > args.budget) {
                    fail(abort, args.err, 5);
                    break;
                }
            }
        }
    } else {
        // -------------------------------------------------------------------- epilogue
        const int lg = warp & 3;
        uint8_t* stg = stg_all + lg * 8192;
        int nbuf = 0;  // staging buffers used so far (alternating)
        // Row `lane` of the warp's 32-row box as 128 bytes, 16-byte chunks XOR-swizzled by the
        // row (the TMA 128-byte swizzle pattern: 8 rows hit 8 different bank groups).
        auto stage_store = [&](const uint4 (&row)[8], int x, int y) {
            uint8_t* buf = stg + (nbuf & 1) * 4096;
            if (lane == 0) bulk_wait_read<1>();  // the store that used this buffer has read it
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                *reinterpret_cast<uint4*>(buf + lane * 128 + ((i ^ (lane & 7)) << 4)) = row[i];
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (EPI == kEpiAddF32) {
                    tma_reduce_add_2d(&tout, buf, x, y);
                } else {
                    tma_store_2d(&tout, buf, x, y);
                }
                bulk_commit();
            }
            ++nbuf;
        };
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
            const int tmn = t % (num_m * num_n);
            const int tm = tmn % num_m, tn = tmn / num_m;
            if (!mbar_wait_warp(&tfull[acc], acc_phase, args.budget, abort)) {
                fail(abort, args.err, 6);
                break;
            }
            tc_fence_after();
            const uint32_t tb_addr = tmem + (static_cast<uint32_t>(lg * 32) << 16) +
                                     static_cast<uint32_t>(acc * BN);
            const int y = tm * BM + lg * 32;  // rows past M are clipped by the TMA store
            if (EPI == kEpiSwiGLU) {
                // 64 hidden columns per box: h = silu(w1 . x) * (w3 . x) as bf16.
#pragma unroll 1
                for (int c = 0; c < BN / 2; c += 64) {
                    uint4 row[8];
#pragma unroll
                    for (int hlf = 0; hlf < 2; ++hlf) {
                        float g[32], u[32];
                        tmem_ld32(tb_addr + c + hlf * 32, g);
                        tmem_ld32(tb_addr + BN / 2 + c + hlf * 32, u);
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            // silu(g) * u (src/inference.cpp:948-950, :1009-1011) with the fast
                            // exponential and division: the result is rounded to bf16.
                            g[i] = __fdividef(g[i], 1.0f + __expf(-g[i])) * u[i];
                        }
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            row[hlf * 4 + i] = args.f16
                                ? make_uint4(pack2_f16(g[8 * i], g[8 * i + 1]), pack2_f16(g[8 * i + 2], g[8 * i + 3]),
                                             pack2_f16(g[8 * i + 4], g[8 * i + 5]), pack2_f16(g[8 * i + 6], g[8 * i + 7]))
                                : make_uint4(pack_bf16(g[8 * i], g[8 * i + 1]), pack_bf16(g[8 * i + 2], g[8 * i + 3]),
                                             pack_bf16(g[8 * i + 4], g[8 * i + 5]), pack_bf16(g[8 * i + 6], g[8 * i + 7]));
                        }
                    }
                    stage_store(row, tn * (BN / 2) + c, y);
                }
            } else if (EPI == kEpiQkvRope) {
                // Two 128-column heads per tile; this thread's row is token y + lane.
                const QkvEpilogue& e = args.qkv;
                const int token = y + lane;
                const bool live = token < args.M;
                const int pos = e.tok_pos ? (live ? __ldg(e.tok_pos + token) : 0) : e.pos0 + token;
                const int nq = e.n_heads, nk = e.n_kv;
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    const int head = tn * 2 + hh;
                    const uint32_t hcol = tb_addr + hh * 128;
                    const bool qk = head < nq + nk;
                    // Pass 1 (q, k): the head's sum of squares.
                    float inv = 1.0f;
                    if (qk) {
                        float ss = 0.0f;
#pragma unroll 1
                        for (int c = 0; c < 128; c += 32) {
                            float t32[32];
                            tmem_ld32(hcol + c, t32);
#pragma unroll
                            for (int i = 0; i < 32; ++i) ss = fmaf(t32[i], t32[i], ss);
                        }
                        inv = 1.0f / sqrtf(ss / 128.0f + e.eps);
                    }
                    uint16_t* dst = nullptr;
                    uint16_t* dst16 = nullptr;  // fp16 copy of a K/V row
                    const bool isq = head < nq;
                    if (live) {
                        if (isq) {
                            dst = e.q_out + static_cast<size_t>(token) * nq * 128 + head * 128;
                        } else {
                            const int g = qk ? head - nq : head - nq - nk;
                            const int crow = e.tok_row ? __ldg(e.tok_row + token)
                                                       : __ldg(e.page_table + pos / 16) * 16 + pos % 16;
                            const size_t page = static_cast<size_t>(crow / 16);
                            const size_t off = ((page * nk + g) * 16 + crow % 16) * 128;
                            dst = (qk ? e.k_cache : e.v_cache) + off;
                            uint16_t* st = qk ? e.k_stage : e.v_stage;
                            if (st) dst16 = st + off;
                        }
                    }
                    const uint16_t* w = head < nq ? e.q_norm : e.k_norm;
                    const float4* cs = reinterpret_cast<const float4*>(
                        e.rope + static_cast<size_t>(live ? pos : e.pos0) * 64);
                    // Pass 2: columns (c .. c+31) and their RoPE partners (c+64 ..), normalised
                    // (:800-807), rotated (:809-810: (a, b) -> (a cos - b sin, b cos + a sin)), bf16.
#pragma unroll 1
                    for (int c = 0; c < 64; c += 32) {
                        float a[32], b[32];
                        tmem_ld32(hcol + c, a);
                        tmem_ld32(hcol + 64 + c, b);
                        if (qk) {
#pragma unroll
                            for (int i = 0; i < 32; i += 8) {
                                const uint4 wa = __ldg(reinterpret_cast<const uint4*>(w + c + i));
                                const uint4 wb = __ldg(reinterpret_cast<const uint4*>(w + 64 + c + i));
                                const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
                                const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    a[i + 2 * j] = (a[i + 2 * j] * inv) * __uint_as_float(wav[j] << 16);
                                    a[i + 2 * j + 1] = (a[i + 2 * j + 1] * inv) * __uint_as_float(wav[j] & 0xffff0000u);
                                    b[i + 2 * j] = (b[i + 2 * j] * inv) * __uint_as_float(wbv[j] << 16);
                                    b[i + 2 * j + 1] = (b[i + 2 * j + 1] * inv) * __uint_as_float(wbv[j] & 0xffff0000u);
                                }
                            }
#pragma unroll
                            for (int i = 0; i < 32; i += 2) {
                                const float4 c2 = __ldg(cs + (c + i) / 2);  // (cos, sin) of c+i, c+i+1
                                const float a0 = a[i], b0 = b[i], a1 = a[i + 1], b1 = b[i + 1];
                                a[i] = a0 * c2.x - b0 * c2.y;
                                b[i] = b0 * c2.x + a0 * c2.y;
                                a[i + 1] = a1 * c2.z - b1 * c2.w;
                                b[i + 1] = b1 * c2.z + a1 * c2.w;
                            }
                        }
                        if (live) {
                            const bool f16q = isq && e.q_f16;
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                uint4 va, vb;
                                if (f16q) {
                                    va = make_uint4(pack2_f16(a[8 * i], a[8 * i + 1]), pack2_f16(a[8 * i + 2], a[8 * i + 3]),
                                                    pack2_f16(a[8 * i + 4], a[8 * i + 5]), pack2_f16(a[8 * i + 6], a[8 * i + 7]));
                                    vb = make_uint4(pack2_f16(b[8 * i], b[8 * i + 1]), pack2_f16(b[8 * i + 2], b[8 * i + 3]),
                                                    pack2_f16(b[8 * i + 4], b[8 * i + 5]), pack2_f16(b[8 * i + 6], b[8 * i + 7]));
                                } else {
                                    va = make_uint4(pack_bf16(a[8 * i], a[8 * i + 1]), pack_bf16(a[8 * i + 2], a[8 * i + 3]),
                                                    pack_bf16(a[8 * i + 4], a[8 * i + 5]), pack_bf16(a[8 * i + 6], a[8 * i + 7]));
                                    vb = make_uint4(pack_bf16(b[8 * i], b[8 * i + 1]), pack_bf16(b[8 * i + 2], b[8 * i + 3]),
                                                    pack_bf16(b[8 * i + 4], b[8 * i + 5]), pack_bf16(b[8 * i + 6], b[8 * i + 7]));
                                }
                                reinterpret_cast<uint4*>(dst + c)[i] = va;
                                reinterpret_cast<uint4*>(dst + 64 + c)[i] = vb;
                                if (dst16) {
                                    // The cache's bf16 values, as fp16 (exact in range).
                                    reinterpret_cast<uint4*>(dst16 + c)[i] = make_uint4(
                                        bf16x2_to_f16x2(va.x), bf16x2_to_f16x2(va.y),
                                        bf16x2_to_f16x2(va.z), bf16x2_to_f16x2(va.w));
                                    reinterpret_cast<uint4*>(dst16 + 64 + c)[i] = make_uint4(
                                        bf16x2_to_f16x2(vb.x), bf16x2_to_f16x2(vb.y),
                                        bf16x2_to_f16x2(vb.z), bf16x2_to_f16x2(vb.w));
                                }
                            }
                        }
                    }
                }
            } else if (EPI == kEpiStoreBF16) {
#pragma unroll 1
                for (int c = 0; c < BN; c += 64) {
                    uint4 row[8];
#pragma unroll
                    for (int hlf = 0; hlf < 2; ++hlf) {
                        float v[32];
                        tmem_ld32(tb_addr + c + hlf * 32, v);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            row[hlf * 4 + i] = args.f16
                                ? make_uint4(pack2_f16(v[8 * i], v[8 * i + 1]), pack2_f16(v[8 * i + 2], v[8 * i + 3]),
                                             pack2_f16(v[8 * i + 4], v[8 * i + 5]), pack2_f16(v[8 * i + 6], v[8 * i + 7]))
                                : make_uint4(pack_bf16(v[8 * i], v[8 * i + 1]), pack_bf16(v[8 * i + 2], v[8 * i + 3]),
                                             pack_bf16(v[8 * i + 4], v[8 * i + 5]), pack_bf16(v[8 * i + 6], v[8 * i + 7]));
                        }
                    }
                    stage_store(row, tn * BN + c, y);
                }
            } else {
                // fp32: 32 columns per box (stored, or added into the residual stream in L2).
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    float v[32];
                    tmem_ld32(tb_addr + c, v);
                    uint4 row[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        row[i] = make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]),
                                            __float_as_uint(v[4 * i + 2]), __float_as_uint(v[4 * i + 3]));
                    }
                    stage_store(row, tn * BN + c, y);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        // Every store has completed (global writes done) before the CTA exits.
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    });
    if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
    return fn;
}

// Large dynamic shared memory is opted into once per kernel instance and device.
template <int BN, int EPI, bool SPLIT = false>
cudaError_t configure_t() {
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (!configured[dev & 63]) {
        e = cudaFuncSetAttribute(gemm_kernel<BN, EPI, SPLIT>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 GemmCfg<BN, SPLIT>::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    return cudaSuccess;
}

template <int BN, int EPI, bool SPLIT = false>
cudaError_t launch_t(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& b2,
                     const CUtensorMap& out, const GemmArgs& args, int num_sms,
                     cudaStream_t stream, const CUtensorMap& a_lo) {
    using C = GemmCfg<BN, SPLIT>;
    auto kern = gemm_kernel<BN, EPI, SPLIT>;
    cudaError_t e = configure_t<BN, EPI, SPLIT>();
    if (e != cudaSuccess) return e;
    GemmArgs g = args;
    const int mn_tiles = ((args.M + BM - 1) / BM) * (args.N / BN);
    g.ksplit = 1;
    if (EPI == kEpiAddF32) {
        // Split K while the tiles fill less than half the SMs (slices reduce-add in L2).
        const int kb = args.K / BK;
        while (g.ksplit < args.max_ksplit && mn_tiles * g.ksplit * 2 <= num_sms &&
               kb % (g.ksplit * 2) == 0 && kb / (g.ksplit * 2) >= args.min_slice_kblocks) {
            g.ksplit *= 2;
        }
    }
    const int tiles = mn_tiles * g.ksplit;
    const int grid = tiles < num_sms ? tiles : num_sms;
    if (grid <= 0) return cudaSuccess;
    launch_dep(g.dependent, kern, dim3(grid), dim3(NTHREADS), C::SMEM_BYTES, stream, a, b, b2, out, a_lo, g);
    return cudaGetLastError();
}

}  // namespace

void make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                    uint32_t box_rows) {
    make_tmap_bf16_strided(map, base, rows, cols, cols, box_rows);
}

void make_tmap_bf16_strided(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                            uint64_t row_stride, uint32_t box_rows) {
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols % 8 != 0 || row_stride % 8 != 0 ||
        row_stride < cols || rows == 0 || box_rows == 0 || box_rows > 256) {
        throw std::invalid_argument("tensor map: misaligned base or unsupported shape");
    }
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_stride * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
    }
}

void make_tmap_out(CUtensorMap* map, void* base, uint64_t rows, uint64_t cols, bool bf16) {
    const uint64_t esz = bf16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (cols * esz) % 128 != 0 || rows == 0) {
        throw std::invalid_argument("tensor map: misaligned output or width not a multiple of 128 B");
    }
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * esz};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esz), 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(
        map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims,
        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
    }
}

void make_tmap_kv_pages(CUtensorMap* map, const void* base, uint64_t n_kv, uint64_t pages) {
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || n_kv == 0 || pages < 8) {
        throw std::invalid_argument("tensor map: misaligned KV cache or too few pages");
    }
    const cuuint64_t dims[4] = {128, 16, n_kv, pages};
    const cuuint64_t strides[3] = {256, 16 * 256, n_kv * 16 * 256};
    const cuuint32_t box[4] = {64, 16, 1, 8};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base),
                                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
    }
}

int gemm_tile_n(int epi, int N) {
    if (epi == kEpiSwiGLU || epi == kEpiQkvRope) return 256;
    return N % 256 == 0 ? 256 : 128;
}

void prepare_gemm_kernels() {
    Q3_CUDA((configure_t<256, kEpiStoreF32>()));
    Q3_CUDA((configure_t<128, kEpiStoreF32>()));
    Q3_CUDA((configure_t<256, kEpiAddF32>()));
    Q3_CUDA((configure_t<128, kEpiAddF32>()));
    Q3_CUDA((configure_t<256, kEpiStoreBF16>()));
    Q3_CUDA((configure_t<128, kEpiStoreBF16>()));
    Q3_CUDA((configure_t<256, kEpiSwiGLU>()));
    Q3_CUDA((configure_t<256, kEpiQkvRope>()));
    Q3_CUDA((configure_t<128, kEpiStoreF32, true>()));
    Q3_CUDA((configure_t<128, kEpiAddF32, true>()));
    Q3_CUDA((configure_t<256, kEpiStoreF32, true>()));
    Q3_CUDA((configure_t<256, kEpiAddF32, true>()));
    Q3_CUDA((configure_t<256, kEpiQkvRope, true>()));
}

cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap* b2,
                        const CUtensorMap& out, const GemmArgs& args, int epi, int num_sms,
                        cudaStream_t stream, const CUtensorMap* a_lo) {
    if (args.K % BK != 0 || args.K <= 0 || args.M <= 0) return cudaErrorInvalidValue;
    const int bn = args.bn ? args.bn : gemm_tile_n(epi, args.N);
    if ((bn != 128 && bn != 256) || args.N % bn != 0) return cudaErrorInvalidValue;
    if (epi == kEpiSwiGLU && (!b2 || bn != 256)) return cudaErrorInvalidValue;
    if (epi == kEpiQkvRope && (bn != 256 || !args.qkv.q_out || !args.qkv.k_cache ||
                               !args.qkv.v_cache || !args.qkv.rope ||
                               (!args.qkv.page_table && !args.qkv.tok_row) ||
                               (!args.qkv.tok_pos != !args.qkv.tok_row))) {
        return cudaErrorInvalidValue;
    }
    const CUtensorMap& bb = b2 ? *b2 : b;
    if (a_lo) {
        if (epi == kEpiStoreF32) {
            return bn == 256 ? launch_t<256, kEpiStoreF32, true>(a, b, bb, out, args, num_sms, stream, *a_lo)
                             : launch_t<128, kEpiStoreF32, true>(a, b, bb, out, args, num_sms, stream, *a_lo);
        }
        if (epi == kEpiAddF32) {
            return bn == 256 ? launch_t<256, kEpiAddF32, true>(a, b, bb, out, args, num_sms, stream, *a_lo)
                             : launch_t<128, kEpiAddF32, true>(a, b, bb, out, args, num_sms, stream, *a_lo);
        }
        if (epi == kEpiQkvRope) {
            return launch_t<256, kEpiQkvRope, true>(a, b, bb, out, args, num_sms, stream, *a_lo);
        }
        return cudaErrorInvalidValue;
    }
    switch (epi) {
        case kEpiStoreF32:
            return bn == 256 ? launch_t<256, kEpiStoreF32>(a, b, bb, out, args, num_sms, stream, a)
                             : launch_t<128, kEpiStoreF32>(a, b, bb, out, args, num_sms, stream, a);
        case kEpiAddF32:
            return bn == 256 ? launch_t<256, kEpiAddF32>(a, b, bb, out, args, num_sms, stream, a)
                             : launch_t<128, kEpiAddF32>(a, b, bb, out, args, num_sms, stream, a);
        case kEpiStoreBF16:
            return bn == 256 ? launch_t<256, kEpiStoreBF16>(a, b, bb, out, args, num_sms, stream, a)
                             : launch_t<128, kEpiStoreBF16>(a, b, bb, out, args, num_sms, stream, a);
        case kEpiSwiGLU:
            return launch_t<256, kEpiSwiGLU>(a, b, bb, out, args, num_sms, stream, a);
        case kEpiQkvRope:
            return launch_t<256, kEpiQkvRope>(a, b, bb, out, args, num_sms, stream, a);
    }
    return cudaErrorInvalidValue;
}

}  // namespace q3

// ------------------------------------------------------------------ C ABI

namespace {
q3_status gemm_entry(void* out, const uint16_t* a, const uint16_t* w, const uint16_t* w3, int M,
                     int N, int K, int epilogue, void* stream, bool f16);
}

extern "C" q3_status q3_gemm_bf16(void* out, const uint16_t* a, const uint16_t* w,
                                  const uint16_t* w3, int M, int N, int K, int epilogue,
                                  void* stream) {
    return gemm_entry(out, a, w, w3, M, N, K, epilogue, stream, false);
}

extern "C" q3_status q3_gemm_f16(void* out, const uint16_t* a, const uint16_t* w,
                                 const uint16_t* w3, int M, int N, int K, int epilogue,
                                 void* stream) {
    return gemm_entry(out, a, w, w3, M, N, K, epilogue, stream, true);
}

namespace {
q3_status gemm_entry(void* out, const uint16_t* a, const uint16_t* w, const uint16_t* w3, int M,
                     int N, int K, int epilogue, void* stream, bool f16) {
    using namespace q3;
    return guard([&] {
        if (!out || !a || !w) throw std::invalid_argument("null argument");
        if (M <= 0 || N <= 0 || K <= 0 || K % 64 != 0 || N % 128 != 0) {
            throw std::invalid_argument("gemm: M, N > 0, K a multiple of 64, N of 128");
        }
        if (epilogue < Q3_GEMM_STORE_F32 || epilogue > Q3_GEMM_STORE_BF16) {
            throw std::invalid_argument("gemm: unknown epilogue");
        }
        const bool swiglu = epilogue == Q3_GEMM_SWIGLU;
        if (swiglu && !w3) throw std::invalid_argument("gemm: SwiGLU needs w3");
        const int tile_space = swiglu ? 2 * N : N;
        const int bn = gemm_tile_n(epilogue, tile_space);
        if (tile_space % bn != 0) throw std::invalid_argument("gemm: N does not tile");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        int dev = 0, sms = 0;
        Q3_CUDA(cudaGetDevice(&dev));
        Q3_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        CUtensorMap ma, mb, mb3;
        make_tmap_bf16(&ma, a, M, K, 128);
        make_tmap_bf16(&mb, w, N, K, swiglu ? 128 : bn);
        if (swiglu) make_tmap_bf16(&mb3, w3, N, K, 128);
        CUtensorMap mo;
        make_tmap_out(&mo, out, M, N, swiglu || epilogue == Q3_GEMM_STORE_BF16);
        unsigned* err = nullptr;
        Q3_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&err), sizeof(unsigned), s));
        Q3_CUDA(cudaMemsetAsync(err, 0, sizeof(unsigned), s));
        GemmArgs g;
        g.M = M;
        g.N = tile_space;
        g.K = K;
        g.err = err;
        g.f16 = f16 ? 1 : 0;
        const cudaError_t le = launch_gemm(ma, mb, swiglu ? &mb3 : nullptr, mo, g, epilogue, sms, s);
        unsigned herr = 0;
        const cudaError_t ce = cudaMemcpyAsync(&herr, err, sizeof(unsigned),
                                               cudaMemcpyDeviceToHost, s);
        const cudaError_t se = cudaStreamSynchronize(s);
        cudaFreeAsync(err, s);
        Q3_CUDA(le);
        Q3_CUDA(ce);
        Q3_CUDA(se);
        if (herr) throw DeviceTimeout("gemm: a pipeline wait gave up (code " + std::to_string(herr) + ")");
    });
}
}  // namespace
