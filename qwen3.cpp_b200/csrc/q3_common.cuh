// Shared device helpers and host error plumbing of the B200 Qwen3 library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>
#include <utility>

#include "q3_b200.h"

namespace q3 {

// ------------------------------------------------------------------ host errors

// Exception types mirror the reference's (std::runtime_error / invalid_argument / out_of_range);
// the C ABI converts them to q3_status at the boundary.
struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct DeviceTimeout : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void cuda_check(cudaError_t e, const char* what, const char* file, int line) {
    if (e != cudaSuccess) {
        throw CudaError(std::string("CUDA error in ") + what + " (" + file + ":" +
                        std::to_string(line) + "): " + cudaGetErrorString(e));
    }
}
#define Q3_CUDA(x) ::q3::cuda_check((x), #x, __FILE__, __LINE__)

void set_last_error(const std::string& msg);

template <typename F>
q3_status guard(F&& fn) {
    try {
        fn();
        return Q3_OK;
    } catch (const std::out_of_range& e) {
        set_last_error(e.what());
        return Q3_ERR_OUT_OF_RANGE;
    } catch (const std::invalid_argument& e) {
        set_last_error(e.what());
        return Q3_ERR_INVALID_ARGUMENT;
    } catch (const DeviceTimeout& e) {
        set_last_error(e.what());
        return Q3_ERR_DEVICE_TIMEOUT;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return Q3_ERR_RUNTIME;
    }
}

// ------------------------------------------------------------------ dependent launches

// Programmatic dependent launch: a kernel launched by launch_dep(dependent = true) may start
// (prologue, shared memory and TMEM set-up) while the kernel before it in the stream finishes; its
// pdl_wait() blocks until that kernel has completed and its writes are visible, so every kernel
// launched this way calls it before its first global-memory access. pdl_trigger() lets the next
// kernel's blocks be scheduled once all blocks of this one have started. Both are no-ops for a
// kernel launched without the attribute. Measured: the prefill's long kernels gain (4.04 -> 3.68 ms
// for 2048 tokens); the graph-captured decode steps of many short kernels lose 4-10%, so they
// launch without it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
void launch_dep(bool dependent, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    Q3_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// ------------------------------------------------------------------ device helpers

__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) {
    return __uint_as_float(packed & 0xffff0000u);
}
__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
// Round to nearest even, as static_cast<std::bfloat16_t>(float) does on the host.
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

// fp16 operands of the prefill's tensor-core contractions and attention (an 11-bit significand
// against bf16's 8, at the same MMA rate). Two fp32 -> one packed f16x2 (a in the low half),
// rounded to nearest even and saturated to +-65504 rather than overflowing to infinity.
__device__ __forceinline__ uint32_t pack2_f16(float a, float b) {
    uint32_t r;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}
__device__ __forceinline__ float f16_lo(uint32_t packed) {
    float f;
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\tcvt.f32.f16 %0, l;\n\t}"
        : "=f"(f) : "r"(packed));
    return f;
}
__device__ __forceinline__ float f16_hi(uint32_t packed) {
    float f;
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\tcvt.f32.f16 %0, h;\n\t}"
        : "=f"(f) : "r"(packed));
    return f;
}
// Packed bf16 pair -> packed fp16 pair holding the same values (exact for magnitudes in
// [2^-17, 65504]: every bf16 value there is an fp16 value; smaller ones round to the fp16
// subnormal grid, larger ones saturate).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t packed) {
    return pack2_f16(bf16_lo(packed), bf16_hi(packed));
}

// Packed fp32 pairs (sm_100): d = a * b + c on two lanes at once.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long pa, pb, pc, pd;
    asm("mov.b64 %0, {%1, %2};" : "=l"(pa) : "f"(a.x), "f"(a.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(pb) : "f"(b.x), "f"(b.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(pc) : "f"(c.x), "f"(c.y));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(pd) : "l"(pa), "l"(pb), "l"(pc));
    float2 d;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(pd));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long pa, pb, pd;
    asm("mov.b64 %0, {%1, %2};" : "=l"(pa) : "f"(a.x), "f"(a.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(pb) : "f"(b.x), "f"(b.y));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(pd) : "l"(pa), "l"(pb));
    float2 d;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(pd));
    return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 8 bf16 weights (one 16-byte load) dotted with 8 fp32 activations.
__device__ __forceinline__ float dot8(const uint4 w, const float4 a, const float4 b, float acc) {
    acc = fmaf(bf16_lo(w.x), a.x, acc);
    acc = fmaf(bf16_hi(w.x), a.y, acc);
    acc = fmaf(bf16_lo(w.y), a.z, acc);
    acc = fmaf(bf16_hi(w.y), a.w, acc);
    acc = fmaf(bf16_lo(w.z), b.x, acc);
    acc = fmaf(bf16_hi(w.z), b.y, acc);
    acc = fmaf(bf16_lo(w.w), b.z, acc);
    acc = fmaf(bf16_hi(w.w), b.w, acc);
    return acc;
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once per token).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Per-step scalars of a decode step, kept in device memory so that a captured CUDA graph can be
// replayed for every step: the sink/ring position math of src/inference.cpp:605-613.
struct StepParams {
    int32_t token;
    int32_t pos;
    int32_t num_sink;
    int32_t kv_pos;
    int32_t kv_len;
    int32_t step;       // index of this step inside a device-driven decode loop
    int32_t n_forced;   // teacher-forced loop: tokens given for steps [0, n_forced)
    int32_t pad;
};

__host__ __device__ inline void step_positions(int pos, int ctx, int* num_sink, int* kv_pos,
                                               int* kv_len) {
    constexpr int kAttentionSinks = 4;
    const int ns = pos >= ctx ? (kAttentionSinks < ctx - 1 ? kAttentionSinks : ctx - 1) : 0;
    *num_sink = ns;
    *kv_pos = pos < ctx ? pos : ns + (pos - ns) % (ctx - ns);
    *kv_len = pos + 1 < ctx ? pos + 1 : ctx;
}

constexpr int kPageTokens = 16;  // KV-cache page size (tokens)

}  // namespace q3
