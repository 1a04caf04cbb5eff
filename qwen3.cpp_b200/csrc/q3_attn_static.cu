// q3_attn_noalloc: the split-K decode attention of q3_attn with its scratch in a file-scope
// device array instead of a caller-provided workspace.
//
// Some callers cannot allocate device memory when they call in: runtimes that own and pre-plan
// every byte of device memory (a serving process with a fixed memory budget, a host plugin that
// forbids allocation), and callers that must not trigger the implicit device-wide
// synchronisation cudaMalloc/cudaFree may cause. For them this entry point takes no workspace and
// allocates nothing: the split partials live in kAttnStaticScratchBytes of static device memory,
// which every GPU that loads this library holds until the process exits.
//
// Device address of the array: in host code the array's name is a host-side stand-in, not a device
// address, so the first call on each device (with that device current) looks the address up with
// cudaGetSymbolAddress and caches it; make that first call before any stream capture. Every call
// on a device shares the one array and overwrites it: calls that can overlap on the GPU (different
// streams, or host threads) race on it and must be ordered by the caller. No part of the array has
// to start at zero: every split writes all of its partial results before the combine reads them.
#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "q3_common.cuh"
#include "q3_kernels.cuh"

namespace {

// Largest workspace q3_attn ever needs: 64 splits x head_dim 256 fp32 partial outputs, 256 bytes of
// alignment, 64 (max, sum) pairs.
constexpr size_t kAttnStaticScratchBytes = 64 * 256 * sizeof(float) + 256 + 64 * sizeof(float2);

static __device__ __align__(256) unsigned char g_attn_scratch[kAttnStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_attn_scratch on the current device (looked up once per device).
void* static_scratch() {
    int dev = 0;
    Q3_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("device index out of range");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || p == nullptr) {
            throw q3::CudaError(std::string("cudaGetSymbolAddress of the attention scratch failed: ") +
                                cudaGetErrorString(e));
        }
        g_scratch_ptr[dev] = p;
    }
    return g_scratch_ptr[dev];
}

}  // namespace

extern "C" {

size_t q3_attn_noalloc_max_scratch(void) { return kAttnStaticScratchBytes; }

q3_status q3_attn_noalloc(float* out, const float* q, const uint16_t* k, const uint16_t* v,
                          int head_dim, int n_kv_heads, int kv_len, void* stream) {
    return q3::guard([&] {
        if (!out || !q || !k || !v || head_dim <= 0 || head_dim > 256 || n_kv_heads <= 0 ||
            kv_len <= 0) {
            throw std::invalid_argument("invalid FastAttn arguments");
        }
        const size_t need = q3_attn_workspace_size(head_dim, kv_len);
        if (need > kAttnStaticScratchBytes) {
            throw std::invalid_argument("attention needs " + std::to_string(need) +
                                        " bytes of scratch, above the static maximum of " +
                                        std::to_string(kAttnStaticScratchBytes));
        }
        unsigned char* ws = static_cast<unsigned char*>(static_scratch());
        const int S = q3::attn_splits_for(kv_len);
        q3::AttnArgs a{};
        a.q = q;
        a.k = k;
        a.v = v;
        a.page_table = nullptr;
        a.sp = nullptr;
        a.kv_len_const = kv_len;
        a.n_heads = 1;
        a.n_kv = 1;
        a.hd = head_dim;
        a.row_stride = n_kv_heads * head_dim;
        a.n_splits = S;
        a.part_o = reinterpret_cast<float*>(ws);
        const size_t o_bytes = (static_cast<size_t>(S) * head_dim * 4 + 255) & ~size_t(255);
        a.part_ml = reinterpret_cast<float2*>(ws + o_bytes);
        a.out = out;
        q3::launch_attention(a, static_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
