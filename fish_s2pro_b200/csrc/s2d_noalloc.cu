// s2d_noalloc.cu -- GQA decode attention that allocates no device memory.
//
// Some callers cannot call cudaMalloc: a real-time audio thread must not
// block in the CUDA allocator (cudaMalloc takes a process-wide lock and may
// synchronize the device), and a host that hands this library a fixed memory
// budget owns every device allocation itself.  For them this file provides a
// variant of s2d_op_gqa_decode_attention whose inputs and outputs are the
// caller's device buffers and whose split-K scratch (per-split softmax
// partials and arrival counters) lives in a file-scope device array below.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>
#include <mutex>

#include "../../include/s2d.h"
#include "s2d_kernels.cuh"

namespace {

// Scratch of the allocation-free attention.  Every GPU that loads this
// library holds these 512 KiB + 256 B until the process exits.  All calls
// share them: two calls that overlap on the GPU (from several host threads or
// streams) race on this memory.
constexpr int kNoAllocPartFloats = 1 << 17;  // 512 KiB of f32 partials
constexpr int kNoAllocCounters = 64;         // one arrival counter per kv head
static __device__ __align__(256) float g_noalloc_part[kNoAllocPartFloats];
static __device__ __align__(256) int32_t g_noalloc_counters[kNoAllocCounters];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
float *g_part_ptr[kMaxDevices] = {};
int32_t *g_counter_ptr[kMaxDevices] = {};

int32_t fail(char *err, size_t cap, int32_t code, const char *msg) {
    if (err && cap) snprintf(err, cap, "%s", msg);
    return code;
}

}  // namespace

extern "C" int32_t s2d_op_gqa_decode_attention_noalloc(
    const float *query, const float *keys, const float *values, int32_t H, int32_t Hkv, int32_t hd,
    int32_t T, float scale, float *out, void *stream, char *err, size_t err_cap) {
    if (!query || !keys || !values || !out || Hkv <= 0 || H % Hkv || hd <= 0 || T <= 0)
        return fail(err, err_cap, S2D_EINVAL, "invalid GQA split or attention dims");
    if (hd % 64 || hd > 256 || H / Hkv > 16)
        return fail(err, err_cap, S2D_EINVAL, "unsupported head_dim or group size");
    // The kernel reads each lane's head_dim/32 key and value elements as one
    // float2 (head_dim 64) or float4s, and query and out as single floats.
    const uintptr_t kv_align = hd == 64 ? 8 : 16;
    if ((uintptr_t)keys % kv_align || (uintptr_t)values % kv_align || (uintptr_t)query % 4 ||
        (uintptr_t)out % 4)
        return fail(err, err_cap, S2D_EINVAL,
                    "misaligned buffer: keys and values must be 16-byte aligned (8 at head_dim 64), "
                    "query and out 4-byte aligned");
    // the same split count as s2d_op_gqa_decode_attention, so both give the same result
    const int S = std::max(1, std::min(16, T / 8));
    if ((int64_t)H * S * (hd + 2) > kNoAllocPartFloats || Hkv > kNoAllocCounters) {
        char msg[256];
        snprintf(msg, sizeof msg,
                 "attention too large for the fixed scratch: head_count*splits*(head_dim+2) = %lld "
                 "floats (limit %d) and head_count_kv = %d (limit %d)",
                 (long long)H * S * (hd + 2), kNoAllocPartFloats, Hkv, kNoAllocCounters);
        return fail(err, err_cap, S2D_EINVAL, msg);
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(err, err_cap, S2D_ECUDA, "cudaGetDevice failed or device ordinal too large");
    float *part = nullptr;
    int32_t *counters = nullptr;
    {
        // Once per device, with that device current: the host-side name of a
        // __device__ array is not a device address, so look the address up.
        // The address belongs to the device's primary context; a
        // cudaDeviceReset ends that context and with it the cached address.
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (!g_part_ptr[dev]) {
            void *p = nullptr, *c = nullptr;
            if ((e = cudaGetSymbolAddress(&p, g_noalloc_part)) != cudaSuccess ||
                (e = cudaGetSymbolAddress(&c, g_noalloc_counters)) != cudaSuccess) {
                char msg[256];
                snprintf(msg, sizeof msg, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
                return fail(err, err_cap, S2D_ECUDA, msg);
            }
            g_part_ptr[dev] = static_cast<float *>(p);
            g_counter_ptr[dev] = static_cast<int32_t *>(c);
        }
        part = g_part_ptr[dev];
        counters = g_counter_ptr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the counters keep the last call's contents: start from zero
    e = cudaMemsetAsync(counters, 0, sizeof(int32_t) * (size_t)Hkv, s);
    if (e == cudaSuccess) {
        s2d::AttnArgs a{};
        a.q = query, a.kcache = keys, a.vcache = values, a.max_seq = T, a.out = out;
        a.part = part, a.counters = counters, a.pos_const = T - 1;
        a.H = H, a.Hkv = Hkv, a.hd = hd, a.S = S, a.M = 1, a.scale = scale;
        e = s2d::launch_attention(a, false, s, false);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        char msg[256];
        snprintf(msg, sizeof msg, "attention: %s", cudaGetErrorString(e));
        return fail(err, err_cap, S2D_ECUDA, msg);
    }
    return S2D_OK;
}
