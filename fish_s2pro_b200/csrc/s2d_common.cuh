// s2d_common.cuh -- shared device helpers for the sm_100a Dual-AR kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s2d {

constexpr int kWarp = 32;

// Streaming 16-byte load of weights: read once per pass, so keep them out of
// L1 (the activation vectors live there).
__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Programmatic dependent launch: a kernel may start while its predecessor in
// the stream is finishing; it must not read the predecessor's outputs before
// grid_dep_wait().  Both are no-ops when the launch did not enable PDL.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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

// f16 bits -> f32, exact (same values as the reference's f16_bits_to_f32,
// crates/fish_s2_infer/src/tensor.rs:266-287, for every non-NaN input).
__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// The f16 in the low / high half of a 32-bit word, as f32 (value operations
// only, so the packed word never has to live in addressable memory).
__device__ __forceinline__ float h_lo(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xffffu))); }
__device__ __forceinline__ float h_hi(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

// 8 f16 weights (one uint4) dotted with 8 f32 activations.
__device__ __forceinline__ float dot8(const uint4 w, const float4 a, const float4 b, float acc) {
    acc = fmaf(h_lo(w.x), a.x, acc);
    acc = fmaf(h_hi(w.x), a.y, acc);
    acc = fmaf(h_lo(w.y), a.z, acc);
    acc = fmaf(h_hi(w.y), a.w, acc);
    acc = fmaf(h_lo(w.z), b.x, acc);
    acc = fmaf(h_hi(w.z), b.y, acc);
    acc = fmaf(h_lo(w.w), b.z, acc);
    acc = fmaf(h_hi(w.w), b.w, acc);
    return acc;
}

}  // namespace s2d

// Host-side launch helper: cudaLaunchKernelEx with optional PDL.
template <typename... KArgs, typename... Args>
static inline cudaError_t s2d_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t stream, bool pdl, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
