// s2d_kernels.cu -- sm_100a kernels of the Dual-AR decode step.
//
// Each kernel replaces one or more functions of the reference's CPU path
// (crate fish_s2_infer, paths relative to the reference repository root);
// the mapping is given above each kernel.  Batch-1 decode is HBM-bound, so
// the kernels are organised around streaming every weight byte exactly once
// per pass with 16-byte coalesced loads, with the small activation vectors
// staged in shared memory and everything elementwise fused into the
// producing GEMV.
#include <math.h>

#include "s2d_common.cuh"
#include "s2d_kernels.cuh"
#include "s2d_sample.cuh"

namespace s2d {

// ---------------------------------------------------------------------------
// GEMV: y = W . rmsnorm(x)  (+ residual | SwiGLU)
//
// Replaces CpuMatmulBackend::linear (backend.rs:55-73) for every linear of a
// layer, matvec_f16_streaming (tensor.rs:220-264) for the tied LM head, and
// fuses the neighbouring elementwise ops of the layer:
//   prologue: rms_norm_f32 (backend.rs:84-102) of the input vector;
//   EPI_RESID: the residual adds (slow_ar.rs:697-701, 839-843);
//   EPI_SWIGLU_*: w1 and w3 in one pass plus swiglu_split
//                 (slow_ar.rs:1215-1232 / fast_ar.rs:472-485).
// One warp owns one output row at a time; lanes stride the row in 16-byte
// chunks.  The activation vector is staged in shared memory in a layout where
// chunk c's low and high halves are stored in separate planes, so the 32
// lanes' float4 reads of a warp hit 32 distinct banks.
// ---------------------------------------------------------------------------

__device__ __forceinline__ int gemv_row(const GemvArgs &a, int row) {
    if (a.n_contig < 0) return row;
    return row < a.n_contig ? a.row_base + row : a.extra_row;
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <int M, int EPI>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
    constexpr int NW = kGemvThreads / kWarp;
    constexpr bool DUAL = EPI == EPI_SWIGLU_SLOW || EPI == EPI_SWIGLU_FAST;
    constexpr int U = (DUAL || M > 2) ? 4 : 8;
    extern __shared__ float4 xs4[];
    __shared__ float red[M][NW];
    __shared__ float scl[M];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K, N = a.N, nchunk = K >> 3;
    const int gw = blockIdx.x * NW + warp, stride = gridDim.x * NW;

    // Weights do not depend on the previous kernel: start pulling this warp's
    // rows into L2 before waiting for the predecessor's activations.
    if (lane == 0) {
        for (int row = gw; row < N; row += stride) {
            prefetch_l2(a.W + (size_t)gemv_row(a, row) * K, (uint32_t)K * 2u);
            if (DUAL) prefetch_l2(a.W2 + (size_t)row * K, (uint32_t)K * 2u);
        }
    }
    grid_dep_launch();
    grid_dep_wait();
    if (a.done && *a.done) return;

    float *xs = reinterpret_cast<float *>(xs4);
    if (a.norm_w) {
        float ss[M];
#pragma unroll
        for (int m = 0; m < M; ++m) ss[m] = 0.f;
        for (int i = tid; i < K; i += kGemvThreads) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float v = a.x[(size_t)m * a.ldx + i];
                ss[m] = fmaf(v, v, ss[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float s = warp_sum(ss[m]);
            if (lane == 0) red[m][warp] = s;
        }
        __syncthreads();
        if (tid < M) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) t += red[tid][w];
            scl[tid] = 1.0f / sqrtf(t / (float)K + a.eps);
        }
        __syncthreads();
    }
    for (int i = tid; i < K; i += kGemvThreads) {
        const int c = i >> 3, k = i & 7;
        const int idx = (((k >> 2) * nchunk) + c) * 4 + (k & 3);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float v = a.x[(size_t)m * a.ldx + i];
            if (a.norm_w) v = __fmul_rn(__fmul_rn(v, scl[m]), a.norm_w[i]);
            xs[m * 2 * nchunk * 4 + idx] = v;
            if (a.x_out && blockIdx.x == 0) a.x_out[(size_t)m * K + i] = v;
        }
    }
    __syncthreads();

    for (int row = gw; row < N; row += stride) {
        const uint4 *w = reinterpret_cast<const uint4 *>(a.W + (size_t)gemv_row(a, row) * K);
        const uint4 *w2 = DUAL ? reinterpret_cast<const uint4 *>(a.W2 + (size_t)row * K) : nullptr;
        float acc[M], acc2[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.f, acc2[m] = 0.f;
        for (int c0 = lane; c0 < nchunk; c0 += 32 * U) {
            uint4 wv[U], wv2[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + 32 * u;
                if (c < nchunk) {
                    wv[u] = ld_stream_u4(w + c);
                    if (DUAL) wv2[u] = ld_stream_u4(w2 + c);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + 32 * u;
                if (c < nchunk) {
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        const float4 xa = xs4[m * 2 * nchunk + c];
                        const float4 xb = xs4[m * 2 * nchunk + nchunk + c];
                        acc[m] = dot8(wv[u], xa, xb, acc[m]);
                        if (DUAL) acc2[m] = dot8(wv2[u], xa, xb, acc2[m]);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            acc[m] = warp_sum(acc[m]);
            if (DUAL) acc2[m] = warp_sum(acc2[m]);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            if (lane != m) continue;
            float out;
            if (EPI == EPI_STORE) {
                out = acc[m];
            } else if (EPI == EPI_RESID) {
                out = __fadd_rn(a.resid[(size_t)m * a.ldr + row], acc[m]);
            } else if (EPI == EPI_SWIGLU_SLOW) {
                const float g = acc[m], up = acc2[m];
                const float sig = 1.0f / (1.0f + expf(-g));
                out = __fmul_rn(__fmul_rn(g, sig), up);
            } else {
                const float g = acc[m], up = acc2[m];
                out = __fmul_rn(g / (1.0f + expf(-g)), up);
            }
            a.y[(size_t)m * a.ldy + row] = out;
        }
    }
}

template <int M, int EPI>
static cudaError_t gemv_launch_t(const GemvArgs &a, cudaStream_t s, bool pdl) {
    const int NW = kGemvThreads / kWarp;
    int blocks = (a.N + NW - 1) / NW;
    if (blocks > 148 * 8) blocks = 148 * 8;
    const size_t smem = (size_t)M * a.K * sizeof(float);
    return s2d_launch(gemv_kernel<M, EPI>, dim3(blocks), dim3(kGemvThreads), smem, s, pdl, a);
}

template <int M>
static cudaError_t gemv_dispatch_epi(const GemvArgs &a, int epi, cudaStream_t s, bool pdl) {
    switch (epi) {
    case EPI_STORE: return gemv_launch_t<M, EPI_STORE>(a, s, pdl);
    case EPI_RESID: return gemv_launch_t<M, EPI_RESID>(a, s, pdl);
    case EPI_SWIGLU_SLOW: return gemv_launch_t<M, EPI_SWIGLU_SLOW>(a, s, pdl);
    case EPI_SWIGLU_FAST: return gemv_launch_t<M, EPI_SWIGLU_FAST>(a, s, pdl);
    }
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// Quantized linears for the per-op path (single steps, short prefills, the
// op-level APIs): one block per output row, threads over 32-element ggml
// sub-blocks, each weight dequantised as the block format defines
// (EngineWeight) and multiplied with the (optionally RMS-normalised) input.
// Not a hot path: decode frames run in the persistent engine.
// ---------------------------------------------------------------------------

// The 6-bit scale and min of sub-block j of a ggml Q4_K superblock.
__device__ __forceinline__ void q4k_scale_min_dev(int j, const uint8_t *p, int *sc, int *mn) {
    if (j < 4) {
        *sc = p[j] & 63;
        *mn = p[j + 4] & 63;
    } else {
        *sc = (p[j + 4] & 0x0f) | ((p[j - 4] >> 6) << 4);
        *mn = (p[j + 4] >> 4) | ((p[j] >> 6) << 4);
    }
}
__device__ __forceinline__ float f16_bits(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}
// Element i (0..31) of 32-element sub-block `blk` of a ggml row.
struct QuantSub {
    float a, b;  // value = a * q - b (Q4_K) or q * a (Q8_0, b unused)
    const uint8_t *q;
    int shift;   // Q4_K nibble shift
    __device__ QuantSub(int wq, const uint8_t *row, int blk) {
        if (wq == 1) {
            const uint8_t *p = row + (size_t)blk * 34;
            a = f16_bits(p), b = 0.f, q = p + 2, shift = 0;
        } else {
            const uint8_t *p = row + (size_t)(blk / 8) * 144;
            const int j = blk % 8;
            int sc, mn;
            q4k_scale_min_dev(j, p + 4, &sc, &mn);
            a = f16_bits(p) * (float)sc, b = f16_bits(p + 2) * (float)mn;
            q = p + 16 + 32 * (j / 2), shift = (j & 1) * 4;
        }
    }
    __device__ __forceinline__ float at(int wq, int i) const {
        if (wq == 1) return __fmul_rn((float)(int8_t)q[i], a);
        return __fsub_rn(__fmul_rn(a, (float)((q[i] >> shift) & 0xf)), b);
    }
};

template <int EPI>
__global__ void __launch_bounds__(128) gemv_quant_kernel(const GemvArgs a, int M) {
    grid_dep_launch();
    grid_dep_wait();
    if (a.done && *a.done) return;
    __shared__ float red[4];
    const int row = blockIdx.x, tid = threadIdx.x;
    const int src = a.n_contig < 0 ? row : (row < a.n_contig ? a.row_base + row : a.extra_row);
    const size_t rb = a.wq == 1 ? (size_t)a.K / 32 * 34 : (size_t)a.K / 256 * 144;
    const uint8_t *wrow = reinterpret_cast<const uint8_t *>(a.W) + (size_t)src * rb;
    const uint8_t *wrow2 = a.W2 ? reinterpret_cast<const uint8_t *>(a.W2) + (size_t)row * rb : nullptr;
    auto block_sum = [&](float v) {
        v = warp_sum(v);
        if ((tid & 31) == 0) red[tid >> 5] = v;
        __syncthreads();
        const float t = red[0] + red[1] + red[2] + red[3];
        __syncthreads();
        return t;
    };
    for (int m = 0; m < M; ++m) {
        const float *x = a.x + (size_t)m * a.ldx;
        float scale = 1.f;
        if (a.norm_w) {
            float ss = 0.f;
            for (int i = tid; i < a.K; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
            scale = 1.0f / sqrtf(block_sum(ss) / (float)a.K + a.eps);
        }
        float acc = 0.f, acc2 = 0.f;
        for (int blk = tid; blk < a.K / 32; blk += blockDim.x) {
            const QuantSub s1(a.wq, wrow, blk);
            const QuantSub s2(a.wq, wrow2 ? wrow2 : wrow, blk);
            for (int i = 0; i < 32; ++i) {
                float xv = x[blk * 32 + i];
                if (a.norm_w) xv = __fmul_rn(__fmul_rn(xv, scale), a.norm_w[blk * 32 + i]);
                acc = fmaf(s1.at(a.wq, i), xv, acc);
                if (wrow2) acc2 = fmaf(s2.at(a.wq, i), xv, acc2);
            }
        }
        acc = block_sum(acc);
        if (EPI == EPI_SWIGLU_SLOW || EPI == EPI_SWIGLU_FAST) acc2 = block_sum(acc2);
        if (tid == 0) {
            float out;
            if (EPI == EPI_STORE) {
                out = acc;
            } else if (EPI == EPI_RESID) {
                out = __fadd_rn(a.resid[(size_t)m * a.ldr + row], acc);
            } else if (EPI == EPI_SWIGLU_SLOW) {
                const float sig = 1.0f / (1.0f + expf(-acc));
                out = __fmul_rn(__fmul_rn(acc, sig), acc2);
            } else {
                out = __fmul_rn(acc / (1.0f + expf(-acc)), acc2);
            }
            a.y[(size_t)m * a.ldy + row] = out;
        }
    }
}

// A tensor's ggml blocks are contiguous, so its elements are one long row.
__global__ void dequant_kernel(int wq, const uint8_t *src, float *dst, int64_t n) {
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= n / 32) return;
    const uint8_t *base = src + (wq == 1 ? (size_t)(blk / 8) * 8 * 34 : (size_t)(blk / 8) * 144);
    const QuantSub s(wq, base, (int)(blk % 8));
    for (int i = 0; i < 32; ++i) dst[blk * 32 + i] = s.at(wq, i);
}

// The same values rounded to f16 (round to nearest even), for the tensor-core
// prefill of quantized models.
__global__ void dequant_f16_kernel(int wq, const uint8_t *src, __half *dst, int64_t n) {
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= n / 32) return;
    const uint8_t *base = src + (wq == 1 ? (size_t)(blk / 8) * 8 * 34 : (size_t)(blk / 8) * 144);
    const QuantSub s(wq, base, (int)(blk % 8));
    __align__(16) __half v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __float2half_rn(s.at(wq, i));
    uint4 *d4 = reinterpret_cast<uint4 *>(dst + blk * 32);
    const uint4 *v4 = reinterpret_cast<const uint4 *>(v);
#pragma unroll
    for (int i = 0; i < 4; ++i) d4[i] = v4[i];
}

cudaError_t launch_dequant_f16(int wq, const void *src, __half *dst, int64_t n, cudaStream_t s) {
    if ((wq != 1 && wq != 2) || n % (wq == 1 ? 32 : 256) || (reinterpret_cast<uintptr_t>(dst) & 15))
        return cudaErrorInvalidValue;
    const int64_t blocks = n / 32;
    dequant_f16_kernel<<<(unsigned)((blocks + 255) / 256), 256, 0, s>>>(wq, reinterpret_cast<const uint8_t *>(src),
                                                                       dst, n);
    return cudaGetLastError();
}

cudaError_t launch_dequant(int gtype, const void *src, float *dst, int64_t n, cudaStream_t s) {
    const int wq = gtype == 8 ? 1 : gtype == 12 ? 2 : 0;
    if (!wq || n % (wq == 1 ? 32 : 256)) return cudaErrorInvalidValue;
    const int64_t blocks = n / 32;
    dequant_kernel<<<(unsigned)((blocks + 255) / 256), 256, 0, s>>>(wq, reinterpret_cast<const uint8_t *>(src), dst, n);
    return cudaGetLastError();
}

cudaError_t launch_gemv(const GemvArgs &a, int M, int epi, cudaStream_t s, bool pdl) {
    if (a.wq != 0) {
        if (a.K % (a.wq == 1 ? 32 : 256)) return cudaErrorInvalidValue;
        switch (epi) {
        case EPI_STORE: return s2d_launch(gemv_quant_kernel<EPI_STORE>, dim3(a.N), dim3(128), 0, s, pdl, a, M);
        case EPI_RESID: return s2d_launch(gemv_quant_kernel<EPI_RESID>, dim3(a.N), dim3(128), 0, s, pdl, a, M);
        case EPI_SWIGLU_SLOW:
            return s2d_launch(gemv_quant_kernel<EPI_SWIGLU_SLOW>, dim3(a.N), dim3(128), 0, s, pdl, a, M);
        case EPI_SWIGLU_FAST:
            return s2d_launch(gemv_quant_kernel<EPI_SWIGLU_FAST>, dim3(a.N), dim3(128), 0, s, pdl, a, M);
        }
        return cudaErrorInvalidValue;
    }
    if (a.K % 8 != 0 || a.K <= 0 || a.N <= 0) return cudaErrorInvalidValue;
    if ((size_t)M * a.K * sizeof(float) > 200 * 1024) return cudaErrorInvalidValue;
    switch (M) {
    case 1: return gemv_dispatch_epi<1>(a, epi, s, pdl);
    case 2: return gemv_dispatch_epi<2>(a, epi, s, pdl);
    case 4: return gemv_dispatch_epi<4>(a, epi, s, pdl);
    }
    return cudaErrorInvalidValue;
}

template <int M>
static cudaError_t gemv_cfg_m() {
    cudaError_t e;
    const int bytes = 200 * 1024;
    if ((e = cudaFuncSetAttribute(gemv_kernel<M, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<M, EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<M, EPI_SWIGLU_SLOW>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes))) return e;
    return cudaFuncSetAttribute(gemv_kernel<M, EPI_SWIGLU_FAST>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

static cudaError_t sample_configure();

cudaError_t configure_kernels() {
    cudaError_t e;
    if ((e = gemv_cfg_m<1>())) return e;
    if ((e = gemv_cfg_m<2>())) return e;
    if ((e = gemv_cfg_m<4>())) return e;
    return sample_configure();
}

// ---------------------------------------------------------------------------
// QK-norm + RoPE + KV write.
// Replaces, per token: the Q/K/V split (slow_ar.rs:743-746), rms_norm_heads
// of Q and K (backend.rs:104-121; Slow-AR only, slow_ar.rs:748-763),
// apply_rope_normal (attention.rs:172-206) and SlowArKvCache::write_token
// (attention.rs:56-76).  One warp per head; the head's elements stay in
// registers.  RoPE angles use the host-computed powf table so the rotation
// matches the reference's theta = pos / base^(pair/hd) to the last bit of
// the denominator; products are rounded separately as in the reference.
// ---------------------------------------------------------------------------

template <typename KV>
__device__ __forceinline__ KV to_kv(float v);
template <>
__device__ __forceinline__ __half to_kv<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float to_kv<float>(float v) { return v; }
__device__ __forceinline__ float from_kv(__half v) { return __half2float(v); }
__device__ __forceinline__ float from_kv(float v) { return v; }

template <typename KV, int EPL>
__global__ void __launch_bounds__(256) rope_kv_kernel(const RopeArgs a) {
    grid_dep_launch();
    grid_dep_wait();
    if (a.done && *a.done) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int head = blockIdx.x * (blockDim.x >> 5) + warp;
    const int m = blockIdx.y;
    if (head >= a.H + a.Hkv) return;
    const int rps = a.rows_per_seq > 0 ? a.rows_per_seq : a.M;
    const int seq = m / rps, j = m - seq * rps;
    if (a.st_b && a.st_b[seq].done) return;
    const int pos = a.pos_const + (a.st_b && a.st_pos ? a.st_b[seq].n_past : (a.pos_dev ? *a.pos_dev : 0)) + j;
    const int hd = a.hd;
    const float *row = a.qkv + (size_t)m * a.ld_qkv;
    const float *row_lo = a.qkv_lo ? a.qkv_lo + (size_t)m * a.ld_qkv : nullptr;
    const float s_lo = a.qkv_lo ? a.inv[m] : 1.0f;
    // element i of the row: the stored value, or the combined GEMM halves
    auto fetch = [&](int i) { return row_lo ? __fadd_rn(row[i], row_lo[i]) * s_lo : row[i]; };
    const bool is_q = head < a.H;
    const int h = is_q ? head : head - a.H;
    const int src = is_q ? h * hd : (a.H + h) * hd;
    float v[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = fetch(src + lane * EPL + e);
    const float *nw = is_q ? a.q_norm : a.k_norm;
    if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) ss = fmaf(v[e], v[e], ss);
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / (float)hd + a.eps);
#pragma unroll
        for (int e = 0; e < EPL; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], scale), nw[lane * EPL + e]);
    }
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
        const int pair = lane * EPL + e;
        const float theta = (float)pos / a.rope_denom[pair >> 1];
        float sn, cs;
        sincosf(theta, &sn, &cs);
        const float x0 = v[e], x1 = v[e + 1];
        v[e] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        v[e + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    }
    if (is_q) {
        float *dst = a.q_out + (size_t)m * a.H * hd + h * hd + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dst[e] = v[e];
        return;
    }
    if (pos < 0 || pos >= a.max_seq) {
        if (lane == 0 && a.error) atomicExch(a.error, 1);
        return;
    }
    const size_t ro = kv_row(a.kv_pages, a.kv_seq_stride, a.max_seq, seq, h, pos, hd);
    KV *kc = reinterpret_cast<KV *>(a.kcache) + ro + lane * EPL;
    KV *vc = reinterpret_cast<KV *>(a.vcache) + ro + lane * EPL;
    const int vsrc = (a.H + a.Hkv + h) * hd + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        kc[e] = to_kv<KV>(v[e]);
        vc[e] = to_kv<KV>(fetch(vsrc + e));
    }
}

template <typename KV>
static cudaError_t rope_launch_t(const RopeArgs &a, cudaStream_t s, bool pdl) {
    const int warps = 8;
    dim3 grid((a.H + a.Hkv + warps - 1) / warps, a.M);
    switch (a.hd / 32) {
    case 2: return s2d_launch(rope_kv_kernel<KV, 2>, grid, dim3(warps * 32), 0, s, pdl, a);
    case 4: return s2d_launch(rope_kv_kernel<KV, 4>, grid, dim3(warps * 32), 0, s, pdl, a);
    case 8: return s2d_launch(rope_kv_kernel<KV, 8>, grid, dim3(warps * 32), 0, s, pdl, a);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_rope_kv(const RopeArgs &a, bool kv_half, cudaStream_t s, bool pdl) {
    if (a.hd % 64 != 0 || a.hd > 256) return cudaErrorInvalidValue;
    return kv_half ? rope_launch_t<__half>(a, s, pdl) : rope_launch_t<float>(a, s, pdl);
}

// ---------------------------------------------------------------------------
// GQA decode attention, split over the sequence.
// Replaces SlowArKvCache::decode_attention_with_backend (attention.rs:106-145)
// + gqa_decode_attention / softmax_in_place (attention.rs:208-247, 296-309)
// for one or more query tokens (prefill: each token sees its causal prefix,
// slow_ar.rs:579-593).  Grid (split, kv head, token); one warp per query head
// of the GQA group, so the group's K/V rows are read from HBM once and hit
// L1 for the other heads.  Each split keeps an online softmax (max, sum,
// weighted V) and writes it to scratch; the last split block to arrive (an
// atomic counter per kv head and token) merges the partials and resets the
// counter for the next launch.
// ---------------------------------------------------------------------------

template <typename KV, int EPL>
__device__ __forceinline__ void load_kv(const KV *p, float *out);
template <>
__device__ __forceinline__ void load_kv<__half, 2>(const __half *p, float *o) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(p));
    o[0] = f.x, o[1] = f.y;
}
template <>
__device__ __forceinline__ void load_kv<__half, 4>(const __half *p, float *o) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    o[0] = f0.x, o[1] = f0.y, o[2] = f1.x, o[3] = f1.y;
}
template <>
__device__ __forceinline__ void load_kv<__half, 8>(const __half *p, float *o) {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        o[2 * i] = f.x, o[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void load_kv<float, 2>(const float *p, float *o) {
    const float2 f = *reinterpret_cast<const float2 *>(p);
    o[0] = f.x, o[1] = f.y;
}
template <>
__device__ __forceinline__ void load_kv<float, 4>(const float *p, float *o) {
    const float4 f = *reinterpret_cast<const float4 *>(p);
    o[0] = f.x, o[1] = f.y, o[2] = f.z, o[3] = f.w;
}
template <>
__device__ __forceinline__ void load_kv<float, 8>(const float *p, float *o) {
    const float4 f = *reinterpret_cast<const float4 *>(p);
    const float4 g = *reinterpret_cast<const float4 *>(p + 4);
    o[0] = f.x, o[1] = f.y, o[2] = f.z, o[3] = f.w, o[4] = g.x, o[5] = g.y, o[6] = g.z, o[7] = g.w;
}

template <typename KV, int EPL>
__global__ void __launch_bounds__(512) attn_kernel(const AttnArgs a) {
    __shared__ int s_last;
    grid_dep_launch();
    grid_dep_wait();
    if (a.done && *a.done) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, rep = blockDim.x >> 5;
    const int sp = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
    const int h = kvh * rep + warp;
    const int hd = a.hd, S = a.S;
    const int pos = a.pos_const + (a.pos_dev ? *a.pos_dev : 0) + m;
    int visible = pos + 1;
    if (visible > a.max_seq) visible = a.max_seq;
    const int chunk = (visible + S - 1) / S;
    const int t0 = sp * chunk;
    const int t1 = min(visible, t0 + chunk);
    float q[EPL], acc[EPL];
    const float *qp = a.q + (size_t)m * a.H * hd + h * hd + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) q[e] = qp[e], acc[e] = 0.f;
    float mrun = -INFINITY, l = 0.f;
    const KV *kb = reinterpret_cast<const KV *>(a.kcache) + (size_t)kvh * a.max_seq * hd + lane * EPL;
    const KV *vb = reinterpret_cast<const KV *>(a.vcache) + (size_t)kvh * a.max_seq * hd + lane * EPL;
    for (int t = t0; t < t1; ++t) {
        float kf[EPL], vf[EPL];
        load_kv<KV, EPL>(kb + (size_t)t * hd, kf);
        load_kv<KV, EPL>(vb + (size_t)t * hd, vf);
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) d = fmaf(q[e], kf[e], d);
        d = warp_sum(d);
        const float sc = d * a.scale;
        const float mn = fmaxf(mrun, sc);
        const float corr = expf(mrun - mn);
        const float p = expf(sc - mn);
        l = fmaf(l, corr, p);
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] = fmaf(acc[e], corr, p * vf[e]);
        mrun = mn;
    }
    float *pp = a.part + (((size_t)m * a.H + h) * S + sp) * (hd + 2);
    if (lane == 0) {
        __stcg(pp, mrun);
        __stcg(pp + 1, l);
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) __stcg(pp + 2 + lane * EPL + e, acc[e]);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(&a.counters[m * a.Hkv + kvh], 1);
        s_last = (prev == S - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float *base = a.part + ((size_t)m * a.H + h) * S * (hd + 2);
    float gmax = -INFINITY;
    for (int j = 0; j < S; ++j) gmax = fmaxf(gmax, __ldcg(base + (size_t)j * (hd + 2)));
    float L = 0.f, o[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = 0.f;
    for (int j = 0; j < S; ++j) {
        const float *pj = base + (size_t)j * (hd + 2);
        const float f = expf(__ldcg(pj) - gmax);
        L = fmaf(__ldcg(pj + 1), f, L);
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[e] = fmaf(__ldcg(pj + 2 + lane * EPL + e), f, o[e]);
    }
    float *op = a.out + (size_t)m * a.H * hd + h * hd + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) op[e] = o[e] / L;
    if (threadIdx.x == 0) a.counters[m * a.Hkv + kvh] = 0;
}

template <typename KV>
static cudaError_t attn_launch_t(const AttnArgs &a, cudaStream_t s, bool pdl) {
    const int rep = a.H / a.Hkv;
    dim3 grid(a.S, a.Hkv, a.M);
    switch (a.hd / 32) {
    case 2: return s2d_launch(attn_kernel<KV, 2>, grid, dim3(rep * 32), 0, s, pdl, a);
    case 4: return s2d_launch(attn_kernel<KV, 4>, grid, dim3(rep * 32), 0, s, pdl, a);
    case 8: return s2d_launch(attn_kernel<KV, 8>, grid, dim3(rep * 32), 0, s, pdl, a);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_attention(const AttnArgs &a, bool kv_half, cudaStream_t s, bool pdl) {
    if (a.Hkv <= 0 || a.H % a.Hkv || a.H / a.Hkv > 16 || a.hd % 64 || a.hd > 256 || a.S <= 0)
        return cudaErrorInvalidValue;
    return kv_half ? attn_launch_t<__half>(a, s, pdl) : attn_launch_t<float>(a, s, pdl);
}

// ---------------------------------------------------------------------------
// Slow-AR input embedding.
// Replaces build_step_input (generate.rs:300-344) and
// embed_slow_ar_time_major (slow_ar.rs:1041-1133): semantic row plus, for a
// semantic id, the codebook rows summed in codebook order, then scaled by
// 1/sqrt(K+1).  The additions and the scaling are rounded exactly as the
// reference does, so this kernel's output is bit-identical to it.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) embed_kernel(const EmbedArgs a) {
    grid_dep_launch();
    grid_dep_wait();
    if (a.done && *a.done) return;
    const int m = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.d) return;
    const int cd = a.K + 1;
    uint32_t main_id;
    if (a.tokens) {
        const int32_t t = a.tokens[(size_t)m * cd];
        if (t < 0) {
            if (i == 0) atomicExch(a.error, 2);
            return;
        }
        main_id = (uint32_t)t;
    } else {
        main_id = a.st[a.batched ? m : 0].main_token;
    }
    const bool is_sem = main_id >= a.sem_begin && main_id <= a.sem_end;
    if (main_id >= (uint32_t)a.vocab) {
        if (i == 0) atomicExch(a.error, 3);
        return;
    }
    float h = h2f(a.emb[(size_t)main_id * a.d + i]);
    if (is_sem) {
        float sum = 0.f;
        for (int cb = 0; cb < a.K; ++cb) {
            const int32_t raw = a.tokens ? a.tokens[(size_t)m * cd + 1 + cb]
                                         : a.frame_codes[(a.batched ? (size_t)m * a.K : 0) + cb];
            const int64_t cid = (int64_t)raw + (int64_t)cb * a.cb_size;
            if (raw < 0 || cid >= a.cb_rows) {
                if (i == 0) atomicExch(a.error, 4);
                return;
            }
            sum = __fadd_rn(sum, h2f(a.cb_emb[(size_t)cid * a.d + i]));
        }
        h = __fadd_rn(h, sum);
    }
    if (a.scale_on) h = __fmul_rn(h, is_sem ? a.sem_scale : 1.0f);
    a.out[(size_t)m * a.d + i] = h;
}

cudaError_t launch_embed(const EmbedArgs &a, cudaStream_t s, bool pdl) {
    dim3 grid((a.d + 255) / 256, a.M);
    return s2d_launch(embed_kernel, grid, dim3(256), 0, s, pdl, a);
}

// ---------------------------------------------------------------------------
// Fast-AR frame start: semantic_to_codebook_id (generate.rs:273-282) and the
// first two positions of the Fast-AR sequence [slow_hidden, fast_emb[c0]]
// (fast_ar.rs:393-403).  code 0 of the frame goes to the output codes
// (generate.rs:176-191).
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) fast_init_kernel(const FastInitArgs a) {
    grid_dep_launch();
    grid_dep_wait();
    const size_t sq = a.batched ? blockIdx.y : 0;
    const DevState *st = a.st + sq;
    if (st->done) return;
    float *fast_x = a.fast_x + sq * a.fast_x_stride;
    int32_t *frame_codes = a.frame_codes + sq * a.frame_stride;
    int32_t *codes_out = a.codes_out ? a.codes_out + sq * a.codes_stride : nullptr;
    const float *slow_hidden = a.slow_hidden + sq * a.hidden_stride;
    uint32_t code;
    if (a.code_override) {
        code = *a.code_override;
    } else {
        const uint32_t mt = st->main_token;
        if (mt < a.sem_begin || mt > a.sem_end) code = 0;
        else {
            code = mt - a.sem_begin;
            if (code >= (uint32_t)a.cb_size) code = (uint32_t)a.cb_size - 1;
        }
    }
    if (code >= (uint32_t)a.cb_size) code = (uint32_t)a.cb_size - 1;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        frame_codes[0] = (int32_t)code;
        if (codes_out) codes_out[st->step_index] = (int32_t)code;
    }
    if (i < a.d) {
        fast_x[i] = slow_hidden[i];
        fast_x[a.d + i] = h2f(a.fast_emb[(size_t)code * a.d + i]);
    }
}

cudaError_t launch_fast_init(const FastInitArgs &a, cudaStream_t s, bool pdl) {
    return s2d_launch(fast_init_kernel, dim3((a.d + 255) / 256), dim3(256), 0, s, pdl, a);
}

cudaError_t launch_fast_init_batch(const FastInitArgs &a, int n_seq, cudaStream_t s) {
    if (!a.batched || n_seq <= 0 || n_seq > 65535) return cudaErrorInvalidValue;
    return s2d_launch(fast_init_kernel, dim3((a.d + 255) / 256, n_seq), dim3(256), 0, s, false, a);
}

// ---------------------------------------------------------------------------
// Device sampler kernel: one 1,024-thread block per sequence running
// sample_block (s2d_sample.cuh), then the next Fast-AR input row.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SampleArgs a) {
    extern __shared__ unsigned long long skeys[];  // [kSampleMax]
    float *probs = reinterpret_cast<float *>(skeys + kSampleMax);  // [kSampleMax + 1]
    __shared__ SampleScratch scratch;
    grid_dep_launch();
    grid_dep_wait();
    const uint32_t sq = a.batched ? blockIdx.x : 0u;
    const DevState *st = a.st ? a.st + sq : nullptr;
    if (a.mode != SAMPLE_PLAIN && st->done) return;
    const uint32_t token = sample_block<kSampleThreads, kSampleMax>(a, sq, a.logits + sq * a.logits_stride, skeys,
                                                                   probs, scratch, [] { __syncthreads(); });
    float *fast_x_next = a.fast_x_next ? a.fast_x_next + sq * a.fast_x_stride : nullptr;
    if (a.mode == SAMPLE_FAST && fast_x_next) {
        for (int i = threadIdx.x; i < a.d; i += kSampleThreads)
            fast_x_next[i] = h2f(a.fast_emb[(size_t)token * a.d + i]);
    }
}

static constexpr size_t kSampleSmem =
    kSampleMax * sizeof(unsigned long long) + (kSampleMax + 1) * sizeof(float);

static cudaError_t sample_configure() {
    return cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kSampleSmem);
}

cudaError_t launch_sample(const SampleArgs &a, cudaStream_t s, bool pdl) {
    if (a.n <= 0 || a.n > kSampleMax || a.batched) return cudaErrorInvalidValue;
    return s2d_launch(sample_kernel, dim3(1), dim3(kSampleThreads), kSampleSmem, s, pdl, a);
}

__global__ void philox_kernel(uint4 c, uint2 k, uint4 *out) { *out = philox4x32_10(c, k); }

cudaError_t launch_philox(const uint32_t counter[4], const uint32_t key[2], uint32_t *out_dev, cudaStream_t s) {
    philox_kernel<<<1, 1, 0, s>>>(make_uint4(counter[0], counter[1], counter[2], counter[3]),
                                  make_uint2(key[0], key[1]), reinterpret_cast<uint4 *>(out_dev));
    return cudaGetLastError();
}

cudaError_t launch_sample_batch(const SampleArgs &a, int n_seq, cudaStream_t s) {
    if (a.n <= 0 || a.n > kSampleMax || !a.batched || !a.st || a.mode == SAMPLE_PLAIN || n_seq <= 0)
        return cudaErrorInvalidValue;
    return s2d_launch(sample_kernel, dim3(n_seq), dim3(kSampleThreads), kSampleSmem, s, false, a);
}

// ---------------------------------------------------------------------------
// Small helpers: exact f16 expansion (tensor.rs:22-75), op-level head
// RMSNorm (backend.rs:104-121), state initialisation.
// ---------------------------------------------------------------------------

__global__ void f16_to_f32_kernel(const uint16_t *src, float *dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = h2f(src[i]);
}

cudaError_t launch_f16_to_f32(const uint16_t *src, float *dst, int64_t n, cudaStream_t s) {
    const int64_t want = (n + 255) / 256;
    int blocks = (int)(want < 148 * 16 ? want : 148 * 16);
    if (blocks < 1) blocks = 1;
    f16_to_f32_kernel<<<blocks, 256, 0, s>>>(src, dst, n);
    return cudaGetLastError();
}

__global__ void rms_norm_heads_kernel(const float *x, const float *w, float *y, int hd, float eps) {
    __shared__ float red[32];
    const float *xh = x + (size_t)blockIdx.x * hd;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) ss = fmaf(xh[i], xh[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
        red[0] = 1.0f / sqrtf(t / (float)hd + eps);
    }
    __syncthreads();
    const float scale = red[0];
    for (int i = threadIdx.x; i < hd; i += blockDim.x)
        y[(size_t)blockIdx.x * hd + i] = __fmul_rn(__fmul_rn(xh[i], scale), w[i]);
}

cudaError_t launch_rms_norm_heads(const float *x, const float *w, float *y, int64_t n, int hd,
                                  float eps, cudaStream_t s) {
    if (hd <= 0 || n % hd) return cudaErrorInvalidValue;
    rms_norm_heads_kernel<<<(unsigned)(n / hd), 256, 0, s>>>(x, w, y, hd, eps);
    return cudaGetLastError();
}

__global__ void set_state_kernel(DevState *st, int32_t n_past, int32_t prompt_cols, uint64_t rng) {
    st->n_past = n_past;
    st->step_index = 0;
    st->done = 0;
    st->main_token = 0;
    st->rng = rng;
    st->error = 0;
    st->prompt_cols = prompt_cols;
}

cudaError_t launch_set_state(DevState *st, int32_t n_past, int32_t prompt_cols, uint64_t rng,
                             cudaStream_t s) {
    set_state_kernel<<<1, 1, 0, s>>>(st, n_past, prompt_cols, rng);
    return cudaGetLastError();
}

}  // namespace s2d
