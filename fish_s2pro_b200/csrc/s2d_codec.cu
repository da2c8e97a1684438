// s2d_codec.cu -- the codec decode on sm_100a: RVQ codes -> 44.1 kHz PCM
// (crates/fish_s2_infer/src/codec.rs:1690 decode_waveform and what it calls).
//
// Activations are frame-major float rows in HBM ([frames][channels]); every
// contraction is one f16 tensor-core GEMM with f32 accumulation:
// * linears and transposed convolutions take float inputs, so their rows go
//   in as power-of-two scaled f16 hi + lo pairs (launch_split_rows, about 22
//   bits) stacked [2T][K], and an epilogue kernel adds the halves back;
// * the causal convolutions round their padded input to f16 in the reference
//   itself (codec.rs:2257-2259), so their im2col rows are exact in f16 and go
//   in alone: one GEMM of K = taps x channels per convolution.
// The transposed convolutions are one GEMM over all kernel taps ([T][k C]
// per input frame) and a col2im pass that sums the overlapping taps in the
// reference's frame order and adds the bias.  Snake, LayerNorm, GELU, RoPE,
// the windowed attention and the output convolution are CUDA-core kernels.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "../../include/s2d.h"
#include "../../include/s2d_codec.h"
#include "s2d_codec.cuh"
#include "s2d_gguf.h"
#include "s2d_prefill.cuh"

namespace s2d {
namespace {

// codec.rs:16-55
constexpr int kHid = 1024, kProj = 8, kFfn = 3072, kHeads = 16, kHd = 64, kWin = 128, kLayers = 8;
constexpr int kExp = 4096, kUpStages = 2, kUp = 2, kDw = 7, kEntry = 1536, kBlocks = 4, kBooks = 10;
constexpr int kRates[kBlocks] = {8, 8, 4, 2};
constexpr int kChan[kBlocks] = {768, 384, 192, 96};  // block_output_channels, codec.rs:2003-2012
constexpr int kSemBook = 4096, kResBook = 1024;
constexpr float kNormEps = 1e-5f, kLnEps = 1e-6f, kRopeBase = 10000.0f;
constexpr int kSamplesPerLatent = 8 * 8 * 4 * 2;
constexpr int kTailTile = 128;

// ---------------------------------------------------------------- kernels --

struct RvqArgs {
    const __half *book[kBooks];   // [n][8]
    const __half *oproj[kBooks];  // [1024][8]
    const __half *obias[kBooks];  // [1024]
    int size[kBooks];
};

// rvq_lookup_codes (codec.rs:2536): per frame and channel, for each codebook
// in order, latents += (sum_j codebook[code][j] * out_proj[c][j]) + bias[c],
// each sum left to right in f32 without fused multiply-adds, as the CPU
// linear / add_bias / add do it: the result is bit-exact.
__global__ void rvq_kernel(RvqArgs a, const int32_t *codes, int T, float *lat, int32_t *error) {
    const int t = blockIdx.x;
    for (int c = threadIdx.x; c < kHid; c += blockDim.x) {
        float acc = 0.f;
        for (int cb = 0; cb < kBooks; ++cb) {
            const int code = codes[(size_t)cb * T + t];
            if (code < 0 || code >= a.size[cb]) {
                if (error) atomicCAS(error, 0, 1);
                continue;
            }
            const __half *row = a.book[cb] + (size_t)code * kProj;
            const __half *w = a.oproj[cb] + (size_t)c * kProj;
            float p = 0.f;
#pragma unroll
            for (int j = 0; j < kProj; ++j) p = __fadd_rn(p, __fmul_rn(__half2float(row[j]), __half2float(w[j])));
            p = __fadd_rn(p, __half2float(a.obias[cb][c]));
            acc = __fadd_rn(acc, p);
        }
        lat[(size_t)t * kHid + c] = acc;
    }
}

__device__ __forceinline__ float combine(const float *Y2, const float *inv, int T, int N, int t, int n) {
    return (Y2[(size_t)t * N + n] + Y2[((size_t)T + t) * N + n]) * inv[t];
}

// The wqkv rows of the stacked GEMM combined, q and k rotated in place
// (apply_rope_normal, attention.rs:172: adjacent pairs, theta = t / freq[i],
// freq[i] = base^(2i / 64) computed on the host in f32).
__global__ void qkv_rope_kernel(const float *Y2, const float *inv, int T, const float *freq, float *qkv) {
    const int t = blockIdx.x;
    constexpr int N = 3 * kHid;
    for (int p = threadIdx.x; p < N / 2; p += blockDim.x) {
        const int n = 2 * p;
        float x0 = combine(Y2, inv, T, N, t, n), x1 = combine(Y2, inv, T, N, t, n + 1);
        if (n < 2 * kHid) {
            const float theta = (float)t / freq[(n % kHd) / 2];
            float s, c;
            sincosf(theta, &s, &c);
            const float r0 = x0 * c - x1 * s, r1 = x0 * s + x1 * c;
            x0 = r0, x1 = r1;
        }
        qkv[(size_t)t * N + n] = x0;
        qkv[(size_t)t * N + n + 1] = x1;
    }
}

// Query row t of head h over keys max(0, t + 1 - WIN) .. t
// (codec.rs:3270-3297 with gqa_decode_attention, attention.rs:208, and
// softmax_in_place, attention.rs:296; WIN 128 in the post and pre modules,
// 512 in the encoder): one block of 128 threads, WIN / 128 visible positions
// per thread for the scores, two half-blocks over positions for P V.
template <int WIN>
__global__ void __launch_bounds__(kWin) window_attn_kernel(const float *qkv, int T, float *out) {
    constexpr int PER = WIN / kWin;
    const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    __shared__ float q[kHd], p[WIN], red[kWin / 32], part[2][kHd];
    constexpr int N = 3 * kHid;
    const int lo = max(0, t + 1 - WIN), n = t + 1 - lo;
    if (tid < kHd) q[tid] = qkv[(size_t)t * N + h * kHd + tid];
    __syncthreads();
    float s[PER], m = -INFINITY;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const int j = tid + kWin * e;
        s[e] = -INFINITY;
        if (j < n) {
            const float4 *k = reinterpret_cast<const float4 *>(qkv + (size_t)(lo + j) * N + kHid + h * kHd);
            float acc = 0.f;
#pragma unroll
            for (int d = 0; d < kHd / 4; ++d) {
                const float4 kv = k[d];
                acc += q[4 * d] * kv.x + q[4 * d + 1] * kv.y + q[4 * d + 2] * kv.z + q[4 * d + 3] * kv.w;
            }
            s[e] = acc * 0.125f;  // 1 / sqrt(64)
        }
        m = fmaxf(m, s[e]);
    }
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        s[e] = tid + kWin * e < n ? expf(s[e] - m) : 0.f;
        sum += s[e];
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((tid & 31) == 0) red[tid >> 5] = sum;
    __syncthreads();
    sum = red[0] + red[1] + red[2] + red[3];
#pragma unroll
    for (int e = 0; e < PER; ++e) p[tid + kWin * e] = s[e] / sum;
    __syncthreads();
    const int d = tid & (kHd - 1), half = tid >> 6;
    float acc = 0.f;
    for (int j = half; j < n; j += 2) acc += p[j] * qkv[(size_t)(lo + j) * N + 2 * kHid + h * kHd + d];
    part[half][d] = acc;
    __syncthreads();
    if (tid < kHd) out[(size_t)t * kHid + h * kHd + tid] = part[0][tid] + part[1][tid];
}

// The same attention with the key / value rows shared by a tile of 32 query
// frames: each chunk of 32 positions of the tile's window is staged in shared
// memory once, and every warp runs an online softmax for 4 frames over it
// (lane = position for the scores, lane = two head dims for P V).  The
// per-frame kernel above re-reads up to WIN rows from L2 for every frame.
constexpr int kWaFrames = 32, kWaChunk = 32;
__global__ void __launch_bounds__(256) window_attn_tiled_kernel(const float *qkv, int T, int window, float *out) {
    __shared__ float qs[kWaFrames][kHd], ks[kWaChunk][kHd + 1];
    __shared__ __align__(8) float vs[kWaChunk][kHd];
    constexpr int N = 3 * kHid;
    const int t0 = blockIdx.x * kWaFrames, h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kWaFrames * kHd; i += blockDim.x) {
        const int f = i / kHd, d = i % kHd, t = t0 + f;
        qs[f][d] = t < T ? qkv[(size_t)t * N + h * kHd + d] : 0.f;
    }
    const int p_lo = max(0, t0 - window + 1), p_hi = min(T, t0 + kWaFrames) - 1;
    float m[4], l[4], o[4][2];
#pragma unroll
    for (int q = 0; q < 4; ++q) m[q] = -INFINITY, l[q] = 0.f, o[q][0] = 0.f, o[q][1] = 0.f;
    for (int p0 = p_lo; p0 <= p_hi; p0 += kWaChunk) {
        __syncthreads();  // the previous chunk (and the q rows) are in place / consumed
        for (int i = threadIdx.x; i < kWaChunk * kHd; i += blockDim.x) {
            const int j = i / kHd, d = i % kHd, p = p0 + j;
            const bool in = p <= p_hi;
            ks[j][d] = in ? qkv[(size_t)p * N + kHid + h * kHd + d] : 0.f;
            vs[j][d] = in ? qkv[(size_t)p * N + 2 * kHid + h * kHd + d] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int f = warp * 4 + q, t = t0 + f, p = p0 + lane;
            const bool vis = t < T && p <= t && p >= t - window + 1 && p <= p_hi;
            float sc = -INFINITY;
            if (vis) {
                float acc = 0.f;
#pragma unroll 16
                for (int d = 0; d < kHd; ++d) acc += qs[f][d] * ks[lane][d];
                sc = acc * 0.125f;  // 1 / sqrt(64)
            }
            float cm = sc;
            for (int off = 16; off; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, off));
            if (cm == -INFINITY) continue;  // nothing of this chunk is visible to frame t (warp-uniform)
            const float mn = fmaxf(m[q], cm);
            const float corr = m[q] == -INFINITY ? 0.f : expf(m[q] - mn);
            const float e = vis ? expf(sc - mn) : 0.f;
            float es = e;
            for (int off = 16; off; off >>= 1) es += __shfl_xor_sync(0xffffffffu, es, off);
            l[q] = l[q] * corr + es;
            float a0 = o[q][0] * corr, a1 = o[q][1] * corr;
#pragma unroll 8
            for (int j = 0; j < kWaChunk; ++j) {
                const float pj = __shfl_sync(0xffffffffu, e, j);
                const float2 v = *reinterpret_cast<const float2 *>(&vs[j][2 * lane]);
                a0 += pj * v.x, a1 += pj * v.y;
            }
            o[q][0] = a0, o[q][1] = a1, m[q] = mn;
        }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int t = t0 + warp * 4 + q;
        if (t < T) {
            float *dst = out + (size_t)t * kHid + h * kHd + 2 * lane;
            dst[0] = o[q][0] / l[q];
            dst[1] = o[q][1] / l[q];
        }
    }
}

enum CodecEpi { CE_STORE = 0, CE_GELU = 1, CE_SWIGLU = 2, CE_SCALE_RESID = 3 };

// erf by Abramowitz & Stegun 7.1.26, the form codec.rs:3890 uses.
__device__ __forceinline__ float erf_as(float v) {
    const float sign = v < 0.f ? -1.f : 1.f, x = fabsf(v);
    const float t = 1.f / (1.f + 0.3275911f * x);
    const float poly = (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t +
                        0.254829592f) * t;
    return sign * (1.f - poly * expf(-x * x));
}

// y[t][n] from the stacked GEMM rows: v = combined + bias[n % nb]; STORE v,
// GELU gelu_erf(v) (codec.rs:3886), SWIGLU silu(v) * u with u combined from
// Y2b (codec.rs:3313-3317), SCALE_RESID r[t][n] + gamma[n] * v (y may alias r).
__global__ void epilogue_kernel(int epi, const float *Y2, const float *Y2b, const float *inv, int T, int N,
                                const float *bias, int nb, const float *gamma, const float *r, float *y) {
    const size_t total = (size_t)T * N;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / N), n = (int)(i % N);
        float v = combine(Y2, inv, T, N, t, n);
        if (bias) v += bias[n % nb];
        if (epi == CE_GELU) {
            v = 0.5f * v * (1.f + erf_as(v * 0.70710678118654752f));
        } else if (epi == CE_SWIGLU) {
            const float u = combine(Y2b, inv, T, N, t, n);
            v = v / (1.f + expf(-v)) * u;
        } else if (epi == CE_SCALE_RESID) {
            v = r[i] + gamma[n] * v;
        }
        y[i] = v;
    }
}

// ConvNeXt front (codec.rs:3438-3458): depthwise causal conv (kernel 7) and
// the affine LayerNorm of each frame, one block per frame.
__global__ void __launch_bounds__(256) dwconv_ln_kernel(const float *x, int T, const float *w, const float *b,
                                                        const float *lnw, const float *lnb, float *out) {
    const int t = blockIdx.x;
    constexpr int PER = kHid / 256;
    __shared__ float red[8];
    float h[PER];
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const int c = threadIdx.x + 256 * e;
        float acc = b[c];
#pragma unroll
        for (int k = 0; k < kDw; ++k) {
            const int src = t + k - (kDw - 1);
            if (src >= 0) acc += x[(size_t)src * kHid + c] * w[c * kDw + k];
        }
        h[e] = acc;
        s += acc;
    }
    auto block_sum = [&](float v) {
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
        __syncthreads();
        float r = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) r += red[i];
        return r;
    };
    const float mean = block_sum(s) / kHid;
    float v2 = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) v2 += (h[e] - mean) * (h[e] - mean);
    const float scale = 1.f / sqrtf(block_sum(v2) / kHid + kLnEps);
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const int c = threadIdx.x + 256 * e;
        out[(size_t)t * kHid + c] = (h[e] - mean) * scale * lnw[c] + lnb[c];
    }
}

// snake (codec.rs:2162): x + sin(a x)^2 / a, with |a| < 1e-8 taken as 1e-8.
__device__ __forceinline__ float snake(float x, float alpha) {
    const float a = fabsf(alpha) < 1e-8f ? 1e-8f : alpha;
    const float s = sinf(a * x);
    return x + s * s / a;
}

// f16 of four floats, stored as 8 bytes.
__device__ __forceinline__ void st_half4(__half *dst, float a, float b, float c, float d) {
    __half2 lo = __floats2half2_rn(a, b), hi = __floats2half2_rn(c, d);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&lo);
    u.y = *reinterpret_cast<uint32_t *>(&hi);
    *reinterpret_cast<uint2 *>(dst) = u;
}

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// A causal convolution's padded input from a float map: P[pad + t][c] =
// f16(snake(x[t][c] + bias[c])) with bias and snake optional, P[0 .. pad) = 0
// (codec.rs:2247-2259).  Four channels per thread (C % 4 == 0).
__global__ void pad_f16_kernel(const float *x, int T, int C, int pad, const float *bias, const float *alpha,
                               __half *P) {
    const int C4 = C / 4;
    const long long total = (long long)(T + pad) * C4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / C4;
        const int c = (int)(i - row * C4) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row >= pad) {
            v = ld4(x + (row - pad) * C + c);
            if (bias) {
                const float4 b = ld4(bias + c);
                v.x += b.x, v.y += b.y, v.z += b.z, v.w += b.w;
            }
            if (alpha) {
                const float4 a = ld4(alpha + c);
                v = make_float4(snake(v.x, a.x), snake(v.y, a.y), snake(v.z, a.z), snake(v.w, a.w));
            }
        }
        st_half4(P + row * C + c, v.x, v.y, v.z, v.w);
    }
}

// The last two steps of a residual unit and the first of the next
// (codec.rs:2085-2160): x += Z + bias (the unit's output, written back; with
// assign x = Z + bias, a strided conv's output starting the next block), and
// the next unit's padded conv input P[pad + t] = f16(snake(x, alpha)),
// P[0 .. pad) = 0.
__global__ void resid_pad_kernel(float *x, const float *Z, const float *bias, int T, int C, const float *alpha,
                                 int pad, __half *P, bool assign) {
    const int C4 = C / 4;
    const long long total = (long long)(T + pad) * C4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / C4;
        const int c = (int)(i - row * C4) * 4;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row >= pad) {
            float *xr = x + (row - pad) * C + c;
            float4 v = assign ? make_float4(0.f, 0.f, 0.f, 0.f) : ld4(xr);
            const float4 z = ld4(Z + (row - pad) * C + c), b = ld4(bias + c);
            v.x += z.x + b.x, v.y += z.y + b.y, v.z += z.z + b.z, v.w += z.w + b.w;
            *reinterpret_cast<float4 *>(xr) = v;
            if (P) {
                const float4 a = ld4(alpha + c);
                s = make_float4(snake(v.x, a.x), snake(v.y, a.y), snake(v.z, a.z), snake(v.w, a.w));
            }
        }
        if (P) st_half4(P + row * C + c, s.x, s.y, s.z, s.w);
    }
}

// The encoder's entry conv (codec.rs:1112-1124): 1 -> 64 channels, kernel 7,
// causal, input rounded to f16: y[t][c] = b[c] + sum_k f16(x[t + k - 6]) w[c][k].
__global__ void enc_entry_kernel(const float *x, int T, const float *w, const float *b, float *y) {
    const long long total = (long long)T * 64;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long t = i >> 6;
        const int c = (int)(i & 63);
        float acc = b[c];
#pragma unroll
        for (int k = 0; k < 7; ++k) {
            const long long src = t + k - 6;
            if (src >= 0) acc += __half2float(__float2half_rn(x[src])) * w[c * 7 + k];
        }
        y[i] = acc;
    }
}

struct VqArgs {
    const __half *in_w[kBooks];  // [8][1024]
    const __half *in_b[kBooks];  // [8]
};

// rvq_encode_latents_nearest (codec.rs:2598) with nearest_code_for_residual
// (codec.rs:2453-2505): one block per frame; per codebook in order, the
// residual's in_proj (+ bias), the codebook row of the largest cosine
// similarity (the first on ties), then residual -= that code's out_proj
// projection (+ bias, summed as rvq_kernel sums it).  codes [10][T],
// l2[t] = the final residual's norm.
constexpr int kVqThreads = 256;
__global__ void __launch_bounds__(kVqThreads) vq_kernel(VqArgs v, RvqArgs a, const float *lat, int T,
                                                        int32_t *codes, float *l2) {
    __shared__ float r[kHid], proj[kProj], bs[kVqThreads / 32];
    __shared__ int bi[kVqThreads / 32];
    __shared__ float red[kVqThreads / 32];
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < kHid; i += kVqThreads) r[i] = lat[(size_t)t * kHid + i];
    __syncthreads();
    for (int cb = 0; cb < kBooks; ++cb) {
        // in_proj: warp j < 8 takes output j
        if (warp < kProj) {
            const __half *wr = v.in_w[cb] + (size_t)warp * kHid;
            float acc = 0.f;
            for (int i = lane; i < kHid; i += 32) acc += r[i] * __half2float(wr[i]);
            for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) proj[warp] = acc + __half2float(v.in_b[cb][warp]);
        }
        __syncthreads();
        float pn = 0.f;
#pragma unroll
        for (int j = 0; j < kProj; ++j) pn += proj[j] * proj[j];
        pn = sqrtf(fmaxf(pn, 1e-12f));
        float pu[kProj];
#pragma unroll
        for (int j = 0; j < kProj; ++j) pu[j] = proj[j] / pn;
        // the best row of this thread's rows, then of the block (first index on ties)
        float best = -INFINITY;
        int besti = 0x7fffffff;
        for (int k = tid; k < a.size[cb]; k += kVqThreads) {
            const __half *row = a.book[cb] + (size_t)k * kProj;
            float cr[kProj], cn = 0.f;
#pragma unroll
            for (int j = 0; j < kProj; ++j) cr[j] = __half2float(row[j]), cn += cr[j] * cr[j];
            cn = sqrtf(fmaxf(cn, 1e-12f));
            float sc = 0.f;
#pragma unroll
            for (int j = 0; j < kProj; ++j) sc += pu[j] * (cr[j] / cn);
            if (sc > best) best = sc, besti = k;
        }
        for (int o = 16; o; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
            if (ob > best || (ob == best && oi < besti)) best = ob, besti = oi;
        }
        if (lane == 0) bs[warp] = best, bi[warp] = besti;
        __syncthreads();
        best = bs[0], besti = bi[0];
        for (int w = 1; w < kVqThreads / 32; ++w)
            if (bs[w] > best || (bs[w] == best && bi[w] < besti)) best = bs[w], besti = bi[w];
        if (tid == 0) codes[(size_t)cb * T + t] = besti;
        // residual -= the code's projection
        const __half *code = a.book[cb] + (size_t)besti * kProj;
        for (int c = tid; c < kHid; c += kVqThreads) {
            const __half *w = a.oproj[cb] + (size_t)c * kProj;
            float p = 0.f;
#pragma unroll
            for (int j = 0; j < kProj; ++j) p = __fadd_rn(p, __fmul_rn(__half2float(code[j]), __half2float(w[j])));
            p = __fadd_rn(p, __half2float(a.obias[cb][c]));
            r[c] -= p;
        }
        __syncthreads();
    }
    float ss = 0.f;
    for (int i = tid; i < kHid; i += kVqThreads) ss += r[i] * r[i];
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float tot = 0.f;
        for (int w = 0; w < kVqThreads / 32; ++w) tot += red[w];
        l2[t] = sqrtf(tot);
    }
}

// A transposed convolution's input row, split for the tensor cores: v =
// x[t] (+ Z[t] + zb: the previous residual unit's output) (+ bias), s =
// snake(v), then the power-of-two scaled hi / lo halves into xs rows t and
// T + t and inv[t] (the scaling of launch_split_rows).  One warp per row,
// NI float2 per lane (C = 64 NI).
template <int NI>
__global__ void __launch_bounds__(256) snake_split_kernel(const float *x, const float *Z, const float *zb,
                                                          const float *bias, const float *alpha, int T,
                                                          __half *xs, float *inv) {
    constexpr int C = 64 * NI;
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    float2 v[NI];
    float mx = 0.f;
#pragma unroll
    for (int j = 0; j < NI; ++j) {
        const int c = 64 * j + 2 * lane;
        float2 a = *reinterpret_cast<const float2 *>(x + (size_t)t * C + c);
        if (Z) {
            const float2 z = *reinterpret_cast<const float2 *>(Z + (size_t)t * C + c);
            const float2 b = *reinterpret_cast<const float2 *>(zb + c);
            a.x += z.x + b.x, a.y += z.y + b.y;
        }
        if (bias) {
            const float2 b = *reinterpret_cast<const float2 *>(bias + c);
            a.x += b.x, a.y += b.y;
        }
        const float2 al = *reinterpret_cast<const float2 *>(alpha + c);
        v[j] = make_float2(snake(a.x, al.x), snake(a.y, al.y));
        mx = fmaxf(mx, fmaxf(fabsf(v[j].x), fabsf(v[j].y)));
    }
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // a power of two p with mx * p in [2^13, 2^14); 1 for an all-zero row
    float p = 1.f;
    if (mx > 0.f && isfinite(mx)) {
        int e;
        frexpf(mx, &e);
        p = ldexpf(1.f, 14 - e);
    }
    if (lane == 0) inv[t] = 1.f / p;
    __half *hi = xs + (size_t)t * C, *lo = xs + ((size_t)T + t) * C;
#pragma unroll
    for (int j = 0; j < NI; ++j) {
        const int c = 64 * j + 2 * lane;
        const float a = v[j].x * p, b = v[j].y * p;
        const __half2 h = __floats2half2_rn(a, b);
        const float2 hf = __half22float2(h);
        *reinterpret_cast<__half2 *>(hi + c) = h;
        *reinterpret_cast<__half2 *>(lo + c) = __floats2half2_rn(a - hf.x, b - hf.y);
    }
}

// im2col of a stride-1 causal convolution: A[t][k Cp + c] = P[t + k d][c] for
// the taps k < K and c < C, zeros for C <= c < Cp; 16 bytes at a time (C and
// Cp multiples of 8).
__global__ void im2col_kernel(const __half *P, int T, int C, int Cp, int K, int d, __half *A) {
    const int cv = C / 8, cvp = Cp / 8, row = K * cvp;  // uint4 per row of P / per tap of A / per row of A
    const long long total = (long long)T * row;
    const uint4 *src = reinterpret_cast<const uint4 *>(P);
    uint4 *dst = reinterpret_cast<uint4 *>(A);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / row;
        const int r = (int)(i - t * row), k = r / cvp, j = r - k * cvp;
        dst[i] = j < cv ? src[(t + (long long)k * d) * cv + j] : make_uint4(0u, 0u, 0u, 0u);
    }
}

// causal_conv_transpose_1d (codec.rs:3505) from the GEMM over every tap, and
// the first residual unit's padded conv input: Y2 holds [T][K C] (stacked hi
// / lo rows); output row u = f s + k sums the taps that land on it in
// increasing f, then adds the bias (rows past T s are not produced) -> x;
// P[pad + u] = f16(snake(x, alpha)), P[0 .. pad) = 0.  Four channels per
// thread.
__global__ void col2im_pad_kernel(const float *Y2, const float *inv, int T, int K, int s, int C, const float *bias,
                                  float *x, const float *alpha, int pad, __half *P) {
    const int C4 = C / 4, N = K * C;
    const long long rows = (long long)T * s, total = (rows + pad) * C4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long prow = i / C4;
        const int c = (int)(i - prow * C4) * 4;
        if (prow < pad) {
            st_half4(P + prow * C + c, 0.f, 0.f, 0.f, 0.f);
            continue;
        }
        const int u = (int)(prow - pad);
        const int f_hi = min(u / s, T - 1);
        int f_lo = u - (K - 1);
        f_lo = f_lo <= 0 ? 0 : (f_lo + s - 1) / s;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int f = f_lo; f <= f_hi; ++f) {
            const size_t col = (size_t)(u - f * s) * C + c;
            const float4 a = ld4(Y2 + (size_t)f * N + col), b = ld4(Y2 + ((size_t)T + f) * N + col);
            const float w = inv[f];
            acc.x += (a.x + b.x) * w, acc.y += (a.y + b.y) * w, acc.z += (a.z + b.z) * w, acc.w += (a.w + b.w) * w;
        }
        const float4 bb = ld4(bias + c), al = ld4(alpha + c);
        acc.x += bb.x, acc.y += bb.y, acc.z += bb.z, acc.w += bb.w;
        *reinterpret_cast<float4 *>(x + (size_t)u * C + c) = acc;
        st_half4(P + prow * C + c, snake(acc.x, al.x), snake(acc.y, al.y), snake(acc.z, al.z), snake(acc.w, al.w));
    }
}

// Decoder tail (codec.rs:1978-1998) after the last residual unit: v = x (+ Z
// + zb when the unit's residual add is still pending), snake, the causal convolution 96 -> 1 (kernel 7,
// input rounded to f16) and tanh.  A block of 128 threads stages its 128
// samples' input rows (and the 6 before) in shared memory as f16 (the
// rounding the reference applies), rows padded to an odd number of words so
// that a warp's threads read different banks, and the weights as floats.
constexpr int kTailC = 96, kTailK = 7, kTailLd = kTailC + 2;  // halves per staged row
__global__ void __launch_bounds__(kTailTile) tail_kernel(const float *x, const float *Z, const float *zb, int T,
                                                         const float *alpha, const float *w, float bias, float *out) {
    __shared__ __half tile[(kTailTile + kTailK - 1) * kTailLd];
    __shared__ float ws[kTailK * kTailC];
    const int t0 = blockIdx.x * kTailTile;
    for (int i = threadIdx.x; i < kTailK * kTailC; i += kTailTile) ws[i] = w[i];
    constexpr int C4 = kTailC / 4, rows = kTailTile + kTailK - 1;
    for (int i = threadIdx.x; i < rows * C4; i += kTailTile) {
        const int r = i / C4, c = (i - r * C4) * 4, src = t0 + r - (kTailK - 1);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (src >= 0 && src < T) {
            const size_t o = (size_t)src * kTailC + c;
            const float4 a = ld4(x + o), al = ld4(alpha + c);
            const float4 z = Z ? ld4(Z + o) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 b = Z ? ld4(zb + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            v = make_float4(snake(a.x + z.x + b.x, al.x), snake(a.y + z.y + b.y, al.y), snake(a.z + z.z + b.z, al.z),
                            snake(a.w + z.w + b.w, al.w));
        }
        __half2 *dst = reinterpret_cast<__half2 *>(tile + r * kTailLd + c);
        dst[0] = __floats2half2_rn(v.x, v.y);
        dst[1] = __floats2half2_rn(v.z, v.w);
    }
    __syncthreads();
    const int t = t0 + threadIdx.x;
    if (t >= T) return;
    float acc = bias;
    for (int k = 0; k < kTailK; ++k) {
        const __half2 *row = reinterpret_cast<const __half2 *>(tile + (threadIdx.x + k) * kTailLd);
        const float *wk = ws + k * kTailC;
#pragma unroll 8
        for (int c = 0; c < kTailC / 2; ++c) {
            const float2 v = __half22float2(row[c]);
            acc += v.x * wk[2 * c] + v.y * wk[2 * c + 1];
        }
    }
    out[t] = tanhf(acc);
}

unsigned grid_for(size_t n, int threads = 256) {
    const size_t b = (n + threads - 1) / threads;
    return (unsigned)(b < 148 * 16 ? (b ? b : 1) : 148 * 16);
}

float h2f_host(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do {
                m <<= 1;
                ++e;
            } while (!(m & 0x400));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ff) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

}  // namespace

// ---------------------------------------------------------------- handle --

struct CodecUnit {
    const float *a0, *a1, *b0, *b1;
    const __half *w0, *w1;  // [C][k0 C] (tap-major columns), [C][k1 C]
    int k0, k1;
};
struct CodecBlock {
    const float *alpha, *bt;
    const __half *wt;  // [k C][C_in]: row (tap, out channel)
    int kernel;
    CodecUnit unit[3];
};
struct CodecLayer {
    const __half *wqkv, *wo, *w1, *w3, *w2;
    const float *an, *fn, *ga, *gf;
};
struct CodecEncBlock {
    CodecUnit unit[3];
    const float *alpha, *down_b;
    const __half *down_w;  // [Co][K C], K = 2 x stride: read as 2 taps of stride x C channels
    int stride;
};
struct CodecUpStage {
    const __half *wt, *pw1, *pw2;  // wt [2 x 1024][1024]
    const float *bt, *dw, *dwb, *lnw, *lnb, *pw1b, *pw2b, *gamma;
};

}  // namespace s2d

struct S2dCodec {
    int device = 0;
    std::string err;
    cudaStream_t stream = nullptr;
    cublasHandle_t blas = nullptr;
    uint8_t *arena = nullptr;
    size_t arena_bytes = 0;
    s2d::RvqArgs rvq{};
    s2d::CodecLayer layer[s2d::kLayers]{};
    const float *post_norm = nullptr, *rope_freq = nullptr;
    s2d::CodecUpStage up[s2d::kUpStages]{};
    const __half *entry_w = nullptr;
    const float *entry_b = nullptr;
    s2d::CodecBlock block[s2d::kBlocks]{};
    const float *tail_alpha = nullptr, *out_w = nullptr;
    float out_b = 0.f;
    // the reference-audio encoder (codec.rs:1056), when the file holds it
    bool has_encoder = false;
    const float *enc_entry_w = nullptr, *enc_entry_b = nullptr;  // [64][7], [64]
    s2d::CodecEncBlock enc[s2d::kBlocks]{};
    s2d::CodecLayer enc_layer[4]{};
    const float *enc_norm = nullptr, *enc_tail_alpha = nullptr, *enc_out_b = nullptr;
    const __half *enc_out_w = nullptr;  // [1024][3 x 1024]
    s2d::CodecUpStage down[s2d::kUpStages]{};  // wt: the stride-2 conv as [1024][2 x 1024]
    s2d::CodecLayer pre_layer[s2d::kLayers]{};
    const float *pre_norm = nullptr;
    s2d::VqArgs vq{};
    size_t enc_samples = 0;  // the encoder workspace's capacity in padded samples
    uint8_t *enc_ws = nullptr;
    size_t enc_ws_bytes = 0;
    float *eaudio = nullptr, *ex = nullptr, *ez = nullptr, *ez2 = nullptr;
    __half *eP = nullptr;
    int32_t *ecodes = nullptr;
    float *el2 = nullptr;
    // workspace, sized for `ws_frames` code frames
    uint32_t ws_frames = 0;
    uint8_t *ws = nullptr;
    size_t ws_bytes = 0;
    float *lat = nullptr, *x = nullptr, *x2 = nullptr, *qkv = nullptr, *att = nullptr, *act = nullptr;
    float *Y2 = nullptr, *Y2b = nullptr, *inv = nullptr, *Z = nullptr;
    __half *xs = nullptr, *P = nullptr, *A = nullptr;
    int32_t *codes = nullptr, *error = nullptr;  // error[0]: a code out of range; [1]: a tcgen05 wait gave up
    float *samples = nullptr;
    bool conv_tc = true;  // causal convolutions on the implicit-GEMM tcgen05 kernel (S2D_CODEC_TC)
    bool conv_one_cta = false;  // ... one CTA per SM with a deeper ring (S2D_CODEC_CONV_CTAS=1)
    bool attn_tiled = true;     // windowed attention over 32-frame tiles (S2D_CODEC_ATTN_TILED=0: per frame)
};

namespace s2d {
namespace {

int32_t cerr(S2dCodec *c, int32_t code, const std::string &m) {
    if (c) c->err = m;
    return code;
}

#define CCK(call)                                                                                    \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) return cerr(c, S2D_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// ---- loading ---------------------------------------------------------------

struct Loader {
    S2dCodec *c;
    const Gguf &g;
    std::vector<uint8_t> host;  // staged arena
    std::string err;
    struct Fix {
        size_t off;
        const void **dst;
    };
    std::vector<Fix> fixes;

    const GgufTensor *get(const std::string &name, std::vector<uint64_t> dims) {
        const GgufTensor *t = g.tensor(name);
        if (!t) {
            if (err.empty()) err = "tensor not found: " + name;
            return nullptr;
        }
        if (t->type != 1) {
            if (err.empty()) err = "expected F16 tensor " + name;
            return nullptr;
        }
        if (!dims.empty() && t->dims != dims) {
            if (err.empty()) {
                err = name + ": expected [";
                for (size_t i = 0; i < dims.size(); ++i) err += (i ? ", " : "") + std::to_string(dims[i]);
                err += "], got [";
                for (size_t i = 0; i < t->dims.size(); ++i) err += (i ? ", " : "") + std::to_string(t->dims[i]);
                err += "]";
            }
            return nullptr;
        }
        return t;
    }
    size_t alloc(size_t bytes) {
        const size_t off = (host.size() + 255) & ~(size_t)255;
        host.resize(off + bytes);
        return off;
    }
    const uint16_t *src(const GgufTensor *t) { return reinterpret_cast<const uint16_t *>(t->data); }
    // f16 tensor as stored
    void f16(const GgufTensor *t, const __half **dst) {
        if (!t) return;
        const size_t off = alloc(t->elements * 2);
        memcpy(host.data() + off, t->data, t->elements * 2);
        fixes.push_back({off, reinterpret_cast<const void **>(dst)});
    }
    // f16 tensor as floats
    void f32(const GgufTensor *t, const float **dst) {
        if (!t) return;
        const size_t off = alloc(t->elements * 4);
        float *o = reinterpret_cast<float *>(host.data() + off);
        const uint16_t *s = src(t);
        for (uint64_t i = 0; i < t->elements; ++i) o[i] = h2f_host(s[i]);
        fixes.push_back({off, reinterpret_cast<const void **>(dst)});
    }
    // causal conv weight ggml [k, in, out] (index tap + k (ic + in oc)) as
    // [out][k inp] with column tap * inp + ic, inp = in rounded up to 64 and
    // zeros in the columns past in
    void conv(const GgufTensor *t, int k, int in, int out, const __half **dst) {
        if (!t) return;
        const int inp = (in + 63) / 64 * 64;
        const size_t off = alloc((size_t)k * inp * out * 2);
        uint16_t *o = reinterpret_cast<uint16_t *>(host.data() + off);
        const uint16_t *s = src(t);
        for (int oc = 0; oc < out; ++oc)
            for (int ic = 0; ic < in; ++ic)
                for (int tap = 0; tap < k; ++tap)
                    o[(size_t)oc * k * inp + (size_t)tap * inp + ic] = s[tap + (size_t)k * (ic + (size_t)in * oc)];
        fixes.push_back({off, reinterpret_cast<const void **>(dst)});
    }
    // transposed conv weight ggml [k, out, in] (index tap + k (oc + out ic))
    // as [k out][in] with row tap * out + oc
    void convt(const GgufTensor *t, int k, int out, int in, const __half **dst) {
        if (!t) return;
        const size_t off = alloc((size_t)k * in * out * 2);
        uint16_t *o = reinterpret_cast<uint16_t *>(host.data() + off);
        const uint16_t *s = src(t);
        for (int ic = 0; ic < in; ++ic)
            for (int oc = 0; oc < out; ++oc)
                for (int tap = 0; tap < k; ++tap)
                    o[((size_t)tap * out + oc) * in + ic] = s[tap + (size_t)k * (oc + (size_t)out * ic)];
        fixes.push_back({off, reinterpret_cast<const void **>(dst)});
    }
    void floats(const std::vector<float> &v, const float **dst) {
        const size_t off = alloc(v.size() * 4);
        memcpy(host.data() + off, v.data(), v.size() * 4);
        fixes.push_back({off, reinterpret_cast<const void **>(dst)});
    }
};

int32_t load(S2dCodec *c, const Gguf &g) {
    Loader L{c, g, {}, {}, {}};
    using D = std::vector<uint64_t>;
    const uint64_t H = kHid;
    // quantizers (codec.rs:2356-2413: in_proj is read and checked there too)
    for (int cb = 0; cb < kBooks; ++cb) {
        const std::string p = cb == 0 ? "quantizer.semantic_quantizer.quantizers.0"
                                      : "quantizer.quantizer.quantizers." + std::to_string(cb - 1);
        const uint64_t n = cb == 0 ? kSemBook : kResBook;
        L.get(p + ".in_proj.weight", D{1, H, kProj});
        L.get(p + ".in_proj.bias", D{kProj});
        L.f16(L.get(p + ".codebook.weight", D{kProj, n}), &c->rvq.book[cb]);
        L.f16(L.get(p + ".out_proj.weight", D{1, kProj, H}), &c->rvq.oproj[cb]);
        L.f16(L.get(p + ".out_proj.bias", D{H}), &c->rvq.obias[cb]);
        c->rvq.size[cb] = (int)n;
    }
    // post module (codec.rs:502-540, 836-910)
    for (int l = 0; l < kLayers; ++l) {
        const std::string p = "quantizer.post_module.layers." + std::to_string(l);
        CodecLayer &y = c->layer[l];
        L.f16(L.get(p + ".attention.wqkv.weight", D{H, 3 * H}), &y.wqkv);
        L.f16(L.get(p + ".attention.wo.weight", D{H, H}), &y.wo);
        L.f32(L.get(p + ".attention_norm.weight", D{H}), &y.an);
        L.f32(L.get(p + ".ffn_norm.weight", D{H}), &y.fn);
        L.f16(L.get(p + ".feed_forward.w1.weight", D{H, kFfn}), &y.w1);
        L.f16(L.get(p + ".feed_forward.w3.weight", D{H, kFfn}), &y.w3);
        L.f16(L.get(p + ".feed_forward.w2.weight", D{kFfn, H}), &y.w2);
        L.f32(L.get(p + ".attention_layer_scale.gamma", D{H}), &y.ga);
        L.f32(L.get(p + ".ffn_layer_scale.gamma", D{H}), &y.gf);
    }
    L.f32(L.get("quantizer.post_module.norm.weight", D{H}), &c->post_norm);
    std::vector<float> freq(kHd / 2);
    for (int i = 0; i < kHd / 2; ++i) freq[i] = powf(kRopeBase, (float)(2 * i) / (float)kHd);
    L.floats(freq, &c->rope_freq);
    // upsample (codec.rs:736-820)
    for (int s = 0; s < kUpStages; ++s) {
        const std::string p = "quantizer.upsample." + std::to_string(s);
        CodecUpStage &u = c->up[s];
        L.convt(L.get(p + ".0.conv.weight", D{kUp, H, H}), kUp, kHid, kHid, &u.wt);
        L.f32(L.get(p + ".0.conv.bias", D{H}), &u.bt);
        L.f32(L.get(p + ".1.gamma", D{H}), &u.gamma);
        // depthwise [7, 1, C] (index tap + 7 c) is already [c][tap]
        L.f32(L.get(p + ".1.dwconv.conv.weight", D{kDw, 1, H}), &u.dw);
        L.f32(L.get(p + ".1.dwconv.conv.bias", D{H}), &u.dwb);
        L.f32(L.get(p + ".1.norm.weight", D{H}), &u.lnw);
        L.f32(L.get(p + ".1.norm.bias", D{H}), &u.lnb);
        L.f16(L.get(p + ".1.pwconv1.weight", D{H, kExp}), &u.pw1);
        L.f32(L.get(p + ".1.pwconv1.bias", D{kExp}), &u.pw1b);
        L.f16(L.get(p + ".1.pwconv2.weight", D{kExp, H}), &u.pw2);
        L.f32(L.get(p + ".1.pwconv2.bias", D{H}), &u.pw2b);
    }
    // decoder (codec.rs:1626-1679; block shapes as the forward pass reads them)
    L.conv(L.get("decoder.model.0.conv.weight", D{7, H, kEntry}), 7, kHid, kEntry, &c->entry_w);
    L.f32(L.get("decoder.model.0.conv.bias", D{kEntry}), &c->entry_b);
    int cin = kEntry;
    for (int b = 0; b < kBlocks; ++b) {
        const std::string p = "decoder.model." + std::to_string(b + 1);
        const int C = kChan[b];
        CodecBlock &k = c->block[b];
        L.f32(L.get(p + ".block.0.alpha", D{1, (uint64_t)cin, 1}), &k.alpha);
        const GgufTensor *wt = L.get(p + ".block.1.conv.weight", {});
        if (wt && (wt->dims.size() != 3 || wt->dims[1] != (uint64_t)C || wt->dims[2] != (uint64_t)cin ||
                   wt->dims[0] < 1 || wt->dims[0] > 64)) {
            if (L.err.empty()) L.err = p + ".block.1.conv.weight: expected [k, " + std::to_string(C) + ", " +
                                       std::to_string(cin) + "]";
            wt = nullptr;
        }
        k.kernel = wt ? (int)wt->dims[0] : 0;
        L.convt(wt, k.kernel, C, cin, &k.wt);
        L.f32(L.get(p + ".block.1.conv.bias", D{(uint64_t)C}), &k.bt);
        for (int u = 0; u < 3; ++u) {
            const std::string q = p + ".block." + std::to_string(u + 2);
            CodecUnit &n = k.unit[u];
            L.f32(L.get(q + ".block.0.alpha", D{1, (uint64_t)C, 1}), &n.a0);
            L.f32(L.get(q + ".block.2.alpha", D{1, (uint64_t)C, 1}), &n.a1);
            for (int j = 0; j < 2; ++j) {
                const GgufTensor *w = L.get(q + (j ? ".block.3.conv.weight" : ".block.1.conv.weight"), {});
                if (w && (w->dims.size() != 3 || w->dims[1] != (uint64_t)C || w->dims[2] != (uint64_t)C ||
                          w->dims[0] < 1 || w->dims[0] > 16)) {
                    if (L.err.empty()) L.err = q + ": conv weight expected [k, C, C]";
                    w = nullptr;
                }
                const int kk = w ? (int)w->dims[0] : 0;
                (j ? n.k1 : n.k0) = kk;
                L.conv(w, kk, C, C, j ? &n.w1 : &n.w0);
            }
            L.f32(L.get(q + ".block.1.conv.bias", D{(uint64_t)C}), &n.b0);
            L.f32(L.get(q + ".block.3.conv.bias", D{(uint64_t)C}), &n.b1);
        }
        cin = C;
    }
    L.f32(L.get("decoder.model.5.alpha", D{1, 96, 1}), &c->tail_alpha);
    const GgufTensor *ow = L.get("decoder.model.6.conv.weight", D{7, 96, 1});
    if (ow) {  // [7, 96, 1]: index tap + 7 ic, kept as [tap][ic]
        std::vector<float> w(7 * 96);
        for (int tap = 0; tap < 7; ++tap)
            for (int ic = 0; ic < 96; ++ic) w[tap * 96 + ic] = h2f_host(L.src(ow)[tap + 7 * ic]);
        L.floats(w, &c->out_w);
    }
    if (const GgufTensor *ob = L.get("decoder.model.6.conv.bias", D{1})) c->out_b = h2f_host(L.src(ob)[0]);
    // the reference-audio encoder and the quantizer's encode side (codec.rs:1519-1584,
    // 546-680, 455-494, and in_proj of 2356-2413), loaded when the file has them
    c->has_encoder = g.tensor("encoder.block.0.conv.weight") != nullptr;
    if (c->has_encoder && L.err.empty()) {
        L.f32(L.get("encoder.block.0.conv.weight", D{7, 1, 64}), &c->enc_entry_w);  // index tap + 7 c
        L.f32(L.get("encoder.block.0.conv.bias", D{64}), &c->enc_entry_b);
        constexpr int kEncRates[kBlocks] = {2, 4, 8, 8};
        constexpr int kEncChan[kBlocks + 1] = {64, 128, 256, 512, 1024};
        for (int b = 0; b < kBlocks; ++b) {
            const std::string p = "encoder.block." + std::to_string(b + 1) + ".block";
            const int C = kEncChan[b], Co = kEncChan[b + 1], st = kEncRates[b];
            CodecEncBlock &k = c->enc[b];
            k.stride = st;
            for (int u = 0; u < 3; ++u) {
                const std::string q = p + "." + std::to_string(u);
                CodecUnit &n = k.unit[u];
                n.k0 = 7, n.k1 = 1;
                L.f32(L.get(q + ".block.0.alpha", D{1, (uint64_t)C, 1}), &n.a0);
                L.conv(L.get(q + ".block.1.conv.weight", D{7, (uint64_t)C, (uint64_t)C}), 7, C, C, &n.w0);
                L.f32(L.get(q + ".block.1.conv.bias", D{(uint64_t)C}), &n.b0);
                L.f32(L.get(q + ".block.2.alpha", D{1, (uint64_t)C, 1}), &n.a1);
                L.conv(L.get(q + ".block.3.conv.weight", D{1, (uint64_t)C, (uint64_t)C}), 1, C, C, &n.w1);
                L.f32(L.get(q + ".block.3.conv.bias", D{(uint64_t)C}), &n.b1);
            }
            L.f32(L.get(p + ".3.alpha", D{1, (uint64_t)C, 1}), &k.alpha);
            // kernel 2 x stride (codec.rs:40): [oc][tap C + ic] is also [oc][j (stride C) + r C + ic]
            L.conv(L.get(p + ".4.conv.weight", D{(uint64_t)(2 * st), (uint64_t)C, (uint64_t)Co}), 2 * st, C, Co,
                   &k.down_w);
            L.f32(L.get(p + ".4.conv.bias", D{(uint64_t)Co}), &k.down_b);
        }
        auto layers = [&](const std::string &module, CodecLayer *out, int n) {
            for (int l = 0; l < n; ++l) {
                const std::string q = module + ".layers." + std::to_string(l);
                CodecLayer &y = out[l];
                L.f16(L.get(q + ".attention.wqkv.weight", D{H, 3 * H}), &y.wqkv);
                L.f16(L.get(q + ".attention.wo.weight", D{H, H}), &y.wo);
                L.f32(L.get(q + ".attention_norm.weight", D{H}), &y.an);
                L.f32(L.get(q + ".ffn_norm.weight", D{H}), &y.fn);
                L.f16(L.get(q + ".feed_forward.w1.weight", D{H, kFfn}), &y.w1);
                L.f16(L.get(q + ".feed_forward.w3.weight", D{H, kFfn}), &y.w3);
                L.f16(L.get(q + ".feed_forward.w2.weight", D{kFfn, H}), &y.w2);
                L.f32(L.get(q + ".attention_layer_scale.gamma", D{H}), &y.ga);
                L.f32(L.get(q + ".ffn_layer_scale.gamma", D{H}), &y.gf);
            }
        };
        layers("encoder.block.4.block.5", c->enc_layer, 4);
        L.f32(L.get("encoder.block.4.block.5.norm.weight", D{H}), &c->enc_norm);
        L.f32(L.get("encoder.block.5.alpha", D{1, H, 1}), &c->enc_tail_alpha);
        L.conv(L.get("encoder.block.6.conv.weight", D{3, H, H}), 3, kHid, kHid, &c->enc_out_w);
        L.f32(L.get("encoder.block.6.conv.bias", D{H}), &c->enc_out_b);
        for (int st = 0; st < kUpStages; ++st) {
            const std::string p = "quantizer.downsample." + std::to_string(st);
            CodecUpStage &u = c->down[st];
            L.conv(L.get(p + ".0.conv.weight", D{2, H, H}), 2, kHid, kHid, &u.wt);
            L.f32(L.get(p + ".0.conv.bias", D{H}), &u.bt);
            L.f32(L.get(p + ".1.gamma", D{H}), &u.gamma);
            L.f32(L.get(p + ".1.dwconv.conv.weight", D{kDw, 1, H}), &u.dw);
            L.f32(L.get(p + ".1.dwconv.conv.bias", D{H}), &u.dwb);
            L.f32(L.get(p + ".1.norm.weight", D{H}), &u.lnw);
            L.f32(L.get(p + ".1.norm.bias", D{H}), &u.lnb);
            L.f16(L.get(p + ".1.pwconv1.weight", D{H, kExp}), &u.pw1);
            L.f32(L.get(p + ".1.pwconv1.bias", D{kExp}), &u.pw1b);
            L.f16(L.get(p + ".1.pwconv2.weight", D{kExp, H}), &u.pw2);
            L.f32(L.get(p + ".1.pwconv2.bias", D{H}), &u.pw2b);
        }
        layers("quantizer.pre_module", c->pre_layer, kLayers);
        L.f32(L.get("quantizer.pre_module.norm.weight", D{H}), &c->pre_norm);
        for (int cb = 0; cb < kBooks; ++cb) {
            const std::string p = cb == 0 ? "quantizer.semantic_quantizer.quantizers.0"
                                          : "quantizer.quantizer.quantizers." + std::to_string(cb - 1);
            L.f16(L.get(p + ".in_proj.weight", D{1, H, kProj}), &c->vq.in_w[cb]);  // [8][1024]
            L.f16(L.get(p + ".in_proj.bias", D{kProj}), &c->vq.in_b[cb]);
        }
    }
    if (!L.err.empty()) return cerr(c, S2D_EINVAL, "codec weights: " + L.err);

    CCK(cudaMalloc(&c->arena, L.host.size()));
    c->arena_bytes = L.host.size();
    CCK(cudaMemcpy(c->arena, L.host.data(), L.host.size(), cudaMemcpyHostToDevice));
    for (const auto &f : L.fixes) *f.dst = c->arena + f.off;
    return S2D_OK;
}

// ---- workspace ---------------------------------------------------------------

int32_t ensure_ws(S2dCodec *c, uint32_t frames) {
    if (frames <= c->ws_frames) return S2D_OK;
    const size_t T = frames, L = 4 * T;  // code frames, latent frames
    // largest row counts x widths over the stages (floats unless noted)
    size_t xf = std::max(L * kHid, (size_t)L * kEntry);
    size_t yf = std::max(2 * T * 3 * (size_t)kHid, 2 * T * (size_t)kFfn);
    yf = std::max(yf, 2 * L * (size_t)kExp);  // pwconv1 of the second stage: 2 x 4T rows of 4096
    size_t pf = (L + 6) * (size_t)kHid, af = L * 7 * (size_t)kHid, xsf = 2 * L * (size_t)kExp;
    size_t zf = L * (size_t)kEntry;
    size_t rows = L, cin = kEntry;
    for (int b = 0; b < kBlocks; ++b) {
        const size_t C = kChan[b], K = c->block[b].kernel, out = rows * kRates[b];
        yf = std::max(yf, 2 * rows * K * C);
        xsf = std::max(xsf, 2 * rows * cin);
        xf = std::max(xf, out * C);
        for (int u = 0; u < 3; ++u) {
            const int d = u == 0 ? 1 : u == 1 ? 3 : 9;
            const size_t k0 = c->block[b].unit[u].k0, k1 = c->block[b].unit[u].k1;
            pf = std::max(pf, (out + (k0 - 1) * d + k1) * C);
            af = std::max(af, out * std::max(k0, k1) * ((C + 63) / 64 * 64));
        }
        zf = std::max(zf, out * C);
        rows = out, cin = C;
    }
    if (c->conv_tc) af = 8;  // the implicit-GEMM convolutions need no im2col rows
    const size_t samples = rows;
    struct Part {
        void **p;
        size_t bytes;
    } parts[] = {
        {(void **)&c->lat, T * kHid * 4},
        {(void **)&c->x, xf * 4},
        {(void **)&c->x2, xf * 4},
        {(void **)&c->qkv, L * 3 * kHid * 4},
        {(void **)&c->att, L * kHid * 4},
        {(void **)&c->act, L * kExp * 4},
        {(void **)&c->Y2, yf * 4},
        {(void **)&c->Y2b, 2 * L * (size_t)kFfn * 4},
        {(void **)&c->inv, std::max(2 * rows, (size_t)L) * 4},
        {(void **)&c->Z, zf * 4},
        {(void **)&c->xs, xsf * 2},
        {(void **)&c->P, pf * 2},
        {(void **)&c->A, af * 2},
        {(void **)&c->codes, T * kBooks * 4},
        {(void **)&c->samples, samples * 4},
        {(void **)&c->error, 8},
    };
    size_t total = 0;
    for (auto &p : parts) total += (p.bytes + 255) & ~(size_t)255;
    if (c->ws) cudaFree(c->ws);
    c->ws = nullptr, c->ws_frames = 0, c->ws_bytes = 0;
    CCK(cudaMalloc(&c->ws, total));
    size_t off = 0;
    for (auto &p : parts) {
        *p.p = c->ws + off;
        off += (p.bytes + 255) & ~(size_t)255;
    }
    CCK(cudaMemset(c->error, 0, 8));
    c->ws_frames = frames, c->ws_bytes = total;
    return S2D_OK;
}

// ---- stages ------------------------------------------------------------------

// C [M][N] = A [M][K] . W [N][K]^T, f16 in, f32 accumulate and out; long
// row counts go in slices of 2^20 rows so that no operand passes 2^31 elements.
int32_t gemm(S2dCodec *c, const __half *A, const __half *W, int M, int N, int K, float *Cm) {
    const float one = 1.f, zero = 0.f;
    constexpr int kSlice = 1 << 20;
    for (int m0 = 0; m0 < M; m0 += kSlice) {
        const int m = std::min(kSlice, M - m0);
        const cublasStatus_t st =
            cublasGemmEx(c->blas, CUBLAS_OP_T, CUBLAS_OP_N, N, m, K, &one, W, CUDA_R_16F, K, A + (size_t)m0 * K,
                         CUDA_R_16F, K, &zero, Cm + (size_t)m0 * N, CUDA_R_32F, N, CUBLAS_COMPUTE_32F,
                         CUBLAS_GEMM_DEFAULT);
        if (st != CUBLAS_STATUS_SUCCESS)
            return cerr(c, S2D_ECUDA, "cublasGemmEx failed (" + std::to_string((int)st) + ")");
    }
    return S2D_OK;
}

// Y2 [2T][N] = the hi / lo split of x [T][K] (RMSNorm with norm_w first when
// given) times W [N][K]^T.
int32_t split_gemm(S2dCodec *c, const float *x, int T, int K, const float *norm_w, const __half *W, int N,
                   float *Y2) {
    CCK(launch_split_rows(x, K, T, K, norm_w, kNormEps, c->xs, c->inv, nullptr, c->stream));
    return gemm(c, c->xs, W, 2 * T, N, K, Y2);
}

int32_t epilogue(S2dCodec *c, int epi, const float *Y2, const float *Y2b, int T, int N, const float *bias, int nb,
                 const float *gamma, const float *r, float *y) {
    epilogue_kernel<<<grid_for((size_t)T * N), 256, 0, c->stream>>>(epi, Y2, Y2b, c->inv, T, N, bias, nb, gamma, r, y);
    CCK(cudaGetLastError());
    return S2D_OK;
}

// n codec transformer layers (codec.rs:3229, attention window `window`) on
// x [T][1024], in place; the module's final RMSNorm lands in `out`
// (forward_codec_post_module, codec.rs:986; the pre module, codec.rs:1038;
// the encoder's last block, codec.rs:1836).
int32_t transformer(S2dCodec *c, const CodecLayer *layers, int n, int window, float *x, int T, const float *norm,
                    float *out) {
    int32_t rc;
    for (int l = 0; l < n; ++l) {
        const CodecLayer &y = layers[l];
        if ((rc = split_gemm(c, x, T, kHid, y.an, y.wqkv, 3 * kHid, c->Y2))) return rc;
        qkv_rope_kernel<<<T, 256, 0, c->stream>>>(c->Y2, c->inv, T, c->rope_freq, c->qkv);
        if (c->attn_tiled)
            window_attn_tiled_kernel<<<dim3((T + kWaFrames - 1) / kWaFrames, kHeads), 256, 0, c->stream>>>(
                c->qkv, T, window, c->att);
        else if (window == 512)
            window_attn_kernel<512><<<dim3(T, kHeads), kWin, 0, c->stream>>>(c->qkv, T, c->att);
        else
            window_attn_kernel<kWin><<<dim3(T, kHeads), kWin, 0, c->stream>>>(c->qkv, T, c->att);
        CCK(cudaGetLastError());
        if ((rc = split_gemm(c, c->att, T, kHid, nullptr, y.wo, kHid, c->Y2))) return rc;
        if ((rc = epilogue(c, CE_SCALE_RESID, c->Y2, nullptr, T, kHid, nullptr, 1, y.ga, x, x))) return rc;
        CCK(launch_split_rows(x, kHid, T, kHid, y.fn, kNormEps, c->xs, c->inv, nullptr, c->stream));
        if ((rc = gemm(c, c->xs, y.w1, 2 * T, kFfn, kHid, c->Y2))) return rc;
        if ((rc = gemm(c, c->xs, y.w3, 2 * T, kFfn, kHid, c->Y2b))) return rc;
        if ((rc = epilogue(c, CE_SWIGLU, c->Y2, c->Y2b, T, kFfn, nullptr, 1, nullptr, nullptr, c->act))) return rc;
        if ((rc = split_gemm(c, c->act, T, kFfn, nullptr, y.w2, kHid, c->Y2))) return rc;
        if ((rc = epilogue(c, CE_SCALE_RESID, c->Y2, nullptr, T, kHid, nullptr, 1, y.gf, x, x))) return rc;
    }
    // the final RMSNorm: split_rows writes the normalised rows to `out`
    CCK(launch_split_rows(x, kHid, T, kHid, norm, kNormEps, c->xs, c->inv, out, c->stream));
    return S2D_OK;
}

int32_t post_module(S2dCodec *c, float *x, int T, float *out) {
    return transformer(c, c->layer, kLayers, kWin, x, T, c->post_norm, out);
}

// The ConvNeXt block of an upsample or downsample stage (codec.rs:3438,
// 3392) on y [T][1024], in place.
int32_t convnext(S2dCodec *c, const CodecUpStage &u, float *y, int T) {
    int32_t rc;
    dwconv_ln_kernel<<<T, 256, 0, c->stream>>>(y, T, u.dw, u.dwb, u.lnw, u.lnb, c->att);
    CCK(cudaGetLastError());
    if ((rc = split_gemm(c, c->att, T, kHid, nullptr, u.pw1, kExp, c->Y2))) return rc;
    if ((rc = epilogue(c, CE_GELU, c->Y2, nullptr, T, kExp, u.pw1b, kExp, nullptr, nullptr, c->act))) return rc;
    if ((rc = split_gemm(c, c->act, T, kExp, nullptr, u.pw2, kHid, c->Y2))) return rc;
    return epilogue(c, CE_SCALE_RESID, c->Y2, nullptr, T, kHid, u.pw2b, kHid, u.gamma, y, y);
}

// One upsample stage (codec.rs:3338): x [T][1024] -> y [2T][1024].
int32_t upsample_stage(S2dCodec *c, const CodecUpStage &u, const float *x, int T, float *y) {
    int32_t rc;
    const int T2 = 2 * T;
    // transposed conv, kernel 2 = stride: output row 2f + k is GEMM row f's
    // columns [k 1024, (k + 1) 1024), so [T][2048] is already [2T][1024]
    if ((rc = split_gemm(c, x, T, kHid, nullptr, u.wt, kUp * kHid, c->Y2))) return rc;
    if ((rc = epilogue(c, CE_STORE, c->Y2, nullptr, T, kUp * kHid, u.bt, kHid, nullptr, nullptr, y))) return rc;
    return convnext(c, u, y, T2);
}

// The GEMM of a stride-1 causal convolution (codec.rs:2212) whose padded f16
// input P ([(K - 1) d + T][C]) is in place, into Z [T][N]: the implicit-GEMM
// tcgen05 kernel, or (S2D_CODEC_TC=0) im2col + cuBLAS.  W is [N][K Cp].
int32_t conv_gemm(S2dCodec *c, int T, int C, const __half *W, int K, int d, int N, float *Z,
                  const __half *P = nullptr) {
    const int Cp = (C + 63) / 64 * 64;
    if (!P) P = c->P;
    if (c->conv_tc) {
        CodecConv cv;
        cv.P = P, cv.W = W, cv.T = T, cv.C = C, cv.N = N, cv.taps = K, cv.d = d, cv.cpb = Cp / 64, cv.Z = Z;
        cv.error = c->error + 1, cv.one_cta = c->conv_one_cta;
        CCK(launch_codec_conv(cv, c->stream));
        return S2D_OK;
    }
    const __half *A = P;
    if (K > 1 || Cp != C) {
        if (P != c->P) return cerr(c, S2D_EINVAL, "the im2col route covers the decoder only");
        im2col_kernel<<<grid_for((size_t)T * K * Cp / 8), 256, 0, c->stream>>>(P, T, C, Cp, K, d, c->A);
        CCK(cudaGetLastError());
        A = c->A;
    }
    return gemm(c, A, W, T, N, K * Cp, Z);
}

// P = the padded f16 input of a convolution: f16(snake(x + bias)).
int32_t pad_input(S2dCodec *c, const float *x, int T, int C, int pad, const float *bias, const float *alpha,
                  __half *P = nullptr) {
    pad_f16_kernel<<<grid_for((size_t)(T + pad) * C / 4), 256, 0, c->stream>>>(x, T, C, pad, bias, alpha,
                                                                                P ? P : c->P);
    CCK(cudaGetLastError());
    return S2D_OK;
}

// xs / inv = the split of snake(x (+ Z + zb) (+ bias)), rows of C channels.
int32_t snake_split(S2dCodec *c, const float *x, const float *Z, const float *zb, const float *bias,
                    const float *alpha, int T, int C) {
    const unsigned g = (unsigned)((T + 7) / 8);
    switch (C) {
    case 1536: snake_split_kernel<24><<<g, 256, 0, c->stream>>>(x, Z, zb, bias, alpha, T, c->xs, c->inv); break;
    case 768: snake_split_kernel<12><<<g, 256, 0, c->stream>>>(x, Z, zb, bias, alpha, T, c->xs, c->inv); break;
    case 384: snake_split_kernel<6><<<g, 256, 0, c->stream>>>(x, Z, zb, bias, alpha, T, c->xs, c->inv); break;
    case 192: snake_split_kernel<3><<<g, 256, 0, c->stream>>>(x, Z, zb, bias, alpha, T, c->xs, c->inv); break;
    default: return cerr(c, S2D_EINVAL, "snake_split: unsupported channel count " + std::to_string(C));
    }
    CCK(cudaGetLastError());
    return S2D_OK;
}

// forward_codec_decoder (codec.rs:1941): hidden [L][1024] -> samples [512 L].
// Elementwise steps ride on the kernels around the GEMMs: the entry conv's
// bias and each block's snake go into the split of the transposed conv's
// input, the transposed conv's col2im writes the first unit's conv input,
// a unit's conv0 bias and snake1 go into conv1's input, and each residual add
// writes the next unit's conv input (or the next block's split, or the tail).
int32_t decoder(S2dCodec *c, const float *hidden, int L, float *samples) {
    int32_t rc;
    // entry conv 1024 -> 1536 (kernel 7), bias left for the split below
    if ((rc = pad_input(c, hidden, L, kHid, 6, nullptr, nullptr))) return rc;
    if ((rc = conv_gemm(c, L, kHid, c->entry_w, 7, 1, kEntry, c->Z))) return rc;
    if ((rc = snake_split(c, c->Z, nullptr, nullptr, c->entry_b, c->block[0].alpha, L, kEntry))) return rc;
    int rows = L;
    float *x = c->x;
    for (int b = 0; b < kBlocks; ++b) {
        const CodecBlock &k = c->block[b];
        const int cin = b == 0 ? kEntry : kChan[b - 1], C = kChan[b], s = kRates[b], out = rows * s;
        // the transposed conv over every tap, col2im + bias -> x, unit 0's conv input -> P
        if ((rc = gemm(c, c->xs, k.wt, 2 * rows, k.kernel * C, cin, c->Y2))) return rc;
        col2im_pad_kernel<<<grid_for(((size_t)out + (k.unit[0].k0 - 1)) * C / 4), 256, 0, c->stream>>>(
            c->Y2, c->inv, rows, k.kernel, s, C, k.bt, x, k.unit[0].a0, k.unit[0].k0 - 1, c->P);
        CCK(cudaGetLastError());
        // residual units, dilations 1, 3, 9 (codec.rs:2040-2042)
        for (int u = 0; u < 3; ++u) {
            const CodecUnit &n = k.unit[u];
            const int d = u == 0 ? 1 : u == 1 ? 3 : 9;
            if ((rc = conv_gemm(c, out, C, n.w0, n.k0, d, C, c->Z))) return rc;
            if ((rc = pad_input(c, c->Z, out, C, n.k1 - 1, n.b0, n.a1))) return rc;
            if ((rc = conv_gemm(c, out, C, n.w1, n.k1, 1, C, c->x2))) return rc;
            if (u < 2) {
                const CodecUnit &nx = k.unit[u + 1];
                const int pad = (nx.k0 - 1) * (u == 0 ? 3 : 9);
                resid_pad_kernel<<<grid_for(((size_t)out + pad) * C / 4), 256, 0, c->stream>>>(x, c->x2, n.b1, out, C,
                                                                                              nx.a0, pad, c->P, false);
                CCK(cudaGetLastError());
            } else if (b + 1 < kBlocks) {
                if ((rc = snake_split(c, x, c->x2, n.b1, nullptr, c->block[b + 1].alpha, out, C))) return rc;
            } else {
                tail_kernel<<<(out + kTailTile - 1) / kTailTile, kTailTile, 0, c->stream>>>(
                    x, c->x2, n.b1, out, c->tail_alpha, c->out_w, c->out_b, samples);
                CCK(cudaGetLastError());
            }
        }
        rows = out;
    }
    return S2D_OK;
}

// ---- reference-audio encoder (codec.rs:1056) --------------------------------

constexpr int kEncChan[kBlocks + 1] = {64, 128, 256, 512, 1024};
constexpr int kFrameLength = 2048;  // codec.rs:46

int32_t ensure_enc_ws(S2dCodec *c, size_t S) {
    if (S <= c->enc_samples) return S2D_OK;
    const size_t frames = S / kFrameLength;
    struct Part {
        void **p;
        size_t bytes;
    } parts[] = {
        {(void **)&c->eaudio, S * 4},
        {(void **)&c->ex, S * 64 * 4},
        {(void **)&c->ez, S * 64 * 4},
        {(void **)&c->ez2, S * 64 * 4},
        {(void **)&c->eP, (S * 64 + 64 * 1024) * 2},
        {(void **)&c->ecodes, frames * kBooks * 4},
        {(void **)&c->el2, frames * 4},
    };
    size_t total = 0;
    for (auto &p : parts) total += (p.bytes + 255) & ~(size_t)255;
    if (c->enc_ws) cudaFree(c->enc_ws);
    c->enc_ws = nullptr, c->enc_samples = 0, c->enc_ws_bytes = 0;
    CCK(cudaMalloc(&c->enc_ws, total));
    size_t off = 0;
    for (auto &p : parts) {
        *p.p = c->enc_ws + off;
        off += (p.bytes + 255) & ~(size_t)255;
    }
    c->enc_samples = S, c->enc_ws_bytes = total;
    return S2D_OK;
}

int32_t resid_pad(S2dCodec *c, float *x, const float *Z, const float *bias, int T, int C, const float *alpha, int pad,
                  __half *P, bool assign) {
    resid_pad_kernel<<<grid_for(((size_t)T + pad) * C / 4), 256, 0, c->stream>>>(x, Z, bias, T, C, alpha, pad, P,
                                                                                  assign);
    CCK(cudaGetLastError());
    return S2D_OK;
}

// forward_codec_encoder_frontend (codec.rs:1104) on c->eaudio [S] (S a
// multiple of 2,048, zero padded): the output conv's rows without their bias
// (c->enc_out_b) in c->ez [S / 512][1024].
int32_t encoder_frontend(S2dCodec *c, int S) {
    int32_t rc;
    enc_entry_kernel<<<grid_for((size_t)S * 64), 256, 0, c->stream>>>(c->eaudio, S, c->enc_entry_w, c->enc_entry_b,
                                                                      c->ex);
    CCK(cudaGetLastError());
    if ((rc = pad_input(c, c->ex, S, 64, 6, nullptr, c->enc[0].unit[0].a0, c->eP))) return rc;
    int rows = S;
    for (int b = 0; b < kBlocks; ++b) {
        const CodecEncBlock &k = c->enc[b];
        const int C = kEncChan[b], Co = kEncChan[b + 1], st = k.stride;
        // residual units, dilations 1, 3, 9 (codec.rs:1749-1790); the last
        // one's residual add writes the down conv's input: snake, then
        // `stride` zero rows of left padding (kernel 2 x stride - stride)
        for (int u = 0; u < 3; ++u) {
            const CodecUnit &n = k.unit[u];
            const int d = u == 0 ? 1 : u == 1 ? 3 : 9;
            if ((rc = conv_gemm(c, rows, C, n.w0, n.k0, d, C, c->ez, c->eP))) return rc;
            if ((rc = pad_input(c, c->ez, rows, C, n.k1 - 1, n.b0, n.a1, c->eP))) return rc;
            if ((rc = conv_gemm(c, rows, C, n.w1, n.k1, 1, C, c->ez2, c->eP))) return rc;
            if (u < 2) {
                const CodecUnit &nx = k.unit[u + 1];
                rc = resid_pad(c, c->ex, c->ez2, n.b1, rows, C, nx.a0, (nx.k0 - 1) * (u == 0 ? 3 : 9), c->eP, false);
            } else {
                rc = resid_pad(c, c->ex, c->ez2, n.b1, rows, C, k.alpha, st, c->eP, false);
            }
            if (rc) return rc;
        }
        // the strided down conv (codec.rs:1808-1820): rows of `stride` x C
        // channels, two taps
        if ((rc = conv_gemm(c, rows / st, st * C, k.down_w, 2, 1, Co, c->ez, c->eP))) return rc;
        rows /= st;
        if (b + 1 < kBlocks)
            rc = resid_pad(c, c->ex, c->ez, k.down_b, rows, Co, c->enc[b + 1].unit[0].a0, 6, c->eP, true);
        else
            rc = resid_pad(c, c->ex, c->ez, k.down_b, rows, Co, nullptr, 0, nullptr, true);
        if (rc) return rc;
    }
    // the last block's 4 transformer layers (window 512) and norm, the tail
    // snake and the output conv (kernel 3)
    if ((rc = transformer(c, c->enc_layer, 4, 512, c->ex, rows, c->enc_norm, c->ez2))) return rc;
    if ((rc = pad_input(c, c->ez2, rows, kHid, 2, nullptr, c->enc_tail_alpha, c->eP))) return rc;
    return conv_gemm(c, rows, kHid, c->enc_out_w, 3, 1, kHid, c->ez, c->eP);
}

// forward_codec_quantizer_encode_stage (codec.rs:1020): h [L][1024] (+ hb)
// -> two downsample stages (stride-2 conv + ConvNeXt) -> pre module -> out
// [L / 4][1024].  L a multiple of 4.
int32_t quantizer_encode(S2dCodec *c, const float *h, const float *hb, int L, float *out) {
    int32_t rc;
    const float *in = h, *in_b = hb;
    float *y[2] = {c->x, c->x2};
    int rows = L;
    for (int st = 0; st < kUpStages; ++st) {
        // kernel 2 = stride 2, no padding: one tap over rows of 2 x 1024
        if ((rc = pad_input(c, in, rows, kHid, 0, in_b, nullptr, c->eP))) return rc;
        if ((rc = conv_gemm(c, rows / 2, 2 * kHid, c->down[st].wt, 1, 1, kHid, c->ez, c->eP))) return rc;
        rows /= 2;
        if ((rc = resid_pad(c, y[st], c->ez, c->down[st].bt, rows, kHid, nullptr, 0, nullptr, true))) return rc;
        if ((rc = convnext(c, c->down[st], y[st], rows))) return rc;
        in = y[st], in_b = nullptr;
    }
    return transformer(c, c->pre_layer, kLayers, kWin, y[1], rows, c->pre_norm, out);
}

int32_t check_encoder(S2dCodec *c) {
    if (!c || !c->arena) return cerr(c, S2D_ESTATE, "codec is not loaded");
    if (!c->has_encoder) return cerr(c, S2D_EINVAL, "the codec file holds no reference-audio encoder");
    if (!c->conv_tc) return cerr(c, S2D_EINVAL, "the reference-audio encoder runs on the tcgen05 convolutions only");
    return S2D_OK;
}

// Zero-padded copy of the audio into the encoder workspace; S = padded samples.
int32_t load_audio(S2dCodec *c, const float *audio, size_t n, size_t *S) {
    if (!audio && n) return cerr(c, S2D_EINVAL, "audio is null");
    if (n > 0xffffffffull) return cerr(c, S2D_EINVAL, "encoder input sample count overflows u32");
    const size_t padded = n == 0 ? kFrameLength : (n + kFrameLength - 1) / kFrameLength * kFrameLength;  // codec.rs:1926
    int32_t rc;
    if ((rc = ensure_enc_ws(c, padded))) return rc;
    if ((rc = ensure_ws(c, (uint32_t)(padded / kFrameLength)))) return rc;
    CCK(cudaMemsetAsync(c->eaudio, 0, padded * 4, c->stream));
    if (n) CCK(cudaMemcpyAsync(c->eaudio, audio, n * 4, cudaMemcpyHostToDevice, c->stream));
    *S = padded;
    return S2D_OK;
}

// RVQ lookup, post module, upsample and decoder on device codes.
int32_t decode_device(S2dCodec *c, const int32_t *codes_dev, int T, float *samples) {
    int32_t rc;
    rvq_kernel<<<T, 256, 0, c->stream>>>(c->rvq, codes_dev, T, c->lat, c->error);
    CCK(cudaGetLastError());
    if ((rc = post_module(c, c->lat, T, c->x))) return rc;
    if ((rc = upsample_stage(c, c->up[0], c->x, T, c->x2))) return rc;
    if ((rc = upsample_stage(c, c->up[1], c->x2, 2 * T, c->Z))) return rc;
    // the entry conv reads hidden (Z) into its padded f16 rows before its GEMM overwrites Z
    return decoder(c, c->Z, 4 * T, samples);
}

int32_t check_codes(S2dCodec *c, const int32_t *codes, uint32_t ncb, uint32_t n) {
    if (!codes) return cerr(c, S2D_EINVAL, "codes is null");
    if (ncb != kBooks) return cerr(c, S2D_EINVAL, "codec codebook count mismatch: expected 10, got " + std::to_string(ncb));
    if (n == 0) return cerr(c, S2D_EINVAL, "codec transformer requires at least one frame");
    for (uint32_t cb = 0; cb < ncb; ++cb)
        for (uint32_t f = 0; f < n; ++f) {
            const int32_t v = codes[(size_t)cb * n + f];
            if (v < 0) return cerr(c, S2D_EINVAL, "codec code must be non-negative, got " + std::to_string(v));
            if (v >= c->rvq.size[cb])
                return cerr(c, S2D_EINVAL, "embedding index " + std::to_string(v) + " out of range for codebook " +
                                               std::to_string(cb));
        }
    return S2D_OK;
}

int32_t sync_and_check(S2dCodec *c) {
    CCK(cudaStreamSynchronize(c->stream));
    int32_t flag[2] = {0, 0};
    CCK(cudaMemcpy(flag, c->error, 8, cudaMemcpyDeviceToHost));
    if (flag[0] || flag[1]) {
        CCK(cudaMemset(c->error, 0, 8));
        return cerr(c, S2D_EDEVICE, flag[0] ? "a codec code was out of range for its codebook"
                                            : "a tensor-core convolution's bounded wait gave up");
    }
    return S2D_OK;
}

}  // namespace
}  // namespace s2d

using namespace s2d;

extern "C" {

int32_t s2d_codec_open(const char *gguf_path, int32_t device, S2dCodec **out) {
    if (!out || !gguf_path) return S2D_EINVAL;
    *out = nullptr;
    S2dCodec *c = new S2dCodec();
    c->device = device;
    Gguf g;
    std::string e;
    int32_t rc = S2D_OK;
    std::string arch;
    if (!g.open(gguf_path, &e)) {
        rc = cerr(c, S2D_EIO, e);
    } else if (!g.meta_str("general.architecture", &arch, &e) || arch != "fish-speech-codec") {
        rc = cerr(c, S2D_EINVAL, "expected fish-speech-codec codec GGUF, got " + (arch.empty() ? e : arch));
    } else if (cudaSetDevice(device) != cudaSuccess) {
        rc = cerr(c, S2D_ECUDA, "cudaSetDevice failed");
    } else if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        rc = cerr(c, S2D_ECUDA, "cudaStreamCreate failed");
    } else if (cublasCreate(&c->blas) != CUBLAS_STATUS_SUCCESS ||
               cublasSetStream(c->blas, c->stream) != CUBLAS_STATUS_SUCCESS) {
        rc = cerr(c, S2D_ECUDA, "cublasCreate failed");
    } else {
        if (const char *v = getenv("S2D_CODEC_TC")) c->conv_tc = v[0] != '0';
        if (const char *v = getenv("S2D_CODEC_CONV_CTAS")) c->conv_one_cta = v[0] == '1';
        if (const char *v = getenv("S2D_CODEC_ATTN_TILED")) c->attn_tiled = v[0] != '0';
        rc = load(c, g);
    }
    *out = c;  // also on failure, so that the caller can read the message
    return rc;
}

void s2d_codec_close(S2dCodec *c) {
    if (!c) return;
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->ws) cudaFree(c->ws);
    if (c->enc_ws) cudaFree(c->enc_ws);
    if (c->arena) cudaFree(c->arena);
    if (c->blas) cublasDestroy(c->blas);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

const char *s2d_codec_last_error(const S2dCodec *c) { return c ? c->err.c_str() : "null codec"; }

int32_t s2d_codec_decode_waveform(S2dCodec *c, const int32_t *codes, uint32_t num_codebooks, uint32_t n_frames,
                                  float *samples, size_t capacity, size_t *num_samples, uint32_t *latent_frames) {
    if (!c || !c->arena) return cerr(c, S2D_ESTATE, "codec is not loaded");
    int32_t rc;
    if ((rc = check_codes(c, codes, num_codebooks, n_frames))) return rc;
    const size_t n = (size_t)n_frames * 4 * kSamplesPerLatent;
    if (!samples || capacity < n) return cerr(c, S2D_EINVAL, "samples buffer holds " + std::to_string(capacity) +
                                                                 " floats, the decode needs " + std::to_string(n));
    if ((rc = ensure_ws(c, n_frames))) return rc;
    CCK(cudaMemcpyAsync(c->codes, codes, (size_t)kBooks * n_frames * 4, cudaMemcpyHostToDevice, c->stream));
    if ((rc = decode_device(c, c->codes, (int)n_frames, c->samples))) return rc;
    CCK(cudaMemcpyAsync(samples, c->samples, n * 4, cudaMemcpyDeviceToHost, c->stream));
    if ((rc = sync_and_check(c))) return rc;
    if (num_samples) *num_samples = n;
    if (latent_frames) *latent_frames = 4 * n_frames;
    return S2D_OK;
}

int32_t s2d_codec_decode_waveform_device(S2dCodec *c, const int32_t *codes_dev, uint32_t num_codebooks,
                                         uint32_t n_frames, float *samples_dev, void *stream) {
    if (!c || !c->arena) return cerr(c, S2D_ESTATE, "codec is not loaded");
    if (!codes_dev || !samples_dev) return cerr(c, S2D_EINVAL, "null device buffer");
    if (num_codebooks != kBooks) return cerr(c, S2D_EINVAL, "codec codebook count mismatch");
    if (n_frames == 0) return cerr(c, S2D_EINVAL, "codec transformer requires at least one frame");
    int32_t rc;
    if ((rc = ensure_ws(c, n_frames))) return rc;
    cudaStream_t own = c->stream;
    if (stream) {
        c->stream = (cudaStream_t)stream;
        cublasSetStream(c->blas, c->stream);
    }
    rc = decode_device(c, codes_dev, (int)n_frames, samples_dev);
    if (stream) {
        c->stream = own;
        cublasSetStream(c->blas, own);
    }
    return rc;
}

int32_t s2d_codec_sync(S2dCodec *c) {
    if (!c || !c->stream) return cerr(c, S2D_ESTATE, "codec is not loaded");
    CCK(cudaDeviceSynchronize());
    return sync_and_check(c);
}

int32_t s2d_codec_rvq_lookup(S2dCodec *c, const int32_t *codes, uint32_t num_codebooks, uint32_t n_frames,
                             float *latents) {
    if (!c || !c->arena) return cerr(c, S2D_ESTATE, "codec is not loaded");
    int32_t rc;
    if ((rc = check_codes(c, codes, num_codebooks, n_frames))) return rc;
    if (!latents) return cerr(c, S2D_EINVAL, "latents is null");
    if ((rc = ensure_ws(c, n_frames))) return rc;
    CCK(cudaMemcpyAsync(c->codes, codes, (size_t)kBooks * n_frames * 4, cudaMemcpyHostToDevice, c->stream));
    rvq_kernel<<<n_frames, 256, 0, c->stream>>>(c->rvq, c->codes, (int)n_frames, c->lat, c->error);
    CCK(cudaGetLastError());
    CCK(cudaMemcpyAsync(latents, c->lat, (size_t)n_frames * kHid * 4, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

int32_t s2d_codec_decode_latents(S2dCodec *c, const float *latents, uint32_t n_frames, float *hidden) {
    if (!c || !c->arena) return cerr(c, S2D_ESTATE, "codec is not loaded");
    if (!latents || !hidden) return cerr(c, S2D_EINVAL, "null buffer");
    if (n_frames == 0) return cerr(c, S2D_EINVAL, "codec transformer requires at least one frame");
    int32_t rc;
    if ((rc = ensure_ws(c, n_frames))) return rc;
    const int T = (int)n_frames;
    CCK(cudaMemcpyAsync(c->lat, latents, (size_t)T * kHid * 4, cudaMemcpyHostToDevice, c->stream));
    if ((rc = post_module(c, c->lat, T, c->x))) return rc;
    if ((rc = upsample_stage(c, c->up[0], c->x, T, c->x2))) return rc;
    if ((rc = upsample_stage(c, c->up[1], c->x2, 2 * T, c->Z))) return rc;
    CCK(cudaMemcpyAsync(hidden, c->Z, (size_t)4 * T * kHid * 4, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

int32_t s2d_codec_decoder(S2dCodec *c, const float *hidden, uint32_t n_frames, uint32_t hidden_dim, float *samples) {
    if (!c || !c->arena) return cerr(c, S2D_ESTATE, "codec is not loaded");
    if (!hidden || !samples) return cerr(c, S2D_EINVAL, "null buffer");
    if (hidden_dim != kHid)
        return cerr(c, S2D_EINVAL, "decoder expects latent dim 1024, got " + std::to_string(hidden_dim));
    if (n_frames == 0) return cerr(c, S2D_EINVAL, "decoder needs at least one frame");
    int32_t rc;
    if ((rc = ensure_ws(c, (n_frames + 3) / 4))) return rc;
    const int L = (int)n_frames;
    CCK(cudaMemcpyAsync(c->x2, hidden, (size_t)L * kHid * 4, cudaMemcpyHostToDevice, c->stream));
    if ((rc = decoder(c, c->x2, L, c->samples))) return rc;
    CCK(cudaMemcpyAsync(samples, c->samples, (size_t)L * kSamplesPerLatent * 4, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

int32_t s2d_codec_memory(const S2dCodec *c, size_t *weight_bytes, size_t *workspace_bytes) {
    if (!c) return S2D_EINVAL;
    if (weight_bytes) *weight_bytes = c->arena_bytes;
    if (workspace_bytes) *workspace_bytes = c->ws_bytes + c->enc_ws_bytes;
    return S2D_OK;
}

int32_t s2d_codec_has_encoder(const S2dCodec *c) { return c && c->has_encoder ? 1 : 0; }

int32_t s2d_codec_encode_reference_audio(S2dCodec *c, const float *audio, size_t n_samples, int32_t *codes,
                                         size_t capacity, uint32_t *quantizer_frames, uint32_t *encoder_frames,
                                         uint32_t *padded_samples, float *final_residual_l2) {
    int32_t rc;
    if ((rc = check_encoder(c))) return rc;
    const size_t need = (n_samples == 0 ? 1 : (n_samples + kFrameLength - 1) / kFrameLength) * kBooks;
    if (!codes || capacity < need)
        return cerr(c, S2D_EINVAL, "codes buffer holds " + std::to_string(capacity) + " codes, the audio needs " +
                                       std::to_string(need));
    size_t S = 0;
    if ((rc = load_audio(c, audio, n_samples, &S))) return rc;
    if ((rc = encoder_frontend(c, (int)S))) return rc;
    const int L = (int)(S / 512), T = L / 4;
    if ((rc = quantizer_encode(c, c->ez, c->enc_out_b, L, c->lat))) return rc;
    vq_kernel<<<T, kVqThreads, 0, c->stream>>>(c->vq, c->rvq, c->lat, T, c->ecodes, c->el2);
    CCK(cudaGetLastError());
    CCK(cudaMemcpyAsync(codes, c->ecodes, (size_t)T * kBooks * 4, cudaMemcpyDeviceToHost, c->stream));
    if (final_residual_l2)
        CCK(cudaMemcpyAsync(final_residual_l2, c->el2, (size_t)T * 4, cudaMemcpyDeviceToHost, c->stream));
    if ((rc = sync_and_check(c))) return rc;
    if (quantizer_frames) *quantizer_frames = (uint32_t)T;
    if (encoder_frames) *encoder_frames = (uint32_t)L;
    if (padded_samples) *padded_samples = (uint32_t)S;
    return S2D_OK;
}

int32_t s2d_codec_encoder_frontend(S2dCodec *c, const float *audio, size_t n_samples, float *hidden, size_t capacity,
                                   uint32_t *frames, uint32_t *padded_samples) {
    int32_t rc;
    if ((rc = check_encoder(c))) return rc;
    const size_t S_need = n_samples == 0 ? kFrameLength : (n_samples + kFrameLength - 1) / kFrameLength * kFrameLength;
    if (!hidden || capacity < S_need / 512 * kHid)
        return cerr(c, S2D_EINVAL, "hidden buffer too small: the audio needs " + std::to_string(S_need / 512 * kHid));
    size_t S = 0;
    if ((rc = load_audio(c, audio, n_samples, &S))) return rc;
    if ((rc = encoder_frontend(c, (int)S))) return rc;
    const int L = (int)(S / 512);
    // the output conv's bias
    if ((rc = resid_pad(c, c->ez2, c->ez, c->enc_out_b, L, kHid, nullptr, 0, nullptr, true))) return rc;
    CCK(cudaMemcpyAsync(hidden, c->ez2, (size_t)L * kHid * 4, cudaMemcpyDeviceToHost, c->stream));
    if ((rc = sync_and_check(c))) return rc;
    if (frames) *frames = (uint32_t)L;
    if (padded_samples) *padded_samples = (uint32_t)S;
    return S2D_OK;
}

int32_t s2d_codec_quantizer_encode(S2dCodec *c, const float *hidden, uint32_t n_frames, float *out) {
    int32_t rc;
    if ((rc = check_encoder(c))) return rc;
    if (!hidden || !out) return cerr(c, S2D_EINVAL, "null buffer");
    if (n_frames < 4 || n_frames % 4)
        return cerr(c, S2D_EINVAL, "codec quantizer encode needs a multiple of 4 frames (two stride-2 downsample "
                                   "stages), got " + std::to_string(n_frames));
    const int L = (int)n_frames;
    if ((rc = ensure_enc_ws(c, (size_t)L * 512))) return rc;
    if ((rc = ensure_ws(c, n_frames / 4))) return rc;
    CCK(cudaMemcpyAsync(c->ez2, hidden, (size_t)L * kHid * 4, cudaMemcpyHostToDevice, c->stream));
    if ((rc = quantizer_encode(c, c->ez2, nullptr, L, c->lat))) return rc;
    CCK(cudaMemcpyAsync(out, c->lat, (size_t)(L / 4) * kHid * 4, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

int32_t s2d_codec_vq_encode(S2dCodec *c, const float *latents, uint32_t n_frames, int32_t *codes,
                            float *final_residual_l2) {
    int32_t rc;
    if ((rc = check_encoder(c))) return rc;
    if (!latents || !codes) return cerr(c, S2D_EINVAL, "null buffer");
    if (n_frames == 0) return cerr(c, S2D_EINVAL, "no frames");
    if ((rc = ensure_ws(c, n_frames))) return rc;
    if ((rc = ensure_enc_ws(c, (size_t)n_frames * kFrameLength))) return rc;
    CCK(cudaMemcpyAsync(c->lat, latents, (size_t)n_frames * kHid * 4, cudaMemcpyHostToDevice, c->stream));
    vq_kernel<<<n_frames, kVqThreads, 0, c->stream>>>(c->vq, c->rvq, c->lat, (int)n_frames, c->ecodes, c->el2);
    CCK(cudaGetLastError());
    CCK(cudaMemcpyAsync(codes, c->ecodes, (size_t)n_frames * kBooks * 4, cudaMemcpyDeviceToHost, c->stream));
    if (final_residual_l2)
        CCK(cudaMemcpyAsync(final_residual_l2, c->el2, (size_t)n_frames * 4, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

}  // extern "C"
