// s2d_prefill.cu -- batched Slow-AR prefill (many prompt tokens per layer pass).
//
// The reference prefills token by token with matvecs
// (forward_slow_ar_block_prefill_layers_cached, slow_ar.rs:1002-1039;
// forward_prefill_sequence, :558-595): every prompt token is a full pass over
// the weights.  Here a layer runs once over T tokens: the linears become
// tensor-core GEMMs (cuBLAS, f16 weights), causal attention runs over the
// KV cache that rope_kv_kernel filled for all T tokens, and the elementwise
// epilogues (residual adds, SwiGLU) are separate passes over [T][N].
//
// Precision: the GEMM operands are f16, the activations f32.  Each activation
// row is scaled by a power of two (so that its largest element lies near
// 2^14) and split into hi = f16(v) and lo = f16(v - hi); one GEMM over the
// stacked [hi; lo] rows gives W.hi + W.lo = W.v to about 2^-22 relative per
// element, with f32 accumulation.  The RMSNorm prologue rounds like the
// reference ((x * scale) * w, backend.rs:84-99).
#include <math.h>

#include "s2d_common.cuh"
#include "s2d_prefill.cuh"

namespace s2d {

namespace {

constexpr int kSplitThreads = 256;

__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    __syncthreads();
    return t;
}
__device__ __forceinline__ float block_max(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = fmaxf(t, red[i]);
    __syncthreads();
    return t;
}

// One block per row t of x [T][ldx]: optional RMSNorm (gain w), then the
// scaled hi/lo split into xs rows t and T + t ([2T][K] f16); inv[t] undoes
// the scaling.  With w, the normalised row is also written to xn (if set).
__global__ void __launch_bounds__(kSplitThreads) split_rows_kernel(const float *x, int ldx, int T, int K,
                                                                   const float *w, float eps, __half *xs,
                                                                   float *inv, float *xn) {
    extern __shared__ float row[];  // [K]
    __shared__ float red[kSplitThreads / 32];
    const int t = blockIdx.x;
    const float *src = x + (size_t)t * ldx;
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = src[i];
        row[i] = v;
        ss = fmaf(v, v, ss);
    }
    float scale = 1.0f;
    if (w) scale = 1.0f / sqrtf(block_sum(ss, red) / (float)K + eps);
    else __syncthreads();
    float mx = 0.f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        float v = row[i];
        if (w) {
            v = __fmul_rn(__fmul_rn(v, scale), w[i]);
            row[i] = v;
            if (xn) xn[(size_t)t * K + i] = v;
        }
        mx = fmaxf(mx, fabsf(v));
    }
    mx = block_max(mx, red);
    // a power of two p with mx * p in [2^13, 2^14); 1 for an all-zero row
    float p = 1.0f;
    if (mx > 0.f && isfinite(mx)) {
        int e;
        frexpf(mx, &e);  // mx = f * 2^e, f in [0.5, 1)
        p = ldexpf(1.0f, 14 - e);
    }
    if (threadIdx.x == 0) inv[t] = 1.0f / p;
    __half *hi = xs + (size_t)t * K, *lo = xs + ((size_t)T + t) * K;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = row[i] * p;  // exact: p is a power of two
        const __half h = __float2half_rn(v);
        hi[i] = h;
        lo[i] = __float2half_rn(v - __half2float(h));
    }
}

// y[t][n] (ldy) from the GEMM of the stacked rows: (Y2[t][n] + Y2[T+t][n]) *
// inv[t], then the epilogue.
template <int EPI>
__global__ void combine_kernel(const float *Y2, const float *Y2b, const float *inv, int T, int N, float *y, int ldy,
                               const float *resid, int ldr) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)T * N) return;
    const int t = (int)(i / N), n = (int)(i % N);
    const size_t top = (size_t)t * N + n, bot = ((size_t)T + t) * N + n;
    const float v = __fadd_rn(Y2[top], Y2[bot]) * inv[t];
    float out;
    if (EPI == PF_STORE) {
        out = v;
    } else if (EPI == PF_RESID) {
        out = __fadd_rn(resid[(size_t)t * ldr + n], v);
    } else {
        const float u = __fadd_rn(Y2b[top], Y2b[bot]) * inv[t];
        if (EPI == PF_SWIGLU_SLOW) {
            const float sig = 1.0f / (1.0f + expf(-v));
            out = __fmul_rn(__fmul_rn(v, sig), u);
        } else {
            out = __fmul_rn(v / (1.0f + expf(-v)), u);
        }
    }
    y[(size_t)t * ldy + n] = out;
}

// Causal GQA attention over the cache for T query tokens at positions
// pos0 .. pos0+T-1 (gqa_decode_attention per token, attention.rs:208-247,
// with the causal prefix of forward_prefill_sequence, slow_ar.rs:579-593).
// Grid (token, kv head); warp r of the block is query head kvh*rep + r.  The
// block copies 32 cached K and V rows at a time into shared memory; lane j
// scores position c0 + j, then every lane accumulates its head dims.
template <typename KV, int EPL>
__global__ void prefill_attn_kernel(const float *q, const void *kcache, const void *vcache, int max_seq, float *out,
                                    int pos0, int H, int Hkv, int hd, float scale) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int rep = H / Hkv;
    const int m = blockIdx.x, kvh = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * rep + warp;
    const int kvb = (int)sizeof(KV), rowb = hd * kvb;
    uint8_t *kt = sm, *vt = sm + 32 * (rowb + 16);
    float *qs = reinterpret_cast<float *>(vt + 32 * (rowb + 16)) + warp * hd;
    const int visible = min(pos0 + m + 1, max_seq);
    const float *qrow = q + (size_t)m * H * hd + h * hd;
    for (int i = lane; i < hd; i += 32) qs[i] = qrow[i];
    const uint8_t *kb = reinterpret_cast<const uint8_t *>(kcache) + (size_t)kvh * max_seq * rowb;
    const uint8_t *vb = reinterpret_cast<const uint8_t *>(vcache) + (size_t)kvh * max_seq * rowb;
    const int units = rowb / 16, nthr = blockDim.x;
    float mrun = -INFINITY, l = 0.f, acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    for (int c0 = 0; c0 < visible; c0 += 32) {
        const int n = min(32, visible - c0);
        __syncthreads();  // the previous chunk's readers are done (and qs is written)
        for (int u = threadIdx.x; u < 2 * n * units; u += nthr) {
            const int which = u >= n * units, r = (u % (n * units)) / units, c = u % units;
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>((which ? vb : kb) + (size_t)(c0 + r) * rowb) + c);
            *reinterpret_cast<uint4 *>((which ? vt : kt) + (size_t)r * (rowb + 16) + c * 16) = v;
        }
        __syncthreads();
        float sc = -INFINITY;
        if (lane < n) {
            const KV *kr = reinterpret_cast<const KV *>(kt + (size_t)lane * (rowb + 16));
            float d0 = 0.f, d1 = 0.f;
            for (int i = 0; i < hd; i += 2) {
                d0 = fmaf(qs[i], float(kr[i]), d0);
                d1 = fmaf(qs[i + 1], float(kr[i + 1]), d1);
            }
            sc = (d0 + d1) * scale;
        }
        const float mn = fmaxf(mrun, warp_max(sc));
        const float corr = expf(mrun - mn);
        const float p = lane < n ? expf(sc - mn) : 0.f;
        l = fmaf(l, corr, warp_sum(p));
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] *= corr;
        for (int j = 0; j < n; ++j) {
            const float pj = __shfl_sync(0xffffffffu, p, j);
            const KV *vr = reinterpret_cast<const KV *>(vt + (size_t)j * (rowb + 16)) + lane * EPL;
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[e] = fmaf(pj, float(vr[e]), acc[e]);
        }
        mrun = mn;
    }
    float *o = out + (size_t)m * H * hd + h * hd + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = acc[e] / l;
}

}  // namespace

cudaError_t launch_split_rows(const float *x, int ldx, int T, int K, const float *norm_w, float eps, __half *xs,
                              float *inv, float *xn, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const size_t smem = (size_t)K * sizeof(float);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(split_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        if (e) return e;
        configured = true;
    }
    if (smem > 64 * 1024) return cudaErrorInvalidValue;
    split_rows_kernel<<<T, kSplitThreads, smem, s>>>(x, ldx, T, K, norm_w, eps, xs, inv, xn);
    return cudaGetLastError();
}

cudaError_t launch_combine(int epi, const float *Y2, const float *Y2b, const float *inv, int T, int N, float *y,
                           int ldy, const float *resid, int ldr, cudaStream_t s) {
    const size_t n = (size_t)T * N;
    if (n == 0) return cudaSuccess;
    const int threads = 256;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    switch (epi) {
    case PF_STORE: combine_kernel<PF_STORE><<<blocks, threads, 0, s>>>(Y2, Y2b, inv, T, N, y, ldy, resid, ldr); break;
    case PF_RESID: combine_kernel<PF_RESID><<<blocks, threads, 0, s>>>(Y2, Y2b, inv, T, N, y, ldy, resid, ldr); break;
    case PF_SWIGLU_SLOW:
        combine_kernel<PF_SWIGLU_SLOW><<<blocks, threads, 0, s>>>(Y2, Y2b, inv, T, N, y, ldy, resid, ldr);
        break;
    case PF_SWIGLU_FAST:
        combine_kernel<PF_SWIGLU_FAST><<<blocks, threads, 0, s>>>(Y2, Y2b, inv, T, N, y, ldy, resid, ldr);
        break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_prefill_attention(const float *q, const void *kcache, const void *vcache, bool kv_half, int max_seq,
                                     float *out, int T, int pos0, int H, int Hkv, int hd, float scale,
                                     cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const int rep = H / Hkv;
    if (rep * Hkv != H || rep > 32 || (hd != 64 && hd != 128)) return cudaErrorInvalidValue;
    const int kvb = kv_half ? 2 : 4;
    const size_t smem = (size_t)2 * 32 * (hd * kvb + 16) + (size_t)rep * hd * 4;
    const dim3 grid(T, Hkv), block(rep * 32);
    if (kv_half) {
        if (hd == 64) prefill_attn_kernel<__half, 2><<<grid, block, smem, s>>>(q, kcache, vcache, max_seq, out, pos0, H, Hkv, hd, scale);
        else prefill_attn_kernel<__half, 4><<<grid, block, smem, s>>>(q, kcache, vcache, max_seq, out, pos0, H, Hkv, hd, scale);
    } else {
        if (hd == 64) prefill_attn_kernel<float, 2><<<grid, block, smem, s>>>(q, kcache, vcache, max_seq, out, pos0, H, Hkv, hd, scale);
        else prefill_attn_kernel<float, 4><<<grid, block, smem, s>>>(q, kcache, vcache, max_seq, out, pos0, H, Hkv, hd, scale);
    }
    return cudaGetLastError();
}

}  // namespace s2d
