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

constexpr int kSplitThreads = 1024;  // one block per row: short passes over the row

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

// The second half of a row split, on row t held in shared memory (`row`,
// K values, with the sum of their squares in ss): optional RMSNorm with gain
// w (the normalised row also to xn when set), then the power-of-two scaled
// f16 hi / lo halves into xs rows t and T + t, and inv[t] = 1 / scale.
__device__ void split_row_tail(float *row, float ss, int t, int T, int K, const float *w, float eps, __half *xs,
                               float *inv, float *xn, float *red) {
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

// One block per row t of x [T][ldx]: optional RMSNorm (gain w), then the
// scaled hi/lo split into xs rows t and T + t ([2T][K] f16); inv[t] undoes
// the scaling.  With w, the normalised row is also written to xn (if set).
// With v4 (K and ldx multiples of 4, x 16-byte aligned) the row arrives in
// one round of float4 loads, up to kRowRounds per thread issued together.
constexpr int kRowRounds = 4;  // float4s per thread: rows of up to 16,384 values in one round
__global__ void __launch_bounds__(kSplitThreads) split_rows_kernel(const float *x, int ldx, int T, int K,
                                                                   const float *w, float eps, __half *xs,
                                                                   float *inv, float *xn, bool v4) {
    extern __shared__ float row[];  // [K]
    __shared__ float red[kSplitThreads / 32];
    const int t = blockIdx.x;
    const float *src = x + (size_t)t * ldx;
    float ss = 0.f;
    if (v4) {
        const int K4 = K >> 2;
        float4 buf[kRowRounds];
#pragma unroll
        for (int j = 0; j < kRowRounds; ++j) {
            const int i4 = threadIdx.x + j * blockDim.x;
            if (i4 < K4) buf[j] = reinterpret_cast<const float4 *>(src)[i4];
        }
#pragma unroll
        for (int j = 0; j < kRowRounds; ++j) {
            const int i4 = threadIdx.x + j * blockDim.x;
            if (i4 < K4) {
                reinterpret_cast<float4 *>(row)[i4] = buf[j];
                ss = fmaf(buf[j].x, buf[j].x, ss);
                ss = fmaf(buf[j].y, buf[j].y, ss);
                ss = fmaf(buf[j].z, buf[j].z, ss);
                ss = fmaf(buf[j].w, buf[j].w, ss);
            }
        }
        for (int i = 4 * (threadIdx.x + kRowRounds * blockDim.x); i < K; i += 4 * blockDim.x) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float v = src[i + e];
                row[i + e] = v;
                ss = fmaf(v, v, ss);
            }
        }
    } else {
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            const float v = src[i];
            row[i] = v;
            ss = fmaf(v, v, ss);
        }
    }
    split_row_tail(row, ss, t, T, K, w, eps, xs, inv, xn, red);
}

// (top + bottom) * s, then the epilogue: the residual r, or SwiGLU with the
// up projection's halves ut + ub
template <int EPI>
__device__ __forceinline__ float combine_vals(float top, float bot, float ut, float ub, float s, float r) {
    const float v = __fadd_rn(top, bot) * s;
    if (EPI == PF_STORE) return v;
    if (EPI == PF_RESID) return __fadd_rn(r, v);
    const float u = __fadd_rn(ut, ub) * s;
    if (EPI == PF_SWIGLU_SLOW) {
        const float sig = 1.0f / (1.0f + expf(-v));
        return __fmul_rn(__fmul_rn(v, sig), u);
    }
    return __fmul_rn(v / (1.0f + expf(-v)), u);
}
template <int EPI>
__device__ __forceinline__ float combine_one(const float *Y2, const float *Y2b, float s, size_t top, size_t bot,
                                             const float *resid) {
    const bool up = EPI == PF_SWIGLU_SLOW || EPI == PF_SWIGLU_FAST;
    return combine_vals<EPI>(Y2[top], Y2[bot], up ? Y2b[top] : 0.f, up ? Y2b[bot] : 0.f, s,
                             EPI == PF_RESID ? *resid : 0.f);
}

// combine_kernel then split_rows_kernel on the same row, in one pass: one
// block per row t; y (optional) receives the combined row, the split goes to
// xs / inv (inv[t] is read before it is replaced).  With v4 (N, ldy, ldr
// multiples of 4, the buffers 16-byte aligned) every operand of the row
// arrives in one round of float4 loads.
template <int EPI>
__global__ void __launch_bounds__(kSplitThreads) combine_split_kernel(const float *Y2, const float *Y2b, float *inv,
                                                                      int T, int N, float *y, int ldy,
                                                                      const float *resid, int ldr, const float *w,
                                                                      float eps, __half *xs, bool v4) {
    extern __shared__ float row[];  // [N]
    __shared__ float red[kSplitThreads / 32];
    const int t = blockIdx.x;
    const float s = inv[t];
    float ss = 0.f;
    constexpr bool up = EPI == PF_SWIGLU_SLOW || EPI == PF_SWIGLU_FAST;
    constexpr int RR = up ? 3 : kRowRounds;  // four operands per element: 3 rounds stay in registers
    if (v4) {
        const int N4 = N >> 2;
        const float4 *yt = reinterpret_cast<const float4 *>(Y2 + (size_t)t * N);
        const float4 *yb = reinterpret_cast<const float4 *>(Y2 + ((size_t)T + t) * N);
        const float4 *ut = reinterpret_cast<const float4 *>((up ? Y2b : Y2) + (size_t)t * N);
        const float4 *ub = reinterpret_cast<const float4 *>((up ? Y2b : Y2) + ((size_t)T + t) * N);
        const float4 *rr = reinterpret_cast<const float4 *>(resid + (size_t)t * ldr);
        float4 A[RR], B[RR], C[RR], D[RR], R[RR];
#pragma unroll
        for (int j = 0; j < RR; ++j) {
            const int i4 = threadIdx.x + j * blockDim.x;
            if (i4 < N4) {
                A[j] = yt[i4], B[j] = yb[i4];
                if (up) C[j] = ut[i4], D[j] = ub[i4];
                if (EPI == PF_RESID) R[j] = rr[i4];
            }
        }
#pragma unroll
        for (int j = 0; j < RR; ++j) {
            const int i4 = threadIdx.x + j * blockDim.x;
            if (i4 < N4) {
                const float4 c = up ? C[j] : A[j], d = up ? D[j] : A[j], r = EPI == PF_RESID ? R[j] : A[j];
                float4 o;
                o.x = combine_vals<EPI>(A[j].x, B[j].x, c.x, d.x, s, r.x);
                o.y = combine_vals<EPI>(A[j].y, B[j].y, c.y, d.y, s, r.y);
                o.z = combine_vals<EPI>(A[j].z, B[j].z, c.z, d.z, s, r.z);
                o.w = combine_vals<EPI>(A[j].w, B[j].w, c.w, d.w, s, r.w);
                reinterpret_cast<float4 *>(row)[i4] = o;
                if (y) reinterpret_cast<float4 *>(y + (size_t)t * ldy)[i4] = o;
                ss = fmaf(o.x, o.x, ss);
                ss = fmaf(o.y, o.y, ss);
                ss = fmaf(o.z, o.z, ss);
                ss = fmaf(o.w, o.w, ss);
            }
        }
        for (int n = 4 * (threadIdx.x + RR * blockDim.x); n < N; n += 4 * blockDim.x) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float v = combine_one<EPI>(Y2, Y2b, s, (size_t)t * N + n + e, ((size_t)T + t) * N + n + e,
                                                 resid + (size_t)t * ldr + n + e);
                row[n + e] = v;
                if (y) y[(size_t)t * ldy + n + e] = v;
                ss = fmaf(v, v, ss);
            }
        }
        split_row_tail(row, ss, t, T, N, w, eps, xs, inv, nullptr, red);
        return;
    }
    for (int n = threadIdx.x; n < N; n += blockDim.x) {
        const float v = combine_one<EPI>(Y2, Y2b, s, (size_t)t * N + n, ((size_t)T + t) * N + n,
                                         resid + (size_t)t * ldr + n);
        row[n] = v;
        if (y) y[(size_t)t * ldy + n] = v;
        ss = fmaf(v, v, ss);
    }
    split_row_tail(row, ss, t, T, N, w, eps, xs, inv, nullptr, red);
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

// ---------------------------------------------------------------------------
// GQA attention of many query rows over their sequences' caches
// (gqa_decode_attention + softmax_in_place per row, attention.rs:208-309; the
// causal prefix of forward_prefill_sequence, slow_ar.rs:579-593).  A row is a
// (sequence, position) pair: the T tokens of one prompt (prefill), one token
// of each of B sequences (batched Slow-AR step), or the Fast-AR positions of
// B frames.  Grid (row, kv head, split); warp r of a block is query head
// kvh*rep + r, so the group's K/V rows are fetched once for its rep heads.
// The block stages 32 cached K and V rows at a time in shared memory with
// cp.async (two stages for f16 caches, so the next chunk streams while this
// one is scored); lane j scores position c0 + j, then every lane accumulates
// its head dims.  With S > 1 splits each block writes its (max, sum, weighted
// V) partial and the last block of the (row, kv head) to arrive merges them.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// q (shared, hd floats) . K row (shared, hd elements), 16-byte reads.
__device__ __forceinline__ float dot_row(const float *q, const __half *k, int hd) {
    float d0 = 0.f, d1 = 0.f;
    for (int i = 0; i < hd; i += 8) {
        const uint4 u = *reinterpret_cast<const uint4 *>(k + i);
        d0 = fmaf(q[i], h_lo(u.x), d0);
        d1 = fmaf(q[i + 1], h_hi(u.x), d1);
        d0 = fmaf(q[i + 2], h_lo(u.y), d0);
        d1 = fmaf(q[i + 3], h_hi(u.y), d1);
        d0 = fmaf(q[i + 4], h_lo(u.z), d0);
        d1 = fmaf(q[i + 5], h_hi(u.z), d1);
        d0 = fmaf(q[i + 6], h_lo(u.w), d0);
        d1 = fmaf(q[i + 7], h_hi(u.w), d1);
    }
    return d0 + d1;
}
__device__ __forceinline__ float dot_row(const float *q, const float *k, int hd) {
    float d0 = 0.f, d1 = 0.f;
    for (int i = 0; i < hd; i += 4) {
        const float4 u = *reinterpret_cast<const float4 *>(k + i);
        d0 = fmaf(q[i], u.x, d0);
        d1 = fmaf(q[i + 1], u.y, d1);
        d0 = fmaf(q[i + 2], u.z, d0);
        d1 = fmaf(q[i + 3], u.w, d1);
    }
    return d0 + d1;
}

template <typename KV, int EPL>
__device__ __forceinline__ void load_v(const KV *p, float *o) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = float(p[e]);
}

template <typename KV, int EPL, int NST>
__device__ __forceinline__ void rows_attn_body(const RowsAttnArgs &a, uint8_t *sm, int &s_last) {
    const int rep = blockDim.x >> 5;
    const int m = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * rep + warp;
    const int hd = a.hd, rowb = hd * (int)sizeof(KV), pitch = rowb + 16;
    const int seq = m / a.rows_per_seq, j = m - seq * a.rows_per_seq;
    if (a.st && a.st[seq].done) return;  // every split of the row returns: no counter use
    const int pos = a.pos_const + (a.st && a.st_pos ? a.st[seq].n_past : 0) + j;
    const int visible = max(1, min(pos + 1, a.max_seq));
    const int nch = (visible + 31) / 32, cps = (nch + a.S - 1) / a.S;
    const int t0 = min(visible, sp * cps * 32), t1 = min(visible, t0 + cps * 32);
    float *qs = reinterpret_cast<float *>(sm + (size_t)NST * 2 * 32 * pitch) + warp * hd;
    const float *qrow = a.q + (size_t)m * a.H * hd + (size_t)h * hd;
    for (int i = lane; i < hd; i += 32) qs[i] = qrow[i];
    const uint8_t *kb = reinterpret_cast<const uint8_t *>(a.kcache);
    const uint8_t *vb = reinterpret_cast<const uint8_t *>(a.vcache);
    const int units = rowb / 16;
    auto issue = [&](int c0, int stg) {
        const int n = min(32, t1 - c0);
        uint8_t *kt = sm + (size_t)stg * 2 * 32 * pitch, *vt = kt + 32 * pitch;
        // the chunk's rows are consecutive in one page (chunks start at multiples of 32)
        const size_t cb = kv_row(a.kv_pages, a.kv_seq_stride, a.max_seq, seq, kvh, c0, hd) * sizeof(KV);
        for (int u = threadIdx.x; u < 2 * n * units; u += blockDim.x) {
            const int which = u >= n * units, uu = which ? u - n * units : u;
            const int r = uu / units, c = uu - r * units;
            cp_async16((which ? vt : kt) + r * pitch + c * 16, (which ? vb : kb) + cb + (size_t)r * rowb + c * 16);
        }
        cp_async_commit();
    };
    float mrun = -INFINITY, l = 0.f, acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    // NST-stage ring: chunks it .. it + NST - 2 are in flight while chunk it
    // is scored (an empty group keeps the group count when no chunk is left)
#pragma unroll
    for (int i = 0; i < NST - 1; ++i) {
        if (t0 + i * 32 < t1) issue(t0 + i * 32, i);
        else cp_async_commit();
    }
    for (int c0 = t0, it = 0; c0 < t1; c0 += 32, ++it) {
        const int stg = it % NST;
        if (NST == 1) {
            issue(c0, 0);  // the previous chunk's readers are done (trailing barrier)
            cp_async_wait<0>();
        } else {
            const int cn = c0 + (NST - 1) * 32;
            if (cn < t1) issue(cn, (it + NST - 1) % NST);
            else cp_async_commit();
            cp_async_wait<NST - 1>();
        }
        __syncthreads();  // this chunk (and, on the first pass, qs) visible to every warp
        const int n = min(32, t1 - c0);
        const uint8_t *kt = sm + (size_t)stg * 2 * 32 * pitch, *vt = kt + 32 * pitch;
        float sc = -INFINITY;
        if (lane < n) sc = dot_row(qs, reinterpret_cast<const KV *>(kt + lane * pitch), hd) * a.scale;
        const float mn = fmaxf(mrun, warp_max(sc));
        const float corr = expf(mrun - mn);
        const float p = lane < n ? expf(sc - mn) : 0.f;
        l = fmaf(l, corr, warp_sum(p));
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] *= corr;
        for (int jj = 0; jj < n; ++jj) {
            const float pj = __shfl_sync(0xffffffffu, p, jj);
            float vf[EPL];
            load_v<KV, EPL>(reinterpret_cast<const KV *>(vt + jj * pitch) + lane * EPL, vf);
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[e] = fmaf(pj, vf[e], acc[e]);
        }
        mrun = mn;
        __syncthreads();  // readers done before the stage is refilled
    }
    if (a.S == 1) {
        float *o = a.out + (size_t)m * a.H * hd + (size_t)h * hd + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[e] = acc[e] / l;
        return;
    }
    float *pp = a.part + (((size_t)m * a.H + h) * a.S + sp) * (hd + 2);
    if (lane == 0) {
        __stcg(pp, mrun);
        __stcg(pp + 1, l);
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) __stcg(pp + 2 + lane * EPL + e, acc[e]);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&a.counters[(size_t)m * a.Hkv + kvh], 1) == a.S - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float *base = a.part + ((size_t)m * a.H + h) * a.S * (hd + 2);
    float gmax = -INFINITY;
    for (int s2 = 0; s2 < a.S; ++s2) gmax = fmaxf(gmax, __ldcg(base + (size_t)s2 * (hd + 2)));
    float L = 0.f, o[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = 0.f;
    for (int s2 = 0; s2 < a.S; ++s2) {
        const float *pj = base + (size_t)s2 * (hd + 2);
        const float f = expf(__ldcg(pj) - gmax);
        L = fmaf(__ldcg(pj + 1), f, L);
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[e] = fmaf(__ldcg(pj + 2 + lane * EPL + e), f, o[e]);
    }
    float *op = a.out + (size_t)m * a.H * hd + (size_t)h * hd + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) op[e] = o[e] / L;
    if (threadIdx.x == 0) a.counters[(size_t)m * a.Hkv + kvh] = 0;
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
    const bool v4 = K % 4 == 0 && ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    split_rows_kernel<<<T, kSplitThreads, smem, s>>>(x, ldx, T, K, norm_w, eps, xs, inv, xn, v4);
    return cudaGetLastError();
}

cudaError_t launch_combine_split(int epi, const float *Y2, const float *Y2b, float *inv, int T, int N, float *y,
                                 int ldy, const float *resid, int ldr, const float *norm_w, float eps, __half *xs,
                                 cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const size_t smem = (size_t)N * sizeof(float);
    if (smem > 64 * 1024 || (epi == PF_RESID && !resid)) return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        const void *ks[] = {(const void *)combine_split_kernel<PF_STORE>, (const void *)combine_split_kernel<PF_RESID>,
                            (const void *)combine_split_kernel<PF_SWIGLU_SLOW>,
                            (const void *)combine_split_kernel<PF_SWIGLU_FAST>};
        for (const void *k : ks) {
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
            if (e) return e;
        }
        configured = true;
    }
    const float *r = resid ? resid : Y2;
    auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool v4 = N % 4 == 0 && a16(Y2) && (!Y2b || a16(Y2b)) && (!y || (ldy % 4 == 0 && a16(y))) &&
                    (epi != PF_RESID || (ldr % 4 == 0 && a16(resid))) &&
                    (!(epi == PF_SWIGLU_SLOW || epi == PF_SWIGLU_FAST) || Y2b);
    switch (epi) {
    case PF_STORE:
        combine_split_kernel<PF_STORE><<<T, kSplitThreads, smem, s>>>(Y2, Y2b, inv, T, N, y, ldy, r, ldr, norm_w, eps, xs, v4);
        break;
    case PF_RESID:
        combine_split_kernel<PF_RESID><<<T, kSplitThreads, smem, s>>>(Y2, Y2b, inv, T, N, y, ldy, r, ldr, norm_w, eps, xs, v4);
        break;
    case PF_SWIGLU_SLOW:
        combine_split_kernel<PF_SWIGLU_SLOW><<<T, kSplitThreads, smem, s>>>(Y2, Y2b, inv, T, N, y, ldy, r, ldr, norm_w,
                                                                            eps, xs, v4);
        break;
    case PF_SWIGLU_FAST:
        combine_split_kernel<PF_SWIGLU_FAST><<<T, kSplitThreads, smem, s>>>(Y2, Y2b, inv, T, N, y, ldy, r, ldr, norm_w,
                                                                            eps, xs, v4);
        break;
    default: return cudaErrorInvalidValue;
    }
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

template <typename KV, int EPL, int NST>
__global__ void __launch_bounds__(256) rows_attn_kernel(const RowsAttnArgs a) {
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ int s_last;
    rows_attn_body<KV, EPL, NST>(a, sm, s_last);
}

// The batched decode step's rows (one per sequence, positions from the
// sequences' states): the same body under its own name, so that profiles
// tell it from the prompt-chunk tails.
template <typename KV, int EPL, int NST>
__global__ void __launch_bounds__(256) decode_rows_attn_kernel(const RowsAttnArgs a) {
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ int s_last;
    rows_attn_body<KV, EPL, NST>(a, sm, s_last);
}


// Causal attention of one sequence's consecutive rows (the prefill case of
// rows_attn_kernel: rows_per_seq = T, no state, one split), QB query rows per
// block so that every staged K/V chunk serves all of them.  Grid (row
// tile, kv head); warp w is query head kvh*rep + w for all QB rows.  Row r
// of the tile sees positions 0 .. pos_const + m0 + r; the chunks past a
// row's end are skipped for that row (warp-uniformly), so no fully masked
// update happens.
template <typename KV, int EPL, int QB>
__global__ void __launch_bounds__(256) prefill_tile_attn_kernel(const RowsAttnArgs a) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int rep = blockDim.x >> 5;
    const int m0 = blockIdx.x * QB, kvh = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * rep + warp;
    const int hd = a.hd, rowb = hd * (int)sizeof(KV), pitch = rowb + 16;
    const int nrows = min(QB, a.T - m0);
    const int last_pos = min(a.pos_const + m0 + nrows - 1, a.max_seq - 1);
    const int t1 = last_pos + 1;
    float *qs = reinterpret_cast<float *>(sm + (size_t)2 * 2 * 32 * pitch) + (size_t)warp * QB * hd;
    for (int r = 0; r < QB; ++r)
        for (int i = lane; i < hd; i += 32)
            qs[r * hd + i] = r < nrows ? a.q[(size_t)(m0 + r) * a.H * hd + (size_t)h * hd + i] : 0.f;
    const uint8_t *kb = reinterpret_cast<const uint8_t *>(a.kcache);
    const uint8_t *vb = reinterpret_cast<const uint8_t *>(a.vcache);
    const int units = rowb / 16;
    auto issue = [&](int c0, int stg) {
        const int n = min(32, t1 - c0);
        uint8_t *kt = sm + (size_t)stg * 2 * 32 * pitch, *vt = kt + 32 * pitch;
        const size_t cb = kv_row(a.kv_pages, 0, a.max_seq, 0, kvh, c0, hd) * sizeof(KV);  // one sequence
        for (int u = threadIdx.x; u < 2 * n * units; u += blockDim.x) {
            const int which = u >= n * units, uu = which ? u - n * units : u;
            const int r = uu / units, c = uu - r * units;
            cp_async16((which ? vt : kt) + r * pitch + c * 16, (which ? vb : kb) + cb + (size_t)r * rowb + c * 16);
        }
        cp_async_commit();
    };
    float mrun[QB], l[QB], acc[QB][EPL];
#pragma unroll
    for (int r = 0; r < QB; ++r) {
        mrun[r] = -INFINITY, l[r] = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[r][e] = 0.f;
    }
    issue(0, 0);
    for (int c0 = 0, it = 0; c0 < t1; c0 += 32, ++it) {
        const int stg = it & 1;
        if (c0 + 32 < t1) {
            issue(c0 + 32, stg ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // this chunk (and, on the first pass, qs) visible to every warp
        const int n = min(32, t1 - c0);
        const uint8_t *kt = sm + (size_t)stg * 2 * 32 * pitch, *vt = kt + 32 * pitch;
        // scores of this lane's position against the QB queries
        float sc[QB];
#pragma unroll
        for (int r = 0; r < QB; ++r) sc[r] = 0.f;
        if (lane < n) {
            const KV *krow = reinterpret_cast<const KV *>(kt + lane * pitch);
            for (int i = 0; i < hd; i += 4) {
                float k4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) k4[e] = float(krow[i + e]);
#pragma unroll
                for (int r = 0; r < QB; ++r) {
                    const float4 q4 = *reinterpret_cast<const float4 *>(qs + r * hd + i);
                    sc[r] = fmaf(q4.x, k4[0], fmaf(q4.y, k4[1], fmaf(q4.z, k4[2], fmaf(q4.w, k4[3], sc[r]))));
                }
            }
        }
        float p[QB];
#pragma unroll
        for (int r = 0; r < QB; ++r) {
            const int pos = a.pos_const + m0 + r;  // row r sees positions <= pos
            p[r] = 0.f;
            if (r >= nrows || c0 > pos) continue;  // uniform over the warp
            const bool ok = lane < n && c0 + lane <= pos;
            const float s = ok ? sc[r] * a.scale : -INFINITY;
            const float mn = fmaxf(mrun[r], warp_max(s));  // finite: position c0 <= pos is valid
            const float corr = expf(mrun[r] - mn);
            p[r] = ok ? expf(s - mn) : 0.f;
            l[r] = fmaf(l[r], corr, warp_sum(p[r]));
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[r][e] *= corr;
            mrun[r] = mn;
        }
        for (int jj = 0; jj < n; ++jj) {
            float vf[EPL];
            load_v<KV, EPL>(reinterpret_cast<const KV *>(vt + jj * pitch) + lane * EPL, vf);
#pragma unroll
            for (int r = 0; r < QB; ++r) {
                const float pj = __shfl_sync(0xffffffffu, p[r], jj);
#pragma unroll
                for (int e = 0; e < EPL; ++e) acc[r][e] = fmaf(pj, vf[e], acc[r][e]);
            }
        }
        if (c0 + 32 < t1) __syncthreads();  // readers done before the stage is refilled
    }
#pragma unroll
    for (int r = 0; r < QB; ++r) {
        if (r >= nrows) break;
        float *o = a.out + (size_t)(m0 + r) * a.H * hd + (size_t)h * hd + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[e] = acc[r][e] / l[r];
    }
}

template <typename KV, int EPL>
static cudaError_t prefill_tile_launch(const RowsAttnArgs &a, cudaStream_t s) {
    constexpr int QB = 8;
    const int rep = a.H / a.Hkv;
    const int pitch = a.hd * (int)sizeof(KV) + 16;
    const size_t smem = (size_t)2 * 2 * 32 * pitch + (size_t)rep * QB * a.hd * sizeof(float);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(prefill_tile_attn_kernel<KV, EPL, QB>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        if (e) return e;
        configured = true;
    }
    if (smem > 160 * 1024) return cudaErrorInvalidValue;
    prefill_tile_attn_kernel<KV, EPL, QB><<<dim3((a.T + QB - 1) / QB, a.Hkv), rep * 32, smem, s>>>(a);
    return cudaGetLastError();
}

template <typename KV, int EPL, int NST>
static cudaError_t rows_attn_launch(const RowsAttnArgs &a, cudaStream_t s) {
    const int rep = a.H / a.Hkv;
    const int pitch = a.hd * (int)sizeof(KV) + 16;
    const size_t smem = (size_t)NST * 2 * 32 * pitch + (size_t)rep * a.hd * sizeof(float);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(rows_attn_kernel<KV, EPL, NST>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        if (!e)
            e = cudaFuncSetAttribute(decode_rows_attn_kernel<KV, EPL, NST>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        if (e) return e;
        configured = true;
    }
    if (smem > 96 * 1024) return cudaErrorInvalidValue;
    if (a.st && a.st_pos)
        decode_rows_attn_kernel<KV, EPL, NST><<<dim3(a.T, a.Hkv, a.S), rep * 32, smem, s>>>(a);
    else
        rows_attn_kernel<KV, EPL, NST><<<dim3(a.T, a.Hkv, a.S), rep * 32, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_rows_attention(const RowsAttnArgs &a, bool kv_half, cudaStream_t s) {
    if (a.T <= 0) return cudaSuccess;
    if (a.Hkv <= 0 || a.H % a.Hkv || a.H / a.Hkv > 8 || (a.hd != 64 && a.hd != 128) || a.rows_per_seq <= 0 ||
        a.S <= 0 || a.S > 65535 || a.T > 0x7fffffff || a.max_seq <= 0 || (a.S > 1 && (!a.part || !a.counters)))
        return cudaErrorInvalidValue;
    // one sequence's consecutive rows (prompt chunks): query rows tiled per block
    if (a.prefill_tc && a.T >= 16 && prefill_tc_supported(a, kv_half)) return launch_prefill_tc_attention(a, s);
    if (a.prefill_mma && a.T >= 16 && prefill_mma_supported(a, kv_half)) return launch_prefill_mma_attention(a, s);
    if (a.rows_per_seq >= a.T && !a.st && a.S == 1 && a.T >= 16 && kv_half)
        return a.hd == 64 ? prefill_tile_launch<__half, 2>(a, s) : prefill_tile_launch<__half, 4>(a, s);
    if (a.decode_mma && decode_mma_supported(a, kv_half)) return launch_decode_mma_attention(a, s);
    // decode rows (one or two per sequence): a deeper ring keeps more of the
    // block's staging in flight
    if (kv_half && a.rows_per_seq <= 2 && a.decode_stages == 4)
        return a.hd == 64 ? rows_attn_launch<__half, 2, 4>(a, s) : rows_attn_launch<__half, 4, 4>(a, s);
    if (kv_half) return a.hd == 64 ? rows_attn_launch<__half, 2, 2>(a, s) : rows_attn_launch<__half, 4, 2>(a, s);
    return a.hd == 64 ? rows_attn_launch<float, 2, 1>(a, s) : rows_attn_launch<float, 4, 1>(a, s);
}

}  // namespace s2d
