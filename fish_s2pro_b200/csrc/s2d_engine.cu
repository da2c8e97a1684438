// s2d_engine.cu -- persistent decode layer engine for sm_100a.
//
// One launch runs a whole program of decode ops (every linear, QK-norm,
// RoPE, KV write and GQA attention of a Slow-AR step or a Fast-AR pass, plus
// the output head): the work of SlowArLayerSkeleton::forward_decode_token +
// forward_feed_forward (slow_ar.rs:637-854) for each layer in turn,
// FastArLayerSkeleton (fast_ar.rs:245-352), forward_logits
// (slow_ar.rs:943-955) and the Fast-AR head (fast_ar.rs:429-435).
//
// Layout: one CTA per SM (cooperative launch).  Warp 8 of each CTA is a
// producer: its lane 0 walks the program and streams this CTA's rows of
// every linear, in program order, into a ring of shared-memory slots with
// cp.async.bulk and mbarrier completion.  Weights do not depend on
// activations, so the producer runs ahead across op and layer boundaries,
// limited only by the ring, and HBM stays busy while the consumers wait at a
// grid barrier or run attention.  Warps 0-7 consume: for each op they wait at
// a grid barrier for the previous op's outputs, stage the input vector (with
// its RMSNorm) in shared memory, then every warp reads every slot, each warp
// owning a few rows of the slot (see GemvTiling).
// Every wait is bounded: on timeout the kernel records an error code in
// DevState::error and returns.
#include <math.h>

#include "s2d_common.cuh"
#include "s2d_kernels.cuh"

namespace s2d {

namespace {

// Bounds of every wait (about a second each): a healthy launch never comes
// close; a broken one records an error and returns instead of hanging.
constexpr uint32_t kMbarSpin = 1u << 20;   // try_wait rounds of <= 1 us each
constexpr uint32_t kGridSpin = 1u << 22;   // grid-barrier polls with a short sleep

__device__ __forceinline__ uint32_t saddr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ int32_t ld_volatile(const int32_t *p) {
    return *reinterpret_cast<const volatile int32_t *>(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait for `parity` of an mbarrier, giving up (and flagging `code`) after a
// bounded number of rounds or when another CTA has already flagged an error.
__device__ bool mbar_wait(uint64_t *bar, uint32_t parity, int32_t *err, int32_t code,
                          bool honor_error = true) {
    for (uint32_t i = 0; i < kMbarSpin; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (honor_error && (i & 1023u) == 1023u && ld_volatile(err)) return false;
    }
    atomicCAS(err, 0, code);
    return false;
}

__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            saddr(dst)),
        "l"(src), "r"(bytes), "r"(saddr(bar))
        : "memory");
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kEngineConsumerWarps * 32) : "memory");
}

__device__ __forceinline__ void group_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// GEMV tiling
//
// A CTA's rows of an op are cut into row tiles of at most rmax rows
// (engine_slice_geom, engine_tile_rows); a tile is streamed through the ring
// in K slices, one slot per slice.  The weights were laid out at load
// time in exactly this order (engine_relayout), so each slot is one
// contiguous bulk copy of [mat][R][kw] f16.  Consumer warp w owns rows
// w, w + 8, w + 16, w + 24 of the tile and its lanes split each row's
// 16-byte column chunks; a row's 32 partial sums meet at the end of the tile.
// ---------------------------------------------------------------------------

constexpr int kRowsPerWarp = kEngineTileRows / kEngineConsumerWarps;  // 4
static_assert(kRowsPerWarp * kEngineConsumerWarps == kEngineTileRows, "tile mapping");

struct GemvTiling {
    int r0, n, ntiles, mats, K;
    SliceGeom sg;
    __device__ __forceinline__ GemvTiling(const EngineOp &op, int slot_bytes) {
        int r1;
        engine_cta_rows(op.N, blockIdx.x, gridDim.x, &r0, &r1);
        n = r1 - r0;
        mats = op.W2 ? 2 : 1;
        K = op.K;
        sg = engine_slice_geom(mats, K, slot_bytes);
        ntiles = engine_tile_count(n, sg.rmax);
    }
    // rows [*tr0, *tr0 + *R) of tile t
    __device__ __forceinline__ void tile(int t, int *tr0, int *R) const {
        int a, b;
        engine_tile_rows(n, t, ntiles, &a, &b);
        *tr0 = r0 + a, *R = b - a;
    }
};

// ---------------------------------------------------------------------------
// producer: lane 0 of the last warp
// ---------------------------------------------------------------------------

__device__ void producer(const EngineArgs &a, uint64_t *full, uint64_t *empty, uint8_t *ring) {
    const int NS = a.nslots;
    uint32_t g = 0;  // slots issued
    int slot = 0;
    uint32_t phase = 0;
    for (int i = 0; i < a.n_ops; ++i) {
        const EngineOp &op = a.ops[i];
        if (op.kind != OP_GEMV) continue;
        const GemvTiling T(op, a.slot_bytes);
        const int K = T.K, mats = T.mats;
        const SliceGeom sg = T.sg;
        for (int t = 0; t < T.ntiles; ++t) {
            int tr0, R;
            T.tile(t, &tr0, &R);
            const uint16_t *src = op.Wt + (size_t)tr0 * K * mats;
            for (int s = 0; s < sg.nk; ++s, ++g) {
                const int kw = min(sg.kt, K - s * sg.kt);
                if (!mbar_wait(&empty[slot], phase ^ 1u, a.error, kErrEngineWeights)) goto drain;
                const uint32_t bytes = (uint32_t)(mats * R * kw * 2);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_copy(ring + (size_t)slot * a.slot_bytes, src + (size_t)s * R * sg.kt * mats, bytes, &full[slot]);
                if (++slot == NS) slot = 0, phase ^= 1u;
            }
        }
        if (a.trace && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1))
            a.trace[((size_t)(blockIdx.x ? 1 : 0) * a.n_ops + i) * 4 + 3] = globaltimer();
    }
drain:
    // Do not leave the CTA while copies may still be landing in it: wait
    // (bounded, also after an error) for the last ring's worth of copies.
    {
        const uint32_t first = g > (uint32_t)NS ? g - (uint32_t)NS : 0u;
        for (uint32_t q = first; q < g; ++q) {
            const int slot = (int)(q % (uint32_t)NS);
            if (!mbar_wait(&full[slot], (q / (uint32_t)NS) & 1u, a.error, kErrEngineWeights, false)) return;
        }
    }
}

// Out-of-place copy of a linear's weights into slot order (see GemvTiling):
// one block per output row.
__global__ void relayout_kernel(const uint16_t *W, const uint16_t *W2, int N, int K, int n_contig, int row_base,
                                int extra_row, int G, int slot_bytes, uint16_t *dst) {
    const int r = blockIdx.x;
    const int mats = W2 ? 2 : 1;
    // the CTA owning row r: the largest c with floor(N c / G) <= r
    const int c = (int)((((long long)r + 1) * G - 1) / N);
    int r0, r1;
    engine_cta_rows(N, c, G, &r0, &r1);
    const SliceGeom sg = engine_slice_geom(mats, K, slot_bytes);
    const int n = r1 - r0, nt = engine_tile_count(n, sg.rmax), rel = r - r0;
    const int t = (int)((((long long)rel + 1) * nt - 1) / n);
    int ta, tb;
    engine_tile_rows(n, t, nt, &ta, &tb);
    const int R = tb - ta, q = rel - ta, tr0 = r0 + ta;
    const int src_row = n_contig < 0 ? r : (r < n_contig ? row_base + r : extra_row);
    uint16_t *tile = dst + (size_t)tr0 * K * mats;
    for (int ch = threadIdx.x; ch < K / 8; ch += blockDim.x) {
        const int col = ch * 8, s = col / sg.kt, kw = min(sg.kt, K - s * sg.kt), cc = col - s * sg.kt;
        uint16_t *slot = tile + (size_t)s * R * sg.kt * mats;
        for (int m = 0; m < mats; ++m) {
            const uint16_t *src = (m ? W2 + (size_t)r * K : W + (size_t)src_row * K) + col;
            *reinterpret_cast<uint4 *>(slot + ((size_t)m * R + q) * kw + cc) = *reinterpret_cast<const uint4 *>(src);
        }
    }
}

// ---------------------------------------------------------------------------
// consumers: warps 0-7
// ---------------------------------------------------------------------------

struct ConsumerShared {
    float red[2][kEngineConsumerWarps];
    int ok;
    int abort;  // a consumer warp's wait failed: all warps leave at the next barrier
    int last[kEngineConsumerWarps];
};

// Stage the op's M input vectors in shared memory as xs[m][K], normalised
// when the op has an RMSNorm prologue; CTA 0 also writes them to x_out.
template <int M>
__device__ void stage_x(const EngineOp &op, float *xs, ConsumerShared &cs) {
    constexpr int T = kEngineConsumerWarps * 32;
    constexpr int J = kEngineMaxK / (T * 4);  // float4 per thread and token
    static_assert(J * T * 4 == kEngineMaxK, "K bound");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = op.K, C = K >> 2;
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float4 *src = reinterpret_cast<const float4 *>(op.x + (size_t)m * op.ldx);
        float4 *dst = reinterpret_cast<float4 *>(xs + (size_t)m * K);
        float4 v[J];
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int c = tid + j * T;
            v[j] = c < C ? __ldcg(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        ss[m] = 0.f;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int c = tid + j * T;
            if (c < C) dst[c] = v[j];
            ss[m] = fmaf(v[j].x, v[j].x, ss[m]);
            ss[m] = fmaf(v[j].y, v[j].y, ss[m]);
            ss[m] = fmaf(v[j].z, v[j].z, ss[m]);
            ss[m] = fmaf(v[j].w, v[j].w, ss[m]);
        }
    }
    float *x_out = blockIdx.x == 0 ? op.x_out : nullptr;
    if (op.norm_w) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) cs.red[m][warp] = t;
        }
        consumers_sync();
        const float4 *nw = reinterpret_cast<const float4 *>(op.norm_w);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float t = 0.f;
#pragma unroll
            for (int k = 0; k < kEngineConsumerWarps; ++k) t += cs.red[m][k];
            const float scale = 1.0f / sqrtf(t / (float)K + op.eps);
            float4 *row = reinterpret_cast<float4 *>(xs + (size_t)m * K);
            for (int c = tid; c < C; c += T) {  // the elements this thread stored
                float4 v = row[c];
                const float4 g = __ldg(nw + c);
                v.x = __fmul_rn(__fmul_rn(v.x, scale), g.x);
                v.y = __fmul_rn(__fmul_rn(v.y, scale), g.y);
                v.z = __fmul_rn(__fmul_rn(v.z, scale), g.z);
                v.w = __fmul_rn(__fmul_rn(v.w, scale), g.w);
                row[c] = v;
                if (x_out) reinterpret_cast<float4 *>(x_out + (size_t)m * K)[c] = v;
            }
        }
    } else if (x_out) {
#pragma unroll
        for (int m = 0; m < M; ++m)
            for (int c = tid; c < C; c += T)
                reinterpret_cast<float4 *>(x_out + (size_t)m * K)[c] = reinterpret_cast<const float4 *>(xs + (size_t)m * K)[c];
    }
    consumers_sync();  // xs is complete; cs.red may be rewritten by the next op
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// One slot's arithmetic for a warp holding NR rows of the tile: per step a
// lane takes CH chunks (c and c + 32), loads their inputs once and the
// chunks of each of its rows, and feeds independent accumulator chains
// (acc[j] for chunk j of the step).
template <int NR, int M, int MATS, int CH>
__device__ __forceinline__ void gemv_slot(uint32_t wbase, uint32_t rstride, uint32_t mstride, uint32_t xbase,
                                          int K, int nch, int lane, float (&acc)[CH][kRowsPerWarp][MATS][M]) {
#pragma unroll 1
    for (int c = lane; c < nch; c += 32 * CH) {
        float4 x0[CH][M], x1[CH][M];
        uint4 w[CH][NR][MATS];
#pragma unroll
        for (int j = 0; j < CH; ++j) {
            const int cj = c + 32 * j;
            const bool ok = j == 0 || cj < nch;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const uint32_t xa = xbase + (uint32_t)((m * K + cj * 8) * 4);
                x0[j][m] = ok ? lds_f4(xa) : make_float4(0.f, 0.f, 0.f, 0.f);
                x1[j][m] = ok ? lds_f4(xa + 16) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < NR; ++i)
#pragma unroll
                for (int q = 0; q < MATS; ++q)
                    w[j][i][q] = ok ? lds_u4(wbase + i * rstride + q * mstride + (uint32_t)cj * 16)
                                    : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < CH; ++j)
#pragma unroll
            for (int i = 0; i < NR; ++i)
#pragma unroll
                for (int q = 0; q < MATS; ++q)
#pragma unroll
                    for (int m = 0; m < M; ++m) acc[j][i][q][m] = dot8(w[j][i][q], x0[j][m], x1[j][m], acc[j][i][q][m]);
    }
}

// Consume this CTA's slots of one GEMV op (see GemvTiling).  Every warp
// takes every slot: per 16-byte column chunk a lane loads the inputs once
// and the chunk of each of its warp's rows.
template <int M, int MATS>
__device__ bool consume_gemv(const EngineArgs &a, const EngineOp &op, uint32_t &g, uint64_t *full,
                             uint64_t *empty, const uint8_t *ring, const float *xs) {
    constexpr int CH = 2 / MATS;  // chunks per lane and step: a slice row has 64 / MATS chunks
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int NS = a.nslots;
    const GemvTiling T(op, a.slot_bytes);
    const SliceGeom sg = T.sg;
    const int K = T.K, epi = op.epi, ldy = op.ldy, ldr = op.ldr;
    float *y = op.y;
    const float *resid = op.resid;
    const uint32_t ring_s = saddr(ring), xs_s = saddr(xs), slot_bytes = (uint32_t)a.slot_bytes;
    int slot = (int)(g % (uint32_t)NS);
    uint32_t phase = (g / (uint32_t)NS) & 1u;
    for (int t = 0; t < T.ntiles; ++t) {
        int tr0, R;
        T.tile(t, &tr0, &R);
        const int nrw = R > warp ? (R - warp + kEngineConsumerWarps - 1) / kEngineConsumerWarps : 0;
        float acc[CH][kRowsPerWarp][MATS][M];
#pragma unroll
        for (int j = 0; j < CH; ++j)
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
                for (int q = 0; q < MATS; ++q)
#pragma unroll
                    for (int m = 0; m < M; ++m) acc[j][i][q][m] = 0.f;
        for (int s = 0; s < sg.nk; ++s) {
            const int k0 = s * sg.kt, kw = min(sg.kt, K - k0), nch = kw >> 3;
            const bool got = mbar_wait(&full[slot], phase, a.error, kErrEngineWeights);
            if (!__all_sync(0xffffffffu, got)) return false;
            const uint32_t wbase = ring_s + (uint32_t)slot * slot_bytes + (uint32_t)(warp * kw * 2);
            const uint32_t rstride = (uint32_t)(kEngineConsumerWarps * kw * 2), mstride = (uint32_t)(R * kw * 2);
            const uint32_t xbase = xs_s + (uint32_t)(k0 * 4);
            switch (nrw) {
            case 4: gemv_slot<4, M, MATS, CH>(wbase, rstride, mstride, xbase, K, nch, lane, acc); break;
            case 3: gemv_slot<3, M, MATS, CH>(wbase, rstride, mstride, xbase, K, nch, lane, acc); break;
            case 2: gemv_slot<2, M, MATS, CH>(wbase, rstride, mstride, xbase, K, nch, lane, acc); break;
            case 1: gemv_slot<1, M, MATS, CH>(wbase, rstride, mstride, xbase, K, nch, lane, acc); break;
            default: break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == NS) slot = 0, phase ^= 1u;
        }
        g += (uint32_t)sg.nk;
        // reduce each row's partial sums; lane i * M + m writes row i, token m
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            if (i >= nrw) break;
            float v[MATS][M];
#pragma unroll
            for (int q = 0; q < MATS; ++q)
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    float t = acc[0][i][q][m];
#pragma unroll
                    for (int j = 1; j < CH; ++j) t += acc[j][i][q][m];
                    v[q][m] = warp_sum(t);
                }
#pragma unroll
            for (int m = 0; m < M; ++m) {
                if (lane != i * M + m) continue;
                const int row = tr0 + warp + i * kEngineConsumerWarps;
                const float g1 = v[0][m], g3 = v[MATS - 1][m];
                float out;
                if (epi == EPI_STORE) {
                    out = g1;
                } else if (epi == EPI_RESID) {
                    out = __fadd_rn(__ldcg(resid + (size_t)m * ldr + row), g1);
                } else if (epi == EPI_SWIGLU_SLOW) {
                    const float sig = 1.0f / (1.0f + expf(-g1));
                    out = __fmul_rn(__fmul_rn(g1, sig), g3);
                } else {
                    out = __fmul_rn(g1 / (1.0f + expf(-g1)), g3);
                }
                y[(size_t)m * ldy + row] = out;
            }
        }
    }
    return true;
}

template <int M>
__device__ bool run_gemv(const EngineArgs &a, const EngineOp &op, uint32_t &g, uint64_t *full, uint64_t *empty,
                         const uint8_t *ring, float *xs, ConsumerShared &cs, unsigned long long *tr) {
    stage_x<M>(op, xs, cs);
    if (tr) tr[1] = globaltimer();
    return op.W2 ? consume_gemv<M, 2>(a, op, g, full, empty, ring, xs)
                 : consume_gemv<M, 1>(a, op, g, full, empty, ring, xs);
}

template <typename KV>
__device__ __forceinline__ KV kv_from(float v);
template <>
__device__ __forceinline__ __half kv_from<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float kv_from<float>(float v) { return v; }
__device__ __forceinline__ float kv_to(__half v) { return __half2float(v); }
__device__ __forceinline__ float kv_to(float v) { return v; }

// QK-norm (optional) + RoPE of one head held as EPL values per lane.
template <int EPL>
__device__ __forceinline__ void norm_rope(float *v, const float *nw, float eps, int hd, int pos,
                                          const float *denom) {
    const int lane = threadIdx.x & 31;
    if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) ss = fmaf(v[e], v[e], ss);
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / (float)hd + eps);
#pragma unroll
        for (int e = 0; e < EPL; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], scale), nw[lane * EPL + e]);
    }
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
        const int pair = lane * EPL + e;
        const float theta = (float)pos / denom[pair >> 1];
        float sn, cs;
        sincosf(theta, &sn, &cs);
        const float x0 = v[e], x1 = v[e + 1];
        v[e] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        v[e + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    }
}

template <typename KV>
__device__ __forceinline__ float4 kv_load4(const uint8_t *p, int i);  // elements 4i..4i+3
template <>
__device__ __forceinline__ float4 kv_load4<__half>(const uint8_t *p, int i) {
    const uint2 u = reinterpret_cast<const uint2 *>(p)[i];
    return make_float4(h_lo(u.x), h_hi(u.x), h_lo(u.y), h_hi(u.y));
}
template <>
__device__ __forceinline__ float4 kv_load4<float>(const uint8_t *p, int i) {
    return reinterpret_cast<const float4 *>(p)[i];
}

// Fused QK-norm + RoPE + KV write + split-K GQA attention (the ops of
// rope_kv_kernel and attn_kernel).  Work items are (token, kv head, split);
// a group of `rep` warps (one per query head of the GQA group) takes one
// item.  Per sub-chunk of at most kAttnCap positions the group copies the
// cached K/V rows into shared memory in one cooperative round trip and adds
// the rows of the new tokens (recomputed from qkv, so no group reads a
// position another group is still writing); scores are then computed with
// one lane per position, P.V with each lane owning head dims.  The group of
// split 0 writes its token's K/V to the cache.  The last group to finish a
// (token, kv head) merges the S partial softmaxes.
constexpr int kAttnSplitLen = 64;  // visible positions per attention split
constexpr int kAttnLoads = 4;      // 16-byte cache loads per thread in flight

template <typename KV, int EPL>
__device__ void consume_attn(const EngineOp &op, float *xs, ConsumerShared &cs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = op.hd, rep = op.H / op.Hkv, M = op.M;
    const int gpc = kEngineConsumerWarps / rep;  // groups per CTA
    const int gid = warp / rep, wr = warp % rep, gtid = wr * 32 + lane;
    const int bar_id = 2 + gid, bar_n = rep * 32;
    constexpr int kvb = (int)sizeof(KV);
    const int cap = attn_cap(op.max_seq), rowb = attn_row_bytes(hd, kvb);
    uint8_t *gbase = reinterpret_cast<uint8_t *>(xs) + (size_t)gid * attn_group_bytes(rep, hd, kvb, op.max_seq);
    float *qsm = reinterpret_cast<float *>(gbase) + wr * hd;
    uint8_t *kc = gbase + rep * hd * 4;
    uint8_t *vc = kc + (size_t)cap * rowb;
    const int pos_base = op.pos_const + (op.pos_dev ? __ldcg(op.pos_dev) : 0);
    // splits of the visible positions: one per kAttnSplitLen of the longest
    // token's context, at most the S that the partial buffers hold
    int S = (min(pos_base + M, op.max_seq) + kAttnSplitLen - 1) / kAttnSplitLen;
    S = S < 1 ? 1 : (S > op.S ? op.S : S);
    const int n_items = M * op.Hkv * S;
    const int units = hd * kvb / 16;  // 16-byte units per row
    for (int item = blockIdx.x * gpc + gid; item < n_items; item += gridDim.x * gpc) {
        const int sp = item % S, kvh = (item / S) % op.Hkv, m = item / (S * op.Hkv);
        const int pos = pos_base + m;
        const KV *kbase = reinterpret_cast<const KV *>(op.kcache) + (size_t)kvh * op.max_seq * hd;
        const KV *vbase = reinterpret_cast<const KV *>(op.vcache) + (size_t)kvh * op.max_seq * hd;
        // the query of this warp's head, normalised and rotated, into shared memory
        const int h = kvh * rep + wr;
        {
            float q[EPL];
            const float *qrow = op.qkv + (size_t)m * op.ld_qkv + h * hd + lane * EPL;
#pragma unroll
            for (int e = 0; e < EPL; ++e) q[e] = __ldcg(qrow + e);
            norm_rope<EPL>(q, op.q_norm, op.eps, hd, pos, op.rope_denom);
#pragma unroll
            for (int e = 0; e < EPL; ++e) qsm[lane * EPL + e] = q[e];
        }
        // split 0 stores this token's K/V in the cache
        if (sp == 0 && wr == 0 && pos < op.max_seq) {
            const float *row = op.qkv + (size_t)m * op.ld_qkv;
            float kf[EPL];
#pragma unroll
            for (int e = 0; e < EPL; ++e) kf[e] = __ldcg(row + (op.H + kvh) * hd + lane * EPL + e);
            norm_rope<EPL>(kf, op.k_norm, op.eps, hd, pos, op.rope_denom);
            KV *kd = const_cast<KV *>(kbase) + (size_t)pos * hd + lane * EPL;
            KV *vd = const_cast<KV *>(vbase) + (size_t)pos * hd + lane * EPL;
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
                kd[e] = kv_from<KV>(kf[e]);
                vd[e] = kv_from<KV>(__ldcg(row + (op.H + op.Hkv + kvh) * hd + lane * EPL + e));
            }
        }
        int visible = pos + 1;
        if (visible > op.max_seq) visible = op.max_seq;
        const int chunk = (visible + S - 1) / S;
        const int t0 = sp * chunk, t1 = min(visible, t0 + chunk);
        float mrun = -INFINITY, l = 0.f, acc[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
        for (int c0 = t0; c0 < t1; c0 += cap) {
            const int c1 = min(t1, c0 + cap), n = c1 - c0;
            group_sync(bar_id, bar_n);  // previous sub-chunk's readers are done; qsm is written
            // cached rows [c0, min(c1, pos_base)) -> shared memory, all loads issued together
            const int ncache = max(0, min(c1, pos_base) - c0);
            const int total = 2 * ncache * units;
            for (int u0 = 0; u0 < total; u0 += kAttnLoads * bar_n) {
                uint4 v[kAttnLoads];
#pragma unroll
                for (int k = 0; k < kAttnLoads; ++k) {
                    const int u = u0 + k * bar_n + gtid;
                    if (u < total) {
                        const int which = u >= ncache * units, r = (u % (ncache * units)) / units, c = u % units;
                        const uint8_t *src = reinterpret_cast<const uint8_t *>(which ? vbase : kbase) +
                                             ((size_t)(c0 + r) * hd) * kvb + (size_t)c * 16;
                        v[k] = __ldcg(reinterpret_cast<const uint4 *>(src));
                    }
                }
#pragma unroll
                for (int k = 0; k < kAttnLoads; ++k) {
                    const int u = u0 + k * bar_n + gtid;
                    if (u < total) {
                        const int which = u >= ncache * units, r = (u % (ncache * units)) / units, c = u % units;
                        *reinterpret_cast<uint4 *>((which ? vc : kc) + (size_t)r * rowb + (size_t)c * 16) = v[k];
                    }
                }
            }
            // rows of the new tokens [pos_base, pos_base + M) that fall in this sub-chunk
            if (wr == 0) {
                for (int t = max(c0, pos_base); t < c1; ++t) {
                    const int mm = t - pos_base;
                    const float *row = op.qkv + (size_t)mm * op.ld_qkv;
                    float kf[EPL];
#pragma unroll
                    for (int e = 0; e < EPL; ++e) kf[e] = __ldcg(row + (op.H + kvh) * hd + lane * EPL + e);
                    norm_rope<EPL>(kf, op.k_norm, op.eps, hd, t, op.rope_denom);
                    KV *kd = reinterpret_cast<KV *>(kc + (size_t)(t - c0) * rowb) + lane * EPL;
                    KV *vd = reinterpret_cast<KV *>(vc + (size_t)(t - c0) * rowb) + lane * EPL;
#pragma unroll
                    for (int e = 0; e < EPL; ++e) {
                        kd[e] = kv_from<KV>(kf[e]);
                        vd[e] = kv_from<KV>(__ldcg(row + (op.H + op.Hkv + kvh) * hd + lane * EPL + e));
                    }
                }
            }
            group_sync(bar_id, bar_n);
            // scores: lane j owns position c0 + j
            float sc = -INFINITY;
            if (lane < n) {
                const uint8_t *krow = kc + (size_t)lane * rowb;
                const float4 *q4 = reinterpret_cast<const float4 *>(qsm);
                float d = 0.f;
                for (int i = 0; i < hd / 4; ++i) {
                    const float4 kk = kv_load4<KV>(krow, i), qq = q4[i];
                    d = fmaf(qq.x, kk.x, d);
                    d = fmaf(qq.y, kk.y, d);
                    d = fmaf(qq.z, kk.z, d);
                    d = fmaf(qq.w, kk.w, d);
                }
                sc = d * op.scale;
            }
            const float mn = fmaxf(mrun, warp_max(sc));
            const float corr = expf(mrun - mn);
            const float p = lane < n ? expf(sc - mn) : 0.f;
            l = fmaf(l, corr, warp_sum(p));
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[e] *= corr;
            for (int j = 0; j < n; ++j) {
                const float pj = __shfl_sync(0xffffffffu, p, j);
                const KV *vr = reinterpret_cast<const KV *>(vc + (size_t)j * rowb) + lane * EPL;
#pragma unroll
                for (int e = 0; e < EPL; ++e) acc[e] = fmaf(pj, kv_to(vr[e]), acc[e]);
            }
            mrun = mn;
        }
        if (S == 1) {  // one split: the group's softmax is final
            float *outp = op.att_out + (size_t)m * op.H * hd + h * hd + lane * EPL;
#pragma unroll
            for (int e = 0; e < EPL; ++e) outp[e] = acc[e] / l;
            continue;
        }
        float *pp = op.part + (((size_t)m * op.H + h) * S + sp) * (hd + 2);
        if (lane == 0) __stcg(pp, mrun), __stcg(pp + 1, l);
#pragma unroll
        for (int e = 0; e < EPL; ++e) __stcg(pp + 2 + lane * EPL + e, acc[e]);
        __threadfence();
        group_sync(bar_id, bar_n);
        if (wr == 0 && lane == 0) {
            const int prev = atomicAdd(&op.counters[m * op.Hkv + kvh], 1);
            cs.last[gid] = prev == S - 1;
        }
        group_sync(bar_id, bar_n);
        if (cs.last[gid]) {
            __threadfence();
            // merge: the S partial (max, sum, P.V) loaded in parallel across lanes
            const float *base = op.part + ((size_t)m * op.H + h) * S * (hd + 2);
            float gmax = -INFINITY;
            for (int j0 = 0; j0 < S; j0 += 32) {
                const int j = j0 + lane;
                gmax = fmaxf(gmax, j < S ? __ldcg(base + (size_t)j * (hd + 2)) : -INFINITY);
            }
            gmax = warp_max(gmax);
            float L = 0.f, o[EPL];
#pragma unroll
            for (int e = 0; e < EPL; ++e) o[e] = 0.f;
            for (int j0 = 0; j0 < S; j0 += 32) {
                const int j = j0 + lane;
                float f = 0.f, lj = 0.f;
                if (j < S) {
                    const float *pj = base + (size_t)j * (hd + 2);
                    f = expf(__ldcg(pj) - gmax);
                    lj = __ldcg(pj + 1);
                }
                L += warp_sum(lj * f);
                const int nj = min(32, S - j0);
                for (int jj = 0; jj < nj; jj += 4) {
                    float a[4][EPL], fs[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        fs[k] = __shfl_sync(0xffffffffu, f, (jj + k) & 31);
                        const float *pk = base + (size_t)(j0 + jj + k) * (hd + 2) + 2 + lane * EPL;
#pragma unroll
                        for (int e = 0; e < EPL; ++e) a[k][e] = jj + k < nj ? __ldcg(pk + e) : 0.f;
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k)
#pragma unroll
                        for (int e = 0; e < EPL; ++e) o[e] = fmaf(a[k][e], jj + k < nj ? fs[k] : 0.f, o[e]);
                }
            }
            float *outp = op.att_out + (size_t)m * op.H * hd + h * hd + lane * EPL;
#pragma unroll
            for (int e = 0; e < EPL; ++e) outp[e] = o[e] / L;
            if (wr == 0 && lane == 0) op.counters[m * op.Hkv + kvh] = 0;
        }
        group_sync(bar_id, bar_n);
    }
}

// Not inlined: attention's register pressure stays out of the GEMV loops.
template <typename KV>
__device__ __noinline__ void consume_attn_dispatch(const EngineOp &op, float *xs, ConsumerShared &cs) {
    switch (op.hd / 32) {
    case 2: consume_attn<KV, 2>(op, xs, cs); break;
    case 4: consume_attn<KV, 4>(op, xs, cs); break;
    }
}

}  // namespace

__global__ void __launch_bounds__(kEngineThreads, 1) engine_kernel(const EngineArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ ConsumerShared cs;
    const int tid = threadIdx.x, warp = tid >> 5;
    // [full | empty mbarriers] [staged inputs / attention tiles] [ring]
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + a.nslots;
    uint8_t *area = smem + kEngineBarrierBytes;
    uint8_t *ring = area + a.area_bytes;
    if ((saddr(ring) & 127u) != 0u) {  // TMA boxes land on 128-byte boundaries
        if (tid == 0) atomicCAS(a.error, 0, kErrEngineAlign);
        return;
    }
    if (tid == 0) {
        cs.abort = 0;
        for (int i = 0; i < a.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kEngineConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (a.done && *a.done) return;
    if (warp == kEngineConsumerWarps) {
        if ((tid & 31) == 0) producer(a, full, empty, ring);
        return;
    }
    uint32_t g = 0;
    for (int i = 0; i < a.n_ops; ++i) {
        const EngineOp &op = a.ops[i];
        if (i > 0) {
            // grid barrier: op i reads what op i-1 wrote on every CTA
            consumers_sync();
            if (tid == 0) {
                int ok = cs.abort ? 0 : 1;
                if (ok) {
                    // release: the CTA's writes, ordered before this thread by
                    // the barrier above, are visible to whoever acquires the count
                    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.barrier) : "memory");
                }
                const uint32_t target = (uint32_t)i * gridDim.x;
                uint32_t it = 0;
                while (ok && ld_acquire(a.barrier) < target) {
                    if (++it > kGridSpin) {
                        atomicCAS(a.error, 0, kErrEngineGrid);
                        ok = 0;
                        break;
                    }
                    if ((it & 63u) == 0 && ld_volatile(a.error)) {
                        ok = 0;
                        break;
                    }
                }
                cs.ok = ok;  // the acquire above orders the reads after the next barrier
            }
            consumers_sync();
            if (!cs.ok) return;
        }
        unsigned long long *tr = nullptr;
        if (a.trace && tid == 0 && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1))
            tr = a.trace + ((size_t)(blockIdx.x ? 1 : 0) * a.n_ops + i) * 4;
        if (tr) tr[0] = globaltimer();
        if (op.kind == OP_GEMV) {
            float *xs = reinterpret_cast<float *>(area);
            const bool okg = op.M == 2 ? run_gemv<2>(a, op, g, full, empty, ring, xs, cs, tr)
                                       : run_gemv<1>(a, op, g, full, empty, ring, xs, cs, tr);
            if (!okg) cs.abort = 1;
        } else {
            if (tr) tr[1] = globaltimer();
            float *xs = reinterpret_cast<float *>(area);
            if (op.kv_half) consume_attn_dispatch<__half>(op, xs, cs);
            else consume_attn_dispatch<float>(op, xs, cs);
        }
        if (a.trace) {  // uniform: every consumer thread takes the barrier
            consumers_sync();
            if (tr) tr[2] = globaltimer();
        }
    }
}

cudaError_t launch_engine(const EngineArgs &a, int grid, size_t smem, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(engine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kEngineSmemMax);
        if (e) return e;
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kEngineThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, engine_kernel, a);
}

cudaError_t launch_engine_relayout(const uint16_t *W, const uint16_t *W2, int N, int K, int n_contig,
                                   int row_base, int extra_row, int grid, int slot_bytes, uint16_t *dst,
                                   cudaStream_t s) {
    if (N <= 0 || K <= 0 || K % 8 || grid <= 0) return cudaErrorInvalidValue;
    relayout_kernel<<<N, 128, 0, s>>>(W, W2, N, K, n_contig, row_base, extra_row, grid, slot_bytes, dst);
    return cudaGetLastError();
}

}  // namespace s2d
