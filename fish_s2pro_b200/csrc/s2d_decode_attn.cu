// s2d_decode_attn.cu -- attention of the batched Slow-AR step on the tensor
// cores.
//
// One query row per sequence attends over that sequence's cached positions
// (gqa_decode_attention + softmax_in_place, attention.rs:208-309, once per
// sequence).  A block takes one (sequence, kv head, split); its warps share
// the split's positions, warp w taking the KC-position chunks w, w + NW, ...
// of it, each through its own cp.async ring in shared memory.  Blocks are
// numbered kv head fastest, then split, then sequence rank, where rank
// follows an optional row order (longest context first, so the long blocks
// start in the first wave and the short ones fill the tail).
//
// One warp serves the whole query group of its kv head (rep <= 8 heads) with
// m16n8k16 f16 MMAs:
//   scores  S[16][32] = Q[16][hd] . K^T   (rows r < rep: f16 hi of head r,
//                                          rows 8 + r: the f16 lo remainder)
//   output  O[16][hd] += P[16][32] . V    (P rows split the same way)
// so rows r and 8 + r of every accumulator sum to head r's value with about
// 22 significant bits in the operands and f32 accumulation, and both halves
// of a head sit in the same thread's accumulator registers.  Each query is
// pre-scaled by scale * log2(e) and a power of two that puts its largest
// element near 2^14 (the power is taken out of the scores exactly), so the
// softmax runs in base 2 with exp2f.
//
// The block merges its warps' (max, sum, weighted V) states in shared memory
// (over the drained rings);
// with S > 1 splits it writes the merged state as a partial and the last
// block of the (sequence, kv head) to arrive merges the S partials.
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>

#include "s2d_common.cuh"
#include "s2d_prefill.cuh"

namespace s2d {

namespace {

__device__ __forceinline__ void cp_async16_zfill(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
// c += A (16x16, row-major fragments) . B (16x8, column fragments), f32 accumulators
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float x, float y) {
    const __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// (x, y) = f16 hi + f16 lo: hi packed into *hi, the remainders into *lo
__device__ __forceinline__ void split_half2(float x, float y, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = pack_half2(x - hf.x, y - hf.y);
}

template <int HD, int NST, int KC>
__global__ void __launch_bounds__(128) decode_mma_attn_kernel(const RowsAttnArgs a) {
    constexpr int KS = HD / 16;         // k-steps of the score MMA
    constexpr int NO = HD / 8;          // n-tiles of the output
    constexpr int NP = KC / 8;          // n-tiles of the scores
    constexpr int UNITS = HD * 2 / 16;  // 16-byte units per cached row
    constexpr int PITCH = HD * 2 + 16;  // staged row pitch: conflict-free ldmatrix rows
    constexpr int STAGE = 2 * KC * PITCH;
    static_assert(KC == 16 || KC == 32, "chunk of 16 or 32 positions");
    static_assert((KC * UNITS) % 32 == 0, "whole copy rounds per lane");
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ int s_last;
    const int nw = blockDim.x >> 5;
    const int rep = a.H / a.Hkv;
    const int kvh = blockIdx.x % a.Hkv, rest = blockIdx.x / a.Hkv, sp = rest % a.S, rank = rest / a.S;
    const int m = a.row_order ? a.row_order[rank] : rank;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    if (a.st[m].done) return;  // every split of the row returns: no counter use
    const int pos = a.pos_const + a.st[m].n_past;
    const int visible = max(1, min(pos + 1, a.max_seq));
    const int nch = (visible + KC - 1) / KC, cps = (nch + a.S - 1) / a.S;
    const int t0 = min(visible, sp * cps * KC), t1 = min(visible, t0 + cps * KC);
    const int nck = (t1 - t0 + KC - 1) / KC;
    const int mine = nck > warp ? (nck - warp + nw - 1) / nw : 0;

    const uint8_t *kb = reinterpret_cast<const uint8_t *>(a.kcache);
    const uint8_t *vb = reinterpret_cast<const uint8_t *>(a.vcache);
    uint8_t *ring = sm + (size_t)warp * NST * STAGE;
    auto issue = [&](int j, int stg) {
        const int c0 = t0 + (warp + nw * j) * KC, n = min(KC, t1 - c0);
        uint8_t *kt = ring + (size_t)stg * STAGE, *vt = kt + KC * PITCH;
        // the chunk's rows are consecutive in one page (chunks start at multiples of KC)
        const size_t cb = kv_row(a.kv_pages, a.kv_seq_stride, a.max_seq, m, kvh, c0, HD) * 2;
#pragma unroll
        for (int i = 0; i < KC * UNITS / 32; ++i) {
            const int u = lane + 32 * i, r = u / UNITS, c = u - r * UNITS;
            const size_t src = cb + (size_t)(r < n ? r : 0) * (HD * 2) + c * 16;
            cp_async16_zfill(kt + r * PITCH + c * 16, kb + src, r < n);
            cp_async16_zfill(vt + r * PITCH + c * 16, vb + src, r < n);
        }
        commit_group();
    };
#pragma unroll
    for (int i = 0; i < NST - 1; ++i) {
        if (i < mine) issue(i, i);
        else commit_group();
    }

    // Q fragments: rows g < rep hi, rows 8 + g lo, of head kvh * rep + g
    uint32_t qa[KS][4];
    float qv[KS][4];
    float amax = 0.f;
    const float qmul = a.scale * 1.4426950408889634f;  // log2(e)
    {
        const float *qrow = a.q + (size_t)m * a.H * HD + (size_t)(kvh * rep + (g < rep ? g : 0)) * HD;
#pragma unroll
        for (int k = 0; k < KS; ++k) {
            float2 v0 = make_float2(0.f, 0.f), v1 = v0;
            if (g < rep) {
                v0 = *reinterpret_cast<const float2 *>(qrow + 16 * k + 2 * t);
                v1 = *reinterpret_cast<const float2 *>(qrow + 16 * k + 2 * t + 8);
            }
            qv[k][0] = v0.x * qmul, qv[k][1] = v0.y * qmul, qv[k][2] = v1.x * qmul, qv[k][3] = v1.y * qmul;
#pragma unroll
            for (int e = 0; e < 4; ++e) amax = fmaxf(amax, fabsf(qv[k][e]));
        }
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    int ex = 0;
    frexpf(amax, &ex);  // amax < 2^ex
    const float qup = ldexpf(1.f, 14 - ex), qdown = ldexpf(1.f, ex - 14);
#pragma unroll
    for (int k = 0; k < KS; ++k) {
        split_half2(qv[k][0] * qup, qv[k][1] * qup, qa[k][0], qa[k][1]);
        split_half2(qv[k][2] * qup, qv[k][3] * qup, qa[k][2], qa[k][3]);
    }

    float o[NO][4];
#pragma unroll
    for (int j = 0; j < NO; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mrun = -INFINITY, lrun = 0.f;

    for (int j = 0; j < mine; ++j) {
        if (j + NST - 1 < mine) issue(j + NST - 1, (j + NST - 1) % NST);
        else commit_group();
        wait_group<NST - 1>();
        __syncwarp();
        const uint8_t *kt = ring + (size_t)(j % NST) * STAGE, *vt = kt + KC * PITCH;
        const int n = min(KC, t1 - (t0 + (warp + nw * j) * KC));
        float s[NP][4];
#pragma unroll
        for (int p = 0; p < NP; ++p) s[p][0] = s[p][1] = s[p][2] = s[p][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < HD / 32; ++kk) {
#pragma unroll
            for (int p = 0; p < NP; ++p) {
                uint32_t b[4];
                ldsm_x4(b, kt + (p * 8 + (lane & 7)) * PITCH + (kk * 32 + (lane >> 3) * 8) * 2);
                mma_16816(s[p], qa[2 * kk], b[0], b[1]);
                mma_16816(s[p], qa[2 * kk + 1], b[2], b[3]);
            }
        }
        // head g's scores of positions 8p + 2t + e: rows g (hi) + 8 + g (lo)
        float sc[NP][2], mx = -INFINITY;
#pragma unroll
        for (int p = 0; p < NP; ++p) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float v = (s[p][e] + s[p][2 + e]) * qdown;
                sc[p][e] = p * 8 + 2 * t + e < n ? v : -INFINITY;
                mx = fmaxf(mx, sc[p][e]);
            }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mnew = fmaxf(mrun, mx);
        const float corr = exp2f(mrun - mnew);
        mrun = mnew;
        float psum = 0.f;
        uint32_t pa[KC / 16][4];
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const float p0 = exp2f(sc[p][0] - mnew), p1 = exp2f(sc[p][1] - mnew);
            psum += p0 + p1;
            // k-step p / 2: regs 0 / 1 = positions 0..7 hi / lo, regs 2 / 3 = 8..15
            split_half2(p0, p1, pa[p >> 1][(p & 1) * 2], pa[p >> 1][(p & 1) * 2 + 1]);
        }
        lrun = fmaf(lrun, corr, psum);
#pragma unroll
        for (int jn = 0; jn < NO; ++jn) {
#pragma unroll
            for (int e = 0; e < 4; ++e) o[jn][e] *= corr;
        }
#pragma unroll
        for (int k2 = 0; k2 < KC / 16; ++k2) {
#pragma unroll
            for (int nd = 0; nd < HD / 16; ++nd) {
                uint32_t b[4];
                ldsm_x4_trans(b, vt + (16 * k2 + (lane & 7) + ((lane >> 3) & 1) * 8) * PITCH +
                                     (nd * 16 + (lane >> 4) * 8) * 2);
                mma_16816(o[2 * nd], pa[k2], b[0], b[1]);
                mma_16816(o[2 * nd + 1], pa[k2], b[2], b[3]);
            }
        }
        __syncwarp();  // every lane's reads of this stage are done before it is refilled
    }
    wait_group<0>();
    __syncthreads();  // every ring drained: the merge area reuses them

    // merge the warps: [warp][head][2 + HD] (max, sum, weighted V) in shared memory
    float *ms = reinterpret_cast<float *>(sm);
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 1);
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 2);
    if (g < rep) {
        float *w = ms + ((size_t)warp * rep + g) * (HD + 2);
        if (t == 0) w[0] = mrun, w[1] = lrun;
#pragma unroll
        for (int jn = 0; jn < NO; ++jn) {
            w[2 + jn * 8 + 2 * t] = o[jn][0] + o[jn][2];
            w[2 + jn * 8 + 2 * t + 1] = o[jn][1] + o[jn][3];
        }
    }
    __syncthreads();
    const bool single = a.S == 1;
    for (int i = threadIdx.x; i < rep * HD; i += blockDim.x) {
        const int hh = i / HD, d = i - hh * HD;
        float gm = -INFINITY;
        for (int w = 0; w < nw; ++w) gm = fmaxf(gm, ms[((size_t)w * rep + hh) * (HD + 2)]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < nw; ++w) {
            const float *ws = ms + ((size_t)w * rep + hh) * (HD + 2);
            const float f = ws[0] == -INFINITY ? 0.f : exp2f(ws[0] - gm);
            L = fmaf(ws[1], f, L);
            O = fmaf(ws[2 + d], f, O);
        }
        const int h = kvh * rep + hh;
        if (single) {
            a.out[(size_t)m * a.H * HD + (size_t)h * HD + d] = O / L;
        } else {
            float *pp = a.part + (((size_t)m * a.H + h) * a.S + sp) * (HD + 2);
            if (d == 0) {
                __stcg(pp, gm);
                __stcg(pp + 1, L);
            }
            __stcg(pp + 2 + d, O);
        }
    }
    if (single) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&a.counters[(size_t)m * a.Hkv + kvh], 1) == a.S - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = threadIdx.x; i < rep * HD; i += blockDim.x) {
        const int hh = i / HD, d = i - hh * HD, h = kvh * rep + hh;
        const float *base = a.part + ((size_t)m * a.H + h) * a.S * (HD + 2);
        float gm = -INFINITY;
        for (int s2 = 0; s2 < a.S; ++s2) gm = fmaxf(gm, __ldcg(base + (size_t)s2 * (HD + 2)));
        float L = 0.f, O = 0.f;
        for (int s2 = 0; s2 < a.S; ++s2) {
            const float *pj = base + (size_t)s2 * (HD + 2);
            const float mj = __ldcg(pj);
            const float f = mj == -INFINITY ? 0.f : exp2f(mj - gm);
            L = fmaf(__ldcg(pj + 1), f, L);
            O = fmaf(__ldcg(pj + 2 + d), f, O);
        }
        a.out[(size_t)m * a.H * HD + (size_t)h * HD + d] = O / L;
    }
    if (threadIdx.x == 0) a.counters[(size_t)m * a.Hkv + kvh] = 0;
}

// One staged chunk of KC positions for one warp's 16 MMA rows: scores
// against the chunk's K rows (positions at or past kmax, a per-row limit,
// masked), the base-2 online softmax of the running (mrun, lrun), and the
// P . V accumulation into o.  Rows g and 8 + g hold the f16 hi / lo halves of
// the same query, as in the decode kernel above.
template <int HD, int KC>
__device__ __forceinline__ void mma_chunk(const uint8_t *kt, const uint8_t *vt, const uint32_t (&qa)[HD / 16][4],
                                          float qdown, int kmax, int lane, float &mrun, float &lrun,
                                          float (&o)[HD / 8][4]) {
    constexpr int NP = KC / 8, NO = HD / 8, PITCH = HD * 2 + 16;
    const int t = lane & 3;
    float s[NP][4];
#pragma unroll
    for (int p = 0; p < NP; ++p) s[p][0] = s[p][1] = s[p][2] = s[p][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 32; ++kk) {
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            uint32_t b[4];
            ldsm_x4(b, kt + (p * 8 + (lane & 7)) * PITCH + (kk * 32 + (lane >> 3) * 8) * 2);
            mma_16816(s[p], qa[2 * kk], b[0], b[1]);
            mma_16816(s[p], qa[2 * kk + 1], b[2], b[3]);
        }
    }
    float sc[NP][2], mx = -INFINITY;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float v = (s[p][e] + s[p][2 + e]) * qdown;
            sc[p][e] = p * 8 + 2 * t + e < kmax ? v : -INFINITY;
            mx = fmaxf(mx, sc[p][e]);
        }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(mrun, mx);
    // a row with every position of the chunk masked keeps its state
    const float corr = mnew == -INFINITY ? 1.f : exp2f(mrun - mnew);
    float psum = 0.f;
    uint32_t pa[KC / 16][4];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const float p0 = mnew == -INFINITY ? 0.f : exp2f(sc[p][0] - mnew);
        const float p1 = mnew == -INFINITY ? 0.f : exp2f(sc[p][1] - mnew);
        psum += p0 + p1;
        split_half2(p0, p1, pa[p >> 1][(p & 1) * 2], pa[p >> 1][(p & 1) * 2 + 1]);
    }
    mrun = mnew;
    lrun = fmaf(lrun, corr, psum);
#pragma unroll
    for (int jn = 0; jn < NO; ++jn) {
#pragma unroll
        for (int e = 0; e < 4; ++e) o[jn][e] *= corr;
    }
#pragma unroll
    for (int k2 = 0; k2 < KC / 16; ++k2) {
#pragma unroll
        for (int nd = 0; nd < HD / 16; ++nd) {
            uint32_t b[4];
            ldsm_x4_trans(b, vt + (16 * k2 + (lane & 7) + ((lane >> 3) & 1) * 8) * PITCH +
                                 (nd * 16 + (lane >> 4) * 8) * 2);
            mma_16816(o[2 * nd], pa[k2], b[0], b[1]);
            mma_16816(o[2 * nd + 1], pa[k2], b[2], b[3]);
        }
    }
}

// Causal attention of one prompt chunk (T consecutive rows of one sequence
// at positions pos_const + m; the prefill case of the rows attention,
// forward_prefill_sequence, slow_ar.rs:579-593) on the tensor cores.  Grid
// (query tile, kv head); the 8 warps of a block take 8 / rep tokens each, so
// a warp's 8 MMA rows are its tokens' rep query heads (f16 hi; rows 8 + r the
// lo halves).  The block stages 32-position K/V chunks in a two-stage cp.async
// ring shared by its warps, up to its last token's position; a warp scores a
// chunk only while it holds one of its tokens' visible positions, and each
// row masks the positions past its own.  Tiles run last first (the longest
// causal ranges start in the first wave).
template <int HD>
__global__ void __launch_bounds__(256, 2) prefill_mma_attn_kernel(const RowsAttnArgs a) {
    constexpr int KC = 32, KS = HD / 16, NO = HD / 8, UNITS = HD * 2 / 16, PITCH = HD * 2 + 16;
    constexpr int STAGE = 2 * KC * PITCH;
    extern __shared__ __align__(16) uint8_t sm[];
    const int nw = blockDim.x >> 5;
    const int rep = a.H / a.Hkv, tpw = 8 / rep, qb = nw * tpw;
    const int ntiles = (a.T + qb - 1) / qb;
    const int tile = ntiles - 1 - (int)blockIdx.x, kvh = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int m0 = tile * qb, mlast = min(m0 + qb, a.T) - 1;
    const int vis_end = min(a.pos_const + mlast + 1, a.max_seq);
    const int wm0 = m0 + warp * tpw, wlast = min(wm0 + tpw, a.T) - 1;
    const int wend = wlast >= wm0 ? min(a.pos_const + wlast + 1, a.max_seq) : 0;
    const int mrow = wm0 + g / rep, h = kvh * rep + g % rep;
    const bool row_ok = mrow < a.T;
    const int prow = a.pos_const + mrow;

    const uint8_t *kb = reinterpret_cast<const uint8_t *>(a.kcache);
    const uint8_t *vb = reinterpret_cast<const uint8_t *>(a.vcache);
    const int nchunks = (vis_end + KC - 1) / KC;
    auto issue = [&](int c, int stg) {
        uint8_t *kt = sm + (size_t)stg * STAGE, *vt = kt + KC * PITCH;
        const size_t cb = kv_row(a.kv_pages, 0, a.max_seq, 0, kvh, c * KC, HD) * 2;  // one sequence
        for (int u = threadIdx.x; u < KC * UNITS; u += blockDim.x) {
            const int r = u / UNITS, cc = u - r * UNITS, key = c * KC + r;
            const bool valid = key < vis_end;
            const size_t src = cb + (size_t)(valid ? r : 0) * (HD * 2) + cc * 16;
            cp_async16_zfill(kt + r * PITCH + cc * 16, kb + src, valid);
            cp_async16_zfill(vt + r * PITCH + cc * 16, vb + src, valid);
        }
        commit_group();
    };
    if (nchunks > 0) issue(0, 0);

    // Q fragments of row g (token mrow, head h), pre-scaled as in the decode kernel
    uint32_t qa[KS][4];
    float qv[KS][4];
    float amax = 0.f;
    const float qmul = a.scale * 1.4426950408889634f;  // log2(e)
    {
        const float *qrow = a.q + (size_t)(row_ok ? mrow : 0) * a.H * HD + (size_t)h * HD;
#pragma unroll
        for (int k = 0; k < KS; ++k) {
            float2 v0 = make_float2(0.f, 0.f), v1 = v0;
            if (row_ok) {
                v0 = *reinterpret_cast<const float2 *>(qrow + 16 * k + 2 * t);
                v1 = *reinterpret_cast<const float2 *>(qrow + 16 * k + 2 * t + 8);
            }
            qv[k][0] = v0.x * qmul, qv[k][1] = v0.y * qmul, qv[k][2] = v1.x * qmul, qv[k][3] = v1.y * qmul;
#pragma unroll
            for (int e = 0; e < 4; ++e) amax = fmaxf(amax, fabsf(qv[k][e]));
        }
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    int ex = 0;
    frexpf(amax, &ex);
    const float qup = ldexpf(1.f, 14 - ex), qdown = ldexpf(1.f, ex - 14);
#pragma unroll
    for (int k = 0; k < KS; ++k) {
        split_half2(qv[k][0] * qup, qv[k][1] * qup, qa[k][0], qa[k][1]);
        split_half2(qv[k][2] * qup, qv[k][3] * qup, qa[k][2], qa[k][3]);
    }
    float o[NO][4];
#pragma unroll
    for (int j = 0; j < NO; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mrun = -INFINITY, lrun = 0.f;

    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) issue(c + 1, (c + 1) & 1);
        else commit_group();
        wait_group<1>();
        __syncthreads();  // chunk c visible to every warp
        const int c0 = c * KC;
        if (c0 < wend) {
            const uint8_t *kt = sm + (size_t)(c & 1) * STAGE;
            mma_chunk<HD, KC>(kt, kt + KC * PITCH, qa, qdown, row_ok ? prow + 1 - c0 : KC, lane, mrun, lrun, o);
        }
        __syncthreads();  // every warp's reads done before the stage is refilled
    }
    wait_group<0>();
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 1);
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 2);
    if (!row_ok) return;
    const float inv_l = 1.f / lrun;
    float *out = a.out + (size_t)mrow * a.H * HD + (size_t)h * HD;
#pragma unroll
    for (int jn = 0; jn < NO; ++jn)
        *reinterpret_cast<float2 *>(out + jn * 8 + 2 * t) =
            make_float2((o[jn][0] + o[jn][2]) * inv_l, (o[jn][1] + o[jn][3]) * inv_l);
}

template <int HD, int NST, int KC>
cudaError_t decode_mma_launch(const RowsAttnArgs &a, int warps, cudaStream_t s) {
    constexpr int PITCH = HD * 2 + 16;
    const int rep = a.H / a.Hkv;
    const size_t smem = std::max((size_t)warps * NST * 2 * KC * PITCH, (size_t)warps * rep * (HD + 2) * sizeof(float));
    const int64_t blocks = (int64_t)a.T * a.Hkv * a.S;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    // the opt-in limit is 227 KB per block, less the kernel's static 16 bytes
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    static size_t configured = 0;
    if (smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(decode_mma_attn_kernel<HD, NST, KC>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e) return e;
        configured = smem;
    }
    decode_mma_attn_kernel<HD, NST, KC><<<(unsigned)blocks, warps * 32, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

bool decode_mma_supported(const RowsAttnArgs &a, bool kv_half) {
    return kv_half && a.st && a.st_pos && a.rows_per_seq == 1 && (a.hd == 64 || a.hd == 128) && a.Hkv > 0 &&
           a.H % a.Hkv == 0 && a.H / a.Hkv <= 8 && (a.kv_seq_stride % 8) == 0 && a.q &&
           (reinterpret_cast<uintptr_t>(a.q) & 7) == 0 && (reinterpret_cast<uintptr_t>(a.kcache) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.vcache) & 15) == 0;
}

cudaError_t launch_decode_mma_attention(const RowsAttnArgs &a, cudaStream_t s) {
    if (a.T <= 0) return cudaSuccess;
    const int warps = a.decode_warps == 2 ? 2 : 4, nst = a.decode_stages == 3 ? 3 : 2;
    if (a.S <= 0 || a.S > 65535 || a.max_seq <= 0 || (a.S > 1 && (!a.part || !a.counters)))
        return cudaErrorInvalidValue;
    if (a.decode_chunk == 32) {
        if (a.hd == 64)
            return nst == 3 ? decode_mma_launch<64, 3, 32>(a, warps, s) : decode_mma_launch<64, 2, 32>(a, warps, s);
        return nst == 3 ? decode_mma_launch<128, 3, 32>(a, warps, s) : decode_mma_launch<128, 2, 32>(a, warps, s);
    }
    if (a.hd == 64)
        return nst == 3 ? decode_mma_launch<64, 3, 16>(a, warps, s) : decode_mma_launch<64, 2, 16>(a, warps, s);
    return nst == 3 ? decode_mma_launch<128, 3, 16>(a, warps, s) : decode_mma_launch<128, 2, 16>(a, warps, s);
}

bool prefill_mma_supported(const RowsAttnArgs &a, bool kv_half) {
    const int rep = a.Hkv > 0 ? a.H / a.Hkv : 0;
    return kv_half && !a.st && a.S == 1 && a.rows_per_seq >= a.T && a.T >= 1 && (a.hd == 64 || a.hd == 128) &&
           a.Hkv > 0 && a.H % a.Hkv == 0 && rep >= 1 && 8 % rep == 0 && a.q &&
           (reinterpret_cast<uintptr_t>(a.q) & 7) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 7) == 0 &&
           (reinterpret_cast<uintptr_t>(a.kcache) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.vcache) & 15) == 0 &&
           a.pos_const >= 0 && a.max_seq > 0;
}

cudaError_t launch_prefill_mma_attention(const RowsAttnArgs &a, cudaStream_t s) {
    if (a.T <= 0) return cudaSuccess;
    const int rep = a.H / a.Hkv, qb = 8 * (8 / rep);
    const unsigned tiles = (unsigned)((a.T + qb - 1) / qb);
    const size_t smem = (size_t)2 * 2 * 32 * (a.hd * 2 + 16);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(prefill_mma_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             64 * 1024);
        if (!e)
            e = cudaFuncSetAttribute(prefill_mma_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     64 * 1024);
        if (e) return e;
        configured = true;
    }
    if (a.Hkv > 65535) return cudaErrorInvalidValue;
    if (a.hd == 64) prefill_mma_attn_kernel<64><<<dim3(tiles, a.Hkv), 256, smem, s>>>(a);
    else prefill_mma_attn_kernel<128><<<dim3(tiles, a.Hkv), 256, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace s2d
