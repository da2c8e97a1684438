// s2d_tc_attn.cu -- the causal attention of a prompt chunk on tcgen05 (sm_100a).
//
// Replaces the attention of forward_prefill_sequence (slow_ar.rs:579-593):
// T consecutive rows of one sequence at positions pos_const + m, each
// attending over positions [0, pos_const + m] of the f16 K / V cache of its
// KV head, GQA with rep = H / Hkv query heads per KV head.
//
// One CTA takes 128 query rows of one KV head (128 / rep tokens x rep heads):
// the M of every MMA.  Positions come in tiles of 64.  Two passes over the
// tiles, so that the output accumulator never needs rescaling:
//   pass 1: S = Q K^T (TMEM), and each row's running max and sum of
//           exp2(s - max) in the softmax threads;
//   pass 2: S = Q K^T again, P = exp2(s - max) / sum written to shared
//           memory, O += P V in TMEM.
// Q and P enter the MMAs as f16 hi + lo pairs (two MMAs accumulating into
// the same TMEM tile), K and V are the cache's f16: about 22 bits of the
// f32 operands with f32 accumulation, the precision of the CUDA-core path.
// As in the mma.sync kernel, each query row is pre-scaled by
// scale * log2(e) and a power of two that puts its largest element near
// 2^14, taken out of the scores exactly, and the softmax runs in base 2.
//
// Warps: 0-7 softmax and epilogue (warps w and w + 4 share TMEM lane quarter
// w, rows 32 w + lane, and take column halves 0 and 1 of every S tile; warp
// 0 also owns the TMEM allocation), 8 the loader (TMA: K and V tiles, one
// 64-position tile = two [64 rows][64 f16] boxes of 128-byte swizzle per
// matrix), 9 the MMA issuer, which issues tile j + 1's S before it waits for
// tile j's P.  TMEM: S in two buffers of 64 columns, O in 128.
// Every wait is bounded; a wait that gives up sets the error flag and the
// CTA drains its copies and MMAs (bounded) and frees its TMEM before leaving.
//
// Shared memory (from a 1024-byte aligned base), all 128-byte swizzled:
//   Q hi, Q lo        [128 rows][128 f16], K-major, two 16 KB halves each;
//   3 K/V stages      K [64 positions][128 f16] (two 8 KB halves, K-major),
//                     V [64 positions][128 f16] (the same bytes read
//                     MN-major by the P V MMA);
//   2 P buffers       P hi, P lo [128 rows][64 positions] (16 KB each).
#include <cuda.h>
#include <cuda_fp16.h>
#include <math.h>

#include "s2d_common.cuh"
#include "s2d_prefill.cuh"
#include "s2d_tc_common.cuh"
#include "s2d_tcgemm.cuh"

namespace s2d {

namespace {

constexpr int kTaRows = 128;   // query rows per CTA: the UMMA M
constexpr int kTaTile = 64;    // positions per K / V tile
constexpr int kTaHd = 128;     // head dim
constexpr int kTaSoftmax = 256;  // softmax threads: warps 0-7, two per TMEM lane quarter
constexpr int kTaThreads = kTaSoftmax + 64;  // + the loader warp and the MMA warp
constexpr int kQHalf = kTaRows * 64 * 2;               // 16 KB: one 64-column half of Q hi or lo
constexpr int kKvHalf = kTaTile * 64 * 2;              // 8 KB: one 64-column half of a K or V tile
constexpr int kStage = 4 * kKvHalf;                    // K halves, then V halves
constexpr int kPMat = kTaRows * kTaTile * 2;           // 16 KB: P hi or P lo
constexpr int kOffKv = 4 * kQHalf;                     // after Q hi, Q lo
constexpr int kStages = 3;                             // K / V stages
constexpr int kOffP = kOffKv + kStages * kStage;
constexpr int kTaSmem = kOffP + 2 * 2 * kPMat;         // 229,376 B
constexpr uint32_t kTaCols = 256;                      // TMEM: S0 [0, 64), S1 [64, 128), O [128, 256)

// Byte offset of 16-byte chunk c (of 8 f16) of row r in a 128-byte-swizzled
// region of 128-byte rows.
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// x = hi + lo with hi = f16(x), lo = f16(x - hi), for 8 values.
__device__ __forceinline__ void split8(const float *x, uint4 &hi, uint4 &lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 hh = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        const float2 hf = __half22float2(hh);
        h[i] = *reinterpret_cast<const uint32_t *>(&hh);
        l[i] = pack2(x[2 * i] - hf.x, x[2 * i + 1] - hf.y);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void st_shared16(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

struct TaShared {
    uint64_t kv_full[kStages], kv_empty[kStages], s_full[2], s_empty[2], p_full[2], p_empty[2], q_full, o_full;
    uint32_t tmem;
    int abort;
};

// The softmax threads' own barrier (warps 0-7).
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kTaSoftmax) : "memory"); }

__global__ void __launch_bounds__(kTaThreads, 1)
    prefill_tc_attn_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv,
                           const RowsAttnArgs a) {
    extern __shared__ uint8_t ta_raw[];
    __shared__ TaShared sh;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(ta_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = su32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rep = a.H / a.Hkv, qb = kTaRows / rep;  // tokens per CTA
    const int ntiles = (a.T + qb - 1) / qb;
    const int tile = ntiles - 1 - (int)blockIdx.x, kvh = blockIdx.y;  // longest causal ranges first
    const int m0 = tile * qb, mlast = min(m0 + qb, a.T) - 1;
    const int vis_end = min(a.pos_const + mlast + 1, a.max_seq);  // positions [0, vis_end) are read
    const int J = (vis_end + kTaTile - 1) / kTaTile;               // K / V tiles per pass
    volatile int *abort_v = &sh.abort;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) mb_init(&sh.kv_full[i], 1), mb_init(&sh.kv_empty[i], 1);
        for (int i = 0; i < 2; ++i) {
            mb_init(&sh.s_full[i], 1), mb_init(&sh.s_empty[i], kTaSoftmax);
            mb_init(&sh.p_full[i], kTaSoftmax), mb_init(&sh.p_empty[i], 1);
        }
        mb_init(&sh.q_full, kTaSoftmax), mb_init(&sh.o_full, 1);
        sh.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&sh.tmem)),
                     "r"(kTaCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem;

    if (warp == kTaSoftmax / 32) {
        // ---- loader: K tiles (pass 1), K and V tiles (pass 2) ----
        if (lane == 0) {
            int issued = 0;
            for (int v = 0; v < 2 * J && !*abort_v; ++v) {
                const int s = v % kStages, use = v / kStages, j = v % J;
                const bool pass2 = v >= J;
                if (use > 0 && !mb_wait(&sh.kv_empty[s], (use & 1) ^ 1, abort_v)) {
                    *abort_v = 1;
                    break;
                }
                // the tile's first cache row: paged (64-position pages of one
                // sequence, the tile inside one page) or contiguous
                int row;
                if (a.kv_pages.pages)
                    row = a.kv_pages.pages[j] * (int)(a.kv_pages.page_elems / kTaHd) + kvh * kTaTile;
                else
                    row = kvh * a.max_seq + j * kTaTile;
                mb_expect_tx(&sh.kv_full[s], pass2 ? kStage : 2 * kKvHalf);
                uint8_t *st = smem + kOffKv + (size_t)s * kStage;
                tma_load_2d(st, &mk, 0, row, &sh.kv_full[s]);
                tma_load_2d(st + kKvHalf, &mk, 64, row, &sh.kv_full[s]);
                if (pass2) {
                    tma_load_2d(st + 2 * kKvHalf, &mv, 0, row, &sh.kv_full[s]);
                    tma_load_2d(st + 3 * kKvHalf, &mv, 64, row, &sh.kv_full[s]);
                }
                ++issued;
            }
            // no copy may still be landing when the CTA leaves
            for (int v = max(0, issued - kStages); v < issued; ++v)
                (void)mb_wait(&sh.kv_full[v % kStages], (v / kStages) & 1, abort_v, false);
        }
    } else if (warp == kTaSoftmax / 32 + 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_f16_f32(kTaRows, kTaTile);      // S: M 128, N 64, K-major
            constexpr uint32_t id_o = idesc_f16_f32_bmn(kTaRows, kTaHd);     // O: M 128, N 128, B MN-major
            const uint32_t q_hi = sbase, q_lo = sbase + 2 * kQHalf;
            // S of use v (tile v % J) into S buffer v & 1: Q_hi K^T + Q_lo K^T,
            // 8 K-steps of 16 over the head dim
            auto issue_s = [&](int v) -> bool {
                const int s = v % kStages, b = v & 1, buse = v >> 1;
                if (!mb_wait(&sh.kv_full[s], (v / kStages) & 1, abort_v)) return false;
                if (buse > 0 && !mb_wait(&sh.s_empty[b], (buse & 1) ^ 1, abort_v)) return false;
                tc_fence_after();
                const uint32_t kst = sbase + kOffKv + (uint32_t)s * kStage;
#pragma unroll
                for (int kk = 0; kk < kTaHd / 16; ++kk) {
                    const uint32_t half = (uint32_t)(kk >> 2), off = (uint32_t)((kk & 3) * 32);
                    const uint64_t dk = desc_k_sw128(kst + half * kKvHalf + off);
                    umma_f16(tmem + (uint32_t)(b * kTaTile), desc_k_sw128(q_hi + half * kQHalf + off), dk, id_s,
                             kk > 0);
                    umma_f16(tmem + (uint32_t)(b * kTaTile), desc_k_sw128(q_lo + half * kQHalf + off), dk, id_s, 1);
                }
                umma_commit(&sh.s_full[b]);
                return true;
            };
            bool ok = mb_wait(&sh.q_full, 0, abort_v);
            tc_fence_after();
            // pass 1: S only; its K stage is free once the MMAs have read it
            for (int v = 0; v < J && ok; ++v) {
                ok = issue_s(v);
                if (ok) umma_commit(&sh.kv_empty[v % kStages]);
            }
            // pass 2: S of tile j + 1 goes out before P of tile j is waited
            // for, so that the softmax of tile j overlaps the next S
            if (ok) ok = issue_s(J);
            for (int j = 0; j < J && ok; ++j) {
                if (j + 1 < J && !(ok = issue_s(J + j + 1))) break;
                const int v = J + j, s = v % kStages, pb = j & 1, puse = j >> 1;
                if (!(ok = mb_wait(&sh.p_full[pb], puse & 1, abort_v))) break;
                tc_fence_after();
                // O += P_hi V + P_lo V: 4 K-steps of 16 positions
                const uint32_t p_hi = sbase + kOffP + (uint32_t)pb * 2 * kPMat, p_lo = p_hi + kPMat;
                const uint32_t vst = sbase + kOffKv + (uint32_t)s * kStage + 2 * kKvHalf;
#pragma unroll
                for (int kk = 0; kk < kTaTile / 16; ++kk) {
                    const uint64_t dv = desc_mn_sw128(vst + (uint32_t)kk * 2048u, kKvHalf);
                    umma_f16(tmem + 128, desc_k_sw128(p_hi + (uint32_t)kk * 32u), dv, id_o, (j | kk) != 0);
                    umma_f16(tmem + 128, desc_k_sw128(p_lo + (uint32_t)kk * 32u), dv, id_o, 1);
                }
                umma_commit(&sh.kv_empty[s]);
                umma_commit(&sh.p_empty[pb]);
            }
            if (!ok) *abort_v = 1;
            umma_commit(&sh.o_full);  // completes once every MMA issued above has
        }
    } else {
        // ---- softmax and epilogue: warp w takes rows 32 (w % 4) + lane (its
        // TMEM lane quarter) and column half ch = w / 4 of every S tile, the
        // Q head-dim half ch and the O head-dim half ch ----
        const int r = 32 * (warp & 3) + lane, ch = warp >> 2;
        const int m = m0 + r / rep, h = kvh * rep + r % rep;
        const bool valid = m < a.T;
        const int prow = a.pos_const + m;  // the row's own position: it sees [0, prow]
        const float qmul = a.scale * 1.4426950408889634f;  // log2(e)
        const float *qrow = a.q + (size_t)(valid ? m : 0) * a.H * kTaHd + (size_t)h * kTaHd + 64 * ch;
        float amax = 0.f;
        for (int c = 0; c < 16; ++c) {
            const float4 v = valid ? reinterpret_cast<const float4 *>(qrow)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        // row exchanges between the column halves go through P buffer 1 (free
        // until pass 2 writes it, which every softmax thread does only after
        // the barrier that closes the exchange)
        float *xq = reinterpret_cast<float *>(smem + kOffP + 3 * kPMat), *xl = xq + 2 * kTaRows;
        xq[ch * kTaRows + r] = amax;
        softmax_sync();
        amax = fmaxf(xq[r], xq[kTaRows + r]) * qmul;
        int ex = 0;
        frexpf(amax, &ex);
        const float qup = ldexpf(qmul, 14 - ex), qdown = ldexpf(1.f, ex - 14);
        // this thread's Q half, scaled, split, written 128-byte swizzled
        for (int c = 0; c < 8; ++c) {
            const float4 v0 = valid ? reinterpret_cast<const float4 *>(qrow)[2 * c] : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 v1 = valid ? reinterpret_cast<const float4 *>(qrow)[2 * c + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
            float x[8] = {v0.x * qup, v0.y * qup, v0.z * qup, v0.w * qup, v1.x * qup, v1.y * qup, v1.z * qup, v1.w * qup};
            uint4 hi, lo;
            split8(x, hi, lo);
            const uint32_t off = (uint32_t)(ch * kQHalf) + sw128(r, c);
            st_shared16(sbase + off, hi);
            st_shared16(sbase + 2 * kQHalf + off, lo);
        }
        fence_proxy_async_smem();
        mb_arrive(&sh.q_full);
        const uint32_t lane_t = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        float mrow = -INFINITY, lrow = 0.f;  // over this thread's columns; both halves after pass 1
        bool ok = true;
        for (int v = 0; v < 2 * J; ++v) {
            const int b = v & 1, use = v >> 1, j = v % J;
            const bool pass2 = v >= J;
            if (v == J) {
                // both column halves' (max, sum) of each row
                xq[ch * kTaRows + r] = mrow, xl[ch * kTaRows + r] = lrow;
                softmax_sync();
                const float m2 = xq[(ch ^ 1) * kTaRows + r], l2 = xl[(ch ^ 1) * kTaRows + r];
                softmax_sync();  // every exchange read before P buffer 1 is written
                const float mm = fmaxf(mrow, m2);
                if (mm > -INFINITY) {
                    lrow = (mrow > -INFINITY ? lrow * exp2f(mrow - mm) : 0.f) + (m2 > -INFINITY ? l2 * exp2f(m2 - mm) : 0.f);
                    mrow = mm;
                }
            }
            // after a failed wait the loop runs on without work, so that every
            // softmax warp reaches the barrier between the passes
            if (!ok) continue;
            const bool got = mb_wait(&sh.s_full[b], use & 1, abort_v);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                continue;
            }
            tc_fence_after();
            float s[32];
            tmem_ld32(lane_t + (uint32_t)(b * kTaTile + 32 * ch), s);  // warp-collective
            tc_fence_before();
            mb_arrive(&sh.s_empty[b]);
            const int t0 = j * kTaTile + 32 * ch, nvis = valid ? min(32, prow + 1 - t0) : 0;  // positions < nvis visible
            if (!pass2) {
                float mx = -INFINITY;
                if (nvis >= 32) {  // the whole half visible: no per-position mask
#pragma unroll
                    for (int i = 0; i < 32; ++i) mx = fmaxf(mx, s[i]);
                    mx *= qdown;
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (i < nvis) mx = fmaxf(mx, s[i] * qdown);
                }
                if (mx > -INFINITY) {
                    const float mnew = fmaxf(mrow, mx);
                    float acc = 0.f;
                    if (nvis >= 32) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) acc += exp2f(fmaf(s[i], qdown, -mnew));
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i < nvis) acc += exp2f(fmaf(s[i], qdown, -mnew));
                    }
                    lrow = fmaf(lrow, exp2f(mrow - mnew), acc);
                    mrow = mnew;
                }
                continue;
            }
            // pass 2: P = exp2(s - max) / sum into P buffer pb, row r, chunks 4 ch ..
            const int pb = j & 1, puse = j >> 1;
            if (puse > 0) {
                const bool free_ = mb_wait(&sh.p_empty[pb], (puse & 1) ^ 1, abort_v);
                if (!__all_sync(0xffffffffu, free_)) {
                    ok = false;
                    continue;
                }
            }
            const float inv_l = lrow > 0.f ? 1.f / lrow : 0.f;
            const uint32_t p_hi = sbase + kOffP + (uint32_t)pb * 2 * kPMat;
            const bool full = nvis >= 32;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float x[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int i = 8 * c + e;
                    x[e] = full || i < nvis ? exp2f(fmaf(s[i], qdown, -mrow)) * inv_l : 0.f;
                }
                uint4 hi, lo;
                split8(x, hi, lo);
                st_shared16(p_hi + sw128(r, 4 * ch + c), hi);
                st_shared16(p_hi + kPMat + sw128(r, 4 * ch + c), lo);
            }
            fence_proxy_async_smem();
            mb_arrive(&sh.p_full[pb]);
        }
        if (!ok) *abort_v = 1;
        // epilogue: O row r, head-dim half ch, normalised already
        const bool done = mb_wait(&sh.o_full, 0, abort_v, false);
        tc_fence_after();
        if (__all_sync(0xffffffffu, done && !*abort_v)) {  // warp-uniform: the loads are collective
            float *out = a.out + (size_t)(valid ? m : 0) * a.H * kTaHd + (size_t)h * kTaHd + 64 * ch;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                float o[32];
                tmem_ld32(lane_t + 128u + (uint32_t)(64 * ch + 32 * c), o);  // warp-collective
                if (valid) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4 *>(out + 32 * c + e) = make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]);
                }
            }
        }
    }
    if (threadIdx.x == 0 && *abort_v && a.error) atomicCAS(a.error, 0, kErrTcWait);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTaCols));
    }
}

}  // namespace

bool prefill_tc_supported(const RowsAttnArgs &a, bool kv_half) {
    const int rep = a.Hkv > 0 ? a.H / a.Hkv : 0;
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return kv_half && !a.st && a.S == 1 && a.rows_per_seq >= a.T && a.T >= 1 && a.hd == kTaHd && a.Hkv > 0 &&
           a.H % a.Hkv == 0 && rep >= 1 && kTaRows % rep == 0 && a.q && al16(a.q) && a.out && al16(a.out) &&
           al16(a.kcache) && al16(a.vcache) && a.k_rows > 0 && a.v_rows > 0 && a.k_rows < (1ull << 31) &&
           a.v_rows < (1ull << 31) && a.pos_const >= 0 && a.max_seq > 0 && encode_fn() &&
           (!a.kv_pages.pages || a.kv_pages.page_elems % kTaHd == 0);
}

cudaError_t launch_prefill_tc_attention(const RowsAttnArgs &a, cudaStream_t s) {
    if (a.T <= 0) return cudaSuccess;
    if (!prefill_tc_supported(a, true)) return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        cudaError_t e =
            cudaFuncSetAttribute(prefill_tc_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTaSmem + 1024);
        if (e) return e;
        configured = true;
    }
    CUtensorMap mk, mv;
    if (!sw128_map(&mk, a.kcache, (int)a.k_rows, kTaHd, kTaTile) || !sw128_map(&mv, a.vcache, (int)a.v_rows, kTaHd, kTaTile))
        return cudaErrorInvalidValue;
    const int rep = a.H / a.Hkv, qb = kTaRows / rep;
    const unsigned tiles = (unsigned)((a.T + qb - 1) / qb);
    if (a.Hkv > 65535) return cudaErrorInvalidValue;
    prefill_tc_attn_kernel<<<dim3(tiles, (unsigned)a.Hkv), kTaThreads, kTaSmem + 1024, s>>>(mk, mv, a);
    return cudaGetLastError();
}

}  // namespace s2d
