// s2d_tc_attn.cu -- the causal attention of a prompt chunk on tcgen05 (sm_100a).
//
// Replaces the attention of forward_prefill_sequence (slow_ar.rs:579-593):
// T consecutive rows of one sequence at positions pos_const + m, each
// attending over positions [0, pos_const + m] of the f16 K / V cache of its
// KV head, GQA with rep = H / Hkv query heads per KV head.
//
// One CTA takes 128 query rows of one KV head (128 / rep tokens x rep heads):
// the M of every MMA.  Positions come in tiles of 64, in one pass: S = Q K^T
// (TMEM), P = exp2(s - m) written to shared memory, O += P V (TMEM).  The
// reference max m of a row moves only when a tile's max exceeds it by more
// than 8 (base-2 units), so P stays below 2^8; then the softmax threads
// rescale the row's O in TMEM (load, multiply, store) after the previous
// P V has landed, which after the first tiles is rare.  O / sum at the end.
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

// 32 consecutive TMEM columns of this thread's lane, stored (warp-collective).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
        "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
        "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
        "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}

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
    float xl[2][kTaRows];  // each row's sum of P over the two column halves
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
        // ---- loader: the K and V tiles of every position tile ----
        if (lane == 0) {
            int issued = 0;
            for (int j = 0; j < J && !*abort_v; ++j) {
                const int s = j % kStages, use = j / kStages;
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
                mb_expect_tx(&sh.kv_full[s], kStage);
                uint8_t *st = smem + kOffKv + (size_t)s * kStage;
                tma_load_2d(st, &mk, 0, row, &sh.kv_full[s]);
                tma_load_2d(st + kKvHalf, &mk, 64, row, &sh.kv_full[s]);
                tma_load_2d(st + 2 * kKvHalf, &mv, 0, row, &sh.kv_full[s]);
                tma_load_2d(st + 3 * kKvHalf, &mv, 64, row, &sh.kv_full[s]);
                ++issued;
            }
            // no copy may still be landing when the CTA leaves
            for (int j = max(0, issued - kStages); j < issued; ++j)
                (void)mb_wait(&sh.kv_full[j % kStages], (j / kStages) & 1, abort_v, false);
        }
    } else if (warp == kTaSoftmax / 32 + 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_f16_f32(kTaRows, kTaTile);      // S: M 128, N 64, K-major
            constexpr uint32_t id_o = idesc_f16_f32_bmn(kTaRows, kTaHd);     // O: M 128, N 128, B MN-major
            const uint32_t q_hi = sbase, q_lo = sbase + 2 * kQHalf;
            // S of tile j into S buffer j & 1: Q_hi K^T + Q_lo K^T, 8 K-steps
            // of 16 over the head dim
            auto issue_s = [&](int j) -> bool {
                const int s = j % kStages, b = j & 1, buse = j >> 1;
                if (!mb_wait(&sh.kv_full[s], (j / kStages) & 1, abort_v)) return false;
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
            // S of tile j + 1 goes out before P of tile j is waited for, so
            // that the softmax of tile j overlaps the next S
            if (ok) ok = issue_s(0);
            for (int j = 0; j < J && ok; ++j) {
                if (j + 1 < J && !(ok = issue_s(j + 1))) break;
                const int s = j % kStages, pb = j & 1, puse = j >> 1;
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
                umma_commit(&sh.p_empty[pb]);  // also: O holds P V of tiles <= j
            }
            if (!ok) *abort_v = 1;
            umma_commit(&sh.o_full);  // completes once every MMA issued above has
        }
    } else {
        // ---- softmax and epilogue: warp w takes rows 32 (w % 4) + lane (its
        // TMEM lane quarter) and half ch = w / 4 of the P columns, of the Q
        // head dim and of the O columns; both threads of a row read the
        // row's whole S tile and so take the same decisions ----
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
        // the row's |q| max: the two halves meet in P buffer 1 (written only
        // after Q is complete, which needs every thread past this point)
        float *xq = reinterpret_cast<float *>(smem + kOffP + 3 * kPMat);
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
        // Online softmax in base 2 with a lazy rescale: mrow is the reference
        // max of P = 2^(s - mrow); it moves (and O and lrow are rescaled)
        // only when a tile's max exceeds it by more than 8, so P stays below
        // 2^8 and O in TMEM is rarely touched.
        float mrow = -INFINITY, lrow = 0.f;  // lrow: this thread's columns
        bool ok = true;
        for (int j = 0; j < J; ++j) {
            if (!ok) break;
            const int b = j & 1, use = j >> 1;
            const bool got = mb_wait(&sh.s_full[b], use & 1, abort_v);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float s0[32], s1[32];  // columns 0-31 and 32-63 of the S row
            tmem_ld32(lane_t + (uint32_t)(b * kTaTile), s0);  // warp-collective
            tmem_ld32(lane_t + (uint32_t)(b * kTaTile + 32), s1);
            tc_fence_before();
            mb_arrive(&sh.s_empty[b]);
            const int nvis = valid ? min(kTaTile, prow + 1 - j * kTaTile) : 0;  // positions < nvis visible
            // all of the warp's rows see the whole tile: no masks (the max is
            // exact in any order, so four independent chains change nothing)
            const bool fullw = __all_sync(0xffffffffu, nvis >= kTaTile);
            float mx = -INFINITY;
            if (fullw) {
                float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    m4[0] = fmaxf(m4[0], s0[i]), m4[1] = fmaxf(m4[1], s0[i + 1]);
                    m4[2] = fmaxf(m4[2], s1[i]), m4[3] = fmaxf(m4[3], s1[i + 1]);
                }
                mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if (i < nvis) mx = fmaxf(mx, s0[i]);
                    if (i + 32 < nvis) mx = fmaxf(mx, s1[i]);
                }
            }
            mx *= qdown;
            // P buffer pb is free once P V of tile j - 2 is done; with j >= 1
            // the wait on tile j - 1's buffer also says O holds tiles < j
            const int pb = j & 1, puse = j >> 1;
            if (puse > 0) {
                const bool free_ = mb_wait(&sh.p_empty[pb], (puse & 1) ^ 1, abort_v);
                if (!__all_sync(0xffffffffu, free_)) {
                    ok = false;
                    break;
                }
            }
            // a new reference max for this row, and the factor for O and lrow
            const bool up = mx > mrow + 8.f;
            const float mnew = up ? mx : mrow;
            const float corr = up && mrow > -INFINITY ? exp2f(mrow - mnew) : 1.f;
            if (__any_sync(0xffffffffu, corr != 1.f)) {
                // O (this thread's 64 columns) *= corr once P V of tile j - 1
                // is done; the TMEM loads and stores are warp-collective
                const int pj = j - 1, ppb = pj & 1, ppuse = pj >> 1;
                const bool ready = mb_wait(&sh.p_empty[ppb], ppuse & 1, abort_v);
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int q = 0; q < 2; ++q) {
                    float o[32];
                    const uint32_t ot = lane_t + 128u + (uint32_t)(64 * ch + 32 * q);
                    tmem_ld32(ot, o);
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] *= corr;
                    tmem_st32(ot, o);
                }
            }
            lrow *= corr;
            mrow = mnew;
            // P = 2^(s - mrow) of this thread's 32 columns into P buffer pb
            // (ch is warp-uniform: each half has its own code, no selects)
            const uint32_t p_hi = sbase + kOffP + (uint32_t)pb * 2 * kPMat;
            auto write_p = [&](const float(&sv)[32], int c0) {
                float a4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float x[8];
                    if (fullw) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) x[e] = exp2f(fmaf(sv[8 * c + e], qdown, -mrow));
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            x[e] = c0 + 8 * c + e < nvis ? exp2f(fmaf(sv[8 * c + e], qdown, -mrow)) : 0.f;
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) a4[e & 3] += x[e];
                    uint4 hi, lo;
                    split8(x, hi, lo);
                    st_shared16(p_hi + sw128(r, 4 * ch + c), hi);
                    st_shared16(p_hi + kPMat + sw128(r, 4 * ch + c), lo);
                }
                lrow += (a4[0] + a4[1]) + (a4[2] + a4[3]);
            };
            if (ch)
                write_p(s1, 32);
            else
                write_p(s0, 0);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            fence_proxy_async_smem();
            mb_arrive(&sh.p_full[pb]);
        }
        if (!ok) *abort_v = 1;
        // the row's sum over both column halves
        sh.xl[ch][r] = lrow;
        softmax_sync();
        const float inv_l = valid ? 1.f / (sh.xl[0][r] + sh.xl[1][r]) : 0.f;
        // epilogue: O row r, head-dim half ch
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
                        *reinterpret_cast<float4 *>(out + 32 * c + e) =
                            make_float4(o[e] * inv_l, o[e + 1] * inv_l, o[e + 2] * inv_l, o[e + 3] * inv_l);
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
