// s2d_tcgemm.cu -- tensor-core GEMM of the rows path on sm_100a: TMA-staged
// operands, tcgen05.mma with the accumulator in TMEM, fused epilogue.
//
// One CTA computes 128 output rows (the M of the MMA: rows of W) for a tile
// of NT activation rows (the N of the MMA: tokens or sequences), over a
// range of K.  Per K block of 64 values (one 128-byte swizzle row):
//   TMA: W tile [128][64] (and W2 for SwiGLU), hi tile [NT][64], lo tile [NT][64]
//        (128-byte swizzle, K-major) into a ring of stages;
//   MMA (one thread): 4 K-steps of 16; the hi and lo tiles sit back to back
//        in the stage, so one MMA of N = 2 NT multiplies both (accumulator
//        columns [0, NT) W.hi, [NT, 2 NT) W.lo) and the epilogue adds the
//        two halves, W.(hi + lo) = W.x in f32;
//   tcgen05.commit frees the stage when its MMAs have read it.
// The epilogue warps (TMEM lanes 0..127, one output row per thread) read the
// accumulator 32 columns at a time and apply inv[t], the residual or SwiGLU.
// Long K with few row tiles splits over a cluster of up to 8 CTAs (blockIdx.z):
// each CTA parks its partial tile in shared memory, and after a cluster
// barrier CTA z sums a slice of the columns over the cluster's CTAs in rank
// order through distributed shared memory, so the result does not depend on
// timing.
//
// Warps: 0-3 epilogue (warp 0 also owns the TMEM allocation), 4 TMA
// producer, 5 MMA issuer.  Every wait is bounded; a wait that gives up sets
// the error flag, the kernel drains its in-flight copies and MMAs (bounded)
// and frees its TMEM before returning.
#include <cuda.h>

#include "s2d_common.cuh"
#include "s2d_prefill.cuh"
#include "s2d_tcgemm.cuh"
#include "s2d_tc_common.cuh"

namespace s2d {

namespace {

constexpr int kTcThreads = 192;
constexpr int kTcRows = 128;   // output rows per CTA (UMMA M)
constexpr int kTcKBlock = 64;  // K values per stage: one 128-byte row
constexpr int kTcMaxStages = 6;
// stage memory per CTA (one CTA per SM): a deep ring keeps enough weight
// bytes in flight per SM to cover the HBM latency
constexpr int kTcStageBudget = 196 * 1024;

// 32 columns of the hi half plus the matching 32 of the lo half (off columns
// later): this lane's W.hi + W.lo for 32 tokens.
__device__ __forceinline__ void tmem_ld_sum(uint32_t taddr, int off, float (&v)[32]) {
    float lo[32];
    tmem_ld32(taddr, v);
    tmem_ld32(taddr + (uint32_t)off, lo);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += lo[j];
}

// Every thread of every CTA of the cluster (not .aligned: the producer and
// MMA lanes arrive apart from the rest of their warps).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// 4 floats of CTA `rank`'s shared memory at this CTA's address `local` (16-byte aligned).
__device__ __forceinline__ float4 ld_dsmem4(const float *local, uint32_t rank) {
    uint32_t remote;
    asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(su32(local)), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote));
    return v;
}

struct TcArgs {
    int N, K, T, ldy, ldr, epi;
    const float *inv;
    float *y;
    const float *resid;
    int32_t *error;
};

__device__ __forceinline__ float tc_epilogue(int epi, float v, float u, const float *resid) {
    if (epi == PF_STORE) return v;
    if (epi == PF_RESID) return __fadd_rn(*resid, v);
    if (epi == PF_SWIGLU_SLOW) {
        const float sig = 1.0f / (1.0f + expf(-v));
        return __fmul_rn(__fmul_rn(v, sig), u);
    }
    return __fmul_rn(v / (1.0f + expf(-v)), u);
}

template <int NT, bool DUAL>
struct TcCfg {
    static constexpr int A = kTcRows * 128;   // W tile bytes
    static constexpr int B = NT * 128;        // hi or lo tile bytes
    static constexpr int STAGE = A * (DUAL ? 2 : 1) + 2 * B;
    static constexpr int ST = kTcStageBudget / STAGE < kTcMaxStages ? kTcStageBudget / STAGE : kTcMaxStages;
    // accumulator columns per matrix: the stacked hi and lo rows (2 NT)
    static constexpr int COLS = 2 * NT * (DUAL ? 2 : 1);  // a power of two here
    static constexpr int RP = NT + 4;  // split-K partial tile row pitch (floats): conflict-free float4s
    static constexpr int RED = kTcRows * RP * 4 * (DUAL ? 2 : 1);  // split-K partial tile bytes
    static constexpr size_t SMEM = (size_t)ST * STAGE + 1024;
    static_assert(ST >= 2, "at least two stages");
    static_assert(COLS <= 512 && (COLS & (COLS - 1)) == 0, "TMEM columns");
};

template <int NT, bool DUAL>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap mw, const __grid_constant__ CUtensorMap mw2,
                   const __grid_constant__ CUtensorMap mhi, const __grid_constant__ CUtensorMap mlo, const TcArgs a) {
    using C = TcCfg<NT, DUAL>;
    extern __shared__ uint8_t tc_raw[];
    __shared__ __align__(8) uint64_t full[C::ST], empty[C::ST], done;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kTcRows, t0 = blockIdx.y * NT;
    const int nks = a.K / kTcKBlock, per = (nks + (int)gridDim.z - 1) / (int)gridDim.z;
    const int ks0 = min(nks, (int)blockIdx.z * per), nit = min(nks, ks0 + per) - ks0;
    auto stage_a = [&](int s) { return smem + (size_t)s * C::STAGE; };
    auto stage_a2 = [&](int s) { return smem + (size_t)s * C::STAGE + C::A; };
    auto stage_hi = [&](int s) { return smem + (size_t)s * C::STAGE + C::A * (DUAL ? 2 : 1); };
    auto stage_lo = [&](int s) { return stage_hi(s) + C::B; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::ST; ++i) mb_init(&full[i], 1), mb_init(&empty[i], 1);
        mb_init(&done, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_slot)),
                     "r"((uint32_t)C::COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_v = &abort_flag;

    if (warp == 4 && lane == 0) {
        // TMA producer
        int issued = 0;
        for (int i = 0; i < nit; ++i) {
            const int s = i % C::ST;
            if (i >= C::ST && !mb_wait(&empty[s], ((i / C::ST) & 1) ^ 1, abort_v)) {
                *abort_v = 1;
                break;
            }
            mb_expect_tx(&full[s], C::STAGE);
            const int x = (ks0 + i) * kTcKBlock;
            tma_load_2d(stage_a(s), &mw, x, n0, &full[s]);
            if (DUAL) tma_load_2d(stage_a2(s), &mw2, x, n0, &full[s]);
            tma_load_2d(stage_hi(s), &mhi, x, t0, &full[s]);
            tma_load_2d(stage_lo(s), &mlo, x, t0, &full[s]);
            ++issued;
        }
        // no copy may still be landing when the CTA leaves
        for (int i = max(0, issued - C::ST); i < issued; ++i)
            (void)mb_wait(&full[i % C::ST], (i / C::ST) & 1, abort_v, false);
    } else if (warp == 5 && lane == 0) {
        // MMA issuer
        // the hi and lo tiles are adjacent in the stage: one MMA of N = 2 NT
        // multiplies both (accumulator columns [0, NT) hi, [NT, 2 NT) lo)
        constexpr uint32_t idesc = idesc_f16_f32(kTcRows, 2 * NT);
        for (int i = 0; i < nit; ++i) {
            const int s = i % C::ST;
            if (!mb_wait(&full[s], (i / C::ST) & 1, abort_v)) {
                *abort_v = 1;
                break;
            }
            tc_fence_after();
            const uint64_t da = desc_k_sw128(su32(stage_a(s))), dhi = desc_k_sw128(su32(stage_hi(s)));
            const uint64_t da2 = DUAL ? desc_k_sw128(su32(stage_a2(s))) : 0ull;
#pragma unroll
            for (int k = 0; k < kTcKBlock / 16; ++k) {
                const uint64_t kk = (uint64_t)(2 * k);  // 32 bytes per K-step of 16 f16
                umma_f16(tmem, da + kk, dhi + kk, idesc, (i | k) != 0);
                if (DUAL) umma_f16(tmem + 2 * NT, da2 + kk, dhi + kk, idesc, (i | k) != 0);
            }
            umma_commit(&empty[s]);
        }
        umma_commit(&done);  // completes once every MMA issued above has
    }

    // epilogue: warps 0-3, thread = output row n0 + threadIdx.x
    const int row = threadIdx.x, n = n0 + row;
    const bool epi_thread = warp < 4;
    bool have = false;
    if (epi_thread) {
        const bool got = mb_wait(&done, 0, abort_v, false);
        if (!got) *abort_v = 1;  // reported below; the output is not written
        have = got && nit > 0;
        tc_fence_after();
        // the TMEM loads below are warp-collective: decide per warp
        have = __all_sync(0xffffffffu, have && !*abort_v);
    }
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * warp) << 16);
    if (gridDim.z == 1) {
        if (epi_thread && have) {
#pragma unroll 1
            for (int c = 0; c < NT / 32; ++c) {
                float v[32], u[32];
                tmem_ld_sum(lane_addr + c * 32, NT, v);
                if (DUAL) tmem_ld_sum(lane_addr + 2 * NT + c * 32, NT, u);
                if (n < a.N) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int t = t0 + c * 32 + j;
                        if (t < a.T) {
                            const float s = a.inv[t];
                            const float r = tc_epilogue(a.epi, v[j] * s, DUAL ? u[j] * s : 0.f,
                                                        a.resid + (size_t)t * a.ldr + n);
                            a.y[(size_t)t * a.ldy + n] = r;
                        }
                    }
                }
            }
        }
    } else {
        // split K over the cluster: each CTA parks its partial tile row-major,
        // [128][RP] (and the W2 tile after it), in its stage memory; then CTA
        // `rank` sums columns [c0, c1) over the cluster, in rank order, with
        // every rank's loads issued before the sums
        constexpr int RP = C::RP;
        float *red = reinterpret_cast<float *>(smem), *red2 = red + kTcRows * RP;
        if (epi_thread) {
#pragma unroll 1
            for (int c = 0; c < NT / 32; ++c) {
                float v[32], u[32];
                if (have) {
                    tmem_ld_sum(lane_addr + c * 32, NT, v);
                    if (DUAL) tmem_ld_sum(lane_addr + 2 * NT + c * 32, NT, u);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0.f, u[j] = 0.f;
                }
                float4 *dst = reinterpret_cast<float4 *>(red + (size_t)row * RP + c * 32);
                float4 *dst2 = reinterpret_cast<float4 *>(red2 + (size_t)row * RP + c * 32);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    if (DUAL) dst2[q] = make_float4(u[4 * q], u[4 * q + 1], u[4 * q + 2], u[4 * q + 3]);
                }
            }
        }
        cluster_sync_all();
        uint32_t rank;
        asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
        const int ks = (int)gridDim.z, share = ((NT / 4 + ks - 1) / ks) * 4;
        const int c0 = (int)rank * share, c1 = min(NT, c0 + share);
        if (epi_thread && n < a.N && !*abort_v) {
            for (int c = c0; c < c1; c += 4) {
                if (t0 + c >= a.T) break;
                float4 pv[8], pu[8];
#pragma unroll
                for (int z = 0; z < 8; ++z)
                    if (z < ks) {
                        pv[z] = ld_dsmem4(red + (size_t)row * RP + c, (uint32_t)z);
                        if (DUAL) pu[z] = ld_dsmem4(red2 + (size_t)row * RP + c, (uint32_t)z);
                    }
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f), u = v;
#pragma unroll
                for (int z = 0; z < 8; ++z)
                    if (z < ks) {
                        v.x += pv[z].x, v.y += pv[z].y, v.z += pv[z].z, v.w += pv[z].w;
                        if (DUAL) u.x += pu[z].x, u.y += pu[z].y, u.z += pu[z].z, u.w += pu[z].w;
                    }
                const float vv[4] = {v.x, v.y, v.z, v.w}, uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int t = t0 + c + q;
                    if (t < a.T) {
                        const float sc = a.inv[t];
                        a.y[(size_t)t * a.ldy + n] =
                            tc_epilogue(a.epi, vv[q] * sc, uu[q] * sc, a.resid + (size_t)t * a.ldr + n);
                    }
                }
            }
        }
        cluster_sync_all();  // no CTA leaves while its partials may be read
    }
    if (threadIdx.x == 0 && *abort_v && a.error) atomicCAS(a.error, 0, kErrTcWait);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::COLS));
    }
}

// Clusters of `ks` CTAs of this kernel that can be resident at once.
template <int NT, bool DUAL>
int tc_max_clusters(int ks) {
    static int cache[9] = {0};
    if (ks < 1 || ks > 8) return 0;
    if (cache[ks]) return cache[ks];
    using C = TcCfg<NT, DUAL>;
    if (cudaFuncSetAttribute(tc_gemm_kernel<NT, DUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM))
        return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, (unsigned)ks);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = (unsigned)ks;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<NT, DUAL>, &cfg) != cudaSuccess) n = 0;
    return cache[ks] = n;
}

// The split-K factor: the most CTAs that still run in one wave (every
// cluster resident at once), every CTA of a cluster with K blocks.
template <int NT, bool DUAL>
int tc_pick_ks(int tiles, int nks) {
    int best = 1;
    long best_ctas = 0;
    for (int ks = 1; ks <= std::min(8, nks); ++ks) {
        const int per = (nks + ks - 1) / ks, k2 = (nks + per - 1) / per;
        if (k2 != ks) continue;
        const int cap = tc_max_clusters<NT, DUAL>(ks);
        if (cap < tiles && ks > 1) continue;
        const long ctas = (long)std::min(tiles, std::max(cap, 1)) * ks;
        if (ctas > best_ctas) best = ks, best_ctas = ctas;
    }
    return best;
}

template <int NT, bool DUAL>
cudaError_t tc_launch(const TcGemm &g, cudaStream_t s, int ks) {
    using C = TcCfg<NT, DUAL>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<NT, DUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)C::SMEM);
        if (e) return e;
        configured = true;
    }
    if (ks > 1 && (size_t)C::RED > (size_t)C::ST * C::STAGE) return cudaErrorInvalidValue;
    CUtensorMap mw, mw2, mhi, mlo;
    if (!sw128_map(&mw, g.W, g.N, g.K, kTcRows) || !sw128_map(&mw2, DUAL ? g.W2 : g.W, g.N, g.K, kTcRows) ||
        !sw128_map(&mhi, g.xs, g.T, g.K, NT) || !sw128_map(&mlo, g.xs + (size_t)g.T * g.K, g.T, g.K, NT))
        return cudaErrorInvalidValue;
    TcArgs a{g.N, g.K, g.T, g.ldy, g.ldr, g.epi, g.inv, g.y, g.resid ? g.resid : g.y, g.error};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((g.N + kTcRows - 1) / kTcRows), (unsigned)((g.T + NT - 1) / NT), (unsigned)ks);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = (unsigned)ks;
    cfg.attrs = attr;
    cfg.numAttrs = ks > 1 ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<NT, DUAL>, mw, mw2, mhi, mlo, a);
}

}  // namespace

bool tc_gemm_supported(const TcGemm &g) {
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const bool dual = g.epi == PF_SWIGLU_SLOW || g.epi == PF_SWIGLU_FAST;
    return encode_fn() && g.K >= kTcKBlock && g.K % kTcKBlock == 0 && g.N >= 1 && g.T >= 1 && g.T <= 4096 &&
           g.W && al16(g.W) && g.xs && al16(g.xs) && (!dual || (g.W2 && al16(g.W2))) && g.inv && g.y;
}

cudaError_t launch_tc_gemm(const TcGemm &g, cudaStream_t s) {
    if (!tc_gemm_supported(g)) return cudaErrorInvalidValue;
    const bool dual = g.epi == PF_SWIGLU_SLOW || g.epi == PF_SWIGLU_FAST;
    const int NT = g.T <= 64 ? 64 : 128;
    const int tiles = ((g.N + kTcRows - 1) / kTcRows) * ((g.T + NT - 1) / NT);
    const int nks = g.K / kTcKBlock;
    if (NT == 64)
        return dual ? tc_launch<64, true>(g, s, tc_pick_ks<64, true>(tiles, nks))
                    : tc_launch<64, false>(g, s, tc_pick_ks<64, false>(tiles, nks));
    return dual ? tc_launch<128, true>(g, s, tc_pick_ks<128, true>(tiles, nks))
                : tc_launch<128, false>(g, s, tc_pick_ks<128, false>(tiles, nks));
}

}  // namespace s2d
