// s2d_codec_conv.cu -- the codec decoder's causal convolutions on tcgen05 as
// implicit GEMMs: no im2col copy.
//
// Z[t][n] = sum over taps k and channels c of P[t + k d][c] . W[n][k Cp + c],
// with P the convolution's padded f16 input ([T + (K - 1) d][C], rounded to
// f16 as the reference rounds it, codec.rs:2257-2259) and W the weights laid
// out [N][K Cp] (Cp = C rounded up to 64, zero columns past C).
//
// One CTA computes a tile of 128 output rows (the M of the MMA) by NT output
// channels.  Its K loop runs over (tap, 64-channel block): the TMA producer
// loads the activation tile straight from P at row t0 + k d (a 2D box of
// [128][64] f16 with 128-byte swizzle; channels past C and rows past the end
// read as zeros) and the weight tile [NT][64]; one thread issues the 4
// K-steps of tcgen05.mma (kind::f16, f32 accumulator in TMEM); the epilogue
// warps read the accumulator back with tcgen05.ld and store it through
// shared memory, so that each global store is a whole 128-byte row piece.
// Two CTAs per SM, so that one's epilogue overlaps the other's main loop.
// (An epilogue that also applied the next bias, snake and f16 rounding, or
// the residual add, measured slower than the separate full-occupancy
// kernels: four epilogue warps per CTA cannot hide those loads and sines.)
//
// Warps: 0-3 epilogue (warp 0 owns the TMEM allocation), 4 TMA producer, 5
// MMA issuer.  Every wait is bounded; a wait that gives up sets the error
// flag, the kernel waits (bounded) for its copies in flight and frees its TMEM.
#include <cuda.h>

#include "s2d_codec.cuh"
#include "s2d_tc_common.cuh"

namespace s2d {

namespace {

constexpr int kCvThreads = 192;
constexpr int kCvRows = 128;  // output rows per CTA (UMMA M)
constexpr int kCvKB = 64;     // channels per K block: one 128-byte swizzle row
// stage memory per CTA: two CTAs per SM with ~100 KB each, or one with ~200 KB
template <int NT, int CTAS>
struct CvCfg {
    static constexpr int kBudget = CTAS == 2 ? 100 * 1024 : 200 * 1024;
    static constexpr int A = kCvRows * 128;  // activation tile bytes
    static constexpr int B = NT * 128;       // weight tile bytes
    static constexpr int STAGE = A + B;
    static constexpr int ST = kBudget / STAGE < 6 ? kBudget / STAGE : 6;
    static constexpr int COLS = NT <= 32 ? 32 : NT <= 64 ? 64 : NT <= 128 ? 128 : 256;  // TMEM columns
    static constexpr size_t SMEM = (size_t)ST * STAGE + 1024;
    static_assert(ST >= 2, "at least two stages");
    static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "UMMA N for M = 128");
};

struct CvArgs {
    int T, N, taps, d, cpb;  // output rows, output channels, taps, dilation, 64-channel blocks per tap
    float *Z;                // [T][N]
    int32_t *error;
};

template <int NT, int CTAS>
__global__ void __launch_bounds__(kCvThreads, CTAS)
    conv_tc_kernel(const __grid_constant__ CUtensorMap mp, const __grid_constant__ CUtensorMap mw, const CvArgs a) {
    using C = CvCfg<NT, CTAS>;
    extern __shared__ uint8_t cv_raw[];
    __shared__ __align__(8) uint64_t full[C::ST], empty[C::ST], done;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(cv_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kCvRows, n0 = blockIdx.y * NT;
    const int nit = a.taps * a.cpb;
    auto stage_a = [&](int s) { return smem + (size_t)s * C::STAGE; };
    auto stage_b = [&](int s) { return smem + (size_t)s * C::STAGE + C::A; };

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
        // TMA producer: K block i = tap i / cpb, channels 64 (i % cpb) ..
        int issued = 0;
        for (int i = 0; i < nit; ++i) {
            const int s = i % C::ST;
            if (i >= C::ST && !mb_wait(&empty[s], ((i / C::ST) & 1) ^ 1, abort_v)) {
                *abort_v = 1;
                break;
            }
            const int tap = i / a.cpb, cb = i - tap * a.cpb;
            mb_expect_tx(&full[s], C::STAGE);
            tma_load_2d(stage_a(s), &mp, cb * kCvKB, t0 + tap * a.d, &full[s]);
            tma_load_2d(stage_b(s), &mw, i * kCvKB, n0, &full[s]);
            ++issued;
        }
        // no copy may still be landing when the CTA leaves
        for (int i = max(0, issued - C::ST); i < issued; ++i)
            (void)mb_wait(&full[i % C::ST], (i / C::ST) & 1, abort_v, false);
    } else if (warp == 5 && lane == 0) {
        // MMA issuer: D[128][NT] += A[128][64] . B[NT][64]^T per K block
        constexpr uint32_t idesc = idesc_f16_f32(kCvRows, NT);
        for (int i = 0; i < nit; ++i) {
            const int s = i % C::ST;
            if (!mb_wait(&full[s], (i / C::ST) & 1, abort_v)) {
                *abort_v = 1;
                break;
            }
            tc_fence_after();
            const uint64_t da = desc_k_sw128(su32(stage_a(s))), db = desc_k_sw128(su32(stage_b(s)));
#pragma unroll
            for (int k = 0; k < kCvKB / 16; ++k) {
                const uint64_t kk = (uint64_t)(2 * k);  // 32 bytes per K-step of 16 f16
                umma_f16(tmem, da + kk, db + kk, idesc, (i | k) != 0);
            }
            umma_commit(&empty[s]);
        }
        umma_commit(&done);  // completes once every MMA issued above has
    }

    // epilogue: warps 0-3, thread = output row t0 + threadIdx.x
    if (warp < 4) {
        const bool got = mb_wait(&done, 0, abort_v, false);
        if (!got) *abort_v = 1;
        tc_fence_after();
        if (__all_sync(0xffffffffu, got && nit > 0 && !*abort_v)) {  // the TMEM loads are warp-collective
            // Per 32-column chunk the warp parks its 32 rows x 32 accumulator
            // columns in shared memory (the stage ring is free once `done`
            // has fired: every MMA has read its operands and every copy has
            // landed), then walks the rows with lane = column, so that every
            // global load and store of the epilogue is one contiguous row piece.
            float *park = reinterpret_cast<float *>(smem) + warp * 32 * 33;
            const uint32_t lane_addr = tmem + ((uint32_t)(32 * warp) << 16);
            const int r0 = t0 + 32 * warp;
#pragma unroll 1
            for (int c = 0; c < NT / 32; ++c) {
                float v[32];
                tmem_ld32(lane_addr + (uint32_t)(c * 32), v);
#pragma unroll
                for (int j = 0; j < 32; ++j) park[lane * 33 + j] = v[j];
                __syncwarp();
                const int n = n0 + c * 32 + lane;
                const int rows = min(32, a.T - r0);  // rows of this warp inside the output
#pragma unroll
                for (int rr = 0; rr < 32; ++rr)
                    if (rr < rows) a.Z[(size_t)(r0 + rr) * a.N + n] = park[rr * 33 + lane];
                __syncwarp();
            }
        }
    }
    if (threadIdx.x == 0 && *abort_v && a.error) atomicCAS(a.error, 0, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::COLS));
    }
}

template <int NT, int CTAS>
cudaError_t launch_nt(const CodecConv &cv, cudaStream_t s) {
    using C = CvCfg<NT, CTAS>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel<NT, CTAS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)C::SMEM);
        if (e) return e;
        configured = true;
    }
    const int cp = cv.cpb * kCvKB;
    CUtensorMap mp, mw;
    if (!sw128_map(&mp, cv.P, cv.T + (cv.taps - 1) * cv.d, cv.C, kCvRows) ||
        !sw128_map(&mw, cv.W, cv.N, cv.taps * cp, NT))
        return cudaErrorInvalidValue;
    CvArgs a{cv.T, cv.N, cv.taps, cv.d, cv.cpb, cv.Z, cv.error};
    const dim3 grid((unsigned)((cv.T + kCvRows - 1) / kCvRows), (unsigned)(cv.N / NT));
    conv_tc_kernel<NT, CTAS><<<grid, kCvThreads, C::SMEM, s>>>(mp, mw, a);
    return cudaGetLastError();
}

}  // namespace

int codec_conv_tile(int N) {
    return N % 256 == 0 ? 256 : N % 192 == 0 ? 192 : N % 128 == 0 ? 128 : N % 96 == 0 ? 96 : N % 64 == 0 ? 64 : 0;
}

bool codec_conv_supported(const CodecConv &cv) {
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return cv.P && cv.W && cv.Z && al16(cv.P) && al16(cv.W) && al16(cv.Z) && cv.T > 0 && cv.C > 0 &&
           (cv.C * 2) % 16 == 0 && cv.cpb == (cv.C + kCvKB - 1) / kCvKB && cv.taps >= 1 && cv.d >= 1 &&
           codec_conv_tile(cv.N) != 0 && (long long)cv.T + (long long)(cv.taps - 1) * cv.d < (1ll << 31) &&
           (cv.T + kCvRows - 1) / kCvRows < (1 << 30) && encode_fn();
}

cudaError_t launch_codec_conv(const CodecConv &cv, cudaStream_t s) {
    if (!codec_conv_supported(cv)) return cudaErrorInvalidValue;
    if (cv.one_cta) switch (codec_conv_tile(cv.N)) {
        case 256: return launch_nt<256, 1>(cv, s);
        case 192: return launch_nt<192, 1>(cv, s);
        case 128: return launch_nt<128, 1>(cv, s);
        case 96: return launch_nt<96, 1>(cv, s);
        default: return launch_nt<64, 1>(cv, s);
        }
    switch (codec_conv_tile(cv.N)) {
    case 256: return launch_nt<256, 2>(cv, s);
    case 192: return launch_nt<192, 2>(cv, s);
    case 128: return launch_nt<128, 2>(cv, s);
    case 96: return launch_nt<96, 2>(cv, s);
    default: return launch_nt<64, 2>(cv, s);
    }
}

}  // namespace s2d
