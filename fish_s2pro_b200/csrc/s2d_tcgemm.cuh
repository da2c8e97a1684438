// s2d_tcgemm.cuh -- tensor-core GEMM of the rows path (s2d_tcgemm.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s2d {

// y[t][n] = epilogue(inv[t] * sum_k W[n][k] * (hi[t][k] + lo[t][k])) for t < T,
// n < N, with hi / lo the stacked f16 rows of launch_split_rows (xs [2T][K])
// and W [N][K] f16 rows.  epi is a PrefillEpi: store, residual add (resid may
// alias y), or SwiGLU with the up projection W2 [N][K] (slow or fast form).
struct TcGemm {
    const uint16_t *W = nullptr, *W2 = nullptr;
    int N = 0, K = 0;
    const __half *xs = nullptr;
    int T = 0;
    const float *inv = nullptr;
    int epi = 0;
    float *y = nullptr;
    int ldy = 0;
    const float *resid = nullptr;
    int ldr = 0;
    int num_sms = 148;
    int32_t *error = nullptr;  // set to kErrTcWait if a wait gave up
};

constexpr int32_t kErrTcWait = 19;

// Whether the tensor-core path takes this GEMM (K a multiple of 64, operands
// 16-byte aligned, T and N in range); otherwise the caller uses cuBLAS.
bool tc_gemm_supported(const TcGemm &g);
cudaError_t launch_tc_gemm(const TcGemm &g, cudaStream_t s);

}  // namespace s2d
