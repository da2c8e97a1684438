// s2d_prefill.cuh -- batched Slow-AR prefill kernels (s2d_prefill.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace s2d {

// Epilogues of a GEMM over stacked hi/lo activation rows.
enum PrefillEpi { PF_STORE = 0, PF_RESID = 1, PF_SWIGLU_SLOW = 2, PF_SWIGLU_FAST = 3 };

// Rows t < T of x [T][ldx] (K values each): optional RMSNorm with gain
// norm_w, then the power-of-two scaled f16 split hi -> xs row t, lo -> row
// T + t ([2T][K]); inv[t] = 1 / scale.  xn (optional, with norm_w) receives
// the normalised rows [T][K] as floats.
cudaError_t launch_split_rows(const float *x, int ldx, int T, int K, const float *norm_w, float eps, __half *xs,
                              float *inv, float *xn, cudaStream_t s);

// y[t][n] = epilogue((Y2[t][n] + Y2[T+t][n]) * inv[t]) for t < T, n < N, Y2
// being [2T][N]; PF_RESID adds resid[t][n] (may alias y), the SwiGLU forms
// take the up projection from Y2b the same way.
cudaError_t launch_combine(int epi, const float *Y2, const float *Y2b, const float *inv, int T, int N, float *y,
                           int ldy, const float *resid, int ldr, cudaStream_t s);

// Causal GQA attention of T query tokens at positions pos0 + t over a
// layer's cache [Hkv][max_seq][hd] (every position up to pos0 + T - 1
// written): q [T][H*hd] (already normalised and rotated) -> out [T][H*hd].
cudaError_t launch_prefill_attention(const float *q, const void *kcache, const void *vcache, bool kv_half, int max_seq,
                                     float *out, int T, int pos0, int H, int Hkv, int hd, float scale,
                                     cudaStream_t s);

}  // namespace s2d
