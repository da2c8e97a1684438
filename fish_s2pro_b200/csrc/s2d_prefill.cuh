// s2d_prefill.cuh -- batched Slow-AR prefill kernels (s2d_prefill.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "s2d_kernels.cuh"

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

// launch_combine then launch_split_rows on its output, in one pass per row:
// y[t] (optional, ldy) = epilogue of the stacked GEMM rows; then RMSNorm
// (norm_w optional) and the hi/lo split of that row into xs, inv[t] replaced
// by the new row scale.  N <= 16384.
cudaError_t launch_combine_split(int epi, const float *Y2, const float *Y2b, float *inv, int T, int N, float *y,
                                 int ldy, const float *resid, int ldr, const float *norm_w, float eps, __half *xs,
                                 cudaStream_t s);

// GQA attention of T query rows over their sequences' caches.  Row m is
// sequence m / rows_per_seq at position pos_const + (m % rows_per_seq), plus
// st[seq].n_past when st_pos is set (rows of a finished sequence,
// st[seq].done, are skipped).  Sequence s's layer caches [Hkv][max_seq][hd] (f16 or f32)
// start kv_seq_stride elements after sequence s-1's; a row attends positions
// 0 .. its own, which must all be written.  q [T][H*hd] is normalised and
// rotated; out [T][H*hd].
struct RowsAttnArgs {
    const float *q;
    const void *kcache, *vcache;
    size_t kv_seq_stride;
    int max_seq;
    KvPages kv_pages;    // paged caches (kv_pages.pages set; see kv_row): kv_seq_stride unused
    float *out;
    int T, rows_per_seq;
    const DevState *st;
    int st_pos;
    int pos_const;
    int H, Hkv, hd;
    float scale;
    int S;               // splits of each row's positions (1: no merge)
    float *part;         // S > 1: [T][H][S][hd + 2]
    int32_t *counters;   // S > 1: [T][Hkv], zero between launches (left zero)
    int decode_stages;   // K/V ring stages of the decode kernels (CUDA cores: 2 or 4; MMA: 2 or 3)
    int decode_mma;      // batched step rows (one per sequence, f16 cache): the tensor-core kernel
    int decode_warps;    // its warps per block, 2 or 4
    int decode_chunk;    // its positions per staged chunk, 16 or 32
    const int32_t *row_order;  // its block order: row of each rank (longest context first), or nullptr
    int prefill_mma;     // prompt chunks (one sequence's consecutive rows, f16 cache): the tensor-core kernel
    int prefill_tc;      // prompt chunks at head dim 128: the tcgen05 kernel (s2d_tc_attn.cu)
    size_t k_rows, v_rows;  // rows of hd f16 from kcache / vcache to the end of their buffer (0: unknown)
    int32_t *error;      // set when a bounded wait of the tcgen05 kernel gives up
};
cudaError_t launch_rows_attention(const RowsAttnArgs &a, bool kv_half, cudaStream_t s);
// A prompt chunk's causal attention on tcgen05 (s2d_tc_attn.cu): one
// sequence's consecutive rows, S == 1, f16 caches (contiguous or paged, with
// k_rows / v_rows set), head dim 128, 128 % (H / Hkv) == 0.
bool prefill_tc_supported(const RowsAttnArgs &a, bool kv_half);
cudaError_t launch_prefill_tc_attention(const RowsAttnArgs &a, cudaStream_t s);
// The batched step's attention on the tensor cores (s2d_decode_attn.cu):
// rows of one position per sequence (st and st_pos set), f16 caches, head
// dim 64 or 128, up to 8 query heads per kv head.
bool decode_mma_supported(const RowsAttnArgs &a, bool kv_half);
cudaError_t launch_decode_mma_attention(const RowsAttnArgs &a, cudaStream_t s);
// A prompt chunk's causal attention on the tensor cores (s2d_decode_attn.cu):
// one sequence's consecutive rows (rows_per_seq >= T, no st), S == 1, f16
// caches, head dim 64 or 128, a GQA group of 1, 2, 4 or 8 heads.
bool prefill_mma_supported(const RowsAttnArgs &a, bool kv_half);
cudaError_t launch_prefill_mma_attention(const RowsAttnArgs &a, cudaStream_t s);

}  // namespace s2d
