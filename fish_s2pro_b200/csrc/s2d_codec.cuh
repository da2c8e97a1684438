// s2d_codec.cuh -- kernels of the codec decode shared between its sources.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s2d {

// A stride-1 causal convolution as an implicit GEMM on tcgen05
// (s2d_codec_conv.cu): Z [T][N] f32 = sum over taps k < taps and channels c < C
// of P[t + k d][c] . W[n][k (64 cpb) + c], P the padded f16 input
// [T + (taps - 1) d][C], W [N][taps 64 cpb] f16 with zero columns past C in
// each tap.  N a multiple of 64 or 96.
struct CodecConv {
    const __half *P = nullptr, *W = nullptr;
    int T = 0, C = 0, N = 0, taps = 1, d = 1, cpb = 1;
    float *Z = nullptr;
    bool one_cta = false;      // one CTA per SM with a deeper stage ring instead of two
    int32_t *error = nullptr;  // set to 1 if a bounded wait gave up
};
int codec_conv_tile(int N);
bool codec_conv_supported(const CodecConv &cv);
cudaError_t launch_codec_conv(const CodecConv &cv, cudaStream_t s);

}  // namespace s2d
