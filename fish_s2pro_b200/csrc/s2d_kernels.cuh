// s2d_kernels.cuh -- kernel argument blocks and host launchers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace s2d {

// Generation state kept in device memory so that a captured frame graph can be
// replayed without host round-trips (generate.rs:117-221 keeps the same
// values in host locals).
struct DevState {
    int32_t n_past;      // Slow-AR positions written (SlowArState::n_past)
    int32_t step_index;  // frames finished (generate.rs:164)
    int32_t done;        // loop exit: im_end sampled or max_new reached
    uint32_t main_token; // last sampled main token (generate.rs:154, 202)
    uint64_t rng;        // SeededRng state (sampling.rs:35-52)
    int32_t error;       // nonzero: a kernel met an out-of-range id
    int32_t prompt_cols; // PromptTensor::cols (generate.rs:198-201)
};

enum GemvEpi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU_SLOW = 2, EPI_SWIGLU_FAST = 3 };

struct GemvArgs {
    const uint16_t *W;   // f16 bits, [N][K] row-major (GGUF dims [K, N])
    const uint16_t *W2;  // second matrix (w3) for the SwiGLU epilogue
    const float *x;      // [M][ldx] input activations
    int ldx;
    const float *norm_w; // RMSNorm gain [K]; nullptr = no norm prologue
    float eps;
    float *y;            // [M][ldy]
    int ldy;
    const float *resid;  // [M][ldr] residual for EPI_RESID (may alias y)
    int ldr;
    float *x_out;        // optional: block 0 writes the normalized input [M][K]
    int K, N;
    int row_base, n_contig, extra_row;  // row remap when n_contig >= 0
    const int32_t *done; // early-exit flag (DevState::done) or nullptr
};

struct RopeArgs {
    const float *qkv;    // [M][ld_qkv]: Q | K | V
    int ld_qkv;
    float *q_out;        // [M][H*hd]
    void *kcache, *vcache; // layer base, [Hkv][max_seq][hd] (half or float)
    int max_seq;
    const float *q_norm, *k_norm;  // nullptr: no QK-norm (Fast-AR)
    float eps;
    const float *rope_denom;       // [hd/2]: rope_base^(2i/hd) (host powf)
    const int32_t *pos_dev;        // position of token 0 = pos_const + *pos_dev
    int pos_const;
    int H, Hkv, hd, M;
    const int32_t *done;
    int32_t *error;
};

struct AttnArgs {
    const float *q;      // [M][H*hd]
    const void *kcache, *vcache;  // layer base, [Hkv][max_seq][hd]
    int max_seq;
    float *out;          // [M][H*hd]
    float *part;         // scratch [M][H][S][hd+2]
    int32_t *counters;   // scratch [M][Hkv], zero between launches
    const int32_t *pos_dev;
    int pos_const;
    int H, Hkv, hd, S, M;
    float scale;
    const int32_t *done;
};

struct EmbedArgs {
    const int32_t *tokens;   // [M][K+1] time-major ids, or nullptr: build from state
    const DevState *st;      // used when tokens == nullptr (frame step input)
    const int32_t *frame_codes; // [K] codes of the current frame (with st)
    const uint16_t *emb, *cb_emb;
    int d, K, cb_size, vocab, cb_rows;
    uint32_t sem_begin, sem_end;
    int scale_on;
    float sem_scale;
    float *out;              // [M][d]
    int M;
    const int32_t *done;
    int32_t *error;
};

struct FastInitArgs {
    DevState *st;
    const float *slow_hidden;   // post-norm hidden [d]
    const uint16_t *fast_emb;   // [cb][d]
    float *fast_x;              // [ctx][d]
    int32_t *frame_codes;       // [K]
    int32_t *codes_out;         // [K][max_new]
    int max_new, d, cb_size;
    uint32_t sem_begin, sem_end;
    const uint32_t *code_override; // tests: fixed semantic code (nullptr in the loop)
};

enum SampleMode { SAMPLE_PLAIN = 0, SAMPLE_SLOW_FIRST = 1, SAMPLE_SLOW_STEP = 2, SAMPLE_FAST = 3 };

struct SampleArgs {
    const float *logits;
    int n;                  // candidate count (<= kSampleMax)
    int n_contig;           // ids: r < n_contig -> id_base + r; r == n_contig -> extra_id
    uint32_t id_base, extra_id;
    int64_t vocab_full;     // total vocabulary (entries beyond the candidates are -inf)
    float temperature, top_p;
    int top_k;
    int64_t force_id;       // SAMPLE_PLAIN: always_include_id (<0 none)
    int mode;
    uint32_t im_end;
    uint32_t min_tokens_before_end;
    int max_new;
    DevState *st;
    uint64_t *rng;          // SAMPLE_PLAIN: rng state; otherwise &st->rng
    int cb_index;           // SAMPLE_FAST: codebook being sampled
    int32_t *frame_codes;
    int32_t *codes_out;
    const uint16_t *fast_emb;
    float *fast_x_next;     // SAMPLE_FAST: row to receive fast_emb[code]
    int d;
    uint32_t *out_token;    // optional result copy
};

constexpr int kSampleMax = 8192;
constexpr int kSampleThreads = 1024;
constexpr int kGemvThreads = 256;

// Host launchers (s2d_kernels.cu). All enqueue on `stream`; pdl enables
// programmatic dependent launch on the kernel.
cudaError_t launch_gemv(const GemvArgs &a, int M, int epi, cudaStream_t s, bool pdl);
cudaError_t launch_rope_kv(const RopeArgs &a, bool kv_half, cudaStream_t s, bool pdl);
cudaError_t launch_attention(const AttnArgs &a, bool kv_half, cudaStream_t s, bool pdl);
cudaError_t launch_embed(const EmbedArgs &a, cudaStream_t s, bool pdl);
cudaError_t launch_fast_init(const FastInitArgs &a, cudaStream_t s, bool pdl);
cudaError_t launch_sample(const SampleArgs &a, cudaStream_t s, bool pdl);
cudaError_t launch_f16_to_f32(const uint16_t *src, float *dst, int64_t n, cudaStream_t s);
cudaError_t launch_rms_norm_heads(const float *x, const float *w, float *y, int64_t n, int hd,
                                  float eps, cudaStream_t s);
cudaError_t launch_set_state(DevState *st, int32_t n_past, int32_t prompt_cols, uint64_t rng,
                             cudaStream_t s);
// Sets the dynamic shared-memory limits of the GEMV and sampler kernels
// (call once per device before launching or capturing them).
cudaError_t configure_kernels();

}  // namespace s2d
