/*
 * s2d.h -- C ABI of libs2d.so, the sm_100a Dual-AR token loop for fish-s2pro.
 *
 * This is the drop-in boundary for the reference's `rust-pure` hot path
 * (crate fish_s2_infer; paths below are relative to the reference repository
 * root).  It follows the conventions of the reference's existing native ABI
 * (crates/fish_s2_infer/ffi/s2_engine_ffi.h:10-37): opaque handle, plain C
 * types, errors returned as a status with the message written into a caller
 * buffer (s2_engine_ffi.cpp:16-22) or kept on the handle.  Caller-provided
 * output buffers are used throughout, so nothing crosses allocators.
 *
 * Status codes: S2D_OK (0) on success, a negative S2D_E* on failure.
 * Threading: a handle is not re-entrant; use one host thread per handle
 * (the reference serialises the same way: engine.rs:159, server.rs:20).
 * Every call is synchronous: it returns after its device work has finished.
 */
#ifndef S2D_H
#define S2D_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define S2D_OK 0
#define S2D_EINVAL (-1)   /* bad argument, shape or token id          */
#define S2D_EIO (-2)      /* GGUF file missing, truncated or malformed */
#define S2D_ECUDA (-3)    /* a CUDA runtime call failed               */
#define S2D_ENOMEM (-4)   /* device or host allocation failed         */
#define S2D_ESTATE (-5)   /* KV cache overflow or call out of order   */
#define S2D_EDEVICE (-6)  /* a kernel reported an error flag           */
#define S2D_EFULL (-7)    /* serving: no free slot or KV pages; collect first */

typedef struct S2dHandle S2dHandle;

/* Open-time configuration (replaces the arguments of SlowArState::open,
 * slow_ar.rs:387, and EngineConfig's device fields, engine.rs:83-127). */
typedef struct S2dConfig {
    int32_t device;       /* CUDA device ordinal                                   */
    int32_t max_seq;      /* Slow-AR KV capacity in positions (SlowArState::open)   */
    int32_t max_batch;    /* sequences of s2d_generate_codes_batch (<= 0: 1); each
                             holds its own Slow-AR KV cache of max_seq positions   */
    int32_t flags;        /* reserved, 0                                             */
    int32_t kv_pages;     /* pages of 64 positions in the batched KV pool (every
                             layer's K and V of one sequence's 64 positions);
                             <= 0: max_batch * ceil(max_seq / 64), room for every
                             sequence at max_seq.  Batched calls give each
                             sequence the pages of its prompt + max_new_tokens. */
} S2dConfig;

/* DualArGraphSpec (registry.rs:30-42, 216-231), shape-parametric. */
typedef struct S2dGraphSpec {
    int32_t slow_layers, hidden, ffn, heads, kv_heads, head_dim, context_length;
    int32_t fast_layers, fast_ffn, fast_heads, fast_kv_heads, fast_head_dim, fast_context_length;
    float rope_base, rms_eps, fast_rope_base, fast_rms_eps;
    int32_t codebook_size, num_codebooks, semantic_begin_id, semantic_end_id;
    int32_t vocab_size, codebook_rows;
    int32_t linear_type; /* ggml type of the linear weights: 1 F16, 8 Q8_0, 12 Q4_K */
} S2dGraphSpec;

/* SamplerParams (sampling.rs:12-27). */
typedef struct S2dSamplerParams {
    float temperature;
    float top_p;
    int32_t top_k;
} S2dSamplerParams;

/* GenerateParams (generate.rs:13-32) plus the tokenizer's <|im_end|> id
 * (S2TokenizerConfig.im_end_id, generate.rs:133-134). */
typedef struct S2dGenParams {
    uint32_t max_new_tokens;
    float temperature;
    float top_p;
    int32_t top_k;
    uint32_t min_tokens_before_end;
    uint32_t im_end_id;
} S2dGenParams;

/* Timing of one generate call, measured with CUDA events on the handle's
 * stream (the device-side counterpart of SlowArDecodeProfile,
 * slow_ar.rs:248-319, which the reference fills with host timers). */
typedef struct S2dProfile {
    double prefill_ms;      /* prompt prefill + first semantic sample            */
    double decode_ms;       /* all frames: Fast-AR codebooks + Slow-AR step      */
    uint32_t frames;        /* frames produced                                   */
    uint32_t kernels_per_frame; /* kernel launches in one captured frame       */
    uint32_t prefill_kernels;   /* kernel launches of the prefill + first sample */
    uint32_t frame_launches;    /* frame graphs launched (>= frames)            */
} S2dProfile;

/* Kernels that s2d_profile_kernel can time in isolation. */
#define S2D_KERNEL_WQKV 0   /* attention_norm + WQKV GEMV            */
#define S2D_KERNEL_WO 1     /* wo GEMV + residual                     */
#define S2D_KERNEL_W13 2    /* ffn_norm + w1/w3 GEMV + SwiGLU          */
#define S2D_KERNEL_W2 3     /* w2 GEMV + residual                     */
#define S2D_KERNEL_LM_HEAD 4 /* final norm + masked LM head GEMV      */

/* Logits requested from s2d_prefill / s2d_step. */
#define S2D_LOGITS_NONE 0
#define S2D_LOGITS_ALLOWED 1 /* semantic rows + im_end only; other entries -inf */
#define S2D_LOGITS_FULL 2    /* all vocab_size rows (debug parity)            */

/* One rank's shard of the Slow-AR under tensor parallelism (s2d_tp_plan). */
typedef struct S2dTpShard {
    int32_t heads, kv_heads;  /* query / KV heads of this rank                     */
    int32_t head0, kv_head0;  /* its first query / KV head                          */
    int32_t ffn, ffn0;        /* its FFN columns [ffn0, ffn0 + ffn)                 */
} S2dTpShard;

/* ---- lifecycle ---------------------------------------------------------- */

/* Replaces SlowArState::open + FastArWeights::from_gguf (slow_ar.rs:387-412,
 * fast_ar.rs:202-223) and TransformerTensorRegistry::from_gguf
 * (registry.rs:515-552): parses the transformer GGUF, validates names and
 * shapes, uploads every tensor to HBM once. */
int32_t s2d_open(const char *transformer_gguf, const S2dConfig *cfg, S2dHandle **out,
                 char *err, size_t err_cap);
/* ---- Slow-AR tensor parallelism ------------------------------------------
 * tp_size ranks (one process or thread per GPU) open the same GGUF with
 * s2d_open_tp; rank r keeps query heads [r*H/n, (r+1)*H/n) of wqkv / wo and
 * the KV cache with their KV heads, and an FFN slice of w1 / w3 / w2 (whole
 * weight blocks; a Q4_K FFN may split unevenly).  The two Slow-AR residual
 * additions of each layer become an NCCL allreduce over the ranks; the LM
 * head, the samplers and the Fast-AR run replicated, so every rank returns
 * the same results.  Every rank must make the same calls in the same order
 * (prefill, step, generate_codes, the batched variant).  The persistent
 * decode engine is single-GPU: a tensor-parallel handle decodes with the
 * per-op kernels captured into the frame graph together with the NCCL calls. */

/* The shard of rank tp_rank of tp_size for this graph (spec.linear_type sets
 * the block width).  S2D_EINVAL if the model does not split that way. */
int32_t s2d_tp_plan(const S2dGraphSpec *spec, int32_t tp_size, int32_t tp_rank, S2dTpShard *out);
/* A fresh NCCL unique id (cap >= 128 bytes) for s2d_open_tp; one rank makes
 * it and hands it to the others by any host channel. */
int32_t s2d_nccl_unique_id(uint8_t *out, size_t cap);
/* s2d_open for rank tp_rank of tp_size (collective: blocks until every rank
 * has joined the communicator).  tp_size 1 is s2d_open. */
int32_t s2d_open_tp(const char *transformer_gguf, const S2dConfig *cfg, int32_t tp_size, int32_t tp_rank,
                    const uint8_t *nccl_id, S2dHandle **out, char *err, size_t err_cap);

/* Replaces s2_engine_destroy (s2_engine_ffi.h:26). NULL is ignored. */
void s2d_close(S2dHandle *h);
/* Message of the last failed call on this handle ("" if none). */
const char *s2d_last_error(const S2dHandle *h);
/* SlowArState::graph_spec (slow_ar.rs:418-420). */
int32_t s2d_graph_spec(const S2dHandle *h, S2dGraphSpec *out);

/* ---- Slow-AR state (SlowArState, slow_ar.rs:372-528) --------------------- */

/* SlowArState::reset (slow_ar.rs:434-438). seq must be 0. */
int32_t s2d_reset(S2dHandle *h, int32_t seq);
/* SlowArState::n_past (slow_ar.rs:422-424). */
int32_t s2d_n_past(const S2dHandle *h, int32_t seq, int32_t *out);
/* SlowArState::prefill / eval (slow_ar.rs:440-442, 456-527): n_flat ids in
 * time-major order (prompt.rs:77-103), a multiple of num_codebooks+1.
 * out_hidden: hidden floats, the post-final-norm hidden of the last token
 * (slow_ar.rs:515-526), or NULL.  out_logits: vocab_size floats or NULL,
 * filled per logits_mode. */
int32_t s2d_prefill(S2dHandle *h, int32_t seq, const int32_t *flat_tokens, int64_t n_flat,
                    float *out_hidden, float *out_logits, int32_t logits_mode,
                    uint32_t im_end_id);
/* SlowArState::step (slow_ar.rs:444-454): exactly num_codebooks+1 ids.
 * With S2D_LOGITS_ALLOWED or S2D_LOGITS_NONE the step runs on the persistent
 * decode engine (the step program every generated frame runs); with
 * S2D_LOGITS_FULL on the per-op kernels, whose LM head covers the vocabulary. */
int32_t s2d_step(S2dHandle *h, int32_t seq, const int32_t *step_input, int64_t n,
                 float *out_hidden, float *out_logits, int32_t logits_mode, uint32_t im_end_id);

/* ---- Fast-AR (fast_ar.rs) ------------------------------------------------ */

/* forward_codebook_prefix (fast_ar.rs:360-437): slow_hidden (hidden floats),
 * prefix codes (n_prefix < num_codebooks) -> codebook_size logits. */
int32_t s2d_fast_prefix_logits(S2dHandle *h, const float *slow_hidden, const uint32_t *prefix,
                               int64_t n_prefix, float *out_logits);
/* generate_codebooks_for_semantic (fast_ar.rs:440-470): out_codes receives
 * num_codebooks codes (out[0] = semantic_code).  *rng_state is the SeededRng
 * state (sampling.rs:35-52), advanced in place. */
int32_t s2d_generate_codebooks(S2dHandle *h, const float *slow_hidden, uint32_t semantic_code,
                               const S2dSamplerParams *sampler, uint64_t *rng_state,
                               uint32_t *out_codes);

/* ---- the generation loop (generate.rs:117-221) --------------------------- */

/* generate_codes: prompt is row-major (num_codebooks+1) x cols
 * (PromptTensor, prompt.rs:59-67).  out_codes needs num_codebooks *
 * max_new_tokens int32 and receives codebook-major codes compacted to
 * *out_n_frames frames (generate.rs:346-390).  *rng_state is advanced like
 * the reference's SeededRng.  profile may be NULL. */
int32_t s2d_generate_codes(S2dHandle *h, const uint32_t *prompt, int32_t rows, int32_t cols,
                           const S2dGenParams *params, uint64_t *rng_state, int32_t *out_codes,
                           uint32_t *out_n_frames, S2dProfile *profile);

/* Random draws of the batched sampler. */
#define S2D_RNG_SEEDED 0 /* the reference's SeededRng LCG; rng_states[i] is its state        */
#define S2D_RNG_PHILOX 1 /* Philox4x32-10, key philox_key, counter (rng_states[i], i):      */
                         /* rng_states[i] counts sequence i's draws                         */

/* generate_codes over n_seq independent prompts at once (the batched
 * variant of generate.rs:117-221; the reference has none).  prompts[i] is
 * row-major rows x cols[i] (rows = num_codebooks+1); every sequence shares
 * params.  Sequence i's codes go to out_codes + i*num_codebooks*max_new_tokens,
 * codebook-major and compacted to out_n_frames[i] frames; rng_states[i] is
 * advanced in place.  With S2D_RNG_SEEDED sequence i produces the codes of
 * s2d_generate_codes on prompt i with state rng_states[i] (up to rounding
 * of the batched GEMMs).  Needs n_seq <= max_batch (S2dConfig) and
 * cols[i] + max_new_tokens <= max_seq.  Q8_0 / Q4_K linears run as GEMMs over
 * an f16 expansion (exact dequantisation rounded to f16) that the first
 * batched call builds and the handle keeps.  Resets the single-sequence
 * state (n_past = 0): sequence 0's cache is reused.  Ends a serving session
 * (s2d_serve_begin) on the handle.  profile (may be NULL) counts frames over
 * all sequences. */
int32_t s2d_generate_codes_batch(S2dHandle *h, int32_t n_seq, const uint32_t *const *prompts,
                                 const int32_t *cols, int32_t rows, const S2dGenParams *params,
                                 int32_t rng_kind, uint64_t philox_key, uint64_t *rng_states,
                                 int32_t *out_codes, uint32_t *out_n_frames, S2dProfile *profile);

/* ---- continuous batching (serving) -----------------------------------------
 * The server-side form of generate_codes.  The reference serves one /v1/tts
 * request at a time under a lock (tts_handler, server.rs:89-120, over
 * InferenceEngine::synthesize_wav, engine.rs:255-287, whose pipeline calls
 * generate_codes, pipeline.rs:174-182).  Here a session holds max_batch
 * slots (S2dConfig) that advance together, one captured batched frame per
 * frame; requests join and leave between frames:
 *   s2d_serve_begin   opens the session with one set of generation params
 *                     and RNG kind, every slot free;
 *   s2d_serve_admit   prefills one request (prompt rows x cols, row-major,
 *                     rows = num_codebooks + 1) into a free slot and samples
 *                     its first semantic token.  The request takes the KV
 *                     pages of positions [0, cols + max_new_tokens) from
 *                     the handle's pool (ceil(.../64) pages of 64
 *                     positions); S2D_EFULL when too few are free;
 *   s2d_serve_step    runs n_frames frames; slot_status[i] (may be NULL)
 *                     receives S2D_SLOT_*, slot_frames[i] the frames slot i
 *                     has produced;
 *   s2d_serve_collect copies a finished slot's codes (codebook-major,
 *                     compacted to *out_n_frames frames, like
 *                     s2d_generate_codes; out_codes holds num_codebooks *
 *                     max_new_tokens) and its final RNG state, and frees the
 *                     slot and its pages.
 * With S2D_RNG_SEEDED a request's codes do not depend on which slot it runs
 * in, on its neighbours or on when it was admitted (each row of the batched
 * frame is computed alone); with S2D_RNG_PHILOX its draws are keyed by the
 * slot index.  Every call is synchronous; no counterpart in the reference
 * beyond the loop it batches. */
#define S2D_SLOT_FREE 0
#define S2D_SLOT_RUNNING 1
#define S2D_SLOT_FINISHED 2
int32_t s2d_serve_begin(S2dHandle *h, const S2dGenParams *params, int32_t rng_kind, uint64_t philox_key);
int32_t s2d_serve_admit(S2dHandle *h, int32_t slot, const uint32_t *prompt, int32_t rows, int32_t cols,
                        uint64_t rng_state);
int32_t s2d_serve_step(S2dHandle *h, int32_t n_frames, int32_t *slot_status, uint32_t *slot_frames);
int32_t s2d_serve_collect(S2dHandle *h, int32_t slot, int32_t *out_codes, uint32_t *out_n_frames,
                          uint64_t *rng_state);
/* KV pages of the pool that no serving slot holds (0 outside a session). */
int32_t s2d_serve_free_pages(const S2dHandle *h, int32_t *out);

/* Device time of one batched frame by kernel category: the frame of the
 * last s2d_generate_codes_batch call (its first n_seq sequences), replayed
 * once outside its graph with a CUDA event after every launch; each gap is
 * charged to the launch it ends.  Every sequence runs the frame (codes are
 * not stored); afterwards every sequence is marked finished.  out_ms[i] for
 * i < n_out: S2D_PROF_* below, out_ms[S2D_PROF_TOTAL] the whole frame. */
#define S2D_PROF_SPLIT 0    /* RMSNorm + hi/lo row split before each GEMM  */
#define S2D_PROF_GEMM 1     /* tensor-core GEMMs over the stacked rows     */
#define S2D_PROF_COMBINE 2  /* hi + lo, residual / SwiGLU epilogues        */
#define S2D_PROF_ROPE 3     /* QK-norm + RoPE + KV writes                  */
#define S2D_PROF_ATTN 4     /* GQA attention of every row                  */
#define S2D_PROF_SAMPLE 5   /* samplers                                    */
#define S2D_PROF_OTHER 6    /* embedding feedback, Fast-AR frame start     */
#define S2D_PROF_TOTAL 7
int32_t s2d_profile_batch(S2dHandle *h, int32_t n_seq, double *out_ms, int32_t n_out);

/* The batched sampler's Philox4x32-10 block function, run on the current
 * device: out = philox(counter[4], key[2]).  For checking the generator
 * against the published known-answer vectors. */
int32_t s2d_philox4x32_10(const uint32_t *counter, const uint32_t *key, uint32_t *out);

/* ---- sampling (sampling.rs:121-241) ------------------------------------- */

/* sample_token on the device sampler: logits (n floats, ids 0..n-1),
 * always_include_id < 0 for None. */
int32_t s2d_sample_token(S2dHandle *h, const float *logits, int64_t n,
                         const S2dSamplerParams *sampler, int64_t always_include_id,
                         uint64_t *rng_state, uint32_t *out_token);

/* ---- weights ------------------------------------------------------------- */

/* Dequantise one resident tensor to f32 on the device and copy it out
 * (n = its element count).  The reference only decodes F16
 * (F16TensorView::from_gguf, tensor.rs:22-45); Q8_0 / Q4_K follow ggml's
 * block formats. */
int32_t s2d_dequant_tensor(S2dHandle *h, const char *name, float *out, int64_t n);

/* ---- measurement ----------------------------------------------------------
 * No counterpart in the reference (which only has host timers,
 * SlowArDecodeProfile, slow_ar.rs:248-319).  Times `iters` back-to-back
 * launches of one decode kernel on the resident Slow-AR weights (cycling
 * through the layers so that no launch finds its weights in L2) with CUDA
 * events on the handle's stream.  *avg_ms: mean duration of one launch;
 * *bytes: algorithmic HBM bytes of one launch (weights read once + the
 * activation vector in and out). */
int32_t s2d_profile_kernel(S2dHandle *h, int32_t kernel, int32_t iters, double *avg_ms,
                           double *bytes);

/* Runs one program of the persistent decode engine once, outside any graph,
 * on the handle's current state (call after s2d_generate_codes): program 0 is
 * the Slow-AR step (all layers + LM head), program k >= 1 the Fast-AR pass
 * that produces codebook k, program -1 the whole Fast-AR of a frame (every
 * pass, head and sampler in one launch; built by the first
 * s2d_generate_codes, absent with S2D_FAST_FRAME=0).  *ms: its CUDA-event
 * duration.  If trace is not
 * NULL it receives n_ops*(8+G) timestamps (ns, %globaltimer), G = the SM
 * count: first for CTA 0 then the last CTA, per op: op started, input staged,
 * op finished, producer done issuing the op's weights; then per op, every
 * CTA's finish time.  *n_ops receives the program length.  No counterpart in
 * the reference. */
int32_t s2d_profile_engine(S2dHandle *h, int32_t program, uint64_t *trace, int64_t trace_cap,
                           int32_t *n_ops, double *ms);

/* ---- op-level seam (MatmulBackend, backend.rs:5-39) ----------------------
 * Host buffers in and out; each call uploads, runs one kernel and copies the
 * result back.  Kept for op-level parity tests; the model path never uses
 * them. */

/* MatmulBackend::linear (backend.rs:55-73) with f16 weights [out_dim][in_dim]
 * (GGUF little-endian bits), i.e. matvec_f16_streaming (tensor.rs:220-264). */
int32_t s2d_op_linear_f16(S2dHandle *h, const float *input, const uint16_t *weight_f16,
                          int64_t in_dim, int64_t out_dim, float *out);
/* The causal attention of forward_prefill_sequence (slow_ar.rs:579-593):
 * T query rows of one sequence, row m at position pos0 + m attending over
 * positions 0..pos0 + m of kcache / vcache [Hkv][max_seq][head_dim] (f16
 * bits); q and out [T][H][head_dim] f32.  impl 0: the tensor-core kernel;
 * 1: the CUDA-core kernels (tiled for T >= 16); 2: the tcgen05 kernel
 * (TMEM accumulators, head_dim 128 only).  pos0 + T <= max_seq,
 * T <= 4096, head_dim 64 or 128, H / Hkv <= 8, host buffers. */
int32_t s2d_op_prefill_attention(S2dHandle *h, const float *q, const uint16_t *kcache, const uint16_t *vcache,
                                 int64_t T, int64_t H, int64_t Hkv, int64_t head_dim, int64_t max_seq,
                                 int64_t pos0, int32_t impl, float *out);
/* gqa_decode_attention + softmax_in_place (attention.rs:208-309) for B
 * sequences at once, the batched Slow-AR step's attention: q [B][H][head_dim]
 * f32; kcache / vcache [B][Hkv][max_seq][head_dim] f16 bits; sequence b's
 * row sits at position n_past[b] and attends over positions 0..n_past[b]
 * (done[b] != 0, when done is given, skips the sequence and leaves its out
 * rows zero).  splits: position splits per (sequence, kv head), 0 for the
 * runtime's choice.  impl 0: the tensor-core kernel; 1: the CUDA-core rows
 * kernel.  head_dim 64 or 128, H / Hkv <= 8, host buffers; out
 * [B][H][head_dim]. */
int32_t s2d_op_batch_attention(S2dHandle *h, const float *q, const uint16_t *kcache, const uint16_t *vcache,
                               int64_t B, int64_t H, int64_t Hkv, int64_t head_dim, int64_t max_seq,
                               const int32_t *n_past, const int32_t *done, int32_t splits, int32_t impl,
                               float *out);
/* MatmulBackend::rms_norm / rms_norm_heads (backend.rs:84-121);
 * head_dim == n gives the plain rms_norm. */
/* MatmulBackend::linear (backend.rs:55-73) over T rows at once, the rows
 * path's GEMM: y[t][n] = epi(sum_k x[t][k] * w[n][k]) for x [T][K] f32, w
 * [N][K] f16 bits.  epi 0 stores, 1 adds resid [T][N], 2 / 3 the slow / fast
 * SwiGLU with the up projection w2 [N][K].  impl 0: the tcgen05 tensor-core
 * GEMM (S2D_EINVAL if it does not take the shape: K a multiple of 64); 1: cuBLAS
 * and the combine pass.  T <= 512, K <= 16384, host buffers. */
int32_t s2d_op_rows_linear_f16(S2dHandle *h, const float *x, int64_t T, int64_t K, const uint16_t *w,
                               const uint16_t *w2, int64_t N, const float *resid, int32_t epi, int32_t impl,
                               float *y);
int32_t s2d_op_rms_norm(S2dHandle *h, const float *input, const float *weight, int64_t n,
                        int64_t head_dim, float eps, float *out);
/* apply_rope_normal (attention.rs:172-206): rotate every head of values (n =
 * heads * head_dim floats, head-major) by position, adjacent pairs (2i, 2i+1)
 * at theta = position / rope_base^(2i/head_dim).  Runs the RoPE of the per-op
 * and rows paths (rope_kv_kernel).  head_dim 64, 128 or 256; host buffers. */
int32_t s2d_op_rope_normal(S2dHandle *h, const float *values, int64_t n, int64_t head_dim,
                           int64_t position, float rope_base, float *out);
/* MatmulBackend::gqa_decode_attention (attention.rs:208-247): keys/values
 * token-major [token_count][head_count_kv][head_dim]. */
int32_t s2d_op_gqa_decode_attention(S2dHandle *h, const float *query, const float *keys,
                                    const float *values, int32_t head_count,
                                    int32_t head_count_kv, int32_t head_dim,
                                    int32_t token_count, float attn_scale, float *out);

/* Allocation-free variant of s2d_op_gqa_decode_attention.  It has no
 * counterpart in the reference.  For callers that cannot call cudaMalloc: a
 * real-time audio thread must not block in the CUDA allocator, and a host that
 * gives this library a fixed memory budget owns every device allocation.
 * query (head_count*head_dim), keys and values (head-major
 * [head_count_kv][token_count][head_dim]) and out (head_count*head_dim) are
 * the caller's DEVICE buffers, f32; keys and values 16-byte aligned (8 bytes
 * suffice at head_dim 64), query and out 4-byte aligned, else S2D_EINVAL
 * before any device work.  The split-K scratch is a fixed device
 * array inside the library: 512 KiB of partials plus 64 counters, held by
 * every GPU that loads the library until the process exits.  Calls needing
 * more (head_count * splits * (head_dim+2) > 131072 floats, with
 * splits = clamp(token_count/8, 1, 16), or head_count_kv > 64) are rejected
 * with S2D_EINVAL.  The first call on a device looks the array's device
 * address up (cudaGetSymbolAddress) and should come before any stream capture
 * on that device; the cached address lives as long as the device's primary
 * context, so do not call this entry point after a cudaDeviceReset of that
 * device in the same process.  All calls share the array, so calls that
 * overlap on the GPU race: serialise them.  The call is synchronous: it is
 * enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream) and
 * returns only after that stream has finished it.  Errors are written into
 * err. */
int32_t s2d_op_gqa_decode_attention_noalloc(const float *query, const float *keys,
                                            const float *values, int32_t head_count,
                                            int32_t head_count_kv, int32_t head_dim,
                                            int32_t token_count, float attn_scale, float *out,
                                            void *stream, char *err, size_t err_cap);

#ifdef __cplusplus
}
#endif
#endif /* S2D_H */
