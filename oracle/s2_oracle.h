/*
 * s2_oracle.h -- CPU restatement of fish-s2pro's `rust-pure` Dual-AR math.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a path and the CPU baseline that bench.py reports beside it.  No
 * product code links or calls it: only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs load it.
 *
 * Every function restates one function of the reference (Rust crate
 * fish_s2_infer, paths relative to the reference repository root) with the
 * same f32 operation order, so that its outputs equal the reference's on the
 * same inputs.  The reference itself is Rust and cannot be compiled in this
 * image (no rustc); the restatement is pinned instead against the
 * known-answer values of the reference's own unit tests
 * (tests/test_oracle_kat.py).
 *
 * Conventions: functions return 0 on success and a negative value on error;
 * the message of the last error on the calling thread is returned by
 * s2o_last_error().
 */
#ifndef S2_ORACLE_H
#define S2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char *s2o_last_error(void);

/* ---- scalar conversions: crates/fish_s2_infer/src/tensor.rs:266-329 ---- */
float s2o_f16_to_f32(uint16_t bits);
uint16_t s2o_f32_to_f16(float value);
float s2o_round_f32_to_f16(float value);

/* ---- op-level math (the MatmulBackend seam, backend.rs:5-121) ---- */
int s2o_rms_norm(const float *input, const float *weight, int64_t n, float eps, float *out);
int s2o_rms_norm_heads(const float *input, const float *weight, int64_t n, int64_t head_dim,
                       float eps, float *out);
int s2o_linear(const float *input, const float *weight, int64_t in_dim, int64_t out_dim,
               float *out);
int s2o_matvec_f16(const float *input, const uint16_t *weight, int64_t in_dim, int64_t out_dim,
                   float *out);
int s2o_rope_normal(float *values, int64_t n, int64_t head_dim, int64_t position,
                    float rope_base);
int s2o_gqa_decode_attention(const float *query, const float *keys, const float *values,
                             int64_t head_count, int64_t head_count_kv, int64_t head_dim,
                             int64_t token_count, float attn_scale, float *out);
int s2o_swiglu_slow(const float *gate, const float *up, int64_t n, float *out);
int s2o_swiglu_fast(const float *gate, const float *up, int64_t n, float *out);

/* ---- sampling: crates/fish_s2_infer/src/sampling.rs ---- */
double s2o_rng_next_unit(uint64_t *state);
int s2o_build_semantic_bias(int64_t vocab, uint32_t sem_begin, uint32_t sem_end,
                            int64_t im_end_id /* <0: none */, float *bias);
int s2o_apply_semantic_bias(float *logits, const float *bias, int64_t n, int block_im_end,
                            int64_t im_end_id);
int s2o_semantic_mask_logits(float *logits, int64_t n, uint32_t sem_begin, uint32_t sem_end,
                             int64_t im_end_id, int block_im_end);
int s2o_sample_token(const float *logits, int64_t vocab, float temperature, float top_p,
                     int32_t top_k, int64_t always_include_id /* <0: none */,
                     uint64_t *rng_state, uint32_t *out_token);

/* ---- toy layer skeleton over caller-provided f32 weights (slow_ar.rs:188-918) ---- */
typedef struct S2oLayerShape {
    int64_t hidden_size;
    int64_t feed_forward_size;
    int64_t head_count;
    int64_t head_count_kv;
    int64_t head_dim;
    float rope_base;
    float rms_norm_eps;
} S2oLayerShape;

typedef struct S2oLayerWeightsF32 {
    const float *attention_norm, *q_norm, *k_norm, *wqkv, *wo, *ffn_norm, *w1, *w2, *w3;
    /* element counts, checked like SlowArLayerSkeleton::validate (slow_ar.rs:856-918) */
    int64_t n_attention_norm, n_q_norm, n_k_norm, n_wqkv, n_wo, n_ffn_norm, n_w1, n_w2, n_w3;
} S2oLayerWeightsF32;

/* Outputs of forward_decode_token + forward_feed_forward, per token (slow_ar.rs:202-228). */
typedef struct S2oLayerTrace {
    float *normalized, *query, *key, *value, *attention, *projected, *attn_hidden;
    float *ffn_normalized, *gate, *up, *activated, *ffn_projected, *hidden;
} S2oLayerTrace;

/* A contiguous f32 KV cache with the reference layout [hd, Hkv, max_seq, layers]
 * (attention.rs:14-170). */
typedef struct S2oKvCache S2oKvCache;
S2oKvCache *s2o_kv_new(int64_t head_dim, int64_t head_count_kv, int64_t max_seq, int64_t layers);
void s2o_kv_free(S2oKvCache *kv);
int s2o_kv_write_token(S2oKvCache *kv, int64_t layer, int64_t token, const float *key,
                       const float *value);
int s2o_kv_read_token(const S2oKvCache *kv, int64_t layer, int64_t token, float *key,
                      float *value);
int s2o_kv_decode_attention(const S2oKvCache *kv, int64_t layer, int64_t token_count,
                            const float *query, int64_t head_count, float attn_scale,
                            float *out);

/* SlowArLayerSkeleton::forward_block_prefill_sequence over n tokens
 * (slow_ar.rs:558-617, 659-854).  `decode_loop` != 0 runs
 * forward_decode_sequence + forward_feed_forward per token instead
 * (slow_ar.rs:539-556).  trace may be NULL; otherwise each array holds
 * n_tokens rows. */
int s2o_layer_forward(const S2oLayerShape *shape, const S2oLayerWeightsF32 *w,
                      const float *hidden_tokens, int64_t n_tokens, S2oKvCache *kv,
                      int64_t layer, int64_t start_position, int decode_loop,
                      S2oLayerTrace *trace, float *hidden_out);

/* ---- model over a GGUF file (gguf.rs, registry.rs, slow_ar.rs, fast_ar.rs) ---- */
typedef struct S2oGraphSpec {
    int32_t slow_context_length, slow_embedding_length, slow_feed_forward_length,
        slow_block_count, slow_head_count, slow_head_count_kv, slow_head_dim;
    float slow_rope_freq_base, slow_rms_norm_eps;
    int32_t slow_attention_qk_norm;
    int32_t fast_context_length, fast_embedding_length, fast_feed_forward_length,
        fast_block_count, fast_head_count, fast_head_count_kv, fast_head_dim;
    float fast_rope_freq_base, fast_rms_norm_eps;
    int32_t fast_attention_qk_norm;
    int32_t codebook_size, num_codebooks, semantic_begin_id, semantic_end_id;
    int32_t scale_codebook_embeddings, tie_word_embeddings, fast_project_in;
    int64_t vocab_size;          /* rows of embeddings.weight */
    int64_t codebook_rows;       /* rows of codebook_embeddings.weight */
    int64_t fast_vocab_size;     /* rows of fast_embeddings.weight */
} S2oGraphSpec;

typedef struct S2oModel S2oModel;

/* mode 0: weights resident, Fast-AR incremental (identical results);
 * mode 1: reference-faithful timing: Slow-AR layer weights re-expanded to f32
 * every step (slow_ar.rs:1189) and Fast-AR prefix recomputed for every
 * codebook (fast_ar.rs:245-292). */
S2oModel *s2o_open(const char *path, int64_t max_seq_len, int mode);
void s2o_close(S2oModel *m);
int s2o_graph_spec(const S2oModel *m, S2oGraphSpec *out);
int s2o_set_threads(int n);
int s2o_get_threads(void);
void s2o_reset(S2oModel *m);
int64_t s2o_n_past(const S2oModel *m);

/* SlowArState::{prefill,step} (slow_ar.rs:440-527): flat time-major tokens,
 * n_tokens*(K+1) ids.  hidden_out: d floats (post-norm, slow_ar.rs:515-526);
 * logits_out: vocab floats, or NULL.  allowed_only != 0 computes only the rows
 * [sem_begin, sem_end] and im_end_id (others set to -inf), which leaves every
 * sampled token unchanged because the semantic bias masks the rest. */
int s2o_eval(S2oModel *m, const int32_t *flat_tokens, int64_t n_flat, float *hidden_out,
             float *logits_out, int allowed_only, int64_t im_end_id);

/* forward_codebook_prefix (fast_ar.rs:360-437): logits over codebook_size. */
int s2o_fast_prefix_logits(S2oModel *m, const float *slow_hidden, const uint32_t *prefix,
                           int64_t n_prefix, float *logits_out);

typedef struct S2oGenParams {
    uint32_t max_new_tokens;
    float temperature;
    float top_p;
    int32_t top_k;
    uint32_t min_tokens_before_end;
    uint32_t im_end_id;
} S2oGenParams;

/* generate_codebooks_for_semantic (fast_ar.rs:440-470). out: num_codebooks codes. */
int s2o_generate_codebooks(S2oModel *m, const float *slow_hidden, uint32_t semantic_code,
                           float temperature, float top_p, int32_t top_k, uint64_t *rng_state,
                           uint32_t *out_codes);

/* generate_codes (generate.rs:117-221).  prompt: row-major (K+1) x cols
 * (prompt.rs:59-67).  out_codes: num_codebooks * max_new_tokens capacity,
 * compacted codebook-major on return (generate.rs:346-390).  If trace_main is
 * not NULL it receives the sampled main tokens (max_new_tokens + 1). */
int s2o_generate_codes(S2oModel *m, const uint32_t *prompt, int64_t rows, int64_t cols,
                       const S2oGenParams *params, uint64_t *rng_state, int32_t *out_codes,
                       uint32_t *out_n_frames, uint32_t *trace_main);

/* transpose_to_time_major (prompt.rs:77-103). */
int s2o_transpose_to_time_major(const uint32_t *data, int64_t rows, int64_t cols, int32_t *flat);
/* compact_codes (generate.rs:346-390): in place; returns new length via *out_len. */
int s2o_compact_codes(int32_t *codes, uint32_t num_codebooks, uint32_t max_new, uint32_t n_frames,
                      int64_t *out_len);

/* GGUF reader restated from crates/fish_s2_core/src/gguf.rs:35-120. */
typedef struct S2oGguf S2oGguf;
S2oGguf *s2o_gguf_open(const char *path);
void s2o_gguf_close(S2oGguf *g);
int64_t s2o_gguf_tensor_count(const S2oGguf *g);
uint32_t s2o_gguf_version(const S2oGguf *g);
uint64_t s2o_gguf_data_start(const S2oGguf *g);
/* tensor directory entry i: name (NUL-terminated, pointer stays valid until
 * close), rank, dims[4], ggml type, relative offset, byte length. */
int s2o_gguf_tensor_info(const S2oGguf *g, int64_t i, const char **name, int32_t *rank,
                         uint64_t *dims, uint32_t *ggml_type, uint64_t *rel_offset,
                         uint64_t *byte_len);
const void *s2o_gguf_tensor_data(const S2oGguf *g, const char *name, uint64_t *byte_len);
/* metadata value rendered as the reference renders it (gguf.rs:396-453). */
int s2o_gguf_metadata(const S2oGguf *g, const char *key, char *buf, size_t cap);
/* ggml block dequantisation to f32 (ggml's public block formats; not in the
 * reference, which is F16-only: crates/fish_s2_core/src/gguf.rs:233-258). */
int s2o_dequant_row(uint32_t ggml_type, const void *src, int64_t n_elements, float *dst);
int64_t s2o_ggml_byte_len(uint32_t ggml_type, int64_t n_elements);

#ifdef __cplusplus
}
#endif
#endif
