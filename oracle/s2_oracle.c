/*
 * s2_oracle.c -- CPU restatement of fish-s2pro's `rust-pure` Dual-AR math.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker and the timed CPU baseline);
 * see s2_oracle.h.  Build flags matter: -ffp-contract=off keeps every
 * `a * b + c` of the reference as two roundings (Rust never fuses them), and
 * no -ffast-math so that every reduction stays in the reference's sequential
 * order.  Row-parallelism over output rows mirrors rayon's par_iter_mut in
 * backend.rs:65-71 / tensor.rs:247-262; each output element is still one
 * sequential f32 sum, so the thread count never changes a result.
 *
 * Citations are `path:line` inside the reference repository.
 */
#define _GNU_SOURCE
#include "s2_oracle.h"

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <omp.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------------- */
/* errors                                                                     */
/* ------------------------------------------------------------------------- */

static __thread char g_err[1024];

const char *s2o_last_error(void) { return g_err; }

static int fail(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return -1;
}

/* ------------------------------------------------------------------------- */
/* f16 <-> f32: crates/fish_s2_infer/src/tensor.rs:266-329                    */
/* ------------------------------------------------------------------------- */

static float bits_f32(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}

static uint32_t f32_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

/* tensor.rs:266-287 */
float s2o_f16_to_f32(uint16_t bits) {
    uint32_t sign = ((uint32_t)(bits & 0x8000u)) << 16;
    uint32_t exponent = (bits >> 10) & 0x1fu;
    uint32_t fraction = bits & 0x03ffu;
    if (exponent == 0 && fraction == 0) return bits_f32(sign);
    if (exponent == 0) {
        float value = (float)fraction * 5.9604644775390625e-8f; /* 2^-24, exact */
        return sign == 0 ? value : -value;
    }
    if (exponent == 0x1f && fraction == 0) return bits_f32(sign | 0x7f800000u);
    if (exponent == 0x1f) return bits_f32(sign | 0x7f800000u | (fraction << 13));
    return bits_f32(sign | ((exponent + 112u) << 23) | (fraction << 13));
}

/* tensor.rs:289-325 */
uint16_t s2o_f32_to_f16(float value) {
    uint32_t bits = f32_bits(value);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exponent = (int32_t)((bits >> 23) & 0xffu);
    uint32_t mantissa = bits & 0x007fffffu;
    if (exponent == 0xff) {
        if (mantissa == 0) return sign | 0x7c00u;
        return sign | 0x7e00u;
    }
    int32_t half_exp = exponent - 127 + 15;
    if (half_exp >= 0x1f) return sign | 0x7c00u;
    if (half_exp <= 0) {
        if (half_exp < -10) return sign;
        uint32_t m = mantissa | 0x00800000u;
        uint32_t shift = (uint32_t)(14 - half_exp);
        uint32_t rounded = m + ((1u << (shift - 1)) - 1) + ((m >> shift) & 1u);
        return sign | (uint16_t)(rounded >> shift);
    }
    uint32_t rounded = mantissa + 0x00000fffu + ((mantissa >> 13) & 1u);
    if (rounded & 0x00800000u) {
        int32_t next_exp = half_exp + 1;
        if (next_exp >= 0x1f) return sign | 0x7c00u;
        return sign | (uint16_t)(next_exp << 10);
    }
    return sign | (uint16_t)(half_exp << 10) | (uint16_t)(rounded >> 13);
}

/* tensor.rs:327-329 */
float s2o_round_f32_to_f16(float value) { return s2o_f16_to_f32(s2o_f32_to_f16(value)); }

static float g_f16_lut[65536];
static int g_f16_lut_ready = 0;

static void f16_lut_init(void) {
    if (__atomic_load_n(&g_f16_lut_ready, __ATOMIC_ACQUIRE)) return;
#pragma omp critical(s2o_lut)
    {
        if (!g_f16_lut_ready) {
            for (uint32_t i = 0; i < 65536u; ++i) g_f16_lut[i] = s2o_f16_to_f32((uint16_t)i);
            __atomic_store_n(&g_f16_lut_ready, 1, __ATOMIC_RELEASE);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* ggml block formats (not in the reference, which is F16-only:              */
/* crates/fish_s2_core/src/gguf.rs:233-258 gives only the block byte sizes). */
/* Restated from ggml's published block layouts, pinned at s2.cpp commit      */
/* 2b9c6d2984f92b186419420e9126c47919b81d3a (docs/S2_CPP_PIN.md:5-6).         */
/* The canonical value is computed with separate roundings (no FMA):          */
/*   Q8_0: v = d * q                                                          */
/*   Q4_K: v = (d*sc) * q - (dmin*m)                                          */
/* ------------------------------------------------------------------------- */

enum { GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8, GGML_Q4_K = 12 };

int64_t s2o_ggml_byte_len(uint32_t t, int64_t n) {
    switch (t) {
    case GGML_F32: return n * 4;
    case GGML_F16: return n * 2;
    case GGML_Q8_0: return (n + 31) / 32 * 34;
    case GGML_Q4_K: return (n + 255) / 256 * 144;
    default: return -1;
    }
}

static void q4k_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = q[j] & 63u;
        *m = q[j + 4] & 63u;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0x0fu) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

int s2o_dequant_row(uint32_t t, const void *src, int64_t n, float *dst) {
    const uint8_t *p = (const uint8_t *)src;
    if (t == GGML_F32) {
        memcpy(dst, src, (size_t)n * 4);
        return 0;
    }
    if (t == GGML_F16) {
        const uint16_t *h = (const uint16_t *)src;
        for (int64_t i = 0; i < n; ++i) dst[i] = s2o_f16_to_f32(h[i]);
        return 0;
    }
    if (t == GGML_Q8_0) {
        if (n % 32) return fail("Q8_0 row length %lld is not a multiple of 32", (long long)n);
        for (int64_t b = 0; b < n / 32; ++b) {
            const uint8_t *blk = p + b * 34;
            uint16_t dbits = (uint16_t)(blk[0] | (blk[1] << 8));
            float d = s2o_f16_to_f32(dbits);
            for (int j = 0; j < 32; ++j) dst[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
        }
        return 0;
    }
    if (t == GGML_Q4_K) {
        if (n % 256) return fail("Q4_K row length %lld is not a multiple of 256", (long long)n);
        for (int64_t b = 0; b < n / 256; ++b) {
            const uint8_t *blk = p + b * 144;
            float d = s2o_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            float dmin = s2o_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const uint8_t *scales = blk + 4;
            const uint8_t *q = blk + 16;
            float *y = dst + b * 256;
            for (int g = 0; g < 4; ++g) {
                uint8_t sc, m;
                q4k_scale_min(2 * g, scales, &sc, &m);
                float d1 = d * (float)sc, m1 = dmin * (float)m;
                q4k_scale_min(2 * g + 1, scales, &sc, &m);
                float d2 = d * (float)sc, m2 = dmin * (float)m;
                for (int l = 0; l < 32; ++l) {
                    float t1 = d1 * (float)(q[l] & 0x0fu);
                    y[l] = t1 - m1;
                }
                for (int l = 0; l < 32; ++l) {
                    float t2 = d2 * (float)(q[l] >> 4);
                    y[32 + l] = t2 - m2;
                }
                q += 32;
                y += 64;
            }
        }
        return 0;
    }
    return fail("unsupported ggml type %u", t);
}

/* ------------------------------------------------------------------------- */
/* threading                                                                  */
/* ------------------------------------------------------------------------- */

int s2o_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
}

int s2o_get_threads(void) { return omp_get_max_threads(); }

/* ------------------------------------------------------------------------- */
/* op-level math: crates/fish_s2_infer/src/backend.rs                         */
/* ------------------------------------------------------------------------- */

/* backend.rs:76-82 dot_f32: `iter().map(a*b).sum()`; Rust's f32 Sum folds
 * from -0.0 (it only changes the sign of an all-zero sum). */
static inline float dot_f32(const float *a, const float *b, int64_t n) {
    float s = -0.0f;
    for (int64_t i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

/* backend.rs:84-102 */
static void rms_norm_f32(const float *x, const float *w, int64_t n, float eps, float *out) {
    float ss = -0.0f;
    for (int64_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float mean_square = ss / (float)n;
    float scale = 1.0f / sqrtf(mean_square + eps);
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

int s2o_rms_norm(const float *input, const float *weight, int64_t n, float eps, float *out) {
    if (n <= 0) return fail("rms_norm input is empty");
    rms_norm_f32(input, weight, n, eps, out);
    return 0;
}

/* backend.rs:104-121 */
int s2o_rms_norm_heads(const float *input, const float *weight, int64_t n, int64_t head_dim,
                       float eps, float *out) {
    if (head_dim <= 0 || n % head_dim)
        return fail("head RMSNorm input length %lld is not a multiple of head_dim %lld",
                    (long long)n, (long long)head_dim);
    for (int64_t h = 0; h < n / head_dim; ++h)
        rms_norm_f32(input + h * head_dim, weight, head_dim, eps, out + h * head_dim);
    return 0;
}

/* backend.rs:55-73: one sequential dot per output row, rows in parallel. */
int s2o_linear(const float *input, const float *weight, int64_t in_dim, int64_t out_dim,
               float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < out_dim; ++o) out[o] = dot_f32(input, weight + o * in_dim, in_dim);
    return 0;
}

/* tensor.rs:220-264: `let mut sum = 0.0; sum += x * w` over f16 row bytes. */
int s2o_matvec_f16(const float *input, const uint16_t *weight, int64_t in_dim, int64_t out_dim,
                   float *out) {
    f16_lut_init();
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < out_dim; ++o) {
        const uint16_t *row = weight + o * in_dim;
        float s = 0.0f;
        for (int64_t i = 0; i < in_dim; ++i) s += input[i] * g_f16_lut[row[i]];
        out[o] = s;
    }
    return 0;
}

/* attention.rs:172-206 (NORMAL mode RoPE: adjacent pairs). */
int s2o_rope_normal(float *values, int64_t n, int64_t head_dim, int64_t position,
                    float rope_base) {
    if (head_dim == 0 || head_dim % 2)
        return fail("RoPE head_dim must be non-zero and even, got %lld", (long long)head_dim);
    if (n % head_dim)
        return fail("RoPE values length %lld is not a multiple of head_dim %lld", (long long)n,
                    (long long)head_dim);
    if (!(rope_base > 0.0f)) return fail("RoPE base must be positive, got %g", rope_base);
    for (int64_t h = 0; h < n / head_dim; ++h) {
        float *head = values + h * head_dim;
        for (int64_t pair = 0; pair < head_dim; pair += 2) {
            float theta = (float)position / powf(rope_base, (float)pair / (float)head_dim);
            float s = sinf(theta), c = cosf(theta);
            float x0 = head[pair], x1 = head[pair + 1];
            head[pair] = x0 * c - x1 * s;
            head[pair + 1] = x0 * s + x1 * c;
        }
    }
    return 0;
}

/* attention.rs:296-309 */
static void softmax_in_place(float *v, int64_t n) {
    float max = -INFINITY;
    for (int64_t i = 0; i < n; ++i) max = fmaxf(max, v[i]);
    float sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        v[i] = expf(v[i] - max);
        sum += v[i];
    }
    for (int64_t i = 0; i < n; ++i) v[i] /= sum;
}

/* attention.rs:208-247; keys/values token-major [T][Hkv][hd]. */
int s2o_gqa_decode_attention(const float *query, const float *keys, const float *values,
                             int64_t H, int64_t Hkv, int64_t hd, int64_t T, float attn_scale,
                             float *out) {
    if (Hkv == 0 || H % Hkv) return fail("invalid GQA split: heads=%lld, kv_heads=%lld",
                                         (long long)H, (long long)Hkv);
    if (hd == 0 || T == 0)
        return fail("invalid attention dims: head_dim=%lld, token_count=%lld", (long long)hd,
                    (long long)T);
    int64_t rep = H / Hkv;
    float *scores = (float *)malloc(sizeof(float) * (size_t)T);
    if (!scores) return fail("out of memory");
    memset(out, 0, sizeof(float) * (size_t)(H * hd));
    for (int64_t qh = 0; qh < H; ++qh) {
        int64_t kvh = qh / rep;
        const float *q = query + qh * hd;
        for (int64_t t = 0; t < T; ++t)
            scores[t] = dot_f32(q, keys + (t * Hkv + kvh) * hd, hd) * attn_scale;
        softmax_in_place(scores, T);
        float *o = out + qh * hd;
        for (int64_t t = 0; t < T; ++t) {
            const float *v = values + (t * Hkv + kvh) * hd;
            for (int64_t d = 0; d < hd; ++d) o[d] += scores[t] * v[d];
        }
    }
    free(scores);
    return 0;
}

/* slow_ar.rs:1215-1232: g * sigmoid(g) * u with sigmoid = 1/(1+exp(-g)). */
int s2o_swiglu_slow(const float *gate, const float *up, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) {
        float sig = 1.0f / (1.0f + expf(-gate[i]));
        out[i] = gate[i] * sig * up[i];
    }
    return 0;
}

/* fast_ar.rs:472-485: g / (1 + exp(-g)) * u. */
int s2o_swiglu_fast(const float *gate, const float *up, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = gate[i] / (1.0f + expf(-gate[i])) * up[i];
    return 0;
}

/* ------------------------------------------------------------------------- */
/* sampling: crates/fish_s2_infer/src/sampling.rs                             */
/* ------------------------------------------------------------------------- */

/* sampling.rs:46-52 */
double s2o_rng_next_unit(uint64_t *state) {
    *state = *state * 6364136223846793005ull + 1ull;
    uint64_t mantissa = (*state >> 11) & ((1ull << 53) - 1ull);
    return (double)mantissa / 9007199254740992.0;
}

/* sampling.rs:55-73 */
int s2o_build_semantic_bias(int64_t vocab, uint32_t sem_begin, uint32_t sem_end,
                            int64_t im_end_id, float *bias) {
    for (int64_t i = 0; i < vocab; ++i) bias[i] = -INFINITY;
    for (uint64_t id = sem_begin; id <= sem_end; ++id)
        if ((int64_t)id < vocab) bias[id] = 0.0f;
    if (im_end_id >= 0 && im_end_id < vocab) bias[im_end_id] = 0.0f;
    return 0;
}

/* sampling.rs:76-100 */
int s2o_apply_semantic_bias(float *logits, const float *bias, int64_t n, int block_im_end,
                            int64_t im_end_id) {
    for (int64_t i = 0; i < n; ++i) logits[i] += bias[i];
    if (block_im_end && im_end_id >= 0 && im_end_id < n) logits[im_end_id] = -INFINITY;
    return 0;
}

/* sampling.rs:103-118 */
int s2o_semantic_mask_logits(float *logits, int64_t n, uint32_t sem_begin, uint32_t sem_end,
                             int64_t im_end_id, int block_im_end) {
    for (int64_t i = 0; i < n; ++i) {
        uint32_t id = (uint32_t)i;
        int in_sem = id >= sem_begin && id <= sem_end;
        int im_end_allowed = im_end_id >= 0 && (int64_t)id == im_end_id && !block_im_end;
        if (!in_sem && !im_end_allowed) logits[i] = -INFINITY;
    }
    return 0;
}

typedef struct {
    float v;
    uint32_t id;
} Item;

/* Stable sort, descending by value, exactly like
 * `items.sort_by(|a, b| b.0.partial_cmp(&a.0).unwrap_or(Equal))`:
 * b is placed before a only when b.v > a.v. */
static void stable_sort_desc(Item *a, int64_t n, Item *tmp) {
    for (int64_t width = 1; width < n; width *= 2) {
        for (int64_t lo = 0; lo < n; lo += 2 * width) {
            int64_t mid = lo + width < n ? lo + width : n;
            int64_t hi = lo + 2 * width < n ? lo + 2 * width : n;
            int64_t i = lo, j = mid, k = lo;
            while (i < mid && j < hi) {
                if (a[j].v > a[i].v) tmp[k++] = a[j++];
                else tmp[k++] = a[i++];
            }
            while (i < mid) tmp[k++] = a[i++];
            while (j < hi) tmp[k++] = a[j++];
        }
        memcpy(a, tmp, sizeof(Item) * (size_t)n);
    }
}

/* sampling.rs:202-225 */
static void apply_softmax(float *p, int64_t n, float temperature) {
    if (n == 0) return;
    float max_val = -INFINITY;
    for (int64_t i = 0; i < n; ++i) max_val = fmaxf(max_val, p[i]);
    float sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        if (temperature > 0.0f) p[i] = expf((p[i] - max_val) / temperature);
        else p[i] = fabsf(p[i] - max_val) < 1e-6f ? 1.0f : 0.0f;
        sum += p[i];
    }
    if (sum > 0.0f)
        for (int64_t i = 0; i < n; ++i) p[i] /= sum;
}

/* sampling.rs:227-241 */
static int64_t sample_discrete(const float *probs, int64_t n, uint64_t *rng) {
    double draw = s2o_rng_next_unit(rng);
    float target = (float)draw;
    if (target < 0.0f) target = 0.0f;
    if (target > 1.0f - 1e-7f) target = 1.0f - 1e-7f;
    float cumsum = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        cumsum += probs[i];
        if (target < cumsum) return i;
    }
    return n - 1;
}

/* sampling.rs:121-200 */
int s2o_sample_token(const float *logits, int64_t vocab, float temperature, float top_p,
                     int32_t top_k, int64_t always_include_id, uint64_t *rng_state,
                     uint32_t *out_token) {
    if (vocab == 0) {
        *out_token = 0;
        return 0;
    }
    Item *items = (Item *)malloc(sizeof(Item) * (size_t)(vocab + 1));
    Item *tmp = (Item *)malloc(sizeof(Item) * (size_t)(vocab + 1));
    float *probs = (float *)malloc(sizeof(float) * (size_t)(vocab + 1));
    if (!items || !tmp || !probs) {
        free(items), free(tmp), free(probs);
        return fail("out of memory");
    }
    for (int64_t i = 0; i < vocab; ++i) items[i] = (Item){logits[i], (uint32_t)i};
    stable_sort_desc(items, vocab, tmp);
    int64_t k = top_k > 0 ? ((int64_t)top_k < vocab ? (int64_t)top_k : vocab) : vocab;
    int64_t n = k;
    if (always_include_id >= 0 && always_include_id < vocab) {
        float force_logit = logits[always_include_id];
        if (force_logit > -1e30f) {
            int present = 0;
            for (int64_t i = 0; i < n; ++i)
                if (items[i].id == (uint32_t)always_include_id) present = 1;
            if (!present) items[n++] = (Item){force_logit, (uint32_t)always_include_id};
        }
    }
    stable_sort_desc(items, n, tmp);
    if (n == 0) {
        *out_token = 0;
        free(items), free(tmp), free(probs);
        return 0;
    }
    for (int64_t i = 0; i < n; ++i) probs[i] = items[i].v;
    apply_softmax(probs, n, temperature);
    int64_t always_pos = -1;
    if (always_include_id >= 0)
        for (int64_t i = 0; i < n; ++i)
            if (items[i].id == (uint32_t)always_include_id) {
                always_pos = i;
                break;
            }
    int64_t p_idx = 0;
    float cumsum = 0.0f;
    while (p_idx < n) {
        cumsum += probs[p_idx];
        p_idx += 1;
        if (cumsum >= top_p) break;
    }
    if (p_idx == 0) p_idx = 1;
    if (always_pos >= 0 && always_pos >= p_idx) p_idx = always_pos + 1;
    float sum_p = -0.0f;
    for (int64_t i = 0; i < p_idx; ++i) sum_p += probs[i];
    if (sum_p > 0.0f)
        for (int64_t i = 0; i < p_idx; ++i) probs[i] /= sum_p;
    int64_t choice = sample_discrete(probs, p_idx, rng_state);
    *out_token = items[choice].id;
    free(items), free(tmp), free(probs);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* KV cache: attention.rs:14-170, layout [hd, Hkv, max_seq, layers]           */
/* ------------------------------------------------------------------------- */

struct S2oKvCache {
    int64_t hd, hkv, max_seq, layers;
    float *keys, *values;
};

S2oKvCache *s2o_kv_new(int64_t hd, int64_t hkv, int64_t max_seq, int64_t layers) {
    S2oKvCache *kv = (S2oKvCache *)calloc(1, sizeof *kv);
    if (!kv) return NULL;
    kv->hd = hd, kv->hkv = hkv, kv->max_seq = max_seq, kv->layers = layers;
    size_t len = (size_t)(hd * hkv * max_seq * layers);
    kv->keys = (float *)calloc(len ? len : 1, sizeof(float));
    kv->values = (float *)calloc(len ? len : 1, sizeof(float));
    if (!kv->keys || !kv->values) {
        s2o_kv_free(kv);
        fail("KV cache allocation failed");
        return NULL;
    }
    return kv;
}

void s2o_kv_free(S2oKvCache *kv) {
    if (!kv) return;
    free(kv->keys);
    free(kv->values);
    free(kv);
}

/* attention.rs:151-169 */
static int64_t kv_offset(const S2oKvCache *kv, int64_t layer, int64_t token) {
    if (layer >= kv->layers || token >= kv->max_seq || layer < 0 || token < 0) {
        fail("KV cache index out of bounds: layer=%lld, token=%lld, kv_head=0, dim=0",
             (long long)layer, (long long)token);
        return -1;
    }
    return kv->hd * kv->hkv * (token + kv->max_seq * layer);
}

/* attention.rs:56-76 */
int s2o_kv_write_token(S2oKvCache *kv, int64_t layer, int64_t token, const float *key,
                       const float *value) {
    int64_t off = kv_offset(kv, layer, token);
    if (off < 0) return -1;
    memcpy(kv->keys + off, key, sizeof(float) * (size_t)(kv->hd * kv->hkv));
    memcpy(kv->values + off, value, sizeof(float) * (size_t)(kv->hd * kv->hkv));
    return 0;
}

int s2o_kv_read_token(const S2oKvCache *kv, int64_t layer, int64_t token, float *key,
                      float *value) {
    int64_t off = kv_offset(kv, layer, token);
    if (off < 0) return -1;
    if (key) memcpy(key, kv->keys + off, sizeof(float) * (size_t)(kv->hd * kv->hkv));
    if (value) memcpy(value, kv->values + off, sizeof(float) * (size_t)(kv->hd * kv->hkv));
    return 0;
}

/* attention.rs:106-145: the visible tokens of one layer are contiguous in this
 * layout, so the reference's per-call copy is a plain view here. */
int s2o_kv_decode_attention(const S2oKvCache *kv, int64_t layer, int64_t token_count,
                            const float *query, int64_t head_count, float attn_scale,
                            float *out) {
    if (token_count > kv->max_seq)
        return fail("token_count %lld exceeds KV cache max_seq_len %lld",
                    (long long)token_count, (long long)kv->max_seq);
    if (layer >= kv->layers)
        return fail("layer %lld exceeds KV cache block_count %lld", (long long)layer,
                    (long long)kv->layers);
    int64_t off = kv->hd * kv->hkv * kv->max_seq * layer;
    return s2o_gqa_decode_attention(query, kv->keys + off, kv->values + off, head_count, kv->hkv,
                                    kv->hd, token_count, attn_scale, out);
}

/* ------------------------------------------------------------------------- */
/* weight views: f32 (toy tests, faithful mode), f16 / Q8_0 / Q4_K (GGUF)     */
/* ------------------------------------------------------------------------- */

typedef struct {
    const void *p;
    uint32_t type;
    int64_t in_dim, out_dim; /* rows of length in_dim, out_dim rows */
} WView;

static size_t wrow_bytes(const WView *w) { return (size_t)s2o_ggml_byte_len(w->type, w->in_dim); }

/* Expand rows [o, o+nr) of w into buf (nr * in_dim floats), exactly. */
static void wrows_f32(const WView *w, int64_t o, int64_t nr, float *buf) {
    if (w->type == GGML_F32) {
        memcpy(buf, (const float *)w->p + o * w->in_dim, sizeof(float) * (size_t)(nr * w->in_dim));
        return;
    }
    const uint8_t *base = (const uint8_t *)w->p + (size_t)o * wrow_bytes(w);
    if (w->type == GGML_F16) {
        const uint16_t *h = (const uint16_t *)base;
        for (int64_t i = 0; i < nr * w->in_dim; ++i) buf[i] = g_f16_lut[h[i]];
        return;
    }
    for (int64_t r = 0; r < nr; ++r)
        s2o_dequant_row(w->type, base + (size_t)r * wrow_bytes(w), w->in_dim, buf + r * w->in_dim);
}

/* Y[t][o] = sum_i X[t][i] * W[o][i] for T tokens, each sum sequential from
 * `init` (-0.0 for backend.rs:76-82 dot_f32, +0.0 for tensor.rs:247-262).
 * Weight-stationary: a block of rows is expanded once and used for all T
 * tokens; four rows advance together to give the CPU independent chains. */
static int linear_multi(const WView *w, const float *X, int64_t T, float *Y, float init) {
    const int64_t in = w->in_dim, out = w->out_dim;
    const int64_t RB = 4;
    int err = 0;
    f16_lut_init();
#pragma omp parallel
    {
        float *buf = (float *)malloc(sizeof(float) * (size_t)(RB * in));
        if (!buf) {
#pragma omp atomic write
            err = 1;
        } else {
#pragma omp for schedule(static)
            for (int64_t ob = 0; ob < (out + RB - 1) / RB; ++ob) {
                int64_t o = ob * RB, nr = out - o < RB ? out - o : RB;
                wrows_f32(w, o, nr, buf);
                for (int64_t t = 0; t < T; ++t) {
                    const float *x = X + t * in;
                    if (nr == 4) {
                        const float *w0 = buf, *w1 = buf + in, *w2 = buf + 2 * in, *w3 = buf + 3 * in;
                        float s0 = init, s1 = init, s2 = init, s3 = init;
                        for (int64_t i = 0; i < in; ++i) {
                            float xi = x[i];
                            s0 += xi * w0[i];
                            s1 += xi * w1[i];
                            s2 += xi * w2[i];
                            s3 += xi * w3[i];
                        }
                        float *y = Y + t * out + o;
                        y[0] = s0, y[1] = s1, y[2] = s2, y[3] = s3;
                    } else {
                        for (int64_t r = 0; r < nr; ++r) {
                            float s = init;
                            const float *wr = buf + r * in;
                            for (int64_t i = 0; i < in; ++i) s += x[i] * wr[i];
                            Y[t * out + o + r] = s;
                        }
                    }
                }
            }
            free(buf);
        }
    }
    return err ? fail("out of memory in linear") : 0;
}

/* ------------------------------------------------------------------------- */
/* one transformer layer (Slow-AR: slow_ar.rs:558-854; Fast-AR: fast_ar.rs)   */
/* ------------------------------------------------------------------------- */

typedef struct {
    int64_t d, F, H, Hkv, hd;
    float rope_base, eps;
    int qk_norm;   /* slow: QK RMSNorm per head (slow_ar.rs:748-763); fast: none */
    int fast_act;  /* SwiGLU rounding: fast_ar.rs:472-485 vs slow_ar.rs:1215-1232 */
} LShape;

typedef struct {
    const float *attn_norm, *q_norm, *k_norm, *ffn_norm; /* f32 (expanded norm gains) */
    WView wqkv, wo, w1, w2, w3;
} LWeights;

/* A per-layer KV store: contiguous [layer][token][Hkv*hd] f32 (the reference
 * layout restricted to one sequence). */
typedef struct {
    float *k, *v;
    int64_t max_seq, width;
} LKv;

/* Run one layer over n tokens at positions start..start+n-1, reference
 * prefill order: prepare all tokens, write the K/V span, attention per token
 * over its visible prefix, then the FFN per token (slow_ar.rs:558-617).
 * Decode of one token is the n == 1 case (slow_ar.rs:637-710).  X is updated
 * in place ([n][d]).  trace (optional) receives intermediate rows. */
static int layer_forward(const LShape *s, const LWeights *w, float *X, int64_t n, float *kbase,
                         float *vbase, int64_t start, S2oLayerTrace *trace) {
    const int64_t d = s->d, qs = s->H * s->hd, kvs = s->Hkv * s->hd, qkv_out = qs + 2 * kvs;
    float *norm = (float *)malloc(sizeof(float) * (size_t)(n * d));
    float *qkv = (float *)malloc(sizeof(float) * (size_t)(n * qkv_out));
    float *q = (float *)malloc(sizeof(float) * (size_t)(n * qs));
    float *att = (float *)malloc(sizeof(float) * (size_t)(n * qs));
    float *proj = (float *)malloc(sizeof(float) * (size_t)(n * d));
    float *gate = (float *)malloc(sizeof(float) * (size_t)(n * s->F));
    float *up = (float *)malloc(sizeof(float) * (size_t)(n * s->F));
    float *act = (float *)malloc(sizeof(float) * (size_t)(n * s->F));
    int rc = 0;
    if (!norm || !qkv || !q || !att || !proj || !gate || !up || !act) {
        rc = fail("out of memory in layer_forward");
        goto done;
    }
    /* prepare_decode_token (slow_ar.rs:722-789) / prepare_token (fast_ar.rs:294-323) */
    for (int64_t t = 0; t < n; ++t) rms_norm_f32(X + t * d, w->attn_norm, d, s->eps, norm + t * d);
    if (trace && trace->normalized) memcpy(trace->normalized, norm, sizeof(float) * (size_t)(n * d));
    if ((rc = linear_multi(&w->wqkv, norm, n, qkv, -0.0f))) goto done;
    for (int64_t t = 0; t < n; ++t) {
        const float *row = qkv + t * qkv_out;
        float *qt = q + t * qs;
        float *kt = kbase + (start + t) * kvs, *vt = vbase + (start + t) * kvs;
        if (s->qk_norm) {
            s2o_rms_norm_heads(row, w->q_norm, qs, s->hd, s->eps, qt);
            s2o_rms_norm_heads(row + qs, w->k_norm, kvs, s->hd, s->eps, kt);
        } else {
            memcpy(qt, row, sizeof(float) * (size_t)qs);
            memcpy(kt, row + qs, sizeof(float) * (size_t)kvs);
        }
        memcpy(vt, row + qs + kvs, sizeof(float) * (size_t)kvs);
        s2o_rope_normal(qt, qs, s->hd, start + t, s->rope_base);
        s2o_rope_normal(kt, kvs, s->hd, start + t, s->rope_base);
        if (trace) {
            if (trace->query) memcpy(trace->query + t * qs, qt, sizeof(float) * (size_t)qs);
            if (trace->key) memcpy(trace->key + t * kvs, kt, sizeof(float) * (size_t)kvs);
            if (trace->value) memcpy(trace->value + t * kvs, vt, sizeof(float) * (size_t)kvs);
        }
    }
    /* finish_decode_token (slow_ar.rs:811-854): attention over visible prefix */
    const float scale = 1.0f / sqrtf((float)s->hd);
    for (int64_t t = 0; t < n; ++t) {
        if ((rc = s2o_gqa_decode_attention(q + t * qs, kbase, vbase, s->H, s->Hkv, s->hd,
                                           start + t + 1, scale, att + t * qs)))
            goto done;
    }
    if (trace && trace->attention) memcpy(trace->attention, att, sizeof(float) * (size_t)(n * qs));
    if ((rc = linear_multi(&w->wo, att, n, proj, -0.0f))) goto done;
    if (trace && trace->projected) memcpy(trace->projected, proj, sizeof(float) * (size_t)(n * d));
    for (int64_t i = 0; i < n * d; ++i) X[i] = X[i] + proj[i];
    if (trace && trace->attn_hidden) memcpy(trace->attn_hidden, X, sizeof(float) * (size_t)(n * d));
    /* forward_feed_forward (slow_ar.rs:659-710, fast_ar.rs:325-352) */
    for (int64_t t = 0; t < n; ++t) rms_norm_f32(X + t * d, w->ffn_norm, d, s->eps, norm + t * d);
    if (trace && trace->ffn_normalized)
        memcpy(trace->ffn_normalized, norm, sizeof(float) * (size_t)(n * d));
    if ((rc = linear_multi(&w->w1, norm, n, gate, -0.0f))) goto done;
    if ((rc = linear_multi(&w->w3, norm, n, up, -0.0f))) goto done;
    if (s->fast_act) s2o_swiglu_fast(gate, up, n * s->F, act);
    else s2o_swiglu_slow(gate, up, n * s->F, act);
    if (trace) {
        if (trace->gate) memcpy(trace->gate, gate, sizeof(float) * (size_t)(n * s->F));
        if (trace->up) memcpy(trace->up, up, sizeof(float) * (size_t)(n * s->F));
        if (trace->activated) memcpy(trace->activated, act, sizeof(float) * (size_t)(n * s->F));
    }
    if ((rc = linear_multi(&w->w2, act, n, proj, -0.0f))) goto done;
    if (trace && trace->ffn_projected)
        memcpy(trace->ffn_projected, proj, sizeof(float) * (size_t)(n * d));
    for (int64_t i = 0; i < n * d; ++i) X[i] = X[i] + proj[i];
    if (trace && trace->hidden) memcpy(trace->hidden, X, sizeof(float) * (size_t)(n * d));
done:
    free(norm), free(qkv), free(q), free(att), free(proj), free(gate), free(up), free(act);
    return rc;
}

/* Toy-weight entry point mirroring SlowArLayerSkeleton (slow_ar.rs:188-918). */
int s2o_layer_forward(const S2oLayerShape *sh, const S2oLayerWeightsF32 *w,
                      const float *hidden_tokens, int64_t n_tokens, S2oKvCache *kv, int64_t layer,
                      int64_t start_position, int decode_loop, S2oLayerTrace *trace,
                      float *hidden_out) {
    /* SlowArLayerShape::validate (slow_ar.rs:63-95) */
    if (sh->hidden_size == 0) return fail("hidden_size must be non-zero");
    if (sh->feed_forward_size == 0) return fail("feed_forward_size must be non-zero");
    if (sh->head_count_kv == 0 || sh->head_count % sh->head_count_kv)
        return fail("invalid GQA split: heads=%lld, kv_heads=%lld", (long long)sh->head_count,
                    (long long)sh->head_count_kv);
    if (sh->head_dim == 0 || sh->head_dim % 2)
        return fail("head_dim must be non-zero and even, got %lld", (long long)sh->head_dim);
    if (!(sh->rope_base > 0.0f)) return fail("rope_base must be positive, got %g", sh->rope_base);
    const int64_t d = sh->hidden_size, qs = sh->head_count * sh->head_dim,
                  kvs = sh->head_count_kv * sh->head_dim, F = sh->feed_forward_size;
    /* SlowArLayerSkeleton::validate (slow_ar.rs:856-918) */
    struct {
        const char *name;
        int64_t got, want;
    } checks[] = {
        {"attention_norm_weight", w->n_attention_norm, d},
        {"q_norm_weight", w->n_q_norm, sh->head_dim},
        {"k_norm_weight", w->n_k_norm, sh->head_dim},
        {"wqkv_weight", w->n_wqkv, d * (qs + 2 * kvs)},
        {"output_weight", w->n_wo, qs * d},
        {"ffn_norm_weight", w->n_ffn_norm, d},
        {"feed_forward_w1_weight", w->n_w1, d * F},
        {"feed_forward_w2_weight", w->n_w2, F * d},
        {"feed_forward_w3_weight", w->n_w3, d * F},
    };
    for (size_t i = 0; i < sizeof checks / sizeof checks[0]; ++i)
        if (checks[i].got != checks[i].want)
            return fail("%s length mismatch: expected %lld, got %lld", checks[i].name,
                        (long long)checks[i].want, (long long)checks[i].got);
    if (kv->hd != sh->head_dim || kv->hkv != sh->head_count_kv)
        return fail("KV token width mismatch");
    if (start_position + n_tokens > kv->max_seq || layer >= kv->layers)
        return fail("KV cache index out of bounds: layer=%lld, token=%lld, kv_head=0, dim=0",
                    (long long)layer, (long long)(start_position + n_tokens - 1));
    LShape s = {d, F, sh->head_count, sh->head_count_kv, sh->head_dim, sh->rope_base,
                sh->rms_norm_eps, 1, 0};
    LWeights lw = {w->attention_norm, w->q_norm, w->k_norm, w->ffn_norm,
                   {w->wqkv, GGML_F32, d, qs + 2 * kvs}, {w->wo, GGML_F32, qs, d},
                   {w->w1, GGML_F32, d, F}, {w->w2, GGML_F32, F, d}, {w->w3, GGML_F32, d, F}};
    float *kbase = kv->keys + kvs * kv->max_seq * layer;
    float *vbase = kv->values + kvs * kv->max_seq * layer;
    memcpy(hidden_out, hidden_tokens, sizeof(float) * (size_t)(n_tokens * d));
    if (!decode_loop) return layer_forward(&s, &lw, hidden_out, n_tokens, kbase, vbase, start_position, trace);
    /* forward_decode_sequence + forward_feed_forward, one token at a time. */
    for (int64_t t = 0; t < n_tokens; ++t) {
        S2oLayerTrace tt, *tp = NULL;
        if (trace) {
#define OFS(field, width) tt.field = trace->field ? trace->field + t * (width) : NULL
            OFS(normalized, d); OFS(query, qs); OFS(key, kvs); OFS(value, kvs);
            OFS(attention, qs); OFS(projected, d); OFS(attn_hidden, d); OFS(ffn_normalized, d);
            OFS(gate, F); OFS(up, F); OFS(activated, F); OFS(ffn_projected, d); OFS(hidden, d);
#undef OFS
            tp = &tt;
        }
        int rc = layer_forward(&s, &lw, hidden_out + t * d, 1, kbase, vbase, start_position + t, tp);
        if (rc) return rc;
    }
    return 0;
}

/* ------------------------------------------------------------------------- */
/* GGUF: crates/fish_s2_core/src/gguf.rs:35-120, 319-503                      */
/* ------------------------------------------------------------------------- */

typedef struct {
    char *key;
    uint32_t type;
    char *text; /* the value rendered as the reference renders it */
    uint64_t u;
    int64_t i;
    double f;
} MetaKV;

typedef struct {
    char *name;
    int32_t rank;
    uint64_t dims[4];
    uint32_t type;
    uint64_t rel;
    uint64_t bytes;
} TInfo;

struct S2oGguf {
    int fd;
    const uint8_t *map;
    size_t size;
    uint32_t version;
    int64_t n_meta, n_tensors;
    MetaKV *meta;
    TInfo *tensors;
    uint64_t data_start;
};

typedef struct {
    const uint8_t *p;
    size_t pos, size;
    int bad;
} Rd;

static int rd_need(Rd *r, size_t n) {
    if (r->bad || r->pos + n > r->size || r->pos + n < r->pos) {
        r->bad = 1;
        return 0;
    }
    return 1;
}
#define RD_SCALAR(name, T)                                                                        \
    static T name(Rd *r) {                                                                        \
        T v = 0;                                                                                  \
        if (rd_need(r, sizeof(T))) memcpy(&v, r->p + r->pos, sizeof(T)), r->pos += sizeof(T);     \
        return v;                                                                                 \
    }
RD_SCALAR(rd_u8, uint8_t)
RD_SCALAR(rd_u16, uint16_t)
RD_SCALAR(rd_u32, uint32_t)
RD_SCALAR(rd_u64, uint64_t)
RD_SCALAR(rd_f32, float)
RD_SCALAR(rd_f64, double)

static char *rd_str(Rd *r) {
    uint64_t len = rd_u64(r);
    if (!rd_need(r, (size_t)len)) return NULL;
    char *s = (char *)malloc((size_t)len + 1);
    if (!s) {
        r->bad = 1;
        return NULL;
    }
    memcpy(s, r->p + r->pos, (size_t)len);
    s[len] = 0;
    r->pos += (size_t)len;
    return s;
}

/* Shortest round-trip rendering of an f32 like Rust's Display (used only for
 * metadata text; numeric getters use the stored value). */
static void render_f32(float v, char *buf, size_t cap) {
    for (int prec = 1; prec <= 9; ++prec) {
        snprintf(buf, cap, "%.*g", prec, (double)v);
        if (strtof(buf, NULL) == v) return;
    }
}

static int skip_value(Rd *r, uint32_t type, int depth) {
    switch (type) {
    case 0: case 1: case 7: rd_u8(r); break;
    case 2: case 3: rd_u16(r); break;
    case 4: case 5: case 6: rd_u32(r); break;
    case 10: case 11: case 12: rd_u64(r); break;
    case 8: free(rd_str(r)); break;
    case 9: {
        if (depth > 4) return fail("GGUF array nesting too deep");
        uint32_t et = rd_u32(r);
        uint64_t len = rd_u64(r);
        for (uint64_t i = 0; i < len && !r->bad; ++i)
            if (skip_value(r, et, depth + 1)) return -1;
        break;
    }
    default: return fail("unknown type %u", type);
    }
    return r->bad ? fail("GGUF truncated") : 0;
}

static int read_value(Rd *r, MetaKV *kv) {
    char buf[64];
    kv->type = rd_u32(r);
    switch (kv->type) {
    case 0: kv->u = rd_u8(r); kv->i = (int64_t)kv->u; snprintf(buf, sizeof buf, "%llu", (unsigned long long)kv->u); break;
    case 1: kv->i = (int8_t)rd_u8(r); kv->u = (uint64_t)kv->i; snprintf(buf, sizeof buf, "%lld", (long long)kv->i); break;
    case 2: kv->u = rd_u16(r); kv->i = (int64_t)kv->u; snprintf(buf, sizeof buf, "%llu", (unsigned long long)kv->u); break;
    case 3: kv->i = (int16_t)rd_u16(r); kv->u = (uint64_t)kv->i; snprintf(buf, sizeof buf, "%lld", (long long)kv->i); break;
    case 4: kv->u = rd_u32(r); kv->i = (int64_t)kv->u; snprintf(buf, sizeof buf, "%llu", (unsigned long long)kv->u); break;
    case 5: kv->i = (int32_t)rd_u32(r); kv->u = (uint64_t)kv->i; snprintf(buf, sizeof buf, "%lld", (long long)kv->i); break;
    case 6: { float f = rd_f32(r); kv->f = f; render_f32(f, buf, sizeof buf); break; }
    case 7: kv->u = rd_u8(r) != 0; snprintf(buf, sizeof buf, "%s", kv->u ? "true" : "false"); break;
    case 8: kv->text = rd_str(r); return r->bad ? fail("GGUF truncated") : 0;
    case 10: kv->u = rd_u64(r); kv->i = (int64_t)kv->u; snprintf(buf, sizeof buf, "%llu", (unsigned long long)kv->u); break;
    case 11: kv->i = (int64_t)rd_u64(r); kv->u = (uint64_t)kv->i; snprintf(buf, sizeof buf, "%lld", (long long)kv->i); break;
    case 12: kv->f = rd_f64(r); snprintf(buf, sizeof buf, "%.17g", kv->f); break;
    case 9: {
        uint32_t et = rd_u32(r);
        uint64_t len = rd_u64(r);
        for (uint64_t i = 0; i < len && !r->bad; ++i)
            if (skip_value(r, et, 1)) return -1;
        snprintf(buf, sizeof buf, "[array len=%llu]", (unsigned long long)len);
        break;
    }
    default: return fail("unknown GGUF value type: %u", kv->type);
    }
    if (r->bad) return fail("GGUF truncated");
    kv->text = strdup(buf);
    return 0;
}

void s2o_gguf_close(S2oGguf *g) {
    if (!g) return;
    for (int64_t i = 0; i < g->n_meta; ++i) free(g->meta[i].key), free(g->meta[i].text);
    for (int64_t i = 0; i < g->n_tensors; ++i) free(g->tensors[i].name);
    free(g->meta);
    free(g->tensors);
    if (g->map && g->map != MAP_FAILED) munmap((void *)g->map, g->size);
    if (g->fd >= 0) close(g->fd);
    free(g);
}

/* gguf.rs:35-73 (+ validate_tensor_bounds 343-362, align_to 371-377) */
S2oGguf *s2o_gguf_open(const char *path) {
    S2oGguf *g = (S2oGguf *)calloc(1, sizeof *g);
    if (!g) return NULL;
    g->fd = open(path, O_RDONLY);
    if (g->fd < 0) {
        fail("IO: %s: %s", path, strerror(errno));
        goto bad;
    }
    struct stat st;
    if (fstat(g->fd, &st)) {
        fail("IO: %s", strerror(errno));
        goto bad;
    }
    g->size = (size_t)st.st_size;
    if (g->size < 4) {
        fail("not a GGUF file: %s", path);
        goto bad;
    }
    g->map = (const uint8_t *)mmap(NULL, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (g->map == MAP_FAILED) {
        fail("IO: mmap %s: %s", path, strerror(errno));
        goto bad;
    }
    Rd r = {g->map, 0, g->size, 0};
    if (memcmp(g->map, "GGUF", 4) != 0) {
        fail("not a GGUF file: %s", path);
        goto bad;
    }
    r.pos = 4;
    g->version = rd_u32(&r);
    uint64_t nt = rd_u64(&r), nm = rd_u64(&r);
    if (r.bad || nt > (1u << 24) || nm > (1u << 24)) {
        fail("GGUF header truncated or implausible");
        goto bad;
    }
    g->meta = (MetaKV *)calloc(nm ? nm : 1, sizeof(MetaKV));
    g->tensors = (TInfo *)calloc(nt ? nt : 1, sizeof(TInfo));
    if (!g->meta || !g->tensors) {
        fail("out of memory");
        goto bad;
    }
    for (uint64_t i = 0; i < nm; ++i) {
        g->n_meta = (int64_t)i + 1;
        g->meta[i].key = rd_str(&r);
        if (!g->meta[i].key || read_value(&r, &g->meta[i])) {
            if (!g_err[0] || r.bad) fail("GGUF metadata truncated");
            goto bad;
        }
    }
    for (uint64_t i = 0; i < nt; ++i) {
        TInfo *t = &g->tensors[i];
        g->n_tensors = (int64_t)i + 1;
        t->name = rd_str(&r);
        uint32_t rank = rd_u32(&r);
        if (r.bad || !t->name || rank > 4) {
            fail("GGUF tensor info truncated or rank > 4");
            goto bad;
        }
        t->rank = (int32_t)rank;
        uint64_t count = 1;
        for (uint32_t k = 0; k < rank; ++k) {
            t->dims[k] = rd_u64(&r);
            if (t->dims[k] && count > UINT64_MAX / t->dims[k]) {
                fail("tensor element count overflow: %s", t->name);
                goto bad;
            }
            count *= t->dims[k];
        }
        t->type = rd_u32(&r);
        t->rel = rd_u64(&r);
        int64_t bl = s2o_ggml_byte_len(t->type, (int64_t)count);
        if (bl < 0) {
            fail("unknown GGML tensor type: %u", t->type);
            goto bad;
        }
        t->bytes = (uint64_t)bl;
    }
    if (r.bad) {
        fail("GGUF truncated");
        goto bad;
    }
    g->data_start = (r.pos + 31) / 32 * 32;
    for (int64_t i = 0; i < g->n_tensors; ++i) {
        TInfo *t = &g->tensors[i];
        uint64_t start = g->data_start + t->rel, end = start + t->bytes;
        if (end < start || end > g->size) {
            fail("tensor %s extends past file end: %llu > %llu", t->name, (unsigned long long)end,
                 (unsigned long long)g->size);
            goto bad;
        }
    }
    return g;
bad:
    s2o_gguf_close(g);
    return NULL;
}

int64_t s2o_gguf_tensor_count(const S2oGguf *g) { return g->n_tensors; }
uint32_t s2o_gguf_version(const S2oGguf *g) { return g->version; }
uint64_t s2o_gguf_data_start(const S2oGguf *g) { return g->data_start; }

int s2o_gguf_tensor_info(const S2oGguf *g, int64_t i, const char **name, int32_t *rank,
                         uint64_t *dims, uint32_t *type, uint64_t *rel, uint64_t *bytes) {
    if (i < 0 || i >= g->n_tensors) return fail("tensor index out of range");
    const TInfo *t = &g->tensors[i];
    if (name) *name = t->name;
    if (rank) *rank = t->rank;
    if (dims) memcpy(dims, t->dims, sizeof t->dims);
    if (type) *type = t->type;
    if (rel) *rel = t->rel;
    if (bytes) *bytes = t->bytes;
    return 0;
}

/* gguf.rs:75-77: linear scan, first match. */
static const TInfo *find_tensor(const S2oGguf *g, const char *name) {
    for (int64_t i = 0; i < g->n_tensors; ++i)
        if (strcmp(g->tensors[i].name, name) == 0) return &g->tensors[i];
    return NULL;
}

const void *s2o_gguf_tensor_data(const S2oGguf *g, const char *name, uint64_t *byte_len) {
    const TInfo *t = find_tensor(g, name);
    if (!t) {
        fail("tensor not found: %s", name);
        return NULL;
    }
    if (byte_len) *byte_len = t->bytes;
    return g->map + g->data_start + t->rel;
}

static const MetaKV *find_meta(const S2oGguf *g, const char *key) {
    for (int64_t i = 0; i < g->n_meta; ++i)
        if (strcmp(g->meta[i].key, key) == 0) return &g->meta[i];
    return NULL;
}

int s2o_gguf_metadata(const S2oGguf *g, const char *key, char *buf, size_t cap) {
    const MetaKV *kv = find_meta(g, key);
    if (!kv) return fail("missing %s", key);
    snprintf(buf, cap, "%s", kv->text ? kv->text : "");
    return 0;
}

/* registry.rs:663-683: the reference parses the rendered text. */
static int meta_u32(const S2oGguf *g, const char *key, int32_t *out) {
    const MetaKV *kv = find_meta(g, key);
    if (!kv) return fail("missing %s", key);
    char *end = NULL;
    errno = 0;
    unsigned long long v = strtoull(kv->text, &end, 10);
    if (errno || !end || *end || kv->text[0] == '-' || kv->text[0] == 0 || v > 0xffffffffull)
        return fail("invalid u32 metadata %s: %s", key, kv->text);
    *out = (int32_t)(uint32_t)v;
    return 0;
}

static int meta_f32(const S2oGguf *g, const char *key, float *out) {
    const MetaKV *kv = find_meta(g, key);
    if (!kv) return fail("missing %s", key);
    if (kv->type == 6) {
        *out = (float)kv->f;
        return 0;
    }
    char *end = NULL;
    float v = strtof(kv->text, &end);
    if (!end || *end || kv->text[0] == 0) return fail("invalid f32 metadata %s: %s", key, kv->text);
    *out = v;
    return 0;
}

static int meta_bool(const S2oGguf *g, const char *key, int32_t *out) {
    const MetaKV *kv = find_meta(g, key);
    if (!kv) return fail("missing %s", key);
    if (strcmp(kv->text, "true") == 0) *out = 1;
    else if (strcmp(kv->text, "false") == 0) *out = 0;
    else return fail("invalid bool metadata %s: %s", key, kv->text);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* model                                                                      */
/* ------------------------------------------------------------------------- */

typedef struct {
    LWeights w;
    float *norms; /* attn_norm | q_norm | k_norm | ffn_norm, expanded f32 */
} LayerStore;

struct S2oModel {
    S2oGguf *g;
    S2oGraphSpec spec;
    LShape slow, fast;
    LayerStore *slow_layers, *fast_layers;
    const uint16_t *emb, *cb_emb, *fast_emb;
    WView fast_out;
    float *norm, *fast_norm;
    float *kslow, *vslow; /* [layer][max_seq][Hkv*hd] */
    int64_t max_seq, n_past;
    int mode;
    /* faithful mode: one layer's weights re-expanded to f32 per step */
    float *fx_wqkv, *fx_wo, *fx_w1, *fx_w2, *fx_w3;
    /* faithful mode: Fast-AR weights expanded once at load (fast_ar.rs:202-213) */
    float **fast_f32;
};

static int expand_norm(const S2oGguf *g, const char *name, int64_t n, float *dst) {
    uint64_t bl = 0;
    const void *p = s2o_gguf_tensor_data(g, name, &bl);
    if (!p) return -1;
    for (uint32_t i = 0; i < (uint32_t)g->n_tensors; ++i)
        if (strcmp(g->tensors[i].name, name) == 0) {
            const TInfo *t = &g->tensors[i];
            if (t->rank != 1 || (int64_t)t->dims[0] != n)
                return fail("%s dimensions mismatch: expected [%lld]", name, (long long)n);
            if (t->type == GGML_F32) memcpy(dst, p, (size_t)n * 4);
            else if (t->type == GGML_F16) s2o_dequant_row(GGML_F16, p, n, dst);
            else return fail("expected F16 tensor %s, got type %u", name, t->type);
            return 0;
        }
    return fail("tensor not found: %s", name);
}

static int bind_matrix(const S2oGguf *g, const char *name, int64_t in, int64_t out, WView *w) {
    const TInfo *t = find_tensor(g, name);
    if (!t) return fail("missing %s", name);
    if (t->rank != 2 || (int64_t)t->dims[0] != in || (int64_t)t->dims[1] != out)
        return fail("%s dimensions mismatch: expected [%lld, %lld], got [%llu, %llu]", name,
                    (long long)in, (long long)out, (unsigned long long)t->dims[0],
                    (unsigned long long)(t->rank > 1 ? t->dims[1] : 0));
    if (t->type != GGML_F16 && t->type != GGML_Q8_0 && t->type != GGML_Q4_K && t->type != GGML_F32)
        return fail("unsupported tensor type %u for %s", t->type, name);
    w->p = g->map + g->data_start + t->rel;
    w->type = t->type;
    w->in_dim = in;
    w->out_dim = out;
    return 0;
}

static int bind_layer(S2oModel *m, const char *prefix, int64_t layer, const LShape *s, int slow,
                      LayerStore *L) {
    char name[256];
    const int64_t d = s->d, qs = s->H * s->hd, kvs = s->Hkv * s->hd, F = s->F;
    L->norms = (float *)calloc((size_t)(2 * d + 2 * s->hd), sizeof(float));
    if (!L->norms) return fail("out of memory");
    float *an = L->norms, *fn = an + d, *qn = fn + d, *kn = qn + s->hd;
#define NM(fmt) (snprintf(name, sizeof name, "%s.%lld." fmt, prefix, (long long)layer), name)
    if (expand_norm(m->g, NM("attention_norm.weight"), d, an)) return -1;
    if (expand_norm(m->g, NM("ffn_norm.weight"), d, fn)) return -1;
    if (slow) {
        if (expand_norm(m->g, NM("attention.q_norm.weight"), s->hd, qn)) return -1;
        if (expand_norm(m->g, NM("attention.k_norm.weight"), s->hd, kn)) return -1;
    }
    if (bind_matrix(m->g, NM("attention.wqkv.weight"), d, qs + 2 * kvs, &L->w.wqkv)) return -1;
    if (bind_matrix(m->g, NM("attention.wo.weight"), qs, d, &L->w.wo)) return -1;
    if (bind_matrix(m->g, NM("feed_forward.w1.weight"), d, F, &L->w.w1)) return -1;
    if (bind_matrix(m->g, NM("feed_forward.w2.weight"), F, d, &L->w.w2)) return -1;
    if (bind_matrix(m->g, NM("feed_forward.w3.weight"), d, F, &L->w.w3)) return -1;
#undef NM
    L->w.attn_norm = an, L->w.ffn_norm = fn, L->w.q_norm = qn, L->w.k_norm = kn;
    return 0;
}

static const uint16_t *bind_f16_table(S2oModel *m, const char *name, int64_t d, int64_t *rows) {
    const TInfo *t = find_tensor(m->g, name);
    if (!t) {
        fail("tensor not found: %s", name);
        return NULL;
    }
    if (t->type != GGML_F16) {
        fail("expected F16 tensor %s, got type %u", name, t->type);
        return NULL;
    }
    if (t->rank != 2 || (int64_t)t->dims[0] != d) {
        fail("%s expected [%lld, rows]", name, (long long)d);
        return NULL;
    }
    *rows = (int64_t)t->dims[1];
    return (const uint16_t *)(m->g->map + m->g->data_start + t->rel);
}

void s2o_close(S2oModel *m) {
    if (!m) return;
    if (m->slow_layers)
        for (int i = 0; i < m->spec.slow_block_count; ++i) free(m->slow_layers[i].norms);
    if (m->fast_layers)
        for (int i = 0; i < m->spec.fast_block_count; ++i) free(m->fast_layers[i].norms);
    if (m->fast_f32) {
        for (int i = 0; i < 5 * m->spec.fast_block_count + 1; ++i) free(m->fast_f32[i]);
        free(m->fast_f32);
    }
    free(m->slow_layers), free(m->fast_layers), free(m->norm), free(m->fast_norm);
    free(m->kslow), free(m->vslow);
    free(m->fx_wqkv), free(m->fx_wo), free(m->fx_w1), free(m->fx_w2), free(m->fx_w3);
    s2o_gguf_close(m->g);
    free(m);
}

static float *expand_view(const WView *w) {
    float *dst = (float *)malloc(sizeof(float) * (size_t)(w->in_dim * w->out_dim));
    if (!dst) return NULL;
    f16_lut_init();
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < w->out_dim; ++o) wrows_f32(w, o, 1, dst + o * w->in_dim);
    return dst;
}

/* SlowArState::open (slow_ar.rs:387-412) + DualArGraphSpec::from_gguf
 * (registry.rs:45-103) with shape-parametric hparams: the slow head_dim is
 * the q_norm length instead of the QK_NORM_SIZE constant (registry.rs:46-52),
 * and the hard-coded S2-Pro shape checks (registry.rs:109-213) are replaced by
 * consistency checks between metadata and tensor shapes. */
S2oModel *s2o_open(const char *path, int64_t max_seq_len, int mode) {
    if (max_seq_len <= 0) {
        fail("max_seq_len must be non-zero");
        return NULL;
    }
    S2oModel *m = (S2oModel *)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->mode = mode;
    m->max_seq = max_seq_len;
    m->g = s2o_gguf_open(path);
    if (!m->g) goto bad;
    char arch[64];
    if (s2o_gguf_metadata(m->g, "general.architecture", arch, sizeof arch)) {
        fail("missing general.architecture");
        goto bad;
    }
    if (strcmp(arch, "fish-speech") != 0) {
        fail("expected fish-speech transformer GGUF, got %s", arch);
        goto bad;
    }
    S2oGraphSpec *s = &m->spec;
    int rc = 0;
    rc |= meta_bool(m->g, "fish_speech.attention_qk_norm", &s->slow_attention_qk_norm);
    rc |= meta_u32(m->g, "fish-speech.context_length", &s->slow_context_length);
    rc |= meta_u32(m->g, "fish-speech.embedding_length", &s->slow_embedding_length);
    rc |= meta_u32(m->g, "fish-speech.feed_forward_length", &s->slow_feed_forward_length);
    rc |= meta_u32(m->g, "fish-speech.block_count", &s->slow_block_count);
    rc |= meta_u32(m->g, "fish-speech.attention.head_count", &s->slow_head_count);
    rc |= meta_u32(m->g, "fish-speech.attention.head_count_kv", &s->slow_head_count_kv);
    rc |= meta_f32(m->g, "fish-speech.rope.freq_base", &s->slow_rope_freq_base);
    rc |= meta_f32(m->g, "fish-speech.attention.layer_norm_rms_epsilon", &s->slow_rms_norm_eps);
    rc |= meta_u32(m->g, "fish_speech.fast_context_length", &s->fast_context_length);
    rc |= meta_u32(m->g, "fish_speech.fast_embedding_length", &s->fast_embedding_length);
    rc |= meta_u32(m->g, "fish_speech.fast_feed_forward_length", &s->fast_feed_forward_length);
    rc |= meta_u32(m->g, "fish_speech.fast_block_count", &s->fast_block_count);
    rc |= meta_u32(m->g, "fish_speech.fast_head_count", &s->fast_head_count);
    rc |= meta_u32(m->g, "fish_speech.fast_head_count_kv", &s->fast_head_count_kv);
    rc |= meta_u32(m->g, "fish_speech.fast_head_dim", &s->fast_head_dim);
    rc |= meta_f32(m->g, "fish_speech.fast_rope_freq_base", &s->fast_rope_freq_base);
    rc |= meta_f32(m->g, "fish_speech.fast_layer_norm_rms_eps", &s->fast_rms_norm_eps);
    rc |= meta_bool(m->g, "fish_speech.fast_attention_qk_norm", &s->fast_attention_qk_norm);
    rc |= meta_u32(m->g, "fish_speech.codebook_size", &s->codebook_size);
    rc |= meta_u32(m->g, "fish_speech.num_codebooks", &s->num_codebooks);
    rc |= meta_u32(m->g, "fish_speech.semantic_begin_id", &s->semantic_begin_id);
    rc |= meta_u32(m->g, "fish_speech.semantic_end_id", &s->semantic_end_id);
    rc |= meta_bool(m->g, "fish_speech.scale_codebook_embeddings", &s->scale_codebook_embeddings);
    rc |= meta_bool(m->g, "fish_speech.tie_word_embeddings", &s->tie_word_embeddings);
    rc |= meta_bool(m->g, "fish_speech.fast_project_in", &s->fast_project_in);
    if (rc) goto bad;
    if (s->fast_project_in) {
        /* fast_ar.rs:366-370 */
        fail("fast_project_in is not implemented in pure Rust yet");
        goto bad;
    }
    if (s->slow_head_count_kv == 0 || s->slow_head_count % s->slow_head_count_kv ||
        s->fast_head_count_kv == 0 || s->fast_head_count % s->fast_head_count_kv) {
        fail("invalid GQA head split");
        goto bad;
    }
    if (s->fast_embedding_length != s->slow_embedding_length) {
        /* fast_ar.rs:380-387: the slow hidden is fed to the Fast-AR as-is */
        fail("slow hidden size mismatch: fast embedding_length %d != slow %d",
             s->fast_embedding_length, s->slow_embedding_length);
        goto bad;
    }
    const int64_t d = s->slow_embedding_length;
    /* slow head_dim: q_norm length when QK-norm is on, else d / heads */
    if (s->slow_attention_qk_norm) {
        const TInfo *qn = find_tensor(m->g, "layers.0.attention.q_norm.weight");
        if (!qn || qn->rank != 1) {
            fail("missing layers.0.attention.q_norm.weight");
            goto bad;
        }
        s->slow_head_dim = (int32_t)qn->dims[0];
    } else {
        s->slow_head_dim = (int32_t)(d / s->slow_head_count);
    }
    m->slow = (LShape){d, s->slow_feed_forward_length, s->slow_head_count, s->slow_head_count_kv,
                       s->slow_head_dim, s->slow_rope_freq_base, s->slow_rms_norm_eps,
                       s->slow_attention_qk_norm, 0};
    m->fast = (LShape){d, s->fast_feed_forward_length, s->fast_head_count, s->fast_head_count_kv,
                       s->fast_head_dim, s->fast_rope_freq_base, s->fast_rms_norm_eps, 0, 1};
    m->emb = bind_f16_table(m, "embeddings.weight", d, &s->vocab_size);
    m->cb_emb = bind_f16_table(m, "codebook_embeddings.weight", d, &s->codebook_rows);
    m->fast_emb = bind_f16_table(m, "fast_embeddings.weight", d, &s->fast_vocab_size);
    if (!m->emb || !m->cb_emb || !m->fast_emb) goto bad;
    if (bind_matrix(m->g, "fast_output.weight", d, s->codebook_size, &m->fast_out)) goto bad;
    m->norm = (float *)malloc(sizeof(float) * (size_t)d);
    m->fast_norm = (float *)malloc(sizeof(float) * (size_t)d);
    if (!m->norm || !m->fast_norm) goto bad;
    if (expand_norm(m->g, "norm.weight", d, m->norm)) goto bad;
    if (expand_norm(m->g, "fast_norm.weight", d, m->fast_norm)) goto bad;
    m->slow_layers = (LayerStore *)calloc((size_t)s->slow_block_count, sizeof(LayerStore));
    m->fast_layers = (LayerStore *)calloc((size_t)s->fast_block_count, sizeof(LayerStore));
    if (!m->slow_layers || !m->fast_layers) goto bad;
    for (int l = 0; l < s->slow_block_count; ++l)
        if (bind_layer(m, "layers", l, &m->slow, 1, &m->slow_layers[l])) goto bad;
    for (int l = 0; l < s->fast_block_count; ++l)
        if (bind_layer(m, "fast_layers", l, &m->fast, 0, &m->fast_layers[l])) goto bad;
    const int64_t kvs = (int64_t)s->slow_head_count_kv * s->slow_head_dim;
    size_t kvlen = (size_t)(kvs * max_seq_len * s->slow_block_count);
    m->kslow = (float *)calloc(kvlen, sizeof(float));
    m->vslow = (float *)calloc(kvlen, sizeof(float));
    if (!m->kslow || !m->vslow) {
        fail("KV cache allocation failed");
        goto bad;
    }
    if (mode == 1) {
        const LWeights *w0 = &m->slow_layers[0].w;
        m->fx_wqkv = (float *)malloc(sizeof(float) * (size_t)(w0->wqkv.in_dim * w0->wqkv.out_dim));
        m->fx_wo = (float *)malloc(sizeof(float) * (size_t)(w0->wo.in_dim * w0->wo.out_dim));
        m->fx_w1 = (float *)malloc(sizeof(float) * (size_t)(w0->w1.in_dim * w0->w1.out_dim));
        m->fx_w2 = (float *)malloc(sizeof(float) * (size_t)(w0->w2.in_dim * w0->w2.out_dim));
        m->fx_w3 = (float *)malloc(sizeof(float) * (size_t)(w0->w3.in_dim * w0->w3.out_dim));
        if (!m->fx_wqkv || !m->fx_wo || !m->fx_w1 || !m->fx_w2 || !m->fx_w3) {
            fail("out of memory (faithful mode buffers)");
            goto bad;
        }
        m->fast_f32 = (float **)calloc((size_t)(5 * s->fast_block_count + 1), sizeof(float *));
        if (!m->fast_f32) goto bad;
        for (int l = 0; l < s->fast_block_count; ++l) {
            LWeights *w = &m->fast_layers[l].w;
            WView *vs[5] = {&w->wqkv, &w->wo, &w->w1, &w->w2, &w->w3};
            for (int k = 0; k < 5; ++k) {
                float *e = expand_view(vs[k]);
                if (!e) {
                    fail("out of memory (fast f32 weights)");
                    goto bad;
                }
                m->fast_f32[5 * l + k] = e;
                vs[k]->p = e;
                vs[k]->type = GGML_F32;
            }
        }
        float *fo = expand_view(&m->fast_out);
        if (!fo) goto bad;
        m->fast_f32[5 * s->fast_block_count] = fo;
        m->fast_out.p = fo;
        m->fast_out.type = GGML_F32;
    }
    return m;
bad:
    s2o_close(m);
    return NULL;
}

int s2o_graph_spec(const S2oModel *m, S2oGraphSpec *out) {
    *out = m->spec;
    return 0;
}

/* slow_ar.rs:434-438 */
void s2o_reset(S2oModel *m) {
    m->n_past = 0;
    const int64_t kvs = (int64_t)m->spec.slow_head_count_kv * m->spec.slow_head_dim;
    size_t kvlen = (size_t)(kvs * m->max_seq * m->spec.slow_block_count);
    memset(m->kslow, 0, kvlen * sizeof(float));
    memset(m->vslow, 0, kvlen * sizeof(float));
}

int64_t s2o_n_past(const S2oModel *m) { return m->n_past; }

/* embed_slow_ar_time_major (slow_ar.rs:1041-1133) + embedding_lookup_rows
 * (tensor.rs:161-193). */
static int embed_tokens(const S2oModel *m, const int32_t *flat, int64_t n_tokens, float *X) {
    const S2oGraphSpec *s = &m->spec;
    const int64_t d = s->slow_embedding_length, K = s->num_codebooks, cd = K + 1;
    const float sem_scale = s->scale_codebook_embeddings ? 1.0f / sqrtf((float)cd) : 1.0f;
    float *cbsum = (float *)malloc(sizeof(float) * (size_t)d);
    if (!cbsum) return fail("out of memory");
    for (int64_t t = 0; t < n_tokens; ++t) {
        const int32_t *tok = flat + t * cd;
        float *h = X + t * d;
        if (tok[0] < 0) {
            free(cbsum);
            return fail("semantic token id must be non-negative, got %d", tok[0]);
        }
        uint32_t id = (uint32_t)tok[0];
        int is_sem = id >= (uint32_t)s->semantic_begin_id && id <= (uint32_t)s->semantic_end_id;
        if ((int64_t)id >= s->vocab_size) {
            free(cbsum);
            return fail("embedding index %u out of range for vocab_dim %lld", id,
                        (long long)s->vocab_size);
        }
        for (int64_t i = 0; i < d; ++i) h[i] = g_f16_lut[m->emb[(int64_t)id * d + i]];
        if (is_sem) {
            for (int64_t i = 0; i < d; ++i) cbsum[i] = 0.0f;
            for (int64_t cb = 0; cb < K; ++cb) {
                int32_t raw = tok[1 + cb];
                if (raw < 0) {
                    free(cbsum);
                    return fail("codebook token must be non-negative, got %d", raw);
                }
                uint64_t cid = (uint64_t)raw + (uint64_t)cb * (uint64_t)s->codebook_size;
                if ((int64_t)cid >= s->codebook_rows) {
                    free(cbsum);
                    return fail("embedding index %llu out of range for vocab_dim %lld",
                                (unsigned long long)cid, (long long)s->codebook_rows);
                }
                const uint16_t *row = m->cb_emb + (int64_t)cid * d;
                for (int64_t i = 0; i < d; ++i) cbsum[i] += g_f16_lut[row[i]];
            }
            for (int64_t i = 0; i < d; ++i) h[i] += cbsum[i];
        }
        if (s->scale_codebook_embeddings) {
            float sc = is_sem ? sem_scale : 1.0f;
            for (int64_t i = 0; i < d; ++i) h[i] *= sc;
        }
    }
    free(cbsum);
    return 0;
}

/* Bind the f32 re-expansion of one Slow-AR layer (faithful mode only):
 * SlowArLayerF16Weights::from_gguf_layer runs per layer per step
 * (slow_ar.rs:1189, 111-133). */
static void faithful_expand(S2oModel *m, const LWeights *src, LWeights *dst) {
    *dst = *src;
    struct {
        const WView *s;
        WView *d;
        float *buf;
    } jobs[5] = {{&src->wqkv, &dst->wqkv, m->fx_wqkv}, {&src->wo, &dst->wo, m->fx_wo},
                 {&src->w1, &dst->w1, m->fx_w1}, {&src->w2, &dst->w2, m->fx_w2},
                 {&src->w3, &dst->w3, m->fx_w3}};
    for (int k = 0; k < 5; ++k) {
        const WView *s = jobs[k].s;
#pragma omp parallel for schedule(static)
        for (int64_t o = 0; o < s->out_dim; ++o) wrows_f32(s, o, 1, jobs[k].buf + o * s->in_dim);
        jobs[k].d->p = jobs[k].buf;
        jobs[k].d->type = GGML_F32;
    }
}

/* SlowArState::eval (slow_ar.rs:456-527) */
int s2o_eval(S2oModel *m, const int32_t *flat, int64_t n_flat, float *hidden_out,
             float *logits_out, int allowed_only, int64_t im_end_id) {
    const S2oGraphSpec *s = &m->spec;
    const int64_t cd = s->num_codebooks + 1, d = s->slow_embedding_length;
    f16_lut_init();
    if (n_flat % cd)
        return fail("flat token length %lld is not a multiple of codebook_dim %lld",
                    (long long)n_flat, (long long)cd);
    const int64_t n = n_flat / cd;
    if (n == 0) return fail("expected at least one token");
    if (m->n_past + n > m->max_seq)
        return fail("KV cache overflow: n_past=%lld n_tokens=%lld max_seq_len=%lld",
                    (long long)m->n_past, (long long)n, (long long)m->max_seq);
    float *X = (float *)malloc(sizeof(float) * (size_t)(n * d));
    if (!X) return fail("out of memory");
    int rc = embed_tokens(m, flat, n, X);
    const int64_t kvs = (int64_t)s->slow_head_count_kv * s->slow_head_dim;
    for (int l = 0; !rc && l < s->slow_block_count; ++l) {
        LWeights w = m->slow_layers[l].w;
        if (m->mode == 1) faithful_expand(m, &m->slow_layers[l].w, &w);
        rc = layer_forward(&m->slow, &w, X, n, m->kslow + kvs * m->max_seq * l,
                           m->vslow + kvs * m->max_seq * l, m->n_past, NULL);
    }
    if (!rc) {
        /* forward_logits (slow_ar.rs:943-955): post-norm hidden of the last
         * token, tied LM head over embeddings.weight rows. */
        float *h = X + (n - 1) * d;
        float *nh = (float *)malloc(sizeof(float) * (size_t)d);
        if (!nh) rc = fail("out of memory");
        else {
            rms_norm_f32(h, m->norm, d, s->slow_rms_norm_eps, nh);
            if (hidden_out) memcpy(hidden_out, nh, sizeof(float) * (size_t)d);
            if (logits_out) {
                if (!allowed_only) {
                    s2o_matvec_f16(nh, m->emb, d, s->vocab_size, logits_out);
                } else {
                    for (int64_t i = 0; i < s->vocab_size; ++i) logits_out[i] = -INFINITY;
                    int64_t b = s->semantic_begin_id, e = s->semantic_end_id;
                    if (e >= s->vocab_size) e = s->vocab_size - 1;
                    if (b <= e) s2o_matvec_f16(nh, m->emb + b * d, d, e - b + 1, logits_out + b);
                    if (im_end_id >= 0 && im_end_id < s->vocab_size)
                        s2o_matvec_f16(nh, m->emb + im_end_id * d, d, 1, logits_out + im_end_id);
                }
            }
            free(nh);
            m->n_past += n;
        }
    }
    free(X);
    return rc;
}

/* Fast-AR over a sequence [slow_hidden, fast_emb[prefix...]]: the last
 * token's logits.  `faithful`: forward_codebook_prefix recomputes every
 * prefix position in every layer (fast_ar.rs:245-292, 360-437).  Otherwise the
 * caller's per-frame KV (fk/fv: [layer][pos][Hkv*hd]) and per-layer hidden
 * tokens are extended by the new positions only; causality makes the two
 * bit-identical. */
typedef struct {
    float *fk, *fv;   /* [L][ctx][kvs] */
    int64_t len;      /* positions already processed */
    int64_t ctx;
} FastKv;

static int fast_run(S2oModel *m, FastKv *kv, const float *new_tokens, int64_t n_new,
                    float *logits) {
    const S2oGraphSpec *s = &m->spec;
    const int64_t d = s->fast_embedding_length;
    const int64_t kvs = (int64_t)s->fast_head_count_kv * s->fast_head_dim;
    if (kv->len + n_new > kv->ctx)
        return fail("fast sequence length %lld exceeds context_length %lld",
                    (long long)(kv->len + n_new), (long long)kv->ctx);
    float *X = (float *)malloc(sizeof(float) * (size_t)(n_new * d));
    if (!X) return fail("out of memory");
    memcpy(X, new_tokens, sizeof(float) * (size_t)(n_new * d));
    int rc = 0;
    for (int l = 0; !rc && l < s->fast_block_count; ++l)
        rc = layer_forward(&m->fast, &m->fast_layers[l].w, X, n_new, kv->fk + l * kv->ctx * kvs,
                           kv->fv + l * kv->ctx * kvs, kv->len, NULL);
    if (!rc) {
        kv->len += n_new;
        float *nh = (float *)malloc(sizeof(float) * (size_t)d);
        if (!nh) rc = fail("out of memory");
        else {
            rms_norm_f32(X + (n_new - 1) * d, m->fast_norm, d, s->fast_rms_norm_eps, nh);
            rc = linear_multi(&m->fast_out, nh, 1, logits, -0.0f);
            free(nh);
        }
    }
    free(X);
    return rc;
}

static int fast_kv_init(S2oModel *m, FastKv *kv) {
    const S2oGraphSpec *s = &m->spec;
    const int64_t kvs = (int64_t)s->fast_head_count_kv * s->fast_head_dim;
    kv->ctx = s->fast_context_length;
    kv->len = 0;
    kv->fk = (float *)calloc((size_t)(s->fast_block_count * kv->ctx * kvs), sizeof(float));
    kv->fv = (float *)calloc((size_t)(s->fast_block_count * kv->ctx * kvs), sizeof(float));
    if (!kv->fk || !kv->fv) {
        free(kv->fk), free(kv->fv);
        return fail("out of memory");
    }
    return 0;
}

static void fast_kv_free(FastKv *kv) { free(kv->fk), free(kv->fv); }

/* Build [slow_hidden, fast_emb rows of codes] (fast_ar.rs:393-403). */
static int fast_sequence(const S2oModel *m, const float *slow_hidden, const uint32_t *prefix,
                         int64_t n_prefix, float *seq) {
    const S2oGraphSpec *s = &m->spec;
    const int64_t d = s->fast_embedding_length;
    memcpy(seq, slow_hidden, sizeof(float) * (size_t)d);
    for (int64_t i = 0; i < n_prefix; ++i) {
        if ((int64_t)prefix[i] >= s->fast_vocab_size)
            return fail("embedding index %u out of range for vocab_dim %lld", prefix[i],
                        (long long)s->fast_vocab_size);
        const uint16_t *row = m->fast_emb + (int64_t)prefix[i] * d;
        for (int64_t k = 0; k < d; ++k) seq[(1 + i) * d + k] = g_f16_lut[row[k]];
    }
    return 0;
}

/* forward_codebook_prefix (fast_ar.rs:360-437) */
int s2o_fast_prefix_logits(S2oModel *m, const float *slow_hidden, const uint32_t *prefix,
                           int64_t n_prefix, float *logits_out) {
    const S2oGraphSpec *s = &m->spec;
    f16_lut_init();
    if (n_prefix >= s->num_codebooks)
        return fail("fast prefix too long: %lld codes (max %d)", (long long)n_prefix,
                    s->num_codebooks - 1);
    const int64_t d = s->fast_embedding_length;
    float *seq = (float *)malloc(sizeof(float) * (size_t)((n_prefix + 1) * d));
    if (!seq) return fail("out of memory");
    FastKv kv;
    int rc = fast_sequence(m, slow_hidden, prefix, n_prefix, seq);
    if (!rc) rc = fast_kv_init(m, &kv);
    if (!rc) {
        rc = fast_run(m, &kv, seq, n_prefix + 1, logits_out);
        fast_kv_free(&kv);
    }
    free(seq);
    return rc;
}

/* generate_codebooks_for_semantic (fast_ar.rs:440-470) */
int s2o_generate_codebooks(S2oModel *m, const float *slow_hidden, uint32_t semantic_code,
                           float temperature, float top_p, int32_t top_k, uint64_t *rng,
                           uint32_t *out) {
    const S2oGraphSpec *s = &m->spec;
    f16_lut_init();
    if (semantic_code >= (uint32_t)s->codebook_size)
        return fail("semantic_code %u >= codebook_size %d", semantic_code, s->codebook_size);
    const int64_t d = s->fast_embedding_length, K = s->num_codebooks, cb = s->codebook_size;
    float *seq = (float *)malloc(sizeof(float) * (size_t)(K * d));
    float *logits = (float *)malloc(sizeof(float) * (size_t)cb);
    uint32_t *prefix = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)K);
    FastKv kv = {0};
    int rc = (!seq || !logits || !prefix) ? fail("out of memory") : 0;
    if (!rc && m->mode != 1) rc = fast_kv_init(m, &kv);
    if (!rc) {
        prefix[0] = semantic_code;
        out[0] = semantic_code;
        for (int64_t k = 1; !rc && k < K; ++k) {
            if (m->mode == 1) {
                rc = s2o_fast_prefix_logits(m, slow_hidden, prefix, k, logits);
            } else {
                /* incremental: first call feeds [slow_hidden, emb(c0)], later
                 * calls feed the newest code only */
                rc = fast_sequence(m, slow_hidden, prefix, k, seq);
                if (!rc) {
                    int64_t first = kv.len;
                    rc = fast_run(m, &kv, seq + first * d, k + 1 - first, logits);
                }
            }
            uint32_t tok = 0;
            if (!rc) rc = s2o_sample_token(logits, cb, temperature, top_p, top_k, -1, rng, &tok);
            if (!rc && tok >= (uint32_t)cb)
                rc = fail("sampled codebook token %u >= codebook_size %lld", tok, (long long)cb);
            if (!rc) prefix[k] = tok, out[k] = tok;
        }
    }
    if (m->mode != 1 && kv.fk) fast_kv_free(&kv);
    free(seq), free(logits), free(prefix);
    return rc;
}

/* prompt.rs:77-103 */
int s2o_transpose_to_time_major(const uint32_t *data, int64_t rows, int64_t cols, int32_t *flat) {
    if (rows == 0) return fail("prompt rows must be non-zero");
    for (int64_t t = 0; t < cols; ++t)
        for (int64_t r = 0; r < rows; ++r) {
            uint32_t v = data[r * cols + t];
            if (v > 0x7fffffffu) return fail("prompt token id does not fit i32");
            flat[t * rows + r] = (int32_t)v;
        }
    return 0;
}

/* generate.rs:346-390 */
int s2o_compact_codes(int32_t *codes, uint32_t K, uint32_t max_new, uint32_t n_frames,
                      int64_t *out_len) {
    if (n_frames >= max_new) {
        *out_len = (int64_t)K * n_frames;
        return 0;
    }
    int32_t *tmp = (int32_t *)malloc(sizeof(int32_t) * ((size_t)K * n_frames + 1));
    if (!tmp) return fail("out of memory");
    for (uint32_t cb = 0; cb < K; ++cb)
        for (uint32_t t = 0; t < n_frames; ++t)
            tmp[(size_t)cb * n_frames + t] = codes[(size_t)cb * max_new + t];
    memcpy(codes, tmp, sizeof(int32_t) * (size_t)K * n_frames);
    free(tmp);
    *out_len = (int64_t)K * n_frames;
    return 0;
}

/* generate.rs:273-282 */
static uint32_t semantic_to_codebook_id(const S2oGraphSpec *s, uint32_t main) {
    if (main < (uint32_t)s->semantic_begin_id || main > (uint32_t)s->semantic_end_id) return 0;
    uint32_t code = main - (uint32_t)s->semantic_begin_id;
    if (code >= (uint32_t)s->codebook_size) return (uint32_t)s->codebook_size - 1;
    return code;
}

/* generate.rs:284-298 */
static int sample_semantic(const S2oModel *m, const float *step_logits, const float *bias,
                           uint32_t im_end, uint64_t generated_after_prefill,
                           const S2oGenParams *p, uint64_t *rng, float *scratch, uint32_t *out) {
    const int64_t V = m->spec.vocab_size;
    memcpy(scratch, step_logits, sizeof(float) * (size_t)V);
    int block = (uint32_t)generated_after_prefill < p->min_tokens_before_end;
    s2o_apply_semantic_bias(scratch, bias, V, block, im_end);
    return s2o_sample_token(scratch, V, p->temperature, p->top_p, p->top_k,
                            block ? -1 : (int64_t)im_end, rng, out);
}

/* generate_codes (generate.rs:117-221) */
int s2o_generate_codes(S2oModel *m, const uint32_t *prompt, int64_t rows, int64_t cols,
                       const S2oGenParams *p, uint64_t *rng, int32_t *out_codes,
                       uint32_t *out_n_frames, uint32_t *trace_main) {
    const S2oGraphSpec *s = &m->spec;
    const int64_t V = s->vocab_size, d = s->slow_embedding_length;
    const uint32_t K = s->num_codebooks > 1 ? (uint32_t)s->num_codebooks : 1u;
    const uint32_t max_new = p->max_new_tokens;
    int32_t *flat = (int32_t *)malloc(sizeof(int32_t) * (size_t)(rows * cols + 1));
    float *logits = (float *)malloc(sizeof(float) * (size_t)V);
    float *scratch = (float *)malloc(sizeof(float) * (size_t)V);
    float *bias = (float *)malloc(sizeof(float) * (size_t)V);
    float *hidden = (float *)malloc(sizeof(float) * (size_t)d);
    uint32_t *cbs = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(K + 1));
    int32_t *step_in = (int32_t *)malloc(sizeof(int32_t) * (size_t)(s->num_codebooks + 1));
    int rc = (!flat || !logits || !scratch || !bias || !hidden || !cbs || !step_in)
                 ? fail("out of memory")
                 : 0;
    const int allowed_only = m->mode != 1;
    if (!rc) rc = s2o_transpose_to_time_major(prompt, rows, cols, flat);
    if (!rc) {
        s2o_reset(m);
        rc = s2o_eval(m, flat, rows * cols, hidden, logits, allowed_only, p->im_end_id);
    }
    if (!rc) s2o_build_semantic_bias(V, (uint32_t)s->semantic_begin_id, (uint32_t)s->semantic_end_id,
                                     p->im_end_id, bias);
    memset(out_codes, 0, sizeof(int32_t) * (size_t)K * max_new);
    uint32_t main = 0, step_index = 0;
    if (!rc) rc = sample_semantic(m, logits, bias, p->im_end_id, 0, p, rng, scratch, &main);
    if (!rc && trace_main) trace_main[0] = main;
    while (!rc && main != p->im_end_id && step_index < max_new) {
        uint32_t sem_code = semantic_to_codebook_id(s, main);
        rc = s2o_generate_codebooks(m, hidden, sem_code, p->temperature, p->top_p, p->top_k, rng,
                                    cbs);
        if (rc) break;
        for (uint32_t cb = 0; cb < K && cb < (uint32_t)s->num_codebooks; ++cb)
            out_codes[(size_t)cb * max_new + step_index] = (int32_t)cbs[cb];
        /* build_step_input (generate.rs:300-344) */
        memset(step_in, 0, sizeof(int32_t) * (size_t)(s->num_codebooks + 1));
        step_in[0] = (int32_t)main;
        if (main >= (uint32_t)s->semantic_begin_id && main <= (uint32_t)s->semantic_end_id)
            for (int cb = 0; cb < s->num_codebooks; ++cb) step_in[1 + cb] = (int32_t)cbs[cb];
        rc = s2o_eval(m, step_in, s->num_codebooks + 1, hidden, logits, allowed_only, p->im_end_id);
        if (rc) break;
        step_index += 1;
        uint64_t gap = (uint64_t)(m->n_past - cols) + step_index;
        rc = sample_semantic(m, logits, bias, p->im_end_id, gap, p, rng, scratch, &main);
        if (!rc && trace_main) trace_main[step_index] = main;
    }
    if (!rc) {
        int64_t len = 0;
        rc = s2o_compact_codes(out_codes, K, max_new, step_index, &len);
        *out_n_frames = step_index;
    }
    free(flat), free(logits), free(scratch), free(bias), free(hidden), free(cbs), free(step_in);
    return rc;
}
