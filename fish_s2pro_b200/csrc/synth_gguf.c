/*
 * synth_gguf.c -- writes seeded synthetic fish-speech transformer GGUF files.
 *
 * No model weights are available offline, so every benchmark and parity run
 * uses a random-init model with the tensor names, shapes and metadata keys the
 * reference's loader reads (crates/fish_s2_infer/src/registry.rs:45-103,
 * 346-496, 625-650) in the GGUF v3 container it parses
 * (crates/fish_s2_core/src/gguf.rs:35-73, 32-byte data alignment at :371-377).
 *
 * Values come from a counter-based hash of (seed, tensor index, element
 * index), so a file is byte-identical whatever the thread count.
 *   linear weights and embeddings: approx. N(0, std) (Irwin-Hall sum of four
 *   uniforms, rescaled), rounded to f16 with the reference's f32->f16 rule
 *   (tensor.rs:289-325); norm gains: 1.0.
 *   Q8_0 linears: int8 uniform in [-127, 127], f16 scale ~U(1e-4, 4e-4).
 *   Q4_K linears: 4-bit quants uniform in 0..15, f16 d/dmin ~U(1e-4, 1e-3),
 *   6-bit sub-block scales/mins uniform (random packed bytes).
 */
#define _GNU_SOURCE
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct S2dSynthConfig {
    int32_t slow_layers, d, heads, kv_heads, head_dim, ffn;
    int32_t vocab, sem_begin, sem_end;
    int32_t fast_layers, fast_heads, fast_kv_heads, fast_head_dim, fast_ffn;
    int32_t num_codebooks, codebook_size;
    int32_t context_length, fast_context_length;
    int32_t linear_type; /* 1 = F16, 8 = Q8_0, 12 = Q4_K; also applied to fast_output */
    float rope_base, eps, weight_std;
    uint64_t seed;
} S2dSynthConfig;

static uint64_t mix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

static float u01(uint64_t h) { return (float)(h >> 40) * (1.0f / 16777216.0f); }

static uint16_t f32_to_f16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exponent = (int32_t)((bits >> 23) & 0xffu);
    uint32_t mantissa = bits & 0x007fffffu;
    if (exponent == 0xff) return mantissa ? (sign | 0x7e00u) : (sign | 0x7c00u);
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

enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12 };
enum { K_NORM = 0, K_NORMAL = 1, K_LINEAR = 2 };

typedef struct {
    char name[96];
    uint64_t dims[2];
    int rank;
    uint32_t type;
    int kind;
    uint64_t offset, bytes;
} Tensor;

static uint64_t byte_len(uint32_t type, uint64_t n) {
    switch (type) {
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    case T_Q8_0: return (n + 31) / 32 * 34;
    case T_Q4_K: return (n + 255) / 256 * 144;
    }
    return 0;
}

/* Fill bytes [b0, b0+nb) of tensor t's payload (b0, nb aligned to the block). */
static void fill(const Tensor *t, uint64_t tid, uint64_t seed, float std, uint64_t b0,
                 uint64_t nb, uint8_t *out) {
    const uint64_t key = mix64(seed ^ mix64(tid + 1));
    if (t->type == T_F16) {
        uint16_t *h = (uint16_t *)out;
        const float scale = std * 1.7320508f; /* Irwin-Hall(4): var 1/3 */
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < (int64_t)(nb / 2); ++i) {
            uint64_t e = b0 / 2 + (uint64_t)i;
            if (t->kind == K_NORM) {
                h[i] = 0x3c00u;
                continue;
            }
            uint64_t a = mix64(key ^ (e * 2 + 0)), b = mix64(key ^ (e * 2 + 1));
            float s = u01(a) + u01(a << 24) + u01(b) + u01(b << 24) - 2.0f;
            h[i] = f32_to_f16(s * scale);
        }
    } else if (t->type == T_Q8_0) {
#pragma omp parallel for schedule(static)
        for (int64_t blk = 0; blk < (int64_t)(nb / 34); ++blk) {
            uint64_t bi = b0 / 34 + (uint64_t)blk;
            uint8_t *p = out + blk * 34;
            uint64_t h0 = mix64(key ^ (bi * 8));
            uint16_t d = f32_to_f16(1e-4f + 3e-4f * u01(h0));
            p[0] = (uint8_t)(d & 0xff), p[1] = (uint8_t)(d >> 8);
            for (int j = 0; j < 32; ++j) {
                uint64_t hj = mix64(key ^ (bi * 8 + 1 + (uint64_t)(j / 8)));
                uint32_t r = (uint32_t)(hj >> (8 * (j % 8))) & 0xffu;
                p[2 + j] = (uint8_t)(int8_t)((int32_t)(r % 255u) - 127);
            }
        }
    } else if (t->type == T_Q4_K) {
#pragma omp parallel for schedule(static)
        for (int64_t blk = 0; blk < (int64_t)(nb / 144); ++blk) {
            uint64_t bi = b0 / 144 + (uint64_t)blk;
            uint8_t *p = out + blk * 144;
            uint64_t h0 = mix64(key ^ (bi * 32));
            uint16_t d = f32_to_f16(1e-4f + 9e-4f * u01(h0));
            uint16_t dm = f32_to_f16(1e-4f + 9e-4f * u01(h0 << 24));
            p[0] = (uint8_t)(d & 0xff), p[1] = (uint8_t)(d >> 8);
            p[2] = (uint8_t)(dm & 0xff), p[3] = (uint8_t)(dm >> 8);
            for (int j = 0; j < 140; ++j) {
                uint64_t hj = mix64(key ^ (bi * 32 + 1 + (uint64_t)(j / 8)));
                p[4 + j] = (uint8_t)(hj >> (8 * (j % 8)));
            }
        }
    } else {
        memset(out, 0, nb);
    }
}

static void put(FILE *f, const void *p, size_t n, int *err) {
    if (!*err && fwrite(p, 1, n, f) != n) *err = errno ? errno : EIO;
}
static void put_u32(FILE *f, uint32_t v, int *e) { put(f, &v, 4, e); }
static void put_u64(FILE *f, uint64_t v, int *e) { put(f, &v, 8, e); }
static void put_str(FILE *f, const char *s, int *e) {
    put_u64(f, (uint64_t)strlen(s), e);
    put(f, s, strlen(s), e);
}
static void kv_u32(FILE *f, const char *k, uint32_t v, int *e) {
    put_str(f, k, e), put_u32(f, 4, e), put_u32(f, v, e);
}
static void kv_f32(FILE *f, const char *k, float v, int *e) {
    put_str(f, k, e), put_u32(f, 6, e), put(f, &v, 4, e);
}
static void kv_bool(FILE *f, const char *k, int v, int *e) {
    uint8_t b = (uint8_t)(v != 0);
    put_str(f, k, e), put_u32(f, 7, e), put(f, &b, 1, e);
}
static void kv_str(FILE *f, const char *k, const char *v, int *e) {
    put_str(f, k, e), put_u32(f, 8, e), put_str(f, v, e);
}

static int add(Tensor *ts, int n, const char *name, uint64_t d0, uint64_t d1, int rank,
               uint32_t type, int kind) {
    Tensor *t = &ts[n];
    memset(t, 0, sizeof *t);
    snprintf(t->name, sizeof t->name, "%s", name);
    t->dims[0] = d0, t->dims[1] = d1, t->rank = rank, t->type = type, t->kind = kind;
    t->bytes = byte_len(type, rank == 2 ? d0 * d1 : d0);
    return n + 1;
}

int s2d_synth_write_gguf(const char *path, const S2dSynthConfig *c, char *err, size_t cap) {
    int lt = c->linear_type;
    if (lt != T_F16 && lt != T_Q8_0 && lt != T_Q4_K) {
        snprintf(err, cap, "linear_type must be 1 (F16), 8 (Q8_0) or 12 (Q4_K)");
        return -1;
    }
    const uint64_t d = (uint64_t)c->d;
    const uint64_t qs = (uint64_t)c->heads * c->head_dim, kvs = (uint64_t)c->kv_heads * c->head_dim;
    const uint64_t fqs = (uint64_t)c->fast_heads * c->fast_head_dim,
                   fkvs = (uint64_t)c->fast_kv_heads * c->fast_head_dim;
    uint64_t blk = lt == T_Q8_0 ? 32 : (lt == T_Q4_K ? 256 : 1);
    if (d % blk || qs % blk || (uint64_t)c->ffn % blk || fqs % blk || (uint64_t)c->fast_ffn % blk) {
        snprintf(err, cap, "input dimensions must be multiples of the quant block (%llu)",
                 (unsigned long long)blk);
        return -1;
    }
    int cap_t = 6 + 9 * c->slow_layers + 7 * c->fast_layers;
    Tensor *ts = (Tensor *)calloc((size_t)cap_t, sizeof(Tensor));
    if (!ts) {
        snprintf(err, cap, "out of memory");
        return -1;
    }
    int n = 0;
    char nm[96];
    /* root tensors: registry.rs:625-650 */
    n = add(ts, n, "codebook_embeddings.weight", d, (uint64_t)c->num_codebooks * c->codebook_size, 2, T_F16, K_NORMAL);
    n = add(ts, n, "embeddings.weight", d, (uint64_t)c->vocab, 2, T_F16, K_NORMAL);
    n = add(ts, n, "fast_embeddings.weight", d, (uint64_t)c->codebook_size, 2, T_F16, K_NORMAL);
    n = add(ts, n, "fast_output.weight", d, (uint64_t)c->codebook_size, 2, (uint32_t)lt, K_LINEAR);
    n = add(ts, n, "fast_norm.weight", d, 0, 1, T_F16, K_NORM);
    n = add(ts, n, "norm.weight", d, 0, 1, T_F16, K_NORM);
    /* slow layers: registry.rs:360-410 */
    for (int l = 0; l < c->slow_layers; ++l) {
#define L(fmt) (snprintf(nm, sizeof nm, "layers.%d." fmt, l), nm)
        n = add(ts, n, L("attention.q_norm.weight"), (uint64_t)c->head_dim, 0, 1, T_F16, K_NORM);
        n = add(ts, n, L("attention.k_norm.weight"), (uint64_t)c->head_dim, 0, 1, T_F16, K_NORM);
        n = add(ts, n, L("attention.wqkv.weight"), d, qs + 2 * kvs, 2, (uint32_t)lt, K_LINEAR);
        n = add(ts, n, L("attention.wo.weight"), qs, d, 2, (uint32_t)lt, K_LINEAR);
        n = add(ts, n, L("attention_norm.weight"), d, 0, 1, T_F16, K_NORM);
        n = add(ts, n, L("ffn_norm.weight"), d, 0, 1, T_F16, K_NORM);
        n = add(ts, n, L("feed_forward.w1.weight"), d, (uint64_t)c->ffn, 2, (uint32_t)lt, K_LINEAR);
        n = add(ts, n, L("feed_forward.w2.weight"), (uint64_t)c->ffn, d, 2, (uint32_t)lt, K_LINEAR);
        n = add(ts, n, L("feed_forward.w3.weight"), d, (uint64_t)c->ffn, 2, (uint32_t)lt, K_LINEAR);
#undef L
    }
    /* fast layers: registry.rs:441-481 */
    for (int l = 0; l < c->fast_layers; ++l) {
#define L(fmt) (snprintf(nm, sizeof nm, "fast_layers.%d." fmt, l), nm)
        n = add(ts, n, L("attention.wqkv.weight"), d, fqs + 2 * fkvs, 2, (uint32_t)lt, K_LINEAR);
        n = add(ts, n, L("attention.wo.weight"), fqs, d, 2, (uint32_t)lt, K_LINEAR);
        n = add(ts, n, L("attention_norm.weight"), d, 0, 1, T_F16, K_NORM);
        n = add(ts, n, L("ffn_norm.weight"), d, 0, 1, T_F16, K_NORM);
        n = add(ts, n, L("feed_forward.w1.weight"), d, (uint64_t)c->fast_ffn, 2, (uint32_t)lt, K_LINEAR);
        n = add(ts, n, L("feed_forward.w2.weight"), (uint64_t)c->fast_ffn, d, 2, (uint32_t)lt, K_LINEAR);
        n = add(ts, n, L("feed_forward.w3.weight"), d, (uint64_t)c->fast_ffn, 2, (uint32_t)lt, K_LINEAR);
#undef L
    }
    uint64_t off = 0;
    for (int i = 0; i < n; ++i) {
        ts[i].offset = off;
        off = (off + ts[i].bytes + 31) / 32 * 32;
    }
    FILE *f = fopen(path, "wb");
    if (!f) {
        snprintf(err, cap, "IO: %s: %s", path, strerror(errno));
        free(ts);
        return -1;
    }
    int e = 0;
    put(f, "GGUF", 4, &e);
    put_u32(f, 3, &e);
    put_u64(f, (uint64_t)n, &e);
    put_u64(f, 28, &e); /* metadata count below */
    kv_str(f, "general.architecture", "fish-speech", &e);
    kv_str(f, "general.name", "s2dualar-synthetic", &e);
    kv_u32(f, "fish-speech.context_length", (uint32_t)c->context_length, &e);
    kv_u32(f, "fish-speech.embedding_length", (uint32_t)c->d, &e);
    kv_u32(f, "fish-speech.feed_forward_length", (uint32_t)c->ffn, &e);
    kv_u32(f, "fish-speech.block_count", (uint32_t)c->slow_layers, &e);
    kv_u32(f, "fish-speech.attention.head_count", (uint32_t)c->heads, &e);
    kv_u32(f, "fish-speech.attention.head_count_kv", (uint32_t)c->kv_heads, &e);
    kv_f32(f, "fish-speech.rope.freq_base", c->rope_base, &e);
    kv_f32(f, "fish-speech.attention.layer_norm_rms_epsilon", c->eps, &e);
    kv_bool(f, "fish_speech.attention_qk_norm", 1, &e);
    kv_u32(f, "fish_speech.fast_context_length", (uint32_t)c->fast_context_length, &e);
    kv_u32(f, "fish_speech.fast_embedding_length", (uint32_t)c->d, &e);
    kv_u32(f, "fish_speech.fast_feed_forward_length", (uint32_t)c->fast_ffn, &e);
    kv_u32(f, "fish_speech.fast_block_count", (uint32_t)c->fast_layers, &e);
    kv_u32(f, "fish_speech.fast_head_count", (uint32_t)c->fast_heads, &e);
    kv_u32(f, "fish_speech.fast_head_count_kv", (uint32_t)c->fast_kv_heads, &e);
    kv_u32(f, "fish_speech.fast_head_dim", (uint32_t)c->fast_head_dim, &e);
    kv_f32(f, "fish_speech.fast_rope_freq_base", c->rope_base, &e);
    kv_f32(f, "fish_speech.fast_layer_norm_rms_eps", c->eps, &e);
    kv_bool(f, "fish_speech.fast_attention_qk_norm", 0, &e);
    kv_u32(f, "fish_speech.codebook_size", (uint32_t)c->codebook_size, &e);
    kv_u32(f, "fish_speech.num_codebooks", (uint32_t)c->num_codebooks, &e);
    kv_u32(f, "fish_speech.semantic_begin_id", (uint32_t)c->sem_begin, &e);
    kv_u32(f, "fish_speech.semantic_end_id", (uint32_t)c->sem_end, &e);
    kv_bool(f, "fish_speech.scale_codebook_embeddings", 1, &e);
    kv_bool(f, "fish_speech.tie_word_embeddings", 1, &e);
    kv_bool(f, "fish_speech.fast_project_in", 0, &e);
    for (int i = 0; i < n; ++i) {
        put_str(f, ts[i].name, &e);
        put_u32(f, (uint32_t)ts[i].rank, &e);
        for (int k = 0; k < ts[i].rank; ++k) put_u64(f, ts[i].dims[k], &e);
        put_u32(f, ts[i].type, &e);
        put_u64(f, ts[i].offset, &e);
    }
    long pos = ftell(f);
    static const uint8_t zeros[32] = {0};
    if (pos < 0) e = EIO;
    else if (pos % 32) put(f, zeros, (size_t)(32 - pos % 32), &e);
    const uint64_t CHUNK = 1ull << 26; /* 64 MiB, a multiple of 34*32 is not needed: see below */
    uint8_t *buf = (uint8_t *)malloc(CHUNK + 144 * 64);
    if (!buf) e = ENOMEM;
    uint64_t written = 0;
    for (int i = 0; i < n && !e; ++i) {
        Tensor *t = &ts[i];
        if (written < t->offset) put(f, zeros, (size_t)(t->offset - written), &e), written = t->offset;
        /* chunk boundaries are multiples of the block size of this tensor */
        uint64_t unit = t->type == T_Q8_0 ? 34 : (t->type == T_Q4_K ? 144 : 2);
        uint64_t step = CHUNK / unit * unit;
        for (uint64_t b = 0; b < t->bytes && !e; b += step) {
            uint64_t nb = t->bytes - b < step ? t->bytes - b : step;
            fill(t, (uint64_t)i, c->seed, c->weight_std, b, nb, buf);
            put(f, buf, (size_t)nb, &e);
            written += nb;
        }
    }
    free(buf);
    if (fclose(f) && !e) e = errno ? errno : EIO;
    free(ts);
    if (e) {
        snprintf(err, cap, "IO: writing %s: %s", path, strerror(e));
        return -1;
    }
    return 0;
}
