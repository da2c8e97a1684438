// s2d_kernels.cuh -- kernel argument blocks and host launchers.
#pragma once

#include <cuda_fp16.h>
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
    const uint16_t *W;   // f16 bits, [N][K] row-major (GGUF dims [K, N]), or ggml blocks (wq)
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
    int wq;              // weight format: 0 f16 rows, 1 ggml Q8_0, 2 ggml Q4_K (EngineWeight)
};

// Paged KV caches of the batched path.  A page holds kKvPage consecutive
// positions of one sequence for every layer: [layer][K | V][kv head]
// [kKvPage][hd]; pages[seq * per_seq + t / kKvPage] is the page of position t
// of sequence seq.  Paged kernels get the layer's K (and V) base inside page
// 0, so every row is base + page * page_elems + (kvh * kKvPage + t % kKvPage)
// * hd.  The rows kernels stage K/V chunks of 16 or 32 positions that start at
// multiples of the chunk, so a chunk never spans two pages.
constexpr int kKvPage = 64;
struct KvPages {
    const int32_t *pages;  // nullptr: contiguous caches
    int per_seq;           // page-table entries per sequence
    size_t page_elems;     // elements (f16 or f32) of one page
};
// Element offset of position t's row of kv head kvh of sequence seq from the
// layer's K (or V) base: paged, or contiguous sequences of seq_stride
// elements with [kv head][max_seq][hd] layer caches.
__host__ __device__ __forceinline__ size_t kv_row(const KvPages &p, size_t seq_stride, int max_seq, int seq,
                                                  int kvh, int t, int hd) {
    if (p.pages)
        return (size_t)p.pages[(size_t)seq * p.per_seq + t / kKvPage] * p.page_elems +
               ((size_t)kvh * kKvPage + t % kKvPage) * hd;
    return (size_t)seq * seq_stride + ((size_t)kvh * max_seq + t) * hd;
}

struct RopeArgs {
    const float *qkv;    // [M][ld_qkv]: Q | K | V
    int ld_qkv;
    // With qkv_lo: row m is (qkv[m] + qkv_lo[m]) * inv[m], the two halves of
    // a rows-path GEMM over the stacked hi / lo rows (the store combine).
    const float *qkv_lo;
    const float *inv;
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
    // Batched rows (0 = one sequence): row m belongs to sequence
    // m / rows_per_seq at position pos_const + j (j = m % rows_per_seq), plus
    // st_b[seq].n_past when st_pos is set; a sequence whose st_b[seq].done
    // is set writes nothing.  Sequence s's caches start kv_seq_stride
    // elements after sequence s-1's.
    int rows_per_seq;
    const DevState *st_b;
    int st_pos;
    size_t kv_seq_stride;
    KvPages kv_pages;    // paged caches (kv_pages.pages set): kv_seq_stride unused
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
    int batched;             // with tokens == nullptr: row m is sequence m (st[m], frame_codes + m*K)
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
    // batched (grid.y = sequences): per-sequence strides of slow_hidden,
    // fast_x, frame_codes and codes_out; st is then an array
    int batched;
    size_t hidden_stride, fast_x_stride, codes_stride, frame_stride;
};

// Random draws of the sampler: the reference's SeededRng LCG (state in
// *rng), or Philox4x32-10 keyed by philox_key with the sequence index and
// the draw counter (*rng) as the counter.
enum RngKind { RNG_SEEDED = 0, RNG_PHILOX = 1 };

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
    int rng_kind;           // RngKind
    uint64_t philox_key;
    uint32_t rng_seq;       // Philox sequence index of block 0
    // batched (one block per sequence, grid.x = sequences): st is an array
    // and the rng is st[seq].rng; logits, frame_codes, codes_out, fast_x_next
    // and out_token advance by these strides per sequence
    int batched;
    size_t logits_stride, codes_stride, fast_x_stride, frame_stride;
};

// ---- persistent layer engine (s2d_engine.cu) -------------------------------

enum EngineOpKind { OP_GEMV = 0, OP_ATTN = 1, OP_SAMPLE = 2, OP_ATTN_CTX = 3 };

constexpr int kEngineMaxPeers = 8;  // tensor-parallel ranks of one engine program
constexpr int kEngineMaxCtx = 16;   // positions of an ATTN op over an LL context (ctx_n)
constexpr int kEngineSampleMax = 4096;  // candidates of a SAMPLE op

// One step of the engine's program.  A GEMV op reads its input vector(s) and
// writes its outputs like gemv_kernel (GemvArgs fields); an ATTN op fuses
// rope_kv_kernel and attn_kernel (RopeArgs / AttnArgs fields).
//
// Values passed between ops of one launch are "LL words": 64-bit words
// holding a float in the low half and a tag in the high half, written with a
// single 64-bit store.  The tag of op i's outputs in a launch with epoch e is
// engine_tag(e, i); a reader polls the words it needs until they carry the
// producer's tag, so no grid-wide barrier separates the ops.  Inputs written
// before the launch are plain floats (src index -1).  A SAMPLE op runs the
// device sampler on one CTA (see the SAMPLE fields).
struct EngineOp {
    int kind, epi, M;
    // GEMV
    const uint16_t *W, *W2;
    const void *x;       // [M][ldx] floats, or LL words of op x_src
    int ldx, x_src;
    const float *norm_w;
    float eps;
    void *y;             // [M][ldy] LL words when y_ll, else floats
    int ldy, y_ll;
    const void *resid;   // [M][ldr] (EPI_RESID) floats, or LL words of op resid_src; may alias y
    int ldr, resid_src;
    float *x_out;        // optional: CTA 0 writes the normalised input [M][K] as floats
    int K, N;
    int row_base, n_contig, extra_row;
    // ATTN
    const uint64_t *qkv; // LL words [M][ld_qkv] of op qkv_src: Q | K | V
    int ld_qkv, qkv_src;
    void *kcache, *vcache;
    int max_seq, kv_half;
    const float *q_norm, *k_norm;
    const float2 *rope_cs;  // [max_seq][hd / 2] (cos, sin) of pos / rope_base^(2i / hd)
    const int32_t *pos_dev;
    int pos_const;
    int H, Hkv, hd, S;
    float scale;
    uint64_t *att_out;   // LL words [M][H * hd]
    uint64_t *part;      // LL words [M][H][S][hd + 2]: split partials (max, sum, P.V with
                         // element lane * hd/32 + e at 2 + e * 32 + lane)
    // GEMV weights in the engine's slot order (engine_relayout): the slot
    // of row tile [tr0, tr0 + R) and K slice s starts at element
    // Wt + tr0 * K * mats + s * R * kt * mats and holds [mat][R][kw].
    const uint16_t *Wt;
    int wt;              // EngineWeight of W (and W2)
    // Tensor parallelism (every field 0 on one GPU).  An input of x_nsum > 1
    // rows is the sum, in rank order, of x_nsum rank rows of LL words
    // x_rstride words apart (each rank's partial sums of the same op); the
    // residual likewise with r_nsum / r_rstride.  With n_peer > 0 every
    // output word also goes to y_peer[q] + m * ldy + row for each rank q (this
    // rank's row of each rank's exchange buffer, the peers' over NVLink).
    int x_nsum, r_nsum, n_peer;
    long long x_rstride, r_rstride;
    uint64_t *y_peer[kEngineMaxPeers];
    // ATTN_CTX: attention over an LL context of ctx_n <= kEngineMaxCtx
    // positions (ATTN fields otherwise): position j's Q | K | V row is the
    // [ld_qkv] LL words ctx_qkv[j] written by op ctx_src[j], the op's own
    // tokens included; K is normed and rotated here, and no cache and no
    // ring slot is used.  Token m attends to positions [0, pos_const + m].
    // SAMPLE and ATTN_CTX ops run only in the frame variant of the engine
    // kernel (launch_engine's `frame`).
    int ctx_n;
    const uint64_t *ctx_qkv[kEngineMaxCtx];
    int ctx_src[kEngineMaxCtx];
    // SAMPLE: CTA sample_cta polls the K <= kEngineSampleMax logits (LL words
    // x of op x_src), draws a token with the device sampler under samp (its
    // logits / fast_x_next fields unused) and writes row `token` of
    // samp.fast_emb, N = d values, as LL words to y (when y is not null).
    int sample_cta;
    SampleArgs samp;
};

// The tag of op `op`'s outputs in the launch of epoch `epoch` (op < 1024).
__host__ __device__ __forceinline__ uint32_t engine_tag(uint32_t epoch, int op) {
    return (epoch << 10) | (uint32_t)op;
}
constexpr int kEngineMaxOps = 1023;

struct EngineArgs {
    const EngineOp *ops;
    int n_ops;
    int nslots, slot_bytes;            // shared-memory weight ring
    int area_bytes;                    // staged inputs / attention tiles (multiple of 128)
    uint32_t *epoch;                   // launch epoch (>= 1): read at start, advanced by CTA 0 at exit
    const int32_t *done;               // DevState::done or nullptr
    int32_t *error;                    // DevState::error
    // Optional timeline (nullptr: off).  CTAs 0 and gridDim-1 record
    // %globaltimer at each op: [cta][op][0] op started, [1] inputs staged,
    // [2] op finished by the consumers, [3] producer issued the op's last slot;
    // then [op][cta] every CTA's finish time.
    unsigned long long *trace;
    int l2_lead;  // weight slots the producer prefetches into L2 ahead of the ring
};

constexpr int kEngineConsumerWarps = 8;
constexpr int kEngineThreads = (kEngineConsumerWarps + 1) * 32;
constexpr int kEngineSlotBytes = 24576;  // default ring slot size
constexpr int kEngineSmemMax = 230400;  // dynamic smem, under the 227 KiB opt-in limit
constexpr int kEngineTileRows = 32;      // output rows of one GEMV row tile
constexpr int kEngineMaxSlots = 64;
constexpr int kEngineBarrierBytes = 1024; // full + empty mbarriers of up to 64 slots
constexpr int kEngineMaxK = 10240;        // longest GEMV input the consumers stage

// Rows [*r0, *r1) of an N-row linear owned by CTA c of G.
__host__ __device__ __forceinline__ void engine_cta_rows(int N, int c, int G, int *r0, int *r1) {
    *r0 = (int)(((long long)N * c) / G);
    *r1 = (int)(((long long)N * (c + 1)) / G);
}

// Weight formats of the engine's GEMVs.  In slot order (engine_relayout) a
// row slice of kw columns is: F16, kw f16 values; Q8_0 (ggml blocks of 32:
// f16 scale d + 32 int8, value d*q), kw int8 quants then kw/32 f16 scales;
// Q4_K (ggml superblocks of 256 in sub-blocks of 32, value (d*sc)*q -
// dmin*m), kw/2 bytes of 4-bit quants (byte k: element 2k in the low
// nibble, 2k+1 in the high one) then per sub-block the f32 pair
// (d*sc, dmin*m).
enum EngineWeight { EW_F16 = 0, EW_Q8_0 = 1, EW_Q4_K = 2 };
__host__ __device__ __forceinline__ int engine_row_bytes(int wt, int kw) {
    return wt == EW_F16 ? 2 * kw : wt == EW_Q8_0 ? kw + kw / 16 : kw / 2 + kw / 4;
}
// Columns per lane chunk: 8 f16 (16 bytes), 16 quantized weights.
__host__ __device__ __forceinline__ int engine_chunk_cols(int wt) { return wt == EW_F16 ? 8 : 16; }

// K-slice geometry of a GEMV: slices of kt columns (64 / mats lane chunks
// per row: two or one per consumer lane), the last one possibly shorter,
// and row tiles of at most rmax rows so that a slot of mats * rmax row
// slices fits slot_bytes.
struct SliceGeom {
    int kt, nk, rmax;
};
__host__ __device__ inline SliceGeom engine_slice_geom(int mats, int K, int slot_bytes, int wt = EW_F16) {
    SliceGeom g;
    const int kt = 64 * engine_chunk_cols(wt) / mats;
    g.kt = kt < K ? kt : K;
    g.nk = (K + g.kt - 1) / g.kt;
    g.rmax = slot_bytes / (mats * engine_row_bytes(wt, g.kt));
    if (g.rmax > kEngineTileRows) g.rmax = kEngineTileRows;
    if (g.rmax < 1) g.rmax = 1;
    return g;
}

// Row tiles of a CTA's n rows: ceil(n / rmax) tiles of near-equal size; tile
// t covers rows [*a, *b) relative to the CTA's first row.
__host__ __device__ __forceinline__ int engine_tile_count(int n, int rmax) { return (n + rmax - 1) / rmax; }
__host__ __device__ __forceinline__ void engine_tile_rows(int n, int t, int ntiles, int *a, int *b) {
    *a = (int)(((long long)n * t) / ntiles);
    *b = (int)(((long long)n * (t + 1)) / ntiles);
}

// Error codes the engine writes into DevState::error.
constexpr int kErrEngineWeights = 16;  // a weight-ring wait ran out
constexpr int kErrEngineWait = 17;     // a wait for another op's outputs ran out
constexpr int kErrEngineAlign = 18;    // the shared-memory ring is not 128-byte aligned

// frame: the kernel variant that also runs SAMPLE and ATTN_CTX ops.
cudaError_t launch_engine(const EngineArgs &a, int grid, size_t smem, cudaStream_t s, bool frame = false);

// Copies a linear's weights into the engine's slot order for a `grid`-CTA
// launch with ring slots of slot_bytes.  W and W2 are GGUF tensors of ggml
// type gtype (F16, Q8_0 or Q4_K: rows of K elements); dst receives
// N * engine_row_bytes(wt, K) * mats bytes in the EngineWeight format wt.
// Output row r reads source row (n_contig < 0 ? r : r < n_contig ?
// row_base + r : extra_row) of W and row r of W2 (when W2 is not null).
cudaError_t launch_engine_relayout(const void *W, const void *W2, int gtype, int N, int K, int n_contig,
                                   int row_base, int extra_row, int grid, int slot_bytes, void *dst,
                                   cudaStream_t s);
// Bytes of the engine copy of an N x K linear of ggml type gtype.
size_t engine_weight_bytes(int gtype, int N, int K, int mats);
int engine_weight_format(int gtype);  // EngineWeight, or -1 if unsupported

// Attention in the engine.  A group's query vectors and the new tokens' K
// and V rows (at most 2 tokens) sit in the shared area (attn_group_bytes per
// group).  The cached K/V rows of a group's item come through the weight
// ring, in program order, as slots of up to attn_slot_rows positions:
// [K rows][V rows] (each tile 128-byte aligned), and in a group's first slot
// a side block: the RoPE (cos, sin) rows of the new positions [2][hd/2], then
// the Q and K norm gains [hd] each.
__host__ __device__ __forceinline__ int attn_round(int b) { return (b + 127) / 128 * 128; }
__host__ __device__ __forceinline__ int attn_group_bytes(int rep, int hd, int kvb) {
    return attn_round(rep * hd * 4 + 4 * hd * kvb);
}
__host__ __device__ __forceinline__ int attn_side_bytes(int hd) { return 16 * hd; }
// Shared area of one group of an ATTN op over an LL context: the rep query
// rows, then ctx K rows and ctx V rows, f32.
__host__ __device__ __forceinline__ int attn_ctx_group_bytes(int rep, int hd, int ctx) {
    return attn_round((rep + 2 * ctx) * hd * 4);
}
// Shared area of a SAMPLE op over n candidates: the logits [n] f32, the sort
// keys [next power of two >= n] u64, the probabilities [n + 1] f32, then
// scratch_bytes of SampleScratch.
__host__ __device__ __forceinline__ int engine_sample_pow2(int n) {
    int p = 2;
    while (p < n) p <<= 1;
    return p;
}
__host__ __device__ __forceinline__ int engine_sample_bytes(int n, int scratch_bytes) {
    return attn_round(n * 4) + engine_sample_pow2(n) * 8 + attn_round((n + 1) * 4) + scratch_bytes;
}
__host__ __device__ __forceinline__ int attn_slot_rows(int hd, int kvb, int slot_bytes) {
    const int p = (slot_bytes - attn_side_bytes(hd) - 256) / (2 * hd * kvb);
    return p > 32 ? 32 : p;
}
__host__ __device__ __forceinline__ int attn_tile_bytes(int rows, int hd, int kvb) { return attn_round(rows * hd * kvb); }

constexpr int kSampleMax = 8192;
constexpr int kSampleThreads = 1024;
// top-k up to this size takes the sampler's radix-select path instead of a full sort
constexpr int kSampleSelMax = 256;
constexpr int kGemvThreads = 256;

// Host launchers (s2d_kernels.cu). All enqueue on `stream`; pdl enables
// programmatic dependent launch on the kernel.
cudaError_t launch_gemv(const GemvArgs &a, int M, int epi, cudaStream_t s, bool pdl);
cudaError_t launch_rope_kv(const RopeArgs &a, bool kv_half, cudaStream_t s, bool pdl);
cudaError_t launch_attention(const AttnArgs &a, bool kv_half, cudaStream_t s, bool pdl);
cudaError_t launch_embed(const EmbedArgs &a, cudaStream_t s, bool pdl);
cudaError_t launch_fast_init(const FastInitArgs &a, cudaStream_t s, bool pdl);
cudaError_t launch_fast_init_batch(const FastInitArgs &a, int n_seq, cudaStream_t s);
cudaError_t launch_sample(const SampleArgs &a, cudaStream_t s, bool pdl);
// The sampler's Philox4x32-10 block function on one counter (out_dev: 4 words).
cudaError_t launch_philox(const uint32_t counter[4], const uint32_t key[2], uint32_t *out_dev, cudaStream_t s);
// Batched sampler: one block per sequence (a.batched set).
cudaError_t launch_sample_batch(const SampleArgs &a, int n_seq, cudaStream_t s);
cudaError_t launch_f16_to_f32(const uint16_t *src, float *dst, int64_t n, cudaStream_t s);
// ggml Q8_0 / Q4_K blocks (gtype 8 / 12) of n elements -> f32 (the block
// formulas d*q and (d*sc)*q - dmin*m, each rounded once in f32).
cudaError_t launch_dequant(int gtype, const void *src, float *dst, int64_t n, cudaStream_t s);
// Q8_0 (wq 1) / Q4_K (wq 2) blocks -> f16 values (n elements, dst 16-byte aligned).
cudaError_t launch_dequant_f16(int wq, const void *src, __half *dst, int64_t n, cudaStream_t s);
cudaError_t launch_rms_norm_heads(const float *x, const float *w, float *y, int64_t n, int hd,
                                  float eps, cudaStream_t s);
cudaError_t launch_set_state(DevState *st, int32_t n_past, int32_t prompt_cols, uint64_t rng,
                             cudaStream_t s);
// Sets the dynamic shared-memory limits of the GEMV and sampler kernels
// (call once per device before launching or capturing them).
cudaError_t configure_kernels();

}  // namespace s2d
