// s2d_runtime.cu -- handle, loader and C ABI of libs2d.so (include/s2d.h).
//
// The handle owns the HBM-resident weights (uploaded once at open), the
// Slow-AR KV cache, the activation and scratch buffers, one CUDA stream, the
// device-resident generation state and the captured frame graph.  The frame
// graph is one full Dual-AR frame: Fast-AR codebooks 1..K-1 (9 sampled passes
// over the 4 Fast-AR layers), the embedding-sum feedback, the 36-layer
// Slow-AR step, the masked LM head and the semantic sampler; it is replayed
// once per frame without any host round-trip.
#include <cublas_v2.h>
#include <dlfcn.h>
#include <nccl.h>
#include <cuda_fp16.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <memory>
#include <tuple>
#include <string>
#include <vector>

#include "../../include/s2d.h"
#include "s2d_gguf.h"
#include "s2d_kernels.cuh"
#include "s2d_sample.cuh"
#include "s2d_prefill.cuh"
#include "s2d_tcgemm.cuh"

using namespace s2d;

namespace {

constexpr int kMaxM = 4;  // tokens per GEMV pass (prefill chunk)

struct LayerDev {
    // linears: f16 rows, or ggml Q8_0 / Q4_K blocks (wq, an EngineWeight)
    const uint16_t *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w2 = nullptr, *w3 = nullptr;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    int wq = EW_F16;
};

int ggml_type_of(int wq) { return wq == EW_Q8_0 ? 8 : wq == EW_Q4_K ? 12 : 1; }

struct TensorDev {
    const GgufTensor *info = nullptr;
    uint8_t *dev = nullptr;
};

struct ArShape {
    int L, d, F, H, Hkv, hd, ctx;
    float rope_base, eps;
    bool qk_norm;
    int qs() const { return H * hd; }
    int kvs() const { return Hkv * hd; }
    int qkv_out() const { return qs() + 2 * kvs(); }
};

// A program of the persistent layer engine (s2d_engine.cu), resident in HBM.
struct EngineProgram {
    EngineOp *ops = nullptr;
    int n_ops = 0;
    bool frame = false;  // has SAMPLE / ATTN_CTX ops: the frame kernel variant
    int nslots = 0, area_bytes = 0;
    size_t smem = 0;
};

struct GenKey {
    uint32_t max_new = 0, min_tokens = 0, im_end = 0;
    float temperature = 0, top_p = 0;
    int32_t top_k = 0;
    bool operator==(const GenKey &o) const {
        return max_new == o.max_new && min_tokens == o.min_tokens && im_end == o.im_end &&
               temperature == o.temperature && top_p == o.top_p && top_k == o.top_k;
    }
};

}  // namespace

struct S2dHandle {
    std::string err;
    int device = 0;
    cudaStream_t stream = nullptr;
    S2dConfig cfg{};
    S2dGraphSpec spec{};
    ArShape slow{}, fast{};
    Gguf gguf;
    std::vector<TensorDev> tensors;  // parallel to gguf.tensors
    uint8_t *arena = nullptr;
    float *norm_arena = nullptr;
    std::vector<LayerDev> slow_layers, fast_layers;
    const uint16_t *emb = nullptr, *cb_emb = nullptr, *fast_emb = nullptr, *fast_out = nullptr;
    int fast_out_wq = EW_F16;
    float *norm = nullptr, *fast_norm = nullptr;
    float *rope_slow = nullptr, *rope_fast = nullptr;
    __half *kv_slow = nullptr;  // [L][2][Hkv][max_seq][hd]
    float *kv_fast = nullptr;   // [Lf][2][Hkv][ctx][hd]
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr, *act = nullptr;
    float *fast_x = nullptr, *hidden_post = nullptr, *logits = nullptr, *logits_fast = nullptr;
    float *part = nullptr;
    int32_t *counters = nullptr;
    int S_slow = 16, S_fast = 1;
    DevState *st = nullptr;
    int32_t *tokens_dev = nullptr;
    size_t tokens_cap = 0;
    int32_t *frame_codes = nullptr, *codes_out = nullptr;
    size_t codes_cap = 0;
    uint32_t *tok_out = nullptr;
    uint32_t *code_override = nullptr;
    int n_allowed_extra = 1;
    int32_t n_past = 0;
    // captured frame
    cudaGraphExec_t frame_exec = nullptr;
    GenKey frame_key;
    uint32_t frame_kernels = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev2 = nullptr;
    bool pdl = true;
    uint32_t launches = 0;  // kernels enqueued through this handle
    // persistent layer engine
    bool use_engine = true;
    int num_sms = 0;
    // batched prefill (s2d_prefill.cu): up to pf_cap tokens per layer pass
    cublasHandle_t blas = nullptr;
    void *blas_ws = nullptr;
    // quantized models: one layer's linears dequantised to f16 for the
    // tensor-core rows path (wqkv, wo, w1, w3, w2)
    __half *qscratch[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    // Batched generation of a quantized model: every quantized linear expanded
    // once to f16 (rounded to nearest), per layer, and fast_output; empty
    // until the first batched call.
    std::vector<LayerDev> slow_f16, fast_f16;
    __half *fast_out_f16 = nullptr;
    std::vector<__half *> f16_bufs;
    // tensor parallelism on the engine (setup_exchange): this rank's exchange
    // buffer and every rank's, mapped here (xchg_peer[tp_rank] == xchg)
    uint64_t *xchg = nullptr;
    uint64_t *xchg_peer[kEngineMaxPeers] = {};
    size_t xchg_words = 0;
    int pf_cap = 0;
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_att = nullptr, *pf_act = nullptr;
    float *pf_inv = nullptr, *pf_y2 = nullptr, *pf_y2b = nullptr;
    __half *pf_xs = nullptr;
    uint32_t *engine_epoch = nullptr;  // launch epoch of the engine's LL words (starts at 1)
    // engine activations as LL words: residual, QKV, attention out, SwiGLU out, split partials
    uint64_t *ll_x = nullptr, *ll_qkv = nullptr, *ll_att = nullptr, *ll_act = nullptr, *ll_part = nullptr;
    float2 *rope_cs_slow = nullptr, *rope_cs_fast = nullptr;  // [positions][hd / 2] (cos, sin)
    std::vector<EngineProgram> fast_progs;  // index = codebook being produced (1..K-1)
    // A frame's whole Fast-AR in one engine launch (build_fast_frame): every
    // pass, its head and its sampler; S2D_FAST_FRAME=0 keeps one launch per
    // pass.  Its passes keep their WQKV words for the later passes'
    // attention (fr_qkv [pass][layer][2][qkv_out]) and exchange the logits
    // (fr_logits) and the next input rows (fr_x [codebook][d]) as LL words.
    EngineProgram fast_frame_prog;
    GenKey fast_frame_key;
    bool fast_frame = true;
    uint64_t *fr_qkv = nullptr, *fr_logits = nullptr, *fr_x = nullptr;
    // engine weight copies in slot order, keyed by (W, W2, N, K, n_contig, row_base, extra_row)
    std::map<std::tuple<const uint16_t *, const uint16_t *, int, int, int, int, int>, uint16_t *> tiled;
    size_t tiled_bytes = 0;
    int slot_bytes = kEngineSlotBytes;  // engine ring slot size (S2D_SLOT_KB)
    int l2_lead = 0;                    // engine L2 prefetch lead in slots (S2D_L2_LEAD)
    int engine_att_splits = 0;          // cap on the Slow-AR attention splits (S2D_ATT_SPLITS; 0: none)
    int attn_blocks_per_sm = 16;        // batched step: rows-attention blocks per SM (S2D_BATCH_ATT_BLOCKS)
    int attn_stages = 2;                // batched step: rows-attention K/V ring stages, 2 or 4 (S2D_BATCH_ATT_STAGES)
    int attn_mma = 1;                   // batched step: tensor-core attention (S2D_DECODE_MMA)
    int attn_mma_warps = 4;             // its warps per block, 2 or 4 (S2D_DECODE_WARPS)
    int attn_mma_stages = 2;            // its K/V ring stages per warp, 2 or 3 (S2D_DECODE_STAGES)
    int attn_mma_blocks_per_sm = 2;     // its blocks per SM when choosing splits (S2D_DECODE_BLOCKS)
    int attn_mma_chunk = 16;            // its positions per staged chunk, 16 or 32 (S2D_DECODE_CHUNK)
    int attn_mma_order = 1;             // its blocks longest context first (S2D_DECODE_ORDER)
    int prefill_mma = 1;                // prompt-chunk attention on the tensor cores (S2D_PREFILL_MMA)
    int prefill_tc = 1;                 // ... on tcgen05 at head dim 128 (S2D_PREFILL_TC)
    EngineProgram slow_prog;
    uint32_t slow_prog_im_end = 0xffffffffu;
    // Slow-AR tensor parallelism (s2d_open_tp): this rank's shard of every
    // Slow-AR layer (heads of wqkv / wo / the KV cache, an FFN slice of
    // w1 / w3 / w2) and the communicator of the two per-layer allreduces
    int tp = 1, tp_rank = 0;
    // rows-path linears on the tcgen05 GEMM (S2D_TCGEMM=1); by default on
    // cuBLAS + the combine pass, which measures faster for now
    bool use_tc = false;
    ncclComm_t comm = nullptr;
    uint8_t *shard_arena = nullptr;
    S2dTpShard shard{};
    // batched generation (s2d_generate_codes_batch): the Slow-AR caches of
    // its sequences live in a pool of kKvPage-position pages (KvPages), with
    // a page table of kv_per_seq entries per sequence; kv_slow holds only the
    // single-sequence calls' cache
    int max_batch = 1;
    size_t kv_slow_seq = 0;
    __half *kv_pool = nullptr;
    int32_t *kv_page_table = nullptr;  // [max_batch][kv_per_seq] page ids (device)
    int kv_per_seq = 0;
    size_t kv_page_elems = 0;
    const int32_t *pf_pages = nullptr;  // set while a batched sequence is prefilled: its page-table row
    DevState *st_b = nullptr;             // [max_batch]
    float *bx = nullptr;                  // [max_batch][d] Slow-AR residual rows
    float *fx = nullptr;                  // [max_batch][2][d] Fast-AR rows of a pass
    float *hidden_b = nullptr;            // [max_batch][d] post-norm hidden
    float *logits_b = nullptr;            // [max_batch][n_sem + 1]
    float *logits_fast_b = nullptr;       // [max_batch][codebook_size]
    float *kv_fast_b = nullptr;           // [max_batch][Lf][2][Hkv][ctx][hd]
    int32_t *frame_codes_b = nullptr;     // [max_batch][K]
    int32_t *codes_b = nullptr;           // [max_batch][K][max_new]
    size_t codes_b_cap = 0;
    float *ra_part = nullptr;             // rows attention split partials
    int32_t *ra_counters = nullptr;
    int32_t *batch_order = nullptr;       // [max_batch]: sequences by prompt length, longest first
    int ra_rows = 0, ra_smax = 0;
    cudaGraphExec_t batch_exec = nullptr;
    // s2d_profile_batch: events recorded after each launch, tagged with the
    // launch's category (null outside profiling); codes are not stored
    std::vector<std::pair<int, cudaEvent_t>> *marks = nullptr;
    bool batch_profile = false;
    GenKey batch_key;
    int batch_n = 0, batch_rng_kind = -1;
    uint64_t batch_philox = 0;
    // Continuous batching (s2d_serve_*): every slot of the batched frame is
    // either free, running or finished; admission hands a sequence the pool
    // pages its prompt and generation need (serve_free lists the pages no
    // slot holds) and writes them into the slot's page-table row.
    bool serving = false;
    GenKey serve_key;
    int serve_rng_kind = 0;
    uint64_t serve_philox = 0;
    std::vector<int32_t> serve_cols;  // per slot: prompt columns, -1 when free
    std::vector<std::vector<int32_t>> serve_pages;
    std::vector<int32_t> serve_free;
    std::vector<int32_t> pool_order;  // the pool's pages in dealing order
    size_t kv_pool_pages = 0;
    uint32_t batch_kernels = 0;
};

namespace {

int32_t set_err(S2dHandle *h, int32_t code, const std::string &msg) {
    if (h) h->err = msg;
    return code;
}

#define CK(call)                                                                              \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess)                                                                \
            return set_err(h, S2D_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// ---------------------------------------------------------------------------
// loading
// ---------------------------------------------------------------------------

// DualArGraphSpec::from_gguf (registry.rs:45-103), shape-parametric: the slow
// head_dim is the q_norm length (the reference forces QK_NORM_SIZE,
// registry.rs:46-52) and the S2-Pro constants of registry.rs:109-213 are
// replaced by metadata/tensor consistency checks in bind_weights().
int32_t read_spec(S2dHandle *h) {
    const Gguf &g = h->gguf;
    std::string e, arch;
    if (!g.meta_str("general.architecture", &arch, &e)) return set_err(h, S2D_EIO, "missing general.architecture");
    if (arch != "fish-speech")
        return set_err(h, S2D_EINVAL, "expected fish-speech transformer GGUF, got " + arch);
    uint32_t u[20];
    float f[4];
    bool b[6];
    bool ok = g.meta_bool("fish_speech.attention_qk_norm", &b[0], &e) &&
              g.meta_u32("fish-speech.context_length", &u[0], &e) &&
              g.meta_u32("fish-speech.embedding_length", &u[1], &e) &&
              g.meta_u32("fish-speech.feed_forward_length", &u[2], &e) &&
              g.meta_u32("fish-speech.block_count", &u[3], &e) &&
              g.meta_u32("fish-speech.attention.head_count", &u[4], &e) &&
              g.meta_u32("fish-speech.attention.head_count_kv", &u[5], &e) &&
              g.meta_f32("fish-speech.rope.freq_base", &f[0], &e) &&
              g.meta_f32("fish-speech.attention.layer_norm_rms_epsilon", &f[1], &e) &&
              g.meta_u32("fish_speech.fast_context_length", &u[6], &e) &&
              g.meta_u32("fish_speech.fast_embedding_length", &u[7], &e) &&
              g.meta_u32("fish_speech.fast_feed_forward_length", &u[8], &e) &&
              g.meta_u32("fish_speech.fast_block_count", &u[9], &e) &&
              g.meta_u32("fish_speech.fast_head_count", &u[10], &e) &&
              g.meta_u32("fish_speech.fast_head_count_kv", &u[11], &e) &&
              g.meta_u32("fish_speech.fast_head_dim", &u[12], &e) &&
              g.meta_f32("fish_speech.fast_rope_freq_base", &f[2], &e) &&
              g.meta_f32("fish_speech.fast_layer_norm_rms_eps", &f[3], &e) &&
              g.meta_bool("fish_speech.fast_attention_qk_norm", &b[1], &e) &&
              g.meta_u32("fish_speech.codebook_size", &u[13], &e) &&
              g.meta_u32("fish_speech.num_codebooks", &u[14], &e) &&
              g.meta_u32("fish_speech.semantic_begin_id", &u[15], &e) &&
              g.meta_u32("fish_speech.semantic_end_id", &u[16], &e) &&
              g.meta_bool("fish_speech.scale_codebook_embeddings", &b[2], &e) &&
              g.meta_bool("fish_speech.tie_word_embeddings", &b[3], &e) &&
              g.meta_bool("fish_speech.fast_project_in", &b[4], &e);
    if (!ok) return set_err(h, S2D_EIO, e);
    if (b[4]) return set_err(h, S2D_EINVAL, "fast_project_in is not supported (fast_ar.rs:366-370)");
    if (!b[2] || !b[3])
        return set_err(h, S2D_EINVAL, "scale_codebook_embeddings and tie_word_embeddings must be true");
    if (b[1]) return set_err(h, S2D_EINVAL, "fast.attention_qk_norm must be false");
    S2dGraphSpec &s = h->spec;
    s.context_length = (int)u[0];
    s.hidden = (int)u[1];
    s.ffn = (int)u[2];
    s.slow_layers = (int)u[3];
    s.heads = (int)u[4];
    s.kv_heads = (int)u[5];
    s.rope_base = f[0];
    s.rms_eps = f[1];
    s.fast_context_length = (int)u[6];
    s.fast_ffn = (int)u[8];
    s.fast_layers = (int)u[9];
    s.fast_heads = (int)u[10];
    s.fast_kv_heads = (int)u[11];
    s.fast_head_dim = (int)u[12];
    s.fast_rope_base = f[2];
    s.fast_rms_eps = f[3];
    s.codebook_size = (int)u[13];
    s.num_codebooks = (int)u[14];
    s.semantic_begin_id = (int)u[15];
    s.semantic_end_id = (int)u[16];
    if (u[7] != u[1])
        return set_err(h, S2D_EINVAL, "slow hidden size mismatch: fast embedding_length != slow (fast_ar.rs:380-387)");
    if (!b[0]) {
        s.head_dim = s.heads ? s.hidden / s.heads : 0;
    } else {
        const GgufTensor *qn = g.tensor("layers.0.attention.q_norm.weight");
        if (!qn || qn->dims.size() != 1) return set_err(h, S2D_EIO, "missing layers.0.attention.q_norm.weight");
        s.head_dim = (int)qn->dims[0];
    }
    if (s.kv_heads <= 0 || s.heads % s.kv_heads || s.fast_kv_heads <= 0 || s.fast_heads % s.fast_kv_heads)
        return set_err(h, S2D_EINVAL, "invalid GQA head split");
    if (s.head_dim % 64 || s.head_dim > 256 || s.fast_head_dim % 64 || s.fast_head_dim > 256)
        return set_err(h, S2D_EINVAL, "head_dim must be a multiple of 64 and <= 256");
    if (s.heads / s.kv_heads > 16 || s.fast_heads / s.fast_kv_heads > 16)
        return set_err(h, S2D_EINVAL, "GQA group larger than 16 heads");
    if (s.num_codebooks < 1 || s.fast_context_length < s.num_codebooks)
        return set_err(h, S2D_EINVAL, "fast_context_length must cover num_codebooks");
    h->slow = ArShape{s.slow_layers, s.hidden, s.ffn, s.heads, s.kv_heads, s.head_dim,
                      s.context_length, s.rope_base, s.rms_eps, b[0]};
    h->fast = ArShape{s.fast_layers, s.hidden, s.fast_ffn, s.fast_heads, s.fast_kv_heads,
                      s.fast_head_dim, s.fast_context_length, s.fast_rope_base, s.fast_rms_eps, false};
    return S2D_OK;
}

const GgufTensor *need(S2dHandle *h, const std::string &name, std::vector<uint64_t> dims, int *rc) {
    const GgufTensor *t = h->gguf.tensor(name);
    if (!t) {
        *rc = set_err(h, S2D_EIO, "missing " + name);
        return nullptr;
    }
    if (t->dims != dims) {
        std::string want, got;
        for (auto d : dims) want += std::to_string(d) + ",";
        for (auto d : t->dims) got += std::to_string(d) + ",";
        *rc = set_err(h, S2D_EINVAL, name + " dimensions mismatch: expected [" + want + "] got [" + got + "]");
        return nullptr;
    }
    return t;
}

int32_t upload_all(S2dHandle *h) {
    // one arena for every tensor, each 256-byte aligned
    size_t total = 0;
    for (const auto &t : h->gguf.tensors) total += align256((size_t)t.bytes);
    CK(cudaMalloc(&h->arena, total ? total : 256));
    const size_t CH = 64u << 20;
    uint8_t *stage[2] = {nullptr, nullptr};
    cudaEvent_t done_ev[2] = {nullptr, nullptr};
    CK(cudaMallocHost(&stage[0], CH));
    CK(cudaMallocHost(&stage[1], CH));
    CK(cudaEventCreateWithFlags(&done_ev[0], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&done_ev[1], cudaEventDisableTiming));
    h->tensors.resize(h->gguf.tensors.size());
    size_t off = 0;
    int slot = 0;
    bool used[2] = {false, false};
    for (size_t i = 0; i < h->gguf.tensors.size(); ++i) {
        const GgufTensor &t = h->gguf.tensors[i];
        h->tensors[i].info = &t;
        h->tensors[i].dev = h->arena + off;
        for (size_t b = 0; b < t.bytes; b += CH) {
            const size_t n = std::min<size_t>(CH, (size_t)t.bytes - b);
            if (used[slot]) CK(cudaEventSynchronize(done_ev[slot]));
            memcpy(stage[slot], t.data + b, n);
            CK(cudaMemcpyAsync(h->arena + off + b, stage[slot], n, cudaMemcpyHostToDevice, h->stream));
            CK(cudaEventRecord(done_ev[slot], h->stream));
            used[slot] = true;
            slot ^= 1;
        }
        off += align256((size_t)t.bytes);
    }
    CK(cudaStreamSynchronize(h->stream));
    cudaFreeHost(stage[0]);
    cudaFreeHost(stage[1]);
    cudaEventDestroy(done_ev[0]);
    cudaEventDestroy(done_ev[1]);
    return S2D_OK;
}

TensorDev *tdev(S2dHandle *h, const GgufTensor *t) {
    return &h->tensors[(size_t)(t - h->gguf.tensors.data())];
}

// TransformerTensorRegistry (registry.rs:346-496, 515-552, 625-650): bind and
// validate every required tensor.  Linear weights must be F16 in this
// version; norms F16 or F32.
int32_t bind_weights(S2dHandle *h) {
    int rc = S2D_OK;
    const S2dGraphSpec &s = h->spec;
    const uint64_t d = (uint64_t)s.hidden, K = (uint64_t)s.num_codebooks, cb = (uint64_t)s.codebook_size;
    const GgufTensor *emb = h->gguf.tensor("embeddings.weight");
    if (!emb || emb->dims.size() != 2 || emb->dims[0] != d)
        return set_err(h, S2D_EINVAL, "embeddings.weight expected [hidden, vocab]");
    s2d::GgufTensor const *ce = h->gguf.tensor("codebook_embeddings.weight");
    if (!ce || ce->dims.size() != 2 || ce->dims[0] != d)
        return set_err(h, S2D_EINVAL, "codebook_embeddings.weight shape mismatch");
    h->spec.vocab_size = (int)emb->dims[1];
    h->spec.codebook_rows = (int)ce->dims[1];
    const GgufTensor *fe = need(h, "fast_embeddings.weight", {d, cb}, &rc);
    const GgufTensor *fo = need(h, "fast_output.weight", {d, cb}, &rc);
    const GgufTensor *nw = need(h, "norm.weight", {d}, &rc);
    const GgufTensor *fnw = need(h, "fast_norm.weight", {d}, &rc);
    if (rc) return rc;
    if (emb->type != 1 || ce->type != 1 || fe->type != 1)
        return set_err(h, S2D_EINVAL, "embedding tables must be F16");
    if ((uint64_t)s.codebook_rows < K * cb)
        return set_err(h, S2D_EINVAL, "codebook_embeddings.weight has fewer than num_codebooks*codebook_size rows");
    if (s.semantic_end_id < s.semantic_begin_id || s.semantic_end_id >= s.vocab_size)
        return set_err(h, S2D_EINVAL, "semantic id range outside the vocabulary");
    if (s.semantic_end_id - s.semantic_begin_id + 1 > kSampleMax - 1)
        return set_err(h, S2D_EINVAL, "semantic range larger than the device sampler supports");
    if (s.codebook_size > kSampleMax) return set_err(h, S2D_EINVAL, "codebook_size larger than the device sampler supports");

    // norms: expanded to f32 once
    std::vector<std::pair<const GgufTensor *, float **>> norms;
    h->slow_layers.resize((size_t)s.slow_layers);
    h->fast_layers.resize((size_t)s.fast_layers);
    uint32_t linear_type = 0;
    // F16, Q8_0 or Q4_K; the five linears of a layer share one format
    auto linear = [&](const std::string &name, LayerDev &L, bool first, uint64_t in,
                      uint64_t out) -> const uint16_t * {
        const GgufTensor *t = need(h, name, {in, out}, &rc);
        if (!t) return nullptr;
        const int wq = engine_weight_format((int)t->type);
        if (wq < 0 || (wq == EW_Q8_0 && in % 32) || (wq == EW_Q4_K && in % 256)) {
            rc = set_err(h, S2D_EINVAL, name + ": linear weights must be F16, Q8_0 or Q4_K (rows of whole blocks)");
            return nullptr;
        }
        if (first) L.wq = wq;
        else if (L.wq != wq) {
            rc = set_err(h, S2D_EINVAL, name + ": the linears of a layer must share one type");
            return nullptr;
        }
        linear_type = t->type;
        return reinterpret_cast<const uint16_t *>(tdev(h, t)->dev);
    };
    for (int l = 0; l < s.slow_layers && !rc; ++l) {
        const ArShape &a = h->slow;
        const std::string p = "layers." + std::to_string(l) + ".";
        LayerDev &L = h->slow_layers[(size_t)l];
        L.wqkv = linear(p + "attention.wqkv.weight", L, true, d, (uint64_t)a.qkv_out());
        L.wo = linear(p + "attention.wo.weight", L, false, (uint64_t)a.qs(), d);
        L.w1 = linear(p + "feed_forward.w1.weight", L, false, d, (uint64_t)a.F);
        L.w2 = linear(p + "feed_forward.w2.weight", L, false, (uint64_t)a.F, d);
        L.w3 = linear(p + "feed_forward.w3.weight", L, false, d, (uint64_t)a.F);
        const GgufTensor *an = need(h, p + "attention_norm.weight", {d}, &rc);
        const GgufTensor *fn = need(h, p + "ffn_norm.weight", {d}, &rc);
        const GgufTensor *qn = need(h, p + "attention.q_norm.weight", {(uint64_t)a.hd}, &rc);
        const GgufTensor *kn = need(h, p + "attention.k_norm.weight", {(uint64_t)a.hd}, &rc);
        if (rc) break;
        norms.push_back({an, &L.attn_norm});
        norms.push_back({fn, &L.ffn_norm});
        norms.push_back({qn, &L.q_norm});
        norms.push_back({kn, &L.k_norm});
    }
    for (int l = 0; l < s.fast_layers && !rc; ++l) {
        const ArShape &a = h->fast;
        const std::string p = "fast_layers." + std::to_string(l) + ".";
        LayerDev &L = h->fast_layers[(size_t)l];
        L.wqkv = linear(p + "attention.wqkv.weight", L, true, d, (uint64_t)a.qkv_out());
        L.wo = linear(p + "attention.wo.weight", L, false, (uint64_t)a.qs(), d);
        L.w1 = linear(p + "feed_forward.w1.weight", L, false, d, (uint64_t)a.F);
        L.w2 = linear(p + "feed_forward.w2.weight", L, false, (uint64_t)a.F, d);
        L.w3 = linear(p + "feed_forward.w3.weight", L, false, d, (uint64_t)a.F);
        const GgufTensor *an = need(h, p + "attention_norm.weight", {d}, &rc);
        const GgufTensor *fn = need(h, p + "ffn_norm.weight", {d}, &rc);
        if (rc) break;
        norms.push_back({an, &L.attn_norm});
        norms.push_back({fn, &L.ffn_norm});
    }
    if (rc) return rc;
    h->fast_out = reinterpret_cast<const uint16_t *>(tdev(h, fo)->dev);
    h->fast_out_wq = engine_weight_format((int)fo->type);
    if (h->fast_out_wq < 0 || (h->fast_out_wq == EW_Q8_0 && s.hidden % 32) || (h->fast_out_wq == EW_Q4_K && s.hidden % 256))
        return set_err(h, S2D_EINVAL, "fast_output.weight must be F16, Q8_0 or Q4_K");
    norms.push_back({nw, &h->norm});
    norms.push_back({fnw, &h->fast_norm});
    h->emb = reinterpret_cast<const uint16_t *>(tdev(h, emb)->dev);
    h->cb_emb = reinterpret_cast<const uint16_t *>(tdev(h, ce)->dev);
    h->fast_emb = reinterpret_cast<const uint16_t *>(tdev(h, fe)->dev);
    h->spec.linear_type = (int)linear_type;
    size_t nfloats = 0;
    for (auto &pr : norms) nfloats += (size_t)(pr.first->elements + 63) / 64 * 64;
    CK(cudaMalloc(&h->norm_arena, nfloats * sizeof(float)));
    size_t off = 0;
    for (auto &pr : norms) {
        const GgufTensor *t = pr.first;
        float *dst = h->norm_arena + off;
        if (t->type == 1) CK(launch_f16_to_f32(reinterpret_cast<const uint16_t *>(tdev(h, t)->dev), dst, (int64_t)t->elements, h->stream));
        else if (t->type == 0) CK(cudaMemcpyAsync(dst, tdev(h, t)->dev, t->elements * 4, cudaMemcpyDeviceToDevice, h->stream));
        else return set_err(h, S2D_EINVAL, t->name + ": norm weights must be F16 or F32");
        *pr.second = dst;
        off += (size_t)(t->elements + 63) / 64 * 64;
    }
    return S2D_OK;
}

// Bytes of `cols` consecutive values of a row in ggml type `gtype`
// (F16, Q8_0 blocks of 32, Q4_K superblocks of 256).
size_t ggml_row_bytes(int gtype, int64_t cols) {
    if (gtype == 8) return (size_t)cols / 32 * 34;
    if (gtype == 12) return (size_t)cols / 256 * 144;
    return (size_t)cols * 2;
}

// This rank's shard of the Slow-AR (tp_plan): rank r of n takes query heads
// [r*H/n, (r+1)*H/n) with their KV heads and the FFN columns of units
// [r*U/n, (r+1)*U/n), a unit being the block width of the weight type (8
// for F16, 32 for Q8_0, 256 for Q4_K) so that w2's column slices are whole
// blocks; a Q4_K FFN may split unevenly.
int32_t tp_plan(const S2dGraphSpec &s, int n, int r, S2dTpShard *out) {
    if (n < 1 || r < 0 || r >= n) return S2D_EINVAL;
    if (s.heads % n || s.kv_heads % n) return S2D_EINVAL;
    const int unit = s.linear_type == 8 ? 32 : s.linear_type == 12 ? 256 : 8;
    if (s.ffn % unit || (s.heads / n * s.head_dim) % unit) return S2D_EINVAL;
    const int units = s.ffn / unit;
    if (units < n) return S2D_EINVAL;
    S2dTpShard t{};
    t.heads = s.heads / n, t.kv_heads = s.kv_heads / n;
    t.head0 = r * t.heads, t.kv_head0 = r * t.kv_heads;
    t.ffn0 = (int32_t)((int64_t)r * units / n) * unit;
    t.ffn = (int32_t)((int64_t)(r + 1) * units / n) * unit - t.ffn0;
    *out = t;
    return S2D_OK;
}

// Copy this rank's shard of every Slow-AR linear out of the file-layout
// arena (rows of wqkv / w1 / w3, column slices of wo / w2) and narrow the
// Slow-AR shape to it.
int32_t shard_slow_weights(S2dHandle *h) {
    const S2dGraphSpec &s = h->spec;
    int32_t rc;
    if ((rc = tp_plan(s, h->tp, h->tp_rank, &h->shard)))
        return set_err(h, rc, "no tensor-parallel split of this model over " + std::to_string(h->tp) +
                                  " ranks (heads, kv heads and the FFN must divide into whole blocks)");
    const S2dTpShard &t = h->shard;
    const int gt = s.linear_type, hd = s.head_dim;
    const int64_t d = s.hidden, qs = (int64_t)s.heads * hd, kvs = (int64_t)s.kv_heads * hd;
    const int64_t qs_r = (int64_t)t.heads * hd, kvs_r = (int64_t)t.kv_heads * hd, F_r = t.ffn;
    const size_t rd = ggml_row_bytes(gt, d);
    const size_t b_qkv = (size_t)(qs_r + 2 * kvs_r) * rd, b_wo = (size_t)d * ggml_row_bytes(gt, qs_r);
    const size_t b_w13 = (size_t)F_r * rd, b_w2 = (size_t)d * ggml_row_bytes(gt, F_r);
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t per_layer = al(b_qkv) + al(b_wo) + 2 * al(b_w13) + al(b_w2);
    CK(cudaMalloc(&h->shard_arena, per_layer * (size_t)s.slow_layers));
    for (int l = 0; l < s.slow_layers; ++l) {
        LayerDev &L = h->slow_layers[(size_t)l];
        uint8_t *p = h->shard_arena + per_layer * (size_t)l;
        uint8_t *qkv = p, *wo = qkv + al(b_qkv), *w1 = wo + al(b_wo), *w3 = w1 + al(b_w13), *w2 = w3 + al(b_w13);
        const uint8_t *src = reinterpret_cast<const uint8_t *>(L.wqkv);
        // [Q heads | K heads | V heads] of this rank, rows of d values
        CK(cudaMemcpyAsync(qkv, src + (size_t)t.head0 * hd * rd, (size_t)qs_r * rd, cudaMemcpyDeviceToDevice, h->stream));
        CK(cudaMemcpyAsync(qkv + (size_t)qs_r * rd, src + (size_t)(qs + (int64_t)t.kv_head0 * hd) * rd,
                           (size_t)kvs_r * rd, cudaMemcpyDeviceToDevice, h->stream));
        CK(cudaMemcpyAsync(qkv + (size_t)(qs_r + kvs_r) * rd, src + (size_t)(qs + kvs + (int64_t)t.kv_head0 * hd) * rd,
                           (size_t)kvs_r * rd, cudaMemcpyDeviceToDevice, h->stream));
        // wo and w2: d rows, this rank's input columns
        CK(cudaMemcpy2DAsync(wo, ggml_row_bytes(gt, qs_r),
                             reinterpret_cast<const uint8_t *>(L.wo) + ggml_row_bytes(gt, (int64_t)t.head0 * hd),
                             ggml_row_bytes(gt, qs), ggml_row_bytes(gt, qs_r), (size_t)d, cudaMemcpyDeviceToDevice,
                             h->stream));
        CK(cudaMemcpy2DAsync(w2, ggml_row_bytes(gt, F_r), reinterpret_cast<const uint8_t *>(L.w2) + ggml_row_bytes(gt, t.ffn0),
                             ggml_row_bytes(gt, s.ffn), ggml_row_bytes(gt, F_r), (size_t)d, cudaMemcpyDeviceToDevice,
                             h->stream));
        // w1 and w3: this rank's FFN rows
        CK(cudaMemcpyAsync(w1, reinterpret_cast<const uint8_t *>(L.w1) + (size_t)t.ffn0 * rd, b_w13,
                           cudaMemcpyDeviceToDevice, h->stream));
        CK(cudaMemcpyAsync(w3, reinterpret_cast<const uint8_t *>(L.w3) + (size_t)t.ffn0 * rd, b_w13,
                           cudaMemcpyDeviceToDevice, h->stream));
        L.wqkv = reinterpret_cast<const uint16_t *>(qkv), L.wo = reinterpret_cast<const uint16_t *>(wo);
        L.w1 = reinterpret_cast<const uint16_t *>(w1), L.w3 = reinterpret_cast<const uint16_t *>(w3);
        L.w2 = reinterpret_cast<const uint16_t *>(w2);
    }
    h->slow.H = t.heads, h->slow.Hkv = t.kv_heads, h->slow.F = t.ffn;
    return S2D_OK;
}

// NCCL, loaded on first use (tensor parallelism only): dlopen of
// S2D_NCCL_LIB, else libnccl.so.2, which is the copy already in the process
// when one is (a framework's), so that loading this library never puts a
// second NCCL beside it.
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclApi &nccl() {
    static NcclApi api = [] {
        NcclApi a;
        const char *env = getenv("S2D_NCCL_LIB");
        void *lib = dlopen(env && env[0] ? env : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) return a;
        a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(lib, "ncclGetUniqueId"));
        a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(lib, "ncclCommInitRank"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(lib, "ncclAllReduce"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(lib, "ncclAllGather"));
        a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(lib, "ncclCommDestroy"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(lib, "ncclGetErrorString"));
        a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.all_gather && a.comm_destroy &&
               a.error_string;
        return a;
    }();
    return api;
}

// The Slow-AR residual exchange of tensor parallelism: every rank's
// wo / w2 output over its input columns, summed in place (rank 0's carries
// the residual, the others' only their partial sums).
cudaError_t tp_allreduce(S2dHandle *h, float *x, size_t n) {
    if (h->tp <= 1) return cudaSuccess;
    const ncclResult_t r = nccl().all_reduce(x, x, n, ncclFloat32, ncclSum, h->comm, h->stream);
    return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

// The residual exchange of tensor parallelism inside the persistent engine.
// Each rank's exchange buffer holds, for every wo and w2 op of the Slow-AR
// step program (2 per layer), one row of d LL words per rank: [op][rank][d].
// Every rank maps every other rank's buffer (CUDA IPC handles, gathered over
// NCCL), so that its engine writes its partial sums straight into the peers'
// buffers over NVLink with plain stores, and every rank sums the rows of an
// op in rank order: the ranks see bit-identical residuals.  Plain peer
// stores and local loads only: no bulk or tensor copies touch peer memory.
int32_t setup_exchange(S2dHandle *h) {
    if (h->tp <= 1 || h->tp > kEngineMaxPeers) return S2D_OK;
    const size_t words = (size_t)2 * h->slow.L * h->tp * h->spec.hidden;
    CK(cudaMalloc(&h->xchg, words * sizeof(uint64_t)));
    CK(cudaMemset(h->xchg, 0, words * sizeof(uint64_t)));
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, h->xchg));
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    uint8_t *dbuf = nullptr;
    CK(cudaMalloc(&dbuf, hb * (size_t)h->tp));
    CK(cudaMemcpy(dbuf + hb * (size_t)h->tp_rank, &mine, hb, cudaMemcpyHostToDevice));
    const ncclResult_t nr = nccl().all_gather(dbuf + hb * (size_t)h->tp_rank, dbuf, hb, ncclUint8, h->comm, h->stream);
    std::vector<cudaIpcMemHandle_t> all((size_t)h->tp);
    cudaError_t e = nr == ncclSuccess ? cudaStreamSynchronize(h->stream) : cudaErrorUnknown;
    if (!e) e = cudaMemcpy(all.data(), dbuf, hb * (size_t)h->tp, cudaMemcpyDeviceToHost);
    cudaFree(dbuf);
    if (nr != ncclSuccess) return set_err(h, S2D_ECUDA, std::string("ncclAllGather: ") + nccl().error_string(nr));
    CK(e);
    for (int q = 0; q < h->tp; ++q) {
        if (q == h->tp_rank) {
            h->xchg_peer[q] = h->xchg;
            continue;
        }
        void *p = nullptr;
        CK(cudaIpcOpenMemHandle(&p, all[(size_t)q], cudaIpcMemLazyEnablePeerAccess));
        h->xchg_peer[q] = static_cast<uint64_t *>(p);
    }
    h->xchg_words = words;
    return S2D_OK;
}

int32_t alloc_buffers(S2dHandle *h) {
    const S2dGraphSpec &s = h->spec;
    const ArShape &a = h->slow, &f = h->fast;
    const int maxseq = h->cfg.max_seq;
    // RoPE denominators rope_base^(pair/hd), computed with the host libm powf
    // exactly as apply_rope_normal does (attention.rs:196-197).
    std::vector<float> rs((size_t)a.hd / 2), rf((size_t)f.hd / 2);
    for (int p = 0; p < a.hd; p += 2) rs[(size_t)p / 2] = powf(a.rope_base, (float)p / (float)a.hd);
    for (int p = 0; p < f.hd; p += 2) rf[(size_t)p / 2] = powf(f.rope_base, (float)p / (float)f.hd);
    CK(cudaMalloc(&h->rope_slow, rs.size() * sizeof(float)));
    CK(cudaMalloc(&h->rope_fast, rf.size() * sizeof(float)));
    CK(cudaMemcpy(h->rope_slow, rs.data(), rs.size() * sizeof(float), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(h->rope_fast, rf.data(), rf.size() * sizeof(float), cudaMemcpyHostToDevice));
    // (cos, sin) of theta = pos / denominator for every position, theta in
    // f32 as above, sin and cos rounded from double
    auto rope_table = [](const std::vector<float> &den, int npos) {
        std::vector<float2> t((size_t)npos * den.size());
        for (int p = 0; p < npos; ++p)
            for (size_t i = 0; i < den.size(); ++i) {
                const float theta = (float)p / den[i];
                t[(size_t)p * den.size() + i] = make_float2((float)cos((double)theta), (float)sin((double)theta));
            }
        return t;
    };
    {
        const std::vector<float2> ts = rope_table(rs, maxseq), tf = rope_table(rf, f.ctx);
        CK(cudaMalloc(&h->rope_cs_slow, std::max<size_t>(ts.size(), 1) * sizeof(float2)));
        CK(cudaMalloc(&h->rope_cs_fast, std::max<size_t>(tf.size(), 1) * sizeof(float2)));
        CK(cudaMemcpy(h->rope_cs_slow, ts.data(), ts.size() * sizeof(float2), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(h->rope_cs_fast, tf.data(), tf.size() * sizeof(float2), cudaMemcpyHostToDevice));
    }
    h->kv_slow_seq = (size_t)a.L * 2 * a.Hkv * maxseq * a.hd;
    const size_t kv_slow = h->kv_slow_seq;
    CK(cudaMalloc(&h->kv_slow, kv_slow * sizeof(__half)));
    CK(cudaMemset(h->kv_slow, 0, kv_slow * sizeof(__half)));
    const size_t kv_fast = (size_t)f.L * 2 * f.Hkv * f.ctx * f.hd;
    CK(cudaMalloc(&h->kv_fast, std::max<size_t>(kv_fast, 1) * sizeof(float)));
    CK(cudaMemset(h->kv_fast, 0, std::max<size_t>(kv_fast, 1) * sizeof(float)));
    const int d = s.hidden;
    const int qkv_out = std::max(a.qkv_out(), f.qkv_out());
    const int qs = std::max(a.qs(), f.qs());
    const int F = std::max(a.F, f.F);
    CK(cudaMalloc(&h->x, (size_t)kMaxM * d * sizeof(float)));
    CK(cudaMalloc(&h->qkv, (size_t)kMaxM * qkv_out * sizeof(float)));
    CK(cudaMalloc(&h->q, (size_t)kMaxM * qs * sizeof(float)));
    CK(cudaMalloc(&h->att, (size_t)kMaxM * qs * sizeof(float)));
    CK(cudaMalloc(&h->act, (size_t)kMaxM * F * sizeof(float)));
    CK(cudaMalloc(&h->fast_x, (size_t)(f.ctx + 1) * d * sizeof(float)));
    CK(cudaMalloc(&h->hidden_post, (size_t)d * sizeof(float)));
    CK(cudaMalloc(&h->logits, (size_t)s.vocab_size * sizeof(float)));
    CK(cudaMalloc(&h->logits_fast, (size_t)std::max(s.codebook_size, kSampleMax) * sizeof(float)));
    // attention split count: ~64 positions per split at full context
    // attention splits: enough items to cover the SMs, ~32 positions per split at full context
    h->S_slow = std::min(128, std::max(32, (maxseq + 31) / 32));
    h->S_fast = 1;
    const int H = std::max(a.H, f.H), hd = std::max(a.hd, f.hd), Hkv = std::max(a.Hkv, f.Hkv);
    CK(cudaMalloc(&h->part, (size_t)kMaxM * H * h->S_slow * (hd + 2) * sizeof(float)));
    CK(cudaMalloc(&h->counters, (size_t)kMaxM * Hkv * sizeof(int32_t)));
    // engine LL words (at most 2 tokens per engine op); zero words carry tag 0,
    // which no launch uses (epochs start at 1)
    {
        const size_t nx = (size_t)2 * d, nq = (size_t)2 * qkv_out, na = (size_t)2 * qs, nf = (size_t)2 * F;
        const size_t np = (size_t)2 * H * h->S_slow * (hd + 2);
        uint64_t **bufs[] = {&h->ll_x, &h->ll_qkv, &h->ll_att, &h->ll_act, &h->ll_part};
        const size_t ns[] = {nx, nq, na, nf, np};
        for (int i = 0; i < 5; ++i) {
            CK(cudaMalloc(bufs[i], ns[i] * sizeof(uint64_t)));
            CK(cudaMemset(*bufs[i], 0, ns[i] * sizeof(uint64_t)));
        }
        {
            const int K = std::max(s.num_codebooks, 1);
            const size_t nq = (size_t)std::max(K - 1, 1) * f.L * 2 * f.qkv_out();
            const size_t nl = (size_t)std::max(s.codebook_size, 2), nxr = (size_t)K * f.d;
            uint64_t **fb[] = {&h->fr_qkv, &h->fr_logits, &h->fr_x};
            const size_t fn[] = {nq, nl, nxr};
            for (int i = 0; i < 3; ++i) {
                CK(cudaMalloc(fb[i], fn[i] * sizeof(uint64_t)));
                CK(cudaMemset(*fb[i], 0, fn[i] * sizeof(uint64_t)));
            }
        }
        const uint32_t one = 1;
        CK(cudaMalloc(&h->engine_epoch, sizeof(uint32_t)));
        CK(cudaMemcpy(h->engine_epoch, &one, sizeof(uint32_t), cudaMemcpyHostToDevice));
    }
    CK(cudaMemset(h->counters, 0, (size_t)kMaxM * Hkv * sizeof(int32_t)));
    CK(cudaMalloc(&h->st, sizeof(DevState)));
    CK(cudaMemset(h->st, 0, sizeof(DevState)));
    CK(cudaMalloc(&h->frame_codes, (size_t)std::max(s.num_codebooks, 1) * sizeof(int32_t)));
    CK(cudaMalloc(&h->tok_out, sizeof(uint32_t)));
    CK(cudaMalloc(&h->code_override, sizeof(uint32_t)));
    return S2D_OK;
}

int32_t ensure_tokens(S2dHandle *h, size_t n) {
    if (n <= h->tokens_cap) return S2D_OK;
    if (h->tokens_dev) cudaFree(h->tokens_dev);
    h->tokens_dev = nullptr;
    h->tokens_cap = 0;
    CK(cudaMalloc(&h->tokens_dev, n * sizeof(int32_t)));
    h->tokens_cap = n;
    return S2D_OK;
}

// ---------------------------------------------------------------------------
// layer sequences
// ---------------------------------------------------------------------------

// One transformer layer over M consecutive tokens at rows x[0..M) of width d:
// SlowArLayerSkeleton::forward_decode_token_with_backend +
// forward_feed_forward_with_backend (slow_ar.rs:637-710) for the Slow-AR,
// FastArLayerSkeleton::forward_prefill for the Fast-AR (fast_ar.rs:245-352).
cudaError_t enqueue_layer(S2dHandle *h, bool is_fast, int l, float *x, int M,
                          const int32_t *pos_dev, int pos_const, const int32_t *done) {
    const ArShape &a = is_fast ? h->fast : h->slow;
    const LayerDev &L = is_fast ? h->fast_layers[(size_t)l] : h->slow_layers[(size_t)l];
    const int d = a.d;
    cudaError_t e;
    GemvArgs g{};
    g.done = done;
    g.n_contig = -1;
    // attention_norm + WQKV
    g.W = L.wqkv, g.x = x, g.ldx = d, g.norm_w = L.attn_norm, g.eps = a.eps;
    g.y = h->qkv, g.ldy = a.qkv_out(), g.K = d, g.N = a.qkv_out(), g.wq = L.wq;
    if ((e = launch_gemv(g, M, EPI_STORE, h->stream, h->pdl))) return e;
    // QK-norm + RoPE + KV write
    RopeArgs r{};
    r.qkv = h->qkv, r.ld_qkv = a.qkv_out(), r.q_out = h->q;
    if (is_fast) {
        float *base = h->kv_fast + (size_t)l * 2 * a.Hkv * a.ctx * a.hd;
        r.kcache = base, r.vcache = base + (size_t)a.Hkv * a.ctx * a.hd, r.max_seq = a.ctx;
        r.rope_denom = h->rope_fast;
    } else {
        __half *base = h->kv_slow + (size_t)l * 2 * a.Hkv * h->cfg.max_seq * a.hd;
        r.kcache = base, r.vcache = base + (size_t)a.Hkv * h->cfg.max_seq * a.hd, r.max_seq = h->cfg.max_seq;
        r.q_norm = L.q_norm, r.k_norm = L.k_norm, r.rope_denom = h->rope_slow;
    }
    r.eps = a.eps, r.pos_dev = pos_dev, r.pos_const = pos_const;
    r.H = a.H, r.Hkv = a.Hkv, r.hd = a.hd, r.M = M, r.done = done, r.error = &h->st->error;
    if ((e = launch_rope_kv(r, !is_fast, h->stream, h->pdl))) return e;
    // GQA attention
    AttnArgs t{};
    t.q = h->q, t.kcache = r.kcache, t.vcache = r.vcache, t.max_seq = r.max_seq, t.out = h->att;
    t.part = h->part, t.counters = h->counters, t.pos_dev = pos_dev, t.pos_const = pos_const;
    t.H = a.H, t.Hkv = a.Hkv, t.hd = a.hd, t.S = is_fast ? h->S_fast : h->S_slow, t.M = M;
    t.scale = 1.0f / sqrtf((float)a.hd);  // SlowArLayerShape::attn_scale (slow_ar.rs:59-61)
    t.done = done;
    if ((e = launch_attention(t, !is_fast, h->stream, h->pdl))) return e;
    // wo + residual
    g = GemvArgs{};
    g.done = done, g.n_contig = -1;
    g.W = L.wo, g.x = h->att, g.ldx = a.qs(), g.y = x, g.ldy = d, g.resid = x, g.ldr = d;
    g.K = a.qs(), g.N = d, g.wq = L.wq;
    // tensor parallel: rank 0 adds the residual, every rank's partial sums
    // are then summed in place
    const bool part = !is_fast && h->tp > 1;
    const int resid_epi = part && h->tp_rank != 0 ? EPI_STORE : EPI_RESID;
    if ((e = launch_gemv(g, M, resid_epi, h->stream, h->pdl))) return e;
    if (part && (e = tp_allreduce(h, x, (size_t)M * d))) return e;
    // ffn_norm + w1/w3 + SwiGLU
    g = GemvArgs{};
    g.done = done, g.n_contig = -1;
    g.W = L.w1, g.W2 = L.w3, g.x = x, g.ldx = d, g.norm_w = L.ffn_norm, g.eps = a.eps;
    g.y = h->act, g.ldy = a.F, g.K = d, g.N = a.F, g.wq = L.wq;
    if ((e = launch_gemv(g, M, is_fast ? EPI_SWIGLU_FAST : EPI_SWIGLU_SLOW, h->stream, h->pdl))) return e;
    // w2 + residual
    g = GemvArgs{};
    g.done = done, g.n_contig = -1;
    g.W = L.w2, g.x = h->act, g.ldx = a.F, g.y = x, g.ldy = d, g.resid = x, g.ldr = d;
    g.K = a.F, g.N = d, g.wq = L.wq;
    h->launches += 6;
    if ((e = launch_gemv(g, M, resid_epi, h->stream, h->pdl))) return e;
    return part ? tp_allreduce(h, x, (size_t)M * d) : cudaSuccess;
}

// Final norm + tied LM head (SlowArOutputHeadF16Weights::forward_logits,
// slow_ar.rs:943-955) on the row `xrow`; writes the post-norm hidden.
// full: every vocabulary row; otherwise the semantic rows + im_end only.
cudaError_t enqueue_lm_head(S2dHandle *h, const float *xrow, bool full, uint32_t im_end,
                            const int32_t *done) {
    const S2dGraphSpec &s = h->spec;
    GemvArgs g{};
    g.done = done;
    g.W = h->emb, g.x = xrow, g.ldx = s.hidden, g.norm_w = h->norm, g.eps = h->slow.eps;
    g.y = h->logits, g.ldy = s.vocab_size, g.x_out = h->hidden_post, g.K = s.hidden;
    if (full) {
        g.n_contig = -1;
        g.N = s.vocab_size;
    } else {
        const int nsem = s.semantic_end_id - s.semantic_begin_id + 1;
        const bool extra = (int64_t)im_end < s.vocab_size &&
                           ((int)im_end < s.semantic_begin_id || (int)im_end > s.semantic_end_id);
        g.row_base = s.semantic_begin_id;
        g.n_contig = nsem;
        g.extra_row = extra ? (int)im_end : s.semantic_begin_id;
        g.N = nsem + (extra ? 1 : 0);
        h->n_allowed_extra = extra ? 1 : 0;
    }
    h->launches += 1;
    return launch_gemv(g, 1, EPI_STORE, h->stream, h->pdl);
}

cudaError_t enqueue_fast_head(S2dHandle *h, const float *xrow, const int32_t *done) {
    GemvArgs g{};
    g.done = done, g.n_contig = -1;
    g.W = h->fast_out, g.x = xrow, g.ldx = h->fast.d, g.norm_w = h->fast_norm, g.eps = h->fast.eps;
    g.y = h->logits_fast, g.ldy = h->spec.codebook_size, g.K = h->fast.d, g.N = h->spec.codebook_size;
    g.wq = h->fast_out_wq;
    h->launches += 1;
    return launch_gemv(g, 1, EPI_STORE, h->stream, h->pdl);
}

SampleArgs slow_sample_args(S2dHandle *h, int mode, const GenKey &k) {
    const S2dGraphSpec &s = h->spec;
    SampleArgs a{};
    a.logits = h->logits;
    const int nsem = s.semantic_end_id - s.semantic_begin_id + 1;
    const bool extra = (int64_t)k.im_end < s.vocab_size &&
                       ((int)k.im_end < s.semantic_begin_id || (int)k.im_end > s.semantic_end_id);
    a.n = nsem + (extra ? 1 : 0);
    a.n_contig = nsem;
    a.id_base = (uint32_t)s.semantic_begin_id;
    a.extra_id = k.im_end;
    a.vocab_full = s.vocab_size;
    a.temperature = k.temperature, a.top_p = k.top_p, a.top_k = k.top_k;
    a.force_id = -1;
    a.mode = mode;
    a.im_end = k.im_end;
    a.min_tokens_before_end = k.min_tokens;
    a.max_new = (int)k.max_new;
    a.st = h->st;
    a.rng = &h->st->rng;
    a.out_token = h->tok_out;
    return a;
}

// Fast-AR codebooks 1..K-1 of one frame (generate_codebooks_for_semantic,
// fast_ar.rs:440-470), with a KV cache over the frame's positions instead
// of the reference's prefix recomputation (identical results: causal).
cudaError_t enqueue_fast_frame(S2dHandle *h, const GenKey &k, bool with_override) {
    const S2dGraphSpec &s = h->spec;
    const int d = s.hidden, K = s.num_codebooks;
    const int32_t *done = &h->st->done;
    cudaError_t e;
    FastInitArgs fi{};
    fi.st = h->st, fi.slow_hidden = h->hidden_post, fi.fast_emb = h->fast_emb, fi.fast_x = h->fast_x;
    fi.frame_codes = h->frame_codes, fi.codes_out = with_override ? nullptr : h->codes_out;
    fi.max_new = (int)k.max_new, fi.d = d, fi.cb_size = s.codebook_size;
    fi.sem_begin = (uint32_t)s.semantic_begin_id, fi.sem_end = (uint32_t)s.semantic_end_id;
    fi.code_override = with_override ? h->code_override : nullptr;
    h->launches += 1;
    if ((e = launch_fast_init(fi, h->stream, h->pdl))) return e;
    for (int cbk = 1; cbk < K; ++cbk) {
        // positions processed this pass: 0 and 1 on the first pass, then cbk
        const int p0 = cbk == 1 ? 0 : cbk;
        const int M = cbk == 1 ? 2 : 1;
        for (int l = 0; l < h->fast.L; ++l)
            if ((e = enqueue_layer(h, true, l, h->fast_x + (size_t)p0 * d, M, nullptr, p0, done))) return e;
        if ((e = enqueue_fast_head(h, h->fast_x + (size_t)cbk * d, done))) return e;
        SampleArgs a{};
        a.logits = h->logits_fast;
        a.n = s.codebook_size;
        a.n_contig = -1;
        a.vocab_full = s.codebook_size;
        a.temperature = k.temperature, a.top_p = k.top_p, a.top_k = k.top_k;
        a.force_id = -1;
        a.mode = SAMPLE_FAST;
        a.max_new = (int)k.max_new;
        a.st = h->st;
        a.rng = &h->st->rng;
        a.cb_index = cbk;
        a.frame_codes = h->frame_codes;
        a.codes_out = with_override ? nullptr : h->codes_out;
        a.fast_emb = h->fast_emb;
        a.fast_x_next = cbk + 1 < K ? h->fast_x + (size_t)(cbk + 1) * d : nullptr;
        a.d = d;
        a.out_token = h->tok_out;
        h->launches += 1;
        if ((e = launch_sample(a, h->stream, h->pdl))) return e;
    }
    return cudaSuccess;
}

// ---------------------------------------------------------------------------
// persistent layer engine programs
// ---------------------------------------------------------------------------

// Whether the engine supports this model's shapes (else the per-op kernels run).
bool engine_supported(const S2dHandle *h) {
    if (h->num_sms <= 0) return false;
    for (const ArShape *a : {&h->slow, &h->fast}) {
        const int rep = a->H / a->Hkv;
        if (rep > kEngineConsumerWarps || kEngineConsumerWarps % rep || (a->hd != 64 && a->hd != 128)) return false;
        if (a->d % 8 || a->qs() % 8 || a->F % 8) return false;
        if (a->d > kEngineMaxK || a->qs() > kEngineMaxK || a->F > kEngineMaxK) return false;  // staged inputs
        // every CTA must own rows of every linear: a CTA's outputs are what
        // orders its reads of a reused buffer before the buffer's next writer
        if (a->d < h->num_sms || a->qkv_out() < h->num_sms || a->F < h->num_sms) return false;
        if (a->L * 5 + 1 > kEngineMaxOps) return false;
    }
    const S2dGraphSpec &s = h->spec;
    return s.codebook_size >= h->num_sms && s.semantic_end_id - s.semantic_begin_id + 1 >= h->num_sms;
}

// A GEMV op reading x (floats when x_src < 0, else LL words of op x_src) and
// writing y (LL words when y_ll).
EngineOp gemv_op(int M, int epi, const uint16_t *W, const uint16_t *W2, const void *x, int ldx, int x_src,
                 const float *norm_w, float eps, void *y, int ldy, int y_ll, const void *resid, int resid_src,
                 int K, int N, int wt = EW_F16) {
    EngineOp o{};
    o.wt = wt;
    o.kind = OP_GEMV, o.epi = epi, o.M = M, o.W = W, o.W2 = W2, o.x = x, o.ldx = ldx, o.x_src = x_src;
    o.norm_w = norm_w, o.eps = eps, o.y = y, o.ldy = ldy, o.y_ll = y_ll, o.resid = resid, o.ldr = ldy;
    o.resid_src = resid_src, o.K = K, o.N = N, o.n_contig = -1;
    return o;
}

// The ops of one transformer layer over M tokens (see enqueue_layer for the
// per-op kernel version).  The residual stream enters as `x` (floats [M][d]
// when *x_src < 0, else the LL residual h->ll_x written by op *x_src) and
// leaves in h->ll_x, written by the op whose index is stored in *x_src.
void layer_ops(S2dHandle *h, bool is_fast, int l, const float *x_in, int M, const int32_t *pos_dev,
               int pos_const, std::vector<EngineOp> &ops, int *x_src) {
    const ArShape &a = is_fast ? h->fast : h->slow;
    const LayerDev &L = is_fast ? h->fast_layers[(size_t)l] : h->slow_layers[(size_t)l];
    const int d = a.d;
    // Tensor parallelism (Slow-AR): wo and w2 leave partial sums over this
    // rank's heads / FFN columns, written into every rank's exchange buffer
    // (setup_exchange: region 2l for wo, 2l + 1 for w2); their readers sum the
    // ranks' rows in rank order.  Rank 0's partials carry the residual.
    const bool xt = !is_fast && h->tp > 1 && h->xchg;
    const int n = h->tp;
    const long long region = (long long)n * M * d;
    const void *x = *x_src < 0 ? static_cast<const void *>(x_in)
                    : xt       ? static_cast<const void *>(h->xchg + (size_t)(2 * l - 1) * region)
                               : static_cast<const void *>(h->ll_x);
    const int x_nsum = xt && *x_src >= 0 ? n : 1;
    auto summed = [&](EngineOp &o, int nsum) {  // o's input: the sum of nsum rank rows
        o.x_nsum = nsum, o.x_rstride = (long long)M * d;
    };
    auto to_peers = [&](EngineOp &o, int e) {  // o's outputs: exchange region e of every rank
        o.n_peer = n;
        for (int q = 0; q < n; ++q) o.y_peer[q] = h->xchg_peer[q] + (size_t)e * region + (size_t)h->tp_rank * M * d;
    };
    const int i_qkv = (int)ops.size();
    ops.push_back(gemv_op(M, EPI_STORE, L.wqkv, nullptr, x, d, *x_src, L.attn_norm, a.eps, h->ll_qkv, a.qkv_out(), 1,
                          nullptr, -1, d, a.qkv_out(), L.wq));
    EngineOp t{};
    t.kind = OP_ATTN, t.M = M, t.qkv = h->ll_qkv, t.ld_qkv = a.qkv_out(), t.qkv_src = i_qkv;
    if (is_fast) {
        float *base = h->kv_fast + (size_t)l * 2 * a.Hkv * a.ctx * a.hd;
        t.kcache = base, t.vcache = base + (size_t)a.Hkv * a.ctx * a.hd, t.max_seq = a.ctx, t.kv_half = 0;
        t.rope_cs = h->rope_cs_fast, t.S = h->S_fast;
    } else {
        __half *base = h->kv_slow + (size_t)l * 2 * a.Hkv * h->cfg.max_seq * a.hd;
        t.kcache = base, t.vcache = base + (size_t)a.Hkv * h->cfg.max_seq * a.hd;
        t.max_seq = h->cfg.max_seq, t.kv_half = 1;
        t.q_norm = L.q_norm, t.k_norm = L.k_norm, t.rope_cs = h->rope_cs_slow;
        t.S = h->engine_att_splits > 0 ? std::min(h->engine_att_splits, h->S_slow) : h->S_slow;
    }
    t.eps = a.eps, t.pos_dev = pos_dev, t.pos_const = pos_const;
    t.H = a.H, t.Hkv = a.Hkv, t.hd = a.hd, t.scale = 1.0f / sqrtf((float)a.hd);
    t.att_out = h->ll_att, t.part = h->ll_part;
    const int i_att = (int)ops.size();
    ops.push_back(t);
    if (xt) summed(ops[(size_t)i_qkv], x_nsum);
    const int i_wo = (int)ops.size();
    const int resid_epi = xt && h->tp_rank != 0 ? EPI_STORE : EPI_RESID;
    ops.push_back(gemv_op(M, resid_epi, L.wo, nullptr, h->ll_att, a.qs(), i_att, nullptr, 0.f, h->ll_x, d, 1, x,
                          *x_src, a.qs(), d, L.wq));
    if (xt) {
        ops.back().r_nsum = x_nsum, ops.back().r_rstride = (long long)M * d;
        to_peers(ops.back(), 2 * l);
    }
    const void *x_att = xt ? static_cast<const void *>(h->xchg + (size_t)(2 * l) * region)
                           : static_cast<const void *>(h->ll_x);
    const int i_w13 = (int)ops.size();
    ops.push_back(gemv_op(M, is_fast ? EPI_SWIGLU_FAST : EPI_SWIGLU_SLOW, L.w1, L.w3, x_att, d, i_wo, L.ffn_norm,
                          a.eps, h->ll_act, a.F, 1, nullptr, -1, d, a.F, L.wq));
    if (xt) summed(ops.back(), n);
    *x_src = (int)ops.size();
    ops.push_back(gemv_op(M, resid_epi, L.w2, nullptr, h->ll_act, a.F, i_w13, nullptr, 0.f, h->ll_x, d, 1, x_att,
                          i_wo, a.F, d, L.wq));
    if (xt) {
        ops.back().r_nsum = n, ops.back().r_rstride = (long long)M * d;
        to_peers(ops.back(), 2 * l + 1);
    }
}

// The weights of a GEMV op in the engine's slot order (engine_relayout),
// built once per (matrices, row mapping) and kept for the handle's lifetime.
int32_t tiled_weights(S2dHandle *h, EngineOp &o) {
    const auto key = std::make_tuple(o.W, o.W2, o.N, o.K, o.n_contig, o.n_contig >= 0 ? o.row_base : 0,
                                     o.n_contig >= 0 ? o.extra_row : 0);
    auto it = h->tiled.find(key);
    if (it == h->tiled.end()) {
        uint16_t *dst = nullptr;
        const int gtype = ggml_type_of(o.wt);
        const size_t n = engine_weight_bytes(gtype, o.N, o.K, o.W2 ? 2 : 1);
        CK(cudaMalloc(&dst, n));
        it = h->tiled.emplace(key, dst).first;
        CK(launch_engine_relayout(o.W, o.W2, gtype, o.N, o.K, o.n_contig, o.row_base, o.extra_row, h->num_sms,
                                  h->slot_bytes, dst, h->stream));
        h->tiled_bytes += n;
    }
    o.Wt = it->second;
    return S2D_OK;
}

int32_t upload_program(S2dHandle *h, const std::vector<EngineOp> &ops_in, EngineProgram *p) {
    if (p->ops) cudaFree(p->ops);
    p->ops = nullptr;
    std::vector<EngineOp> ops = ops_in;
    if ((int)ops.size() > kEngineMaxOps) return set_err(h, S2D_EINVAL, "engine: program too long");
    // Shared area: a GEMV's staged inputs, or an attention op's groups (query
    // vectors and new K/V rows); the cached K/V rows come through the ring.
    int ab = 0;
    for (EngineOp &o : ops) {
        if (o.kind == OP_GEMV) {
            ab = std::max(ab, o.M * o.K * 4);
            const int32_t rc = tiled_weights(h, o);
            if (rc) return rc;
        } else if (o.kind == OP_SAMPLE) {
            if (o.K < 2 || o.K % 2 || o.K > kEngineSampleMax || o.samp.n != o.K || o.sample_cta < 0 ||
                o.sample_cta >= h->num_sms)
                return set_err(h, S2D_EINVAL, "engine: unsupported sample op");
            ab = std::max(ab, engine_sample_bytes(o.K, (int)sizeof(SampleScratch)));
        } else if (o.kind == OP_ATTN_CTX) {
            if (o.ctx_n > kEngineMaxCtx || o.pos_const + o.M > o.ctx_n || (o.hd != 64 && o.hd != 128) ||
                o.H % o.Hkv || (o.H / o.Hkv) > kEngineConsumerWarps)
                return set_err(h, S2D_EINVAL, "engine: unsupported context attention op");
            const int rep = o.H / o.Hkv;
            ab = std::max(ab, (kEngineConsumerWarps / rep) * attn_ctx_group_bytes(rep, o.hd, o.ctx_n));
        } else {
            if (o.M > 2) return set_err(h, S2D_EINVAL, "engine: attention over more than 2 tokens");
            const int kvb = o.kv_half ? 2 : 4;
            if (attn_slot_rows(o.hd, kvb, h->slot_bytes) < 1)
                return set_err(h, S2D_EINVAL, "engine: ring slots too small for a cache row");
            ab = std::max(ab, (kEngineConsumerWarps / (o.H / o.Hkv)) * attn_group_bytes(o.H / o.Hkv, o.hd, kvb));
        }
    }
    ab = (ab + 127) / 128 * 128;
    const int ns = (int)std::min<long>(kEngineMaxSlots,
                                       ((long)kEngineSmemMax - kEngineBarrierBytes - ab) / h->slot_bytes);
    if (ns < 2) return set_err(h, S2D_EINVAL, "engine: inputs too large for shared memory");
    CK(cudaMalloc(&p->ops, ops.size() * sizeof(EngineOp)));
    CK(cudaMemcpy(p->ops, ops.data(), ops.size() * sizeof(EngineOp), cudaMemcpyHostToDevice));
    p->n_ops = (int)ops.size();
    p->frame = false;
    for (const EngineOp &o : ops) p->frame |= o.kind == OP_SAMPLE || o.kind == OP_ATTN_CTX;
    p->area_bytes = ab;
    p->nslots = ns;
    p->smem = (size_t)kEngineBarrierBytes + (size_t)ab + (size_t)ns * h->slot_bytes;
    if (p->smem > (size_t)kEngineSmemMax) return set_err(h, S2D_EINVAL, "engine: shared memory layout too large");
    return S2D_OK;
}

// Fast-AR pass programs (codebook 1..K-1) and the Slow-AR step program.
int32_t build_programs(S2dHandle *h, uint32_t im_end) {
    const S2dGraphSpec &s = h->spec;
    const int d = s.hidden, K = s.num_codebooks;
    int32_t rc;
    if (h->fast_progs.empty()) {
        h->fast_progs.resize((size_t)std::max(K, 1));
        for (int cbk = 1; cbk < K; ++cbk) {
            const int p0 = cbk == 1 ? 0 : cbk, M = cbk == 1 ? 2 : 1;
            std::vector<EngineOp> ops;
            int x_src = -1;
            for (int l = 0; l < h->fast.L; ++l)
                layer_ops(h, true, l, h->fast_x + (size_t)p0 * d, M, nullptr, p0, ops, &x_src);
            // the head reads the residual of the pass's last token (position cbk)
            ops.push_back(gemv_op(1, EPI_STORE, h->fast_out, nullptr, h->ll_x + (size_t)(M - 1) * d, d, x_src,
                                  h->fast_norm, h->fast.eps, h->logits_fast, s.codebook_size, 0, nullptr, -1, d,
                                  s.codebook_size, h->fast_out_wq));
            if ((rc = upload_program(h, ops, &h->fast_progs[(size_t)cbk]))) return rc;
        }
    }
    if (!h->slow_prog.ops || h->slow_prog_im_end != im_end) {
        std::vector<EngineOp> ops;
        int x_src = -1;
        for (int l = 0; l < h->slow.L; ++l) layer_ops(h, false, l, h->x, 1, &h->st->n_past, 0, ops, &x_src);
        const int nsem = s.semantic_end_id - s.semantic_begin_id + 1;
        const bool extra = (int64_t)im_end < s.vocab_size &&
                           ((int)im_end < s.semantic_begin_id || (int)im_end > s.semantic_end_id);
        // the final residual: LL words of the last w2, or on a tensor-parallel
        // handle the ranks' rows of its exchange region
        const bool xt = h->tp > 1 && h->xchg;
        const void *xf = xt ? static_cast<const void *>(h->xchg + (size_t)(2 * h->slow.L - 1) * h->tp * d)
                            : static_cast<const void *>(h->ll_x);
        EngineOp head = gemv_op(1, EPI_STORE, h->emb, nullptr, xf, d, x_src, h->norm, h->slow.eps, h->logits,
                                s.vocab_size, 0, nullptr, -1, d, nsem + (extra ? 1 : 0));
        if (xt) head.x_nsum = h->tp, head.x_rstride = d;
        head.row_base = s.semantic_begin_id, head.n_contig = nsem;
        head.extra_row = extra ? (int)im_end : s.semantic_begin_id;
        head.x_out = h->hidden_post;
        ops.push_back(head);
        if ((rc = upload_program(h, ops, &h->slow_prog))) return rc;
        h->slow_prog_im_end = im_end;
        h->n_allowed_extra = extra ? 1 : 0;
    }
    return S2D_OK;
}

// The Fast-AR of one frame as a single engine program (the loop of
// generate_codebooks_for_semantic, fast_ar.rs:440-470): for each codebook
// k = 1..K-1 the pass's layers (pass 1 over positions 0 and 1, pass k > 1
// over position k), the head (fast_ar.rs:429-435) and a SAMPLE op on CTA 0
// (sample_token, sampling.rs:121-241) that writes code k and the next
// pass's input row fast_emb[code k].  Attention reads the earlier positions
// from the WQKV words of the passes that produced them (ctx_qkv), so no KV
// cache and no launch boundary sits between the passes.  The sampling
// parameters are part of the program: rebuilt when the key changes.
int32_t build_fast_frame(S2dHandle *h, const GenKey &k) {
    const S2dGraphSpec &s = h->spec;
    const ArShape &f = h->fast;
    const int d = s.hidden, K = s.num_codebooks, L = f.L, q_out = f.qkv_out();
    if (!h->fast_frame || K < 2 || K > kEngineMaxCtx || (f.hd != 64 && f.hd != 128) ||
        s.codebook_size > kEngineSampleMax || s.codebook_size % 2 ||
        (size_t)(K - 1) * (5 * L + 2) > (size_t)kEngineMaxOps) {
        if (h->fast_frame_prog.ops) cudaFree(h->fast_frame_prog.ops);
        h->fast_frame_prog = EngineProgram{};
        return S2D_OK;  // one launch per pass
    }
    if (h->fast_frame_prog.ops && h->fast_frame_key == k) return S2D_OK;
    std::vector<EngineOp> ops;
    std::vector<std::vector<int>> qkv_op((size_t)K, std::vector<int>((size_t)L, -1));
    auto qbuf = [&](int pass, int l) { return h->fr_qkv + ((size_t)(pass - 1) * L + l) * 2 * q_out; };
    int prev_sample = -1;
    for (int cbk = 1; cbk < K; ++cbk) {
        const int p0 = cbk == 1 ? 0 : cbk, M = cbk == 1 ? 2 : 1;
        int x_src = -1;
        for (int l = 0; l < L; ++l) {
            const size_t base = ops.size();
            layer_ops(h, true, l, h->fast_x + (size_t)p0 * d, M, nullptr, p0, ops, &x_src);
            EngineOp &q = ops[base], &at = ops[base + 1], &wo = ops[base + 2];
            q.y = qbuf(cbk, l);
            at.qkv = qbuf(cbk, l);
            if (l == 0 && cbk > 1) {  // the previous sample op's input row
                q.x = h->fr_x + (size_t)cbk * d, q.x_src = prev_sample;
                wo.resid = q.x, wo.resid_src = prev_sample;
            }
            qkv_op[(size_t)cbk][(size_t)l] = (int)base;
            at.kind = OP_ATTN_CTX, at.ctx_n = p0 + M;
            for (int j = 0; j < p0 + M; ++j) {
                const int pass = j <= 1 ? 1 : j, row = j <= 1 ? j : 0;
                at.ctx_qkv[j] = qbuf(pass, l) + (size_t)row * q_out;
                at.ctx_src[j] = qkv_op[(size_t)pass][(size_t)l];
            }
        }
        const int i_head = (int)ops.size();
        ops.push_back(gemv_op(1, EPI_STORE, h->fast_out, nullptr, h->ll_x + (size_t)(M - 1) * d, d, x_src,
                              h->fast_norm, h->fast.eps, h->fr_logits, s.codebook_size, 1, nullptr, -1, d,
                              s.codebook_size, h->fast_out_wq));
        EngineOp sm{};
        sm.kind = OP_SAMPLE, sm.M = 1, sm.x = h->fr_logits, sm.x_src = i_head, sm.K = s.codebook_size, sm.N = d;
        sm.y = cbk + 1 < K ? static_cast<void *>(h->fr_x + (size_t)(cbk + 1) * d) : nullptr;
        sm.sample_cta = 0;
        SampleArgs &a = sm.samp;
        a.logits = nullptr, a.n = s.codebook_size, a.n_contig = -1, a.vocab_full = s.codebook_size;
        a.temperature = k.temperature, a.top_p = k.top_p, a.top_k = k.top_k, a.force_id = -1;
        a.mode = SAMPLE_FAST, a.max_new = (int)k.max_new, a.st = h->st, a.rng = &h->st->rng;
        a.cb_index = cbk, a.frame_codes = h->frame_codes, a.codes_out = h->codes_out;
        a.fast_emb = h->fast_emb, a.fast_x_next = nullptr, a.d = d, a.out_token = h->tok_out;
        prev_sample = (int)ops.size();
        ops.push_back(sm);
    }
    int32_t rc = upload_program(h, ops, &h->fast_frame_prog);
    if (rc) return rc;
    h->fast_frame_key = k;
    return S2D_OK;
}

cudaError_t enqueue_engine(S2dHandle *h, const EngineProgram &p) {
    EngineArgs a{};
    a.ops = p.ops, a.n_ops = p.n_ops, a.nslots = p.nslots, a.slot_bytes = h->slot_bytes;
    a.area_bytes = p.area_bytes, a.epoch = h->engine_epoch, a.done = &h->st->done, a.error = &h->st->error;
    a.l2_lead = h->l2_lead;
    h->launches += 1;
    return launch_engine(a, h->num_sms, p.smem, h->stream, p.frame);
}

// One frame with the persistent engine: 9 Fast-AR pass programs and one
// Slow-AR step program, with the samplers and the embedding between them.
cudaError_t enqueue_frame_engine(S2dHandle *h, const GenKey &k) {
    const S2dGraphSpec &s = h->spec;
    const int d = s.hidden, K = s.num_codebooks;
    const int32_t *done = &h->st->done;
    cudaError_t e;
    FastInitArgs fi{};
    fi.st = h->st, fi.slow_hidden = h->hidden_post, fi.fast_emb = h->fast_emb, fi.fast_x = h->fast_x;
    fi.frame_codes = h->frame_codes, fi.codes_out = h->codes_out;
    fi.max_new = (int)k.max_new, fi.d = d, fi.cb_size = s.codebook_size;
    fi.sem_begin = (uint32_t)s.semantic_begin_id, fi.sem_end = (uint32_t)s.semantic_end_id;
    h->launches += 1;
    if ((e = launch_fast_init(fi, h->stream, false))) return e;
    if (h->fast_frame_prog.ops) {
        if ((e = enqueue_engine(h, h->fast_frame_prog))) return e;
    }
    for (int cbk = 1; cbk < K && !h->fast_frame_prog.ops; ++cbk) {
        if ((e = enqueue_engine(h, h->fast_progs[(size_t)cbk]))) return e;
        SampleArgs a{};
        a.logits = h->logits_fast, a.n = s.codebook_size, a.n_contig = -1, a.vocab_full = s.codebook_size;
        a.temperature = k.temperature, a.top_p = k.top_p, a.top_k = k.top_k, a.force_id = -1;
        a.mode = SAMPLE_FAST, a.max_new = (int)k.max_new, a.st = h->st, a.rng = &h->st->rng;
        a.cb_index = cbk, a.frame_codes = h->frame_codes, a.codes_out = h->codes_out;
        a.fast_emb = h->fast_emb, a.fast_x_next = cbk + 1 < K ? h->fast_x + (size_t)(cbk + 1) * d : nullptr;
        a.d = d, a.out_token = h->tok_out;
        h->launches += 1;
        if ((e = launch_sample(a, h->stream, false))) return e;
    }
    EmbedArgs ea{};
    ea.tokens = nullptr, ea.st = h->st, ea.frame_codes = h->frame_codes;
    ea.emb = h->emb, ea.cb_emb = h->cb_emb, ea.d = s.hidden, ea.K = s.num_codebooks;
    ea.cb_size = s.codebook_size, ea.vocab = s.vocab_size, ea.cb_rows = s.codebook_rows;
    ea.sem_begin = (uint32_t)s.semantic_begin_id, ea.sem_end = (uint32_t)s.semantic_end_id;
    ea.scale_on = 1, ea.sem_scale = 1.0f / sqrtf((float)(s.num_codebooks + 1));
    ea.out = h->x, ea.M = 1, ea.done = done, ea.error = &h->st->error;
    h->launches += 1;
    if ((e = launch_embed(ea, h->stream, false))) return e;
    if ((e = enqueue_engine(h, h->slow_prog))) return e;
    SampleArgs a = slow_sample_args(h, SAMPLE_SLOW_STEP, k);
    h->launches += 1;
    return launch_sample(a, h->stream, false);
}

// One full frame (the loop body of generate_codes, generate.rs:165-211).
cudaError_t enqueue_frame(S2dHandle *h, const GenKey &k) {
    if (h->use_engine) return enqueue_frame_engine(h, k);
    const S2dGraphSpec &s = h->spec;
    const int32_t *done = &h->st->done;
    cudaError_t e;
    if ((e = enqueue_fast_frame(h, k, false))) return e;
    EmbedArgs ea{};
    ea.tokens = nullptr, ea.st = h->st, ea.frame_codes = h->frame_codes;
    ea.emb = h->emb, ea.cb_emb = h->cb_emb, ea.d = s.hidden, ea.K = s.num_codebooks;
    ea.cb_size = s.codebook_size, ea.vocab = s.vocab_size, ea.cb_rows = s.codebook_rows;
    ea.sem_begin = (uint32_t)s.semantic_begin_id, ea.sem_end = (uint32_t)s.semantic_end_id;
    ea.scale_on = 1, ea.sem_scale = 1.0f / sqrtf((float)(s.num_codebooks + 1));
    ea.out = h->x, ea.M = 1, ea.done = done, ea.error = &h->st->error;
    h->launches += 1;
    if ((e = launch_embed(ea, h->stream, h->pdl))) return e;
    for (int l = 0; l < h->slow.L; ++l)
        if ((e = enqueue_layer(h, false, l, h->x, 1, &h->st->n_past, 0, done))) return e;
    if ((e = enqueue_lm_head(h, h->x, false, k.im_end, done))) return e;
    SampleArgs a = slow_sample_args(h, SAMPLE_SLOW_STEP, k);
    h->launches += 1;
    return launch_sample(a, h->stream, h->pdl);
}

int32_t check_device_error(S2dHandle *h) {
    int32_t err = 0;
    CK(cudaMemcpyAsync(&err, &h->st->error, sizeof(int32_t), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    if (err) {
        cudaMemsetAsync(&h->st->error, 0, sizeof(int32_t), h->stream);
        return set_err(h, S2D_EDEVICE, "device error flag " + std::to_string(err) +
                                           " (1: KV position out of range, 2-4: token id out of range)");
    }
    return S2D_OK;
}

// Slow-AR eval over n tokens at positions n_past.. (SlowArState::eval,
// slow_ar.rs:456-527).  Leaves the post-norm hidden in hidden_post and the
// logits in h->logits.
// Prefill chunk length of the batched path, and the smallest prompt it takes.
constexpr int kPrefillChunk = 512;
constexpr size_t kBlasWorkspace = (size_t)32 << 20;
constexpr int kPrefillMin = 8;

int32_t ensure_prefill(S2dHandle *h) {
    if (h->pf_cap) return S2D_OK;
    if (!h->blas) {
        if (cublasCreate(&h->blas) != CUBLAS_STATUS_SUCCESS) return set_err(h, S2D_ECUDA, "cublasCreate failed");
        if (cublasSetStream(h->blas, h->stream) != CUBLAS_STATUS_SUCCESS)
            return set_err(h, S2D_ECUDA, "cublasSetStream failed");
        // a workspace of our own, so that GEMMs captured into the batched
        // frame graph never allocate
        CK(cudaMalloc(&h->blas_ws, kBlasWorkspace));
        if (cublasSetWorkspace(h->blas, h->blas_ws, kBlasWorkspace) != CUBLAS_STATUS_SUCCESS)
            return set_err(h, S2D_ECUDA, "cublasSetWorkspace failed");
    }
    // row buffers for both stacks (the batched Fast-AR passes use them too)
    // and the heads (masked LM head, fast_output)
    const ArShape &a = h->slow, &f = h->fast;
    const S2dGraphSpec &sp = h->spec;
    const size_t T = kPrefillChunk;
    const size_t d = (size_t)std::max(a.d, f.d), qo = (size_t)std::max(a.qkv_out(), f.qkv_out());
    const size_t qs = (size_t)std::max(a.qs(), f.qs()), F = (size_t)std::max(a.F, f.F);
    const size_t kmax = std::max(std::max(d, qs), F);
    const size_t heads_n = (size_t)std::max(sp.semantic_end_id - sp.semantic_begin_id + 2, sp.codebook_size);
    const size_t nmax = std::max(std::max(std::max(d, qo), F), heads_n);
    CK(cudaMalloc(&h->pf_x, T * d * sizeof(float)));
    CK(cudaMalloc(&h->pf_qkv, T * qo * sizeof(float)));
    CK(cudaMalloc(&h->pf_q, T * qs * sizeof(float)));
    CK(cudaMalloc(&h->pf_att, T * qs * sizeof(float)));
    CK(cudaMalloc(&h->pf_act, T * F * sizeof(float)));
    CK(cudaMalloc(&h->pf_inv, T * sizeof(float)));
    CK(cudaMalloc(&h->pf_y2, 2 * T * nmax * sizeof(float)));
    CK(cudaMalloc(&h->pf_y2b, 2 * T * nmax * sizeof(float)));
    CK(cudaMalloc(&h->pf_xs, 2 * T * kmax * sizeof(__half)));
    h->pf_cap = (int)T;
    return S2D_OK;
}

// Y2 [2T][N] = xs [2T][K] (f16) x W^T, W [N][K] f16 row-major, f32 accumulation.
int32_t prefill_gemm(S2dHandle *h, const uint16_t *W, int N, int K, int T, float *Y2) {
    const float one = 1.0f, zero = 0.0f;
    const cublasStatus_t st =
        cublasGemmEx(h->blas, CUBLAS_OP_T, CUBLAS_OP_N, N, 2 * T, K, &one, W, CUDA_R_16F, K, h->pf_xs, CUDA_R_16F, K,
                     &zero, Y2, CUDA_R_32F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    if (st != CUBLAS_STATUS_SUCCESS) return set_err(h, S2D_ECUDA, "cublasGemmEx failed (" + std::to_string((int)st) + ")");
    return S2D_OK;
}

// Kernel categories of s2d_profile_batch (S2D_PROF_* in include/s2d.h).
enum ProfCat { PC_SPLIT = 0, PC_GEMM = 1, PC_COMBINE = 2, PC_ROPE = 3, PC_ATTN = 4, PC_SAMPLE = 5, PC_OTHER = 6,
               PC_COUNT = 7 };

// While profiling, an event after the launch just enqueued, tagged cat.
void mark(S2dHandle *h, int cat) {
    if (!h->marks) return;
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return;
    cudaEventRecord(e, h->stream);
    h->marks->emplace_back(cat, e);
}

// Whether rows_linear takes the tcgen05 GEMM for an N x K weight over T rows.
bool tc_gemm_supported_rows(const S2dHandle *h, int N, int K, int T) {
    TcGemm g;
    g.W = reinterpret_cast<const uint16_t *>(16), g.N = N, g.K = K, g.xs = h->pf_xs, g.T = T, g.inv = h->pf_inv;
    g.y = h->pf_y2, g.ldy = N;
    return tc_gemm_supported(g);
}

// y = epilogue(W . x) over the T rows split into pf_xs / pf_inv: the tcgen05
// GEMM with the epilogue fused when it takes the shape, else cuBLAS over the
// stacked rows followed by the combine pass.  W2 is the up projection of the
// SwiGLU forms.

int32_t rows_linear(S2dHandle *h, const uint16_t *W, const uint16_t *W2, int N, int K, int T, int epi, float *y,
                    int ldy, const float *resid, int ldr) {
    TcGemm g;
    g.W = W, g.W2 = W2, g.N = N, g.K = K, g.xs = h->pf_xs, g.T = T, g.inv = h->pf_inv, g.epi = epi;
    g.y = y, g.ldy = ldy, g.resid = resid, g.ldr = ldr, g.num_sms = h->num_sms > 0 ? h->num_sms : 148;
    g.error = &h->st->error;
    if (h->use_tc && tc_gemm_supported(g)) {
        CK(launch_tc_gemm(g, h->stream));
        mark(h, PC_GEMM);
        h->launches += 1;
        return S2D_OK;
    }
    int32_t rc;
    if ((rc = prefill_gemm(h, W, N, K, T, h->pf_y2))) return rc;
    if (W2 && (rc = prefill_gemm(h, W2, N, K, T, h->pf_y2b))) return rc;
    mark(h, PC_GEMM);
    CK(launch_combine(epi, h->pf_y2, W2 ? h->pf_y2b : nullptr, h->pf_inv, T, N, y, ldy, resid, ldr, h->stream));
    mark(h, PC_COMBINE);
    h->launches += 1;
    return S2D_OK;
}

// Rows of one layered pass (rows_layers): T rows of the residual x, row m
// of sequence m / rps at position pos_const + m % rps (+ st[seq].n_past with
// st_pos); sequence s's KV cache starts kv_seq_stride elements after
// sequence 0's (kv).  Rows of finished sequences (st[seq].done) write no KV.
struct RowsPlan {
    int T = 0, rps = 1, pos_const = 0, st_pos = 0, S = 1;
    const DevState *st = nullptr;
    const int32_t *order = nullptr;  // one row per sequence: the attention's block order
    void *kv = nullptr;
    size_t kv_seq_stride = 0;
    int max_seq = 0;
    KvPages pages{};  // paged caches (pages.pages set): kv is the pool, kv_seq_stride unused
    size_t kv_bytes = 0;  // bytes of the buffer kv points into (the tcgemm attention's bounds)
};

// Every layer of the Slow-AR (is_fast false) or the Fast-AR over T rows of
// x [T][ldx] in place, a layer at a time: the linears are GEMMs over the
// stacked hi/lo rows, RoPE + KV write and GQA attention are per row
// (SlowArLayerSkeleton::forward_decode_token_with_backend +
// forward_feed_forward_with_backend, slow_ar.rs:637-710, for each row;
// forward_slow_ar_block_prefill_layers_cached, slow_ar.rs:1002-1039, when the
// rows are one prompt; FastArLayerSkeleton::forward_prefill,
// fast_ar.rs:245-352, for the Fast-AR).
// A quantized layer's linears as f16 rows in qscratch (rounded to nearest):
// L's weight pointers are redirected there.
int32_t dequant_layer(S2dHandle *h, const ArShape &a, LayerDev *L) {
    if (!h->qscratch[0]) {
        const ArShape &sl = h->slow, &fa = h->fast;
        const size_t d = (size_t)std::max(sl.d, fa.d);
        const size_t n[5] = {(size_t)std::max(sl.qkv_out(), fa.qkv_out()) * d,
                             d * (size_t)std::max(sl.qs(), fa.qs()), (size_t)std::max(sl.F, fa.F) * d,
                             (size_t)std::max(sl.F, fa.F) * d, d * (size_t)std::max(sl.F, fa.F)};
        for (int i = 0; i < 5; ++i) CK(cudaMalloc(&h->qscratch[i], n[i] * sizeof(__half)));
    }
    const uint16_t **w[5] = {&L->wqkv, &L->wo, &L->w1, &L->w3, &L->w2};
    const int64_t n[5] = {(int64_t)a.qkv_out() * a.d, (int64_t)a.d * a.qs(), (int64_t)a.F * a.d,
                          (int64_t)a.F * a.d, (int64_t)a.d * a.F};
    for (int i = 0; i < 5; ++i) {
        CK(launch_dequant_f16(L->wq, *w[i], h->qscratch[i], n[i], h->stream));
        *w[i] = reinterpret_cast<const uint16_t *>(h->qscratch[i]);
    }
    L->wq = EW_F16;
    h->launches += 5;
    return S2D_OK;
}

// The resident f16 expansion of every quantized linear (batched generation):
// the rows path then streams f16 weights once per frame step instead of
// dequantising each layer again.  Exact dequantisation, rounded to f16, as the
// per-layer scratch of the quantized prefill.
int32_t ensure_f16_linears(S2dHandle *h) {
    auto expand = [&](int wq, const uint16_t *src, int64_t n, const uint16_t **dst) -> int32_t {
        __half *p = nullptr;
        CK(cudaMalloc(&p, (size_t)n * sizeof(__half)));
        h->f16_bufs.push_back(p);
        CK(launch_dequant_f16(wq, src, p, n, h->stream));
        *dst = reinterpret_cast<const uint16_t *>(p);
        return S2D_OK;
    };
    int32_t rc;
    for (int fast = 0; fast < 2; ++fast) {
        const ArShape &a = fast ? h->fast : h->slow;
        std::vector<LayerDev> &src = fast ? h->fast_layers : h->slow_layers;
        std::vector<LayerDev> &dst = fast ? h->fast_f16 : h->slow_f16;
        if (!dst.empty()) continue;
        std::vector<LayerDev> out = src;
        for (LayerDev &L : out) {
            if (L.wq == EW_F16) continue;
            const int64_t n[5] = {(int64_t)a.qkv_out() * a.d, (int64_t)a.d * a.qs(), (int64_t)a.F * a.d,
                                  (int64_t)a.F * a.d, (int64_t)a.d * a.F};
            const uint16_t **w[5] = {&L.wqkv, &L.wo, &L.w1, &L.w3, &L.w2};
            for (int i = 0; i < 5; ++i)
                if ((rc = expand(L.wq, *w[i], n[i], w[i]))) return rc;
            L.wq = EW_F16;
            h->launches += 5;
        }
        dst = std::move(out);
    }
    if (h->fast_out_wq != EW_F16 && !h->fast_out_f16) {
        const uint16_t *p = nullptr;
        if ((rc = expand(h->fast_out_wq, h->fast_out, (int64_t)h->spec.codebook_size * h->spec.hidden, &p))) return rc;
        h->fast_out_f16 = const_cast<__half *>(reinterpret_cast<const __half *>(p));
    }
    return S2D_OK;
}

int32_t rows_layers(S2dHandle *h, bool is_fast, float *x, int ldx, const RowsPlan &rp) {
    const ArShape &a = is_fast ? h->fast : h->slow;
    const int d = a.d, qo = a.qkv_out(), qs = a.qs(), F = a.F, T = rp.T;
    const size_t kvb = is_fast ? sizeof(float) : sizeof(__half);
    // a layer's K and V: contiguous [Hkv][max_seq][hd] each, or (paged) the
    // layer's slice of page 0 of the pool, [Hkv][kKvPage][hd] each
    const size_t layer_bytes = (size_t)2 * a.Hkv * (rp.pages.pages ? kKvPage : rp.max_seq) * a.hd * kvb;
    // tensor parallel (Slow-AR rows in one block of d floats each): rank 0
    // adds the residual, the others store their partial sums; summed in place
    const bool part = !is_fast && h->tp > 1;
    const int resid_epi = part && h->tp_rank != 0 ? PF_STORE : PF_RESID;
    if (part && ldx != d) return set_err(h, S2D_EINVAL, "tensor-parallel rows must be contiguous");
    // on the cuBLAS path without an exchange between them, each combine pass
    // also makes the next GEMM's row split (one pass per row instead of two)
    const bool fuse = !h->use_tc && !part;
    // the rows' split for `lin` (N outputs, K inputs) followed by the next
    // GEMM's split of the result (norm_w optional); y may be null when fused
    auto linear_then_split = [&](const uint16_t *W, const uint16_t *W2, int N, int K, int epi, float *y, int ldy,
                                 const float *resid, int ldr, const float *norm_w) -> int32_t {
        int32_t r2;
        if (fuse) {
            if ((r2 = prefill_gemm(h, W, N, K, T, h->pf_y2))) return r2;
            if (W2 && (r2 = prefill_gemm(h, W2, N, K, T, h->pf_y2b))) return r2;
            mark(h, PC_GEMM);
            CK(launch_combine_split(epi, h->pf_y2, W2 ? h->pf_y2b : nullptr, h->pf_inv, T, N, y, ldy, resid, ldr,
                                    norm_w, a.eps, h->pf_xs, h->stream));
            mark(h, PC_COMBINE);
            h->launches += 1;
            return S2D_OK;
        }
        if ((r2 = rows_linear(h, W, W2, N, K, T, epi, y, ldy, resid, ldr))) return r2;
        if (part && epi == resid_epi) CK(tp_allreduce(h, y, (size_t)T * d));
        CK(launch_split_rows(y, ldy, T, N, norm_w, a.eps, h->pf_xs, h->pf_inv, nullptr, h->stream));
        mark(h, PC_SPLIT);
        h->launches += 1;
        return S2D_OK;
    };
    int32_t rc;
    bool presplit = false;  // pf_xs / pf_inv already hold this layer's attention-norm split
    for (int l = 0; l < a.L; ++l) {
        LayerDev L = is_fast ? h->fast_layers[(size_t)l] : h->slow_layers[(size_t)l];
        const std::vector<LayerDev> &x16 = is_fast ? h->fast_f16 : h->slow_f16;
        if (L.wq != EW_F16 && !x16.empty()) L = x16[(size_t)l];  // the resident f16 expansion
        if (L.wq != EW_F16 && (rc = dequant_layer(h, a, &L))) return rc;
        // attention_norm + WQKV
        if (!presplit) {
            CK(launch_split_rows(x, ldx, T, d, L.attn_norm, a.eps, h->pf_xs, h->pf_inv, nullptr, h->stream));
            mark(h, PC_SPLIT);
            h->launches += 1;
        }
        presplit = false;
        // On cuBLAS, RoPE reads the GEMM's stacked hi / lo rows itself (the
        // store combine folded into its loads); the tcgen05 epilogue combines.
        const bool qkv_fold = !(h->use_tc && tc_gemm_supported_rows(h, qo, d, T));
        if (qkv_fold) {
            if ((rc = prefill_gemm(h, L.wqkv, qo, d, T, h->pf_y2))) return rc;
            mark(h, PC_GEMM);
        } else if ((rc = rows_linear(h, L.wqkv, nullptr, qo, d, T, PF_STORE, h->pf_qkv, qo, nullptr, 0))) {
            return rc;
        }
        // QK-norm (Slow-AR) + RoPE + KV write for every row
        uint8_t *base = reinterpret_cast<uint8_t *>(rp.kv) + (size_t)l * layer_bytes;
        RopeArgs r{};
        r.qkv = h->pf_qkv, r.ld_qkv = qo, r.q_out = h->pf_q;
        if (qkv_fold) r.qkv = h->pf_y2, r.qkv_lo = h->pf_y2 + (size_t)T * qo, r.inv = h->pf_inv;
        r.kcache = base, r.vcache = base + layer_bytes / 2, r.max_seq = rp.max_seq;
        if (!is_fast) r.q_norm = L.q_norm, r.k_norm = L.k_norm;
        r.rope_denom = is_fast ? h->rope_fast : h->rope_slow;
        r.eps = a.eps, r.pos_dev = nullptr, r.pos_const = rp.pos_const;
        r.H = a.H, r.Hkv = a.Hkv, r.hd = a.hd, r.M = T, r.done = nullptr, r.error = &h->st->error;
        r.rows_per_seq = rp.rps, r.st_b = rp.st, r.st_pos = rp.st_pos, r.kv_seq_stride = rp.kv_seq_stride;
        r.kv_pages = rp.pages;
        CK(launch_rope_kv(r, !is_fast, h->stream, false));
        mark(h, PC_ROPE);
        // GQA attention of every row over its sequence's cache
        RowsAttnArgs t{};
        t.q = h->pf_q, t.kcache = r.kcache, t.vcache = r.vcache, t.kv_seq_stride = rp.kv_seq_stride;
        t.kv_pages = rp.pages;
        t.max_seq = rp.max_seq, t.out = h->pf_att, t.T = T, t.rows_per_seq = rp.rps, t.st = rp.st;
        t.st_pos = rp.st_pos, t.pos_const = rp.pos_const, t.H = a.H, t.Hkv = a.Hkv, t.hd = a.hd;
        t.scale = 1.0f / sqrtf((float)a.hd);  // SlowArLayerShape::attn_scale (slow_ar.rs:59-61)
        t.S = rp.S, t.part = h->ra_part, t.counters = h->ra_counters, t.decode_stages = h->attn_stages;
        t.prefill_mma = h->prefill_mma;
        t.prefill_tc = h->prefill_tc && !is_fast && rp.kv_bytes > 0;
        if (t.prefill_tc) {
            const size_t kb = base - reinterpret_cast<uint8_t *>(rp.kv), rowb = (size_t)a.hd * 2;
            t.k_rows = (rp.kv_bytes - kb) / rowb, t.v_rows = (rp.kv_bytes - kb - layer_bytes / 2) / rowb;
        }
        t.error = &h->st->error;
        if (h->attn_mma && rp.st && rp.st_pos && rp.rps == 1) {
            t.decode_mma = 1, t.decode_warps = h->attn_mma_warps, t.decode_stages = h->attn_mma_stages;
            t.decode_chunk = h->attn_mma_chunk, t.row_order = rp.order;
        }
        CK(launch_rows_attention(t, !is_fast, h->stream));
        mark(h, PC_ATTN);
        // wo + residual, then the ffn_norm split
        CK(launch_split_rows(h->pf_att, qs, T, qs, nullptr, 0.f, h->pf_xs, h->pf_inv, nullptr, h->stream));
        mark(h, PC_SPLIT);
        if ((rc = linear_then_split(L.wo, nullptr, d, qs, resid_epi, x, ldx, x, ldx, L.ffn_norm))) return rc;
        // w1 / w3 + SwiGLU, then the split for w2 (the SwiGLU row is not kept when fused)
        if ((rc = linear_then_split(L.w1, L.w3, F, d, is_fast ? PF_SWIGLU_FAST : PF_SWIGLU_SLOW,
                                    fuse ? nullptr : h->pf_act, F, nullptr, 0, nullptr)))
            return rc;
        // w2 + residual (with the next layer's attention-norm split when fused)
        if (fuse && l + 1 < a.L) {
            const LayerDev &N2 = is_fast ? h->fast_layers[(size_t)l + 1] : h->slow_layers[(size_t)l + 1];
            if ((rc = linear_then_split(L.w2, nullptr, d, F, resid_epi, x, ldx, x, ldx, N2.attn_norm))) return rc;
            presplit = true;
        } else {
            if ((rc = rows_linear(h, L.w2, nullptr, d, F, T, resid_epi, x, ldx, x, ldx))) return rc;
            if (part) CK(tp_allreduce(h, x, (size_t)T * d));
        }
        h->launches += 3;  // rope, attention, the attention split
    }
    return S2D_OK;
}

// The Slow-AR layers over T (<= pf_cap) embedded tokens in pf_x at positions
// pos0 .. pos0 + T - 1 of sequence 0's cache.
int32_t prefill_layers(S2dHandle *h, int T, int pos0) {
    RowsPlan rp;
    rp.T = T, rp.rps = T, rp.pos_const = pos0, rp.kv = h->kv_slow, rp.max_seq = h->cfg.max_seq;
    rp.kv_bytes = h->kv_slow_seq * sizeof(__half);
    if (h->pf_pages) {  // a batched sequence: its pages of the pool
        rp.kv = h->kv_pool, rp.kv_bytes = h->kv_pool_pages * h->kv_page_elems * sizeof(__half);
        rp.pages = KvPages{h->pf_pages, h->kv_per_seq, h->kv_page_elems};
    }
    return rows_layers(h, false, h->pf_x, h->slow.d, rp);
}

// The checks of SlowArState::eval on n_flat time-major ids (slow_ar.rs:456-474)
// and of embed_slow_ar_time_major (slow_ar.rs:1071-1105, tensor.rs:177-185).
int32_t check_eval_ids(S2dHandle *h, const int32_t *flat, int64_t n_flat) {
    const S2dGraphSpec &s = h->spec;
    const int64_t cd = s.num_codebooks + 1;
    if (n_flat <= 0 || n_flat % cd)
        return set_err(h, S2D_EINVAL, "flat token length " + std::to_string(n_flat) +
                                          " is not a multiple of codebook_dim " + std::to_string(cd));
    const int64_t n = n_flat / cd;
    if (h->n_past + n > h->cfg.max_seq)
        return set_err(h, S2D_ESTATE, "KV cache overflow: n_past=" + std::to_string(h->n_past) +
                                          " n_tokens=" + std::to_string(n) +
                                          " max_seq_len=" + std::to_string(h->cfg.max_seq));
    for (int64_t t = 0; t < n; ++t) {
        const int32_t id = flat[t * cd];
        if (id < 0) return set_err(h, S2D_EINVAL, "semantic token id must be non-negative, got " + std::to_string(id));
        if (id >= s.vocab_size)
            return set_err(h, S2D_EINVAL, "embedding index " + std::to_string(id) + " out of range for vocab_dim " +
                                              std::to_string(s.vocab_size));
        if (id < s.semantic_begin_id || id > s.semantic_end_id) continue;
        for (int cb = 0; cb < s.num_codebooks; ++cb) {
            const int32_t raw = flat[t * cd + 1 + cb];
            if (raw < 0) return set_err(h, S2D_EINVAL, "codebook token must be non-negative, got " + std::to_string(raw));
            const int64_t cid = (int64_t)raw + (int64_t)cb * s.codebook_size;
            if (cid >= s.codebook_rows)
                return set_err(h, S2D_EINVAL, "embedding index " + std::to_string(cid) + " out of range for vocab_dim " +
                                                  std::to_string(s.codebook_rows));
        }
    }
    return S2D_OK;
}

int32_t slow_eval(S2dHandle *h, const int32_t *flat, int64_t n_flat, int32_t logits_mode,
                  uint32_t im_end) {
    const S2dGraphSpec &s = h->spec;
    const int64_t cd = s.num_codebooks + 1;
    int32_t rc = check_eval_ids(h, flat, n_flat);
    if (rc) return rc;
    const int64_t n = n_flat / cd;
    rc = ensure_tokens(h, (size_t)n_flat);
    if (rc) return rc;
    CK(cudaMemcpyAsync(h->tokens_dev, flat, (size_t)n_flat * sizeof(int32_t), cudaMemcpyHostToDevice, h->stream));
    // a batched sequence's prompt always takes the rows path (its cache is paged)
    if (n >= kPrefillMin || h->pf_pages) {
        if ((rc = ensure_prefill(h))) return rc;
        for (int64_t c0 = 0; c0 < n; c0 += h->pf_cap) {
            const int T = (int)std::min<int64_t>(h->pf_cap, n - c0);
            EmbedArgs ea{};
            ea.tokens = h->tokens_dev + c0 * cd, ea.emb = h->emb, ea.cb_emb = h->cb_emb, ea.d = s.hidden;
            ea.K = s.num_codebooks, ea.cb_size = s.codebook_size, ea.vocab = s.vocab_size;
            ea.cb_rows = s.codebook_rows, ea.sem_begin = (uint32_t)s.semantic_begin_id;
            ea.sem_end = (uint32_t)s.semantic_end_id, ea.scale_on = 1;
            ea.sem_scale = 1.0f / sqrtf((float)(s.num_codebooks + 1));
            ea.out = h->pf_x, ea.M = T, ea.error = &h->st->error;
            h->launches += 1;
            CK(launch_embed(ea, h->stream, false));
            if ((rc = prefill_layers(h, T, (int)(h->n_past + c0)))) return rc;
            if (c0 + T >= n)
                CK(enqueue_lm_head(h, h->pf_x + (size_t)(T - 1) * s.hidden, logits_mode == S2D_LOGITS_FULL, im_end,
                                   nullptr));
        }
        rc = check_device_error(h);
        if (rc) return rc;
        h->n_past += (int32_t)n;
        return S2D_OK;
    }
    for (int64_t c0 = 0; c0 < n;) {
        int M = (int)std::min<int64_t>(kMaxM, n - c0);
        if (M == 3) M = 2;  // GEMV instantiations: 1, 2, 4
        EmbedArgs ea{};
        ea.tokens = h->tokens_dev + c0 * cd, ea.emb = h->emb, ea.cb_emb = h->cb_emb, ea.d = s.hidden;
        ea.K = s.num_codebooks, ea.cb_size = s.codebook_size, ea.vocab = s.vocab_size;
        ea.cb_rows = s.codebook_rows, ea.sem_begin = (uint32_t)s.semantic_begin_id;
        ea.sem_end = (uint32_t)s.semantic_end_id, ea.scale_on = 1;
        ea.sem_scale = 1.0f / sqrtf((float)(s.num_codebooks + 1));
        ea.out = h->x, ea.M = M, ea.error = &h->st->error;
        h->launches += 1;
        CK(launch_embed(ea, h->stream, false));
        for (int l = 0; l < h->slow.L; ++l)
            CK(enqueue_layer(h, false, l, h->x, M, nullptr, (int)(h->n_past + c0), nullptr));
        if (c0 + M >= n) {
            CK(enqueue_lm_head(h, h->x + (size_t)(M - 1) * s.hidden, logits_mode == S2D_LOGITS_FULL, im_end, nullptr));
        }
        c0 += M;
    }
    rc = check_device_error(h);
    if (rc) return rc;
    h->n_past += (int32_t)n;
    return S2D_OK;
}

// One Slow-AR step (SlowArState::step, slow_ar.rs:444-454) on the persistent
// engine: the step program that every generated frame runs, fed with the
// caller's step input instead of the sampled one.  Leaves the post-norm
// hidden in hidden_post and the allowed logits (semantic rows + im_end) in
// h->logits, like slow_eval with S2D_LOGITS_ALLOWED.
int32_t engine_step(S2dHandle *h, const int32_t *flat, int64_t n_flat, uint32_t im_end) {
    const S2dGraphSpec &s = h->spec;
    int32_t rc = check_eval_ids(h, flat, n_flat);
    if (rc) return rc;
    if ((rc = ensure_tokens(h, (size_t)n_flat))) return rc;
    if (h->slow_prog.ops && h->slow_prog_im_end != im_end && h->frame_exec) {
        // the captured frame graph points at the program about to be replaced
        cudaGraphExecDestroy(h->frame_exec);
        h->frame_exec = nullptr;
    }
    if ((rc = build_programs(h, im_end))) return rc;
    CK(cudaMemcpyAsync(h->tokens_dev, flat, (size_t)n_flat * sizeof(int32_t), cudaMemcpyHostToDevice, h->stream));
    // the program reads the step's position from the device state
    CK(launch_set_state(h->st, h->n_past, 0, 0, h->stream));
    EmbedArgs ea{};
    ea.tokens = h->tokens_dev, ea.emb = h->emb, ea.cb_emb = h->cb_emb, ea.d = s.hidden;
    ea.K = s.num_codebooks, ea.cb_size = s.codebook_size, ea.vocab = s.vocab_size;
    ea.cb_rows = s.codebook_rows, ea.sem_begin = (uint32_t)s.semantic_begin_id;
    ea.sem_end = (uint32_t)s.semantic_end_id, ea.scale_on = 1;
    ea.sem_scale = 1.0f / sqrtf((float)(s.num_codebooks + 1));
    ea.out = h->x, ea.M = 1, ea.error = &h->st->error;
    h->launches += 2;
    CK(launch_embed(ea, h->stream, false));
    CK(enqueue_engine(h, h->slow_prog));
    if ((rc = check_device_error(h))) return rc;
    h->n_past += 1;
    return S2D_OK;
}

int32_t copy_eval_outputs(S2dHandle *h, float *out_hidden, float *out_logits, int32_t mode,
                          uint32_t im_end) {
    const S2dGraphSpec &s = h->spec;
    if (out_hidden)
        CK(cudaMemcpyAsync(out_hidden, h->hidden_post, (size_t)s.hidden * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
    if (out_logits && mode == S2D_LOGITS_FULL)
        CK(cudaMemcpyAsync(out_logits, h->logits, (size_t)s.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
    if (out_logits && mode == S2D_LOGITS_ALLOWED) {
        const int nsem = s.semantic_end_id - s.semantic_begin_id + 1;
        for (int i = 0; i < s.vocab_size; ++i) out_logits[i] = -INFINITY;
        CK(cudaMemcpyAsync(out_logits + s.semantic_begin_id, h->logits, (size_t)nsem * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
        if (h->n_allowed_extra)
            CK(cudaMemcpyAsync(out_logits + im_end, h->logits + nsem, sizeof(float), cudaMemcpyDeviceToHost, h->stream));
    }
    CK(cudaStreamSynchronize(h->stream));
    return S2D_OK;
}

// ---------------------------------------------------------------------------
// batched generation: B independent sequences advance one frame per graph
// launch, every linear a GEMM over the B (or 2B) rows of the frame
// ---------------------------------------------------------------------------

constexpr int kBatchMaxSeq = kPrefillChunk / 2;  // rows of the first Fast-AR pass fit one row block

int32_t ensure_batch(S2dHandle *h, uint32_t max_new) {
    const S2dGraphSpec &s = h->spec;
    const ArShape &a = h->slow, &f = h->fast;
    const size_t B = (size_t)h->max_batch, d = (size_t)s.hidden, K = (size_t)std::max(s.num_codebooks, 1);
    int32_t rc;
    if ((rc = ensure_prefill(h))) return rc;
    if (!h->st_b) {
        const size_t nsem = (size_t)(s.semantic_end_id - s.semantic_begin_id + 1);
        const size_t kvf = (size_t)f.L * 2 * f.Hkv * f.ctx * f.hd;
        // The Slow-AR caches of the batch: a pool of kKvPage-position pages
        // ([layer][K | V][kv head][kKvPage][hd] f16 each) and a page table
        // of kv_per_seq entries per slot.  Pages are dealt out per call
        // (deal_pages) or per admitted request (s2d_serve_admit) in a seeded
        // random order of the pool (pool_order), so that no sequence's cache
        // is contiguous.
        h->kv_per_seq = (h->cfg.max_seq + kKvPage - 1) / kKvPage;
        h->kv_page_elems = (size_t)a.L * 2 * a.Hkv * kKvPage * a.hd;
        const size_t n_rows = B * (size_t)h->kv_per_seq;  // page-table entries
        const size_t n_pages = h->cfg.kv_pages > 0 ? (size_t)h->cfg.kv_pages : n_rows;
        h->kv_pool_pages = n_pages;
        CK(cudaMalloc(&h->kv_pool, n_pages * h->kv_page_elems * sizeof(__half)));
        CK(cudaMemset(h->kv_pool, 0, n_pages * h->kv_page_elems * sizeof(__half)));
        std::vector<int32_t> table(n_pages);
        for (size_t i = 0; i < n_pages; ++i) table[i] = (int32_t)i;
        uint64_t x = 0x9e3779b97f4a7c15ull;  // splitmix64 stream for a Fisher-Yates shuffle
        for (size_t i = n_pages; i > 1; --i) {
            x += 0x9e3779b97f4a7c15ull;
            uint64_t z = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
            z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
            std::swap(table[i - 1], table[(z ^ (z >> 31)) % i]);
        }
        CK(cudaMalloc(&h->kv_page_table, n_rows * sizeof(int32_t)));
        CK(cudaMemset(h->kv_page_table, 0, n_rows * sizeof(int32_t)));
        h->pool_order = table;
        CK(cudaMalloc(&h->st_b, B * sizeof(DevState)));
        CK(cudaMemset(h->st_b, 0, B * sizeof(DevState)));
        CK(cudaMalloc(&h->bx, B * d * sizeof(float)));
        CK(cudaMemset(h->bx, 0, B * d * sizeof(float)));
        CK(cudaMalloc(&h->fx, B * 2 * d * sizeof(float)));
        CK(cudaMemset(h->fx, 0, B * 2 * d * sizeof(float)));
        CK(cudaMalloc(&h->hidden_b, B * d * sizeof(float)));
        CK(cudaMemset(h->hidden_b, 0, B * d * sizeof(float)));
        CK(cudaMalloc(&h->logits_b, B * (nsem + 1) * sizeof(float)));
        CK(cudaMalloc(&h->logits_fast_b, B * (size_t)s.codebook_size * sizeof(float)));
        CK(cudaMalloc(&h->kv_fast_b, std::max<size_t>(B * kvf, 1) * sizeof(float)));
        CK(cudaMemset(h->kv_fast_b, 0, std::max<size_t>(B * kvf, 1) * sizeof(float)));
        CK(cudaMalloc(&h->frame_codes_b, B * K * sizeof(int32_t)));
        CK(cudaMemset(h->frame_codes_b, 0, B * K * sizeof(int32_t)));
        // split partials of the rows attention: up to 2 rows per sequence
        h->ra_rows = (int)(2 * B), h->ra_smax = 16;
        const size_t H = (size_t)std::max(a.H, f.H), Hkv = (size_t)std::max(a.Hkv, f.Hkv);
        const size_t hd = (size_t)std::max(a.hd, f.hd);
        CK(cudaMalloc(&h->ra_part, (size_t)h->ra_rows * H * h->ra_smax * (hd + 2) * sizeof(float)));
        CK(cudaMalloc(&h->ra_counters, (size_t)h->ra_rows * Hkv * sizeof(int32_t)));
        CK(cudaMemset(h->ra_counters, 0, (size_t)h->ra_rows * Hkv * sizeof(int32_t)));
        CK(cudaMalloc(&h->batch_order, B * sizeof(int32_t)));
        std::vector<int32_t> ident(B);
        for (size_t i = 0; i < B; ++i) ident[i] = (int32_t)i;
        CK(cudaMemcpy(h->batch_order, ident.data(), B * sizeof(int32_t), cudaMemcpyHostToDevice));
    }
    const size_t need = B * K * std::max<uint32_t>(max_new, 1);
    if (need > h->codes_b_cap) {
        if (h->codes_b) cudaFree(h->codes_b);
        h->codes_b = nullptr;
        h->codes_b_cap = 0;
        CK(cudaMalloc(&h->codes_b, need * sizeof(int32_t)));
        h->codes_b_cap = need;
        if (h->batch_exec) {  // the captured frame points at the old buffer
            cudaGraphExecDestroy(h->batch_exec);
            h->batch_exec = nullptr;
        }
    }
    return S2D_OK;
}

// Attention splits of the batched Slow-AR step: enough blocks for ~8 per SM.
int batch_splits(const S2dHandle *h, int B) {
    const int blocks = B * h->slow.Hkv;
    const int per_sm = h->attn_mma ? h->attn_mma_blocks_per_sm : h->attn_blocks_per_sm;
    return std::max(1, std::min(h->ra_smax, (per_sm * std::max(h->num_sms, 1) + blocks - 1) / blocks));
}

// One frame of B sequences (the loop body of generate_codes,
// generate.rs:165-211, for each sequence): Fast-AR codebooks 1..K-1 over all
// sequences' rows, the embedding-sum feedback, the Slow-AR step over B rows,
// the masked LM head and the semantic sampler.  Finished sequences keep their
// state and caches (every kernel that writes them checks the sequence's done
// flag).
int32_t enqueue_frame_batch(S2dHandle *h, const GenKey &k, int B, int rng_kind, uint64_t philox_key) {
    const S2dGraphSpec &s = h->spec;
    const int d = s.hidden, K = s.num_codebooks, cb = s.codebook_size;
    const int nsem = s.semantic_end_id - s.semantic_begin_id + 1;
    const bool extra = (int64_t)k.im_end < s.vocab_size &&
                       ((int)k.im_end < s.semantic_begin_id || (int)k.im_end > s.semantic_end_id);
    const size_t codes_stride = (size_t)K * k.max_new;
    const ArShape &f = h->fast;
    int32_t rc;
    FastInitArgs fi{};
    fi.st = h->st_b, fi.slow_hidden = h->hidden_b, fi.fast_emb = h->fast_emb, fi.fast_x = h->fx;
    fi.frame_codes = h->frame_codes_b, fi.codes_out = h->batch_profile ? nullptr : h->codes_b;
    fi.max_new = (int)k.max_new, fi.d = d, fi.cb_size = cb;
    fi.sem_begin = (uint32_t)s.semantic_begin_id, fi.sem_end = (uint32_t)s.semantic_end_id;
    fi.batched = 1, fi.hidden_stride = (size_t)d, fi.fast_x_stride = (size_t)2 * d;
    fi.codes_stride = codes_stride, fi.frame_stride = (size_t)K;
    CK(launch_fast_init_batch(fi, B, h->stream));
    mark(h, PC_OTHER);
    h->launches += 1;
    for (int cbk = 1; cbk < K; ++cbk) {
        // positions 0 and 1 on the first pass (rows (seq, 0), (seq, 1) of fx),
        // then position cbk in row (seq, 0)
        const int M = cbk == 1 ? 2 : 1;
        RowsPlan rp;
        rp.T = B * M, rp.rps = M, rp.pos_const = cbk == 1 ? 0 : cbk, rp.st = h->st_b, rp.st_pos = 0, rp.S = 1;
        rp.kv = h->kv_fast_b, rp.kv_seq_stride = (size_t)f.L * 2 * f.Hkv * f.ctx * f.hd, rp.max_seq = f.ctx;
        if ((rc = rows_layers(h, true, h->fx, M == 2 ? d : 2 * d, rp))) return rc;
        // fast_norm + fast_output on each sequence's last row
        CK(launch_split_rows(h->fx + (size_t)(M - 1) * d, 2 * d, B, d, h->fast_norm, f.eps, h->pf_xs, h->pf_inv,
                             nullptr, h->stream));
        mark(h, PC_SPLIT);
        const uint16_t *fo = h->fast_out_wq == EW_F16 ? h->fast_out : reinterpret_cast<const uint16_t *>(h->fast_out_f16);
        if ((rc = rows_linear(h, fo, nullptr, cb, d, B, PF_STORE, h->logits_fast_b, cb, nullptr, 0))) return rc;
        SampleArgs a{};
        a.logits = h->logits_fast_b, a.n = cb, a.n_contig = -1, a.vocab_full = cb;
        a.temperature = k.temperature, a.top_p = k.top_p, a.top_k = k.top_k, a.force_id = -1;
        a.mode = SAMPLE_FAST, a.max_new = (int)k.max_new, a.st = h->st_b, a.cb_index = cbk;
        a.frame_codes = h->frame_codes_b, a.codes_out = h->batch_profile ? nullptr : h->codes_b;
        a.fast_emb = h->fast_emb;
        a.fast_x_next = cbk + 1 < K ? h->fx : nullptr, a.d = d;
        a.rng_kind = rng_kind, a.philox_key = philox_key;
        a.batched = 1, a.logits_stride = (size_t)cb, a.codes_stride = codes_stride;
        a.fast_x_stride = (size_t)2 * d, a.frame_stride = (size_t)K;
        CK(launch_sample_batch(a, B, h->stream));
        mark(h, PC_SAMPLE);
        h->launches += 3;
    }
    // step input embedding (build_step_input + embed_slow_ar_time_major)
    EmbedArgs ea{};
    ea.tokens = nullptr, ea.st = h->st_b, ea.frame_codes = h->frame_codes_b, ea.batched = 1;
    ea.emb = h->emb, ea.cb_emb = h->cb_emb, ea.d = d, ea.K = K;
    ea.cb_size = cb, ea.vocab = s.vocab_size, ea.cb_rows = s.codebook_rows;
    ea.sem_begin = (uint32_t)s.semantic_begin_id, ea.sem_end = (uint32_t)s.semantic_end_id;
    ea.scale_on = 1, ea.sem_scale = 1.0f / sqrtf((float)(K + 1));
    ea.out = h->bx, ea.M = B, ea.done = nullptr, ea.error = &h->st->error;
    CK(launch_embed(ea, h->stream, false));
    mark(h, PC_OTHER);
    // Slow-AR step: one row per sequence at its own position
    RowsPlan rp;
    rp.T = B, rp.rps = 1, rp.pos_const = 0, rp.st = h->st_b, rp.st_pos = 1, rp.S = batch_splits(h, B);
    rp.order = h->attn_mma_order ? h->batch_order : nullptr;
    rp.kv = h->kv_pool, rp.max_seq = h->cfg.max_seq;
    rp.kv_bytes = h->kv_pool_pages * h->kv_page_elems * sizeof(__half);
    rp.pages = KvPages{h->kv_page_table, h->kv_per_seq, h->kv_page_elems};
    if ((rc = rows_layers(h, false, h->bx, d, rp))) return rc;
    // final norm (post-norm hidden for the next frame's Fast-AR) + masked LM head
    CK(launch_split_rows(h->bx, d, B, d, h->norm, h->slow.eps, h->pf_xs, h->pf_inv, h->hidden_b, h->stream));
    mark(h, PC_SPLIT);
    if ((rc = rows_linear(h, h->emb + (size_t)s.semantic_begin_id * d, nullptr, nsem, d, B, PF_STORE, h->logits_b,
                          nsem + 1, nullptr, 0)))
        return rc;
    if (extra &&
        (rc = rows_linear(h, h->emb + (size_t)k.im_end * d, nullptr, 1, d, B, PF_STORE, h->logits_b + nsem, nsem + 1,
                          nullptr, 0)))
        return rc;
    SampleArgs a = slow_sample_args(h, SAMPLE_SLOW_STEP, k);
    a.logits = h->logits_b, a.st = h->st_b, a.rng = nullptr, a.out_token = nullptr;
    a.rng_kind = rng_kind, a.philox_key = philox_key;
    a.batched = 1, a.logits_stride = (size_t)nsem + 1;
    CK(launch_sample_batch(a, B, h->stream));
    mark(h, PC_SAMPLE);
    h->launches += 4 + (extra ? 1 : 0);
    return S2D_OK;
}

void free_handle(S2dHandle *h) {
    if (!h) return;
    if (h->device >= 0) cudaSetDevice(h->device);
    // graphs that hold NCCL calls go before the communicator
    if (h->frame_exec) cudaGraphExecDestroy(h->frame_exec);
    if (h->batch_exec) cudaGraphExecDestroy(h->batch_exec);
    h->frame_exec = nullptr, h->batch_exec = nullptr;
    if (h->stream) cudaStreamSynchronize(h->stream);
    for (int q = 0; q < kEngineMaxPeers; ++q)
        if (h->xchg_peer[q] && h->xchg_peer[q] != h->xchg) cudaIpcCloseMemHandle(h->xchg_peer[q]);
    if (h->xchg) cudaFree(h->xchg);
    if (h->comm) nccl().comm_destroy(h->comm);
    if (h->shard_arena) cudaFree(h->shard_arena);
    for (void *p : {(void *)h->st_b, (void *)h->bx, (void *)h->fx, (void *)h->hidden_b, (void *)h->logits_b,
                    (void *)h->logits_fast_b, (void *)h->kv_fast_b, (void *)h->frame_codes_b, (void *)h->codes_b,
                    (void *)h->ra_part, (void *)h->ra_counters, (void *)h->batch_order})
        if (p) cudaFree(p);
    void *bufs[] = {h->arena, h->norm_arena, h->rope_slow, h->rope_fast, h->kv_slow, h->kv_fast, h->kv_pool, h->kv_page_table,
                    h->x, h->qkv, h->q, h->att, h->act, h->fast_x, h->hidden_post, h->logits,
                    h->logits_fast, h->part, h->counters, h->st, h->tokens_dev, h->frame_codes,
                    h->codes_out, h->tok_out, h->code_override, h->engine_epoch, h->slow_prog.ops,
                    h->ll_x, h->ll_qkv, h->ll_att, h->ll_act, h->ll_part, h->rope_cs_slow, h->rope_cs_fast};
    for (void *p : bufs)
        if (p) cudaFree(p);
    for (EngineProgram &p : h->fast_progs)
        if (p.ops) cudaFree(p.ops);
    if (h->fast_frame_prog.ops) cudaFree(h->fast_frame_prog.ops);
    for (void *p : {(void *)h->fr_qkv, (void *)h->fr_logits, (void *)h->fr_x})
        if (p) cudaFree(p);
    for (auto &kv : h->tiled) cudaFree(kv.second);
    for (void *p : {(void *)h->pf_x, (void *)h->pf_qkv, (void *)h->pf_q, (void *)h->pf_att, (void *)h->pf_act,
                    (void *)h->pf_inv, (void *)h->pf_y2, (void *)h->pf_y2b, (void *)h->pf_xs})
        if (p) cudaFree(p);
    for (__half *p : h->f16_bufs) cudaFree(p);
    for (__half *p : h->qscratch)
        if (p) cudaFree(p);
    if (h->blas) cublasDestroy(h->blas);
    if (h->blas_ws) cudaFree(h->blas_ws);
    if (h->ev0) cudaEventDestroy(h->ev0);
    if (h->ev1) cudaEventDestroy(h->ev1);
    if (h->ev2) cudaEventDestroy(h->ev2);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================

extern "C" {

namespace {
int32_t open_handle(const char *path, const S2dConfig *cfg, int32_t tp_size, int32_t tp_rank, const uint8_t *nccl_id,
                    S2dHandle **out, char *err, size_t err_cap) {
    auto report = [&](S2dHandle *h, int32_t rc) {
        if (err && err_cap) {
            snprintf(err, err_cap, "%s", h ? h->err.c_str() : "out of memory");
        }
        free_handle(h);
        return rc;
    };
    if (out) *out = nullptr;
    if (!path || !out) {
        if (err && err_cap) snprintf(err, err_cap, "s2d_open: path and out must not be NULL");
        return S2D_EINVAL;
    }
    S2dHandle *h = new (std::nothrow) S2dHandle();
    if (!h) return report(nullptr, S2D_ENOMEM);
    h->cfg = cfg ? *cfg : S2dConfig{0, 4096, 1, 0, 0};
    if (h->cfg.max_seq <= 0) {
        h->err = "max_seq_len must be non-zero";
        return report(h, S2D_EINVAL);
    }
    if (h->cfg.max_batch > 4096) {
        h->err = "max_batch must be at most 4096";
        return report(h, S2D_EINVAL);
    }
    h->max_batch = std::max(1, h->cfg.max_batch);
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size || (tp_size > 1 && !nccl_id)) {
        h->err = "invalid tensor-parallel rank, size or NCCL id";
        return report(h, S2D_EINVAL);
    }
    h->tp = tp_size, h->tp_rank = tp_rank;
    h->device = h->cfg.device;
    cudaError_t ce = cudaSetDevice(h->device);
    if (ce) {
        h->err = std::string("cudaSetDevice: ") + cudaGetErrorString(ce);
        h->device = -1;
        return report(h, S2D_ECUDA);
    }
    if ((ce = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking)) ||
        (ce = cudaEventCreate(&h->ev0)) || (ce = cudaEventCreate(&h->ev1)) ||
        (ce = cudaEventCreate(&h->ev2)) || (ce = configure_kernels())) {
        h->err = std::string("CUDA init: ") + cudaGetErrorString(ce);
        return report(h, S2D_ECUDA);
    }
    std::string e;
    if (!h->gguf.open(path, &e)) {
        h->err = e;
        return report(h, S2D_EIO);
    }
    int32_t rc;
    if ((rc = read_spec(h))) return report(h, rc);
    if ((rc = upload_all(h))) return report(h, rc);
    if ((rc = bind_weights(h))) return report(h, rc);
    if (h->tp > 1) {
        if ((rc = shard_slow_weights(h))) return report(h, rc);
        if (!nccl().ok) {
            h->err = "NCCL (libnccl.so.2, or S2D_NCCL_LIB) could not be loaded";
            return report(h, S2D_ECUDA);
        }
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof(id));
        const ncclResult_t nr = nccl().comm_init_rank(&h->comm, h->tp, id, h->tp_rank);
        if (nr != ncclSuccess) {
            h->comm = nullptr;
            h->err = std::string("ncclCommInitRank: ") + nccl().error_string(nr);
            return report(h, S2D_ECUDA);
        }
    }
    if ((rc = alloc_buffers(h))) return report(h, rc);
    if (h->tp > 1 && (rc = setup_exchange(h))) return report(h, rc);
    {
        int coop = 0;
        cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, h->device);
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, h->device);
        const char *env = getenv("S2D_ENGINE");
        // a tensor-parallel handle runs the engine when the ranks' exchange
        // buffers are mapped (setup_exchange); otherwise the per-op kernels
        // with NCCL allreduces
        h->use_engine = coop && (h->tp == 1 || h->xchg) && engine_supported(h) && !(env && env[0] == '0');
        if (const char *lead = getenv("S2D_L2_LEAD")) h->l2_lead = std::max(0, std::min(64, atoi(lead)));
        if (const char *ff = getenv("S2D_FAST_FRAME")) h->fast_frame = ff[0] != '0';
        if (const char *sp = getenv("S2D_ATT_SPLITS")) h->engine_att_splits = std::max(0, atoi(sp));
        if (const char *tc = getenv("S2D_TCGEMM")) h->use_tc = tc[0] == '1';
        if (const char *ab = getenv("S2D_BATCH_ATT_BLOCKS")) h->attn_blocks_per_sm = std::max(1, std::min(64, atoi(ab)));
        if (const char *st = getenv("S2D_BATCH_ATT_STAGES")) h->attn_stages = atoi(st) == 2 ? 2 : 4;
        if (const char *v = getenv("S2D_DECODE_MMA")) h->attn_mma = atoi(v) != 0;
        if (const char *v = getenv("S2D_DECODE_WARPS")) h->attn_mma_warps = atoi(v) == 2 ? 2 : 4;
        if (const char *v = getenv("S2D_DECODE_STAGES")) h->attn_mma_stages = atoi(v) == 3 ? 3 : 2;
        if (const char *v = getenv("S2D_DECODE_BLOCKS")) h->attn_mma_blocks_per_sm = std::max(1, std::min(64, atoi(v)));
        if (const char *v = getenv("S2D_DECODE_CHUNK")) h->attn_mma_chunk = atoi(v) == 32 ? 32 : 16;
        if (const char *v = getenv("S2D_DECODE_ORDER")) h->attn_mma_order = atoi(v) != 0;
        if (const char *v = getenv("S2D_PREFILL_MMA")) h->prefill_mma = atoi(v) != 0;
        if (const char *v = getenv("S2D_PREFILL_TC")) h->prefill_tc = atoi(v) != 0;
        if (const char *kb = getenv("S2D_SLOT_KB")) {
            const int v = atoi(kb);
            if (v >= 4 && v <= 96) h->slot_bytes = v * 1024;
        }
    }
    if ((ce = cudaStreamSynchronize(h->stream))) {
        h->err = std::string("CUDA: ") + cudaGetErrorString(ce);
        return report(h, S2D_ECUDA);
    }
    *out = h;
    return S2D_OK;
}
}  // namespace

int32_t s2d_open(const char *path, const S2dConfig *cfg, S2dHandle **out, char *err, size_t err_cap) {
    return open_handle(path, cfg, 1, 0, nullptr, out, err, err_cap);
}

int32_t s2d_open_tp(const char *path, const S2dConfig *cfg, int32_t tp_size, int32_t tp_rank, const uint8_t *nccl_id,
                    S2dHandle **out, char *err, size_t err_cap) {
    return open_handle(path, cfg, tp_size, tp_rank, nccl_id, out, err, err_cap);
}

int32_t s2d_tp_plan(const S2dGraphSpec *spec, int32_t tp_size, int32_t tp_rank, S2dTpShard *out) {
    if (!spec || !out) return S2D_EINVAL;
    return tp_plan(*spec, tp_size, tp_rank, out);
}

int32_t s2d_nccl_unique_id(uint8_t *out, size_t cap) {
    if (!out || cap < sizeof(ncclUniqueId)) return S2D_EINVAL;
    ncclUniqueId id;
    if (!nccl().ok || nccl().get_unique_id(&id) != ncclSuccess) return S2D_ECUDA;
    memcpy(out, &id, sizeof(id));
    return S2D_OK;
}

void s2d_close(S2dHandle *h) { free_handle(h); }

const char *s2d_last_error(const S2dHandle *h) { return h ? h->err.c_str() : ""; }

int32_t s2d_graph_spec(const S2dHandle *h, S2dGraphSpec *out) {
    if (!h || !out) return S2D_EINVAL;
    *out = h->spec;
    return S2D_OK;
}

int32_t s2d_reset(S2dHandle *h, int32_t seq) {
    if (!h) return S2D_EINVAL;
    if (seq != 0) return set_err(h, S2D_EINVAL, "seq must be 0");
    h->n_past = 0;
    return S2D_OK;
}

int32_t s2d_n_past(const S2dHandle *h, int32_t seq, int32_t *out) {
    if (!h || !out || seq != 0) return S2D_EINVAL;
    *out = h->n_past;
    return S2D_OK;
}

int32_t s2d_prefill(S2dHandle *h, int32_t seq, const int32_t *flat, int64_t n_flat, float *out_hidden,
                    float *out_logits, int32_t logits_mode, uint32_t im_end) {
    if (!h) return S2D_EINVAL;
    if (seq != 0 || !flat) return set_err(h, S2D_EINVAL, "bad arguments");
    CK(cudaSetDevice(h->device));
    int32_t rc = slow_eval(h, flat, n_flat, logits_mode, im_end);
    if (rc) return rc;
    return copy_eval_outputs(h, out_hidden, out_logits, logits_mode, im_end);
}

int32_t s2d_step(S2dHandle *h, int32_t seq, const int32_t *step_input, int64_t n, float *out_hidden,
                 float *out_logits, int32_t logits_mode, uint32_t im_end) {
    if (!h) return S2D_EINVAL;
    if (n != h->spec.num_codebooks + 1)
        return set_err(h, S2D_EINVAL, "step token width mismatch: expected " +
                                          std::to_string(h->spec.num_codebooks + 1) + ", got " + std::to_string(n));
    // Full-vocabulary logits need the per-op LM head; every other step runs
    // the engine's step program, the one the generated frames run.
    if (h->use_engine && logits_mode != S2D_LOGITS_FULL && seq == 0 && step_input) {
        CK(cudaSetDevice(h->device));
        int32_t rc = engine_step(h, step_input, n, im_end);
        if (rc) return rc;
        return copy_eval_outputs(h, out_hidden, out_logits, logits_mode, im_end);
    }
    return s2d_prefill(h, seq, step_input, n, out_hidden, out_logits, logits_mode, im_end);
}

int32_t s2d_fast_prefix_logits(S2dHandle *h, const float *slow_hidden, const uint32_t *prefix, int64_t n_prefix,
                               float *out_logits) {
    if (!h || !slow_hidden || (!prefix && n_prefix) || !out_logits) return S2D_EINVAL;
    const S2dGraphSpec &s = h->spec;
    if (n_prefix >= s.num_codebooks)
        return set_err(h, S2D_EINVAL, "fast prefix too long: " + std::to_string(n_prefix) + " codes (max " +
                                          std::to_string(s.num_codebooks - 1) + ")");
    if (n_prefix + 1 > h->fast.ctx)
        return set_err(h, S2D_EINVAL, "fast sequence length exceeds context_length");
    CK(cudaSetDevice(h->device));
    const int d = s.hidden;
    CK(cudaMemcpyAsync(h->fast_x, slow_hidden, (size_t)d * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    for (int64_t i = 0; i < n_prefix; ++i) {
        if (prefix[i] >= (uint32_t)s.codebook_size)
            return set_err(h, S2D_EINVAL, "embedding index " + std::to_string(prefix[i]) + " out of range");
        CK(launch_f16_to_f32(h->fast_emb + (size_t)prefix[i] * d, h->fast_x + (size_t)(1 + i) * d, d, h->stream));
    }
    const int n = (int)n_prefix + 1;
    for (int c0 = 0; c0 < n;) {
        int M = std::min(kMaxM, n - c0);
        if (M == 3) M = 2;
        for (int l = 0; l < h->fast.L; ++l)
            CK(enqueue_layer(h, true, l, h->fast_x + (size_t)c0 * d, M, nullptr, c0, nullptr));
        c0 += M;
    }
    CK(enqueue_fast_head(h, h->fast_x + (size_t)(n - 1) * d, nullptr));
    CK(cudaMemcpyAsync(out_logits, h->logits_fast, (size_t)s.codebook_size * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return check_device_error(h);
}

int32_t s2d_generate_codebooks(S2dHandle *h, const float *slow_hidden, uint32_t semantic_code,
                               const S2dSamplerParams *sp, uint64_t *rng_state, uint32_t *out_codes) {
    if (!h || !slow_hidden || !sp || !rng_state || !out_codes) return S2D_EINVAL;
    const S2dGraphSpec &s = h->spec;
    if (semantic_code >= (uint32_t)s.codebook_size)
        return set_err(h, S2D_EINVAL, "semantic_code " + std::to_string(semantic_code) + " >= codebook_size " +
                                          std::to_string(s.codebook_size));
    CK(cudaSetDevice(h->device));
    GenKey k;
    k.temperature = sp->temperature, k.top_p = sp->top_p, k.top_k = sp->top_k, k.max_new = 1;
    CK(cudaMemcpyAsync(h->hidden_post, slow_hidden, (size_t)s.hidden * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(h->code_override, &semantic_code, sizeof(uint32_t), cudaMemcpyHostToDevice, h->stream));
    CK(launch_set_state(h->st, 0, 0, *rng_state, h->stream));
    CK(enqueue_fast_frame(h, k, true));
    std::vector<int32_t> codes((size_t)s.num_codebooks);
    DevState st{};
    CK(cudaMemcpyAsync(codes.data(), h->frame_codes, codes.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaMemcpyAsync(&st, h->st, sizeof(DevState), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    for (size_t i = 0; i < codes.size(); ++i) out_codes[i] = (uint32_t)codes[i];
    *rng_state = st.rng;
    return st.error ? set_err(h, S2D_EDEVICE, "device error flag") : S2D_OK;
}

int32_t s2d_sample_token(S2dHandle *h, const float *logits, int64_t n, const S2dSamplerParams *sp,
                         int64_t always_include_id, uint64_t *rng_state, uint32_t *out_token) {
    if (!h || !logits || !sp || !rng_state || !out_token) return S2D_EINVAL;
    if (n <= 0 || n > kSampleMax) return set_err(h, S2D_EINVAL, "n must be in 1..8192");
    CK(cudaSetDevice(h->device));
    CK(cudaMemcpyAsync(h->logits_fast, logits, (size_t)n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    CK(launch_set_state(h->st, 0, 0, *rng_state, h->stream));
    SampleArgs a{};
    a.logits = h->logits_fast, a.n = (int)n, a.n_contig = -1, a.vocab_full = n;
    a.temperature = sp->temperature, a.top_p = sp->top_p, a.top_k = sp->top_k;
    a.force_id = always_include_id, a.mode = SAMPLE_PLAIN, a.st = h->st, a.rng = &h->st->rng;
    a.out_token = h->tok_out;
    CK(launch_sample(a, h->stream, false));
    DevState st{};
    CK(cudaMemcpyAsync(out_token, h->tok_out, sizeof(uint32_t), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaMemcpyAsync(&st, h->st, sizeof(DevState), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    *rng_state = st.rng;
    return S2D_OK;
}

int32_t s2d_generate_codes(S2dHandle *h, const uint32_t *prompt, int32_t rows, int32_t cols,
                           const S2dGenParams *p, uint64_t *rng_state, int32_t *out_codes,
                           uint32_t *out_n_frames, S2dProfile *profile) {
    if (!h) return S2D_EINVAL;
    if (!prompt || !p || !rng_state || !out_codes || !out_n_frames)
        return set_err(h, S2D_EINVAL, "s2d_generate_codes: NULL argument");
    const S2dGraphSpec &s = h->spec;
    const int K = std::max(s.num_codebooks, 1);
    if (rows != s.num_codebooks + 1) return set_err(h, S2D_EINVAL, "prompt rows must be num_codebooks+1");
    if (cols <= 0) return set_err(h, S2D_EINVAL, "expected at least one token");
    if ((int64_t)cols + (int64_t)p->max_new_tokens > h->cfg.max_seq)
        return set_err(h, S2D_ESTATE, "prompt + max_new_tokens exceeds max_seq");
    CK(cudaSetDevice(h->device));
    // transpose_to_time_major (prompt.rs:77-103)
    std::vector<int32_t> flat((size_t)rows * cols);
    for (int t = 0; t < cols; ++t)
        for (int r = 0; r < rows; ++r) {
            const uint32_t v = prompt[(size_t)r * cols + t];
            if (v > 0x7fffffffu) return set_err(h, S2D_EINVAL, "prompt token id does not fit i32");
            flat[(size_t)t * rows + r] = (int32_t)v;
        }
    const size_t need_codes = (size_t)K * std::max<uint32_t>(p->max_new_tokens, 1);
    if (need_codes > h->codes_cap) {
        if (h->codes_out) cudaFree(h->codes_out);
        h->codes_out = nullptr;
        h->codes_cap = 0;
        CK(cudaMalloc(&h->codes_out, need_codes * sizeof(int32_t)));
        h->codes_cap = need_codes;
        if (h->frame_exec) {  // captured frames point at the old buffer
            cudaGraphExecDestroy(h->frame_exec);
            h->frame_exec = nullptr;
        }
    }
    CK(cudaMemsetAsync(h->codes_out, 0, need_codes * sizeof(int32_t), h->stream));
    GenKey k;
    k.max_new = p->max_new_tokens, k.min_tokens = p->min_tokens_before_end, k.im_end = p->im_end_id;
    k.temperature = p->temperature, k.top_p = p->top_p, k.top_k = p->top_k;

    // prefill + first semantic sample (generate.rs:126-162)
    CK(cudaEventRecord(h->ev0, h->stream));
    const uint32_t launches0 = h->launches;
    h->n_past = 0;
    int32_t rc = slow_eval(h, flat.data(), (int64_t)flat.size(), S2D_LOGITS_ALLOWED, p->im_end_id);
    if (rc) return rc;
    CK(launch_set_state(h->st, h->n_past, cols, *rng_state, h->stream));
    SampleArgs first = slow_sample_args(h, SAMPLE_SLOW_FIRST, k);
    CK(launch_sample(first, h->stream, false));
    h->launches += 2;
    const uint32_t prefill_kernels = h->launches - launches0;
    CK(cudaEventRecord(h->ev1, h->stream));

    // frames (generate.rs:165-211): one captured graph per frame
    if (!h->frame_exec || !(h->frame_key == k)) {
        if (h->use_engine && (rc = build_programs(h, k.im_end))) return rc;
        if (h->use_engine && (rc = build_fast_frame(h, k))) return rc;
        if (h->frame_exec) cudaGraphExecDestroy(h->frame_exec);
        h->frame_exec = nullptr;
        cudaGraph_t graph = nullptr;
        CK(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = enqueue_frame(h, k);
        cudaError_t e2 = cudaStreamEndCapture(h->stream, &graph);
        if (e || e2) {
            if (graph) cudaGraphDestroy(graph);
            return set_err(h, S2D_ECUDA, std::string("frame capture: ") + cudaGetErrorString(e ? e : e2));
        }
        size_t nn = 0;
        cudaGraphGetNodes(graph, nullptr, &nn);
        h->frame_kernels = (uint32_t)nn;
        e = cudaGraphInstantiateWithFlags(&h->frame_exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e) return set_err(h, S2D_ECUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
        h->frame_key = k;
    }
    // Launch the frame graph up to max_new times; a frame whose state says
    // `done` exits in every kernel, so frames past the end are no-ops.  The
    // host polls `done` every few frames to stop launching early.
    const uint32_t poll = 8;
    DevState st{};
    uint32_t launched = 0;
    while (launched < p->max_new_tokens) {
        const uint32_t batch = std::min(poll, p->max_new_tokens - launched);
        for (uint32_t i = 0; i < batch; ++i) CK(cudaGraphLaunch(h->frame_exec, h->stream));
        launched += batch;
        CK(cudaMemcpyAsync(&st, h->st, sizeof(DevState), cudaMemcpyDeviceToHost, h->stream));
        CK(cudaStreamSynchronize(h->stream));
        if (st.done || st.error) break;
    }
    CK(cudaEventRecord(h->ev2, h->stream));
    CK(cudaMemcpyAsync(&st, h->st, sizeof(DevState), cudaMemcpyDeviceToHost, h->stream));
    std::vector<int32_t> codes(need_codes);
    CK(cudaMemcpyAsync(codes.data(), h->codes_out, need_codes * sizeof(int32_t), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    if (st.error) return set_err(h, S2D_EDEVICE, "device error flag " + std::to_string(st.error));
    if (!st.done) return set_err(h, S2D_ESTATE, "generation did not finish");
    const uint32_t frames = (uint32_t)st.step_index;
    // compact_codes (generate.rs:346-390)
    for (int cb = 0; cb < K; ++cb)
        for (uint32_t t = 0; t < frames; ++t)
            out_codes[(size_t)cb * frames + t] = codes[(size_t)cb * p->max_new_tokens + t];
    *out_n_frames = frames;
    *rng_state = st.rng;
    h->n_past = st.n_past;
    if (profile) {
        float a = 0, b = 0;
        cudaEventElapsedTime(&a, h->ev0, h->ev1);
        cudaEventElapsedTime(&b, h->ev1, h->ev2);
        profile->prefill_ms = a;
        profile->decode_ms = b;
        profile->frames = frames;
        profile->kernels_per_frame = h->frame_kernels;
        profile->prefill_kernels = prefill_kernels;
        profile->frame_launches = launched;
    }
    return S2D_OK;
}

namespace {

// Prefill of batch slot i (generate.rs:126-162 for one sequence): the
// prompt (rows x cols, row-major, transposed to time-major here) into the
// slot's pages of the pool, then the first semantic sample into the slot's
// DevState with RNG state `rng`; the post-norm hidden goes to the slot's row
// of hidden_b.  The single-sequence state is reset afterwards.
int32_t batch_admit_seq(S2dHandle *h, int i, const uint32_t *prompt, int rows, int cols, const GenKey &k,
                        uint64_t rng, int rng_kind, uint64_t philox_key) {
    const S2dGraphSpec &s = h->spec;
    std::vector<int32_t> flat((size_t)rows * cols);
    for (int t = 0; t < cols; ++t)
        for (int r = 0; r < rows; ++r) {
            const uint32_t v = prompt[(size_t)r * cols + t];
            if (v > 0x7fffffffu) return set_err(h, S2D_EINVAL, "prompt token id does not fit i32");
            flat[(size_t)t * rows + r] = (int32_t)v;
        }
    h->pf_pages = h->kv_page_table + (size_t)i * h->kv_per_seq;  // slot i's pages
    h->n_past = 0;
    int32_t rc = slow_eval(h, flat.data(), (int64_t)flat.size(), S2D_LOGITS_ALLOWED, k.im_end);
    h->pf_pages = nullptr;
    const int32_t n_past = h->n_past;
    h->n_past = 0;  // the single-sequence state is reset
    if (rc) return rc;
    CK(launch_set_state(h->st_b + i, n_past, cols, rng, h->stream));
    SampleArgs first = slow_sample_args(h, SAMPLE_SLOW_FIRST, k);
    first.st = h->st_b + i, first.rng = &h->st_b[i].rng, first.out_token = nullptr;
    first.rng_kind = rng_kind, first.philox_key = philox_key, first.rng_seq = (uint32_t)i;
    CK(launch_sample(first, h->stream, false));
    CK(cudaMemcpyAsync(h->hidden_b + (size_t)i * s.hidden, h->hidden_post, (size_t)s.hidden * sizeof(float),
                       cudaMemcpyDeviceToDevice, h->stream));
    h->launches += 2;
    return S2D_OK;
}

// The captured frame of n_seq batch slots for key k (re-captured when any of
// the key, the slot count or the RNG changes).
int32_t ensure_batch_graph(S2dHandle *h, const GenKey &k, int n_seq, int rng_kind, uint64_t philox_key) {
    if (h->batch_exec && h->batch_key == k && h->batch_n == n_seq && h->batch_rng_kind == rng_kind &&
        h->batch_philox == philox_key)
        return S2D_OK;
    if (h->batch_exec) cudaGraphExecDestroy(h->batch_exec);
    h->batch_exec = nullptr;
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    const uint32_t l0 = h->launches;
    const int32_t rc = enqueue_frame_batch(h, k, n_seq, rng_kind, philox_key);
    h->batch_kernels = h->launches - l0;
    cudaError_t e2 = cudaStreamEndCapture(h->stream, &graph);
    if (rc || e2) {
        if (graph) cudaGraphDestroy(graph);
        if (rc) return rc;
        return set_err(h, S2D_ECUDA, std::string("batch frame capture: ") + cudaGetErrorString(e2));
    }
    cudaError_t e = cudaGraphInstantiateWithFlags(&h->batch_exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e) return set_err(h, S2D_ECUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    h->batch_key = k, h->batch_n = n_seq, h->batch_rng_kind = rng_kind, h->batch_philox = philox_key;
    return S2D_OK;
}

}  // namespace

int32_t s2d_generate_codes_batch(S2dHandle *h, int32_t n_seq, const uint32_t *const *prompts,
                                 const int32_t *cols, int32_t rows, const S2dGenParams *p, int32_t rng_kind,
                                 uint64_t philox_key, uint64_t *rng_states, int32_t *out_codes,
                                 uint32_t *out_n_frames, S2dProfile *profile) {
    if (!h) return S2D_EINVAL;
    if (!prompts || !cols || !p || !rng_states || !out_codes || !out_n_frames)
        return set_err(h, S2D_EINVAL, "s2d_generate_codes_batch: NULL argument");
    const S2dGraphSpec &s = h->spec;
    const int K = std::max(s.num_codebooks, 1);
    if (n_seq <= 0 || n_seq > h->max_batch || n_seq > kBatchMaxSeq)
        return set_err(h, S2D_EINVAL, "n_seq must be in 1..min(max_batch, " + std::to_string(kBatchMaxSeq) +
                                          "), max_batch = " + std::to_string(h->max_batch));
    if (rng_kind != S2D_RNG_SEEDED && rng_kind != S2D_RNG_PHILOX) return set_err(h, S2D_EINVAL, "unknown rng_kind");
    if (rows != s.num_codebooks + 1) return set_err(h, S2D_EINVAL, "prompt rows must be num_codebooks+1");
    for (int i = 0; i < n_seq; ++i) {
        if (!prompts[i]) return set_err(h, S2D_EINVAL, "prompt " + std::to_string(i) + " is NULL");
        if (cols[i] <= 0) return set_err(h, S2D_EINVAL, "expected at least one token in prompt " + std::to_string(i));
        if ((int64_t)cols[i] + (int64_t)p->max_new_tokens > h->cfg.max_seq)
            return set_err(h, S2D_ESTATE, "prompt " + std::to_string(i) + " + max_new_tokens exceeds max_seq");
    }
    CK(cudaSetDevice(h->device));
    int32_t rc;
    if ((rc = ensure_batch(h, p->max_new_tokens))) return rc;
    // quantized linears: GEMMs over their resident f16 expansion
    if ((s.linear_type != 1 || h->fast_out_wq != EW_F16) && (rc = ensure_f16_linears(h))) return rc;
    const size_t codes_stride = (size_t)K * std::max<uint32_t>(p->max_new_tokens, 1);
    CK(cudaMemsetAsync(h->codes_b, 0, (size_t)n_seq * codes_stride * sizeof(int32_t), h->stream));
    GenKey k;
    k.max_new = p->max_new_tokens, k.min_tokens = p->min_tokens_before_end, k.im_end = p->im_end_id;
    k.temperature = p->temperature, k.top_p = p->top_p, k.top_k = p->top_k;

    // each sequence's prefill + first semantic sample (generate.rs:126-162),
    // into its own KV cache
    CK(cudaEventRecord(h->ev0, h->stream));
    const uint32_t launches0 = h->launches;
    h->serving = false;  // any serving slots are dropped
    {
        // each sequence gets the pages of positions [0, cols + max_new), in
        // the pool's dealing order
        std::vector<int32_t> table((size_t)n_seq * h->kv_per_seq);
        size_t next = 0;
        for (int i = 0; i < n_seq; ++i) {
            const size_t need = ((size_t)cols[i] + p->max_new_tokens + kKvPage - 1) / kKvPage;
            if (next + need > h->pool_order.size())
                return set_err(h, S2D_EFULL, "the KV pool has " + std::to_string(h->pool_order.size()) +
                                                 " pages; the batch needs more");
            for (int j = 0; j < h->kv_per_seq; ++j)
                table[(size_t)i * h->kv_per_seq + j] = h->pool_order[next + std::min((size_t)j, need - 1)];
            next += need;
        }
        CK(cudaMemcpyAsync(h->kv_page_table, table.data(), table.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                           h->stream));
    }
    for (int i = 0; i < n_seq; ++i)
        if ((rc = batch_admit_seq(h, i, prompts[i], rows, cols[i], k, rng_states[i], rng_kind, philox_key)))
            return rc;
    const uint32_t prefill_kernels = h->launches - launches0;
    // the batched attention's block order: longest context first (every
    // sequence advances one position per frame, so the order holds)
    std::vector<int32_t> order((size_t)n_seq);
    for (int i = 0; i < n_seq; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int32_t x, int32_t y) { return cols[x] > cols[y]; });
    CK(cudaMemcpyAsync(h->batch_order, order.data(), order.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                       h->stream));
    CK(cudaEventRecord(h->ev1, h->stream));

    // frames: one captured graph advances every sequence by one frame
    if ((rc = ensure_batch_graph(h, k, n_seq, rng_kind, philox_key))) return rc;
    const uint32_t poll = 8;
    std::vector<DevState> st((size_t)n_seq);
    uint32_t launched = 0;
    while (launched < p->max_new_tokens) {
        const uint32_t batch = std::min(poll, p->max_new_tokens - launched);
        for (uint32_t i = 0; i < batch; ++i) CK(cudaGraphLaunch(h->batch_exec, h->stream));
        launched += batch;
        CK(cudaMemcpyAsync(st.data(), h->st_b, st.size() * sizeof(DevState), cudaMemcpyDeviceToHost, h->stream));
        CK(cudaStreamSynchronize(h->stream));
        bool all_done = true, err = false;
        for (const DevState &x : st) all_done &= x.done != 0, err |= x.error != 0;
        if (all_done || err) break;
    }
    CK(cudaEventRecord(h->ev2, h->stream));
    CK(cudaMemcpyAsync(st.data(), h->st_b, st.size() * sizeof(DevState), cudaMemcpyDeviceToHost, h->stream));
    std::vector<int32_t> codes((size_t)n_seq * codes_stride);
    CK(cudaMemcpyAsync(codes.data(), h->codes_b, codes.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    if ((rc = check_device_error(h))) return rc;
    uint32_t total = 0;
    for (int i = 0; i < n_seq; ++i) {
        if (st[(size_t)i].error)
            return set_err(h, S2D_EDEVICE, "sequence " + std::to_string(i) + ": device error flag " +
                                               std::to_string(st[(size_t)i].error));
        if (!st[(size_t)i].done)
            return set_err(h, S2D_ESTATE, "sequence " + std::to_string(i) + ": generation did not finish");
        const uint32_t frames = (uint32_t)st[(size_t)i].step_index;
        // compact_codes (generate.rs:346-390), per sequence
        int32_t *dst = out_codes + (size_t)i * codes_stride;
        const int32_t *src = codes.data() + (size_t)i * codes_stride;
        for (int cb = 0; cb < K; ++cb)
            for (uint32_t t = 0; t < frames; ++t) dst[(size_t)cb * frames + t] = src[(size_t)cb * p->max_new_tokens + t];
        out_n_frames[i] = frames;
        rng_states[i] = st[(size_t)i].rng;
        total += frames;
    }
    if (profile) {
        float a = 0, b = 0;
        cudaEventElapsedTime(&a, h->ev0, h->ev1);
        cudaEventElapsedTime(&b, h->ev1, h->ev2);
        profile->prefill_ms = a;
        profile->decode_ms = b;
        profile->frames = total;
        profile->kernels_per_frame = h->batch_kernels;
        profile->prefill_kernels = prefill_kernels;
        profile->frame_launches = launched;
    }
    return S2D_OK;
}

// ---- continuous batching ---------------------------------------------------

namespace {

// The batched attention's block order over the session's slots: running
// slots by descending prompt length (their contexts grow in step), then the
// others.
int32_t serve_order(S2dHandle *h) {
    const int B = h->max_batch;
    std::vector<int32_t> order((size_t)B);
    for (int i = 0; i < B; ++i) order[(size_t)i] = i;
    std::stable_sort(order.begin(), order.end(),
                     [&](int32_t x, int32_t y) { return h->serve_cols[(size_t)x] > h->serve_cols[(size_t)y]; });
    CK(cudaMemcpyAsync(h->batch_order, order.data(), order.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                       h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return S2D_OK;
}

}  // namespace

int32_t s2d_serve_begin(S2dHandle *h, const S2dGenParams *p, int32_t rng_kind, uint64_t philox_key) {
    if (!h) return S2D_EINVAL;
    if (!p) return set_err(h, S2D_EINVAL, "s2d_serve_begin: NULL params");
    if (rng_kind != S2D_RNG_SEEDED && rng_kind != S2D_RNG_PHILOX) return set_err(h, S2D_EINVAL, "unknown rng_kind");
    if (p->max_new_tokens == 0) return set_err(h, S2D_EINVAL, "max_new_tokens must be positive");
    const int B = h->max_batch;
    if (B > kBatchMaxSeq)
        return set_err(h, S2D_EINVAL, "max_batch must be at most " + std::to_string(kBatchMaxSeq) + " for serving");
    if ((int64_t)p->max_new_tokens >= h->cfg.max_seq) return set_err(h, S2D_EINVAL, "max_new_tokens exceeds max_seq");
    CK(cudaSetDevice(h->device));
    const S2dGraphSpec &s = h->spec;
    int32_t rc;
    if ((rc = ensure_batch(h, p->max_new_tokens))) return rc;
    if ((s.linear_type != 1 || h->fast_out_wq != EW_F16) && (rc = ensure_f16_linears(h))) return rc;
    GenKey k;
    k.max_new = p->max_new_tokens, k.min_tokens = p->min_tokens_before_end, k.im_end = p->im_end_id;
    k.temperature = p->temperature, k.top_p = p->top_p, k.top_k = p->top_k;
    // every slot free: a finished DevState, so that every kernel skips it
    std::vector<DevState> st((size_t)B);
    for (DevState &x : st) x = DevState{}, x.done = 1;
    CK(cudaMemcpyAsync(h->st_b, st.data(), st.size() * sizeof(DevState), cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemsetAsync(h->codes_b, 0, (size_t)B * s.num_codebooks * p->max_new_tokens * sizeof(int32_t),
                       h->stream));
    h->serve_key = k, h->serve_rng_kind = rng_kind, h->serve_philox = philox_key;
    h->serve_cols.assign((size_t)B, -1);
    h->serve_pages.assign((size_t)B, {});
    h->serve_free = h->pool_order;  // the pool's pages, in the dealing (shuffled) order
    h->serving = true;
    if ((rc = ensure_batch_graph(h, k, B, rng_kind, philox_key))) return rc;
    if ((rc = serve_order(h))) return rc;
    return check_device_error(h);
}

int32_t s2d_serve_admit(S2dHandle *h, int32_t slot, const uint32_t *prompt, int32_t rows, int32_t cols,
                        uint64_t rng_state) {
    if (!h) return S2D_EINVAL;
    if (!h->serving) return set_err(h, S2D_ESTATE, "s2d_serve_admit needs s2d_serve_begin first");
    if (!prompt) return set_err(h, S2D_EINVAL, "s2d_serve_admit: NULL prompt");
    if (slot < 0 || slot >= h->max_batch) return set_err(h, S2D_EINVAL, "slot out of range");
    if (h->serve_cols[(size_t)slot] >= 0) return set_err(h, S2D_ESTATE, "slot is not free");
    if (rows != h->spec.num_codebooks + 1) return set_err(h, S2D_EINVAL, "prompt rows must be num_codebooks+1");
    if (cols <= 0) return set_err(h, S2D_EINVAL, "expected at least one prompt token");
    const GenKey &k = h->serve_key;
    if ((int64_t)cols + (int64_t)k.max_new > h->cfg.max_seq)
        return set_err(h, S2D_ESTATE, "prompt + max_new_tokens exceeds max_seq");
    // the pages of positions [0, cols + max_new): the prompt, then one per frame
    const size_t need = ((size_t)cols + k.max_new + kKvPage - 1) / kKvPage;
    if (need > h->serve_free.size())
        return set_err(h, S2D_EFULL, "not enough free KV pages: " + std::to_string(need) + " needed, " +
                                         std::to_string(h->serve_free.size()) + " free");
    CK(cudaSetDevice(h->device));
    std::vector<int32_t> row((size_t)h->kv_per_seq);
    std::vector<int32_t> pages(h->serve_free.begin(), h->serve_free.begin() + (ptrdiff_t)need);
    for (size_t j = 0; j < row.size(); ++j) row[j] = pages[std::min(j, need - 1)];  // unused entries: never read
    CK(cudaMemcpyAsync(h->kv_page_table + (size_t)slot * h->kv_per_seq, row.data(), row.size() * sizeof(int32_t),
                       cudaMemcpyHostToDevice, h->stream));
    const size_t codes_stride = (size_t)h->spec.num_codebooks * k.max_new;
    CK(cudaMemsetAsync(h->codes_b + (size_t)slot * codes_stride, 0, codes_stride * sizeof(int32_t), h->stream));
    int32_t rc = batch_admit_seq(h, slot, prompt, rows, cols, k, rng_state, h->serve_rng_kind, h->serve_philox);
    if (rc) {
        // leave the slot free and finished again
        DevState x{};
        x.done = 1;
        cudaMemcpyAsync(h->st_b + slot, &x, sizeof(DevState), cudaMemcpyHostToDevice, h->stream);
        cudaStreamSynchronize(h->stream);
        return rc;
    }
    h->serve_free.erase(h->serve_free.begin(), h->serve_free.begin() + (ptrdiff_t)need);
    h->serve_pages[(size_t)slot] = std::move(pages);
    h->serve_cols[(size_t)slot] = cols;
    if ((rc = serve_order(h))) return rc;
    return check_device_error(h);
}

int32_t s2d_serve_step(S2dHandle *h, int32_t n_frames, int32_t *slot_status, uint32_t *slot_frames) {
    if (!h) return S2D_EINVAL;
    if (!h->serving) return set_err(h, S2D_ESTATE, "s2d_serve_step needs s2d_serve_begin first");
    if (n_frames < 0) return set_err(h, S2D_EINVAL, "n_frames must not be negative");
    CK(cudaSetDevice(h->device));
    const int B = h->max_batch;
    std::vector<DevState> st((size_t)B);
    bool running = false;
    for (int i = 0; i < B; ++i) running |= h->serve_cols[(size_t)i] >= 0;
    if (running)
        for (int32_t f = 0; f < n_frames; ++f) CK(cudaGraphLaunch(h->batch_exec, h->stream));
    CK(cudaMemcpyAsync(st.data(), h->st_b, st.size() * sizeof(DevState), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    int32_t rc;
    if ((rc = check_device_error(h))) return rc;
    for (int i = 0; i < B; ++i) {
        const DevState &x = st[(size_t)i];
        if (x.error)
            return set_err(h, S2D_EDEVICE, "slot " + std::to_string(i) + ": device error flag " + std::to_string(x.error));
        const bool busy = h->serve_cols[(size_t)i] >= 0;
        if (slot_status) slot_status[i] = !busy ? S2D_SLOT_FREE : x.done ? S2D_SLOT_FINISHED : S2D_SLOT_RUNNING;
        if (slot_frames) slot_frames[i] = busy ? (uint32_t)x.step_index : 0u;
    }
    return S2D_OK;
}

int32_t s2d_serve_collect(S2dHandle *h, int32_t slot, int32_t *out_codes, uint32_t *out_n_frames,
                          uint64_t *rng_state) {
    if (!h) return S2D_EINVAL;
    if (!h->serving) return set_err(h, S2D_ESTATE, "s2d_serve_collect needs s2d_serve_begin first");
    if (!out_codes || !out_n_frames) return set_err(h, S2D_EINVAL, "s2d_serve_collect: NULL argument");
    if (slot < 0 || slot >= h->max_batch) return set_err(h, S2D_EINVAL, "slot out of range");
    if (h->serve_cols[(size_t)slot] < 0) return set_err(h, S2D_ESTATE, "slot holds no request");
    CK(cudaSetDevice(h->device));
    const int K = h->spec.num_codebooks;
    const uint32_t max_new = h->serve_key.max_new;
    DevState x{};
    std::vector<int32_t> codes((size_t)K * max_new);
    CK(cudaMemcpyAsync(&x, h->st_b + slot, sizeof(DevState), cudaMemcpyDeviceToHost, h->stream));
    CK(cudaMemcpyAsync(codes.data(), h->codes_b + (size_t)slot * codes.size(), codes.size() * sizeof(int32_t),
                       cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    if (!x.done) return set_err(h, S2D_ESTATE, "slot " + std::to_string(slot) + " has not finished");
    // compact_codes (generate.rs:346-390)
    const uint32_t frames = (uint32_t)x.step_index;
    for (int cb = 0; cb < K; ++cb)
        for (uint32_t t = 0; t < frames; ++t) out_codes[(size_t)cb * frames + t] = codes[(size_t)cb * max_new + t];
    *out_n_frames = frames;
    if (rng_state) *rng_state = x.rng;
    std::vector<int32_t> &pg = h->serve_pages[(size_t)slot];
    h->serve_free.insert(h->serve_free.end(), pg.begin(), pg.end());
    pg.clear();
    h->serve_cols[(size_t)slot] = -1;
    return serve_order(h);
}

int32_t s2d_serve_free_pages(const S2dHandle *h, int32_t *out) {
    if (!h || !out) return S2D_EINVAL;
    *out = h->serving ? (int32_t)h->serve_free.size() : 0;
    return S2D_OK;
}

int32_t s2d_profile_batch(S2dHandle *h, int32_t n_seq, double *out_ms, int32_t n_out) {
    if (!h || !out_ms || n_out <= 0) return S2D_EINVAL;
    if (!h->st_b || h->batch_n <= 0)
        return set_err(h, S2D_ESTATE, "s2d_profile_batch needs a previous s2d_generate_codes_batch call");
    if (n_seq <= 0 || n_seq > h->batch_n)
        return set_err(h, S2D_EINVAL, "n_seq must be in 1..the last batch's sequence count");
    CK(cudaSetDevice(h->device));
    // every sequence active again for one more frame (codes are not stored)
    for (int i = 0; i < n_seq; ++i) CK(cudaMemsetAsync(&h->st_b[i].done, 0, sizeof(int32_t), h->stream));
    std::vector<std::pair<int, cudaEvent_t>> marks;
    cudaEvent_t start = nullptr;
    CK(cudaEventCreate(&start));
    CK(cudaEventRecord(start, h->stream));
    h->marks = &marks;
    h->batch_profile = true;
    const int32_t rc = enqueue_frame_batch(h, h->batch_key, n_seq, h->batch_rng_kind, h->batch_philox);
    h->marks = nullptr;
    h->batch_profile = false;
    cudaError_t e = cudaStreamSynchronize(h->stream);
    double sums[PC_COUNT + 1] = {0};
    cudaEvent_t prev = start;
    for (auto &m : marks) {
        float ms = 0.f;
        if (!e) cudaEventElapsedTime(&ms, prev, m.second);
        sums[m.first] += ms;
        sums[PC_COUNT] += ms;
        prev = m.second;
    }
    for (auto &m : marks) cudaEventDestroy(m.second);
    cudaEventDestroy(start);
    // this extra frame may reach max_seq for some sequence: not an error here
    cudaMemsetAsync(&h->st->error, 0, sizeof(int32_t), h->stream);
    for (int i = 0; i < n_seq; ++i) cudaMemsetAsync(&h->st_b[i].done, 0xff, sizeof(int32_t), h->stream);
    cudaStreamSynchronize(h->stream);
    if (rc) return rc;
    if (e) return set_err(h, S2D_ECUDA, std::string("profile_batch: ") + cudaGetErrorString(e));
    for (int i = 0; i < n_out && i <= PC_COUNT; ++i) out_ms[i] = sums[i];
    return S2D_OK;
}

int32_t s2d_philox4x32_10(const uint32_t *counter, const uint32_t *key, uint32_t *out) {
    if (!counter || !key || !out) return S2D_EINVAL;
    uint32_t *dev = nullptr;
    if (cudaMalloc(&dev, 4 * sizeof(uint32_t)) != cudaSuccess) return S2D_ENOMEM;
    cudaError_t e = launch_philox(counter, key, dev, nullptr);
    if (!e) e = cudaMemcpy(out, dev, 4 * sizeof(uint32_t), cudaMemcpyDeviceToHost);
    cudaFree(dev);
    return e ? S2D_ECUDA : S2D_OK;
}

int32_t s2d_dequant_tensor(S2dHandle *h, const char *name, float *out, int64_t n) {
    if (!h || !name || !out) return S2D_EINVAL;
    const GgufTensor *t = h->gguf.tensor(name);
    if (!t) return set_err(h, S2D_EINVAL, std::string("tensor not found: ") + name);
    if ((uint64_t)n != t->elements) return set_err(h, S2D_EINVAL, "element count mismatch");
    CK(cudaSetDevice(h->device));
    float *dst = nullptr;
    CK(cudaMalloc(&dst, (size_t)n * sizeof(float)));
    cudaError_t e;
    if (t->type == 1) e = launch_f16_to_f32(reinterpret_cast<const uint16_t *>(tdev(h, t)->dev), dst, n, h->stream);
    else if (t->type == 0) e = cudaMemcpyAsync(dst, tdev(h, t)->dev, (size_t)n * 4, cudaMemcpyDeviceToDevice, h->stream);
    else if (t->type == 8 || t->type == 12) e = launch_dequant((int)t->type, tdev(h, t)->dev, dst, n, h->stream);
    else e = cudaErrorNotSupported;
    if (!e) e = cudaMemcpyAsync(out, dst, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost, h->stream);
    if (!e) e = cudaStreamSynchronize(h->stream);
    cudaFree(dst);
    if (e) return set_err(h, S2D_ECUDA, std::string("dequant: ") + cudaGetErrorString(e));
    return S2D_OK;
}

int32_t s2d_profile_kernel(S2dHandle *h, int32_t kernel, int32_t iters, double *avg_ms, double *bytes) {
    if (!h || !avg_ms || !bytes || iters <= 0) return S2D_EINVAL;
    CK(cudaSetDevice(h->device));
    const S2dGraphSpec &s = h->spec;
    const ArShape &a = h->slow;
    const int d = s.hidden;
    // finite activations for the inputs the kernels read
    CK(cudaMemsetAsync(h->x, 0, (size_t)kMaxM * d * sizeof(float), h->stream));
    CK(cudaMemsetAsync(h->att, 0, (size_t)kMaxM * a.qs() * sizeof(float), h->stream));
    CK(cudaMemsetAsync(h->act, 0, (size_t)kMaxM * a.F * sizeof(float), h->stream));
    auto args = [&](int l, int *epi) {
        const LayerDev &L = h->slow_layers[(size_t)l];
        GemvArgs g{};
        g.n_contig = -1;
        switch (kernel) {
        case S2D_KERNEL_WQKV:
            g.W = L.wqkv, g.x = h->x, g.ldx = d, g.norm_w = L.attn_norm, g.eps = a.eps;
            g.y = h->qkv, g.ldy = a.qkv_out(), g.K = d, g.N = a.qkv_out(), *epi = EPI_STORE;
            break;
        case S2D_KERNEL_WO:
            g.W = L.wo, g.x = h->att, g.ldx = a.qs(), g.y = h->x, g.ldy = d, g.resid = h->x, g.ldr = d;
            g.K = a.qs(), g.N = d, *epi = EPI_RESID;
            break;
        case S2D_KERNEL_W13:
            g.W = L.w1, g.W2 = L.w3, g.x = h->x, g.ldx = d, g.norm_w = L.ffn_norm, g.eps = a.eps;
            g.y = h->act, g.ldy = a.F, g.K = d, g.N = a.F, *epi = EPI_SWIGLU_SLOW;
            break;
        case S2D_KERNEL_W2:
            g.W = L.w2, g.x = h->act, g.ldx = a.F, g.y = h->x, g.ldy = d, g.resid = h->x, g.ldr = d;
            g.K = a.F, g.N = d, *epi = EPI_RESID;
            break;
        default: {
            const int nsem = s.semantic_end_id - s.semantic_begin_id + 1;
            g.W = h->emb, g.x = h->x, g.ldx = d, g.norm_w = h->norm, g.eps = a.eps;
            g.y = h->logits, g.ldy = s.vocab_size, g.x_out = h->hidden_post, g.K = d;
            // a different block of rows per launch so that no launch hits L2
            const int span = nsem + 1;
            const int base = (int)(((int64_t)l * span) % std::max(1, s.vocab_size - span));
            g.row_base = base, g.n_contig = nsem, g.extra_row = base + nsem;
            g.N = span, *epi = EPI_STORE;
        }
        }
        return g;
    };
    if (kernel < S2D_KERNEL_WQKV || kernel > S2D_KERNEL_LM_HEAD) return set_err(h, S2D_EINVAL, "unknown kernel");
    if (kernel != S2D_KERNEL_LM_HEAD && h->slow_layers[0].wq != EW_F16)
        return set_err(h, S2D_EINVAL, "profile_kernel times the f16 GEMV kernels; this model's linears are quantized");
    int epi = 0;
    GemvArgs g0 = args(0, &epi);
    const double wbytes = (double)g0.K * g0.N * 2.0 * (g0.W2 ? 2 : 1);
    *bytes = wbytes + (double)g0.K * 4.0 + (double)g0.N * 4.0 * (epi == EPI_RESID ? 2 : 1);
    for (int i = 0; i < 3; ++i) CK(launch_gemv(args(i % a.L, &epi), 1, epi, h->stream, h->pdl));
    CK(cudaEventRecord(h->ev0, h->stream));
    for (int i = 0; i < iters; ++i) {
        const int l = kernel == S2D_KERNEL_LM_HEAD ? i : i % a.L;
        CK(launch_gemv(args(l, &epi), 1, epi, h->stream, h->pdl));
    }
    CK(cudaEventRecord(h->ev1, h->stream));
    CK(cudaEventSynchronize(h->ev1));
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, h->ev0, h->ev1));
    *avg_ms = ms / iters;
    return S2D_OK;
}

int32_t s2d_profile_engine(S2dHandle *h, int32_t program, uint64_t *trace, int64_t trace_cap,
                           int32_t *n_ops, double *ms) {
    if (!h || !n_ops || !ms) return S2D_EINVAL;
    if (!h->use_engine) return set_err(h, S2D_ESTATE, "the persistent engine is not in use");
    CK(cudaSetDevice(h->device));
    int32_t rc = build_programs(h, h->slow_prog.ops ? h->slow_prog_im_end : 0xffffffffu);
    if (rc) return rc;
    if (program < -1 || program >= (int)h->fast_progs.size()) return set_err(h, S2D_EINVAL, "no such program");
    const EngineProgram &p = program == -1  ? h->fast_frame_prog
                             : program == 0 ? h->slow_prog
                                            : h->fast_progs[(size_t)program];
    if (!p.ops) return set_err(h, S2D_EINVAL, "no such program");
    *n_ops = p.n_ops;
    unsigned long long *dtr = nullptr;
    const size_t need = (size_t)p.n_ops * (8 + h->num_sms);
    if (trace) {
        if ((int64_t)need > trace_cap) return set_err(h, S2D_EINVAL, "trace buffer too small");
        CK(cudaMalloc(&dtr, need * sizeof(unsigned long long)));
        CK(cudaMemsetAsync(dtr, 0, need * sizeof(unsigned long long), h->stream));
    }
    EngineArgs a{};
    a.ops = p.ops, a.n_ops = p.n_ops, a.nslots = p.nslots, a.slot_bytes = h->slot_bytes;
    a.area_bytes = p.area_bytes, a.epoch = h->engine_epoch, a.done = nullptr, a.error = &h->st->error;
    a.l2_lead = h->l2_lead;
    a.trace = dtr;
    cudaError_t e = cudaEventRecord(h->ev0, h->stream);
    if (!e) e = launch_engine(a, h->num_sms, p.smem, h->stream, p.frame);
    if (!e) e = cudaEventRecord(h->ev1, h->stream);
    if (!e) e = cudaEventSynchronize(h->ev1);
    float t = 0.f;
    if (!e) e = cudaEventElapsedTime(&t, h->ev0, h->ev1);
    if (!e && trace) e = cudaMemcpy(trace, dtr, need * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    if (dtr) cudaFree(dtr);
    if (e) return set_err(h, S2D_ECUDA, std::string("profile_engine: ") + cudaGetErrorString(e));
    *ms = t;
    return check_device_error(h);
}

// ---- op-level seam -------------------------------------------------------

namespace {
struct DevBuf {
    void *p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};
}  // namespace

int32_t s2d_op_linear_f16(S2dHandle *h, const float *input, const uint16_t *w, int64_t in_dim, int64_t out_dim,
                          float *out) {
    if (!input || !w || !out || in_dim <= 0 || out_dim <= 0) return set_err(h, S2D_EINVAL, "bad arguments");
    if (in_dim % 8) return set_err(h, S2D_EINVAL, "in_dim must be a multiple of 8");
    if (in_dim * 4 > 200 * 1024) return set_err(h, S2D_EINVAL, "in_dim too large for the op-level GEMV");
    cudaStream_t st = h ? h->stream : nullptr;
    if (h) CK(cudaSetDevice(h->device));
    DevBuf x, W, y;
    CK(configure_kernels());
    CK(cudaMalloc(&x.p, (size_t)in_dim * 4));
    CK(cudaMalloc(&W.p, (size_t)in_dim * out_dim * 2));
    CK(cudaMalloc(&y.p, (size_t)out_dim * 4));
    CK(cudaMemcpyAsync(x.p, input, (size_t)in_dim * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(W.p, w, (size_t)in_dim * out_dim * 2, cudaMemcpyHostToDevice, st));
    GemvArgs g{};
    g.W = (const uint16_t *)W.p, g.x = (const float *)x.p, g.ldx = (int)in_dim, g.y = (float *)y.p;
    g.ldy = (int)out_dim, g.K = (int)in_dim, g.N = (int)out_dim, g.n_contig = -1;
    CK(launch_gemv(g, 1, EPI_STORE, st, false));
    CK(cudaMemcpyAsync(out, y.p, (size_t)out_dim * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return S2D_OK;
}

int32_t s2d_op_rows_linear_f16(S2dHandle *h, const float *x, int64_t T, int64_t K, const uint16_t *w,
                               const uint16_t *w2, int64_t N, const float *resid, int32_t epi, int32_t impl, float *y) {
    if (!h) return S2D_EINVAL;
    if (!x || !w || !y || T <= 0 || K <= 0 || N <= 0 || epi < 0 || epi > 3 || (epi >= 2) != (w2 != nullptr) ||
        (epi == 1 && !resid))
        return set_err(h, S2D_EINVAL, "s2d_op_rows_linear_f16: bad arguments");
    if (T > kPrefillChunk) return set_err(h, S2D_EINVAL, "at most 512 rows per call");
    if (K % 8 || K * 4 > 64 * 1024) return set_err(h, S2D_EINVAL, "K must be a multiple of 8 and at most 16384");
    CK(cudaSetDevice(h->device));
    int32_t rc;
    if ((rc = ensure_prefill(h))) return rc;  // the cuBLAS handle
    // row buffers of this call's size, in place of the handle's for its duration
    DevBuf dx, dw, dw2, dy, xs, inv, y2, y2b;
    CK(cudaMalloc(&xs.p, (size_t)2 * T * K * sizeof(__half)));
    CK(cudaMalloc(&inv.p, (size_t)T * sizeof(float)));
    CK(cudaMalloc(&y2.p, (size_t)2 * T * N * sizeof(float)));
    CK(cudaMalloc(&y2b.p, (size_t)2 * T * N * sizeof(float)));
    struct Swap {
        S2dHandle *h;
        __half *xs;
        float *inv, *y2, *y2b;
        ~Swap() { h->pf_xs = xs, h->pf_inv = inv, h->pf_y2 = y2, h->pf_y2b = y2b; }
    } keep{h, h->pf_xs, h->pf_inv, h->pf_y2, h->pf_y2b};
    h->pf_xs = (__half *)xs.p, h->pf_inv = (float *)inv.p, h->pf_y2 = (float *)y2.p, h->pf_y2b = (float *)y2b.p;
    CK(cudaMalloc(&dx.p, (size_t)T * K * 4));
    CK(cudaMalloc(&dw.p, (size_t)N * K * 2));
    if (w2) CK(cudaMalloc(&dw2.p, (size_t)N * K * 2));
    CK(cudaMalloc(&dy.p, (size_t)T * N * 4));
    CK(cudaMemcpyAsync(dx.p, x, (size_t)T * K * 4, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(dw.p, w, (size_t)N * K * 2, cudaMemcpyHostToDevice, h->stream));
    if (w2) CK(cudaMemcpyAsync(dw2.p, w2, (size_t)N * K * 2, cudaMemcpyHostToDevice, h->stream));
    if (resid) CK(cudaMemcpyAsync(dy.p, resid, (size_t)T * N * 4, cudaMemcpyHostToDevice, h->stream));
    CK(launch_split_rows((const float *)dx.p, (int)K, (int)T, (int)K, nullptr, 0.f, h->pf_xs, h->pf_inv, nullptr,
                         h->stream));
    const bool tc = h->use_tc;
    h->use_tc = impl == 0;
    if (impl == 0) {
        TcGemm g;
        g.W = (const uint16_t *)dw.p, g.W2 = (const uint16_t *)dw2.p, g.N = (int)N, g.K = (int)K, g.xs = h->pf_xs;
        g.T = (int)T, g.inv = h->pf_inv, g.epi = epi, g.y = (float *)dy.p, g.ldy = (int)N;
        if (!tc_gemm_supported(g)) {
            h->use_tc = tc;
            return set_err(h, S2D_EINVAL, "the tensor-core GEMM does not take this shape");
        }
    }
    rc = rows_linear(h, (const uint16_t *)dw.p, (const uint16_t *)dw2.p, (int)N, (int)K, (int)T, epi, (float *)dy.p,
                     (int)N, (const float *)dy.p, (int)N);
    h->use_tc = tc;
    if (rc) return rc;
    CK(cudaMemcpyAsync(y, dy.p, (size_t)T * N * 4, cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return check_device_error(h);
}

int32_t s2d_op_batch_attention(S2dHandle *h, const float *q, const uint16_t *kcache, const uint16_t *vcache,
                               int64_t B, int64_t H, int64_t Hkv, int64_t head_dim, int64_t max_seq,
                               const int32_t *n_past, const int32_t *done, int32_t splits, int32_t impl, float *out) {
    if (!h) return S2D_EINVAL;
    if (!q || !kcache || !vcache || !n_past || !out || B <= 0 || B > 4096 || Hkv <= 0 || H % Hkv ||
        H / Hkv > 8 || (head_dim != 64 && head_dim != 128) || max_seq <= 0 || max_seq > (1 << 20) || splits < 0 ||
        splits > 64 || impl < 0 || impl > 1)
        return set_err(h, S2D_EINVAL, "s2d_op_batch_attention: bad arguments");
    for (int64_t b = 0; b < B; ++b)
        if (n_past[b] < 0 || n_past[b] >= max_seq)
            return set_err(h, S2D_EINVAL, "s2d_op_batch_attention: n_past out of range");
    CK(cudaSetDevice(h->device));
    const size_t per_seq = (size_t)Hkv * max_seq * head_dim, nq = (size_t)B * H * head_dim;
    const int S = splits ? splits : std::max(1, std::min(16, (int)((h->attn_mma_blocks_per_sm * h->num_sms +
                                                                    B * Hkv - 1) / (B * Hkv))));
    std::vector<DevState> st((size_t)B);
    for (int64_t b = 0; b < B; ++b) st[b] = DevState{}, st[b].n_past = n_past[b], st[b].done = done ? done[b] : 0;
    DevBuf dq, dk, dv, dout, dst, part, cnt;
    CK(cudaMalloc(&dq.p, nq * 4));
    CK(cudaMalloc(&dk.p, (size_t)B * per_seq * 2));
    CK(cudaMalloc(&dv.p, (size_t)B * per_seq * 2));
    CK(cudaMalloc(&dout.p, nq * 4));
    CK(cudaMalloc(&dst.p, (size_t)B * sizeof(DevState)));
    CK(cudaMalloc(&part.p, nq / head_dim * S * (head_dim + 2) * 4));
    CK(cudaMalloc(&cnt.p, (size_t)B * Hkv * 4));
    CK(cudaMemsetAsync(cnt.p, 0, (size_t)B * Hkv * 4, h->stream));
    CK(cudaMemsetAsync(dout.p, 0, nq * 4, h->stream));
    CK(cudaMemcpyAsync(dq.p, q, nq * 4, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(dk.p, kcache, (size_t)B * per_seq * 2, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(dv.p, vcache, (size_t)B * per_seq * 2, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(dst.p, st.data(), (size_t)B * sizeof(DevState), cudaMemcpyHostToDevice, h->stream));
    RowsAttnArgs t{};
    t.q = (const float *)dq.p, t.kcache = dk.p, t.vcache = dv.p, t.kv_seq_stride = per_seq, t.max_seq = (int)max_seq;
    t.out = (float *)dout.p, t.T = (int)B, t.rows_per_seq = 1, t.st = (const DevState *)dst.p, t.st_pos = 1;
    t.pos_const = 0, t.H = (int)H, t.Hkv = (int)Hkv, t.hd = (int)head_dim;
    t.scale = 1.0f / sqrtf((float)head_dim), t.S = S, t.part = (float *)part.p, t.counters = (int32_t *)cnt.p;
    t.decode_stages = impl == 0 ? h->attn_mma_stages : h->attn_stages;
    t.decode_mma = impl == 0, t.decode_warps = h->attn_mma_warps, t.decode_chunk = h->attn_mma_chunk;
    std::vector<int32_t> order((size_t)B);
    for (int64_t b = 0; b < B; ++b) order[b] = (int32_t)b;
    std::stable_sort(order.begin(), order.end(), [&](int32_t x, int32_t y) { return n_past[x] > n_past[y]; });
    DevBuf dorder;
    CK(cudaMalloc(&dorder.p, (size_t)B * sizeof(int32_t)));
    CK(cudaMemcpyAsync(dorder.p, order.data(), (size_t)B * sizeof(int32_t), cudaMemcpyHostToDevice, h->stream));
    t.row_order = (const int32_t *)dorder.p;
    if (impl == 0 && !decode_mma_supported(t, true))
        return set_err(h, S2D_EINVAL, "the tensor-core attention does not take these arguments");
    CK(launch_rows_attention(t, true, h->stream));
    CK(cudaMemcpyAsync(out, dout.p, nq * 4, cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return S2D_OK;
}

int32_t s2d_op_prefill_attention(S2dHandle *h, const float *q, const uint16_t *kcache, const uint16_t *vcache,
                                 int64_t T, int64_t H, int64_t Hkv, int64_t head_dim, int64_t max_seq, int64_t pos0,
                                 int32_t impl, float *out) {
    if (!h) return S2D_EINVAL;
    if (!q || !kcache || !vcache || !out || T <= 0 || T > 4096 || Hkv <= 0 || H % Hkv || H / Hkv > 8 ||
        (head_dim != 64 && head_dim != 128) || max_seq <= 0 || max_seq > (1 << 20) || pos0 < 0 ||
        pos0 + T > max_seq || impl < 0 || impl > 2)
        return set_err(h, S2D_EINVAL, "s2d_op_prefill_attention: bad arguments");
    CK(cudaSetDevice(h->device));
    const size_t kvn = (size_t)Hkv * max_seq * head_dim, nq = (size_t)T * H * head_dim;
    DevBuf dq, dk, dv, dout;
    CK(cudaMalloc(&dq.p, nq * 4));
    CK(cudaMalloc(&dk.p, kvn * 2));
    CK(cudaMalloc(&dv.p, kvn * 2));
    CK(cudaMalloc(&dout.p, nq * 4));
    CK(cudaMemcpyAsync(dq.p, q, nq * 4, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(dk.p, kcache, kvn * 2, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(dv.p, vcache, kvn * 2, cudaMemcpyHostToDevice, h->stream));
    RowsAttnArgs t{};
    t.q = (const float *)dq.p, t.kcache = dk.p, t.vcache = dv.p, t.kv_seq_stride = 0, t.max_seq = (int)max_seq;
    t.out = (float *)dout.p, t.T = (int)T, t.rows_per_seq = (int)T, t.st = nullptr, t.st_pos = 0;
    t.pos_const = (int)pos0, t.H = (int)H, t.Hkv = (int)Hkv, t.hd = (int)head_dim;
    t.scale = 1.0f / sqrtf((float)head_dim), t.S = 1, t.decode_stages = 2, t.prefill_mma = impl == 0;
    t.k_rows = t.v_rows = (size_t)Hkv * max_seq, t.error = &h->st->error;
    if (impl == 0 && !prefill_mma_supported(t, true))
        return set_err(h, S2D_EINVAL, "the tensor-core prefill attention does not take these arguments");
    if (impl == 2 && !prefill_tc_supported(t, true))
        return set_err(h, S2D_EINVAL, "the tcgen05 prefill attention does not take these arguments");
    if (impl == 0) CK(launch_prefill_mma_attention(t, h->stream));
    else if (impl == 2) CK(launch_prefill_tc_attention(t, h->stream));
    else CK(launch_rows_attention(t, true, h->stream));
    if (impl == 2) {
        int32_t rc = check_device_error(h);
        if (rc) return rc;
    }
    CK(cudaMemcpyAsync(out, dout.p, nq * 4, cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return S2D_OK;
}

int32_t s2d_op_rms_norm(S2dHandle *h, const float *input, const float *weight, int64_t n, int64_t head_dim,
                        float eps, float *out) {
    if (!input || !weight || !out || n <= 0 || head_dim <= 0 || n % head_dim)
        return set_err(h, S2D_EINVAL, "bad arguments");
    cudaStream_t st = h ? h->stream : nullptr;
    if (h) CK(cudaSetDevice(h->device));
    DevBuf x, w, y;
    CK(cudaMalloc(&x.p, (size_t)n * 4));
    CK(cudaMalloc(&w.p, (size_t)head_dim * 4));
    CK(cudaMalloc(&y.p, (size_t)n * 4));
    CK(cudaMemcpyAsync(x.p, input, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(w.p, weight, (size_t)head_dim * 4, cudaMemcpyHostToDevice, st));
    CK(launch_rms_norm_heads((const float *)x.p, (const float *)w.p, (float *)y.p, n, (int)head_dim, eps, st));
    CK(cudaMemcpyAsync(out, y.p, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return S2D_OK;
}

int32_t s2d_op_rope_normal(S2dHandle *h, const float *values, int64_t n, int64_t head_dim, int64_t position,
                           float rope_base, float *out) {
    if (!values || !out || n <= 0 || head_dim <= 0 || n % head_dim || position < 0 || position > INT32_MAX)
        return set_err(h, S2D_EINVAL, "bad arguments");
    if (head_dim != 64 && head_dim != 128 && head_dim != 256)
        return set_err(h, S2D_EINVAL, "head_dim must be 64, 128 or 256");
    cudaStream_t st = h ? h->stream : nullptr;
    if (h) CK(cudaSetDevice(h->device));
    // the denominators as the model's tables hold them (alloc_buffers)
    std::vector<float> den((size_t)head_dim / 2);
    for (int64_t p = 0; p < head_dim; p += 2) den[(size_t)p / 2] = powf(rope_base, (float)p / (float)head_dim);
    DevBuf x, dn, y;
    CK(cudaMalloc(&x.p, (size_t)n * 4));
    CK(cudaMalloc(&dn.p, den.size() * 4));
    CK(cudaMalloc(&y.p, (size_t)n * 4));
    CK(cudaMemcpyAsync(x.p, values, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(dn.p, den.data(), den.size() * 4, cudaMemcpyHostToDevice, st));
    // every head as a query head of rope_kv_kernel: no QK-norm, no KV write
    RopeArgs a{};
    a.qkv = (const float *)x.p, a.ld_qkv = (int)n, a.q_out = (float *)y.p;
    a.rope_denom = (const float *)dn.p, a.pos_const = (int)position;
    a.H = (int)(n / head_dim), a.Hkv = 0, a.hd = (int)head_dim, a.M = 1, a.max_seq = 1;
    CK(launch_rope_kv(a, false, st, false));
    CK(cudaMemcpyAsync(out, y.p, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return S2D_OK;
}

int32_t s2d_op_gqa_decode_attention(S2dHandle *h, const float *query, const float *keys, const float *values,
                                    int32_t H, int32_t Hkv, int32_t hd, int32_t T, float scale, float *out) {
    if (!query || !keys || !values || !out || Hkv <= 0 || H % Hkv || hd <= 0 || T <= 0)
        return set_err(h, S2D_EINVAL, "invalid GQA split or attention dims");
    if (hd % 64 || hd > 256 || H / Hkv > 16) return set_err(h, S2D_EINVAL, "unsupported head_dim or group size");
    cudaStream_t st = h ? h->stream : nullptr;
    if (h) CK(cudaSetDevice(h->device));
    // token-major [T][Hkv][hd] -> per-head [Hkv][T][hd]
    std::vector<float> kt((size_t)Hkv * T * hd), vt((size_t)Hkv * T * hd);
    for (int t = 0; t < T; ++t)
        for (int k = 0; k < Hkv; ++k)
            for (int e = 0; e < hd; ++e) {
                kt[((size_t)k * T + t) * hd + e] = keys[((size_t)t * Hkv + k) * hd + e];
                vt[((size_t)k * T + t) * hd + e] = values[((size_t)t * Hkv + k) * hd + e];
            }
    const int S = std::max(1, std::min(16, T / 8));
    DevBuf q, K, V, o, part, cnt;
    CK(cudaMalloc(&q.p, (size_t)H * hd * 4));
    CK(cudaMalloc(&K.p, kt.size() * 4));
    CK(cudaMalloc(&V.p, vt.size() * 4));
    CK(cudaMalloc(&o.p, (size_t)H * hd * 4));
    CK(cudaMalloc(&part.p, (size_t)H * S * (hd + 2) * 4));
    CK(cudaMalloc(&cnt.p, (size_t)Hkv * 4));
    CK(cudaMemsetAsync(cnt.p, 0, (size_t)Hkv * 4, st));
    CK(cudaMemcpyAsync(q.p, query, (size_t)H * hd * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(K.p, kt.data(), kt.size() * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(V.p, vt.data(), vt.size() * 4, cudaMemcpyHostToDevice, st));
    AttnArgs a{};
    a.q = (const float *)q.p, a.kcache = K.p, a.vcache = V.p, a.max_seq = T, a.out = (float *)o.p;
    a.part = (float *)part.p, a.counters = (int32_t *)cnt.p, a.pos_const = T - 1;
    a.H = H, a.Hkv = Hkv, a.hd = hd, a.S = S, a.M = 1, a.scale = scale;
    CK(launch_attention(a, false, st, false));
    CK(cudaMemcpyAsync(out, o.p, (size_t)H * hd * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return S2D_OK;
}

}  // extern "C"
