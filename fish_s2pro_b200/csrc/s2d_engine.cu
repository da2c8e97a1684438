// s2d_engine.cu -- persistent decode layer engine for sm_100a.
//
// One launch runs a whole program of decode ops (every linear, QK-norm,
// RoPE, KV write and GQA attention of a Slow-AR step or a Fast-AR pass, plus
// the output head): the work of SlowArLayerSkeleton::forward_decode_token +
// forward_feed_forward (slow_ar.rs:637-854) for each layer in turn,
// FastArLayerSkeleton (fast_ar.rs:245-352), forward_logits
// (slow_ar.rs:943-955) and the Fast-AR head (fast_ar.rs:429-435).
//
// Layout: one CTA per SM (cooperative launch).  Warp 8 of each CTA is a
// producer: its lane 0 walks the program and streams this CTA's rows of
// every linear, in program order, into a ring of shared-memory slots with
// cp.async.bulk and mbarrier completion.  Weights do not depend on
// activations, so the producer runs ahead across op and layer boundaries,
// limited only by the ring, and HBM stays busy while the consumers wait for
// inputs or run attention.  Warps 0-7 consume: for each op they poll its
// input words (LL words, see EngineOp) until the producing op's tag appears,
// stage the input vector (with its RMSNorm) in shared memory, then every
// warp reads every slot, each warp owning a few rows of it (see GemvTiling).
// Every wait is bounded: on timeout the kernel records an error code in
// DevState::error and returns.
#include <math.h>

#include "s2d_common.cuh"
#include "s2d_kernels.cuh"
#include "s2d_sample.cuh"

namespace s2d {

namespace {

// Bounds of every wait (about a second each): a healthy launch never comes
// close; a broken one records an error and returns instead of hanging.
constexpr uint32_t kMbarSpin = 1u << 20;   // try_wait rounds of <= 1 us each

__device__ __forceinline__ uint32_t saddr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ int32_t ld_volatile(const int32_t *p) {
    return *reinterpret_cast<const volatile int32_t *>(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}


// Wait for `parity` of an mbarrier, giving up (and flagging `code`) after a
// bounded number of rounds or when another CTA has already flagged an error.
__device__ bool mbar_wait(uint64_t *bar, uint32_t parity, int32_t *err, int32_t code,
                          bool honor_error = true) {
    for (uint32_t i = 0; i < kMbarSpin; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (honor_error && (i & 1023u) == 1023u && ld_volatile(err)) return false;
    }
    atomicCAS(err, 0, code);
    return false;
}

__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            saddr(dst)),
        "l"(src), "r"(bytes), "r"(saddr(bar))
        : "memory");
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kEngineConsumerWarps * 32) : "memory");
}
// consumers_sync that also returns whether any consumer thread passed true.
__device__ __forceinline__ bool consumers_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kEngineConsumerWarps * 32)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void group_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// GEMV tiling
//
// A CTA's rows of an op are cut into row tiles of at most rmax rows
// (engine_slice_geom, engine_tile_rows); a tile is streamed through the ring
// in K slices, one slot per slice.  The weights were laid out at load
// time in exactly this order (engine_relayout), so each slot is one
// contiguous bulk copy of [mat][R][kw] f16.  Consumer warp w owns rows
// w, w + 8, w + 16, w + 24 of the tile and its lanes split each row's
// 16-byte column chunks; a row's 32 partial sums meet at the end of the tile.
// ---------------------------------------------------------------------------

constexpr int kRowsPerWarp = kEngineTileRows / kEngineConsumerWarps;  // 4
static_assert(kRowsPerWarp * kEngineConsumerWarps == kEngineTileRows, "tile mapping");

struct GemvTiling {
    int r0, n, ntiles, mats, K, wt;
    SliceGeom sg;
    __device__ __forceinline__ GemvTiling(const EngineOp &op, int slot_bytes) {
        int r1;
        engine_cta_rows(op.N, blockIdx.x, gridDim.x, &r0, &r1);
        n = r1 - r0;
        mats = op.W2 ? 2 : 1;
        K = op.K;
        wt = op.wt;
        sg = engine_slice_geom(mats, K, slot_bytes, op.wt);
        ntiles = engine_tile_count(n, sg.rmax);
    }
    // rows [*tr0, *tr0 + *R) of tile t
    __device__ __forceinline__ void tile(int t, int *tr0, int *R) const {
        int a, b;
        engine_tile_rows(n, t, ntiles, &a, &b);
        *tr0 = r0 + a, *R = b - a;
    }
};

// Attention splits of an ATTN op (shared by the consumers, which run the
// items, and the producer, which streams their cache rows): one split per
// kAttnSplitLen positions of the longest visible context, at most
// kAttnMaxSplits and op.S, and few enough that every item has its own group
// (split 0 waits for the others).
constexpr int kAttnSplitLen = 32;
constexpr int kAttnMaxSplits = 32;
__device__ __forceinline__ int attn_splits(const EngineOp &op, int pos_base, int groups) {
    int S = (min(pos_base + op.M, op.max_seq) + kAttnSplitLen - 1) / kAttnSplitLen;
    S = min(min(S, kAttnMaxSplits), min(op.S, groups / (op.M * op.Hkv)));
    return S < 1 ? 1 : S;
}
// Positions [*t0, *t1) of split sp of token m's visible context.
__device__ __forceinline__ void attn_range(const EngineOp &op, int pos_base, int m, int sp, int S, int *t0, int *t1) {
    const int visible = min(pos_base + m + 1, op.max_seq);
    const int chunk = (visible + S - 1) / S;
    *t0 = min(visible, sp * chunk);
    *t1 = min(visible, *t0 + chunk);
}
__device__ __forceinline__ int attn_pos_base(const EngineOp &op) {
    return op.pos_const + (op.pos_dev ? *reinterpret_cast<const volatile int32_t *>(op.pos_dev) : 0);
}
// First RoPE row a side block holds: the new positions, clamped to the table.
__device__ __forceinline__ int attn_rope_r0(const EngineOp &op, int pos_base) { return min(pos_base, op.max_seq - 1); }

// The ring slots of an ATTN op on this CTA: `rounds` rounds of one slot per
// group (gpc groups), round k of a group carrying positions
// [t0 + k * P, t0 + (k + 1) * P) of its item's range.
struct AttnPlan {
    int rep = 1, gpc = 1, kvb = 2, P = 1, S = 1, n_items = 0, rounds = 0, pos_base = 0;
    __device__ void init(const EngineOp &op, int slot_bytes) {
        rep = op.H / op.Hkv, gpc = kEngineConsumerWarps / rep, kvb = op.kv_half ? 2 : 4;
        P = attn_slot_rows(op.hd, kvb, slot_bytes);
        pos_base = attn_pos_base(op);
        S = attn_splits(op, pos_base, gridDim.x * gpc);
        n_items = op.M * op.Hkv * S;
        const int vmax = min(pos_base + op.M, op.max_seq), chunk = (vmax + S - 1) / S;
        rounds = max(1, (chunk + P - 1) / P);
    }
    __device__ int slots() const { return rounds * gpc; }
};

// One slot's bulk copies, in fixed places (a zero size: no copy), so that
// the producer keeps them in registers: a weight slot uses copy 0; an
// attention slot K rows (0), V rows (1), RoPE rows (2), Q gains (3) and K
// gains (4).
struct SlotCopies {
    const void *src[5];
    uint32_t off[5], bytes[5];
    __device__ __forceinline__ void clear() {
#pragma unroll
        for (int q = 0; q < 5; ++q) src[q] = nullptr, off[q] = 0, bytes[q] = 0;
    }
    __device__ __forceinline__ uint32_t total() const {
        uint32_t t = 0;
#pragma unroll
        for (int q = 0; q < 5; ++q) t += bytes[q];
        return t;
    }
};

// The copies of slot j (round j / gpc, group j % gpc) of an ATTN op.
__device__ void attn_slot(const EngineOp &op, const AttnPlan &pl, int j, SlotCopies &c) {
    const int k = j / pl.gpc, gg = j % pl.gpc, item = gg * gridDim.x + blockIdx.x;
    if (item >= pl.n_items) return;
    const int sp = item % pl.S, kvh = (item / pl.S) % op.Hkv, m = item / (pl.S * op.Hkv);
    int t0, t1;
    attn_range(op, pl.pos_base, m, sp, pl.S, &t0, &t1);
    const int hd = op.hd, rowb = hd * pl.kvb, tile = attn_tile_bytes(pl.P, hd, pl.kvb);
    const int c0 = t0 + k * pl.P, nc = min(min(t1, c0 + pl.P), pl.pos_base) - c0;
    if (nc > 0) {
        const size_t off = ((size_t)kvh * op.max_seq + c0) * rowb;
        c.src[0] = reinterpret_cast<const uint8_t *>(op.kcache) + off, c.off[0] = 0, c.bytes[0] = (uint32_t)(nc * rowb);
        c.src[1] = reinterpret_cast<const uint8_t *>(op.vcache) + off, c.off[1] = (uint32_t)tile;
        c.bytes[1] = (uint32_t)(nc * rowb);
    }
    if (k == 0) {
        const int r0 = attn_rope_r0(op, pl.pos_base), nr = min(op.M, op.max_seq - r0);
        c.src[2] = op.rope_cs + (size_t)r0 * (hd >> 1), c.off[2] = (uint32_t)(2 * tile);
        c.bytes[2] = (uint32_t)(nr * (hd >> 1) * 8);
        if (op.q_norm) c.src[3] = op.q_norm, c.off[3] = (uint32_t)(2 * tile + 8 * hd), c.bytes[3] = (uint32_t)(hd * 4);
        if (op.k_norm) c.src[4] = op.k_norm, c.off[4] = (uint32_t)(2 * tile + 12 * hd), c.bytes[4] = (uint32_t)(hd * 4);
    }
}

// ---------------------------------------------------------------------------
// producer: lane 0 of the last warp
// ---------------------------------------------------------------------------

// Walks this CTA's ring slots in program order: the weight slots of GEMV
// ops and the cache-row slots of ATTN ops.
template <bool FRAME>
struct SlotIter {
    int i = -1, t = 0, s = 0;  // op, tile (ATTN: slot), slice of the next slot
    bool attn = false;
    int r0 = 0, n = 0, ntiles = 0, mats = 1, K = 0, tr0 = 0, R = 0, wt = 0;
    SliceGeom sg{};
    const uint8_t *Wt = nullptr;
    __device__ void set_tile() {
        int a0, b0;
        engine_tile_rows(n, t, ntiles, &a0, &b0);
        tr0 = r0 + a0, R = b0 - a0;
    }
    // Fills c with the next slot's copies and returns its op; -1 at the end.
    __device__ int next(const EngineArgs &a, SlotCopies &c, AttnPlan &plan) {
        for (;;) {
            if (t < ntiles) {
                const int opi = i;
                c.clear();
                if (attn) {
                    attn_slot(a.ops[i], plan, t, c);
                    ++t;
                } else {
                    const int kw = min(sg.kt, K - s * sg.kt);
                    c.src[0] = Wt + (size_t)tr0 * engine_row_bytes(wt, K) * mats +
                               (size_t)s * R * engine_row_bytes(wt, sg.kt) * mats;
                    c.bytes[0] = (uint32_t)(mats * R * engine_row_bytes(wt, kw));
                    if (++s == sg.nk) {
                        s = 0;
                        if (++t < ntiles) set_tile();
                    }
                }
                return opi;
            }
            if (++i >= a.n_ops) return -1;
            const EngineOp &op = a.ops[i];
            t = s = 0;
            attn = FRAME ? op.kind == OP_ATTN : op.kind != OP_GEMV;
            if (attn) {
                plan.init(op, a.slot_bytes);
                ntiles = plan.slots();
            } else if (FRAME && op.kind != OP_GEMV) {  // SAMPLE, ATTN_CTX: no slots
                ntiles = 0;
            } else {
                const GemvTiling T(op, a.slot_bytes);
                r0 = T.r0, n = T.n, ntiles = T.ntiles, mats = T.mats, K = T.K, sg = T.sg, wt = T.wt;
                Wt = reinterpret_cast<const uint8_t *>(op.Wt);
                if (ntiles) set_tile();
            }
        }
    }
};

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <bool FRAME>
__device__ void producer(const EngineArgs &a, uint64_t *full, uint64_t *empty, uint8_t *ring) {
    const int NS = a.nslots;
    uint32_t g = 0;   // slots issued
    uint32_t pf = 0;  // slots the prefetch cursor has passed
    int slot = 0;
    uint32_t phase = 0;
    SlotIter<FRAME> cur, ahead;
    AttnPlan cur_plan, ahead_plan;
    SlotCopies c, pc;
    for (;;) {
        const int opi = cur.next(a, c, cur_plan);
        if (opi < 0) break;
        // keep the L2 prefetch cursor l2_lead slots ahead of the ring
        while (a.l2_lead > 0 && pf <= g + (uint32_t)a.l2_lead) {
            if (ahead.next(a, pc, ahead_plan) < 0) {
                pf = 0xffffffffu;
                break;
            }
            if (pf > g) {
#pragma unroll
                for (int q = 0; q < 5; ++q)
                    if (pc.bytes[q]) prefetch_l2(pc.src[q], pc.bytes[q]);
            }
            ++pf;
        }
        if (!mbar_wait(&empty[slot], phase ^ 1u, a.error, kErrEngineWeights)) break;
        uint8_t *dst = ring + (size_t)slot * a.slot_bytes;
        mbar_arrive_expect_tx(&full[slot], c.total());  // 0 bytes: the phase completes here
#pragma unroll
        for (int q = 0; q < 5; ++q)
            if (c.bytes[q]) bulk_copy(dst + c.off[q], c.src[q], c.bytes[q], &full[slot]);
        ++g;
        if (++slot == NS) slot = 0, phase ^= 1u;
        if (a.trace && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1))
            a.trace[((size_t)(blockIdx.x ? 1 : 0) * a.n_ops + opi) * 4 + 3] = globaltimer();
    }
    // Do not leave the CTA while copies may still be landing in it: wait
    // (bounded, also after an error) for the last ring's worth of copies.
    const uint32_t first = g > (uint32_t)NS ? g - (uint32_t)NS : 0u;
    for (uint32_t q = first; q < g; ++q) {
        const int sl = (int)(q % (uint32_t)NS);
        if (!mbar_wait(&full[sl], (q / (uint32_t)NS) & 1u, a.error, kErrEngineWeights, false)) return;
    }
}

// The 6-bit scale and min of sub-block j of a ggml Q4_K superblock from its
// 12 packed bytes (the published Q4_K block format).
__device__ __forceinline__ void q4k_sub_scale(int j, const uint8_t *p, int *sc, int *mn) {
    if (j < 4) {
        *sc = p[j] & 63;
        *mn = p[j + 4] & 63;
    } else {
        *sc = (p[j + 4] & 0x0f) | ((p[j - 4] >> 6) << 4);
        *mn = (p[j + 4] >> 4) | ((p[j] >> 6) << 4);
    }
}

// Out-of-place copy of a linear's weights into slot order (see GemvTiling
// and EngineWeight): one block per output row, threads over 32-element
// units (8-element ones for F16).
__global__ void relayout_kernel(const uint8_t *W, const uint8_t *W2, int gtype, int wt, int N, int K, int n_contig,
                                int row_base, int extra_row, int G, int slot_bytes, uint8_t *dst) {
    const int r = blockIdx.x;
    const int mats = W2 ? 2 : 1;
    // the CTA owning row r: the largest c with floor(N c / G) <= r
    const int c = (int)((((long long)r + 1) * G - 1) / N);
    int r0, r1;
    engine_cta_rows(N, c, G, &r0, &r1);
    const SliceGeom sg = engine_slice_geom(mats, K, slot_bytes, wt);
    const int n = r1 - r0, nt = engine_tile_count(n, sg.rmax), rel = r - r0;
    const int t = (int)((((long long)rel + 1) * nt - 1) / n);
    int ta, tb;
    engine_tile_rows(n, t, nt, &ta, &tb);
    const int R = tb - ta, q = rel - ta, tr0 = r0 + ta;
    const int src_row = n_contig < 0 ? r : (r < n_contig ? row_base + r : extra_row);
    uint8_t *tile = dst + (size_t)tr0 * engine_row_bytes(wt, K) * mats;
    const size_t src_row_bytes = gtype == 1 ? (size_t)K * 2 : gtype == 8 ? (size_t)K / 32 * 34 : (size_t)K / 256 * 144;
    const int unit = wt == EW_F16 ? 8 : 32;
    for (int u = threadIdx.x; u < K / unit; u += blockDim.x) {
        const int col = u * unit, s = col / sg.kt, kw = min(sg.kt, K - s * sg.kt), cc = col - s * sg.kt;
        uint8_t *slot = tile + (size_t)s * R * engine_row_bytes(wt, sg.kt) * mats;
        for (int m = 0; m < mats; ++m) {
            const uint8_t *srow = (m ? W2 + (size_t)r * src_row_bytes : W + (size_t)src_row * src_row_bytes);
            uint8_t *drow = slot + ((size_t)m * R + q) * engine_row_bytes(wt, kw);
            if (wt == EW_F16) {
                *reinterpret_cast<uint4 *>(drow + (size_t)cc * 2) = *reinterpret_cast<const uint4 *>(srow + (size_t)col * 2);
            } else if (wt == EW_Q8_0) {
                const uint8_t *blk = srow + (size_t)u * 34;
                for (int i = 0; i < 32; ++i) drow[cc + i] = blk[2 + i];
                drow[kw + cc / 16] = blk[0], drow[kw + cc / 16 + 1] = blk[1];
            } else {
                // sub-block j of superblock sb: elements 32j.. of the superblock
                const int sb = col / 256, j = (col % 256) / 32;
                const uint8_t *blk = srow + (size_t)sb * 144;
                const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(blk[2] | (blk[3] << 8))));
                int sc, mn;
                q4k_sub_scale(j, blk + 4, &sc, &mn);
                const uint8_t *qs = blk + 16 + 32 * (j / 2);  // group j/2: low nibbles j even, high j odd
                for (int i = 0; i < 16; ++i) {
                    const int lo = (j & 1) ? qs[2 * i] >> 4 : qs[2 * i] & 0x0f;
                    const int hi = (j & 1) ? qs[2 * i + 1] >> 4 : qs[2 * i + 1] & 0x0f;
                    drow[cc / 2 + i] = (uint8_t)(lo | (hi << 4));
                }
                float2 ab = make_float2(d * (float)sc, dmin * (float)mn);
                *reinterpret_cast<float2 *>(drow + kw / 2 + (cc / 32) * 8) = ab;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// consumers: warps 0-7
// ---------------------------------------------------------------------------

constexpr uint32_t kPollSpin = 1u << 21;  // polls of one LL word (an L2 round trip each)

struct ConsumerShared {
    float red[2][kEngineConsumerWarps];
    uint32_t epoch;
    int abort;  // a consumer wait failed: all warps leave after the current op
};

__device__ __forceinline__ unsigned long long ll_word(float v, uint32_t tag) {
    return ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
}
__device__ __forceinline__ void ll_store(uint64_t *p, float v, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(ll_word(v, tag)) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load(const uint64_t *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ ulonglong2 ll_load2(const uint64_t *p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0,%1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
// System-scope forms for the tensor-parallel exchange: the words are written
// by other GPUs (over NVLink) into this GPU's exchange buffer.
__device__ __forceinline__ void ll_store_sys(uint64_t *p, float v, uint32_t tag) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(ll_word(v, tag)) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load_sys(const uint64_t *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ ulonglong2 ll_load2_sys(const uint64_t *p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0,%1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool ll_fresh(unsigned long long w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float ll_value(unsigned long long w) { return __uint_as_float((uint32_t)w); }

// Wait until the N words w[i] = *addr(i) (addr(i) == nullptr: no word) carry
// `tag`.  Words start as 0 (tag 0 is never used), so the first pass issues
// every load at once and later passes re-read only the stale ones.  Bounded:
// on timeout kErrEngineWait is flagged; when another CTA has flagged an
// error the wait gives up; either way it returns false.
template <bool SYS = false, int N, class Addr>
__device__ __forceinline__ bool ll_wait(unsigned long long (&w)[N], Addr addr, uint32_t tag, int32_t *err) {
    for (uint32_t spin = 0;; ++spin) {
        bool all = true;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint64_t *p = addr(i);
            if (p && !ll_fresh(w[i], tag)) {
                all = false;
                w[i] = SYS ? ll_load_sys(p) : ll_load(p);
            }
        }
        if (all) return true;
        if ((spin & 255u) == 255u && ld_volatile(err)) return false;
        if (spin >= kPollSpin) {
            atomicCAS(err, 0, kErrEngineWait);
            return false;
        }
    }
}
template <bool SYS = false, int N, class Addr>
__device__ __forceinline__ bool ll_wait2(ulonglong2 (&w)[N], Addr addr, uint32_t tag, int32_t *err) {
    for (uint32_t spin = 0;; ++spin) {
        bool all = true;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint64_t *p = addr(i);
            if (p && !(ll_fresh(w[i].x, tag) && ll_fresh(w[i].y, tag))) {
                all = false;
                w[i] = SYS ? ll_load2_sys(p) : ll_load2(p);
            }
        }
        if (all) return true;
        if ((spin & 255u) == 255u && ld_volatile(err)) return false;
        if (spin >= kPollSpin) {
            atomicCAS(err, 0, kErrEngineWait);
            return false;
        }
    }
}

// One input value of an op: a float written before the launch (src < 0), an
// LL word of op src, or (nsum > 1) the sum in rank order of nsum ranks' LL
// words of op src, rstride words apart.
__device__ __forceinline__ bool read_input(const void *base, size_t idx, int src, uint32_t epoch, float &v,
                                           int32_t *err, int nsum = 1, long long rstride = 0) {
    if (src < 0) {
        v = __ldcg(reinterpret_cast<const float *>(base) + idx);
        return true;
    }
    if (nsum > 1) {
        const uint64_t *p = reinterpret_cast<const uint64_t *>(base) + idx;
        unsigned long long w[kEngineMaxPeers];
#pragma unroll
        for (int r = 0; r < kEngineMaxPeers; ++r) w[r] = 0ull;
        const bool ok =
            ll_wait<true>(w, [&](int r) { return r < nsum ? p + r * rstride : nullptr; }, engine_tag(epoch, src), err);
        float t = ll_value(w[0]);
#pragma unroll
        for (int r = 1; r < kEngineMaxPeers; ++r)
            if (r < nsum) t = __fadd_rn(t, ll_value(w[r]));
        v = t;
        return ok;
    }
    const uint64_t *p = reinterpret_cast<const uint64_t *>(base) + idx;
    unsigned long long w[1] = {0ull};
    const bool ok = ll_wait(w, [&](int) { return p; }, engine_tag(epoch, src), err);
    v = ll_value(w[0]);
    return ok;
}

// Stage the op's M input vectors in shared memory as xs[m][K], normalised
// when the op has an RMSNorm prologue; CTA 0 also writes them to x_out.
// Returns false (for every thread) when an input wait failed.
template <int M>
__device__ bool stage_x(const EngineOp &op, float *xs, ConsumerShared &cs, int32_t *err) {
    constexpr int T = kEngineConsumerWarps * 32;
    constexpr int B = 8;  // 16-byte chunks in flight per thread
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = op.K;
    float ss[M];
    bool ok = true;
#pragma unroll
    for (int m = 0; m < M; ++m) {
        ss[m] = 0.f;
        float *dst = xs + (size_t)m * K;
        if (op.x_src < 0) {
            const float4 *src = reinterpret_cast<const float4 *>(op.x) + (size_t)m * (op.ldx >> 2);
            for (int c0 = tid; c0 < (K >> 2); c0 += B * T) {
                float4 v[B];
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const int c = c0 + b * T;
                    v[b] = c < (K >> 2) ? __ldcg(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const int c = c0 + b * T;
                    if (c < (K >> 2)) reinterpret_cast<float4 *>(dst)[c] = v[b];
                    ss[m] = fmaf(v[b].x, v[b].x, ss[m]);
                    ss[m] = fmaf(v[b].y, v[b].y, ss[m]);
                    ss[m] = fmaf(v[b].z, v[b].z, ss[m]);
                    ss[m] = fmaf(v[b].w, v[b].w, ss[m]);
                }
            }
        } else if (op.x_nsum > 1) {
            // tensor parallelism: the sum in rank order of every rank's
            // partial sums; nb chunks of the n rows in flight per thread
            const uint32_t tag = engine_tag(cs.epoch, op.x_src);
            const uint64_t *src = reinterpret_cast<const uint64_t *>(op.x) + (size_t)m * op.ldx;
            const int n = op.x_nsum, nb = kEngineMaxPeers / n;
            const long long rs = op.x_rstride;
            for (int c0 = tid; c0 < (K >> 1); c0 += nb * T) {
                ulonglong2 v[kEngineMaxPeers];
#pragma unroll
                for (int i = 0; i < kEngineMaxPeers; ++i) v[i] = make_ulonglong2(0ull, 0ull);
                ok = ll_wait2<true>(v,
                                    [&](int i) {
                                        const int b = i / n, r = i - b * n, c = c0 + b * T;
                                        return b < nb && c < (K >> 1) ? src + r * rs + 2 * c : nullptr;
                                    },
                                    tag, err) && ok;
                for (int b = 0; b < nb; ++b) {
                    const int c = c0 + b * T;
                    if (c >= (K >> 1)) break;
                    float f0 = ll_value(v[b * n].x), f1 = ll_value(v[b * n].y);
                    for (int r = 1; r < n; ++r) {
                        f0 = __fadd_rn(f0, ll_value(v[b * n + r].x));
                        f1 = __fadd_rn(f1, ll_value(v[b * n + r].y));
                    }
                    reinterpret_cast<float2 *>(dst)[c] = make_float2(f0, f1);
                    ss[m] = fmaf(f0, f0, ss[m]);
                    ss[m] = fmaf(f1, f1, ss[m]);
                }
            }
        } else {
            const uint32_t tag = engine_tag(cs.epoch, op.x_src);
            const uint64_t *src = reinterpret_cast<const uint64_t *>(op.x) + (size_t)m * op.ldx;
            for (int c0 = tid; c0 < (K >> 1); c0 += B * T) {
                ulonglong2 v[B];
#pragma unroll
                for (int b = 0; b < B; ++b) v[b] = make_ulonglong2(0ull, 0ull);
                ok = ll_wait2(v, [&](int b) { return c0 + b * T < (K >> 1) ? src + 2 * (c0 + b * T) : nullptr; },
                              tag, err) && ok;
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const int c = c0 + b * T;
                    if (c < (K >> 1)) {
                        const float f0 = ll_value(v[b].x), f1 = ll_value(v[b].y);
                        reinterpret_cast<float2 *>(dst)[c] = make_float2(f0, f1);
                        ss[m] = fmaf(f0, f0, ss[m]);
                        ss[m] = fmaf(f1, f1, ss[m]);
                    }
                }
            }
        }
    }
    if (!ok) cs.abort = 1;
    float *x_out = blockIdx.x == 0 ? op.x_out : nullptr;
    if (op.norm_w) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) cs.red[m][warp] = t;
        }
        consumers_sync();
        const float4 *nw = reinterpret_cast<const float4 *>(op.norm_w);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float t = 0.f;
#pragma unroll
            for (int k = 0; k < kEngineConsumerWarps; ++k) t += cs.red[m][k];
            const float scale = 1.0f / sqrtf(t / (float)K + op.eps);
            float4 *row = reinterpret_cast<float4 *>(xs + (size_t)m * K);
            for (int c = tid; c < (K >> 2); c += T) {
                float4 v = row[c];
                const float4 g = __ldg(nw + c);
                v.x = __fmul_rn(__fmul_rn(v.x, scale), g.x);
                v.y = __fmul_rn(__fmul_rn(v.y, scale), g.y);
                v.z = __fmul_rn(__fmul_rn(v.z, scale), g.z);
                v.w = __fmul_rn(__fmul_rn(v.w, scale), g.w);
                row[c] = v;
                if (x_out) reinterpret_cast<float4 *>(x_out + (size_t)m * K)[c] = v;
            }
        }
    } else {
        consumers_sync();
        if (x_out) {
#pragma unroll
            for (int m = 0; m < M; ++m)
                for (int c = tid; c < (K >> 2); c += T)
                    reinterpret_cast<float4 *>(x_out + (size_t)m * K)[c] =
                        reinterpret_cast<const float4 *>(xs + (size_t)m * K)[c];
        }
    }
    consumers_sync();  // xs is complete; cs.red may be rewritten by the next op
    return !cs.abort;
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// One slot's arithmetic for a warp holding NR rows of the tile: per step a
// lane takes CH chunks (c and c + 32), loads their inputs once and the
// chunks of each of its rows, and feeds independent accumulator chains
// (acc[j] for chunk j of the step).
template <int NR, int M, int MATS, int CH>
__device__ __forceinline__ void gemv_slot(uint32_t wbase, uint32_t rstride, uint32_t mstride, uint32_t xbase,
                                          int K, int nch, int lane, float (&acc)[CH][kRowsPerWarp][MATS][M]) {
#pragma unroll 1
    for (int c = lane; c < nch; c += 32 * CH) {
        float4 x0[CH][M], x1[CH][M];
        uint4 w[CH][NR][MATS];
#pragma unroll
        for (int j = 0; j < CH; ++j) {
            const int cj = c + 32 * j;
            const bool ok = j == 0 || cj < nch;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const uint32_t xa = xbase + (uint32_t)((m * K + cj * 8) * 4);
                x0[j][m] = ok ? lds_f4(xa) : make_float4(0.f, 0.f, 0.f, 0.f);
                x1[j][m] = ok ? lds_f4(xa + 16) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < NR; ++i)
#pragma unroll
                for (int q = 0; q < MATS; ++q)
                    w[j][i][q] = ok ? lds_u4(wbase + i * rstride + q * mstride + (uint32_t)cj * 16)
                                    : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < CH; ++j)
#pragma unroll
            for (int i = 0; i < NR; ++i)
#pragma unroll
                for (int q = 0; q < MATS; ++q)
#pragma unroll
                    for (int m = 0; m < M; ++m) acc[j][i][q][m] = dot8(w[j][i][q], x0[j][m], x1[j][m], acc[j][i][q][m]);
    }
}

__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ unsigned short lds_u16(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

// acc += sum over the 4 int8 of `q` of (d * q_i) * x_i (ggml Q8_0 value d*q).
__device__ __forceinline__ float dot4_q8(uint32_t q, float d, float4 x, float acc) {
    acc = fmaf(__fmul_rn((float)(int8_t)(q & 0xff), d), x.x, acc);
    acc = fmaf(__fmul_rn((float)(int8_t)((q >> 8) & 0xff), d), x.y, acc);
    acc = fmaf(__fmul_rn((float)(int8_t)((q >> 16) & 0xff), d), x.z, acc);
    acc = fmaf(__fmul_rn((float)(int8_t)(q >> 24), d), x.w, acc);
    return acc;
}
// acc += sum over the 8 nibbles of `q` (element 2i low, 2i+1 high of byte
// i) of (a * n - b) * x (ggml Q4_K value (d*sc)*q - dmin*m).
__device__ __forceinline__ float dot8_q4(uint32_t q, float a, float b, float4 x0, float4 x1, float acc) {
    const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fmaf(__fsub_rn(__fmul_rn(a, (float)((q >> (4 * i)) & 0xf)), b), xs[i], acc);
    return acc;
}

// One slot's arithmetic for quantized weights (EW_Q8_0 / EW_Q4_K): like
// gemv_slot over 16-column chunks; a row slice of kw columns holds the
// chunk quants at q_off + chunk * qb and the scales at s_off.
template <int WT, int NR, int M, int MATS, int CH>
__device__ __forceinline__ void gemv_slot_q(uint32_t wbase, uint32_t rstride, uint32_t mstride, uint32_t xbase,
                                            int K, int kw, int nch, int lane,
                                            float (&acc)[CH][kRowsPerWarp][MATS][M]) {
#pragma unroll 1
    for (int c = lane; c < nch; c += 32 * CH) {
#pragma unroll
        for (int j = 0; j < CH; ++j) {
            const int cj = c + 32 * j;
            if (j > 0 && cj >= nch) break;
            float4 x[M][4];
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const uint32_t xa = xbase + (uint32_t)((m * K + cj * 16) * 4);
#pragma unroll
                for (int v = 0; v < 4; ++v) x[m][v] = lds_f4(xa + 16 * v);
            }
#pragma unroll
            for (int i = 0; i < NR; ++i)
#pragma unroll
                for (int q = 0; q < MATS; ++q) {
                    const uint32_t row = wbase + i * rstride + q * mstride;
                    if (WT == EW_Q8_0) {
                        const uint4 w = lds_u4(row + (uint32_t)cj * 16);
                        const float d = __half2float(__ushort_as_half(lds_u16(row + (uint32_t)(kw + (cj >> 1) * 2))));
#pragma unroll
                        for (int m = 0; m < M; ++m) {
                            float t = acc[j][i][q][m];
                            t = dot4_q8(w.x, d, x[m][0], t);
                            t = dot4_q8(w.y, d, x[m][1], t);
                            t = dot4_q8(w.z, d, x[m][2], t);
                            t = dot4_q8(w.w, d, x[m][3], t);
                            acc[j][i][q][m] = t;
                        }
                    } else {
                        const uint2 w = lds_u2(row + (uint32_t)cj * 8);
                        const uint32_t sa = row + (uint32_t)(kw / 2 + (cj >> 1) * 8);
                        const float a = __uint_as_float(lds_u32(sa)), b = __uint_as_float(lds_u32(sa + 4));
#pragma unroll
                        for (int m = 0; m < M; ++m) {
                            float t = acc[j][i][q][m];
                            t = dot8_q4(w.x, a, b, x[m][0], x[m][1], t);
                            t = dot8_q4(w.y, a, b, x[m][2], x[m][3], t);
                            acc[j][i][q][m] = t;
                        }
                    }
                }
        }
    }
}

// Consume this CTA's slots of one GEMV op (see GemvTiling).  Every warp
// takes every slot: per 16-byte column chunk a lane loads the inputs once
// and the chunk of each of its warp's rows.
template <int M, int MATS>
__device__ bool consume_gemv(const EngineArgs &a, const EngineOp &op, int opi, uint32_t epoch, uint32_t &g,
                             uint64_t *full, uint64_t *empty, const uint8_t *ring, const float *xs) {
    constexpr int CH = 2 / MATS;  // chunks per lane and step: a slice row has 64 / MATS chunks
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int NS = a.nslots;
    const GemvTiling T(op, a.slot_bytes);
    const SliceGeom sg = T.sg;
    const int K = T.K, epi = op.epi, ldy = op.ldy, ldr = op.ldr, resid_src = op.resid_src;
    const int r_nsum = op.r_nsum, n_peer = op.n_peer;
    const long long r_rstride = op.r_rstride;
    const bool y_ll = op.y_ll != 0;
    void *y = op.y;
    const void *resid = op.resid;
    const uint32_t out_tag = engine_tag(epoch, opi);
    const uint32_t ring_s = saddr(ring), xs_s = saddr(xs), slot_bytes = (uint32_t)a.slot_bytes;
    int slot = (int)(g % (uint32_t)NS);
    uint32_t phase = (g / (uint32_t)NS) & 1u;
    bool ok = true;
    for (int t = 0; t < T.ntiles; ++t) {
        int tr0, R;
        T.tile(t, &tr0, &R);
        const int nrw = R > warp ? (R - warp + kEngineConsumerWarps - 1) / kEngineConsumerWarps : 0;
        float acc[CH][kRowsPerWarp][MATS][M];
#pragma unroll
        for (int j = 0; j < CH; ++j)
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
                for (int q = 0; q < MATS; ++q)
#pragma unroll
                    for (int m = 0; m < M; ++m) acc[j][i][q][m] = 0.f;
        for (int s = 0; s < sg.nk; ++s) {
            const int k0 = s * sg.kt, kw = min(sg.kt, K - k0), nch = kw >> 3;
            const bool got = mbar_wait(&full[slot], phase, a.error, kErrEngineWeights);
            if (!__all_sync(0xffffffffu, got)) return false;
            const uint32_t rb = (uint32_t)engine_row_bytes(T.wt, kw);  // one row slice
            const uint32_t wbase = ring_s + (uint32_t)slot * slot_bytes + (uint32_t)warp * rb;
            const uint32_t rstride = (uint32_t)kEngineConsumerWarps * rb, mstride = (uint32_t)R * rb;
            const uint32_t xbase = xs_s + (uint32_t)(k0 * 4);
            if (T.wt == EW_F16) {
                switch (nrw) {
                case 4: gemv_slot<4, M, MATS, CH>(wbase, rstride, mstride, xbase, K, nch, lane, acc); break;
                case 3: gemv_slot<3, M, MATS, CH>(wbase, rstride, mstride, xbase, K, nch, lane, acc); break;
                case 2: gemv_slot<2, M, MATS, CH>(wbase, rstride, mstride, xbase, K, nch, lane, acc); break;
                case 1: gemv_slot<1, M, MATS, CH>(wbase, rstride, mstride, xbase, K, nch, lane, acc); break;
                default: break;
                }
            } else if (T.wt == EW_Q8_0) {
                const int nq = kw >> 4;
                switch (nrw) {
                case 4: gemv_slot_q<EW_Q8_0, 4, M, MATS, CH>(wbase, rstride, mstride, xbase, K, kw, nq, lane, acc); break;
                case 3: gemv_slot_q<EW_Q8_0, 3, M, MATS, CH>(wbase, rstride, mstride, xbase, K, kw, nq, lane, acc); break;
                case 2: gemv_slot_q<EW_Q8_0, 2, M, MATS, CH>(wbase, rstride, mstride, xbase, K, kw, nq, lane, acc); break;
                case 1: gemv_slot_q<EW_Q8_0, 1, M, MATS, CH>(wbase, rstride, mstride, xbase, K, kw, nq, lane, acc); break;
                default: break;
                }
            } else {
                const int nq = kw >> 4;
                switch (nrw) {
                case 4: gemv_slot_q<EW_Q4_K, 4, M, MATS, CH>(wbase, rstride, mstride, xbase, K, kw, nq, lane, acc); break;
                case 3: gemv_slot_q<EW_Q4_K, 3, M, MATS, CH>(wbase, rstride, mstride, xbase, K, kw, nq, lane, acc); break;
                case 2: gemv_slot_q<EW_Q4_K, 2, M, MATS, CH>(wbase, rstride, mstride, xbase, K, kw, nq, lane, acc); break;
                case 1: gemv_slot_q<EW_Q4_K, 1, M, MATS, CH>(wbase, rstride, mstride, xbase, K, kw, nq, lane, acc); break;
                default: break;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == NS) slot = 0, phase ^= 1u;
        }
        g += (uint32_t)sg.nk;
        // reduce each row's partial sums; lane i * M + m writes row i, token m
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            if (i >= nrw) break;
            float v[MATS][M];
#pragma unroll
            for (int q = 0; q < MATS; ++q)
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    float s = acc[0][i][q][m];
#pragma unroll
                    for (int j = 1; j < CH; ++j) s += acc[j][i][q][m];
                    v[q][m] = warp_sum(s);
                }
#pragma unroll
            for (int m = 0; m < M; ++m) {
                if (lane != i * M + m) continue;
                const int row = tr0 + warp + i * kEngineConsumerWarps;
                const float g1 = v[0][m], g3 = v[MATS - 1][m];
                float out;
                if (epi == EPI_STORE) {
                    out = g1;
                } else if (epi == EPI_RESID) {
                    float r;
                    ok = read_input(resid, (size_t)m * ldr + row, resid_src, epoch, r, a.error, r_nsum, r_rstride) &&
                         ok;
                    out = __fadd_rn(r, g1);
                } else if (epi == EPI_SWIGLU_SLOW) {
                    const float sig = 1.0f / (1.0f + expf(-g1));
                    out = __fmul_rn(__fmul_rn(g1, sig), g3);
                } else {
                    out = __fmul_rn(g1 / (1.0f + expf(-g1)), g3);
                }
                if (n_peer > 0) {
                    // tensor parallelism: this rank's partial sum into every rank's exchange buffer
                    for (int q = 0; q < n_peer; ++q) ll_store_sys(op.y_peer[q] + (size_t)m * ldy + row, out, out_tag);
                } else if (y_ll) {
                    ll_store(reinterpret_cast<uint64_t *>(y) + (size_t)m * ldy + row, out, out_tag);
                } else {
                    reinterpret_cast<float *>(y)[(size_t)m * ldy + row] = out;
                }
            }
        }
    }
    return ok;
}

template <int M>
__device__ bool run_gemv(const EngineArgs &a, const EngineOp &op, int opi, uint32_t &g, uint64_t *full,
                         uint64_t *empty, const uint8_t *ring, float *xs, ConsumerShared &cs, unsigned long long *tr) {
    if (!stage_x<M>(op, xs, cs, a.error)) return false;
    if (tr) tr[1] = globaltimer();
    return op.W2 ? consume_gemv<M, 2>(a, op, opi, cs.epoch, g, full, empty, ring, xs)
                 : consume_gemv<M, 1>(a, op, opi, cs.epoch, g, full, empty, ring, xs);
}

template <typename KV>
__device__ __forceinline__ KV kv_from(float v);
template <>
__device__ __forceinline__ __half kv_from<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float kv_from<float>(float v) { return v; }
__device__ __forceinline__ float kv_to(__half v) { return __half2float(v); }
__device__ __forceinline__ float kv_to(float v) { return v; }

// This lane's QK-norm gains and RoPE (cos, sin) pairs of one head, from the
// group's side block in shared memory.
template <int EPL>
struct RopeNorm {
    float g[EPL];
    float2 cs[EPL / 2];
    __device__ __forceinline__ void load(const float *gains, const float2 *rope_row) {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int e = 0; e < EPL; ++e) g[e] = gains[lane * EPL + e];
#pragma unroll
        for (int e = 0; e < EPL; e += 2) cs[e / 2] = rope_row[(lane * EPL + e) >> 1];
    }
    // the same from global memory; gains may be null (no QK-norm)
    __device__ __forceinline__ void load_global(const float *gains, const float2 *rope_row) {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int e = 0; e < EPL; ++e) g[e] = gains ? __ldg(gains + lane * EPL + e) : 1.f;
#pragma unroll
        for (int e = 0; e < EPL; e += 2) cs[e / 2] = __ldg(rope_row + ((lane * EPL + e) >> 1));
    }
    // QK-norm (when `norm`) + RoPE of one head held as EPL values per lane
    __device__ __forceinline__ void apply(float *v, bool norm, float eps, int hd) const {
        if (norm) {
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < EPL; ++e) ss = fmaf(v[e], v[e], ss);
            ss = warp_sum(ss);
            const float scale = 1.0f / sqrtf(ss / (float)hd + eps);
#pragma unroll
            for (int e = 0; e < EPL; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], scale), g[e]);
        }
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
            const float2 r = cs[e / 2];
            const float x0 = v[e], x1 = v[e + 1];
            v[e] = __fsub_rn(__fmul_rn(x0, r.x), __fmul_rn(x1, r.y));
            v[e + 1] = __fadd_rn(__fmul_rn(x0, r.y), __fmul_rn(x1, r.x));
        }
    }
};

template <typename KV>
__device__ __forceinline__ float4 kv_load4(const uint8_t *p, int i);  // elements 4i..4i+3
template <>
__device__ __forceinline__ float4 kv_load4<__half>(const uint8_t *p, int i) {
    const uint2 u = reinterpret_cast<const uint2 *>(p)[i];
    return make_float4(h_lo(u.x), h_hi(u.x), h_lo(u.y), h_hi(u.y));
}
template <>
__device__ __forceinline__ float4 kv_load4<float>(const uint8_t *p, int i) {
    return reinterpret_cast<const float4 *>(p)[i];
}



// This lane's EPL elements (lane * EPL ...) of a K or V row, as floats.
template <typename KV, int EPL>
__device__ __forceinline__ void kv_load_lane(const uint8_t *row, float (&v)[EPL]) {
    const int lane = threadIdx.x & 31;
    if constexpr (EPL % 4 == 0) {
#pragma unroll
        for (int e = 0; e < EPL; e += 4) {
            const float4 f = kv_load4<KV>(row, (lane * EPL + e) >> 2);
            v[e] = f.x, v[e + 1] = f.y, v[e + 2] = f.z, v[e + 3] = f.w;
        }
    } else {
        const KV *r = reinterpret_cast<const KV *>(row) + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) v[e] = kv_to(r[e]);
    }
}

// Fused QK-norm + RoPE + KV write + split GQA attention (the ops of
// rope_kv_kernel and attn_kernel).  Work items are (token, kv head, split);
// a group of `rep` warps (one per query head of the GQA group) takes one
// item.  Cached K/V rows stream through one or two shared-memory buffers of
// kAttnRows rows with cp.async, the next sub-chunk's copies in flight while
// the current one is scored; the new tokens' rows are rebuilt from the QKV
// words, so no group reads a position another group is still writing.  The
// group holding a token's own position writes it to the cache.  With S > 1
// splits, split 0 merges the other splits' partials (LL words).
// Fused QK-norm + RoPE + KV write + split GQA attention (the ops of
// rope_kv_kernel and attn_kernel).  Work items are (token, kv head, split);
// a group of `rep` warps (one per query head of the GQA group) takes one
// item.  The item's cached K/V rows arrive through the weight ring (see
// AttnPlan), round by round; every consumer warp waits on every slot, in
// order, and the owning group reads it.  The new tokens' rows are rebuilt
// from the QKV words, so no group reads a position another group is still
// writing; the group holding a token's own position writes it to the cache.
// With S > 1 splits, split 0 merges the other splits' partials (LL words).
template <typename KV, int EPL>
__device__ bool consume_attn(const EngineArgs &a, const EngineOp &op, int opi, uint32_t epoch, uint8_t *area,
                             uint32_t g, uint64_t *full, uint64_t *empty, const uint8_t *ring,
                             unsigned long long *tr) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = op.hd, M = op.M;
    AttnPlan pl;
    pl.init(op, a.slot_bytes);
    const int rep = pl.rep, gid = warp / rep, wr = warp % rep, gtid = wr * 32 + lane;
    const int bar_id = 2 + gid, bar_n = rep * 32;
    constexpr int kvb = (int)sizeof(KV);
    const int rowb = hd * kvb, tile = attn_tile_bytes(pl.P, hd, kvb);
    uint8_t *gbase = area + (size_t)gid * attn_group_bytes(rep, hd, kvb);
    float *qsm = reinterpret_cast<float *>(gbase) + wr * hd;
    KV *newk = reinterpret_cast<KV *>(gbase + rep * hd * 4);  // [2][hd]
    KV *newv = newk + 2 * hd;
    const int pos_base = pl.pos_base, rope_r0 = attn_rope_r0(op, pos_base), S = pl.S;
    const uint32_t in_tag = engine_tag(epoch, op.qkv_src), out_tag = engine_tag(epoch, opi);
    const int NS = a.nslots;
    int slot = (int)(g % (uint32_t)NS);
    uint32_t phase = (g / (uint32_t)NS) & 1u;
    const int item = gid * gridDim.x + blockIdx.x;  // CTA-major: items spread over the SMs first
    const bool has = item < pl.n_items;
    const int sp = has ? item % S : 0, kvh = has ? (item / S) % op.Hkv : 0, m = has ? item / (S * op.Hkv) : 0;
    const int pos = pos_base + m, h = kvh * rep + wr;
    int t0 = 0, t1 = 0;
    if (has) attn_range(op, pos_base, m, sp, S, &t0, &t1);
    KV *kbase = reinterpret_cast<KV *>(op.kcache) + (size_t)kvh * op.max_seq * hd;
    KV *vbase = reinterpret_cast<KV *>(op.vcache) + (size_t)kvh * op.max_seq * hd;
    bool ok = true;
    float mrun = -INFINITY, l = 0.f, acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    for (int k = 0; k < pl.rounds; ++k) {
        for (int gg = 0; gg < pl.gpc; ++gg) {
            const bool got = mbar_wait(&full[slot], phase, a.error, kErrEngineWeights);
            if (!__all_sync(0xffffffffu, got)) return false;
            if (gg == gid && has) {
                const uint8_t *sb = ring + (size_t)slot * a.slot_bytes;
                if (k == 0) {
                    // the side block: RoPE rows of the new positions, QK-norm gains
                    const float2 *rope = reinterpret_cast<const float2 *>(sb + 2 * tile);
                    const float *qn = reinterpret_cast<const float *>(sb + 2 * tile + 8 * hd), *kn = qn + hd;
                    {
                        RopeNorm<EPL> rn;
                        rn.load(qn, rope + (size_t)(min(pos, op.max_seq - 1) - rope_r0) * (hd >> 1));
                        float q[EPL];
                        const uint64_t *qp = op.qkv + (size_t)m * op.ld_qkv + h * hd + lane * EPL;
                        unsigned long long w[EPL];
#pragma unroll
                        for (int e = 0; e < EPL; ++e) w[e] = 0ull;
                        ok = ll_wait(w, [&](int e) { return qp + e; }, in_tag, a.error) && ok;
#pragma unroll
                        for (int e = 0; e < EPL; ++e) q[e] = ll_value(w[e]);
                        rn.apply(q, op.q_norm != nullptr, op.eps, hd);
#pragma unroll
                        for (int e = 0; e < EPL; ++e) qsm[lane * EPL + e] = q[e];
                    }
                    // the new tokens' K/V rows this item sees, rebuilt by warp
                    // 0; the row of the item's own position also goes to the cache
                    if (wr == 0) {
                        for (int mm = 0; mm < M; ++mm) {
                            const int t = pos_base + mm;
                            if (t < t0 || t >= t1) continue;
                            RopeNorm<EPL> rn;
                            rn.load(kn, rope + (size_t)(t - rope_r0) * (hd >> 1));
                            const uint64_t *kp = op.qkv + (size_t)mm * op.ld_qkv + (op.H + kvh) * hd + lane * EPL;
                            const uint64_t *vp = kp + (size_t)op.Hkv * hd;
                            unsigned long long w[2 * EPL];
#pragma unroll
                            for (int e = 0; e < 2 * EPL; ++e) w[e] = 0ull;
                            ok = ll_wait(w, [&](int e) { return e < EPL ? kp + e : vp + (e - EPL); }, in_tag,
                                         a.error) && ok;
                            float kf[EPL], vf[EPL];
#pragma unroll
                            for (int e = 0; e < EPL; ++e) kf[e] = ll_value(w[e]), vf[e] = ll_value(w[EPL + e]);
                            rn.apply(kf, op.k_norm != nullptr, op.eps, hd);
                            KV *kd = newk + mm * hd + lane * EPL, *vd = newv + mm * hd + lane * EPL;
#pragma unroll
                            for (int e = 0; e < EPL; ++e) kd[e] = kv_from<KV>(kf[e]), vd[e] = kv_from<KV>(vf[e]);
                            if (t == pos) {
                                KV *kc = kbase + (size_t)t * hd + lane * EPL, *vc = vbase + (size_t)t * hd + lane * EPL;
#pragma unroll
                                for (int e = 0; e < EPL; ++e) kc[e] = kd[e], vc[e] = vd[e];
                            }
                        }
                    }
                    group_sync(bar_id, bar_n);  // qsm and the new rows are complete
                    if (tr && gtid == 0) tr[1] = globaltimer();
                }
                const int c0 = t0 + k * pl.P, c1 = min(t1, c0 + pl.P), n = max(0, c1 - c0);
                const uint8_t *kt = sb, *vt = sb + tile;
                // scores: lane j owns position c0 + j; lanes start at different
                // 4-element groups of the row so that they hit different banks
                float sc = -INFINITY;
                if (lane < n) {
                    const int t = c0 + lane;
                    const uint8_t *krow = t < pos_base ? kt + (size_t)lane * rowb
                                                       : reinterpret_cast<const uint8_t *>(newk + (t - pos_base) * hd);
                    const float4 *q4 = reinterpret_cast<const float4 *>(qsm);
                    const int ng = hd / 4;  // a power of two
                    float d0 = 0.f, d1 = 0.f;
                    for (int i = 0; i < ng; i += 2) {
                        const int i0 = (i + lane) & (ng - 1), i1 = (i + 1 + lane) & (ng - 1);
                        const float4 k0 = kv_load4<KV>(krow, i0), k1 = kv_load4<KV>(krow, i1);
                        const float4 a0 = q4[i0], a1 = q4[i1];
                        d0 = fmaf(a0.x, k0.x, d0);
                        d0 = fmaf(a0.y, k0.y, d0);
                        d0 = fmaf(a0.z, k0.z, d0);
                        d0 = fmaf(a0.w, k0.w, d0);
                        d1 = fmaf(a1.x, k1.x, d1);
                        d1 = fmaf(a1.y, k1.y, d1);
                        d1 = fmaf(a1.z, k1.z, d1);
                        d1 = fmaf(a1.w, k1.w, d1);
                    }
                    sc = (d0 + d1) * op.scale;
                }
                if (n > 0) {
                    const float mn = fmaxf(mrun, warp_max(sc));
                    const float corr = expf(mrun - mn);
                    const float p = lane < n ? expf(sc - mn) : 0.f;
                    l = fmaf(l, corr, warp_sum(p));
#pragma unroll
                    for (int e = 0; e < EPL; ++e) acc[e] *= corr;
                    for (int j0 = 0; j0 < n; j0 += 4) {
                        float pj[4], vv[4][EPL];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int j = j0 + u, t = c0 + j;
                            pj[u] = __shfl_sync(0xffffffffu, p, j & 31);
                            const uint8_t *vr = t < pos_base ? vt + (size_t)j * rowb
                                                             : reinterpret_cast<const uint8_t *>(newv + (t - pos_base) * hd);
                            if (j < n) {
                                kv_load_lane<KV, EPL>(vr, vv[u]);
                            } else {
                                pj[u] = 0.f;
#pragma unroll
                                for (int e = 0; e < EPL; ++e) vv[u][e] = 0.f;
                            }
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u)
#pragma unroll
                            for (int e = 0; e < EPL; ++e) acc[e] = fmaf(pj[u], vv[u][e], acc[e]);
                    }
                    mrun = mn;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == NS) slot = 0, phase ^= 1u;
        }
    }
    if (!has) return ok;
    uint64_t *outp = op.att_out + (size_t)m * op.H * hd + h * hd + lane * EPL;
    if (S == 1) {
#pragma unroll
        for (int e = 0; e < EPL; ++e) ll_store(outp + e, acc[e] / l, out_tag);
        return ok;
    }
    uint64_t *pbase = op.part + ((size_t)m * op.H + h) * op.S * (hd + 2);
    if (sp != 0) {
        uint64_t *pp = pbase + (size_t)sp * (hd + 2);
        if (lane == 0) ll_store(pp, mrun, out_tag), ll_store(pp + 1, l, out_tag);
#pragma unroll
        for (int e = 0; e < EPL; ++e) ll_store(pp + 2 + e * 32 + lane, acc[e], out_tag);  // lane-contiguous
        return ok;
    }
    // split 0 merges the other splits of its (token, head): lane j reads
    // split j + 1's (max, sum) and the lanes' dims of P.V come in batches
    if (tr && gtid == 0) tr[3] = globaltimer();
    float mj = -INFINITY, lj = 0.f;
    {
        const uint64_t *pj = lane < S - 1 ? pbase + (size_t)(lane + 1) * (hd + 2) : nullptr;
        unsigned long long w[2] = {0ull, 0ull};
        ok = ll_wait(w, [&](int i) { return pj ? pj + i : nullptr; }, out_tag, a.error) && ok;
        if (pj) mj = ll_value(w[0]), lj = ll_value(w[1]);
    }
    const float gmax = fmaxf(mrun, warp_max(mj));
    const float fj = lane < S - 1 ? expf(mj - gmax) : 0.f, fown = expf(mrun - gmax);
    const float L = fmaf(l, fown, warp_sum(lj * fj));
    float o[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = acc[e] * fown;
    constexpr int kB = 8;  // splits per batch of loads
    for (int j0 = 1; j0 < S; j0 += kB) {
        unsigned long long w[kB * EPL];
#pragma unroll
        for (int i = 0; i < kB * EPL; ++i) w[i] = 0ull;
        ok = ll_wait(w,
                     [&](int i) {
                         const int j = j0 + i / EPL;
                         return j < S ? pbase + (size_t)j * (hd + 2) + 2 + (i % EPL) * 32 + lane : nullptr;
                     },
                     out_tag, a.error) && ok;
#pragma unroll
        for (int b = 0; b < kB; ++b) {
            const float f = __shfl_sync(0xffffffffu, fj, (j0 + b - 1) & 31);
            if (j0 + b < S) {
#pragma unroll
                for (int e = 0; e < EPL; ++e) o[e] = fmaf(ll_value(w[b * EPL + e]), f, o[e]);
            }
        }
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) ll_store(outp + e, o[e] / L, out_tag);
    return ok;
}

// An ATTN op over an LL context (EngineOp::ctx_n > 0).  Group gid of the CTA
// takes item (KV head kvh, token m) like consume_attn with one split: its
// warps rebuild the visible K / V rows [0, pos] from the words of the ops
// that produced them (QK-norm and RoPE of K as when those rows were cached),
// then warp wr scores query head kvh * rep + wr, lane j owning position j,
// with consume_attn's arithmetic.  Group area: q [rep][hd], K [ctx_n][hd],
// V [ctx_n][hd].
template <int EPL>
__device__ __forceinline__ bool consume_attn_ctx(const EngineArgs &a, const EngineOp &op, int opi, uint32_t epoch,
                                              uint8_t *area) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hd = op.hd, rep = op.H / op.Hkv, gpc = kEngineConsumerWarps / rep;
    const int gid = warp / rep, wr = warp % rep;
    if (gid >= gpc) return true;
    const int item = gid * gridDim.x + blockIdx.x;
    if (item >= op.M * op.Hkv) return true;
    const int kvh = item % op.Hkv, m = item / op.Hkv, h = kvh * rep + wr;
    const int pos = op.pos_const + m, np = pos + 1;  // np <= ctx_n <= 32 (host-checked)
    float *qsm = reinterpret_cast<float *>(area + (size_t)gid * attn_ctx_group_bytes(rep, hd, op.ctx_n));
    float *ks = qsm + rep * hd, *vs = ks + (size_t)op.ctx_n * hd;
    bool ok = true;
    for (int j = wr; j < np; j += rep) {
        const uint64_t *kp = op.ctx_qkv[j] + (size_t)(op.H + kvh) * hd + lane * EPL;
        const uint64_t *vp = kp + (size_t)op.Hkv * hd;
        unsigned long long w[2 * EPL];
#pragma unroll
        for (int e = 0; e < 2 * EPL; ++e) w[e] = 0ull;
        ok = ll_wait(w, [&](int e) { return e < EPL ? kp + e : vp + (e - EPL); }, engine_tag(epoch, op.ctx_src[j]),
                     a.error) && ok;
        float kf[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) kf[e] = ll_value(w[e]), vs[(size_t)j * hd + lane * EPL + e] = ll_value(w[EPL + e]);
        RopeNorm<EPL> rn;
        rn.load_global(op.k_norm, op.rope_cs + (size_t)j * (hd >> 1));
        rn.apply(kf, op.k_norm != nullptr, op.eps, hd);
#pragma unroll
        for (int e = 0; e < EPL; ++e) ks[(size_t)j * hd + lane * EPL + e] = kf[e];
    }
    {
        const uint64_t *qp = op.qkv + (size_t)m * op.ld_qkv + (size_t)h * hd + lane * EPL;
        unsigned long long w[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) w[e] = 0ull;
        ok = ll_wait(w, [&](int e) { return qp + e; }, engine_tag(epoch, op.qkv_src), a.error) && ok;
        float q[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) q[e] = ll_value(w[e]);
        RopeNorm<EPL> rn;
        rn.load_global(op.q_norm, op.rope_cs + (size_t)pos * (hd >> 1));
        rn.apply(q, op.q_norm != nullptr, op.eps, hd);
#pragma unroll
        for (int e = 0; e < EPL; ++e) qsm[wr * hd + lane * EPL + e] = q[e];
    }
    group_sync(2 + gid, rep * 32);  // the group's K / V rows and queries are complete
    float sc = -INFINITY;
    if (lane < np) {
        const uint8_t *krow = reinterpret_cast<const uint8_t *>(ks + (size_t)lane * hd);
        const float4 *q4 = reinterpret_cast<const float4 *>(qsm + wr * hd);
        const int ng = hd / 4;  // a power of two
        float d0 = 0.f, d1 = 0.f;
        for (int i = 0; i < ng; i += 2) {
            const int i0 = (i + lane) & (ng - 1), i1 = (i + 1 + lane) & (ng - 1);
            const float4 k0 = kv_load4<float>(krow, i0), k1 = kv_load4<float>(krow, i1);
            const float4 a0 = q4[i0], a1 = q4[i1];
            d0 = fmaf(a0.x, k0.x, d0);
            d0 = fmaf(a0.y, k0.y, d0);
            d0 = fmaf(a0.z, k0.z, d0);
            d0 = fmaf(a0.w, k0.w, d0);
            d1 = fmaf(a1.x, k1.x, d1);
            d1 = fmaf(a1.y, k1.y, d1);
            d1 = fmaf(a1.z, k1.z, d1);
            d1 = fmaf(a1.w, k1.w, d1);
        }
        sc = (d0 + d1) * op.scale;
    }
    const float mn = warp_max(sc);
    const float p = lane < np ? expf(sc - mn) : 0.f;
    const float l = warp_sum(p);
    float acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    for (int j = 0; j < np; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const float *vr = vs + (size_t)j * hd + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] = fmaf(pj, vr[e], acc[e]);
    }
    uint64_t *outp = op.att_out + (size_t)m * op.H * hd + (size_t)h * hd + lane * EPL;
    const uint32_t out_tag = engine_tag(epoch, opi);
#pragma unroll
    for (int e = 0; e < EPL; ++e) ll_store(outp + e, acc[e] / l, out_tag);
    return ok;
}

// A SAMPLE op: CTA sample_cta stages the logits, runs the device sampler
// (sample_block, the 256 consumer threads) and writes the sampled code's
// Fast-AR embedding row as the next pass's input words.  Area layout:
// engine_sample_bytes.
__device__ __forceinline__ bool run_sample(const EngineArgs &a, const EngineOp &op, int opi, uint32_t epoch,
                                        uint8_t *area) {
    if ((int)blockIdx.x != op.sample_cta) return true;
    constexpr int T = kEngineConsumerWarps * 32;
    constexpr int B = 8;  // word pairs in flight per thread
    const int tid = threadIdx.x, n = op.K;
    float *lg = reinterpret_cast<float *>(area);
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(area + attn_round(n * 4));
    float *probs = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(keys) + (size_t)engine_sample_pow2(n) * 8);
    SampleScratch *scr =
        reinterpret_cast<SampleScratch *>(reinterpret_cast<uint8_t *>(probs) + attn_round((n + 1) * 4));
    const uint32_t tag = engine_tag(epoch, op.x_src);
    const uint64_t *src = reinterpret_cast<const uint64_t *>(op.x);
    bool ok = true;
    for (int c0 = tid; c0 < (n >> 1); c0 += B * T) {
        ulonglong2 v[B];
#pragma unroll
        for (int b = 0; b < B; ++b) v[b] = make_ulonglong2(0ull, 0ull);
        ok = ll_wait2(v, [&](int b) { return c0 + b * T < (n >> 1) ? src + 2 * (c0 + b * T) : nullptr; }, tag,
                      a.error) && ok;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int c = c0 + b * T;
            if (c < (n >> 1)) lg[2 * c] = ll_value(v[b].x), lg[2 * c + 1] = ll_value(v[b].y);
        }
    }
    if (consumers_sync_or(!ok)) return false;
    const uint32_t token =
        sample_block<T, kEngineSampleMax>(op.samp, 0, lg, keys, probs, *scr, [] { consumers_sync(); });
    if (op.y) {
        uint64_t *y = reinterpret_cast<uint64_t *>(op.y);
        const uint16_t *row = op.samp.fast_emb + (size_t)token * op.N;
        const uint32_t out_tag = engine_tag(epoch, opi);
        for (int i = tid; i < op.N; i += T) ll_store(y + i, h2f(row[i]), out_tag);
    }
    return true;
}

// The ops that only whole-frame programs use (engine_kernel<true>).  Inlined:
// with them as calls the frame kernel's program ran 2.8% slower (2.907
// against 2.827 ms for C2's nine passes).
__device__ __forceinline__ bool run_frame_op(const EngineArgs &a, const EngineOp &op, int opi, uint32_t epoch,
                                          uint8_t *area) {
    if (op.kind == OP_SAMPLE) return run_sample(a, op, opi, epoch, area);
    return op.hd == 64 ? consume_attn_ctx<2>(a, op, opi, epoch, area) : consume_attn_ctx<4>(a, op, opi, epoch, area);
}

// Not inlined: attention's register pressure stays out of the GEMV loops.
template <typename KV>
__device__ __noinline__ bool consume_attn_dispatch(const EngineArgs &a, const EngineOp &op, int opi, uint32_t epoch,
                                                   uint8_t *area, uint32_t g, uint64_t *full, uint64_t *empty,
                                                   const uint8_t *ring, unsigned long long *tr) {
    switch (op.hd / 32) {
    case 2: return consume_attn<KV, 2>(a, op, opi, epoch, area, g, full, empty, ring, tr);
    case 4: return consume_attn<KV, 4>(a, op, opi, epoch, area, g, full, empty, ring, tr);
    }
    return false;
}

}  // namespace

template <bool FRAME>
__global__ void __launch_bounds__(kEngineThreads, 1) engine_kernel(const EngineArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ ConsumerShared cs;
    const int tid = threadIdx.x, warp = tid >> 5;
    // [full | empty mbarriers] [staged inputs / attention groups] [ring]
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + a.nslots;
    uint8_t *area = smem + kEngineBarrierBytes;
    uint8_t *ring = area + a.area_bytes;
    if ((saddr(ring) & 127u) != 0u) {  // bulk copies land on 128-byte boundaries
        if (tid == 0) atomicCAS(a.error, 0, kErrEngineAlign);
        return;
    }
    if (tid == 0) {
        cs.abort = 0;
        cs.epoch = *reinterpret_cast<volatile uint32_t *>(a.epoch);
        for (int i = 0; i < a.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kEngineConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (a.done && *a.done) return;
    if (warp == kEngineConsumerWarps) {
        if ((tid & 31) == 0) producer<FRAME>(a, full, empty, ring);
        return;
    }
    const uint32_t epoch = cs.epoch;
    uint32_t g = 0;  // ring slots consumed
    for (int i = 0; i < a.n_ops; ++i) {
        const EngineOp &op = a.ops[i];
        unsigned long long *tr = nullptr;
        if (a.trace && tid == 0 && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1))
            tr = a.trace + ((size_t)(blockIdx.x ? 1 : 0) * a.n_ops + i) * 4;
        if (tr) tr[0] = globaltimer();
        bool ok;
        if (op.kind == OP_GEMV) {
            float *xs = reinterpret_cast<float *>(area);
            ok = op.M == 2 ? run_gemv<2>(a, op, i, g, full, empty, ring, xs, cs, tr)
                           : run_gemv<1>(a, op, i, g, full, empty, ring, xs, cs, tr);
        } else if (FRAME && op.kind != OP_ATTN) {
            ok = run_frame_op(a, op, i, epoch, area);
        } else {
            // attention timeline (group 0 of the CTA): [1] inputs ready, [3] merge started
            unsigned long long *atr = a.trace && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1)
                                          ? a.trace + ((size_t)(blockIdx.x ? 1 : 0) * a.n_ops + i) * 4
                                          : nullptr;
            ok = op.kv_half ? consume_attn_dispatch<__half>(a, op, i, epoch, area, g, full, empty, ring, atr)
                            : consume_attn_dispatch<float>(a, op, i, epoch, area, g, full, empty, ring, atr);
            AttnPlan pl;
            pl.init(op, a.slot_bytes);
            g += (uint32_t)pl.slots();
        }
        if (!ok) cs.abort = 1;
        consumers_sync();  // every consumer thread: the op is done (and the area reusable)
        if (tr) tr[2] = globaltimer();
        if (a.trace && tid == 0) a.trace[(size_t)a.n_ops * 8 + (size_t)i * gridDim.x + blockIdx.x] = globaltimer();
        if (cs.abort) break;
    }
    // Every CTA read the epoch before producing its first outputs, and CTA 0's
    // last op consumed outputs of every CTA: the next launch may use e + 1.
    // (Also after a failed wait, so that no later launch mistakes this one's
    // words for its own.)
    if (blockIdx.x == 0 && tid == 0) *reinterpret_cast<volatile uint32_t *>(a.epoch) = epoch + 1;
}

cudaError_t launch_engine(const EngineArgs &a, int grid, size_t smem, cudaStream_t s, bool frame) {
    static bool configured = false;
    if (!configured) {
        for (auto k : {engine_kernel<false>, engine_kernel<true>}) {
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kEngineSmemMax);
            if (e) return e;
        }
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kEngineThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return frame ? cudaLaunchKernelEx(&cfg, engine_kernel<true>, a) : cudaLaunchKernelEx(&cfg, engine_kernel<false>, a);
}

int engine_weight_format(int gtype) {
    switch (gtype) {
    case 1: return EW_F16;
    case 8: return EW_Q8_0;
    case 12: return EW_Q4_K;
    }
    return -1;
}

size_t engine_weight_bytes(int gtype, int N, int K, int mats) {
    const int wt = engine_weight_format(gtype);
    return wt < 0 ? 0 : (size_t)N * engine_row_bytes(wt, K) * mats;
}

cudaError_t launch_engine_relayout(const void *W, const void *W2, int gtype, int N, int K, int n_contig,
                                   int row_base, int extra_row, int grid, int slot_bytes, void *dst,
                                   cudaStream_t s) {
    const int wt = engine_weight_format(gtype);
    if (wt < 0 || N <= 0 || K <= 0 || grid <= 0) return cudaErrorInvalidValue;
    if (K % (wt == EW_F16 ? 8 : wt == EW_Q8_0 ? 256 : 256)) return cudaErrorInvalidValue;
    relayout_kernel<<<N, 128, 0, s>>>(reinterpret_cast<const uint8_t *>(W), reinterpret_cast<const uint8_t *>(W2),
                                      gtype, wt, N, K, n_contig, row_base, extra_row, grid, slot_bytes,
                                      reinterpret_cast<uint8_t *>(dst));
    return cudaGetLastError();
}

}  // namespace s2d
