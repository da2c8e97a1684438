// s2d_sample.cuh -- the device sampler shared by sample_kernel
// (s2d_kernels.cu) and the persistent engine's sample op (s2d_engine.cu).
#pragma once

#include <math.h>
#include <stdint.h>

#include "s2d_common.cuh"
#include "s2d_kernels.cuh"

namespace s2d {

// ---------------------------------------------------------------------------
// Device sampler: sample_token (sampling.rs:121-200) with apply_softmax
// (:202-225), sample_discrete (:227-241) and the SeededRng LCG (:46-52), plus
// the semantic masking of sample_semantic_token (generate.rs:284-298,
// sampling.rs:76-100) and the loop bookkeeping of generate_codes
// (generate.rs:165-211).
//
// Candidates are the unmasked rows only (the allowed semantic rows and
// <|im_end|> for the Slow-AR head; every code for the Fast-AR head).  The
// reference sorts the whole vocabulary; all other entries are -inf there, so
// they sit after the finite entries in id order and carry zero probability.
// The sampler reproduces the reference's item list exactly, including those
// -inf entries when top-k/top-p reach them:
//   greedy fast path: temperature 0, top_p <= 1 and a unique maximum (no
//   other logit within 1e-6) -> the reference's draw always picks item 0;
//   general path: one block bitonic-sorts (value desc, id asc) keys, which is
//   the order of the reference's stable sort, then thread 0 runs the
//   reference's sequential top-k / force-include / softmax / top-p /
//   renormalise / draw steps with the same f32 sums.
// Every call consumes exactly one RNG draw, like the reference.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t f2ord(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float draw_to_target(uint64_t bits) {
    const uint64_t mant = (bits >> 11) & ((1ull << 53) - 1ull);
    const double draw = (double)mant / 9007199254740992.0;
    float t = __double2float_rn(draw);
    t = fminf(fmaxf(t, 0.0f), 1.0f - 1e-7f);
    return t;
}

__device__ __forceinline__ float rng_target(uint64_t *state) {
    *state = *state * 6364136223846793005ull + 1ull;
    return draw_to_target(*state);
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011): ten rounds of two 32x32->64 multiplies with the
// Weyl-sequence key schedule.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += 0x9E3779B9u;
        k.y += 0xBB67AE85u;
    }
    return c;
}

// One draw in [0, 1 - 1e-7]: the LCG step, or Philox on the counter
// (draw index, sequence) with the draw index advanced.
__device__ __forceinline__ float rng_draw(uint64_t *state, int kind, uint64_t key, uint32_t seq) {
    if (kind != RNG_PHILOX) return rng_target(state);
    const uint64_t n = *state;
    *state = n + 1;
    const uint4 r = philox4x32_10(make_uint4((uint32_t)n, (uint32_t)(n >> 32), seq, 0u),
                                  make_uint2((uint32_t)key, (uint32_t)(key >> 32)));
    return draw_to_target(((uint64_t)r.y << 32) | r.x);
}

struct SampleShared {
    float maxv;
    int count;      // logits within 1e-6 of the max
    int first_tie;  // candidate index of the (unique) maximum
    int nfin;       // finite candidates
    int kk;         // finite items inside top-k
    int appended;   // force id appended after top-k
    int nf;         // finite items in the list
    int token;
    int force_pos;  // sorted position of the force id if its logit is finite
    float force_v;
    int fin_below;  // finite candidates with an id below the force id
    long long always_pos;
    int general;
};

// The shared memory of one sampler block besides its key and probability
// arrays.
struct SampleScratch {
    SampleShared sh;
    float rv[32];
    int ri[32], rj[32];
    int sel_hist[256];
    unsigned long long sel_keys[kSampleSelMax], sel_prefix, sel_fkey;
    int sel_need, sel_level, sel_count, sel_rank;
};

// One sampler block of T threads (thread index tid = threadIdx.x < T) over
// the candidates logits[0, a.n) of sequence sq: returns the token and applies
// the mode's DevState / code bookkeeping (thread 0).  skeys holds up to
// max(MAXN rounded up to a power of two) keys and probs MAXN + 1 floats;
// MAXN bounds a.n (the caller checks).  sync() is a barrier of exactly the
// T threads.  The caller has already returned for a finished sequence.
template <int T, int MAXN, class Sync>
__device__ uint32_t sample_block(const SampleArgs &a, uint32_t sq, const float *logits, unsigned long long *skeys,
                                 float *probs, SampleScratch &S, Sync sync) {
    static_assert(MAXN % T == 0, "candidates per thread");
    SampleShared &sh = S.sh;
    float *rv = S.rv;
    int *ri = S.ri, *rj = S.rj, *sel_hist = S.sel_hist;
    unsigned long long *sel_keys = S.sel_keys;
    unsigned long long &sel_prefix = S.sel_prefix, &sel_fkey = S.sel_fkey;
    int &sel_need = S.sel_need, &sel_level = S.sel_level, &sel_count = S.sel_count, &sel_rank = S.sel_rank;
    const uint32_t rseq = a.rng_seq + sq;
    DevState *st = a.st ? a.st + sq : nullptr;
    uint64_t *rng = a.batched ? &st->rng : a.rng;
    int32_t *frame_codes = a.frame_codes ? a.frame_codes + sq * a.frame_stride : nullptr;
    int32_t *codes_out = a.codes_out ? a.codes_out + sq * a.codes_stride : nullptr;
    uint32_t *out_token = a.out_token ? a.out_token + sq : nullptr;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = a.n;

    bool block = false;
    int64_t force = a.force_id;
    int32_t new_npast = 0, new_step = 0;
    if (a.mode == SAMPLE_SLOW_FIRST) {
        block = 0u < a.min_tokens_before_end;
        force = block ? -1 : (int64_t)a.im_end;
    } else if (a.mode == SAMPLE_SLOW_STEP) {
        new_npast = st->n_past + 1;
        new_step = st->step_index + 1;
        const uint32_t gen = (uint32_t)(new_npast - st->prompt_cols + new_step);
        block = gen < a.min_tokens_before_end;
        force = block ? -1 : (int64_t)a.im_end;
    } else if (a.mode == SAMPLE_FAST) {
        force = -1;
    }
    const bool slow = a.mode == SAMPLE_SLOW_FIRST || a.mode == SAMPLE_SLOW_STEP;
    auto cid = [&](int r) -> uint32_t {
        return a.n_contig < 0 ? (uint32_t)r : (r < a.n_contig ? a.id_base + (uint32_t)r : a.extra_id);
    };
    // -0.0 is folded into +0.0: the reference's partial_cmp sees them equal,
    // so their order must come from the id alone.
    auto cval = [&](int r) -> float {
        const float v = logits[r];
        return (slow && block && cid(r) == a.im_end) ? -INFINITY : (v == 0.0f ? 0.0f : v);
    };

    // pass 1: max and finite count
    float mx = -INFINITY;
    int fin = 0;
    for (int r = tid; r < n; r += T) {
        const float v = cval(r);
        mx = fmaxf(mx, v);
        fin += v > -INFINITY;
    }
    mx = warp_max(mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) fin += __shfl_xor_sync(0xffffffffu, fin, o);
    if (lane == 0) rv[warp] = mx, ri[warp] = fin;
    sync();
    if (tid == 0) {
        float m2 = -INFINITY;
        int f2 = 0;
        for (int w = 0; w < T / 32; ++w) m2 = fmaxf(m2, rv[w]), f2 += ri[w];
        sh.maxv = m2;
        sh.nfin = f2;
    }
    sync();
    // pass 2: entries within 1e-6 of the max
    int cnt = 0, first = 0x7fffffff;
    for (int r = tid; r < n; r += T) {
        const float v = cval(r);
        if (fabsf(v - sh.maxv) < 1e-6f) {
            ++cnt;
            first = min(first, r);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
        first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    }
    if (lane == 0) ri[warp] = cnt, rj[warp] = first;
    sync();
    const int64_t k_eff = a.top_k > 0 ? min((int64_t)a.top_k, a.vocab_full) : a.vocab_full;
    if (tid == 0) {
        int c2 = 0, f2 = 0x7fffffff;
        for (int w = 0; w < T / 32; ++w) c2 += ri[w], f2 = min(f2, rj[w]);
        sh.count = c2;
        sh.first_tie = f2;
        sh.general = !(a.temperature == 0.0f && a.top_p <= 1.0f && isfinite(sh.maxv) && c2 == 1 &&
                       k_eff >= 1);
        if (!sh.general) {
            (void)rng_draw(rng, a.rng_kind, a.philox_key, rseq);
            sh.token = (int)cid(f2);
        }
    }
    sync();

    if (sh.general) {
        const int nkeep = (int)min(k_eff, (int64_t)sh.nfin);  // the top-k items that are finite
        const bool select = k_eff <= kSampleSelMax;
        if (tid == 0) sh.force_pos = 0x7fffffff, sh.force_v = -INFINITY, sh.fin_below = 0;
        if (select) {
            // Only the first nkeep entries of the sorted list are read (the
            // -inf entries behind them only when nkeep == nfin): radix-select
            // the nkeep smallest (value desc, id asc) keys, 8 bits a level,
            // then place each by its rank among them.
            unsigned long long kr[MAXN / T];
#pragma unroll
            for (int i = 0; i < MAXN / T; ++i) {
                const int r = tid + i * T;
                kr[i] = r < n ? ((unsigned long long)(~f2ord(cval(r))) << 32) | cid(r) : ~0ull;
            }
            if (tid == 0) sel_prefix = 0ull, sel_need = nkeep, sel_level = 0, sel_count = 0, sel_fkey = ~0ull, sel_rank = 0;
            sync();
            for (int lev = 1; lev <= 8 && nkeep > 0; ++lev) {
                const int shift = 64 - 8 * lev;
                if (tid < 256) sel_hist[tid] = 0;
                sync();
                const unsigned long long pre = sel_prefix;
#pragma unroll
                for (int i = 0; i < MAXN / T; ++i)
                    if (lev == 1 || (kr[i] >> (shift + 8)) == pre) atomicAdd(&sel_hist[(kr[i] >> shift) & 255u], 1);
                sync();
                if (warp == 0) {
                    int c[8], tot = 0;
#pragma unroll
                    for (int j = 0; j < 8; ++j) c[j] = sel_hist[lane * 8 + j], tot += c[j];
                    int incl = tot;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int y = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= o) incl += y;
                    }
                    const int need = sel_need;
                    int b = incl - tot;
                    if (b < need && need <= incl) {
                        int d = 0;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            if (b + c[j] >= need) {
                                d = j;
                                break;
                            }
                            b += c[j];
                        }
                        // the need-th key lies in bin lane * 8 + d: every key of a
                        // lower bin is kept, and the whole bin once it holds no more
                        sel_prefix = (pre << 8) | (unsigned long long)(lane * 8 + d);
                        sel_need = need - b;
                        if (c[d] == need - b) sel_level = lev;
                    }
                }
                sync();
                if (sel_level) break;
            }
            if (nkeep > 0) {
                const int shift = 64 - 8 * sel_level;
                const unsigned long long pre = sel_prefix;
#pragma unroll
                for (int i = 0; i < MAXN / T; ++i)
                    if ((shift == 64 ? 0ull : kr[i] >> shift) <= pre) {
                        const int pos = atomicAdd(&sel_count, 1);
                        if (pos < kSampleSelMax) sel_keys[pos] = kr[i];
                    }
            }
            sync();
            if (tid < nkeep) {
                const unsigned long long key = sel_keys[tid];
                int rank = 0;
                for (int j = 0; j < nkeep; ++j) rank += sel_keys[j] < key;
                skeys[rank] = key;
            }
            // Position of a finite force id among the sorted entries: the
            // number of keys below its own.
            if (force >= 0 && force < a.vocab_full) {
#pragma unroll
                for (int i = 0; i < MAXN / T; ++i) {
                    const int r = tid + i * T;
                    if (r < n && (int64_t)cid(r) == force && cval(r) > -INFINITY) sel_fkey = kr[i], sh.force_v = cval(r);
                }
            }
            sync();
            const unsigned long long fk = sel_fkey;
            if (fk != ~0ull) {
                int less = 0;
#pragma unroll
                for (int i = 0; i < MAXN / T; ++i) less += kr[i] < fk;
                if (less) atomicAdd(&sel_rank, less);
            }
            sync();
            if (tid == 0 && fk != ~0ull) sh.force_pos = sel_rank;
            sync();
        } else {
            // bitonic sort of (value desc, id asc) keys
            int np2 = 2;
            while (np2 < n) np2 <<= 1;
            for (int r = tid; r < np2; r += T) {
                if (r < n) {
                    const float v = cval(r);
                    skeys[r] = ((unsigned long long)(~f2ord(v)) << 32) | cid(r);
                } else {
                    skeys[r] = ~0ull;
                }
            }
            sync();
            for (int k = 2; k <= np2; k <<= 1) {
                for (int j = k >> 1; j > 0; j >>= 1) {
                    for (int i = tid; i < np2; i += T) {
                        const int ixj = i ^ j;
                        if (ixj > i) {
                            const unsigned long long x = skeys[i], y = skeys[ixj];
                            const bool up = (i & k) == 0;
                            if ((x > y) == up) skeys[i] = y, skeys[ixj] = x;
                        }
                    }
                    sync();
                }
            }
            // Position of the force id in the reference's sorted list: among the
            // sorted finite entries if its logit is finite (sampling.rs:146-168).
            if (force >= 0 && force < a.vocab_full) {
                for (int r = tid; r < sh.nfin; r += T) {
                    if ((uint32_t)(skeys[r] & 0xffffffffu) == (uint32_t)force) {
                        sh.force_pos = r;
                        const uint32_t ord = ~(uint32_t)(skeys[r] >> 32);
                        sh.force_v = __uint_as_float((ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord);
                    }
                }
            }
            sync();
        }
        // otherwise among the -inf entries, which follow in id order
        if (force >= 0 && force < a.vocab_full) {
            int below = 0;
            for (int r = tid; r < n; r += T)
                below += (cval(r) > -INFINITY) && ((int64_t)cid(r) < force);
            if (below) atomicAdd(&sh.fin_below, below);
        }
        sync();
        if (tid == 0) {
            const int64_t kk = min(k_eff, (int64_t)sh.nfin);
            int appended = 0;
            int64_t always_pos = -1;
            if (force >= 0 && force < a.vocab_full) {
                const bool finite = sh.force_pos != 0x7fffffff;
                const int64_t P = finite ? (int64_t)sh.force_pos
                                         : (int64_t)sh.nfin + force - (int64_t)sh.fin_below;
                if (!finite) sh.force_v = -INFINITY;
                if (P < k_eff) {
                    always_pos = P;
                } else if (sh.force_v > -1e30f) {
                    appended = 1;
                    always_pos = kk;  // appended right after the top-k items
                }
            }
            sh.kk = (int)kk;
            sh.appended = appended;
            sh.nf = (int)kk + appended;
            sh.always_pos = always_pos;
        }
        sync();
        const int nf = sh.nf;
        // item values and probabilities (apply_softmax), in parallel
        const float top = nf > 0 ? sh.maxv : -INFINITY;
        for (int i = tid; i < nf; i += T) {
            float v;
            if (i < sh.kk) {
                const uint32_t ord = ~(uint32_t)(skeys[i] >> 32);
                v = __uint_as_float((ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord);
            } else {
                v = sh.force_v;
            }
            probs[i] = a.temperature > 0.0f ? expf((v - top) / a.temperature)
                                            : (fabsf(v - top) < 1e-6f ? 1.0f : 0.0f);
        }
        sync();
        if (tid == 0) {
            const int64_t n_items = k_eff + sh.appended;
            int64_t choice;
            if (nf == 0) {
                (void)rng_draw(rng, a.rng_kind, a.philox_key, rseq);
                choice = n_items - 1;
            } else {
                float sum = 0.0f;
                for (int i = 0; i < nf; ++i) sum += probs[i];
                if (sum > 0.0f)
                    for (int i = 0; i < nf; ++i) probs[i] /= sum;
                const int64_t always_pos = sh.always_pos;
                int64_t p_idx = 0;
                float cum = 0.0f;
                bool broke = false;
                for (int i = 0; i < nf; ++i) {
                    cum += probs[i];
                    p_idx = i + 1;
                    if (cum >= a.top_p) {
                        broke = true;
                        break;
                    }
                }
                if (!broke) p_idx = n_items;
                if (p_idx == 0) p_idx = 1;
                if (always_pos >= 0 && always_pos >= p_idx) p_idx = always_pos + 1;
                const int lim = (int)min(p_idx, (int64_t)nf);
                float sum_p = -0.0f;
                for (int i = 0; i < lim; ++i) sum_p += probs[i];
                if (sum_p > 0.0f)
                    for (int i = 0; i < lim; ++i) probs[i] /= sum_p;
                const float target = rng_draw(rng, a.rng_kind, a.philox_key, rseq);
                choice = p_idx - 1;
                float c2 = 0.0f;
                for (int i = 0; i < lim; ++i) {
                    c2 += probs[i];
                    if (target < c2) {
                        choice = i;
                        break;
                    }
                }
            }
            if (choice < sh.kk) {
                sh.token = (int)(uint32_t)(skeys[choice] & 0xffffffffu);
            } else if (sh.appended && choice == sh.kk) {
                sh.token = (int)force;
            } else {
                // the j-th -inf entry in id order: ids that are not finite candidates
                const int64_t j = choice - sh.kk;
                int64_t ans = j;
                for (int it = 0; it < 64; ++it) {
                    int64_t c = 0;
                    for (int r = 0; r < sh.nfin; ++r)
                        c += (int64_t)(uint32_t)(skeys[r] & 0xffffffffu) <= ans;
                    if (j + c == ans) break;
                    ans = j + c;
                }
                sh.token = (int)ans;
            }
        }
        sync();
    }

    const uint32_t token = (uint32_t)sh.token;
    if (tid == 0) {
        if (out_token) *out_token = token;
        if (a.mode == SAMPLE_SLOW_FIRST) {
            st->main_token = token;
            st->done = (token == a.im_end) || (a.max_new <= 0);
        } else if (a.mode == SAMPLE_SLOW_STEP) {
            st->n_past = new_npast;
            st->step_index = new_step;
            st->main_token = token;
            st->done = (token == a.im_end) || (new_step >= a.max_new);
        } else if (a.mode == SAMPLE_FAST) {
            frame_codes[a.cb_index] = (int32_t)token;
            if (codes_out) codes_out[(size_t)a.cb_index * a.max_new + st->step_index] = (int32_t)token;
        }
    }
    return token;
}

}  // namespace s2d
