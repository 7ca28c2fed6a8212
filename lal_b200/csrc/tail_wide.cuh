/*
 * tail_wide.cuh -- the select and draw of a candidate set of any size, by one
 * CTA, for the inputs the fast selects cannot hold:
 *
 *  - ties at the threshold T that crowd a CTA's slot of the small-k select or
 *    exceed the shared-memory superset and candidate arrays.  An all-zero
 *    hidden vector makes every logit 0.0, so every row of the vocabulary is a
 *    candidate; LM-head rows duplicated bit for bit tie exactly;
 *  - a vocab-sharded slice whose tie-complete set {l >= T_s} does not fit its
 *    candidate record.
 *
 * The reference returns a token for every such input
 * (runtime/lal_sampling.h:70-124): T is the k-th largest logit counted with
 * multiplicity, every row with l >= T is a candidate, max_l is the largest of
 * them, and the weights expf((l - max_l) / temp) are summed in ascending row
 * order before the draw scans the same order.  Here:
 *
 *   1. T exactly, by an MSB-first radix select over the slice's logits in
 *      global memory (4 passes of 8 bits);
 *   2. the rows with l > T -- fewer than k -- as an explicit list in ascending
 *      row order, and the number of rows with l == T;
 *   3. the walk: one thread adds the weights in ascending row order, the
 *      explicit rows' own and one shared weight for every tie, reading the
 *      ties as a bitmap that the CTA stages 8192 rows at a time.  The running
 *      sum at each chunk end is kept, so the draw re-walks one chunk.
 *
 * A sharded slice in this case exports its rows l > T_s explicitly and its
 * ties as a bitmap of its rows (the record's wide form); the merge walks the
 * records in rank order with the same walk.
 */
#pragma once

#include "tail_device.cuh"

namespace lal {
namespace {

/* bitmap words staged per chunk of the walk (8192 rows) */
constexpr int kWideChunkWords = 256;
/* chunks whose running sums the draw can revisit; with more, it re-walks */
constexpr int kWideChunkTab = 512;

struct WideChunk {
    int unit, w0, nw, pe0;
    float acc0, acc1; /* running sum before and after the chunk */
};

/* shared memory of the walk: the staged bitmap words and the chunk table */
constexpr int kWideWalkBytes = 4 * kWideChunkWords + 24 * kWideChunkTab;
static_assert(sizeof(WideChunk) == 24, "WideChunk layout");

/* shared memory of the dense wide path holding up to cap explicit rows
 * (unsorted keys + rows, sorted keys + rows + weights) */
__host__ __device__ constexpr int wide_area_bytes(int cap) {
    return 20 * ((cap + 3) / 4 * 4) + kWideWalkBytes;
}

__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, Misc *ms) {
    v = __reduce_max_sync(0xffffffffu, v);
    if ((threadIdx.x & 31) == 0) ms->scan[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t r = ms->scan[0];
    for (int w = 1; w < NWARP; ++w) r = max(r, ms->scan[w]);
    __syncthreads();
    return r;
}
__device__ __forceinline__ uint32_t block_min_u32(uint32_t v, Misc *ms) {
    v = __reduce_min_sync(0xffffffffu, v);
    if ((threadIdx.x & 31) == 0) ms->scan[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t r = ms->scan[0];
    for (int w = 1; w < NWARP; ++w) r = min(r, ms->scan[w]);
    __syncthreads();
    return r;
}

/* k-th largest key of a multiset given as n entries, entry i standing for
 * `weight` copies of `key` (get(i, key, weight) returns whether it takes
 * part); 1 <= k <= the total weight.  MSB-first radix select, 8-bit digits. */
template <class Get>
__device__ uint32_t block_kth_largest_w(Get get, int n, uint32_t k, Misc *ms) {
    uint32_t prefix = 0, mask = 0, krem = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += NT) ms->hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += NT) {
            uint32_t key = 0u, w = 0u;
            if (get(i, key, w) && w > 0u && (key & mask) == prefix)
                atomicAdd(&ms->hist[(key >> shift) & 0xFFu], w);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t run = 0u;
            int d = 255;
            for (; d > 0; --d) {
                if (run + ms->hist[d] >= krem) break;
                run += ms->hist[d];
            }
            ms->sh[0] = (uint32_t)d;
            ms->sh[1] = run;
        }
        __syncthreads();
        prefix |= ms->sh[0] << shift;
        mask |= 0xFFu << shift;
        krem -= ms->sh[1];
        __syncthreads();
    }
    return prefix;
}

/* expf((l - max_l) / temp) exactly as glibc computes it (the sampler's
 * weight, runtime/lal_sampling.h:112) */
struct ExpfTables {
    const uint32_t *x, *y, *bits, *off;
    const uint4 *hash;
    int hash_probe;
    __device__ float weight(float l, float max_l, float temp) const {
        const float v = __fdiv_rn(__fsub_rn(l, max_l), temp);
        return hash ? expf_hash_finish(v, expf_hash_load(v, hash), hash, hash_probe)
                    : sampler_expf(v, x, y, bits, off);
    }
};

/* One unit of the walk: explicit candidates (keys, global rows, weights, in
 * ascending row order) and, when `tie` is set, the unit's rows whose key
 * equals T, given as a bitmap of rows [row0, row0 + rows) that the walk's
 * fill stages into shared memory.  Explicit rows lie inside the unit's rows;
 * in a tie unit every explicit row is above T. */
struct WalkUnit {
    const uint32_t *key;
    const int *row;
    const float *w;
    int n;
    int tie;
    int row0, rows;
};

/* Thread 0: add one chunk's candidates to acc in ascending row order (a
 * chunk of a tie unit is nw staged bitmap words from word w0; a unit without
 * ties is one chunk of its explicit rows l >= T).  pe = the next explicit
 * entry.  In draw mode, stops at the first candidate with r <= acc. */
__device__ __noinline__ bool walk_chunk(const WalkUnit &U, const uint32_t *bm, int w0, int nw,
                                        int &pe, uint32_t T, float wT, float &acc, bool draw,
                                        float r, int &tok) {
    if (!U.tie) {
        for (; pe < U.n; ++pe) {
            if (U.key[pe] < T) continue;
            acc = __fadd_rn(acc, U.w[pe]);
            if (draw && r <= acc) {
                tok = U.row[pe];
                ++pe;
                return true;
            }
        }
        return false;
    }
    for (int w = 0; w < nw; ++w) {
        const int rlo = U.row0 + 32 * (w0 + w), rhi = rlo + 32;
        uint32_t bits = bm[w];
        if (!draw && bits == 0xffffffffu && !(pe < U.n && U.row[pe] < rhi)) {
            /* 32 ties in a row: the same 32 sequential adds, unrolled */
#pragma unroll
            for (int q = 0; q < 32; ++q) acc = __fadd_rn(acc, wT);
            continue;
        }
        for (;;) {
            const bool he = pe < U.n && U.row[pe] < rhi;
            if (!he && bits == 0u) break;
            const int te = he ? U.row[pe] : 0x7fffffff;
            const int tb = bits ? rlo + __ffs(bits) - 1 : 0x7fffffff;
            float wt;
            int rw;
            if (te < tb) {
                wt = U.w[pe];
                rw = te;
                ++pe;
            } else {
                wt = wT;
                rw = tb;
                bits &= bits - 1u;
            }
            acc = __fadd_rn(acc, wt);
            if (draw && r <= acc) {
                tok = rw;
                return true;
            }
        }
    }
    return false;
}

struct WalkResult {
    float sum, r;
    int token; /* the row drawn, or -1: none reached r (the caller's fallthrough) */
    int drew;
    int ok;    /* every fill succeeded (peer words arrived in time) */
};

/* The sum and the draw over n_units units in order (every thread of the CTA
 * calls it).  unit_of(u) describes unit u; fill(u, w0, nw, dst) stages nw
 * bitmap words of unit u from word w0 into dst (all threads; it clears
 * ms->sh[12] when a word cannot be had).  Greedy: the first candidate (all
 * weights must then be 0).  SERVER with sum <= 0: row 0, no draw -- every
 * candidate then lies at or below -1e30, where the reference's argmax keeps
 * its initial row (tools/server/qwen7b_server.c:285-286). */
template <class UnitOf, class Fill>
__device__ WalkResult wide_walk(int n_units, UnitOf unit_of, Fill fill, uint32_t T, float wT,
                                bool greedy, float u, int variant, uint32_t *bm, WideChunk *tab,
                                Misc *ms, float r_direct = -1.0f) {
    const int tid = threadIdx.x;
    float acc = 0.0f;
    int ntab = 0, tok = -1;
    if (tid == 0) {
        ms->sh[12] = 1u;
        ms->found = -1;
        ms->sum = 0.0f;
        ms->sh[13] = 0u;
    }
    __syncthreads();
    if (!greedy) {
        for (int uu = 0; uu < n_units; ++uu) {
            const WalkUnit U = unit_of(uu);
            int pe = 0;
            if (!U.tie) {
                if (tid == 0) {
                    const float a0 = acc;
                    walk_chunk(U, bm, 0, 0, pe, T, wT, acc, false, 0.0f, tok);
                    if (ntab < kWideChunkTab) tab[ntab] = WideChunk{uu, 0, 0, 0, a0, acc};
                    ++ntab;
                }
                continue;
            }
            const int words = (U.rows + 31) >> 5;
            for (int w0 = 0; w0 < words; w0 += kWideChunkWords) {
                const int nw = min(kWideChunkWords, words - w0);
                __syncthreads(); /* the previous chunk's words are consumed */
                fill(uu, w0, nw, bm);
                __syncthreads();
                if (tid == 0) {
                    const int pe0 = pe;
                    const float a0 = acc;
                    walk_chunk(U, bm, w0, nw, pe, T, wT, acc, false, 0.0f, tok);
                    if (ntab < kWideChunkTab) tab[ntab] = WideChunk{uu, w0, nw, pe0, a0, acc};
                    ++ntab;
                }
            }
        }
        if (tid == 0) {
            ms->sum = acc;
            ms->sh[13] = (uint32_t)ntab;
        }
    }
    __syncthreads();
    WalkResult res;
    res.ok = ms->sh[12] != 0u;
    res.sum = ms->sum;
    res.r = 0.0f;
    res.drew = 0;
    res.token = -1;
    if (!res.ok) return res;
    if (!greedy && r_direct < 0.0f && variant == VARIANT_SERVER && res.sum <= 0.0f) {
        res.token = 0;
        return res;
    }
    /* r_direct >= 0: find the first row whose running sum reaches it */
    const float r = greedy ? -1.0f : r_direct >= 0.0f ? r_direct : __fmul_rn(u, res.sum);
    if (!greedy) {
        res.r = r;
        res.drew = 1;
    }
    const int nt = (int)ms->sh[13];
    if (!greedy && nt <= kWideChunkTab) {
        /* the first chunk whose running sum reaches r holds the row */
        if (tid == 0) {
            int c = -1;
            for (int i = 0; i < nt; ++i)
                if (r <= tab[i].acc1) {
                    c = i;
                    break;
                }
            ms->sh[11] = (uint32_t)c;
        }
        __syncthreads();
        const int c = (int)ms->sh[11];
        if (c >= 0) {
            const WideChunk ch = tab[c];
            const WalkUnit U = unit_of(ch.unit);
            if (U.tie) fill(ch.unit, ch.w0, ch.nw, bm);
            __syncthreads();
            if (tid == 0) {
                float a = ch.acc0;
                int pe = ch.pe0, t = -1;
                if (walk_chunk(U, bm, ch.w0, ch.nw, pe, T, wT, a, true, r, t)) ms->found = t;
            }
        }
    } else {
        /* greedy (the first candidate), or more chunks than the table holds:
         * walk from the start until the row is found */
        acc = 0.0f;
        for (int uu = 0; uu < n_units; ++uu) {
            const WalkUnit U = unit_of(uu);
            int pe = 0;
            if (!U.tie) {
                if (tid == 0) {
                    int t = -1;
                    if (walk_chunk(U, bm, 0, 0, pe, T, wT, acc, true, r, t)) ms->found = t;
                }
            } else {
                const int words = (U.rows + 31) >> 5;
                for (int w0 = 0; w0 < words; w0 += kWideChunkWords) {
                    const int nw = min(kWideChunkWords, words - w0);
                    __syncthreads();
                    fill(uu, w0, nw, bm);
                    __syncthreads();
                    if (tid == 0) {
                        int t = -1;
                        if (walk_chunk(U, bm, w0, nw, pe, T, wT, acc, true, r, t)) ms->found = t;
                    }
                    __syncthreads();
                    if (ms->found >= 0) break;
                }
            }
            __syncthreads();
            if (ms->found >= 0) break;
        }
    }
    __syncthreads();
    res.ok = ms->sh[12] != 0u;
    res.token = ms->found;
    __syncthreads();
    return res;
}

/* Inputs and outputs of the dense wide path: the select of one slice's
 * logits and then one of -- the draw (token, diagnostics, history push); the
 * wide form of the slice's shard record (gathered, or stored into every
 * rank's receive buffer); the candidate export of the filter hook. */
struct WideDense {
    const float *lg; /* the slice's penalised logits [rows], global memory */
    int rows, row_base, vocab, k, variant, greedy;
    float temp, u;
    int cap; /* explicit rows the area holds: >= k - 1 */
    ExpfTables ex;
    /* the draw */
    int *token;
    unsigned long long *host_tok; /* completion word (notify_host), or null */
    unsigned host_seq;
    StreamDiag *diag;
    int *hist_ids, *hist_n, *hist_head;
    int hist_cap, push_history, hn, hhead;
    /* the shard record: gathered (rec) or peer stores (peer_recv) */
    uint8_t *rec;
    int rec_cap;
    uint8_t *const *peer_recv;
    int n_ranks, rank, rec_bytes;
    unsigned seq;
    /* the filter hook's candidate export */
    float *cand_val;
    int *cand_idx;
    int cand_cap, candidates_only;
    /* VARIANT_GPT2: the server's nucleus when 0 < top_p < 1 */
    float top_p;
};

/* The GPT-2 server's nucleus (gpt2_server.c:2908-2955) over the m
 * candidates of a step: Oi their rows in ascending order, Ce their terms
 * expf((l - max_l) / T).  Every thread calls it.  The terms are summed in row
 * order, inv = 1 / (sum + 1e-12f), each probability is term * inv; the rows
 * are taken in the order of the server's insertion sort (descending
 * probability, equal probabilities by ascending row) until the running
 * probability reaches top_p, the row that reaches it included.  The largest
 * term stays (it is first in that order), so the kept rows' softmax over
 * their own maximum has the same terms: on return Ce holds them for kept rows
 * and 0 for the rest.  P, R, Q: scratch of m entries.  Returns the count
 * kept. */
__device__ __noinline__ int gpt2_nucleus(float top_p, int m, float *Ce, float *P, int *R,
                                         float *Q, Misc *ms) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        float acc = 0.0f;
        for (int i = 0; i < m; ++i) acc = __fadd_rn(acc, Ce[i]);
        ms->sum = acc;
    }
    __syncthreads();
    const float inv = __fdiv_rn(1.0f, __fadd_rn(ms->sum, 1e-12f));
    for (int i = tid; i < m; i += NT) P[i] = __fmul_rn(Ce[i], inv);
    __syncthreads();
    for (int i = tid; i < m; i += NT) {
        const float pi = P[i];
        int r = 0;
        for (int j = 0; j < m; ++j) r += (P[j] > pi) || (P[j] == pi && j < i);
        R[i] = r;
        Q[r] = pi;
    }
    __syncthreads();
    if (tid == 0) {
        float cum = 0.0f;
        int n = m;
        for (int j = 0; j < m; ++j) {
            cum = __fadd_rn(cum, Q[j]);
            if (cum >= top_p) {
                n = j + 1;
                break;
            }
        }
        ms->sh[0] = (uint32_t)n;
    }
    __syncthreads();
    const int n_keep = (int)ms->sh[0];
    for (int i = tid; i < m; i += NT)
        if (R[i] >= n_keep) Ce[i] = 0.0f;
    __syncthreads();
    return n_keep;
}

/* bitmap word w of a slice: bit j set when row 32w + j equals T (warp-wide) */
__device__ __forceinline__ uint32_t tie_word(const float *lg, int rows, int w, uint32_t T) {
    const int row = 32 * w + (int)(threadIdx.x & 31);
    const bool in = row < rows;
    const uint32_t key = in ? f2key(__ldcg(lg + row)) : 0u;
    return __ballot_sync(0xffffffffu, in && key == T);
}

__device__ __forceinline__ void st_sys_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

/* The dense wide path (every thread of the CTA; area >= wide_area_bytes(cap),
 * 16-byte aligned). */
__device__ __noinline__ void wide_dense(const WideDense &a, uint8_t *area, Misc *ms) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c4 = (a.cap + 3) / 4 * 4;
    uint32_t *tk = reinterpret_cast<uint32_t *>(area);
    int *ti = reinterpret_cast<int *>(tk + c4);
    uint32_t *Xk = reinterpret_cast<uint32_t *>(ti + c4);
    int *Xi = reinterpret_cast<int *>(Xk + c4);
    float *Xw = reinterpret_cast<float *>(Xi + c4);
    uint32_t *bm = reinterpret_cast<uint32_t *>(Xw + c4);
    WideChunk *tab = reinterpret_cast<WideChunk *>(bm + kWideChunkWords);
    const float *lg = a.lg;
    const int rows = a.rows;
    const int k = max(1, min(a.k, rows));

    /* 1. T, the k-th largest key with multiplicity */
    const uint32_t T = block_kth_largest(
        [&](int i, uint32_t &key) {
            key = f2key(__ldcg(lg + i));
            return true;
        },
        rows, k, ms);
    /* 2. the rows above T (fewer than k), the ties, the largest key */
    if (tid == 0) ms->cnt = 0u;
    __syncthreads();
    uint32_t n_eq = 0u, top = 0u, first = 0xffffffffu;
    for (int i = tid; i < rows; i += NT) {
        const uint32_t key = f2key(__ldcg(lg + i));
        top = max(top, key);
        if (key == T) {
            ++n_eq;
            first = min(first, (uint32_t)i);
        } else if (key > T) {
            const uint32_t pos = atomicAdd(&ms->cnt, 1u);
            if (pos < (uint32_t)a.cap) {
                tk[pos] = key;
                ti[pos] = i;
            }
        }
    }
    uint32_t ties;
    block_scan_excl(n_eq, ms, &ties);
    top = block_max_u32(top, ms);
    first = block_min_u32(first, ms);
    const int ne = min((int)ms->cnt, a.cap);
    for (int i = tid; i < ne; i += NT) {
        const int me = ti[i];
        int r = 0;
        for (int j = 0; j < ne; ++j) r += ti[j] < me;
        Xk[r] = tk[i];
        Xi[r] = a.row_base + me;
    }
    __syncthreads();
    StreamDiag dg;
    dg.threshold = key2f(T);
    dg.max_l = 0.0f;
    dg.sum = 0.0f;
    dg.r = 0.0f;
    dg.n_cand = ne + (int)ties;
    dg.greedy = a.greedy ? 1 : 0;
    dg.drew = 0;
    dg.token = -1;

    /* 3a. the record's wide form: the rows above T_s, then the tie bitmap */
    const int words = (rows + 31) >> 5;
    if (a.rec != nullptr) {
        ShardRecordHead *h = reinterpret_cast<ShardRecordHead *>(a.rec);
        float *rv = reinterpret_cast<float *>(a.rec + sizeof(ShardRecordHead));
        int *ri = reinterpret_cast<int *>(rv + a.rec_cap);
        uint32_t *rb = reinterpret_cast<uint32_t *>(ri + a.rec_cap);
        for (int i = tid; i < ne; i += NT) {
            rv[i] = key2f(Xk[i]);
            ri[i] = Xi[i];
        }
        for (int w = warp; w < words; w += NWARP) {
            const uint32_t b = tie_word(lg, rows, w, T);
            if (lane == 0) rb[w] = b;
        }
        if (tid == 0) {
            h->count = ne;
            h->status = 0;
            h->ties = (int)ties;
            h->tkey = T;
            if (a.diag) *a.diag = dg;
        }
        return;
    }
    if (a.peer_recv != nullptr) {
        /* 64-bit stores tagged with the step's sequence number (see
         * peer_publish): [count], [status], [ties], [T_s key], the entries
         * (value, row), then the bitmap words after rec_cap entries */
        const size_t slot = ((size_t)(a.seq & 1u) * a.n_ranks + a.rank) * a.rec_bytes;
        const uint64_t hi = (uint64_t)a.seq << 32;
        for (int r = 0; r < a.n_ranks; ++r) {
            uint64_t *w64 = reinterpret_cast<uint64_t *>(a.peer_recv[r] + slot);
            for (int i = tid; i < ne; i += NT)
                st_sys_pair(w64 + 4 + 2 * i, hi | __float_as_uint(key2f(Xk[i])),
                            hi | (uint32_t)Xi[i]);
            for (int w = warp; w < words; w += NWARP) {
                const uint32_t b = tie_word(lg, rows, w, T);
                if (lane == 0) st_sys_u64(w64 + 4 + 2 * a.rec_cap + w, hi | b);
            }
            if (tid == 0) {
                st_sys_pair(w64, hi | (uint32_t)ne, hi);
                st_sys_pair(w64 + 2, hi | ties, hi | T);
            }
        }
        if (tid == 0 && a.diag) *a.diag = dg;
        __syncthreads();
        return;
    }

    const float max_l = fmaxf(-1e30f, key2f(top));
    dg.max_l = max_l;
    /* 3b. the filter hook: every candidate, ascending rows */
    if (a.candidates_only) {
        uint32_t base = 0u;
        for (int i0 = 0; i0 < rows; i0 += NT) {
            const int i = i0 + tid;
            const uint32_t key = i < rows ? f2key(__ldcg(lg + i)) : 0u;
            const bool c = i < rows && key >= T;
            uint32_t tot;
            const uint32_t pos = base + block_scan_excl(c ? 1u : 0u, ms, &tot);
            if (c && pos < (uint32_t)a.cand_cap) {
                a.cand_val[pos] = key2f(key);
                a.cand_idx[pos] = a.row_base + i;
            }
            base += tot;
        }
        if (tid == 0 && a.diag) *a.diag = dg;
        return;
    }

    /* 3c. the draw */
    int token;
    WalkResult res;
    res.sum = 0.0f;
    res.r = 0.0f;
    res.drew = 0;
    if (a.greedy) {
        token = a.row_base + (int)first; /* k = 1: T is the maximum */
    } else {
        for (int i = tid; i < ne; i += NT) Xw[i] = a.ex.weight(key2f(Xk[i]), max_l, a.temp);
        if (tid == 0) ms->fred[0] = a.ex.weight(key2f(T), max_l, a.temp);
        __syncthreads();
        float wT = ms->fred[0];
        /* ties count only up to row tie_end (the nucleus may cut them) */
        int tie_end = rows;
        auto fill = [&](int, int w0, int nw, uint32_t *dst) {
            for (int w = warp; w < nw; w += NWARP) {
                uint32_t b = tie_word(lg, rows, w0 + w, T);
                const int lo = 32 * (w0 + w);
                if (lo + 32 > tie_end) b &= lo >= tie_end ? 0u : (1u << (tie_end - lo)) - 1u;
                if (lane == 0) dst[w] = b;
            }
        };
        WalkUnit U{Xk, Xi, Xw, ne, 1, a.row_base, rows};
        if (a.variant == VARIANT_GPT2 && a.top_p > 0.0f && a.top_p < 1.0f) {
            /* gpt2_server.c:2908-2955 with every tie sharing one probability
             * pT: the explicit rows' probabilities are >= pT (a larger logit
             * never weighs less), so the server's order is the rows above pT
             * (descending, equal ones by row), then every row at exactly pT
             * by row -- the ties and the explicit rows that round to pT */
            const WalkResult s1 = wide_walk(1, [&](int) { return U; }, fill, T, wT, false, 0.0f,
                                            VARIANT_LIBRARY, bm, tab, ms, 0.0f);
            const float inv = __fdiv_rn(1.0f, __fadd_rn(s1.sum, 1e-12f));
            const float pT = __fmul_rn(wT, inv);
            float *P = reinterpret_cast<float *>(tk); /* free after the sort */
            int *ord = ti;
            for (int i = tid; i < ne; i += NT) P[i] = __fmul_rn(Xw[i], inv);
            __syncthreads();
            for (int i = tid; i < ne; i += NT)
                if (P[i] > pT) {
                    int r = 0;
                    for (int j = 0; j < ne; ++j) r += P[j] > P[i] || (P[j] == P[i] && j < i);
                    ord[r] = i;
                }
            __syncthreads();
            if (tid == 0) {
                int nA = 0;
                for (int i = 0; i < ne; ++i) nA += P[i] > pT;
                float cum = 0.0f;
                int cut = -1; /* rows of the first group kept: ranks < cut */
                for (int j = 0; j < nA && cut < 0; ++j) {
                    cum = __fadd_rn(cum, P[ord[j]]);
                    if (cum >= a.top_p) cut = j + 1;
                }
                /* c rows at pT, in row order, complete the nucleus */
                int nE = (int)ties;
                for (int i = 0; i < ne; ++i) nE += P[i] == pT;
                int c = 0;
                if (cut < 0)
                    while (c < nE) {
                        cum = __fadd_rn(cum, pT);
                        ++c;
                        if (cum >= a.top_p) break;
                    }
                ms->sh[0] = (uint32_t)(cut < 0 ? nA : cut);
                ms->sh[1] = (uint32_t)c;
            }
            __syncthreads();
            const int keepA = (int)ms->sh[0], c = (int)ms->sh[1];
            /* the row of the c-th row at pT: a walk counting those rows */
            int cut_row = a.row_base - 1;
            if (c > 0) {
                for (int i = tid; i < ne; i += NT) P[i] = P[i] == pT ? 1.0f : 0.0f;
                __syncthreads();
                const WalkUnit Uc{Xk, Xi, P, ne, 1, a.row_base, rows};
                const WalkResult cw = wide_walk(1, [&](int) { return Uc; }, fill, T, 1.0f, false,
                                                0.0f, VARIANT_LIBRARY, bm, tab, ms, (float)c);
                cut_row = cw.token >= 0 ? cw.token : a.row_base + rows - 1;
                __syncthreads();
                for (int i = tid; i < ne; i += NT) P[i] = __fmul_rn(Xw[i], inv);
                __syncthreads();
            }
            /* the kept rows' terms (the largest stays, so they are unchanged) */
            for (int i = tid; i < ne; i += NT) {
                const bool inA = P[i] > pT;
                int r = 0;
                if (inA)
                    for (int j = 0; j < ne; ++j) r += P[j] > P[i] || (P[j] == P[i] && j < i);
                const bool kept = inA ? r < keepA : (c > 0 && Xi[i] <= cut_row);
                if (!kept) Xw[i] = 0.0f;
            }
            tie_end = c > 0 ? cut_row - a.row_base + 1 : 0;
            __syncthreads();
            dg.n_cand = keepA + c;
        }
        res = wide_walk(1, [&](int) { return U; }, fill, T, wT, false, a.u, a.variant, bm, tab,
                        ms);
        token = res.token >= 0 ? res.token : a.vocab - 1;
        /* gpt2_server.c:2996-3001 walks every row: a draw of exactly 0 stops
         * at row 0 */
        if (a.variant == VARIANT_GPT2 && res.drew && res.r == 0.0f) token = 0;
    }
    if (tid == 0) {
        dg.sum = res.sum;
        dg.r = res.r;
        dg.drew = res.drew;
        dg.token = token;
        if (a.token) *a.token = token;
        if (a.diag) *a.diag = dg;
        if (a.push_history && a.hist_cap > 0) {
            /* runtime/lal_sampling.h:133-136 as a ring: FIFO at hist_cap */
            if (a.hn < a.hist_cap) {
                a.hist_ids[a.hn] = token;
                *a.hist_n = a.hn + 1;
            } else {
                a.hist_ids[a.hhead] = token;
                *a.hist_head = (a.hhead + 1) % a.hist_cap;
            }
        }
        notify_host(a.host_tok, a.host_seq, token);
    }
    __syncthreads();
}

}  // namespace
}  // namespace lal
