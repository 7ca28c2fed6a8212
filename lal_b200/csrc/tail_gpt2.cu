/*
 * tail_gpt2.cu -- the GPT-2 server's LM-head tail (tools/server/gpt2_server.c)
 * as a second drop-in, for contexts created with LAL_SAMPLER_GPT2.
 *
 * One step of one stream is three launches on the context's stream, each a
 * programmatic dependent launch that waits for its predecessor before its
 * first dependent read:
 *   tail_kernel<LMHEAD>    the int8 logits of every row (gpt2_server.c:2013-
 *                          2095: exact int32 dots, scale_x*scale_w[v]*dot),
 *                          x quantized per CTA as lm_head_quantize_x does
 *                          (:1982-1998: scale = max|x|/127 floored at 1e-8,
 *                          xq = clamp((int)(x/scale), +-127), truncation for
 *                          every element); it streams the LM head while the
 *                          previous step's last launch finishes;
 *   gpt2_select_kernel     one CTA of 1024 threads with the V int8 logits in
 *                          shared memory: the rows the server's min-heap of
 *                          RERANK_N = 512 keeps (:2160-2197);
 *   gpt2_rerank_kernel     their float re-score (gpt2_server.c:2203-2212):
 *                          logits[v] = sum over eight lanes of fused
 *                          multiply-adds x[i] * ((float)wq[i] * scale[v]),
 *                          lane j taking i = j (mod 8) in index order, the
 *                          lanes summed left to right (v8f_hsum, :110-113);
 *                          then, in its last CTA, the server's sampler
 *                          (:2862-3013): the repetition penalty in place, the
 *                          k-th largest logit (its k passes of find-max-and-
 *                          mask give the k-th largest with multiplicity), the
 *                          nucleus when 0 < top_p < 1, the softmax over the
 *                          kept rows summed in ascending vocab order, r = u *
 *                          sum with u = (rand() % 1000000) / 1e6f drawn by the
 *                          caller, the first v whose running sum reaches r
 *                          (v = 0 when r == 0: the server's running sum also
 *                          walks the rows below T, adding zeros); argmax
 *                          without the penalty when temperature <= 0 or
 *                          top_k <= 0.  The candidates lie among the 512
 *                          re-scored rows whenever k of them beat every row
 *                          the heap left out (gpt2_finish below); otherwise
 *                          the wide path (tail_wide.cuh) runs over the whole
 *                          vocabulary.
 *
 * Which rows the heap keeps.  Every row above the RERANK_N-th largest int8
 * logit T is kept.  When more rows than places tie at T, the rows kept among
 * them depend on the heap's history: the select kernel then replays the
 * server's heap exactly (one thread over the keys in shared memory, index
 * order) -- a slow path that only exact logit ties at the boundary take.
 */
#include "tail_device.cuh"
#include "tail_wide.cuh"

#include <algorithm>
#include <cstring>

namespace lal {
namespace {

constexpr int kRerankWarps = 8;          /* warps of a CTA that re-score rows   */
constexpr int kRerankRows = 32;          /* rows a CTA of the re-score kernel   */
constexpr int kGpt2SelCap = 2048;        /* keys gathered above the bound L     */

/* The 512 rows the server's min-heap keeps (gpt2_server.c:2160-2197), from
 * the int8 logits of all V rows held as order keys in one CTA's shared memory
 * (V <= kGpt2MaxV; one bulk copy brings them in): a lower bound L of T, the
 * N-th largest key with multiplicity, from the maxima of 1024 groups of rows;
 * the few keys >= L gathered; T by a radix select among them (among all keys
 * when more than kGpt2SelCap reach L).  When exactly N rows
 * reach T they are the heap's rows, listed in any order; otherwise rows tie
 * at T across the boundary and thread 0 replays the heap's pushes and root
 * replacements over the keys in index order (keys compare as the floats do:
 * -0 and +0 share one).  Writes the rows to cand_out, their count to *n_out
 * and T to *bound_out: every row left out has a logit <= T. */
__global__ void __launch_bounds__(kGpt2SelThreads, 1)
    gpt2_select_kernel(const float *logits, int V, int N, int *cand_out, int *n_out,
                       uint32_t *bound_out, int *status) {
    extern __shared__ __align__(16) uint32_t keys[];
    __shared__ __align__(16) uint32_t gat[2 * kGpt2SelCap]; /* the gathered keys, then rows */
    __shared__ __align__(16) uint32_t aux[2 * kGpt2RerankN]; /* refinement bins, or the heap */
    __shared__ uint32_t sh[4];
    __shared__ int cnt;
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag, never;
    __shared__ int wsum[kGpt2SelThreads / 32];
    uint32_t *heap_key = aux;
    int *heap_idx = reinterpret_cast<int *>(aux + kGpt2RerankN);
    static_assert(2 * kGpt2RerankN >= 1024, "refinement bins");
    /* programmatic dependent launch: the LM head's logits are complete and
     * visible after the wait; the re-score launch may then be scheduled */
    grid_dep_wait();
    grid_dep_launch_dependents();
    if (*status != 0) return; /* the LM head failed: the step reports it */
    const int tid = threadIdx.x, lane = tid & 31;
    /* the logits into shared memory: one bulk copy of the 16-byte multiple,
     * plain loads for the rest */
    const bool al16 = (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
    const int nb16 = al16 ? V * 4 / 16 * 16 : 0;
    if (tid == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
        abort_flag = 0;
        never = 0;
    }
    __syncthreads();
    if (tid == 0 && nb16 > 0) {
        mbar_expect_tx(&bar, (uint32_t)nb16);
        bulk_g2s(keys, logits, (uint32_t)nb16, &bar, policy_evict_first());
    }
    for (int i = nb16 / 4 + tid; i < V; i += kGpt2SelThreads)
        keys[i] = __float_as_uint(__ldcg(logits + i));
    if (nb16 > 0 && !mbar_wait(&bar, 0u, &abort_flag)) {
        /* the copy is still in flight: wait for it on time alone, then fail */
        mbar_wait(&bar, 0u, &never);
        if (tid == 0) atomicCAS(status, 0, (int)DEV_TIMEOUT);
        return;
    }
    __syncthreads();
    /* The N-th largest of a multiset of keys that the threads hold (each
     * thread's each(f) calls f(key) for its keys; 1 <= krem <= the count): an
     * MSB-first radix select, 8-bit digits counted in aux. */
    auto kth_largest = [&](auto each, uint32_t krem, int top_shift) {
        uint32_t prefix = 0u, mask = 0u;
        for (int shift = top_shift; shift >= 0; shift -= 8) {
            if (tid < 256) aux[tid] = 0u;
            __syncthreads();
            each([&](uint32_t key) {
                if ((key & mask) == prefix) atomicAdd(&aux[(key >> shift) & 0xFFu], 1u);
            });
            __syncthreads();
            if (tid < 32) {
                /* from the top: lane l holds digits 255-8l .. 248-8l */
                uint32_t c[8], sum = 0u;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c[j] = aux[255 - 8 * lane - j];
                    sum += c[j];
                }
                uint32_t incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                const uint32_t excl = incl - sum;
                if (excl < krem && krem <= incl) {
                    uint32_t run = excl;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (run < krem && run + c[j] >= krem) {
                            sh[0] = 255u - 8u * (uint32_t)lane - (uint32_t)j;
                            sh[1] = run;
                        }
                        run += c[j];
                    }
                }
            }
            __syncthreads();
            prefix |= sh[0] << shift;
            mask |= 0xFFu << shift;
            krem -= sh[1];
            __syncthreads();
        }
        return prefix;
    };
    /* the rows with key >= T, listed when there are exactly N of them */
    auto list_if_n = [&](auto key_of, auto row_of, int count, uint32_t T) {
        int c = 0;
        for (int e = tid; e < count; e += kGpt2SelThreads) c += key_of(e) >= T;
        if (tid == 0) cnt = 0;
        __syncthreads();
        c = __reduce_add_sync(0xffffffffu, c);
        if (lane == 0 && c) atomicAdd(&cnt, c);
        __syncthreads();
        const int mt = cnt;
        __syncthreads();
        if (mt != N) return false;
        if (tid == 0) cnt = 0;
        __syncthreads();
        const int cr = (count + kGpt2SelThreads - 1) / kGpt2SelThreads * kGpt2SelThreads;
        for (int e = tid; e < cr; e += kGpt2SelThreads) {
            const bool take = e < count && key_of(e) >= T;
            const unsigned bal = __ballot_sync(0xffffffffu, take);
            if (bal) {
                int base = 0;
                if (lane == 0) base = atomicAdd(&cnt, __popc(bal));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (take) cand_out[base + __popc(bal & ((1u << lane) - 1u))] = row_of(e);
            }
        }
        if (tid == 0) {
            *n_out = N;
            *bound_out = T;
        }
        return true;
    };
    /* order keys in place; thread t's keys t, t + 1024, ... form a group
     * whose largest key it keeps */
    uint32_t gmx = 0u;
    {
        constexpr int U = 4; /* independent shared-memory round trips in flight */
        for (int i0 = tid; i0 < V; i0 += U * kGpt2SelThreads) {
            uint32_t v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * kGpt2SelThreads;
                v[u] = i < V ? keys[i] : 0u;
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * kGpt2SelThreads;
                if (i < V) {
                    const uint32_t key = f2key(__uint_as_float(v[u]));
                    keys[i] = key;
                    gmx = max(gmx, key);
                }
            }
        }
    }
    __syncthreads();
    /* L, the lower edge of the 12-bit bin holding the N-th largest group
     * maximum (empty groups count 0): N distinct rows reach L, so T >= L and
     * every row at or above T has a key >= L -- few rows, gathered in one
     * pass.  One histogram pass (in the gather area, free until then). */
    for (int i = tid; i < 4096; i += kGpt2SelThreads) gat[i] = 0u;
    if (tid == 0) sh[3] = 0u;
    __syncthreads();
    atomicAdd(&gat[gmx >> 20], 1u);
    {
        const uint32_t wm = __reduce_max_sync(0xffffffffu, gmx);
        if (lane == 0) atomicMax(&sh[3], wm);
    }
    __syncthreads();
    if (tid < 32) {
        const uint32_t b = warp_boundary_bin_4096(gat, sh[3] >> 20, (uint32_t)N);
        if (lane == 0) sh[2] = b;
    }
    __syncthreads();
    const uint32_t L = sh[2] << 20, top_key = sh[3];
    __syncthreads();
    /* the keys >= L: counted per thread, placed by a block scan (thread
     * order, then row order within a thread) */
    uint32_t *ck = gat;
    int *ci = reinterpret_cast<int *>(gat + kGpt2SelCap);
    int mine = 0;
    for (int i = tid; i < V; i += kGpt2SelThreads) mine += keys[i] >= L;
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) wsum[tid >> 5] = incl;
    __syncthreads();
    if (tid < 32) {
        const int w = wsum[lane];
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        wsum[lane] = wi - w;
        if (lane == 31) cnt = wi;
    }
    __syncthreads();
    int pos = wsum[tid >> 5] + incl - mine;
    if (mine > 0)
        for (int i = tid; i < V; i += kGpt2SelThreads)
            if (keys[i] >= L) {
                if (pos < kGpt2SelCap) {
                    ck[pos] = keys[i];
                    ci[pos] = i;
                }
                ++pos;
            }
    __syncthreads();
    const int na = cnt;
    uint32_t T;
    if (na <= kGpt2SelCap) {
        /* every gathered key lies in [L, top_key]: the digits above the
         * first byte where the two differ are known */
        const uint32_t diff = L ^ top_key;
        const int top_shift = diff == 0u ? 0 : (31 - __clz(diff)) / 8 * 8;
        T = kth_largest(
            [&](auto f) {
                for (int e = tid; e < na; e += kGpt2SelThreads) f(ck[e]);
            },
            (uint32_t)N, top_shift);
        T |= L & (top_shift >= 24 ? 0u : 0xFFFFFFFFu << (top_shift + 8));
        if (list_if_n([&](int e) { return ck[e]; }, [&](int e) { return ci[e]; }, na, T)) return;
    } else {
        /* a crowded boundary: the radix select over all keys */
        T = kth_largest(
            [&](auto f) {
                for (int i = tid; i < V; i += kGpt2SelThreads) f(keys[i]);
            },
            (uint32_t)N, 24);
        if (list_if_n([&](int i) { return keys[i]; }, [&](int i) { return i; }, V, T)) return;
    }
    __syncthreads(); /* the refinement bins are read before the heap reuses them */
    /* more rows than places tie at T: the server's heap (gpt2_server.c:
     * 2167-2197) replayed over the keys in index order (keys compare as the
     * floats do: -0 and +0 share one) */
    if (tid == 0) {
        int hn = 0;
        for (int v = 0; v < V; ++v) {
            const uint32_t val = keys[v];
            if (hn < N) {
                int ch = hn++;
                heap_key[ch] = val;
                heap_idx[ch] = v;
                while (ch > 0) {
                    const int pa = (ch - 1) >> 1;
                    if (heap_key[pa] <= heap_key[ch]) break;
                    const uint32_t tk = heap_key[pa];
                    heap_key[pa] = heap_key[ch];
                    heap_key[ch] = tk;
                    const int ti = heap_idx[pa];
                    heap_idx[pa] = heap_idx[ch];
                    heap_idx[ch] = ti;
                    ch = pa;
                }
            } else if (val > heap_key[0]) {
                heap_key[0] = val;
                heap_idx[0] = v;
                int pa = 0;
                for (;;) {
                    const int l = 2 * pa + 1, r = 2 * pa + 2;
                    int sm = pa;
                    if (l < hn && heap_key[l] < heap_key[sm]) sm = l;
                    if (r < hn && heap_key[r] < heap_key[sm]) sm = r;
                    if (sm == pa) break;
                    const uint32_t tk = heap_key[pa];
                    heap_key[pa] = heap_key[sm];
                    heap_key[sm] = tk;
                    const int ti = heap_idx[pa];
                    heap_idx[pa] = heap_idx[sm];
                    heap_idx[sm] = ti;
                    pa = sm;
                }
            }
        }
        for (int j = 0; j < hn; ++j) cand_out[j] = heap_idx[j];
        *n_out = hn;
        *bound_out = T;
    }
}

/* k-th largest (with multiplicity) of the keys the block's threads hold --
 * each thread's each(f) calls f(key) for its keys; 1 <= krem <= their count
 * -- by an MSB-first radix select of 8-bit digits with plain shared-memory
 * counters (a few hundred keys: little contention), from the digit at
 * top_shift down: the caller passes keys whose bits above it are all equal,
 * and the result holds only the bits from top_shift + 7 down. */
template <class Each>
__device__ uint32_t kth_largest_small(Each each, uint32_t krem, int top_shift, Misc *ms) {
    const int tid = threadIdx.x, lane = tid & 31;
    uint32_t prefix = 0u, mask = 0u;
    for (int shift = top_shift; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += NT) ms->hist[i] = 0u;
        __syncthreads();
        each([&](uint32_t key) {
            if ((key & mask) == prefix) atomicAdd(&ms->hist[(key >> shift) & 0xFFu], 1u);
        });
        __syncthreads();
        if (tid < 32) {
            uint32_t c[8], sum = 0u;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = ms->hist[255 - 8 * lane - j];
                sum += c[j];
            }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t excl = incl - sum;
            if (excl < krem && krem <= incl) {
                uint32_t run = excl;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (run < krem && run + c[j] >= krem) {
                        ms->sh[0] = 255u - 8u * (uint32_t)lane - (uint32_t)j;
                        ms->sh[1] = run;
                    }
                    run += c[j];
                }
            }
        }
        __syncthreads();
        prefix |= ms->sh[0] << shift;
        mask |= 0xFFu << shift;
        krem -= ms->sh[1];
        __syncthreads();
    }
    return prefix;
}

constexpr uint32_t kHashEmpty = 0xFFFFFFFFu;
constexpr int kFinishPer = (kGpt2RerankN + NT - 1) / NT; /* kept rows a thread holds */

/* shared memory of the sampler below: the kept rows and their logits, the
 * history hash, the candidates and the nucleus scratch (kGpt2RerankN entries
 * each), or the wide path's area */
__host__ __device__ constexpr size_t gpt2_finish_bytes(int cap, int h_slots) {
    return (size_t)8 * kGpt2RerankN + (size_t)8 * h_slots + (size_t)24 * kGpt2RerankN >
                   (size_t)wide_area_bytes(cap)
               ? (size_t)8 * kGpt2RerankN + (size_t)8 * h_slots + (size_t)24 * kGpt2RerankN
               : (size_t)wide_area_bytes(cap);
}

/* The nucleus marks of a pool the wide path exported (the filter hook's
 * first half): every row kept without top-p; with it, the pool's weights over
 * its largest value and gpt2_nucleus, for a pool of at most kGpt2RerankN rows
 * (a larger one -- ties across most of the vocabulary -- reports
 * DEV_CAPACITY). */
__device__ __noinline__ void gpt2_pool_nucleus(const Gpt2Finish &f, uint8_t *smem, Misc *ms) {
    const int tid = threadIdx.x;
    __syncthreads();
    const int m = min(f.diag->n_cand, f.pool_cap);
    const bool nucleus = f.top_p > 0.0f && f.top_p < 1.0f;
    if (!nucleus) {
        for (int i = tid; i < m; i += NT) f.pool_keep[i] = 1;
        return;
    }
    if (m > kGpt2RerankN) {
        if (tid == 0) atomicCAS(f.status, 0, (int)DEV_CAPACITY);
        return;
    }
    float *Ce = reinterpret_cast<float *>(smem);
    float *P = Ce + kGpt2RerankN, *Q = P + kGpt2RerankN;
    int *R = reinterpret_cast<int *>(Q + kGpt2RerankN);
    float mx = -1e30f;
    for (int i = tid; i < m; i += NT) mx = fmaxf(mx, __ldcg(f.pool_val + i));
    const float max_l = block_max_f(mx, ms);
    const ExpfTables ex{f.expf_x, f.expf_y, f.expf_bits, f.expf_off, f.expf_hash,
                        f.expf_hash_probe};
    const float temp = f.temperature[0];
    for (int i = tid; i < m; i += NT) Ce[i] = ex.weight(__ldcg(f.pool_val + i), max_l, temp);
    __syncthreads();
    const int n_keep = gpt2_nucleus(f.top_p, m, Ce, P, R, Q, ms);
    for (int i = tid; i < m; i += NT) f.pool_keep[i] = R[i] < n_keep ? 1 : 0;
}

/* The server's sampler (gpt2_server.c:2862-3013) after the re-score, by one
 * CTA.  Every row the heap left out has an int8 logit <= the bound B (the
 * heap kept every row above it), and the repetition penalty never raises a
 * logit.  So when k of the kept rows' penalised logits lie above B, the k-th
 * largest logit T of the vocabulary lies above every left-out row: the
 * candidates {l >= T} are kept rows only, and the select, softmax and draw
 * run over the 512 kept rows.  Greedy likewise when the kept rows' largest
 * raw logit is above B.  Any other step takes the wide path over the whole
 * vocabulary (penalised in global memory first).  The penalised logits of
 * every history row are written back, as the server's in-place penalty
 * leaves them. */
__device__ __noinline__ void gpt2_finish(const Gpt2Finish &f, uint8_t *smem, Misc *ms) {
    const int tid = threadIdx.x;
    const int V = f.V;
    const int n = min(__ldcg(f.n_ptr), kGpt2RerankN);
    const bool all_rows = n >= V;
    const uint32_t B = __ldcg(f.bound);
    const float temp = f.temperature[0], pen = f.rep_penalty[0], u0 = f.u[0];
    const int topk = f.top_k[0];
    const int hn = f.hist_n ? f.hist_n[0] : 0, hhead = f.hist_head ? f.hist_head[0] : 0;
    const bool greedy = temp <= 0.0f || topk <= 0;
    const int k = greedy ? 1 : min(topk, V);
    const bool use_pen = !greedy && pen > 1.0f && hn > 0;
    const ExpfTables ex{f.expf_x, f.expf_y, f.expf_bits, f.expf_off, f.expf_hash,
                        f.expf_hash_probe};
    float *Rv = reinterpret_cast<float *>(smem);
    int *Ri = reinterpret_cast<int *>(Rv + kGpt2RerankN);
    uint32_t *hkey = reinterpret_cast<uint32_t *>(Ri + kGpt2RerankN);
    uint32_t *hcnt = hkey + f.h_slots;
    float *Ov = reinterpret_cast<float *>(hcnt + f.h_slots);
    int *Oi = reinterpret_cast<int *>(Ov + kGpt2RerankN);
    float *Ce = reinterpret_cast<float *>(Oi + kGpt2RerankN);
    float *P = Ce + kGpt2RerankN;
    int *Rk = reinterpret_cast<int *>(P + kGpt2RerankN);
    float *Q = reinterpret_cast<float *>(Rk + kGpt2RerankN);

    /* 1. the kept rows and their re-scored logits (written in list order by
     * the re-score), the history ids and the history rows' logits: every
     * load goes out before any is used */
    const uint32_t mask = (uint32_t)f.h_slots - 1u;
    if (use_pen)
        for (int i = tid; i < f.h_slots; i += NT) {
            hkey[i] = kHashEmpty;
            hcnt[i] = 0u;
        }
    constexpr int kHReg = 4;
    int hid[kHReg];
#pragma unroll
    for (int q = 0; q < kHReg; ++q) {
        const int i = tid + q * NT;
        hid[q] = use_pen && i < hn ? __ldcg(f.hist_ids + i) : -1;
    }
#pragma unroll
    for (int q = 0; q < kFinishPer; ++q) {
        const int j = tid + q * NT;
        if (j < n) {
            Ri[j] = __ldcg(f.cand + j);
            Rv[j] = __ldcg(f.kept_val + j);
        }
    }
    float hl[kHReg];
#pragma unroll
    for (int q = 0; q < kHReg; ++q)
        hl[q] = hid[q] >= 0 && hid[q] < V ? __ldcg(f.logits + hid[q]) : 0.0f;
    /* 2. the penalty (gpt2_server.c:2868-2876): each history id in [0, V)
     * once per occurrence, on the vocabulary's logits and on the kept copies;
     * the thread that inserts an id first writes its row back */
    if (use_pen) {
        __syncthreads();
        auto insert = [&](int id) {
            if (id < 0 || id >= V) return false;
            uint32_t slot = ((uint32_t)id * 2654435761u) & mask;
            for (int probe = 0; probe < f.h_slots; ++probe) {
                const uint32_t prev = atomicCAS(&hkey[slot], kHashEmpty, (uint32_t)id);
                if (prev == kHashEmpty || prev == (uint32_t)id) {
                    atomicAdd(&hcnt[slot], 1u);
                    return prev == kHashEmpty;
                }
                slot = (slot + 1u) & mask;
            }
            return false;
        };
        auto count_of = [&](uint32_t id) {
            uint32_t slot = (id * 2654435761u) & mask;
            for (int probe = 0; probe < f.h_slots; ++probe) {
                const uint32_t kk = hkey[slot];
                if (kk == id) return hcnt[slot];
                if (kk == kHashEmpty) break;
                slot = (slot + 1u) & mask;
            }
            return 0u;
        };
        bool owner[kHReg];
#pragma unroll
        for (int q = 0; q < kHReg; ++q) owner[q] = insert(hid[q]);
        for (int i = tid + kHReg * NT; i < hn; i += NT) insert(__ldcg(f.hist_ids + i));
        __syncthreads();
        if (hn <= kHReg * NT) {
#pragma unroll
            for (int q = 0; q < kHReg; ++q)
                if (owner[q]) f.logits[hid[q]] = penalise(hl[q], count_of((uint32_t)hid[q]), pen);
        } else {
            /* a history past the registers' reach: every distinct id's row
             * with a load of its own */
            for (int i = tid; i < f.h_slots; i += NT) {
                const uint32_t id = hkey[i];
                if (id != kHashEmpty) f.logits[id] = penalise(__ldcg(f.logits + id), hcnt[i], pen);
            }
        }
        for (int j = tid; j < n; j += NT) {
            const uint32_t id = (uint32_t)Ri[j];
            uint32_t slot = (id * 2654435761u) & mask;
            for (int probe = 0; probe < f.h_slots; ++probe) {
                const uint32_t kk = hkey[slot];
                if (kk == id) {
                    Rv[j] = penalise(Rv[j], hcnt[slot], pen);
                    break;
                }
                if (kk == kHashEmpty) break;
                slot = (slot + 1u) & mask;
            }
        }
    }
    __syncthreads();
    /* 3. do the kept rows hold the step? */
    float rv[kFinishPer];
    uint32_t top = 0u, above = 0u;
#pragma unroll
    for (int q = 0; q < kFinishPer; ++q) {
        const int j = tid + q * NT;
        rv[q] = j < n ? Rv[j] : 0.0f;
        if (j < n) {
            const uint32_t key = f2key(rv[q]);
            top = max(top, key);
            above += key > B;
        }
    }
    top = block_max_u32(top, ms);
    uint32_t n_above;
    block_scan_excl(above, ms, &n_above);
    const bool fast = all_rows || (greedy ? top > B : (int)n_above >= k);
    if (!fast) {
        WideDense a = {};
        a.lg = f.logits;
        a.rows = V;
        a.row_base = 0;
        a.vocab = V;
        a.k = k;
        a.variant = VARIANT_GPT2;
        a.greedy = greedy ? 1 : 0;
        a.temp = temp;
        a.u = u0;
        a.cap = max(1, f.cap);
        a.ex = ex;
        a.token = f.tokens;
        a.diag = f.diag;
        a.hist_ids = f.hist_ids;
        a.hist_n = f.hist_n;
        a.hist_head = f.hist_head;
        a.hist_cap = f.hist_cap;
        a.push_history = f.push_history;
        a.hn = hn;
        a.hhead = hhead;
        a.top_p = f.top_p;
        if (f.candidates_only) {
            a.candidates_only = 1;
            a.cand_val = f.pool_val;
            a.cand_idx = f.pool_idx;
            a.cand_cap = f.pool_cap;
        }
        __syncthreads();
        wide_dense(a, smem, ms);
        if (f.candidates_only) gpt2_pool_nucleus(f, smem, ms);
        return;
    }
    StreamDiag dg;
    dg.max_l = 0.0f;
    dg.sum = 0.0f;
    dg.r = 0.0f;
    dg.greedy = greedy ? 1 : 0;
    dg.drew = 0;
    int token;
    if (greedy) {
        /* argmax without the penalty, the lowest row among equals */
        int first = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < kFinishPer; ++q) {
            const int j = tid + q * NT;
            if (j < n && f2key(rv[q]) == top) first = min(first, Ri[j]);
        }
        token = (int)block_min_u32((uint32_t)first, ms);
        dg.threshold = key2f(top);
        dg.n_cand = 1;
    } else {
        /* the weights' table loads go out now (every candidate's weight is
         * expf((l - max_l) / temp) with max_l the largest kept logit) and land
         * while T is selected */
        const float max_l = fmaxf(-1e30f, key2f(top));
        float xw[kFinishPer], yr[kFinishPer];
        uint4 hp[kFinishPer];
#pragma unroll
        for (int q = 0; q < kFinishPer; ++q) {
            xw[q] = __fdiv_rn(__fsub_rn(rv[q], max_l), temp);
            if (f.expf_hash) {
                hp[q] = expf_hash_load(xw[q], f.expf_hash);
                yr[q] = lal_expf_rounded(xw[q]);
            }
        }
        /* 4. T, the k-th largest of the kept rows' logits with multiplicity
         * (the server's k passes of find-max-and-mask) */
        /* Unless every row was kept, T > B: only the keys above B take part
         * (at least k of them), and their digits above the first byte where
         * B + 1 and the largest key differ are known. */
        const uint32_t lo = all_rows ? 0u : B + 1u;
        const uint32_t diff = lo ^ top;
        const int top_shift = diff == 0u ? 0 : (31 - __clz(diff)) / 8 * 8;
        uint32_t T = kth_largest_small(
            [&](auto add) {
#pragma unroll
                for (int q = 0; q < kFinishPer; ++q) {
                    const uint32_t key = f2key(rv[q]);
                    if (tid + q * NT < n && key >= lo) add(key);
                }
            },
            (uint32_t)k, top_shift, ms);
        T |= top & (top_shift >= 24 ? 0u : 0xFFFFFFFFu << (top_shift + 8));
        /* the candidates {l >= T} with their weights: listed (Rk, Q, P),
         * then placed in ascending row order by their rank among themselves */
        int *Ci = Rk;
        float *Cv = Q, *Cw = P;
        uint32_t c = 0u;
#pragma unroll
        for (int q = 0; q < kFinishPer; ++q) c += tid + q * NT < n && f2key(rv[q]) >= T;
        uint32_t mt;
        uint32_t pos = block_scan_excl(c, ms, &mt);
#pragma unroll
        for (int q = 0; q < kFinishPer; ++q) {
            const int j = tid + q * NT;
            if (j < n && f2key(rv[q]) >= T) {
                Ci[pos] = Ri[j];
                Cv[pos] = rv[q];
                Cw[pos] = f.expf_hash ? expf_hash_resolve(xw[q], yr[q], hp[q], f.expf_hash,
                                                          f.expf_hash_probe)
                                      : sampler_expf(xw[q], f.expf_x, f.expf_y, f.expf_bits,
                                                     f.expf_off);
                ++pos;
            }
        }
        __syncthreads();
        const int m = (int)mt;
        for (int i = tid; i < m; i += NT) {
            const int me = Ci[i];
            int r = 0;
            for (int j = 0; j < m; ++j) r += Ci[j] < me;
            Oi[r] = me;
            Ov[r] = Cv[i];
            Ce[r] = Cw[i];
        }
        __syncthreads();
        int n_cand = m;
        const bool nucleus = f.top_p > 0.0f && f.top_p < 1.0f;
        if (nucleus) n_cand = gpt2_nucleus(f.top_p, m, Ce, P, Rk, Q, ms);
        if (f.candidates_only) {
            /* the filter hook's pool: every candidate, the nucleus's mark */
            for (int i = tid; i < m && i < f.pool_cap; i += NT) {
                f.pool_val[i] = Ov[i];
                f.pool_idx[i] = Oi[i];
                f.pool_keep[i] = !nucleus || Rk[i] < n_cand ? 1 : 0;
            }
            if (tid == 0) {
                dg.threshold = key2f(T);
                dg.max_l = max_l;
                dg.n_cand = m;
                dg.token = -1;
                *f.diag = dg;
            }
            return;
        }
        if (tid == 0) {
            float acc = 0.0f;
            for (int i = 0; i < m; ++i) {
                acc = __fadd_rn(acc, Ce[i]);
                Ce[i] = acc;
            }
            ms->sum = acc;
            ms->found = 0x7fffffff;
        }
        __syncthreads();
        const float sum = ms->sum;
        /* the draw (gpt2_server.c:2995-3002): the first row whose running sum
         * reaches r = u * sum; a draw of exactly 0 stops at row 0 */
        const float r = __fmul_rn(u0, sum);
        int first = 0x7fffffff;
        for (int i = tid; i < m; i += NT)
            if (r <= Ce[i]) {
                first = i;
                break;
            }
        if (first != 0x7fffffff) atomicMin(&ms->found, first);
        __syncthreads();
        token = ms->found != 0x7fffffff ? Oi[ms->found] : V - 1;
        if (r == 0.0f) token = 0;
        dg.threshold = key2f(T);
        dg.max_l = max_l;
        dg.sum = sum;
        dg.r = r;
        dg.drew = 1;
        dg.n_cand = n_cand;
    }
    if (tid == 0) {
        dg.token = token;
        *f.tokens = token;
        *f.diag = dg;
        if (f.push_history && f.hist_cap > 0) {
            /* runtime/lal_sampling.h:133-136 as a ring: FIFO at hist_cap */
            if (hn < f.hist_cap) {
                f.hist_ids[hn] = token;
                *f.hist_n = hn + 1;
            } else {
                f.hist_ids[hhead] = token;
                *f.hist_head = (hhead + 1) % f.hist_cap;
            }
        }
    }
}

/* The float re-score (gpt2_server.c:2203-2211) of up to kRerankRows listed
 * rows a CTA: x and the rows are staged into shared memory with 16-byte
 * asynchronous copies, then eight lanes a row sum x[i] * ((float)wq[i] *
 * scale) as fused multiply-adds, lane j over i = j (mod 8) in index order,
 * and add the lanes left to right (v8f_hsum, :110-113).  The last CTA to
 * finish (an acquire-release ticket) runs the sampler. */
__global__ void __launch_bounds__(NT)
    gpt2_rerank_kernel(const float *x, int d, const int8_t *W, int ld, const float *sw,
                       const __grid_constant__ Gpt2Finish f) {
    extern __shared__ __align__(16) uint8_t rsm[];
    __shared__ Misc msh;
    /* programmatic dependent launch: the select's rows are complete and
     * visible after the wait; the next step's LM head may then be scheduled
     * (it streams the LM head, and waits for this launch before it writes) */
    grid_dep_wait();
    grid_dep_launch_dependents();
    if (*f.status != 0) return; /* the LM head failed: the step reports it */
    const int n = *f.n_ptr;
    const int j0 = blockIdx.x * kRerankRows;
    const int rn = max(0, min(kRerankRows, n - j0));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (rn > 0) {
        uint8_t *rows = rsm;
        float *xs = reinterpret_cast<float *>(rsm + (size_t)kRerankRows * ld);
        if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
            for (int e = tid; e < d / 4; e += blockDim.x) cp_async16(xs + 4 * e, x + 4 * e);
        } else {
            for (int i = tid; i < d; i += blockDim.x) xs[i] = x[i];
        }
        const int rp = ld / 16;
        for (int e = tid; e < rn * rp; e += blockDim.x) {
            const int r = e / rp, q = e - r * rp;
            cp_async16(rows + (size_t)r * ld + 16 * q, W + (size_t)f.cand[j0 + r] * ld + 16 * q);
        }
        cp_async_wait_all();
        __syncthreads();
        const int sub = lane >> 3, lane8 = lane & 7;
        for (int r0 = warp * 4; warp < kRerankWarps && r0 < rn; r0 += kRerankWarps * 4) {
            const int r = r0 + sub;
            const bool on = r < rn;
            const int8_t *wr = reinterpret_cast<const int8_t *>(rows + (size_t)(on ? r : 0) * ld);
            const int v = on ? f.cand[j0 + r] : 0;
            const float scale = on ? sw[v] : 0.0f;
            float acc = 0.0f;
#pragma unroll 4
            for (int i = lane8; i < d; i += 8)
                acc = __fmaf_rn(xs[i], __fmul_rn((float)wr[i], scale), acc);
            const int base = lane & ~7;
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float t = __shfl_sync(0xffffffffu, acc, base + j);
                s = j == 0 ? t : __fadd_rn(s, t);
            }
            if (on && lane8 == 0) {
                f.logits[v] = s;
                f.kept_val[j0 + r] = s; /* list order, for the sampler */
            }
        }
    }
    /* the barrier orders this CTA's logit writes before thread 0's
     * acquire-release ticket; in the last CTA the same atomic acquires every
     * other CTA's writes */
    __syncthreads();
    if (tid == 0) msh.ticket = (int)atom_add_acq_rel_gpu(f.ticket, 1u);
    __syncthreads();
    if (msh.ticket != (int)gridDim.x - 1) return;
    if (tid == 0) *f.ticket = 0u; /* for the next launch */
    gpt2_finish(f, rsm, &msh);
}

/* a launch that may begin while the previous kernel on the stream runs
 * (the kernel waits for it before its first dependent read) */
cudaError_t launch_dependent_gpt2(const void *fn, int grid, int block, size_t smem,
                                  cudaStream_t st, void **args) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_gpt2_select(const float *logits, int V, int N, int *cand_out, int *n_out,
                               uint32_t *bound_out, int *status, cudaStream_t st) {
    const int bytes = 4 * V;
    cudaError_t e = raise_smem((const void *)gpt2_select_kernel, bytes);
    if (e != cudaSuccess) return e;
    void *args[] = {const_cast<float **>(&logits), &V, &N, &cand_out, &n_out, &bound_out, &status};
    return launch_dependent_gpt2((const void *)gpt2_select_kernel, 1, kGpt2SelThreads,
                                 (size_t)bytes, st, args);
}

size_t gpt2_finish_smem(int cap, int h_slots) { return gpt2_finish_bytes(cap, h_slots); }

cudaError_t launch_gpt2_rerank(const float *x, int d, const int8_t *W, int ld, const float *sw,
                               const Gpt2Finish &f, int N, cudaStream_t st) {
    const size_t bytes = std::max((size_t)kRerankRows * ld + 4 * (size_t)d,
                                  gpt2_finish_bytes(f.cap, f.h_slots));
    cudaError_t e = raise_smem((const void *)gpt2_rerank_kernel, (int)bytes);
    if (e != cudaSuccess) return e;
    const int grid = std::max(1, (N + kRerankRows - 1) / kRerankRows);
    /* NT threads: the sampler's block-wide helpers span the whole block */
    void *args[] = {const_cast<float **>(&x), &d, const_cast<int8_t **>(&W), &ld,
                    const_cast<float **>(&sw), const_cast<Gpt2Finish *>(&f)};
    return launch_dependent_gpt2((const void *)gpt2_rerank_kernel, grid, NT, bytes, st, args);
}

}  // namespace lal
