/*
 * tail_gpt2.cu -- the GPT-2 server's LM-head tail (tools/server/gpt2_server.c)
 * as a second drop-in, for contexts created with LAL_SAMPLER_GPT2.
 *
 * One step of one stream is five launches on the context's stream:
 *   gpt2_quantize_kernel   lm_head_quantize_x (gpt2_server.c:1982-1998): the
 *                          max of |x|, scale = max/127 floored at 1e-8,
 *                          inv = 1/scale, xq = clamp((int)(x*inv), +-127) --
 *                          truncation for every element;
 *   tail_kernel<LMHEAD>    the int8 logits of every row (gpt2_server.c:2013-
 *                          2095: exact int32 dots, scale_x*scale_w[v]*dot);
 *   gpt2_select_kernel     one CTA of 1024 threads with the V int8 logits in
 *                          shared memory: the rows the server's min-heap of
 *                          RERANK_N = 512 keeps (:2160-2197);
 *   gpt2_rerank_kernel     their float re-score (gpt2_server.c:2203-2212):
 *                          logits[v] = sum over eight lanes of fused
 *                          multiply-adds x[i] * ((float)wq[i] * scale[v]),
 *                          lane j taking i = j (mod 8) in index order, the
 *                          lanes summed left to right (v8f_hsum, :110-113);
 *   tail_kernel<SAMPLE>    the server's sampler (gpt2_server.c:2862-3013 with
 *                          top-p off): the repetition penalty in place, the
 *                          k-th largest logit (its k passes of find-max-and-
 *                          mask give the k-th largest with multiplicity), the
 *                          softmax over {l >= T} summed in ascending vocab
 *                          order, r = u * sum with u = (rand() % 1000000) /
 *                          1e6f drawn by the caller, the first v whose
 *                          running sum reaches r (v = 0 when r == 0: the
 *                          server's running sum also walks the rows below T,
 *                          adding zeros); argmax without the penalty when
 *                          temperature <= 0 or top_k <= 0.
 *
 * Which rows the heap keeps.  Every row above the RERANK_N-th largest int8
 * logit T is kept.  When more rows than places tie at T, the rows kept among
 * them depend on the heap's history: the select kernel then replays the
 * server's heap exactly (one thread over the keys in shared memory, index
 * order) -- a slow path that only exact logit ties at the boundary take.
 */
#include "tail_device.cuh"

namespace lal {
namespace {

constexpr int kRerankWarps = 8;          /* warps a CTA of the re-score kernel  */
constexpr int kRerankRows = 32;          /* rows a CTA of the re-score kernel   */
constexpr int kGpt2SelCap = 2048;        /* keys gathered above the bin's edge  */

/* gpt2_server.c:1982-1998 */
__global__ void __launch_bounds__(NT) gpt2_quantize_kernel(const float *x, int d, int8_t *xq,
                                                           int ld, float *scale_out) {
    __shared__ Misc ms;
    float m = 0.0f;
    /* the server keeps the larger of max_abs and |x[i]| with '>': the same
     * value as fmaxf (NaN never wins either) */
    for (int i = threadIdx.x; i < d; i += NT) m = fmaxf(m, fabsf(x[i]));
    m = block_max_f(m, &ms);
    float scale = __fdiv_rn(m, 127.0f);
    if (scale < 1e-8f) scale = 1e-8f;
    const float inv = __fdiv_rn(1.0f, scale);
    for (int i = threadIdx.x; i < ld; i += NT) {
        int v = 0;
        if (i < d) {
            const float s = __fmul_rn(x[i], inv);
            /* (int)NaN is the x86 integer indefinite, clamped to -127 */
            if (s != s) v = -127;
            else {
                v = __float2int_rz(s);
                v = v > 127 ? 127 : (v < -127 ? -127 : v);
            }
        }
        xq[i] = (int8_t)v;
    }
    if (threadIdx.x == 0) *scale_out = scale;
}

/* The 512 rows the server's min-heap keeps (gpt2_server.c:2160-2197), from
 * the int8 logits of all V rows held as order keys in one CTA's shared memory
 * (V <= kGpt2MaxV): T, the N-th largest key with multiplicity, from a 12-bit
 * histogram of the keys (the bin where the count from the top reaches N,
 * searched by one warp down from the largest key's bin) and a count among the
 * keys of that bin (a radix select over all keys when the bin is crowded).  When
 * exactly N rows reach T they are the heap's rows, listed in any order;
 * otherwise rows tie at T across the boundary and thread 0 replays the
 * heap's pushes and root replacements over the keys in index order (keys
 * compare as the floats do: -0 and +0 share one).  Writes the rows to
 * cand_out and their count to *n_out. */
__global__ void __launch_bounds__(kGpt2SelThreads, 1)
    gpt2_select_kernel(const float *logits, int V, int N, int *cand_out, int *n_out,
                       const int *status) {
    extern __shared__ __align__(16) uint32_t keys[];
    __shared__ __align__(16) uint32_t hist[4096]; /* then the boundary bin's keys */
    __shared__ uint32_t sh[4];
    __shared__ int cnt;
    __shared__ uint32_t heap_key[kGpt2RerankN];
    __shared__ int heap_idx[kGpt2RerankN];
    if (*status != 0) return; /* the LM head failed: the step reports it */
    const int tid = threadIdx.x, lane = tid & 31;
    const int Vr = (V + kGpt2SelThreads - 1) / kGpt2SelThreads * kGpt2SelThreads;
    for (int i = tid; i < 4096; i += kGpt2SelThreads) hist[i] = 0u;
    if (tid == 0) sh[3] = 0u;
    __syncthreads();
    /* keys, their 12-bit histogram and the largest key (16-byte reads when
     * the logits start on a 16-byte boundary) */
    uint32_t mk = 0u;
    auto take_key = [&](int i, float l) {
        const uint32_t key = f2key(l);
        keys[i] = key;
        atomicAdd(&hist[key >> 20], 1u);
        mk = max(mk, key);
    };
    const bool al16 = (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
    const int nv = al16 ? V / 4 : 0;
#pragma unroll 2
    for (int e = tid; e < nv; e += kGpt2SelThreads) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(logits) + e);
        take_key(4 * e, v.x);
        take_key(4 * e + 1, v.y);
        take_key(4 * e + 2, v.z);
        take_key(4 * e + 3, v.w);
    }
    for (int i = 4 * nv + tid; i < V; i += kGpt2SelThreads) take_key(i, __ldcg(logits + i));
    mk = __reduce_max_sync(0xffffffffu, mk);
    if (lane == 0) atomicMax(&sh[3], mk);
    __syncthreads();
    /* the bin holding the N-th largest key, the count above it and its own */
    if (tid < 32) {
        const uint32_t bin = warp_boundary_bin_4096(hist, sh[3] >> 20, (uint32_t)N);
        uint32_t above = 0u;
        for (int q = (int)bin + 1 + lane; q <= (int)(sh[3] >> 20); q += 32) above += hist[q];
        above = __reduce_add_sync(0xffffffffu, above);
        if (lane == 0) {
            sh[0] = bin;
            sh[1] = above;
            sh[2] = hist[bin];
        }
    }
    __syncthreads();
    const uint32_t bin = sh[0], above = sh[1], nb = sh[2];
    const uint32_t edge = bin << 20;
    if (above + nb <= (uint32_t)kGpt2SelCap) {
        /* one pass: every key at or above the bin's lower edge with its row
         * (into the histogram's memory); T and the rows come from them */
        uint32_t *ck = hist;
        int *ci = reinterpret_cast<int *>(hist + kGpt2SelCap);
        if (tid == 0) cnt = 0;
        __syncthreads();
        for (int i = tid; i < Vr; i += kGpt2SelThreads) {
            const uint32_t key = i < V ? keys[i] : 0u;
            const bool in = i < V && key >= edge;
            const unsigned bal = __ballot_sync(0xffffffffu, in);
            if (bal) {
                int base = 0;
                if (lane == 0) base = atomicAdd(&cnt, __popc(bal));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (in) {
                    const int pos = base + __popc(bal & ((1u << lane) - 1u));
                    ck[pos] = key;
                    ci[pos] = i;
                }
            }
        }
        __syncthreads();
        const int na = cnt; /* = above + nb */
        /* T = min{ key of the bin : #{gathered keys > key} < N } */
        uint32_t best = 0xffffffffu;
        for (int e = tid; e < na; e += kGpt2SelThreads) {
            const uint32_t me = ck[e];
            if ((me >> 20) != bin) continue;
            uint32_t gt = 0u;
            for (int j = 0; j < na; ++j) gt += ck[j] > me;
            if (gt < (uint32_t)N) best = min(best, me);
        }
        best = __reduce_min_sync(0xffffffffu, best);
        if (tid == 0) sh[0] = 0xffffffffu;
        __syncthreads();
        if (lane == 0) atomicMin(&sh[0], best);
        __syncthreads();
        const uint32_t T = sh[0];
        /* the rows at or above T: the heap's rows when there are exactly N */
        int c = 0;
        for (int e = tid; e < na; e += kGpt2SelThreads) c += ck[e] >= T;
        if (tid == 0) cnt = 0;
        __syncthreads();
        c = __reduce_add_sync(0xffffffffu, c);
        if (lane == 0 && c) atomicAdd(&cnt, c);
        __syncthreads();
        const int mt = cnt;
        if (mt == N) {
            __syncthreads();
            if (tid == 0) cnt = 0;
            __syncthreads();
            const int nar = (na + kGpt2SelThreads - 1) / kGpt2SelThreads * kGpt2SelThreads;
            for (int e = tid; e < nar; e += kGpt2SelThreads) {
                const bool take = e < na && ck[e] >= T;
                const unsigned bal = __ballot_sync(0xffffffffu, take);
                if (bal) {
                    int base = 0;
                    if (lane == 0) base = atomicAdd(&cnt, __popc(bal));
                    base = __shfl_sync(0xffffffffu, base, 0);
                    if (take) cand_out[base + __popc(bal & ((1u << lane) - 1u))] = ci[e];
                }
            }
            if (tid == 0) *n_out = N;
            return;
        }
        /* ties across the boundary: the heap replay below */
    } else {
        /* a crowded boundary: radix select over all keys (8-bit digits) */
        uint32_t prefix = 0u, mask = 0u;
        uint32_t krem = (uint32_t)N;
        for (int shift = 24; shift >= 0; shift -= 8) {
            if (tid < 256) hist[tid] = 0u;
            __syncthreads();
            for (int i = tid; i < Vr; i += kGpt2SelThreads) {
                const uint32_t key = i < V ? keys[i] : 0u;
                const bool m = i < V && (key & mask) == prefix;
                const uint32_t digit = (key >> shift) & 0xFFu;
                const unsigned voters = __ballot_sync(0xffffffffu, m);
                if (m) {
                    const unsigned peers = __match_any_sync(voters, digit);
                    if (lane == __ffs(peers) - 1) atomicAdd(&hist[digit], (uint32_t)__popc(peers));
                }
            }
            __syncthreads();
            if (tid < 32) {
                /* from the top: lane l holds digits 255-8l .. 248-8l */
                uint32_t c[8], sum = 0u;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c[j] = hist[255 - 8 * lane - j];
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
        const uint32_t T = prefix;
        /* rows at or above T */
        if (tid == 0) cnt = 0;
        __syncthreads();
        int c = 0;
        for (int i = tid; i < V; i += kGpt2SelThreads) c += keys[i] >= T;
        c = __reduce_add_sync(0xffffffffu, c);
        if (lane == 0 && c) atomicAdd(&cnt, c);
        __syncthreads();
        const int m = cnt;
        __syncthreads();
        if (m == N) {
            if (tid == 0) cnt = 0;
            __syncthreads();
            for (int i = tid; i < Vr; i += kGpt2SelThreads) {
                const bool take = i < V && keys[i] >= T;
                const unsigned bal = __ballot_sync(0xffffffffu, take);
                if (bal) {
                    int base = 0;
                    if (lane == 0) base = atomicAdd(&cnt, __popc(bal));
                    base = __shfl_sync(0xffffffffu, base, 0);
                    if (take) cand_out[base + __popc(bal & ((1u << lane) - 1u))] = i;
                }
            }
            if (tid == 0) *n_out = N;
            return;
        }
    }
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
    }
}

/* The float re-score (gpt2_server.c:2203-2211) of up to kRerankRows listed
 * rows a CTA: x and the rows are staged into shared memory with 16-byte
 * asynchronous copies, then eight lanes a row sum x[i] * ((float)wq[i] *
 * scale) as fused multiply-adds, lane j over i = j (mod 8) in index order,
 * and add the lanes left to right (v8f_hsum, :110-113). */
__global__ void __launch_bounds__(kRerankWarps * 32)
    gpt2_rerank_kernel(const float *x, int d, const int8_t *W, int ld, const float *sw,
                       float *logits, const int *cand, const int *n_ptr, const int *status) {
    extern __shared__ __align__(16) uint8_t rsm[];
    if (*status != 0) return;
    const int n = *n_ptr;
    const int j0 = blockIdx.x * kRerankRows;
    if (j0 >= n) return;
    const int rn = min(kRerankRows, n - j0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
        cp_async16(rows + (size_t)r * ld + 16 * q, W + (size_t)cand[j0 + r] * ld + 16 * q);
    }
    cp_async_wait_all();
    __syncthreads();
    const int sub = lane >> 3, lane8 = lane & 7;
    for (int r0 = warp * 4; r0 < rn; r0 += kRerankWarps * 4) {
        const int r = r0 + sub;
        const bool on = r < rn;
        const int8_t *wr = reinterpret_cast<const int8_t *>(rows + (size_t)(on ? r : 0) * ld);
        const int v = on ? cand[j0 + r] : 0;
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
        if (on && lane8 == 0) logits[v] = s;
    }
}

}  // namespace

cudaError_t launch_gpt2_quantize(const float *x, int d, int8_t *xq, int ld, float *scale_out,
                                 cudaStream_t st) {
    gpt2_quantize_kernel<<<1, NT, 0, st>>>(x, d, xq, ld, scale_out);
    return cudaGetLastError();
}

cudaError_t launch_gpt2_select(const float *logits, int V, int N, int *cand_out, int *n_out,
                               const int *status, cudaStream_t st) {
    const int bytes = 4 * V;
    cudaError_t e = raise_smem((const void *)gpt2_select_kernel, bytes);
    if (e != cudaSuccess) return e;
    gpt2_select_kernel<<<1, kGpt2SelThreads, bytes, st>>>(logits, V, N, cand_out, n_out, status);
    return cudaGetLastError();
}

cudaError_t launch_gpt2_rerank(const float *x, int d, const int8_t *W, int ld, const float *sw,
                               float *logits, const int *cand, const int *n_dev, int N,
                               const int *status, cudaStream_t st) {
    const int bytes = kRerankRows * ld + 4 * d;
    cudaError_t e = raise_smem((const void *)gpt2_rerank_kernel, bytes);
    if (e != cudaSuccess) return e;
    const int grid = (N + kRerankRows - 1) / kRerankRows;
    gpt2_rerank_kernel<<<grid, kRerankWarps * 32, bytes, st>>>(x, d, W, ld, sw, logits, cand,
                                                              n_dev, status);
    return cudaGetLastError();
}

}  // namespace lal
