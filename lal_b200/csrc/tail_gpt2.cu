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
 *   tail_kernel<SAMPLE>    candidates only, k = RERANK_N: the threshold T of
 *                          the RERANK_N largest int8 logits and every row at
 *                          or above it, in ascending vocab order;
 *   gpt2_rerank_kernel     the float re-score of the RERANK_N rows picked by
 *                          the server's min-heap (gpt2_server.c:2160-2212):
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
 * them depend on the heap's history: the candidates launch reports more than
 * RERANK_N rows, and the rerank kernel then replays the server's heap exactly
 * (one thread over the logits in index order, staged through shared memory)
 * before re-scoring -- a slow path (about a millisecond) that only exact
 * logit ties at the boundary take.
 */
#include "tail_device.cuh"

namespace lal {
namespace {

constexpr int kRerankWarps = 8;          /* warps a CTA of the rerank kernel    */
constexpr int kHeapChunk = 4096;         /* logits staged a round (heap replay)  */

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

/* The float re-score of row v (gpt2_server.c:2203-2211), by the eight lanes
 * sub*8 .. sub*8+7 of the calling warp; returns the score in lane sub*8. */
__device__ __forceinline__ float rescore_row(const float *x, int d, const int8_t *wrow,
                                             float scale, int lane8) {
    float acc = 0.0f;
#pragma unroll 4
    for (int i = lane8; i < d; i += 8)
        acc = __fmaf_rn(x[i], __fmul_rn((float)wrow[i], scale), acc);
    /* v8f_hsum: t[0]+t[1]+...+t[7], left to right */
    const int base = (threadIdx.x & 31) & ~7;
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float t = __shfl_sync(0xffffffffu, acc, base + j);
        s = j == 0 ? t : __fadd_rn(s, t);
    }
    return s;
}

/* Re-scores the rows the server's heap keeps.  sel_diag->n_cand is the
 * candidates launch's count of rows at or above the N-th largest logit; the
 * common case (== N) takes the listed rows, all CTAs, four rows a warp; any
 * other count takes the exact heap replay in CTA 0 alone. */
__global__ void __launch_bounds__(kRerankWarps * 32)
    gpt2_rerank_kernel(const float *x, int d, const int8_t *W, int ld, const float *sw,
                       float *logits, int V, const int *cand_i, int cand_cap,
                       const StreamDiag *sel_diag, int N, const int *status) {
    __shared__ float heap_val[kGpt2RerankN];
    __shared__ int heap_idx[kGpt2RerankN];
    __shared__ float chunk[kHeapChunk];
    __shared__ int heap_n_s;
    if (*status != 0) return; /* the select failed: the step reports it */
    const int m = sel_diag->n_cand;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane >> 3, lane8 = lane & 7;
    if (m == N && m <= cand_cap) {
        const int gw = blockIdx.x * kRerankWarps + warp;
        const int nw = gridDim.x * kRerankWarps;
        for (int j0 = gw * 4; j0 < N; j0 += nw * 4) {
            const int j = j0 + sub;
            const bool on = j < N;
            const int v = on ? cand_i[j] : 0;
            const float s = rescore_row(x, d, W + (size_t)v * ld, on ? sw[v] : 0.0f, lane8);
            if (on && lane8 == 0) logits[v] = s;
        }
        return;
    }
    if (blockIdx.x != 0) return;
    /* the server's heap (gpt2_server.c:2167-2197), replayed by thread 0 over
     * the int8 logits in index order; the block stages them */
    int heap_n = 0;
    for (int c0 = 0; c0 < V; c0 += kHeapChunk) {
        const int cn = min(kHeapChunk, V - c0);
        __syncthreads();
        for (int i = threadIdx.x; i < cn; i += blockDim.x) chunk[i] = logits[c0 + i];
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int q = 0; q < cn; ++q) {
                const float val = chunk[q];
                const int v = c0 + q;
                if (heap_n < N) {
                    int c = heap_n++;
                    heap_val[c] = val;
                    heap_idx[c] = v;
                    while (c > 0) {
                        const int p = (c - 1) >> 1;
                        if (heap_val[p] <= heap_val[c]) break;
                        const float tv = heap_val[p];
                        heap_val[p] = heap_val[c];
                        heap_val[c] = tv;
                        const int ti = heap_idx[p];
                        heap_idx[p] = heap_idx[c];
                        heap_idx[c] = ti;
                        c = p;
                    }
                } else if (val > heap_val[0]) {
                    heap_val[0] = val;
                    heap_idx[0] = v;
                    int p = 0;
                    for (;;) {
                        const int l = 2 * p + 1, r = 2 * p + 2;
                        int s = p;
                        if (l < heap_n && heap_val[l] < heap_val[s]) s = l;
                        if (r < heap_n && heap_val[r] < heap_val[s]) s = r;
                        if (s == p) break;
                        const float tv = heap_val[p];
                        heap_val[p] = heap_val[s];
                        heap_val[s] = tv;
                        const int ti = heap_idx[p];
                        heap_idx[p] = heap_idx[s];
                        heap_idx[s] = ti;
                        p = s;
                    }
                }
            }
            heap_n_s = heap_n;
        }
    }
    __syncthreads();
    const int hn = heap_n_s;
    for (int j0 = warp * 4; j0 < hn; j0 += kRerankWarps * 4) {
        const int j = j0 + sub;
        const bool on = j < hn;
        const int v = on ? heap_idx[j] : 0;
        const float s = rescore_row(x, d, W + (size_t)v * ld, on ? sw[v] : 0.0f, lane8);
        if (on && lane8 == 0) logits[v] = s;
    }
}

}  // namespace

cudaError_t launch_gpt2_quantize(const float *x, int d, int8_t *xq, int ld, float *scale_out,
                                 cudaStream_t st) {
    gpt2_quantize_kernel<<<1, NT, 0, st>>>(x, d, xq, ld, scale_out);
    return cudaGetLastError();
}

cudaError_t launch_gpt2_rerank(const float *x, int d, const int8_t *W, int ld, const float *sw,
                               float *logits, int V, const int *cand_i, int cand_cap,
                               const StreamDiag *sel_diag, int N, const int *status,
                               int num_sms, cudaStream_t st) {
    const int grid = std::max(1, std::min(num_sms, (N + kRerankWarps * 4 - 1) / (kRerankWarps * 4)));
    gpt2_rerank_kernel<<<grid, kRerankWarps * 32, 0, st>>>(x, d, W, ld, sw, logits, V, cand_i,
                                                          cand_cap, sel_diag, N, status);
    return cudaGetLastError();
}

}  // namespace lal
