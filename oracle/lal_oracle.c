/*
 * lal_oracle.c -- CPU restatement of the LAL decode tail.
 *
 * TEST INFRASTRUCTURE ONLY (see lal_oracle.h).  Written from the reference's
 * behaviour, in plain scalar C, so that every arithmetic step is visible:
 * float32 operations in the reference's order, no FMA contraction (the build
 * passes -ffp-contract=off), glibc expf for the softmax exactly as the
 * reference calls it.
 */
#include "lal_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- quantisation of the hidden vector ------------------------------------
 * runtime/lal_q8_kernel.h:375-424.  The servers build with -march=native, so
 * the AVX2+FMA branch is the reference: absmax over all n (order-free),
 * scale = max/127 floored at 1e-8, inv = 1/scale; the first n&~7 elements go
 * through _mm256_cvtps_epi32 (round to nearest even, :409) and the last n%8
 * through a C cast (truncation, :418-423); both clamp to [-127, 127].
 */
static int cvt_rne(float v) {
    /* _mm256_cvtps_epi32 on a NaN or out-of-range value yields INT_MIN. */
    if (!(v > -2147483648.0f && v < 2147483648.0f)) return (int)0x80000000u;
    return (int)nearbyintf(v); /* default rounding mode: nearest-even */
}

/* runtime/lal_simd_optim.h:32-58, for n a multiple of 8 (returns without
 * writing otherwise: the reference's scalar tail loop at :45 is compiled by
 * its compiler into a mix of separately rounded and fused products that no
 * fixed rule reproduces).  Eight lane accumulators: lane j takes x[i]^2 for
 * i = j (mod 8) as fused multiply-adds in index order (_mm256_fmadd_ps,
 * :39-43); lal_hsum_m256 (:21-28) adds the 128-bit halves (v_j + v_{j+4})
 * and then two horizontal adds: ((s0+s1)+(s2+s3)).  inv_rms =
 * 1/sqrtf(ms/n + eps) (:47); the output is (x * inv_rms) * w (:52-56). */
void orc_rms_norm(float *out, const float *x, const float *w, int n, float eps) {
    if (n <= 0 || n % 8 != 0) return;
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < n; i += 8)
        for (int j = 0; j < 8; ++j) v[j] = fmaf(x[i + j], x[i + j], v[j]);
    const float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    const float ms = (s0 + s1) + (s2 + s3);
    const float inv = 1.0f / sqrtf(ms / (float)n + eps);
    for (int i = 0; i < n; ++i) out[i] = (x[i] * inv) * w[i];
}

float orc_quantize_x_int8(const float *x, int8_t *xq, int n) {
    float max_abs = 0.0f;
    for (int i = 0; i < n; i++) {
        float a = fabsf(x[i]);
        if (a > max_abs) max_abs = a;
    }
    float scale = max_abs / 127.0f;
    if (scale < 1e-8f) scale = 1e-8f;
    float inv = 1.0f / scale;
    int n8 = n & ~7;
    for (int i = 0; i < n; i++) {
        float s = x[i] * inv;
        int v = (i < n8) ? cvt_rne(s) : (int)s;
        if (v > 127) v = 127;
        if (v < -127) v = -127;
        xq[i] = (int8_t)v;
    }
    return scale;
}

/* runtime/lal_q8_kernel.h:450-460: |xq| as uint8. */
void orc_compute_abs_xq(const int8_t *xq, uint8_t *ax, int n) {
    for (int i = 0; i < n; i++) ax[i] = (uint8_t)(xq[i] < 0 ? -xq[i] : xq[i]);
}

/* ---- LM head ----------------------------------------------------------------
 * runtime/lal_q8_kernel.h:463-499 (and the _abs / _abs_8row forms at
 * :506-543 / :551-640, which produce identical values): an exact int32 dot
 * per vocab row, then logits[v] = scale_x * scale_w[v] * (float)dot,
 * evaluated left to right (:489).  The AVX2 sign trick equals the signed dot
 * whenever |xq| <= 127 and |w| <= 127, which both quantizers guarantee.
 */
void orc_lm_head_dots(int32_t *dots, const int8_t *xq, const int8_t *wte_q,
                      int v_start, int v_end, int n_embd) {
    for (int v = v_start; v < v_end; v++) {
        const int8_t *w = wte_q + (size_t)v * n_embd;
        int32_t acc = 0;
        for (int i = 0; i < n_embd; i++) acc += (int32_t)xq[i] * (int32_t)w[i];
        dots[v - v_start] = acc;
    }
}

/* Rows are independent, so large ranges are split over OpenMP threads (the
 * reference splits its vocab the same way, qwen7b_server.c:833-845); every
 * row's dot product and logit are the same whatever the split. */
void orc_lm_head_int8_range(float *logits, const int8_t *xq, float scale_x,
                            const int8_t *wte_q, const float *scale_w,
                            int v_start, int v_end, int n_embd) {
    #pragma omp parallel for schedule(static) if ((long)(v_end - v_start) * n_embd > (1L << 22))
    for (int v = v_start; v < v_end; v++) {
        int32_t dot;
        orc_lm_head_dots(&dot, xq, wte_q, v, v + 1, n_embd);
        float s = scale_x * scale_w[v];
        logits[v] = s * (float)dot;
    }
}

/* The same logits for B quantized vectors at once (a batched decode step
 * restated as B calls of the 1-row form above): logits[b][v] for v in
 * [0, vocab).  Rows are taken in blocks of 16 that every vector visits
 * while they are in cache; each logit is the 1-row form's
 * (scale_x[b] * scale_w[v]) * (float)dot, exact int32 dot. */
void orc_lm_head_multi(float *logits, const int8_t *xq, const float *scale_x,
                       const int8_t *wte_q, const float *scale_w, int vocab, int n_embd,
                       int n_vec) {
    #pragma omp parallel for schedule(static)
    for (int v0 = 0; v0 < vocab; v0 += 16) {
        const int v1 = v0 + 16 < vocab ? v0 + 16 : vocab;
        for (int b = 0; b < n_vec; b++) {
            const int8_t *x = xq + (size_t)b * n_embd;
            for (int v = v0; v < v1; v++) {
                const int8_t *w = wte_q + (size_t)v * n_embd;
                int32_t acc = 0;
                for (int i = 0; i < n_embd; i++) acc += (int32_t)x[i] * (int32_t)w[i];
                float s = scale_x[b] * scale_w[v];
                logits[(size_t)b * vocab + v] = s * (float)acc;
            }
        }
    }
}

/* runtime/lal_q8_kernel.h:551-640.  Rows taken in full groups of 8 from
 * v_start (:562) sum only the first n_embd & ~31 columns -- the group body
 * (:577-611) has no scalar tail, unlike the 1-row forms (:488, :532) and the
 * 1-row remainder (:614-631), which sum all columns. */
void orc_lm_head_int8_range_abs_8row(float *logits, const int8_t *xq, float scale_x,
                                     const int8_t *wte_q, const float *scale_w,
                                     int v_start, int v_end, int n_embd) {
    int v = v_start;
    const int n32 = n_embd & ~31;
    for (; v + 8 <= v_end; v += 8)
        for (int r = 0; r < 8; r++) {
            const int8_t *w = wte_q + (size_t)(v + r) * n_embd;
            int32_t dot = 0;
            for (int i = 0; i < n32; i++) dot += (int32_t)xq[i] * (int32_t)w[i];
            float s = scale_x * scale_w[v + r];
            logits[v + r] = s * (float)dot;
        }
    orc_lm_head_int8_range(logits, xq, scale_x, wte_q, scale_w, v, v_end, n_embd);
}

/* ---- per-row weight quantisation ------------------------------------------
 * runtime/lal_q8_kernel.h:357-372: scale = max|row|/127 floored at 1e-8,
 * q = clamp(lroundf(w * (1/scale)), +-127) -- round half AWAY from zero.
 */
void orc_quantize_q8_rows(const float *W, int8_t *q8_T, float *scale,
                          int in_dim, int n_rows) {
    for (int j = 0; j < n_rows; j++) {
        const float *row = W + (size_t)j * in_dim;
        float mx = 0.0f;
        for (int i = 0; i < in_dim; i++) {
            float a = fabsf(row[i]);
            if (a > mx) mx = a;
        }
        float s = mx / 127.0f;
        if (s < 1e-8f) s = 1e-8f;
        scale[j] = s;
        float inv = 1.0f / s;
        for (int i = 0; i < in_dim; i++) {
            long q = lroundf(row[i] * inv);
            if (q > 127) q = 127;
            if (q < -127) q = -127;
            q8_T[(size_t)j * in_dim + i] = (int8_t)q;
        }
    }
}

void orc_quantize_q8_per_row(const float *W, int8_t *q8_T, float *scale,
                             int in_dim, int out_dim) {
    orc_quantize_q8_rows(W, q8_T, scale, in_dim, out_dim);
}

/* ---- sampling ---------------------------------------------------------------*/

/* Repetition penalty, runtime/lal_sampling.h:59-67 (and the identical loop at
 * tools/server/qwen7b_server.c:223-230): once per occurrence, in order. */
static void apply_penalty(float *logits, int vocab_size, float rep_penalty,
                          const int *recent, int n_recent) {
    if (!(rep_penalty > 1.0f) || !recent || n_recent <= 0) return;
    for (int i = 0; i < n_recent; i++) {
        int t = recent[i];
        if (t < 0 || t >= vocab_size) continue;
        if (logits[t] > 0) logits[t] /= rep_penalty;
        else logits[t] *= rep_penalty;
    }
}

/* Greedy argmax with strict '>' (lowest index wins ties):
 * runtime/lal_sampling.h:51-56. */
static int argmax_first(const float *logits, int vocab_size) {
    int best = 0;
    for (int v = 1; v < vocab_size; v++)
        if (logits[v] > logits[best]) best = v;
    return best;
}

/* Top-k threshold by a min-heap of capacity k (runtime/lal_sampling.h:70-104,
 * tools/server/qwen7b_server.c:237-256).  The heap takes the first k values,
 * then replaces its root only on a STRICTLY larger value; its final root is
 * the k-th largest value counted with multiplicity.  The capacity here is k
 * itself, so k larger than the reference's static 64 / 512 is defined. */
static float heap_threshold(const float *logits, int vocab_size, int k) {
    float *h = (float *)malloc(sizeof(float) * (size_t)k);
    int hn = 0;
    for (int v = 0; v < vocab_size; v++) {
        float val = logits[v];
        if (hn < k) {
            int c = hn++;
            h[c] = val;
            while (c > 0) {               /* sift up */
                int p = (c - 1) / 2;
                if (h[p] <= h[c]) break;
                float t = h[p]; h[p] = h[c]; h[c] = t;
                c = p;
            }
        } else if (val > h[0]) {
            h[0] = val;
            int p = 0;
            for (;;) {                    /* sift down */
                int l = 2 * p + 1, r = l + 1, s = p;
                if (l < hn && h[l] < h[s]) s = l;
                if (r < hn && h[r] < h[s]) s = r;
                if (s == p) break;
                float t = h[p]; h[p] = h[s]; h[s] = t;
                p = s;
            }
        }
    }
    float th = h[0];
    free(h);
    return th;
}

int orc_sample_token(float *logits, int vocab_size, float temperature,
                     int top_k, float rep_penalty, const int *recent,
                     int n_recent, float u, orc_sample_info *info) {
    orc_sample_info tmp;
    if (!info) info = &tmp;
    memset(info, 0, sizeof(*info));
    /* lal_sampling.h:51-56: greedy BEFORE the penalty in the library form. */
    if (temperature <= 0.0f || top_k <= 0) {
        info->greedy = 1;
        return argmax_first(logits, vocab_size);
    }
    apply_penalty(logits, vocab_size, rep_penalty, recent, n_recent);
    int k = top_k;
    if (k > vocab_size) k = vocab_size;                   /* :70-71 */
    float threshold = heap_threshold(logits, vocab_size, k);
    float max_l = -1e30f;                                 /* :107-109 */
    int n_cand = 0;
    for (int v = 0; v < vocab_size; v++)
        if (logits[v] >= threshold) {
            n_cand++;
            if (logits[v] > max_l) max_l = logits[v];
        }
    float sum = 0;                                        /* :110-113 */
    for (int v = 0; v < vocab_size; v++)
        if (logits[v] >= threshold) sum += expf((logits[v] - max_l) / temperature);
    float r = u * sum;                                    /* :116 */
    info->threshold = threshold; info->max_l = max_l; info->sum = sum;
    info->r = r; info->n_cand = n_cand; info->drew = 1;
    float acc = 0;                                        /* :117-123 */
    for (int v = 0; v < vocab_size; v++) {
        if (logits[v] >= threshold) {
            acc += expf((logits[v] - max_l) / temperature);
            if (r <= acc) return v;
        }
    }
    return vocab_size - 1;                                /* :124 */
}

int orc_sample_token_filtered(float *logits, int vocab_size, float temperature,
                              int top_k, float rep_penalty, const int *recent,
                              int n_recent, orc_filter_fn filter,
                              orc_decode_fn decode, orc_draw_fn draw,
                              void *draw_ctx, orc_sample_info *info) {
    orc_sample_info tmp;
    if (!info) info = &tmp;
    memset(info, 0, sizeof(*info));
    /* qwen7b_server.c:223-230: penalty first, then the greedy check :231-234 */
    apply_penalty(logits, vocab_size, rep_penalty, recent, n_recent);
    if (temperature <= 0.0f || top_k <= 0) {
        info->greedy = 1;
        return argmax_first(logits, vocab_size);
    }
    int k = top_k;                                        /* :236 */
    if (k < 1) k = 1;
    if (k > vocab_size) k = vocab_size;
    float threshold = heap_threshold(logits, vocab_size, k);
    /* :258-270: keep_mask = candidates, optional filter, restore if empty */
    int *keep = (int *)malloc(sizeof(int) * (size_t)vocab_size);
    for (int v = 0; v < vocab_size; v++) keep[v] = (logits[v] >= threshold) ? 1 : 0;
    if (filter) {
        int last = (n_recent > 0) ? recent[n_recent - 1] : -1;
        (void)filter(keep, vocab_size, last, recent, n_recent, decode);
    }
    int any = 0;
    for (int v = 0; v < vocab_size; v++) if (keep[v]) { any = 1; break; }
    if (!any)
        for (int v = 0; v < vocab_size; v++) if (logits[v] >= threshold) keep[v] = 1;
    /* :275-284: max then sum over kept & >= threshold */
    float max_l = -1e30f, sum = 0;
    int n_cand = 0;
    for (int v = 0; v < vocab_size; v++)
        if (keep[v] && logits[v] >= threshold) {
            n_cand++;
            if (logits[v] > max_l) max_l = logits[v];
        }
    for (int v = 0; v < vocab_size; v++)
        if (keep[v] && logits[v] >= threshold)
            sum += expf((logits[v] - max_l) / temperature);
    info->threshold = threshold; info->max_l = max_l; info->sum = sum;
    info->n_cand = n_cand;
    int tok;
    if (sum <= 0) {                                        /* :285-286 */
        int best = 0; float bv = -1e30f;
        for (int v = 0; v < vocab_size; v++)
            if (keep[v] && logits[v] > bv) { bv = logits[v]; best = v; }
        tok = best;
    } else {
        float u = draw ? draw(draw_ctx) : 0.0f;            /* :287 */
        float r = u * sum, acc = 0;
        info->r = r; info->drew = 1;
        tok = vocab_size - 1;                              /* :294 */
        for (int v = 0; v < vocab_size; v++) {
            if (keep[v] && logits[v] >= threshold) {
                acc += expf((logits[v] - max_l) / temperature);
                if (r <= acc) { tok = v; break; }
            }
        }
    }
    free(keep);
    return tok;
}

/* runtime/lal_sampling.h:133-136 (FIFO by memmove), capacity cap. */
void orc_recent_push(int *tokens, int *n, int cap, int tok) {
    if (*n < cap) { tokens[(*n)++] = tok; return; }
    memmove(tokens, tokens + 1, (size_t)(cap - 1) * sizeof(int));
    tokens[cap - 1] = tok;
}

/* glibc expf over an array: the softmax weight function of
 * runtime/lal_sampling.h:112,120, for checking the device's weights. */
void orc_expf_batch(const float *x, float *y, long n) {
    for (long i = 0; i < n; i++) y[i] = expf(x[i]);
}

static float fixed_draw(void *ctx) { return *(const float *)ctx; }

int orc_tail_step(const float *hidden, int n_embd, const int8_t *wte_q,
                  const float *scale_w, int vocab_size, float temperature,
                  int top_k, float rep_penalty, int *recent, int *n_recent,
                  int hist_cap, float u, int variant, float *logits_out,
                  orc_sample_info *info) {
    int8_t *xq = (int8_t *)malloc((size_t)n_embd);
    float *logits = logits_out ? logits_out
                               : (float *)malloc(sizeof(float) * (size_t)vocab_size);
    float sx = orc_quantize_x_int8(hidden, xq, n_embd);
    orc_lm_head_int8_range(logits, xq, sx, wte_q, scale_w, 0, vocab_size, n_embd);
    int tok;
    if (variant == 0)
        tok = orc_sample_token(logits, vocab_size, temperature, top_k, rep_penalty,
                               recent, *n_recent, u, info);
    else
        tok = orc_sample_token_filtered(logits, vocab_size, temperature, top_k,
                                        rep_penalty, recent, *n_recent, NULL, NULL,
                                        fixed_draw, &u, info);
    orc_recent_push(recent, n_recent, hist_cap, tok);
    free(xq);
    if (!logits_out) free(logits);
    return tok;
}


/* ------------------------------------------------------------------ *
 * The GPT-2 server's LM-head tail (tools/server/gpt2_server.c)       *
 * ------------------------------------------------------------------ */

/* gpt2_server.c:1982-1998: max |x| kept with '>', scale = max/127 floored at
 * 1e-8, inv = 1/scale, (int)(x*inv) truncated and clamped to +-127 ((int)NaN
 * is the x86 integer indefinite: -127 after the clamp). */
float orc_gpt2_quantize_x(const float *x, int8_t *xq, int n) {
    float max_abs = 0.0f;
    for (int i = 0; i < n; i++) {
        const float a = fabsf(x[i]);
        if (a > max_abs) max_abs = a;
    }
    float scale = max_abs / 127.0f;
    if (scale < 1e-8f) scale = 1e-8f;
    const float inv = 1.0f / scale;
    for (int i = 0; i < n; i++) {
        const float s = x[i] * inv;
        int v = (s != s || s >= 2147483648.0f || s < -2147483648.0f) ? INT32_MIN : (int)s;
        if (v > 127) v = 127;
        if (v < -127) v = -127;
        xq[i] = (int8_t)v;
    }
    return scale;
}

#define ORC_GPT2_RERANK_N 512

/* gpt2_server.c:2125-2214.  Pass 1 (:2013-2095): exact int32 dots, logits =
 * scale_x * scale_w[v] * (float)dot left to right.  Pass 2 (:2160-2197): a
 * min-heap of RERANK_N (value, row) entries over v = 0..V-1: the first N are
 * pushed with sift-up (stop when parent <= child); later rows replace the
 * root only when strictly greater, then sift down to the strictly smaller
 * child (left first).  Re-score (:2203-2211): w_row[i] = (float)wq[i] *
 * scale_w[v]; eight lane sums of fused multiply-adds x[i] * w_row[i], lane j
 * over i = j (mod 8) in index order; v8f_hsum (:110-113) adds the lanes left
 * to right. */
int orc_gpt2_lm_head(float *logits, const float *x, const int8_t *wte_q, const float *scale_w,
                     int vocab_size, int n, int *kept) {
    int8_t *xq = (int8_t *)malloc((size_t)n);
    const float sx = orc_gpt2_quantize_x(x, xq, n);
    for (int v = 0; v < vocab_size; v++) {
        const int8_t *w = wte_q + (size_t)v * n;
        int32_t dot = 0;
        for (int i = 0; i < n; i++) dot += (int32_t)xq[i] * (int32_t)w[i];
        logits[v] = sx * scale_w[v] * (float)dot;
    }
    free(xq);
    static int heap_idx[ORC_GPT2_RERANK_N];
    static float heap_val[ORC_GPT2_RERANK_N];
    int heap_n = 0;
    for (int v = 0; v < vocab_size; v++) {
        const float val = logits[v];
        if (heap_n < ORC_GPT2_RERANK_N) {
            int c = heap_n++;
            heap_val[c] = val;
            heap_idx[c] = v;
            while (c > 0) {
                const int p = (c - 1) >> 1;
                if (heap_val[p] <= heap_val[c]) break;
                float tv = heap_val[p]; heap_val[p] = heap_val[c]; heap_val[c] = tv;
                int ti = heap_idx[p]; heap_idx[p] = heap_idx[c]; heap_idx[c] = ti;
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
                float tv = heap_val[p]; heap_val[p] = heap_val[s]; heap_val[s] = tv;
                int ti = heap_idx[p]; heap_idx[p] = heap_idx[s]; heap_idx[s] = ti;
                p = s;
            }
        }
    }
    for (int k = 0; k < heap_n; k++) {
        const int v = heap_idx[k];
        const int8_t *wq = wte_q + (size_t)v * n;
        const float scale = scale_w[v];
        float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int i = 0; i + 8 <= n; i += 8)
            for (int j = 0; j < 8; j++) lane[j] = fmaf(x[i + j], (float)wq[i + j] * scale, lane[j]);
        float s = lane[0];
        for (int j = 1; j < 8; j++) s = s + lane[j];
        logits[v] = s;
        if (kept) kept[k] = v;
    }
    return heap_n;
}

/* gpt2_server.c:2862-3013 with g_top_p = 0 (its default, :2343) and the
 * weak no-op filter (the keep mask unchanged).  Sampling branch
 * (temperature > 0 and top_k > 0): the penalty per recent occurrence in order
 * (l > 0 ? l /= p : l *= p) when p > 1; k = min(top_k, V); k passes of
 * find-max (strict '>', lowest row) and mask with -1e30f leave threshold =
 * the k-th largest logit with multiplicity; keep = {l >= threshold};
 * actual_max over the kept rows with '>' from -1e30f; sum_exp +=
 * expf((l - actual_max) / T) for kept rows in ascending order (the others add
 * 0.0f, which leaves the sum unchanged); r = u * sum_exp; the running sum
 * walks every row (zeros below the threshold) and returns the first row
 * where it reaches r, else V-1.  Otherwise argmax (strict '>', lowest row),
 * no penalty. */
int orc_gpt2_sample(float *logits, int vocab_size, float temperature, int top_k,
                    float rep_penalty, const int *recent, int n_recent, float u,
                    orc_sample_info *info) {
    return orc_gpt2_sample_p(logits, vocab_size, temperature, top_k, 0.0f, rep_penalty, recent,
                             n_recent, u, info);
}

/* The same with the server's nucleus branch (gpt2_server.c:2895-2960, on
 * when 0 < top_p < 1): the rows l >= threshold (ascending index), their
 * temperature softmax over the largest of them -- expf terms summed in that
 * order, inv = 1 / (sum + 1e-12f), each term times inv -- an insertion sort
 * descending by probability (stable: equal probabilities keep ascending
 * index), and rows kept in that order until the running probability sum
 * reaches top_p (the row that reaches it is kept).  No level-2 filter is
 * linked (the weak lal_filter_topk keeps the mask, :2969-2979).  The softmax
 * and draw then run over the kept rows (:2981-3002). */
int orc_gpt2_sample_p(float *logits, int vocab_size, float temperature, int top_k, float top_p,
                      float rep_penalty, const int *recent, int n_recent, float u,
                      orc_sample_info *info) {
    return orc_gpt2_sample_f(logits, vocab_size, temperature, top_k, top_p, rep_penalty, recent,
                             n_recent, NULL, NULL, u, info);
}

/* The same with the server's level-2 filter hook (gpt2_server.c:2962-2978):
 * after the top-k (and top-p) keep mask, filter(keep_mask, V, last token,
 * recent, n_recent, decode) may change any entry; if no entry is left, the
 * top-k pool {l >= threshold} is restored.  The softmax and the draw then
 * run over every row the mask keeps (gpt2_server.c:2981-3002). */
int orc_gpt2_sample_f(float *logits, int vocab_size, float temperature, int top_k, float top_p,
                      float rep_penalty, const int *recent, int n_recent,
                      orc_filter_fn filter, orc_decode_fn decode, float u,
                      orc_sample_info *info) {
    orc_sample_info loc;
    if (!info) info = &loc;
    memset(info, 0, sizeof(*info));
    if (temperature > 0.0f && top_k > 0) {
        if (rep_penalty > 1.0f)
            for (int i = 0; i < n_recent; i++) {
                const int t = recent[i];
                if (t >= 0 && t < vocab_size) {
                    if (logits[t] > 0) logits[t] /= rep_penalty;
                    else logits[t] *= rep_penalty;
                }
            }
        int k = top_k > vocab_size ? vocab_size : top_k;
        float *copy = (float *)malloc(sizeof(float) * (size_t)vocab_size);
        memcpy(copy, logits, sizeof(float) * (size_t)vocab_size);
        float threshold = -1e30f;
        for (int sel = 0; sel < k; sel++) {
            int max_v = 0;
            float max_val = copy[0];
            for (int v = 1; v < vocab_size; v++)
                if (copy[v] > max_val) { max_val = copy[v]; max_v = v; }
            threshold = max_val;
            copy[max_v] = -1e30f;
        }
        int *keep = (int *)calloc((size_t)vocab_size, sizeof(int));
        if (top_p > 0.0f && top_p < 1.0f) {
            int *top_idx = (int *)malloc(sizeof(int) * (size_t)vocab_size);
            float *top_val = (float *)malloc(sizeof(float) * (size_t)vocab_size);
            int n_top = 0;
            for (int v = 0; v < vocab_size; v++)
                if (logits[v] >= threshold) {
                    top_idx[n_top] = v;
                    top_val[n_top] = logits[v];
                    n_top++;
                }
            float top_max = -1e30f;
            for (int i = 0; i < n_top; i++)
                if (top_val[i] > top_max) top_max = top_val[i];
            float top_sum = 0.0f;
            for (int i = 0; i < n_top; i++) {
                top_val[i] = expf((top_val[i] - top_max) / temperature);
                top_sum += top_val[i];
            }
            const float inv = 1.0f / (top_sum + 1e-12f);
            for (int i = 0; i < n_top; i++) top_val[i] *= inv;
            for (int i = 1; i < n_top; i++) {
                const float vp = top_val[i];
                const int vi = top_idx[i];
                int j = i - 1;
                while (j >= 0 && top_val[j] < vp) {
                    top_val[j + 1] = top_val[j];
                    top_idx[j + 1] = top_idx[j];
                    j--;
                }
                top_val[j + 1] = vp;
                top_idx[j + 1] = vi;
            }
            float cum = 0.0f;
            for (int i = 0; i < n_top; i++) {
                keep[top_idx[i]] = 1;
                cum += top_val[i];
                if (cum >= top_p) break;
            }
            free(top_idx);
            free(top_val);
        } else {
            for (int v = 0; v < vocab_size; v++)
                if (logits[v] >= threshold) keep[v] = 1;
        }
        if (filter) {
            const int last = n_recent > 0 ? recent[n_recent - 1] : -1;
            (void)filter(keep, vocab_size, last, recent, n_recent, decode);
            int any = 0;
            for (int v = 0; v < vocab_size && !any; v++) any = keep[v] != 0;
            if (!any)
                for (int v = 0; v < vocab_size; v++)
                    if (logits[v] >= threshold) keep[v] = 1;
        }
        float actual_max = -1e30f;
        int n_cand = 0;
        for (int v = 0; v < vocab_size; v++)
            if (keep[v]) {
                n_cand++;
                if (logits[v] > actual_max) actual_max = logits[v];
            }
        float sum_exp = 0.0f;
        for (int v = 0; v < vocab_size; v++) {
            if (keep[v]) {
                copy[v] = expf((logits[v] - actual_max) / temperature);
                sum_exp += copy[v];
            } else {
                copy[v] = 0.0f;
            }
        }
        free(keep);
        const float r = u * sum_exp;
        info->threshold = threshold;
        info->max_l = actual_max;
        info->sum = sum_exp;
        info->r = r;
        info->n_cand = n_cand;
        info->drew = 1;
        float cum = 0.0f;
        int tok = vocab_size - 1;
        for (int v = 0; v < vocab_size; v++) {
            cum += copy[v];
            if (cum >= r) { tok = v; break; }
        }
        free(copy);
        return tok;
    }
    info->greedy = 1;
    int best = 0;
    float best_val = logits[0];
    for (int v = 1; v < vocab_size; v++)
        if (logits[v] > best_val) { best_val = logits[v]; best = v; }
    return best;
}
