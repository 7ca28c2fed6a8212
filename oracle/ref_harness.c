/*
 * ref_harness.c -- exposes the reference's own decode-tail code as a shared
 * library (oracle/_ref/liblal_ref.so) for parity checks and the CPU baseline.
 *
 * TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile from the reference
 * sources where they lie (LAL_REF points at the samaidev/lal checkout); no
 * reference source is copied into this repository.  The whole server
 * translation unit tools/server/qwen7b_server.c is included, with its main()
 * renamed, so that the server's static sampler lal_sample_token_filtered
 * (qwen7b_server.c:219-295) and its filter hook global are reachable, and so
 * that runtime/lal_q8_kernel.h and runtime/lal_sampling.h are compiled exactly
 * as the server compiles them (XQ_MAX 18944, VOCAB_SIZE 152064, -O3
 * -march=native per Makefile:12-17,30).
 */
#define main lal_ref_qwen7b_server_main
#include "tools/server/qwen7b_server.c"
#undef main

#include <omp.h>

#define REF_API __attribute__((visibility("default")))

REF_API int ref_vocab_max(void) { return VOCAB_SIZE; }
REF_API int ref_xq_max(void) { return XQ_MAX; }

/* the server's final RMSNorm (qwen7b_server.c:624-626, 820) */
REF_API void ref_rms_norm(float *out, const float *x, const float *w, int n, float eps) {
    lal_rms_norm_simd(out, x, w, n, eps);
}

REF_API float ref_quantize_x_int8(const float *x, int8_t *xq, int n) {
    return lal_quantize_x_int8(x, xq, n);
}

/* lal_compute_abs_xq walks 32-byte chunks (lal_q8_kernel.h:452): callers
 * must pad both buffers to a multiple of 32 bytes. */
REF_API void ref_compute_abs_xq(const int8_t *xq, uint8_t *ax, int n) {
    lal_compute_abs_xq(xq, ax, n);
}

REF_API void ref_lm_head_int8_range(float *logits, const int8_t *xq, float sx,
                                    const int8_t *w, const float *sw,
                                    int v0, int v1, int n) {
    lal_lm_head_int8_range(logits, xq, sx, w, sw, v0, v1, n);
}

REF_API void ref_lm_head_int8_range_abs(float *logits, const int8_t *xq,
                                        const uint8_t *ax, float sx,
                                        const int8_t *w, const float *sw,
                                        int v0, int v1, int n) {
    lal_lm_head_int8_range_abs(logits, xq, ax, sx, w, sw, v0, v1, n);
}

REF_API void ref_lm_head_int8_range_abs_8row(float *logits, const int8_t *xq,
                                             const uint8_t *ax, float sx,
                                             const int8_t *w, const float *sw,
                                             int v0, int v1, int n) {
    lal_lm_head_int8_range_abs_8row(logits, xq, ax, sx, w, sw, v0, v1, n);
}

/* The server's OpenMP vocab split around the _abs kernel
 * (qwen7b_server.c:833-845), for an arbitrary vocab size and thread count. */
REF_API void ref_lm_head_omp(float *logits, const int8_t *xq, const uint8_t *ax,
                             float sx, const int8_t *w, const float *sw,
                             int vocab, int n, int n_threads) {
    #pragma omp parallel num_threads(n_threads)
    {
        int tid = omp_get_thread_num();
        int nthreads = omp_get_num_threads();
        int v_per = (vocab + nthreads - 1) / nthreads;
        int v_start = tid * v_per;
        int v_end = v_start + v_per;
        if (v_end > vocab) v_end = vocab;
        if (v_start < vocab)
            lal_lm_head_int8_range_abs(logits, xq, ax, sx, w, sw, v_start, v_end, n);
    }
}

REF_API void ref_quantize_q8_per_row(const float *W, int8_t *q, float *s,
                                     int in_dim, int out_dim) {
    lal_quantize_q8_per_row(W, q, s, in_dim, out_dim);
}

/* runtime/lal_sampling.h:46-125.  Its heap is static float[64]
 * (lal_sampling.h:74): top_k above 64 overflows it, so it is refused here. */
REF_API int ref_sample_token(float *logits, int vocab, float temperature, int top_k,
                             float rep_penalty, const int *recent, int n_recent) {
    if ((top_k < vocab ? top_k : vocab) > 64 && temperature > 0.0f && top_k > 0) return -2;
    return lal_sample_token(logits, vocab, temperature, top_k, rep_penalty, recent,
                            n_recent);
}

/* qwen7b_server.c:219-295.  Heap capacity 512 (:239), keep_mask[VOCAB_SIZE]
 * (:258). */
REF_API int ref_sample_token_filtered(float *logits, int vocab, float temperature,
                                      int top_k, float rep_penalty,
                                      const int *recent, int n_recent) {
    if (((top_k < vocab ? top_k : vocab) > 512 && temperature > 0.0f) || vocab > VOCAB_SIZE) return -2;
    return lal_sample_token_filtered(logits, vocab, temperature, top_k, rep_penalty,
                                     recent, n_recent);
}

/* Install (or clear with NULL) the level-2 filter the server would have
 * loaded with --lal-filter (qwen7b_server.c:208-211). */
REF_API void ref_set_filter(int (*f)(int *, int, int, const int *, int,
                                     lal_token_decode_fn)) {
    g_lal_filter = f;
}

REF_API void ref_srand(unsigned seed) { srand(seed); }
REF_API int ref_rand(void) { return rand(); }

REF_API void ref_recent_push(LalRecentTokens *rt, int tok) { lal_recent_push(rt, tok); }

/* The decode tail of one forward() call, qwen7b_server.c:829-850, for a
 * caller-sized vocab: quantize, |xq|, OpenMP LM head, sampler, history push.
 * variant 0 = lal_sample_token, 1 = lal_sample_token_filtered.  The scratch
 * buffers must hold n rounded up to 32 bytes.  Draws come from the process's
 * glibc rand() state, as in the server. */
REF_API int ref_tail_step(const float *hidden, int8_t *xq, uint8_t *ax,
                          float *logits, const int8_t *w, const float *sw,
                          int vocab, int n, float temperature, int top_k,
                          float rep_penalty, int *recent, int *n_recent,
                          int hist_cap, int n_threads, int variant) {
    float sx = lal_quantize_x_int8(hidden, xq, n);
    lal_compute_abs_xq(xq, ax, n);
    ref_lm_head_omp(logits, xq, ax, sx, w, sw, vocab, n, n_threads);
    int next = variant == 0
        ? ref_sample_token(logits, vocab, temperature, top_k, rep_penalty, recent, *n_recent)
        : ref_sample_token_filtered(logits, vocab, temperature, top_k, rep_penalty,
                                    recent, *n_recent);
    if (next < 0) return next;
    if (*n_recent < hist_cap) recent[(*n_recent)++] = next;
    else { memmove(recent, recent + 1, (size_t)(hist_cap - 1) * sizeof(int)); recent[hist_cap - 1] = next; }
    return next;
}
