/*
 * lal_oracle.h -- CPU restatement of the LAL decode tail.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library, and only as the checker.
 * The product (lal_b200/liblal_tail.so) never links, loads or calls it.
 *
 * Every function restates one reference function; the citation names the file
 * and lines (paths relative to the samaidev/lal project root).  Parity of this
 * restatement with the reference itself is pinned by tests/test_oracle.py,
 * which runs the reference's own C (compiled by oracle/Makefile into
 * oracle/_ref/liblal_ref.so) on the same inputs, and by the golden vectors in
 * tests/golden/ that tests/golden/make_golden.py produced from that build.
 */
#ifndef LAL_ORACLE_H
#define LAL_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Intermediates of one sampling call, reported so tests can compare them. */
typedef struct {
    float threshold;   /* k-th largest penalised logit (min-heap root)   */
    float max_l;       /* max over candidates, floored at -1e30f          */
    float sum;         /* sequential sum of expf((l-max_l)/T), ascending v */
    float r;           /* u * sum                                          */
    int   n_cand;      /* |{v : l[v] >= threshold}|                        */
    int   greedy;      /* 1 when the argmax path was taken                 */
    int   drew;        /* 1 when the reference would have called rand()    */
} orc_sample_info;

/* runtime/lal_simd_optim.h:32-58 (AVX2+FMA build): the final RMSNorm,
 * tools/server/qwen7b_server.c:820; n a multiple of 8. */
void  orc_rms_norm(float *out, const float *x, const float *w, int n, float eps);
/* tools/server/gpt2_server.c:1982-1998: the GPT-2 server's quantizer
 * (truncation for every element). */
float orc_gpt2_quantize_x(const float *x, int8_t *xq, int n);
/* gpt2_server.c:2125-2214 (AVX2 build, n a multiple of 8): int8 logits of all
 * V rows, then the rows its 512-entry min-heap keeps re-scored in float.
 * kept (may be NULL) receives the kept rows in heap order; returns their
 * count. */
int   orc_gpt2_lm_head(float *logits, const float *x, const int8_t *wte_q,
                       const float *scale_w, int vocab_size, int n, int *kept);
/* gpt2_server.c:2862-3013 with top-p off and no filter: returns the token;
 * u = (float)(rand() % 1000000) / 1000000.0f. */
int   orc_gpt2_sample(float *logits, int vocab_size, float temperature, int top_k,
                      float rep_penalty, const int *recent, int n_recent, float u,
                      orc_sample_info *info);
/* with the server's top-p branch (gpt2_server.c:2895-2960); top_p outside
 * (0, 1) keeps every row of the top-k pool */
int   orc_gpt2_sample_p(float *logits, int vocab_size, float temperature, int top_k,
                        float top_p, float rep_penalty, const int *recent, int n_recent,
                        float u, orc_sample_info *info);
/* runtime/lal_q8_kernel.h:375-424 (AVX2+FMA build, the one the servers use). */
float orc_quantize_x_int8(const float *x, int8_t *xq, int n);
/* runtime/lal_q8_kernel.h:450-460 */
void  orc_compute_abs_xq(const int8_t *xq, uint8_t *ax, int n);
/* runtime/lal_q8_kernel.h:463-499 (also :506-543 and :551-640: same values) */
void  orc_lm_head_int8_range(float *logits, const int8_t *xq, float scale_x,
                             const int8_t *wte_q, const float *scale_w,
                             int v_start, int v_end, int n_embd);
/* logits[b][v] of n_vec quantized vectors xq[b][n_embd] (scales scale_x[b]) */
void  orc_lm_head_multi(float *logits, const int8_t *xq, const float *scale_x,
                        const int8_t *wte_q, const float *scale_w, int vocab, int n_embd,
                        int n_vec);
/* runtime/lal_q8_kernel.h:551-640: rows in full 8-row groups from v_start
 * sum only the first n_embd & ~31 columns (no scalar tail in :577-611). */
void  orc_lm_head_int8_range_abs_8row(float *logits, const int8_t *xq, float scale_x,
                                      const int8_t *wte_q, const float *scale_w,
                                      int v_start, int v_end, int n_embd);
/* Same, but also returns the exact int32 dot products for [v_start, v_end). */
void  orc_lm_head_dots(int32_t *dots, const int8_t *xq, const int8_t *wte_q,
                       int v_start, int v_end, int n_embd);
/* runtime/lal_q8_kernel.h:357-372 */
void  orc_quantize_q8_per_row(const float *W, int8_t *q8_T, float *scale,
                              int in_dim, int out_dim);
/* The same with a row stride (for quantizing a slice of a larger matrix). */
void  orc_quantize_q8_rows(const float *W, int8_t *q8_T, float *scale,
                           int in_dim, int n_rows);

/* runtime/lal_sampling.h:46-125, with the heap uncapped (capacity = k) and
 * the draw supplied as u = (float)rand()/(float)RAND_MAX (lal_sampling.h:116).
 * Mutates logits exactly as the reference does. */
int   orc_sample_token(float *logits, int vocab_size, float temperature,
                       int top_k, float rep_penalty, const int *recent,
                       int n_recent, float u, orc_sample_info *info);

/* tools/server/qwen7b_server.c:219-295 (lal_sample_token_filtered), heap
 * uncapped.  filter may be NULL (the weak no-op of qwen7b_server.c:179-186).
 * draw() is called exactly where the reference calls rand() (only when
 * sum > 0); it returns u.  decode is passed through to the filter. */
typedef int   (*orc_decode_fn)(int token_id, char *out_buf, int max_len);
typedef int   (*orc_filter_fn)(int *keep_mask, int n_vocab, int last_token,
                               const int *recent, int n_recent,
                               orc_decode_fn decode_fn);
typedef float (*orc_draw_fn)(void *ctx);
int   orc_sample_token_filtered(float *logits, int vocab_size, float temperature,
                                int top_k, float rep_penalty, const int *recent,
                                int n_recent, orc_filter_fn filter,
                                orc_decode_fn decode, orc_draw_fn draw,
                                void *draw_ctx, orc_sample_info *info);
int   orc_gpt2_sample_f(float *logits, int vocab_size, float temperature, int top_k,
                        float top_p, float rep_penalty, const int *recent, int n_recent,
                        orc_filter_fn filter, orc_decode_fn decode, float u,
                        orc_sample_info *info);

/* glibc expf element-wise (runtime/lal_sampling.h:112,120 call expf). */
void  orc_expf_batch(const float *x, float *y, long n);

/* runtime/lal_sampling.h:133-136 generalised to capacity cap (256 there). */
void  orc_recent_push(int *tokens, int *n, int cap, int tok);

/* One decode-tail step for one stream, the sequence of
 * tools/server/qwen7b_server.c:829-850: quantize, LM head over all rows,
 * sample (variant 0 = lal_sample_token, 1 = the server's filtered sampler
 * with no filter loaded), push into the history.  Returns the token. */
int   orc_tail_step(const float *hidden, int n_embd, const int8_t *wte_q,
                    const float *scale_w, int vocab_size, float temperature,
                    int top_k, float rep_penalty, int *recent, int *n_recent,
                    int hist_cap, float u, int variant, float *logits_out,
                    orc_sample_info *info);

#ifdef __cplusplus
}
#endif
#endif
