/*
 * lal_tail.h -- C ABI of liblal_tail.so, the B200 (sm_100a) decode tail of LAL.
 *
 * The decode tail is the end of every forward() in the LAL servers
 * (tools/server/qwen7b_server.c:819-851): quantize the final hidden vector to
 * int8, contract it with the per-row-scaled int8 LM head, apply the
 * repetition penalty, then top-k select, softmax with temperature, draw.
 *
 * Two layers are exported, both plain C: host pointers, sizes, int status.
 *
 *  1. Drop-ins.  The functions the reference defines as static inline in
 *     runtime/lal_q8_kernel.h and runtime/lal_sampling.h, with the same names
 *     and signatures, computed on the GPU (declared in include/runtime/, the
 *     drop-in copies of those headers), and their status-returning lal_tail_*
 *     forms below.  Host pointers in and out; the sampler mutates logits in
 *     place and consumes glibc rand() exactly where the reference does.  The
 *     reference-named forms have no error channel (the originals return void
 *     or a token): on failure they print the reason to stderr and abort().
 *     There is no CPU fallback.
 *
 *  2. The fused decode tail (lal_tail_*): one context per GPU holding its
 *     vocab slice of the LM head in HBM, the per-stream penalty histories and
 *     sampling parameters; lal_tail_step() takes B hidden vectors and B draws
 *     and returns B token ids, in one kernel per step.  Multi-GPU contexts
 *     each own a contiguous vocab slice and merge the per-slice top-k
 *     candidates across GPUs.
 *
 * Every lal_tail_* function returns LAL_TAIL_OK (0) or an error code;
 * lal_tail_last_error() gives the calling thread's last message.
 */
#ifndef LAL_TAIL_H
#define LAL_TAIL_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LAL_TAIL_OK              0
#define LAL_TAIL_ERR_ARG         1   /* bad argument or size                  */
#define LAL_TAIL_ERR_CUDA        2   /* CUDA runtime error                    */
#define LAL_TAIL_ERR_NOMEM       3   /* device or pinned allocation failed    */
#define LAL_TAIL_ERR_TIMEOUT     4   /* a bounded device wait ran out         */
#define LAL_TAIL_ERR_CAPACITY    5   /* tie set or list above the built limit */
#define LAL_TAIL_ERR_STATE       6   /* call out of order (e.g. no LM head)   */
#define LAL_TAIL_ERR_COMM        7   /* multi-GPU exchange failed             */
#define LAL_TAIL_ERR_UNSUPPORTED 8   /* shape outside what the kernels handle */

/* Sampler semantics.  LIBRARY = runtime/lal_sampling.h:46-125 (greedy check
 * before the penalty).  SERVER = tools/server/qwen7b_server.c:219-295
 * (penalty first, k clamped to [1,V], argmax fallback when the kept softmax
 * mass is not positive). */
#define LAL_SAMPLER_LIBRARY 0
#define LAL_SAMPLER_SERVER  1
/* GPT2 = the GPT-2 server's int8 LM head and sampler, a second drop-in for
 * lm_head_int8_parallel (tools/server/gpt2_server.c:2125-2214) and its
 * sampling block (gpt2_server.c:2862-3013; top-p with lal_tail_set_top_p,
 * the level-2 filter call with lal_tail_set_filter):
 * truncating quantizer, int8 logits of every row, the 512 rows the server's
 * min-heap keeps re-scored in float, then LIBRARY's arithmetic on the
 * re-scored logits, except that a draw of exactly 0 returns row 0.  u[b] is
 * the caller's (float)(rand() % 1000000) / 1000000.0f.  One shard, n_embd a
 * multiple of 8, vocab_size <= 51200 (the select holds the vocab's logits in
 * one CTA's shared memory); lal_tail_get_logits returns the re-scored, penalised
 * logits (the server's g_logits after the step). */
#define LAL_SAMPLER_GPT2    2

/* The calling thread's last error message ("" if none). */
const char *lal_tail_last_error(void);
/* Library version and build string. */
const char *lal_tail_version(void);

/* ======================================================================
 * 1. Status-returning forms of the drop-ins
 *
 * The functions with the reference's own names (lal_quantize_x_int8,
 * lal_lm_head_int8_range, lal_sample_token, ...) are exported by the same
 * library and declared in include/runtime/lal_q8_kernel.h and
 * include/runtime/lal_sampling.h, the drop-in copies of the reference
 * headers.  This header declares only lal_tail_* names, so it can be
 * included next to the reference's original headers.
 * ====================================================================== */


/* Level-2 filter hook types (tools/server/qwen7b_server.c:175-186). */
typedef int (*lal_token_decode_fn)(int token_id, char *out_buf, int max_len);
typedef int (*lal_filter_topk_fn)(int *keep_mask, int n_vocab, int last_token,
                                  const int *recent_tokens, int n_recent,
                                  lal_token_decode_fn decode_fn);
/* A draw source: returns u = (float)rand()/(float)RAND_MAX or equivalent. */
typedef float (*lal_draw_fn)(void *ctx);

int lal_tail_quantize_x_int8(const float *x, int8_t *xq, int n, float *scale_out);
int lal_tail_compute_abs_xq(const int8_t *xq, uint8_t *ax, int n);
int lal_tail_lm_head_int8_range(float *logits, const int8_t *xq, float scale_x,
                                const int8_t *wte_q, const float *scale_w,
                                int v_start, int v_end, int n_embd);
int lal_tail_quantize_q8_per_row(const float *W, int8_t *q8_T, float *scale,
                                 int in_dim, int out_dim);
/* lal_sample_token with the draw u supplied (used only on the non-greedy
 * path).  Writes the token to *token_out and mutates logits like the
 * reference. */
int lal_tail_sample_token(float *logits, int vocab_size, float temperature,
                          int top_k, float rep_penalty, const int *recent,
                          int n_recent, float u, int *token_out);
/* tools/server/qwen7b_server.c:219-295 (lal_sample_token_filtered), with the
 * level-2 filter hook: filter (may be NULL) sees the top-k keep_mask on the
 * host; draw() is called exactly where the reference calls rand() (only when
 * the kept softmax mass is positive).  decode is handed to the filter. */
int lal_tail_sample_token_filtered(float *logits, int vocab_size, float temperature,
                                   int top_k, float rep_penalty, const int *recent,
                                   int n_recent, lal_filter_topk_fn filter,
                                   lal_token_decode_fn decode, lal_draw_fn draw,
                                   void *draw_ctx, int *token_out);
/* lal_sample_token on logits already in device memory, allocating nothing
 * (no counterpart in the reference, whose sampler runs on the host).  For
 * callers that must not allocate device memory inside their decode loop:
 * all working memory is a fixed static device region (2.1 MB of scratch +
 * 3.1 MB for the expf table), so vocab_size <= 262144; larger sizes return
 * LAL_TAIL_ERR_ARG.  d_logits [vocab_size] is penalised in place like the
 * reference's logits; d_recent [n_recent] are device ids; u is the draw
 * (used only on the non-greedy path); stream is a cudaStream_t (NULL = the
 * legacy default stream); the call waits for its stream and writes the token
 * to *token_out.  The first call on a device does the set-up with that device
 * current: make it before any stream capture.  Calls that overlap on one
 * device share the scratch and race: serialise them. */
int lal_tail_sample_token_noalloc(float *d_logits, int vocab_size, float temperature,
                                  int top_k, float rep_penalty, const int *d_recent,
                                  int n_recent, float u, void *stream, int *token_out);
/* Register (copy to the device) or drop a host LM head used by the range
 * drop-ins.  Registration is optional: first use registers on demand. */
int lal_tail_lm_head_register(const int8_t *wte_q, const float *scale_w,
                              int vocab_size, int n_embd);
int lal_tail_lm_head_forget(const int8_t *wte_q);

/* ======================================================================
 * 2. Fused decode tail
 * ====================================================================== */

typedef struct lal_tail lal_tail;

typedef struct {
    int vocab_size;    /* V: the whole vocabulary (all slices)              */
    int n_embd;        /* d                                                 */
    int max_streams;   /* B capacity                                        */
    int max_top_k;     /* largest top_k a step will use                     */
    int history_cap;   /* per-stream penalty-history capacity (server: 256) */
    int sampler;       /* LAL_SAMPLER_LIBRARY, _SERVER or _GPT2             */
    int device;        /* CUDA device ordinal; -1 = the current device      */
    int shard_rank;    /* this context owns vocab rows                      */
    int shard_count;   /*   [rank*V/count, (rank+1)*V/count)                */
} lal_tail_config;

/* Per-stream outputs of the last step, for inspection and parity tests. */
typedef struct {
    float threshold;   /* k-th largest penalised logit                      */
    float max_l;       /* softmax max, floored at -1e30f                    */
    float sum;         /* sequential sum of the candidate weights           */
    float r;           /* u * sum                                           */
    int   n_cand;      /* candidates {v : l[v] >= threshold}                */
    int   greedy;      /* 1 if the argmax path was taken                    */
    int   drew;        /* 1 if the draw u was consumed                      */
    int   token;
} lal_tail_diag;

int lal_tail_create(const lal_tail_config *cfg, lal_tail **out);
int lal_tail_destroy(lal_tail *t);
/* This context's vocab slice: first row and row count. */
int lal_tail_shard_rows(const lal_tail *t, int *row0, int *n_rows);

/* Load this slice of the LM head: int8 rows [n_rows, n_embd] + fp32 scales,
 * from host memory. */
int lal_tail_load_lm_head_q8(lal_tail *t, const int8_t *wte_q_rows,
                             const float *scale_w_rows);
/* Load this slice from fp32 rows and quantize it on the GPU exactly as
 * lal_quantize_q8_per_row does (runtime/lal_q8_kernel.h:357-372).  rows may
 * be given in chunks: [row_begin, row_begin + n) of the slice. */
int lal_tail_load_lm_head_f32(lal_tail *t, const float *W_rows, int row_begin,
                              int n_rows);
/* GPQ8 weight files (the Qwen-7B server's format, tools/server/
 * qwen7b_server.c:499-563).  lal_tail_gpq8_find locates a tensor in a GPQ8
 * blob (host memory, e.g. an mmap of the file) without touching the GPU;
 * offsets are from the start of the blob.  lal_tail_load_lm_head_gpq8 loads
 * this context's slice of the [vocab_size, n_embd] tensor `key` (NULL =
 * "lm_head.weight"): an F32 tensor is quantized on the GPU exactly as
 * lal_quantize_q8_per_row does at the server's load, a Q8 tensor (per-row
 * scales) is copied as it is. */
typedef struct {
    int ndim;
    int shape[4];
    int qtype;              /* 0 = F32, 1 = Q8                                   */
    uint64_t data_offset;
    uint64_t data_len;
    int n_scale;
    uint64_t scale_offset;
} lal_gpq8_tensor;
int lal_tail_gpq8_find(const void *blob, size_t size, const char *key, lal_gpq8_tensor *out);
int lal_tail_load_lm_head_gpq8(lal_tail *t, const void *blob, size_t size, const char *key);

/* Read back this slice's quantized LM head (n_rows x n_embd, and scales). */
int lal_tail_read_lm_head(lal_tail *t, int8_t *wte_q_rows, float *scale_w_rows);

/* Per-stream sampling parameters (host arrays of n_streams). */
int lal_tail_set_sampling(lal_tail *t, int n_streams, const float *temperature,
                          const int *top_k, const float *rep_penalty);
/* Replace one stream's penalty history (oldest first; n <= history_cap). */
int lal_tail_set_history(lal_tail *t, int stream, const int *recent, int n_recent);
/* Read one stream's history, oldest first; *n_out receives its length. */
int lal_tail_get_history(lal_tail *t, int stream, int *recent_out, int *n_out);

/* One decode-tail step for n_streams streams.  hidden: host [n_streams,
 * n_embd] fp32; u: host [n_streams] draws (read only for non-greedy
 * streams); tokens_out: host [n_streams].  Each sampled token is appended to
 * its stream's history (FIFO at history_cap, runtime/lal_sampling.h:133-136). */
int lal_tail_step(lal_tail *t, const float *hidden, int n_streams, const float *u,
                  int *tokens_out);
/* The same with device pointers, enqueued on the context's stream without a
 * host synchronisation (tokens land in d_tokens_out). */
int lal_tail_step_device(lal_tail *t, const float *d_hidden, int n_streams,
                         const float *d_u, int *d_tokens_out);
/* Wait for the context's stream; returns a device-side error if one was
 * recorded (e.g. LAL_TAIL_ERR_TIMEOUT). */
int lal_tail_sync(lal_tail *t);

/* Host staging of one step's inputs (pinned copy, then one H2D into the
 * context's device buffers, see lal_tail_device_buffers) and the matching
 * read of the tokens (D2H + wait + status check).  lal_tail_step is
 * stage_inputs + the step on the device buffers + fetch_tokens for GPT-2
 * sampler contexts and for shards that are not peer-connected; otherwise
 * (unsharded, or one stream on peer-connected shards) a small kernel pulls
 * the inputs from mapped pinned memory and the token comes back in a mapped
 * completion word that the calling thread waits on. */
int lal_tail_stage_inputs(lal_tail *t, const float *hidden, int n_streams, const float *u);
int lal_tail_fetch_tokens(lal_tail *t, int n_streams, int *tokens_out);

/* Vocab-sharded step (shard_count > 1; no counterpart in the reference,
 * which samples from one process).  Per step, on every rank, in order on the
 * context's stream:
 *   1. lal_tail_shard_select: the fused kernel over this rank's slice writes,
 *      per stream, a candidate record (its tie-complete local top-k set, in
 *      ascending vocab order; when the set outgrows the record, its rows
 *      above the slice's threshold plus a bitmap of the rows tied at it)
 *      into the send buffer;
 *   2. the caller all-gathers bytes_per_rank bytes of the send buffer of
 *      every rank into the receive buffer, in rank order, on the context's
 *      stream (ncclAllGather or any equivalent);
 *   3. lal_tail_shard_merge: every rank merges the same records and draws
 *      the same token (the unsharded step's result, bit for bit), pushes it
 *      into its history copy and writes d_tokens_out.
 * A failing shard (status in its record) fails the step on every rank. */
int lal_tail_shard_select(lal_tail *t, const float *d_hidden, int n_streams);
/* Peer exchange (single-stream steps, one process per GPU): every rank
 * exports the IPC handle of its receive buffer, gathers all ranks' handles
 * (rank order) and connects; afterwards lal_tail_step / lal_tail_step_device
 * with one stream run the whole sharded step in one kernel per rank: the last
 * CTA writes its record into every rank's buffer over NVLink (plain stores),
 * waits -- bounded, LAL_TAIL_ERR_TIMEOUT after 2 s -- for every rank's
 * record of the step, merges them and draws.  Every rank must step in
 * lockstep (the step's sequence number is counted per context; connecting
 * again restarts it).  lal_tail_exchange_handle clears the receive buffer
 * before the handle is returned, so every rank must have exported its handle
 * before any rank steps (gathering the handles is that point); connecting
 * does not clear it again. */
#define LAL_TAIL_IPC_HANDLE_BYTES 64
int lal_tail_exchange_handle(lal_tail *t, void *handle_out);
int lal_tail_connect_peers(lal_tail *t, const void *handles);
int lal_tail_disconnect_peers(lal_tail *t);
int lal_tail_exchange_buffers(lal_tail *t, int n_streams, void **d_send, void **d_recv,
                              size_t *bytes_per_rank);
int lal_tail_shard_merge(lal_tail *t, int n_streams, const float *d_u, int *d_tokens_out);
/* Level-2 filter hook in the fused context (tools/server/qwen7b_server.c:
 * 175-186, 257-270).  With a filter or a draw callback set, lal_tail_step
 * samples each non-greedy stream as the server's lal_sample_token_filtered:
 * the fused kernel selects the candidates, the host builds the keep mask and
 * calls filter (restoring the mask if it comes back empty), the GPU finishes
 * the kept softmax, and draw(draw_ctx) is called only when the kept mass is
 * positive (with no draw callback, the step's u[b] is used there).  Greedy
 * streams take the normal path.  Needs LAL_SAMPLER_SERVER or LAL_SAMPLER_GPT2
 * and one shard; lal_tail_step_device is not filtered.  All NULL switches it
 * off.  With LAL_SAMPLER_GPT2 it is the GPT-2 server's call
 * (tools/server/gpt2_server.c:2962-2978): the mask holds the top-k pool
 * narrowed by top-p, an empty mask gets the whole top-k pool back, the
 * softmax runs over every row the mask keeps (rows the filter adds too), and
 * the draw is taken every non-greedy step. */
int lal_tail_set_filter(lal_tail *t, lal_filter_topk_fn filter, lal_token_decode_fn decode,
                        lal_draw_fn draw, void *draw_ctx);
/* The model's final RMSNorm fused as the tail's prologue: replaces
 * qwen7b_rms_norm(g_ln, g_x, g_norm_f_w, N_EMBD) at
 * tools/server/qwen7b_server.c:820 (runtime/lal_simd_optim.h:32-58, the AVX2
 * build; eps RMS_EPS = 1e-6f there).  With norm_w set (n_embd floats, copied
 * to the device), every later step's hidden input is the residual stream x,
 * and the step quantizes (x * inv_rms) * w with the reference's exact sum
 * order instead of the hidden itself; the per-stream, batched and sharded
 * steps all apply it.  NULL switches it off.  n_embd <= 4096 and a multiple of 8
 * (the reference's scalar tail loop, whose rounding its compiler decides, is
 * then empty; LAL_TAIL_ERR_UNSUPPORTED otherwise). */
int lal_tail_set_final_norm(lal_tail *t, const float *norm_w, float eps);
/* The GPT-2 server's nucleus (top-p) step, applied after top-k and before
 * the softmax (tools/server/gpt2_server.c:2895-2960, its --top-p; 0 = off,
 * the server's default, :2343): the top-k pool's temperature softmax,
 * sorted by descending probability (ties by ascending row), keeps rows until
 * the running probability reaches top_p.  Values are clamped to [0, 1] as
 * the server clamps them (:3147-3148).  Only LAL_SAMPLER_GPT2 contexts. */
int lal_tail_set_top_p(lal_tail *t, float top_p);
/* How a step of n_streams streams runs on this context (no counterpart in
 * the reference): one fused launch per stream, the batched tensor-core step
 * (quantize, one tcgen05 GEMM pass over the LM head for every stream, a
 * select CTA per stream), or the GPT-2 server's tail.  A batched shape whose
 * select does not fit shared memory falls back to the per-stream launches.
 * Returns the kind, or minus an LAL_TAIL_ERR_* code. */
#define LAL_TAIL_STEP_PER_STREAM 0
#define LAL_TAIL_STEP_BATCHED 1
#define LAL_TAIL_STEP_GPT2 2
int lal_tail_step_kind(lal_tail *t, int n_streams);
/* Measurement aid (no counterpart in the reference): keep `copies` identical
 * device copies of this slice's LM head and row scales (the loaded one and
 * copies - 1 duplicates) and let the single-stream steps use them in turn,
 * one per step.  A slice smaller than the GPU's L2 cache (the Qwen head split
 * 4 or 8 ways is 136 or 68 MB against 126 MB of L2) is then read from HBM at
 * every step, as a full-size head is, so steps can be timed back to back.
 * Results do not change.  1 drops the duplicates; loading an LM head drops
 * them too.  Batched (B >= 2) steps always read the loaded copy. */
int lal_tail_set_lm_head_copies(lal_tail *t, int copies);
/* Diagnostics and penalised logits (this slice's rows) of the last step. */
int lal_tail_get_diag(lal_tail *t, int stream, lal_tail_diag *out);
int lal_tail_get_logits(lal_tail *t, int stream, float *logits_rows);
/* Device buffers of the context, for callers that keep inputs on the GPU. */
int lal_tail_device_buffers(lal_tail *t, float **d_hidden, float **d_u,
                            int **d_tokens);
/* The context's CUDA stream (a cudaStream_t), for callers that order their
 * own work or timing events with the tail's launches. */
int lal_tail_get_stream(lal_tail *t, void **stream);
/* Turn on (1) or off (0) CUDA-event timing of each step's dominant kernel:
 * the fused kernel of a single-stream step (one launch per stream), or the
 * tensor-core GEMM of a batched step (B >= 2 streams). */
int lal_tail_set_timing(lal_tail *t, int on);
/* Average duration in milliseconds of that kernel over the launches since
 * the last call (CUDA events on the context's stream), and their count. */
int lal_tail_kernel_time(lal_tail *t, double *avg_ms, int *n_launches);

/* Phase timing of the fused kernel (inspection hook).  When on, every launch
 * writes globaltimer stamps (ns): per CTA c, out[c*8 + 0..7] = start,
 * prologue done, rows done, the previous kernel complete (small-k select) or
 * histogram levels 0/1/2 merged (grid select), -, -, -, arrival at the final
 * ticket; for the last CTA, out[grid*8 + 0..7] = select start, CTA bound,
 * superset, threshold, candidates in vocab order, (peer exchange) record
 * published, every rank's record arrived, token written; and for the peer
 * exchange's merge, out[(grid+1)*8 + 0..4] = maximum, threshold, candidates,
 * sum, draw.  read copies the last launch's (grid+2)*8 stamps. */
int lal_tail_debug_phases(lal_tail *t, int on);
int lal_tail_debug_phase_read(lal_tail *t, unsigned long long *out, int cap, int *grid);

/* Glibc-exact expf as the device computes it (test hook). */
int lal_tail_debug_expf(const float *x, float *y, int n);

#ifdef __cplusplus
}
#endif
#endif /* LAL_TAIL_H */
