/*
 * tail_internal.h -- structures shared by the sm_100a kernels (tail_kernels.cu)
 * and the C-ABI implementation (tail_api.cu).  Not installed.
 */
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace lal {

/* Block shape of the streaming kernel: 8 consumer warps (dp4a) + 1 TMA
 * producer warp. */
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxStages = 8;
/* stages the fused kernel's producer issues before waiting for the previous
 * kernel on the stream (programmatic dependent launch), unless a CTA's slice
 * is short enough that it prefetches its whole ring (plan_launch) */
constexpr int kEarlyStages = 2;
/* Largest grid (one CTA per SM on B200 is 148). */
constexpr int kMaxGrid = 256;
/* Global key histogram of the threshold search: level 0 = the top 12 bits
 * of the order key, levels 1 and 2 = the next 10 + 10 bits, used only while
 * the boundary bin holds more than kRefineMax keys. */
constexpr int kHistWords = 4096 + 1024 + 1024;
constexpr int kRefineMax = 2048;
/* Small-k select: per-CTA slot of the sorted local superset; the strategy is
 * used only for k <= kLocalMaxK (and 2k <= the rows of a CTA: each CTA's own
 * boundary then bounds T usefully; correctness never depends on it). */
/* the longest hidden vector the fused final RMSNorm accepts (it holds the
 * vector in the consumer warps' registers, 16 values a thread) */
constexpr int kNormMaxD = 4096;
constexpr int kSlot = 128;
constexpr int kLocalMaxK = 64;
/* Each CTA also publishes a 48-byte head record {max key, slot count, the
 * slot's last kept key when its tail was dropped (else 0), -, the slot's
 * first 4 keys, their 4 vocab ids} at kSlotHeads words into the
 * superset buffer, so the last CTA reads three 16-byte vectors per CTA. */
constexpr int kSlotHeads = kMaxGrid * kSlot;
constexpr int kSlotHeadWords = 12;
constexpr int kSelectCapMin = kSlotHeads + kMaxGrid * kSlotHeadWords;
/* words of the expf exception bitmap: bit (b >> 8) for b = bits(x) - 2^31,
 * x from -0 down to -inf (0x7F800000 >> 8 buckets) */
constexpr int kExpfBitmapWords = ((0x7F800000u >> 8) >> 5) + 1;
/* The fix-up table as an open-addressed hash: kExpfHashPairs 16-byte buckets
 * of two (x bits, y bits) slots, linear probing by bucket from
 * expf_hash_bucket(x); key 0 (never a fix-up input, all of which are
 * negative) marks an empty slot.  One aligned 16-byte load resolves most
 * lookups, and its address depends on x alone. */
constexpr unsigned kExpfHashPairs = 1u << 18;
__host__ __device__ inline unsigned expf_hash_bucket(uint32_t xb) {
    return ((xb * 2654435761u) >> 13) & (kExpfHashPairs - 1u);
}
/* Largest per-CTA row slice (smem holds its logits, scales, penalty counts). */
constexpr int kMaxRowsPerCta = 4096;
/* Largest shard count of a vocab-sharded context. */
constexpr int kMaxRanks = 64;

enum Mode : int { MODE_FUSED = 0, MODE_LMHEAD = 1, MODE_SAMPLE = 2 };
/* LIBRARY: runtime/lal_sampling.h; SERVER: qwen7b_server.c's
 * lal_sample_token_filtered; GPT2: gpt2_server.c's sampler (LIBRARY's
 * arithmetic; a draw of r == 0 returns row 0) */
enum Variant : int { VARIANT_LIBRARY = 0, VARIANT_SERVER = 1, VARIANT_GPT2 = 2 };
/* rows the GPT-2 server re-scores in float (gpt2_server.c:2123) */
constexpr int kGpt2RerankN = 512;
/* the GPT-2 tail's select holds the vocab's keys in one CTA's shared memory */
constexpr int kGpt2SelThreads = 1024;
constexpr int kGpt2MaxV = 51200;

/* Device status word values (mirrors LAL_TAIL_ERR_* in include/lal_tail.h).
 * DEV_CAPACITY remains for a merge whose gathered entries exceed the
 * capacity it was built with (the selects and the merge otherwise take the
 * wide path, tail_wide.cuh). */
enum DevStatus : int { DEV_OK = 0, DEV_TIMEOUT = 4, DEV_CAPACITY = 5 };

/* Per-stream outputs of a sampling launch (same layout as lal_tail_diag). */
struct StreamDiag {
    float threshold, max_l, sum, r;
    int n_cand, greedy, drew, token;
};

/* The GPT-2 tail's re-score launch: its last CTA runs the server's sampler
 * (tail_gpt2.cu). */
struct Gpt2Finish {
    float *logits; /* [V]: int8 logits, the re-scored rows written by the launch */
    int V;
    const int *cand;        /* the rows the heap kept, any order */
    float *kept_val;        /* their re-scored logits, in the same order */
    const int *n_ptr;       /* their count */
    const uint32_t *bound;  /* order key: every row left out has a logit <= it */
    const float *temperature, *rep_penalty, *u;
    const int *top_k;
    float top_p;
    int *hist_ids, *hist_n, *hist_head;
    int hist_cap, push_history;
    int *tokens;
    StreamDiag *diag;
    const uint32_t *expf_x, *expf_y, *expf_bits, *expf_off;
    const uint4 *expf_hash;
    int expf_hash_probe;
    int cap;      /* explicit rows of the wide path: >= the largest k */
    int h_slots;  /* history hash slots: a power of two >= 2 * hist_cap */
    unsigned *ticket;
    int *status;
    /* the level-2 filter hook's first half: no draw; the top-k pool {l >= T}
     * in ascending rows (values, rows, 1 where the top-p nucleus keeps the
     * row) and its size in diag->n_cand */
    int candidates_only;
    float *pool_val;
    int *pool_idx, *pool_keep;
    int pool_cap;
};

/* Vocab-sharded step: the candidate record one shard exports per stream.
 * A 32-byte header, then cap values and cap global vocab indices in
 * ascending index order, then a bitmap of the shard's rows.  Every global
 * candidate {l >= T} lies in its shard's set {l >= T_shard} (T >= T_shard,
 * T_shard the shard's own k-th largest penalised logit), so the union of the
 * records carries the whole step.  Two forms:
 *   - list form (ties == 0): the entries are the whole set {l >= T_shard};
 *   - wide form (ties > 0), when the set does not fit cap entries: the
 *     entries are the rows l > T_shard (fewer than k), and bit j of the
 *     bitmap marks local row j when its logit equals T_shard (`ties` rows;
 *     tkey is T_shard's order key). */
struct ShardRecordHead {
    int count;        /* entries in the record                                */
    int status;       /* DEV_* of the shard's launch (0 = ok)                 */
    unsigned seq;     /* step sequence number (peer exchange)                 */
    int ties;         /* 0: list form; else the rows equal to T_shard         */
    uint32_t tkey;    /* wide form: T_shard as an order key                   */
    int pad[3];
};
static_assert(sizeof(ShardRecordHead) == 32, "record header layout");
/* rows of the largest slice of a vocabulary split n ways */
inline int shard_rows_max(int vocab, int n) {
    int m = 0;
    for (int r = 0; r < n; ++r) {
        const int a = (int)((long long)r * vocab / n), b = (int)((long long)(r + 1) * vocab / n);
        if (b - a > m) m = b - a;
    }
    return m;
}
inline int shard_bitmap_words(int rows) { return (rows + 31) / 32; }
/* bytes of a gathered record (16-byte multiple) */
inline int shard_record_bytes(int cap, int rows_max) {
    return (32 + 8 * cap + 4 * shard_bitmap_words(rows_max) + 15) / 16 * 16;
}
/* bytes of a peer-exchange record: 64-bit words tagged with the step's
 * sequence number -- count, status, ties, T_shard key, then (value, vocab
 * index) per entry, then the bitmap words after cap entries; a 16-byte
 * multiple, so that every pair of words is one aligned 16-byte access */
inline int peer_record_bytes(int cap, int rows_max) {
    return (8 * (4 + 2 * cap + shard_bitmap_words(rows_max)) + 15) / 16 * 16;
}

/* Merge of the gathered records of one stream (one CTA per stream): the
 * records of stream b from rank r are at recv + (r * rank_stride +
 * b * rec_bytes). */
struct MergeParams {
    const uint8_t *recv;
    long long rank_stride;
    int rec_bytes, rec_cap, n_ranks;
    int vocab, variant;
    const float *temperature;
    const int *top_k;
    const float *u;
    int *hist_ids, *hist_n, *hist_head;
    int hist_cap, push_history;
    int *tokens;
    StreamDiag *diag;
    int *status;
    const uint32_t *expf_x, *expf_y;
    int expf_n;
    const uint32_t *expf_bits;
    const uint32_t *expf_off;
    const uint4 *expf_hash;   /* hash form of the fix-ups, or null            */
    int expf_hash_probe;
    int smem_cap;     /* candidates the CTA's shared memory holds             */
    /* optional globaltimer stamps of the merge's phases ([8], or null) */
    unsigned long long *phase_ts;
};

struct TailParams {
    int mode, variant;
    /* LM head slice: row-major [rows][ld] int8, ld % 16 == 0, zero padded. */
    const int8_t *W;
    const float *scale_w;
    int rows;          /* rows covered by this launch                        */
    int row_base;      /* vocab index of local row 0                         */
    int vocab;         /* the whole vocabulary V                             */
    int d, ld;
    /* inputs */
    const float *hidden;     /* FUSED: [B][d]                                 */
    /* FUSED: when set, hidden is the residual stream before the final RMSNorm
     * (weights norm_w [d], epsilon norm_eps), applied in the prologue */
    const float *norm_w;
    float norm_eps;
    const int8_t *xq_in;     /* LMHEAD: quantized vector [d]                  */
    float scale_x_in;        /* LMHEAD                                        */
    const float *scale_x_dev; /* LMHEAD: the scale in device memory, if set    */
    /* LMHEAD: local rows < trunc_rows_end sum only columns < trunc_cols (the
     * 8-row form's dropped tail, runtime/lal_q8_kernel.h:577-611); otherwise
     * trunc_cols = ld. */
    int trunc_cols, trunc_rows_end;
    float *logits;           /* [B][rows]: written (FUSED/LMHEAD), in/out (SAMPLE) */
    int B;
    const float *temperature;
    const int *top_k;
    const float *rep_penalty;
    const float *u;
    /* penalty history: ids[b*hist_cap + i] for i < hist_n[b] */
    int *hist_ids, *hist_n, *hist_head;
    int hist_cap;
    int push_history;
    /* outputs */
    int *tokens;
    StreamDiag *diag;
    /* scratch (global memory beyond inputs and outputs); every word returns
     * to zero (or, for the barrier generation, to a consistent value) by
     * the end of a launch */
    unsigned *ghist;         /* [kHistWords] global key histogram             */
    unsigned *gbar;          /* [2] grid barrier: arrivals, generation        */
    unsigned *gcount;        /* [1] superset entries appended                 */
    unsigned *gL;            /* [1] largest per-CTA boundary edge (small k)   */
    unsigned *gmax;          /* [kMaxGrid] each CTA's largest key (small k)   */
    unsigned *gslot_n;       /* [kMaxGrid] each CTA's slot count (small k)    */
    uint32_t *gcand_key;     /* [gcand_cap] superset {key >= boundary}        */
    int *gcand_idx;          /* [gcand_cap] their vocab indices               */
    int gcand_cap;
    unsigned int *counter;   /* [1] arrival tickets, self-resetting           */
    int *status;             /* device status word                            */
    /* optional export of the candidate set (ascending vocab order) */
    float *cand_val_out;
    int *cand_idx_out;
    int cand_out_cap;
    int candidates_only;     /* stop after exporting candidates (no draw)     */
    /* VARIANT_GPT2: the server's nucleus over the candidates when
     * 0 < top_p < 1 (gpt2_server.c:2908-2955), else off */
    float top_p;
    /* vocab-sharded step: write this stream's candidate record (status,
     * count, ascending-index list of at most rec_cap) and stop */
    uint8_t *shard_out;
    int rec_cap;
    /* vocab-sharded step with the peer exchange (one stream): the last CTA
     * writes its record into every rank's receive buffer peer_recv[r]
     * ([2 parities][n_ranks][rec_bytes], NVLink stores), publishes seq, waits
     * (bounded) for every rank's record of this step and merges them */
    uint8_t *const *peer_recv;
    int n_ranks, rank, rec_bytes;
    unsigned seq;
    /* glibc expf fix-ups; expf_bits has one bit per 256 consecutive negative
     * float bit patterns, set where the table holds an entry */
    const uint32_t *expf_x, *expf_y;
    int expf_n;
    const uint32_t *expf_bits;
    const uint32_t *expf_off; /* [words+1]: first table entry of each bitmap word */
    /* the same fix-ups as an open-addressed hash (null: use the bitmap) */
    const uint4 *expf_hash;
    int expf_hash_probe;     /* longest probe (buckets) of any table entry    */
    /* optional globaltimer stamps: [cta*8 + i] per CTA (start, prologue done,
     * rows done, list written) and [grid*8 + i] for the merge */
    unsigned long long *phase_ts;
    /* optional completion word in mapped pinned host memory: the step's token
     * (or -1) in the low half, the step's sequence number (*seq_in, device
     * memory, read after the previous kernel completes) in the high half */
    unsigned long long *host_tok;
    const unsigned *seq_in;
    /* shared-memory layout (bytes) */
    int stages, rows_per_stage, stage_bytes, area_bytes;
    int off_bars, off_xq, off_sw, off_lg, off_cnt, off_hist, off_misc, smem_total;
    int rows_per_cta_max;
    int early_stages;        /* stages streamed before griddepcontrol.wait    */
    int nch;                 /* 512-byte column chunks per row                */
    int max_k;               /* largest k a launch may use (planning)         */
    int local_edges;         /* select strategy (use_local_edges); 0 = grid
                              * histogram with grid barriers, which needs a
                              * cooperative launch                            */
};

/* Second half of the server sampler with a level-2 filter
 * (tools/server/qwen7b_server.c:271-294) over an exported candidate list:
 * phase 0 computes max, weights, running sums and the argmax fallback over
 * the kept candidates; phase 1 draws with u. */
struct FinishParams {
    const float *cand_val;   /* or null: the values are logits[cand_idx[i]]     */
    const float *logits;
    const int *cand_idx;
    const int *keep;         /* or null: every entry is kept                   */
    int variant;             /* VARIANT_GPT2: a draw of exactly 0 takes row 0   */
    int m;
    float temperature;
    int vocab;
    const float *u;
    float *prefix;           /* [m] scratch                                    */
    StreamDiag *diag;
    int *token;
    int phase;
    const uint32_t *expf_x, *expf_y;
    int expf_n;
    const uint32_t *expf_bits;
    const uint32_t *expf_off;
};

/* The select strategy of a launch whose effective k (greedy: 1; else
 * min(top_k, V, rows)) is k: per-CTA histogram edges (no grid barrier) when k
 * is small against a CTA's slice, else the grid-wide histogram. */
inline int use_local_edges(int k, int rows_per_cta_max) {
    return k <= kLocalMaxK && 2 * k <= rows_per_cta_max;
}
inline int effective_k(float temperature, int top_k, int vocab, int rows) {
    int k = (temperature <= 0.0f || top_k <= 0) ? 1 : top_k;
    if (k > vocab) k = vocab;
    if (k > rows) k = rows;
    return k < 1 ? 1 : k;
}

/* Host-side launchers (tail_kernels.cu). */
cudaError_t launch_finish(const FinishParams &f, cudaStream_t st);
cudaError_t launch_merge(const MergeParams &m, int n_streams, cudaStream_t st);
/* candidates a merge CTA can hold (the gathered records of one stream), or
 * -1 when n_candidates_max does not fit in shared memory */
int merge_smem_cap(int n_candidates_max);
/* candidates the fused kernel's last CTA can merge in the peer exchange */
int peer_merge_cap(const TailParams &p);

/* Allocation-free sampler entry (tail_noalloc.cu): build the expf bitmap and
 * offset index from a device copy of the sorted fix-up table (kernels, no
 * host buffers); raise the SAMPLE kernel's shared-memory limit once; launch
 * the SAMPLE kernel with that limit already raised. */
cudaError_t launch_expf_index(const uint32_t *tx, int n, uint32_t *bits, uint32_t *off,
                              cudaStream_t st);
cudaError_t prepare_sample_kernel();
cudaError_t launch_sample_prepared(const TailParams &p, int grid, cudaStream_t st);
/* Records the calling thread's last error message (tail_api.cu). */
int set_error(int code, const char *msg);
/* Raise a kernel's dynamic shared-memory limit once per (device, kernel). */
cudaError_t raise_smem(const void *fn, int bytes);

/* Batched step (tail_batch.cu): B >= 2 streams share one pass over W on the
 * tensor cores.  BatchPlan is per context (W, the quantized-vector buffer,
 * cached TMA descriptors); BatchStep is per launch. */
struct BatchPlan {
    const int8_t *W;
    const float *scale_w;
    int rows, ld, num_sms, kblocks;
    int8_t *xq;        /* [256][ld] quantized hidden vectors                     */
    float *sx;         /* [256] their scales                                     */
    uint32_t *gmax;    /* [256][n_groups] raw maxima of 32-row groups, per stream */
    int n_groups;
    int s_cap, c_cap, h_slots;
    int wide_cap; /* explicit rows of the select's wide path */
    /* candidate groups the select stages a round when a step has more
     * streams than SMs (0 = not chosen yet): the smaller round that lets two
     * select CTAs share an SM, when they fit */
    int stage_groups_many;
    /* TMA descriptors (CUtensorMap, 128 bytes each): W, and X for N = 32..256 */
    alignas(64) unsigned char tm_w[128];
    alignas(64) unsigned char tm_x[8][128];
    unsigned x_ready;
    int w_ready;
    /* the GEMM's split tiles (those left over after its last whole wave):
     * int32 partial dots [rem][chunks][N][128] of a launch, or null */
    int *split_part;
    int split_rem;
    size_t split_ints;
};
struct BatchStep {
    const float *hidden;
    const float *norm_w; /* the final RMSNorm first, when set */
    float norm_eps;
    int d, B;
    float *logits; /* [B][rows] */
    int row_base, vocab, variant;
    const float *temperature;
    const int *top_k;
    const float *rep_penalty;
    const float *u;
    int *hist_ids, *hist_n, *hist_head;
    int hist_cap, hist_stride, push_history;
    int *tokens;
    StreamDiag *diag;
    int *status;
    const uint32_t *expf_x, *expf_y;
    int expf_n;
    const uint32_t *expf_bits;
    const uint32_t *expf_off;
    uint8_t *shard_out; /* per-stream records (vocab-sharded select), or null */
    int rec_cap, rec_bytes;
    cudaEvent_t gemm_ev0, gemm_ev1; /* optional: recorded around the GEMM launch */
    /* optional per-stream completion words in mapped host memory (TailParams) */
    unsigned long long *host_tok;
    const unsigned *seq_in;
};
/* 0 when the shape takes the batched path (d >= 128, 2 <= max_B <= 256). */
int batch_plan(BatchPlan &bp, const int8_t *W, const float *scale_w, int rows, int ld,
               int num_sms, int8_t *xq, float *sx, uint32_t *gmax, int *split_scratch,
               int max_B, int hist_cap, int max_top_k);
/* bytes of the GEMM's split scratch for this shape and up to max_B streams
 * (0: no tile is split); each launch writes what it reads */
size_t batch_split_bytes(int rows, int ld, int num_sms, int max_B);
/* 32-row groups of a slice of `rows` rows (the gmax buffer holds 256 streams of them) */
inline int batch_groups(int rows) { return (rows + 127) / 128 * 4; }
cudaError_t batch_launch(BatchPlan &bp, const BatchStep &s, cudaStream_t st);
int plan_launch(TailParams &p, int num_sms, int min_rows_per_cta);
cudaError_t launch_tail(const TailParams &p, int grid, cudaStream_t st);
cudaError_t launch_gpt2_select(const float *logits, int V, int N, int *cand_out, int *n_out,
                               uint32_t *bound_out, int *status, cudaStream_t st);
/* the re-score of the kept rows, then the sampler in the launch's last CTA */
cudaError_t launch_gpt2_rerank(const float *x, int d, const int8_t *W, int ld, const float *sw,
                               const Gpt2Finish &f, int N, cudaStream_t st);
size_t gpt2_finish_smem(int cap, int h_slots);
cudaError_t launch_quantize_x(const float *x, int8_t *xq, float *scale, int n,
                              cudaStream_t st);
/* One step's inputs from mapped pinned host memory into device memory: words
 * [0, n0) and [off1, off1 + n1) of src to the same offsets of dst, by one
 * small kernel that lets the next kernel on the stream launch at once
 * (programmatic dependent launch). */
cudaError_t launch_stage_inputs(const float *src, float *dst, int n0, int off1, int n1,
                                cudaStream_t st);
cudaError_t launch_abs_xq(const int8_t *xq, uint8_t *ax, int n, cudaStream_t st);
cudaError_t launch_quantize_rows(const float *W, int d, int8_t *q, int ld,
                                 float *scale, int n_rows, cudaStream_t st);
cudaError_t launch_debug_expf(const float *x, float *y, int n, const uint32_t *tx,
                              const uint32_t *ty, int tn, const uint32_t *bits,
                              const uint32_t *off, const uint4 *hash, int hash_probe,
                              cudaStream_t st);

}  // namespace lal
