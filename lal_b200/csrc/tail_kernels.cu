/*
 * tail_kernels.cu -- sm_100a kernels of the LAL decode tail.
 *
 * The streaming kernel (tail_kernel) handles one stream (B = 1) and has three
 * modes that share one body:
 *
 *   MODE_FUSED   hidden fp32 -> int8 quantize (prologue, every CTA) -> int8
 *                GEMV over this CTA's slice of vocab rows -> logits with the
 *                reference's scale epilogue -> repetition penalty -> per-CTA
 *                tie-complete top-k list -> the last CTA to finish merges the
 *                lists, runs the ordered softmax and the draw, and pushes
 *                the token into the device-resident history.
 *   MODE_LMHEAD  the GEMV + scale epilogue only (runtime/lal_q8_kernel.h:463
 *                drop-in): quantized vector in, logits out.
 *   MODE_SAMPLE  logits in (host copy), penalty written back, then the same
 *                select / merge / draw (runtime/lal_sampling.h:46 drop-in).
 *
 * Data movement: each CTA owns a contiguous slice of rows, which is one
 * contiguous byte range of the row-major LM head; a producer warp streams it
 * into a ring of shared-memory stages with cp.async.bulk (untiled TMA into
 * this CTA's own shared memory, L2 evict-first) completing on mbarriers, and
 * 8 consumer warps
 * each take whole rows: every lane holds its 16-byte columns of the quantized
 * vector in registers and does 4 dp4a per 16 bytes of weights; a warp
 * reduction (redux.sync) gives the exact int32 dot.
 *
 * Exactness: all float steps use explicit round-to-nearest intrinsics in the
 * reference's order (scale_x*scale_w[v] then *(float)dot; penalty divide or
 * multiply once per history occurrence; (l-max_l)/T; sequential float sum in
 * ascending vocab order); the file is compiled with -fmad=false.  The
 * softmax weights use lal_expf_glibc (lal_expf.h), equal to glibc expf.
 */
#include "tail_device.cuh"
#include "tail_wide.cuh"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <utility>
#include <vector>

namespace lal {
namespace {

/* The head of the merge's shared-memory area: per-rank offsets of the
 * gathered entries, the load's failure word, and each record's form. */
struct MergeHead {
    int roff[kMaxRanks + 1]; /* prefix offsets of the records' entries        */
    int rbad;                /* DEV_* failure of the load, or 0               */
    int wide;                /* some record is in the wide form               */
    int rties[kMaxRanks];    /* each record's ties (0: list form)             */
    uint32_t rtkey[kMaxRanks]; /* each wide record's T_shard key              */
    int pad;
};
constexpr int kMergeHead = (int)((sizeof(MergeHead) + 15) / 16 * 16);
template <class Load>
__device__ void merge_sample(const MergeParams &mp, int b, uint8_t *area, Misc *ms, Load load);

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

/* Peer exchange of the sharded step.  A record slot in a rank's receive
 * buffer ([2 parities][n_ranks][rec_bytes]) is a run of 64-bit words whose
 * high half is the step's sequence number: [count | seq], [status | seq],
 * [ties | seq], [T_shard key | seq], then per entry [value bits | seq],
 * [vocab id | seq], and after rec_cap entries the wide form's bitmap words
 * [word | seq] (peer_record_bytes).  A 64-bit store is single-copy atomic, so
 * a reader that sees seq in a word has that word's data: no fence orders the
 * data before a flag, and a stale word (a step two back, same parity) never
 * matches.  This writes the list form (ties 0), or a failure record. */
__device__ void peer_publish(const TailParams &p, int status, int m, const float *Ov,
                             const int *Oi) {
    const size_t slot = ((size_t)(p.seq & 1u) * p.n_ranks + p.rank) * p.rec_bytes;
    const bool fits = status == 0 && m <= p.rec_cap;
    const uint64_t hi = (uint64_t)p.seq << 32;
    for (int r = 0; r < p.n_ranks; ++r) {
        uint64_t *w = reinterpret_cast<uint64_t *>(p.peer_recv[r] + slot);
        if (fits)
            for (int i = threadIdx.x; i < m; i += NT)
                st_sys_pair(w + 4 + 2 * i, hi | __float_as_uint(Ov[i]), hi | (uint32_t)Oi[i]);
        if (threadIdx.x == 0) {
            st_sys_pair(w, hi | (uint32_t)(fits ? m : 0),
                        hi | (uint32_t)(fits ? 0 : (status != 0 ? status : (int)DEV_CAPACITY)));
            st_sys_pair(w + 2, hi, hi);
        }
    }
}

/* Wait until w carries this step's sequence number (bounded: the deadline
 * is a globaltimer value); false on timeout. */
__device__ __forceinline__ bool poll_word(const uint64_t *w, uint32_t seq, uint64_t deadline,
                                          uint64_t *out) {
    for (uint32_t it = 0;; ++it) {
        const uint64_t v = ld_relaxed_sys_u64(w);
        if ((uint32_t)(v >> 32) == seq) {
            *out = v;
            return true;
        }
        if ((it & 15u) == 15u && gtimer() > deadline) return false;
    }
}

/* The four header words of a peer record, loaded together (two 16-byte
 * loads) until every one carries this step's sequence number (bounded by
 * deadline). */
__device__ __forceinline__ bool poll_head4(const uint64_t *w, uint32_t seq, uint64_t deadline,
                                           uint64_t *v) {
    for (uint32_t it = 0;; ++it) {
        ld_sys_pair(w, v[0], v[1]);
        ld_sys_pair(w + 2, v[2], v[3]);
        bool all = true;
#pragma unroll
        for (int q = 0; q < 4; ++q) all = all && (uint32_t)(v[q] >> 32) == seq;
        if (all) return true;
        if ((it & 15u) == 15u && gtimer() > deadline) return false;
    }
}

/* Loader of the peers' records in this rank's own receive buffer. */
struct PeerRecords {
    const TailParams &p;
    Misc *ms;
    __device__ const uint64_t *rec(int r) const {
        return reinterpret_cast<const uint64_t *>(
            p.peer_recv[p.rank] + ((size_t)(p.seq & 1u) * p.n_ranks + r) * p.rec_bytes);
    }
    __device__ void operator()(MergeHead &hd, uint32_t *Mk, int *Mi, int cap,
                               float *scratch) const {
        const int tid = threadIdx.x;
        const uint64_t deadline = gtimer() + kWaitNs;
        int *rstat = reinterpret_cast<int *>(scratch);
        if (tid == 0) ms->found = 1;
        __syncthreads();
        if (tid < p.n_ranks) {
            uint64_t v[4];
            if (poll_head4(rec(tid), p.seq, deadline, v)) {
                hd.roff[tid] = (int)(uint32_t)v[0];
                rstat[tid] = (int)(uint32_t)v[1];
                hd.rties[tid] = (int)(uint32_t)v[2];
                hd.rtkey[tid] = (uint32_t)v[3];
            } else {
                ms->found = 0;
            }
        }
        __syncthreads();
        if (tid == 0) {
            int acc = 0, st = ms->found ? 0 : (int)DEV_TIMEOUT, wide = 0;
            for (int r = 0; r < p.n_ranks && st == 0; ++r) {
                const int c = hd.roff[r], s = rstat[r];
                if (s != 0) st = s;
                else if (c < 0 || c > p.rec_cap || hd.rties[r] < 0) st = DEV_CAPACITY;
                if (hd.rties[r] > 0) wide = 1;
                hd.roff[r] = acc;
                acc += c;
            }
            hd.roff[p.n_ranks] = acc;
            if ((acc > cap || (acc < 1 && !wide)) && st == 0) st = DEV_CAPACITY;
            hd.rbad = st;
            hd.wide = wide;
        }
        __syncthreads();
        if (hd.rbad != 0) return;
        const int M = hd.roff[p.n_ranks];
        for (int e = tid; e < M; e += NT) {
            int r = 0;
            while (hd.roff[r + 1] <= e) ++r;
            const int j = e - hd.roff[r];
            const uint64_t *w = rec(r);
            uint64_t v = 0, x = 0;
            if (poll_pair(w + 4 + 2 * j, p.seq, deadline, v, x)) {
                Mk[e] = f2key(__uint_as_float((uint32_t)v));
                Mi[e] = (int)(uint32_t)x;
            } else {
                ms->found = 0;
            }
        }
        __syncthreads();
        if (tid == 0) {
            if (!ms->found) hd.rbad = DEV_TIMEOUT;
            stamp(p, (int)gridDim.x * 8 + 6); /* every rank's record is here */
        }
        __syncthreads();
    }
    /* nw bitmap words of rank r's wide record from word w0 (every thread);
     * a word that does not arrive in time clears ms->sh[12] */
    __device__ void bitmap(int r, int w0, int nw, uint32_t *dst) const {
        const uint64_t *w = rec(r) + 4 + 2 * p.rec_cap + w0;
        const uint64_t deadline = gtimer() + kWaitNs;
        for (int i = threadIdx.x; i < nw; i += NT) {
            uint64_t v = 0;
            if (poll_word(w + i, p.seq, deadline, &v)) dst[i] = (uint32_t)v;
            else {
                dst[i] = 0u;
                ms->sh[12] = 0u;
            }
        }
    }
};

/* The peer exchange's merge of this step (the fused kernel's last CTA, after
 * it published its record): wait for every rank's record, merge and draw
 * like merge_kernel.  With a host waiting on the step's completion word
 * (lal_tail_step), thread 0 -- the thread that writes the token on every
 * path of the merge -- then hands it the token, or -1 when the step failed
 * (the host then reads the status); the token slot is set to -1 first, so
 * no path can pass on an earlier step's token. */
__device__ __noinline__ void peer_merge(const TailParams &p, uint8_t *smem, Misc *ms) {
    if (threadIdx.x == 0 && p.host_tok != nullptr) p.tokens[0] = -1;
    MergeParams mp;
    mp.recv = p.peer_recv[p.rank] + (size_t)(p.seq & 1u) * p.n_ranks * p.rec_bytes;
    mp.rank_stride = p.rec_bytes;
    mp.rec_bytes = p.rec_bytes;
    mp.rec_cap = p.rec_cap;
    mp.n_ranks = p.n_ranks;
    mp.vocab = p.vocab;
    mp.variant = p.variant;
    mp.temperature = p.temperature;
    mp.top_k = p.top_k;
    mp.u = p.u;
    mp.hist_ids = p.hist_ids;
    mp.hist_n = p.hist_n;
    mp.hist_head = p.hist_head;
    mp.hist_cap = p.hist_cap;
    mp.push_history = p.push_history;
    mp.tokens = p.tokens;
    mp.diag = p.diag;
    mp.status = p.status;
    mp.expf_x = p.expf_x;
    mp.expf_y = p.expf_y;
    mp.expf_n = p.expf_n;
    mp.expf_bits = p.expf_bits;
    mp.expf_off = p.expf_off;
    mp.expf_hash = p.expf_hash;
    mp.expf_hash_probe = p.expf_hash_probe;
    mp.smem_cap = (p.area_bytes - kMergeHead - kWideWalkBytes) / 24;
    mp.phase_ts = p.phase_ts ? p.phase_ts + ((size_t)gridDim.x + 1) * 8 : nullptr;
    merge_sample(mp, 0, smem, ms, PeerRecords{p, ms});
    if (threadIdx.x == 0 && p.host_tok != nullptr)
        notify_host(p.host_tok, __ldcg(p.seq_in), p.tokens[0]);
}

/* The wide path (tail_wide.cuh) of a launch whose candidates did not fit the
 * fast select: the exact select over this launch's logits in global memory
 * (every CTA wrote its rows before its ticket), then the launch's own output
 * -- the draw, the shard record in its wide form, or the candidate export.
 * k is the launch's effective k; hn / hhead the history ring's words. */
__device__ __noinline__ void tail_wide(const TailParams &p, int k, bool greedy, float temp,
                                       float u0, int hn, int hhead, uint8_t *smem, Misc *ms) {
    WideDense a;
    a.lg = p.logits;
    a.rows = p.rows;
    a.row_base = p.row_base;
    a.vocab = p.vocab;
    a.k = k;
    a.variant = p.variant;
    a.greedy = greedy ? 1 : 0;
    a.temp = temp;
    a.u = u0;
    a.cap = max(1, p.max_k);
    a.ex = ExpfTables{p.expf_x, p.expf_y, p.expf_bits, p.expf_off, p.expf_hash,
                      p.expf_hash_probe};
    a.token = p.tokens;
    a.host_tok = p.host_tok;
    a.host_seq = p.host_tok ? __ldcg(p.seq_in) : 0u;
    a.diag = p.diag;
    a.hist_ids = p.hist_ids;
    a.hist_n = p.hist_n;
    a.hist_head = p.hist_head;
    a.hist_cap = p.hist_cap;
    a.push_history = p.push_history;
    a.hn = hn;
    a.hhead = hhead;
    a.rec = p.shard_out;
    a.rec_cap = p.rec_cap;
    a.peer_recv = p.peer_recv;
    a.n_ranks = p.n_ranks;
    a.rank = p.rank;
    a.rec_bytes = p.rec_bytes;
    a.seq = p.seq;
    a.cand_val = p.cand_val_out;
    a.cand_idx = p.cand_idx_out;
    a.cand_cap = p.cand_val_out ? p.cand_out_cap : 0;
    a.candidates_only = p.candidates_only;
    a.top_p = p.variant == VARIANT_GPT2 ? p.top_p : 0.0f;
    wide_dense(a, smem, ms);
}

/* ----------------------------------------------------- the kernel --- */
template <int MODE, int NCH>
__global__ void __launch_bounds__(NT, 1) tail_kernel(const __grid_constant__ TailParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, cta = blockIdx.x;
    const int c0 = (int)((long long)p.rows * cta / G);
    const int c1 = (int)((long long)p.rows * (cta + 1) / G);
    const int nloc = c1 - c0;

    uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + p.off_bars);
    uint64_t *empty_bar = full_bar + kMaxStages;
    int8_t *xq_s = reinterpret_cast<int8_t *>(smem + p.off_xq);
    float *sw_s = reinterpret_cast<float *>(smem + p.off_sw);
    float *lg_s = reinterpret_cast<float *>(smem + p.off_lg);
    uint32_t *cnt_s = reinterpret_cast<uint32_t *>(smem + p.off_cnt);
    uint32_t *hist_s = reinterpret_cast<uint32_t *>(smem + p.off_hist); /* 4096 bins */
    Misc *ms = reinterpret_cast<Misc *>(smem + p.off_misc);

    /* stream 0 sampling parameters (the last CTA also uses u0 and the ring
     * words) */
    float temp = 0.0f, pen = 1.0f, u0 = 0.0f;
    int topk = 0, hn = 0, hhead = 0;
    bool greedy = false, use_pen = false;
    auto load_params = [&]() {
        if (MODE != MODE_LMHEAD) {
            temp = p.temperature[0];
            topk = p.top_k[0];
            pen = p.rep_penalty[0];
            hn = p.hist_n ? p.hist_n[0] : 0;
            hhead = p.hist_head ? p.hist_head[0] : 0;
            u0 = p.u[0];
        }
        greedy = (temp <= 0.0f) || (topk <= 0);
        use_pen = (MODE != MODE_LMHEAD) && (pen > 1.0f) && hn > 0 &&
                  (p.variant == VARIANT_SERVER || !greedy);
    };
    const bool stream_warp = MODE != MODE_SAMPLE && warp == kConsumerWarps;

    /* ---- phase 0: barriers -------------------------------------------- */
    if (tid == 0) {
        stamp(p, cta * 8 + 0);
        ms->abort_flag = 0;
        ms->cnt = 0u;
        for (int w = 0; w < NWARP; ++w) ms->wmax[w] = 0u;
        if (MODE != MODE_SAMPLE) {
            for (int s = 0; s < p.stages; ++s) {
                mbar_init(&full_bar[s], 1);
                mbar_init(&empty_bar[s], kConsumerWarps);
            }
            mbar_fence_init();
        }
    }
    __syncthreads();
    /* The fused launch may start while the previous kernel on the stream is
     * still running (programmatic dependent launch).  The LM head and its row
     * scales are never written by a step, so the producer warp streams the
     * rows and the consumer warps load the scales at once; every other read
     * (hidden vector, history ring, sampling parameters, select scratch)
     * waits for the previous kernel to complete. */
    if (MODE != MODE_SAMPLE && warp < kConsumerWarps)
#pragma unroll 4
        for (int i = tid; i < nloc; i += kConsumerWarps * 32) sw_s[i] = __ldg(p.scale_w + c0 + i);
    if (!stream_warp) {
        grid_dep_wait();
        if (tid == 0) stamp(p, cta * 8 + 3); /* the previous kernel is complete */
        load_params();
    }

    /* ---- the consumer warps' prologue (the producer streams meanwhile):
     * quantized vector, row scales, penalty counts ------------------------ */
    if (warp < kConsumerWarps) {
        const int ctid = tid; /* 0 .. kConsumerWarps*32-1 */
        constexpr int NC = kConsumerWarps * 32;
        /* every global load of the prologue is issued before any result is
         * used: hidden values and history ids into registers, scales to smem */
        constexpr int kHReg = 16;
        const float *h = p.hidden;
        float hv[kHReg];
        int ids[kHReg];
        /* the hidden vector is quantized here (per CTA) by the fused launch,
         * and by an LM-head launch given the hidden vector (the GPT-2 tail:
         * its server's truncating quantizer) */
        const bool qin = MODE == MODE_FUSED || (MODE == MODE_LMHEAD && p.hidden != nullptr);
        if (qin) {
#pragma unroll
            for (int j = 0; j < kHReg; ++j) {
                const int i = ctid + j * NC;
                hv[j] = i < p.d ? __ldg(h + i) : 0.0f;
            }
        }
        if (MODE != MODE_LMHEAD) {
            /* the ring's slots, loaded with the parameters rather than after
             * them (one round trip): only i < hn count, and only with a
             * penalty */
#pragma unroll
            for (int j = 0; j < kHReg; ++j) {
                const int i = ctid + j * NC;
                ids[j] = i < p.hist_cap ? __ldcg(p.hist_ids + i) : -1;
            }
        }
        /* the final RMSNorm's weights, when the step takes the residual
         * stream (d <= kHReg * NC: the whole vector sits in registers) */
        const bool norm = MODE == MODE_FUSED && p.norm_w != nullptr;
        float wv[kHReg];
        if (norm) {
#pragma unroll
            for (int j = 0; j < kHReg; ++j) {
                const int i = ctid + j * NC;
                wv[j] = i < p.d ? __ldg(p.norm_w + i) : 0.0f;
            }
        }
        if (norm) {
            /* runtime/lal_simd_optim.h:32-58 through the key histogram's
             * shared memory (zeroed after): eight lane sums, combined and
             * inverted by one thread, then x * inv_rms * w in registers */
            float *xs = reinterpret_cast<float *>(hist_s);
#pragma unroll
            for (int j = 0; j < kHReg; ++j) {
                const int i = ctid + j * NC;
                if (i < p.d) xs[i] = hv[j];
            }
            consumer_sync();
            if (ctid < 8) ms->nrm[ctid] = rmsnorm_lane(xs, p.d, ctid);
            consumer_sync();
            if (ctid == 0) ms->ninv = rmsnorm_inv(ms->nrm, p.d, p.norm_eps);
            consumer_sync();
            const float inv_rms = ms->ninv;
#pragma unroll
            for (int j = 0; j < kHReg; ++j) hv[j] = rmsnorm_apply(hv[j], inv_rms, wv[j]);
        }
        /* The fused launch stages x in the key histogram's words (zeroed
         * after the quantizer), so that the quantizer takes four consecutive
         * elements a thread and writes them as one word. */
        const bool stage_x = MODE == MODE_FUSED && p.d <= 4096 && (p.ld & 3) == 0;
        float *xs_q = reinterpret_cast<float *>(hist_s);
        if (stage_x) {
#pragma unroll
            for (int j = 0; j < kHReg; ++j) {
                const int i = ctid + j * NC;
                if (i < p.d) xs_q[i] = hv[j];
            }
        }
        if (MODE != MODE_LMHEAD) {
            for (int i = ctid; i < nloc; i += NC) cnt_s[i] = 0u;
            if (!stage_x)
                for (int i = ctid; i < 4096; i += NC) hist_s[i] = 0u;
        }
        float m = 0.0f;
        if (qin) {
#pragma unroll
            for (int j = 0; j < kHReg; ++j) m = fmaxf(m, fabsf(hv[j]));
            for (int i = ctid + kHReg * NC; i < p.d; i += NC) m = fmaxf(m, fabsf(__ldg(h + i)));
        }
        m = consumer_max_f(m, ms); /* also orders the zeroing before the adds */
        if (ctid == 0) stamp(p, cta * 8 + 6); /* the hidden vector's maximum */
        if (MODE != MODE_LMHEAD && use_pen) {
            /* runtime/lal_sampling.h:60-66: ids outside [0, V) are skipped */
            auto count = [&](int t) {
                if (t < 0 || t >= p.vocab) return;
                const int g = t - p.row_base;
                if (g >= c0 && g < c1) atomicAdd(&cnt_s[g - c0], 1u);
            };
#pragma unroll
            for (int j = 0; j < kHReg; ++j)
                if (ctid + j * NC < hn) count(ids[j]);
            for (int i = ctid + kHReg * NC; i < hn; i += NC) count(__ldcg(p.hist_ids + i));
        }
        if (qin) {
            /* lal_quantize_x_int8 (runtime/lal_q8_kernel.h:375-424), redundantly
             * per CTA: absmax, scale = max/127 floored at 1e-8, inv = 1/scale,
             * RNE for the first d&~7 elements and truncation for the tail; the
             * GPT-2 server's lm_head_quantize_x (gpt2_server.c:1982-1998)
             * truncates every element. */
            float scale = __fdiv_rn(m, 127.0f);
            if (scale < 1e-8f) scale = 1e-8f;
            const float inv = __fdiv_rn(1.0f, scale);
            const int n8 = MODE == MODE_LMHEAD ? 0 : p.d & ~7;
            auto quant = [&](int i, float x) {
                int v = 0;
                if (i < p.d) {
                    const float s = __fmul_rn(x, inv);
                    if (s != s) v = -127;
                    else {
                        v = (i < n8) ? __float2int_rn(s) : __float2int_rz(s);
                        v = v > 127 ? 127 : (v < -127 ? -127 : v);
                    }
                }
                return (int8_t)v;
            };
            if (stage_x) {
                uint32_t *xq32 = reinterpret_cast<uint32_t *>(xq_s);
                const float4 *xs4 = reinterpret_cast<const float4 *>(xs_q);
                for (int e = ctid; e < p.ld / 4; e += NC) {
                    const int i = 4 * e;
                    const float4 v = xs4[e]; /* elements >= d quantize to 0 */
                    xq32[e] = (uint32_t)(uint8_t)quant(i, v.x) |
                              (uint32_t)(uint8_t)quant(i + 1, v.y) << 8 |
                              (uint32_t)(uint8_t)quant(i + 2, v.z) << 16 |
                              (uint32_t)(uint8_t)quant(i + 3, v.w) << 24;
                }
                consumer_sync(); /* x is read before its words are zeroed */
                for (int i = ctid; i < 4096; i += NC) hist_s[i] = 0u;
            } else {
#pragma unroll
                for (int j = 0; j < kHReg; ++j) {
                    const int i = ctid + j * NC;
                    if (i < p.ld) xq_s[i] = quant(i, hv[j]);
                }
                for (int i = ctid + kHReg * NC; i < p.ld; i += NC)
                    xq_s[i] = quant(i, i < p.d ? __ldg(h + i) : 0.0f);
            }
            if (ctid == 0) ms->sx = scale;
        } else if (MODE == MODE_LMHEAD) {
            for (int i = ctid; i < p.ld; i += NC) xq_s[i] = i < p.d ? p.xq_in[i] : (int8_t)0;
            if (ctid == 0) ms->sx = p.scale_x_dev ? *p.scale_x_dev : p.scale_x_in;
        }
        consumer_sync();
        if (ctid == 0) stamp(p, cta * 8 + 1);
    }

    /* ---- phase 1: logits of this CTA's rows --------------------------- */
    if (MODE != MODE_SAMPLE) {
        const int R = p.rows_per_stage;
        const int n_chunks = (nloc + R - 1) / R;
        if (warp == kConsumerWarps) {
            /* producer: one elected lane streams the slice, chunk by chunk */
            if (lane == 0) {
                const uint64_t pol = policy_evict_first();
                int c = 0;
                for (; c < n_chunks; ++c) {
                    const int s = c % p.stages;
                    const uint32_t use = (uint32_t)(c / p.stages);
                    if (c >= p.stages && !mbar_wait(&empty_bar[s], (use & 1u) ^ 1u, &ms->abort_flag)) {
                        ms->abort_flag = 1;
                        break;
                    }
                    const int r0 = c0 + c * R;
                    const int nr = min(R, c1 - r0);
                    const uint32_t bytes = (uint32_t)nr * (uint32_t)p.ld;
                    mbar_expect_tx(&full_bar[s], bytes);
                    bulk_g2s(smem + (size_t)s * p.stage_bytes, p.W + (size_t)r0 * p.ld, bytes,
                             &full_bar[s], pol);
                    /* at most two stages ahead of the previous kernel on the
                     * stream: a full ring's burst (25 MB over the grid) slows
                     * that kernel's serial tail; measured 93.0 against 93.4 us
                     * a step back to back */
                    if (c == p.early_stages - 1) grid_dep_wait();
                }
                /* Do not leave copies in flight: wait (bounded) for the last
                 * issued stages to land before the CTA may exit. */
                for (int q = max(0, c - p.stages); q < c; ++q) {
                    const int s = q % p.stages;
                    mbar_wait(&full_bar[s], (uint32_t)(q / p.stages) & 1u, &ms->abort_flag);
                }
            }
        } else {
            const float sx = ms->sx;
            uint32_t wmax = 0u; /* lane 0: largest key of this warp's rows */
            int4 xr[NCH];
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int col = j * 512 + lane * 16;
                xr[j] = col < p.ld ? *reinterpret_cast<const int4 *>(xq_s + col)
                                   : make_int4(0, 0, 0, 0);
            }
            for (int c = 0; c < n_chunks; ++c) {
                const int s = c % p.stages;
                if (!mbar_wait(&full_bar[s], (uint32_t)(c / p.stages) & 1u, &ms->abort_flag)) {
                    ms->abort_flag = 1;
                    break;
                }
                const int r0 = c0 + c * R;
                const int nr = min(R, c1 - r0);
                const uint8_t *st = smem + (size_t)s * p.stage_bytes;
                for (int rr = warp; rr < nr; rr += kConsumerWarps) {
                    const uint8_t *row = st + (size_t)rr * p.ld;
                    int acc = 0, acc_tail = 0;
#pragma unroll
                    for (int j = 0; j < NCH; ++j) {
                        const int col = j * 512 + lane * 16;
                        if (col < p.ld) {
                            const int4 w = *reinterpret_cast<const int4 *>(row + col);
                            int part = __dp4a(w.x, xr[j].x, 0);
                            part = __dp4a(w.y, xr[j].y, part);
                            part = __dp4a(w.z, xr[j].z, part);
                            part = __dp4a(w.w, xr[j].w, part);
                            if (MODE == MODE_LMHEAD && col >= p.trunc_cols) acc_tail += part;
                            else acc += part;
                        }
                    }
                    acc = __reduce_add_sync(0xffffffffu, acc);
                    if (MODE == MODE_LMHEAD && p.trunc_cols < p.ld) {
                        acc_tail = __reduce_add_sync(0xffffffffu, acc_tail);
                        if (r0 + rr >= p.trunc_rows_end) acc += acc_tail;
                    }
                    if (lane == 0) {
                        const int lr = r0 + rr - c0;
                        /* runtime/lal_q8_kernel.h:489: scale_x*scale_w[v]*(float)dot */
                        float l = __fmul_rn(__fmul_rn(sx, sw_s[lr]), __int2float_rn(acc));
                        if (MODE == MODE_FUSED) {
                            l = penalise(l, cnt_s[lr], pen);
                            lg_s[lr] = l;
                            const uint32_t key = f2key(l);
                            atomicAdd(&hist_s[key >> 20], 1u); /* level-0 bins */
                            wmax = max(wmax, key);
                        }
                        p.logits[c0 + lr] = l;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty_bar[s]);
            }
            if (lane == 0) ms->wmax[warp] = wmax;
        }
        __syncthreads();
        if (tid == 0) stamp(p, cta * 8 + 2);
        /* this CTA's rows are done: the next launch may begin to stream */
        grid_dep_launch_dependents();
        if (stream_warp) {
            grid_dep_wait();
            load_params();
        }
        if (MODE == MODE_LMHEAD) {
            if (tid == 0 && ms->abort_flag) atomicCAS(p.status, 0, (int)DEV_TIMEOUT);
            return;
        }
    } else {
        __syncthreads(); /* penalty counts come from the consumers' prologue */
        uint32_t wmax = 0u;
        for (int i = tid; i < nloc; i += NT) {
            float l = p.logits[c0 + i];
            const uint32_t cnt = cnt_s[i];
            if (cnt) {
                l = penalise(l, cnt, pen);
                p.logits[c0 + i] = l; /* the reference mutates logits in place */
            }
            lg_s[i] = l;
            const uint32_t key = f2key(l);
            atomicAdd(&hist_s[key >> 20], 1u); /* level-0 bins */
            wmax = max(wmax, key);
        }
        wmax = __reduce_max_sync(0xffffffffu, wmax);
        if (lane == 0) ms->wmax[warp] = wmax;
        __syncthreads();
    }

    /* ---- phase 2: the global threshold ---------------------------------- *
     * k = min(top_k, V) (runtime/lal_sampling.h:70-71); greedy is k = 1 and
     * takes the lowest index among the maxima.  T, the k-th largest
     * penalised logit counted with multiplicity, is located with a global
     * histogram of the order keys, built by all CTAs: a 12-bit level, then 10
     * + 10 bits only while the boundary bin is large.  Every key >= the
     * boundary bin's lower edge Lb (a tie-complete superset of {l >= T}) is
     * appended to a global buffer; the last CTA selects T exactly from it. */
    int k = greedy ? 1 : topk;
    if (k > p.vocab) k = p.vocab;
    if (k > p.rows) k = p.rows;
    if (k < 1) k = 1;
    uint32_t *lh = reinterpret_cast<uint32_t *>(smem); /* stage area is free now */
    uint32_t prefix = 0u, pmask = 0u;
    int above = 0, binc = 0;
    bool ok = ms->abort_flag == 0;
    /* Small k against the slice (the common case): no grid barrier.  Each
     * CTA's own boundary bin (from its level-0 histogram) has a lower edge
     * below its local k-th largest, hence below the global T; the union of
     * every CTA's keys >= its own edge contains {l >= T}, and the largest
     * edge L is a lower bound of T that the last CTA filters with.  Large k
     * (k comparable to a slice) takes the global histogram below. */
    const bool local_edges = p.local_edges != 0; /* = use_local_edges(k, ...) */
    if (local_edges) {
        /* warp 0 finds the boundary bin from the top, starting at the bin of
         * this CTA's largest key (the warps' running maxima of the rows).
         * That key also goes out with the head record: the k-th largest of
         * the CTAs' maxima is a second lower bound of T (distinct elements),
         * usually much tighter.  (A CTA with fewer than k rows would give no
         * bound: it keeps all.) */
        if (warp == 0) {
            uint32_t mx = ms->wmax[0];
            for (int w = 1; w < NWARP; ++w) mx = max(mx, ms->wmax[w]);
            const uint32_t bin = warp_boundary_bin_4096(hist_s, mx >> 20, (uint32_t)min(k, nloc));
            if (lane == 0) {
                ms->sh[0] = bin;
                if (nloc >= k) atomicMax(p.gL, bin << 20);
                p.gmax[cta] = mx;
                p.gcand_key[kSlotHeads + cta * kSlotHeadWords] = mx;
            }
        }
        __syncthreads();
        prefix = nloc >= k ? ms->sh[0] << 20 : 0u;
    }
    for (int level = 0; level < 3 && !local_edges; ++level) {
        const int bits = level == 0 ? 12 : 10;
        const int shift = level == 0 ? 20 : (level == 1 ? 10 : 0);
        const int nb = 1 << bits;
        unsigned *gh = p.ghist + (level == 0 ? 0 : (level == 1 ? 4096 : 5120));
        /* this CTA's histogram: level 0 was accumulated as the logits were
         * produced; deeper levels take a pass over the keys in the bin */
        uint32_t *loc = level == 0 ? hist_s : lh;
        if (level > 0) {
            for (int i = tid; i < nb; i += NT) lh[i] = 0u;
            __syncthreads();
            for (int i0 = 0; i0 < nloc; i0 += NT) {
                const int i = i0 + tid;
                const uint32_t key = i < nloc ? f2key(lg_s[i]) : 0u;
                const bool m = i < nloc && (key & pmask) == prefix;
                const uint32_t digit = (key >> shift) & (uint32_t)(nb - 1);
                const unsigned voters = __ballot_sync(0xffffffffu, m);
                if (m) {
                    const unsigned peers = __match_any_sync(voters, digit);
                    if ((int)(threadIdx.x & 31) == __ffs(peers) - 1)
                        atomicAdd(&lh[digit], (uint32_t)__popc(peers));
                }
            }
        }
        __syncthreads();
        for (int i = tid; i < nb; i += NT) {
            const uint32_t c = loc[i];
            if (c) atomicAdd(&gh[i], c);
        }
        ok = grid_sync(p.gbar, (unsigned)G, ms, p.status) && ok;
        if (tid == 0) stamp(p, cta * 8 + 3 + level);
        /* boundary bin, from the top: every CTA reads the same histogram */
        for (int i = tid; i < nb; i += NT) lh[i] = __ldcg(gh + i);
        __syncthreads();
        uint32_t ab, cnt;
        const uint32_t bin = boundary_bin(lh, nb, (uint32_t)(k - above), ms, &ab, &cnt);
        above += (int)ab;
        binc = (int)cnt;
        prefix |= bin << shift;
        pmask |= (uint32_t)(nb - 1) << shift;
        if (binc <= kRefineMax) break;
    }
    const uint32_t Lb = prefix; /* lower edge of this CTA's (or the global) bin */
    const int S_hist = above + binc; /* global histogram: keys >= Lb, all CTAs */

    /* append this CTA's keys >= Lb */
    if (local_edges) {
        /* into this CTA's fixed slot of kSlot entries, in descending key order
         * (ties by index), so that the last CTA reads only the head of each
         * slot; the slot count may exceed kSlot (the tail is dropped and the
         * last CTA checks that nothing dropped can be a candidate) */
        /* gather the keys >= Lb in any order (one shared-memory atomic per
         * warp and round) as 64-bit words key << 32 | ~row: a larger word is
         * a larger key, or the same key at a smaller row, so the rank below
         * is one comparison an element */
        uint64_t *tw = reinterpret_cast<uint64_t *>(lh);
        const unsigned below = (1u << lane) - 1u;
        for (int i0 = 0; i0 < nloc; i0 += NT) {
            const int i = i0 + tid;
            const uint32_t key = i < nloc ? f2key(lg_s[i]) : 0u;
            const bool take = i < nloc && key >= Lb;
            const unsigned mask = __ballot_sync(0xffffffffu, take);
            if (mask) {
                const int lead = __ffs(mask) - 1;
                uint32_t base = 0u;
                if (lane == lead) base = atomicAdd(&ms->cnt, (uint32_t)__popc(mask));
                base = __shfl_sync(0xffffffffu, base, lead);
                if (take)
                    tw[base + (uint32_t)__popc(mask & below)] =
                        ((uint64_t)key << 32) | (uint32_t)~(uint32_t)i;
            }
        }
        __syncthreads();
        const uint32_t n = ms->cnt;
        uint32_t *slot_k = p.gcand_key + (size_t)cta * kSlot;
        int *slot_i = p.gcand_idx + (size_t)cta * kSlot;
        uint32_t *head = p.gcand_key + kSlotHeads + cta * kSlotHeadWords;
        for (int j = tid; j < (int)n; j += NT) {
            const uint64_t w = tw[j];
            const uint32_t me = (uint32_t)(w >> 32);
            const int row = p.row_base + c0 + (int)~(uint32_t)w;
            int r = 0;
#pragma unroll 8
            for (int q = 0; q < (int)n; ++q) r += tw[q] > w;
            if (r < kSlot) {
                slot_k[r] = me;
                slot_i[r] = row;
            }
            if (r < 4) {
                head[4 + r] = me;
                head[8 + r] = (uint32_t)row;
            }
            if (r == kSlot - 1 && n > (uint32_t)kSlot) head[2] = me;
        }
        if (tid == 0) {
            p.gslot_n[cta] = n;
            head[1] = n;
            if (n <= (uint32_t)kSlot) head[2] = 0u;
        }
    } else {
        const int seg = (nloc + NT - 1) / NT;
        const int i0 = min(nloc, tid * seg), i1 = min(nloc, i0 + seg);
        uint32_t c = 0;
        for (int i = i0; i < i1; ++i) c += f2key(lg_s[i]) >= Lb;
        uint32_t tot;
        uint32_t pos = block_scan_excl(c, ms, &tot);
        if (tid == 0) ms->sh[3] = tot ? atomicAdd(p.gcount, tot) : 0u;
        __syncthreads();
        pos += ms->sh[3];
        for (int i = i0; i < i1; ++i) {
            const uint32_t key = f2key(lg_s[i]);
            if (key >= Lb) {
                if (pos < (uint32_t)p.gcand_cap) {
                    p.gcand_key[pos] = key;
                    p.gcand_idx[pos] = p.row_base + c0 + i;
                }
                ++pos;
            }
        }
    }

    /* ---- phase 3: the last CTA to arrive selects and samples ------------ *
     * The barrier orders every thread's writes above before thread 0's
     * acquire-release ticket, which publishes them at GPU scope; in the last
     * CTA the same atomic acquires every other CTA's writes, and the barrier
     * after it orders all of its threads' reads behind that. */
    __syncthreads();
    if (tid == 0) {
        ms->ticket = (int)atom_add_acq_rel_gpu(&p.counter[0], 1u);
        stamp(p, cta * 8 + 7);
    }
    __syncthreads();
    if (ms->ticket != G - 1) return;
    if (tid == 0) stamp(p, G * 8 + 0);

    /* shared-memory plan of the stage area: superset keys + indices (Sk, Si),
     * then the superset weights (Ws), the candidates (Cv, Ci, Cw) and their
     * ascending-index copies (Ov, Oi, Ce = weights, then running sums), ccap
     * a power of two */
    /* grid-histogram path: the superset size is known (S_hist); small-k
     * path: the slot heads are small, a sixteenth of the area suffices */
    /* a multiple of 4 entries: Si and the arrays after it start on 16-byte
     * boundaries */
    const int s_cap = local_edges ? p.area_bytes / 16 / 4 * 4
                                  : max(4, min((S_hist + 3) & ~3, (p.area_bytes / 8 - 28 * 64) & ~3));
    int ccap = 1;
    while (ccap * 2 * 28 <= p.area_bytes - 8 * s_cap) ccap *= 2;
    uint32_t *Sk = reinterpret_cast<uint32_t *>(smem);
    int *Si = reinterpret_cast<int *>(Sk + s_cap);
    float *Ws = reinterpret_cast<float *>(Si + s_cap);
    float *Cv = Ws + ccap;
    int *Ci = reinterpret_cast<int *>(Cv + ccap);
    float *Cw = reinterpret_cast<float *>(Ci + ccap);
    float *Ov = Cw + ccap;
    int *Oi = reinterpret_cast<int *>(Ov + ccap);
    float *Ce = reinterpret_cast<float *>(Oi + ccap);

    /* one batch of global loads: status, counts, the bound words and, on the
     * small-k path, thread g's slot count, maximum and its slot's first 4
     * entries (read whatever the count; only the first min(n, kSlot) count) */
    const int dev_status = __ldcg(p.status);
    const int Sg = (int)__ldcg(p.gcount);
    uint32_t Lg = 0u, gmx = 0u, gdrop = 0u, hk[4] = {0u, 0u, 0u, 0u};
    int g_n = 0, hi[4] = {0, 0, 0, 0};
    if (local_edges) {
        Lg = __ldcg(p.gL);
        if (tid < G) {
            const uint4 *h4 =
                reinterpret_cast<const uint4 *>(p.gcand_key + kSlotHeads + tid * kSlotHeadWords);
            const uint4 a = __ldcg(h4), b = __ldcg(h4 + 1), c = __ldcg(h4 + 2);
            gmx = a.x;
            g_n = (int)a.y;
            gdrop = a.z;
            hk[0] = b.x;
            hk[1] = b.y;
            hk[2] = b.z;
            hk[3] = b.w;
            hi[0] = (int)c.x;
            hi[1] = (int)c.y;
            hi[2] = (int)c.z;
            hi[3] = (int)c.w;
        }
    }
    int m = 0;
    uint32_t T = 0u;
    uint32_t top_key = 0u; /* the superset's largest key, when known early */
    bool top_known = false;
    bool fine = ok && dev_status == 0 &&
                (local_edges || (Sg <= p.gcand_cap && Sg >= 1));
    int S = S_hist;
    if (fine && local_edges) {
        /* keep the slot entries >= L* = max(largest CTA edge, k-th largest
         * CTA maximum): each slot is sorted descending, so only its head is
         * read */
        uint32_t L = Lg;
        if (k <= G) {
            /* L2 = k-th largest of the G per-CTA maxima <= T */
            if (tid < G) ms->gm[tid] = gmx;
            __syncthreads();
            if (tid == 0) stamp(p, cta * 8 + 4);
            /* (the gm tail up to a multiple of 4 is zero: it never counts) */
            if (tid >= G && tid < ((G + 3) & ~3)) ms->gm[tid] = 0u;
            __syncthreads();
            uint32_t best = 0xffffffffu;
            const uint4 *g4 = reinterpret_cast<const uint4 *>(ms->gm);
            for (int g = tid; g < G; g += NT) {
                const uint32_t me = ms->gm[g];
                int gt = 0;
#pragma unroll 4
                for (int j = 0; j < (G + 3) >> 2; ++j) {
                    const uint4 v = g4[j];
                    gt += (v.x > me) + (v.y > me) + (v.z > me) + (v.w > me);
                }
                if (gt < k) best = min(best, me);
            }
            best = __reduce_min_sync(0xffffffffu, best);
            /* with it, the largest of the maxima: the superset's maximum */
            const uint32_t gw = __reduce_max_sync(0xffffffffu, gmx);
            if ((tid & 31) == 0) {
                ms->scan[tid >> 5] = best;
                ms->wmax[tid >> 5] = gw;
            }
            __syncthreads();
            if (tid == 0) stamp(p, cta * 8 + 5);
            uint32_t L2 = ms->scan[0];
            for (int w = 1; w < NWARP; ++w) L2 = min(L2, ms->scan[w]);
            L = max(L, L2);
            for (int w = 0; w < NWARP; ++w) top_key = max(top_key, ms->wmax[w]);
            top_known = true;
            __syncthreads();
        }
        if (tid == 0) stamp(p, G * 8 + 1);
        /* thread g scans slot g's head in groups of 4 keys; gm[g] becomes the
         * slot's dropped-tail bound (0 if the slot held all of its entries) */
        uint32_t c = 0;
        const int g = tid;
        if (g < G) {
            const int lim = min(g_n, kSlot);
            const uint32_t *sk = p.gcand_key + (size_t)g * kSlot;
            bool more = true;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const bool take = more && q < lim && hk[q] >= L;
                c += take;
                more = take;
            }
            /* rarely more than 4 survivors in one slot: read on */
            for (int j = 4; more && j < lim; j += 4) {
                uint32_t kv[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) kv[q] = j + q < lim ? __ldcg(sk + j + q) : 0u;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const bool take = more && j + q < lim && kv[q] >= L;
                    c += take;
                    more = take;
                }
            }
        }
        __syncthreads();
        if (g < G) ms->gm[g] = gdrop;
        uint32_t tot;
        uint32_t pos = block_scan_excl(c, ms, &tot);
        S = (int)tot;
        fine = S >= 1 && S <= s_cap;
        if (fine && g < G) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if ((uint32_t)q < c) {
                    Sk[pos + q] = hk[q];
                    Si[pos + q] = hi[q];
                }
            for (uint32_t j = 4; j < c; ++j) {
                Sk[pos + j] = __ldcg(p.gcand_key + (size_t)g * kSlot + j);
                Si[pos + j] = __ldcg(p.gcand_idx + (size_t)g * kSlot + j);
            }
        }
        if (tid == 0) stamp(p, G * 8 + 2);
    } else if (fine) {
        fine = Sg == S && S <= s_cap;
        if (fine)
#pragma unroll 4
            for (int i = tid; i < S; i += NT) {
                Sk[i] = __ldcg(p.gcand_key + i);
                Si[i] = __ldcg(p.gcand_idx + i);
            }
    }
    /* pad the superset to a multiple of 4 (s_cap is one) */
    if (fine && tid < ((S + 3) & ~3) - S) {
        Sk[S + tid] = 0u;
        Si[S + tid] = 0x7fffffff;
    }
    __syncthreads();
    /* Early weights: the superset holds every candidate and the maximum, so
     * max_l (runtime/lal_sampling.h:107-109) is known before T; the weights'
     * exception-bitmap loads are issued now and consumed after the select,
     * hiding their latency behind it. */
    const bool early = fine && !greedy && S <= 2 * NT && S <= ccap && p.peer_recv == nullptr &&
                       p.shard_out == nullptr;
    float max_l = -1e30f;
    float xw[2] = {0.0f, 0.0f};
    uint32_t bw[2] = {0u, 0u}, olo[2] = {0u, 0u}, ohi[2] = {0u, 0u};
    uint4 hp[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
    float yr[2] = {0.0f, 0.0f};
    if (early) {
        uint32_t mx = top_key;
        if (!top_known) {
            uint32_t mk = 0u;
            for (int j = tid; j < S; j += NT) mk = max(mk, Sk[j]);
            mk = __reduce_max_sync(0xffffffffu, mk);
            if ((tid & 31) == 0) ms->scan[tid >> 5] = mk;
            __syncthreads();
            mx = ms->scan[0];
            for (int w = 1; w < NWARP; ++w) mx = max(mx, ms->scan[w]);
            __syncthreads();
        }
        max_l = fmaxf(-1e30f, key2f(mx));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int j = tid + r * NT;
            if (j < S) {
                xw[r] = __fdiv_rn(__fsub_rn(key2f(Sk[j]), max_l), temp);
                if (p.expf_hash) {
                    hp[r] = expf_hash_load(xw[r], p.expf_hash);
                    yr[r] = lal_expf_rounded(xw[r]);
                } else {
                    bw[r] = expf_bitmap_word(xw[r], p.expf_bits);
                    expf_offsets(xw[r], p.expf_off, &olo[r], &ohi[r]);
                }
            }
        }
    }
    /* at most one superset entry a thread: the candidates are placed in
     * ascending vocab order straight from the superset */
    const bool small = fine && S <= NT;
    /* A shard whose slots dropped nothing exports its whole superset (every
     * key >= the bound L, a set holding {l >= T_shard}) in vocab order: the
     * merge selects the global T among the records in any case, so this
     * rank's own threshold search is left out.  Threshold key 1 is below
     * every real key and above the superset's zero padding. */
    bool export_all = false;
    if (small && local_edges && (p.peer_recv != nullptr || p.shard_out != nullptr) &&
        S <= p.rec_cap) {
        const uint32_t drop = tid < G ? ms->gm[tid] : 0u;
        export_all = __syncthreads_or(drop != 0u) == 0;
    }
    if (fine) {
        /* the superset is padded with zero keys (never greater, never a
         * candidate) to a multiple of 4 for 16-byte reads */
        const int S4 = (S + 3) & ~3;
        const uint4 *K4 = reinterpret_cast<const uint4 *>(Sk);
        if (export_all) {
            T = 1u;
        } else if (S <= 256) {
            /* T = min{ key : #{keys > key} < k } -- one pass per element */
            uint32_t best = 0xffffffffu;
            for (int t = tid; t < S; t += NT) {
                const uint32_t me = Sk[t];
                int gt = 0;
                /* four 16-byte loads in flight: the loop is bound by their
                 * latency, not by the compares */
#pragma unroll 4
                for (int j = 0; j < S4 / 4; ++j) {
                    const uint4 v = K4[j];
                    gt += (v.x > me) + (v.y > me) + (v.z > me) + (v.w > me);
                }
                if (gt < k) best = min(best, me);
            }
            best = __reduce_min_sync(0xffffffffu, best);
            if ((tid & 31) == 0) ms->scan[tid >> 5] = best;
            __syncthreads();
            T = ms->scan[0];
            for (int w = 1; w < NWARP; ++w) T = min(T, ms->scan[w]);
        } else {
            T = block_kth_largest(
                [&](int i, uint32_t &key) {
                    key = Sk[i];
                    return true;
                },
                S, min(k, S), ms);
        }
        /* a slot whose dropped tail reaches T lost candidates: refuse (the
         * barrier also keeps ms->scan until every thread has read T) */
        const uint32_t drop = (local_edges && tid < G) ? ms->gm[tid] : 0u;
        const bool lost = __syncthreads_or(drop != 0u && drop >= T) != 0;
        if (tid == 0) stamp(p, G * 8 + 3);
        if (small) {
            /* a candidate's rank by vocab index among the candidates is its
             * place; the barrier counts them */
            const bool cand = tid < S && Sk[tid] >= T;
            if (cand) {
                const uint32_t me = Sk[tid];
                const int mi = Si[tid];
                const int4 *I4 = reinterpret_cast<const int4 *>(Si);
                int r = 0;
#pragma unroll 4
                for (int j = 0; j < S4 / 4; ++j) {
                    const uint4 v = K4[j];
                    const int4 ix = I4[j];
                    r += (v.x >= T && ix.x < mi) + (v.y >= T && ix.y < mi) +
                         (v.z >= T && ix.z < mi) + (v.w >= T && ix.w < mi);
                }
                if (r < ccap) {
                    Oi[r] = mi;
                    Ov[r] = key2f(me);
                    Ce[r] = !early ? 0.0f
                            : p.expf_hash ? expf_hash_resolve(xw[0], yr[0], hp[0], p.expf_hash,
                                                              p.expf_hash_probe)
                                          : expf_with_range(xw[0], bw[0], olo[0], ohi[0],
                                                            p.expf_x, p.expf_y);
                }
            }
            m = __syncthreads_count(cand);
            fine = m >= 1 && m <= ccap && !lost;
        } else {
            if (early) {
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const int j = tid + r * NT;
                    if (j < S)
                        Ws[j] = p.expf_hash ? expf_hash_resolve(xw[r], yr[r], hp[r], p.expf_hash,
                                                                p.expf_hash_probe)
                                            : expf_with_range(xw[r], bw[r], olo[r], ohi[r],
                                                              p.expf_x, p.expf_y);
                }
            }
            /* candidates {v : l[v] >= T} (superset order) */
            const int seg = (S + NT - 1) / NT;
            const int e0 = min(S, tid * seg), e1 = min(S, e0 + seg);
            uint32_t c = 0;
            for (int e = e0; e < e1; ++e) c += Sk[e] >= T;
            uint32_t mt;
            uint32_t pos = block_scan_excl(c, ms, &mt);
            m = (int)mt;
            if (m <= ccap)
                for (int e = e0; e < e1; ++e)
                    if (Sk[e] >= T) {
                        Cv[pos] = key2f(Sk[e]);
                        Ci[pos] = Si[e];
                        Cw[pos] = early ? Ws[e] : 0.0f;
                        ++pos;
                    }
            fine = m >= 1 && m <= ccap && !lost;
        }
    }
    __syncthreads();

    StreamDiag dg;
    dg.threshold = key2f(T);
    dg.max_l = 0.0f;
    dg.sum = 0.0f;
    dg.r = 0.0f;
    dg.n_cand = m;
    dg.greedy = greedy ? 1 : 0;
    dg.drew = 0;
    dg.token = -1;

    /* leave the scratch clean for the next launch */
    if (!local_edges)
        for (int i = tid; i < kHistWords; i += NT) p.ghist[i] = 0u;
    if (tid == 0) {
        *p.gcount = 0u;
        *p.gL = 0u;
        p.counter[0] = 0u;
    }
    /* ties (or a superset) beyond the fast path's shared memory, or a
     * slice's set beyond its record: the exact wide path */
    const bool shard_wide = fine && (p.peer_recv != nullptr || p.shard_out != nullptr) &&
                            m > p.rec_cap;
    if ((!fine && ok && dev_status == 0) || shard_wide) {
        tail_wide(p, k, greedy, temp, u0, hn, hhead, smem, ms);
        if (p.peer_recv != nullptr) {
            __syncthreads();
            if (tid == 0) stamp(p, G * 8 + 5);
            peer_merge(p, smem, ms);
            if (tid == 0) stamp(p, G * 8 + 7);
        }
        return;
    }
    if (!fine) {
        /* a failed slice still publishes (a failure record): the peers fail
         * the step at once instead of waiting */
        if (p.peer_recv != nullptr) peer_publish(p, ok ? (int)DEV_CAPACITY : (int)DEV_TIMEOUT, 0,
                                                 nullptr, nullptr);
        if (tid == 0) {
            const int st = ok ? (int)DEV_CAPACITY : (int)DEV_TIMEOUT;
            /* a shard reports through its record: the merge fails the step
             * on every rank alike */
            if (dev_status == 0 && p.shard_out == nullptr) atomicCAS(p.status, 0, st);
            if (p.shard_out != nullptr) {
                ShardRecordHead *h = reinterpret_cast<ShardRecordHead *>(p.shard_out);
                h->count = 0;
                h->status = st;
            } else {
                p.tokens[0] = -1;
            }
            p.diag[0] = dg;
            if (p.host_tok) notify_host(p.host_tok, __ldcg(p.seq_in), -1);
        }
        return;
    }

    /* ascending vocab order (placed already for a small superset): rank by
     * counting for small sets, else bitonic */
    if (small) {
    } else if (m <= 64) {
        for (int i = tid; i < m; i += NT) {
            const int me = Ci[i];
            int r = 0;
#pragma unroll 8
            for (int j = 0; j < m; ++j) r += Ci[j] < me;
            Oi[r] = me;
            Ov[r] = Cv[i];
            Ce[r] = Cw[i];
        }
    } else {
        int n2 = 1;
        while (n2 < m) n2 <<= 1;
        for (int i = tid; i < n2; i += NT) {
            Oi[i] = i < m ? Ci[i] : 0x7fffffff;
            Ov[i] = i < m ? Cv[i] : 0.0f;
            Ce[i] = i < m ? Cw[i] : 0.0f;
        }
        __syncthreads();
        for (int size = 2; size <= n2; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < (n2 >> 1); i += NT) {
                    const int lo = (i / stride) * stride * 2 + (i % stride);
                    const int hi = lo + stride;
                    const bool asc = (lo & size) == 0;
                    const int a = Oi[lo], b = Oi[hi];
                    if ((a > b) == asc) {
                        Oi[lo] = b;
                        Oi[hi] = a;
                        float t = Ov[lo];
                        Ov[lo] = Ov[hi];
                        Ov[hi] = t;
                        t = Ce[lo];
                        Ce[lo] = Ce[hi];
                        Ce[hi] = t;
                    }
                }
                __syncthreads();
            }
    }
    __syncthreads();
    if (tid == 0) stamp(p, G * 8 + 4);

    if (p.cand_val_out != nullptr && m <= p.cand_out_cap) {
        for (int i = tid; i < m; i += NT) {
            p.cand_val_out[i] = Ov[i];
            p.cand_idx_out[i] = Oi[i];
        }
    }
    if (p.peer_recv != nullptr) {
        /* vocab-sharded step, peer exchange: publish, wait for every rank's
         * record of this step, merge and draw like merge_kernel */
        peer_publish(p, 0, m, Ov, Oi);
        __syncthreads(); /* Ov / Oi are read before the merge reuses the area */
        if (tid == 0) stamp(p, G * 8 + 5);
        peer_merge(p, smem, ms);
        if (tid == 0) stamp(p, G * 8 + 7);
        return;
    }
    if (p.shard_out != nullptr) {
        /* vocab-sharded step: this slice's record (list form); the merge draws */
        ShardRecordHead *h = reinterpret_cast<ShardRecordHead *>(p.shard_out);
        float *rv = reinterpret_cast<float *>(p.shard_out + sizeof(ShardRecordHead));
        int *ri = reinterpret_cast<int *>(rv + p.rec_cap);
        for (int i = tid; i < m; i += NT) {
            rv[i] = Ov[i];
            ri[i] = Oi[i];
        }
        if (tid == 0) {
            h->count = m;
            h->status = 0;
            h->ties = 0;
            h->tkey = 0u;
            p.diag[0] = dg;
        }
        return;
    }
    if (p.candidates_only) {
        if (tid == 0) p.diag[0] = dg;
        return;
    }

    /* max over candidates, floored at -1e30f (runtime/lal_sampling.h:107-109) */
    if (!early) {
        float mx = -1e30f;
        for (int i = tid; i < m; i += NT) mx = fmaxf(mx, Ov[i]);
        max_l = block_max_f(mx, ms);
    }
    if (tid == 0) stamp(p, G * 8 + 5);
    dg.max_l = max_l;
    int token;
    if (greedy) {
        token = Oi[0];
    } else {
        /* weights expf((l - max_l) / T) (runtime/lal_sampling.h:112), unless
         * they came with the candidates */
        if (!early)
            for (int i = tid; i < m; i += NT) {
                const float x = __fdiv_rn(__fsub_rn(Ov[i], max_l), temp);
                Ce[i] = p.expf_hash ? expf_hash_finish(x, expf_hash_load(x, p.expf_hash),
                                                       p.expf_hash, p.expf_hash_probe)
                                    : sampler_expf(x, p.expf_x, p.expf_y, p.expf_bits, p.expf_off);
            }
        __syncthreads();
        /* the GPT-2 server's nucleus: the dropped rows' terms become 0 (its
         * draw walks every row, zeros included) */
        if (p.variant == VARIANT_GPT2 && p.top_p > 0.0f && p.top_p < 1.0f)
            dg.n_cand = gpt2_nucleus(p.top_p, m, Ce, Cv, Ci, Cw, ms);
        /* sequential float sum in ascending vocab order; keep the prefix
         * (values fetched eight at a time, the adds stay in order) */
        if (tid == 0) {
            float acc = 0.0f;
            int i = 0;
            for (; i + 8 <= m; i += 8) {
                float v[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) v[q] = Ce[i + q];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    acc = __fadd_rn(acc, v[q]);
                    Ce[i + q] = acc;
                }
            }
            for (; i < m; ++i) {
                acc = __fadd_rn(acc, Ce[i]);
                Ce[i] = acc;
            }
            ms->sum = acc;
            ms->found = 0x7fffffff;
        }
        __syncthreads();
        const float sum = ms->sum;
        if (tid == 0) stamp(p, G * 8 + 6);
        dg.sum = sum;
        if (p.variant == VARIANT_SERVER && sum <= 0.0f) {
            /* tools/server/qwen7b_server.c:285-286: argmax over the kept
             * candidates with '>' from -1e30f, no draw */
            token = 0;
            float bv = -1e30f;
            if (tid == 0)
                for (int i = 0; i < m; ++i)
                    if (Ov[i] > bv) {
                        bv = Ov[i];
                        token = Oi[i];
                    }
        } else {
            /* r = u * sum; first candidate with r <= running sum
             * (runtime/lal_sampling.h:116-124) */
            const float r = __fmul_rn(u0, sum);
            dg.r = r;
            dg.drew = 1;
            int first = 0x7fffffff;
            for (int i = tid; i < m; i += NT)
                if (r <= Ce[i]) {
                    first = i;
                    break;
                }
            if (first != 0x7fffffff) atomicMin(&ms->found, first);
            __syncthreads();
            token = ms->found != 0x7fffffff ? Oi[ms->found] : p.vocab - 1;
            /* gpt2_server.c:2996-3001 walks every row, adding zeros below T:
             * a draw of exactly 0 stops at row 0 */
            if (p.variant == VARIANT_GPT2 && r == 0.0f) token = 0;
        }
    }
    if (tid == 0) {
        dg.token = token;
        p.tokens[0] = token;
        p.diag[0] = dg;
        if (p.push_history && p.hist_cap > 0) {
            /* runtime/lal_sampling.h:133-136 as a ring: FIFO at hist_cap */
            const int n = hn;
            if (n < p.hist_cap) {
                p.hist_ids[n] = token;
                p.hist_n[0] = n + 1;
            } else {
                const int h = hhead;
                p.hist_ids[h] = token;
                p.hist_head[0] = (h + 1) % p.hist_cap;
            }
        }
        if (p.host_tok) notify_host(p.host_tok, __ldcg(p.seq_in), token);
        stamp(p, G * 8 + 7);
    }
}

/* ------------------------------------------------- auxiliary kernels --- */

/* lal_quantize_x_int8 for the drop-in: one CTA. */
__global__ void __launch_bounds__(NT) quantize_x_kernel(const float *x, int8_t *xq,
                                                        float *scale_out, int n) {
    __shared__ Misc ms;
    float m = 0.0f;
    for (int i = threadIdx.x; i < n; i += NT) m = fmaxf(m, fabsf(x[i]));
    m = block_max_f(m, &ms);
    float scale = __fdiv_rn(m, 127.0f);
    if (scale < 1e-8f) scale = 1e-8f;
    const float inv = __fdiv_rn(1.0f, scale);
    const int n8 = n & ~7;
    for (int i = threadIdx.x; i < n; i += NT) {
        const float s = __fmul_rn(x[i], inv);
        int v;
        if (s != s) v = -127;
        else {
            v = (i < n8) ? __float2int_rn(s) : __float2int_rz(s);
            v = v > 127 ? 127 : (v < -127 ? -127 : v);
        }
        xq[i] = (int8_t)v;
    }
    if (threadIdx.x == 0) *scale_out = scale;
}

/* A step's inputs from mapped pinned host memory (src) into device memory
 * (dst): words [0, n0) and [off1, off1 + n1).  The next kernel may launch at
 * once (it streams the LM head, which no step writes) and waits for this
 * one's completion before it reads the inputs. */
__global__ void __launch_bounds__(256) stage_inputs_kernel(const float *src, float *dst, int n0,
                                                           int off1, int n1) {
    grid_dep_launch_dependents();
    const int stride = gridDim.x * blockDim.x;
    const int i0 = blockIdx.x * blockDim.x + threadIdx.x;
    if (((n0 | off1) & 3) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int i = i0; i < n0 / 4; i += stride) d4[i] = s4[i];
    } else {
        for (int i = i0; i < n0; i += stride) dst[i] = src[i];
    }
    for (int i = i0; i < n1; i += stride) dst[off1 + i] = src[off1 + i];
}

__global__ void abs_xq_kernel(const int8_t *xq, uint8_t *ax, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const int v = xq[i];
        ax[i] = (uint8_t)(v < 0 ? -v : v);
    }
}

/* lroundf without the library: round half away from zero (exact for the
 * |v| < 2^23 range the quantizer sees; larger values are already integers). */
__device__ __forceinline__ int round_half_away(float v) {
    const float t = truncf(v);
    const float frac = __fsub_rn(v, t);
    float r = t;
    if (frac >= 0.5f) r = __fadd_rn(t, 1.0f);
    else if (frac <= -0.5f) r = __fsub_rn(t, 1.0f);
    if (r > 2147483520.0f) return 0x7fffffff;
    if (r < -2147483648.0f) return (int)0x80000000u;
    return (int)r;
}

/* lal_quantize_q8_per_row (runtime/lal_q8_kernel.h:357-372): one warp per
 * row; absmax, scale = max/127 floored at 1e-8, q = clamp(lroundf(w*inv)). */
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float *W, int d, int8_t *q,
                                                            int ld, float *scale, int n_rows) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= n_rows) return;
    const float *row = W + (size_t)warp * d;
    float m = 0.0f;
    for (int i = lane; i < d; i += 32) m = fmaxf(m, fabsf(row[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = __fdiv_rn(m, 127.0f);
    if (s < 1e-8f) s = 1e-8f;
    const float inv = __fdiv_rn(1.0f, s);
    int8_t *out = q + (size_t)warp * ld;
    for (int i = lane; i < ld; i += 32) {
        int v = 0;
        if (i < d) {
            v = round_half_away(__fmul_rn(row[i], inv));
            v = v > 127 ? 127 : (v < -127 ? -127 : v);
        }
        out[i] = (int8_t)v;
    }
    if (lane == 0) scale[warp] = s;
}

/* One CTA: the kept-candidate softmax of qwen7b_server.c:271-294. */
__global__ void __launch_bounds__(NT) finish_kernel(const FinishParams f) {
    __shared__ Misc ms;
    const int tid = threadIdx.x;
    auto val = [&](int i) { return f.cand_val ? f.cand_val[i] : __ldcg(f.logits + f.cand_idx[i]); };
    auto kept = [&](int i) { return f.keep == nullptr || f.keep[i] != 0; };
    if (f.phase == 0) {
        /* the largest kept value with '>' from -1e30f (max over equal values
         * is the same as fmaxf's) */
        float mx = -1e30f;
        for (int i = tid; i < f.m; i += NT)
            if (kept(i)) mx = fmaxf(mx, val(i));
        const float max_l = block_max_f(mx, &ms);
        for (int i = tid; i < f.m; i += NT)
            f.prefix[i] = kept(i) ? sampler_expf(__fdiv_rn(__fsub_rn(val(i), max_l),
                                                           f.temperature),
                                                 f.expf_x, f.expf_y, f.expf_bits, f.expf_off)
                                  : 0.0f;
        __syncthreads();
        if (tid == 0) {
            float acc = 0.0f, bv = -1e30f;
            int best = 0;
            for (int i = 0; i < f.m; ++i) {
                if (!kept(i)) continue;
                acc = __fadd_rn(acc, f.prefix[i]);
                f.prefix[i] = acc;
                const float v = val(i);
                if (v > bv) {
                    bv = v;
                    best = f.cand_idx[i];
                }
            }
            f.diag->max_l = max_l;
            f.diag->sum = acc;
            f.diag->token = best; /* argmax fallback, used when sum <= 0 */
        }
    } else {
        if (tid == 0) ms.found = 0x7fffffff;
        __syncthreads();
        const float r = __fmul_rn(f.u[0], f.diag->sum);
        int first = 0x7fffffff;
        for (int i = tid; i < f.m; i += NT)
            if (kept(i) && r <= f.prefix[i]) {
                first = i;
                break;
            }
        if (first != 0x7fffffff) atomicMin(&ms.found, first);
        __syncthreads();
        if (tid == 0) {
            int tok = ms.found != 0x7fffffff ? f.cand_idx[ms.found] : f.vocab - 1;
            /* gpt2_server.c:2996-3001 walks every row: a draw of exactly 0
             * stops at row 0 */
            if (f.variant == VARIANT_GPT2 && r == 0.0f) tok = 0;
            f.diag->r = r;
            f.diag->drew = 1;
            f.diag->token = tok;
            *f.token = tok;
        }
    }
}

__global__ void debug_expf_kernel(const float *x, float *y, int n, const uint32_t *tx,
                                  const uint32_t *ty, const uint32_t *bits,
                                  const uint32_t *off, const uint4 *hash, int hash_probe) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        y[i] = hash ? expf_hash_finish(x[i], expf_hash_load(x[i], hash), hash, hash_probe)
                    : sampler_expf(x[i], tx, ty, bits, off);
}

/* Vocab-sharded step, second half: CTA b merges stream b's records from every
 * rank and samples exactly as the unsharded last CTA does.  The records are
 * concatenated in rank order; the slices are contiguous and rank-ordered, so
 * the concatenation is in ascending vocab order, the order of the
 * reference's sequential softmax sums (runtime/lal_sampling.h:110-124).
 * Every rank runs the same merge on the same bytes and gets the same token. */
/* The history push of a merged stream (runtime/lal_sampling.h:133-136 as a
 * ring: FIFO at hist_cap). */
__device__ __forceinline__ void merge_push(const MergeParams &mp, int b, int token, int hn,
                                           int hhead) {
    if (mp.push_history && mp.hist_cap > 0) {
        int *ids = mp.hist_ids + (size_t)b * mp.hist_cap;
        if (hn < mp.hist_cap) {
            ids[hn] = token;
            mp.hist_n[b] = hn + 1;
        } else {
            ids[hhead] = token;
            mp.hist_head[b] = (hhead + 1) % mp.hist_cap;
        }
    }
}

/* The merge when some record is in the wide form (tail_wide.cuh): T is the
 * k-th largest of the entries and of every wide record's ties (each T_shard
 * counted `ties` times); the candidates are the entries >= T and the ties of
 * the records whose T_shard equals T; the walk adds their weights record by
 * record in rank order, a record's entries and bitmap rows in ascending
 * index order. */
template <class Load>
__device__ void merge_wide(const MergeParams &mp, int b, MergeHead &hd, const uint32_t *Mk,
                           const int *Mi, float *Mw, uint8_t *walk, Misc *ms, const Load &load,
                           StreamDiag dg, bool greedy, float temp, int topk, float u0, int hn,
                           int hhead) {
    const int tid = threadIdx.x;
    const int M = hd.roff[mp.n_ranks];
    uint32_t total = (uint32_t)M;
    for (int r = 0; r < mp.n_ranks; ++r) total += (uint32_t)hd.rties[r];
    uint32_t k = greedy ? 1u : (uint32_t)max(topk, 1);
    if (k > (uint32_t)mp.vocab) k = (uint32_t)mp.vocab;
    if (k > total) k = total;
    if (k < 1u) k = 1u;
    uint32_t mk = 0u;
    for (int e = tid; e < M; e += NT) mk = max(mk, Mk[e]);
    if (tid < mp.n_ranks && hd.rties[tid] > 0) mk = max(mk, hd.rtkey[tid]);
    const uint32_t top = block_max_u32(mk, ms);
    const uint32_t T = block_kth_largest_w(
        [&](int i, uint32_t &key, uint32_t &w) {
            if (i < M) {
                key = Mk[i];
                w = 1u;
                return true;
            }
            key = hd.rtkey[i - M];
            w = (uint32_t)hd.rties[i - M];
            return hd.rties[i - M] > 0;
        },
        M + mp.n_ranks, k, ms);
    const float max_l = fmaxf(-1e30f, key2f(top));
    const ExpfTables ex{mp.expf_x, mp.expf_y, mp.expf_bits, mp.expf_off, mp.expf_hash,
                        mp.expf_hash_probe};
    uint32_t c = 0u;
    for (int e = tid; e < M; e += NT) {
        Mw[e] = greedy ? 0.0f : ex.weight(key2f(Mk[e]), max_l, temp);
        c += Mk[e] >= T;
    }
    uint32_t n_exp;
    block_scan_excl(c, ms, &n_exp);
    uint32_t n_tie = 0u;
    for (int r = 0; r < mp.n_ranks; ++r)
        if (hd.rties[r] > 0 && hd.rtkey[r] == T) n_tie += (uint32_t)hd.rties[r];
    if (tid == 0) ms->fred[0] = greedy ? 0.0f : ex.weight(key2f(T), max_l, temp);
    __syncthreads();
    const float wT = ms->fred[0];
    uint32_t *bm = reinterpret_cast<uint32_t *>(walk);
    WideChunk *tab = reinterpret_cast<WideChunk *>(bm + kWideChunkWords);
    const WalkResult res = wide_walk(
        mp.n_ranks,
        [&](int r) {
            const int r0 = (int)((long long)r * mp.vocab / mp.n_ranks);
            const int r1 = (int)((long long)(r + 1) * mp.vocab / mp.n_ranks);
            const int o = hd.roff[r];
            return WalkUnit{Mk + o, Mi + o, Mw + o, hd.roff[r + 1] - o,
                            hd.rties[r] > 0 && hd.rtkey[r] == T, r0, r1 - r0};
        },
        [&](int r, int w0, int nw, uint32_t *dst) { load.bitmap(r, w0, nw, dst); }, T, wT,
        greedy, u0, mp.variant, bm, tab, ms);
    dg.threshold = key2f(T);
    dg.max_l = max_l;
    dg.n_cand = (int)(n_exp + n_tie);
    dg.sum = greedy ? 0.0f : res.sum;
    dg.r = res.r;
    dg.drew = res.drew;
    if (tid == 0) {
        if (!res.ok) {
            atomicCAS(mp.status, 0, (int)DEV_TIMEOUT);
            mp.tokens[b] = -1;
            mp.diag[b] = dg;
        } else {
            const int token = res.token >= 0 ? res.token : mp.vocab - 1;
            dg.token = token;
            mp.tokens[b] = token;
            mp.diag[b] = dg;
            merge_push(mp, b, token, hn, hhead);
        }
    }
    __syncthreads();
}

/* The merge when the gathered entries fit two a thread (M <= 2 NT: N
 * records of about k entries each, the usual case).  Thread t holds entries
 * t and t + NT; the concatenated records are in ascending vocab order
 * already, so a candidate's place in the draw order is the number of
 * candidates before it in entry order.  Five barriers: threshold and
 * maximum, places, weights in place, the sequential sum (one thread), the
 * draw. */
__device__ __noinline__ void merge_small(const MergeParams &mp, int b, int M, const uint32_t *Mk,
                                         const int *Mi, float *Cw, Misc *ms, StreamDiag dg,
                                         bool greedy, float temp, int topk, float u0, int hn,
                                         int hhead) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    auto mstamp = [&](int i) {
        if (mp.phase_ts && tid == 0) mp.phase_ts[i] = gtimer();
    };
    bool have[2];
    uint32_t me[2];
    int mi[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int e = tid + h * NT;
        have[h] = e < M;
        me[h] = have[h] ? Mk[e] : 0u;
        mi[h] = have[h] ? Mi[e] : 0;
    }
    /* k = min(top_k, V) (runtime/lal_sampling.h:70-71), 1 for greedy; every
     * shard exported at least min(k, its rows) entries */
    int k = greedy ? 1 : topk;
    if (k > mp.vocab) k = mp.vocab;
    if (k > M) k = M;
    if (k < 1) k = 1;
    /* the largest key first (max_l, runtime/lal_sampling.h:107-109): every
     * entry's weight table load then goes out before the threshold count,
     * which hides its latency */
    {
        const uint32_t wmx = __reduce_max_sync(0xffffffffu, max(me[0], me[1]));
        if (lane == 0) ms->wmax[warp] = wmx;
    }
    __syncthreads();
    uint32_t mx = ms->wmax[0];
    for (int w = 1; w < NWARP; ++w) mx = max(mx, ms->wmax[w]);
    const float max_l = fmaxf(-1e30f, key2f(mx));
    float xw[2] = {0.0f, 0.0f}, yr[2] = {0.0f, 0.0f};
    uint4 hp[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
    const bool early_w = !greedy && mp.expf_hash != nullptr;
    if (early_w)
#pragma unroll
        for (int h = 0; h < 2; ++h)
            if (have[h]) {
                xw[h] = __fdiv_rn(__fsub_rn(key2f(me[h]), max_l), temp);
                hp[h] = expf_hash_load(xw[h], mp.expf_hash);
                yr[h] = lal_expf_rounded(xw[h]);
            }
    /* T = min{ key : #{keys > key} < k } (the k-th largest with
     * multiplicity) */
    int gt[2] = {0, 0};
    {
        const uint4 *K4 = reinterpret_cast<const uint4 *>(Mk);
        int j = 0;
        if ((reinterpret_cast<uintptr_t>(Mk) & 15u) == 0)
#pragma unroll 4
            for (; j + 4 <= M; j += 4) {
                const uint4 v = K4[j >> 2];
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    gt[h] += (v.x > me[h]) + (v.y > me[h]) + (v.z > me[h]) + (v.w > me[h]);
            }
        for (; j < M; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) gt[h] += Mk[j] > me[h];
    }
    uint32_t best = 0xffffffffu;
#pragma unroll
    for (int h = 0; h < 2; ++h)
        if (have[h] && gt[h] < k) best = min(best, me[h]);
    best = __reduce_min_sync(0xffffffffu, best);
    if (lane == 0) ms->scan[warp] = best;
    if (tid == 0) ms->found = -1;
    __syncthreads();
    uint32_t T = ms->scan[0];
    for (int w = 1; w < NWARP; ++w) T = min(T, ms->scan[w]);
    mstamp(0);
    /* candidates {l >= T} and their places; each one's weight
     * expf((l - max_l) / T) (runtime/lal_sampling.h:107-112) */
    const ExpfTables ex{mp.expf_x, mp.expf_y, mp.expf_bits, mp.expf_off, mp.expf_hash,
                        mp.expf_hash_probe};
    bool cand[2];
    unsigned bal[2];
    float w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        cand[h] = have[h] && me[h] >= T;
        bal[h] = __ballot_sync(0xffffffffu, cand[h]);
        if (lane == 0) ms->hist[h * NWARP + warp] = (uint32_t)__popc(bal[h]);
        w[h] = !cand[h] || greedy ? 0.0f
               : early_w ? expf_hash_resolve(xw[h], yr[h], hp[h], mp.expf_hash, mp.expf_hash_probe)
                         : ex.weight(key2f(me[h]), max_l, temp);
    }
    __syncthreads();
    int off[2] = {0, 0}, m = 0;
    for (int v = 0; v < 2 * NWARP; ++v) {
        const int c = (int)ms->hist[v];
        off[0] += v < warp ? c : 0;
        off[1] += v < NWARP + warp ? c : 0;
        m += c;
    }
    int pos[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        pos[h] = off[h] + __popc(bal[h] & ((1u << lane) - 1u));
        if (cand[h]) Cw[pos[h]] = w[h];
        if (cand[h] && pos[h] == 0) ms->sh[15] = (uint32_t)mi[h]; /* the first candidate */
    }
    __syncthreads();
    mstamp(1);
    dg.threshold = key2f(T);
    dg.max_l = max_l;
    dg.n_cand = m;
    int token = (int)ms->sh[15];
    if (!greedy) {
        /* sequential float sum in ascending vocab order, the running sums in
         * place (values fetched eight at a time, the adds in order) */
        if (tid == 0) {
            float acc = 0.0f;
            int i = 0;
            for (; i + 8 <= m; i += 8) {
                float v[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) v[q] = Cw[i + q];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    acc = __fadd_rn(acc, v[q]);
                    Cw[i + q] = acc;
                }
            }
            for (; i < m; ++i) {
                acc = __fadd_rn(acc, Cw[i]);
                Cw[i] = acc;
            }
            ms->sum = acc;
        }
        __syncthreads();
        mstamp(2);
        const float sum = ms->sum;
        dg.sum = sum;
        if (mp.variant == VARIANT_SERVER && sum <= 0.0f) {
            /* tools/server/qwen7b_server.c:285-286, the argmax over the kept
             * candidates with '>' from -1e30f: the sum is 0 only when every
             * candidate lies at or below -1e30 (the largest one weighs
             * expf(0) = 1 otherwise), so that argmax keeps row 0 */
            token = 0;
        } else {
            /* r = u * sum; the first candidate with r <= its running sum
             * (runtime/lal_sampling.h:116-124): the sums do not decrease, so
             * it is the one whose predecessor's sum is below r */
            const float r = __fmul_rn(u0, sum);
            dg.r = r;
            dg.drew = 1;
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (cand[h] && r <= Cw[pos[h]] && !(pos[h] > 0 && r <= Cw[pos[h] - 1]))
                    ms->found = mi[h];
            __syncthreads();
            token = ms->found >= 0 ? ms->found : mp.vocab - 1;
            if (mp.variant == VARIANT_GPT2 && r == 0.0f) token = 0;
        }
    }
    mstamp(4);
    if (tid == 0) {
        dg.token = token;
        mp.tokens[b] = token;
        mp.diag[b] = dg;
        merge_push(mp, b, token, hn, hhead);
    }
}

/* The merge of stream b's N shard records and its draw, by one CTA (NT
 * threads): shared by merge_kernel (records all-gathered into global memory)
 * and the fused kernel's peer exchange (records written by the peers over
 * NVLink, polled word by word).  load() fills the MergeHead (prefix offsets
 * of the entries, a DEV_* failure or 0, each record's form) and the keys /
 * vocab ids of the concatenated records' entries in ascending vocab order,
 * then synchronises the CTA; load.bitmap() stages a wide record's bitmap.
 * area: kMergeHead bytes + 24 bytes per entry (mp.smem_cap of them) +
 * kWideWalkBytes. */
template <class Load>
__device__ void merge_sample(const MergeParams &mp, int b, uint8_t *area, Misc *ms, Load load) {
    MergeHead &hd = *reinterpret_cast<MergeHead *>(area);
    const int tid = threadIdx.x;
    const int cap = mp.smem_cap;
    uint32_t *Mk = reinterpret_cast<uint32_t *>(area + kMergeHead);
    int *Mi = reinterpret_cast<int *>(Mk + cap);
    float *Mw = reinterpret_cast<float *>(Mi + cap);
    float *Cv = Mw + cap;
    int *Ci = reinterpret_cast<int *>(Cv + cap);
    float *Ce = reinterpret_cast<float *>(Ci + cap);

    const float temp = mp.temperature[b];
    const int topk = mp.top_k[b];
    const float u0 = mp.u[b];
    const int hn = mp.hist_n ? mp.hist_n[b] : 0;
    const int hhead = mp.hist_head ? mp.hist_head[b] : 0;
    const bool greedy = (temp <= 0.0f) || (topk <= 0);
    load(hd, Mk, Mi, cap, Ce);
    StreamDiag dg;
    dg.threshold = 0.0f;
    dg.max_l = 0.0f;
    dg.sum = 0.0f;
    dg.r = 0.0f;
    dg.n_cand = 0;
    dg.greedy = greedy ? 1 : 0;
    dg.drew = 0;
    dg.token = -1;
    if (hd.rbad != 0) {
        if (tid == 0) {
            atomicCAS(mp.status, 0, hd.rbad);
            mp.tokens[b] = -1;
            mp.diag[b] = dg;
        }
        return;
    }
    if (hd.wide) {
        merge_wide(mp, b, hd, Mk, Mi, Mw, area + kMergeHead + 24 * cap, ms, load, dg, greedy, temp,
                   topk, u0, hn, hhead);
        return;
    }
    const int M = hd.roff[mp.n_ranks];
    if (M <= 2 * NT) {
        merge_small(mp, b, M, Mk, Mi, Ce, ms, dg, greedy, temp, topk, u0, hn, hhead);
        return;
    }
    /* k = min(top_k, V) (runtime/lal_sampling.h:70-71), 1 for greedy; every
     * shard exported at least min(k, its rows) entries, so M >= k */
    int k = greedy ? 1 : topk;
    if (k > mp.vocab) k = mp.vocab;
    if (k > M) k = M;
    if (k < 1) k = 1;
    /* max_l = the largest entry (every shard's record holds its maximum, and
     * the overall maximum is a candidate), floored at -1e30f
     * (runtime/lal_sampling.h:107-109): the weights need not wait for T */
    uint32_t mk = 0u;
    for (int e = tid; e < M; e += NT) mk = max(mk, Mk[e]);
    mk = __reduce_max_sync(0xffffffffu, mk);
    if ((tid & 31) == 0) ms->scan[tid >> 5] = mk;
    __syncthreads();
    uint32_t mx = ms->scan[0];
    for (int w = 1; w < NWARP; ++w) mx = max(mx, ms->scan[w]);
    __syncthreads();
    const float max_l = fmaxf(-1e30f, key2f(mx));
    dg.max_l = max_l;
    auto mstamp = [&](int i) {
        if (mp.phase_ts && tid == 0) mp.phase_ts[i] = gtimer();
    };
    mstamp(0);
    /* weights expf((l - max_l) / T) (runtime/lal_sampling.h:112) of every
     * entry, then T by the radix select (more than 2 NT entries) */
    if (!greedy)
        for (int e = tid; e < M; e += NT) {
            const float x = __fdiv_rn(__fsub_rn(key2f(Mk[e]), max_l), temp);
            Mw[e] = mp.expf_hash ? expf_hash_finish(x, expf_hash_load(x, mp.expf_hash),
                                                    mp.expf_hash, mp.expf_hash_probe)
                                 : sampler_expf(x, mp.expf_x, mp.expf_y, mp.expf_bits,
                                                mp.expf_off);
        }
    const uint32_t T = block_kth_largest(
        [&](int i, uint32_t &key) {
            key = Mk[i];
            return true;
        },
        M, k, ms);
    mstamp(1);
    /* candidates {l >= T}, order kept (stable compaction), with weights */
    const int seg = (M + NT - 1) / NT;
    const int e0 = min(M, tid * seg), e1 = min(M, e0 + seg);
    uint32_t c = 0;
    for (int e = e0; e < e1; ++e) c += Mk[e] >= T;
    uint32_t mt;
    uint32_t pos = block_scan_excl(c, ms, &mt);
    const int m = (int)mt;
    for (int e = e0; e < e1; ++e)
        if (Mk[e] >= T) {
            Cv[pos] = key2f(Mk[e]);
            Ci[pos] = Mi[e];
            Ce[pos] = greedy ? 0.0f : Mw[e];
            ++pos;
        }
    __syncthreads();
    mstamp(2);
    dg.threshold = key2f(T);
    dg.n_cand = m;
    int token;
    if (greedy) {
        token = Ci[0];
    } else {
        /* sequential float sum in ascending vocab order; keep the prefix */
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
        mstamp(3);
        const float sum = ms->sum;
        dg.sum = sum;
        if (mp.variant == VARIANT_SERVER && sum <= 0.0f) {
            /* tools/server/qwen7b_server.c:285-286 */
            token = 0;
            float bv = -1e30f;
            for (int i = 0; i < m; ++i)
                if (Cv[i] > bv) {
                    bv = Cv[i];
                    token = Ci[i];
                }
        } else {
            /* r = u * sum; first candidate with r <= running sum
             * (runtime/lal_sampling.h:116-124) */
            const float r = __fmul_rn(u0, sum);
            dg.r = r;
            dg.drew = 1;
            int first = 0x7fffffff;
            for (int i = tid; i < m; i += NT)
                if (r <= Ce[i]) {
                    first = i;
                    break;
                }
            if (first != 0x7fffffff) atomicMin(&ms->found, first);
            __syncthreads();
            token = ms->found != 0x7fffffff ? Ci[ms->found] : mp.vocab - 1;
        }
    }
    mstamp(4);
    if (tid == 0) {
        dg.token = token;
        mp.tokens[b] = token;
        mp.diag[b] = dg;
        merge_push(mp, b, token, hn, hhead);
    }
}

/* Loader of all-gathered records (ShardRecordHead + values + ids + bitmap)
 * in global memory: records of stream b from rank r at recv + r*rank_stride
 * + b*rec_bytes. */
struct GatheredRecords {
    const MergeParams &mp;
    int b;
    __device__ const uint8_t *rec(int r) const {
        return mp.recv + r * mp.rank_stride + (long long)b * mp.rec_bytes;
    }
    __device__ void operator()(MergeHead &hd, uint32_t *Mk, int *Mi, int cap, float *) const {
        const int tid = threadIdx.x;
        if (tid == 0) {
            int acc = 0, st = 0, wide = 0;
            for (int r = 0; r < mp.n_ranks; ++r) {
                const ShardRecordHead *h = reinterpret_cast<const ShardRecordHead *>(rec(r));
                const int c = __ldcg(&h->count), s = __ldcg(&h->status);
                const int ties = __ldcg(&h->ties);
                if (s != 0 && st == 0) st = s;
                const bool bad = c < 0 || c > mp.rec_cap || ties < 0;
                if (bad && st == 0) st = DEV_CAPACITY;
                hd.rties[r] = bad ? 0 : ties;
                hd.rtkey[r] = __ldcg(&h->tkey);
                if (!bad && ties > 0) wide = 1;
                hd.roff[r] = acc;
                acc += bad ? 0 : c;
            }
            hd.roff[mp.n_ranks] = acc;
            if ((acc > cap || (acc < 1 && !wide)) && st == 0) st = DEV_CAPACITY;
            hd.rbad = st;
            hd.wide = wide;
        }
        __syncthreads();
        if (hd.rbad != 0) return;
        for (int r = 0; r < mp.n_ranks; ++r) {
            const int c = hd.roff[r + 1] - hd.roff[r];
            const float *rv = reinterpret_cast<const float *>(rec(r) + sizeof(ShardRecordHead));
            const int *ri = reinterpret_cast<const int *>(rv + mp.rec_cap);
            for (int i = tid; i < c; i += NT) {
                Mk[hd.roff[r] + i] = f2key(__ldcg(rv + i));
                Mi[hd.roff[r] + i] = __ldcg(ri + i);
            }
        }
        __syncthreads();
    }
    /* nw bitmap words of rank r's wide record from word w0 (every thread) */
    __device__ void bitmap(int r, int w0, int nw, uint32_t *dst) const {
        const uint32_t *bm = reinterpret_cast<const uint32_t *>(
            rec(r) + sizeof(ShardRecordHead) + 8 * (size_t)mp.rec_cap);
        for (int i = threadIdx.x; i < nw; i += NT) dst[i] = __ldcg(bm + w0 + i);
    }
};

__global__ void __launch_bounds__(NT) merge_kernel(const MergeParams mp) {
    extern __shared__ __align__(16) uint8_t msm[];
    __shared__ Misc msh;
    merge_sample(mp, blockIdx.x, msm, &msh, GatheredRecords{mp, (int)blockIdx.x});
}

/* -------------------------------------------------- host planning --- */
template <int MODE>
void *pick_kernel(int nch) {
    switch (nch) {
        case 1: return (void *)tail_kernel<MODE, 1>;
        case 2: return (void *)tail_kernel<MODE, 2>;
        case 4: return (void *)tail_kernel<MODE, 4>;
        case 7: return (void *)tail_kernel<MODE, 7>;
        case 8: return (void *)tail_kernel<MODE, 8>;
        case 16: return (void *)tail_kernel<MODE, 16>;
        default: return nullptr;
    }
}

int round_nch(int ld) {
    const int need = (ld + 511) / 512;
    const int opts[] = {1, 2, 4, 7, 8, 16};
    for (int o : opts)
        if (o >= need) return o;
    return -1;
}

constexpr int kSmemLimit = 232448; /* 227 KB dynamic per block on sm_100 */
constexpr int kStageTargetBytes = 57344; /* bytes of W per bulk-copy stage */

int align_up(int v, int a) { return (v + a - 1) / a * a; }

}  // namespace

/* Fills the launch geometry and shared-memory layout of p; returns the grid
 * size, or a negative value when the shape is unsupported. */
int plan_launch(TailParams &p, int num_sms, int min_rows_per_cta) {
    if (p.rows < 1) return -1;
    int G = (p.rows + min_rows_per_cta - 1) / min_rows_per_cta;
    G = std::min(G, std::min(num_sms, kMaxGrid));
    G = std::max(G, 1);
    p.rows_per_cta_max = (p.rows + G - 1) / G;
    if (p.rows_per_cta_max > kMaxRowsPerCta) return -2;
    p.nch = p.mode == MODE_SAMPLE ? 1 : round_nch(p.ld);
    if (p.nch < 0) return -3;
    const int rpc = align_up(p.rows_per_cta_max, 4);
    int off = 0;
    const int hist_bytes = p.mode == MODE_LMHEAD ? 0 : 4 * 4096;
    const int fixed = 16 * kMaxStages + align_up(p.ld, 16) + 3 * 4 * rpc + hist_bytes +
                      align_up((int)sizeof(Misc), 128) + 3 * 128;
    const int budget = (kSmemLimit - fixed) / 128 * 128;
    if (p.mode == MODE_SAMPLE) {
        p.stages = 0;
        p.rows_per_stage = 0;
        p.stage_bytes = 0;
        p.area_bytes = budget;
    } else {
        /* Few large stages: on B200 a ring of 3 x 56 KB bulk copies streams a
         * 545 MB slice in 94 us/step, 6 x 28 KB in 106 us and 14 KB copies
         * slower still.  A stage is about 56 KB of whole rows, a multiple of
         * 4 KB where the row length allows it. */
        const int unit = 4096 / std::gcd(p.ld, 4096);
        int R = (kStageTargetBytes / p.ld) / unit * unit;
        if (R < 1) R = std::max(1, kStageTargetBytes / p.ld);
        p.rows_per_stage = R;
        p.stage_bytes = align_up(R * p.ld, 128);
        p.stages = std::min(kMaxStages, budget / p.stage_bytes);
        if (p.stages < 2) return -4;
        /* stages issued before the previous kernel completes: two, or the
         * whole ring when a CTA's slice is short (a vocab shard), where the
         * prefetched part is a large share of its rows */
        p.early_stages = (long long)p.rows_per_cta_max * p.ld <= 12ll * p.stage_bytes
                             ? p.stages : std::min(kEarlyStages, p.stages);
        p.area_bytes = p.stages * p.stage_bytes;
        /* after the rows, the stage area holds the local key histogram and,
         * in the last CTA, the superset and the candidates */
        if (p.mode == MODE_FUSED) p.area_bytes = std::max(p.area_bytes, std::min(budget, 96 << 10));
    }
    /* the last CTA needs room for the candidates (k plus ties) and the key
     * histogram of 4096 bins */
    if (p.mode != MODE_LMHEAD) {
        /* k plus ties in power-of-two candidate arrays (28 B an entry) next to
         * a superset of k plus a boundary bin (8 B an entry) */
        int c2 = 1;
        while (c2 < p.max_k + 64) c2 <<= 1;
        if (p.area_bytes < 16384 || 28 * c2 + 8 * (p.max_k + 64 + kRefineMax) > p.area_bytes)
            return -5;
        /* the wide path's explicit rows (fewer than k) and walk tables */
        if (wide_area_bytes(std::max(1, p.max_k)) > p.area_bytes) return -7;
    }
    off = align_up(p.area_bytes, 128);
    p.off_bars = off;
    off += 16 * kMaxStages;
    p.off_xq = off;
    off += align_up(p.ld, 16);
    off = align_up(off, 16);
    p.off_sw = off;
    off += 4 * rpc;
    p.off_lg = off;
    off += 4 * rpc;
    p.off_cnt = off;
    off += 4 * rpc;
    off = align_up(off, 128);
    p.off_hist = off;
    off += hist_bytes;
    p.off_misc = off;
    off += (int)sizeof(Misc);
    p.smem_total = align_up(off, 128);
    if (p.smem_total > kSmemLimit) return -6;
    return G;
}

/* Raise a kernel's dynamic shared-memory limit once per (device, kernel). */
cudaError_t raise_smem(const void *fn, int bytes) {
    thread_local std::vector<std::pair<int, const void *>> raised;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    for (const auto &r : raised)
        if (r.first == dev && r.second == fn) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    raised.emplace_back(dev, fn);
    return cudaSuccess;
}

cudaError_t launch_tail(const TailParams &p, int grid, cudaStream_t st) {
    void *fn = nullptr;
    if (p.mode == MODE_FUSED) fn = pick_kernel<MODE_FUSED>(p.nch);
    else if (p.mode == MODE_LMHEAD) fn = pick_kernel<MODE_LMHEAD>(p.nch);
    else fn = (void *)tail_kernel<MODE_SAMPLE, 1>;
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = raise_smem(fn, kSmemLimit);
    if (e != cudaSuccess) return e;
    void *args[] = {const_cast<TailParams *>(&p)};
    if ((p.mode == MODE_FUSED && p.local_edges) || (p.mode == MODE_LMHEAD && p.hidden)) {
        /* programmatic dependent launch: the kernel streams W while the
         * previous kernel on the stream finishes, and waits for it before
         * any other read */
        cudaLaunchConfig_t cfg;
        memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(NT);
        cfg.dynamicSmemBytes = (size_t)p.smem_total;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelExC(&cfg, fn, args);
    }
    /* The select's grid barriers need every CTA resident: a cooperative
     * launch guarantees it (or fails to launch). */
    if (p.mode == MODE_LMHEAD || p.local_edges)
        return cudaLaunchKernel(fn, dim3(grid), dim3(NT), args, (size_t)p.smem_total, st);
    return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(NT), args, (size_t)p.smem_total, st);
}

cudaError_t launch_quantize_x(const float *x, int8_t *xq, float *scale, int n,
                              cudaStream_t st) {
    quantize_x_kernel<<<1, NT, 0, st>>>(x, xq, scale, n);
    return cudaGetLastError();
}

cudaError_t launch_stage_inputs(const float *src, float *dst, int n0, int off1, int n1,
                                cudaStream_t st) {
    /* 16 KB of the first range a CTA (the PCIe reads of one CTA overlap) */
    const int grid = std::max(1, std::min(64, (n0 + 4095) / 4096));
    stage_inputs_kernel<<<grid, 256, 0, st>>>(src, dst, n0, off1, n1);
    return cudaGetLastError();
}

cudaError_t launch_abs_xq(const int8_t *xq, uint8_t *ax, int n, cudaStream_t st) {
    abs_xq_kernel<<<(n + 255) / 256, 256, 0, st>>>(xq, ax, n);
    return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const float *W, int d, int8_t *q, int ld, float *scale,
                                 int n_rows, cudaStream_t st) {
    const int warps_per_block = 8;
    const int blocks = (n_rows + warps_per_block - 1) / warps_per_block;
    quantize_rows_kernel<<<blocks, 32 * warps_per_block, 0, st>>>(W, d, q, ld, scale, n_rows);
    return cudaGetLastError();
}

cudaError_t launch_finish(const FinishParams &f, cudaStream_t st) {
    finish_kernel<<<1, NT, 0, st>>>(f);
    return cudaGetLastError();
}

/* Six words per candidate: gathered key + index + weight, candidate value +
 * index + weight / running sum; then the wide walk's bitmap stage and chunk
 * table; the static part (Misc) stays below 8 KB. */
constexpr int kMergeDynLimit = kSmemLimit - 8192;
constexpr int kMergeMaxCap = (kMergeDynLimit - kMergeHead - kWideWalkBytes) / 24;

int peer_merge_cap(const TailParams &p) {
    return (p.area_bytes - kMergeHead - kWideWalkBytes) / 24;
}

int merge_smem_cap(int n_candidates_max) {
    return n_candidates_max <= kMergeMaxCap ? n_candidates_max : -1;
}

cudaError_t launch_merge(const MergeParams &m, int n_streams, cudaStream_t st) {
    if (m.smem_cap < 1 || m.smem_cap > kMergeMaxCap || m.n_ranks < 1 ||
        m.n_ranks > kMaxRanks)
        return cudaErrorInvalidValue;
    cudaError_t e = raise_smem((const void *)merge_kernel, kMergeDynLimit);
    if (e != cudaSuccess) return e;
    merge_kernel<<<n_streams, NT, kMergeHead + 24ull * (size_t)m.smem_cap + kWideWalkBytes, st>>>(m);
    return cudaGetLastError();
}

/* ---- support of the allocation-free sampler entry (tail_noalloc.cu) ---- */
namespace {
/* bit (b >> 8) of every table entry, b = bits(x) - 2^31 (the table holds
 * negative x only, so b >> 8 < kExpfBitmapWords * 32) */
__global__ void expf_bits_kernel(const uint32_t *tx, int n, uint32_t *bits) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const uint32_t b = (tx[i] - 0x80000000u) >> 8;
        atomicOr(bits + (b >> 5), 1u << (b & 31));
    }
}
/* off[w] = first entry whose bitmap word is >= w (the table is sorted by bit
 * pattern), for w in [0, words] */
__global__ void expf_off_kernel(const uint32_t *tx, int n, uint32_t *off, int words) {
    const int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w > words) return;
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (((tx[mid] - 0x80000000u) >> 13) >= (uint32_t)w) hi = mid;
        else lo = mid + 1;
    }
    off[w] = (uint32_t)lo;
}
}  // namespace

cudaError_t launch_expf_index(const uint32_t *tx, int n, uint32_t *bits, uint32_t *off,
                              cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(bits, 0, 4ull * kExpfBitmapWords, st);
    if (e != cudaSuccess) return e;
    if (n > 0) expf_bits_kernel<<<(n + 255) / 256, 256, 0, st>>>(tx, n, bits);
    expf_off_kernel<<<(kExpfBitmapWords + 1 + 255) / 256, 256, 0, st>>>(tx, n, off,
                                                                        kExpfBitmapWords);
    return cudaGetLastError();
}

cudaError_t prepare_sample_kernel() {
    return cudaFuncSetAttribute((const void *)tail_kernel<MODE_SAMPLE, 1>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
}

cudaError_t launch_sample_prepared(const TailParams &p, int grid, cudaStream_t st) {
    if (p.mode != MODE_SAMPLE) return cudaErrorInvalidValue;
    void *fn = (void *)tail_kernel<MODE_SAMPLE, 1>;
    void *args[] = {const_cast<TailParams *>(&p)};
    if (p.local_edges)
        return cudaLaunchKernel(fn, dim3(grid), dim3(NT), args, (size_t)p.smem_total, st);
    return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(NT), args, (size_t)p.smem_total, st);
}

cudaError_t launch_debug_expf(const float *x, float *y, int n, const uint32_t *tx,
                              const uint32_t *ty, int tn, const uint32_t *bits,
                              const uint32_t *off, const uint4 *hash, int hash_probe,
                              cudaStream_t st) {
    (void)tn;
    debug_expf_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, y, n, tx, ty, bits, off, hash,
                                                        hash_probe);
    return cudaGetLastError();
}

}  // namespace lal
