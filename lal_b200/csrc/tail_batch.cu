/*
 * tail_batch.cu -- the batched decode tail (B >= 2 streams) on sm_100a.
 *
 * With B streams the LM-head contraction is a GEMM, logits[b][v] =
 * (scale_x[b] * scale_w[v]) * sum_k xq[b][k] * W[v][k]; one pass over the
 * 545 MB of W serves every stream.  Three launches per step:
 *
 *   quantize_batch_kernel  lal_quantize_x_int8 (runtime/lal_q8_kernel.h:375-442)
 *                          for each stream: int8 rows X [N][ld] + scale_x [B];
 *   gemm_i8_kernel         the 5th-gen tensor cores: tcgen05.mma kind::i8
 *                          with int32 accumulators in tensor memory.  W is
 *                          the M operand (128 vocab rows a tile), the B
 *                          streams the N operand (N = B rounded up to 32, at
 *                          most 256), K = d in 128-byte TMA boxes with the
 *                          128-byte swizzle.  A persistent CTA per SM walks
 *                          its tiles: warp 0 issues the TMA loads into a ring
 *                          of shared-memory stages, warp 1 issues the MMAs
 *                          (one thread) and owns the tensor memory, warps
 *                          2-5 read the accumulators (tcgen05.ld), apply the
 *                          reference's scale expression and store the logits
 *                          [B][rows] (fp32, L2-resident for the next kernel).
 *                          Two accumulator buffers let the epilogue of one
 *                          tile overlap the MMAs of the next.  int8 products
 *                          accumulate exactly in int32, so the logits equal
 *                          the reference's bit for bit.  The tiles left over
 *                          after the last whole wave (4 of Qwen's 1188 on 148
 *                          SMs) would cost a whole extra wave: they are split
 *                          along K instead, one chunk a CTA after its own
 *                          tiles, each chunk's int32 partial dots stored to
 *                          its own slot (still in L2 when the select runs);
 *                          the select adds a stream's slots (exact in any
 *                          order) into its logits.
 *   batch_select_kernel    one CTA per stream: the repetition penalty
 *                          (runtime/lal_sampling.h:59-67; occurrences counted
 *                          in a shared-memory hash of the history), a key
 *                          histogram for a tie-complete superset of the top k,
 *                          the exact threshold, the candidates in ascending
 *                          vocab order, then the softmax sums and the draw
 *                          exactly as the single-stream kernel, the history
 *                          push, or (vocab-sharded) the stream's record.
 *
 * Every wait is bounded (kWaitNs); a wait that runs out sets DEV_TIMEOUT, the
 * MMA issuer drains its MMAs before the tensor memory is released, and the
 * producer waits for its copies in flight before the CTA exits.
 */
#include "tail_device.cuh"
#include "tail_wide.cuh"

#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>

namespace lal {
namespace {

constexpr int kBM = 128;           /* W rows per tile (MMA M)                  */
constexpr int kBK = 128;           /* K bytes per TMA box = one swizzle row    */
constexpr int kMmaK = 32;          /* K of one tcgen05.mma kind::i8            */
constexpr int kGemmThreads = 192;  /* warp 0 TMA, warp 1 MMA, warps 2-5 epilogue */
constexpr int kGemmStagesMax = 8;
constexpr int kGemmSmemLimit = 232448;
constexpr int kStageGroups = 512;  /* 32-row logit groups staged a round (select) */
/* the smallest round tried when a step has more streams than SMs (the
 * largest round, in steps of 32 groups, with which two select CTAs fit on
 * one SM, so that every stream's CTA is resident at once instead of a
 * second wave waiting for the first) */
constexpr int kStageGroupsMin = 64;
constexpr int kPenGroupWords = 512; /* bitmap words of groups holding a penalised row */
constexpr int kSplitChunksMax = 32; /* K chunks of a split tile (the select keeps a row's in registers) */
constexpr int kSplitGroupsMax = 4 * 74; /* 32-row groups of the split tiles (>= 2 chunks a tile, 148 SMs) */

/* ------------------------------------------------------------ PTX --- */
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
/* arrive on bar when every tcgen05.mma this thread issued before has completed */
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                     "r"(smem_u32(bar))
                 : "memory");
}
/* D[tmem] (+)= A[smem desc] * B[smem desc]^T, int8 x int8 -> int32 */
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    const uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1),
        "r"(mask2), "r"(mask3));
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

/* Shared-memory matrix descriptor of a K-major tile written by TMA with the
 * 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride
 * byte offset), leading byte offset unused (1), descriptor version 1, layout
 * type 2 = 128-byte swizzle.  The tile base is 1024-byte aligned; a K step of
 * 32 bytes inside the swizzle row advances the start address. */
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;                 /* leading byte offset (unused) */
    d |= (uint64_t)(1024u >> 4) << 32;       /* stride byte offset           */
    d |= (uint64_t)1u << 46;                 /* version                      */
    d |= (uint64_t)2u << 61;                 /* 128-byte swizzle             */
    return d;
}
/* Instruction descriptor: int32 accumulate, signed int8 A and B, both K-major,
 * N >> 3 at bit 17, M >> 4 at bit 24. */
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

/* -------------------------------------------------- batch quantize --- */
__global__ void __launch_bounds__(NT) quantize_batch_kernel(const float *x, int d, int8_t *xq,
                                                            int ld, float *scale_out,
                                                            const float *norm_w, float norm_eps) {
    __shared__ Misc ms;
    __shared__ float xs[kNormMaxD];
    /* the GEMM may launch now: it streams the LM head and waits for this
     * kernel's completion before it reads X */
    grid_dep_launch_dependents();
    const int b = blockIdx.x;
    const float *row = x + (size_t)b * d;
    int8_t *out = xq + (size_t)b * ld;
    /* the final RMSNorm first when the step takes the residual stream
     * (runtime/lal_simd_optim.h:32-58): the normalised row replaces x */
    float inv_rms = 0.0f;
    if (norm_w != nullptr) {
        for (int i = threadIdx.x; i < d; i += NT) xs[i] = row[i];
        __syncthreads();
        if (threadIdx.x < 8) ms.nrm[threadIdx.x] = rmsnorm_lane(xs, d, threadIdx.x);
        __syncthreads();
        if (threadIdx.x == 0) ms.ninv = rmsnorm_inv(ms.nrm, d, norm_eps);
        __syncthreads();
        inv_rms = ms.ninv;
    }
    auto value = [&](int i) {
        return norm_w != nullptr ? rmsnorm_apply(xs[i], inv_rms, __ldg(norm_w + i)) : row[i];
    };
    float m = 0.0f;
    for (int i = threadIdx.x; i < d; i += NT) m = fmaxf(m, fabsf(value(i)));
    m = block_max_f(m, &ms);
    float scale = __fdiv_rn(m, 127.0f);
    if (scale < 1e-8f) scale = 1e-8f;
    const float inv = __fdiv_rn(1.0f, scale);
    const int n8 = d & ~7;
    for (int i = threadIdx.x; i < ld; i += NT) {
        int v = 0;
        if (i < d) {
            const float s = __fmul_rn(value(i), inv);
            if (s != s) v = -127;
            else {
                v = (i < n8) ? __float2int_rn(s) : __float2int_rz(s);
                v = v > 127 ? 127 : (v < -127 ? -127 : v);
            }
        }
        out[i] = (int8_t)v;
    }
    if (threadIdx.x == 0) scale_out[b] = scale;
}

/* ---------------------------------------------------- the tcgen05 GEMM --- */
struct GemmParams {
    CUtensorMap tmW; /* [rows][ld] int8, box 128 x 128, 128-byte swizzle */
    CUtensorMap tmX; /* [N][ld] int8, box 128 x N, 128-byte swizzle      */
    const float *scale_w;
    const float *scale_x;
    float *logits; /* [B][rows] */
    uint32_t *gmax; /* [B][n_groups] order key of each 32-row group's largest logit */
    int n_groups;
    int rows, B, N, kblocks, stages, stage_bytes, tmem_cols;
    int *status;
    /* tiles [0, reg_end) whole, tile t by CTA t mod grid; tiles [reg_end,
     * n_tiles) in split_chunks K chunks of split_cb boxes, chunk c of tile
     * reg_end + u / split_chunks by CTA u < split_units */
    int reg_end, split_units, split_chunks, split_cb;
    int *split_part; /* [n_tiles - reg_end][split_chunks][N][128] int32 partial dots */
};

/* logits and group maxima of 32 streams (c0 ..) of one warp's 32 rows from
 * their int32 dots r[j] (stream c0 + j, this lane's row) */
__device__ __forceinline__ void emit_logits32(const GemmParams &p, const float *sx, float sw,
                                              int row, int group, int c0, const uint32_t (&r)[32],
                                              int lane) {
    uint32_t mine = 0u;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const int b = c0 + j;
        /* runtime/lal_q8_kernel.h:489: scale_x*scale_w[v]*(float)dot */
        const float l = __fmul_rn(__fmul_rn(sx[b], sw), __int2float_rn((int)r[j]));
        if (row < p.rows && b < p.B) p.logits[(size_t)b * p.rows + row] = l;
        /* the group maximum of stream b, kept by lane j */
        const uint32_t gm = __reduce_max_sync(0xffffffffu, row < p.rows ? f2key(l) : 0u);
        if (lane == j) mine = gm;
    }
    if (c0 + lane < p.B) p.gmax[(size_t)(c0 + lane) * p.n_groups + group] = mine;
}

__device__ __forceinline__ bool bwait(uint64_t *b, uint32_t parity, volatile int *abort_flag) {
    return mbar_wait(b, parity, abort_flag);
}

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_i8_kernel(const __grid_constant__ GemmParams p) {
    extern __shared__ uint8_t gsm_raw[];
    uint8_t *gsm = gsm_raw + ((1024u - (smem_u32(gsm_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *full = reinterpret_cast<uint64_t *>(gsm + (size_t)p.stages * p.stage_bytes);
    uint64_t *empty = full + kGemmStagesMax;
    uint64_t *tfull = empty + kGemmStagesMax;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tholder = reinterpret_cast<uint32_t *>(drain + 1);
    int *abort_i = reinterpret_cast<int *>(tholder + 1);
    volatile int *abort_flag = abort_i;
    /* the drains at exit wait on time alone (never on the abort flag): no
     * copy or MMA may be in flight when the CTA leaves */
    volatile int *never = reinterpret_cast<int *>(tholder + 2);
    float *sx = reinterpret_cast<float *>(tholder + 4);
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);
        }
        mbar_init(drain, 1);
        *abort_i = 0;
        *never = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tholder)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tholder;

    /* Programmatic dependent launch: the LM head is written by no step, so
     * the first W boxes are requested while the previous kernel on the
     * stream (the quantizer) still runs; X, the scales and every output wait
     * for that kernel's completion.  Two boxes only: X's first boxes queue
     * behind this burst when the launches do not overlap (measured: a full
     * ring of W first cost 5 us a launch at B=64). */
    const uint32_t bytes = (uint32_t)(kBM * kBK + p.N * kBK);
    const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
    /* this CTA's work: its whole tiles, then its K chunk of a split tile (u_n
     * boxes) as accumulator round a = n_reg when there is one */
    const int G = (int)gridDim.x, bid = (int)blockIdx.x;
    const bool has_unit = bid < p.split_units;
    const int u_tile = has_unit ? p.reg_end + bid / p.split_chunks : 0;
    const int u_kb0 = has_unit ? (bid % p.split_chunks) * p.split_cb : 0;
    const int u_n = has_unit ? min(p.kblocks, u_kb0 + p.split_cb) - u_kb0 : 0;
    const int n_reg = bid < p.reg_end ? (p.reg_end - 1 - bid) / G + 1 : 0;
    const int n_acc = (u_n > 0 ? 1 : 0) + n_reg;
    const int my_iters = u_n + n_reg * p.kblocks;
    auto coord = [&](int it, int &tile, int &kb) {
        if (it < n_reg * p.kblocks) {
            tile = bid + (it / p.kblocks) * G;
            kb = it % p.kblocks;
        } else {
            tile = u_tile;
            kb = u_kb0 + (it - n_reg * p.kblocks);
        }
    };
    const int pre = min(2, my_iters);
    if (warp == 0 && lane == 0)
        for (int it = 0; it < pre; ++it) {
            int tile, kb;
            coord(it, tile, kb);
            mbar_expect_tx(&full[it], bytes);
            tma_load_2d(gsm + (size_t)it * p.stage_bytes, &p.tmW, kb * kBK, tile * kBM, &full[it],
                        pol_w);
        }
    grid_dep_wait();
    grid_dep_launch_dependents();
    for (int i = threadIdx.x; i < p.N; i += kGemmThreads) sx[i] = i < p.B ? p.scale_x[i] : 0.0f;
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            /* producer: one W box and one X box per stage (the first `pre`
             * stages' W boxes are on their way already) */
            int it = 0;
            for (; it < my_iters; ++it) {
                int tile, kb;
                coord(it, tile, kb);
                const int s = it % p.stages;
                const uint32_t use = (uint32_t)(it / p.stages);
                uint8_t *st = gsm + (size_t)s * p.stage_bytes;
                if (it < pre) {
                    tma_load_2d(st + kBM * kBK, &p.tmX, kb * kBK, 0, &full[s], pol_x);
                    continue;
                }
                if (!bwait(&empty[s], (use & 1u) ^ 1u, abort_flag)) {
                    *abort_flag = 1;
                    break;
                }
                mbar_expect_tx(&full[s], bytes);
                tma_load_2d(st, &p.tmW, kb * kBK, tile * kBM, &full[s], pol_w);
                tma_load_2d(st + kBM * kBK, &p.tmX, kb * kBK, 0, &full[s], pol_x);
            }
            /* no copy may be in flight when the CTA exits */
            for (int q = max(0, it - p.stages); q < it; ++q)
                bwait(&full[q % p.stages], (uint32_t)(q / p.stages) & 1u, never);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            /* MMA issuer */
            const uint32_t idesc = idesc_i8(kBM, p.N);
            int it = 0;
            bool ok = true;
            for (int a = 0; a < n_acc && ok; ++a) {
                const int acc = a & 1;
                const uint32_t ause = (uint32_t)(a >> 1);
                if (a >= 2 && !bwait(&tempty[acc], (ause & 1u) ^ 1u, abort_flag)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tbase + (uint32_t)(acc * p.N);
                const int nkb = a == n_reg ? u_n : p.kblocks;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % p.stages;
                    if (!bwait(&full[s], (uint32_t)(it / p.stages) & 1u, abort_flag)) {
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(gsm + (size_t)s * p.stage_bytes);
                    const uint32_t b0 = a0 + kBM * kBK;
#pragma unroll
                    for (int kk = 0; kk < kBK / kMmaK; ++kk)
                        tc_mma_i8(d_tmem, sw128_desc(a0 + kk * kMmaK), sw128_desc(b0 + kk * kMmaK),
                                  idesc, (kb | kk) != 0 ? 1u : 0u);
                    tc_commit(&empty[s]); /* the stage is free once these MMAs are done */
                }
                if (ok) tc_commit(&tfull[acc]);
            }
            /* every MMA issued is complete before the tensor memory is freed */
            tc_commit(drain);
            if (!bwait(drain, 0u, never)) *abort_flag = 1;
        }
    } else {
        /* epilogue (warps 2-5): warp w reads tensor-memory lanes
         * 32*(w%4) .. +31 */
        const int q = warp & 3;
        for (int a = 0; a < n_acc; ++a) {
            const int acc = a & 1;
            const uint32_t ause = (uint32_t)(a >> 1);
            if (!bwait(&tfull[acc], ause & 1u, abort_flag)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const bool part = a == n_reg;
            const int tile = part ? u_tile : bid + a * G;
            const int row = tile * kBM + q * 32 + lane;
            const float sw = row < p.rows ? __ldg(p.scale_w + row) : 0.0f;
            const int group = tile * 4 + q; /* this warp's 32 rows */
            if (part) {
                /* a K chunk: its partial dots into its own slot, for the
                 * select to add up */
                const int slot = (tile - p.reg_end) * p.split_chunks + bid % p.split_chunks;
                int *dst = p.split_part + (size_t)slot * p.N * kBM + q * 32 + lane;
                for (int c0 = 0; c0 < p.N; c0 += 32) {
                    uint32_t r[32];
                    tmem_ld32(tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * p.N + c0), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (c0 + j < p.B) dst[(size_t)(c0 + j) * kBM] = (int)r[j];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[acc]);
                continue;
            }
            for (int c0 = 0; c0 < p.N; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * p.N + c0), r);
                tmem_ld_wait();
                emit_logits32(p, sx, sw, row, group, c0, r, lane);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase),
                     "r"(p.tmem_cols)
                     : "memory");
    }
    if (threadIdx.x == 0 && *abort_flag) atomicCAS(p.status, 0, (int)DEV_TIMEOUT);
}

/* --------------------------------------------- per-stream select + draw --- */
struct BatchSelectParams {
    float *logits; /* [B][rows], penalised in place */
    int rows, row_base, vocab, variant;
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
    uint8_t *shard_out; /* [B][rec_bytes] records, or null */
    int rec_cap, rec_bytes;
    int s_cap, c_cap, h_slots; /* superset, candidate and hash capacities */
    uint32_t *gmax;            /* [B][n_groups] raw group maxima (GEMM) */
    int n_groups;
    /* the GEMM's split tiles (rows [split_row0, split_row0 + 128 * split_rem)):
     * int32 partial dots [split_rem][split_chunks][split_n][128], or null */
    const int *split_part;
    int split_rem, split_chunks, split_n, split_row0;
    const float *scale_w, *scale_x;
    int wide_cap;              /* explicit rows of the wide path (>= max k - 1) */
    int stage_groups;          /* candidate groups staged a round */
    unsigned long long *host_tok; /* [B] completion words in mapped host memory, or null */
    const unsigned *seq_in;
};

constexpr uint32_t kEmptySlot = 0xFFFFFFFFu;

/* The wide path (tail_wide.cuh) of stream b, whose candidates did not fit
 * the select's shared memory or whose shard set did not fit its record: the
 * exact select over the stream's penalised logits, then the draw or the
 * record's wide form. */
__device__ __noinline__ void batch_wide(const BatchSelectParams &p, int b, int k, bool greedy,
                                        float temp, float u0, int hn, int hhead, uint8_t *area,
                                        Misc *ms) {
    WideDense a = {};
    a.lg = p.logits + (size_t)b * p.rows;
    a.rows = p.rows;
    a.row_base = p.row_base;
    a.vocab = p.vocab;
    a.k = k;
    a.variant = p.variant;
    a.greedy = greedy ? 1 : 0;
    a.temp = temp;
    a.u = u0;
    a.cap = max(1, p.wide_cap);
    a.ex = ExpfTables{p.expf_x, p.expf_y, p.expf_bits, p.expf_off, nullptr, 0};
    a.diag = p.diag + b;
    if (p.shard_out != nullptr) {
        a.rec = p.shard_out + (size_t)b * p.rec_bytes;
        a.rec_cap = p.rec_cap;
    } else {
        a.token = p.tokens + b;
        if (p.host_tok) {
            a.host_tok = p.host_tok + b;
            a.host_seq = __ldcg(p.seq_in);
        }
        a.hist_ids = p.hist_ids + (size_t)b * p.hist_stride;
        a.hist_n = p.hist_n + b;
        a.hist_head = p.hist_head + b;
        a.hist_cap = p.hist_cap;
        a.push_history = p.push_history;
        a.hn = hn;
        a.hhead = hhead;
    }
    wide_dense(a, area, ms);
}


__global__ void __launch_bounds__(NT, 1) batch_select_kernel(const __grid_constant__ BatchSelectParams p) {
    extern __shared__ __align__(16) uint8_t bsm[];
    __shared__ Misc msh;
    __shared__ int s_count;
    Misc *ms = &msh;
    const int tid = threadIdx.x, b = blockIdx.x;
    uint32_t *hist = reinterpret_cast<uint32_t *>(bsm);            /* 4096 bins        */
    uint32_t *Sk = hist + 4096;                                     /* superset keys    */
    int *Si = reinterpret_cast<int *>(Sk + p.s_cap);                /* superset rows    */
    float *Cv = reinterpret_cast<float *>(Si + p.s_cap);           /* candidates       */
    int *Ci = reinterpret_cast<int *>(Cv + p.c_cap);
    float *Ov = reinterpret_cast<float *>(Ci + p.c_cap);           /* index order      */
    int *Oi = reinterpret_cast<int *>(Ov + p.c_cap);
    float *Ce = reinterpret_cast<float *>(Oi + p.c_cap);           /* weights, sums    */
    int *Gl = reinterpret_cast<int *>(Ce + p.c_cap);               /* candidate groups */
    /* one 16-byte aligned region, used twice: the history hash of the
     * penalty (step 1), then the staging of p.stage_groups candidate groups'
     * 32 logits a round (step 3) */
    uint8_t *shared2 = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(Gl + p.n_groups) + 15) & ~static_cast<uintptr_t>(15));
    uint32_t *hkey = reinterpret_cast<uint32_t *>(shared2);        /* history hash     */
    uint32_t *hcnt = hkey + p.h_slots;
    float *Gv = reinterpret_cast<float *>(shared2);

    float *lg = p.logits + (size_t)b * p.rows;
    const float temp = p.temperature[b];
    const int topk = p.top_k[b];
    const float pen = p.rep_penalty[b];
    const float u0 = p.u ? p.u[b] : 0.0f;
    int *hids = p.hist_ids + (size_t)b * p.hist_stride;
    const int hn = p.hist_n ? p.hist_n[b] : 0;
    const int hhead = p.hist_head ? p.hist_head[b] : 0;
    const bool greedy = (temp <= 0.0f) || (topk <= 0);
    const bool use_pen = pen > 1.0f && hn > 0 && (p.variant == VARIANT_SERVER || !greedy);

    constexpr int kGroupRegs = 24;
    uint32_t gpre[kGroupRegs];
    const bool gpre_ok = p.gmax != nullptr && p.n_groups <= NT * kGroupRegs;

    /* 1. repetition penalty: occurrences of each history id in this slice,
     * counted in an open-addressing hash, applied once per occurrence
     * (runtime/lal_sampling.h:60-66; ids outside [0, V) are skipped).
     *
     * Programmatic dependent launch: the history (the previous step's
     * select, complete before this step's quantizer ran) is hashed while the
     * GEMM finishes; the wait comes before the first read of its outputs. */
    for (int i = tid; i < 4096; i += NT) hist[i] = 0u;
    __shared__ int s_pen; /* distinct history ids inside this slice */
    /* which 32-row groups hold a penalised row (slices of up to
     * kPenGroupWords * 32 groups) */
    __shared__ uint32_t pen_groups[kPenGroupWords];
    const bool mark = p.n_groups <= kPenGroupWords * 32;
    if (tid == 0) {
        s_pen = 0;
    }
    for (int i = tid; i < kPenGroupWords; i += NT) pen_groups[i] = 0u;
    if (use_pen) {
        for (int i = tid; i < p.h_slots; i += NT) {
            hkey[i] = kEmptySlot;
            hcnt[i] = 0u;
        }
        __syncthreads();
        const uint32_t mask = (uint32_t)p.h_slots - 1u;
        for (int i = tid; i < hn; i += NT) {
            const int id = hids[i];
            if (id < 0 || id >= p.vocab) continue;
            const int g = id - p.row_base;
            if (g < 0 || g >= p.rows) continue;
            uint32_t slot = ((uint32_t)id * 2654435761u) & mask;
            for (int probe = 0; probe < p.h_slots; ++probe) {
                const uint32_t prev = atomicCAS(&hkey[slot], kEmptySlot, (uint32_t)id);
                if (prev == kEmptySlot || prev == (uint32_t)id) {
                    atomicAdd(&hcnt[slot], 1u);
                    if (prev == kEmptySlot) {
                        atomicAdd(&s_pen, 1);
                        if (mark) {
                            const int gi = g >> 5;
                            const uint32_t bit = 1u << (gi & 31);
                            atomicOr(&pen_groups[gi >> 5], bit);
                        }
                    }
                    break;
                }
                slot = (slot + 1u) & mask;
            }
        }
        __syncthreads();
    }
    grid_dep_wait();
    /* this stream's group maxima, loaded now so that their latency overlaps
     * the penalty (one batch when the slice has at most NT * kGroupRegs
     * groups) */
    if (gpre_ok) {
        const uint32_t *gm = p.gmax + (size_t)b * p.n_groups;
#pragma unroll
        for (int j = 0; j < kGroupRegs; ++j) {
            const int g = j * NT + tid;
            gpre[j] = g < p.n_groups ? __ldcg(gm + g) : 0u;
        }
    }
    /* the GEMM's split tiles: this stream's rows of them are the sums of
     * their K chunks' partial dots (int32, exact in any order), scaled like
     * every other logit (runtime/lal_q8_kernel.h:489), with their groups'
     * maxima (which replace the ones just loaded); before the penalty,
     * which may change them */
    if (p.split_part != nullptr) {
        __shared__ uint32_t s_split_gmax[kSplitGroupsMax];
        const int R = p.split_rem * kBM; /* a multiple of 32, as NT: whole warps */
        const int g0 = p.split_row0 >> 5;
        const float sxb = __ldcg(p.scale_x + b);
        const size_t cstride = (size_t)p.split_n * kBM;
        for (int i = tid; i < R; i += NT) {
            const int *src = p.split_part +
                             ((size_t)(i >> 7) * p.split_chunks * p.split_n + b) * kBM + (i & 127);
            /* every chunk's load in flight at once */
            int v[kSplitChunksMax];
#pragma unroll
            for (int c = 0; c < kSplitChunksMax; ++c)
                v[c] = c < p.split_chunks ? __ldcg(src + c * cstride) : 0;
            int dot = 0;
#pragma unroll
            for (int c = 0; c < kSplitChunksMax; ++c) dot += v[c];
            const int row = p.split_row0 + i;
            const bool in = row < p.rows;
            const float sw = in ? __ldg(p.scale_w + row) : 0.0f;
            const float l = __fmul_rn(__fmul_rn(sxb, sw), __int2float_rn(dot));
            if (in) lg[row] = l;
            const uint32_t gm = __reduce_max_sync(0xffffffffu, in ? f2key(l) : 0u);
            if ((tid & 31) == 0) {
                p.gmax[(size_t)b * p.n_groups + (row >> 5)] = gm;
                s_split_gmax[(row >> 5) - g0] = gm;
            }
        }
        __syncthreads();
        if (gpre_ok) {
#pragma unroll
            for (int j = 0; j < kGroupRegs; ++j) {
                const int g = j * NT + tid;
                if (g >= g0 && g < g0 + 4 * p.split_rem) gpre[j] = s_split_gmax[g - g0];
            }
        }
    }
    if (use_pen) {
        for (int i = tid; i < p.h_slots; i += NT) {
            const uint32_t id = hkey[i];
            if (id != kEmptySlot) {
                const int g = (int)id - p.row_base;
                lg[g] = penalise(lg[g], hcnt[i], pen);
            }
        }
    }
    __syncthreads();

    /* 2. k = min(top_k, V) (runtime/lal_sampling.h:70-71), 1 for greedy */
    int k = greedy ? 1 : topk;
    if (k > p.vocab) k = p.vocab;
    if (k > p.rows) k = p.rows;
    if (k < 1) k = 1;
    constexpr int U = 8;
    StreamDiag dg;
    dg.threshold = 0.0f;
    dg.max_l = 0.0f;
    dg.sum = 0.0f;
    dg.r = 0.0f;
    dg.n_cand = 0;
    dg.greedy = greedy ? 1 : 0;
    dg.drew = 0;
    dg.token = -1;

    /* 3. a tie-complete superset of {l >= T}: keys >= a lower bound L of T.
     *
     * Group bound (the GEMM recorded each 32-row group's largest raw logit):
     * with every group's maximum a logit of the step (the penalised groups'
     * taken again below), the k-th largest group maximum L is <= T -- k
     * groups hold k distinct logits >= L -- and only groups whose maximum
     * reaches L can hold a key >= L.  Without the group marks (a slice of
     * more than kPenGroupWords * 32 groups), with P distinct penalised ids,
     * the (k+P)-th largest raw maximum is: its k+P groups hold k+P distinct
     * logits >= L, at most P of them penalised, and a penalty (p > 1) never
     * raises a logit.  When the bound is weak the full histogram pass below
     * is used instead. */
    auto hist_add = [&](uint32_t *h, uint32_t digit, bool act) {
        const unsigned voters = __ballot_sync(0xffffffffu, act);
        if (act) {
            const unsigned peers = __match_any_sync(voters, digit);
            if ((tid & 31) == __ffs(peers) - 1) atomicAdd(&h[digit], (uint32_t)__popc(peers));
        }
    };
    uint32_t L = 0u;
    int S = -1;
    bool ordered = false; /* the superset is in vocab order (the group path) */
    /* with the penalised groups marked, only the groups free of penalised
     * rows count towards the bound: their maxima are unchanged logits of k
     * distinct rows, so the k-th largest of them is <= T; otherwise every
     * group counts and the (k+P)-th largest maximum is the bound */
    /* With the penalised groups marked, each one's maximum is taken again
     * after the penalty (the GEMM's is of the raw logits): every group
     * maximum is then a logit of the step, k groups reach their k-th largest,
     * and that maximum bounds T from below.  Without the marks, the (k+P)-th
     * largest raw maximum does (see above). */
    const bool exact = mark;
    const int kp = exact ? k : k + s_pen;
    const bool groups = p.gmax != nullptr && kp <= p.n_groups / 2 && p.n_groups <= p.s_cap;
    auto counts = [&](int g) { return g < p.n_groups; };
    if (groups) {
        /* the group maxima (contiguous per stream) into Sk and the top 12 key
         * bits of the counted ones into the histogram; the lower edge of the
         * bin holding the kp-th largest counted maximum is <= that maximum,
         * hence a bound of T */
        uint32_t *Gk = Sk; /* the group maxima, then the superset */
        const uint32_t *gm = p.gmax + (size_t)b * p.n_groups;
        if (gpre_ok) {
#pragma unroll
            for (int j = 0; j < kGroupRegs; ++j) {
                const int g = j * NT + tid;
                if (g < p.n_groups) Gk[g] = gpre[j];
            }
        } else {
            for (int g = tid; g < p.n_groups; g += NT) Gk[g] = __ldcg(gm + g);
        }
        if (exact && use_pen) {
            /* the marked groups, listed in Gl (free until the candidate
             * groups), then each one's maximum after the penalty, one group a
             * thread with eight 16-byte loads */
            if (tid == 0) s_count = 0;
            __syncthreads();
            const int words = (p.n_groups + 31) >> 5;
            for (int w0 = 0; w0 < words; w0 += NT) {
                const int w = w0 + tid;
                const uint32_t bits = w < words ? pen_groups[w] : 0u;
                const int c = __popc(bits);
                const int lane = tid & 31;
                int incl = c;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                int base = 0;
                if (lane == 31) base = atomicAdd(&s_count, incl);
                base = __shfl_sync(0xffffffffu, base, 31) + incl - c;
                uint32_t rest = bits;
                while (rest) {
                    Gl[base++] = 32 * w + __ffs(rest) - 1;
                    rest &= rest - 1u;
                }
            }
            __syncthreads();
            const int nm = s_count;
            const bool lg16 = (reinterpret_cast<uintptr_t>(lg) & 15u) == 0;
            for (int i = tid; i < nm; i += NT) {
                const int g = Gl[i];
                const int r0 = g * 32, r1 = min(p.rows, r0 + 32);
                uint32_t mx = 0u;
                if (lg16 && r1 == r0 + 32) {
                    const float4 *v4 = reinterpret_cast<const float4 *>(lg + r0);
                    float4 v[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) v[q] = __ldcg(v4 + q);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        mx = max(max(max(mx, f2key(v[q].x)), f2key(v[q].y)),
                                 max(f2key(v[q].z), f2key(v[q].w)));
                } else {
                    for (int r = r0; r < r1; ++r) mx = max(mx, f2key(__ldcg(lg + r)));
                }
                Gk[g] = mx;
            }
        }
        __syncthreads();
        uint32_t gtop = 0u;
        for (int g0 = 0; g0 < p.n_groups; g0 += NT) {
            const int g = g0 + tid;
            const uint32_t key = g < p.n_groups ? Gk[g] : 0u;
            gtop = max(gtop, key);
            hist_add(hist, key >> 20, counts(g));
        }
        gtop = __reduce_max_sync(0xffffffffu, gtop);
        if ((tid & 31) == 0) ms->wmax[tid >> 5] = gtop;
        __syncthreads();
        /* one warp, down from the largest maximum's bin (the answer is near
         * the top: kp of thousands of groups) */
        if (tid < 32) {
            uint32_t top = ms->wmax[0];
            for (int w = 1; w < NWARP; ++w) top = max(top, ms->wmax[w]);
            const uint32_t bin = warp_boundary_bin_4096(hist, top >> 20, (uint32_t)kp);
            if (tid == 0) ms->sh[0] = bin;
        }
        __syncthreads();
        L = ms->sh[0] << 20;
        for (int i = tid; i < 4096; i += NT) hist[i] = 0u; /* for the fallback */
        /* the candidate groups, listed in Gl in ascending order (a thread a
         * contiguous run of groups: count, one scan, write), so that the
         * superset gathered from them, and the candidates, are in vocab
         * order without a sort */
        const int gper = (p.n_groups + NT - 1) / NT;
        const int ga = min(p.n_groups, tid * gper), gb = min(p.n_groups, ga + gper);
        uint32_t gc = 0;
        for (int g = ga; g < gb; ++g) gc += Gk[g] >= L;
        uint32_t ngt;
        uint32_t gpos = block_scan_excl(gc, ms, &ngt);
        for (int g = ga; g < gb; ++g)
            if (Gk[g] >= L) Gl[gpos++] = g;
        __syncthreads();
        const int ng = (int)ngt;
        if (ng <= p.n_groups / 2) {
            if (tid == 0) s_count = 0;
            /* gather the groups' keys >= L (32 consecutive rows a group):
             * each round copies up to p.stage_groups groups into shared memory
             * with 16-byte asynchronous copies, all in flight together (a
             * piece that is misaligned or crosses the slice end is read one
             * value at a time), then a warp takes a group a ballot */
            const bool al16 = (reinterpret_cast<uintptr_t>(lg) & 15u) == 0;
            for (int c0 = 0; c0 < ng; c0 += p.stage_groups) {
                const int cn = min(p.stage_groups, ng - c0);
                __syncthreads(); /* the previous round's staging is consumed */
                for (int e = tid; e < cn * 8; e += NT) {
                    const int r = Gl[c0 + (e >> 3)] * 32 + (e & 7) * 4;
                    float *dst = Gv + (size_t)(e >> 3) * 32 + (e & 7) * 4;
                    if (al16 && r + 4 <= p.rows) {
                        cp_async16(dst, lg + r);
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q) dst[q] = r + q < p.rows ? lg[r + q] : 0.0f;
                    }
                }
                cp_async_wait_all();
                __syncthreads();
                /* a thread a contiguous run of the staged values: count, one
                 * scan, write (no atomics on the way) */
                const int tot = cn * 32;
                const int per = (tot + NT - 1) / NT;
                const int e0 = min(tot, tid * per), e1 = min(tot, e0 + per);
                uint32_t c = 0;
                for (int e = e0; e < e1; ++e)
                    c += (Gl[c0 + (e >> 5)] * 32 + (e & 31) < p.rows) && f2key(Gv[e]) >= L;
                uint32_t got;
                uint32_t pos = block_scan_excl(c, ms, &got) + (uint32_t)s_count;
                for (int e = e0; e < e1; ++e) {
                    const int r = Gl[c0 + (e >> 5)] * 32 + (e & 31);
                    const uint32_t key = f2key(Gv[e]);
                    if (r < p.rows && key >= L) {
                        if (pos < (uint32_t)p.s_cap) {
                            Sk[pos] = key;
                            Si[pos] = r;
                        }
                        ++pos;
                    }
                }
                __syncthreads(); /* every thread read s_count before it moves */
                if (tid == 0) s_count += (int)got;
            }
            __syncthreads();
            S = s_count;
            if (S > p.s_cap) {
                batch_wide(p, b, k, greedy, temp, u0, hn, hhead, bsm, ms);
                return;
            }
            ordered = true;
        }
    }
    if (S < 0) {
    /* full pass: the top 12 key bits of every logit into the histogram */
    for (int i0 = 0; i0 < p.rows; i0 += NT * U) {
        float v[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int i = i0 + j * NT + tid;
            v[j] = i < p.rows ? lg[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int i = i0 + j * NT + tid;
            hist_add(hist, f2key(v[j]) >> 20, i < p.rows);
        }
    }
    __syncthreads();
    uint32_t ab, cnt;
    uint32_t bin = boundary_bin(hist, 4096, (uint32_t)k, ms, &ab, &cnt);
    uint32_t prefix = bin << 20, pmask = 0xFFF00000u;
    uint32_t above = ab;
    /* refine (10 + 10 bits) while the boundary bin does not fit the superset */
    for (int level = 1; level <= 2 && above + cnt > (uint32_t)p.s_cap; ++level) {
        const int shift = level == 1 ? 10 : 0;
        for (int i = tid; i < 1024; i += NT) hist[i] = 0u;
        __syncthreads();
        for (int i0 = 0; i0 < p.rows; i0 += NT * U) {
            float v[U];
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const int i = i0 + j * NT + tid;
                v[j] = i < p.rows ? lg[i] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const int i = i0 + j * NT + tid;
                const uint32_t key = f2key(v[j]);
                hist_add(hist, (key >> shift) & 1023u, i < p.rows && (key & pmask) == prefix);
            }
        }
        __syncthreads();
        uint32_t ab2, cnt2;
        const uint32_t bin2 = boundary_bin(hist, 1024, (uint32_t)k - above, ms, &ab2, &cnt2);
        above += ab2;
        cnt = cnt2;
        prefix |= bin2 << shift;
        pmask |= 1023u << shift;
    }
    L = prefix;
    S = (int)(above + cnt);
    if (S > p.s_cap) {
        batch_wide(p, b, k, greedy, temp, u0, hn, hhead, bsm, ms);
        return;
    }

    /* the superset {key >= L} (every candidate is in it) */
    if (tid == 0) s_count = 0;
    __syncthreads();
    for (int i0 = 0; i0 < p.rows; i0 += NT * U) {
        float v[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int i = i0 + j * NT + tid;
            v[j] = i < p.rows ? lg[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int i = i0 + j * NT + tid;
            const uint32_t key = f2key(v[j]);
            const bool take = i < p.rows && key >= L;
            const unsigned bal = __ballot_sync(0xffffffffu, take);
            int base = 0;
            if ((tid & 31) == 0 && bal) base = atomicAdd(&s_count, __popc(bal));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (take) {
                const int pos = base + __popc(bal & ((1u << (tid & 31)) - 1u));
                if (pos < p.s_cap) {
                    Sk[pos] = key;
                    Si[pos] = i;
                }
            }
        }
    }
    __syncthreads();
    }  /* full pass */

    /* Early weights (a superset of at most NT keys: one a thread): the
     * superset holds every candidate and the largest logit, so max_l
     * (runtime/lal_sampling.h:107-109) is known before T, and each key's
     * weight-table loads go out now and land during the select of T. */
    const bool early = !greedy && S <= NT;
    float max_l_e = -1e30f, xw = 0.0f;
    uint32_t bw = 0u, olo = 0u, ohi = 0u;
    if (early) {
        uint32_t mk = tid < S ? Sk[tid] : 0u;
        mk = __reduce_max_sync(0xffffffffu, mk);
        if ((tid & 31) == 0) ms->wmax[tid >> 5] = mk;
        __syncthreads();
        for (int w = 0; w < NWARP; ++w) mk = max(mk, ms->wmax[w]);
        max_l_e = fmaxf(-1e30f, key2f(mk));
        if (tid < S) {
            xw = __fdiv_rn(__fsub_rn(key2f(Sk[tid]), max_l_e), temp);
            bw = expf_bitmap_word(xw, p.expf_bits);
            expf_offsets(xw, p.expf_off, &olo, &ohi);
        }
        __syncthreads(); /* wmax is read before anything reuses it */
    }
    /* 4. T exactly: the k-th largest key of the superset (counting for a
     * small superset: T = min{ key : #{keys > key} < k }) */
    uint32_t T;
    if (S <= 128) {
        /* pad to a multiple of 4 with zero keys (never greater) and count with
         * 16-byte reads, two keys a thread in one pass */
        const int S4 = (S + 3) & ~3;
        if (tid < S4 - S) Sk[S + tid] = 0u;
        __syncthreads();
        uint32_t best = 0xffffffffu;
        const int kk = min(k, S);
        const uint32_t me0 = tid < S ? Sk[tid] : 0u;
        const uint32_t me1 = tid + NT < S ? Sk[tid + NT] : 0u;
        int g0 = 0, g1 = 0;
        const uint4 *K4 = reinterpret_cast<const uint4 *>(Sk);
#pragma unroll 4
        for (int j = 0; j < S4 / 4; ++j) {
            const uint4 v = K4[j];
            g0 += (v.x > me0) + (v.y > me0) + (v.z > me0) + (v.w > me0);
            g1 += (v.x > me1) + (v.y > me1) + (v.z > me1) + (v.w > me1);
        }
        if (tid < S && g0 < kk) best = me0;
        if (tid + NT < S && g1 < kk) best = min(best, me1);
        best = __reduce_min_sync(0xffffffffu, best);
        if ((tid & 31) == 0) ms->scan[tid >> 5] = best;
        __syncthreads();
        T = ms->scan[0];
        for (int w = 1; w < NWARP; ++w) T = min(T, ms->scan[w]);
        __syncthreads();
    } else {
        T = block_kth_largest(
            [&](int i, uint32_t &key) {
                key = Sk[i];
                return true;
            },
            S, min(k, S), ms);
    }
    /* candidates {l >= T} */
    const int seg = (S + NT - 1) / NT;
    const int e0 = min(S, tid * seg), e1 = min(S, e0 + seg);
    uint32_t c = 0;
    for (int e = e0; e < e1; ++e) c += Sk[e] >= T;
    uint32_t mt;
    uint32_t pos = block_scan_excl(c, ms, &mt);
    const int m = (int)mt;
    dg.threshold = key2f(T);
    dg.n_cand = m;
    if (m < 1 || m > p.c_cap || (p.shard_out != nullptr && m > p.rec_cap)) {
        batch_wide(p, b, k, greedy, temp, u0, hn, hhead, bsm, ms);
        return;
    }
    /* the candidates with their weights when early (Ce in the list's order;
     * with S <= NT the thread of superset entry e holds its loads) */
    for (int e = e0; e < e1; ++e)
        if (Sk[e] >= T) {
            Cv[pos] = key2f(Sk[e]);
            Ci[pos] = p.row_base + Si[e];
            if (early) Ce[pos] = expf_with_range(xw, bw, olo, ohi, p.expf_x, p.expf_y);
            ++pos;
        }
    __syncthreads();
    /* ascending vocab order (the early weights move with their rows) */
    if (ordered) {
        for (int i = tid; i < m; i += NT) {
            Oi[i] = Ci[i];
            Ov[i] = Cv[i];
        }
    } else if (m <= 64) {
        int me = 0, r = 0;
        float mv = 0.0f, mw = 0.0f;
        if (tid < m) {
            me = Ci[tid];
            mv = Cv[tid];
            mw = early ? Ce[tid] : 0.0f;
#pragma unroll 8
            for (int j = 0; j < m; ++j) r += Ci[j] < me;
        }
        __syncthreads();
        if (tid < m) {
            Oi[r] = me;
            Ov[r] = mv;
            if (early) Ce[r] = mw;
        }
    } else {
        int n2 = 1;
        while (n2 < m) n2 <<= 1;
        for (int i = tid; i < n2; i += NT) {
            Oi[i] = i < m ? Ci[i] : 0x7fffffff;
            Ov[i] = i < m ? Cv[i] : 0.0f;
            if (early && i >= m) Ce[i] = 0.0f;
        }
        __syncthreads();
        for (int size = 2; size <= n2; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < (n2 >> 1); i += NT) {
                    const int lo = (i / stride) * stride * 2 + (i % stride);
                    const int hi = lo + stride;
                    const bool asc = (lo & size) == 0;
                    const int a = Oi[lo], bb = Oi[hi];
                    if ((a > bb) == asc) {
                        Oi[lo] = bb;
                        Oi[hi] = a;
                        float t = Ov[lo];
                        Ov[lo] = Ov[hi];
                        Ov[hi] = t;
                        if (early) {
                            t = Ce[lo];
                            Ce[lo] = Ce[hi];
                            Ce[hi] = t;
                        }
                    }
                }
                __syncthreads();
            }
    }
    __syncthreads();

    if (p.shard_out != nullptr) {
        /* vocab-sharded step: this slice's record for the merge */
        uint8_t *rec = p.shard_out + (size_t)b * p.rec_bytes;
        ShardRecordHead *h = reinterpret_cast<ShardRecordHead *>(rec);
        float *rv = reinterpret_cast<float *>(rec + sizeof(ShardRecordHead));
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
            p.diag[b] = dg;
        }
        return;
    }

    /* 5. max over candidates floored at -1e30 (runtime/lal_sampling.h:107-109),
     * weights expf((l - max_l)/T), sequential sums in vocab order, draw */
    float max_l = max_l_e;
    if (!early) {
        float mx = -1e30f;
        for (int i = tid; i < m; i += NT) mx = fmaxf(mx, Ov[i]);
        max_l = block_max_f(mx, ms);
    }
    dg.max_l = max_l;
    int token;
    if (greedy) {
        token = Oi[0];
    } else {
        if (!early)
            for (int i = tid; i < m; i += NT) {
                const float x = __fdiv_rn(__fsub_rn(Ov[i], max_l), temp);
                Ce[i] = sampler_expf(x, p.expf_x, p.expf_y, p.expf_bits, p.expf_off);
            }
        __syncthreads();
        if (tid == 0) {
            /* values fetched eight at a time, the adds in order */
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
        dg.sum = sum;
        if (p.variant == VARIANT_SERVER && sum <= 0.0f) {
            /* tools/server/qwen7b_server.c:285-286 */
            token = 0;
            float bv = -1e30f;
            for (int i = 0; i < m; ++i)
                if (Ov[i] > bv) {
                    bv = Ov[i];
                    token = Oi[i];
                }
        } else {
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
        }
    }
    if (tid == 0) {
        dg.token = token;
        p.tokens[b] = token;
        p.diag[b] = dg;
        if (p.push_history && p.hist_cap > 0) {
            if (hn < p.hist_cap) {
                hids[hn] = token;
                p.hist_n[b] = hn + 1;
            } else {
                hids[hhead] = token;
                p.hist_head[b] = (hhead + 1) % p.hist_cap;
            }
        }
        if (p.host_tok) notify_host(p.host_tok + b, __ldcg(p.seq_in), token);
    }
}

/* ------------------------------------------------------------ host --- */
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

/* A launch that may begin while the previous kernel on the stream runs
 * (programmatic stream serialization); the kernel calls griddepcontrol.wait
 * before it reads anything that kernel writes. */
cudaError_t launch_dependent(const void *fn, int grid, int block, size_t smem, cudaStream_t st,
                             void **args) {
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

/* 2-D int8 tensor [dim1][dim0] (row pitch `pitch` bytes), box 128 x box1,
 * 128-byte swizzle; out-of-range rows and columns read as zero. */
bool encode_i8(CUtensorMap *m, const void *base, int dim0, int dim1, int pitch, int box1) {
    EncodeTiledFn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)dim0, (cuuint64_t)dim1};
    const cuuint64_t strides[1] = {(cuuint64_t)pitch};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box1};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

/* The tiles left over after the GEMM's last whole wave, split along K: rem
 * tiles in `chunks` chunks of `cb` boxes, one chunk a CTA (rem * chunks <=
 * grid), so the slowest CTA streams cb boxes more than the others instead
 * of a whole tile (kblocks boxes) more.  The partial dots, rem * chunks *
 * 128 * N ints, are kept to about 2^20 by longer chunks at large N: the
 * select adds each stream's share.  rem = 0: nothing is split. */
constexpr long kSplitPartsMax = 1l << 20;
struct SplitShape {
    int rem, chunks, cb;
};
SplitShape split_shape(int rows, int kblocks, int num_sms, int N) {
    const int n_tiles = (rows + kBM - 1) / kBM;
    const int grid = std::min(n_tiles, num_sms);
    SplitShape sh = {0, 0, 0};
    const int rem = grid > 0 ? n_tiles % grid : 0;
    if (rem == 0) return sh;
    const long per_chunk = (long)rem * kBM * std::max(1, N);
    const int by_adds = (int)std::min<long>(kblocks, std::max<long>(2, kSplitPartsMax / per_chunk));
    const int want = std::min({grid / rem, by_adds, kSplitChunksMax});
    if (want < 2) return sh;
    const int cb = (kblocks + want - 1) / want;
    const int chunks = (kblocks + cb - 1) / cb;
    if (chunks < 2 || rem * chunks > grid || 4 * rem > kSplitGroupsMax) return sh;
    sh.rem = rem;
    sh.chunks = chunks;
    sh.cb = cb;
    return sh;
}

}  // namespace

/* ---- the batched step, as seen by tail_api.cu ---- */
int batch_n_for(int B) { return (B + 31) / 32 * 32; }

size_t batch_split_bytes(int rows, int ld, int num_sms, int max_B) {
    size_t ints = 0;
    for (int N = 32; N <= batch_n_for(max_B); N += 32) {
        const SplitShape sh = split_shape(rows, (ld + kBK - 1) / kBK, num_sms, N);
        ints = std::max(ints, (size_t)sh.rem * sh.chunks * N * kBM);
    }
    return 4 * ints;
}

size_t batch_select_smem(int s_cap, int c_cap, int h_slots, int n_groups,
                         int stage_groups = kStageGroups) {
    const size_t fixed = 4ull * 4096 + 8ull * s_cap + 20ull * c_cap + 4ull * n_groups;
    return (fixed + 15) / 16 * 16 + std::max(8ull * h_slots, 128ull * stage_groups);
}

int batch_plan(BatchPlan &bp, const int8_t *W, const float *scale_w, int rows, int ld,
               int num_sms, int8_t *xq, float *sx, uint32_t *gmax, int *split_scratch,
               int max_B, int hist_cap, int max_top_k) {
    memset(&bp, 0, sizeof(bp));
    if (!encoder()) return -3;
    if (ld < kBK || ld % 16 != 0 || max_B < 2 || max_B > 256 || rows < 1) return -1;
    bp.W = W;
    bp.scale_w = scale_w;
    bp.rows = rows;
    bp.ld = ld;
    bp.xq = xq;
    bp.sx = sx;
    bp.gmax = gmax;
    bp.n_groups = batch_groups(rows);
    bp.num_sms = num_sms;
    bp.kblocks = (ld + kBK - 1) / kBK;
    if (split_scratch != nullptr) {
        bp.split_part = split_scratch;
        bp.split_ints = batch_split_bytes(rows, ld, num_sms, max_B) / 4;
        bp.split_rem = split_shape(rows, bp.kblocks, num_sms, 32).rem;
    }
    /* select capacities: superset, candidates, history hash (>= 2x the
     * history, a power of two) */
    /* superset >= the group maxima and 8x the largest k; candidates k plus
     * ties; small enough for several select CTAs per SM at small k */
    bp.s_cap = std::max({2048, batch_groups(rows), 8 * max_top_k});
    bp.s_cap = (bp.s_cap + 31) / 32 * 32;
    bp.c_cap = 256;
    while (bp.c_cap < 2 * max_top_k) bp.c_cap <<= 1;
    int hs = 64;
    while (hs < 2 * std::max(1, hist_cap)) hs <<= 1;
    bp.h_slots = hs;
    bp.wide_cap = std::max(1, std::min(max_top_k, rows));
    if (batch_select_smem(bp.s_cap, bp.c_cap, bp.h_slots, bp.n_groups) >
            (size_t)(kGemmSmemLimit - 8192) ||
        batch_select_smem(bp.s_cap, bp.c_cap, bp.h_slots, bp.n_groups) <
            (size_t)wide_area_bytes(bp.wide_cap))
        return -2;
    return 0;
}

cudaError_t batch_launch(BatchPlan &bp, const BatchStep &s, cudaStream_t st) {
    const int N = batch_n_for(s.B);
    if (s.B < 1 || N > 256) return cudaErrorInvalidValue;
    static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
    if (!bp.w_ready) {
        if (!encode_i8(reinterpret_cast<CUtensorMap *>(bp.tm_w), bp.W, bp.ld, bp.rows, bp.ld, kBM))
            return cudaErrorInvalidValue;
        bp.w_ready = 1;
    }
    const int xi = N / 32 - 1;
    if (!(bp.x_ready & (1u << xi))) {
        if (!encode_i8(reinterpret_cast<CUtensorMap *>(bp.tm_x[xi]), bp.xq, bp.ld, N, bp.ld, N))
            return cudaErrorInvalidValue;
        bp.x_ready |= 1u << xi;
    }
    /* 1. quantize the B hidden vectors */
    quantize_batch_kernel<<<s.B, NT, 0, st>>>(s.hidden, s.d, bp.xq, bp.ld, bp.sx, s.norm_w,
                                              s.norm_eps);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    /* 2. logits = X W^T on the tensor cores */
    GemmParams g;
    memset(&g, 0, sizeof(g));
    memcpy(&g.tmW, bp.tm_w, sizeof(CUtensorMap));
    memcpy(&g.tmX, bp.tm_x[xi], sizeof(CUtensorMap));
    g.scale_w = bp.scale_w;
    g.scale_x = bp.sx;
    g.logits = s.logits;
    g.gmax = bp.gmax;
    g.n_groups = bp.n_groups;
    g.rows = bp.rows;
    g.B = s.B;
    g.N = N;
    g.kblocks = bp.kblocks;
    g.stage_bytes = kBM * kBK + N * kBK;
    const int fixed = 1024 + 64 * 8 + 4 * 256 + 64; /* alignment, barriers, scales */
    g.stages = std::min(kGemmStagesMax, (kGemmSmemLimit - fixed) / g.stage_bytes);
    if (g.stages < 2) return cudaErrorInvalidValue;
    int cols = 32;
    while (cols < 2 * N) cols <<= 1;
    g.tmem_cols = cols;
    g.status = s.status;
    const size_t gsmem = (size_t)g.stages * g.stage_bytes + fixed;
    e = raise_smem((const void *)gemm_i8_kernel, kGemmSmemLimit);
    if (e != cudaSuccess) return e;
    const int n_tiles = (bp.rows + kBM - 1) / kBM;
    const int grid = std::min(n_tiles, bp.num_sms);
    g.reg_end = n_tiles;
    const SplitShape sh = split_shape(bp.rows, bp.kblocks, bp.num_sms, N);
    if (bp.split_part != nullptr && sh.rem > 0 && sh.rem == bp.split_rem &&
        (size_t)sh.rem * sh.chunks * N * kBM <= bp.split_ints) {
        g.reg_end = n_tiles - sh.rem;
        g.split_units = sh.rem * sh.chunks;
        g.split_chunks = sh.chunks;
        g.split_cb = sh.cb;
        g.split_part = bp.split_part;
    }
    if (s.gemm_ev0) {
        e = cudaEventRecord(s.gemm_ev0, st);
        if (e != cudaSuccess) return e;
    }
    {
        void *args[] = {&g};
        e = launch_dependent((const void *)gemm_i8_kernel, grid, kGemmThreads, gsmem, st, args);
        if (e != cudaSuccess) return e;
    }
    if (s.gemm_ev1) {
        e = cudaEventRecord(s.gemm_ev1, st);
        if (e != cudaSuccess) return e;
    }
    /* 3. per stream: penalty, select, draw (or the shard record) */
    BatchSelectParams q;
    memset(&q, 0, sizeof(q));
    q.logits = s.logits;
    q.rows = bp.rows;
    q.row_base = s.row_base;
    q.vocab = s.vocab;
    q.variant = s.variant;
    q.temperature = s.temperature;
    q.top_k = s.top_k;
    q.rep_penalty = s.rep_penalty;
    q.u = s.u;
    q.hist_ids = s.hist_ids;
    q.hist_n = s.hist_n;
    q.hist_head = s.hist_head;
    q.hist_cap = s.hist_cap;
    q.hist_stride = s.hist_stride;
    q.push_history = s.push_history;
    q.tokens = s.tokens;
    q.diag = s.diag;
    q.status = s.status;
    q.expf_x = s.expf_x;
    q.expf_y = s.expf_y;
    q.expf_n = s.expf_n;
    q.expf_bits = s.expf_bits;
    q.expf_off = s.expf_off;
    q.shard_out = s.shard_out;
    q.rec_cap = s.rec_cap;
    q.rec_bytes = s.rec_bytes;
    q.s_cap = bp.s_cap;
    q.c_cap = bp.c_cap;
    q.h_slots = bp.h_slots;
    q.gmax = bp.gmax;
    q.n_groups = bp.n_groups;
    q.wide_cap = bp.wide_cap;
    q.host_tok = s.shard_out ? nullptr : s.host_tok;
    q.seq_in = s.seq_in;
    if (g.split_part != nullptr) {
        q.split_part = g.split_part;
        q.split_rem = n_tiles - g.reg_end;
        q.split_chunks = g.split_chunks;
        q.split_n = N;
        q.split_row0 = g.reg_end * kBM;
        q.scale_w = bp.scale_w;
        q.scale_x = bp.sx;
    }
    e = raise_smem((const void *)batch_select_kernel, kGemmSmemLimit - 8192);
    if (e != cudaSuccess) return e;
    /* one select CTA a stream: with more streams than SMs, the largest
     * staging round that lets two CTAs share an SM, if any (decided once) */
    if (s.B > bp.num_sms && bp.stage_groups_many == 0) {
        bp.stage_groups_many = kStageGroups;
        for (int sg = kStageGroups; sg >= kStageGroupsMin; sg -= 32) {
            const size_t sm_bytes =
                batch_select_smem(bp.s_cap, bp.c_cap, bp.h_slots, bp.n_groups, sg);
            if (sm_bytes < (size_t)wide_area_bytes(bp.wide_cap)) break;
            int per_sm = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                    &per_sm, (const void *)batch_select_kernel, NT, sm_bytes) != cudaSuccess) {
                (void)cudaGetLastError(); /* the failed query leaves no error behind */
                break;
            }
            if (per_sm >= 2) {
                bp.stage_groups_many = sg;
                break;
            }
        }
    }
    q.stage_groups = s.B > bp.num_sms ? bp.stage_groups_many : kStageGroups;
    const size_t ssmem =
        batch_select_smem(bp.s_cap, bp.c_cap, bp.h_slots, bp.n_groups, q.stage_groups);
    void *args[] = {&q};
    return launch_dependent((const void *)batch_select_kernel, s.B, NT, ssmem, st, args);
}

}  // namespace lal
