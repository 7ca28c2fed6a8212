/*
 * tail_device.cuh -- device helpers shared by the sm_100a kernels
 * (tail_kernels.cu, tail_batch.cu): mbarrier and bulk-copy PTX, bounded
 * waits, the glibc-exact expf lookup, float order keys, block-wide scans,
 * maxima, histogram boundaries and the radix k-th-largest select.  Every
 * function has internal linkage (each kernel file gets its own copy).
 */
#pragma once

#include <cstddef>

#include "tail_internal.h"
#include "lal_expf.h"

namespace lal {
namespace {

constexpr int NT = kThreads;
constexpr int NWARP = NT / 32;

/* ---------------------------------------------------------------- PTX --- */
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

/* 16-byte asynchronous global -> shared copy (L2 only) and the wait for all
 * of this thread's copies */
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
/* Every wait is bounded: it gives up after kWaitNs of wall time (globaltimer)
 * or as soon as another warp of the CTA has given up. */
constexpr uint64_t kWaitNs = 2000000000ull;
__device__ bool mbar_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try(b, parity)) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try(b, parity)) return true;
        if ((it & 63u) == 0) {
            if (*abort_flag) return false;
            if (gtimer() - t0 > kWaitNs) return false;
        }
    }
}
/* Programmatic dependent launch: wait until the preceding kernel on the
 * stream has completed and its writes are visible (returns at once when the
 * launch did not overlap one); let the next launch begin to schedule. */
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
/* Bulk (non-tensor) TMA copy global -> this CTA's shared memory. */
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

/* The glibc fix-up of x, whose bitmap bit is set: the entries of x's bitmap
 * word (8192 bit patterns) are tx[off[w] .. off[w+1]), a few at most. */
__device__ __forceinline__ float expf_fixup(float x, const uint32_t *tx, const uint32_t *ty,
                                            const uint32_t *off) {
    const uint32_t xb = __float_as_uint(x);
    const uint32_t w = (xb - 0x80000000u) >> 13;
    const uint32_t lo = __ldg(off + w), hi = __ldg(off + w + 1);
    for (uint32_t i = lo; i < hi; ++i)
        if (__ldg(tx + i) == xb) return __uint_as_float(__ldg(ty + i));
    return lal_expf_rounded(x);
}

/* The sampler's weight function: glibc-exact expf (lal_expf.h) with the
 * fix-up table gated by a membership bitmap, so that nearly every call costs
 * one bitmap load, and a flagged one two more plus a short scan. */
__device__ __forceinline__ float sampler_expf(float x, const uint32_t *tx, const uint32_t *ty,
                                              const uint32_t *bits, const uint32_t *off) {
    const uint32_t xb = __float_as_uint(x);
    if (!(xb & 0x80000000u) || !(x <= 0.0f)) return lal_expf_rounded(x);
    const uint32_t b = (xb - 0x80000000u) >> 8;
    if (!((__ldg(bits + (b >> 5)) >> (b & 31)) & 1u)) return lal_expf_rounded(x);
    return expf_fixup(x, tx, ty, off);
}

/* sampler_expf in two halves, so the bitmap load can be in flight while
 * other work runs: the first returns the raw bitmap word (0 when x takes no
 * fix-up), the second finishes with it. */
__device__ __forceinline__ uint32_t expf_bitmap_word(float x, const uint32_t *bits) {
    const uint32_t xb = __float_as_uint(x);
    if (!(xb & 0x80000000u) || !(x <= 0.0f)) return 0u;
    return __ldg(bits + (((xb - 0x80000000u) >> 8) >> 5));
}
__device__ __forceinline__ float expf_with_word(float x, uint32_t word, const uint32_t *tx,
                                                const uint32_t *ty, const uint32_t *off) {
    const uint32_t xb = __float_as_uint(x);
    const uint32_t b = (xb - 0x80000000u) >> 8;
    if ((xb & 0x80000000u) && x <= 0.0f && ((word >> (b & 31)) & 1u))
        return expf_fixup(x, tx, ty, off);
    return lal_expf_rounded(x);
}

/* The table range of x's bitmap word (loaded beside the word itself, so a
 * flagged x needs one more round trip, not two); 0..0 for x the table never
 * holds (x > 0, NaN). */
__device__ __forceinline__ void expf_offsets(float x, const uint32_t *off, uint32_t *lo,
                                             uint32_t *hi) {
    const uint32_t xb = __float_as_uint(x);
    if ((xb & 0x80000000u) && x <= 0.0f) {
        const uint32_t w = (xb - 0x80000000u) >> 13;
        *lo = __ldg(off + w);
        *hi = __ldg(off + w + 1);
    } else {
        *lo = 0u;
        *hi = 0u;
    }
}
__device__ __forceinline__ float expf_with_range(float x, uint32_t word, uint32_t lo, uint32_t hi,
                                                 const uint32_t *tx, const uint32_t *ty) {
    const uint32_t xb = __float_as_uint(x);
    const uint32_t b = (xb - 0x80000000u) >> 8;
    if ((xb & 0x80000000u) && x <= 0.0f && ((word >> (b & 31)) & 1u))
        for (uint32_t i = lo; i < hi; ++i)
            if (__ldg(tx + i) == xb) return __uint_as_float(__ldg(ty + i));
    return lal_expf_rounded(x);
}

/* Hash form of the fix-up lookup, in two halves: the first issues the one
 * 16-byte load of x's bucket (volatile, so it goes out where it is written,
 * ahead of the work that hides its latency); the second resolves it, probing
 * further buckets only when x's is full and holds neither x nor a gap. */
__device__ __forceinline__ uint4 expf_hash_load(float x, const uint4 *hash) {
    const uint32_t xb = __float_as_uint(x);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if ((xb & 0x80000000u) && x <= 0.0f) {
        const uint4 *a = hash + expf_hash_bucket(xb);
        asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(a));
    }
    return v;
}
__device__ __forceinline__ float expf_hash_finish(float x, uint4 pr, const uint4 *hash,
                                                  int max_probe) {
    const uint32_t xb = __float_as_uint(x);
    if ((xb & 0x80000000u) && x <= 0.0f) {
        uint32_t bk = expf_hash_bucket(xb);
        for (int probe = 0; probe < max_probe; ++probe) {
            if (pr.x == xb) return __uint_as_float(pr.y);
            if (pr.x == 0u) break;
            if (pr.z == xb) return __uint_as_float(pr.w);
            if (pr.z == 0u) break;
            bk = (bk + 1u) & (kExpfHashPairs - 1u);
            pr = __ldg(hash + bk);
        }
    }
    return lal_expf_rounded(x);
}

/* expf_hash_finish with the rounded value yr = lal_expf_rounded(x) computed
 * earlier (so its double-precision latency hides behind other work). */
__device__ __forceinline__ float expf_hash_resolve(float x, float yr, uint4 pr, const uint4 *hash,
                                                   int max_probe) {
    const uint32_t xb = __float_as_uint(x);
    if ((xb & 0x80000000u) && x <= 0.0f) {
        uint32_t bk = expf_hash_bucket(xb);
        for (int probe = 0; probe < max_probe; ++probe) {
            if (pr.x == xb) return __uint_as_float(pr.y);
            if (pr.x == 0u) break;
            if (pr.z == xb) return __uint_as_float(pr.w);
            if (pr.z == 0u) break;
            bk = (bk + 1u) & (kExpfHashPairs - 1u);
            pr = __ldg(hash + bk);
        }
    }
    return yr;
}

/* ------------------------------------------------------- order keys --- */
/* Monotone map float -> uint32 (larger float, larger key).  -0 maps like +0,
 * so key equality is float equality, as the reference's comparisons treat it. */
__device__ __forceinline__ uint32_t f2key(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

/* ------------------------------------------------- block primitives --- */
struct Misc {
    uint32_t hist[256];
    uint32_t scan[NWARP + 1];
    uint32_t sh[16];
    float fred[NWARP];
    float sx;
    float nrm[8];  /* the RMSNorm lane sums */
    float ninv;    /* inv_rms */
    float sum;
    int abort_flag;
    int ticket;
    int found;
    uint32_t cnt;           /* compaction counter of the small-k select */
    uint32_t wmax[NWARP];   /* per-warp largest key of the CTA's rows */
    /* the last CTA's copy of the per-CTA maxima (read as 16-byte vectors) */
    alignas(16) uint32_t gm[kMaxGrid];
};
static_assert(offsetof(Misc, gm) % 16 == 0, "Misc::gm must be 16-byte aligned");

/* Grid-wide barrier of a cooperative launch (every CTA resident).  The
 * wait is bounded: after kWaitNs it records DEV_TIMEOUT and returns false.
 * bar[0] counts arrivals, bar[1] is the generation; the last arriver resets
 * the count before publishing the next generation (release), so the words
 * are ready for the next barrier and the next launch. */
__device__ bool grid_sync(unsigned *bar, unsigned G, Misc *ms, int *status) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned gen = ld_acquire_gpu(bar + 1);
        __threadfence();
        const unsigned arrived = atomicAdd(bar, 1u) + 1u;
        unsigned ok = 1u;
        if (arrived == G) {
            bar[0] = 0u;
            __threadfence();
            st_release_gpu(bar + 1, gen + 1u);
        } else {
            const uint64_t t0 = gtimer();
            while (ld_acquire_gpu(bar + 1) == gen) {
                if (gtimer() - t0 > kWaitNs) {
                    ok = 0u;
                    atomicCAS(status, 0, (int)DEV_TIMEOUT);
                    break;
                }
            }
        }
        ms->sh[15] = ok;
    }
    __syncthreads();
    return ms->sh[15] != 0u;
}

/* Exclusive prefix (thread order) of one value per thread; *total = sum. */
__device__ __forceinline__ uint32_t block_scan_excl(uint32_t v, Misc *ms, uint32_t *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) ms->scan[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < NWARP ? ms->scan[lane] : 0u;
        uint32_t incl = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane < NWARP) ms->scan[lane] = incl - w;
        if (lane == NWARP - 1) ms->scan[NWARP] = incl;
    }
    __syncthreads();
    const uint32_t res = ms->scan[warp] + x - v;
    *total = ms->scan[NWARP];
    __syncthreads();
    return res;
}

/* Barrier among the kConsumerWarps consumer warps only (named barrier 1), so
 * the producer warp can stream while the consumers run the prologue. */
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

/* max over the consumer warps' values (consumer threads only) */
__device__ __forceinline__ float consumer_max_f(float v, Misc *ms) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) ms->fred[warp] = v;
    consumer_sync();
    float r = ms->fred[0];
#pragma unroll
    for (int w = 1; w < kConsumerWarps; ++w) r = fmaxf(r, ms->fred[w]);
    consumer_sync();
    return r;
}

__device__ __forceinline__ void stamp(const TailParams &p, int slot) {
    if (p.phase_ts) p.phase_ts[slot] = gtimer();
}

__device__ __forceinline__ float block_max_f(float v, Misc *ms) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) ms->fred[warp] = v;
    __syncthreads();
    float r = ms->fred[0];
#pragma unroll
    for (int w = 1; w < NWARP; ++w) r = fmaxf(r, ms->fred[w]);
    __syncthreads();
    return r;
}

/* Boundary bin of a histogram h[0..nb) scanned from the top bin down: the bin
 * holding the krem-th largest entry (1 <= krem <= total).  Returns the bin;
 * *above gets the count in higher bins, *count the bin's own count.  All
 * threads of the block call it. */
__device__ uint32_t boundary_bin(const uint32_t *h, int nb, uint32_t krem, Misc *ms,
                                 uint32_t *above, uint32_t *count) {
    const int per = (nb + NT - 1) / NT;
    const int q0 = threadIdx.x * per; /* descending positions q <-> bin nb-1-q */
    const int q1 = min(nb, q0 + per);
    uint32_t s = 0;
    for (int q = q0; q < q1; ++q) s += h[nb - 1 - q];
    uint32_t tot;
    const uint32_t ex = block_scan_excl(s, ms, &tot);
    if (ex < krem && krem <= ex + s) {
        uint32_t run = ex;
        for (int q = q0; q < q1; ++q) {
            const uint32_t c = h[nb - 1 - q];
            if (run + c >= krem) {
                ms->sh[0] = (uint32_t)(nb - 1 - q);
                ms->sh[1] = run;
                ms->sh[2] = c;
                break;
            }
            run += c;
        }
    }
    __syncthreads();
    const uint32_t bin = ms->sh[0];
    *above = ms->sh[1];
    *count = ms->sh[2];
    __syncthreads();
    return bin;
}

/* The reference's final RMSNorm (runtime/lal_simd_optim.h:32-58, the
 * AVX2+FMA build the servers use; called at tools/server/qwen7b_server.c:820),
 * for n a multiple of 8 (the reference's scalar tail loop is then empty):
 *   lane j of eight accumulates x[i]^2 for i = j (mod 8) with fused
 *   multiply-adds in index order (rmsnorm_lane, one thread a lane); the
 *   lanes combine as ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)) -- the two 128-bit
 *   halves added, then two horizontal adds; inv_rms = 1 / sqrtf(ms / n + eps);
 *   the output is (x[i] * inv_rms) * w[i]. */
__device__ __forceinline__ float rmsnorm_lane(const float *xs, int n, int j) {
    float acc = 0.0f;
#pragma unroll 8
    for (int i = j; i < n; i += 8) acc = __fmaf_rn(xs[i], xs[i], acc);
    return acc;
}
__device__ __forceinline__ float rmsnorm_inv(const float *v, int n, float eps) {
    const float s0 = __fadd_rn(v[0], v[4]), s1 = __fadd_rn(v[1], v[5]);
    const float s2 = __fadd_rn(v[2], v[6]), s3 = __fadd_rn(v[3], v[7]);
    const float ms = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ms, (float)n), eps)));
}
__device__ __forceinline__ float rmsnorm_apply(float x, float inv, float w) {
    return __fmul_rn(__fmul_rn(x, inv), w);
}

/* boundary_bin for one warp on a 4096-bin histogram whose highest non-empty
 * bin is top: lanes sum 16 bins each (four 16-byte reads) in windows of 512
 * bins going down from top, a warp scan finds the window, the lane and the
 * bin where the count from the top reaches krem (1 <= krem <= the total).
 * Every lane returns the bin. */
__device__ __forceinline__ uint32_t warp_boundary_bin_4096(const uint32_t *h, uint32_t top,
                                                           uint32_t krem) {
    const int lane = threadIdx.x & 31;
    uint32_t run = 0u;
    for (int hi = (int)(top | 15u); hi >= 0; hi -= 512) {
        const int base = hi - 16 * lane - 15; /* this lane's group [base, base + 15] */
        uint32_t c[16];
        uint32_t sum = 0u;
        if (base >= 0) {
            const uint4 *g = reinterpret_cast<const uint4 *>(h + base);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const uint4 x = g[v];
                c[15 - 4 * v] = x.x; /* c[q] = bin base + 15 - q: descending */
                c[14 - 4 * v] = x.y;
                c[13 - 4 * v] = x.z;
                c[12 - 4 * v] = x.w;
            }
        } else {
#pragma unroll
            for (int q = 0; q < 16; ++q) c[q] = 0u;
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) sum += c[q];
        uint32_t incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
        if (run + total >= krem) {
            const uint32_t ex = run + incl - sum;
            const unsigned who = __ballot_sync(0xffffffffu, ex < krem && krem <= ex + sum);
            uint32_t bin = 0u;
            if (lane == __ffs(who) - 1) {
                uint32_t r = ex;
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    if (r < krem && r + c[q] >= krem) bin = (uint32_t)(base + 15 - q);
                    r += c[q];
                }
            }
            return __shfl_sync(0xffffffffu, bin, __ffs(who) - 1);
        }
        run += total;
    }
    return 0u;
}

/* k-th largest key of the valid entries among i in [0, n): get(i, key)
 * returns whether entry i takes part and sets its key; 1 <= k <= the number
 * of valid entries.  MSB-first radix select with 8-bit digits; histogram adds
 * are aggregated per warp (match.any). */
template <class Get>
__device__ uint32_t block_kth_largest(Get get, int n, int k, Misc *ms) {
    uint32_t prefix = 0, mask = 0;
    int krem = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += NT) ms->hist[i] = 0;
        __syncthreads();
        for (int i0 = 0; i0 < n; i0 += NT) {
            const int i = i0 + threadIdx.x;
            uint32_t key = 0u;
            const bool act = i < n && get(i, key);
            const bool m = act && ((key & mask) == prefix);
            const uint32_t digit = (key >> shift) & 0xFFu;
            const unsigned voters = __ballot_sync(0xffffffffu, m);
            if (m) {
                const unsigned peers = __match_any_sync(voters, digit);
                if ((int)(threadIdx.x & 31) == __ffs(peers) - 1)
                    atomicAdd(&ms->hist[digit], (uint32_t)__popc(peers));
            }
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            uint32_t c[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = ms->hist[255 - 8 * lane - j];
                s += c[j];
            }
            uint32_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t excl = incl - s;
            if (excl < (uint32_t)krem && (uint32_t)krem <= incl) {
                uint32_t run = excl;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (run + c[j] >= (uint32_t)krem) {
                        ms->sh[0] = 255u - 8u * lane - j;
                        ms->sh[1] = run;
                        break;
                    }
                    run += c[j];
                }
            }
        }
        __syncthreads();
        const uint32_t digit = ms->sh[0];
        krem -= (int)ms->sh[1];
        prefix |= digit << shift;
        mask |= 0xFFu << shift;
        __syncthreads();
    }
    return prefix;
}

/* A pair of 64-bit words of a peer record, stored and loaded as one aligned
 * 16-byte access (each word single-copy atomic on its own; readers check the
 * sequence number in both). */
__device__ __forceinline__ void st_sys_pair(uint64_t *p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b)
                 : "memory");
}
__device__ __forceinline__ void ld_sys_pair(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p)
                 : "memory");
}
/* Wait (bounded by the globaltimer deadline) until both words of a pair
 * carry sequence number seq. */
__device__ __forceinline__ bool poll_pair(const uint64_t *w, uint32_t seq, uint64_t deadline,
                                          uint64_t &a, uint64_t &b) {
    for (uint32_t it = 0;; ++it) {
        ld_sys_pair(w, a, b);
        if ((uint32_t)(a >> 32) == seq && (uint32_t)(b >> 32) == seq) return true;
        if ((it & 15u) == 15u && gtimer() > deadline) return false;
    }
}

/* The step's token (or -1) into the caller's completion word in mapped
 * pinned host memory, tagged with the step's sequence number in the high
 * half; one 64-bit system-scope store after a system fence, so the host
 * that sees the sequence number has the token and every earlier write. */
__device__ __forceinline__ void notify_host(unsigned long long *w, unsigned seq, int token) {
    if (w == nullptr) return;
    __threadfence_system();
    const unsigned long long v = ((unsigned long long)seq << 32) | (uint32_t)token;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(w), "l"(v) : "memory");
}

/* Penalty for one logit with `count` history occurrences, one step per
 * occurrence as runtime/lal_sampling.h:63-64 does (not a power). */
__device__ __forceinline__ float penalise(float l, uint32_t count, float pen) {
    for (uint32_t c = 0; c < count; ++c) l = (l > 0.0f) ? __fdiv_rn(l, pen) : __fmul_rn(l, pen);
    return l;
}

}  // namespace
}  // namespace lal
