/*
 * tail_api.cu -- the C ABI of liblal_tail.so (include/lal_tail.h): contexts,
 * device memory, streams, the host-LM-head registry of the drop-ins, and the
 * launch of the kernels in tail_kernels.cu.  Host code only.
 *
 * There is no CPU path: every computation is a kernel launch; a missing GPU
 * or a CUDA error is reported (status-returning functions) or aborts the
 * process (the void / token-returning drop-ins, which have no error channel).
 */
#define LAL_TAIL_BUILDING 1
#include "../../include/lal_tail.h"
#include "../../include/runtime/lal_q8_kernel.h"
#include "../../include/runtime/lal_sampling.h"
#include "tail_internal.h"

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

/* glibc-expf fix-up table, embedded at build time (expf_blob.S). */
extern "C" const unsigned char lal_expf_fixups_blob[];
extern "C" const unsigned char lal_expf_fixups_blob_end[];

using namespace lal;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CU(call)                                                                       \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess)                                                         \
            return fail(LAL_TAIL_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                        __FILE__, __LINE__);                                           \
    } while (0)

#define CHECK(expr)                                                                    \
    do {                                                                               \
        int rc_ = (expr);                                                              \
        if (rc_ != LAL_TAIL_OK) return rc_;                                            \
    } while (0)

/* Drop-ins without an error channel: report and stop (no CPU fallback). */
[[noreturn]] void die(const char *where) {
    fprintf(stderr, "liblal_tail: %s failed: %s\n", where, g_err.c_str());
    fflush(stderr);
    abort();
}

/* ---- per-device state: SM count and the expf fix-up table ------------ */
struct DeviceState {
    bool ready = false;
    int num_sms = 0;
    uint32_t *d_expf_x = nullptr, *d_expf_y = nullptr, *d_expf_bits = nullptr,
             *d_expf_off = nullptr;
    int expf_n = 0;
    uint4 *d_expf_hash = nullptr; /* kExpfHashPairs buckets of two (x, y) slots */
    int expf_hash_probe = 0;
};
std::mutex g_dev_mu;
DeviceState g_dev[64];

int device_state(int dev, DeviceState **out) {
    if (dev < 0 || dev >= 64) return fail(LAL_TAIL_ERR_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceState &ds = g_dev[dev];
    if (!ds.ready) {
        CU(cudaSetDevice(dev));
        CU(cudaDeviceGetAttribute(&ds.num_sms, cudaDevAttrMultiProcessorCount, dev));
        int major = 0;
        CU(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10)
            return fail(LAL_TAIL_ERR_UNSUPPORTED, "device %d is sm_%d0; this library is built for sm_100a",
                        dev, major);
        const size_t blob = (size_t)(lal_expf_fixups_blob_end - lal_expf_fixups_blob);
        uint32_t n = 0;
        if (blob < 4) return fail(LAL_TAIL_ERR_STATE, "expf fix-up table missing from the build");
        memcpy(&n, lal_expf_fixups_blob, 4);
        if (blob < 4 + 8ull * n) return fail(LAL_TAIL_ERR_STATE, "expf fix-up table truncated");
        CU(cudaMalloc(&ds.d_expf_x, 4ull * n + 4));
        CU(cudaMalloc(&ds.d_expf_y, 4ull * n + 4));
        CU(cudaMemcpy(ds.d_expf_x, lal_expf_fixups_blob + 4, 4ull * n, cudaMemcpyHostToDevice));
        CU(cudaMemcpy(ds.d_expf_y, lal_expf_fixups_blob + 4 + 4ull * n, 4ull * n,
                      cudaMemcpyHostToDevice));
        /* membership bitmap: most lookups end after one load */
        std::vector<uint32_t> bits(kExpfBitmapWords, 0u);
        for (uint32_t i = 0; i < n; ++i) {
            uint32_t xb;
            memcpy(&xb, lal_expf_fixups_blob + 4 + 4ull * i, 4);
            const uint32_t b = (xb - 0x80000000u) >> 8;
            bits[b >> 5] |= 1u << (b & 31);
        }
        CU(cudaMalloc(&ds.d_expf_bits, 4ull * kExpfBitmapWords));
        CU(cudaMemcpy(ds.d_expf_bits, bits.data(), 4ull * kExpfBitmapWords, cudaMemcpyHostToDevice));
        /* off[w] = first table entry whose bitmap word is >= w (table sorted) */
        std::vector<uint32_t> off(kExpfBitmapWords + 1, n);
        {
            uint32_t i = 0;
            for (uint32_t w = 0; w <= (uint32_t)kExpfBitmapWords; ++w) {
                while (i < n) {
                    uint32_t xb;
                    memcpy(&xb, lal_expf_fixups_blob + 4 + 4ull * i, 4);
                    if (((xb - 0x80000000u) >> 13) >= w) break;
                    ++i;
                }
                off[w] = i;
            }
        }
        CU(cudaMalloc(&ds.d_expf_off, 4ull * (kExpfBitmapWords + 1)));
        CU(cudaMemcpy(ds.d_expf_off, off.data(), 4ull * (kExpfBitmapWords + 1),
                      cudaMemcpyHostToDevice));
        /* the hash form: linear probing by bucket, the first free slot */
        std::vector<uint32_t> hash(4ull * kExpfHashPairs, 0u);
        int probe_max = 1;
        for (uint32_t i = 0; i < n; ++i) {
            uint32_t xb, yb;
            memcpy(&xb, lal_expf_fixups_blob + 4 + 4ull * i, 4);
            memcpy(&yb, lal_expf_fixups_blob + 4 + 4ull * n + 4ull * i, 4);
            uint32_t bk = expf_hash_bucket(xb);
            for (int probe = 1;; ++probe) {
                uint32_t *slot = &hash[4ull * bk];
                const int at = slot[0] == 0u ? 0 : (slot[2] == 0u ? 2 : -1);
                if (at >= 0) {
                    slot[at] = xb;
                    slot[at + 1] = yb;
                    probe_max = std::max(probe_max, probe);
                    break;
                }
                bk = (bk + 1u) & (kExpfHashPairs - 1u);
            }
        }
        CU(cudaMalloc(&ds.d_expf_hash, 16ull * kExpfHashPairs));
        CU(cudaMemcpy(ds.d_expf_hash, hash.data(), 16ull * kExpfHashPairs,
                      cudaMemcpyHostToDevice));
        ds.expf_hash_probe = probe_max;
        ds.expf_n = (int)n;
        ds.ready = true;
    }
    *out = &ds;
    return LAL_TAIL_OK;
}

int current_device(int *dev) {
    CU(cudaGetDevice(dev));
    return LAL_TAIL_OK;
}

int ld_for(int d) { return (d + 15) / 16 * 16; }

/* an environment switch is on when set to anything but "" or "0" */
bool getenv_flag(const char *name) {
    const char *v = getenv(name);
    return v && v[0] && !(v[0] == '0' && v[1] == 0);
}

/* ---- growable device buffer ------------------------------------------- */
struct DevBuf {
    void *p = nullptr;
    size_t cap = 0;
    int ensure(size_t bytes) {
        if (bytes <= cap) return LAL_TAIL_OK;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        size_t want = bytes < 256 ? 256 : bytes;
        CU(cudaMalloc(&p, want));
        cap = want;
        return LAL_TAIL_OK;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

/* Scratch of the select (global memory beyond inputs and outputs): the key
 * histogram, grid-barrier words, superset buffer, arrival ticket. */
struct SelectScratch {
    unsigned *ghist = nullptr, *gbar = nullptr, *gcount = nullptr, *counter = nullptr,
             *gL = nullptr, *gmax = nullptr, *gslot_n = nullptr;
    uint32_t *gkey = nullptr;
    int *gidx = nullptr;
    int cap = 0;
    static constexpr size_t kWords = kHistWords + 8 + 2 * kMaxGrid;
    int alloc(int cap_) {
        CU(cudaMalloc(&ghist, 4ull * kWords));
        gbar = ghist + kHistWords;
        gcount = gbar + 2;
        counter = gbar + 3;
        gL = gbar + 4;
        gmax = gbar + 8;
        gslot_n = gmax + kMaxGrid;
        CU(cudaMemset(ghist, 0, 4ull * kWords));
        /* the small-k path uses one slot of kSlot entries per CTA */
        cap = std::max(cap_, kSelectCapMin);
        CU(cudaMalloc(&gkey, 4ull * cap));
        CU(cudaMalloc(&gidx, 4ull * cap));
        return LAL_TAIL_OK;
    }
    /* after a device error the words may be mid-update: start clean */
    int reset(cudaStream_t st) {
        CU(cudaMemsetAsync(ghist, 0, 4ull * kWords, st));
        return LAL_TAIL_OK;
    }
    void free_all() {
        if (ghist) cudaFree(ghist);
        if (gkey) cudaFree(gkey);
        if (gidx) cudaFree(gidx);
        ghist = gbar = gcount = counter = gL = gmax = gslot_n = nullptr;
        gkey = nullptr;
        gidx = nullptr;
    }
    void fill(TailParams &p) const {
        p.ghist = ghist;
        p.gbar = gbar;
        p.gcount = gcount;
        p.gL = gL;
        p.gmax = gmax;
        p.gslot_n = gslot_n;
        p.counter = counter;
        p.gcand_key = gkey;
        p.gcand_idx = gidx;
        p.gcand_cap = cap;
    }
};

/* Scratch of the drop-ins' launches (one set per host thread). */
struct LaunchScratch {
    DevBuf status, diag, tokens, params, hist, cand_v, cand_i, keep, prefix, u;
    SelectScratch sel;
    bool ready = false;
    ~LaunchScratch() { sel.free_all(); }
    int ensure(int vocab) {
        if (ready && vocab <= sel.cap) return LAL_TAIL_OK;
        if (sel.ghist) {
            CU(cudaDeviceSynchronize());
            sel.free_all();
        }
        CHECK(sel.alloc(std::max(vocab, 1 << 16)));
        CHECK(status.ensure(64));
        CU(cudaMemset(status.p, 0, 64));
        CHECK(diag.ensure(sizeof(StreamDiag)));
        CHECK(tokens.ensure(64));
        CHECK(params.ensure(64));
        ready = true;
        return LAL_TAIL_OK;
    }
};

/* ---- per-thread state of the drop-ins ---------------------------------- */
struct DropinState {
    int device = -1;
    cudaStream_t stream = nullptr;
    DevBuf x, xq, ax, logits, W, q, s;
    LaunchScratch ls;
    ~DropinState() {
        if (stream) cudaStreamDestroy(stream);
    }
};
thread_local std::unique_ptr<DropinState> t_drop;

int dropin(DropinState **out, DeviceState **ds) {
    int dev;
    CHECK(current_device(&dev));
    CHECK(device_state(dev, ds));
    if (!t_drop || t_drop->device != dev) {
        t_drop.reset(new DropinState());
        t_drop->device = dev;
        CU(cudaStreamCreateWithFlags(&t_drop->stream, cudaStreamNonBlocking));
    }
    *out = t_drop.get();
    return LAL_TAIL_OK;
}

/* ---- registry of host LM heads used by the range drop-ins -------------- */
struct LmHead {
    int device = -1;
    int d = 0, ld = 0, rows = 0;
    const float *host_scale = nullptr;
    int8_t *W = nullptr;
    float *sw = nullptr;
};
std::mutex g_reg_mu;
std::map<const int8_t *, LmHead> g_reg;
std::vector<void *> g_retired; /* buffers replaced while a launch may still read them */

int upload_rows(const int8_t *host, int rows, int d, int ld, int8_t *dst, cudaStream_t st) {
    if (ld == d) {
        CU(cudaMemcpyAsync(dst, host, (size_t)rows * d, cudaMemcpyHostToDevice, st));
    } else {
        CU(cudaMemset2DAsync(dst, ld, 0, ld, rows, st));
        CU(cudaMemcpy2DAsync(dst, ld, host, d, d, rows, cudaMemcpyHostToDevice, st));
    }
    return LAL_TAIL_OK;
}

/* Look up (registering or growing on demand) a host LM head covering rows
 * [0, rows_needed).  Called with g_reg_mu held. */
int registry_get(const int8_t *wte_q, const float *scale_w, int rows_needed, int d, int dev,
                 LmHead *out) {
    auto it = g_reg.find(wte_q);
    if (it != g_reg.end() && it->second.device == dev && it->second.d == d &&
        it->second.rows >= rows_needed && it->second.host_scale == scale_w) {
        *out = it->second;
        return LAL_TAIL_OK;
    }
    LmHead h;
    h.device = dev;
    h.d = d;
    h.ld = ld_for(d);
    h.rows = rows_needed;
    h.host_scale = scale_w;
    /* on any failure the new buffers are freed, the old entry stays */
    int rc = LAL_TAIL_OK;
    cudaError_t e = cudaMalloc(&h.W, (size_t)h.rows * h.ld);
    if (e == cudaSuccess) e = cudaMalloc(&h.sw, sizeof(float) * (size_t)h.rows);
    if (e == cudaSuccess) rc = upload_rows(wte_q, h.rows, d, h.ld, h.W, 0);
    if (e == cudaSuccess && rc == LAL_TAIL_OK)
        e = cudaMemcpy(h.sw, scale_w, sizeof(float) * (size_t)h.rows, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && rc == LAL_TAIL_OK) e = cudaDeviceSynchronize();
    if (e != cudaSuccess || rc != LAL_TAIL_OK) {
        if (e != cudaSuccess)
            rc = fail(LAL_TAIL_ERR_CUDA, "LM head registry: %s", cudaGetErrorString(e));
        cudaDeviceSynchronize(); /* no copy into the buffers may be in flight */
        if (h.W) cudaFree(h.W);
        if (h.sw) cudaFree(h.sw);
        (void)cudaGetLastError(); /* reported through rc; leave no stale error behind */
        return rc;
    }
    if (it != g_reg.end()) {
        g_retired.push_back(it->second.W);
        g_retired.push_back(it->second.sw);
    }
    g_reg[wte_q] = h;
    *out = h;
    return LAL_TAIL_OK;
}

/* Launch parameters common to the streaming kernel's modes. */
void base_params(TailParams &p, const DeviceState *ds) {
    memset(&p, 0, sizeof(p));
    p.expf_x = ds->d_expf_x;
    p.expf_y = ds->d_expf_y;
    p.expf_n = ds->expf_n;
    p.expf_bits = ds->d_expf_bits;
    p.expf_off = ds->d_expf_off;
    p.expf_hash = ds->d_expf_hash;
    p.expf_hash_probe = ds->expf_hash_probe;
}

int sample_launch(DropinState *S, DeviceState *ds, float *logits, int V, float temperature,
                  int top_k, float rep_penalty, const int *recent, int n_recent, float u,
                  int variant, bool candidates_only, int *token_out, StreamDiag *diag_out,
                  int *n_cand_out) {
    if (!logits || V < 1) return fail(LAL_TAIL_ERR_ARG, "sample: bad logits/vocab");
    if (n_recent < 0 || (n_recent > 0 && !recent)) return fail(LAL_TAIL_ERR_ARG, "sample: bad recent");
    const bool greedy = temperature <= 0.0f || top_k <= 0;
    int k = greedy ? 1 : (top_k > V ? V : top_k);
    cudaStream_t st = S->stream;
    TailParams p;
    base_params(p, ds);
    p.mode = MODE_SAMPLE;
    p.variant = variant;
    p.rows = V;
    p.row_base = 0;
    p.vocab = V;
    p.d = p.ld = 16;
    p.B = 1;
    p.max_k = k;
    const int grid = plan_launch(p, ds->num_sms, 64);
    if (grid < 1) return fail(LAL_TAIL_ERR_UNSUPPORTED, "sample: shape unsupported (plan %d)", grid);
    CHECK(S->ls.ensure(V));
    CHECK(S->logits.ensure(sizeof(float) * (size_t)V));
    CHECK(S->ls.hist.ensure(sizeof(int) * (size_t)(n_recent + 1)));
    CHECK(S->ls.cand_v.ensure(sizeof(float) * (size_t)V));
    CHECK(S->ls.cand_i.ensure(sizeof(int) * (size_t)V));
    /* param block: temperature, top_k, penalty, u, hist_n */
    struct {
        float t;
        int k;
        float pen;
        float u;
        int hn;
        int head;
    } hp = {temperature, top_k, rep_penalty, u, n_recent, 0};
    CU(cudaMemcpyAsync(S->ls.params.p, &hp, sizeof(hp), cudaMemcpyHostToDevice, st));
    CU(cudaMemcpyAsync(S->logits.p, logits, sizeof(float) * (size_t)V, cudaMemcpyHostToDevice, st));
    if (n_recent > 0)
        CU(cudaMemcpyAsync(S->ls.hist.p, recent, sizeof(int) * (size_t)n_recent,
                           cudaMemcpyHostToDevice, st));
    char *pb = (char *)S->ls.params.p;
    p.logits = (float *)S->logits.p;
    p.temperature = (const float *)(pb + 0);
    p.top_k = (const int *)(pb + 4);
    p.rep_penalty = (const float *)(pb + 8);
    p.u = (const float *)(pb + 12);
    p.hist_n = (int *)(pb + 16);
    p.hist_head = (int *)(pb + 20);
    p.hist_ids = (int *)S->ls.hist.p;
    p.hist_cap = n_recent;
    p.push_history = 0;
    p.tokens = (int *)S->ls.tokens.p;
    p.diag = (StreamDiag *)S->ls.diag.p;
    S->ls.sel.fill(p);
    p.status = (int *)S->ls.status.p;
    p.cand_val_out = (float *)S->ls.cand_v.p;
    p.cand_idx_out = (int *)S->ls.cand_i.p;
    p.cand_out_cap = V;
    p.candidates_only = candidates_only ? 1 : 0;
    p.local_edges = use_local_edges(effective_k(temperature, top_k, V, V), p.rows_per_cta_max);
    CU(launch_tail(p, grid, st));
    int status = 0;
    StreamDiag dg;
    CU(cudaMemcpyAsync(logits, S->logits.p, sizeof(float) * (size_t)V, cudaMemcpyDeviceToHost, st));
    CU(cudaMemcpyAsync(&dg, S->ls.diag.p, sizeof(dg), cudaMemcpyDeviceToHost, st));
    CU(cudaMemcpyAsync(&status, S->ls.status.p, sizeof(int), cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    if (status != 0) {
        CU(cudaMemset(S->ls.status.p, 0, sizeof(int)));
        CHECK(S->ls.sel.reset(st));
        CU(cudaStreamSynchronize(st));
        return fail(status, "sample kernel reported device status %d (%s)", status,
                    status == LAL_TAIL_ERR_TIMEOUT ? "bounded wait expired"
                                                   : "candidate set above the built capacity");
    }
    if (token_out) *token_out = dg.token;
    if (diag_out) *diag_out = dg;
    if (n_cand_out) *n_cand_out = dg.n_cand;
    return LAL_TAIL_OK;
}

}  // namespace

namespace lal {
int set_error(int code, const char *msg) { return fail(code, "%s", msg); }
}  // namespace lal

/* ======================================================================
 * 1. drop-ins and their status-returning forms
 * ====================================================================== */
extern "C" {

const char *lal_tail_last_error(void) { return g_err.c_str(); }

const char *lal_tail_version(void) {
    return "liblal_tail 0.1 (sm_100a; int8 GEMV via cp.async.bulk + dp4a; fused top-k sampler)";
}

int lal_tail_quantize_x_int8(const float *x, int8_t *xq, int n, float *scale_out) {
    if (!x || !xq || n < 1) return fail(LAL_TAIL_ERR_ARG, "quantize_x: bad arguments");
    DropinState *S;
    DeviceState *ds;
    CHECK(dropin(&S, &ds));
    cudaStream_t st = S->stream;
    CHECK(S->x.ensure(4ull * n + 64));
    CHECK(S->xq.ensure((size_t)n + 64));
    CU(cudaMemcpyAsync(S->x.p, x, 4ull * n, cudaMemcpyHostToDevice, st));
    float *d_scale = (float *)((char *)S->x.p + 4ull * n);
    CU(launch_quantize_x((const float *)S->x.p, (int8_t *)S->xq.p, d_scale, n, st));
    float sc = 0.0f;
    CU(cudaMemcpyAsync(xq, S->xq.p, (size_t)n, cudaMemcpyDeviceToHost, st));
    CU(cudaMemcpyAsync(&sc, d_scale, 4, cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    if (scale_out) *scale_out = sc;
    return LAL_TAIL_OK;
}

float lal_quantize_x_int8(const float *x, int8_t *xq, int n) {
    float s = 0.0f;
    if (lal_tail_quantize_x_int8(x, xq, n, &s) != LAL_TAIL_OK) die("lal_quantize_x_int8");
    return s;
}

int lal_tail_compute_abs_xq(const int8_t *xq, uint8_t *ax, int n) {
    if (!xq || !ax || n < 1) return fail(LAL_TAIL_ERR_ARG, "compute_abs_xq: bad arguments");
    DropinState *S;
    DeviceState *ds;
    CHECK(dropin(&S, &ds));
    cudaStream_t st = S->stream;
    CHECK(S->xq.ensure((size_t)n));
    CHECK(S->ax.ensure((size_t)n));
    CU(cudaMemcpyAsync(S->xq.p, xq, (size_t)n, cudaMemcpyHostToDevice, st));
    CU(launch_abs_xq((const int8_t *)S->xq.p, (uint8_t *)S->ax.p, n, st));
    CU(cudaMemcpyAsync(ax, S->ax.p, (size_t)n, cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    return LAL_TAIL_OK;
}

void lal_compute_abs_xq(const int8_t *xq, uint8_t *ax, int n_embd) {
    if (lal_tail_compute_abs_xq(xq, ax, n_embd) != LAL_TAIL_OK) die("lal_compute_abs_xq");
}

int lal_tail_lm_head_register(const int8_t *wte_q, const float *scale_w, int vocab_size,
                              int n_embd) {
    if (!wte_q || !scale_w || vocab_size < 1 || n_embd < 1)
        return fail(LAL_TAIL_ERR_ARG, "lm_head_register: bad arguments");
    int dev;
    CHECK(current_device(&dev));
    DeviceState *ds;
    CHECK(device_state(dev, &ds));
    std::lock_guard<std::mutex> lk(g_reg_mu);
    LmHead h;
    return registry_get(wte_q, scale_w, vocab_size, n_embd, dev, &h);
}

int lal_tail_lm_head_forget(const int8_t *wte_q) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    auto it = g_reg.find(wte_q);
    if (it == g_reg.end()) return LAL_TAIL_OK;
    CU(cudaDeviceSynchronize());
    cudaFree(it->second.W);
    cudaFree(it->second.sw);
    g_reg.erase(it);
    for (void *p : g_retired) cudaFree(p);
    g_retired.clear();
    return LAL_TAIL_OK;
}

}  // extern "C"

namespace {

/* The LM-head range drop-ins.  eight_row selects the 8-row form's column
 * tail behaviour (runtime/lal_q8_kernel.h:562-611): rows in full 8-row groups
 * from v_start sum only the first n_embd & ~31 columns. */
int lm_head_range(float *logits, const int8_t *xq, float scale_x, const int8_t *wte_q,
                  const float *scale_w, int v_start, int v_end, int n_embd, bool eight_row) {
    if (!logits || !xq || !wte_q || !scale_w || n_embd < 1 || v_start < 0)
        return fail(LAL_TAIL_ERR_ARG, "lm_head_int8_range: bad arguments");
    if (v_end <= v_start) return LAL_TAIL_OK;
    DropinState *S;
    DeviceState *ds;
    CHECK(dropin(&S, &ds));
    LmHead h;
    {
        std::lock_guard<std::mutex> lk(g_reg_mu);
        CHECK(registry_get(wte_q, scale_w, v_end, n_embd, S->device, &h));
    }
    cudaStream_t st = S->stream;
    const int rows = v_end - v_start;
    TailParams p;
    base_params(p, ds);
    p.mode = MODE_LMHEAD;
    p.W = h.W + (size_t)v_start * h.ld;
    p.scale_w = h.sw + v_start;
    p.rows = rows;
    p.row_base = v_start;
    p.vocab = v_end;
    p.d = n_embd;
    p.ld = h.ld;
    p.B = 1;
    p.max_k = 1;
    p.trunc_cols = h.ld;
    p.trunc_rows_end = 0;
    if (eight_row && (n_embd & 31) != 0) {
        p.trunc_cols = n_embd & ~31;
        p.trunc_rows_end = rows / 8 * 8;
    }
    const int grid = plan_launch(p, ds->num_sms, 8);
    if (grid < 1) return fail(LAL_TAIL_ERR_UNSUPPORTED, "lm_head: shape unsupported (plan %d)", grid);
    CHECK(S->ls.ensure(1));
    CHECK(S->xq.ensure((size_t)n_embd));
    CHECK(S->logits.ensure(4ull * rows));
    CU(cudaMemcpyAsync(S->xq.p, xq, (size_t)n_embd, cudaMemcpyHostToDevice, st));
    p.xq_in = (const int8_t *)S->xq.p;
    p.scale_x_in = scale_x;
    p.logits = (float *)S->logits.p;
    p.status = (int *)S->ls.status.p;
    CU(launch_tail(p, grid, st));
    int status = 0;
    CU(cudaMemcpyAsync(logits + v_start, S->logits.p, 4ull * rows, cudaMemcpyDeviceToHost, st));
    CU(cudaMemcpyAsync(&status, S->ls.status.p, sizeof(int), cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    if (status != 0) {
        CU(cudaMemset(S->ls.status.p, 0, sizeof(int)));
        return fail(status, "lm_head kernel reported device status %d", status);
    }
    return LAL_TAIL_OK;
}

}  // namespace

extern "C" {

int lal_tail_lm_head_int8_range(float *logits, const int8_t *xq, float scale_x,
                                const int8_t *wte_q, const float *scale_w, int v_start,
                                int v_end, int n_embd) {
    return lm_head_range(logits, xq, scale_x, wte_q, scale_w, v_start, v_end, n_embd, false);
}

void lal_lm_head_int8_range(float *logits, const int8_t *xq, float scale_x,
                            const int8_t *wte_q, const float *scale_w, int v_start, int v_end,
                            int n_embd) {
    if (lal_tail_lm_head_int8_range(logits, xq, scale_x, wte_q, scale_w, v_start, v_end,
                                    n_embd) != LAL_TAIL_OK)
        die("lal_lm_head_int8_range");
}

void lal_lm_head_int8_range_abs(float *logits, const int8_t *xq, const uint8_t *ax,
                                float scale_x, const int8_t *wte_q, const float *scale_w,
                                int v_start, int v_end, int n_embd) {
    (void)ax;
    if (lal_tail_lm_head_int8_range(logits, xq, scale_x, wte_q, scale_w, v_start, v_end,
                                    n_embd) != LAL_TAIL_OK)
        die("lal_lm_head_int8_range_abs");
}

void lal_lm_head_int8_range_abs_8row(float *logits, const int8_t *xq, const uint8_t *ax,
                                     float scale_x, const int8_t *wte_q, const float *scale_w,
                                     int v_start, int v_end, int n_embd) {
    (void)ax;
    if (lm_head_range(logits, xq, scale_x, wte_q, scale_w, v_start, v_end, n_embd, true) !=
        LAL_TAIL_OK)
        die("lal_lm_head_int8_range_abs_8row");
}

int lal_tail_quantize_q8_per_row(const float *W, int8_t *q8_T, float *scale, int in_dim,
                                 int out_dim) {
    if (!W || !q8_T || !scale || in_dim < 1 || out_dim < 0)
        return fail(LAL_TAIL_ERR_ARG, "quantize_q8_per_row: bad arguments");
    DropinState *S;
    DeviceState *ds;
    CHECK(dropin(&S, &ds));
    cudaStream_t st = S->stream;
    /* chunks of ~64 MB of fp32 input */
    const int chunk = std::max(1, (int)((64ull << 20) / (4ull * in_dim)));
    CHECK(S->W.ensure(4ull * chunk * in_dim));
    CHECK(S->q.ensure((size_t)chunk * in_dim));
    CHECK(S->s.ensure(4ull * chunk));
    for (int r0 = 0; r0 < out_dim; r0 += chunk) {
        const int n = std::min(chunk, out_dim - r0);
        CU(cudaMemcpyAsync(S->W.p, W + (size_t)r0 * in_dim, 4ull * n * in_dim,
                           cudaMemcpyHostToDevice, st));
        CU(launch_quantize_rows((const float *)S->W.p, in_dim, (int8_t *)S->q.p, in_dim,
                                (float *)S->s.p, n, st));
        CU(cudaMemcpyAsync(q8_T + (size_t)r0 * in_dim, S->q.p, (size_t)n * in_dim,
                           cudaMemcpyDeviceToHost, st));
        CU(cudaMemcpyAsync(scale + r0, S->s.p, 4ull * n, cudaMemcpyDeviceToHost, st));
        CU(cudaStreamSynchronize(st));
    }
    return LAL_TAIL_OK;
}

void lal_quantize_q8_per_row(const float *W, int8_t *q8_T, float *scale, int in_dim,
                             int out_dim) {
    if (lal_tail_quantize_q8_per_row(W, q8_T, scale, in_dim, out_dim) != LAL_TAIL_OK)
        die("lal_quantize_q8_per_row");
}

int lal_tail_sample_token(float *logits, int vocab_size, float temperature, int top_k,
                          float rep_penalty, const int *recent, int n_recent, float u,
                          int *token_out) {
    DropinState *S;
    DeviceState *ds;
    CHECK(dropin(&S, &ds));
    return sample_launch(S, ds, logits, vocab_size, temperature, top_k, rep_penalty, recent,
                         n_recent, u, VARIANT_LIBRARY, false, token_out, nullptr, nullptr);
}

int lal_sample_token(float *logits, int vocab_size, float temperature, int top_k,
                     float rep_penalty, const int *recent, int n_recent) {
    /* runtime/lal_sampling.h:116 draws once on the non-greedy path; no other
     * rand() call happens inside the function, so drawing first keeps the
     * caller's global sequence identical. */
    float u = 0.0f;
    if (!(temperature <= 0.0f || top_k <= 0)) u = (float)rand() / (float)RAND_MAX;
    int tok = 0;
    if (lal_tail_sample_token(logits, vocab_size, temperature, top_k, rep_penalty, recent,
                              n_recent, u, &tok) != LAL_TAIL_OK)
        die("lal_sample_token");
    return tok;
}

int lal_tail_sample_token_filtered(float *logits, int vocab_size, float temperature,
                                   int top_k, float rep_penalty, const int *recent,
                                   int n_recent, lal_filter_topk_fn filter,
                                   lal_token_decode_fn decode, lal_draw_fn draw,
                                   void *draw_ctx, int *token_out) {
    DropinState *S;
    DeviceState *ds;
    CHECK(dropin(&S, &ds));
    const bool greedy = temperature <= 0.0f || top_k <= 0;
    if (greedy) /* penalty then argmax (qwen7b_server.c:223-234) */
        return sample_launch(S, ds, logits, vocab_size, temperature, top_k, rep_penalty, recent,
                             n_recent, 0.0f, VARIANT_SERVER, false, token_out, nullptr, nullptr);
    /* 1. penalty, threshold and the candidate set on the device */
    StreamDiag dg;
    int m = 0;
    CHECK(sample_launch(S, ds, logits, vocab_size, temperature, top_k, rep_penalty, recent,
                        n_recent, 0.0f, VARIANT_SERVER, true, nullptr, &dg, &m));
    cudaStream_t st = S->stream;
    std::vector<int> cand(m);
    CU(cudaMemcpyAsync(cand.data(), S->ls.cand_i.p, sizeof(int) * (size_t)m,
                       cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    /* 2. keep_mask and the level-2 filter on the host (qwen7b_server.c:258-270) */
    std::vector<int> keep_c(m, 1);
    if (filter) {
        std::vector<int> mask((size_t)vocab_size, 0);
        for (int i = 0; i < m; ++i) mask[cand[i]] = 1;
        const int last = n_recent > 0 ? recent[n_recent - 1] : -1;
        (void)filter(mask.data(), vocab_size, last, recent, n_recent, decode);
        bool any = false;
        for (int v = 0; v < vocab_size && !any; ++v) any = mask[v] != 0;
        if (any) {
            /* a filter only clears bits; kept non-candidates never count
             * because the reference also requires logits[v] >= threshold */
            for (int i = 0; i < m; ++i) keep_c[i] = mask[cand[i]] ? 1 : 0;
        }
    }
    /* 3. kept softmax on the device; draw only when the mass is positive */
    CHECK(S->ls.keep.ensure(sizeof(int) * (size_t)(m + 1)));
    CHECK(S->ls.prefix.ensure(sizeof(float) * (size_t)(m + 1)));
    CHECK(S->ls.u.ensure(64));
    CU(cudaMemcpyAsync(S->ls.keep.p, keep_c.data(), sizeof(int) * (size_t)m,
                       cudaMemcpyHostToDevice, st));
    FinishParams f;
    memset(&f, 0, sizeof(f));
    f.cand_val = (const float *)S->ls.cand_v.p;
    f.cand_idx = (const int *)S->ls.cand_i.p;
    f.keep = (const int *)S->ls.keep.p;
    f.m = m;
    f.temperature = temperature;
    f.vocab = vocab_size;
    f.u = (const float *)S->ls.u.p;
    f.prefix = (float *)S->ls.prefix.p;
    f.diag = (StreamDiag *)S->ls.diag.p;
    f.token = (int *)S->ls.tokens.p;
    f.expf_x = ds->d_expf_x;
    f.expf_y = ds->d_expf_y;
    f.expf_n = ds->expf_n;
    f.expf_bits = ds->d_expf_bits;
    f.expf_off = ds->d_expf_off;
    f.phase = 0;
    CU(launch_finish(f, st));
    CU(cudaMemcpyAsync(&dg, S->ls.diag.p, sizeof(dg), cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    if (dg.sum <= 0.0f) { /* qwen7b_server.c:285-286 */
        if (token_out) *token_out = dg.token;
        return LAL_TAIL_OK;
    }
    const float u = draw ? draw(draw_ctx) : 0.0f;
    CU(cudaMemcpyAsync(S->ls.u.p, &u, sizeof(float), cudaMemcpyHostToDevice, st));
    f.phase = 1;
    CU(launch_finish(f, st));
    int tok = -1;
    CU(cudaMemcpyAsync(&tok, S->ls.tokens.p, sizeof(int), cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    if (token_out) *token_out = tok;
    return LAL_TAIL_OK;
}

void lal_recent_push(LalRecentTokens *rt, int tok) {
    /* runtime/lal_sampling.h:133-136 */
    if (rt->n < 256) {
        rt->tokens[rt->n++] = tok;
    } else {
        memmove(rt->tokens, rt->tokens + 1, 255 * sizeof(int));
        rt->tokens[255] = tok;
    }
}

int lal_tail_debug_expf(const float *x, float *y, int n) {
    if (!x || !y || n < 0) return fail(LAL_TAIL_ERR_ARG, "debug_expf: bad arguments");
    if (n == 0) return LAL_TAIL_OK;
    DropinState *S;
    DeviceState *ds;
    CHECK(dropin(&S, &ds));
    cudaStream_t st = S->stream;
    CHECK(S->x.ensure(4ull * n));
    CHECK(S->logits.ensure(4ull * n));
    CU(cudaMemcpyAsync(S->x.p, x, 4ull * n, cudaMemcpyHostToDevice, st));
    CU(launch_debug_expf((const float *)S->x.p, (float *)S->logits.p, n, ds->d_expf_x,
                         ds->d_expf_y, ds->expf_n, ds->d_expf_bits, ds->d_expf_off,
                         ds->d_expf_hash, ds->expf_hash_probe, st));
    CU(cudaMemcpyAsync(y, S->logits.p, 4ull * n, cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    return LAL_TAIL_OK;
}

}  // extern "C"

/* ======================================================================
 * 2. fused decode-tail contexts
 * ====================================================================== */
struct lal_tail {
    lal_tail_config cfg;
    int device = 0;
    DeviceState *ds = nullptr;
    int row0 = 0, nrows = 0, ld = 0;
    cudaStream_t stream = nullptr;
    bool loaded = false;
    int8_t *W = nullptr;
    float *sw = nullptr;
    /* inputs: hidden [B][d] followed by u [B] (one H2D per step) */
    float *io_in = nullptr;
    /* outputs: tokens [B] followed by the status word (one D2H per step) */
    int *io_out = nullptr;
    float *logits = nullptr;                   /* [B][nrows] */
    float *temp = nullptr;                     /* [B] */
    int *topk = nullptr;                       /* [B] */
    float *pen = nullptr;                      /* [B] */
    int *hist_ids = nullptr, *hist_n = nullptr, *hist_head = nullptr;
    StreamDiag *diag = nullptr;                /* [B] */
    SelectScratch sel;                         /* shared by the streams' launches */
    float *h_in = nullptr;                     /* pinned staging (mapped) */
    float *d_h_in = nullptr;                   /* its device address */
    int *h_out = nullptr;
    /* per-stream completion words of lal_tail_step (mapped pinned): the
     * kernel that draws a stream's token stores [step number | token] */
    unsigned long long *h_tok = nullptr, *d_h_tok = nullptr;
    unsigned host_seq = 0;
    std::vector<float> h_temp;
    std::vector<int> h_topk;
    std::vector<float> h_pen;
    int n_set = 0;
    TailParams plan;
    int grid = 0;
    bool timing = false;
    std::vector<cudaEvent_t> ev;
    int ev_used = 0;
    unsigned long long *phase_ts = nullptr;    /* [(kMaxGrid+1)*8] when on */
    bool phases = false;
    /* vocab-sharded step: this rank's records [max_streams][rec_bytes] and
     * the gathered records of all ranks [shard_count][n][rec_bytes] */
    int rec_cap = 0, rec_bytes = 0, merge_cap = 0;
    uint8_t *x_send = nullptr, *x_recv = nullptr;
    /* batched step (B >= 2): quantized vectors, scales, cached descriptors */
    bool batch_ok = false;
    int8_t *xq_b = nullptr;
    float *sx_b = nullptr;
    uint32_t *gmax_b = nullptr;
    int *ksplit_b = nullptr; /* the GEMM's split tiles' partial dots */
    size_t ksplit_bytes = 0;
    BatchPlan bplan;
    /* peer exchange of the sharded step: this rank's receive buffer
     * [2][shard_count][rec_bytes] (exported by IPC handle), the device array
     * of every rank's buffer, the peers' opened mappings, the step counter */
    uint8_t *x_peer = nullptr;
    uint8_t **d_peer = nullptr;
    int peer_rec_bytes = 0; /* peer_record_bytes(rec_cap, largest slice) */
    std::vector<void *> peer_open;
    bool p2p = false;
    unsigned seq = 1;
    /* level-2 filter hook (qwen7b_server.c:257-270) for the host-buffer step:
     * device candidate list, keep flags, prefix scratch, draw and token words;
     * host keep mask and copies */
    lal_filter_topk_fn filter = nullptr;
    lal_token_decode_fn decode = nullptr;
    lal_draw_fn draw = nullptr;
    void *draw_ctx = nullptr;
    bool filtered = false;
    float *f_cand_v = nullptr, *f_prefix = nullptr, *f_u = nullptr;
    int *f_cand_i = nullptr, *f_keep = nullptr, *f_tok = nullptr;
    StreamDiag *f_diag = nullptr;
    std::vector<int> f_mask, f_ids, f_ring, f_keep_h;
    /* the final RMSNorm's weights on the device (lal_tail_set_final_norm) */
    float *d_norm_w = nullptr;
    /* lal_tail_set_lm_head_copies: extra device copies of the slice and its
     * scales, used in turn by the per-stream steps */
    std::vector<int8_t *> w_copies;
    std::vector<float *> sw_copies;
    unsigned rot = 0;
    /* LAL_SAMPLER_GPT2: the launch plans of the LM head and the sampler; the
     * quantized vector and its scale, the re-scored rows and their count */
    TailParams g2_lm;
    int g2_grid_lm = 0, g2_n = 0, g2_h_slots = 0;
    float g2_top_p = 0.0f;
    int *g2_cand_i = nullptr, *g2_count = nullptr;
    uint32_t *g2_bound = nullptr;
    float *g2_kept_v = nullptr;
    unsigned *g2_ticket = nullptr;
};

namespace {

void close_peers(lal_tail *t) {
    for (void *q : t->peer_open)
        if (q) cudaIpcCloseMemHandle(q);
    t->peer_open.clear();
    t->p2p = false;
}

void free_copies(lal_tail *t) {
    for (int8_t *w : t->w_copies) cudaFree(w);
    for (float *f : t->sw_copies) cudaFree(f);
    t->w_copies.clear();
    t->sw_copies.clear();
    t->rot = 0;
}

void destroy_ctx(lal_tail *t) {
    if (!t) return;
    if (t->device >= 0) cudaSetDevice(t->device);
    if (t->stream) cudaStreamSynchronize(t->stream);
    close_peers(t);
    free_copies(t);
    void *bufs[] = {t->W, t->sw, t->io_in, t->io_out, t->logits, t->temp, t->topk, t->pen,
                    t->hist_ids, t->hist_n, t->hist_head, t->diag, t->phase_ts,
                    t->x_send, t->x_recv, t->xq_b, t->sx_b, t->gmax_b, t->ksplit_b, t->x_peer, t->d_peer,
                    t->f_cand_v, t->f_prefix, t->f_u, t->f_cand_i, t->f_keep, t->f_tok,
                    t->f_diag, t->d_norm_w, t->g2_cand_i, t->g2_count,
                    t->g2_bound, t->g2_ticket, t->g2_kept_v};
    for (void *b : bufs)
        if (b) cudaFree(b);
    t->sel.free_all();
    if (t->h_in) cudaFreeHost(t->h_in);
    if (t->h_out) cudaFreeHost(t->h_out);
    if (t->h_tok) cudaFreeHost(t->h_tok);
    for (cudaEvent_t e : t->ev) cudaEventDestroy(e);
    if (t->stream) cudaStreamDestroy(t->stream);
    delete t;
}

/* LAL_SAMPLER_GPT2 contexts (one shard): the plans and buffers of the five
 * launches of a step (tail_gpt2.cu) */
int gpt2_alloc(lal_tail *t) {
    const lal_tail_config &c = t->cfg;
    const int V = c.vocab_size, num_sms = t->ds->num_sms;
    if (V > kGpt2MaxV)
        return fail(LAL_TAIL_ERR_UNSUPPORTED,
                    "gpt2 tail: vocab %d above %d (its select holds the vocab's logits in one "
                    "CTA's shared memory)", V, kGpt2MaxV);
    t->g2_n = std::min(kGpt2RerankN, V);
    TailParams &lm = t->g2_lm;
    base_params(lm, t->ds);
    lm.mode = MODE_LMHEAD;
    lm.rows = t->nrows;
    lm.row_base = 0;
    lm.vocab = V;
    lm.d = c.n_embd;
    lm.ld = t->ld;
    lm.B = 1;
    lm.max_k = 1;
    lm.trunc_cols = t->ld;
    lm.trunc_rows_end = 0;
    t->g2_grid_lm = plan_launch(lm, num_sms, 8);
    if (t->g2_grid_lm < 1)
        return fail(LAL_TAIL_ERR_UNSUPPORTED, "gpt2 tail: shape V=%d d=%d unsupported", V,
                    c.n_embd);
    /* the sampler's history hash: a power of two >= twice the history */
    int hs = 64;
    while (hs < 2 * std::max(1, c.history_cap)) hs <<= 1;
    t->g2_h_slots = hs;
    if (gpt2_finish_smem(std::max(1, std::min(c.max_top_k, V)), hs) > (size_t)200 * 1024)
        return fail(LAL_TAIL_ERR_UNSUPPORTED,
                    "gpt2 tail: history_cap %d / max_top_k %d beyond the sampler's shared memory",
                    c.history_cap, c.max_top_k);
    CU(cudaMalloc(&t->g2_cand_i, sizeof(int) * (size_t)kGpt2RerankN));
    CU(cudaMalloc(&t->g2_count, sizeof(int)));
    CU(cudaMalloc(&t->g2_bound, sizeof(uint32_t)));
    CU(cudaMalloc(&t->g2_kept_v, sizeof(float) * (size_t)kGpt2RerankN));
    CU(cudaMalloc(&t->g2_ticket, sizeof(unsigned)));
    CU(cudaMemset(t->g2_ticket, 0, sizeof(unsigned)));
    return LAL_TAIL_OK;
}

/* One stream of a LAL_SAMPLER_GPT2 step (tail_gpt2.cu has the sequence). */
int enqueue_gpt2(lal_tail *t, int b, const float *d_hidden, const float *d_u, int *d_tokens,
                 bool candidates_only = false) {
    const int d = t->cfg.n_embd, V = t->cfg.vocab_size;
    const int hc = std::max(1, t->cfg.history_cap);
    cudaStream_t st = t->stream;
    const float *x = d_hidden + (size_t)b * d;
    float *logits = t->logits + (size_t)b * t->nrows;
    int *status = t->io_out + t->cfg.max_streams;
    /* the LM head (its launch quantizes x: gpt2_server.c:1982-1998) */
    TailParams lm = t->g2_lm;
    lm.W = t->W;
    lm.scale_w = t->sw;
    lm.hidden = x;
    lm.logits = logits;
    lm.status = status;
    const bool time_it = t->timing && t->ev_used + 2 <= (int)t->ev.size();
    if (time_it) CU(cudaEventRecord(t->ev[t->ev_used], st));
    CU(launch_tail(lm, t->g2_grid_lm, st));
    if (time_it) {
        CU(cudaEventRecord(t->ev[t->ev_used + 1], st));
        t->ev_used += 2;
    }
    /* the rows the server's heap keeps, then their float re-score and the
     * server's sampler (the re-score launch's last CTA) */
    CU(launch_gpt2_select(logits, V, t->g2_n, t->g2_cand_i, t->g2_count, t->g2_bound, status,
                          st));
    Gpt2Finish f;
    memset(&f, 0, sizeof(f));
    f.logits = logits;
    f.V = V;
    f.cand = t->g2_cand_i;
    f.kept_val = t->g2_kept_v;
    f.n_ptr = t->g2_count;
    f.bound = t->g2_bound;
    f.temperature = t->temp + b;
    f.rep_penalty = t->pen + b;
    f.u = d_u + b;
    f.top_k = t->topk + b;
    f.top_p = t->g2_top_p;
    f.hist_ids = t->hist_ids + (size_t)b * hc;
    f.hist_n = t->hist_n + b;
    f.hist_head = t->hist_head + b;
    f.hist_cap = t->cfg.history_cap;
    f.push_history = t->cfg.history_cap > 0 ? 1 : 0;
    f.tokens = d_tokens + b;
    f.diag = t->diag + b;
    f.expf_x = t->ds->d_expf_x;
    f.expf_y = t->ds->d_expf_y;
    f.expf_bits = t->ds->d_expf_bits;
    f.expf_off = t->ds->d_expf_off;
    f.expf_hash = t->ds->d_expf_hash;
    f.expf_hash_probe = t->ds->expf_hash_probe;
    f.cap = std::max(1, std::min(t->cfg.max_top_k, V));
    f.h_slots = t->g2_h_slots;
    f.ticket = t->g2_ticket;
    f.status = status;
    if (candidates_only) {
        f.candidates_only = 1;
        f.pool_val = t->f_cand_v;
        f.pool_idx = t->f_cand_i;
        f.pool_keep = t->f_keep;
        f.pool_cap = t->nrows;
        f.push_history = 0;
    }
    CU(launch_gpt2_rerank(x, d, t->W, t->ld, t->sw, f, t->g2_n, st));
    return LAL_TAIL_OK;
}

int ctx_alloc(lal_tail *t) {
    const lal_tail_config &c = t->cfg;
    const int B = c.max_streams, d = c.n_embd;
    CU(cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking));
    CU(cudaMalloc(&t->W, (size_t)t->nrows * t->ld));
    CU(cudaMemset(t->W, 0, (size_t)t->nrows * t->ld));
    CU(cudaMalloc(&t->sw, 4ull * t->nrows));
    /* [B][d] hidden, [B] draws, the step number */
    CU(cudaMalloc(&t->io_in, 4ull * ((size_t)B * d + B + 1)));
    CU(cudaMalloc(&t->io_out, 4ull * (B + 1)));
    CU(cudaMemset(t->io_out, 0, 4ull * (B + 1)));
    CU(cudaMalloc(&t->logits, 4ull * B * t->nrows));
    CU(cudaMalloc(&t->temp, 4ull * B));
    CU(cudaMalloc(&t->topk, 4ull * B));
    CU(cudaMalloc(&t->pen, 4ull * B));
    const int hc = std::max(1, c.history_cap);
    CU(cudaMalloc(&t->hist_ids, 4ull * B * hc));
    CU(cudaMalloc(&t->hist_n, 4ull * B));
    CU(cudaMalloc(&t->hist_head, 4ull * B));
    CU(cudaMemset(t->hist_n, 0, 4ull * B));
    CU(cudaMemset(t->hist_head, 0, 4ull * B));
    CU(cudaMalloc(&t->diag, sizeof(StreamDiag) * B));
    CU(cudaMemset(t->diag, 0, sizeof(StreamDiag) * B));
    CHECK(t->sel.alloc(t->nrows));
    CU(cudaHostAlloc(&t->h_in, 4ull * ((size_t)B * d + B + 1), cudaHostAllocMapped));
    CU(cudaHostGetDevicePointer((void **)&t->d_h_in, t->h_in, 0));
    CU(cudaMallocHost(&t->h_out, 4ull * (B + 1)));
    CU(cudaHostAlloc(&t->h_tok, 8ull * B, cudaHostAllocMapped));
    memset(t->h_tok, 0, 8ull * B);
    CU(cudaHostGetDevicePointer((void **)&t->d_h_tok, t->h_tok, 0));
    t->h_temp.assign(B, 0.0f);
    t->h_topk.assign(B, 0);
    t->h_pen.assign(B, 1.0f);
    /* plan the fused launch for this slice */
    TailParams &p = t->plan;
    base_params(p, t->ds);
    p.mode = MODE_FUSED;
    p.variant = c.sampler == LAL_SAMPLER_SERVER ? VARIANT_SERVER
                : c.sampler == LAL_SAMPLER_GPT2 ? VARIANT_GPT2
                                                : VARIANT_LIBRARY;
    p.rows = t->nrows;
    p.row_base = t->row0;
    p.vocab = c.vocab_size;
    p.d = d;
    p.ld = t->ld;
    p.B = 1;
    p.max_k = std::min(c.max_top_k, t->nrows);
    t->grid = plan_launch(p, t->ds->num_sms, 8);
    if (t->grid < 1)
        return fail(LAL_TAIL_ERR_UNSUPPORTED, "fused tail: shape V=%d d=%d k=%d unsupported (plan %d)",
                    c.vocab_size, d, c.max_top_k, t->grid);
    /* candidate records of the sharded step: a slice exports its
     * tie-complete set, k entries plus room for ties at its threshold, or in
     * the wide form its rows above its threshold and a bitmap of its ties */
    const int want = (std::min(c.max_top_k, c.vocab_size) + 64 + 3) / 4 * 4;
    t->rec_cap = std::min(want, (t->nrows + 3) / 4 * 4);
    const int rows_max = shard_rows_max(c.vocab_size, c.shard_count);
    t->rec_bytes = shard_record_bytes(t->rec_cap, rows_max);
    t->merge_cap = merge_smem_cap(c.shard_count * t->rec_cap);
    if (t->merge_cap < 1)
        return fail(LAL_TAIL_ERR_UNSUPPORTED,
                    "sharded merge: %d shards x %d candidates exceed shared memory",
                    c.shard_count, t->rec_cap);
    CU(cudaMalloc(&t->x_send, (size_t)B * t->rec_bytes));
    CU(cudaMemset(t->x_send, 0, (size_t)B * t->rec_bytes));
    CU(cudaMalloc(&t->x_recv, (size_t)c.shard_count * B * t->rec_bytes));
    CU(cudaMemset(t->x_recv, 0, (size_t)c.shard_count * B * t->rec_bytes));
    if (c.shard_count > 1) {
        t->peer_rec_bytes = peer_record_bytes(t->rec_cap, rows_max);
        const size_t pb = 2ull * c.shard_count * t->peer_rec_bytes;
        CU(cudaMalloc(&t->x_peer, pb));
        CU(cudaMemset(t->x_peer, 0, pb));
        CU(cudaMalloc(&t->d_peer, sizeof(uint8_t *) * c.shard_count));
    }
    if (c.sampler == LAL_SAMPLER_GPT2) return gpt2_alloc(t);
    /* batched step: one pass over W for all streams on the tensor cores */
    if (B >= 2 && B <= 256) {
        CU(cudaMalloc(&t->xq_b, (size_t)256 * t->ld));
        CU(cudaMemset(t->xq_b, 0, (size_t)256 * t->ld));
        CU(cudaMalloc(&t->sx_b, 4ull * 256));
        CU(cudaMalloc(&t->gmax_b, 4ull * 256 * batch_groups(t->nrows)));
        t->ksplit_bytes = batch_split_bytes(t->nrows, t->ld, t->ds->num_sms, B);
        if (t->ksplit_bytes) CU(cudaMalloc(&t->ksplit_b, t->ksplit_bytes));
        t->batch_ok = batch_plan(t->bplan, t->W, t->sw, t->nrows, t->ld, t->ds->num_sms, t->xq_b,
                                 t->sx_b, t->gmax_b, t->ksplit_b, B, c.history_cap,
                                 std::min(c.max_top_k, c.vocab_size)) == 0;
    }
    return LAL_TAIL_OK;
}

int ctx_check(lal_tail *t) {
    if (!t) return fail(LAL_TAIL_ERR_ARG, "null context");
    CU(cudaSetDevice(t->device));
    return LAL_TAIL_OK;
}

/* Enqueue the fused kernel for streams [0, n) on the context stream; with
 * shard_export, each launch writes stream b's candidate record into x_send
 * instead of sampling (d_u and d_tokens unused). */
int enqueue_step(lal_tail *t, const float *d_hidden, int n, const float *d_u, int *d_tokens,
                 bool shard_export = false, bool notify = false) {
    const unsigned *seq_in =
        reinterpret_cast<const unsigned *>(t->io_in + (size_t)t->cfg.max_streams * t->cfg.n_embd +
                                           t->cfg.max_streams);
    if (!t->loaded) return fail(LAL_TAIL_ERR_STATE, "step before the LM head was loaded");
    if (n < 1 || n > t->cfg.max_streams) return fail(LAL_TAIL_ERR_ARG, "n_streams %d out of range", n);
    if (t->n_set < n) return fail(LAL_TAIL_ERR_STATE, "sampling parameters not set for %d streams", n);
    const bool peer = !shard_export && t->cfg.shard_count > 1 && t->p2p && n == 1;
    if (!shard_export && t->cfg.shard_count > 1 && !peer)
        return fail(LAL_TAIL_ERR_STATE,
                    "vocab-sharded context: step one stream after lal_tail_connect_peers, or "
                    "use lal_tail_shard_select, an all-gather of the records and "
                    "lal_tail_shard_merge");
    const int hc = std::max(1, t->cfg.history_cap);
    if (t->cfg.sampler == LAL_SAMPLER_GPT2) {
        if (shard_export)
            return fail(LAL_TAIL_ERR_UNSUPPORTED, "the GPT-2 sampler has no sharded step");
        for (int b = 0; b < n; ++b) CHECK(enqueue_gpt2(t, b, d_hidden, d_u, d_tokens));
        return LAL_TAIL_OK;
    }
    if (t->batch_ok && n >= 2 && !getenv_flag("LAL_TAIL_PER_STREAM")) {
        BatchStep bs;
        memset(&bs, 0, sizeof(bs));
        bs.hidden = d_hidden;
        bs.norm_w = t->plan.norm_w;
        bs.norm_eps = t->plan.norm_eps;
        bs.d = t->cfg.n_embd;
        bs.B = n;
        bs.logits = t->logits;
        bs.row_base = t->row0;
        bs.vocab = t->cfg.vocab_size;
        bs.variant = t->plan.variant;
        bs.temperature = t->temp;
        bs.top_k = t->topk;
        bs.rep_penalty = t->pen;
        bs.u = shard_export ? nullptr : d_u;
        bs.hist_ids = t->hist_ids;
        bs.hist_n = t->hist_n;
        bs.hist_head = t->hist_head;
        bs.hist_cap = t->cfg.history_cap;
        bs.hist_stride = hc;
        bs.push_history = shard_export ? 0 : (t->cfg.history_cap > 0 ? 1 : 0);
        bs.tokens = d_tokens;
        bs.diag = t->diag;
        bs.status = t->io_out + t->cfg.max_streams;
        bs.expf_x = t->ds->d_expf_x;
        bs.expf_y = t->ds->d_expf_y;
        bs.expf_n = t->ds->expf_n;
        bs.expf_bits = t->ds->d_expf_bits;
        bs.expf_off = t->ds->d_expf_off;
        if (shard_export) {
            bs.shard_out = t->x_send;
            bs.rec_cap = t->rec_cap;
            bs.rec_bytes = t->rec_bytes;
        }
        if (notify) {
            bs.host_tok = t->d_h_tok;
            bs.seq_in = seq_in;
        }
        /* timing covers the GEMM launch (the step's dominant kernel) */
        const bool time_it = t->timing && t->ev_used + 2 <= (int)t->ev.size();
        if (time_it) {
            bs.gemm_ev0 = t->ev[t->ev_used];
            bs.gemm_ev1 = t->ev[t->ev_used + 1];
        }
        CU(batch_launch(t->bplan, bs, t->stream));
        if (time_it) t->ev_used += 2;
        return LAL_TAIL_OK;
    }
    /* the LM head copy of this step (lal_tail_set_lm_head_copies) */
    const int8_t *W = t->W;
    const float *sw = t->sw;
    if (!t->w_copies.empty()) {
        const unsigned c = t->rot++ % (unsigned)(t->w_copies.size() + 1);
        if (c > 0) {
            W = t->w_copies[c - 1];
            sw = t->sw_copies[c - 1];
        }
    }
    for (int b = 0; b < n; ++b) {
        TailParams p = t->plan;
        p.W = W;
        p.scale_w = sw;
        p.hidden = d_hidden + (size_t)b * t->cfg.n_embd;
        p.logits = t->logits + (size_t)b * t->nrows;
        p.temperature = t->temp + b;
        p.top_k = t->topk + b;
        p.rep_penalty = t->pen + b;
        p.u = d_u + b;
        p.hist_ids = t->hist_ids + (size_t)b * hc;
        p.hist_n = t->hist_n + b;
        p.hist_head = t->hist_head + b;
        p.hist_cap = t->cfg.history_cap;
        p.push_history = t->cfg.history_cap > 0 ? 1 : 0;
        p.tokens = shard_export ? nullptr : d_tokens + b;
        p.u = shard_export ? t->temp + b : d_u + b; /* read, unused */
        p.diag = t->diag + b;
        if (shard_export) {
            p.shard_out = t->x_send + (size_t)b * t->rec_bytes;
            p.rec_cap = t->rec_cap;
        }
        if (peer) {
            p.peer_recv = t->d_peer;
            p.n_ranks = t->cfg.shard_count;
            p.rank = t->cfg.shard_rank;
            p.rec_bytes = t->peer_rec_bytes;
            p.rec_cap = t->rec_cap;
            p.seq = t->seq++;
            if (t->seq == 0) t->seq = 1; /* 0 never matches: buffers start zeroed */
        }
        t->sel.fill(p);
        p.status = t->io_out + t->cfg.max_streams;
        p.phase_ts = t->phases ? t->phase_ts : nullptr;
        if (notify) {
            p.host_tok = t->d_h_tok + b;
            p.seq_in = seq_in;
        }
        p.local_edges = use_local_edges(
            effective_k(t->h_temp[b], t->h_topk[b], t->cfg.vocab_size, t->nrows), p.rows_per_cta_max);
        const bool time_it = t->timing && t->ev_used + 2 <= (int)t->ev.size();
        if (time_it) CU(cudaEventRecord(t->ev[t->ev_used], t->stream));
        CU(launch_tail(p, t->grid, t->stream));
        if (time_it) {
            CU(cudaEventRecord(t->ev[t->ev_used + 1], t->stream));
            t->ev_used += 2;
        }
    }
    return LAL_TAIL_OK;
}

/* The normal fused launch of stream b alone (hidden and u in io_in, the
 * token into io_out). */
int enqueue_one(lal_tail *t, int b) {
    const int B = t->cfg.max_streams, d = t->cfg.n_embd;
    const int hc = std::max(1, t->cfg.history_cap);
    TailParams p = t->plan;
    p.W = t->W;
    p.scale_w = t->sw;
    p.hidden = t->io_in + (size_t)b * d;
    p.logits = t->logits + (size_t)b * t->nrows;
    p.temperature = t->temp + b;
    p.top_k = t->topk + b;
    p.rep_penalty = t->pen + b;
    p.u = t->io_in + (size_t)B * d + b;
    p.hist_ids = t->hist_ids + (size_t)b * hc;
    p.hist_n = t->hist_n + b;
    p.hist_head = t->hist_head + b;
    p.hist_cap = t->cfg.history_cap;
    p.push_history = t->cfg.history_cap > 0 ? 1 : 0;
    p.tokens = t->io_out + b;
    p.diag = t->diag + b;
    t->sel.fill(p);
    p.status = t->io_out + B;
    p.local_edges = use_local_edges(
        effective_k(t->h_temp[b], t->h_topk[b], t->cfg.vocab_size, t->nrows), p.rows_per_cta_max);
    CU(launch_tail(p, t->grid, t->stream));
    return LAL_TAIL_OK;
}

/* One stream's step with the level-2 filter hook: the server's sampler
 * (tools/server/qwen7b_server.c:219-295) with the candidate set handed to the
 * host between the select and the draw.  hidden is already on the device;
 * u_fallback is the draw used when no draw callback is set. */
int filtered_stream_step(lal_tail *t, int b, const float *d_hidden, float u_fallback,
                         int *token_out) {
    const int hc = std::max(1, t->cfg.history_cap);
    const int V = t->cfg.vocab_size;
    TailParams p = t->plan;
    p.W = t->W;
    p.scale_w = t->sw;
    p.hidden = d_hidden + (size_t)b * t->cfg.n_embd;
    p.logits = t->logits + (size_t)b * t->nrows;
    p.temperature = t->temp + b;
    p.top_k = t->topk + b;
    p.rep_penalty = t->pen + b;
    p.u = t->f_u;
    p.hist_ids = t->hist_ids + (size_t)b * hc;
    p.hist_n = t->hist_n + b;
    p.hist_head = t->hist_head + b;
    p.hist_cap = t->cfg.history_cap;
    p.push_history = 0;
    p.tokens = t->f_tok;
    p.diag = t->diag + b;
    p.candidates_only = 1;
    p.cand_val_out = t->f_cand_v;
    p.cand_idx_out = t->f_cand_i;
    p.cand_out_cap = t->nrows;
    t->sel.fill(p);
    p.status = t->io_out + t->cfg.max_streams;
    p.local_edges = use_local_edges(
        effective_k(t->h_temp[b], t->h_topk[b], V, t->nrows), p.rows_per_cta_max);
    CU(launch_tail(p, t->grid, t->stream));
    /* 1. the candidate count, the status and the history ring */
    StreamDiag dg;
    int status = 0, n = 0, head = 0;
    CU(cudaMemcpyAsync(&dg, t->diag + b, sizeof(dg), cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(&status, p.status, 4, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(&n, t->hist_n + b, 4, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(&head, t->hist_head + b, 4, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    if (status != 0) {
        CU(cudaMemset(p.status, 0, 4));
        CHECK(t->sel.reset(t->stream));
        CU(cudaStreamSynchronize(t->stream));
        return fail(status, "device status %d in the filtered step", status);
    }
    const int m = dg.n_cand;
    if (m < 1 || m > t->nrows) return fail(LAL_TAIL_ERR_CAPACITY, "filtered step: %d candidates", m);
    CU(cudaMemcpyAsync(t->f_ids.data(), t->f_cand_i, 4ull * m, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(t->f_ring.data(), p.hist_ids, 4ull * hc, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    /* the recent tokens, oldest first, as the server keeps them */
    std::vector<int> recent((size_t)n);
    for (int i = 0; i < n; ++i)
        recent[i] = t->f_ring[(size_t)((n < hc ? 0 : head) + i) % (size_t)hc];
    /* 2. keep mask, filter, restore when emptied (qwen7b_server.c:258-270) */
    std::vector<int> &keep = t->f_keep_h;
    keep.assign((size_t)m, 1);
    if (t->filter) {
        std::fill(t->f_mask.begin(), t->f_mask.end(), 0);
        for (int i = 0; i < m; ++i) t->f_mask[t->f_ids[i]] = 1;
        const int last = n > 0 ? recent[n - 1] : -1;
        (void)t->filter(t->f_mask.data(), V, last, recent.data(), n, t->decode);
        bool any = false;
        for (int v = 0; v < V && !any; ++v) any = t->f_mask[v] != 0;
        if (any)
            for (int i = 0; i < m; ++i) keep[i] = t->f_mask[t->f_ids[i]] ? 1 : 0;
    }
    /* 3. kept softmax on the device; the draw only when the mass is positive */
    CU(cudaMemcpyAsync(t->f_keep, keep.data(), 4ull * m, cudaMemcpyHostToDevice, t->stream));
    FinishParams f;
    memset(&f, 0, sizeof(f));
    f.cand_val = t->f_cand_v;
    f.cand_idx = t->f_cand_i;
    f.keep = t->f_keep;
    f.m = m;
    f.temperature = t->h_temp[b];
    f.vocab = V;
    f.u = t->f_u;
    f.prefix = t->f_prefix;
    f.diag = t->f_diag;
    f.token = t->f_tok;
    f.expf_x = t->ds->d_expf_x;
    f.expf_y = t->ds->d_expf_y;
    f.expf_n = t->ds->expf_n;
    f.expf_bits = t->ds->d_expf_bits;
    f.expf_off = t->ds->d_expf_off;
    f.phase = 0;
    CU(launch_finish(f, t->stream));
    StreamDiag fd;
    CU(cudaMemcpyAsync(&fd, t->f_diag, sizeof(fd), cudaMemcpyDeviceToHost, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    int tok = fd.token;
    if (fd.sum > 0.0f) { /* qwen7b_server.c:285-290 */
        const float u = t->draw ? t->draw(t->draw_ctx) : u_fallback;
        CU(cudaMemcpyAsync(t->f_u, &u, 4, cudaMemcpyHostToDevice, t->stream));
        f.phase = 1;
        CU(launch_finish(f, t->stream));
        CU(cudaMemcpyAsync(&tok, t->f_tok, 4, cudaMemcpyDeviceToHost, t->stream));
        CU(cudaStreamSynchronize(t->stream));
    }
    /* 4. the history push (FIFO at history_cap) */
    if (t->cfg.history_cap > 0) {
        const int pos = n < hc ? n : head;
        const int n2 = n < hc ? n + 1 : n, head2 = n < hc ? head : (head + 1) % hc;
        CU(cudaMemcpy(p.hist_ids + pos, &tok, 4, cudaMemcpyHostToDevice));
        CU(cudaMemcpy(t->hist_n + b, &n2, 4, cudaMemcpyHostToDevice));
        CU(cudaMemcpy(t->hist_head + b, &head2, 4, cudaMemcpyHostToDevice));
    }
    *token_out = tok;
    return LAL_TAIL_OK;
}

/* One stream's GPT-2 step with the level-2 filter hook (gpt2_server.c:
 * 2962-2978): the device exports the top-k pool with the nucleus's marks, the
 * host builds the keep mask over the vocabulary, calls the filter and restores
 * the pool when the mask comes back empty; the device then runs the softmax
 * and the draw over every row the mask keeps, in ascending order (rows the
 * filter added included, at their penalised logits).  Non-greedy only. */
int gpt2_filtered_step(lal_tail *t, int b, const float *d_hidden, const float *d_u,
                       float u_fallback, int *token_out) {
    const int hc = std::max(1, t->cfg.history_cap);
    const int V = t->cfg.vocab_size;
    int *status_p = t->io_out + t->cfg.max_streams;
    CHECK(enqueue_gpt2(t, b, d_hidden, d_u, t->f_tok, true));
    /* 1. the pool size, the status and the history ring */
    StreamDiag dg;
    int status = 0, n = 0, head = 0;
    CU(cudaMemcpyAsync(&dg, t->diag + b, sizeof(dg), cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(&status, status_p, 4, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(&n, t->hist_n + b, 4, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(&head, t->hist_head + b, 4, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    if (status != 0) {
        CU(cudaMemset(status_p, 0, 4));
        CU(cudaStreamSynchronize(t->stream));
        return fail(status, "device status %d in the filtered GPT-2 step", status);
    }
    const int m = dg.n_cand;
    if (m < 1 || m > t->nrows) return fail(LAL_TAIL_ERR_CAPACITY, "filtered step: %d candidates", m);
    std::vector<int> pool_keep((size_t)m);
    CU(cudaMemcpyAsync(t->f_ids.data(), t->f_cand_i, 4ull * m, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(pool_keep.data(), t->f_keep, 4ull * m, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaMemcpyAsync(t->f_ring.data(), t->hist_ids + (size_t)b * hc, 4ull * hc,
                       cudaMemcpyDeviceToHost, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    std::vector<int> recent((size_t)n);
    for (int i = 0; i < n; ++i)
        recent[i] = t->f_ring[(size_t)((n < hc ? 0 : head) + i) % (size_t)hc];
    /* 2. keep mask (top-k, narrowed by top-p), the filter, the restore of
     * the top-k pool when it keeps nothing */
    std::fill(t->f_mask.begin(), t->f_mask.end(), 0);
    for (int i = 0; i < m; ++i) t->f_mask[t->f_ids[i]] = pool_keep[i];
    if (t->filter) {
        const int last = n > 0 ? recent[n - 1] : -1;
        (void)t->filter(t->f_mask.data(), V, last, recent.data(), n, t->decode);
    }
    bool any = false;
    for (int v = 0; v < V && !any; ++v) any = t->f_mask[v] != 0;
    if (!any)
        for (int i = 0; i < m; ++i) t->f_mask[t->f_ids[i]] = 1;
    std::vector<int> &rows = t->f_keep_h;
    rows.clear();
    for (int v = 0; v < V; ++v)
        if (t->f_mask[v]) rows.push_back(v);
    const int mk = (int)rows.size();
    /* 3. softmax over the kept rows and the draw, on the device */
    CU(cudaMemcpyAsync(t->f_cand_i, rows.data(), 4ull * mk, cudaMemcpyHostToDevice, t->stream));
    FinishParams f;
    memset(&f, 0, sizeof(f));
    f.cand_val = nullptr;
    f.logits = t->logits + (size_t)b * t->nrows;
    f.cand_idx = t->f_cand_i;
    f.keep = nullptr;
    f.variant = VARIANT_GPT2;
    f.m = mk;
    f.temperature = t->h_temp[b];
    f.vocab = V;
    f.u = t->f_u;
    f.prefix = t->f_prefix;
    f.diag = t->f_diag;
    f.token = t->f_tok;
    f.expf_x = t->ds->d_expf_x;
    f.expf_y = t->ds->d_expf_y;
    f.expf_n = t->ds->expf_n;
    f.expf_bits = t->ds->d_expf_bits;
    f.expf_off = t->ds->d_expf_off;
    f.phase = 0;
    CU(launch_finish(f, t->stream));
    /* gpt2_server.c:2996: one draw every step, after the filter */
    const float u = t->draw ? t->draw(t->draw_ctx) : u_fallback;
    CU(cudaMemcpyAsync(t->f_u, &u, 4, cudaMemcpyHostToDevice, t->stream));
    f.phase = 1;
    CU(launch_finish(f, t->stream));
    int tok = -1;
    CU(cudaMemcpyAsync(&tok, t->f_tok, 4, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    /* 4. the history push (FIFO at history_cap) */
    if (t->cfg.history_cap > 0) {
        const int pos = n < hc ? n : head;
        const int n2 = n < hc ? n + 1 : n, head2 = n < hc ? head : (head + 1) % hc;
        CU(cudaMemcpy(t->hist_ids + (size_t)b * hc + pos, &tok, 4, cudaMemcpyHostToDevice));
        CU(cudaMemcpy(t->hist_n + b, &n2, 4, cudaMemcpyHostToDevice));
        CU(cudaMemcpy(t->hist_head + b, &head2, 4, cudaMemcpyHostToDevice));
    }
    *token_out = tok;
    return LAL_TAIL_OK;
}

}  // namespace

extern "C" {

int lal_tail_create(const lal_tail_config *cfg, lal_tail **out) {
    if (!cfg || !out) return fail(LAL_TAIL_ERR_ARG, "create: null argument");
    *out = nullptr;
    const lal_tail_config &c = *cfg;
    if (c.vocab_size < 1 || c.n_embd < 1 || c.max_streams < 1 || c.max_top_k < 1 ||
        c.history_cap < 0 || c.shard_count < 1 || c.shard_rank < 0 || c.shard_rank >= c.shard_count)
        return fail(LAL_TAIL_ERR_ARG, "create: bad config");
    if (c.sampler != LAL_SAMPLER_LIBRARY && c.sampler != LAL_SAMPLER_SERVER &&
        c.sampler != LAL_SAMPLER_GPT2)
        return fail(LAL_TAIL_ERR_ARG, "create: unknown sampler %d", c.sampler);
    /* the GPT-2 tail re-scores rows with eight-lane sums and no scalar tail
     * (gpt2_server.c:2207-2210 has one, which its compiler may contract) */
    if (c.sampler == LAL_SAMPLER_GPT2 && (c.shard_count != 1 || c.n_embd % 8 != 0))
        return fail(LAL_TAIL_ERR_UNSUPPORTED,
                    "create: the GPT-2 sampler needs one shard and n_embd a multiple of 8");
    lal_tail *t = new lal_tail();
    t->cfg = c;
    int dev = c.device;
    if (dev < 0) {
        int rc = current_device(&dev);
        if (rc) { delete t; return rc; }
    }
    t->device = dev;
    int rc = device_state(dev, &t->ds);
    if (rc == LAL_TAIL_OK) {
        cudaError_t e = cudaSetDevice(dev);
        if (e != cudaSuccess) rc = fail(LAL_TAIL_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    }
    if (rc == LAL_TAIL_OK) {
        t->row0 = (int)((long long)c.shard_rank * c.vocab_size / c.shard_count);
        t->nrows = (int)((long long)(c.shard_rank + 1) * c.vocab_size / c.shard_count) - t->row0;
        t->ld = ld_for(c.n_embd);
        if (t->nrows < 1) rc = fail(LAL_TAIL_ERR_ARG, "create: empty vocab slice");
    }
    if (rc == LAL_TAIL_OK) rc = ctx_alloc(t);
    if (rc != LAL_TAIL_OK) {
        std::string keep = g_err;
        destroy_ctx(t);
        g_err = keep;
        return rc;
    }
    *out = t;
    return LAL_TAIL_OK;
}

int lal_tail_destroy(lal_tail *t) {
    destroy_ctx(t);
    return LAL_TAIL_OK;
}

int lal_tail_shard_rows(const lal_tail *t, int *row0, int *n_rows) {
    if (!t) return fail(LAL_TAIL_ERR_ARG, "null context");
    if (row0) *row0 = t->row0;
    if (n_rows) *n_rows = t->nrows;
    return LAL_TAIL_OK;
}

int lal_tail_load_lm_head_q8(lal_tail *t, const int8_t *wte_q_rows, const float *scale_w_rows) {
    CHECK(ctx_check(t));
    CU(cudaStreamSynchronize(t->stream));
    free_copies(t);
    if (!wte_q_rows || !scale_w_rows) return fail(LAL_TAIL_ERR_ARG, "load_lm_head_q8: null");
    CHECK(upload_rows(wte_q_rows, t->nrows, t->cfg.n_embd, t->ld, t->W, t->stream));
    CU(cudaMemcpyAsync(t->sw, scale_w_rows, 4ull * t->nrows, cudaMemcpyHostToDevice, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    t->loaded = true;
    return LAL_TAIL_OK;
}

int lal_tail_load_lm_head_f32(lal_tail *t, const float *W_rows, int row_begin, int n_rows) {
    CHECK(ctx_check(t));
    CU(cudaStreamSynchronize(t->stream));
    free_copies(t);
    if (!W_rows || row_begin < 0 || n_rows < 0 || row_begin + n_rows > t->nrows)
        return fail(LAL_TAIL_ERR_ARG, "load_lm_head_f32: bad row range");
    const int d = t->cfg.n_embd;
    const int chunk = std::max(1, (int)((64ull << 20) / (4ull * d)));
    float *dW = nullptr;
    CU(cudaMalloc(&dW, 4ull * std::min(chunk, std::max(1, n_rows)) * d));
    int rc = LAL_TAIL_OK;
    for (int r = 0; r < n_rows && rc == LAL_TAIL_OK; r += chunk) {
        const int n = std::min(chunk, n_rows - r);
        cudaError_t e = cudaMemcpyAsync(dW, W_rows + (size_t)r * d, 4ull * n * d,
                                        cudaMemcpyHostToDevice, t->stream);
        if (e == cudaSuccess)
            e = launch_quantize_rows(dW, d, t->W + (size_t)(row_begin + r) * t->ld, t->ld,
                                     t->sw + row_begin + r, n, t->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(t->stream);
        if (e != cudaSuccess) rc = fail(LAL_TAIL_ERR_CUDA, "load_lm_head_f32: %s", cudaGetErrorString(e));
    }
    cudaFree(dW);
    if (rc == LAL_TAIL_OK && row_begin + n_rows == t->nrows) t->loaded = true;
    return rc;
}

int lal_tail_read_lm_head(lal_tail *t, int8_t *wte_q_rows, float *scale_w_rows) {
    CHECK(ctx_check(t));
    if (wte_q_rows)
        CU(cudaMemcpy2D(wte_q_rows, t->cfg.n_embd, t->W, t->ld, t->cfg.n_embd, t->nrows,
                        cudaMemcpyDeviceToHost));
    if (scale_w_rows) CU(cudaMemcpy(scale_w_rows, t->sw, 4ull * t->nrows, cudaMemcpyDeviceToHost));
    return LAL_TAIL_OK;
}

int lal_tail_set_sampling(lal_tail *t, int n_streams, const float *temperature,
                          const int *top_k, const float *rep_penalty) {
    CHECK(ctx_check(t));
    if (n_streams < 1 || n_streams > t->cfg.max_streams || !temperature || !top_k || !rep_penalty)
        return fail(LAL_TAIL_ERR_ARG, "set_sampling: bad arguments");
    for (int b = 0; b < n_streams; ++b) {
        const bool greedy = temperature[b] <= 0.0f || top_k[b] <= 0;
        if (!greedy && top_k[b] > t->cfg.max_top_k)
            return fail(LAL_TAIL_ERR_ARG, "top_k %d above the context's max_top_k %d", top_k[b],
                        t->cfg.max_top_k);
    }
    CU(cudaMemcpyAsync(t->temp, temperature, 4ull * n_streams, cudaMemcpyHostToDevice, t->stream));
    CU(cudaMemcpyAsync(t->topk, top_k, 4ull * n_streams, cudaMemcpyHostToDevice, t->stream));
    CU(cudaMemcpyAsync(t->pen, rep_penalty, 4ull * n_streams, cudaMemcpyHostToDevice, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    for (int b = 0; b < n_streams; ++b) {
        t->h_temp[b] = temperature[b];
        t->h_topk[b] = top_k[b];
        t->h_pen[b] = rep_penalty[b];
    }
    t->n_set = n_streams;
    return LAL_TAIL_OK;
}

int lal_tail_set_history(lal_tail *t, int stream, const int *recent, int n_recent) {
    CHECK(ctx_check(t));
    if (stream < 0 || stream >= t->cfg.max_streams || n_recent < 0 ||
        n_recent > t->cfg.history_cap || (n_recent > 0 && !recent))
        return fail(LAL_TAIL_ERR_ARG, "set_history: bad arguments");
    const int hc = std::max(1, t->cfg.history_cap);
    if (n_recent > 0)
        CU(cudaMemcpyAsync(t->hist_ids + (size_t)stream * hc, recent, 4ull * n_recent,
                           cudaMemcpyHostToDevice, t->stream));
    const int zero = 0;
    CU(cudaMemcpyAsync(t->hist_n + stream, &n_recent, 4, cudaMemcpyHostToDevice, t->stream));
    CU(cudaMemcpyAsync(t->hist_head + stream, &zero, 4, cudaMemcpyHostToDevice, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    return LAL_TAIL_OK;
}

int lal_tail_get_history(lal_tail *t, int stream, int *recent_out, int *n_out) {
    CHECK(ctx_check(t));
    if (stream < 0 || stream >= t->cfg.max_streams)
        return fail(LAL_TAIL_ERR_ARG, "get_history: bad stream");
    const int hc = std::max(1, t->cfg.history_cap);
    int n = 0, head = 0;
    CU(cudaStreamSynchronize(t->stream));
    CU(cudaMemcpy(&n, t->hist_n + stream, 4, cudaMemcpyDeviceToHost));
    CU(cudaMemcpy(&head, t->hist_head + stream, 4, cudaMemcpyDeviceToHost));
    std::vector<int> ring(hc);
    CU(cudaMemcpy(ring.data(), t->hist_ids + (size_t)stream * hc, 4ull * hc, cudaMemcpyDeviceToHost));
    if (n_out) *n_out = n;
    if (recent_out) /* oldest first: [head, n) then [0, head) */
        for (int i = 0; i < n; ++i) recent_out[i] = ring[(head + i) % (n < hc ? std::max(n, 1) : hc)];
    return LAL_TAIL_OK;
}

int lal_tail_device_buffers(lal_tail *t, float **d_hidden, float **d_u, int **d_tokens) {
    if (!t) return fail(LAL_TAIL_ERR_ARG, "null context");
    if (d_hidden) *d_hidden = t->io_in;
    if (d_u) *d_u = t->io_in + (size_t)t->cfg.max_streams * t->cfg.n_embd;
    if (d_tokens) *d_tokens = t->io_out;
    return LAL_TAIL_OK;
}

int lal_tail_get_stream(lal_tail *t, void **stream) {
    if (!t || !stream) return fail(LAL_TAIL_ERR_ARG, "get_stream: null argument");
    *stream = (void *)t->stream;
    return LAL_TAIL_OK;
}

int lal_tail_step_device(lal_tail *t, const float *d_hidden, int n_streams, const float *d_u,
                         int *d_tokens_out) {
    CHECK(ctx_check(t));
    if (!d_hidden || !d_u || !d_tokens_out) return fail(LAL_TAIL_ERR_ARG, "step_device: null");
    return enqueue_step(t, d_hidden, n_streams, d_u, d_tokens_out);
}

int lal_tail_sync(lal_tail *t) {
    CHECK(ctx_check(t));
    int status = 0;
    CU(cudaMemcpyAsync(&status, t->io_out + t->cfg.max_streams, 4, cudaMemcpyDeviceToHost, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    if (status != 0) {
        CU(cudaMemset(t->io_out + t->cfg.max_streams, 0, 4));
        CHECK(t->sel.reset(t->stream));
        CU(cudaStreamSynchronize(t->stream));
        return fail(status, "device status %d (%s)", status,
                    status == LAL_TAIL_ERR_TIMEOUT ? "bounded wait expired"
                                                   : "candidate set above the built capacity");
    }
    return LAL_TAIL_OK;
}

}  // extern "C"

namespace {
/* The step's inputs into io_in ([B][d] hidden, then the B draws) through the
 * pinned staging buffer: one copy when all B streams step (the two parts are
 * then contiguous), else one for each part. */
int upload_inputs(lal_tail *t, const float *hidden, int n, const float *u) {
    const int B = t->cfg.max_streams, d = t->cfg.n_embd;
    memcpy(t->h_in, hidden, 4ull * n * d);
    memcpy(t->h_in + (size_t)B * d, u, 4ull * n);
    if (n == B) {
        CU(cudaMemcpyAsync(t->io_in, t->h_in, 4ull * ((size_t)B * d + B), cudaMemcpyHostToDevice,
                           t->stream));
    } else {
        CU(cudaMemcpyAsync(t->io_in, t->h_in, 4ull * n * d, cudaMemcpyHostToDevice, t->stream));
        CU(cudaMemcpyAsync(t->io_in + (size_t)B * d, t->h_in + (size_t)B * d, 4ull * n,
                           cudaMemcpyHostToDevice, t->stream));
    }
    return LAL_TAIL_OK;
}
/* tokens [B] and the status word: one copy of the whole block */
int download_outputs(lal_tail *t) {
    CU(cudaMemcpyAsync(t->h_out, t->io_out, 4ull * (t->cfg.max_streams + 1),
                       cudaMemcpyDeviceToHost, t->stream));
    return LAL_TAIL_OK;
}

int step_status_error(lal_tail *t, int status) {
    const int B = t->cfg.max_streams;
    CU(cudaMemset(t->io_out + B, 0, 4));
    CHECK(t->sel.reset(t->stream));
    CU(cudaStreamSynchronize(t->stream));
    return fail(status, "device status %d (%s)", status,
                status == LAL_TAIL_ERR_TIMEOUT ? "bounded wait expired"
                                               : "candidate set above the built capacity");
}

/* lal_tail_step of an unsharded context, or of one stream on a vocab shard
 * connected to its peers: the inputs are staged in mapped
 * pinned memory and pulled onto the device by a small kernel (the step's
 * kernel begins streaming the LM head meanwhile), and each stream's kernel
 * stores [step number | token] into a mapped completion word that this
 * thread waits on -- no device-to-host copy and no stream synchronisation
 * on the way.  A stream whose step failed stores -1; its status is then read
 * the usual way.  If the stream completes without the words (a launch
 * error), the tokens are read back the usual way too. */
int notified_step(lal_tail *t, const float *hidden, int n, const float *u, int *tokens_out) {
    const int B = t->cfg.max_streams, d = t->cfg.n_embd;
    const unsigned seq = ++t->host_seq == 0 ? ++t->host_seq : t->host_seq;
    memcpy(t->h_in, hidden, 4ull * n * d);
    memcpy(t->h_in + (size_t)B * d, u, 4ull * n);
    memcpy(t->h_in + (size_t)B * d + B, &seq, 4);
    CU(launch_stage_inputs(t->d_h_in, t->io_in, n * d, B * d, B + 1, t->stream));
    CHECK(enqueue_step(t, t->io_in, n, t->io_in + (size_t)B * d, t->io_out, false, true));
    const auto t0 = std::chrono::steady_clock::now();
    bool done = false, drained = false;
    for (unsigned it = 1;; ++it) {
        done = true;
        for (int b = 0; b < n && done; ++b) {
            const unsigned long long v = __atomic_load_n(&t->h_tok[b], __ATOMIC_ACQUIRE);
            done = (unsigned)(v >> 32) == seq;
        }
        if (done || drained) break;
        if ((it & 1023u) == 0) {
            const cudaError_t q = cudaStreamQuery(t->stream);
            if (q == cudaSuccess) drained = true; /* one more look at the words */
            else if (q != cudaErrorNotReady) return fail(LAL_TAIL_ERR_CUDA, "step: %s", cudaGetErrorString(q));
            else if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60))
                return fail(LAL_TAIL_ERR_TIMEOUT, "step: no completion within 60 s");
        }
#if defined(__x86_64__)
        __builtin_ia32_pause();
#endif
    }
    bool failed = !done;
    for (int b = 0; b < n && !failed; ++b) {
        tokens_out[b] = (int)(uint32_t)t->h_tok[b];
        failed = tokens_out[b] < 0;
    }
    if (!failed) return LAL_TAIL_OK;
    CHECK(download_outputs(t));
    CU(cudaStreamSynchronize(t->stream));
    const int status = t->h_out[B];
    if (status != 0) return step_status_error(t, status);
    memcpy(tokens_out, t->h_out, 4ull * n);
    return LAL_TAIL_OK;
}
}  // namespace

extern "C" {

int lal_tail_step(lal_tail *t, const float *hidden, int n_streams, const float *u,
                  int *tokens_out) {
    CHECK(ctx_check(t));
    if (!hidden || !u || !tokens_out) return fail(LAL_TAIL_ERR_ARG, "step: null argument");
    if (n_streams < 1 || n_streams > t->cfg.max_streams)
        return fail(LAL_TAIL_ERR_ARG, "n_streams %d out of range", n_streams);
    if (t->filtered) {
        if (!t->loaded) return fail(LAL_TAIL_ERR_STATE, "step before the LM head was loaded");
        if (t->n_set < n_streams)
            return fail(LAL_TAIL_ERR_STATE, "sampling parameters not set for %d streams", n_streams);
        CHECK(lal_tail_stage_inputs(t, hidden, n_streams, u));
        const int Bmax = t->cfg.max_streams;
        for (int b = 0; b < n_streams; ++b) {
            if (t->cfg.sampler == LAL_SAMPLER_GPT2) {
                if (t->h_temp[b] <= 0.0f || t->h_topk[b] <= 0) {
                    /* greedy: argmax, no penalty, no filter (gpt2_server.c:3005) */
                    CHECK(enqueue_gpt2(t, b, t->io_in, t->io_in + (size_t)Bmax * t->cfg.n_embd,
                                       t->io_out));
                    CU(cudaMemcpyAsync(tokens_out + b, t->io_out + b, 4, cudaMemcpyDeviceToHost,
                                       t->stream));
                    CHECK(lal_tail_sync(t));
                } else {
                    CHECK(gpt2_filtered_step(t, b, t->io_in,
                                             t->io_in + (size_t)Bmax * t->cfg.n_embd, u[b],
                                             tokens_out + b));
                }
                continue;
            }
            if (t->h_temp[b] <= 0.0f || t->h_topk[b] <= 0) {
                /* greedy: penalty then argmax, no filter (qwen7b_server.c:233-234) */
                CHECK(enqueue_one(t, b));
                CU(cudaMemcpyAsync(tokens_out + b, t->io_out + b, 4, cudaMemcpyDeviceToHost,
                                   t->stream));
                CHECK(lal_tail_sync(t));
            } else {
                CHECK(filtered_stream_step(t, b, t->io_in, u[b], tokens_out + b));
            }
        }
        return LAL_TAIL_OK;
    }
    const int B = t->cfg.max_streams, d = t->cfg.n_embd;
    /* unsharded steps, and single-stream steps of a vocab shard connected to
     * its peers (one kernel per rank draws the token): inputs pulled from
     * mapped memory, the token handed back through the completion word */
    if (t->cfg.sampler != LAL_SAMPLER_GPT2 &&
        (t->cfg.shard_count == 1 || (t->p2p && n_streams == 1)))
        return notified_step(t, hidden, n_streams, u, tokens_out);
    CHECK(upload_inputs(t, hidden, n_streams, u));
    CHECK(enqueue_step(t, t->io_in, n_streams, t->io_in + (size_t)B * d, t->io_out));
    CHECK(download_outputs(t));
    CU(cudaStreamSynchronize(t->stream));
    const int status = t->h_out[B];
    if (status != 0) {
        CU(cudaMemset(t->io_out + B, 0, 4));
        CHECK(t->sel.reset(t->stream));
        CU(cudaStreamSynchronize(t->stream));
        return fail(status, "device status %d (%s)", status,
                    status == LAL_TAIL_ERR_TIMEOUT ? "bounded wait expired"
                                                   : "candidate set above the built capacity");
    }
    memcpy(tokens_out, t->h_out, 4ull * n_streams);
    return LAL_TAIL_OK;
}

int lal_tail_stage_inputs(lal_tail *t, const float *hidden, int n_streams, const float *u) {
    CHECK(ctx_check(t));
    if (!hidden || !u) return fail(LAL_TAIL_ERR_ARG, "stage_inputs: null argument");
    if (n_streams < 1 || n_streams > t->cfg.max_streams)
        return fail(LAL_TAIL_ERR_ARG, "n_streams %d out of range", n_streams);
    return upload_inputs(t, hidden, n_streams, u);
}

int lal_tail_fetch_tokens(lal_tail *t, int n_streams, int *tokens_out) {
    CHECK(ctx_check(t));
    if (!tokens_out || n_streams < 1 || n_streams > t->cfg.max_streams)
        return fail(LAL_TAIL_ERR_ARG, "fetch_tokens: bad arguments");
    const int B = t->cfg.max_streams;
    CHECK(download_outputs(t));
    CU(cudaStreamSynchronize(t->stream));
    const int status = t->h_out[B];
    if (status != 0) {
        CU(cudaMemset(t->io_out + B, 0, 4));
        CHECK(t->sel.reset(t->stream));
        CU(cudaStreamSynchronize(t->stream));
        return fail(status, "device status %d (%s)", status,
                    status == LAL_TAIL_ERR_TIMEOUT ? "bounded wait expired"
                                                   : "candidate set above the built capacity");
    }
    memcpy(tokens_out, t->h_out, 4ull * n_streams);
    return LAL_TAIL_OK;
}

int lal_tail_shard_select(lal_tail *t, const float *d_hidden, int n_streams) {
    CHECK(ctx_check(t));
    if (!d_hidden) return fail(LAL_TAIL_ERR_ARG, "shard_select: null hidden");
    return enqueue_step(t, d_hidden, n_streams, nullptr, nullptr, true);
}

int lal_tail_exchange_buffers(lal_tail *t, int n_streams, void **d_send, void **d_recv,
                              size_t *bytes_per_rank) {
    if (!t) return fail(LAL_TAIL_ERR_ARG, "null context");
    if (n_streams < 1 || n_streams > t->cfg.max_streams)
        return fail(LAL_TAIL_ERR_ARG, "n_streams %d out of range", n_streams);
    if (d_send) *d_send = t->x_send;
    if (d_recv) *d_recv = t->x_recv;
    if (bytes_per_rank) *bytes_per_rank = (size_t)n_streams * t->rec_bytes;
    return LAL_TAIL_OK;
}

int lal_tail_shard_merge(lal_tail *t, int n_streams, const float *d_u, int *d_tokens_out) {
    CHECK(ctx_check(t));
    if (!d_u || !d_tokens_out) return fail(LAL_TAIL_ERR_ARG, "shard_merge: null argument");
    if (n_streams < 1 || n_streams > t->cfg.max_streams)
        return fail(LAL_TAIL_ERR_ARG, "n_streams %d out of range", n_streams);
    if (t->n_set < n_streams)
        return fail(LAL_TAIL_ERR_STATE, "sampling parameters not set for %d streams", n_streams);
    MergeParams m;
    memset(&m, 0, sizeof(m));
    m.recv = t->x_recv;
    m.rank_stride = (long long)n_streams * t->rec_bytes;
    m.rec_bytes = t->rec_bytes;
    m.rec_cap = t->rec_cap;
    m.n_ranks = t->cfg.shard_count;
    m.vocab = t->cfg.vocab_size;
    m.variant = t->cfg.sampler == LAL_SAMPLER_SERVER ? VARIANT_SERVER : VARIANT_LIBRARY;
    m.temperature = t->temp;
    m.top_k = t->topk;
    m.u = d_u;
    m.hist_ids = t->hist_ids;
    m.hist_n = t->hist_n;
    m.hist_head = t->hist_head;
    m.hist_cap = t->cfg.history_cap;
    m.push_history = t->cfg.history_cap > 0 ? 1 : 0;
    m.tokens = d_tokens_out;
    m.diag = t->diag;
    m.status = t->io_out + t->cfg.max_streams;
    m.expf_x = t->ds->d_expf_x;
    m.expf_y = t->ds->d_expf_y;
    m.expf_n = t->ds->expf_n;
    m.expf_bits = t->ds->d_expf_bits;
    m.expf_off = t->ds->d_expf_off;
    m.expf_hash = t->ds->d_expf_hash;
    m.expf_hash_probe = t->ds->expf_hash_probe;
    m.smem_cap = t->merge_cap;
    CU(launch_merge(m, n_streams, t->stream));
    return LAL_TAIL_OK;
}

int lal_tail_exchange_handle(lal_tail *t, void *handle_out) {
    CHECK(ctx_check(t));
    if (!handle_out) return fail(LAL_TAIL_ERR_ARG, "exchange_handle: null");
    if (!t->x_peer) return fail(LAL_TAIL_ERR_STATE, "exchange_handle: context is not sharded");
    static_assert(sizeof(cudaIpcMemHandle_t) == LAL_TAIL_IPC_HANDLE_BYTES, "IPC handle size");
    /* the receive buffer starts clean before any peer can learn its address:
     * a peer that connects first and steps at once then writes into a buffer
     * that no later clear can erase */
    CU(cudaStreamSynchronize(t->stream));
    CU(cudaMemsetAsync(t->x_peer, 0, 2ull * t->cfg.shard_count * t->peer_rec_bytes, t->stream));
    CU(cudaStreamSynchronize(t->stream));
    cudaIpcMemHandle_t h;
    CU(cudaIpcGetMemHandle(&h, t->x_peer));
    memcpy(handle_out, &h, sizeof(h));
    return LAL_TAIL_OK;
}

int lal_tail_connect_peers(lal_tail *t, const void *handles) {
    CHECK(ctx_check(t));
    if (!handles) return fail(LAL_TAIL_ERR_ARG, "connect_peers: null");
    if (!t->x_peer) return fail(LAL_TAIL_ERR_STATE, "connect_peers: context is not sharded");
    const int N = t->cfg.shard_count;
    if (peer_merge_cap(t->plan) < N * t->rec_cap)
        return fail(LAL_TAIL_ERR_UNSUPPORTED, "connect_peers: %d shards x %d candidates exceed "
                    "the fused kernel's merge area", N, t->rec_cap);
    CU(cudaStreamSynchronize(t->stream));
    close_peers(t);
    std::vector<uint8_t *> ptrs(N, nullptr);
    for (int r = 0; r < N; ++r) {
        if (r == t->cfg.shard_rank) {
            ptrs[r] = t->x_peer;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *)handles + (size_t)r * sizeof(h), sizeof(h));
        void *q = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&q, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            close_peers(t);
            return fail(LAL_TAIL_ERR_COMM, "connect_peers: rank %d: %s", r, cudaGetErrorString(e));
        }
        t->peer_open.push_back(q);
        ptrs[r] = (uint8_t *)q;
    }
    CU(cudaMemcpyAsync(t->d_peer, ptrs.data(), sizeof(uint8_t *) * N, cudaMemcpyHostToDevice,
                       t->stream));
    CU(cudaStreamSynchronize(t->stream));
    /* (the receive buffer was cleared by lal_tail_exchange_handle, before its
     * handle left this rank) */
    t->seq = 1;
    t->p2p = true;
    return LAL_TAIL_OK;
}

int lal_tail_disconnect_peers(lal_tail *t) {
    CHECK(ctx_check(t));
    CU(cudaStreamSynchronize(t->stream));
    close_peers(t);
    return LAL_TAIL_OK;
}

/* GPQ8 tensor directory (tools/server/qwen7b_server.c:499-505, 524-563):
 * "GPQ8", int32 count, then per tensor: int32 key length, key bytes, int32
 * ndim, int32 shape[ndim], uint8 qtype (0 = F32, 1 = Q8), uint64 data length,
 * data, int32 scale count, float scales (keys up to 127 bytes, the server's
 * char key[128]).  Every field is bounds-checked against the blob (the server
 * trusts its file; a library must not). */
int lal_tail_gpq8_find(const void *blob, size_t size, const char *key, lal_gpq8_tensor *out) {
    if (!blob || !key || !out) return fail(LAL_TAIL_ERR_ARG, "gpq8: null argument");
    const unsigned char *b = (const unsigned char *)blob;
    size_t off = 0;
    auto take = [&](void *dst, size_t n) {
        if (n > size || off > size - n) return false;
        memcpy(dst, b + off, n);
        off += n;
        return true;
    };
    char magic[4];
    int32_t count = 0;
    if (!take(magic, 4) || memcmp(magic, "GPQ8", 4) != 0) return fail(LAL_TAIL_ERR_ARG, "gpq8: bad magic");
    if (!take(&count, 4) || count < 0) return fail(LAL_TAIL_ERR_ARG, "gpq8: bad tensor count");
    const size_t klen_want = strlen(key);
    for (int32_t i = 0; i < count; ++i) {
        int32_t klen = 0, ndim = 0, n_scale = 0;
        uint8_t qtype = 0;
        uint64_t dlen = 0;
        if (!take(&klen, 4) || klen < 0 || klen > 127 || (size_t)klen > size - off)
            return fail(LAL_TAIL_ERR_ARG, "gpq8: tensor %d: bad key", (int)i);
        const bool match = (size_t)klen == klen_want && memcmp(b + off, key, (size_t)klen) == 0;
        off += (size_t)klen;
        if (!take(&ndim, 4) || ndim < 0 || ndim > 4)
            return fail(LAL_TAIL_ERR_ARG, "gpq8: tensor %d: bad ndim", (int)i);
        int32_t shape[4] = {0, 0, 0, 0};
        for (int d = 0; d < ndim; ++d)
            if (!take(&shape[d], 4) || shape[d] < 0)
                return fail(LAL_TAIL_ERR_ARG, "gpq8: tensor %d: bad shape", (int)i);
        if (!take(&qtype, 1) || qtype > 1 || !take(&dlen, 8) || dlen > size - off)
            return fail(LAL_TAIL_ERR_ARG, "gpq8: tensor %d: bad data", (int)i);
        const uint64_t data_off = off;
        off += (size_t)dlen;
        if (!take(&n_scale, 4) || n_scale < 0 || (size_t)n_scale * 4 > size - off)
            return fail(LAL_TAIL_ERR_ARG, "gpq8: tensor %d: bad scales", (int)i);
        const uint64_t scale_off = off;
        off += (size_t)n_scale * 4;
        if (match) {
            out->ndim = ndim;
            for (int d = 0; d < 4; ++d) out->shape[d] = shape[d];
            out->qtype = qtype;
            out->data_offset = data_off;
            out->data_len = dlen;
            out->n_scale = n_scale;
            out->scale_offset = scale_off;
            return LAL_TAIL_OK;
        }
    }
    return fail(LAL_TAIL_ERR_ARG, "gpq8: tensor %s not found", key);
}

int lal_tail_load_lm_head_gpq8(lal_tail *t, const void *blob, size_t size, const char *key) {
    CHECK(ctx_check(t));
    const char *name = key ? key : "lm_head.weight";
    lal_gpq8_tensor e;
    CHECK(lal_tail_gpq8_find(blob, size, name, &e));
    const long long V = t->cfg.vocab_size, d = t->cfg.n_embd;
    if (e.ndim != 2 || e.shape[0] != V || e.shape[1] != d)
        return fail(LAL_TAIL_ERR_ARG, "gpq8: %s is not [%lld, %lld]", name, V, d);
    const unsigned char *b = (const unsigned char *)blob;
    if (e.qtype == 0) {
        /* F32: quantized on the GPU as lal_quantize_q8_per_row does at load
         * (qwen7b_server.c:1106-1112), this context's rows only */
        if (e.data_len != (uint64_t)(V * d * 4)) return fail(LAL_TAIL_ERR_ARG, "gpq8: F32 size");
        std::vector<float> rows;
        const float *src = (const float *)(b + e.data_offset) + (size_t)t->row0 * d;
        if (((uintptr_t)src & 3u) != 0) { /* the file's float data need not be aligned */
            rows.resize((size_t)t->nrows * d);
            memcpy(rows.data(), b + e.data_offset + 4ull * t->row0 * d, 4ull * t->nrows * d);
            src = rows.data();
        }
        return lal_tail_load_lm_head_f32(t, src, 0, t->nrows);
    }
    if (e.data_len != (uint64_t)(V * d) || e.n_scale != V)
        return fail(LAL_TAIL_ERR_ARG, "gpq8: Q8 size");
    const int8_t *q = (const int8_t *)(b + e.data_offset) + (size_t)t->row0 * d;
    std::vector<float> sc((size_t)t->nrows);
    memcpy(sc.data(), b + e.scale_offset + 4ull * t->row0, 4ull * t->nrows);
    return lal_tail_load_lm_head_q8(t, q, sc.data());
}

int lal_tail_set_top_p(lal_tail *t, float top_p) {
    CHECK(ctx_check(t));
    if (t->cfg.sampler != LAL_SAMPLER_GPT2)
        return fail(LAL_TAIL_ERR_UNSUPPORTED,
                    "set_top_p: only the GPT-2 server's sampler has a nucleus step");
    if (top_p != top_p) return fail(LAL_TAIL_ERR_ARG, "set_top_p: NaN");
    /* gpt2_server.c:3147-3148 clamps the request to [0, 1]; 0 and 1 keep the
     * whole top-k pool */
    if (top_p < 0.0f) top_p = 0.0f;
    if (top_p > 1.0f) top_p = 1.0f;
    CU(cudaStreamSynchronize(t->stream));
    t->g2_top_p = top_p;
    return LAL_TAIL_OK;
}

int lal_tail_step_kind(lal_tail *t, int n_streams) {
    if (!t) return -fail(LAL_TAIL_ERR_ARG, "null context");
    if (n_streams < 1 || n_streams > t->cfg.max_streams)
        return -fail(LAL_TAIL_ERR_ARG, "n_streams %d out of range", n_streams);
    if (t->cfg.sampler == LAL_SAMPLER_GPT2) return LAL_TAIL_STEP_GPT2;
    if (t->batch_ok && n_streams >= 2 && !getenv_flag("LAL_TAIL_PER_STREAM"))
        return LAL_TAIL_STEP_BATCHED;
    return LAL_TAIL_STEP_PER_STREAM;
}

int lal_tail_set_lm_head_copies(lal_tail *t, int copies) {
    CHECK(ctx_check(t));
    if (copies < 1 || copies > 64) return fail(LAL_TAIL_ERR_ARG, "set_lm_head_copies: 1..64");
    if (!t->loaded) return fail(LAL_TAIL_ERR_STATE, "set_lm_head_copies before the LM head was loaded");
    CU(cudaStreamSynchronize(t->stream));
    free_copies(t);
    const size_t wb = (size_t)t->nrows * t->ld, sb = 4ull * t->nrows;
    for (int c = 1; c < copies; ++c) {
        int8_t *w = nullptr;
        float *f = nullptr;
        cudaError_t e = cudaMalloc(&w, wb);
        if (e == cudaSuccess) e = cudaMalloc(&f, sb);
        if (e == cudaSuccess) e = cudaMemcpyAsync(w, t->W, wb, cudaMemcpyDeviceToDevice, t->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(f, t->sw, sb, cudaMemcpyDeviceToDevice, t->stream);
        if (w) t->w_copies.push_back(w);
        if (f) t->sw_copies.push_back(f);
        if (e != cudaSuccess) {
            cudaStreamSynchronize(t->stream);
            free_copies(t);
            return fail(LAL_TAIL_ERR_CUDA, "set_lm_head_copies: %s", cudaGetErrorString(e));
        }
    }
    CU(cudaStreamSynchronize(t->stream));
    return LAL_TAIL_OK;
}

int lal_tail_set_final_norm(lal_tail *t, const float *norm_w, float eps) {
    CHECK(ctx_check(t));
    if (!norm_w) {
        CU(cudaStreamSynchronize(t->stream));
        t->plan.norm_w = nullptr;
        t->plan.norm_eps = 0.0f;
        return LAL_TAIL_OK;
    }
    const int d = t->cfg.n_embd;
    /* n_embd % 8 == 0: the reference's SIMD loop then covers every element;
     * its scalar tail loop (lal_simd_optim.h:45) is compiled by the
     * reference's compiler into a mix of separately rounded and fused
     * products, which no fixed rule reproduces */
    if (d > kNormMaxD || d % 8 != 0)
        return fail(LAL_TAIL_ERR_UNSUPPORTED,
                    "set_final_norm: n_embd %d must be a multiple of 8 and <= %d", d, kNormMaxD);
    if (!(eps >= 0.0f) || eps == INFINITY)
        return fail(LAL_TAIL_ERR_ARG, "set_final_norm: eps must be finite and >= 0");
    if (!t->d_norm_w) CU(cudaMalloc(&t->d_norm_w, sizeof(float) * (size_t)d));
    /* on the context's stream: steps already queued keep reading the old
     * weights until they finish, later steps see the new ones */
    CU(cudaMemcpyAsync(t->d_norm_w, norm_w, sizeof(float) * (size_t)d, cudaMemcpyHostToDevice,
                       t->stream));
    CU(cudaStreamSynchronize(t->stream));
    t->plan.norm_w = t->d_norm_w;
    t->plan.norm_eps = eps;
    return LAL_TAIL_OK;
}

int lal_tail_set_filter(lal_tail *t, lal_filter_topk_fn filter, lal_token_decode_fn decode,
                        lal_draw_fn draw, void *draw_ctx) {
    CHECK(ctx_check(t));
    if (!filter && !draw) {
        t->filtered = false;
        t->filter = nullptr;
        t->decode = nullptr;
        t->draw = nullptr;
        t->draw_ctx = nullptr;
        return LAL_TAIL_OK;
    }
    if ((t->cfg.sampler != LAL_SAMPLER_SERVER && t->cfg.sampler != LAL_SAMPLER_GPT2) ||
        t->cfg.shard_count != 1)
        return fail(LAL_TAIL_ERR_UNSUPPORTED,
                    "set_filter: the filter hook needs the server or GPT-2 sampler and one shard");
    if (!t->f_cand_v) {
        const size_t r = (size_t)t->nrows;
        CU(cudaMalloc(&t->f_cand_v, 4 * r));
        CU(cudaMalloc(&t->f_cand_i, 4 * r));
        CU(cudaMalloc(&t->f_keep, 4 * r));
        CU(cudaMalloc(&t->f_prefix, 4 * r));
        CU(cudaMalloc(&t->f_u, 4));
        CU(cudaMalloc(&t->f_tok, 4));
        CU(cudaMalloc(&t->f_diag, sizeof(StreamDiag)));
        t->f_mask.assign((size_t)t->cfg.vocab_size, 0);
        t->f_ids.assign(r, 0);
        t->f_ring.assign((size_t)std::max(1, t->cfg.history_cap), 0);
    }
    t->filter = filter;
    t->decode = decode;
    t->draw = draw;
    t->draw_ctx = draw_ctx;
    t->filtered = true;
    return LAL_TAIL_OK;
}

int lal_tail_get_diag(lal_tail *t, int stream, lal_tail_diag *out) {
    CHECK(ctx_check(t));
    if (stream < 0 || stream >= t->cfg.max_streams || !out)
        return fail(LAL_TAIL_ERR_ARG, "get_diag: bad arguments");
    static_assert(sizeof(StreamDiag) == sizeof(lal_tail_diag), "diag layout");
    CU(cudaStreamSynchronize(t->stream));
    CU(cudaMemcpy(out, t->diag + stream, sizeof(StreamDiag), cudaMemcpyDeviceToHost));
    return LAL_TAIL_OK;
}

int lal_tail_get_logits(lal_tail *t, int stream, float *logits_rows) {
    CHECK(ctx_check(t));
    if (stream < 0 || stream >= t->cfg.max_streams || !logits_rows)
        return fail(LAL_TAIL_ERR_ARG, "get_logits: bad arguments");
    CU(cudaStreamSynchronize(t->stream));
    CU(cudaMemcpy(logits_rows, t->logits + (size_t)stream * t->nrows, 4ull * t->nrows,
                  cudaMemcpyDeviceToHost));
    return LAL_TAIL_OK;
}

int lal_tail_set_timing(lal_tail *t, int on) {
    CHECK(ctx_check(t));
    t->timing = on != 0;
    if (t->timing && t->ev.empty()) {
        t->ev.resize(8192);
        for (auto &e : t->ev) CU(cudaEventCreate(&e));
    }
    t->ev_used = 0;
    return LAL_TAIL_OK;
}

int lal_tail_debug_phases(lal_tail *t, int on) {
    CHECK(ctx_check(t));
    if (on && !t->phase_ts) {
        CU(cudaMalloc(&t->phase_ts, sizeof(unsigned long long) * (kMaxGrid + 1) * 8));
        CU(cudaMemset(t->phase_ts, 0, sizeof(unsigned long long) * (kMaxGrid + 1) * 8));
    }
    t->phases = on != 0;
    return LAL_TAIL_OK;
}

int lal_tail_debug_phase_read(lal_tail *t, unsigned long long *out, int cap, int *grid) {
    CHECK(ctx_check(t));
    if (grid) *grid = t->grid;
    if (!t->phase_ts || !out) return LAL_TAIL_OK;
    const int n = std::min(cap, (t->grid + 2) * 8);
    CU(cudaStreamSynchronize(t->stream));
    CU(cudaMemcpy(out, t->phase_ts, sizeof(unsigned long long) * n, cudaMemcpyDeviceToHost));
    return LAL_TAIL_OK;
}

int lal_tail_kernel_time(lal_tail *t, double *avg_ms, int *n_launches) {
    CHECK(ctx_check(t));
    CU(cudaStreamSynchronize(t->stream));
    double tot = 0.0;
    const int n = t->ev_used / 2;
    for (int i = 0; i < n; ++i) {
        float ms = 0.0f;
        CU(cudaEventElapsedTime(&ms, t->ev[2 * i], t->ev[2 * i + 1]));
        tot += ms;
    }
    if (avg_ms) *avg_ms = n ? tot / n : 0.0;
    if (n_launches) *n_launches = n;
    t->ev_used = 0;
    return LAL_TAIL_OK;
}

}  // extern "C"
