/*
 * tail_noalloc.cu -- lal_tail_sample_token_noalloc: lal_sample_token
 * (runtime/lal_sampling.h:46-125, library semantics) on logits that already
 * live in device memory, with all of its working memory in two fixed
 * file-scope device arrays.  A call allocates nothing: no cudaMalloc, no
 * pinned or heap buffer, no library routine that allocates.
 *
 * Who needs it: a caller whose device memory is planned up front and must
 * not move while its decode loop runs -- e.g. a server that has handed the
 * rest of HBM to its KV cache and LM head, or one that keeps kernels queued
 * back to back and cannot afford the device-wide synchronisation that
 * cudaMalloc / cudaFree imply.  The drop-in lal_sample_token grows buffers
 * on demand (the first call at a vocab size allocates, a larger vocab
 * reallocates); this entry never does.
 *
 * Limits and rules:
 *  - vocab_size <= kNaMaxVocab (262,144; Qwen2.5's 152,064 and GPT-2's
 *    50,257 fit); larger sizes are rejected with LAL_TAIL_ERR_ARG before any
 *    device work.  The arrays take 2.1 MB (scratch) + 3.1 MB (expf table).
 *  - The first call on a device does the set-up (symbol addresses, the expf
 *    table copied in and indexed, the kernel's shared-memory limit), with
 *    that device current; make that first call before any stream capture.
 *  - The scratch words [0, kNaParams) -- key histogram, grid-barrier
 *    arrivals, append count, arrival ticket, edge word, status -- must be
 *    zero when a launch starts.  Static device memory is zero when the
 *    module loads, every launch returns them to zero, and an error return
 *    clears them again before it reports.
 *  - One scratch per device: calls that overlap on one device (two host
 *    threads, or two streams in flight) race on it and give wrong results.
 *    Serialise them.
 */
#include "../../include/lal_tail.h"
#include "tail_internal.h"

#include <cstdio>
#include <cstring>
#include <mutex>

/* glibc-expf fix-up table, embedded at build time (expf_blob.S) */
extern "C" const unsigned char lal_expf_fixups_blob[];
extern "C" const unsigned char lal_expf_fixups_blob_end[];

using namespace lal;

namespace {

constexpr int kNaMaxVocab = 1 << 18;
constexpr int kNaMaxFixups = 1 << 17;

/* word offsets inside the scratch array */
constexpr int kNaBar = kHistWords;              /* barrier arrivals, generation,
                                                 * append count, ticket, edge */
constexpr int kNaMax = kNaBar + 8;              /* per-CTA maxima [kMaxGrid]   */
constexpr int kNaSlotN = kNaMax + kMaxGrid;     /* per-CTA slot counts         */
constexpr int kNaStatus = kNaSlotN + kMaxGrid;  /* status, token               */
constexpr int kNaParams = kNaStatus + 8;        /* temperature, top_k, penalty,
                                                 * u, history length, head     */
constexpr int kNaDiag = kNaParams + 8;          /* StreamDiag                  */
constexpr int kNaKeys = kNaDiag + 8;            /* superset keys [kNaMaxVocab] */
constexpr int kNaIdx = kNaKeys + kNaMaxVocab;   /* superset ids [kNaMaxVocab]  */
constexpr int kNaWords = kNaIdx + kNaMaxVocab;
static_assert(kNaMaxVocab >= kSelectCapMin, "slot layout of the small-k select");

/* expf table: x [kNaMaxFixups], y [kNaMaxFixups], bitmap, offsets */
constexpr int kNaExpfY = kNaMaxFixups;
constexpr int kNaExpfBits = 2 * kNaMaxFixups;
constexpr int kNaExpfOff = kNaExpfBits + kExpfBitmapWords;
constexpr int kNaExpfWords = kNaExpfOff + kExpfBitmapWords + 1;

static __device__ __align__(256) uint32_t g_na_scratch[kNaWords];
static __device__ __align__(256) uint32_t g_na_expf[kNaExpfWords];

struct NaDevice {
    bool ready = false;
    int num_sms = 0;
    uint32_t *scratch = nullptr;
    uint32_t *expf = nullptr;
    int expf_n = 0;
};
std::mutex g_na_mu;
NaDevice g_na[64];

int cuda_fail(const char *what, cudaError_t e) {
    char buf[256];
    snprintf(buf, sizeof(buf), "sample_token_noalloc: %s: %s", what, cudaGetErrorString(e));
    return set_error(LAL_TAIL_ERR_CUDA, buf);
}

#define NA_CU(call)                                        \
    do {                                                   \
        cudaError_t e_ = (call);                           \
        if (e_ != cudaSuccess) return cuda_fail(#call, e_); \
    } while (0)

/* Once per device, with that device current. */
int na_setup(int dev, NaDevice **out) {
    std::lock_guard<std::mutex> lk(g_na_mu);
    NaDevice &d = g_na[dev];
    if (!d.ready) {
        int major = 0;
        NA_CU(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10)
            return set_error(LAL_TAIL_ERR_UNSUPPORTED,
                             "sample_token_noalloc: this library is built for sm_100a");
        NA_CU(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev));
        NA_CU(cudaGetSymbolAddress((void **)&d.scratch, g_na_scratch));
        NA_CU(cudaGetSymbolAddress((void **)&d.expf, g_na_expf));
        const size_t blob = (size_t)(lal_expf_fixups_blob_end - lal_expf_fixups_blob);
        uint32_t n = 0;
        if (blob >= 4) memcpy(&n, lal_expf_fixups_blob, 4);
        if (blob < 4 || blob < 4 + 8ull * n)
            return set_error(LAL_TAIL_ERR_STATE, "sample_token_noalloc: expf table missing");
        if (n > (uint32_t)kNaMaxFixups)
            return set_error(LAL_TAIL_ERR_STATE,
                             "sample_token_noalloc: expf table above its static capacity");
        NA_CU(cudaMemcpy(d.expf, lal_expf_fixups_blob + 4, 4ull * n, cudaMemcpyHostToDevice));
        NA_CU(cudaMemcpy(d.expf + kNaExpfY, lal_expf_fixups_blob + 4 + 4ull * n, 4ull * n,
                         cudaMemcpyHostToDevice));
        NA_CU(launch_expf_index(d.expf, (int)n, d.expf + kNaExpfBits, d.expf + kNaExpfOff, 0));
        NA_CU(cudaMemset(d.scratch, 0, 4ull * kNaParams));
        NA_CU(cudaStreamSynchronize(0));
        NA_CU(prepare_sample_kernel());
        d.expf_n = (int)n;
        d.ready = true;
    }
    *out = &d;
    return LAL_TAIL_OK;
}

}  // namespace

extern "C" int lal_tail_sample_token_noalloc(float *d_logits, int vocab_size, float temperature,
                                             int top_k, float rep_penalty, const int *d_recent,
                                             int n_recent, float u, void *stream,
                                             int *token_out) {
    if (!d_logits || !token_out || vocab_size < 1 || n_recent < 0 || (n_recent > 0 && !d_recent))
        return set_error(LAL_TAIL_ERR_ARG, "sample_token_noalloc: bad arguments");
    if (vocab_size > kNaMaxVocab) {
        char buf[160];
        snprintf(buf, sizeof(buf),
                 "sample_token_noalloc: vocab_size %d above the static scratch limit %d",
                 vocab_size, kNaMaxVocab);
        return set_error(LAL_TAIL_ERR_ARG, buf);
    }
    int dev = 0;
    NA_CU(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(LAL_TAIL_ERR_ARG, "sample_token_noalloc: device");
    NaDevice *d = nullptr;
    int rc = na_setup(dev, &d);
    if (rc != LAL_TAIL_OK) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    uint32_t *s = d->scratch;

    const bool greedy = temperature <= 0.0f || top_k <= 0;
    TailParams p;
    memset(&p, 0, sizeof(p));
    p.mode = MODE_SAMPLE;
    p.variant = VARIANT_LIBRARY;
    p.rows = vocab_size;
    p.row_base = 0;
    p.vocab = vocab_size;
    p.d = p.ld = 16;
    p.B = 1;
    p.max_k = greedy ? 1 : (top_k > vocab_size ? vocab_size : top_k);
    const int grid = plan_launch(p, d->num_sms, 64);
    if (grid < 1)
        return set_error(LAL_TAIL_ERR_UNSUPPORTED, "sample_token_noalloc: shape unsupported");

    /* the per-call scalars, through the stream into the scratch (a pageable
     * source is staged by the driver before the call returns) */
    struct {
        float t;
        int k;
        float pen;
        float u;
        int hn;
        int head;
    } hp = {temperature, top_k, rep_penalty, u, n_recent, 0};
    NA_CU(cudaMemcpyAsync(s + kNaParams, &hp, sizeof(hp), cudaMemcpyHostToDevice, st));

    p.logits = d_logits; /* penalised in place, as the reference does */
    p.temperature = reinterpret_cast<const float *>(s + kNaParams + 0);
    p.top_k = reinterpret_cast<const int *>(s + kNaParams + 1);
    p.rep_penalty = reinterpret_cast<const float *>(s + kNaParams + 2);
    p.u = reinterpret_cast<const float *>(s + kNaParams + 3);
    p.hist_n = reinterpret_cast<int *>(s + kNaParams + 4);
    p.hist_head = reinterpret_cast<int *>(s + kNaParams + 5);
    p.hist_ids = const_cast<int *>(d_recent);
    p.hist_cap = n_recent;
    p.push_history = 0;
    p.tokens = reinterpret_cast<int *>(s + kNaStatus + 1);
    p.diag = reinterpret_cast<StreamDiag *>(s + kNaDiag);
    p.ghist = s;
    p.gbar = s + kNaBar;
    p.gcount = s + kNaBar + 2;
    p.counter = s + kNaBar + 3;
    p.gL = s + kNaBar + 4;
    p.gmax = s + kNaMax;
    p.gslot_n = s + kNaSlotN;
    p.gcand_key = s + kNaKeys;
    p.gcand_idx = reinterpret_cast<int *>(s + kNaIdx);
    p.gcand_cap = kNaMaxVocab;
    p.status = reinterpret_cast<int *>(s + kNaStatus);
    p.expf_x = d->expf;
    p.expf_y = d->expf + kNaExpfY;
    p.expf_n = d->expf_n;
    p.expf_bits = d->expf + kNaExpfBits;
    p.expf_off = d->expf + kNaExpfOff;
    p.local_edges = use_local_edges(effective_k(temperature, top_k, vocab_size, vocab_size),
                                    p.rows_per_cta_max);
    NA_CU(launch_sample_prepared(p, grid, st));

    int res[2] = {0, -1}; /* status, token */
    NA_CU(cudaMemcpyAsync(res, s + kNaStatus, sizeof(res), cudaMemcpyDeviceToHost, st));
    NA_CU(cudaStreamSynchronize(st));
    if (res[0] != 0) {
        NA_CU(cudaMemsetAsync(s, 0, 4ull * kNaParams, st));
        NA_CU(cudaStreamSynchronize(st));
        return set_error(res[0], res[0] == LAL_TAIL_ERR_TIMEOUT
                                     ? "sample_token_noalloc: bounded device wait expired"
                                     : "sample_token_noalloc: candidate set above capacity");
    }
    *token_out = res[1];
    return LAL_TAIL_OK;
}
