// C ABI of the B200 sampler: contexts, argument checks, host-buffer staging,
// the reference RNG and the reference-convention single-row / row-sequence
// calls.  All sampling goes through the CUDA kernel in bm_kernel.cu; there is
// no host fallback.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "bm_kernel.cuh"
#include "bm_lmhead.cuh"
#include "bm_sampler.h"

struct bm_ctx {
    int device;
    int sms;
    size_t smem_optin;
    int max_vocab;
    cudaStream_t stream;
    int *d_err;
    // staging for the host-buffer entry points (grown on demand)
    float *d_logits;
    size_t cap_logits;
    int32_t *d_hist;
    size_t cap_hist;
    int64_t *d_off;
    size_t cap_off;
    bm_knobs_t *d_knobs;
    size_t cap_knobs;
    float *d_u;
    int32_t *d_id;
    float *d_prob;
    bm_row_stats_t *d_stats;
    size_t cap_rows;
    // lm_head: normalised bf16 hidden states and the logits of the fused call
    uint16_t *d_a;
    size_t cap_a;
    float *d_lm;
    size_t cap_lm;
    int lm_ready;
    // ternary lm_head: int8 activations and per-row output scales
    int8_t *d_q;
    size_t cap_q;
    float *d_isc;
    size_t cap_isc;
    // fused lm_head + sampler: the rows' history bits, the GEMM's per-tile
    // lists, the fallback row lists and the gathered activations of the rows
    // whose lists cannot decide them
    uint32_t *d_pb;
    size_t cap_pb;
    uint64_t *d_summ;
    size_t cap_summ;
    int *d_fb;
    size_t cap_fb;
    int *d_nl;
    size_t cap_nl;
    unsigned char *d_a2;
    size_t cap_a2;
    float *d_isc2;
    size_t cap_isc2;
    int sum_ready;
    // small host-buffer calls: one pinned host region and its device mirror,
    // laid out [words | outputs | inputs]; uploaded whole, [words | outputs]
    // read back (one copy each way, one synchronisation)
    unsigned char *h_stage;
    unsigned char *d_stage;
    size_t cap_stage;
};

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    int code = (e == cudaErrorMemoryAllocation) ? BM_ERR_OOM : BM_ERR_CUDA;
    return fail(code, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call)                                             \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);  \
    } while (0)

template <class T>
int grow(T **p, size_t *cap, size_t need) {
    if (need <= *cap) return BM_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    size_t n = need + need / 4 + 16;
    cudaError_t e = cudaMalloc(reinterpret_cast<void **>(p), n * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(staging)");
    *cap = n;
    return BM_OK;
}

int check_args(int max_vocab, const void *logits, int B, int V, int64_t ld, const void *hist,
               const void *off, const void *knobs, int64_t knob_stride, const void *uniform,
               const void *out_id) {
    if (B < 0) return fail(BM_ERR_INVALID_ARG, "B = %d < 0", B);
    if (B == 0) return BM_OK;
    if (V < 1) return fail(BM_ERR_INVALID_ARG, "V = %d < 1", V);
    if (V > max_vocab)
        return fail(BM_ERR_UNSUPPORTED, "V = %d exceeds the row buffer limit %d", V,
                    max_vocab);
    if (ld < V) return fail(BM_ERR_INVALID_ARG, "ld = %lld < V = %d", (long long)ld, V);
    if (!logits || !knobs || !out_id)
        return fail(BM_ERR_INVALID_ARG, "logits, knobs and out_id must be non-NULL");
    if (!uniform) return fail(BM_ERR_INVALID_ARG, "uniform must be non-NULL");
    if ((hist == nullptr) != (off == nullptr))
        return fail(BM_ERR_INVALID_ARG, "hist and hist_off must both be NULL or both set");
    if (knob_stride != 0 && knob_stride != 1)
        return fail(BM_ERR_INVALID_ARG, "knob_stride must be 0 or 1");
    if (reinterpret_cast<uintptr_t>(logits) % 4)
        return fail(BM_ERR_INVALID_ARG, "logits not 4-byte aligned");
    return BM_OK;
}

int check_batch_args(const bm_ctx_t *ctx, const void *logits, int B, int V, int64_t ld,
                     const void *hist, const void *off, const void *knobs,
                     int64_t knob_stride, const void *uniform, const void *out_id) {
    if (!ctx) return fail(BM_ERR_INVALID_ARG, "ctx is NULL");
    return check_args(ctx->max_vocab, logits, B, V, ld, hist, off, knobs, knob_stride, uniform,
                      out_id);
}

// The sampler's grid: one CTA per SM, never more CTAs than rows.
int launch_grid(int B, int sms) { return B < sms ? B : sms; }

// The fused lm_head + sampler on activations A ([B x d]: bf16, or int8 with
// per-row output scales isc) and weights W ([V x d]), on stream s:
//   1. the rows' history bits (penalty), when there are histories;
//   2. the GEMM with the summary epilogue: per row and 128 columns the KS
//      best penalised, scaled logits (greedy and top_k rows), or the row's
//      logits (rows of the full-vocabulary path);
//   3. the merge kernel: greedy and top_k rows resolved from the lists; the
//      rest appended to the fallback lists (fb: to sample; nl: logits
//      missing, the rows whose lists could not decide them);
//   4. the nl rows' activations gathered and their logits computed (a GEMM
//      of those rows only; its row count is read on the device);
//   5. the sampler on the fb rows (row count and row map read on the device).
// Steps 4-5 find empty lists in the common case and return at once.  No
// logits cross HBM for rows the lists decide, and nothing here waits for the
// host.
int fused_sample(bm_ctx_t *c, bool i8, const void *A, const float *isc, const void *W, int B,
                 int d, int V, const int32_t *d_hist, const int64_t *d_hist_off,
                 const bm_knobs_t *d_knobs, int64_t knob_stride, const float *d_uniform,
                 int32_t *d_out_id, float *d_out_prob, bm_row_stats_t *d_stats, cudaStream_t s) {
    const int lists = bml::summary_lists(V);
    const int pw = (V + 31) / 32;
    const int64_t ld = ((int64_t)V + 3) / 4 * 4;  // 16-byte rows for the GEMM's stores
    const size_t esz = i8 ? 1 : 2;
    int rc;
    if ((rc = grow(&c->d_summ, &c->cap_summ, (size_t)B * lists * bml::KS)) != BM_OK) return rc;
    if (d_hist && (rc = grow(&c->d_pb, &c->cap_pb, (size_t)B * pw)) != BM_OK) return rc;
    if ((rc = grow(&c->d_fb, &c->cap_fb, (size_t)B + 1)) != BM_OK) return rc;
    if ((rc = grow(&c->d_nl, &c->cap_nl, (size_t)B + 1)) != BM_OK) return rc;
    if ((rc = grow(&c->d_lm, &c->cap_lm, (size_t)B * (size_t)ld)) != BM_OK) return rc;
    if ((rc = grow(&c->d_a2, &c->cap_a2, (size_t)B * d * esz)) != BM_OK) return rc;
    if (i8 && (rc = grow(&c->d_isc2, &c->cap_isc2, (size_t)B)) != BM_OK) return rc;
    if (!c->sum_ready) {
        CK(bmk::prepare_summary(c->max_vocab, bml::summary_lists(c->max_vocab), bml::KS));
        c->sum_ready = 1;
    }
    if (d_hist) CK(bml::penalty_bits(d_hist, d_hist_off, B, V, c->d_pb, pw, s));
    bml::SumArgs sg;
    sg.pbits = d_hist ? c->d_pb : nullptr;
    sg.pw = pw;
    sg.knobs = d_knobs;
    sg.knob_stride = knob_stride;
    sg.summ = c->d_summ;
    if (i8)
        CK(bml::gemm_i8_summary(static_cast<const int8_t *>(A), static_cast<const int8_t *>(W), B,
                                V, d, isc, sg, c->d_lm, ld, c->d_err, s));
    else
        CK(bml::gemm_bf16_summary(static_cast<const uint16_t *>(A),
                                  static_cast<const uint16_t *>(W), B, V, d, sg, c->d_lm, ld,
                                  c->d_err, s));
    CK(cudaMemsetAsync(c->d_fb, 0, sizeof(int), s));
    CK(cudaMemsetAsync(c->d_nl, 0, sizeof(int), s));
    bmk::SumParams sp;
    sp.summ = c->d_summ;
    sp.tiles = lists;
    sp.ks = bml::KS;
    sp.B = B;
    sp.V = V;
    sp.knobs = d_knobs;
    sp.knob_stride = knob_stride;
    sp.uniform = d_uniform;
    sp.out_id = d_out_id;
    sp.out_prob = d_out_prob;
    sp.stats = d_stats;
    sp.fb = c->d_fb;
    sp.nl = c->d_nl;
    sp.err = c->d_err;
    const int mgrid = bmk::MERGE_CTAS_PER_SM * c->sms;
    CK(bmk::launch_summary(sp, B < mgrid ? B : mgrid, s));
    CK(bml::gather_rows(A, (int64_t)d * (int64_t)esz, c->d_nl, c->d_a2, isc, c->d_isc2, B, s));
    if (i8)
        CK(bml::gemm_i8(reinterpret_cast<const int8_t *>(c->d_a2),
                        static_cast<const int8_t *>(W), B, V, d, c->d_isc2, c->d_lm, ld, c->d_err,
                        s, c->d_nl, c->d_nl + 1));
    else
        CK(bml::gemm_bf16(reinterpret_cast<const uint16_t *>(c->d_a2),
                          static_cast<const uint16_t *>(W), B, V, d, c->d_lm, ld, c->d_err, s,
                          c->d_nl, c->d_nl + 1));
    bmk::Params p;
    p.logits = c->d_lm;
    p.ld = ld;
    p.B = B;
    p.V = V;
    p.hist = d_hist;
    p.hist_off = d_hist_off;
    p.knobs = d_knobs;
    p.knob_stride = knob_stride;
    p.uniform = d_uniform;
    p.out_id = d_out_id;
    p.out_prob = d_out_prob;
    p.stats = d_stats;
    p.err = c->d_err;
    p.sched = c->d_err + 1;
    p.dB = c->d_fb;
    p.row_map = c->d_fb + 1;
    CK(bmk::launch(p, launch_grid(B, c->sms), s));
    return BM_OK;
}

// Per-device state of the allocation-free entry point: the scratch address
// and the launch shape, set up once.
constexpr int NOALLOC_MAXDEV = 64;
constexpr int NOALLOC_MAX_ROWS = 1 << 30;  // keeps the row counter inside int
struct NoallocDev {
    int ready;
    int sms;
    int max_vocab;
    int *scratch;
};
NoallocDev g_noalloc[NOALLOC_MAXDEV];
std::mutex g_noalloc_mu;

int noalloc_setup(int dev, const NoallocDev **out) {
    if (dev < 0 || dev >= NOALLOC_MAXDEV)
        return fail(BM_ERR_UNSUPPORTED, "device %d beyond the %d devices supported", dev,
                    NOALLOC_MAXDEV);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoallocDev &d = g_noalloc[dev];
    if (!d.ready) {
        int major = 0, sms = 0, optin = 0;
        CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10)
            return fail(BM_ERR_NO_DEVICE, "device %d is sm_%dx; this library is built for sm_100a",
                        dev, major);
        CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        int *scratch = nullptr;
        CK(bmk::noalloc_scratch(&scratch));
        const int mv = bmk::max_vocab((size_t)optin);
        CK(bmk::prepare(mv));
        d.sms = sms;
        d.max_vocab = mv;
        d.scratch = scratch;
        d.ready = 1;
    }
    *out = &d;
    return BM_OK;
}

}  // namespace

extern "C" {

const char *bm_last_error(void) { return g_err; }
int bm_abi_version(void) { return BM_SAMPLER_ABI_VERSION; }

int bm_knobs_init(bm_knobs_t *k, float temp, float penalty, float min_p, float top_p,
                  int top_k) {
    if (!k) return fail(BM_ERR_INVALID_ARG, "knobs is NULL");
    k->temp = temp;
    k->penalty = penalty;
    k->min_p = min_p;
    k->top_p = top_p;
    k->top_k = top_k;
    // IEEE division and the host libm's logf, as src/model.c:157 and :173
    volatile float one = 1.0f;
    k->inv_temp = one / temp;
    k->log_min_p = (min_p > 0.0f && min_p < 1.0f) ? logf(min_p) : 0.0f;
    k->flags = 0;
    return BM_OK;
}

int bm_ctx_create(int device, bm_ctx_t **out) {
    if (!out) return fail(BM_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return fail(BM_ERR_NO_DEVICE, "no CUDA device (%s)",
                    e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
    if (device < 0 || device >= n)
        return fail(BM_ERR_NO_DEVICE, "device %d out of range (%d devices)", device, n);
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(BM_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a",
                    device, prop.major, prop.minor);
    CK(cudaSetDevice(device));
    bm_ctx_t *c = static_cast<bm_ctx_t *>(calloc(1, sizeof(bm_ctx_t)));
    if (!c) return fail(BM_ERR_OOM, "host allocation failed");
    c->device = device;
    c->sms = prop.multiProcessorCount;
    c->smem_optin = prop.sharedMemPerBlockOptin;
    c->max_vocab = bmk::max_vocab(c->smem_optin);
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    // error word and the two row-schedule counters
    if (e == cudaSuccess) e = cudaMalloc(&c->d_err, 4 * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, 4 * sizeof(int));
    if (e == cudaSuccess) e = bmk::prepare(c->max_vocab);
    if (e != cudaSuccess) {
        int rc = cuda_fail(e, "context setup");
        bm_ctx_destroy(c);
        return rc;
    }
    *out = c;
    return BM_OK;
}

void bm_ctx_destroy(bm_ctx_t *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    cudaFree(c->d_err);
    cudaFree(c->d_logits);
    cudaFree(c->d_hist);
    cudaFree(c->d_off);
    cudaFree(c->d_knobs);
    cudaFree(c->d_u);
    cudaFree(c->d_id);
    cudaFree(c->d_prob);
    cudaFree(c->d_stats);
    cudaFree(c->d_a);
    cudaFree(c->d_lm);
    cudaFree(c->d_q);
    cudaFree(c->d_isc);
    cudaFree(c->d_stage);
    cudaFree(c->d_pb);
    cudaFree(c->d_summ);
    cudaFree(c->d_fb);
    cudaFree(c->d_nl);
    cudaFree(c->d_a2);
    cudaFree(c->d_isc2);
    if (c->h_stage) cudaFreeHost(c->h_stage);
    if (c->stream) cudaStreamDestroy(c->stream);
    free(c);
}

int bm_max_vocab(const bm_ctx_t *c) { return c ? c->max_vocab : 0; }

void *bm_ctx_stream(bm_ctx_t *c) { return c ? static_cast<void *>(c->stream) : nullptr; }

int bm_ctx_device(const bm_ctx_t *c, int *device) {
    if (!c || !device) return fail(BM_ERR_INVALID_ARG, "ctx or device is NULL");
    *device = c->device;
    return BM_OK;
}

int bm_ctx_check(bm_ctx_t *c) {
    if (!c) return fail(BM_ERR_INVALID_ARG, "ctx is NULL");
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    int h = 0;
    CK(cudaMemcpy(&h, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        // a CTA that stopped early may leave the schedule counters behind
        CK(cudaMemset(c->d_err, 0, 4 * sizeof(int)));
        return fail(BM_ERR_DEVICE, "device error flag 0x%x (bounded wait expired or select "
                                   "did not converge)", h);
    }
    return BM_OK;
}

int bm_sample_batch(bm_ctx_t *c, const float *d_logits, int B, int V, int64_t ld,
                    const int32_t *d_hist, const int64_t *d_hist_off,
                    const bm_knobs_t *d_knobs, int64_t knob_stride, const float *d_uniform,
                    int32_t *d_out_id, float *d_out_prob, bm_row_stats_t *d_stats,
                    void *stream) {
    int rc = check_batch_args(c, d_logits, B, V, ld, d_hist, d_hist_off, d_knobs, knob_stride,
                              d_uniform, d_out_id);
    if (rc != BM_OK || B == 0) return rc;
    CK(cudaSetDevice(c->device));
    bmk::Params p;
    p.logits = d_logits;
    p.ld = ld;
    p.B = B;
    p.V = V;
    p.hist = d_hist;
    p.hist_off = d_hist_off;
    p.knobs = d_knobs;
    p.knob_stride = knob_stride;
    p.uniform = d_uniform;
    p.out_id = d_out_id;
    p.out_prob = d_out_prob;
    p.stats = d_stats;
    p.err = c->d_err;
    p.sched = c->d_err + 1;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    int grid = B < c->sms ? B : c->sms;
    CK(bmk::launch(p, grid, s));
    return BM_OK;
}

int bm_lmhead_logits(bm_ctx_t *c, const float *d_hidden, int B, int d_model,
                     const float *d_norm_w, const uint16_t *d_W, int V, float *d_logits,
                     int64_t ld, void *stream) {
    if (!c) return fail(BM_ERR_INVALID_ARG, "ctx is NULL");
    if (B < 0 || V < 1 || ld < V)
        return fail(BM_ERR_INVALID_ARG, "B = %d, V = %d, ld = %lld", B, V, (long long)ld);
    if (B == 0) return BM_OK;
    if (!d_hidden || !d_norm_w || !d_W || !d_logits)
        return fail(BM_ERR_INVALID_ARG, "hidden, norm weight, W and logits must be non-NULL");
    if (d_model <= 0 || d_model % 8 || d_model > 4096)
        return fail(BM_ERR_UNSUPPORTED, "d_model = %d (needs a multiple of 8, <= 4096)", d_model);
    if ((reinterpret_cast<uintptr_t>(d_W) & 15) || (reinterpret_cast<uintptr_t>(d_hidden) & 15) ||
        (reinterpret_cast<uintptr_t>(d_norm_w) & 15) || (reinterpret_cast<uintptr_t>(d_logits) & 3))
        return fail(BM_ERR_INVALID_ARG,
                    "W / hidden / norm weight not 16-byte or logits not 4-byte aligned");
    if ((V + 255) / 256 > 65535) return fail(BM_ERR_UNSUPPORTED, "V = %d too large", V);
    CK(cudaSetDevice(c->device));
    if (!c->lm_ready) {
        CK(bml::prepare());
        c->lm_ready = 1;
    }
    int rc = grow(&c->d_a, &c->cap_a, (size_t)B * d_model);
    if (rc != BM_OK) return rc;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    CK(bml::rmsnorm_bf16(d_hidden, B, d_model, d_norm_w, c->d_a, s));
    CK(bml::gemm_bf16(c->d_a, d_W, B, V, d_model, d_logits, ld, c->d_err, s));
    return BM_OK;
}

int bm_lmhead_sample_batch(bm_ctx_t *c, const float *d_hidden, int B, int d_model,
                           const float *d_norm_w, const uint16_t *d_W, int V,
                           const int32_t *d_hist, const int64_t *d_hist_off,
                           const bm_knobs_t *d_knobs, int64_t knob_stride, const float *d_uniform,
                           int32_t *d_out_id, float *d_out_prob, bm_row_stats_t *d_stats,
                           void *stream) {
    if (!c) return fail(BM_ERR_INVALID_ARG, "ctx is NULL");
    // the sampler's checks first (the hidden states stand in for the logits)
    const int64_t ld = ((int64_t)V + 3) / 4 * 4;
    int rc = check_batch_args(c, d_hidden, B, V, ld, d_hist, d_hist_off, d_knobs, knob_stride,
                              d_uniform, d_out_id);
    if (rc != BM_OK || B == 0) return rc;
    if (!d_norm_w || !d_W)
        return fail(BM_ERR_INVALID_ARG, "hidden, norm weight and W must be non-NULL");
    if (d_model <= 0 || d_model % 8 || d_model > 4096)
        return fail(BM_ERR_UNSUPPORTED, "d_model = %d (needs a multiple of 8, <= 4096)", d_model);
    if ((reinterpret_cast<uintptr_t>(d_W) & 15) || (reinterpret_cast<uintptr_t>(d_hidden) & 15) ||
        (reinterpret_cast<uintptr_t>(d_norm_w) & 15))
        return fail(BM_ERR_INVALID_ARG, "W / hidden / norm weight not 16-byte aligned");
    CK(cudaSetDevice(c->device));
    if (!c->lm_ready) {
        CK(bml::prepare());
        c->lm_ready = 1;
    }
    if ((rc = grow(&c->d_a, &c->cap_a, (size_t)B * d_model)) != BM_OK) return rc;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    CK(bml::rmsnorm_bf16(d_hidden, B, d_model, d_norm_w, c->d_a, s));
    return fused_sample(c, false, c->d_a, nullptr, d_W, B, d_model, V, d_hist, d_hist_off, d_knobs,
                        knob_stride, d_uniform, d_out_id, d_out_prob, d_stats, s);
}

int bm_fused_fallback_rows(bm_ctx_t *c, int *n_sampled, int *n_computed) {
    if (!c || !n_sampled || !n_computed) return fail(BM_ERR_INVALID_ARG, "NULL argument");
    *n_sampled = *n_computed = 0;
    if (!c->d_fb) return BM_OK;
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(n_sampled, c->d_fb, sizeof(int), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(n_computed, c->d_nl, sizeof(int), cudaMemcpyDeviceToHost));
    return BM_OK;
}

int bm_ternary_unpack(bm_ctx_t *c, const uint8_t *d_packed, int V, int d_model, int8_t *d_w8,
                      void *stream) {
    if (!c) return fail(BM_ERR_INVALID_ARG, "ctx is NULL");
    if (V < 1 || !d_packed || !d_w8)
        return fail(BM_ERR_INVALID_ARG, "V = %d, packed and w8 must be non-NULL", V);
    if (d_model <= 0 || d_model % 32 || d_model > 4096)
        return fail(BM_ERR_UNSUPPORTED, "d_model = %d (needs a multiple of 32, <= 4096)", d_model);
    if ((reinterpret_cast<uintptr_t>(d_packed) & 3) || (reinterpret_cast<uintptr_t>(d_w8) & 15))
        return fail(BM_ERR_INVALID_ARG, "packed not 4-byte or w8 not 16-byte aligned");
    CK(cudaSetDevice(c->device));
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    CK(bml::ternary_unpack(d_packed, V, d_model, d_w8, s));
    return BM_OK;
}

int bm_ternary_logits(bm_ctx_t *c, const float *d_hidden, int B, int d_model,
                      const float *d_norm_f, const float *d_lmh_norm, const int8_t *d_w8,
                      float w_scale, int V, float *d_logits, int64_t ld, void *stream) {
    if (!c) return fail(BM_ERR_INVALID_ARG, "ctx is NULL");
    if (B < 0 || V < 1 || ld < V)
        return fail(BM_ERR_INVALID_ARG, "B = %d, V = %d, ld = %lld", B, V, (long long)ld);
    if (B == 0) return BM_OK;
    if (!d_hidden || !d_lmh_norm || !d_w8 || !d_logits)
        return fail(BM_ERR_INVALID_ARG, "hidden, lm_head norm, w8 and logits must be non-NULL");
    if (d_model <= 0 || d_model % 32 || d_model > 4096)
        return fail(BM_ERR_UNSUPPORTED, "d_model = %d (needs a multiple of 32, <= 4096)", d_model);
    if ((reinterpret_cast<uintptr_t>(d_w8) & 15) || (reinterpret_cast<uintptr_t>(d_hidden) & 15) ||
        (reinterpret_cast<uintptr_t>(d_lmh_norm) & 15) ||
        (d_norm_f && (reinterpret_cast<uintptr_t>(d_norm_f) & 15)) ||
        (reinterpret_cast<uintptr_t>(d_logits) & 3))
        return fail(BM_ERR_INVALID_ARG,
                    "w8 / hidden / norm weights not 16-byte or logits not 4-byte aligned");
    if (!(w_scale == w_scale)) return fail(BM_ERR_INVALID_ARG, "w_scale is NaN");
    CK(cudaSetDevice(c->device));
    if (!c->lm_ready) {
        CK(bml::prepare());
        c->lm_ready = 1;
    }
    int rc = grow(&c->d_q, &c->cap_q, (size_t)B * d_model);
    if (rc != BM_OK) return rc;
    if ((rc = grow(&c->d_isc, &c->cap_isc, (size_t)B)) != BM_OK) return rc;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    CK(bml::ternary_prep(d_hidden, B, d_model, d_norm_f, d_lmh_norm, w_scale, c->d_q, c->d_isc, s));
    CK(bml::gemm_i8(c->d_q, d_w8, B, V, d_model, c->d_isc, d_logits, ld, c->d_err, s));
    return BM_OK;
}

int bm_ternary_sample_batch(bm_ctx_t *c, const float *d_hidden, int B, int d_model,
                            const float *d_norm_f, const float *d_lmh_norm, const int8_t *d_w8,
                            float w_scale, int V, const int32_t *d_hist,
                            const int64_t *d_hist_off, const bm_knobs_t *d_knobs,
                            int64_t knob_stride, const float *d_uniform, int32_t *d_out_id,
                            float *d_out_prob, bm_row_stats_t *d_stats, void *stream) {
    if (!c) return fail(BM_ERR_INVALID_ARG, "ctx is NULL");
    const int64_t ld = ((int64_t)V + 3) / 4 * 4;
    int rc = check_batch_args(c, d_hidden, B, V, ld, d_hist, d_hist_off, d_knobs, knob_stride,
                              d_uniform, d_out_id);
    if (rc != BM_OK || B == 0) return rc;
    if (!d_lmh_norm || !d_w8)
        return fail(BM_ERR_INVALID_ARG, "hidden, lm_head norm and w8 must be non-NULL");
    if (d_model <= 0 || d_model % 32 || d_model > 4096)
        return fail(BM_ERR_UNSUPPORTED, "d_model = %d (needs a multiple of 32, <= 4096)", d_model);
    if ((reinterpret_cast<uintptr_t>(d_w8) & 15) || (reinterpret_cast<uintptr_t>(d_hidden) & 15) ||
        (reinterpret_cast<uintptr_t>(d_lmh_norm) & 15) ||
        (d_norm_f && (reinterpret_cast<uintptr_t>(d_norm_f) & 15)))
        return fail(BM_ERR_INVALID_ARG, "w8 / hidden / norm weights not 16-byte aligned");
    if (!(w_scale == w_scale)) return fail(BM_ERR_INVALID_ARG, "w_scale is NaN");
    CK(cudaSetDevice(c->device));
    if (!c->lm_ready) {
        CK(bml::prepare());
        c->lm_ready = 1;
    }
    if ((rc = grow(&c->d_q, &c->cap_q, (size_t)B * d_model)) != BM_OK) return rc;
    if ((rc = grow(&c->d_isc, &c->cap_isc, (size_t)B)) != BM_OK) return rc;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    CK(bml::ternary_prep(d_hidden, B, d_model, d_norm_f, d_lmh_norm, w_scale, c->d_q, c->d_isc, s));
    return fused_sample(c, true, c->d_q, c->d_isc, d_w8, B, d_model, V, d_hist, d_hist_off,
                        d_knobs, knob_stride, d_uniform, d_out_id, d_out_prob, d_stats, s);
}

int bm_sample_batch_noalloc(const float *d_logits, int B, int V, int64_t ld,
                            const int32_t *d_hist, const int64_t *d_hist_off,
                            const bm_knobs_t *d_knobs, int64_t knob_stride,
                            const float *d_uniform, int32_t *d_out_id, float *d_out_prob,
                            bm_row_stats_t *d_stats, void *stream) {
    if (B > NOALLOC_MAX_ROWS)
        return fail(BM_ERR_INVALID_ARG, "B = %d exceeds %d rows per call", B, NOALLOC_MAX_ROWS);
    int dev = 0;
    CK(cudaGetDevice(&dev));
    const NoallocDev *d = nullptr;
    int rc = noalloc_setup(dev, &d);
    if (rc != BM_OK) return rc;
    rc = check_args(d->max_vocab, d_logits, B, V, ld, d_hist, d_hist_off, d_knobs, knob_stride,
                    d_uniform, d_out_id);
    if (rc != BM_OK || B == 0) return rc;
    bmk::Params p;
    p.logits = d_logits;
    p.ld = ld;
    p.B = B;
    p.V = V;
    p.hist = d_hist;
    p.hist_off = d_hist_off;
    p.knobs = d_knobs;
    p.knob_stride = knob_stride;
    p.uniform = d_uniform;
    p.out_id = d_out_id;
    p.out_prob = d_out_prob;
    p.stats = d_stats;
    p.err = d->scratch;
    p.sched = d->scratch + 1;
    p.mark_failed_rows = 1;
    const int grid = B < d->sms ? B : d->sms;
    CK(bmk::launch(p, grid, static_cast<cudaStream_t>(stream)));
    return BM_OK;
}

namespace {

// Host-buffer calls whose staged bytes fit STAGE_MAX (B = 1 is 201 KB at
// V = 50257): every input is packed into one pinned host region together with
// a zeroed error / row-schedule word group for the launch, uploaded with one
// copy, and the word group and outputs come back with one copy, so a call
// costs two copies, one launch and one synchronisation instead of a copy per
// buffer (pageable copies each wait for the host) and a separate read of the
// context's error word.
constexpr size_t STAGE_MAX = size_t(16) << 20;
constexpr size_t r16h(size_t x) { return (x + 15) & ~size_t(15); }

// Byte offsets of the staging region's sections (16-byte aligned):
// [logits | knobs | uniforms | history ids | history offsets | words 16 B |
//  ids | probabilities | stats].  The upload is [0, o_w + 16): the inputs and
// the zeroed words; the read-back is [o_w, total): the words and the outputs.
struct StageLayout {
    size_t o_log, o_kn, o_u, o_h, o_off, o_w, o_id, o_prob, o_st, total;
};
StageLayout stage_layout(size_t rows, int64_t ld, size_t nk, int64_t h1, bool hist) {
    StageLayout L;
    L.o_log = 0;
    L.o_kn = L.o_log + r16h(rows * (size_t)ld * sizeof(float));
    L.o_u = L.o_kn + r16h(nk * sizeof(bm_knobs_t));
    L.o_h = L.o_u + r16h(rows * sizeof(float));
    L.o_off = L.o_h + (hist ? r16h((size_t)h1 * sizeof(int32_t)) : 0);
    L.o_w = L.o_off + (hist ? r16h((rows + 1) * sizeof(int64_t)) : 0);
    L.o_id = L.o_w + 16;
    L.o_prob = L.o_id + r16h(rows * sizeof(int32_t));
    L.o_st = L.o_prob + r16h(rows * sizeof(float));
    L.total = L.o_st + r16h(rows * sizeof(bm_row_stats_t));
    return L;
}

int sample_host_small(bm_ctx_t *c, const float *h_logits, int B, int V, int64_t ld,
                      const int32_t *h_hist, const int64_t *h_hist_off,
                      const bm_knobs_t *h_knobs, int64_t knob_stride, const float *h_uniform,
                      int32_t *h_out_id, float *h_out_prob, bm_row_stats_t *h_stats,
                      size_t nk, int64_t h1, const StageLayout &L) {
    const size_t rows = (size_t)B;
    const size_t o_id = L.o_id, o_prob = L.o_prob, o_st = L.o_st, o_w = L.o_w;
    const size_t o_log = L.o_log, o_kn = L.o_kn, o_u = L.o_u, o_h = L.o_h, o_off = L.o_off;
    const size_t total = L.total;
    cudaStream_t s = c->stream;
    if (total > c->cap_stage) {
        CK(cudaStreamSynchronize(s));
        cudaFree(c->d_stage);
        if (c->h_stage) cudaFreeHost(c->h_stage);
        c->d_stage = nullptr;
        c->h_stage = nullptr;
        c->cap_stage = 0;
        const size_t n = total + total / 4 + 256;
        cudaError_t e = cudaMalloc(reinterpret_cast<void **>(&c->d_stage), n);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(small staging)");
        e = cudaHostAlloc(reinterpret_cast<void **>(&c->h_stage), n, cudaHostAllocDefault);
        if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(small staging)");
        c->cap_stage = n;
    }
    // (every call leaves the stream idle, so no copy still reads the region)
    unsigned char *h = c->h_stage, *d = c->d_stage;
    memset(h + o_w, 0, 16);  // error word and the two row-schedule counters
    memcpy(h + o_log, h_logits, rows * (size_t)ld * sizeof(float));
    memcpy(h + o_kn, h_knobs, nk * sizeof(bm_knobs_t));
    memcpy(h + o_u, h_uniform, rows * sizeof(float));
    if (h_hist) {
        if (h1 > 0) memcpy(h + o_h, h_hist, (size_t)h1 * sizeof(int32_t));
        memcpy(h + o_off, h_hist_off, (rows + 1) * sizeof(int64_t));
    }
    CK(cudaMemcpyAsync(d, h, o_w + 16, cudaMemcpyHostToDevice, s));
    bmk::Params p;
    p.logits = reinterpret_cast<const float *>(d + o_log);
    p.ld = ld;
    p.B = B;
    p.V = V;
    p.hist = h_hist ? reinterpret_cast<const int32_t *>(d + o_h) : nullptr;
    p.hist_off = h_hist ? reinterpret_cast<const int64_t *>(d + o_off) : nullptr;
    p.knobs = reinterpret_cast<const bm_knobs_t *>(d + o_kn);
    p.knob_stride = knob_stride;
    p.uniform = reinterpret_cast<const float *>(d + o_u);
    p.out_id = reinterpret_cast<int32_t *>(d + o_id);
    p.out_prob = h_out_prob ? reinterpret_cast<float *>(d + o_prob) : nullptr;
    p.stats = h_stats ? reinterpret_cast<bm_row_stats_t *>(d + o_st) : nullptr;
    p.err = reinterpret_cast<int *>(d + o_w);
    p.sched = reinterpret_cast<int *>(d + o_w) + 1;
    const int grid = B < c->sms ? B : c->sms;
    cudaError_t e = bmk::launch(p, grid, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h + o_w, d + o_w, total - o_w, cudaMemcpyDeviceToHost, s);
    // synchronise on the failure path too: the upload may still read the region
    const cudaError_t es = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "small host-buffer call");
    if (es != cudaSuccess) return cuda_fail(es, "cudaStreamSynchronize");
    int err = 0;
    memcpy(&err, h + o_w, sizeof(int));
    if (err)
        return fail(BM_ERR_DEVICE, "device error flag 0x%x (bounded wait expired or select "
                                   "did not converge)", err);
    memcpy(h_out_id, h + o_id, rows * sizeof(int32_t));
    if (h_out_prob) memcpy(h_out_prob, h + o_prob, rows * sizeof(float));
    if (h_stats) memcpy(h_stats, h + o_st, rows * sizeof(bm_row_stats_t));
    return BM_OK;
}

}  // namespace

int bm_sample_batch_host(bm_ctx_t *c, const float *h_logits, int B, int V, int64_t ld,
                         const int32_t *h_hist, const int64_t *h_hist_off,
                         const bm_knobs_t *h_knobs, int64_t knob_stride,
                         const float *h_uniform, int32_t *h_out_id, float *h_out_prob,
                         bm_row_stats_t *h_stats) {
    int rc = check_batch_args(c, h_logits, B, V, ld, h_hist, h_hist_off, h_knobs, knob_stride,
                              h_uniform, h_out_id);
    if (rc != BM_OK || B == 0) return rc;
    CK(cudaSetDevice(c->device));
    cudaStream_t s = c->stream;
    const size_t rows = (size_t)B;
    {
        const size_t nk = knob_stride ? rows : 1;
        int64_t h1 = 0;
        if (h_hist) {
            const int64_t h0 = h_hist_off[0];
            h1 = h_hist_off[B];
            if (h0 < 0 || h1 < h0) return fail(BM_ERR_INVALID_ARG, "hist_off not monotone");
        }
        const StageLayout L = stage_layout(rows, ld, nk, h1, h_hist != nullptr);
        if (L.total <= STAGE_MAX)
            return sample_host_small(c, h_logits, B, V, ld, h_hist, h_hist_off, h_knobs,
                                     knob_stride, h_uniform, h_out_id, h_out_prob, h_stats, nk,
                                     h1, L);
    }
    if ((rc = grow(&c->d_logits, &c->cap_logits, rows * (size_t)ld)) != BM_OK) return rc;
    if (rows > c->cap_rows) {
        // the four per-row buffers share one capacity
        cudaFree(c->d_u); cudaFree(c->d_id); cudaFree(c->d_prob); cudaFree(c->d_stats);
        c->d_u = nullptr; c->d_id = nullptr; c->d_prob = nullptr; c->d_stats = nullptr;
        c->cap_rows = 0;
        size_t t0 = 0, t1 = 0, t2 = 0, t3 = 0;
        if ((rc = grow(&c->d_u, &t0, rows)) != BM_OK) return rc;
        if ((rc = grow(&c->d_id, &t1, rows)) != BM_OK) return rc;
        if ((rc = grow(&c->d_prob, &t2, rows)) != BM_OK) return rc;
        if ((rc = grow(&c->d_stats, &t3, rows)) != BM_OK) return rc;
        c->cap_rows = t0;
    }
    const size_t nk = knob_stride ? rows : 1;
    if ((rc = grow(&c->d_knobs, &c->cap_knobs, nk)) != BM_OK) return rc;
    CK(cudaMemcpyAsync(c->d_logits, h_logits, rows * (size_t)ld * sizeof(float),
                       cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(c->d_knobs, h_knobs, nk * sizeof(bm_knobs_t), cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(c->d_u, h_uniform, rows * sizeof(float), cudaMemcpyHostToDevice, s));
    const int32_t *dh = nullptr;
    const int64_t *doff = nullptr;
    if (h_hist) {
        const int64_t h0 = h_hist_off[0], h1 = h_hist_off[B];
        if (h0 < 0 || h1 < h0) return fail(BM_ERR_INVALID_ARG, "hist_off not monotone");
        if ((rc = grow(&c->d_off, &c->cap_off, rows + 1)) != BM_OK) return rc;
        if ((rc = grow(&c->d_hist, &c->cap_hist, (size_t)(h1 > 0 ? h1 : 1))) != BM_OK) return rc;
        if (h1 > 0)
            CK(cudaMemcpyAsync(c->d_hist, h_hist, (size_t)h1 * sizeof(int32_t),
                               cudaMemcpyHostToDevice, s));
        CK(cudaMemcpyAsync(c->d_off, h_hist_off, (rows + 1) * sizeof(int64_t),
                           cudaMemcpyHostToDevice, s));
        dh = c->d_hist;
        doff = c->d_off;
    }
    rc = bm_sample_batch(c, c->d_logits, B, V, ld, dh, doff, c->d_knobs, knob_stride, c->d_u,
                         c->d_id, h_out_prob ? c->d_prob : nullptr,
                         h_stats ? c->d_stats : nullptr, s);
    if (rc != BM_OK) return rc;
    CK(cudaMemcpyAsync(h_out_id, c->d_id, rows * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    if (h_out_prob)
        CK(cudaMemcpyAsync(h_out_prob, c->d_prob, rows * sizeof(float), cudaMemcpyDeviceToHost,
                           s));
    if (h_stats)
        CK(cudaMemcpyAsync(h_stats, c->d_stats, rows * sizeof(bm_row_stats_t),
                           cudaMemcpyDeviceToHost, s));
    return bm_ctx_check(c);
}

// ---- reference RNG (src/utils.c:117-140) ---------------------------------
static uint64_t g_rng = 0x853c49e6748fea9bULL;

void bm_rng_seed(uint64_t seed) { g_rng = seed ? seed : 0x853c49e6748fea9bULL; }

uint64_t bm_rng_next(void) {
    uint64_t x = g_rng;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    g_rng = x;
    return x * 0x2545F4914F6CDD1DULL;
}

float bm_rng_float(void) {
    return (float)(bm_rng_next() >> 11) * (1.0f / 9007199254740992.0f);
}

uint64_t bm_rng_get_state(void) { return g_rng; }
void bm_rng_set_state(uint64_t s) { g_rng = s; }

// ---- reference calling convention ----------------------------------------
static std::mutex g_default_mu;
static bm_ctx_t *g_default = nullptr;

static int default_ctx(bm_ctx_t **out) {
    std::lock_guard<std::mutex> lk(g_default_mu);
    if (!g_default) {
        const char *s = getenv("BM_DEVICE");
        int dev = s ? atoi(s) : 0;
        int rc = bm_ctx_create(dev, &g_default);
        if (rc != BM_OK) return rc;
    }
    *out = g_default;
    return BM_OK;
}

int bm_sample_rows(const float *h_logits, int B, int V, int64_t ld, const int32_t *h_hist,
                   const int64_t *h_hist_off, const bm_knobs_t *h_knobs, int64_t knob_stride,
                   int32_t *h_out_id) {
    if (B < 0 || !h_knobs || !h_out_id || (B > 0 && !h_logits))
        return fail(BM_ERR_INVALID_ARG, "bad arguments to bm_sample_rows");
    if (B == 0) return BM_OK;
    bm_ctx_t *c;
    int rc = default_ctx(&c);
    if (rc != BM_OK) return rc;
    std::vector<float> u(B);
    std::vector<bm_row_stats_t> st(B);
    // draw in row order for rows that will draw; greedy rows never do
    // (src/model.c:144-154).  A row whose candidate set turns out empty
    // (argmax guard) does not draw either; that is only known after the
    // kernel, so the stream is re-assigned and the later rows re-run.
    const uint64_t state0 = g_rng;
    std::vector<char> draws(B);
    for (int r = 0; r < B; ++r) {
        const bm_knobs_t &k = h_knobs[knob_stride ? r : 0];
        draws[r] = !(k.temp < 0.05f);
        u[r] = draws[r] ? bm_rng_float() : 0.0f;
    }
    rc = bm_sample_batch_host(c, h_logits, B, V, ld, h_hist, h_hist_off, h_knobs, knob_stride,
                              u.data(), h_out_id, nullptr, st.data());
    if (rc != BM_OK) {
        g_rng = state0;
        return rc;
    }
    int first_fix = -1;
    for (int r = 0; r < B; ++r)
        if (draws[r] && !st[r].consumed) {
            draws[r] = 0;
            if (first_fix < 0) first_fix = r;
        }
    if (first_fix >= 0) {
        g_rng = state0;
        for (int r = 0; r < B; ++r) u[r] = draws[r] ? bm_rng_float() : 0.0f;
        // rows after the first non-drawing row see shifted uniforms
        int start = first_fix + 1;
        if (start < B) {
            const int32_t *hh = h_hist;
            std::vector<int64_t> off;
            if (h_hist) {
                off.assign(h_hist_off + start, h_hist_off + B + 1);
            }
            rc = bm_sample_batch_host(c, h_logits + (size_t)start * ld, B - start, V, ld, hh,
                                      h_hist ? off.data() : nullptr,
                                      knob_stride ? h_knobs + start : h_knobs, knob_stride,
                                      u.data() + start, h_out_id + start, nullptr, nullptr);
            if (rc != BM_OK) return rc;
        }
    }
    return BM_OK;
}

int bm_sample_row(float *logits, int V, const int *history, int history_len, float penalty,
                  float temp, float min_p, float top_p, int top_k) {
    if (!logits || V < 1 || history_len < 0 || (history_len > 0 && !history))
        return fail(BM_ERR_INVALID_ARG, "bad arguments to bm_sample_row");
    bm_knobs_t k;
    bm_knobs_init(&k, temp, penalty, min_p, top_p, top_k);
    int64_t off[2] = {0, history_len};
    int32_t id = -1;
    int rc = bm_sample_rows(logits, 1, V, V, history_len > 0 ? history : nullptr,
                            history_len > 0 ? off : nullptr, &k, 0, &id);
    return rc != BM_OK ? rc : id;
}

}  // extern "C"

// The library's error channel for the other translation units (bm_decode.cu).
int bm_detail_fail(int code, const char *msg) { return fail(code, "%s", msg); }
