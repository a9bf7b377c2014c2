// Device-resident decode loop state: the reference generation loop's
// bookkeeping (src/main.c:42-50, 455-500) kept on the GPU, so that repeated
// decode steps (logits -> token -> history -> stop check) need no host round
// trip.
//
//   history   src/main.c:42-50 (history_push): a sliding window of the last
//             256 ids.  Here a ring of 256 slots per row, slot p % 256 taking
//             the p-th pushed id, empty slots -1.  The sampler reads the ring
//             as its history CSR (row r at [256 r, 256 r + 256)): the penalty
//             works on the set of distinct in-range ids and skips -1
//             (src/model.c:1276-1281), so the ring gives the reference's
//             window exactly.
//   step      src/main.c:476-499: sample `next`, count it, current = next,
//             push it, stop on EOS (50256) or 0; the loop bound max_tokens;
//             the chat loop's user stop tokens (src/chat.c:1069-1081).
//
// A row that has stopped is still sampled by the batched kernel (rows are
// independent); its result is discarded and its id reported as -1.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include <cuda_runtime.h>

#include "bm_sampler.h"

namespace {

constexpr int HMAX = BM_HISTORY_MAX;
constexpr int TOKEN_EOS = 50256;  // src/bitmamba.h:21

__global__ void decode_update_kernel(const int32_t *ids, int B, int32_t *ring, int32_t *pos,
                                     int32_t *cur, int32_t *status, int32_t *ngen,
                                     const int32_t *stop, int n_stop, int max_tokens,
                                     int32_t *active, int32_t *out_id) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= B) return;
    if (status[r] != BM_DECODE_ACTIVE) {
        if (out_id) out_id[r] = -1;
        return;
    }
    const int id = ids[r];
    const int p = pos[r];
    ring[(int64_t)r * HMAX + (p % HMAX)] = id;  // history_push (src/main.c:42-50)
    pos[r] = p + 1;
    cur[r] = id;
    const int n = ngen[r] + 1;
    ngen[r] = n;
    int st = BM_DECODE_ACTIVE;
    if (id == TOKEN_EOS || id == 0) {  // src/main.c:498-499
        st = BM_DECODE_STOP_EOS;
    } else {
        for (int j = 0; j < n_stop; ++j)
            if (id == stop[j]) st = BM_DECODE_STOP_TOKEN;  // src/chat.c:1069-1081
        if (st == BM_DECODE_ACTIVE && max_tokens > 0 && n >= max_tokens)
            st = BM_DECODE_STOP_MAX;  // the loop bound, src/main.c:473
    }
    status[r] = st;
    if (st != BM_DECODE_ACTIVE) atomicSub(active, 1);
    if (out_id) out_id[r] = id;
}

}  // namespace

// the library's error channel (bm_sampler.cu): bm_last_error reads it
int bm_detail_fail(int code, const char *msg);

struct bm_decode {
    bm_ctx_t *ctx;
    int B, max_tokens, n_stop;
    int32_t *d_ring;   // [B x 256]
    int64_t *d_off;    // [B + 1], 256 r
    int32_t *d_pos;    // ids pushed so far (prompt included)
    int32_t *d_cur;    // the token the next forward step consumes
    int32_t *d_status; // BM_DECODE_*
    int32_t *d_ngen;   // tokens generated
    int32_t *d_stop;   // [n_stop]
    int32_t *d_active; // rows still active
    int32_t *d_id;     // the step's sampled ids
    int32_t *h_active; // pinned
};

namespace {

int dfail(int code, const char *what, cudaError_t e = cudaSuccess) {
    char buf[256];
    if (e != cudaSuccess)
        snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    else
        snprintf(buf, sizeof(buf), "%s", what);
    return bm_detail_fail(code, buf);
}

#define DCK(call)                                                                        \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess)                                                           \
            return dfail(e_ == cudaErrorMemoryAllocation ? BM_ERR_OOM : BM_ERR_CUDA, #call, e_); \
    } while (0)

void release(bm_decode_t *d) {
    cudaFree(d->d_ring);
    cudaFree(d->d_off);
    cudaFree(d->d_pos);
    cudaFree(d->d_cur);
    cudaFree(d->d_status);
    cudaFree(d->d_ngen);
    cudaFree(d->d_stop);
    cudaFree(d->d_active);
    cudaFree(d->d_id);
    if (d->h_active) cudaFreeHost(d->h_active);
}

int launch_update(bm_decode_t *d, int32_t *d_out_id, cudaStream_t s) {
    const int threads = 256, blocks = (d->B + threads - 1) / threads;
    decode_update_kernel<<<blocks, threads, 0, s>>>(d->d_id, d->B, d->d_ring, d->d_pos, d->d_cur,
                                                    d->d_status, d->d_ngen, d->d_stop, d->n_stop,
                                                    d->max_tokens, d->d_active, d_out_id);
    DCK(cudaGetLastError());
    return BM_OK;
}

}  // namespace

extern "C" {

int bm_decode_create(bm_ctx_t *ctx, int B, int max_tokens, const int32_t *stop_ids, int n_stop,
                     bm_decode_t **out) {
    if (!out) return dfail(BM_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (!ctx || B < 1 || n_stop < 0 || (n_stop > 0 && !stop_ids) || max_tokens < 0)
        return dfail(BM_ERR_INVALID_ARG, "ctx NULL, B < 1, n_stop < 0 or max_tokens < 0");
    int dev = 0;
    int rc = bm_ctx_device(ctx, &dev);
    if (rc != BM_OK) return rc;
    DCK(cudaSetDevice(dev));
    bm_decode_t *d = static_cast<bm_decode_t *>(calloc(1, sizeof(bm_decode_t)));
    if (!d) return dfail(BM_ERR_OOM, "calloc");
    d->ctx = ctx;
    d->B = B;
    d->max_tokens = max_tokens;
    d->n_stop = n_stop;
    cudaError_t e = cudaSuccess;
    auto al = [&](void **p, size_t n) {
        if (e == cudaSuccess) e = cudaMalloc(p, n ? n : 4);
    };
    al(reinterpret_cast<void **>(&d->d_ring), (size_t)B * HMAX * 4);
    al(reinterpret_cast<void **>(&d->d_off), (size_t)(B + 1) * 8);
    al(reinterpret_cast<void **>(&d->d_pos), (size_t)B * 4);
    al(reinterpret_cast<void **>(&d->d_cur), (size_t)B * 4);
    al(reinterpret_cast<void **>(&d->d_status), (size_t)B * 4);
    al(reinterpret_cast<void **>(&d->d_ngen), (size_t)B * 4);
    al(reinterpret_cast<void **>(&d->d_stop), (size_t)n_stop * 4);
    al(reinterpret_cast<void **>(&d->d_active), 4);
    al(reinterpret_cast<void **>(&d->d_id), (size_t)B * 4);
    if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void **>(&d->h_active), 4);
    if (e == cudaSuccess) {
        std::vector<int64_t> off((size_t)B + 1);
        for (int r = 0; r <= B; ++r) off[(size_t)r] = (int64_t)r * HMAX;
        e = cudaMemcpy(d->d_off, off.data(), off.size() * 8, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess && n_stop)
        e = cudaMemcpy(d->d_stop, stop_ids, (size_t)n_stop * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        release(d);
        free(d);
        return dfail(e == cudaErrorMemoryAllocation ? BM_ERR_OOM : BM_ERR_CUDA, "decode setup", e);
    }
    // every row starts stopped until a prompt is pushed
    std::vector<int32_t> st((size_t)B, BM_DECODE_STOP_MAX);
    const int32_t zero = 0;
    e = cudaMemcpy(d->d_status, st.data(), (size_t)B * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(d->d_active, &zero, 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        release(d);
        free(d);
        return dfail(BM_ERR_CUDA, "decode setup", e);
    }
    *out = d;
    return BM_OK;
}

int bm_decode_destroy(bm_decode_t *d) {
    if (!d) return BM_OK;
    int dev = 0;
    if (bm_ctx_device(d->ctx, &dev) == BM_OK) cudaSetDevice(dev);
    release(d);
    free(d);
    return BM_OK;
}

int bm_decode_reset(bm_decode_t *d, const int32_t *h_prompt, const int64_t *h_prompt_off) {
    if (!d || !h_prompt_off || (!h_prompt && h_prompt_off[d->B] > h_prompt_off[0]))
        return dfail(BM_ERR_INVALID_ARG, "decode NULL or prompt offsets missing");
    const int B = d->B;
    std::vector<int32_t> ring((size_t)B * HMAX, -1), pos((size_t)B), cur((size_t)B);
    for (int r = 0; r < B; ++r) {
        const int64_t a = h_prompt_off[r], b = h_prompt_off[r + 1];
        if (b < a) return dfail(BM_ERR_INVALID_ARG, "prompt offsets decrease");
        const int64_t n = b - a;
        if (n > INT32_MAX / 2) return dfail(BM_ERR_INVALID_ARG, "prompt too long");
        // history_push of every prompt id keeps the last 256 (src/main.c:455-456)
        for (int64_t p = (n > HMAX ? n - HMAX : 0); p < n; ++p)
            ring[(size_t)r * HMAX + (size_t)(p % HMAX)] = h_prompt[a + p];
        pos[(size_t)r] = (int32_t)n;
        cur[(size_t)r] = n ? h_prompt[b - 1] : 0;  // current = prompt_ids[n_prompt - 1]
    }
    int dev = 0;
    int rc = bm_ctx_device(d->ctx, &dev);
    if (rc != BM_OK) return rc;
    DCK(cudaSetDevice(dev));
    const int32_t active = B;
    DCK(cudaMemcpy(d->d_ring, ring.data(), ring.size() * 4, cudaMemcpyHostToDevice));
    DCK(cudaMemcpy(d->d_pos, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice));
    DCK(cudaMemcpy(d->d_cur, cur.data(), cur.size() * 4, cudaMemcpyHostToDevice));
    DCK(cudaMemset(d->d_status, 0, (size_t)B * 4));
    DCK(cudaMemset(d->d_ngen, 0, (size_t)B * 4));
    DCK(cudaMemcpy(d->d_active, &active, 4, cudaMemcpyHostToDevice));
    return BM_OK;
}

int bm_decode_step(bm_decode_t *d, const float *d_logits, int V, int64_t ld,
                   const bm_knobs_t *d_knobs, int64_t knob_stride, const float *d_uniform,
                   int32_t *d_out_id, void *stream) {
    if (!d) return dfail(BM_ERR_INVALID_ARG, "decode is NULL");
    int rc = bm_sample_batch(d->ctx, d_logits, d->B, V, ld, d->d_ring, d->d_off, d_knobs,
                             knob_stride, d_uniform, d->d_id, nullptr, nullptr, stream);
    if (rc != BM_OK) return rc;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream)
                            : static_cast<cudaStream_t>(bm_ctx_stream(d->ctx));
    return launch_update(d, d_out_id, s);
}

int bm_decode_ternary_step(bm_decode_t *d, const float *d_hidden, int d_model,
                           const float *d_norm_f, const float *d_lmh_norm, const int8_t *d_w8,
                           float w_scale, int V, const bm_knobs_t *d_knobs, int64_t knob_stride,
                           const float *d_uniform, int32_t *d_out_id, void *stream) {
    if (!d) return dfail(BM_ERR_INVALID_ARG, "decode is NULL");
    int rc = bm_ternary_sample_batch(d->ctx, d_hidden, d->B, d_model, d_norm_f, d_lmh_norm, d_w8,
                                     w_scale, V, d->d_ring, d->d_off, d_knobs, knob_stride,
                                     d_uniform, d->d_id, nullptr, nullptr, stream);
    if (rc != BM_OK) return rc;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream)
                            : static_cast<cudaStream_t>(bm_ctx_stream(d->ctx));
    return launch_update(d, d_out_id, s);
}

int bm_decode_views(const bm_decode_t *d, bm_decode_views_t *v) {
    if (!d || !v) return dfail(BM_ERR_INVALID_ARG, "decode or views NULL");
    v->ring = d->d_ring;
    v->ring_off = d->d_off;
    v->current = d->d_cur;
    v->status = d->d_status;
    v->n_generated = d->d_ngen;
    v->n_pushed = d->d_pos;
    v->n_active = d->d_active;
    return BM_OK;
}

int bm_decode_read(bm_decode_t *d, int32_t *h_current, int32_t *h_status, int32_t *h_n_generated,
                   int32_t *h_ring) {
    if (!d) return dfail(BM_ERR_INVALID_ARG, "decode is NULL");
    int dev = 0;
    int rc = bm_ctx_device(d->ctx, &dev);
    if (rc != BM_OK) return rc;
    DCK(cudaSetDevice(dev));
    DCK(cudaStreamSynchronize(static_cast<cudaStream_t>(bm_ctx_stream(d->ctx))));
    const size_t n = (size_t)d->B * 4;
    if (h_current) DCK(cudaMemcpy(h_current, d->d_cur, n, cudaMemcpyDeviceToHost));
    if (h_status) DCK(cudaMemcpy(h_status, d->d_status, n, cudaMemcpyDeviceToHost));
    if (h_n_generated) DCK(cudaMemcpy(h_n_generated, d->d_ngen, n, cudaMemcpyDeviceToHost));
    if (h_ring) DCK(cudaMemcpy(h_ring, d->d_ring, n * HMAX, cudaMemcpyDeviceToHost));
    return BM_OK;
}

int bm_decode_active(bm_decode_t *d, void *stream, int32_t *h_n_active) {
    if (!d || !h_n_active) return dfail(BM_ERR_INVALID_ARG, "decode or output NULL");
    int dev = 0;
    int rc = bm_ctx_device(d->ctx, &dev);
    if (rc != BM_OK) return rc;
    DCK(cudaSetDevice(dev));
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream)
                            : static_cast<cudaStream_t>(bm_ctx_stream(d->ctx));
    DCK(cudaMemcpyAsync(d->h_active, d->d_active, 4, cudaMemcpyDeviceToHost, s));
    DCK(cudaStreamSynchronize(s));
    *h_n_active = *d->h_active;
    return BM_OK;
}

}  // extern "C"
