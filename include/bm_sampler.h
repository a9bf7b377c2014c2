/*
 * bm_sampler.h - C ABI of the B200 decode-step token sampler.
 *
 * Drop-in replacement for the sampling tail of jserv/bitmamba.c:
 *   repetition penalty (src/model.c:1268-1305) -> sample_advanced /
 *   filter_and_sample (src/model.c:37-361) -> rng_float (src/utils.c:117-140).
 * The batched entry points run a hand-written sm_100a CUDA kernel: one
 * persistent CTA per SM, one logits row at a time in shared memory.  There is
 * no CPU fallback: every sampling entry point fails with BM_ERR_NO_DEVICE /
 * BM_ERR_CUDA when no usable B200 is present.
 *
 * Semantics kept from the reference, row by row:
 *   - penalty applied once per distinct history id in [0, V), skipping the
 *     protected GPT-2 ids {50256, 198, 628, 13}: l > 0 ? l / penalty
 *     : l * penalty (src/model.c:1283-1304; ids src/bitmamba.h:21-24);
 *   - temp < 0.05 -> argmax of the penalised logits, lowest id on ties, no
 *     uniform consumed (src/model.c:144-154);
 *   - otherwise logits * (1/temp), min_p threshold max + logf(min_p), the
 *     128-bucket histogram top_k path for 1 <= top_k <= 256 (heap top-k,
 *     survivor softmax, stable descending sort when top_p < 1), or the
 *     full-vocabulary path for other top_k (lazy id-order walk, top-256
 *     partial sort, full sort), then the nucleus cut and the CDF walk against
 *     r = u * (float)new_sum (src/model.c:156-360, 72-118).
 * Token ids equal the reference's except where the draw or the nucleus cut
 * lies within 1e-5 of a CDF boundary; probabilities agree to a few ulps (the
 * device exp is within 3 ulp of the correctly rounded value).
 *
 * Thread safety: a bm_ctx_t may be used by one host thread at a time.  The
 * reference-convention calls (bm_sample_row, bm_sample_rows) share one
 * process-global RNG and default context, like the reference's globals
 * (src/utils.c:119), and are not reentrant.
 */
#ifndef BM_SAMPLER_H
#define BM_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BM_SAMPLER_ABI_VERSION 1

/* Status codes.  Sampling entry points return >= 0 on success (a token id
 * for the single-row calls, BM_OK for the batched calls). */
enum {
    BM_OK = 0,
    BM_ERR_INVALID_ARG = -1,  /* bad pointer, size, stride or knob layout */
    BM_ERR_CUDA = -2,         /* a CUDA runtime call failed */
    BM_ERR_OOM = -3,          /* device or pinned-host allocation failed */
    BM_ERR_UNSUPPORTED = -4,  /* V larger than one row buffer (bm_max_vocab) */
    BM_ERR_NO_DEVICE = -5,    /* no CUDA device, or not an sm_100 part */
    BM_ERR_DEVICE = -6        /* the kernel raised its error flag (a bounded
                                 wait timed out); the context stays usable */
};

/* Per-row sampling knobs in the reference's units (src/main.c:316-321).
 * The derived fields are filled by bm_knobs_init on the host so that
 * 1.0f/temp is an IEEE division and logf(min_p) comes from the host libm, as
 * in the reference (src/model.c:157, 173).  32 bytes, device-copyable. */
typedef struct bm_knobs {
    float temp;
    float penalty;
    float min_p;
    float top_p;
    int32_t top_k;
    float inv_temp;  /* derived: 1.0f / temp */
    float log_min_p; /* derived: logf(min_p) when 0 < min_p < 1, else 0 */
    int32_t flags;   /* reserved, 0 */
} bm_knobs_t;

/* Optional per-row diagnostics written by the batched calls. */
typedef struct bm_row_stats {
    int32_t path;     /* 1 greedy, 2 top_k guard, 3 top_k, 4 full guard,
                         5 lazy id-order walk, 6 top-256 partial, 7 full */
    int32_t n_cand;   /* candidates after min_p / histogram extraction */
    int32_t n_final;  /* size of the set the CDF walk ran over */
    int32_t consumed; /* 1 when the reference would have drawn a uniform */
} bm_row_stats_t;

typedef struct bm_ctx bm_ctx_t;

/* ---- knobs --------------------------------------------------------------- */

/* Fills *k from the reference's five knobs.  Any float is accepted (NaN and
 * infinities keep the reference's behaviour).  Returns BM_OK or
 * BM_ERR_INVALID_ARG for k == NULL. */
int bm_knobs_init(bm_knobs_t *k, float temp, float penalty, float min_p,
                  float top_p, int top_k);

/* ---- contexts -------------------------------------------------------------- */

/* Creates a sampling context on CUDA device `device` (its stream, staging
 * buffers, error flag).  Fails with BM_ERR_NO_DEVICE when the device is
 * absent or is not compute capability 10.x. */
int bm_ctx_create(int device, bm_ctx_t **out);
void bm_ctx_destroy(bm_ctx_t *ctx);

/* Largest vocabulary one row buffer holds on this device (V * 4 bytes plus
 * scratch must fit one CTA's shared memory). */
int bm_max_vocab(const bm_ctx_t *ctx);

/* Reads and clears the device error flag (synchronises the context stream).
 * Returns BM_OK or BM_ERR_DEVICE. */
int bm_ctx_check(bm_ctx_t *ctx);

/* The context's CUDA stream (a cudaStream_t), on which bm_sample_batch_host
 * and bm_sample_batch with stream == NULL run; lets callers order their own
 * work (events, copies) against the sampler.  No reference counterpart: the
 * reference sampler is synchronous on the calling thread. */
void *bm_ctx_stream(bm_ctx_t *ctx);

/* The CUDA device ordinal the context was created on. */
int bm_ctx_device(const bm_ctx_t *ctx, int *device);

/* ---- batched sampling, device buffers -------------------------------------- */

/*
 * Samples one token per row of a [B x V] fp32 logits matrix in device memory
 * (row pitch ld >= V elements).  Replaces, per row, the penalty block and
 * sample_advanced call of model_forward_step (src/model.c:1268-1307).
 *
 *   d_hist, d_hist_off  CSR token histories: row r owns
 *                       d_hist[d_hist_off[r] .. d_hist_off[r+1]).
 *                       Both NULL = no history.  Out-of-range ids are
 *                       skipped, duplicates penalised once.
 *   d_knobs             per-row knobs; knob_stride = 1 for one struct per
 *                       row, 0 to apply d_knobs[0] to every row.
 *   d_uniform           one uniform in [0,1] per row (the value the
 *                       reference's rng_float() would return for that row);
 *                       ignored for rows that do not draw.
 *   d_out_id            [B] sampled ids.
 *   d_out_prob          optional [B]: probability of the sampled id in the
 *                       final candidate array (1.0 for greedy/guard rows).
 *   d_stats             optional [B] diagnostics.
 *   stream              a cudaStream_t (NULL = the context's stream).
 * Logits are read-only (the reference scales them in place; this does not).
 * Asynchronous: returns after enqueueing.  Call bm_ctx_check to collect the
 * device error flag.  Rows are handed to SMs by a counter that lives in the
 * context: launches on one context must not overlap (issue them on one
 * stream, or order them); use one context per concurrently running stream.
 */
int bm_sample_batch(bm_ctx_t *ctx, const float *d_logits, int B, int V,
                    int64_t ld, const int32_t *d_hist,
                    const int64_t *d_hist_off, const bm_knobs_t *d_knobs,
                    int64_t knob_stride, const float *d_uniform,
                    int32_t *d_out_id, float *d_out_prob,
                    bm_row_stats_t *d_stats, void *stream);

/*
 * bm_sample_batch without a context and without any allocation (no
 * cudaMalloc, no host allocation).  No reference counterpart: the reference
 * samples one row on the CPU and owns its buffers.  Same arguments and
 * semantics as bm_sample_batch, on the calling thread's current CUDA device;
 * stream NULL is the legacy default stream.
 *
 * Scratch: one file-scope device array per device (64 ints = 256 bytes,
 * 256-byte aligned): an error word and the two row-schedule counters.  The
 * counters must start at zero; they are zero when the module loads and every
 * launch returns them to zero.  The first call on a device takes the array's
 * address (cudaGetSymbolAddress) and sets the kernel's shared-memory
 * attribute; that first call must come before any stream capture on that
 * device.  All calls on one device share the scratch: calls that overlap in
 * time (different streams, or threads without ordering) race on the row
 * schedule and must not be made; order them on one stream.
 *
 * Limits: V <= bm_max_vocab (50268 on a B200) else BM_ERR_UNSUPPORTED;
 * B <= 2^30 rows per call else BM_ERR_INVALID_ARG.  There is no context
 * error flag to check: a row whose bounded wait in the kernel expired, or
 * whose exact selection (the rare fallback over global memory) did not
 * converge, gets id -1; the launch leaves the error word cleared.
 */
int bm_sample_batch_noalloc(const float *d_logits, int B, int V, int64_t ld,
                            const int32_t *d_hist, const int64_t *d_hist_off,
                            const bm_knobs_t *d_knobs, int64_t knob_stride,
                            const float *d_uniform, int32_t *d_out_id,
                            float *d_out_prob, bm_row_stats_t *d_stats,
                            void *stream);

/* ---- final RMSNorm + bf16 lm_head feeding the sampler ---------------------- */

/*
 * logits[r, n] = sum_k bf16(rmsnorm(hidden[r, :]))[k] * W[n, k] for B rows of
 * d_model hidden states (fp32, row-major) and a V x d_model bf16 lm_head (raw
 * bf16 bits, row-major), accumulated in fp32 on the tensor cores, into
 * d_logits (fp32, row pitch ld >= V).  rmsnorm is the reference's
 * scalar_rms_norm (src/kernel.c:72-91: x * (1 / sqrtf(sum_sq / d + 1e-6f)) * w,
 * the sum of squares in four strided fp32 accumulators), bit for bit, rounded
 * to bf16 for the tensor cores.  The reference's own lm_head is a ternary
 * BitLinear (src/model.c:1239-1262); this bf16 projection has no counterpart
 * there.  d_model % 8 == 0, d_model <= 4096; hidden, norm weight and W
 * 16-byte aligned.
 * Stream-ordered; errors of the kernels show in bm_ctx_check.
 */
int bm_lmhead_logits(bm_ctx_t *ctx, const float *d_hidden, int B, int d_model,
                     const float *d_norm_w, const uint16_t *d_W, int V,
                     float *d_logits, int64_t ld, void *stream);

/*
 * The fused decode step from the final hidden state to the next token: the
 * final RMSNorm and the bf16 lm_head GEMM of bm_lmhead_logits, and the
 * sampler of bm_sample_batch on those logits (same arguments, same results),
 * without the logits making a round trip through HBM for greedy rows and
 * rows of the top_k path (1 <= top_k <= 256): the GEMM's epilogue keeps, per
 * row and 256-column output tile, the 8 largest penalised and
 * temperature-scaled logits, and a merge kernel finishes the reference's
 * top_k sampler (src/model.c:175-280) from those lists.  A row is finished
 * from its lists only when no tile's omitted logits can reach the top_k
 * histogram's cut buckets or the extracted candidates; other rows, and rows
 * of the full-vocabulary path (their logits are stored by the same GEMM),
 * go through the logits and bm_sample_batch's kernel, on the device without
 * a host round trip.  No counterpart in the reference (see
 * bm_lmhead_logits); the sampling part replaces the tail of
 * model_forward_step (src/model.c:1268-1307).
 */
int bm_lmhead_sample_batch(bm_ctx_t *ctx, const float *d_hidden, int B, int d_model,
                           const float *d_norm_w, const uint16_t *d_W, int V,
                           const int32_t *d_hist, const int64_t *d_hist_off,
                           const bm_knobs_t *d_knobs, int64_t knob_stride,
                           const float *d_uniform, int32_t *d_out_id,
                           float *d_out_prob, bm_row_stats_t *d_stats,
                           void *stream);

/*
 * Diagnostics of the last fused call on this context (bm_lmhead_sample_batch
 * or bm_ternary_sample_batch): rows sampled from logits (n_sampled: rows of
 * the full-vocabulary path and rows their lists could not decide) and, of
 * those, rows whose logits took a GEMM of their own (n_computed).
 * Synchronises the device.  No reference counterpart.
 */
int bm_fused_fallback_rows(bm_ctx_t *ctx, int *n_sampled, int *n_computed);

/* ---- the reference's ternary BitLinear lm_head feeding the sampler --------- */

/*
 * Decodes the lm_head's 2-bit ternary weights (the model file's packed
 * layout, src/model.c:367-475 loads it; 4 codes per byte, lowest bits first,
 * code c -> min(c, 2) - 1, src/quantization.c:27-31; rows of d_model / 4
 * bytes) into int8 {-1, 0, 1}, V x d_model row-major, on the device: the
 * one-time weight preparation of bm_ternary_logits.  d_model % 32 == 0;
 * d_packed 4-byte and d_w8 16-byte aligned.  Stream-ordered.
 */
int bm_ternary_unpack(bm_ctx_t *ctx, const uint8_t *d_packed, int V, int d_model,
                      int8_t *d_w8, void *stream);

/*
 * The reference's logits producer (src/model.c:1222-1262) for B rows of
 * d_model fp32 hidden states: the final RMSNorm with d_norm_f (skipped when
 * NULL), the BitLinear's RMSNorm with d_lmh_norm, int8 absmax quantisation
 * (scale_x = 127 / (max|x| + 1e-5f)), the ternary product on the tensor
 * cores with exact int32 accumulation, logits = (float) dot * (1 / (scale_x *
 * w_scale)).  The arithmetic follows the reference's x86 AVX2 kernels
 * (src/arch/avx2.c:22-83 norm, 276-315 quantisation, 159 output), so the
 * logits are bit-identical to the reference's on such a host.  d_w8 comes
 * from bm_ternary_unpack.  d_model % 32 == 0, d_model <= 4096; hidden and
 * norm weights 16-byte aligned, logits 4-byte aligned, ld >= V.
 * Stream-ordered; errors of the kernels show in bm_ctx_check.
 */
int bm_ternary_logits(bm_ctx_t *ctx, const float *d_hidden, int B, int d_model,
                      const float *d_norm_f, const float *d_lmh_norm,
                      const int8_t *d_w8, float w_scale, int V, float *d_logits,
                      int64_t ld, void *stream);

/*
 * The reference's decode-step tail from the last layer's output to the next
 * token (src/model.c:1222-1307): bm_ternary_logits and the sampler of
 * bm_sample_batch on its logits (same arguments, same results), fused as
 * bm_lmhead_sample_batch is: greedy rows and rows of the top_k path are
 * finished from the GEMM epilogue's per-tile lists, the others from logits.
 */
int bm_ternary_sample_batch(bm_ctx_t *ctx, const float *d_hidden, int B, int d_model,
                            const float *d_norm_f, const float *d_lmh_norm,
                            const int8_t *d_w8, float w_scale, int V,
                            const int32_t *d_hist, const int64_t *d_hist_off,
                            const bm_knobs_t *d_knobs, int64_t knob_stride,
                            const float *d_uniform, int32_t *d_out_id,
                            float *d_out_prob, bm_row_stats_t *d_stats,
                            void *stream);

/* ---- device-resident decode loop state ------------------------------------- */

/*
 * The reference generation loop's bookkeeping kept on the GPU
 * (src/main.c:42-50, 455-500), so that repeated decode steps run without a
 * host round trip: per row a 256-id history window (src/main.c:19,
 * history_push), the token the next forward step consumes, the number of
 * tokens generated and a stop status.  A step samples every row with the
 * window as its penalty history, then for each active row counts the token,
 * makes it current, pushes it and stops the row on EOS (50256) or token 0
 * (src/main.c:498-499), on a user stop token (src/chat.c:1069-1081) or at
 * max_tokens (the loop bound, src/main.c:473; 0 = no bound).  Stopped rows
 * are still sampled (rows are independent) but left unchanged, and their id
 * is reported as -1.
 *
 * The window is a ring of BM_HISTORY_MAX slots per row (slot p % 256 holds
 * the p-th pushed id, empty slots -1), read by the sampler as the history
 * CSR ring[256 r .. 256 r + 256): the penalty uses the set of distinct
 * in-range ids, so this equals the reference's shifted array.
 */
#define BM_HISTORY_MAX 256

enum {
    BM_DECODE_ACTIVE = 0,
    BM_DECODE_STOP_EOS = 1,    /* sampled 50256 or 0 */
    BM_DECODE_STOP_TOKEN = 2,  /* sampled a user stop token */
    BM_DECODE_STOP_MAX = 3     /* max_tokens generated, or no prompt pushed yet */
};

typedef struct bm_decode bm_decode_t;

/* Device views of a decode state (row-major, B rows). */
typedef struct {
    int32_t *ring;         /* [B x 256] history windows, -1 = empty */
    int64_t *ring_off;     /* [B + 1] = 256 r: the windows as a history CSR */
    int32_t *current;      /* [B] token of the next forward step */
    int32_t *status;       /* [B] BM_DECODE_* */
    int32_t *n_generated;  /* [B] tokens generated since the reset */
    int32_t *n_pushed;     /* [B] ids pushed (prompt + generated) */
    int32_t *n_active;     /* [1] rows with status BM_DECODE_ACTIVE */
} bm_decode_views_t;

/* B rows on ctx's device; every row starts stopped until bm_decode_reset.
 * stop_ids (host, n_stop entries) may be NULL when n_stop == 0. */
int bm_decode_create(bm_ctx_t *ctx, int B, int max_tokens, const int32_t *stop_ids,
                     int n_stop, bm_decode_t **out);
int bm_decode_destroy(bm_decode_t *d);

/* Starts every row from its prompt (host CSR: row r's ids at
 * h_prompt[h_prompt_off[r] .. h_prompt_off[r + 1])): pushes the prompt ids
 * (the window keeps the last 256), current = the last prompt id (0 for an
 * empty prompt), n_generated = 0, every row active.  Synchronous. */
int bm_decode_reset(bm_decode_t *d, const int32_t *h_prompt, const int64_t *h_prompt_off);

/* One decode step from this step's logits (B rows, as bm_sample_batch):
 * sample with the windows as history, then update the state.  d_out_id
 * (optional, [B]) receives the step's tokens, -1 for stopped rows.
 * Stream-ordered (stream NULL: the context stream). */
int bm_decode_step(bm_decode_t *d, const float *d_logits, int V, int64_t ld,
                   const bm_knobs_t *d_knobs, int64_t knob_stride,
                   const float *d_uniform, int32_t *d_out_id, void *stream);

/* The same step from the last layer's output through the reference's final
 * RMSNorm + ternary lm_head (bm_ternary_sample_batch). */
int bm_decode_ternary_step(bm_decode_t *d, const float *d_hidden, int d_model,
                           const float *d_norm_f, const float *d_lmh_norm,
                           const int8_t *d_w8, float w_scale, int V,
                           const bm_knobs_t *d_knobs, int64_t knob_stride,
                           const float *d_uniform, int32_t *d_out_id, void *stream);

/* Device pointers of the state (valid until bm_decode_destroy). */
int bm_decode_views(const bm_decode_t *d, bm_decode_views_t *views);

/* Copies the state to host buffers (each optional: [B] current, status,
 * n_generated; [B x 256] ring).  Synchronises the context stream and the
 * device; for inspection, not for the step loop. */
int bm_decode_read(bm_decode_t *d, int32_t *h_current, int32_t *h_status,
                   int32_t *h_n_generated, int32_t *h_ring);

/* Reads the active-row count (4 bytes to pinned host memory; synchronises
 * the stream). */
int bm_decode_active(bm_decode_t *d, void *stream, int32_t *h_n_active);

/* ---- model file: the decode tail's tensors --------------------------------- */

/*
 * Reads jserv/bitmamba.c's packed model file (magic 0x42495432; written by
 * scripts/export-bin.py:110-200, loaded by src/model.c:477-783) for the
 * tensors the decode tail needs: norm_f, lm_head.norm and the ternary
 * lm_head with its scale.  The file is walked tensor by tensor, as the
 * reference loader does, with the loader's checks (header bounds, per-tensor
 * bounds, shapes and float / packed types); a malformed file fails with
 * BM_ERR_INVALID_ARG and bm_last_error naming the check.
 */
typedef struct {
    int32_t vocab_size, d_model, n_layers, n_heads;
    float w_scale;          /* lm_head scale (the exporter's 1 / mean|W|) */
    float *norm_f;          /* [d_model] */
    float *lm_head_norm;    /* [d_model] */
    uint8_t *packed;        /* [vocab_size x (d_model + 3) / 4] 2-bit codes */
} bm_model_head_host_t;

/* Host only (no GPU needed): fills *out with copies; free with
 * bm_model_head_host_free. */
int bm_model_head_read(const char *path, bm_model_head_host_t *out);
void bm_model_head_host_free(bm_model_head_host_t *h);

typedef struct bm_model_head bm_model_head_t;

typedef struct {
    int32_t vocab_size, d_model, n_layers, n_heads;
    float w_scale;
    const float *d_norm_f;      /* [d_model] on the device */
    const float *d_lmh_norm;    /* [d_model] */
    const int8_t *d_w8;         /* [vocab_size x d_model] decoded ternary weights */
    const uint8_t *d_packed;    /* [vocab_size x d_model / 4] as stored */
} bm_model_head_info_t;

/* Reads the file, uploads the tensors to ctx's device and decodes the
 * ternary weights (bm_ternary_unpack), ready for bm_ternary_logits /
 * bm_ternary_sample_batch / bm_decode_ternary_step.  d_model must be a
 * multiple of 32 (<= 4096), else BM_ERR_UNSUPPORTED.  Synchronous. */
int bm_model_head_load(bm_ctx_t *ctx, const char *path, bm_model_head_t **out);
int bm_model_head_info(const bm_model_head_t *head, bm_model_head_info_t *info);
void bm_model_head_free(bm_model_head_t *head);

/* ---- batched sampling, host buffers ---------------------------------------- */

/*
 * Same as bm_sample_batch with every buffer in host memory: copies the
 * inputs to the context's device staging buffers, samples, copies ids (and
 * probabilities / stats when non-NULL) back, and synchronises.  Host buffers
 * may be pageable or pinned (pinned is faster).  h_logits holds B * ld
 * floats (the last row's pitch included: the rows are copied whole).
 * h_hist_off may be NULL with h_hist NULL.  Calls whose buffers total at
 * most 16 MB (B = 1 through about
 * 80 rows at V = 50257) pack every input into one pinned staging region of
 * the context (grown on demand), so they make one copy each way and one
 * synchronisation.
 */
int bm_sample_batch_host(bm_ctx_t *ctx, const float *h_logits, int B, int V,
                         int64_t ld, const int32_t *h_hist,
                         const int64_t *h_hist_off, const bm_knobs_t *h_knobs,
                         int64_t knob_stride, const float *h_uniform,
                         int32_t *h_out_id, float *h_out_prob,
                         bm_row_stats_t *h_stats);

/* ---- reference calling convention ------------------------------------------ */

/* The reference RNG (src/utils.c:117-140): XorShift64*, default state
 * 0x853c49e6748fea9b, seed 0 keeps the default; process-global. */
void bm_rng_seed(uint64_t seed);
uint64_t bm_rng_next(void);
float bm_rng_float(void);
uint64_t bm_rng_get_state(void);
void bm_rng_set_state(uint64_t state);

/*
 * One row in the reference's argument order (the tail of model_forward_step,
 * src/model.c:1268-1307, with sample_advanced's knobs; prototype of the
 * caller src/bitmamba.h:285-293).  `logits` is host memory and is left
 * unchanged.  Draws from the process-global RNG exactly when the reference
 * would (non-greedy rows whose candidate set is not empty).  Runs on the
 * default context (device from BM_DEVICE, else 0).  Returns the token id, or
 * a negative BM_ERR_* code.
 */
int bm_sample_row(float *logits, int V, const int *history, int history_len,
                  float penalty, float temp, float min_p, float top_p,
                  int top_k);

/*
 * B rows in one launch, equivalent to calling bm_sample_row on rows
 * 0..B-1 in order: rows draw from the global RNG in row order, only when they
 * consume.  Host buffers; histories in CSR form (may be NULL).  Returns
 * BM_OK or a BM_ERR_* code.
 */
int bm_sample_rows(const float *h_logits, int B, int V, int64_t ld,
                   const int32_t *h_hist, const int64_t *h_hist_off,
                   const bm_knobs_t *h_knobs, int64_t knob_stride,
                   int32_t *h_out_id);

/* ---- misc ------------------------------------------------------------------ */

/* Human-readable text of the last error on the calling thread. */
const char *bm_last_error(void);
int bm_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif
