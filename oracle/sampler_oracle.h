/*
 * CPU oracle for the decode-step sampler (TEST INFRASTRUCTURE ONLY).
 *
 * A plain-C restatement of jserv/bitmamba.c's sampling tail: the repetition
 * penalty block of model_forward_step (src/model.c:1268-1305) followed by
 * sample_advanced / filter_and_sample (src/model.c:37-361).  It exists so the
 * tests and the bench's CPU baseline can check the CUDA path; nothing in the
 * product library links, loads or calls it.
 *
 * Differences from the reference, all deliberate and output-neutral:
 *   - the uniform draw is an argument instead of a call to rng_float();
 *   - the float->int conversion of the histogram bucket follows x86
 *     cvttss2si explicitly (NaN / out-of-range -> INT_MIN) so the oracle
 *     reproduces the x86 build on any host;
 *   - qsort (glibc 2.39: stable merge sort) is replaced by an explicit stable
 *     merge sort with the same comparator, so tie order does not depend on
 *     the host libc;
 *   - a diagnostics record describes the path taken and the margins the
 *     parity tests use to classify rows near a CDF / top_p boundary.
 */
#ifndef BM_SAMPLER_ORACLE_H
#define BM_SAMPLER_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Path codes, shared with the CUDA library's optional per-row stats. */
enum {
    BMO_PATH_GREEDY = 1,     /* temp < 0.05: argmax, no draw      (model.c:144-154) */
    BMO_PATH_K_GUARD = 2,    /* top_k path, nothing extracted      (model.c:227-237) */
    BMO_PATH_K = 3,          /* histogram top_k path               (model.c:178-280) */
    BMO_PATH_FULL_GUARD = 4, /* fallback, nothing passed min_p     (model.c:296-303) */
    BMO_PATH_LAZY = 5,       /* fallback, CDF walk in id order     (model.c:319-320) */
    BMO_PATH_PARTIAL = 6,    /* fallback, top-256 heap covers top_p(model.c:327-356) */
    BMO_PATH_FULL = 7        /* fallback, full sort                (model.c:359-360) */
};

typedef struct {
    int32_t id;
    float val;
} bmo_cand_t; /* same layout as token_prob_t (src/bitmamba.h:99-102) */

typedef struct {
    int32_t token;     /* sampled id */
    float prob;        /* probability of the sampled id in the final candidate
                          array; 1.0 for greedy / guard rows */
    int32_t consumed;  /* 1 when the reference would have called rng_float() */
    int32_t path;      /* BMO_PATH_* */
    int32_t n_cand;    /* candidates after min_p / histogram extraction */
    int32_t n_final;   /* size of the array the CDF walk ran over */
    int32_t pos;       /* position of the sampled id in that array */
    float r;           /* u * (float)new_sum */
    double new_sum;    /* renormalisation sum of filter_and_sample */
    double r_margin;   /* min |r - cdf_i| over the walked prefix, / new_sum */
    double cut_margin; /* min |cs_i - top_p| over the nucleus scan (1 if no cut) */
    float max_logit;   /* after temperature */
    float thresh;      /* extraction threshold (min_p or histogram) */
} bmo_result_t;

/* Repetition penalty, in place (src/model.c:1268-1305).  `visited` is caller
 * scratch of (V+63)/64 words. */
void bmo_apply_penalty(float *logits, int V, const int32_t *history,
                       int history_len, float penalty, uint64_t *visited);

/* sample_advanced (src/model.c:135-361) with `u` standing in for the one
 * rng_float() call; logits are modified in place exactly like the reference.
 * `probs` is scratch of V entries.  Returns the token id. */
int32_t bmo_sample_advanced(float *logits, int V, float temp, float min_p,
                            float top_p, int top_k, float u, bmo_cand_t *probs,
                            bmo_result_t *res);

/* Penalty + sample_advanced on a private copy of one row (logits untouched).
 * `work` must hold V floats, `probs` V entries, `visited` (V+63)/64 words. */
int32_t bmo_sample_row(const float *logits, int V, const int32_t *history,
                       int history_len, float penalty, float temp, float min_p,
                       float top_p, int top_k, float u, float *work,
                       bmo_cand_t *probs, uint64_t *visited,
                       bmo_result_t *res);

/* Batched form used by the tests and the CPU baseline.  Rows are
 * [B x ld] floats; histories are CSR (hist_off has B+1 entries, may be NULL
 * for no history); knobs are per-row arrays.  Runs `n_threads` pthreads over
 * rows (row-parallel; each thread has its own scratch).  `res` may be NULL.
 * Returns 0 on success, -1 on allocation failure. */
int bmo_sample_batch(const float *logits, int B, int V, int64_t ld,
                     const int32_t *hist, const int64_t *hist_off,
                     const float *temp, const float *penalty,
                     const float *min_p, const float *top_p,
                     const int32_t *top_k, const float *uniform,
                     int32_t *out_id, float *out_prob, bmo_result_t *res,
                     int n_threads);

/* Reference RNG (src/utils.c:117-140): XorShift64* with the reference's
 * default state and its float conversion. */
void bmo_rng_seed(uint64_t *state, uint64_t seed);
uint64_t bmo_rng_next(uint64_t *state);
float bmo_rng_float(uint64_t *state);

#ifdef __cplusplus
}
#endif

#endif
