/*
 * CPU oracle for the decode-step sampler (TEST INFRASTRUCTURE ONLY).
 *
 * Restates jserv/bitmamba.c's sampling tail so that the CUDA library can be
 * checked row by row.  Only tests/, __graft_entry__.smoke() and the bench's
 * CPU-baseline leg use this file; the product library never links it.
 * Each function names the reference lines it follows (paths relative to the
 * reference project root).  See sampler_oracle.h for the list of deliberate
 * (output-neutral) differences.
 */
#define _GNU_SOURCE
#include "sampler_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* GPT-2 ids exempt from the repetition penalty (src/bitmamba.h:21-24). */
static const int32_t kProtected[4] = {50256, 198, 628, 13};

/* src/model.c:132-133 */
#define HIST_BUCKETS 128
#define HIST_RANGE 20.0f
/* src/model.c:326 */
#define PARTIAL_K 256

/* (int)f as the x86 cvttss2si instruction computes it: truncation toward
 * zero, and the "integer indefinite" INT_MIN for NaN or out-of-range inputs.
 * The reference's histogram bucket (src/model.c:188) is computed this way on
 * x86 builds, which sends any logit more than ~3.4e8 below the maximum to
 * bucket 0 after the clamp at src/model.c:191-192. */
static int32_t x86_cvtt(float t)
{
    if (!(t < 2147483648.0f && t >= -2147483648.0f))
        return INT32_MIN;
    return (int32_t) t;
}

/* ---- repetition penalty: src/model.c:1268-1305 ------------------------- */
void bmo_apply_penalty(float *logits, int V, const int32_t *history,
                       int history_len, float penalty, uint64_t *visited)
{
    size_t words = ((size_t) V + 63) / 64;
    memset(visited, 0, words * sizeof(uint64_t));
    for (int i = 0; i < history_len; i++) {
        int32_t id = history[i];
        if (id < 0 || id >= V)
            continue;
        uint64_t bit = 1ULL << (id % 64);
        if (visited[id / 64] & bit)
            continue; /* one application per distinct id */
        visited[id / 64] |= bit;
        int prot = 0;
        for (int p = 0; p < 4; p++)
            prot |= (kProtected[p] == id);
        if (prot || !(penalty > 0.0f))
            continue;
        float l = logits[id];
        logits[id] = (l > 0) ? l / penalty : l * penalty;
    }
}

/* ---- min-heap on .val: src/model.c:50-66 -------------------------------- */
static void heap_down(bmo_cand_t *h, int n, int i)
{
    for (;;) {
        int m = i, a = 2 * i + 1, b = 2 * i + 2;
        if (a < n && h[a].val < h[m].val)
            m = a;
        if (b < n && h[b].val < h[m].val)
            m = b;
        if (m == i)
            return;
        bmo_cand_t t = h[i];
        h[i] = h[m];
        h[m] = t;
        i = m;
    }
}

/* Keep the k largest of c[0..n) the way src/model.c:241-252 (and 330-341)
 * does: heapify the first k, then replace the root by every later element
 * that is strictly greater.  Result (in heap layout) is left in dst[0..k). */
static void heap_select(bmo_cand_t *dst, const bmo_cand_t *c, int n, int k)
{
    if (dst != c)
        memcpy(dst, c, (size_t) k * sizeof(bmo_cand_t));
    for (int i = k / 2 - 1; i >= 0; i--)
        heap_down(dst, k, i);
    for (int i = k; i < n; i++) {
        if (c[i].val > dst[0].val) {
            dst[0] = c[i];
            heap_down(dst, k, 0);
        }
    }
}

/* Ordering of compare_token_prob_desc (src/model.c:38-43): a goes before b
 * when b.val - a.val < 0.  NaN differences compare equal. */
static int before(const bmo_cand_t *a, const bmo_cand_t *b)
{
    float d = b->val - a->val;
    return d < 0;
}

/* Stable merge sort by that ordering: the result glibc's merge-sort qsort
 * produces (ties keep their input order). */
static void stable_sort_desc(bmo_cand_t *a, int n, bmo_cand_t *tmp)
{
    if (n < 2)
        return;
    int h = n / 2;
    stable_sort_desc(a, h, tmp);
    stable_sort_desc(a + h, n - h, tmp);
    int i = 0, j = h, o = 0;
    while (i < h && j < n) {
        if (before(&a[j], &a[i]))
            tmp[o++] = a[j++];
        else
            tmp[o++] = a[i++];
    }
    while (i < h)
        tmp[o++] = a[i++];
    while (j < n)
        tmp[o++] = a[j++];
    memcpy(a, tmp, (size_t) n * sizeof(bmo_cand_t));
}

static void sort_desc(bmo_cand_t *a, int n)
{
    if (n < 2)
        return;
    bmo_cand_t *tmp = (bmo_cand_t *) malloc((size_t) n * sizeof(bmo_cand_t));
    if (!tmp)
        abort(); /* the reference exits on OOM (src/utils.c:12-20) */
    stable_sort_desc(a, n, tmp);
    free(tmp);
}

/* ---- filter_and_sample: src/model.c:72-118 ------------------------------ */
static int32_t filter_and_sample(bmo_cand_t *probs, int n, float min_p,
                                 float top_p, int top_k, float u,
                                 bmo_result_t *res)
{
    /* min_p on sorted probabilities (src/model.c:79-87); both callers pass 0 */
    if (min_p > 0.0f) {
        float thr = probs[0].val * min_p;
        for (int i = 1; i < n; i++)
            if (probs[i].val < thr) {
                n = i;
                break;
            }
    }
    double cut_margin = 1.0;
    /* nucleus cut (src/model.c:90-98) */
    if (top_p < 1.0f) {
        double cs = 0.0, prev = 0.0;
        int cut = -1;
        for (int i = 0; i < n; i++) {
            prev = cs;
            cs += probs[i].val;
            if (cs >= top_p) {
                cut = i + 1;
                break;
            }
        }
        if (cut > 0) {
            double a = cs - top_p, b = top_p - prev;
            cut_margin = a < b ? a : b;
            n = cut;
        } else {
            cut_margin = top_p - cs;
        }
    }
    /* top_k truncation (src/model.c:102-103) */
    if (top_k > 0 && top_k < n)
        n = top_k;
    /* renormalise and draw (src/model.c:106-117) */
    double new_sum = 0.0;
    for (int i = 0; i < n; i++)
        new_sum += probs[i].val;
    float r = u * (float) new_sum;
    double cdf = 0.0, lo = -1.0;
    int pos = n - 1;
    double hi = 0.0;
    for (int i = 0; i < n; i++) {
        lo = cdf;
        cdf += probs[i].val;
        if (r < cdf) {
            pos = i;
            break;
        }
    }
    hi = cdf;
    if (res) {
        double m1 = fabs(hi - (double) r);
        double m0 = (pos > 0) ? fabs((double) r - lo) : m1;
        double m = m0 < m1 ? m0 : m1;
        res->consumed = 1;
        res->n_final = n;
        res->pos = pos;
        res->r = r;
        res->new_sum = new_sum;
        res->r_margin = new_sum > 0 ? m / new_sum : m;
        res->cut_margin = cut_margin;
        res->prob = probs[pos].val;
    }
    return probs[pos].id;
}

/* ---- sample_advanced: src/model.c:135-361 ------------------------------- */
int32_t bmo_sample_advanced(float *logits, int V, float temp, float min_p,
                            float top_p, int top_k, float u, bmo_cand_t *probs,
                            bmo_result_t *res)
{
    bmo_result_t dummy;
    if (!res)
        res = &dummy;
    memset(res, 0, sizeof(*res));
    res->cut_margin = 1.0;
    res->r_margin = 1.0;
    res->prob = 1.0f;

    /* greedy (src/model.c:144-154) */
    if (temp < 0.05f) {
        int32_t best = 0;
        float m = -1e9f;
        for (int i = 0; i < V; i++)
            if (logits[i] > m) {
                m = logits[i];
                best = i;
            }
        res->path = BMO_PATH_GREEDY;
        res->token = best;
        return best;
    }

    /* temperature in place + max (src/model.c:157-163) */
    float inv_temp = 1.0f / temp;
    float mx = -1e30f;
    for (int i = 0; i < V; i++) {
        logits[i] *= inv_temp;
        if (logits[i] > mx)
            mx = logits[i];
    }
    res->max_logit = mx;

    /* pre-softmax min_p threshold (src/model.c:169-173) */
    float thr = -1e30f;
    if (min_p >= 1.0f)
        thr = mx;
    else if (min_p > 0.0f)
        thr = mx + logf(min_p);

    int k = (top_k > 0 && top_k <= 256) ? top_k : 0; /* src/model.c:175 */

    if (k > 0) {
        /* 128-bucket histogram of (max - l) over survivors of min_p
         * (src/model.c:181-195) */
        int32_t hist[HIST_BUCKETS];
        memset(hist, 0, sizeof(hist));
        float scale = (float) (HIST_BUCKETS - 1) / HIST_RANGE;
        for (int i = 0; i < V; i++) {
            if (logits[i] >= thr) {
                int32_t b = x86_cvtt((mx - logits[i]) * scale);
                if (b >= HIST_BUCKETS)
                    b = HIST_BUCKETS - 1;
                if (b < 0)
                    b = 0;
                hist[b]++;
            }
        }
        /* first bucket whose running count reaches k (src/model.c:199-207) */
        int cut = HIST_BUCKETS - 1, acc = 0;
        for (int b = 0; b < HIST_BUCKETS; b++) {
            acc += hist[b];
            if (acc >= k) {
                cut = b;
                break;
            }
        }
        float bthr = mx - (float) (cut + 1) / scale; /* src/model.c:210-211 */
        float ethr = bthr > thr ? bthr : thr;       /* src/model.c:213-214 */
        res->thresh = ethr;

        /* extraction in id order (src/model.c:217-224) */
        int n = 0;
        for (int i = 0; i < V; i++)
            if (logits[i] >= ethr) {
                probs[n].id = i;
                probs[n].val = logits[i];
                n++;
            }
        res->n_cand = n;
        if (n == 0) { /* argmax guard (src/model.c:227-237) */
            int32_t best = 0;
            float bv = logits[0];
            for (int i = 1; i < V; i++)
                if (logits[i] > bv) {
                    bv = logits[i];
                    best = i;
                }
            res->path = BMO_PATH_K_GUARD;
            res->token = best;
            return best;
        }
        if (n > k) { /* heap top-k (src/model.c:240-254) */
            heap_select(probs, probs, n, k);
            n = k;
        }
        /* softmax over survivors (src/model.c:257-269) */
        float lmax = -1e30f;
        for (int i = 0; i < n; i++)
            if (probs[i].val > lmax)
                lmax = probs[i].val;
        double s = 0.0;
        for (int i = 0; i < n; i++) {
            probs[i].val = expf(probs[i].val - lmax);
            s += probs[i].val;
        }
        float inv = 1.0f / (float) s;
        for (int i = 0; i < n; i++)
            probs[i].val *= inv;
        if (top_p < 1.0f) /* src/model.c:275-276 */
            sort_desc(probs, n);
        res->path = BMO_PATH_K;
        int32_t t = filter_and_sample(probs, n, 0, top_p, 0, u, res);
        res->token = t;
        return t;
    }

    /* fallback: extraction by min_p only (src/model.c:286-293) */
    int n = 0;
    for (int i = 0; i < V; i++)
        if (logits[i] >= thr) {
            probs[n].id = i;
            probs[n].val = logits[i];
            n++;
        }
    res->n_cand = n;
    res->thresh = thr;
    if (n == 0) { /* argmax guard (src/model.c:296-303) */
        int32_t best = 0;
        for (int i = 1; i < V; i++)
            if (logits[i] > logits[best])
                best = i;
        res->path = BMO_PATH_FULL_GUARD;
        res->token = best;
        return best;
    }
    /* softmax against the global max (src/model.c:306-313) */
    double s = 0.0;
    for (int i = 0; i < n; i++) {
        probs[i].val = expf(probs[i].val - mx);
        s += probs[i].val;
    }
    float inv = 1.0f / (float) s;
    for (int i = 0; i < n; i++)
        probs[i].val *= inv;

    /* no sort when nothing truncates (src/model.c:319-320) */
    if (top_p >= 1.0f && (top_k <= 0 || top_k >= n)) {
        res->path = BMO_PATH_LAZY;
        int32_t t = filter_and_sample(probs, n, 0, top_p, top_k, u, res);
        res->token = t;
        return t;
    }
    /* top-256 partial sort (src/model.c:327-356) */
    if (top_p < 1.0f && n > PARTIAL_K) {
        bmo_cand_t top[PARTIAL_K];
        heap_select(top, probs, n, PARTIAL_K);
        sort_desc(top, PARTIAL_K);
        double cs = 0.0;
        for (int i = 0; i < PARTIAL_K; i++) {
            cs += top[i].val;
            if (cs >= top_p) {
                res->path = BMO_PATH_PARTIAL;
                int32_t t = filter_and_sample(top, PARTIAL_K, 0, top_p, top_k,
                                              u, res);
                res->token = t;
                return t;
            }
        }
    }
    /* full sort (src/model.c:359-360) */
    sort_desc(probs, n);
    res->path = BMO_PATH_FULL;
    int32_t t = filter_and_sample(probs, n, 0, top_p, top_k, u, res);
    res->token = t;
    return t;
}

int32_t bmo_sample_row(const float *logits, int V, const int32_t *history,
                       int history_len, float penalty, float temp, float min_p,
                       float top_p, int top_k, float u, float *work,
                       bmo_cand_t *probs, uint64_t *visited,
                       bmo_result_t *res)
{
    memcpy(work, logits, (size_t) V * sizeof(float));
    bmo_apply_penalty(work, V, history, history_len, penalty, visited);
    return bmo_sample_advanced(work, V, temp, min_p, top_p, top_k, u, probs,
                               res);
}

/* ---- batched driver (row-parallel pthreads) ----------------------------- */
typedef struct {
    const float *logits;
    int B, V;
    int64_t ld;
    const int32_t *hist;
    const int64_t *hist_off;
    const float *temp, *penalty, *min_p, *top_p;
    const int32_t *top_k;
    const float *uniform;
    int32_t *out_id;
    float *out_prob;
    bmo_result_t *res;
    int n_threads, tid, failed;
} batch_job_t;

static void *batch_worker(void *arg)
{
    batch_job_t *j = (batch_job_t *) arg;
    int V = j->V;
    float *work = (float *) malloc((size_t) V * sizeof(float));
    bmo_cand_t *probs = (bmo_cand_t *) malloc((size_t) V * sizeof(bmo_cand_t));
    uint64_t *vis = (uint64_t *) malloc(((size_t) V + 63) / 64 * 8);
    if (!work || !probs || !vis) {
        j->failed = 1;
        free(work);
        free(probs);
        free(vis);
        return NULL;
    }
    for (int r = j->tid; r < j->B; r += j->n_threads) {
        const int32_t *h = NULL;
        int hl = 0;
        if (j->hist && j->hist_off) {
            h = j->hist + j->hist_off[r];
            hl = (int) (j->hist_off[r + 1] - j->hist_off[r]);
        }
        bmo_result_t rr;
        int32_t t = bmo_sample_row(j->logits + (int64_t) r * j->ld, V, h, hl,
                                   j->penalty[r], j->temp[r], j->min_p[r],
                                   j->top_p[r], j->top_k[r], j->uniform[r],
                                   work, probs, vis, &rr);
        j->out_id[r] = t;
        if (j->out_prob)
            j->out_prob[r] = rr.prob;
        if (j->res)
            j->res[r] = rr;
    }
    free(work);
    free(probs);
    free(vis);
    return NULL;
}

int bmo_sample_batch(const float *logits, int B, int V, int64_t ld,
                     const int32_t *hist, const int64_t *hist_off,
                     const float *temp, const float *penalty,
                     const float *min_p, const float *top_p,
                     const int32_t *top_k, const float *uniform,
                     int32_t *out_id, float *out_prob, bmo_result_t *res,
                     int n_threads)
{
    if (n_threads < 1)
        n_threads = 1;
    if (n_threads > B)
        n_threads = B > 0 ? B : 1;
    batch_job_t *jobs = (batch_job_t *) calloc((size_t) n_threads,
                                               sizeof(batch_job_t));
    pthread_t *th = (pthread_t *) calloc((size_t) n_threads,
                                         sizeof(pthread_t));
    if (!jobs || !th) {
        free(jobs);
        free(th);
        return -1;
    }
    for (int t = 0; t < n_threads; t++) {
        batch_job_t j = {logits, B, V, ld, hist, hist_off, temp, penalty,
                         min_p, top_p, top_k, uniform, out_id, out_prob,
                         res, n_threads, t, 0};
        jobs[t] = j;
    }
    int rc = 0;
    if (n_threads == 1) {
        batch_worker(&jobs[0]);
    } else {
        for (int t = 0; t < n_threads; t++)
            if (pthread_create(&th[t], NULL, batch_worker, &jobs[t]) != 0) {
                batch_worker(&jobs[t]); /* run inline if no thread */
                th[t] = 0;
            }
        for (int t = 0; t < n_threads; t++)
            if (th[t])
                pthread_join(th[t], NULL);
    }
    for (int t = 0; t < n_threads; t++)
        rc |= jobs[t].failed;
    free(jobs);
    free(th);
    return rc ? -1 : 0;
}

/* ---- reference RNG: src/utils.c:117-140 --------------------------------- */
void bmo_rng_seed(uint64_t *state, uint64_t seed)
{
    *state = seed ? seed : 0x853c49e6748fea9bULL;
}

uint64_t bmo_rng_next(uint64_t *state)
{
    uint64_t x = *state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return x * 0x2545F4914F6CDD1DULL;
}

float bmo_rng_float(uint64_t *state)
{
    return (float) (bmo_rng_next(state) >> 11) * (1.0f / 9007199254740992.0f);
}
