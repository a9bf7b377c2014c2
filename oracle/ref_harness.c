/*
 * Reference harness (TEST INFRASTRUCTURE ONLY).
 *
 * Builds the reference's own sampler, unmodified, into oracle/_ref/ so the
 * C restatement in sampler_oracle.c (and through it the CUDA path) can be
 * pinned against it.  The reference's src/model.c is compiled as part of this
 * translation unit, taken from where it lies in the reference tree (the
 * include path is set by oracle/Makefile); nothing from it is copied into this
 * repository.  rng_float is redirected to a function that returns the uniform
 * supplied by the caller and counts the calls, which is the only change to
 * the reference's code path.
 *
 * The penalty block is inline in model_forward_step (src/model.c:1268-1305),
 * which needs a loaded model, so bm_ref_sample_row restates those few lines
 * (same bitset dedup, protected ids and in-place update) before calling the
 * reference's static sample_advanced (src/model.c:135-361).
 */
#define rng_float bm_ref_harness_uniform
#include "model.c"
#undef rng_float

static __thread float g_uniform;
static __thread int g_calls;

float bm_ref_harness_uniform(void)
{
    g_calls++;
    return g_uniform;
}

/* Returns the sampled id; *consumed = number of rng_float() calls (0 or 1);
 * *prob = value stored for that id in the reference's probs array (1.0 for
 * greedy and argmax-guard rows).  `logits` is modified in place, as the
 * reference does.  `probs` must hold V entries, `visited` (V+63)/64 words. */
int bm_ref_sample_row(float *logits, int V, const int *history,
                      int history_len, float penalty, float temp, float min_p,
                      float top_p, int top_k, float u, int *consumed,
                      float *prob, token_prob_t *probs, uint64_t *visited)
{
    static const int prot[4] = {TOKEN_EOS, TOKEN_NL, TOKEN_NLNL, TOKEN_PERIOD};
    memset(visited, 0, (((size_t) V + 63) / 64) * sizeof(uint64_t));
    for (int i = 0; i < history_len; i++) {
        int id = history[i];
        if (id < 0 || id >= V)
            continue;
        if (visited[id / 64] & (1ULL << (id % 64)))
            continue;
        visited[id / 64] |= (1ULL << (id % 64));
        int is_prot = 0;
        for (int p = 0; p < 4; p++)
            if (prot[p] == id)
                is_prot = 1;
        if (!is_prot && penalty > 0.0f) {
            if (logits[id] > 0)
                logits[id] /= penalty;
            else
                logits[id] *= penalty;
        }
    }
    for (int i = 0; i < V; i++)
        probs[i].id = -1;
    g_uniform = u;
    g_calls = 0;
    int t = sample_advanced(logits, V, temp, min_p, top_p, top_k, probs);
    *consumed = g_calls;
    *prob = 1.0f;
    if (g_calls) {
        for (int i = 0; i < V; i++)
            if (probs[i].id == t) {
                *prob = probs[i].val;
                break;
            }
    }
    return t;
}

int bm_ref_sizeof_token_prob(void)
{
    return (int) sizeof(token_prob_t);
}

/* Row-parallel driver over the reference sampler for the CPU baseline: rows
 * [B x ld], per-row knobs, CSR histories (may be NULL), one uniform per row.
 * Each thread owns a logits copy, a probs buffer and a bitset, so the
 * reference's shared model buffers are not needed.  Returns 0 or -1. */
#include <pthread.h>
typedef struct {
    const float *logits; int B, V; long long ld;
    const int *hist; const long long *off;
    const float *temp, *penalty, *min_p, *top_p; const int *top_k;
    const float *u; int *out; int nt, tid, failed;
} ref_job_t;

static void *ref_worker(void *arg)
{
    ref_job_t *j = (ref_job_t *) arg;
    float *row = malloc((size_t) j->V * sizeof(float));
    token_prob_t *probs = malloc((size_t) j->V * sizeof(token_prob_t));
    uint64_t *vis = malloc(((size_t) j->V + 63) / 64 * 8);
    if (!row || !probs || !vis) {
        j->failed = 1;
        free(row); free(probs); free(vis);
        return NULL;
    }
    for (int r = j->tid; r < j->B; r += j->nt) {
        memcpy(row, j->logits + (long long) r * j->ld, (size_t) j->V * sizeof(float));
        const int *h = j->hist ? j->hist + j->off[r] : NULL;
        int hl = j->hist ? (int) (j->off[r + 1] - j->off[r]) : 0;
        int c; float p;
        j->out[r] = bm_ref_sample_row(row, j->V, h, hl, j->penalty[r], j->temp[r],
                                      j->min_p[r], j->top_p[r], j->top_k[r], j->u[r],
                                      &c, &p, probs, vis);
    }
    free(row); free(probs); free(vis);
    return NULL;
}

int bm_ref_sample_batch(const float *logits, int B, int V, long long ld,
                        const int *hist, const long long *off, const float *temp,
                        const float *penalty, const float *min_p, const float *top_p,
                        const int *top_k, const float *u, int *out, int n_threads)
{
    if (n_threads < 1) n_threads = 1;
    if (n_threads > B) n_threads = B > 0 ? B : 1;
    ref_job_t *jobs = calloc((size_t) n_threads, sizeof(ref_job_t));
    pthread_t *th = calloc((size_t) n_threads, sizeof(pthread_t));
    if (!jobs || !th) { free(jobs); free(th); return -1; }
    int rc = 0;
    for (int t = 0; t < n_threads; t++) {
        ref_job_t jb = {logits, B, V, ld, hist, off, temp, penalty, min_p, top_p, top_k,
                        u, out, n_threads, t, 0};
        jobs[t] = jb;
        if (pthread_create(&th[t], NULL, ref_worker, &jobs[t]) != 0) {
            ref_worker(&jobs[t]);
            th[t] = 0;
        }
    }
    for (int t = 0; t < n_threads; t++) {
        if (th[t]) pthread_join(th[t], NULL);
        rc |= jobs[t].failed;
    }
    free(jobs); free(th);
    return rc ? -1 : 0;
}

/*
 * The reference's logits producer, unmodified: the final RMSNorm
 * (src/model.c:1225) and the ternary BitLinear lm_head (src/model.c:1257,
 * the single-node branch), through the kernel table dispatch_init() fills
 * for this host (AVX2 on x86-64 with AVX2+FMA, src/dispatch.c:31-38).  Row b
 * of x [B x d] gives logits out[b * ld .. + V).  When xq_out / inv_out are
 * given, the BitLinear's own prepare step (src/arch/avx2.c:276-318) is run
 * once more to expose its int8 activations and 1 / (scale_x * w_scale).
 * n_threads > 0 sizes the reference's thread pool (bm_set_threads).
 * Returns 1 when the AVX2 kernels ran, 0 for the scalar ones.
 */
static pthread_once_t g_disp_once = PTHREAD_ONCE_INIT;
static int g_pool_threads = -1;

static void bm_ref_disp_init(void)
{
    dispatch_init();
    init_lut();
}

int bm_ref_ternary_lmhead(const float *x, int B, int d, const float *norm_f,
                          const float *lmh_norm, const uint8_t *packed, int V,
                          float w_scale, float *out, long long ld, int8_t *xq_out,
                          float *inv_out, int n_threads)
{
    pthread_once(&g_disp_once, bm_ref_disp_init);
    if (n_threads > 0 && n_threads != g_pool_threads) {
        bm_set_threads(n_threads);
        g_pool_threads = n_threads;
    }
    tensor_t w;
    memset(&w, 0, sizeof(w));
    w.packed_data = packed;
    w.rows = V;
    w.cols = d;
    w.n_elements = (size_t) V * (size_t) d;
    w.is_bitnet = true;
    w.scale = w_scale;
    tensor_t nw;
    memset(&nw, 0, sizeof(nw));
    nw.data = lmh_norm;
    nw.rows = 1;
    nw.cols = d;
    nw.n_elements = (size_t) d;
    float *feat = malloc((size_t) d * sizeof(float));
    float *xn = malloc((size_t) d * sizeof(float));
    int8_t *xq = malloc((size_t) d);
    if (!feat || !xn || !xq) {
        free(feat); free(xn); free(xq);
        return -1;
    }
    for (int b = 0; b < B; b++) {
        const float *xr = x + (size_t) b * d;
        if (norm_f) {
            g_kernels.rms_norm(xr, d, norm_f, feat);
            xr = feat;
        }
        g_kernels.bitlinear_forward(xr, d, &w, &nw, out + (size_t) b * ld, xn, xq);
        if (xq_out)
            memcpy(xq_out + (size_t) b * d, xq, (size_t) d);
        if (inv_out && g_kernels.bitlinear_prepare) {
            const float sx = g_kernels.bitlinear_prepare(xr, d, &nw, xn, xq);
            inv_out[b] = 1.0f / (sx * w_scale);
        }
    }
    free(feat); free(xn); free(xq);
    return strcmp(g_kernels.name, "avx2") == 0 ? 1 : 0;
}

/*
 * The reference's own model loader (src/model.c:477-783) on a packed model
 * file, then its logits producer on caller-supplied last-layer outputs: the
 * final RMSNorm and the ternary lm_head read from the loaded model
 * (src/model.c:1225, 1257).  Returns -1 when model_load rejects the file,
 * else the vocabulary size; *d_model_out receives d_model.  `out` holds
 * B x ld floats (ld >= vocab).
 */
int bm_ref_model_lmhead(const char *path, const float *x, int B, float *out, long long ld,
                        int *d_model_out)
{
    pthread_once(&g_disp_once, bm_ref_disp_init);
    bitmamba_model_t m;
    memset(&m, 0, sizeof(m));
    if (!model_load(&m, path))
        return -1;
    const int d = m.config.d_model, V = m.config.vocab_size;
    if (d_model_out)
        *d_model_out = d;
    if (x && out) {
        float *feat = malloc((size_t) d * sizeof(float));
        float *xn = malloc((size_t) d * sizeof(float));
        int8_t *xq = malloc((size_t) d);
        for (int b = 0; feat && xn && xq && b < B; b++) {
            g_kernels.rms_norm(x + (size_t) b * d, d, m.norm_f.data, feat);
            g_kernels.bitlinear_forward(feat, d, &m.lm_head, &m.lm_head_norm,
                                        out + (size_t) b * ld, xn, xq);
        }
        free(feat); free(xn); free(xq);
    }
    model_free(&m);
    return V;
}
