// Decode-step token sampler for sm_100a: one persistent CTA per SM, one logits
// row at a time resident in shared memory.
//
// Per row (reference: jserv/bitmamba.c src/model.c:1268-1307, 37-361):
//   load      bulk async copy of the row's 16-byte-aligned interior into shared
//             memory in NCHUNK pieces (one mbarrier each), ragged head/tail by
//             plain loads, next row of this CTA prefetched into L2.  The
//             repetition penalty is applied while the row is consumed, from a
//             bitset of the row's distinct history ids (src/model.c:1277-1304),
//             and the pass computes max / min of the scaled logits
//             (src/model.c:156-163) or the greedy argmax (src/model.c:144-154).
//   top_k     1 <= top_k <= 256: the reference's 128-bucket histogram cut
//             (src/model.c:181-214), extraction, exact emulation of its
//             min-heap (heap layout decides the CDF walk order), survivor
//             softmax, stable descending sort, nucleus cut and draw.
//   full      other top_k: expf against the global max into shared memory with
//             a logit-bucket count histogram, then either the id-order walk
//             (src/model.c:319-320) or a select in (prob desc, id asc) order
//             (the order the reference's stable qsort produces) through
//             estimated windows verified by exact passes.  Rows where the
//             reference's top-256 heap path applies and ties make its layout
//             visible are replayed exactly (src/model.c:327-356).
//
// Arithmetic that decides ids is done with the reference's fp32 operations
// (no contraction: explicit __fmul_rn/__fadd_rn/__fdiv_rn), sums in fp64.
#include "bm_kernel.cuh"

#include <cfloat>
#include <climits>

namespace bmk {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr unsigned long long WAIT_NS = 2000000000ull;  // bounded mbarrier waits: 2 s
constexpr float DCAP = 40.0f;                // bucket range cap (e^-40 ~ 4e-18)
constexpr float MAGIC = 12582912.0f;         // 1.5 * 2^23: round-to-int trick

// GPT-2 ids the reference never penalises (src/bitmamba.h:21-24).
__device__ __forceinline__ bool protected_id(int id) {
    return id == 50256 || id == 198 || id == 628 || id == 13;
}

struct __align__(16) Vars {
    float mx, thr, xmin, inv_temp;
    float temp, penalty, min_p, top_p;
    float log_min_p, u, inv_sum, dmax;
    int top_k, greedy, pen, k;
    int sh, nslots, s_int0, s_int1;
    int res_id, n_cand, n_final, path;
    int consumed, kcut, kcnt, list_n;
    int bhat, cnt_above, last_cand, fail;
    int sel_j, sel_found, sel_tie, own;
    float res_p, w, inv_w, pad0;
    double S, above, cs, aux;
};

struct Layout {
    size_t mbar, red, vars, bits, scr, row, total;
    int nbw;
};

__host__ __device__ inline size_t r16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline Layout layout(int V) {
    Layout L;
    size_t o = 0;
    L.mbar = o;
    o += NCHUNK * 8;
    L.red = o;
    o += 1024;
    L.vars = o;
    o += r16(sizeof(Vars));
    L.nbw = (V + 3 + 31) / 32 + 1;
    L.bits = o;
    o += r16((size_t)L.nbw * 4);
    L.scr = o;
    o += SCRATCH;
    L.row = o;
    o += r16((size_t)(V + 8) * 4);
    L.total = o;
    return L;
}

// ---------------------------------------------------------------- PTX glue --
__device__ __forceinline__ uint32_t sa(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *b) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(sa(dst)),
        "l"(src), "r"(bytes), "r"(sa(b))
        : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(sa(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Wait for a phase with a wall-clock bound; false when the bound expired.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity) {
    if (mbar_try(b, parity)) return true;
    const unsigned long long t0 = gtimer();
    for (unsigned it = 0; it < (1u << 30); ++it) {
        if (mbar_try(b, parity)) return true;
        if (gtimer() - t0 > WAIT_NS) return false;
    }
    return false;
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// --------------------------------------------------------- small helpers --
// (int)t as x86 cvttss2si computes it (NaN / out of range -> INT_MIN), the
// conversion the reference's bucket index uses on x86 (src/model.c:188).
__device__ __forceinline__ int x86_cvtt(float t) {
    if (!(t < 2147483648.0f && t >= -2147483648.0f)) return INT_MIN;
    return __float2int_rz(t);
}
__device__ __forceinline__ float penalize(float l, float pen) {
    return (l > 0.0f) ? __fdiv_rn(l, pen) : __fmul_rn(l, pen);
}
__device__ __forceinline__ unsigned long long canon_key(float p, int id) {
    // ascending key order == probability descending, id ascending (p >= 0)
    return ((unsigned long long)(~__float_as_uint(p)) << 32) | (unsigned)id;
}
__device__ __forceinline__ float key_p(unsigned long long k) {
    return __uint_as_float(~(unsigned)(k >> 32));
}
__device__ __forceinline__ int key_id(unsigned long long k) { return (int)(unsigned)(k & 0xffffffffu); }

template <class T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fminf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}
__device__ __forceinline__ int warp_imax(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(FULL, v, o));
    return v;
}
__device__ __forceinline__ int warp_imin(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(FULL, v, o));
    return v;
}
// inclusive warp scan
template <class T>
__device__ __forceinline__ T warp_iscan(T v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T n = __shfl_up_sync(FULL, v, o);
        if (lane >= o) v += n;
    }
    return v;
}
// (value, index) with "larger value, then smaller index" preference; idx
// INT_MAX means none.
__device__ __forceinline__ void argmax_combine(float &v, int &i, float v2, int i2) {
    bool take = (i == INT_MAX) ? (i2 != INT_MAX)
                               : (i2 != INT_MAX && (v2 > v || (v2 == v && i2 < i)));
    if (take) { v = v2; i = i2; }
}
__device__ __forceinline__ void warp_argmax(float &v, int &i) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        float v2 = __shfl_xor_sync(FULL, v, o);
        int i2 = __shfl_xor_sync(FULL, i, o);
        argmax_combine(v, i, v2, i2);
    }
}

// Block-level reductions.  `rd` holds NW doubles, `ri` NW ints (two arrays
// laid side by side in the red area).  Every thread gets the result.
struct Red {
    double *d;
    int *i;
    float *f;
};

__device__ __forceinline__ double block_sum_d(double v, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) r.d[warp] = v;
    __syncthreads();
    double t = r.d[lane];
    t = warp_sum(t);
    __syncthreads();
    return t;
}
__device__ __forceinline__ int block_sum_i(int v, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) r.i[warp] = v;
    __syncthreads();
    int t = r.i[lane];
    t = warp_sum(t);
    __syncthreads();
    return t;
}
__device__ __forceinline__ int block_max_i(int v, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_imax(v);
    if (lane == 0) r.i[warp] = v;
    __syncthreads();
    int t = warp_imax(r.i[lane]);
    __syncthreads();
    return t;
}
__device__ __forceinline__ int block_min_i(int v, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_imin(v);
    if (lane == 0) r.i[warp] = v;
    __syncthreads();
    int t = warp_imin(r.i[lane]);
    __syncthreads();
    return t;
}
__device__ __forceinline__ void block_maxmin_f(float &mx, float &mn, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    mx = warp_max(mx);
    mn = warp_min(mn);
    if (lane == 0) { r.f[warp] = mx; r.f[NW + warp] = mn; }
    __syncthreads();
    mx = warp_max(r.f[lane]);
    mn = warp_min(r.f[NW + lane]);
    __syncthreads();
}
__device__ __forceinline__ void block_argmax(float &v, int &i, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    warp_argmax(v, i);
    if (lane == 0) { r.f[warp] = v; r.i[warp] = i; }
    __syncthreads();
    v = r.f[lane];
    i = r.i[lane];
    warp_argmax(v, i);
    __syncthreads();
}
// exclusive block scan of doubles; returns exclusive prefix, sets total
__device__ __forceinline__ double block_xscan_d(double v, double &total, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double inc = warp_iscan(v, lane);
    if (lane == 31) r.d[warp] = inc;
    __syncthreads();
    double w = r.d[lane];
    double winc = warp_iscan(w, lane);
    double woff = __shfl_sync(FULL, winc - w, warp);
    total = __shfl_sync(FULL, winc, 31);
    __syncthreads();
    return woff + inc - v;
}
__device__ __forceinline__ int block_xscan_i(int v, int &total, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = warp_iscan(v, lane);
    if (lane == 31) r.i[warp] = inc;
    __syncthreads();
    int w = r.i[lane];
    int winc = warp_iscan(w, lane);
    int woff = __shfl_sync(FULL, winc - w, warp);
    total = __shfl_sync(FULL, winc, 31);
    __syncthreads();
    return woff + inc - v;
}

// In-place ascending bitonic sort of n <= cap 64-bit keys in shared memory,
// padded to a power of two with ~0.  All threads call it.
__device__ void block_sort_u64(unsigned long long *a, int n, int cap) {
    int P = 1;
    while (P < n) P <<= 1;
    if (P > cap) P = cap;
    for (int i = n + threadIdx.x; i < P; i += NT) a[i] = ~0ull;
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int t = threadIdx.x; t < (P >> 1); t += NT) {
                int i = ((t / j) * (j << 1)) + (t % j);
                int l = i + j;
                bool up = ((i & k) == 0);
                unsigned long long x = a[i], y = a[l];
                if ((x > y) == up) { a[i] = y; a[l] = x; }
            }
            __syncthreads();
        }
    }
}

// Min-heap sift-down on parallel arrays, exactly src/model.c:50-66
// (strict '<', left child checked first).
__device__ void heap_down(float *hv, int *hi, int n, int i) {
    for (;;) {
        int m = i, a = 2 * i + 1, b = 2 * i + 2;
        if (a < n && hv[a] < hv[m]) m = a;
        if (b < n && hv[b] < hv[m]) m = b;
        if (m == i) return;
        float tv = hv[i]; hv[i] = hv[m]; hv[m] = tv;
        int ti = hi[i]; hi[i] = hi[m]; hi[m] = ti;
        i = m;
    }
}
// Floyd heapify (src/model.c:242-243, 330-331) by one warp, level by level:
// nodes of one level root disjoint subtrees, and every deeper node has a
// larger index, so this is the reference's sequential order.
__device__ void warp_heapify(float *hv, int *hi, int k, int lane) {
    int last = k / 2 - 1;
    if (last < 0) return;
    int top = 31 - __clz(last + 1);
    for (int lev = top; lev >= 0; --lev) {
        int a = (1 << lev) - 1, b = min((1 << (lev + 1)) - 2, last);
        for (int i = a + lane; i <= b; i += 32) heap_down(hv, hi, k, i);
        __syncwarp();
    }
}

// ------------------------------------------------------------ the kernel --
struct Ctx {
    Params P;
    Layout L;
    uint64_t *mbar;
    Red red;
    Vars *v;
    uint32_t *bits;
    unsigned char *scr;
    float *row;  // 16-byte aligned; element e lives at row[e + sh]
    const float *g;
    int rowid;
    uint32_t parity;
};

// Walk a list (in shared memory, n entries, key form) from a starting mass:
// finds the first j with start + cum(j) >= T (mode 0), > T (mode 1).  Runs on
// one warp; results go to vars (sel_found/sel_j, cs).
__device__ void warp_walk(const unsigned long long *keys, int n, double start, int mode,
                          double T, Vars *v, int lane) {
    const int per = (n + 31) / 32;
    const int b = lane * per, e = min(n, b + per);
    double s = 0.0;
    for (int j = b; j < e; ++j) s += (double)key_p(keys[j]);
    double inc = warp_iscan(s, lane);
    double pre = start + (inc - s);
    int hit = INT_MAX;
    double hit_cs = 0.0;
    if (b < e) {
        double cs = pre;
        for (int j = b; j < e; ++j) {
            cs += (double)key_p(keys[j]);
            bool ok = (mode == 0) ? (cs >= T) : (cs > T);
            if (ok) { hit = j; hit_cs = cs; break; }
        }
    }
    int best = warp_imin(hit);
    if (best != INT_MAX) {
        int owner = (best / per);
        double cs = __shfl_sync(FULL, hit_cs, owner);
        if (lane == 0) { v->sel_found = 1; v->sel_j = best; v->cs = cs; }
    } else if (lane == 0) {
        v->sel_found = 0;
        v->sel_j = n;
        v->cs = start + __shfl_sync(FULL, inc, 31);
    }
    if (best == INT_MAX) (void)__shfl_sync(FULL, inc, 31);
}

// ---- full-vocabulary select ------------------------------------------------
// Candidates hold e = expf(l - max) >= 0 in the row buffer (non-candidates
// -1).  p = e * inv_sum.  Canonical order: p descending, id ascending (the
// order the reference's stable qsort leaves the id-ordered candidates in).
struct Sel {
    int found;  // 1 = crossing found; 0 = beyond the last candidate
    int pos;    // position in canonical order (0-based)
    int id;
    float p;
    double cs;  // cumulative mass through `pos`
    int tie;    // another candidate has the same p
};

struct PassOut {
    double above, in_mass;
    int cnt_above, in_cnt;
};

// One exact pass over the candidates for the probability window [plo, phi]:
// mass / count strictly above phi, mass / count inside, and the inside
// elements collected into `list` as canonical keys (only the first WCAP).
__device__ PassOut exact_pass(Ctx &c, float plo, float phi, unsigned long long *list) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Vars *v = c.v;
    const float inv_sum = v->inv_sum;
    const int sh = v->sh, nslots = v->nslots;
    if (threadIdx.x == 0) v->list_n = 0;
    __syncthreads();
    double acc_up = 0.0, acc_in = 0.0;
    int cnt_up = 0;
    const float4 *r4 = reinterpret_cast<const float4 *>(c.row);
    for (int base = warp * 32; base < nslots; base += NT) {
        int s = base + lane;
        float4 e4 = make_float4(-1.f, -1.f, -1.f, -1.f);
        if (s < nslots) e4 = r4[s];
        float ev[4] = {e4.x, e4.y, e4.z, e4.w};
        float gu0 = 0.f, gu1 = 0.f, gi0 = 0.f, gi1 = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float e = ev[q];
            bool cand = (e >= 0.0f);
            float p = __fmul_rn(cand ? e : 0.0f, inv_sum);
            bool up = cand && (p > phi);
            bool in = cand && !up && (p >= plo);
            if (q < 2) { gu0 = __fadd_rn(gu0, up ? p : 0.f); gi0 = __fadd_rn(gi0, in ? p : 0.f); }
            else { gu1 = __fadd_rn(gu1, up ? p : 0.f); gi1 = __fadd_rn(gi1, in ? p : 0.f); }
            cnt_up += up;
            unsigned m = __ballot_sync(FULL, in);
            if (m) {
                int leader = __ffs(m) - 1;
                int bpos = 0;
                if (lane == leader) bpos = atomicAdd(&v->list_n, __popc(m));
                bpos = __shfl_sync(FULL, bpos, leader);
                if (in) {
                    int pos = bpos + __popc(m & ((1u << lane) - 1));
                    if (pos < WCAP) list[pos] = canon_key(p, 4 * s + q - sh);
                }
            }
        }
        acc_up += (double)__fadd_rn(gu0, gu1);
        acc_in += (double)__fadd_rn(gi0, gi1);
    }
    PassOut o;
    o.above = block_sum_d(acc_up, c.red);
    o.in_mass = block_sum_d(acc_in, c.red);
    o.cnt_above = block_sum_i(cnt_up, c.red);
    o.in_cnt = v->list_n;
    __syncthreads();
    return o;
}

// Ordered select inside one probability value: the j-th (0-based, id order)
// candidate whose p equals `pv`.  Contiguous slot segments per thread.
__device__ int ordered_pick(Ctx &c, float pv, int j) {
    Vars *v = c.v;
    const float inv_sum = v->inv_sum;
    const int sh = v->sh, nslots = v->nslots;
    const int Q = (nslots + NT - 1) / NT;
    const int s0 = threadIdx.x * Q, s1 = min(nslots, s0 + Q);
    const float4 *r4 = reinterpret_cast<const float4 *>(c.row);
    int cnt = 0;
    for (int s = s0; s < s1; ++s) {
        float4 e4 = r4[s];
        float ev[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
            cnt += (ev[q] >= 0.0f) && (__fmul_rn(ev[q], inv_sum) == pv);
    }
    int tot;
    int ex = block_xscan_i(cnt, tot, c.red);
    if (threadIdx.x == 0) v->own = -1;
    __syncthreads();
    if (j >= ex && j < ex + cnt) {
        int k = ex;
        for (int s = s0; s < s1; ++s) {
            float4 e4 = r4[s];
            float ev[4] = {e4.x, e4.y, e4.z, e4.w};
            for (int q = 0; q < 4; ++q) {
                if ((ev[q] >= 0.0f) && (__fmul_rn(ev[q], inv_sum) == pv)) {
                    if (k == j) v->own = 4 * s + q - sh;
                    ++k;
                }
            }
        }
    }
    __syncthreads();
    int id = v->own;
    __syncthreads();
    return id;
}

// where the target lies relative to a window
enum { W_INSIDE = 0, W_HIGH = 1, W_LOW = 2 };
__device__ __forceinline__ int classify(const PassOut &o, int mode, double T, int m) {
    if (mode == 2) {
        if (m < o.cnt_above) return W_HIGH;
        if (m >= o.cnt_above + o.in_cnt) return W_LOW;
        return W_INSIDE;
    }
    bool hi = (mode == 0) ? (o.above >= T) : (o.above > T);
    if (hi && o.cnt_above > 0) return W_HIGH;
    double tot = o.above + o.in_mass;
    bool reach = (mode == 0) ? (tot >= T) : (tot > T);
    return reach ? W_INSIDE : W_LOW;
}

// Sort the collected window and find the crossing inside it.  Returns 1 and
// fills `out` on success; 0 when the walk disagrees with the pass sums.
__device__ int finish_window(Ctx &c, unsigned long long *list, const PassOut &o, int mode,
                             double T, int m, Sel &out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Vars *v = c.v;
    const int n = o.in_cnt;
    block_sort_u64(list, n, WCAP);
    if (warp == 0) {
        if (mode == 2) {
            int j = m - o.cnt_above;
            const int per = (j + 1 + 31) / 32;
            const int bb = lane * per, ee = min(j + 1, bb + per);
            double s = 0.0;
            for (int q = bb; q < ee; ++q) s += (double)key_p(list[q]);
            s = warp_sum(s);
            if (lane == 0) { v->sel_found = 1; v->sel_j = j; v->cs = o.above + s; }
        } else {
            warp_walk(list, n, o.above, mode, T, v, lane);
        }
    }
    __syncthreads();
    int f = v->sel_found, j = v->sel_j;
    double cs = v->cs;
    __syncthreads();
    if (!f) return 0;
    unsigned long long kk = list[j];
    out.found = 1;
    out.pos = o.cnt_above + j;
    out.id = key_id(kk);
    out.p = key_p(kk);
    out.cs = cs;
    out.tie = (j > 0 && key_p(list[j - 1]) == out.p) || (j + 1 < n && key_p(list[j + 1]) == out.p);
    __syncthreads();
    return 1;
}

// The last candidate in canonical order (smallest p, then largest id) and
// whether its probability is shared.
__device__ Sel last_canon(Ctx &c) {
    Vars *v = c.v;
    const float inv_sum = v->inv_sum;
    const int sh = v->sh, nslots = v->nslots;
    const float4 *r4 = reinterpret_cast<const float4 *>(c.row);
    float pmin = __int_as_float(0x7f800000);
    for (int s = threadIdx.x; s < nslots; s += NT) {
        float4 e4 = r4[s];
        float ev[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (ev[q] >= 0.0f) pmin = fminf(pmin, __fmul_rn(ev[q], inv_sum));
    }
    float dummy = 0.f;
    block_maxmin_f(dummy, pmin, c.red);
    int idmax = -1, cnt = 0;
    for (int s = threadIdx.x; s < nslots; s += NT) {
        float4 e4 = r4[s];
        float ev[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (ev[q] >= 0.0f && __fmul_rn(ev[q], inv_sum) == pmin) {
                idmax = max(idmax, 4 * s + q - sh);
                ++cnt;
            }
    }
    idmax = block_max_i(idmax, c.red);
    cnt = block_sum_i(cnt, c.red);
    Sel out;
    out.found = 0;
    out.pos = v->n_cand - 1;
    out.id = idmax;
    out.p = pmin;
    out.cs = 0.0;
    out.tie = cnt > 1;
    return out;
}

// mode 0: first position with cs >= T; mode 1: cs > T; mode 2: position m.
// Window estimate from the count histogram, verified by exact passes,
// widened on a miss, bisected in probability when too dense.
__device__ Sel select_canon(Ctx &c, int mode, double T, int m) {
    Vars *v = c.v;
    const uint32_t *hcnt = reinterpret_cast<const uint32_t *>(c.scr);
    unsigned long long *list = reinterpret_cast<unsigned long long *>(c.scr + NB * 4);
    const float inv_sum = v->inv_sum, w = v->w;
    const int n_cand = v->n_cand;
    const float PINF = __int_as_float(0x7f800000);
    Sel out;
    out.found = 0; out.pos = n_cand - 1; out.id = -1; out.p = 0.f; out.cs = 0.0; out.tie = 0;

    // 1. estimate the crossing bucket from counts x bucket-centre probability
    const int b0 = 2 * threadIdx.x, b1 = b0 + 1;
    const int c0 = (int)hcnt[b0], c1 = (int)hcnt[b1];
    const double m0 = (double)c0 * (double)__fmul_rn(expf(-(float)b0 * w), inv_sum);
    const double m1 = (double)c1 * (double)__fmul_rn(expf(-(float)b1 * w), inv_sum);
    double mt;
    const double mex = block_xscan_d(m0 + m1, mt, c.red);
    int ct;
    const int cex = block_xscan_i(c0 + c1, ct, c.red);
    if (threadIdx.x == 0) v->bhat = NB - 1;
    __syncthreads();
    int hitb = INT_MAX;
    if (mode == 2) {
        if (m >= cex && m < cex + c0) hitb = b0;
        else if (m >= cex + c0 && m < cex + c0 + c1) hitb = b1;
    } else {
        bool h0 = (mode == 0) ? (mex + m0 >= T) : (mex + m0 > T);
        bool h1 = (mode == 0) ? (mex + m0 + m1 >= T) : (mex + m0 + m1 > T);
        if (h0) hitb = b0;
        else if (h1) hitb = b1;
    }
    if (hitb != INT_MAX) atomicMin(&v->bhat, hitb);
    __syncthreads();
    const int bh = v->bhat;
    __syncthreads();

    // 2. windows around the estimate, widening on a miss; [lo, hi] is the
    //    probability interval the crossing is known to lie in
    float lo = -1.0f, hi = PINF;
    const int deltas[3] = {0, 2, 16};
    PassOut o;
    bool dense = false;
    for (int a = 0; a < 3; ++a) {
        const int blo = max(0, bh - deltas[a]), bhi = min(NB - 1, bh + deltas[a]);
        float phi = (blo == 0) ? PINF : __fmul_rn(expf(-((float)blo - 0.5f) * w), inv_sum);
        float plo = (bhi == NB - 1) ? -1.0f : __fmul_rn(expf(-((float)bhi + 0.5f) * w), inv_sum);
        phi = fminf(phi, hi);
        plo = fmaxf(plo, lo);
        o = exact_pass(c, plo, phi, list);
        int cl = classify(o, mode, T, m);
        if (cl == W_INSIDE) {
            lo = plo; hi = phi;
            if (o.in_cnt <= WCAP) {
                if (finish_window(c, list, o, mode, T, m, out)) return out;
            } else {
                dense = true;
                break;
            }
        } else if (cl == W_HIGH) {
            lo = __uint_as_float(__float_as_uint(phi) + 1u);  // p > phi
        } else {
            if (plo <= 0.0f) {
                // nothing below the window: the target lies beyond the last
                // candidate (total mass under the target)
                out = last_canon(c);
                out.found = 0;
                out.cs = o.above + o.in_mass;
                return out;
            }
            hi = __uint_as_float(__float_as_uint(plo) - 1u);  // p < plo
            if (hi < 0.0f) hi = 0.0f;
        }
    }
    // 3. bisection on the probability bits of [lo, hi]
    (void)dense;
    for (int it = 0; it < 64; ++it) {
        unsigned ub = (hi == PINF) ? 0x3f800001u : __float_as_uint(hi);
        unsigned lb = (lo < 0.0f) ? 0u : __float_as_uint(lo);
        if (ub > 0x3f800001u) ub = 0x3f800001u;
        if (lb > ub) lb = ub;
        o = exact_pass(c, (lo < 0.0f) ? -1.0f : __uint_as_float(lb), __uint_as_float(ub), list);
        int cl = classify(o, mode, T, m);
        if (cl == W_INSIDE && o.in_cnt <= WCAP) {
            if (finish_window(c, list, o, mode, T, m, out)) return out;
        }
        if (cl == W_LOW && lb == 0u) {
            out = last_canon(c);
            out.found = 0;
            out.cs = o.above + o.in_mass;
            return out;
        }
        if (cl != W_INSIDE) {
            // the estimate drifted outside [lo, hi]; reopen the interval
            if (cl == W_HIGH) { lo = __uint_as_float(ub + 1u); hi = PINF; }
            else { hi = (lb == 0u) ? 0.0f : __uint_as_float(lb - 1u); lo = -1.0f; }
            continue;
        }
        if (lb == ub) {
            // more than WCAP candidates share one probability value: the
            // position inside the tie group is arithmetic, then the j-th id
            const float pv = __uint_as_float(ub);
            const int n = o.in_cnt;
            int j;
            if (mode == 2) {
                j = m - o.cnt_above;
            } else {
                j = 0;
                while (j < n - 1 && !((mode == 0) ? (o.above + (double)(j + 1) * pv >= T)
                                                  : (o.above + (double)(j + 1) * pv > T))) {
                    double need = (T - o.above) / (double)pv;
                    int jj = (int)need - 1;
                    j = (jj > j) ? jj : j + 1;
                    if (j > n - 1) j = n - 1;
                }
            }
            out.found = 1;
            out.pos = o.cnt_above + j;
            out.p = pv;
            out.cs = o.above + (double)(j + 1) * pv;
            out.tie = (n > 1);
            out.id = ordered_pick(c, pv, j);
            return out;
        }
        const unsigned mid = lb + (ub - lb) / 2;
        // upper half (mid, ub]
        PassOut u = exact_pass(c, __uint_as_float(mid + 1u), __uint_as_float(ub), list);
        int cu = classify(u, mode, T, m);
        if (cu == W_INSIDE) {
            lo = __uint_as_float(mid + 1u);
            hi = __uint_as_float(ub);
            if (u.in_cnt <= WCAP && finish_window(c, list, u, mode, T, m, out)) return out;
        } else {
            lo = (lb == 0u && lo < 0.0f) ? -1.0f : __uint_as_float(lb);
            hi = __uint_as_float(mid);
        }
    }
    if (threadIdx.x == 0) atomicOr(c.P.err, 2);
    return out;
}

// Exact replay of the reference's top-256 heap (src/model.c:327-356) over the
// candidates in id order, by one warp: heapify the first 256, then replace
// the root by every later candidate that is strictly greater.  The result is
// left in `outk` sorted as the stable qsort leaves it: probability
// descending, ties in heap-array order (low word = heap slot).
__device__ __noinline__ void replay_top256(Ctx &c, unsigned long long *outk, float *hv,
                                           int *hi) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Vars *v = c.v;
    const float inv_sum = v->inv_sum;
    const int sh = v->sh, V = c.P.V;
    if (warp == 0) {
        int filled = 0;
        for (int base = 0; base < V; base += 32) {
            const int id = base + lane;
            const float e = (id < V) ? c.row[id + sh] : -1.0f;
            const bool cand = e >= 0.0f;
            const float p = __fmul_rn(cand ? e : 0.0f, inv_sum);
            const unsigned mk = __ballot_sync(FULL, cand);
            bool rest = cand;
            if (filled < 256) {
                const int rank = __popc(mk & ((1u << lane) - 1));
                const int take = min(__popc(mk), 256 - filled);
                if (cand && rank < take) { hv[filled + rank] = p; hi[filled + rank] = id; }
                rest = cand && rank >= take;
                filled += take;
                __syncwarp();
                if (filled < 256) continue;
                if (filled - take < 256 && take > 0) warp_heapify(hv, hi, 256, lane);
            }
            const float root = hv[0];
            unsigned mr = __ballot_sync(FULL, rest && p > root);
            while (mr) {
                const int src = __ffs(mr) - 1;
                const float pb = __shfl_sync(FULL, p, src);
                const int ib = __shfl_sync(FULL, id, src);
                if (lane == 0 && pb > hv[0]) { hv[0] = pb; hi[0] = ib; heap_down(hv, hi, 256, 0); }
                __syncwarp();
                mr &= mr - 1;
            }
        }
        __syncwarp();
        for (int q = lane; q < 256; q += 32) outk[q] = canon_key(hv[q], q);
    }
    __syncthreads();
    block_sort_u64(outk, 256, 256);
}

// ------------------------------------------------------------ row passes --
// Pass 1: consume the freshly loaded row (waiting chunk by chunk), apply the
// penalty bitset, and reduce.  greedy: argmax of raw penalised logits.
__device__ void load_pass(Ctx &c, bool greedy, float &mx, float &xmin, float &gv, int &gi) {
    Vars *v = c.v;
    const int sh = v->sh, nslots = v->nslots, s0 = v->s_int0, s1 = v->s_int1;
    const int V = c.P.V;
    const bool pen = v->pen != 0;
    const float penalty = v->penalty, inv_temp = v->inv_temp;
    const bool scale = (inv_temp != 1.0f);
    const int nint = s1 - s0;
    unsigned waited = 0;
    float4 *r4 = reinterpret_cast<float4 *>(c.row);
    mx = -1e30f;
    xmin = __int_as_float(0x7f800000);
    gv = -1e9f;
    gi = INT_MAX;
    for (int s = threadIdx.x; s < nslots; s += NT) {
        float4 x;
        if (s >= s0 && s < s1) {
            int j = s - s0;
            int ch = (j * NCHUNK) / nint;
            if (((ch + 1) * nint) / NCHUNK <= j) ++ch;
            if (!((waited >> ch) & 1u)) {
                if (!mbar_wait(&c.mbar[ch], c.parity)) {
                    atomicOr(c.P.err, 1);
                    v->fail = 1;
                }
                waited |= 1u << ch;
            }
            x = r4[s];
        } else {
            float t[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                int e = 4 * s + q - sh;
                t[q] = (e >= 0 && e < V) ? __ldg(c.g + e) : 0.0f;
            }
            x = make_float4(t[0], t[1], t[2], t[3]);
            r4[s] = x;
        }
        float t[4] = {x.x, x.y, x.z, x.w};
        if (pen) {
            unsigned nib = (c.bits[s >> 3] >> ((s & 7) * 4)) & 0xfu;
            if (nib) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if ((nib >> q) & 1u) t[q] = penalize(t[q], penalty);
                r4[s] = make_float4(t[0], t[1], t[2], t[3]);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int e = 4 * s + q - sh;
            if (e < 0 || e >= V) continue;
            if (greedy) {
                if (t[q] > gv) { gv = t[q]; gi = e; }
            } else {
                float l = scale ? __fmul_rn(t[q], inv_temp) : t[q];
                mx = fmaxf(mx, l);
                xmin = fminf(xmin, l);
            }
        }
    }
}

// Argmax over the scaled (penalised) logits with the guard semantics of
// src/model.c:227-237 and 296-303: start from element 0, strict '>'.
// Reloads from global memory (the row buffer may hold probabilities).
__device__ int guard_argmax(Ctx &c) {
    Vars *v = c.v;
    const int V = c.P.V;
    const bool pen = v->pen != 0;
    const float penalty = v->penalty, inv_temp = v->inv_temp;
    const bool scale = (inv_temp != 1.0f);
    const int sh = v->sh;
    float bv = 0.f;
    int bi = INT_MAX;
    for (int e = threadIdx.x; e < V; e += NT) {
        float x = __ldg(c.g + e);
        int s = (e + sh) >> 2, q = (e + sh) & 3;
        if (pen && ((c.bits[s >> 3] >> ((s & 7) * 4 + q)) & 1u)) x = penalize(x, penalty);
        float l = scale ? __fmul_rn(x, inv_temp) : x;
        if (l == l) argmax_combine(bv, bi, l, e);
    }
    block_argmax(bv, bi, c.red);
    float l0 = __ldg(c.g);
    {
        int s = sh >> 2, q = sh & 3;
        if (pen && ((c.bits[s >> 3] >> ((s & 7) * 4 + q)) & 1u)) l0 = penalize(l0, penalty);
    }
    l0 = scale ? __fmul_rn(l0, inv_temp) : l0;
    if (l0 != l0 || bi == INT_MAX) return 0;
    return bi;
}

__device__ void write_result(Ctx &c, int id, float p, int path, int n_cand, int n_final,
                             int consumed) {
    if (threadIdx.x == 0) {
        c.P.out_id[c.rowid] = id;
        if (c.P.out_prob) c.P.out_prob[c.rowid] = p;
        if (c.P.stats) {
            bm_row_stats_t st;
            st.path = path; st.n_cand = n_cand; st.n_final = n_final; st.consumed = consumed;
            c.P.stats[c.rowid] = st;
        }
    }
}

// ---------------------------------------------------------------- top_k --
__device__ void topk_path(Ctx &c) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Vars *v = c.v;
    const int sh = v->sh, nslots = v->nslots, V = c.P.V, k = v->k;
    const float mx = v->mx, thr = v->thr, inv_temp = v->inv_temp;
    const bool scale = (inv_temp != 1.0f);
    const float4 *r4 = reinterpret_cast<const float4 *>(c.row);
    uint32_t *kh = reinterpret_cast<uint32_t *>(c.scr);                       // 8 x 128
    unsigned long long *kc = reinterpret_cast<unsigned long long *>(c.scr + 4096);  // KCAP
    const float bscale = __fdiv_rn(127.0f, 20.0f);  // src/model.c:184

    for (int i = threadIdx.x; i < 8 * HB; i += NT) kh[i] = 0;
    if (threadIdx.x == 0) v->kcnt = 0;
    __syncthreads();
    // histogram of (max - l) over l >= thr (src/model.c:185-195); the last
    // bucket never decides the cut, so it is not counted
    uint32_t *myh = kh + (warp & 7) * HB;
    for (int s = threadIdx.x; s < nslots; s += NT) {
        float4 x = r4[s];
        float t[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int e = 4 * s + q - sh;
            if (e < 0 || e >= V) continue;
            float l = scale ? __fmul_rn(t[q], inv_temp) : t[q];
            if (l >= thr) {
                int b = x86_cvtt(__fmul_rn(__fsub_rn(mx, l), bscale));
                b = min(max(b, 0), HB - 1);
                if (b < HB - 1) atomicAdd(&myh[b], 1u);
            }
        }
    }
    __syncthreads();
    // cut bucket: first bucket whose running count reaches k (src/model.c:199-207)
    if (warp == 0) {
        uint32_t cq[4];
        uint32_t ls = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t s = 0;
            for (int cp = 0; cp < 8; ++cp) s += kh[cp * HB + 4 * lane + q];
            cq[q] = s;
            ls += s;
        }
        uint32_t inc = warp_iscan(ls, lane);
        uint32_t run = inc - ls;
        int hit = INT_MAX;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            run += cq[q];
            if (hit == INT_MAX && run >= (uint32_t)k) hit = 4 * lane + q;
        }
        hit = warp_imin(hit);
        if (lane == 0) v->kcut = (hit == INT_MAX) ? HB - 1 : hit;
    }
    __syncthreads();
    const int cut = v->kcut;
    const float bthr = __fsub_rn(mx, __fdiv_rn((float)(cut + 1), bscale));  // src/model.c:210-211
    const float ethr = bthr > thr ? bthr : thr;                          // src/model.c:213-214
    // extraction (src/model.c:217-224), unordered here, ordered by id below
    for (int base = warp * 32; base < nslots; base += NT) {
        int s = base + lane;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s < nslots) x = r4[s];
        float t[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int e = 4 * s + q - sh;
            bool ok = false;
            float l = 0.f;
            if (s < nslots && e >= 0 && e < V) {
                l = scale ? __fmul_rn(t[q], inv_temp) : t[q];
                ok = (l >= ethr);
            }
            unsigned m = __ballot_sync(FULL, ok);
            if (m) {
                int leader = __ffs(m) - 1, bpos = 0;
                if (lane == leader) bpos = atomicAdd(&v->kcnt, __popc(m));
                bpos = __shfl_sync(FULL, bpos, leader);
                if (ok) {
                    int pos = bpos + __popc(m & ((1u << lane) - 1));
                    if (pos < KCAP)
                        kc[pos] = ((unsigned long long)(unsigned)e << 32) | __float_as_uint(l);
                }
            }
        }
    }
    __syncthreads();
    const int n = v->kcnt;
    if (n == 0) {  // argmax guard (src/model.c:227-237)
        int id = guard_argmax(c);
        write_result(c, id, 1.0f, 2, 0, 0, 0);
        return;
    }
    float *hv = reinterpret_cast<float *>(c.scr);            // 256 (reuses histogram)
    int *hi = reinterpret_cast<int *>(c.scr + 1024);         // 256
    float *pv = reinterpret_cast<float *>(c.scr + 2048);     // 256: probabilities
    int *rk = reinterpret_cast<int *>(c.scr + 3072);         // 256: ranks
    int ns;  // survivors
    if (n <= KCAP) {
        block_sort_u64(kc, n, KCAP);  // by id (ids are unique)
        if (warp == 0) {
            int first = min(n, k);
            for (int q = lane; q < first; q += 32) {
                hv[q] = __uint_as_float((unsigned)(kc[q] & 0xffffffffu));
                hi[q] = (int)(kc[q] >> 32);
            }
            __syncwarp();
            if (n > k) {  // heap top-k (src/model.c:240-254)
                warp_heapify(hv, hi, k, lane);
                for (int base = k; base < n; base += 32) {
                    int j = base + lane;
                    float val = 0.f;
                    int id = 0;
                    if (j < n) { val = __uint_as_float((unsigned)(kc[j] & 0xffffffffu)); id = (int)(kc[j] >> 32); }
                    float root = hv[0];
                    unsigned mr = __ballot_sync(FULL, j < n && val > root);
                    while (mr) {
                        int src = __ffs(mr) - 1;
                        float vb = __shfl_sync(FULL, val, src);
                        int ib = __shfl_sync(FULL, id, src);
                        if (lane == 0 && vb > hv[0]) { hv[0] = vb; hi[0] = ib; heap_down(hv, hi, k, 0); }
                        __syncwarp();
                        mr &= mr - 1;
                    }
                }
            }
        }
    } else {
        // more candidates than the list holds: stream them in id order
        // straight from the row buffer through the same heap rules
        if (warp == 0) {
            int filled = 0;
            for (int base = 0; base < V; base += 32) {
                const int e = base + lane;
                float l = 0.f;
                bool ok = false;
                if (e < V) {
                    const float x = c.row[e + sh];
                    l = scale ? __fmul_rn(x, inv_temp) : x;
                    ok = (l >= ethr);
                }
                const unsigned mk = __ballot_sync(FULL, ok);
                bool rest = ok;
                if (filled < k) {
                    const int rank = __popc(mk & ((1u << lane) - 1));
                    const int take = min(__popc(mk), k - filled);
                    if (ok && rank < take) { hv[filled + rank] = l; hi[filled + rank] = e; }
                    rest = ok && rank >= take;
                    filled += take;
                    __syncwarp();
                    if (filled < k) continue;
                    if (take > 0) warp_heapify(hv, hi, k, lane);
                }
                const float root = hv[0];
                unsigned mr = __ballot_sync(FULL, rest && l > root);
                while (mr) {
                    const int src = __ffs(mr) - 1;
                    const float vb = __shfl_sync(FULL, l, src);
                    const int ib = __shfl_sync(FULL, e, src);
                    if (lane == 0 && vb > hv[0]) { hv[0] = vb; hi[0] = ib; heap_down(hv, hi, k, 0); }
                    __syncwarp();
                    mr &= mr - 1;
                }
            }
        }
    }
    ns = min(n, k);
    __syncthreads();
    // survivor softmax (src/model.c:257-269), warp 0, <= 8 per lane in order
    if (warp == 0) {
        float val[8];
        float lm = -1e30f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            int j = lane * 8 + q;
            val[q] = (j < ns) ? hv[j] : -1e30f;
            if (j < ns) lm = fmaxf(lm, val[q]);
        }
        lm = warp_max(lm);
        float ev[8];
        double s = 0.0;
        float emin = __int_as_float(0x7f800000);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            int j = lane * 8 + q;
            ev[q] = (j < ns) ? expf(__fsub_rn(val[q], lm)) : 0.0f;
            s += (double)ev[q];
            if (j < ns && ev[q] > 0.0f) emin = fminf(emin, ev[q]);
        }
        emin = warp_min(emin);
        double S = warp_sum(s);
        // the tree sum equals the reference's sequential one when every term
        // is a multiple of ulp(emin) and the sum stays below 2^53 of those
        if (!(emin >= 0x1p-22f) && S == S) {
            double q0 = 0.0;
            for (int j = 0; j < ns; ++j) q0 += (double)__shfl_sync(FULL, ev[j & 7], j >> 3);
            S = q0;
        }
        float inv = __fdiv_rn(1.0f, __double2float_rn(S));
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            int j = lane * 8 + q;
            if (j < ns) pv[j] = __fmul_rn(ev[q], inv);
        }
        if (lane == 0) v->S = S;
    }
    __syncthreads();
    const double S = v->S;
    const float top_p = v->top_p;
    if (S != S) {  // NaN mass: every comparison fails, the walk returns the last
        write_result(c, hi[ns - 1], pv[ns - 1], 3, n, ns, 1);
        return;
    }
    // stable descending sort when top_p < 1 (src/model.c:275-276)
    unsigned long long *srt = kc;  // reuse
    if (top_p < 1.0f) {
        for (int j = threadIdx.x; j < ns; j += NT) rk[j] = 0;
        __syncthreads();
        int G = NT / ns;  // >= 4
        if (threadIdx.x < G * ns) {
            int j = threadIdx.x % ns, g = threadIdx.x / ns;
            int per = (ns + G - 1) / G;
            int a = g * per, b = min(ns, a + per);
            float pj = pv[j];
            int r = 0;
            for (int i = a; i < b; ++i) {
                float pi = pv[i];
                r += (pi > pj) || (pi == pj && i < j);
            }
            if (r) atomicAdd(&rk[j], r);
        }
        __syncthreads();
        for (int j = threadIdx.x; j < ns; j += NT)
            srt[rk[j]] = ((unsigned long long)(unsigned)hi[j] << 32) | __float_as_uint(pv[j]);
    } else {
        for (int j = threadIdx.x; j < ns; j += NT)
            srt[j] = ((unsigned long long)(unsigned)hi[j] << 32) | __float_as_uint(pv[j]);
    }
    __syncthreads();
    // filter_and_sample(probs, ns, 0, top_p, 0) (src/model.c:72-118), warp 0
    if (warp == 0) {
        const int per = (ns + 31) / 32;
        const int b = lane * per, e = min(ns, b + per);
        float pmin = __int_as_float(0x7f800000);
        double ls = 0.0;
        for (int j = b; j < e; ++j) {
            float p = __uint_as_float((unsigned)(srt[j] & 0xffffffffu));
            ls += (double)p;
            if (p > 0.0f) pmin = fminf(pmin, p);
        }
        pmin = warp_min(pmin);
        double inc = warp_iscan(ls, lane);
        double pre = inc - ls;
        bool exact = (pmin >= 0x1p-29f);
        // nucleus cut: first j with cs_j >= top_p
        int nf = ns;
        double cs_cut = __shfl_sync(FULL, inc, 31);
        if (top_p < 1.0f) {
            int hit = INT_MAX;
            double hcs = 0.0;
            if (exact) {
                double cs = pre;
                for (int j = b; j < e; ++j) {
                    cs += (double)__uint_as_float((unsigned)(srt[j] & 0xffffffffu));
                    if (cs >= (double)top_p) { hit = j; hcs = cs; break; }
                }
                int best = warp_imin(hit);
                if (best != INT_MAX) {
                    hcs = __shfl_sync(FULL, hcs, best / per);
                    nf = best + 1;
                    cs_cut = hcs;
                }
            } else {
                double cs = 0.0;
                for (int j = 0; j < ns; ++j) {
                    cs += (double)__uint_as_float((unsigned)(srt[j] & 0xffffffffu));
                    if (cs >= (double)top_p) { nf = j + 1; break; }
                }
                cs_cut = cs;
            }
        }
        // renormalise and draw: r = u * (float)new_sum, first j with r < cdf_j
        const double new_sum = cs_cut;
        const float r = __fmul_rn(v->u, __double2float_rn(new_sum));
        int pos = nf - 1;
        if (exact) {
            int hit = INT_MAX;
            double cs = pre;
            for (int j = b; j < min(e, nf); ++j) {
                cs += (double)__uint_as_float((unsigned)(srt[j] & 0xffffffffu));
                if ((double)r < cs) { hit = j; break; }
            }
            int best = warp_imin(hit);
            if (best != INT_MAX) pos = best;
        } else {
            double cs = 0.0;
            for (int j = 0; j < nf; ++j) {
                cs += (double)__uint_as_float((unsigned)(srt[j] & 0xffffffffu));
                if ((double)r < cs) { pos = j; break; }
            }
        }
        if (lane == 0) {
            unsigned long long kk = srt[pos];
            v->res_id = (int)(kk >> 32);
            v->res_p = __uint_as_float((unsigned)(kk & 0xffffffffu));
            v->n_final = nf;
        }
    }
    __syncthreads();
    write_result(c, v->res_id, v->res_p, 3, n, v->n_final, 1);
}

// ------------------------------------------------------ full vocabulary --
__device__ void full_path(Ctx &c) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Vars *v = c.v;
    const int sh = v->sh, nslots = v->nslots, V = c.P.V;
    const float mx = v->mx, thr = v->thr, inv_temp = v->inv_temp;
    const bool scale = (inv_temp != 1.0f);
    float4 *r4 = reinterpret_cast<float4 *>(c.row);
    uint32_t *hcnt = reinterpret_cast<uint32_t *>(c.scr);

    for (int i = threadIdx.x; i < NB; i += NT) hcnt[i] = 0;
    // bucket geometry over d = max - l
    float dmax = __fsub_rn(mx, v->xmin);
    if (v->min_p > 0.0f) dmax = fminf(dmax, __fsub_rn(mx, thr));
    dmax = fminf(dmax, DCAP);
    if (!(dmax > 1e-30f)) dmax = 1.0f;
    const float inv_w = __fdiv_rn((float)NB - 1.5f, dmax);
    const float w = __fdiv_rn(1.0f, inv_w);
    __syncthreads();
    // exp pass (src/model.c:306-310): e = expf(l - max) for l >= thr, stored in
    // place; non-candidates -1.  fp64 sum in groups of four.
    double S = 0.0;
    int ncand = 0, last = -1;
    for (int s = threadIdx.x; s < nslots; s += NT) {
        float4 x = r4[s];
        float t[4] = {x.x, x.y, x.z, x.w};
        float ev[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int e = 4 * s + q - sh;
            float l = scale ? __fmul_rn(t[q], inv_temp) : t[q];
            bool cand = (e >= 0 && e < V) && (l >= thr);
            ev[q] = -1.0f;
            if (cand) {
                ev[q] = expf(__fsub_rn(l, mx));
                ++ncand;
                last = e;
                float d = fminf(__fsub_rn(mx, l), dmax);
                int key = __float_as_int(__fmaf_rn(d, inv_w, MAGIC)) - __float_as_int(MAGIC);
                key = min(max(key, 0), NB - 1);
                atomicAdd(&hcnt[key], 1u);
            }
        }
        float g0 = __fadd_rn(fmaxf(ev[0], 0.f), fmaxf(ev[1], 0.f));
        float g1 = __fadd_rn(fmaxf(ev[2], 0.f), fmaxf(ev[3], 0.f));
        // NaN e (inf logits) must poison the sum like the reference's
        if (ev[0] != ev[0] || ev[1] != ev[1] || ev[2] != ev[2] || ev[3] != ev[3])
            S += (double)__int_as_float(0x7fc00000);
        else
            S += (double)__fadd_rn(g0, g1);
        r4[s] = make_float4(ev[0], ev[1], ev[2], ev[3]);
    }
    S = block_sum_d(S, c.red);
    ncand = block_sum_i(ncand, c.red);
    last = block_max_i(last, c.red);
    const float top_p = v->top_p;
    const int top_k = v->top_k;
    const bool lazy = (top_p >= 1.0f) && (top_k <= 0 || top_k >= ncand);
    if (ncand == 0) {  // argmax guard (src/model.c:296-303)
        int id = guard_argmax(c);
        write_result(c, id, 1.0f, 4, 0, 0, 0);
        return;
    }
    if (S != S) {  // NaN mass: the walk falls through to the last candidate
        write_result(c, last, __int_as_float(0x7fc00000), lazy ? 5 : 7, ncand, ncand, 1);
        return;
    }
    const float inv_sum = __fdiv_rn(1.0f, __double2float_rn(S));  // src/model.c:311
    if (threadIdx.x == 0) {
        v->inv_sum = inv_sum;
        v->n_cand = ncand;
        v->w = w;
        v->inv_w = inv_w;
        v->last_cand = last;
    }
    __syncthreads();

    if (lazy) {
        // CDF walk in id order (src/model.c:319-320): contiguous segments
        const int Q = (nslots + NT - 1) / NT;
        const int s0 = threadIdx.x * Q, s1 = min(nslots, s0 + Q);
        double seg = 0.0;
        for (int s = s0; s < s1; ++s) {
            float4 x = r4[s];
            float ev[4] = {x.x, x.y, x.z, x.w};
            float g = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q)
                g = __fadd_rn(g, ev[q] >= 0.f ? __fmul_rn(ev[q], inv_sum) : 0.f);
            seg += (double)g;
        }
        double total;
        double pre = block_xscan_d(seg, total, c.red);
        const float r = __fmul_rn(v->u, __double2float_rn(total));
        int cand_t = ((double)r < pre + seg && seg > 0.0) ? (int)threadIdx.x : INT_MAX;
        int owner = block_min_i(cand_t, c.red);
        if (threadIdx.x == 0) { v->res_id = -1; v->res_p = 0.f; }
        __syncthreads();
        if ((int)threadIdx.x == owner) {
            // rescan from this segment on (a rounding difference at the
            // segment start can push the crossing one segment further)
            double cdf = pre;
            int id = -1;
            float pp = 0.f;
            for (int s = s0; s < nslots && id < 0; ++s) {
                float4 x = r4[s];
                float ev[4] = {x.x, x.y, x.z, x.w};
                for (int q = 0; q < 4; ++q) {
                    if (ev[q] >= 0.f) {
                        float p = __fmul_rn(ev[q], inv_sum);
                        cdf += (double)p;
                        if ((double)r < cdf) { id = 4 * s + q - sh; pp = p; break; }
                    }
                }
            }
            if (id >= 0) { v->res_id = id; v->res_p = pp; }
        }
        __syncthreads();
        int id = v->res_id;
        float pp = v->res_p;
        if (id < 0) {
            // r at or beyond the last cdf: the reference returns the last
            // candidate (src/model.c:117)
            id = last;
            pp = __fmul_rn(c.row[last + sh], inv_sum);
        }
        write_result(c, id, pp, 5, ncand, ncand, 1);
        return;
    }

    // sorted order: nucleus cut, optional top_k truncation, draw
    int n = ncand;
    double new_sum = 0.0;
    Sel tail;  // the element at position n-1
    tail.found = 0;
    bool partial = false;
    if (top_p < 1.0f) {
        Sel cut = select_canon(c, 0, (double)top_p, 0);
        if (cut.found) {
            n = cut.pos + 1;
            new_sum = cut.cs;
            tail = cut;
            partial = (ncand > 256) && (cut.pos < 256);  // src/model.c:327-356
        } else {
            new_sum = cut.cs;  // whole candidate mass
            tail = cut;
        }
    }
    if (top_k > 0 && top_k < n) {  // src/model.c:102-103
        Sel tk = select_canon(c, 2, 0.0, top_k - 1);
        n = top_k;
        new_sum = tk.cs;
        tail = tk;
    }
    const float r = __fmul_rn(v->u, __double2float_rn(new_sum));
    Sel d = select_canon(c, 1, (double)r, 0);
    int id;
    float pp;
    if (d.found && d.pos < n) { id = d.id; pp = d.p; }
    else { id = tail.id; pp = tail.p; d.tie = tail.tie; }
    if (partial && d.tie) {
        // the reference's heap layout decides the order among equal
        // probabilities: replay it exactly
        unsigned long long *hk = reinterpret_cast<unsigned long long *>(c.scr + NB * 4);
        float *hv = reinterpret_cast<float *>(c.scr + NB * 4 + WCAP * 8);
        int *hix = reinterpret_cast<int *>(c.scr + NB * 4 + WCAP * 8 + 256 * 4);
        replay_top256(c, hk, hv, hix);
        if (warp == 0) {
            // walk the replayed order with the same cut and draw
            double cs = 0.0;
            int pos = n - 1;
            if (lane == 0) {
                for (int j = 0; j < n; ++j) {
                    cs += (double)key_p(hk[j]);
                    if ((double)r < cs) { pos = j; break; }
                }
                int hp = key_id(hk[pos]);
                v->res_id = hix[hp];
                v->res_p = hv[hp];
            }
        }
        __syncthreads();
        id = v->res_id;
        pp = v->res_p;
    }
    write_result(c, id, pp, partial ? 6 : 7, ncand, n, 1);
}

__global__ void __launch_bounds__(NT, 1) sample_kernel(const Params P) {
    extern __shared__ __align__(128) unsigned char smem[];
    Ctx c;
    c.P = P;
    c.L = layout(P.V);
    c.mbar = reinterpret_cast<uint64_t *>(smem + c.L.mbar);
    c.red.d = reinterpret_cast<double *>(smem + c.L.red);
    c.red.i = reinterpret_cast<int *>(smem + c.L.red + NW * 8);
    c.red.f = reinterpret_cast<float *>(smem + c.L.red + NW * 12);
    c.v = reinterpret_cast<Vars *>(smem + c.L.vars);
    c.bits = reinterpret_cast<uint32_t *>(smem + c.L.bits);
    c.scr = smem + c.L.scr;
    c.row = reinterpret_cast<float *>(smem + c.L.row);
    Vars *v = c.v;
    const int V = P.V;
    const int tid = threadIdx.x;

    if (tid == 0) {
        for (int i = 0; i < NCHUNK; ++i) mbar_init(&c.mbar[i], 1);
        fence_mbar_init();
        v->fail = 0;
    }
    __syncthreads();

    uint32_t it = 0;
    for (int row = blockIdx.x; row < P.B; row += gridDim.x, ++it) {
        c.rowid = row;
        c.parity = it & 1u;
        c.g = P.logits + (int64_t)row * P.ld;
        // geometry of this row inside 16-byte slots
        const int sh = (int)(((uintptr_t)c.g & 15u) >> 2);
        const int nslots = (V + sh + 3) >> 2;
        int i0 = sh ? 4 - sh : 0;
        if (i0 > V) i0 = V;
        int n4 = ((V - i0) >> 2) << 2;
        if (n4 < 4 * NCHUNK * 4) n4 = 0;  // tiny rows: plain loads only
        const int s_int0 = (i0 + sh) >> 2, s_int1 = s_int0 + (n4 >> 2);
        if (tid == 0) {
            // issue this row's bulk copies (the buffer is free: previous row
            // finished with a barrier and an async-proxy fence)
            const int nint = s_int1 - s_int0;
            for (int ch = 0; ch < NCHUNK; ++ch) {
                int a = (ch * nint) / NCHUNK, b = ((ch + 1) * nint) / NCHUNK;
                uint32_t bytes = (uint32_t)(b - a) * 16u;
                mbar_expect_tx(&c.mbar[ch], bytes);
                if (bytes)
                    bulk_load(c.row + 4 * (s_int0 + a), c.g + i0 + 4 * a, bytes, &c.mbar[ch]);
            }
            // and warm L2 with the next row this CTA will take
            const int nrow = row + gridDim.x;
            if (nrow < P.B) {
                const float *ng = P.logits + (int64_t)nrow * P.ld;
                int nsh = (int)(((uintptr_t)ng & 15u) >> 2);
                int ni0 = nsh ? 4 - nsh : 0;
                if (ni0 < V) {
                    int nn4 = ((V - ni0) >> 2) << 2;
                    if (nn4 >= 16) prefetch_l2(ng + ni0, (uint32_t)nn4 * 4u);
                }
            }
            // knobs of this row
            const bm_knobs_t kn = P.knobs[(int64_t)row * P.knob_stride];
            v->temp = kn.temp;
            v->penalty = kn.penalty;
            v->min_p = kn.min_p;
            v->top_p = kn.top_p;
            v->top_k = kn.top_k;
            v->inv_temp = kn.inv_temp;
            v->log_min_p = kn.log_min_p;
            v->u = P.uniform ? P.uniform[row] : 0.0f;
            v->greedy = (kn.temp < 0.05f);  // src/model.c:144
            v->sh = sh;
            v->nslots = nslots;
            v->s_int0 = s_int0;
            v->s_int1 = s_int1;
            int h0 = 0, h1 = 0;
            if (P.hist && P.hist_off) { h0 = (int)P.hist_off[row]; h1 = (int)P.hist_off[row + 1]; }
            v->pen = (h1 > h0) && (kn.penalty > 0.0f) && (kn.penalty != 1.0f);
            v->kcut = h0;
            v->kcnt = h1;
        }
        __syncthreads();
        // penalty bitset over this row's distinct, in-range, unprotected ids
        if (v->pen) {
            const int h0 = v->kcut, h1 = v->kcnt;
            for (int i = tid; i < c.L.nbw; i += NT) c.bits[i] = 0u;
            __syncthreads();
            for (int i = h0 + tid; i < h1; i += NT) {
                int id = P.hist[i];
                if (id >= 0 && id < V && !protected_id(id)) {
                    int b = id + sh;
                    atomicOr(&c.bits[b >> 5], 1u << (b & 31));
                }
            }
            __syncthreads();
        }
        const bool greedy = v->greedy != 0;
        float mx, xmin, gv;
        int gi;
        load_pass(c, greedy, mx, xmin, gv, gi);
        if (__syncthreads_or(v->fail)) {
            // a bounded wait expired: wait (bounded) for this row's copies,
            // then stop; the host sees the error flag
            if (tid == 0)
                for (int ch = 0; ch < NCHUNK; ++ch) (void)mbar_wait(&c.mbar[ch], c.parity);
            __syncthreads();
            return;
        }
        if (greedy) {
            block_argmax(gv, gi, c.red);
            write_result(c, gi == INT_MAX ? 0 : gi, 1.0f, 1, 0, 0, 0);
        } else {
            block_maxmin_f(mx, xmin, c.red);
            if (tid == 0) {
                v->mx = mx;
                v->xmin = xmin;
                // src/model.c:169-173 (logf from the host)
                float thr = -1e30f;
                if (v->min_p >= 1.0f) thr = mx;
                else if (v->min_p > 0.0f) thr = __fadd_rn(mx, v->log_min_p);
                v->thr = thr;
                v->k = (v->top_k > 0 && v->top_k <= 256) ? v->top_k : 0;  // src/model.c:175
            }
            __syncthreads();
            if (v->k > 0) topk_path(c);
            else full_path(c);
        }
        fence_proxy_async();
        __syncthreads();
    }
}

}  // namespace

size_t smem_bytes(int V) { return layout(V).total; }

int max_vocab(size_t limit) {
    int lo = 1, hi = 1 << 20;
    if (smem_bytes(1) > limit) return 0;
    while (lo < hi) {
        int mid = lo + (hi - lo + 1) / 2;
        if (smem_bytes(mid) <= limit) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

cudaError_t prepare(int V) {
    return cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem_bytes(V));
}

cudaError_t launch(const Params &p, int grid, cudaStream_t s) {
    sample_kernel<<<grid, NT, smem_bytes(p.V), s>>>(p);
    return cudaGetLastError();
}

}  // namespace bmk
