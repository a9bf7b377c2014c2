// Decode-step token sampler for sm_100a: one persistent CTA per SM, one logits
// row at a time resident in shared memory.
//
// Per row (reference: jserv/bitmamba.c src/model.c:1268-1307, 37-361):
//   load      bulk async copy of the row's 16-byte-aligned interior into shared
//             memory in NCHUNK pieces (one mbarrier each; the copy for the
//             next row is issued as soon as this row's buffer is free, and the
//             row after that is prefetched into L2), ragged head/tail by plain
//             loads with NaN in the junk lanes so every later pass runs over
//             whole 16-byte slots.  The repetition penalty is applied in
//             place once the row has landed, once per distinct history id (a
//             bitset; src/model.c:1277-1304); the pass then reduces max / min
//             of the scaled logits
//             (src/model.c:156-163) or the greedy argmax (src/model.c:144-154).
//   top_k     1 <= top_k <= 256: with a real min_p threshold the candidates
//             are listed first (threads whose own maximum lies below it skip
//             their slots); up to 64 in value order finish on one warp: a
//             bitonic sort of the occupied part of the list, the reference's
//             128-bucket cut and extraction (src/model.c:181-224) as prefixes
//             of it, survivor softmax, nucleus cut and draw.  Otherwise the
//             128-bucket histogram cut, exact emulation of the reference's
//             min-heap (the heap layout decides the CDF walk order), survivor
//             softmax, stable descending sort, nucleus cut and draw.
//   full      other top_k: rows with a real min_p threshold and at most 64
//             candidates take the same one-warp end without the cut.  Else a
//             bucket-mass histogram over d = max - l (one shared atomic per
//             candidate adds its fixed-point e-mass), then either the id-order
//             walk (src/model.c:319-320) or, for the sorted order, windows of
//             buckets around the nucleus cut, the top_k position and the
//             draw: a membership pass flags the window elements, a gather
//             lists them with exact probabilities, and order statistics over
//             the list in (probability desc, id asc) order -- the order the
//             reference's stable sort produces -- resolve every target
//             block-parallel.  Rows where the reference's top-256 heap path
//             applies and ties make its layout visible are replayed exactly
//             (src/model.c:327-356); a target that falls outside its window
//             takes exact passes over global memory.
//   schedule  the first gridDim.x rows go one per CTA; at each release a CTA
//             claims the row after the one whose copy it issues there (atomic
//             counter, rewound by the last CTA to finish), so rows of unequal
//             cost keep every SM busy to the end of the launch.
//
// Arithmetic that decides ids uses the reference's fp32 operations (no
// contraction: explicit __fmul_rn/__fadd_rn/__fdiv_rn; the library is built
// with --fmad=false), sums in fp64.
#include "bm_kernel.cuh"

#include <cfloat>
#include <climits>

namespace bmk {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr unsigned long long WAIT_NS = 2000000000ull;  // bounded waits: 2 s
constexpr float DCAP = 40.0f;                          // bucket range cap
constexpr float MAGIC = 12582912.0f;                   // 1.5 * 2^23
constexpr int MAGIC_I = 0x4B400000;                    // bits of MAGIC
constexpr int LISTCAP = 2048;                          // window list cap (entries)
constexpr int MASKW = 4;                               // top_k path: mask words per thread
constexpr int KREG = 2;                                // top_k path: slots per thread
constexpr int KOVF = KCAP - KREG * NT;                 // top_k path: overflow entries
constexpr int BPT = NB / NT;                            // estimate buckets per thread
constexpr int SLOW_CAP = 256;                          // rare-path list cap
constexpr int SLOW_OFF = LISTCAP * 8 + 2048;           // rare-path scratch offset
constexpr float PINF = __builtin_huge_valf();
// Junk lanes of the ragged head / tail slots hold NaN (never a candidate,
// whatever the temperature).  The branch-free CLEAN passes need a finite
// value instead: JUNK, rewritten into those lanes for CLEAN rows, whose
// temperature-scaled value (1e-6 <= 1/temp <= 20) lies below every min_p
// threshold (>= -1e30 - 104) while max - value stays finite, so its exp is 0
// and its bucket key lies beyond the last bucket.
constexpr float JUNK = -1e37f;
constexpr size_t RED_BYTES = 2048;

// GPT-2 ids the reference never penalises (src/bitmamba.h:21-24).
__device__ __forceinline__ bool protected_id(int id) {
    return id == 50256 || id == 198 || id == 628 || id == 13;
}

struct __align__(16) Vars {
    double S, cs, aux0, aux1;
    int64_t nh[2];    // the next row's history offsets, knobs and uniform,
    bm_knobs_t nk;    // copied in asynchronously at the release
    float nu;
    int nclaim;       // the row claimed to follow the next one
    double mc, ec, mk, ek, md;
    double adj[3];    // per target: mass of the band elements above its buckets
    double lbm[3];    // per target: mass of the listed elements in front of its range
    const bm_knobs_t *p_knobs;  // launch parameters the row release prefetches from
    const float *p_uniform;
    const int64_t *p_hist_off;
    int64_t p_knob_stride;
    float mx, thr, xmin, inv_temp;
    float temp, penalty, min_p, top_p;
    float log_min_p, u, inv_sum, res_p;
    int top_k, greedy, pen, k;
    int sh, nslots, s_int0, s_int1;
    int h0, h1, released, fail;
    int fail2;      // the exact select of this row did not converge
    int fb;         // summary rows: the lists cannot decide the row (full path)
    float sumvk;    // summary rows: the largest value a tile's list may omit
    int kcut, kcnt, n_cand, own;
    int clean, ln0, ln2, ln3;
    int sel_found, sel_j, res_id, n_final;
    int wt;         // the one-warp top_k tail decided the row
    int bc, bk, bd0, bc_hi, bd_hi, next_row, lastb;
    int amax;       // index of the maximum (lowest among equal maxima)
    uint32_t h0b;   // fixed-point mass sum of bucket 0
    int frk[3];   // per target: rank of its range's first listed element
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
    o += RED_BYTES;
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
// 4-byte asynchronous global -> shared copy (the ragged row edges)
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2_line(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
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
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// three-input max / min (sm_100): NaN inputs are ignored like fmaxf / fminf
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
    float r;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
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
// exp(x) for x <= 0 as 2^y * 2^c with y = fl(x*L1) and c the exact residual
// of x*L1 plus x*L2 (L1 + L2 = log2 e); 2^c = 1 + c ln2 to fp32 accuracy
// since |c| < 2^-16.  Error: that of ex2.approx plus one rounding.
__device__ __forceinline__ float2 exp_pair(float2 x) {
    const float2 L1 = make_float2(1.4426950216293335f, 1.4426950216293335f);
    const float2 L2 = make_float2(1.925963033500011e-08f, 1.925963033500011e-08f);
    const float2 LN2 = make_float2(0.6931471824645996f, 0.6931471824645996f);
    const float2 y = __fmul2_rn(x, L1);
    float2 c = __ffma2_rn(x, L1, make_float2(-y.x, -y.y));
    c = __ffma2_rn(x, L2, c);
    const float2 e = make_float2(ex2_approx(y.x), ex2_approx(y.y));
    const float2 t = __fmul2_rn(e, c);
    return __ffma2_rn(t, LN2, e);
}
__device__ __forceinline__ float exp_one(float x) { return exp_pair(make_float2(x, x)).x; }
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
template <class T>
__device__ __forceinline__ T warp_iscan(T v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T n = __shfl_up_sync(FULL, v, o);
        if (lane >= o) v += n;
    }
    return v;
}
// (value, index): larger value, then smaller index; idx INT_MAX = none.
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

// Block reductions over NT threads; every thread gets the result.  The red
// area holds 2*NW doubles, 4*NW ints and 2*NW floats side by side.
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
    double t = warp_sum(lane < NW ? r.d[lane] : 0.0);
    __syncthreads();
    return t;
}
__device__ __forceinline__ int block_sum_i(int v, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) r.i[warp] = v;
    __syncthreads();
    int t = warp_sum(lane < NW ? r.i[lane] : 0);
    __syncthreads();
    return t;
}
__device__ __forceinline__ int block_max_i(int v, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_imax(v);
    if (lane == 0) r.i[warp] = v;
    __syncthreads();
    int t = warp_imax(lane < NW ? r.i[lane] : INT_MIN);
    __syncthreads();
    return t;
}
__device__ __forceinline__ int block_min_i(int v, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_imin(v);
    if (lane == 0) r.i[warp] = v;
    __syncthreads();
    int t = warp_imin(lane < NW ? r.i[lane] : INT_MAX);
    __syncthreads();
    return t;
}
__device__ __forceinline__ void block_maxmin_f(float &mx, float &mn, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    mx = warp_max(mx);
    mn = warp_min(mn);
    if (lane == 0) { r.f[warp] = mx; r.f[NW + warp] = mn; }
    __syncthreads();
    mx = warp_max(lane < NW ? r.f[lane] : -PINF);
    mn = warp_min(lane < NW ? r.f[NW + lane] : PINF);
    __syncthreads();
}
// max, min and sum at once (the sum carries the non-finite check)
__device__ __forceinline__ void block_maxmin_chk(float &mx, float &mn, float &ck, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    mx = warp_max(mx);
    mn = warp_min(mn);
    ck = warp_sum(ck);
    if (lane == 0) { r.f[warp] = mx; r.f[NW + warp] = mn; r.f[2 * NW + warp] = ck; }
    __syncthreads();
    mx = warp_max(lane < NW ? r.f[lane] : -PINF);
    mn = warp_min(lane < NW ? r.f[NW + lane] : PINF);
    ck = warp_sum(lane < NW ? r.f[2 * NW + lane] : 0.0f);
    __syncthreads();
}
__device__ __forceinline__ void block_argmax(float &v, int &i, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    warp_argmax(v, i);
    if (lane == 0) { r.f[warp] = v; r.i[warp] = i; }
    __syncthreads();
    v = lane < NW ? r.f[lane] : 0.f;
    i = lane < NW ? r.i[lane] : INT_MAX;
    warp_argmax(v, i);
    __syncthreads();
}
// several sums at once: doubles a, b and ints c, d
__device__ __forceinline__ void block_sum4(double &a, double &b, int &c, int &d, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    a = warp_sum(a);
    b = warp_sum(b);
    c = warp_sum(c);
    d = warp_sum(d);
    if (lane == 0) {
        r.d[warp] = a;
        r.d[NW + warp] = b;
        r.i[2 * NW + warp] = c;
        r.i[3 * NW + warp] = d;
    }
    __syncthreads();
    a = warp_sum(lane < NW ? r.d[lane] : 0.0);
    b = warp_sum(lane < NW ? r.d[NW + lane] : 0.0);
    c = warp_sum(lane < NW ? r.i[2 * NW + lane] : 0);
    d = warp_sum(lane < NW ? r.i[3 * NW + lane] : 0);
    __syncthreads();
}
// exclusive block scans; return the exclusive prefix, set the total
__device__ __forceinline__ double block_xscan_d(double v, double &total, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double inc = warp_iscan(v, lane);
    if (lane == 31) r.d[warp] = inc;
    __syncthreads();
    double w = lane < NW ? r.d[lane] : 0.0;
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
    int w = lane < NW ? r.i[lane] : 0;
    int winc = warp_iscan(w, lane);
    int woff = __shfl_sync(FULL, winc - w, warp);
    total = __shfl_sync(FULL, winc, 31);
    __syncthreads();
    return woff + inc - v;
}

// exclusive block scan of a double and an int at once (in place); totals out
__device__ __forceinline__ void block_xscan_di(double &vd, int &vi, double &td, int &ti, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const double incd = warp_iscan(vd, lane);
    const int inci = warp_iscan(vi, lane);
    if (lane == 31) { r.d[warp] = incd; r.i[warp] = inci; }
    __syncthreads();
    const double wd = lane < NW ? r.d[lane] : 0.0;
    const int wi = lane < NW ? r.i[lane] : 0;
    const double wincd = warp_iscan(wd, lane);
    const int winci = warp_iscan(wi, lane);
    const double woffd = __shfl_sync(FULL, wincd - wd, warp);
    const int woffi = __shfl_sync(FULL, winci - wi, warp);
    td = __shfl_sync(FULL, wincd, 31);
    ti = __shfl_sync(FULL, winci, 31);
    __syncthreads();
    vd = woffd + incd - vd;
    vi = woffi + inci - vi;
}

// exclusive block scan of v (returned, total in `total`) and block sums of
// three ints s (in place)
__device__ __forceinline__ int block_xscan_i4(int v, int (&s)[3], int &total, Red r) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int inc = warp_iscan(v, lane);
    int ws[3];
#pragma unroll
    for (int t = 0; t < 3; ++t) ws[t] = warp_sum(s[t]);
    if (lane == 31) {
        r.i[warp] = inc;
#pragma unroll
        for (int t = 0; t < 3; ++t) r.i[(t + 1) * NW + warp] = ws[t];
    }
    __syncthreads();
    const int w = lane < NW ? r.i[lane] : 0;
    const int winc = warp_iscan(w, lane);
    const int woff = __shfl_sync(FULL, winc - w, warp);
    total = __shfl_sync(FULL, winc, 31);
#pragma unroll
    for (int t = 0; t < 3; ++t) s[t] = warp_sum(lane < NW ? r.i[(t + 1) * NW + lane] : 0);
    __syncthreads();
    return woff + inc - v;
}

// In-place ascending bitonic sort of n <= cap 64-bit keys, padded to a power
// of two with ~0 (cap a power of two).  All threads call it.
__device__ void bitonic_u64(unsigned long long *a, int n, int cap) {
    int P = 1;
    while (P < n) P <<= 1;
    if (P > cap) P = cap;
    for (int i = n + threadIdx.x; i < P; i += NT) a[i] = ~0ull;
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int t = threadIdx.x; t < (P >> 1); t += NT) {
                const int i = ((t / j) * (j << 1)) + (t % j);
                const int l = i + j;
                const bool up = ((i & k) == 0);
                const unsigned long long x = a[i], y = a[l];
                if ((x > y) == up) { a[i] = y; a[l] = x; }
            }
            __syncthreads();
        }
    }
}

// Ascending sort of n unique 64-bit keys in shared memory.  n <= 32: one warp
// by register ranks; n <= NT: ranks summed from slices of the comparisons
// with integer shared atomics into `rank` (n ints), then a scatter; larger n:
// bitonic with capacity `cap`.  All threads call it.
__device__ void sort_keys(unsigned long long *a, int n, int *rank, int cap) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (n <= 1) return;
    if (n <= 32) {
        if (warp == 0) {
            const unsigned long long k = (lane < n) ? a[lane] : ~0ull;
            int r = 0;
            for (int j = 0; j < n; ++j) r += (__shfl_sync(FULL, k, j) < k);
            __syncwarp();
            if (lane < n) a[r] = k;
        }
        __syncthreads();
        return;
    }
    if (n > 256) {  // rank sort costs n*n/NT comparisons per thread
        bitonic_u64(a, n, cap);
        return;
    }
    for (int i = threadIdx.x; i < n; i += NT) rank[i] = 0;
    __syncthreads();
    const int G = NT / n;
    const int per = (n + G - 1) / G;
    if ((int)threadIdx.x < n * G) {
        const int i = threadIdx.x % n, g = threadIdx.x / n;
        const unsigned long long ki = a[i];
        const int j0 = g * per, j1 = min(n, j0 + per);
        int r = 0;
        for (int j = j0; j < j1; ++j) r += (a[j] < ki);
        if (r) atomicAdd(&rank[i], r);
    }
    __syncthreads();
    const unsigned long long mine = ((int)threadIdx.x < n) ? a[threadIdx.x] : 0ull;
    __syncthreads();
    if ((int)threadIdx.x < n) a[rank[threadIdx.x]] = mine;
    __syncthreads();
}

// Ascending bitonic sort of n <= NT keys in shared memory `a`, one key per
// thread in registers: exchanges within a warp by shuffles, across warps
// through two alternating shared buffers (a and a + NT; one barrier each).
__device__ __forceinline__ void sort_reg(unsigned long long *a, int n) {
    const int t = threadIdx.x;
    unsigned long long k = (t < n) ? a[t] : ~0ull;
    int P = 2;
    while (P < n) P <<= 1;
    int buf = 0;
    // (each thread read its own a[t]; the first exchange writes only a[t])
    for (int size = 2; size <= P; size <<= 1) {
        for (int j = size >> 1; j > 0; j >>= 1) {
            unsigned long long o;
            if (j >= 32) {
                unsigned long long *x = a + buf * NT;
                x[t] = k;
                __syncthreads();
                o = x[t ^ j];
                buf ^= 1;
            } else {
                const unsigned lo32 = __shfl_xor_sync(FULL, (unsigned)k, j);
                const unsigned hi32 = __shfl_xor_sync(FULL, (unsigned)(k >> 32), j);
                o = ((unsigned long long)hi32 << 32) | lo32;
            }
            const bool up = (t & size) == 0, lower = (t & j) == 0;
            k = (lower == up) ? (o < k ? o : k) : (o > k ? o : k);
        }
    }
    __syncthreads();  // the last exchange's reads are done
    if (t < n) a[t] = k;
    __syncthreads();
}

__device__ __forceinline__ unsigned long long shfl_xor64(unsigned long long v, int m) {
    const unsigned lo = __shfl_xor_sync(FULL, (unsigned)v, m);
    const unsigned hi = __shfl_xor_sync(FULL, (unsigned)(v >> 32), m);
    return ((unsigned long long)hi << 32) | lo;
}

// The end of the top_k path for up to 64 candidates when the survivors'
// order is their value order, on one warp with everything in registers (two
// entries per lane: entry x = 2 * lane + r):
//   - the candidates (kc: (id << 32) | bits(l)) sorted by value descending,
//     ties by id (a bitonic network); the k survivors are the first
//     min(n, k).  The reference's heap (src/model.c:239-254) holds exactly
//     these k largest when no two of the k + 1 largest values are equal,
//     and its stable sort by probability (src/model.c:275-276) then lists
//     them in value order when no two probabilities are equal;
//   - the survivor softmax (src/model.c:257-269): expf(l - max), fp64 sum,
//     p = e * (1 / (float) sum);
//   - filter_and_sample (src/model.c:72-118): the nucleus cut (cumulative
//     fp64 sum >= top_p), r = u * (float) cut sum, the first r < cumulative.
// The fp64 sums are exact in any order when every term is a multiple of
// ulp(smallest term) below 2^53 of them (e >= 2^-22, p >= 2^-29); returns
// false (nothing decided) when a value or probability tie, a +inf value or
// an inexact sum makes the order matter: the block path then decides.
__device__ __forceinline__ bool warp_tail(const unsigned long long *kc, int cnt, int k, float top_p,
                                          float u, bool cut, float mx, float thr, int lane,
                                          int &res_id, float &res_p, int &res_nf, int &res_n) {
    unsigned long long key[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int x = 2 * lane + r;
        key[r] = ~0ull;
        if (x < cnt) {
            const unsigned long long e = kc[x];
            const unsigned b = (unsigned)(e & 0xffffffffu);
            const unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
            key[r] = ((unsigned long long)(~ord) << 32) | (unsigned)(e >> 32);
        }
    }
    // ascending bitonic sort of the 64 keys (padding ~0 sorts last).  Only
    // the first `lim` (a power of two >= cnt) hold keys: the network's
    // stages up to that size sort them, and the padding behind them is
    // already in order.
    const int lim = (cnt <= 2) ? 2 : 1 << (32 - __clz(cnt - 1));
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1) {
        if (size > lim) break;
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            unsigned long long o[2];
            if (j == 1) {
                o[0] = key[1];
                o[1] = key[0];
            } else {
                o[0] = shfl_xor64(key[0], j >> 1);
                o[1] = shfl_xor64(key[1], j >> 1);
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int x = 2 * lane + r;
                const bool up = (x & size) == 0, lower = (x & j) == 0;
                key[r] = (lower == up) ? (o[r] < key[r] ? o[r] : key[r])
                                       : (o[r] > key[r] ? o[r] : key[r]);
            }
        }
    }
    float l[2], e[2], p[2];
    int id[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const unsigned ord = ~(unsigned)(key[r] >> 32);
        l[r] = __uint_as_float((ord & 0x80000000u) ? (ord ^ 0x80000000u) : ~ord);
        id[r] = (int)(unsigned)(key[r] & 0xffffffffu);
    }
    int n = cnt;
    if (cut) {
        // the candidates' cut and extraction (src/model.c:181-224) on the
        // sorted list: a bucket grows as the value falls, so the counted
        // candidates (buckets below the last) are a prefix, the cut bucket
        // is that of the k-th of them, and the extraction set (l >= ethr) is
        // a prefix too
        const float bscale = __fdiv_rn(127.0f, 20.0f);  // src/model.c:184
        int b[2];
#pragma unroll
        for (int r = 0; r < 2; ++r)
            b[r] = min(max(x86_cvtt(__fmul_rn(__fsub_rn(mx, l[r]), bscale)), 0), HB - 1);
        const bool c0 = 2 * lane < cnt && b[0] < HB - 1, c1 = 2 * lane + 1 < cnt && b[1] < HB - 1;
        const int counted = __popc(__ballot_sync(FULL, c0)) + __popc(__ballot_sync(FULL, c1));
        const int bk0 = __shfl_sync(FULL, b[0], (k - 1) >> 1), bk1 = __shfl_sync(FULL, b[1], (k - 1) >> 1);
        const int kcut = (k - 1 < counted) ? (((k - 1) & 1) ? bk1 : bk0) : HB - 1;
        const float bthr = __fsub_rn(mx, __fdiv_rn((float)(kcut + 1), bscale));  // src/model.c:210-211
        const float ethr = bthr > thr ? bthr : thr;                                // src/model.c:213-214
        const bool x0 = 2 * lane < cnt && l[0] >= ethr, x1 = 2 * lane + 1 < cnt && l[1] >= ethr;
        n = __popc(__ballot_sync(FULL, x0)) + __popc(__ballot_sync(FULL, x1));
    }
    res_n = n;
    if (n == 0) return false;
    const int ns = min(n, k), m = min(n, k + 1);
    // equal values among the first k + 1, or a +inf maximum
    const unsigned hi0 = (unsigned)(key[0] >> 32), hi1 = (unsigned)(key[1] >> 32);
    const unsigned nxt = __shfl_down_sync(FULL, hi0, 1);
    bool tie = (2 * lane + 1 < m && hi0 == hi1) || (2 * lane + 2 < m && hi1 == nxt);
    if (lane == 0) tie |= (~hi0) == 0xff800000u;
    if (__any_sync(FULL, tie)) return false;
    const float lm = __shfl_sync(FULL, l[0], 0);  // the largest survivor
    double s = 0.0;
    float emin = PINF;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const bool sv = 2 * lane + r < ns;
        e[r] = sv ? expf(__fsub_rn(l[r], lm)) : 0.0f;
        s += (double)e[r];
        if (sv && e[r] > 0.0f) emin = fminf(emin, e[r]);
    }
    emin = warp_min(emin);
    if (!(emin >= 0x1p-22f)) return false;
    const double S = warp_sum(s);
    const float inv = __fdiv_rn(1.0f, __double2float_rn(S));
    float pmin = PINF;
    double ls = 0.0;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const bool sv = 2 * lane + r < ns;
        p[r] = sv ? __fmul_rn(e[r], inv) : 0.0f;
        ls += (double)p[r];
        if (sv && p[r] > 0.0f) pmin = fminf(pmin, p[r]);
    }
    // equal probabilities: the stable sort keeps heap order among them
    const float pn = __shfl_down_sync(FULL, p[0], 1);
    const bool ptie = (2 * lane + 1 < ns && p[0] == p[1]) || (2 * lane + 2 < ns && p[1] == pn);
    if (__any_sync(FULL, ptie)) return false;
    pmin = warp_min(pmin);
    if (!(pmin >= 0x1p-29f)) return false;
    const double inc = warp_iscan(ls, lane);
    const double pre = inc - ls;
    // nucleus cut: the first entry whose cumulative sum reaches top_p
    int hit = INT_MAX;
    double hcs = 0.0, cs = pre;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        if (2 * lane + r < ns && hit == INT_MAX) {
            cs += (double)p[r];
            if (cs >= (double)top_p) { hit = 2 * lane + r; hcs = cs; }
        }
    }
    int nf = ns;
    double cs_cut = __shfl_sync(FULL, inc, 31);
    const int best = warp_imin(hit);
    if (best != INT_MAX) {
        cs_cut = __shfl_sync(FULL, hcs, best >> 1);
        nf = best + 1;
    }
    // the draw: the first entry of the nucleus whose cumulative sum exceeds r
    const float rr = __fmul_rn(u, __double2float_rn(cs_cut));
    int hit2 = INT_MAX;
    cs = pre;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        if (2 * lane + r < nf && hit2 == INT_MAX) {
            cs += (double)p[r];
            if ((double)rr < cs) hit2 = 2 * lane + r;
        }
    }
    int pos = warp_imin(hit2);
    if (pos == INT_MAX) pos = nf - 1;
    const int sl = pos >> 1;
    const int i0 = __shfl_sync(FULL, id[0], sl), i1 = __shfl_sync(FULL, id[1], sl);
    const float p0 = __shfl_sync(FULL, p[0], sl), p1 = __shfl_sync(FULL, p[1], sl);
    res_id = (pos & 1) ? i1 : i0;
    res_p = (pos & 1) ? p1 : p0;
    res_nf = nf;
    return true;
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
// nodes of one level root disjoint subtrees and every deeper node has a
// larger index, so this equals the reference's sequential order.
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

// ---------------------------------------------------------- row context --
struct Ctx {
    const float *logits;
    int64_t ld;
    int B, V;
    int *err;
    int *sched;
    uint64_t *mbar;
    Red red;
    Vars *v;
    uint32_t *bits;
    unsigned char *scr;
    float *row;  // 16-byte aligned; element e lives at row[e + sh]
    const float *g;
    int32_t *out_id;
    float *out_prob;
    bm_row_stats_t *stats;
    int rowid;
    int claim;  // thread 0: the row claimed to follow this one
    int succ;   // thread 32 + 1: the row claimed at the release to follow that one
    int mark;   // failed rows get id -1 (the allocation-free entry point)
    int summary;  // the merge kernel: candidates come from per-tile lists
    const int32_t *row_map;  // launch row -> row of the per-row arrays (or NULL)
    uint32_t parity;
    // Point the shared-memory fields at the dynamic shared array.  Called at
    // the top of every non-inlined function: pointers that arrive as
    // arguments lose their address space and every access through them would
    // become a generic load, store or atomic.
    __device__ __forceinline__ void attach() {
        extern __shared__ __align__(128) unsigned char smem_dyn[];
        const Layout L = layout(V);
        mbar = reinterpret_cast<uint64_t *>(smem_dyn + L.mbar);
        red.d = reinterpret_cast<double *>(smem_dyn + L.red);
        red.i = reinterpret_cast<int *>(smem_dyn + L.red + 2 * NW * 8);
        red.f = reinterpret_cast<float *>(smem_dyn + L.red + 2 * NW * 8 + 4 * NW * 4);
        v = reinterpret_cast<Vars *>(smem_dyn + L.vars);
        bits = reinterpret_cast<uint32_t *>(smem_dyn + L.bits);
        scr = smem_dyn + L.scr;
        row = reinterpret_cast<float *>(smem_dyn + L.row);
    }
};

// Issue the bulk copies of one row into the row buffer (one thread).
__device__ __forceinline__ void issue_chunk(const float *g, int V, uint64_t *mbar, float *rowbuf,
                                            int ch) {
    const int sh = (int)(((uintptr_t)g & 15u) >> 2);
    int i0 = sh ? 4 - sh : 0;
    if (i0 > V) i0 = V;
    int n4 = ((V - i0) >> 2) << 2;
    if (n4 < 4 * NCHUNK * 4) n4 = 0;  // tiny rows: plain loads only
    const int s_int0 = (i0 + sh) >> 2;
    const int nint = n4 >> 2;
    const int a = (ch * nint) / NCHUNK, b = ((ch + 1) * nint) / NCHUNK;
    const uint32_t bytes = (uint32_t)(b - a) * 16u;
    mbar_expect_tx(&mbar[ch], bytes);
    if (bytes) bulk_load(rowbuf + 4 * (s_int0 + a), g + i0 + 4 * a, bytes, &mbar[ch]);
}
__device__ __forceinline__ void issue_row(const float *g, int V, uint64_t *mbar, float *rowbuf) {
    for (int ch = 0; ch < NCHUNK; ++ch) issue_chunk(g, V, mbar, rowbuf, ch);
}

// L2 prefetch of a row's 16-byte-aligned interior.
__device__ __forceinline__ void prefetch_row(const float *g, int V) {
    const int sh = (int)(((uintptr_t)g & 15u) >> 2);
    const int i0 = sh ? 4 - sh : 0;
    if (i0 < V) {
        const int n4 = ((V - i0) >> 2) << 2;
        if (n4 >= 16) prefetch_l2(g + i0, (uint32_t)n4 * 4u);
    }
}

// The row buffer is no longer read for this row: let the next row's copy in.
// Warp `cw` issues the copies (one lane per chunk); warp 1 the prefetches,
// so the two sets of instructions do not run one after the other.  The top_k
// path passes cw = 2: its warp 0 finishes short lists right after the
// release.
__device__ __forceinline__ void release_row(Ctx &c, int cw = 0) {
    if (threadIdx.x == 0) {
        // the row claimed to follow this one (thread 0 holds it)
        c.v->released = 1;
        c.v->next_row = c.claim;
    }
    fence_proxy_async();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 1 || warp == cw) {
        const int next_row = c.v->next_row;
        if (next_row < c.B) {
            const int nr = c.row_map ? (int)c.row_map[next_row] : next_row;
            if (warp == cw) {
                if (lane < NCHUNK)
                    issue_chunk(c.logits + (int64_t)nr * c.ld, c.V, c.mbar, c.row, lane);
            } else {
                // the next row's knobs, uniform and history offsets into the
                // staging fields (4-byte asynchronous copies; waited for at
                // the end of this row)
                Vars *v = c.v;
                if (lane >= 8 && lane < 16)
                    cp_async4(reinterpret_cast<uint32_t *>(&v->nk) + (lane - 8),
                              reinterpret_cast<const uint32_t *>(v->p_knobs +
                                                                 (int64_t)nr * v->p_knob_stride) +
                                  (lane - 8));
                if (lane == 16 && v->p_uniform) cp_async4(&v->nu, v->p_uniform + nr);
                if (lane >= 17 && lane < 21 && v->p_hist_off)
                    cp_async4(reinterpret_cast<uint32_t *>(v->nh) + (lane - 17),
                              reinterpret_cast<const uint32_t *>(v->p_hist_off + nr) + (lane - 17));
                if (lane >= 8 && lane < 21) cp_async_commit();
                // the row to follow the next one (published at this row's end)
                if (lane == 1) c.succ = (int)gridDim.x + atomicAdd(c.sched, 1);
                // warm L2 with the row claimed about one round later
                const int pre = next_row + (int)gridDim.x;
                if (lane == 0 && pre < c.B)
                    prefetch_row(c.logits + (int64_t)(c.row_map ? (int)c.row_map[pre] : pre) * c.ld,
                                 c.V);
            }
        }
    }
}

__device__ __forceinline__ void write_result(const Ctx &c, int id, float p, int path, int n_cand,
                                             int n_final, int consumed) {
    if (threadIdx.x == 0) {
        // an exact select that did not converge leaves the row unresolved
        if (c.mark && c.v->fail2) id = -1;
        c.out_id[c.rowid] = id;
        if (c.out_prob) c.out_prob[c.rowid] = p;
        if (c.stats) {
            bm_row_stats_t st;
            st.path = path; st.n_cand = n_cand; st.n_final = n_final; st.consumed = consumed;
            c.stats[c.rowid] = st;
        }
    }
}

// The penalised (and optionally temperature-scaled) logit of element e read
// from global memory; used by the rare paths once the buffer is released.
__device__ __forceinline__ float logit_g(const Ctx &c, int e, bool scale) {
    float x = __ldg(c.g + e);
    const int b = e + c.v->sh;
    if (c.v->pen && ((c.bits[b >> 5] >> (b & 31)) & 1u)) x = penalize(x, c.v->penalty);
    return scale ? __fmul_rn(x, c.v->inv_temp) : x;
}

// ------------------------------------------------------------ load pass --
// Consume the freshly loaded row chunk by chunk: apply the penalty, fill the
// junk lanes of the ragged first / last slots with NaN, and reduce.
template <bool GREEDY, bool PEN, bool SCALE>
__device__ __forceinline__ void load_pass(Ctx &c, const int32_t *hist, float &mx, float &xmin,
                                          float &chk, float &gv, int &gi) {
    Vars *v = c.v;
    const int sh = v->sh, nslots = v->nslots, s0 = v->s_int0, s1 = v->s_int1;
    const int V = c.V;
    const float penalty = v->penalty, inv_temp = v->inv_temp;
    float4 *r4 = reinterpret_cast<float4 *>(c.row);
    mx = -1e30f;
    xmin = PINF;
    chk = 0.0f;  // stays 0 while every logit is finite (l * 0 is NaN for NaN / inf)
    gv = -1e9f;
    gi = INT_MAX;
    // `valid`: lanes that hold elements (junk lanes of the ragged head / tail
    // slots hold NaN and take no part in the reductions)
    float2 chk2 = make_float2(0.0f, 0.0f);
    const float2 it2 = make_float2(inv_temp, inv_temp), z2 = make_float2(0.0f, 0.0f);
    auto consume = [&](int s, float4 x, unsigned valid) {
        const float t[4] = {x.x, x.y, x.z, x.w};
        if (!GREEDY && valid == 0xfu) {
            // whole slot: two three-input max / min, two packed checks
            float2 a = make_float2(t[0], t[1]), b = make_float2(t[2], t[3]);
            if (SCALE) { a = __fmul2_rn(a, it2); b = __fmul2_rn(b, it2); }
            // (gi: the slot of this thread's maximum)
            const float m4 = fmaxf(max3f(a.x, a.y, b.x), b.y);
            if (m4 > mx) { mx = m4; gi = s; }
            xmin = min3f(xmin, min3f(a.x, a.y, b.x), b.y);
            chk2 = __ffma2_rn(a, z2, chk2);
            chk2 = __ffma2_rn(b, z2, chk2);
            return;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (!((valid >> q) & 1u)) continue;
            if (GREEDY) {
                // (the ragged head slot comes last: ties keep the lower id)
                const int e = 4 * s + q - sh;
                if (t[q] > gv || (t[q] == gv && gi != INT_MAX && e < gi)) { gv = t[q]; gi = e; }
            } else {
                const float l = SCALE ? __fmul_rn(t[q], inv_temp) : t[q];
                if (l > mx) gi = s;
                mx = fmaxf(mx, l);
                xmin = fminf(xmin, l);
                chk = __fmaf_rn(l, 0.0f, chk);
            }
        }
    };
    auto plain = [&](int s) -> unsigned {
        float t[4];
        unsigned valid = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int e = 4 * s + q - sh;
            const bool in = e >= 0 && e < V;
            t[q] = in ? __ldg(c.g + e) : __int_as_float(0x7fc00000);
            valid |= (unsigned)in << q;
        }
        const float4 x = make_float4(t[0], t[1], t[2], t[3]);
        r4[s] = x;
        return valid;
    };
    // lanes of slot s that hold elements
    auto valid_of = [&](int s) {
        unsigned valid = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int e = 4 * s + q - sh;
            valid |= (unsigned)(e >= 0 && e < V) << q;
        }
        return valid;
    };
    const int nint = s1 - s0;
    // rows with a bulk-copied interior have at most one ragged head slot and
    // two tail slots: the last threads load them first and consume them after
    // the interior, so the global-load latency overlaps the chunk waits
    int es = -1;
    unsigned evld = 0;
    if (nint > 0) {
        const int ntl = nslots - s1, nedge = s0 + ntl;
        const int i = (int)threadIdx.x - (NT - nedge);
        if (i >= 0) {
            es = (i < s0) ? i : s1 + (i - s0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int e = 4 * es + q - sh;
                const bool in = e >= 0 && e < V;
                if (in) cp_async4(c.row + 4 * es + q, c.g + e);
                else c.row[4 * es + q] = __int_as_float(0x7fc00000);
                evld |= (unsigned)in << q;
            }
            cp_async_commit();
        }
    } else if (!PEN) {
        // tiny row: every slot by plain loads
        for (int s = threadIdx.x; s < nslots; s += NT) {
            const unsigned vl = plain(s);
            consume(s, r4[s], vl);
        }
    } else {
        for (int s = threadIdx.x; s < nslots; s += NT) (void)plain(s);
    }
    bool ok = true;
    if (PEN) {
        // The row lands whole first; then the logit of each distinct history
        // id is penalised in place by one thread (the bit's previous value
        // tells the first claimant), and the pass reads the penalised row.
        // (A per-slot test inside the pass diverges in most warps: about one
        // lane in 32 holds a history id, and the division is long.)
        const int h0 = v->h0, h1 = v->h1;
        int i = h0 + (int)threadIdx.x;
        int ids[4];
        auto fetch_ids = [&]() {
#pragma unroll
            for (int q = 0; q < 4; ++q) ids[q] = (i + q * NT < h1) ? __ldg(&hist[i + q * NT]) : -1;
        };
        fetch_ids();  // (in flight during the waits)
        if (nint > 0) {
            for (int ch = 0; ch < NCHUNK; ++ch)
                if (!mbar_wait(&c.mbar[ch], c.parity)) { ok = false; break; }
            if (es >= 0) cp_async_wait_all();
        }
        if (!ok) {
            atomicOr(c.err, 1);
            v->fail = 1;
        }
        __syncthreads();
        if (!v->fail) {
            for (;;) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int id = ids[q];
                    if (id >= 0 && id < V && !protected_id(id)) {
                        const int b = id + sh;
                        const uint32_t m = 1u << (b & 31);
                        if (!(atomicOr(&c.bits[b >> 5], m) & m)) c.row[b] = penalize(c.row[b], penalty);
                    }
                }
                i += 4 * NT;
                if (i >= h1) break;
                fetch_ids();
            }
        }
        __syncthreads();
        ok = !v->fail;
        if (ok && nint > 0) {
            int s = s0 + ((int)threadIdx.x - s0 % NT + NT) % NT;
            if (s < s1) {
                float4 xn = r4[s];
                for (; s < s1; s += NT) {
                    const float4 x = xn;
                    if (s + NT < s1) xn = r4[s + NT];
                    consume(s, x, 0xfu);
                }
            }
        } else if (ok) {
            for (int s = threadIdx.x; s < nslots; s += NT) consume(s, r4[s], valid_of(s));
        }
    } else if (nint > 0) {
        // interior, chunk by chunk; each thread takes its slots of a chunk
        // (s = tid mod NT) in ascending order, the next slot's load issued
        // before the current slot's work (one dependent shared load a slot
        // would leave the pass latency-bound)
        for (int ch = 0; ch < NCHUNK; ++ch) {
            const int a = s0 + (ch * nint) / NCHUNK, b = s0 + ((ch + 1) * nint) / NCHUNK;
            int s = a + ((int)threadIdx.x - a % NT + NT) % NT;
            if (s >= b) continue;
            if (!mbar_wait(&c.mbar[ch], c.parity)) {
                atomicOr(c.err, 1);
                v->fail = 1;
                ok = false;
                break;
            }
            float4 xn = r4[s];
            for (; s < b; s += NT) {
                const float4 x = xn;
                if (s + NT < b) xn = r4[s + NT];
                consume(s, x, 0xfu);
            }
        }
    }
    if (es >= 0) {
        if (!PEN) cp_async_wait_all();
        if (ok) consume(es, r4[es], evld);
    }
    chk = __fadd_rn(chk, __fadd_rn(chk2.x, chk2.y));
}

// Argmax over the scaled penalised logits with the guard semantics of
// src/model.c:227-237 and 296-303 (start from element 0, strict '>'),
// read from global memory.
__device__ __noinline__ int guard_argmax(Ctx c) {
    c.attach();
    const int V = c.V;
    const bool scale = (c.v->inv_temp != 1.0f);
    float bv = 0.f;
    int bi = INT_MAX;
    for (int e = threadIdx.x; e < V; e += NT) {
        const float l = logit_g(c, e, scale);
        if (l == l) argmax_combine(bv, bi, l, e);
    }
    block_argmax(bv, bi, c.red);
    const float l0 = logit_g(c, 0, scale);
    if (l0 != l0 || bi == INT_MAX) return 0;
    return bi;
}

// The candidates (l >= thr) of a row with a real min_p threshold, listed in
// kc as (id << 32) | bits(l) when they are at most KCAP; returns their count.
// Each thread marks its candidates, a bit per element, in registers.  A
// thread whose own maximum in the load pass (tmax: the same scaled values of
// the same interior slots) lies below thr has none there and skips its
// slots; the ragged head / tail slots were consumed by other threads in the
// load pass, so their threads here always scan.  The count's block scan
// ends the mask reads; the caller's next barrier orders the list writes.
template <bool SCALE>
__device__ __forceinline__ int list_candidates(Ctx &c, float tmax, unsigned long long *kc) {
    const int lane = threadIdx.x & 31;
    Vars *v = c.v;
    const int sh = v->sh, nslots = v->nslots;
    const float thr = v->thr, inv_temp = v->inv_temp;
    const float4 *r4 = reinterpret_cast<const float4 *>(c.row);
    bool edge = (int)threadIdx.x < v->s_int0;
    for (int s = v->s_int1; s < nslots; ++s) edge |= (s % NT) == (int)threadIdx.x;
    const bool need = edge || !(tmax < thr);
    // candidate bits of slot s: bit q for element q of the slot
    auto bits4 = [&](int s) -> uint32_t {
        const float4 x = r4[s];
        const float t[4] = {x.x, x.y, x.z, x.w};
        uint32_t b4 = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float l = SCALE ? __fmul_rn(t[q], inv_temp) : t[q];
            b4 |= (l >= thr ? 1u : 0u) << q;
        }
        return b4;
    };
    uint32_t wv[MASKW] = {0u, 0u, 0u, 0u};
    const uint32_t scanners = __ballot_sync(FULL, need);
    if (__popc(scanners) <= 8) {
        // few threads of this warp have candidates: the whole warp scans
        // each one's slots (lane i takes its slot i), and groups of 8
        // lanes assemble its mask words (word q = slots 8q..8q+7)
        for (uint32_t m = scanners; m; m &= m - 1) {
            const int ln = __ffs(m) - 1;
            const int s = (int)(threadIdx.x & ~31u) + ln + lane * NT;
            uint32_t w = (s < nslots) ? bits4(s) << (4 * (lane & 7)) : 0u;
            w |= __shfl_xor_sync(FULL, w, 1);
            w |= __shfl_xor_sync(FULL, w, 2);
            w |= __shfl_xor_sync(FULL, w, 4);
#pragma unroll
            for (int q = 0; q < MASKW; ++q) {
                const uint32_t wq = __shfl_sync(FULL, w, 8 * q);
                if (lane == ln) wv[q] = wq;
            }
        }
    } else if (need) {
        uint32_t w = 0;
        int i = 0;
        for (int s = threadIdx.x; s < nslots; s += NT, ++i) {
            w |= bits4(s) << (4 * (i & 7));
            if ((i & 7) == 7) {
#pragma unroll
                for (int q = 0; q < MASKW; ++q)
                    if (q == (i >> 3)) wv[q] = w;
                w = 0;
            }
        }
        if (i & 7) {
#pragma unroll
            for (int q = 0; q < MASKW; ++q)
                if (q == (i >> 3)) wv[q] = w;
        }
    }
    int nb = 0;
#pragma unroll
    for (int q = 0; q < MASKW; ++q) nb += __popc(wv[q]);
    int tot;
    int j = block_xscan_i(nb, tot, c.red);
    if (tot <= KCAP) {
#pragma unroll
        for (int q = 0; q < MASKW; ++q) {
            uint32_t m = wv[q];
            while (m) {
                const int bp = __ffs(m) - 1;
                m &= m - 1;
                const int s = threadIdx.x + (8 * q + (bp >> 2)) * NT;
                const int r = min(4 * s + (bp & 3), 4 * nslots - 1);
                const float l = SCALE ? __fmul_rn(c.row[r], inv_temp) : c.row[r];
                kc[j++] = ((unsigned long long)(unsigned)(r - sh) << 32) | __float_as_uint(l);
            }
        }
    }
    return tot;
}

// ---------------------------------------------------------------- top_k --
template <bool SCALE>
__device__ __forceinline__ void topk_path(Ctx &c, float tmax) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Vars *v = c.v;
    const int sh = v->sh, nslots = v->nslots, V = c.V, k = v->k;
    const float mx = v->mx, thr = v->thr, inv_temp = v->inv_temp;
    const float4 *r4 = reinterpret_cast<const float4 *>(c.row);
    uint32_t *kh = reinterpret_cast<uint32_t *>(c.scr);                            // 8 x 128
    unsigned long long *kc = reinterpret_cast<unsigned long long *>(c.scr + 4096);  // KCAP
    const float bscale = __fdiv_rn(127.0f, 20.0f);  // src/model.c:184
    constexpr bool collect = false;  // the streaming branch lists after the cut
    float ethr;
    // cut bucket: first bucket whose running count reaches k (src/model.c:199-207)
    auto cut_of = [&]() {
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
            const uint32_t inc = warp_iscan(ls, lane);
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
    };
    // Above a real min_p threshold the candidates are usually few: one pass
    // marks them (a bit per element, no branch), a gather lists them, and the
    // histogram, cut and extraction work on that list.
    bool listed = false;
    bool early = false;  // the row buffer was released right after the listing
    if (c.summary) {
        // The merge kernel listed every tile-list entry with l >= thr.  Each
        // tile's list holds its KS largest values, so it holds every value of
        // the tile above the tile's KS-th (v->sumvk: their largest).  The
        // cut's buckets and the extraction set are exact when every value
        // they contain lies above sumvk; otherwise the row takes the full
        // path (v->fb).
        listed = true;
        if (v->kcnt > KCAP) {  // more than the list holds: the full path
            if (threadIdx.x == 0) v->fb = 1;
            __syncthreads();
            return;
        }
        for (int q = threadIdx.x; q < 8 * HB; q += NT) kh[q] = 0;
        __syncthreads();
        const int tot = v->kcnt;
        for (int q = threadIdx.x; q < tot; q += NT) {
            const float l = __uint_as_float((unsigned)(kc[q] & 0xffffffffu));
            int b = x86_cvtt(__fmul_rn(__fsub_rn(mx, l), bscale));
            b = min(max(b, 0), HB - 1);
            if (b < HB - 1) atomicAdd(&kh[b], 1u);
        }
        __syncthreads();
        cut_of();
        const int cut = v->kcut;
        const float bthr = __fsub_rn(mx, __fdiv_rn((float)(cut + 1), bscale));  // src/model.c:210-211
        ethr = bthr > thr ? bthr : thr;                                      // src/model.c:213-214
        // lowest value in buckets 0..cut (half a bucket of margin) or at or
        // above ethr
        const float lb = __fsub_rn(mx, __fdiv_rn((float)cut + 1.5f, bscale));
        const float need = fmaxf(thr, fminf(lb, ethr));
        if (!(v->sumvk < need) || !(fabsf(mx) < 1e30f)) {
            if (threadIdx.x == 0) v->fb = 1;
            __syncthreads();
            return;
        }
        constexpr int PQ = KCAP / NT;
        unsigned long long e[PQ];
        bool keep[PQ];
        int mine = 0;
#pragma unroll
        for (int q = 0; q < PQ; ++q) {
            const int jj = threadIdx.x + q * NT;
            e[q] = (jj < tot) ? kc[jj] : 0ull;
            keep[q] = jj < tot && __uint_as_float((unsigned)(e[q] & 0xffffffffu)) >= ethr;
            mine += keep[q] ? 1 : 0;
        }
        int n2;
        int o = block_xscan_i(mine, n2, c.red);
#pragma unroll
        for (int q = 0; q < PQ; ++q)
            if (keep[q]) kc[o++] = e[q];
        if (threadIdx.x == 0) v->kcnt = n2;
        __syncthreads();
    } else if (v->min_p > 0.0f) {
        const int tot = list_candidates<SCALE>(c, tmax, kc);
        if (tot <= KCAP) {
            listed = true;
            for (int q = 0; q < 8 * HB; q += NT)
                if (q + (int)threadIdx.x < 8 * HB) kh[q + threadIdx.x] = 0;
            // the row buffer is no longer read (its barrier orders the list
            // writes above before the reads below): the next row's copy
            // starts here, beside the cut and the extraction
            release_row(c, 2);
            early = true;
            if (tot <= 64 && v->top_p < 1.0f) {
                // few candidates: cut, extraction and the end of the row on
                // one warp (the block path below when the warp cannot decide)
                if (warp == 0) {
                    int rid = 0, rnf = 0, rn = 0;
                    float rp = 0.0f;
                    const bool ok = warp_tail(kc, tot, k, v->top_p, v->u, true, mx, thr, lane, rid,
                                              rp, rnf, rn);
                    if (lane == 0) {
                        v->wt = ok ? 1 : 0;
                        v->res_id = rid;
                        v->res_p = rp;
                        v->n_final = rnf;
                        v->kcnt = rn;
                    }
                }
                __syncthreads();
                if (v->wt) {
                    write_result(c, v->res_id, v->res_p, 3, v->kcnt, v->n_final, 1);
                    return;
                }
            }
            // histogram of the listed candidates (src/model.c:185-195); the last
            // bucket never decides the cut, so it is not counted
            for (int q = threadIdx.x; q < tot; q += NT) {
                const float l = __uint_as_float((unsigned)(kc[q] & 0xffffffffu));
                int b = x86_cvtt(__fmul_rn(__fsub_rn(mx, l), bscale));
                b = min(max(b, 0), HB - 1);
                if (b < HB - 1) atomicAdd(&kh[b], 1u);
            }
            __syncthreads();
            cut_of();
            const int cut = v->kcut;
            const float bthr = __fsub_rn(mx, __fdiv_rn((float)(cut + 1), bscale));  // src/model.c:210-211
            ethr = bthr > thr ? bthr : thr;                                      // src/model.c:213-214
            // the extraction set (src/model.c:217-224): the listed candidates
            // with l >= ethr, compacted
            constexpr int PQ = KCAP / NT;
            unsigned long long e[PQ];
            bool keep[PQ];
            int mine = 0;
#pragma unroll
            for (int q = 0; q < PQ; ++q) {
                const int jj = threadIdx.x + q * NT;
                e[q] = (jj < tot) ? kc[jj] : 0ull;
                keep[q] = jj < tot && __uint_as_float((unsigned)(e[q] & 0xffffffffu)) >= ethr;
                mine += keep[q] ? 1 : 0;
            }
            int n2;
            int o = block_xscan_i(mine, n2, c.red);
#pragma unroll
            for (int q = 0; q < PQ; ++q)
                if (keep[q]) kc[o++] = e[q];
            if (threadIdx.x == 0) v->kcnt = n2;
            __syncthreads();
        } else {
            __syncthreads();
        }
    }
    if (!listed) {
        for (int i = threadIdx.x; i < 8 * HB; i += NT) kh[i] = 0;
        if (threadIdx.x == 0) v->kcnt = 0;
        __syncthreads();
        uint32_t *myh = kh + (warp & 7) * HB;
        unsigned long long lo8 = 0, hi8 = 0;  // per-thread counts of buckets 0..15
        // candidates: every thread keeps its first KREG in its own list slots
        // (index q * NT + tid), further ones go to the shared overflow part
        // through an atomic (v->kcnt counts them)
        int cnt = 0;
        auto put = [&](unsigned long long ent) {
            if (cnt < KREG) {
                kc[cnt * NT + threadIdx.x] = ent;
            } else {
                const int pos = atomicAdd(&v->kcnt, 1);
                if (pos < KOVF) kc[KREG * NT + pos] = ent;
            }
            ++cnt;
        };
        // histogram of (max - l) over l >= thr (src/model.c:185-195); the last
        // bucket never decides the cut, so it is not counted
        for (int s = threadIdx.x; s < nslots; s += NT) {
            const float4 x = r4[s];
            const float t[4] = {x.x, x.y, x.z, x.w};
    #pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float l = SCALE ? __fmul_rn(t[q], inv_temp) : t[q];
                if (l >= thr) {
                    int b = x86_cvtt(__fmul_rn(__fsub_rn(mx, l), bscale));
                    b = min(max(b, 0), HB - 1);
                    // buckets 0..15 (where the cut of a top_k <= 256 nearly always
                    // lies, and where flat rows pile up) in 8-bit register fields
                    if (b < 8) lo8 += 1ull << (8 * b);
                    else if (b < 16) hi8 += 1ull << (8 * (b - 8));
                    else if (b < HB - 1) atomicAdd(&myh[b], 1u);
                    if (collect)
                        put(((unsigned long long)(unsigned)(4 * s + q - sh) << 32) | __float_as_uint(l));
                }
            }
        }
        {
            // widen the 8-bit fields to 16 bits (a warp holds at most 32 * 100
            // per bucket), sum over the warp, add 16 counts to the histogram
            const unsigned long long M = 0x00ff00ff00ff00ffull;
            unsigned long long f[4] = {lo8 & M, (lo8 >> 8) & M, hi8 & M, (hi8 >> 8) & M};
    #pragma unroll
            for (int j = 0; j < 4; ++j) f[j] = warp_sum(f[j]);
            if (lane < 16) {
                const int j = lane >> 3, q = lane & 7;  // bucket = 8j + q
                const unsigned long long fw = f[2 * j + (q & 1)];
                const unsigned cnt16 = (unsigned)((fw >> (16 * (q >> 1))) & 0xffffu);
                if (cnt16) atomicAdd(&kh[lane], cnt16);
            }
        }
        __syncthreads();
        cut_of();
        const int cut = v->kcut;
        const float bthr = __fsub_rn(mx, __fdiv_rn((float)(cut + 1), bscale));  // src/model.c:210-211
        ethr = bthr > thr ? bthr : thr;                                      // src/model.c:213-214
        int novf = v->kcnt;
        if (!(collect && novf <= KOVF)) {
            // extraction pass (src/model.c:217-224), unordered here
            __syncthreads();
            if (threadIdx.x == 0) v->kcnt = 0;
            cnt = 0;
            __syncthreads();
            for (int s = threadIdx.x; s < nslots; s += NT) {
                const float4 x = r4[s];
                const float t[4] = {x.x, x.y, x.z, x.w};
    #pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float l = SCALE ? __fmul_rn(t[q], inv_temp) : t[q];
                    if (l >= ethr)
                        put(((unsigned long long)(unsigned)(4 * s + q - sh) << 32) | __float_as_uint(l));
                }
            }
            __syncthreads();
            novf = v->kcnt;
        }
        // the extraction set: the listed candidates with l >= ethr, compacted
        // (block scan of the per-thread counts; fixed-size register staging)
        {
            constexpr int OQ = KOVF / NT;
            unsigned long long e[KREG + OQ];
            bool keep[KREG + OQ];
            const int own = min(cnt, KREG);
            const bool fits = novf <= KOVF;
    #pragma unroll
            for (int q = 0; q < KREG; ++q) {
                e[q] = (q < own) ? kc[q * NT + threadIdx.x] : 0ull;
                keep[q] = fits && q < own && __uint_as_float((unsigned)(e[q] & 0xffffffffu)) >= ethr;
            }
    #pragma unroll
            for (int q = 0; q < OQ; ++q) {
                const int i = threadIdx.x + q * NT;
                e[KREG + q] = (fits && i < novf) ? kc[KREG * NT + i] : 0ull;
                keep[KREG + q] = fits && i < novf &&
                                 __uint_as_float((unsigned)(e[KREG + q] & 0xffffffffu)) >= ethr;
            }
            int mine = 0;
    #pragma unroll
            for (int q = 0; q < KREG + OQ; ++q) mine += keep[q] ? 1 : 0;
            int tot;
            int j = block_xscan_i(mine, tot, c.red);
            __syncthreads();
    #pragma unroll
            for (int q = 0; q < KREG + OQ; ++q)
                if (keep[q]) kc[j++] = e[q];
            // more candidates than the list holds: the global-memory path below
            if (threadIdx.x == 0) v->kcnt = fits ? tot : KCAP + 1;
            __syncthreads();
        }
    }
    const int n = v->kcnt;
    if (c.summary && (n == 0 || n > KCAP)) {
        // the guard and the overflow paths read the logits: the full path
        if (threadIdx.x == 0) v->fb = 1;
        __syncthreads();
        return;
    }
    // the buffer is no longer needed: the rest works on the candidate list
    // (or re-reads global memory on the rare overflow / guard paths)
    if (!c.summary && !early) release_row(c);
    if (n == 0) {  // argmax guard (src/model.c:227-237)
        const int id = guard_argmax(c);
        write_result(c, id, 1.0f, 2, 0, 0, 0);
        return;
    }
    if (n <= 64 && v->top_p < 1.0f) {
        // short lists in value order: one warp, no block barrier
        if (warp == 0) {
            int rid = 0, rnf = 0;
            float rp = 0.0f;
            int rn = 0;
            const bool ok = warp_tail(kc, n, k, v->top_p, v->u, false, 0.0f, 0.0f, lane, rid, rp,
                                      rnf, rn);
            if (lane == 0) {
                v->wt = ok ? 1 : 0;
                v->res_id = rid;
                v->res_p = rp;
                v->n_final = rnf;
            }
        }
        __syncthreads();
        if (v->wt) {
            write_result(c, v->res_id, v->res_p, 3, n, v->n_final, 1);
            return;
        }
    }
    float *hv = reinterpret_cast<float *>(c.scr);         // 256 (reuses the histogram)
    int *hi = reinterpret_cast<int *>(c.scr + 1024);      // 256
    float *pv = reinterpret_cast<float *>(c.scr + 2048);  // 256 probabilities
    int *rk = reinterpret_cast<int *>(c.scr + 3072);      // 256 ranks
    const float top_p = v->top_p;
    const int ns = min(n, k);
    // Survivors in the reference's heap layout (src/model.c:239-254): the
    // candidates by id, a Floyd heap of the first k, root replacements.
    auto exact_select = [&]() {
        if (n <= KCAP) {
            // by id (ids are unique)
            if (n <= NT) sort_reg(kc, n);
            else sort_keys(kc, n, reinterpret_cast<int *>(c.scr), KCAP);
            if (warp == 0) {
                const int first = min(n, k);
                for (int q = lane; q < first; q += 32) {
                    hv[q] = __uint_as_float((unsigned)(kc[q] & 0xffffffffu));
                    hi[q] = (int)(kc[q] >> 32);
                }
                __syncwarp();
                if (n > k) {  // heap top-k (src/model.c:240-254)
                    warp_heapify(hv, hi, k, lane);
                    for (int base = k; base < n; base += 32) {
                        const int j = base + lane;
                        float val = 0.f;
                        int id = 0;
                        if (j < n) {
                            val = __uint_as_float((unsigned)(kc[j] & 0xffffffffu));
                            id = (int)(kc[j] >> 32);
                        }
                        const float root = hv[0];
                        unsigned mr = __ballot_sync(FULL, j < n && val > root);
                        while (mr) {
                            const int src = __ffs(mr) - 1;
                            const float vb = __shfl_sync(FULL, val, src);
                            const int ib = __shfl_sync(FULL, id, src);
                            if (lane == 0 && vb > hv[0]) { hv[0] = vb; hi[0] = ib; heap_down(hv, hi, k, 0); }
                            __syncwarp();
                            mr &= mr - 1;
                        }
                    }
                }
            }
        } else {
            // more candidates than the list holds: stream them in id order from
            // global memory through the same heap rules
            if (warp == 0) {
                int filled = 0;
                for (int base = 0; base < V; base += 32) {
                    const int e = base + lane;
                    float l = 0.f;
                    bool ok = false;
                    if (e < V) {
                        l = logit_g(c, e, SCALE);
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
    };
    // Survivors by value: when top_p < 1 and no two of the k + 1 largest
    // values are equal, the heap holds exactly the k largest and the stable
    // sort by probability puts them in value order, so the heap layout is not
    // needed (probability ties are checked after the softmax).  Sorts a copy
    // of the candidates; false when a tie needs the heap layout.
    auto value_select = [&]() -> bool {
        unsigned long long *kv = kc + 1024;  // n <= NT: room for sort_reg's buffers
        for (int i = threadIdx.x; i < n; i += NT) {
            const unsigned long long e0 = kc[i];
            const unsigned u = (unsigned)(e0 & 0xffffffffu);
            const unsigned ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            kv[i] = ((unsigned long long)(~ord) << 32) | (unsigned)(e0 >> 32);
        }
        __syncthreads();
        sort_reg(kv, n);
        bool tie = false;
        const int m = min(n, k + 1);
        for (int j = threadIdx.x; j + 1 < m; j += NT)
            tie |= (kv[j] >> 32) == (kv[j + 1] >> 32);
        // a +inf value makes the sums NaN: the walk's fallback element then
        // depends on the heap layout
        if (threadIdx.x == 0) tie |= (~(unsigned)(kv[0] >> 32)) == 0xff800000u;
        tie = __syncthreads_or(tie);
        if (!tie) {
            for (int j = threadIdx.x; j < ns; j += NT) {
                const unsigned ord = ~(unsigned)(kv[j] >> 32);
                const unsigned u = (ord & 0x80000000u) ? (ord ^ 0x80000000u) : ~ord;
                hv[j] = __uint_as_float(u);
                hi[j] = (int)(unsigned)(kv[j] & 0xffffffffu);
            }
        }
        __syncthreads();
        return !tie;
    };
    // survivor softmax (src/model.c:257-269) over hv[0..ns), warp 0, <= 8 per
    // lane in array order; v->ln2 = 1 when the fp64 sum is order-independent
    auto softmax = [&]() {
        // survivor softmax (src/model.c:257-269), warp 0, <= 8 per lane in order
        if (warp == 0) {
            float val[8];
            float lm = -1e30f;
    #pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int j = lane * 8 + q;
                val[q] = (j < ns) ? hv[j] : -1e30f;
                if (j < ns) lm = fmaxf(lm, val[q]);
            }
            lm = warp_max(lm);
            float ev[8];
            double s = 0.0;
            float emin = PINF;
    #pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int j = lane * 8 + q;
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
            const float inv = __fdiv_rn(1.0f, __double2float_rn(S));
    #pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int j = lane * 8 + q;
                if (j < ns) pv[j] = __fmul_rn(ev[q], inv);
            }
            if (lane == 0) { v->S = S; v->ln2 = (emin >= 0x1p-22f) ? 1 : 0; }
        }
        __syncthreads();
    };
    bool by_value = (top_p < 1.0f) && n <= NT && value_select();
    if (!by_value) exact_select();
    __syncthreads();
    softmax();
    if (by_value) {
        // equal probabilities keep heap order in the stable sort; a sum that
        // depends on the order must follow the heap layout too
        bool tie = !v->ln2;
        for (int j = threadIdx.x; j + 1 < ns; j += NT) tie |= pv[j] == pv[j + 1];
        if (__syncthreads_or(tie)) {
            by_value = false;
            exact_select();
            __syncthreads();
            softmax();
        }
    }
    const double S = v->S;
    if (S != S) {  // NaN mass: every comparison fails, the walk returns the last
        write_result(c, hi[ns - 1], pv[ns - 1], 3, n, ns, 1);
        return;
    }
    // stable descending sort when top_p < 1 (src/model.c:275-276); the value
    // selection is in that order already
    unsigned long long *srt = kc;
    if (top_p < 1.0f && !by_value) {
        for (int j = threadIdx.x; j < ns; j += NT) rk[j] = 0;
        __syncthreads();
        const int G = NT / ns;
        if ((int)threadIdx.x < G * ns) {
            const int j = threadIdx.x % ns, g = threadIdx.x / ns;
            const int per = (ns + G - 1) / G;
            const int a = g * per, b = min(ns, a + per);
            const float pj = pv[j];
            int r = 0;
            for (int i = a; i < b; ++i) {
                const float pi = pv[i];
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
        float pmin = PINF;
        double ls = 0.0;
        for (int j = b; j < e; ++j) {
            const float p = __uint_as_float((unsigned)(srt[j] & 0xffffffffu));
            ls += (double)p;
            if (p > 0.0f) pmin = fminf(pmin, p);
        }
        pmin = warp_min(pmin);
        const double inc = warp_iscan(ls, lane);
        const double pre = inc - ls;
        const bool exact = (pmin >= 0x1p-29f);
        int nf = ns;
        double cs_cut = __shfl_sync(FULL, inc, 31);
        if (top_p < 1.0f) {
            if (exact) {
                int hit = INT_MAX;
                double hcs = 0.0, cs = pre;
                for (int j = b; j < e; ++j) {
                    cs += (double)__uint_as_float((unsigned)(srt[j] & 0xffffffffu));
                    if (cs >= (double)top_p) { hit = j; hcs = cs; break; }
                }
                const int best = warp_imin(hit);
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
        const float r = __fmul_rn(v->u, __double2float_rn(cs_cut));
        int pos = nf - 1;
        if (exact) {
            int hit = INT_MAX;
            double cs = pre;
            for (int j = b; j < min(e, nf); ++j) {
                cs += (double)__uint_as_float((unsigned)(srt[j] & 0xffffffffu));
                if ((double)r < cs) { hit = j; break; }
            }
            const int best = warp_imin(hit);
            if (best != INT_MAX) pos = best;
        } else {
            double cs = 0.0;
            for (int j = 0; j < nf; ++j) {
                cs += (double)__uint_as_float((unsigned)(srt[j] & 0xffffffffu));
                if ((double)r < cs) { pos = j; break; }
            }
        }
        if (lane == 0) {
            const unsigned long long kk = srt[pos];
            v->res_id = (int)(kk >> 32);
            v->res_p = __uint_as_float((unsigned)(kk & 0xffffffffu));
            v->n_final = nf;
        }
    }
    __syncthreads();
    write_result(c, v->res_id, v->res_p, 3, n, v->n_final, 1);
}

// ------------------------------------------------------ full vocabulary --
// Selection targets in canonical order (p desc, id asc).
enum { T_MASS_GE = 0, T_MASS_GT = 1, T_POS = 2 };

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

// e of element `e` recomputed from global memory (bit-identical to the exp
// pass): -0 for non-candidates.
__device__ __forceinline__ float e_global(const Ctx &c, int e, bool scale) {
    const float l = logit_g(c, e, scale);
    if (!(l >= c.v->thr)) return -0.0f;
    return exp_one(__fsub_rn(l, c.v->mx));
}

// One exact pass over global memory (rare paths): mass / count above phi,
// mass / count inside [plo, phi], inside elements appended to `list`.
__device__ __forceinline__ PassOut exact_pass_g(Ctx &c, bool scale, float plo, float phi,
                                                unsigned long long *list, int cap) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Vars *v = c.v;
    const float inv_sum = v->inv_sum;
    const int V = c.V;
    if (threadIdx.x == 0) v->ln3 = 0;
    __syncthreads();
    double au = 0.0, ai = 0.0;
    int cu = 0, ci = 0;
    for (int base = warp * 32; base < V; base += NT) {
        const int e = base + lane;
        float p = -0.0f;
        if (e < V) p = __fmul_rn(e_global(c, e, scale), inv_sum);
        const int pb = __float_as_int(p);
        const bool up = pb > __float_as_int(phi);
        const bool in = !up && pb >= __float_as_int(plo);
        au += up ? (double)p : 0.0;
        ai += in ? (double)p : 0.0;
        cu += up;
        ci += in;
        const unsigned m = __ballot_sync(FULL, in);
        if (m) {
            const int leader = __ffs(m) - 1;
            int bpos = 0;
            if (lane == leader) bpos = atomicAdd(&v->ln3, __popc(m));
            bpos = __shfl_sync(FULL, bpos, leader);
            if (in) {
                const int pos = bpos + __popc(m & ((1u << lane) - 1));
                if (pos < cap) list[pos] = canon_key(p, e);
            }
        }
    }
    PassOut o;
    o.above = au;
    o.in_mass = ai;
    o.cnt_above = cu;
    o.in_cnt = ci;
    block_sum4(o.above, o.in_mass, o.cnt_above, o.in_cnt, c.red);
    return o;
}

// Walk a sorted key list from a starting mass, on one warp: first j with
// start + cum(j) >= T (mode 0), > T (mode 1), or j == j2 (mode 2).
__device__ __forceinline__ void warp_walk(const unsigned long long *keys, int n, double start,
                                          int mode, double T, int j2, Vars *v, int lane) {
    const int per = (n + 31) / 32;
    const int b = lane * per, e = min(n, b + per);
    double s = 0.0;
    for (int j = b; j < e; ++j) s += (double)key_p(keys[j]);
    const double inc = warp_iscan(s, lane);
    const double pre = start + (inc - s);
    int hit = INT_MAX;
    double hit_cs = 0.0;
    double cs = pre;
    for (int j = b; j < e; ++j) {
        cs += (double)key_p(keys[j]);
        const bool ok = (mode == T_MASS_GE) ? (cs >= T) : (mode == T_MASS_GT) ? (cs > T) : (j == j2);
        if (ok) { hit = j; hit_cs = cs; break; }
    }
    const int best = warp_imin(hit);
    if (best != INT_MAX) {
        const double hcs = __shfl_sync(FULL, hit_cs, best / per);
        if (lane == 0) { v->sel_found = 1; v->sel_j = best; v->cs = hcs; }
    } else {
        const double tot = __shfl_sync(FULL, inc, 31);
        if (lane == 0) { v->sel_found = 0; v->sel_j = n; v->cs = start + tot; }
    }
}

__device__ __forceinline__ int classify(const PassOut &o, int mode, double T, int m) {
    // 0 inside, 1 above the window, 2 below it
    if (mode == T_POS) {
        if (m < o.cnt_above) return 1;
        if (m >= o.cnt_above + o.in_cnt) return 2;
        return 0;
    }
    const bool hi = (mode == T_MASS_GE) ? (o.above >= T) : (o.above > T);
    if (hi && o.cnt_above > 0) return 1;
    const double tot = o.above + o.in_mass;
    const bool reach = (mode == T_MASS_GE) ? (tot >= T) : (tot > T);
    return reach ? 0 : 2;
}

// Resolve one target from a collected, sorted window list.  Returns 1 and
// fills `out` when the crossing lies in the list.
__device__ __forceinline__ int resolve_list(Ctx &c, const unsigned long long *list,
                                            const PassOut &o, int mode, double T, int m,
                                            Sel &out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Vars *v = c.v;
    const int n = o.in_cnt;
    if (classify(o, mode, T, m) != 0) return 0;
    if (warp == 0) warp_walk(list, n, o.above, mode, T, m - o.cnt_above, v, lane);
    __syncthreads();
    const int f = v->sel_found, j = v->sel_j;
    const double cs = v->cs;
    __syncthreads();
    if (!f) return 0;
    const unsigned long long kk = list[j];
    out.found = 1;
    out.pos = o.cnt_above + j;
    out.id = key_id(kk);
    out.p = key_p(kk);
    out.cs = cs;
    out.tie = (j > 0 && key_p(list[j - 1]) == out.p) || (j + 1 < n && key_p(list[j + 1]) == out.p);
    return 1;
}

// Last candidate in canonical order (smallest p, then largest id), and
// whether its probability is shared; from global memory.
__device__ __forceinline__ Sel last_canon(Ctx &c, bool scale) {
    Vars *v = c.v;
    const float inv_sum = v->inv_sum;
    float pmin = PINF;
    for (int e = threadIdx.x; e < c.V; e += NT) {
        const float ev = e_global(c, e, scale);
        if (__float_as_int(ev) >= 0) pmin = fminf(pmin, __fmul_rn(ev, inv_sum));
    }
    float dummy = 0.f;
    block_maxmin_f(dummy, pmin, c.red);
    int idmax = -1, cnt = 0;
    for (int e = threadIdx.x; e < c.V; e += NT) {
        const float ev = e_global(c, e, scale);
        if (__float_as_int(ev) >= 0 && __fmul_rn(ev, inv_sum) == pmin) {
            idmax = max(idmax, e);
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

// j-th (0-based, id order) candidate whose p equals pv; from global memory.
__device__ __forceinline__ int ordered_pick(Ctx &c, bool scale, float pv, int j) {
    Vars *v = c.v;
    const float inv_sum = v->inv_sum;
    const int V = c.V;
    const int Q = (V + NT - 1) / NT;
    const int e0 = threadIdx.x * Q, e1 = min(V, e0 + Q);
    int cnt = 0;
    for (int e = e0; e < e1; ++e) {
        const float ev = e_global(c, e, scale);
        cnt += (__float_as_int(ev) >= 0) && (__fmul_rn(ev, inv_sum) == pv);
    }
    int tot;
    const int ex = block_xscan_i(cnt, tot, c.red);
    if (threadIdx.x == 0) v->own = -1;
    __syncthreads();
    if (j >= ex && j < ex + cnt) {
        int k = ex;
        for (int e = e0; e < e1; ++e) {
            const float ev = e_global(c, e, scale);
            if ((__float_as_int(ev) >= 0) && (__fmul_rn(ev, inv_sum) == pv)) {
                if (k == j) v->own = e;
                ++k;
            }
        }
    }
    __syncthreads();
    const int id = v->own;
    __syncthreads();
    return id;
}

// General select (rare path: the exact bucket windows could not decide):
// the probability window [plo0, phi0] first, then bisection of the
// probability interval, each step one exact pass over global memory.  Uses
// the upper part of the scratch area.
__device__ __noinline__ Sel select_slow(Ctx c, bool scale, int mode, double T, int m, float plo0,
                                        float phi0) {
    c.attach();
    Vars *v = c.v;
    unsigned long long *list = reinterpret_cast<unsigned long long *>(c.scr + SLOW_OFF);
    int *rank = reinterpret_cast<int *>(c.scr + SLOW_OFF + SLOW_CAP * 8);
    Sel out;
    out.found = 0; out.pos = v->n_cand - 1; out.id = -1; out.p = 0.f; out.cs = 0.0; out.tie = 0;
    unsigned lb = 0u, ub = 0x7f800000u;  // probability interval as bits
    for (int it = 0; it < 100; ++it) {
        float plo, phi;
        if (it == 0) {
            phi = phi0;
            plo = plo0;
        } else {
            phi = __uint_as_float(ub);
            plo = __uint_as_float(lb);
        }
        PassOut o = exact_pass_g(c, scale, plo, phi, list, SLOW_CAP);
        const int cl = classify(o, mode, T, m);
        if (cl == 2 && __float_as_uint(plo) == 0u) {
            // beyond the last candidate: total mass under the target
            out = last_canon(c, scale);
            out.found = 0;
            out.cs = o.above + o.in_mass;
            return out;
        }
        if (cl == 1) { lb = __float_as_uint(phi) + 1u; continue; }
        if (cl == 2) { ub = __float_as_uint(plo) - 1u; continue; }
        lb = __float_as_uint(plo);
        ub = __float_as_uint(phi);
        if (o.in_cnt <= SLOW_CAP) {
            sort_keys(list, o.in_cnt, rank, SLOW_CAP);
            if (resolve_list(c, list, o, mode, T, m, out)) return out;
        }
        if (lb == ub) {
            // more than SLOW_CAP candidates share one probability value: the
            // position inside the tie group is arithmetic, then the j-th id
            const float pv = __uint_as_float(lb);
            const int n = o.in_cnt;
            int j = 0;
            if (mode == T_POS) {
                j = m - o.cnt_above;
            } else {
                while (j < n - 1 && !((mode == T_MASS_GE) ? (o.above + (double)(j + 1) * pv >= T)
                                                           : (o.above + (double)(j + 1) * pv > T))) {
                    const double need = (T - o.above) / (double)pv;
                    const int jj = (int)need - 1;
                    j = (jj > j) ? jj : j + 1;
                    if (j > n - 1) j = n - 1;
                }
            }
            out.found = 1;
            out.pos = o.cnt_above + j;
            out.p = pv;
            out.cs = o.above + (double)(j + 1) * pv;
            out.tie = (n > 1);
            out.id = ordered_pick(c, scale, pv, j);
            return out;
        }
        // keep the half that holds the crossing
        const unsigned mid = lb + (ub - lb) / 2;
        const PassOut u = exact_pass_g(c, scale, __uint_as_float(mid + 1u), __uint_as_float(ub),
                                       list, SLOW_CAP);
        if (classify(u, mode, T, m) == 0) lb = mid + 1u;
        else ub = mid;
    }
    // did not converge: the error word says so, and on the allocation-free
    // path the row's id is -1 (write_result)
    if (threadIdx.x == 0) { atomicOr(c.err, 2); v->fail2 = 1; }
    __syncthreads();
    return out;
}

// Exact replay of the reference's top-256 heap (src/model.c:327-356) over the
// candidates in id order, by one warp, from global memory; then the walk over
// the replayed order (stable sort: ties in heap-array order) for the nucleus
// of n elements and the draw r held in vars.
__device__ __noinline__ void replay_top256(Ctx c, bool scale, int n) {
    c.attach();
    // runs after every walk: the window list area is free
    unsigned long long *outk = reinterpret_cast<unsigned long long *>(c.scr);
    float *hv = reinterpret_cast<float *>(c.scr + 256 * 8);
    int *hi = reinterpret_cast<int *>(c.scr + 256 * 8 + 256 * 4);
    int *rank = reinterpret_cast<int *>(c.scr + 256 * 8 + 512 * 4);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float inv_sum = c.v->inv_sum;
    const int V = c.V;
    // chunks of probabilities computed by every thread from global memory
    // (-1 for non-candidates), then fed to the heap by warp 0 in id order
    constexpr int CH = 2048;
    float *pch = reinterpret_cast<float *>(c.scr + 8192);  // 8 KB
    int filled = 0;
    for (int c0 = 0; c0 < V; c0 += CH) {
        for (int i = threadIdx.x; i < CH; i += NT) {
            const int id = c0 + i;
            float pv = -1.0f;
            if (id < V) {
                const float ev = e_global(c, id, scale);
                if (__float_as_int(ev) >= 0) pv = __fmul_rn(ev, inv_sum);
            }
            pch[i] = pv;
        }
        __syncthreads();
        if (warp == 0) {
            for (int base = 0; base < CH && c0 + base < V; base += 32) {
                const int id = c0 + base + lane;
                const float pv = pch[base + lane];
                const bool cand = pv >= 0.0f;
                const float p = cand ? pv : 0.0f;
                const unsigned mk = __ballot_sync(FULL, cand);
                bool rest = cand;
                if (filled < 256) {
                    const int rk = __popc(mk & ((1u << lane) - 1));
                    const int take = min(__popc(mk), 256 - filled);
                    if (cand && rk < take) { hv[filled + rk] = p; hi[filled + rk] = id; }
                    rest = cand && rk >= take;
                    filled += take;
                    __syncwarp();
                    if (filled < 256) continue;
                    if (take > 0) warp_heapify(hv, hi, 256, lane);
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
        }
        __syncthreads();
    }
    if (warp == 0) {
        __syncwarp();
        for (int q = lane; q < 256; q += 32) outk[q] = canon_key(hv[q], q);
    }
    __syncthreads();
    sort_keys(outk, 256, rank, 256);
    if (threadIdx.x == 0) {
        const float r = (float)c.v->aux1;
        double cs = 0.0;
        int pos = n - 1;
        for (int j = 0; j < n; ++j) {
            cs += (double)key_p(outk[j]);
            if ((double)r < cs) { pos = j; break; }
        }
        const int hp = key_id(outk[pos]);
        c.v->res_id = hi[hp];
        c.v->res_p = hv[hp];
    }
    __syncthreads();
}

// ---- full-vocabulary path: buckets over d = max - l ------------------------
// A candidate's bucket is key = round(d * inv_w), d = max - l, computed as
// kf = fma(d, inv_w, MAGIC) on the FMA pipe (kf - MAGIC = key, exactly).
// Non-candidates get d = 1e30: exp(-d) is then 0 and every bucket test fails.
// Bucket tests use saturating FMAs (FMA pipe), not compares/selects.
constexpr float DNC = 1e30f;  // d of non-candidates

// d = max - l for a pair of scaled logits; DNC for non-candidates (l < thr)
__device__ __forceinline__ float2 d_pair(float2 l, float mx, float thr) {
    const float2 d = __fadd2_rn(make_float2(mx, mx), make_float2(-l.x, -l.y));
    return make_float2(l.x >= thr ? d.x : DNC, l.y >= thr ? d.y : DNC);
}
// bucket key floats of a pair (clamped to the last bucket when CLAMP)
template <bool CLAMP>
__device__ __forceinline__ float2 kf_pair(float2 d, float2 iw2, float2 mg2, float dmax) {
    // non-candidates keep d = DNC (clamping them would file them in the last
    // bucket)
    if (CLAMP)
        d = make_float2(d.x == DNC ? DNC : fminf(d.x, dmax), d.y == DNC ? DNC : fminf(d.y, dmax));
    return __ffma2_rn(d, iw2, mg2);
}

// Pass 1 of the sorted path: per bucket the e-mass of its candidates, one
// 32-bit shared atomic per candidate (plus a count atomic when CNT: only rows
// whose top_k position is needed).  A member with d = b*w + t (|t| <= w/2;
// t = fma(-b, w, d), exact to one rounding) has e = exp(-d) = E_b * exp(-t),
// E_b = exp(-b*w).  The pass adds G = round(2^16 exp(-t)) (the quadratic
// Taylor polynomial: |t| < 0.01, error below 1.7e-7 relative, odd in t; G in
// [64880, 66200], so a bucket's sum stays below 2^32 for any V <= 64880), so
// that
//   mass_b = E_b * 2^-16 * sum_b
// is the members' e-sum to within 2^-17 = 7.6e-6 relative per member: below
// 7.6e-6 of the row's total mass in the worst case (equal logits round
// alike), ~1e-9 when the roundings are independent.
// CLEAN rows skip the candidate test (junk lanes have keys beyond the last
// bucket); CLAMP rows file every d > dmax at dmax (e < e^-40 there).  Returns
// this thread's candidate count (non-CLEAN rows).
template <bool SCALE, bool CLAMP, bool CLEAN, bool CNT>
__device__ __forceinline__ int hist_pass(Ctx &c, float inv_w, float w, float dmax) {
    Vars *v = c.v;
    const int nslots = v->nslots;
    const float mx = v->mx, thr = v->thr;
    const float4 *r4 = reinterpret_cast<const float4 *>(c.row);
    uint32_t *hsh = reinterpret_cast<uint32_t *>(c.scr) - MAGIC_I;
    const float2 it2 = make_float2(v->inv_temp, v->inv_temp);
    const float2 iw2 = make_float2(inv_w, inv_w), mg2 = make_float2(MAGIC, MAGIC);
    const float2 nmg2 = make_float2(-MAGIC, -MAGIC), nw2 = make_float2(-w, -w);
    const float2 mx2 = make_float2(mx, mx);
    // 2^16 exp(-t) ~ 2^16 - 2^16 t + 2^15 t^2, rounded to an integer by the
    // bias 2^23 (bits 0x4B000000 + G)
    const float2 c2 = make_float2(0x1p15f, 0x1p15f), c1 = make_float2(-0x1p16f, -0x1p16f);
    const float2 g0 = make_float2(0x1p23f + 0x1p16f, 0x1p23f + 0x1p16f);
    const int KT = MAGIC_I + NB - 1;
    int ncand = 0;
    auto dpair = [&](float2 l) -> float2 {
        if (SCALE) l = __fmul2_rn(l, it2);
        if (CLEAN) return __fadd2_rn(mx2, make_float2(-l.x, -l.y));
        float2 d = d_pair(l, mx, thr);
        if (CLAMP)
            d = make_float2(d.x == DNC ? DNC : fminf(d.x, dmax), d.y == DNC ? DNC : fminf(d.y, dmax));
        return d;
    };
    auto slot = [&](int s, bool check) {
        const float4 x = r4[s];
        const float2 da = dpair(make_float2(x.x, x.y)), db = dpair(make_float2(x.z, x.w));
        const float2 ka = __ffma2_rn(da, iw2, mg2), kb = __ffma2_rn(db, iw2, mg2);
        const float2 ta = __ffma2_rn(__fadd2_rn(ka, nmg2), nw2, da);
        const float2 tb = __ffma2_rn(__fadd2_rn(kb, nmg2), nw2, db);
        const float2 ga = __ffma2_rn(ta, __ffma2_rn(ta, c2, c1), g0);
        const float2 gb = __ffma2_rn(tb, __ffma2_rn(tb, c2, c1), g0);
        const int kk[4] = {__float_as_int(ka.x), __float_as_int(ka.y), __float_as_int(kb.x),
                           __float_as_int(kb.y)};
        const uint32_t gg[4] = {__float_as_uint(ga.x), __float_as_uint(ga.y), __float_as_uint(gb.x),
                                __float_as_uint(gb.y)};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (check && kk[q] > KT) continue;  // non-candidate or junk lane
            atomicAdd(&hsh[kk[q]], gg[q] & 0x7fffffu);
            if (CNT) atomicAdd(&hsh[kk[q] + NB], 1u);
            if (!CLEAN) ++ncand;
        }
    };
    if (CLEAN) {
        // interior slots hold candidates only; the ragged head / tail slots
        // (junk lanes: keys beyond the last bucket) take the key test
        const int s0 = v->s_int0, s1 = max(v->s_int1, s0), nh = s0, nt = nslots - s1;
        int s = s0 + threadIdx.x;
        for (; s + NT < s1; s += 2 * NT) {  // two slots in flight
            slot(s, false);
            slot(s + NT, false);
        }
        if (s < s1) slot(s, false);
        for (int i = threadIdx.x; i < nh + nt; i += NT) slot(i < nh ? i : s1 + (i - nh), true);
    } else {
        for (int s = threadIdx.x; s < nslots; s += NT) slot(s, true);
    }
    return ncand;
}

// Pass 2 of the sorted path: one flag per 16-byte slot holding an element of
// the union of the windows, each a range of d given as float bits
// [lo_t, lo_t + span_t] (d >= 0, so its bits order like its value), and
// (COUNT) per window the number of candidates above it (d below the range).
// Two slots per thread and trip, the flags of up to 16 trips in one 32-bit
// word per thread (the dead histogram); the gather re-tests the flagged
// slots' elements.  No branch or store per element.
template <bool SCALE, bool CLAMP, bool CLEAN, int NR, bool COUNT>
__device__ __forceinline__ void member_pass(Ctx &c, float dmax, const uint32_t *wlo,
                                            const uint32_t *wsp, int *above) {
    Vars *v = c.v;
    const int nslots = v->nslots;
    const float mx = v->mx, thr = v->thr;
    const float4 *r4 = reinterpret_cast<const float4 *>(c.row);
    const float2 it2 = make_float2(v->inv_temp, v->inv_temp);
    const float2 mx2 = make_float2(mx, mx);
    const int lane = threadIdx.x & 31;
    uint32_t lo[NR], sp[NR];
    int cnt[NR];
#pragma unroll
    for (int t = 0; t < NR; ++t) { lo[t] = wlo[t]; sp[t] = wsp[t]; cnt[t] = 0; }
    auto dpair = [&](float2 l) -> float2 {
        if (SCALE) l = __fmul2_rn(l, it2);
        if (CLEAN) return __fadd2_rn(mx2, make_float2(-l.x, -l.y));
        float2 d = d_pair(l, mx, thr);
        if (CLAMP)
            d = make_float2(d.x == DNC ? DNC : fminf(d.x, dmax), d.y == DNC ? DNC : fminf(d.y, dmax));
        return d;
    };
    auto slot_in = [&](float4 x) -> uint32_t {
        const float2 a = dpair(make_float2(x.x, x.y)), b = dpair(make_float2(x.z, x.w));
        const uint32_t k0 = __float_as_uint(a.x), k1 = __float_as_uint(a.y);
        const uint32_t k2 = __float_as_uint(b.x), k3 = __float_as_uint(b.y);
        bool in = false;
#pragma unroll
        for (int t = 0; t < NR; ++t) {
            const uint32_t u0 = k0 - lo[t], u1 = k1 - lo[t], u2 = k2 - lo[t], u3 = k3 - lo[t];
            in |= min(min(u0, u1), min(u2, u3)) <= sp[t];
            if (COUNT) cnt[t] += (int)((u0 >> 31) + (u1 >> 31) + (u2 >> 31) + (u3 >> 31));
        }
        return in ? 1u : 0u;
    };
    uint32_t *mw = reinterpret_cast<uint32_t *>(c.scr);
    uint32_t bits = 0;
    // out-of-range slots: d beyond every range, never counted
    const float ov_ = CLEAN ? JUNK : __int_as_float(0x7fc00000);
    const float4 OUT = make_float4(ov_, ov_, ov_, ov_);
    int iter = 0;
    // warp-uniform trip count: every lane of a warp takes the same trips
    const int wbase = (threadIdx.x & ~31);
    for (int base = wbase; base < nslots; base += 2 * NT, ++iter) {
        const int s0 = base + lane, s1 = base + NT + lane;
        const float4 x0 = (s0 < nslots) ? r4[s0] : OUT;
        const float4 x1 = (s1 < nslots) ? r4[s1] : OUT;
        bits |= (slot_in(x0) | (slot_in(x1) << 1)) << (2 * iter);
    }
    mw[threadIdx.x] = bits;
#pragma unroll
    for (int t = 0; t < NR; ++t) above[t] = COUNT ? cnt[t] : 0;
}

// Candidates with d below float bits `a` (d as the passes compute it), over
// global memory: the exact count of candidates above a window when the
// membership pass did not count (rare).
__device__ __noinline__ int count_below_g(Ctx c, bool scale, bool clamp, float dmax, uint32_t a) {
    c.attach();
    const float mx = c.v->mx, thr = c.v->thr;
    int n = 0;
    for (int e = threadIdx.x; e < c.V; e += NT) {
        const float l = logit_g(c, e, scale);
        if (!(l >= thr)) continue;
        float d = __fsub_rn(mx, l);
        if (clamp) d = fminf(d, dmax);
        n += __float_as_uint(d) < a;
    }
    return block_sum_i(n, c.red);
}

// exp pass of the id-order path: e stored in place (-0 for non-candidates),
// fp64 sum of fp32 groups of four.
template <bool SCALE>
__device__ __forceinline__ double exp_store_pass(Ctx &c) {
    Vars *v = c.v;
    const int nslots = v->nslots;
    const float mx = v->mx, thr = v->thr;
    float4 *r4 = reinterpret_cast<float4 *>(c.row);
    const float2 it2 = make_float2(v->inv_temp, v->inv_temp);
    double S = 0.0;
    for (int s = threadIdx.x; s < nslots; s += NT) {
        const float4 x = r4[s];
        float2 a = make_float2(x.x, x.y), b = make_float2(x.z, x.w);
        if (SCALE) { a = __fmul2_rn(a, it2); b = __fmul2_rn(b, it2); }
        const float2 xa = make_float2(a.x >= thr ? __fsub_rn(a.x, mx) : -DNC,
                                      a.y >= thr ? __fsub_rn(a.y, mx) : -DNC);
        const float2 xb = make_float2(b.x >= thr ? __fsub_rn(b.x, mx) : -DNC,
                                      b.y >= thr ? __fsub_rn(b.y, mx) : -DNC);
        float2 ea = exp_pair(xa), eb = exp_pair(xb);
        const float2 g = __fadd2_rn(ea, eb);
        S += (double)__fadd_rn(g.x, g.y);
        ea.x = a.x >= thr ? ea.x : -0.0f;
        ea.y = a.y >= thr ? ea.y : -0.0f;
        eb.x = b.x >= thr ? eb.x : -0.0f;
        eb.y = b.y >= thr ? eb.y : -0.0f;
        r4[s] = make_float4(ea.x, ea.y, eb.x, eb.y);
    }
    return block_sum_d(S, c.red);
}

// Window list entries after the membership pass, self-contained 64-bit keys:
//   bits 63..32  ~bits(p)        (probability descending)
//   bits 31..16  id              (then id ascending: the stable sort's order)
//   bits 11..0   per target t (0 cut, 1 top_k, 2 draw), bits 4t..4t+3:
//                in the target's d range / in its band above the target's
//                buckets / in its band below them / below the range's d
__device__ __forceinline__ unsigned long long list_key(float p, int id, uint32_t flags) {
    return ((unsigned long long)(~__float_as_uint(p)) << 32) | (((unsigned)id << 16) | flags);
}
__device__ __forceinline__ int lk_id(unsigned long long k) { return (int)((unsigned)k >> 16); }
struct __align__(16) Ent {
    unsigned long long k;
    double p;
};
__device__ __forceinline__ Ent make_ent(unsigned long long k) {
    Ent e;
    e.k = k;
    e.p = (double)key_p(k);
    return e;
}
// small lists live past the membership mask words (read into registers by the
// gather before any entry is written) and below the sort's rank area
constexpr int ENT_OFF = 8192;
static_assert(ENT_OFF + NT * 16 <= LISTCAP * 8, "entry area inside the list area");

// Exclusive block scan of three doubles m and three ints n, and block sums of
// three doubles a (in place; scratch `wd`: 6 * NW doubles, `wi`: 3 * NW ints).
__device__ __forceinline__ void block_xscan3a(double (&m)[3], int (&n)[3], double (&a)[3],
                                              double *wd, int *wi) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double im[3], sa[3];
    int in[3];
#pragma unroll
    for (int t = 0; t < 3; ++t) {
        im[t] = warp_iscan(m[t], lane);
        in[t] = warp_iscan(n[t], lane);
        sa[t] = warp_sum(a[t]);
    }
    if (lane == 31) {
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            wd[3 * warp + t] = im[t]; wi[3 * warp + t] = in[t]; wd[3 * NW + 3 * warp + t] = sa[t];
        }
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 3; ++t) {
        double bm = 0.0, ba = 0.0;
        int bn = 0;
        for (int w = 0; w < NW; ++w) {
            if (w < warp) { bm += wd[3 * w + t]; bn += wi[3 * w + t]; }
            ba += wd[3 * NW + 3 * w + t];
        }
        m[t] = bm + (im[t] - m[t]);
        n[t] = bn + (in[t] - n[t]);
        a[t] = ba;
    }
    __syncthreads();
}

// A target's crossing over the sorted window list, published by its owner.
struct Hit {
    double cs;
    float p;
    int id, pos, flags;  // flags: 1 found, 2 near an outer window edge, 4 tie
    int jmin;            // list index of the crossing (lowest claimant)
};
struct Cand {
    int j, pos;
    double cs;
};

// The first entry of this thread's run [j0, j1) of the sorted list that lies
// in target t's d range and where the running mass from m0 crosses T (GE /
// GT) or whose position from cnt0 equals m (POS); (pre_m, pre_n) is the
// range's exclusive prefix in front of the run.  j = INT_MAX when none.  Runs
// of two threads can both claim a crossing within fp64 rounding of T: the
// lowest list index wins (run_publish).
__device__ __forceinline__ Cand run_find(const unsigned long long *list, int j0, int j1, int t,
                                         double m0, int cnt0, double pre_m, int pre_n, int mode,
                                         double T, int m) {
    Cand r;
    r.j = INT_MAX;
    r.pos = 0;
    r.cs = 0.0;
    double cs = m0 + pre_m;
    int pos = cnt0 + pre_n;
    for (int j = j0; j < j1; ++j) {
        const unsigned long long k = list[j];
        if (!(((uint32_t)k >> (4 * t)) & 1u)) continue;
        const double prev = cs;
        cs += (double)key_p(k);
        const bool hit = (mode == T_MASS_GE) ? ((pos == 0 || prev < T) && cs >= T)
                         : (mode == T_MASS_GT) ? ((pos == 0 || prev <= T) && cs > T)
                                               : (pos == m);
        if (hit) { r.j = j; r.pos = pos; r.cs = cs; return r; }
        ++pos;
    }
    return r;
}

__device__ __forceinline__ void run_publish(const unsigned long long *list, int nl, const Cand &h,
                                            int t, Hit *out) {
    const unsigned long long k = list[h.j];
    const int j = h.j;
    const float p = key_p(k);
    const bool tie = (j > 0 && key_p(list[j - 1]) == p) || (j + 1 < nl && key_p(list[j + 1]) == p);
    // a crossing in the band outside the target's buckets: the estimate
    // missed; the exact fallback decides
    const bool outer = (((uint32_t)k >> (4 * t)) & 6u) != 0;
    out->cs = h.cs;
    out->p = p;
    out->id = lk_id(k);
    out->pos = h.pos;
    out->flags = 1 | (outer ? 2 : 0) | (tie ? 4 : 0);
}

// A published crossing as a selection; false when missing or at an outer edge.
__device__ __forceinline__ bool hit_sel(const Hit &h, Sel &out) {
    const int f = h.flags;
    if (!(f & 1)) return false;
    out.found = 1;
    out.cs = h.cs;
    out.p = h.p;
    out.id = h.id;
    out.pos = h.pos;
    out.tie = (f & 4) ? 1 : 0;
    return !(f & 2);
}


// Probability window [plo, phi] covering buckets [b0, b1] of width w (for
// the slow path's first exact pass).
__device__ __forceinline__ void pwin_of(int b0, int b1, float w, float inv_sum, float &plo,
                                        float &phi) {
    phi = (b0 <= 0) ? PINF : __fmul_rn(exp_one(-((float)b0 - 0.5f) * w), inv_sum);
    plo = __fmul_rn(exp_one(-((float)b1 + 0.5f) * w), inv_sum);
}

// A full-path row's candidates when they are at most 64 (listed into the
// scratch area), finished on one warp; returns their count when the warp
// decided the row (v->res_id, v->res_p, v->n_final), else 0.  Out of line:
// the rows of the bucket path run none of it.
template <bool SCALE>
__device__ __noinline__ int few_candidates(Ctx c, float tmax) {
    c.attach();
    Vars *v = c.v;
    unsigned long long *kl = reinterpret_cast<unsigned long long *>(c.scr + 4096);
    const int tot = list_candidates<SCALE>(c, tmax, kl);
    __syncthreads();  // the list writes (the buckets of the caller reuse the area)
    if (tot > 64) return 0;
    if (threadIdx.x < 32) {
        int rid = 0, rnf = 0, rn = 0;
        float rp = 0.0f;
        const bool ok = warp_tail(kl, tot, tot, v->top_p, v->u, false, v->mx, v->thr,
                                  (int)threadIdx.x, rid, rp, rnf, rn);
        if (threadIdx.x == 0) {
            v->wt = ok ? 1 : 0;
            v->res_id = rid;
            v->res_p = rp;
            v->n_final = rnf;
        }
    }
    __syncthreads();
    return v->wt ? tot : 0;
}

template <bool SCALE>
__device__ __forceinline__ void full_path(Ctx &c, float tmax) {
    Vars *v = c.v;
    const int sh = v->sh, nslots = v->nslots;
    const float mx = v->mx, thr = v->thr;
    float4 *r4 = reinterpret_cast<float4 *>(c.row);
    uint32_t *hc = reinterpret_cast<uint32_t *>(c.scr);
    unsigned long long *list = reinterpret_cast<unsigned long long *>(c.scr);
    const float top_p = v->top_p;
    const int top_k = v->top_k;

    if (mx == PINF) {
        // +inf logit: expf(inf - inf) is NaN, the reference's sums are NaN and
        // every walk falls through to the last candidate
        int last = -1, cnt = 0;
        for (int e = threadIdx.x; e < c.V; e += NT)
            if (logit_g(c, e, SCALE) >= thr) { last = max(last, e); ++cnt; }
        last = block_max_i(last, c.red);
        cnt = block_sum_i(cnt, c.red);
        release_row(c);
        const bool lazy = (top_p >= 1.0f) && (top_k <= 0 || top_k >= cnt);
        write_result(c, last, __int_as_float(0x7fc00000), lazy ? 5 : 7, cnt, cnt, 1);
        return;
    }
    // A real min_p threshold usually leaves few candidates: they are listed
    // as on the top_k path and, up to 64 of them, finish the row on one warp.
    // The reference's softmax over them and its stable sort by probability
    // (src/model.c:306-313, 359-360) list them in value order when no two
    // values or probabilities are equal; otherwise the warp leaves the row
    // undecided and the bucket path below takes it (the row is still
    // resident).  Rows where more than 64 threads hold a candidate skip it.
    if (!v->clean && v->min_p > 0.0f && top_p < 1.0f && __syncthreads_count(!(tmax < thr)) <= 64) {
        const int tot = few_candidates<SCALE>(c, tmax);
        if (tot > 0) {
            release_row(c);
            write_result(c, v->res_id, v->res_p, 7, tot, v->n_final, 1);  // src/model.c:359-360
            return;
        }
    }
    // bucket geometry over d = max - l
    float dmax = __fsub_rn(mx, v->xmin);
    if (v->min_p > 0.0f) dmax = fminf(dmax, __fsub_rn(mx, thr));
    const bool clamp = !(dmax <= DCAP);
    dmax = fminf(dmax, DCAP);
    if (!(dmax > 1e-30f)) dmax = 1.0f;
    const float inv_w = __fdiv_rn((float)NB - 1.5f, dmax);
    const float w = __fdiv_rn(1.0f, inv_w);
    const bool cntv = top_k > 0;  // bucket counts needed (the top_k position)
    for (int i = threadIdx.x; i < (cntv ? 2 : 1) * NB; i += NT) hc[i] = 0;
    if (threadIdx.x == 0) { v->ln0 = 0; v->lastb = -1; }
    __syncthreads();
    // CLEAN variants only without clamping (junk lanes must stay beyond the
    // last bucket)
    const bool clean = v->clean && !clamp;
    if (clean) {
        // junk lanes of the ragged head / tail slots: NaN -> JUNK
        // (the bulk-copied interior slots [s_int0, s_int1) hold no junk)
        const int s0 = v->s_int0, s1 = max(v->s_int1, s0), V = c.V;
        const int nh = s0, nt = nslots - s1;
        for (int i = threadIdx.x; i < nh + nt; i += NT) {
            const int s = (i < nh) ? i : s1 + (i - nh);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int e = 4 * s + q - sh;
                if (e < 0 || e >= V) c.row[4 * s + q] = JUNK;
            }
        }
        __syncthreads();
    }
    int my_nc;
    if (clamp) {
        my_nc = cntv ? hist_pass<SCALE, true, false, true>(c, inv_w, w, dmax)
                     : hist_pass<SCALE, true, false, false>(c, inv_w, w, dmax);
    } else if (clean) {
        my_nc = cntv ? hist_pass<SCALE, false, true, true>(c, inv_w, w, dmax)
                     : hist_pass<SCALE, false, true, false>(c, inv_w, w, dmax);
    } else {
        my_nc = cntv ? hist_pass<SCALE, false, false, true>(c, inv_w, w, dmax)
                     : hist_pass<SCALE, false, false, false>(c, inv_w, w, dmax);
    }
    __syncthreads();
    // bucket scan: e-masses (and counts when cntv)
    const int bb = BPT * threadIdx.x;
    int cb[BPT];
    double mb[BPT];
    int csum = 0;
    double msum = 0.0;
    {
        // E_b = exp(-b*w) of the first bucket (2^-16 scaled) and exp(-w), to
        // ~2e-7: 2^-x as 2^-n * ex2(-f) with x = n + f from an exact product
        auto e2neg = [](double x) -> double {
            const double n = floor(x);
            return ldexp((double)ex2_approx((float)(n - x)), -(int)n);
        };
        const double L2E = 1.4426950408889634;
        if (threadIdx.x == 0) v->h0b = hc[0];
        double E = e2neg((double)bb * (double)w * L2E) * 0x1p-16;
        const double qd = e2neg((double)w * L2E);
#pragma unroll
        for (int q = 0; q < BPT; ++q) {
            cb[q] = cntv ? (int)hc[NB + bb + q] : 0;
            mb[q] = E * (double)hc[bb + q];
            E *= qd;
            csum += cb[q];
            msum += mb[q];
        }
    }
    double mt;
    int ncand;
    double mex = msum;
    int cex = cntv ? csum : my_nc;
    // the window buckets start unset; the scan's barriers order this before
    // the bucket owners' writes below
    if (threadIdx.x == 0) { v->bc = NB; v->bc_hi = NB; v->bk = NB; v->bd0 = NB; v->bd_hi = NB; }
    block_xscan_di(mex, cex, mt, ncand, c.red);
    if (clean && !cntv) ncand = c.V;  // every logit finite and a candidate
    if (threadIdx.x == 0) v->n_cand = ncand;
    if (ncand == 0) {  // argmax guard (src/model.c:296-303)
        release_row(c);
        const int id = guard_argmax(c);
        write_result(c, id, 1.0f, 4, 0, 0, 0);
        return;
    }
    const bool lazy = (top_p >= 1.0f) && (top_k <= 0 || top_k >= ncand);
    if (lazy) {
        const double S = exp_store_pass<SCALE>(c);
        const float inv_sum = __fdiv_rn(1.0f, __double2float_rn(S));  // src/model.c:311
        // CDF walk in id order (src/model.c:319-320): contiguous segments
        const int Q = (nslots + NT - 1) / NT;
        const int s0 = threadIdx.x * Q, s1 = min(nslots, s0 + Q);
        const float2 is2 = make_float2(inv_sum, inv_sum);
        double seg = 0.0;
        int last = -1;
        for (int s = s0; s < s1; ++s) {
            const float4 x = r4[s];
            const float2 pa = __fmul2_rn(make_float2(x.x, x.y), is2);
            const float2 pb = __fmul2_rn(make_float2(x.z, x.w), is2);
            const float2 gg = __fadd2_rn(pa, pb);
            seg += (double)__fadd_rn(gg.x, gg.y);
            if (__float_as_int(x.w) >= 0) last = 4 * s + 3 - sh;
            else if (__float_as_int(x.z) >= 0) last = 4 * s + 2 - sh;
            else if (__float_as_int(x.y) >= 0) last = 4 * s + 1 - sh;
            else if (__float_as_int(x.x) >= 0) last = 4 * s - sh;
        }
        last = block_max_i(last, c.red);
        double total;
        const double pre = block_xscan_d(seg, total, c.red);
        const float r = __fmul_rn(v->u, __double2float_rn(total));
        const int cand_t = ((double)r < pre + seg && seg > 0.0) ? (int)threadIdx.x : INT_MAX;
        const int owner = block_min_i(cand_t, c.red);
        if (threadIdx.x == 0) { v->res_id = -1; v->res_p = 0.f; v->inv_sum = inv_sum; }
        __syncthreads();
        if ((int)threadIdx.x == owner) {
            // a rounding difference at a segment start can push the crossing
            // one segment further: rescan from here on
            double cdf = pre;
            int id = -1;
            float pp = 0.f;
            for (int s = s0; s < nslots && id < 0; ++s) {
                const float4 x = r4[s];
                const float ev[4] = {x.x, x.y, x.z, x.w};
                for (int q = 0; q < 4; ++q) {
                    if (__float_as_int(ev[q]) >= 0) {
                        const float p = __fmul_rn(ev[q], inv_sum);
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
        if (id < 0) {  // r at or beyond the last cdf: the last candidate (src/model.c:117)
            id = last;
            pp = __fmul_rn(c.row[last + sh], inv_sum);
        }
        release_row(c);
        write_result(c, id, pp, 5, ncand, ncand, 1);
        return;
    }

    // ---- sorted order: nucleus cut, top_k truncation, draw -----------------
    // Windows: the buckets each target can fall in, from the exact bucket
    // masses (normalised by the reference's inv_sum they are within 8e-6 of
    // the reference's cumulative sums of rounded probabilities, hence the EPS
    // margins) and counts (top_k).  Each window becomes a range of d with a
    // band of 1.2e-6 (+5e-7 relative) beyond its bucket edges: two candidates
    // with one probability lie within 5e-7 of each other in d, so every
    // candidate tied with one inside the buckets is inside the range.  The
    // walks run over each range's elements in exact (p desc, id asc) order
    // from the mass and count of the candidates below the range's d.
    const bool want_cut = top_p < 1.0f;
    const bool want_k = top_k > 0 && top_k < ncand;
    const double S = mt;
    const float inv_sum = __fdiv_rn(1.0f, __double2float_rn(S));  // src/model.c:311
    const double ip = (double)inv_sum;
    constexpr double EPS = 8e-6;
    int lastb = -1;  // last non-empty bucket
    {
        const double tlo = fmax((double)top_p - EPS, 0.0), thi = (double)top_p + EPS;
        double run = mex;
        int crun = cex;
#pragma unroll
        for (int q = 0; q < BPT; ++q) {
            const double nxt = run + mb[q];
            if (mb[q] > 0.0) {
                const int b = bb + q;
                const double pr = run * ip, pn = nxt * ip;
                lastb = b;
                if (want_cut && (pr < tlo || pr == 0.0) && pn >= tlo) { v->bc = b; v->mc = run; }
                if (want_cut && pr < thi && pn >= thi) { v->bc_hi = b; v->ec = pn; }
                if (want_k && top_k - 1 >= crun && top_k - 1 < crun + cb[q]) {
                    v->bk = b; v->mk = run; v->aux0 = pr; v->ek = pn;
                }
            }
            run = nxt;
            crun += cb[q];
        }
    }
    if (lastb >= 0) atomicMax(&v->lastb, lastb);
    __syncthreads();
    if (want_cut && !want_k && v->bc == 0 && v->bc_hi == 0 && v->h0b < 2u * 64880u &&
        v->amax != INT_MAX) {
        // bucket 0 holds one element (each adds at least 64880), the maximum
        // (e = 1, p = inv_sum), and its probability alone reaches top_p: the
        // nucleus is that element (n = 1; src/model.c:84-118, 327-356), the
        // draw r = u * p < p picks it (u = 1: the last element, the same)
        release_row(c);
        write_result(c, v->amax, inv_sum, (ncand > 256) ? 6 : 7, ncand, 1, 1);
        return;
    }
    // Every thread derives the draw range and then the window ranges itself
    // (no serial step between the barriers); thread 0 publishes the fixed-up
    // fields once every thread has read the old ones.
    const int lastb_all = v->lastb;
    const double mtot = S * ip;
    int bc_hi = v->bc_hi;
    double ec = v->ec;
    if (want_cut && v->bc < NB && bc_hi == NB) { bc_hi = lastb_all; ec = mtot; }
    {
        // range of new_sum (the cumulative mass where the walk stops), then of
        // r = u * (float)new_sum
        double lo = mtot, hi = mtot;
        if (want_cut && v->bc < NB) { lo = (double)top_p; hi = ec; }
        if (want_k && v->bk < NB) { lo = fmin(lo, v->aux0); hi = fmin(hi, v->ek); }
        const double rlo = fmax((double)v->u * lo * (1.0 - 1e-6) - EPS, 0.0);
        const double rhi = (double)v->u * hi * (1.0 + 1e-6) + EPS;
        double run = mex;
#pragma unroll
        for (int q = 0; q < BPT; ++q) {
            const double nxt = run + mb[q];
            if (mb[q] > 0.0) {
                const double pr = run * ip, pn = nxt * ip;
                if (pr <= rlo && pn > rlo) { v->bd0 = bb + q; v->md = run; }
                if (pr <= rhi && pn > rhi) v->bd_hi = bb + q;
            }
            run = nxt;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        v->inv_sum = inv_sum;
        v->S = S;
        v->adj[0] = v->adj[1] = v->adj[2] = 0.0;
        v->frk[0] = v->frk[1] = v->frk[2] = INT_MAX;
        v->bc_hi = bc_hi;
        v->ec = ec;
    }
    const int bc = want_cut ? v->bc : NB, bk = want_k ? v->bk : NB, bd = v->bd0;
    int bd_hi = v->bd_hi;
    if (bd < NB && bd_hi == NB) bd_hi = lastb_all;
    // d range of target t as float bits (inactive: empty)
    int tlo_b[3], thi_b[3];
    uint32_t ta[3], tsp[3];
    {
        const double rw = 1.0 / (double)inv_w;
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const int lo_b = (t == 0) ? bc : (t == 1) ? bk : bd;
            const int hi_b = (t == 0) ? bc_hi : (t == 1) ? lo_b : bd_hi;
            uint32_t a = 0xffffffffu, sp = 0u;
            if (lo_b < NB) {
                const double dl = ((double)lo_b - 0.5) * rw, dh = ((double)hi_b + 0.5) * rw;
                a = (lo_b == 0) ? 0u
                                : __float_as_uint(fmaxf(0.0f, __double2float_rd(dl * (1.0 - 5e-7) - 1.2e-6)));
                const uint32_t b = (hi_b >= NB - 1)
                                       ? __float_as_uint(DNC) - 1u
                                       : min(__float_as_uint(__double2float_ru(dh * (1.0 + 5e-7) + 1.2e-6)),
                                             __float_as_uint(DNC) - 1u);
                sp = b - a;
            }
            ta[t] = a;
            tsp[t] = sp;
            tlo_b[t] = lo_b;
            thi_b[t] = hi_b;
        }
    }
    // distinct ranges for the pass; rng[t] = the range of target t
    uint32_t wl[3] = {0u, 0u, 0u}, ws[3] = {0u, 0u, 0u};
    int rng[3] = {-1, -1, -1};
    int ntg = 0;
#pragma unroll
    for (int t = 0; t < 3; ++t) {
        if (tlo_b[t] >= NB) continue;
        int f = -1;
        if (ntg > 0 && wl[0] == ta[t] && ws[0] == tsp[t]) f = 0;
        else if (ntg > 1 && wl[1] == ta[t] && ws[1] == tsp[t]) f = 1;
        if (f < 0) {
            if (ntg == 0) { wl[0] = ta[t]; ws[0] = tsp[t]; }
            else if (ntg == 1) { wl[1] = ta[t]; ws[1] = tsp[t]; }
            else { wl[2] = ta[t]; ws[2] = tsp[t]; }
            f = ntg++;
        }
        rng[t] = f;
    }
    int abv[3] = {0, 0, 0};
    // counts of the candidates above each window: needed for positions (the
    // top_k target, stats) and for the cut's position unless its mass bound
    // already puts it at 256 or beyond (checked exactly after the gather)
    const bool cntp = cntv || (c.stats != nullptr) || (want_cut && bc > 0 && bc < NB && v->mc < 1024.0);
#define BM_MEMBER(CL, CN, N)                                                           \
    (cntp ? member_pass<SCALE, CL, CN, N, true>(c, dmax, wl, ws, abv)                  \
          : member_pass<SCALE, CL, CN, N, false>(c, dmax, wl, ws, abv))
    if (clamp) {
        if (ntg == 1) member_pass<SCALE, true, false, 1, true>(c, dmax, wl, ws, abv);
        else if (ntg == 2) member_pass<SCALE, true, false, 2, true>(c, dmax, wl, ws, abv);
        else if (ntg == 3) member_pass<SCALE, true, false, 3, true>(c, dmax, wl, ws, abv);
    } else if (clean) {
        if (ntg == 1) BM_MEMBER(false, true, 1);
        else if (ntg == 2) BM_MEMBER(false, true, 2);
        else if (ntg == 3) BM_MEMBER(false, true, 3);
    } else {
        if (ntg == 1) BM_MEMBER(false, false, 1);
        else if (ntg == 2) BM_MEMBER(false, false, 2);
        else if (ntg == 3) BM_MEMBER(false, false, 3);
    }
#undef BM_MEMBER
    const bool counted = cntp || clamp;
    // entries of lists of up to NT elements: the key and its probability as a
    // double, side by side (one 16-byte load per pair in the rank loop)
    Ent *ent = reinterpret_cast<Ent *>(c.scr + ENT_OFF);
    // exact probability and window flags of a listed element as its key
    auto to_key = [&](int id, float l) -> unsigned long long {
        const float pe = __fmul_rn(exp_one(__fsub_rn(l, mx)), inv_sum);
        float d = __fsub_rn(mx, l);
        if (clamp) d = fminf(d, dmax);
        const int kb = __float_as_int(__fmaf_rn(d, inv_w, MAGIC)) - MAGIC_I;
        const uint32_t db = __float_as_uint(d);
        uint32_t f = 0;
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            if (db - ta[t] <= tsp[t]) {
                f |= 1u << (4 * t);
                if (kb < tlo_b[t]) f |= 2u << (4 * t);
                if (kb > thi_b[t]) f |= 4u << (4 * t);
            } else if (tlo_b[t] < NB && db < ta[t]) {
                f |= 8u << (4 * t);
            }
        }
        return list_key(pe, id, f);
    };
    // gather the window elements of the flagged slots into keys: count them,
    // block scan of the counts, then every thread writes its own
    int tot;
    {
        const uint32_t *mw = reinterpret_cast<const uint32_t *>(c.scr);
        const int wbase = threadIdx.x & ~31, lane = threadIdx.x & 31;
        const uint32_t fl = (ntg > 0) ? mw[threadIdx.x] : 0u;
        const float it = v->inv_temp;
        // element q of slot `sl` in a window: its value (scaled) or NaN
        auto member = [&](int sl, int q) -> float {
            const int e = 4 * sl + q - sh;
            if (sl >= nslots || e < 0 || e >= c.V) return __int_as_float(0x7fc00000);
            const float l = SCALE ? __fmul_rn(c.row[4 * sl + q], it) : c.row[4 * sl + q];
            if (!(l >= thr)) return __int_as_float(0x7fc00000);
            float d = __fsub_rn(mx, l);
            if (clamp) d = fminf(d, dmax);
            const uint32_t db = __float_as_uint(d);
            bool in = false;
#pragma unroll
            for (int t = 0; t < 3; ++t) in |= (db - ta[t] <= tsp[t]);
            return in ? l : __int_as_float(0x7fc00000);
        };
        auto slot_of = [&](int bpos) { return wbase + (bpos >> 1) * 2 * NT + (bpos & 1) * NT + lane; };
        // member lanes of the first 8 flagged slots, 4 bits each (later
        // slots are re-tested in the write loop)
        uint32_t mm = 0;
        int nb = 0, k = 0;
        for (uint32_t m = fl; m; m &= m - 1, ++k) {
            const int sl = slot_of(__ffs(m) - 1);
            uint32_t m4 = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float l = member(sl, q);
                m4 |= (l == l) ? (1u << q) : 0u;
            }
            nb += __popc(m4);
            if (k < 8) mm |= m4 << (4 * k);
        }
        // the block scan of the member counts also sums the per-range counts
        // of candidates above the ranges
        int j = block_xscan_i4(nb, abv, tot, c.red);  // (its barriers end the flag reads)
        k = 0;
        for (uint32_t m = fl; m; m &= m - 1, ++k) {
            const int sl = slot_of(__ffs(m) - 1);
            uint32_t m4 = (mm >> (4 * k)) & 15u;
            if (k >= 8) {
                m4 = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float l = member(sl, q);
                    m4 |= (l == l) ? (1u << q) : 0u;
                }
            }
            for (; m4; m4 &= m4 - 1) {
                const int q = __ffs(m4) - 1;
                const float l = SCALE ? __fmul_rn(c.row[4 * sl + q], it) : c.row[4 * sl + q];
                const unsigned long long key = to_key(4 * sl + q - sh, l);
                if (tot <= NT) ent[j] = make_ent(key);
                else if (j < LISTCAP) list[j] = key;
                ++j;
            }
        }
    }
    // (every thread read v->bd_hi before the gather's barriers)
    if (threadIdx.x == 0) v->bd_hi = bd_hi;
    // release: the row buffer is no longer read on the common path (the list
    // holds the window elements, visible after its barrier; the rare
    // fallbacks read global memory)
    release_row(c);
    const bool list_ok = tot <= LISTCAP;
    const int nl = list_ok ? tot : 0;
    // Order statistics of the list.  Up to NT entries (the common case): no
    // sort; each entry's rank and per-target exclusive prefix (mass, count)
    // in canonical order are counted over the whole list by G threads per
    // entry (comparisons of self-contained keys), so every entry is a run of
    // one.  Longer lists: block sort, then runs of ceil(nl / NT) entries.
    Hit *hits = reinterpret_cast<Hit *>(c.scr + LISTCAP * 8 + 1024);
    if (threadIdx.x < 3) { hits[threadIdx.x].flags = 0; hits[threadIdx.x].jmin = INT_MAX; }
    const bool small = list_ok && nl <= NT;
    double pm[3] = {0.0, 0.0, 0.0}, pa[3] = {0.0, 0.0, 0.0};
    int pn[3] = {0, 0, 0};
    int j0 = 0, j1 = 0;
    unsigned long long ki = ~0ull;  // small lists: this thread's entry
    int rank = 0, own = 0;
    if (small) {
        // per pair: the rank and the mass of all entries in front.  A
        // target's range is contiguous in canonical order (no tie crosses its
        // band), so the prefix at an entry of the range is that mass minus
        // the mass in front of the range's first entry.
        const int lg = (nl <= NT / 4) ? 2 : (nl <= NT / 2) ? 1 : 0;  // G = 1 << lg
        const int i = (int)threadIdx.x >> lg, sub = (int)threadIdx.x & ((1 << lg) - 1);
        own = (sub == 0 && i < nl);
        ki = (i < nl) ? ent[i].k : ~0ull;
        const int per = (nl + (1 << lg) - 1) >> lg;
        const int jb = min(nl, sub * per), je = min(nl, jb + per);
        double pall = 0.0;
        for (int j = jb; j < je; ++j) {
            const Ent e = ent[j];
            const bool lt = e.k < ki;
            rank += lt;
            pall += lt ? e.p : 0.0;
        }
        for (int o = 1; o < (1 << lg); o <<= 1) {
            rank += __shfl_xor_sync(FULL, rank, o);
            pall += __shfl_xor_sync(FULL, pall, o);
        }
        const uint32_t fi = own ? (uint32_t)ki : 0u;
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            // lowest rank of the range: a warp minimum, one atomic a warp
            const int rmin = __reduce_min_sync(FULL, ((fi >> (4 * t)) & 1u) ? rank : INT_MAX);
            if ((threadIdx.x & 31) == 0 && rmin != INT_MAX) atomicMin(&v->frk[t], rmin);
            if ((fi >> (4 * t)) & 2u) atomicAdd(&v->adj[t], (double)key_p(ki));  // (rare)
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < 3; ++t)
            if (((fi >> (4 * t)) & 1u) && rank == v->frk[t]) v->lbm[t] = pall;
        __syncthreads();
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            pa[t] = v->adj[t];
            pm[t] = pall - v->lbm[t];
            pn[t] = rank - v->frk[t];
        }
    } else if (list_ok) {
        sort_keys(list, nl, reinterpret_cast<int *>(c.scr + LISTCAP * 8), LISTCAP);
        const int RQ = (nl + NT - 1) / NT;
        j0 = min(nl, (int)threadIdx.x * RQ);
        j1 = min(nl, j0 + RQ);
        for (int j = j0; j < j1; ++j) {
            const unsigned long long k = list[j];
            const uint32_t f = (uint32_t)k;
            const double p = (double)key_p(k);
#pragma unroll
            for (int t = 0; t < 3; ++t) {
                if ((f >> (4 * t)) & 1u) { pm[t] += p; ++pn[t]; }
                if ((f >> (4 * t)) & 2u) pa[t] += p;
            }
        }
        block_xscan3a(pm, pn, pa, reinterpret_cast<double *>(c.scr + LISTCAP * 8),
                      reinterpret_cast<int *>(c.scr + LISTCAP * 8 + 6 * NW * 8));
    }
    // mass and count of the candidates below each target's d range
    double m0[3];
    int c0[3];
    {
        const double mh[3] = {v->mc, v->mk, v->md};
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            m0[t] = mh[t] * ip - pa[t];
            c0[t] = (rng[t] == 0) ? abv[0] : (rng[t] == 1) ? abv[1] : (rng[t] == 2) ? abv[2] : 0;
            // uncounted: nothing lies below a range that starts at d = 0;
            // otherwise a large placeholder (the cut's bound is checked below)
            if (!counted) c0[t] = (tlo_b[t] == 0) ? 0 : (1 << 28);
        }
    }
    // the crossing of target t in this thread's run (small lists: its entry,
    // j = the entry's rank), and its publication by the lowest claimant
    // (the per-target values are passed by value: an array indexed by a
    // runtime target would leave registers for local memory)
    auto find = [&](int t, double m0t, int c0t, double pmt, int pnt, int mode, double T,
                    int m) -> Cand {
        if (!small) return run_find(list, j0, j1, t, m0t, c0t, pmt, pnt, mode, T, m);
        Cand r = {INT_MAX, 0, 0.0};
        if (own && (((uint32_t)ki >> (4 * t)) & 1u)) {
            const double prev = m0t + pmt;
            const double cs = prev + (double)key_p(ki);
            const int pos = c0t + pnt;
            const bool hit = (mode == T_MASS_GE) ? ((pos == 0 || prev < T) && cs >= T)
                             : (mode == T_MASS_GT) ? ((pos == 0 || prev <= T) && cs > T)
                                                   : (pos == m);
            if (hit) { r.j = rank; r.pos = pos; r.cs = cs; }
        }
        return r;
    };
    auto publish = [&](const Cand &h, int t) {
        if (!small) { run_publish(list, nl, h, t, &hits[t]); return; }
        Hit *o = &hits[t];
        o->cs = h.cs;
        o->p = key_p(ki);
        o->id = lk_id(ki);
        o->pos = h.pos;
        const bool outer = (((uint32_t)ki >> (4 * t)) & 6u) != 0;
        o->flags = 1 | (outer ? 2 : 0);
    };
    // small lists: a published crossing's tie flag (another entry with the
    // same probability), one comparison per entry; only the top-256 heap
    // path (a nucleus of fewer than 256) reads it
    auto mark_ties = [&](int t_a, int t_b, bool need) {
        if (!small || !need) return;
        if (own) {
            const float pi = key_p(ki);
            const int id = lk_id(ki);
            if ((hits[t_a].flags & 1) && hits[t_a].p == pi && hits[t_a].id != id) atomicOr(&hits[t_a].flags, 4);
            if ((hits[t_b].flags & 1) && hits[t_b].p == pi && hits[t_b].id != id) atomicOr(&hits[t_b].flags, 4);
        }
        __syncthreads();
    };

    if (!counted && want_cut && bc > 0 && bc < NB && !(v->mc - pa[0] * S * 1.001 >= 256.5)) {
        // the placeholder stands for at least 256 candidates above the cut's
        // range only while their e-mass (each e <= 1) reaches 256: count
        c0[0] = count_below_g(c, SCALE, clamp, dmax, ta[0]);
    }
    // nucleus cut and top_k position: the owners of the crossings publish them
    const bool try_c = want_cut && list_ok && bc < NB && !(m0[0] >= (double)top_p && c0[0] > 0);
    const bool try_k = want_k && list_ok && bk < NB && !(top_k - 1 < c0[1]);
    Cand hc_ = {INT_MAX, 0, 0.0}, hk_ = {INT_MAX, 0, 0.0};
    if (try_c)
        hc_ = find(0, m0[0], c0[0], pm[0], pn[0], T_MASS_GE, (double)top_p, 0);
    if (try_k)
        hk_ = find(1, m0[1], c0[1], pm[1], pn[1], T_POS, 0.0, top_k - 1);
    if (hc_.j != INT_MAX) atomicMin(&hits[0].jmin, hc_.j);
    if (hk_.j != INT_MAX) atomicMin(&hits[1].jmin, hk_.j);
    __syncthreads();
    if (hc_.j != INT_MAX && hc_.j == hits[0].jmin) publish(hc_, 0);
    if (hk_.j != INT_MAX && hk_.j == hits[1].jmin) publish(hk_, 1);
    __syncthreads();
    mark_ties(0, 1, (hits[0].flags & 1) && hits[0].pos < 256 && ncand > 256);

    int n = ncand;
    double new_sum = S * ip;  // total probability mass (fallback when no cut)
    Sel tail;
    tail.found = 0; tail.id = -1; tail.p = 0.f; tail.tie = 0; tail.pos = ncand - 1; tail.cs = 0.0;
    bool partial = false;
    float pw_lo = 0.0f, pw_hi = PINF;
    if (want_cut) {
        Sel cut;
        if (!(try_c && hit_sel(hits[0], cut))) {
            if (bc < NB) pwin_of(bc - 4, v->bc_hi + 4, w, inv_sum, pw_lo, pw_hi);
            cut = select_slow(c, SCALE, T_MASS_GE, (double)top_p, 0, pw_lo, pw_hi);
        }
        if (cut.found) {
            n = cut.pos + 1;
            partial = (ncand > 256) && (cut.pos < 256);  // src/model.c:327-356
        }
        new_sum = cut.cs;
        tail = cut;
    }
    if (want_k && top_k < n) {  // src/model.c:102-103
        Sel tk;
        if (!(try_k && hit_sel(hits[1], tk))) {
            pw_lo = 0.0f; pw_hi = PINF;
            if (bk < NB) pwin_of(bk - 4, bk + 4, w, inv_sum, pw_lo, pw_hi);
            tk = select_slow(c, SCALE, T_POS, 0.0, top_k - 1, pw_lo, pw_hi);
        }
        n = top_k;
        new_sum = tk.cs;
        tail = tk;
    }
    const float r = __fmul_rn(v->u, __double2float_rn(new_sum));
    Sel d;
    {
        const bool try_d = list_ok && bd < NB && !(m0[2] > (double)r && c0[2] > 0);
        Cand hd_ = {INT_MAX, 0, 0.0};
        if (try_d)
            hd_ = find(2, m0[2], c0[2], pm[2], pn[2], T_MASS_GT, (double)r, 0);
        if (hd_.j != INT_MAX) atomicMin(&hits[2].jmin, hd_.j);
        __syncthreads();
        if (hd_.j != INT_MAX && hd_.j == hits[2].jmin) publish(hd_, 2);
        __syncthreads();
        mark_ties(2, 2, partial);
        if (!(try_d && hit_sel(hits[2], d))) {
            pw_lo = 0.0f; pw_hi = PINF;
            if (bd < NB) pwin_of(bd - 4, v->bd_hi + 4, w, inv_sum, pw_lo, pw_hi);
            d = select_slow(c, SCALE, T_MASS_GT, (double)r, 0, pw_lo, pw_hi);
        }
    }
    int id;
    float pp;
    // the draw's crossing lies in the nucleus when it is at or before the
    // nucleus' last element in canonical order (p desc, id asc)
    const bool in_nucleus = !tail.found || d.p > tail.p || (d.p == tail.p && d.id <= tail.id);
    if (d.found && in_nucleus) { id = d.id; pp = d.p; }
    else { id = tail.id; pp = tail.p; d.tie = tail.tie; }
    if (partial && d.tie) {
        // the reference's heap layout decides the order among equal
        // probabilities: replay it exactly
        if (threadIdx.x == 0) v->aux1 = (double)r;
        __syncthreads();
        replay_top256(c, SCALE, n);
        id = v->res_id;
        pp = v->res_p;
    }
    write_result(c, id, pp, partial ? 6 : 7, ncand, n, 1);
}

__global__ void __launch_bounds__(NT, 1) sample_kernel(const Params P) {
    const Layout L = layout(P.V);
    Ctx c;
    // the launch's rows: B, or a count an earlier kernel wrote
    const int B = P.dB ? min(*P.dB, P.B) : P.B;
    // launch row r is row orow(r) of the per-row arrays
    auto orow = [&](int r) { return P.row_map ? (int)P.row_map[r] : r; };
    c.logits = P.logits;
    c.ld = P.ld;
    c.B = B;
    c.V = P.V;
    c.err = P.err;
    c.sched = P.sched;
    c.out_id = P.out_id;
    c.out_prob = P.out_prob;
    c.stats = P.stats;
    c.mark = P.mark_failed_rows;
    c.summary = 0;
    c.row_map = P.row_map;
    c.attach();
    Vars *v = c.v;
    const int V = P.V;
    const int tid = threadIdx.x;

    if (tid == 0) {
        v->p_knobs = P.knobs;
        v->p_uniform = P.uniform;
        v->p_hist_off = P.hist_off;
        v->p_knob_stride = P.knob_stride;
        for (int i = 0; i < NCHUNK; ++i) mbar_init(&c.mbar[i], 1);
        fence_mbar_init();
        v->fail = 0;
        if ((int)blockIdx.x < B)
            issue_row(P.logits + (int64_t)orow(blockIdx.x) * P.ld, V, c.mbar, c.row);
        const int pre = (int)(blockIdx.x + gridDim.x);
        if (pre < B) prefetch_row(P.logits + (int64_t)orow(pre) * P.ld, V);
    }
    __syncthreads();

    uint32_t it = 0;
    for (int lrow = blockIdx.x; lrow < B; ++it) {
        const int row = orow(lrow);
        c.rowid = row;
        c.parity = it & 1u;
        c.g = P.logits + (int64_t)row * P.ld;
        if (tid == 0) {
            // dynamic schedule: the first gridDim.x rows go one per CTA, every
            // later row to the CTA that asks first (rows of unequal cost would
            // otherwise leave SMs idle at the end of the launch).  The row to
            // follow this one was claimed at the last release (the first row:
            // claimed now); its copy is issued at this row's release
            c.claim = (it == 0) ? (int)gridDim.x + atomicAdd(&P.sched[0], 1) : v->nclaim;
            const int sh = (int)(((uintptr_t)c.g & 15u) >> 2);
            int i0 = sh ? 4 - sh : 0;
            if (i0 > V) i0 = V;
            int n4 = ((V - i0) >> 2) << 2;
            if (n4 < 4 * NCHUNK * 4) n4 = 0;
            v->sh = sh;
            v->nslots = (V + sh + 3) >> 2;
            v->s_int0 = (i0 + sh) >> 2;
            v->s_int1 = v->s_int0 + (n4 >> 2);
            v->released = 0;
            v->fail2 = 0;
            v->amax = INT_MAX;
            // (rows after a CTA's first: the values staged at the release)
            const bool st = it > 0;
            const bm_knobs_t kn = st ? v->nk : P.knobs[(int64_t)row * P.knob_stride];
            v->temp = kn.temp;
            v->penalty = kn.penalty;
            v->min_p = kn.min_p;
            v->top_p = kn.top_p;
            v->top_k = kn.top_k;
            v->inv_temp = kn.inv_temp;
            v->log_min_p = kn.log_min_p;
            v->u = P.uniform ? (st ? v->nu : P.uniform[row]) : 0.0f;
            v->greedy = (kn.temp < 0.05f);  // src/model.c:144
            int h0 = 0, h1 = 0;
            if (P.hist && P.hist_off) {
                h0 = (int)(st ? v->nh[0] : P.hist_off[row]);
                h1 = (int)(st ? v->nh[1] : P.hist_off[row + 1]);
            }
            v->pen = (h1 > h0) && (kn.penalty > 0.0f) && (kn.penalty != 1.0f);
            v->h0 = h0;
            v->h1 = h1;
        }
        __syncthreads();
        const int sh = v->sh;
        // penalty bitset over this row's distinct, in-range, unprotected ids:
        // cleared here, set by the load pass once the row has landed
        if (v->pen) {
            for (int i = tid; i < L.nbw; i += NT) c.bits[i] = 0u;
            __syncthreads();
        }
        const bool greedy = v->greedy != 0, pen = v->pen != 0;
        const bool scale = v->inv_temp != 1.0f;
        float mx, xmin, chk, gv;
        int gi;
        if (greedy) {
            if (pen) load_pass<true, true, false>(c, P.hist, mx, xmin, chk, gv, gi);
            else load_pass<true, false, false>(c, P.hist, mx, xmin, chk, gv, gi);
        } else if (pen) {
            if (scale) load_pass<false, true, true>(c, P.hist, mx, xmin, chk, gv, gi);
            else load_pass<false, true, false>(c, P.hist, mx, xmin, chk, gv, gi);
        } else {
            if (scale) load_pass<false, false, true>(c, P.hist, mx, xmin, chk, gv, gi);
            else load_pass<false, false, false>(c, P.hist, mx, xmin, chk, gv, gi);
        }
        // the block reductions (their barriers also make a failed wait's flag
        // visible to every thread)
        const float lmx = mx;
        if (greedy) block_argmax(gv, gi, c.red);
        else block_maxmin_chk(mx, xmin, chk, c.red);
        if (v->fail) {
            // a bounded wait expired: wait (bounded) for this row's copies,
            // then stop; the host sees the error flag
            if (tid == 0) {
                for (int ch = 0; ch < NCHUNK; ++ch) (void)mbar_wait(&c.mbar[ch], c.parity);
                if (P.mark_failed_rows) {
                    // this row and the one claimed for after it stay unsampled
                    P.out_id[row] = -1;
                    if (c.claim < B) P.out_id[orow(c.claim)] = -1;
                }
            }
            __syncthreads();
            break;
        }
        if (greedy) {
            release_row(c);
            write_result(c, gi == INT_MAX ? 0 : gi, 1.0f, 1, 0, 0, 0);
        } else {
            if (lmx == mx && gi != INT_MAX) {
                // this thread saw the maximum in slot gi: its index
                const float4 x = reinterpret_cast<const float4 *>(c.row)[gi];
                const float xv[4] = {x.x, x.y, x.z, x.w};
                int idx = INT_MAX;
#pragma unroll
                for (int q = 3; q >= 0; --q) {
                    const int e = 4 * gi + q - sh;
                    const float l = scale ? __fmul_rn(xv[q], v->inv_temp) : xv[q];
                    if (e >= 0 && e < V && l == mx) idx = e;
                }
                if (idx != INT_MAX) atomicMin(&v->amax, idx);
            }
            {
                // every thread derives the row's values and writes them (the
                // same values) before it reads them: no barrier needed here
                // src/model.c:169-173 (logf from the host)
                float thr = -1e30f;
                if (v->min_p >= 1.0f) thr = mx;
                else if (v->min_p > 0.0f) thr = __fadd_rn(mx, v->log_min_p);
                // every logit finite and a candidate: the streaming passes
                // need no candidate test
                const int clean = (chk == 0.0f) && (xmin >= thr) && (fabsf(mx) < 1e30f) &&
                                  (v->inv_temp >= 1e-6f);
                const int kk = (v->top_k > 0 && v->top_k <= 256) ? v->top_k : 0;  // src/model.c:175
                v->mx = mx;
                v->xmin = xmin;
                v->thr = thr;
                v->clean = clean;
                v->k = kk;
            }
            if (v->k > 0) {
                if (scale) topk_path<true>(c, lmx);
                else topk_path<false>(c, lmx);
            } else {
                if (scale) full_path<true>(c, lmx);
                else full_path<false>(c, lmx);
            }
        }
        __syncthreads();
        if (!v->released) release_row(c);
        if ((tid >> 5) == 1) {
            // the next row's staged values have landed; its history ids into
            // L2 (up to 256 lines), so the load pass finds them there
            cp_async_wait_all();
            if (tid == 33) v->nclaim = c.succ;
            __syncwarp();
            const int nxt = v->next_row;
            if (P.hist && P.hist_off && nxt < B) {
                const int64_t a = v->nh[0], b = v->nh[1];
                const int64_t lines = min((b - a + 31) / 32, (int64_t)256);
                for (int64_t q = tid & 31; q < lines; q += 32) prefetch_l2_line(P.hist + a + 32 * q);
            }
        }
        __syncthreads();
        lrow = v->next_row;
    }
    // the last release of this CTA claimed a row >= B and issued nothing, so
    // no copy is in flight when the kernel ends.  The last CTA to finish
    // rewinds the schedule for the next launch (and, on the allocation-free
    // path, clears the error word: failed rows carry id -1 instead).
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&P.sched[1], 1) == (int)gridDim.x - 1) {
            P.sched[0] = 0;
            P.sched[1] = 0;
            if (P.mark_failed_rows) P.err[0] = 0;
            __threadfence();
        }
    }
}

// ------------------------------------------------------------ merge --
// The fused lm_head + sampler's second kernel: one CTA per row at a time.
// The row's lists (the GEMM's summary epilogue: per 128 columns the KS
// largest penalised, scaled logits, unordered) are staged in the row
// buffer's place.  Every column's maximum is in its list, and a list that is
// not full holds every value of its columns.
//   greedy rows: the argmax over the lists (the lowest id among equal
//     maxima), strict '>' from -1e9 (src/model.c:144-154);
//   top_k rows (1 <= top_k <= 256): the maximum, the min_p threshold
//     (src/model.c:165-173), every listed value at or above it, and the top_k
//     path on that list, which checks that no full list's omitted values (at
//     most its smallest entry) can reach the cut's buckets or the extraction
//     set (else the row goes to the fallback lists);
//   other rows (their logits were stored by the GEMM): the fallback list.
__global__ void __launch_bounds__(NT, MERGE_CTAS_PER_SM) summary_kernel(const SumParams P) {
    Ctx c;
    c.logits = nullptr;
    c.ld = 0;
    c.B = P.B;
    c.V = P.V;
    c.err = P.err;
    c.sched = nullptr;
    c.out_id = P.out_id;
    c.out_prob = P.out_prob;
    c.stats = P.stats;
    c.mark = 0;
    c.summary = 1;
    c.row_map = nullptr;
    c.g = nullptr;
    c.claim = 0;
    c.parity = 0;
    c.attach();
    Vars *v = c.v;
    const int tid = threadIdx.x;
    const int ks = P.ks, ne = P.tiles * P.ks;
    unsigned long long *se = reinterpret_cast<unsigned long long *>(c.row);
    unsigned long long *kc = reinterpret_cast<unsigned long long *>(c.scr + 4096);
    constexpr unsigned NONE = 0xffffffffu;  // unused list slot
    for (int row = blockIdx.x; row < P.B; row += gridDim.x) {
        c.rowid = row;
        if (tid == 0) {
            const bm_knobs_t kn = P.knobs[(int64_t)row * P.knob_stride];
            v->temp = kn.temp;
            v->penalty = kn.penalty;
            v->min_p = kn.min_p;
            v->top_p = kn.top_p;
            v->top_k = kn.top_k;
            v->inv_temp = kn.inv_temp;
            v->log_min_p = kn.log_min_p;
            v->u = P.uniform ? P.uniform[row] : 0.0f;
            v->greedy = (kn.temp < 0.05f);                                   // src/model.c:144
            v->k = (kn.top_k > 0 && kn.top_k <= 256) ? kn.top_k : 0;        // src/model.c:175
            v->pen = 0;
            v->fb = 0;
            v->fail2 = 0;
            v->kcnt = 0;
            v->released = 1;
            v->sh = 0;
            v->nslots = 0;
        }
        // the row's lists, 16-byte loads (ne is even: ks is)
        const uint4 *src = reinterpret_cast<const uint4 *>(P.summ + (int64_t)row * ne);
        for (int i = tid; i < ne / 2; i += NT) reinterpret_cast<uint4 *>(se)[i] = src[i];
        __syncthreads();
        if (v->greedy) {
            float gv = -1e9f;
            int gi = INT_MAX;
            for (int i = tid; i < ne; i += NT) {
                const unsigned long long e = se[i];
                const unsigned id = (unsigned)e;
                const float x = __uint_as_float((unsigned)(e >> 32));
                if (id != NONE && (x > gv || (x == gv && gi != INT_MAX && (int)id < gi))) {
                    gv = x;
                    gi = (int)id;
                }
            }
            block_argmax(gv, gi, c.red);
            write_result(c, gi == INT_MAX ? 0 : gi, 1.0f, 1, 0, 0, 0);
            __syncthreads();
            continue;
        }
        if (v->k > 0) {
            // the maximum, and the largest value a full list may have left
            // out (at most its smallest entry)
            float mx = -1e30f, nvk = PINF;
            for (int t = tid; t < P.tiles; t += NT) {
                float lmax = -PINF, lmin = PINF;
                int cnt = 0;
                for (int k = 0; k < ks; ++k) {
                    const unsigned long long e = se[(int64_t)t * ks + k];
                    if ((unsigned)e == NONE) continue;
                    const float x = __uint_as_float((unsigned)(e >> 32));
                    lmax = fmaxf(lmax, x);
                    lmin = fminf(lmin, x);
                    ++cnt;
                }
                mx = fmaxf(mx, lmax);
                if (cnt == ks) nvk = fminf(nvk, -lmin);
            }
            block_maxmin_f(mx, nvk, c.red);
            if (tid == 0) {
                v->mx = mx;
                // src/model.c:169-173 (logf from the host)
                float thr = -1e30f;
                if (v->min_p >= 1.0f) thr = mx;
                else if (v->min_p > 0.0f) thr = __fadd_rn(mx, v->log_min_p);
                v->thr = thr;
                v->sumvk = -nvk;
            }
            // the listed candidates (l >= thr, src/model.c:185).  More entries
            // than the candidate list holds: only those in the reference's
            // 128 buckets up to one past the first bucket where their count
            // reaches top_k (it lies at or past the row's own cut: the lists
            // hold a subset of the row, so every candidate the cut or the
            // extraction can need lies there)
            uint32_t *hb = reinterpret_cast<uint32_t *>(c.scr);
            const float bscale = __fdiv_rn(127.0f, 20.0f);  // src/model.c:184
            const bool all_fit = ne <= KCAP;
            if (!all_fit)
                for (int q = tid; q < HB; q += NT) hb[q] = 0u;
            __syncthreads();
            const float thr = v->thr, mxr = v->mx;
            auto bucket_of = [&](float l) {
                const int b = x86_cvtt(__fmul_rn(__fsub_rn(mxr, l), bscale));
                return min(max(b, 0), HB - 1);
            };
            int lim = HB - 1;
            if (!all_fit) {
                for (int i = tid; i < ne; i += NT) {
                    const unsigned long long e = se[i];
                    if ((unsigned)e == NONE) continue;
                    const float x = __uint_as_float((unsigned)(e >> 32));
                    if (x >= thr) {
                        const int b = bucket_of(x);
                        if (b < HB - 1) atomicAdd(&hb[b], 1u);
                    }
                }
                __syncthreads();
                if (tid < 32) {
                    uint32_t cq[4], ls = 0;
#pragma unroll
                    for (int q = 0; q < 4; ++q) { cq[q] = hb[4 * tid + q]; ls += cq[q]; }
                    const uint32_t inc = warp_iscan(ls, tid);
                    uint32_t run = inc - ls;
                    int hit = INT_MAX;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        run += cq[q];
                        if (hit == INT_MAX && run >= (uint32_t)v->k) hit = 4 * tid + q;
                    }
                    hit = warp_imin(hit);
                    if (tid == 0) v->kcut = (hit == INT_MAX) ? HB - 1 : hit;
                }
                __syncthreads();
                lim = min(v->kcut + 1, HB - 1);
            }
            // the kept entries, one shared atomic a warp
            const int lane = tid & 31;
            for (int base = 0; base < ne; base += NT) {
                const int i = base + tid;
                bool keep = false;
                unsigned long long ent = 0ull;
                if (i < ne) {
                    const unsigned long long e = se[i];
                    if ((unsigned)e != NONE) {
                        const float x = __uint_as_float((unsigned)(e >> 32));
                        keep = x >= thr && bucket_of(x) <= lim;
                        ent = ((unsigned long long)(unsigned)e << 32) | (e >> 32);
                    }
                }
                const unsigned m = __ballot_sync(FULL, keep);
                int pos0 = 0;
                if (lane == 0 && m) pos0 = atomicAdd(&v->kcnt, __popc(m));
                pos0 = __shfl_sync(FULL, pos0, 0);
                if (keep) {
                    const int pos = pos0 + __popc(m & ((1u << lane) - 1u));
                    if (pos < KCAP) kc[pos] = ent;
                }
            }
            __syncthreads();
            topk_path<false>(c, PINF);  // (the lists: no candidate scan)
        } else if (tid == 0) {
            v->fb = 1;
        }
        __syncthreads();
        if (tid == 0 && v->fb) {
            // left for the full sampler: with its logits (stored by the GEMM)
            // or after a GEMM of its own (a top_k row the lists cannot decide)
            P.fb[1 + atomicAdd(&P.fb[0], 1)] = row;
            if (v->k > 0) P.nl[1 + atomicAdd(&P.nl[0], 1)] = row;
        }
        __syncthreads();
    }
}

// Scratch of the allocation-free entry point (one copy per device).
static __device__ __align__(256) int g_noalloc_scratch[NOALLOC_WORDS];

}  // namespace

size_t smem_bytes(int V) { return layout(V).total; }

cudaError_t noalloc_scratch(int **out) {
    return cudaGetSymbolAddress(reinterpret_cast<void **>(out), g_noalloc_scratch);
}

int max_vocab(size_t limit) {
    int lo = 1, hi = 1 << 20;
    if (smem_bytes(1) > limit) return 0;
    while (lo < hi) {
        const int mid = lo + (hi - lo + 1) / 2;
        if (smem_bytes(mid) <= limit) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

cudaError_t prepare(int V) {
    return cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem_bytes(V));
}

static size_t summary_smem(int V, int tiles, int ks) {
    return layout(V).row + (size_t)tiles * ks * 8;
}

cudaError_t prepare_summary(int V, int tiles, int ks) {
    cudaError_t e = cudaFuncSetAttribute(summary_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)summary_smem(V, tiles, ks));
    if (e != cudaSuccess) return e;
    // MERGE_CTAS_PER_SM CTAs' shared memory per SM
    return cudaFuncSetAttribute(summary_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                (int)cudaSharedmemCarveoutMaxShared);
}

cudaError_t launch_summary(const SumParams &p, int grid, cudaStream_t s) {
    if (p.ks % 2 || p.tiles <= 0) return cudaErrorInvalidValue;
    summary_kernel<<<grid, NT, summary_smem(p.V, p.tiles, p.ks), s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch(const Params &p, int grid, cudaStream_t s) {
    sample_kernel<<<grid, NT, smem_bytes(p.V), s>>>(p);
    return cudaGetLastError();
}

}  // namespace bmk
