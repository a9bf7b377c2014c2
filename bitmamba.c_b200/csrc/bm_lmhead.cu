// Final RMSNorm + bf16 lm_head GEMM on the sm_100a tensor cores, the producer
// of the sampler's logits (the optional fused variant of the sampling path).
//
//   rmsnorm   a[r, :] = bf16(x[r, :] * rms_r * w), the normalisation of
//             jserv/bitmamba.c src/kernel.c:72-91 (scalar_rms_norm: four
//             strided fp32 accumulators, 1 / sqrtf(sum / size + 1e-6f)),
//             bit for bit, then rounded to bf16 for the tensor cores.
//   gemm      logits[r, n] = sum_k a[r, k] * W[n, k] in 128 x 256 output
//             tiles on persistent CTAs (one per SM): a TMA producer thread
//             streams 128 x 64 (a) and 256 x 64 (W) bf16 tiles with 128-byte
//             swizzle through a 4-stage shared-memory ring (plain loads),
//             one thread issues tcgen05.mma (kind::f16, M=128, N=256, K=16)
//             into one of two 256-column fp32 accumulators in tensor memory
//             and frees each stage with tcgen05.commit; eight warps drain the
//             other accumulator with tcgen05.ld and store fp32 logits while
//             the next tile's MMAs run.  Tiles go M-index first, so CTAs
//             running together share W tiles and W streams from HBM once.
//   summary   (the fused top_k path) the drain warps store no logits: each
//             thread owns one row and 128 columns of the tile, applies the
//             row's repetition penalty (a per-row bitset of its history ids)
//             and temperature, and writes the KS largest values of those
//             columns (ties: lower id first) with their ids -- 64 bytes per
//             row and 128 columns instead of 512 bytes of logits.  A merge
//             kernel finishes the sampler's top_k path from these lists
//             (bm_kernel.cu).
//
// The reference computes its lm_head as a ternary BitLinear (src/model.c:
// 1239-1262); this bf16 variant has no counterpart there and is checked
// against a CPU GEMM of the same bf16 operands.  Every wait is bounded.
#include "bm_lmhead.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <climits>
#include <mutex>

namespace bml {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
// producer, MMA and the drain warps: four (one per accumulator lane quarter)
// storing logits, eight (two per quarter, each taking half of the tile's 256
// columns) for the summary epilogue
template <bool SUM>
__host__ __device__ constexpr int epi_warps() { return SUM ? 8 : 4; }
template <bool SUM>
__host__ __device__ constexpr int gemm_threads() { return 32 * (2 + epi_warps<SUM>()); }
constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t TMEM_COLS = 2 * BN;  // two fp32 accumulators, one column per n
constexpr size_t GEMM_SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
// the summary epilogue's staging: 32 columns x 256 drain threads of fp32
// (column j of drain thread t at [j][t]: bank t % 32, conflict-free for any
// column per thread)
constexpr size_t EPI_STAGE = 32 * 256 * 4;
constexpr size_t GEMM_SMEM_SUM = GEMM_SMEM + EPI_STAGE;
constexpr unsigned long long WAIT_NS = 2000000000ull;  // bounded waits: 2 s

// GPT-2 ids the reference never penalises (src/bitmamba.h:21-24).
__device__ __forceinline__ bool protected_id(int id) {
    return id == 50256 || id == 198 || id == 628 || id == 13;
}
// src/model.c:1298-1304: l > 0 ? l / penalty : l * penalty
__device__ __forceinline__ float penalize(float l, float pen) {
    return (l > 0.0f) ? __fdiv_rn(l, pen) : __fmul_rn(l, pen);
}
// (a, ia) ahead of (b, ib): larger value, then lower id (NaN never ahead)
__device__ __forceinline__ bool ahead(float a, int ia, float b, int ib) {
    return a > b || (a == b && ia < ib);
}

__device__ __forceinline__ uint32_t sa(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)),
                 "r"(bytes)
                 : "memory");
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
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity) {
    if (mbar_try(b, parity)) return true;
    const unsigned long long t0 = gtimer();
    for (unsigned it = 0; it < (1u << 30); ++it) {
        if (mbar_try(b, parity)) return true;
        if (gtimer() - t0 > WAIT_NS) return false;
    }
    return false;
}
// 16-byte asynchronous global -> shared copy (every copy of a row in flight
// at once), and the wait for this thread's copies
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_own() {
    asm volatile("cp.async.commit_group;\n cp.async.wait_all;" ::: "memory");
}
// 2-D tiled TMA load into this CTA only: box at (x = k, y = row) into smem
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
        "{%2, %3}], [%4];" ::"r"(sa(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(sa(bar))
        : "memory");
}
// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), version 1, layout 2.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_i8(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     sa(bar))
                 : "memory");
}
// 32 consecutive fp32 accumulator columns of this thread's lane
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Persistent: CTA c takes tiles c, c + grid, ... (M-tile index fastest, so
// CTAs running together share W tiles).  Warp 0 lane 0 is the TMA producer,
// warp 1 lane 0 issues the MMAs, warps 2-5 drain the accumulators.  Two
// 256-column accumulators in tensor memory let the drain of tile i overlap
// the MMAs of tile i + 1.
//
// I8: int8 operands (kind::i8, K = 32 per instruction, so a 128-byte stage row
// holds 128 elements), exact int32 accumulation, and the epilogue
// out = (float) acc * row_scale[row]; otherwise bf16 operands (kind::f16,
// 64 elements per stage row) and fp32 accumulators stored as they are.  The
// shared-memory tiles are byte-identical in shape either way.
template <bool I8, bool SUM>
__global__ void __launch_bounds__(gemm_threads<SUM>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                float *out, int M, int N, int K, int64_t ldo, const float *row_scale, int *err,
                const SumArgs sg, const int *dM, const int *out_rows) {
    constexpr int BKE = I8 ? 128 : BK;  // elements per 128-byte stage row
    if (dM) M = *dM;  // a row count the previous kernel wrote (0: no tiles)
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the 128-byte swizzle pattern repeats every 1024 bytes: tiles start on
    // a 1024-byte boundary
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~static_cast<uintptr_t>(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *accf = empty + STAGES;  // [2] accumulator b complete
    uint64_t *acce = accf + 2;        // [2] accumulator b drained
    uint32_t *tslot = reinterpret_cast<uint32_t *>(acce + 2);
    int *abort_ = reinterpret_cast<int *>(tslot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int MT = (M + BM - 1) / BM, NTL = (N + BN - 1) / BN;
    const int tiles = MT * NTL;
    const int KT = (K + BKE - 1) / BKE;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], epi_warps<SUM>());
        }
        *abort_ = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         sa(tslot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tslot;
    auto fail = [&]() { atomicOr(abort_, 1); };
    auto aborted = [&]() { return *reinterpret_cast<volatile int *>(abort_) != 0; };

    if (threadIdx.x == 0) {
        // producer: stage s is free once the MMAs that read it completed
        int g = 0;
        for (int t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x) {
            const int m0 = (t % MT) * BM, n0 = (t / MT) * BN;
            for (int kt = 0; kt < KT; ++kt, ++g) {
                const int s = g % STAGES;
                if (g >= STAGES && !mbar_wait(&empty[s], ((g / STAGES) - 1) & 1)) {
                    fail();
                    break;
                }
                unsigned char *st = smem + (size_t)s * STAGE_BYTES;
                mbar_expect_tx(&full[s], STAGE_BYTES);
                tma_load_2d(st, &tmA, kt * BKE, m0, &full[s]);
                tma_load_2d(st + A_BYTES, &tmB, kt * BKE, n0, &full[s]);
            }
        }
    } else if (threadIdx.x == 32) {
        // MMA issuer, A and B K-major, M=128, N=256: bf16 x bf16 -> fp32
        // (D format 1, A/B format 1 = bf16) or s8 x s8 -> s32 (D format 2,
        // A/B format 1 = signed)
        const uint32_t idesc = ((I8 ? 2u : 1u) << 4) | (1u << 7) | (1u << 10) |
                               ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
        int g = 0, i = 0;
        for (int t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x, ++i) {
            const int b = i & 1;
            if (i >= 2 && !mbar_wait(&acce[b], ((i >> 1) - 1) & 1)) {
                fail();
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t acc = tmem + (uint32_t)(b * BN);
            for (int kt = 0; kt < KT; ++kt, ++g) {
                const int s = g % STAGES;
                if (!mbar_wait(&full[s], (g / STAGES) & 1)) {
                    fail();
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t a0 = sa(smem + (size_t)s * STAGE_BYTES), b0 = a0 + A_BYTES;
                // four instructions of 32 bytes of K each (16 bf16 or 32 int8)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (I8)
                        umma_i8(acc, sdesc(a0 + k * 32), sdesc(b0 + k * 32), idesc,
                                (kt > 0 || k > 0) ? 1u : 0u);
                    else
                        umma_f16(acc, sdesc(a0 + k * 32), sdesc(b0 + k * 32), idesc,
                                 (kt > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(&accf[b]);  // arrives once every MMA of this tile completed
        }
    } else if (warp >= 2) {
        // drain: warp w reads accumulator lanes (rows) 32 (w % 4) .. + 31 and
        // (summary) columns 128 h .. + 127 of the tile, h = (w - 2) / 4
        constexpr int CPW = (BN / 32) * 4 / epi_warps<SUM>();  // 32-column chunks per warp
        const int q = warp & 3, h = (warp - 2) >> 2, td = (warp - 2) * 32 + lane;
        const bool vec = ((ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
        // this drain thread's column of the staging area
        float *cv = reinterpret_cast<float *>(smem + STAGES * STAGE_BYTES + 256) + td;
        int i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
            const int b = i & 1;
            const bool ok = !aborted() && mbar_wait(&accf[b], (i >> 1) & 1);
            if (!ok) {
                fail();
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int m0 = (t % MT) * BM, n0 = (t / MT) * BN;
            const int row = m0 + q * 32 + lane;
            const uint32_t tb = tmem + (uint32_t)(b * BN) + ((uint32_t)(q * 32) << 16);
            const float sc = (I8 && row < M) ? row_scale[row] : 1.0f;
            // summary: the row's knobs (greedy rows keep the raw penalised
            // logits, src/model.c:144-154; others are scaled by 1 / temp,
            // :156-163) and the KS best (value, id) of the 128 columns, as an
            // unordered set with its worst entry (wv, wi in slot ws) tracked
            float pen = 1.0f, inv = 1.0f;
            bool has_pen = false, row_full = false;
            float tv[KS], wv = -__builtin_huge_valf();
            int ti[KS], wi = INT_MAX, ws = 0;
#pragma unroll
            for (int k = 0; k < KS; ++k) { tv[k] = -__builtin_huge_valf(); ti[k] = INT_MAX; }
            // (value, id) into the set in place of its worst entry when ahead
            // of it; then the new worst by a three-level comparison tree
            auto put = [&](float x, int col) {
                if (!ahead(x, col, wv, wi)) return;
#pragma unroll
                for (int k = 0; k < KS; ++k) {
                    tv[k] = (k == ws) ? x : tv[k];
                    ti[k] = (k == ws) ? col : ti[k];
                }
                float v4[KS / 2];
                int i4[KS / 2], s4[KS / 2];
#pragma unroll
                for (int k = 0; k < KS / 2; ++k) {
                    const bool a = ahead(tv[2 * k], ti[2 * k], tv[2 * k + 1], ti[2 * k + 1]);
                    v4[k] = a ? tv[2 * k + 1] : tv[2 * k];
                    i4[k] = a ? ti[2 * k + 1] : ti[2 * k];
                    s4[k] = a ? 2 * k + 1 : 2 * k;
                }
#pragma unroll
                for (int n = KS / 4; n >= 1; n >>= 1) {
#pragma unroll
                    for (int k = 0; k < n; ++k) {
                        const bool a = ahead(v4[2 * k], i4[2 * k], v4[2 * k + 1], i4[2 * k + 1]);
                        v4[k] = a ? v4[2 * k + 1] : v4[2 * k];
                        i4[k] = a ? i4[2 * k + 1] : i4[2 * k];
                        s4[k] = a ? s4[2 * k + 1] : s4[2 * k];
                    }
                }
                wv = v4[0];
                wi = i4[0];
                ws = s4[0];
            };
            if (SUM && row < M) {
                const bm_knobs_t kn = sg.knobs[(int64_t)row * sg.knob_stride];
                inv = (kn.temp < 0.05f) ? 1.0f : kn.inv_temp;
                pen = kn.penalty;
                // rows of the full-vocabulary path (src/model.c:282-360) get
                // their logits stored instead
                row_full = !(kn.temp < 0.05f) && !(kn.top_k > 0 && kn.top_k <= 256);
                has_pen = sg.pbits && (kn.penalty > 0.0f) && (kn.penalty != 1.0f);
            }
#pragma unroll 1
            for (int c = CPW * h; c < CPW * h + CPW; ++c) {
                uint32_t r[32];
                tmem_ld32(tb + c * 32, r);
                if (I8) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        r[j] = __float_as_uint(__fmul_rn(__int2float_rn((int)r[j]), sc));
                }
                const int col0 = n0 + c * 32;
                if (SUM && !row_full) {
                    if (row < M && col0 < N) {
                        // stage the chunk, mark the columns ahead of the set's
                        // worst entry (branch-free), insert only those; the
                        // penalised columns (history ids, rare) separately
                        const int nv = min(32, N - col0);
                        const uint32_t live = nv < 32 ? (1u << nv) - 1u : 0xffffffffu;
                        const uint32_t pm =
                            (has_pen ? sg.pbits[(int64_t)row * sg.pw + (col0 >> 5)] : 0u) & live;
                        const float lv = wv;
                        const int li = wi;
                        uint32_t mask = 0;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float x = __uint_as_float(r[j]);
                            cv[j * 256] = x;
                            const float y = __fmul_rn(x, inv);
                            mask |= (ahead(y, col0 + j, lv, li) ? 1u : 0u) << j;
                        }
                        mask &= live & ~pm;
                        for (; mask; mask &= mask - 1) {
                            const int j = __ffs(mask) - 1;
                            put(__fmul_rn(cv[j * 256], inv), col0 + j);
                        }
                        for (uint32_t m = pm; m; m &= m - 1) {
                            const int j = __ffs(m) - 1;
                            put(__fmul_rn(penalize(cv[j * 256], pen), inv), col0 + j);
                        }
                    }
                    continue;
                }
                if (row < M && col0 < N) {
                    float *o = out + (int64_t)(out_rows ? out_rows[row] : row) * ldo + col0;
                    if (vec && col0 + 32 <= N) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4 *>(o + j) =
                                make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                            __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < N) o[j] = __uint_as_float(r[j]);
                    }
                }
            }
            if (SUM && row < M && !row_full) {
                // entries (bits(value) << 32) | id in no order, unused slots
                // id 0xffffffff; list 2 t' + h of the row for tile column t'
                uint4 *o = reinterpret_cast<uint4 *>(
                    sg.summ + ((int64_t)row * 2 * NTL + 2 * (t / MT) + h) * KS);
#pragma unroll
                for (int k = 0; k < KS; k += 2) {
                    const uint32_t i0 = ti[k] == INT_MAX ? 0xffffffffu : (uint32_t)ti[k];
                    const uint32_t i1 = ti[k + 1] == INT_MAX ? 0xffffffffu : (uint32_t)ti[k + 1];
                    o[k / 2] = make_uint4(i0, __float_as_uint(tv[k]), i1, __float_as_uint(tv[k + 1]));
                }
            }
            // the accumulator is free for the MMAs of tile i + 2
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(&acce[b])) : "memory");
        }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS)
                     : "memory");
    if (threadIdx.x == 0 && *abort_) atomicOr(err, 4);
}

// One warp per row: the row is staged in shared memory with 16-byte loads,
// lanes 0-3 keep the reference's four strided accumulators (multiply, then
// add: the library is built without contraction), lane 0 adds them left to
// right with the tail; the norm weight is staged once per block.  D % 4 == 0.
constexpr int RN_WARPS = 8;
constexpr int RN_MAXD = 4096;  // floats staged per warp

__global__ void __launch_bounds__(RN_WARPS * 32)
    rmsnorm_kernel(const float *x, int B, int D, const float *w, __nv_bfloat16 *a) {
    extern __shared__ float4 rn_smem4[];
    float *wbuf = reinterpret_cast<float *>(rn_smem4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *buf = wbuf + D + (size_t)warp * D;
    const int D4 = D / 4;
    for (int i = threadIdx.x; i < D4; i += blockDim.x)
        reinterpret_cast<float4 *>(wbuf)[i] = reinterpret_cast<const float4 *>(w)[i];
    __syncthreads();
    for (int r = blockIdx.x * RN_WARPS + warp; r < B; r += gridDim.x * RN_WARPS) {
        const float4 *xr = reinterpret_cast<const float4 *>(x + (int64_t)r * D);
        for (int i = lane; i < D4; i += 32) cp_async16(buf + 4 * i, xr + i);
        cp_async_wait_own();
        __syncwarp();
        float s = 0.0f;
        if (lane < 4) {
#pragma unroll 8
            for (int i = lane; i < 4 * D4; i += 4) s = __fadd_rn(s, __fmul_rn(buf[i], buf[i]));
        }
        const float s1 = __shfl_sync(0xffffffffu, s, 1), s2 = __shfl_sync(0xffffffffu, s, 2),
                    s3 = __shfl_sync(0xffffffffu, s, 3);
        float rms = 0.0f;
        if (lane == 0) {
            const float sum = __fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3);
            rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)D), 1e-6f)));
        }
        rms = __shfl_sync(0xffffffffu, rms, 0);
        __nv_bfloat162 *ar = reinterpret_cast<__nv_bfloat162 *>(a + (int64_t)r * D);
#pragma unroll 4
        for (int i = lane; i < D / 2; i += 32) {
            const float v0 = __fmul_rn(__fmul_rn(buf[2 * i], rms), wbuf[2 * i]);
            const float v1 = __fmul_rn(__fmul_rn(buf[2 * i + 1], rms), wbuf[2 * i + 1]);
            ar[i] = __halves2bfloat162(__float2bfloat16_rn(v0), __float2bfloat16_rn(v1));
        }
        __syncwarp();
    }
}

// ------------------------------------------------------ ternary lm_head --
// The reference's logits producer on x86-64 (AVX2 kernels):
//   final_feat = rms_norm(x, norm_f)                  src/model.c:1225
//   xn = rms_norm(final_feat, lm_head_norm), max|xn|  src/arch/avx2.c:278
//   scale_x = 127 / (max|xn| + 1e-5f)                 src/arch/avx2.c:279
//   xq = int8(round_even(max(-128, min(xn * scale_x, 127))))
//                                                      src/arch/avx2.c:290-315
//   inv_scale = 1 / (scale_x * w_scale)               src/arch/avx2.c:684
// rms_norm in avx2_rms_norm's order (src/arch/avx2.c:22-83, D % 32 == 0):
// lane j of the warp is the reference's accumulator j (four 8-wide vectors),
// taking x[j], x[j + 32], ... by fused multiply-add; lanes combine as
// (s[l] + s[l + 8]) + (s[l + 16] + s[l + 24]), l = 0..7, added left to right
// from 0; rms = 1 / sqrtf(sum / D + 1e-6f); out = (x * rms) * w.
__device__ __forceinline__ float rms_x86(const float *buf, int D, int lane) {
    float s = 0.0f;
#pragma unroll 8
    for (int i = lane; i < D; i += 32) s = __fmaf_rn(buf[i], buf[i], s);
    const float a = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 8));
    const float t = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 16));
    float sum = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, t, l));
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)D), 1e-6f)));
}

// One warp per row; both norm weights staged once per block, the row in
// shared memory.  xq: [B x D] int8, inv_scale: [B].
__global__ void __launch_bounds__(RN_WARPS * 32)
    ternary_prep_kernel(const float *x, int B, int D, const float *norm_f, const float *lmh_norm,
                        float w_scale, int8_t *xq, float *inv_scale) {
    extern __shared__ float4 tp_smem4[];
    float *wl = reinterpret_cast<float *>(tp_smem4);
    float *wf = wl + D;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *buf = wf + D + (size_t)warp * D;
    const int D4 = D / 4;
    for (int i = threadIdx.x; i < D4; i += blockDim.x) {
        reinterpret_cast<float4 *>(wl)[i] = reinterpret_cast<const float4 *>(lmh_norm)[i];
        if (norm_f) reinterpret_cast<float4 *>(wf)[i] = reinterpret_cast<const float4 *>(norm_f)[i];
    }
    __syncthreads();
    for (int r = blockIdx.x * RN_WARPS + warp; r < B; r += gridDim.x * RN_WARPS) {
        const float4 *xr = reinterpret_cast<const float4 *>(x + (int64_t)r * D);
        for (int i = lane; i < D4; i += 32) cp_async16(buf + 4 * i, xr + i);
        cp_async_wait_own();
        __syncwarp();
        if (norm_f) {
            const float rms = rms_x86(buf, D, lane);
            for (int i = lane; i < D; i += 32) buf[i] = __fmul_rn(__fmul_rn(buf[i], rms), wf[i]);
            __syncwarp();
        }
        const float rms = rms_x86(buf, D, lane);
        float ma = 0.0f;
        for (int i = lane; i < D; i += 32) {
            const float v = __fmul_rn(__fmul_rn(buf[i], rms), wl[i]);
            buf[i] = v;
            ma = fmaxf(ma, fabsf(v));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
        __syncwarp();
        const float scale_x = __fdiv_rn(127.0f, __fadd_rn(ma, 1e-5f));
        char4 *qr = reinterpret_cast<char4 *>(xq + (int64_t)r * D);
        for (int i = lane; i < D4; i += 32) {
            const float4 v4 = reinterpret_cast<const float4 *>(buf)[i];
            const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
            signed char qv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float v = __fmul_rn(vv[j], scale_x);
                v = v < 127.0f ? v : 127.0f;
                v = -128.0f > v ? -128.0f : v;
                qv[j] = (signed char)__float2int_rn(v);
            }
            qr[i] = make_char4(qv[0], qv[1], qv[2], qv[3]);
        }
        if (lane == 0) inv_scale[r] = __fdiv_rn(1.0f, __fmul_rn(scale_x, w_scale));
        __syncwarp();
    }
}

// 2-bit codes (four per byte, lowest bits first; src/quantization.c:27-31
// decodes code c as min(c, 2) - 1) to int8 {-1, 0, 1}: 4 packed bytes in,
// 16 weights out per step.  The packed rows are D / 4 bytes, the int8 rows D
// bytes, so the flat byte order carries over.
__global__ void ternary_unpack_kernel(const uint32_t *packed, int64_t n4, uint4 *w8) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t p = packed[i];
        uint32_t o[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            uint32_t w = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t c = (p >> (8 * b + 2 * j)) & 3u;
                const uint32_t v = (uint32_t)((int)(c < 2u ? c : 2u) - 1) & 0xffu;
                w |= v << (8 * j);
            }
            o[b] = w;
        }
        w8[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_mu;

cudaError_t get_encode() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode) return cudaSuccess;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return cudaSuccess;
}

// rows x K row-major (bf16, or int8 when i8), box of one 128-byte row of K
// (64 bf16 / 128 int8) x box_rows, 128-byte swizzle, zero fill
cudaError_t make_map(CUtensorMap *m, const void *base, int rows, int K, int box_rows, bool i8) {
    const int esz = i8 ? 1 : 2;
    const cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)K * esz};
    const cuuint32_t box[2] = {(cuuint32_t)(128 / esz), (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(m, i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                2, const_cast<void *>(base),
                                gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// a, W: [M x K] and [N x K] K-major (int8 when row_scale is given, else bf16);
// sg.summ set: the summary epilogue instead of the logits
cudaError_t launch_gemm(const void *a, const void *W, int M, int N, int K, const float *row_scale,
                        float *out, int64_t ldo, int *err, cudaStream_t s, const SumArgs &sg,
                        const int *dM, const int *out_rows) {
    const bool i8 = row_scale != nullptr;
    const bool sum = sg.summ != nullptr;
    CUtensorMap ma, mb;
    cudaError_t e;
    if ((e = make_map(&ma, a, M, K, BM, i8)) != cudaSuccess) return e;
    if ((e = make_map(&mb, W, N, K, BN, i8)) != cudaSuccess) return e;
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    const long long tiles = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    if (tiles > (1LL << 30)) return cudaErrorInvalidValue;
    const int grid = (int)(tiles < sms ? tiles : sms);
    if (i8 && sum)
        gemm_kernel<true, true><<<grid, gemm_threads<true>(), GEMM_SMEM_SUM, s>>>(ma, mb, out, M, N, K, ldo, row_scale,
                                                            err, sg, dM, out_rows);
    else if (i8)
        gemm_kernel<true, false><<<grid, gemm_threads<false>(), GEMM_SMEM, s>>>(ma, mb, out, M, N, K, ldo, row_scale,
                                                             err, sg, dM, out_rows);
    else if (sum)
        gemm_kernel<false, true><<<grid, gemm_threads<true>(), GEMM_SMEM_SUM, s>>>(ma, mb, out, M, N, K, ldo, nullptr,
                                                             err, sg, dM, out_rows);
    else
        gemm_kernel<false, false><<<grid, gemm_threads<false>(), GEMM_SMEM, s>>>(ma, mb, out, M, N, K, ldo, nullptr,
                                                              err, sg, dM, out_rows);
    return cudaGetLastError();
}

// One CTA per row: clear the row's bits, then set those of its history.
__global__ void __launch_bounds__(256) penbits_kernel(const int32_t *hist, const int64_t *off,
                                                      int V, uint32_t *bits, int pw) {
    const int r = blockIdx.x;
    uint32_t *b = bits + (int64_t)r * pw;
    for (int i = threadIdx.x; i < pw; i += blockDim.x) b[i] = 0u;
    __syncthreads();
    const int64_t h0 = off[r], h1 = off[r + 1];
    for (int64_t i = h0 + threadIdx.x; i < h1; i += blockDim.x) {
        const int id = hist[i];
        if (id >= 0 && id < V && !protected_id(id)) atomicOr(&b[id >> 5], 1u << (id & 31));
    }
}

// Rows of 16-byte words: block-stride over the listed rows.
__global__ void gather_kernel(const uint4 *src, int64_t w16, const int *list, uint4 *dst,
                              const float *ssc, float *dsc) {
    const int n = list[0];
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        const int r = list[1 + i];
        const uint4 *sr = src + (int64_t)r * w16;
        uint4 *dr = dst + (int64_t)i * w16;
        for (int64_t k = threadIdx.x; k < w16; k += blockDim.x) dr[k] = sr[k];
        if (ssc && threadIdx.x == 0) dsc[i] = ssc[r];
    }
}

}  // namespace

cudaError_t prepare() {
    cudaError_t e = get_encode();
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(gemm_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)GEMM_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(gemm_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)GEMM_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(gemm_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)GEMM_SMEM_SUM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(gemm_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)GEMM_SMEM_SUM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(ternary_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)((RN_WARPS + 2) * RN_MAXD * sizeof(float)));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)((RN_WARPS + 1) * RN_MAXD * sizeof(float)));
}

cudaError_t rmsnorm_bf16(const float *x, int B, int D, const float *w, uint16_t *a,
                         cudaStream_t s) {
    if (B <= 0) return cudaSuccess;
    if (D <= 0 || D > RN_MAXD || D % 4 || (reinterpret_cast<uintptr_t>(x) & 15) ||
        (reinterpret_cast<uintptr_t>(w) & 15))
        return cudaErrorInvalidValue;
    int grid = (B + RN_WARPS - 1) / RN_WARPS;
    if (grid > 148 * 8) grid = 148 * 8;
    rmsnorm_kernel<<<grid, RN_WARPS * 32, (size_t)(RN_WARPS + 1) * D * sizeof(float), s>>>(
        x, B, D, w, reinterpret_cast<__nv_bfloat16 *>(a));
    return cudaGetLastError();
}

cudaError_t gemm_bf16(const uint16_t *a, const uint16_t *W, int M, int N, int K, float *out,
                      int64_t ldo, int *err, cudaStream_t s, const int *dM, const int *out_rows) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (K <= 0 || K % 8 || (reinterpret_cast<uintptr_t>(a) & 15) ||
        (reinterpret_cast<uintptr_t>(W) & 15) || ldo < N)
        return cudaErrorInvalidValue;
    cudaError_t e = get_encode();
    if (e != cudaSuccess) return e;
    return launch_gemm(a, W, M, N, K, nullptr, out, ldo, err, s, SumArgs{}, dM, out_rows);
}

cudaError_t gemm_i8(const int8_t *a, const int8_t *W, int M, int N, int K, const float *row_scale,
                    float *out, int64_t ldo, int *err, cudaStream_t s, const int *dM,
                    const int *out_rows) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (K <= 0 || K % 16 || (reinterpret_cast<uintptr_t>(a) & 15) ||
        (reinterpret_cast<uintptr_t>(W) & 15) || ldo < N || !row_scale)
        return cudaErrorInvalidValue;
    cudaError_t e = get_encode();
    if (e != cudaSuccess) return e;
    return launch_gemm(a, W, M, N, K, row_scale, out, ldo, err, s, SumArgs{}, dM, out_rows);
}

cudaError_t gemm_bf16_summary(const uint16_t *a, const uint16_t *W, int M, int N, int K,
                              const SumArgs &sg, float *out, int64_t ldo, int *err,
                              cudaStream_t s) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (K <= 0 || K % 8 || (reinterpret_cast<uintptr_t>(a) & 15) || !out || ldo < N ||
        (reinterpret_cast<uintptr_t>(W) & 15) || !sg.summ || !sg.knobs ||
        (reinterpret_cast<uintptr_t>(sg.summ) & 15) || (sg.pbits && sg.pw < (N + 31) / 32))
        return cudaErrorInvalidValue;
    cudaError_t e = get_encode();
    if (e != cudaSuccess) return e;
    return launch_gemm(a, W, M, N, K, nullptr, out, ldo, err, s, sg, nullptr, nullptr);
}

cudaError_t gemm_i8_summary(const int8_t *a, const int8_t *W, int M, int N, int K,
                            const float *row_scale, const SumArgs &sg, float *out, int64_t ldo,
                            int *err, cudaStream_t s) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (K <= 0 || K % 16 || (reinterpret_cast<uintptr_t>(a) & 15) || !out || ldo < N ||
        (reinterpret_cast<uintptr_t>(W) & 15) || !row_scale || !sg.summ || !sg.knobs ||
        (reinterpret_cast<uintptr_t>(sg.summ) & 15) || (sg.pbits && sg.pw < (N + 31) / 32))
        return cudaErrorInvalidValue;
    cudaError_t e = get_encode();
    if (e != cudaSuccess) return e;
    return launch_gemm(a, W, M, N, K, row_scale, out, ldo, err, s, sg, nullptr, nullptr);
}

cudaError_t penalty_bits(const int32_t *hist, const int64_t *hist_off, int B, int V,
                         uint32_t *bits, int pw, cudaStream_t s) {
    if (B <= 0) return cudaSuccess;
    if (!hist || !hist_off || !bits || pw < (V + 31) / 32) return cudaErrorInvalidValue;
    penbits_kernel<<<B, 256, 0, s>>>(hist, hist_off, V, bits, pw);
    return cudaGetLastError();
}

cudaError_t gather_rows(const void *src, int64_t row_bytes, const int *list, void *dst,
                        const float *ssc, float *dsc, int max_rows, cudaStream_t s) {
    if (max_rows <= 0) return cudaSuccess;
    if (row_bytes % 16 || (reinterpret_cast<uintptr_t>(src) & 15) ||
        (reinterpret_cast<uintptr_t>(dst) & 15))
        return cudaErrorInvalidValue;
    const int grid = max_rows < 148 * 4 ? max_rows : 148 * 4;
    gather_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const uint4 *>(src), row_bytes / 16, list,
                                       reinterpret_cast<uint4 *>(dst), ssc, dsc);
    return cudaGetLastError();
}

cudaError_t ternary_prep(const float *x, int B, int D, const float *norm_f, const float *lmh_norm,
                         float w_scale, int8_t *xq, float *inv_scale, cudaStream_t s) {
    if (B <= 0) return cudaSuccess;
    if (D <= 0 || D > RN_MAXD || D % 32 || (reinterpret_cast<uintptr_t>(x) & 15) ||
        (reinterpret_cast<uintptr_t>(lmh_norm) & 15) ||
        (norm_f && (reinterpret_cast<uintptr_t>(norm_f) & 15)) ||
        (reinterpret_cast<uintptr_t>(xq) & 3))
        return cudaErrorInvalidValue;
    int grid = (B + RN_WARPS - 1) / RN_WARPS;
    if (grid > 148 * 8) grid = 148 * 8;
    ternary_prep_kernel<<<grid, RN_WARPS * 32, (size_t)(RN_WARPS + 2) * D * sizeof(float), s>>>(
        x, B, D, norm_f, lmh_norm, w_scale, xq, inv_scale);
    return cudaGetLastError();
}

cudaError_t ternary_unpack(const uint8_t *packed, int V, int D, int8_t *w8, cudaStream_t s) {
    if (V <= 0) return cudaSuccess;
    if (D <= 0 || D % 16 || (reinterpret_cast<uintptr_t>(packed) & 3) ||
        (reinterpret_cast<uintptr_t>(w8) & 15))
        return cudaErrorInvalidValue;
    const int64_t n4 = (int64_t)V * (D / 16);
    int64_t grid = (n4 + 255) / 256;
    if (grid > 148 * 16) grid = 148 * 16;
    ternary_unpack_kernel<<<(int)grid, 256, 0, s>>>(reinterpret_cast<const uint32_t *>(packed), n4,
                                                   reinterpret_cast<uint4 *>(w8));
    return cudaGetLastError();
}

}  // namespace bml
