// Internal interface of the final RMSNorm + bf16 lm_head GEMM (bm_lmhead.cu)
// that feeds the sampler.  Not part of the public ABI.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "bm_sampler.h"

namespace bml {

constexpr int LIST_N = 128;  // columns per summary list
constexpr int KS = 4;        // entries per summary list

// Summary lists per row for V columns (two per 256-column GEMM tile).
inline int summary_lists(int V) { return 2 * ((V + 255) / 256); }

// The summary epilogue's inputs and output.  List j of row r covers the
// columns [128 j, 128 j + 128); its entries summ[(r * lists + j) * KS + k],
// k < KS, are (bits(value) << 32) | id of the KS largest penalised,
// temperature-scaled logits of the row in those columns (greedy rows:
// unscaled; ties by lower id first), in no particular order; unused slots
// have id 0xffffffff.
struct SumArgs {
    const uint32_t *pbits;  // [M x pw] the rows' history bits (NULL: no penalty)
    int pw;                 // words per row of pbits
    const bm_knobs_t *knobs;
    int64_t knob_stride;
    uint64_t *summ;
};

// a[r, :] = bf16(x[r, :] * rms_r * w), rms_r = 1 / sqrtf(sum_sq / D + 1e-6f)
// with the sum of squares accumulated as jserv/bitmamba.c src/kernel.c:72-91
// does (four strided fp32 accumulators, added left to right).
cudaError_t rmsnorm_bf16(const float *x, int B, int D, const float *w, uint16_t *a,
                         cudaStream_t s);

// out[r, n] = sum_k a[r, k] * W[n, k] (bf16 inputs, fp32 accumulation on the
// tensor cores), out row pitch ldo floats.  a: [M x K] and W: [N x K]
// row-major bf16 (K-major operands), both 16-byte aligned, K % 8 == 0.
// err: device word, bit 2 set when a bounded wait expired.
// dM (optional): the row count is read from this device word at launch
// instead (a count an earlier kernel wrote; rows beyond it are not computed).
// out_rows (optional): row r of the product is stored at out row out_rows[r].
cudaError_t gemm_bf16(const uint16_t *a, const uint16_t *W, int M, int N, int K, float *out,
                      int64_t ldo, int *err, cudaStream_t s, const int *dM = nullptr,
                      const int *out_rows = nullptr);

// out[r, n] = (float) sum_k a[r, k] * W[n, k] * row_scale[r]: int8 inputs,
// exact int32 accumulation on the tensor cores, one conversion and one fp32
// multiply per element.  a: [M x K], W: [N x K] row-major int8, 16-byte
// aligned, K % 16 == 0.
cudaError_t gemm_i8(const int8_t *a, const int8_t *W, int M, int N, int K, const float *row_scale,
                    float *out, int64_t ldo, int *err, cudaStream_t s, const int *dM = nullptr,
                    const int *out_rows = nullptr);

// The same GEMMs with the summary epilogue (SumArgs) for greedy rows and
// rows of the sampler's top_k path (1 <= top_k <= 256); the other rows' logits
// are stored in out (pitch ldo) as the plain GEMM stores them.
cudaError_t gemm_bf16_summary(const uint16_t *a, const uint16_t *W, int M, int N, int K,
                              const SumArgs &sg, float *out, int64_t ldo, int *err,
                              cudaStream_t s);
cudaError_t gemm_i8_summary(const int8_t *a, const int8_t *W, int M, int N, int K,
                            const float *row_scale, const SumArgs &sg, float *out, int64_t ldo,
                            int *err, cudaStream_t s);

// bits[r * pw + (id >> 5)] bit (id & 31) set for every distinct history id
// of row r in [0, V) that the reference penalises (src/model.c:1276-1281,
// protected ids src/bitmamba.h:21-24).  pw >= (V + 31) / 32.
cudaError_t penalty_bits(const int32_t *hist, const int64_t *hist_off, int B, int V,
                         uint32_t *bits, int pw, cudaStream_t s);

// dst row i = src row list[1 + i] for i < list[0] (rows of row_bytes bytes,
// a multiple of 16, 16-byte aligned); also dsc[i] = ssc[list[1 + i]] when
// ssc is given.  At most max_rows rows.
cudaError_t gather_rows(const void *src, int64_t row_bytes, const int *list, void *dst,
                        const float *ssc, float *dsc, int max_rows, cudaStream_t s);

// The ternary BitLinear's activations: per row, the final RMSNorm (norm_f;
// skipped when NULL), the BitLinear's RMSNorm (lmh_norm), int8 absmax
// quantisation, inv_scale[r] = 1 / (scale_x * w_scale), all in the order of
// jserv/bitmamba.c's AVX2 kernels (src/arch/avx2.c:22-83, 276-315).
// D % 32 == 0, D <= 4096.
cudaError_t ternary_prep(const float *x, int B, int D, const float *norm_f, const float *lmh_norm,
                         float w_scale, int8_t *xq, float *inv_scale, cudaStream_t s);

// 2-bit packed ternary weights [V x D/4] -> int8 [V x D].  D % 16 == 0.
cudaError_t ternary_unpack(const uint8_t *packed, int V, int D, int8_t *w8, cudaStream_t s);

// One-time per-device setup (dynamic shared memory opt-in, driver entry point).
cudaError_t prepare();

}  // namespace bml
