// Internal interface of the final RMSNorm + bf16 lm_head GEMM (bm_lmhead.cu)
// that feeds the sampler.  Not part of the public ABI.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace bml {

// a[r, :] = bf16(x[r, :] * rms_r * w), rms_r = 1 / sqrtf(sum_sq / D + 1e-6f)
// with the sum of squares accumulated as jserv/bitmamba.c src/kernel.c:72-91
// does (four strided fp32 accumulators, added left to right).
cudaError_t rmsnorm_bf16(const float *x, int B, int D, const float *w, uint16_t *a,
                         cudaStream_t s);

// out[r, n] = sum_k a[r, k] * W[n, k] (bf16 inputs, fp32 accumulation on the
// tensor cores), out row pitch ldo floats.  a: [M x K] and W: [N x K]
// row-major bf16 (K-major operands), both 16-byte aligned, K % 8 == 0.
// err: device word, bit 2 set when a bounded wait expired.
cudaError_t gemm_bf16(const uint16_t *a, const uint16_t *W, int M, int N, int K, float *out,
                      int64_t ldo, int *err, cudaStream_t s);

// out[r, n] = (float) sum_k a[r, k] * W[n, k] * row_scale[r]: int8 inputs,
// exact int32 accumulation on the tensor cores, one conversion and one fp32
// multiply per element.  a: [M x K], W: [N x K] row-major int8, 16-byte
// aligned, K % 16 == 0.
cudaError_t gemm_i8(const int8_t *a, const int8_t *W, int M, int N, int K, const float *row_scale,
                    float *out, int64_t ldo, int *err, cudaStream_t s);

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
