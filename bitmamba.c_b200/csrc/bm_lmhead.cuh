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

// One-time per-device setup (dynamic shared memory opt-in, driver entry point).
cudaError_t prepare();

}  // namespace bml
