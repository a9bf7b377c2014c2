/*
 * CPU oracle for the ternary BitLinear lm_head (TEST INFRASTRUCTURE ONLY).
 * Restates jserv/bitmamba.c src/model.c:1225-1262 with the x86 AVX2 kernels
 * (src/arch/avx2.c:22-83, 99-230, 276-315, 666-714); see ternary_oracle.c.
 */
#ifndef BM_TERNARY_ORACLE_H
#define BM_TERNARY_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out = rms_norm(x) * w in avx2_rms_norm's order; returns max|out|.
 * d % 32 == 0. */
float bmo_rms_norm_x86(const float *x, int d, const float *w, float *out);

/* Per row: the final norm (skipped when norm_f is NULL), the BitLinear's
 * own norm, int8 absmax quantisation; inv_scale[b] = 1 / (scale_x * w_scale).
 * scratch: 2 * d floats.  Returns -1 unless d % 32 == 0. */
int bmo_ternary_prep(const float *x, int B, int d, const float *norm_f,
                     const float *lmh_norm, float w_scale, float *scratch,
                     int8_t *xq, float *inv_scale);

/* 2-bit packed [V x (d + 3) / 4] -> int8 [V x d] in {-1, 0, 1}. */
void bmo_ternary_unpack(const uint8_t *packed, int V, int d, int8_t *w8);

/* out[b * ld + v] = (float) dot(xq[b], W[v]) * inv_scale[b]. */
void bmo_ternary_logits(const int8_t *xq, const float *inv_scale, int B, int d,
                        const uint8_t *packed, int V, float *out, int64_t ld);

#ifdef __cplusplus
}
#endif

#endif
