/*
 * CPU oracle for the ternary BitLinear lm_head (TEST INFRASTRUCTURE ONLY).
 *
 * A plain-C restatement of the logits producer of jserv/bitmamba.c's decode
 * step on x86-64 hosts with AVX2+FMA (the kernels src/dispatch.c:31-38
 * selects there):
 *
 *   final_feat = rms_norm(x, norm_f)              src/model.c:1225
 *   xn         = rms_norm(final_feat, lm_head_norm)   src/arch/avx2.c:278
 *   scale_x    = 127 / (max|xn| + 1e-5f)          src/arch/avx2.c:279
 *   xq         = int8(round_even(clamp(xn * scale_x, -128, 127)))
 *                                                  src/arch/avx2.c:290-315
 *   logits[v]  = (float) sum_k xq[k] * W[v][k] * (1 / (scale_x * w_scale))
 *                                                  src/arch/avx2.c:159, 684
 *
 * rms_norm follows avx2_rms_norm (src/arch/avx2.c:22-83) for d % 32 == 0:
 * 32 fp32 accumulators, accumulator j taking x[j], x[j+32], ... by fused
 * multiply-add (the reference uses _mm256_fmadd_ps), lanes combined as
 * (s[l] + s[l+8]) + (s[l+16] + s[l+24]) for l = 0..7, those eight added
 * left to right from 0, rms = 1 / sqrtf(sum / d + 1e-6f), out = (x * rms) * w
 * (two roundings), max|out| tracked.  The weights are the exporter's 2-bit
 * codes (scripts/export-bin.py:99-107: code = w + 1, four per byte, lowest
 * bits first), decoded as min(code, 2) - 1 (src/quantization.c:27-31).  The
 * integer dot product is exact, so the logits are one int->float conversion
 * and one multiply per element.
 *
 * Nothing in the product library links, loads or calls this file.
 */
#include "ternary_oracle.h"

#include <math.h>
#include <stddef.h>

float bmo_rms_norm_x86(const float *x, int d, const float *w, float *out)
{
    float s[32];
    for (int j = 0; j < 32; j++)
        s[j] = 0.0f;
    for (int i = 0; i < d; i += 32)
        for (int j = 0; j < 32; j++)
            s[j] = fmaf(x[i + j], x[i + j], s[j]);
    float sum = 0.0f;
    for (int l = 0; l < 8; l++)
        sum += (s[l] + s[l + 8]) + (s[l + 16] + s[l + 24]);
    const float rms = 1.0f / sqrtf(sum / (float) d + 1e-6f);
    float ma = 0.0f;
    for (int i = 0; i < d; i++) {
        const float t = x[i] * rms;
        const float v = t * w[i];
        out[i] = v;
        const float a = fabsf(v);
        if (a > ma)
            ma = a;
    }
    return ma;
}

int bmo_ternary_prep(const float *x, int B, int d, const float *norm_f,
                     const float *lmh_norm, float w_scale, float *scratch,
                     int8_t *xq, float *inv_scale)
{
    if (d <= 0 || d % 32)
        return -1;
    float *feat = scratch, *xn = scratch + d;
    for (int b = 0; b < B; b++) {
        const float *xr = x + (size_t) b * d;
        if (norm_f) {
            (void) bmo_rms_norm_x86(xr, d, norm_f, feat);
            xr = feat;
        }
        const float ma = bmo_rms_norm_x86(xr, d, lmh_norm, xn);
        const float scale_x = 127.0f / (ma + 1e-5f);
        int8_t *q = xq + (size_t) b * d;
        for (int i = 0; i < d; i++) {
            float v = xn[i] * scale_x;
            v = v < 127.0f ? v : 127.0f;   /* _mm256_min_ps(v, 127) */
            v = -128.0f > v ? -128.0f : v; /* _mm256_max_ps(-128, v) */
            q[i] = (int8_t) nearbyintf(v); /* round half to even */
        }
        const float t = scale_x * w_scale;
        inv_scale[b] = 1.0f / t;
    }
    return 0;
}

static inline int decode(unsigned code)
{
    return (int) (code < 2u ? code : 2u) - 1;
}

void bmo_ternary_unpack(const uint8_t *packed, int V, int d, int8_t *w8)
{
    const int stride = (d + 3) / 4;
    for (int v = 0; v < V; v++)
        for (int k = 0; k < d; k++) {
            const unsigned byte = packed[(size_t) v * stride + k / 4];
            w8[(size_t) v * d + k] = (int8_t) decode((byte >> (2 * (k & 3))) & 3u);
        }
}

void bmo_ternary_logits(const int8_t *xq, const float *inv_scale, int B, int d,
                        const uint8_t *packed, int V, float *out, int64_t ld)
{
    const int stride = (d + 3) / 4;
    for (int v = 0; v < V; v++) {
        const uint8_t *row = packed + (size_t) v * stride;
        for (int b = 0; b < B; b++) {
            const int8_t *q = xq + (size_t) b * d;
            int32_t total = 0;
            for (int k = 0; k < d; k++)
                total += decode((row[k / 4] >> (2 * (k & 3))) & 3u) * q[k];
            out[(size_t) b * ld + v] = (float) total * inv_scale[b];
        }
    }
}
