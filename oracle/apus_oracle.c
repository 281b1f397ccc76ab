/*
 * apus_oracle.c — CPU restatement of the apus speculative-decode path.
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels.  Built with
 * -ffp-contract=off like the reference (Makefile:27), so every a*b+c below
 * is two IEEE roundings.
 */
#include "apus_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ num */

/* c/num.h:162-166 — exact widen */
float orc_bf16_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* c/num.h:153-160 — RNE via the 0x7FFF + lsb bias, NaN keeps its high bits */
uint16_t orc_bf16_bits(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(u >> 16);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* c/num.h:143-151 */
float orc_bf16_round(float x) { return orc_bf16_f32(orc_bf16_bits(x)); }

/* c/num.h:136-141 — exact; e=15,m=7 decodes as the normal 480 */
float orc_e4m3_f32(uint8_t c) {
    int e = (c >> 3) & 15, m = c & 7;
    float v = e ? ldexpf((float)(8 + m), e - 10) : ldexpf((float)m, -9);
    return (c & 0x80) ? -v : v;
}

/* c/num.h:110-134 — RNE to E4M3, clamped to +-448 */
static uint32_t orc_rne_shift(uint32_t m, int sh) {
    uint32_t half = 1u << (sh - 1), mask = (1u << sh) - 1u;
    uint32_t r = m & mask, v = m >> sh;
    if (r > half || (r == half && (v & 1u))) v++;
    return v;
}

uint8_t orc_e4m3_quant(float x) {
    if (x > 448.0f) x = 448.0f;
    else if (x < -448.0f) x = -448.0f;
    uint32_t u;
    memcpy(&u, &x, 4);
    uint32_t sign = (u >> 31) << 7, a = u & 0x7fffffffu;
    if (!a) return (uint8_t)sign;
    int e = (int)(a >> 23) - 127;
    uint32_t m23 = (a & 0x7fffffu) | 0x800000u, code;
    if (e >= -6) {
        uint32_t v = orc_rne_shift(m23, 20);
        if (v == 16) { v = 8; e++; }
        code = (e > 8) ? 0x7Eu : (((uint32_t)(e + 7) << 3) | (v & 7u));
    } else if (e >= -10) {
        code = orc_rne_shift(m23, 14 - e);
    } else {
        code = 0;
    }
    return (uint8_t)(sign | code);
}

/* c/gmhc.h:157-160 — numpy's numerically stable sigmoid */
float orc_sigmoid(float x) {
    float e = expf(-fabsf(x));
    return x >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
}

/* c/gmhc.h:165-185 — numpy pairwise summation order */
float orc_pw_sum(const float *a, size_t n) {
    if (!n) return 0.0f;
    if (n < 8) {
        float r = a[0];
        for (size_t i = 1; i < n; i++) r += a[i];
        return r;
    }
    if (n <= 128) {
        float r[8];
        size_t i;
        for (int j = 0; j < 8; j++) r[j] = a[j];
        for (i = 8; i + 8 <= n; i += 8)
            for (int j = 0; j < 8; j++) r[j] += a[i + (size_t)j];
        float s = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (; i < n; i++) s += a[i];
        return s;
    }
    size_t n2 = (n / 2) & ~(size_t)7;
    return orc_pw_sum(a, n2) + orc_pw_sum(a + n2, n - n2);
}

/* ---------------------------------------------------------- linear leaf */

/* c/fp8blk.h:115-136 — one fp32 multiply, then BF16 RNE */
void orc_fp8_dequant(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K) {
    size_t nkb = (K + 127) / 128;
    for (size_t o = 0; o < O; o++)
        for (size_t k = 0; k < K; k++)
            out[o * K + k] = orc_bf16_bits(orc_e4m3_f32(w[o * K + k]) * ws[(o / 128) * nkb + k / 128]);
}

/* c/bf16.h:202-217 — fp32 accumulate from +0, strictly ascending k */
void orc_bf16_gemm_f32(const uint16_t *w, const uint16_t *x, float *y, size_t M, size_t O, size_t K) {
    for (size_t m = 0; m < M; m++)
        for (size_t o = 0; o < O; o++) {
            const uint16_t *wr = w + o * K, *xr = x + m * K;
            float acc = 0.0f;
            for (size_t k = 0; k < K; k++) acc += orc_bf16_f32(wr[k]) * orc_bf16_f32(xr[k]);
            y[m * O + o] = acc;
        }
}

void orc_bf16_gemm(const uint16_t *w, const uint16_t *x, uint16_t *y, size_t M, size_t O, size_t K) {
    for (size_t m = 0; m < M; m++)
        for (size_t o = 0; o < O; o++) {
            const uint16_t *wr = w + o * K, *xr = x + m * K;
            float acc = 0.0f;
            for (size_t k = 0; k < K; k++) acc += orc_bf16_f32(wr[k]) * orc_bf16_f32(xr[k]);
            y[m * O + o] = orc_bf16_bits(acc);
        }
}

/* c/gdsa.h:525-534 — dequant -> BF16 -> BF16 GEMM */
void orc_fp8_linear(const uint8_t *codes, const float *scales, const uint16_t *x, uint16_t *y,
                    size_t M, size_t O, size_t K) {
    uint16_t *wb = (uint16_t *)malloc(O * K * sizeof(uint16_t));
    orc_fp8_dequant(codes, scales, wb, O, K);
    orc_bf16_gemm(wb, x, y, M, O, K);
    free(wb);
}

/* c/sample.h:76-81 over widened BF16 codes: strict >, lowest index wins */
int orc_argmax_bf16(const uint16_t *logits, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
        if (orc_bf16_f32(logits[i]) > orc_bf16_f32(logits[best])) best = i;
    return (int)best;
}
