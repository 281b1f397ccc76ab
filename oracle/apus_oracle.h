/*
 * apus_oracle.h — CPU restatement of the apus GLM-5.3-Flash speculative
 * decode path, used ONLY as the checker for the CUDA path (tests, smoke,
 * the bench's CPU-baseline leg).  It is not part of the product: nothing in
 * libapus_gcuda.so calls it.
 *
 * Each function restates one reference function (cited file:line, paths
 * inside the apus repository).  The arithmetic keeps the reference's
 * rounding points and summation orders, so with an identical libm expf the
 * outputs are bitwise those of the reference; oracle/ref_glue.c lets the
 * tests prove that against the reference sources themselves.
 */
#ifndef APUS_ORACLE_H
#define APUS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numerics (c/num.h:110-166) ---- */
float    orc_bf16_f32(uint16_t b);
uint16_t orc_bf16_bits(float x);
float    orc_bf16_round(float x);
float    orc_e4m3_f32(uint8_t c);
uint8_t  orc_e4m3_quant(float x);
float    orc_sigmoid(float x);                 /* c/gmhc.h:157-160 */
float    orc_pw_sum(const float *a, size_t n); /* c/gmhc.h:165-185 */

/* ---- linear leaf ---- */
void orc_fp8_dequant(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K);
void orc_bf16_gemm(const uint16_t *w, const uint16_t *x, uint16_t *y, size_t M, size_t O, size_t K);
void orc_bf16_gemm_f32(const uint16_t *w, const uint16_t *x, float *y, size_t M, size_t O, size_t K);
void orc_fp8_linear(const uint8_t *codes, const float *scales, const uint16_t *x, uint16_t *y,
                    size_t M, size_t O, size_t K);
int  orc_argmax_bf16(const uint16_t *logits, size_t n);   /* c/sample.h:76-81 on widened codes */

/* ---- sampling (c/sample.h:91-177) ---- */
uint64_t orc_rng_next(uint64_t *s);                       /* splitmix64, c/sample.h:159-166 */
/* apus_sample_logits_u on the widened BF16 row (c/sample.h:134-157, :91-132) */
int orc_sample_logits_u(const uint16_t *logits, size_t n, float temp, float top_p, double u);
/* the same draw in the B200 sampler's exact arithmetic, u = u53 * 2^-53 */
int orc_sample_exact(const uint16_t *logits, size_t n, float temp, float top_p, uint64_t u53);

/* ---- chunked KDA prefill core (c/gkda.h:350-539 apus_gkda_chunk) ---- */
void orc_kda_chunk(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *g,
                   const uint16_t *beta, float *S, uint16_t *out, size_t s, size_t H, size_t D);

#ifdef __cplusplus
}
#endif
#endif
