/*
 * apus_gcuda.h — C ABI of the B200 (sm_100a) backend for the apus
 * GLM-5.3-Flash engine: the linear-layer leaf (FP8 128x128 block dequant,
 * FP8/BF16 decode GEMV) behind the reference's own entry points.
 *
 * Drop-in rules:
 *   - Host-pointer entry points keep the reference signatures exactly, so a C
 *     engine that stops compiling the CPU implementation of c/fp8blk.h /
 *     c/bf16.h and links libapus_gcuda.so instead runs unchanged.
 *   - The hook-table entries have the signatures of ApusGmetalHooks
 *     (c/backend_gmetal.h:120-126): 0 = handled, nonzero = not handled.
 *   - `_dev` twins take device pointers plus a cudaStream_t passed as void*.
 *   - No CPU fallback: when the CUDA path cannot run, entry points return
 *     nonzero (or, for the void reference signatures, record the error in
 *     apus_gcuda_last_error() and leave the output untouched).
 * Numerics: dequant is bitwise c/fp8blk.h; GEMV rows are the reference
 * dequant->BF16->fp32-accumulate->BF16 composition with a different (fixed,
 * row-count independent) fp32 summation order.
 */
#ifndef APUS_GCUDA_H
#define APUS_GCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- backend control (mirrors c/backend_gmetal.h:131-156) --------------- */

/* Initialise the CUDA device (must be sm_100). 0 on success, -1 + err. */
int  apus_gcuda_enable(char *err, size_t errcap);        /* c/backend_gmetal.h:134 */
void apus_gcuda_disable(void);                           /* c/backend_gmetal.h:136 */
int  apus_gcuda_is_enabled(void);                        /* c/backend_gmetal.h:137 */
/* Last error message of the calling thread ("" when none); the message
 * stays until the next failure or apus_gcuda_clear_error. */
const char *apus_gcuda_last_error(void);
void apus_gcuda_clear_error(void);
/* Device-side error word of the pipelined kernels (0 = none; nonzero = a
 * bounded wait gave up: 1 producer, 2 consumer), read and cleared.
 * Synchronises the device. */
int apus_gcuda_kernel_error(void);

/* Persistent HBM residency for a model-owned host weight region: the bytes
 * are uploaded once; hooked ops whose weight pointer lies inside a
 * registered region read the resident copy (c/backend_gmetal.h:147-148). */
int  apus_gcuda_register_region(const void *ptr, size_t len);
void apus_gcuda_unregister_region(const void *ptr);
uint64_t apus_gcuda_bytes_pinned(void);                  /* c/backend_gmetal.h:154 */
uint64_t apus_gcuda_dispatches(void);                    /* c/backend_gmetal.h:155 */
uint64_t apus_gcuda_offload_bf16(void);                  /* c/backend_gmetal.h:156 */
uint64_t apus_gcuda_offload_fp8blk(void);                /* c/backend_gmetal.h:157 */

/* Hook table with the layout of ApusGmetalHooks (c/backend_gmetal.h:120-126). */
typedef struct {
    int (*bf16_gemm)(const uint16_t *w, const uint16_t *x, uint16_t *y,
                     size_t M, size_t O, size_t K);
    int (*fp8blk_linear)(const uint8_t *codes, const float *scales,
                         const uint16_t *x, uint16_t *y,
                         size_t M, size_t O, size_t K);
} ApusGcudaHooks;
void apus_gcuda_fill_hooks(ApusGcudaHooks *out);

/* Direct hook entries (c/backend_gmetal.h:163-167): host pointers, any M. */
int apus_gcuda_bf16_gemm(const uint16_t *w, const uint16_t *x, uint16_t *y,
                         size_t M, size_t O, size_t K);
int apus_gcuda_fp8blk_linear(const uint8_t *codes, const float *scales,
                             const uint16_t *x, uint16_t *y,
                             size_t M, size_t O, size_t K);

/* ---- c/fp8blk.h drop-ins ------------------------------------------------- */
size_t apus_fp8blk_nblocks(size_t n);                    /* c/fp8blk.h:63 */
void apus_fp8blk_dequant(const uint8_t *w, const float *ws,
                         uint16_t *out, size_t O, size_t K);   /* c/fp8blk.h:81-82 */
void apus_fp8blk_dequant_mt(const uint8_t *w, const float *ws,
                            uint16_t *out, size_t O, size_t K); /* c/fp8blk.h:88-89 */

/* ---- c/bf16.h drop-ins (xf scratch is accepted and unused) --------------- */
void apus_bf16_gemv_mt(const uint16_t *w, const uint16_t *x, float *xf,
                       uint16_t *y, size_t O, size_t K);       /* c/bf16.h:146-147 */
void apus_bf16_gemm_mt(const uint16_t *w, const uint16_t *x, float *xf,
                       uint16_t *y, size_t M, size_t O, size_t K); /* c/bf16.h:150-151 */

/* ---- device-pointer twins ------------------------------------------------ */
/* Launch the `_dev` linears as programmatic dependents of the previous kernel
 * in the stream (their weight stream starts while it drains).  Only safe when
 * no kernel immediately before a linear writes that linear's weights. Off by
 * default. */
void apus_gcuda_set_pdl(int on);
int apus_fp8blk_dequant_dev(const uint8_t *w, const float *ws, uint16_t *out,
                            size_t O, size_t K, void *stream);
/* y [M,O] BF16 codes; M <= 8 per launch (larger M is split into 8-row
 * launches, each row bitwise independent of the others). */
int apus_gcuda_fp8blk_linear_dev(const uint8_t *codes, const float *scales,
                                 const uint16_t *x, uint16_t *y,
                                 size_t M, size_t O, size_t K, void *stream);
int apus_gcuda_bf16_gemm_dev(const uint16_t *w, const uint16_t *x, uint16_t *y,
                             size_t M, size_t O, size_t K, void *stream);
/* fp32 output, no rounding (router logits c/gmoe.h:168-173, mHC mixes
 * c/gmhc.h:250-258). */
int apus_gcuda_bf16_gemm_f32_dev(const uint16_t *w, const uint16_t *x, float *y,
                                 size_t M, size_t O, size_t K, void *stream);
/* BF16 GEMV fused with the greedy pick of c/sample.h:76-81 on the
 * BF16-rounded outputs (lowest index wins ties): ids [M]; y (optional) gets
 * the BF16 logits. */
int apus_gcuda_bf16_gemm_argmax_dev(const uint16_t *w, const uint16_t *x, uint16_t *y,
                                    int32_t *ids, size_t M, size_t O, size_t K,
                                    void *stream);
/* No counterpart in the reference.  The same fused GEMV + greedy pick with
 * its scratch (keys, split-K partials and tickets) in a fixed 4 MiB
 * file-scope device array instead of the grow-only pool, for callers that
 * may not call cudaMalloc/cudaFree (an HBM budget already handed out, or
 * streams that cannot take the implied device synchronisation).  Limits:
 * M <= 64 and O, K whose split-K scratch fits the array.  Split-K scratch
 * is only needed when the shape splits K (a function of O and K: small O
 * splits even a K of 2048); every K <= 4096 fits, and K = 8192 fits O up to
 * about 65,000.  Larger shapes return -1 with the reason in
 * apus_gcuda_last_error().  The first call on a device sets up the array's
 * address (make it before any stream capture).  Calls that overlap in time
 * share the array and race; serialising them is the caller's job, while the
 * library's own per-device set-up (kernel attributes, SM count) is
 * thread-safe.  Outputs are bitwise those of
 * apus_gcuda_bf16_gemm_argmax_dev. */
int apus_gcuda_bf16_gemm_argmax_static_dev(const uint16_t *w, const uint16_t *x, uint16_t *y,
                                           int32_t *ids, size_t M, size_t O, size_t K,
                                           void *stream);
/* c/sample.h:63 apus_sample over `rows` BF16 logits rows (device, row r at
 * logits + r*ld): row r is drawn with the (r+1)-th splitmix64 uniform after
 * rng_state, as if apus_sample were called on the rows in order with an
 * ApusRng holding rng_state (the caller advances its state by `rows`).
 * temp <= 0: the lowest-index argmax, no uniform.  temp > 0: softmax of
 * logits/temp, nucleus top_p (c/sample.h:91-132), CDF draw, computed in exact
 * integer arithmetic for the cumulative masses and a correctly rounded exp
 * (the token is the reference's unless u * kept or top_p lies within about
 * 1e-7 of a cumulative-mass boundary).  n <= 256000, ld >= n; ids [rows]. */
int apus_gcuda_sample_rows_dev(const uint16_t *logits, size_t rows, size_t ld, size_t n, float temp,
                               float top_p, uint64_t rng_state, int32_t *out, void *stream);
/* c/gkda.h:140-143 apus_gkda_chunk (the chunked KDA prefill core, chunks of
 * 64 rows): q/k/v [s, H*D] BF16 codes (post-conv), g [s, H*D] fp32, beta
 * [s, H] BF16 codes, S [H*D*D] fp32 in/out, out [s, H*D] BF16 codes, all
 * device pointers.  Each head's sums run in the reference's order; results
 * differ from it only through expf's last bits.  D must be 128. */
int apus_gcuda_kda_chunk_dev(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *g,
                             const uint16_t *beta, float *S, uint16_t *out, size_t s, size_t H, size_t D,
                             void *stream);

#ifdef __cplusplus
}
#endif

#endif /* APUS_GCUDA_H */
