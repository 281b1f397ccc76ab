/*
 * apus_oracle.c — CPU restatement of the apus speculative-decode path.
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels.  Built with
 * -ffp-contract=off like the reference (Makefile:27), so every a*b+c below
 * is two IEEE roundings.
 */
#include "apus_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>
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
/* Large loops over output rows are split over host threads: every output
 * element is still computed by one thread in the reference's order, so the
 * results do not depend on the thread count (ORC_THREADS, default: the
 * online cores). */
typedef void (*par_fn)(void *ctx, size_t i0, size_t i1);
typedef struct { par_fn fn; void *ctx; size_t i0, i1; } ParJob;

static void *par_run(void *a) {
    ParJob *j = (ParJob *)a;
    j->fn(j->ctx, j->i0, j->i1);
    return NULL;
}

static int par_threads(void) {
    static int n = 0;
    if (!n) {
        const char *e = getenv("ORC_THREADS");
        n = e ? atoi(e) : (int)sysconf(_SC_NPROCESSORS_ONLN);
        if (n < 1) n = 1;
        if (n > 64) n = 64;
    }
    return n;
}

static void par_for(size_t n, size_t work, par_fn fn, void *ctx) {
    int nt = par_threads();
    if (work < ((size_t)1 << 22) || nt < 2 || n < 2) { fn(ctx, 0, n); return; }
    if ((size_t)nt > n) nt = (int)n;
    pthread_t th[64];
    ParJob jb[64];
    for (int t = 0; t < nt; t++) {
        jb[t].fn = fn; jb[t].ctx = ctx;
        jb[t].i0 = n * (size_t)t / (size_t)nt;
        jb[t].i1 = n * (size_t)(t + 1) / (size_t)nt;
    }
    int started[64] = {0};
    for (int t = 1; t < nt; t++) started[t] = pthread_create(&th[t], NULL, par_run, &jb[t]) == 0;
    par_run(&jb[0]);
    for (int t = 1; t < nt; t++) {
        if (started[t]) pthread_join(th[t], NULL);
        else par_run(&jb[t]);
    }
}

typedef struct { const uint8_t *w; const float *ws; uint16_t *out; size_t K, nkb; } DeqCtx;

static void deq_rows(void *a, size_t o0, size_t o1) {
    DeqCtx *c = (DeqCtx *)a;
    for (size_t o = o0; o < o1; o++)
        for (size_t k = 0; k < c->K; k++)
            c->out[o * c->K + k] =
                orc_bf16_bits(orc_e4m3_f32(c->w[o * c->K + k]) * c->ws[(o / 128) * c->nkb + k / 128]);
}

void orc_fp8_dequant(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K) {
    DeqCtx c = {w, ws, out, K, (K + 127) / 128};
    par_for(O, O * K, deq_rows, &c);
}

/* c/bf16.h:202-217 — fp32 accumulate from +0, strictly ascending k */
typedef struct { const uint16_t *w, *x; float *yf; uint16_t *y; size_t M, O, K; } GemmCtx;

/* rows o0..o1 of W against every activation row; each output sums from +0
 * in strictly ascending k */
static void gemm_rows(void *a, size_t o0, size_t o1) {
    GemmCtx *c = (GemmCtx *)a;
    for (size_t m = 0; m < c->M; m++)
        for (size_t o = o0; o < o1; o++) {
            const uint16_t *wr = c->w + o * c->K, *xr = c->x + m * c->K;
            float acc = 0.0f;
            for (size_t k = 0; k < c->K; k++) acc += orc_bf16_f32(wr[k]) * orc_bf16_f32(xr[k]);
            if (c->yf) c->yf[m * c->O + o] = acc;
            else c->y[m * c->O + o] = orc_bf16_bits(acc);
        }
}

void orc_bf16_gemm_f32(const uint16_t *w, const uint16_t *x, float *y, size_t M, size_t O, size_t K) {
    GemmCtx c = {w, x, y, NULL, M, O, K};
    par_for(O, M * O * K, gemm_rows, &c);
}

void orc_bf16_gemm(const uint16_t *w, const uint16_t *x, uint16_t *y, size_t M, size_t O, size_t K) {
    GemmCtx c = {w, x, NULL, y, M, O, K};
    par_for(O, M * O * K, gemm_rows, &c);
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

/* --------------------------------------------------------------- sample */

/* splitmix64 (c/sample.h:159-170) */
uint64_t orc_rng_next(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static float *g_sort_p;   /* qsort comparator context (single-threaded checker) */

/* probability descending, exact ties by lower index (c/sample.h:97-110) */
static int cmp_prob_desc(const void *a, const void *b) {
    const int32_t i = *(const int32_t *)a, j = *(const int32_t *)b;
    const float pi = g_sort_p[i], pj = g_sort_p[j];
    if (pi > pj) return -1;
    if (pi < pj) return 1;
    return i < j ? -1 : (i > j ? 1 : 0);
}

/* c/sample.h:134-157 then :91-132 on the widened BF16 row: softmax of
 * logits/temp in fp32 with a double sum, nucleus by the HF shift rule,
 * renormalised CDF draw with u.  The sort is qsort on the same total order
 * as the reference's shell sort, so the permutation is the same. */
int orc_sample_logits_u(const uint16_t *logits, size_t n, float temp, float top_p, double u) {
    if (temp <= 0.0f) return orc_argmax_bf16(logits, n);
    float *p = (float *)malloc(n * sizeof(float));
    int32_t *ord = (int32_t *)malloc(n * sizeof(int32_t));
    float mx = orc_bf16_f32(logits[0]);
    for (size_t i = 1; i < n; i++)
        if (orc_bf16_f32(logits[i]) > mx) mx = orc_bf16_f32(logits[i]);
    double sum = 0.0;
    for (size_t i = 0; i < n; i++) {
        p[i] = expf((orc_bf16_f32(logits[i]) - mx) / temp);
        sum += p[i];
    }
    for (size_t i = 0; i < n; i++) p[i] = (float)(p[i] / sum);
    for (size_t i = 0; i < n; i++) ord[i] = (int32_t)i;
    g_sort_p = p;
    qsort(ord, n, sizeof(int32_t), cmp_prob_desc);
    double cum = 0.0, kept = 0.0;
    size_t nk = 0;
    for (size_t i = 0; i < n; i++) {
        if (cum <= (double)top_p) {
            cum += p[ord[i]];
            kept = cum;
            nk = i + 1;
        } else {
            break;
        }
    }
    if (nk == 0) { nk = 1; kept = p[ord[0]]; }
    int tok = ord[nk - 1];
    double c = 0.0;
    for (size_t i = 0; i < nk; i++) {
        c += (double)p[ord[i]] / kept;
        if (u < c) { tok = ord[i]; break; }
    }
    free(p);
    free(ord);
    return tok;
}

/* The same draw in the exact arithmetic the B200 sampler uses (the
 * bitwise checker of apus-glm5.3-flash_b200/csrc/sample.cu), computed here
 * element by element with a full sort instead of the kernel's key
 * histogram:
 *   p = e^z rounded to float, e^z by a Cody-Waite reduction by ln 2 and
 *       the degree-13 Taylor polynomial in double (one rounding per op);
 *   sum = the exact sum of p at 2^-100 resolution, rounded once to double;
 *   q = (float)(p / sum) as the reference;
 *   cumulative masses exact in integers of 2^-62; nucleus = through the
 *   first sorted token whose cumulative mass exceeds floor(top_p * 2^62);
 *   draw = the first sorted token whose cumulative mass exceeds
 *   floor(u53 * kept / 2^53), u = u53 * 2^-53. */
typedef unsigned __int128 orc_u128;

static double orc_exp_cw(double z) {
    static const double c[14] = {1.0, 1.0, 0x1.0p-1, 0x1.5555555555555p-3, 0x1.5555555555555p-5,
                                 0x1.1111111111111p-7, 0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13,
                                 0x1.a01a01a01a01ap-16, 0x1.71de3a556c734p-19, 0x1.27e4fb7789f5cp-22,
                                 0x1.ae64567f544e4p-26, 0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33};
    const double inv_ln2 = 0x1.71547652b82fep+0, ln2_hi = 0x1.62e42fee00000p-1, ln2_lo = 0x1.a39ef35793c76p-33;
    const double k = rint(z * inv_ln2);
    const double r = (z - k * ln2_hi) - k * ln2_lo;
    double e = c[13];
    for (int i = 12; i >= 0; i--) e = e * r + c[i];
    const uint64_t kb = (uint64_t)((int64_t)k + 1023) << 52;
    double s;
    memcpy(&s, &kb, 8);
    return e * s;
}

static float orc_smp_p(float l, float mx, float temp) {
    const float z = (l - mx) / temp;
    if (!(z >= -105.0f)) return 0.0f;
    return (float)orc_exp_cw((double)z);
}

static void orc_float_parts(float v, uint64_t *M, int *E) {
    uint32_t b;
    memcpy(&b, &v, 4);
    const uint32_t e = b >> 23;
    *M = b & 0x7FFFFFu;
    *E = -149;
    if (e) { *M |= 0x800000u; *E = (int)e - 150; }
}

static uint64_t orc_fix62(float v) {
    uint64_t M;
    int E;
    orc_float_parts(v, &M, &E);
    const int s = E + 62;
    return s >= 0 ? M << s : (s > -64 ? M >> -s : 0);
}

static orc_u128 orc_fix100(float v) {
    uint64_t M;
    int E;
    orc_float_parts(v, &M, &E);
    const int s = E + 100;
    return s >= 0 ? (orc_u128)M << s : (orc_u128)(s > -64 ? M >> -s : 0);
}

static double orc_u128_scaled_rn(orc_u128 x) {
    if (x < ((orc_u128)1 << 53)) return (double)(uint64_t)x * 0x1.0p-100;
    int nb = 0;
    for (orc_u128 t = x; t; t >>= 1) nb++;
    const int sh = nb - 53;
    orc_u128 mant = x >> sh;
    const orc_u128 rem = x - (mant << sh), half = (orc_u128)1 << (sh - 1);
    if (rem > half || (rem == half && (mant & 1))) mant += 1;
    return ldexp((double)(uint64_t)mant, sh - 100);
}

static uint64_t *g_sort_f;
static float *g_sort_q;

static int cmp_q_desc(const void *a, const void *b) {
    const int32_t i = *(const int32_t *)a, j = *(const int32_t *)b;
    const float qi = g_sort_q[i], qj = g_sort_q[j];
    if (qi > qj) return -1;
    if (qi < qj) return 1;
    return i < j ? -1 : (i > j ? 1 : 0);
}

int orc_sample_exact(const uint16_t *logits, size_t n, float temp, float top_p, uint64_t u53) {
    if (!(temp > 0.0f)) return orc_argmax_bf16(logits, n);
    float *q = (float *)malloc(n * sizeof(float));
    uint64_t *f = (uint64_t *)malloc(n * sizeof(uint64_t));
    int32_t *ord = (int32_t *)malloc(n * sizeof(int32_t));
    float mx = orc_bf16_f32(logits[0]);
    for (size_t i = 1; i < n; i++)
        if (orc_bf16_f32(logits[i]) > mx) mx = orc_bf16_f32(logits[i]);
    orc_u128 acc = 0;
    for (size_t i = 0; i < n; i++) {
        q[i] = orc_smp_p(orc_bf16_f32(logits[i]), mx, temp);
        acc += orc_fix100(q[i]);
    }
    const double S = orc_u128_scaled_rn(acc);
    uint64_t total = 0;
    for (size_t i = 0; i < n; i++) {
        q[i] = (float)((double)q[i] / S);
        f[i] = orc_fix62(q[i]);
        total += f[i];
        ord[i] = (int32_t)i;
    }
    g_sort_q = q;
    g_sort_f = f;
    qsort(ord, n, sizeof(int32_t), cmp_q_desc);
    const uint64_t TP = !(top_p >= 0.0f) ? 0 : (top_p >= 4.0f ? ~0ull : (uint64_t)((double)top_p * 0x1.0p62));
    uint64_t kept = total, cum = 0;
    for (size_t i = 0; i < n; i++) {
        if (cum + f[ord[i]] > TP) { kept = cum + f[ord[i]]; break; }
        cum += f[ord[i]];
    }
    const uint64_t X = (uint64_t)(((orc_u128)u53 * kept) >> 53);
    int tok = ord[0];
    cum = 0;
    for (size_t i = 0; i < n; i++) {
        cum += f[ord[i]];
        if (cum > X) { tok = ord[i]; break; }
    }
    free(q);
    free(f);
    free(ord);
    return tok;
}

/* ------------------------------------------------------------ chunked KDA */

/* c/gkda.h:350-539 apus_gkda_chunk (the chunked delta rule, chunks of 64):
 * per head, rows l2-normalised (numpy pairwise sum of squares), q scaled by
 * D^-1/2, k and v weighted by beta; the gate summed within each chunk; the
 * strictly-lower attn with per-dimension decay, its UT transform row by row
 * (+ I after the whole solve); value, kcd, v_new, inter, intra, the output
 * rows and the state update, every sum ascending from +0.  Rows past s are
 * zero.  S [H*D*D] fp32 in/out. */
#define ORC_KDA_C 64
void orc_kda_chunk(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *g,
                   const uint16_t *beta, float *S, uint16_t *out, size_t s, size_t H, size_t D) {
    const size_t C = ORC_KDA_C, pad = (C - s % C) % C, sp = s + pad, N = sp / C, hd = H * D;
    const float qscale = (float)pow((double)D, -0.5);
    float *qp = calloc(sp * D, 4), *kp = calloc(sp * D, 4), *gc = calloc(sp * D, 4);
    float *kb = calloc(sp * D, 4), *vb = calloc(sp * D, 4), *sq = malloc(D * 4);
    float *attn = malloc(C * C * 4), *intra = malloc(C * C * 4), *value = malloc(C * D * 4);
    float *kcd = malloc(C * D * 4), *vnew = malloc(C * D * 4), *inter = malloc(C * D * 4);
    for (size_t h = 0; h < H; h++) {
        memset(qp, 0, sp * D * 4); memset(kp, 0, sp * D * 4); memset(gc, 0, sp * D * 4);
        memset(kb, 0, sp * D * 4); memset(vb, 0, sp * D * 4);
        for (size_t t = 0; t < s; t++) {
            float *rows[2] = {qp + t * D, kp + t * D};
            const uint16_t *src[2] = {q + t * hd + h * D, k + t * hd + h * D};
            for (int w = 0; w < 2; w++) {
                for (size_t d = 0; d < D; d++) {
                    rows[w][d] = orc_bf16_f32(src[w][d]);
                    sq[d] = rows[w][d] * rows[w][d];
                }
                const float root = sqrtf(orc_pw_sum(sq, D) + 1e-6f);
                for (size_t d = 0; d < D; d++) rows[w][d] = rows[w][d] / root;
            }
            const float bt = orc_bf16_f32(beta[t * H + h]);
            for (size_t d = 0; d < D; d++) {
                qp[t * D + d] = qp[t * D + d] * qscale;
                gc[t * D + d] = g[t * hd + h * D + d];
                kb[t * D + d] = kp[t * D + d] * bt;
                vb[t * D + d] = orc_bf16_f32(v[t * hd + h * D + d]) * bt;
            }
        }
        for (size_t n = 0; n < N; n++)
            for (size_t i = 1; i < C; i++)
                for (size_t d = 0; d < D; d++)
                    gc[(n * C + i) * D + d] = gc[(n * C + i - 1) * D + d] + gc[(n * C + i) * D + d];
        float *Sh = S + h * D * D;
        for (size_t n = 0; n < N; n++) {
            const float *qc = qp + n * C * D, *kc = kp + n * C * D, *gn = gc + n * C * D;
            const float *kbc = kb + n * C * D, *vbc = vb + n * C * D;
            memset(attn, 0, C * C * 4);
            memset(intra, 0, C * C * 4);
            for (size_t i = 0; i < C; i++)
                for (size_t j = 0; j <= i; j++) {
                    float a = 0.0f, b = 0.0f;
                    for (size_t d = 0; d < D; d++) {
                        const float dec = expf(gn[i * D + d] - gn[j * D + d]);
                        a += (kbc[i * D + d] * kc[j * D + d]) * dec;
                        b += (qc[i * D + d] * kc[j * D + d]) * dec;
                    }
                    if (j < i) attn[i * C + j] = -a;
                    intra[i * C + j] = b;
                }
            for (size_t i = 1; i < C; i++)
                for (size_t j = 0; j < i; j++) {
                    float a = 0.0f;
                    for (size_t m = 0; m < i; m++) a += attn[i * C + m] * attn[m * C + j];
                    attn[i * C + j] = attn[i * C + j] + a;
                }
            for (size_t i = 0; i < C; i++) attn[i * C + i] = attn[i * C + i] + 1.0f;
            for (size_t i = 0; i < C; i++)
                for (size_t d = 0; d < D; d++) {
                    float a = 0.0f, b = 0.0f;
                    for (size_t j = 0; j < C; j++) {
                        a += attn[i * C + j] * vbc[j * D + d];
                        b += attn[i * C + j] * (kbc[j * D + d] * expf(gn[j * D + d]));
                    }
                    value[i * D + d] = a;
                    kcd[i * D + d] = b;
                }
            for (size_t i = 0; i < C; i++)
                for (size_t c = 0; c < D; c++) {
                    float a = 0.0f, b = 0.0f;
                    for (size_t d = 0; d < D; d++) {
                        b += (qc[i * D + d] * expf(gn[i * D + d])) * Sh[d * D + c];
                        a += kcd[i * D + d] * Sh[d * D + c];
                    }
                    inter[i * D + c] = b;
                    vnew[i * D + c] = value[i * D + c] - a;
                }
            for (size_t i = 0; i < C && n * C + i < s; i++)
                for (size_t c = 0; c < D; c++) {
                    float a = 0.0f;
                    for (size_t j = 0; j < C; j++) a += intra[i * C + j] * vnew[j * D + c];
                    out[(n * C + i) * hd + h * D + c] = orc_bf16_bits(inter[i * D + c] + a);
                }
            const float *gl = gn + (C - 1) * D;
            for (size_t m = 0; m < D; m++) {
                const float egl = expf(gl[m]);
                for (size_t c = 0; c < D; c++) {
                    float a = 0.0f;
                    for (size_t j = 0; j < C; j++) a += (kc[j * D + m] * expf(gl[m] - gn[j * D + m])) * vnew[j * D + c];
                    Sh[m * D + c] = Sh[m * D + c] * egl + a;
                }
            }
        }
    }
    free(qp); free(kp); free(gc); free(kb); free(vb); free(sq);
    free(attn); free(intra); free(value); free(kcd); free(vnew); free(inter);
}
