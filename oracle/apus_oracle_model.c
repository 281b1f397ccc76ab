/*
 * apus_oracle_model.c — CPU restatement of the apus decode stack.
 * TEST INFRASTRUCTURE ONLY (the checker of the CUDA engine).  Compiled with
 * -ffp-contract=off; every rounding point and summation order follows the
 * cited reference function.
 */
#include "apus_oracle_model.h"
#include "apus_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define NEG_INF (-3.4028234663852886e+38f)   /* c/gdsa.h:91 */

typedef struct { const uint8_t *c; const float *s; } Fp8;

typedef struct {
    const uint16_t *input_norm, *post_norm;
    const uint16_t *hc_fn[2];
    const float *hc_base[2], *hc_scale[2];
    /* KDA */
    const uint16_t *q_w, *k_w, *v_w, *conv[3], *f_a, *f_b, *b_w, *g_a, *g_b, *o_norm, *o_w;
    const float *A_log, *dt_bias;
    /* DSA */
    Fp8 q_a, q_b, kv_a, o;
    const uint16_t *q_a_norm, *kv_a_norm, *kv_b;
    const uint16_t *idx_wq_b, *idx_wk, *idx_knorm_w, *idx_knorm_b, *idx_wproj, *idx_ape, *idx_gate;
    /* MLP */
    Fp8 mlp_g, mlp_u, mlp_d;
    const uint16_t *gate_w;
    const float *gate_bias;
    Fp8 *eg, *eu, *ed;
    Fp8 sg, su, sd;
    /* MTP glue */
    const uint16_t *enorm, *hnorm, *eh_proj, *shared_norm;
} OLayer;

typedef struct { const uint8_t *c; uint16_t *deq; } DeqEntry;

struct OrcModel {
    OrcConfig c;
    int has_mtp;
    OLayer *L;                       /* [num_hidden_layers + has_mtp] */
    const uint16_t *embed, *norm, *head;
    /* BF16 copies of the FP8 matrices, made on first use (the reference
     * engine likewise holds dequantized experts, c/gmodel.h:1003-1073); the
     * arithmetic is orc_fp8_dequant's either way */
    DeqEntry *deq;
    size_t ndeq, capdeq;
};

typedef struct {
    uint16_t *k, *v, *ik, *ig;
    size_t cap, n;
} ODsa;

struct OrcState {
    const OrcModel *m;
    size_t pos, cap;
    uint16_t **conv;                 /* [L] KDA conv states */
    float **rec;                     /* [L] KDA recurrent states */
    ODsa *dsa;                       /* [L] */
};

struct OrcMtpState {
    size_t cap, pos;
    ODsa dsa;
};

/* ------------------------------------------------------------ helpers */

static void *xc(size_t n) { void *p = calloc(n ? n : 1, 1); if (!p) abort(); return p; }
static size_t kda_bytes(const OrcConfig *c, int rec);

static void gemm(const uint16_t *w, const uint16_t *x, uint16_t *y, size_t M, size_t O, size_t K) {
    orc_bf16_gemm(w, x, y, M, O, K);
}

static const uint16_t *deq_of(const OrcModel *cm, Fp8 w, size_t O, size_t K) {
    OrcModel *m = (OrcModel *)cm;
    size_t h = ((uintptr_t)w.c >> 4) * 0x9E3779B97F4A7C15ull;
    if (m->capdeq) {
        for (size_t i = h % m->capdeq;; i = (i + 1) % m->capdeq) {
            if (!m->deq[i].c) break;
            if (m->deq[i].c == w.c) return m->deq[i].deq;
        }
    }
    if (2 * (m->ndeq + 1) > m->capdeq) {   /* grow and rehash */
        size_t nc = m->capdeq ? 2 * m->capdeq : 256;
        DeqEntry *nt = xc(nc * sizeof *nt);
        for (size_t j = 0; j < m->capdeq; j++) {
            if (!m->deq[j].c) continue;
            size_t i = (((uintptr_t)m->deq[j].c >> 4) * 0x9E3779B97F4A7C15ull) % nc;
            while (nt[i].c) i = (i + 1) % nc;
            nt[i] = m->deq[j];
        }
        free(m->deq);
        m->deq = nt;
        m->capdeq = nc;
    }
    uint16_t *b = malloc(O * K * 2);
    if (!b) abort();
    orc_fp8_dequant(w.c, w.s, b, O, K);
    size_t i = h % m->capdeq;
    while (m->deq[i].c) i = (i + 1) % m->capdeq;
    m->deq[i].c = w.c;
    m->deq[i].deq = b;
    m->ndeq++;
    return b;
}

/* c/gdsa.h:525-534 fp8_linear: dequant -> BF16 -> BF16 GEMM */
static void fp8lin(const OrcModel *m, Fp8 w, const uint16_t *x, uint16_t *y, size_t M, size_t O, size_t K) {
    orc_bf16_gemm(deq_of(m, w, O, K), x, y, M, O, K);
}

/* c/gdsa.h:258-274 — weighted RMSNorm: f32 pairwise mean, bf16 round, x w */
void orc_rmsnorm(const uint16_t *x, const uint16_t *w, uint16_t *y, size_t n, float eps) {
    float *sq = xc(n * 4), *xf = xc(n * 4);
    for (size_t i = 0; i < n; i++) { xf[i] = orc_bf16_f32(x[i]); sq[i] = xf[i] * xf[i]; }
    float var = orc_pw_sum(sq, n) / (float)n;
    float inv = 1.0f / sqrtf(var + eps);
    for (size_t i = 0; i < n; i++) {
        float t = orc_bf16_round(xf[i] * inv);
        y[i] = orc_bf16_bits(orc_bf16_f32(w[i]) * t);
    }
    free(xf); free(sq);
}

/* c/gdsa.h:276-305 — LayerNorm, pairwise mean/var, one bf16 rounding */
void orc_layernorm(const uint16_t *x, const uint16_t *w, const uint16_t *b, uint16_t *y,
                   size_t n, float eps) {
    float *xf = xc(n * 4), *d = xc(n * 4), *sq = xc(n * 4);
    for (size_t i = 0; i < n; i++) xf[i] = orc_bf16_f32(x[i]);
    float mu = orc_pw_sum(xf, n) / (float)n;
    for (size_t i = 0; i < n; i++) { d[i] = xf[i] - mu; sq[i] = d[i] * d[i]; }
    float var = orc_pw_sum(sq, n) / (float)n;
    float inv = 1.0f / sqrtf(var + eps);
    for (size_t i = 0; i < n; i++) {
        float t = d[i] * inv;
        t = t * orc_bf16_f32(w[i]) + orc_bf16_f32(b[i]);
        y[i] = orc_bf16_bits(t);
    }
    free(sq); free(d); free(xf);
}

/* ---------------------------------------------------------------- mHC */

/* c/gmhc.h:225-232 Sinkhorn-20 with the reference's eps placement */
static void sinkhorn(float *c, size_t n, int iters, float eps) {
    for (size_t j = 0; j < n; j++) {                       /* :197-206 */
        float *r = c + j * n, mx = r[0];
        for (size_t k = 1; k < n; k++) if (r[k] > mx) mx = r[k];
        for (size_t k = 0; k < n; k++) r[k] = expf(r[k] - mx);
        float sum = orc_pw_sum(r, n);
        for (size_t k = 0; k < n; k++) r[k] = r[k] / sum + eps;
    }
    for (int it = 0; it < iters; it++) {
        if (it) {                                          /* :208-214 rows */
            for (size_t j = 0; j < n; j++) {
                float *r = c + j * n, den = orc_pw_sum(r, n) + eps;
                for (size_t k = 0; k < n; k++) r[k] /= den;
            }
        }
        for (size_t k = 0; k < n; k++) {                   /* :216-223 cols */
            float sum = c[k];
            for (size_t j = 1; j < n; j++) sum += c[j * n + k];
            float den = sum + eps;
            for (size_t j = 0; j < n; j++) c[j * n + k] /= den;
        }
    }
}

/* c/gmhc.h:234-276 maps + collapse; fn is the BF16 [mix, n*d] tensor
 * (widened exactly, as c/gmodel.h:716-729 does at load). */
void orc_hc_pre(const OrcModel *m, int layer, int ffn, const uint16_t *h4, uint16_t *x,
                float *post, float *comb) {
    const OrcConfig *c = &m->c;
    const OLayer *Ly = &m->L[layer];
    size_t n = (size_t)c->hc_mult, d = (size_t)c->hidden_size, nx = n * d, nmix = (2 + n) * n;
    const uint16_t *fn = Ly->hc_fn[ffn];
    const float *scale = Ly->hc_scale[ffn], *base = Ly->hc_base[ffn];
    float *x4 = xc(nx * 4), *flat = xc(nx * 4), *sq = xc(nx * 4), *mix = xc(nmix * 4), pre[16];
    for (size_t i = 0; i < nx; i++) { x4[i] = orc_bf16_f32(h4[i]); sq[i] = x4[i] * x4[i]; }
    float var = orc_pw_sum(sq, nx) / (float)nx;            /* :187-195 */
    float inv = 1.0f / sqrtf(var + c->rms_norm_eps);
    for (size_t i = 0; i < nx; i++) flat[i] = x4[i] * inv;
    for (size_t j = 0; j < nmix; j++) {                    /* :250-258 */
        float acc = 0.0f;
        for (size_t i = 0; i < nx; i++) acc += orc_bf16_f32(fn[j * nx + i]) * flat[i];
        mix[j] = acc;
    }
    for (size_t j = 0; j < n; j++)
        pre[j] = orc_sigmoid(mix[j] * scale[0] + base[j]) + c->hc_eps;
    for (size_t j = 0; j < n; j++)
        post[j] = 2.0f * orc_sigmoid(mix[n + j] * scale[1] + base[n + j]);
    for (size_t j = 0; j < n; j++)
        for (size_t k = 0; k < n; k++) {
            size_t idx = 2 * n + j * n + k;
            comb[j * n + k] = mix[idx] * scale[2] + base[idx];
        }
    sinkhorn(comb, n, c->hc_sinkhorn_iters, c->hc_eps);
    for (size_t i = 0; i < d; i++) {                       /* :267-276 */
        float acc = pre[0] * x4[i];
        for (size_t j = 1; j < n; j++) acc += pre[j] * x4[j * d + i];
        x[i] = orc_bf16_bits(acc);
    }
    free(mix); free(sq); free(flat); free(x4);
}

/* c/gmhc.h:278-294 expand */
void orc_hc_post(const uint16_t *x, const uint16_t *res4, const float *post, const float *comb,
                 uint16_t *y4, size_t d, size_t n) {
    for (size_t j = 0; j < n; j++) {
        float pb = orc_bf16_round(post[j]);
        for (size_t i = 0; i < d; i++) {
            float t1 = orc_bf16_round(pb * orc_bf16_f32(x[i]));
            float acc = 0.0f;
            for (size_t k = 0; k < n; k++)
                acc += orc_bf16_round(comb[k * n + j]) * orc_bf16_f32(res4[k * d + i]);
            y4[j * d + i] = orc_bf16_bits(t1 + orc_bf16_round(acc));
        }
    }
}

/* c/gmhc.h:296-304 HyperHead mean */
void orc_hc_head(const uint16_t *x4, uint16_t *y, size_t d, size_t n) {
    for (size_t i = 0; i < d; i++) {
        float acc = orc_bf16_f32(x4[i]);
        for (size_t j = 1; j < n; j++) acc += orc_bf16_f32(x4[j * d + i]);
        y[i] = orc_bf16_bits(acc / (float)n);
    }
}

/* ---------------------------------------------------------------- MoE */

/* c/gmoe.h:175-189 */
static void topk_stable(const float *row, int n, int k, int32_t *idx) {
    for (int j = 0; j < k; j++) {
        int best = -1;
        for (int i = 0; i < n; i++) {
            int used = 0;
            for (int q = 0; q < j; q++) if (idx[q] == i) { used = 1; break; }
            if (used) continue;
            if (best < 0 || row[i] > row[best]) best = i;
        }
        idx[j] = best;
    }
}

/* c/gmoe.h:191-208 */
/* the last router call's gap between the topk-th and the next biased
 * score (how close its selection came to a tie); test inspection only */
static float g_route_gap;

static void router(const OrcModel *m, const OLayer *Ly, const uint16_t *x, int32_t *idx, float *w) {
    const OrcConfig *c = &m->c;
    int E = c->n_routed_experts, topk = c->num_experts_per_tok;
    size_t d = (size_t)c->hidden_size;
    float *scores = xc((size_t)E * 4), *b = xc((size_t)E * 4);
    for (int e = 0; e < E; e++) {
        float acc = 0.0f;
        for (size_t i = 0; i < d; i++)
            acc += orc_bf16_f32(Ly->gate_w[(size_t)e * d + i]) * orc_bf16_f32(x[i]);
        scores[e] = orc_sigmoid(acc);
        b[e] = scores[e] + Ly->gate_bias[e];
    }
    topk_stable(b, E, topk, idx);
    {
        float kth = b[idx[topk - 1]], next = -INFINITY;
        for (int e = 0; e < E; e++) {
            int used = 0;
            for (int j = 0; j < topk; j++) if (idx[j] == e) { used = 1; break; }
            if (!used && b[e] > next) next = b[e];
        }
        g_route_gap = kth - next;
    }
    for (int j = 0; j < topk; j++) w[j] = scores[idx[j]];
    float sum = orc_pw_sum(w, (size_t)topk);
    for (int j = 0; j < topk; j++) w[j] = w[j] / (sum + 1e-20f) * c->routed_scaling_factor;
    free(b); free(scores);
}

/* c/gmoe.h:210-227 SwiGLU expert on FP8 weights (dequant -> BF16 GEMV) */
static void expert(const OrcModel *m, Fp8 g, Fp8 u, Fp8 dn, const uint16_t *x, size_t d, size_t inter,
                   float limit, uint16_t *out) {
    uint16_t *gv = xc(inter * 2), *uv = xc(inter * 2), *h = xc(inter * 2);
    fp8lin(m, g, x, gv, 1, inter, d);
    fp8lin(m, u, x, uv, 1, inter, d);
    for (size_t i = 0; i < inter; i++) {
        float a = orc_bf16_f32(gv[i]), b = orc_bf16_f32(uv[i]);
        if (a > limit) a = limit;
        if (b > limit) b = limit;
        else if (b < -limit) b = -limit;
        float hv = orc_bf16_round(a * orc_sigmoid(a));
        h[i] = orc_bf16_bits(orc_bf16_round(hv * b));
    }
    fp8lin(m, dn, h, out, 1, d, inter);
    free(h); free(uv); free(gv);
}

/* c/gmoe.h:265-337 forward2 (per token, ascending expert, shared last) */
static void moe_forward(const OrcModel *m, int layer, const uint16_t *x, size_t s, uint16_t *out,
                        int32_t *idx_out, float *w_out, const int32_t *forced, float *gap_out);

void orc_moe_forward(const OrcModel *m, int layer, const uint16_t *x, size_t s, uint16_t *out,
                     int32_t *idx_out, float *w_out, const int32_t *forced) {
    moe_forward(m, layer, x, s, out, idx_out, w_out, forced, NULL);
}

/* c/gmodel.h dense MLP layers (the first first_k_dense_replace): the SwiGLU
 * expert of c/gmoe.h:210-227 on the layer's mlp.{gate,up,down}_proj */
void orc_mlp_forward(const OrcModel *m, int layer, const uint16_t *x, size_t s, uint16_t *out) {
    const OLayer *Ly = &m->L[layer];
    size_t d = (size_t)m->c.hidden_size, inter = (size_t)m->c.intermediate_size;
    for (size_t t = 0; t < s; t++)
        expert(m, Ly->mlp_g, Ly->mlp_u, Ly->mlp_d, x + t * d, d, inter, m->c.swiglu_limit, out + t * d);
}

static void moe_forward(const OrcModel *m, int layer, const uint16_t *x, size_t s, uint16_t *out,
                        int32_t *idx_out, float *w_out, const int32_t *forced, float *gap_out) {
    const OrcConfig *c = &m->c;
    const OLayer *Ly = &m->L[layer];
    int E = c->n_routed_experts, topk = c->num_experts_per_tok;
    size_t d = (size_t)c->hidden_size, inter = (size_t)c->moe_intermediate_size;
    size_t sinter = inter * (size_t)c->n_shared_experts;
    float *y = xc(d * 4), wt[64];
    int32_t idx[64];
    uint16_t *eo = xc(d * 2), *sh = xc(d * 2);
    for (size_t t = 0; t < s; t++) {
        const uint16_t *xt = x + t * d;
        router(m, Ly, xt, idx, wt);
        if (gap_out) gap_out[t] = g_route_gap;
        if (forced) {   /* c/gmoe.h:287-297: weights re-gathered at the forced indices */
            float scores_f[64];
            for (int j = 0; j < topk; j++) {
                idx[j] = forced[t * topk + j];
                float acc = 0.0f;
                for (size_t i = 0; i < d; i++)
                    acc += orc_bf16_f32(Ly->gate_w[(size_t)idx[j] * d + i]) * orc_bf16_f32(xt[i]);
                scores_f[j] = orc_sigmoid(acc);
            }
            float sum = orc_pw_sum(scores_f, (size_t)topk);
            for (int j = 0; j < topk; j++) wt[j] = scores_f[j] / (sum + 1e-20f) * c->routed_scaling_factor;
        }
        if (idx_out) memcpy(idx_out + t * topk, idx, (size_t)topk * 4);
        if (w_out) memcpy(w_out + t * topk, wt, (size_t)topk * 4);
        memset(y, 0, d * 4);
        for (int e = 0; e < E; e++) {
            int slot = -1;
            for (int j = 0; j < topk; j++) if (idx[j] == e) { slot = j; break; }
            if (slot < 0) continue;
            expert(m, Ly->eg[e], Ly->eu[e], Ly->ed[e], xt, d, inter, c->swiglu_limit, eo);
            for (size_t i = 0; i < d; i++) {
                float contrib = orc_bf16_round(orc_bf16_f32(eo[i]) * wt[slot]);
                y[i] = orc_bf16_round(y[i] + contrib);
            }
        }
        expert(m, Ly->sg, Ly->su, Ly->sd, xt, d, sinter, c->swiglu_limit, sh);
        for (size_t i = 0; i < d; i++) out[t * d + i] = orc_bf16_bits(y[i] + orc_bf16_f32(sh[i]));
    }
    free(sh); free(eo); free(y);
}

/* ---------------------------------------------------------------- KDA */

/* c/gkda.h:263-273 */
static void l2norm_row(const uint16_t *x, float *y, size_t D) {
    float *sq = xc(D * 4);
    for (size_t i = 0; i < D; i++) { float v = orc_bf16_f32(x[i]); y[i] = v; sq[i] = v * v; }
    float root = sqrtf(orc_pw_sum(sq, D) + 1e-6f);
    for (size_t i = 0; i < D; i++) y[i] = y[i] / root;
    free(sq);
}

/* c/gkda.h:279-331 one token, one head */
static void recurrent_head(float *S, const uint16_t *qh, const uint16_t *kh, const uint16_t *vh,
                           const float *gh, uint16_t beta, uint16_t *oh, size_t D, float qscale) {
    float *qf = xc(D * 4), *kf = xc(D * 4), *vf = xc(D * 4), *kv = xc(D * 4), *dl = xc(D * 4);
    l2norm_row(qh, qf, D);
    l2norm_row(kh, kf, D);
    for (size_t i = 0; i < D; i++) { qf[i] = qf[i] * qscale; vf[i] = orc_bf16_f32(vh[i]); }
    float bt = orc_bf16_f32(beta);
    for (size_t i = 0; i < D; i++) {
        float dec = expf(gh[i]);
        for (size_t j = 0; j < D; j++) S[i * D + j] = S[i * D + j] * dec;
    }
    for (size_t j = 0; j < D; j++) {
        float acc = 0.0f;
        for (size_t i = 0; i < D; i++) acc += S[i * D + j] * kf[i];
        kv[j] = acc;
    }
    for (size_t j = 0; j < D; j++) dl[j] = (vf[j] - kv[j]) * bt;
    for (size_t i = 0; i < D; i++)
        for (size_t j = 0; j < D; j++) S[i * D + j] = S[i * D + j] + kf[i] * dl[j];
    for (size_t j = 0; j < D; j++) {
        float acc = 0.0f;
        for (size_t i = 0; i < D; i++) acc += S[i * D + j] * qf[i];
        oh[j] = orc_bf16_bits(acc);
    }
    free(dl); free(kv); free(vf); free(kf); free(qf);
}

/* c/gkda.h:581-683: conv chained per token, then the core: recurrent per
 * token (decode = 1) or the chunked delta rule over the s rows (decode = 0,
 * the prefill's apus_gkda_chunk) */
static void kda_forward(const OrcModel *m, int layer, const uint16_t *x, size_t s, uint16_t *conv_state,
                        float *rec_state, int decode, uint16_t *out);

void orc_kda_decode(const OrcModel *m, int layer, const uint16_t *x, size_t s,
                    uint16_t *conv_state, float *rec_state, uint16_t *out) {
    kda_forward(m, layer, x, s, conv_state, rec_state, 1, out);
}

void orc_kda_prefill(const OrcModel *m, int layer, const uint16_t *x, size_t s,
                     uint16_t *conv_state, float *rec_state, uint16_t *out) {
    kda_forward(m, layer, x, s, conv_state, rec_state, 0, out);
}

static void kda_forward(const OrcModel *m, int layer, const uint16_t *x, size_t s, uint16_t *conv_state,
                        float *rec_state, int decode, uint16_t *out) {
    const OrcConfig *c = &m->c;
    const OLayer *W = &m->L[layer];
    size_t d = (size_t)c->hidden_size, H = (size_t)c->linear_num_heads, D = (size_t)c->linear_head_dim;
    size_t qkv = H * D, Dr = D, K = (size_t)c->linear_conv_kernel_dim;
    uint16_t *mq = xc(s * qkv * 2), *mk = xc(s * qkv * 2), *mv = xc(s * qkv * 2);
    uint16_t *fg1 = xc(s * Dr * 2), *fg2 = xc(s * qkv * 2), *bt = xc(s * H * 2), *beta = xc(s * H * 2);
    uint16_t *ga = xc(s * Dr * 2), *gate = xc(s * qkv * 2), *core = xc(s * qkv * 2), *on = xc(s * qkv * 2);
    float *g = xc(s * qkv * 4);
    gemm(W->q_w, x, mq, s, qkv, d);
    gemm(W->k_w, x, mk, s, qkv, d);
    gemm(W->v_w, x, mv, s, qkv, d);
    /* conv over the concatenated [q|k|v] channels (c/gkda.h:227-257);
     * conv weight rows: q_conv1d, k_conv1d, v_conv1d, each [qkv, K] */
    for (size_t t = 0; t < s; t++) {
        uint16_t *parts[3] = {mq + t * qkv, mk + t * qkv, mv + t * qkv};
        for (int pi = 0; pi < 3; pi++)
            for (size_t ch = 0; ch < qkv; ch++) {
                size_t cc = (size_t)pi * qkv + ch;
                uint16_t *stt = conv_state + cc * (K - 1);
                const uint16_t *wc = W->conv[pi] + ch * K;
                uint16_t xcv = parts[pi][ch];
                float acc = 0.0f;
                for (size_t i = 0; i < K - 1; i++) acc += orc_bf16_f32(wc[i]) * orc_bf16_f32(stt[i]);
                acc += orc_bf16_f32(wc[K - 1]) * orc_bf16_f32(xcv);
                parts[pi][ch] = orc_bf16_bits(acc * orc_sigmoid(acc));
                for (size_t j = 0; j + 1 < K - 1; j++) stt[j] = stt[j + 1];
                stt[K - 2] = xcv;
            }
    }
    gemm(W->f_a, x, fg1, s, Dr, d);
    gemm(W->f_b, fg1, fg2, s, qkv, Dr);
    for (size_t t = 0; t < s; t++)
        for (size_t hh = 0; hh < H; hh++) {
            float dec = expf(W->A_log[hh]);
            for (size_t q = 0; q < D; q++) {
                size_t i = hh * D + q;
                float z = orc_bf16_f32(fg2[t * qkv + i]) + W->dt_bias[i];
                g[t * qkv + i] = c->linear_lower_bound * orc_sigmoid(dec * z);
            }
        }
    gemm(W->b_w, x, bt, s, H, d);
    for (size_t i = 0; i < s * H; i++) beta[i] = orc_bf16_bits(orc_sigmoid(orc_bf16_f32(bt[i])));
    float qscale = (float)pow((double)D, -0.5);
    if (decode) {
        for (size_t t = 0; t < s; t++)
            for (size_t hh = 0; hh < H; hh++)
                recurrent_head(rec_state + hh * D * D, mq + t * qkv + hh * D, mk + t * qkv + hh * D,
                               mv + t * qkv + hh * D, g + t * qkv + hh * D, beta[t * H + hh],
                               core + t * qkv + hh * D, D, qscale);
    } else {
        orc_kda_chunk(mq, mk, mv, g, beta, rec_state, core, s, H, D);
    }
    gemm(W->g_a, x, ga, s, Dr, d);
    gemm(W->g_b, ga, gate, s, qkv, Dr);
    /* c/gkda.h:543-569 gated o_norm */
    float *sq = xc(D * 4);
    for (size_t r = 0; r < s * H; r++) {
        for (size_t q = 0; q < D; q++) { float v = orc_bf16_f32(core[r * D + q]); sq[q] = v * v; }
        float var = orc_pw_sum(sq, D) / (float)D;
        float inv = 1.0f / sqrtf(var + c->rms_norm_eps);
        for (size_t q = 0; q < D; q++) {
            float t = orc_bf16_f32(core[r * D + q]) * inv;
            t = orc_bf16_f32(W->o_norm[q]) * t;
            t = t * orc_sigmoid(orc_bf16_f32(gate[r * D + q]));
            on[r * D + q] = orc_bf16_bits(t);
        }
    }
    free(sq);
    gemm(W->o_w, on, out, s, d, qkv);
    free(g); free(on); free(core); free(gate); free(ga); free(beta); free(bt); free(fg2); free(fg1);
    free(mv); free(mk); free(mq);
}

/* ---------------------------------------------------------------- DSA */

static size_t dsa_width(const OrcConfig *c) {
    return (size_t)c->index_topk + (c->index_kpool_always_select_tail ? (size_t)c->index_kpool - 1 : 0);
}

/* c/gdsa.h:307-449 indexer: appends this call's idx rows at st->n, rebuilds
 * every full pool, scores, selects. */
static void indexer(const OrcModel *m, const OLayer *W, const uint16_t *x, const uint16_t *qres,
                    size_t s, ODsa *st, int32_t *topk, float *score_out, size_t score_ld) {
    const OrcConfig *c = &m->c;
    size_t d = (size_t)c->hidden_size, ql = (size_t)c->q_lora_rank;
    size_t IH = (size_t)c->index_n_heads, ID = (size_t)c->index_head_dim, kp = (size_t)c->index_kpool;
    size_t width = dsa_width(c), base = st->n, n = base + s, nf = n / kp;
    float idx_scale = (float)pow((double)ID, -0.5), ih_scale = (float)pow((double)IH, -0.5);
    uint16_t *iq = xc(s * IH * ID * 2), *kpre = xc(s * ID * 2), *gnew = xc(s * ID * 2), *wp = xc(s * IH * 2);
    gemm(W->idx_wq_b, qres, iq, s, IH * ID, ql);
    gemm(W->idx_wk, x, kpre, s, ID, d);
    gemm(W->idx_gate, x, gnew, s, ID, d);
    for (size_t t = 0; t < s; t++) {
        orc_layernorm(kpre + t * ID, W->idx_knorm_w, W->idx_knorm_b, st->ik + (base + t) * ID, ID, 1e-6f);
        memcpy(st->ig + (base + t) * ID, gnew + t * ID, ID * 2);
    }
    float *pkey = xc((nf ? nf : 1) * ID * 4), lg[64], e[64];
    for (size_t p = 0; p < nf; p++)
        for (size_t q = 0; q < ID; q++) {
            for (size_t cc = 0; cc < kp; cc++)
                lg[cc] = orc_bf16_f32(st->ig[(p * kp + cc) * ID + q]) + orc_bf16_f32(W->idx_ape[cc * ID + q]);
            float mx = lg[0];
            for (size_t cc = 1; cc < kp; cc++) if (lg[cc] > mx) mx = lg[cc];
            float sum = 0.0f;
            for (size_t cc = 0; cc < kp; cc++) { e[cc] = expf(lg[cc] - mx); sum += e[cc]; }
            float acc = 0.0f;
            for (size_t cc = 0; cc < kp; cc++)
                acc += orc_bf16_round(e[cc] / sum) * orc_bf16_f32(st->ik[(p * kp + cc) * ID + q]);
            pkey[p * ID + q] = orc_bf16_round(acc);
        }
    gemm(W->idx_wproj, x, wp, s, IH, d);
    float *sm = xc((nf ? nf : 1) * 4), *sc = xc(IH * 4), *w32 = xc(IH * 4);
    int32_t *sel = xc(((size_t)c->index_topk / kp + 1) * 4);
    for (size_t t = 0; t < s; t++) {
        size_t q_pos = base + t;
        for (size_t h = 0; h < IH; h++) w32[h] = orc_bf16_f32(wp[t * IH + h]) * ih_scale;
        for (size_t p = 0; p < nf; p++) {
            float acc = 0.0f;
            for (size_t h = 0; h < IH; h++) {
                float dot = 0.0f;
                for (size_t i = 0; i < ID; i++)
                    dot += orc_bf16_f32(iq[t * IH * ID + h * ID + i]) * pkey[p * ID + i];
                float v = dot * idx_scale;
                sc[h] = v > 0.0f ? v : 0.0f;
            }
            for (size_t h = 0; h < IH; h++) acc += w32[h] * sc[h];
            sm[p] = acc;
        }
        for (size_t p = 0; p < nf; p++)
            if (p * kp + (kp - 1) > q_pos) sm[p] = NEG_INF;
        if (score_out)
            for (size_t p = 0; p < nf && p < score_ld; p++) score_out[t * score_ld + p] = sm[p];
        size_t sk = (size_t)c->index_topk / kp;
        if (sk > nf) sk = nf;
        int32_t *row = topk + t * width;
        for (size_t i = 0; i < width; i++) row[i] = -1;
        if (sk) {
            topk_stable(sm, (int)nf, (int)sk, sel);
            for (size_t j = 0; j < sk; j++) {
                int valid = (size_t)sel[j] * kp + (kp - 1) <= q_pos;
                for (size_t o = 0; o < kp; o++)
                    row[j * kp + o] = valid ? sel[j] * (int32_t)kp + (int32_t)o : -1;
            }
        }
        if (c->index_kpool_always_select_tail) {
            size_t vis = q_pos + 1, tc = vis % kp, ts = vis - tc;
            for (size_t o = 0; o + 1 < kp; o++) row[sk * kp + o] = o < tc ? (int32_t)(ts + o) : -1;
        }
    }
    free(sel); free(w32); free(sc); free(sm); free(pkey); free(wp); free(gnew); free(kpre); free(iq);
}

/* c/gdsa.h:451-517 attention over the full cache with the additive mask */
static void attention(const OrcModel *m, const uint16_t *q, const ODsa *st, size_t s,
                      const int32_t *topk, uint16_t *out) {
    const OrcConfig *c = &m->c;
    size_t H = (size_t)c->num_attention_heads, qd = (size_t)c->qk_nope_head_dim;
    size_t vd = (size_t)c->v_head_dim, n = st->n, width = dsa_width(c);
    float scale = (float)pow((double)qd, -0.5);
    uint16_t *qh = xc(s * qd * 2), *scb = xc(s * n * 2);
    float *sc = xc(n * 4), *e = xc(n * 4);
    unsigned char *vis = xc(n);
    for (size_t h = 0; h < H; h++) {
        for (size_t t = 0; t < s; t++) memcpy(qh + t * qd, q + t * H * qd + h * qd, qd * 2);
        gemm(st->k + h * st->cap * qd, qh, scb, s, n, qd);
        for (size_t t = 0; t < s; t++) {
            const int32_t *ids = topk + t * width;
            memset(vis, 0, n);
            for (size_t i = 0; i < width; i++)
                if (ids[i] >= 0 && (size_t)ids[i] < n) vis[ids[i]] = 1;
            float mx = NEG_INF;
            for (size_t j = 0; j < n; j++) {
                float v = orc_bf16_round(orc_bf16_f32(scb[t * n + j]) * scale);
                v = v + (vis[j] ? 0.0f : NEG_INF);
                sc[j] = v;
                if (v > mx) mx = v;
            }
            for (size_t j = 0; j < n; j++) e[j] = expf(sc[j] - mx);
            float sum = orc_pw_sum(e, n);
            for (size_t j = 0; j < n; j++) e[j] = e[j] / sum;
            const uint16_t *vc = st->v + h * st->cap * vd;
            for (size_t dv = 0; dv < vd; dv++) {
                float acc = 0.0f;
                for (size_t j = 0; j < n; j++) acc += orc_bf16_round(e[j]) * orc_bf16_f32(vc[j * vd + dv]);
                out[t * H * vd + h * vd + dv] = orc_bf16_bits(acc);
            }
        }
    }
    free(vis); free(e); free(sc); free(scb); free(qh);
}

/* c/gdsa.h:555-674 forward3: s tokens in one shot (s = 1 for decode) */
static void dsa_forward(const OrcModel *m, const OLayer *W, const uint16_t *x, size_t s, ODsa *st,
                        uint16_t *out, int32_t *topk_out, float *score_out, size_t score_ld) {
    const OrcConfig *c = &m->c;
    size_t d = (size_t)c->hidden_size, H = (size_t)c->num_attention_heads, qd = (size_t)c->qk_nope_head_dim;
    size_t vd = (size_t)c->v_head_dim, ql = (size_t)c->q_lora_rank, kl = (size_t)c->kv_lora_rank;
    size_t base = st->n, width = dsa_width(c);
    uint16_t *qa = xc(s * ql * 2), *qres = xc(s * ql * 2), *q = xc(s * H * qd * 2), *kv = xc(s * kl * 2);
    uint16_t *kpass = xc(s * kl * 2), *kvb = xc(s * H * (qd + vd) * 2), *attn = xc(s * H * vd * 2);
    int32_t *topk = xc(s * width * 4);
    fp8lin(m, W->q_a, x, qa, s, ql, d);
    for (size_t t = 0; t < s; t++) orc_rmsnorm(qa + t * ql, W->q_a_norm, qres + t * ql, ql, c->rms_norm_eps);
    fp8lin(m, W->q_b, qres, q, s, H * qd, ql);
    fp8lin(m, W->kv_a, x, kv, s, kl, d);
    for (size_t t = 0; t < s; t++) orc_rmsnorm(kv + t * kl, W->kv_a_norm, kpass + t * kl, kl, c->rms_norm_eps);
    gemm(W->kv_b, kpass, kvb, s, H * (qd + vd), kl);
    for (size_t t = 0; t < s; t++)
        for (size_t h = 0; h < H; h++) {
            memcpy(st->k + h * st->cap * qd + (base + t) * qd, kvb + t * H * (qd + vd) + h * (qd + vd), qd * 2);
            memcpy(st->v + h * st->cap * vd + (base + t) * vd, kvb + t * H * (qd + vd) + h * (qd + vd) + qd,
                   vd * 2);
        }
    indexer(m, W, x, qres, s, st, topk, score_out, score_ld);
    if (topk_out) memcpy(topk_out, topk, s * width * 4);
    st->n = base + s;
    attention(m, q, st, s, topk, attn);
    fp8lin(m, W->o, attn, out, s, d, H * vd);
    free(topk); free(attn); free(kvb); free(kpass); free(kv); free(q); free(qres); free(qa);
}

/* c/gdsa.h:682-690 decode_batch2: per-token interleave */
void orc_dsa_decode(const OrcModel *m, int layer, const uint16_t *x, size_t s, OrcState *st,
                    uint16_t *out) {
    orc_dsa_decode_sel(m, layer, x, s, st, out, NULL, NULL, 0);
}

size_t orc_dsa_width(const OrcModel *m) { return dsa_width(&m->c); }

void orc_dsa_decode_sel(const OrcModel *m, int layer, const uint16_t *x, size_t s, OrcState *st,
                        uint16_t *out, int32_t *topk, float *scores, size_t score_ld) {
    size_t d = (size_t)m->c.hidden_size, width = dsa_width(&m->c);
    for (size_t t = 0; t < s; t++)
        dsa_forward(m, &m->L[layer], x + t * d, 1, &st->dsa[layer], out + t * d, topk ? topk + t * width : NULL,
                    scores ? scores + t * score_ld : NULL, score_ld);
}

/* -------------------------------------------------------------- model */

OrcModel *orc_model_new(const OrcConfig *c, int has_mtp) {
    OrcModel *m = xc(sizeof *m);
    m->c = *c;
    m->has_mtp = has_mtp;
    int nl = c->num_hidden_layers + (has_mtp ? 1 : 0);
    m->L = xc((size_t)nl * sizeof(OLayer));
    for (int l = 0; l < nl; l++) {
        m->L[l].eg = xc((size_t)c->n_routed_experts * sizeof(Fp8));
        m->L[l].eu = xc((size_t)c->n_routed_experts * sizeof(Fp8));
        m->L[l].ed = xc((size_t)c->n_routed_experts * sizeof(Fp8));
    }
    return m;
}

void orc_model_free(OrcModel *m) {
    if (!m) return;
    int nl = m->c.num_hidden_layers + (m->has_mtp ? 1 : 0);
    for (int l = 0; l < nl; l++) { free(m->L[l].eg); free(m->L[l].eu); free(m->L[l].ed); }
    for (size_t i = 0; i < m->capdeq; i++) free(m->deq[i].deq);
    free(m->deq);
    free(m->L);
    free(m);
}

static int set_fp8(Fp8 *f, const char *rest, const char *stem, const void *data) {
    char a[160], b[160];
    snprintf(a, sizeof a, "%s.weight", stem);
    snprintf(b, sizeof b, "%s.weight_scale_inv", stem);
    if (!strcmp(rest, a)) { f->c = data; return 1; }
    if (!strcmp(rest, b)) { f->s = data; return 1; }
    return 0;
}

int orc_model_set(OrcModel *m, const char *name, const void *data) {
    if (!strcmp(name, "embed_tokens.weight")) { m->embed = data; return 0; }
    if (!strcmp(name, "norm.weight")) { m->norm = data; return 0; }
    if (!strcmp(name, "lm_head.weight")) { m->head = data; return 0; }
    int l = -1, off = 0;
    if (sscanf(name, "layers.%d.%n", &l, &off) != 1 || off <= 0) return -1;
    int nl = m->c.num_hidden_layers + (m->has_mtp ? 1 : 0);
    if (l < 0 || l >= nl) return -1;
    OLayer *Y = &m->L[l];
    const char *r = name + off;
    struct { const char *n; const void **p; } tab[] = {
        {"input_layernorm.weight", (const void **)&Y->input_norm},
        {"post_attention_layernorm.weight", (const void **)&Y->post_norm},
        {"hc_attn_fn", (const void **)&Y->hc_fn[0]}, {"hc_ffn_fn", (const void **)&Y->hc_fn[1]},
        {"hc_attn_base", (const void **)&Y->hc_base[0]}, {"hc_ffn_base", (const void **)&Y->hc_base[1]},
        {"hc_attn_scale", (const void **)&Y->hc_scale[0]}, {"hc_ffn_scale", (const void **)&Y->hc_scale[1]},
        {"self_attn.q_proj.weight", (const void **)&Y->q_w}, {"self_attn.k_proj.weight", (const void **)&Y->k_w},
        {"self_attn.v_proj.weight", (const void **)&Y->v_w},
        {"self_attn.q_conv1d.weight", (const void **)&Y->conv[0]},
        {"self_attn.k_conv1d.weight", (const void **)&Y->conv[1]},
        {"self_attn.v_conv1d.weight", (const void **)&Y->conv[2]},
        {"self_attn.f_a_proj.weight", (const void **)&Y->f_a}, {"self_attn.f_b_proj.weight", (const void **)&Y->f_b},
        {"self_attn.A_log", (const void **)&Y->A_log}, {"self_attn.dt_bias", (const void **)&Y->dt_bias},
        {"self_attn.b_proj.weight", (const void **)&Y->b_w},
        {"self_attn.g_a_proj.weight", (const void **)&Y->g_a}, {"self_attn.g_b_proj.weight", (const void **)&Y->g_b},
        {"self_attn.o_norm.weight", (const void **)&Y->o_norm},
        {"self_attn.q_a_layernorm.weight", (const void **)&Y->q_a_norm},
        {"self_attn.kv_a_layernorm.weight", (const void **)&Y->kv_a_norm},
        {"self_attn.kv_b_proj.weight", (const void **)&Y->kv_b},
        {"self_attn.indexer.wq_b.weight", (const void **)&Y->idx_wq_b},
        {"self_attn.indexer.wk.weight", (const void **)&Y->idx_wk},
        {"self_attn.indexer.k_norm.weight", (const void **)&Y->idx_knorm_w},
        {"self_attn.indexer.k_norm.bias", (const void **)&Y->idx_knorm_b},
        {"self_attn.indexer.weights_proj.weight", (const void **)&Y->idx_wproj},
        {"self_attn.indexer.index_kpool_compress_ape", (const void **)&Y->idx_ape},
        {"self_attn.indexer.index_kpool_compress_gate", (const void **)&Y->idx_gate},
        {"mlp.gate.weight", (const void **)&Y->gate_w},
        {"mlp.gate.e_score_correction_bias", (const void **)&Y->gate_bias},
        {"enorm.weight", (const void **)&Y->enorm}, {"hnorm.weight", (const void **)&Y->hnorm},
        {"eh_proj.weight", (const void **)&Y->eh_proj},
        {"shared_head.norm.weight", (const void **)&Y->shared_norm},
    };
    for (size_t i = 0; i < sizeof tab / sizeof tab[0]; i++)
        if (!strcmp(r, tab[i].n)) { *tab[i].p = data; return 0; }
    if (!strcmp(r, "self_attn.o_proj.weight") && !m->c.layer_is_dsa[l < m->c.num_hidden_layers ? l : 0]
        && l < m->c.num_hidden_layers) { Y->o_w = data; return 0; }
    if (set_fp8(&Y->q_a, r, "self_attn.q_a_proj", data) || set_fp8(&Y->q_b, r, "self_attn.q_b_proj", data) ||
        set_fp8(&Y->kv_a, r, "self_attn.kv_a_proj_with_mqa", data) || set_fp8(&Y->o, r, "self_attn.o_proj", data) ||
        set_fp8(&Y->mlp_g, r, "mlp.gate_proj", data) || set_fp8(&Y->mlp_u, r, "mlp.up_proj", data) ||
        set_fp8(&Y->mlp_d, r, "mlp.down_proj", data) || set_fp8(&Y->sg, r, "mlp.shared_experts.gate_proj", data) ||
        set_fp8(&Y->su, r, "mlp.shared_experts.up_proj", data) ||
        set_fp8(&Y->sd, r, "mlp.shared_experts.down_proj", data))
        return 0;
    int e = -1, off2 = 0;
    if (sscanf(r, "mlp.experts.%d.%n", &e, &off2) == 1 && off2 > 0 && e >= 0 && e < m->c.n_routed_experts) {
        const char *q = r + off2;
        if (set_fp8(&Y->eg[e], q, "gate_proj", data) || set_fp8(&Y->eu[e], q, "up_proj", data) ||
            set_fp8(&Y->ed[e], q, "down_proj", data))
            return 0;
    }
    return -1;
}

const char *orc_model_missing(const OrcModel *m) {
    if (!m->embed) return "embed_tokens.weight";
    if (!m->norm) return "norm.weight";
    if (!m->head) return "lm_head.weight";
    return NULL;
}

static void dsa_alloc(ODsa *d, const OrcConfig *c, size_t cap) {
    size_t H = (size_t)c->num_attention_heads;
    d->cap = cap;
    d->n = 0;
    d->k = xc(H * cap * (size_t)c->qk_nope_head_dim * 2);
    d->v = xc(H * cap * (size_t)c->v_head_dim * 2);
    d->ik = xc(cap * (size_t)c->index_head_dim * 2);
    d->ig = xc(cap * (size_t)c->index_head_dim * 2);
}

static void dsa_free(ODsa *d) { free(d->k); free(d->v); free(d->ik); free(d->ig); }

OrcState *orc_state_new(const OrcModel *m, size_t cap) {
    const OrcConfig *c = &m->c;
    int L = c->num_hidden_layers;
    OrcState *st = xc(sizeof *st);
    st->m = m;
    st->cap = cap;
    st->conv = xc((size_t)L * sizeof(void *));
    st->rec = xc((size_t)L * sizeof(void *));
    st->dsa = xc((size_t)L * sizeof(ODsa));
    size_t qkv = (size_t)c->linear_num_heads * (size_t)c->linear_head_dim;
    for (int l = 0; l < L; l++) {
        if (!c->layer_is_dsa[l]) {
            st->conv[l] = xc(3 * qkv * ((size_t)c->linear_conv_kernel_dim - 1) * 2);
            st->rec[l] = xc(qkv * (size_t)c->linear_head_dim * 4);
        } else {
            dsa_alloc(&st->dsa[l], c, cap);
        }
    }
    return st;
}

void orc_state_free(OrcState *st) {
    if (!st) return;
    for (int l = 0; l < st->m->c.num_hidden_layers; l++) {
        free(st->conv[l]);
        free(st->rec[l]);
        if (st->m->c.layer_is_dsa[l]) dsa_free(&st->dsa[l]);
    }
    free(st->conv); free(st->rec); free(st->dsa); free(st);
}

size_t orc_state_pos(const OrcState *st) { return st->pos; }

void orc_state_set_pos(OrcState *st, size_t pos) { st->pos = pos; }

static int dsa_load(ODsa *d, const OrcConfig *c, const uint16_t *k, const uint16_t *v, const uint16_t *ik,
                    const uint16_t *ig, size_t n) {
    size_t H = (size_t)c->num_attention_heads, qd = (size_t)c->qk_nope_head_dim, vd = (size_t)c->v_head_dim;
    size_t ID = (size_t)c->index_head_dim;
    if (n > d->cap) return -1;
    for (size_t h = 0; h < H; h++) {
        memcpy(d->k + h * d->cap * qd, k + h * n * qd, n * qd * 2);
        memcpy(d->v + h * d->cap * vd, v + h * n * vd, n * vd * 2);
    }
    memcpy(d->ik, ik, n * ID * 2);
    memcpy(d->ig, ig, n * ID * 2);
    d->n = n;
    return 0;
}

int orc_state_load_kda(OrcState *st, int layer, const uint16_t *conv, const float *rec) {
    const OrcConfig *c = &st->m->c;
    if (layer < 0 || layer >= c->num_hidden_layers || c->layer_is_dsa[layer]) return -1;
    memcpy(st->conv[layer], conv, kda_bytes(c, 0));
    memcpy(st->rec[layer], rec, kda_bytes(c, 1));
    return 0;
}

int orc_state_load_dsa(OrcState *st, int layer, const uint16_t *k, const uint16_t *v, const uint16_t *ik,
                       const uint16_t *ig, size_t n) {
    const OrcConfig *c = &st->m->c;
    if (layer < 0 || layer >= c->num_hidden_layers || !c->layer_is_dsa[layer]) return -1;
    return dsa_load(&st->dsa[layer], c, k, v, ik, ig, n);
}

int orc_decode_batch(OrcModel *m, OrcState *st, const int32_t *ids, size_t s,
                     uint16_t *logits, uint16_t *h_out, uint16_t *yn_out) {
    return orc_decode_batch_ex(m, st, ids, s, logits, h_out, yn_out, NULL, NULL, NULL);
}

/* c/gmodel.h:1439-1626 apus_gm_run.  decode = 1: recurrent KDA, DSA one
 * token at a time (the decode batch); decode = 0: chunked KDA, DSA over the s
 * tokens in one call (the prefill).  logits: [s][V], or [V] of the last row
 * only when last_only (the rows are independent, so it is the same row). */
static int run(OrcModel *m, OrcState *st, const int32_t *ids, size_t s, int decode, uint16_t *logits,
               int last_only, uint16_t *h_out, uint16_t *yn_out, const int32_t *forced, int32_t *sel_out,
               float *gap_out);

int orc_decode_batch_ex(OrcModel *m, OrcState *st, const int32_t *ids, size_t s, uint16_t *logits,
                        uint16_t *h_out, uint16_t *yn_out, const int32_t *forced, int32_t *sel_out,
                        float *gap_out) {
    return run(m, st, ids, s, 1, logits, 0, h_out, yn_out, forced, sel_out, gap_out);
}

/* c/gmodel.h:1658-1666 apus_gmodel_prefill_h */
int orc_prefill_h(OrcModel *m, OrcState *st, const int32_t *ids, size_t s, uint16_t *logits,
                  uint16_t *h_out, uint16_t *yn_out) {
    return run(m, st, ids, s, 0, logits, 0, h_out, yn_out, NULL, NULL, NULL);
}

/* The same prompt pass with the logits of the last row only ([V]). */
int orc_prefill_last(OrcModel *m, OrcState *st, const int32_t *ids, size_t s, uint16_t *logits_last,
                     uint16_t *h_out, uint16_t *yn_out) {
    return run(m, st, ids, s, 0, logits_last, 1, h_out, yn_out, NULL, NULL, NULL);
}

static int run(OrcModel *m, OrcState *st, const int32_t *ids, size_t s, int decode, uint16_t *logits,
               int last_only, uint16_t *h_out, uint16_t *yn_out, const int32_t *forced, int32_t *sel_out,
               float *gap_out) {
    const OrcConfig *c = &m->c;
    if (s < 1) return -1;
    if (st->pos + s > st->cap) return -1;
    size_t d = (size_t)c->hidden_size, hc = (size_t)c->hc_mult, V = (size_t)c->vocab_size;
    uint16_t *h = xc(s * hc * d * 2), *h2 = xc(s * hc * d * 2), *x = xc(s * d * 2), *sub = xc(s * d * 2);
    uint16_t *yh = xc(s * d * 2);
    float *post = xc(s * hc * 4), *comb = xc(s * hc * hc * 4);
    for (size_t t = 0; t < s; t++)
        for (size_t j = 0; j < hc; j++) memcpy(h + (t * hc + j) * d, m->embed + (size_t)ids[t] * d, d * 2);
    for (int l = 0; l < c->num_hidden_layers; l++) {
        for (int site = 0; site < 2; site++) {
            for (size_t t = 0; t < s; t++) {
                orc_hc_pre(m, l, site, h + t * hc * d, x + t * d, post + t * hc, comb + t * hc * hc);
                orc_rmsnorm(x + t * d, site ? m->L[l].post_norm : m->L[l].input_norm, x + t * d, d,
                            c->rms_norm_eps);
            }
            if (site == 0) {
                if (!c->layer_is_dsa[l]) kda_forward(m, l, x, s, st->conv[l], st->rec[l], decode, sub);
                else if (decode) orc_dsa_decode(m, l, x, s, st, sub);
                else dsa_forward(m, &m->L[l], x, s, &st->dsa[l], sub, NULL, NULL, 0);
            } else if (!c->mlp_is_sparse[l]) {
                size_t inter = (size_t)c->intermediate_size;
                for (size_t t = 0; t < s; t++)
                    expert(m, m->L[l].mlp_g, m->L[l].mlp_u, m->L[l].mlp_d, x + t * d, d, inter,
                           c->swiglu_limit, sub + t * d);
            } else {
                const size_t lk = (size_t)l * s * (size_t)c->num_experts_per_tok;
                moe_forward(m, l, x, s, sub, sel_out ? sel_out + lk : NULL, NULL, forced ? forced + lk : NULL,
                            gap_out ? gap_out + (size_t)l * s : NULL);
            }
            for (size_t t = 0; t < s; t++)
                orc_hc_post(sub + t * d, h + t * hc * d, post + t * hc, comb + t * hc * hc, h2 + t * hc * d, d, hc);
            uint16_t *tmp = h; h = h2; h2 = tmp;
        }
    }
    if (h_out) memcpy(h_out, h, s * hc * d * 2);
    for (size_t t = 0; t < s; t++) {
        orc_hc_head(h + t * hc * d, yh + t * d, d, hc);
        orc_rmsnorm(yh + t * d, m->norm, yh + t * d, d, c->rms_norm_eps);
    }
    if (yn_out) memcpy(yn_out, yh, s * d * 2);
    if (logits && last_only) gemm(m->head, yh + (s - 1) * d, logits, 1, V, d);
    else if (logits) gemm(m->head, yh, logits, s, V, d);
    st->pos += s;
    free(comb); free(post); free(yh); free(sub); free(x); free(h2); free(h);
    return 0;
}

/* ---------------------------------------------------------------- MTP */

OrcMtpState *orc_mtp_state_new(const OrcModel *m, size_t cap) {
    OrcMtpState *st = xc(sizeof *st);
    st->cap = cap;
    dsa_alloc(&st->dsa, &m->c, cap);
    return st;
}

int orc_mtp_state_load(const OrcModel *m, OrcMtpState *mst, const uint16_t *k, const uint16_t *v,
                       const uint16_t *ik, const uint16_t *ig, size_t n) {
    if (dsa_load(&mst->dsa, &m->c, k, v, ik, ig, n)) return -1;
    mst->pos = n;
    return 0;
}

void orc_mtp_state_free(OrcMtpState *st) {
    if (!st) return;
    dsa_free(&st->dsa);
    free(st);
}

/* c/gmtp.h:471-541 */
int orc_mtp_forward(OrcModel *m, OrcMtpState *mst, const int32_t *ids, const uint16_t *prev_h,
                    size_t s, uint16_t *logits, uint16_t *out_h) {
    const OrcConfig *c = &m->c;
    size_t d = (size_t)c->hidden_size, V = (size_t)c->vocab_size;
    int Lm = c->num_hidden_layers;
    const OLayer *W = &m->L[Lm];
    float eps = c->rms_norm_eps;
    if (mst->pos + s > mst->cap) return -1;
    uint16_t *eh = xc(s * 2 * d * 2), *x = xc(s * d * 2), *xn = xc(s * d * 2), *sub = xc(s * d * 2);
    for (size_t t = 0; t < s; t++) {
        orc_rmsnorm(m->embed + (size_t)ids[t] * d, W->enorm, eh + t * 2 * d, d, eps);
        orc_rmsnorm(prev_h + t * d, W->hnorm, eh + t * 2 * d + d, d, eps);
    }
    gemm(W->eh_proj, eh, x, s, d, 2 * d);
    for (size_t t = 0; t < s; t++) orc_rmsnorm(x + t * d, W->input_norm, xn + t * d, d, eps);
    dsa_forward(m, W, xn, s, &mst->dsa, sub, NULL, NULL, 0);
    for (size_t i = 0; i < s * d; i++) x[i] = orc_bf16_bits(orc_bf16_f32(x[i]) + orc_bf16_f32(sub[i]));
    for (size_t t = 0; t < s; t++) orc_rmsnorm(x + t * d, W->post_norm, xn + t * d, d, eps);
    orc_moe_forward(m, Lm, xn, s, sub, NULL, NULL, NULL);
    for (size_t i = 0; i < s * d; i++) x[i] = orc_bf16_bits(orc_bf16_f32(x[i]) + orc_bf16_f32(sub[i]));
    for (size_t t = 0; t < s; t++) orc_rmsnorm(x + t * d, W->shared_norm, out_h + t * d, d, eps);
    gemm(m->head, out_h, logits, s, V, d);
    mst->pos += s;
    free(sub); free(xn); free(x); free(eh);
    return 0;
}

/* --------------------------------------------------------- spec decode */

struct OrcSpec {
    OrcModel *m;
    OrcState *st;
    OrcMtpState *mst;
    int depth, V, d, hc;
    OrcDraftHook hook;
    void *hook_ctx;
    int hook_after_chain;            /* 1: the MTP chain runs, then the hook edits its drafts */
    int32_t *raw;                    /* the chain's own drafts (before the hook) */
    float *margin;                   /* top-1 minus top-2 of each chain row */
    uint64_t emitted, batches, refeed, offered, accepted;
    size_t q;
    int32_t held;
    int32_t *drafts, *batch;
    uint16_t *logits16, *H, *Yn, *ph, *h_prev, *oh, *hmtp_a, *hmtp_b, *mtp_row;
    /* snapshot: pos + per-KDA conv/rec, per-DSA n; MTP pos/n */
    size_t snap_pos, *snap_n, mtp_snap_pos, mtp_snap_n;
    uint16_t **snap_conv;
    float **snap_rec;
};

OrcSpec *orc_spec_new(OrcModel *m, OrcState *st, OrcMtpState *mst, int depth) {
    OrcSpec *sp = xc(sizeof *sp);
    const OrcConfig *c = &m->c;
    sp->m = m; sp->st = st; sp->mst = mst;
    sp->depth = depth > 0 ? depth : 1;
    sp->V = c->vocab_size; sp->d = c->hidden_size; sp->hc = c->hc_mult;
    size_t D = (size_t)sp->depth, V = (size_t)sp->V, d = (size_t)sp->d, hcd = (size_t)sp->hc * d;
    sp->drafts = xc(D * 4); sp->batch = xc(D * 4);
    sp->raw = xc(D * 4); sp->margin = xc(D * 4);
    sp->logits16 = xc(D * V * 2); sp->H = xc(D * hcd * 2); sp->Yn = xc(D * d * 2);
    sp->ph = xc(D * d * 2); sp->h_prev = xc(d * 2); sp->oh = xc(D * d * 2);
    sp->hmtp_a = xc(d * 2); sp->hmtp_b = xc(d * 2); sp->mtp_row = xc(V * 2);
    int L = c->num_hidden_layers;
    size_t qkv = (size_t)c->linear_num_heads * (size_t)c->linear_head_dim;
    sp->snap_n = xc((size_t)L * sizeof(size_t));
    sp->snap_conv = xc((size_t)L * sizeof(void *));
    sp->snap_rec = xc((size_t)L * sizeof(void *));
    for (int l = 0; l < L; l++)
        if (!c->layer_is_dsa[l]) {
            sp->snap_conv[l] = xc(3 * qkv * ((size_t)c->linear_conv_kernel_dim - 1) * 2);
            sp->snap_rec[l] = xc(qkv * (size_t)c->linear_head_dim * 4);
        }
    return sp;
}

void orc_spec_free(OrcSpec *sp) {
    if (!sp) return;
    for (int l = 0; l < sp->m->c.num_hidden_layers; l++) { free(sp->snap_conv[l]); free(sp->snap_rec[l]); }
    free(sp->snap_conv); free(sp->snap_rec); free(sp->snap_n);
    free(sp->raw); free(sp->margin);
    free(sp->drafts); free(sp->batch); free(sp->logits16); free(sp->H); free(sp->Yn); free(sp->ph);
    free(sp->h_prev); free(sp->oh); free(sp->hmtp_a); free(sp->hmtp_b); free(sp->mtp_row);
    free(sp);
}

void orc_spec_set_draft_hook(OrcSpec *sp, OrcDraftHook hook, void *ctx) {
    sp->hook = hook;
    sp->hook_ctx = ctx;
    sp->hook_after_chain = 0;
}

void orc_spec_set_force_hook(OrcSpec *sp, OrcDraftHook hook, void *ctx) {
    sp->hook = hook;
    sp->hook_ctx = ctx;
    sp->hook_after_chain = 1;
}

void orc_spec_raw_drafts(const OrcSpec *sp, int32_t *drafts, float *margins) {
    memcpy(drafts, sp->raw, (size_t)sp->depth * 4);
    if (margins) memcpy(margins, sp->margin, (size_t)sp->depth * 4);
}

/* (top-1 - top-2) / |top-1| of a BF16 logits row: how far the pick is
 * from a tie, relative to the row's scale */
static float top2_margin(const uint16_t *row, size_t n) {
    float a = -INFINITY, b = -INFINITY;
    for (size_t i = 0; i < n; i++) {
        float v = orc_bf16_f32(row[i]);
        if (v > a) { b = a; a = v; } else if (v > b) b = v;
    }
    return (a - b) / fmaxf(fabsf(a), 1e-30f);
}

/* c/gmtp.h:807-831, greedy: the accept walk over the verify rows' BF16
 * logits (row j-1 verifies draft j); out[0] = held, then each accepted
 * draft; the token that ends the walk (replacement or bonus) becomes the
 * next held token.  Returns the emitted count. */
int orc_spec_walk(const uint16_t *logits16, int De, size_t V, const int32_t *drafts, int32_t held, int32_t *out,
                  int *matched_out, int32_t *next_held) {
    int ne = 0, matched = 0, last = -1;
    out[ne++] = held;
    for (int j = 1; j < De; j++) {
        int x = orc_argmax_bf16(logits16 + (size_t)(j - 1) * V, V);
        if (drafts[j] == x) { matched++; out[ne++] = x; }
        else { last = x; break; }
    }
    if (last < 0) last = orc_argmax_bf16(logits16 + (size_t)(De - 1) * V, V);
    *matched_out = matched;
    *next_held = last;
    return ne;
}

static size_t kda_bytes(const OrcConfig *c, int rec) {
    size_t qkv = (size_t)c->linear_num_heads * (size_t)c->linear_head_dim;
    return rec ? qkv * (size_t)c->linear_head_dim * 4 : 3 * qkv * ((size_t)c->linear_conv_kernel_dim - 1) * 2;
}

/* c/gmtp.h:577-603 */
static void snap_take(OrcSpec *sp) {
    const OrcConfig *c = &sp->m->c;
    sp->snap_pos = sp->st->pos;
    for (int l = 0; l < c->num_hidden_layers; l++) {
        if (!c->layer_is_dsa[l]) {
            memcpy(sp->snap_conv[l], sp->st->conv[l], kda_bytes(c, 0));
            memcpy(sp->snap_rec[l], sp->st->rec[l], kda_bytes(c, 1));
        } else {
            sp->snap_n[l] = sp->st->dsa[l].n;
        }
    }
}

static void snap_restore(OrcSpec *sp) {
    const OrcConfig *c = &sp->m->c;
    sp->st->pos = sp->snap_pos;
    for (int l = 0; l < c->num_hidden_layers; l++) {
        if (!c->layer_is_dsa[l]) {
            memcpy(sp->st->conv[l], sp->snap_conv[l], kda_bytes(c, 0));
            memcpy(sp->st->rec[l], sp->snap_rec[l], kda_bytes(c, 1));
        } else {
            sp->st->dsa[l].n = sp->snap_n[l];
        }
    }
}

/* c/gmtp.h:677-696 draft chain (greedy) */
static void chain(OrcSpec *sp) {
    size_t V = (size_t)sp->V, d = (size_t)sp->d;
    sp->drafts[0] = orc_argmax_bf16(sp->mtp_row, V);
    sp->margin[0] = top2_margin(sp->mtp_row, V);
    uint16_t *cur = sp->hmtp_a, *nxt = sp->hmtp_b;
    for (int i = 1; i < sp->depth; i++) {
        if (orc_mtp_forward(sp->m, sp->mst, &sp->drafts[i - 1], cur, 1, sp->logits16, nxt)) {
            for (int j = i; j < sp->depth; j++) sp->drafts[j] = 0;
            break;
        }
        memcpy(sp->mtp_row, sp->logits16, V * 2);
        sp->drafts[i] = orc_argmax_bf16(sp->mtp_row, V);
        sp->margin[i] = top2_margin(sp->mtp_row, V);
        uint16_t *tmp = cur; cur = nxt; nxt = tmp;
    }
    if (cur != sp->hmtp_a) memcpy(sp->hmtp_a, cur, d * 2);
    memcpy(sp->raw, sp->drafts, (size_t)sp->depth * 4);
    if (sp->hook && sp->hook_after_chain) sp->hook(sp->hook_ctx, (int64_t)sp->q, sp->drafts, sp->depth);
}

/* c/gmtp.h:698-774 apus_gspec_prefill: the main model's prompt pass
 * (apus_gmodel_prefill_h: chunked KDA, DSA over the prompt in one call), the
 * held token from its last row, then the MTP true-pair replay over the
 * n - 1 pairs in one call (lag 1, postnorm source: c/gmtp.h:99-119). */
int orc_spec_prefill(OrcSpec *sp, const int32_t *ids, size_t n) {
    size_t V = (size_t)sp->V, d = (size_t)sp->d, hcd = (size_t)sp->hc * d;
    if (n < 1) return -1;
    uint16_t *h_all = xc(n * hcd * 2), *yn_all = xc(n * d * 2), *lg = xc(V * 2);
    if (orc_prefill_last(sp->m, sp->st, ids, n, lg, h_all, yn_all)) { free(lg); free(yn_all); free(h_all); return -1; }
    memcpy(sp->mtp_row, lg, V * 2);
    sp->held = orc_argmax_bf16(sp->mtp_row, V);
    sp->q = n;
    if (sp->hook && !sp->hook_after_chain) {
        sp->hook(sp->hook_ctx, (int64_t)sp->q, sp->drafts, sp->depth);
    } else if (n >= 2) {
        uint16_t *l16 = xc(n * V * 2), *oh = xc(n * d * 2);
        /* postnorm source: the hnorm input of position t is yn[t] */
        int rc = orc_mtp_forward(sp->m, sp->mst, ids + 1, yn_all, n - 1, l16, oh);
        memcpy(sp->h_prev, yn_all + (n - 1) * d, d * 2);
        if (!rc) {
            memcpy(sp->mtp_row, l16 + (n - 2) * V, V * 2);
            memcpy(sp->hmtp_a, oh + (n - 2) * d, d * 2);
            sp->mtp_snap_pos = sp->mst->pos;
            sp->mtp_snap_n = sp->mst->dsa.n;
            chain(sp);
        } else {
            for (int i = 0; i < sp->depth; i++) sp->drafts[i] = 0;
        }
        free(oh); free(l16);
    }
    free(lg); free(yn_all); free(h_all);
    return 0;
}

/* c/gmtp.h:776-891, greedy (temp 0) */
int orc_spec_step(OrcSpec *sp, int *out, int cap) {
    int D = sp->depth;
    size_t V = (size_t)sp->V, d = (size_t)sp->d;
    if (cap < D + 1) return 0;
    int De = D;
    if (sp->q + (size_t)De > sp->st->cap) De = (int)(sp->st->cap - sp->q);
    if (De <= 0) return 0;
    snap_take(sp);
    sp->batch[0] = sp->held;
    for (int j = 1; j < De; j++) sp->batch[j] = sp->drafts[j];
    if (orc_decode_batch(sp->m, sp->st, sp->batch, (size_t)De, sp->logits16, sp->H, sp->Yn)) return 0;
    sp->batches++;
    int matched = 0;
    int32_t last = -1;
    int ne = orc_spec_walk(sp->logits16, De, V, sp->drafts, sp->held, out, &matched, &last);
    sp->offered += (uint64_t)(matched < De - 1 ? matched + 1 : matched);
    sp->accepted += (uint64_t)matched;
    sp->emitted += (uint64_t)ne;
    if (matched < De - 1) {
        snap_restore(sp);
        if (orc_decode_batch(sp->m, sp->st, sp->batch, (size_t)(matched + 1), sp->logits16, NULL, NULL)) return 0;
        sp->refeed += (uint64_t)(matched + 1);
    }
    sp->held = last;
    sp->q += (size_t)(matched + 1);
    if (!sp->hook || sp->hook_after_chain) {
        memcpy(sp->ph, sp->h_prev, d * 2);
        for (int j = 1; j <= matched; j++) memcpy(sp->ph + (size_t)j * d, sp->Yn + (size_t)(j - 1) * d, d * 2);
        sp->mst->pos = sp->mtp_snap_pos;
        sp->mst->dsa.n = sp->mtp_snap_n;
        if (orc_mtp_forward(sp->m, sp->mst, sp->batch, sp->ph, (size_t)(matched + 1), sp->logits16, sp->oh)) {
            for (int i = 0; i < D; i++) sp->drafts[i] = 0;
            return ne;
        }
        memcpy(sp->mtp_row, sp->logits16 + (size_t)matched * V, V * 2);
        memcpy(sp->hmtp_a, sp->oh + (size_t)matched * d, d * 2);
        memcpy(sp->h_prev, sp->Yn + (size_t)matched * d, d * 2);
        sp->mtp_snap_pos = sp->mst->pos;
        sp->mtp_snap_n = sp->mst->dsa.n;
        chain(sp);
    } else {
        sp->hook(sp->hook_ctx, (int64_t)sp->q, sp->drafts, D);
    }
    return ne;
}

void orc_spec_stats(const OrcSpec *sp, uint64_t *o) {
    o[0] = sp->emitted; o[1] = sp->batches; o[2] = sp->refeed; o[3] = sp->offered; o[4] = sp->accepted;
    o[5] = sp->q; o[6] = (uint64_t)(int64_t)sp->held;
}

int orc_greedy(OrcModel *m, OrcState *st, const int32_t *ids, size_t n, int n_gen, int32_t *out) {
    size_t V = (size_t)m->c.vocab_size;
    uint16_t *lg = xc(V * 2);
    /* the prompt through the prefill (c/apus.c:1079), then one-token decodes */
    if (orc_prefill_last(m, st, ids, n, lg, NULL, NULL)) { free(lg); return -1; }
    int32_t tok = orc_argmax_bf16(lg, V);
    for (int i = 0; i < n_gen; i++) {
        out[i] = tok;
        if (i + 1 == n_gen) break;
        if (orc_decode_batch(m, st, &tok, 1, lg, NULL, NULL)) { free(lg); return -1; }
        tok = orc_argmax_bf16(lg, V);
    }
    free(lg);
    return 0;
}
