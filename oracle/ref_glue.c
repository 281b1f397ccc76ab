/*
 * ref_glue.c — instantiates the apus reference's own header-only C engine
 * (c/*.h, compiled where it lies, never copied) into oracle/_ref/libapus_ref.so
 * so the tests can pin the oracle restatement against the reference itself
 * and the bench can time the reference CPU path.  TEST INFRASTRUCTURE ONLY.
 * The single-TU instantiation list mirrors tests/m8g/test_m8g.c:48-60.
 */
#define APUS_JSON_IMPLEMENTATION
#define APUS_ST_IMPLEMENTATION
#define APUS_COMPAT_IMPLEMENTATION
#define APUS_BF16_IMPLEMENTATION
#define APUS_FP8BLK_IMPLEMENTATION
#define APUS_GMHC_IMPLEMENTATION
#define APUS_GMOE_IMPLEMENTATION
#define APUS_GKDA_IMPLEMENTATION
#define APUS_GDSA_IMPLEMENTATION
#define APUS_GCACHE_IMPLEMENTATION
#define APUS_GMODEL_IMPLEMENTATION
#define APUS_SAMPLE_IMPLEMENTATION
#define APUS_GMTP_IMPLEMENTATION
#include "gmodel.h"
#include "gmtp.h"
#include "sample.h"
#include "bf16.h"
#include "fp8blk.h"

/* thread count the reference pool will use (c/pool.h APUS_THREADS) */
int apus_ref_threads(void) { return apus_pool_default_threads(); }

/* The reference MoE sublayer (c/gmoe.h apus_gmoe_forward2) on caller-owned
 * BF16 (dequantized) expert views; eg/eu/ed are [E] pointer arrays whose
 * unselected entries are never dereferenced. */
int ref_moe_forward(int E, int topk, size_t dim, size_t inter, float route_scale, float limit,
                    const uint16_t *gate_w, const float *gate_bias, const uint16_t *const *eg,
                    const uint16_t *const *eu, const uint16_t *const *ed, const uint16_t *sg,
                    const uint16_t *su, const uint16_t *sd, const uint16_t *x, size_t s, uint16_t *out) {
    ApusGmoeW w;
    memset(&w, 0, sizeof w);
    w.router.E = E; w.router.topk = topk; w.router.dim = dim; w.router.route_scale = route_scale;
    w.router.gate_w = gate_w; w.router.gate_bias = gate_bias;
    w.inter = inter; w.eg = eg; w.eu = eu; w.ed = ed;
    w.sg = sg; w.su = su; w.sd = sd; w.sinter = inter; w.limit = limit;
    ApusGmoeScratch sc;
    apus_gmoe_scratch_init(&sc, &w, s);
    apus_gmoe_forward2(&w, x, s, out, NULL, &sc, NULL);
    apus_gmoe_scratch_free(&sc);
    return 0;
}

/* ------------------------------------------------------------------------
 * Building a reference ApusGmodel from caller-owned arrays.  The reference
 * loads weights from its safetensors container (c/gmodel.h:622-1106); the
 * tests have no container, so this glue fills the SAME struct fields the
 * loader fills (c/gmodel.h:484-526), with the same derived buffers (mHC fn
 * widened to f32, q|k|v conv concatenated, FP8 MLP/expert weights
 * dequantized with apus_fp8blk_dequant_mt), and then calls the reference's
 * own forward / MTP / speculative functions unchanged.
 * ---------------------------------------------------------------------- */
#include "apus_oracle_model.h"

typedef struct { const uint8_t *c; const float *s; } RFp8;

typedef struct {
    const uint16_t *hc_fn16[2];
    const uint16_t *conv[3];
    RFp8 mlp[3], shr[3], *ex;   /* ex: [E*3] gate/up/down */
} RPend;

typedef struct {
    ApusGmodel *m;
    RPend *pend;
    int nl;
} RefModel;

RefModel *ref_model_new(const OrcConfig *oc, int has_mtp) {
    RefModel *R = calloc(1, sizeof *R);
    ApusGmodel *m = calloc(1, sizeof *m);
    ApusGmodelConfig *c = &m->cfg;
    c->hidden_size = oc->hidden_size; c->vocab_size = oc->vocab_size;
    c->num_hidden_layers = oc->num_hidden_layers; c->rms_norm_eps = oc->rms_norm_eps;
    c->hc_mult = oc->hc_mult; c->hc_sinkhorn_iters = oc->hc_sinkhorn_iters; c->hc_eps = oc->hc_eps;
    c->first_k_dense_replace = oc->first_k_dense_replace;
    c->intermediate_size = oc->intermediate_size; c->moe_intermediate_size = oc->moe_intermediate_size;
    c->n_routed_experts = oc->n_routed_experts; c->n_shared_experts = oc->n_shared_experts;
    c->num_experts_per_tok = oc->num_experts_per_tok; c->routed_scaling_factor = oc->routed_scaling_factor;
    c->norm_topk_prob = oc->norm_topk_prob; c->swiglu_limit = oc->swiglu_limit;
    c->num_attention_heads = oc->num_attention_heads; c->q_lora_rank = oc->q_lora_rank;
    c->kv_lora_rank = oc->kv_lora_rank; c->qk_nope_head_dim = oc->qk_nope_head_dim;
    c->v_head_dim = oc->v_head_dim; c->index_n_heads = oc->index_n_heads;
    c->index_head_dim = oc->index_head_dim; c->index_topk = oc->index_topk;
    c->index_kpool = oc->index_kpool; c->index_kpool_always_select_tail = oc->index_kpool_always_select_tail;
    c->linear_num_heads = oc->linear_num_heads; c->linear_head_dim = oc->linear_head_dim;
    c->linear_conv_kernel_dim = oc->linear_conv_kernel_dim; c->linear_lower_bound = oc->linear_lower_bound;
    c->num_nextn_predict_layers = has_mtp;
    int L = c->num_hidden_layers;
    c->layer_is_dsa = malloc((size_t)L * sizeof(int));
    c->mlp_is_sparse = malloc((size_t)L * sizeof(int));
    for (int l = 0; l < L; l++) { c->layer_is_dsa[l] = oc->layer_is_dsa[l]; c->mlp_is_sparse[l] = oc->mlp_is_sparse[l]; }
    R->nl = L + (has_mtp ? 1 : 0);
    m->layers = calloc((size_t)R->nl, sizeof(ApusGmodelLayer));
    R->pend = calloc((size_t)R->nl, sizeof(RPend));
    for (int l = 0; l < R->nl; l++) R->pend[l].ex = calloc((size_t)c->n_routed_experts * 3, sizeof(RFp8));
    m->has_mtp = has_mtp;
    m->prefill_moe_chunk = 8;
    R->m = m;
    return R;
}

static int rset_fp8(RFp8 *f, const char *rest, const char *stem, const void *data) {
    char a[160], b[160];
    snprintf(a, sizeof a, "%s.weight", stem);
    snprintf(b, sizeof b, "%s.weight_scale_inv", stem);
    if (!strcmp(rest, a)) { f->c = data; return 1; }
    if (!strcmp(rest, b)) { f->s = data; return 1; }
    return 0;
}

int ref_model_set(RefModel *R, const char *name, const void *data) {
    ApusGmodel *m = R->m;
    if (!strcmp(name, "embed_tokens.weight")) { m->embed = data; return 0; }
    if (!strcmp(name, "norm.weight")) { m->norm = data; return 0; }
    if (!strcmp(name, "lm_head.weight")) { m->head = data; return 0; }
    int l = -1, off = 0;
    if (sscanf(name, "layers.%d.%n", &l, &off) != 1 || off <= 0 || l < 0 || l >= R->nl) return -1;
    ApusGmodelLayer *Y = &m->layers[l];
    RPend *P = &R->pend[l];
    const char *r = name + off;
    ApusGkdaW *k = &Y->kda;
    ApusGdsaW *d = &Y->dsa;
    struct { const char *n; const void **p; } tab[] = {
        {"input_layernorm.weight", (const void **)&Y->input_norm},
        {"post_attention_layernorm.weight", (const void **)&Y->post_norm},
        {"hc_attn_fn", (const void **)&P->hc_fn16[0]}, {"hc_ffn_fn", (const void **)&P->hc_fn16[1]},
        {"hc_attn_base", (const void **)&Y->hc_attn_base}, {"hc_ffn_base", (const void **)&Y->hc_ffn_base},
        {"hc_attn_scale", (const void **)&Y->hc_attn_scale}, {"hc_ffn_scale", (const void **)&Y->hc_ffn_scale},
        {"self_attn.q_proj.weight", (const void **)&k->q_w}, {"self_attn.k_proj.weight", (const void **)&k->k_w},
        {"self_attn.v_proj.weight", (const void **)&k->v_w},
        {"self_attn.q_conv1d.weight", (const void **)&P->conv[0]},
        {"self_attn.k_conv1d.weight", (const void **)&P->conv[1]},
        {"self_attn.v_conv1d.weight", (const void **)&P->conv[2]},
        {"self_attn.f_a_proj.weight", (const void **)&k->f_a}, {"self_attn.f_b_proj.weight", (const void **)&k->f_b},
        {"self_attn.A_log", (const void **)&k->A_log}, {"self_attn.dt_bias", (const void **)&k->dt_bias},
        {"self_attn.b_proj.weight", (const void **)&k->b_w},
        {"self_attn.g_a_proj.weight", (const void **)&k->g_a}, {"self_attn.g_b_proj.weight", (const void **)&k->g_b},
        {"self_attn.o_norm.weight", (const void **)&k->o_norm},
        {"self_attn.q_a_layernorm.weight", (const void **)&d->q_a_norm},
        {"self_attn.kv_a_layernorm.weight", (const void **)&d->kv_a_norm},
        {"self_attn.kv_b_proj.weight", (const void **)&d->kv_b},
        {"self_attn.indexer.wq_b.weight", (const void **)&d->idx_wq_b},
        {"self_attn.indexer.wk.weight", (const void **)&d->idx_wk},
        {"self_attn.indexer.k_norm.weight", (const void **)&d->idx_knorm_w},
        {"self_attn.indexer.k_norm.bias", (const void **)&d->idx_knorm_b},
        {"self_attn.indexer.weights_proj.weight", (const void **)&d->idx_wproj},
        {"self_attn.indexer.index_kpool_compress_ape", (const void **)&d->idx_ape},
        {"self_attn.indexer.index_kpool_compress_gate", (const void **)&d->idx_gate},
        {"mlp.gate.weight", (const void **)&Y->router.gate_w},
        {"mlp.gate.e_score_correction_bias", (const void **)&Y->router.gate_bias},
        {"enorm.weight", (const void **)&m->mtp_enorm}, {"hnorm.weight", (const void **)&m->mtp_hnorm},
        {"eh_proj.weight", (const void **)&m->mtp_eh_proj},
        {"shared_head.norm.weight", (const void **)&m->mtp_shared_norm},
    };
    for (size_t i = 0; i < sizeof tab / sizeof tab[0]; i++)
        if (!strcmp(r, tab[i].n)) { *tab[i].p = data; return 0; }
    int is_dsa = (l >= m->cfg.num_hidden_layers) || m->cfg.layer_is_dsa[l];
    if (!is_dsa && !strcmp(r, "self_attn.o_proj.weight")) { k->o_w = data; return 0; }
    RFp8 qa = {d->q_a_c, d->q_a_s}, qb = {d->q_b_c, d->q_b_s}, kva = {d->kv_a_c, d->kv_a_s}, oo = {d->o_c, d->o_s};
    if (rset_fp8(&qa, r, "self_attn.q_a_proj", data)) { d->q_a_c = qa.c; d->q_a_s = qa.s; return 0; }
    if (rset_fp8(&qb, r, "self_attn.q_b_proj", data)) { d->q_b_c = qb.c; d->q_b_s = qb.s; return 0; }
    if (rset_fp8(&kva, r, "self_attn.kv_a_proj_with_mqa", data)) { d->kv_a_c = kva.c; d->kv_a_s = kva.s; return 0; }
    if (rset_fp8(&oo, r, "self_attn.o_proj", data)) { d->o_c = oo.c; d->o_s = oo.s; return 0; }
    if (rset_fp8(&P->mlp[0], r, "mlp.gate_proj", data) || rset_fp8(&P->mlp[1], r, "mlp.up_proj", data) ||
        rset_fp8(&P->mlp[2], r, "mlp.down_proj", data) ||
        rset_fp8(&P->shr[0], r, "mlp.shared_experts.gate_proj", data) ||
        rset_fp8(&P->shr[1], r, "mlp.shared_experts.up_proj", data) ||
        rset_fp8(&P->shr[2], r, "mlp.shared_experts.down_proj", data))
        return 0;
    int e = -1, off2 = 0;
    if (sscanf(r, "mlp.experts.%d.%n", &e, &off2) == 1 && off2 > 0 && e >= 0 && e < m->cfg.n_routed_experts) {
        const char *q = r + off2;
        if (rset_fp8(&P->ex[e * 3 + 0], q, "gate_proj", data) || rset_fp8(&P->ex[e * 3 + 1], q, "up_proj", data) ||
            rset_fp8(&P->ex[e * 3 + 2], q, "down_proj", data))
            return 0;
    }
    return -1;
}

static uint16_t *rdeq(RFp8 f, size_t O, size_t K) {
    uint16_t *o = malloc(O * K * sizeof(uint16_t));
    apus_fp8blk_dequant_mt(f.c, f.s, o, O, K);
    return o;
}

/* Derived buffers, as apus_gmodel_open2 builds them. */
void ref_model_finalize(RefModel *R) {
    ApusGmodel *m = R->m;
    const ApusGmodelConfig *c = &m->cfg;
    size_t d = (size_t)c->hidden_size, hc = (size_t)c->hc_mult, mix = (2 + hc) * hc;
    size_t inter = (size_t)c->intermediate_size, mi = (size_t)c->moe_intermediate_size;
    size_t si = mi * (size_t)c->n_shared_experts;
    int E = c->n_routed_experts;
    for (int l = 0; l < R->nl; l++) {
        ApusGmodelLayer *Y = &m->layers[l];
        RPend *P = &R->pend[l];
        int is_mtp = l >= c->num_hidden_layers;
        for (int sub = 0; sub < 2 && !is_mtp; sub++) {
            float *fn = malloc(mix * hc * d * sizeof(float));
            for (size_t i = 0; i < mix * hc * d; i++) fn[i] = apus_bf16_f32(P->hc_fn16[sub][i]);
            if (sub) Y->hc_ffn_fn = fn; else Y->hc_attn_fn = fn;
        }
        if (!is_mtp && !c->layer_is_dsa[l]) {
            ApusGkdaW *w = &Y->kda;
            size_t H = (size_t)c->linear_num_heads, D = (size_t)c->linear_head_dim, qkv = H * D;
            size_t ck = (size_t)c->linear_conv_kernel_dim;
            w->dim = d; w->H = H; w->D = D; w->Dr = D;
            w->lower_bound = c->linear_lower_bound; w->eps = c->rms_norm_eps;
            Y->kda_conv = malloc(3 * qkv * ck * sizeof(uint16_t));
            for (int p = 0; p < 3; p++) memcpy(Y->kda_conv + (size_t)p * qkv * ck, P->conv[p], qkv * ck * 2);
            w->conv_w = Y->kda_conv;
        } else {
            ApusGdsaW *w = &Y->dsa;
            w->dim = d; w->H = (size_t)c->num_attention_heads; w->qd = (size_t)c->qk_nope_head_dim;
            w->vd = (size_t)c->v_head_dim; w->ql = (size_t)c->q_lora_rank; w->kl = (size_t)c->kv_lora_rank;
            w->eps = c->rms_norm_eps; w->IH = (size_t)c->index_n_heads; w->ID = (size_t)c->index_head_dim;
            w->topk = (size_t)c->index_topk; w->kpool = (size_t)c->index_kpool;
            w->tail = c->index_kpool_always_select_tail;
        }
        int sparse = is_mtp || c->mlp_is_sparse[l];
        if (!sparse) {
            Y->mlp_g = rdeq(P->mlp[0], inter, d);
            Y->mlp_u = rdeq(P->mlp[1], inter, d);
            Y->mlp_d = rdeq(P->mlp[2], d, inter);
        } else {
            Y->router.E = E; Y->router.topk = c->num_experts_per_tok; Y->router.dim = d;
            Y->router.route_scale = c->routed_scaling_factor;
            Y->shr_g = rdeq(P->shr[0], si, d);
            Y->shr_u = rdeq(P->shr[1], si, d);
            Y->shr_d = rdeq(P->shr[2], d, si);
            Y->experts = calloc((size_t)E, sizeof *Y->experts);
            Y->expert_arena = malloc((size_t)E * 3 * mi * d * sizeof(uint16_t));
            for (int e = 0; e < E; e++) {
                uint16_t *base = Y->expert_arena + (size_t)e * 3 * mi * d;
                apus_fp8blk_dequant_mt(P->ex[e * 3 + 0].c, P->ex[e * 3 + 0].s, base, mi, d);
                apus_fp8blk_dequant_mt(P->ex[e * 3 + 1].c, P->ex[e * 3 + 1].s, base + mi * d, mi, d);
                apus_fp8blk_dequant_mt(P->ex[e * 3 + 2].c, P->ex[e * 3 + 2].s, base + 2 * mi * d, d, mi);
                Y->experts[e].gate = base;
                Y->experts[e].up = base + mi * d;
                Y->experts[e].down = base + 2 * mi * d;
            }
        }
    }
}

ApusGmodelState *ref_state_new(RefModel *R, size_t cap) { return apus_gmodel_state_new(R->m, cap); }
void ref_state_free(ApusGmodelState *st) { apus_gmodel_state_free(st); }

int ref_decode_batch(RefModel *R, ApusGmodelState *st, const int32_t *ids, size_t s,
                     uint16_t *logits, uint16_t *h_out, uint16_t *yn_out) {
    return apus_gmodel_decode_batch(R->m, st, ids, s, logits, NULL, h_out, yn_out);
}

/* apus_gmodel_prefill_h (c/gmodel.h:1658-1666): the prompt pass */
int ref_prefill_h(RefModel *R, ApusGmodelState *st, const int32_t *ids, size_t s, uint16_t *logits,
                  uint16_t *h_out, uint16_t *yn_out) {
    return apus_gmodel_prefill_h(R->m, st, ids, s, logits, NULL, h_out, yn_out);
}

/* The reference spec engine (c/gmtp.h:617-891), greedy, rng seeded 12345. */
typedef struct {
    ApusGspec sp;
    ApusGmtp mt;
    ApusGmtpState *mst;
    ApusRng rng;
} RefSpec;

RefSpec *ref_spec_new(RefModel *R, ApusGmodelState *st, size_t mtp_cap, int depth) {
    RefSpec *S = calloc(1, sizeof *S);
    char err[128];
    if (apus_gmtp_bind(&S->mt, R->m, err, sizeof err)) { free(S); return NULL; }
    S->mst = apus_gmtp_state_new(&S->mt, mtp_cap);
    apus_rng_seed(&S->rng, 12345);
    apus_gspec_init(&S->sp, R->m, st, &S->mt, S->mst, depth, 0.0f, 1.0f, &S->rng, NULL);
    return S;
}

void ref_spec_free(RefSpec *S) {
    if (!S) return;
    apus_gspec_free(&S->sp);
    apus_gmtp_state_free(S->mst);
    free(S);
}

void ref_spec_set_draft_hook(RefSpec *S, void (*hook)(void *, int64_t, int32_t *, int), void *ctx) {
    S->sp.draft_override = hook;
    S->sp.draft_ctx = ctx;
}

int ref_spec_prefill(RefSpec *S, const int32_t *ids, size_t n) {
    return apus_gspec_prefill(&S->sp, ids, n);
}

int ref_spec_step(RefSpec *S, int *out, int cap) { return apus_gspec_step(&S->sp, out, cap); }

void ref_spec_stats(const RefSpec *S, uint64_t *o) {
    const ApusGspec *sp = &S->sp;
    o[0] = sp->emitted; o[1] = sp->batches; o[2] = sp->refeed_tokens; o[3] = sp->offered;
    o[4] = sp->accepted; o[5] = sp->q; o[6] = (uint64_t)(int64_t)sp->held;
}

int ref_mtp_forward(RefSpec *S, const int32_t *ids, const uint16_t *prev_h, size_t s,
                    uint16_t *logits, uint16_t *out_h) {
    return apus_gmtp_forward(&S->mt, S->mst, ids, prev_h, s, logits, out_h, NULL);
}
