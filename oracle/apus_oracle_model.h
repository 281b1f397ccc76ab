/*
 * apus_oracle_model.h — CPU restatement (TEST INFRASTRUCTURE ONLY) of the
 * apus GLM-5.3-Flash decode stack: mHC, MoE, KDA, DSA, the layer loop, the
 * MTP draft head and the greedy speculative step.  The checker of the CUDA
 * engine; never linked into it.
 */
#ifndef APUS_ORACLE_MODEL_H
#define APUS_ORACLE_MODEL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_MAX_LAYERS 64

/* Field names and meaning of ApusGmodelConfig (c/gmodel.h:88-108); the two
 * per-layer pattern arrays are inline. */
typedef struct {
    int hidden_size, vocab_size, num_hidden_layers;
    float rms_norm_eps;
    int hc_mult, hc_sinkhorn_iters;
    float hc_eps;
    int first_k_dense_replace;
    int intermediate_size, moe_intermediate_size;
    int n_routed_experts, n_shared_experts, num_experts_per_tok;
    float routed_scaling_factor;
    int norm_topk_prob;
    float swiglu_limit;
    int num_attention_heads, q_lora_rank, kv_lora_rank;
    int qk_nope_head_dim, v_head_dim;
    int index_n_heads, index_head_dim, index_topk, index_kpool;
    int index_kpool_always_select_tail;
    int linear_num_heads, linear_head_dim, linear_conv_kernel_dim;
    float linear_lower_bound;
    int num_nextn_predict_layers;
    int layer_is_dsa[ORC_MAX_LAYERS];
    int mlp_is_sparse[ORC_MAX_LAYERS];
} OrcConfig;

typedef struct OrcModel OrcModel;
typedef struct OrcState OrcState;
typedef struct OrcMtpState OrcMtpState;
typedef struct OrcSpec OrcSpec;

/* model: weights are caller-owned arrays registered by checkpoint name
 * ("layers.3.self_attn.q_a_proj.weight", "embed_tokens.weight", ...). */
OrcModel *orc_model_new(const OrcConfig *c, int has_mtp);
void orc_model_free(OrcModel *m);
int  orc_model_set(OrcModel *m, const char *name, const void *data);  /* 0 ok, -1 unknown */
const char *orc_model_missing(const OrcModel *m);   /* first unset tensor or NULL */

OrcState *orc_state_new(const OrcModel *m, size_t cap);
void orc_state_free(OrcState *st);
size_t orc_state_pos(const OrcState *st);

/* apus_gmodel_decode_batch (c/gmodel.h:1648-1656): s tokens, RECURRENT KDA,
 * per-token DSA interleave.  logits [s,V], h_out [s,hc*d], yn_out [s,d]
 * (BF16 codes; h_out/yn_out may be NULL). */
int orc_decode_batch(OrcModel *m, OrcState *st, const int32_t *ids, size_t s,
                     uint16_t *logits, uint16_t *h_out, uint16_t *yn_out);
/* The same with the MoE routing exposed (test inspection): forced
 * [L][s][topk] replaces each sparse layer's selection (top-k order, the
 * teacher-forcing hook of c/gmoe.h:145-152); sel_out [L][s][topk] gets the
 * selections, gap_out [L][s] the router's biased-score gap between the
 * topk-th selection and the best unselected expert (any may be NULL; dense
 * layers are left untouched). */
int orc_decode_batch_ex(OrcModel *m, OrcState *st, const int32_t *ids, size_t s, uint16_t *logits,
                        uint16_t *h_out, uint16_t *yn_out, const int32_t *forced, int32_t *sel_out,
                        float *gap_out);

/* apus_gmodel_prefill_h (c/gmodel.h:1658-1666): the prompt pass, s tokens
 * in one call with CHUNKED KDA and the DSA over the s tokens at once.
 * logits [s,V] (or NULL).  orc_prefill_last: the same with the logits of the
 * last row only ([V]). */
int orc_prefill_h(OrcModel *m, OrcState *st, const int32_t *ids, size_t s, uint16_t *logits,
                  uint16_t *h_out, uint16_t *yn_out);
int orc_prefill_last(OrcModel *m, OrcState *st, const int32_t *ids, size_t s, uint16_t *logits_last,
                     uint16_t *h_out, uint16_t *yn_out);

/* Sublayer entry points for unit parity (state passed explicitly). */
void orc_rmsnorm(const uint16_t *x, const uint16_t *w, uint16_t *y, size_t n, float eps);
void orc_layernorm(const uint16_t *x, const uint16_t *w, const uint16_t *b, uint16_t *y,
                   size_t n, float eps);
void orc_hc_pre(const OrcModel *m, int layer, int ffn, const uint16_t *h4, uint16_t *x,
                float *post, float *comb);
void orc_hc_post(const uint16_t *x, const uint16_t *res4, const float *post, const float *comb,
                 uint16_t *y4, size_t d, size_t n);
void orc_hc_head(const uint16_t *x4, uint16_t *y, size_t d, size_t n);
void orc_moe_forward(const OrcModel *m, int layer, const uint16_t *x, size_t s, uint16_t *out,
                     int32_t *idx_out, float *w_out, const int32_t *forced);
void orc_mlp_forward(const OrcModel *m, int layer, const uint16_t *x, size_t s, uint16_t *out);
void orc_kda_decode(const OrcModel *m, int layer, const uint16_t *x, size_t s,
                    uint16_t *conv_state, float *rec_state, uint16_t *out);
/* c/gkda.h:581-683 with decode = 0 (the chunked core over the s rows) */
void orc_kda_prefill(const OrcModel *m, int layer, const uint16_t *x, size_t s,
                     uint16_t *conv_state, float *rec_state, uint16_t *out);
void orc_dsa_decode(const OrcModel *m, int layer, const uint16_t *x, size_t s,
                    OrcState *st, uint16_t *out);
/* The same with the indexer's selection of every token (topk [s][width],
 * token ids, -1 padded; width = orc_dsa_width) and its pool scores (scores
 * [s][score_ld], -FLT_MAX for pools a token cannot see); both may be NULL. */
size_t orc_dsa_width(const OrcModel *m);
void orc_dsa_decode_sel(const OrcModel *m, int layer, const uint16_t *x, size_t s, OrcState *st,
                        uint16_t *out, int32_t *topk, float *scores, size_t score_ld);

/* State transplant (tests feed the oracle the engine's committed state so a
 * sublayer is checked on identical inputs): KDA conv [3*qkv][K-1] BF16 and
 * rec [H][D][D] f32; DSA k [H][n][qd], v [H][n][vd], ik / ig [n][ID] BF16. */
void orc_state_set_pos(OrcState *st, size_t pos);
int orc_state_load_kda(OrcState *st, int layer, const uint16_t *conv, const float *rec);
int orc_state_load_dsa(OrcState *st, int layer, const uint16_t *k, const uint16_t *v, const uint16_t *ik,
                       const uint16_t *ig, size_t n);

/* MTP head (c/gmtp.h:471-541) and its DSA-cache state. */
OrcMtpState *orc_mtp_state_new(const OrcModel *m, size_t cap);
void orc_mtp_state_free(OrcMtpState *st);
int orc_mtp_forward(OrcModel *m, OrcMtpState *mst, const int32_t *ids, const uint16_t *prev_h,
                    size_t s, uint16_t *logits, uint16_t *out_h);
int orc_mtp_state_load(const OrcModel *m, OrcMtpState *mst, const uint16_t *k, const uint16_t *v,
                       const uint16_t *ik, const uint16_t *ig, size_t n);

/* Greedy speculative decode (c/gmtp.h:617-891), depth D = verify rows. */
typedef void (*OrcDraftHook)(void *ctx, int64_t q, int32_t *drafts, int n);
OrcSpec *orc_spec_new(OrcModel *m, OrcState *st, OrcMtpState *mst, int depth);
void orc_spec_free(OrcSpec *sp);
void orc_spec_set_draft_hook(OrcSpec *sp, OrcDraftHook hook, void *ctx);
/* The B200 engine's forced agreement: the MTP chain still runs and the hook
 * then edits its drafts (the reference's draft_override replaces the MTP). */
void orc_spec_set_force_hook(OrcSpec *sp, OrcDraftHook hook, void *ctx);
/* The last chain's own drafts (before any hook) and each chain row's
 * (top-1 - top-2) / |top-1| logit margin. */
void orc_spec_raw_drafts(const OrcSpec *sp, int32_t *drafts, float *margins);
/* c/gmtp.h:807-831, greedy: the accept walk over De verify rows of BF16
 * logits; out[0..ne) = held then the accepted drafts; returns ne. */
int orc_spec_walk(const uint16_t *logits16, int De, size_t V, const int32_t *drafts, int32_t held, int32_t *out,
                  int *matched, int32_t *next_held);
int  orc_spec_prefill(OrcSpec *sp, const int32_t *ids, size_t n);
int  orc_spec_step(OrcSpec *sp, int *out, int cap);
/* stats: emitted, batches, refeed, offered, accepted, q, held */
void orc_spec_stats(const OrcSpec *sp, uint64_t *out7);

/* Non-speculative greedy decode: prefill then n_gen argmax tokens. */
int orc_greedy(OrcModel *m, OrcState *st, const int32_t *ids, size_t n, int n_gen, int32_t *out);

#ifdef __cplusplus
}
#endif
#endif
