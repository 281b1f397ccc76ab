/*
 * apus_gmtp_gcuda.h — the glm5_next decode stack and the MTP speculative
 * decode step on the B200, behind the reference's engine entry points
 * (c/gmodel.h, c/gmtp.h).
 *
 * The reference's ApusGmodel is opaque and filled from its safetensors
 * container (c/gmodel.h:622-1106); here the model is filled tensor by tensor
 * under the same checkpoint names (or from seeded synthetic weights) and is
 * resident in HBM.  ApusGcudaModel bundles what the reference splits over
 * ApusGmodel + ApusGmodelState + ApusGmtp + ApusGmtpState + ApusGspec
 * (c/gmodel.h:129-320, c/gmtp.h:123-259): one sequence, one stream.
 *
 * Numerics: every sublayer keeps the reference's rounding points; fp32
 * summation orders differ where a GPU reduction replaces a sequential loop,
 * so logits match the reference within tolerance, while inside this engine a
 * verify row is bitwise the one-token decode of the same context.  The
 * speculative stream is therefore bitwise the engine's own non-speculative
 * stream, greedy or sampled.  The greedy pick is c/sample.h:76-81 on the
 * BF16 logits (lowest index wins ties), fused into the lm_head GEMV; the
 * sampled draw is apus_gcuda_sample_rows_dev's (include/apus_gcuda.h).
 */
#ifndef APUS_GMTP_GCUDA_H
#define APUS_GMTP_GCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define APUS_GCUDA_MAX_LAYERS 64

/* Field names and meaning of ApusGmodelConfig (c/gmodel.h:88-108); the two
 * per-layer pattern arrays are inline (c/gmodel.h:344-350 rule or explicit). */
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
    int layer_is_dsa[APUS_GCUDA_MAX_LAYERS];
    int mlp_is_sparse[APUS_GCUDA_MAX_LAYERS];
} ApusGcudaConfig;

typedef struct ApusGcudaModel ApusGcudaModel;

/* Model + one sequence state with kv_cap token positions and a speculative
 * depth (verify rows per step, 1..8; the reference's APUS_SPEC_K).  has_mtp
 * loads the NextN block as layer num_hidden_layers (c/gmodel.h:186-209).
 * c/gmodel.h:161-164 (open2) + :244 (state_new) + c/gmtp.h:133,145,245. */
ApusGcudaModel *apus_gcuda_model_new(const ApusGcudaConfig *cfg, int has_mtp, size_t kv_cap, int depth);
void apus_gcuda_model_free(ApusGcudaModel *m);

/* Expert parallelism over `world` GPUs, one process and one model per GPU.
 * Rank r keeps routed experts [r*E/world, (r+1)*E/world), the shared expert
 * and vocabulary rows [r*ceil(V/world), ...) of the lm_head; everything else
 * is replicated.  Each MoE layer exchanges the weighted expert outputs and the
 * lm_head exchanges its argmax keys through peer memory; every rank emits the
 * same tokens as a one-GPU model.  The reference runs the whole model in one
 * process (c/gmodel.h:161-164); this is its multi-GPU form.  Bootstrap: every
 * rank calls _ep_handle (64 bytes out), the handles are all-gathered by the
 * host, then every rank calls _ep_connect with the world*64 bytes in rank
 * order.  set() returns 1 for another rank's expert tensor (nothing stored),
 * and decode_batch / mtp_forward refuse to return logits. */
ApusGcudaModel *apus_gcuda_model_new_ep(const ApusGcudaConfig *cfg, int has_mtp, size_t kv_cap, int depth,
                                        int rank, int world);
int apus_gcuda_model_ep_handle(ApusGcudaModel *m, void *handle_out /* 64 bytes */);
int apus_gcuda_model_ep_connect(ApusGcudaModel *m, const void *handles /* world * 64 bytes */);

/* The reference's weight container (c/gmodel.h:123-137, c/st.h:25-80):
 * config.json in either layout the reference accepts (the real
 * "text_config" + "linear_attn_config" file or the flat fixture file;
 * explicit layer_types / mlp_layer_types lists win over the i % 4 == 3 and
 * first_k_dense_replace rule), and a directory with
 * model.safetensors.index.json naming the safetensors shard of every tensor
 * (container names: checkpoint names minus "model.language_model.").
 * apus_gcuda_config_load fills cfg (0 / -1 + err).  apus_gcuda_container_check
 * verifies, without a GPU, that every tensor the model of cfg needs is present
 * with its dtype and size; it returns their count or -1.
 * apus_gcuda_container_read copies one tensor's raw bytes to host (or, with
 * host == NULL, only reports its size); it returns the byte count or -1.
 * apus_gcuda_model_load_container uploads every tensor the model stores on
 * this rank (an expert-parallel rank reads only its own experts and its
 * lm_head rows); the shards are memory-mapped, not copied on the host. */
int apus_gcuda_config_load(const char *path, ApusGcudaConfig *cfg, char *err, size_t errcap);
int apus_gcuda_container_check(const char *dir, const ApusGcudaConfig *cfg, int has_mtp, char *err,
                               size_t errcap);
long apus_gcuda_container_read(const char *dir, const char *name, void *host, size_t cap, char *err,
                               size_t errcap);
int apus_gcuda_model_load_container(ApusGcudaModel *m, const char *dir, char *err, size_t errcap);

/* Tensor by checkpoint name (c/gmodel.h:622-1106 names, minus the
 * "model.language_model." prefix), host pointer, synchronous. */
int apus_gcuda_model_set(ApusGcudaModel *m, const char *name, const void *host, size_t bytes);
int apus_gcuda_model_get(ApusGcudaModel *m, const char *name, void *host, size_t bytes);
/* Seeded synthetic weights generated on the device (BASELINE distributions). */
int apus_gcuda_model_init_random(ApusGcudaModel *m, uint64_t seed);
/* Fresh sequence: position 0, all states zero. */
int apus_gcuda_model_reset(ApusGcudaModel *m);
size_t apus_gcuda_model_pos(const ApusGcudaModel *m);            /* c/gmodel.h:246 */

/* c/gmodel.h:311-314 apus_gmodel_decode_batch: s <= 8 tokens at the current
 * position, committed.  logits [s,V], h_out [s,hc*dim] (last-layer stream),
 * yn_out [s,dim] (post-final-norm rows): host arrays, each may be NULL. */
int apus_gcuda_decode_batch(ApusGcudaModel *m, const int32_t *ids, size_t s, uint16_t *logits,
                            uint16_t *h_out, uint16_t *yn_out);

/* c/gmodel.h:317-320 apus_gmodel_prefill_h on a fresh sequence (reset
 * first): the prompt ids[n] in one pass, chunked KDA and the DSA over the
 * prompt as the reference's prefill, committed.  The prompt's rows go through
 * each layer together (chunks of 256), the linears on the tensor-core GEMM.
 * logits [n,V] (every row's; the rows' lm_head runs only when asked),
 * yn_out [n,dim] (post-final-norm rows); host arrays, each may be NULL.
 * Expert-parallel models return the logits gathered from every rank's slice. */
int apus_gcuda_prefill(ApusGcudaModel *m, const int32_t *ids, size_t n, uint16_t *logits, uint16_t *yn_out);

/* c/gmtp.h:169-172 apus_gmtp_forward: s <= 8 pairs (ids[t], prev_h[t]) at the
 * MTP block's current position, committed.  logits [s,V], out_h [s,dim]. */
int apus_gcuda_mtp_forward(ApusGcudaModel *m, const int32_t *ids, const uint16_t *prev_h, size_t s,
                           uint16_t *logits, uint16_t *out_h);

/* c/gmtp.h:245-248 apus_gspec_init's temp / top_p / rng (seeded as
 * apus_rng_seed, c/sample.h:159): temp <= 0 decodes greedily (the default),
 * temp > 0 samples every emitted token with one splitmix64 draw, in position
 * order (c/gmtp.h:800-831); drafts stay the MTP argmax.  The stream state
 * persists across prefills like a caller-owned ApusRng.  Expert-parallel
 * models sample too: each rank's vocabulary slice of the logits rows is
 * gathered on every rank, which then draws the same tokens.
 * NaN temp is rejected; -1 on error. */
int apus_gcuda_gspec_sampling(ApusGcudaModel *m, float temp, float top_p, uint64_t seed);
/* The splitmix64 state (c/sample.h:57 ApusRng.s) after the draws so far. */
int apus_gcuda_rng_state(ApusGcudaModel *m, uint64_t *state);

/* c/gmtp.h:253 apus_gspec_prefill: prompt in 8-token decode batches, held
 * token (greedy or sampled), MTP true-pair replay (postnorm source, lag 1,
 * c/gmtp.h:99-119) and the first draft chain.  0 on success. */
int apus_gcuda_gspec_prefill(ApusGcudaModel *m, const int32_t *ids, size_t n);
/* c/gmtp.h:259 apus_gspec_step: one verify step entirely on the
 * device (verify forward, accept walk, KDA checkpoint select + DSA rewind,
 * MTP replay, draft chain); appends the emitted tokens to out (cap >=
 * depth+1) and returns their count (0 at capacity). */
int apus_gcuda_gspec_step(ApusGcudaModel *m, int *out, int cap);
/* The same step enqueued on the model's stream without waiting (emitted
 * tokens go to a device-resident log); gspec_emitted synchronises and copies
 * up to cap logged tokens, returning how many were logged since prefill. */
int apus_gcuda_gspec_step_async(ApusGcudaModel *m);
int apus_gcuda_gspec_emitted(ApusGcudaModel *m, int32_t *out, size_t cap);
/* Device-resident step counters (c/apus.c:1061-1075): emitted, batches,
 * offered, accepted, position, held. */
int apus_gcuda_gspec_stats(ApusGcudaModel *m, uint64_t *out6);
/* Forced draft agreement (the reference's draft_override test hook,
 * c/gmtp.h:211-215, generalised): after each chain, draft i for position
 * q+i becomes truth[q+i-base] with probability p (splitmix64 of seed and the
 * position), else (truth+1) mod V.  truth == NULL switches it off. */
int apus_gcuda_gspec_force(ApusGcudaModel *m, const int32_t *truth, size_t n, size_t base, double p,
                           uint64_t seed);

/* Non-speculative greedy decode (the reference run loop's --no-spec path,
 * c/apus.c:1079-1143): prefill ids[n], then n_gen argmax tokens into out. */
int apus_gcuda_greedy(ApusGcudaModel *m, const int32_t *ids, size_t n, int n_gen, int32_t *out);
/* The same non-speculative decode drawing each token with the model's
 * sampling settings (tests/m8g/test_m8g.c:649-678 nonspec_run): greedy when
 * temp <= 0, else one splitmix64 draw per token from the stream state. */
int apus_gcuda_generate(ApusGcudaModel *m, const int32_t *ids, size_t n, int n_gen, int32_t *out);

/* Digest (FNV-1a 64) of the committed KDA states and DSA caches (the
 * rollback check of tests/m8g/test_m8g.c:383-424). */
uint64_t apus_gcuda_state_digest(ApusGcudaModel *m);

/* Replay the full-depth step from a CUDA graph captured on its first use
 * (the step is fixed-shape and keeps its control state on the device). */
int apus_gcuda_gspec_use_graph(ApusGcudaModel *m, int on);
/* The model's CUDA stream (cudaStream_t), for timing with events. */
void *apus_gcuda_model_stream(ApusGcudaModel *m);
/* Counters: [0] MoE expert problems run (routed union + shared, summed over
 * calls), [1] main-model forwards, [2] MTP forwards enqueued, [3] kernels in
 * the captured step graph (0 before capture), [4] bytes of the control
 * block a synchronous step reads back (twice per step). */
int apus_gcuda_model_counters(ApusGcudaModel *m, uint64_t *out, size_t n);

/* Inspection hooks (no reference counterpart; the reference dumps through
 * its APUS_DEBUG logging): stop the main forward after (layer, stage) —
 * stage 0 mHC pre (attn), 1 attention, 2 mHC post, 3 mHC pre (ffn), 4 MLP —
 * and read a scratch buffer by name ("x", "sub", "h4", "h4b", "kp", "core",
 * "q", "kvb", "attn", ...).  layer -1 clears the stop. */
int apus_gcuda_model_debug_stop(ApusGcudaModel *m, int layer, int stage);
int apus_gcuda_model_debug_read(ApusGcudaModel *m, const char *name, void *host, size_t bytes);
/* More inspection names for debug_read: "moe_idx" / "moe_w" (the last MoE
 * call's routing, [rows][top-k] int32 / f32, ascending experts), "moe_sel"
 * (the same selections in top-k order), "hmtp" / "hcarry" ([d] BF16: the
 * MTP hidden the next chain step starts from / the hnorm input carried to
 * the next replay), "oh" (the last MTP forward's post-shared_head.norm
 * rows), "logits" ([8][V]
 * BF16 rows of the last forward that wrote logits), "drafts" / "raw_drafts"
 * (int32, the verify drafts of the next step / the MTP chain's own drafts
 * before forced agreement), and the committed sequence state: "kda_conv.L"
 * [3*qkv][K-1] BF16, "kda_rec.L" [H][D][D] f32, "dsa_k.L" [AH][n][qd],
 * "dsa_v.L" [AH][n][vd], "dsa_ik.L" / "dsa_ig.L" [n][ID] BF16 (n committed
 * rows; L = num_hidden_layers names the MTP block).  A decode_batch stopped
 * by debug_stop commits nothing.  gspec_keep_logits(1): every speculative
 * step also writes its verify rows' BF16 logits (rows 0..depth-1 of
 * "logits"), so a test can replay the accept walk on them. */
int apus_gcuda_gspec_keep_logits(ApusGcudaModel *m, int on);

#ifdef __cplusplus
}
#endif
#endif
