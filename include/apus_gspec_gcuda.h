/*
 * apus_gspec_gcuda.h — the reference's speculative-engine API (c/gmtp.h,
 * c/gmodel.h, c/sample.h), names, argument order and return conventions
 * kept, implemented over the B200 engine of apus_gmtp_gcuda.h.
 *
 * A host written against the reference's spec loop (c/apus.c:1016-1077:
 * apus_gmtp_bind, apus_gmtp_state_new, apus_gspec_init, apus_gspec_prefill,
 * apus_gspec_step, the ApusGspec counters, apus_gspec_free,
 * apus_gmtp_state_free) compiles against this header unchanged and links
 * libapus_gcuda.so instead of compiling the reference's implementation.
 *
 * What differs behind the names:
 *   - ApusGmodel / ApusGmodelState stay opaque (c/gmodel.h:129, :239).
 *     apus_gmodel_open2 reads the container's config and checks the
 *     container; the weights are uploaded to HBM when the sequence state is
 *     made (apus_gmodel_state_new), because the B200 engine keeps one
 *     sequence beside its resident weights: one state per model at a time.
 *     The tier settings (NVMe expert cache) are accepted and unused: every
 *     expert is resident.
 *   - ApusGmtp is complete (callers declare it on the stack) but its fields
 *     are this engine's; ApusGmtpState is opaque (callers only hold the
 *     pointer).
 *   - ApusGspec keeps the reference's public fields and counters
 *     (c/gmtp.h:202-243).  The counters are the device's, copied after every
 *     prefill and step.  refeed_tokens counts the tokens the reference's
 *     partial-reject path re-decodes (this engine rolls back to a checkpoint
 *     and re-decodes none; the count keeps the reference's meaning).
 *   - draft_override (c/gmtp.h:211-215) is honoured after every prefill and
 *     step: the hook edits the next drafts on the host and they are written
 *     back to the device (one round trip a step).  The MTP chain still runs
 *     (the reference skips it when the hook is set).
 *   - The sampler's scratch is not needed (pass NULL or any buffer); the
 *     caller's ApusRng is advanced by the tokens each step draws, as the
 *     reference's apus_sample calls would advance it.
 * Errors: 0 / -1 (+ err text where the reference fills err), NULL from
 * allocators, apus_gspec_step returns 0 at capacity or failure; the last
 * error string is apus_gcuda_last_error() (apus_gcuda.h).
 */
#ifndef APUS_GSPEC_GCUDA_H
#define APUS_GSPEC_GCUDA_H

#include <stddef.h>
#include <stdint.h>

#include "apus_gcuda.h"
#include "apus_gmtp_gcuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* c/sample.h:57-59 */
typedef struct { uint64_t s; } ApusRng;
void apus_rng_seed(ApusRng *r, uint64_t seed);
size_t apus_sample_scratch_size(size_t n);   /* c/sample.h:39 (the buffer is unused here) */

/* c/gmodel.h:88-108: same field names (the per-layer patterns inline) */
typedef ApusGcudaConfig ApusGmodelConfig;

typedef struct ApusGmodel ApusGmodel;             /* c/gmodel.h:129 */
typedef struct ApusGmodelState ApusGmodelState;   /* c/gmodel.h:239 */

/* c/gmodel.h:143-160 (accepted, unused: every expert is resident) */
typedef struct {
    int tiered;
    size_t cache_bytes;
    int slots_per_layer;
    int io_threads;
    int nocache;
    size_t rss_budget_bytes;
    int want_mtp;
} ApusGmodelTierCfg;

/* c/gmodel.h:138-141, :161-164: config_path NULL = <dir>/config.json */
ApusGmodel *apus_gmodel_open(const char *container_dir, const char *config_path, char *err, size_t errcap);
ApusGmodel *apus_gmodel_open2(const char *container_dir, const char *config_path, const ApusGmodelTierCfg *tier,
                              char *err, size_t errcap);
void apus_gmodel_close(ApusGmodel *m);                                  /* c/gmodel.h:165 */
const ApusGmodelConfig *apus_gmodel_config(const ApusGmodel *m);        /* c/gmodel.h:170 */
int apus_gmodel_has_mtp(const ApusGmodel *m);                           /* c/gmodel.h:193 */
/* c/gmodel.h:244-248: uploads the weights (one state per model at a time) */
ApusGmodelState *apus_gmodel_state_new(const ApusGmodel *m, size_t kv_cap);
void apus_gmodel_state_free(ApusGmodelState *st);
size_t apus_gmodel_pos(const ApusGmodelState *st);
size_t apus_gmodel_state_cap(const ApusGmodelState *st);
/* The B200 model behind a state (for the apus_gmtp_gcuda.h calls). */
ApusGcudaModel *apus_gmodel_state_gcuda(ApusGmodelState *st);

/* c/gmtp.h:123-135 */
typedef struct {
    const ApusGmodel *m;
    int layer;        /* the MTP block's layer id (num_hidden_layers) */
    size_t dim;
    int V;
} ApusGmtp;
int apus_gmtp_bind(ApusGmtp *mt, const ApusGmodel *m, char *err, size_t errcap);

typedef struct ApusGmtpState ApusGmtpState;   /* c/gmtp.h:137-145 (opaque here) */
ApusGmtpState *apus_gmtp_state_new(const ApusGmtp *mt, size_t kv_cap);
void apus_gmtp_state_free(ApusGmtpState *st);

/* c/gmtp.h:202-243: the public fields of the reference, then this engine's */
typedef struct ApusGspec {
    ApusGmodel *m;
    ApusGmodelState *st;
    const ApusGmtp *mt;
    ApusGmtpState *mst;
    int depth;
    float temp, top_p;
    ApusRng *rng;
    void *sample_scratch;
    void (*draft_override)(void *ctx, int64_t q, int32_t *drafts, int n);
    void *draft_ctx;
    uint64_t emitted;
    uint64_t batches;
    uint64_t batch_tokens;
    uint64_t refeed_tokens;
    uint64_t offered;
    uint64_t accepted;
    uint64_t d1_offered, d1_hits;
    /* internals (opaque to callers) */
    size_t q;         /* position of the held token */
    int32_t held;
    int32_t drafts[8];
    int sampling_set;
} ApusGspec;

/* c/gmtp.h:245-259 */
void apus_gspec_init(ApusGspec *sp, ApusGmodel *m, ApusGmodelState *st, const ApusGmtp *mt, ApusGmtpState *mst,
                     int depth, float temp, float top_p, ApusRng *rng, void *sample_scratch);
void apus_gspec_free(ApusGspec *sp);
int apus_gspec_prefill(ApusGspec *sp, const int32_t *ids, size_t n);
int apus_gspec_step(ApusGspec *sp, int *out, int cap);

/* Counters of the device control block (emitted, batches, offered,
 * accepted, position, held, d1_hits, d1_offered, refeed_tokens,
 * batch_tokens), read after synchronising; n <= 10. */
int apus_gcuda_gspec_counters(ApusGcudaModel *m, uint64_t *out, size_t n);

#ifdef __cplusplus
}
#endif
#endif
