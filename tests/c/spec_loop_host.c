/*
 * A C host of the speculative loop written against the reference's engine
 * API (the run_glm spec branch, c/apus.c:1016-1077: bind the MTP block,
 * make its state, init the spec engine, prefill, step until done, report
 * the ApusGspec counters, free), compiled against include/apus_gspec_gcuda.h
 * and linked with libapus_gcuda.so instead of the reference's
 * implementation (test build).
 *
 * spec_loop: prompt ids[n_ids], depth spec_k, up to max_tokens emitted into
 * out; stats[8] = emitted, batches, refeed_tokens, accepted, offered,
 * d1_hits, d1_offered, position.  force (optional, n_force tokens from
 * position force_base): a draft_override that proposes the true tokens, so
 * every draft is accepted.  Returns the token count, -1 on failure.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "apus_gspec_gcuda.h"

typedef struct {
    const int32_t *truth;
    int64_t n, base;
} Force;

static void force_truth(void *ctx, int64_t q, int32_t *drafts, int n) {
    const Force *f = (const Force *)ctx;
    /* d1 is compared with the held token (position q), d2.. are verified */
    for (int i = 0; i < n; i++) {
        const int64_t p = q + i - f->base;
        if (p >= 0 && p < f->n) drafts[i] = f->truth[p];
    }
}

int spec_loop(const char *dir, const int32_t *ids, int n_ids, int spec_k, int max_tokens, size_t kv_cap,
              const int32_t *force, int n_force, int32_t *out, uint64_t *stats, char *err, size_t errcap) {
    ApusGmodel *gm = apus_gmodel_open2(dir, NULL, NULL, err, errcap);
    if (!gm) return -1;
    ApusGmodelState *st = apus_gmodel_state_new(gm, kv_cap);
    if (!st) {
        snprintf(err, errcap, "state: %s", apus_gcuda_last_error());
        apus_gmodel_close(gm);
        return -1;
    }
    ApusGmtp mt;
    if (apus_gmtp_bind(&mt, gm, err, errcap)) {
        apus_gmodel_close(gm);
        return -1;
    }
    ApusGmtpState *mst = apus_gmtp_state_new(&mt, kv_cap + (size_t)spec_k);
    const int V = apus_gmodel_config(gm)->vocab_size;
    void *scratch = malloc(apus_sample_scratch_size((size_t)V));
    ApusRng rng;
    apus_rng_seed(&rng, 12345);
    ApusGspec sp;
    apus_gspec_init(&sp, gm, st, &mt, mst, spec_k, 0.0f, 1.0f, &rng, scratch);
    Force f = {force, n_force, n_ids};
    if (force) {
        sp.draft_override = force_truth;
        sp.draft_ctx = &f;
    }
    int n_gen = -1;
    if (apus_gspec_prefill(&sp, ids, (size_t)n_ids) == 0) {
        int step_out[64];
        n_gen = 0;
        while (n_gen < max_tokens) {
            const int ne = apus_gspec_step(&sp, step_out, 64);
            if (ne <= 0) break;
            for (int i = 0; i < ne && n_gen < max_tokens; i++) out[n_gen++] = step_out[i];
        }
        stats[0] = sp.emitted; stats[1] = sp.batches; stats[2] = sp.refeed_tokens; stats[3] = sp.accepted;
        stats[4] = sp.offered; stats[5] = sp.d1_hits; stats[6] = sp.d1_offered; stats[7] = apus_gmodel_pos(st);
    } else {
        snprintf(err, errcap, "prefill: %s", apus_gcuda_last_error());
    }
    apus_gspec_free(&sp);
    apus_gmtp_state_free(mst);
    free(scratch);
    apus_gmodel_close(gm);     /* frees the state too */
    return n_gen;
}
