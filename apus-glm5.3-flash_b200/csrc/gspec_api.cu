// gspec_api.cu — the reference's speculative-engine entry points
// (c/gmtp.h:123-259, c/gmodel.h:129-248, c/sample.h:39-59) over the B200
// engine, declared in include/apus_gspec_gcuda.h.  Host code only: every
// call forwards to the resident model of apus_gmtp_gcuda.h.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "gcuda.h"
#include "../../include/apus_gcuda.h"
#include "../../include/apus_gspec_gcuda.h"

// engine internals (model.cu)
int model_drafts_rw(ApusGcudaModel *m, int32_t *drafts, int n, int write);
int model_set_depth(ApusGcudaModel *m, int depth);
size_t model_cap(const ApusGcudaModel *m);

struct ApusGmodel {
    ApusGcudaConfig cfg;
    std::string dir;
    int has_mtp;
    ApusGmodelState *state;      // the one sequence bound to the resident weights
};

struct ApusGmodelState {
    ApusGmodel *owner;
    ApusGcudaModel *g;
};

struct ApusGmtpState {
    ApusGmodelState *st;
    size_t cap;
};

static void put_err(char *err, size_t cap, const char *msg) {
    if (err && cap) snprintf(err, cap, "%s", msg);
    gcuda_set_error("%s", msg);
}

extern "C" void apus_rng_seed(ApusRng *r, uint64_t seed) { r->s = seed; }

extern "C" size_t apus_sample_scratch_size(size_t n) { return n * (sizeof(float) + sizeof(int32_t)); }

extern "C" ApusGmodel *apus_gmodel_open2(const char *dir, const char *config_path, const ApusGmodelTierCfg *tier,
                                         char *err, size_t errcap) {
    (void)tier;
    if (!dir) { put_err(err, errcap, "gmodel_open: no container directory"); return nullptr; }
    std::string cp = config_path ? std::string(config_path) : std::string(dir) + "/config.json";
    ApusGmodel *m = new ApusGmodel();
    char e[512] = "";
    if (apus_gcuda_config_load(cp.c_str(), &m->cfg, e, sizeof e)) {
        put_err(err, errcap, e);
        delete m;
        return nullptr;
    }
    // the MTP block is loaded when the container carries it
    m->has_mtp = m->cfg.num_nextn_predict_layers > 0 &&
                 apus_gcuda_container_check(dir, &m->cfg, 1, e, sizeof e) >= 0;
    if (!m->has_mtp && apus_gcuda_container_check(dir, &m->cfg, 0, e, sizeof e) < 0) {
        put_err(err, errcap, e);
        delete m;
        return nullptr;
    }
    m->dir = dir;
    m->state = nullptr;
    return m;
}

extern "C" ApusGmodel *apus_gmodel_open(const char *dir, const char *config_path, char *err, size_t errcap) {
    return apus_gmodel_open2(dir, config_path, nullptr, err, errcap);
}

extern "C" void apus_gmodel_close(ApusGmodel *m) {
    if (!m) return;
    if (m->state) apus_gmodel_state_free(m->state);
    delete m;
}

extern "C" const ApusGmodelConfig *apus_gmodel_config(const ApusGmodel *m) { return &m->cfg; }

extern "C" int apus_gmodel_has_mtp(const ApusGmodel *m) { return m->has_mtp; }

extern "C" ApusGmodelState *apus_gmodel_state_new(const ApusGmodel *cm, size_t kv_cap) {
    ApusGmodel *m = const_cast<ApusGmodel *>(cm);
    if (m->state) { gcuda_set_error("gmodel_state_new: the model already has a sequence state"); return nullptr; }
    ApusGcudaModel *g = apus_gcuda_model_new(&m->cfg, m->has_mtp, kv_cap, 1);
    if (!g) return nullptr;
    char e[512] = "";
    if (apus_gcuda_model_load_container(g, m->dir.c_str(), e, sizeof e)) {
        gcuda_set_error("%s", e);
        apus_gcuda_model_free(g);
        return nullptr;
    }
    apus_gcuda_gspec_use_graph(g, 1);   // full-depth steps replay one captured graph
    ApusGmodelState *st = new ApusGmodelState{m, g};
    m->state = st;
    return st;
}

extern "C" void apus_gmodel_state_free(ApusGmodelState *st) {
    if (!st) return;
    if (st->owner && st->owner->state == st) st->owner->state = nullptr;
    apus_gcuda_model_free(st->g);
    delete st;
}

extern "C" size_t apus_gmodel_pos(const ApusGmodelState *st) { return apus_gcuda_model_pos(st->g); }

extern "C" size_t apus_gmodel_state_cap(const ApusGmodelState *st) { return model_cap(st->g); }

extern "C" ApusGcudaModel *apus_gmodel_state_gcuda(ApusGmodelState *st) { return st ? st->g : nullptr; }

extern "C" int apus_gmtp_bind(ApusGmtp *mt, const ApusGmodel *m, char *err, size_t errcap) {
    if (!m || !m->has_mtp) {
        put_err(err, errcap, "gmtp: model has no MTP block loaded");
        return -1;
    }
    mt->m = m;
    mt->layer = m->cfg.num_hidden_layers;
    mt->dim = (size_t)m->cfg.hidden_size;
    mt->V = m->cfg.vocab_size;
    return 0;
}

// The MTP block's caches live beside the main model's in the resident
// sequence state; this handle records the capacity the caller asked for.
extern "C" ApusGmtpState *apus_gmtp_state_new(const ApusGmtp *mt, size_t kv_cap) {
    if (!mt || !mt->m) { gcuda_set_error("gmtp_state_new: unbound ApusGmtp"); return nullptr; }
    return new ApusGmtpState{mt->m->state, kv_cap};
}

extern "C" void apus_gmtp_state_free(ApusGmtpState *st) { delete st; }

// Device counters -> the reference's ApusGspec fields; the caller's rng
// follows the device's stream state when sampling.
static int spec_sync(ApusGspec *sp) {
    ApusGcudaModel *g = sp->st->g;
    uint64_t c[10];
    if (apus_gcuda_gspec_counters(g, c, 10)) return -1;
    sp->emitted = c[0]; sp->batches = c[1]; sp->offered = c[2]; sp->accepted = c[3];
    sp->q = (size_t)c[4]; sp->held = (int32_t)(int64_t)c[5];
    sp->d1_hits = c[6]; sp->d1_offered = c[7]; sp->refeed_tokens = c[8]; sp->batch_tokens = c[9];
    if (sp->rng && sp->temp > 0.0f && apus_gcuda_rng_state(g, &sp->rng->s)) return -1;
    return 0;
}

// c/gmtp.h:211-215: the caller's hook edits the next drafts
static int spec_override(ApusGspec *sp) {
    if (!sp->draft_override) return 0;
    ApusGcudaModel *g = sp->st->g;
    if (model_drafts_rw(g, sp->drafts, sp->depth, 0)) return -1;
    sp->draft_override(sp->draft_ctx, (int64_t)sp->q, sp->drafts, sp->depth);
    return model_drafts_rw(g, sp->drafts, sp->depth, 1);
}

extern "C" void apus_gspec_init(ApusGspec *sp, ApusGmodel *m, ApusGmodelState *st, const ApusGmtp *mt,
                                ApusGmtpState *mst, int depth, float temp, float top_p, ApusRng *rng,
                                void *sample_scratch) {
    memset(sp, 0, sizeof *sp);
    sp->m = m; sp->st = st; sp->mt = mt; sp->mst = mst;
    sp->depth = depth < 1 ? 1 : (depth > 8 ? 8 : depth);
    sp->temp = temp; sp->top_p = top_p; sp->rng = rng; sp->sample_scratch = sample_scratch;
    sp->held = -1;
    if (!st || model_set_depth(st->g, sp->depth)) return;
    // the engine samples with the caller's stream state (greedy when temp <= 0)
    sp->sampling_set = apus_gcuda_gspec_sampling(st->g, temp, top_p, rng ? rng->s : 0) == 0;
}

extern "C" void apus_gspec_free(ApusGspec *sp) { (void)sp; }

extern "C" int apus_gspec_prefill(ApusGspec *sp, const int32_t *ids, size_t n) {
    if (!sp->st || !sp->sampling_set) { gcuda_set_error("gspec_prefill: spec not initialised"); return -1; }
    if (sp->rng && sp->temp > 0.0f &&
        apus_gcuda_gspec_sampling(sp->st->g, sp->temp, sp->top_p, sp->rng->s))
        return -1;
    if (apus_gcuda_gspec_prefill(sp->st->g, ids, n)) return -1;
    if (spec_sync(sp)) return -1;
    return spec_override(sp);
}

extern "C" int apus_gspec_step(ApusGspec *sp, int *out, int cap) {
    if (!sp->st || !sp->sampling_set) return 0;
    const int ne = apus_gcuda_gspec_step(sp->st->g, out, cap);
    if (ne <= 0) return 0;
    if (spec_sync(sp) || spec_override(sp)) return 0;
    return ne;
}
