// model.cu — the resident glm5_next model, its decode forward, the MTP head
// and the on-device speculative step (include/apus_gmtp_gcuda.h).
//
// HBM layout (chosen for one-launch decode GEMVs): per KDA layer the six
// projections that read the same normed input are one row-concatenated BF16
// matrix (q|k|v|f_a|g_a|b); per DSA layer q_a|kv_a are one FP8 matrix and
// the indexer's wk|compress_gate|weights_proj one BF16 matrix; MoE experts
// are packed per layer (see gmoe.cu); the dense MLP is the "shared expert"
// of an MoE with no routed experts.
//
// Speculative step (c/gmtp.h:776-891, greedy), all launches fixed-shape so no
// host round-trip happens inside a step:
//   k_spec_begin   batch = [held, d2..dD]
//   main forward   D rows at pos..pos+D-1, lm_head GEMV fused with argmax
//   MTP replay     D pairs (h_prev|yn[0..D-2], batch) at the MTP position;
//                  rows past the accepted prefix land in dead cache rows
//   k_spec_walk    accept walk, emit, commit pos/KDA checkpoint/MTP position,
//                  pick draft 1 and the chaining hidden of the accepted row
//   chain          D-1 single-row MTP forwards, each argmax -> next draft
// Rollback is a checkpoint-slot select for KDA (the recurrent kernel wrote
// the state after every row) and a position rewind for the DSA caches.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "gcuda.h"
#include "model_dev.h"
#include "../../include/apus_gcuda.h"
#include "../../include/apus_gmtp_gcuda.h"

// Rows of one prompt chunk.  Every prompt row takes the same arithmetic
// whatever the chunk size (the GEMM sums each row alike, the KDA chunks are
// the prompt's 64-row chunks, the DSA rows attend to positions <= their own),
// so this only trades memory for fewer weight passes.
#define PROMPT_ROWS 256

// ------------------------------------------------------------ device kernels
namespace apus {

__global__ void k_commit(Ctl *c, int R) {
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        c->pos += R;
        c->kda_cur = (c->kda_cur + R) % NSLOT;
    }
}

// The prompt pass leaves each KDA layer's state in the committed slot itself:
// only the position advances.
__global__ void k_commit_rows(Ctl *c, int R) {
    if (threadIdx.x == 0) c->pos += R;
}

__global__ void k_mtp_commit(Ctl *c, int R) {
    pdl_launch_dependents();
    if (threadIdx.x == 0) c->mtp_n += R;
}

// rows r < n0 -> dst[r], rows r >= n0 -> dst2[r - n0]
__global__ void k_extract_picks(const unsigned long long *keys, int R, int *dst, int n0, int *dst2) {
    pdl_launch_dependents();
    const int r = threadIdx.x;
    if (r >= R) return;
    const int v = (int)argmax_key_index(keys[r]);
    if (r < n0) dst[r] = v;
    else dst2[r - n0] = v;
}

// Step start.  A step whose rows would pass the capacity freezes the
// sequence (err) instead: the launches still run (into the slack rows past
// the capacity) but commit nothing.
__global__ void k_spec_begin(Ctl *c, int D, int cap, int32_t *ids) {
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        if (c->pos + D > cap) c->err = 1;
        c->batch[0] = c->held;
        for (int j = 1; j < D; j++) c->batch[j] = c->drafts[j];
        for (int j = 0; j < D; j++) ids[j] = c->batch[j];
    }
}

// MTP replay input rows: row 0 pairs the held token with the carried hnorm
// input of position q-1, row j the draft batch[j] with yn[j-1] (lag 1,
// postnorm source, c/gmtp.h:855-866).
__global__ void k_replay_rows(const uint16_t *hprev_carry, const uint16_t *yn, int D, int d, uint16_t *rows) {
    pdl_launch_dependents();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D * d; i += gridDim.x * blockDim.x) {
        const int r = i / d, e = i % d;
        rows[i] = r == 0 ? hprev_carry[e] : yn[(size_t)(r - 1) * d + e];
    }
}

// Accept walk (c/gmtp.h:807-831) and state fixup (:833-848, :867-884).
__global__ void k_spec_walk(Ctl *c, int D, int32_t *log, int log_cap) {
    pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    if (c->err) { c->n_emitted = 0; return; }
    c->stat_d1_offered++;
    if (c->drafts[0] == c->held) c->stat_d1_hits++;
    c->stat_batch_tokens += D;
    int matched = 0, last = -1;
    c->emitted[0] = c->held;
    for (int j = 1; j < D; j++) {
        const int x = c->picks[j - 1];
        c->stat_offered++;
        if (c->drafts[j] == x) { matched++; c->stat_accepted++; c->emitted[matched] = x; }
        else { last = x; break; }
    }
    if (last < 0) last = c->picks[D - 1];
    c->n_emitted = matched + 1;
    c->matched = matched;
    if (matched < D - 1) c->stat_refeed += matched + 1;
    for (int i = 0; i <= matched && c->log_n + i < log_cap; i++) log[c->log_n + i] = c->emitted[i];
    c->log_n += matched + 1;
    c->stat_emitted += matched + 1;
    c->stat_batches++;
    if (c->temp > 0.0f) c->rng_s += (unsigned long long)(matched + 1) * 0x9E3779B97F4A7C15ull;
    c->pos += matched + 1;
    c->kda_cur = (c->kda_cur + matched + 1) % NSLOT;
    c->held = last;
    // MTP: the replay wrote D rows at mtp_n; keep the accepted prefix
    c->mtp_n += matched + 1;
    c->drafts[0] = c->mtp_picks[matched];
    for (int i = 1; i < MAXR; i++) c->chain_pos[i] = c->mtp_n + i - 1;
}

__global__ void k_copy_row(const uint16_t *src, long row, int d, uint16_t *dst) {
    pdl_launch_dependents();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x)
        dst[i] = src[row * d + i];
}

// copy row `matched` (device-selected) of a [D][d] block
__global__ void k_copy_sel_row(const uint16_t *src, const Ctl *c, int d, uint16_t *dst) {
    pdl_launch_dependents();
    const int row = c->matched;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x)
        dst[i] = src[(size_t)row * d + i];
}

__global__ void k_chain_first(const Ctl *c, int32_t *ids) {
    pdl_launch_dependents();
    if (threadIdx.x == 0) ids[0] = c->drafts[0];
}

__global__ void k_chain_next(Ctl *c, int i, int32_t *ids) {
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        c->drafts[i] = c->mtp_picks[0];
        ids[0] = c->drafts[i];
    }
}

__device__ unsigned long long sm64(unsigned long long z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void k_force(Ctl *c, const int32_t *truth, int D, int V) {
    pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    for (int i = 0; i < D; i++) c->raw_drafts[i] = c->drafts[i];
    if (!c->force_on) return;
    for (int i = 0; i < D; i++) {
        const long pos = (long)c->pos + i - c->force_base;
        if (pos < 0 || pos >= c->force_n) continue;
        const double u = (double)(sm64(c->force_seed ^ (unsigned long long)(c->pos + i)) >> 11) * 0x1.0p-53;
        const int t = truth[pos];
        c->drafts[i] = u < c->force_p ? t : (t + 1) % V;
    }
}

__global__ void k_greedy_prep(Ctl *c, int32_t *ids) {
    pdl_launch_dependents();
    if (threadIdx.x == 0) ids[0] = c->held;
}

__global__ void k_greedy_post(Ctl *c, int32_t *log, int log_cap) {
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        if (c->log_n < log_cap) log[c->log_n] = c->held;
        c->log_n++;
        c->held = c->picks[0];
    }
}

// n sampled tokens consumed n splitmix64 draws (c/sample.h:173-177)
__global__ void k_rng_advance(Ctl *c, int n) {
    if (threadIdx.x == 0) c->rng_s += (unsigned long long)n * 0x9E3779B97F4A7C15ull;
}

__global__ void k_set_held_from_pick(Ctl *c, int row) {
    pdl_launch_dependents();
    if (threadIdx.x == 0) c->held = c->picks[row];
}

}  // namespace apus
using namespace apus;

// ------------------------------------------------------------------- host

struct ApusGcudaModel {
    ApusGcudaConfig cfg;
    Dims D;
    int has_mtp, depth, cap, nL;
    std::vector<LayerW> L;
    uint16_t *embed = nullptr, *norm = nullptr, *head = nullptr;
    uint16_t *enorm = nullptr, *hnorm = nullptr, *eh_proj = nullptr, *shared_norm = nullptr;
    std::vector<KdaState> kda;
    std::vector<DsaState> dsa;
    DsaState mtp_dsa{};
    Scratch S{};
    float *part = nullptr;
    int *tick = nullptr;
    Ctl *ctl = nullptr;
    int32_t *log = nullptr;
    int log_cap = 0;
    int32_t *truth = nullptr;
    Ctl force{};                         // forced-draft settings (survive reset)
    float temp = 0.0f, top_p = 1.0f;     // sampling settings (survive reset)
    int dbg_layer = -1, dbg_stage = -1;  // inspection stop inside main_forward
    int keep_logits = 0;                 // speculative steps also write the verify rows' logits
    uint16_t *yn_prompt = nullptr;       // [cap][d] post-norm rows of the prompt
    uint16_t *hcarry = nullptr, *hmtp = nullptr, *mtp_rows = nullptr;
    int32_t *ids = nullptr;
    cudaStream_t st = nullptr;
    std::vector<void *> allocs;
    // shared MoE scratch
    MoeDev moe_scr{};
    unsigned long long *moe_problems = nullptr;   // device counter (expert problems run)
    uint64_t n_main_fwd = 0, n_mtp_fwd = 0;       // forwards enqueued (host count)
    cudaGraph_t graph = nullptr;                  // captured full-depth step
    cudaGraphExec_t gexec = nullptr;
    int use_graph = 0;
    size_t graph_kernels = 0;
    // the control block as the last synchronous step read it back, valid
    // while no other work has touched the control block since (ctl_epoch
    // counts the calls that do)
    Ctl ctl_cache{};
    uint64_t ctl_epoch = 0, cache_epoch = ~0ull;
    // expert / vocabulary parallelism (one process per GPU)
    int ep_rank = 0, ep_world = 1;
    EpCtx ep{};
    uint8_t *ep_region = nullptr;             // this rank's exchange region
    void *ep_opened[EP_MAX_RANKS] = {};       // peers' regions opened through IPC
    long v0 = 0, vn = 0;                      // this rank's lm_head rows [v0, v0+vn)
    // the prompt pass's row buffers (allocated by the first prompt)
    struct Wide {
        int W = 0;                            // rows of one prompt chunk
        uint16_t *h4 = nullptr, *h4b = nullptr;   // [W][hc*d]
        uint16_t *x = nullptr, *sub = nullptr;    // [W][d]
        float *mix = nullptr, *post = nullptr, *comb = nullptr;
        KdaRows kda{};
        DsaRows dsa{};
        MlpRows mlp{};
        MoeRows moe{};                        // one GPU: the MoE over all the chunk's rows
        uint16_t *eh = nullptr, *mx = nullptr, *mxn = nullptr, *oh = nullptr;   // MTP block rows
        uint16_t *wbuf = nullptr;             // one FP8 matrix dequantised to BF16
        int32_t *ids = nullptr;               // [cap] prompt ids
        int *pos = nullptr;                   // 0, 1, 2, ... (row positions)
    } wide;
};

static void *dmalloc(ApusGcudaModel *m, size_t n, bool zero = true) {
    void *p = nullptr;
    if (cudaMalloc(&p, n ? n : 16) != cudaSuccess) return nullptr;
    if (zero) cudaMemset(p, 0, n ? n : 16);
    m->allocs.push_back(p);
    return p;
}

static Dims dims_of(const ApusGcudaConfig &c) {
    Dims D{};
    D.d = c.hidden_size; D.V = c.vocab_size; D.L = c.num_hidden_layers; D.hc = c.hc_mult;
    D.eps = c.rms_norm_eps; D.hc_eps = c.hc_eps; D.lower_bound = c.linear_lower_bound;
    D.route_scale = c.routed_scaling_factor; D.limit = c.swiglu_limit; D.sinkhorn_iters = c.hc_sinkhorn_iters;
    D.H = c.linear_num_heads; D.D = c.linear_head_dim; D.Dr = c.linear_head_dim; D.K = c.linear_conv_kernel_dim;
    D.qkv = D.H * D.D;
    D.AH = c.num_attention_heads; D.qd = c.qk_nope_head_dim; D.vd = c.v_head_dim; D.ql = c.q_lora_rank;
    D.kl = c.kv_lora_rank; D.IH = c.index_n_heads; D.ID = c.index_head_dim; D.topk = c.index_topk;
    D.kpool = c.index_kpool; D.tail = c.index_kpool_always_select_tail;
    D.E = c.n_routed_experts; D.ktop = c.num_experts_per_tok; D.inter = c.moe_intermediate_size;
    D.dense_inter = c.intermediate_size;
    return D;
}

// MoE weights + per-layer views into the shared scratch
// The router is replicated; the routed experts are split evenly over the
// expert-parallel ranks (this rank keeps [e0, e0+eloc) in local slots
// 0..eloc-1) and the shared expert sits in local slot eloc on every rank.
static bool alloc_moe(ApusGcudaModel *m, MoeDev &md, int E, int topk, int inter) {
    const Dims &D = m->D;
    md = m->moe_scr;
    md.E = E; md.topk = topk; md.inter = inter; md.dim = D.d; md.max_r = MAXR; md.pdl = 1;
    md.route_scale = D.route_scale; md.limit = D.limit;
    md.eloc = E / m->ep_world;
    md.e0 = md.eloc * m->ep_rank;
    md.ep = m->ep;
    const int L = md.eloc + 1;                // local expert slots
    const size_t nkd = (D.d + 127) / 128, nki = (inter + 127) / 128;
    md.gate_w = E ? (uint16_t *)dmalloc(m, (size_t)E * D.d * 2) : nullptr;
    md.gate_bias = E ? (float *)dmalloc(m, (size_t)E * 4) : nullptr;
    md.gu_codes = (uint8_t *)dmalloc(m, (size_t)L * 2 * inter * D.d, false);
    md.gu_scales = (float *)dmalloc(m, (size_t)L * (2 * inter / 128) * nkd * 4, false);
    md.d_codes = (uint8_t *)dmalloc(m, (size_t)L * D.d * inter, false);
    md.d_scales = (float *)dmalloc(m, (size_t)L * nkd * nki * 4, false);
    return md.gu_codes && md.gu_scales && md.d_codes && md.d_scales && (!E || (md.gate_w && md.gate_bias));
}

static bool alloc_dsa_w(ApusGcudaModel *m, DsaW &w) {
    const Dims &D = m->D;
    const size_t nkd = (D.d + 127) / 128;
    w.qkva_c = (uint8_t *)dmalloc(m, (size_t)(D.ql + D.kl) * D.d, false);
    w.qkva_s = (float *)dmalloc(m, (size_t)((D.ql + D.kl) / 128) * nkd * 4, false);
    w.q_a_norm = (uint16_t *)dmalloc(m, (size_t)D.ql * 2);
    w.kv_a_norm = (uint16_t *)dmalloc(m, (size_t)D.kl * 2);
    w.q_b_c = (uint8_t *)dmalloc(m, (size_t)D.AH * D.qd * D.ql, false);
    w.q_b_s = (float *)dmalloc(m, (size_t)((D.AH * D.qd + 127) / 128) * ((D.ql + 127) / 128) * 4, false);
    w.kv_b = (uint16_t *)dmalloc(m, (size_t)D.AH * (D.qd + D.vd) * D.kl * 2, false);
    w.o_c = (uint8_t *)dmalloc(m, (size_t)D.d * D.AH * D.vd, false);
    w.o_s = (float *)dmalloc(m, nkd * (((size_t)D.AH * D.vd + 127) / 128) * 4, false);
    w.idx_wq_b = (uint16_t *)dmalloc(m, (size_t)D.IH * D.ID * D.ql * 2, false);
    w.idx_kgw = (uint16_t *)dmalloc(m, (size_t)(2 * D.ID + D.IH) * D.d * 2, false);
    w.idx_knorm_w = (uint16_t *)dmalloc(m, (size_t)D.ID * 2);
    w.idx_knorm_b = (uint16_t *)dmalloc(m, (size_t)D.ID * 2);
    w.idx_ape = (uint16_t *)dmalloc(m, (size_t)D.kpool * D.ID * 2);
    return w.qkva_c && w.qkva_s && w.q_b_c && w.kv_b && w.o_c && w.idx_wq_b && w.idx_kgw && w.idx_ape;
}

// DSA caches hold SLACK rows past the sequence capacity: the MTP draft chain
// runs up to depth-1 rows ahead of the committed position, and a step that
// overruns the capacity (frozen by k_spec_begin) still writes its rows.
#define SLACK (3 * MAXR)
static bool alloc_dsa_state(ApusGcudaModel *m, DsaState &s) {
    const Dims &D = m->D;
    const size_t rows = (size_t)m->cap + SLACK;
    s.cap = (int)rows;
    s.k = (uint16_t *)dmalloc(m, (size_t)D.AH * rows * D.qd * 2);
    s.v = (uint16_t *)dmalloc(m, (size_t)D.AH * rows * D.vd * 2);
    s.ik = (uint16_t *)dmalloc(m, rows * D.ID * 2);
    s.ig = (uint16_t *)dmalloc(m, rows * D.ID * 2);
    s.pkey = (uint16_t *)dmalloc(m, (rows / D.kpool + 1) * D.ID * 2);
    return s.k && s.v && s.ik && s.ig && s.pkey;
}

static void model_release(ApusGcudaModel *m) {
    if (!m) return;
    if (m->st) cudaStreamSynchronize(m->st);
    if (m->gexec) cudaGraphExecDestroy(m->gexec);
    if (m->graph) cudaGraphDestroy(m->graph);
    if (m->st) cudaStreamDestroy(m->st);
    for (int p = 0; p < EP_MAX_RANKS; p++)
        if (m->ep_opened[p]) cudaIpcCloseMemHandle(m->ep_opened[p]);
    for (void *p : m->allocs) cudaFree(p);
    delete m;
}

static ApusGcudaModel *model_create(const ApusGcudaConfig *cfg, int has_mtp, size_t kv_cap, int depth, int rank,
                                    int world) {
    char err[128];
    if (apus_gcuda_enable(err, sizeof err)) return nullptr;
    const Dims D = dims_of(*cfg);
    bool any_kda = false;
    for (int l = 0; l < D.L && l < APUS_GCUDA_MAX_LAYERS; l++) any_kda |= !cfg->layer_is_dsa[l];
    if (depth < 1 || depth > MAXR || D.L < 1 || D.L > APUS_GCUDA_MAX_LAYERS || (any_kda && D.D != 128) ||
        D.hc < 1 || D.hc > 8 || cfg->n_shared_experts != 1 || D.kpool < 1 || D.ktop > D.E ||
        D.d % 128 || D.d > 8192 || D.qd > 256 || D.qd % 32 || D.vd % 32 || D.IH > 32 || D.ID > 128 ||
        D.kpool > 16 || D.ql % 128 || D.kl % 128 || D.inter % 128 || D.dense_inter % 128 || D.E > MOE_MAX_E ||
        D.ktop > MOE_MAX_TOPK || kv_cap < 16) {
        gcuda_set_error("gmodel: unsupported configuration");
        return nullptr;
    }
    if (world < 1 || world > EP_MAX_RANKS || rank < 0 || rank >= world ||
        (world > 1 && (D.E % world || D.ktop > MOE_MAX_TOPK || D.V < world))) {
        gcuda_set_error("gmodel: expert-parallel split needs experts divisible by the %d ranks", world);
        return nullptr;
    }
    if (layers_prepare(D)) {
        cudaGetLastError();
        gcuda_set_error("gmodel: unsupported layer shapes");
        return nullptr;
    }
    ApusGcudaModel *m = new ApusGcudaModel();
    m->cfg = *cfg;
    m->D = D;
    m->has_mtp = has_mtp ? 1 : 0;
    m->depth = depth;
    m->cap = (int)kv_cap;
    m->nL = D.L + m->has_mtp;
    m->ep_rank = rank;
    m->ep_world = world;
    {   // vocabulary rows of this rank's lm_head slice
        const long per = ((long)D.V + world - 1) / world;
        m->v0 = per * rank < D.V ? per * rank : D.V;
        m->vn = (m->v0 + per < D.V ? m->v0 + per : D.V) - m->v0;
    }
    bool ok = cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) == cudaSuccess;
    // shared scratch (all layers run one after another on one stream)
    Scratch &S = m->S;
    const int R = MAXR, d = D.d, qkv = D.qkv, ldkp = kda_ldkp(D);
    auto A = [&](size_t n) { void *p = dmalloc(m, n); ok = ok && p; return p; };
    S.h4 = (uint16_t *)A((size_t)R * D.hc * d * 2);
    S.h4b = (uint16_t *)A((size_t)R * D.hc * d * 2);
    S.x = (uint16_t *)A((size_t)R * d * 2);
    S.sub = (uint16_t *)A((size_t)R * d * 2);
    S.mix = (float *)A((size_t)R * hc_nchunk(D) * ((2 + D.hc) * D.hc + 1) * 4);   // pre-mix partials
    S.post = (float *)A((size_t)R * D.hc * 4);
    S.comb = (float *)A((size_t)R * D.hc * D.hc * 4);
    S.kp = (uint16_t *)A((size_t)R * ldkp * 2);
    S.fgo = (uint16_t *)A((size_t)2 * R * qkv * 2);
    S.qkvc = (uint16_t *)A((size_t)R * 3 * qkv * 2);
    S.core = (uint16_t *)A((size_t)R * qkv * 2);
    S.qkva = (uint16_t *)A((size_t)R * (D.ql + D.kl) * 2);
    S.qres = (uint16_t *)A((size_t)R * D.ql * 2);
    S.kpass = (uint16_t *)A((size_t)R * D.kl * 2);
    S.q = (uint16_t *)A((size_t)R * D.AH * D.qd * 2);
    S.kvb = (uint16_t *)A((size_t)R * D.AH * (D.qd + D.vd) * 2);
    S.iq = (uint16_t *)A((size_t)R * D.IH * D.ID * 2);
    S.ikgw = (uint16_t *)A((size_t)R * (2 * D.ID + D.IH) * 2);
    S.maxpools = (m->cap + SLACK) / D.kpool + 1;
    S.iscore = (float *)A((size_t)R * S.maxpools * 4);
    S.isel = (uint8_t *)A((size_t)R * S.maxpools);
    S.attn = (uint16_t *)A((size_t)R * D.AH * D.vd * 2);
    // scores row: every position a call can see, plus a full attention tile
    // past it (the tile loader reads whole tiles), in 16-byte units
    S.attn_sstride = (m->cap + SLACK + MAXR + 128 + 7) & ~7;
    S.attn_scores = (float *)A((size_t)D.AH * R * S.attn_sstride * 4);
    S.attn_p = (uint16_t *)A((size_t)D.AH * R * S.attn_sstride * 2);
    S.yn = (uint16_t *)A((size_t)R * d * 2);
    S.logits = (uint16_t *)A((size_t)R * D.V * 2);
    S.amax = (unsigned long long *)A(R * 8);
    S.ids = (int32_t *)A(R * 4);
    S.eh = (uint16_t *)A((size_t)R * 2 * d * 2);
    S.mx = (uint16_t *)A((size_t)R * d * 2);
    S.mxn = (uint16_t *)A((size_t)R * d * 2);
    S.oh = (uint16_t *)A((size_t)R * d * 2);
    S.hprev = (uint16_t *)A((size_t)R * d * 2);
    S.two_problems = (int *)A(3 * sizeof(int));
    if (ok) {
        const int tp[3] = {0, 1, 2};
        ok = cudaMemcpy(S.two_problems, tp, sizeof tp, cudaMemcpyHostToDevice) == cudaSuccess;
    }
    // split-K scratch sized for the largest split GEMV: K up to 4 ranges of
    // 4096 over up to V rows
    {
        size_t pf1, nt1, pf2, nt2;
        gemv_scratch_need(D.V, 2L * d, &pf1, &nt1);
        gemv_scratch_need(16384, (long)D.AH * D.vd > qkv ? (long)D.AH * D.vd : qkv, &pf2, &nt2);
        size_t pf = pf1 > pf2 ? pf1 : pf2, nt = nt1 > nt2 ? nt1 : nt2;
        const size_t pd = (size_t)d / 16 * 4 * 128;
        if (pf < pd) pf = pd;
        if (nt < (size_t)d / 16) nt = d / 16;
        m->part = (float *)A(pf * 4);
        m->tick = (int *)A(nt * 4);
    }
    m->ctl = (Ctl *)A(sizeof(Ctl));
    m->ep.rank = rank;
    m->ep.world = world;
    if (world > 1) {   // this rank's exchange region (peers open it through IPC)
        const size_t contrib = (size_t)2 * MOE_MAX_R * MOE_MAX_TOPK * d * 2;
        const size_t rb0 = (ep_region_bytes(d) + 255) & ~(size_t)255;
        const int wk = D.ktop > 0 ? D.ktop : 1;
        const size_t rbw = rb0 + ep_wide_bytes(PROMPT_ROWS, wk, d);   // + the prompt pass's outputs
        const size_t rb = rbw + (size_t)MOE_MAX_R * D.V * 2;            // + lm_head logits rows
        m->ep.off_wide = (long)rb0;
        m->ep.off_logits = (long)rbw;
        m->ep.vocab = D.V;
        m->ep.wide_rows = PROMPT_ROWS;
        m->ep.wide_k = wk;
        m->ep_region = (uint8_t *)A(rb > (2u << 20) ? rb : (2u << 20));   // its own IPC-mappable allocation
        m->ep.peer[rank] = m->ep_region;
        m->ep.off_keys = (long)contrib;
        m->ep.off_flags = (long)(contrib + 2 * MOE_MAX_R * 8);
        m->ep.epoch = (int *)A(2 * sizeof(int));     // epoch, CTA arrivals
    }
    m->log_cap = m->cap + 2 * MAXR;
    m->log = (int32_t *)A((size_t)m->log_cap * 4);
    m->yn_prompt = (uint16_t *)A((size_t)(m->cap + MAXR) * d * 2);
    m->hcarry = (uint16_t *)A((size_t)d * 2);
    m->hmtp = (uint16_t *)A((size_t)d * 2);
    m->mtp_rows = (uint16_t *)A((size_t)R * d * 2);
    m->ids = (int32_t *)A(R * 4);
    // MoE scratch shared by every sparse layer
    {
        MoeDev &ms = m->moe_scr;
        m->moe_problems = (unsigned long long *)A(sizeof(unsigned long long));
        ms.stat_problems = m->moe_problems;
        ms.part = m->part;       // the router GEMV shares the model's split-K scratch
        ms.tick = m->tick;
        const int maxi = D.inter > D.dense_inter ? D.inter : D.dense_inter;
        const size_t P = (size_t)R * (D.ktop > 0 ? D.ktop : 1) + 1;
        ms.logits = (float *)A((size_t)R * (D.E > 0 ? D.E : 1) * 4);
        ms.row_expert = (int32_t *)A((size_t)R * MOE_MAX_TOPK * 4);
        ms.row_weight = (float *)A((size_t)R * MOE_MAX_TOPK * 4);
        ms.row_sel = (int32_t *)A((size_t)R * MOE_MAX_TOPK * 4);
        ms.row_prob = (int32_t *)A((size_t)R * MOE_MAX_TOPK * 4);
        ms.row_prob_shared = (int32_t *)A((size_t)R * 4);
        ms.prob_slot = world > 1 ? (int32_t *)A(P * 8 * 4) : nullptr;
        ms.prob_expert = (int32_t *)A(P * 4);
        ms.prob_count = (int32_t *)A(4);
        ms.gu = (uint16_t *)A(P * R * 2 * (size_t)maxi * 2);
        ms.yd = (uint16_t *)A(P * R * (size_t)d * 2);
    }
    // weights
    m->embed = (uint16_t *)A((size_t)D.V * d * 2);
    m->norm = (uint16_t *)A((size_t)d * 2);
    m->head = (uint16_t *)A((size_t)m->vn * d * 2);
    m->L.resize(m->nL);
    m->kda.resize(D.L);
    m->dsa.resize(D.L);
    const int mix = (2 + D.hc) * D.hc;
    for (int l = 0; l < m->nL && ok; l++) {
        LayerW &W = m->L[l];
        const bool mtp = l >= D.L;
        W.is_dsa = mtp ? 1 : cfg->layer_is_dsa[l];
        W.sparse = mtp ? 1 : cfg->mlp_is_sparse[l];
        W.input_norm = (uint16_t *)A((size_t)d * 2);
        W.post_norm = (uint16_t *)A((size_t)d * 2);
        if (!mtp)
            for (int s = 0; s < 2; s++) {
                W.hc_fn[s] = (uint16_t *)A((size_t)mix * D.hc * d * 2);
                W.hc_base[s] = (float *)A((size_t)mix * 4);
                W.hc_scale[s] = (float *)A(3 * 4);
            }
        if (!W.is_dsa) {
            W.kda.proj = (uint16_t *)A((size_t)kda_nproj(D) * d * 2);
            W.kda.fg_b = (uint16_t *)A((size_t)2 * qkv * D.Dr * 2);
            W.kda.conv = (uint16_t *)A((size_t)3 * qkv * D.K * 2);
            W.kda.A_log = (float *)A((size_t)D.H * 4);
            W.kda.dt_bias = (float *)A((size_t)qkv * 4);
            W.kda.o_norm = (uint16_t *)A((size_t)D.D * 2);
            W.kda.o_w = (uint16_t *)A((size_t)d * qkv * 2);
            m->kda[l].conv = (uint16_t *)A((size_t)NSLOT * 3 * qkv * (D.K - 1) * 2);
            m->kda[l].rec = (float *)A((size_t)NSLOT * D.H * D.D * D.D * 4);
        } else {
            ok = ok && alloc_dsa_w(m, W.dsa);
            if (!mtp) ok = ok && alloc_dsa_state(m, m->dsa[l]);
        }
        if (W.sparse) ok = ok && alloc_moe(m, W.moe, D.E, D.ktop, D.inter);
        else ok = ok && alloc_moe(m, W.moe, 0, 0, D.dense_inter);
    }
    if (m->has_mtp) {
        m->enorm = (uint16_t *)A((size_t)d * 2);
        m->hnorm = (uint16_t *)A((size_t)d * 2);
        m->eh_proj = (uint16_t *)A((size_t)d * 2 * d * 2);
        m->shared_norm = (uint16_t *)A((size_t)d * 2);
        ok = ok && alloc_dsa_state(m, m->mtp_dsa);
    }
    if (!ok) {
        gcuda_set_error("gmodel: device allocation failed");
        model_release(m);
        return nullptr;
    }
    apus_gcuda_model_reset(m);
    return m;
}

extern "C" ApusGcudaModel *apus_gcuda_model_new(const ApusGcudaConfig *cfg, int has_mtp, size_t kv_cap, int depth) {
    return model_create(cfg, has_mtp, kv_cap, depth, 0, 1);
}

extern "C" ApusGcudaModel *apus_gcuda_model_new_ep(const ApusGcudaConfig *cfg, int has_mtp, size_t kv_cap, int depth,
                                                   int rank, int world) {
    return model_create(cfg, has_mtp, kv_cap, depth, rank, world);
}

extern "C" int apus_gcuda_model_ep_handle(ApusGcudaModel *m, void *handle_out) {
    if (m->ep_world < 2) { gcuda_set_error("gmodel: not an expert-parallel model"); return -1; }
    cudaIpcMemHandle_t h;
    if (gcuda_check(cudaIpcGetMemHandle(&h, m->ep_region), "ep handle")) return -1;
    memcpy(handle_out, &h, sizeof h);
    return 0;
}

// Opens every peer's exchange region and points every MoE layer and the
// lm_head exchange at them.  A captured step graph is dropped (its launches
// hold the old pointers).
extern "C" int apus_gcuda_model_ep_connect(ApusGcudaModel *m, const void *handles) {
    if (m->ep_world < 2) { gcuda_set_error("gmodel: not an expert-parallel model"); return -1; }
    const cudaIpcMemHandle_t *h = (const cudaIpcMemHandle_t *)handles;
    for (int p = 0; p < m->ep_world; p++) {
        if (p == m->ep_rank || m->ep_opened[p]) continue;
        void *ptr = nullptr;
        if (gcuda_check(cudaIpcOpenMemHandle(&ptr, h[p], cudaIpcMemLazyEnablePeerAccess), "ep connect")) return -1;
        m->ep_opened[p] = ptr;
        m->ep.peer[p] = (uint8_t *)ptr;
    }
    m->moe_scr.ep = m->ep;
    for (LayerW &W : m->L) W.moe.ep = m->ep;
    if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = nullptr; }
    if (m->graph) { cudaGraphDestroy(m->graph); m->graph = nullptr; }
    return 0;
}

extern "C" void apus_gcuda_model_free(ApusGcudaModel *m) { model_release(m); }

// ---- tensor name -> packed device location --------------------------------

static int resolve_moe(const ApusGcudaModel *m, const MoeDev &md, const std::string &n, void **dst, size_t *want) {
    const size_t dim = m->D.d, inter = md.inter, E = md.E;
    const size_t nkd = (dim + 127) / 128, nki = (inter + 127) / 128;
    if (n == "mlp.gate.weight" && E) { *dst = (void *)md.gate_w; *want = E * dim * 2; return 0; }
    if (n == "mlp.gate.e_score_correction_bias" && E) { *dst = (void *)md.gate_bias; *want = E * 4; return 0; }
    int e = -1;
    char part[64] = {0}, kind[64] = {0};
    if (E && sscanf(n.c_str(), "mlp.experts.%d.%63[a-z]_proj.%63s", &e, part, kind) == 3) {
        if (e < 0 || e >= (int)E) return -1;
        if (e < md.e0 || e >= md.e0 + md.eloc) return 1;   // another rank's expert
        e -= md.e0;                                       // local slot
    } else if (E && sscanf(n.c_str(), "mlp.shared_experts.%63[a-z]_proj.%63s", part, kind) == 2) {
        e = md.eloc;
    } else if (!E && sscanf(n.c_str(), "mlp.%63[a-z]_proj.%63s", part, kind) == 2) {
        e = 0;     // dense MLP = the lone "shared" expert
    } else {
        return -1;
    }
    const bool scale = !strcmp(kind, "weight_scale_inv");
    if (!scale && strcmp(kind, "weight")) return -1;
    const size_t gus = (2 * inter / 128) * nkd, ds = nkd * nki;
    if (!strcmp(part, "gate") || !strcmp(part, "up")) {
        const int up = !strcmp(part, "up");
        if (scale) { *dst = (void *)(md.gu_scales + (size_t)e * gus + up * (inter / 128) * nkd); *want = (inter / 128) * nkd * 4; }
        else { *dst = (void *)(md.gu_codes + (size_t)e * 2 * inter * dim + up * inter * dim); *want = inter * dim; }
    } else if (!strcmp(part, "down")) {
        if (scale) { *dst = (void *)(md.d_scales + (size_t)e * ds); *want = ds * 4; }
        else { *dst = (void *)(md.d_codes + (size_t)e * dim * inter); *want = dim * inter; }
    } else {
        return -1;
    }
    return 0;
}

static int resolve(const ApusGcudaModel *m, const char *name, void **dst, size_t *want) {
    const Dims &D = m->D;
    const size_t d = D.d, V = D.V, qkv = D.qkv, Dr = D.Dr, H = D.H;
    std::string n(name);
    if (n == "embed_tokens.weight") { *dst = m->embed; *want = V * d * 2; return 0; }
    if (n == "norm.weight") { *dst = m->norm; *want = d * 2; return 0; }
    if (n == "lm_head.weight") { *dst = m->head; *want = V * d * 2; return 2; }   // vocabulary slice
    int l = -1, off = 0;
    if (sscanf(name, "layers.%d.%n", &l, &off) != 1 || off <= 0 || l < 0 || l >= m->nL) return -1;
    const LayerW &W = m->L[l];
    const bool mtp = l >= D.L;
    const std::string r = n.substr(off);
    const int mix = (2 + D.hc) * D.hc;
    auto is = [&](const char *s) { return r == s; };
    if (is("input_layernorm.weight")) { *dst = (void *)W.input_norm; *want = d * 2; return 0; }
    if (is("post_attention_layernorm.weight")) { *dst = (void *)W.post_norm; *want = d * 2; return 0; }
    if (mtp) {
        if (is("enorm.weight")) { *dst = m->enorm; *want = d * 2; return 0; }
        if (is("hnorm.weight")) { *dst = m->hnorm; *want = d * 2; return 0; }
        if (is("eh_proj.weight")) { *dst = m->eh_proj; *want = d * 2 * d * 2; return 0; }
        if (is("shared_head.norm.weight")) { *dst = m->shared_norm; *want = d * 2; return 0; }
    } else {
        for (int s = 0; s < 2; s++) {
            const std::string site = s ? "ffn" : "attn";
            if (r == "hc_" + site + "_fn") { *dst = (void *)W.hc_fn[s]; *want = (size_t)mix * D.hc * d * 2; return 0; }
            if (r == "hc_" + site + "_base") { *dst = (void *)W.hc_base[s]; *want = (size_t)mix * 4; return 0; }
            if (r == "hc_" + site + "_scale") { *dst = (void *)W.hc_scale[s]; *want = 3 * 4; return 0; }
        }
    }
    if (!W.is_dsa) {
        const KdaW &k = W.kda;
        uint16_t *proj = (uint16_t *)k.proj;
        if (is("self_attn.q_proj.weight")) { *dst = proj; *want = qkv * d * 2; return 0; }
        if (is("self_attn.k_proj.weight")) { *dst = proj + qkv * d; *want = qkv * d * 2; return 0; }
        if (is("self_attn.v_proj.weight")) { *dst = proj + 2 * qkv * d; *want = qkv * d * 2; return 0; }
        if (is("self_attn.f_a_proj.weight")) { *dst = proj + 3 * qkv * d; *want = Dr * d * 2; return 0; }
        if (is("self_attn.g_a_proj.weight")) { *dst = proj + (3 * qkv + Dr) * d; *want = Dr * d * 2; return 0; }
        if (is("self_attn.b_proj.weight")) { *dst = proj + (3 * qkv + 2 * Dr) * d; *want = H * d * 2; return 0; }
        if (is("self_attn.f_b_proj.weight")) { *dst = (void *)k.fg_b; *want = qkv * Dr * 2; return 0; }
        if (is("self_attn.g_b_proj.weight")) { *dst = (void *)(k.fg_b + qkv * Dr); *want = qkv * Dr * 2; return 0; }
        for (int p = 0; p < 3; p++) {
            const std::string nm = std::string("self_attn.") + "qkv"[p] + "_conv1d.weight";
            if (r == nm) { *dst = (void *)(k.conv + (size_t)p * qkv * D.K); *want = qkv * D.K * 2; return 0; }
        }
        if (is("self_attn.A_log")) { *dst = (void *)k.A_log; *want = H * 4; return 0; }
        if (is("self_attn.dt_bias")) { *dst = (void *)k.dt_bias; *want = qkv * 4; return 0; }
        if (is("self_attn.o_norm.weight")) { *dst = (void *)k.o_norm; *want = D.D * 2; return 0; }
        if (is("self_attn.o_proj.weight")) { *dst = (void *)k.o_w; *want = d * qkv * 2; return 0; }
    } else {
        const DsaW &w = W.dsa;
        const size_t ql = D.ql, kl = D.kl, nkd = (d + 127) / 128;
        const size_t aq = (size_t)D.AH * D.qd, av = (size_t)D.AH * D.vd;
        if (is("self_attn.q_a_proj.weight")) { *dst = (void *)w.qkva_c; *want = ql * d; return 0; }
        if (is("self_attn.q_a_proj.weight_scale_inv")) { *dst = (void *)w.qkva_s; *want = (ql / 128) * nkd * 4; return 0; }
        if (is("self_attn.kv_a_proj_with_mqa.weight")) { *dst = (void *)(w.qkva_c + ql * d); *want = kl * d; return 0; }
        if (is("self_attn.kv_a_proj_with_mqa.weight_scale_inv")) {
            *dst = (void *)(w.qkva_s + (ql / 128) * nkd); *want = (kl / 128) * nkd * 4; return 0;
        }
        if (is("self_attn.q_a_layernorm.weight")) { *dst = (void *)w.q_a_norm; *want = ql * 2; return 0; }
        if (is("self_attn.kv_a_layernorm.weight")) { *dst = (void *)w.kv_a_norm; *want = kl * 2; return 0; }
        if (is("self_attn.q_b_proj.weight")) { *dst = (void *)w.q_b_c; *want = aq * ql; return 0; }
        if (is("self_attn.q_b_proj.weight_scale_inv")) {
            *dst = (void *)w.q_b_s; *want = ((aq + 127) / 128) * ((ql + 127) / 128) * 4; return 0;
        }
        if (is("self_attn.kv_b_proj.weight")) { *dst = (void *)w.kv_b; *want = (aq + av) * kl * 2; return 0; }
        if (is("self_attn.o_proj.weight")) { *dst = (void *)w.o_c; *want = d * av; return 0; }
        if (is("self_attn.o_proj.weight_scale_inv")) { *dst = (void *)w.o_s; *want = nkd * ((av + 127) / 128) * 4; return 0; }
        if (is("self_attn.indexer.wq_b.weight")) { *dst = (void *)w.idx_wq_b; *want = (size_t)D.IH * D.ID * ql * 2; return 0; }
        if (is("self_attn.indexer.wk.weight")) { *dst = (void *)w.idx_kgw; *want = (size_t)D.ID * d * 2; return 0; }
        if (is("self_attn.indexer.index_kpool_compress_gate")) {
            *dst = (void *)(w.idx_kgw + (size_t)D.ID * d); *want = (size_t)D.ID * d * 2; return 0;
        }
        if (is("self_attn.indexer.weights_proj.weight")) {
            *dst = (void *)(w.idx_kgw + (size_t)2 * D.ID * d); *want = (size_t)D.IH * d * 2; return 0;
        }
        if (is("self_attn.indexer.k_norm.weight")) { *dst = (void *)w.idx_knorm_w; *want = D.ID * 2; return 0; }
        if (is("self_attn.indexer.k_norm.bias")) { *dst = (void *)w.idx_knorm_b; *want = D.ID * 2; return 0; }
        if (is("self_attn.indexer.index_kpool_compress_ape")) {
            *dst = (void *)w.idx_ape; *want = (size_t)D.kpool * D.ID * 2; return 0;
        }
    }
    return resolve_moe(m, W.moe, r, dst, want);
}

// The configuration a model was created with (the container loader's view).
int model_config_get(const ApusGcudaModel *m, ApusGcudaConfig *cfg, int *has_mtp) {
    if (!m) return -1;
    *cfg = m->cfg;
    *has_mtp = m->has_mtp;
    return 0;
}

// 1 = this rank stores the checkpoint tensor, 0 = another expert-parallel
// rank does, -1 = not a tensor of this model.
int model_tensor_here(const ApusGcudaModel *m, const char *name) {
    void *dst;
    size_t want;
    const int rc = resolve(m, name, &dst, &want);
    return rc < 0 ? -1 : rc == 1 ? 0 : 1;
}

// 0 = stored; 1 = another expert-parallel rank's expert (nothing stored);
// -1 = unknown tensor or wrong size.  The lm_head is stored as this rank's
// vocabulary rows of the full host tensor.
extern "C" int apus_gcuda_model_set(ApusGcudaModel *m, const char *name, const void *host, size_t bytes) {
    void *dst;
    size_t want;
    const int rc = resolve(m, name, &dst, &want);
    if (rc == 1) return 1;
    if (rc < 0) { gcuda_set_error("gmodel: unknown tensor %s", name); return -1; }
    if (bytes != want) { gcuda_set_error("gmodel: %s has %zu bytes, expected %zu", name, bytes, want); return -1; }
    if (rc == 2) {
        const size_t row = (size_t)m->D.d * 2;
        return gcuda_check(cudaMemcpy(dst, (const uint8_t *)host + m->v0 * row, m->vn * row, cudaMemcpyHostToDevice),
                           "gmodel set");
    }
    return gcuda_check(cudaMemcpy(dst, host, bytes, cudaMemcpyHostToDevice), "gmodel set");
}

extern "C" int apus_gcuda_model_get(ApusGcudaModel *m, const char *name, void *host, size_t bytes) {
    void *src;
    size_t want;
    const int rc = resolve(m, name, &src, &want);
    if (rc == 1) return 1;
    if (rc < 0 || bytes != want) { gcuda_set_error("gmodel: bad get %s", name); return -1; }
    cudaStreamSynchronize(m->st);
    if (rc == 2) {   // this rank's rows, at their place in the full tensor
        const size_t row = (size_t)m->D.d * 2;
        return gcuda_check(cudaMemcpy((uint8_t *)host + m->v0 * row, src, m->vn * row, cudaMemcpyDeviceToHost),
                           "gmodel get");
    }
    return gcuda_check(cudaMemcpy(host, src, bytes, cudaMemcpyDeviceToHost), "gmodel get");
}

// ---- synthetic weights ------------------------------------------------------

extern "C" int apus_gcuda_model_init_random(ApusGcudaModel *m, uint64_t seed) {
    const Dims &D = m->D;
    const size_t d = D.d, qkv = D.qkv;
    uint64_t sid = 100;
    int rc = 0;
    cudaStream_t st = m->st;
    auto bf16n = [&](const void *p, size_t n, float std, float mean = 0.f) {
        rc |= fill_launch(FILL_BF16_NORMAL, (void *)p, n, seed, sid++, std, mean, st);
    };
    auto f32n = [&](const void *p, size_t n, float std, float mean = 0.f) {
        rc |= fill_launch(FILL_F32_NORMAL, (void *)p, n, seed, sid++, std, mean, st);
    };
    auto fp8 = [&](const void *c, const void *s, size_t n, size_t ns) {  // BASELINE config-0/1 FP8 blocks
        rc |= fill_launch(FILL_E4M3_NORMAL, (void *)c, n, seed, sid++, 64.f, 0.f, st);
        rc |= fill_launch(FILL_F32_LOGUNIFORM, (void *)s, ns, seed, sid++, 1e-4f, 1e-2f, st);
    };
    // Expert blocks of an MoE layer: one random stream over the (E+1) experts
    // of the whole model; this rank draws its routed slice [e0, e0+eloc) and
    // the shared expert E, so every rank count yields the same weights.
    auto fp8_experts = [&](const MoeDev &md, const uint8_t *c, const float *s, size_t per, size_t per_s) {
        const size_t E = md.E, e0 = md.e0, el = md.eloc;
        rc |= fill_launch(FILL_E4M3_NORMAL, (void *)c, el * per, seed, sid, 64.f, 0.f, st, e0 * per);
        rc |= fill_launch(FILL_E4M3_NORMAL, (void *)(c + el * per), per, seed, sid, 64.f, 0.f, st, E * per);
        sid++;
        rc |= fill_launch(FILL_F32_LOGUNIFORM, (void *)s, el * per_s, seed, sid, 1e-4f, 1e-2f, st, e0 * per_s);
        rc |= fill_launch(FILL_F32_LOGUNIFORM, (void *)(s + el * per_s), per_s, seed, sid, 1e-4f, 1e-2f, st,
                          E * per_s);
        sid++;
    };
    auto norm = [&](const void *p, size_t n) { bf16n(p, n, 0.05f, 1.0f); };
    bf16n(m->embed, (size_t)D.V * d, 0.02f);          // BASELINE: N(0, 0.02) embeddings and head
    rc |= fill_launch(FILL_BF16_NORMAL, m->head, (size_t)m->vn * d, seed, sid++, 0.02f, 0.f, st, (size_t)m->v0 * d);
    norm(m->norm, d);
    const int mix = (2 + D.hc) * D.hc;
    for (int l = 0; l < m->nL; l++) {
        LayerW &W = m->L[l];
        const bool mtp = l >= D.L;
        norm(W.input_norm, d);
        norm(W.post_norm, d);
        if (!mtp)
            for (int s = 0; s < 2; s++) {
                bf16n(W.hc_fn[s], (size_t)mix * D.hc * d, 1.0f / sqrtf((float)(D.hc * d)));
                f32n(W.hc_base[s], mix, 0.25f);
                f32n(W.hc_scale[s], 3, 0.1f, 1.0f);
            }
        if (!W.is_dsa) {
            bf16n(W.kda.proj, (size_t)kda_nproj(D) * d, 1.0f / sqrtf((float)d));
            bf16n(W.kda.fg_b, 2 * qkv * D.Dr, 1.0f / sqrtf((float)D.Dr));
            bf16n(W.kda.conv, 3 * qkv * D.K, 0.25f);
            f32n(W.kda.A_log, D.H, 0.5f);
            f32n(W.kda.dt_bias, qkv, 0.5f);
            norm(W.kda.o_norm, D.D);
            bf16n(W.kda.o_w, d * qkv, 1.0f / sqrtf((float)qkv));
        } else {
            const DsaW &w = W.dsa;
            const size_t nkd = (d + 127) / 128, aq = (size_t)D.AH * D.qd, av = (size_t)D.AH * D.vd;
            fp8(w.qkva_c, w.qkva_s, (size_t)(D.ql + D.kl) * d, ((D.ql + D.kl) / 128) * nkd);
            fp8(w.q_b_c, w.q_b_s, aq * D.ql, ((aq + 127) / 128) * ((D.ql + 127) / 128));
            fp8(w.o_c, w.o_s, d * av, nkd * ((av + 127) / 128));
            norm(w.q_a_norm, D.ql);
            norm(w.kv_a_norm, D.kl);
            bf16n(w.kv_b, (aq + av) * D.kl, 1.0f / sqrtf((float)D.kl));
            bf16n(w.idx_wq_b, (size_t)D.IH * D.ID * D.ql, 1.0f / sqrtf((float)D.ql));
            bf16n(w.idx_kgw, (size_t)(2 * D.ID + D.IH) * d, 1.0f / sqrtf((float)d));
            norm(w.idx_knorm_w, D.ID);
            bf16n(w.idx_knorm_b, D.ID, 0.05f);
            bf16n(w.idx_ape, (size_t)D.kpool * D.ID, 0.05f);
        }
        MoeDev &md = W.moe;
        const size_t nkd = (d + 127) / 128, nki = (md.inter + 127) / 128;
        if (md.E) {
            bf16n(md.gate_w, (size_t)md.E * d, 0.02f);           // N(0, 0.02), bias 0
            rc |= fill_launch(FILL_F32_CONST, (void *)md.gate_bias, md.E, seed, sid++, 0.f, 0.f, st);
        }
        fp8_experts(md, md.gu_codes, md.gu_scales, 2 * md.inter * d, (2 * md.inter / 128) * nkd);
        fp8_experts(md, md.d_codes, md.d_scales, d * md.inter, nkd * nki);
    }
    if (m->has_mtp) {
        norm(m->enorm, d);
        norm(m->hnorm, d);
        bf16n(m->eh_proj, d * 2 * d, 1.0f / sqrtf((float)(2 * d)));
        norm(m->shared_norm, d);
    }
    if (rc) return gcuda_check(cudaGetLastError(), "gmodel init");
    return gcuda_check(cudaStreamSynchronize(st), "gmodel init sync");
}

extern "C" int apus_gcuda_model_reset(ApusGcudaModel *m) {
    const Dims &D = m->D;
    m->ctl_epoch++;
    cudaStreamSynchronize(m->st);
    for (int l = 0; l < D.L; l++) {
        if (!m->L[l].is_dsa) {
            cudaMemsetAsync(m->kda[l].conv, 0, (size_t)NSLOT * 3 * D.qkv * (D.K - 1) * 2, m->st);
            cudaMemsetAsync(m->kda[l].rec, 0, (size_t)NSLOT * D.H * D.D * D.D * 4, m->st);
        }
    }
    if (m->hcarry) cudaMemsetAsync(m->hcarry, 0, (size_t)D.d * 2, m->st);
    if (m->hmtp) cudaMemsetAsync(m->hmtp, 0, (size_t)D.d * 2, m->st);
    Ctl old{};
    cudaMemcpy(&old, m->ctl, sizeof old, cudaMemcpyDeviceToHost);
    Ctl c{};
    c.one = 1;
    for (int i = 1; i < MAXR; i++) c.chain_pos[i] = i - 1;
    c.temp = m->temp; c.top_p = m->top_p;
    c.rng_s = old.rng_s;                 // the caller's stream continues (an ApusRng outlives a sequence)
    c.force_on = m->force.force_on; c.force_base = m->force.force_base; c.force_n = m->force.force_n;
    c.force_seed = m->force.force_seed; c.force_p = m->force.force_p;
    if (gcuda_check(cudaMemcpyAsync(m->ctl, &c, sizeof c, cudaMemcpyHostToDevice, m->st), "reset")) return -1;
    return gcuda_check(cudaStreamSynchronize(m->st), "reset sync");
}

static Ctl read_ctl(ApusGcudaModel *m) {
    Ctl c{};
    cudaStreamSynchronize(m->st);
    cudaMemcpy(&c, m->ctl, sizeof c, cudaMemcpyDeviceToHost);
    return c;
}

extern "C" size_t apus_gcuda_model_pos(const ApusGcudaModel *m) {
    return (size_t)read_ctl((ApusGcudaModel *)m).pos;
}

// ---- forward passes -----------------------------------------------------------

// lm_head over `yn` rows with the fused greedy pick into picks[R] (and the
// BF16 logits when want_logits).
// The argmax keys S.amax were zeroed by the norm that produced yn.
static int lm_head(ApusGcudaModel *m, const uint16_t *yn, int R, int *picks, bool want_logits, int n0 = -1,
                   int *picks2 = nullptr) {
    if (n0 < 0 || n0 > R) n0 = R;
    const Dims &D = m->D;
    GemvDesc g{};
    g.W = m->head; g.x = yn; g.ldx = D.d; g.R = R; g.O = m->vn; g.K = D.d; g.fp8 = 0;
    g.row_base = m->v0; g.plan_o = D.V;     // a vocabulary slice sums like the whole head
    if (want_logits) {
        // expert parallelism: this rank's columns go into its region's logits
        // area, gathered into S.logits on every rank after the picks exchange
        g.y = m->ep_world > 1 ? (uint16_t *)(m->ep_region + m->ep.off_logits) + m->v0 : m->S.logits;
        g.ldy = D.V;
    }
    g.amax = m->S.amax; g.part = m->part; g.ticket = m->tick;
    g.pdl = 1;
    if (gemv_launch(g, m->st)) return -1;
    if (m->ep_world > 1) {
        // the largest key over every rank's slice: publish, barrier, reduce
        if (ep_picks_exchange_launch(m->ep, m->S.amax, R, picks, m->st, n0, picks2)) return -1;
        return want_logits ? ep_logits_gather_launch(m->ep, R, m->S.logits, D.V, m->st) : 0;
    }
    k_extract_picks<<<1, 32, 0, m->st>>>(m->S.amax, R, picks, n0, picks2);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Main model over R rows at positions ctl->pos.., not committed.  yn_out
// (device, [R][d]) receives the post-norm rows.
static int main_forward(ApusGcudaModel *m, const int32_t *ids_dev, int R, uint16_t *yn_out, bool want_logits,
                        bool head = true) {
    const Dims &D = m->D;
    Scratch &S = m->S;
    cudaStream_t st = m->st;
    m->n_main_fwd++;
    m->ctl_epoch++;
    if (k_embed_launch(m->embed, ids_dev, R, D.d, D.hc, S.h4, st)) return -1;
    uint16_t *h = S.h4, *h2 = S.h4b;
    auto stop = [&](int l, int stage) { return l == m->dbg_layer && stage == m->dbg_stage; };
    // each expand also leaves the next site's pre-mix partials in S.mix
    if (hc_postmix_launch(D, nullptr, nullptr, h, R, S, nullptr, m->L[0].hc_fn[0], st)) return -1;
    const bool ep = m->ep_world > 1;
    for (int l = 0; l < D.L; l++) {
        LayerW &W = m->L[l];
        if (hc_pre_launch(D, W, 0, h, R, S, st)) return -1;
        if (stop(l, 0)) return 0;
        if (!W.is_dsa) {
            if (kda_launch(D, W, m->kda[l], m->ctl, R, S, m->part, m->tick, st)) return -1;
        } else {
            if (dsa_launch(D, W.dsa, m->dsa[l], &m->ctl->pos, R, S, S.x, S.sub, m->part, m->tick, st)) return -1;
        }
        if (stop(l, 1)) return 0;
        if (hc_postmix_launch(D, S.sub, nullptr, h, R, S, h2, W.hc_fn[1], st)) return -1;
        std::swap(h, h2);
        if (stop(l, 2)) return 0;
        if (hc_pre_launch(D, W, 1, h, R, S, st)) return -1;
        if (stop(l, 3)) return 0;
        // one GPU: the combine of the expert outputs happens inside the expand
        if (moe_forward_launch(W.moe, S.x, D.d, R, ep ? S.sub : nullptr, D.d, nullptr, st)) return -1;
        if (stop(l, 4)) return ep ? 0 : moe_combine_launch(W.moe, R, S.sub, D.d, st);
        const uint16_t *fn_next = l + 1 < D.L ? m->L[l + 1].hc_fn[0] : nullptr;
        if (hc_postmix_launch(D, ep ? S.sub : nullptr, ep ? nullptr : &W.moe, h, R, S, h2, fn_next, st)) return -1;
        std::swap(h, h2);
    }
    if (h != S.h4) cudaMemcpyAsync(S.h4, h, (size_t)R * D.hc * D.d * 2, cudaMemcpyDeviceToDevice, st);
    if (head_norm_launch(D, S.h4, m->norm, R, yn_out, S.amax, st)) return -1;
    if (!head) return 0;      // the caller runs the lm_head (keys S.amax[0..R) are zeroed)
    return lm_head(m, yn_out, R, m->ctl->picks, want_logits);
}

// MTP block (c/gmtp.h:471-541) over R pairs (ids, prev_h rows) whose DSA
// cache rows start at *base_n; out_h -> S.oh, picks -> ctl->mtp_picks.
static int mtp_forward(ApusGcudaModel *m, const int32_t *ids_dev, const uint16_t *prev_h, int R, const int *base_n,
                       bool want_logits, uint16_t *out_h = nullptr, unsigned long long *keys = nullptr,
                       bool head = true) {
    const Dims &D = m->D;
    Scratch &S = m->S;
    cudaStream_t st = m->st;
    const LayerW &W = m->L[D.L];
    const int d = D.d;
    m->n_mtp_fwd++;
    m->ctl_epoch++;
    // eh = [enorm(embed[id]) | hnorm(prev_h)], the embed rows gathered by id
    {
        NormSeg sg[2] = {{m->embed, d, ids_dev, nullptr, 0, m->enorm, d, S.eh, 2L * d},
                         {prev_h, d, nullptr, nullptr, 0, m->hnorm, d, S.eh + d, 2L * d}};
        if (norm_seg_launch(sg, 2, R, D.eps, nullptr, st)) return -1;
    }
    GemvDesc g{};
    g.W = m->eh_proj; g.x = S.eh; g.ldx = 2L * d; g.R = R; g.O = d; g.K = 2L * d; g.fp8 = 0;
    g.y = S.mx; g.ldy = d; g.part = m->part; g.ticket = m->tick;
    g.pdl = 1;
    if (gemv_launch(g, st)) return -1;
    if (rmsnorm_rows_launch(S.mx, d, W.input_norm, d, R, D.eps, S.mxn, d, st)) return -1;
    if (dsa_launch(D, W.dsa, m->mtp_dsa, base_n, R, S, S.mxn, S.sub, m->part, m->tick, st)) return -1;
    {   // x = bf16(x + attn); post_attention_layernorm
        NormSeg sg = {S.mx, d, nullptr, S.sub, d, W.post_norm, d, S.mxn, d};
        if (norm_seg_launch(&sg, 1, R, D.eps, nullptr, st)) return -1;
    }
    if (moe_forward_launch(W.moe, S.mxn, d, R, S.sub, d, nullptr, st)) return -1;
    if (!out_h) out_h = S.oh;
    {   // x = bf16(x + moe); shared_head.norm; zero the lm_head argmax keys
        NormSeg sg = {S.mx, d, nullptr, S.sub, d, m->shared_norm, d, out_h, d};
        if (norm_seg_launch(&sg, 1, R, D.eps, keys ? keys : S.amax, st)) return -1;
    }
    if (!head) return 0;      // the caller runs the lm_head
    return lm_head(m, out_h, R, m->ctl->mtp_picks, want_logits);
}

// ---- the prompt pass (c/gmodel.h:1658-1666 apus_gmodel_prefill_h) --------


static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

static int ensure_wide(ApusGcudaModel *m) {
    auto &X = m->wide;
    if (X.W) return 0;
    const Dims &D = m->D;
    const int W = PROMPT_ROWS, d = D.d, qkv = D.qkv, ldkp = kda_ldkp(D), hc = D.hc;
    const int mp = m->S.maxpools;
    bool any_dense = false, any_kda = false;
    for (int l = 0; l < D.L; l++) { any_dense |= !m->L[l].sparse; any_kda |= !m->L[l].is_dsa; }
    // one arena for the sublayer that runs (KDA, DSA or the dense MLP)
    const size_t kda_b = any_kda ? al256((size_t)W * ldkp * 2) + al256((size_t)W * 3 * qkv * 2) +
                                       al256((size_t)2 * W * qkv * 2) + al256((size_t)W * qkv * 4) +
                                       al256((size_t)W * D.H * 2) + 2 * al256((size_t)W * qkv * 2)
                                 : 0;
    const size_t dsa_b = al256((size_t)W * (D.ql + D.kl) * 2) + al256((size_t)W * D.ql * 2) +
                         al256((size_t)W * D.kl * 2) + al256((size_t)W * D.AH * D.qd * 2) +
                         al256((size_t)W * D.AH * (D.qd + D.vd) * 2) + al256((size_t)W * D.IH * D.ID * 2) +
                         al256((size_t)W * (2 * D.ID + D.IH) * 2) + al256((size_t)W * D.AH * D.vd * 2) +
                         al256((size_t)W * mp * 4) + al256((size_t)W * mp);
    const size_t mlp_b = any_dense ? al256((size_t)W * 2 * D.dense_inter * 2) + al256((size_t)W * D.dense_inter * 2) : 0;
    size_t arena_b = kda_b > dsa_b ? kda_b : dsa_b;
    arena_b = arena_b > mlp_b ? arena_b : mlp_b;
    size_t wb = (size_t)(D.ql + D.kl) * d;
    wb = std::max(wb, (size_t)D.AH * D.qd * D.ql);
    wb = std::max(wb, (size_t)d * D.AH * D.vd);
    if (any_dense) wb = std::max(wb, (size_t)2 * D.dense_inter * d);
    bool ok = true;
    auto A = [&](size_t n) { void *p = dmalloc(m, n, false); ok = ok && p; return p; };
    X.h4 = (uint16_t *)A((size_t)W * hc * d * 2);
    X.h4b = (uint16_t *)A((size_t)W * hc * d * 2);
    X.x = (uint16_t *)A((size_t)W * d * 2);
    X.sub = (uint16_t *)A((size_t)W * d * 2);
    X.mix = (float *)A((size_t)W * hc_nchunk(D) * ((2 + hc) * hc + 1) * 4);
    X.post = (float *)A((size_t)W * hc * 4);
    X.comb = (float *)A((size_t)W * hc * hc * 4);
    uint8_t *arena = (uint8_t *)A(arena_b);
    X.wbuf = (uint16_t *)A(wb * 2);
    X.ids = (int32_t *)A((size_t)(m->cap + MAXR) * 4);
    const int npos = m->cap + SLACK + W + MAXR;
    X.pos = (int *)A((size_t)npos * 4);
    if (m->has_mtp) {
        X.eh = (uint16_t *)A((size_t)W * 2 * d * 2);
        X.mx = (uint16_t *)A((size_t)W * d * 2);
        X.mxn = (uint16_t *)A((size_t)W * d * 2);
        X.oh = (uint16_t *)A((size_t)W * d * 2);
    }
    if (D.E > 0) {
        MoeRows &w = X.moe;
        const int K = D.ktop, P = W * K / 8 + D.E + W / 8 + 1;
        w.W = W;
        w.pmax = P;
        w.logits = (float *)A((size_t)W * D.E * 4);
        w.row_expert = (int32_t *)A((size_t)W * K * 4);
        w.row_weight = (float *)A((size_t)W * K * 4);
        w.row_sel = (int32_t *)A((size_t)W * K * 4);
        w.pair_slot = (int32_t *)A((size_t)W * K * 4);
        w.shared_slot = (int32_t *)A((size_t)W * 4);
        w.prob_rows = (int32_t *)A((size_t)P * 8 * 4);
        w.prob_expert = (int32_t *)A((size_t)P * 4);
        w.prob_count = (int32_t *)A(4);
        w.xg = (uint16_t *)A((size_t)P * 8 * d * 2);
        w.gu = (uint16_t *)A((size_t)P * 8 * 2 * D.inter * 2);
        w.yd = (uint16_t *)A((size_t)P * 8 * d * 2);
    }
    if (!ok) { gcuda_set_error("gmodel: prompt-pass buffers: device allocation failed"); return -1; }
    {
        uint8_t *p = arena;
        auto C = [&](size_t n) { uint8_t *q = p; p += al256(n); return (void *)q; };
        X.kda.W = W;
        if (any_kda) {
            X.kda.kp = (uint16_t *)C((size_t)W * ldkp * 2);
            X.kda.qkvc = (uint16_t *)C((size_t)W * 3 * qkv * 2);
            X.kda.fgo = (uint16_t *)C((size_t)2 * W * qkv * 2);
            X.kda.g = (float *)C((size_t)W * qkv * 4);
            X.kda.beta = (uint16_t *)C((size_t)W * D.H * 2);
            X.kda.core = (uint16_t *)C((size_t)W * qkv * 2);
            X.kda.onorm = (uint16_t *)C((size_t)W * qkv * 2);
        }
        p = arena;
        X.dsa.qkva = (uint16_t *)C((size_t)W * (D.ql + D.kl) * 2);
        X.dsa.qres = (uint16_t *)C((size_t)W * D.ql * 2);
        X.dsa.kpass = (uint16_t *)C((size_t)W * D.kl * 2);
        X.dsa.q = (uint16_t *)C((size_t)W * D.AH * D.qd * 2);
        X.dsa.kvb = (uint16_t *)C((size_t)W * D.AH * (D.qd + D.vd) * 2);
        X.dsa.iq = (uint16_t *)C((size_t)W * D.IH * D.ID * 2);
        X.dsa.ikgw = (uint16_t *)C((size_t)W * (2 * D.ID + D.IH) * 2);
        X.dsa.attn = (uint16_t *)C((size_t)W * D.AH * D.vd * 2);
        X.dsa.iscore = (float *)C((size_t)W * mp * 4);
        X.dsa.isel = (uint8_t *)C((size_t)W * mp);
        p = arena;
        if (any_dense) {
            X.mlp.gu = (uint16_t *)C((size_t)W * 2 * D.dense_inter * 2);
            X.mlp.h = (uint16_t *)C((size_t)W * D.dense_inter * 2);
        }
    }
    if (iota_launch(X.pos, npos, m->st)) return gcuda_check(cudaGetLastError(), "prompt-pass positions");
    X.W = W;
    return 0;
}

// Scratch view of prompt rows r0.. for the per-row mHC kernels.
static Scratch wide_view(ApusGcudaModel *m, int r0) {
    Scratch v = m->S;
    const auto &X = m->wide;
    const Dims &D = m->D;
    v.x = X.x + (size_t)r0 * D.d;
    v.mix = X.mix + (size_t)r0 * hc_nchunk(D) * ((2 + D.hc) * D.hc + 1);
    v.post = X.post + (size_t)r0 * D.hc;
    v.comb = X.comb + (size_t)r0 * D.hc * D.hc;
    return v;
}

// The main model over prompt rows ids_dev[0..R) at positions p0.. (the layer
// loop of c/gmodel.h:1439-1626 with decode = 0), every sublayer over all R
// rows (the MoE gathers each expert's rows; with expert parallelism each rank
// runs its own experts and the outputs meet in one exchange a layer).  The
// KDA state is read from and left in checkpoint slot `slot`.  yn_out [R][d]
// gets the post-final-norm rows.
static int main_rows(ApusGcudaModel *m, const int32_t *ids_dev, int p0, int R, int slot, uint16_t *yn_out) {
    const Dims &D = m->D;
    auto &X = m->wide;
    cudaStream_t st = m->st;
    m->n_main_fwd++;
    m->ctl_epoch++;
    if (k_embed_launch(m->embed, ids_dev, R, D.d, D.hc, X.h4, st)) return -1;
    uint16_t *h = X.h4, *h2 = X.h4b;
    Scratch v0 = wide_view(m, 0);
    if (hc_postmix_rows_launch(D, nullptr, h, R, v0, nullptr, m->L[0].hc_fn[0], st)) return -1;
    for (int l = 0; l < D.L; l++) {
        LayerW &W = m->L[l];
        if (hc_pre_launch(D, W, 0, h, R, v0, st)) return -1;
        if (!W.is_dsa) {
            KdaState &K = m->kda[l];
            uint16_t *cs = K.conv + (size_t)slot * 3 * D.qkv * (D.K - 1);
            float *rs = K.rec + (size_t)slot * D.H * D.D * D.D;
            if (kda_rows_launch(D, W, cs, rs, R, X.kda, X.x, X.sub, st)) return -1;
        } else if (dsa_rows_launch(D, W.dsa, m->dsa[l], X.pos, p0, R, X.dsa, m->S, X.wbuf, X.x, X.sub, st)) {
            return -1;
        }
        if (hc_postmix_rows_launch(D, X.sub, h, R, v0, h2, W.hc_fn[1], st)) return -1;
        std::swap(h, h2);
        if (hc_pre_launch(D, W, 1, h, R, v0, st)) return -1;
        const uint16_t *fn_next = l + 1 < D.L ? m->L[l + 1].hc_fn[0] : nullptr;
        if (!W.sparse && mlp_rows_launch(W.moe, R, X.mlp, X.wbuf, X.x, X.sub, st)) return -1;
        if (W.sparse && moe_rows_launch(W.moe, X.moe, X.x, D.d, R, X.sub, D.d, st)) return -1;
        if (hc_postmix_rows_launch(D, X.sub, h, R, v0, h2, fn_next, st)) return -1;
        std::swap(h, h2);
    }
    return head_norm_launch(D, h, m->norm, R, yn_out, nullptr, st);
}

// The MTP block (c/gmtp.h:471-541) over R true pairs (ids_dev[t],
// prev_h[t]) at MTP cache positions p0..; out rows -> wide.oh.
static int mtp_rows(ApusGcudaModel *m, const int32_t *ids_dev, const uint16_t *prev_h, int p0, int R) {
    const Dims &D = m->D;
    auto &X = m->wide;
    cudaStream_t st = m->st;
    const LayerW &W = m->L[D.L];
    const int d = D.d;
    m->n_mtp_fwd++;
    m->ctl_epoch++;
    {
        NormSeg sg[2] = {{m->embed, d, ids_dev, nullptr, 0, m->enorm, d, X.eh, 2L * d},
                         {prev_h, d, nullptr, nullptr, 0, m->hnorm, d, X.eh + d, 2L * d}};
        if (norm_seg_launch(sg, 2, R, D.eps, nullptr, st)) return -1;
    }
    if (gemm_tc_launch(X.eh, 2L * d, m->eh_proj, 2L * d, X.mx, d, nullptr, 0, R, d, 2L * d, st)) return -1;
    if (rmsnorm_rows_launch(X.mx, d, W.input_norm, d, R, D.eps, X.mxn, d, st)) return -1;
    if (dsa_rows_launch(D, W.dsa, m->mtp_dsa, X.pos, p0, R, X.dsa, m->S, X.wbuf, X.mxn, X.sub, st)) return -1;
    {   // x = bf16(x + attn); post_attention_layernorm
        NormSeg sg = {X.mx, d, nullptr, X.sub, d, W.post_norm, d, X.mxn, d};
        if (norm_seg_launch(&sg, 1, R, D.eps, nullptr, st)) return -1;
    }
    if (moe_rows_launch(W.moe, X.moe, X.mxn, d, R, X.sub, d, st)) return -1;
    {   // x = bf16(x + moe); shared_head.norm
        NormSeg sg = {X.mx, d, nullptr, X.sub, d, m->shared_norm, d, X.oh, d};
        return norm_seg_launch(&sg, 1, R, D.eps, nullptr, st);
    }
}

// The prompt ids[0..n) from a reset sequence: chunks of PROMPT_ROWS rows
// through the main model, committed chunk by chunk, every position's
// post-norm row kept in yn_prompt; then the lm_head of the last row (pick in
// ctl->picks[0], its logits in S.logits row 0 when want_logits).
static int prompt_pass(ApusGcudaModel *m, const int32_t *ids, size_t n, bool want_logits) {
    if (ensure_wide(m)) return -1;
    auto &X = m->wide;
    const int d = m->D.d;
    if (gcuda_check(cudaMemcpyAsync(X.ids, ids, n * 4, cudaMemcpyHostToDevice, m->st), "prompt upload")) return -1;
    const int slot = read_ctl(m).kda_cur;
    for (size_t c0 = 0; c0 < n; c0 += X.W) {
        const int R = (int)std::min((size_t)X.W, n - c0);
        if (main_rows(m, X.ids + c0, (int)c0, R, slot, m->yn_prompt + c0 * d)) return -1;
        k_commit_rows<<<1, 32, 0, m->st>>>(m->ctl, R);
    }
    if (cudaMemsetAsync(m->S.amax, 0, sizeof(unsigned long long), m->st) != cudaSuccess) return -1;
    return lm_head(m, m->yn_prompt + (n - 1) * d, 1, m->ctl->picks, want_logits);
}

static bool ids_ok(const ApusGcudaModel *m, const int32_t *ids, size_t n, const char *what) {
    for (size_t i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= m->D.V) {
            gcuda_set_error("%s: token id %d outside [0, %d)", what, (int)ids[i], m->D.V);
            return false;
        }
    return true;
}

// held = the draw from logits row `row` of the last forward: the fused
// argmax pick when greedy, else one sampled token (one splitmix64 draw).
static int draw_held(ApusGcudaModel *m, int row) {
    if (!(m->temp > 0.0f)) {
        k_set_held_from_pick<<<1, 32, 0, m->st>>>(m->ctl, row);
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    }
    if (sample_launch(m->S.logits + (size_t)row * m->D.V, m->D.V, m->D.V, 1, m->temp, m->top_p, &m->ctl->rng_s, 0,
                      &m->ctl->held, m->st))
        return -1;
    k_rng_advance<<<1, 32, 0, m->st>>>(m->ctl, 1);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

static int fail_ctl(ApusGcudaModel *m, const char *what) {
    if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(m->st) != cudaSuccess)
        return gcuda_check(cudaGetLastError(), what);
    gcuda_set_error("%s failed", what);
    return -1;
}

extern "C" int apus_gcuda_decode_batch(ApusGcudaModel *m, const int32_t *ids, size_t s, uint16_t *logits,
                                       uint16_t *h_out, uint16_t *yn_out) {
    const Dims &D = m->D;
    if (s < 1 || s > MAXR) { gcuda_set_error("decode_batch: %zu rows (1..%d)", s, MAXR); return -1; }
    if (!ids_ok(m, ids, s, "decode_batch")) return -1;
    Ctl c = read_ctl(m);
    if ((size_t)c.pos + s > (size_t)m->cap) { gcuda_set_error("decode_batch: capacity"); return -1; }
    cudaMemcpyAsync(m->ids, ids, s * 4, cudaMemcpyHostToDevice, m->st);
    if (main_forward(m, m->ids, (int)s, m->S.yn, logits != nullptr)) return fail_ctl(m, "decode_batch");
    // a forward stopped for inspection commits nothing (the sequence stays
    // at its position and committed state)
    if (m->dbg_layer < 0) k_commit<<<1, 32, 0, m->st>>>(m->ctl, (int)s);
    if (logits) cudaMemcpyAsync(logits, m->S.logits, s * D.V * 2, cudaMemcpyDeviceToHost, m->st);
    if (h_out) cudaMemcpyAsync(h_out, m->S.h4, s * D.hc * D.d * 2, cudaMemcpyDeviceToHost, m->st);
    if (yn_out) cudaMemcpyAsync(yn_out, m->S.yn, s * D.d * 2, cudaMemcpyDeviceToHost, m->st);
    return gcuda_check(cudaStreamSynchronize(m->st), "decode_batch");
}

extern "C" int apus_gcuda_prefill(ApusGcudaModel *m, const int32_t *ids, size_t n, uint16_t *logits,
                                  uint16_t *yn_out) {
    const Dims &D = m->D;
    if (n < 1 || n > (size_t)m->cap) { gcuda_set_error("prefill: %zu prompt tokens", n); return -1; }
    if (!ids_ok(m, ids, n, "prefill")) return -1;
    if (apus_gcuda_model_reset(m)) return -1;
    if (prompt_pass(m, ids, n, false)) return fail_ctl(m, "prefill");
    if (logits) {       // every row's logits, 8 rows a launch of the head
        for (size_t t0 = 0; t0 < n; t0 += MAXR) {
            const int k = (int)std::min((size_t)MAXR, n - t0);
            if (cudaMemsetAsync(m->S.amax, 0, k * sizeof(unsigned long long), m->st) != cudaSuccess ||
                lm_head(m, m->yn_prompt + t0 * D.d, k, m->ctl->picks, true))
                return fail_ctl(m, "prefill head");
            if (gcuda_check(cudaMemcpyAsync(logits + t0 * D.V, m->S.logits, (size_t)k * D.V * 2,
                                            cudaMemcpyDeviceToHost, m->st), "prefill logits"))
                return -1;
        }
    }
    if (yn_out && gcuda_check(cudaMemcpyAsync(yn_out, m->yn_prompt, n * D.d * 2, cudaMemcpyDeviceToHost, m->st),
                              "prefill rows"))
        return -1;
    if (gcuda_check(cudaStreamSynchronize(m->st), "prefill")) return -1;
    return tc_error_read_and_clear() ? (gcuda_set_error("prefill: a GEMM wait gave up"), -1) : 0;
}

extern "C" int apus_gcuda_mtp_forward(ApusGcudaModel *m, const int32_t *ids, const uint16_t *prev_h, size_t s,
                                      uint16_t *logits, uint16_t *out_h) {
    const Dims &D = m->D;
    if (!m->has_mtp) { gcuda_set_error("gmtp: model has no MTP block loaded"); return -1; }
    if (s < 1 || s > MAXR) { gcuda_set_error("mtp_forward: %zu rows", s); return -1; }
    if (!ids_ok(m, ids, s, "mtp_forward")) return -1;
    Ctl c = read_ctl(m);
    if ((size_t)c.mtp_n + s > (size_t)m->cap) { gcuda_set_error("mtp_forward: capacity"); return -1; }
    cudaMemcpyAsync(m->ids, ids, s * 4, cudaMemcpyHostToDevice, m->st);
    cudaMemcpyAsync(m->mtp_rows, prev_h, s * D.d * 2, cudaMemcpyHostToDevice, m->st);
    if (mtp_forward(m, m->ids, m->mtp_rows, (int)s, &m->ctl->mtp_n, logits != nullptr))
        return fail_ctl(m, "mtp_forward");
    k_mtp_commit<<<1, 32, 0, m->st>>>(m->ctl, (int)s);
    if (logits) cudaMemcpyAsync(logits, m->S.logits, s * D.V * 2, cudaMemcpyDeviceToHost, m->st);
    if (out_h) cudaMemcpyAsync(out_h, m->S.oh, s * D.d * 2, cudaMemcpyDeviceToHost, m->st);
    return gcuda_check(cudaStreamSynchronize(m->st), "mtp_forward");
}

// ---- speculative decoding --------------------------------------------------

// D-1 chained single-row MTP forwards (c/gmtp.h:677-696): draft i from the
// previous draft and the previous step's post-shared_head.norm hidden.
static int draft_chain(ApusGcudaModel *m) {
    const int D = m->depth, d = m->D.d;
    k_chain_first<<<1, 32, 0, m->st>>>(m->ctl, m->ids);              // ids[0] = drafts[0]
    for (int i = 1; i < D; i++) {
        if (mtp_forward(m, m->ids, m->hmtp, 1, &m->ctl->chain_pos[i], false)) return -1;
        k_copy_row<<<(d + 255) / 256, 256, 0, m->st>>>(m->S.oh, 0, d, m->hmtp);
        k_chain_next<<<1, 32, 0, m->st>>>(m->ctl, i, m->ids);       // drafts[i] = pick
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

extern "C" int apus_gcuda_gspec_prefill(ApusGcudaModel *m, const int32_t *ids, size_t n) {
    const Dims &D = m->D;
    const int d = D.d;
    if (!m->has_mtp) { gcuda_set_error("gspec: model has no MTP block loaded"); return -1; }
    if (n < 1 || n > (size_t)m->cap) { gcuda_set_error("gspec_prefill: %zu prompt tokens", n); return -1; }
    if (!ids_ok(m, ids, n, "gspec_prefill")) return -1;
    if (apus_gcuda_model_reset(m)) return -1;
    // the main model's prompt pass (c/gmtp.h:708-711); the first held token is
    // exactly the non-speculative first draw (c/gmtp.h:724-727)
    if (prompt_pass(m, ids, n, m->temp > 0.0f)) return fail_ctl(m, "gspec_prefill");
    if (draw_held(m, 0)) return fail_ctl(m, "gspec_prefill draw");
    // a one-token prompt has no true pair: drafts stay 0 (c/gmtp.h:741-757)
    if (n < 2) return gcuda_check(cudaStreamSynchronize(m->st), "gspec_prefill");
    // MTP true-pair replay (h_{t-1}, tok_t), t = 1..n-1, chunk by chunk
    auto &X = m->wide;
    int R = 0;
    for (size_t c0 = 0; c0 + 1 < n; c0 += X.W) {
        R = (int)std::min((size_t)X.W, n - 1 - c0);
        if (mtp_rows(m, X.ids + 1 + c0, m->yn_prompt + c0 * d, (int)c0, R)) return fail_ctl(m, "gspec_prefill replay");
        k_mtp_commit<<<1, 32, 0, m->st>>>(m->ctl, R);
    }
    // drafts[0] = argmax of the last replay row; its hidden starts the chain
    const uint16_t *last = X.oh + (size_t)(R - 1) * d;
    k_copy_row<<<(d + 255) / 256, 256, 0, m->st>>>(last, 0, d, m->hmtp);
    if (cudaMemsetAsync(m->S.amax, 0, sizeof(unsigned long long), m->st) != cudaSuccess ||
        lm_head(m, last, 1, m->ctl->mtp_picks, false))
        return fail_ctl(m, "gspec_prefill replay head");
    {
        Ctl tmp = read_ctl(m);
        tmp.drafts[0] = tmp.mtp_picks[0];
        for (int i = 1; i < MAXR; i++) tmp.chain_pos[i] = tmp.mtp_n + i - 1;
        if (gcuda_check(cudaMemcpy(m->ctl, &tmp, sizeof tmp, cudaMemcpyHostToDevice), "gspec_prefill ctl")) return -1;
    }
    // the hnorm input carried to the next step: yn of position n-1
    k_copy_row<<<(d + 255) / 256, 256, 0, m->st>>>(m->yn_prompt, (long)n - 1, d, m->hcarry);
    if (draft_chain(m)) return fail_ctl(m, "gspec_prefill chain");
    k_force<<<1, 32, 0, m->st>>>(m->ctl, m->truth, m->depth, D.V);
    if (gcuda_check(cudaStreamSynchronize(m->st), "gspec_prefill")) return -1;
    return tc_error_read_and_clear() ? (gcuda_set_error("gspec_prefill: a GEMM wait gave up"), -1) : 0;
}

// One verify step of Dp <= depth rows (fewer only at the capacity edge,
// c/gmtp.h:783-786); the draft chain always runs the full depth.
static int spec_step(ApusGcudaModel *m, int Dp) {
    const Dims &D = m->D;
    const int d = D.d;
    cudaStream_t st = m->st;
    const bool smp = m->temp > 0.0f;
    // The verify rows' lm_head waits for the MTP replay so that both row
    // sets share one stream of the 1.27 GB head (the replay needs the verify
    // rows' hidden states, not their picks): rows [0, Dp) of S.yn are the
    // verify rows, rows [Dp, 2 Dp) the replay's shared-head outputs.
    const bool one_head = 2 * Dp <= MAXR;
    uint16_t *mtp_out = one_head ? m->S.yn + (size_t)Dp * d : m->S.oh;
    const bool want = smp || m->keep_logits;
    k_spec_begin<<<1, 32, 0, st>>>(m->ctl, Dp, m->cap, m->ids);
    if (main_forward(m, m->ids, Dp, m->S.yn, want, !one_head)) return -1;
    // MTP replay of the D candidate pairs (rows past the accepted prefix are
    // overwritten by the chain / the next replay)
    k_replay_rows<<<(Dp * d + 255) / 256, 256, 0, st>>>(m->hcarry, m->S.yn, Dp, d, m->mtp_rows);
    if (one_head) {
        if (mtp_forward(m, m->ids, m->mtp_rows, Dp, &m->ctl->mtp_n, false, mtp_out, m->S.amax + Dp, false))
            return -1;
        if (lm_head(m, m->S.yn, 2 * Dp, m->ctl->picks, want, Dp, m->ctl->mtp_picks)) return -1;
    } else if (mtp_forward(m, m->ids, m->mtp_rows, Dp, &m->ctl->mtp_n, false)) {
        return -1;
    }
    // sampled: every verify row's own draw replaces its argmax pick; the walk
    // consumes the draws of the rows it reaches (c/gmtp.h:800-831)
    if (smp && sample_launch(m->S.logits, D.V, D.V, Dp, m->temp, m->top_p, &m->ctl->rng_s, 0, m->ctl->picks, st))
        return -1;
    k_spec_walk<<<1, 32, 0, st>>>(m->ctl, Dp, m->log, m->log_cap);
    k_copy_sel_row<<<(d + 255) / 256, 256, 0, st>>>(mtp_out, m->ctl, d, m->hmtp);
    k_copy_sel_row<<<(d + 255) / 256, 256, 0, st>>>(m->S.yn, m->ctl, d, m->hcarry);
    if (draft_chain(m)) return -1;
    k_force<<<1, 32, 0, st>>>(m->ctl, m->truth, m->depth, D.V);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// The full-depth step is fixed-shape and reads all of its control state
// from device memory, so it is captured once into a CUDA graph and replayed.
static int graph_build(ApusGcudaModel *m) {
    if (cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return gcuda_check(cudaGetLastError(), "graph capture begin");
    const int rc = spec_step(m, m->depth);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (rc || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        gcuda_set_error("gspec: step capture failed");
        return -1;
    }
    if (cudaGraphInstantiate(&m->gexec, g, 0) != cudaSuccess) {
        cudaGraphDestroy(g);
        return gcuda_check(cudaGetLastError(), "graph instantiate");
    }
    m->graph = g;
    size_t n = 0;
    cudaGraphGetNodes(g, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    cudaGraphGetNodes(g, nodes.data(), &n);
    size_t k = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) k++;
    }
    m->graph_kernels = k;
    return 0;
}

extern "C" int apus_gcuda_gspec_step_async(ApusGcudaModel *m) {
    if (!m->has_mtp) { gcuda_set_error("gspec: model has no MTP block loaded"); return -1; }
    m->ctl_epoch++;
    if (!m->use_graph) return spec_step(m, m->depth);
    if (!m->gexec && graph_build(m)) return -1;
    return gcuda_check(cudaGraphLaunch(m->gexec, m->st), "graph launch");
}

extern "C" int apus_gcuda_gspec_use_graph(ApusGcudaModel *m, int on) {
    m->use_graph = on ? 1 : 0;
    return 0;
}

extern "C" void *apus_gcuda_model_stream(ApusGcudaModel *m) { return (void *)m->st; }

extern "C" int apus_gcuda_model_counters(ApusGcudaModel *m, uint64_t *out, size_t n) {
    uint64_t v[5] = {0, m->n_main_fwd, m->n_mtp_fwd, (uint64_t)m->graph_kernels, (uint64_t)sizeof(Ctl)};
    cudaStreamSynchronize(m->st);
    unsigned long long p = 0;
    if (gcuda_check(cudaMemcpy(&p, m->moe_problems, sizeof p, cudaMemcpyDeviceToHost), "counters")) return -1;
    v[0] = p;
    for (size_t i = 0; i < n && i < 5; i++) out[i] = v[i];
    return 0;
}

// One synchronous step: the capacity check uses the control block the
// previous synchronous step read back (when nothing has touched it since),
// a full-depth step replays the captured graph when graphs are on, and the
// one read-back per step returns the emitted tokens.
extern "C" int apus_gcuda_gspec_step(ApusGcudaModel *m, int *out, int cap) {
    if (!m->has_mtp || cap < m->depth + 1) return 0;
    Ctl c = m->cache_epoch == m->ctl_epoch ? m->ctl_cache : read_ctl(m);
    const int De = m->cap - c.pos < m->depth ? m->cap - c.pos : m->depth;
    if (c.err || De <= 0) return 0;
    const int rc = (De == m->depth && m->use_graph) ? apus_gcuda_gspec_step_async(m) : spec_step(m, De);
    m->ctl_epoch++;
    if (rc) { fail_ctl(m, "gspec_step"); return 0; }
    c = read_ctl(m);
    m->ctl_cache = c;
    m->cache_epoch = m->ctl_epoch;
    for (int i = 0; i < c.n_emitted; i++) out[i] = c.emitted[i];
    return c.n_emitted;
}

extern "C" int apus_gcuda_gspec_emitted(ApusGcudaModel *m, int32_t *out, size_t cap) {
    Ctl c = read_ctl(m);
    const size_t n = (size_t)c.log_n < cap ? (size_t)c.log_n : cap;
    if (n && gcuda_check(cudaMemcpy(out, m->log, n * 4, cudaMemcpyDeviceToHost), "emitted")) return -1;
    return c.log_n;
}

extern "C" int apus_gcuda_gspec_stats(ApusGcudaModel *m, uint64_t *o) {
    Ctl c = read_ctl(m);
    o[0] = (uint64_t)c.stat_emitted; o[1] = (uint64_t)c.stat_batches; o[2] = (uint64_t)c.stat_offered;
    o[3] = (uint64_t)c.stat_accepted; o[4] = (uint64_t)c.pos; o[5] = (uint64_t)(int64_t)c.held;
    return c.err ? -1 : 0;
}

// Counters for the reference's ApusGspec fields (apus_gspec_gcuda.h).
extern "C" int apus_gcuda_gspec_counters(ApusGcudaModel *m, uint64_t *o, size_t n) {
    Ctl c = read_ctl(m);
    const uint64_t v[10] = {(uint64_t)c.stat_emitted, (uint64_t)c.stat_batches, (uint64_t)c.stat_offered,
                            (uint64_t)c.stat_accepted, (uint64_t)c.pos, (uint64_t)(int64_t)c.held,
                            (uint64_t)c.stat_d1_hits, (uint64_t)c.stat_d1_offered, (uint64_t)c.stat_refeed,
                            (uint64_t)c.stat_batch_tokens};
    for (size_t i = 0; i < n && i < 10; i++) o[i] = v[i];
    return gcuda_check(cudaGetLastError(), "gspec counters");
}

// The next step's drafts d1..dD (host copy), read or replaced: the
// reference's draft_override hook edits them between steps.
int model_drafts_rw(ApusGcudaModel *m, int32_t *drafts, int n, int write) {
    if (n < 0 || n > MAXR) { gcuda_set_error("drafts: %d entries (0..%d)", n, MAXR); return -1; }
    m->ctl_epoch++;
    Ctl c = read_ctl(m);
    if (!write) {
        memcpy(drafts, c.drafts, (size_t)n * 4);
        return 0;
    }
    for (int i = 0; i < n; i++)
        if (drafts[i] < 0 || drafts[i] >= m->D.V) {
            gcuda_set_error("drafts: token id %d outside [0, %d)", drafts[i], m->D.V);
            return -1;
        }
    return gcuda_check(cudaMemcpy(m->ctl->drafts, drafts, (size_t)n * 4, cudaMemcpyHostToDevice), "drafts write");
}

// Verify rows per step (1..8): the reference's depth, chosen at
// apus_gspec_init; the captured step graph is dropped.
int model_set_depth(ApusGcudaModel *m, int depth) {
    if (depth < 1 || depth > MAXR) { gcuda_set_error("depth %d (1..%d)", depth, MAXR); return -1; }
    if (depth == m->depth) return 0;
    m->depth = depth;
    if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = nullptr; }
    if (m->graph) { cudaGraphDestroy(m->graph); m->graph = nullptr; }
    return 0;
}

size_t model_cap(const ApusGcudaModel *m) { return (size_t)m->cap; }

extern "C" int apus_gcuda_gspec_force(ApusGcudaModel *m, const int32_t *truth, size_t n, size_t base, double p,
                                      uint64_t seed) {
    m->ctl_epoch++;
    Ctl c = read_ctl(m);
    if (!truth) {
        c.force_on = 0;
        m->force.force_on = 0;
    } else {
        if (!m->truth) m->truth = (int32_t *)dmalloc(m, (size_t)m->log_cap * 4 + (size_t)m->cap * 4);
        if (!m->truth || n > (size_t)m->cap + m->log_cap) { gcuda_set_error("gspec_force: truth too long"); return -1; }
        if (!ids_ok(m, truth, n, "gspec_force")) return -1;
        cudaMemcpy(m->truth, truth, n * 4, cudaMemcpyHostToDevice);
        c.force_on = 1; c.force_base = (int)base; c.force_n = (int)n; c.force_p = p; c.force_seed = seed;
        m->force = c;
    }
    return gcuda_check(cudaMemcpy(m->ctl, &c, sizeof c, cudaMemcpyHostToDevice), "gspec_force");
}

// Non-speculative decode: prompt in 8-row batches, then one token per
// forward, each the draw from its own logits row (greedy pick, or a sampled
// token when the model samples: tests/m8g/test_m8g.c:649-678).
static int generate(ApusGcudaModel *m, const int32_t *ids, size_t n, int n_gen, int32_t *out, bool smp,
                    const char *what) {
    if (n < 1 || n_gen < 1 || n + (size_t)n_gen > (size_t)m->cap) { gcuda_set_error("%s: capacity", what); return -1; }
    if (!ids_ok(m, ids, n, what)) return -1;
    if (apus_gcuda_model_reset(m)) return -1;
    const float temp = m->temp;
    if (!smp) m->temp = 0.0f;            // draw_held picks greedily
    int rc = 0;
    // the prompt through the prefill (c/apus.c:1079), then one-token decodes
    rc = prompt_pass(m, ids, n, smp);
    if (!rc) rc = draw_held(m, 0);
    for (int i = 0; i < n_gen && !rc; i++) {
        k_greedy_prep<<<1, 32, 0, m->st>>>(m->ctl, m->ids);
        if (i + 1 < n_gen) {
            rc = main_forward(m, m->ids, 1, m->S.yn, smp);
            if (!rc) k_commit<<<1, 32, 0, m->st>>>(m->ctl, 1);
            if (!rc && smp) {
                rc = sample_launch(m->S.logits, m->D.V, m->D.V, 1, m->temp, m->top_p, &m->ctl->rng_s, 0,
                                   m->ctl->picks, m->st);
                if (!rc) k_rng_advance<<<1, 32, 0, m->st>>>(m->ctl, 1);
            }
        }
        if (!rc) k_greedy_post<<<1, 32, 0, m->st>>>(m->ctl, m->log, m->log_cap);
    }
    m->temp = temp;
    if (rc) return fail_ctl(m, what);
    if (gcuda_check(cudaStreamSynchronize(m->st), what)) return -1;
    return gcuda_check(cudaMemcpy(out, m->log, (size_t)n_gen * 4, cudaMemcpyDeviceToHost), what);
}

extern "C" int apus_gcuda_greedy(ApusGcudaModel *m, const int32_t *ids, size_t n, int n_gen, int32_t *out) {
    return generate(m, ids, n, n_gen, out, false, "greedy");
}

extern "C" int apus_gcuda_generate(ApusGcudaModel *m, const int32_t *ids, size_t n, int n_gen, int32_t *out) {
    return generate(m, ids, n, n_gen, out, m->temp > 0.0f, "generate");
}

// Sampling settings of the speculative and non-speculative decode
// (apus_gspec_init's temp / top_p / rng, c/gmtp.h:617-629, seeded as
// apus_rng_seed, c/sample.h:159).  A captured step graph is dropped: the
// sampled step launches the sampler, the greedy one does not.
extern "C" int apus_gcuda_gspec_sampling(ApusGcudaModel *m, float temp, float top_p, uint64_t seed) {
    if (temp != temp) { gcuda_set_error("sampling: temperature is NaN"); return -1; }
    if (temp > 0.0f && sample_prepare(m->D.V)) return -1;
    m->ctl_epoch++;
    m->temp = temp;
    m->top_p = top_p;
    Ctl c = read_ctl(m);
    c.temp = temp; c.top_p = top_p; c.rng_s = seed;
    if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = nullptr; }
    if (m->graph) { cudaGraphDestroy(m->graph); m->graph = nullptr; }
    return gcuda_check(cudaMemcpy(m->ctl, &c, sizeof c, cudaMemcpyHostToDevice), "sampling");
}

extern "C" int apus_gcuda_rng_state(ApusGcudaModel *m, uint64_t *state) {
    Ctl c = read_ctl(m);
    *state = c.rng_s;
    return gcuda_check(cudaGetLastError(), "rng state");
}

extern "C" int apus_gcuda_gspec_keep_logits(ApusGcudaModel *m, int on) {
    m->keep_logits = on ? 1 : 0;
    if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = nullptr; }
    if (m->graph) { cudaGraphDestroy(m->graph); m->graph = nullptr; }
    return 0;
}

extern "C" int apus_gcuda_model_debug_stop(ApusGcudaModel *m, int layer, int stage) {
    m->dbg_layer = layer;
    m->dbg_stage = stage;
    return 0;
}

// Committed sequence state by name, for inspection: "kda_conv.L" [3*qkv][K-1]
// and "kda_rec.L" [H][D][D] (the committed checkpoint slot of KDA layer L),
// "dsa_k.L" [AH][n][qd], "dsa_v.L" [AH][n][vd], "dsa_ik.L" / "dsa_ig.L"
// [n][ID] (the n committed cache rows of DSA layer L; L = num_hidden_layers
// names the MTP block's caches, n = its committed rows).  -2: not a state name.
static int state_read(ApusGcudaModel *m, const char *name, void *host, size_t bytes) {
    const Dims &D = m->D;
    const char *dot = strchr(name, '.');
    if (!dot) return -2;
    const std::string kind(name, dot - name);
    const int l = atoi(dot + 1);
    if (kind != "kda_conv" && kind != "kda_rec" && kind != "dsa_k" && kind != "dsa_v" && kind != "dsa_ik" &&
        kind != "dsa_ig")
        return -2;
    Ctl c = read_ctl(m);
    auto need = [&](size_t n) {
        if (bytes != n) { gcuda_set_error("debug_read %s: %zu bytes, expected %zu", name, bytes, n); return false; }
        return true;
    };
    uint8_t *h = (uint8_t *)host;
    if (kind == "kda_conv" || kind == "kda_rec") {
        if (l < 0 || l >= D.L || m->L[l].is_dsa) { gcuda_set_error("debug_read %s: not a KDA layer", name); return -1; }
        const size_t cs = (size_t)3 * D.qkv * (D.K - 1) * 2, rs = (size_t)D.H * D.D * D.D * 4;
        if (kind == "kda_conv")
            return need(cs) ? gcuda_check(cudaMemcpy(h, (uint8_t *)m->kda[l].conv + c.kda_cur * cs, cs,
                                                     cudaMemcpyDeviceToHost), "debug_read") : -1;
        return need(rs) ? gcuda_check(cudaMemcpy(h, (uint8_t *)m->kda[l].rec + c.kda_cur * rs, rs,
                                                 cudaMemcpyDeviceToHost), "debug_read") : -1;
    }
    const bool mtp = l == D.L && m->has_mtp;
    if (!mtp && (l < 0 || l >= D.L || !m->L[l].is_dsa)) {
        gcuda_set_error("debug_read %s: not a DSA layer", name);
        return -1;
    }
    const DsaState &ds = mtp ? m->mtp_dsa : m->dsa[l];
    const size_t n = (size_t)(mtp ? c.mtp_n : c.pos);
    if (kind == "dsa_k" || kind == "dsa_v") {
        const size_t w = kind == "dsa_k" ? D.qd : D.vd;
        const uint16_t *src = kind == "dsa_k" ? ds.k : ds.v;
        if (!need((size_t)D.AH * n * w * 2)) return -1;
        for (int hh = 0; hh < D.AH; hh++)
            if (gcuda_check(cudaMemcpy(h + (size_t)hh * n * w * 2, src + (size_t)hh * ds.cap * w, n * w * 2,
                                       cudaMemcpyDeviceToHost), "debug_read"))
                return -1;
        return 0;
    }
    if (!need(n * D.ID * 2)) return -1;
    return gcuda_check(cudaMemcpy(h, kind == "dsa_ik" ? ds.ik : ds.ig, n * D.ID * 2, cudaMemcpyDeviceToHost),
                       "debug_read");
}

extern "C" int apus_gcuda_model_debug_read(ApusGcudaModel *m, const char *name, void *host, size_t bytes) {
    {
        const int rc = state_read(m, name, host, bytes);
        if (rc != -2) return rc;
    }
    if (!strcmp(name, "raw_drafts") || !strcmp(name, "drafts")) {
        Ctl c = read_ctl(m);
        const int *src = name[0] == 'r' ? c.raw_drafts : c.drafts;
        if (bytes > sizeof c.drafts) { gcuda_set_error("debug_read %s: at most %zu bytes", name, sizeof c.drafts); return -1; }
        memcpy(host, src, bytes);
        return 0;
    }
    const Scratch &S = m->S;
    const struct { const char *n; const void *p; } tab[] = {
        {"h4", S.h4}, {"h4b", S.h4b}, {"x", S.x}, {"sub", S.sub}, {"post", S.post}, {"comb", S.comb},
        {"kp", S.kp}, {"qkvc", S.qkvc}, {"fgo", S.fgo}, {"core", S.core}, {"qkva", S.qkva}, {"q", S.q},
        {"kvb", S.kvb}, {"iq", S.iq}, {"ikgw", S.ikgw}, {"attn", S.attn}, {"yn", S.yn}, {"mix", S.mix},
        {"qres", S.qres}, {"kpass", S.kpass}, {"isel", S.isel}, {"iscore", S.iscore},
        {"moe_idx", m->moe_scr.row_expert}, {"moe_w", m->moe_scr.row_weight}, {"moe_sel", m->moe_scr.row_sel},
        {"logits", S.logits}, {"hmtp", m->hmtp}, {"hcarry", m->hcarry}, {"oh", S.oh},
    };
    for (const auto &e : tab)
        if (!strcmp(e.n, name)) {
            cudaStreamSynchronize(m->st);
            return gcuda_check(cudaMemcpy(host, e.p, bytes, cudaMemcpyDeviceToHost), "debug_read");
        }
    gcuda_set_error("debug_read: unknown buffer %s", name);
    return -1;
}

extern "C" uint64_t apus_gcuda_state_digest(ApusGcudaModel *m) {
    const Dims &D = m->D;
    Ctl c = read_ctl(m);
    uint64_t h = 14695981039346656037ull;
    auto eat = [&](const void *dev, size_t bytes) {
        std::vector<uint8_t> b(bytes);
        cudaMemcpy(b.data(), dev, bytes, cudaMemcpyDeviceToHost);
        for (uint8_t x : b) { h ^= x; h *= 1099511628211ull; }
    };
    for (int l = 0; l < D.L; l++) {
        if (!m->L[l].is_dsa) {
            const size_t cs = (size_t)3 * D.qkv * (D.K - 1) * 2, rs = (size_t)D.H * D.D * D.D * 4;
            eat((uint8_t *)m->kda[l].conv + c.kda_cur * cs, cs);
            eat((uint8_t *)m->kda[l].rec + c.kda_cur * rs, rs);
        } else {
            for (int hh = 0; hh < D.AH; hh++) {
                eat(m->dsa[l].k + ((size_t)hh * m->dsa[l].cap) * D.qd, (size_t)c.pos * D.qd * 2);
                eat(m->dsa[l].v + ((size_t)hh * m->dsa[l].cap) * D.vd, (size_t)c.pos * D.vd * 2);
            }
            eat(m->dsa[l].ik, (size_t)c.pos * D.ID * 2);
        }
    }
    return h;
}

