// moe_api.cu — C ABI of include/apus_gmoe_gcuda.h: a resident MoE sublayer.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "gcuda.h"
#include "gmoe_dev.h"
#include "../../include/apus_gcuda.h"
#include "../../include/apus_gmoe_gcuda.h"

struct ApusGcudaMoe {
    MoeDev d;
    std::vector<void *> allocs;
    cudaStream_t st = nullptr;
    uint16_t *xbuf = nullptr, *obuf = nullptr;
    int32_t *fbuf = nullptr;
    size_t nkb_d, nkb_i;
};

static void *dalloc(ApusGcudaMoe *m, size_t n) {
    void *p = nullptr;
    if (cudaMalloc(&p, n ? n : 16) != cudaSuccess) return nullptr;
    m->allocs.push_back(p);
    return p;
}

extern "C" {

ApusGcudaMoe *apus_gcuda_moe_new(int E, int topk, size_t dim, size_t inter, float route_scale,
                                 float swiglu_limit, int max_rows) {
    char err[128];
    if (apus_gcuda_enable(err, sizeof err)) return nullptr;
    if (E < 1 || E > MOE_MAX_E || topk < 1 || topk > MOE_MAX_TOPK || topk > E || max_rows < 1 ||
        max_rows > MOE_MAX_R || inter % 128 || dim % 128) {
        gcuda_set_error("gmoe: unsupported shape E=%d topk=%d dim=%zu inter=%zu rows=%d", E, topk, dim,
                        inter, max_rows);
        return nullptr;
    }
    ApusGcudaMoe *m = new ApusGcudaMoe();
    MoeDev &d = m->d;
    d.E = E; d.topk = topk; d.dim = (int)dim; d.inter = (int)inter; d.max_r = max_rows; d.pdl = 0;
    d.e0 = 0; d.eloc = E;          // every expert local, no exchange (d.ep.world == 0)
    d.route_scale = route_scale; d.limit = swiglu_limit;
    m->nkb_d = (dim + 127) / 128;
    m->nkb_i = (inter + 127) / 128;
    const size_t P = (size_t)max_rows * topk + 1;
    bool ok = true;
    auto A = [&](size_t n) { void *p = dalloc(m, n); ok = ok && p; return p; };
    d.gate_w = (uint16_t *)A((size_t)E * dim * 2);
    d.gate_bias = (float *)A((size_t)E * 4);
    d.gu_codes = (uint8_t *)A((size_t)(E + 1) * 2 * inter * dim);
    d.gu_scales = (float *)A((size_t)(E + 1) * (2 * inter / 128) * m->nkb_d * 4);
    d.d_codes = (uint8_t *)A((size_t)(E + 1) * dim * inter);
    d.d_scales = (float *)A((size_t)(E + 1) * m->nkb_d * m->nkb_i * 4);
    d.logits = (float *)A((size_t)max_rows * E * 4);
    {   // router split-K scratch (tickets start at zero; every launch leaves them zeroed)
        size_t pf, nt;
        gemv_scratch_need(E, (long)dim, &pf, &nt);
        d.part = (float *)A((pf ? pf : 1) * 4);
        d.tick = (int *)A((nt ? nt : 1) * 4);
        if (d.tick) cudaMemset(d.tick, 0, (nt ? nt : 1) * 4);
    }
    d.row_expert = (int32_t *)A((size_t)max_rows * topk * 4);
    d.row_weight = (float *)A((size_t)max_rows * topk * 4);
    d.row_sel = (int32_t *)A((size_t)max_rows * topk * 4);
    d.row_prob = (int32_t *)A((size_t)max_rows * topk * 4);
    d.row_prob_shared = (int32_t *)A((size_t)max_rows * 4);
    d.prob_expert = (int32_t *)A(P * 4);
    d.prob_count = (int32_t *)A(4);
    d.gu = (uint16_t *)A(P * max_rows * 2 * inter * 2);
    d.yd = (uint16_t *)A(P * max_rows * dim * 2);
    m->xbuf = (uint16_t *)A((size_t)max_rows * dim * 2);
    m->obuf = (uint16_t *)A((size_t)max_rows * dim * 2);
    m->fbuf = (int32_t *)A((size_t)max_rows * topk * 4);
    if (ok) ok = cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) == cudaSuccess;
    if (ok) ok = cudaMemset((void *)d.gate_bias, 0, (size_t)E * 4) == cudaSuccess;
    if (!ok) {
        gcuda_set_error("gmoe: device allocation failed");
        apus_gcuda_moe_free(m);
        return nullptr;
    }
    return m;
}

void apus_gcuda_moe_free(ApusGcudaMoe *m) {
    if (!m) return;
    if (m->st) { cudaStreamSynchronize(m->st); cudaStreamDestroy(m->st); }
    for (void *p : m->allocs) cudaFree(p);
    delete m;
}

static int moe_resolve(ApusGcudaMoe *m, const char *name, void **dst_out, size_t *want_out) {
    const MoeDev &d = m->d;
    std::string n(name);
    if (n.rfind("layers.", 0) == 0) {
        size_t dot = n.find('.', 7);
        if (dot == std::string::npos) return -1;
        n = n.substr(dot + 1);
    }
    const size_t dim = d.dim, inter = d.inter, E = d.E;
    void *dst = nullptr;
    size_t want = 0;
    int e = -1;
    char part[64] = {0}, kind[64] = {0};
    if (n == "mlp.gate.weight") { dst = (void *)d.gate_w; want = E * dim * 2; }
    else if (n == "mlp.gate.e_score_correction_bias") { dst = (void *)d.gate_bias; want = E * 4; }
    else {
        if (sscanf(n.c_str(), "mlp.experts.%d.%63[a-z]_proj.%63s", &e, part, kind) == 3) {
            if (e < 0 || e >= (int)E) return -1;
        } else if (sscanf(n.c_str(), "mlp.shared_experts.%63[a-z]_proj.%63s", part, kind) == 2) {
            e = (int)E;
        } else {
            return -1;
        }
        const bool scale = !strcmp(kind, "weight_scale_inv");
        if (!scale && strcmp(kind, "weight")) return -1;
        const size_t gus = (2 * inter / 128) * m->nkb_d, ds = m->nkb_d * m->nkb_i;
        if (!strcmp(part, "gate") || !strcmp(part, "up")) {
            const int up = !strcmp(part, "up");
            if (scale) {
                dst = (void *)(d.gu_scales + (size_t)e * gus + up * (inter / 128) * m->nkb_d);
                want = (inter / 128) * m->nkb_d * 4;
            } else {
                dst = (void *)(d.gu_codes + (size_t)e * 2 * inter * dim + up * inter * dim);
                want = inter * dim;
            }
        } else if (!strcmp(part, "down")) {
            if (scale) { dst = (void *)(d.d_scales + (size_t)e * ds); want = ds * 4; }
            else { dst = (void *)(d.d_codes + (size_t)e * dim * inter); want = dim * inter; }
        } else {
            return -1;
        }
    }
    *dst_out = dst;
    *want_out = want;
    return 0;
}

int apus_gcuda_moe_set(ApusGcudaMoe *m, const char *name, const void *host, size_t bytes) {
    void *dst;
    size_t want;
    if (moe_resolve(m, name, &dst, &want)) { gcuda_set_error("gmoe: unknown tensor %s", name); return -1; }
    if (bytes != want) {
        gcuda_set_error("gmoe: %s has %zu bytes, expected %zu", name, bytes, want);
        return -1;
    }
    return gcuda_check(cudaMemcpy(dst, host, bytes, cudaMemcpyHostToDevice), "gmoe set");
}

int apus_gcuda_moe_get(ApusGcudaMoe *m, const char *name, void *host, size_t bytes) {
    void *src;
    size_t want;
    if (moe_resolve(m, name, &src, &want) || bytes != want) { gcuda_set_error("gmoe: bad get %s", name); return -1; }
    cudaDeviceSynchronize();
    return gcuda_check(cudaMemcpy(host, src, bytes, cudaMemcpyDeviceToHost), "gmoe get");
}

int apus_gcuda_moe_init_random(ApusGcudaMoe *m, uint64_t seed) {
    const MoeDev &d = m->d;
    const size_t E = d.E, dim = d.dim, inter = d.inter;
    int rc = 0;
    rc |= fill_launch(FILL_BF16_NORMAL, (void *)d.gate_w, E * dim, seed, 1, 0.02f, 0.f, m->st);
    rc |= fill_launch(FILL_F32_CONST, (void *)d.gate_bias, E, seed, 2, 0.f, 0.f, m->st);
    rc |= fill_launch(FILL_E4M3_NORMAL, (void *)d.gu_codes, (E + 1) * 2 * inter * dim, seed, 3, 64.f, 0.f, m->st);
    rc |= fill_launch(FILL_E4M3_NORMAL, (void *)d.d_codes, (E + 1) * dim * inter, seed, 4, 64.f, 0.f, m->st);
    rc |= fill_launch(FILL_F32_LOGUNIFORM, (void *)d.gu_scales, (E + 1) * (2 * inter / 128) * m->nkb_d, seed, 5,
                      1e-4f, 1e-2f, m->st);
    rc |= fill_launch(FILL_F32_LOGUNIFORM, (void *)d.d_scales, (E + 1) * m->nkb_d * m->nkb_i, seed, 6, 1e-4f,
                      1e-2f, m->st);
    if (rc) return gcuda_check(cudaGetLastError(), "gmoe init");
    return gcuda_check(cudaStreamSynchronize(m->st), "gmoe init sync");
}

int apus_gcuda_moe_forward_dev(ApusGcudaMoe *m, const uint16_t *x, size_t s, uint16_t *out,
                               const int32_t *forced_idx, void *stream) {
    if (s < 1 || (int)s > m->d.max_r) {
        gcuda_set_error("gmoe: %zu rows (max %d)", s, m->d.max_r);
        return -1;
    }
    if (moe_forward_launch(m->d, x, m->d.dim, (int)s, out, m->d.dim, forced_idx, (cudaStream_t)stream))
        return gcuda_check(cudaGetLastError(), "gmoe forward") ? -1 : -1;
    return 0;
}

int apus_gcuda_moe_forward2(ApusGcudaMoe *m, const uint16_t *x, size_t s, uint16_t *out,
                            const int32_t *forced_idx) {
    const MoeDev &d = m->d;
    if (s < 1 || (int)s > d.max_r) {
        gcuda_set_error("gmoe: %zu rows (max %d)", s, d.max_r);
        return -1;
    }
    if (gcuda_check(cudaMemcpyAsync(m->xbuf, x, s * d.dim * 2, cudaMemcpyHostToDevice, m->st), "x upload"))
        return -1;
    const int32_t *f = nullptr;
    if (forced_idx) {
        if (gcuda_check(cudaMemcpyAsync(m->fbuf, forced_idx, s * d.topk * 4, cudaMemcpyHostToDevice, m->st),
                        "forced upload"))
            return -1;
        f = m->fbuf;
    }
    if (apus_gcuda_moe_forward_dev(m, m->xbuf, s, m->obuf, f, m->st)) return -1;
    if (gcuda_check(cudaMemcpyAsync(out, m->obuf, s * d.dim * 2, cudaMemcpyDeviceToHost, m->st), "out download"))
        return -1;
    return gcuda_check(cudaStreamSynchronize(m->st), "gmoe sync");
}

int apus_gcuda_moe_last_routing(ApusGcudaMoe *m, size_t s, int32_t *idx, float *w) {
    const MoeDev &d = m->d;
    std::vector<int32_t> sel(s * d.topk), ex(s * d.topk);
    std::vector<float> wt(s * d.topk);
    cudaDeviceSynchronize();
    if (gcuda_check(cudaMemcpy(sel.data(), d.row_sel, s * d.topk * 4, cudaMemcpyDeviceToHost), "routing") ||
        gcuda_check(cudaMemcpy(ex.data(), d.row_expert, s * d.topk * 4, cudaMemcpyDeviceToHost), "routing") ||
        gcuda_check(cudaMemcpy(wt.data(), d.row_weight, s * d.topk * 4, cudaMemcpyDeviceToHost), "routing"))
        return -1;
    for (size_t r = 0; r < s; r++)
        for (int j = 0; j < d.topk; j++) {
            const int32_t e = sel[r * d.topk + j];
            if (idx) idx[r * d.topk + j] = e;
            if (w)
                for (int q = 0; q < d.topk; q++)
                    if (ex[r * d.topk + q] == e) w[r * d.topk + j] = wt[r * d.topk + q];
        }
    return 0;
}

uint64_t apus_gcuda_moe_last_bytes(ApusGcudaMoe *m) {
    const MoeDev &d = m->d;
    int32_t cnt = 0;
    cudaDeviceSynchronize();
    if (cudaMemcpy(&cnt, d.prob_count, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    const uint64_t per = (uint64_t)3 * d.inter * d.dim +
                         4ull * ((2 * d.inter / 128) * m->nkb_d + m->nkb_d * m->nkb_i);
    return (uint64_t)cnt * per + (uint64_t)d.E * d.dim * 2;
}

}  // extern "C"
