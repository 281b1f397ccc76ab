// container.cu — the reference's weight container on the host: the model
// configuration (config.json), the standard shard index
// (model.safetensors.index.json) and its safetensors shards, read straight
// into a resident model.
//
// Restates the loading contract of c/gmodel.h:373-480 (config: the real
// "text_config" + "linear_attn_config" layout or the flat fixture layout,
// explicit layer lists winning over the i % 4 == 3 / first_k_dense rule)
// and c/st.h:25-80 (a directory with model.safetensors.index.json whose
// weight_map names the shard of every tensor; a safetensors shard is an
// 8-byte little-endian header length, a JSON header mapping each name to
// dtype, shape and data_offsets relative to the end of the header, then the
// data).  Tensor names are the container names (checkpoint names minus
// "model.language_model.", lm_head.weight verbatim), the names
// apus_gcuda_model_set takes.  Shards are memory-mapped; each tensor the
// model stores on this rank is copied to the device once, another rank's
// experts are never read.
#include "gcuda.h"
#include "../../include/apus_gcuda.h"
#include "../../include/apus_gmtp_gcuda.h"

#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

// model.cu: the configuration a model was created with; whether a
// checkpoint tensor is stored on this rank (1), belongs to another
// expert-parallel rank (0) or is not a tensor of this model (-1).
int model_config_get(const ApusGcudaModel *m, ApusGcudaConfig *cfg, int *has_mtp);
int model_tensor_here(const ApusGcudaModel *m, const char *name);

namespace {

// ---- a small JSON reader ----------------------------------------------------

struct JVal {
    enum Type { NUL, BOOL, NUM, STR, ARR, OBJ } t = NUL;
    bool b = false;
    double n = 0;
    std::string s;
    std::vector<JVal> a;
    std::vector<std::pair<std::string, JVal>> o;
    const JVal *get(const char *k) const {
        if (t != OBJ) return nullptr;
        for (const auto &kv : o)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char *p, *end;
    std::string err;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
    }
    bool fail(const char *what) {
        if (err.empty()) err = what;
        return false;
    }
    bool str(std::string &out) {
        if (p >= end || *p != '"') return fail("expected a string");
        p++;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c != '\\') { out += c; continue; }
            if (p >= end) return fail("bad escape");
            c = *p++;
            switch (c) {
            case 'n': out += '\n'; break;
            case 't': out += '\t'; break;
            case 'r': out += '\r'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'u': {
                if (end - p < 4) return fail("bad \\u escape");
                unsigned v = 0;
                for (int i = 0; i < 4; i++) {
                    const char h = *p++;
                    v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : (h | 32) >= 'a' && (h | 32) <= 'f' ? (h | 32) - 'a' + 10 : 0);
                }
                if (v < 0x80) out += (char)v;          // names here are ASCII; others kept as UTF-8
                else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 63)); }
                else { out += (char)(0xE0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 63)); out += (char)(0x80 | (v & 63)); }
                break;
            }
            default: out += c;
            }
        }
        if (p >= end) return fail("unterminated string");
        p++;
        return true;
    }
    bool val(JVal &v, int depth) {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end");
        const char c = *p;
        if (c == '{') {
            v.t = JVal::OBJ;
            p++;
            ws();
            if (p < end && *p == '}') { p++; return true; }
            while (true) {
                ws();
                std::string k;
                if (!str(k)) return false;
                ws();
                if (p >= end || *p != ':') return fail("expected ':'");
                p++;
                v.o.emplace_back(std::move(k), JVal());
                if (!val(v.o.back().second, depth + 1)) return false;
                ws();
                if (p < end && *p == ',') { p++; continue; }
                if (p < end && *p == '}') { p++; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.t = JVal::ARR;
            p++;
            ws();
            if (p < end && *p == ']') { p++; return true; }
            while (true) {
                v.a.emplace_back();
                if (!val(v.a.back(), depth + 1)) return false;
                ws();
                if (p < end && *p == ',') { p++; continue; }
                if (p < end && *p == ']') { p++; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') { v.t = JVal::STR; return str(v.s); }
        if (end - p >= 4 && !strncmp(p, "true", 4)) { v.t = JVal::BOOL; v.b = true; p += 4; return true; }
        if (end - p >= 5 && !strncmp(p, "false", 5)) { v.t = JVal::BOOL; v.b = false; p += 5; return true; }
        if (end - p >= 4 && !strncmp(p, "null", 4)) { v.t = JVal::NUL; p += 4; return true; }
        // number (also the non-standard Infinity / NaN some writers emit)
        std::string num;
        while (p < end && (isdigit((unsigned char)*p) || strchr("+-.eEInfityNa", *p))) num += *p++;
        if (num.empty()) return fail("unexpected character");
        char *e = nullptr;
        v.t = JVal::NUM;
        v.n = strtod(num.c_str(), &e);
        if (!e || *e) return fail("bad number");
        return true;
    }
};

bool json_parse(const char *text, size_t len, JVal &out, std::string &err) {
    JParser ps{text, text + len, {}};
    if (!ps.val(out, 0)) { err = ps.err; return false; }
    ps.ws();
    if (ps.p != ps.end) { err = "trailing characters"; return false; }
    return true;
}

bool read_file(const std::string &path, std::string &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[1 << 16];
    size_t k;
    while ((k = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, k);
    fclose(f);
    return true;
}

void put_err(char *err, size_t cap, const std::string &msg) {
    gcuda_set_error("%s", msg.c_str());
    if (err && cap) snprintf(err, cap, "%s", msg.c_str());
}

// ---- the shard set ----------------------------------------------------------

struct StTensor {
    std::string dtype;
    std::vector<long> shape;
    const uint8_t *data = nullptr;
    size_t nbytes = 0;
};

struct Shard {
    int fd = -1;
    void *map = nullptr;
    size_t size = 0;
    std::map<std::string, StTensor> tensors;
    ~Shard() {
        if (map && map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) close(fd);
    }
};

size_t dtype_size(const std::string &dt) {
    if (dt == "BF16" || dt == "F16" || dt == "U16" || dt == "I16") return 2;
    if (dt == "F32" || dt == "I32" || dt == "U32") return 4;
    if (dt == "F8_E4M3" || dt == "F8_E5M2" || dt == "U8" || dt == "I8" || dt == "BOOL") return 1;
    if (dt == "F64" || dt == "I64" || dt == "U64") return 8;
    return 0;
}

struct ShardSet {
    std::string dir;
    std::map<std::string, std::string> where;                 // tensor -> shard file
    std::map<std::string, std::unique_ptr<Shard>> shards;     // opened lazily
    std::string err;

    bool open(const char *d) {
        dir = d;
        std::string text;
        if (!read_file(dir + "/model.safetensors.index.json", text)) {
            err = "container: cannot read " + dir + "/model.safetensors.index.json";
            return false;
        }
        JVal idx;
        std::string je;
        if (!json_parse(text.data(), text.size(), idx, je)) {
            err = "container: model.safetensors.index.json: " + je;
            return false;
        }
        const JVal *wm = idx.get("weight_map");
        if (!wm || wm->t != JVal::OBJ) {
            err = "container: model.safetensors.index.json has no weight_map";
            return false;
        }
        for (const auto &kv : wm->o)
            if (kv.second.t == JVal::STR) where[kv.first] = kv.second.s;
        return true;
    }

    Shard *shard(const std::string &file) {
        auto it = shards.find(file);
        if (it != shards.end()) return it->second.get();
        std::unique_ptr<Shard> s(new Shard());
        const std::string path = dir + "/" + file;
        s->fd = ::open(path.c_str(), O_RDONLY);
        struct stat stt;
        if (s->fd < 0 || fstat(s->fd, &stt) || stt.st_size < 8) {
            err = "container: cannot open shard " + path;
            return nullptr;
        }
        s->size = (size_t)stt.st_size;
        s->map = mmap(nullptr, s->size, PROT_READ, MAP_SHARED, s->fd, 0);
        if (s->map == MAP_FAILED) {
            err = "container: cannot map shard " + path;
            return nullptr;
        }
        const uint8_t *base = (const uint8_t *)s->map;
        uint64_t hlen = 0;
        for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | base[i];
        if (hlen > s->size - 8) {
            err = "container: bad header length in " + path;
            return nullptr;
        }
        JVal hdr;
        std::string je;
        if (!json_parse((const char *)base + 8, (size_t)hlen, hdr, je) || hdr.t != JVal::OBJ) {
            err = "container: bad header in " + path + ": " + je;
            return nullptr;
        }
        const uint8_t *data = base + 8 + hlen;
        const size_t dsize = s->size - 8 - hlen;
        for (const auto &kv : hdr.o) {
            if (kv.first == "__metadata__") continue;
            const JVal *dt = kv.second.get("dtype"), *sh = kv.second.get("shape"),
                       *off = kv.second.get("data_offsets");
            if (!dt || dt->t != JVal::STR || !sh || sh->t != JVal::ARR || !off || off->t != JVal::ARR ||
                off->a.size() != 2) {
                err = "container: bad entry " + kv.first + " in " + path;
                return nullptr;
            }
            StTensor t;
            t.dtype = dt->s;
            size_t numel = 1;
            for (const auto &x : sh->a) {
                t.shape.push_back((long)x.n);
                numel *= (size_t)x.n;
            }
            const size_t b = (size_t)off->a[0].n, e = (size_t)off->a[1].n;
            if (e < b || e > dsize || e - b != numel * dtype_size(t.dtype)) {
                err = "container: tensor " + kv.first + " in " + path + " has inconsistent offsets";
                return nullptr;
            }
            t.data = data + b;
            t.nbytes = e - b;
            s->tensors[kv.first] = t;
        }
        Shard *r = s.get();
        shards[file] = std::move(s);
        return r;
    }

    const StTensor *get(const std::string &name) {
        auto w = where.find(name);
        if (w == where.end()) {
            err = "container: no tensor " + name;
            return nullptr;
        }
        Shard *s = shard(w->second);
        if (!s) return nullptr;
        auto t = s->tensors.find(name);
        if (t == s->tensors.end()) {
            err = "container: " + name + " is not in its shard " + w->second;
            return nullptr;
        }
        return &t->second;
    }
};

// ---- the tensors a model needs -----------------------------------------------

struct Need {
    std::string name, dtype;
    size_t numel;
};

// Every checkpoint tensor of cfg's model (c/gmodel.h:622-1106 names), with
// its dtype and element count; the MTP block as layer num_hidden_layers.
std::vector<Need> needed(const ApusGcudaConfig &c, bool mtp) {
    std::vector<Need> v;
    const size_t d = c.hidden_size, V = c.vocab_size, hc = c.hc_mult, mix = (2 + hc) * hc;
    const size_t H = c.linear_num_heads, D = c.linear_head_dim, K = c.linear_conv_kernel_dim, qkv = H * D;
    const size_t AH = c.num_attention_heads, qd = c.qk_nope_head_dim, vd = c.v_head_dim;
    const size_t ql = c.q_lora_rank, kl = c.kv_lora_rank, IH = c.index_n_heads, ID = c.index_head_dim;
    const size_t E = c.n_routed_experts, inter = c.moe_intermediate_size, dense = c.intermediate_size;
    auto cb = [](size_t n) { return (n + 127) / 128; };
    auto t = [&](const std::string &n, const char *dt, size_t numel) { v.push_back({n, dt, numel}); };
    auto fp8 = [&](const std::string &n, size_t O, size_t Kk) {
        t(n + ".weight", "F8_E4M3", O * Kk);
        t(n + ".weight_scale_inv", "F32", cb(O) * cb(Kk));
    };
    auto dsa = [&](const std::string &p) {
        fp8(p + "self_attn.q_a_proj", ql, d);
        t(p + "self_attn.q_a_layernorm.weight", "BF16", ql);
        fp8(p + "self_attn.q_b_proj", AH * qd, ql);
        fp8(p + "self_attn.kv_a_proj_with_mqa", kl, d);
        t(p + "self_attn.kv_a_layernorm.weight", "BF16", kl);
        t(p + "self_attn.kv_b_proj.weight", "BF16", AH * (qd + vd) * kl);
        fp8(p + "self_attn.o_proj", d, AH * vd);
        t(p + "self_attn.indexer.wq_b.weight", "BF16", IH * ID * ql);
        t(p + "self_attn.indexer.wk.weight", "BF16", ID * d);
        t(p + "self_attn.indexer.k_norm.weight", "BF16", ID);
        t(p + "self_attn.indexer.k_norm.bias", "BF16", ID);
        t(p + "self_attn.indexer.weights_proj.weight", "BF16", IH * d);
        t(p + "self_attn.indexer.index_kpool_compress_ape", "BF16", (size_t)c.index_kpool * ID);
        t(p + "self_attn.indexer.index_kpool_compress_gate", "BF16", ID * d);
    };
    auto moe = [&](const std::string &p) {
        t(p + "mlp.gate.weight", "BF16", E * d);
        t(p + "mlp.gate.e_score_correction_bias", "F32", E);
        for (size_t e = 0; e < E; e++) {
            const std::string q = p + "mlp.experts." + std::to_string(e) + ".";
            fp8(q + "gate_proj", inter, d);
            fp8(q + "up_proj", inter, d);
            fp8(q + "down_proj", d, inter);
        }
        fp8(p + "mlp.shared_experts.gate_proj", inter, d);
        fp8(p + "mlp.shared_experts.up_proj", inter, d);
        fp8(p + "mlp.shared_experts.down_proj", d, inter);
    };
    t("embed_tokens.weight", "BF16", V * d);
    t("norm.weight", "BF16", d);
    t("lm_head.weight", "BF16", V * d);
    const int L = c.num_hidden_layers;
    for (int l = 0; l < L; l++) {
        const std::string p = "layers." + std::to_string(l) + ".";
        t(p + "input_layernorm.weight", "BF16", d);
        t(p + "post_attention_layernorm.weight", "BF16", d);
        for (const char *site : {"attn", "ffn"}) {
            t(p + "hc_" + site + "_fn", "BF16", mix * hc * d);
            t(p + "hc_" + site + "_base", "F32", mix);
            t(p + "hc_" + site + "_scale", "F32", 3);
        }
        if (!c.layer_is_dsa[l]) {
            for (const char *n : {"q", "k", "v"}) {
                t(p + "self_attn." + n + "_proj.weight", "BF16", qkv * d);
                t(p + "self_attn." + n + "_conv1d.weight", "BF16", qkv * K);
            }
            t(p + "self_attn.f_a_proj.weight", "BF16", D * d);
            t(p + "self_attn.f_b_proj.weight", "BF16", qkv * D);
            t(p + "self_attn.g_a_proj.weight", "BF16", D * d);
            t(p + "self_attn.g_b_proj.weight", "BF16", qkv * D);
            t(p + "self_attn.b_proj.weight", "BF16", H * d);
            t(p + "self_attn.A_log", "F32", H);
            t(p + "self_attn.dt_bias", "F32", qkv);
            t(p + "self_attn.o_norm.weight", "BF16", D);
            t(p + "self_attn.o_proj.weight", "BF16", d * qkv);
        } else {
            dsa(p);
        }
        if (c.mlp_is_sparse[l]) {
            moe(p);
        } else {
            fp8(p + "mlp.gate_proj", dense, d);
            fp8(p + "mlp.up_proj", dense, d);
            fp8(p + "mlp.down_proj", d, dense);
        }
    }
    if (mtp) {
        const std::string p = "layers." + std::to_string(L) + ".";
        t(p + "enorm.weight", "BF16", d);
        t(p + "hnorm.weight", "BF16", d);
        t(p + "eh_proj.weight", "BF16", d * 2 * d);
        t(p + "input_layernorm.weight", "BF16", d);
        t(p + "post_attention_layernorm.weight", "BF16", d);
        dsa(p);
        moe(p);
        t(p + "shared_head.norm.weight", "BF16", d);
    }
    return v;
}

bool cfg_num(const JVal *o, const char *k, double &out) {
    const JVal *v = o ? o->get(k) : nullptr;
    if (!v || v->t != JVal::NUM) return false;
    out = v->n;
    return true;
}

bool cfg_bool(const JVal *o, const char *k, int &out) {
    const JVal *v = o ? o->get(k) : nullptr;
    if (!v) return false;
    if (v->t == JVal::BOOL) { out = v->b; return true; }
    if (v->t == JVal::NUM) { out = (int)v->n != 0; return true; }
    return false;
}

// The v2 manifest apus.index.json when the container has one (the reference
// loader requires it, c/gmodel.h:647-660; the expert cache reads its slab
// records, c/gcache.h:865-930): format_version 2 and model_type glm5_next;
// every tensor_map entry naming a tensor of the safetensors index agrees with
// that tensor's shard, absolute file offset, size and dtype; every expert
// slab record is the six members (gate, up, down weight + scale, in the
// manifest's member order) laid end to end at its offset in its shard.
int check_manifest(ShardSet &set, std::string &err) {
    std::string text, je;
    if (!read_file(set.dir + "/apus.index.json", text)) return 0;      // a plain safetensors container
    JVal man;
    if (!json_parse(text.data(), text.size(), man, je) || man.t != JVal::OBJ) {
        err = "container: apus.index.json: " + je;
        return -1;
    }
    const JVal *fv = man.get("format_version"), *mt = man.get("model_type"), *ob = man.get("offset_base");
    if (!fv || fv->t != JVal::NUM || (long)fv->n != 2 || !mt || mt->t != JVal::STR || mt->s != "glm5_next") {
        err = "container: apus.index.json not a glm5_next v2 container";
        return -1;
    }
    if (ob && (ob->t != JVal::STR || ob->s != "file")) {
        err = "container: apus.index.json offsets are not file offsets";
        return -1;
    }
    auto file_off = [&](const std::string &name, const std::string &shard, size_t *off, const StTensor **tp) {
        const StTensor *t = set.get(name);
        if (!t) return false;
        auto w = set.where.find(name);
        if (w == set.where.end() || w->second != shard) return false;
        *off = (size_t)(t->data - (const uint8_t *)set.shards[shard]->map);
        *tp = t;
        return true;
    };
    const JVal *tm = man.get("tensor_map");
    if (tm && tm->t == JVal::OBJ)
        for (const auto &kv : tm->o) {
            if (!set.where.count(kv.first)) continue;
            const JVal *sh = kv.second.get("shard"), *off = kv.second.get("offset"), *nb = kv.second.get("nbytes"),
                       *dt = kv.second.get("dtype");
            size_t o = 0;
            const StTensor *t = nullptr;
            if (!sh || sh->t != JVal::STR || !off || off->t != JVal::NUM || !nb || nb->t != JVal::NUM ||
                !file_off(kv.first, sh->s, &o, &t) || o != (size_t)off->n || t->nbytes != (size_t)nb->n ||
                (dt && dt->t == JVal::STR && dt->s != t->dtype)) {
                err = "container: apus.index.json disagrees with the shards for " + kv.first;
                return -1;
            }
        }
    std::vector<std::string> members = {"gate_proj.weight", "gate_proj.weight_scale_inv", "up_proj.weight",
                                        "up_proj.weight_scale_inv", "down_proj.weight", "down_proj.weight_scale_inv"};
    const JVal *mem = man.get("expert_slab_members");
    if (mem && mem->t == JVal::ARR) {
        members.clear();
        for (const auto &x : mem->a)
            if (x.t == JVal::STR) members.push_back(x.s);
    }
    const JVal *slabs = man.get("expert_slabs");
    if (slabs && slabs->t == JVal::ARR)
        for (const auto &r : slabs->a) {
            const JVal *blk = r.get("block"), *ex = r.get("expert"), *sh = r.get("shard"), *off = r.get("offset"),
                       *nb = r.get("nbytes");
            if (!blk || blk->t != JVal::STR || !ex || ex->t != JVal::NUM || !sh || sh->t != JVal::STR || !off ||
                off->t != JVal::NUM || !nb || nb->t != JVal::NUM) {
                err = "container: apus.index.json has a bad expert slab record";
                return -1;
            }
            const std::string base = blk->s + ".mlp.experts." + std::to_string((long)ex->n) + ".";
            size_t at = (size_t)off->n, total = 0;
            for (const std::string &m : members) {
                size_t o = 0;
                const StTensor *t = nullptr;
                if (!file_off(base + m, sh->s, &o, &t) || o != at) {
                    err = "container: expert slab " + blk->s + "/" + std::to_string((long)ex->n) +
                          " is not its members laid end to end (" + m + ")";
                    return -1;
                }
                at += t->nbytes;
                total += t->nbytes;
            }
            if (total != (size_t)nb->n) {
                err = "container: expert slab " + blk->s + "/" + std::to_string((long)ex->n) + " size " +
                      std::to_string((size_t)nb->n) + " != its members' " + std::to_string(total);
                return -1;
            }
        }
    return 0;
}

int check_all(ShardSet &set, const ApusGcudaConfig &c, bool mtp, std::string &err) {
    if (check_manifest(set, err)) return -1;
    int n = 0;
    for (const Need &nd : needed(c, mtp)) {
        const StTensor *t = set.get(nd.name);
        if (!t) { err = set.err; return -1; }
        if (t->dtype != nd.dtype || t->nbytes != nd.numel * dtype_size(nd.dtype)) {
            err = "container: " + nd.name + " is " + t->dtype + " with " + std::to_string(t->nbytes) +
                  " bytes, expected " + nd.dtype + " with " + std::to_string(nd.numel * dtype_size(nd.dtype));
            return -1;
        }
        n++;
    }
    return n;
}

}  // namespace

extern "C" int apus_gcuda_config_load(const char *path, ApusGcudaConfig *cfg, char *err, size_t errcap) {
    std::string text, je;
    JVal root;
    if (!read_file(path, text)) { put_err(err, errcap, std::string("gcuda cfg: cannot read ") + path); return -1; }
    if (!json_parse(text.data(), text.size(), root, je)) {
        put_err(err, errcap, std::string("gcuda cfg: ") + path + ": " + je);
        return -1;
    }
    memset(cfg, 0, sizeof *cfg);
    const JVal *tc = root.get("text_config");
    if (!tc) tc = &root;                           // flat fixture config
    bool ok = true;
    double d;
    const struct { const char *k; int *o; } ints[] = {
        {"hidden_size", &cfg->hidden_size}, {"vocab_size", &cfg->vocab_size},
        {"num_hidden_layers", &cfg->num_hidden_layers}, {"hc_mult", &cfg->hc_mult},
        {"hc_sinkhorn_iters", &cfg->hc_sinkhorn_iters}, {"first_k_dense_replace", &cfg->first_k_dense_replace},
        {"intermediate_size", &cfg->intermediate_size}, {"moe_intermediate_size", &cfg->moe_intermediate_size},
        {"n_routed_experts", &cfg->n_routed_experts}, {"n_shared_experts", &cfg->n_shared_experts},
        {"num_experts_per_tok", &cfg->num_experts_per_tok}, {"num_attention_heads", &cfg->num_attention_heads},
        {"q_lora_rank", &cfg->q_lora_rank}, {"kv_lora_rank", &cfg->kv_lora_rank},
        {"qk_nope_head_dim", &cfg->qk_nope_head_dim}, {"v_head_dim", &cfg->v_head_dim},
        {"index_n_heads", &cfg->index_n_heads}, {"index_head_dim", &cfg->index_head_dim},
        {"index_topk", &cfg->index_topk}, {"index_kpool", &cfg->index_kpool},
    };
    for (const auto &e : ints) {
        if (cfg_num(tc, e.k, d)) *e.o = (int)d;
        else ok = false;
    }
    const struct { const char *k; float *o; } flts[] = {
        {"rms_norm_eps", &cfg->rms_norm_eps}, {"hc_eps", &cfg->hc_eps},
        {"routed_scaling_factor", &cfg->routed_scaling_factor}, {"swiglu_limit", &cfg->swiglu_limit},
    };
    for (const auto &e : flts) {
        if (cfg_num(tc, e.k, d)) *e.o = (float)d;
        else ok = false;
    }
    ok = cfg_bool(tc, "norm_topk_prob", cfg->norm_topk_prob) && ok;
    ok = cfg_bool(tc, "index_kpool_always_select_tail", cfg->index_kpool_always_select_tail) && ok;
    if (cfg_num(tc, "num_nextn_predict_layers", d)) cfg->num_nextn_predict_layers = (int)d;   // optional
    const JVal *la = tc->get("linear_attn_config");      // the real layout nests the KDA keys
    const char *kn[4] = {"num_heads", "head_dim", "short_conv_kernel_size", "gate_lower_bound"};
    const char *fk[4] = {"linear_num_heads", "linear_head_dim", "linear_conv_kernel_dim", "linear_lower_bound"};
    const JVal *src = la ? la : tc;
    const char **keys = la ? kn : fk;
    if (cfg_num(src, keys[0], d)) cfg->linear_num_heads = (int)d; else ok = false;
    if (cfg_num(src, keys[1], d)) cfg->linear_head_dim = (int)d; else ok = false;
    if (cfg_num(src, keys[2], d)) cfg->linear_conv_kernel_dim = (int)d; else ok = false;
    if (cfg_num(src, keys[3], d)) cfg->linear_lower_bound = (float)d; else ok = false;
    const int L = cfg->num_hidden_layers;
    if (!ok || L <= 0) {
        put_err(err, errcap, std::string("gcuda cfg: missing/invalid keys in ") + path);
        return -1;
    }
    if (L > APUS_GCUDA_MAX_LAYERS) {
        put_err(err, errcap, std::string("gcuda cfg: more than ") + std::to_string(APUS_GCUDA_MAX_LAYERS) +
                                 " layers in " + path);
        return -1;
    }
    for (int i = 0; i < L; i++) {             // the pattern rule (c/gmodel.h:343-349) ...
        cfg->layer_is_dsa[i] = i % 4 == 3;
        cfg->mlp_is_sparse[i] = i >= cfg->first_k_dense_replace;
    }
    const JVal *lt = tc->get("layer_types");  // ... unless explicit lists are given
    if (lt && lt->t == JVal::ARR && lt->a.size() == (size_t)L)
        for (int i = 0; i < L; i++)
            cfg->layer_is_dsa[i] = lt->a[i].t == JVal::STR && lt->a[i].s == "deepseek_sparse_attention";
    const JVal *mt = tc->get("mlp_layer_types");
    if (mt && mt->t == JVal::ARR && mt->a.size() == (size_t)L)
        for (int i = 0; i < L; i++) cfg->mlp_is_sparse[i] = mt->a[i].t == JVal::STR && mt->a[i].s == "sparse";
    return 0;
}

extern "C" int apus_gcuda_container_check(const char *dir, const ApusGcudaConfig *cfg, int has_mtp, char *err,
                                          size_t errcap) {
    ShardSet set;
    if (!set.open(dir)) { put_err(err, errcap, set.err); return -1; }
    std::string e;
    const int n = check_all(set, *cfg, has_mtp != 0, e);
    if (n < 0) put_err(err, errcap, e);
    return n;
}

extern "C" long apus_gcuda_container_read(const char *dir, const char *name, void *host, size_t cap, char *err,
                                          size_t errcap) {
    ShardSet set;
    if (!set.open(dir)) { put_err(err, errcap, set.err); return -1; }
    const StTensor *t = set.get(name);
    if (!t) { put_err(err, errcap, set.err); return -1; }
    if (host) {
        if (cap < t->nbytes) {
            put_err(err, errcap, std::string("container: ") + name + " needs " + std::to_string(t->nbytes) + " bytes");
            return -1;
        }
        memcpy(host, t->data, t->nbytes);
    }
    return (long)t->nbytes;
}

extern "C" int apus_gcuda_model_load_container(ApusGcudaModel *m, const char *dir, char *err, size_t errcap) {
    ApusGcudaConfig cfg;
    int has_mtp = 0;
    if (model_config_get(m, &cfg, &has_mtp)) { put_err(err, errcap, "container: bad model"); return -1; }
    ShardSet set;
    if (!set.open(dir)) { put_err(err, errcap, set.err); return -1; }
    std::string e;
    if (check_all(set, cfg, has_mtp != 0, e) < 0) { put_err(err, errcap, e); return -1; }
    for (const Need &nd : needed(cfg, has_mtp != 0)) {
        const int here = model_tensor_here(m, nd.name.c_str());
        if (here < 0) { put_err(err, errcap, "container: the model does not take " + nd.name); return -1; }
        if (!here) continue;                      // another expert-parallel rank's expert: not read
        const StTensor *t = set.get(nd.name);
        if (!t || apus_gcuda_model_set(m, nd.name.c_str(), t->data, t->nbytes) < 0) {
            put_err(err, errcap, t ? std::string(apus_gcuda_last_error()) : set.err);
            return -1;
        }
    }
    return 0;
}
