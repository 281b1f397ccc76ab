"""Parity of the decode stack at the layer dims the bench runs (BASELINE
config 2): hidden 4096, three KDA layers of 32 heads x 128, one DSA layer
with 64 heads (qk_nope = v = 256, q_lora 1536, kv_lora 512) and the
Lightning indexer at 32 x 128 with index_topk 2048, MoE with top-8 of the
routed experts at inter 1024, mHC 4 streams with Sinkhorn-20, an MTP block.
The routed experts (16 instead of 288) and the vocabulary (16384 instead of
154880) are cut so the CPU oracle finishes in seconds; every per-row shape a
kernel sees is the benched one.

Each sublayer is checked teacher-forced: the engine stops after one stage
(apus_gcuda_model_debug_stop) and the oracle restatement of that stage
(oracle/apus_oracle_model.c, pinned bitwise to the reference engine) runs on
the engine's own inputs and committed state (read back and transplanted into
the oracle's state).  Bound per row (north_star): relative L2 error <= 1e-2
and cosine >= 0.9999.  Router selections are compared exactly.  The one
long-context case decodes 2200 tokens first, so the indexer's top-2048
(512 pools of 4) selection binds: selected pools must equal the oracle's
except where the oracle's own scores tie within the observed score error at
the cut.
"""
import numpy as np
import pytest

import oracle as O
import synth

pytestmark = pytest.mark.gpu

KW = synth.c2_config(small=True)
CAP = 2400
COS_MIN, REL_MAX = 0.9999, 1e-2


def f32(a):
    return O.f32_of(np.ascontiguousarray(a, np.uint16)).astype(np.float64)


def close_rows(got, ref, what, cos_min=COS_MIN, rel_max=REL_MAX, to_f=f32):
    g = to_f(got).reshape(len(ref), -1)
    r = to_f(ref).reshape(len(ref), -1)
    worst = (1.0, 0.0)
    for i in range(len(r)):
        a, b = g[i], r[i]
        nb = np.linalg.norm(b)
        cos = float(a @ b / (np.linalg.norm(a) * nb + 1e-30))
        rel = float(np.linalg.norm(a - b) / (nb + 1e-30))
        assert cos >= cos_min and rel <= rel_max, f"{what} row {i}: cosine {cos:.7f}, relative L2 {rel:.3g}"
        worst = (min(worst[0], cos), max(worst[1], rel))
    return worst


def ident(a):
    return np.asarray(a, np.float64)


@pytest.fixture(scope="module")
def c2(gcuda):
    W = synth.c2_weights(KW, seed=20261202)
    g = gcuda.GModel(gcuda.make_config(**KW), has_mtp=True, kv_cap=CAP, depth=4)
    g.load(W)
    o = O.Model(O.make_config(**KW), W, True, "orc")
    yield W, g, o
    g.close()


def transplant(g, o, pos):
    """An oracle state holding the engine's committed state at `pos`."""
    st = o.state(CAP)
    for l in range(KW["num_hidden_layers"]):
        if KW["layer_is_dsa"][l]:
            k, v, ik, ig = g.dsa_state(l, pos)
            assert O.ORC.orc_state_load_dsa(st, l, O.p(k), O.p(v), O.p(ik), O.p(ig), pos) == 0
        else:
            conv, rec = g.kda_state(l)
            assert O.ORC.orc_state_load_kda(st, l, O.p(conv), O.p(rec)) == 0
    O.ORC.orc_state_set_pos(st, pos)
    return st


def stage(g, l, s, ids, reads):
    g.debug_stop(l, s)
    try:
        g.decode_batch(ids)
        return {n: g.debug_read(n, shp, dt) for n, (shp, dt) in reads.items()}
    finally:
        g.debug_stop(-1, 0)


def test_c2_sublayers_vs_oracle(c2):
    W, g, o = c2
    d, hc, R = KW["hidden_size"], KW["hc_mult"], 4
    qkv = KW["linear_num_heads"] * KW["linear_head_dim"]
    rng = np.random.default_rng(5)
    prefix = rng.integers(0, KW["vocab_size"], 13).astype(np.int32)
    ids = rng.integers(0, KW["vocab_size"], R).astype(np.int32)
    g.reset()
    for a in range(0, len(prefix), 8):
        g.decode(prefix[a:a + 8])
    pos = len(prefix)
    assert g.pos() == pos
    u16, f4 = np.uint16, np.float32
    rows = lambda n: ((R, n), u16)
    report = {}
    for l in range(KW["num_hidden_layers"]):
        # stage 0: mHC pre (attention site) + input RMSNorm
        r0 = stage(g, l, 0, ids, {"h4": rows(hc * d), "x": rows(d), "post": ((R, hc), f4),
                                  "comb": ((R, hc, hc), f4)})
        x0 = np.empty((R, d), u16)
        post0, comb0 = np.empty((R, hc), f4), np.empty((R, hc, hc), f4)
        for t in range(R):
            O.ORC.orc_hc_pre(o.h, l, 0, O.p(r0["h4"][t]), O.p(x0[t]), O.p(post0[t]), O.p(comb0[t]))
            O.ORC.orc_rmsnorm(O.p(x0[t]), O.p(W[f"layers.{l}.input_layernorm.weight"]), O.p(x0[t]), d,
                              KW["rms_norm_eps"])
        report[f"L{l} hc_pre"] = close_rows(r0["x"], x0, f"layer {l} mHC pre x")
        close_rows(r0["post"], post0, f"layer {l} mHC pre post", to_f=ident)
        close_rows(r0["comb"], comb0, f"layer {l} mHC pre comb", to_f=ident)
        # stage 1: the attention sublayer on the engine's x and committed state
        r1 = stage(g, l, 1, ids, {"x": rows(d), "sub": rows(d)})
        assert np.array_equal(r1["x"], r0["x"]), "the stage-0 output moved"
        st = transplant(g, o, pos)
        out = np.empty((R, d), u16)
        if KW["layer_is_dsa"][l]:
            O.ORC.orc_dsa_decode(o.h, l, O.p(r1["x"]), R, st, O.p(out))
            name = "DSA"
        else:
            conv, rec = g.kda_state(l)
            O.ORC.orc_kda_decode(o.h, l, O.p(r1["x"]), R, O.p(conv), O.p(rec), O.p(out))
            name = "KDA"
        O.ORC.orc_state_free(st)
        report[f"L{l} {name}"] = close_rows(r1["sub"], out, f"layer {l} {name}")
        # stage 2: mHC post (expand with the attention output)
        r2 = stage(g, l, 2, ids, {"h4": rows(hc * d), "h4b": rows(hc * d), "sub": rows(d),
                                  "post": ((R, hc), f4), "comb": ((R, hc, hc), f4)})
        y4 = np.empty((R, hc * d), u16)
        for t in range(R):
            O.ORC.orc_hc_post(O.p(r2["sub"][t]), O.p(r2["h4"][t]), O.p(r2["post"][t]), O.p(r2["comb"][t]),
                              O.p(y4[t]), d, hc)
        report[f"L{l} hc_post"] = close_rows(r2["h4b"], y4, f"layer {l} mHC post")
        # stage 3: mHC pre (FFN site) + post-attention RMSNorm
        r3 = stage(g, l, 3, ids, {"h4b": rows(hc * d), "x": rows(d), "post": ((R, hc), f4),
                                  "comb": ((R, hc, hc), f4)})
        x3 = np.empty((R, d), u16)
        post3, comb3 = np.empty((R, hc), f4), np.empty((R, hc, hc), f4)
        for t in range(R):
            O.ORC.orc_hc_pre(o.h, l, 1, O.p(r3["h4b"][t]), O.p(x3[t]), O.p(post3[t]), O.p(comb3[t]))
            O.ORC.orc_rmsnorm(O.p(x3[t]), O.p(W[f"layers.{l}.post_attention_layernorm.weight"]), O.p(x3[t]), d,
                              KW["rms_norm_eps"])
        report[f"L{l} hc_pre_ffn"] = close_rows(r3["x"], x3, f"layer {l} mHC pre (ffn) x")
        close_rows(r3["post"], post3, f"layer {l} mHC pre (ffn) post", to_f=ident)
        close_rows(r3["comb"], comb3, f"layer {l} mHC pre (ffn) comb", to_f=ident)
        # stage 4: the MoE on the engine's x; routing exact
        K = KW["num_experts_per_tok"]
        r4 = stage(g, l, 4, ids, {"x": rows(d), "sub": rows(d), "moe_idx": ((8, 16), np.int32)})
        out = np.empty((R, d), u16)
        idx = np.empty((R, K), np.int32)
        wts = np.empty((R, K), f4)
        O.ORC.orc_moe_forward(o.h, l, O.p(r4["x"]), R, O.p(out), O.p(idx), O.p(wts), None)
        for t in range(R):
            assert sorted(idx[t].tolist()) == r4["moe_idx"][t, :K].tolist(), f"layer {l} routing row {t}"
        report[f"L{l} MoE"] = close_rows(r4["sub"], out, f"layer {l} MoE")
    # the whole forward from the transplanted state: head norm + lm_head too
    st = transplant(g, o, pos)
    lg, hg, yg = g.decode_batch(ids, want_h=True)
    lo, ho, yo = o.decode_batch(st, ids, want_h=True)
    O.ORC.orc_state_free(st)
    report["yn"] = close_rows(yg, yo, "final norm rows")
    report["logits"] = close_rows(lg, lo, "logits")
    print("\nconfig-2 stage parity (min cosine, max relative L2):")
    for k, (c, r) in report.items():
        print(f"  {k:16s} {c:.8f} {r:.3g}")


def test_c2_decode_and_mtp_vs_oracle(c2):
    """Fresh sequences on both sides, no transplant: a 12-token prompt in
    batches of 5, 4 and 3 rows, then the MTP block on the true pairs."""
    W, g, o = c2
    rng = np.random.default_rng(11)
    ids = rng.integers(0, KW["vocab_size"], 12).astype(np.int32)
    g.reset()
    st = o.state(CAP)
    yns = []
    for a, b in ((0, 5), (5, 9), (9, 12)):
        lg, _, yg = g.decode_batch(ids[a:b], want_h=True)
        lo, _, yo = o.decode_batch(st, ids[a:b], want_h=True)
        close_rows(lg, lo, f"logits@{a}")
        yns.append(yo)
    O.ORC.orc_state_free(st)
    yn = np.concatenate(yns)
    mst = O.ORC.orc_mtp_state_new(o.h, CAP)
    V, d = KW["vocab_size"], KW["hidden_size"]
    for a, b in ((0, 4), (4, 11)):
        pid = np.ascontiguousarray(ids[1 + a:1 + b])
        ph = np.ascontiguousarray(yn[a:b])
        lo = np.empty((b - a, V), np.uint16)
        oo = np.empty((b - a, d), np.uint16)
        assert O.ORC.orc_mtp_forward(o.h, mst, O.p(pid), O.p(ph), b - a, O.p(lo), O.p(oo)) == 0
        lg, og = g.mtp_forward(pid, ph)
        close_rows(og, oo, f"mtp out_h@{a}")
        close_rows(lg, lo, f"mtp logits@{a}")
    O.ORC.orc_mtp_state_free(mst)


def test_c2_long_context_indexer_selection(c2):
    """2200 committed tokens (550 full pools > 512 selected): the indexer's
    scores, its top-512 pool selection and the DSA sublayer output against
    the oracle on the same cache."""
    W, g, o = c2
    R, d, kp = 4, KW["hidden_size"], KW["index_kpool"]
    layer = KW["layer_is_dsa"].index(1)
    rng = np.random.default_rng(23)
    ctx = rng.integers(0, KW["vocab_size"], 2200).astype(np.int32)
    ids = rng.integers(0, KW["vocab_size"], R).astype(np.int32)
    g.reset()
    for a in range(0, len(ctx), 8):
        g.decode(ctx[a:a + 8])
    pos = len(ctx)
    maxp = (CAP + 24) // kp + 1
    r = stage(g, layer, 1, ids, {"x": ((R, d), np.uint16), "sub": ((R, d), np.uint16),
                                 "iscore": ((R, maxp), np.float32), "isel": ((R, maxp), np.uint8)})
    st = transplant(g, o, pos)
    width = O.ORC.orc_dsa_width(o.h)
    out = np.empty((R, d), np.uint16)
    topk = np.empty((R, width), np.int32)
    scores = np.full((R, maxp), np.nan, np.float32)
    O.ORC.orc_dsa_decode_sel(o.h, layer, O.p(r["x"]), R, st, O.p(out), O.p(topk), O.p(scores), maxp)
    O.ORC.orc_state_free(st)
    ksel = KW["index_topk"] // kp
    for t in range(R):
        nvalid = (pos + t + 1) // kp
        assert nvalid > ksel
        so, sg = scores[t, :nvalid].astype(np.float64), r["iscore"][t, :nvalid].astype(np.float64)
        err = float(np.abs(sg - so).max())
        assert err <= 1e-3 * float(np.abs(so).max()) + 1e-6, f"row {t}: indexer score error {err}"
        ref_sel = set((topk[t][:ksel * kp][topk[t][:ksel * kp] >= 0] // kp).tolist())
        got_sel = set(np.nonzero(r["isel"][t, :nvalid])[0].tolist())
        assert len(ref_sel) == ksel and len(got_sel) == ksel, (len(ref_sel), len(got_sel))
        cut = np.sort(so)[::-1][ksel - 1]
        for p in ref_sel ^ got_sel:
            assert abs(so[p] - cut) <= 2 * err + 1e-7, f"row {t}: pool {p} differs away from the cut"
        # the tail tokens (the partial pool) are selected too
        tail = [i for i in topk[t][ksel * kp:] if i >= 0]
        assert tail == list(range((pos + t + 1) // kp * kp, pos + t + 1))
    close_rows(r["sub"], out, "DSA output at 2200 tokens")
