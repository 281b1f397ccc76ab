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
and cosine >= 0.9999.  Router selections are compared exactly.

Composites of stages (a whole forward, an MTP forward) compound the stages'
BF16 rounding-point flips and have a looser, measured bound; they run with
the MoE routing of both sides the same (the oracle forced to the engine's
selections), and the oracle's own routing may differ from the engine's only
at a near tie of its top-k scores.

The same checks run at the config-3 (full model) per-layer dims too: four
layers of the reference's config.json shapes -- the first three dense MLPs of
intermediate 12288, KDA at 64 heads, MoE at inter 2048 -- with the routed
experts and the vocabulary cut as above.

The long-context case decodes 2200 tokens first, so the indexer's top-2048
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
KW3 = dict(synth.c3_config(4), n_routed_experts=16, vocab_size=16384)
CAP = 2400
COS_MIN, REL_MAX = 0.9999, 1e-2
E2E_COS, E2E_REL = 0.999, 5e-2
# The routing may only differ where the oracle's own top-k selection is a
# near tie: biased-score gap between the k-th selection and the next expert
# below ROUTE_TIE (the scores are sigmoids; an x error of 1e-2 relative moves
# a logit by about 1e-2 and a score by at most a quarter of that).
ROUTE_TIE = 5e-3


def f32(a):
    return O.f32_of(np.ascontiguousarray(a, np.uint16)).astype(np.float64)


def ident(a):
    return np.asarray(a, np.float64)


def row_stats(got, ref, to_f=None):
    """(min cosine, max relative L2, fraction of bitwise-equal elements) over rows."""
    to_f = to_f or f32
    g = to_f(got).reshape(len(ref), -1)
    r = to_f(ref).reshape(len(ref), -1)
    cmin, rmax = 1.0, 0.0
    for i in range(len(r)):
        a, b = g[i], r[i]
        nb = np.linalg.norm(b)
        cmin = min(cmin, float(a @ b / (np.linalg.norm(a) * nb + 1e-30)))
        rmax = max(rmax, float(np.linalg.norm(a - b) / (nb + 1e-30)))
    same = float(np.mean(np.asarray(got).reshape(-1) == np.asarray(ref).reshape(-1)))
    return cmin, rmax, same


class Report:
    """Collects every stage's figures, prints them all, then fails on the
    stages outside their bound (so one run shows the whole picture)."""

    def __init__(self, title):
        self.title, self.rows, self.bad = title, [], []

    def check(self, what, got, ref, cos_min=COS_MIN, rel_max=REL_MAX, to_f=None):
        c, r, same = row_stats(got, ref, to_f)
        ok = c >= cos_min and r <= rel_max
        self.rows.append((what, c, r, same, ok))
        if not ok:
            self.bad.append(f"{what}: cosine {c:.7f} (>= {cos_min}), relative L2 {r:.3g} (<= {rel_max})")

    def fact(self, what, ok, detail=""):
        self.rows.append((what, float("nan"), float("nan"), float("nan"), ok))
        if not ok:
            self.bad.append(f"{what}: {detail}")

    def finish(self):
        print(f"\n{self.title}: stage, min cosine, max relative L2, bitwise-equal fraction")
        for what, c, r, same, ok in self.rows:
            print(f"  {'ok ' if ok else 'BAD'} {what:34s} {c:.8f} {r:.3e} {same:.4f}")
        assert not self.bad, "; ".join(self.bad)


def make_case(gcuda, kw, seed):
    W = synth.c2_weights(kw, seed=seed)
    g = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=CAP, depth=4)
    g.load(W)
    o = O.Model(O.make_config(**kw), W, True, "orc")
    return W, g, o


@pytest.fixture(scope="module")
def c2(gcuda):
    W, g, o = make_case(gcuda, KW, 20261202)
    yield W, g, o
    g.close()


@pytest.fixture(scope="module", params=["config2", "config3"])
def case(request, gcuda):
    """(kw, W, engine model, oracle model) at the config-2 or the config-3
    per-layer dims."""
    if request.param == "config2":
        yield (KW,) + request.getfixturevalue("c2")
        return
    W, g, o = make_case(gcuda, KW3, 20261205)
    yield KW3, W, g, o
    g.close()


def engine_state(g, pos, kw=KW):
    """The engine's committed state at `pos`, per layer (host copies)."""
    return [g.dsa_state(l, pos) if kw["layer_is_dsa"][l] else g.kda_state(l)
            for l in range(kw["num_hidden_layers"])]


def oracle_state(o, saved, pos, kw=KW):
    """A fresh oracle state holding a saved engine state."""
    st = o.state(CAP)
    for l, a in enumerate(saved):
        if kw["layer_is_dsa"][l]:
            assert O.ORC.orc_state_load_dsa(st, l, *(O.p(x) for x in a), pos) == 0
        else:
            assert O.ORC.orc_state_load_kda(st, l, *(O.p(x) for x in a)) == 0
    O.ORC.orc_state_set_pos(st, pos)
    return st


def transplant(g, o, pos, kw=KW):
    """An oracle state holding the engine's committed state at `pos`."""
    return oracle_state(o, engine_state(g, pos, kw), pos, kw)


def stage(g, l, s, ids, reads):
    g.debug_stop(l, s)
    try:
        g.decode_batch(ids)
        return {n: g.debug_read(n, shp, dt) for n, (shp, dt) in reads.items()}
    finally:
        g.debug_stop(-1, 0)


def gpu_routing(g, ids, kw=KW):
    """The engine's MoE selections of a forward over ids, top-k order,
    [L][R][K] (stage-4 stops; nothing is committed)."""
    R, K, L = len(ids), kw["num_experts_per_tok"], kw["num_hidden_layers"]
    sel = np.zeros((L, R, K), np.int32)
    for l in range(L):
        if kw["mlp_is_sparse"][l]:
            sel[l] = stage(g, l, 4, ids, {"moe_sel": ((8 * 16,), np.int32)})["moe_sel"][:R * K].reshape(R, K)
    return sel


def oracle_forward(o, st, ids, forced, kw=KW):
    R, L, K = len(ids), kw["num_hidden_layers"], kw["num_experts_per_tok"]
    V, d, hc = kw["vocab_size"], kw["hidden_size"], kw["hc_mult"]
    ids = np.ascontiguousarray(ids, np.int32)
    lo, ho, yo = np.empty((R, V), np.uint16), np.empty((R, hc * d), np.uint16), np.empty((R, d), np.uint16)
    osel, gap = np.zeros((L, R, K), np.int32), np.zeros((L, R), np.float32)
    fp = O.p(np.ascontiguousarray(forced)) if forced is not None else None
    assert O.ORC.orc_decode_batch_ex(o.h, st, O.p(ids), R, O.p(lo), O.p(ho), O.p(yo), fp, O.p(osel),
                                     O.p(gap)) == 0
    return lo, yo, osel, gap


def whole_forward(rep, o, new_state, ids, sel, yg, lg, tag="", kw=KW):
    """Oracle forwards from fresh copies of the same state: forced to the
    engine's routing (within the composite bound), and free (its routing may
    differ only at a near tie; without a difference, within bound)."""
    R, L = len(ids), kw["num_hidden_layers"]
    st = new_state()
    lo, yo, _, _ = oracle_forward(o, st, ids, sel, kw)
    O.ORC.orc_state_free(st)
    rep.check(f"{tag}final norm rows (engine routing)", yg, yo, cos_min=E2E_COS, rel_max=E2E_REL)
    rep.check(f"{tag}logits (engine routing)", lg, lo, cos_min=E2E_COS, rel_max=E2E_REL)
    st = new_state()
    lo, yo, osel, gap = oracle_forward(o, st, ids, None, kw)
    O.ORC.orc_state_free(st)
    diff = [(l, t) for l in range(L) if kw["mlp_is_sparse"][l] for t in range(R)
            if sorted(osel[l, t].tolist()) != sorted(sel[l, t].tolist())]
    if diff:
        l0 = diff[0][0]
        for l, t in diff:
            if l == l0:
                rep.fact(f"{tag}own routing L{l} row {t}", gap[l, t] < ROUTE_TIE,
                         f"differs at a top-k gap of {gap[l, t]:.3g}")
        print(f"{tag}oracle's own routing first differs at layer {l0} (rows "
              f"{[t for l, t in diff if l == l0]}, gaps {[float(gap[l, t]) for l, t in diff if l == l0]})")
    else:
        rep.check(f"{tag}logits (own routing)", lg, lo, cos_min=E2E_COS, rel_max=E2E_REL)


def test_sublayers_vs_oracle(case):
    KW, W, g, o = case
    d, hc, R = KW["hidden_size"], KW["hc_mult"], 4
    K = KW["num_experts_per_tok"]
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
    rep = Report(f"stage parity at {KW['num_hidden_layers']} layers of {KW['linear_num_heads']}-head KDA, "
                 f"MoE inter {KW['moe_intermediate_size']}")
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
        rep.check(f"L{l} mHC pre x", r0["x"], x0)
        rep.check(f"L{l} mHC pre post", r0["post"], post0, to_f=ident)
        rep.check(f"L{l} mHC pre comb", r0["comb"], comb0, to_f=ident)
        # stage 1: the attention sublayer on the engine's x and committed state
        r1 = stage(g, l, 1, ids, {"x": rows(d), "sub": rows(d)})
        rep.fact(f"L{l} stage-1 input = stage-0 output", np.array_equal(r1["x"], r0["x"]), "moved")
        out = np.empty((R, d), u16)
        if KW["layer_is_dsa"][l]:
            st = transplant(g, o, pos, KW)
            O.ORC.orc_dsa_decode(o.h, l, O.p(r1["x"]), R, st, O.p(out))
            O.ORC.orc_state_free(st)
            name = "DSA"
        else:
            conv, rec = g.kda_state(l)
            O.ORC.orc_kda_decode(o.h, l, O.p(r1["x"]), R, O.p(conv), O.p(rec), O.p(out))
            name = "KDA"
        rep.check(f"L{l} {name}", r1["sub"], out)
        # stage 2: mHC post (expand with the attention output)
        r2 = stage(g, l, 2, ids, {"h4": rows(hc * d), "h4b": rows(hc * d), "sub": rows(d),
                                  "post": ((R, hc), f4), "comb": ((R, hc, hc), f4)})
        y4 = np.empty((R, hc * d), u16)
        for t in range(R):
            O.ORC.orc_hc_post(O.p(r2["sub"][t]), O.p(r2["h4"][t]), O.p(r2["post"][t]), O.p(r2["comb"][t]),
                              O.p(y4[t]), d, hc)
        rep.check(f"L{l} mHC post", r2["h4b"], y4)
        # stage 3: mHC pre (FFN site) + post-attention RMSNorm
        r3 = stage(g, l, 3, ids, {"h4b": rows(hc * d), "x": rows(d), "post": ((R, hc), f4),
                                  "comb": ((R, hc, hc), f4)})
        x3 = np.empty((R, d), u16)
        post3, comb3 = np.empty((R, hc), f4), np.empty((R, hc, hc), f4)
        for t in range(R):
            O.ORC.orc_hc_pre(o.h, l, 1, O.p(r3["h4b"][t]), O.p(x3[t]), O.p(post3[t]), O.p(comb3[t]))
            O.ORC.orc_rmsnorm(O.p(x3[t]), O.p(W[f"layers.{l}.post_attention_layernorm.weight"]), O.p(x3[t]), d,
                              KW["rms_norm_eps"])
        rep.check(f"L{l} mHC pre (ffn) x", r3["x"], x3)
        rep.check(f"L{l} mHC pre (ffn) post", r3["post"], post3, to_f=ident)
        rep.check(f"L{l} mHC pre (ffn) comb", r3["comb"], comb3, to_f=ident)
        # stage 4: the MoE (routing exact) or the dense MLP on the engine's x
        r4 = stage(g, l, 4, ids, {"x": rows(d), "sub": rows(d), "moe_idx": ((8 * 16,), np.int32)})
        out = np.empty((R, d), u16)
        if not KW["mlp_is_sparse"][l]:
            O.ORC.orc_mlp_forward(o.h, l, O.p(r4["x"]), R, O.p(out))
            rep.check(f"L{l} dense MLP (inter {KW['intermediate_size']})", r4["sub"], out)
            continue
        idx = np.empty((R, K), np.int32)
        wts = np.empty((R, K), f4)
        O.ORC.orc_moe_forward(o.h, l, O.p(r4["x"]), R, O.p(out), O.p(idx), O.p(wts), None)
        gidx = r4["moe_idx"][:R * K].reshape(R, K)
        for t in range(R):
            rep.fact(f"L{l} routing row {t}", sorted(idx[t].tolist()) == gidx[t].tolist(),
                     f"{gidx[t].tolist()} vs {sorted(idx[t].tolist())}")
        rep.check(f"L{l} MoE", r4["sub"], out)
    # the whole forward from the transplanted state (the MoE expand and the
    # head norm + lm_head included), with the engine's routing and the
    # oracle's own
    sel = gpu_routing(g, ids, KW)
    saved = engine_state(g, pos, KW)
    lg, _, yg = g.decode_batch(ids, want_h=True)
    whole_forward(rep, o, lambda: oracle_state(o, saved, pos, KW), ids, sel, yg, lg, kw=KW)
    rep.finish()


def test_decode_and_mtp_vs_oracle(case):
    """Fresh sequences on both sides, no transplant: a 12-token prompt in
    batches of 5, 4 and 3 rows (the oracle following the engine's routing),
    then the MTP block on the engine's true pairs and three chained MTP
    steps."""
    KW, W, g, o = case
    rng = np.random.default_rng(11)
    ids = rng.integers(0, KW["vocab_size"], 12).astype(np.int32)
    g.reset()
    st = o.state(CAP)
    yns = []
    rep = Report(f"fresh decode + MTP ({KW['linear_num_heads']}-head KDA)")
    for a, b in ((0, 5), (5, 9), (9, 12)):
        chunk = np.ascontiguousarray(ids[a:b])
        sel = gpu_routing(g, chunk, KW)
        lg, _, yg = g.decode_batch(chunk, want_h=True)
        lo, yo, _, _ = oracle_forward(o, st, chunk, sel, KW)
        rep.check(f"yn@{a} (engine routing)", yg, yo, cos_min=E2E_COS, rel_max=E2E_REL)
        rep.check(f"logits@{a} (engine routing)", lg, lo, cos_min=E2E_COS, rel_max=E2E_REL)
        yns.append(yg)
    O.ORC.orc_state_free(st)
    # the MTP block on the engine's own yn rows (both sides the same input)
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
        rep.check(f"mtp out_h@{a}", og, oo, cos_min=E2E_COS, rel_max=E2E_REL)
        rep.check(f"mtp logits@{a}", lg, lo, cos_min=E2E_COS, rel_max=E2E_REL)
    # three chained MTP steps past the replayed rows, teacher-forced on the
    # engine's picks and hidden rows (the draft chain, c/gmtp.h:677-696)
    tok, prev = int(np.argmax(f32(lg[-1]))), np.ascontiguousarray(og[-1:])
    for i in range(3):
        lo = np.empty((1, V), np.uint16)
        oo = np.empty((1, d), np.uint16)
        pid = np.array([tok], np.int32)
        assert O.ORC.orc_mtp_forward(o.h, mst, O.p(pid), O.p(prev), 1, O.p(lo), O.p(oo)) == 0
        lg1, og1 = g.mtp_forward(pid, prev)
        rep.check(f"chain step {i + 1} out_h", og1, oo, cos_min=E2E_COS, rel_max=E2E_REL)
        rep.check(f"chain step {i + 1} logits", lg1, lo, cos_min=E2E_COS, rel_max=E2E_REL)
        mo = np.sort(f32(lo[0]))
        if (mo[-1] - mo[-2]) > 4 * float(np.abs(f32(lg1[0]) - f32(lo[0])).max()):
            rep.fact(f"chain step {i + 1} pick", int(np.argmax(f32(lg1[0]))) == O.argmax_bf16(lo[0]), "differs")
        tok, prev = int(np.argmax(f32(lg1[0]))), np.ascontiguousarray(og1)
    O.ORC.orc_mtp_state_free(mst)
    rep.finish()


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
    rep = Report("indexer at 2200 tokens")
    for t in range(R):
        nvalid = (pos + t + 1) // kp
        assert nvalid > ksel
        so, sg = scores[t, :nvalid].astype(np.float64), r["iscore"][t, :nvalid].astype(np.float64)
        err = float(np.abs(sg - so).max())
        rep.check(f"row {t} pool scores", sg[None], so[None], to_f=ident)
        ref_sel = set((topk[t][:ksel * kp][topk[t][:ksel * kp] >= 0] // kp).tolist())
        got_sel = set(np.nonzero(r["isel"][t, :nvalid])[0].tolist())
        rep.fact(f"row {t} selects {ksel} pools", len(ref_sel) == ksel and len(got_sel) == ksel,
                 f"{len(ref_sel)} / {len(got_sel)}")
        cut = np.sort(so)[::-1][ksel - 1]
        away = [p for p in ref_sel ^ got_sel if abs(so[p] - cut) > 2 * err + 1e-7]
        rep.fact(f"row {t} selection ({len(ref_sel ^ got_sel)} differ at the cut)", not away,
                 f"pools {away[:8]} differ away from the cut")
        # the tail tokens (the partial pool) are selected too
        tail = [i for i in topk[t][ksel * kp:] if i >= 0]
        assert tail == list(range((pos + t + 1) // kp * kp, pos + t + 1))
    rep.check("DSA output at 2200 tokens", r["sub"], out)
    rep.finish()
