"""The model-level oracle restatement (oracle/apus_oracle_model.c) against
the reference's own C engine (oracle/_ref) on a tiny seeded model: the
decode batch, the MTP forward and the full greedy speculative loop must be
BITWISE equal (same host libm on both sides, same rounding points), and the
speculative stream must equal plain greedy decoding (the reference's own
equivalence property, c/gmtp.h:40-52)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from modelgen import gen_weights, tiny_config

needs_ref = pytest.mark.skipif(O.REF is None, reason="reference engine not built")


@pytest.fixture(scope="module")
def tiny():
    kw = tiny_config()
    cfg = O.make_config(**kw)
    W = gen_weights(kw, seed=20261201)
    return kw, cfg, W


@needs_ref
def test_decode_batch_bitwise_vs_reference(tiny):
    kw, cfg, W = tiny
    mo, mr = O.Model(cfg, W, True, "orc"), O.Model(cfg, W, True, "ref")
    so, sr = mo.state(64), mr.state(64)
    ids = np.array([5, 17, 300, 2, 99, 42, 7, 381, 0, 11], np.int32)
    for chunk in (ids[:3], ids[3:4], ids[4:10]):
        lo, ho, yo = mo.decode_batch(so, chunk, True)
        lr, hr, yr = mr.decode_batch(sr, chunk, True)
        assert np.array_equal(lo, lr)
        assert np.array_equal(ho, hr)
        assert np.array_equal(yo, yr)


@needs_ref
@pytest.mark.parametrize("n", [1, 11, 64, 150])
def test_prefill_bitwise_vs_reference(tiny, n):
    """apus_gmodel_prefill_h: the prompt in one call (chunked KDA over 64-row
    chunks, the DSA over the whole prompt); logits, streams and post-norm
    rows of every position, then one decode batch on the state it left."""
    kw, cfg, W = tiny
    mo, mr = O.Model(cfg, W, True, "orc"), O.Model(cfg, W, True, "ref")
    so, sr = mo.state(256), mr.state(256)
    ids = np.random.default_rng(n).integers(0, kw["vocab_size"], n).astype(np.int32)
    lo, ho, yo = mo.prefill(so, ids, True)
    lr, hr, yr = mr.prefill(sr, ids, True)
    assert np.array_equal(lo, lr)
    assert np.array_equal(ho, hr)
    assert np.array_equal(yo, yr)
    # the last row alone is the same row
    st = mo.state(256)
    ll, yl = mo.prefill_last(st, ids)
    assert np.array_equal(ll, lo[-1]) and np.array_equal(yl, yo)
    nxt = np.array([7, 3], np.int32)
    assert np.array_equal(mo.decode_batch(so, nxt), mr.decode_batch(sr, nxt))


def test_prefill_differs_from_decode_batches(tiny):
    """The prompt pass is not the decode batch: the chunked KDA core sums in
    another order, so the two orderings agree closely but not bitwise."""
    kw, cfg, W = tiny
    m = O.Model(cfg, W, True, "orc")
    ids = np.random.default_rng(5).integers(0, kw["vocab_size"], 40).astype(np.int32)
    lp = m.prefill(m.state(64), ids)
    sd = m.state(64)
    ld = np.concatenate([m.decode_batch(sd, ids[i:i + 8]) for i in range(0, 40, 8)])
    a, b = O.f32_of(lp).astype(np.float64), O.f32_of(ld).astype(np.float64)
    cos = (a * b).sum(1) / np.sqrt((a * a).sum(1) * (b * b).sum(1))
    assert cos.min() > 0.999
    assert not np.array_equal(lp, ld)


def test_batch_equals_sequential_in_oracle(tiny):
    """Decode-batch interleave: R rows == R one-token decodes (c/gmodel.h:302-310)."""
    kw, cfg, W = tiny
    m = O.Model(cfg, W, True, "orc")
    s1, s2 = m.state(64), m.state(64)
    ids = np.array([3, 1, 4, 1, 5, 9, 2, 6], np.int32)
    full = m.decode_batch(s1, ids)
    one = np.concatenate([m.decode_batch(s2, ids[i:i + 1]) for i in range(len(ids))])
    assert np.array_equal(full, one)


def _run_spec(kind, tiny, depth, n_steps, prompt, hook=None):
    kw, cfg, W = tiny
    m = O.Model(cfg, W, True, kind)
    st = m.state(256)
    if kind == "orc":
        mst = O.ORC.orc_mtp_state_new(m.h, 256)
        sp = O.ORC.orc_spec_new(m.h, st, mst, depth)
        lib, pre = O.ORC, "orc_"
    else:
        sp = O.REF.ref_spec_new(m.h, st, 256, depth)
        lib, pre = O.REF, "ref_"
    if hook is not None:
        getattr(lib, pre + "spec_set_draft_hook")(sp, C.cast(hook, C.c_void_p), None)
    ids = np.asarray(prompt, np.int32)
    assert getattr(lib, pre + "spec_prefill")(sp, O.p(ids), len(ids)) == 0
    out = []
    buf = np.zeros(depth + 1, np.int32)
    for _ in range(n_steps):
        n = getattr(lib, pre + "spec_step")(sp, O.p(buf), depth + 1)
        assert n >= 1
        out.extend(buf[:n].tolist())
    stats = np.zeros(7, np.uint64)
    getattr(lib, pre + "spec_stats")(sp, O.p(stats))
    return out, stats, m


@needs_ref
@pytest.mark.parametrize("depth", [2, 4])
def test_spec_loop_bitwise_vs_reference(tiny, depth):
    prompt = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]
    so, sto, _ = _run_spec("orc", tiny, depth, 6, prompt)
    sr, str_, _ = _run_spec("ref", tiny, depth, 6, prompt)
    assert so == sr
    assert np.array_equal(sto, str_)


@pytest.mark.parametrize("depth", [1, 2, 4])
def test_spec_equals_greedy_in_oracle(tiny, depth):
    kw, cfg, W = tiny
    prompt = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]
    out, stats, _ = _run_spec("orc", tiny, depth, 8, prompt)
    m = O.Model(cfg, W, True, "orc")
    st = m.state(256)
    ref = np.zeros(len(out), np.int32)
    ids = np.asarray(prompt, np.int32)
    assert O.ORC.orc_greedy(m.h, st, O.p(ids), len(ids), len(out), O.p(ref)) == 0
    assert out == ref.tolist()


def test_forced_drafts_full_accept(tiny):
    """draft_override pattern (tests/m8g/test_m8g.c:686-694): truth drafts are
    all accepted with a bonus token each step."""
    kw, cfg, W = tiny
    prompt = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]
    m = O.Model(cfg, W, True, "orc")
    st = m.state(256)
    truth = np.zeros(40, np.int32)
    ids = np.asarray(prompt, np.int32)
    O.ORC.orc_greedy(m.h, st, O.p(ids), len(ids), 40, O.p(truth))
    n0 = len(prompt)

    @O.DRAFT_HOOK
    def hook(ctx, q, drafts, n):
        for i in range(n):   # d_i predicts position q + i
            drafts[i] = int(truth[q + i - n0]) if q + i - n0 < len(truth) else 0

    out, stats, _ = _run_spec("orc", tiny, 4, 5, prompt, hook=hook)
    assert out == truth[:len(out)].tolist()
    assert stats[4] == stats[3]          # every offered draft accepted
    assert len(out) == 5 * 4             # held + 3 accepted drafts per step
