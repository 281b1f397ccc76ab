"""The resident glm5_next model and the on-device MTP speculative step
(include/apus_gmtp_gcuda.h) against the oracle restatement
(oracle/apus_oracle_model.c, itself bitwise equal to the reference engine).

Two kinds of checks:
  * against the oracle, within tolerance: the GPU reductions sum fp32 in a
    different order than the reference's sequential loops, and a flipped BF16
    rounding point propagates through the layers.  Tolerance per logits row:
    cosine >= 0.999 and max |gpu - oracle| <= 0.05 * max |oracle|; greedy
    picks must agree wherever the oracle's top-2 margin exceeds 4x the
    row's observed error.
  * inside the engine, bitwise: a verify row equals the one-token decode of
    the same context, so the speculative stream IS the engine's greedy
    stream (c/gmtp.h:40-52), and the committed state after accept/rollback
    equals a plain decode of the emitted tokens (tests/m8g/test_m8g.c:383-424).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from modelgen import gen_weights, tiny_config

pytestmark = pytest.mark.gpu

PROMPT = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]


@pytest.fixture(scope="module")
def tiny():
    kw = tiny_config()
    W = gen_weights(kw, seed=20261201)
    return kw, W


def gpu_model(gcuda, kw, W, cap=256, depth=4):
    m = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=cap, depth=depth)
    m.load(W)
    return m


def orc_model(kw, W):
    return O.Model(O.make_config(**kw), W, True, "orc")


def f32(a):
    return O.f32_of(np.ascontiguousarray(a, np.uint16))


def assert_rows_close(g, o, what, cos_min=0.999, rel=0.05):
    g, o = f32(g).reshape(len(g), -1), f32(o).reshape(len(o), -1)
    for r in range(len(o)):
        a, b = g[r].astype(np.float64), o[r].astype(np.float64)
        cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))
        err = float(np.abs(a - b).max())
        bound = rel * float(np.abs(b).max())
        assert cos >= cos_min and err <= bound, f"{what} row {r}: cos {cos:.6f} err {err:.4g} > {bound:.4g}"


def margin(row):
    v = np.sort(f32(row))
    return float(v[-1] - v[-2])


def test_decode_batch_vs_oracle(gcuda, tiny):
    kw, W = tiny
    g, o = gpu_model(gcuda, kw, W), orc_model(kw, W)
    st = o.state(256)
    ids = np.array(PROMPT + [1, 2, 3, 200, 100, 50, 25, 12, 6, 3, 383, 382], np.int32)
    p = 0
    for k in (3, 1, 8, 6, 5):
        chunk = ids[p:p + k]
        lg, hg, yg = g.decode_batch(chunk, want_h=True)
        lo, ho, yo = o.decode_batch(st, chunk, want_h=True)
        assert_rows_close(yg, yo, f"yn@{p}")
        assert_rows_close(hg, ho, f"h@{p}")
        assert_rows_close(lg, lo, f"logits@{p}")
        for r in range(k):
            err = float(np.abs(f32(lg[r]) - f32(lo[r])).max())
            if margin(lo[r]) > 4 * err:
                assert int(np.argmax(f32(lg[r]))) == O.argmax_bf16(lo[r])
        p += k
    assert g.pos() == p


def test_mtp_forward_vs_oracle(gcuda, tiny):
    kw, W = tiny
    g, o = gpu_model(gcuda, kw, W), orc_model(kw, W)
    st = o.state(256)
    ids = np.array(PROMPT, np.int32)
    _, _, yn = o.decode_batch(st, ids, want_h=True)
    mst = O.ORC.orc_mtp_state_new(o.h, 256)
    V, d = kw["vocab_size"], kw["hidden_size"]
    n = len(ids) - 1
    for a, b in ((0, 6), (6, 7), (7, n)):
        pid = np.ascontiguousarray(ids[1 + a:1 + b])
        ph = np.ascontiguousarray(yn[a:b])
        lo = np.empty((b - a, V), np.uint16)
        oo = np.empty((b - a, d), np.uint16)
        assert O.ORC.orc_mtp_forward(o.h, mst, O.p(pid), O.p(ph), b - a, O.p(lo), O.p(oo)) == 0
        lg, og = g.mtp_forward(pid, ph)
        assert_rows_close(og, oo, f"mtp h@{a}")
        assert_rows_close(lg, lo, f"mtp logits@{a}")
    O.ORC.orc_mtp_state_free(mst)


def test_greedy_vs_oracle(gcuda, tiny):
    """Long enough for the indexer's pool selection to bind (index_topk 8 of
    kpool 4: 2 pools + the tail out of up to 10)."""
    kw, W = tiny
    n_gen = 30
    o = orc_model(kw, W)
    ids = np.array(PROMPT, np.int32)
    ref = np.zeros(n_gen, np.int32)
    assert O.ORC.orc_greedy(o.h, o.state(256), O.p(ids), len(ids), n_gen, O.p(ref)) == 0
    g = gpu_model(gcuda, kw, W)
    out = g.greedy(ids, n_gen)
    if out != ref.tolist():
        j = next(i for i in range(n_gen) if out[i] != ref[i])
        # teacher-forced oracle logits of the step that differs (the prompt
        # pass, then one-token decodes): only a near tie may flip
        st = o.state(256)
        lo = o.prefill(st, ids)
        for a in range(0, j, 8):
            lo = o.decode_batch(st, ref[a:min(a + 8, j)].astype(np.int32))
        assert margin(lo[-1]) < 0.05 * float(np.abs(f32(lo[-1])).max()), f"greedy differs at {j}"


@pytest.mark.parametrize("depth", [1, 2, 3, 4, 8])
def test_spec_equals_greedy(gcuda, tiny, depth):
    kw, W = tiny
    g = gpu_model(gcuda, kw, W, depth=depth)
    g.spec_prefill(PROMPT)
    out = []
    for _ in range(10):
        e = g.spec_step()
        assert 1 <= len(e) <= depth
        out += e
    stats, rc = g.stats()
    assert rc == 0 and stats["emitted"] == len(out) and stats["batches"] == 10
    assert stats["pos"] == len(PROMPT) + len(out)
    assert g.emitted() == out
    ref = gpu_model(gcuda, kw, W).greedy(PROMPT, len(out) + 1)
    assert out == ref[:len(out)]
    assert stats["held"] == ref[len(out)]


def test_spec_forced_full_accept(gcuda, tiny):
    """draft_override pattern (tests/m8g/test_m8g.c:686-694): truth drafts are
    all accepted, depth tokens per step."""
    kw, W = tiny
    depth = 4
    truth = gpu_model(gcuda, kw, W).greedy(PROMPT, 60)
    g = gpu_model(gcuda, kw, W, depth=depth)
    g.force(truth, base=len(PROMPT), p=1.0)
    g.spec_prefill(PROMPT)
    out = []
    for _ in range(6):
        e = g.spec_step()
        assert len(e) == depth
        out += e
    stats, _ = g.stats()
    assert stats["accepted"] == stats["offered"] == 6 * (depth - 1)
    assert out == truth[:len(out)]


def test_spec_forced_partial_accept_rollback(gcuda, tiny):
    """Drafts right with probability 1/2: rejections roll the KDA state back
    to a checkpoint and rewind the DSA caches; the committed state must be
    bitwise that of decoding the emitted tokens."""
    kw, W = tiny
    depth = 5
    truth = gpu_model(gcuda, kw, W).greedy(PROMPT, 80)
    g = gpu_model(gcuda, kw, W, depth=depth)
    g.force(truth, base=len(PROMPT), p=0.5, seed=7)
    g.spec_prefill(PROMPT)
    out = []
    for _ in range(12):
        out += g.spec_step()
    stats, _ = g.stats()
    assert 0 < stats["accepted"] < stats["offered"]
    assert out == truth[:len(out)]
    dig = g.digest()
    # the prompt pass on a fresh sequence, then a plain decode of the emitted tokens
    g.prefill(PROMPT, want_logits=False)
    ctx = np.array(out, np.int32)
    for a in range(0, len(ctx), 8):
        g.decode_batch(ctx[a:a + 8])
    assert g.digest() == dig


def test_async_steps_equal_sync(gcuda, tiny):
    kw, W = tiny
    a = gpu_model(gcuda, kw, W, depth=3)
    a.spec_prefill(PROMPT)
    sync = []
    for _ in range(8):
        sync += a.spec_step()
    b = gpu_model(gcuda, kw, W, depth=3)
    b.spec_prefill(PROMPT)
    for _ in range(8):
        b.spec_step_async()
    assert b.emitted() == sync


def test_graph_steps_equal_sync(gcuda, tiny):
    """The full-depth step captured once into a CUDA graph and replayed."""
    kw, W = tiny
    a = gpu_model(gcuda, kw, W, depth=4)
    a.spec_prefill(PROMPT)
    sync = []
    for _ in range(10):
        sync += a.spec_step()
    b = gpu_model(gcuda, kw, W, depth=4)
    b.use_graph(True)
    b.spec_prefill(PROMPT)
    for _ in range(10):
        b.spec_step_async()
    assert b.emitted() == sync
    c = b.counters()
    assert c["graph_kernels"] > 20 and c["moe_problems"] > 0
    assert b.digest() == a.digest()


def test_capacity_edge(gcuda, tiny):
    """Near the capacity the verify batch shrinks to cap - q rows
    (c/gmtp.h:783-786); at the capacity a step emits nothing."""
    kw, W = tiny
    cap = 40
    g = gpu_model(gcuda, kw, W, cap=cap, depth=4)
    g.spec_prefill(PROMPT)
    out = []
    for _ in range(cap):
        e = g.spec_step()
        if not e:
            break
        out += e
    assert len(out) == cap - len(PROMPT)
    assert g.spec_step() == []
    ref = gpu_model(gcuda, kw, W).greedy(PROMPT, len(out))
    assert out == ref


def test_errors(gcuda, tiny):
    kw, W = tiny
    g = gpu_model(gcuda, kw, W, cap=32)
    with pytest.raises(gcuda.GcudaError):
        g.set("layers.0.self_attn.q_proj.weight", np.zeros(3, np.uint16))
    with pytest.raises(gcuda.GcudaError):
        g.set("layers.0.no_such_tensor", np.zeros(3, np.uint16))
    with pytest.raises(gcuda.GcudaError):
        g.decode_batch(np.zeros(9, np.int32))      # more than 8 rows
    bad = dict(kw, hc_mult=9)
    with pytest.raises(gcuda.GcudaError):
        gcuda.GModel(gcuda.make_config(**bad))


def test_sync_steps_replay_graph(gcuda, tiny):
    """With graphs on, the synchronous step replays the captured step; mixing
    synchronous and enqueued steps (the control block read back by the
    previous synchronous step is stale then) keeps the same stream."""
    kw, W = tiny
    a = gpu_model(gcuda, kw, W, depth=4)
    a.spec_prefill(PROMPT)
    eager = []
    for _ in range(9):
        eager += a.spec_step()
    b = gpu_model(gcuda, kw, W, depth=4)
    b.use_graph(True)
    b.spec_prefill(PROMPT)
    got = []
    for i in range(9):
        if i == 4:
            b.spec_step_async()
            got = b.emitted()
        else:
            got += b.spec_step()
    assert got == eager
    assert b.emitted() == eager
    assert b.counters()["graph_kernels"] > 20
    assert b.digest() == a.digest()
