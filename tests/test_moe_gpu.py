"""The MoE sublayer (c/gmoe.h) on the B200 against the oracle restatement
(orc_moe_forward, bitwise equal to the reference engine on the CPU): routing
exact (teacher-forced and free), outputs within the GEMV tolerance, row-count
invariance bitwise."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from modelgen import fp8_store, tiny_config
from test_linear_gpu import assert_close_rows

pytestmark = pytest.mark.gpu


def moe_weights(rng, E, d, inter):
    W = {"mlp.gate.weight": O.bf16_of((0.05 * rng.standard_normal((E, d))).astype(np.float32)),
         "mlp.gate.e_score_correction_bias": (0.1 * rng.standard_normal(E)).astype(np.float32)}

    def fp8(name, a):
        c, s = fp8_store(a)
        W[name + ".weight"] = c
        W[name + ".weight_scale_inv"] = s

    for e in range(E):
        fp8(f"mlp.experts.{e}.gate_proj", (rng.standard_normal((inter, d)) / np.sqrt(d)).astype(np.float32))
        fp8(f"mlp.experts.{e}.up_proj", (rng.standard_normal((inter, d)) / np.sqrt(d)).astype(np.float32))
        fp8(f"mlp.experts.{e}.down_proj", (rng.standard_normal((d, inter)) / np.sqrt(inter)).astype(np.float32))
    for p, shp in (("gate", (inter, d)), ("up", (inter, d)), ("down", (d, inter))):
        fp8(f"mlp.shared_experts.{p}_proj", (rng.standard_normal(shp) / np.sqrt(shp[1])).astype(np.float32))
    return W


def oracle_moe(kw, W, x, forced=None):
    """orc_moe_forward on a one-layer oracle model holding only the MoE."""
    cfg = O.make_config(**kw)
    m = O.ORC.orc_model_new(C.byref(cfg), 0)
    for n, a in W.items():
        assert O.ORC.orc_model_set(m, ("layers.0." + n).encode(), O.p(a)) == 0, n
    s = x.shape[0]
    out = np.empty_like(x)
    idx = np.empty((s, kw["num_experts_per_tok"]), np.int32)
    w = np.empty((s, kw["num_experts_per_tok"]), np.float32)
    f = None if forced is None else O.p(np.ascontiguousarray(forced, np.int32))
    O.ORC.orc_moe_forward(m, 0, O.p(x), s, O.p(out), O.p(idx), O.p(w), f)
    O.ORC.orc_model_free(m)
    return out, idx, w


def make_moe(G, kw, W, rows=8):
    h = G.apus_gcuda_moe_new(kw["n_routed_experts"], kw["num_experts_per_tok"], kw["hidden_size"],
                             kw["moe_intermediate_size"], kw["routed_scaling_factor"], kw["swiglu_limit"], rows)
    assert h, G.apus_gcuda_last_error()
    for n, a in W.items():
        G.check(G.apus_gcuda_moe_set(h, n.encode(), O.p(a), a.nbytes), n)
    return h


def run_moe(G, h, x, forced=None):
    out = np.zeros_like(x)
    f = None if forced is None else O.p(np.ascontiguousarray(forced, np.int32))
    G.check(G.apus_gcuda_moe_forward2(h, O.p(x), x.shape[0], O.p(out), f), "moe forward2")
    return out


@pytest.fixture(scope="module")
def small(gcuda):
    kw = tiny_config(hidden_size=512, n_routed_experts=16, num_experts_per_tok=4, moe_intermediate_size=256)
    rng = np.random.default_rng(77)
    W = moe_weights(rng, 16, 512, 256)
    h = make_moe(gcuda, kw, W)
    yield kw, W, h
    gcuda.apus_gcuda_moe_free(h)


def test_moe_small_vs_oracle(gcuda, small):
    kw, W, h = small
    rng = np.random.default_rng(5)
    x = O.bf16_of(rng.standard_normal((4, 512)).astype(np.float32))
    got = run_moe(gcuda, h, x)
    idx = np.zeros((4, 4), np.int32)
    w = np.zeros((4, 4), np.float32)
    gcuda.check(gcuda.apus_gcuda_moe_last_routing(h, 4, O.p(idx), O.p(w)))
    ref, ridx, rw = oracle_moe(kw, W, x)
    assert np.array_equal(idx, ridx), (idx, ridx)
    np.testing.assert_allclose(w, rw, rtol=1e-5)
    assert_close_rows(got, ref, fp8=True, elem=4e-2)


def test_moe_forced_selection(gcuda, small):
    kw, W, h = small
    rng = np.random.default_rng(6)
    x = O.bf16_of(rng.standard_normal((3, 512)).astype(np.float32))
    forced = np.array([[15, 0, 7, 3], [1, 2, 3, 4], [9, 8, 7, 6]], np.int32)
    got = run_moe(gcuda, h, x, forced)
    idx = np.zeros((3, 4), np.int32)
    gcuda.check(gcuda.apus_gcuda_moe_last_routing(h, 3, O.p(idx), None))
    assert np.array_equal(idx, forced)
    ref, ridx, _ = oracle_moe(kw, W, x, forced)
    assert np.array_equal(ridx, forced)
    assert_close_rows(got, ref, fp8=True, elem=4e-2)


def test_moe_row_invariance_bitwise(gcuda, small):
    kw, W, h = small
    rng = np.random.default_rng(8)
    x = O.bf16_of(rng.standard_normal((8, 512)).astype(np.float32))
    full = run_moe(gcuda, h, x)
    for m in range(8):
        one = run_moe(gcuda, h, x[m:m + 1])
        assert np.array_equal(one[0], full[m]), m
    assert np.array_equal(run_moe(gcuda, h, x[:4]), full[:4])


def test_moe_config1_vs_oracle(gcuda):
    """288 experts top-8 + shared, hidden 4096, inter 1024,
    4 rows, device-generated weights (seed 1).  The oracle runs on the
    routed experts, downloaded from HBM."""
    kw = tiny_config(hidden_size=4096, n_routed_experts=288, num_experts_per_tok=8, moe_intermediate_size=1024)
    h = gcuda.apus_gcuda_moe_new(288, 8, 4096, 1024, 2.5, 10.0, 4)
    assert h
    try:
        gcuda.check(gcuda.apus_gcuda_moe_init_random(h, 1), "init")
        rng = np.random.default_rng(1)
        x = O.bf16_of(rng.standard_normal((4, 4096)).astype(np.float32))
        got = run_moe(gcuda, h, x)
        idx = np.zeros((4, 8), np.int32)
        gcuda.check(gcuda.apus_gcuda_moe_last_routing(h, 4, O.p(idx), None))
        assert gcuda.apus_gcuda_moe_last_bytes(h) > 0
        # download router + the routed/shared experts; unselected experts get zeros
        W = {}

        def get(name, shape, dt):
            a = np.empty(shape, dt)
            gcuda.check(gcuda.apus_gcuda_moe_get(h, name.encode(), O.p(a), a.nbytes), name)
            W[name] = a

        get("mlp.gate.weight", (288, 4096), np.uint16)
        get("mlp.gate.e_score_correction_bias", (288,), np.float32)
        used = sorted(set(idx.ravel().tolist()))
        for e in range(288):
            for p, shp in (("gate", (1024, 4096)), ("up", (1024, 4096)), ("down", (4096, 1024))):
                sshp = ((shp[0] + 127) // 128, (shp[1] + 127) // 128)
                if e in used:
                    get(f"mlp.experts.{e}.{p}_proj.weight", shp, np.uint8)
                    get(f"mlp.experts.{e}.{p}_proj.weight_scale_inv", sshp, np.float32)
                else:
                    W[f"mlp.experts.{e}.{p}_proj.weight"] = np.zeros(shp, np.uint8)
                    W[f"mlp.experts.{e}.{p}_proj.weight_scale_inv"] = np.zeros(sshp, np.float32)
        for p, shp in (("gate", (1024, 4096)), ("up", (1024, 4096)), ("down", (4096, 1024))):
            get(f"mlp.shared_experts.{p}_proj.weight", shp, np.uint8)
            get(f"mlp.shared_experts.{p}_proj.weight_scale_inv", ((shp[0] + 127) // 128, (shp[1] + 127) // 128),
                np.float32)
        ref, ridx, _ = oracle_moe(kw, W, x)
        assert np.array_equal(idx, ridx)
        assert_close_rows(got, ref, fp8=True, elem=4e-2)
    finally:
        gcuda.apus_gcuda_moe_free(h)
