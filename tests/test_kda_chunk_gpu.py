"""The chunked KDA prefill core on the B200 (apus_gcuda_kda_chunk_dev)
against the reference's own apus_gkda_chunk (c/gkda.h:350-539, compiled from
the reference sources into oracle/_ref): ragged chunk edges, several heads,
a carried-in state.  Each head's sums run in the reference's order, so the
outputs differ only through expf's last bits: per row cosine >= 0.9999 and
max |diff| <= 1e-2 of the row's max (the north-star logits bound), the
state within 1e-3 of its max.  The recurrent core (apus_gkda_recurrent) is
the same function of the inputs up to rounding and is held to the same
bound."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def inputs(rng, s, H, D=128):
    q = O.bf16_of(rng.standard_normal((s, H * D)).astype(np.float32))
    k = O.bf16_of(rng.standard_normal((s, H * D)).astype(np.float32))
    v = O.bf16_of(rng.standard_normal((s, H * D)).astype(np.float32))
    g = (-5.0 / (1.0 + np.exp(-rng.standard_normal((s, H * D)) - 2.0))).astype(np.float32)  # in (-5, 0)
    beta = O.bf16_of((1.0 / (1.0 + np.exp(-rng.standard_normal((s, H))))).astype(np.float32))
    S0 = (rng.standard_normal((H, D, D)) * 0.05).astype(np.float32)
    return q, k, v, g, beta, S0


def ref(fn, q, k, v, g, beta, S0, s, H, D=128):
    S = S0.copy()
    out = np.zeros((s, H * D), np.uint16)
    fn(O.p(q), O.p(k), O.p(v), O.p(g), O.p(beta), O.p(S), O.p(out), s, H, D)
    return out, S


def dev(gcuda, q, k, v, g, beta, S0, s, H, D=128):
    import torch
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dq, dk, dv = (t(a.view(np.int16)) for a in (q, k, v))
    dg, db, dS = t(g), t(beta.view(np.int16)), t(S0.copy())
    dout = torch.zeros((s, H * D), dtype=torch.int16, device="cuda")
    gcuda.check(gcuda.apus_gcuda_kda_chunk_dev(gcuda.ptr(dq), gcuda.ptr(dk), gcuda.ptr(dv), gcuda.ptr(dg),
                                               gcuda.ptr(db), gcuda.ptr(dS), gcuda.ptr(dout), s, H, D,
                                               gcuda.stream_of()), "kda_chunk")
    torch.cuda.synchronize()
    return dout.cpu().numpy().view(np.uint16), dS.cpu().numpy()


def close(got, want, H, D=128):
    g = O.f32_of(got).astype(np.float64).reshape(len(got), H, D)
    w = O.f32_of(want).astype(np.float64).reshape(len(want), H, D)
    for t in range(len(w)):
        for h in range(H):
            a, b = g[t, h], w[t, h]
            nb = np.linalg.norm(b)
            if nb == 0:
                assert np.abs(a).max() == 0
                continue
            assert a @ b / (np.linalg.norm(a) * nb) >= 0.9999, (t, h)
            assert np.abs(a - b).max() <= 1e-2 * np.abs(b).max(), (t, h)


@pytest.mark.parametrize("s,H", [(1, 2), (64, 2), (100, 3), (300, 4)])
def test_chunk_vs_reference(gcuda, s, H):
    """Against the oracle's restatement (bitwise the reference's
    apus_gkda_chunk, tests/test_oracle_kda_cpu.py) and, when oracle/_ref is
    built, the reference's own chunked and recurrent cores."""
    rng = np.random.default_rng(s * 10 + H)
    args = inputs(rng, s, H)
    got_o, got_S = dev(gcuda, *args, s, H)
    fns = [O.ORC.orc_kda_chunk]
    if O.REF is not None:
        fns += [O.REF.apus_gkda_chunk, O.REF.apus_gkda_recurrent]
    for fn in fns:
        want_o, want_S = ref(fn, *args, s, H)
        close(got_o, want_o, H)
        assert np.abs(got_S - want_S).max() <= 1e-3 * np.abs(want_S).max()


def test_chunk_rejects_other_head_dims(gcuda):
    import torch
    z = torch.zeros(64, dtype=torch.int16, device="cuda")
    assert gcuda.apus_gcuda_kda_chunk_dev(gcuda.ptr(z), gcuda.ptr(z), gcuda.ptr(z), gcuda.ptr(z), gcuda.ptr(z),
                                          gcuda.ptr(z), gcuda.ptr(z), 1, 1, 64, gcuda.stream_of()) == -1
    gcuda.apus_gcuda_clear_error()
