"""The oracle's chunked KDA core (orc_kda_chunk, a restatement of
c/gkda.h:350-539) against the reference's own apus_gkda_chunk compiled from
the reference sources (oracle/_ref): bitwise equal outputs and state (same
libm expf, the same summation orders), ragged chunk edges, several heads,
a carried-in state."""
import numpy as np
import pytest

import oracle as O


def inputs(rng, s, H, D=128):
    q = O.bf16_of(rng.standard_normal((s, H * D)).astype(np.float32))
    k = O.bf16_of(rng.standard_normal((s, H * D)).astype(np.float32))
    v = O.bf16_of(rng.standard_normal((s, H * D)).astype(np.float32))
    g = (-5.0 / (1.0 + np.exp(-rng.standard_normal((s, H * D)) - 2.0))).astype(np.float32)
    beta = O.bf16_of((1.0 / (1.0 + np.exp(-rng.standard_normal((s, H))))).astype(np.float32))
    S0 = (rng.standard_normal((H, D, D)) * 0.05).astype(np.float32)
    return q, k, v, g, beta, S0


def run(fn, q, k, v, g, beta, S0, s, H, D=128):
    S = S0.copy()
    out = np.zeros((s, H * D), np.uint16)
    fn(O.p(q), O.p(k), O.p(v), O.p(g), O.p(beta), O.p(S), O.p(out), s, H, D)
    return out, S


@pytest.mark.skipif(O.REF is None, reason="oracle/_ref is not built (reference sources absent)")
@pytest.mark.parametrize("s,H", [(1, 1), (63, 2), (64, 1), (130, 2)])
def test_kda_chunk_restatement_bitwise(s, H):
    rng = np.random.default_rng(31 * s + H)
    args = inputs(rng, s, H)
    o1, S1 = run(O.ORC.orc_kda_chunk, *args, s, H)
    o2, S2 = run(O.REF.apus_gkda_chunk, *args, s, H)
    assert np.array_equal(o1, o2)
    assert np.array_equal(S1.view(np.uint32), S2.view(np.uint32))
