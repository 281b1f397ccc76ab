"""The sampler restatements (oracle/apus_oracle.c) pinned against the
reference's own sampler (c/sample.h): the golden tokens of
tests/golden/sample.npz, made by tests/golden/gen_sample_golden.py from the
compiled reference, and fresh rows against oracle/_ref when it is built.

Two restatements: orc_sample_logits_u follows the reference's arithmetic
(libm expf, sequential double sums) and must equal it bitwise;
orc_sample_exact is the B200 sampler's exact-integer arithmetic (the
bitwise checker of the CUDA kernel) and must give the reference's token on
every golden case."""
import os

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN

import sys
sys.path.insert(0, GOLDEN)
from sample_cases import cases  # noqa: E402

G = np.load(os.path.join(GOLDEN, "sample.npz"))
CASES = cases()


def test_case_list_matches_fixture():
    assert [c[0] for c in CASES] == list(G["names"])


def test_rng_golden():
    for seed, want in zip(G["rng_seeds"], G["rng_draws"]):
        got, state = O.rng_draws(int(seed), 8)
        assert got == [int(x) for x in want]
        assert state == (int(seed) + 8 * O.GOLDEN) & O.M64


@pytest.mark.parametrize("i", range(len(CASES)))
def test_restatement_golden(i):
    name, row, temp, top_p, u53 = CASES[i]
    assert O.sample_logits_u(row, temp, top_p, u53 * 2.0 ** -53) == G["tokens"][i], name


@pytest.mark.parametrize("i", range(len(CASES)))
def test_exact_arithmetic_golden(i):
    name, row, temp, top_p, u53 = CASES[i]
    assert O.sample_exact(row, temp, top_p, u53) == G["tokens"][i], name


def test_zero_signs_tie_to_lowest_index():
    """-0 and +0 are one value: the greedy pick is the lowest index holding
    either (c/sample.h:76-81, strict >)."""
    name, row, temp, top_p, u53 = next(c for c in CASES if c[0] == "zeros_t0.0_p1.0")
    assert O.sample_exact(row, 0.0, 1.0, 0) == 3 == O.sample_logits_u(row, 0.0, 1.0, 0.0)


@pytest.mark.skipif(O.REF is None, reason="oracle/_ref is not built (reference sources absent)")
def test_restatement_equals_reference_fresh_rows():
    rng = np.random.default_rng(77)
    agree_exact = 0
    n = 0
    for V, sigma in ((154880, 1.0), (154880, 3.0), (4096, 0.3), (384, 2.0)):
        for temp, top_p in ((0.8, 0.95), (1.0, 1.0), (0.6, 0.8)):
            for _ in range(3):
                row = O.bf16_of(rng.standard_normal(V).astype(np.float32) * sigma)
                u53 = int(rng.integers(0, 1 << 53))
                ref = O.ref_sample_logits_u(row, temp, top_p, u53 * 2.0 ** -53)
                assert O.sample_logits_u(row, temp, top_p, u53 * 2.0 ** -53) == ref
                agree_exact += O.sample_exact(row, temp, top_p, u53) == ref
                n += 1
    # the exact arithmetic differs only when u * kept or top_p lies within
    # ~1e-7 of a cumulative-mass boundary
    assert agree_exact >= n - 1, (agree_exact, n)
