"""The oracle restatement (oracle/apus_oracle.c) pinned against the
reference: the golden fixtures generated from the reference's numpy oracle
(tests/golden/gen_golden.py) and, when built, the reference's own C engine
(oracle/_ref/libapus_ref.so)."""
import os

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN

LIN = np.load(os.path.join(GOLDEN, "linear.npz"))
COD = np.load(os.path.join(GOLDEN, "codec.npz"))


def test_e4m3_decode_all_codes():
    tab = COD["e4m3_table"]
    for c in range(256):
        v = O.ORC.orc_e4m3_f32(c)
        if np.isnan(tab[c]):            # oracle table NaN; C engine decodes +-480
            assert abs(v) == 480.0
        else:
            assert np.float32(v).view(np.uint32) == tab[c].view(np.uint32), c


def test_e4m3_quant_rne():
    xin, want = COD["e4m3_in"], COD["e4m3_out"]
    got = np.array([O.ORC.orc_e4m3_quant(float(v)) for v in xin], np.uint8)
    assert np.array_equal(got, want)


def test_bf16_rounding():
    xin, want = COD["bf16_in"], COD["bf16_out"]
    got = np.array([O.ORC.orc_bf16_bits(float(v)) for v in xin], np.uint16)
    assert np.array_equal(got, want)
    assert np.array_equal(O.bf16_of(xin), want)


@pytest.mark.parametrize("i", range(8))
def test_dequant_golden(i):
    c, s, want = LIN[f"deq{i}_codes"], LIN[f"deq{i}_scales"], LIN[f"deq{i}_out"]
    assert np.array_equal(O.fp8_dequant(c, s), want)


@pytest.mark.parametrize("i", range(9))
def test_gemm_golden(i):
    w, x, want = LIN[f"gem{i}_w"], LIN[f"gem{i}_x"], LIN[f"gem{i}_y"]
    assert np.array_equal(O.bf16_gemm(w, x), want)


@pytest.mark.parametrize("i", range(4))
def test_fp8_linear_golden(i):
    c, s, x, want = (LIN[f"lin{i}_{k}"] for k in ("codes", "scales", "x", "y"))
    assert np.array_equal(O.fp8_linear(c, s, x), want)


def test_argmax_ties_lowest_index():
    row = np.array([0x3F80, 0x4000, 0x4000, 0x3F00], np.uint16)
    assert O.argmax_bf16(row) == 1
    row = np.full(100, 0xBF80, np.uint16)
    assert O.argmax_bf16(row) == 0


def test_pw_sum_matches_numpy():
    rng = np.random.default_rng(3)
    for n in (1, 7, 8, 9, 127, 128, 129, 300, 4096, 16384, 5000):
        a = rng.standard_normal(n).astype(np.float32)
        got = np.float32(O.ORC.orc_pw_sum(O.p(a), n))
        assert got.view(np.uint32) == np.float32(a.sum()).view(np.uint32), n


needs_ref = pytest.mark.skipif(O.REF is None, reason="reference engine not built")


@needs_ref
def test_restatement_equals_reference_engine():
    rng = np.random.default_rng(11)
    for (M, Ov, K) in [(1, 130, 257), (4, 256, 512), (3, 128, 128)]:
        c = rng.integers(0, 256, size=(Ov, K), dtype=np.uint8)
        c[c == 0x7F] = 0
        c[c == 0xFF] = 0
        s = np.exp2(rng.uniform(-9, -5, size=((Ov + 127) // 128, (K + 127) // 128))).astype(np.float32)
        ref = np.empty((Ov, K), np.uint16)
        O.REF.apus_fp8blk_dequant_scalar(O.p(c), O.p(s), O.p(ref), Ov, K)
        assert np.array_equal(O.fp8_dequant(c, s), ref)
        x = O.bf16_of(rng.standard_normal((M, K)).astype(np.float32))
        yref = np.empty((M, Ov), np.uint16)
        O.REF.apus_bf16_gemm_scalar(O.p(ref), O.p(x), O.p(yref), M, Ov, K)
        assert np.array_equal(O.bf16_gemm(ref, x), yref)
