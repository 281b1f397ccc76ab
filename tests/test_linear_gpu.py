"""Parity of the linear leaf on the B200: FP8 block dequant (bitwise),
FP8/BF16 decode GEMV (tolerance per row: relative L2 error <= 1e-2 and
cosine >= 0.9999, the north-star bound for GEMM logits, plus an elementwise
ceiling), row-count invariance (bitwise) and the fused greedy pick (bitwise
given the kernel's own logits)."""
import os

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
LIN = np.load(os.path.join(GOLDEN, "linear.npz"))

REL_TOL = 1e-2        # per row: ||got - ref|| / ||ref||
COS_TOL = 0.9999
# Elementwise ceiling, relative to max(|ref|, rms(ref row)).  BF16 weights:
# only the fp32 summation order differs, so 1e-2.  FP8 weights: the kernel
# applies each 128x128 block scale to the MMA partial instead of rounding
# every dequantized weight to BF16 (<= 2^-9 relative per weight), so an
# output may sit one more BF16 ulp (<= 0.78 %) from the reference: 2e-2.
# A whole MoE layer (FP8 gate/up -> BF16 SwiGLU -> FP8 down -> BF16-rounded
# weighted adds) can compound that to a few ulps: callers pass elem=4e-2.
ELEM_TOL = {False: 1e-2, True: 2e-2}


def assert_close_rows(got_codes, ref_codes, fp8=False, elem=None):
    g = O.f32_of(got_codes).astype(np.float64)
    r = O.f32_of(ref_codes).astype(np.float64)
    for m in range(r.shape[0]):
        scale = np.sqrt(np.mean(r[m] ** 2)) + 1e-30
        err = np.abs(g[m] - r[m])
        tol = elem if elem is not None else ELEM_TOL[fp8]
        assert np.all(err <= tol * np.maximum(np.abs(r[m]), scale)), (m, err.max(), scale)
        nr = np.linalg.norm(r[m])
        if nr > 0:
            assert np.linalg.norm(g[m] - r[m]) <= REL_TOL * nr, (m, np.linalg.norm(g[m] - r[m]) / nr)
            cos = g[m] @ r[m] / (np.linalg.norm(g[m]) * nr)
            assert cos >= COS_TOL, (m, cos)


def fp8_weights(rng, O_, K):
    """BASELINE config-0 distribution: round-to-E4M3 of N(0,1)*64 (no NaN
    codes), F32 scales log-uniform in [1e-4, 1e-2]."""
    v = np.clip(rng.standard_normal((O_, K)).astype(np.float32) * 64, -448, 448)
    codes = np.vectorize(lambda f: O.ORC.orc_e4m3_quant(float(f)), otypes=[np.uint8])(v) \
        if O_ * K <= 4096 else _quant_np(v)
    s = np.exp(rng.uniform(np.log(1e-4), np.log(1e-2),
                           size=((O_ + 127) // 128, (K + 127) // 128))).astype(np.float32)
    return codes, s


def _quant_np(v):
    """Vectorised E4M3 RNE quantiser equal to c/num.h:110-134 (checked
    against the oracle on a sample below)."""
    import torch
    t = torch.from_numpy(v).to(torch.float8_e4m3fn)
    return t.view(torch.uint8).numpy().copy()


def test_quant_np_matches_oracle():
    rng = np.random.default_rng(1)
    v = np.clip(rng.standard_normal(5000).astype(np.float32) * 64, -448, 448)
    want = np.array([O.ORC.orc_e4m3_quant(float(f)) for f in v], np.uint8)
    assert np.array_equal(_quant_np(v), want)


@pytest.mark.parametrize("i", range(8))
def test_dequant_host_dropin_bitwise(gcuda, i):
    c, s, want = LIN[f"deq{i}_codes"], LIN[f"deq{i}_scales"], LIN[f"deq{i}_out"]
    out = np.zeros_like(want)
    gcuda.apus_gcuda_clear_error()
    gcuda.apus_fp8blk_dequant(O.p(c), O.p(s), O.p(out), c.shape[0], c.shape[1])
    assert gcuda.apus_gcuda_last_error().decode() == ""
    assert np.array_equal(out, want)


def test_dequant_dev_bitwise_all_codes(gcuda):
    import torch
    rng = np.random.default_rng(7)
    O_, K = 384, 1024
    c = rng.integers(0, 256, size=(O_, K), dtype=np.uint8)   # includes 0x7F/0xFF
    s = np.exp2(rng.uniform(-30, 30, size=(3, 8))).astype(np.float32)
    want = O.fp8_dequant(c, s)
    dc, ds = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    dout = torch.empty((O_, K), dtype=torch.int16, device="cuda")
    gcuda.check(gcuda.apus_fp8blk_dequant_dev(gcuda.ptr(dc), gcuda.ptr(ds), gcuda.ptr(dout), O_, K,
                                              gcuda.stream_of()), "dequant")
    torch.cuda.synchronize()
    assert np.array_equal(dout.cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("i", range(9))
def test_bf16_gemm_golden(gcuda, i):
    w, x, want = LIN[f"gem{i}_w"], LIN[f"gem{i}_x"], LIN[f"gem{i}_y"]
    y = np.zeros_like(want)
    assert gcuda.apus_gcuda_bf16_gemm(O.p(w), O.p(x), O.p(y), x.shape[0], w.shape[0], w.shape[1]) == 0
    assert_close_rows(y, want)


@pytest.mark.parametrize("i", range(4))
def test_fp8_linear_golden(gcuda, i):
    c, s, x, want = (LIN[f"lin{i}_{k}"] for k in ("codes", "scales", "x", "y"))
    y = np.zeros_like(want)
    assert gcuda.apus_gcuda_fp8blk_linear(O.p(c), O.p(s), O.p(x), O.p(y),
                                          x.shape[0], c.shape[0], c.shape[1]) == 0
    assert_close_rows(y, want, fp8=True)


def _dev_linear(gcuda, fp8, W, S, x):
    import torch
    dW = torch.from_numpy(np.ascontiguousarray(W)).cuda()
    dS = torch.from_numpy(S).cuda() if fp8 else None
    dx = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda()
    M, O_ = x.shape[0], W.shape[0]
    dy = torch.zeros((M, O_), dtype=torch.int16, device="cuda")
    if fp8:
        rc = gcuda.apus_gcuda_fp8blk_linear_dev(gcuda.ptr(dW), gcuda.ptr(dS), gcuda.ptr(dx), gcuda.ptr(dy),
                                                M, O_, W.shape[1], gcuda.stream_of())
    else:
        rc = gcuda.apus_gcuda_bf16_gemm_dev(gcuda.ptr(dW), gcuda.ptr(dx), gcuda.ptr(dy),
                                            M, O_, W.shape[1], gcuda.stream_of())
    gcuda.check(rc, "linear_dev")
    torch.cuda.synchronize()
    assert gcuda.apus_gcuda_kernel_error() == 0
    return dy.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("shape", [(4, 4096, 4096), (1, 1536, 4096), (8, 512, 4096), (3, 4096, 1024),
                                   (4, 300, 1536), (4, 520, 16384), (6, 256, 12288)])
def test_fp8_gemv_vs_oracle(gcuda, shape):
    M, O_, K = shape
    rng = np.random.default_rng(hash(shape) & 0xffff)
    c, s = fp8_weights(rng, O_, K)
    x = O.bf16_of(rng.standard_normal((M, K)).astype(np.float32))
    got = _dev_linear(gcuda, True, c, s, x)
    assert_close_rows(got, O.fp8_linear(c, s, x), fp8=True)


@pytest.mark.parametrize("shape", [(4, 4096, 4096), (1, 2048, 8192), (5, 288, 4096), (2, 40, 512),
                                   (4, 1000, 8192), (8, 64, 6144)])
def test_bf16_gemv_vs_oracle(gcuda, shape):
    M, O_, K = shape
    rng = np.random.default_rng(hash(shape) & 0xffff)
    w = O.bf16_of((rng.standard_normal((O_, K)) * 0.02).astype(np.float32))
    x = O.bf16_of(rng.standard_normal((M, K)).astype(np.float32))
    got = _dev_linear(gcuda, False, w, None, x)
    assert_close_rows(got, O.bf16_gemm(w, x))


@pytest.mark.parametrize("fp8,K", [(True, 2048), (False, 2048), (True, 12288), (False, 8192)])
def test_row_count_invariance_bitwise(gcuda, fp8, K):
    """Row m of an R-row call is bitwise the 1-row call on row m (the
    property speculative verify == sequential decode rests on), with and
    without the split-K reduction."""
    rng = np.random.default_rng(5)
    O_ = 1024
    if fp8:
        W, S = fp8_weights(rng, O_, K)
    else:
        W, S = O.bf16_of((rng.standard_normal((O_, K)) * 0.05).astype(np.float32)), None
    x = O.bf16_of(rng.standard_normal((8, K)).astype(np.float32))
    full = _dev_linear(gcuda, fp8, W, S, x)
    for R in (1, 3, 8):
        part = _dev_linear(gcuda, fp8, W, S, x[:R])
        assert np.array_equal(part, full[:R])
    for m in range(8):
        one = _dev_linear(gcuda, fp8, W, S, x[m:m + 1])
        assert np.array_equal(one[0], full[m])


def test_argmax_fused(gcuda):
    import torch
    rng = np.random.default_rng(9)
    V, K, M = 20000, 1024, 4
    w = O.bf16_of((rng.standard_normal((V, K)) * 0.02).astype(np.float32))
    w[777] = w[123]            # exact duplicate rows -> possible exact ties
    x = O.bf16_of(rng.standard_normal((M, K)).astype(np.float32))
    x[2] = O.bf16_of(O.f32_of(w[123]) * 4)   # row 2 peaks at rows 123 and 777
    dW = torch.from_numpy(w.view(np.int16)).cuda()
    dx = torch.from_numpy(x.view(np.int16)).cuda()
    dy = torch.zeros((M, V), dtype=torch.int16, device="cuda")
    ids = torch.full((M,), -1, dtype=torch.int32, device="cuda")
    gcuda.check(gcuda.apus_gcuda_bf16_gemm_argmax_dev(gcuda.ptr(dW), gcuda.ptr(dx), gcuda.ptr(dy), gcuda.ptr(ids),
                                                      M, V, K, gcuda.stream_of()), "argmax")
    torch.cuda.synchronize()
    logits = dy.cpu().numpy().view(np.uint16)
    got = ids.cpu().numpy()
    for m in range(M):
        assert got[m] == O.argmax_bf16(logits[m])
    assert got[2] == 123
    assert_close_rows(logits, O.bf16_gemm(w, x))
