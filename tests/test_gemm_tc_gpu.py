"""The tcgen05 GEMM (csrc/gemm_tc.cu) behind the linear-leaf drop-ins for 64
rows or more: BF16 and FP8-block (dequantised to BF16 first, c/fp8blk.h)
weights, BF16 and fp32 outputs, ragged edges in every dimension.  The
reference is the exact product rounded once (float64 numpy), held to the
linear leaf's tolerance (per row relative L2 <= 1e-2, cosine >= 0.9999,
elementwise ceiling); the fp32 output must sit within fp32 accumulation
error of the exact product.  The dispatch counter shows that one tensor-core
launch, not 8-row GEMV launches, produced the result."""
import numpy as np
import pytest

import oracle as O
from test_linear_gpu import assert_close_rows, fp8_weights

pytestmark = pytest.mark.gpu


def exact_bf16(w_codes, x_codes):
    r = O.f32_of(x_codes).astype(np.float64) @ O.f32_of(w_codes).astype(np.float64).T
    return O.bf16_of(r.astype(np.float32)), r


def run(gcuda, W, x, S=None, f32=False):
    import torch
    fp8 = S is not None
    dW = torch.from_numpy(np.ascontiguousarray(W).view(np.uint8 if fp8 else np.int16)).cuda()
    dS = torch.from_numpy(S).cuda() if fp8 else None
    dx = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda()
    M, O_, K = x.shape[0], W.shape[0], W.shape[1]
    dy = torch.zeros((M, O_), dtype=torch.float32 if f32 else torch.int16, device="cuda")
    d0 = gcuda.apus_gcuda_dispatches()
    st = gcuda.stream_of()
    if fp8:
        rc = gcuda.apus_gcuda_fp8blk_linear_dev(gcuda.ptr(dW), gcuda.ptr(dS), gcuda.ptr(dx), gcuda.ptr(dy),
                                                M, O_, K, st)
    elif f32:
        rc = gcuda.apus_gcuda_bf16_gemm_f32_dev(gcuda.ptr(dW), gcuda.ptr(dx), gcuda.ptr(dy), M, O_, K, st)
    else:
        rc = gcuda.apus_gcuda_bf16_gemm_dev(gcuda.ptr(dW), gcuda.ptr(dx), gcuda.ptr(dy), M, O_, K, st)
    gcuda.check(rc, "linear")
    torch.cuda.synchronize()
    assert gcuda.apus_gcuda_kernel_error() == 0
    launches = gcuda.apus_gcuda_dispatches() - d0
    out = dy.cpu().numpy()
    return (out if f32 else out.view(np.uint16)), launches


SHAPES = [(64, 256, 512), (128, 128, 64), (200, 300, 136), (256, 1024, 128), (512, 4096, 4096),
          (130, 2048, 8192), (1000, 96, 1024), (128, 4096, 4096), (96, 1536, 4096)]


@pytest.mark.parametrize("shape", SHAPES)
def test_bf16(gcuda, shape):
    M, O_, K = shape
    rng = np.random.default_rng(M * 7 + O_ + K)
    w = O.bf16_of((rng.standard_normal((O_, K)) * 0.02).astype(np.float32))
    x = O.bf16_of(rng.standard_normal((M, K)).astype(np.float32))
    got, launches = run(gcuda, w, x)
    assert launches == 1
    want, _ = exact_bf16(w, x)
    assert_close_rows(got, want)


@pytest.mark.parametrize("shape", [(64, 512, 4096), (256, 4096, 4096), (96, 1536, 4096), (300, 2048, 1024)])
def test_fp8(gcuda, shape):
    M, O_, K = shape
    rng = np.random.default_rng(M + O_ * 3 + K)
    c, s = fp8_weights(rng, O_, K)
    x = O.bf16_of(rng.standard_normal((M, K)).astype(np.float32))
    got, launches = run(gcuda, c, x, S=s)
    assert launches == 1
    want, _ = exact_bf16(O.fp8_dequant(c, s), x)     # bf16(sum x * bf16(dequant(W)))
    assert_close_rows(got, want, fp8=False)


def test_f32_output(gcuda):
    rng = np.random.default_rng(3)
    M, O_, K = 192, 288, 4096                    # the router's shape at a prefill chunk
    w = O.bf16_of((rng.standard_normal((O_, K)) * 0.02).astype(np.float32))
    x = O.bf16_of(rng.standard_normal((M, K)).astype(np.float32))
    got, launches = run(gcuda, w, x, f32=True)
    assert launches == 1
    _, exact = exact_bf16(w, x)
    # fp32 accumulation of exact BF16 products: |error| <= K * 2^-24 * sum |terms|
    bound = K * 2.0 ** -24 * (np.abs(O.f32_of(x)).astype(np.float64) @ np.abs(O.f32_of(w)).astype(np.float64).T)
    assert np.all(np.abs(got.astype(np.float64) - exact) <= bound + 1e-30)


def test_small_row_counts_stay_on_the_gemv(gcuda):
    """Fewer than 64 rows keep the batch-invariant 8-row GEMV launches."""
    rng = np.random.default_rng(4)
    w = O.bf16_of((rng.standard_normal((512, 1024)) * 0.02).astype(np.float32))
    x = O.bf16_of(rng.standard_normal((63, 1024)).astype(np.float32))
    got, launches = run(gcuda, w, x)
    assert launches == 8
    assert_close_rows(got, exact_bf16(w, x)[0])


def test_repeatable(gcuda):
    """Repeated calls are bitwise equal (a fixed tile plan and summation
    order)."""
    rng = np.random.default_rng(8)
    w = O.bf16_of((rng.standard_normal((2048, 4096)) * 0.02).astype(np.float32))
    x = O.bf16_of(rng.standard_normal((128, 4096)).astype(np.float32))
    a, _ = run(gcuda, w, x)
    b, _ = run(gcuda, w, x)
    assert np.array_equal(a, b)
    assert_close_rows(a, exact_bf16(w, x)[0])
