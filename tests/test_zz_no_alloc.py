"""apus_gcuda_bf16_gemm_argmax_static_dev: the fused BF16 GEMV + greedy pick
whose scratch is a fixed file-scope device array (no cudaMalloc/cudaFree on
any call).  Checked against apus_gcuda_bf16_gemm_argmax_dev on the same
inputs, two calls in a row: the same kernels run on the same split, so the
BF16 outputs and the picks must be bitwise equal (the GEMV test tolerance,
elementwise |err| <= 1e-2 * max(|ref|, rms(ref row)) and cosine >= 0.9999,
is checked too, as a diagnostic that names the row when they are not); plus
the size limits.  This file is collected last on purpose and needs nothing
from the other tests."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)


def _close_rows(got, ref):
    got, ref = got.float().cpu().numpy(), ref.float().cpu().numpy()
    for r in range(ref.shape[0]):
        a, b = got[r].astype(np.float64), ref[r].astype(np.float64)
        rms = float(np.sqrt((b * b).mean()))
        assert np.all(np.abs(a - b) <= 1e-2 * np.maximum(np.abs(b), rms)), f"row {r}"
        cos = a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30)
        assert cos >= 0.9999, f"row {r}: cosine {cos}"


@pytest.mark.parametrize("M,O,K", [(5, 4096, 8192), (1, 40000, 4096), (8, 1000, 6144), (64, 512, 2048)])
def test_static_scratch_matches_pooled(gcuda, M, O, K):
    import torch
    rng = np.random.default_rng(M * 7 + O + K)
    dev = torch.device("cuda:0")
    w = _bf16(rng.standard_normal((O, K)) / np.sqrt(K)).to(dev)
    x = _bf16(rng.standard_normal((M, K))).to(dev)
    y_ref = torch.empty((M, O), dtype=torch.bfloat16, device=dev)
    id_ref = torch.empty(M, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    P = lambda t: C.c_void_p(t.data_ptr())
    assert gcuda.apus_gcuda_bf16_gemm_argmax_dev(P(w), P(x), P(y_ref), P(id_ref), M, O, K, C.c_void_p(st)) == 0
    # one set-up call; then the free device memory must not move across
    # either of two calls (measured tightly around the call itself)
    y = torch.empty_like(y_ref)
    ids = torch.empty_like(id_ref)
    assert gcuda.apus_gcuda_bf16_gemm_argmax_static_dev(P(w), P(x), P(y), P(ids), M, O, K, C.c_void_p(st)) == 0
    for _ in range(2):
        y.fill_(0)
        ids.fill_(-1)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = gcuda.apus_gcuda_bf16_gemm_argmax_static_dev(P(w), P(x), P(y), P(ids), M, O, K, C.c_void_p(st))
        assert rc == 0, gcuda.apus_gcuda_last_error()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0
        _close_rows(y, y_ref)
        assert torch.equal(y, y_ref), "static-scratch outputs differ bitwise from the pooled entry point"
        assert torch.equal(ids, id_ref)
    assert gcuda.apus_gcuda_kernel_error() == 0


def test_static_scratch_limits(gcuda):
    import torch
    dev = torch.device("cuda:0")
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    w = torch.zeros((16, 64), dtype=torch.bfloat16, device=dev)
    x = torch.zeros((65, 64), dtype=torch.bfloat16, device=dev)
    ids = torch.zeros(65, dtype=torch.int32, device=dev)
    P = lambda t: C.c_void_p(t.data_ptr())
    assert gcuda.apus_gcuda_bf16_gemm_argmax_static_dev(P(w), P(x), None, P(ids), 65, 16, 64, st) == -1
    assert b"static maximum" in gcuda.apus_gcuda_last_error()
    # split-K scratch beyond the array: rejected before any launch
    assert gcuda.apus_gcuda_bf16_gemm_argmax_static_dev(P(w), P(x), None, P(ids), 1, 1 << 20, 8192, st) == -1
    assert b"scratch bytes" in gcuda.apus_gcuda_last_error()
