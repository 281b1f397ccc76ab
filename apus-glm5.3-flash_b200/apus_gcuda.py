"""apus_gcuda — Python host mirror of the apus B200 engine's C ABI.

Loads libapus_gcuda.so (built in-tree by this folder's Makefile) with ctypes
and exposes the entry points of include/apus_gcuda.h and
include/apus_gmodel_gcuda.h with the reference's names and argument meaning
(c/fp8blk.h, c/bf16.h, c/gmoe.h, c/gmtp.h).  There is no CPU fallback: if
the shared library is missing or fails to load, importing this module
raises.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libapus_gcuda.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"apus_gcuda: {LIB_PATH} is not built (run make in {HERE})")

lib = C.CDLL(LIB_PATH)

_vp, _sz, _i, _u64 = C.c_void_p, C.c_size_t, C.c_int, C.c_uint64


def _fn(name, res, *args):
    f = getattr(lib, name)
    f.restype = res
    f.argtypes = list(args)
    return f


apus_gcuda_enable = _fn("apus_gcuda_enable", _i, C.c_char_p, _sz)
apus_gcuda_disable = _fn("apus_gcuda_disable", None)
apus_gcuda_is_enabled = _fn("apus_gcuda_is_enabled", _i)
apus_gcuda_last_error = _fn("apus_gcuda_last_error", C.c_char_p)
apus_gcuda_kernel_error = _fn("apus_gcuda_kernel_error", _i)
apus_gcuda_register_region = _fn("apus_gcuda_register_region", _i, _vp, _sz)
apus_gcuda_unregister_region = _fn("apus_gcuda_unregister_region", None, _vp)
apus_gcuda_bytes_pinned = _fn("apus_gcuda_bytes_pinned", _u64)
apus_gcuda_dispatches = _fn("apus_gcuda_dispatches", _u64)
apus_gcuda_offload_bf16 = _fn("apus_gcuda_offload_bf16", _u64)
apus_gcuda_offload_fp8blk = _fn("apus_gcuda_offload_fp8blk", _u64)
apus_gcuda_bf16_gemm = _fn("apus_gcuda_bf16_gemm", _i, _vp, _vp, _vp, _sz, _sz, _sz)
apus_gcuda_fp8blk_linear = _fn("apus_gcuda_fp8blk_linear", _i, _vp, _vp, _vp, _vp, _sz, _sz, _sz)
apus_fp8blk_nblocks = _fn("apus_fp8blk_nblocks", _sz, _sz)
apus_fp8blk_dequant = _fn("apus_fp8blk_dequant", None, _vp, _vp, _vp, _sz, _sz)
apus_fp8blk_dequant_mt = _fn("apus_fp8blk_dequant_mt", None, _vp, _vp, _vp, _sz, _sz)
apus_bf16_gemv_mt = _fn("apus_bf16_gemv_mt", None, _vp, _vp, _vp, _vp, _sz, _sz)
apus_bf16_gemm_mt = _fn("apus_bf16_gemm_mt", None, _vp, _vp, _vp, _vp, _sz, _sz, _sz)
apus_gcuda_set_pdl = _fn("apus_gcuda_set_pdl", None, _i)
apus_fp8blk_dequant_dev = _fn("apus_fp8blk_dequant_dev", _i, _vp, _vp, _vp, _sz, _sz, _vp)
apus_gcuda_fp8blk_linear_dev = _fn("apus_gcuda_fp8blk_linear_dev", _i, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp)
apus_gcuda_bf16_gemm_dev = _fn("apus_gcuda_bf16_gemm_dev", _i, _vp, _vp, _vp, _sz, _sz, _sz, _vp)
apus_gcuda_bf16_gemm_f32_dev = _fn("apus_gcuda_bf16_gemm_f32_dev", _i, _vp, _vp, _vp, _sz, _sz, _sz, _vp)
apus_gcuda_bf16_gemm_argmax_dev = _fn("apus_gcuda_bf16_gemm_argmax_dev", _i, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp)

_f = C.c_float
apus_gcuda_moe_new = _fn("apus_gcuda_moe_new", _vp, _i, _i, _sz, _sz, _f, _f, _i)
apus_gcuda_moe_free = _fn("apus_gcuda_moe_free", None, _vp)
apus_gcuda_moe_set = _fn("apus_gcuda_moe_set", _i, _vp, C.c_char_p, _vp, _sz)
apus_gcuda_moe_get = _fn("apus_gcuda_moe_get", _i, _vp, C.c_char_p, _vp, _sz)
apus_gcuda_moe_init_random = _fn("apus_gcuda_moe_init_random", _i, _vp, C.c_uint64)
apus_gcuda_moe_forward_dev = _fn("apus_gcuda_moe_forward_dev", _i, _vp, _vp, _sz, _vp, _vp, _vp)
apus_gcuda_moe_forward2 = _fn("apus_gcuda_moe_forward2", _i, _vp, _vp, _sz, _vp, _vp)
apus_gcuda_moe_last_routing = _fn("apus_gcuda_moe_last_routing", _i, _vp, _sz, _vp, _vp)
apus_gcuda_moe_last_bytes = _fn("apus_gcuda_moe_last_bytes", _u64, _vp)


class GcudaError(RuntimeError):
    pass


def check(rc, what=""):
    if rc != 0:
        raise GcudaError(f"{what}: {apus_gcuda_last_error().decode(errors='replace')}")


def enable():
    err = C.create_string_buffer(256)
    if apus_gcuda_enable(err, 256) != 0:
        raise GcudaError(err.value.decode())


def ptr(a):
    """Address of a numpy array or torch tensor (host or device)."""
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return C.c_void_p(a.ctypes.data)


def stream_of(torch_stream=None):
    import torch
    s = torch_stream if torch_stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)
