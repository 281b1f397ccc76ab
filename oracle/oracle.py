"""ctypes access to the oracle (TEST INFRASTRUCTURE ONLY).

  ORC — liboracle.so, the C restatement of the reference algorithm
        (oracle/apus_oracle.c), the checker of the CUDA path.
  REF — _ref/libapus_ref.so, the reference's own C engine compiled from its
        sources (oracle/ref_glue.c); None when it was not built.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
import this module.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libapus_ref.so")

ORC = C.CDLL(ORC_PATH)
REF = C.CDLL(REF_PATH) if os.path.exists(REF_PATH) else None

_vp, _sz, _i, _f = C.c_void_p, C.c_size_t, C.c_int, C.c_float


def _decl(lib, name, res, *args):
    f = getattr(lib, name)
    f.restype = res
    f.argtypes = list(args)
    return f


_decl(ORC, "orc_bf16_f32", _f, C.c_uint16)
_decl(ORC, "orc_bf16_bits", C.c_uint16, _f)
_decl(ORC, "orc_e4m3_f32", _f, C.c_uint8)
_decl(ORC, "orc_e4m3_quant", C.c_uint8, _f)
_decl(ORC, "orc_sigmoid", _f, _f)
_decl(ORC, "orc_pw_sum", _f, _vp, _sz)
_decl(ORC, "orc_fp8_dequant", None, _vp, _vp, _vp, _sz, _sz)
_decl(ORC, "orc_bf16_gemm", None, _vp, _vp, _vp, _sz, _sz, _sz)
_decl(ORC, "orc_bf16_gemm_f32", None, _vp, _vp, _vp, _sz, _sz, _sz)
_decl(ORC, "orc_fp8_linear", None, _vp, _vp, _vp, _vp, _sz, _sz, _sz)
_decl(ORC, "orc_argmax_bf16", _i, _vp, _sz)

if REF is not None:
    _decl(REF, "apus_fp8blk_dequant_scalar", None, _vp, _vp, _vp, _sz, _sz)
    _decl(REF, "apus_fp8blk_dequant_mt", None, _vp, _vp, _vp, _sz, _sz)
    _decl(REF, "apus_bf16_gemm_scalar", None, _vp, _vp, _vp, _sz, _sz, _sz)
    _decl(REF, "apus_bf16_gemm_mt", None, _vp, _vp, _vp, _vp, _sz, _sz, _sz)
    _decl(REF, "apus_e4m3_dequant_f32", _f, C.c_uint8)
    _decl(REF, "apus_e4m3_quant_f32", C.c_uint8, _f)
    _decl(REF, "apus_ref_threads", _i)


def p(a):
    return C.c_void_p(a.ctypes.data)


def fp8_dequant(codes, scales):
    O, K = codes.shape
    out = np.empty((O, K), np.uint16)
    ORC.orc_fp8_dequant(p(np.ascontiguousarray(codes)), p(np.ascontiguousarray(scales, np.float32)), p(out), O, K)
    return out


def bf16_gemm(w, x):
    O, K = w.shape
    M = x.shape[0]
    y = np.empty((M, O), np.uint16)
    ORC.orc_bf16_gemm(p(np.ascontiguousarray(w)), p(np.ascontiguousarray(x)), p(y), M, O, K)
    return y


def bf16_gemm_f32(w, x):
    O, K = w.shape
    M = x.shape[0]
    y = np.empty((M, O), np.float32)
    ORC.orc_bf16_gemm_f32(p(np.ascontiguousarray(w)), p(np.ascontiguousarray(x)), p(y), M, O, K)
    return y


def fp8_linear(codes, scales, x):
    O, K = codes.shape
    M = x.shape[0]
    y = np.empty((M, O), np.uint16)
    ORC.orc_fp8_linear(p(np.ascontiguousarray(codes)), p(np.ascontiguousarray(scales, np.float32)),
                       p(np.ascontiguousarray(x)), p(y), M, O, K)
    return y


def argmax_bf16(row):
    row = np.ascontiguousarray(row, np.uint16)
    return ORC.orc_argmax_bf16(p(row), row.size)


# ---- numpy helpers shared by tests and bench -------------------------------

def f32_of(codes):
    return (np.asarray(codes, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_of(x):
    """RNE f32 -> BF16 codes (the 0x7FFF + lsb rule of c/num.h:153-160)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    return np.where(nan, (u >> 16) & 0xFFFF, r).astype(np.uint16)
