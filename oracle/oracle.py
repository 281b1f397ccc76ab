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
_decl(ORC, "orc_rng_next", C.c_uint64, C.POINTER(C.c_uint64))
_decl(ORC, "orc_sample_logits_u", _i, _vp, _sz, _f, _f, C.c_double)
_decl(ORC, "orc_sample_exact", _i, _vp, _sz, _f, _f, C.c_uint64)
_decl(ORC, "orc_kda_chunk", None, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz)

if REF is not None:
    _decl(REF, "apus_fp8blk_dequant_scalar", None, _vp, _vp, _vp, _sz, _sz)
    _decl(REF, "apus_fp8blk_dequant_mt", None, _vp, _vp, _vp, _sz, _sz)
    _decl(REF, "apus_bf16_gemm_scalar", None, _vp, _vp, _vp, _sz, _sz, _sz)
    _decl(REF, "apus_bf16_gemm_mt", None, _vp, _vp, _vp, _vp, _sz, _sz, _sz)
    _decl(REF, "apus_e4m3_dequant_f32", _f, C.c_uint8)
    _decl(REF, "apus_e4m3_quant_f32", C.c_uint8, _f)
    _decl(REF, "apus_ref_threads", _i)
    _decl(REF, "apus_sample_logits_u", _i, _vp, _sz, _f, _f, C.c_double, _vp)
    _decl(REF, "apus_sample", _i, _vp, _sz, _f, _f, _vp, _vp)
    _decl(REF, "apus_gkda_chunk", None, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz)
    _decl(REF, "apus_gkda_recurrent", None, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz)


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


# ---- model-level restatement (apus_oracle_model.c) -------------------------

MAX_LAYERS = 64
_CFG_FIELDS = [
    ("hidden_size", C.c_int), ("vocab_size", C.c_int), ("num_hidden_layers", C.c_int),
    ("rms_norm_eps", C.c_float), ("hc_mult", C.c_int), ("hc_sinkhorn_iters", C.c_int),
    ("hc_eps", C.c_float), ("first_k_dense_replace", C.c_int), ("intermediate_size", C.c_int),
    ("moe_intermediate_size", C.c_int), ("n_routed_experts", C.c_int), ("n_shared_experts", C.c_int),
    ("num_experts_per_tok", C.c_int), ("routed_scaling_factor", C.c_float), ("norm_topk_prob", C.c_int),
    ("swiglu_limit", C.c_float), ("num_attention_heads", C.c_int), ("q_lora_rank", C.c_int),
    ("kv_lora_rank", C.c_int), ("qk_nope_head_dim", C.c_int), ("v_head_dim", C.c_int),
    ("index_n_heads", C.c_int), ("index_head_dim", C.c_int), ("index_topk", C.c_int),
    ("index_kpool", C.c_int), ("index_kpool_always_select_tail", C.c_int), ("linear_num_heads", C.c_int),
    ("linear_head_dim", C.c_int), ("linear_conv_kernel_dim", C.c_int), ("linear_lower_bound", C.c_float),
    ("num_nextn_predict_layers", C.c_int), ("layer_is_dsa", C.c_int * MAX_LAYERS),
    ("mlp_is_sparse", C.c_int * MAX_LAYERS),
]


class Config(C.Structure):
    """Field names of ApusGmodelConfig (c/gmodel.h:88-108); also the layout of
    OrcConfig and ApusGcudaConfig."""
    _fields_ = _CFG_FIELDS


def make_config(**kw):
    c = Config()
    for name, _ in _CFG_FIELDS:
        if name in ("layer_is_dsa", "mlp_is_sparse"):
            continue
        setattr(c, name, kw[name])
    L = kw["num_hidden_layers"]
    for i in range(L):
        c.layer_is_dsa[i] = int(kw["layer_is_dsa"][i])
        c.mlp_is_sparse[i] = int(kw["mlp_is_sparse"][i])
    return c


_decl(ORC, "orc_model_new", _vp, _vp, _i)
_decl(ORC, "orc_model_free", None, _vp)
_decl(ORC, "orc_model_set", _i, _vp, C.c_char_p, _vp)
_decl(ORC, "orc_state_new", _vp, _vp, _sz)
_decl(ORC, "orc_state_free", None, _vp)
_decl(ORC, "orc_state_pos", _sz, _vp)
_decl(ORC, "orc_decode_batch", _i, _vp, _vp, _vp, _sz, _vp, _vp, _vp)
_decl(ORC, "orc_mtp_state_new", _vp, _vp, _sz)
_decl(ORC, "orc_mtp_state_free", None, _vp)
_decl(ORC, "orc_mtp_forward", _i, _vp, _vp, _vp, _vp, _sz, _vp, _vp)
_decl(ORC, "orc_spec_new", _vp, _vp, _vp, _vp, _i)
_decl(ORC, "orc_spec_free", None, _vp)
_decl(ORC, "orc_spec_set_draft_hook", None, _vp, _vp, _vp)
_decl(ORC, "orc_spec_prefill", _i, _vp, _vp, _sz)
_decl(ORC, "orc_spec_step", _i, _vp, _vp, _i)
_decl(ORC, "orc_spec_stats", None, _vp, _vp)
_decl(ORC, "orc_greedy", _i, _vp, _vp, _vp, _sz, _i, _vp)
_decl(ORC, "orc_rmsnorm", None, _vp, _vp, _vp, _sz, _f)
_decl(ORC, "orc_hc_pre", None, _vp, _i, _i, _vp, _vp, _vp, _vp)
_decl(ORC, "orc_hc_post", None, _vp, _vp, _vp, _vp, _vp, _sz, _sz)
_decl(ORC, "orc_hc_head", None, _vp, _vp, _sz, _sz)
_decl(ORC, "orc_moe_forward", None, _vp, _i, _vp, _sz, _vp, _vp, _vp, _vp)
_decl(ORC, "orc_kda_decode", None, _vp, _i, _vp, _sz, _vp, _vp, _vp)
_decl(ORC, "orc_dsa_decode", None, _vp, _i, _vp, _sz, _vp, _vp)
_decl(ORC, "orc_dsa_width", _sz, _vp)
_decl(ORC, "orc_mlp_forward", None, _vp, _i, _vp, _sz, _vp)
_decl(ORC, "orc_decode_batch_ex", _i, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp)
_decl(ORC, "orc_dsa_decode_sel", None, _vp, _i, _vp, _sz, _vp, _vp, _vp, _vp, _sz)
_decl(ORC, "orc_state_set_pos", None, _vp, _sz)
_decl(ORC, "orc_state_load_kda", _i, _vp, _i, _vp, _vp)
_decl(ORC, "orc_state_load_dsa", _i, _vp, _i, _vp, _vp, _vp, _vp, _sz)
_decl(ORC, "orc_mtp_state_load", _i, _vp, _vp, _vp, _vp, _vp, _vp, _sz)
_decl(ORC, "orc_spec_set_force_hook", None, _vp, _vp, _vp)
_decl(ORC, "orc_spec_raw_drafts", None, _vp, _vp, _vp)
_decl(ORC, "orc_prefill_h", _i, _vp, _vp, _vp, _sz, _vp, _vp, _vp)
_decl(ORC, "orc_prefill_last", _i, _vp, _vp, _vp, _sz, _vp, _vp, _vp)
_decl(ORC, "orc_kda_prefill", None, _vp, _i, _vp, _sz, _vp, _vp, _vp)
_decl(ORC, "orc_spec_walk", _i, _vp, _i, _sz, _vp, C.c_int32, _vp, C.POINTER(C.c_int), C.POINTER(C.c_int32))

DRAFT_HOOK = C.CFUNCTYPE(None, _vp, C.c_int64, C.POINTER(C.c_int32), C.c_int)

if REF is not None:
    _decl(REF, "ref_model_new", _vp, _vp, _i)
    _decl(REF, "ref_model_set", _i, _vp, C.c_char_p, _vp)
    _decl(REF, "ref_model_finalize", None, _vp)
    _decl(REF, "ref_state_new", _vp, _vp, _sz)
    _decl(REF, "ref_state_free", None, _vp)
    _decl(REF, "ref_decode_batch", _i, _vp, _vp, _vp, _sz, _vp, _vp, _vp)
    _decl(REF, "ref_prefill_h", _i, _vp, _vp, _vp, _sz, _vp, _vp, _vp)
    _decl(REF, "ref_spec_new", _vp, _vp, _vp, _sz, _i)
    _decl(REF, "ref_spec_free", None, _vp)
    _decl(REF, "ref_spec_set_draft_hook", None, _vp, _vp, _vp)
    _decl(REF, "ref_spec_prefill", _i, _vp, _vp, _sz)
    _decl(REF, "ref_spec_step", _i, _vp, _vp, _i)
    _decl(REF, "ref_spec_stats", None, _vp, _vp)
    _decl(REF, "ref_mtp_forward", _i, _vp, _vp, _vp, _sz, _vp, _vp)


class Model:
    """A weight dict (name -> numpy array, caller-owned) bound to the oracle
    restatement (kind='orc') or the reference engine (kind='ref')."""

    def __init__(self, cfg, weights, has_mtp, kind="orc"):
        self.cfg, self.w, self.kind = cfg, weights, kind
        self.lib = ORC if kind == "orc" else REF
        if kind == "orc":
            self.h = ORC.orc_model_new(C.byref(cfg), int(has_mtp))
            setter = ORC.orc_model_set
        else:
            self.h = REF.ref_model_new(C.byref(cfg), int(has_mtp))
            setter = REF.ref_model_set
        for name, arr in weights.items():
            if setter(self.h, name.encode(), p(arr)) != 0:
                raise KeyError(name)
        if kind == "ref":
            REF.ref_model_finalize(self.h)

    def state(self, cap):
        return (ORC.orc_state_new if self.kind == "orc" else REF.ref_state_new)(self.h, cap)

    def decode_batch(self, st, ids, want_h=False):
        cfg = self.cfg
        s = len(ids)
        ids = np.ascontiguousarray(ids, np.int32)
        logits = np.empty((s, cfg.vocab_size), np.uint16)
        h = np.empty((s, cfg.hc_mult * cfg.hidden_size), np.uint16)
        yn = np.empty((s, cfg.hidden_size), np.uint16)
        fn = ORC.orc_decode_batch if self.kind == "orc" else REF.ref_decode_batch
        rc = fn(self.h, st, p(ids), s, p(logits), p(h), p(yn))
        assert rc == 0
        return (logits, h, yn) if want_h else logits

    def prefill(self, st, ids, want_h=False):
        """apus_gmodel_prefill_h: the prompt pass (chunked KDA, DSA over the
        prompt in one call); logits of every row."""
        cfg = self.cfg
        s = len(ids)
        ids = np.ascontiguousarray(ids, np.int32)
        logits = np.empty((s, cfg.vocab_size), np.uint16)
        h = np.empty((s, cfg.hc_mult * cfg.hidden_size), np.uint16)
        yn = np.empty((s, cfg.hidden_size), np.uint16)
        fn = ORC.orc_prefill_h if self.kind == "orc" else REF.ref_prefill_h
        rc = fn(self.h, st, p(ids), s, p(logits), p(h), p(yn))
        assert rc == 0
        return (logits, h, yn) if want_h else logits

    def prefill_last(self, st, ids):
        """The prompt pass with the last row's logits only: (logits [V], yn [s][d])."""
        assert self.kind == "orc"
        cfg = self.cfg
        s = len(ids)
        ids = np.ascontiguousarray(ids, np.int32)
        logits = np.empty(cfg.vocab_size, np.uint16)
        yn = np.empty((s, cfg.hidden_size), np.uint16)
        assert ORC.orc_prefill_last(self.h, st, p(ids), s, p(logits), None, p(yn)) == 0
        return logits, yn


def spec_walk(logits16, drafts, held):
    """c/gmtp.h:807-831 (greedy) on De rows of BF16 logits: (emitted,
    matched, next held)."""
    lg = np.ascontiguousarray(logits16, np.uint16)
    De, V = lg.shape
    dr = np.zeros(max(De, 1), np.int32)
    dr[:len(drafts)] = drafts[:De]
    out = np.zeros(De + 1, np.int32)
    matched, nh = C.c_int(0), C.c_int32(0)
    ne = ORC.orc_spec_walk(p(lg), De, V, p(dr), int(held), p(out), C.byref(matched), C.byref(nh))
    return out[:ne].tolist(), matched.value, nh.value


# ---- sampling (c/sample.h:91-177) ----

GOLDEN = 0x9E3779B97F4A7C15
M64 = (1 << 64) - 1


def rng_draws(state, n):
    """The next n splitmix64 outputs after `state` and the state after them
    (c/sample.h:159-166)."""
    s = C.c_uint64(state)
    out = [ORC.orc_rng_next(C.byref(s)) for _ in range(n)]
    return out, s.value


def sample_logits_u(row, temp, top_p, u):
    """c/sample.h apus_sample_logits_u on a BF16 codes row (restatement)."""
    row = np.ascontiguousarray(row, np.uint16)
    return ORC.orc_sample_logits_u(p(row), row.size, temp, top_p, u)


def sample_exact(row, temp, top_p, u53):
    """The same draw in the B200 sampler's exact arithmetic (u = u53 * 2^-53)."""
    row = np.ascontiguousarray(row, np.uint16)
    return ORC.orc_sample_exact(p(row), row.size, temp, top_p, u53)


def ref_sample_logits_u(row, temp, top_p, u):
    """The reference's own apus_sample_logits_u on the widened row (REF only)."""
    lf = np.ascontiguousarray(f32_of(np.ascontiguousarray(row, np.uint16)))
    scratch = np.empty(row.size * 8, np.uint8)
    return REF.apus_sample_logits_u(p(lf), row.size, temp, top_p, u, p(scratch))
