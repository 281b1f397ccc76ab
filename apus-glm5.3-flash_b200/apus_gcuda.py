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

import synth

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
apus_gcuda_clear_error = _fn("apus_gcuda_clear_error", None)
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
apus_gcuda_bf16_gemm_argmax_static_dev = _fn("apus_gcuda_bf16_gemm_argmax_static_dev", _i, _vp, _vp, _vp, _vp,
                                             _sz, _sz, _sz, _vp)
apus_gcuda_sample_rows_dev = _fn("apus_gcuda_sample_rows_dev", _i, _vp, _sz, _sz, _sz, C.c_float, C.c_float,
                                 _u64, _vp, _vp)
apus_gcuda_kda_chunk_dev = _fn("apus_gcuda_kda_chunk_dev", _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz,
                               _vp)

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


# ---- the resident model + speculative step (include/apus_gmtp_gcuda.h) ----

MAX_LAYERS = 64
_CFG_FIELDS = [
    ("hidden_size", _i), ("vocab_size", _i), ("num_hidden_layers", _i), ("rms_norm_eps", _f),
    ("hc_mult", _i), ("hc_sinkhorn_iters", _i), ("hc_eps", _f), ("first_k_dense_replace", _i),
    ("intermediate_size", _i), ("moe_intermediate_size", _i), ("n_routed_experts", _i),
    ("n_shared_experts", _i), ("num_experts_per_tok", _i), ("routed_scaling_factor", _f),
    ("norm_topk_prob", _i), ("swiglu_limit", _f), ("num_attention_heads", _i), ("q_lora_rank", _i),
    ("kv_lora_rank", _i), ("qk_nope_head_dim", _i), ("v_head_dim", _i), ("index_n_heads", _i),
    ("index_head_dim", _i), ("index_topk", _i), ("index_kpool", _i), ("index_kpool_always_select_tail", _i),
    ("linear_num_heads", _i), ("linear_head_dim", _i), ("linear_conv_kernel_dim", _i),
    ("linear_lower_bound", _f), ("num_nextn_predict_layers", _i),
    ("layer_is_dsa", _i * MAX_LAYERS), ("mlp_is_sparse", _i * MAX_LAYERS),
]


class GcudaConfig(C.Structure):
    """ApusGcudaConfig: the field names and meaning of ApusGmodelConfig
    (c/gmodel.h:88-108) with the per-layer patterns inline."""
    _fields_ = _CFG_FIELDS


def make_config(**kw):
    c = GcudaConfig()
    for name, _ in _CFG_FIELDS:
        if name not in ("layer_is_dsa", "mlp_is_sparse"):
            setattr(c, name, kw[name])
    for i in range(kw["num_hidden_layers"]):
        c.layer_is_dsa[i] = int(kw["layer_is_dsa"][i])
        c.mlp_is_sparse[i] = int(kw["mlp_is_sparse"][i])
    return c


_cs = C.c_char_p
apus_gcuda_model_new = _fn("apus_gcuda_model_new", _vp, _vp, _i, _sz, _i)
apus_gcuda_model_free = _fn("apus_gcuda_model_free", None, _vp)
apus_gcuda_config_load = _fn("apus_gcuda_config_load", _i, _cs, _vp, _vp, _sz)
apus_gcuda_container_check = _fn("apus_gcuda_container_check", _i, _cs, _vp, _i, _vp, _sz)
apus_gcuda_container_read = _fn("apus_gcuda_container_read", C.c_long, _cs, _cs, _vp, _sz, _vp, _sz)
apus_gcuda_model_load_container = _fn("apus_gcuda_model_load_container", _i, _vp, _cs, _vp, _sz)
apus_gcuda_model_new_ep = _fn("apus_gcuda_model_new_ep", _vp, _vp, _i, _sz, _i, _i, _i)
apus_gcuda_model_ep_handle = _fn("apus_gcuda_model_ep_handle", _i, _vp, _vp)
apus_gcuda_model_ep_connect = _fn("apus_gcuda_model_ep_connect", _i, _vp, _vp)
apus_gcuda_model_set = _fn("apus_gcuda_model_set", _i, _vp, _cs, _vp, _sz)
apus_gcuda_model_get = _fn("apus_gcuda_model_get", _i, _vp, _cs, _vp, _sz)
apus_gcuda_model_init_random = _fn("apus_gcuda_model_init_random", _i, _vp, _u64)
apus_gcuda_model_reset = _fn("apus_gcuda_model_reset", _i, _vp)
apus_gcuda_model_pos = _fn("apus_gcuda_model_pos", _sz, _vp)
apus_gcuda_decode_batch = _fn("apus_gcuda_decode_batch", _i, _vp, _vp, _sz, _vp, _vp, _vp)
apus_gcuda_mtp_forward = _fn("apus_gcuda_mtp_forward", _i, _vp, _vp, _vp, _sz, _vp, _vp)
apus_gcuda_prefill = _fn("apus_gcuda_prefill", _i, _vp, _vp, _sz, _vp, _vp)
apus_gcuda_gspec_prefill = _fn("apus_gcuda_gspec_prefill", _i, _vp, _vp, _sz)
apus_gcuda_gspec_step = _fn("apus_gcuda_gspec_step", _i, _vp, _vp, _i)
apus_gcuda_gspec_step_async = _fn("apus_gcuda_gspec_step_async", _i, _vp)
apus_gcuda_gspec_emitted = _fn("apus_gcuda_gspec_emitted", _i, _vp, _vp, _sz)
apus_gcuda_gspec_stats = _fn("apus_gcuda_gspec_stats", _i, _vp, _vp)
apus_gcuda_gspec_force = _fn("apus_gcuda_gspec_force", _i, _vp, _vp, _sz, _sz, C.c_double, _u64)
apus_gcuda_greedy = _fn("apus_gcuda_greedy", _i, _vp, _vp, _sz, _i, _vp)
apus_gcuda_generate = _fn("apus_gcuda_generate", _i, _vp, _vp, _sz, _i, _vp)
apus_gcuda_gspec_sampling = _fn("apus_gcuda_gspec_sampling", _i, _vp, C.c_float, C.c_float, _u64)
apus_gcuda_rng_state = _fn("apus_gcuda_rng_state", _i, _vp, C.POINTER(_u64))
apus_gcuda_state_digest = _fn("apus_gcuda_state_digest", _u64, _vp)
apus_gcuda_gspec_use_graph = _fn("apus_gcuda_gspec_use_graph", _i, _vp, _i)
apus_gcuda_model_stream = _fn("apus_gcuda_model_stream", _vp, _vp)
apus_gcuda_model_counters = _fn("apus_gcuda_model_counters", _i, _vp, _vp, _sz)
apus_gcuda_model_debug_stop = _fn("apus_gcuda_model_debug_stop", _i, _vp, _i, _i)
apus_gcuda_model_debug_read = _fn("apus_gcuda_model_debug_read", _i, _vp, _cs, _vp, _sz)
apus_gcuda_gspec_keep_logits = _fn("apus_gcuda_gspec_keep_logits", _i, _vp, _i)
apus_gcuda_gspec_counters = _fn("apus_gcuda_gspec_counters", _i, _vp, _vp, _sz)

# ---- the reference's spec-engine names (include/apus_gspec_gcuda.h) --------
# Structs the C host declares (ApusGmtp, ApusGspec, ApusRng) are passed as
# pointers to caller memory; a C host uses them directly (tests/c/).
apus_rng_seed = _fn("apus_rng_seed", None, _vp, _u64)
apus_sample_scratch_size = _fn("apus_sample_scratch_size", _sz, _sz)
apus_gmodel_open = _fn("apus_gmodel_open", _vp, _cs, _cs, _vp, _sz)
apus_gmodel_open2 = _fn("apus_gmodel_open2", _vp, _cs, _cs, _vp, _vp, _sz)
apus_gmodel_close = _fn("apus_gmodel_close", None, _vp)
apus_gmodel_config = _fn("apus_gmodel_config", _vp, _vp)
apus_gmodel_has_mtp = _fn("apus_gmodel_has_mtp", _i, _vp)
apus_gmodel_state_new = _fn("apus_gmodel_state_new", _vp, _vp, _sz)
apus_gmodel_state_free = _fn("apus_gmodel_state_free", None, _vp)
apus_gmodel_pos = _fn("apus_gmodel_pos", _sz, _vp)
apus_gmodel_state_cap = _fn("apus_gmodel_state_cap", _sz, _vp)
apus_gmodel_state_gcuda = _fn("apus_gmodel_state_gcuda", _vp, _vp)
apus_gmtp_bind = _fn("apus_gmtp_bind", _i, _vp, _vp, _vp, _sz)
apus_gmtp_state_new = _fn("apus_gmtp_state_new", _vp, _vp, _sz)
apus_gmtp_state_free = _fn("apus_gmtp_state_free", None, _vp)
apus_gspec_init = _fn("apus_gspec_init", None, _vp, _vp, _vp, _vp, _vp, _i, C.c_float, C.c_float, _vp, _vp)
apus_gspec_free = _fn("apus_gspec_free", None, _vp)
apus_gspec_prefill = _fn("apus_gspec_prefill", _i, _vp, _vp, _sz)
apus_gspec_step = _fn("apus_gspec_step", _i, _vp, _vp, _i)


EP_HANDLE_BYTES = 64   # sizeof(cudaIpcMemHandle_t)


def ep_handles_blob(handles, world):
    """Concatenate the ranks' exchange handles in rank order (host side of
    apus_gcuda_model_ep_connect)."""
    if len(handles) != world:
        raise GcudaError(f"ep_connect: {len(handles)} handles for {world} ranks")
    for r, h in enumerate(handles):
        if len(h) != EP_HANDLE_BYTES:
            raise GcudaError(f"ep_connect: rank {r} handle has {len(h)} bytes")
    return b"".join(bytes(h) for h in handles)


def ep_all_gather(group=None):
    """An all_gather(bytes) -> [bytes] over a torch.distributed group (any
    backend): every rank's payload, in rank order."""
    import torch.distributed as dist

    def gather(payload):
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, bytes(payload), group=group)
        return out
    return gather


class GModel:
    """One resident model + sequence on the current CUDA device (the
    reference's ApusGmodel/ApusGmodelState/ApusGmtp/ApusGspec bundle,
    c/gmodel.h:161-320, c/gmtp.h:123-259).  Arrays are numpy (host)."""

    def __init__(self, cfg, has_mtp=True, kv_cap=1024, depth=4, rank=0, world=1):
        import numpy as np
        self.np = np
        enable()
        self.cfg, self.depth, self.rank, self.world = cfg, depth, rank, world
        if world > 1:
            self.h = apus_gcuda_model_new_ep(C.byref(cfg), int(has_mtp), kv_cap, depth, rank, world)
        else:
            self.h = apus_gcuda_model_new(C.byref(cfg), int(has_mtp), kv_cap, depth)
        if not self.h:
            raise GcudaError(f"model_new: {apus_gcuda_last_error().decode(errors='replace')}")

    def load_container(self, path):
        """Upload every tensor this model (this rank) stores from the
        reference's weight container directory `path`."""
        err = C.create_string_buffer(512)
        if apus_gcuda_model_load_container(self.h, os.fsencode(path), err, 512) != 0:
            raise GcudaError(err.value.decode(errors="replace"))

    def ep_handle(self):
        """This rank's 64-byte exchange-region handle."""
        buf = C.create_string_buffer(EP_HANDLE_BYTES)
        check(apus_gcuda_model_ep_handle(self.h, buf), "ep_handle")
        return buf.raw

    def ep_connect(self, handles):
        """Open every rank's exchange region; `handles` lists the ranks'
        64-byte handles in rank order."""
        blob = ep_handles_blob(handles, self.world)
        buf = C.create_string_buffer(blob, len(blob))
        check(apus_gcuda_model_ep_connect(self.h, buf), "ep_connect")

    def ep_bootstrap(self, all_gather):
        """Exchange handles with `all_gather(bytes) -> [bytes per rank]` (for
        example ep_all_gather over a torch.distributed group), then connect."""
        self.ep_connect(all_gather(self.ep_handle()))

    def close(self):
        if self.h:
            apus_gcuda_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set(self, name, arr):
        """Store one checkpoint tensor; returns False for another
        expert-parallel rank's expert (nothing stored)."""
        arr = self.np.ascontiguousarray(arr)
        rc = apus_gcuda_model_set(self.h, name.encode(), ptr(arr), arr.nbytes)
        if rc == 1:
            return False
        check(rc, f"set {name}")
        return True

    def get(self, name, shape, dtype):
        a = self.np.empty(shape, dtype)
        check(apus_gcuda_model_get(self.h, name.encode(), ptr(a), a.nbytes), f"get {name}")
        return a

    def load(self, weights):
        for k, v in weights.items():
            self.set(k, v)

    def init_random(self, seed):
        check(apus_gcuda_model_init_random(self.h, seed), "init_random")

    def reset(self):
        check(apus_gcuda_model_reset(self.h), "reset")

    def pos(self):
        return apus_gcuda_model_pos(self.h)

    def decode_batch(self, ids, want_h=False):
        np, cfg = self.np, self.cfg
        ids = np.ascontiguousarray(ids, np.int32)
        s = len(ids)
        logits = np.empty((s, cfg.vocab_size), np.uint16)
        h = np.empty((s, cfg.hc_mult * cfg.hidden_size), np.uint16)
        yn = np.empty((s, cfg.hidden_size), np.uint16)
        check(apus_gcuda_decode_batch(self.h, ptr(ids), s, ptr(logits), ptr(h), ptr(yn)), "decode_batch")
        return (logits, h, yn) if want_h else logits

    def prefill(self, ids, want_logits=True):
        """The prompt pass on a fresh sequence: (logits [n][V] or None, yn [n][d])."""
        np, cfg = self.np, self.cfg
        ids = np.ascontiguousarray(ids, np.int32)
        n = len(ids)
        logits = np.empty((n, cfg.vocab_size), np.uint16) if want_logits else None
        yn = np.empty((n, cfg.hidden_size), np.uint16)
        check(apus_gcuda_prefill(self.h, ptr(ids), n, ptr(logits) if want_logits else None, ptr(yn)), "prefill")
        return logits, yn

    def mtp_forward(self, ids, prev_h):
        np, cfg = self.np, self.cfg
        ids = np.ascontiguousarray(ids, np.int32)
        prev_h = np.ascontiguousarray(prev_h, np.uint16)
        s = len(ids)
        logits = np.empty((s, cfg.vocab_size), np.uint16)
        oh = np.empty((s, cfg.hidden_size), np.uint16)
        check(apus_gcuda_mtp_forward(self.h, ptr(ids), ptr(prev_h), s, ptr(logits), ptr(oh)), "mtp_forward")
        return logits, oh

    def spec_prefill(self, ids):
        ids = self.np.ascontiguousarray(ids, self.np.int32)
        check(apus_gcuda_gspec_prefill(self.h, ptr(ids), len(ids)), "gspec_prefill")

    def spec_step(self):
        out = (C.c_int * 16)()
        n = apus_gcuda_gspec_step(self.h, out, 16)
        return list(out[:n])

    def spec_step_async(self):
        check(apus_gcuda_gspec_step_async(self.h), "gspec_step_async")

    def emitted(self, cap=1 << 16):
        out = self.np.empty(cap, self.np.int32)
        n = apus_gcuda_gspec_emitted(self.h, ptr(out), cap)
        if n < 0:
            raise GcudaError(apus_gcuda_last_error().decode(errors="replace"))
        return out[:min(n, cap)].tolist()

    def stats(self):
        o = (C.c_uint64 * 6)()
        rc = apus_gcuda_gspec_stats(self.h, o)
        return dict(zip(("emitted", "batches", "offered", "accepted", "pos", "held"), list(o))), rc

    def force(self, truth, base, p=1.0, seed=0):
        if truth is None:
            check(apus_gcuda_gspec_force(self.h, None, 0, 0, 0.0, 0), "force off")
            return
        t = self.np.ascontiguousarray(truth, self.np.int32)
        check(apus_gcuda_gspec_force(self.h, ptr(t), len(t), base, float(p), seed), "force")

    def greedy(self, ids, n_gen):
        np = self.np
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(n_gen, np.int32)
        check(apus_gcuda_greedy(self.h, ptr(ids), len(ids), n_gen, ptr(out)), "greedy")
        return out.tolist()

    def generate(self, ids, n_gen):
        """Non-speculative decode with the sampling settings (greedy when temp <= 0)."""
        np = self.np
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(n_gen, np.int32)
        check(apus_gcuda_generate(self.h, ptr(ids), len(ids), n_gen, ptr(out)), "generate")
        return out.tolist()

    def sampling(self, temp, top_p=1.0, seed=0):
        """apus_gspec_init's temp / top_p and apus_rng_seed(seed)."""
        check(apus_gcuda_gspec_sampling(self.h, float(temp), float(top_p), int(seed) & ((1 << 64) - 1)), "sampling")

    def rng_state(self):
        s = _u64(0)
        check(apus_gcuda_rng_state(self.h, C.byref(s)), "rng_state")
        return s.value

    def digest(self):
        return apus_gcuda_state_digest(self.h)

    def use_graph(self, on=True):
        check(apus_gcuda_gspec_use_graph(self.h, int(on)), "use_graph")

    def stream(self):
        return apus_gcuda_model_stream(self.h)

    def decode(self, ids):
        """decode_batch without copying anything back (state only)."""
        ids = self.np.ascontiguousarray(ids, self.np.int32)
        check(apus_gcuda_decode_batch(self.h, ptr(ids), len(ids), None, None, None), "decode_batch")

    def debug_stop(self, layer, stage):
        """Stop the next forwards after (layer, stage); layer -1 clears it."""
        check(apus_gcuda_model_debug_stop(self.h, int(layer), int(stage)), "debug_stop")

    def debug_read(self, name, shape, dtype):
        a = self.np.empty(shape, dtype)
        check(apus_gcuda_model_debug_read(self.h, name.encode(), ptr(a), a.nbytes), f"debug_read {name}")
        return a

    def keep_logits(self, on=True):
        check(apus_gcuda_gspec_keep_logits(self.h, int(on)), "keep_logits")

    def kda_state(self, layer):
        """Committed KDA state of `layer`: (conv [3*qkv][K-1] BF16, rec [H][D][D] f32)."""
        c, np = self.cfg, self.np
        qkv = c.linear_num_heads * c.linear_head_dim
        conv = self.debug_read(f"kda_conv.{layer}", (3 * qkv, c.linear_conv_kernel_dim - 1), np.uint16)
        rec = self.debug_read(f"kda_rec.{layer}", (c.linear_num_heads, c.linear_head_dim, c.linear_head_dim),
                              np.float32)
        return conv, rec

    def dsa_state(self, layer, n):
        """The n committed cache rows of DSA `layer` (num_hidden_layers: the MTP
        block): k [AH][n][qd], v [AH][n][vd], ik / ig [n][ID] BF16."""
        c, np = self.cfg, self.np
        AH, ID = c.num_attention_heads, c.index_head_dim
        return (self.debug_read(f"dsa_k.{layer}", (AH, n, c.qk_nope_head_dim), np.uint16),
                self.debug_read(f"dsa_v.{layer}", (AH, n, c.v_head_dim), np.uint16),
                self.debug_read(f"dsa_ik.{layer}", (n, ID), np.uint16),
                self.debug_read(f"dsa_ig.{layer}", (n, ID), np.uint16))

    def counters(self):
        o = (C.c_uint64 * 5)()
        check(apus_gcuda_model_counters(self.h, o, 5), "counters")
        return dict(zip(("moe_problems", "main_forwards", "mtp_forwards", "graph_kernels", "ctl_bytes"),
                        list(o)))


def ep_owns(kw, rank, world):
    """synth.ep_owns (the split apus_gcuda_model_set applies), raising
    GcudaError for a split that does not divide the experts."""
    try:
        return synth.ep_owns(kw, rank, world)
    except ValueError as e:
        raise GcudaError(str(e)) from None


tensor_specs = synth.tensor_specs


def config_load(path):
    """ApusGcudaConfig from a config.json in either layout the reference
    reads (apus_gcuda_config_load)."""
    cfg = GcudaConfig()
    err = C.create_string_buffer(512)
    if apus_gcuda_config_load(os.fsencode(path), C.byref(cfg), err, 512) != 0:
        raise GcudaError(err.value.decode(errors="replace"))
    return cfg


def config_dict(cfg):
    """The fields of an ApusGcudaConfig as the keyword dict make_config takes."""
    kw = {name: getattr(cfg, name) for name, _ in _CFG_FIELDS if name not in ("layer_is_dsa", "mlp_is_sparse")}
    L = cfg.num_hidden_layers
    kw["layer_is_dsa"] = [cfg.layer_is_dsa[i] for i in range(L)]
    kw["mlp_is_sparse"] = [cfg.mlp_is_sparse[i] for i in range(L)]
    return kw


def container_check(path, cfg, has_mtp=True):
    """Number of tensors the model of cfg needs, all found in the container
    with their dtype and size; raises on the first problem."""
    err = C.create_string_buffer(512)
    n = apus_gcuda_container_check(os.fsencode(path), C.byref(cfg), int(has_mtp), err, 512)
    if n < 0:
        raise GcudaError(err.value.decode(errors="replace"))
    return n


def container_read(path, name):
    """Raw bytes of one container tensor."""
    err = C.create_string_buffer(512)
    n = apus_gcuda_container_read(os.fsencode(path), name.encode(), None, 0, err, 512)
    if n < 0:
        raise GcudaError(err.value.decode(errors="replace"))
    buf = C.create_string_buffer(max(n, 1))
    if apus_gcuda_container_read(os.fsencode(path), name.encode(), buf, n, err, 512) != n:
        raise GcudaError(err.value.decode(errors="replace"))
    return buf.raw[:n]
