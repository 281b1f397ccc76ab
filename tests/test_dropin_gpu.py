"""The drop-in boundary, exercised from C hosts compiled here with gcc.

  * Linear-leaf hooks: tests/c/hooks_host.c fills the reference engine's own
    hook table (apus_gmetal_hooks, c/backend_gmetal.h:120-128) from
    apus_gcuda_fill_hooks.  The reference engine (compiled from the
    reference's sources, oracle/_ref) then runs its decode batch and its
    speculative loop (apus_gspec_prefill / apus_gspec_step) with every BF16
    GEMM and fused FP8-block linear on the B200.  Its logits stay within the
    linear leaf's tolerance of the pure-CPU run, its token stream equals the
    CPU run's up to a near tie of the CPU logits, and the offload counters
    prove the hooks ran.
  * Spec-engine API: tests/c/spec_loop_host.c is a spec loop in the shape of
    the reference's run_glm (c/apus.c:1016-1077) written against
    include/apus_gspec_gcuda.h (the reference's names and ApusGspec
    counters) and linked with libapus_gcuda.so.  Its tokens are the engine's
    own greedy stream, its counters are consistent, and a draft_override
    that proposes the true tokens gets every draft accepted.
"""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

import oracle as O
from container import write_container
from modelgen import gen_weights, tiny_config

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "apus-glm5.3-flash_b200")
REF_DIR = os.path.join(ROOT, "oracle", "_ref")
PROMPT = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]


def build(src, out, with_ref):
    libs = ["-L", PKG, "-lapus_gcuda", f"-Wl,-rpath,{PKG}"]
    if with_ref:
        libs = ["-L", REF_DIR, "-lapus_ref", f"-Wl,-rpath,{REF_DIR}"] + libs
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-Werror", "-shared", "-fPIC", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", src), "-o", str(out)] + libs
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return C.CDLL(str(out))


def f32(a):
    return O.f32_of(np.ascontiguousarray(a, np.uint16)).astype(np.float64)


def test_reference_engine_with_cuda_leaf(gcuda, tmp_path):
    if O.REF is None:
        pytest.skip("the reference engine (oracle/_ref) is not built")
    host = build("hooks_host.c", tmp_path / "hooks_host.so", with_ref=True)
    host.host_attach.argtypes = [C.c_char_p, C.c_size_t]
    # every expert selected and the indexer's selection never binding: no
    # discrete decision (a top-k routing or pool pick) can flip on the leaf's
    # last-bit differences, so the logits compare at the leaf's tolerance
    kw = tiny_config(n_routed_experts=4, num_experts_per_tok=4, index_topk=256)
    W = gen_weights(kw, seed=20261204)
    ref = O.Model(O.make_config(**kw), W, True, "ref")
    depth, steps, cap = 4, 10, 256
    ids = np.array(PROMPT, np.int32)

    def run():
        st = ref.state(cap)
        lg = ref.decode_batch(st, ids[:8])
        O.REF.ref_state_free(st)
        st = ref.state(cap)
        sp = O.REF.ref_spec_new(ref.h, st, cap, depth)
        assert O.REF.ref_spec_prefill(sp, O.p(ids), len(ids)) == 0
        buf = (C.c_int * (depth + 1))()
        toks = []
        for _ in range(steps):
            n = O.REF.ref_spec_step(sp, buf, depth + 1)
            assert n > 0
            toks += list(buf[:n])
        O.REF.ref_spec_free(sp)
        O.REF.ref_state_free(st)
        return lg, toks

    lg_cpu, toks_cpu = run()
    c0 = (gcuda.apus_gcuda_dispatches(), gcuda.apus_gcuda_offload_bf16(), gcuda.apus_gcuda_offload_fp8blk())
    err = C.create_string_buffer(256)
    assert host.host_attach(err, 256) == 0, err.value
    try:
        assert host.host_attached() == 1
        lg_gpu, toks_gpu = run()
    finally:
        host.host_detach()
    c1 = (gcuda.apus_gcuda_dispatches(), gcuda.apus_gcuda_offload_bf16(), gcuda.apus_gcuda_offload_fp8blk())
    assert c1[0] > c0[0] and c1[1] > c0[1] and c1[2] > c0[2], (c0, c1)
    # the linear leaf's tolerance, compounded through the tiny model as in
    # the engine's own tiny-model tests
    for r in range(len(lg_cpu)):
        a, b = f32(lg_gpu[r]), f32(lg_cpu[r])
        cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
        assert cos >= 0.999 and np.abs(a - b).max() <= 0.05 * np.abs(b).max(), (r, cos)
    if toks_gpu != toks_cpu:
        j = next(i for i in range(min(len(toks_gpu), len(toks_cpu))) if toks_gpu[i] != toks_cpu[i])
        st = ref.state(cap)
        ctx = np.array(PROMPT + toks_cpu[:j], np.int32)
        for a in range(0, len(ctx), 8):
            lo = ref.decode_batch(st, ctx[a:a + 8])
        O.REF.ref_state_free(st)
        v = np.sort(f32(lo[-1]))
        assert v[-1] - v[-2] < 0.05 * np.abs(v).max(), f"streams differ at {j} away from a near tie"


@pytest.fixture(scope="module")
def tiny_container(tmp_path_factory):
    import synth
    kw = tiny_config()
    W = gen_weights(kw, seed=20261201)
    d = tmp_path_factory.mktemp("container")
    write_container(str(d), kw, W, synth.tensor_specs(kw))
    return kw, W, str(d)


def spec_loop(host, path, ids, depth, max_tokens, cap, force=None):
    host.spec_loop.restype = C.c_int
    host.spec_loop.argtypes = [C.c_char_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p,
                               C.c_int, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.zeros(max_tokens, np.int32)
    stats = np.zeros(8, np.uint64)
    err = C.create_string_buffer(512)
    fa = np.ascontiguousarray(force, np.int32) if force is not None else None
    n = host.spec_loop(path.encode(), ids.ctypes.data, len(ids), depth, max_tokens, cap,
                       fa.ctypes.data if fa is not None else None, len(fa) if fa is not None else 0,
                       out.ctypes.data, stats.ctypes.data, err, 512)
    assert n >= 0, err.value
    keys = ("emitted", "batches", "refeed_tokens", "accepted", "offered", "d1_hits", "d1_offered", "pos")
    return out[:n].tolist(), dict(zip(keys, (int(x) for x in stats)))


def test_spec_loop_host_on_the_gspec_api(gcuda, tiny_container, tmp_path):
    kw, W, path = tiny_container
    host = build("spec_loop_host.c", tmp_path / "spec_loop_host.so", with_ref=False)
    depth, n_tok, cap = 4, 30, 256
    toks, s = spec_loop(host, path, PROMPT, depth, n_tok, cap)
    ref = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=cap, depth=depth)
    ref.load(W)
    truth = ref.greedy(PROMPT, 80)
    ref.close()
    assert toks == truth[:len(toks)] and len(toks) == n_tok
    assert s["emitted"] >= n_tok and s["batches"] >= 1 and s["pos"] == len(PROMPT) + s["emitted"]
    assert s["accepted"] <= s["offered"] and s["d1_offered"] == s["batches"]
    # a partial reject re-feeds the drafts it checked (matched + 1 of them);
    # a full accept checks depth - 1 and re-feeds none
    assert s["refeed_tokens"] <= s["offered"] and (s["offered"] - s["refeed_tokens"]) % (depth - 1) == 0
    # a draft_override proposing the true tokens: every draft accepted,
    # depth tokens a step, no re-fed tokens
    toks_f, sf = spec_loop(host, path, PROMPT, depth, n_tok, cap, force=truth)
    assert toks_f == truth[:len(toks_f)]
    assert sf["accepted"] == sf["offered"] > 0 and sf["refeed_tokens"] == 0
    assert sf["emitted"] == depth * sf["batches"]
    assert sf["d1_hits"] == sf["d1_offered"]
