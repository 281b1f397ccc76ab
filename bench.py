#!/usr/bin/env python3
"""bench.py — throughput of the apus B200 engine on the BASELINE workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 0|1|2]

Prints ONE JSON line (rank 0).  Workloads:
  0  FP8-E4M3 128x128 block-dequant GEMV, M=4 rows, N=K=4096.  A step is one
     linear call; weights rotate over a set of buffers larger than L2.
  1  one MoE verify layer (4 rows, hidden 4096, 288 experts top-8 + shared,
     inter 1024, FP8 experts).  A step is one layer call.
  2  the scaled glm5_next stack + MTP speculative decode (the headline).
With --impl reference the reference's own CPU engine (oracle/_ref, compiled
from the reference sources) runs a bounded sample of the same workload on
the host cores.
"""
import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "apus-glm5.3-flash_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
from synth import c2_config, c2_weights, ep_owns  # noqa: E402  (pure Python: loads no CUDA library)

METRIC = "accepted tok/s (MTP depth 3, 1 seq) at 1/2/4/8 B200; FP8 GEMV % HBM peak"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a while to start: wait (bounded) for its first
            # sample so that a short timed region is still covered
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.05)
            self.lines.clear()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return ws, rank, local


def max_over_ranks(v, ws):
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


# --------------------------------------------------------------------------
# config 0: FP8 GEMV
C0 = dict(M=4, N=4096, K=4096)


def c0_inputs(seed=0):
    import numpy as np
    import torch
    M, N, K = C0["M"], C0["N"], C0["K"]
    g = torch.Generator(device="cpu").manual_seed(seed)
    v = torch.clamp(torch.randn((N, K), generator=g) * 64, -448, 448)
    codes = v.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()
    lo, hi = np.log(1e-4), np.log(1e-2)
    s = torch.exp(lo + (hi - lo) * torch.rand((N // 128, K // 128), generator=g)).numpy().astype(np.float32)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    return codes, s, x


def c0_algo_bytes():
    M, N, K = C0["M"], C0["N"], C0["K"]
    return N * K + (N // 128) * (K // 128) * 4 + M * K * 2 + M * N * 2


def bench_c0(args, ws, rank):
    import numpy as np
    import torch
    import apus_gcuda as G
    G.enable()
    M, N, K = C0["M"], C0["N"], C0["K"]
    codes, s, x = c0_inputs(0)
    nbuf = 16  # 16 x 16.8 MB = 270 MB > 2x L2: every timed call streams from HBM
    dW = [torch.from_numpy(codes).cuda() for _ in range(nbuf)]
    dS = torch.from_numpy(s).cuda()
    dx = torch.from_numpy(x.view(np.int16)).cuda()
    dy = torch.empty((M, N), dtype=torch.int16, device="cuda")
    st = torch.cuda.Stream()
    sp = G.C.c_void_p(st.cuda_stream)
    G.apus_gcuda_set_pdl(1)   # consecutive linears overlap their weight streams

    def step(i):
        G.check(G.apus_gcuda_fp8blk_linear_dev(G.ptr(dW[i % nbuf]), G.ptr(dS), G.ptr(dx), G.ptr(dy),
                                               M, N, K, sp), "linear")

    with torch.cuda.stream(st):
        for i in range(args.warmup):
            step(i)
    st.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        time.sleep(0.3)
        e0.record(st)
        for i in range(args.steps):
            step(i)
        e1.record(st)
        st.synchronize()
    ms = e0.elapsed_time(e1)
    barrier(ws)
    ms = max_over_ranks(ms, ws)
    per = ms / args.steps
    hbm, _, src = peaks()
    algo = c0_algo_bytes()
    gbs = algo / (per * 1e-3) / 1e9
    if args.quick:
        return {"metric": METRIC, "value": round(gbs * ws, 2), "ms_per_step": per, "n_gpus": ws,
                "roofline": {"achieved": round(gbs, 1), "peak": hbm, "frac": round(gbs / hbm, 4)}}
    # e2e: the reference-facing host-pointer hook with resident weights
    for i in range(nbuf):
        G.check(G.apus_gcuda_register_region(G.ptr(_hold(codes, i)), codes.nbytes), "register")
    G.check(G.apus_gcuda_register_region(G.ptr(s), s.nbytes), "register scales")
    yh = np.empty((M, N), np.uint16)
    for i in range(args.warmup):
        G.apus_gcuda_fp8blk_linear(G.ptr(_hold(codes, i % nbuf)), G.ptr(s), G.ptr(x), G.ptr(yh), M, N, K)
    t0 = time.perf_counter()
    for i in range(args.steps):
        if G.apus_gcuda_fp8blk_linear(G.ptr(_hold(codes, i % nbuf)), G.ptr(s), G.ptr(x), G.ptr(yh), M, N, K):
            raise RuntimeError(G.apus_gcuda_last_error())
    e2e_s = (time.perf_counter() - t0) / args.steps
    e2e_s = max_over_ranks(e2e_s, ws)
    out = {
        "metric": METRIC, "value": round(gbs * ws, 2), "unit": "GB/s (FP8 GEMV algorithmic bytes, config 0)",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp8e4m3->bf16, f32 acc",
        "data": "synthetic (BASELINE config 0 distributions, seed 0)",
        "config": {"workload": "config0: FP8 128x128 block-dequant GEMV M=4 N=4096 K=4096",
                   "l2": "16 rotating weight buffers (270 MB > L2)", "parallelism": f"replicas x{ws}"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "traffic": None, "peak_source": src,
                     "algo_bytes_per_launch": algo},
        "e2e": {"value": round(algo / e2e_s / 1e9 * ws, 3), "unit": "GB/s through apus_gcuda_fp8blk_linear (host x/y)",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    return out


def _graph_us(torch, st, body, n_calls, replays=5):
    """Device time of one call of `body` (n_calls calls on stream st), the
    calls captured into a CUDA graph and replayed (as the engine runs its
    kernels: no host launch cost between them), CUDA events on st."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        body()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        g.replay()
        e0.record(st)
        for _ in range(replays):
            g.replay()
        e1.record(st)
    st.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (replays * n_calls)
    del g
    return us


def fp8_gemv_leg(reps=200, warmup=10):
    """The metric's second half, FP8 GEMV % of HBM peak.
      * BASELINE config 0 (M=4 rows, 4096x4096 E4M3 with 128x128 block
        scales): `reps` back-to-back programmatic launches over 16 rotating
        weight copies (270 MB > L2, so every launch streams its weights from
        HBM), captured in a CUDA graph and replayed, CUDA events on the
        launching stream.  A 16.8 MB launch is bounded by its fixed latency
        (launch, tensor-map fetch, first copy) as much as by the bandwidth.
      * the shape the decode step streams most FP8 bytes through: one MoE
        layer call of BASELINE config 1 (4 rows, 288 experts top-8 + shared,
        inter 1024), the router and grouped expert GEMVs over the realised
        union (~30 experts, ~400 MB), over 16 rotating input batches, graph
        replayed; algorithmic bytes = the union's expert bytes + router."""
    import numpy as np
    import torch
    import apus_gcuda as G
    M, N, K = C0["M"], C0["N"], C0["K"]
    codes, s, x = c0_inputs(0)
    nbuf = 16
    dW = [torch.from_numpy(codes).cuda() for _ in range(nbuf)]
    dS = torch.from_numpy(s).cuda()
    dx = torch.from_numpy(x.view(np.int16)).cuda()
    dy = torch.empty((M, N), dtype=torch.int16, device="cuda")
    st = torch.cuda.Stream()
    sp = G.C.c_void_p(st.cuda_stream)
    G.apus_gcuda_set_pdl(1)

    def step(i):
        G.check(G.apus_gcuda_fp8blk_linear_dev(G.ptr(dW[i % nbuf]), G.ptr(dS), G.ptr(dx), G.ptr(dy),
                                               M, N, K, sp), "linear")
    for i in range(warmup):
        step(i)
    st.synchronize()
    us = _graph_us(torch, st, lambda: [step(i) for i in range(reps)], reps)
    G.apus_gcuda_set_pdl(0)
    hbm, _, src = peaks()
    algo = c0_algo_bytes()
    gbs = algo / us / 1e3
    del dW
    torch.cuda.empty_cache()
    out = {"workload": "config0: FP8 128x128 block-dequant GEMV, M=4, N=K=4096", "kernel": "k_gemv_tma<true>",
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(gbs / hbm, 4), "peak_source": src, "algo_bytes_per_launch": algo,
                        "avg_launch_us": round(us, 3), "launches": reps,
                        "timing": "graph-replayed back-to-back launches, CUDA events",
                        "l2": "16 rotating weight copies (270 MB > L2)"}}
    # the same kernel on a matrix large enough that its fixed latency is small
    # beside the stream, K within one k-range (no split-K pass): 4 rows x
    # 65536 x 4096 E4M3 (268 MB), 2 rotating copies
    NO, NK = 65536, 4096
    wl = [torch.randint(0, 120, (NO, NK), dtype=torch.uint8, device="cuda") for _ in range(2)]
    sl = torch.full((NO // 128, NK // 128), 1e-3, device="cuda")
    xl = torch.randn(M, NK, device="cuda").to(torch.bfloat16)
    yl = torch.empty(M, NO, dtype=torch.bfloat16, device="cuda")
    G.apus_gcuda_set_pdl(1)

    def big(i):
        G.check(G.apus_gcuda_fp8blk_linear_dev(G.ptr(wl[i % 2]), G.ptr(sl), G.ptr(xl), G.ptr(yl), M, NO, NK, sp),
                "linear")
    for i in range(4):
        big(i)
    st.synchronize()
    nb = 20
    usl = _graph_us(torch, st, lambda: [big(i) for i in range(nb)], nb)
    G.apus_gcuda_set_pdl(0)
    al = NO * NK + sl.numel() * 4 + M * (NK + NO) * 2
    out["large_matrix"] = {"workload": "FP8 128x128 block-dequant GEMV, M=4, N=65536, K=4096 (268 MB)",
                           "achieved": round(al / usl / 1e3, 1), "peak": hbm, "unit": "GB/s",
                           "frac": round(al / usl / 1e3 / hbm, 4), "avg_launch_us": round(usl, 2),
                           "timing": "graph-replayed back-to-back launches over 2 copies (537 MB > L2)"}
    del wl
    torch.cuda.empty_cache()
    # one MoE layer (config 1): the grouped FP8 GEMVs at the step's shapes
    R, d = C1["R"], C1["dim"]
    h = G.apus_gcuda_moe_new(C1["E"], C1["topk"], d, C1["inter"], 2.5, 10.0, R)
    assert h, G.apus_gcuda_last_error()
    G.check(G.apus_gcuda_moe_init_random(h, 1), "init")
    xs = c1_inputs(1)
    mx = torch.from_numpy(xs.view(np.int16)).cuda()
    my = torch.empty((R, d), dtype=torch.int16, device="cuda")
    algo1 = []
    for i in range(C1["nx"]):
        G.check(G.apus_gcuda_moe_forward_dev(h, G.ptr(mx[i]), R, G.ptr(my), None, sp), "moe")
        st.synchronize()
        algo1.append(G.apus_gcuda_moe_last_bytes(h) + R * d * 4)
    n1 = C1["nx"] * 4
    us1 = _graph_us(torch, st, lambda: [G.check(G.apus_gcuda_moe_forward_dev(
        h, G.ptr(mx[i % C1["nx"]]), R, G.ptr(my), None, sp), "moe") for i in range(n1)], n1)
    G.apus_gcuda_moe_free(h)
    a1 = float(np.mean(algo1))
    out["moe_layer"] = {"workload": "config1: one MoE layer call, 4 rows, 288 experts top-8 + shared, inter 1024",
                        "kernels": "router GEMV + k_moe_route + grouped k_gemv_tma<true> gate|up and down + combine",
                        "achieved": round(a1 / us1 / 1e3, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(a1 / us1 / 1e3 / hbm, 4), "us_per_call": round(us1, 2),
                        "algo_bytes_per_call": round(a1), "timing": "graph-replayed calls, CUDA events"}
    return out


_HOLD = {}


def _hold(codes, i):
    """Distinct host copies of the weights (one registered region each)."""
    if i not in _HOLD:
        _HOLD[i] = codes.copy()
    return _HOLD[i]


def cpu_c0(budget_s=10.0):
    """Reference CPU fp8_linear (c/gdsa.h:525-534 = apus_fp8blk_dequant_mt +
    apus_bf16_gemm_mt) on the host cores, bounded to ~budget_s."""
    import numpy as np
    import oracle as O
    if O.REF is None:
        return None
    M, N, K = C0["M"], C0["N"], C0["K"]
    codes, s, x = c0_inputs(0)
    wb = np.empty((N, K), np.uint16)
    xf = np.empty((M * K,), np.float32)
    y = np.empty((M, N), np.uint16)
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        O.REF.apus_fp8blk_dequant_mt(O.p(codes), O.p(s), O.p(wb), N, K)
        O.REF.apus_bf16_gemm_mt(O.p(wb), O.p(x), O.p(xf), O.p(y), M, N, K)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(c0_algo_bytes() / dt / 1e9, 3), "unit": "GB/s", "cores": O.REF.apus_ref_threads(),
            "kind": "reference", "sample": f"{n} fp8_linear calls (dequant_mt + bf16_gemm_mt), {dt * 1e3:.2f} ms each"}


# --------------------------------------------------------------------------
# config 1: one MoE verify layer
C1 = dict(R=4, E=288, topk=8, dim=4096, inter=1024, nx=16)


def c1_inputs(seed=1):
    import numpy as np
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    xs = torch.randn((C1["nx"], C1["R"], C1["dim"]), generator=g).to(torch.bfloat16)
    return xs.view(torch.int16).numpy().view(np.uint16).copy()


def bench_c1(args, ws, rank):
    """A step = one MoE layer call on 4 rows (router + top-8 of 288 + shared,
    FP8 experts resident in HBM).  Activations rotate over 16 seeded batches
    so the routed union changes step to step; the union (~30 experts, ~380 MB)
    exceeds L2, so every call streams its experts from HBM."""
    import numpy as np
    import torch
    import apus_gcuda as G
    G.enable()
    R, d = C1["R"], C1["dim"]
    h = G.apus_gcuda_moe_new(C1["E"], C1["topk"], d, C1["inter"], 2.5, 10.0, R)
    assert h, G.apus_gcuda_last_error()
    G.check(G.apus_gcuda_moe_init_random(h, 1), "init")
    xs = c1_inputs(1)
    dx = torch.from_numpy(xs.view(np.int16)).cuda()
    dy = torch.empty((R, d), dtype=torch.int16, device="cuda")
    st = torch.cuda.Stream()
    sp = G.C.c_void_p(st.cuda_stream)
    # algorithmic bytes per call, from each input batch's realised routing
    algo = []
    for i in range(C1["nx"]):
        G.check(G.apus_gcuda_moe_forward_dev(h, G.ptr(dx[i]), R, G.ptr(dy), None, sp), "moe")
        st.synchronize()
        algo.append(G.apus_gcuda_moe_last_bytes(h) + R * d * 4)
    algo_mean = float(np.mean(algo))

    def step(i):
        G.check(G.apus_gcuda_moe_forward_dev(h, G.ptr(dx[i % C1["nx"]]), R, G.ptr(dy), None, sp), "moe")

    with torch.cuda.stream(st):
        for i in range(args.warmup):
            step(i)
    st.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        time.sleep(0.3)
        e0.record(st)
        for i in range(args.steps):
            step(i)
        e1.record(st)
        st.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), ws)
    per = ms / args.steps
    hbm, _, src = peaks()
    gbs = algo_mean / (per * 1e-3) / 1e9
    out = {"metric": METRIC, "value": round(1e3 / per * ws, 2), "unit": "MoE layer calls/s (config 1)",
           "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp8e4m3->bf16, f32 acc",
           "data": "synthetic (BASELINE config 1 distributions, seed 1)",
           "config": {"workload": "config1: MoE verify layer, 4 rows, 288 experts top-8 + shared, hidden 4096, "
                                  "inter 1024", "l2": "routed union ~380 MB > L2; 16 rotating input batches",
                      "parallelism": f"replicas x{ws}"},
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(gbs / hbm, 4), "traffic": None, "peak_source": src,
                        "algo_bytes_per_launch": algo_mean},
           "gpu_launches": 5 * args.steps, "clocks": clk.summary()}
    if args.quick:
        return out
    # e2e: the host-pointer apus_gmoe_forward2 drop-in
    yh = np.empty((R, d), np.uint16)
    for i in range(args.warmup):
        G.check(G.apus_gcuda_moe_forward2(h, G.ptr(xs[i % C1["nx"]]), R, G.ptr(yh), None), "moe2")
    t0 = time.perf_counter()
    for i in range(args.steps):
        G.check(G.apus_gcuda_moe_forward2(h, G.ptr(xs[i % C1["nx"]]), R, G.ptr(yh), None), "moe2")
    e2e = max_over_ranks((time.perf_counter() - t0) / args.steps, ws)
    out["e2e"] = {"value": round(ws / e2e, 2), "unit": "MoE layer calls/s through apus_gcuda_moe_forward2",
                  "h2d_bytes_per_step": R * d * 2, "d2h_bytes_per_step": R * d * 2}
    out["_moe"] = h
    return out


def cpu_c1(h, budget_s=10.0):
    """The reference apus_gmoe_forward2 (c/gmoe.h:265-337) on the same weights:
    the experts routed by the sample batches are read back from HBM and
    dequantized to BF16 with the reference's apus_fp8blk_dequant_mt, as its
    engine does at load (c/gmodel.h:1003-1073; not timed)."""
    import ctypes as C
    import numpy as np
    import apus_gcuda as G
    import oracle as O
    if O.REF is None:
        return None
    R, d, E, inter, K = C1["R"], C1["dim"], C1["E"], C1["inter"], C1["topk"]
    O._decl(O.REF, "ref_moe_forward", O._i, O._i, O._i, O._sz, O._sz, O._f, O._f, O._vp, O._vp, O._vp, O._vp,
            O._vp, O._vp, O._vp, O._vp, O._vp, O._sz, O._vp)
    xs = c1_inputs(1)
    nb = 2
    used = set()
    idx = np.zeros((R, K), np.int32)
    for i in range(nb):
        y = np.empty((R, d), np.uint16)
        G.check(G.apus_gcuda_moe_forward2(h, G.ptr(xs[i]), R, G.ptr(y), None), "moe2")
        G.check(G.apus_gcuda_moe_last_routing(h, R, O.p(idx), None), "routing")
        used |= set(idx.ravel().tolist())

    def get(name, shape, dt):
        a = np.empty(shape, dt)
        G.check(G.apus_gcuda_moe_get(h, name.encode(), O.p(a), a.nbytes), name)
        return a

    def deq(name, O_, K_):
        c = get(name + ".weight", (O_, K_), np.uint8)
        s = get(name + ".weight_scale_inv", ((O_ + 127) // 128, (K_ + 127) // 128), np.float32)
        out = np.empty((O_, K_), np.uint16)
        O.REF.apus_fp8blk_dequant_mt(O.p(c), O.p(s), O.p(out), O_, K_)
        return out

    gate_w = get("mlp.gate.weight", (E, d), np.uint16)
    bias = get("mlp.gate.e_score_correction_bias", (E,), np.float32)
    keep = []
    PP = C.c_void_p * E
    eg, eu, ed = PP(), PP(), PP()
    for e in sorted(used):
        for arr, p, shp in ((eg, "gate", (inter, d)), (eu, "up", (inter, d)), (ed, "down", (d, inter))):
            a = deq(f"mlp.experts.{e}.{p}_proj", *shp)
            keep.append(a)
            arr[e] = a.ctypes.data
    sg = deq("mlp.shared_experts.gate_proj", inter, d)
    su = deq("mlp.shared_experts.up_proj", inter, d)
    sd = deq("mlp.shared_experts.down_proj", d, inter)
    out = np.empty((R, d), np.uint16)
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or n < 1:
        O.REF.ref_moe_forward(E, K, d, inter, 2.5, 10.0, O.p(gate_w), O.p(bias), eg, eu, ed, O.p(sg), O.p(su),
                              O.p(sd), O.p(xs[n % nb]), R, O.p(out))
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(1.0 / dt, 3), "unit": "MoE layer calls/s", "cores": O.REF.apus_ref_threads(),
            "kind": "reference",
            "sample": f"{n} apus_gmoe_forward2 calls (4 rows, 288 experts top-8 + shared, experts pre-dequantized "
                      f"to BF16 as the reference engine holds them), {dt * 1e3:.1f} ms each"}


# --------------------------------------------------------------------------
# config 2: the scaled glm5_next stack + MTP speculative decode (headline)
C2 = dict(prompt=512, depth=4, seed=2)   # BASELINE "depth 3" = 4 verify rows (reference APUS_SPEC_K 4)


def c2_workload(temp=0.0, top_p=1.0, seed=0):
    return ("config2: scaled glm5_next (4 layers: 3 KDA 32x128 + 1 DSA, MoE 288 top-8 inter 1024, vocab 154880)"
            " + 1 NextN MTP layer, " + (f"sampled spec decode (temp {temp}, top_p {top_p}, seed {seed})"
                                       if temp > 0 else "greedy spec decode"))


def c2_prompt(kw, seed):
    import numpy as np
    return np.random.default_rng(seed).integers(0, kw["vocab_size"], C2["prompt"]).astype(np.int32)


def c2_algo_bytes(kw, depth, n_ctx, moe_problems, world=1):
    """Algorithmic HBM bytes of one speculative step: every weight byte the
    step's forwards must read once (main forward over `depth` rows, the MTP
    replay and depth-1 chain forwards; the replay and the verify rows share
    one pass over the lm_head when 2*depth <= 8), the realised MoE expert union
    (`moe_problems` expert GEMV pairs, shared expert included, counted on the
    device), the KDA state read + final write, the DSA K/V and pool-key rows
    visible at context n_ctx, and the new cache rows.  Checkpoint copies and
    L2 reuse are not counted.  Expert-parallel ranks (world > 1) read their
    vocabulary slice of the lm_head and count their own expert problems."""
    d, V, hc, L = kw["hidden_size"], kw["vocab_size"], kw["hc_mult"], kw["num_hidden_layers"]
    H, D, K = kw["linear_num_heads"], kw["linear_head_dim"], kw["linear_conv_kernel_dim"]
    qkv, mix = H * D, (2 + hc) * hc
    AH, qd, vd = kw["num_attention_heads"], kw["qk_nope_head_dim"], kw["v_head_dim"]
    ql, kl, IH, ID, kp = (kw["q_lora_rank"], kw["kv_lora_rank"], kw["index_n_heads"], kw["index_head_dim"],
                          kw["index_kpool"])
    E, inter = kw["n_routed_experts"], kw["moe_intermediate_size"]
    cb = lambda n: (n + 127) // 128
    fp8 = lambda O_, K_: O_ * K_ + cb(O_) * cb(K_) * 4
    kda = (3 * qkv + 2 * D + H) * d * 2 + 2 * qkv * D * 2 + 3 * qkv * K * 2 + d * qkv * 2 + 2 * H * D * D * 4
    dsa_w = (fp8(ql + kl, d) + fp8(AH * qd, ql) + AH * (qd + vd) * kl * 2 + fp8(d, AH * vd) + IH * ID * ql * 2
             + (2 * ID + IH) * d * 2)

    def dsa(rows, n):
        return dsa_w + n * AH * (qd + vd) * 2 + (n // kp) * ID * 2 + rows * (AH * (qd + vd) + 2 * ID) * 2

    router = E * d * 2 + E * 4
    expert = fp8(2 * inter, d) + fp8(d, inter)
    # dense-MLP layers (the first first_k_dense_replace): one "problem" of
    # the device counter each per main forward, at the dense width, no router
    dense_l = [l for l in range(L) if not kw["mlp_is_sparse"][l]]
    dn = kw["intermediate_size"]
    dense = len(dense_l) * (fp8(2 * dn, d) + fp8(d, dn))
    hcb = 2 * mix * hc * d * 2
    main = sum(hcb + (dsa(depth, n_ctx) if kw["layer_is_dsa"][l] else kda)
               + (router if kw["mlp_is_sparse"][l] else 0) for l in range(L)) + dense
    head = -(-V // world) * d * 2
    main += head
    mtp_fwd = lambda rows, n: 2 * d * d * 2 + dsa(rows, n) + router + head
    mtp = mtp_fwd(depth, n_ctx) + sum(mtp_fwd(1, n_ctx + i) for i in range(depth - 1))
    if 2 * depth <= 8:      # the replay rows share the verify rows' pass over the head
        mtp -= head
    n_moe_calls = L + 1 + (depth - 1)
    return main + mtp + (moe_problems - len(dense_l)) * expert, n_moe_calls


def profile_value(fname, key):
    """A number recorded in a committed ncu summary under profiles/ (a line
    `key: value`), or None."""
    path = os.path.join(ROOT, "profiles", fname)
    try:
        for line in open(path):
            if line.strip().startswith(key + ":"):
                return float(line.split(":", 1)[1].split()[0].replace(",", ""))
    except OSError:
        pass
    return None


def lm_head_gemv_time(kw, rows, world=1, reps=20):
    """Average device time of the dominant kernel of the step, the lm_head
    GEMV with the fused greedy pick (BF16 [vocab][hidden], `rows` rows), timed
    with CUDA events on its stream over `reps` back-to-back launches (the
    matrix exceeds L2, so every launch streams it from HBM).  Expert-parallel
    ranks time their vocabulary slice."""
    import torch
    import apus_gcuda as G
    V, d = -(-kw["vocab_size"] // world), kw["hidden_size"]
    w = (torch.randn(V, d, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(rows, d, device="cuda").to(torch.bfloat16)
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    st = torch.cuda.Stream()
    sp = G.C.c_void_p(st.cuda_stream)

    def call():
        G.check(G.apus_gcuda_bf16_gemm_argmax_dev(G.ptr(w), G.ptr(x), None, G.ptr(ids), rows, V, d, sp), "lm_head")
    for _ in range(3):
        call()
    st.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        call()
    e1.record(st)
    st.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    del w
    torch.cuda.empty_cache()
    return us, V * d * 2 + rows * d * 2


def bench_c2(args, ws, rank, W=None):
    import numpy as np
    import torch
    import apus_gcuda as G
    G.enable()
    kw = c2_config(args.small)
    depth = C2["depth"]
    ep = ws > 1 and args.mode == "ep"
    if W is None:
        W = c2_weights(kw, C2["seed"], keep=ep_owns(kw, rank, ws) if ep else None)
    prompt = c2_prompt(kw, C2["seed"])[:args.prompt or C2["prompt"]]
    cap = len(prompt) + depth * (2 * args.steps + 2 * args.warmup) + 64
    m = G.GModel(G.make_config(**kw), has_mtp=True, kv_cap=cap, depth=depth,
                 rank=rank if ep else 0, world=ws if ep else 1)
    if ep:   # one sequence over every GPU: experts and lm_head rows split
        m.ep_bootstrap(G.ep_all_gather())
    m.load(W)
    m.use_graph(True)
    if args.temp > 0:
        m.sampling(args.temp, args.top_p, args.seed)
    # every rank reaches the first device-side exchange together (its waits
    # are bounded at about a second)
    barrier(ws)
    m.spec_prefill(prompt)
    st = torch.cuda.ExternalStream(m.stream())
    for _ in range(args.warmup):
        m.spec_step_async()
    st.synchronize()
    s0, _ = m.stats()
    c0 = m.counters()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        time.sleep(0.3)
        torch.cuda.nvtx.range_push("timed")
        e0.record(st)
        for _ in range(args.steps):
            m.spec_step_async()
        e1.record(st)
        st.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = e0.elapsed_time(e1)
    s1, rc = m.stats()
    c1 = m.counters()
    if rc != 0:
        raise RuntimeError("sequence ran past its capacity")
    barrier(ws)
    ms = max_over_ranks(ms, ws)
    emitted = s1["emitted"] - s0["emitted"]
    per = ms / args.steps
    tok_s = emitted / (ms * 1e-3)
    n_ctx = (s0["pos"] + s1["pos"]) // 2
    probs = (c1["moe_problems"] - c0["moe_problems"]) / args.steps
    algo, _ = c2_algo_bytes(kw, depth, n_ctx, probs, ws if ep else 1)
    hbm, _, src = peaks()
    gbs = algo / (per * 1e-3) / 1e9
    offered = s1["offered"] - s0["offered"]
    accepted = s1["accepted"] - s0["accepted"]
    agg = 1 if ep else ws       # EP: one sequence across the GPUs; replicas: ws sequences
    out = {"metric": METRIC, "value": round(tok_s * agg, 2), "unit": "accepted tok/s",
           "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per, 4),
           "higher_is_better": True, "scaling": "strong" if ep else "weak", "vs_baseline": None,
           "dtype": "bf16 activations, fp8e4m3/bf16 weights, f32 accumulation",
           "data": f"synthetic random-init weights (seed {C2['seed']}), {len(prompt)} uniform random prompt ids",
           "config": {"workload": c2_workload(args.temp, args.top_p, args.seed),
                      "depth": "BASELINE depth 3 = 4 verify rows (reference APUS_SPEC_K 4)",
                      "prompt": len(prompt),
                      "parallelism": (f"ep{ws}: routed experts and lm_head rows split over {ws} GPUs, "
                                      "peer-memory exchange per MoE layer and per lm_head") if ep
                      else f"replicas x{ws}",
                      "l2": "inputs larger than L2: each step streams ~10 GB of weights",
                      "step": "one device-resident speculative step replayed from a CUDA graph"},
           "spec": {"tokens_per_step": round(emitted / args.steps, 4), "offered": offered, "accepted": accepted,
                    "acceptance": round(accepted / offered, 4) if offered else None,
                    "context_avg": n_ctx},
           "step_roofline": {"achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4),
                             "algo_bytes_per_step": int(algo), "moe_expert_problems_per_step": round(probs, 2),
                             "note": "algorithmic bytes per step / device step time"},
           "gpu_launches": int(c1["graph_kernels"]) * args.steps,
           "clocks": clk.summary()}
    # the dominant kernel: the lm_head GEMV, ~1/3 of the step.  Per step one
    # launch over the verify rows and the MTP replay rows together (2*depth
    # rows) and depth-1 one-row launches of the draft chain; timed in that mix
    rows_main = 2 * depth if 2 * depth <= 8 else depth
    n_one = depth - 1 if rows_main == 2 * depth else depth
    us_m, hb_m = lm_head_gemv_time(kw, rows_main, ws if ep else 1)
    us_1, hb_1 = lm_head_gemv_time(kw, 1, ws if ep else 1)
    us, hb = us_m + n_one * us_1, hb_m + n_one * hb_1
    # DRAM bytes of one full-vocabulary launch from the committed ncu capture;
    # a vocabulary slice moves its share of them
    traffic = profile_value("lm_head_gemv_k_gemv_tma.md", "dram_bytes_per_launch")
    if traffic is not None and ep:
        traffic = round(traffic / ws)
    hgbs = hb / us / 1e3
    nl = 1 + n_one
    out["roofline"] = {"bound": "hbm", "kernel": f"k_gemv_tma<false> lm_head (BF16 {-(-kw['vocab_size'] // (ws if ep else 1))}"
                                                  f"x{kw['hidden_size']} per rank, fused argmax)",
                       "achieved": round(hgbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(hgbs / hbm, 4),
                       "traffic": traffic,
                       "algo_bytes_per_launch": round(hb / nl), "avg_launch_us": round(us / nl, 2),
                       "peak_source": src, "launches_per_step": nl,
                       "launch_mix": {f"{rows_main}_rows_us": round(us_m, 2), "1_row_us": round(us_1, 2),
                                      "1_row_launches": n_one}}
    if args.quick:
        m.close()
        return out, W
    # e2e: the reference-facing synchronous apus_gspec_step drop-in, host tokens out
    for _ in range(min(args.warmup, 3)):
        m.spec_step()
    t0 = time.perf_counter()
    n_e2e = 0
    for _ in range(args.steps):
        n_e2e += len(m.spec_step())
    e2e = max_over_ranks(time.perf_counter() - t0, ws)
    out["e2e"] = {"value": round(n_e2e / e2e * agg, 2), "unit": "accepted tok/s",
                  "path": "apus_gcuda_gspec_step per step, emitted tokens copied to the host",
                  "h2d_bytes_per_step": 0, "d2h_bytes_per_step": int(c1["ctl_bytes"]),
                  "note": "no per-step inputs cross to the device (the held token and drafts stay resident); "
                          "the control block with the emitted tokens is read back once a step"}
    # the same decode with the prompt upload and prefill inside the timed
    # region: host prompt ids in, host tokens out (a whole request)
    barrier(ws)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    m.spec_prefill(prompt)
    t_pf = time.perf_counter()
    n_req = 0
    for _ in range(args.steps):
        n_req += len(m.spec_step())
    t1 = time.perf_counter()
    req = max_over_ranks(t1 - t0, ws)
    out["e2e_request"] = {"value": round(n_req / req * agg, 2), "unit": "accepted tok/s",
                          "path": "apus_gcuda_gspec_prefill (host prompt ids) + apus_gcuda_gspec_step x steps",
                          "prompt": len(prompt), "prefill_ms": round((t_pf - t0) * 1e3, 2),
                          "h2d_bytes": int(len(prompt) * 4), "d2h_bytes_per_step": int(c1["ctl_bytes"])}
    m.close()
    out["fp8_gemv"] = fp8_gemv_leg()
    return out, W


# --------------------------------------------------------------------------
# config 3: the full-depth model, expert-parallel over the GPUs
C3 = dict(prompt=4096, depth=4, seed=3, sweep=(0.0, 0.5, 0.9))


def bench_c3(args, ws, rank):
    """the 45-layer real-dims glm5_next (~306 GiB of FP8
    experts) split expert-parallel over the ws GPUs (routed experts and
    lm_head rows; everything else replicated), synthetic weights generated on
    each device for its own slice (seed 3), a 4096-token random prompt, then
    speculative steps at depth 3 (4 verify rows) with draft agreement forced
    at p in {0, 0.5, 0.9}: each draft is the model's own greedy token with
    probability p, else that token + 1 (splitmix64 of the seed and the
    position).  The headline is p = 0: every step emits one token, as with
    random weights' own drafts.  A step is timed on the device (CUDA events
    on the model's stream), max over ranks."""
    import numpy as np
    import torch
    import apus_gcuda as G
    from synth import c3_config
    G.enable()
    kw = c3_config(args.layers or 45)
    depth = C3["depth"]
    n_prompt = args.prompt or C3["prompt"]
    prompt = np.random.default_rng(C3["seed"]).integers(0, kw["vocab_size"], n_prompt).astype(np.int32)
    n_truth = depth * (args.steps + args.warmup + 4) + 16
    cap = n_prompt + n_truth + 64
    m = G.GModel(G.make_config(**kw), has_mtp=True, kv_cap=cap, depth=depth, rank=rank, world=ws)
    if ws > 1:
        m.ep_bootstrap(G.ep_all_gather())
    t0 = time.perf_counter()
    m.init_random(C3["seed"])
    t_init = time.perf_counter() - t0
    m.use_graph(True)
    barrier(ws)
    t0 = time.perf_counter()
    truth = m.greedy(prompt, n_truth)       # the model's own greedy stream: the forcing's truth
    t_truth = time.perf_counter() - t0
    st = torch.cuda.ExternalStream(m.stream())
    hbm, _, src = peaks()
    runs = {}
    clk_sum = None
    for p in C3["sweep"]:
        m.force(truth, base=n_prompt, p=p, seed=C3["seed"])
        barrier(ws)
        t0 = time.perf_counter()
        m.spec_prefill(prompt)
        t_pf = time.perf_counter() - t0
        for _ in range(args.warmup):
            m.spec_step_async()
        st.synchronize()
        s0, _ = m.stats()
        c0 = m.counters()
        barrier(ws)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
            time.sleep(0.3)
            e0.record(st)
            for _ in range(args.steps):
                m.spec_step_async()
            e1.record(st)
            st.synchronize()
        ms = e0.elapsed_time(e1)
        s1, rc = m.stats()
        c1 = m.counters()
        if rc != 0:
            raise RuntimeError("sequence ran past its capacity")
        barrier(ws)
        ms = max_over_ranks(ms, ws)
        emitted = s1["emitted"] - s0["emitted"]
        per = ms / args.steps
        n_ctx = (s0["pos"] + s1["pos"]) // 2
        probs = (c1["moe_problems"] - c0["moe_problems"]) / args.steps
        algo, _ = c2_algo_bytes(kw, depth, n_ctx, probs, ws)
        algo = max_over_ranks(algo, ws)      # the busiest rank bounds the step
        gbs = algo / (per * 1e-3) / 1e9
        runs[p] = {"tok_s": round(emitted / (ms * 1e-3), 2), "ms_per_step": round(per, 4),
                   "tokens_per_step": round(emitted / args.steps, 4),
                   "acceptance": round((s1["accepted"] - s0["accepted"]) / max(1, s1["offered"] - s0["offered"]), 4),
                   "step_roofline": {"achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                     "frac": round(gbs / hbm, 4), "algo_bytes_per_step_busiest_rank": int(algo),
                                     "moe_expert_problems_per_step": round(probs, 2)},
                   "prefill_ms": round(t_pf * 1e3, 1), "context_avg": n_ctx}
        if p == C3["sweep"][0]:
            clk_sum = clk.summary()
            graph_kernels = int(c1["graph_kernels"])
    head = runs[C3["sweep"][0]]
    out = {"metric": METRIC, "value": head["tok_s"], "unit": "accepted tok/s", "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None,
           "dtype": "bf16 activations, fp8e4m3/bf16 weights, f32 accumulation",
           "data": f"synthetic random-init weights generated on each GPU for its slice (seed {C3['seed']}), "
                   f"{n_prompt} uniform random prompt ids",
           "config": {"workload": f"config3: full-depth glm5_next ({kw['num_hidden_layers']} layers: "
                                  f"{kw['num_hidden_layers'] - sum(kw['layer_is_dsa'])} KDA 64x128 + "
                                  f"{sum(kw['layer_is_dsa'])} DSA, 3 dense MLP + MoE 288 top-8 inter 2048, "
                                  "vocab 154880, real config.json dims) + 1 NextN MTP layer, greedy spec decode, "
                                  "draft agreement forced at p = 0 (headline)",
                      "depth": "BASELINE depth 3 = 4 verify rows (reference APUS_SPEC_K 4)",
                      "prompt": n_prompt,
                      "parallelism": f"ep{ws}: routed experts ({kw['n_routed_experts'] // ws} per GPU) and lm_head "
                                     f"rows split over {ws} GPUs, dense/attention/MTP replicated, peer-memory "
                                     "exchange per MoE layer and per lm_head",
                      "l2": "inputs larger than L2: each step streams tens of GB of weights per GPU",
                      "step": "one device-resident speculative step replayed from a CUDA graph"},
           "spec": {"tokens_per_step": head["tokens_per_step"], "acceptance": head["acceptance"],
                    "context_avg": head["context_avg"]},
           "forced_agreement": {str(p): r for p, r in runs.items()},
           "step_roofline": head["step_roofline"],
           "setup_s": {"init_random": round(t_init, 1), "truth_greedy": round(t_truth, 1)},
           "gpu_launches": graph_kernels * args.steps, "clocks": clk_sum}
    # the dominant kernel: the lm_head slice GEMV (as config 2's line)
    us_m, hb_m = lm_head_gemv_time(kw, 2 * depth, ws)
    us_1, hb_1 = lm_head_gemv_time(kw, 1, ws)
    n_one = depth - 1
    us, hb = us_m + n_one * us_1, hb_m + n_one * hb_1
    traffic = profile_value("lm_head_gemv_k_gemv_tma.md", "dram_bytes_per_launch")
    hgbs = hb / us / 1e3
    out["roofline"] = {"bound": "hbm", "kernel": f"k_gemv_tma<false> lm_head (BF16 {-(-kw['vocab_size'] // ws)}"
                                                  f"x{kw['hidden_size']} per rank, fused argmax)",
                       "achieved": round(hgbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(hgbs / hbm, 4),
                       "traffic": round(traffic / ws) if traffic is not None else None,
                       "algo_bytes_per_launch": round(hb / (1 + n_one)), "avg_launch_us": round(us / (1 + n_one), 2),
                       "peak_source": src, "launches_per_step": 1 + n_one}
    if not args.quick:
        # e2e: the synchronous apus_gcuda_gspec_step (host tokens out each step)
        m.force(truth, base=n_prompt, p=C3["sweep"][0], seed=C3["seed"])
        m.spec_prefill(prompt)
        for _ in range(min(args.warmup, 3)):
            m.spec_step()
        barrier(ws)
        t0 = time.perf_counter()
        n_e2e = 0
        for _ in range(args.steps):
            n_e2e += len(m.spec_step())
        e2e = max_over_ranks(time.perf_counter() - t0, ws)
        out["e2e"] = {"value": round(n_e2e / e2e, 2), "unit": "accepted tok/s",
                      "path": "apus_gcuda_gspec_step per step on every rank, emitted tokens copied to the host",
                      "h2d_bytes_per_step": 0, "d2h_bytes_per_step": int(m.counters()["ctl_bytes"])}
    m.close()
    return out


def cpu_c2(W, budget_s=20.0, prompt_len=C2["prompt"], log=None):
    """The reference's own speculative engine (oracle/_ref: apus_gspec_* over
    apus_gmodel, compiled from the reference sources) on the host cores with
    the same weights: prefill of the first prompt_len prompt tokens (not
    timed), then apus_gspec_step until budget_s.  Experts are dequantized to
    BF16 at load as the reference engine holds them (not timed)."""
    import numpy as np
    import oracle as O
    if O.REF is None:
        return None
    kw = c2_config()
    depth = C2["depth"]
    cfg = O.make_config(**kw)
    t_load = time.perf_counter()
    R = O.REF.ref_model_new(C.byref(cfg), 1)
    for name, arr in W.items():
        if O.REF.ref_model_set(R, name.encode(), O.p(arr)) != 0:
            raise KeyError(name)
    O.REF.ref_model_finalize(R)
    cap = prompt_len + 4096
    st = O.REF.ref_state_new(R, cap)
    sp = O.REF.ref_spec_new(R, st, cap, depth)
    ids = np.ascontiguousarray(c2_prompt(kw, C2["seed"])[:prompt_len])
    assert O.REF.ref_spec_prefill(sp, O.p(ids), len(ids)) == 0
    t_load = time.perf_counter() - t_load
    buf = np.zeros(depth + 1, np.int32)
    n = tok = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or n < 1:
        k = O.REF.ref_spec_step(sp, O.p(buf), depth + 1)
        if k <= 0:
            break
        tok += k
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(tok / dt, 4), "unit": "accepted tok/s", "cores": O.REF.apus_ref_threads(),
            "kind": "reference",
            "sample": f"{n} apus_gspec_step calls ({tok} tokens, {dt:.1f} s) after the {prompt_len}-token prompt's "
                      f"prefill (weights, expert dequant and prefill {t_load:.0f} s, untimed)"}


def tc_table(rows=(512, 2048), reps=20):
    """Prefill-chunk linears of the config-2 model on the tcgen05 GEMM
    (--tc-table): BF16 weights, M rows of activations, fp32 accumulation,
    CUDA events on the launching stream over back-to-back launches, with
    torch.matmul (cuBLAS) on the same operands beside it.  Prints one JSON
    line per (matrix, rows)."""
    import torch
    import apus_gcuda as G
    G.enable()
    kw = c2_config()
    d, V, qkv = kw["hidden_size"], kw["vocab_size"], kw["linear_num_heads"] * kw["linear_head_dim"]
    D, H = kw["linear_head_dim"], kw["linear_num_heads"]
    shapes = [("kda_proj", 3 * qkv + 2 * D + H, d), ("kda_o", d, qkv), ("eh_proj", d, 2 * d),
              ("dsa_o", d, kw["num_attention_heads"] * kw["v_head_dim"]), ("lm_head", V, d),
              ("square8k", 8192, 4096)]
    st = torch.cuda.Stream()
    sp = G.C.c_void_p(st.cuda_stream)
    _, tf_peak, src = peaks()
    for name, O_, K_ in shapes:
        for M in rows:
            w = (torch.randn(O_, K_, device="cuda") * 0.02).to(torch.bfloat16)
            x = torch.randn(M, K_, device="cuda").to(torch.bfloat16)
            y = torch.empty(M, O_, device="cuda", dtype=torch.bfloat16)
            fl = 2.0 * M * O_ * K_
            res = {}
            for arm in ("tc", "cublas"):
                with torch.cuda.stream(st):
                    def run():
                        if arm == "tc":
                            G.check(G.apus_gcuda_bf16_gemm_dev(G.ptr(w), G.ptr(x), G.ptr(y), M, O_, K_, sp))
                        else:
                            torch.matmul(x, w.t(), out=y)
                    for _ in range(3):
                        run()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    for _ in range(reps):
                        run()
                    e1.record(st)
                st.synchronize()
                res[arm] = e0.elapsed_time(e1) * 1e3 / reps
            print(json.dumps({"matrix": name, "M": M, "O": O_, "K": K_, "kernel": "k_gemm_tc (tcgen05, 128x256 tiles)",
                              "us": round(res["tc"], 2), "tflops": round(fl / res["tc"] / 1e6, 1),
                              "frac_of_peak": round(fl / res["tc"] / 1e6 / tf_peak, 3), "peak_tflops": tf_peak,
                              "peak_source": src, "cublas_us": round(res["cublas"], 2),
                              "cublas_tflops": round(fl / res["cublas"] / 1e6, 1),
                              "kernel_error": G.apus_gcuda_kernel_error()}), flush=True)
            del w, x, y
    torch.cuda.empty_cache()


def gemv_table(only="all", rows=(8, 4, 1), reps=50):
    """Per-shape GEMV timings of the config-2 step's matrices (profiling aid,
    --gemv-table): back-to-back PDL launches over rotating weight copies
    (>= 512 MB per shape, so every launch streams from HBM), CUDA events on
    the launching stream.  Prints one JSON line per (matrix, rows)."""
    import numpy as np
    import torch
    import apus_gcuda as G
    G.enable()
    G.apus_gcuda_set_pdl(1)
    kw = c2_config()
    d, V, qkv = kw["hidden_size"], kw["vocab_size"], kw["linear_num_heads"] * kw["linear_head_dim"]
    D, H = kw["linear_head_dim"], kw["linear_num_heads"]
    AH, qd, vd, ql, kl = (kw["num_attention_heads"], kw["qk_nope_head_dim"], kw["v_head_dim"], kw["q_lora_rank"],
                          kw["kv_lora_rank"])
    IH, ID, E = kw["index_n_heads"], kw["index_head_dim"], kw["n_routed_experts"]
    shapes = [("lm_head", V, d, "bf16"), ("kda_proj", 3 * qkv + 2 * D + H, d, "bf16"), ("kda_o", d, qkv, "bf16"),
              ("eh_proj", d, 2 * d, "bf16"), ("router", E, d, "f32"), ("dsa_qa_kva", ql + kl, d, "fp8"),
              ("dsa_qb", AH * qd, ql, "fp8"), ("dsa_kvb", AH * (qd + vd), kl, "bf16"),
              ("idx_wqb", IH * ID, ql, "bf16"), ("idx_kgw", 2 * ID + IH, d, "bf16"), ("dsa_o", d, AH * vd, "fp8"),
              ("config0", C0["N"], C0["K"], "fp8"), ("expert_gu", 2 * kw["moe_intermediate_size"], d, "fp8"),
              ("expert_down", d, kw["moe_intermediate_size"], "fp8")]
    st = torch.cuda.Stream()
    sp = G.C.c_void_p(st.cuda_stream)
    hbm, _, _ = peaks()
    for name, O_, K_, kind in shapes:
        if only not in ("all", name):
            continue
        wb = O_ * K_ * (1 if kind == "fp8" else 2)
        nbuf = max(1, -(-(512 << 20) // wb))
        if kind == "fp8":
            Ws = [torch.randint(0, 120, (O_, K_), dtype=torch.uint8, device="cuda") for _ in range(nbuf)]
            S = torch.full(((O_ + 127) // 128, (K_ + 127) // 128), 1e-3, device="cuda")
        else:
            Ws = [torch.randn(O_, K_, device="cuda").to(torch.bfloat16) * 0.02 for _ in range(nbuf)]
        for R in rows:
            x = torch.randn(R, K_, device="cuda").to(torch.bfloat16)
            y = torch.empty(R, O_, device="cuda", dtype=torch.float32 if kind == "f32" else torch.bfloat16)

            def call(i):
                w = Ws[i % nbuf]
                if kind == "fp8":
                    rc = G.apus_gcuda_fp8blk_linear_dev(G.ptr(w), G.ptr(S), G.ptr(x), G.ptr(y), R, O_, K_, sp)
                elif kind == "f32":
                    rc = G.apus_gcuda_bf16_gemm_f32_dev(G.ptr(w), G.ptr(x), G.ptr(y), R, O_, K_, sp)
                else:
                    rc = G.apus_gcuda_bf16_gemm_dev(G.ptr(w), G.ptr(x), G.ptr(y), R, O_, K_, sp)
                G.check(rc, name)
            for i in range(5):
                call(i)
            st.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for i in range(reps):
                call(i)
            e1.record(st)
            st.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / reps
            algo = wb + (S.numel() * 4 if kind == "fp8" else 0)
            print(json.dumps({"matrix": name, "O": O_, "K": K_, "weights": kind, "rows": R,
                              "us": round(us, 2), "GB/s": round(algo / us / 1e3, 1),
                              "frac": round(algo / us / 1e3 / hbm, 3)}), flush=True)
        del Ws
        torch.cuda.empty_cache()


def prefill_table(reps=3):
    """The prompt pass of config 2 (512 prompt tokens, the MTP replay
    included: apus_gcuda_gspec_prefill) timed with CUDA events after one
    untimed call, `reps` calls (profiling aid, --prefill-table).  Prints one
    JSON line."""
    import numpy as np
    import torch
    import apus_gcuda as G
    G.enable()
    kw = c2_config()
    W = c2_weights(kw, C2["seed"])
    prompt = c2_prompt(kw, C2["seed"])[:C2["prompt"]]
    m = G.GModel(G.make_config(**kw), has_mtp=True, kv_cap=len(prompt) + 64, depth=C2["depth"])
    m.load(W)
    m.spec_prefill(prompt)
    st = torch.cuda.ExternalStream(m.stream())
    ms = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("prefill")
        e0.record(st)
        m.spec_prefill(prompt)
        e1.record(st)
        st.synchronize()
        torch.cuda.nvtx.range_pop()
        ms.append(e0.elapsed_time(e1))
    m.close()
    print(json.dumps({"workload": "config2 prompt pass: apus_gcuda_gspec_prefill, 512 tokens", "calls": reps,
                      "ms": [round(x, 2) for x in ms], "ms_min": round(min(ms), 2)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: 256 for config 2, else 200)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=None,
                    help="BASELINE config (default: 2 on one GPU, 3 -- the full model, expert-parallel -- on several)")
    ap.add_argument("--layers", type=int, default=0, help="config 3: layers (default 45; fewer for quick checks)")
    ap.add_argument("--prompt", type=int, default=0, help="config 2: prompt tokens (default 512; profiling only)")
    ap.add_argument("--small", action="store_true",
                    help="config 2 layer shapes with 16 experts and a 16384 vocab (profiling captures only)")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of reference CPU decode sampled")
    ap.add_argument("--mode", default="ep", choices=["ep", "replicas"],
                    help="config 2 with several GPUs: one sequence expert-parallel over all of them (ep), "
                         "or one independent sequence per GPU (replicas)")
    ap.add_argument("--gemv-table", nargs="?", const="all", default=None,
                    help="per-matrix GEMV timings of the config-2 step (profiling aid, one GPU); "
                         "optionally one matrix name")
    ap.add_argument("--tc-table", nargs="*", type=int, default=None,
                    help="prefill-chunk linears on the tcgen05 GEMM vs cuBLAS (profiling aid, one GPU); "
                         "optionally the row counts (default 512 2048)")
    ap.add_argument("--prefill-table", action="store_true",
                    help="config 2's 512-token prompt pass timed alone (profiling aid, one GPU)")
    ap.add_argument("--temp", type=float, default=0.0,
                    help="config 2: sampled decode at this temperature (default 0: greedy, the headline)")
    ap.add_argument("--top-p", type=float, default=0.95, help="config 2 sampled decode: nucleus top_p")
    ap.add_argument("--seed", type=int, default=12345, help="config 2 sampled decode: splitmix64 seed")
    ap.add_argument("--quick", action="store_true",
                    help="device-timed kernels only (no e2e, no CPU baseline): the profiling command")
    args = ap.parse_args()
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.config is None:
        args.config = 2 if ws == 1 and args.gpus <= 1 else 3
    if args.steps is None:
        args.steps = {2: 256, 3: 32}.get(args.config, 200)
    if args.impl == "reference":
        if rank != 0:
            return
        line = {"metric": METRIC, "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True}
        if args.config == 2:
            import oracle as O
            if O.REF is None:
                line["unavailable"] = "reference CPU engine (oracle/_ref/libapus_ref.so) not built"
            else:
                cb = cpu_c2(c2_weights(c2_config(), C2["seed"]), budget_s=args.cpu_budget)
                line.update({"value": cb["value"], "unit": cb["unit"],
                             "config": {"workload": c2_workload(),
                                        "depth": "BASELINE depth 3 = 4 verify rows (reference APUS_SPEC_K 4)",
                                        "prompt": C2["prompt"],
                                        "parallelism": f"the reference's CPU engine on {cb['cores']} host threads"},
                             "cpu_baseline": cb,
                             "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                                     "d2h_bytes_per_step": 0}})
        elif args.config == 3:
            line["unavailable"] = ("config 3 is the 306 GiB 45-layer model; the reference CPU engine holds its "
                                   "experts dequantized in host RAM and cannot load it on this host")
        else:
            cb = cpu_c0(budget_s=max(3.0, 0.05 * args.steps))
            if cb is None:
                line["unavailable"] = "reference CPU engine (oracle/_ref/libapus_ref.so) not built"
            else:
                line.update({"value": cb["value"], "unit": "GB/s (FP8 GEMV algorithmic bytes, config 0)",
                             "config": {"workload": "config0 on host cores"}, "cpu_baseline": cb,
                             "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                                     "d2h_bytes_per_step": 0}})
        print(json.dumps(line), flush=True)
        return
    ws, rank, local = dist_init()
    if args.temp > 0 and ws > 1 and args.mode == "ep":
        raise SystemExit("sampled decode runs on one GPU per sequence (use --mode replicas)")
    if args.gemv_table:
        gemv_table(args.gemv_table)
        return
    if args.tc_table is not None:
        tc_table(tuple(args.tc_table) or (512, 2048))
        return
    if args.prefill_table:
        prefill_table()
        return
    if args.config == 3:
        out = bench_c3(args, ws, rank)
        if rank == 0:
            print(json.dumps(out), flush=True)
    elif args.config == 2:
        out, W = bench_c2(args, ws, rank)
        if rank == 0 and not args.quick and ws == 1 and args.temp <= 0:   # the reference leg decodes greedily
            out["cpu_baseline"] = cpu_c2(W, budget_s=args.cpu_budget)
            if "fp8_gemv" in out:
                out["fp8_gemv"]["cpu_baseline"] = cpu_c0(budget_s=5.0)
        if rank == 0:
            print(json.dumps(out), flush=True)
    elif args.config == 1:
        out = bench_c1(args, ws, rank)
        h = out.pop("_moe", None)
        if rank == 0 and not args.quick and h:
            out["cpu_baseline"] = cpu_c1(h, budget_s=10.0)
        if rank == 0:
            print(json.dumps(out), flush=True)
    else:
        out = bench_c0(args, ws, rank)
        if rank == 0:
            if not args.quick:
                out["cpu_baseline"] = cpu_c0(budget_s=10.0)
            print(json.dumps(out), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
