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
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=0)
    ap.add_argument("--quick", action="store_true",
                    help="device-timed kernels only (no e2e, no CPU baseline): the profiling command")
    args = ap.parse_args()
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_c0(budget_s=max(3.0, 0.05 * args.steps))
        line = {"metric": METRIC, "impl": "reference"}
        if cb is None:
            line["unavailable"] = "reference CPU engine (oracle/_ref/libapus_ref.so) not built"
        else:
            line.update({"value": cb["value"], "unit": "GB/s (FP8 GEMV algorithmic bytes, config 0)",
                         "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                         "higher_is_better": True, "config": {"workload": "config0 on host cores"},
                         "cpu_baseline": cb,
                         "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                                 "d2h_bytes_per_step": 0}})
        print(json.dumps(line), flush=True)
        return
    ws, rank, local = dist_init()
    if args.config == 1:
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
