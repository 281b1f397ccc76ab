"""Expert-parallel worker for tests/test_ep_gpu.py: one process per GPU under
torch.distributed.run (gloo carries only the 64-byte handle exchange and the
host-side result gather; the per-layer exchange runs in the engine's own
kernels over peer memory).

Every rank builds the tiny glm5_next model with its slice of the routed
experts and lm_head rows, runs greedy decode, plain / forced-accept /
forced-rollback speculative steps and CUDA-graph steps, and rank 0 compares
each token stream and state digest with a one-GPU model of the same weights:
the expert-parallel engine must reproduce the one-GPU engine bit for bit.

usage: python -m torch.distributed.run --nproc-per-node N tests/ep_worker.py OUT.json
"""
import datetime
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (HERE, ROOT, os.path.join(ROOT, "apus-glm5.3-flash_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

PROMPT = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]
# a prompt over two 256-row chunks of the prompt pass (its MoE exchange runs once a chunk)
LONG = [(i * 7919 + 13) % 1024 for i in range(300)]


def ep_config():
    from modelgen import tiny_config
    # 16 experts and 1024 vocabulary rows split evenly over 2, 4 or 8 ranks
    return tiny_config(n_routed_experts=16, num_experts_per_tok=4, vocab_size=1024)


def run(G, kw, W, rank, world, seed_random=None):
    """Every stream the comparison needs, from one model."""
    m = G.GModel(G.make_config(**kw), has_mtp=True, kv_cap=400, depth=4, rank=rank, world=world)
    res = {}
    if world > 1:
        m.ep_bootstrap(G.ep_all_gather())
    owns = G.ep_owns(kw, rank, world)
    stored = {k: m.set(k, v) for k, v in W.items()}
    res["stored_ok"] = all(stored[k] == owns(k) for k in W)
    if world > 1:    # the device-side exchanges wait at most about a second
        import torch.distributed as dist
        dist.barrier()
    res["long_greedy"] = m.greedy(LONG, 12)
    m.reset()
    m.spec_prefill(LONG)
    res["long_spec"] = m.spec_step() + m.spec_step()
    res["long_digest"] = m.digest()
    m.reset()
    res["greedy"] = m.greedy(PROMPT, 40)
    truth = res["greedy"]
    m.reset()
    m.spec_prefill(PROMPT)
    spec = []
    for _ in range(8):
        spec += m.spec_step()
    res["spec"] = spec
    res["spec_digest"] = m.digest()
    for name, p in (("forced_full", 1.0), ("forced_half", 0.5)):
        m.reset()
        m.force(truth, base=len(PROMPT), p=p, seed=3)
        m.spec_prefill(PROMPT)
        out = []
        for _ in range(6):
            out += m.spec_step()
        res[name] = out
        res[name + "_stats"] = m.stats()[0]
        res[name + "_digest"] = m.digest()
    m.force(None, 0)
    m.reset()
    m.use_graph(True)
    m.spec_prefill(PROMPT)
    for _ in range(8):
        m.spec_step_async()
    res["graph"] = m.emitted()
    res["graph_digest"] = m.digest()
    m.use_graph(False)
    # sampled decode: every rank gathers the full logits rows and draws the same tokens
    m.sampling(0.8, 0.95, 4242)
    res["sampled_generate"] = m.generate(PROMPT, 24)
    m.reset()
    m.spec_prefill(PROMPT)
    sspec = []
    for _ in range(8):
        sspec += m.spec_step()
    res["sampled_spec"] = sspec
    res["sampled_rng"] = m.rng_state()
    m.sampling(0.0)
    m.reset()
    import hashlib
    res["logits_sha"] = hashlib.sha256(m.decode_batch(PROMPT[:8]).tobytes()).hexdigest()
    if seed_random is not None:   # on-device synthetic weights, drawn per rank slice
        m.init_random(seed_random)
        res["random_greedy"] = m.greedy(PROMPT, 16)
    res["kernel_error"] = G.apus_gcuda_kernel_error()
    m.close()
    return res


def main():
    import torch
    import torch.distributed as dist
    out_path = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    import apus_gcuda as G
    from modelgen import gen_weights
    G.enable()
    kw = ep_config()
    W = gen_weights(kw, seed=20261207)
    ep = run(G, kw, W, rank, world, seed_random=11)
    every = [None] * world
    dist.all_gather_object(every, ep)
    if rank == 0:
        one = run(G, kw, W, 0, 1, seed_random=11)
        report = {"world": world, "one_gpu": one, "ranks": every}
        with open(out_path, "w") as f:
            json.dump(report, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
