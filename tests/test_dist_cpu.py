"""The bench's multi-rank plumbing on CPU: two gloo ranks (127.0.0.1) take
the max of their timings and meet at the barriers, the way `bench.py --gpus N`
ranks do over NCCL, and the expert-parallel bootstrap exchanges every rank's
64-byte exchange-region handle in rank order.  The per-layer expert exchange
itself runs in the engine's kernels over peer memory (tests/test_ep_gpu.py)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, ws, port, q):
    import datetime
    import sys
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        bench.barrier(ws)
        m = bench.max_over_ranks(10.0 + rank, ws)
        bench.barrier(ws)
        sys.path.insert(0, os.path.join(ROOT, "apus-glm5.3-flash_b200"))
        import apus_gcuda as G
        hs = G.ep_all_gather()(bytes([rank]) * G.EP_HANDLE_BYTES)
        blob = G.ep_handles_blob(hs, ws)
        q.put((rank, m, blob == b"".join(bytes([r]) * G.EP_HANDLE_BYTES for r in range(ws))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ws", [2])
def test_max_over_ranks_gloo(ws):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(ws))
    assert got == [(r, 10.0 + ws - 1, True) for r in range(ws)]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ep_owns_partitions_experts(world):
    """Every routed expert tensor is stored by exactly one rank, every other
    tensor by all ranks; bad handle lists are refused."""
    import sys
    sys.path.insert(0, os.path.join(ROOT, "apus-glm5.3-flash_b200"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import apus_gcuda as G
    from modelgen import tiny_config
    kw = tiny_config(n_routed_experts=16, num_experts_per_tok=4, vocab_size=1024)
    names = [s[0] for s in G.tensor_specs(kw)]
    owners = [G.ep_owns(kw, r, world) for r in range(world)]
    for n in names:
        k = sum(o(n) for o in owners)
        assert k == (1 if ".mlp.experts." in n else world), n
    e3 = [n for n in names if ".mlp.experts.3." in n]
    assert e3 and all(owners[3 * world // 16](n) for n in e3)
    with pytest.raises(G.GcudaError):
        G.ep_owns(kw, 0, 3)
    with pytest.raises(G.GcudaError):
        G.ep_handles_blob([b"x" * 64], 2)
    with pytest.raises(G.GcudaError):
        G.ep_handles_blob([b"x" * 64, b"y" * 63], 2)
