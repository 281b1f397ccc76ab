"""The bench's multi-rank plumbing on CPU: two gloo ranks (127.0.0.1) take
the max of their timings and meet at the barriers, the way `bench.py --gpus N`
ranks do over NCCL.  Config 2 runs one replica per GPU with no data-path
collective, so these are the only cross-rank steps."""
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
        q.put((rank, m))
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
    assert got == [(r, 10.0 + ws - 1) for r in range(ws)]
