"""Expert parallelism across GPUs (include/apus_gmtp_gcuda.h, _new_ep /
_ep_handle / _ep_connect): one process per GPU, routed experts and lm_head
rows split over the ranks, every MoE layer and every lm_head exchanging
through peer memory.  The token streams (greedy, speculative, forced full
accept, forced partial accept with rollback, CUDA-graph replay, on-device
random weights, a 300-token prompt whose prompt pass runs two 256-row
chunks through the gathered MoE's exchange, sampled decode, speculative and
not, on the logits rows gathered from every rank's vocabulary slice, and the
decode batch's logits) and the committed-state digests
must equal the one-GPU engine's bit for bit on every rank.  Needs as many
GPUs as ranks."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _n_gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_streams_equal_one_gpu(world, tmp_path):
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "ep.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "ep_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    rep = json.loads(out.read_text())
    one = rep["one_gpu"]
    assert one["kernel_error"] == 0
    assert one["forced_full_stats"]["accepted"] == one["forced_full_stats"]["offered"] > 0
    assert 0 < one["forced_half_stats"]["accepted"] < one["forced_half_stats"]["offered"]
    for rank, ep in enumerate(rep["ranks"]):
        assert ep["kernel_error"] == 0, f"rank {rank}: exchange error {ep['kernel_error']}"
        assert ep["stored_ok"], f"rank {rank}: set() stored the wrong expert slice"
        for key in ("long_greedy", "long_spec", "long_digest", "sampled_generate", "sampled_spec", "sampled_rng",
                    "logits_sha", "greedy", "spec", "spec_digest", "forced_full",
                    "forced_full_digest", "forced_half",
                    "forced_half_stats", "forced_half_digest", "graph", "graph_digest", "random_greedy"):
            assert ep[key] == one[key], f"rank {rank}: {key} differs from the one-GPU engine"
