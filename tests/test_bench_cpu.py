"""bench.py's host-side pieces, no GPU: the committed ncu figure the
roofline's traffic comes from, and the algorithmic bytes of a step (the
replay rows share the verify rows' pass over the head when 2*depth <= 8)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_profile_value_for_roofline_traffic():
    v = bench.profile_value("lm_head_gemv_k_gemv_tma.md", "dram_bytes_per_launch")
    kw = bench.c2_config(False)
    head = kw["vocab_size"] * kw["hidden_size"] * 2
    assert v is not None and head <= v <= 1.01 * head      # no re-reads of the 1.27 GB head
    assert bench.profile_value("lm_head_gemv_k_gemv_tma.md", "no_such_key") is None


def test_algo_bytes_share_the_head_pass():
    kw = bench.c2_config(False)
    head = kw["vocab_size"] * kw["hidden_size"] * 2
    # ~190 expert GEMV pairs a step on one GPU (routed unions + shared experts)
    b4, calls4 = bench.c2_algo_bytes(kw, 4, 640, 190.0)
    b5, _ = bench.c2_algo_bytes(kw, 5, 640, 190.0)
    # depth 4: the verify rows and the replay share one pass (4 passes a step);
    # depth 5 (10 rows > 8): a separate replay pass, plus one more chain step
    assert 8e9 < b4 < 11e9
    assert b5 - b4 > 2 * head * 0.99
    assert calls4 == kw["num_hidden_layers"] + 1 + 3
    # expert parallelism: each rank reads its vocabulary slice of the head
    b4_ep, _ = bench.c2_algo_bytes(kw, 4, 640, 97.0, world=2)
    assert b4_ep < b4
