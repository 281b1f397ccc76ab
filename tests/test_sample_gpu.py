"""Temperature / top-p sampling on the B200 (apus_gcuda_sample_rows_dev and
the sampled speculative step) against the reference's sampler.

  * the kernel on the golden cases of tests/golden/sample.npz gives the
    reference's own tokens (c/sample.h apus_sample_logits_u, compiled from
    the reference sources by tests/golden/gen_sample_golden.py): the stream
    state handed to the kernel is chosen so that its first draw is the
    case's uniform;
  * on fresh rows it equals the oracle's exact-arithmetic restatement
    bitwise, row r drawing the (r+1)-th splitmix64 uniform;
  * inside the engine the sampled speculative stream is bitwise the
    engine's own sampled non-speculative stream with the same seed, one
    uniform per emitted token (tests/m8g/test_m8g.c:730-772, sampled leg
    temp 0.8, top_p 0.95, seed 12345), and the committed state after
    accept/rollback is that of decoding the emitted tokens.
"""
import os
import sys

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN
from modelgen import gen_weights, tiny_config

sys.path.insert(0, GOLDEN)
from sample_cases import cases  # noqa: E402

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(GOLDEN, "sample.npz"))
C1, C2 = 0xBF58476D1CE4E5B9, 0x94D049BB133111EB
M64 = (1 << 64) - 1
PROMPT = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]


def _unxorshift(y, k):
    x = y
    for _ in range(64 // k + 1):
        x = y ^ (x >> k)
    return x


def state_for_u53(u53):
    """A splitmix64 state whose next draw has top 53 bits u53 (the mix is a
    bijection: undo its xor-shifts and odd multiplications)."""
    z = u53 << 11
    z = _unxorshift(z, 31)
    z = (z * pow(C2, -1, 1 << 64)) & M64
    z = _unxorshift(z, 27)
    z = (z * pow(C1, -1, 1 << 64)) & M64
    z = _unxorshift(z, 30)
    return (z - O.GOLDEN) & M64


def dev_sample(gcuda, rows, temp, top_p, state, ld=None):
    import torch
    rows = np.atleast_2d(np.ascontiguousarray(rows, np.uint16))
    R, V = rows.shape
    ld = ld or V
    buf = np.zeros((R, ld), np.uint16)
    buf[:, :V] = rows
    t = torch.from_numpy(buf.view(np.int16)).cuda()
    out = torch.full((R,), -1, dtype=torch.int32, device="cuda")
    gcuda.check(gcuda.apus_gcuda_sample_rows_dev(gcuda.ptr(t), R, ld, V, float(temp), float(top_p),
                                                 state & M64, gcuda.ptr(out), gcuda.stream_of()), "sample_rows")
    torch.cuda.synchronize()
    return out.cpu().numpy().tolist()


def test_state_inversion():
    for u53 in (0, 1, 12345, (1 << 53) - 1):
        draws, _ = O.rng_draws(state_for_u53(u53), 1)
        assert draws[0] >> 11 == u53


def test_golden_cases(gcuda):
    bad = []
    for i, (name, row, temp, top_p, u53) in enumerate(cases()):
        got = dev_sample(gcuda, row, temp, top_p, state_for_u53(u53))[0]
        if got != GOLD["tokens"][i]:
            bad.append((name, got, int(GOLD["tokens"][i])))
    assert not bad, bad


@pytest.mark.parametrize("V,sigma,temp,top_p", [(154880, 1.0, 0.8, 0.95), (154880, 4.0, 1.0, 1.0),
                                                (154880, 0.02, 0.8, 0.95), (4096, 2.0, 0.5, 0.5),
                                                (384, 1.0, 1.3, 0.9), (997, 2.0, 0.7, 0.9)])
def test_rows_equal_exact_restatement(gcuda, V, sigma, temp, top_p):
    rng = np.random.default_rng(V + int(sigma * 100))
    R = 8
    rows = O.bf16_of(rng.standard_normal((R, V)).astype(np.float32) * sigma)
    state = int(rng.integers(0, 1 << 62))
    got = dev_sample(gcuda, rows, temp, top_p, state)
    draws, _ = O.rng_draws(state, R)
    want = [O.sample_exact(rows[r], temp, top_p, draws[r] >> 11) for r in range(R)]
    assert got == want
    faithful = [O.sample_logits_u(rows[r], temp, top_p, (draws[r] >> 11) * 2.0 ** -53) for r in range(R)]
    assert sum(a == b for a, b in zip(got, faithful)) >= R - 1


def test_unaligned_rows_and_stride(gcuda):
    """Rows not on a 16-byte boundary take the scalar load path."""
    rng = np.random.default_rng(5)
    V = 1001
    rows = O.bf16_of(rng.standard_normal((3, V)).astype(np.float32))
    for ld in (V, 1008):
        got = dev_sample(gcuda, rows, 0.9, 0.9, 99, ld=ld)
        draws, _ = O.rng_draws(99, 3)
        assert got == [O.sample_exact(rows[r], 0.9, 0.9, draws[r] >> 11) for r in range(3)]


def test_greedy_rows(gcuda):
    rng = np.random.default_rng(3)
    rows = O.bf16_of(np.round(rng.standard_normal((4, 5000)) * 4).astype(np.float32))   # many exact ties
    got = dev_sample(gcuda, rows, 0.0, 1.0, 0)
    assert got == [O.argmax_bf16(rows[r]) for r in range(4)]
    z = next(c for c in cases() if c[0] == "zeros_t0.0_p1.0")[1]
    assert dev_sample(gcuda, z, 0.0, 1.0, 0) == [3]          # -0 at 3 ties +0 at 7


# ---- the sampled speculative step ------------------------------------------------

@pytest.fixture(scope="module")
def tiny():
    kw = tiny_config()
    return kw, gen_weights(kw, seed=20261201)


def gpu_model(gcuda, kw, W, cap=256, depth=4):
    m = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=cap, depth=depth)
    m.load(W)
    return m


@pytest.mark.parametrize("depth", [1, 2, 3, 4])
def test_spec_sampled_equals_nonspec(gcuda, tiny, depth):
    kw, W = tiny
    temp, top_p, seed = 0.8, 0.95, 12345
    g = gpu_model(gcuda, kw, W, depth=depth)
    g.sampling(temp, top_p, seed)
    g.spec_prefill(PROMPT)
    out = []
    for _ in range(12):
        out += g.spec_step()
    stats, rc = g.stats()
    assert rc == 0 and stats["emitted"] == len(out) and stats["pos"] == len(PROMPT) + len(out)
    # one uniform per token: the prefill's held token plus every emitted one
    assert g.rng_state() == (seed + (len(out) + 1) * O.GOLDEN) & M64
    dig = g.digest()
    ref_m = gpu_model(gcuda, kw, W)
    ref_m.sampling(temp, top_p, seed)
    ref = ref_m.generate(PROMPT, len(out) + 1)
    assert out == ref[:len(out)] and stats["held"] == ref[len(out)]
    assert ref_m.rng_state() == g.rng_state()
    assert ref_m.digest() == dig
    if depth > 1:
        assert stats["offered"] > 0


def test_sampled_prefill_draw(gcuda, tiny):
    """The held token after a sampled prefill is the sampler's draw on the
    last prompt row's logits with the first uniform of the stream."""
    kw, W = tiny
    g = gpu_model(gcuda, kw, W)
    lg, _ = g.prefill(PROMPT)
    draws, _ = O.rng_draws(777, 1)
    want = O.sample_exact(lg[-1], 0.7, 0.9, draws[0] >> 11)
    g.sampling(0.7, 0.9, 777)
    g.spec_prefill(PROMPT)
    assert g.stats()[0]["held"] == want
    g.sampling(0.7, 0.9, 777)
    assert g.generate(PROMPT, 1) == [want]


def test_sampled_graph_equals_sync(gcuda, tiny):
    kw, W = tiny
    a = gpu_model(gcuda, kw, W, depth=4)
    a.sampling(1.0, 1.0, 5)
    a.spec_prefill(PROMPT)
    sync = []
    for _ in range(10):
        sync += a.spec_step()
    b = gpu_model(gcuda, kw, W, depth=4)
    b.use_graph(True)
    b.sampling(1.0, 1.0, 5)
    b.spec_prefill(PROMPT)
    for _ in range(10):
        b.spec_step_async()
    assert b.emitted() == sync
    assert b.rng_state() == a.rng_state() and b.digest() == a.digest()
    # back to greedy: the captured sampled step is dropped
    b.sampling(0.0, 1.0, 0)
    b.spec_prefill(PROMPT)
    for _ in range(4):
        b.spec_step_async()
    greedy = gpu_model(gcuda, kw, W).greedy(PROMPT, 40)
    e = b.emitted()
    assert e == greedy[:len(e)]


def test_sampling_errors(gcuda, tiny):
    kw, W = tiny
    g = gpu_model(gcuda, kw, W, cap=32)
    with pytest.raises(gcuda.GcudaError, match="NaN"):
        g.sampling(float("nan"), 1.0, 0)
    import torch
    t = torch.zeros(8, dtype=torch.int16, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert gcuda.apus_gcuda_sample_rows_dev(gcuda.ptr(t), 1, 4, 8, 1.0, 1.0, 0, gcuda.ptr(out),
                                            gcuda.stream_of()) == -1   # ld < n
    gcuda.apus_gcuda_clear_error()
