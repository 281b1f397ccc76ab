"""The speculative step's decisions and drafts against the oracle.

  * Accept walk, bitwise: the engine keeps each step's verify-row logits
    (apus_gcuda_gspec_keep_logits); the oracle's walk (orc_spec_walk, the
    walk of c/gmtp.h:807-831 that orc_spec_step runs, itself pinned bitwise
    to the reference engine's apus_gspec_step) replays it on those logits
    and the drafts the step verified.  Emitted tokens, the matched count,
    the next held token and the new position must be equal.
  * Drafts: the engine's MTP chain (replay of the step's candidate pairs,
    then depth-1 chained forwards) against the oracle's speculative loop
    (replay of the accepted prefix after the walk, then the chain,
    c/gmtp.h:851-884 and :677-696) on the same prompt, with the same forced
    agreement (truth with probability p, else truth+1, keyed by splitmix64
    of the seed and the position).  The MTP's own drafts, before the
    forcing, must be equal wherever the oracle's pick is not a near tie
    (relative top-2 margin above a per-dims MARGIN); the emitted streams must be equal
    up to the first position where the two engines' greedy picks may
    differ (a near tie of the oracle's logits).  Seeded extra prompts run
    until at least depth - 1 drafts were compared away from near ties.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import synth
from modelgen import gen_weights, tiny_config

pytestmark = pytest.mark.gpu

PROMPT = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]
# near-tie margins: a few times the relative error of the MTP logits at the
# dims, grown over a loop in which both engines' MTP caches drift apart
# (tiny model: cosine 0.999, up to 5 % of the row max per forward;
# config-2 dims: relative L2 about 1e-2)
MARGIN_TINY, MARGIN_C2 = 0.2, 0.04
M64 = (1 << 64) - 1


def sm64(z):
    """splitmix64's output function on z (the forced-agreement hash of
    apus_gcuda_gspec_force)."""
    z = (z + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def force_rule(truth, base, p, seed, V):
    def hook(ctx, q, drafts, n):
        for i in range(n):
            pos = q + i - base
            if 0 <= pos < len(truth):
                u = (sm64((seed ^ (q + i)) & M64) >> 11) * 2.0 ** -53
                drafts[i] = truth[pos] if u < p else (truth[pos] + 1) % V
    return O.DRAFT_HOOK(hook)


@pytest.fixture(scope="module")
def tiny():
    kw = tiny_config()
    return kw, gen_weights(kw, seed=20261201)


def walk_steps(g, depth, V, n_steps):
    """Run n_steps engine steps with logits kept; replay each on the oracle
    walk and compare."""
    g.keep_logits(True)
    for _ in range(n_steps):
        s0, rc = g.stats()
        assert rc == 0
        drafts = g.debug_read("drafts", (depth,), np.int32)
        out = g.spec_step()
        s1, _ = g.stats()
        logits = g.debug_read("logits", (depth, V), np.uint16)
        emitted, matched, nh = O.spec_walk(logits, drafts.tolist(), s0["held"])
        assert out == emitted, (out, emitted)
        assert len(out) == matched + 1
        assert s1["held"] == nh
        assert s1["pos"] == s0["pos"] + matched + 1
        assert s1["accepted"] - s0["accepted"] == matched
    g.keep_logits(False)


@pytest.mark.parametrize("p", [0.0, 0.5, 1.0])
def test_walk_bitwise_on_device_logits(gcuda, tiny, p):
    kw, W = tiny
    depth, V = 4, kw["vocab_size"]
    ref = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=256, depth=depth)
    ref.load(W)
    truth = ref.greedy(PROMPT, 80)
    ref.close()
    g = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=256, depth=depth)
    g.load(W)
    g.force(truth, base=len(PROMPT), p=p, seed=9)
    g.spec_prefill(PROMPT)
    walk_steps(g, depth, V, 14)
    g.close()


def draft_parity(gcuda, kw, W, depth, p, n_steps, cap, margin, prompt=PROMPT):
    """Drafts compared on one prompt: (drafts compared away from a near tie,
    drafts equal)."""
    V = kw["vocab_size"]
    # the oracle's own greedy stream is the truth the forcing uses on both sides
    o = O.Model(O.make_config(**kw), W, True, "orc")
    truth = np.zeros(n_steps * depth + 8, np.int32)
    ids = np.array(prompt, np.int32)
    st0 = o.state(cap)
    assert O.ORC.orc_greedy(o.h, st0, O.p(ids), len(ids), len(truth), O.p(truth)) == 0
    O.ORC.orc_state_free(st0)
    truth = truth.tolist()
    seed = 31
    st, mst = o.state(cap), O.ORC.orc_mtp_state_new(o.h, cap)
    sp = O.ORC.orc_spec_new(o.h, st, mst, depth)
    hook = force_rule(truth, len(prompt), p, seed, V)
    O.ORC.orc_spec_set_force_hook(sp, hook, None)
    g = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=cap, depth=depth)
    g.load(W)
    g.keep_logits(True)
    g.force(truth, base=len(prompt), p=p, seed=seed)
    assert O.ORC.orc_spec_prefill(sp, O.p(ids), len(ids)) == 0
    g.spec_prefill(prompt)
    raw_o = np.zeros(depth, np.int32)
    marg = np.zeros(depth, np.float32)
    buf = (C.c_int * (depth + 1))()
    checked = agreed = 0
    for step in range(n_steps + 1):
        O.ORC.orc_spec_raw_drafts(sp, O.p(raw_o), O.p(marg))
        raw_g = g.debug_read("raw_drafts", (depth,), np.int32)
        print(f"step {step}: engine drafts {raw_g.tolist()}, oracle {raw_o.tolist()}, "
              f"oracle margins {[round(float(x), 4) for x in marg]}")
        # each chain draft feeds the next chain step: after the first
        # difference (only allowed at a near tie) the rest of the chain
        # starts from other tokens and is not comparable
        for i in range(depth):
            if raw_g[i] != raw_o[i]:
                assert marg[i] <= margin, f"step {step} draft {i}: engine {raw_g[i]}, oracle {raw_o[i]} " \
                                          f"(margin {marg[i]:.3g})"
                break
            checked += int(marg[i] > margin)
            agreed += 1
        q = g.stats()[0]["pos"]
        assert g.debug_read("drafts", (depth,), np.int32).tolist() == \
            O_forced(truth, len(prompt), p, seed, V, q, raw_g)
        if step == n_steps:
            break
        ne = O.ORC.orc_spec_step(sp, buf, depth + 1)
        out_o = list(buf[:ne])
        out_g = g.spec_step()
        if out_g != out_o:
            # the two engines' greedy streams split (a near tie of the main
            # model's logits): the drafts after it are not comparable.  Token
            # i >= 1 of a step is draft i accepted on verify row i-1's pick, so
            # the rows disagree at k = (first differing token) - 1, or at the
            # last row of the shorter step when one is a prefix of the other;
            # the engine's own pick there must be a near tie (token 0 is the
            # previous step's last pick, checked no further)
            diff = [i for i in range(min(len(out_g), len(out_o))) if out_g[i] != out_o[i]]
            k = diff[0] - 1 if diff else min(len(out_g), len(out_o)) - 1
            if k >= 0:
                row = O.f32_of(g.debug_read("logits", (depth, V), np.uint16)[k]).astype(np.float64)
                top = np.sort(row)
                tie = (top[-1] - top[-2]) / max(abs(top[-1]), 1e-30)   # the oracle's top2_margin
                assert tie <= margin, f"streams split at verify row {k} away from a near tie ({tie:.3g})"
            break
    O.ORC.orc_spec_free(sp)
    O.ORC.orc_mtp_state_free(mst)
    O.ORC.orc_state_free(st)
    g.close()
    return checked, agreed


def draft_parity_prompts(gcuda, kw, W, depth, p, n_steps, cap, margin, n_prompts):
    """draft_parity over the fixed prompt and seeded random ones until at
    least depth - 1 drafts were compared away from near ties (a run ends where
    the two engines' greedy streams split at a near tie, which may come early)."""
    rng = np.random.default_rng(20261208)
    prompts = [PROMPT] + [rng.integers(0, kw["vocab_size"], 11 + 4 * i).tolist() for i in range(n_prompts - 1)]
    checked = agreed = 0
    for pr in prompts:
        c, a = draft_parity(gcuda, kw, W, depth, p, n_steps, cap, margin, pr)
        checked, agreed = checked + c, agreed + a
        if checked >= depth - 1:
            break
    assert checked >= depth - 1, f"only {checked} drafts compared away from near ties"
    print(f"{agreed} drafts equal, {checked} of them away from near ties")


def O_forced(truth, base, p, seed, V, q, drafts):
    """The forced drafts the engine verifies next: its own raw drafts edited
    by the forcing rule at position q."""
    out = [int(x) for x in drafts]
    for i in range(len(out)):
        pos = q + i - base
        if 0 <= pos < len(truth):
            u = (sm64((seed ^ (q + i)) & M64) >> 11) * 2.0 ** -53
            out[i] = truth[pos] if u < p else (truth[pos] + 1) % V
    return out


@pytest.mark.parametrize("p", [0.0, 0.5])
def test_drafts_vs_oracle_tiny(gcuda, tiny, p):
    kw, W = tiny
    draft_parity_prompts(gcuda, kw, W, depth=4, p=p, n_steps=16, cap=256, margin=MARGIN_TINY, n_prompts=4)


def test_drafts_vs_oracle_config2_dims(gcuda):
    kw = synth.c2_config(small=True)
    W = synth.c2_weights(kw, seed=20261203)
    draft_parity_prompts(gcuda, kw, W, depth=4, p=0.5, n_steps=6, cap=128, margin=MARGIN_C2, n_prompts=3)
