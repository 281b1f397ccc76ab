"""The NDJSON serve loop on the B200 engine (tiny model): a greedy
`generate` streams the engine's greedy tokens and stops at an end id; a
sampled one streams the engine's own sampled stream for the seed."""
import io
import json

import pytest

import serve as S
from modelgen import gen_weights, tiny_config

pytestmark = pytest.mark.gpu
PROMPT = [5, 17, 300, 2, 99, 42, 7, 381, 0, 11, 13]


@pytest.fixture(scope="module")
def tiny():
    kw = tiny_config()
    return kw, gen_weights(kw, seed=20261201)


def model(gcuda, kw, W):
    m = gcuda.GModel(gcuda.make_config(**kw), has_mtp=True, kv_cap=128, depth=4)
    m.load(W)
    m.use_graph(True)
    return m


def serve(srv, req):
    fout = io.StringIO()
    srv.run(io.StringIO(json.dumps(req) + "\n"), fout)
    return [json.loads(l) for l in fout.getvalue().splitlines()]


def test_serve_greedy_and_eos(gcuda, tiny):
    kw, W = tiny
    greedy = model(gcuda, kw, W).greedy(PROMPT, 20)
    srv = S.Server(model(gcuda, kw, W), eos=[10 ** 6])
    out = serve(srv, {"id": 1, "cmd": "generate", "ids": PROMPT, "max_tokens": 20, "temperature": 0})
    assert [o["token_id"] for o in out if o["type"] == "token"] == greedy
    assert out[-1]["finish_reason"] == "length" and out[-1]["completion_tokens"] == 20
    eos = greedy[6]
    stop = greedy.index(eos)
    srv = S.Server(model(gcuda, kw, W), eos=[eos])
    out = serve(srv, {"id": 2, "cmd": "generate", "ids": PROMPT, "max_tokens": 20, "temperature": 0})
    assert [o["token_id"] for o in out if o["type"] == "token"] == greedy[:stop]
    assert out[-1]["finish_reason"] == "stop"


def test_serve_sampled_equals_engine_stream(gcuda, tiny):
    kw, W = tiny
    ref = model(gcuda, kw, W)
    ref.sampling(0.8, 0.95, 12345)
    want = ref.generate(PROMPT, 15)
    srv = S.Server(model(gcuda, kw, W), eos=[10 ** 6])
    out = serve(srv, {"id": 3, "cmd": "generate", "ids": PROMPT, "max_tokens": 15, "temperature": 0.8,
                      "top_p": 0.95, "seed": 12345})
    assert [o["token_id"] for o in out if o["type"] == "token"] == want
