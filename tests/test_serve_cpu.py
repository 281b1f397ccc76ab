"""The NDJSON serve loop (apus-glm5.3-flash_b200/serve.py, the `generate`
command of c/apus.c:644-875) on a stand-in engine, no GPU: the message
sequence, end ids, max_tokens, the sampling settings handed to the engine,
generation_config.json defaults, and the reference's error answers."""
import io
import json

import pytest

import serve as S


class FakeModel:
    """Emits `stream` in steps of `per_step` tokens, [] past its end (the
    engine at its KV capacity); records the calls."""

    def __init__(self, stream, per_step=3, fail=None):
        self.stream, self.per_step, self.fail = list(stream), per_step, fail
        self.calls = []

    def sampling(self, temp, top_p, seed):
        self.calls.append(("sampling", temp, top_p, seed))

    def spec_prefill(self, ids):
        if self.fail:
            raise RuntimeError(self.fail)
        self.calls.append(("prefill", list(ids)))
        self.pos = 0

    def spec_step(self):
        out = self.stream[self.pos:self.pos + self.per_step]
        self.pos += len(out)
        return out


def lines(server, reqs):
    fout = io.StringIO()
    server.run(io.StringIO("".join(json.dumps(r) + "\n" for r in reqs)), fout)
    return [json.loads(l) for l in fout.getvalue().splitlines()]


def test_generate_until_eos():
    m = FakeModel([5, 6, 7, 154820, 9, 10])
    out = lines(S.Server(m), [{"id": 1, "cmd": "generate", "ids": [1, 2, 3], "seed": 4, "temperature": 0.7}])
    assert out[0] == {"id": 1, "type": "prompt", "prompt_tokens": 3}
    assert [o["token_id"] for o in out[1:-1]] == [5, 6, 7]
    assert out[-1] == {"id": 1, "type": "done", "finish_reason": "stop", "prompt_tokens": 3,
                       "completion_tokens": 3, "text": ""}
    assert m.calls[0] == ("sampling", 0.7, 1.0, 4) and m.calls[1] == ("prefill", [1, 2, 3])


def test_max_tokens_and_capacity():
    m = FakeModel(range(100, 120))
    out = lines(S.Server(m), [{"id": "a", "cmd": "generate", "ids": [1], "max_tokens": 4}])
    assert [o["token_id"] for o in out if o["type"] == "token"] == [100, 101, 102, 103]
    assert out[-1]["finish_reason"] == "length" and out[-1]["completion_tokens"] == 4
    m = FakeModel([1, 2])                      # the engine stops emitting (KV capacity)
    out = lines(S.Server(m, eos=[99]), [{"id": 2, "cmd": "generate", "ids": [3]}])
    assert out[-1]["finish_reason"] == "length" and out[-1]["completion_tokens"] == 2
    out = lines(S.Server(FakeModel([1])), [{"id": 3, "cmd": "generate", "ids": [3], "max_tokens": 0}])
    assert [o["type"] for o in out] == ["prompt", "done"]


def test_errors():
    srv = S.Server(FakeModel([1]))
    out = lines(srv, [{"id": 1, "cmd": "generate", "text": "hi"}, {"id": 2, "cmd": "encode", "text": "x"},
                      {"id": 3, "cmd": "generate"}, {"id": 4, "cmd": "generate", "ids": []},
                      {"id": 5, "cmd": "generate", "ids": [1, "x"]}, {"id": 6, "cmd": "nope"}])
    msgs = [(o["id"], o["code"], o["message"]) for o in out]
    assert msgs == [(1, "bad_request", "no tokenizer in model dir"), (2, "bad_request", "no tokenizer in model dir"),
                    (3, "bad_request", "generate needs messages, text, or ids"), (4, "bad_request", "empty prompt"),
                    (5, "bad_request", "ids must be an array of numbers"),
                    (6, "bad_request", "unknown cmd (want encode|generate)")]
    assert srv.handle_line("[1, 2]") == [{"id": None, "type": "error", "code": "bad_request",
                                          "message": "bad request line (not a JSON object)"}]
    out = lines(S.Server(FakeModel([1], fail="capacity")), [{"id": 7, "cmd": "generate", "ids": [1]}])
    assert out[-1] == {"id": 7, "type": "error", "code": "engine_error", "message": "capacity"}


def test_generation_config(tmp_path):
    assert S.gen_config(str(tmp_path)) == (S.GLM_EOS_IDS, 1.0, 1.0)
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [7, 8], "temperature": 0.6,
                                                                 "top_p": 0.95}))
    assert S.gen_config(str(tmp_path)) == ((7, 8), 0.6, 0.95)
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": 5}))
    assert S.gen_config(str(tmp_path)) == ((5,), 1.0, 1.0)
    m = FakeModel([1, 2, 5, 3])
    eos, t, p = S.gen_config(str(tmp_path))
    out = lines(S.Server(m, eos, t, p), [{"id": 1, "cmd": "generate", "ids": [4]}])
    assert [o["token_id"] for o in out if o["type"] == "token"] == [1, 2]
    assert m.calls[0] == ("sampling", 1.0, 1.0, 0)
