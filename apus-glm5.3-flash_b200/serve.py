"""NDJSON serve loop over the B200 engine: the `generate` command of the
reference's `apus serve` (c/apus.c:644-875) on the speculative path, token
ids in and out (the tokenizer is not part of this engine).

Protocol (one JSON object per line on stdin, responses on stdout), as the
reference:
  {"id": X, "cmd": "generate", "ids": [...], "max_tokens": N,
   "temperature": T, "top_p": P, "seed": S}
    -> {"id": X, "type": "prompt", "prompt_tokens": n}
    -> {"id": X, "type": "token", "token_id": t}            per emitted token
    -> {"id": X, "type": "done", "finish_reason": "stop"|"length",
        "prompt_tokens": n, "completion_tokens": m, "text": ""}
  errors: {"id": X, "type": "error", "code": "bad_request"|"engine_error",
           "message": ...}
Sampling defaults and the end-of-sequence set come from the container's
generation_config.json (c/apus.c:250-287): eos_token_id (a number or a
list), temperature and top_p, else GLM's end ids {154820, 154827, 154829}
and 1.0 / 1.0.  max_tokens absent means until an end id (bounded by
APUS_GSERVE_MAX_TOKENS, default 65536, c/apus.c:653-655).  Requests carrying
"text" or "messages", and "encode", need the tokenizer and answer as the
reference does without one.  The engine's KV capacity is fixed when it is
created: a request that reaches it ends with "length".

Usage: python serve.py --model CONTAINER_DIR [--spec-k K] [--kv-cap N]
"""
import json
import os
import sys

GLM_EOS_IDS = (154820, 154827, 154829)


def gen_config(model_dir):
    """(eos ids, default temperature, default top_p) of a container
    (c/apus.c:256-287)."""
    eos, temp, top_p = [], 1.0, 1.0
    path = os.path.join(model_dir, "generation_config.json") if model_dir else None
    if path and os.path.exists(path):
        try:
            gc = json.load(open(path))
        except ValueError:
            gc = None
        if isinstance(gc, dict):
            v = gc.get("eos_token_id")
            if isinstance(v, (int, float)) and not isinstance(v, bool):
                eos = [int(v)]
            elif isinstance(v, list):
                eos = [int(x) for x in v if isinstance(x, (int, float)) and not isinstance(x, bool)][:8]
            if isinstance(gc.get("temperature"), (int, float)):
                temp = float(gc["temperature"])
            if isinstance(gc.get("top_p"), (int, float)):
                top_p = float(gc["top_p"])
    return tuple(eos or GLM_EOS_IDS), temp, top_p


def _num(v):
    return isinstance(v, (int, float)) and not isinstance(v, bool)


class Server:
    """Serves requests on one resident model (apus_gcuda.GModel or any
    object with sampling / spec_prefill / spec_step)."""

    def __init__(self, model, eos=GLM_EOS_IDS, temperature=1.0, top_p=1.0):
        self.model, self.eos = model, set(int(e) for e in eos)
        self.temperature, self.top_p = temperature, top_p

    @staticmethod
    def _resp(rid, typ, **kw):
        d = {"id": rid, "type": typ}
        d.update(kw)
        return d

    def _error(self, rid, msg, code="bad_request"):
        return self._resp(rid, "error", code=code, message=msg)

    def handle_line(self, line):
        """All responses to one request line, in order."""
        try:
            req = json.loads(line)
        except ValueError:
            req = None
        if not isinstance(req, dict):
            return [self._error(None, "bad request line (not a JSON object)")]
        rid, cmd = req.get("id"), req.get("cmd")
        if cmd == "encode":
            return [self._error(rid, "no tokenizer in model dir")]
        if cmd != "generate":
            return [self._error(rid, "unknown cmd (want encode|generate)")]
        return list(self.generate(req))

    def generate(self, req):
        rid = req.get("id")
        ids = req.get("ids")
        if isinstance(ids, list):
            if not all(_num(v) for v in ids):
                yield self._error(rid, "ids must be an array of numbers")
                return
            ids = [int(v) for v in ids]
        elif isinstance(req.get("text"), str) or "messages" in req:
            yield self._error(rid, "no tokenizer in model dir")
            return
        else:
            yield self._error(rid, "generate needs messages, text, or ids")
            return
        if not ids:
            yield self._error(rid, "empty prompt")
            return
        max_tokens = int(req["max_tokens"]) if _num(req.get("max_tokens")) else \
            int(os.environ.get("APUS_GSERVE_MAX_TOKENS", "65536"))
        max_tokens = max(max_tokens, 0)
        temp = float(req["temperature"]) if _num(req.get("temperature")) else self.temperature
        top_p = float(req["top_p"]) if _num(req.get("top_p")) else self.top_p
        seed = int(req["seed"]) if _num(req.get("seed")) else 0
        yield self._resp(rid, "prompt", prompt_tokens=len(ids))
        completion, finish = 0, "length"
        try:
            self.model.sampling(temp, top_p, seed)
            self.model.spec_prefill(ids)
            done = False
            while completion < max_tokens and not done:
                emitted = self.model.spec_step()
                if not emitted:
                    break                      # the KV capacity is reached
                for t in emitted:
                    if completion >= max_tokens:
                        break
                    if t in self.eos:
                        finish, done = "stop", True
                        break
                    completion += 1
                    yield self._resp(rid, "token", token_id=int(t))
        except Exception as e:  # noqa: BLE001 - every engine failure is reported, as the reference does
            yield self._error(rid, str(e), code="engine_error")
            return
        yield self._resp(rid, "done", finish_reason=finish, prompt_tokens=len(ids), completion_tokens=completion,
                         text="")

    def run(self, fin=sys.stdin, fout=sys.stdout):
        for line in fin:
            if not line.strip():
                continue
            for r in self.handle_line(line):
                fout.write(json.dumps(r) + "\n")
                fout.flush()


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", required=True, help="weight container directory (config.json + safetensors)")
    ap.add_argument("--spec-k", type=int, default=int(os.environ.get("APUS_SPEC_K", "3")))
    ap.add_argument("--kv-cap", type=int, default=65536)
    args = ap.parse_args(argv)
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import apus_gcuda as G
    G.enable()
    cfg = G.config_load(os.path.join(args.model, "config.json"))
    m = G.GModel(cfg, has_mtp=cfg.num_nextn_predict_layers > 0, kv_cap=args.kv_cap, depth=args.spec_k)
    m.load_container(args.model)
    m.use_graph(True)
    eos, temp, top_p = gen_config(args.model)
    Server(m, eos, temp, top_p).run()


if __name__ == "__main__":
    main()
