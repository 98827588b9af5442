"""The batch front end over the real engine: a /v1/decide/batch body gives the
answers of one direct decide_batch call, in request order."""
import json

import numpy as np
import pytest

from laya_goish_b200 import engine, frontend, synth
from laya_goish_b200.engine import Question

pytestmark = pytest.mark.gpu


def test_batch_endpoint_matches_engine(tiny_paths):
    path = tiny_paths["tiny-llama-q8_0"]
    rng = np.random.default_rng(21)
    states = [synth.token_ids(rng, 1000, int(n)).tolist() for n in (12, 70, 33, 5)]
    q = {"pick": {"type": "choice", "criteria": {"x": 11, "y": 12, "z": 13}, "suffix": [7, 8]},
         "lvl": {"type": "score", "criteria": [[3, 4], [5, 6], [7, 9]]},
         "ok": {"type": "noul", "criteria": {"false": 21, "true": 22}}}
    with engine.Engine(path) as e:
        svc = frontend.DecideService(e, raw=True)
        r = svc.handle("POST", "/v1/decide/batch", json.dumps({"states": states, "questions": q}).encode())
        assert r.status == 200, r.body
        direct = e.decide_batch(states, [Question("choice", [11, 12, 13], [7, 8]),
                                         Question("score", [[3, 4], [5, 6], [7, 9]]),
                                         Question("noul", [21, 22])])
        bad = svc.handle("POST", "/v1/decide/batch", json.dumps({"states": states + [[1, 5000]], "questions": q}))
        assert bad.status == 422
    res = r.body["results"]
    assert len(res) == len(states)
    for i in range(len(states)):
        a = res[i]["answers"]
        d = direct[i]
        assert a["pick"]["choice"] == "xyz"[d[0]["choice"]]
        assert np.allclose(list(a["pick"]["probabilities"].values()), d[0]["probabilities"])
        assert a["lvl"]["score"] == pytest.approx(d[1]["score"])
        assert a["ok"]["noul"] == pytest.approx(d[2]["noul"])
        assert a["ok"]["logits"] == pytest.approx(d[2]["logits"])


def test_text_state_matches_token_ids(tiny_paths):
    from laya_goish_b200.tokenizer import Tokenizer

    path = tiny_paths["tiny-llama-q8_0-tok"]
    tok = Tokenizer.from_gguf(path)
    text = "hello world, the email is urgent. answer yes or no"
    q_text = {"ok": {"type": "noul", "criteria": {"false": "no", "true": "yes"}, "suffix": " answer"}}
    q_ids = {"ok": {"type": "noul", "criteria": {"false": tok.encode("no"), "true": tok.encode("yes")},
                    "suffix": tok.encode(" answer")}}
    with engine.Engine(path) as e:
        svc = frontend.DecideService(e, tokenizer=tok)
        a = svc.handle("POST", "/v1/decide", json.dumps({"state": text, "questions": q_text}))
        b = svc.handle("POST", "/v1/decide", json.dumps({"state": tok.encode(text), "questions": q_ids}))
    assert a.status == 200 and b.status == 200
    assert a.body["answers"] == b.body["answers"]


def test_batch_endpoint_matches_oracle(tiny_paths):
    # The served answers against the oracle's decide (the reference's
    # decision rules on its CPU forward), not only against the same engine.
    import oracle

    path = tiny_paths["tiny-llama-q4_k_m"]
    rng = np.random.default_rng(22)
    states = [synth.token_ids(rng, 1000, int(n)).tolist() for n in (9, 64, 130)]
    q = {"pick": {"type": "choice", "criteria": {"a": 31, "b": 32, "c": 33, "d": 34}},
         "lvl": {"type": "score", "criteria": [[3, 4, 5], [6, 7, 8]], "suffix": [40, 41]},
         "ok": {"type": "noul", "criteria": {"false": 51, "true": 52}, "suffix": [9]}}
    with engine.Engine(path) as e:
        svc = frontend.DecideService(e)
        r = svc.handle("POST", "/v1/decide/batch", json.dumps({"states": states, "questions": q}))
    assert r.status == 200, r.body
    o = oracle.Model(open(path, "rb").read(), threads=4, attn_threads=4)
    for st, res in zip(states, r.body["results"]):
        a = res["answers"]
        pick = o.decide(st, 0, [31, 32, 33, 34])
        lvl = o.decide(st, 1, [[3, 4, 5], [6, 7, 8]], suffix=[40, 41])
        ok = o.decide(st, 2, [51, 52], suffix=[9])
        assert np.allclose(list(a["pick"]["probabilities"].values()), pick["probabilities"], atol=1e-3, rtol=1e-2)
        if sorted(pick["probabilities"])[-1] - sorted(pick["probabilities"])[-2] > 2e-3:
            assert a["pick"]["choice"] == "abcd"[pick["choice"]]
        assert a["lvl"]["score"] == pytest.approx(lvl["score"], abs=2e-3)
        assert a["ok"]["noul"] == pytest.approx(ok["noul"], abs=1e-3, rel=1e-2)
    o.close()
