"""The OpenThai request path of the front end (src/server.rs:235-331 over
src/models/openthai/decision.rs:234-390) on CPU: `OpenThaiService` around an
`openthai.Model` whose forward is the oracle's (the checker stands in for the
GPU here; the GPU forward itself is checked in test_gpu_openthai.py)."""
import io
import json

import numpy as np
import pytest

import oracle
from laya_goish_b200 import frontend, openthai, synth
from laya_goish_b200._lib import E_CUDA, LayaError
from laya_goish_b200.tokenizer import Tokenizer


@pytest.fixture(scope="module")
def served(tmp_path_factory):
    path = synth.write_openthai(str(tmp_path_factory.mktemp("ots") / "ot.gguf"), tokenizer=True, seed=4)
    w = openthai.load_weights(path, strict=False)
    m = object.__new__(openthai.Model)  # no device: the forward below is the oracle's
    m._h = None
    m.config = w["config"]
    m.temperature = w["temperature"]
    calls = []

    def forward(ids, positions):
        calls.append(len(ids))
        return oracle.ot_forward(w, ids, positions)

    m.forward = forward
    return m, Tokenizer.from_gguf(path), w, calls


REQ = {"state": {"ticket": "refund please", "n": 3},
       "questions": {"c": {"type": "choice", "instructions": "route",
                           "criteria": {"a": "billing", "b": None, "c": "other"}},
                     "s": {"type": "score", "instructions": "urgency", "criteria": ["low", "mid", "high"]},
                     "n": {"type": "noul", "instructions": "spam?"}},
       "order_invariant": True, "id": "r-1"}


def test_single_request_result_object(served):
    m, tok, w, calls = served
    svc = frontend.OpenThaiService(m, tok)
    calls.clear()
    r = svc.handle("POST", "/v1/decide", json.dumps(REQ))
    assert r.status == 200 and "X-Response-Time-Ms" in r.headers
    b = r.body
    assert b["model"] == "openthai-systemone" and b["id"] == "r-1" and "_raw" not in b
    u = b["usage"]
    assert u["permutations"] == 3 and u["output_tokens"] == 0 and u["truncated_state"] is False
    assert u["input_tokens"] == calls[0] and len(calls) == 3
    # the answers are the slot decoding of the oracle's passes
    qs = openthai.questions(REQ)
    passes = []
    for p in range(3):
        e = openthai.encode(tok, REQ, qs, 3, p, m.config["answer_token_id"], 512, 256)
        passes.append((oracle.ot_forward(w, e.ids, e.positions), e.order))
    want = openthai.decide(qs, passes, w["temperature"])
    assert json.loads(json.dumps(b["answers"])) == json.loads(json.dumps(want))
    assert set(b["answers"]["c"]["probabilities"]) == {"a", "b", "c"}
    assert sum(b["answers"]["c"]["probabilities"].values()) == pytest.approx(1.0, abs=1e-5)


def test_raw_output_and_batch(served):
    m, tok, _, _ = served
    svc = frontend.OpenThaiService(m, tok, raw=True)
    single = {"state": "hello there", "questions": {"n": {"type": "noul", "instructions": "greeting?"}}}
    r = svc.handle("POST", "/v1/decide", json.dumps(single))
    raw = r.body["_raw"]
    assert len(raw) == 1 and len(raw[0]["logits"]) == 256
    ids, pos = raw[0]["input_ids"], raw[0]["answer_positions"]
    assert ids[pos[0]] == m.config["answer_token_id"] and r.body["usage"]["input_tokens"] == len(ids)
    batch = {"states": ["hello there", {"x": 1}], "questions": single["questions"]}
    rb = svc.handle("POST", "/v1/decide/batch", json.dumps(batch))
    assert rb.status == 200 and len(rb.body["results"]) == 2
    assert rb.body["results"][0]["answers"] == r.body["answers"]
    assert rb.body["results"][1]["answers"] != r.body["answers"]


@pytest.mark.parametrize("body,msg", [
    ({"questions": REQ["questions"]}, "state is required"),
    ({"state": 5, "questions": REQ["questions"]}, "OpenThai state must be"),
    ({"state": "s", "questions": {"q": {"type": "rank", "instructions": ""}}}, "invalid question type"),
    ({"state": "s", "questions": REQ["questions"], "permutations": 0}, "permutations must be 1..32"),
    ({"state": "x" * 3000, "questions": {"q": {"type": "choice", "instructions": "y" * 2000,
                                              "criteria": {"a": None}}}}, "context budget"),
])
def test_validation_errors_are_422(served, body, msg):
    m, tok, _, calls = served
    svc = frontend.OpenThaiService(m, tok)
    calls.clear()
    r = svc.handle("POST", "/v1/decide", json.dumps(body))
    assert r.status == 422 and msg in r.body["error"]["message"] and not calls


def test_batch_limits(served):
    m, tok, _, calls = served
    svc = frontend.OpenThaiService(m, tok)
    qs = {f"q{i}": {"type": "noul", "instructions": ""} for i in range(130)}
    calls.clear()
    budget = m.config["max_tokens"]
    m.config["max_tokens"] = 8192  # room for 130 question blocks in one prompt
    try:
        r = svc.handle("POST", "/v1/decide/batch", json.dumps({"states": ["a", "b"], "questions": qs}))
    finally:
        m.config["max_tokens"] = budget
    assert r.status == 422 and "At most 256 total questions" in r.body["error"]["message"] and not calls
    r = svc.handle("POST", "/v1/decide/batch", json.dumps({"states": [], "questions": qs}))
    assert r.status == 422 and "1..256 states" in r.body["error"]["message"]
    # one bad state fails the whole batch before any pass runs
    r = svc.handle("POST", "/v1/decide/batch", json.dumps({"states": ["ok", 7], "questions": REQ["questions"]}))
    assert r.status == 422 and not calls


def test_cancel_busy_and_failures(served):
    m, tok, _, calls = served
    svc = frontend.OpenThaiService(m, tok)
    r = svc.handle("POST", "/v1/decide", json.dumps(REQ), canceled=lambda: True)
    assert r.status == 408 and r.body["error"]["type"] == "request_canceled"
    svc._busy.acquire()
    try:
        r = svc.handle("POST", "/v1/decide", json.dumps(REQ))
        assert r.status == 429 and r.headers["Retry-After"] == "1"
    finally:
        svc._busy.release()
    fwd = m.forward

    def broken(ids, positions):
        raise LayaError(E_CUDA, "device lost")

    m.forward = broken
    try:
        r = svc.handle("POST", "/v1/decide", json.dumps(REQ))
        assert r.status == 500 and r.body["error"]["message"] == "device lost"
    finally:
        m.forward = fwd
    h = svc.handle("GET", "/health", None).body
    assert h["model"] == "openthai-systemone" and h["layers"] == 4 and h["busy"] is False
    # the model key must name the loaded model (validation/test_openthai_http.py)
    r = svc.handle("POST", "/v1/decide", json.dumps(dict(REQ, model="laya")))
    assert r.status == 422 and r.body["error"]["message"] == "unknown model laya; see /v1/models"
    r = svc.handle("POST", "/v1/systemone", json.dumps(dict(REQ, model="openthai-systemone")))
    assert r.status == 200 and r.body["id"] == "r-1"
    with pytest.raises(ValueError, match="tokenizer"):
        frontend.OpenThaiService(m, None)


def test_daemon_lines(served):
    m, tok, _, _ = served
    svc = frontend.OpenThaiService(m, tok)
    out = io.StringIO()
    frontend.run_daemon(svc, io.StringIO(json.dumps(REQ) + "\n\n" + json.dumps({"state": 1}) + "\n"), out)
    lines = [json.loads(x) for x in out.getvalue().splitlines()]
    assert lines[0]["model"] == "openthai-systemone" and "error" in lines[1]
    assert np.isfinite(lines[0]["answers"]["s"]["score"])


def _model_like(m, forward):
    c = object.__new__(openthai.Model)
    c._h = None
    c.config, c.temperature = m.config, m.temperature
    c.forward = forward
    return c


def test_batch_shared_over_several_models(served):
    import threading
    import time

    m, tok, w, _ = served
    used = {}

    def on(k):
        def forward(ids, positions):
            used.setdefault(k, 0)
            used[k] += 1
            time.sleep(0.02)
            return oracle.ot_forward(w, ids, positions)
        return forward

    models = [_model_like(m, on(0)), _model_like(m, on(1))]
    batch = {"states": ["a", {"b": 1}, "ccc", "d d", ["e"]], "questions": REQ["questions"], "order_invariant": True}
    one = frontend.OpenThaiService(m, tok).handle("POST", "/v1/decide/batch", json.dumps(batch))
    two = frontend.OpenThaiService(models, tok).handle("POST", "/v1/decide/batch", json.dumps(batch))
    assert one.status == two.status == 200
    strip = [{k: v for k, v in r.items() if k != "usage"} for r in one.body["results"]]
    assert strip == [{k: v for k, v in r.items() if k != "usage"} for r in two.body["results"]]
    assert set(used) == {0, 1} and sum(used.values()) == 5 * 3
    # a failure on one device fails the batch and stops the other
    stop = threading.Event()

    def broken(ids, positions):
        stop.set()
        raise LayaError(E_CUDA, "device lost")

    r = frontend.OpenThaiService([_model_like(m, on(0)), _model_like(m, broken)], tok).handle(
        "POST", "/v1/decide/batch", json.dumps(batch))
    assert r.status == 500 and r.body["error"]["message"] == "device lost" and stop.is_set()
    r = frontend.OpenThaiService(models, tok).handle("POST", "/v1/decide/batch", json.dumps(batch),
                                                    canceled=lambda: True)
    assert r.status == 408


def test_non_library_failure_on_one_device_fails_the_batch(served):
    # A worker's exception that is not a LayaError (here a RuntimeError from
    # one model's forward on the third state) still stops the other worker
    # and maps to 500, never a 200 with missing results.
    import threading

    m, tok, w, _ = served
    seen = []
    lock = threading.Lock()

    def flaky(ids, positions):
        with lock:
            seen.append(1)
            n = len(seen)
        if n == 3:
            raise RuntimeError("numpy blew up")
        return oracle.ot_forward(w, ids, positions)

    batch = {"states": ["a", "b", "c", "d", "e", "f"], "questions": REQ["questions"], "order_invariant": True}
    models = [_model_like(m, flaky), _model_like(m, flaky)]
    r = frontend.OpenThaiService(models, tok).handle("POST", "/v1/decide/batch", json.dumps(batch))
    assert r.status == 500 and "numpy blew up" in r.body["error"]["message"]
    assert len(seen) < 6 * 3  # the batch stopped early


def test_model_without_gpu_fails_cleanly(tmp_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    path = synth.write_openthai(str(tmp_path / "ot.gguf"), d=128, ffn=256, hd=64, lin_dim=64)
    with pytest.raises(openthai.OpenThaiError, match="unsupported OpenThai config"):
        openthai.Model(path)  # the reference's one size only, unless strict=False
    with pytest.raises(LayaError):
        openthai.Model(path, strict=False)
    m = object.__new__(openthai.Model)
    m._h = None
    with pytest.raises(openthai.OpenThaiError, match="closed"):
        openthai.Model.forward(m, [1, 2], [1])
