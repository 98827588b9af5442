"""Host logic of the batch front end (src/server.rs:65-332, src/main.rs:139-151)
against a fake engine: routes, validation order, busy, cancel, errors, order."""
import io
import json
import threading

import pytest

from laya_goish_b200 import frontend
from laya_goish_b200._lib import E_CANCELED, E_CUDA, E_INVALID, LayaError


class FakeEngine:
    """Answers choice with the option whose first token id is largest."""

    info = {"architecture": "llama"}

    def __init__(self, vocab=1000):
        self.vocab = vocab
        self.calls = []
        self.gate = None
        self.fail = None

    def layers(self):
        return 2

    def validate(self, prompts, questions):
        for p in prompts:
            if any(t < 0 or t >= self.vocab for t in p):
                raise LayaError(E_INVALID, "token id out of range")

    def decide_batch(self, prompts, questions, canceled=None):
        self.calls.append((len(prompts), len(questions)))
        if self.gate:
            self.gate.wait(5)
        if canceled and canceled():
            raise LayaError(E_CANCELED, "request canceled")
        if self.fail:
            raise LayaError(self.fail, "boom")
        out = []
        for p in prompts:
            row = []
            for q in questions:
                _, opts, _ = q.arrays()
                k = opts.shape[0]
                best = int(max(range(k), key=lambda i: (opts[i, 0] + p[0]) % 7))
                probs = [0.0] * k
                probs[best] = 1.0
                row.append({"type": q.kind, "probabilities": probs, "logits": [float(i) for i in range(k)],
                            "confidence": 1.0, "choice": best, "score": float(best), "noul": probs[-1]})
            out.append(row)
        return out


CHOICE = {"pick": {"type": "choice", "criteria": {"a": 5, "b": 6, "c": 7}}}


def body(**kw):
    return json.dumps(kw).encode()


def test_routes_and_methods():
    s = frontend.DecideService(FakeEngine())
    assert s.handle("GET", "/nope", None).status == 404
    r = s.handle("GET", "/v1/decide", None)
    assert r.status == 405 and r.headers["Allow"] == "POST"
    assert s.handle("POST", "/health", b"").status == 405
    r = s.handle("GET", "/health", None)
    assert r.status == 200 and r.body["status"] == "ok"
    assert r.headers["X-Request-Id"].startswith("laya-")


def test_bad_json_and_validation():
    s = frontend.DecideService(FakeEngine())
    assert s.handle("POST", "/v1/decide", b"{").status == 400
    r = s.handle("POST", "/v1/decide", body(questions=CHOICE))
    assert r.status == 422 and "state" in r.body["error"]["message"]
    r = s.handle("POST", "/v1/decide", body(state=[1, 2], questions={"q": {"type": "bogus"}}))
    assert r.status == 422 and "type must be" in r.body["error"]["message"]
    r = s.handle("POST", "/v1/decide", body(state=[1, 2], questions={"q": {"type": "score", "criteria": [1]}}))
    assert r.status == 422
    r = s.handle("POST", "/v1/decide", body(state=[1, 2], questions={"q": {"type": "noul", "criteria": {"true": 3}}}))
    assert r.status == 422
    r = s.handle("POST", "/v1/decide", body(state=[1, 2],
                                           questions={"q": {"type": "choice", "criteria": {"a": 1, "b": [2, 3]}}}))
    assert r.status == 422 and "same number of tokens" in r.body["error"]["message"]
    r = s.handle("POST", "/v1/decide", body(state=[1, 5000], questions=CHOICE))
    assert r.status == 422 and "out of range" in r.body["error"]["message"]
    many = {f"q{i}": {"type": "choice", "criteria": {"a": 1, "b": 2}} for i in range(257)}
    assert s.handle("POST", "/v1/decide", body(state=[1], questions=many)).status == 422


def test_batch_validates_everything_first():
    eng = FakeEngine()
    s = frontend.DecideService(eng)
    assert s.handle("POST", "/v1/decide/batch", body(states=[], questions=CHOICE)).status == 422
    assert s.handle("POST", "/v1/decide/batch", body(states=[[1]] * 257, questions=CHOICE)).status == 422
    # one bad state anywhere fails the batch before any inference
    r = s.handle("POST", "/v1/decide/batch", body(states=[[1, 2], [3], [9999]], questions=CHOICE))
    assert r.status == 422 and eng.calls == []
    # 2 questions x 129 states > 256
    two = {"x": CHOICE["pick"], "y": CHOICE["pick"]}
    r = s.handle("POST", "/v1/decide/batch", body(states=[[1]] * 129, questions=two))
    assert r.status == 422 and "256" in r.body["error"]["message"] and eng.calls == []


def test_batch_answers_in_order_one_call():
    eng = FakeEngine()
    s = frontend.DecideService(eng)
    states = [[i, 2, 3] for i in range(10)]
    r = s.handle("POST", "/v1/decide/batch", body(states=states, questions=CHOICE))
    assert r.status == 200 and eng.calls == [(10, 1)]
    assert "X-Response-Time-Ms" in r.headers
    res = r.body["results"]
    assert len(res) == 10
    for i, st in enumerate(states):
        want = max(range(3), key=lambda k: ([5, 6, 7][k] + st[0]) % 7)
        a = res[i]["answers"]["pick"]
        assert a["choice"] == "abc"[want]
        assert set(a["probabilities"]) == {"a", "b", "c"}
        assert res[i]["usage"]["tokens"] == 3


def test_score_and_noul_shapes():
    s = frontend.DecideService(FakeEngine(), raw=True)
    q = {"s": {"type": "score", "criteria": [[4, 5], [6, 7], [8, 9]]},
         "n": {"type": "noul", "criteria": {"false": 3, "true": 4}, "suffix": [1, 2]}}
    r = s.handle("POST", "/v1/decide", body(state={"ids": [1, 2]}, questions=q))
    assert r.status == 200
    a = r.body["answers"]
    assert set(a["s"]) >= {"score", "legend", "confidence", "probabilities", "logits"}
    assert a["s"]["legend"] == {"0": [4, 5], "1": [6, 7], "2": [8, 9]}
    assert set(a["n"]["probabilities"]) == {"false", "true"} and "noul" in a["n"]
    assert r.body["usage"]["tokens"] == 2 + 4


def test_busy_cancel_and_internal_errors():
    eng = FakeEngine()
    s = frontend.DecideService(eng)
    eng.gate = threading.Event()
    first = {}
    t = threading.Thread(target=lambda: first.update(r=s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE))))
    t.start()
    for _ in range(500):
        if eng.calls:
            break
        threading.Event().wait(0.01)
    r = s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE))
    assert r.status == 429 and r.headers["Retry-After"] == "1" and r.body["error"]["type"] == "busy_error"
    eng.gate.set()
    t.join()
    assert first["r"].status == 200
    eng.gate = None
    r = s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE), canceled=lambda: True)
    assert r.status == 408 and r.body["error"]["type"] == "request_canceled"
    eng.fail = E_CUDA
    r = s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE))
    assert r.status == 500 and r.body["error"]["type"] == "internal_error"
    eng.fail = None
    assert s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE)).status == 200  # busy flag released


def test_daemon_lines():
    s = frontend.DecideService(FakeEngine())
    inp = io.StringIO(json.dumps({"state": [1, 2], "questions": CHOICE}) + "\n\n{bad\n" +
                      json.dumps({"state": [1], "questions": {"q": {"type": "x"}}}) + "\n")
    out = io.StringIO()
    frontend.run_daemon(s, inp, out)
    lines = [json.loads(x) for x in out.getvalue().splitlines()]
    assert len(lines) == 3
    assert "answers" in lines[0]
    assert "error" in lines[1] and "error" in lines[2]
    # the daemon hands each line to the model: a `model` key is not checked
    out = io.StringIO()
    frontend.run_daemon(s, io.StringIO(json.dumps({"state": [1, 2], "questions": CHOICE, "model": "x"}) + "\n"), out)
    assert "answers" in json.loads(out.getvalue())


def test_http_round_trip():
    import urllib.error
    import urllib.request

    srv = frontend.make_server(frontend.DecideService(FakeEngine()), "127.0.0.1", 0)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    try:
        url = f"http://127.0.0.1:{srv.server_address[1]}"
        req = urllib.request.Request(url + "/v1/decide/batch", data=body(states=[[1], [2]], questions=CHOICE),
                                     method="POST", headers={"Content-Type": "application/json; charset=utf-8"})
        with urllib.request.urlopen(req, timeout=10) as r:
            assert r.status == 200
            assert r.headers["Content-Type"].startswith("application/json")
            assert len(json.loads(r.read())["results"]) == 2
        with pytest.raises(urllib.error.HTTPError) as e:
            urllib.request.urlopen(url + "/missing", timeout=10)
        assert e.value.code == 404
        # no JSON content type: 415 (src/server.rs:175-189)
        with pytest.raises(urllib.error.HTTPError) as e:
            urllib.request.urlopen(urllib.request.Request(url + "/v1/decide", data=b"{}", method="POST"), timeout=10)
        assert e.value.code == 415
    finally:
        srv.shutdown()
        srv.server_close()


def _raw_http(port, head: bytes, chunks) -> tuple[int, dict]:
    import socket

    with socket.create_connection(("127.0.0.1", port), timeout=10) as c:
        c.sendall(head)
        for ch in chunks:
            c.sendall(b"%x\r\n" % len(ch) + ch + b"\r\n")
        c.sendall(b"0\r\n\r\n")
        data = b""
        while b"\r\n\r\n" not in data:
            data += c.recv(65536)
        h, rest = data.split(b"\r\n\r\n", 1)
        n = int([x for x in h.split(b"\r\n") if x.lower().startswith(b"content-length")][0].split(b":")[1])
        while len(rest) < n:
            rest += c.recv(65536)
    return int(h.split(b" ")[1]), json.loads(rest[:n])


def test_http_chunked_bodies():
    srv = frontend.make_server(frontend.DecideService(FakeEngine()), "127.0.0.1", 0)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    try:
        port = srv.server_address[1]
        head = (b"POST /v1/decide HTTP/1.1\r\nHost: x\r\nContent-Type: application/json\r\n"
                b"Transfer-Encoding: chunked\r\nConnection: close\r\n\r\n")
        b = body(state=[1, 2], questions=CHOICE)
        status, out = _raw_http(port, head, [b[:17], b[17:]])
        assert status == 200 and set(out["answers"]["pick"]["probabilities"]) == {"a", "b", "c"}
        status, out = _raw_http(port, head, [b"x" * 600000, b"x" * 600000])
        assert status == 413 and "1 MiB" in out["error"]["message"]
    finally:
        srv.shutdown()
        srv.server_close()


def test_reference_routes_and_request_checks():
    eng = FakeEngine()
    s = frontend.DecideService(eng)
    h = s.handle("GET", "/health", None).body
    assert h["model"] == "llama" and h["busy"] is False and h["models"] == ["llama"] and h["layers"] == 2
    assert s.handle("GET", "/", None).body["decide"] == "/v1/systemone"
    m = s.handle("GET", "/v1/models", None).body["models"]
    assert [x["name"] for x in m] == ["llama"] and m[0]["default"] is True
    assert s.handle("HEAD", "/v1/models", None).status == 200
    assert s.handle("POST", "/v1/presets", b"{}").status == 404  # presets are not served
    # /v1/systemone is /v1/decide
    a = s.handle("POST", "/v1/systemone", body(state=[1, 2], questions=CHOICE))
    b = s.handle("POST", "/v1/decide", body(state=[1, 2], questions=CHOICE))
    assert a.status == b.status == 200 and a.body == b.body
    # 415, 400 (not UTF-8, repeated key), 422 (model selection)
    assert s.handle("POST", "/v1/decide", b"{}", content_type="text/plain").status == 415
    assert s.handle("POST", "/v1/decide", b"{}", content_type=None).status == 415
    r = s.handle("POST", "/v1/decide", b'{"state": "\xff"}')
    assert r.status == 400 and "UTF-8" in r.body["error"]["message"]
    r = s.handle("POST", "/v1/decide", b'{"x": 1, "x": 2}')
    assert r.status == 400 and "duplicate" in r.body["error"]["message"]
    r = s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE, model="missing"))
    assert r.status == 422 and r.body["error"]["message"] == "unknown model missing; see /v1/models"
    r = s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE, model=3))
    assert r.status == 422 and "must be a string" in r.body["error"]["message"]
    r = s.handle("POST", "/v1/decide", b"[]")
    assert r.status == 422 and "JSON object" in r.body["error"]["message"]
    assert s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE, model="llama")).status == 200


def test_text_requests_with_tokenizer():
    from laya_goish_b200 import synth
    from laya_goish_b200.tokenizer import Tokenizer

    tok = Tokenizer(synth._meta(synth.TINY["tiny-llama-q8_0-tok"]))
    eng = FakeEngine()
    s = frontend.DecideService(eng, tokenizer=tok)
    q = {"q": {"type": "choice", "criteria": {"yes": "yes", "no": "no"}, "suffix": " the answer"}}
    r = s.handle("POST", "/v1/decide", body(state="hello world, is this spam?", questions=q))
    assert r.status == 200, r.body
    assert r.body["usage"]["tokens"] == len(tok.encode("hello world, is this spam?")) + len(tok.encode(" the answer"))
    ids = s.handle("POST", "/v1/decide", body(state=tok.encode("hello world, is this spam?"),
                                              questions={"q": {"type": "choice",
                                                               "criteria": {"yes": tok.encode("yes"), "no": tok.encode("no")},
                                                               "suffix": tok.encode(" the answer")}}))
    assert ids.body["answers"] == r.body["answers"]
    lv = s.handle("POST", "/v1/decide", body(state="x", questions={"s": {"type": "score", "criteria": ["bad", "good"]}}))
    assert lv.status == 200 and lv.body["answers"]["s"]["legend"] == {"0": "bad", "1": "good"}
    # without a tokenizer, text is a 422
    r = frontend.DecideService(FakeEngine()).handle("POST", "/v1/decide", body(state="hello", questions=CHOICE))
    assert r.status == 422 and "tokenizer" in r.body["error"]["message"]


def test_draining_refuses_new_work():
    s = frontend.DecideService(FakeEngine())
    s.draining = True
    h = s.handle("GET", "/health", None)
    assert h.status == 503 and h.body["status"] == "draining"
    r = s.handle("POST", "/v1/decide", body(state=[1], questions=CHOICE))
    assert r.status == 503 and r.body["error"]["type"] == "unavailable_error"


class SlowEngine(FakeEngine):
    """Runs until canceled (or 5 s), recording whether it saw the cancel."""

    def __init__(self):
        super().__init__()
        self.saw_cancel = threading.Event()
        self.started = threading.Event()

    def decide_batch(self, prompts, questions, canceled=None):
        self.started.set()
        import time

        end = time.monotonic() + 5
        while time.monotonic() < end:
            if canceled and canceled():
                self.saw_cancel.set()
                raise LayaError(E_CANCELED, "request canceled")
            time.sleep(0.01)
        return super().decide_batch(prompts, questions)


def test_client_disconnect_cancels_running_request():
    import socket

    eng = SlowEngine()
    srv = frontend.make_server(frontend.DecideService(eng), "127.0.0.1", 0)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    try:
        b = body(state=[1, 2], questions=CHOICE)
        c = socket.create_connection(("127.0.0.1", srv.server_address[1]), timeout=10)
        c.sendall(b"POST /v1/decide HTTP/1.1\r\nHost: x\r\nContent-Type: application/json\r\n"
                  b"Content-Length: %d\r\n\r\n" % len(b) + b)
        assert eng.started.wait(5)
        c.close()
        assert eng.saw_cancel.wait(3)
        assert srv.inflight.wait_idle(5)
    finally:
        srv.shutdown()
        srv.server_close()


CHILD = r"""
import sys, time
sys.path.insert(0, sys.argv[1])
from laya_goish_b200 import frontend

class Eng:
    info = {"architecture": "llama"}
    def layers(self): return 1
    def validate(self, prompts, questions): pass
    def decide_batch(self, prompts, questions, canceled=None):
        time.sleep(1.5)
        return [[{"type": 0, "probabilities": [1.0, 0.0], "logits": [1.0, 0.0], "confidence": 1.0, "choice": 0,
                  "score": 0.0, "noul": 0.0} for _ in questions] for _ in prompts]

def ready(srv):
    print(srv.server_address[1], flush=True)

frontend.serve(frontend.DecideService(Eng()), "127.0.0.1", 0, ready=ready)
print("drained", flush=True)
"""


def test_sigterm_drains_running_request(tmp_path):
    import os
    import signal
    import subprocess
    import sys
    import urllib.request

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    p = subprocess.Popen([sys.executable, "-c", CHILD, root], stdout=subprocess.PIPE, text=True)
    try:
        port = int(p.stdout.readline())
        url = f"http://127.0.0.1:{port}"
        out = {}

        def call():
            req = urllib.request.Request(url + "/v1/decide", method="POST",
                                         data=body(state=[1], questions={"q": {"type": "choice",
                                                                               "criteria": {"a": 1, "b": 2}}}),
                                         headers={"Content-Type": "application/json"})
            with urllib.request.urlopen(req, timeout=20) as r:
                out["status"], out["body"] = r.status, json.loads(r.read())

        t = threading.Thread(target=call)
        t.start()
        import time

        for _ in range(200):  # until the request runs
            with urllib.request.urlopen(url + "/health", timeout=5) as r:
                if json.loads(r.read())["busy"]:
                    break
            time.sleep(0.01)
        p.send_signal(signal.SIGTERM)
        t.join(20)
        assert out.get("status") == 200 and out["body"]["answers"]["q"]["choice"] == "a"
        assert p.wait(timeout=20) == 0
        assert p.stdout.read().strip() == "drained"
    finally:
        if p.poll() is None:
            p.kill()
            p.wait()


def test_command_line_without_a_model_load(tmp_path, capsys):
    import types

    from laya_goish_b200 import synth

    path = synth.write_openthai(str(tmp_path / "ot.gguf"), tokenizer=True)
    assert frontend.main(["info", path]) == 0
    info = json.loads(capsys.readouterr().out)
    assert info["model"] == "openthai-systemone" and info["max_len"] == 512 and info["tensors"] > 0
    assert frontend.main(["tokenize", path, "--text", "th<|ts_q|>"]) == 0
    ids = json.loads(capsys.readouterr().out)
    assert ids == [274, 256]  # the merge "t h", then <|ts_q|> (the first control token)
    # decide needs a request, or a state and questions (no presets)
    assert frontend.main(["decide", path, "--state", "hi"]) == 1
    assert "presets are not served" in capsys.readouterr().err
    with pytest.raises(SystemExit):
        frontend.main(["bogus", path])
    # the request builder (src/main.rs:155-189)
    ns = dict(request=None, state=None, state_file=None, questions=None, questions_file=None)
    q = '{"q": {"type": "noul", "instructions": "?"}}'
    r = frontend.build_request(types.SimpleNamespace(**dict(ns, state="plain text", questions=q)))
    assert r == {"state": "plain text", "questions": {"q": {"type": "noul", "instructions": "?"}}}
    r = frontend.build_request(types.SimpleNamespace(**dict(ns, state='{"a": 1}', questions=q)))
    assert r["state"] == {"a": 1}
    f = tmp_path / "req.json"
    f.write_text(json.dumps({"state": "s", "questions": {}}))
    assert frontend.build_request(types.SimpleNamespace(**dict(ns, request=str(f))))["state"] == "s"
