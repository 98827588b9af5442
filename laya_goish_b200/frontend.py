"""Batch front end over the decision hot path: the request handling of the
reference's HTTP server (`/v1/decide`, `/v1/decide/batch`,
src/server.rs:65-332) and of its JSON-lines daemon (src/main.rs:139-151),
calling one batched `Engine.decide_batch` (laya_decide_batch) per request.

What is kept from the reference, in the same order:

* routes and methods: `/`, `/health` (status, model, busy, layers),
  `/v1/models` (the one loaded model), `/v1/systemone` = `/v1/decide`,
  `/v1/decide/batch`; unknown path -> 404 `not_found_error`; wrong method ->
  405 with `Allow` (src/server.rs:82-158);
* POST bodies: Content-Type must be application/json (415), at most 1 MiB,
  fixed-length or chunked (413), UTF-8 JSON without repeated object keys
  (400), an object whose optional `model` names the loaded model and which
  has a `state` (422, src/server.rs:65-75, 175-233, src/registry.rs:58-73);
* `/v1/decide/batch`: `states` is an array of 1..256 states sharing
  `questions` (src/server.rs:235-258);
* the whole batch is validated before any work starts, the first failure is
  a 422, and at most 256 questions are counted over the batch
  (src/server.rs:259-282);
* one inference at a time: a second request while one runs gets 429
  `busy_error` with `Retry-After: 1` (src/server.rs:283-297);
* a canceled call maps to 408 `request_canceled` (an HTTP client that
  disconnects cancels its request), any other failure to 500
  `internal_error`; success is 200 with `X-Response-Time-Ms`, answers in
  request order (src/server.rs:298-331);
* `serve` drains on SIGTERM / SIGINT: new requests get 503, `/health`
  reports "draining", running requests are answered, then it returns;
* the daemon answers each non-empty input line with one output line, the
  result or `{"error": message}` (src/main.rs:139-151).

`state` is the prompt's token ids (a list, or an object with `ids`), or
text when the service has a tokenizer (the model file's own BPE vocabulary,
`tokenizer.Tokenizer`); every option of a question is a token id, a list of
ids (a continuation) or, with a tokenizer, text.  Question objects follow
src/models/laya/decision.rs:19-98:

    {"type": "choice", "criteria": {"label": option, ...}, "suffix": [ids] | text}
    {"type": "score",  "criteria": [option, ...]}              (>= 2 levels)
    {"type": "noul",   "criteria": {"false": option, "true": option}}

Prompt templates (how a product phrases the question around the state) sit
above this layer: the caller writes them into the state text or the suffix.

Answers follow src/models/laya/decision.rs:214-268 (`choice` label, `score`
with its `legend`, `noul`, `confidence`, `probabilities` by label; `logits`
when raw).  The Laya encoder's `action` head is not part of this path.
Authentication, presets, the model registry and draining are not part of it
either.

An OpenThai GGUF (`general.architecture` "openthai_systemone",
src/models/mod.rs:64-70) is served by `OpenThaiService` over the same routes:
its requests and answer objects are OpenThai's own
(src/models/openthai/decision.rs), one `openthai.Model.respond` per state.
"""
from __future__ import annotations

import json
import select
import signal
import socket
import sys
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Callable

from ._lib import E_CANCELED, E_INVALID, LayaError

MAX_STATES = 256
MAX_QUESTIONS = 256
MAX_OPTIONS = 16
MAX_BODY = 1024 * 1024  # src/server.rs:22

# src/server.rs:82-89; /v1/systemone is the reference's other name for /v1/decide
ROUTES = {"/": "GET, HEAD", "/health": "GET, HEAD", "/v1/models": "GET, HEAD", "/v1/systemone": "POST",
          "/v1/decide": "POST", "/v1/decide/batch": "POST"}


def _no_duplicate_keys(pairs):
    """JSON objects with a repeated key are rejected (400), as the
    reference's parser does."""
    out = {}
    for k, v in pairs:
        if k in out:
            raise ValueError(f"duplicate object key {k}")
        out[k] = v
    return out


def parse_body(body: bytes | str | None):
    """The request body as JSON: UTF-8 text, no repeated object keys
    (src/server.rs:214-227); ValueError with the message of the 400."""
    if isinstance(body, (bytes, bytearray)):
        try:
            body = bytes(body).decode("utf-8")
        except UnicodeDecodeError:
            raise ValueError("Request body is not UTF-8") from None
    return json.loads(body or "", object_pairs_hook=_no_duplicate_keys)


class RequestError(ValueError):
    """A request that fails validation (422 over HTTP)."""


def _encode(tok, text: str, what: str) -> list[int]:
    if tok is None:
        raise RequestError(f"{what}: text needs a model with a tokenizer; send token ids")
    try:
        ids = tok.encode(text)
    except ValueError as e:
        raise RequestError(f"{what}: {e}") from e
    if not ids:
        raise RequestError(f"{what}: text encodes to no tokens")
    return ids


def _ids(v, what: str, tok=None) -> list[int]:
    if isinstance(v, str):
        return _encode(tok, v, what)
    if isinstance(v, bool) or not isinstance(v, (int, list)):
        raise RequestError(f"{what} must be a token id or a list of token ids")
    ids = [v] if isinstance(v, int) else v
    if not ids or any(isinstance(t, bool) or not isinstance(t, int) for t in ids):
        raise RequestError(f"{what} must be a token id or a non-empty list of token ids")
    return ids


def state_ids(state, tok=None) -> list[int]:
    """The prompt of one request: a list of token ids, {"ids": [...]}, or text."""
    if isinstance(state, dict):
        state = state.get("ids")
    if isinstance(state, str):
        return _encode(tok, state, "state")
    if not isinstance(state, list) or not state:
        raise RequestError("state must be a non-empty list of token ids (or an object with ids)")
    return _ids(state, "state")


class ParsedQuestion:
    def __init__(self, qid: str, kind: str, labels: list[str], options: list[list[int]], suffix: list[int],
                 given=None):
        self.id, self.kind, self.labels, self.options, self.suffix = qid, kind, labels, options, suffix
        self.given = given  # the criteria as sent (the score legend)


def parse_questions(obj, tok=None) -> list[ParsedQuestion]:
    """src/models/laya/decision.rs:19-98 on token-level (or tokenised) criteria."""
    if not isinstance(obj, dict) or not obj or len(obj) > MAX_QUESTIONS:
        raise RequestError("questions must contain 1..256 named questions")
    out = []
    for qid, q in obj.items():
        if not isinstance(q, dict):
            raise RequestError(f"{qid}: question must be an object")
        kind = q.get("type")
        if kind not in ("choice", "score", "noul"):
            raise RequestError(f"{qid}: type must be choice, score, or noul")
        c = q.get("criteria")
        if kind == "choice":
            if not isinstance(c, dict) or not c:
                raise RequestError(f"{qid}: choice requires a criteria object")
            labels = list(c)
            opts = [_ids(c[k], f"{qid}.{k}", tok) for k in labels]
        elif kind == "score":
            if not isinstance(c, list) or len(c) < 2:
                raise RequestError(f"{qid}: score requires at least two ordered criteria")
            labels = [str(i) for i in range(len(c))]
            opts = [_ids(v, f"{qid}[{i}]", tok) for i, v in enumerate(c)]
        else:
            if not isinstance(c, dict) or "false" not in c or "true" not in c:
                raise RequestError(f"{qid}: noul requires criteria with false and true token ids")
            labels = ["false", "true"]
            opts = [_ids(c["false"], f"{qid}.false", tok), _ids(c["true"], f"{qid}.true", tok)]
        if not opts or len(opts) > MAX_OPTIONS:
            raise RequestError(f"{qid}: requires 1..16 options")
        if len({len(o) for o in opts}) != 1:
            raise RequestError(f"{qid}: all options must have the same number of tokens")
        suffix = q.get("suffix", [])
        if suffix is None:
            suffix = []
        if isinstance(suffix, str):
            suffix = _encode(tok, suffix, f"{qid}.suffix")
        if not isinstance(suffix, list) or any(isinstance(t, bool) or not isinstance(t, int) for t in suffix):
            raise RequestError(f"{qid}: suffix must be a list of token ids")
        out.append(ParsedQuestion(str(qid), kind, labels, opts, suffix, c))
    return out


def _engine_questions(qs: list[ParsedQuestion]):
    from .engine import Question

    return [Question(q.kind, [o[0] for o in q.options] if len(q.options[0]) == 1 else q.options, q.suffix)
            for q in qs]


def answer_json(q: ParsedQuestion, a: dict, raw: bool) -> dict:
    """src/models/laya/decision.rs:214-268 for one question."""
    p = a["probabilities"]
    out = {"type": q.kind}
    if q.kind == "choice":
        out["choice"] = q.labels[a["choice"]]
    elif q.kind == "score":
        out["score"] = a["score"]
        out["legend"] = {str(i): v for i, v in enumerate(q.given)}
    else:
        out["noul"] = a["noul"]
    out["confidence"] = a["confidence"]
    out["probabilities"] = {lab: v for lab, v in zip(q.labels, p)}
    if raw:
        out["logits"] = a["logits"]
    return out


class Response:
    def __init__(self, status: int, body: dict, headers: dict | None = None):
        self.status, self.body, self.headers = status, body, headers or {}

    def json(self) -> str:
        return json.dumps(self.body) + "\n"


def _error(status: int, kind: str, message: str, headers: dict | None = None) -> Response:
    return Response(status, {"error": {"type": kind, "message": message}}, headers)


class DecideService:
    """The server's request handling around one loaded Engine (or any object
    with the same `validate` / `decide_batch` / `info` interface)."""

    def __init__(self, engine, raw: bool = False, tokenizer=None, name: str | None = None,
                 family: str | None = None):
        self.engine = engine
        self.raw = raw
        self.tokenizer = tokenizer
        self.name = name or str(engine.info.get("architecture"))
        self.family = family or self.name
        self._busy = threading.Lock()
        self._requests = 0
        self._count_lock = threading.Lock()
        self.draining = False  # set on SIGTERM: new work is refused, running work finishes

    def _select(self, req) -> None:
        """The request's optional `model` must name the loaded model
        (src/registry.rs:58-73, one model loaded)."""
        if not isinstance(req, dict):
            raise RequestError("request body must be a JSON object")
        m = req.get("model")
        if m is None:
            return
        if not isinstance(m, str):
            raise RequestError("model must be a string naming a loaded model")
        if m != self.name:
            raise RequestError(f"unknown model {m}; see /v1/models")

    def _info(self, path: str) -> Response:
        if path == "/":
            return Response(200, {"service": "laya-goish B200", "health": "/health", "decide": "/v1/systemone"})
        if path == "/v1/models":
            return Response(200, {"models": [{
                "name": self.name, "canonical_name": self.name, "architecture": str(self.engine.info.get("architecture")),
                "family": self.family, "default": True,
                "description": f"Locally loaded {self.name} decision model on B200"}]})
        return Response(503 if self.draining else 200,
                        {"status": "draining" if self.draining else "ok", "model": self.name, "family": self.family,
                         "device": "cuda", "models": [self.name], "busy": self._busy.locked(),
                         "layers": self.engine.layers()})

    def _prepare(self, req) -> tuple[list[list[int]], list[ParsedQuestion]]:
        if not isinstance(req, dict):
            raise RequestError("request body must be a JSON object")
        if req.get("state") is None:
            raise RequestError("state is required")
        return [state_ids(req["state"], self.tokenizer)], parse_questions(req.get("questions"), self.tokenizer)

    def handle(self, method: str, path: str, body: bytes | str | None,
               canceled: Callable[[], bool] | None = None,
               content_type: str | None = "application/json") -> Response:
        """One HTTP request.  `content_type` is its Content-Type header
        (in-process callers without headers keep the default)."""
        with self._count_lock:
            self._requests += 1
            rid = self._requests
        r = self._handle(method, path, body, canceled, content_type)
        r.headers.setdefault("X-Request-Id", f"laya-{rid}")
        return r

    def _handle(self, method, path, body, canceled, content_type) -> Response:
        allowed = ROUTES.get(path)
        if allowed is None:
            return _error(404, "not_found_error", "Endpoint not found")
        if (allowed == "POST") != (method == "POST") or (allowed != "POST" and method not in ("GET", "HEAD")):
            return _error(405, "invalid_request_error", "Method not allowed", {"Allow": allowed})
        if allowed != "POST":
            return self._info(path)
        if self.draining:
            return _error(503, "unavailable_error", "Server is shutting down")
        if (content_type or "").split(";")[0].strip().lower() != "application/json":
            return _error(415, "invalid_request_error", "Content-Type must be application/json")
        if body is not None and len(body) > MAX_BODY:
            return _error(413, "invalid_request_error", "Request body exceeds 1 MiB")
        try:
            req = parse_body(body)
        except ValueError as e:
            return _error(400, "invalid_request_error", str(e))
        try:
            self._select(req)
        except RequestError as e:
            return _error(422, "invalid_request_error", str(e))
        return self._decide(req, path == "/v1/decide/batch", canceled)

    def _decide(self, req, batch: bool, canceled) -> Response:
        # Validate the whole batch before starting any expensive work.
        try:
            if batch:
                if not isinstance(req, dict):
                    raise RequestError("request body must be a JSON object")
                states = req.get("states")
                if not isinstance(states, list) or not 1 <= len(states) <= MAX_STATES:
                    raise RequestError("states must be an array of 1..256 states")
                prompts = [state_ids(s, self.tokenizer) for s in states]
                qs = parse_questions(req.get("questions"), self.tokenizer)
            else:
                prompts, qs = self._prepare(req)
            eqs = _engine_questions(qs)
            self.engine.validate(prompts, eqs)
            if len(qs) * len(prompts) > MAX_QUESTIONS:
                raise RequestError("At most 256 total questions per request")
        except RequestError as e:
            return _error(422, "invalid_request_error", str(e))
        except LayaError as e:
            if e.code == E_INVALID:
                return _error(422, "invalid_request_error", e.message)
            return _error(500, "internal_error", e.message)
        if not self._busy.acquire(blocking=False):
            return _error(429, "busy_error", "An inference request is running; retry later", {"Retry-After": "1"})
        try:
            start = time.perf_counter()
            try:
                ans = self.engine.decide_batch(prompts, eqs, canceled=canceled)
            except LayaError as e:
                if e.code == E_CANCELED:
                    return _error(408, "request_canceled", e.message)
                return _error(500, "internal_error", e.message)
            ms = int((time.perf_counter() - start) * 1000)
        finally:
            self._busy.release()
        results = []
        for prompt, row in zip(prompts, ans):
            tokens = sum(len(prompt) + len(q.suffix) for q in qs)
            results.append({"model": self.engine.info.get("architecture"),
                            "answers": {q.id: answer_json(q, a, self.raw) for q, a in zip(qs, row)},
                            "usage": {"tokens": tokens}})
        body = {"results": results} if batch else results[0]
        return Response(200, body, {"X-Response-Time-Ms": str(ms)})


class OpenThaiService(DecideService):
    """The same routes over an OpenThai model (`openthai.Model`), whose
    requests keep OpenThai's own shape (decision.rs:20-109): `state` is text
    or any JSON object / array written into the prompt, questions carry
    `instructions` and `criteria`, plus `order_invariant` / `permutations`.
    Each request (each state of a batch, with the shared questions and
    options, src/server.rs:235-258) is validated through every permutation
    pass before any runs, then answered by one `Model.respond`; the answer
    objects are the model's own (model, answers, usage, id, _raw).

    `model` may be a list with one model per GPU: the states of a batch are
    then shared out over them (each device thread takes the next unanswered
    state), answers stay in request order, and the first failure stops the
    others before their next state and fails the batch."""

    def __init__(self, model, tokenizer, raw: bool = False):
        if tokenizer is None:
            raise ValueError("an OpenThai model needs its tokenizer")
        self.models = list(model) if isinstance(model, (list, tuple)) else [model]
        if not self.models:
            raise ValueError("no OpenThai model")
        super().__init__(self.models[0], raw=raw, tokenizer=tokenizer, name="openthai-systemone",
                         family="openthai-systemone")

    def _run(self, reqs, canceled):
        """Answers of `reqs` in order, over every model; raises the first
        LayaError (a cancel wins over later failures)."""
        if len(self.models) == 1 or len(reqs) == 1:
            return [self.engine.respond(self.tokenizer, r, self.raw, canceled) for r in reqs]
        results = [None] * len(reqs)
        errors = []
        lock = threading.Lock()
        nxt = [0]

        def stop():
            return bool(errors) or (canceled is not None and canceled())

        def worker(m):
            while True:
                with lock:
                    if errors or nxt[0] >= len(reqs):
                        return
                    i = nxt[0]
                    nxt[0] += 1
                try:
                    results[i] = m.respond(self.tokenizer, reqs[i], self.raw, stop)
                except Exception as e:  # any failure stops the other workers and fails the batch
                    with lock:
                        errors.append((i, e))
                    return

        threads = [threading.Thread(target=worker, args=(m,)) for m in self.models[:len(reqs)]]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            # the failure that stopped the others, not the cancels it caused
            first = [e for _, e in errors if getattr(e, "code", None) != E_CANCELED] or [e for _, e in errors]
            if canceled is not None and canceled():
                raise LayaError(E_CANCELED, "request canceled")
            raise first[0]
        return results

    def _decide(self, req, batch: bool, canceled) -> Response:
        from .openthai import OpenThaiError

        try:
            if not isinstance(req, dict):
                raise RequestError("request body must be a JSON object")
            if batch:
                states = req.get("states")
                if not isinstance(states, list) or not 1 <= len(states) <= MAX_STATES:
                    raise RequestError("states must be an array of 1..256 states")
                reqs = [{"state": st, "questions": req.get("questions"), "model": req.get("model"),
                         "order_invariant": req.get("order_invariant"), "permutations": req.get("permutations")}
                        for st in states]
            else:
                reqs = [req]
            count = 0
            for r in reqs:
                if r.get("state") is None:
                    raise RequestError("state is required")
                self.engine.validate(self.tokenizer, r)
                count += len(r["questions"])
            if count > MAX_QUESTIONS:
                raise RequestError("At most 256 total questions per request")
        except (RequestError, OpenThaiError) as e:
            return _error(422, "invalid_request_error", str(e))
        if not self._busy.acquire(blocking=False):
            return _error(429, "busy_error", "An inference request is running; retry later", {"Retry-After": "1"})
        try:
            start = time.perf_counter()
            try:
                results = self._run(reqs, canceled)
            except LayaError as e:
                if e.code == E_CANCELED:
                    return _error(408, "request_canceled", e.message)
                return _error(500, "internal_error", e.message)
            except Exception as e:  # a failure outside the library (model wrapper, tokenizer) is a 500 too
                return _error(500, "internal_error", str(e) or type(e).__name__)
            ms = int((time.perf_counter() - start) * 1000)
        finally:
            self._busy.release()
        return Response(200, {"results": results} if batch else results[0], {"X-Response-Time-Ms": str(ms)})


def run_daemon(service: DecideService, inp=None, out=None) -> None:
    """JSON lines: each non-empty input line is one decide request, given to
    the model as it is (no route, content-type or `model` checks); the
    answer or {"error": message} is written as one line (src/main.rs:139-151)."""
    inp = inp or sys.stdin
    out = out or sys.stdout
    for line in inp:
        if not line.strip():
            continue
        try:
            r = service._decide(parse_body(line), False, None)  # no HTTP checks: the line goes to decide
        except ValueError as e:
            r = _error(400, "invalid_request_error", str(e))
        if r.status == 200:
            out.write(r.json())
        else:
            out.write(json.dumps({"error": r.body["error"]["message"]}) + "\n")
        out.flush()


class _InFlight:
    """Requests between their first byte and their last response byte."""

    def __init__(self):
        self.n = 0
        self.cv = threading.Condition()

    def __enter__(self):
        with self.cv:
            self.n += 1

    def __exit__(self, *exc):
        with self.cv:
            self.n -= 1
            self.cv.notify_all()

    def wait_idle(self, timeout: float) -> bool:
        with self.cv:
            return self.cv.wait_for(lambda: self.n == 0, timeout)


def make_server(service: DecideService, host: str = "127.0.0.1", port: int = 8080) -> ThreadingHTTPServer:
    """An HTTP server over `service` (serve with .serve_forever(), or `serve`
    for the signal handling).  `server.inflight` counts requests being
    answered."""
    inflight = _InFlight()

    class Handler(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def _body(self):
            """The request body (Content-Length or chunked); None past 1 MiB
            or when it cannot be read.  Bodies over 1 MiB are still read and
            dropped up to 16 MiB (the reference's transport buffers that
            much before dispatch), so the client gets the 413 instead of a
            reset connection."""
            hard = 16 * MAX_BODY
            if "chunked" in (self.headers.get("Transfer-Encoding") or "").lower():
                out, total = bytearray(), 0
                while True:
                    line = self.rfile.readline(64)
                    try:
                        n = int(line.split(b";")[0].strip() or b"x", 16)
                    except ValueError:
                        return None
                    if n == 0:
                        while self.rfile.readline(1024) not in (b"\r\n", b"\n", b""):
                            pass  # trailers
                        return bytes(out) if total <= MAX_BODY else None
                    total += n
                    if total > hard:
                        return None
                    data = self.rfile.read(n)
                    if total <= MAX_BODY:
                        out += data
                    self.rfile.readline(8)  # the chunk's CRLF
            n = int(self.headers.get("Content-Length") or 0)
            if n > MAX_BODY:
                if n <= hard:
                    while n > 0:
                        got = len(self.rfile.read(min(n, 1 << 16)))
                        if not got:
                            break
                        n -= got
                return None
            return self.rfile.read(n) if n else b""

        def _client_gone(self) -> bool:
            """True once the client has closed its side: the request is
            canceled between steps (src/server.rs:297-313, the request
            context ends on disconnect)."""
            try:
                readable, _, _ = select.select([self.connection], [], [], 0)
                return bool(readable) and self.connection.recv(1, socket.MSG_PEEK) == b""
            except OSError:
                return True

        def _go(self, method):
            with inflight:
                self._answer(method)

        def _answer(self, method):
            body = self._body() if method == "POST" else b""
            if body is None:
                self.close_connection = True
                r = _error(413, "invalid_request_error", "Request body exceeds 1 MiB or could not be read")
            else:
                r = service.handle(method, self.path.split("?", 1)[0], body, canceled=self._client_gone,
                                   content_type=self.headers.get("Content-Type"))
            data = r.json().encode()
            try:
                self.send_response(r.status)
                self.send_header("Content-Type", "application/json; charset=utf-8")
                self.send_header("Cache-Control", "no-store")
                self.send_header("X-Content-Type-Options", "nosniff")
                self.send_header("Content-Length", str(len(data)))
                for k, v in r.headers.items():
                    self.send_header(k, v)
                self.end_headers()
                if method != "HEAD":
                    self.wfile.write(data)
            except (BrokenPipeError, ConnectionResetError):
                self.close_connection = True  # the client left (a canceled request)

        def do_GET(self):
            self._go("GET")

        def do_HEAD(self):
            self._go("HEAD")

        def do_POST(self):
            self._go("POST")

        def log_message(self, *a):
            pass

    srv = ThreadingHTTPServer((host, port), Handler)
    srv.inflight = inflight
    return srv


def serve(service: DecideService, host: str = "127.0.0.1", port: int = 8080, ready=None,
          drain_timeout: float = 600.0) -> None:
    """Serves until SIGTERM or SIGINT, then drains (the reference's
    shutdown): new requests get 503 and /health reports "draining", requests
    already running finish and are answered, and the call returns.
    `ready(server)` is called once the socket listens."""
    srv = make_server(service, host, port)

    def stop(*_):
        service.draining = True
        threading.Thread(target=srv.shutdown, daemon=True).start()

    old = {sig: signal.signal(sig, stop) for sig in (signal.SIGTERM, signal.SIGINT)}
    try:
        if ready is not None:
            ready(srv)
        srv.serve_forever()
        srv.inflight.wait_idle(drain_timeout)
    finally:
        srv.server_close()
        for sig, h in old.items():
            signal.signal(sig, h)


MODES = ("decide", "daemon", "serve", "tokenize", "info")


def build_request(a) -> dict:
    """The `decide` command's request (src/main.rs:155-189): the --request
    file, or a state (--state as JSON, else as text; --state-file) and the
    questions (--questions / --questions-file).  Presets are not served, so
    the questions must be given."""
    if a.request:
        with open(a.request, encoding="utf-8") as f:
            return parse_body(f.read())
    if a.state is not None:
        try:
            state = parse_body(a.state)
        except ValueError:
            state = a.state
    elif a.state_file:
        with open(a.state_file, encoding="utf-8") as f:
            state = parse_body(f.read())
    else:
        raise RequestError("--request, --state or --state-file is required")
    if a.questions is not None:
        questions = parse_body(a.questions)
    elif a.questions_file:
        with open(a.questions_file, encoding="utf-8") as f:
            questions = parse_body(f.read())
    else:
        raise RequestError("--questions or --questions-file is required (presets are not served)")
    return {"state": state, "questions": questions}


def gguf_info(path: str) -> dict:
    """The `info` command (Gguf::info, src/gguf.rs:204-224) for this build."""
    from .gguf_meta import _parse

    with open(path, "rb") as f:
        meta, infos, _ = _parse(memoryview(f.read()), tensors=True)
    arch = meta.get("general.architecture")
    return {"name": meta.get("general.name"),
            "model": "openthai-systemone" if arch == "openthai_systemone" else meta.get("laya.model_name", arch),
            "architecture": arch, "checkpoint": meta.get("laya.checkpoint"),
            "max_len": int(meta.get("openthai.context_length", meta.get("laya.max_len", 512))),
            "tensors": len(infos), "runtime": "laya-goish B200 (CUDA, sm_100a)"}


def main(argv=None) -> int:
    """`python -m laya_goish_b200.frontend COMMAND MODEL [options]`, the
    reference's command line (src/main.rs:33-192) for the commands on the
    decision path: decide, daemon, serve, plus tokenize and info.  The older
    `MODEL COMMAND` order is accepted too."""
    import argparse

    ap = argparse.ArgumentParser(prog="python -m laya_goish_b200.frontend")
    ap.add_argument("first", help="command (decide, daemon, serve, tokenize, info) or GGUF file")
    ap.add_argument("second", help="GGUF file or command")
    ap.add_argument("--devices", default="0", help="comma-separated CUDA devices")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8080)
    ap.add_argument("--raw", action="store_true")
    ap.add_argument("--request", help="decide: request JSON file")
    ap.add_argument("--state", help="decide: state (JSON, or text)")
    ap.add_argument("--state-file", help="decide: state JSON file")
    ap.add_argument("--questions", help="decide: questions JSON")
    ap.add_argument("--questions-file", help="decide: questions JSON file")
    ap.add_argument("--text", help="tokenize: text")
    ap.add_argument("--threads", type=int, help="accepted for compatibility; the GPU path ignores it")
    a = ap.parse_args(argv)
    mode, model = (a.first, a.second) if a.first in MODES else (a.second, a.first)
    if mode not in MODES:
        ap.error(f"unknown command {mode}")
    if not 1 <= a.port <= 65535:
        ap.error("--port must be 1..65535")
    from .gguf_meta import read_metadata
    from .tokenizer import Tokenizer

    if mode == "info":
        print(json.dumps(gguf_info(model), ensure_ascii=False))
        return 0
    if mode == "tokenize":
        if a.text is None:
            ap.error("missing --text")
        print(json.dumps(Tokenizer.from_gguf(model).encode(a.text)))
        return 0
    req = None
    if mode == "decide":
        try:
            req = build_request(a)
        except (RequestError, ValueError, OSError) as e:
            print(str(e), file=sys.stderr)
            return 1
    try:
        tok = Tokenizer.from_gguf(model)
    except ValueError:
        tok = None  # no usable vocabulary in the file: token-id requests only
    devices = [int(d) for d in a.devices.split(",")]
    if read_metadata(model).get("general.architecture") == "openthai_systemone":
        from .openthai import Model

        models = [Model(model, device=d) for d in devices]
        svc = OpenThaiService(models, tok, raw=a.raw)
    else:
        from .engine import Engine

        models = [Engine(model, devices=devices)]
        svc = DecideService(models[0], raw=a.raw, tokenizer=tok)
    rc = 0
    try:
        if mode == "decide":
            r = svc.handle("POST", "/v1/decide", json.dumps(req))
            if r.status == 200:
                print(json.dumps(r.body, ensure_ascii=False))
            else:
                print(r.body["error"]["message"], file=sys.stderr)
                rc = 1
        elif mode == "daemon":
            run_daemon(svc)
        else:
            serve(svc, a.host, a.port)
    finally:
        for m in models:
            m.close()
    return rc


if __name__ == "__main__":
    sys.exit(main())
