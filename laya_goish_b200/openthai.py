"""Host side of OpenThai decisions: the request rules, the control-token
prompt, the option-order permutations and the calibrated slot decoding of
src/models/openthai/decision.rs, restated for the GPU forward (the layers'
mixers are `engine.gated_attention` / `engine.gated_delta_mixer`).

A request's questions become text blocks

    <|ts_q|><|ts_{choice|score|noul}|> {instructions}\\n
    <|ts_opt_{slot}|> {name}[: {description}]\\n      (one per option, in pass order)
    <|ts_answer|>\\n

after a state block `<|ts_state|> {state}\\n` (decision.rs:169-233); the slot
head's 256 logits at each block's answer token give, per question, a softmax
over its k option slots and the abstain slot 255, scaled by the per-kind
temperature; choice questions are asked in several cyclic option orders and
the slot probabilities are averaged back onto the options (decision.rs:
243-391).

Where the reference leaves the exact text to its own JSON writer (numbers in
non-string states), the standard library's JSON formatting is used; that
corner is not pinned.
"""
from __future__ import annotations

import json
import math
import time

import numpy as np

KINDS = ("choice", "score", "noul")
ABSTAIN_SLOT = 255
SLOTS = 256
# Unicode White_Space (Rust's str::trim)
_WS = frozenset([0x9, 0xA, 0xB, 0xC, 0xD, 0x20, 0x85, 0xA0, 0x1680, *range(0x2000, 0x200B), 0x2028, 0x2029,
                 0x202F, 0x205F, 0x3000])


class OpenThaiError(ValueError):
    pass


def trim(s: str) -> str:
    i, j = 0, len(s)
    while i < j and ord(s[i]) in _WS:
        i += 1
    while j > i and ord(s[j - 1]) in _WS:
        j -= 1
    return s[i:j]


def clean(s: str) -> str:
    """Control-token text inside user strings is broken with a zero-width
    space (decision.rs:17-19)."""
    return s.replace("<|ts_", "<\u200b|ts_")


class Spec:
    def __init__(self, qid, kind, ins, names, desc):
        self.id, self.kind, self.ins, self.names, self.desc = qid, kind, ins, names, desc


def questions(req: dict) -> list[Spec]:
    """Request validation (decision.rs:20-109)."""
    qs = req.get("questions")
    if not isinstance(qs, dict) or not qs or len(qs) > 256:
        raise OpenThaiError("questions must contain 1..256 named questions")
    if not isinstance(req.get("state"), (str, dict, list)):
        raise OpenThaiError("OpenThai state must be a string, object, or array")
    out = []

    def text(qid, v):
        if isinstance(v, str):
            return v
        if v is None:
            return ""
        raise OpenThaiError(f"{qid}: descriptions must be strings or null")

    for qid, q in qs.items():
        q = q if isinstance(q, dict) else {}
        kind = q.get("type")
        if kind not in KINDS:
            raise OpenThaiError(f"{qid}: invalid question type")
        kind = KINDS.index(kind)
        ins = q.get("instructions")
        if not isinstance(ins, str):
            raise OpenThaiError(f"{qid}: instructions must be a string")
        c = q.get("criteria")
        names, desc = [], []
        if kind == 0:
            if not isinstance(c, dict) or not 1 <= len(c) <= 255:
                raise OpenThaiError(f"{qid}: choice requires 1..255 options")
            for name, d in c.items():
                if not trim(name):
                    raise OpenThaiError(f"{qid}: option name is empty")
                names.append(name)
                desc.append(text(qid, d))
        elif kind == 1:
            if not isinstance(c, list) or not 2 <= len(c) <= 10:
                raise OpenThaiError(f"{qid}: score requires 2..10 levels")
            for i, d in enumerate(c):
                if not isinstance(d, str):
                    raise OpenThaiError(f"{qid}: score descriptions must be strings")
                names.append(str(i))
                desc.append(d)
        else:
            if not (c is None or isinstance(c, dict)) or (isinstance(c, dict) and any(k not in ("false", "true")
                                                                                      for k in c)):
                raise OpenThaiError(f"{qid}: noul criteria keys must be false/true")
            c = c or {}
            names = ["no", "yes"]
            desc = [text(qid, c.get("false")), text(qid, c.get("true"))]
        out.append(Spec(str(qid), kind, ins, names, desc))
    oi = req.get("order_invariant")
    if oi is not None and not isinstance(oi, bool):
        raise OpenThaiError("order_invariant must be boolean")
    p = req.get("permutations")
    if p is not None:
        if isinstance(p, bool) or not isinstance(p, (int, float)) or not 1 <= p <= 32 or p != int(p):
            raise OpenThaiError("permutations must be 1..32")
    return out


def orders(k: int, n: int) -> list[list[int]]:
    """The n cyclic option orders of a k-option question (decision.rs:120-135):
    offsets j*k/n rounded half to even, deduplicated, ascending."""
    n = max(1, min(n, k))
    offs = set()
    for j in range(n):
        a = j * k
        d, rem = a // n, a % n
        offs.add((d + (1 if rem * 2 > n or (rem * 2 == n and d % 2 == 1) else 0)) % k)
    return [[(i + off) % k for i in range(k)] for off in sorted(offs)]


def permutation_count(req: dict, qs: list[Spec]) -> int:
    """Passes over the prompt (decision.rs:136-162)."""
    k = max([len(q.names) for q in qs if q.kind == 0], default=1)
    p = req.get("permutations")
    if p is not None:
        n = int(p)
    elif req.get("order_invariant") is False:
        n = 1
    elif req.get("order_invariant") is True:
        n = 8
    else:
        n = 8 if k >= 11 else 1
    return max(1, min(n, k))


def py_state(v) -> str:
    """A non-string state as text (decision.rs:110-119): strings JSON-quoted,
    arrays `[a, b]`, objects `{"k": v}`, other values as JSON."""
    if isinstance(v, str):
        return json.dumps(v, ensure_ascii=False)
    if isinstance(v, list):
        return "[" + ", ".join(py_state(x) for x in v) + "]"
    if isinstance(v, dict):
        return "{" + ", ".join(f"{json.dumps(k, ensure_ascii=False)}: {py_state(x)}" for k, x in v.items()) + "}"
    return json.dumps(v)


class Encoded:
    def __init__(self, ids, positions, order, truncated):
        self.ids, self.positions, self.order, self.truncated = ids, positions, order, truncated


def encode(tok, req: dict, qs: list[Spec], n: int, npass: int, answer_id: int, max_tokens: int = 4096,
           max_state: int = 2048) -> Encoded:
    """Pass `npass` of the prompt (decision.rs:169-233): question blocks in
    that pass's option order, the state block truncated to its budget
    (keeping its first token), answer positions at each block's last answer
    token."""
    blocks, order = [], []
    for q in qs:
        if q.kind == 0:
            all_ = orders(len(q.names), n)
            ordq = all_[npass % len(all_)]
        else:
            ordq = list(range(len(q.names)))
        text = f"<|ts_q|><|ts_{KINDS[q.kind]}|> {trim(clean(q.ins))}\n"
        for slot, i in enumerate(ordq):
            text += f"<|ts_opt_{slot}|> {trim(clean(q.names[i]))}"
            if q.desc[i]:
                text += f": {trim(clean(q.desc[i]))}"
            text += "\n"
        text += "<|ts_answer|>\n"
        blocks.append(tok.encode(text))
        order.append(ordq)
    total = sum(len(b) for b in blocks)
    if total >= max_tokens:
        raise OpenThaiError("question tokens exceed OpenThai context budget")
    state = req["state"] if isinstance(req["state"], str) else py_state(req["state"])
    ids = tok.encode(f"<|ts_state|> {trim(clean(state))}\n")
    budget = min(max_state, max_tokens - total)
    truncated = len(ids) > budget
    if truncated:
        ids = ids[:1] + ids[len(ids) - (budget - 1):]
    positions = []
    for b in blocks:
        if answer_id not in b:
            raise OpenThaiError("missing OpenThai answer token")
        p = len(b) - 1 - b[::-1].index(answer_id)
        positions.append(len(ids) + p)
        ids = ids + b
    return Encoded(ids, positions, order, truncated)


def _softmax32(x: np.ndarray) -> np.ndarray:
    """tensor::softmax (src/tensor.rs:132-140) in F32."""
    x = x.astype(np.float32)
    e = np.exp(x - x.max()).astype(np.float32)
    s = np.float32(0)
    for v in e:
        s = np.float32(s + v)
    return (e / s).astype(np.float32)


def decide(qs: list[Spec], passes, temperature) -> dict:
    """Calibrated slot decoding (decision.rs:264-380).  passes: one (logits,
    order) per permutation pass, logits [len(qs)][256] slot-head rows at the
    answer positions, order the pass's option order per question;
    temperature[kind] from the model.  Returns {question id: answer}."""
    n = len(passes)
    probs = [np.zeros(len(q.names), np.float32) for q in qs]
    abstain = [np.float32(0)] * len(qs)
    for logits, order in passes:
        for i, q in enumerate(qs):
            k = len(q.names)
            row = np.asarray(logits[i], np.float32)
            t = np.float32(temperature[q.kind])
            valid = np.concatenate([row[:k] / t, [row[ABSTAIN_SLOT] / t]]).astype(np.float32)
            p = _softmax32(valid)
            ssum = np.float32(0)
            for v in p[:k]:
                ssum = np.float32(ssum + v)
            ssum = max(ssum, np.float32(1e-12))
            for slot in range(k):
                probs[i][order[i][slot]] += p[slot] / ssum / np.float32(n)
            abstain[i] = np.float32(abstain[i] + p[k] / np.float32(n))
    out = {}
    for i, q in enumerate(qs):
        p = probs[i]
        s = np.float32(0)
        for v in p:
            s = np.float32(s + v)
        p = (p / max(s, np.float32(1e-12))).astype(np.float32)
        k = len(p)
        ent = np.float32(0)
        for v in p:
            v = max(v, np.float32(1e-12))
            ent = np.float32(ent + v * np.float32(math.log(v)))
        ent = -ent
        conf = 1.0 if k <= 1 else float(min(max(1 - ent / np.float32(math.log(k)), 0.0), 1.0))
        a = {"type": KINDS[q.kind]}
        if q.kind == 2:
            a["noul"] = float(p[1])
        else:
            a["probabilities"] = {name: float(v) for name, v in zip(q.names, p)}
            a["confidence"] = conf
            if q.kind == 0:
                best = 0
                for j in range(1, k):
                    if p[j] > p[best]:
                        best = j
                a["choice"] = q.names[best]
                a["abstain"] = float(abstain[i])
            else:
                a["score"] = float(sum(np.float32(j) * v for j, v in enumerate(p)))
                a["legend"] = {str(j): (d if d else str(j)) for j, d in enumerate(q.desc)}
        out[q.id] = a
    return out


# Model::new's fixed text_config (src/models/openthai/model.rs:99-125)
REFERENCE_CONFIG = {"hidden_size": 1024, "intermediate_size": 3584, "num_hidden_layers": 24, "head_dim": 256,
                    "num_attention_heads": 8, "num_key_value_heads": 2, "linear_conv_kernel_dim": 4,
                    "linear_key_head_dim": 128, "linear_value_head_dim": 128, "linear_num_key_heads": 16,
                    "linear_num_value_heads": 16, "vocab_size": 248339}


def load_config(meta: dict, strict: bool = True) -> dict:
    """The model shape from a GGUF's `openthai.config` JSON
    (src/models/openthai/model.rs:99-135).  strict: the reference's checks
    (its one supported size, 256 slots with abstain slot 255, answer token
    248082, eps 1e-6, rope theta 1e7 on a quarter of each head); otherwise any
    consistent shape (small models for tests)."""
    try:
        cfg = json.loads(meta.get("openthai.config", ""))
    except ValueError as e:
        raise OpenThaiError(f"openthai.config: {e}") from e
    c = cfg.get("text_config") or {}
    if strict:
        for k, n in REFERENCE_CONFIG.items():
            if c.get(k) != n:
                raise OpenThaiError(f"unsupported OpenThai config {k}")
        rp = c.get("rope_parameters") or {}
        if (cfg.get("n_slots") != 256 or cfg.get("abstain_slot") != 255 or cfg.get("answer_token_id") != 248082
                or c.get("rms_norm_eps") != 1e-6 or rp.get("rope_theta") != 1e7
                or rp.get("partial_rotary_factor") != 0.25 or rp.get("rope_type") != "default"):
            raise OpenThaiError("unsupported OpenThai head/normalization/rotary configuration")
    if c.get("linear_num_key_heads") != c.get("linear_num_value_heads") or \
            c.get("linear_key_head_dim") != c.get("linear_value_head_dim"):
        raise OpenThaiError("DeltaNet key and value heads must match")
    rp = c.get("rope_parameters") or {}
    hd = int(c["head_dim"])
    types = list(c.get("layer_types") or [])
    if len(types) != int(c["num_hidden_layers"]) or any(t not in ("full_attention", "linear_attention")
                                                           for t in types):
        raise OpenThaiError("unsupported OpenThai layer type")
    max_tokens = int(meta.get("openthai.context_length", 4096))
    max_state = int(meta.get("openthai.state_length", 2048))
    if not 32 <= max_tokens <= 8192 or not 1 <= max_state <= max_tokens:
        raise OpenThaiError("invalid OpenThai sequence budgets")
    return {"d": int(c["hidden_size"]), "ffn": int(c["intermediate_size"]), "heads": int(c["num_attention_heads"]),
            "kv_heads": int(c["num_key_value_heads"]), "head_dim": hd,
            "rot": int(round(hd * float(rp.get("partial_rotary_factor", 0.25)))),
            "theta": float(rp.get("rope_theta", 1e7)), "lin_heads": int(c["linear_num_key_heads"]),
            "lin_dim": int(c["linear_key_head_dim"]), "vocab": int(c["vocab_size"]), "layer_types": types,
            "slots": int(cfg.get("n_slots", 256)), "answer_token_id": int(cfg.get("answer_token_id", 248082)),
            "max_tokens": max_tokens, "max_state": max_state}


def load_weights(path: str, strict: bool = True, decode=None) -> dict:
    """Config and F32 weights of an OpenThai GGUF under its tensor names
    (model.rs:103-174), with `temperature` = exp(log_temperature).
    Block-quantised tensors need `decode(kind, raw_bytes)`."""
    from .gguf_meta import read_tensors_f32

    meta, t = read_tensors_f32(path, decode=decode)
    cfg = load_config(meta, strict)
    t["config"] = cfg
    t["temperature"] = np.exp(t["log_temperature"].astype(np.float32)).astype(np.float32)
    return t


class Model:
    """An OpenThai GGUF on one GPU (laya_openthai_open / _forward / _close):
    the config from the file's `openthai.config` (checked as `load_config`),
    the per-kind temperatures from `log_temperature`, and `decide(tok, req)`
    running every permutation pass of a request through the GPU forward and
    the calibrated slot decoding (decision.rs:243-391)."""

    def __init__(self, path: str, device: int = 0, strict: bool = True):
        import ctypes

        from . import _lib
        from .gguf_meta import read_tensors_f32

        meta, t = read_tensors_f32(path, names={"log_temperature"})
        self.config = c = load_config(meta, strict)
        if "log_temperature" not in t or t["log_temperature"].size != 3:
            raise OpenThaiError("missing or invalid tensor log_temperature")
        self.temperature = np.exp(t["log_temperature"].astype(np.float32)).astype(np.float32)
        self._full = np.array([ty == "full_attention" for ty in c["layer_types"]], np.uint8)
        eps = float(json.loads(meta["openthai.config"]).get("text_config", {}).get("rms_norm_eps", 1e-6))
        cfg = _lib.OtConfig(c["d"], c["ffn"], c["heads"], c["kv_heads"], c["head_dim"], c["rot"], c["lin_heads"],
                            c["lin_dim"], c["vocab"], c["slots"], len(c["layer_types"]), c["theta"], eps,
                            self._full.ctypes.data_as(ctypes.c_void_p))
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().laya_openthai_open(path.encode(), device, ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        from . import _lib

        if self._h:
            _lib.lib().laya_openthai_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, ids, positions) -> np.ndarray:
        """Slot logits [len(positions)][slots] of one encoded pass."""
        import ctypes

        from . import _lib

        if not self._h:
            raise OpenThaiError("model is closed")
        ids = np.ascontiguousarray(np.asarray(ids, np.int32))
        pos = np.ascontiguousarray(np.asarray(positions, np.int32))
        out = np.zeros((len(pos), self.config["slots"]), np.float32)
        _lib.check(_lib.lib().laya_openthai_forward(self._h, ids.ctypes.data_as(ctypes.c_void_p), len(ids),
                                                    pos.ctypes.data_as(ctypes.c_void_p), len(pos),
                                                    out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def forward_batch(self, passes) -> list:
        """Slot logits of several encoded passes [(ids, positions), ...] in
        one forward (laya_openthai_forward_batch): each pass is its own causal
        sequence.  A model without a native handle (a forward stood in by
        another implementation) runs the passes one at a time."""
        import ctypes

        from . import _lib

        if not self._h:
            return [self.forward(ids, pos) for ids, pos in passes]
        if len(passes) == 1:
            return [self.forward(*passes[0])]
        ids = [np.asarray(i, np.int32) for i, _ in passes]
        for (i, p) in zip(ids, (p for _, p in passes)):
            if len(i) == 0 or any(not 0 <= int(x) < len(i) for x in p):
                # a position past its own pass would read the next pass's row
                raise _lib.LayaError(_lib.E_INVALID, "invalid OpenThai token sequence")
        lens = np.ascontiguousarray([len(i) for i in ids], np.int32)
        offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        allids = np.ascontiguousarray(np.concatenate(ids))
        pos = [np.asarray(p, np.int64) for _, p in passes]
        allpos = np.ascontiguousarray(np.concatenate([p + o for p, o in zip(pos, offs)]).astype(np.int32))
        out = np.zeros((len(allpos), self.config["slots"]), np.float32)
        _lib.check(_lib.lib().laya_openthai_forward_batch(
            self._h, allids.ctypes.data_as(ctypes.c_void_p), lens.ctypes.data_as(ctypes.c_void_p), len(lens),
            allpos.ctypes.data_as(ctypes.c_void_p), len(allpos), out.ctypes.data_as(ctypes.c_void_p)))
        bounds = np.cumsum([0] + [len(p) for p in pos])
        return [out[bounds[i]:bounds[i + 1]] for i in range(len(passes))]

    info = {"architecture": "openthai_systemone"}

    def layers(self) -> int:
        return len(self.config["layer_types"])

    def _encode(self, tok, req, qs, n, p) -> Encoded:
        c = self.config
        return encode(tok, req, qs, n, p, c["answer_token_id"], c["max_tokens"], c["max_state"])

    def validate(self, tok, req: dict) -> None:
        """validate (decision.rs:234-242): the questions, then every
        permutation pass's prompt against the context budget (option order
        can change the token count)."""
        qs = questions(req)
        n = permutation_count(req, qs)
        for p in range(n):
            self._encode(tok, req, qs, n, p)

    def respond(self, tok, req: dict, raw: bool = False, canceled=None) -> dict:
        """decide (decision.rs:243-390): every permutation pass through the
        forward, the calibrated slot decoding, and the result object: model,
        answers, usage (input tokens of the first pass, permutations, whether
        the state was truncated, latency), the request's `id` if it has one,
        and with `raw` each pass's input ids, answer positions and logits.
        `canceled()` is polled before the passes run (LayaError E_CANCELED):
        once before the single batched GPU forward of all passes, or before
        each pass when the forward is another implementation's."""
        from ._lib import E_CANCELED, LayaError

        start = time.perf_counter()
        qs = questions(req)
        n = permutation_count(req, qs)
        passes, debug, tokens, truncated = [], [], 0, False
        if canceled is not None and canceled():
            raise LayaError(E_CANCELED, "request canceled")
        enc = [self._encode(tok, req, qs, n, p) for p in range(n)]
        tokens = len(enc[0].ids)
        # every permutation pass in one forward on the GPU (one at a time
        # when the forward is another implementation's)
        if self._h:
            all_logits = self.forward_batch([(e.ids, e.positions) for e in enc])
        else:
            all_logits = []
            for e in enc:
                if canceled is not None and canceled():
                    raise LayaError(E_CANCELED, "request canceled")
                all_logits.append(self.forward(e.ids, e.positions))
        for e, logits in zip(enc, all_logits):
            truncated |= e.truncated
            passes.append((logits, e.order))
            if raw:
                debug.append({"input_ids": [int(v) for v in e.ids], "answer_positions": [int(v) for v in e.positions],
                              "logits": [float(v) for v in logits.reshape(-1)]})
        out = {"model": "openthai-systemone", "answers": decide(qs, passes, self.temperature),
               "usage": {"input_tokens": tokens, "output_tokens": 0, "permutations": n,
                         "truncated_state": truncated, "latency_ms": int((time.perf_counter() - start) * 1000)}}
        if req.get("id") is not None:
            out["id"] = req["id"]
        if raw:
            out["_raw"] = debug
        return out

    def decide(self, tok, req: dict) -> dict:
        """The answers of `respond`: {question id: answer}."""
        return self.respond(tok, req)["answers"]
