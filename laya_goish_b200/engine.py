"""Python host interface of the decision hot path, mirroring the reference
engine's plugin boundary:

* ``Engine(path, devices)``      — Engine::new / models::load (src/engine.rs:16-39)
* ``Engine.layers()``             — Backend::layers (src/models/mod.rs:14)
* ``Engine.validate(...)``        — Backend::validate (src/models/mod.rs:15)
* ``Engine.decide(...)``          — Backend::decide for one request (src/models/mod.rs:16-22)
* ``Engine.decide_batch(...)``    — /v1/decide/batch: many requests sharing the questions
                                     (src/server.rs:235-332), sharded across GPUs
* ``dequantize`` / ``matrix_apply`` — gguf::decode (src/gguf.rs:250-336) and
                                     Matrix::apply (src/tensor.rs:10-39)

Requests arrive as token ids (the reference's tokenizer and prompt templates
sit above this boundary).  Every call goes through liblaya_cuda.so; errors
raise LayaError carrying the library's status code and message.
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Callable, Sequence

import numpy as np

from . import _lib
from ._lib import CHOICE, NOUL, SCORE, LayaError, check  # noqa: F401

KINDS = {"choice": CHOICE, "score": SCORE, "noul": NOUL}
KIND_NAMES = {v: k for k, v in KINDS.items()}


def _ptr(a: np.ndarray, ctype=ctypes.c_int32):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


@dataclasses.dataclass
class Question:
    """kind: "choice" | "score" | "noul"; options: (k,) single tokens or (k, L)
    continuations; suffix: ids appended to every prompt before reading."""

    kind: str | int
    options: Sequence
    suffix: Sequence = ()

    def arrays(self):
        opts = np.ascontiguousarray(np.asarray(self.options, dtype=np.int32))
        if opts.ndim == 1:
            opts = opts.reshape(-1, 1)
        suf = np.ascontiguousarray(np.asarray(self.suffix, dtype=np.int32).reshape(-1))
        kind = KINDS[self.kind] if isinstance(self.kind, str) else int(self.kind)
        return kind, opts, suf


class _BatchArgs:
    """Keeps the numpy buffers of a laya_batch alive for the duration of a call."""

    def __init__(self, prompts, questions):
        prompts = [np.asarray(p, dtype=np.int32).reshape(-1) for p in prompts]
        self.offsets = np.zeros(len(prompts) + 1, np.int64)
        if prompts:
            self.offsets[1:] = np.cumsum([len(p) for p in prompts])
        self.ids = np.ascontiguousarray(np.concatenate(prompts) if prompts else np.zeros(1, np.int32))
        self.qarrays = [q.arrays() for q in questions]
        self.qs = (_lib.Question * max(1, len(questions)))()
        for i, (kind, opts, suf) in enumerate(self.qarrays):
            self.qs[i] = _lib.Question(kind, opts.shape[0], opts.shape[1], _ptr(opts), len(suf),
                                       _ptr(suf) if len(suf) else None)
        self.batch = _lib.Batch(len(prompts), _ptr(self.ids), _ptr(self.offsets, ctypes.c_int64), len(questions),
                                self.qs)


def answer_dict(a: _lib.Answer) -> dict:
    k = a.n_options
    d = {"type": KIND_NAMES[a.kind], "probabilities": list(a.probabilities[:k]), "logits": list(a.logits[:k]),
         "confidence": a.confidence}
    if a.kind == CHOICE:
        d["choice"] = a.choice
    elif a.kind == SCORE:
        d["score"] = a.score
    else:
        d["noul"] = a.noul
    return d


class Engine:
    """A GGUF decoder loaded as one immutable weight replica per listed GPU."""

    def __init__(self, path: str | None = None, devices: Sequence[int] = (0,), image: bytes | None = None):
        L = _lib.lib()
        devs = np.ascontiguousarray(np.asarray(devices, dtype=np.int32))
        h = ctypes.c_void_p()
        if image is not None:
            buf = np.frombuffer(image, dtype=np.uint8)
            check(L.laya_open_memory(buf.ctypes.data_as(ctypes.c_void_p), len(buf), devs.ctypes.data_as(ctypes.c_void_p),
                                     len(devs), ctypes.byref(h)))
        else:
            check(L.laya_open(path.encode(), devs.ctypes.data_as(ctypes.c_void_p), len(devs), ctypes.byref(h)))
        self._h = h
        info = _lib.ModelInfo()
        check(L.laya_info(self._h, ctypes.byref(info)))
        self.info = {f: getattr(info, f) for f, _ in _lib.ModelInfo._fields_}
        self.info["architecture"] = info.architecture.decode()

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().laya_close(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def layers(self) -> int:
        return check(_lib.lib().laya_layers(self._h))

    def validate(self, prompts, questions) -> None:
        args = _BatchArgs(prompts, questions)
        check(_lib.lib().laya_validate(self._h, ctypes.byref(args.batch)))

    def decide_batch(self, prompts, questions, canceled: Callable[[], bool] | None = None, raw: bool = False):
        """Answers for every (request, question), request-major: list of lists of dicts
        (or the raw laya_answer array when raw=True)."""
        args = _BatchArgs(prompts, questions)
        n = len(prompts) * len(questions)
        out = (_lib.Answer * max(1, n))()
        cb = _lib.CANCEL_FN(lambda _u: int(bool(canceled()))) if canceled else _lib.CANCEL_FN()
        check(_lib.lib().laya_decide_batch(self._h, ctypes.byref(args.batch), out, cb, None))
        if raw:
            return out
        nq = len(questions)
        return [[answer_dict(out[i * nq + j]) for j in range(nq)] for i in range(len(prompts))]

    def decide(self, prompt, questions, canceled=None):
        return self.decide_batch([prompt], questions, canceled)[0]

    def decode(self, contexts, steps: int):
        """Greedy decode: returns (tokens [n, steps], {"prefill_ms", "decode_ms"})."""
        args = _BatchArgs(contexts, [])
        out = np.zeros((len(contexts), steps), np.int32)
        stats = np.zeros(2, np.float32)
        check(_lib.lib().laya_decode(self._h, args.ids.ctypes.data_as(ctypes.c_void_p),
                                     args.offsets.ctypes.data_as(ctypes.c_void_p), len(contexts), steps,
                                     out.ctypes.data_as(ctypes.c_void_p), stats.ctypes.data_as(ctypes.c_void_p)))
        return out, {"prefill_ms": float(stats[0]), "decode_ms": float(stats[1])}

    def forward(self, ids, read) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(ids, np.int32))
        read = np.ascontiguousarray(np.asarray(read, np.int32))
        out = np.zeros((len(read), self.info["d_model"]), np.float32)
        check(_lib.lib().laya_forward(self._h, ids.ctypes.data_as(ctypes.c_void_p), len(ids),
                                      read.ctypes.data_as(ctypes.c_void_p), len(read),
                                      out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def tensor(self, name: str, count: int) -> np.ndarray:
        out = np.zeros(count, np.float32)
        check(_lib.lib().laya_tensor_f32(self._h, name.encode(), out.ctypes.data_as(ctypes.c_void_p), count))
        return out

    def timing(self) -> dict:
        """Device time, launches and host<->device bytes of the last decide/decode call."""
        t = _lib.Timing()
        check(_lib.lib().laya_last_timing(self._h, ctypes.byref(t)))
        return {"device_ms": t.device_ms, "launches": t.launches, "h2d_bytes": t.h2d_bytes, "d2h_bytes": t.d2h_bytes}

    def profile(self, enable: bool = True) -> None:
        check(_lib.lib().laya_profile_enable(self._h, int(enable)))

    def profile_read(self) -> dict:
        buf = (_lib.ProfileEntry * 64)()
        n = check(_lib.lib().laya_profile_read(self._h, buf, 64))
        return {buf[i].name.decode(): (buf[i].launches, buf[i].total_ms) for i in range(min(n, 64))}


def dequantize(kind: int, raw, device: int = 0) -> np.ndarray:
    """gguf::decode on the GPU: GGUF block bytes → float32, bit-exact."""
    b = np.ascontiguousarray(np.frombuffer(bytes(raw), np.uint8) if not isinstance(raw, np.ndarray) else raw, np.uint8)
    block, size = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210)}[kind]
    out = np.zeros(len(b) // size * block, np.float32)
    check(_lib.lib().laya_dequantize(device, kind, b.ctypes.data_as(ctypes.c_void_p), len(b),
                                     out.ctypes.data_as(ctypes.c_void_p)))
    return out


def matrix_apply(kind: int, w_bytes, rows: int, cols: int, x, bias=None, device: int = 0) -> np.ndarray:
    """Matrix::apply on the tcgen05 GEMM: x [m][cols] · W^T (+bias) → [m][rows]."""
    w = np.ascontiguousarray(np.frombuffer(bytes(w_bytes), np.uint8) if not isinstance(w_bytes, np.ndarray) else w_bytes, np.uint8)
    x = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, cols))
    out = np.zeros((x.shape[0], rows), np.float32)
    b = None if bias is None else np.ascontiguousarray(np.asarray(bias, np.float32))
    check(_lib.lib().laya_matrix_apply(device, kind, w.ctypes.data_as(ctypes.c_void_p), rows, cols,
                                       x.ctypes.data_as(ctypes.c_void_p), x.shape[0],
                                       None if b is None else b.ctypes.data_as(ctypes.c_void_p),
                                       out.ctypes.data_as(ctypes.c_void_p)))
    return out


def gated_delta(qkv, a, b, dt, alog, nh: int, hk: int, device: int = 0) -> np.ndarray:
    """OpenThai's gated DeltaNet recurrence on the GPU (Delta::run,
    src/models/openthai/model.rs:322-355): qkv [s][3 nh hk] after the
    convolution and SiLU, a / b [s][nh], dt / A_log [nh] -> [s][nh hk]."""
    q = np.ascontiguousarray(np.asarray(qkv, np.float32))
    s = q.shape[0]
    arrs = [np.ascontiguousarray(np.asarray(v, np.float32)) for v in (a, b, dt, alog)]
    out = np.zeros((s, nh * hk), np.float32)
    check(_lib.lib().laya_gated_delta(device, q.ctypes.data_as(ctypes.c_void_p),
                                      *[v.ctypes.data_as(ctypes.c_void_p) for v in arrs], s, nh, hk,
                                      out.ctypes.data_as(ctypes.c_void_p)))
    return out


def gated_attention(qgate, k, v, qn, kn, H: int, KV: int, hd: int, rot: int, theta: float,
                    device: int = 0) -> np.ndarray:
    """OpenThai's gated full attention after the projections on the GPU
    (Full::run, src/models/openthai/model.rs:248-296): qgate [s][H 2hd], k / v
    [s][KV hd], q / k norm weights [hd] -> [s][H hd] before o_proj."""
    q = np.ascontiguousarray(np.asarray(qgate, np.float32))
    s = q.shape[0]
    arrs = [np.ascontiguousarray(np.asarray(a, np.float32)) for a in (k, v, qn, kn)]
    out = np.zeros((s, H * hd), np.float32)
    check(_lib.lib().laya_gated_attention(device, q.ctypes.data_as(ctypes.c_void_p),
                                          *[a.ctypes.data_as(ctypes.c_void_p) for a in arrs], s, H, KV, hd, rot,
                                          theta, out.ctypes.data_as(ctypes.c_void_p)))
    return out


def gated_delta_mixer(raw, z, a, b, conv, dt, alog, normw, nh: int, hk: int, device: int = 0) -> np.ndarray:
    """OpenThai's DeltaNet mixer after its projections on the GPU (Delta::run,
    src/models/openthai/model.rs:309-360): raw [s][3 nh hk], z [s][nh hk],
    a / b [s][nh], conv [3 nh hk][4], dt / A_log [nh], norm [hk] -> [s][nh hk]
    before out_proj."""
    r = np.ascontiguousarray(np.asarray(raw, np.float32))
    s = r.shape[0]
    arrs = [np.ascontiguousarray(np.asarray(v, np.float32)) for v in (z, a, b, conv, dt, alog, normw)]
    out = np.zeros((s, nh * hk), np.float32)
    check(_lib.lib().laya_gated_delta_mixer(device, r.ctypes.data_as(ctypes.c_void_p),
                                            *[v.ctypes.data_as(ctypes.c_void_p) for v in arrs], s, nh, hk,
                                            out.ctypes.data_as(ctypes.c_void_p)))
    return out
