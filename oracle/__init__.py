"""ctypes bindings for the CPU oracle (oracle.c).  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, as the parity checker.  The product library never uses it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "liblaya_oracle.so")


def build() -> str:
    """Compile liblaya_oracle.so with its Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB


class Question(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("n_options", ctypes.c_int32),
                ("option_len", ctypes.c_int32), ("suffix_len", ctypes.c_int32),
                ("options", ctypes.POINTER(ctypes.c_int32)),
                ("suffix", ctypes.POINTER(ctypes.c_int32))]


class Answer(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("n_options", ctypes.c_int32),
                ("choice", ctypes.c_int32), ("score", ctypes.c_float),
                ("noul", ctypes.c_float), ("confidence", ctypes.c_float),
                ("probabilities", ctypes.c_float * 16), ("logits", ctypes.c_float * 16)]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        srcs = [os.path.join(_HERE, f) for f in ("oracle.c", "openthai.c", "oracle.h")]
        if not os.path.exists(_LIB) or os.path.getmtime(_LIB) < max(os.path.getmtime(f) for f in srcs):
            build()
        L = ctypes.CDLL(_LIB)
        P = ctypes.c_void_p
        L.or_half.restype = ctypes.c_float
        L.or_half.argtypes = [ctypes.c_uint16]
        L.or_decode.argtypes = [ctypes.c_uint32, P, ctypes.c_size_t, P]
        L.or_gguf_check.argtypes = [P, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
        L.or_matrix_apply.argtypes = [P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P, ctypes.c_int, P]
        L.or_softmax.argtypes = [P, ctypes.c_int, P]
        L.or_confidence.restype = ctypes.c_float
        L.or_confidence.argtypes = [P, ctypes.c_int]
        L.or_model_load.restype = P
        L.or_model_load.argtypes = [P, ctypes.c_size_t, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        L.or_model_free.argtypes = [P]
        L.or_model_dim.argtypes = [P, ctypes.c_int]
        L.or_forward.argtypes = [P, P, ctypes.c_int, P, ctypes.c_int, P]
        L.or_cache_new.restype = P
        L.or_cache_new.argtypes = [P, ctypes.c_int]
        L.or_cache_free.argtypes = [P]
        L.or_cache_len.argtypes = [P]
        L.or_cache_truncate.argtypes = [P, ctypes.c_int]
        L.or_cache_forward.argtypes = [P, P, P, ctypes.c_int, P, ctypes.c_int, P]
        L.or_cache_fill_timing.argtypes = [P, P, ctypes.c_int]
        L.or_model_attn_threads.argtypes = [P, ctypes.c_int]
        i = ctypes.c_int
        L.or_ot_full.argtypes = [P, i, i, i, i, i, i, ctypes.c_float, P, P, P, P, P, P, i, P]
        L.or_ot_delta.argtypes = [P, i, i, i, i, P, P, P, P, P, P, P, P, P, i, P]
        L.or_ot_delta_core.argtypes = [P, P, P, P, P, i, i, i, P]
        L.or_ot_full_core.argtypes = [P, P, P, P, P, i, i, i, i, i, ctypes.c_float, P]
        L.or_ot_delta_mid.argtypes = [P, P, P, P, P, P, P, P, i, i, i, P]
        L.or_head.argtypes = [P, P, ctypes.c_int, P, ctypes.c_int, P]
        L.or_decide.argtypes = [P, P, ctypes.c_int, ctypes.POINTER(Question), ctypes.POINTER(Answer)]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def half(x: int) -> float:
    return lib().or_half(x)


def layout(kind: int) -> tuple[int, int]:
    return {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210)}[kind]


def decode(kind: int, raw: bytes | np.ndarray) -> np.ndarray:
    b = np.frombuffer(bytes(raw), dtype=np.uint8) if not isinstance(raw, np.ndarray) else np.ascontiguousarray(raw, dtype=np.uint8)
    block, size = layout(kind)
    out = np.zeros(len(b) // size * block, dtype=np.float32)
    if lib().or_decode(kind, _p(b), len(b), _p(out)) != 0:
        raise ValueError(f"unsupported kind {kind}")
    return out


def gguf_check(blob: bytes) -> str | None:
    """None when the image parses, else the loader's error message."""
    b = np.frombuffer(blob, dtype=np.uint8) if blob else np.zeros(1, np.uint8)
    err = ctypes.create_string_buffer(256)
    rc = lib().or_gguf_check(_p(b), len(blob), err, 256)
    return None if rc == 0 else err.value.decode()


def matrix_apply(w: np.ndarray, x: np.ndarray, bias: np.ndarray | None = None, threads: int = 1) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = w.shape
    m = x.size // cols
    out = np.zeros((m, rows), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().or_matrix_apply(_p(w), rows, cols, _p(x), m, None if b is None else _p(b), threads, _p(out))
    return out


def softmax(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    p = np.zeros_like(x)
    lib().or_softmax(_p(x), len(x), _p(p))
    return p


def confidence(p) -> float:
    p = np.ascontiguousarray(p, np.float32)
    return lib().or_confidence(_p(p), len(p))


class Model:
    """The oracle decoder: GGUF image → F32 weights (as the reference loads them)."""

    def __init__(self, blob: bytes | np.ndarray, threads: int = 1, attn_threads: int = 1):
        """threads: Matrix::apply workers.  attn_threads: workers of the
        attention loop; 1 keeps the reference's single-threaded loop (the
        timed baseline), more give the same bits sooner (the checkers)."""
        self._buf = np.frombuffer(blob, dtype=np.uint8) if not isinstance(blob, np.ndarray) else blob
        err = ctypes.create_string_buffer(256)
        h = lib().or_model_load(_p(self._buf), len(self._buf), threads, err, 256)
        if not h:
            raise ValueError(err.value.decode())
        self.h = ctypes.c_void_p(h)
        L = lib()
        L.or_model_attn_threads(self.h, attn_threads)
        self.d, self.layers, self.vocab, self.heads, self.kv, self.hd, self.ffn, self.ctx = (
            L.or_model_dim(self.h, i) for i in range(8))

    def close(self):
        if self.h:
            lib().or_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def forward(self, ids, read) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        read = np.ascontiguousarray(read, np.int32)
        out = np.zeros((len(read), self.d), np.float32)
        if lib().or_forward(self.h, _p(ids), len(ids), _p(read), len(read), _p(out)):
            raise ValueError("invalid token sequence")
        return out

    def cache(self, capacity: int) -> "Cache":
        """A K/V cache over this model for up to `capacity` tokens."""
        return Cache(self, capacity)

    def greedy(self, ctx, steps: int):
        """Greedy decode with the K/V cache: the context once, then one token
        per step (argmax over the full vocabulary, ties to the lowest id).
        Returns (tokens, top-2 logit margins)."""
        c = self.cache(len(ctx) + steps)
        h = c.forward(ctx, [len(ctx) - 1])
        toks, margins = [], []
        for s in range(steps):
            logits = self.head(h)[0]
            order = np.argsort(-logits, kind="stable")
            toks.append(int(order[0]))
            margins.append(float(logits[order[0]] - logits[order[1]]))
            if s + 1 < steps:
                h = c.forward([toks[-1]], [0])
        c.close()
        return toks, margins

    def head(self, hidden, cand=None) -> np.ndarray:
        hidden = np.ascontiguousarray(hidden, np.float32).reshape(-1, self.d)
        n = 0 if cand is None else len(cand)
        c = np.ascontiguousarray(cand if cand is not None else [0], np.int32)
        out = np.zeros((hidden.shape[0], n or self.vocab), np.float32)
        if lib().or_head(self.h, _p(hidden), hidden.shape[0], _p(c), n, _p(out)):
            raise ValueError("invalid candidate id")
        return out

    def decide(self, ids, kind: int, options, suffix=()) -> dict:
        ids = np.ascontiguousarray(ids, np.int32)
        opts = np.ascontiguousarray(options, np.int32)
        if opts.ndim == 1:
            opts = opts.reshape(-1, 1)
        suf = np.ascontiguousarray(suffix if len(suffix) else [0], np.int32)
        q = Question(kind, opts.shape[0], opts.shape[1], len(suffix),
                     opts.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                     suf.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
        a = Answer()
        rc = lib().or_decide(self.h, _p(ids), len(ids), ctypes.byref(q), ctypes.byref(a))
        if rc:
            raise ValueError(f"oracle decide failed ({rc})")
        k = a.n_options
        return {"kind": a.kind, "choice": a.choice, "score": a.score, "noul": a.noul,
                "confidence": a.confidence, "probabilities": list(a.probabilities[:k]),
                "logits": list(a.logits[:k])}


class Cache:
    """Model::forward extended token by token: forward() appends ids at the
    next positions and returns the final-normed hidden rows at `read`
    (indices into the appended ids); truncate(n) drops positions >= n, so a
    shared prefix is computed once and branched.  Same bits as one forward
    over the whole sequence."""

    def __init__(self, model: Model, capacity: int):
        self.m = model
        h = lib().or_cache_new(model.h, capacity)
        if not h:
            raise ValueError("cache capacity out of range")
        self.h = ctypes.c_void_p(h)

    def __len__(self):
        return lib().or_cache_len(self.h)

    def forward(self, ids, read) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        read = np.ascontiguousarray(read, np.int32)
        out = np.zeros((len(read), self.m.d), np.float32)
        if lib().or_cache_forward(self.m.h, self.h, _p(ids), len(ids), _p(read), len(read), _p(out)):
            raise ValueError("invalid token sequence or cache overflow")
        return out

    def fill_for_timing(self, n: int) -> None:
        """Timing only: positions 0..n-1 hold arbitrary K/V values."""
        if lib().or_cache_fill_timing(self.h, self.m.h, n):
            raise ValueError("fill past the cache capacity")

    def truncate(self, n: int) -> None:
        if lib().or_cache_truncate(self.h, n):
            raise ValueError("truncate past the cached length")

    def close(self):
        if self.h:
            lib().or_cache_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def ot_full(x, wq, wk, wv, wo, qn, kn, H, KV, hd, rot, theta, threads=4) -> np.ndarray:
    """OpenThai gated full attention of one sequence x [s][d] (Full::run)."""
    x = _f32(x)
    s, d = x.shape
    args = [_f32(a) for a in (wq, wk, wv, wo, qn, kn)]
    out = np.zeros((s, d), np.float32)
    rc = lib().or_ot_full(x.ctypes.data, s, d, H, KV, hd, rot, theta, *[a.ctypes.data for a in args], threads,
                          out.ctypes.data)
    if rc:
        raise ValueError(f"or_ot_full failed ({rc})")
    return out


def ot_delta(x, wqkv, wz, wa, wb, wo, conv, dt, alog, normw, nh, hk, threads=4) -> np.ndarray:
    """OpenThai gated DeltaNet mixer of one sequence x [s][d] (Delta::run)."""
    x = _f32(x)
    s, d = x.shape
    args = [_f32(a) for a in (wqkv, wz, wa, wb, wo, conv, dt, alog, normw)]
    out = np.zeros((s, d), np.float32)
    rc = lib().or_ot_delta(x.ctypes.data, s, d, nh, hk, *[a.ctypes.data for a in args], threads, out.ctypes.data)
    if rc:
        raise ValueError(f"or_ot_delta failed ({rc})")
    return out


def ot_delta_core(qkv, a, b, dt, alog, nh, hk) -> np.ndarray:
    """The DeltaNet recurrence alone: qkv [s][3 nh hk] (after conv + SiLU),
    a / b [s][nh], dt / A_log [nh] -> [s][nh hk] before the output norm."""
    qkv = _f32(qkv)
    s = qkv.shape[0]
    args = [_f32(v) for v in (a, b, dt, alog)]
    out = np.zeros((s, nh * hk), np.float32)
    rc = lib().or_ot_delta_core(qkv.ctypes.data, *[v.ctypes.data for v in args], s, nh, hk, out.ctypes.data)
    if rc:
        raise ValueError(f"or_ot_delta_core failed ({rc})")
    return out


def ot_full_core(qgate, k, v, qn, kn, H, KV, hd, rot, theta) -> np.ndarray:
    """Gated attention after the projections: qgate [s][H 2hd], k / v
    [s][KV hd] -> [s][H hd] before o_proj."""
    qgate = _f32(qgate)
    s = qgate.shape[0]
    args = [_f32(a) for a in (k, v, qn, kn)]
    out = np.zeros((s, H * hd), np.float32)
    rc = lib().or_ot_full_core(qgate.ctypes.data, *[a.ctypes.data for a in args], s, H, KV, hd, rot, theta,
                               out.ctypes.data)
    if rc:
        raise ValueError(f"or_ot_full_core failed ({rc})")
    return out


def ot_delta_mid(raw, z, a, b, conv, dt, alog, normw, nh, hk) -> np.ndarray:
    """The DeltaNet mixer after its projections: raw [s][3 nh hk], z [s][nh hk],
    a / b [s][nh] -> [s][nh hk] before out_proj."""
    raw = _f32(raw)
    s = raw.shape[0]
    args = [_f32(v) for v in (z, a, b, conv, dt, alog, normw)]
    out = np.zeros((s, nh * hk), np.float32)
    rc = lib().or_ot_delta_mid(raw.ctypes.data, *[v.ctypes.data for v in args], s, nh, hk, out.ctypes.data)
    if rc:
        raise ValueError(f"or_ot_delta_mid failed ({rc})")
    return out


def _rms(x: np.ndarray, w: np.ndarray, off: float) -> np.ndarray:
    """rms (src/models/openthai/model.rs:84-94) in F32: rows of len(w), eps 1e-6."""
    d = w.shape[0]
    r = x.reshape(-1, d).astype(np.float32)
    dot = np.add.accumulate(r * r, axis=1, dtype=np.float32)[:, -1]  # sequential, as tensor::dot
    scale = (np.float32(1) / np.sqrt(dot / np.float32(d) + np.float32(1e-6))).astype(np.float32)
    return (r * scale[:, None] * (np.float32(off) + w.astype(np.float32))).reshape(x.shape).astype(np.float32)


def ot_forward(m: dict, ids, positions, threads: int = 4) -> np.ndarray:
    """OpenThai Model::forward (src/models/openthai/model.rs:192-241) on
    weights given as a dict of F32 arrays under the OpenThai GGUF tensor
    names, composed from the C mixers and Matrix::apply:
    embedding rows; per layer x += mixer(rms(x, n1, 1)), x += down(silu(gate
    h) * up h) with h = rms(x, n2, 1); the slot head (+ bias) on
    rms(x[positions], norm, 1).  Returns [len(positions)][slots]."""
    c = m["config"]
    H, KV, hd, rot, theta = c["heads"], c["kv_heads"], c["head_dim"], c["rot"], c["theta"]
    nh, hk = c["lin_heads"], c["lin_dim"]
    x = m["model.embed_tokens.weight"][np.asarray(ids)].astype(np.float32)
    for i, kind in enumerate(c["layer_types"]):
        p = f"model.layers.{i}"
        h = _rms(x, m[f"{p}.input_layernorm.weight"], 1.0)
        if kind == "full_attention":
            y = ot_full(h, m[f"{p}.self_attn.q_proj.weight"], m[f"{p}.self_attn.k_proj.weight"],
                        m[f"{p}.self_attn.v_proj.weight"], m[f"{p}.self_attn.o_proj.weight"],
                        m[f"{p}.self_attn.q_norm.weight"], m[f"{p}.self_attn.k_norm.weight"], H, KV, hd, rot, theta,
                        threads)
        else:
            y = ot_delta(h, m[f"{p}.linear_attn.in_proj_qkv.weight"], m[f"{p}.linear_attn.in_proj_z.weight"],
                         m[f"{p}.linear_attn.in_proj_a.weight"], m[f"{p}.linear_attn.in_proj_b.weight"],
                         m[f"{p}.linear_attn.out_proj.weight"], m[f"{p}.linear_attn.conv1d.weight"],
                         m[f"{p}.linear_attn.dt_bias"], m[f"{p}.linear_attn.A_log"],
                         m[f"{p}.linear_attn.norm.weight"], nh, hk, threads)
        x = (x + y).astype(np.float32)
        h = _rms(x, m[f"{p}.post_attention_layernorm.weight"], 1.0)
        g = matrix_apply(m[f"{p}.mlp.gate_proj.weight"], h, threads=threads)
        u = matrix_apply(m[f"{p}.mlp.up_proj.weight"], h, threads=threads)
        act = (g * (np.float32(1) / (np.float32(1) + np.exp(-g))) * u).astype(np.float32)
        x = (x + matrix_apply(m[f"{p}.mlp.down_proj.weight"], act, threads=threads)).astype(np.float32)
    ans = _rms(x[np.asarray(positions)], m["model.norm.weight"], 1.0)
    return matrix_apply(m["slot_head.weight"], ans, m["slot_head.bias"], threads=threads)
