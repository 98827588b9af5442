"""GGUF v3 metadata reader (header and key/value section only).

The device loader parses the container natively (csrc/gguf.cpp) and skips
array values; the host tokenizer needs them (`tokenizer.ggml.tokens`,
`.merges`, `.token_type`), so this reads the same layout in Python:
magic "GGUF", version 3, tensor count, KV count, then per KV a string key,
a u32 value type and the value (src/gguf.rs:48-79, 95-125).  Tensors are
not read.
"""
from __future__ import annotations

import mmap
import struct

_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
MAX_ARRAY = 1 << 24


class GGUFError(ValueError):
    pass


class _Reader:
    def __init__(self, buf):
        self.b = buf
        self.p = 0

    def take(self, n: int):
        if n < 0 or self.p + n > len(self.b):
            raise GGUFError("truncated GGUF")
        v = self.b[self.p:self.p + n]
        self.p += n
        return v

    def fmt(self, f: str):
        return struct.unpack(f, self.take(struct.calcsize(f)))[0]

    def string(self) -> str:
        n = self.fmt("<Q")
        if n > len(self.b):
            raise GGUFError("GGUF string length overflow")
        try:
            return bytes(self.take(n)).decode("utf-8")
        except UnicodeDecodeError as e:
            raise GGUFError("invalid GGUF UTF-8") from e

    def value(self, t: int, depth: int = 0):
        if depth > 4:
            raise GGUFError("GGUF metadata nesting too deep")
        if t in _SCALARS:
            return self.fmt(_SCALARS[t])
        if t == 8:
            return self.string()
        if t == 9:
            et, n = self.fmt("<I"), self.fmt("<Q")
            if n > MAX_ARRAY:
                raise GGUFError("GGUF array too large")
            if et in _SCALARS:  # one unpack for the whole numeric array
                f = _SCALARS[et]
                size = struct.calcsize(f)
                return list(struct.unpack("<%d%s" % (n, f[1]), self.take(n * size)))
            return [self.value(et, depth + 1) for _ in range(n)]
        raise GGUFError(f"unsupported GGUF metadata type {t}")


def read_metadata(path_or_bytes) -> dict:
    """All metadata key/values of a GGUF file (path) or image (bytes)."""
    if isinstance(path_or_bytes, (bytes, bytearray, memoryview)):
        return _parse(memoryview(path_or_bytes))
    with open(path_or_bytes, "rb") as f:
        with mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as m:
            mv = memoryview(m)
            try:
                return _parse(mv)
            finally:
                mv.release()


def _parse(buf, tensors: bool = False):
    r = _Reader(buf)
    try:
        if bytes(r.take(4)) != b"GGUF":
            raise GGUFError("not a GGUF file")
        if r.fmt("<I") != 3:
            raise GGUFError("unsupported GGUF version")
        n_t = r.fmt("<Q")
        n_kv = r.fmt("<Q")
        if n_kv > 1 << 20 or n_t > 1 << 20:
            raise GGUFError("too many GGUF entries")
        out = {}
        for _ in range(n_kv):
            k = r.string()
            out[k] = r.value(r.fmt("<I"))
        if not tensors:
            return out
        infos = []
        for _ in range(n_t):
            name = r.string()
            nd = r.fmt("<I")
            if nd > 4:
                raise GGUFError("GGUF tensor rank above 4")
            dims = [r.fmt("<Q") for _ in range(nd)]
            kind, off = r.fmt("<I"), r.fmt("<Q")
            infos.append((name, dims, kind, off))
        align = int(out.get("general.alignment", 32))
        base = (r.p + align - 1) // align * align
        return out, infos, base
    finally:
        r.b = None


_ELEM = {0: (4, "<f4"), 1: (2, "<f2")}
# (elements, bytes) per block of the block-quantised GGML types (src/gguf.rs:81-93)
_BLOCK = {2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


def read_tensors_f32(path: str, names=None, decode=None) -> tuple[dict, dict]:
    """Metadata and the F32 / F16 tensors of a GGUF file (all of them, or
    those in `names`) as F32 arrays of shape dims reversed (GGUF dims are
    innermost first: a matrix [K, N] is N rows of K).  Block-quantised
    tensors (Q4_0, Q8_0, Q4_K, Q6_K) go through `decode(kind, raw_bytes)`
    when one is given; without it, and for other types, GGUFError."""
    import numpy as np

    with open(path, "rb") as f:
        with mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as data:
            mv = memoryview(data)
            try:
                meta, infos, base = _parse(mv, tensors=True)
                out = {}
                for name, dims, kind, off in infos:
                    if names is not None and name not in names:
                        continue
                    n = 1
                    for d in dims:
                        n *= d
                    start = base + off
                    if kind in _BLOCK and decode is not None:
                        block, bsize = _BLOCK[kind]
                        if n % block or start + n // block * bsize > len(data):
                            raise GGUFError(f"{name}: tensor data out of range")
                        a = np.asarray(decode(kind, bytes(mv[start:start + n // block * bsize])), np.float32)
                        out[name] = a.reshape(list(reversed(dims))) if dims else a
                        continue
                    if kind not in _ELEM:
                        raise GGUFError(f"{name}: tensor type {kind} is not F32/F16")
                    size, dt = _ELEM[kind]
                    if start + n * size > len(data):
                        raise GGUFError(f"{name}: tensor data out of range")
                    a = np.frombuffer(mv[start:start + n * size], dtype=dt, count=n).astype(np.float32)
                    out[name] = a.reshape(list(reversed(dims))) if dims else a
            finally:
                mv.release()
    return meta, out
