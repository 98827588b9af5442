"""Host tokenizer for text requests: the GGUF byte-level BPE of the reference
(src/tokenizer.rs:17-331), restated over the model file's own vocabulary.

Three pre-tokenizers, chosen by `tokenizer.ggml.pre` as the reference does
(src/tokenizer.rs:19-21):

* "gpt2": ASCII pre-tokenization on bytes — the contractions 's 't 're 've
  'm 'll 'd (case-sensitive), runs of letters / digits / other bytes with one
  optional leading space, whitespace runs that leave their last space to the
  next word (src/tokenizer.rs:139-201);
* "qwen3" (also accepted as "qwen2"): NFC-normalised text split by Unicode
  general category — case-insensitive contractions, an optional non-letter
  prefix before a letter run, single digits, punctuation runs with their
  trailing newlines, whitespace runs (src/tokenizer.rs:204-303);
* "gemma": SentencePiece-style pieces starting at each U+2581 (spaces mapped
  to it, one prepended), with <0xXX> byte fallback (src/tokenizer.rs:123-137).

Every piece is mapped to GPT-2's printable byte alphabet (except gemma) and
merged by BPE: repeatedly the adjacent pair with the lowest merge rank,
leftmost on ties (src/tokenizer.rs:85-118).  Special tokens are cut out first:
at each step the earliest occurrence of any special token, longest first
among those starting at the same place (src/tokenizer.rs:305-331).  Special
tokens are "<...>" / "[...]" tokens of 3+ characters, or for qwen3 the
tokens whose `token_type` is 3 (control) or 4 (user-defined).

Unlike the reference, a vocabulary without `laya.mask_token_id` inside it is
accepted (the decoders here have no mask token); `mask` is then None.
"""
from __future__ import annotations

import unicodedata

from .gguf_meta import read_metadata

MAX_TEXT_BYTES = 1024 * 1024  # src/tokenizer.rs:306-308
CONTRACTIONS = ("'s", "'t", "'re", "'ve", "'m", "'ll", "'d")
# Unicode White_Space (Rust char::is_whitespace)
_WS = frozenset([0x9, 0xA, 0xB, 0xC, 0xD, 0x20, 0x85, 0xA0, 0x1680, *range(0x2000, 0x200B), 0x2028, 0x2029,
                 0x202F, 0x205F, 0x3000])


class TokenizerError(ValueError):
    pass


def byte_alphabet() -> list[str]:
    """GPT-2's byte -> printable character map: bytes 33-126, 161-172 and
    174-255 stand for themselves, the others take code points 256, 257, ...
    in byte order (src/tokenizer.rs:36-51)."""
    out, extra = [], 256
    for b in range(256):
        if 33 <= b <= 126 or 161 <= b <= 172 or 174 <= b <= 255:
            out.append(chr(b))
        else:
            out.append(chr(extra))
            extra += 1
    return out


def _is_ws(c: str) -> bool:
    return ord(c) in _WS


def _letter(c: str) -> bool:
    return unicodedata.category(c) in ("Lu", "Ll", "Lt", "Lm", "Lo")


def _number(c: str) -> bool:
    return unicodedata.category(c) in ("Nd", "Nl", "No")


def _punct(c: str) -> bool:
    return not _is_ws(c) and not _letter(c) and not _number(c)


def _ascii_ws(b: int) -> bool:
    return b in (0x20, 0x09, 0x0D, 0x0A, 0x0B, 0x0C)


def _ascii_cat(b: int) -> int:
    if 65 <= b <= 90 or 97 <= b <= 122:
        return 1
    if 48 <= b <= 57:
        return 2
    if _ascii_ws(b):
        return 0
    return 3


def split_gpt2(data: bytes) -> list[bytes]:
    """ASCII GPT-2 pre-tokenization on bytes (src/tokenizer.rs:139-201)."""
    out, i, n = [], 0, len(data)
    while i < n:
        start, end = i, None
        if data[i] == 0x27:  # '
            for c in CONTRACTIONS:
                if data.startswith(c.encode(), i):
                    end = i + len(c)
                    break
        if end is None:
            j = i + 1 if data[i] == 0x20 and i + 1 < n and not _ascii_ws(data[i + 1]) else i
            c = _ascii_cat(data[j])
            if c != 0:
                k = j + 1
                while k < n and _ascii_cat(data[k]) == c:
                    k += 1
                end = k
            else:
                k = i + 1
                while k < n and _ascii_ws(data[k]):
                    k += 1
                if k < n and k - i > 1:
                    k -= 1
                end = k
        out.append(data[start:end])
        i = end
    return out


def split_qwen(text: str) -> list[bytes]:
    """Unicode-category pre-tokenization of NFC text (src/tokenizer.rs:204-303),
    as UTF-8 byte pieces."""
    s = unicodedata.normalize("NFC", text)
    out, i, n = [], 0, len(s)
    while i < n:
        start, end = i, None
        if s[i] == "'":
            for c in CONTRACTIONS:
                # ASCII case-insensitive match of the suffix
                w = s[i:i + len(c)]
                if len(w) == len(c) and all(x == y or (x.isascii() and x.lower() == y) for x, y in zip(w, c)):
                    end = i + len(c)
                    break
        if end is None:
            c, j = s[i], i
            if c not in "\r\n" and not _letter(c) and not _number(c):
                j += 1
            if j < n and _letter(s[j]):
                j += 1
                while j < n and _letter(s[j]):
                    j += 1
                end = j
        if end is None and _number(s[i]):
            end = i + 1
        if end is None:
            j = i
            if s[j] == " ":
                j += 1
            if j < n and _punct(s[j]):
                j += 1
                while j < n and _punct(s[j]):
                    j += 1
                while j < n and s[j] in "\r\n":
                    j += 1
                end = j
        if end is None and _is_ws(s[i]):
            j, newline = i, None
            while j < n and _is_ws(s[j]):
                if s[j] in "\r\n":
                    newline = j + 1
                j += 1
            end = newline if newline is not None else (j - 1 if j < n and j > i + 1 else j)
        if end is None:
            raise TokenizerError("unsupported Qwen pretokenization character")
        out.append(s[start:end].encode("utf-8"))
        i = end
    return out


class Tokenizer:
    def __init__(self, meta: dict):
        pre = meta.get("tokenizer.ggml.pre", "")
        if pre == "qwen2":
            pre = "qwen3"
        if pre not in ("gpt2", "gemma", "qwen3"):
            raise TokenizerError(f"unsupported tokenizer {pre}")
        tokens = meta.get("tokenizer.ggml.tokens") or []
        if not tokens:
            raise TokenizerError("missing vocabulary")
        self.pre = pre
        self.tokens = list(tokens)
        self.vocab = {t: i for i, t in enumerate(tokens)}  # a repeated token keeps its last id
        self.ranks = {}
        for i, m in enumerate(meta.get("tokenizer.ggml.merges") or []):
            a, sep, b = m.partition(" ")
            if sep:
                self.ranks[(a, b)] = i
        self.bytes = byte_alphabet()
        if pre == "qwen3":
            tt = meta.get("tokenizer.ggml.token_type") or []
            special = [(t, i) for t, i in sorted(self.vocab.items()) if i < len(tt) and tt[i] in (3, 4)]
        else:
            special = [(t, i) for t, i in sorted(self.vocab.items())
                       if len(t.encode()) >= 3 and ((t[0] == "<" and t[-1] == ">") or (t[0] == "[" and t[-1] == "]"))]
        special.sort(key=lambda x: -len(x[0].encode()))  # stable: ties keep token order
        self.special = special
        mask_id = int(meta.get("laya.mask_token_id", 50284))
        self.mask = self.tokens[mask_id] if 0 <= mask_id < len(self.tokens) else None

    @classmethod
    def from_gguf(cls, path_or_bytes) -> "Tokenizer":
        return cls(read_metadata(path_or_bytes))

    def _bpe(self, word: list[str], out: list[int]) -> None:
        while len(word) > 1:
            best = None
            for i in range(len(word) - 1):
                r = self.ranks.get((word[i], word[i + 1]))
                if r is not None and (best is None or r < best[0]):
                    best = (r, i)
            if best is None:
                break
            i = best[1]
            word[i:i + 2] = [word[i] + word[i + 1]]
        for p in word:
            t = self.vocab.get(p)
            if t is not None:
                out.append(t)
            elif self.pre == "gemma":
                for b in p.encode("utf-8"):
                    t = self.vocab.get(f"<0x{b:02X}>")
                    if t is None:
                        raise TokenizerError("missing byte fallback")
                    out.append(t)
            else:
                raise TokenizerError(f"missing BPE piece {p}")

    def _normal(self, s: str, out: list[int]) -> None:
        if self.pre == "gemma":
            s = s.replace(" ", "▁")
            if not s.startswith("▁"):
                s = "▁" + s
            start = 0
            while start < len(s):
                end = s.find("▁", start + 1)
                end = len(s) if end < 0 else end
                self._bpe(list(s[start:end]), out)
                start = end
            return
        pieces = split_qwen(s) if self.pre == "qwen3" else split_gpt2(s.encode("utf-8"))
        for p in pieces:
            self._bpe([self.bytes[b] for b in p], out)

    def encode(self, s: str) -> list[int]:
        if len(s.encode("utf-8")) > MAX_TEXT_BYTES:
            raise TokenizerError("text exceeds 1 MiB")
        out: list[int] = []
        pos = 0
        while pos < len(s):
            found = None
            for t, i in self.special:
                p = s.find(t, pos)
                if p >= 0 and (found is None or p < found[0]):
                    found = (p, len(t), i)
            if found is None:
                self._normal(s[pos:], out)
                break
            self._normal(s[pos:found[0]], out)
            out.append(found[2])
            pos = found[0] + found[1]
        return out

    def decode(self, ids) -> str:
        """Inverse of the byte alphabet for gpt2/qwen3 vocabularies (gemma:
        U+2581 -> space); special tokens are emitted as their text."""
        inv = {c: b for b, c in enumerate(self.bytes)}
        if self.pre == "gemma":
            return "".join(self.tokens[i] for i in ids).replace("▁", " ")
        data = bytearray()
        for i in ids:
            t = self.tokens[i]
            if all(c in inv for c in t):
                data.extend(inv[c] for c in t)
            else:
                data.extend(t.encode("utf-8"))
        return data.decode("utf-8", errors="replace")
