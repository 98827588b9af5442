"""Host tokenizer (src/tokenizer.rs:17-331) on synthetic vocabularies.

No reference output is available here (the reference's tokenizer parity
script needs the real model files and the reference binary), so these cases
pin the restated algorithm: the byte alphabet, both pre-tokenizers on the
texts the reference's tokenizer parity script feeds, BPE rank order and
leftmost ties, special-token cutting, gemma byte fallback, limits and errors,
and the GGUF metadata round trip of the synthetic models."""
import pytest

from laya_goish_b200 import synth
from laya_goish_b200.gguf_meta import GGUFError, read_metadata
from laya_goish_b200.tokenizer import (Tokenizer, TokenizerError, byte_alphabet, split_gpt2, split_qwen)


def gpt2(text):
    return [p.decode("utf-8", "replace") for p in split_gpt2(text.encode())]


def qwen(text):
    return [p.decode() for p in split_qwen(text)]


def test_byte_alphabet():
    a = byte_alphabet()
    assert len(set(a)) == 256
    assert all(a[b] == chr(b) for b in range(33, 127))
    assert a[0x20] == "Ġ" and a[0x0A] == "Ċ" and a[0] == "Ā"
    assert a[0xAD] == "Ń" and a[0xA1] == "\xa1"


def test_gpt2_pretokenization():
    assert gpt2("Hello, world!") == ["Hello", ",", " world", "!"]
    assert gpt2("I'm you're we've he'll she'd can't I'M") == [
        "I", "'m", " you", "'re", " we", "'ve", " he", "'ll", " she", "'d", " can", "'t", " I", "'", "M"]
    assert gpt2("  word   next\n\n\tlast  ") == [" ", " word", "  ", " next", "\n\n", "\t", "last", "  "]
    assert gpt2("1234567890 + 42.5") == ["1234567890", " +", " 42", ".", "5"]
    assert gpt2(" a  b   c") == [" a", " ", " b", "  ", " c"]
    assert gpt2("\r\n\t \v\f") == ["\r\n\t \v\f"]
    assert gpt2("") == []
    # non-ASCII bytes are "other" bytes, grouped into one run
    assert b"".join(split_gpt2("café ไทย".encode())) == "café ไทย".encode()


def test_qwen_pretokenization():
    assert qwen("café Café 日本語 🙂 ไทย") == ["café", " Café", " 日本語", " 🙂", " ไทย"]  # NFC first
    assert qwen("I'M you're 12 ab!!\n\nx") == ["I", "'M", " you", "'re", " ", "1", "2", " ab", "!!\n\n", "x"]
    assert qwen("  word   next\n\n\tlast  ") == [" ", " word", "  ", " next", "\n\n", "\tlast", "  "]
    assert qwen("1234567890 + 42.5")[:3] == ["1", "2", "3"]
    assert qwen("https://example.com?a=1&b=2")[:3] == ["https", "://", "example"]


def meta(tokens, merges, pre="gpt2", types=None):
    m = {"tokenizer.ggml.pre": pre, "tokenizer.ggml.tokens": tokens, "tokenizer.ggml.merges": merges}
    if types is not None:
        m["tokenizer.ggml.token_type"] = types
    return m


def test_bpe_rank_order_and_leftmost_ties():
    a = byte_alphabet()
    toks = a + ["ab", "bc", "abc", "aa"]
    t = Tokenizer(meta(toks, ["b c", "a b", "a bc", "a a"]))
    # "abc": b+c has the lower rank, then a+bc
    assert t.encode("abc") == [toks.index("abc")]
    # "aaa": a+a at both places has one rank; the leftmost merges first
    assert t.encode("aaa") == [toks.index("aa"), toks.index("a")]
    # unknown piece without byte fallback is an error
    t2 = Tokenizer(meta(["a", "b"], ["a b"]))
    with pytest.raises(TokenizerError):
        t2.encode("c")


def test_special_tokens_cut_first():
    a = byte_alphabet()
    toks = a + ["[CLS]", "[SEP]", "[MASK]", "<|ts|>", "<|ts_q|>"]
    t = Tokenizer(meta(toks, []))
    ids = t.encode("[CLS][SEP][MASK]x")
    assert ids[:3] == [toks.index("[CLS]"), toks.index("[SEP]"), toks.index("[MASK]")]
    assert ids[3] == a.index("x")
    # longest special first among those starting at the same place
    assert t.encode("<|ts_q|>")[0] == toks.index("<|ts_q|>")
    assert t.decode(t.encode("before [MASK] after")) == "before [MASK] after"


def test_qwen_specials_by_token_type():
    a = byte_alphabet()
    toks = a + ["<|im_start|>", "<fake>"]
    types = [1] * 256 + [3, 1]
    t = Tokenizer(meta(toks, [], pre="qwen2", types=types))
    assert t.encode("<|im_start|>")[0] == toks.index("<|im_start|>")
    assert len(t.encode("<fake>")) > 1  # token_type 1: not special under qwen3 rules


def test_gemma_pieces_and_byte_fallback():
    toks = ["▁hi", "▁", "h", "i", "<0x21>"]
    t = Tokenizer(meta(toks, ["h i", "▁ hi"], pre="gemma"))
    assert t.encode("hi") == [toks.index("▁hi")]
    assert t.encode("hi!") == [toks.index("▁hi"), toks.index("<0x21>")]


def test_limits_and_errors():
    with pytest.raises(TokenizerError):
        Tokenizer(meta(["a"], [], pre="llama-bpe"))
    with pytest.raises(TokenizerError):
        Tokenizer(meta([], []))
    t = Tokenizer(meta(byte_alphabet(), []))
    with pytest.raises(TokenizerError):
        t.encode("a" * (1024 * 1024 + 1))
    assert t.mask is None


def test_synthetic_model_vocabulary_round_trip(tmp_path):
    cfg = synth.TINY["tiny-llama-q8_0-tok"]
    m = synth._meta(cfg)
    path = tmp_path / "tok.gguf"
    synth.write_gguf(str(path), m, [])
    got = read_metadata(str(path))
    assert got["tokenizer.ggml.tokens"] == m["tokenizer.ggml.tokens"]
    assert got["tokenizer.ggml.merges"] == m["tokenizer.ggml.merges"]
    assert got["tokenizer.ggml.token_type"] == m["tokenizer.ggml.token_type"]
    assert len(got["tokenizer.ggml.tokens"]) == cfg.vocab
    t = Tokenizer(got)
    ids = t.encode("hello world, the answer is yes!")
    assert all(0 <= i < cfg.vocab for i in ids)
    assert t.decode(ids) == "hello world, the answer is yes!"
    assert t.encode("the") == [t.vocab["the"]]
    with pytest.raises(GGUFError):
        read_metadata(b"GGUF" + b"\x02\x00\x00\x00")


def test_gguf_metadata_reader_errors_and_types():
    import struct

    def kv_str(k, v):
        kb, vb = k.encode(), v.encode()
        return struct.pack("<Q", len(kb)) + kb + struct.pack("<IQ", 8, len(vb)) + vb

    head = b"GGUF" + struct.pack("<IQQ", 3, 0, 3)
    body = kv_str("general.name", "x")
    body += struct.pack("<Q", 1) + b"f" + struct.pack("<Id", 12, 2.5)          # f64 scalar
    body += struct.pack("<Q", 1) + b"a" + struct.pack("<IIQ", 9, 4, 3) + struct.pack("<3I", 7, 8, 9)  # u32 array
    m = read_metadata(head + body)
    assert m == {"general.name": "x", "f": 2.5, "a": [7, 8, 9]}
    with pytest.raises(GGUFError):
        read_metadata(b"GGUX" + head[4:] + body)  # bad magic
    with pytest.raises(GGUFError):
        read_metadata(head + body[:-3])  # truncated
    bad_type = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", 1) + b"k" + struct.pack("<I", 13)
    with pytest.raises(GGUFError):
        read_metadata(bad_type)
    bad_utf8 = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", 1) + b"k" + struct.pack("<IQ", 8, 2) + b"\xff\xfe"
    with pytest.raises(GGUFError):
        read_metadata(bad_utf8)
