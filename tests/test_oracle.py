"""CPU tests: pin the oracle against the reference's known-answer tests and
the golden vectors, before it is trusted as the parity checker."""
import os
import struct

import numpy as np
import pytest

import oracle
from laya_goish_b200 import synth

GOLD = os.path.join(os.path.dirname(__file__), "golden", "dequant.npz")


def test_half_known_answers():
    # src/tensor.rs:215-217
    assert abs(oracle.half(0x3C00) - 1.0) <= 1e-8
    assert oracle.half(1) == 1.0 / 16777216.0


def test_matrix_self_test():
    # src/tensor.rs:196-214: 17x11 W, 9 rows of x, bias 0.25, 1/2/4 threads, tol 1e-4
    w = ((np.arange(187, dtype=np.float32) - 83.0) / 71.0).reshape(11, 17)
    x = ((np.arange(153, dtype=np.float32) - 71.0) / 43.0).reshape(9, 17)
    b = np.full(11, 0.25, np.float32)
    want = np.array([[np.dot(x[r], w[c]) + 0.25 for c in range(11)] for r in range(9)], np.float32)
    for threads in (1, 2, 4):
        y = oracle.matrix_apply(w, x, b, threads)
        assert np.abs(y - want).max() <= 1e-4


def test_matrix_thread_count_bit_equal():
    # validation/smoke.py:28 — thread count never changes results
    rng = np.random.default_rng(5)
    w = rng.standard_normal((37, 131), dtype=np.float32)
    x = rng.standard_normal((23, 131), dtype=np.float32)
    ys = [oracle.matrix_apply(w, x, None, t) for t in (1, 3, 8)]
    assert all(np.array_equal(ys[0], y) for y in ys[1:])


def test_confidence_known_answers():
    # src/models/laya/decision.rs:331-333
    assert abs(oracle.confidence([0.5, 0.5])) <= 1e-6
    assert oracle.confidence([1.0, 0.0]) >= 0.9999


@pytest.mark.parametrize("kind", [0, 1, 2, 8, 12, 14])
def test_decode_golden_bit_exact(kind):
    g = np.load(GOLD)
    got = oracle.decode(kind, g[f"raw_{kind}"])
    want = g[f"want_{kind}"]
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _string(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


@pytest.mark.parametrize("blob,msg", [
    (b"", "truncated"),
    (b"GGUF", "truncated"),
    (b"GGUF" + struct.pack("<IQQ", 3, 999999999, 0), "too large"),
    (b"NOPE" + bytes(20), "not a GGUF"),
    (b"GGUF" + struct.pack("<IQQ", 2, 0, 0), "version 3"),
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + _string("k") + struct.pack("<I", 13), "metadata type"),
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 2) + (_string("k") + struct.pack("<II", 4, 1)) * 2, "duplicate"),
    (b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + _string("t") + struct.pack("<IQ", 1, 0), "empty tensor"),
    (b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + _string("t") + struct.pack("<IQIQ", 1, 32, 3, 0), "unsupported GGML"),
    (b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + _string("t") + struct.pack("<IQIQ", 1, 33, 8, 0), "row alignment"),
    (b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + _string("t") + struct.pack("<IQIQ", 1, 32, 8, 0), "truncated tensor"),
    (b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + _string("t") + struct.pack("<IQIQ", 1, 32, 8, 5), "unaligned"),
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + _string("general.alignment") + struct.pack("<II", 4, 48), "alignment"),
    (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", 2) + b"\xff\xfe" + struct.pack("<II", 4, 1), "UTF-8"),
])
def test_malformed_gguf_rejected(blob, msg):
    # validation/smoke.py:13 (the first four blobs) and the src/gguf.rs:95-180 checks
    err = oracle.gguf_check(blob)
    assert err is not None and msg in err, err


def test_unsupported_architecture_rejected():
    # validation/test_registry.py:34-35
    blob = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + _string("general.architecture") + struct.pack("<I", 8) + _string("unsupported")
    assert oracle.gguf_check(blob) is None
    with pytest.raises(ValueError, match="unsupported GGUF architecture"):
        oracle.Model(blob)


def test_writer_readable_by_gguf_py(tiny_paths):
    gguf = pytest.importorskip("gguf")
    path = tiny_paths["tiny-llama-q4_k_m"]
    r = gguf.GGUFReader(path)
    names = {t.name: t for t in r.tensors}
    assert names["blk.0.attn_v.weight"].tensor_type.name == "Q6_K"
    assert names["blk.0.attn_q.weight"].tensor_type.name == "Q4_K"
    assert oracle.gguf_check(open(path, "rb").read()) is None


@pytest.mark.parametrize("name", ["tiny-llama-f16", "tiny-qwen2-f16", "tiny-llama-q4_k_m", "tiny-llama-q8_0"])
def test_oracle_forward_matches_float64_torch(tiny_paths, name):
    pytest.importorskip("gguf")
    import torch_ref
    m = oracle.Model(open(tiny_paths[name], "rb").read(), threads=2)
    rng = np.random.default_rng(3)
    ids = synth.token_ids(rng, m.vocab, 33)
    h = m.forward(ids, [32, 0, 7])
    th, W = torch_ref.forward(tiny_paths[name], ids, [32, 0, 7])
    assert np.abs(h - th.numpy()).max() < 1e-4
    cand = synth.candidates(rng, m.vocab, 4)
    assert np.abs(m.head(h, cand) - (th @ W.T)[:, cand].numpy()).max() < 1e-4


def test_oracle_rejects_bad_ids(tiny_paths):
    m = oracle.Model(open(tiny_paths["tiny-llama-f16"], "rb").read())
    with pytest.raises(ValueError):
        m.forward([1, 2, m.vocab], [2])  # id >= V (src/models/openthai/model.rs:198-204)
    with pytest.raises(ValueError):
        m.forward([1, 2, 3], [3])  # read position past the end


def test_decision_rules(tiny_paths):
    m = oracle.Model(open(tiny_paths["tiny-llama-f16"], "rb").read())
    ids = synth.token_ids(np.random.default_rng(9), m.vocab, 20)
    a = m.decide(ids, 0, [10, 11, 12, 13])
    p = np.array(a["probabilities"])
    assert abs(p.sum() - 1) < 1e-6 and a["choice"] == int(np.argmax(p))
    assert np.allclose(p, oracle.softmax(np.array(a["logits"], np.float32)))
    # identical options tie: the lowest index wins (src/models/laya/decision.rs:233-235)
    a = m.decide(ids, 0, [10, 10, 10])
    assert a["choice"] == 0
    s = m.decide(ids, 1, [[5, 6, 7], [8, 9, 10]])
    ps = np.array(s["probabilities"])
    assert abs(s["score"] - float((np.arange(2) * ps).sum())) < 1e-6
    c = m.decide(ids, 2, [20, 21], suffix=[30, 31])
    assert c["noul"] == c["probabilities"][1]
    assert abs(c["confidence"] - max(c["noul"], 1 - c["noul"])) < 1e-7


@pytest.mark.parametrize("name", ["tiny-llama-q8_0", "tiny-qwen2-f16"])
def test_cached_forward_bit_equal_to_whole_sequence(tiny_paths, name):
    # Extending a cached prefix gives the same bits as one forward over the
    # whole sequence: each row depends on its own token and earlier keys, and
    # Matrix::apply computes every token row alone (src/tensor.rs:58-102).
    m = oracle.Model(open(tiny_paths[name], "rb").read(), threads=3, attn_threads=3)
    rng = np.random.default_rng(11)
    ids = synth.token_ids(rng, m.vocab, 41)
    whole = m.forward(ids, list(range(41)))
    c = m.cache(60)
    parts = [c.forward(ids[:17], list(range(17))), c.forward(ids[17:18], [0]), c.forward(ids[18:], list(range(23)))]
    assert len(c) == 41
    assert np.array_equal(np.concatenate(parts), whole)
    # branch off the prefix: truncate and append a different tail
    c.truncate(30)
    tail = synth.token_ids(rng, m.vocab, 5)
    got = c.forward(tail, [4])
    want = m.forward(np.concatenate([ids[:30], tail]), [34])
    assert np.array_equal(got, want)
    with pytest.raises(ValueError):
        c.truncate(40)
    c.close()


def test_cached_greedy_matches_recompute(tiny_paths):
    m = oracle.Model(open(tiny_paths["tiny-llama-f16"], "rb").read(), threads=2)
    ctx = list(synth.token_ids(np.random.default_rng(12), m.vocab, 25))
    toks, margins = m.greedy(ctx, 5)
    seq = list(ctx)
    for s in range(5):
        logits = m.head(m.forward(np.array(seq, np.int32), [len(seq) - 1]))[0]
        assert toks[s] == int(np.argmax(logits))
        seq.append(toks[s])
    assert all(g >= 0 for g in margins)


def test_attention_threads_bit_equal(tiny_paths):
    blob = open(tiny_paths["tiny-qwen2-f16"], "rb").read()
    ids = synth.token_ids(np.random.default_rng(13), 1000, 50)
    outs = [oracle.Model(blob, threads=t, attn_threads=t).forward(ids, [0, 25, 49]) for t in (1, 4, 7)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
