"""OpenThai on the GPU against the oracle's restatement of
src/models/openthai/model.rs: the gated DeltaNet recurrence
(laya_gated_delta, Delta::run 322-355) and its whole mixer after the
projections, the gated attention (Full::run 248-296), the native forward
(laya_openthai_forward, Model::forward 192-241), with F16 or block-quantised
matrices (Q8_0, Q4_K: decoded at load as the reference's g.floats does), and
a whole decision through it.  Parity of the forward with the reference itself is unpinned (its
goldens need the real OpenThai weights)."""
import numpy as np
import pytest

import oracle
from laya_goish_b200 import engine
from laya_goish_b200._lib import E_INVALID, LayaError

pytestmark = pytest.mark.gpu


def inputs(rng, s, nh, hk):
    raw = rng.normal(0, 1, (s, 3 * nh * hk))
    qkv = raw / (1 + np.exp(-raw))  # SiLU output, as after the causal convolution
    a = rng.normal(0, 1, (s, nh))
    b = rng.normal(0, 1, (s, nh))
    dt = rng.normal(0, 0.5, nh)
    alog = rng.normal(-1, 0.5, nh)
    return qkv, a, b, dt, alog


@pytest.mark.parametrize("s,nh,hk", [(1, 2, 128), (37, 3, 128), (200, 16, 128), (64, 4, 64)])
def test_gated_delta_matches_oracle(s, nh, hk):
    rng = np.random.default_rng(s * 7 + nh)
    qkv, a, b, dt, alog = inputs(rng, s, nh, hk)
    got = engine.gated_delta(qkv, a, b, dt, alog, nh, hk)
    want = oracle.ot_delta_core(qkv, a, b, dt, alog, nh, hk)
    assert np.allclose(got, want, atol=1e-4, rtol=1e-3), np.abs(got - want).max()
    # causal: a prefix gives the prefix's rows
    if s > 8:
        head = engine.gated_delta(qkv[:8], a[:8], b[:8], dt, alog, nh, hk)
        assert np.allclose(head, got[:8], atol=1e-6)


def test_gated_delta_rejects_bad_head_dim():
    rng = np.random.default_rng(1)
    qkv, a, b, dt, alog = inputs(rng, 4, 2, 32)
    with pytest.raises(LayaError) as e:
        engine.gated_delta(qkv, a, b, dt, alog, 2, 32)
    assert e.value.code == E_INVALID


@pytest.mark.parametrize("s,H,KV,hd,rot", [(1, 8, 2, 256, 64), (23, 8, 2, 256, 64), (130, 8, 2, 256, 64),
                                           (40, 4, 4, 128, 128), (17, 6, 2, 64, 16)])
def test_gated_attention_matches_oracle(s, H, KV, hd, rot):
    rng = np.random.default_rng(s + hd)
    qgate = rng.normal(0, 1, (s, H * 2 * hd))
    k = rng.normal(0, 1, (s, KV * hd))
    v = rng.normal(0, 1, (s, KV * hd))
    qn, kn = rng.normal(0, 0.1, hd), rng.normal(0, 0.1, hd)
    got = engine.gated_attention(qgate, k, v, qn, kn, H, KV, hd, rot, 1e7)
    want = oracle.ot_full_core(qgate, k, v, qn, kn, H, KV, hd, rot, 1e7)
    # tensor-core operands: q, k, v, the softmax weights and the output are
    # rounded to F16 (relative 2^-11 each), scores and sums are F32
    err = np.abs(got - want).max()
    print(f"[parity] gated attention s={s} H={H}/{KV} hd={hd}: max |d| = {err:.2e}")
    assert np.allclose(got, want, atol=5e-3, rtol=2e-2), err


def test_gated_attention_rejects_bad_shapes():
    z = np.zeros((2, 512), np.float32)
    with pytest.raises(LayaError) as e:
        engine.gated_attention(z, z, z, np.zeros(256), np.zeros(256), H=3, KV=2, hd=256, rot=64, theta=1e7)
    assert e.value.code == E_INVALID


@pytest.mark.parametrize("s,nh,hk", [(3, 2, 128), (90, 16, 128), (33, 4, 64)])
def test_gated_delta_mixer_matches_oracle(s, nh, hk):
    rng = np.random.default_rng(1000 + s)
    w = nh * hk
    raw = rng.normal(0, 1, (s, 3 * w))
    z = rng.normal(0, 1, (s, w))
    a, b = rng.normal(0, 1, (s, nh)), rng.normal(0, 1, (s, nh))
    conv = rng.normal(0, 0.5, (3 * w, 4))
    dt, alog, normw = rng.normal(0, 0.5, nh), rng.normal(-1, 0.5, nh), rng.normal(1, 0.1, hk)
    got = engine.gated_delta_mixer(raw, z, a, b, conv, dt, alog, normw, nh, hk)
    want = oracle.ot_delta_mid(raw, z, a, b, conv, dt, alog, normw, nh, hk)
    assert np.allclose(got, want, atol=1e-4, rtol=1e-3), np.abs(got - want).max()


@pytest.fixture(scope="module")
def ot_model(tmp_path_factory):
    from laya_goish_b200 import openthai, synth

    path = synth.write_openthai(str(tmp_path_factory.mktemp("ot") / "ot.gguf"), d=128, ffn=256, heads=4, kv=2,
                                hd=64, lin_heads=2, lin_dim=64, seed=11)
    weights = openthai.load_weights(path, strict=False)
    with openthai.Model(path, strict=False) as m:
        yield m, weights


def test_openthai_forward_matches_oracle(ot_model):
    m, w = ot_model
    rng = np.random.default_rng(3)
    for s, pos in [(40, [0, 20, 39]), (1, [0]), (200, [7, 150, 199])]:
        ids = rng.integers(0, 300, s)
        got = m.forward(ids, pos)
        want = oracle.ot_forward(w, ids, pos)
        # F16 GEMM operands (activations rounded to 2^-11 relative) against F32;
        # a NumPy emulation of that rounding lands near 1e-3 of the largest logit
        tol = 5e-3 * np.abs(want).max()
        assert got.shape == (len(pos), 256)
        assert np.abs(got - want).max() < tol, (s, np.abs(got - want).max(), tol)
    # causal: a prefix's last position gives the same logits as in the full pass
    ids = rng.integers(0, 300, 40)
    full = m.forward(ids, [20])
    head = m.forward(ids[:21], [20])
    assert np.allclose(full, head, atol=1e-4, rtol=1e-4)
    # a repeated request after a different one is bitwise identical:
    # no state survives a pass in the reused scratch (validation/openthai_edges.py)
    assert np.array_equal(m.forward(ids, [20]), full)
    with pytest.raises(LayaError):
        m.forward([0, 1, 300], [0])
    with pytest.raises(LayaError):
        m.forward([0, 1, 2], [3])


def test_openthai_forward_batch_matches_single_passes(ot_model):
    """Several passes in one forward (laya_openthai_forward_batch): each
    sequence causal on its own, mixers on side streams (five sequences: more
    than the four side streams), the same logits as one pass at a time and
    the oracle's."""
    m, w = ot_model
    rng = np.random.default_rng(21)
    shapes = [(40, [0, 39]), (1, [0]), (200, [7, 150, 199]), (65, [64]), (130, [3, 129])]
    passes = [(rng.integers(0, 300, s), pos) for s, pos in shapes]
    got = m.forward_batch(passes)
    assert len(got) == len(passes)
    for (ids, pos), g in zip(passes, got):
        one = m.forward(ids, pos)
        want = oracle.ot_forward(w, ids, pos)
        assert g.shape == one.shape == (len(pos), 256)
        # the batch's GEMMs may split K differently from one pass's
        assert np.allclose(g, one, atol=1e-3 * np.abs(one).max() + 1e-5), np.abs(g - one).max()
        assert np.abs(g - want).max() < 5e-3 * np.abs(want).max()
    with pytest.raises(LayaError):
        m.forward_batch([([0, 1, 2], [0]), ([0, 1], [2])])  # a position past its own pass
    with pytest.raises(LayaError):
        m.forward_batch([([0, 1, 2], [3]), ([0, 1], [1])])  # ... that would land in the next pass


def test_openthai_forward_reference_head_geometry(tmp_path):
    """The reference's head layout (8/2 attention heads of 256 with a 64-wide
    rotary part, 16 DeltaNet heads of 128) on a small width; a NumPy
    emulation of the F16 operand rounding lands near 1.5e-3 of the largest
    logit here."""
    from laya_goish_b200 import openthai, synth

    path = synth.write_openthai(str(tmp_path / "ot_ref.gguf"), d=256, ffn=256, heads=8, kv=2, hd=256,
                                lin_heads=16, lin_dim=128, seed=12, width_scaled=True)
    w = openthai.load_weights(path, strict=False)
    rng = np.random.default_rng(5)
    with openthai.Model(path, strict=False) as m:
        for s, pos in [(40, [0, 39]), (200, [99, 199])]:
            ids = rng.integers(0, 300, s)
            got = m.forward(ids, pos)
            want = oracle.ot_forward(w, ids, pos)
            tol = 5e-3 * np.abs(want).max()
            assert np.abs(got - want).max() < tol, (s, np.abs(got - want).max(), tol)


def test_openthai_decide_matches_oracle(ot_model):
    from laya_goish_b200 import openthai
    from laya_goish_b200.tokenizer import Tokenizer, byte_alphabet

    m, w = ot_model
    control = ["<|ts_q|>", "<|ts_choice|>", "<|ts_score|>", "<|ts_noul|>", "<|ts_answer|>", "<|ts_state|>"] + \
              [f"<|ts_opt_{i}|>" for i in range(12)]
    tok = Tokenizer({"tokenizer.ggml.pre": "gpt2", "tokenizer.ggml.tokens": byte_alphabet() + control,
                     "tokenizer.ggml.merges": []})
    m.config["answer_token_id"] = w["config"]["answer_token_id"] = tok.vocab["<|ts_answer|>"]
    req = {"state": {"ticket": "refund please", "n": 3},
           "questions": {"c": {"type": "choice", "instructions": "route", "criteria": {"a": "billing", "b": None,
                                                                                       "c": "other"}},
                         "s": {"type": "score", "instructions": "urgency", "criteria": ["low", "mid", "high"]},
                         "n": {"type": "noul", "instructions": "spam?"}},
           "order_invariant": True}
    got = m.decide(tok, req)
    qs = openthai.questions(req)
    n = openthai.permutation_count(req, qs)
    assert n == 3
    passes = []
    for p in range(n):
        e = openthai.encode(tok, req, qs, n, p, w["config"]["answer_token_id"], 512, 256)
        passes.append((oracle.ot_forward(w, e.ids, e.positions), e.order))
    want = openthai.decide(qs, passes, w["temperature"])
    for k in ("a", "b", "c"):
        assert abs(got["c"]["probabilities"][k] - want["c"]["probabilities"][k]) < 1e-2
    assert abs(got["s"]["score"] - want["s"]["score"]) < 5e-2
    assert abs(got["n"]["noul"] - want["n"]["noul"]) < 1e-2


def test_openthai_batch_over_two_gpus(tmp_path):
    """A batch of states shared over one model per GPU (OpenThaiService with
    a model list) gives the one-GPU answers, in request order."""
    import json

    import torch

    from laya_goish_b200 import frontend, openthai, synth
    from laya_goish_b200.tokenizer import Tokenizer

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    path = synth.write_openthai(str(tmp_path / "ot2.gguf"), d=128, ffn=256, heads=4, kv=2, hd=64, lin_heads=2,
                                lin_dim=64, seed=13, tokenizer=True)
    tok = Tokenizer.from_gguf(path)
    batch = {"states": ["a", {"b": 1}, "ccc", "d d", ["e"], "ff"],
             "questions": {"c": {"type": "choice", "instructions": "route",
                                 "criteria": {"a": "billing", "b": None, "c": "other"}},
                           "n": {"type": "noul", "instructions": "spam?"}},
             "order_invariant": True}
    with openthai.Model(path, device=0, strict=False) as m0, openthai.Model(path, device=1, strict=False) as m1:
        one = frontend.OpenThaiService(m0, tok).handle("POST", "/v1/decide/batch", json.dumps(batch))
        two = frontend.OpenThaiService([m0, m1], tok).handle("POST", "/v1/decide/batch", json.dumps(batch))
    assert one.status == two.status == 200
    strip = lambda b: [{k: v for k, v in r.items() if k not in ("usage", "id")} for r in b["results"]]
    assert strip(one.body) == strip(two.body)


@pytest.mark.parametrize("quant,shape", [
    (8, dict(d=128, ffn=256, heads=4, kv=2, hd=64, lin_heads=2, lin_dim=64)),      # Q8_0
    (12, dict(d=256, ffn=512, heads=4, kv=2, hd=64, lin_heads=2, lin_dim=128)),    # Q4_K
])
def test_openthai_forward_quantised_matrices_match_oracle(tmp_path, quant, shape):
    # every matrix and the embedding table in a block type: the library
    # decodes them at load with the reference's block arithmetic
    # (src/models/openthai/model.rs:61, src/gguf.rs:250-336); the oracle gets
    # the same values from its own pinned decoder
    from laya_goish_b200 import openthai, synth

    path = synth.write_openthai(str(tmp_path / f"ot_q{quant}.gguf"), seed=12, quant=quant, **shape)
    w = openthai.load_weights(path, strict=False, decode=oracle.decode)
    rng = np.random.default_rng(5)
    with openthai.Model(path, strict=False) as m:
        for s, pos in [(33, [0, 16, 32]), (130, [7, 129])]:
            ids = rng.integers(0, 300, s)
            got = m.forward(ids, pos)
            want = oracle.ot_forward(w, ids, pos)
            tol = 5e-3 * np.abs(want).max()
            assert np.abs(got - want).max() < tol, (quant, s, np.abs(got - want).max(), tol)
