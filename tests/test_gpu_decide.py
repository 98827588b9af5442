"""GPU parity of the decision hot path against the CPU oracle on seeded
synthetic GGUF decoders: the forward's hidden states, and decide answers
(probabilities within 1e-3 absolute / 1e-2 relative, identical argmax) for
choice / score / noul questions, single-token and multi-token options,
suffixes over a shared prefix, ragged prompt lengths, batch invariance,
waves, validation errors and cancellation."""
import numpy as np
import pytest

import oracle
from laya_goish_b200 import engine, synth
from laya_goish_b200.engine import Question

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-2


@pytest.fixture(scope="module")
def models(tiny_paths):
    out = {}
    for name, path in tiny_paths.items():
        out[name] = (engine.Engine(path), oracle.Model(open(path, "rb").read(), threads=8, attn_threads=8))
    yield out
    for e, o in out.values():
        e.close()
        o.close()


def assert_answer(got, want, tag=""):
    p, q = np.array(got["probabilities"]), np.array(want["probabilities"])
    assert np.allclose(p, q, atol=ATOL, rtol=RTOL), (tag, p, q, got["logits"], want["logits"])
    top = np.sort(q)[::-1]
    if want["kind"] == 0 and (len(q) < 2 or top[0] - top[1] > 2 * ATOL):
        assert got["choice"] == want["choice"], tag
    if want["kind"] == 1:
        assert abs(got["score"] - want["score"]) < 1e-2, tag
    if want["kind"] == 2:
        assert abs(got["noul"] - want["noul"]) <= ATOL + RTOL * want["noul"], tag


def oracle_answer(o, ids, q: Question):
    kind, opts, suf = q.arrays()
    a = o.decide(ids, kind, opts, suf)
    return a


@pytest.mark.parametrize("name", ["tiny-llama-f16", "tiny-llama-q8_0", "tiny-llama-q4_k_m", "tiny-qwen2-f16",
                                  "small-llama-q8_0"])
@pytest.mark.parametrize("n", [1, 7, 64, 65, 200])
def test_forward_hidden_matches_oracle(models, name, n):
    e, o = models[name]
    rng = np.random.default_rng(n)
    ids = synth.token_ids(rng, o.vocab, n)
    read = sorted({0, n // 2, n - 1})
    got = e.forward(ids, read)
    want = o.forward(ids, read)
    err = np.abs(got - want)
    assert err.max() < 3e-2 and err.mean() < 3e-3, (err.max(), err.mean())


@pytest.mark.parametrize("name", ["tiny-llama-f16", "tiny-llama-q8_0", "tiny-llama-q4_k_m", "tiny-llama-q4_0",
                                  "tiny-qwen2-f16", "small-llama-q8_0"])
def test_decide_matches_oracle(models, name):
    e, o = models[name]
    rng = np.random.default_rng(42)
    V = o.vocab
    prompts = [synth.token_ids(rng, V, n) for n in (1, 5, 63, 64, 65, 130, 300)]
    questions = [
        Question("choice", synth.candidates(rng, V, 4)),
        Question("noul", synth.candidates(rng, V, 2)),
        Question("noul", synth.candidates(rng, V, 2), suffix=synth.token_ids(rng, V, 16)),
        Question("score", synth.candidates(rng, V, 15 * 3 // 3 * 1)[:5].reshape(5, 1)),
        Question("score", synth.token_ids(rng, V, 15).reshape(5, 3)),
        Question("choice", synth.token_ids(rng, V, 8).reshape(4, 2), suffix=synth.token_ids(rng, V, 3)),
    ]
    got = e.decide_batch(prompts, questions)
    for i, p in enumerate(prompts):
        for j, q in enumerate(questions):
            assert_answer(got[i][j], oracle_answer(o, p, q), (name, i, j))


def test_batch_invariance_and_determinism(models):
    e, _ = models["small-llama-q8_0"]
    rng = np.random.default_rng(7)
    prompts = [synth.token_ids(rng, 4000, n) for n in (17, 64, 100, 257)]
    qs = [Question("choice", synth.candidates(rng, 4000, 4)), Question("score", synth.token_ids(rng, 4000, 6).reshape(3, 2))]
    a = e.decide_batch(prompts, qs)
    b = e.decide_batch(prompts, qs)
    assert a == b  # repeated requests are bit-identical (validation/smoke.py:25)
    # Alone, a request runs with fewer token rows, so its residual GEMMs may
    # split K (partial sums merged in split order): the same sums, associated
    # differently in F32, hence a tolerance rather than bit equality.
    for i, p in enumerate(prompts):
        alone = e.decide_batch([p], qs)[0]
        for j in range(len(qs)):
            assert np.allclose(alone[j]["probabilities"], a[i][j]["probabilities"], atol=2e-4), (i, j)


def test_waves_match_single_wave(models, monkeypatch):
    e, o = models["tiny-llama-q8_0"]
    rng = np.random.default_rng(8)
    prompts = [synth.token_ids(rng, o.vocab, n) for n in (90, 33, 140, 2, 77)]
    qs = [Question("noul", synth.candidates(rng, o.vocab, 2), suffix=[5, 6, 7])]
    one = e.decide_batch(prompts, qs)
    # smaller waves may split the residual GEMMs' K differently (2e-4 below)
    monkeypatch.setenv("LAYA_WAVE_TOKENS", "100")
    many = e.decide_batch(prompts, qs)
    for i in range(len(prompts)):
        assert np.allclose(one[i][0]["probabilities"], many[i][0]["probabilities"], atol=2e-4)


def test_validation_rejects_before_launch(models):
    e, o = models["tiny-llama-f16"]
    good = synth.token_ids(np.random.default_rng(1), o.vocab, 10)
    q = Question("choice", [3, 4])
    with pytest.raises(engine.LayaError) as ex:
        e.decide_batch([good, np.array([1, o.vocab])], [q])  # id >= V (src/models/openthai/model.rs:198-204)
    assert ex.value.code == engine._lib.E_INVALID
    with pytest.raises(engine.LayaError):
        e.decide_batch([good, np.array([], np.int32)], [q])
    with pytest.raises(engine.LayaError):
        e.decide_batch([good], [Question("noul", [3, 4, 5])])
    with pytest.raises(engine.LayaError):
        e.decide_batch([good], [Question("choice", list(range(3, 20)))])
    with pytest.raises(engine.LayaError):
        e.decide_batch([np.zeros(o.ctx + 1, np.int32)], [q])
    assert e.decide_batch([], [q]) == []
    # the engine still works after rejected batches
    assert len(e.decide_batch([good], [q])[0]) == 1


def test_cancellation_then_recovery(models):
    e, o = models["small-llama-q8_0"]
    rng = np.random.default_rng(3)
    prompts = [synth.token_ids(rng, o.vocab, 64)]
    q = [Question("choice", [3, 4, 5])]
    calls = []

    def cancel():
        calls.append(1)
        return len(calls) >= 2  # fires at the second layer poll

    with pytest.raises(engine.LayaError) as ex:
        e.decide_batch(prompts, q, canceled=cancel)
    assert ex.value.code == engine._lib.E_CANCELED
    ok = e.decide_batch(prompts, q, canceled=lambda: False)
    assert_answer(ok[0][0], oracle_answer(o, prompts[0], q[0]))


def test_open_rejects_malformed_gguf():
    for blob in [b"GGUF", b"NOPE" + bytes(20)]:
        with pytest.raises(engine.LayaError) as ex:
            engine.Engine(image=blob)
        assert ex.value.code == engine._lib.E_FORMAT
    with pytest.raises(engine.LayaError) as ex:
        engine.Engine("/nonexistent/model.gguf")
    assert ex.value.code == engine._lib.E_IO


def test_multi_replica_sharding_matches_single(tiny_paths):
    # Two replicas on one GPU exercise the in-process request sharding (one host
    # thread per replica, contiguous request ranges, answers in request order).
    path = tiny_paths["tiny-llama-q8_0"]
    rng = np.random.default_rng(11)
    prompts = [synth.token_ids(rng, 1000, int(n)) for n in (30, 200, 5, 64, 90, 17, 128)]
    qs = [Question("choice", [10, 11, 12]), Question("score", [[3, 4], [5, 6]], suffix=[7])]
    with engine.Engine(path, devices=[0]) as one, engine.Engine(path, devices=[0, 0]) as two:
        assert two.info["n_devices"] == 2
        a = one.decide_batch(prompts, qs)
        b = two.decide_batch(prompts, qs)
    for i in range(len(prompts)):
        for j in range(len(qs)):
            assert np.allclose(a[i][j]["probabilities"], b[i][j]["probabilities"], atol=2e-4), (i, j)


@pytest.mark.parametrize("peer", ["1", "0"])
def test_replicas_on_distinct_gpus(tiny_paths, monkeypatch, peer):
    # Replicas on other GPUs are copied from the first over NVLink (or, with
    # LAYA_LOAD_PEER=0, each read from the file); both give the one-GPU answers.
    import torch

    n = min(torch.cuda.device_count(), 4)
    if n < 2:
        pytest.skip("needs 2 GPUs")
    monkeypatch.setenv("LAYA_LOAD_PEER", peer)
    path = tiny_paths["small-llama-q8_0"] if "small-llama-q8_0" in tiny_paths else tiny_paths["tiny-llama-q8_0"]
    rng = np.random.default_rng(12)
    prompts = [synth.token_ids(rng, 1000, int(n_)) for n_ in (40, 7, 300, 64, 90, 12, 128, 33)]
    qs = [Question("choice", [10, 11, 12, 13])]
    with engine.Engine(path, devices=[0]) as one, engine.Engine(path, devices=list(range(n))) as many:
        assert many.info["n_devices"] == n
        assert many.info["device_bytes"] == one.info["device_bytes"]
        a = one.decide_batch(prompts, qs)
        b = many.decide_batch(prompts, qs)
    for i in range(len(prompts)):
        assert np.allclose(a[i][0]["probabilities"], b[i][0]["probabilities"], atol=2e-4), i
