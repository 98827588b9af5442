"""OpenThai's decision rules pinned to the reference's saved upstream outputs
(tests/golden/openthai_slots.json, made by make_openthai_slots.py from the
reference's validation/openthai.reference.json): ten requests with the slot
head's raw logits of their first pass and the upstream answers.

* Slot decoding (decision.rs:264-380): for every request answered in one
  pass, `openthai.decide` on the saved logits gives the saved answers.  The
  model's three temperatures are not in the fixture; they are fitted from
  one request (the ratio of two option probabilities fixes the logit scale)
  and the fit must agree with every other single-pass request.
* Permutation counts (decision.rs:136-162) for all ten.
* The prompt's control tokens (decision.rs:169-233): with a vocabulary that
  puts <|ts_*|> at the model's ids (248077..), the first pass's sequence of
  control tokens and the answer positions' tokens match the saved prompt.
  Text between them depends on the model's BPE merges, which the fixture
  does not carry.
"""
import json
import os

import numpy as np
import pytest

from laya_goish_b200 import openthai as ot
from laya_goish_b200.tokenizer import Tokenizer, byte_alphabet

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "openthai_slots.json")
STATE_ID, ANSWER_ID, OPT0_ID, VOCAB = 248077, 248082, 248083, 248339


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN, encoding="utf-8") as f:
        return json.load(f)


def logits(g, nq):
    return np.array(g["raw_logits"], np.float32).reshape(nq, 256)


def fitted_temperature(row, p_hi, p_lo):
    # softmax over slots divided by T: log(p1 / p0) = (l1 - l0) / T
    return float((row[1] - row[0]) / np.log(p_hi / p_lo))


def temperatures(golden):
    g = golden[1]  # choice, score and noul questions in one request
    L, a = logits(g, 3), g["response"]["answers"]
    return [fitted_temperature(L[0], a["department"]["probabilities"]["technical"],
                               a["department"]["probabilities"]["billing"]),
            fitted_temperature(L[1], a["frustration"]["probabilities"]["1"], a["frustration"]["probabilities"]["0"]),
            fitted_temperature(L[2], a["refund_requested"]["noul"], 1 - a["refund_requested"]["noul"])]


def test_fixture_shape(golden):
    assert len(golden) == 10
    for g in golden:
        nq = len(g["request"]["questions"])
        assert len(g["raw_logits"]) == 256 * nq and len(g["answer_positions"]) == nq
        assert g["response"]["usage"]["input_tokens"] == g["n_tokens"]
        ctl = dict((p, t) for p, t in g["control"])
        assert ctl[0] == STATE_ID and all(ctl[p] == ANSWER_ID for p in g["answer_positions"])


def test_temperature_fit_is_consistent(golden):
    T = temperatures(golden)
    for i, g in enumerate(golden):
        qs = ot.questions(g["request"])
        if ot.permutation_count(g["request"], qs) != 1:
            continue
        L, ans = logits(g, len(qs)), g["response"]["answers"]
        for j, q in enumerate(qs):
            a = ans[q.id]
            if q.kind == 2:
                t = fitted_temperature(L[j], a["noul"], 1 - a["noul"])
            elif len(q.names) >= 2:
                pr = a["probabilities"]
                keys = q.names if q.kind == 0 else ["0", "1"]
                t = fitted_temperature(L[j], pr[keys[1]], pr[keys[0]])
            else:
                continue
            assert t == pytest.approx(T[q.kind], rel=2e-5), (i, q.id)


def test_slot_decoding_matches_upstream(golden):
    T = np.array(temperatures(golden), np.float32)
    checked = 0
    for i, g in enumerate(golden):
        qs = ot.questions(g["request"])
        if ot.permutation_count(g["request"], qs) != 1:
            continue
        got = ot.decide(qs, [(logits(g, len(qs)), [list(range(len(q.names))) for q in qs])], T)
        for q in qs:
            a, b = got[q.id], g["response"]["answers"][q.id]
            assert set(a) == set(b), (i, q.id)
            for k, want in b.items():
                if k == "probabilities":
                    assert set(a[k]) == set(want)
                    assert max(abs(a[k][x] - want[x]) for x in want) < 1e-6, (i, q.id)
                elif isinstance(want, float):
                    assert a[k] == pytest.approx(want, abs=1e-6), (i, q.id, k)
                else:
                    assert a[k] == want, (i, q.id, k)
            checked += 1
    assert checked == 10  # the eight single-pass requests hold ten questions


def test_permutation_counts_match_upstream(golden):
    for g in golden:
        qs = ot.questions(g["request"])
        assert ot.permutation_count(g["request"], qs) == g["response"]["usage"]["permutations"]


@pytest.fixture(scope="module")
def model_ids_tokenizer():
    control = ["<|ts_state|>", "<|ts_q|>", "<|ts_choice|>", "<|ts_score|>", "<|ts_noul|>", "<|ts_answer|>"] + \
              [f"<|ts_opt_{i}|>" for i in range(256)]
    tokens = byte_alphabet() + [f"<pad_{i}>" for i in range(256, STATE_ID)] + control
    assert len(tokens) == VOCAB and tokens[ANSWER_ID] == "<|ts_answer|>" and tokens[OPT0_ID] == "<|ts_opt_0|>"
    types = [1] * STATE_ID + [3] * len(control)
    return Tokenizer({"tokenizer.ggml.pre": "qwen2", "tokenizer.ggml.tokens": tokens,
                      "tokenizer.ggml.token_type": types, "tokenizer.ggml.merges": []})


def test_prompt_control_tokens_match_upstream(golden, model_ids_tokenizer):
    tok = model_ids_tokenizer
    for i, g in enumerate(golden):
        req = g["request"]
        qs = ot.questions(req)
        n = ot.permutation_count(req, qs)
        e = ot.encode(tok, req, qs, n, 0, ANSWER_ID)
        ours = [t for t in e.ids if t >= STATE_ID]
        assert ours == [t for _, t in g["control"]], i
        assert [e.ids[p] for p in e.positions] == [ANSWER_ID] * len(qs)
        assert all(e.ids[p + 1] == tok.vocab["Ċ"] for p in e.positions)  # each answer token ends its line
        assert not e.truncated
