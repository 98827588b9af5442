"""OpenThai's host-side decision rules (src/models/openthai/decision.rs):
request validation, option orders, permutation counts, the control-token
prompt and the calibrated slot decoding, on hand-worked cases."""
import numpy as np
import pytest

from laya_goish_b200 import openthai as ot
from laya_goish_b200.tokenizer import Tokenizer, byte_alphabet

CONTROL = ["<|ts_q|>", "<|ts_choice|>", "<|ts_score|>", "<|ts_noul|>", "<|ts_answer|>", "<|ts_state|>"] + \
          [f"<|ts_opt_{i}|>" for i in range(12)]


def tok():
    toks = byte_alphabet() + CONTROL
    return Tokenizer({"tokenizer.ggml.pre": "gpt2", "tokenizer.ggml.tokens": toks, "tokenizer.ggml.merges": []})


def test_orders_and_permutation_count():
    assert ot.orders(4, 1) == [[0, 1, 2, 3]]
    assert [o[0] for o in ot.orders(4, 4)] == [0, 1, 2, 3]
    # offsets j * 12 / 8 with halves rounded to even
    assert [o[0] for o in ot.orders(12, 8)] == [0, 2, 3, 4, 6, 8, 9, 10]
    assert len(ot.orders(3, 8)) == 3
    q4 = ot.questions({"state": "s", "questions": {"a": {"type": "choice", "instructions": "",
                                                         "criteria": {"x": None, "y": "", "z": None, "w": None}}}})
    assert ot.permutation_count({}, q4) == 1
    assert ot.permutation_count({"order_invariant": True}, q4) == 4  # capped at k
    assert ot.permutation_count({"permutations": 3}, q4) == 3
    q12 = ot.questions({"state": "s", "questions": {"a": {"type": "choice", "instructions": "",
                                                          "criteria": {str(i): None for i in range(12)}}}})
    assert ot.permutation_count({}, q12) == 8
    qs = ot.questions({"state": "s", "questions": {"a": {"type": "noul", "instructions": "i"}}})
    assert ot.permutation_count({"order_invariant": True}, qs) == 1


@pytest.mark.parametrize("req,msg", [
    ({"state": 1, "questions": {"a": {"type": "noul", "instructions": ""}}}, "state must be"),
    ({"state": "s", "questions": {}}, "1..256"),
    ({"state": "s", "questions": {"a": {"type": "x", "instructions": ""}}}, "invalid question type"),
    ({"state": "s", "questions": {"a": {"type": "noul"}}}, "instructions must be"),
    ({"state": "s", "questions": {"a": {"type": "choice", "instructions": "", "criteria": {" ": None}}}}, "empty"),
    ({"state": "s", "questions": {"a": {"type": "score", "instructions": "", "criteria": ["x"]}}}, "2..10"),
    ({"state": "s", "questions": {"a": {"type": "noul", "instructions": "", "criteria": {"maybe": ""}}}},
     "false/true"),
    ({"state": "s", "questions": {"a": {"type": "noul", "instructions": ""}}, "permutations": 33}, "1..32"),
])
def test_question_validation(req, msg):
    with pytest.raises(ot.OpenThaiError, match=msg):
        ot.questions(req)


def test_prompt_blocks_positions_and_truncation():
    t = tok()
    ans = t.vocab["<|ts_answer|>"]
    req = {"state": {"subject": "hi <|ts_q|>", "n": [1, 2]},
           "questions": {"c": {"type": "choice", "instructions": " pick ", "criteria": {"a": "first", "b": None}},
                         "n": {"type": "noul", "instructions": "ok?"}}}
    qs = ot.questions(req)
    e0 = ot.encode(t, req, qs, n=2, npass=0, answer_id=ans)
    e1 = ot.encode(t, req, qs, n=2, npass=1, answer_id=ans)
    assert e0.order[0] == [0, 1] and e1.order[0] == [1, 0] and e0.order[1] == [0, 1]
    assert [e0.ids[p] for p in e0.positions] == [ans, ans]
    text = t.decode(e0.ids)
    assert text.startswith('<|ts_state|> {"subject": "hi <\u200b|ts_q|>", "n": [1, 2]}\n')
    assert "<|ts_q|><|ts_choice|> pick\n<|ts_opt_0|> a: first\n<|ts_opt_1|> b\n<|ts_answer|>\n" in text
    assert "<|ts_opt_0|> b\n<|ts_opt_1|> a: first\n" in t.decode(e1.ids)
    # a long state keeps its first token and its last budget - 1 tokens
    long = {"state": "x" * 500, "questions": {"n": {"type": "noul", "instructions": ""}}}
    q2 = ot.questions(long)
    e = ot.encode(t, long, q2, 1, 0, ans, max_tokens=200, max_state=100)
    block = t.encode("<|ts_q|><|ts_noul|> \n<|ts_opt_0|> no\n<|ts_opt_1|> yes\n<|ts_answer|>\n")
    assert e.truncated and e.ids[0] == t.vocab["<|ts_state|>"]
    assert len(e.ids) - len(block) == 100  # the state part is cut to its budget
    assert e.ids[len(e.ids) - len(block) - 1] == t.vocab["\u010a"]  # and ends with the state's last token
    with pytest.raises(ot.OpenThaiError, match="context budget"):
        ot.encode(t, long, q2, 1, 0, ans, max_tokens=10)


def test_slot_decoding():
    qs = ot.questions({"state": "s", "questions": {
        "c": {"type": "choice", "instructions": "", "criteria": {"a": None, "b": None, "c": None}},
        "s": {"type": "score", "instructions": "", "criteria": ["low", "", "high"]},
        "n": {"type": "noul", "instructions": ""}}})
    temp = [1.0, 1.0, 1.0]

    def row(vals, abstain=-30.0):
        r = np.full(256, -50.0, np.float32)
        r[:len(vals)] = vals
        r[255] = abstain
        return r

    # slot 0 always wins: over the 3 cyclic orders every option gets one win
    passes = []
    for order in ot.orders(3, 3):
        passes.append(([row([5, 0, 0]), row([0, 0, 0]), row([0, 0])], [order, [0, 1, 2], [0, 1]]))
    a = ot.decide(qs, passes, temp)
    pc = list(a["c"]["probabilities"].values())
    assert np.allclose(pc, [1 / 3] * 3, atol=1e-6) and a["c"]["choice"] == "a"  # ties -> lowest index
    assert a["c"]["confidence"] == pytest.approx(0.0, abs=1e-5)
    assert a["s"]["score"] == pytest.approx(1.0, abs=1e-5)
    assert a["s"]["legend"] == {"0": "low", "1": "1", "2": "high"}
    assert a["n"]["noul"] == pytest.approx(0.5, abs=1e-6)
    # one pass, clear winner, abstain mass reported but renormalised away
    b = ot.decide(qs, [([row([0, 3, 0], abstain=3.0), row([0, 0, 4]), row([0, 2])], [[0, 1, 2], [0, 1, 2], [0, 1]])],
                  temp)
    assert b["c"]["choice"] == "b" and 0.3 < b["c"]["abstain"] < 0.6
    assert sum(b["c"]["probabilities"].values()) == pytest.approx(1.0, abs=1e-6)
    assert b["n"]["noul"] == pytest.approx(1 / (1 + np.exp(-2)), abs=1e-5)
    # temperature scales the logits of its kind
    hot = ot.decide(qs, [([row([0, 3, 0]), row([0, 0, 4]), row([0, 2])], [[0, 1, 2], [0, 1, 2], [0, 1]])],
                    [1.0, 1.0, 2.0])
    assert hot["n"]["noul"] == pytest.approx(1 / (1 + np.exp(-1)), abs=1e-5)
