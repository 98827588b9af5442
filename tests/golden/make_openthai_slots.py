"""Generates the committed OpenThai decision goldens (openthai_slots.json).

Source: the reference's saved upstream outputs for its OpenThai validation
requests (validation/openthai.requests.json and openthai.reference.json in
the laya-goish project, written by validation/openthai_reference.py from the
upstream CPU/F32 model).  Kept per request: the request, the number of
prompt tokens, the control tokens of the first pass's prompt (position and
id, ids >= 248077), its answer positions, the slot head's raw logits of that
pass and the upstream response (answers and usage).

Run: python tests/golden/make_openthai_slots.py <laya-goish checkout>
"""
import json
import os
import sys

CONTROL_MIN = 248077  # <|ts_state|>; the <|ts_*|> control tokens follow it


def main(root: str) -> None:
    v = os.path.join(root, "validation")
    with open(os.path.join(v, "openthai.requests.json"), encoding="utf-8") as f:
        reqs = json.load(f)
    with open(os.path.join(v, "openthai.reference.json"), encoding="utf-8") as f:
        refs = json.load(f)
    if len(reqs) != len(refs):
        raise SystemExit("requests and reference outputs differ in length")
    out = []
    for req, ref in zip(reqs, refs):
        ids = ref["input_ids"]
        out.append({"request": req, "n_tokens": len(ids),
                    "control": [[i, t] for i, t in enumerate(ids) if t >= CONTROL_MIN],
                    "answer_positions": ref["answer_positions"], "raw_logits": ref["raw_logits"],
                    "response": ref["response"]})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "openthai_slots.json")
    with open(path, "w", encoding="utf-8") as f:
        json.dump(out, f, ensure_ascii=False, separators=(",", ":"))
        f.write("\n")
    print(path, os.path.getsize(path))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
