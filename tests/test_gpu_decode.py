"""KV-cached greedy decode against the oracle's recompute-everything greedy
loop (parity unpinned: the reference has no decode).  Tokens must agree
until the oracle's top-2 logit margin falls inside the F16 tolerance."""
import numpy as np
import pytest

import oracle
from laya_goish_b200 import engine, synth

pytestmark = pytest.mark.gpu


def oracle_greedy(o, ctx, steps):
    seq = list(ctx)
    toks, margins = [], []
    for _ in range(steps):
        h = o.forward(np.array(seq, np.int32), [len(seq) - 1])
        logits = o.head(h)[0]
        order = np.argsort(-logits, kind="stable")
        toks.append(int(order[0]))
        margins.append(float(logits[order[0]] - logits[order[1]]))
        seq.append(int(order[0]))
    return toks, margins


@pytest.mark.parametrize("name,nseq", [("tiny-llama-q8_0", 1), ("tiny-llama-f16", 3), ("tiny-qwen2-f16", 2),
                                       ("tiny-llama-q4_k_m", 8), ("tiny-llama-q8_0", 20),
                                       ("small-llama-q8_0", 16), ("tiny-llama-q8_0", 9), ("tiny-llama-f16", 12),
                                       # past the GEMV batch on F16 operands: K-split GEMMs
                                       ("small-llama-f16", 20), ("tiny-llama-q4_k_m", 24)])
def test_greedy_decode_matches_oracle(tiny_paths, name, nseq):
    path = tiny_paths[name]
    o = oracle.Model(open(path, "rb").read(), threads=8, attn_threads=8)
    rng = np.random.default_rng(nseq)
    ctxs = [synth.token_ids(rng, o.vocab, int(n)) for n in rng.integers(5, 140, size=nseq)]
    steps = 6
    with engine.Engine(path) as e:
        toks, stats = e.decode(ctxs, steps)
    assert toks.shape == (nseq, steps) and stats["decode_ms"] >= 0
    for i, c in enumerate(ctxs):
        want, margins = oracle_greedy(o, c, steps)
        for s in range(steps):
            if margins[s] < 2e-2:
                break  # near-tie: F16 rounding may pick the other token; later steps diverge
            assert toks[i, s] == want[s], (name, i, s, toks[i], want)
    o.close()


@pytest.mark.parametrize("name,nseq,lo,hi", [("tiny-llama-q8_0", 2, 250, 400), ("tiny-qwen2-f16", 3, 450, 520),
                                            ("small-llama-q8_0", 2, 700, 900)])
def test_greedy_decode_mid_contexts_match_oracle(tiny_paths, name, nseq, lo, hi):
    # 4-15 pages per sequence: the decode attention's key splits run as
    # clusters of 4 or 8 CTAs that merge in the leader's shared memory
    path = tiny_paths[name]
    o = oracle.Model(open(path, "rb").read(), threads=8, attn_threads=8)
    rng = np.random.default_rng(77 + nseq)
    ctxs = [synth.token_ids(rng, o.vocab, int(n)) for n in rng.integers(lo, hi, size=nseq)]
    steps = 4
    with engine.Engine(path) as e:
        toks, _ = e.decode(ctxs, steps)
    for i, c in enumerate(ctxs):
        want, margins = oracle_greedy(o, c, steps)
        for s in range(steps):
            if margins[s] < 2e-2:
                break
            assert toks[i, s] == want[s], (name, i, s, toks[i], want)
    o.close()


@pytest.mark.parametrize("name,nseq", [("small-llama-q8_0", 1), ("small-llama-q8_0", 8), ("tiny-llama-f16", 4)])
def test_chained_gemv_step_matches_per_launch_step(tiny_paths, monkeypatch, name, nseq):
    # One cooperative launch per layer (grid barriers between the GEMV phases)
    # does the same arithmetic as one launch per GEMV: identical tokens.
    path = tiny_paths[name]
    rng = np.random.default_rng(100 + nseq)
    ctxs = [synth.token_ids(rng, 1000, int(n)) for n in rng.integers(5, 90, size=nseq)]
    with engine.Engine(path) as e:
        chained, _ = e.decode(ctxs, 12)
        monkeypatch.setenv("LAYA_DECODE_SEQ", "0")
        separate, _ = e.decode(ctxs, 12)
    assert np.array_equal(chained, separate)
