"""GPU checks of the GEMM that decodes Q8_0 blocks in its shared-memory
staging (gemm_q8_launch), used for passes of at most 256 token rows over
Q8_0 models: the forward against the CPU oracle, bitwise agreement with the
resident-F16-operand path when neither splits K (both round d * q once to
F16 and issue the same MMAs), no F16 operand cache allocated, and batched
decode steps (K-split Q8_0 GEMMs, Q8_0 lm_head) against the oracle's greedy
loop.  LAYA_Q8_FUSED / LAYA_KSPLIT are read by the library at every call."""
import numpy as np
import pytest

import oracle
from laya_goish_b200 import engine, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_q8(tiny_paths):
    path = tiny_paths["small-llama-q8_0"]
    o = oracle.Model(open(path, "rb").read(), threads=8, attn_threads=8)
    yield path, o
    o.close()


@pytest.mark.parametrize("n", [1, 37, 128, 129, 256])
def test_fused_forward_matches_oracle(small_q8, n):
    path, o = small_q8
    rng = np.random.default_rng(300 + n)
    ids = synth.token_ids(rng, o.vocab, n)
    read = sorted({0, n // 2, n - 1})
    with engine.Engine(path) as e:
        got = e.forward(ids, read)
    want = o.forward(ids, read)
    err = np.abs(got - want)
    assert err.max() < 3e-2 and err.mean() < 3e-3, (err.max(), err.mean())


@pytest.mark.parametrize("n", [130, 256])
def test_fused_forward_bitwise_equal_to_f16_operands(small_q8, monkeypatch, n):
    # with K unsplit both paths run the same 256 x 256 CTA-pair tiles over
    # identical F16 operand values, so the hidden rows agree bit for bit
    path, o = small_q8
    monkeypatch.setenv("LAYA_KSPLIT", "0")
    rng = np.random.default_rng(500 + n)
    ids = synth.token_ids(rng, o.vocab, n)
    read = list(range(0, n, 7))
    with engine.Engine(path) as e:
        fused = e.forward(ids, read)
        monkeypatch.setenv("LAYA_Q8_FUSED", "0")
        cached = e.forward(ids, read)
    assert np.array_equal(fused.view(np.uint32), cached.view(np.uint32)), np.abs(fused - cached).max()


def test_fused_forward_allocates_no_f16_cache(small_q8, monkeypatch):
    import torch

    path, o = small_q8
    cfg = synth.TINY["small-llama-q8_0"]
    cache_bytes = 2 * cfg.matrix_params()
    rng = np.random.default_rng(9)
    ids = synth.token_ids(rng, o.vocab, 100)
    with engine.Engine(path) as e:
        e.forward(ids, [99])
        free0 = torch.cuda.mem_get_info(0)[0]
        e.forward(ids, [99])  # fused again: nothing new to allocate
        free1 = torch.cuda.mem_get_info(0)[0]
        monkeypatch.setenv("LAYA_Q8_FUSED", "0")
        e.forward(ids, [99])  # the F16 path builds its resident operand cache now
        free2 = torch.cuda.mem_get_info(0)[0]
    assert free0 - free1 < cache_bytes // 4, (free0, free1)
    assert free1 - free2 >= cache_bytes * 9 // 10, (free1, free2, cache_bytes)


@pytest.mark.parametrize("nseq", [24, 64, 200])
def test_batched_decode_on_q8_blocks_matches_oracle(small_q8, nseq):
    path, o = small_q8
    rng = np.random.default_rng(nseq)
    ctxs = [synth.token_ids(rng, o.vocab, int(n)) for n in rng.integers(5, 60, size=nseq)]
    steps = 3
    with engine.Engine(path) as e:
        toks, _ = e.decode(ctxs, steps)
    checked = 0
    for i in range(0, nseq, max(1, nseq // 12)):
        seq = list(ctxs[i])
        for s in range(steps):
            h = o.forward(np.array(seq, np.int32), [len(seq) - 1])
            logits = o.head(h)[0]
            order = np.argsort(-logits, kind="stable")
            if logits[order[0]] - logits[order[1]] < 2e-2:
                break  # near-tie: F16 rounding may pick the other token; later steps diverge
            assert toks[i, s] == order[0], (i, s, toks[i], int(order[0]))
            checked += 1
            seq.append(int(order[0]))
    assert checked >= nseq // max(1, nseq // 12)
