"""OpenThai's gated DeltaNet recurrence on the GPU (laya_gated_delta) against
the oracle's restatement of Delta::run (src/models/openthai/model.rs:322-355).
Parity with the reference itself is unpinned (its goldens need the real
OpenThai weights)."""
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
    assert np.allclose(got, want, atol=1e-4, rtol=1e-3), np.abs(got - want).max()


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
