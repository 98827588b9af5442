"""The oracle's OpenThai sequence mixers (oracle/openthai.c) against an
independent float64 NumPy restatement of the same equations
(src/models/openthai/model.rs:243-363), at the reference's head layouts on
small widths, plus the properties the equations imply (causality, the gate
at zero, the decay limit).  Parity with the reference itself is unpinned:
its goldens need the real OpenThai weights."""
import numpy as np
import pytest

import oracle


def rms(x, w, off):
    d = w.shape[0]
    x = x.reshape(-1, d)
    return x / np.sqrt((x * x).sum(1, keepdims=True) / d + 1e-6) * (off + w)


def sigmoid(x):
    return 1 / (1 + np.exp(-x))


def ref_full(x, wq, wk, wv, wo, qn, kn, H, KV, hd, rot, theta):
    s = x.shape[0]
    qg = (x @ wq.T).reshape(s, H, 2 * hd)
    q, gate = qg[:, :, :hd], qg[:, :, hd:]
    q = rms(q, qn, 1).reshape(s, H, hd)
    k = rms(x @ wk.T, kn, 1).reshape(s, KV, hd)
    v = (x @ wv.T).reshape(s, KV, hd)
    half = rot // 2
    ang = np.arange(s)[:, None] / theta ** (2 * np.arange(half) / rot)[None, :]
    co, si = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    for t in (q, k):
        a, b = t[:, :, :half].copy(), t[:, :, half:rot].copy()
        t[:, :, :half] = a * co - b * si
        t[:, :, half:rot] = b * co + a * si
    out = np.zeros((s, H, hd))
    g = H // KV
    for h in range(H):
        sc = q[:, h] @ k[:, h // g].T / np.sqrt(hd)
        sc[np.triu_indices(s, 1)] = -np.inf
        p = np.exp(sc - sc.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        out[:, h] = p @ v[:, h // g]
    out = out * sigmoid(gate)
    return out.reshape(s, H * hd) @ wo.T


def ref_delta(x, wqkv, wz, wa, wb, wo, conv, dt, alog, normw, nh, hk):
    s = x.shape[0]
    w = nh * hk
    raw = x @ wqkv.T
    z, a, b = x @ wz.T, x @ wa.T, x @ wb.T
    pad = np.vstack([np.zeros((3, raw.shape[1])), raw])
    conv_out = sum(pad[j:j + s] * conv[:, j][None, :] for j in range(4))
    qkv = conv_out * sigmoid(conv_out)
    out = np.zeros((s, w))
    for h in range(nh):
        st = np.zeros((hk, hk))
        for i in range(s):
            q = qkv[i, h * hk:(h + 1) * hk]
            k = qkv[i, w + h * hk:w + (h + 1) * hk]
            v = qkv[i, 2 * w + h * hk:2 * w + (h + 1) * hk]
            q = q / np.sqrt(q @ q + 1e-6) / np.sqrt(hk)
            k = k / np.sqrt(k @ k + 1e-6)
            sp = a[i, h] + dt[h]
            sp = sp if sp > 20 else np.log1p(np.exp(sp))
            st *= np.exp(-np.exp(alog[h]) * sp)
            delta = (v - k @ st) * sigmoid(b[i, h])
            st += np.outer(k, delta)
            out[i, h * hk:(h + 1) * hk] = q @ st
    out = rms(out, normw, 0).reshape(s, w) * (z * sigmoid(z))
    return out @ wo.T


@pytest.mark.parametrize("s", [1, 5, 37])
def test_gated_full_attention_matches_float64(s):
    rng = np.random.default_rng(s)
    d, H, KV, hd, rot = 48, 4, 2, 32, 8  # the reference: 1024, 8, 2, 256, 64
    x = rng.normal(0, 1, (s, d))
    wq = rng.normal(0, 0.1, (2 * H * hd, d))
    wk, wv = rng.normal(0, 0.1, (KV * hd, d)), rng.normal(0, 0.1, (KV * hd, d))
    wo = rng.normal(0, 0.1, (d, H * hd))
    qn, kn = rng.normal(0, 0.1, hd), rng.normal(0, 0.1, hd)
    got = oracle.ot_full(x, wq, wk, wv, wo, qn, kn, H, KV, hd, rot, 1e7)
    want = ref_full(x, wq, wk, wv, wo, qn, kn, H, KV, hd, rot, 1e7)
    assert np.allclose(got, want, atol=2e-4, rtol=2e-3), np.abs(got - want).max()
    # causal: the first rows do not see later tokens
    if s > 3:
        got2 = oracle.ot_full(x[:3], wq, wk, wv, wo, qn, kn, H, KV, hd, rot, 1e7)
        assert np.array_equal(got2, got[:3])


@pytest.mark.parametrize("s", [1, 4, 29])
def test_gated_deltanet_matches_float64(s):
    rng = np.random.default_rng(100 + s)
    d, nh, hk = 40, 3, 16  # the reference: 1024, 16, 128
    w = nh * hk
    x = rng.normal(0, 1, (s, d))
    wqkv = rng.normal(0, 0.2, (3 * w, d))
    wz, wa, wb = rng.normal(0, 0.2, (w, d)), rng.normal(0, 0.5, (nh, d)), rng.normal(0, 0.5, (nh, d))
    wo = rng.normal(0, 0.1, (d, w))
    conv = rng.normal(0, 0.5, (3 * w, 4))
    dt, alog, normw = rng.normal(0, 0.5, nh), rng.normal(-1, 0.3, nh), rng.normal(1, 0.1, hk)
    got = oracle.ot_delta(x, wqkv, wz, wa, wb, wo, conv, dt, alog, normw, nh, hk)
    want = ref_delta(x, wqkv, wz, wa, wb, wo, conv, dt, alog, normw, nh, hk)
    assert np.allclose(got, want, atol=2e-4, rtol=2e-3), np.abs(got - want).max()
    if s > 2:
        got2 = oracle.ot_delta(x[:2], wqkv, wz, wa, wb, wo, conv, dt, alog, normw, nh, hk)
        assert np.array_equal(got2, got[:2])  # causal (conv and recurrence)


def test_bad_shapes_rejected():
    x = np.zeros((2, 8), np.float32)
    z = np.zeros(64, np.float32)
    with pytest.raises(ValueError):
        oracle.ot_full(x, z, z, z, z, z, z, H=3, KV=2, hd=4, rot=4, theta=1e7)  # H % KV != 0
