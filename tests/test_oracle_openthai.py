"""The oracle's OpenThai sequence mixers (oracle/openthai.c) and the forward
composed from them (oracle.ot_forward) against an independent float64 NumPy
restatement of the same equations (src/models/openthai/model.rs:192-363),
at the reference's head layouts on small widths, plus causality.  Parity
with the reference itself is unpinned: its goldens need the real OpenThai
weights."""
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


def ref_forward(m, ids, positions):
    c = m["config"]
    x = m["model.embed_tokens.weight"][np.asarray(ids)].astype(np.float64)
    for i, kind in enumerate(c["layer_types"]):
        p = f"model.layers.{i}"
        h = rms(x, m[f"{p}.input_layernorm.weight"], 1).reshape(x.shape)
        if kind == "full_attention":
            y = ref_full(h, m[f"{p}.self_attn.q_proj.weight"], m[f"{p}.self_attn.k_proj.weight"],
                         m[f"{p}.self_attn.v_proj.weight"], m[f"{p}.self_attn.o_proj.weight"],
                         m[f"{p}.self_attn.q_norm.weight"], m[f"{p}.self_attn.k_norm.weight"], c["heads"],
                         c["kv_heads"], c["head_dim"], c["rot"], c["theta"])
        else:
            y = ref_delta(h, m[f"{p}.linear_attn.in_proj_qkv.weight"], m[f"{p}.linear_attn.in_proj_z.weight"],
                          m[f"{p}.linear_attn.in_proj_a.weight"], m[f"{p}.linear_attn.in_proj_b.weight"],
                          m[f"{p}.linear_attn.out_proj.weight"], m[f"{p}.linear_attn.conv1d.weight"],
                          m[f"{p}.linear_attn.dt_bias"], m[f"{p}.linear_attn.A_log"],
                          m[f"{p}.linear_attn.norm.weight"], c["lin_heads"], c["lin_dim"])
        x = x + y
        h = rms(x, m[f"{p}.post_attention_layernorm.weight"], 1).reshape(x.shape)
        g, u = h @ m[f"{p}.mlp.gate_proj.weight"].T, h @ m[f"{p}.mlp.up_proj.weight"].T
        x = x + (g * sigmoid(g) * u) @ m[f"{p}.mlp.down_proj.weight"].T
    ans = rms(x[np.asarray(positions)], m["model.norm.weight"], 1).reshape(len(positions), -1)
    return ans @ m["slot_head.weight"].T + m["slot_head.bias"]


def tiny_openthai(rng):
    d, ffn, V, slots = 48, 96, 300, 16
    c = {"heads": 4, "kv_heads": 2, "head_dim": 32, "rot": 8, "theta": 1e7, "lin_heads": 2, "lin_dim": 16,
         "layer_types": ["linear_attention", "linear_attention", "full_attention", "linear_attention"]}
    H, KV, hd, nh, hk = c["heads"], c["kv_heads"], c["head_dim"], c["lin_heads"], c["lin_dim"]
    w = nh * hk
    n = lambda *shape, sd=0.05: rng.normal(0, sd, shape).astype(np.float32)  # noqa: E731
    m = {"config": c, "model.embed_tokens.weight": n(V, d, sd=1.0), "model.norm.weight": n(d),
         "slot_head.weight": n(slots, d, sd=0.2), "slot_head.bias": n(slots)}
    for i, kind in enumerate(c["layer_types"]):
        p = f"model.layers.{i}"
        m.update({f"{p}.input_layernorm.weight": n(d), f"{p}.post_attention_layernorm.weight": n(d),
                  f"{p}.mlp.gate_proj.weight": n(ffn, d, sd=0.1), f"{p}.mlp.up_proj.weight": n(ffn, d, sd=0.1),
                  f"{p}.mlp.down_proj.weight": n(d, ffn, sd=0.1)})
        if kind == "full_attention":
            m.update({f"{p}.self_attn.q_proj.weight": n(2 * H * hd, d, sd=0.1),
                      f"{p}.self_attn.k_proj.weight": n(KV * hd, d, sd=0.1),
                      f"{p}.self_attn.v_proj.weight": n(KV * hd, d, sd=0.1),
                      f"{p}.self_attn.o_proj.weight": n(d, H * hd, sd=0.1),
                      f"{p}.self_attn.q_norm.weight": n(hd), f"{p}.self_attn.k_norm.weight": n(hd)})
        else:
            m.update({f"{p}.linear_attn.in_proj_qkv.weight": n(3 * w, d, sd=0.2),
                      f"{p}.linear_attn.in_proj_z.weight": n(w, d, sd=0.2),
                      f"{p}.linear_attn.in_proj_a.weight": n(nh, d, sd=0.3),
                      f"{p}.linear_attn.in_proj_b.weight": n(nh, d, sd=0.3),
                      f"{p}.linear_attn.out_proj.weight": n(d, w, sd=0.1),
                      f"{p}.linear_attn.conv1d.weight": n(3 * w, 4, sd=0.5),
                      f"{p}.linear_attn.dt_bias": n(nh, sd=0.5), f"{p}.linear_attn.A_log": n(nh, sd=0.3) - 1,
                      f"{p}.linear_attn.norm.weight": 1 + n(hk)})
    return m


@pytest.mark.parametrize("s", [1, 9, 40])
def test_openthai_forward_matches_float64(s):
    rng = np.random.default_rng(300 + s)
    m = tiny_openthai(rng)
    ids = rng.integers(0, 300, size=s)
    pos = sorted({0, s // 2, s - 1})
    got = oracle.ot_forward(m, ids, pos)
    want = ref_forward(m, ids, pos)
    assert got.shape == (len(pos), 16)
    assert np.allclose(got, want, atol=2e-3, rtol=2e-3), np.abs(got - want).max()


def test_openthai_gguf_round_trip_and_forward(tmp_path):
    from laya_goish_b200 import openthai, synth

    path = synth.write_openthai(str(tmp_path / "ot.gguf"), seed=5)
    with pytest.raises(openthai.OpenThaiError, match="unsupported OpenThai config"):
        openthai.load_weights(path)  # the reference loads only its one size
    m = openthai.load_weights(path, strict=False)
    c = m["config"]
    assert (c["d"], c["heads"], c["kv_heads"], c["head_dim"], c["rot"]) == (48, 4, 2, 32, 8)
    assert c["layer_types"][2] == "full_attention" and c["max_state"] == 256
    assert m["model.layers.0.linear_attn.in_proj_qkv.weight"].shape == (96, 48)
    assert m["model.layers.0.linear_attn.conv1d.weight"].shape == (96 * 4,)
    for i in (0, 1, 3):  # the [3w][4] view of the convolution kernel for the float64 restatement
        k = f"model.layers.{i}.linear_attn.conv1d.weight"
        m[k] = m[k].reshape(-1, 4)
    rng = np.random.default_rng(9)
    ids = rng.integers(0, 300, size=23)
    pos = [0, 11, 22]
    got = oracle.ot_forward(m, ids, pos)
    want = ref_forward(m, ids, pos)
    assert got.shape == (3, 256)
    assert np.allclose(got, want, atol=2e-3, rtol=2e-3), np.abs(got - want).max()
    assert np.allclose(m["temperature"], np.exp(m["log_temperature"]))


def test_openthai_quantised_gguf_decodes_through_the_oracle(tmp_path):
    # the reference decodes any supported block type when it loads OpenThai
    # matrices (src/models/openthai/model.rs:61 -> src/gguf.rs:250-336)
    from laya_goish_b200 import openthai, synth
    from laya_goish_b200.gguf_meta import GGUFError

    path = synth.write_openthai(str(tmp_path / "ot_q8.gguf"), seed=5, d=64, ffn=128, quant=synth.Q8_0)
    with pytest.raises(GGUFError, match="not F32/F16"):
        openthai.load_weights(path, strict=False)  # a block type needs a decoder
    m = openthai.load_weights(path, strict=False, decode=oracle.decode)
    f = openthai.load_weights(synth.write_openthai(str(tmp_path / "ot_f16.gguf"), seed=5, d=64, ffn=128),
                              strict=False)
    w = "model.layers.0.mlp.gate_proj.weight"
    assert m[w].shape == f[w].shape == (128, 64)
    # Q8_0 of the same F16 draw: within half a quantisation step per block
    step = np.abs(f[w]).reshape(-1, 32).max(axis=1) / 127
    assert (np.abs(m[w] - f[w]).reshape(-1, 32).max(axis=1) <= 0.5 * step + 1e-3).all()
    assert np.array_equal(m["model.norm.weight"], f["model.norm.weight"])  # vectors stay F32
