"""GPU parity of the single-function entry points against the CPU oracle:
gguf::decode (bit-exact), Matrix::apply, and the upload transcoding of
every GGUF tensor type into its HBM layout (bit-exact)."""
import os

import numpy as np
import pytest

import oracle
from laya_goish_b200 import engine, synth

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "dequant.npz")


@pytest.mark.parametrize("kind", [0, 1, 2, 8, 12, 14])
def test_dequantize_golden_bit_exact(kind):
    g = np.load(GOLD)
    got = engine.dequantize(kind, g[f"raw_{kind}"])
    want = g[f"want_{kind}"]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kind", [2, 8, 12, 14])
def test_dequantize_large_matches_oracle(kind):
    rng = np.random.default_rng(kind)
    x = (rng.standard_normal(256 * 4096, dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
    raw = synth.encode(kind, x)
    assert np.array_equal(engine.dequantize(kind, raw).view(np.uint32), oracle.decode(kind, raw).view(np.uint32))


def test_dequantize_empty():
    assert engine.dequantize(8, b"").size == 0


def test_matrix_self_test():
    # src/tensor.rs:196-214 with inputs rounded to F16 (the tensor-core
    # operand type), so products are exact and only summation order differs.
    w = ((np.arange(187, dtype=np.float32) - 83.0) / 71.0).astype(np.float16).astype(np.float32).reshape(11, 17)
    x = ((np.arange(153, dtype=np.float32) - 71.0) / 43.0).astype(np.float16).astype(np.float32).reshape(9, 17)
    b = np.full(11, 0.25, np.float32)
    y = engine.matrix_apply(0, w.tobytes(), 11, 17, x, b)
    want = oracle.matrix_apply(w, x, b, 4)
    assert np.abs(y - want).max() <= 1e-4


@pytest.mark.parametrize("kind,m,rows,cols", [(1, 1, 256, 512), (8, 3, 300, 2048), (12, 17, 520, 1024),
                                              (14, 130, 256, 768), (2, 257, 384, 256), (1, 1000, 1000, 2048)])
def test_matrix_apply_matches_oracle(kind, m, rows, cols):
    rng = np.random.default_rng(m + rows)
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
    raw = synth.encode(kind, w)
    wd = oracle.decode(kind, raw).reshape(rows, cols)
    x = rng.standard_normal((m, cols), dtype=np.float32).astype(np.float16).astype(np.float32)
    bias = rng.standard_normal(rows, dtype=np.float32)
    y = engine.matrix_apply(kind, raw, rows, cols, x, bias)
    want = oracle.matrix_apply(wd, x, bias, 8)
    # F16 operands: x exact, decoded weights rounded to F16 (rel 2^-11)
    tol = 2e-3 * np.sqrt(cols) * 0.02 * 4 + 1e-4
    assert np.abs(y - want).max() < tol


@pytest.mark.parametrize("name", ["tiny-llama-f16", "tiny-llama-q8_0", "tiny-llama-q4_k_m", "tiny-llama-q4_0",
                                  "tiny-qwen2-f16"])
def test_upload_transcoding_bit_exact(tiny_paths, name):
    blob = open(tiny_paths[name], "rb").read()
    om = oracle.Model(blob)
    import gguf  # noqa: F401  (tensor table via the oracle-independent reader)
    r = gguf.GGUFReader(tiny_paths[name])
    with engine.Engine(tiny_paths[name]) as e:
        for t in r.tensors:
            if len(t.shape) != 2 or t.name.endswith("ffn_gate.weight") or t.name.endswith("ffn_up.weight"):
                continue
            if e.info["weight_kind"] in (0, 1) and t.name.startswith("blk."):
                if not any(t.name.endswith(s) for s in ("attn_q.weight", "attn_k.weight", "attn_v.weight",
                                                         "attn_output.weight", "ffn_down.weight")):
                    continue
            n = int(np.prod(t.shape))
            got = e.tensor(t.name, n)
            raw = np.array(t.data).reshape(-1).view(np.uint8)
            want = oracle.decode(int(t.tensor_type), raw)
            if int(t.tensor_type) in (0, 1) or int(t.tensor_type) in (2, 8, 12, 14):
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), t.name
    om.close()


def test_device_wait_that_runs_out_reports_timeout_and_context_survives():
    # A device-side wait that nothing completes (a fresh mbarrier nobody
    # arrives at), bounded by ~1 ms of SM cycles: the kernel records the
    # expiry and returns, the host maps it to LAYA_E_TIMEOUT, and the next
    # call on the same context succeeds.  No fault, trap or hang is involved.
    from laya_goish_b200 import _lib

    L = _lib.lib()
    assert L.laya_wait_selftest(0, 2_000_000) == _lib.E_TIMEOUT
    assert b"budget" in L.laya_last_error()
    assert L.laya_wait_selftest(0, 0) == _lib.E_INVALID
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 256), dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
    x = rng.standard_normal((5, 256), dtype=np.float32).astype(np.float16).astype(np.float32)
    got = engine.matrix_apply(1, synth.encode(1, w), 64, 256, x)
    assert np.abs(got - x @ w.T).max() < 1e-3
