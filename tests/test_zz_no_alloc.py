"""laya_matrix_apply_static: the allocation-free Matrix::apply.

Callers whose process already hands all of HBM to its own pool, or whose
thread must not stall on cudaMalloc/cudaFree, pass device buffers they own;
the library stages the GEMM operands in its fixed static array instead of
allocating.  This file is collected last so that a failure here, under -x,
comes after every other test has run.  The inputs below are allocated by the
test (with torch) — only the entry point itself must not allocate.  Two
calls in a row check that the shared array is reused correctly; each result
is compared with the existing laya_matrix_apply on the same inputs and with
the oracle, and the second call must leave the device's free memory as it
was."""
import ctypes

import numpy as np
import pytest

import oracle
from laya_goish_b200 import _lib, engine, synth

pytestmark = pytest.mark.gpu


def _static_apply(kind, raw, rows, cols, x, bias, free_bytes=None):
    """Runs the entry point on device buffers the test owns; free_bytes, when
    given, receives the device's free memory just before and just after the
    call (cudaMemGetInfo), which stays the same if the call allocates
    nothing."""
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    w_d = torch.from_numpy(np.ascontiguousarray(raw, np.uint8)).to(dev)
    x_d = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev)
    b_d = torch.from_numpy(np.ascontiguousarray(bias, np.float32)).to(dev)
    out_d = torch.full((x.shape[0], rows), float("nan"), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize()
    before = torch.cuda.mem_get_info(dev)[0]
    rc = _lib.lib().laya_matrix_apply_static(kind, ctypes.c_void_p(w_d.data_ptr()), rows, cols,
                                             ctypes.c_void_p(x_d.data_ptr()), x.shape[0],
                                             ctypes.c_void_p(b_d.data_ptr()), ctypes.c_void_p(out_d.data_ptr()),
                                             ctypes.c_void_p(stream.cuda_stream))
    after = torch.cuda.mem_get_info(dev)[0]
    _lib.check(rc)
    if free_bytes is not None:
        free_bytes.append((before, after))
    return out_d.cpu().numpy()


# (type, m, rows, cols): m <= 128 runs the one-CTA GEMM, m > 128 the CTA-pair
# GEMM whose tensor maps then point into the static array as well
@pytest.mark.parametrize("kind,m,rows,cols", [(8, 37, 300, 1024), (1, 5, 256, 512), (8, 300, 256, 512),
                                              (12, 200, 384, 768)])
def test_static_matches_existing_entry_point_twice(kind, m, rows, cols):
    rng = np.random.default_rng(kind * 100 + m)
    free = []
    for call in range(2):
        w = (rng.standard_normal((rows, cols), dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
        raw = synth.encode(kind, w)
        x = rng.standard_normal((m, cols), dtype=np.float32)
        bias = rng.standard_normal(rows, dtype=np.float32)
        got = _static_apply(kind, raw, rows, cols, x, bias, free)
        want = engine.matrix_apply(kind, raw, rows, cols, x, bias)
        tol = 2e-3 * np.sqrt(cols) * 0.02 * 4 + 1e-4
        assert np.abs(got - want).max() < tol, (call, np.abs(got - want).max())
        # and against the oracle's Matrix::apply on the F32-decoded weight
        ref = oracle.matrix_apply(oracle.decode(kind, raw).reshape(rows, cols), x, bias, threads=4)
        assert np.abs(got - ref).max() < tol, (call, np.abs(got - ref).max())
    # the second call (set-up done) leaves the device's free memory unchanged
    before, after = free[1]
    assert before == after, (before, after)


def test_static_rejects_sizes_beyond_the_limit():
    torch = pytest.importorskip("torch")
    rows, cols = 4096, 2048  # 16 MiB of F16 weight operand alone
    w_d = torch.zeros(rows * cols * 2, dtype=torch.uint8, device="cuda")
    x_d = torch.zeros((1, cols), dtype=torch.float32, device="cuda")
    out_d = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
    rc = _lib.lib().laya_matrix_apply_static(1, ctypes.c_void_p(w_d.data_ptr()), rows, cols,
                                             ctypes.c_void_p(x_d.data_ptr()), 1, None,
                                             ctypes.c_void_p(out_d.data_ptr()), None)
    assert rc == _lib.E_INVALID
    assert b"static scratch" in _lib.lib().laya_last_error()
