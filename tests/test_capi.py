"""CPU checks of the C-ABI library: it is built for sm_100a, loads, and
exports every entry point that include/laya_cuda.h declares."""
import ctypes
import subprocess

import pytest

from laya_goish_b200 import _lib


def test_header_declares_the_boundary():
    syms = _lib.declared_symbols()
    for name in ["laya_open", "laya_open_memory", "laya_layers", "laya_validate", "laya_decide_batch",
                 "laya_decode", "laya_close", "laya_last_error", "laya_dequantize", "laya_matrix_apply"]:
        assert name in syms


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in _lib.declared_symbols():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(_lib.declared_symbols()) <= exported


def test_open_without_gpu_fails_cleanly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = _lib.lib()
    h = ctypes.c_void_p()
    rc = L.laya_open(b"/nonexistent.gguf", None, 0, ctypes.byref(h))
    assert rc < 0 and not h.value
    assert L.laya_last_error()


def test_null_arguments_rejected():
    L = _lib.lib()
    assert L.laya_layers(None) == _lib.E_INVALID
    assert L.laya_decide_batch(None, None, None, _lib.CANCEL_FN(), None) == _lib.E_INVALID
    assert b"null" in L.laya_last_error()


def test_openthai_entry_points_reject_bad_arguments():
    L = _lib.lib()
    h = ctypes.c_void_p()
    full = (ctypes.c_uint8 * 2)(1, 0)
    cfg = _lib.OtConfig(128, 256, 4, 2, 96, 24, 2, 64, 300, 256, 2, 1e7, 1e-6,
                        ctypes.cast(full, ctypes.c_void_p))
    assert L.laya_openthai_open(b"/nonexistent.gguf", 0, ctypes.byref(cfg), ctypes.byref(h)) == _lib.E_INVALID
    assert b"unsupported OpenThai shape" in L.laya_last_error() and not h.value
    assert L.laya_openthai_open(b"x", 0, None, ctypes.byref(h)) == _lib.E_INVALID
    img = b"GGUF" + bytes(60)
    assert L.laya_openthai_open_memory(img, len(img), 0, ctypes.byref(cfg), ctypes.byref(h)) == _lib.E_INVALID
    cfg.head_dim = 64
    assert L.laya_openthai_open_memory(img, 8, 0, ctypes.byref(cfg), ctypes.byref(h)) == _lib.E_FORMAT
    assert L.laya_openthai_open_memory(None, 0, 0, ctypes.byref(cfg), ctypes.byref(h)) == _lib.E_INVALID
    assert L.laya_openthai_forward(None, None, 0, None, 0, None) == _lib.E_INVALID
    assert L.laya_openthai_forward_batch(None, None, None, 0, None, 0, None) == _lib.E_INVALID
    L.laya_openthai_close(None)
