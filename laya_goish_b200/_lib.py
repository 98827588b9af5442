"""ctypes binding of liblaya_cuda.so (the C ABI declared in include/laya_cuda.h).

There is no fallback: if the in-tree library is missing, loading fails with an
error that says how to build it.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblaya_cuda.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "laya_cuda.h")

OK, E_INVALID, E_CANCELED, E_CUDA, E_TIMEOUT, E_NONFINITE, E_NOMEM, E_IO, E_FORMAT = 0, -1, -2, -3, -4, -5, -6, -7, -8
CODE_NAMES = {E_INVALID: "invalid", E_CANCELED: "canceled", E_CUDA: "cuda", E_TIMEOUT: "timeout",
              E_NONFINITE: "nonfinite", E_NOMEM: "nomem", E_IO: "io", E_FORMAT: "format"}
MAX_OPTIONS = 16
CHOICE, SCORE, NOUL = 0, 1, 2


class LayaError(RuntimeError):
    """A failed library call: .code is the LAYA_E_* status, the message is laya_last_error()."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{CODE_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class Question(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("n_options", ctypes.c_int32), ("option_len", ctypes.c_int32),
                ("options", ctypes.POINTER(ctypes.c_int32)), ("suffix_len", ctypes.c_int32),
                ("suffix", ctypes.POINTER(ctypes.c_int32))]


class Batch(ctypes.Structure):
    _fields_ = [("n_requests", ctypes.c_int32), ("ids", ctypes.POINTER(ctypes.c_int32)),
                ("offsets", ctypes.POINTER(ctypes.c_int64)), ("n_questions", ctypes.c_int32),
                ("questions", ctypes.POINTER(Question))]


class Answer(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("n_options", ctypes.c_int32), ("choice", ctypes.c_int32),
                ("score", ctypes.c_float), ("noul", ctypes.c_float), ("confidence", ctypes.c_float),
                ("probabilities", ctypes.c_float * MAX_OPTIONS), ("logits", ctypes.c_float * MAX_OPTIONS)]


class ModelInfo(ctypes.Structure):
    _fields_ = [("architecture", ctypes.c_char * 32), ("layers", ctypes.c_int32), ("d_model", ctypes.c_int32),
                ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("ffn", ctypes.c_int32), ("vocab", ctypes.c_int32), ("context", ctypes.c_int32),
                ("weight_kind", ctypes.c_int32), ("n_devices", ctypes.c_int32), ("device_bytes", ctypes.c_int64)]


class Timing(ctypes.Structure):
    _fields_ = [("device_ms", ctypes.c_double), ("launches", ctypes.c_int64), ("h2d_bytes", ctypes.c_int64),
                ("d2h_bytes", ctypes.c_int64)]


class OtConfig(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int32) for k in ("d", "ffn", "heads", "kv_heads", "head_dim", "rot", "lin_heads",
                                              "lin_dim", "vocab", "slots", "n_layers")] + \
               [("theta", ctypes.c_float), ("eps", ctypes.c_float), ("layer_full", ctypes.c_void_p)]


class ProfileEntry(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_int64), ("total_ms", ctypes.c_double)]


CANCEL_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)

_lib = None


def declared_symbols() -> list[str]:
    """Every function declared in include/laya_cuda.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(laya_\w+)\s*\(", text, re.M)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built: run `python -m laya_goish_b200.build` (needs nvcc)")
    L = ctypes.CDLL(LIB_PATH)
    P, I, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    L.laya_last_error.restype = ctypes.c_char_p
    L.laya_open.argtypes = [ctypes.c_char_p, P, I, ctypes.POINTER(P)]
    L.laya_open_memory.argtypes = [P, SZ, P, I, ctypes.POINTER(P)]
    L.laya_layers.argtypes = [P]
    L.laya_info.argtypes = [P, ctypes.POINTER(ModelInfo)]
    L.laya_validate.argtypes = [P, ctypes.POINTER(Batch)]
    L.laya_decide_batch.argtypes = [P, ctypes.POINTER(Batch), ctypes.POINTER(Answer), CANCEL_FN, P]
    L.laya_decode.argtypes = [P, P, P, I, I, P, P]
    L.laya_close.argtypes = [P]
    L.laya_close.restype = None
    L.laya_dequantize.argtypes = [I, ctypes.c_uint32, P, SZ, P]
    L.laya_matrix_apply.argtypes = [I, ctypes.c_uint32, P, I, I, P, I, P, P]
    L.laya_gated_delta.argtypes = [I, P, P, P, P, P, I, I, I, P]
    L.laya_gated_attention.argtypes = [I, P, P, P, P, P, I, I, I, I, I, ctypes.c_float, P]
    L.laya_gated_delta_mixer.argtypes = [I, P, P, P, P, P, P, P, P, I, I, I, P]
    L.laya_forward.argtypes = [P, P, I, P, I, P]
    L.laya_tensor_f32.argtypes = [P, ctypes.c_char_p, P, SZ]
    L.laya_matrix_apply_static.argtypes = [ctypes.c_uint32, P, I, I, P, I, P, P, P]
    L.laya_wait_selftest.argtypes = [I, ctypes.c_longlong]
    L.laya_last_timing.argtypes = [P, ctypes.POINTER(Timing)]
    L.laya_profile_enable.argtypes = [P, I]
    L.laya_profile_read.argtypes = [P, ctypes.POINTER(ProfileEntry), I]
    L.laya_openthai_open.argtypes = [ctypes.c_char_p, I, ctypes.POINTER(OtConfig), ctypes.POINTER(P)]
    L.laya_openthai_open_memory.argtypes = [P, SZ, I, ctypes.POINTER(OtConfig), ctypes.POINTER(P)]
    L.laya_openthai_forward.argtypes = [P, P, I, P, I, P]
    L.laya_openthai_forward_batch.argtypes = [P, P, P, I, P, I, P]
    L.laya_openthai_close.argtypes = [P]
    L.laya_openthai_close.restype = None
    _lib = L
    return L


def check(rc: int) -> int:
    if rc < 0:
        raise LayaError(rc, lib().laya_last_error().decode(errors="replace"))
    return rc
