"""Generates the committed golden dequantisation vectors (dequant.npz).

Each kind gets raw GGUF block bytes — both encoder output and random bytes
with finite scales, so every bit pattern of the packed scales and quants is
exercised — and the float32 values produced by gguf-py's independent
decoder (gguf 0.19.0, ``gguf.quants.dequantize``), which follows the ggml
block formats that the reference decoder restates (src/gguf.rs:250-336).
F16 vectors cover zeros, subnormals, normals, infinities and the largest
finite values (src/gguf.rs:226-246).

Run: python tests/golden/make_golden.py   (needs gguf-py; the GPU box does not)
"""
import os
import sys

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", ".."))
from laya_goish_b200 import synth  # noqa: E402

rng = np.random.default_rng(20261201)


def finite_f16(n):
    v = rng.integers(0, 0x7C00, size=n, dtype=np.uint16)  # exponent < 31: finite
    v |= (rng.integers(0, 2, size=n, dtype=np.uint16) << 15)
    return v


def random_blocks(kind, nblocks):
    block, size = synth.LAYOUT[kind]
    raw = rng.integers(0, 256, size=(nblocks, size), dtype=np.uint8)
    scale_at = {synth.Q8_0: [0], synth.Q4_0: [0], synth.Q4_K: [0, 2], synth.Q6_K: [208]}[kind]
    for off in scale_at:
        raw[:, off:off + 2] = finite_f16(nblocks).view(np.uint8).reshape(-1, 2)
    return raw.reshape(-1)


out = {}
x = (rng.standard_normal(256 * 8, dtype=np.float32) * 0.02).astype(np.float16).astype(np.float32)
for kind, t in [(synth.Q8_0, T.Q8_0), (synth.Q4_0, T.Q4_0), (synth.Q4_K, T.Q4_K), (synth.Q6_K, T.Q6_K)]:
    raw = np.concatenate([synth.encode(kind, x), random_blocks(kind, 8)])
    out[f"raw_{kind}"] = raw
    out[f"want_{kind}"] = quants.dequantize(raw, t).astype(np.float32).reshape(-1)
f16 = np.concatenate([
    np.array([0x0000, 0x8000, 0x0001, 0x8001, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF, 0x7C00, 0xFC00], np.uint16),
    finite_f16(500)])
out[f"raw_{synth.F16}"] = f16.view(np.uint8)
out[f"want_{synth.F16}"] = f16.view(np.float16).astype(np.float32)
f32 = rng.standard_normal(64, dtype=np.float32)
out[f"raw_{synth.F32}"] = f32.view(np.uint8)
out[f"want_{synth.F32}"] = f32
np.savez_compressed(os.path.join(os.path.dirname(__file__), "dequant.npz"), **out)
print({k: v.shape for k, v in out.items()})
