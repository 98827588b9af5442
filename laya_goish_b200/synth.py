"""Seeded synthetic GGUF models and inputs for the decision hot path.

The reference ships no decoder weights for these shapes, so every model used
by the tests and the benchmark is written here from a seed: weights
N(0, 0.02) rounded to F16, norm weights 1.0, Qwen2 QKV biases N(0, 0.02),
then quantised to Q8_0 / Q4_K / Q6_K by round-to-nearest encoders.  Any valid
encoding will do: parity is always on decoding the same bytes.

The container layout follows the GGUF v3 rules that the reference reader
enforces (src/gguf.rs:95-180): little-endian header, metadata, tensor table,
32-byte aligned data.  Tensor and metadata names follow the llama.cpp
convention (``blk.N.attn_q.weight`` ..., ``llama.block_count`` ...).
A matrix with GGUF dims ``[K, N]`` is stored as N rows of K elements,
quantised along K (src/gguf.rs:141; src/models/openthai/model.rs:53-63).
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
import struct

import numpy as np

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
LAYOUT = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


# ---------------------------------------------------------------- encoders

def _f16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16)


def _div(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    with np.errstate(divide="ignore", invalid="ignore"):
        return np.where(b != 0, a / np.where(b != 0, b, 1), 0).astype(np.float32)


def quant_q8_0(x: np.ndarray) -> np.ndarray:
    """x: (..., K) float32, K % 32 == 0 → uint8 blocks of 34 bytes (d f16, 32 x int8)."""
    b = x.reshape(-1, 32).astype(np.float32)
    d16 = _f16(np.abs(b).max(axis=1) / 127.0)
    q = np.clip(np.rint(_div(b, d16.astype(np.float32)[:, None])), -127, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quant_q4_0(x: np.ndarray) -> np.ndarray:
    """x → 18-byte blocks: d f16, 16 bytes of nibbles (element j low, j+16 high)."""
    b = x.reshape(-1, 32).astype(np.float32)
    idx = np.abs(b).argmax(axis=1)
    mx = b[np.arange(b.shape[0]), idx]
    d16 = _f16(mx / -8.0)
    q = np.clip(np.rint(_div(b, d16.astype(np.float32)[:, None])) + 8, 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], 18), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def quant_q4_k(x: np.ndarray) -> np.ndarray:
    """x → 144-byte superblocks: d, dmin (f16), 12 bytes of packed 6-bit
    scales/mins, 128 bytes of nibbles.  Inverse of src/gguf.rs:281-307."""
    b = x.reshape(-1, 8, 32).astype(np.float32)
    nb = b.shape[0]
    mn = np.minimum(b.min(axis=2), 0.0)
    mx = b.max(axis=2)
    scale = (mx - mn) / 15.0
    mins = -mn
    d16 = _f16(scale.max(axis=1) / 63.0)
    dm16 = _f16(mins.max(axis=1) / 63.0)
    df = d16.astype(np.float32)[:, None]
    dmf = dm16.astype(np.float32)[:, None]
    sc = np.clip(np.rint(_div(scale, df)), 0, 63).astype(np.uint8)
    m = np.clip(np.rint(_div(mins, dmf)), 0, 63).astype(np.uint8)
    eff_s = (df * sc).astype(np.float32)[:, :, None]
    eff_m = (dmf * m).astype(np.float32)[:, :, None]
    q = np.clip(np.rint(_div(b + eff_m, np.broadcast_to(eff_s, b.shape))), 0, 15).astype(np.uint8)
    packed = np.zeros((nb, 12), np.uint8)
    for j in range(4):
        packed[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        packed[:, j + 4] = (m[:, j] & 63) | ((m[:, j + 4] >> 4) << 6)
        packed[:, j + 8] = (sc[:, j + 4] & 15) | ((m[:, j + 4] & 15) << 4)
    qs = np.empty((nb, 4, 32), np.uint8)
    for g in range(4):
        qs[:, g] = q[:, 2 * g] | (q[:, 2 * g + 1] << 4)
    out = np.empty((nb, 144), np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(-1, 2)
    out[:, 4:16] = packed
    out[:, 16:] = qs.reshape(nb, 128)
    return out.reshape(-1)


def quant_q6_k(x: np.ndarray) -> np.ndarray:
    """x → 210-byte superblocks: ql[128], qh[64], int8 scales[16], d f16.
    Inverse of src/gguf.rs:308-332."""
    b = x.reshape(-1, 16, 16).astype(np.float32)
    nb = b.shape[0]
    amax = np.abs(b).max(axis=2)
    scale = amax / 31.0
    d16 = _f16(scale.max(axis=1) / 127.0)
    df = d16.astype(np.float32)[:, None]
    sc = np.clip(np.rint(_div(scale, df)), -128, 127).astype(np.int8)
    eff = (df * sc.astype(np.float32))[:, :, None]
    q = (np.clip(np.rint(_div(b, np.broadcast_to(eff, b.shape))), -32, 31) + 32).astype(np.uint8)
    q = q.reshape(nb, 2, 4, 32)  # element n*128 + j*32 + l
    ql = np.empty((nb, 2, 2, 32), np.uint8)
    ql[:, :, 0] = (q[:, :, 0] & 15) | ((q[:, :, 2] & 15) << 4)
    ql[:, :, 1] = (q[:, :, 1] & 15) | ((q[:, :, 3] & 15) << 4)
    qh = ((q[:, :, 0] >> 4) | ((q[:, :, 1] >> 4) << 2) | ((q[:, :, 2] >> 4) << 4) | ((q[:, :, 3] >> 4) << 6)).astype(np.uint8)
    out = np.empty((nb, 210), np.uint8)
    out[:, :128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d16.view(np.uint8).reshape(-1, 2)
    return out.reshape(-1)


def encode(kind: int, x: np.ndarray) -> np.ndarray:
    """Encode a float array (rows of K contiguous elements) as GGUF tensor bytes."""
    if kind == F32:
        return np.ascontiguousarray(x, np.float32).view(np.uint8).reshape(-1)
    if kind == F16:
        return np.ascontiguousarray(x, np.float16).view(np.uint8).reshape(-1)
    return {Q8_0: quant_q8_0, Q4_0: quant_q4_0, Q4_K: quant_q4_k, Q6_K: quant_q6_k}[kind](x)


def nbytes(kind: int, count: int) -> int:
    block, size = LAYOUT[kind]
    return count // block * size


# ---------------------------------------------------------------- GGUF writer

def _gstr(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, value) -> bytes:
    if isinstance(value, str):
        return _gstr(key) + struct.pack("<I", 8) + _gstr(value)
    if isinstance(value, float):
        return _gstr(key) + struct.pack("<If", 6, value)
    if isinstance(value, bool):
        return _gstr(key) + struct.pack("<IB", 7, int(value))
    return _gstr(key) + struct.pack("<II", 4, int(value))


def write_gguf(path: str, meta: dict, tensors: list, align: int = 32) -> None:
    """tensors: list of (name, dims, kind, producer) where producer() returns the bytes."""
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta) + 1)
    head += b"".join(_kv(k, v) for k, v in meta.items()) + _kv("general.alignment", align)
    offs, off = [], 0
    for name, dims, kind, _ in tensors:
        count = int(np.prod(dims))
        offs.append(off)
        off += nbytes(kind, count)
        off = (off + align - 1) // align * align
    for (name, dims, kind, _), o in zip(tensors, offs):
        head += _gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", kind, o)
    pad = (-len(head)) % align
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(head + b"\0" * pad)
        pos = 0
        for (name, dims, kind, produce), o in zip(tensors, offs):
            if o > pos:
                f.write(b"\0" * (o - pos))
                pos = o
            data = produce()
            assert data.nbytes == nbytes(kind, int(np.prod(dims))), name
            f.write(memoryview(np.ascontiguousarray(data)))
            pos += data.nbytes
    os.replace(tmp, path)


# ---------------------------------------------------------------- decoder configs

@dataclasses.dataclass(frozen=True)
class Decoder:
    name: str
    arch: str          # "llama" or "qwen2"
    layers: int
    d: int
    heads: int
    kv: int
    ffn: int
    vocab: int
    theta: float
    eps: float = 1e-5
    bias: bool = False
    quant: str = "f16"  # f16 | q8_0 | q4_k_m | q4_0
    seed: int = 0
    ctx: int = 8192

    @property
    def hd(self) -> int:
        return self.d // self.heads

    def kind_of(self, role: str) -> int:
        """Tensor type per role.  Q4_K_M keeps attn_v, ffn_down and output at Q6_K."""
        if role == "norm" or role == "bias":
            return F32
        if self.quant == "f16":
            return F16
        if self.quant == "q8_0":
            return Q8_0
        if self.quant == "q4_0":
            return Q4_0
        if self.quant == "q4_k_m":
            return Q6_K if role in ("attn_v", "ffn_down", "output") else Q4_K
        raise ValueError(self.quant)

    def matrix_params(self) -> int:
        qd, kd = self.heads * self.hd, self.kv * self.hd
        per = self.d * (qd + 2 * kd) + qd * self.d + 3 * self.d * self.ffn
        return per * self.layers


LLAMA = dict(arch="llama", layers=16, d=2048, heads=32, kv=8, ffn=8192, vocab=32000, theta=1e4)
QWEN2 = dict(arch="qwen2", layers=28, d=3584, heads=28, kv=4, ffn=18944, vocab=152064, theta=1e6, bias=True)

CONFIGS = {
    "cfg0": Decoder("cfg0-llama16-f16", quant="f16", seed=0, **LLAMA),
    "cfg1": Decoder("cfg1-llama16-q8_0", quant="q8_0", seed=1, **LLAMA),
    "cfg2": Decoder("cfg2-llama16-q4_k_m", quant="q4_k_m", seed=2, **LLAMA),
    "cfg3": Decoder("cfg3-qwen2-28-f16", quant="f16", seed=3, **QWEN2),
    "cfg4": Decoder("cfg1-llama16-q8_0", quant="q8_0", seed=1, **LLAMA),
}

# Small decoders for the parity tests (the oracle finishes them in seconds).
TINY = {
    "tiny-llama-f16": Decoder("tiny-llama-f16", "llama", 2, 256, 4, 2, 512, 1000, 1e4, quant="f16", seed=11),
    "tiny-llama-q8_0": Decoder("tiny-llama-q8_0", "llama", 2, 256, 4, 2, 512, 1000, 1e4, quant="q8_0", seed=12),
    "tiny-llama-q4_k_m": Decoder("tiny-llama-q4_k_m", "llama", 2, 256, 4, 2, 512, 1000, 1e4, quant="q4_k_m", seed=13),
    "tiny-llama-q4_0": Decoder("tiny-llama-q4_0", "llama", 2, 256, 4, 2, 512, 1000, 1e4, quant="q4_0", seed=14),
    "tiny-qwen2-f16": Decoder("tiny-qwen2-f16", "qwen2", 2, 256, 2, 1, 768, 1000, 1e6, quant="f16", bias=True, seed=15),
    "small-llama-q8_0": Decoder("small-llama-q8_0", "llama", 4, 512, 8, 2, 1536, 4000, 1e4, quant="q8_0", seed=16),
}


def tensor_plan(cfg: Decoder) -> list:
    """(name, dims, kind, role, std) in file order; matrices [K, N] = N rows of K."""
    qd, kd = cfg.heads * cfg.hd, cfg.kv * cfg.hd
    plan = [("token_embd.weight", [cfg.d, cfg.vocab], cfg.kind_of("token_embd"), "w")]
    for i in range(cfg.layers):
        p = f"blk.{i}."
        plan += [
            (p + "attn_norm.weight", [cfg.d], F32, "norm"),
            (p + "attn_q.weight", [cfg.d, qd], cfg.kind_of("attn_q"), "w"),
            (p + "attn_k.weight", [cfg.d, kd], cfg.kind_of("attn_k"), "w"),
            (p + "attn_v.weight", [cfg.d, kd], cfg.kind_of("attn_v"), "w"),
        ]
        if cfg.bias:
            plan += [(p + "attn_q.bias", [qd], F32, "bias"), (p + "attn_k.bias", [kd], F32, "bias"),
                     (p + "attn_v.bias", [kd], F32, "bias")]
        plan += [
            (p + "attn_output.weight", [qd, cfg.d], cfg.kind_of("attn_output"), "w"),
            (p + "ffn_norm.weight", [cfg.d], F32, "norm"),
            (p + "ffn_gate.weight", [cfg.d, cfg.ffn], cfg.kind_of("ffn_gate"), "w"),
            (p + "ffn_up.weight", [cfg.d, cfg.ffn], cfg.kind_of("ffn_up"), "w"),
            (p + "ffn_down.weight", [cfg.ffn, cfg.d], cfg.kind_of("ffn_down"), "w"),
        ]
    plan += [("output_norm.weight", [cfg.d], F32, "norm"),
             ("output.weight", [cfg.d, cfg.vocab], cfg.kind_of("output"), "w")]
    return plan


def _meta(cfg: Decoder) -> dict:
    a = cfg.arch
    return {
        "general.architecture": a,
        "general.name": cfg.name,
        f"{a}.context_length": cfg.ctx,
        f"{a}.embedding_length": cfg.d,
        f"{a}.block_count": cfg.layers,
        f"{a}.feed_forward_length": cfg.ffn,
        f"{a}.attention.head_count": cfg.heads,
        f"{a}.attention.head_count_kv": cfg.kv,
        f"{a}.attention.layer_norm_rms_epsilon": float(cfg.eps),
        f"{a}.rope.freq_base": float(cfg.theta),
        f"{a}.vocab_size": cfg.vocab,
    }


def write_model(cfg: Decoder, path: str) -> str:
    rng = np.random.default_rng(cfg.seed)
    tensors = []
    for name, dims, kind, role in tensor_plan(cfg):
        count = int(np.prod(dims))

        def produce(role=role, kind=kind, count=count, dims=dims):
            if role == "norm":
                return np.ones(count, np.float32).view(np.uint8)
            x = (rng.standard_normal(count, dtype=np.float32) * np.float32(0.02)).astype(np.float16)
            if role == "bias":
                return x.astype(np.float32).view(np.uint8)
            return encode(kind, x.astype(np.float32).reshape(-1, dims[0]) if kind != F16 else x)

        tensors.append((name, dims, kind, produce))
    write_gguf(path, _meta(cfg), tensors)
    return path


def cache_dir() -> str:
    d = os.environ.get("LAYA_SYNTH_DIR") or os.path.join("/tmp", "laya_synth")
    os.makedirs(d, exist_ok=True)
    return d


def model_path(cfg: Decoder | str) -> str:
    """Path of the seeded GGUF for cfg, writing it on first use."""
    if isinstance(cfg, str):
        cfg = CONFIGS.get(cfg) or TINY[cfg]
    tag = hashlib.sha1(json.dumps(dataclasses.asdict(cfg), sort_keys=True).encode()).hexdigest()[:10]
    path = os.path.join(cache_dir(), f"{cfg.name}-{tag}.gguf")
    if not os.path.exists(path):
        write_model(cfg, path)
    return path


# ---------------------------------------------------------------- inputs

def token_ids(rng: np.random.Generator, vocab: int, n: int) -> np.ndarray:
    """Token ids uniform in [3, vocab)."""
    return rng.integers(3, vocab, size=n, dtype=np.int32)


def candidates(rng: np.random.Generator, vocab: int, k: int) -> np.ndarray:
    """k distinct candidate ids uniform in [3, vocab)."""
    return (rng.choice(vocab - 3, size=k, replace=False) + 3).astype(np.int32)
