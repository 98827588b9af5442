"""Independent float64 PyTorch restatement of the decoder forward, used only
to cross-check the C oracle on tiny shapes.  Weights are read with gguf-py's
GGUFReader and decoded with gguf-py, so no code is shared with the oracle."""
import numpy as np
import torch
from gguf import GGUFReader
from gguf import quants


def load(path):
    r = GGUFReader(path)
    meta = {}
    for f in r.fields.values():
        if f.types and f.types[0].name == "STRING":
            meta[f.name] = bytes(f.parts[f.data[0]]).decode()
        elif f.data:
            meta[f.name] = f.parts[f.data[0]][0].item()
    w = {}
    for t in r.tensors:
        raw = np.array(t.data)
        if t.tensor_type.name in ("F32", "F16"):
            v = raw.astype(np.float32).reshape(-1)
        else:
            v = quants.dequantize(raw.reshape(-1).view(np.uint8), t.tensor_type).reshape(-1)
        dims = [int(d) for d in t.shape]
        w[t.name] = torch.tensor(v, dtype=torch.float64).reshape(list(reversed(dims)) if len(dims) > 1 else dims)
    return meta, w


def forward(path, ids, read):
    meta, w = load(path)
    a = meta["general.architecture"]
    L = meta[f"{a}.block_count"]
    H = meta[f"{a}.attention.head_count"]
    KV = meta[f"{a}.attention.head_count_kv"]
    eps = meta[f"{a}.attention.layer_norm_rms_epsilon"]
    theta = meta[f"{a}.rope.freq_base"]
    x = w["token_embd.weight"][torch.tensor(ids, dtype=torch.long)]
    s, d = x.shape
    hd = d // H

    def rms(v, g):
        return v / torch.sqrt((v * v).mean(-1, keepdim=True) + eps) * g

    pos = torch.arange(s, dtype=torch.float64)
    inv = theta ** (-(torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    ang = pos[:, None] * inv[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)

    def rope(t):  # t: s, heads, hd — rotate-half pairs (j, j + hd/2)
        a_, b_ = t[..., : hd // 2], t[..., hd // 2:]
        c, sn = cos[:, None, :], sin[:, None, :]
        return torch.cat([a_ * c - b_ * sn, b_ * c + a_ * sn], -1)

    mask = torch.full((s, s), float("-inf"), dtype=torch.float64).triu(1)
    for i in range(L):
        p = f"blk.{i}."
        h = rms(x, w[p + "attn_norm.weight"])
        q = h @ w[p + "attn_q.weight"].T
        k = h @ w[p + "attn_k.weight"].T
        v = h @ w[p + "attn_v.weight"].T
        if p + "attn_q.bias" in w:
            q, k, v = q + w[p + "attn_q.bias"], k + w[p + "attn_k.bias"], v + w[p + "attn_v.bias"]
        q = rope(q.reshape(s, H, hd))
        k = rope(k.reshape(s, KV, hd)).repeat_interleave(H // KV, dim=1)
        v = v.reshape(s, KV, hd).repeat_interleave(H // KV, dim=1)
        sc = torch.einsum("ihd,jhd->hij", q, k) / np.sqrt(hd) + mask
        o = torch.einsum("hij,jhd->ihd", torch.softmax(sc, -1), v).reshape(s, H * hd)
        x = x + o @ w[p + "attn_output.weight"].T
        h = rms(x, w[p + "ffn_norm.weight"])
        g = h @ w[p + "ffn_gate.weight"].T
        u = h @ w[p + "ffn_up.weight"].T
        x = x + (torch.nn.functional.silu(g) * u) @ w[p + "ffn_down.weight"].T
    hid = rms(x[torch.tensor(read, dtype=torch.long)], w["output_norm.weight"])
    return hid, w["output.weight"]
