"""An independent float64 numpy forward pass of the reference model (cpu.go).

Test helper: it shares no code with the C oracle (its own GGUF reader, block
dequantisation and layer loop) and computes in float64, so agreement to about
1e-5 relative pins the structure of the oracle's restatement (block layouts,
nibble order, RoPE pairing, GQA head mapping, bias and residual placement) where
no golden vector exists. Follows cpu.go:225-366 and cpu.go:371-385.
"""

from __future__ import annotations

import struct

import numpy as np

_VT_SIZE = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
_VT_FMT = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


def read_gguf(path: str):
    data = np.memmap(path, np.uint8, mode="r")
    b = bytes(data[: min(len(data), 1 << 24)])
    pos = 8
    nt, nkv = struct.unpack_from("<QQ", b, pos)
    pos += 16

    def rstr():
        nonlocal pos
        (n,) = struct.unpack_from("<Q", b, pos)
        s = b[pos + 8: pos + 8 + n].decode()
        pos += 8 + n
        return s

    def rval(t):
        nonlocal pos
        if t == 8:
            return rstr()
        if t == 9:
            (et,) = struct.unpack_from("<I", b, pos)
            (n,) = struct.unpack_from("<Q", b, pos + 4)
            pos += 12
            return [rval(et) for _ in range(n)]
        (v,) = struct.unpack_from(_VT_FMT[t], b, pos)
        pos += _VT_SIZE[t]
        return v

    meta = {}
    for _ in range(nkv):
        k = rstr()
        (t,) = struct.unpack_from("<I", b, pos)
        pos += 4
        meta[k] = rval(t)
    tensors = {}
    for _ in range(nt):
        name = rstr()
        (nd,) = struct.unpack_from("<I", b, pos)
        dims = list(struct.unpack_from(f"<{nd}Q", b, pos + 4))
        ty, off = struct.unpack_from("<IQ", b, pos + 4 + 8 * nd)
        pos += 4 + 8 * nd + 12
        tensors[name] = (dims, ty, off)
    align = meta.get("general.alignment", 32)
    data_off = (pos + align - 1) // align * align
    return meta, tensors, data, data_off


def dequant(data, data_off, dims, ty) -> np.ndarray:
    """The [out, in] float64 matrix (or vector) of a GGUF tensor."""
    n = int(np.prod(dims))
    if ty == 0:
        return np.frombuffer(bytes(data[data_off: data_off + 4 * n]), "<f4").astype(np.float64).reshape(dims[::-1])
    bb = {2: 18, 3: 20, 8: 34}[ty]
    nblk = n // 32
    raw = np.asarray(data[data_off: data_off + nblk * bb]).reshape(nblk, bb)
    d = raw[:, 0:2].copy().view(np.float16).astype(np.float64)
    if ty == 2:
        qs = raw[:, 2:18]
        q = np.concatenate([(qs & 15).astype(np.float64) - 8, (qs >> 4).astype(np.float64) - 8], axis=1)
        v = d * q
    elif ty == 3:
        mn = raw[:, 2:4].copy().view(np.float16).astype(np.float64)
        qs = raw[:, 4:20]
        q = np.concatenate([(qs & 15).astype(np.float64), (qs >> 4).astype(np.float64)], axis=1)
        v = d * q + mn
    else:
        v = d * raw[:, 2:34].copy().view(np.int8).astype(np.float64)
    return v.reshape(dims[::-1])


class NumpyModel:
    def __init__(self, path: str, ctx: int):
        meta, ts, data, off = read_gguf(path)
        a = meta["general.architecture"]
        self.arch = a
        self.L = meta[f"{a}.block_count"]
        self.E = meta[f"{a}.embedding_length"]
        self.H = meta[f"{a}.attention.head_count"]
        self.KV = meta.get(f"{a}.attention.head_count_kv", self.H)
        self.HD = self.E // self.H
        self.base = float(np.float32(meta.get(f"{a}.rope.freq_base", 10000.0)))
        self.eps = float(np.float32(meta[f"{a}.attention.layer_norm_rms_epsilon"]))
        self.neox = a == "qwen2"
        self.w = {k: dequant(data, off + o, dims, ty) for k, (dims, ty, o) in ts.items()}
        self.out = self.w.get("output.weight", self.w["token_embd.weight"])
        self.kc = np.zeros((self.L, ctx, self.KV * self.HD))
        self.vc = np.zeros_like(self.kc)
        self.pos = 0

    def rope(self, x: np.ndarray, heads: int) -> np.ndarray:
        x = x.copy().reshape(heads, self.HD)
        i = np.arange(self.HD // 2)
        theta = self.pos * np.power(self.base, -(2.0 * i) / self.HD)
        c, s = np.cos(theta), np.sin(theta)
        if self.neox:
            a, b = x[:, : self.HD // 2].copy(), x[:, self.HD // 2:].copy()
            x[:, : self.HD // 2], x[:, self.HD // 2:] = a * c - b * s, a * s + b * c
        else:
            a, b = x[:, 0::2].copy(), x[:, 1::2].copy()
            x[:, 0::2], x[:, 1::2] = a * c - b * s, a * s + b * c
        return x.reshape(-1)

    def rms(self, x, w):
        return x / np.sqrt(np.mean(x * x) + self.eps) * w

    def forward(self, tok: int) -> np.ndarray:
        x = self.w["token_embd.weight"][tok].copy()
        grp = self.H // self.KV
        for l in range(self.L):
            p = f"blk.{l}."
            W = lambda n: self.w[p + n]
            h = self.rms(x, W("attn_norm.weight"))
            q, k, v = W("attn_q.weight") @ h, W("attn_k.weight") @ h, W("attn_v.weight") @ h
            if self.arch == "qwen2":
                q, k, v = q + W("attn_q.bias"), k + W("attn_k.bias"), v + W("attn_v.bias")
            q, k = self.rope(q, self.H), self.rope(k, self.KV)
            self.kc[l, self.pos], self.vc[l, self.pos] = k, v
            att = np.zeros(self.H * self.HD)
            for hd in range(self.H):
                g = hd // grp
                K = self.kc[l, : self.pos + 1, g * self.HD:(g + 1) * self.HD]
                V = self.vc[l, : self.pos + 1, g * self.HD:(g + 1) * self.HD]
                s = K @ q[hd * self.HD:(hd + 1) * self.HD] / np.sqrt(self.HD)
                e = np.exp(s - s.max())
                att[hd * self.HD:(hd + 1) * self.HD] = (e / e.sum()) @ V
            x = x + W("attn_output.weight") @ att
            h = self.rms(x, W("ffn_norm.weight"))
            g, u = W("ffn_gate.weight") @ h, W("ffn_up.weight") @ h
            x = x + W("ffn_down.weight") @ (g / (1 + np.exp(-g)) * u)
        self.pos += 1
        return self.out @ self.rms(x, self.w["output_norm.weight"])
