"""Seeded synthetic GGUF v3 model files for the benchmark configurations.

The reference is measured on real instruct weights that are not available here,
so every configuration is a GGUF v3 file written from a fixed seed with the
shapes, tensor types and value distributions the benchmark specification
names. The CPU oracle and the GPU backend read the identical bytes.

Layout follows what the reference reads: metadata keys of ``ConfigFrom``
(config.go:29-73), tensor names of ``Forward`` (cpu.go:231-363) and
``fusedLayer`` (fused.go:199-217), dims ``[in, out]`` with ne[0] contiguous
(gguf/gguf.go:98, cpu.go:144), data aligned to 32 bytes (gguf/gguf.go:335).
Block formats (cpu.go:164-215): Q4_0 = f16 d + 16 bytes (byte j: low nibble is
element j, high nibble element j+16), Q4_1 = f16 d + f16 min + 16 bytes,
Q8_0 = f16 d + 32 int8.
"""

from __future__ import annotations

import os
import struct
import tempfile
from dataclasses import dataclass, field

import numpy as np

GGUF_MAGIC = b"GGUF"
T_F32, T_Q4_0, T_Q4_1, T_Q8_0 = 0, 2, 3, 8
VT_U32, VT_F32, VT_STRING = 4, 6, 8
ALIGN = 32


@dataclass(frozen=True)
class Spec:
    """A synthetic model: architecture, shape and the ggml type of each matrix."""

    name: str
    seed: int
    arch: str  # "llama" (NORM rope) or "qwen2" (NEOX rope, QKV biases)
    embd: int
    layers: int
    heads: int
    kv_heads: int
    ff: int
    vocab: int
    rope_base: float
    eps: float
    ctx: int = 2048  # <arch>.context_length; runs pass their own ctx <= this
    emb_type: int = T_Q4_0
    out_type: int | None = None  # None: tied output (token_embd is the head)
    types: dict = field(default_factory=dict)  # per matrix kind, default Q4_0
    # Rows of the output matrix written as copies of others, so that logits tie
    # exactly at every step: "far" copies row i to row i + vocab/2 (tiles far
    # apart, so different CTAs of the head), "near" copies row 2i to 2i + 1
    # (the same 8-row tile).  The argmax must return the lower index
    # (kernels.go:351-353, cpu.go:389-397).
    tie: str = ""

    def mtype(self, kind: str) -> int:
        return self.types.get(kind, T_Q4_0)

    @property
    def head_dim(self) -> int:
        return self.embd // self.heads


# BASELINE configurations. C4 runs on C3's file, C5 on C1's.
C1 = Spec("c1-smollm2-q4_0", 1, "llama", 576, 30, 9, 3, 1536, 49152, 1e5, 1e-5)
C2 = Spec("c2-smollm2-mixed", 2, "llama", 576, 30, 9, 3, 1536, 49152, 1e5, 1e-5,
          out_type=T_Q8_0, types={"attn_v": T_Q4_1, "ffn_down": T_Q4_1})
C3 = Spec("c3-qwen2.5-0.5b", 3, "qwen2", 896, 24, 14, 2, 4864, 151936, 1e6, 1e-6,
          out_type=T_Q8_0)
# Small models of the same families, for tests that run the oracle over many tokens.
TINY_LLAMA = Spec("tiny-llama", 11, "llama", 256, 3, 4, 2, 512, 1024, 1e4, 1e-5)
TINY_MIXED = Spec("tiny-mixed", 12, "llama", 256, 3, 4, 1, 512, 1024, 1e4, 1e-5,
                  emb_type=T_Q8_0, out_type=T_Q8_0, types={"attn_v": T_Q4_1, "ffn_down": T_Q4_1})
TINY_QWEN = Spec("tiny-qwen2", 13, "qwen2", 384, 3, 6, 2, 768, 1536, 1e6, 1e-6, out_type=T_Q8_0)
# head_dim 128 (the other supported head size)
TINY_HD128 = Spec("tiny-hd128", 14, "llama", 512, 2, 4, 2, 1024, 1024, 1e4, 1e-5)

# Every logit has an exact twin (untied Q4_0 / Q8_0 output): the greedy tie rule on the GPU.
TINY_TIE_FAR = Spec("tiny-tie-far", 15, "llama", 256, 3, 4, 2, 512, 1024, 1e4, 1e-5, out_type=T_Q4_0, tie="far")
TINY_TIE_NEAR = Spec("tiny-tie-near", 16, "llama", 256, 3, 4, 2, 512, 1024, 1e4, 1e-5, out_type=T_Q8_0, tie="near")

SPECS = {s.name: s for s in (C1, C2, C3, TINY_LLAMA, TINY_MIXED, TINY_QWEN, TINY_HD128, TINY_TIE_FAR,
                              TINY_TIE_NEAR)}

# The five BASELINE.json configurations: which file, prompt length, greedy tokens, context.
WORKLOADS = {
    1: dict(spec=C1, prompt=128, gen=128, ctx=512),
    2: dict(spec=C2, prompt=32, gen=256, ctx=512),
    3: dict(spec=C3, prompt=128, gen=128, ctx=512),
    4: dict(spec=C3, prompt=512, gen=16, ctx=528),
    5: dict(spec=C1, streams=64, prompt_range=(16, 512), gen=128, ctx=640),
}


def prompt_ids(vocab: int, n: int, seed: int) -> np.ndarray:
    """Uniform-random token ids (the benchmark prompts), seeded."""
    return np.random.default_rng(1000 + seed).integers(0, vocab, n, dtype=np.int64).astype(np.int32)


def workload_prompts(k: int, rank: int = 0) -> list[np.ndarray]:
    """The prompts of BASELINE workload k as the benchmark runs them.

    Workloads 1-4: one prompt of the workload's length, ids uniform over the
    vocab, seeded by the model's seed. Workload 5: the streams of one GPU
    (rank), lengths uniform on the prompt range and ids uniform, seeded per
    rank and per stream."""
    w = WORKLOADS[k]
    s = w["spec"]
    if k != 5:
        return [prompt_ids(s.vocab, w["prompt"], seed=s.seed)]
    rng = np.random.default_rng(5000 + rank)
    lo, hi = w["prompt_range"]
    lens = rng.integers(lo, hi + 1, w["streams"])
    return [prompt_ids(s.vocab, int(n), seed=10000 * (rank + 1) + i) for i, n in enumerate(lens)]


def _blocks(rng: np.random.Generator, ty: int, rows: int, cols: int) -> np.ndarray:
    """Raw GGUF blocks of a [cols, rows] matrix (rows of cols elements)."""
    nblk = rows * (cols // 32)
    if ty == T_Q4_0:
        out = np.empty((nblk, 18), np.uint8)
        out[:, 0:2] = rng.uniform(0.002, 0.02, nblk).astype(np.float16).view(np.uint8).reshape(nblk, 2)
        out[:, 2:] = rng.integers(0, 256, (nblk, 16), dtype=np.uint8)
    elif ty == T_Q4_1:
        out = np.empty((nblk, 20), np.uint8)
        out[:, 0:2] = rng.uniform(0.002, 0.02, nblk).astype(np.float16).view(np.uint8).reshape(nblk, 2)
        out[:, 2:4] = rng.uniform(-0.1, 0.0, nblk).astype(np.float16).view(np.uint8).reshape(nblk, 2)
        out[:, 4:] = rng.integers(0, 256, (nblk, 16), dtype=np.uint8)
    elif ty == T_Q8_0:
        out = np.empty((nblk, 34), np.uint8)
        out[:, 0:2] = rng.uniform(1e-4, 1e-3, nblk).astype(np.float16).view(np.uint8).reshape(nblk, 2)
        out[:, 2:] = rng.integers(-127, 128, (nblk, 32), dtype=np.int8).view(np.uint8)
    else:
        raise ValueError(f"no synthetic blocks for ggml type {ty}")
    return out


def _tensors(s: Spec):
    """(name, dims, type, generator) in file order."""
    kvd = s.kv_heads * s.head_dim
    ts = [("token_embd.weight", (s.embd, s.vocab), s.emb_type),
          ("output_norm.weight", (s.embd,), T_F32)]
    if s.out_type is not None:
        ts.append(("output.weight", (s.embd, s.vocab), s.out_type))
    for l in range(s.layers):
        p = f"blk.{l}."
        ts += [(p + "attn_norm.weight", (s.embd,), T_F32),
               (p + "attn_q.weight", (s.embd, s.embd), s.mtype("attn_q")),
               (p + "attn_k.weight", (s.embd, kvd), s.mtype("attn_k")),
               (p + "attn_v.weight", (s.embd, kvd), s.mtype("attn_v"))]
        if s.arch == "qwen2":
            ts += [(p + "attn_q.bias", (s.embd,), T_F32), (p + "attn_k.bias", (kvd,), T_F32),
                   (p + "attn_v.bias", (kvd,), T_F32)]
        ts += [(p + "attn_output.weight", (s.embd, s.embd), s.mtype("attn_output")),
               (p + "ffn_norm.weight", (s.embd,), T_F32),
               (p + "ffn_gate.weight", (s.embd, s.ff), s.mtype("ffn_gate")),
               (p + "ffn_up.weight", (s.embd, s.ff), s.mtype("ffn_up")),
               (p + "ffn_down.weight", (s.ff, s.embd), s.mtype("ffn_down"))]
    return ts


def _nbytes(dims, ty) -> int:
    n = int(np.prod(dims))
    return {T_F32: 4 * n, T_Q4_0: n // 32 * 18, T_Q4_1: n // 32 * 20, T_Q8_0: n // 32 * 34}[ty]


def _str(b: bytearray, s: str) -> None:
    e = s.encode()
    b += struct.pack("<Q", len(e)) + e


def header(s: Spec) -> tuple[bytes, list]:
    """The GGUF header and the (name, dims, type, offset, size) of each tensor."""
    a = s.arch
    kv = [("general.architecture", VT_STRING, a), ("general.name", VT_STRING, f"synthetic {s.name} seed {s.seed}"),
          (f"{a}.block_count", VT_U32, s.layers), (f"{a}.context_length", VT_U32, s.ctx),
          (f"{a}.embedding_length", VT_U32, s.embd), (f"{a}.feed_forward_length", VT_U32, s.ff),
          (f"{a}.attention.head_count", VT_U32, s.heads), (f"{a}.attention.head_count_kv", VT_U32, s.kv_heads),
          (f"{a}.rope.dimension_count", VT_U32, s.head_dim), (f"{a}.rope.freq_base", VT_F32, s.rope_base),
          (f"{a}.attention.layer_norm_rms_epsilon", VT_F32, s.eps)]
    ts = _tensors(s)
    b = bytearray(GGUF_MAGIC + struct.pack("<IQQ", 3, len(ts), len(kv)))
    for k, vt, v in kv:
        _str(b, k)
        b += struct.pack("<I", vt)
        if vt == VT_STRING:
            _str(b, v)
        elif vt == VT_U32:
            b += struct.pack("<I", v)
        else:
            b += struct.pack("<f", v)
    infos, off = [], 0
    for name, dims, ty in ts:
        size = _nbytes(dims, ty)
        _str(b, name)
        b += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        b += struct.pack("<IQ", ty, off)
        infos.append((name, dims, ty, off, size))
        off = (off + size + ALIGN - 1) // ALIGN * ALIGN
    b += b"\0" * ((-len(b)) % ALIGN)
    return bytes(b), infos


def write(s: Spec, path: str) -> None:
    """Writes the model file of s to path (atomically: a temporary file, then a rename)."""
    rng = np.random.default_rng(s.seed)
    hdr, infos = header(s)
    d = os.path.dirname(os.path.abspath(path))
    os.makedirs(d, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=d, suffix=".part")
    try:
        with os.fdopen(fd, "wb") as f:
            f.write(hdr)
            for name, dims, ty, off, size in infos:
                f.seek(len(hdr) + off)
                if ty == T_F32:
                    if name.endswith("norm.weight"):
                        v = 1.0 + rng.normal(0.0, 0.05, dims[0])
                    else:  # qwen2 QKV biases
                        v = rng.normal(0.0, 0.02, dims[0])
                    f.write(v.astype("<f4").tobytes())
                else:
                    blk = _blocks(rng, ty, dims[1], dims[0])
                    if name == "output.weight" and s.tie:
                        rows = blk.reshape(dims[1], -1)
                        if s.tie == "far":
                            rows[dims[1] // 2:] = rows[: dims[1] // 2]
                        else:
                            rows[1::2] = rows[0::2]
                    assert blk.size == size
                    f.write(blk.tobytes())
            end = len(hdr) + infos[-1][3] + infos[-1][4]
            f.truncate(end)
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise


def model_dir() -> str:
    return os.environ.get("LLMB_MODEL_DIR", os.path.join(tempfile.gettempdir(), "llmb_models"))


def ensure(s: Spec | str) -> str:
    """Path of the model file of s, written once into the model directory."""
    if isinstance(s, str):
        s = SPECS[s]
    path = os.path.join(model_dir(), f"{s.name}-seed{s.seed}.gguf")
    if not os.path.exists(path):
        write(s, path)
    return path


def algorithmic_bytes_per_token(s: Spec) -> int:
    """GGUF bytes every decoded token reads once: all layer matrices, the head,
    and the norm/bias vectors (the embedding row is not counted)."""
    total = 0
    for name, dims, ty, _, size in header(s)[1]:
        if name == "token_embd.weight" and s.out_type is not None:
            continue
        total += size
    return total


def kv_bytes_per_position(s: Spec) -> int:
    """f32 K and V of one cached position in every layer."""
    return 2 * s.layers * s.kv_heads * s.head_dim * 4
