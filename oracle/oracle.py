"""ctypes wrapper of the CPU oracle (oracle/cpu_ref.c).

TEST INFRASTRUCTURE: imported only by tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline legs, as the checker. The product never imports it.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

ERRORS = {0: "ok", 1: "magic", 2: "version", 3: "bound", 4: "format", 5: "eof", 6: "config",
          7: "tensor", 8: "io", 9: "ctx", 10: "arg"}


class Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("layers", "embd", "ff", "heads", "kv_heads", "head_dim", "vocab", "ctx")] + \
               [("rope_base", C.c_float), ("eps", C.c_float)] + \
               [(n, C.c_int32) for n in ("rope_neox", "bias", "tied_output", "arch_qwen2")]


def build() -> str:
    """Compiles the oracle with its Makefile (gcc; seconds)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "cpu_ref.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        L = C.CDLL(LIB_PATH)
        P, I, U64, F = C.c_void_p, C.c_int, C.c_uint64, C.c_float
        L.orc_f16_to_f32.argtypes, L.orc_f16_to_f32.restype = [C.c_uint16], F
        L.orc_f32_to_f16.argtypes, L.orc_f32_to_f16.restype = [F], C.c_uint16
        L.orc_round_f16.argtypes, L.orc_round_f16.restype = [F], F
        L.orc_gguf_parse.argtypes, L.orc_gguf_parse.restype = [C.c_char_p, U64, C.POINTER(P)], I
        L.orc_gguf_free.argtypes = [P]
        L.orc_gguf_find.argtypes, L.orc_gguf_find.restype = [P, C.c_char_p], I
        L.orc_gguf_uint.argtypes, L.orc_gguf_uint.restype = [P, C.c_char_p, C.POINTER(U64)], I
        L.orc_gguf_float.argtypes, L.orc_gguf_float.restype = [P, C.c_char_p, C.POINTER(C.c_double)], I
        L.orc_gguf_str.argtypes, L.orc_gguf_str.restype = [P, C.c_char_p], C.c_char_p
        for n in ("orc_gguf_ntensors", "orc_gguf_nkv", "orc_gguf_data_offset", "orc_gguf_alignment"):
            getattr(L, n).argtypes, getattr(L, n).restype = [P], U64
        L.orc_gguf_tensor.argtypes = [P, U64, C.POINTER(C.c_char_p), C.POINTER(C.c_uint32), C.POINTER(U64),
                                      C.POINTER(C.c_uint32), C.POINTER(U64), C.POINTER(U64)]
        L.orc_gguf_tensor.restype = I
        L.orc_set_threads.argtypes = [I]
        L.orc_rmsnorm.argtypes = [P, P, P, I, F]
        L.orc_matvec.argtypes, L.orc_matvec.restype = [C.c_uint32, I, I, P, P, P], I
        L.orc_rope.argtypes = [P, I, I, I, F, I]
        L.orc_neox_map.argtypes, L.orc_neox_map.restype = [I, I], I
        L.orc_argmax.argtypes, L.orc_argmax.restype = [P, I], C.c_int32
        L.orc_load.argtypes, L.orc_load.restype = [C.c_char_p, I, C.POINTER(P), C.c_char_p, I], I
        L.orc_free.argtypes = [P]
        L.orc_get_config.argtypes = [P, C.POINTER(Config)]
        L.orc_reset.argtypes = [P]
        L.orc_pos.argtypes, L.orc_pos.restype = [P], I
        L.orc_set_max_layers.argtypes = [P, I]
        L.orc_last_x.argtypes, L.orc_last_x.restype = [P], C.POINTER(F)
        L.orc_forward.argtypes, L.orc_forward.restype = [P, C.c_int32, P], I
        L.orc_generate.argtypes, L.orc_generate.restype = [P, P, I, I, P, P], I
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


class GGUF:
    """A parsed GGUF header (gguf.Parse)."""

    def __init__(self, data: bytes):
        self._h = C.c_void_p()
        self.data = data
        self.err = lib().orc_gguf_parse(data, len(data), C.byref(self._h))

    @property
    def error(self) -> str | None:
        return None if self.err == 0 else ERRORS[self.err]

    def __del__(self):
        if getattr(self, "_h", None) and self._h:
            lib().orc_gguf_free(self._h)
            self._h = None

    def tensors(self):
        out = []
        for i in range(lib().orc_gguf_ntensors(self._h)):
            name = C.c_char_p()
            nd = C.c_uint32()
            dims = (C.c_uint64 * 4)()
            ty = C.c_uint32()
            off, size = C.c_uint64(), C.c_uint64()
            lib().orc_gguf_tensor(self._h, i, C.byref(name), C.byref(nd), dims, C.byref(ty), C.byref(off), C.byref(size))
            out.append(dict(name=name.value.decode(), dims=list(dims[:nd.value]), type=ty.value, offset=off.value,
                            size=size.value))
        return out

    def uint(self, key: str):
        v = C.c_uint64()
        return v.value if lib().orc_gguf_uint(self._h, key.encode(), C.byref(v)) else None

    def float(self, key: str):
        v = C.c_double()
        return v.value if lib().orc_gguf_float(self._h, key.encode(), C.byref(v)) else None

    def str(self, key: str):
        v = lib().orc_gguf_str(self._h, key.encode())
        return None if v is None else v.decode()

    @property
    def data_offset(self) -> int:
        return lib().orc_gguf_data_offset(self._h)

    @property
    def alignment(self) -> int:
        return lib().orc_gguf_alignment(self._h)


class CPU:
    """The CPU forward pass (cpu.go's CPU: LoadCPU, Forward, Reset, Pos)."""

    def __init__(self, path: str, max_ctx: int):
        self._h = C.c_void_p()
        err = C.create_string_buffer(512)
        e = lib().orc_load(path.encode(), max_ctx, C.byref(self._h), err, 512)
        if e:
            raise RuntimeError(f"oracle load: {ERRORS.get(e, e)}: {err.value.decode()}")
        self.cfg = Config()
        lib().orc_get_config(self._h, C.byref(self.cfg))

    def __del__(self):
        if getattr(self, "_h", None) and self._h:
            lib().orc_free(self._h)
            self._h = None

    def reset(self) -> None:
        lib().orc_reset(self._h)

    @property
    def pos(self) -> int:
        return lib().orc_pos(self._h)

    def set_max_layers(self, n: int) -> None:
        lib().orc_set_max_layers(self._h, n)

    def last_x(self) -> np.ndarray:
        return np.ctypeslib.as_array(lib().orc_last_x(self._h), shape=(self.cfg.embd,)).copy()

    def forward(self, tok: int) -> np.ndarray:
        logits = np.zeros(self.cfg.vocab, np.float32)
        e = lib().orc_forward(self._h, int(tok), _p(logits))
        if e not in (0, 1):
            raise RuntimeError(f"oracle forward: {ERRORS.get(e, e)}")
        return logits

    def generate(self, prompt, n: int, step_logits: bool = False):
        """Greedy tokens after the prompt (and the logits that chose each)."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(n, np.int32)
        sl = np.zeros((n, self.cfg.vocab), np.float32) if step_logits else None
        e = lib().orc_generate(self._h, _p(prompt), len(prompt), n, _p(toks), _p(sl) if sl is not None else None)
        if e:
            raise RuntimeError(f"oracle generate: {ERRORS.get(e, e)}")
        return (toks, sl) if step_logits else toks


def f16_to_f32(h: int) -> float:
    return lib().orc_f16_to_f32(h)


def f32_to_f16(f: float) -> int:
    return lib().orc_f32_to_f16(f)


def round_f16(f: float) -> float:
    return lib().orc_round_f16(f)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib().orc_rmsnorm(_p(out), _p(x), _p(w), len(x), eps)
    return out


def matvec(ty: int, n_in: int, n_out: int, blocks: np.ndarray, x: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks).view(np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(n_out, np.float32)
    e = lib().orc_matvec(ty, n_in, n_out, _p(blocks), _p(x), _p(out))
    if e:
        raise RuntimeError(f"oracle matvec: {ERRORS.get(e, e)}")
    return out


def rope(x: np.ndarray, pos: int, heads: int, dim: int, base: float, neox: bool) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().orc_rope(_p(x), pos, heads, dim, base, int(neox))
    return x


def neox_map(nr: int, hd: int) -> int:
    return lib().orc_neox_map(nr, hd)


def argmax(l: np.ndarray) -> int:
    l = np.ascontiguousarray(l, np.float32)
    return lib().orc_argmax(_p(l), len(l))
