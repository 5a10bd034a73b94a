"""B200 forward pass for go-wasmcontainers/llm: the host-side mirror of ``llm.GPU``.

The compute path is libllmb200.so (hand-written sm_100a CUDA behind the C ABI
of include/llm_b200.h). This module binds that ABI with ctypes and mirrors the
reference's Go API (gpu.go): ``NewGPU`` opens a GGUF model onto a device,
``GPU.generate`` decodes greedily (``Generate``, gpu.go:946),
``GPU.prefill_logits`` returns the last prompt token's logits
(``PrefillLogits``, gpu.go:904), ``GPU.peek`` reads a named buffer (``Peek``,
gpu.go:1018), ``GPU.memory_used`` (gpu.go:767), ``GPU.stats`` (gpu.go:56),
``GPU.layers`` (gpu.go:143-146) and the package knobs ``DecodeBatch`` and
``PrefillBatch`` (gpu.go:1052,165). Errors raise ``LlmError`` with the
library's status code, as the Go functions return ``error``.

There is no CPU fallback: importing this package fails when the library has
not been built (``python -m llm_b200.build``).
"""

from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libllmb200.so")

OK, ERR_ARG, ERR_IO, ERR_FORMAT, ERR_BOUND, ERR_CONFIG, ERR_TENSOR, ERR_MEMORY, ERR_CONTEXT, ERR_CUDA, ERR_DEVICE = range(11)

# Every function include/llm_b200.h declares.
EXPORTS = ("llmb_open", "llmb_open_reader", "llmb_close", "llmb_last_error", "llmb_get_config", "llmb_memory_used",
           "llmb_get_stats", "llmb_generate", "llmb_generate_batch", "llmb_prefill_logits", "llmb_generate_logits",
           "llmb_peek",
           "llmb_set_layers", "llmb_set_knob", "llmb_get_knob", "llmb_attention_noalloc")


class LlmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{msg} (status {code})")
        self.code = code


class _Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("layers", "embd", "ff", "heads", "kv_heads", "head_dim", "vocab", "ctx")] + \
               [("rope_base", C.c_float), ("eps", C.c_float)] + \
               [(n, C.c_int32) for n in ("rope_neox", "bias", "tied_output")] + [("arch", C.c_char * 16)]


class _Stats(C.Structure):
    _fields_ = [("submits", C.c_int64), ("dispatches", C.c_int64), ("tokens", C.c_int64)]


class _Timing(C.Structure):
    _fields_ = [("prefill_ms", C.c_double), ("decode_ms", C.c_double), ("prompt_tokens", C.c_int32),
                ("generated", C.c_int32), ("submits", C.c_int64), ("dispatches", C.c_int64),
                ("record_ms", C.c_double), ("submit_ms", C.c_double), ("gpu_prefill_ms", C.c_double),
                ("gpu_decode_ms", C.c_double), ("decode_kernel_ms", C.c_double), ("decode_launches", C.c_int64)]


READ_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint64, C.c_void_p, C.c_uint64)
EMIT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int32)

_lib = None


def lib() -> C.CDLL:
    """The loaded C-ABI library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m llm_b200.build` (no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        P, I = C.c_void_p, C.c_int
        L.llmb_open.argtypes, L.llmb_open.restype = [C.c_char_p, I, I, C.POINTER(P)], I
        L.llmb_open_reader.argtypes, L.llmb_open_reader.restype = [READ_FN, P, C.c_uint64, I, I, C.POINTER(P)], I
        L.llmb_close.argtypes, L.llmb_close.restype = [P], None
        L.llmb_last_error.argtypes, L.llmb_last_error.restype = [P], C.c_char_p
        L.llmb_get_config.argtypes, L.llmb_get_config.restype = [P, C.POINTER(_Config)], I
        L.llmb_memory_used.argtypes, L.llmb_memory_used.restype = [P], C.c_uint64
        L.llmb_get_stats.argtypes, L.llmb_get_stats.restype = [P, C.POINTER(_Stats)], I
        L.llmb_generate.argtypes = [P, P, I, I, C.c_int32, EMIT_FN, P, P, C.POINTER(I), C.POINTER(_Timing)]
        L.llmb_generate.restype = I
        L.llmb_generate_batch.argtypes = [P, P, P, I, I, C.c_int32, P, P, C.POINTER(_Timing)]
        L.llmb_generate_batch.restype = I
        L.llmb_prefill_logits.argtypes, L.llmb_prefill_logits.restype = [P, P, I, P], I
        L.llmb_generate_logits.argtypes, L.llmb_generate_logits.restype = [P, P, I, I, P, P], I
        L.llmb_peek.argtypes, L.llmb_peek.restype = [P, C.c_char_p, P, I], I
        L.llmb_set_layers.argtypes, L.llmb_set_layers.restype = [P, I], I
        L.llmb_set_knob.argtypes, L.llmb_set_knob.restype = [C.c_char_p, C.c_int64], I
        L.llmb_get_knob.argtypes, L.llmb_get_knob.restype = [C.c_char_p], C.c_int64
        L.llmb_attention_noalloc.argtypes = [P, P, P, I, I, I, I, I, P, P]
        L.llmb_attention_noalloc.restype = I
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def set_knob(name: str, value: int) -> None:
    """Sets a package knob: decode_batch, prefill_batch, memory_budget, decode_mode, prefill_mode, tag_reset,
    attn_positions, decode_trace, wait_limit_us or drop_publish (include/llm_b200.h describes each)."""
    if lib().llmb_set_knob(name.encode(), int(value)) != OK:
        raise LlmError(ERR_ARG, f"llm: no knob {name!r}")


def get_knob(name: str) -> int:
    return lib().llmb_get_knob(name.encode())


@dataclass
class Config:
    """llm.Config (config.go:11-23)."""

    layers: int
    embd: int
    ff: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    ctx: int
    rope_base: float
    eps: float
    rope_neox: bool
    bias: bool
    tied_output: bool
    arch: str


@dataclass
class Timing:
    """llm.Timing (gpu.go:929-939) plus device time from CUDA events."""

    prefill_ms: float
    decode_ms: float
    prompt_tokens: int
    generated: int
    submits: int
    dispatches: int
    record_ms: float
    submit_ms: float
    gpu_prefill_ms: float
    gpu_decode_ms: float
    decode_kernel_ms: float
    decode_launches: int


class GPU:
    """The forward pass on one B200 (llm.GPU, gpu.go:115-159)."""

    def __init__(self, path: str | None = None, ctx: int = 0, device: int = 0, reader=None, size: int = 0):
        self._h = C.c_void_p()
        self._keep = None
        if reader is not None:
            def _read(_user, off, buf, n):
                try:
                    data = reader(off, n)
                    if len(data) < n:
                        return 1
                    C.memmove(buf, data, n)
                    return 0
                except Exception:
                    return 1

            self._keep = READ_FN(_read)
            rc = lib().llmb_open_reader(self._keep, None, size, ctx, device, C.byref(self._h))
        else:
            rc = lib().llmb_open(os.fsencode(path), ctx, device, C.byref(self._h))
        if rc != OK:
            raise LlmError(rc, lib().llmb_last_error(None).decode(errors="replace"))
        c = _Config()
        lib().llmb_get_config(self._h, C.byref(c))
        self.cfg = Config(c.layers, c.embd, c.ff, c.heads, c.kv_heads, c.head_dim, c.vocab, c.ctx, c.rope_base, c.eps,
                          bool(c.rope_neox), bool(c.bias), bool(c.tied_output), c.arch.decode())

    def _check(self, rc: int) -> None:
        if rc != OK:
            raise LlmError(rc, lib().llmb_last_error(self._h).decode(errors="replace"))

    def close(self) -> None:
        if self._h:
            lib().llmb_close(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def memory_used(self) -> int:
        return lib().llmb_memory_used(self._h)

    @property
    def stats(self) -> dict:
        s = _Stats()
        self._check(lib().llmb_get_stats(self._h, C.byref(s)))
        return dict(submits=s.submits, dispatches=s.dispatches, tokens=s.tokens)

    @property
    def layers(self) -> int:
        return getattr(self, "_layers", 0)

    @layers.setter
    def layers(self, n: int) -> None:
        self._check(lib().llmb_set_layers(self._h, int(n)))
        self._layers = int(n)

    def generate(self, prompt, n: int, eos: int = -1, emit=None) -> tuple[np.ndarray, Timing]:
        """Greedy decoding (Generate, gpu.go:946): returns the emitted tokens and the timing."""
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(n, 1), np.int32)
        n_out = C.c_int()
        tm = _Timing()
        cb = EMIT_FN()
        if emit is not None:
            cb = EMIT_FN(lambda _u, t: 1 if emit(int(t)) else 0)
        self._check(lib().llmb_generate(self._h, _ptr(p), len(p), n, eos, cb, None, _ptr(out), C.byref(n_out),
                                        C.byref(tm)))
        t = Timing(tm.prefill_ms, tm.decode_ms, tm.prompt_tokens, tm.generated, tm.submits, tm.dispatches,
                   tm.record_ms, tm.submit_ms, tm.gpu_prefill_ms, tm.gpu_decode_ms, tm.decode_kernel_ms,
                   tm.decode_launches)
        return out[: n_out.value].copy(), t

    def generate_batch(self, prompts, n: int, eos: int = -1) -> tuple[list[np.ndarray], Timing]:
        """Independent greedy sequences, one KV cache each (llmb_generate_batch): the tokens of each, and the timing."""
        ps = [np.ascontiguousarray(p, np.int32) for p in prompts]
        flat = np.concatenate(ps) if ps else np.zeros(0, np.int32)
        lens = np.array([len(p) for p in ps], np.int32)
        out = np.zeros((len(ps), max(n, 1)), np.int32)
        n_out = np.zeros(len(ps), np.int32)
        tm = _Timing()
        self._check(lib().llmb_generate_batch(self._h, _ptr(flat), _ptr(lens), len(ps), n, eos, _ptr(out),
                                              _ptr(n_out), C.byref(tm)))
        t = Timing(tm.prefill_ms, tm.decode_ms, tm.prompt_tokens, tm.generated, tm.submits, tm.dispatches,
                   tm.record_ms, tm.submit_ms, tm.gpu_prefill_ms, tm.gpu_decode_ms, tm.decode_kernel_ms,
                   tm.decode_launches)
        return [out[i, : n_out[i]].copy() for i in range(len(ps))], t

    def prefill_logits(self, prompt) -> np.ndarray:
        """The logits of the prompt's last token (PrefillLogits, gpu.go:904)."""
        p = np.ascontiguousarray(prompt, np.int32)
        logits = np.zeros(self.cfg.vocab, np.float32)
        self._check(lib().llmb_prefill_logits(self._h, _ptr(p), len(p), _ptr(logits)))
        return logits

    def generate_logits(self, prompt, n: int) -> tuple[np.ndarray, np.ndarray]:
        """Greedy tokens and the logits that chose each (a test hook)."""
        p = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(n, np.int32)
        logits = np.zeros((n, self.cfg.vocab), np.float32)
        self._check(lib().llmb_generate_logits(self._h, _ptr(p), len(p), n, _ptr(toks), _ptr(logits)))
        return toks, logits

    def peek(self, name: str, n: int) -> np.ndarray:
        """The first n words of a named device buffer, as float32 (Peek, gpu.go:1018)."""
        out = np.zeros(n, np.float32)
        self._check(lib().llmb_peek(self._h, name.encode(), _ptr(out), n))
        return out


def NewGPU(path: str, ctx: int = 0, device: int = 0) -> GPU:
    """NewGPU (gpu.go:465): parses the model, allocates its buffers and streams its weights to the device."""
    return GPU(path, ctx, device)
