"""The C ABI on the CPU: the library loads, exports every declared symbol,
keeps its knobs, and refuses bad model files before any device work.

The GGUF parse and ConfigFrom run on the host before the first CUDA call, so
the product's parser is checked here against the restated reference tests
(gguf/gguf_test.go:42-85, config.go:29-73) and against the oracle's parser.
"""

import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

import llm_b200
from llm_b200 import synth
from tests.test_oracle import build_tiny_gguf, load_corpus, _refusal_cases

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "llm_b200.h")).read()
    return re.findall(r"LLMB_API\s+[\w\s\*]+?\b(llmb_\w+)\s*\(", src)


def test_library_exports_every_declared_symbol():
    L = llm_b200.lib()
    names = declared_functions()
    assert sorted(names) == sorted(llm_b200.EXPORTS)
    for n in names:
        assert hasattr(L, n), n


def test_knobs():
    """DecodeBatch clamps to 1..MaxBatch (gpu.go:1046,1054), PrefillBatch to 1..64."""
    old = {k: llm_b200.get_knob(k) for k in ("decode_batch", "prefill_batch", "memory_budget", "decode_mode",
                                              "attn_positions")}
    try:
        llm_b200.set_knob("decode_batch", 100)
        assert llm_b200.get_knob("decode_batch") == 16
        llm_b200.set_knob("decode_batch", 0)
        assert llm_b200.get_knob("decode_batch") == 1
        llm_b200.set_knob("prefill_batch", 1000)
        assert llm_b200.get_knob("prefill_batch") == 64
        llm_b200.set_knob("attn_positions", 100)
        assert llm_b200.get_knob("attn_positions") == 96
        llm_b200.set_knob("attn_positions", 1000)
        assert llm_b200.get_knob("attn_positions") == 256
        llm_b200.set_knob("attn_positions", 0)
        assert llm_b200.get_knob("attn_positions") == 0
        with pytest.raises(llm_b200.LlmError):
            llm_b200.set_knob("tpr", 8)
        assert llm_b200.get_knob("nothing") == -1
    finally:
        for k, v in old.items():
            llm_b200.set_knob(k, v)


def open_bytes(data: bytes):
    """llmb_open_reader over bytes in memory: returns (status, message)."""
    L = llm_b200.lib()
    h = C.c_void_p()

    def rd(_u, off, buf, n):
        if off + n > len(data):
            return 1
        C.memmove(buf, data[off:off + n], n)
        return 0

    fn = llm_b200.READ_FN(rd)
    rc = L.llmb_open_reader(fn, None, len(data), 64, 0, C.byref(h))
    msg = L.llmb_last_error(None).decode(errors="replace")
    if rc == 0:
        L.llmb_close(h)
    return rc, msg


def test_parse_refusals_through_the_abi():
    """TestRefusals (gguf/gguf_test.go:60-78) through llmb_open_reader."""
    want = {"magic": llm_b200.ERR_FORMAT, "version": llm_b200.ERR_FORMAT, "tensors": llm_b200.ERR_BOUND,
            "truncated": None, "past end": llm_b200.ERR_BOUND}
    for name, (data, _) in _refusal_cases().items():
        rc, msg = open_bytes(data)
        assert rc != 0, name
        if want[name] is not None:
            assert rc == want[name], (name, rc, msg)
        assert rc in (llm_b200.ERR_FORMAT, llm_b200.ERR_BOUND), (name, rc, msg)


def test_valid_header_reaches_config():
    """TestParse's file (gguf/gguf_test.go:13-58) parses; ConfigFrom then refuses it (no hyperparameters)."""
    rc, msg = open_bytes(build_tiny_gguf())
    assert rc == llm_b200.ERR_CONFIG, msg
    assert "implausible llama hyperparameters" in msg


def test_open_missing_file():
    with pytest.raises(llm_b200.LlmError) as e:
        llm_b200.GPU("/nonexistent/model.gguf")
    assert e.value.code == llm_b200.ERR_IO


def test_fuzz_corpus_agrees_with_oracle(oracle):
    """Both parsers accept and refuse the same FuzzParse inputs, with the same error class."""
    cls = {"magic": llm_b200.ERR_FORMAT, "version": llm_b200.ERR_FORMAT, "format": llm_b200.ERR_FORMAT,
           "bound": llm_b200.ERR_BOUND}
    for name, data in load_corpus().items():
        ref = oracle.GGUF(data).error
        rc, msg = open_bytes(data)
        if ref is None:
            assert rc not in (llm_b200.ERR_FORMAT, llm_b200.ERR_BOUND), (name, rc, msg)
        else:
            assert rc == cls[ref], (name, ref, rc, msg)


def _config_file(tmp_path, mutate):
    s = synth.TINY_LLAMA
    hdr, infos = synth.header(s)
    data = bytearray(hdr)
    mutate(data)
    end = max(o + n for _, _, _, o, n in infos)
    data += bytes(end)
    return bytes(data)


@pytest.mark.parametrize("arch,want", [(b"llama", None), (b"gpt2x", "architecture")])
def test_config_refusals(arch, want):
    """ConfigFrom refusals (config.go:31-33) through the ABI."""
    s = synth.TINY_LLAMA
    hdr, infos = synth.header(s)
    data = bytearray(hdr.replace(b"llama", arch, 1) if len(arch) == 5 else hdr)
    end = len(hdr) + max(o + n for _, _, _, o, n in infos)
    data += bytes(end - len(data))
    rc, msg = open_bytes(bytes(data))
    if want is None:
        assert rc not in (llm_b200.ERR_FORMAT, llm_b200.ERR_BOUND, llm_b200.ERR_CONFIG), msg
    else:
        assert rc == llm_b200.ERR_CONFIG and want in msg, msg


def test_rope_scaling_refused():
    """config.go:47-53: any rope scaling key is refused."""
    s = synth.TINY_LLAMA
    hdr, infos = synth.header(s)
    key = b"llama.rope.scaling.type"
    kv = struct.pack("<Q", len(key)) + key + struct.pack("<IQ", 8, 4) + b"yarn"
    n_kv = struct.unpack_from("<Q", hdr, 16)[0]
    body = hdr[:16] + struct.pack("<Q", n_kv + 1) + hdr[24:]
    # the new key/value goes right after the counts; tensor data offsets stay relative
    data = bytearray(body[:24] + kv + body[24:])
    data += bytes((-len(data)) % 32)
    end = len(data) + max(o + n for _, _, _, o, n in infos)
    data += bytes(end - len(data))
    rc, msg = open_bytes(bytes(data))
    assert rc == llm_b200.ERR_CONFIG and "rope scaling" in msg, msg
