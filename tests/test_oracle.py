"""Pins the CPU oracle (oracle/cpu_ref.c) before anything is compared with it.

The reference is Go and cannot run here, so its own tests are restated against
the restatement: f16 known answers (tokenizer_test.go:42-53), the NEOX
permutation identity (kernels_test.go:24-58), the GGUF parse and refusal cases
(gguf/gguf_test.go:13-78) and the FuzzParse corpus (gguf_test.go:80-85). The
forward pass is pinned structurally against an independent float64 numpy
forward pass (tests/np_forward.py).
"""

import json
import os
import struct

import numpy as np
import pytest

from tests.np_forward import NumpyModel

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# ---------------------------------------------------------------- f16 --


def test_f16_round_trip(oracle):
    """TestF16RoundTrip, tokenizer_test.go:42-53."""
    for v in [0, 1, -2, 0.5, 65504, 6.1e-5, 5.96e-8, 3.14159]:
        v = float(np.float32(v))
        h = oracle.f32_to_f16(v)
        assert oracle.f32_to_f16(oracle.f16_to_f32(h)) == h, v
    assert oracle.f32_to_f16(1.0) == 0x3C00
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f32_to_f16(65520.0) == 0x7C00


def test_f16_to_f32_exhaustive(oracle):
    """F16ToF32 (f16.go:6-28) is exact: every binary16 value against numpy's conversion."""
    for h in range(0, 1 << 16):
        want = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        got = np.float32(oracle.f16_to_f32(h))
        if np.isnan(want):
            assert np.isnan(got), hex(h)
        else:
            assert got.view(np.uint32) == want.view(np.uint32), hex(h)


def test_f32_to_f16_round_to_nearest_even(oracle):
    """F32ToF16 (f16.go:30-65) rounds to nearest even, as numpy does (NaN payloads aside)."""
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 1 << 32, 20000, dtype=np.uint64).astype(np.uint32)
    vals = bits.view(np.float32)
    specials = np.array([0.0, -0.0, 65504, 65519.99, 65520, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 1e-9, np.inf, -np.inf],
                        np.float32)
    for f in np.concatenate([vals, specials]):
        if np.isnan(f):
            assert oracle.f32_to_f16(float(f)) & 0x7E00 == 0x7E00
            continue
        want = int(np.array([f], np.float32).astype(np.float16).view(np.uint16)[0])
        assert oracle.f32_to_f16(float(f)) == want, (f, hex(want))


# ------------------------------------------------------------ NEOX rope --


def test_neox_rows_equal_neox_rope(oracle):
    """TestNeoxRowsEqualNeoxRope, kernels_test.go:24-58: the adjacent-pair rotation
    of rows permuted by neoxMap equals the NEOX rotation, bit for bit."""
    hd, heads = 64, 3
    x = np.array([((i * 7919) % 101) / 17 - 3 for i in range(hd * heads)], np.float32)
    perm = lambda v: np.array([v[oracle.neox_map(nr, hd)] for nr in range(len(v))], np.float32)
    assert len({oracle.neox_map(nr, hd) for nr in range(hd * heads)}) == hd * heads
    want = perm(oracle.rope(x, 37, heads, hd, 1e6, True))
    got = oracle.rope(perm(x), 37, heads, hd, 1e6, False)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # neoxRows on 2-byte rows of 4: new row 1 is old row 2 (kernels_test.go:54-56)
    b = bytes(range(8))
    rows = b"".join(b[2 * oracle.neox_map(nr, 4): 2 * oracle.neox_map(nr, 4) + 2] for nr in range(4))
    assert rows[2] == 4 and rows[4] == 2


# ------------------------------------------------------------------ GGUF --

VT_STRING, VT_U32, T_F32 = 8, 4, 0


def build_tiny_gguf(mut=None) -> bytes:
    """`build`, gguf/gguf_test.go:13-40: one metadata string, one u32, one F32 tensor of 4."""
    b = bytearray()
    s = lambda t: b.extend(struct.pack("<Q", len(t)) + t.encode())
    b += b"GGUF" + struct.pack("<IQQ", 3, 1, 2)
    s("general.architecture")
    b += struct.pack("<I", VT_STRING)
    s("llama")
    s("x.count")
    b += struct.pack("<II", VT_U32, 7)
    s("w")
    b += struct.pack("<IQIQ", 1, 4, T_F32, 0)
    while len(b) % 32:
        b.append(0)
    b += bytes(16)
    if mut:
        mut(b)
    return bytes(b)


def test_gguf_parse(oracle):
    """TestParse, gguf/gguf_test.go:42-58."""
    f = oracle.GGUF(build_tiny_gguf())
    assert f.error is None
    assert f.str("general.architecture") == "llama"
    assert f.uint("x.count") == 7
    (w,) = f.tensors()
    assert w["name"] == "w" and w["size"] == 16 and f.data_offset % 32 == 0


def _refusal_cases():
    d = build_tiny_gguf()
    ver = bytearray(d)
    ver[4] = 2
    tens = bytearray(d)
    tens[8 + 7] = 0x7F
    return {
        "magic": (b"GGUX" + d[4:], "magic"),
        "version": (bytes(ver), "version"),
        "tensors": (bytes(tens), "bound"),
        "truncated": (d[:40], None),
        "past end": (d[:-4], "bound"),
    }


@pytest.mark.parametrize("case", list(_refusal_cases()))
def test_gguf_refusals(oracle, case):
    """TestRefusals, gguf/gguf_test.go:60-78."""
    data, want = _refusal_cases()[case]
    f = oracle.GGUF(data)
    assert f.error is not None
    if want is not None:
        assert f.error == want


def load_corpus():
    with open(os.path.join(GOLDEN, "gguf_fuzz_corpus.json")) as f:
        return {k: bytes.fromhex(v) for k, v in json.load(f)["inputs"].items()}


def test_gguf_fuzz_corpus(oracle):
    """FuzzParse, gguf/gguf_test.go:80-85: every corpus input parses or is refused
    without a crash, and an accepted header's tensors lie inside the input."""
    corpus = load_corpus()
    assert len(corpus) == 216
    accepted = 0
    for name, data in corpus.items():
        f = oracle.GGUF(data)
        if f.error is None:
            accepted += 1
            for t in f.tensors():
                assert f.data_offset + t["offset"] + t["size"] <= len(data), name
    assert accepted < len(corpus)


def test_gguf_bounds(oracle):
    """Bounded reads (gguf/gguf.go:18-26,195-208,270-277): oversized counts and lengths are ErrBound."""
    big_str = lambda b: b.__setitem__(slice(24, 32), struct.pack("<Q", 1 << 25))
    assert oracle.GGUF(build_tiny_gguf(big_str)).error == "bound"
    nkv = lambda b: b.__setitem__(slice(16, 24), struct.pack("<Q", (1 << 16) + 1))
    assert oracle.GGUF(build_tiny_gguf(nkv)).error == "bound"
    # an array longer than the rest of the header
    b = bytearray(b"GGUF" + struct.pack("<IQQ", 3, 0, 1))
    b += struct.pack("<Q", 1) + b"a" + struct.pack("<IIQ", 9, 4, 1 << 20)
    assert oracle.GGUF(bytes(b)).error == "bound"
    # a nested array is a format error
    b = bytearray(b"GGUF" + struct.pack("<IQQ", 3, 0, 1))
    b += struct.pack("<Q", 1) + b"a" + struct.pack("<IIQ", 9, 9, 1) + struct.pack("<IQ", 4, 0) + bytes(16)
    assert oracle.GGUF(bytes(b)).error == "format"


def test_gguf_alignment_rules(oracle):
    """general.alignment must be an unsigned multiple of 8 (gguf/gguf.go:335-342)."""

    def with_align(vt, payload):
        b = bytearray(b"GGUF" + struct.pack("<IQQ", 3, 0, 1))
        k = b"general.alignment"
        b += struct.pack("<Q", len(k)) + k + struct.pack("<I", vt) + payload
        return bytes(b)

    assert oracle.GGUF(with_align(4, struct.pack("<I", 64))).alignment == 64
    assert oracle.GGUF(with_align(4, struct.pack("<I", 12))).error == "format"
    assert oracle.GGUF(with_align(5, struct.pack("<i", 64))).error == "format"  # int64 kind
    assert oracle.GGUF(with_align(4, struct.pack("<I", 0))).error == "format"


# ------------------------------------------------------- matvec pieces --


@pytest.mark.parametrize("ty", [2, 3, 8])
def test_matvec_blocks(oracle, ty):
    """matvec (cpu.go:143-222) on random blocks against float64 dequantisation."""
    from llm_b200 import synth
    from tests.np_forward import dequant

    rng = np.random.default_rng(ty)
    n_in, n_out = 256, 40
    blk = synth._blocks(rng, ty, n_out, n_in)
    x = rng.normal(0, 1, n_in).astype(np.float32)
    got = oracle.matvec(ty, n_in, n_out, blk, x)
    W = dequant(blk.reshape(-1), 0, [n_in, n_out], ty)
    want = W @ x.astype(np.float64)
    assert np.max(np.abs(got - want)) <= 1e-5 * np.max(np.abs(want))


def test_rmsnorm_and_argmax(oracle):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, 576).astype(np.float32)
    w = (1 + rng.normal(0, 0.05, 576)).astype(np.float32)
    got = oracle.rmsnorm(x, w, 1e-5)
    want = x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-5) * w
    assert np.allclose(got, want, rtol=2e-6, atol=1e-7)
    assert oracle.argmax(np.array([1, 3, 3, 2], np.float32)) == 1  # the first on ties (cpu.go:387-397)


# ------------------------------------------------------------ forward --


@pytest.mark.parametrize("spec", ["tiny-llama", "tiny-mixed", "tiny-qwen2", "tiny-hd128"])
def test_forward_matches_float64(oracle, model_path, spec):
    """The oracle's Forward against the independent float64 forward over 12 tokens."""
    path = model_path(spec)
    cpu = oracle.CPU(path, 64)
    ref = NumpyModel(path, 64)
    toks = np.random.default_rng(3).integers(0, cpu.cfg.vocab, 12)
    for t in toks:
        got = cpu.forward(int(t))
        want = ref.forward(int(t))
        rel = np.max(np.abs(got - want)) / np.max(np.abs(want))
        assert rel < 2e-5, rel
    assert cpu.pos == 12


def test_forward_threads_bit_identical(oracle, model_path):
    """Rows spread over threads are summed in the same order: identical logits."""
    path = model_path("tiny-qwen2")
    prompt = np.arange(5, dtype=np.int32) * 37
    outs = []
    for n in (1, 4):
        oracle.set_threads(n)
        cpu = oracle.CPU(path, 32)
        toks, sl = cpu.generate(prompt, 4, step_logits=True)
        outs.append((toks, sl))
    oracle.set_threads(min(8, os.cpu_count() or 1))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1].view(np.uint32), outs[1][1].view(np.uint32))


def test_context_full_is_an_error(oracle, model_path):
    """cpu.go:227-229 panics on a full context; the restatement returns an error."""
    cpu = oracle.CPU(model_path("tiny-llama"), 2)
    cpu.forward(1)
    cpu.forward(2)
    with pytest.raises(RuntimeError, match="ctx"):
        cpu.forward(3)


def test_trace_max_layers(oracle, model_path):
    """MaxLayers / LastX (cpu.go:29-33,352-356): truncated passes give the residual, no logits."""
    path = model_path("tiny-llama")
    cpu = oracle.CPU(path, 8)
    cpu.set_max_layers(-1)
    cpu.forward(7)
    x0 = cpu.last_x()
    ref = NumpyModel(path, 8)
    assert np.allclose(x0, ref.w["token_embd.weight"][7], rtol=0, atol=1e-7)
    assert cpu.pos == 1


@pytest.mark.parametrize("spec", ["tiny-tie-far", "tiny-tie-near"])
def test_tie_models_tie_every_step(oracle, model_path, spec):
    """The tie models (an output matrix of identical row pairs) give every logit an exact twin in the oracle,
    and its greedy tokens are always the lower index of the pair (cpu.go:389-397)."""
    from llm_b200 import synth

    s = synth.SPECS[spec]
    cpu = oracle.CPU(model_path(spec), 256)
    toks, lg = cpu.generate(synth.prompt_ids(s.vocab, 12, seed=3), 16, step_logits=True)
    a, b = (lg[:, : s.vocab // 2], lg[:, s.vocab // 2:]) if s.tie == "far" else (lg[:, 0::2], lg[:, 1::2])
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.all(toks < s.vocab // 2) if s.tie == "far" else np.all(toks % 2 == 0)
