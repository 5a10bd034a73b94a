"""The allocation-free decode attention (llmb_attention_noalloc).

Callers that cannot allocate device memory (a host whose GPU memory is a
fixed grant, like the reference's WebAssembly guest, or code recording a CUDA
graph, where it may not allocate) get one entry point whose scratch is a
fixed device array inside the library.  These tests call it through the C
ABI, two calls in a row each time (they share the library's scratch array):

  - on the inputs the model itself used for its last layer's attention after
    llmb_prefill_logits (the query and the KV cache, read with llmb_peek),
    against the attention the existing entry point computed (llmb_peek
    "att"), within the tolerance the parity tests use;
  - on seeded random q, K, V against a float64 softmax attention in numpy
    (cpu.go:304-335), up to the scratch's limits (32 heads, head_dim 128,
    4096 positions) and at position counts that are not a multiple of the
    64-position chunk.

The file is collected last on purpose: it runs after every other test, and
it also passes alone in a fresh process.
"""

import ctypes as C

import numpy as np
import pytest

import llm_b200
from llm_b200 import synth

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5  # max|a - b| / max|b|, as the parity tests


def _call(dq, dk, dv, n_pos, heads, kv_heads, hd, stride, out, stream):
    return llm_b200.lib().llmb_attention_noalloc(C.c_void_p(dq.data_ptr()), C.c_void_p(dk.data_ptr()),
                                                 C.c_void_p(dv.data_ptr()), n_pos, heads, kv_heads, hd, stride,
                                                 C.c_void_p(out.data_ptr()), stream)


def _rel(got, want):
    return float(np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want)))


def attention_f64(q, k, v, heads, kv_heads, hd):
    """softmax(q k / sqrt(hd)) v per query head, in float64 (query head h reads kv head h / (heads / kv_heads))."""
    grp = heads // kv_heads
    out = np.zeros(heads * hd)
    for h in range(heads):
        g = h // grp
        qh = q[h * hd:(h + 1) * hd].astype(np.float64)
        kh = k[:, g * hd:(g + 1) * hd].astype(np.float64)
        vh = v[:, g * hd:(g + 1) * hd].astype(np.float64)
        s = kh @ qh / np.sqrt(hd)
        e = np.exp(s - s.max())
        out[h * hd:(h + 1) * hd] = (e @ vh) / e.sum()
    return out


@pytest.mark.parametrize("spec,n_prompt", [("tiny-qwen2", 70), ("tiny-llama", 150)])
def test_attention_noalloc_matches_model(spec, n_prompt):
    import torch

    ctx = 256
    g = llm_b200.GPU(synth.ensure(spec), ctx=ctx)
    try:
        c = g.cfg
        prompt = synth.prompt_ids(c.vocab, n_prompt, seed=5)
        g.prefill_logits(prompt)
        E, hd, kvd = c.embd, c.head_dim, c.kv_heads * c.head_dim
        m = n_prompt % 64 or 64  # tokens of the last prefill chunk
        q = g.peek("q", m * E).reshape(m, E)[-1]
        want = g.peek("att", m * E).reshape(m, E)[-1]
        kv = g.peek(f"kvblk.{c.layers - 1}.", 2 * ctx * kvd).reshape(2, ctx, kvd)
    finally:
        g.close()
    dev = torch.device("cuda", 0)
    dq = torch.from_numpy(q.copy()).to(dev)
    dk = torch.from_numpy(kv[0, :n_prompt].copy()).to(dev)
    dv = torch.from_numpy(kv[1, :n_prompt].copy()).to(dev)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for call in range(2):  # two calls in a row share the library's scratch array
        out = torch.full((E,), float("nan"), device=dev)
        rc = _call(dq, dk, dv, n_prompt, c.heads, c.kv_heads, hd, kvd, out, stream)
        assert rc == llm_b200.OK, rc
        torch.cuda.synchronize(dev)
        got = out.cpu().numpy()
        assert _rel(got, want) <= REL_TOL, (call, _rel(got, want))
        # and the model's own attention against float64 over the same inputs
        ref = attention_f64(q, kv[0, :n_prompt], kv[1, :n_prompt], c.heads, c.kv_heads, hd)
        assert _rel(got, ref) <= REL_TOL, (call, _rel(got, ref))


@pytest.mark.parametrize("n_pos,heads,kv_heads,hd,pad", [
    (4096, 32, 8, 128, 0),   # every limit of the scratch at once
    (4095, 32, 32, 128, 0),  # one position short of the limit, no GQA sharing
    (1, 14, 2, 64, 0),       # a single position
    (777, 9, 3, 64, 16),     # ragged: not a multiple of 64, rows wider than the heads (kv_stride > kv_heads * hd)
    (130, 7, 1, 128, 0),     # one kv head for every query head
])
def test_attention_noalloc_against_float64(n_pos, heads, kv_heads, hd, pad):
    import torch

    rng = np.random.default_rng(n_pos * 131 + heads)
    stride = kv_heads * hd + pad
    q = rng.normal(0, 1, heads * hd).astype(np.float32)
    k = rng.normal(0, 1, (n_pos, stride)).astype(np.float32)
    v = rng.normal(0, 1, (n_pos, stride)).astype(np.float32)
    ref = attention_f64(q, k, v, heads, kv_heads, hd)
    dev = torch.device("cuda", 0)
    dq, dk, dv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    outs = []
    for call in range(2):
        out = torch.full((heads * hd,), float("nan"), device=dev)
        assert _call(dq, dk, dv, n_pos, heads, kv_heads, hd, stride, out, stream) == llm_b200.OK
        torch.cuda.synchronize(dev)
        got = out.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert _rel(got, ref) <= REL_TOL, (call, _rel(got, ref))
        outs.append(got)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))  # deterministic across calls


def test_attention_noalloc_refuses_oversize():
    """Sizes beyond the fixed scratch are refused before any work (no device pointer is touched)."""
    L = llm_b200.lib()
    fake = C.c_void_p(16)  # never dereferenced: the checks come first
    assert L.llmb_attention_noalloc(fake, fake, fake, 4097, 8, 8, 64, 512, fake, None) == llm_b200.ERR_ARG
    assert L.llmb_attention_noalloc(fake, fake, fake, 16, 64, 8, 64, 512, fake, None) == llm_b200.ERR_ARG
    assert L.llmb_attention_noalloc(fake, fake, fake, 16, 8, 8, 256, 2048, fake, None) == llm_b200.ERR_ARG
    assert L.llmb_attention_noalloc(fake, fake, fake, 16, 9, 2, 64, 128, fake, None) == llm_b200.ERR_ARG
