"""The allocation-free decode attention (llmb_attention_noalloc).

Callers that cannot allocate device memory (a host whose GPU memory is a
fixed grant, like the reference's WebAssembly guest, or code running where
cudaMalloc is not allowed) get one entry point whose scratch is a fixed
device array inside the library.  This test calls it through the C ABI, twice
in a row, on the inputs the model itself used for its last layer's attention
after llmb_prefill_logits (the query and the KV cache, read with llmb_peek),
and checks each output against the attention the existing entry point
computed (llmb_peek "att"), within the tolerance the parity tests use.

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
    L = llm_b200.lib()
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for call in range(2):  # two calls in a row share the library's scratch array
        out = torch.full((E,), float("nan"), device=dev)
        rc = L.llmb_attention_noalloc(C.c_void_p(dq.data_ptr()), C.c_void_p(dk.data_ptr()), C.c_void_p(dv.data_ptr()),
                                      n_prompt, c.heads, c.kv_heads, hd, kvd, C.c_void_p(out.data_ptr()), stream)
        assert rc == llm_b200.OK, rc
        torch.cuda.synchronize(dev)
        got = out.cpu().numpy()
        rel = float(np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want)))
        assert rel <= REL_TOL, (call, rel)


def test_attention_noalloc_refuses_oversize():
    """Sizes beyond the fixed scratch are refused before any work (no device pointer is touched)."""
    L = llm_b200.lib()
    fake = C.c_void_p(16)  # never dereferenced: the checks come first
    assert L.llmb_attention_noalloc(fake, fake, fake, 4097, 8, 8, 64, 512, fake, None) == llm_b200.ERR_ARG
    assert L.llmb_attention_noalloc(fake, fake, fake, 16, 64, 8, 64, 512, fake, None) == llm_b200.ERR_ARG
    assert L.llmb_attention_noalloc(fake, fake, fake, 16, 8, 8, 256, 2048, fake, None) == llm_b200.ERR_ARG
    assert L.llmb_attention_noalloc(fake, fake, fake, 16, 9, 2, 64, 128, fake, None) == llm_b200.ERR_ARG
