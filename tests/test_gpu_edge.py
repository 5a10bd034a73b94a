"""Edge semantics of the forward pass on the GPU, through the C ABI.

1. The greedy tie rule: the first index of the largest logit wins
   (kernels.go:351-353, cpu.go:389-397).  The tie models (synth
   TINY_TIE_FAR / TINY_TIE_NEAR) have an output matrix whose rows come in
   identical pairs, so every logit has an exact twin and every step's argmax
   is a tie: across CTAs (rows i and i + vocab/2) or inside one 8-row tile
   (rows 2i and 2i + 1).  Each argmax implementation must pick the lower
   index: the persistent decode kernel's head (decode_mode 0), the per-phase
   head k_head (decode_mode 1, and the prefill's first token), the
   multi-stream head over the chunked products (k_argmax_rows) and its
   per-token twin k_head_batch (prefill_mode 1).
2. A bounded device wait that runs out: with the knobs wait_limit_us and
   drop_publish, one publish of the persistent kernel is skipped, the
   consumers' wait ends at the limit, the call returns LLMB_ERR_DEVICE, and
   the next call (knobs off) decodes correctly.  Nothing faults or hangs:
   every wait in the kernel is bounded and the kernel returns.
"""

import numpy as np
import pytest

import llm_b200
from llm_b200 import synth

pytestmark = pytest.mark.gpu


def _knobs(**kv):
    old = {k: llm_b200.get_knob(k) for k in kv}
    for k, v in kv.items():
        llm_b200.set_knob(k, v)
    return old


def _restore(old):
    for k, v in old.items():
        llm_b200.set_knob(k, v)


def _twin_ok(spec, toks):
    """Every sampled token is the lower index of its twin pair."""
    v = synth.SPECS[spec].vocab
    toks = np.asarray(toks)
    return bool(np.all(toks < v // 2)) if synth.SPECS[spec].tie == "far" else bool(np.all(toks % 2 == 0))


@pytest.mark.parametrize("spec", ["tiny-tie-far", "tiny-tie-near"])
@pytest.mark.parametrize("mode", [0, 1], ids=["persistent", "per-phase"])
@pytest.mark.parametrize("batch", [1, 8])
def test_argmax_ties_generate(oracle, spec, mode, batch):
    old = _knobs(decode_mode=mode, decode_batch=batch)
    try:
        with llm_b200.GPU(synth.ensure(spec), ctx=256) as g:
            prompt = synth.prompt_ids(g.cfg.vocab, 12, seed=3)
            got, _ = g.generate(prompt, 40)
            toks, logits = g.generate_logits(prompt, 8)
    finally:
        _restore(old)
    want, want_logits = oracle.CPU(synth.ensure(spec), 256).generate(prompt, 40, step_logits=True)
    v = synth.SPECS[spec].vocab
    # the oracle's logits tie exactly at every step (the premise of the test)
    lw = want_logits
    twins = (lw[:, : v // 2], lw[:, v // 2:]) if synth.SPECS[spec].tie == "far" else (lw[:, 0::2], lw[:, 1::2])
    assert np.array_equal(twins[0].view(np.uint32), twins[1].view(np.uint32))
    assert _twin_ok(spec, want)
    assert np.array_equal(got, want), (got.tolist(), want.tolist())
    assert np.array_equal(toks, want[:8])
    # and the GPU's own logits tie too (the pairs are computed identically)
    lg = logits
    gt = (lg[:, : v // 2], lg[:, v // 2:]) if synth.SPECS[spec].tie == "far" else (lg[:, 0::2], lg[:, 1::2])
    assert np.array_equal(gt[0].view(np.uint32), gt[1].view(np.uint32))


@pytest.mark.parametrize("spec", ["tiny-tie-far", "tiny-tie-near"])
@pytest.mark.parametrize("pmode", [0, 1], ids=["products", "per-token"])
def test_argmax_ties_generate_batch(oracle, spec, pmode):
    old = _knobs(prefill_mode=pmode)
    try:
        with llm_b200.GPU(synth.ensure(spec), ctx=256) as g:
            prompts = [synth.prompt_ids(g.cfg.vocab, n, seed=40 + n) for n in (5, 33, 70, 9)]
            outs, _ = g.generate_batch(prompts, 24)
    finally:
        _restore(old)
    cpu = oracle.CPU(synth.ensure(spec), 256)
    for p, got in zip(prompts, outs):
        want = cpu.generate(p, 24)
        assert _twin_ok(spec, want)
        assert np.array_equal(got, want), (got.tolist(), want.tolist())


def test_device_wait_runs_out(oracle):
    """A publish the persistent kernel skips: the wait for it ends at the limit with LLMB_ERR_DEVICE."""
    spec = "tiny-llama"
    with llm_b200.GPU(synth.ensure(spec), ctx=256) as g:
        prompt = synth.prompt_ids(g.cfg.vocab, 20, seed=17)
        want = oracle.CPU(synth.ensure(spec), 256).generate(prompt, 30)
        old = _knobs(decode_mode=0, decode_batch=8, wait_limit_us=20000, drop_publish=len(prompt) + 2)
        try:
            with pytest.raises(llm_b200.LlmError) as e:
                g.generate(prompt, 30)
        finally:
            _restore(old)
        assert e.value.code == llm_b200.ERR_DEVICE
        assert "did not arrive in time" in str(e.value)
        # the context and the model stay usable: the next call decodes correctly, twice
        for _ in range(2):
            got, _ = g.generate(prompt, 30)
            assert np.array_equal(got, want)
        # a drop past the tokens of the call changes nothing
        old = _knobs(wait_limit_us=20000, drop_publish=len(prompt) + 100)
        try:
            got, _ = g.generate(prompt, 30)
        finally:
            _restore(old)
        assert np.array_equal(got, want)
