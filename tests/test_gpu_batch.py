"""Multi-stream generation (llmb_generate_batch) against the CPU oracle.

The multi-stream workload runs many independent
sequences on one GPU, each with its own KV cache; each sequence's output
must be token-identical to its own single-stream run of the CPU path
(cpu.go Forward + Argmax, driven as examples/generate does).  The cases
cover ragged prompt lengths across the 64-token batch boundaries, more
sequences than one launch set holds, eos per sequence, the error paths, and
that the single-stream path is unaffected afterwards.
"""

import numpy as np
import pytest

import llm_b200
from llm_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpus():
    opened = {}

    def get(spec, ctx):
        key = (spec, ctx)
        if key not in opened:
            opened[key] = llm_b200.GPU(synth.ensure(spec), ctx=ctx)
        return opened[key]

    yield get
    for g in opened.values():
        g.close()


def prompts_for(vocab, lens, seed):
    return [synth.prompt_ids(vocab, n, seed=seed + i) for i, n in enumerate(lens)]


@pytest.mark.parametrize("spec", ["tiny-llama", "tiny-mixed", "tiny-qwen2"])
def test_batch_matches_single_stream(oracle, gpus, spec):
    g = gpus(spec, 256)
    lens = [1, 5, 64, 70, 17, 130, 33]
    prompts = prompts_for(g.cfg.vocab, lens, seed=40)
    n = 24
    got, tm = g.generate_batch(prompts, n)
    assert tm.prompt_tokens == sum(lens) and tm.generated == n * len(lens)
    cpu = oracle.CPU(synth.ensure(spec), 256)
    for i, p in enumerate(prompts):
        want = cpu.generate(p, n)
        assert np.array_equal(got[i], want), (i, got[i], want)


def test_batch_more_sequences_than_a_launch(oracle, gpus):
    """70 sequences: two launch sets per decode step, prompts packed across many batches."""
    g = gpus("tiny-llama", 128)
    rng = np.random.default_rng(5)
    lens = [int(v) for v in rng.integers(1, 40, size=70)]
    prompts = prompts_for(g.cfg.vocab, lens, seed=100)
    n = 6
    got, tm = g.generate_batch(prompts, n)
    cpu = oracle.CPU(synth.ensure("tiny-llama"), 128)
    for i, p in enumerate(prompts):
        assert np.array_equal(got[i], cpu.generate(p, n)), i


@pytest.mark.parametrize("mode", [1, 2], ids=["per-token", "fp32-products"])
def test_batch_other_paths(oracle, gpus, mode):
    """prefill_mode 1 (the per-token kernels) and 2 (the float32 CUDA-core products): the same batches."""
    g = gpus("tiny-mixed", 256)
    prompts = prompts_for(g.cfg.vocab, [3, 66, 20], seed=80)
    old = llm_b200.get_knob("prefill_mode")
    llm_b200.set_knob("prefill_mode", mode)
    try:
        got, _ = g.generate_batch(prompts, 12)
    finally:
        llm_b200.set_knob("prefill_mode", old)
    cpu = oracle.CPU(synth.ensure("tiny-mixed"), 256)
    for i, p in enumerate(prompts):
        assert np.array_equal(got[i], cpu.generate(p, 12)), i


def test_batch_benchmark_model(oracle, gpus):
    g = gpus("c1-smollm2-q4_0", 512)
    lens = [16, 40, 9]
    prompts = prompts_for(g.cfg.vocab, lens, seed=7)
    n = 8
    got, _ = g.generate_batch(prompts, n)
    cpu = oracle.CPU(synth.ensure("c1-smollm2-q4_0"), 512)
    for i, p in enumerate(prompts):
        assert np.array_equal(got[i], cpu.generate(p, n)), i


def test_batch_eos_per_sequence(oracle, gpus):
    """eos stops only the sequences that sample it, and is not emitted (gpu.go:973-976)."""
    g = gpus("tiny-qwen2", 256)
    prompts = prompts_for(g.cfg.vocab, [12, 30, 7, 50], seed=60)
    n = 20
    cpu = oracle.CPU(synth.ensure("tiny-qwen2"), 256)
    want = [cpu.generate(p, n) for p in prompts]
    eos = int(want[1][9])
    got, tm = g.generate_batch(prompts, n, eos=eos)
    for i in range(len(prompts)):
        w = want[i]
        stop = int(np.argmax(w == eos)) if (w == eos).any() else n
        assert np.array_equal(got[i], w[:stop]), (i, got[i], w[:stop])
    assert tm.generated == sum(len(x) for x in got)


def test_batch_errors_and_single_stream_after(oracle, gpus):
    g = gpus("tiny-llama", 64)
    with pytest.raises(llm_b200.LlmError) as e:
        g.generate_batch([np.arange(10, dtype=np.int32), np.arange(60, dtype=np.int32)], 10)
    assert e.value.code == llm_b200.ERR_CONTEXT
    with pytest.raises(llm_b200.LlmError) as e:
        g.generate_batch([np.arange(4, dtype=np.int32), np.zeros(0, np.int32)], 3)
    assert e.value.code == llm_b200.ERR_ARG
    with pytest.raises(llm_b200.LlmError) as e:
        g.generate_batch([np.array([1, g.cfg.vocab], np.int32)], 3)
    assert e.value.code == llm_b200.ERR_ARG
    prompts = prompts_for(g.cfg.vocab, [9, 20], seed=3)
    got, _ = g.generate_batch(prompts, 5)
    # the single-stream path still matches after a batch call on the same model
    toks, _ = g.generate(prompts[0], 12)
    assert np.array_equal(toks, oracle.CPU(synth.ensure("tiny-llama"), 64).generate(prompts[0], 12))
    assert np.array_equal(got[0], toks[:5])
