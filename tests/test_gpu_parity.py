"""Parity of the CUDA forward pass with the CPU oracle, through the C ABI.

The bar (the benchmark specification, restating examples/generate check,
main.go:141-181, and the strict oracle tolerance of oracle_test.go:374):
  - greedy tokens identical to the oracle's at every step;
  - step-1 logits (after the prompt) within a relative error
    max|gpu - cpu| / max|cpu| <= REL_TOL;
  - at every decoded step, log-probabilities within NATS_TOL of the oracle's
    over the oracle's top-10 (the oracle_test.go:213-224 measure), and the
    relative logit error within STEP_REL_TOL.
Later steps get the reference's nats tolerance rather than 1e-5 relative:
at ill-conditioned steps of the seeded models every float32 implementation
moves about 1e-5 from the exact result (measured against a float64 forward
pass: the oracle itself is 6.8e-6 off at step 36 of tiny-mixed, where this
path differs from it by 1.8e-5).
"""

import numpy as np
import pytest

import llm_b200
from llm_b200 import synth

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5       # step 1: max|gpu-cpu| / max|cpu| (main.go:159-165 definition)
NATS_TOL = 1e-4      # every step: log-prob differences over the top-10 (f32RefTol, oracle_test.go:374)
STEP_REL_TOL = 5e-5  # every step: relative logit error


def rel_err(got, want):
    return float(np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want)))


def logprob_diff(got, want, k=10):
    """max over the oracle's top-k of |(lp_i - lp_top) - (ref_i - ref_top)|, in nats (oracle_test.go:213-224)."""
    def lsm(x):
        x = x.astype(np.float64)
        m = x.max()
        return x - m - np.log(np.sum(np.exp(x - m)))
    lg, lw = lsm(got), lsm(want)
    top = np.argsort(-want)[:k]
    t0 = top[0]
    return float(np.max(np.abs((lg[top] - lg[t0]) - (lw[top] - lw[t0]))))


def check_step(i, got, want):
    rel = rel_err(got, want)
    assert rel <= (REL_TOL if i == 0 else STEP_REL_TOL), (i, rel)
    nats = logprob_diff(got, want)
    assert nats <= NATS_TOL, (i, nats)


def top2_gap(l):
    s = np.sort(l)
    return float(s[-1] - s[-2])


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


@pytest.fixture(params=[0, 1], ids=["persistent", "per-phase"])
def decode_mode(request):
    old = llm_b200.get_knob("decode_mode")
    llm_b200.set_knob("decode_mode", request.param)
    yield request.param
    llm_b200.set_knob("decode_mode", old)


@pytest.mark.parametrize("spec", ["tiny-llama", "tiny-mixed", "tiny-qwen2"])
@pytest.mark.parametrize("n_prompt", [1, 5, 64, 70, 150])
def test_prefill_logits(oracle, gpus, spec, n_prompt):
    """PrefillLogits (gpu.go:904) against the oracle: chunk boundaries (64) and several attention chunks."""
    g = gpus(spec, 256)
    prompt = synth.prompt_ids(g.cfg.vocab, n_prompt, seed=n_prompt)
    got = g.prefill_logits(prompt)
    cpu = oracle.CPU(synth.ensure(spec), 256)
    for t in prompt:
        want = cpu.forward(int(t))
    assert rel_err(got, want) <= REL_TOL
    assert int(np.argmax(got)) == oracle.argmax(want)


@pytest.mark.parametrize("spec", ["tiny-llama", "tiny-mixed", "tiny-qwen2", "c3-qwen2.5-0.5b"])
def test_prefill_per_token_kernels(oracle, gpus, spec):
    """prefill_mode 1 (one matvec per token and phase) against the oracle, and against the products' path."""
    old = llm_b200.get_knob("prefill_mode")
    g = gpus(spec, 256)
    prompt = synth.prompt_ids(g.cfg.vocab, 70, seed=21)
    try:
        llm_b200.set_knob("prefill_mode", 1)
        got1 = g.prefill_logits(prompt)
    finally:
        llm_b200.set_knob("prefill_mode", old)
    got0 = g.prefill_logits(prompt)
    cpu = oracle.CPU(synth.ensure(spec), 256)
    for t in prompt:
        want = cpu.forward(int(t))
    for got in (got0, got1):
        assert rel_err(got, want) <= REL_TOL
        assert int(np.argmax(got)) == oracle.argmax(want)


@pytest.mark.parametrize("spec", ["tiny-llama", "tiny-mixed", "tiny-qwen2", "tiny-hd128", "c2-smollm2-mixed"])
@pytest.mark.parametrize("n_prompt", [3, 64, 150])
def test_prefill_products_tensor_and_fp32(oracle, gpus, spec, n_prompt):
    """The chunked products on the tensor cores (prefill_mode 0, tcgen05 with split bf16 pieces) and in float32
    on the CUDA cores (prefill_mode 2): the last prompt token's logits against the oracle, both within 1e-5."""
    old = llm_b200.get_knob("prefill_mode")
    g = gpus(spec, 256)
    prompt = synth.prompt_ids(g.cfg.vocab, n_prompt, seed=n_prompt + 3)
    got = {}
    try:
        for mode in (0, 2):
            llm_b200.set_knob("prefill_mode", mode)
            got[mode] = g.prefill_logits(prompt)
    finally:
        llm_b200.set_knob("prefill_mode", old)
    cpu = oracle.CPU(synth.ensure(spec), 256)
    for t in prompt:
        want = cpu.forward(int(t))
    for mode in (0, 2):
        assert rel_err(got[mode], want) <= REL_TOL, (mode, rel_err(got[mode], want))
        assert int(np.argmax(got[mode])) == oracle.argmax(want)


@pytest.mark.parametrize("spec", ["tiny-llama", "tiny-mixed", "tiny-qwen2"])
def test_generate_every_step(oracle, gpus, decode_mode, spec):
    """Every decoded step's logits and token against the oracle's greedy run."""
    g = gpus(spec, 256)
    prompt = synth.prompt_ids(g.cfg.vocab, 20, seed=7)
    n = 40
    want_toks, want_logits = oracle.CPU(synth.ensure(spec), 256).generate(prompt, n, step_logits=True)
    toks, logits = g.generate_logits(prompt, n)
    for i in range(n):
        check_step(i, logits[i], want_logits[i])
        assert toks[i] == want_toks[i], (i, toks[i], want_toks[i], top2_gap(want_logits[i]))


@pytest.mark.parametrize("spec", ["tiny-llama", "tiny-mixed", "tiny-qwen2"])
@pytest.mark.parametrize("batch", [1, 3, 8, 16])
def test_generate_tokens(oracle, gpus, decode_mode, spec, batch):
    """Generate (gpu.go:946) in launches of DecodeBatch tokens: identical greedy tokens."""
    old = llm_b200.get_knob("decode_batch")
    llm_b200.set_knob("decode_batch", batch)
    try:
        g = gpus(spec, 256)
        prompt = synth.prompt_ids(g.cfg.vocab, 33, seed=batch)
        want = oracle.CPU(synth.ensure(spec), 256).generate(prompt, 60)
        got, tm = g.generate(prompt, 60)
        assert np.array_equal(got, want)
        assert tm.generated == 60 and tm.prompt_tokens == 33
    finally:
        llm_b200.set_knob("decode_batch", old)


@pytest.mark.parametrize("spec,n_prompt,n", [("c1-smollm2-q4_0", 16, 16), ("c2-smollm2-mixed", 8, 24),
                                             ("c3-qwen2.5-0.5b", 12, 12)])
def test_benchmark_models_every_step(oracle, gpus, spec, n_prompt, n):
    """The three benchmark files: every step's logits and tokens."""
    g = gpus(spec, 512)
    prompt = synth.prompt_ids(g.cfg.vocab, n_prompt, seed=1)
    want_toks, want_logits = oracle.CPU(synth.ensure(spec), 512).generate(prompt, n, step_logits=True)
    toks, logits = g.generate_logits(prompt, n)
    for i in range(n):
        check_step(i, logits[i], want_logits[i])
    assert np.array_equal(toks, want_toks)


@pytest.mark.parametrize("n_prompt", [5, 150])
def test_head_dim_128(oracle, gpus, decode_mode, n_prompt):
    """A model with 128-wide heads: prefill and every decoded step against the oracle."""
    g = gpus("tiny-hd128", 512)
    prompt = synth.prompt_ids(g.cfg.vocab, n_prompt, seed=31)
    n = 24
    want_toks, want_logits = oracle.CPU(synth.ensure("tiny-hd128"), 512).generate(prompt, n, step_logits=True)
    toks, logits = g.generate_logits(prompt, n)
    for i in range(n):
        check_step(i, logits[i], want_logits[i])
    assert np.array_equal(toks, want_toks)


@pytest.mark.parametrize("spec,positions", [("tiny-qwen2", 64), ("tiny-qwen2", 96), ("tiny-qwen2", 256),
                                            ("tiny-hd128", 64)])
def test_attention_positions(oracle, spec, positions):
    """The decode kernel's attention items of 64, 96 or 256 positions (knob attn_positions): with the shorter
    ones a head's context spans several items whose partials are merged.  Every step against the oracle."""
    old = llm_b200.get_knob("attn_positions")
    llm_b200.set_knob("attn_positions", positions)
    try:
        g = llm_b200.GPU(synth.ensure(spec), ctx=512)
    finally:
        llm_b200.set_knob("attn_positions", old)
    try:
        prompt = synth.prompt_ids(g.cfg.vocab, 150, seed=positions)
        toks, logits = g.generate_logits(prompt, 40)
    finally:
        g.close()
    want_toks, want_logits = oracle.CPU(synth.ensure(spec), 512).generate(prompt, 40, step_logits=True)
    for i in range(40):
        check_step(i, logits[i], want_logits[i])
    assert np.array_equal(toks, want_toks)


def test_config1_full_workload(oracle, gpus):
    """BASELINE config 1 at full size: 128 prompt tokens, 128 greedy tokens, token-identical."""
    g = gpus("c1-smollm2-q4_0", 512)
    prompt = synth.prompt_ids(g.cfg.vocab, 128, seed=1)
    want = oracle.CPU(synth.ensure("c1-smollm2-q4_0"), 512).generate(prompt, 128)
    got, tm = g.generate(prompt, 128)
    assert np.array_equal(got, want), int(np.argmax(got != want))


def test_config4_full_workload(oracle):
    """BASELINE config 4 at full size: a 512-token prompt through 8 chunks of 64 (Qwen2.5 architecture), then
    16 greedy tokens, token-identical; the last prompt token's logits within 1e-5 relative."""
    path = synth.ensure("c3-qwen2.5-0.5b")
    w = synth.WORKLOADS[4]
    g = llm_b200.GPU(path, ctx=w["ctx"])
    try:
        prompt = synth.prompt_ids(g.cfg.vocab, w["prompt"], seed=4)
        toks, logits = g.generate_logits(prompt, w["gen"])
    finally:
        g.close()
    want_toks, want_logits = oracle.CPU(path, w["ctx"]).generate(prompt, w["gen"], step_logits=True)
    assert rel_err(logits[0], want_logits[0]) <= REL_TOL
    for i in range(w["gen"]):
        check_step(i, logits[i], want_logits[i])
    assert np.array_equal(toks, want_toks)


def test_tag_reset(oracle, gpus):
    """The decode kernel's exchange tags restart (buffers cleared, epoch 0) between launches: tokens unchanged."""
    old = llm_b200.get_knob("tag_reset")
    llm_b200.set_knob("tag_reset", 3)
    try:
        g = gpus("tiny-qwen2", 256)
        prompt = synth.prompt_ids(g.cfg.vocab, 15, seed=9)
        got, _ = g.generate(prompt, 40)
        again, _ = g.generate(prompt, 40)
    finally:
        llm_b200.set_knob("tag_reset", old)
    want = oracle.CPU(synth.ensure("tiny-qwen2"), 256).generate(prompt, 40)
    assert np.array_equal(got, want) and np.array_equal(again, want)


def test_deterministic(gpus):
    g = gpus("tiny-qwen2", 256)
    prompt = synth.prompt_ids(g.cfg.vocab, 40, seed=3)
    a = g.generate_logits(prompt, 10)[1]
    b = g.generate_logits(prompt, 10)[1]
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_eos_and_emit_stop(oracle, gpus):
    """eos stops generation and is not emitted (gpu.go:973-976); emit returning false stops too."""
    g = gpus("tiny-llama", 256)
    prompt = synth.prompt_ids(g.cfg.vocab, 10, seed=11)
    want = oracle.CPU(synth.ensure("tiny-llama"), 256).generate(prompt, 30)
    k = 17
    eos = int(want[k])
    first = int(np.argmax(want == eos))
    got, tm = g.generate(prompt, 30, eos=eos)
    assert np.array_equal(got, want[:first]) and tm.generated == first
    seen = []
    got, _ = g.generate(prompt, 30, emit=lambda t: (seen.append(t), len(seen) < 5)[1])
    assert seen == list(want[:5]) and np.array_equal(got, want[:5])


def test_errors(gpus):
    g = gpus("tiny-llama", 64)
    with pytest.raises(llm_b200.LlmError) as e:
        g.generate(np.arange(60, dtype=np.int32), 10)
    assert e.value.code == llm_b200.ERR_CONTEXT
    with pytest.raises(llm_b200.LlmError) as e:
        g.generate(np.zeros(0, np.int32), 3)
    assert e.value.code == llm_b200.ERR_ARG
    with pytest.raises(llm_b200.LlmError) as e:
        g.prefill_logits(np.array([1, g.cfg.vocab], np.int32))
    assert e.value.code == llm_b200.ERR_ARG
    with pytest.raises(llm_b200.LlmError) as e:
        g.prefill_logits(np.zeros(64, np.int32))
    assert e.value.code == llm_b200.ERR_CONTEXT
    # the largest prompt that fits, and generation up to the last position
    toks, _ = g.generate(np.arange(54, dtype=np.int32), 10)
    assert len(toks) == 10


def test_peek_state_tokens(gpus):
    g = gpus("tiny-llama", 256)
    prompt = synth.prompt_ids(g.cfg.vocab, 9, seed=2)
    got, _ = g.generate(prompt, 7)
    toks = g.peek("tokens", 9 + 7).view(np.int32)
    assert np.array_equal(toks[:9], prompt) and np.array_equal(toks[9:], got)
    state = g.peek("state", 2).view(np.uint32)
    assert state[0] >= 9 + 6 and state[0] == state[1]
    with pytest.raises(llm_b200.LlmError):
        g.peek("nothing", 1)


def test_trace_layers(oracle, gpus):
    """`trace` (main.go:212-240): the residual after 0, 1 and 2 layers against the oracle's LastX."""
    g = gpus("tiny-qwen2", 256)
    path = synth.ensure("tiny-qwen2")
    tok = 123
    try:
        for layers in (-1, 1, 2):
            g.layers = layers
            cpu = oracle.CPU(path, 8)
            cpu.set_max_layers(layers)
            cpu.forward(tok)
            want = cpu.last_x()
            g.prefill_logits(np.array([tok], np.int32))
            got = g.peek("x", g.cfg.embd)
            assert rel_err(got, want) <= REL_TOL, layers
    finally:
        g.layers = 0


def test_memory_budget():
    """Limits.MemoryBudget (gpu.go:175-177): a model larger than the budget is refused."""
    old = llm_b200.get_knob("memory_budget")
    llm_b200.set_knob("memory_budget", 1 << 20)
    try:
        with pytest.raises(llm_b200.LlmError) as e:
            llm_b200.GPU(synth.ensure("tiny-llama"), ctx=64)
        assert e.value.code == llm_b200.ERR_MEMORY
    finally:
        llm_b200.set_knob("memory_budget", old)


def test_reader_callback_matches_path(gpus):
    """llmb_open_reader (an io.ReaderAt, gpu.go:290,365) loads the same model as a path."""
    path = synth.ensure("tiny-mixed")
    data = open(path, "rb").read()
    g2 = llm_b200.GPU(reader=lambda off, n: data[off:off + n], size=len(data), ctx=256)
    try:
        prompt = synth.prompt_ids(g2.cfg.vocab, 12, seed=4)
        a = g2.prefill_logits(prompt)
        b = gpus("tiny-mixed", 256).prefill_logits(prompt)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert g2.memory_used() > 0
    finally:
        g2.close()
