"""Every BASELINE workload at the size the benchmark runs it, token for token
against the CPU oracle (the reference's `check`, examples/generate/main.go
:159-180: identical greedy sequences).

The oracle's tokens come from committed fixtures (tests/golden/parity/,
written by tests/golden/make_parity_fixtures.py; each records the SHA-256 of
the model file it was made from): at these sizes the oracle takes minutes to
hours (workload 5 is ~200K forward passes for eight ranks' streams).

  - workload 1: 128-token prompt + 128 greedy tokens (SmolLM2 arch, Q4_0);
  - workload 2: 32 + 256 (mixed Q4_0 / Q4_1 / Q8_0);
  - workload 3: 128 + 128 (Qwen2.5-0.5B arch, NEOX, biases, Q8_0 head);
  - workload 4: a 512-token prompt in 8 chunks of 64, then 16 tokens;
  - workload 5: each rank's 64 streams (prompts on [16, 512]) through
    llmb_generate_batch, 128 tokens each, every stream against its own
    single-stream oracle run.
For workloads 1-4 the step-1 logits are also checked on the oracle's top 16
(relative to the largest |logit|, as main.go:159-165 defines the error).
"""

import hashlib
import os

import numpy as np
import pytest

import llm_b200
from llm_b200 import synth

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = os.path.join(HERE, "golden", "parity")
REL_TOL = 1e-5
_sha = {}


def load(name, spec):
    path = os.path.join(FIX, name)
    if not os.path.exists(path):
        pytest.skip(f"no fixture {name} (tests/golden/make_parity_fixtures.py writes it)")
    f = np.load(path)
    mp = synth.ensure(spec)
    if mp not in _sha:
        h = hashlib.sha256()
        with open(mp, "rb") as fh:
            for b in iter(lambda: fh.read(1 << 24), b""):
                h.update(b)
        _sha[mp] = h.hexdigest()
    assert str(f["model_sha256"]) == _sha[mp], f"{name} was made from another model file: regenerate it"
    return f


def first_divergence(got, want):
    d = np.nonzero(got[: len(want)] != want[: len(got)])[0]
    return int(d[0]) if len(d) else min(len(got), len(want))


@pytest.mark.parametrize("k", [1, 2, 3, 4])
def test_workload_full_size(k):
    w = synth.WORKLOADS[k]
    f = load(f"c{k}.npz", w["spec"])
    prompt = synth.workload_prompts(k)[0]
    assert np.array_equal(f["prompt"], prompt)
    with llm_b200.GPU(synth.ensure(w["spec"]), ctx=w["ctx"]) as g:
        got, tm = g.generate(prompt, w["gen"])
        logits = g.prefill_logits(prompt)
    want = f["tokens"]
    assert tm.generated == w["gen"]
    assert np.array_equal(got, want), f"first divergence at step {first_divergence(got, want)}"
    top, top_v = f["top_ids"], f["top_logits"]
    rel = float(np.max(np.abs(logits[top].astype(np.float64) - top_v)) / float(f["max_abs_logit"]))
    assert rel <= REL_TOL, rel
    assert int(np.argmax(logits)) == int(top[0])


@pytest.mark.parametrize("rank", range(8))
def test_workload5_streams(rank):
    w = synth.WORKLOADS[5]
    f = load(f"c5_r{rank}.npz", w["spec"])
    prompts = synth.workload_prompts(5, rank)
    assert np.array_equal(f["prompt_lens"], [len(p) for p in prompts])
    with llm_b200.GPU(synth.ensure(w["spec"]), ctx=w["ctx"]) as g:
        outs, tm = g.generate_batch(prompts, w["gen"])
    want = f["tokens"]
    bad = [i for i, (a, b) in enumerate(zip(outs, want)) if not np.array_equal(a, b)]
    assert not bad, [(i, first_divergence(outs[i], want[i])) for i in bad[:8]]
    assert tm.generated == w["streams"] * w["gen"]
