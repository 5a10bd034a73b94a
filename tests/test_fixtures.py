"""The full-size parity fixtures (tests/golden/parity/) against the CPU oracle, on CPU.

The GPU tests and bench.py compare the CUDA path's greedy tokens at the
benchmark sizes with these files; here each file is checked against what it
claims to be: the prompt the benchmark runs, the model file it was made from
(SHA-256), and a prefix of its tokens recomputed by the oracle (the whole
sequences take the oracle minutes to hours; tests/golden/make_parity_fixtures.py
regenerates them).
"""

import hashlib
import os

import numpy as np
import pytest

from llm_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = os.path.join(HERE, "golden", "parity")
_sha = {}


def sha256(path):
    if path not in _sha:
        h = hashlib.sha256()
        with open(path, "rb") as f:
            for b in iter(lambda: f.read(1 << 24), b""):
                h.update(b)
        _sha[path] = h.hexdigest()
    return _sha[path]


@pytest.mark.parametrize("k,prefix", [(1, 4), (2, 8), (3, 2), (4, 1)])
def test_workload_fixture(oracle, k, prefix):
    w = synth.WORKLOADS[k]
    f = np.load(os.path.join(FIX, f"c{k}.npz"))
    path = synth.ensure(w["spec"])
    assert str(f["model_sha256"]) == sha256(path)
    prompt = synth.workload_prompts(k)[0]
    assert np.array_equal(f["prompt"], prompt)
    assert len(f["tokens"]) == w["gen"] and int(f["gen"]) == w["gen"] and int(f["ctx"]) == w["ctx"]
    if k == 4:
        # the 512-token prompt is the benchmark's prefill case; its first 128 ids are config 3's prompt
        assert np.array_equal(prompt[:128], synth.workload_prompts(3)[0])
        return
    toks, logits = oracle.CPU(path, w["ctx"]).generate(prompt, prefix, step_logits=True)
    assert np.array_equal(toks, f["tokens"][:prefix])
    top = f["top_ids"]
    assert np.array_equal(logits[0][top].view(np.uint32), f["top_logits"].view(np.uint32))
    assert float(np.abs(logits[0]).max()) == float(f["max_abs_logit"])


def test_workload5_fixtures(oracle):
    w = synth.WORKLOADS[5]
    path = synth.ensure(w["spec"])
    cpu = oracle.CPU(path, w["ctx"])
    for rank in range(8):
        f = np.load(os.path.join(FIX, f"c5_r{rank}.npz"))
        assert str(f["model_sha256"]) == sha256(path) and int(f["rank"]) == rank
        prompts = synth.workload_prompts(5, rank)
        assert np.array_equal(f["prompt_lens"], [len(p) for p in prompts])
        assert f["tokens"].shape == (w["streams"], w["gen"])
        lens = [len(p) for p in prompts]
        assert min(lens) >= w["prompt_range"][0] and max(lens) <= w["prompt_range"][1]
        i = int(np.argmin(lens))  # the shortest stream: its first tokens from the oracle
        assert np.array_equal(cpu.generate(prompts[i], 4), f["tokens"][i, :4])
