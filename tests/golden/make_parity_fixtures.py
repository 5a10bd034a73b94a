#!/usr/bin/env python
"""Writes the full-size parity fixtures: the CPU oracle's greedy tokens for
every BASELINE workload, at the sizes the benchmark runs them.

TEST INFRASTRUCTURE. The oracle (oracle/cpu_ref.c, the C restatement of the
reference's CPU forward pass, cpu.go:225-397) runs each workload's seeded
prompts through the seeded synthetic model, and the greedy token ids are
saved, as the reference's `check` command compares greedy sequences
(examples/generate/main.go:159-180):

    parity/c1.npz .. c4.npz   workloads 1-4: prompt, tokens, step-1 top-16
    parity/c5_r{R}.npz        workload 5, rank R's 64 streams: prompt
                              lengths, tokens [64, 128]

Each file records the SHA-256 of the model file it was made from, so a test
can tell a stale fixture from a wrong result. The GPU tests
(tests/test_gpu_fixtures.py) and bench.py compare against these files; the
oracle is too slow to rerun at full size there (config 5 is ~200K forward
passes for eight ranks).

    python tests/golden/make_parity_fixtures.py [--workloads 1 2 3 4 5]
        [--ranks 0 1 ...] [--procs N]

Sequences run in parallel processes (spawn), one oracle thread each.
"""

from __future__ import annotations

import argparse
import hashlib
import multiprocessing as mp
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "parity")
sys.path.insert(0, ROOT)


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 24), b""):
            h.update(b)
    return h.hexdigest()


def _job(args):
    """One greedy sequence on the oracle: (key, tokens, step-1 logits top-16 or None)."""
    key, path, ctx, prompt, n, want_top = args
    from oracle import oracle

    oracle.set_threads(1)
    cpu = _job.cache.get(path)
    if cpu is None:
        cpu = _job.cache[path] = oracle.CPU(path, ctx)
    if want_top:
        toks, logits = cpu.generate(prompt, n, step_logits=True)
        first = logits[0]
        top = np.argsort(-first.astype(np.float64), kind="stable")[:16]
        return key, toks, (top.astype(np.int32), first[top].astype(np.float32), float(np.abs(first).max()))
    return key, cpu.generate(prompt, n), None


_job.cache = {}


def main():
    from llm_b200 import synth

    ap = argparse.ArgumentParser()
    ap.add_argument("--workloads", type=int, nargs="*", default=[1, 2, 3, 4, 5])
    ap.add_argument("--ranks", type=int, nargs="*", default=list(range(8)))
    ap.add_argument("--procs", type=int, default=os.cpu_count() or 1)
    a = ap.parse_args()
    os.makedirs(OUT, exist_ok=True)
    jobs, meta = [], {}
    for k in a.workloads:
        w = synth.WORKLOADS[k]
        path = synth.ensure(w["spec"])
        meta[k] = dict(spec=w["spec"].name, seed=w["spec"].seed, model_sha256=sha256(path), ctx=w["ctx"],
                       gen=w["gen"], path=path)
        if k != 5:
            p = synth.workload_prompts(k)[0]
            jobs.append(((k, 0, 0), path, w["ctx"], p, w["gen"], True))
        else:
            for r in a.ranks:
                for i, p in enumerate(synth.workload_prompts(5, r)):
                    jobs.append(((5, r, i), path, w["ctx"], p, w["gen"], False))
    # longest first, so the pool's tail is short
    jobs.sort(key=lambda j: -(len(j[3]) + j[4]) * (4 if j[0][0] in (3, 4) else 1))
    res = {}
    t0 = time.time()
    with mp.get_context("spawn").Pool(a.procs) as pool:
        for i, (key, toks, top) in enumerate(pool.imap_unordered(_job, jobs)):
            res[key] = (toks, top)
            if (i + 1) % 16 == 0 or i + 1 == len(jobs):
                print(f"{i + 1}/{len(jobs)} sequences, {time.time() - t0:.0f} s", flush=True)
    for k in a.workloads:
        m = meta[k]
        common = dict(spec=np.array(m["spec"]), seed=np.int32(m["seed"]), model_sha256=np.array(m["model_sha256"]),
                      ctx=np.int32(m["ctx"]), gen=np.int32(m["gen"]))
        if k != 5:
            toks, (ti, tv, amax) = res[(k, 0, 0)]
            np.savez_compressed(os.path.join(OUT, f"c{k}.npz"), prompt=synth.workload_prompts(k)[0],
                                tokens=np.asarray(toks, np.int32), top_ids=ti, top_logits=tv,
                                max_abs_logit=np.float32(amax), **common)
        else:
            for r in a.ranks:
                ps = synth.workload_prompts(5, r)
                toks = np.stack([np.asarray(res[(5, r, i)][0], np.int32) for i in range(len(ps))])
                np.savez_compressed(os.path.join(OUT, f"c5_r{r}.npz"),
                                    prompt_lens=np.array([len(p) for p in ps], np.int32), tokens=toks,
                                    rank=np.int32(r), **common)
    print("wrote", sorted(os.listdir(OUT)))


if __name__ == "__main__":
    main()
