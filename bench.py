#!/usr/bin/env python
"""Decode / prefill throughput of the B200 forward pass.

One step is one ``Generate`` of config 1 (SmolLM2-135M architecture, Q4_0,
seeded synthetic GGUF): a 128-token prompt, then 128 greedy tokens, context
512 -- one round of the reference's ``bench`` (examples/generate/main.go
:183-207). ``value`` is decode tok/s: tokens produced by decode launches over
the device time of the decode loop (CUDA events on the library's stream,
weights and prompt already in HBM), summed over GPUs, each GPU running its own
sequence (weak scaling, no collective). ``e2e`` is the same metric through
the C ABI call with host buffers (prompt in, tokens out), by wall clock.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import os
import re
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from llm_b200 import synth  # noqa: E402

METRIC = "decode/prefill tok/s per B200, SmolLM2-135M-arch Q4_0; box total at 1-8 GPUs"
CFG = synth.WORKLOADS[1]
SPEC, NP, NGEN, CTX = CFG["spec"], CFG["prompt"], CFG["gen"], CFG["ctx"]
DECODED = NGEN - 1  # the first generated token is sampled by the prefill
FALLBACK_HBM_GBS = 6650.0


def config_block(extra=None):
    c = {"workload": f"config 1: {SPEC.name} seed {SPEC.seed} (SmolLM2-135M architecture, Q4_0, tied output), "
                     f"{NP}-token prompt + {NGEN} greedy tokens, ctx {CTX}, batch 1",
         "model": "SmolLM2-135M-arch (synthetic weights)", "global_batch": 1, "seq_len": NP + NGEN,
         "parallelism": "independent sequence per GPU (no collective)", "seed": SPEC.seed,
         "l2": "flushed between steps (256 MiB write); within a step every token re-reads the weights "
               "the previous token left in L2, as the workload does"}
    if extra:
        c.update(extra)
    return c


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    return ws, rank, local


def all_max(vals, ws):
    if ws == 1:
        return list(vals)
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(vals), dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def all_sum(vals, ws):
    if ws == 1:
        return list(vals)
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(vals), dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


class Clocks:
    """nvidia-smi samples during the timed region (SM clock and throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.p:
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                self.out = ""

    def summary(self):
        rows = [r for r in csv.reader(io.StringIO(self.out)) if len(r) >= 9]
        rows = [[c.strip() for c in r] for r in rows if r[0].strip().isdigit() and int(r[0]) in self.gpus]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": FALLBACK_HBM_GBS}, "fallback"


def profiled_traffic():
    """DRAM bytes per k_decode launch from the committed ncu summary (None if absent)."""
    p = os.path.join(ROOT, "profiles", "k_decode_c1.md")
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.e+]+)", open(p).read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


def kv_bytes(p0, n):
    """KV cache bytes the tokens at positions p0..p0+n-1 read (all cached positions, K and V)."""
    per = synth.kv_bytes_per_position(SPEC)
    return sum(per * (p + 1) for p in range(p0, p0 + n))


def cpu_baseline(threads=1, prompt_len=32, gen=64):
    """The oracle (C restatement of the reference's cpu.go) on a bounded sample of config 1."""
    from oracle import oracle

    oracle.set_threads(threads)
    cpu = oracle.CPU(synth.ensure(SPEC), CTX)
    prompt = synth.prompt_ids(SPEC.vocab, prompt_len, seed=SPEC.seed)
    t0 = time.perf_counter()
    for t in prompt:
        logits = cpu.forward(int(t))
    t1 = time.perf_counter()
    tok = oracle.argmax(logits)
    for _ in range(gen):
        tok = oracle.argmax(cpu.forward(tok))
    t2 = time.perf_counter()
    return {"value": gen / (t2 - t1), "prefill_tok_s": prompt_len / (t1 - t0), "unit": "tok/s", "cores": threads,
            "kind": "port",
            "sample": f"config 1 weights, {prompt_len}-token prompt then {gen} greedy tokens (positions 0..{prompt_len + gen - 1} "
                      f"of the {NP + NGEN}-position workload); C restatement of the reference cpu.go, "
                      f"{threads} thread(s), {os.cpu_count()} host cores"}


def run_reference(args, ws, rank):
    """`--impl reference`: the reference's CPU path (the oracle port; Go cannot run here) on the host cores."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    from oracle import oracle

    oracle.set_threads(threads)
    cpu = oracle.CPU(synth.ensure(SPEC), CTX)
    prompt = synth.prompt_ids(SPEC.vocab, 16, seed=SPEC.seed)
    gen = 16
    dec_s, pre_s = [], []
    for i in range(args.warmup + args.steps):
        cpu.reset()
        t0 = time.perf_counter()
        for t in prompt:
            logits = cpu.forward(int(t))
        t1 = time.perf_counter()
        tok = oracle.argmax(logits)
        for _ in range(gen):
            tok = oracle.argmax(cpu.forward(tok))
        t2 = time.perf_counter()
        if i >= args.warmup:
            pre_s.append(t1 - t0)
            dec_s.append(t2 - t1)
    value = gen * len(dec_s) / sum(dec_s)
    sample = (f"config 1 weights, each step a 16-token prompt then {gen} greedy tokens; C restatement of the "
              f"reference cpu.go (Go is not installed), {threads} threads over the matrix rows")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * (sum(dec_s) + sum(pre_s)) / len(dec_s),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block({"reference_sample": sample}),
        "prefill_tok_s": 16 * len(pre_s) / sum(pre_s),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


C5 = synth.WORKLOADS[5]


def c5_prompts(vocab, rank):
    """Config 5's prompts for one GPU: lengths uniform on the range, uniform ids (seeded per rank)."""
    import numpy as np

    rng = np.random.default_rng(5000 + rank)
    lo, hi = C5["prompt_range"]
    lens = rng.integers(lo, hi + 1, C5["streams"])
    return [synth.prompt_ids(vocab, int(n), seed=10000 * (rank + 1) + i) for i, n in enumerate(lens)]


def run_multi_stream(args, ws, rank, local):
    """Config 5: 64 independent sequences per GPU through llmb_generate_batch; box-total decode tok/s."""
    import torch

    import llm_b200

    g = llm_b200.GPU(synth.ensure(C5["spec"]), ctx=C5["ctx"], device=local)
    prompts = c5_prompts(g.cfg.vocab, rank)
    ngen = args.c5_gen or C5["gen"]
    g.generate_batch(prompts, ngen)  # warm-up (allocates the KV arena)
    torch.cuda.synchronize()
    barrier(ws)
    rounds = max(1, args.c5_rounds)
    dec = pre = 0.0
    gen = ptoks = launches = 0
    for _ in range(rounds):
        outs, tm = g.generate_batch(prompts, ngen)
        dec += tm.gpu_decode_ms
        pre += tm.gpu_prefill_ms
        gen += tm.generated - len(prompts)  # the first token of each sequence is sampled by the prefill
        ptoks += tm.prompt_tokens
        launches += tm.dispatches
    torch.cuda.synchronize()
    barrier(ws)
    g.close()
    mdec, mpre = all_max([dec, pre], ws)
    tgen, tpro, tl = all_sum([gen, ptoks, launches], ws)
    return {"workload": f"config 5: {C5['streams']} sequences per GPU on {C5['spec'].name}, prompts uniform on "
                        f"{list(C5['prompt_range'])}, {ngen} greedy tokens each, ctx {C5['ctx']}",
            "decode_tok_s": tgen / (mdec / 1000.0), "prefill_tok_s": tpro / (mpre / 1000.0), "unit": "tok/s",
            "rounds": rounds, "decode_ms_per_round": mdec / rounds, "prefill_ms_per_round": mpre / rounds,
            "gpu_launches": int(tl), "timing": "CUDA events on the library stream, max over ranks; box total"}


def run_other_configs(local):
    """Configs 2-4 once each (after a warm-up run): decode and prefill tok/s by CUDA events, one GPU."""
    import llm_b200

    out = {}
    for k in (2, 3, 4):
        w = synth.WORKLOADS[k]
        g = llm_b200.GPU(synth.ensure(w["spec"]), ctx=w["ctx"], device=local)
        prompt = synth.prompt_ids(g.cfg.vocab, w["prompt"], seed=w["spec"].seed)
        g.generate(prompt, w["gen"])
        _, tm = g.generate(prompt, w["gen"])
        g.close()
        out[f"config{k}"] = {"workload": f"{w['spec'].name}: {w['prompt']}-token prompt + {w['gen']} greedy tokens, "
                                         f"ctx {w['ctx']}",
                             "decode_tok_s": (tm.generated - 1) / (tm.gpu_decode_ms / 1000.0) if tm.generated > 1 else None,
                             "prefill_tok_s": tm.prompt_tokens / (tm.gpu_prefill_ms / 1000.0), "unit": "tok/s"}
    return out


def run_ours(args, ws, rank, local):
    import torch

    import llm_b200

    torch.cuda.set_device(local)
    path = synth.ensure(SPEC)
    g = llm_b200.GPU(path, ctx=CTX, device=local)
    prompt = synth.prompt_ids(g.cfg.vocab, NP, seed=SPEC.seed)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=f"cuda:{local}")
    for _ in range(args.warmup):
        g.generate(prompt, NGEN)
    barrier(ws)
    torch.cuda.synchronize()
    acc = dict(dec=0.0, pre=0.0, kern=0.0, launches=0, wall_dec=0.0, wall_pre=0.0, dispatches=0, gen=0)
    with Clocks(list(range(torch.cuda.device_count())) if rank == 0 else []) as clk:
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            toks, tm = g.generate(prompt, NGEN)
            assert tm.generated == NGEN
            acc["dec"] += tm.gpu_decode_ms
            acc["pre"] += tm.gpu_prefill_ms
            acc["kern"] += tm.decode_kernel_ms
            acc["launches"] += tm.decode_launches
            acc["wall_dec"] += tm.decode_ms
            acc["wall_pre"] += tm.prefill_ms
            acc["dispatches"] += tm.dispatches
        torch.cuda.synchronize()
        barrier(ws)
    mx = dict(zip(["dec", "pre", "kern", "wall_dec", "wall_pre"],
                  all_max([acc["dec"], acc["pre"], acc["kern"], acc["wall_dec"], acc["wall_pre"]], ws)))
    launches_total, dispatches_total = all_sum([acc["launches"], acc["dispatches"]], ws)
    g.close()
    multi = None if args.no_multi_stream else run_multi_stream(args, ws, rank, local)
    if rank != 0:
        return
    others = run_other_configs(local) if (ws == 1 and not args.no_other_configs) else None
    K = args.steps
    value = ws * K * DECODED / (mx["dec"] / 1000.0)
    prefill = ws * K * NP / (mx["pre"] / 1000.0)
    e2e = ws * K * DECODED / (mx["wall_dec"] / 1000.0)
    # roofline of the persistent decode kernel: algorithmic bytes per launch / its event-timed duration
    weights = synth.algorithmic_bytes_per_token(SPEC)
    per_step_bytes = DECODED * weights + kv_bytes(NP, DECODED)
    launches_per_step = acc["launches"] / K
    bytes_per_launch = per_step_bytes / launches_per_step
    launch_ms = acc["kern"] / acc["launches"]
    achieved = bytes_per_launch / (launch_ms / 1000.0) / 1e9
    peaks, kind = measured_peaks()
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    cpu = cpu_baseline() if (ws == 1 and not args.no_cpu_baseline) else None
    out = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": args.warmup,
        "ms_per_step": (mx["dec"] + mx["pre"]) / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF and uniform-random prompt ids)",
        "config": config_block({"decode_batch": llm_b200.get_knob("decode_batch"),
                                "prefill_batch": llm_b200.get_knob("prefill_batch"),
                                "decode_tokens_per_step": DECODED}),
        "prefill_tok_s": prefill,
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 * NP + 8,
                "d2h_bytes_per_step": 4 * NGEN + 4 * int(1 + launches_per_step)},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"hbm_gbs of {kind}", "traffic": profiled_traffic(),
                     "kernel": "k_decode (persistent decode kernel, one launch per DecodeBatch tokens)",
                     "bytes_per_launch": bytes_per_launch, "launch_ms": launch_ms},
        "gpu_launches": int(dispatches_total),
        "clocks": clk.summary(),
    }
    if cpu:
        out["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if multi:
        out["multi_stream"] = multi
    if others:
        out["other_configs"] = others
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-multi-stream", action="store_true", help="skip the config 5 (64-sequence) measurement")
    ap.add_argument("--no-other-configs", action="store_true", help="skip the single runs of configs 2-4 (N=1 only)")
    ap.add_argument("--c5-rounds", type=int, default=1, help="timed rounds of config 5")
    ap.add_argument("--c5-gen", type=int, default=0, help="greedy tokens per config 5 sequence (0: the workload's 128)")
    ap.add_argument("--only-multi-stream", action="store_true",
                    help="run only the config 5 measurement and print its object (a profiling aid)")
    args = ap.parse_args()
    ws, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, ws, rank)
        elif args.only_multi_stream:
            import torch

            torch.cuda.set_device(local)
            multi = run_multi_stream(args, ws, rank, local)
            if rank == 0:
                print(json.dumps({"multi_stream": multi}), flush=True)
        else:
            run_ours(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
