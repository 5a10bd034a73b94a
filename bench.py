#!/usr/bin/env python
"""Decode / prefill throughput of the B200 forward pass.

One step is one ``Generate`` of config 1 (SmolLM2-135M architecture, Q4_0,
seeded synthetic GGUF): a 128-token prompt, then 128 greedy tokens, context
512 -- one round of the reference's ``bench`` (examples/generate/main.go
:183-207). ``value`` is decode tok/s: tokens produced by decode launches over
the device time of the decode loop (CUDA events on the library's stream,
weights and prompt already in HBM), summed over GPUs, each GPU running its own
sequence (weak scaling, no collective). ``e2e`` is the whole ``Generate`` call
through the C ABI with host buffers: the 128 generated tokens over the wall
time of the call (prompt upload, prefill, decode launches, token read-back).
Every configuration's greedy tokens are compared with the CPU oracle's
(fixtures made by tests/golden/make_parity_fixtures.py): ``parity``.

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


FIXTURES = os.path.join(ROOT, "tests", "golden", "parity")
_sha = {}


def fixture(k, rank=0):
    """The oracle's greedy tokens for workload k (rank's streams for k = 5), or (None, why)."""
    import hashlib

    import numpy as np

    name = f"c{k}.npz" if k != 5 else f"c5_r{rank}.npz"
    try:
        f = np.load(os.path.join(FIXTURES, name))
    except OSError:
        return None, f"no fixture {name}"
    path = synth.ensure(synth.WORKLOADS[k]["spec"])
    if path not in _sha:
        h = hashlib.sha256()
        with open(path, "rb") as fh:
            for b in iter(lambda: fh.read(1 << 24), b""):
                h.update(b)
        _sha[path] = h.hexdigest()
    if str(f["model_sha256"]) != _sha[path]:
        return None, f"fixture {name} was made from another model file"
    return f["tokens"], None


def parity_of(k, got, rank=0):
    """True/False: got (tokens, or the list of each stream's) equals the oracle's fixture; None if none applies."""
    import numpy as np

    want, why = fixture(k, rank)
    if want is None:
        return None, why
    if k == 5:
        return bool(len(got) == len(want) and all(np.array_equal(g, w) for g, w in zip(got, want))), None
    return bool(np.array_equal(got, want)), None


def decode_bytes(spec, starts, ntok):
    """Algorithmic bytes of decoding ntok tokens from each start position (weights once per token and
    sequence, plus every cached position's K and V read)."""
    w = synth.algorithmic_bytes_per_token(spec)
    per = synth.kv_bytes_per_position(spec)
    return sum(ntok * w + per * sum(p + 1 for p in range(p0, p0 + ntok)) for p0 in starts)


def hbm_roofline(achieved_gbs):
    peaks, kind = measured_peaks()
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    return {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s", "frac": achieved_gbs / peak,
            "peak_source": f"hbm_gbs of {kind}"}


# FP32 CUDA-core peak (no measured figure exists for it): 148 SMs x 128 lanes x 2 flops x 1.965 GHz.
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def prefill_flops(spec, n):
    """Flops of a prompt of n tokens: 2 per weight element per token in the layers, plus causal attention
    (q.k and the V sum, 4 * heads * head_dim per cached position) and one head product."""
    layer = 0
    for name, dims, ty, _, _ in synth.header(spec)[1]:
        if name.startswith("blk.") and len(dims) == 2:
            layer += dims[0] * dims[1]
    att = 4 * spec.heads * spec.head_dim * spec.layers * sum(p + 1 for p in range(n))
    return 2 * layer * n + att + 2 * spec.embd * spec.vocab


def oracle_generate(cpu, oracle, prompt, gen):
    """One greedy Generate of the CPU oracle: (tokens, prefill seconds, decode seconds).  The prompt's forward
    passes sample the first token; each of the other gen - 1 tokens takes one more forward pass."""
    cpu.reset()
    t0 = time.perf_counter()
    for t in prompt:
        logits = cpu.forward(int(t))
    t1 = time.perf_counter()
    toks = [oracle.argmax(logits)]
    for _ in range(gen - 1):
        toks.append(oracle.argmax(cpu.forward(toks[-1])))
    t2 = time.perf_counter()
    return toks, t1 - t0, t2 - t1


def cpu_baseline(threads=1):
    """The oracle (C restatement of the reference's cpu.go, single-threaded as cpu.go is) on config 1's
    whole workload, once: decode tok/s over the same 127 decoded tokens as the GPU's value."""
    from oracle import oracle

    oracle.set_threads(threads)
    cpu = oracle.CPU(synth.ensure(SPEC), CTX)
    prompt = synth.workload_prompts(1)[0]
    _, pre, dec = oracle_generate(cpu, oracle, prompt, NGEN)
    return {"value": DECODED / dec, "prefill_tok_s": NP / pre, "e2e_tok_s": NGEN / (pre + dec), "unit": "tok/s",
            "cores": threads, "kind": "port",
            "sample": f"config 1 whole workload once ({NP}-token prompt, {NGEN} greedy tokens, ctx {CTX}); "
                      f"C restatement of the reference cpu.go, {threads} thread(s) of {os.cpu_count()} host cores"}


def run_reference(args, ws, rank):
    """`--impl reference`: the reference's CPU path (the oracle port; Go cannot run here) on the host cores,
    on the same workload as our arm: each step one Generate of config 1 (128-token prompt, 128 greedy
    tokens, ctx 512).  value = decode tok/s (127 decoded tokens per step over their time), e2e = 128
    generated tokens over the whole call, as our arm's."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    from oracle import oracle

    oracle.set_threads(threads)
    cpu = oracle.CPU(synth.ensure(SPEC), CTX)
    prompt = synth.workload_prompts(1)[0]
    dec_s, pre_s, par = [], [], []
    for i in range(args.warmup + args.steps):
        toks, pre, dec = oracle_generate(cpu, oracle, prompt, NGEN)
        if i >= args.warmup:
            pre_s.append(pre)
            dec_s.append(dec)
        par.append(parity_of(1, np_array(toks))[0])
    value = DECODED * len(dec_s) / sum(dec_s)
    e2e = NGEN * len(dec_s) / (sum(dec_s) + sum(pre_s))
    sample = (f"config 1 whole workload per step ({NP}-token prompt, {NGEN} greedy tokens, ctx {CTX}); C restatement "
              f"of the reference cpu.go (Go is not installed), {threads} threads over the matrix rows")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * (sum(dec_s) + sum(pre_s)) / len(dec_s),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block({"decode_tokens_per_step": DECODED}),
        "prefill_tok_s": NP * len(pre_s) / sum(pre_s),
        "parity": all(p is True for p in par),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                "what": "128 generated tokens over the wall time of the whole Generate (prefill + decode)"},
    }), flush=True)


def np_array(toks):
    import numpy as np

    return np.asarray(toks, np.int32)


C5 = synth.WORKLOADS[5]


def c5_prompts(rank):
    """Config 5's prompts for one GPU (synth.workload_prompts)."""
    return synth.workload_prompts(5, rank)


def run_multi_stream(args, ws, rank, local):
    """Config 5: 64 independent sequences per GPU through llmb_generate_batch; box-total decode tok/s, each
    rank's streams compared with the oracle's fixture, and the decode's HBM roofline (the weights once per
    decode step for all streams, plus every stream's KV reads)."""
    import torch

    import llm_b200

    g = llm_b200.GPU(synth.ensure(C5["spec"]), ctx=C5["ctx"], device=local)
    prompts = c5_prompts(rank)
    ngen = args.c5_gen or C5["gen"]
    g.generate_batch(prompts, ngen)  # warm-up (allocates the KV arena)
    torch.cuda.synchronize()
    barrier(ws)
    rounds = max(1, args.c5_rounds)
    dec = pre = 0.0
    gen = ptoks = launches = 0
    ok = []
    for _ in range(rounds):
        outs, tm = g.generate_batch(prompts, ngen)
        dec += tm.gpu_decode_ms
        pre += tm.gpu_prefill_ms
        gen += tm.generated - len(prompts)  # the first token of each sequence is sampled by the prefill
        ptoks += tm.prompt_tokens
        launches += tm.dispatches
        ok.append(parity_of(5, outs, rank)[0] if ngen == C5["gen"] else None)
    torch.cuda.synchronize()
    barrier(ws)
    g.close()
    n_true = sum(1 for o in ok if o is True)
    n_none = sum(1 for o in ok if o is None)
    # the weights cross HBM once per decode step for all streams; each stream reads its own KV rows
    starts = [len(p) for p in prompts]
    nbytes = rounds * (decode_bytes(C5["spec"], starts, ngen - 1)
                       - (len(starts) - 1) * (ngen - 1) * synth.algorithmic_bytes_per_token(C5["spec"]))
    mdec, mpre = all_max([dec, pre], ws)
    tgen, tpro, tl, tt, tn, tb = all_sum([gen, ptoks, launches, n_true, n_none, nbytes], ws)
    parity = None if tn > 0 else bool(tt == ws * rounds)
    flops = all_sum([rounds * sum(prefill_flops(C5["spec"], len(p)) - 2 * C5["spec"].embd * C5["spec"].vocab
                                  for p in prompts)], ws)[0]
    return {"workload": f"config 5: {C5['streams']} sequences per GPU on {C5['spec'].name}, prompts uniform on "
                        f"{list(C5['prompt_range'])}, {ngen} greedy tokens each, ctx {C5['ctx']}",
            "decode_tok_s": tgen / (mdec / 1000.0), "prefill_tok_s": tpro / (mpre / 1000.0), "unit": "tok/s",
            "rounds": rounds, "decode_ms_per_round": mdec / rounds, "prefill_ms_per_round": mpre / rounds,
            "parity": parity,
            "roofline": dict(hbm_roofline(tb / ws / (mdec / 1000.0) / 1e9),
                             bytes_per_round_per_gpu=tb / ws / rounds,
                             what="decode: weights once per step (all streams share them) + every stream's KV reads"),
            "prefill_roofline": fp32_roofline(flops / ws / (mpre / 1000.0) / 1e12),
            "gpu_launches": int(tl), "timing": "CUDA events on the library stream, max over ranks; box total"}


def fp32_roofline(achieved_tflops):
    return {"bound": "fp32", "achieved": achieved_tflops, "peak": FP32_NOMINAL_TFLOPS, "unit": "TFLOP/s",
            "frac": achieved_tflops / FP32_NOMINAL_TFLOPS,
            "peak_source": "nominal FP32 (148 SMs x 128 lanes x 2 x 1.965 GHz; no measured FP32 peak)"}


def run_other_configs(local, ks=(2, 3, 4)):
    """Configs 2-4 (or those of ks) once each (after a warm-up run): decode and prefill tok/s by CUDA events,
    one GPU, tokens against the oracle's fixture, and the decode's HBM roofline (prefill's FP32 roofline)."""
    import llm_b200

    out = {}
    for k in ks:
        w = synth.WORKLOADS[k]
        g = llm_b200.GPU(synth.ensure(w["spec"]), ctx=w["ctx"], device=local)
        prompt = synth.workload_prompts(k)[0]
        g.generate(prompt, w["gen"])
        toks, tm = g.generate(prompt, w["gen"])
        g.close()
        par, why = parity_of(k, toks)
        dec_s, pre_s = tm.gpu_decode_ms / 1000.0, tm.gpu_prefill_ms / 1000.0
        o = {"workload": f"{w['spec'].name}: {w['prompt']}-token prompt + {w['gen']} greedy tokens, ctx {w['ctx']}",
             "decode_tok_s": (tm.generated - 1) / dec_s if tm.generated > 1 else None,
             "prefill_tok_s": tm.prompt_tokens / pre_s, "unit": "tok/s", "parity": par,
             "roofline": hbm_roofline(decode_bytes(w["spec"], [w["prompt"]], w["gen"] - 1) / dec_s / 1e9),
             "prefill_roofline": fp32_roofline(prefill_flops(w["spec"], w["prompt"]) / pre_s / 1e12)}
        if why:
            o["parity_note"] = why
        out[f"config{k}"] = o
    return out


def run_ours(args, ws, rank, local):
    import torch

    import llm_b200

    torch.cuda.set_device(local)
    path = synth.ensure(SPEC)
    g = llm_b200.GPU(path, ctx=CTX, device=local)
    prompt = synth.workload_prompts(1)[0]
    flush = torch.empty(64 << 20, dtype=torch.float32, device=f"cuda:{local}")
    for _ in range(args.warmup):
        g.generate(prompt, NGEN)
    barrier(ws)
    torch.cuda.synchronize()
    acc = dict(dec=0.0, pre=0.0, kern=0.0, launches=0, wall=0.0, dispatches=0, gen=0, ok=0)
    with Clocks(list(range(torch.cuda.device_count())) if rank == 0 else []) as clk:
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            toks, tm = g.generate(prompt, NGEN)  # the public call: host prompt in, host tokens out
            acc["wall"] += time.perf_counter() - t0
            assert tm.generated == NGEN
            acc["dec"] += tm.gpu_decode_ms
            acc["pre"] += tm.gpu_prefill_ms
            acc["kern"] += tm.decode_kernel_ms
            acc["launches"] += tm.decode_launches
            acc["dispatches"] += tm.dispatches
            acc["ok"] += int(parity_of(1, toks)[0] is True)
        torch.cuda.synchronize()
        barrier(ws)
    mx = dict(zip(["dec", "pre", "kern", "wall"], all_max([acc["dec"], acc["pre"], acc["kern"], acc["wall"]], ws)))
    launches_total, dispatches_total, ok_total = all_sum([acc["launches"], acc["dispatches"], acc["ok"]], ws)
    g.close()
    multi = None if args.no_multi_stream else run_multi_stream(args, ws, rank, local)
    if rank != 0:
        return
    others = run_other_configs(local) if (ws == 1 and not args.no_other_configs) else None
    K = args.steps
    value = ws * K * DECODED / (mx["dec"] / 1000.0)
    prefill = ws * K * NP / (mx["pre"] / 1000.0)
    e2e = ws * K * NGEN / mx["wall"]
    # roofline of the persistent decode kernel: algorithmic bytes per launch / its event-timed duration
    per_step_bytes = decode_bytes(SPEC, [NP], DECODED)
    launches_per_step = acc["launches"] / K
    bytes_per_launch = per_step_bytes / launches_per_step
    launch_ms = acc["kern"] / acc["launches"]
    achieved = bytes_per_launch / (launch_ms / 1000.0) / 1e9
    par_note = parity_of(1, np_array([0]))[1]
    cpu = cpu_baseline() if (ws == 1 and not args.no_cpu_baseline) else None
    out = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": args.warmup,
        "ms_per_step": (mx["dec"] + mx["pre"]) / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF and uniform-random prompt ids)",
        "config": config_block({"decode_batch": llm_b200.get_knob("decode_batch"),
                                "prefill_batch": llm_b200.get_knob("prefill_batch"),
                                "decode_tokens_per_step": DECODED}),
        "prefill_tok_s": prefill,
        "parity": None if par_note else bool(ok_total == ws * K),
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 * NP + 8,
                "d2h_bytes_per_step": 4 * NGEN + 4 * int(1 + launches_per_step),
                "what": "128 generated tokens over the wall time of the whole llmb_generate call (prompt upload, "
                        "prefill, decode launches, token read-back), max over ranks"},
        "roofline": dict(hbm_roofline(achieved), traffic=profiled_traffic(),
                         kernel="k_decode2 (persistent decode kernel, one launch per DecodeBatch tokens)",
                         bytes_per_launch=bytes_per_launch, launch_ms=launch_ms),
        "prefill_roofline": fp32_roofline(prefill_flops(SPEC, NP) * ws * K / (mx["pre"] / 1000.0) / 1e12 / ws),
        "gpu_launches": int(dispatches_total),
        "clocks": clk.summary(),
    }
    if par_note:
        out["parity_note"] = par_note
    if cpu:
        out["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        out["cpu_baseline"]["e2e_tok_s"] = cpu["e2e_tok_s"]
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
    ap.add_argument("--only-config", type=int, choices=[2, 3, 4], default=0,
                    help="run only this config's single-stream measurement and print its object (a profiling aid)")
    ap.add_argument("--knob", action="append", default=[], metavar="NAME=VALUE",
                    help="set a package knob before any model opens (e.g. decode_mode=1 times the per-phase "
                         "kernels, prefill_mode=2 the FP32 products)")
    args = ap.parse_args()
    if args.knob and args.impl == "ours":
        import llm_b200

        for kv in args.knob:
            name, _, val = kv.partition("=")
            llm_b200.set_knob(name, int(val))
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
        elif args.only_config:
            import torch

            torch.cuda.set_device(local)
            if rank == 0:
                print(json.dumps({"other_configs": run_other_configs(local, (args.only_config,))}), flush=True)
        else:
            run_ours(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
