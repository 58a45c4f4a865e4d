#!/usr/bin/env python3
"""bench.py -- B200 benchmark of the Effort-style dynamic-sparse decode path.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload decode|bucketmul|prefill] [--effort 0.25]

Prints ONE JSON line (rank 0).

`decode` (default; the 32-layer decode workload): the 32-layer Mistral-7B shape (d 4096, 32/8 heads,
head_dim 128, ffn 14336, vocab 32000, tied embeddings) with random-init N(0, 0.02) fp16
weights bucketized on the GPU, RMSNorm gains 1.0, a 128-token prompt drawn uniformly from
[3, 32000) with seed 1, then greedy decoding at `--effort`.  One step = one generated token
(32 layers + LM head + argmax); W untimed tokens, then K timed tokens, all replays of one
captured CUDA graph.  `value` = generated tokens/s on the device clock; `e2e` = the same
through iam_model_forward from the host with the logits read back and argmaxed on the host
every token (the reference driver's loop, test_generation.cpp:239-291).  The roofline is the
fused bucketMul kernel's effective HBM bandwidth: its algorithmic bytes (2|S|C + 2R + 4N +
2*4096 + 4M per bucketMul, |S| reported by the kernel) over its CUDA-event time inside the
captured step.  Weights (13.9 GB) exceed the 126 MB L2 by two orders of magnitude.

`bucketmul` (the Mistral FFN and attention shapes): one step = the 7 bucketMuls of one Mistral layer on
alternating weight sets; value = effective GB/s.

`prefill`: one step = the config-4 prompt (128 tokens) ingested in one batched pass on the dense
tensor-core path (iam_model_prefill: every bucket row selected, tcgen05 products); value =
prompt tokens/s.  The roofline is the dense GEMM kernel's tensor throughput: 2 x tokens x
(out x in) flops per product over the GEMM launches' CUDA-event time at the prefill's shapes
(the fp16 hi + lo activation split doubles the tensor work; flops are counted once).  The
reference ingests a prompt one forward() at a time (test_generation.cpp:202-213); the decode
line reports that time beside the batched prefill.

`--impl reference` times the CPU restatement of the reference's kernels (oracle/, every
host thread) on the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "input-adaptive-matrix-inference-optimization_b200")
METRIC = "Mistral-7B batch-1 decode tok/s vs effort; bucketMul effective HBM GB/s"
LAYER_SHAPES = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
                ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]
N_SETS = 2


def load_pkg():
    import importlib.util
    if "iam_b200" in sys.modules:
        return sys.modules["iam_b200"]
    spec = importlib.util.spec_from_file_location("iam_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["iam_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


TRAFFIC_PROFILE = os.path.join(ROOT, "profiles", "decode_step_launch_list.md")
TRAFFIC_EFFORT = 0.25  # the effort the committed ncu traffic capture ran at


def profiled_traffic(effort):
    """DRAM bytes (read + write) per bm_fused_kernel launch from the committed ncu summary of
    the decode step, when this run's effort is the one that was profiled; else None."""
    if abs(effort - TRAFFIC_EFFORT) > 1e-9:
        return None
    try:
        with open(TRAFFIC_PROFILE) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [v.strip() for v in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- bucketmul workload


def algorithmic_bytes(sel, out_dim, in_dim):
    """2|S|C (selected weights) + 2R (stats ch.3) + 4N (x) + 2*4096 (probes) + 4M (out)."""
    C, R = out_dim // 16, 16 * in_dim
    return 2 * sel * C + 2 * R + 4 * in_dim + 2 * min(in_dim, 4096) + 4 * out_dim


def make_layer_sets(iam, torch, dev, seed):
    gen = torch.Generator(device=dev).manual_seed(seed)
    sets = []
    for _ in range(N_SETS):
        mats = []
        for name, o, i in LAYER_SHAPES:
            W = (torch.randn((o, i), generator=gen, device=dev) * 0.02).half().view(torch.int16)
            buckets = torch.empty((16 * i, o // 16), dtype=torch.int16, device=dev)
            s1 = torch.empty(16 * i, dtype=torch.int16, device=dev)
            pr = torch.empty(i, dtype=torch.int16, device=dev)
            iam.bucketize(W, buckets, None, s1, pr)
            del W
            x = torch.randn(i, generator=gen, device=dev)
            k = max(1, i // 100)
            idx = torch.randperm(i, generator=gen, device=dev)[:k]
            x[idx] *= 20.0
            out = torch.empty(o, dtype=torch.float32, device=dev)
            cnt = torch.zeros(1, dtype=torch.int32, device=dev)
            mats.append(dict(name=name, o=o, i=i, buckets=buckets, stats=s1, probes=pr, x=x, out=out, cnt=cnt))
        sets.append(mats)
    torch.cuda.synchronize()
    return sets


def run_bucketmul(args, rank, world):
    import torch
    iam = load_pkg()
    dev = torch.device(f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}")
    torch.cuda.set_device(dev)
    bm = iam.BucketMul(dev.index)
    sets = make_layer_sets(iam, torch, dev, seed=1234 + rank)
    stream = torch.cuda.current_stream()

    def step(k, events=None):
        for j, m in enumerate(sets[k % N_SETS]):
            if events is not None:
                events[j][0].record(stream)
            bm.full_mul(m["x"], m["stats"], m["probes"], m["buckets"], 0, m["i"], m["o"] // 16, 16 * m["i"],
                        args.effort, m["out"], stats_stride=1, count=m["cnt"])
            if events is not None:
                events[j][1].record(stream)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    sel = [[int(m["cnt"].item()) for m in s] for s in sets]
    step_bytes = [sum(algorithmic_bytes(sel[si][j], m["o"], m["i"]) for j, m in enumerate(s))
                  for si, s in enumerate(sets)]

    # device-timed region: K steps, per-launch events for the roofline
    per_launch = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in LAYER_SHAPES] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        t0.record(stream)
        for k in range(args.steps):
            step(args.warmup + k, per_launch[k])
        t1.record(stream)
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if world > 1:
        torch.distributed.barrier()
    launch_ms = [sum(e[0].elapsed_time(e[1]) for e in per_launch[k]) for k in range(args.steps)]
    total_bytes = sum(step_bytes[(args.warmup + k) % N_SETS] for k in range(args.steps))
    # max over ranks of the device time; sum of bytes
    if world > 1:
        t = torch.tensor([ms, float(total_bytes)], dtype=torch.float64, device=dev)
        tm = t.clone()
        torch.distributed.all_reduce(tm[:1], op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(t[1:], op=torch.distributed.ReduceOp.SUM)
        ms, total_bytes = float(tm[0]), float(t[1])
    gbs = total_bytes / (ms * 1e-3) / 1e9

    # e2e: the C ABI with host buffers, H2D of every x and D2H of every output inside the region
    pinned_x = [[m["x"].cpu().pin_memory() for m in s] for s in sets]
    pinned_o = [[torch.empty(m["o"], dtype=torch.float32).pin_memory() for m in s] for s in sets]
    h2d = sum(m["i"] * 4 for m in sets[0])
    d2h = sum(m["o"] * 4 for m in sets[0])
    e_steps = max(3, min(args.steps, 20))
    torch.cuda.synchronize()
    e0 = time.perf_counter()
    for k in range(e_steps):
        s = sets[k % N_SETS]
        for j, m in enumerate(s):
            m["x"].copy_(pinned_x[k % N_SETS][j], non_blocking=True)
            bm.full_mul(m["x"], m["stats"], m["probes"], m["buckets"], 0, m["i"], m["o"] // 16, 16 * m["i"],
                        args.effort, m["out"], stats_stride=1, count=m["cnt"])
            pinned_o[k % N_SETS][j].copy_(m["out"], non_blocking=True)
        torch.cuda.synchronize()
    e_sec = time.perf_counter() - e0
    e2e_bytes = sum(step_bytes[k % N_SETS] for k in range(e_steps))
    e2e_gbs = e2e_bytes / e_sec / 1e9 * (world if world > 1 else 1)

    peak, peak_kind = measured_peaks()
    launch_avg_bytes = total_bytes / (world * args.steps * len(LAYER_SHAPES)) if world > 1 else \
        total_bytes / (args.steps * len(LAYER_SHAPES))
    achieved = total_bytes / max(1e-9, sum(launch_ms) * 1e-3) / 1e9 / (world if world > 1 else 1)
    sel_frac = float(np.mean([sel[0][j] / (16 * m["i"]) for j, m in enumerate(sets[0])]))
    res = {
        "metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "bucketmul: the 7 Mistral-7B layer bucketMuls (config 2 shapes) per step",
                   "effort": args.effort, "x": "N(0,1), 1% channels x20", "weights": "N(0,0.02) fp16, GPU-bucketized",
                   "l2": "inputs larger than L2: 2 alternating weight sets, 0.9 GB", "selected_row_fraction":
                   round(sel_frac, 4), "bytes_per_step": int(step_bytes[0])},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_kind,
                     "kernel": "bg_kernel", "bytes_per_launch": int(launch_avg_bytes)},
        "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps * len(LAYER_SHAPES),
        "clocks": clk.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_bucketmul(sets, args.effort, budget_s=args.cpu_seconds)
    bm.close()
    return res


def host_set(m):
    return dict(buckets=m["buckets"].cpu().numpy().view(np.uint16), stats=m["stats"].cpu().numpy().view(np.uint16),
                probes=m["probes"].cpu().numpy().view(np.uint16), x=m["x"].cpu().numpy(), o=m["o"], i=m["i"])


def cpu_baseline_bucketmul(sets, effort, budget_s=10.0, steps=None):
    """The oracle (CPU restatement of bucketMul.cl) on the same layer set, all host threads."""
    sys.path.insert(0, ROOT)
    from oracle import ora
    threads = os.cpu_count() or 1
    hs = [host_set(m) for m in sets[0]]
    t0 = time.perf_counter()
    done, nbytes = 0, 0
    while True:
        for m in hs:
            _, n, _ = ora.bucketmul_full(m["x"], m["stats"], 1, m["probes"], m["buckets"], effort, nthreads=threads)
            nbytes += algorithmic_bytes(n, m["o"], m["i"])
        done += 1
        el = time.perf_counter() - t0
        if (steps is not None and done >= steps) or (steps is None and el >= budget_s):
            break
    return {"value": round(nbytes / el / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{done} steps of the 7 layer bucketMuls (one weight set) in {el:.1f} s",
            "seconds": round(el, 2), "ms_per_step": round(1e3 * el / done, 2)}


# ---------------------------------------------------------------- decode workload

PROMPT_LEN = 128


def mistral_cfg(iam, max_ctx, n_layers=None):
    d = dict(iam.MISTRAL_7B, max_ctx=max_ctx)
    if n_layers:
        d["n_layers"] = n_layers
    return iam.ModelConfig.make(**d)


def prompt_tokens(vocab):
    return np.random.default_rng(1).integers(3, vocab, PROMPT_LEN).tolist()


def decode_plan(args):
    """(start position, max_ctx, effort sweep, sweep tokens, profiled steps, e2e tokens) of the
    decode workload; the reference arm builds its model from the same numbers."""
    sweep = [e for e in (0.5, 1.0) if e != args.effort] if not args.no_sweep else []
    n_sweep = max(8, args.steps // 4)
    n_prof = 4
    n_e2e = max(3, min(args.steps, 32))
    # config 4: a 128-token prompt ingested token by token; config 5 (--kv-prefix 8192): a
    # random fp16 KV prefix, decoding starts after it
    start = args.kv_prefix if args.kv_prefix > 0 else PROMPT_LEN
    max_ctx = start + args.warmup + args.steps + n_sweep * len(sweep) + n_prof + n_e2e + 8
    return start, max_ctx, sweep, n_sweep, n_prof, n_e2e


def decode_config(args, cfg, world):
    """The workload description both arms print (the timed tokens are positions
    start + W .. start + W + K - 1 of the same model and prompt)."""
    start = args.kv_prefix if args.kv_prefix > 0 else PROMPT_LEN
    return {"workload": ("decode: config 5 context, Mistral-7B shape, 32 layers, random N(0,0.02) weights, "
                         f"tied embeddings, greedy batch-1 decode after a random fp16 KV prefix of "
                         f"{args.kv_prefix} tokens") if args.kv_prefix > 0 else
                        ("decode: config 4, Mistral-7B shape, 32 layers, random N(0,0.02) weights, "
                         "tied embeddings, greedy batch-1 decode after a 128-token prompt (seed 1)"),
            "model": "Mistral-7B (random init)" + (f", {cfg.n_layers} layers" if args.layers else ""),
            "effort": args.effort, "global_batch": 1, "seq_len": start + args.warmup + args.steps,
            "timed_positions": [start + args.warmup, start + args.warmup + args.steps - 1],
            "parallelism": f"tp{world}" if world > 1 else "single",
            "l2": "inputs larger than L2: 13.9 GB of bucket weights streamed per token"}


def tp_exchanges_per_layer():
    """Exchange launches per decoder layer under the NVLink tensor-parallel path."""
    if os.environ.get("IAM_TP_FUSED", "1") == "0":
        return 4
    return 2 if os.environ.get("IAM_TP_PUSH", "1") == "0" else 0


def run_decode(args, rank, world):
    import torch
    iam = load_pkg()
    dev = torch.device(f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}")
    torch.cuda.set_device(dev)
    start, max_ctx, sweep, n_sweep, n_prof, n_e2e = decode_plan(args)
    cfg = mistral_cfg(iam, max_ctx, args.layers)
    tp = None
    if world > 1:  # one decode stream, tensor-parallel over the ranks (NCCL inside the library)
        uid = [iam.tp_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(uid, src=0)
        tp = (rank, world, uid[0])
    t_build = time.perf_counter()
    model, logits, first = prepared_decode_model(args, iam, torch, cfg, dev, tp)
    build_s = time.perf_counter() - t_build
    stream = torch.cuda.current_stream()
    toks = torch.empty(max_ctx, dtype=torch.int32, device=dev)
    model.generate(first, start, args.warmup, args.effort, toks)  # includes the graph capture
    torch.cuda.synchronize()
    timed_first = int(toks[args.warmup - 1].item())  # the token the first timed step takes in

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        t0.record(stream)
        model.generate(-1, 0, args.steps, args.effort, toks)
        t1.record(stream)
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if world > 1:
        torch.distributed.barrier()
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t[0])
    ctx_end = start + args.warmup + args.steps
    sel_rows = model.selected_rows()
    step_bytes = model.step_bytes(ctx_end)  # this rank's share
    if world > 1:
        t = torch.tensor([float(step_bytes)], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t)
        step_bytes = int(t[0])
    tok_s = args.steps / (ms * 1e-3)  # one token stream, whatever the number of GPUs

    # roofline of the fused bucketMul kernel: CUDA events between the kernels of a captured step
    print(f"[bench] timed {args.steps} tokens in {ms:.2f} ms", file=sys.stderr, flush=True)
    prof = model.profile_steps(args.effort, n_prof)
    bm_ms = sum(t for k, t in prof if k == "bucketmul")
    all_ms = sum(t for _, t in prof)
    by_kind = {}
    for k, t in prof:
        by_kind[k] = by_kind.get(k, 0.0) + t
    total_bytes = model.step_bytes(ctx_end + n_prof)  # this rank's share
    lm_bytes = 2 * (cfg.vocab // world) * cfg.dim
    kv_bytes = 2 * cfg.n_layers * (cfg.n_kv_heads // world) * (ctx_end + n_prof) * cfg.head_dim * 2
    bm_bytes = total_bytes - lm_bytes - kv_bytes
    peak, peak_kind = measured_peaks()
    # Events between the kernels of an eager profiled step add their own gaps, so their sum is
    # longer than a graph-replayed step: each kernel kind is given its share of the events'
    # total, applied to the graph-timed step.
    share = bm_ms / all_ms if all_ms > 0 else 1.0
    bm_graph_ms = (ms / args.steps) * share
    achieved = bm_bytes / (bm_graph_ms * 1e-3) / 1e9

    # effort sweep (same graph machinery, fewer tokens)
    sweep_res = {}
    for e in sweep:
        model.generate(-1, 0, 2, e, toks)  # capture for this effort
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        model.generate(-1, 0, n_sweep, e, toks)
        b.record(stream)
        torch.cuda.synchronize()
        sweep_res[str(e)] = round(n_sweep / (a.elapsed_time(b) * 1e-3), 1)
    sweep_res[str(args.effort)] = round(args.steps / (ms * 1e-3), 1)

    # e2e: the host API loop -- token in as a launch argument, logits back to pinned memory,
    # argmax on the host, one synchronisation per token
    host_logits = torch.empty(cfg.vocab, dtype=torch.float32).pin_memory()
    tok = int(toks[0].item())
    pos = int(ctx_end + n_prof + 2 * len(sweep) + n_sweep * len(sweep))
    pos = min(pos, max_ctx - n_e2e - 1)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0 = time.perf_counter()
    for i in range(n_e2e):
        model.forward(tok, pos + i, args.effort, logits)  # every rank: the same token, gathered logits
        host_logits.copy_(logits, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        tok = int(np.argmax(host_logits.numpy()))
    e2e_s = time.perf_counter() - e0
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_s = float(t[0])
    e2e_tok_s = n_e2e / e2e_s

    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:  # the CPU port runs on rank 0 at N=1 only
        # a bounded sample from the GPU's cache at the first timed position (the later
        # positions are rewritten as the oracle goes), before the prefill below rewrites the prompt's
        cpu_base = cpu_baseline_decode(model, cfg, args.effort, start + args.warmup, timed_first,
                                       budget_s=args.cpu_seconds)

    prefill = None
    if world == 1:  # the prompt again, in one batched pass on the dense tensor-core path
        prompt = prompt_tokens(cfg.vocab)
        model.prefill(prompt, 0, None)  # builds the dense weight copies once
        pf_ms = time_prefill(model, prompt, 3)
        prefill = {"prompt_tokens": len(prompt), "ms": round(pf_ms, 3),
                   "tokens_per_s": round(len(prompt) / (pf_ms * 1e-3), 1),
                   "path": "iam_model_prefill (every bucket row selected, tcgen05 products)",
                   "note": "the timed decode above ingested the prompt token by token (the reference's way)"}

    res = {
        "metric": METRIC, "value": round(tok_s, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": decode_config(args, cfg, world),
        "detail": {"tokens_per_s_by_effort": sweep_res, "selected_rows_per_step": sel_rows,
                   "algorithmic_bytes_per_step": step_bytes,
                   "step_effective_GBps": round(step_bytes / (ms / args.steps * 1e-3) / 1e9, 1),
                   "model_build_s": round(build_s, 1)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": profiled_traffic(args.effort),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per bg_kernel launch, "
                                       "mean over the 8 launches of a 2-layer decode step (profiles/"
                                       "decode_step_launch_list.md); the per-launch bytes do not depend on depth",
                     "peak_source": peak_kind,
                     "kernel": "bg_kernel", "bytes_per_launch": int(bm_bytes / (4 * cfg.n_layers)),
                     "kernel_ms_per_step": round(bm_graph_ms, 4),
                     "kernel_share_of_step": round(share, 4),
                     "timing": "the kernel's share of the CUDA-event times of profiled steps, applied to the "
                               "graph-timed ms_per_step",
                     "kernel_ms_per_step_events": round(bm_ms, 4), "step_ms_events": round(all_ms, 4),
                     "ms_per_step_by_kernel_events": {k: round(v, 4) for k, v in by_kind.items()}},
        "e2e": {"value": round(e2e_tok_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * cfg.vocab},
        # ours per step and rank: embed, key clear, 32 x (4 bucketMul + attention), LM head,
        # advance; under TP the argmax-key exchange (NVLink one-shot) and, per layer, no
        # exchange launch (the o / down partials are exchanged inside their bucketMul launches,
        # heads and gate/up slices pushed by their producers), 2 with IAM_TP_PUSH=0, 4 with
        # IAM_TP_FUSED=0
        "gpu_launches": world * args.steps * (2 + 5 * cfg.n_layers + 2 +
                                              ((tp_exchanges_per_layer() * cfg.n_layers + 1) if world > 1 and
                                               os.environ.get("IAM_TP_COLL", "p2p") != "nccl" else 0)),
        "clocks": clk.summary(),
    }
    if prefill:
        res["prefill"] = prefill
    if cpu_base:
        res["cpu_baseline"] = cpu_base
    model.close()  # its captured graph holds NCCL work: released before the process group
    return res


def dense_split_for(m, k, n, sms=148):
    """The split-K the library picks for one dense product (dense_auto_split in iam_dense.cu)."""
    tiles = -(-m // 256) * -(-n // 128)
    kb = -(-k // 64)
    if tiles >= sms:
        return 1
    split = min(max(1, sms // tiles), 8, max(1, kb // 4))
    per = -(-kb // split)
    return -(-kb // per)


def prefill_shapes(cfg):
    qn, kvn = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    return [(qn + 2 * kvn, cfg.dim), (cfg.dim, qn), (2 * cfg.ffn_dim, cfg.dim), (cfg.dim, cfg.ffn_dim)]


def time_prefill(model, tokens, reps):
    import torch
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(reps):
        model.prefill(tokens, 0, None)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def gemm_roofline(iam, torch, dev, cfg, n, reps=5):
    """CUDA-event time of the dense GEMM launches of one prefill layer at n tokens (random
    weights of the same shapes: the kernel's time depends on the shapes only)."""
    shapes = prefill_shapes(cfg)
    d = iam.Dense(max_tokens=n, max_in_dim=max(k for _, k in shapes), max_out_dim=max(m for m, _ in shapes),
                  device=dev.index)
    flops, ms = 0.0, 0.0
    for m, k in shapes:
        w = (torch.randn(m, k, device=dev) * 0.02).half()
        x = torch.randn(n, k, device=dev)
        y = torch.empty(n, m, device=dev)
        d.gemm(w, x, y)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            d.gemm(w, x, y)
        b.record()
        torch.cuda.synchronize()
        ms += a.elapsed_time(b) / reps
        flops += 2.0 * n * m * k
        del w, x, y
    d.status()
    d.close()
    return flops, ms


def run_prefill(args, rank, world):
    """Batched dense prefill of the config-4 prompt; under torchrun every rank runs its own
    replica (the prefill does not shard) and value is the sum over ranks."""
    import torch
    iam = load_pkg()
    dev = torch.device(f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}")
    torch.cuda.set_device(dev)
    cfg = mistral_cfg(iam, PROMPT_LEN + 8, args.layers)
    model = iam.Model.random(cfg, seed=0, device=dev.index)
    tokens = prompt_tokens(cfg.vocab)
    P = len(tokens)
    t_dense = time.perf_counter()
    model.prefill(tokens, 0, None)  # builds the dense weight copies once
    torch.cuda.synchronize()
    dense_build_s = time.perf_counter() - t_dense
    time_prefill(model, tokens, args.warmup)
    if world > 1:
        torch.distributed.barrier()
    with ClockSampler(dev.index) as clk:
        ms = time_prefill(model, tokens, args.steps)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t[0])
    tok_s = world * P / (ms * 1e-3)
    # the reference's way: the same prompt through the decode step, one token at a time
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device=dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for pos, tok in enumerate(tokens):
        model.forward(tok, pos, args.effort, logits)
    b.record()
    torch.cuda.synchronize()
    tbt_ms = a.elapsed_time(b)
    # e2e: host tokens in, the last token's logits back to pinned host memory
    host_logits = torch.empty(cfg.vocab, dtype=torch.float32).pin_memory()
    reps = max(3, min(args.steps, 10))
    torch.cuda.synchronize()
    e0 = time.perf_counter()
    for _ in range(reps):
        model.prefill(tokens, 0, logits)
        host_logits.copy_(logits, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2e_tok_s = world * P * reps / (time.perf_counter() - e0)
    flops, gemm_ms = gemm_roofline(iam, torch, dev, cfg, P)
    peak = measured_tensor_peak()
    achieved = flops / (gemm_ms * 1e-3) / 1e12
    splits = [dense_split_for(m, k, P) for m, k in prefill_shapes(cfg)]
    launches = 1 + cfg.n_layers * (4 + sum(1 for sp in splits if sp > 1) + 2 + 1 + 1 + 1 + 1) + 2
    res = {
        "metric": METRIC, "value": round(tok_s, 1), "unit": "prompt tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 x (f16 hi + f16 lo), f32 accumulate",
        "data": "synthetic",
        "config": {"workload": ("prefill: config 4 prompt (128 tokens, seed 1) through the 32-layer Mistral-7B "
                                "shape in one batched pass on the dense tensor-core path"),
                   "model": "Mistral-7B (random init)" + (f", {cfg.n_layers} layers" if args.layers else ""),
                   "prompt_tokens": P, "global_batch": 1, "seq_len": P,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2: 13.9 GB of dense weights streamed per prefill",
                   "token_by_token_ms": round(tbt_ms, 2),
                   "token_by_token_effort": args.effort,
                   "speedup_vs_token_by_token": round(tbt_ms / ms, 1),
                   "dense_weights_build_s": round(dense_build_s, 2)},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak[0], "unit": "TFLOP/s",
                     "frac": round(achieved / peak[0], 4), "traffic": None, "peak_source": peak[1],
                     "kernel": "dense_gemm_kernel",
                     "flops_per_layer": flops, "gemm_ms_per_layer": round(gemm_ms, 4),
                     "note": "flops counted once per product; the hi + lo activation halves run two MMAs each"},
        "e2e": {"value": round(e2e_tok_s, 1), "unit": "prompt tokens/s", "h2d_bytes_per_step": 4 * P,
                "d2h_bytes_per_step": 4 * cfg.vocab},
        "gpu_launches": world * args.steps * launches,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_prefill(model, cfg, budget_s=args.cpu_seconds)
    model.close()
    return res


def measured_tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            v = json.load(f).get("bf16_tflops")
        if v:
            return float(v), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        pass
    return 1590.0, "fallback (1.59 PFLOP/s)"


def cpu_baseline_prefill(model, cfg, budget_s=10.0, tokens=2):
    """The oracle's dense decode step (every bucket row selected) on every host core, token by
    token: the reference's way of ingesting a prompt, on its CPU restatement."""
    sys.path.insert(0, ROOT)
    from oracle import ora
    om = ora.OracleModel(cfg.as_dict(), model.export_weights())
    threads = os.cpu_count() or 1
    prompt = prompt_tokens(cfg.vocab)
    t0 = time.perf_counter()
    n = 0
    for pos, tok in enumerate(prompt):
        om.forward_dense(tok, pos, nthreads=threads)
        n += 1
        if n >= tokens or time.perf_counter() - t0 >= budget_s:
            break
    sec = time.perf_counter() - t0
    return {"value": round(n / sec, 3), "unit": "prompt tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} prompt tokens of config 4 through the oracle's dense decode step ({cfg.n_layers} layers)"}


def cpu_baseline_decode(model, cfg, effort, start_pos, first_tok, budget_s=10.0, steps=None, warmup=0):
    """The oracle decode step (CPU restatement of the reference's kernels), every host thread,
    on the same weights, continuing from the GPU model's KV cache: `warmup` untimed steps at
    start_pos.., then timed steps (all `steps`, or as many as fit in budget_s)."""
    sys.path.insert(0, ROOT)
    from oracle import ora
    iam = sys.modules["iam_b200"]
    threads = os.cpu_count() or 1
    t_pre = time.perf_counter()
    om = ora.OracleModel(cfg.as_dict(), model.export_weights())
    om.set_kv(np.stack([model.read_weight(iam.W_K_CACHE, l) for l in range(cfg.n_layers)]),
              np.stack([model.read_weight(iam.W_V_CACHE, l) for l in range(cfg.n_layers)]))
    tok, pos = first_tok, start_pos
    for _ in range(warmup):
        tok, _, _ = om.forward(tok, pos, effort, nthreads=threads)
        pos += 1
    t0 = time.perf_counter()
    done, p0 = 0, pos
    while True:
        tok, _, _ = om.forward(tok, pos, effort, nthreads=threads)
        pos += 1
        done += 1
        el = time.perf_counter() - t0
        if (steps is not None and done >= steps) or (steps is None and el >= budget_s):
            break
    return {"value": round(done / el, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{done} greedy decode steps at positions {p0}..{pos - 1} of the same 32-layer model, "
                      f"continuing from the GPU-built KV cache, {el:.1f} s", "seconds": round(el, 2),
            "steps": done, "setup_s": round(t0 - t_pre, 1)}


def prepared_decode_model(args, iam, torch, cfg, dev, tp=None):
    """The decode model after its context: the 128-token prompt ingested token by token
    (test_generation.cpp:202-210) or, for --kv-prefix, a random fp16 KV prefix.  Returns
    (model, logits, first greedy token)."""
    model = iam.Model.random(cfg, seed=0, device=dev.index, tp=tp)
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device=dev)
    if args.kv_prefix > 0:
        model.fill_kv_random(args.kv_prefix, seed=1)
        model.forward(int(prompt_tokens(cfg.vocab)[0]), args.kv_prefix - 1, args.effort, logits)
    else:
        for pos, tok in enumerate(prompt_tokens(cfg.vocab)):
            model.forward(tok, pos, args.effort, logits)
    return model, logits, int(torch.argmax(logits).item())


def run_reference(args, rank, world):
    """--impl reference: the oracle port of the reference's kernels on the host cores."""
    if rank != 0:
        return None
    if args.workload == "decode":
        # the GPU arm's workload: the same model, context and timed positions (the context is
        # built on the GPU, as the GPU arm builds it; the oracle then runs W untimed and K
        # timed steps from there)
        import torch
        iam = load_pkg()
        dev = torch.device("cuda:0")
        torch.cuda.set_device(dev)
        start, max_ctx, _, _, _, _ = decode_plan(args)
        cfg = mistral_cfg(iam, max_ctx, args.layers)
        model, _, first = prepared_decode_model(args, iam, torch, cfg, dev)
        torch.cuda.synchronize()
        cb = cpu_baseline_decode(model, cfg, args.effort, start, first, steps=args.steps, warmup=args.warmup)
        model.close()
        return {
            "metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": world, "steps": cb["steps"],
            "warmup": args.warmup, "ms_per_step": round(1e3 * cb["seconds"] / cb["steps"], 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": decode_config(args, cfg, world),
            "reference_path": "the CPU restatement (oracle) of the reference's decode step: bucketMul.cl, aux.cl, "
                              "matrix.cl, transformer_layer.hpp, every host thread",
            "cpu_baseline": {"value": cb["value"], "unit": "tokens/s", "cores": cb["cores"], "kind": "port",
                             "sample": cb["sample"]},
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    if args.workload == "prefill":  # the reference's way: the prompt through the dense step, token by token
        import torch
        iam = load_pkg()
        cfg = mistral_cfg(iam, PROMPT_LEN + 8, args.layers)
        model = iam.Model.random(cfg, seed=0)
        cb = cpu_baseline_prefill(model, cfg, budget_s=args.cpu_seconds, tokens=max(1, min(args.steps, 4)))
        model.close()
        return {
            "metric": METRIC, "value": cb["value"], "unit": "prompt tokens/s", "n_gpus": world,
            "steps": max(1, min(args.steps, 4)), "warmup": args.warmup, "ms_per_step": round(1e3 / cb["value"], 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "prefill: the config-4 prompt through the CPU restatement (oracle) of the "
                                   "reference's step with every bucket row selected, one token at a time",
                       "model": "Mistral-7B (random init)", "prompt_tokens": PROMPT_LEN, "global_batch": 1},
            "cpu_baseline": {"value": cb["value"], "unit": cb["unit"], "cores": cb["cores"], "kind": "port",
                             "sample": cb["sample"]},
            "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    import torch
    iam = load_pkg()
    dev = torch.device("cuda:0") if torch.cuda.is_available() else None
    if dev is None:
        return {"impl": "reference", "unavailable": "workload generation needs the GPU bucketizer"}
    sets = make_layer_sets(iam, torch, dev, seed=1234)
    for _ in range(args.warmup):
        pass
    cb = cpu_baseline_bucketmul(sets, args.effort, steps=args.steps)
    per_step_ms = cb["ms_per_step"]
    res = {
        "metric": METRIC, "value": cb["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "bucketmul: the 7 Mistral-7B layer bucketMuls (config 2 shapes) per step",
                   "effort": args.effort},
        "cpu_baseline": {"value": cb["value"], "unit": "GB/s", "cores": cb["cores"], "kind": "port",
                         "sample": cb["sample"]},
        "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "bucketmul", "prefill"])
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--effort", type=float, default=0.25)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers of the decode model (default 32; fewer only for small profiling captures)")
    ap.add_argument("--kv-prefix", type=int, default=0,
                    help="decode after a random KV prefix of this many tokens (config 5: 8192) instead of the prompt")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    # stdout carries the one JSON line: whatever the libraries print there (NCCL's version
    # banner, for one) goes to stderr instead
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)

    def emit(res):
        if rank == 0 and res is not None:
            os.write(json_fd, (json.dumps(res) + "\n").encode())

    if args.impl == "reference":  # rank 0 alone times the reference's CPU path: no collective at all
        emit(run_reference(args, rank, world))
        return
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        if args.workload == "decode":
            res = run_decode(args, rank, world)
        elif args.workload == "prefill":
            res = run_prefill(args, rank, world)
        else:
            res = run_bucketmul(args, rank, world)
        emit(res)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
