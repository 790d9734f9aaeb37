#!/usr/bin/env python
"""Throughput of the SMO8bit optimizer step on B200 (params stepped/s, HBM GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One "step" is one optimizer step over the whole parameter set of the workload
(default: the ~700M-parameter decoder, SMO8bit k=0.25 low_peak, fp32 params,
synthetic grads ~N(0, 1e-3)).  With N > 1 (launched by torch.distributed.run)
the tensors are sharded ZeRO-1 style: each rank steps the tensors it owns, and
``value`` is all ranks' params / the slowest rank's device time.  The NCCL
all-gather of the flat parameter buffer that completes a ZeRO-1 step is timed
separately (``zero1``).  Rank 0 prints one JSON line.

``--impl reference`` times the reference's own CPU step (its PyTorch
SMO8bit / SMO, installed unmodified in baseline/_ref) on all host cores over
the same workload: whole-set steps when K + W of them fit about two minutes,
else round-robin samples of the set; without baseline/_ref it times the C
restatement of the step (the oracle) the same way.  Same metric and config.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "params stepped/sec per SMO-8bit step"
UNIT = "params/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="decoder700m")
    ap.add_argument("--dtype", default="f32", choices=sorted(DTYPES),
                    help="parameter and gradient dtype (the reference steps half-precision parameters in their dtype)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--e2e-chunks", type=int, default=24)
    ap.add_argument("--cpu-sample-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="one process: step only the share of the tensors that rank --shard-rank owns "
                         "when the set is split ZeRO-1 style over this many ranks (per-rank profiling)")
    ap.add_argument("--shard-rank", type=int, default=0)
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            peaks = json.load(f)
        return float(peaks["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(workload, kernel, world=1, rank=0):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary: the whole set at one GPU, or rank ``rank``'s share when the set
    is split over ``world`` ranks (``<workload>@<world>`` entries)."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            data = json.load(f)
        if world > 1:
            return data[f"{workload}@{world}"][str(rank)]
        return data[workload][kernel]
    except Exception:
        return None


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


DTYPES = {"f32": "float32", "bf16": "bfloat16", "f16": "float16"}


def build_workload(wl, seed, device, owned, dtype="f32"):
    """Params (all tensors) and grads (owned tensors) filled on the device by
    the synthetic generator (fp32 draws, rounded to ``dtype``)."""
    import torch
    from smo_optimizer_b200 import ops, synthetic

    tdt = getattr(torch, DTYPES[dtype])
    params, grads = [], []
    for i, (name, shape) in enumerate(wl.tensors):
        p = torch.empty(shape, dtype=torch.float32, device=device)
        ops.synth_normal_(p, seed, synthetic.stream_id(synthetic.STREAM_PARAM, 0, i), 0.02)
        params.append(torch.nn.Parameter(p.to(tdt) if tdt != torch.float32 else p))
        if owned[i]:
            g = torch.empty(shape, dtype=torch.float32, device=device)
            ops.synth_normal_(g, seed, synthetic.stream_id(synthetic.STREAM_GRAD, 1, i), 1e-3)
            if wl.bf16_grads:
                g = g.to(torch.bfloat16).to(torch.float32)
            params[-1].grad = g.to(tdt) if tdt != torch.float32 else g
        grads.append(params[-1].grad)
    return params, grads


def _all_host_threads():
    """Every host core: torch.distributed.run sets OMP_NUM_THREADS=1 for its
    ranks, which the CPU legs override."""
    return max(1, os.cpu_count() or 1)


def cpu_baseline(wl, seed, seconds):
    """The oracle (C restatement of the reference step, OpenMP) on a sample of the workload."""
    import numpy as np

    from oracle import oracle
    from smo_optimizer_b200 import synthetic

    oracle.build()
    oracle.set_num_threads(_all_host_threads())
    # one decoder layer's tensors (or the first few of another workload)
    take = []
    total = 0
    for i, (name, shape) in enumerate(wl.tensors):
        take.append((i, shape))
        total += int(np.prod(shape))
        if total >= 25_000_000:
            break
    params = [synthetic.synth_param(seed, i, s) for i, s in take]
    grads = [synthetic.synth_grad(seed, 1, i, s, bf16=wl.bf16_grads) for i, s in take]
    opt = oracle.OracleOptimizer(wl.optimizer, [{"params": params}], **wl.kwargs)
    opt.step(grads)  # warm-up (init + first step)
    steps, t0 = 0, time.perf_counter()
    while True:
        opt.step(grads)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds or steps >= 1000:
            break
    return {"value": total * steps / el, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{len(take)} tensors ({total / 1e6:.1f}M params) of {wl.name}, {steps} steps, "
                      f"{el:.1f} s, OpenMP C oracle"}


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def import_reference():
    """The reference's own optimizer classes, installed unmodified into
    baseline/_ref (``pip install --target baseline/_ref``); None when absent."""
    if not os.path.isdir(os.path.join(REF_DIR, "smo")):
        return None, "reference not installed in baseline/_ref"
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        from smo.optimizers.spatial import SMO as RefSMO
        from smo.optimizers.spatial_8bit import SMO8bit as RefSMO8bit
    except Exception as e:  # pragma: no cover - depends on the install
        return None, f"reference import failed: {e!r}"
    import smo
    if not os.path.abspath(smo.__file__).startswith(REF_DIR):
        return None, f"an smo package outside baseline/_ref shadows the reference ({smo.__file__})"
    return {"SMO8bit": RefSMO8bit, "SMO": RefSMO}, None


class ReferenceLeg:
    """The reference's PyTorch step (SMO8bit / SMO from baseline/_ref) on the
    host cores over the workload's tensors, timed as
    benchmarks/suites/optimizer_step/benchmark_step_time.py:22-38 times it
    (warm-up, then time.perf_counter around optimizer.step()).

    Inputs are seeded torch CPU draws with the workload's shapes and
    distributions (params N(0, 0.02), grads N(0, 1e-3), bf16-rounded where the
    workload says so).  ``step(members)`` steps the tensors listed: one
    optimizer per tensor, so that a bounded sample of the set can be timed when
    the whole set does not fit the time budget."""

    def __init__(self, wl, seed, classes):
        import torch

        from smo_optimizer_b200 import protected_param_groups

        torch.set_num_threads(_all_host_threads())
        self.torch = torch
        self.wl = wl
        gen = torch.Generator().manual_seed(seed)
        cls = classes[wl.optimizer]
        self.params, self.opts = [], []
        flags = {}
        if wl.protect_output:
            # the reference harness's grouping rule (t4_memory_benchmark.py:117-133)
            named = [(n, i) for i, (n, _) in enumerate(wl.tensors)]
            for g in protected_param_groups(named, wl.protect_output, quant_capable=wl.optimizer == "SMO8bit"):
                for i in g["params"]:
                    flags[i] = g.get("compress", True)
        for i, (_, shape) in enumerate(wl.tensors):
            p = torch.nn.Parameter(torch.randn(shape, generator=gen) * 0.02)
            g = torch.randn(shape, generator=gen) * 1e-3
            if wl.bf16_grads:
                g = g.to(torch.bfloat16).to(torch.float32)
            p.grad = g
            group = {"params": [p]}
            if i in flags:
                group["compress"] = flags[i]
            self.params.append(p)
            self.opts.append(cls([group], **wl.kwargs))
        self.numel = [p.numel() for p in self.params]

    def step(self, members):
        t0 = time.perf_counter()
        for i in members:
            self.opts[i].step()
        return time.perf_counter() - t0

    def cores(self):
        return self.torch.get_num_threads()


def reference_baseline(wl, seed, seconds):
    """cpu_baseline of kind "reference": the reference's own step on a sample
    of the workload (about ``seconds`` of host time), or None if the reference
    is not installed."""
    classes, why = import_reference()
    if classes is None:
        return None
    # about 25M params (the sample of the port leg)
    take, total = [], 0
    for i, (_, shape) in enumerate(wl.tensors):
        take.append(i)
        total += _numel(shape)
        if total >= 25_000_000:
            break
    sub = type(wl)(wl.name, tuple(wl.tensors[i] for i in take), wl.optimizer, wl.kwargs, wl.protect_output,
                   wl.bf16_grads)
    leg = ReferenceLeg(sub, seed, classes)
    members = list(range(len(take)))
    leg.step(members)  # state init
    steps, el = 0, 0.0
    while el < seconds and steps < 1000:
        el += leg.step(members)
        steps += 1
    return {"value": total * steps / el, "unit": UNIT, "cores": leg.cores(), "kind": "reference",
            "sample": f"{len(take)} tensors ({total / 1e6:.1f}M params) of {wl.name}, {steps} steps, {el:.1f} s, "
                      f"the reference's PyTorch {wl.optimizer}.step (baseline/_ref) on the host cores"}


def _numel(shape):
    n = 1
    for s in shape:
        n *= int(s)
    return n


def run_reference(args, rank, world):
    """The reference arm: the reference's own CPU step (its PyTorch SMO8bit /
    SMO, installed unmodified in baseline/_ref) on the host cores, on the
    workload of the GPU arm.  Only rank 0 works; other ranks exit at once.

    A step is one optimizer step over the whole parameter set when K + W such
    steps fit the time budget (about two minutes), else over a round-robin
    sample of the tensors sized to fit it.  Without baseline/_ref the C
    restatement of the step (the oracle) is timed the same way."""
    if rank != 0:
        return 0
    from smo_optimizer_b200 import workloads

    wl = workloads.get(args.workload)
    n = len(wl.tensors)
    classes, why = import_reference()
    budget = float(os.environ.get("SMO_REFERENCE_BUDGET_S", "120"))
    if classes is not None:
        leg = ReferenceLeg(wl, args.seed, classes)
        kind = "reference"
        what = f"the reference's PyTorch {wl.optimizer}.step (baseline/_ref)"
        step_fn, cores = leg.step, leg.cores
        numel = leg.numel
    else:
        from oracle import oracle
        from smo_optimizer_b200 import synthetic

        oracle.build()
        oracle.set_num_threads(_all_host_threads())
        opts = []
        for i, (_, shape) in enumerate(wl.tensors):
            p = synthetic.synth_param(args.seed, i, shape)
            g = synthetic.synth_grad(args.seed, 1, i, shape, bf16=wl.bf16_grads)
            opts.append((oracle.OracleOptimizer(wl.optimizer, [{"params": [p]}], **wl.kwargs), g))

        def step_fn(members):
            t0 = time.perf_counter()
            for i in members:
                opts[i][0].step([opts[i][1]])
            return time.perf_counter() - t0

        kind = "port"
        what = f"the C restatement of the step (OpenMP oracle; {why})"
        cores = oracle.num_threads
        numel = [_numel(s) for _, s in wl.tensors]

    full = list(range(n))
    t_full = step_fn(full)  # state init + first step over the whole set
    t_full = min(t_full, step_fn(full))
    per_step = budget / max(1, args.steps + args.warmup)
    if t_full <= per_step:
        chunks = [full]
        sample = f"whole set ({sum(numel) / 1e6:.1f}M params, {n} tensors) per step"
    else:
        # contiguous round-robin chunks of tensors, each about per_step long
        frac = per_step / t_full
        target = max(1, int(sum(numel) * frac))
        chunks, cur, acc = [], [], 0
        for i in full:
            cur.append(i)
            acc += numel[i]
            if acc >= target:
                chunks.append(cur)
                cur, acc = [], 0
        if cur:
            chunks.append(cur)
        sample = f"round-robin chunks of ~{target / 1e6:.0f}M params of the {sum(numel) / 1e6:.1f}M-param set per step"
    for w in range(args.warmup):
        step_fn(chunks[w % len(chunks)])
    stepped, el = 0, 0.0
    for k in range(args.steps):
        c = chunks[(args.warmup + k) % len(chunks)]
        el += step_fn(c)
        stepped += sum(numel[i] for i in c)
    value = stepped / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32+int8",
        "data": "synthetic (seeded host draws, params N(0,0.02), grads N(0,1e-3))",
        "config": _config(wl, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores(), "kind": kind,
                         "sample": f"{sample}; {what}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _config(wl, world, dtype="f32"):
    gb = (8 if dtype == "f32" else 4) * wl.numel / 1e9  # params and grads
    l2 = (f"inputs ({gb:.1f} GB of params and grads) larger than L2; no flush" if gb > 0.5 else
          f"inputs ({gb * 1e3:.0f} MB) fit in L2: a step re-reads what the previous step left there")
    cfg = {"workload": wl.name, "params": wl.numel, "tensors": len(wl.tensors),
           "parallelism": f"zero1-dp{world}" if world > 1 else "single", **_cfg(wl), "l2": l2}
    if dtype != "f32":
        cfg["param_dtype"] = dtype
    return cfg


def _cfg(wl):
    kw = wl.kwargs
    cfg = {"optimizer": wl.optimizer, "k_ratio": kw.get("k_ratio"), "block_size": kw.get("block_size"),
           "low_peak": kw.get("low_peak", False), "weight_decay": kw.get("weight_decay"),
           "protect_output": wl.protect_output, "bf16_grads": wl.bf16_grads}
    if wl.compress is not True:
        cfg["compress"] = wl.compress
    if wl.general_path:
        cfg["kernels"] = "general two-launch path pinned"
    return cfg


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import numpy as np
    import torch
    import torch.distributed as dist

    from smo_optimizer_b200 import SMO, SMO8bit, _lib, workloads, zero

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    wl = workloads.get(args.workload)
    cls = SMO8bit if wl.optimizer == "SMO8bit" else SMO
    kw = dict(wl.kwargs)

    shapes = [s for _, s in wl.tensors]
    elem = 4 if args.dtype == "f32" else 2
    costs = [zero.step_bytes(s, wl.optimizer, kw.get("k_ratio", 0.25), kw.get("block_size", 64), elem=elem,
                             compress=wl.compress) for s in shapes]
    shard_of = args.shard_of if world == 1 and args.shard_of > 1 else 0
    if shard_of:
        # one rank's share of a ZeRO-1 split, stepped alone on this GPU
        owner = zero.lpt_partition(costs, shard_of)
        owned = [o == args.shard_rank for o in owner]
    else:
        owner = zero.lpt_partition(costs, world)
        owned = [o == rank for o in owner]
    # N > 1: every rank holds every gradient (a replicated model's backward), which
    # the gradient reduce-scatter timing below needs; the local step reads only
    # the owned ones
    params, grads = build_workload(wl, args.seed, device, owned if world == 1 else [True] * len(owned), args.dtype)
    flat = None
    if world > 1:
        # ZeRO-1 layout: parameters rebound into one rank-contiguous buffer so the
        # exchange after the step is a single in-place all-gather
        flat = zero.FlatParams(params, owner, world, rank).bind()
    mine = [p for p, o in zip(params, owned) if o]
    if wl.protect_output:
        named = [(n, p) for (n, _), p, o in zip(wl.tensors, params, owned) if o]
        opt = cls(named, protect_output=wl.protect_output, **kw)
    else:
        opt = cls([{"params": mine, "compress": wl.compress}], **kw)
    if wl.general_path:
        opt._kernel_flags = _lib.SMO_FLAG_GENERAL_PATH
    my_params = sum(p.numel() for p in mine)
    my_bytes = sum(c for c, o in zip(costs, owned) if o)
    total_params = wl.numel
    lib = _lib.load()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # ---- warm-up
    for _ in range(max(3, args.warmup)):
        opt.step()
    torch.cuda.synchronize()
    status = opt.workspace_status()
    if status:
        raise RuntimeError(f"device status {status} after warm-up")

    # ---- timed region: device events, per-step events bracket the launch(es)
    K = args.steps
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local_rank)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    launches0 = lib.smo_launch_count()
    t_start.record(stream)
    host_t = []
    for k in range(K):
        ev[k][0].record(stream)
        h0 = time.perf_counter()
        opt.step()
        host_t.append(time.perf_counter() - h0)
        ev[k][1].record(stream)
    t_end.record(stream)
    # host time of one step() call: the median of the first ten (launches are
    # asynchronous; later calls of a long run can wait for room in the launch queue)
    host_ms = float(np.median(host_t[:10])) * 1e3
    host_ms_max = float(np.max(host_t)) * 1e3
    torch.cuda.synchronize()
    launches = lib.smo_launch_count() - launches0
    barrier()
    clk = clocks.stop()
    elapsed_ms = t_start.elapsed_time(t_end)
    kern_ms = [a.elapsed_time(b) for a, b in ev]
    step_ms_local = sum(kern_ms) / K
    if world > 1:
        t = torch.tensor([elapsed_ms, step_ms_local], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, step_ms = float(t[0]), float(t[1])
    else:
        step_ms = step_ms_local
    status = opt.workspace_status()
    if status:
        raise RuntimeError(f"device status {status} after the timed region")

    ms_per_step = elapsed_ms / K
    if shard_of:
        total_params = my_params
    value = total_params / (ms_per_step * 1e-3)
    peak, peak_src = load_peaks()
    achieved = my_bytes / (step_ms_local * 1e-3) / 1e9
    roof = {"bound": "hbm", "kernel": "smo step (all launches of one step)", "achieved": achieved,
            "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_src,
            "algorithmic_bytes_per_launch": my_bytes,
            "traffic": load_traffic(wl.name if args.dtype == "f32" else f"{wl.name}:{args.dtype}", "step",
                                    shard_of or world, args.shard_rank if shard_of else rank)}

    # ---- ZeRO-1 completion: one in-place all-gather of the flat parameter buffer
    zero1 = None
    if world > 1:
        for _ in range(3):
            flat.all_gather()
        torch.cuda.synchronize()
        barrier()
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        nb = 10
        a.record(stream)
        for _ in range(nb):
            flat.all_gather()
        b.record(stream)
        for _ in range(nb):
            opt.step()
            flat.all_gather()
        c.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / nb, b.elapsed_time(c) / nb], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ag_ms, zms = float(t[0]), float(t[1])
        zero1 = {"step_plus_allgather_ms": zms, "allgather_ms": ag_ms,
                 "params_per_s": total_params / (zms * 1e-3),
                 "allgather_bytes_per_rank": flat.bytes_per_rank,
                 "allgather_busbw_gbs": flat.bytes_per_rank / (ag_ms * 1e-3) / 1e9}
        # gradient reduce-scatter (ZeRO-2 communication) + local step + all-gather;
        # every rank holds the same synthetic gradients, so averaging keeps them
        flat.bind_grads()
        grads = [p.grad for p in params]
        for _ in range(3):
            flat.reduce_scatter_grads()
            opt.step()
            flat.all_gather()
        torch.cuda.synchronize()
        barrier()
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record(stream)
        for _ in range(nb):
            flat.reduce_scatter_grads()
        b.record(stream)
        for _ in range(nb):
            flat.reduce_scatter_grads()
            opt.step()
            flat.all_gather()
        c.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / nb, b.elapsed_time(c) / nb], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        zero1["reduce_scatter_ms"] = float(t[0])
        zero1["reduce_scatter_step_allgather_ms"] = float(t[1])
        zero1["reduce_scatter_step_allgather_params_per_s"] = total_params / (float(t[1]) * 1e-3)

    # ---- e2e through the public API with host buffers (pinned): H2D grads, step, D2H params.
    # The owned tensors are split into chunks of about equal size, each with its
    # own optimizer instance; chunk k's grads go in on one stream while chunk
    # k-1 steps on a second and chunk k-2's params come out on a third, so the
    # two PCIe directions run at the same time.
    e2e = None
    if not args.no_e2e:
        idx = [i for i, o in enumerate(owned) if o]
        host_g = {i: grads[i].detach().cpu().pin_memory() for i in idx}
        host_p = {i: torch.empty(params[i].shape, dtype=params[i].dtype, pin_memory=True) for i in idx}
        h2d = sum(host_g[i].numel() * host_g[i].element_size() for i in idx)
        d2h = sum(host_p[i].numel() * host_p[i].element_size() for i in idx)
        n_chunks = min(len(idx), args.e2e_chunks)
        target = sum(params[i].numel() for i in idx) / max(n_chunks, 1)
        chunks, cur, acc = [], [], 0
        for i in sorted(idx, key=lambda i: -params[i].numel()):
            cur.append(i)
            acc += params[i].numel()
            if acc >= target and len(chunks) < n_chunks - 1:
                chunks.append(cur)
                cur, acc = [], 0
        if cur:
            chunks.append(cur)

        def chunk_opt(members):
            if wl.protect_output:
                return cls([(wl.tensors[i][0], params[i]) for i in members], protect_output=wl.protect_output, **kw)
            o = cls([{"params": [params[i] for i in members], "compress": wl.compress}], **kw)
            if wl.general_path:
                o._kernel_flags = _lib.SMO_FLAG_GENERAL_PATH
            return o

        opts = [chunk_opt(c) for c in chunks]
        s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        ev_in = [torch.cuda.Event() for _ in chunks]
        ev_comp = [torch.cuda.Event() for _ in chunks]
        ev_out = [torch.cuda.Event() for _ in chunks]

        def pipelined_step(first):
            for k, members in enumerate(chunks):
                with torch.cuda.stream(s_in):
                    if not first:
                        s_in.wait_event(ev_comp[k])  # the previous step has read these grads
                    for i in members:
                        grads[i].copy_(host_g[i], non_blocking=True)
                    ev_in[k].record(s_in)
                with torch.cuda.stream(s_comp):
                    s_comp.wait_event(ev_in[k])
                    if not first:
                        s_comp.wait_event(ev_out[k])  # the previous step's params are out
                    opts[k].step()
                    ev_comp[k].record(s_comp)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_comp[k])
                    for i in members:
                        host_p[i].copy_(params[i].detach(), non_blocking=True)
                    ev_out[k].record(s_out)

        for w_ in range(2):  # state init and warm-up of the chunk optimizers
            pipelined_step(w_ == 0)
        torch.cuda.synchronize()
        KE = args.e2e_steps
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for st_ in (s_in, s_comp, s_out):
            st_.wait_event(a)
        for _ in range(KE):
            pipelined_step(False)
        for st_ in (s_in, s_comp, s_out):
            stream.wait_stream(st_)
        b.record(stream)
        torch.cuda.synchronize()
        ems = a.elapsed_time(b) / KE
        if world > 1:
            t = torch.tensor([ems], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t[0])
        status = max(o.workspace_status() for o in opts)
        if status:
            raise RuntimeError(f"device status {status} in the e2e run")
        e2e = {"value": total_params / (ems * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": ems, "steps": KE, "chunks": len(chunks),
               "path": "SMO8bit.step() via the C ABI, one optimizer per chunk of tensors; pinned host grads "
                       "H2D, step and params D2H pipelined over chunks on three streams"}

    cpu = cpu_ref = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.dtype == "f32":
        cpu = cpu_baseline(wl, args.seed, args.cpu_sample_seconds)
        cpu_ref = reference_baseline(wl, args.seed, args.cpu_sample_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": f"{args.dtype}+int8", "data": "synthetic (seeded counter-hash N(0,0.02) params, N(0,1e-3) grads)",
            "config": dict(_config(wl, world, args.dtype), **({"shard": f"rank {args.shard_rank} of {shard_of}",
                                                   "params": my_params} if shard_of else {})),
            "hbm_gbs": (my_bytes if shard_of else sum(costs)) / (ms_per_step * 1e-3) / 1e9,
            "kernel_ms_per_step": step_ms,
            "host_ms_per_step": host_ms,
            "host_ms_max": host_ms_max,
            "roofline": roof,
            "cpu_baseline": cpu_ref or cpu,
            "cpu_baseline_port": cpu,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "clocks": clk,
            "impl": "ours",
        }
        if zero1:
            line["zero1"] = zero1
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
