#!/usr/bin/env python
"""Benchmark of the laya encoder forward on B200.

Metric: encoder tokens/s, reported on REAL tokens (padding is
never computed; padded tokens/s is reported beside it).  A step is one forward
of the workload.  The default workload is the --max-tokens 16384 budget
(configuration 2: 128 sequences x 128 padded tokens, real lengths U[24,128]).

  value     device-resident: the request is uploaded once (a plan) and each
            step replays the forward's CUDA graph; CUDA events on the engine
            stream around K steps, max over ranks.
  e2e       through the public call (Engine.forward -> laya_forward): host
            index arrays in, host logits/act out, every step; wall clock
            around K calls after a barrier, max over ranks.
  roofline  the dominant kernel family (the tcgen05 GEMM, all its launches):
            algorithmic real-token FLOPs / device time from CUDA events
            recorded after every launch over K more steps.

N GPUs (torchrun): one engine per GPU, each rank runs its own seeded batch
(seed = rank), no collective on the data path; weak scaling.

--impl reference: the reference's CPU algorithm (the C restatement in
oracle/, the Rust reference cannot be built here) on a bounded sample of the
same workload with all host threads; rank 0 only.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "encoder tokens/sec"
UNIT = "real tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="forward-16k", choices=["forward-16k", "long-state"])
    ap.add_argument("--cpu-sample", type=int, default=4, help="sequences in the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def workload(name, seed):
    from laya_rust_b200 import workloads
    return workloads.forward_16k(seed) if name == "forward-16k" else workloads.long_state(seed + 3)


def config_of(args, req, n):
    from laya_rust_b200 import workloads
    return {"workload": args.config, "model": "laya (ModernBERT-large 28L + 2L head), random-init f16 GGUF seed 0",
            "global_batch": req.n * n, "seq_len": req.l, "k_markers": req.k,
            "real_tokens_per_forward": workloads.real_tokens(req),
            "padded_tokens_per_forward": workloads.padded_tokens(req),
            "parallelism": f"request-dp{n}", "l2": "working set > L2 (843 MB f16 weights streamed per forward)"}


def sub_request(req, m):
    from laya_rust_b200.engine import Req
    n, l, k = req.n, req.l, req.k
    return Req(m, l, k, req.ids.reshape(n, l)[:m], req.att.reshape(n, l)[:m], req.mpos.reshape(n, k)[:m],
               req.mmask.reshape(n, k)[:m], req.qtype[:m])


def cpu_run(req, steps, warmup):
    """Times the oracle (the reference CPU algorithm) on `req`; returns seconds per step."""
    from laya_rust_b200 import modelgen
    from oracle.oracle import OracleModel
    m = OracleModel(modelgen.cached_model(seed=0))
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        m.forward(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    m.close()
    return statistics.mean(times)


def cpu_threads():
    v = os.environ.get("LAYA_CPU_THREADS")
    return int(v) if v and int(v) > 0 else os.cpu_count()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={','.join(map(str, gpus))}",
                                       f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f:
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1]))
                mx.append(float(c[2]))
            except ValueError:
                continue
            for nm, v in zip(names, c[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def run_reference(args):
    rank, _, world = env_rank()
    if rank != 0:
        return
    req = workload(args.config, 0)
    sample = sub_request(req, args.cpu_sample)
    from laya_rust_b200 import workloads
    real = workloads.real_tokens(sample)
    sec = cpu_run(sample, args.steps, args.warmup)
    v = real / sec
    cores = cpu_threads()
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded ids, random-init weights)",
            "impl": "reference", "config": config_of(args, req, args.gpus),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"first {args.cpu_sample} sequences of the {args.config} batch "
                                       f"({real} real / {sample.n * sample.l} padded tokens) per step; "
                                       "C restatement of the reference CPU backend (Rust reference not "
                                       "buildable: no cargo in the image)"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_b200(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from laya_rust_b200 import modelgen, workloads
    from laya_rust_b200.engine import Engine

    rank, local, world = env_rank()
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)

    def barrier():
        if world > 1:
            dist.barrier()

    def allmax(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def allsum(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    if rank == 0:
        path = modelgen.cached_model(seed=0)
    barrier()
    path = modelgen.cached_model(seed=0)
    eng = Engine(path, device=local)
    req = workload(args.config, rank)
    plan = eng.plan(req)
    plan.capture()
    real, launches, upload = plan.stats()
    stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))

    for _ in range(args.warmup):
        plan.run()
    torch.cuda.synchronize()
    clocks = ClockSampler(list(range(world))) if rank == 0 else None
    barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        plan.run()
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = t0.elapsed_time(t1)
    ms_max = allmax(ms)
    clk = clocks.stop() if clocks else None
    out = plan.outputs()
    assert np.all(np.isfinite(out.logits)) and np.all(np.isfinite(out.act))

    total_real = allsum(real) * args.steps
    total_padded = allsum(req.n * req.l) * args.steps
    value = total_real / (ms_max / 1e3)

    # roofline of the dominant kernel family from per-launch events
    prof = plan.profile(args.steps)
    gemm_kinds = ["gemm_qkv", "gemm_attn_out", "gemm_ffn_in_geglu", "gemm_ffn_out", "gemm_head_scorer"]
    gemm_ms = sum(prof[k][0] for k in gemm_kinds)
    gemm_launches = sum(prof[k][1] for k in gemm_kinds)
    flops = workloads.gemm_flops(req) * args.steps
    pk, pk_src = peaks()
    achieved = flops / (gemm_ms / 1e3) / 1e12
    peak = pk["bf16_tflops_sustained"]
    prof_total = sum(v[0] for v in prof.values())
    kernels = {k: {"ms_per_step": v[0] / args.steps, "launches_per_step": v[1] // args.steps,
                   "share": v[0] / prof_total} for k, v in prof.items()}
    kernels["attention"]["tflops"] = workloads.attention_flops(req) * args.steps / (prof["attention"][0] / 1e3) / 1e12

    # e2e through the public call: host arrays in, host logits/act out
    for _ in range(2):
        eng.forward(req)
    barrier()
    e0 = time.perf_counter()
    for _ in range(args.steps):
        eng.forward(req)
    e_sec = allmax(time.perf_counter() - e0)
    barrier()
    e2e = {"value": total_real / e_sec, "unit": UNIT, "h2d_bytes_per_step": upload,
           "d2h_bytes_per_step": 4 * (req.n * req.k + 2 * req.n), "ms_per_step": e_sec * 1e3 / args.steps,
           "path": "laya_forward (validate + compact on host, one pinned H2D, graph-free launch, D2H)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = sub_request(req, args.cpu_sample)
        sec = cpu_run(sample, 1, 0)
        cpu = {"value": workloads.real_tokens(sample) / sec, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
               "sample": f"first {args.cpu_sample} sequences of the batch ({workloads.real_tokens(sample)} real / "
                         f"{sample.n * sample.l} padded tokens), one forward"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f16 operands, f32 accumulate",
                "data": "synthetic (seeded ids, random-init weights)",
                "padded_tokens_per_s": total_padded / (ms_max / 1e3),
                "config": config_of(args, req, world),
                "roofline": {"bound": "tensor", "kernel": "gemm_tc_kernel (tcgen05, all launches)",
                             "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                             "peak_source": f"{pk_src} bf16_tflops_sustained", "traffic": None,
                             "launches_per_step": gemm_launches // args.steps,
                             "flops_per_step": workloads.gemm_flops(req)},
                "kernels": kernels, "e2e": e2e, "gpu_launches": launches * args.steps,
                "clocks": clk, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    plan.close()
    eng.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
