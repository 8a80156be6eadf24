#!/usr/bin/env python
"""Benchmark of the laya encoder forward on B200.

Metric: encoder tokens/s, counted on REAL tokens (padding is
never computed; padded tokens/s is reported beside it), plus request latency.
Workloads (--config), all seeded synthetic data on a random-init f16 model:

  forward-16k  config 2 (default): the --max-tokens 16384 budget, 128
               sequences x 128 padded tokens, real lengths U[24,128].  A step
               is one forward.
  long-state   config 3: 8 sequences x 512 tokens.  A step is one forward.
  layer        config 1: one encoder layer alone on 32 sequences padded to
               256 (real lengths U[16,256]), f16 N(0,1) activations; global
               layer 0 and local layer 1 timed separately, L2 flushed before
               every step (the layer's weights and activations fit in L2).
  request      config 0: one System One request (JSON: 48-word state, a
               choice question with 2 criteria, a noul question) through the
               C++ front end (planned once; per step group_by_budget,
               build_batch, forward, scoring, response JSON); the metric is
               its latency (ms, p50 over the steps).
  stream       config 4: 4096 seeded JSON requests planned by the C++ front end
               on the host threads, assigned to the GPUs greedily by token
               cost; each GPU packs its share across requests into
               <=16384-token forwards.  Steps are the forwards of one pass.
  gemm         diagnostic: the encoder's four GEMM shapes at 9872 rows, this
               build's kernel with its fused epilogues against cuBLAS (torch)
               on the same shapes and operands, L2 flushed per launch.

  value     device-resident: requests uploaded once (plans), forwards
            enqueued back to back (CUDA graph replay where one plan repeats);
            CUDA events on the engine stream, max over ranks.
  e2e       through the public call (Engine.forward -> laya_forward): host
            index arrays in, host logits/act out, every step; wall clock
            after a barrier, max over ranks.
  roofline  the dominant kernel family (the tcgen05 GEMM, all its launches):
            algorithmic real-token FLOPs / device time from CUDA events
            recorded after every launch over K more steps.

N GPUs (torchrun): one engine per GPU, each rank works on its own requests,
no collective on the data path (NCCL only for the barrier and the final
reductions); weak scaling.

--impl reference: the reference's CPU algorithm (the C restatement in
oracle/, the Rust reference cannot be built here) on a bounded sample of the
same workload with all host threads; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
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
LAT_METRIC = "request latency p50"
CONFIGS = ["forward-16k", "long-state", "layer", "request", "stream", "gemm"]
DATA = "synthetic (seeded ids, random-init weights)"
MODEL = "laya (ModernBERT-large 28L + 2L head), random-init f16 GGUF seed 0"
LAYERS = (("global", 0), ("local", 1))
# Mean DRAM bytes (read + write) per GEMM launch from one ncu capture
# (--set full) of layer 1's four GEMMs in the 16384-token forward (cold L2).
GEMM_TRAFFIC = 58.4e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="forward-16k", choices=CONFIGS)
    ap.add_argument("--cpu-sample", type=int, default=4, help="sequences in the CPU baseline sample")
    ap.add_argument("--requests", type=int, default=4096, help="requests in the stream configuration")
    ap.add_argument("--stream-window", type=int, default=0,
                    help="stream: group questions by length within windows of this many consecutive "
                         "requests (0, the default: pack in dispatch order)")
    ap.add_argument("--stream-requests", type=int, default=1024,
                    help="forward-16k: requests of the request-stream sweep carried in the line's `stream` key "
                         "(0: none)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def pct(sorted_vals, p):
    """main.rs:559-565: element round(p/100 * (n-1)) of the sorted sample."""
    if not sorted_vals:
        return 0.0
    i = int(math.floor(p / 100.0 * (len(sorted_vals) - 1) + 0.5))
    return sorted_vals[min(i, len(sorted_vals) - 1)]


def latency_summary(ms):
    s = sorted(ms)
    return {"min": s[0], "p50": pct(s, 50), "p90": pct(s, 90), "p99": pct(s, 99), "max": s[-1],
            "mean": sum(s) / len(s), "count": len(s)}


def workload(name, seed):
    from laya_rust_b200 import workloads
    if name == "forward-16k":
        return workloads.forward_16k(seed)
    if name == "long-state":
        return workloads.long_state(seed + 3)
    if name == "layer":
        return workloads.layer_batch(seed + 1)
    raise ValueError(name)


def config_of(args, req, n):
    from laya_rust_b200 import workloads
    return {"workload": args.config, "model": MODEL,
            "global_batch": req.n * n, "seq_len": req.l, "k_markers": req.k,
            "real_tokens_per_forward": workloads.real_tokens(req),
            "padded_tokens_per_forward": workloads.padded_tokens(req),
            "parallelism": f"request-dp{n}", "l2": "working set > L2 (843 MB f16 weights streamed per forward)"}


def sub_request(req, m):
    from laya_rust_b200.engine import Req
    n, l, k = req.n, req.l, req.k
    return Req(m, l, k, req.ids.reshape(n, l)[:m], req.att.reshape(n, l)[:m], req.mpos.reshape(n, k)[:m],
               req.mmask.reshape(n, k)[:m], req.qtype[:m])


def cpu_threads():
    v = os.environ.get("LAYA_CPU_THREADS")
    return int(v) if v and int(v) > 0 else os.cpu_count()


def oracle_model():
    from laya_rust_b200 import modelgen
    from oracle.oracle import OracleModel
    return OracleModel(modelgen.cached_model(seed=0))


def cpu_run(req, steps, warmup):
    """Times the oracle (the reference CPU algorithm) on `req`; returns seconds per step."""
    m = oracle_model()
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        m.forward(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    m.close()
    return statistics.mean(times)


def cpu_layer_run(req, steps, warmup):
    """Times the oracle's one-layer call (global then local layer) on `req`;
    returns seconds per layer."""
    import numpy as np
    m = oracle_model()
    x = np.random.default_rng(1).standard_normal((req.n * req.l, 1024)).astype(np.float16).astype(np.float32)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        for _, layer in LAYERS:
            m.encoder_layer(req.n, req.l, req.att, layer, x)
        if i >= warmup:
            times.append((time.perf_counter() - t0) / len(LAYERS))
    m.close()
    return statistics.mean(times)


def cpu_request_run(requests, steps, warmup):
    """Times run_all (main.rs:520-557) of each request on the reference CPU
    algorithm: the restated front end (oracle/frontend_ref.py) planning,
    batching and scoring around the C oracle's forward.  Returns per-step
    milliseconds and the tokens of one step."""
    from laya_rust_b200 import tokgen
    from oracle import frontend_ref as F
    tok = F.Tokenizer(tokgen.tokenizer_json(0))
    m = oracle_model()
    times, toks = [], 0
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        toks = 0
        for req in requests:
            out = F.run_all(m.forward, tok, req)
            toks += out["usage"]["input_tokens"]
        if i >= warmup:
            times.append((time.perf_counter() - t0) * 1e3)
    m.close()
    return times, toks


def request_words():
    from laya_rust_b200 import tokgen, workloads
    return workloads.vocab_words(tokgen.tokenizer_json(0))


def stream_sample():
    """The CPU sample of the stream: request 0 with its first 4 questions."""
    from laya_rust_b200 import workloads
    req = workloads.request_stream_json(request_words(), 1, 4)[0]
    keep = list(req["questions"])[:4]
    return {"state": req["state"], "questions": {k: req["questions"][k] for k in keep}}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms; the
    constructor returns once the first sample is written, so sampling is live
    when the timed region starts."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={','.join(map(str, gpus))}",
                                       f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
            return
        t_end = time.time() + 5.0
        while time.time() < t_end and self.p.poll() is None and os.path.getsize(self.f.name) == 0:
            time.sleep(0.02)

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


def base_line(args, metric, value, unit, n, ms_per_step, config, hib=True, **extra):
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": hib, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 operands, f32 accumulate", "data": DATA, "config": config}
    line.update(extra)
    return line


# ---- reference arm -------------------------------------------------------------------

def reference_gpu_schedule(req, iters=3):
    """The reference's GPU algorithm on this GPU, for context beside the CPU
    arm: its own CUDA kernels (src/backend/cuda/kernels.rs) and cuBLAS FP32
    op sequence (src/backend/cuda/mod.rs:466-812) on the full padded batch,
    built into oracle/_ref/ from the reference tree.  None without a GPU or
    without that build."""
    try:
        import torch
        if not torch.cuda.is_available():
            return None
        from oracle import ref_gpu
        if not ref_gpu.available():
            return {"unavailable": "oracle/_ref/libref_gpu.so not built (needs the reference tree at build time)"}
        from laya_rust_b200 import workloads
        m = oracle_model()
        rg = ref_gpu.RefGpuSchedule(m)
        ms = rg.time(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype, iters)
        rg.close()
        m.close()
        real = workloads.real_tokens(req)
        return {"value": real / (ms / 1e3), "unit": UNIT, "ms_per_forward": ms, "iters": iters,
                "what": "reference kernels + cuBLAS FP32 (default math) on the padded batch, device time per "
                        "forward incl. its request copies"}
    except Exception as e:  # a baseline for context only: never fail the arm
        return {"unavailable": f"{type(e).__name__}: {e}"}


def run_reference(args):
    rank, _, world = env_rank()
    if rank != 0:
        return
    from laya_rust_b200 import workloads
    cores = cpu_threads()
    note = "C restatement of the reference CPU backend (Rust reference not buildable: no cargo in the image)"
    if args.config in ("forward-16k", "long-state", "layer"):
        req = workload(args.config, 0)
        sample = sub_request(req, args.cpu_sample if args.config != "layer" else 2 * args.cpu_sample)
        real = workloads.real_tokens(sample)
        if args.config == "layer":
            sec = cpu_layer_run(sample, args.steps, args.warmup)
            what = "one encoder layer (global layer 0 and local layer 1 alternately)"
        else:
            sec = cpu_run(sample, args.steps, args.warmup)
            what = "one forward"
        v = real / sec
        cfg = config_of(args, req, args.gpus)
        sample_txt = (f"first {sample.n} sequences of the {args.config} batch ({real} real / "
                      f"{sample.n * sample.l} padded tokens), {what} per step; {note}")
        line = base_line(args, METRIC, v, UNIT, args.gpus, sec * 1e3, cfg, dtype="f32", impl="reference")
    else:
        req = workloads.single_request_json(request_words(), 0) if args.config == "request" else stream_sample()
        times, toks = cpu_request_run([req], args.steps, args.warmup)
        lat = latency_summary(times)
        nq = len(req["questions"])
        if args.config == "request":
            v, unit, metric, hib = lat["p50"], "ms", LAT_METRIC, False
        else:
            v, unit, metric, hib = toks / (lat["mean"] / 1e3), UNIT, METRIC, True
        cfg = {"workload": args.config, "model": MODEL, "questions": nq, "real_tokens": toks}
        sample_txt = (f"{'the request' if args.config == 'request' else 'request 0 with its first 4 questions'} "
                      f"({nq} questions, {toks} tokens) through run_all (restated front end + C oracle forward) "
                      f"per step; {note}")
        line = base_line(args, metric, v, unit, args.gpus, lat["mean"], cfg, hib=hib, dtype="f32",
                         impl="reference", latency_ms=lat)
    line["cpu_baseline"] = {"value": line["value"], "unit": line["unit"], "cores": cores, "kind": "port",
                            "sample": sample_txt}
    if args.config in ("forward-16k", "long-state"):
        line["reference_gpu_schedule"] = reference_gpu_schedule(workload(args.config, 0))
    line["e2e"] = {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    print(json.dumps(line), flush=True)


# ---- B200 arm ------------------------------------------------------------------------

class Dist:
    def __init__(self):
        import torch
        self.torch = torch
        self.rank, self.local, self.world = env_rank()
        self.cuda = torch.cuda.is_available()
        if self.world > 1:
            import torch.distributed as dist
            from datetime import timedelta
            # short: a rank that waits for a peer that never comes ends with an error
            if self.cuda:
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                        device_id=torch.device("cuda", self.local))
            else:  # host-only runs (tests of the collective steps)
                dist.init_process_group("gloo", timeout=timedelta(seconds=60))
            self.dist = dist
        if self.cuda:
            torch.cuda.set_device(self.local)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def _reduce(self, x, op):
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device="cuda" if self.cuda else "cpu")
        self.dist.all_reduce(t, op=op)
        return float(t.item())

    def allmax(self, x):
        return self._reduce(x, self.dist.ReduceOp.MAX if self.world > 1 else None)

    def allsum(self, x):
        return self._reduce(x, self.dist.ReduceOp.SUM if self.world > 1 else None)

    def gather(self, obj):
        if self.world == 1:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def open_engine(d):
    from laya_rust_b200 import modelgen
    from laya_rust_b200.engine import Engine
    if d.rank == 0:
        modelgen.cached_model(seed=0)
    d.barrier()
    return Engine(modelgen.cached_model(seed=0), device=d.local)


def ext_stream(d, eng):
    return d.torch.cuda.ExternalStream(eng.stream(), device=d.torch.device("cuda", d.local))


def cpu_baseline_line(value, unit, sample):
    return {"value": value, "unit": unit, "cores": cpu_threads(), "kind": "port", "sample": sample}


def run_forward(args, d, eng):
    """forward-16k / long-state: one forward of a fixed batch per step."""
    import numpy as np
    from laya_rust_b200 import workloads
    torch = d.torch
    req = workload(args.config, d.rank)
    plan = eng.plan(req)
    plan.capture()
    real, launches, upload = plan.stats()
    stream = ext_stream(d, eng)

    for _ in range(args.warmup):
        plan.run()
    torch.cuda.synchronize()
    clocks = ClockSampler(list(range(d.world))) if d.rank == 0 else None
    d.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        plan.run()
    t1.record(stream)
    torch.cuda.synchronize()
    d.barrier()
    ms = t0.elapsed_time(t1)
    ms_max = d.allmax(ms)
    clk = clocks.stop() if clocks else None
    out = plan.outputs()
    parity = fixture_parity(args.config, req, out)

    total_real = d.allsum(real) * args.steps
    total_padded = d.allsum(req.n * req.l) * args.steps
    value = total_real / (ms_max / 1e3)

    # roofline of the dominant kernel family from per-launch events
    prof = plan.profile(args.steps)
    gemm_kinds = ["gemm_qkv", "gemm_attn_out", "gemm_ffn_in_geglu", "gemm_ffn_out", "gemm_head_scorer"]
    gemm_ms = sum(prof[k][0] for k in gemm_kinds)
    gemm_launches = sum(prof[k][1] for k in gemm_kinds)
    flops = workloads.gemm_flops(req) * args.steps
    pk, pk_src = peaks()
    achieved = flops / (gemm_ms / 1e3) / 1e12
    # the burst figure (cuBLAS timed alone at the clocks this run also holds);
    # the sustained figure was measured at a lower median SM clock under the
    # power cap, and is reported beside it only
    peak = pk["bf16_tflops"]
    sustained = pk.get("bf16_tflops_sustained")
    sustained_mhz = (pk.get("clocks_under_load") or {}).get("sm_mhz_median")
    prof_total = sum(v[0] for v in prof.values())
    fwd_flops = workloads.gemm_flops(req) + workloads.attention_flops(req)
    forward_frac = fwd_flops / (ms_max / args.steps / 1e3) / 1e12 / peak
    kernels = {k: {"ms_per_step": v[0] / args.steps, "launches_per_step": v[1] // args.steps,
                   "share": v[0] / prof_total} for k, v in prof.items()}
    kernels["attention"]["tflops"] = workloads.attention_flops(req) * args.steps / (prof["attention"][0] / 1e3) / 1e12

    # e2e through the public call: host arrays in, host logits/act out
    for _ in range(2):
        eng.forward(req)
    d.barrier()
    e_ms = []
    for _ in range(args.steps):
        e0 = time.perf_counter()
        eng.forward(req)
        e_ms.append((time.perf_counter() - e0) * 1e3)
    e_sec = d.allmax(sum(e_ms) / 1e3)
    d.barrier()
    e2e = {"value": total_real / e_sec, "unit": UNIT, "h2d_bytes_per_step": upload,
           "d2h_bytes_per_step": 4 * (req.n * req.k + 2 * req.n), "ms_per_step": e_sec * 1e3 / args.steps,
           "latency_ms": latency_summary(e_ms),
           "path": "laya_forward (validate + compact on host, one pinned H2D, graph-free launch, D2H)"}

    # every rank: the bounded request-stream sweep (collective steps inside)
    stream_info = stream_key(args, d, eng) if args.config == "forward-16k" else None

    cpu = None
    if d.rank == 0 and d.world == 1 and not args.no_cpu_baseline:
        sample = sub_request(req, args.cpu_sample)
        sec = cpu_run(sample, 1, 0)
        cpu = cpu_baseline_line(workloads.real_tokens(sample) / sec, UNIT,
                                f"first {args.cpu_sample} sequences of the batch ({workloads.real_tokens(sample)} "
                                f"real / {sample.n * sample.l} padded tokens), one forward")

    if d.rank == 0:
        line = base_line(args, METRIC, value, UNIT, d.world, ms_max / args.steps, config_of(args, req, d.world),
                         padded_tokens_per_s=total_padded / (ms_max / 1e3),
                         roofline={"bound": "tensor", "kernel": "gemm_tc_kernel (tcgen05, all launches)",
                                   "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                                   "peak_source": f"{pk_src} bf16_tflops (burst)",
                                   "frac_of_sustained": achieved / sustained if sustained else None,
                                   "sustained_peak": sustained, "sustained_peak_sm_mhz": sustained_mhz,
                                   "forward_frac": forward_frac,
                                   "forward_tflops": forward_frac * peak,
                                   "traffic": GEMM_TRAFFIC if args.config == "forward-16k" else None,
                                   "traffic_source": "ncu, layer 1's four GEMMs of the 16384-token forward, "
                                                     "cold L2 (ncu --set full, gemm_tc_kernel, -s 4 -c 4)",
                                   "launches_per_step": gemm_launches // args.steps,
                                   "flops_per_step": workloads.gemm_flops(req)},
                         kernels=kernels, e2e=e2e, gpu_launches=launches * args.steps, clocks=clk,
                         cpu_baseline=cpu, parity=parity, stream=stream_info)
        print(json.dumps(line), flush=True)
    plan.close()


FIXTURES = os.path.join(ROOT, "tests", "golden", "fullsize_outputs.json")


def fixture_parity(config, req, out):
    """Checks a benchmarked forward against the reference algorithm's output
    committed for that exact batch (tests/golden/fullsize_outputs.json, made
    by the C oracle): the contract's tolerance (max-abs 2e-2, rel 1e-2),
    masked markers -10000, identical argmax.  Rank 0 runs the fixture's
    batch (seed 0); other ranks' batches have no fixture and are checked for
    finite outputs only.  Raises on a mismatch, so no number is printed for
    a wrong forward."""
    import hashlib
    import numpy as np
    assert np.all(np.isfinite(out.logits)) and np.all(np.isfinite(out.act)), "non-finite outputs"
    entry = None
    if config in ("forward-16k", "long-state") and os.path.exists(FIXTURES):
        h = hashlib.sha256()
        for a in (req.ids, req.att, req.mpos, req.mmask, req.qtype):
            h.update(np.ascontiguousarray(a, dtype="<i8").tobytes())
        h.update(f"{req.n},{req.l},{req.k}".encode())
        entry = next((e for e in json.load(open(FIXTURES)).get(config, []) if e["sha256"] == h.hexdigest()), None)
    if entry is None:
        return {"checked": "finite outputs only (no fixture for this rank's batch)"}
    mm = (req.mmask != 0).reshape(req.n, req.k)
    gl, wl = out.logits.reshape(req.n, req.k), np.array(entry["logits"], np.float32).reshape(req.n, req.k)
    ga, wa = out.act, np.array(entry["act"], np.float32)
    assert np.all(gl[~mm] == -10000.0), "masked marker logits must be -10000"
    el, ea = np.abs(gl[mm] - wl[mm]), np.abs(ga - wa)
    assert el.max() <= 2e-2 and np.all(el <= 2e-2 + 1e-2 * np.abs(wl[mm])), f"logits off by {el.max()}"
    assert ea.max() <= 2e-2 and np.all(ea <= 2e-2 + 1e-2 * np.abs(wa)), f"act off by {ea.max()}"
    rows = [b for b in range(req.n) if mm[b].sum() > 1]
    same = sum(int(np.argmax(gl[b][mm[b]]) == np.argmax(wl[b][mm[b]])) for b in rows)
    assert same == len(rows), f"argmax differs on {len(rows) - same} rows"
    return {"checked": f"against the C oracle's output for this batch ({os.path.relpath(FIXTURES, ROOT)})",
            "max_abs_dlogit": float(el.max()), "max_abs_dact": float(ea.max()),
            "argmax_equal_rows": f"{same}/{len(rows)}"}


def layer_launches(req):
    """Kernels laya_plan_run_layer enqueues: two row norms, four GEMMs and one
    attention launch per kind of sequence present (at most 128 tokens: the
    single-pass kernel over packed tiles; longer: the flash kernel)."""
    lens = (req.att.reshape(req.n, req.l) != 0).sum(1)
    return 6 + int((lens <= 128).any()) + int((lens > 128).any())


def layer_flops(req, global_layer):
    import numpy as np
    lens = (req.att.reshape(req.n, req.l) != 0).sum(1).astype(np.float64)
    real = float(lens.sum())
    gemm = 2.0 * real * (1024 * 3072 + 1024 * 1024 + 1024 * 5248 + 2624 * 1024)
    if global_layer:
        pairs = float((lens ** 2).sum())
    else:
        pairs = 0.0
        for r in lens.astype(np.int64):
            i = np.arange(r)
            pairs += float((np.minimum(i + 64, r - 1) - np.maximum(i - 64, 0) + 1).sum())
    return gemm, 4.0 * 1024 * pairs


def run_layer(args, d, eng):
    """Config 1: one encoder layer alone, L2 flushed before every timed step."""
    import numpy as np
    from laya_rust_b200 import workloads
    torch = d.torch
    req = workload("layer", d.rank)
    plan = eng.plan(req)
    real = plan.stats()[0]
    x = np.random.default_rng(1 + d.rank).standard_normal((real, 1024)).astype(np.float16).astype(np.float32)
    stream = ext_stream(d, eng)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")   # 256 MiB > 126 MB L2
    clocks = ClockSampler(list(range(d.world))) if d.rank == 0 else None
    per_kind = {}
    for kind, layer in LAYERS:
        plan.set_hidden(x)
        for _ in range(args.warmup):
            plan.run_layer(layer)
        torch.cuda.synchronize()
        d.barrier()
        evs = []
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                flush.zero_()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                plan.run_layer(layer)
                b.record(stream)
                evs.append((a, b))
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
        per_kind[kind] = {"layer": layer, "ms": d.allmax(ms)}
    clk = clocks.stop() if clocks else None
    y = plan.hidden()
    assert np.all(np.isfinite(y))

    pk, pk_src = peaks()
    peak = pk["bf16_tflops"]
    for kind, layer in LAYERS:
        g, a = layer_flops(req, kind == "global")
        per_kind[kind]["tflops"] = (g + a) / (per_kind[kind]["ms"] / 1e3) / 1e12
        per_kind[kind]["gemm_flops"], per_kind[kind]["attention_flops"] = g, a
    mean_ms = sum(v["ms"] for v in per_kind.values()) / len(per_kind)
    total_real = d.allsum(real)
    value = total_real / (mean_ms / 1e3)
    flops = sum(v["gemm_flops"] + v["attention_flops"] for v in per_kind.values())
    achieved = flops / (sum(v["ms"] for v in per_kind.values()) / 1e3) / 1e12

    # e2e: host residual stream in, one layer, host residual stream out
    d.barrier()
    e_ms = []
    for i in range(args.steps):
        kind, layer = LAYERS[i % len(LAYERS)]
        e0 = time.perf_counter()
        plan.set_hidden(x)
        plan.run_layer(layer)
        plan.hidden()
        e_ms.append((time.perf_counter() - e0) * 1e3)
    e_sec = d.allmax(sum(e_ms) / 1e3)
    e2e = {"value": total_real * args.steps / e_sec, "unit": UNIT, "h2d_bytes_per_step": real * 4096,
           "d2h_bytes_per_step": real * 4096, "ms_per_step": e_sec * 1e3 / args.steps,
           "path": "laya_plan_set_hidden (H2D f32 stream) + laya_plan_run_layer + laya_plan_hidden (D2H)"}

    cpu = None
    if d.rank == 0 and d.world == 1 and not args.no_cpu_baseline:
        sample = sub_request(req, 2 * args.cpu_sample)
        sec = cpu_layer_run(sample, 1, 0)
        cpu = cpu_baseline_line(workloads.real_tokens(sample) / sec, UNIT,
                                f"first {sample.n} sequences ({workloads.real_tokens(sample)} real / "
                                f"{sample.n * sample.l} padded tokens), layers 0 and 1 once each")
    padded_all = d.allsum(req.n * req.l)   # every rank takes the same collective steps
    if d.rank == 0:
        cfg = config_of(args, req, d.world)
        cfg["l2"] = "flushed (256 MiB memset) before every timed step"
        cfg["layers"] = {k: v for k, v in LAYERS}
        line = base_line(args, METRIC + " (one encoder layer)", value, UNIT, d.world, mean_ms, cfg,
                         padded_tokens_per_s=padded_all / (mean_ms / 1e3), layers=per_kind,
                         roofline={"bound": "tensor", "kernel": "one encoder layer (4 tcgen05 GEMMs, attention, 2 norms)",
                                   "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                                   "peak_source": f"{pk_src} bf16_tflops (burst: a layer is timed alone)",
                                   "traffic": None},
                         e2e=e2e, gpu_launches=layer_launches(req) * args.steps * len(LAYERS), clocks=clk,
                         cpu_baseline=cpu)
        print(json.dumps(line), flush=True)
    plan.close()


def run_request(args, d, eng):
    """Config 0: one System One request (JSON) through the C++ front end and
    the engine.  As the reference's bench (main.rs:661-694: prepare once,
    then time run_all), the request is planned (parsed, tokenized, laid out)
    once; each step packs it (group_by_budget), builds the batches, runs
    laya_forward per forward, scores and writes the response JSON.  The
    planning time is reported beside it."""
    from laya_rust_b200 import frontend as FE, modelgen, workloads
    torch = d.torch
    tok = FE.Tokenizer(gguf_path=modelgen.cached_model(seed=0))
    req = workloads.single_request_json(request_words(), 0)
    plan_ms = []
    for _ in range(max(args.steps, 5)):
        t = time.perf_counter()
        FE.Requests(tok, [req], threads=1).close()
        plan_ms.append((time.perf_counter() - t) * 1e3)
    rq = FE.Requests(tok, [req], threads=1)
    nf = rq.pack(16384, False)
    batches = [rq.batch(f) for f in range(nf)]
    toks = sum(int(b.att.sum()) for b in batches)

    # device time of the request's forwards (plans replayed as graphs)
    plans = [eng.plan(b) for b in batches]
    for p in plans:
        p.capture()
    stream = ext_stream(d, eng)
    for _ in range(args.warmup):
        for p in plans:
            p.run()
    torch.cuda.synchronize()
    d.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        for p in plans:
            p.run()
    t1.record(stream)
    torch.cuda.synchronize()
    dev_ms = d.allmax(t0.elapsed_time(t1) / args.steps)
    launches = sum(p.stats()[1] for p in plans)
    upload = sum(p.stats()[2] for p in plans)
    # the GEMM family's share from per-launch events: at 179 rows it runs far
    # below both rooflines (per-launch latency bound); reported as measured
    gemm_kinds = ["gemm_qkv", "gemm_attn_out", "gemm_ffn_in_geglu", "gemm_ffn_out", "gemm_head_scorer"]
    gemm_ms, gemm_launches, flops = 0.0, 0, 0.0
    for p, b in zip(plans, batches):
        prof = p.profile(args.steps)
        gemm_ms += sum(prof[k][0] for k in gemm_kinds) / args.steps
        gemm_launches += sum(prof[k][1] for k in gemm_kinds) // args.steps
        flops += workloads.gemm_flops(b)
    for p in plans:
        p.close()
    pk, pk_src = peaks()
    achieved = flops / (gemm_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "kernel": "gemm_tc_kernel (tcgen05, all launches)", "achieved": achieved,
                "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                "peak_source": f"{pk_src} bf16_tflops", "traffic": None,
                "launches_per_step": gemm_launches, "gemm_ms_per_step": gemm_ms,
                "regime": "per-launch latency: 256-row tiles fill at most 21 of 74 clusters "
                          "(the residual GEMMs split K)"}

    def run_all():
        for f in range(rq.pack(16384, False)):
            out = eng.forward(rq.batch(f))
            rq.score(f, out.logits, out.act)
        return rq.response_text(0)

    clocks = ClockSampler(list(range(d.world))) if d.rank == 0 else None
    for _ in range(args.warmup):
        run_all()
    d.barrier()
    times = []
    for _ in range(args.steps):
        e0 = time.perf_counter()
        resp = run_all()
        times.append((time.perf_counter() - e0) * 1e3)
    clk = clocks.stop() if clocks else None
    assert json.loads(resp)["usage"]["input_tokens"] == toks
    lat = latency_summary(times)
    p50 = d.allmax(lat["p50"])

    cpu = None
    if d.rank == 0 and d.world == 1 and not args.no_cpu_baseline:
        ct, _ = cpu_request_run([req], 1, 0)
        cpu = cpu_baseline_line(ct[0], "ms", f"the same request ({len(req['questions'])} questions, {toks} tokens) "
                                             "through run_all (restated front end + C oracle forward), one run")
    if d.rank == 0:
        cfg = {"workload": "request", "model": MODEL, "questions": len(req["questions"]), "forwards": nf,
               "real_tokens": toks, "seq_lens": [int(x) for b in batches for x in b.att.reshape(b.n, b.l).sum(1)],
               "parallelism": f"replicas{d.world}", "l2": "working set > L2 (843 MB f16 weights streamed per forward)"}
        e2e = {"value": p50, "unit": "ms", "h2d_bytes_per_step": upload,
               "d2h_bytes_per_step": sum(4 * (b.n * b.k + 2 * b.n) for b in batches),
               "path": "C++ front end (pack, build_batch) -> laya_forward per forward -> score -> response JSON"}
        line = base_line(args, LAT_METRIC, p50, "ms", d.world, lat["mean"], cfg, hib=False,
                         latency_ms=lat, device_ms_per_request=dev_ms,
                         frontend_plan_ms=statistics.median(plan_ms),
                         tokens_per_s=toks / (lat["mean"] / 1e3), e2e=e2e, roofline=roofline,
                         gpu_launches=launches * args.steps, clocks=clk, cpu_baseline=cpu)
        print(json.dumps(line), flush=True)
    rq.close()
    tok.close()


def stream_pass(args, d, eng, n_requests, window, warmup):
    """One pass over the first `n_requests` requests of the request stream
    (configuration 4, JSON) through the C++ front end: every rank plans all
    of them on its host threads to learn their token costs, takes the share
    the greedy cost assignment gives it, and packs its questions across
    requests into <=16384-token forwards in dispatch order (window W > 0:
    grouped by length within windows of W consecutive requests; measured
    2.4% more tokens/s for 2.8x the median service latency at W = 64, so not
    the default).  The forwards run once device-resident (plans, CUDA events,
    max over ranks), then once through the public call with scoring and
    response JSON (wall clock).  Every rank takes the same collective steps;
    the returned figures are whole-job aggregates."""
    from laya_rust_b200 import frontend as FE, modelgen, workloads
    torch = d.torch
    tok = FE.Tokenizer(gguf_path=modelgen.cached_model(seed=0))
    texts = [json.dumps(r) for r in workloads.request_stream_json(request_words(), n_requests, 4)]
    t = time.perf_counter()
    allq = FE.Requests(tok, texts, threads=0)
    plan_all_s = time.perf_counter() - t
    cost = [0] * len(texts)
    for i in range(allq.questions()):
        r, ln, _, _ = allq.question_shape(i)
        cost[r] += ln
    allq.close()
    mine = workloads.assign_by_cost(cost, d.world)[d.rank]   # greedy by token cost, in dispatch order
    t = time.perf_counter()
    rq = FE.Requests(tok, [texts[i] for i in mine], threads=0)
    plan_s = time.perf_counter() - t
    nf = rq.pack_windows(16384, window) if window > 0 else rq.pack(16384, True)
    batches = [rq.batch(f) for f in range(nf)]
    fq = [rq.forward_questions(f) for f in range(nf)]
    q_req = [rq.question_shape(i)[0] for i in range(rq.questions())]
    plans = [eng.plan(b) for b in batches]
    real = sum(p.stats()[0] for p in plans)
    upload = sum(p.stats()[2] for p in plans)
    padded = sum(b.n * b.l for b in batches)
    stream = ext_stream(d, eng)

    # warm-up: the forwards with the most rows, markers, sequences and the
    # longest rows (they size the activation arena and the RoPE tables), then
    # the first W
    idx = range(len(plans))
    big = {max(idx, key=lambda i: plans[i].stats()[0]), max(idx, key=lambda i: batches[i].n * batches[i].k),
           max(idx, key=lambda i: batches[i].n), max(idx, key=lambda i: batches[i].l)} if plans else set()
    for i in sorted(big) + list(range(min(warmup, len(plans)))):
        plans[i].run()
    torch.cuda.synchronize()
    clocks = ClockSampler(list(range(d.world))) if d.rank == 0 else None
    d.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for p in plans:
        p.run()
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    ms_max = d.allmax(ms)
    launches = sum(p.stats()[1] for p in plans)
    for p in plans:
        p.close()

    # e2e: every forward through laya_forward and the C++ scorer, then every
    # response.  A request's service latency runs from the start of the
    # forward holding its first question to the end of the one holding its
    # last; its completion latency is measured from the start of the pass
    # (all requests queued at t = 0).
    d.barrier()
    start = time.perf_counter()
    t_beg, t_end = [], []
    for f, b in enumerate(batches):
        t_beg.append(time.perf_counter() - start)
        out = eng.forward(b)
        rq.score(f, out.logits, out.act)
        t_end.append(time.perf_counter() - start)
    for r in range(len(mine)):
        rq.response_text(r)
    e_sec = d.allmax(time.perf_counter() - start)
    clk = clocks.stop() if clocks else None
    first, last = {}, {}
    for f, qs in enumerate(fq):
        for q in qs:
            r = q_req[q]
            first.setdefault(r, f)
            last[r] = f
    service = [(t_end[last[r]] - t_beg[first[r]]) * 1e3 for r in first]
    completion = [t_end[last[r]] * 1e3 for r in first]
    all_service = [v for part in d.gather(service) for v in part]
    all_completion = [v for part in d.gather(completion) for v in part]
    total_real = d.allsum(real)
    forwards = d.allsum(nf)
    plan_s_max = d.allmax(plan_s)
    questions_all = d.allsum(rq.questions())   # every rank takes the same collective steps
    padded_all = d.allsum(padded)
    gpus_active = d.allsum(1 if nf > 0 else 0)
    res = {"requests": len(texts), "questions": int(questions_all), "forwards": int(forwards),
           "real_tokens": int(total_real), "ms_max": ms_max, "value": total_real / (ms_max / 1e3),
           "padded_tokens_per_s": padded_all / (ms_max / 1e3), "e2e_s": e_sec, "e2e_value": total_real / e_sec,
           "service_latency_ms": latency_summary(all_service),
           "completion_latency_ms": latency_summary(all_completion), "gpus_active": int(gpus_active),
           "launches": launches, "upload": upload, "plan_s_max": plan_s_max, "plan_all_s": plan_all_s,
           "nf": nf, "d2h": sum(4 * (b.n * b.k + 2 * b.n) for b in batches), "clocks": clk,
           "warmup": min(warmup, len(plans)) + len(big)}
    rq.close()
    tok.close()
    return res


def run_stream(args, d, eng):
    """Config 4: the request stream (JSON) through the C++ front end, one
    pass over --requests requests (stream_pass)."""
    res = stream_pass(args, d, eng, args.requests, args.stream_window, args.warmup)
    cpu = None
    if d.rank == 0 and d.world == 1 and not args.no_cpu_baseline:
        ct, toks = cpu_request_run([stream_sample()], 1, 0)
        cpu = cpu_baseline_line(toks / (ct[0] / 1e3), UNIT,
                                f"request 0 with its first 4 questions ({toks} tokens) through run_all "
                                "(restated front end + C oracle forward), one run")
    if d.rank == 0:
        cfg = {"workload": "stream", "model": MODEL, "requests": res["requests"], "questions": res["questions"],
               "forwards": res["forwards"], "real_tokens": res["real_tokens"], "max_tokens_per_forward": 16384,
               "packing": (f"group_by_budget within windows of {args.stream_window} requests"
                           if args.stream_window > 0 else "dispatch order"),
               "parallelism": f"request-dp{d.world} (greedy by token cost, no collective)",
               "l2": "working set > L2 (843 MB f16 weights streamed per forward)"}
        steps = res["nf"]
        e2e = {"value": res["e2e_value"], "unit": UNIT, "h2d_bytes_per_step": res["upload"] / steps,
               "d2h_bytes_per_step": res["d2h"] / steps,
               "makespan_s": res["e2e_s"], "service_latency_ms": res["service_latency_ms"],
               "completion_latency_ms": res["completion_latency_ms"],
               "path": "laya_forward per packed forward, C++ scoring and response JSON"}
        frontend = {"plan_s": res["plan_s_max"], "plan_tokens_per_s": res["real_tokens"] / res["plan_s_max"],
                    "plan_all_requests_s": res["plan_all_s"], "host_threads": os.cpu_count(),
                    "what": "parse + tokenize + System One layout of the rank's requests on all host threads"}
        line = base_line(args, METRIC + " (request stream)", res["value"], UNIT, d.world,
                         res["ms_max"] / steps, cfg, padded_tokens_per_s=res["padded_tokens_per_s"],
                         device_makespan_s=res["ms_max"] / 1e3, e2e=e2e, frontend=frontend,
                         gpus_active=res["gpus_active"], gpu_launches=res["launches"], clocks=res["clocks"],
                         cpu_baseline=cpu)
        line["steps"] = steps
        line["warmup"] = res["warmup"]
        print(json.dumps(line), flush=True)


def stream_key(args, d, eng):
    """The bounded request-stream sweep carried by the forward-16k line (the
    one the 1/2/4/8-GPU scaling run records): the first --stream-requests
    requests of configuration 4, sharded over the ranks by token cost."""
    if args.stream_requests <= 0:
        return None
    res = stream_pass(args, d, eng, args.stream_requests, 0, 2)
    svc, cmp_ = res["service_latency_ms"], res["completion_latency_ms"]
    return {"requests": res["requests"], "questions": res["questions"], "forwards": res["forwards"],
            "real_tokens": res["real_tokens"], "value": res["value"], "unit": UNIT,
            "device_makespan_s": res["ms_max"] / 1e3, "e2e_value": res["e2e_value"], "e2e_makespan_s": res["e2e_s"],
            "service_latency_ms": {"p50": svc["p50"], "p99": svc["p99"]},
            "completion_latency_ms": {"p50": cmp_["p50"], "p99": cmp_["p99"]},
            "gpus_active": res["gpus_active"],
            "parallelism": f"request-dp{d.world} (greedy by token cost, no collective)",
            "what": "configuration 4's first requests: value = real tokens / device makespan (max over ranks); "
                    "e2e_value through laya_forward + scoring + response JSON (wall clock, max over ranks)"}


# The encoder's four GEMMs at the 16384-token forward's 9872 real rows:
# (name, N as launched, N of the layer, K, epilogue code of laya_bench_gemm,
# f32 residual output).  Wi is launched with gate and up co-tiled and padded
# to 21 tiles of 256 columns; its FLOPs count the layer's 2 x 2624 columns.
GEMM_SHAPES = (("Wqkv", 3072, 3072, 1024, 0, False), ("Wo", 1024, 1024, 1024, 2, True),
               ("Wi", 5376, 5248, 1024, 3, False), ("Wo_mlp", 1024, 1024, 2624, 2, True))
GEMM_M = 9872


def run_gemm(args, d):
    """Diagnostic (not a configuration of the reference): the encoder's four
    GEMM shapes alone, this build's tcgen05 kernel with its fused epilogue
    (RoPE + scale, f32 residual reduce-add, GeGLU) against cuBLAS through
    torch on the same shapes and operand values (f16 operands, f32
    accumulation; f16 output, or for the residual shapes an f32 output that
    adds the residual: addmm with out_dtype f32).  L2 is flushed before every
    launch; CUDA events around each launch; rank 0 only."""
    from laya_rust_b200 import engine as E
    torch = d.torch
    if d.rank != 0:
        return
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    clocks = ClockSampler([0])
    rows, tot_flops, tot_laya, tot_lib = [], 0.0, 0.0, 0.0
    for name, n_launch, n, k, epi, resid in GEMM_SHAPES:
        flops = 2.0 * GEMM_M * n * k
        laya_ms = E.bench_gemm(GEMM_M, n_launch, k, epi, args.steps)
        # the operand bit patterns laya_bench_gemm writes (f16 1.0039, 0.0655)
        a = torch.full((GEMM_M, k), 0x3C3C, dtype=torch.int16, device="cuda").view(torch.float16)
        w = torch.full((n, k), 0x2C2C, dtype=torch.int16, device="cuda").view(torch.float16)
        x = torch.zeros((GEMM_M, n), dtype=torch.float32, device="cuda") if resid else None
        if resid:
            try:
                call = lambda: torch.addmm(x, a, w.t(), out_dtype=torch.float32)
                call()
                lib_form = "addmm(f32 residual, f16, f16, out_dtype=f32)"
            except RuntimeError:
                call = lambda: torch.mm(a, w.t())
                lib_form = "mm (f16 out; addmm with out_dtype f32 unavailable)"
        else:
            call = lambda: torch.mm(a, w.t())
            lib_form = "mm (f16 out)"
        for _ in range(max(3, args.warmup)):
            call()
        torch.cuda.synchronize()
        evs = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            call()
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        lib_ms = sum(p.elapsed_time(q) for p, q in evs) / args.steps
        rows.append({"gemm": name, "m": GEMM_M, "n": n, "k": k, "laya_us": laya_ms * 1e3,
                     "laya_tflops": flops / (laya_ms / 1e3) / 1e12, "cublas_us": lib_ms * 1e3,
                     "cublas_tflops": flops / (lib_ms / 1e3) / 1e12, "cublas_call": lib_form,
                     "laya_over_cublas_time": laya_ms / lib_ms})
        tot_flops += flops
        tot_laya += laya_ms
        tot_lib += lib_ms
        del a, w, x
    clk = clocks.stop()
    pk, pk_src = peaks()
    peak = pk["bf16_tflops"]
    achieved = tot_flops / (tot_laya / 1e3) / 1e12
    line = base_line(args, "encoder GEMM TFLOP/s (four shapes, fused epilogues)", achieved, "TFLOP/s", 1,
                     tot_laya, {"workload": f"Wqkv, Wo, Wi, Wo_mlp at M = {GEMM_M} (one layer of forward-16k)",
                                "l2": "flushed (256 MiB memset) before every launch",
                                "operands": "constant f16 patterns, the same for both kernels"},
                     shapes=rows,
                     cublas={"tflops": tot_flops / (tot_lib / 1e3) / 1e12, "ms_per_layer": tot_lib,
                             "epilogues": "none fused (plain GEMM; residual shapes add an f32 input)"},
                     roofline={"bound": "tensor", "kernel": "gemm_tc_kernel", "achieved": achieved, "peak": peak,
                               "unit": "TFLOP/s", "frac": achieved / peak,
                               "peak_source": f"{pk_src} bf16_tflops (burst)", "traffic": None},
                     gpu_launches=4 * (args.steps + 3), clocks=clk)
    print(json.dumps(line), flush=True)


def run_b200(args):
    d = Dist()
    if args.config == "gemm":
        try:
            run_gemm(args, d)
        finally:
            d.close()
        return
    eng = open_engine(d)
    try:
        if args.config in ("forward-16k", "long-state"):
            run_forward(args, d, eng)
        elif args.config == "layer":
            run_layer(args, d, eng)
        elif args.config == "request":
            run_request(args, d, eng)
        else:
            run_stream(args, d, eng)
    finally:
        eng.close()
        d.close()


def main():
    args = parse()
    # the CPU baseline and the reference arm time the oracle with the
    # reference's own traversal, never the test suite's faster one
    os.environ.pop("LAYA_ORACLE_FAST", None)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
