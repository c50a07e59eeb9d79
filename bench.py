"""Benchmark: HGRN-Bit 1.3B lockstep decode tok/s (configuration 3) on N B200s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload decode|prefill] [--op sweep|M,K,N]
  (N > 1: launched by torch.distributed.run, one rank per GPU)

Workload: the seeded random-init 1.3B blob (seed 0), 64
independent streams with 256-id seeded prompts, FixedQ510 greedy decode. Every GPU serves its
own 64 streams (rank r: seeds 1000 + 64 r + b; no inter-GPU communication, the streams share
nothing but the weights), so the per-GPU batch stays b=64 and scaling is "weak". One step =
one lockstep decode step of every stream (64 N new tokens); value = 64 N K / (max over ranks
of the device time of K steps).
The prefill of the prompts happens before the timed region (untimed), so the timed steps
start from resident state. Weights (325 MB packed) exceed the 126 MB L2, so consecutive
steps stream them from HBM without an explicit flush.

Also reported: e2e (the same metric through the public serving API, one
mmfree_cuda_serve_step call per step: pinned host ids in, next ids out), b=1 decode tok/s
(configuration 2 shape, rank 0), the per-kernel roofline of the dominant kernel class and
the reference CPU engine timed on this host on a bounded sample (rank 0, N=1).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_STREAMS = 64
PROMPT_LEN = 256
GEN_TOKENS = 512          # configuration 3: 512 generated tokens per stream
B1_PROMPT, B1_GEN = 128, 256
METRIC = "HGRN-Bit 1.3B decode tok/s (b=64 lockstep, 64 streams per GPU)"
DTYPE = "q5.10-int16 x ternary(2-bit) -> int32"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def prompts_for(rank: int):
    """The 64 independent streams of one GPU (weak scaling: every rank serves its own 64;
    rank 0's are the configuration's streams, seeds 1000 + b)."""
    from matmulfreellmcpu_b200.blob import seeded_ids
    return [seeded_ids(PROMPT_LEN, 1000 + N_STREAMS * rank + b) for b in range(N_STREAMS)]


def host_threads() -> int:
    """Host cores this process may use (torchrun sets OMP_NUM_THREADS=1 per worker, so the
    CPU reference sets its thread count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class Clocks:
    """nvidia-smi sampler for the timed region (clocks and throttle reasons)."""
    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        self.dev, self.p = dev, None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "-i", str(self.dev),
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.p:
            time.sleep(0.2)
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                self.out, _ = self.p.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 6:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[2 + i] == "Active"})
        load = [s for s in sm if mx and s >= 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allmax(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"  # gloo groups reduce on the host
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def blob_path(rank, world, name="1.3B"):
    from matmulfreellmcpu_b200 import blob as B
    cache = os.environ.get("MMFREE_BLOB_CACHE", "/tmp/mmfree_blobs")
    if rank == 0:
        p = B.cached_blob(name, 0, cache)
    barrier(world)
    if rank != 0:
        p = B.cached_blob(name, 0, cache)  # written by rank 0 already
    return p


# ------------------------------------------------------------------ reference (CPU) arm
def cpu_reference(steps: int, warmup: int, threads: int | None = None):
    """The reference engine (oracle/_ref, compiled from the reference sources) on this host:
    Model::generate_serve with 64 streams; the decode window of one call is timed by the
    reference's own token callbacks. Prompts are 4 ids (state cost per step does not depend
    on prompt length), so the sample is `steps` lockstep decode steps of 64 streams."""
    import oracle
    from matmulfreellmcpu_b200.blob import seeded_ids
    R = oracle.Reference()
    R.set_threads(threads or host_threads())
    path = blob_path(0, 1)
    m = R.model(path, 1)
    prompts = [seeded_ids(4, 1000 + b) for b in range(N_STREAMS)]
    if warmup > 0:
        m.bench_serve(prompts[:8], 2)
    pre_s, dec_s, dec_tok = m.bench_serve(prompts, steps + 1)
    m.close()
    value = dec_tok / dec_s if dec_s > 0 else 0.0
    return {"value": value, "unit": "tok/s", "cores": R.threads(), "kind": "reference",
            "sample": f"64 streams x {steps} lockstep decode steps (4-id seeded prompts, "
                      f"prefill excluded; {dec_tok} tokens in {dec_s:.2f} s)",
            "ms_per_step": 1e3 * dec_s / max(steps, 1)}


def load_traffic():
    """DRAM bytes per launch by kernel class, summarised from ncu captures in profiles/."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def run_reference_arm(a, rank, world):
    if rank != 0:
        return
    if getattr(a, "workload", "decode") == "prefill":
        cb = cpu_prefill()
        line = {"impl": "reference", "metric": "HGRN-Bit 2.7B prefill tok/s (8 x 2048 tokens)",
                "value": cb["value"], "unit": "tok/s", "n_gpus": world, "steps": 1, "warmup": 1,
                "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": DTYPE, "data": "synthetic (seeded random-init blob)",
                "config": {"workload": "config4: 2.7B prefill (CPU sample: one prompt)",
                           "model": "HGRN-Bit 2.7B random-init seed 0", "mode": "fixed",
                           "engine": "reference CPU (AVX2 + OpenMP)"},
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    steps = max(1, min(a.steps, 4))
    cb = cpu_reference(steps, min(a.warmup, 1))
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tok/s",
            "n_gpus": world, "steps": steps, "warmup": min(a.warmup, 1),
            "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": DTYPE, "data": "synthetic (seeded random-init blob)",
            "config": {"workload": "config3: 1.3B lockstep decode, 64 streams",
                       "model": "HGRN-Bit 1.3B random-init seed 0", "streams": N_STREAMS,
                       "mode": "fixed", "engine": "reference CPU (AVX2 + OpenMP)"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(a, rank, world, local):
    import torch

    from matmulfreellmcpu_b200 import api

    torch.cuda.set_device(local)
    path = blob_path(rank, world)
    model = api.Model(path, a.mode, 10, device=local)
    stream = torch.cuda.ExternalStream(model.stream_ptr, device=torch.device("cuda", local))
    shard = prompts_for(rank)  # weak scaling: 64 independent streams on every GPU
    S = len(shard)
    budget = GEN_TOKENS - 1  # decode steps available after the prefill token
    K = min(a.steps, budget)
    W = a.warmup

    # warm-up session (graph capture for K steps, clocks up), then a fresh session for the
    # timed steps; W warm-up steps run first, then K so that the timed call reuses the graph
    model.serve_begin(shard)
    model.serve_run(max(W, 1))
    model.serve_end()
    model.serve_begin(shard)
    model.serve_run(K)
    model.serve_end()
    model.serve_begin(shard)
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.nvtx.range_push("timed")  # lets ncu --nvtx-include "timed/" capture it
        ev0.record(stream)
        model.serve_run(K)
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier(world)
    ms = allmax(ev0.elapsed_time(ev1), world)
    value = N_STREAMS * world * K / (ms / 1e3)  # all ranks' tokens / the slowest rank's time

    # per-kernel-class breakdown of the same decode steps (event pairs, not graph-captured)
    prof_steps = min(16, max(1, budget - K)) if budget - K > 0 else 8
    if budget - K <= 0:
        model.serve_end()
        model.serve_begin(shard)
    prof = model.serve_profile(prof_steps)
    model.serve_end()
    launches_per_step = sum(v["launches"] for v in prof.values()) / prof_steps

    # e2e through the public per-step API: pinned host ids in, next ids out, every step
    first = model.serve_begin(shard)
    K_e2e = max(1, min(K, a.e2e_steps))
    hin = torch.empty(S, dtype=torch.int64).pin_memory()
    hout = torch.empty(S, dtype=torch.int64).pin_memory()
    hin.copy_(torch.from_numpy(first))
    model.serve_step_ptr(hin.data_ptr(), hout.data_ptr())  # first step outside timing
    hin.copy_(hout)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K_e2e):
        model.serve_step_ptr(hin.data_ptr(), hout.data_ptr())
        hin.copy_(hout)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = allmax(e0.elapsed_time(e1), world)
    model.serve_end()
    e2e = N_STREAMS * world * K_e2e / (ms_e2e / 1e3)

    # b = 1 decode (configuration 2 shape: 128-id prompt, 255 decode steps), rank 0
    b1 = None
    b1_steps = max(1, min(a.b1_steps, B1_GEN - 1))
    if rank == 0 and a.b1_steps > 0:
        from matmulfreellmcpu_b200.blob import seeded_ids
        model.serve_begin([seeded_ids(B1_PROMPT, 0)])
        model.serve_run(b1_steps)  # captures the graph the timed call reuses
        model.serve_end()
        model.serve_begin([seeded_ids(B1_PROMPT, 0)])
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("b1")
        f0.record(stream)
        model.serve_run(b1_steps)
        f1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        b1_ms = f0.elapsed_time(f1)
        prof1 = model.serve_profile(8)
        model.serve_end()
        b1 = {"decode_tok_s": b1_steps / (b1_ms / 1e3), "steps": b1_steps,
              "ms_per_token": b1_ms / b1_steps,
              "kernel_ms_per_token": {k: v["ms"] / 8 for k, v in prof1.items()}}
        mm = prof1["bitlinear_matmul"]
        b1["bitlinear_hbm_gbs"] = mm["bytes"] / (mm["ms"] / 1e3) / 1e9 if mm["ms"] else None
    barrier(world)

    if rank != 0:
        model.close()
        return
    peaks, src = load_peaks()
    mm = prof["bitlinear_matmul"]
    t = mm["ms"] / 1e3
    gbs = mm["bytes"] / t / 1e9
    tops = mm["ops"] / t / 1e12
    int8_peak = 2.0 * float(peaks["bf16_tflops"])
    t_hbm = mm["bytes"] / (float(peaks["hbm_gbs"]) * 1e9)
    t_tc = mm["ops"] / (int8_peak * 1e12)
    if t_tc > t_hbm:
        roof = {"bound": "tensor", "achieved": tops, "peak": int8_peak, "unit": "TOP/s",
                "frac": tops / int8_peak, "traffic": None,
                "peak_source": f"int8 dense = 2 x bf16_tflops of {src} peaks (no int8 entry)",
                "alt_hbm": {"achieved": gbs, "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                            "frac": gbs / float(peaks["hbm_gbs"])}}
    else:
        roof = {"bound": "hbm", "achieved": gbs, "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                "frac": gbs / float(peaks["hbm_gbs"]), "traffic": None,
                "peak_source": f"hbm_gbs of {src} peaks"}
    # DRAM traffic per launch of the same kernel class from an ncu capture (profiles/)
    tr = load_traffic().get("bitlinear_matmul")
    if tr:
        # the class's packed weight bytes per launch (every projection of every layer once
        # per step) times the DRAM bytes per weight byte the capture measured
        H, I, L = 2048, 5632, 24
        pk = lambda n, k: -(-n // 32) * -(-k // 64) * 512
        wstep = L * (4 * pk(H, H) + pk(2 * I, H) + pk(H, I))
        per_launch = wstep / (mm["launches"] / prof_steps)
        roof["traffic"] = tr["dram_bytes_per_weight_byte"] * per_launch
        roof["traffic_source"] = tr["source"]
    roof.update({"kernel": "bitlinear_matmul (all per-layer BitLinear projections)",
                 "launches_per_step": mm["launches"] / prof_steps,
                 "avg_launch_us": 1e3 * mm["ms"] / mm["launches"],
                 "algorithmic_bytes_per_launch": mm["bytes"] / mm["launches"],
                 "share_of_step": mm["ms"] / sum(v["ms"] for v in prof.values())})

    cpu = None
    if world == 1 and not a.no_cpu:
        try:
            cb = cpu_reference(2, 0)
            cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "reference",
                   "sample": f"unavailable: {ex}"}

    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded random-init 1.3B blob, seeded prompt ids)",
            "config": {"workload": "config3: 1.3B lockstep decode, 64 streams, 256-id prompts",
                       "model": "HGRN-Bit 1.3B random-init seed 0 (L24 H2048 I5632 V32000)",
                       "streams": N_STREAMS * world, "streams_per_gpu": S, "prompt_len": PROMPT_LEN,
                       "mode": a.mode,
                       "parallelism": f"dp{world} (64 independent streams per GPU, no collective)",
                       "l2": "no flush: 325 MB packed weights > 126 MB L2 per step"},
            "e2e": {"value": e2e, "unit": "tok/s", "steps": K_e2e,
                    "h2d_bytes_per_step": 8 * S + 16, "d2h_bytes_per_step": 8 * S},
            "gpu_launches": int(round(launches_per_step * K)),
            "roofline": roof, "cpu_baseline": cpu, "b1": b1,
            "kernel_ms_per_step": {k: v["ms"] / prof_steps for k, v in prof.items()},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    model.close()


# ------------------------------------------------------------------ configuration 4: prefill
P4_SEQS, P4_LEN = 8, 2048   # 2.7B, 8 x 2048 seeded tokens, prefill only
P4_CPU_LEN = 64             # CPU reference sample: one prompt of this length


def p4_prompts():
    from matmulfreellmcpu_b200.blob import seeded_ids
    return [seeded_ids(P4_LEN, 4000 + b) for b in range(P4_SEQS)]


def p4_ops_per_token():
    """Algorithmic int ops per prefill token: 2 x the per-layer BitLinear weights (the head
    runs on one row per sequence and is left out)."""
    H, I, L = 2560, 6912, 32
    return 2.0 * L * (4 * H * H + 2 * I * H + I * H)


def cpu_prefill(threads=0):
    """The reference engine's Model::forward on one P4_CPU_LEN-token prompt of the 2.7B blob,
    timed on this host; tok/s = prompt tokens / seconds."""
    import oracle
    from matmulfreellmcpu_b200.blob import seeded_ids
    R = oracle.Reference()
    R.set_threads(threads or host_threads())
    m = R.model(blob_path(0, 1, "2.7B"), 1)
    ids = seeded_ids(P4_CPU_LEN, 4000)
    m.forward(ids[:8])  # warm-up (page the weights in)
    t0 = time.perf_counter()
    m.forward(ids)
    dt = time.perf_counter() - t0
    m.close()
    return {"value": P4_CPU_LEN / dt, "unit": "tok/s", "cores": R.threads(), "kind": "reference",
            "sample": f"Model::forward of one {P4_CPU_LEN}-token prompt (2.7B, fixed) in {dt:.2f} s",
            "ms_per_step": 1e3 * dt}


def run_prefill(a, rank, world, local):
    """Configuration 4: batched prefill of 8 x 2048 tokens on the 2.7B model (the last
    position's logits and argmax plus the final recurrent states of every sequence).
    Sequences are sharded over ranks (sequence-parallel, no data-path collective)."""
    import torch

    from matmulfreellmcpu_b200 import api
    from matmulfreellmcpu_b200.dp import shard_bounds

    torch.cuda.set_device(local)
    model = api.Model(blob_path(rank, world, "2.7B"), a.mode, 10, device=local)
    stream = torch.cuda.ExternalStream(model.stream_ptr, device=torch.device("cuda", local))
    b0, b1 = shard_bounds(P4_SEQS, rank, world)
    shard = p4_prompts()[b0:b1]
    K, W = max(1, min(a.steps, 20)), a.warmup
    for _ in range(max(W, 1)):
        if shard:
            model.serve_begin(shard)
            model.serve_end()
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        ev0.record(stream)
        for _ in range(K):
            if shard:
                model.serve_begin(shard)  # host ids in, first ids out: the public API call
                model.serve_end()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = allmax(ev0.elapsed_time(ev1), world)
    tokens = P4_SEQS * P4_LEN * K
    value = tokens / (ms / 1e3)
    if rank != 0:
        model.close()
        return
    peaks, src = load_peaks()
    int8_peak = 2.0 * float(peaks["bf16_tflops"])
    tops = p4_ops_per_token() * tokens / (ms / 1e3) / 1e12
    cpu = None
    if world == 1 and not a.no_cpu:
        try:
            cb = cpu_prefill()
            cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as ex:
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "reference",
                   "sample": f"unavailable: {ex}"}
    line = {"metric": "HGRN-Bit 2.7B prefill tok/s (8 x 2048 tokens)", "value": value,
            "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms / K,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded random-init 2.7B blob, seeded prompt ids)",
            "config": {"workload": "config4: 2.7B prefill, 8 sequences x 2048 tokens",
                       "model": "HGRN-Bit 2.7B random-init seed 0 (L32 H2560 I6912 V32000)",
                       "mode": a.mode, "parallelism": f"sp{world} (sequences sharded, no collective)",
                       "l2": "no flush: 655 MB packed weights > 126 MB L2 per forward"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 8 * P4_SEQS * P4_LEN,
                    "d2h_bytes_per_step": 8 * P4_SEQS,
                    "note": "each step is the public serve_begin call: host ids in, first ids out"},
            "roofline": {"bound": "tensor", "achieved": tops, "peak": int8_peak, "unit": "TOP/s",
                         "frac": tops / int8_peak, "traffic": None,
                         "kernel": "whole prefill forward (algorithmic 2*T*weights int ops)",
                         "peak_source": f"int8 dense = 2 x bf16_tflops of {src} peaks (no int8 entry)"},
            "cpu_baseline": cpu, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    model.close()


SWEEP_M = (1, 16, 64, 512, 4096)
SWEEP_KN = ((1024, 1024), (1024, 5632), (2048, 2048), (2048, 11264), (5632, 2048),
            (2560, 13824), (6912, 2560))


def run_op(a):
    """Configuration 1: the isolated BitLinear op (mmfree_cuda_bitlinear) per (M, K, N).
    Inputs as in the config (N(0,1) activations with 1% x20 outliers, ternary p=(.3,.4,.3),
    scale 20); weights rotate over enough packed copies to exceed L2 (>= 512 MB), so every
    timed call streams its weights from HBM. One JSON line per shape."""
    import torch

    from matmulfreellmcpu_b200 import api
    peaks, src = load_peaks()
    dev = torch.device("cuda", 0)
    shapes = []
    if a.op == "sweep":
        shapes = [(m, k, n) for (k, n) in SWEEP_KN for m in SWEEP_M]
    else:
        shapes = [tuple(int(v) for v in a.op.split(","))]
    for M, K, N in shapes:
        rng = np.random.default_rng(M + K + N)
        x = rng.standard_normal((M, K)).astype(np.float32)
        x[rng.random((M, K)) < 0.01] *= np.float32(20.0)
        wq = torch.from_numpy(rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K),
                                         p=[0.3, 0.4, 0.3])).to(dev)
        wp0 = api.repack_ternary(wq)
        copies = max(1, -(-(512 << 20) // wp0.numel()))
        wps = [wp0] + [wp0.clone() for _ in range(copies - 1)]
        xd = torch.from_numpy(x).to(dev)
        nw = torch.ones(K, device=dev)
        s = torch.cuda.current_stream()
        for i in range(3):
            api.bitlinear(xd, nw, wps[i % copies], 20.0, N, act_quant=a.mode)
        reps = max(1, a.op_reps)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(reps):
            api.bitlinear(xd, nw, wps[i % copies], 20.0, N, act_quant=a.mode)
        e1.record(s)
        torch.cuda.synchronize()
        us = 1e3 * e0.elapsed_time(e1) / reps
        byts = K * N / 4 + 4 * K + 4 * M * K + 4 * M * N + 4
        ops = 2.0 * M * K * N
        gbs = byts / us / 1e3
        print(json.dumps({"metric": "BitLinear op (config 1)", "M": M, "K": K, "N": N,
                          "mode": a.mode, "us_per_call": us, "hbm_gbs": gbs,
                          "hbm_frac": gbs / float(peaks["hbm_gbs"]), "tops": ops / us / 1e6,
                          "weight_copies": copies, "reps": reps, "peak_source": src}),
              flush=True)
        del wps, wp0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--op", default=None,
                    help="configuration 1 instead: 'sweep' or 'M,K,N' (isolated BitLinear)")
    ap.add_argument("--op-reps", type=int, default=50)
    ap.add_argument("--e2e-steps", type=int, default=128,
                    help="decode steps of the end-to-end (host ids in/out) measurement")
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "prefill"], default="decode",
                    help="decode: configuration 3 (default); prefill: configuration 4")
    ap.add_argument("--mode", choices=["fixed", "float"], default="fixed")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--b1-steps", type=int, default=B1_GEN - 1,
                    help="decode steps of the b=1 figure (0 skips it)")
    a = ap.parse_args()
    if a.op:
        run_op(a)
        return
    if a.impl == "reference":
        # rank 0 alone times the CPU reference; the other ranks exit without work
        rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
        run_reference_arm(a, rank, world)
        return
    rank, world, local = dist_setup()
    try:
        if a.workload == "prefill":
            run_prefill(a, rank, world, local)
        else:
            run_ours(a, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
