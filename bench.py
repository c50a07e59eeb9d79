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
(configuration 2 shape, rank 0), the per-kernel roofline of the dominant kernel class, the
configuration-4 prefill (2.7B, 8 x 2048 tokens; N=1, `prefill_2.7B`, --no-prefill skips it)
and the reference CPU engine timed on this host on a bounded sample (rank 0, N=1).
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


def load_shares():
    """Launch-list shares of the timed decode step (ncu gpu__time_duration of every launch of
    the same command, summarised in profiles/launch_shares.json)."""
    path = os.path.join(ROOT, "profiles", "launch_shares.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


KERNEL_CLASSES = (("tc_matmul_kernel", "bitlinear"), ("dec_kernel", "bitlinear"),
                  ("matmul_fixed_kernel", "bitlinear"), ("matmul_float_kernel", "bitlinear"),
                  ("prep_kernel", "prep"), ("mixer", "mixer"), ("swiglu", "swiglu"),
                  ("argmax", "argmax"), ("embed", "embed"))


def summarize_launches(csv_path, steps, key, command):
    """Per-class launches and share of gpu__time_duration in an ncu launch list (the --csv
    log of `ncu --metrics gpu__time_duration.sum --nvtx-include timed/ ...` over `steps`
    decode steps), merged into profiles/launch_shares.json under `key`."""
    import csv
    per = {}
    with open(csv_path, newline="") as f:
        rows = [r for r in csv.reader(f) if r]
    hdr = next(i for i, r in enumerate(rows) if "Kernel Name" in r and "Metric Value" in r)
    cols = rows[hdr]
    kn, mn, mv = cols.index("Kernel Name"), cols.index("Metric Name"), cols.index("Metric Value")
    unit = cols.index("Metric Unit") if "Metric Unit" in cols else None
    for r in rows[hdr + 1:]:
        if len(r) <= mv or r[mn] != "gpu__time_duration.sum":
            continue
        v = float(r[mv].replace(",", ""))
        u = r[unit] if unit is not None else "ns"
        v *= {"ns": 1e-3, "nsecond": 1e-3, "us": 1.0, "usecond": 1.0, "ms": 1e3, "msecond": 1e3}.get(u, 1e-3)
        name = r[kn]
        cls = next((c for pat, c in KERNEL_CLASSES if pat in name), "other")
        d = per.setdefault(cls, {"launches": 0, "us": 0.0, "kernels": set()})
        d["launches"] += 1
        d["us"] += v
        d["kernels"].add(name.split("(")[0])
    total = sum(d["us"] for d in per.values())
    out = {"command": command, "steps": steps, "total_us_serialised": total,
           "note": "ncu serialises launches with cold caches: use the shares, not the times",
           "classes": {c: {"launches_per_step": d["launches"] / steps, "share": d["us"] / total,
                           "us_per_launch_serialised": d["us"] / d["launches"],
                           "kernels": sorted(d["kernels"])} for c, d in per.items()}}
    path = os.path.join(ROOT, "profiles", "launch_shares.json")
    try:
        with open(path) as f:
            allv = json.load(f)
    except (OSError, ValueError):
        allv = {}
    allv[key] = out
    with open(path, "w") as f:
        json.dump(allv, f, indent=1, sort_keys=True)
        f.write("\n")
    return out


def golden(name):
    """A committed fixture of the reference's own outputs (tests/golden/), or None."""
    path = os.path.join(ROOT, "tests", "golden", name)
    if not os.path.exists(path):
        return None
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def packed_step_bytes(H, I, L, V):
    """Packed 2-bit weight bytes of one decode step: every projection of every layer + lm_head."""
    pk = lambda n, k: -(-n // 32) * -(-k // 64) * 512
    return L * (4 * pk(H, H) + pk(2 * I, H) + pk(H, I)) + pk(V, H)


OP_M1_SHAPES = ((2048, 2048), (2048, 11264), (5632, 2048), (2048, 32000))  # 1.3B shapes


def op_rows(shapes, mode, reps, peaks, src):
    """Configuration 1 rows (isolated mmfree_cuda_bitlinear) for (M, K, N) shapes; weights
    rotate over copies totalling >= 512 MB so every timed call streams them from HBM. The
    `reps` calls are captured once in a CUDA graph and the replay is timed, so the figure is
    the calls' device time (their two kernels and the gaps between them), not the host's
    per-call launch cost (which us_per_call_host reports: the same calls issued one by one
    from Python)."""
    import torch

    from matmulfreellmcpu_b200 import api
    from matmulfreellmcpu_b200._lib import lib, check
    dev = torch.device("cuda", torch.cuda.current_device())
    aq = api.ActQuant[mode]
    rows = []
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
        out = torch.empty(M, N, device=dev)

        def call(i, stream):
            check(lib().mmfree_cuda_bitlinear(out.data_ptr(), xd.data_ptr(), nw.data_ptr(),
                                              wps[i % copies].data_ptr(), 20.0, M, K, N, 1e-6,
                                              None, aq, 10, None, stream))

        s = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(s):
            for i in range(3):  # scratch sized and kernel attributes set before capture
                call(i, s.cuda_stream)
        torch.cuda.synchronize()
        # host-issued calls (Python + C ABI launch cost per call)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            for i in range(reps):
                call(i, s.cuda_stream)
            e1.record(s)
        torch.cuda.synchronize()
        us_host = 1e3 * e0.elapsed_time(e1) / reps
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(reps):
                call(i, s.cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            e0.record(s)
            g.replay()
            e1.record(s)
        torch.cuda.synchronize()
        api.kernel_status(s)
        us = 1e3 * e0.elapsed_time(e1) / reps
        byts = K * N / 4 + 4 * K + 4 * M * K + 4 * M * N + 4
        gbs = byts / us / 1e3
        rows.append({"M": M, "K": K, "N": N, "mode": mode, "us_per_call": us, "hbm_gbs": gbs,
                     "hbm_frac": gbs / float(peaks["hbm_gbs"]), "tops": 2.0 * M * K * N / us / 1e6,
                     "us_per_call_host": us_host, "timing": "CUDA graph of the calls",
                     "weight_copies": copies, "reps": reps, "peak_source": src})
        del g, wps, wp0
    return rows


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
                       "mode": "fixed", "engine": "reference CPU (AVX2 + OpenMP)",
                       "sample_note": "4-id prompts and at most 4 timed steps keep the CPU run "
                                      "bounded; an HGRN decode step costs the same for any "
                                      "prompt length (the recurrent state is [L, B, H]), so "
                                      "tok/s per step is comparable with the GPU arm's"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
H13, I13, L13, V13 = 2048, 5632, 24, 32000  # the 1.3B model


def timed_serve(model, stream, shard, K, world, local, clocks=False):
    """First ids (serve_begin, untimed) and K lockstep steps timed on the model's stream;
    returns (first [S], ids [S, K], max-over-ranks ms, clock summary or None)."""
    import torch
    first = model.serve_begin(shard)
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = Clocks(local) if clocks else None
    if clk:
        clk.__enter__()
    torch.cuda.nvtx.range_push("timed")  # lets ncu --nvtx-include "timed/" capture it
    ev0.record(stream)
    ids = model.serve_run(K)
    ev1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    if clk:
        clk.__exit__(None, None, None)
    barrier(world)
    ms = allmax(ev0.elapsed_time(ev1), world)
    return first, ids, ms, (clk.summary() if clk else None)


def serve_parity(first, ids, rows):
    """The timed run's ids against the reference's generate_serve of the same streams
    (tests/golden/config3_serve_1.3B.npz: first token + 16 steps of each of the 64 streams);
    rows = the configuration's stream indices this rank served."""
    g = golden("config3_serve_1.3B.npz")
    if g is None:
        return {"ok": None, "why": "fixture tests/golden/config3_serve_1.3B.npz absent"}
    ref = g["gen_ids"][rows]
    n = min(ids.shape[1], ref.shape[1] - 1)
    ok = bool(np.array_equal(first, ref[:, 0]) and np.array_equal(ids[:, :n], ref[:, 1:1 + n]))
    return {"ok": ok, "checked": f"{len(rows)} streams: first id + {n} decode steps, bit-exact "
                                 "vs the reference engine's generate_serve"}


def step_roofline(ms_per_step, prof, prof_steps, peaks, src):
    """Roofline of the dominant kernel class of the timed step. The class's time per step is
    its share of the step in the ncu launch list of the same command
    (profiles/launch_shares.json) times the timed ms_per_step, so the class times sum to the
    step; the per-launch algorithmic work comes from the model's own counters (serve_profile).
    Without the launch list the serialised event-pair times are used and labelled so."""
    int8_peak = 2.0 * float(peaks["bf16_tflops"])
    hbm = float(peaks["hbm_gbs"])
    mm = prof["bitlinear_matmul"]
    lm = prof.get("lm_head_matmul", {"ms": 0.0, "launches": 0, "bytes": 0.0, "ops": 0.0})
    launches = (mm["launches"] + lm["launches"]) / prof_steps
    byts = (mm["bytes"] + lm["bytes"]) / prof_steps / launches
    ops = (mm["ops"] + lm["ops"]) / prof_steps / launches
    sh = load_shares().get("decode_b64_1.3B", {}).get("classes", {}).get("bitlinear")
    if sh:
        us = 1e3 * sh["share"] * ms_per_step / launches
        basis = (f"share {sh['share']:.3f} of the timed step in the ncu launch list "
                 f"(profiles/launch_shares.json) x ms_per_step / launches")
    else:
        us = 1e3 * (mm["ms"] + lm["ms"]) / prof_steps / launches
        basis = "serialised CUDA-event pairs around each launch (no launch list found)"
    tops, gbs = ops / us / 1e6, byts / us / 1e3
    roof = {"bound": "tensor", "achieved": tops, "peak": int8_peak, "unit": "TOP/s",
            "frac": tops / int8_peak, "traffic": None,
            "peak_source": f"int8 dense = 2 x bf16_tflops of {src} peaks (no int8 entry)",
            "alt_hbm": {"achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}}
    if byts / hbm / 1e3 > ops / int8_peak / 1e6:  # bytes bound the launch instead
        roof.update({"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "peak_source": f"hbm_gbs of {src} peaks"})
    tr = load_traffic().get("bitlinear_matmul")
    if tr:
        # DRAM bytes per packed weight byte of an ncu capture, times the class's packed
        # weight bytes per launch
        roof["traffic"] = tr["dram_bytes_per_weight_byte"] * packed_step_bytes(H13, I13, L13, V13) / launches
        roof["traffic_source"] = tr["source"]
    roof.update({"kernel": "tc_matmul_kernel: every BitLinear of the step (96 per-layer + lm_head)",
                 "launches_per_step": launches, "avg_launch_us": us,
                 "algorithmic_bytes_per_launch": byts, "algorithmic_ops_per_launch": ops,
                 "time_basis": basis})
    return roof


def run_b1(model, stream, steps, mode):
    """Batch-1 decode (configuration 2 shape: 128-id seeded prompt, up to 255 decode steps) on
    an open model; tok/s from CUDA events around the graph replays, the weight stream rate as
    packed step bytes / time per token, and parity against the reference's stream."""
    import torch
    from matmulfreellmcpu_b200.blob import seeded_ids
    prompt = seeded_ids(B1_PROMPT, 0)
    model.serve_begin([prompt])
    model.serve_run(steps)  # captures the graph the timed call reuses
    model.serve_end()
    first = model.serve_begin([prompt])
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("b1")
    f0.record(stream)
    ids = model.serve_run(steps)
    f1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    b1_ms = f0.elapsed_time(f1)
    model.serve_end()
    ms_tok = b1_ms / steps
    wbytes = packed_step_bytes(H13, I13, L13, V13)
    out = {"mode": mode, "decode_tok_s": steps / (b1_ms / 1e3), "steps": steps,
           "ms_per_token": ms_tok, "weight_stream_gbs": wbytes / (ms_tok / 1e3) / 1e9,
           "weight_bytes_per_token": wbytes}
    g = golden("config_1.3B.npz")
    if g is not None:
        ref = g[f"{mode}_stream"]
        got = np.concatenate([first, ids[0]])
        n = min(got.size, ref.size - B1_PROMPT)
        if mode == "fixed":
            out["parity"] = {"ok": bool(np.array_equal(got[:n], ref[B1_PROMPT:B1_PROMPT + n])),
                             "checked": f"{n} generated ids bit-exact vs the reference"}
        else:  # Float: the logits of the reference's stream, within 1e-3 of their range
            lg, rl = model.forward_last(ref), g["float_logits"]
            err = float(np.abs(lg - rl).max()) / float(rl.max() - rl.min())
            out["parity"] = {"ok": err <= 1e-3, "max_abs_over_range": err,
                             "checked": "last-position logits of the reference's float stream"}
    return out


def run_ours(a, rank, world, local):
    import torch

    from matmulfreellmcpu_b200 import api
    from matmulfreellmcpu_b200.dp import shard_bounds

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
    first, ids, ms, clk = timed_serve(model, stream, shard, K, world, local, clocks=True)
    value = N_STREAMS * world * K / (ms / 1e3)  # all ranks' tokens / the slowest rank's time
    parity = serve_parity(first, ids, list(range(N_STREAMS))) if rank == 0 else None

    # per-kernel-class work counters of the same decode steps (event pairs, not captured)
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

    # strong scaling (N > 1): configuration 3's own 64 streams sharded 64/N per GPU
    strong = None
    if world > 1:
        b0, b1 = shard_bounds(N_STREAMS, rank, world)
        mine = prompts_for(0)[b0:b1]
        model.serve_begin(mine)
        model.serve_run(K)  # graph capture for this batch
        model.serve_end()
        sf, sids, sms, _ = timed_serve(model, stream, mine, K, world, local)
        model.serve_end()
        sp = serve_parity(sf, sids, list(range(b0, b1)))
        ok = allmax(0.0 if sp["ok"] else 1.0, world) == 0.0 if sp["ok"] is not None else None
        strong = {"value": N_STREAMS * K / (sms / 1e3), "unit": "tok/s", "ms_per_step": sms / K,
                  "streams_total": N_STREAMS, "streams_per_gpu": b1 - b0,
                  "parity": {"ok": ok, "checked": "every rank's shard vs the fixture"}}

    # b = 1 decode (configuration 2 shape), rank 0: fixed (this model) and float
    b1 = b1f = None
    b1_steps = max(1, min(a.b1_steps, B1_GEN - 1))
    if rank == 0 and a.b1_steps > 0:
        b1 = run_b1(model, stream, b1_steps, a.mode)
        if a.mode == "fixed":
            with api.Model(path, "float", 10, device=local) as mf:
                sf_ = torch.cuda.ExternalStream(mf.stream_ptr, device=torch.device("cuda", local))
                b1f = run_b1(mf, sf_, b1_steps, "float")
    prefill = None
    if rank == 0 and world == 1 and not a.no_prefill:
        try:
            prefill = prefill_extra(a.mode, local)
        except Exception as ex:  # reported beside the headline, never required
            prefill = {"unavailable": str(ex)}
    op_m1 = None
    if rank == 0 and not a.no_op:
        peaks_, src_ = load_peaks()
        op_m1 = op_rows([(1, k, n) for k, n in OP_M1_SHAPES], "fixed", 50, peaks_, src_) + \
            op_rows([(1, k, n) for k, n in OP_M1_SHAPES], "float", 50, peaks_, src_)
    barrier(world)

    if rank != 0:
        model.close()
        return
    peaks, src = load_peaks()
    roof = step_roofline(ms / K, prof, prof_steps, peaks, src)

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
            "parity": parity,
            "e2e": {"value": e2e, "unit": "tok/s", "steps": K_e2e,
                    "h2d_bytes_per_step": 8 * S + 16, "d2h_bytes_per_step": 8 * S},
            "gpu_launches": int(round(launches_per_step * K)),
            "roofline": roof, "cpu_baseline": cpu, "b1": b1, "b1_float": b1f, "op_m1": op_m1,
            "prefill_2.7B": prefill,
            "strong_scaling": strong,
            "kernel_ms_per_step_serialised": {k: v["ms"] / prof_steps for k, v in prof.items()},
            "clocks": clk}
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


def prefill_extra(mode, local, steps=3):
    """Configuration 4 on one GPU, attached to the default decode line: the 8 x 2048-token
    prefill of the 2.7B model through the public serve_begin call, one warm-up forward and
    `steps` timed ones (CUDA events on the model's stream), sequence 0's first id checked
    against the reference's fixture; the roofline as `--workload prefill` reports it."""
    import torch

    from matmulfreellmcpu_b200 import api

    seqs = p4_prompts()
    with api.Model(blob_path(0, 1, "2.7B"), mode, 10, device=local) as m:
        st = torch.cuda.ExternalStream(m.stream_ptr, device=torch.device("cuda", local))
        m.serve_begin(seqs)
        m.serve_end()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            first = m.serve_begin(seqs)
            m.serve_end()
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
    peaks, src = load_peaks()
    int8_peak = 2.0 * float(peaks["bf16_tflops"])
    tokens = P4_SEQS * P4_LEN * steps
    tops = p4_ops_per_token() * tokens / (ms / 1e3) / 1e12
    g4 = golden("config4_prefill_2.7B.npz")
    parity = None
    if g4 is not None:
        parity = {"ok": bool(first[0] == int(g4[f"{mode}_argmax"][0])),
                  "checked": "sequence 0's first id vs the reference's argmax of its last position"}
    return {"metric": "HGRN-Bit 2.7B prefill tok/s (8 x 2048 tokens, config 4)",
            "value": tokens / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / steps, "steps": steps,
            "warmup": 1, "mode": mode, "parity": parity,
            "roofline": {"bound": "tensor", "achieved": tops, "peak": int8_peak, "unit": "TOP/s",
                         "frac": tops / int8_peak,
                         "kernel": "whole prefill forward (algorithmic 2*T*weights int ops)",
                         "peak_source": f"int8 dense = 2 x bf16_tflops of {src} peaks"}}


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
    sp_first = model.serve_begin(shard) if shard else np.zeros(0, np.int64)
    if shard:
        model.serve_end()
    model.close()
    # the sequence split's first ids of all 8 sequences, for the parity checks below
    if world > 1:
        import torch.distributed as dist
        parts = [None] * world
        dist.all_gather_object(parts, [int(v) for v in sp_first])
        all_first = np.array([v for p in parts for v in p], np.int64)
    else:
        all_first = sp_first
    g4 = golden("config4_prefill_2.7B.npz")
    parity = None
    if g4 is not None and a.mode in ("fixed", "float"):
        parity = {"ok": bool(all_first[0] == int(g4[f"{a.mode}_argmax"][0])),
                  "checked": "sequence 0's first id vs the reference's argmax of its last "
                             "position (tests/golden/config4_prefill_2.7B.npz)"}

    # tensor-parallel prefill of all 8 sequences on every rank (column/row split, NCCL)
    tp_res = None
    if world > 1 and not a.no_tp:
        from matmulfreellmcpu_b200 import tp
        tp_res = {}
        for mode in (("fixed", "float") if a.tp_float else ("fixed",)):
            m = tp.open_model(blob_path(rank, world, "2.7B"), mode, rank, world, local)
            st = torch.cuda.ExternalStream(m.stream_ptr, device=torch.device("cuda", local))
            first = m.serve_begin(p4_prompts())  # warm-up (workspace, clocks)
            m.serve_end()
            Kt = 1 if mode == "float" else max(1, min(K, 3))
            barrier(world)
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(st)
            for _ in range(Kt):
                first = m.serve_begin(p4_prompts())
                m.serve_end()
            t1.record(st)
            torch.cuda.synchronize()
            barrier(world)
            tms = allmax(t0.elapsed_time(t1), world)
            m.close()
            r = {"value": P4_SEQS * P4_LEN * Kt / (tms / 1e3), "unit": "tok/s",
                 "ms_per_step": tms / Kt, "steps": Kt,
                 "split": ("column-parallel projections, NCCL all-gather of column slices "
                           "before each exact norm" if mode == "fixed" else
                           "i/f/g/gate column-parallel, o/down row-parallel, NCCL all-reduce "
                           "of partial sums of squares and of the row-parallel outputs")}
            if mode == a.mode:
                r["first_ids_equal_sequence_split"] = bool(np.array_equal(first, all_first))
            tp_res[mode] = r
    if rank != 0:
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
            "cpu_baseline": cpu, "clocks": clk.summary(), "parity": parity,
            "tensor_parallel": tp_res}
    print(json.dumps(line), flush=True)


SWEEP_M = (1, 16, 64, 512, 4096)
SWEEP_KN = ((1024, 1024), (1024, 5632), (2048, 2048), (2048, 11264), (5632, 2048),
            (2560, 13824), (6912, 2560))


def run_op(a):
    """Configuration 1: the isolated BitLinear op (mmfree_cuda_bitlinear) per (M, K, N).
    Inputs as in the config (N(0,1) activations with 1% x20 outliers, ternary p=(.3,.4,.3),
    scale 20); weights rotate over enough packed copies to exceed L2 (>= 512 MB), so every
    timed call streams its weights from HBM. One JSON line per shape."""
    import torch
    torch.cuda.set_device(0)
    peaks, src = load_peaks()
    if a.op == "sweep":
        shapes = [(m, k, n) for (k, n) in SWEEP_KN for m in SWEEP_M]
    else:
        shapes = [tuple(int(v) for v in a.op.split(","))]
    for M, K, N in shapes:
        row = op_rows([(M, K, N)], a.mode, max(1, a.op_reps), peaks, src)[0]
        print(json.dumps({"metric": "BitLinear op (config 1)", **row}), flush=True)


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
    ap.add_argument("--no-op", action="store_true", help="skip the op_m1 rows (config 1, M=1)")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the config-4 prefill attached to the default decode line")
    ap.add_argument("--no-tp", action="store_true",
                    help="prefill at N > 1: skip the tensor-parallel leg")
    ap.add_argument("--tp-float", action="store_true",
                    help="prefill at N > 1: also time the Float-mode tensor-parallel split")
    ap.add_argument("--b1-steps", type=int, default=B1_GEN - 1,
                    help="decode steps of the b=1 figure (0 skips it)")
    ap.add_argument("--summarize-launches", nargs=3, metavar=("CSV", "STEPS", "KEY"),
                    help="write profiles/launch_shares.json[KEY] from an ncu launch-list CSV")
    a = ap.parse_args()
    if a.summarize_launches:
        csv_path, steps, key = a.summarize_launches
        cmd = os.environ.get("MMFREE_NCU_COMMAND", "see profiles/ summary of this key")
        print(json.dumps(summarize_launches(csv_path, int(steps), key, cmd), indent=1))
        return
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
