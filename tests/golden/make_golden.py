"""Generate the golden fixtures under tests/golden/ from the reference engine itself.

The reference (matmulfreellmCPU) ships no golden vectors on its main branch, so these pins
come from running its own code: ``oracle/_ref/libmmfree_ref.so`` (built from the reference
sources by ``oracle/Makefile``) through ``oracle/ref_ops.cpp``. Run from the repo root:

    make -C oracle all && python tests/golden/make_golden.py [--big]

``--big`` also records the 370M (16-token prompt, 32 greedy tokens) and 1.3B (128-token
prompt, 256 greedy tokens) streams of the benchmark configurations; those need the seeded
blobs (about 0.5 GB and 1.6 GB, written to $MMFREE_BLOB_CACHE or /tmp/mmfree_blobs).
``--bench-configs`` (or ``--only-bench-configs``) records the benchmarked configurations at
their full sizes: config 3 (1.3B, 64 streams x 256-id prompts, generate_serve) and config 4
(2.7B, a 2048-id prefill); they need the 1.3B and 2.7B blobs (1.6 GB and 3.2 GB).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from matmulfreellmcpu_b200 import blob as B  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

#: (M, K, N) op shapes: ragged K and N, K%8 tails, a saturating outlier row.
OP_SHAPES = [(1, 64, 32), (3, 100, 37), (4, 256, 96), (2, 1024, 64), (5, 1003, 77)]
EDGE = np.array([np.nan, np.inf, -np.inf, 88.0, 88.3, 88.37, 88.4, -88.0, -88.3, -88.37, -88.4,
                 87.5, -87.5, 0.0, -0.0, 1e-30, -1e-30, 3e38, -3e38, 40.0, 32.0, 31.99951,
                 -32.0, -32.0005, 2.2e6, -2.2e6, 3e9, -3e9, 1e-45, 20.5, -20.5, 0.5],
                np.float32)


def sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def op_inputs(M, K, N, seed):
    """Config-1 style inputs: N(0,1) activations with 1% outliers x20, p=(.3,.4,.3) ternary."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    out_mask = rng.random((M, K)) < 0.01
    x[out_mask] *= np.float32(20.0)
    x[-1, : min(K, 4)] = np.float32(600.0)  # forces y*1024 past +-32767 on the last row
    wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])
    nw = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    return x, nw, wq


def make_ops(R: oracle.Reference) -> None:
    arrays = {}
    for idx, (M, K, N) in enumerate(OP_SHAPES):
        x, nw, wq = op_inputs(M, K, N, 100 + idx)
        for aq in (1, 0):
            out, acc, norm = R.bitlinear(x, nw, wq, 20.0, act_quant=aq, want_norm=True)
            p = f"bl{idx}_{'fixed' if aq else 'float'}"
            arrays[f"{p}_out"] = out
            if acc is not None:
                arrays[f"{p}_acc"] = acc
        arrays[f"bl{idx}_x"], arrays[f"bl{idx}_nw"], arrays[f"bl{idx}_wq"] = x, nw, wq
        arrays[f"bl{idx}_norm"] = norm
    rng = np.random.default_rng(7)
    for n in (8, 29, 1000, 1003):
        v = (rng.standard_normal(n) * rng.choice([0.01, 1.0, 30.0], n)).astype(np.float32)
        v[: min(n, EDGE.size)] = EDGE[: min(n, EDGE.size)]
        b = rng.standard_normal(n).astype(np.float32)
        arrays[f"ew{n}_x"], arrays[f"ew{n}_b"] = v, b
        arrays[f"ew{n}_sigmoid"] = R.sigmoid(v)
        arrays[f"ew{n}_silu"] = R.silu(v)
        arrays[f"ew{n}_swiglu"] = R.swiglu(v, b)
        arrays[f"ew{n}_quant"] = R.quant_q510(v)
        arrays[f"ew{n}_sumsq"] = np.array([R.sumsq(v[np.isfinite(v)])], np.float32)
    for T, D in ((1, 64), (5, 37), (16, 256)):
        i = rng.standard_normal((T, D)).astype(np.float32)
        f = rng.random((T, D)).astype(np.float32)
        g = rng.standard_normal((T, D)).astype(np.float32)
        w = rng.random(D).astype(np.float32)
        s0 = rng.standard_normal(D).astype(np.float32)
        out, st = R.hgrn_scan(i, f, s0)
        p = f"sc{T}x{D}"
        arrays.update({f"{p}_i": i, f"{p}_f": f, f"{p}_g": g, f"{p}_w": w, f"{p}_s0": s0,
                       f"{p}_out": out, f"{p}_state": st,
                       f"{p}_swishgate": R.rmsnorm_swishgate(g, i, w),
                       f"{p}_rmsnorm": R.rmsnorm(g, w)})
    np.savez_compressed(os.path.join(OUT, "ops.npz"), **arrays)


def make_models(R: oracle.Reference, names, cache) -> None:
    for name in names:
        path = B.cached_blob(name, 0, cache)
        V = B.CONFIGS[name]["vocab_size"]
        arrays = {"blob_sha256": np.frombuffer(bytes.fromhex(sha256_file(path)), np.uint8)}
        ids = B.seeded_ids(7, 0, V)
        prompts = [B.seeded_ids(5 + k, 100 + k, V) for k in range(3)]
        arrays["prompt"] = ids
        for k, p in enumerate(prompts):
            arrays[f"serve_prompt{k}"] = p
        for aq, mode in ((1, "fixed"), (0, "float")):
            m = R.model(path, aq)
            stream = m.generate(ids, 9)
            arrays[f"{mode}_stream"] = stream
            arrays[f"{mode}_logits"] = m.forward(stream)[-1]
            arrays[f"{mode}_prefix_logits"] = m.forward(ids)
            for k, s in enumerate(m.generate_serve(prompts, 6)):
                arrays[f"{mode}_serve{k}"] = s
            m.close()
        np.savez_compressed(os.path.join(OUT, f"model_{name}.npz"), **arrays)


def make_big(R: oracle.Reference, cache) -> None:
    for name, n_prompt, gen, modes in (("370M", 16, 32, ("fixed", "float")),
                                       ("1.3B", 128, 256, ("fixed", "float"))):
        path = B.cached_blob(name, 0, cache)
        ids = B.seeded_ids(n_prompt, 0)
        arrays = {"blob_sha256": np.frombuffer(bytes.fromhex(sha256_file(path)), np.uint8),
                  "prompt": ids}
        for mode in modes:
            m = R.model(path, 1 if mode == "fixed" else 0)
            stream = m.generate(ids, gen)
            arrays[f"{mode}_stream"] = stream
            arrays[f"{mode}_logits"] = m.forward(stream)[-1]
            m.close()
        np.savez_compressed(os.path.join(OUT, f"config_{name}.npz"), **arrays)


#: configuration 3: 64 streams with 256-id prompts (seeds 1000 + b), first token + 16 steps
SERVE_STREAMS, SERVE_PROMPT, SERVE_GEN = 64, 256, 17
#: configuration 4: one of the 8 prefill sequences (2048 ids, seed 4000)
PREFILL_LEN, PREFILL_SEED = 2048, 4000


def make_bench_configs(R: oracle.Reference, cache) -> None:
    """The two benchmarked workloads at their own sizes: config 3 (1.3B, 64 x 256-id prompts,
    Model::generate_serve, fixed) and config 4 (2.7B, a 2048-id sequence, the last row of
    Model::forward in fixed and float mode). Takes several minutes of CPU."""
    path = B.cached_blob("1.3B", 0, cache)
    prompts = [B.seeded_ids(SERVE_PROMPT, 1000 + b) for b in range(SERVE_STREAMS)]
    m = R.model(path, 1)
    streams = m.generate_serve(prompts, SERVE_GEN)
    m.close()
    gen = np.stack([s[SERVE_PROMPT:] for s in streams])  # [64, 17]: first id + 16 steps
    np.savez_compressed(os.path.join(OUT, "config3_serve_1.3B.npz"),
                        blob_sha256=np.frombuffer(bytes.fromhex(sha256_file(path)), np.uint8),
                        prompt_seeds=np.arange(1000, 1000 + SERVE_STREAMS), gen_ids=gen)
    path = B.cached_blob("2.7B", 0, cache)
    ids = B.seeded_ids(PREFILL_LEN, PREFILL_SEED)
    arrays = {"blob_sha256": np.frombuffer(bytes.fromhex(sha256_file(path)), np.uint8),
              "ids": ids}
    for aq, mode in ((1, "fixed"), (0, "float")):
        m = R.model(path, aq)
        last = m.forward(ids)[-1].copy()
        m.close()
        arrays[f"{mode}_logits"] = last
        arrays[f"{mode}_argmax"] = np.array([int(np.argmax(last))], np.int64)
    np.savez_compressed(os.path.join(OUT, "config4_prefill_2.7B.npz"), **arrays)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--big", action="store_true")
    ap.add_argument("--bench-configs", action="store_true",
                    help="also record configurations 3 and 4 at their full sizes")
    ap.add_argument("--only-bench-configs", action="store_true")
    ap.add_argument("--cache", default=os.environ.get("MMFREE_BLOB_CACHE", "/tmp/mmfree_blobs"))
    a = ap.parse_args()
    R = oracle.Reference()
    if a.only_bench_configs:
        make_bench_configs(R, a.cache)
        return
    make_ops(R)
    make_models(R, ("tiny", "ragged", "small"), a.cache)
    if a.big:
        make_big(R, a.cache)
    if a.bench_configs:
        make_bench_configs(R, a.cache)


if __name__ == "__main__":
    main()
