"""Tensor-parallel split of the BitLinear projections (matmulfreellmcpu_b200/tp.py and the
library's layers_tp) checked on the CPU with two gloo ranks.

Each rank takes the shard ``tp.shard_plan`` gives it, computes its part with the CPU oracle
(the restatement of the reference's bitlinear, bitlinear.cpp:39-116), and the ranks exchange
results with the collectives the GPU path uses (all-gather of column slices, all-reduce of
partial sums). The exchanged result must equal the unsharded oracle:
  * FixedQ510 column-parallel (i/f/g/o/down and the gate_proj SwiGLU pair): bit for bit;
  * Float row-parallel (o/down: all-reduced partial sums of squares, then partial outputs):
    within the Float tolerance.
The GPU path itself (NCCL, sharded weight upload) is tested by tests/test_gpu_tp.py.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import traceback

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from matmulfreellmcpu_b200.tp import PROJ, shard_plan  # noqa: E402

H, I = 256, 640  # multiples of 32 x 2


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("mode", ["fixed", "float"])
def test_shard_plan_covers_every_weight_once(world, mode):
    for p in PROJ:
        out = 2 * I if p == "gate_proj" else H
        k = I if p == "down_proj" else H
        hit = np.zeros((out, k), np.int32)
        for r in range(world):
            s = shard_plan(H, I, r, world, mode)[p]
            for b, e in s.rows:
                hit[b:e, s.cols[0]:s.cols[1]] += 1
        assert (hit == 1).all(), p


def test_shard_plan_rejects_unaligned_sizes():
    with pytest.raises(ValueError):
        shard_plan(96, 640, 0, 2, "fixed")  # 96 is not a multiple of 64
    with pytest.raises(ValueError):
        shard_plan(H, I, 2, 2, "fixed")


def _inputs(T, K, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, K)).astype(np.float32)
    wq = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])
    nw = (0.5 + rng.random(K)).astype(np.float32)
    return x, nw, wq


def _worker(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist

        import oracle
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        orc = oracle.Oracle()
        res = {}
        T = 5
        # FixedQ510, column-parallel o_proj on whole rows: all-gather the column slices
        x, nw, wq = _inputs(T, H, H, 1)
        s = shard_plan(H, I, rank, world, "fixed")["o_proj"]
        (b, e), = s.rows
        part, _, _ = orc.bitlinear(x, nw, wq[b:e], 20.0, act_quant=1)
        parts = [torch.empty(T, e - b) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        res["fixed_col"] = torch.cat(parts, 1).numpy()
        # FixedQ510 gate_proj SwiGLU pair: local swiglu of (gate rows, up rows), gathered
        xg, nwg, wg = _inputs(T, H, 2 * I, 2)
        s = shard_plan(H, I, rank, world, "fixed")["gate_proj"]
        rows = np.concatenate([np.arange(b, e) for b, e in s.rows])
        y, _, _ = orc.bitlinear(xg, nwg, wg[rows], 20.0, act_quant=1)
        half = y.shape[1] // 2
        z = orc.swiglu(np.ascontiguousarray(y[:, :half]).ravel(),
                       np.ascontiguousarray(y[:, half:]).ravel()).reshape(T, half)
        parts = [torch.empty(T, half) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(z))
        res["fixed_swiglu"] = torch.cat(parts, 1).numpy()
        # Float, row-parallel down_proj: partial sums of squares, then partial outputs
        xd, nwd, wd = _inputs(T, I, H, 3)
        s = shard_plan(H, I, rank, world, "float")["down_proj"]
        c0, c1 = s.cols
        xs = xd[:, c0:c1].astype(np.float64)
        ss = torch.from_numpy((xs * xs).sum(1))
        dist.all_reduce(ss)
        rstd = 1.0 / np.sqrt(ss.numpy() / I + 1e-6)
        y = xs * rstd[:, None] * nwd[c0:c1]
        out = torch.from_numpy(y @ wd[:, c0:c1].T.astype(np.float64) / 20.0)
        dist.all_reduce(out)
        res["float_row"] = out.numpy()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception:  # report instead of hanging the parent
        q.put((rank, traceback.format_exc()))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp_split_two_gloo_ranks(orc):
    T = 5
    x, nw, wq = _inputs(T, H, H, 1)
    ref_col, _, _ = orc.bitlinear(x, nw, wq, 20.0, act_quant=1)
    xg, nwg, wg = _inputs(T, H, 2 * I, 2)
    y, _, _ = orc.bitlinear(xg, nwg, wg, 20.0, act_quant=1)
    ref_sw = orc.swiglu(np.ascontiguousarray(y[:, :I]).ravel(),
                        np.ascontiguousarray(y[:, I:]).ravel()).reshape(T, I)
    xd, nwd, wd = _inputs(T, I, H, 3)
    ref_row, _, _ = orc.bitlinear(xd, nwd, wd, 20.0, act_quant=0)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, res = q.get(timeout=240)
            results[rank] = res
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank in (0, 1):
        res = results[rank]
        assert not isinstance(res, str), res
        assert np.array_equal(res["fixed_col"].view(np.uint32), ref_col.view(np.uint32))
        assert np.array_equal(res["fixed_swiglu"].view(np.uint32), ref_sw.view(np.uint32))
        tol = 1e-4 * max(1.0, float(np.abs(ref_row).max()))
        assert np.abs(res["float_row"] - ref_row).max() <= tol
