"""Tensor-parallel prefill on 2 GPUs (one process per GPU, NCCL over NVLink) against one GPU
and, for configuration 4 (2.7B), against the reference's own logits.

Runs tests/tp_worker.py under torch.distributed.run. It needs two visible GPUs; with fewer
it is skipped and says so (two NCCL ranks never share one GPU).
FixedQ510 must be bit-identical to one GPU; Float within max|d| <= 1e-3 * (max - min) of the
logits.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _gpus() -> int:
    import torch
    return torch.cuda.device_count()


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(names, out_dir, world=2, timeout=1500):
    cmd = ["timeout", "-k", "60", str(timeout), sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), os.path.join(ROOT, "tests", "tp_worker.py"), *names]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MMFREE_TP_OUT=str(out_dir))
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = []
    for rank in range(world):
        with open(os.path.join(out_dir, f"rank{rank}.json")) as f:
            res.append(json.load(f))
    return res


@pytest.mark.parametrize("name", ["370M", "2.7B"])
def test_tp2_prefill_matches_one_gpu(cuda, name, tmp_path):
    if _gpus() < 2:
        pytest.skip("tensor-parallel prefill needs 2 visible GPUs")
    for res in _run([name], tmp_path):
        f, fl = res[f"{name}/fixed"], res[f"{name}/float"]
        assert f["logits_bits_equal_1gpu"] and f["first_ids_equal_1gpu"], res
        assert fl["max_abs_over_range_1gpu"] <= 1e-3, res
        if name == "2.7B":
            assert f["logits_bits_equal_reference"], res
            assert fl["max_abs_over_range_reference"] <= 1e-3, res
