"""Data-parallel serving logic (matmulfreellmcpu_b200/dp.py) on two gloo ranks on the CPU.

The GPU path shards the 64 streams of configuration 3 across ranks with no data-path
collective; what needs checking without a GPU is the host logic: the shard bounds, the
ordered gather, the error path, and the max-over-ranks timing reduction of bench.py. The
"model" of each rank is the reference restatement (oracle) of the same blob, so the sharded
result is compared with an unsharded run of the same streams.
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

from matmulfreellmcpu_b200.dp import shard_bounds  # noqa: E402


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (64, 8), (5, 2), (3, 4), (0, 2), (7, 3)])
def test_shard_bounds_partition(n, world):
    spans = [shard_bounds(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (b0, e0), (b1, _) in zip(spans, spans[1:]):
        assert e0 == b1  # contiguous, in rank order
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(8, 2, 2)
    with pytest.raises(ValueError):
        shard_bounds(8, 0, 0)


class _ShortModel:
    """Returns one stream too few on rank 1 (the gather must notice)."""

    def __init__(self, inner, rank):
        self.inner, self.rank = inner, rank

    def generate_serve(self, prompts, n, **kw):
        out = self.inner.generate_serve(prompts, n, **kw)
        return out[:-1] if self.rank == 1 and out else out


def _worker(rank, world, port, blob, prompts, gen, q):
    try:
        import torch.distributed as dist

        import oracle
        from matmulfreellmcpu_b200 import blob as B
        from matmulfreellmcpu_b200.dp import generate_serve_dp

        sys.path.insert(0, ROOT)
        import bench

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        om = oracle.Oracle().model(B.Blob.open(blob))
        got = generate_serve_dp(om, prompts, gen, rank, world)
        t = bench.allmax(float(rank + 1), world)
        err = None
        try:
            generate_serve_dp(_ShortModel(om, rank), prompts, gen, rank, world)
        except RuntimeError as ex:
            err = str(ex)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, [list(map(int, s)) for s in got], t, err))
    except Exception:  # report instead of hanging the parent
        q.put((rank, traceback.format_exc(), None, None))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_generate_serve_dp_two_gloo_ranks(orc, blob_cache):
    from matmulfreellmcpu_b200 import blob as B

    blob = B.cached_blob("tiny", 0, blob_cache)
    prompts = [B.seeded_ids(3 + (k % 3), 300 + k, 512) for k in range(5)]  # ragged, odd count
    gen = 4
    ref = orc.model(B.Blob.open(blob)).generate_serve(prompts, gen)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, blob, prompts, gen, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, streams, t, err = q.get(timeout=240)
            results[rank] = (streams, t, err)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank in (0, 1):
        streams, t, err = results[rank]
        assert not isinstance(streams, str), streams
        assert len(streams) == len(prompts)
        for a, b in zip(streams, ref):
            assert np.array_equal(np.asarray(a), np.asarray(b))
        assert t == 2.0  # max over ranks
        assert err is not None and "expected" in err
