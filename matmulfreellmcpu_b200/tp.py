"""Tensor-parallel prefill across GPUs (configuration 4): one process per GPU, NCCL over NVLink.

Each rank holds a shard of every per-layer BitLinear of matmulfreellmCPU's block
(cpp/src/model/hgrn_model.cpp:80-195); the library does the split and the NCCL collectives
itself (``mmfree_cuda_model_open_tp``). This module is the host side: the shard plan, the
distribution of the NCCL unique id over an existing ``torch.distributed`` group, and the
opening of a handle.

Shard plan (P ranks, rank r; H hidden, I intermediate; both multiples of 32 P):

* FixedQ510 -- every projection column-parallel: i/f/g/o/down own output rows
  [r H/P, (r+1) H/P), gate_proj owns the SwiGLU pair rows [r I/P, (r+1) I/P) and
  [I + r I/P, I + (r+1) I/P). Whole rows are all-gathered before every exact norm.
* Float -- i/f/g and gate_proj as above; o_proj and down_proj row-parallel: they own input
  columns [r H/P, (r+1) H/P) and [r I/P, (r+1) I/P); partial sums of squares and the
  row-parallel outputs are all-reduced.
"""
from __future__ import annotations

from dataclasses import dataclass

PROJ = ("i_proj", "f_proj", "g_proj", "o_proj", "gate_proj", "down_proj")


@dataclass(frozen=True)
class Shard:
    """The part of one projection's int8 weight [out, in] a rank holds."""
    rows: tuple  # tuple of (begin, end) output-row ranges, concatenated in this order
    cols: tuple  # (begin, end) input-column range


def shard_plan(hidden: int, inter: int, rank: int, world: int, mode: str) -> dict:
    """{projection: Shard} of one rank (the layout the library uploads)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if hidden % (32 * world) or inter % (32 * world):
        raise ValueError("hidden and intermediate sizes must be multiples of 32 x world")
    hs, is_ = hidden // world, inter // world
    hr, ir = (rank * hs, (rank + 1) * hs), (rank * is_, (rank + 1) * is_)
    plan = {}
    for p in PROJ:
        k = inter if p == "down_proj" else hidden
        if p == "gate_proj":
            plan[p] = Shard(rows=(ir, (inter + ir[0], inter + ir[1])), cols=(0, hidden))
        elif mode == "float" and p == "o_proj":
            plan[p] = Shard(rows=((0, hidden),), cols=hr)
        elif mode == "float" and p == "down_proj":
            plan[p] = Shard(rows=((0, hidden),), cols=ir)
        else:
            plan[p] = Shard(rows=(hr,), cols=(0, k))
    return plan


def broadcast_nccl_id(rank: int, group=None) -> bytes:
    """NCCL unique id created on rank 0 and broadcast over a torch.distributed group
    (collective)."""
    import torch.distributed as dist

    from . import api
    obj = [api.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def open_model(blob_path: str, mode: str, rank: int, world: int, device: int, group=None):
    """A tensor-parallel handle of this rank (collective over the group's ranks)."""
    from . import api
    nid = broadcast_nccl_id(rank, group)
    return api.Model.open_tp(blob_path, mode, rank, world, nid, device=device)
