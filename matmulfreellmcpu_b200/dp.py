"""Data-parallel serving across GPUs: one process per GPU, independent streams.

HGRN-Bit streams share nothing but the weights (the recurrent state [L, B, H] has no
cross-stream term, matmulfreellmCPU hgrn_model.cpp:139-146, :362-364), so a batch of B
streams is split into contiguous shards, each rank runs ``Model.generate_serve`` (or a
serving session) on its shard with a full weight replica, and the id streams are gathered
once at the end. Every row's arithmetic is independent of batch composition, so the
sharded result equals the single-GPU result bit for bit. No collective runs on the data path.
"""
from __future__ import annotations


def shard_bounds(n_streams: int, rank: int, world: int) -> tuple[int, int]:
    """[begin, end) of rank's contiguous shard; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(n_streams, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def gather_streams(local_streams: list, n_streams: int, rank: int, world: int, group=None):
    """All ranks' shards, in stream order (collective: every rank must call it)."""
    import torch.distributed as dist
    if world == 1:
        return list(local_streams)
    parts = [None] * world
    dist.all_gather_object(parts, [list(map(int, s)) for s in local_streams], group=group)
    out = []
    for r in range(world):
        b, e = shard_bounds(n_streams, r, world)
        if len(parts[r]) != e - b:
            raise RuntimeError(f"rank {r} returned {len(parts[r])} streams, expected {e - b}")
        out.extend(parts[r])
    return out


def generate_serve_dp(model, prompts, new_tokens: int, rank: int, world: int, **kw):
    """Model.generate_serve over this rank's shard, then gather every stream on all ranks."""
    b, e = shard_bounds(len(prompts), rank, world)
    local = model.generate_serve(prompts[b:e], new_tokens, **kw) if e > b else []
    return gather_streams(local, len(prompts), rank, world)
