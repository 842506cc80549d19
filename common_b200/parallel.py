"""Host-side plumbing of tensor parallelism: one process per GPU.

The library forms its own NCCL communicator from a 128-byte unique id (qw_get_unique_id on rank 0,
qw_create on every rank).  These helpers move that id and the per-rank timings over an existing
torch.distributed process group (NCCL on the GPU box, gloo on CPU in the tests); the data path
never goes through them.  The reference has no parallelism for this path (a single
AutoregressiveModel per process, engine/ml/src/main/java/org/almostrealism/ml/AutoregressiveModel.java).
"""
from __future__ import annotations

import os
from typing import Callable


def launch_env() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) as set by torch.distributed.run; (0, 1, 0) for a plain launch."""
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def share_unique_id(make_id: Callable[[], bytes]) -> bytes | None:
    """Rank 0 calls make_id() (normally native.unique_id) and every rank receives the same bytes;
    None when no process group is initialised (a single process)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return None
    obj = [make_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    nid = obj[0]
    if not isinstance(nid, (bytes, bytearray)) or len(nid) != 128:
        raise RuntimeError("NCCL unique id must be 128 bytes")
    return bytes(nid)


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of `value` over all ranks (the job's time is its slowest rank's)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard_rows(n: int, rank: int, world: int) -> tuple[int, int]:
    """The contiguous slice [lo, hi) of n rows (heads, vocabulary rows, intermediate rows) that a rank
    keeps under Megatron-style sharding; n must divide by world (the library enforces the same)."""
    if n % world:
        raise ValueError(f"{n} rows do not divide over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per
