"""Episode (batch) sharding across the GPUs of one node.

Episodes are independent — no score, softmax or selection crosses an episode
— so the attention core shards over B with no data-path collective: each rank
(one process per GPU) receives a contiguous slice of episodes, runs the same
kernels on its own stream, and returns its slice of the output. The only
inter-process traffic is host plumbing: a barrier around timed regions and a
max-reduction of elapsed times (``torch.distributed``; NCCL on GPUs, gloo on
CPU).
"""

from __future__ import annotations

import datetime as _dt
import os

import torch
import torch.distributed as dist


def shard_range(B: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice [b0, b1) of B episodes for ``rank`` of ``world``:
    ceil(B / world) episodes per rank, the last ranks possibly shorter (or
    empty)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    per = -(-B // world)
    b0 = min(B, rank * per)
    return b0, min(B, b0 + per)


def env_world() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def init(backend: str, timeout_s: float = 120.0) -> bool:
    """Initialise the default process group from the environment when more
    than one rank runs; returns whether a group exists. A short timeout makes
    ranks that wait on a dead peer fail instead of hanging."""
    _, _, world = env_world()
    if world <= 1:
        return False
    if not dist.is_initialized():
        dist.init_process_group(backend=backend,
                                timeout=_dt.timedelta(seconds=timeout_s))
    return True


def barrier(device: torch.device | None = None) -> None:
    if dist.is_available() and dist.is_initialized():
        if device is not None and device.type == "cuda":
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()


def max_over_ranks(x: float, device: torch.device | None = None) -> float:
    """Maximum of a per-rank scalar (e.g. elapsed ms) over all ranks."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, device: torch.device | None = None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def shutdown() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
