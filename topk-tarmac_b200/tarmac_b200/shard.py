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


def local_cpus(pci_bus_id: str, nvml=None) -> list[int] | None:
    """The host CPUs NVML reports as local to the GPU at ``pci_bus_id``
    (its NUMA node), intersected with this process's current affinity; None
    when NVML is unavailable or reports nothing usable. Reads only."""
    try:
        if nvml is None:
            import pynvml as nvml  # nvidia-ml-py
        nvml.nvmlInit()
    except Exception:
        return None
    try:
        h = nvml.nvmlDeviceGetHandleByPciBusId(pci_bus_id)
        words = 64  # 64-bit words: 4096 CPUs
        mask = nvml.nvmlDeviceGetCpuAffinity(h, words)
        cpus = {64 * w + b for w, m in enumerate(mask) for b in range(64) if (int(m) >> b) & 1}
    except Exception:
        return None
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:
            pass
    cpus &= set(os.sched_getaffinity(0))
    return sorted(cpus) or None


def bind_to_gpu_cpus(device: torch.device, nvml=None) -> list[int] | None:
    """Restrict this process (one rank) to the host CPUs local to its GPU, so
    its pinned host buffers are allocated and copied from that GPU's NUMA
    node. Changes only this process's CPU affinity; returns the CPU list, or
    None when it left the affinity unchanged."""
    props = torch.cuda.get_device_properties(device)
    bus = getattr(props, "pci_bus_id", None)
    if bus is None:
        return None
    dom = getattr(props, "pci_domain_id", 0)
    dev_id = getattr(props, "pci_device_id", 0)
    cpus = local_cpus(f"{dom:08X}:{bus:02X}:{dev_id:02X}.0", nvml)
    if cpus:
        os.sched_setaffinity(0, cpus)
    return cpus


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
