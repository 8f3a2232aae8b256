"""Request-level replicas across GPUs: one process per GPU, each holding a full model replica and
serving its own requests; no collective on the data path (the reference's natural sharding is by
request: seeded request i goes to GPU i mod N). The only cross-rank traffic is host control:
barriers around the timed region, the max-over-ranks of device-timed durations, and failure
detection (a short process-group timeout turns a rank that died or never joined into an error on
the survivors instead of a hang).

Used by ``bench.py`` under ``torch.distributed.run`` (NCCL on GPUs) and tested with ``gloo`` on CPU.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist

SEED_STRIDE = 1000  # request seeds of rank r: SEED_STRIDE * r + i (disjoint while i < SEED_STRIDE)


def dist_env() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the launcher's environment (1 process when absent)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, timeout_s: float = 300.0, device: torch.device | None = None) -> bool:
    """Joins the process group when the launcher started more than one rank; returns whether it
    did. Rendezvous comes from MASTER_ADDR / MASTER_PORT (use 127.0.0.1 on one node)."""
    _, world, _ = dist_env()
    if world <= 1:
        return False
    kwargs = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None and device.type == "cuda":
        kwargs["device_id"] = device
    dist.init_process_group(backend, **kwargs)
    return True


def request_seed(rank: int, i: int) -> int:
    """Seed of the i-th request served by `rank` (distinct across ranks)."""
    if not 0 <= i < SEED_STRIDE:
        raise ValueError(f"request index {i} outside [0, {SEED_STRIDE})")
    return SEED_STRIDE * rank + i


def requests_for_rank(n_requests: int, world: int, rank: int) -> list[int]:
    """Global request ids served by `rank`: i with i mod world == rank."""
    return list(range(rank, n_requests, world))


def max_over_ranks(x: float, device: torch.device | None = None) -> float:
    """Maximum of a host value over all ranks (the device-timed duration a job takes is that of its
    slowest rank); the value itself when running alone."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier() -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def aggregate_rate(count_per_rank: float, seconds_max: float, world: int) -> float:
    """Whole-job throughput of `world` replicas that each processed `count_per_rank` units, timed
    as the slowest rank's duration (weak scaling: per-rank work fixed as ranks are added)."""
    if seconds_max <= 0:
        raise ValueError("duration must be positive")
    return world * count_per_rank / seconds_max


def shutdown() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
