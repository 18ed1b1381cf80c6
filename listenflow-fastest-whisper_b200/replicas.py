"""Data-parallel replicas: one process per GPU, each with a full copy of the
FP8 weights, each running its own audio streams.  The path has no exchange
step (the reference runs one engine per device, python/src/listenflow/
fastest_whisper/_engine.py:81-88), so torch.distributed is used only for
plumbing: a barrier around timed regions and the max-over-ranks reduction of
elapsed times.
"""

from __future__ import annotations

import datetime
import os


def env_rank() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def shard(units: int, rank: int, world: int) -> range:
    """The contiguous block of `units` (streams, batch rows) owned by `rank`.
    Blocks differ in size by at most one and cover every unit exactly once."""
    if world < 1 or not 0 <= rank < world or units < 0:
        raise ValueError(f"bad shard request: units={units} rank={rank} world={world}")
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def init(backend: str, timeout_s: float = 120.0, device=None):
    """Initialise the default process group (short timeout: a rank that dies
    makes the others fail fast at their next collective instead of hanging)."""
    import torch.distributed as dist

    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kwargs["device_id"] = device
    dist.init_process_group(backend, **kwargs)
    return dist


def max_over_ranks(values, dist=None, device=None):
    """Element-wise maximum of a list of floats across ranks (identity when alone)."""
    import torch

    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu().tolist()]


def whole_job_rate(units_per_rank: float, world: int, seconds: float) -> float:
    """Aggregate throughput: units processed by all ranks over the slowest rank's time."""
    if seconds <= 0:
        raise ValueError("elapsed time must be positive")
    return units_per_rank * world / seconds
