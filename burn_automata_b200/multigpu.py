"""One process per GPU over independent rollout shards.

Batches of independent rollouts (the reference keeps them as separate lanes:
crates/burn_automata_kernels/src/hashgrid.rs:33-58) shard across GPUs with no
exchange on the step path.  This module holds the rank plumbing around that:
shard assignment, process-group set-up with a short timeout, the
max-over-ranks reduction used for timing, and one optional gather of
per-shard checksums of the final states for validation.  Nothing here runs
inside the timed region.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta
from typing import Optional, Tuple

import numpy as np


@dataclass
class RankInfo:
    rank: int
    world: int
    local_rank: int


def env_rank() -> RankInfo:
    def get(name, default):
        try:
            return int(os.environ.get(name, default))
        except ValueError:
            return default

    return RankInfo(get("RANK", 0), get("WORLD_SIZE", 1), get("LOCAL_RANK", 0))


def shard(total_rollouts: int, world: int, rank: int, strong: bool) -> Tuple[int, int]:
    """(first rollout index, rollouts on this rank).

    strong: the `total_rollouts` rollouts are split as evenly as possible
    (the first `total % world` ranks take one more).  weak: every rank runs its
    own `total_rollouts` rollouts, numbered after the previous ranks'."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    if not strong:
        return rank * total_rollouts, total_rollouts
    base, extra = divmod(total_rollouts, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def init(backend: str, info: RankInfo, timeout_s: float = 120.0, device=None):
    """Process group over the torchrun environment (127.0.0.1 rendezvous)."""
    import torch.distributed as dist

    if info.world <= 1:
        return None
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kwargs = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None:
        kwargs["device_id"] = device
    dist.init_process_group(backend, **kwargs)
    return dist


def max_over_ranks(values, device=None):
    """Element-wise max over ranks of a small list of floats."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]


def shard_checksum(positions: np.ndarray, states: np.ndarray) -> Tuple[float, float]:
    """Order-dependent float64 checksums of a shard's final particles."""
    p = np.asarray(positions, np.float64).reshape(-1)
    s = np.asarray(states, np.float64).reshape(-1)
    wp = np.arange(1, p.size + 1, dtype=np.float64)
    ws = np.arange(1, s.size + 1, dtype=np.float64)
    return float(np.dot(p, 1.0 / wp)), float(np.dot(s, 1.0 / ws))


def gather_checksums(local: Tuple[float, float], device=None):
    """All ranks' checksums, in rank order (one all_gather, after timing)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(local), dtype=torch.float64, device=device)
    if not (dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1):
        return [tuple(float(v) for v in t.cpu())]
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [tuple(float(v) for v in o.cpu()) for o in out]


def barrier_or_fail(timeout_s: Optional[float] = None) -> None:
    """Barrier that raises (instead of hanging) when a rank is gone.

    With gloo, monitored_barrier names the ranks that did not arrive; other
    backends rely on the process group's timeout."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() <= 1:
        return
    if dist.get_backend() == "gloo" and timeout_s is not None:
        dist.monitored_barrier(timeout=timedelta(seconds=timeout_s))
    else:
        dist.barrier()


def finish() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
