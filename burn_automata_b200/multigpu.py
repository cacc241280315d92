"""One process per GPU over independent rollout shards.

Batches of independent rollouts (the reference keeps them as separate lanes:
crates/burn_automata_kernels/src/hashgrid.rs:33-58) shard across GPUs with no
exchange on the step path.  This module holds the rank plumbing around that:
shard assignment, process-group set-up with a short timeout, the
max-over-ranks reduction used for timing, and one gather of per-rollout
digests of the final states, which rank 0 compares with a 1-GPU rerun of
the same rollouts (rollouts are independent and the kernels deterministic,
so a sharded run reproduces it bit for bit).  Nothing here runs inside the
timed region.
"""

from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass
from datetime import timedelta
from typing import Dict, Iterable, List, Optional, Tuple

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


def rollout_digests(batch: int, first: int, positions: np.ndarray,
                    states: np.ndarray) -> Dict[int, str]:
    """{global rollout index: 64-bit digest of that rollout's bytes}.

    positions / states hold `batch` consecutive rollouts (any per-rollout
    layout: each array splits evenly into `batch` rows).  Equal digests mean
    bit-identical rollouts."""
    p = np.ascontiguousarray(positions).reshape(batch, -1)
    s = np.ascontiguousarray(states).reshape(batch, -1)
    return {first + b: hashlib.blake2b(p[b].tobytes() + s[b].tobytes(),
                                       digest_size=8).hexdigest() for b in range(batch)}


def compare_digests(gathered: Iterable[Dict[int, str]],
                    expected: Dict[int, str]) -> Tuple[int, List[int]]:
    """(rollouts checked, rollouts whose digest differs from `expected` or
    that `expected` lacks), over every rank's gathered digests."""
    got: Dict[int, str] = {}
    for d in gathered:
        got.update(d)
    bad = sorted(k for k, v in got.items() if expected.get(k) != v)
    return len(got), bad


def gather_floats(value: float, device=None):
    """Every rank's `value`, in rank order (one all_gather, outside timing)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if not (dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1):
        return [float(t.item())]
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def gather_objects(obj):
    """Every rank's picklable `obj`, in rank order (validation data only: one
    all_gather_object after the timed region)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1):
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


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
