"""Checkpoint / resume of a resident rollout.

A checkpoint holds what continues a rollout bit for bit: the particles
(positions [B*N, 4], states [B*N*C] f32), the executor's step index and its
stochastic-mask settings (update_prob, seed, optional per-lane seeds; the mask
of step s depends on them and on s, crates/burn_automata/src/gpu_step.wgsl:1019-1056).
The file is a NumPy .npz with a format tag and the shape fields, so a loader
rejects a checkpoint of another batch or channel count instead of reading it
wrongly.  The reference's counterpart is the final state that
`infer --output` writes (crates/burn_automata/src/cli/commands/basic.rs);
a rollout trace JSON from `bpk.infer` can be turned into a checkpoint with
`from_trace`.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

from .config import InvalidArgument

FORMAT = "burn_automata_b200.checkpoint/1"


@dataclass
class Checkpoint:
    positions: np.ndarray      # [B*N, 4] f32
    states: np.ndarray         # [B*N*C] f32
    batch_size: int
    particle_count: int
    state_dims: int
    step_index: int = 0
    update_prob: float = 1.0
    seed: int = 0
    lane_seeds: Optional[np.ndarray] = None  # [B] u64

    def validate(self) -> None:
        total = self.batch_size * self.particle_count
        if self.batch_size < 0 or self.particle_count < 0 or self.state_dims < 0:
            raise InvalidArgument("checkpoint sizes must be non-negative")
        if self.positions.shape != (total, 4) or self.positions.dtype != np.float32:
            raise InvalidArgument(f"checkpoint positions must be float32 [{total}, 4], got "
                                  f"{self.positions.dtype} {list(self.positions.shape)}")
        if self.states.shape != (total * self.state_dims,) or self.states.dtype != np.float32:
            raise InvalidArgument(f"checkpoint states must be float32 [{total * self.state_dims}]"
                                  f", got {self.states.dtype} {list(self.states.shape)}")
        if not 0 <= self.step_index <= 0xFFFFFFFF:
            raise InvalidArgument("checkpoint step index outside the executor's u32 counter")
        if self.lane_seeds is not None and self.lane_seeds.shape != (self.batch_size,):
            raise InvalidArgument("checkpoint lane seeds do not match the batch size")


def save(path: str, ck: Checkpoint) -> None:
    """Writes `ck` to `path` (.npz), atomically (temporary file + rename)."""
    ck.validate()
    meta = {"format": FORMAT, "batch_size": ck.batch_size, "particle_count": ck.particle_count,
            "state_dims": ck.state_dims, "step_index": int(ck.step_index),
            "update_prob": float(ck.update_prob), "seed": int(ck.seed) & 0xFFFFFFFFFFFFFFFF,
            "has_lane_seeds": ck.lane_seeds is not None}
    arrays = {"positions": ck.positions, "states": ck.states,
              "meta": np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)}
    if ck.lane_seeds is not None:
        arrays["lane_seeds"] = np.asarray(ck.lane_seeds, dtype=np.uint64)
    tmp = f"{path}.tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        np.savez(f, **arrays)
    os.replace(tmp, path)


def load(path: str) -> Checkpoint:
    """Reads a checkpoint written by `save`; InvalidArgument when the file is
    not one or its arrays do not match its own shape fields."""
    try:
        with np.load(path, allow_pickle=False) as z:
            meta = json.loads(bytes(z["meta"]).decode())
            pos = np.array(z["positions"])
            st = np.array(z["states"])
            lanes = np.array(z["lane_seeds"]) if meta.get("has_lane_seeds") else None
    except (OSError, KeyError, ValueError) as e:
        raise InvalidArgument(f"not a rollout checkpoint: {path}: {e}") from e
    if meta.get("format") != FORMAT:
        raise InvalidArgument(f"unknown checkpoint format {meta.get('format')!r}")
    ck = Checkpoint(pos, st, int(meta["batch_size"]), int(meta["particle_count"]),
                    int(meta["state_dims"]), int(meta["step_index"]),
                    float(meta["update_prob"]), int(meta["seed"]), lanes)
    ck.validate()
    return ck


def from_trace(trace_json: str, step_index: int = 0) -> Checkpoint:
    """A checkpoint from the RolloutTrace JSON that `bpk.infer` writes
    (crates/burn_automata/src/rollout/mod.rs:152-161: positions as [x, y, z, w]
    records, states flat, batch_size / particle_count / state_dims): the final
    particles, mask off."""
    try:
        with open(trace_json) as f:
            d = json.load(f)
        pos = np.asarray(d["positions"], dtype=np.float32).reshape(-1, 4)
        st = np.asarray(d["states"], dtype=np.float32).reshape(-1)
        b, n, c = int(d["batch_size"]), int(d["particle_count"]), int(d["state_dims"])
    except (OSError, KeyError, ValueError, TypeError) as e:
        raise InvalidArgument(f"not a rollout trace: {trace_json}: {e}") from e
    ck = Checkpoint(pos, st, b, n, c, int(step_index))
    ck.validate()
    return ck
