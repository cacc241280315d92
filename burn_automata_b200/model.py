"""NpaModel, the rollout driver and the resident executor, backed by the CUDA library.

Mirrors crates/burn_automata:
  NpaWeights / NpaModel::{step_cpu, forward_update_from_features,
                          forward_from_features_with_eps}   src/model.rs:11-17, :768-940
  RolloutConfig / RolloutTrace / run_rollout_from_particles  src/rollout/mod.rs:102-283
  WgpuAutomataExecutor::{create_state, step_state_many, read_state}
                                                              src/gpu/executor/*
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import _lib
from .config import InvalidArgument, NpaConfig, HashGridConfig


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _fp(a):
    return None if a is None else a.ctypes.data_as(_lib.f32p)


@dataclass
class NpaWeights:
    """model.rs:11-17: w1 [hidden, perception_dims], b1 [hidden], w2 [update_dims, hidden], b2."""

    w1: np.ndarray
    b1: np.ndarray
    w2: np.ndarray
    b2: np.ndarray

    @staticmethod
    def zeros(cfg: NpaConfig) -> "NpaWeights":
        f, h, o = cfg.perception_dims(), cfg.hidden_dims, cfg.update_dims()
        return NpaWeights(np.zeros(h * f, np.float32), np.zeros(h, np.float32),
                          np.zeros(o * h, np.float32), np.zeros(o, np.float32))


@dataclass
class StepOutput:
    """model.rs:735-744 (perception carries the features and density)."""

    next_positions: np.ndarray
    next_states: np.ndarray
    dx: np.ndarray
    ds: np.ndarray
    features: np.ndarray
    density: np.ndarray


class NpaModel:
    """NpaModel { config, weights } with the weights resident on one CUDA device."""

    def __init__(self, config: NpaConfig, weights, device: int = 0):
        self.config = config
        self.weights = weights
        self.device = int(device)
        L = _lib.lib()
        m = _lib.model_c(config)
        ws = [_f32(getattr(weights, k)).reshape(-1) for k in ("w1", "b1", "w2", "b2")]
        handle = ctypes.c_void_p()
        _lib.check(L.npa_model_create(ctypes.byref(m), _fp(ws[0]), ws[0].shape[0], _fp(ws[1]),
                                      ws[1].shape[0], _fp(ws[2]), ws[2].shape[0], _fp(ws[3]),
                                      ws[3].shape[0], self.device, ctypes.byref(handle)),
                   "NpaModel")
        self._handle = handle

    @property
    def handle(self):
        return self._handle

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None and self._handle.value:
            _lib.lib().npa_model_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward_update_from_features(self, features) -> np.ndarray:
        """model.rs:900-940."""
        f = _f32(features).reshape(-1)
        F = self.config.perception_dims()
        rows = f.shape[0] // F if F else 0
        out = np.zeros(rows * self.config.update_dims(), np.float32)
        _lib.check(_lib.lib().npa_model_forward_update_from_features(
            self._handle, _fp(f), f.shape[0], _fp(out), out.shape[0]),
            "forward_update_from_features")
        return out

    def forward_from_features_with_eps(self, features, eps: float):
        """model.rs:867-898 (host-side composition of the device MLP)."""
        update = self.forward_update_from_features(features).reshape(-1, self.config.update_dims())
        D, C = self.config.spatial_dims, self.config.state_dims
        rows = update.shape[0]
        dx = np.zeros((rows, 4), np.float32)
        ds = np.zeros((rows, C), np.float32)
        motion_eps = np.float32(self.config.motion_eps(eps))
        alpha = np.float32(self.config.alpha)
        for r in range(rows):
            u = update[r]
            norm = np.float32(0.0)
            for a in range(D):
                norm = np.float32(norm + np.float32(u[a] * u[a]))
            norm = np.float32(np.sqrt(norm))
            for a in range(D):
                dx[r, a] = np.float32(np.float32(np.float32(alpha * u[a]) * motion_eps)
                                      / np.float32(1.0 + norm))
            ds[r] = u[D:D + C]
        return dx, ds.reshape(-1)

    def step(self, positions, states, batch_size: int, particle_count: int,
             grid: HashGridConfig, dt: float, update_mask=None,
             outputs=("dx", "ds", "features", "density"), out=None) -> StepOutput:
        """NpaModel::step_cpu (model.rs:768-858), executed on the GPU.

        `outputs` selects which of the StepOutput extras are copied back (the
        reference always builds all of them); `out` = (next_positions,
        next_states) or (next_positions, next_states, dx, ds, features,
        density) reuses caller-owned float32 host arrays (None entries fall
        back to `outputs`).  With page-locked buffers throughout, a batch of
        several rollouts is stepped in rollout chunks whose copies overlap the
        neighbouring chunks' kernels."""
        pos = _f32(positions).reshape(-1, 4) if np.size(positions) else np.zeros((0, 4), np.float32)
        st = _f32(states).reshape(-1)
        total = batch_size * particle_count
        C = self.config.state_dims
        F = self.config.perception_dims()
        mask = _f32(update_mask).reshape(-1) if update_mask is not None else None
        sizes = {"next_positions": max(total, 0) * 4, "next_states": max(total * C, 0),
                 "dx": max(total, 0) * 4, "ds": max(total * C, 0),
                 "features": max(total * F, 0), "density": max(total, 0)}
        given = {}
        if out is not None:
            if len(out) not in (2, 6) or out[0] is None or out[1] is None:
                raise InvalidArgument("out is (next_positions, next_states[, dx, ds, features, "
                                      "density])")
            given = {k: a for k, a in zip(sizes, out) if a is not None}
            for k, a in given.items():
                if (not isinstance(a, np.ndarray) or a.dtype != np.float32
                        or not a.flags.c_contiguous or a.size != sizes[k]):
                    raise InvalidArgument(f"out buffer {k} must be contiguous float32 of the "
                                          "step's size")
        want = set(outputs or ()) | {"next_positions", "next_states"}

        def buf(k, shape):
            if k in given:
                return given[k]
            return np.zeros(shape, np.float32) if k in want else None
        npos = buf("next_positions", (max(total, 0), 4))
        nst = buf("next_states", max(total * C, 0))
        dx = buf("dx", (max(total, 0), 4))
        ds = buf("ds", max(total * C, 0))
        feats = buf("features", max(total * F, 0))
        dens = buf("density", max(total, 0))
        g = _lib.grid_c(grid)
        _lib.check(_lib.lib().npa_model_step(
            self._handle, ctypes.byref(g), _fp(pos), pos.shape[0], _fp(st), st.shape[0],
            batch_size, particle_count, float(dt), _fp(mask), _fp(npos), _fp(nst), _fp(dx),
            _fp(ds), _fp(feats), _fp(dens)), "step")
        return StepOutput(npos, nst, dx, ds, feats, dens)

    # step_cpu is the reference's name for the same operation.
    step_cpu = step


@dataclass
class RolloutConfig:
    """rollout/mod.rs:102-124 (seeding fields are unused: inputs are given)."""

    batch_size: int = 1
    particle_count: int = 4096
    steps: int = 32
    dt: float = 1.0
    update_prob: float = 1.0
    seed: int = 42
    seed_scale: float = 0.2


@dataclass
class RolloutTrace:
    """rollout/mod.rs:152-161."""

    positions: np.ndarray
    states: np.ndarray
    batch_size: int
    particle_count: int
    state_dims: int
    steps: int
    mean_dx: np.ndarray = None


def run_rollout_from_particles(model: NpaModel, grid: HashGridConfig, cfg: RolloutConfig,
                               positions, states) -> RolloutTrace:
    """rollout/mod.rs:222-283: cfg.steps steps from the given particles.  With
    update_prob < 1 every step's update is masked by the reference's
    stochastic_mask stream (StdRng seeded with cfg.seed ^ 0x5eed; see
    rollout_update_masks)."""
    pos = _f32(positions).reshape(-1, 4).copy()
    st = _f32(states).reshape(-1).copy()
    g = _lib.grid_c(grid)
    mean_dx = np.zeros(max(cfg.steps, 1), np.float32)
    _lib.check(_lib.lib().npa_model_run_rollout_seeded(
        model.handle, ctypes.byref(g), _fp(pos), pos.shape[0], _fp(st), st.shape[0],
        cfg.batch_size, cfg.particle_count, cfg.steps, float(cfg.dt), float(cfg.update_prob),
        int(cfg.seed) & 0xFFFFFFFFFFFFFFFF, _fp(mean_dx)), "run_rollout")
    return RolloutTrace(pos, st, cfg.batch_size, cfg.particle_count, model.config.state_dims,
                        cfg.steps, mean_dx[:cfg.steps])


def rollout_update_masks(seed: int, update_prob: float, count: int, steps: int,
                         first_step: int = 0) -> np.ndarray:
    """stochastic_mask (rollout/mod.rs:644-651) as run_rollout_from_particles
    with cfg.seed = seed draws it: [steps, count] for steps first_step.. (0-based).
    The stream is rand 0.9's StdRng (ChaCha12) seeded by seed_from_u64(seed ^
    0x5eed), restated and computed on the GPU."""
    out = np.zeros((steps, count), np.float32)
    _lib.check(_lib.lib().npa_rollout_update_masks(int(seed) & 0xFFFFFFFFFFFFFFFF,
                                                   float(update_prob), count, first_step, steps,
                                                   _fp(out)), "rollout_update_masks")
    return out


class CudaAutomataExecutor:
    """Resident rollout state on one GPU (the CUDA counterpart of WgpuAutomataExecutor)."""

    def __init__(self, model: NpaModel, grid: HashGridConfig, batch_size: int,
                 particle_count: int):
        self.model = model
        self.grid = grid
        self.batch_size = batch_size
        self.particle_count = particle_count
        h = ctypes.c_void_p()
        g = _lib.grid_c(grid)
        _lib.check(_lib.lib().npa_executor_create(model.handle, ctypes.byref(g), batch_size,
                                                  particle_count, ctypes.byref(h)), "executor")
        self._handle = h

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None and self._handle.value:
            _lib.lib().npa_executor_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def create_state(self, positions, states, update_prob: float = 1.0, seed: int = 0,
                     lane_seeds=None) -> None:
        """create_state / create_state_with_update_prob (gpu/executor/state.rs:6-55):
        uploads the particles and restarts the step index at 0.  update_prob < 1
        applies the executor's counter-based stochastic update mask (see
        set_update_prob)."""
        pos = _f32(positions).reshape(-1, 4)
        st = _f32(states).reshape(-1)
        _lib.check(_lib.lib().npa_executor_upload_state(self._handle, _fp(pos), _fp(st)),
                   "create_state")
        self.set_step_index(0)
        self.set_update_prob(update_prob, seed, lane_seeds)

    def set_update_prob(self, update_prob: float, seed: int = 0, lane_seeds=None) -> None:
        """Stochastic update mask of later steps: particle i of lane l updates
        when random01(i, step_index, lane seed) < update_prob; lane seeds are
        fold(seed) ^ (l * particle_count), or fold(lane_seeds[l]) when given."""
        ls = None
        arr = None
        if lane_seeds is not None:
            arr = np.ascontiguousarray(np.asarray(lane_seeds, dtype=np.uint64))
            if arr.size != self.batch_size:
                raise InvalidArgument(f"lane seed count {arr.size} does not match batch size "
                                      f"{self.batch_size}")
            ls = arr.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
        _lib.check(_lib.lib().npa_executor_set_update_prob(
            self._handle, float(update_prob), int(seed) & 0xFFFFFFFFFFFFFFFF, ls),
            "set_update_prob")
        self._mask = (float(update_prob), int(seed) & 0xFFFFFFFFFFFFFFFF,
                      None if arr is None else arr.copy())

    def save_checkpoint(self, path: str) -> None:
        """Writes the resident particles, the step index and the mask settings
        (checkpoint.py); load_checkpoint on an executor of the same shape
        continues the rollout bit for bit."""
        from . import checkpoint

        pos, st = self.read_state()
        prob, seed, lanes = getattr(self, "_mask", (1.0, 0, None))
        checkpoint.save(path, checkpoint.Checkpoint(
            pos, st, self.batch_size, self.particle_count, self.model.config.state_dims,
            self.step_index, prob, seed, lanes))

    def load_checkpoint(self, path: str) -> None:
        """Restores a checkpoint written by save_checkpoint (same batch, particle
        count and channel count)."""
        from . import checkpoint

        ck = checkpoint.load(path)
        if (ck.batch_size, ck.particle_count, ck.state_dims) != (
                self.batch_size, self.particle_count, self.model.config.state_dims):
            raise InvalidArgument(
                f"checkpoint of {ck.batch_size} x {ck.particle_count} particles with "
                f"{ck.state_dims} channels does not fit this executor ({self.batch_size} x "
                f"{self.particle_count}, {self.model.config.state_dims})")
        self.create_state(ck.positions, ck.states, ck.update_prob, ck.seed, ck.lane_seeds)
        self.set_step_index(ck.step_index)

    @property
    def step_index(self) -> int:
        v = ctypes.c_uint32(0)
        _lib.check(_lib.lib().npa_executor_step_index(self._handle, ctypes.byref(v)), "step_index")
        return v.value

    def set_step_index(self, step_index: int) -> None:
        _lib.check(_lib.lib().npa_executor_set_step_index(self._handle,
                                                          int(step_index) & 0xFFFFFFFF),
                   "set_step_index")

    def set_state_device(self, d_positions, d_states, stream=None) -> None:
        _lib.check(_lib.lib().npa_executor_set_state_device(
            self._handle, d_positions.data_ptr(), d_states.data_ptr(), stream), "set_state")

    def step_state_many(self, steps: int, dt: float, use_graph: bool = True, stream=None) -> None:
        _lib.check(_lib.lib().npa_executor_step_many(self._handle, int(steps), float(dt),
                                                     1 if use_graph else 0, stream),
                   "step_state_many")

    def step_state_many_profiled(self, steps: int, dt: float, use_graph: bool = True,
                                 stream=None):
        """step_state_many with CUDA events around every phase of every step.
        Returns (phase_ms [steps, 4] for hashgrid / density / perception / MLP step,
        total_ms)."""
        phase = np.zeros((int(steps), 4), np.float32)
        total = ctypes.c_float(0.0)
        _lib.check(_lib.lib().npa_executor_step_many_profiled(
            self._handle, int(steps), float(dt), 1 if use_graph else 0, stream, _fp(phase),
            ctypes.byref(total)), "step_state_many_profiled")
        return phase, float(total.value)

    def read_state(self):
        total = self.batch_size * self.particle_count
        pos = np.zeros((total, 4), np.float32)
        st = np.zeros(total * self.model.config.state_dims, np.float32)
        _lib.check(_lib.lib().npa_executor_read_state(self._handle, _fp(pos), _fp(st)),
                   "read_state")
        return pos, st

    def state_device_ptrs(self):
        p, s = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(_lib.lib().npa_executor_state_device(self._handle, ctypes.byref(p),
                                                        ctypes.byref(s)), "state_device")
        return p.value, s.value

    def set_fused_step(self, fused=True) -> None:
        """Run perception, the MLP and the Euler step as one kernel per step
        (feature rows kept in shared memory) instead of two; same results.
        fused = 2 selects the warp-specialised form (perception warps and
        MLP warps in one block per SM)."""
        mode = 2 if fused == 2 else int(bool(fused))
        _lib.check(_lib.lib().npa_executor_set_fused_step(self._handle, mode), "set_fused_step")

    def set_step_groups(self, groups: int) -> None:
        """Replay the batch as `groups` independent chains of rollouts (1..4),
        overlapping their latency-bound phases; same results."""
        _lib.check(_lib.lib().npa_executor_set_step_groups(self._handle, int(groups)),
                   "set_step_groups")

    @property
    def step_groups(self) -> int:
        v = ctypes.c_int32(0)
        _lib.check(_lib.lib().npa_executor_step_groups(self._handle, ctypes.byref(v)),
                   "step_groups")
        return v.value

    def launches_per_step(self) -> int:
        v = ctypes.c_int64(0)
        _lib.check(_lib.lib().npa_executor_launches_per_step(self._handle, ctypes.byref(v)),
                   "launches_per_step")
        return v.value
