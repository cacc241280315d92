"""The training rollout's f32 backprop through time, on the GPU.

Mirrors crates/burn_automata:
  SupervisedGradients / mlp_backward_from_output_gradients  src/training.rs:110-116, :558-640
  RolloutForTraining / rollout_for_training                 src/target2d.rs:982-997, :3414-3466
  bptt_gradients                                            src/target2d.rs:3550-3722
The loss that produces the final-state adjoints (target2d.rs:3469-3548) is
the caller's: bptt_gradients takes its position and state gradients.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _lib
from .config import HashGridConfig, InvalidArgument
from .model import NpaModel, _f32, _fp


@dataclass
class SupervisedGradients:
    """training.rs:110-116 (features: the gradient of the rows' features;
    bptt_gradients leaves it empty, as the reference's total does not
    accumulate it)."""

    w1: np.ndarray
    b1: np.ndarray
    w2: np.ndarray
    b2: np.ndarray
    features: np.ndarray


@dataclass
class RolloutForTraining:
    """target2d.rs:989-997 with the snapshots stacked: snapshot_positions
    [steps, B*N, 4], snapshot_states [steps, B*N*C], snapshot_masks
    [steps, B*N] are step k's inputs."""

    snapshot_positions: np.ndarray
    snapshot_states: np.ndarray
    snapshot_masks: np.ndarray
    final_positions: np.ndarray
    final_states: np.ndarray
    mean_dx_norm_sum: float
    steps: int
    batch_size: int
    particle_count: int


def _weight_buffers(model: NpaModel):
    c = model.config
    f, h, o = c.perception_dims(), c.hidden_dims, c.update_dims()
    return (np.zeros(h * f, np.float32), np.zeros(h, np.float32), np.zeros(o * h, np.float32),
            np.zeros(o, np.float32))


def mlp_backward_from_output_gradients(model: NpaModel, features,
                                       output_gradients) -> SupervisedGradients:
    """training.rs:558-640: the MLP's weight and feature gradients for the
    rows of `features` given the adjoint of their raw update."""
    feats = _f32(features).reshape(-1)
    grads = _f32(output_gradients).reshape(-1)
    gw1, gb1, gw2, gb2 = _weight_buffers(model)
    F = model.config.perception_dims()
    gf = np.zeros(feats.size if F and feats.size % F == 0 else 0, np.float32)
    _lib.check(_lib.lib().npa_model_mlp_backward(
        model.handle, _fp(feats), feats.size, _fp(grads), grads.size, _fp(gw1), _fp(gb1),
        _fp(gw2), _fp(gb2), _fp(gf) if gf.size else _fp(np.zeros(1, np.float32))),
        "mlp_backward_from_output_gradients")
    return SupervisedGradients(gw1, gb1, gw2, gb2, gf)


def rollout_for_training(model: NpaModel, grid: HashGridConfig, positions, states,
                         batch_size: int, particle_count: int, steps: int,
                         update_prob: float = 1.0, seed: int = 0) -> RolloutForTraining:
    """target2d.rs:3414-3466: `steps` Euler steps with dt = 1, each update
    masked by stochastic_mask of StdRng::seed_from_u64(seed ^ 0x5eed2d),
    recording every step's input."""
    pos = _f32(positions).reshape(-1, 4)
    st = _f32(states).reshape(-1)
    total = batch_size * particle_count
    C = model.config.state_dims
    if steps < 0:
        raise InvalidArgument("steps must be >= 0")
    sp = np.zeros((steps, max(total, 0), 4), np.float32)
    ss = np.zeros((steps, max(total * C, 0)), np.float32)
    sm = np.zeros((steps, max(total, 0)), np.float32)
    fp = np.zeros((max(total, 0), 4), np.float32)
    fs = np.zeros(max(total * C, 0), np.float32)
    mean = np.zeros(1, np.float32)
    g = _lib.grid_c(grid)
    _lib.check(_lib.lib().npa_model_rollout_for_training(
        model.handle, ctypes.byref(g), _fp(pos), pos.shape[0], _fp(st), st.shape[0], batch_size,
        particle_count, steps, float(update_prob), int(seed) & 0xFFFFFFFFFFFFFFFF, _fp(sp),
        _fp(ss), _fp(sm), _fp(fp), _fp(fs), _fp(mean)), "rollout_for_training")
    return RolloutForTraining(sp, ss, sm, fp, fs, float(mean[0]), steps, batch_size,
                              particle_count)


@dataclass
class BpttResult:
    """bptt_gradients' total plus the adjoints at the rollout's input."""

    gradients: SupervisedGradients
    position_adjoint: np.ndarray
    state_adjoint: np.ndarray


def bptt_gradients(model: NpaModel, grid: HashGridConfig, rollout: RolloutForTraining,
                   position_gradients, state_gradients,
                   displacement_regularizer_weight: float = 0.0,
                   stopgrad_pos: Optional[bool] = None,
                   stopgrad_state: Optional[bool] = None) -> BpttResult:
    """target2d.rs:3550-3722: the MLP weight gradients of the rollout given
    the loss adjoints of its final positions [B*N, 4] and states [B*N*C].
    stopgrad_pos / stopgrad_state default to the model config's."""
    cfg = model.config
    sgp = cfg.stopgrad_pos if stopgrad_pos is None else stopgrad_pos
    sgs = cfg.stopgrad_state if stopgrad_state is None else stopgrad_state
    total = rollout.batch_size * rollout.particle_count
    C = cfg.state_dims
    pg = _f32(position_gradients).reshape(-1, 4)
    sg = _f32(state_gradients).reshape(-1)
    if pg.shape[0] != total or sg.size != total * C:
        raise InvalidArgument("loss gradients do not match the rollout's particles")
    sp = _f32(rollout.snapshot_positions)
    ss = _f32(rollout.snapshot_states)
    sm = _f32(rollout.snapshot_masks)
    if (sp.size != rollout.steps * total * 4 or ss.size != rollout.steps * total * C
            or sm.size != rollout.steps * total):
        raise InvalidArgument("snapshots do not match the rollout's steps and particles")
    gw1, gb1, gw2, gb2 = _weight_buffers(model)
    pa = np.zeros((total, 4), np.float32)
    sa = np.zeros(total * C, np.float32)
    g = _lib.grid_c(grid)
    _lib.check(_lib.lib().npa_model_bptt_gradients(
        model.handle, ctypes.byref(g), _fp(sp), _fp(ss), _fp(sm), rollout.batch_size,
        rollout.particle_count, rollout.steps, _fp(pg), _fp(sg),
        float(displacement_regularizer_weight), int(bool(sgp)), int(bool(sgs)), _fp(gw1),
        _fp(gb1), _fp(gw2), _fp(gb2), _fp(pa), _fp(sa)), "bptt_gradients")
    return BpttResult(SupervisedGradients(gw1, gb1, gw2, gb2, np.zeros(0, np.float32)), pa, sa)
