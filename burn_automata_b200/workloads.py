"""Seeded synthetic inputs for the five benchmark configurations.

No public dataset is involved: every config is a seeded draw with the shapes
and value distributions the configuration names.  Seeds: positions use
numpy PCG64(seed), states PCG64(seed + 1), weights PCG64(seed + 2).

cfg0  2D fixed NPA, 4,096 particles, 64 steps, C=16, MLP 64->128->18
cfg1  hashgrid + perception microbench, 1,048,576 particles, C=32, eps 0.004
cfg2  256 independent cfg0 rollouts x 128 steps, one shared MLP
cfg3  3D torus (R=0.6, r=0.25), 16,384 particles, C=32, MLP 160->256->35
cfg4  Gaussian-mixture 2D cluster, 4,194,304 particles, C=16, cfg0 MLP

Model weights are Kaiming-normal (std = sqrt(2 / fan_in)) with zero biases.
The reference's own initialisers (uniform / Xavier, model.rs:29-63) draw from
Rust's StdRng through rand's distributions, with no golden values to check a
restatement against; the weights are an input, identical for the oracle and
the GPU.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from .config import (GaussianDecodeConfig, GaussianDecodeMode, HashGridConfig, HashGridMode,
                     Boundary, NpaConfig, PerceptionOptions)


@dataclass
class NpaWeightsHost:
    """NpaWeights (model.rs:11-17) as host arrays: w1 [H, F], b1 [H], w2 [O, H], b2 [O]."""

    w1: np.ndarray
    b1: np.ndarray
    w2: np.ndarray
    b2: np.ndarray


@dataclass
class Workload:
    name: str
    batch: int
    n: int
    steps: int
    dt: float
    grid: HashGridConfig
    model: Optional[NpaConfig]
    options: PerceptionOptions
    decode: Optional[GaussianDecodeConfig]
    positions: np.ndarray  # [B*N, 4] f32
    states: np.ndarray  # [B*N*C] f32
    weights: Optional[NpaWeightsHost] = None
    state_dims: int = 16
    notes: dict = field(default_factory=dict)


def kaiming_weights(cfg: NpaConfig, seed: int) -> NpaWeightsHost:
    rng = np.random.Generator(np.random.PCG64(seed))
    f, h, o = cfg.perception_dims(), cfg.hidden_dims, cfg.update_dims()
    w1 = (rng.standard_normal((h, f)) * np.sqrt(2.0 / f)).astype(np.float32)
    w2 = (rng.standard_normal((o, h)) * np.sqrt(2.0 / h)).astype(np.float32)
    return NpaWeightsHost(w1.reshape(-1), np.zeros(h, np.float32), w2.reshape(-1),
                          np.zeros(o, np.float32))


def uniform_positions_2d(count: int, seed: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    pos = np.zeros((count, 4), np.float32)
    pos[:, :2] = rng.uniform(lo, hi, size=(count, 2)).astype(np.float32)
    return pos


def normal_states(count: int, c: int, std: float, seed: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.standard_normal(count * c) * std).astype(np.float32)


def torus_positions(count: int, seed: int, major: float = 0.6, minor: float = 0.25) -> np.ndarray:
    """Area-uniform samples on a torus: uniform major angle, tube angle by rejection
    with acceptance (R + r cos(phi)) / (R + r)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = np.zeros((count, 4), np.float32)
    filled = 0
    while filled < count:
        m = (count - filled) * 2 + 64
        theta = rng.uniform(0.0, 2.0 * np.pi, m)
        phi = rng.uniform(0.0, 2.0 * np.pi, m)
        keep = rng.uniform(0.0, 1.0, m) < (major + minor * np.cos(phi)) / (major + minor)
        theta, phi = theta[keep], phi[keep]
        take = min(count - filled, theta.shape[0])
        theta, phi = theta[:take], phi[:take]
        ring = major + minor * np.cos(phi)
        out[filled:filled + take, 0] = (ring * np.cos(theta)).astype(np.float32)
        out[filled:filled + take, 1] = (ring * np.sin(theta)).astype(np.float32)
        out[filled:filled + take, 2] = (minor * np.sin(phi)).astype(np.float32)
        filled += take
    return out


def mixture_positions_2d(count: int, seed: int, components: int = 64,
                         sigma: float = 0.02) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    centres = rng.uniform(-1.0, 1.0, size=(components, 2))
    which = rng.integers(0, components, size=count)
    pos = np.zeros((count, 4), np.float32)
    pos[:, :2] = (centres[which] + rng.standard_normal((count, 2)) * sigma).astype(np.float32)
    return pos


def cfg0_model() -> NpaConfig:
    """growing_2d (config.rs:56) with density_grad off: F = 2C + C*D = 64."""
    return NpaConfig.growing_2d().with_(density_grad=False)


def cfg0_grid(eps: float = 0.05) -> HashGridConfig:
    return HashGridConfig.growing_2d().with_(eps=eps, grid_size=(64, 64, 1))


def learned_scale_decode() -> GaussianDecodeConfig:
    return GaussianDecodeConfig(mode=GaussianDecodeMode.GaussianSh0LearnedScale)


def make(name: str, seed: int = 0, *, batch: Optional[int] = None, n: Optional[int] = None,
         steps: Optional[int] = None, first: int = 0,
         components: Optional[int] = None) -> Workload:
    """Build one configuration.  batch / n / steps override the sizes for
    reduced parity cases; everything else stays as the configuration names it.
    `first` is the global index of the first rollout, so a shard of a batched
    configuration draws exactly the rollouts the full batch would.
    `components` (cfg4 only) sets the number of mixture components; 1 with
    n = 65,536 is one component of the full draw at its particle density."""
    if name == "cfg0":
        b = batch or 1
        n_ = n or 4096
        model = cfg0_model()
        grid = cfg0_grid()
        pos = np.concatenate([uniform_positions_2d(n_, seed + 1000 * (first + k)) for k in range(b)])
        st = np.concatenate([normal_states(n_, 16, 0.1, seed + 1 + 1000 * (first + k)) for k in range(b)])
        return Workload("cfg0", b, n_, steps or 64, 0.1, grid, model, model.perception_options(),
                        learned_scale_decode(), pos, st, kaiming_weights(model, seed + 2), 16)
    if name == "cfg1":
        b = batch or 1
        n_ = n or (1 << 20)
        grid = HashGridConfig.growing_2d().with_(eps=0.004, grid_size=(512, 512, 1))
        opt = NpaConfig.growing_2d().perception_options()
        pos = np.concatenate([uniform_positions_2d(n_, seed + 1000 * (first + k)) for k in range(b)])
        st = np.concatenate([normal_states(n_, 32, 1.0, seed + 1 + 1000 * (first + k)) for k in range(b)])
        return Workload("cfg1", b, n_, steps or 1, 0.1, grid, None, opt, None, pos, st, None, 32)
    if name == "cfg2":
        b = batch or 256
        n_ = n or 4096
        model = cfg0_model()
        grid = cfg0_grid()
        pos = np.concatenate([uniform_positions_2d(n_, seed + 1000 * (first + k)) for k in range(b)])
        st = np.concatenate([normal_states(n_, 16, 0.1, seed + 1 + 1000 * (first + k)) for k in range(b)])
        return Workload("cfg2", b, n_, steps or 128, 0.1, grid, model, model.perception_options(),
                        learned_scale_decode(), pos, st, kaiming_weights(model, seed + 2), 16)
    if name == "cfg3":
        b = batch or 1
        n_ = n or 16384
        model = NpaConfig.growing_3dgs().with_(state_dims=32, hidden_dims=256, density_grad=False,
                                               decoder_dims=None, output_dims=None)
        grid = HashGridConfig.growing_3dgs().with_(eps=0.06, grid_size=(32, 32, 32))
        pos = np.concatenate([torus_positions(n_, seed + 1000 * (first + k)) for k in range(b)])
        st = np.concatenate([normal_states(n_, 32, 0.1, seed + 1 + 1000 * (first + k)) for k in range(b)])
        dec = GaussianDecodeConfig(mode=GaussianDecodeMode.GaussianSh0Oriented, sh_degree=0)
        return Workload("cfg3", b, n_, steps or 256, 0.1, grid, model, model.perception_options(),
                        dec, pos, st, kaiming_weights(model, seed + 2), 32)
    if name == "cfg4":
        b = batch or 1
        n_ = n or (1 << 22)
        model = cfg0_model()
        grid = cfg0_grid()
        comp = components or 64
        pos = np.concatenate([mixture_positions_2d(n_, seed + 1000 * (first + k), comp)
                              for k in range(b)])
        st = np.concatenate([normal_states(n_, 16, 0.1, seed + 1 + 1000 * (first + k)) for k in range(b)])
        return Workload("cfg4", b, n_, steps or 32, 0.1, grid, model, model.perception_options(),
                        learned_scale_decode(), pos, st, kaiming_weights(model, seed + 2), 16)
    raise ValueError(f"unknown workload {name!r}")
