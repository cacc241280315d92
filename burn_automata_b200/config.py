"""Host-side mirror of the reference's configuration types.

Mirrors, field for field:
  HashGridConfig / Boundary / HashGridMode   crates/burn_automata_kernels/src/config.rs:4-99
  KernelError                                crates/burn_automata_kernels/src/config.rs:101-139
  PerceptionOptions                          crates/burn_automata_kernels/src/reference/types.rs:4-31
  NpaConfig / EquivarianceMode               crates/burn_automata/src/config.rs:22-205
  GaussianDecodeConfig / GaussianDecodeMode  crates/burn_automata_kernels/src/gaussian.rs:13-51

Validation raises the same error kinds, in the same order, as the reference.
"""

from __future__ import annotations

import enum
import math
from dataclasses import dataclass, field, replace
from typing import Tuple


class Boundary(enum.IntEnum):
    Periodic = 0
    Clamped = 1


class HashGridMode(enum.IntEnum):
    Grid = 0
    Particle = 1


class EquivarianceMode(enum.IntEnum):
    NoEquivariance = 0
    ParticleDensity = 1
    ParticleDensityAndScale = 2


class GaussianDecodeMode(enum.IntEnum):
    ParticlePoint = 0
    GaussianSh0FixedScale = 1
    GaussianSh0LearnedScale = 2
    GaussianSh0Oriented = 3


# Status codes of the C ABI (include/npa_b200.h); 1..9 map 1:1 onto KernelError /
# AutomataError variants of the reference.
STATUS_NAMES = {
    0: "Ok",
    1: "InvalidDim",
    2: "InvalidEps",
    3: "InvalidGridSize",
    4: "ParticleModeRequiresPowerOfTwo",
    5: "PositionShape",
    6: "StateShape",
    7: "OutputShape",
    8: "InvalidArgument",
    9: "InvalidModel",
    20: "Cuda",
    21: "DeviceStatus",
    22: "Timeout",
    23: "OutOfMemory",
    24: "Unsupported",
    25: "NoDevice",
}


class KernelError(Exception):
    """Base of the reference's KernelError / AutomataError variants."""

    code = -1

    def __init__(self, message: str = "", code: int | None = None):
        super().__init__(message)
        if code is not None:
            self.code = code


def _make_error(name: str, code: int):
    return type(name, (KernelError,), {"code": code})


InvalidDim = _make_error("InvalidDim", 1)
InvalidEps = _make_error("InvalidEps", 2)
InvalidGridSize = _make_error("InvalidGridSize", 3)
ParticleModeRequiresPowerOfTwo = _make_error("ParticleModeRequiresPowerOfTwo", 4)
PositionShape = _make_error("PositionShape", 5)
StateShape = _make_error("StateShape", 6)
OutputShape = _make_error("OutputShape", 7)
InvalidArgument = _make_error("InvalidArgument", 8)
InvalidModel = _make_error("InvalidModel", 9)
CudaError = _make_error("CudaError", 20)
DeviceStatusError = _make_error("DeviceStatusError", 21)
TimeoutError_ = _make_error("DeviceTimeout", 22)
OutOfMemory = _make_error("OutOfMemory", 23)
Unsupported = _make_error("Unsupported", 24)
NoDevice = _make_error("NoDevice", 25)

ERRORS_BY_CODE = {
    cls.code: cls
    for cls in (InvalidDim, InvalidEps, InvalidGridSize, ParticleModeRequiresPowerOfTwo,
                PositionShape, StateShape, OutputShape, InvalidArgument, InvalidModel, CudaError,
                DeviceStatusError, TimeoutError_, OutOfMemory, Unsupported, NoDevice)
}


# The fields each KernelError variant carries (config.rs:102-137), filled from
# the C ABI's npa_last_error_detail: (attribute, source) pairs.
PAYLOAD_FIELDS = {
    1: (("dim", "a"),),
    2: (("eps", "eps"),),
    4: (("axis", "a"), ("value", "b")),
    5: (("positions", "a"), ("expected", "b")),
    6: (("states", "a"), ("expected", "b")),
    7: (("actual", "a"), ("expected", "b")),
}


def error_for(code: int, message: str = "", detail=None) -> KernelError:
    """The exception for a status code; `detail` (a = ..., b = ..., eps = ...)
    becomes the variant's fields, e.g. OutputShape.actual / .expected."""
    cls = ERRORS_BY_CODE.get(int(code), KernelError)
    err = cls(message or STATUS_NAMES.get(int(code), f"status {code}"), int(code))
    if detail is not None:
        for attr, src in PAYLOAD_FIELDS.get(int(code), ()):
            setattr(err, attr, detail[src])
    return err


@dataclass
class HashGridConfig:
    """config.rs:20-29."""

    dim: int = 2
    boundary: Boundary = Boundary.Clamped
    mode: HashGridMode = HashGridMode.Particle
    grid_size: Tuple[int, int, int] = (64, 64, 1)
    eps: float = 0.1
    max_particles_per_block: int = 32

    @staticmethod
    def growing_2d() -> "HashGridConfig":
        return HashGridConfig(2, Boundary.Clamped, HashGridMode.Particle, (64, 64, 1), 0.1, 32)

    @staticmethod
    def texture_2d() -> "HashGridConfig":
        return HashGridConfig(2, Boundary.Periodic, HashGridMode.Grid, (10, 10, 1), 0.2, 32)

    @staticmethod
    def growing_3dgs() -> "HashGridConfig":
        return HashGridConfig(3, Boundary.Clamped, HashGridMode.Particle, (32, 32, 32), 0.1, 64)

    def with_(self, **kw) -> "HashGridConfig":
        return replace(self, **kw)

    def validate(self) -> None:
        """config.rs:65-84."""
        if self.dim not in (2, 3):
            raise InvalidDim(f"expected spatial dim 2 or 3, got {self.dim}")
        eps32 = float(_f32(self.eps))
        if not math.isfinite(eps32) or eps32 <= 0.0:
            raise InvalidEps(f"eps must be finite and positive, got {self.eps}")
        for axis in range(self.dim):
            size = int(self.grid_size[axis])
            if size == 0:
                raise InvalidGridSize("grid sizes must be non-zero for active dimensions")
            if self.mode == HashGridMode.Particle and (size & (size - 1)) != 0:
                raise ParticleModeRequiresPowerOfTwo(
                    f"particle hashgrid mode requires power-of-two grid size at axis {axis}, "
                    f"got {size}")

    def cell_count(self) -> int:
        c = 1
        for axis in range(self.dim):
            c *= int(self.grid_size[axis])
        return c

    def spatial_mem_dims(self) -> int:
        return 4 if self.dim == 3 else 2


@dataclass
class PerceptionOptions:
    """reference/types.rs:4-31 (PerceptionOptions::new defaults)."""

    state_grad: bool = True
    density_grad: bool = True
    eps0: float = 0.1
    scale_equivariance: bool = True
    particle_density_equivariance: bool = True
    log_norm_grad: bool = False
    log_norm_density_grad: bool = False
    hybrid_state_gradient: bool = True
    position_features: bool = False

    @staticmethod
    def new(state_grad: bool, density_grad: bool, eps0: float) -> "PerceptionOptions":
        return PerceptionOptions(state_grad, density_grad, eps0)


def feature_dims(cfg: HashGridConfig, opt: PerceptionOptions, state_dims: int) -> int:
    """forward.rs:100-103."""
    return (state_dims * 2 + int(opt.state_grad) * state_dims * cfg.dim
            + int(opt.density_grad) * cfg.dim + int(opt.position_features) * cfg.dim)


@dataclass
class NpaConfig:
    """burn_automata/src/config.rs:30-53 (decoder_dims / output_dims are not read by the step)."""

    spatial_dims: int = 2
    state_dims: int = 16
    hidden_dims: int = 128
    eps0: float = 0.1
    alpha: float = 0.5
    density_grad: bool = True
    state_grad: bool = True
    log_norm_grad: bool = True
    log_norm_density_grad: bool = True
    stopgrad_pos: bool = True
    stopgrad_state: bool = False
    equivariance: EquivarianceMode = EquivarianceMode.ParticleDensityAndScale
    position_features: bool = False
    auxiliary_input_dims: int = 0
    decoder_dims: int | None = None
    output_dims: int | None = None

    @staticmethod
    def growing_2d() -> "NpaConfig":
        return NpaConfig()

    @staticmethod
    def texture_2d() -> "NpaConfig":
        return NpaConfig(eps0=0.2)

    @staticmethod
    def growing_3dgs() -> "NpaConfig":
        return NpaConfig(spatial_dims=3, state_dims=24, hidden_dims=256, eps0=0.1, alpha=1.0,
                         decoder_dims=256, output_dims=20)

    @staticmethod
    def point_mnist() -> "NpaConfig":
        return NpaConfig(hidden_dims=256, alpha=1.0, decoder_dims=256, output_dims=10)

    @staticmethod
    def torus_field_3dgs() -> "NpaConfig":
        return replace(NpaConfig.growing_3dgs(), position_features=True)

    def with_(self, **kw) -> "NpaConfig":
        return replace(self, **kw)

    def perception_dims(self) -> int:
        return (self.state_dims * 2 + int(self.state_grad) * self.state_dims * self.spatial_dims
                + int(self.density_grad) * self.spatial_dims
                + int(self.position_features) * self.spatial_dims + self.auxiliary_input_dims)

    def update_dims(self) -> int:
        return self.spatial_dims + self.state_dims

    def scale_equivariant(self) -> bool:
        return self.equivariance == EquivarianceMode.ParticleDensityAndScale

    def particle_density_equivariant(self) -> bool:
        return self.equivariance in (EquivarianceMode.ParticleDensity,
                                     EquivarianceMode.ParticleDensityAndScale)

    def motion_eps(self, grid_eps: float) -> float:
        return grid_eps if self.scale_equivariant() else self.eps0

    def perception_options(self) -> PerceptionOptions:
        """The options step_cpu passes to perceive_with_options (model.rs:785-801)."""
        return PerceptionOptions(
            state_grad=self.state_grad,
            density_grad=self.density_grad,
            eps0=self.eps0,
            scale_equivariance=self.scale_equivariant(),
            particle_density_equivariance=self.particle_density_equivariant(),
            log_norm_grad=self.log_norm_grad,
            log_norm_density_grad=self.log_norm_density_grad,
            hybrid_state_gradient=True,
            position_features=self.position_features,
        )


@dataclass
class GaussianDecodeConfig:
    """gaussian.rs:23-51."""

    mode: GaussianDecodeMode = GaussianDecodeMode.GaussianSh0FixedScale
    sigma: float = 0.02
    min_scale: float = 0.001
    max_scale: float = 0.08
    max_anisotropy: float = 0.1
    opacity_scale: float = 0.15
    min_opacity: float = 0.001
    max_opacity: float = 0.95
    sh_degree: int = 0

    def with_(self, **kw) -> "GaussianDecodeConfig":
        return replace(self, **kw)

    def sh_coeffs(self) -> int:
        if self.mode == GaussianDecodeMode.GaussianSh0Oriented:
            return (self.sh_degree + 1) ** 2
        return 1

    def record_floats(self) -> int:
        """Floats per decoded Gaussian in the C ABI record:
        [position_visibility 4][rotation 4][scale_opacity 4][sh 3*k]."""
        return 12 + 3 * self.sh_coeffs()


def _f32(x: float):
    import numpy as np

    return np.float32(x)


@dataclass
class Splat2dConfig:
    """splat.rs:4-28 (defaults as Splat2dConfig::default)."""

    image_size: int = 128
    sigma: float = 1.0
    lo: float = -1.0
    hi: float = 1.0
    normalize_color: bool = True
    y_up: bool = True
    pixel_size: float = 2.0 / 128.0

    def with_(self, **kw) -> "Splat2dConfig":
        return replace(self, **kw)
