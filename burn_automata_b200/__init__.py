"""B200-native (sm_100a) implementation of the burn_automata NPA rollout path.

The CUDA kernels and the C ABI live in csrc/ and build into libnpa_b200.so;
this package is the Python mirror of the reference's operator surface
(crates/burn_automata_kernels and NpaModel / run_rollout of crates/burn_automata).
"""

from .config import (Boundary, EquivarianceMode, GaussianDecodeConfig, GaussianDecodeMode,
                     HashGridConfig, HashGridMode, KernelError, NpaConfig, PerceptionOptions,
                     Splat2dConfig,
                     feature_dims)
from .kernels import (DevicePerception, Gaussian3d, HashGridSnapshot, PerceptionOutput, build_hashgrid,
                      decode_gaussians_3d, decode_gaussians_3d_records, euler_step, perceive,
                      perceive_adjoint_with_options, perceive_state_adjoint_with_options,
                      perceive_with_options, splat_particles_2d)
from .model import (CudaAutomataExecutor, NpaModel, NpaWeights, RolloutConfig, RolloutTrace,
                    StepOutput, rollout_update_masks, run_rollout_from_particles)
from . import bpk
from ._lib import build as build_library, lib as load_library

__all__ = [
    "Boundary", "EquivarianceMode", "GaussianDecodeConfig", "GaussianDecodeMode",
    "HashGridConfig", "HashGridMode", "KernelError", "NpaConfig", "PerceptionOptions",
    "feature_dims", "Gaussian3d", "HashGridSnapshot", "PerceptionOutput", "build_hashgrid",
    "decode_gaussians_3d", "decode_gaussians_3d_records", "euler_step", "perceive",
    "perceive_with_options", "CudaAutomataExecutor", "NpaModel", "NpaWeights", "RolloutConfig",
    "RolloutTrace", "StepOutput", "rollout_update_masks", "run_rollout_from_particles",
    "build_library", "load_library",
]
