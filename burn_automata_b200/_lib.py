"""ctypes binding of libnpa_b200.so (include/npa_b200.h).

The library is built in-tree by burn_automata_b200/csrc/Makefile.  Loading
fails loudly when it is missing: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

from . import config as _cfg

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libnpa_b200.so"
CSRC = PKG_DIR / "csrc"

c_i32, c_i64, c_u32, c_u64, c_f32 = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32,
                                     ctypes.c_uint64, ctypes.c_float)
P = ctypes.POINTER
f32p = P(c_f32)
u32p = P(c_u32)
vp = ctypes.c_void_p


class GridConfigC(ctypes.Structure):
    _fields_ = [("dim", c_i32), ("boundary", c_i32), ("mode", c_i32),
                ("max_particles_per_block", c_i32), ("grid_size", c_i64 * 3), ("eps", c_f32),
                ("reserved", c_i32)]


class PerceptionOptionsC(ctypes.Structure):
    _fields_ = [("state_grad", ctypes.c_uint8), ("density_grad", ctypes.c_uint8),
                ("scale_equivariance", ctypes.c_uint8),
                ("particle_density_equivariance", ctypes.c_uint8),
                ("log_norm_grad", ctypes.c_uint8), ("log_norm_density_grad", ctypes.c_uint8),
                ("hybrid_state_gradient", ctypes.c_uint8), ("position_features", ctypes.c_uint8),
                ("eps0", c_f32), ("reserved", c_i32)]


class ModelConfigC(ctypes.Structure):
    _fields_ = [("spatial_dims", c_i32), ("state_dims", c_i32), ("hidden_dims", c_i32),
                ("auxiliary_input_dims", c_i32), ("eps0", c_f32), ("alpha", c_f32),
                ("equivariance", c_i32), ("density_grad", ctypes.c_uint8),
                ("state_grad", ctypes.c_uint8), ("log_norm_grad", ctypes.c_uint8),
                ("log_norm_density_grad", ctypes.c_uint8), ("position_features", ctypes.c_uint8),
                ("reserved", ctypes.c_uint8 * 7)]


class DecodeConfigC(ctypes.Structure):
    _fields_ = [("mode", c_i32), ("sh_degree", c_i32), ("sigma", c_f32), ("min_scale", c_f32),
                ("max_scale", c_f32), ("max_anisotropy", c_f32), ("opacity_scale", c_f32),
                ("min_opacity", c_f32), ("max_opacity", c_f32), ("reserved", c_i32)]


class ErrorDetailC(ctypes.Structure):
    _fields_ = [("status", c_i32), ("eps", c_f32), ("a", c_i64), ("b", c_i64)]


class Splat2dConfigC(ctypes.Structure):
    _fields_ = [("image_size", ctypes.c_int64), ("sigma", ctypes.c_float),
                ("lo", ctypes.c_float), ("hi", ctypes.c_float),
                ("normalize_color", ctypes.c_int32), ("y_up", ctypes.c_int32),
                ("pixel_size", ctypes.c_float), ("reserved", ctypes.c_int32)]


# (name, restype, argtypes) for every entry point of include/npa_b200.h.
SIGNATURES = [
    ("npa_abi_version", c_i32, []),
    ("npa_status_string", ctypes.c_char_p, [c_i32]),
    ("npa_last_error_message", ctypes.c_char_p, []),
    ("npa_kernel_launch_count", c_u64, []),
    ("npa_bulk_copy_timeouts", c_u64, []),
    ("npa_last_error_detail", c_i32, [P(ErrorDetailC)]),
    ("npa_prepare_host_tables", c_i32, [P(c_i64)]),
    ("npa_prepare_device", c_i32, [c_i32]),
    ("npa_dev_ln_1p", c_i32, [vp, c_i64, vp, vp]),
    ("npa_grid_validate", c_i32, [P(GridConfigC)]),
    ("npa_grid_cell_count", c_i32, [P(GridConfigC), P(c_i64)]),
    ("npa_feature_dims", c_i32, [P(GridConfigC), P(PerceptionOptionsC), c_i64, P(c_i64)]),
    ("npa_gaussian_record_floats", c_i32, [P(DecodeConfigC), P(c_i64)]),
    ("npa_build_hashgrid", c_i32,
     [P(GridConfigC), f32p, c_i64, c_i64, c_i64, u32p, c_i64, u32p, u32p, c_i64]),
    ("npa_perceive_with_options", c_i32,
     [P(GridConfigC), P(PerceptionOptionsC), f32p, c_i64, f32p, c_i64, c_i64, c_i64, c_i64, f32p,
      c_i64, f32p, f32p, f32p, f32p]),
    ("npa_euler_step", c_i32,
     [P(GridConfigC), f32p, c_i64, f32p, c_i64, f32p, c_i64, f32p, c_i64, c_i64, c_i64, c_i64,
      c_f32, f32p, f32p, f32p]),
    ("npa_decode_gaussians_3d", c_i32,
     [P(DecodeConfigC), f32p, c_i64, f32p, c_i64, c_i64, f32p, c_i64]),
    ("npa_model_create", c_i32,
     [P(ModelConfigC), f32p, c_i64, f32p, c_i64, f32p, c_i64, f32p, c_i64, c_i32, P(vp)]),
    ("npa_model_destroy", None, [vp]),
    ("npa_model_forward_update_from_features", c_i32, [vp, f32p, c_i64, f32p, c_i64]),
    ("npa_model_step", c_i32,
     [vp, P(GridConfigC), f32p, c_i64, f32p, c_i64, c_i64, c_i64, c_f32, f32p, f32p, f32p, f32p,
      f32p, f32p, f32p]),
    ("npa_model_run_rollout", c_i32,
     [vp, P(GridConfigC), f32p, c_i64, f32p, c_i64, c_i64, c_i64, c_i64, c_f32]),
    ("npa_model_run_rollout_trace", c_i32,
     [vp, P(GridConfigC), f32p, c_i64, f32p, c_i64, c_i64, c_i64, c_i64, c_f32, f32p]),
    ("npa_model_run_rollout_seeded", c_i32,
     [vp, P(GridConfigC), f32p, c_i64, f32p, c_i64, c_i64, c_i64, c_i64, c_f32, c_f32,
      ctypes.c_uint64, f32p]),
    ("npa_rollout_update_masks", c_i32, [ctypes.c_uint64, c_f32, c_i64, c_i64, c_i64, f32p]),
    ("npa_model_mlp_backward", c_i32,
     [vp, f32p, c_i64, f32p, c_i64, f32p, f32p, f32p, f32p, f32p]),
    ("npa_model_rollout_for_training", c_i32,
     [vp, P(GridConfigC), f32p, c_i64, f32p, c_i64, c_i64, c_i64, c_i64, c_f32, ctypes.c_uint64,
      f32p, f32p, f32p, f32p, f32p, f32p]),
    ("npa_model_bptt_gradients", c_i32,
     [vp, P(GridConfigC), f32p, f32p, f32p, c_i64, c_i64, c_i64, f32p, f32p, c_f32, c_i32, c_i32,
      f32p, f32p, f32p, f32p, f32p, f32p]),
    ("npa_dev_hashgrid_workspace_size", c_i32, [P(GridConfigC), c_i64, c_i64, P(ctypes.c_size_t)]),
    ("npa_dev_build_hashgrid", c_i32,
     [P(GridConfigC), vp, c_i64, c_i64, vp, vp, vp, vp, ctypes.c_size_t, vp]),
    ("npa_dev_build_hashgrid_noalloc", c_i32,
     [P(GridConfigC), vp, c_i64, c_i64, vp, vp, vp, vp]),
    ("npa_perceive_adjoint_with_options", c_i32,
     [P(GridConfigC), P(PerceptionOptionsC), f32p, c_i64, f32p, c_i64, c_i64, c_i64, c_i64, f32p,
      c_i64, f32p, f32p]),
    ("npa_dev_perceive_adjoint_workspace_size", c_i32,
     [P(GridConfigC), c_i64, c_i64, c_i64, P(ctypes.c_size_t)]),
    ("npa_dev_perceive_adjoint_with_options", c_i32,
     [P(GridConfigC), P(PerceptionOptionsC), vp, vp, c_i64, c_i64, c_i64, vp, vp, vp, vp,
      ctypes.c_size_t, vp]),
    ("npa_splat_particles_2d", c_i32, [P(Splat2dConfigC), f32p, f32p, c_i64, f32p, c_i64]),
    ("npa_dev_splat_workspace_size", c_i32, [c_i64, P(ctypes.c_size_t)]),
    ("npa_dev_splat_particles_2d", c_i32,
     [P(Splat2dConfigC), vp, vp, c_i64, vp, vp, ctypes.c_size_t, vp]),
    ("npa_dev_perceive_workspace_size", c_i32,
     [P(GridConfigC), c_i64, c_i64, c_i64, P(ctypes.c_size_t)]),
    ("npa_dev_perceive_with_options", c_i32,
     [P(GridConfigC), P(PerceptionOptionsC), vp, vp, c_i64, c_i64, c_i64, vp, vp, vp, vp, vp, vp,
      ctypes.c_size_t, vp]),
    ("npa_dev_perceive_many_profiled", c_i32,
     [P(GridConfigC), P(PerceptionOptionsC), vp, vp, c_i64, c_i64, c_i64, vp, vp, vp,
      ctypes.c_size_t, c_i64, vp, f32p, f32p]),
    ("npa_dev_model_forward_update", c_i32, [vp, vp, c_i64, vp, vp]),
    ("npa_dev_euler_step", c_i32,
     [P(GridConfigC), vp, vp, vp, vp, c_i64, c_i64, c_i64, c_f32, vp, vp, vp, vp]),
    ("npa_dev_decode_gaussians_3d", c_i32, [P(DecodeConfigC), vp, vp, c_i64, c_i64, vp, vp]),
    ("npa_dev_step_workspace_size", c_i32, [vp, P(GridConfigC), c_i64, c_i64, P(ctypes.c_size_t)]),
    ("npa_dev_model_step", c_i32,
     [vp, P(GridConfigC), vp, vp, c_i64, c_i64, c_f32, vp, vp, vp, vp, vp, vp, vp, vp,
      ctypes.c_size_t, vp]),
    ("npa_executor_create", c_i32, [vp, P(GridConfigC), c_i64, c_i64, P(vp)]),
    ("npa_executor_destroy", None, [vp]),
    ("npa_executor_upload_state", c_i32, [vp, f32p, f32p]),
    ("npa_executor_set_state_device", c_i32, [vp, vp, vp, vp]),
    ("npa_executor_step_many", c_i32, [vp, c_i64, c_f32, c_i32, vp]),
    ("npa_executor_step_many_profiled", c_i32, [vp, c_i64, c_f32, c_i32, vp, f32p, f32p]),
    ("npa_executor_set_update_prob", c_i32, [vp, c_f32, c_u64, P(c_u64)]),
    ("npa_executor_set_step_index", c_i32, [vp, ctypes.c_uint32]),
    ("npa_executor_step_index", c_i32, [vp, P(ctypes.c_uint32)]),
    ("npa_executor_read_state", c_i32, [vp, f32p, f32p]),
    ("npa_executor_state_device", c_i32, [vp, P(vp), P(vp)]),
    ("npa_executor_launches_per_step", c_i32, [vp, P(c_i64)]),
    ("npa_executor_set_fused_step", c_i32, [vp, c_i32]),
    ("npa_executor_set_step_groups", c_i32, [vp, c_i32]),
    ("npa_executor_step_groups", c_i32, [vp, P(c_i32)]),
]

# Symbols exported beyond the public header (test hooks).
EXTRA_SIGNATURES = [
    ("npa_debug_set_allocation_cap", None, [c_u64]),
    ("npa_debug_fp32_tile_rate", c_i32, [c_i32, P(ctypes.c_double), P(ctypes.c_double)]),
]


def build(force: bool = False) -> Path:
    """Compile the library with the committed Makefile (nvcc, sm_100a)."""
    if force or not LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(CSRC), "-j4"], check=True)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `make -C {CSRC}` "
                "(burn_automata_b200 has no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES + EXTRA_SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, where: str = "") -> None:
    if status != 0:
        L = lib()
        msg = L.npa_last_error_message().decode(errors="replace")
        d = ErrorDetailC()
        L.npa_last_error_detail(ctypes.byref(d))
        detail = {"a": int(d.a), "b": int(d.b), "eps": float(d.eps)} if d.status == status else None
        raise _cfg.error_for(status, f"{where}: {msg}" if where else msg, detail)


def grid_c(cfg: _cfg.HashGridConfig) -> GridConfigC:
    g = GridConfigC()
    g.dim = int(cfg.dim)
    g.boundary = int(cfg.boundary)
    g.mode = int(cfg.mode)
    g.max_particles_per_block = int(cfg.max_particles_per_block)
    for i in range(3):
        g.grid_size[i] = int(cfg.grid_size[i])
    g.eps = float(cfg.eps)
    return g


def options_c(opt: _cfg.PerceptionOptions) -> PerceptionOptionsC:
    o = PerceptionOptionsC()
    for name in ("state_grad", "density_grad", "scale_equivariance",
                 "particle_density_equivariance", "log_norm_grad", "log_norm_density_grad",
                 "hybrid_state_gradient", "position_features"):
        setattr(o, name, int(bool(getattr(opt, name))))
    o.eps0 = float(opt.eps0)
    return o


def model_c(cfg: _cfg.NpaConfig) -> ModelConfigC:
    m = ModelConfigC()
    m.spatial_dims = int(cfg.spatial_dims)
    m.state_dims = int(cfg.state_dims)
    m.hidden_dims = int(cfg.hidden_dims)
    m.auxiliary_input_dims = int(cfg.auxiliary_input_dims)
    m.eps0 = float(cfg.eps0)
    m.alpha = float(cfg.alpha)
    m.equivariance = int(cfg.equivariance)
    for name in ("density_grad", "state_grad", "log_norm_grad", "log_norm_density_grad",
                 "position_features"):
        setattr(m, name, int(bool(getattr(cfg, name))))
    return m


def decode_c(cfg: _cfg.GaussianDecodeConfig) -> DecodeConfigC:
    d = DecodeConfigC()
    d.mode = int(cfg.mode)
    d.sh_degree = int(cfg.sh_degree)
    for name in ("sigma", "min_scale", "max_scale", "max_anisotropy", "opacity_scale",
                 "min_opacity", "max_opacity"):
        setattr(d, name, float(getattr(cfg, name)))
    return d
