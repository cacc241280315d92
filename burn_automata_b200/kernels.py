"""Operator surface of crates/burn_automata_kernels, backed by the CUDA library.

Same names, argument meaning and error behaviour as the reference:
  build_hashgrid         hashgrid.rs:16
  perceive               reference/forward.rs:4
  perceive_with_options  reference/forward.rs:26
  euler_step             reference/step.rs:4
  decode_gaussians_3d    gaussian.rs:53
Host numpy arrays go through the host-buffer C entry points (copy in, compute
on the GPU, copy out); torch CUDA tensors go through the npa_dev_* entry
points on the current torch stream.  Errors raise the KernelError subclass
matching the reference's variant.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from . import _lib
from .config import (GaussianDecodeConfig, GaussianDecodeMode, HashGridConfig, InvalidArgument,
                     PerceptionOptions, feature_dims)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _fp(a):
    return None if a is None else a.ctypes.data_as(_lib.f32p)


def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch") and hasattr(x, "is_cuda")


@dataclass
class HashGridSnapshot:
    """hashgrid.rs:3-14."""

    batch_size: int
    particle_count: int
    cell_count: int
    bin_offsets: np.ndarray
    permutation: np.ndarray
    inverse_permutation: np.ndarray


@dataclass
class PerceptionOutput:
    """reference/types.rs:33-41."""

    features: np.ndarray
    density: np.ndarray
    blurred_state: np.ndarray
    state_gradient: np.ndarray
    density_gradient: np.ndarray
    feature_dims: int


@dataclass
class Gaussian3d:
    """gaussian.rs:4-11."""

    position_visibility: List[float]
    spherical_harmonic: List[List[float]]
    rotation: List[float]
    scale_opacity: List[float]


def build_hashgrid(positions, batch_size: int, particle_count: int,
                   cfg: HashGridConfig) -> HashGridSnapshot:
    pos = _f32(positions).reshape(-1, 4) if np.size(positions) else np.zeros((0, 4), np.float32)
    L = _lib.lib()
    g = _lib.grid_c(cfg)
    cells = ctypes.c_int64(0)
    _lib.check(L.npa_grid_cell_count(ctypes.byref(g), ctypes.byref(cells)), "build_hashgrid")
    total = batch_size * particle_count
    offsets = np.zeros(batch_size * cells.value + 1, np.uint32)
    perm = np.zeros(max(total, 0), np.uint32)
    inv = np.zeros(max(total, 0), np.uint32)
    _lib.check(L.npa_build_hashgrid(ctypes.byref(g), _fp(pos), pos.shape[0], batch_size,
                                    particle_count, offsets.ctypes.data_as(_lib.u32p),
                                    offsets.shape[0], perm.ctypes.data_as(_lib.u32p),
                                    inv.ctypes.data_as(_lib.u32p), perm.shape[0]),
               "build_hashgrid")
    return HashGridSnapshot(batch_size, particle_count, cells.value, offsets, perm, inv)


def perceive_with_options(positions, states, batch_size: int, particle_count: int,
                          state_dims: int, cfg: HashGridConfig, options: PerceptionOptions,
                          outputs=("blurred_state", "state_gradient", "density_gradient"),
                          out=None) -> PerceptionOutput:
    """perceive_with_options (forward.rs:26-143).  Host arrays are copied to
    the GPU and back; torch CUDA tensors stay on the device.  Host calls may
    skip the intermediate outputs (`outputs`) and reuse caller-owned float32
    arrays for (features, density) via `out`."""
    if _is_torch(positions):
        return _perceive_device(positions, states, batch_size, particle_count, state_dims, cfg,
                                options)
    pos = _f32(positions).reshape(-1, 4) if np.size(positions) else np.zeros((0, 4), np.float32)
    st = _f32(states).reshape(-1)
    total = batch_size * particle_count
    fd = feature_dims(cfg, options, state_dims) if cfg.dim in (2, 3) else 0
    if out is not None:
        feats, dens = out
        if (feats.dtype != np.float32 or dens.dtype != np.float32
                or not feats.flags.c_contiguous or not dens.flags.c_contiguous
                or feats.size != max(total * fd, 0) or dens.size != max(total, 0)):
            raise InvalidArgument("out buffers must be contiguous float32 of the output's size")
    else:
        feats = np.zeros(max(total * fd, 0), np.float32)
        dens = np.zeros(max(total, 0), np.float32)
    want = set(outputs or ())
    blur = np.zeros(max(total * state_dims, 0), np.float32) if "blurred_state" in want else None
    sgrad = (np.zeros(max(total * state_dims * cfg.dim, 0) if options.state_grad else 0,
                      np.float32) if "state_gradient" in want else None)
    dgrad = (np.zeros(max(total * cfg.dim, 0) if options.density_grad else 0, np.float32)
             if "density_gradient" in want else None)
    L = _lib.lib()
    g, o = _lib.grid_c(cfg), _lib.options_c(options)
    _lib.check(L.npa_perceive_with_options(
        ctypes.byref(g), ctypes.byref(o), _fp(pos), pos.shape[0], _fp(st), st.shape[0],
        batch_size, particle_count, state_dims, _fp(feats), feats.shape[0], _fp(dens),
        _fp(blur), _fp(sgrad) if options.state_grad else None,
        _fp(dgrad) if options.density_grad else None), "perceive_with_options")
    return PerceptionOutput(feats, dens, blur, sgrad, dgrad, fd)


class DevicePerception:
    """Repeated perceive_with_options over one particle set's shape on the
    device: the workspace and the feature / density outputs are allocated
    once and reused (the hashgrid + perception pass of a caller that keeps
    its particles in GPU memory)."""

    def __init__(self, cfg: HashGridConfig, options: PerceptionOptions, batch: int, n: int,
                 state_dims: int, device=None):
        import torch

        self.cfg, self.options = cfg, options
        self.batch, self.n, self.state_dims = batch, n, state_dims
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else device)
        self.feature_dims = feature_dims(cfg, options, state_dims)
        self._g, self._o = _lib.grid_c(cfg), _lib.options_c(options)
        ws = ctypes.c_size_t(0)
        _lib.check(_lib.lib().npa_dev_perceive_workspace_size(
            ctypes.byref(self._g), batch, n, state_dims, ctypes.byref(ws)), "perceive")
        self._ws_bytes = ws.value
        total = batch * n
        self.workspace = torch.empty(max(ws.value, 1), dtype=torch.uint8, device=self.device)
        self.features = torch.empty(max(total * self.feature_dims, 1), dtype=torch.float32,
                                    device=self.device)
        self.density = torch.empty(max(total, 1), dtype=torch.float32, device=self.device)

    def _stream(self, stream):
        import torch

        return stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream

    def __call__(self, positions, states, stream=None):
        """Features and density of device tensors positions [B*N, 4], states [B*N*C]."""
        _lib.check(_lib.lib().npa_dev_perceive_with_options(
            ctypes.byref(self._g), ctypes.byref(self._o), positions.data_ptr(),
            states.data_ptr(), self.batch, self.n, self.state_dims, self.features.data_ptr(),
            self.density.data_ptr(), None, None, None, self.workspace.data_ptr(),
            self._ws_bytes, self._stream(stream)), "perceive")
        return self.features, self.density

    def run_profiled(self, positions, states, repeats: int, stream=None):
        """`repeats` back-to-back passes with CUDA events between phases:
        (phase_ms [repeats, 3] = hashgrid, density, perception; total_ms)."""
        phase = np.zeros(max(repeats, 1) * 3, np.float32)
        total = ctypes.c_float(0.0)
        _lib.check(_lib.lib().npa_dev_perceive_many_profiled(
            ctypes.byref(self._g), ctypes.byref(self._o), positions.data_ptr(),
            states.data_ptr(), self.batch, self.n, self.state_dims, self.features.data_ptr(),
            self.density.data_ptr(), self.workspace.data_ptr(), self._ws_bytes, repeats,
            self._stream(stream), phase.ctypes.data_as(_lib.f32p), ctypes.byref(total)),
            "perceive_many_profiled")
        return phase[:repeats * 3].reshape(repeats, 3), float(total.value)


def perceive(positions, states, batch_size, particle_count, state_dims, cfg, state_grad: bool,
             density_grad: bool) -> PerceptionOutput:
    return perceive_with_options(positions, states, batch_size, particle_count, state_dims, cfg,
                                 PerceptionOptions.new(state_grad, density_grad, cfg.eps))


def _perceive_device(positions, states, batch, n, c, cfg, options) -> PerceptionOutput:
    import torch

    dev = positions.device
    total = batch * n
    fd = feature_dims(cfg, options, c)
    L = _lib.lib()
    g, o = _lib.grid_c(cfg), _lib.options_c(options)
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(L.npa_dev_perceive_workspace_size(ctypes.byref(g), batch, n, c,
                                                 ctypes.byref(ws_bytes)), "perceive")
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=dev)
    feats = torch.empty(total * fd, dtype=torch.float32, device=dev)
    dens = torch.empty(total, dtype=torch.float32, device=dev)
    blur = torch.empty(total * c, dtype=torch.float32, device=dev)
    sgrad = torch.empty(total * c * cfg.dim if options.state_grad else 0, dtype=torch.float32,
                        device=dev)
    dgrad = torch.empty(total * cfg.dim if options.density_grad else 0, dtype=torch.float32,
                        device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.npa_dev_perceive_with_options(
        ctypes.byref(g), ctypes.byref(o), positions.data_ptr(), states.data_ptr(), batch, n, c,
        feats.data_ptr(), dens.data_ptr(), blur.data_ptr(),
        sgrad.data_ptr() if options.state_grad else None,
        dgrad.data_ptr() if options.density_grad else None, ws.data_ptr(), ws_bytes.value,
        stream), "perceive")
    return PerceptionOutput(feats, dens, blur, sgrad, dgrad, fd)


def euler_step(positions, states, dx, ds, batch_size: int, particle_count: int, state_dims: int,
               cfg: HashGridConfig, dt: float, update_mask=None):
    pos = _f32(positions).reshape(-1, 4) if np.size(positions) else np.zeros((0, 4), np.float32)
    st = _f32(states).reshape(-1)
    dxa = _f32(dx).reshape(-1, 4) if np.size(dx) else np.zeros((0, 4), np.float32)
    dsa = _f32(ds).reshape(-1)
    mask = _f32(update_mask).reshape(-1) if update_mask is not None else None
    npos = np.zeros_like(pos)
    nst = np.zeros_like(st)
    L = _lib.lib()
    g = _lib.grid_c(cfg)
    _lib.check(L.npa_euler_step(ctypes.byref(g), _fp(pos), pos.shape[0], _fp(st), st.shape[0],
                                _fp(dxa), dxa.shape[0], _fp(dsa), dsa.shape[0], batch_size,
                                particle_count, state_dims, float(dt), _fp(mask), _fp(npos),
                                _fp(nst)), "euler_step")
    return npos, nst


def decode_gaussians_3d_records(positions, states, state_dims: int,
                                cfg: GaussianDecodeConfig) -> np.ndarray:
    """Decoded Gaussians as the C ABI's flat records [count, 12 + 3k]:
    [position_visibility 4][rotation 4][scale_opacity 4][spherical_harmonic 3k]."""
    pos = _f32(positions).reshape(-1, 4) if np.size(positions) else np.zeros((0, 4), np.float32)
    st = _f32(states).reshape(-1)
    rec = cfg.record_floats()
    out = np.zeros(pos.shape[0] * rec, np.float32)
    L = _lib.lib()
    d = _lib.decode_c(cfg)
    _lib.check(L.npa_decode_gaussians_3d(ctypes.byref(d), _fp(pos), pos.shape[0], _fp(st),
                                         st.shape[0], state_dims, _fp(out), out.shape[0]),
               "decode_gaussians_3d")
    return out.reshape(pos.shape[0], rec)


def decode_gaussians_3d(positions, states, state_dims: int,
                        cfg: GaussianDecodeConfig) -> List[Gaussian3d]:
    recs = decode_gaussians_3d_records(positions, states, state_dims, cfg)
    k = cfg.sh_coeffs()
    out = []
    for r in recs:
        sh = [list(map(float, r[12 + 3 * q:15 + 3 * q])) for q in range(k)]
        out.append(Gaussian3d(list(map(float, r[0:4])), sh, list(map(float, r[4:8])),
                              list(map(float, r[8:12]))))
    return out


def splat_particles_2d(positions, colors, cfg) -> np.ndarray:
    """splat_particles_2d (crates/burn_automata_kernels/src/splat.rs:30-93):
    [image_size * image_size, 4] (RGB + weight).  Host arrays go through the
    host entry point; torch CUDA tensors stay on the device (a tensor result)."""
    c = _lib.Splat2dConfigC(int(cfg.image_size), float(cfg.sigma), float(cfg.lo), float(cfg.hi),
                            1 if cfg.normalize_color else 0, 1 if cfg.y_up else 0,
                            float(cfg.pixel_size), 0)
    size = int(cfg.image_size)
    if _is_torch(positions):
        import torch

        count = positions.numel() // 4
        if colors.numel() != count * 3:
            raise InvalidArgument("colors must hold 3 values per particle")
        ws_bytes = ctypes.c_size_t(0)
        _lib.check(_lib.lib().npa_dev_splat_workspace_size(count, ctypes.byref(ws_bytes)),
                   "splat")
        ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=positions.device)
        out = torch.empty((max(size * size, 1), 4), dtype=torch.float32, device=positions.device)
        stream = torch.cuda.current_stream(positions.device).cuda_stream
        _lib.check(_lib.lib().npa_dev_splat_particles_2d(
            ctypes.byref(c), positions.data_ptr(), colors.data_ptr(), count, out.data_ptr(),
            ws.data_ptr(), ws_bytes.value, stream), "splat")
        return out[:size * size]
    pos = _f32(positions).reshape(-1, 4) if np.size(positions) else np.zeros((0, 4), np.float32)
    col = _f32(colors).reshape(-1)
    if col.size != pos.shape[0] * 3:  # assert_eq!(positions.len(), colors.len())
        raise InvalidArgument(f"{pos.shape[0]} positions but {col.size // 3} colors")
    out = np.zeros((size * size, 4), np.float32)
    _lib.check(_lib.lib().npa_splat_particles_2d(ctypes.byref(c), _fp(pos), _fp(col),
                                                 pos.shape[0], _fp(out), out.size), "splat")
    return out


@dataclass
class PerceptionAdjointOutput:
    """types.rs:44-47."""

    state: np.ndarray     # [B*N*C]
    position: np.ndarray  # [B*N, 4]


def perceive_adjoint_with_options(positions, states, batch_size: int, particle_count: int,
                                  state_dims: int, cfg: HashGridConfig,
                                  options: PerceptionOptions,
                                  feature_adjoint) -> PerceptionAdjointOutput:
    """perceive_adjoint_with_options (reference/adjoint.rs:28-136) on the GPU."""
    pos = _f32(positions).reshape(-1, 4) if np.size(positions) else np.zeros((0, 4), np.float32)
    st = _f32(states).reshape(-1)
    fa = _f32(feature_adjoint).reshape(-1)
    total = batch_size * particle_count
    sadj = np.zeros(max(total * state_dims, 0), np.float32)
    padj = np.zeros((max(total, 0), 4), np.float32)
    L = _lib.lib()
    g, o = _lib.grid_c(cfg), _lib.options_c(options)
    _lib.check(L.npa_perceive_adjoint_with_options(
        ctypes.byref(g), ctypes.byref(o), _fp(pos), pos.shape[0], _fp(st), st.shape[0],
        batch_size, particle_count, state_dims, _fp(fa), fa.shape[0], _fp(sadj), _fp(padj)),
        "perceive_adjoint_with_options")
    return PerceptionAdjointOutput(sadj, padj)


def perceive_state_adjoint_with_options(positions, states, batch_size: int, particle_count: int,
                                        state_dims: int, cfg: HashGridConfig,
                                        options: PerceptionOptions, feature_adjoint) -> np.ndarray:
    """perceive_state_adjoint_with_options (reference/adjoint.rs:4-26)."""
    return perceive_adjoint_with_options(positions, states, batch_size, particle_count,
                                         state_dims, cfg, options, feature_adjoint).state
