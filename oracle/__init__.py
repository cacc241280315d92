"""ctypes front end of the CPU oracle (oracle/npa_oracle.c).

TEST INFRASTRUCTURE ONLY.  The oracle is the parity checker for the CUDA
product and the timed CPU baseline; it restates the reference's CPU path
(crates/burn_automata_kernels/src/{hashgrid.rs,reference/*.rs,gaussian.rs},
crates/burn_automata/src/model.rs:768-940).  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline legs import this module; the product package never
does.

Config arguments are duck-typed: any object with the attribute names of the
reference structs (HashGridConfig, PerceptionOptions, NpaConfig,
GaussianDecodeConfig) works, including burn_automata_b200's mirrors.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "libnpa_oracle.so"


class OracleError(RuntimeError):
    def __init__(self, code: int, where: str):
        super().__init__(f"oracle {where} failed with status {code}")
        self.code = code


class _Grid(ctypes.Structure):
    _fields_ = [
        ("dim", ctypes.c_int32),
        ("boundary", ctypes.c_int32),
        ("mode", ctypes.c_int32),
        ("max_particles_per_block", ctypes.c_int32),
        ("grid_size", ctypes.c_int64 * 3),
        ("eps", ctypes.c_float),
        ("reserved", ctypes.c_int32),
    ]


class _Opt(ctypes.Structure):
    _fields_ = [
        ("state_grad", ctypes.c_uint8),
        ("density_grad", ctypes.c_uint8),
        ("scale_equivariance", ctypes.c_uint8),
        ("particle_density_equivariance", ctypes.c_uint8),
        ("log_norm_grad", ctypes.c_uint8),
        ("log_norm_density_grad", ctypes.c_uint8),
        ("hybrid_state_gradient", ctypes.c_uint8),
        ("position_features", ctypes.c_uint8),
        ("eps0", ctypes.c_float),
        ("reserved", ctypes.c_int32),
    ]


class _Model(ctypes.Structure):
    _fields_ = [
        ("spatial_dims", ctypes.c_int32),
        ("state_dims", ctypes.c_int32),
        ("hidden_dims", ctypes.c_int32),
        ("auxiliary_input_dims", ctypes.c_int32),
        ("eps0", ctypes.c_float),
        ("alpha", ctypes.c_float),
        ("equivariance", ctypes.c_int32),
        ("density_grad", ctypes.c_uint8),
        ("state_grad", ctypes.c_uint8),
        ("log_norm_grad", ctypes.c_uint8),
        ("log_norm_density_grad", ctypes.c_uint8),
        ("position_features", ctypes.c_uint8),
        ("reserved", ctypes.c_uint8 * 7),
    ]


class _Decode(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32),
        ("sh_degree", ctypes.c_int32),
        ("sigma", ctypes.c_float),
        ("min_scale", ctypes.c_float),
        ("max_scale", ctypes.c_float),
        ("max_anisotropy", ctypes.c_float),
        ("opacity_scale", ctypes.c_float),
        ("min_opacity", ctypes.c_float),
        ("max_opacity", ctypes.c_float),
        ("reserved", ctypes.c_int32),
    ]


class _Splat(ctypes.Structure):
    _fields_ = [("image_size", ctypes.c_int64), ("sigma", ctypes.c_float),
                ("lo", ctypes.c_float), ("hi", ctypes.c_float),
                ("normalize_color", ctypes.c_int32), ("y_up", ctypes.c_int32),
                ("pixel_size", ctypes.c_float)]


_BOUNDARY = {"Periodic": 0, "Clamped": 1}
_MODE = {"Grid": 0, "Particle": 1}
_EQUIV = {"None": 0, "ParticleDensity": 1, "ParticleDensityAndScale": 2}
_DECODE = {
    "ParticlePoint": 0,
    "GaussianSh0FixedScale": 1,
    "GaussianSh0LearnedScale": 2,
    "GaussianSh0Oriented": 3,
}


def _enum_value(v, table):
    if isinstance(v, (int, np.integer)):
        return int(v)
    name = getattr(v, "name", v)
    return table[str(name)]


def build(force: bool = False) -> Path:
    """Compile libnpa_oracle.so with the committed Makefile if it is missing."""
    if force or not _LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        P = ctypes.POINTER
        f32p = P(ctypes.c_float)
        i64p = P(ctypes.c_int64)
        i64 = ctypes.c_int64
        L.ora_grid_validate.argtypes = [P(_Grid)]
        L.ora_cell_count.argtypes = [P(_Grid)]
        L.ora_cell_count.restype = i64
        L.ora_cell_for_position.argtypes = [P(_Grid), f32p]
        L.ora_cell_for_position.restype = i64
        L.ora_build_hashgrid.argtypes = [P(_Grid), f32p, i64, i64, i64p, i64p, i64p]
        L.ora_feature_dims.argtypes = [P(_Grid), P(_Opt), i64]
        L.ora_feature_dims.restype = i64
        L.ora_perceive.argtypes = [P(_Grid), P(_Opt), f32p, f32p, i64, i64, i64, f32p, f32p,
                                   f32p, f32p, f32p]
        L.ora_moment_det.argtypes = [P(_Grid), f32p, i64, i64, f32p]
        L.ora_forward_update.argtypes = [f32p, i64, i64, i64, i64, f32p, f32p, f32p, f32p, f32p]
        L.ora_euler_step.argtypes = [P(_Grid), f32p, f32p, f32p, f32p, i64, i64, i64,
                                     ctypes.c_float, f32p, f32p, f32p]
        L.ora_model_perception_dims.argtypes = [P(_Model)]
        L.ora_model_perception_dims.restype = i64
        L.ora_step.argtypes = [P(_Model), f32p, f32p, f32p, f32p, P(_Grid), f32p, f32p, i64, i64,
                               ctypes.c_float, f32p, f32p, f32p, f32p, f32p, f32p, f32p]
        L.ora_rollout.argtypes = [P(_Model), f32p, f32p, f32p, f32p, P(_Grid), f32p, f32p, i64,
                                  i64, i64, ctypes.c_float, f32p, f32p]
        L.ora_gaussian_record_floats.argtypes = [P(_Decode)]
        L.ora_gaussian_record_floats.restype = i64
        L.ora_decode_gaussians.argtypes = [P(_Decode), f32p, f32p, i64, i64, f32p]
        L.ora_gpu_update_mask.argtypes = [i64, i64, ctypes.c_float, ctypes.c_uint32,
                                          P(ctypes.c_uint32), f32p]
        L.ora_splat_particles_2d.argtypes = [P(_Splat), f32p, f32p, i64, f32p]
        L.ora_perceive_adjoint.argtypes = [P(_Grid), P(_Opt), f32p, f32p, i64, i64, i64, f32p,
                                           f32p, f32p]
        u32p = P(ctypes.c_uint32)
        L.ora_stdrng_key.argtypes = [ctypes.c_uint64, u32p]
        L.ora_chacha_block.argtypes = [u32p, ctypes.c_uint64, ctypes.c_int, u32p]
        L.ora_rollout_masks.argtypes = [ctypes.c_uint64, ctypes.c_float, i64, i64, i64, f32p]
        L.ora_mlp_backward.argtypes = [f32p, i64, i64, i64, i64, f32p, f32p, f32p, f32p, f32p,
                                       f32p, f32p, f32p, f32p]
        L.ora_rollout_for_training.argtypes = [P(_Model), f32p, f32p, f32p, f32p, P(_Grid), f32p,
                                               f32p, i64, i64, i64, ctypes.c_float,
                                               ctypes.c_uint64, f32p, f32p, f32p, f32p, f32p,
                                               f32p]
        L.ora_bptt_gradients.argtypes = [P(_Model), f32p, f32p, f32p, f32p, P(_Grid), f32p, f32p,
                                         f32p, i64, i64, i64, f32p, f32p, ctypes.c_float,
                                         ctypes.c_int, ctypes.c_int, f32p, f32p, f32p, f32p, f32p,
                                         f32p]
        L.ora_set_threads.argtypes = [ctypes.c_int]
        L.ora_set_log1p_mode.argtypes = [ctypes.c_int]
        L.ora_ln_1p.argtypes = [f32p, i64, f32p]
        L.ora_get_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def mlp_backward(features, rows: int, in_dims: int, hidden: int, out_dims: int, w1, b1, w2,
                 output_gradients):
    """training.rs:558 mlp_backward_from_output_gradients -> (gw1, gb1, gw2, gb2, gfeatures)."""
    f = _f32(features).reshape(-1)
    g = _f32(output_gradients).reshape(-1)
    ws = [_f32(w).reshape(-1) for w in (w1, b1, w2)]
    out = [np.zeros(hidden * in_dims, np.float32), np.zeros(hidden, np.float32),
           np.zeros(out_dims * hidden, np.float32), np.zeros(out_dims, np.float32),
           np.zeros(rows * in_dims, np.float32)]
    _check(lib().ora_mlp_backward(_ptr(f), rows, in_dims, hidden, out_dims, *[_ptr(w) for w in ws],
                                  _ptr(g), *[_ptr(o) for o in out]), "mlp_backward")
    return tuple(out)


def rollout_for_training(model_cfg, weights, grid, positions, states, batch, n, steps,
                         update_prob=1.0, seed=0):
    """target2d.rs:3414 rollout_for_training -> dict(snapshot positions [steps, B*N, 4],
    states [steps, B*N*C], masks [steps, B*N], final positions / states, mean_dx_norm_sum)."""
    m = model_struct(model_cfg)
    g = grid_struct(grid)
    c = model_cfg.state_dims
    total = batch * n
    w1, b1, w2, b2 = [_f32(w) for w in (weights.w1, weights.b1, weights.w2, weights.b2)]
    pos = _f32(positions).reshape(-1, 4)
    st = _f32(states).reshape(-1)
    sp = np.zeros((steps, total, 4), np.float32)
    ss = np.zeros((steps, total * c), np.float32)
    sm = np.zeros((steps, total), np.float32)
    fp = np.zeros((total, 4), np.float32)
    fs = np.zeros(total * c, np.float32)
    mean = np.zeros(1, np.float32)
    _check(lib().ora_rollout_for_training(ctypes.byref(m), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2),
                                          ctypes.byref(g), _ptr(pos), _ptr(st), batch, n, steps,
                                          float(update_prob), int(seed) & 0xFFFFFFFFFFFFFFFF,
                                          _ptr(sp), _ptr(ss), _ptr(sm), _ptr(fp), _ptr(fs),
                                          _ptr(mean)), "rollout_for_training")
    return {"snapshot_positions": sp, "snapshot_states": ss, "snapshot_masks": sm,
            "final_positions": fp, "final_states": fs, "mean_dx_norm_sum": float(mean[0])}


def bptt_gradients(model_cfg, weights, grid, rollout, batch, n, position_gradients,
                   state_gradients, regularizer_weight=0.0, stopgrad_pos=False,
                   stopgrad_state=False):
    """target2d.rs:3550 bptt_gradients -> dict(w1, b1, w2, b2, position_adjoint, state_adjoint)."""
    m = model_struct(model_cfg)
    g = grid_struct(grid)
    c = model_cfg.state_dims
    total = batch * n
    steps = rollout["snapshot_masks"].shape[0]
    f = int(lib().ora_model_perception_dims(ctypes.byref(m)))
    h, o = model_cfg.hidden_dims, model_cfg.spatial_dims + c
    w1, b1, w2, b2 = [_f32(w) for w in (weights.w1, weights.b1, weights.w2, weights.b2)]
    sp = _f32(rollout["snapshot_positions"]).reshape(-1)
    ss = _f32(rollout["snapshot_states"]).reshape(-1)
    sm = _f32(rollout["snapshot_masks"]).reshape(-1)
    pg = _f32(position_gradients).reshape(-1)
    sg = _f32(state_gradients).reshape(-1)
    out = {"w1": np.zeros(h * f, np.float32), "b1": np.zeros(h, np.float32),
           "w2": np.zeros(o * h, np.float32), "b2": np.zeros(o, np.float32),
           "position_adjoint": np.zeros((total, 4), np.float32),
           "state_adjoint": np.zeros(total * c, np.float32)}
    _check(lib().ora_bptt_gradients(ctypes.byref(m), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2),
                                    ctypes.byref(g), _ptr(sp), _ptr(ss), _ptr(sm), batch, n, steps,
                                    _ptr(pg), _ptr(sg), float(regularizer_weight),
                                    int(bool(stopgrad_pos)), int(bool(stopgrad_state)),
                                    _ptr(out["w1"]), _ptr(out["b1"]), _ptr(out["w2"]),
                                    _ptr(out["b2"]), _ptr(out["position_adjoint"]),
                                    _ptr(out["state_adjoint"])), "bptt_gradients")
    return out


def ln_1p(x) -> np.ndarray:
    """f32::ln_1p as the reference binds it: the host C library's log1pf."""
    a = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty_like(a)
    lib().ora_ln_1p(_ptr(a), a.shape[0], _ptr(out))
    return out


class device_log1p:
    """Context: the oracle's ln_1p evaluated as the device library does (f64
    log1p rounded once to f32) instead of the reference's libm log1pf.  With
    it the whole rollout path, log-normalisation included, is predicted bit
    for bit; outside it the oracle is the reference's arithmetic."""

    def __enter__(self):
        lib().ora_set_log1p_mode(1)
        return self

    def __exit__(self, *exc):
        lib().ora_set_log1p_mode(0)
        return False


def set_threads(n: int) -> None:
    lib().ora_set_threads(int(n))


def get_threads() -> int:
    return int(lib().ora_get_threads())


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a, ctype=ctypes.c_float):
    if a is None:
        return None
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def _check(code: int, where: str) -> None:
    if code != 0:
        raise OracleError(code, where)


def grid_struct(cfg) -> _Grid:
    g = _Grid()
    g.dim = int(cfg.dim)
    g.boundary = _enum_value(cfg.boundary, _BOUNDARY)
    g.mode = _enum_value(cfg.mode, _MODE)
    g.max_particles_per_block = int(getattr(cfg, "max_particles_per_block", 32))
    for i in range(3):
        g.grid_size[i] = int(cfg.grid_size[i])
    g.eps = float(cfg.eps)
    return g


def options_struct(opt) -> _Opt:
    o = _Opt()
    for name in ("state_grad", "density_grad", "scale_equivariance",
                 "particle_density_equivariance", "log_norm_grad", "log_norm_density_grad",
                 "hybrid_state_gradient", "position_features"):
        setattr(o, name, int(bool(getattr(opt, name))))
    o.eps0 = float(opt.eps0)
    return o


def model_struct(cfg) -> _Model:
    m = _Model()
    m.spatial_dims = int(cfg.spatial_dims)
    m.state_dims = int(cfg.state_dims)
    m.hidden_dims = int(cfg.hidden_dims)
    m.auxiliary_input_dims = int(getattr(cfg, "auxiliary_input_dims", 0))
    m.eps0 = float(cfg.eps0)
    m.alpha = float(cfg.alpha)
    m.equivariance = _enum_value(cfg.equivariance, _EQUIV)
    for name in ("density_grad", "state_grad", "log_norm_grad", "log_norm_density_grad",
                 "position_features"):
        setattr(m, name, int(bool(getattr(cfg, name))))
    return m


def decode_struct(cfg) -> _Decode:
    d = _Decode()
    d.mode = _enum_value(cfg.mode, _DECODE)
    d.sh_degree = int(cfg.sh_degree)
    for name in ("sigma", "min_scale", "max_scale", "max_anisotropy", "opacity_scale",
                 "min_opacity", "max_opacity"):
        setattr(d, name, float(getattr(cfg, name)))
    return d


def cell_for_position(cfg, pos4) -> int:
    g = grid_struct(cfg)
    p = _f32(pos4).reshape(4)
    return int(lib().ora_cell_for_position(ctypes.byref(g), _ptr(p)))


def build_hashgrid(positions, batch: int, n: int, cfg):
    """hashgrid.rs:16 build_hashgrid -> (bin_offsets, permutation, inverse_permutation)."""
    g = grid_struct(cfg)
    pos = _f32(positions).reshape(-1, 4)
    cells = int(lib().ora_cell_count(ctypes.byref(g))) if cfg.dim in (2, 3) else 1
    offsets = np.zeros(batch * cells + 1, dtype=np.int64)
    perm = np.zeros(batch * n, dtype=np.int64)
    inv = np.zeros(batch * n, dtype=np.int64)
    _check(lib().ora_build_hashgrid(ctypes.byref(g), _ptr(pos), batch, n,
                                    _ptr(offsets, ctypes.c_int64), _ptr(perm, ctypes.c_int64),
                                    _ptr(inv, ctypes.c_int64)), "build_hashgrid")
    return offsets, perm, inv


def perceive_with_options(positions, states, batch: int, n: int, c: int, cfg, opt):
    """forward.rs:26 perceive_with_options -> dict of features and intermediates."""
    g = grid_struct(cfg)
    o = options_struct(opt)
    pos = _f32(positions).reshape(-1, 4)
    st = _f32(states).reshape(-1)
    total = batch * n
    fd = int(lib().ora_feature_dims(ctypes.byref(g), ctypes.byref(o), c))
    feats = np.zeros(total * fd, dtype=np.float32)
    dens = np.zeros(total, dtype=np.float32)
    blur = np.zeros(total * c, dtype=np.float32)
    sgrad = np.zeros(total * c * cfg.dim, dtype=np.float32) if opt.state_grad else None
    dgrad = np.zeros(total * cfg.dim, dtype=np.float32) if opt.density_grad else None
    _check(lib().ora_perceive(ctypes.byref(g), ctypes.byref(o), _ptr(pos), _ptr(st), batch, n, c,
                              _ptr(feats), _ptr(dens), _ptr(blur), _ptr(sgrad), _ptr(dgrad)),
           "perceive")
    return {
        "features": feats,
        "density": dens,
        "blurred_state": blur,
        "state_gradient": sgrad if sgrad is not None else np.zeros(0, np.float32),
        "density_gradient": dgrad if dgrad is not None else np.zeros(0, np.float32),
        "feature_dims": fd,
    }


def moment_determinants(positions, batch: int, n: int, cfg) -> np.ndarray:
    """det of each particle's hybrid moment matrix (moment_matrix,
    forward.rs:357-382), as safe_inverse_symmetric (kernels.rs:3-51) forms it."""
    g = grid_struct(cfg)
    pos = _f32(positions).reshape(-1, 4)
    det = np.zeros(batch * n, dtype=np.float32)
    _check(lib().ora_moment_det(ctypes.byref(g), _ptr(pos), batch, n, _ptr(det)),
           "moment_det")
    return det


def forward_update(features, rows: int, in_dims: int, hidden: int, out_dims: int, w1, b1, w2, b2):
    """model.rs:900 forward_update_from_features."""
    f = _f32(features).reshape(-1)
    out = np.zeros(rows * out_dims, dtype=np.float32)
    ws = [_f32(w) for w in (w1, b1, w2, b2)]
    _check(lib().ora_forward_update(_ptr(f), rows, in_dims, hidden, out_dims,
                                    *[_ptr(w) for w in ws], _ptr(out)), "forward_update")
    return out


def euler_step(positions, states, dx, ds, batch, n, c, cfg, dt, mask=None):
    """step.rs:4 euler_step -> (next_positions, next_states)."""
    g = grid_struct(cfg)
    pos = _f32(positions).reshape(-1, 4)
    st = _f32(states).reshape(-1)
    dxa = _f32(dx).reshape(-1, 4)
    dsa = _f32(ds).reshape(-1)
    m = _f32(mask).reshape(-1) if mask is not None else None
    npos = np.zeros_like(pos)
    nst = np.zeros_like(st)
    _check(lib().ora_euler_step(ctypes.byref(g), _ptr(pos), _ptr(st), _ptr(dxa), _ptr(dsa), batch,
                                n, c, float(dt), _ptr(m), _ptr(npos), _ptr(nst)), "euler_step")
    return npos, nst


def step(model_cfg, weights, grid, positions, states, batch, n, dt, mask=None):
    """model.rs:768 NpaModel::step_cpu -> dict(next_positions, next_states, dx, ds, features, density)."""
    m = model_struct(model_cfg)
    g = grid_struct(grid)
    w1, b1, w2, b2 = [_f32(w) for w in (weights.w1, weights.b1, weights.w2, weights.b2)]
    pos = _f32(positions).reshape(-1, 4)
    st = _f32(states).reshape(-1)
    total = batch * n
    c = int(model_cfg.state_dims)
    o = _Opt()
    o.state_grad, o.density_grad = m.state_grad, m.density_grad
    o.position_features = m.position_features
    fd = int(lib().ora_feature_dims(ctypes.byref(g), ctypes.byref(o), c))
    mk = _f32(mask).reshape(-1) if mask is not None else None
    npos = np.zeros_like(pos)
    nst = np.zeros_like(st)
    dx = np.zeros((total, 4), np.float32)
    ds = np.zeros(total * c, np.float32)
    feats = np.zeros(total * fd, np.float32)
    dens = np.zeros(total, np.float32)
    _check(lib().ora_step(ctypes.byref(m), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), ctypes.byref(g),
                          _ptr(pos), _ptr(st), batch, n, float(dt), _ptr(mk), _ptr(npos), _ptr(nst),
                          _ptr(dx), _ptr(ds), _ptr(feats), _ptr(dens)), "step")
    return {"next_positions": npos, "next_states": nst, "dx": dx, "ds": ds, "features": feats,
            "density": dens}


def rollout(model_cfg, weights, grid, positions, states, batch, n, steps, dt, masks=None):
    """rollout/mod.rs:240 run_rollout_from_particles (mask of ones unless given)."""
    m = model_struct(model_cfg)
    g = grid_struct(grid)
    w1, b1, w2, b2 = [_f32(w) for w in (weights.w1, weights.b1, weights.w2, weights.b2)]
    pos = _f32(positions).reshape(-1, 4).copy()
    st = _f32(states).reshape(-1).copy()
    mk = _f32(masks).reshape(-1) if masks is not None else None
    mean_dx = np.zeros(steps, np.float32)
    _check(lib().ora_rollout(ctypes.byref(m), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2),
                             ctypes.byref(g), _ptr(pos), _ptr(st), batch, n, steps, float(dt),
                             _ptr(mk), _ptr(mean_dx)), "rollout")
    return pos, st, mean_dx


def gpu_lane_seeds(batch: int, n: int, seed: int, lane_seeds=None) -> np.ndarray:
    """gpu_random_seed / gpu_lane_seeds (gpu/helpers/params.rs:186-188,
    gpu/executor/state.rs:1282-1312)."""
    fold = lambda v: (int(v) & 0xFFFFFFFF) ^ ((int(v) >> 32) & 0xFFFFFFFF)
    if lane_seeds is not None:
        return np.array([fold(v) for v in lane_seeds], np.uint32)
    return np.array([fold(seed) ^ ((lane * n) & 0xFFFFFFFF) for lane in range(batch)], np.uint32)


def gpu_update_masks(batch: int, n: int, update_prob: float, steps: int, seed: int = 0,
                     first_step: int = 0, lane_seeds=None) -> np.ndarray:
    """The executor's masks for `steps` consecutive steps: [steps, batch * n]."""
    seeds = gpu_lane_seeds(batch, n, seed, lane_seeds)
    out = np.zeros((steps, batch * n), np.float32)
    for k in range(steps):
        _check(lib().ora_gpu_update_mask(batch, n, float(update_prob),
                                         (first_step + k) & 0xFFFFFFFF,
                                         seeds.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                                         _ptr(out[k])), "gpu_update_mask")
    return out


def stdrng_key(rng_seed: int) -> np.ndarray:
    """rand_core 0.9 seed_from_u64 as the ChaCha key words (parity unpinned)."""
    key = np.zeros(8, np.uint32)
    lib().ora_stdrng_key(int(rng_seed) & 0xFFFFFFFFFFFFFFFF,
                         key.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return key


def chacha_block(key, counter: int, rounds: int) -> np.ndarray:
    """One ChaCha block (64-bit counter in words 12-13, stream 0) as 16 words."""
    k = np.ascontiguousarray(key, np.uint32)
    out = np.zeros(16, np.uint32)
    u32p = ctypes.POINTER(ctypes.c_uint32)
    lib().ora_chacha_block(k.ctypes.data_as(u32p), int(counter), int(rounds),
                           out.ctypes.data_as(u32p))
    return out


def rollout_masks(rollout_seed: int, update_prob: float, count: int, steps: int,
                  first_step: int = 0) -> np.ndarray:
    """The masks run_rollout_from_particles (rollout/mod.rs:222-238) draws for
    `steps` steps from step `first_step` (0-based): [steps, count].  Restated
    StdRng stream; parity unpinned (no Rust, no golden values)."""
    out = np.zeros((steps, count), np.float32)
    _check(lib().ora_rollout_masks(int(rollout_seed) & 0xFFFFFFFFFFFFFFFF, float(update_prob),
                                   count, first_step, steps, _ptr(out)), "rollout_masks")
    return out


def perceive_adjoint_with_options(positions, states, batch: int, n: int, c: int, cfg, opt,
                                  feature_adjoint):
    """adjoint.rs:28 perceive_adjoint_with_options -> (state [B*N*C], position [B*N, 4])."""
    g = grid_struct(cfg)
    o = options_struct(opt)
    pos = _f32(positions).reshape(-1, 4)
    st = _f32(states).reshape(-1)
    fa = _f32(feature_adjoint).reshape(-1)
    total = batch * n
    sadj = np.zeros(max(total * c, 1), np.float32)
    padj = np.zeros((max(total, 1), 4), np.float32)
    _check(lib().ora_perceive_adjoint(ctypes.byref(g), ctypes.byref(o), _ptr(pos), _ptr(st), batch,
                                      n, c, _ptr(fa), _ptr(sadj), _ptr(padj)), "perceive_adjoint")
    return sadj[:total * c], padj[:total]


def splat_particles_2d(positions, colors, cfg) -> np.ndarray:
    """splat.rs:30-93 -> [image_size^2, 4]."""
    c = _Splat(int(cfg.image_size), float(cfg.sigma), float(cfg.lo), float(cfg.hi),
               1 if cfg.normalize_color else 0, 1 if cfg.y_up else 0, float(cfg.pixel_size))
    pos = _f32(positions).reshape(-1, 4)
    col = _f32(colors).reshape(-1)
    out = np.zeros((int(cfg.image_size) ** 2, 4), np.float32)
    _check(lib().ora_splat_particles_2d(ctypes.byref(c), _ptr(pos), _ptr(col), pos.shape[0],
                                        _ptr(out)), "splat")
    return out


def decode_gaussians(positions, states, c: int, cfg):
    """gaussian.rs:53 decode_gaussians_3d -> records [count, 12 + 3k]."""
    d = decode_struct(cfg)
    pos = _f32(positions).reshape(-1, 4)
    st = _f32(states).reshape(-1)
    count = pos.shape[0]
    rec = int(lib().ora_gaussian_record_floats(ctypes.byref(d)))
    out = np.zeros(count * rec, np.float32)
    _check(lib().ora_decode_gaussians(ctypes.byref(d), _ptr(pos), _ptr(st), count, c, _ptr(out)),
           "decode_gaussians")
    return out.reshape(count, rec)
