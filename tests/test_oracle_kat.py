"""Known-answer tests of the CPU oracle, taken from the reference's own unit
tests (crates/burn_automata_kernels/src/lib.rs).  They pin the oracle before
it is trusted as the parity checker."""

import numpy as np
import pytest

from burn_automata_b200.config import (GaussianDecodeConfig, GaussianDecodeMode, HashGridConfig,
                                       PerceptionOptions)


def test_hashgrid_counts_particles_per_cell(oracle_mod):
    # lib.rs:73-84
    cfg = HashGridConfig.growing_2d().with_(grid_size=(4, 4, 1))
    pos = np.array([[-0.9, -0.9, 0, 0], [0.9, 0.9, 0, 0]], np.float32)
    offsets, perm, inv = oracle_mod.build_hashgrid(pos, 1, 2, cfg)
    assert offsets.shape[0] == cfg.cell_count() + 1
    assert perm.shape[0] == 2
    assert np.any(np.diff(offsets) > 0)


def test_perceive_returns_finite_reference_features(oracle_mod):
    # lib.rs:87-98
    cfg = HashGridConfig.growing_2d()
    pos = np.array([[-0.05, 0, 0, 0], [0.05, 0, 0, 0]], np.float32)
    st = np.array([1, 0, 0, 1], np.float32)
    out = oracle_mod.perceive_with_options(pos, st, 1, 2, 2, cfg,
                                           PerceptionOptions.new(True, True, cfg.eps))
    assert out["feature_dims"] == 2 * 2 + 2 * cfg.dim + cfg.dim
    assert out["features"].shape[0] == 2 * out["feature_dims"]
    assert np.all(np.isfinite(out["features"]))
    assert np.all(out["density"] > 0)


def sph_constants_case():
    cfg = HashGridConfig.growing_2d().with_(grid_size=(4, 4, 1), eps=0.1)
    pos = np.array([[0, 0, 0, 0], [0.05, 0, 0, 0]], np.float32)
    st = np.array([1, 0, 0, 1], np.float32)
    return cfg, pos, st


def check_sph_constants(density, blurred, sgrad, dgrad):
    # lib.rs:100-121 (tolerances as in the reference's assert_close calls)
    assert abs(density[0] - 181.03874) <= 1e-3
    assert abs(density[1] - 181.03874) <= 1e-3
    assert abs(blurred[0] - 0.7032967) <= 1e-5
    assert abs(blurred[1] - 0.2967033) <= 1e-5
    assert abs(blurred[2] - 0.2967033) <= 1e-5
    assert abs(blurred[3] - 0.7032967) <= 1e-5
    assert abs(sgrad[0] - -13.186813) <= 1e-4
    assert abs(sgrad[2] - 13.186813) <= 1e-4
    assert abs(dgrad[0] - 1193.662) <= 1e-3
    assert abs(dgrad[2] - -1193.662) <= 1e-3


def test_perceive_matches_upstream_sph_kernel_constants(oracle_mod):
    cfg, pos, st = sph_constants_case()
    out = oracle_mod.perceive_with_options(pos, st, 1, 2, 2, cfg,
                                           PerceptionOptions.new(True, True, cfg.eps))
    check_sph_constants(out["density"], out["blurred_state"], out["state_gradient"],
                        out["density_gradient"])


def euler_mask_case():
    cfg = HashGridConfig.growing_2d()
    pos = np.array([[0, 0, 0, 0], [0.9, 0, 0, 0]], np.float32)
    st = np.array([0.0, 1.0], np.float32)
    dx = np.array([[0.5, 0, 0, 0], [0.5, 0, 0, 0]], np.float32)
    ds = np.array([1.0, 1.0], np.float32)
    mask = np.array([1.0, 0.0], np.float32)
    return cfg, pos, st, dx, ds, mask


def test_euler_step_applies_masks_and_boundaries(oracle_mod):
    # lib.rs:359-384
    cfg, pos, st, dx, ds, mask = euler_mask_case()
    npos, nst = oracle_mod.euler_step(pos, st, dx, ds, 1, 2, 1, cfg, 1.0, mask)
    assert npos[0, 0] == 0.5
    assert npos[1, 0] == np.float32(0.9)
    assert list(nst) == [1.0, 1.0]


@pytest.mark.parametrize("s0,d0,expected", [(23.0, 10.0, 24.0), (-7.0, -10.0, -8.0)])
def test_euler_step_clamps_3d_opacity_logit(oracle_mod, s0, d0, expected):
    # lib.rs:386-404
    cfg = HashGridConfig.growing_3dgs()
    pos = np.zeros((1, 4), np.float32)
    st = np.array([0, 0, 0, s0], np.float32)
    ds = np.array([0, 0, 0, d0], np.float32)
    _, nst = oracle_mod.euler_step(pos, st, np.zeros((1, 4), np.float32), ds, 1, 1, 4, cfg, 1.0)
    assert nst[3] == expected


def test_gaussian_decode_default_rgb_tail(oracle_mod):
    # lib.rs:406-435 (decode half): RGB tail (0.4, -0.2, 0.1) -> [0.9, 0.3, 0.6]
    st = np.zeros(20, np.float32)
    st[17:20] = [0.4, -0.2, 0.1]
    rec = oracle_mod.decode_gaussians(np.zeros((1, 4), np.float32), st, 20, GaussianDecodeConfig())
    assert rec.shape == (1, 15)
    assert list(rec[0, 12:15]) == [np.float32(0.9), np.float32(0.3), np.float32(0.6)]
    assert rec[0, 11] > 0


def test_gaussian_decode_modes(oracle_mod):
    # lib.rs:437-483
    pos = np.array([[0.1, -0.2, 0.3, 0.0]], np.float32)
    learned = np.zeros(8, np.float32)
    learned[3:8] = [2.0, 1.5, 0.25, -0.25, 0.0]
    cfg = GaussianDecodeConfig(mode=GaussianDecodeMode.GaussianSh0LearnedScale, sigma=0.01,
                               opacity_scale=1.0)
    r = oracle_mod.decode_gaussians(pos, learned, 8, cfg)[0]
    assert list(r[12:15]) == [0.75, 0.25, 0.5]
    assert r[8] > 0.01 and r[11] > 0.5
    assert list(r[4:8]) == [1.0, 0.0, 0.0, 0.0]
    oriented = np.zeros(20, np.float32)
    oriented[4], oriented[12], oriented[16], oriented[17] = 1.0, 1.0, 0.5, -0.5
    cfg = GaussianDecodeConfig(mode=GaussianDecodeMode.GaussianSh0Oriented, sh_degree=1)
    r = oracle_mod.decode_gaussians(pos, oriented, 20, cfg)[0]
    assert r.shape[0] == 12 + 3 * 4
    assert abs(r[4] - 1.0) <= 1e-6
    assert np.isfinite(r[8])
