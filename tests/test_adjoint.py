"""perceive_adjoint_with_options (crates/burn_automata_kernels/src/reference/adjoint.rs).

The reference has no known-answer vectors for the adjoint, so the oracle's
restatement is pinned by central finite differences of the oracle's own
(pinned) forward perception; the CUDA adjoint is then checked against the
oracle.  The GPU scatters with atomics (the reference adds serially), so the
bar is f32 summation error: allclose with rtol 1e-3 and an absolute floor of
1e-4 of the largest entry, and a normwise relative error below 1e-4."""

import numpy as np
import pytest

import oracle
from burn_automata_b200 import workloads
from burn_automata_b200.config import HashGridConfig, NpaConfig


def fd_case(log_norm):
    n, c = 48, 2
    rng = np.random.default_rng(0)
    grid = HashGridConfig.growing_2d().with_(eps=0.25, grid_size=(8, 8, 1))
    pos = np.zeros((n, 4), np.float32)
    pos[:, :2] = rng.uniform(-0.5, 0.5, (n, 2))
    st = rng.standard_normal(n * c).astype(np.float32)
    opt = NpaConfig.growing_2d().with_(log_norm_grad=log_norm,
                                       log_norm_density_grad=log_norm).perception_options()
    F = oracle.perceive_with_options(pos, st, 1, n, c, grid, opt)["features"].size // n
    fa = rng.standard_normal(n * F).astype(np.float32)
    return n, c, grid, pos, st, opt, fa


@pytest.mark.parametrize("log_norm,tol_state,tol_pos", [(False, 1e-4, 1e-3), (True, 2e-3, 1e-3)])
def test_oracle_adjoint_matches_finite_differences(log_norm, tol_state, tol_pos):
    n, c, grid, pos, st, opt, fa = fd_case(log_norm)
    sadj, padj = oracle.perceive_adjoint_with_options(pos, st, 1, n, c, grid, opt, fa)

    def f(p, s):
        feats = oracle.perceive_with_options(p, s, 1, n, c, grid, opt)["features"]
        return float(np.dot(feats.astype(np.float64), fa))

    eye = np.eye(n * c, dtype=np.float32)
    h = 1e-2
    fd_s = np.array([(f(pos, st + h * eye[i]) - f(pos, st - h * eye[i])) / (2 * h)
                     for i in range(n * c)])
    hp = 1e-4
    fd_p = np.zeros((n, 2))
    for i in range(n):
        for a in range(2):
            e = np.zeros_like(pos)
            e[i, a] = hp
            fd_p[i, a] = (f(pos + e, st) - f(pos - e, st)) / (2 * hp)
    assert np.linalg.norm(sadj - fd_s) / np.linalg.norm(fd_s) < tol_state
    assert np.linalg.norm(padj[:, :2] - fd_p) / np.linalg.norm(fd_p) < tol_pos


def adjoint_cases():
    out = []
    w = workloads.make("cfg0", n=2048, steps=1)
    for name, opt in (("growing_full", NpaConfig.growing_2d().perception_options()),
                      ("cfg0_options", w.options),
                      ("no_log_norm", NpaConfig.growing_2d().with_(
                          log_norm_grad=False, log_norm_density_grad=False).perception_options()),
                      ("no_hybrid", NpaConfig.growing_2d().perception_options())):
        if name == "no_hybrid":
            opt.hybrid_state_gradient = False
        out.append((name, w.grid, w.positions, w.states, 1, w.n, 16, opt))
    pg = HashGridConfig.texture_2d()
    pp = workloads.uniform_positions_2d(1500, 5, -1.0, 1.0)
    ps = workloads.normal_states(1500, 4, 0.3, 6)
    out.append(("periodic_grid", pg, pp, ps, 1, 1500, 4, NpaConfig.texture_2d().perception_options()))
    w3 = workloads.make("cfg3", n=3000, steps=1)
    o3 = NpaConfig.growing_3dgs().with_(position_features=True).perception_options()
    out.append(("3d_position_features", w3.grid, w3.positions, w3.states, 1, w3.n, 32, o3))
    w2 = workloads.make("cfg2", batch=3, n=1024, steps=1)
    out.append(("batched", w2.grid, w2.positions, w2.states, 3, 1024, 16, w2.options))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("case", adjoint_cases(), ids=lambda c: c[0])
def test_gpu_adjoint_matches_oracle(case):
    import burn_automata_b200 as ba

    _, grid, pos, st, b, n, c, opt = case
    F = oracle.perceive_with_options(pos, st, b, n, c, grid, opt)["features"].size // (b * n)
    fa = np.random.default_rng(7).standard_normal(b * n * F).astype(np.float32)
    got = ba.perceive_adjoint_with_options(pos, st, b, n, c, grid, opt, fa)
    sref, pref = oracle.perceive_adjoint_with_options(pos, st, b, n, c, grid, opt, fa)
    for g_, r_ in ((got.state, sref), (got.position, pref)):
        scale = float(np.abs(r_).max()) or 1.0
        np.testing.assert_allclose(g_, r_, rtol=1e-3, atol=1e-4 * scale)
        assert np.linalg.norm(g_ - r_) <= 1e-4 * max(np.linalg.norm(r_), 1e-30)
    np.testing.assert_array_equal(got.position[:, 3], 0.0)


def test_feature_adjoint_length_is_an_output_shape_error():
    import burn_automata_b200 as ba
    from burn_automata_b200.config import OutputShape

    w = workloads.make("cfg0", n=64, steps=1)
    with pytest.raises(OutputShape):
        ba.perceive_adjoint_with_options(w.positions, w.states, 1, 64, 16, w.grid, w.options,
                                         np.zeros(10, np.float32))
