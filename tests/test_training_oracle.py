"""The oracle's training rollout (rollout_for_training + bptt_gradients +
mlp_backward_from_output_gradients, crates/burn_automata/src/target2d.rs:3414-3722
and training.rs:558-640) pinned by finite differences, as the reference pins
its own (target2d.rs:4310 bptt_weight_gradients_match_rollout_finite_difference):
for the loss L = sum(final positions * A_p) + sum(final states * A_s) +
w * mean_dx_norm_sum, the BPTT weight gradients given dL/d(final state) = (A_p,
A_s) and the displacement regularizer weight w must equal central differences
of L on the largest-gradient entries of b2, w2, b1 and w1.  Test
infrastructure only: the GPU path is compared with this oracle in
tests/test_training_gpu.py."""

import numpy as np
import pytest

from burn_automata_b200 import workloads


def small_case():
    w = workloads.make("cfg0", n=24)
    rng = np.random.default_rng(3)
    # a small patch so that the particles interact (eps 0.05)
    w.positions[:, :2] = rng.uniform(-0.06, 0.06, size=(24, 2)).astype(np.float32)
    w.weights = workloads.kaiming_weights(w.model, 5)
    w.weights.w1 = (w.weights.w1 * 0.5).astype(np.float32)
    return w


def loss(oracle_mod, w, weights, ap, as_, reg):
    r = oracle_mod.rollout_for_training(w.model, weights, w.grid, w.positions, w.states, 1, w.n, 2,
                                        1.0, 9)
    return (np.sum(r["final_positions"][:, :2].astype(np.float64) * ap[:, :2])
            + np.sum(r["final_states"].astype(np.float64) * as_) + reg * r["mean_dx_norm_sum"])


@pytest.mark.parametrize("reg", [0.0, 0.5])
def test_bptt_matches_finite_differences(oracle_mod, reg):
    w = small_case()
    rng = np.random.default_rng(11)
    ap = rng.standard_normal((w.n, 4)).astype(np.float32)
    ap[:, 2:] = 0.0
    as_ = (rng.standard_normal(w.n * w.state_dims) * 0.1).astype(np.float32)
    r = oracle_mod.rollout_for_training(w.model, w.weights, w.grid, w.positions, w.states, 1, w.n,
                                        2, 1.0, 9)
    g = oracle_mod.bptt_gradients(w.model, w.weights, w.grid, r, 1, w.n, ap, as_, reg)
    for name in ("b2", "w2", "b1", "w1"):
        analytic = g[name]
        idx = int(np.argmax(np.abs(analytic)))
        base = getattr(w.weights, name).astype(np.float64)
        h = 3e-3 * max(1.0, abs(base[idx]))  # the log-normalisation is strongly curved
        vals = []
        for sign in (1, -1):
            p = base.copy()
            p[idx] += sign * h
            ws = type(w.weights)(**{k: getattr(w.weights, k) for k in ("w1", "b1", "w2", "b2")})
            setattr(ws, name, p.astype(np.float32))
            vals.append(loss(oracle_mod, w, ws, ap, as_, reg))
        fd = (vals[0] - vals[1]) / (2 * h)
        assert abs(fd - analytic[idx]) <= 3e-2 * max(1.0, abs(fd)), (name, idx, analytic[idx], fd)


def test_mlp_backward_matches_finite_differences(oracle_mod):
    rng = np.random.default_rng(2)
    rows, f, h, o = 5, 7, 6, 4
    feats = rng.standard_normal(rows * f).astype(np.float32)
    w1 = rng.standard_normal(h * f).astype(np.float32) * 0.5
    b1 = rng.standard_normal(h).astype(np.float32) * 0.1
    w2 = rng.standard_normal(o * h).astype(np.float32) * 0.5
    b2 = np.zeros(o, np.float32)
    go = rng.standard_normal(rows * o).astype(np.float32)
    gw1, gb1, gw2, gb2, gf = oracle_mod.mlp_backward(feats, rows, f, h, o, w1, b1, w2, go)

    def out(f_, w1_, b1_, w2_):
        hid = np.maximum(f_.reshape(rows, f) @ w1_.reshape(h, f).T + b1_, 0.0)
        return float(np.sum((hid @ w2_.reshape(o, h).T + b2) * go.reshape(rows, o)))

    f64 = [a.astype(np.float64) for a in (feats, w1, b1, w2)]
    for k, grad in ((0, gf), (1, gw1), (2, gb1), (3, gw2)):
        for idx in range(0, grad.size, max(1, grad.size // 7)):
            e = 1e-4
            plus = [a.copy() for a in f64]
            minus = [a.copy() for a in f64]
            plus[k][idx] += e
            minus[k][idx] -= e
            fd = (out(*plus) - out(*minus)) / (2 * e)
            assert abs(fd - grad[idx]) <= 1e-3 * max(1.0, abs(fd)), (k, idx)
