"""The training rollout on the GPU against the oracle (through the C ABI).

  mlp_backward_from_output_gradients (training.rs:558-640): bit for bit
      (every sum in the reference's order);
  rollout_for_training (target2d.rs:3414-3466): snapshots, masks and final
      particles bit for bit; mean_dx_norm_sum to the f64-vs-f32 summation of
      the per-step means;
  bptt_gradients (target2d.rs:3550-3722): with one step the weight
      gradients are the MLP backward of the loss adjoint, bit for bit; over
      several steps the perception adjoint (atomic scatter, summation order
      differs) feeds back, so the gradients agree normwise to 1e-4 and the
      adjoints at the rollout's input to 1e-4.
The oracle's own gradients are pinned by finite differences in
test_training_oracle.py.
"""

import numpy as np
import pytest

from burn_automata_b200 import workloads
from burn_automata_b200.model import NpaModel, NpaWeights
from burn_automata_b200 import training

pytestmark = pytest.mark.gpu

NORMWISE = 1e-4


def normwise(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def make_model(w):
    return NpaModel(w.model, NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2, w.weights.b2))


def case(name, n, seed=0, **model_changes):
    w = workloads.make(name, seed, batch=1, n=n)
    if model_changes:
        w.model = w.model.with_(**model_changes)
        w.weights = workloads.kaiming_weights(w.model, seed + 2)
    return w


def loss_gradients(w, seed):
    rng = np.random.default_rng(seed)
    total = w.batch * w.n
    ap = rng.standard_normal((total, 4)).astype(np.float32)
    ap[:, w.grid.dim:] = 0.0
    as_ = (rng.standard_normal(total * w.state_dims) * 0.1).astype(np.float32)
    return ap, as_


@pytest.mark.parametrize("name,n", [("cfg0", 4096), ("cfg3", 2048)])
def test_mlp_backward_bit_exact(oracle_mod, name, n):
    w = case(name, n)
    m = make_model(w)
    rng = np.random.default_rng(5)
    F, O = w.model.perception_dims(), w.model.update_dims()
    feats = rng.standard_normal(n * F).astype(np.float32)
    go = rng.standard_normal(n * O).astype(np.float32)
    g = training.mlp_backward_from_output_gradients(m, feats, go)
    ref = oracle_mod.mlp_backward(feats, n, F, w.model.hidden_dims, O, w.weights.w1, w.weights.b1,
                                  w.weights.w2, go)
    for got, want, key in zip((g.w1, g.b1, g.w2, g.b2, g.features), ref,
                              ("w1", "b1", "w2", "b2", "features")):
        np.testing.assert_array_equal(got, want, err_msg=key)


def test_mlp_backward_rejects_like_the_reference():
    w = case("cfg0", 64)
    m = make_model(w)
    F, O = w.model.perception_dims(), w.model.update_dims()
    with pytest.raises(Exception, match="whole perception rows"):
        training.mlp_backward_from_output_gradients(m, np.zeros(F + 1, np.float32),
                                                    np.zeros(O, np.float32))
    feats = np.zeros(2 * F, np.float32)
    feats[3] = np.nan
    with pytest.raises(Exception, match="features contain non-finite"):
        training.mlp_backward_from_output_gradients(m, feats, np.zeros(2 * O, np.float32))


ROLLOUTS = [("cfg0", 4096, 1.0), ("cfg0", 4096, 0.6), ("cfg3", 4096, 0.8)]


@pytest.mark.parametrize("name,n,p", ROLLOUTS, ids=[f"{r[0]}_p{r[2]}" for r in ROLLOUTS])
def test_rollout_for_training_bit_exact(oracle_mod, name, n, p):
    kw = {"position_features": False} if name == "cfg3" else {}
    w = case(name, n, **kw)
    m = make_model(w)
    steps = 8
    r = training.rollout_for_training(m, w.grid, w.positions, w.states, 1, n, steps, p, 77)
    ref = oracle_mod.rollout_for_training(w.model, w.weights, w.grid, w.positions, w.states, 1, n,
                                          steps, p, 77)
    np.testing.assert_array_equal(r.snapshot_masks, ref["snapshot_masks"])
    np.testing.assert_array_equal(r.snapshot_positions, ref["snapshot_positions"])
    np.testing.assert_array_equal(r.snapshot_states, ref["snapshot_states"])
    np.testing.assert_array_equal(r.final_positions, ref["final_positions"])
    np.testing.assert_array_equal(r.final_states, ref["final_states"])
    assert abs(r.mean_dx_norm_sum - ref["mean_dx_norm_sum"]) <= 1e-5 * abs(ref["mean_dx_norm_sum"])
    if p < 1.0:
        frac = float(np.mean(r.snapshot_masks))
        assert 0.0 < frac < 1.0


def test_rollout_for_training_rejects_3d_position_features():
    w = case("cfg3", 256, position_features=True)
    m = make_model(w)
    with pytest.raises(Exception, match="position gates"):
        training.rollout_for_training(m, w.grid, w.positions, w.states, 1, w.n, 1)


def test_bptt_one_step_weight_gradients_bit_exact(oracle_mod):
    w = case("cfg0", 4096)
    m = make_model(w)
    ap, as_ = loss_gradients(w, 1)
    r = training.rollout_for_training(m, w.grid, w.positions, w.states, 1, w.n, 1, 0.7, 3)
    ref_r = oracle_mod.rollout_for_training(w.model, w.weights, w.grid, w.positions, w.states, 1,
                                            w.n, 1, 0.7, 3)
    got = training.bptt_gradients(m, w.grid, r, ap, as_, 0.5, stopgrad_pos=False,
                                  stopgrad_state=False)
    ref = oracle_mod.bptt_gradients(w.model, w.weights, w.grid, ref_r, 1, w.n, ap, as_, 0.5,
                                    False, False)
    for key in ("w1", "b1", "w2", "b2"):
        np.testing.assert_array_equal(getattr(got.gradients, key), ref[key], err_msg=key)
    assert normwise(got.position_adjoint, ref["position_adjoint"]) <= NORMWISE
    assert normwise(got.state_adjoint, ref["state_adjoint"]) <= NORMWISE


BPTT = [("cfg0", 2048, 0.0, False, False), ("cfg0", 2048, 0.5, True, False),
        ("cfg0", 2048, 0.25, False, True), ("cfg3", 2048, 0.5, False, False)]


@pytest.mark.parametrize("name,n,reg,sgp,sgs", BPTT,
                         ids=[f"{b[0]}_reg{b[2]}_sgp{int(b[3])}_sgs{int(b[4])}" for b in BPTT])
def test_bptt_gradients_match_oracle(oracle_mod, name, n, reg, sgp, sgs):
    kw = {"position_features": False} if name == "cfg3" else {}
    w = case(name, n, **kw)
    m = make_model(w)
    ap, as_ = loss_gradients(w, 2)
    steps = 4
    r = training.rollout_for_training(m, w.grid, w.positions, w.states, 1, n, steps, 0.9, 5)
    ref_r = oracle_mod.rollout_for_training(w.model, w.weights, w.grid, w.positions, w.states, 1,
                                            n, steps, 0.9, 5)
    np.testing.assert_array_equal(r.final_states, ref_r["final_states"])
    got = training.bptt_gradients(m, w.grid, r, ap, as_, reg, stopgrad_pos=sgp,
                                  stopgrad_state=sgs)
    ref = oracle_mod.bptt_gradients(w.model, w.weights, w.grid, ref_r, 1, n, ap, as_, reg, sgp,
                                    sgs)
    for key in ("w1", "b1", "w2", "b2"):
        err = normwise(getattr(got.gradients, key), ref[key])
        assert err <= NORMWISE, (key, err)
    assert normwise(got.position_adjoint, ref["position_adjoint"]) <= NORMWISE
    assert normwise(got.state_adjoint, ref["state_adjoint"]) <= NORMWISE
    if sgp:  # the loss adjoint reaches the input unchanged
        np.testing.assert_array_equal(got.position_adjoint, ap)
