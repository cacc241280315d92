"""The executor's fused step (perception + MLP + Euler in one kernel after the
density pass) against the split kernels and the oracle.

The fused kernel runs the same per-particle perception code and the same MLP
tile code as the split path, so the two must agree bit for bit; both are
compared with the oracle rollout (crates/burn_automata/src/rollout/mod.rs:240-283)
as well.  Cases: cfg2 x 8 (4,096-particle rollouts, log-normalised
gradients), cfg0 with the GPU executor's stochastic mask, a ragged single
rollout whose last tile is partly empty, and a model whose options differ
from the rollout models' (density gradient on: the generic option path).
"""

import numpy as np
import pytest

from burn_automata_b200 import workloads

pytestmark = pytest.mark.gpu


def run(w, steps, fused, prob=1.0, seed=0):
    import torch

    import burn_automata_b200 as ba

    m = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                           w.weights.b2))
    ex = ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)
    ex.create_state(w.positions, w.states, update_prob=prob, seed=seed)
    if fused:
        ex.set_fused_step(fused)
    s = torch.cuda.Stream()
    ex.step_state_many(steps, w.dt, use_graph=True, stream=s.cuda_stream)
    out = ex.read_state()
    launches = ex.launches_per_step()
    ex.close()
    m.close()
    return out, launches


CASES = [("cfg2", 8, 4096, 1.0, 16), ("cfg0", 1, 4096, 0.5, 12), ("cfg0", 1, 3001, 1.0, 8)]


@pytest.mark.parametrize("name,batch,n,prob,steps", CASES,
                         ids=[f"{c[0]}x{c[1]}_n{c[2]}_p{c[3]}" for c in CASES])
def test_fused_equals_split(name, batch, n, prob, steps):
    w = workloads.make(name, batch=batch, n=n)
    (fp, fs), lf = run(w, steps, True, prob, 7)
    (sp, ss), ls = run(w, steps, False, prob, 7)
    np.testing.assert_array_equal(fs, ss)
    np.testing.assert_array_equal(fp, sp)
    assert lf == ls - 1  # one kernel instead of perception tiles + MLP step


def test_fused_matches_oracle(oracle_mod):
    w = workloads.make("cfg2", batch=4, n=4096)
    steps = 8
    (pos, st), _ = run(w, steps, True)
    rpos, rst, _ = oracle_mod.rollout(w.model, w.weights, w.grid, w.positions, w.states, w.batch,
                                      w.n, steps, w.dt)
    np.testing.assert_array_equal(st, rst)
    np.testing.assert_array_equal(pos, rpos)


def test_fused_generic_options(oracle_mod):
    w = workloads.make("cfg0", n=2048)
    w.model = w.model.with_(density_grad=True)
    w.weights = workloads.kaiming_weights(w.model, 4)
    (pos, st), _ = run(w, 4, True)
    (spos, sst), _ = run(w, 4, False)
    np.testing.assert_array_equal(st, sst)
    np.testing.assert_array_equal(pos, spos)


def test_fused_unsupported_outside_its_range():
    import burn_automata_b200 as ba

    w = workloads.make("cfg3", n=1024)
    m = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                           w.weights.b2))
    ex = ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)
    with pytest.raises(Exception, match="fused step"):
        ex.set_fused_step(True)
    ex.close()
    m.close()


def run_grouped(w, steps, groups, prob=1.0, seed=0):
    import torch

    import burn_automata_b200 as ba

    m = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                           w.weights.b2))
    ex = ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)
    ex.create_state(w.positions, w.states, update_prob=prob, seed=seed)
    ex.set_step_groups(groups)
    s = torch.cuda.Stream()
    ex.step_state_many(steps, w.dt, use_graph=True, stream=s.cuda_stream)
    ex.step_state_many(1, w.dt, use_graph=True, stream=s.cuda_stream)  # odd count: single-step graph
    out = ex.read_state()
    idx = ex.step_index
    ex.close()
    m.close()
    return out, idx


@pytest.mark.parametrize("groups,prob", [(2, 1.0), (3, 0.5), (4, 1.0)])
def test_step_groups_equal_one_chain(groups, prob):
    """Rollout groups replayed as independent graph chains give the batch's
    results bit for bit (the stochastic mask's per-group step counters
    included)."""
    w = workloads.make("cfg2", batch=7, n=4096)
    (gp, gs), gi = run_grouped(w, 6, groups, prob, 3)
    (op, os_), oi = run_grouped(w, 6, 1, prob, 3)
    assert gi == oi == 7
    np.testing.assert_array_equal(gs, os_)
    np.testing.assert_array_equal(gp, op)


def test_step_groups_range():
    import burn_automata_b200 as ba

    w = workloads.make("cfg2", batch=2, n=512)
    m = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                           w.weights.b2))
    ex = ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)
    for bad in (0, 3, 5):
        with pytest.raises(Exception, match="step groups"):
            ex.set_step_groups(bad)
    ex.set_step_groups(2)
    ex.set_step_groups(1)
    ex.close()
    m.close()


WS_CASES = [("cfg2", 8, 4096, 1.0, 12), ("cfg0", 1, 4096, 0.5, 8), ("cfg0", 1, 3001, 1.0, 6)]


@pytest.mark.parametrize("name,batch,n,prob,steps", WS_CASES,
                         ids=[f"{c[0]}x{c[1]}_n{c[2]}_p{c[3]}" for c in WS_CASES])
def test_warp_specialised_step_equals_split(name, batch, n, prob, steps):
    """The warp-specialised fused step (perception warps and MLP warps of one
    block handing feature tiles over in shared memory) gives the split
    kernels' bits, and its bounded waits all complete."""
    import burn_automata_b200 as ba

    lib = ba.load_library()
    before = lib.npa_bulk_copy_timeouts()
    w = workloads.make(name, batch=batch, n=n)
    (fp, fs), lf = run(w, steps, 2, prob, 7)
    (sp, ss), ls = run(w, steps, False, prob, 7)
    np.testing.assert_array_equal(fs, ss)
    np.testing.assert_array_equal(fp, sp)
    assert lf == ls - 1
    assert lib.npa_bulk_copy_timeouts() == before
