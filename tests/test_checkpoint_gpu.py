"""Resume: an executor restored from a checkpoint continues the rollout bit
for bit, stochastic update mask and step index included (the mask of step s
depends on s and the lane seeds, crates/burn_automata/src/gpu_step.wgsl:1019-1056)."""

import numpy as np
import pytest

from burn_automata_b200 import workloads

pytestmark = pytest.mark.gpu


def executor(w):
    import burn_automata_b200 as ba

    m = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                           w.weights.b2))
    return m, ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)


@pytest.mark.parametrize("prob,lanes", [(1.0, None), (0.5, None), (0.7, [11, 2**40 + 3])])
def test_resume_is_bit_exact(tmp_path, prob, lanes):
    import torch

    w = workloads.make("cfg2", batch=2, n=4096)
    s = torch.cuda.Stream()
    m, ex = executor(w)
    ex.create_state(w.positions, w.states, update_prob=prob, seed=99, lane_seeds=lanes)
    ex.step_state_many(7, w.dt, use_graph=True, stream=s.cuda_stream)
    straight = ex.read_state()
    ex.close()

    ex = __import__("burn_automata_b200").CudaAutomataExecutor(m, w.grid, w.batch, w.n)
    ex.create_state(w.positions, w.states, update_prob=prob, seed=99, lane_seeds=lanes)
    ex.step_state_many(3, w.dt, use_graph=True, stream=s.cuda_stream)
    path = str(tmp_path / "ck.npz")
    ex.save_checkpoint(path)
    ex.close()

    ex = __import__("burn_automata_b200").CudaAutomataExecutor(m, w.grid, w.batch, w.n)
    ex.load_checkpoint(path)
    assert ex.step_index == 3
    ex.step_state_many(4, w.dt, use_graph=True, stream=s.cuda_stream)
    resumed = ex.read_state()
    ex.close()
    m.close()
    np.testing.assert_array_equal(resumed[0], straight[0])
    np.testing.assert_array_equal(resumed[1], straight[1])


def test_load_rejects_other_shapes(tmp_path):
    w = workloads.make("cfg2", batch=2, n=1024)
    m, ex = executor(w)
    ex.create_state(w.positions, w.states)
    path = str(tmp_path / "ck.npz")
    ex.save_checkpoint(path)
    ex.close()
    w1 = workloads.make("cfg2", batch=1, n=1024)
    import burn_automata_b200 as ba

    ex1 = ba.CudaAutomataExecutor(m, w1.grid, 1, 1024)
    with pytest.raises(Exception, match="does not fit"):
        ex1.load_checkpoint(path)
    ex1.close()
    m.close()
