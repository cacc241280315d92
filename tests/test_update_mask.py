"""The resident executor's stochastic update mask (the reference's GPU executor
mask, crates/burn_automata/src/gpu_step.wgsl:1019-1056).

CPU: the oracle's twin against a direct restatement of the reference's test
helper (crates/burn_automata/tests/gpu_wgpu/common.rs:115-137).
GPU: executor rollouts with update_prob < 1 against the oracle rollout fed the
twin's masks, step by step."""

import numpy as np
import pytest

import oracle
from burn_automata_b200 import workloads

M32 = 0xFFFFFFFF


def hash_u32(value):
    x = value & M32
    x = (x ^ 61) ^ (x >> 16)
    x = (x + (x << 3)) & M32
    x ^= x >> 4
    x = (x * 0x27D4EB2D) & M32
    return x ^ (x >> 15)


def gpu_random01(particle, step, seed):
    mixed = hash_u32(particle ^ hash_u32((step + 0x9E3779B9) & M32) ^ seed)
    return np.float32(mixed >> 8) * np.float32(1.0 / 16777216.0)


def gpu_update_mask(count, update_prob, step, seed):
    seed = (seed & M32) ^ ((seed >> 32) & M32)
    return np.array([np.float32(gpu_random01(i, step, seed) < np.float32(update_prob))
                     for i in range(count)], np.float32)


@pytest.mark.parametrize("prob,step,seed", [(0.5, 0, 0), (0.25, 7, 123456789),
                                            (0.9, 2**32 - 1, 2**40 + 17)])
def test_twin_matches_the_reference_helper(prob, step, seed):
    want = gpu_update_mask(500, prob, step, seed)
    got = oracle.gpu_update_masks(1, 500, prob, 1, seed=seed, first_step=step)[0]
    np.testing.assert_array_equal(got, want)
    assert abs(float(got.mean()) - prob) < 0.08


def test_lane_seeds_follow_the_executor():
    n, seed = 300, 99
    masks = oracle.gpu_update_masks(3, n, 0.5, 1, seed=seed, first_step=4)[0].reshape(3, n)
    base = (seed & M32) ^ (seed >> 32)
    for lane in range(3):
        lane_seed = base ^ (lane * n)
        want = np.array([np.float32(gpu_random01(i, 4, lane_seed) < np.float32(0.5))
                         for i in range(n)], np.float32)
        np.testing.assert_array_equal(masks[lane], want)
    own = oracle.gpu_update_masks(2, n, 0.5, 1, lane_seeds=[5, 2**33 + 1])[0].reshape(2, n)
    np.testing.assert_array_equal(own[1], gpu_update_mask(n, 0.5, 0, 2**33 + 1))


def test_probability_edges():
    assert oracle.gpu_update_masks(1, 64, 1.0, 1)[0].min() == 1.0
    assert oracle.gpu_update_masks(1, 64, 0.0, 1)[0].max() == 0.0
    assert oracle.gpu_update_masks(1, 64, float("nan"), 1)[0].max() == 0.0


def _executor_case(w, prob, steps, seed, lane_seeds=None, first_step=0):
    import torch

    import burn_automata_b200 as ba

    m = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                           w.weights.b2))
    ex = ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)
    ex.create_state(w.positions, w.states, update_prob=prob, seed=seed, lane_seeds=lane_seeds)
    if first_step:
        ex.set_step_index(first_step)
    s = torch.cuda.Stream()
    ex.step_state_many(steps, w.dt, use_graph=True, stream=s.cuda_stream)
    assert ex.step_index == first_step + steps
    got = ex.read_state()
    ex.close()
    masks = oracle.gpu_update_masks(w.batch, w.n, prob, steps, seed=seed, first_step=first_step,
                                    lane_seeds=lane_seeds)
    ref = oracle.rollout(w.model, w.weights, w.grid, w.positions, w.states, w.batch, w.n, steps,
                         w.dt, masks=masks)
    return got, ref


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [4, 8])  # 8: the 384-thread MLP tiles
def test_executor_mask_is_bit_exact_without_log_norm(batch):
    w = workloads.make("cfg2", batch=batch, steps=1)
    w.model = w.model.with_(log_norm_grad=False, log_norm_density_grad=False)
    (pos, st), (rpos, rst, _) = _executor_case(w, 0.5, 6, seed=2024)
    np.testing.assert_array_equal(st, rst)
    np.testing.assert_array_equal(pos, rpos)


@pytest.mark.gpu
def test_executor_mask_with_lane_seeds_and_offset_step():
    w = workloads.make("cfg2", batch=3, steps=1)
    (pos, st), (rpos, rst, _) = _executor_case(w, 0.3, 5, seed=0, lane_seeds=[11, 22, 2**35 + 3],
                                               first_step=1000)
    np.testing.assert_allclose(st, rst, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(pos, rpos, rtol=1e-4, atol=1e-5)


@pytest.mark.gpu
def test_executor_mask_zero_probability_freezes_particles():
    w = workloads.make("cfg0", n=2048, steps=1)
    (pos, st), _ = _executor_case(w, 0.0, 3, seed=5)
    np.testing.assert_array_equal(st, w.states)
    np.testing.assert_array_equal(pos, w.positions)
