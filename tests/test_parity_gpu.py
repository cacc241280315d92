"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Bars, from the path's parity contract:
  - hashgrid (bin_offsets, permutation, inverse_permutation): bit-exact;
  - per-step perception, MLP output and decoded Gaussians: within
    rtol 1e-5 / atol 1e-6 (np.allclose);
  - final state after 64 steps: within 1e-3 relative (normwise, since the
    rollout is chaotic).
The device arithmetic follows the reference's f32 operation order, so the
only sources of difference are log1p (correctly rounded on the device, the host
libm's log1pf on the oracle side) and exp/tanh in the decode.  With log
normalisation switched off the step is therefore checked for bit equality.
"""

import numpy as np
import pytest

import burn_automata_b200 as ba
from burn_automata_b200 import workloads
from burn_automata_b200.config import (Boundary, GaussianDecodeConfig, GaussianDecodeMode,
                                       HashGridConfig, HashGridMode, NpaConfig,
                                       PerceptionOptions)
from burn_automata_b200.model import NpaModel, NpaWeights
from tests.golden_cases import CASES, load_case

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def assert_hashgrid_equal(oracle_mod, pos, batch, n, grid):
    snap = ba.build_hashgrid(pos, batch, n, grid)
    off, perm, inv = oracle_mod.build_hashgrid(pos, batch, n, grid)
    np.testing.assert_array_equal(snap.bin_offsets.astype(np.int64), off)
    np.testing.assert_array_equal(snap.permutation.astype(np.int64), perm)
    np.testing.assert_array_equal(snap.inverse_permutation.astype(np.int64), inv)
    return snap


@pytest.mark.parametrize("name,batch,n", [("cfg0", 1, 4096), ("cfg2", 8, 4096),
                                          ("cfg3", 1, 16384), ("cfg1", 1, 1 << 16),
                                          ("cfg4", 1, 1 << 16)])
def test_hashgrid_bit_exact_on_configs(oracle_mod, name, batch, n):
    w = workloads.make(name, batch=batch, n=n, steps=1)
    assert_hashgrid_equal(oracle_mod, w.positions, w.batch, w.n, w.grid)


def test_hashgrid_full_size_cfg1(oracle_mod):
    w = workloads.make("cfg1")
    assert_hashgrid_equal(oracle_mod, w.positions, w.batch, w.n, w.grid)


@pytest.mark.parametrize("name", ["cfg2", "cfg4"])
def test_hashgrid_full_size_batched_and_clustered(oracle_mod, name):
    """The benchmark's own shapes: 256 x 4,096 (shared-memory sort) and one
    4,194,304-particle clustered rollout (device-wide radix sort)."""
    w = workloads.make(name)
    assert_hashgrid_equal(oracle_mod, w.positions, w.batch, w.n, w.grid)


def test_full_size_cfg2_step_bit_exact_without_log_norm(oracle_mod):
    """One step of the whole benchmark workload (1,048,576 particles) through
    the resident executor, bit for bit against the oracle."""
    import torch

    w = workloads.make("cfg2", steps=1)
    w.model = w.model.with_(log_norm_grad=False, log_norm_density_grad=False)
    m = make_model(w)
    ex = ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)
    ex.create_state(w.positions, w.states)
    ex.step_state_many(1, w.dt, use_graph=True, stream=torch.cuda.Stream().cuda_stream)
    pos, st = ex.read_state()
    ex.close()
    rpos, rst, _ = oracle_mod.rollout(w.model, w.weights, w.grid, w.positions, w.states, w.batch,
                                      w.n, 1, w.dt)
    np.testing.assert_array_equal(st, rst)
    np.testing.assert_array_equal(pos, rpos)


def test_hashgrid_edge_cases(oracle_mod):
    g2 = HashGridConfig.growing_2d()
    # empty batch and empty rollouts
    snap = ba.build_hashgrid(np.zeros((0, 4), np.float32), 3, 0, g2)
    assert np.all(snap.bin_offsets == 0) and snap.bin_offsets.shape[0] == 3 * 4096 + 1
    # one particle
    assert_hashgrid_equal(oracle_mod, np.array([[0.3, -0.2, 0, 0]], np.float32), 1, 1, g2)
    # every particle in one cell (ties resolved by index)
    same = np.tile(np.array([[0.01, 0.02, 0, 0]], np.float32), (5000, 1))
    assert_hashgrid_equal(oracle_mod, same, 2, 2500, g2)
    # far outside the domain, negative coordinates, huge values and NaN
    rng = np.random.default_rng(3)
    wild = np.zeros((4096, 4), np.float32)
    wild[:, :2] = rng.uniform(-1e6, 1e6, size=(4096, 2))
    wild[:10, 0] = [np.nan, np.inf, -np.inf, 3e38, -3e38, 1e20, -1e20, 0.0, -0.0, 1e-40]
    assert_hashgrid_equal(oracle_mod, wild, 1, 4096, g2)
    # Grid mode, periodic and clamped, non power-of-two grids
    for boundary in (Boundary.Periodic, Boundary.Clamped):
        gg = HashGridConfig(2, boundary, HashGridMode.Grid, (10, 7, 1), 0.2, 32)
        assert_hashgrid_equal(oracle_mod, wild, 4, 1024, gg)
    g3 = HashGridConfig.growing_3dgs()
    p3 = np.zeros((3000, 4), np.float32)
    p3[:, :3] = rng.uniform(-2, 2, size=(3000, 3))
    assert_hashgrid_equal(oracle_mod, p3, 3, 1000, g3)


def perception_cases():
    rng = np.random.default_rng(7)
    cases = []
    g = HashGridConfig.growing_2d().with_(eps=0.05, grid_size=(64, 64, 1))
    pos = workloads.uniform_positions_2d(2048, 1, -0.5, 0.5)
    for c in (1, 5, 16):
        st = (rng.standard_normal(2048 * c) * 0.3).astype(np.float32)
        for opt in (PerceptionOptions.new(True, True, 0.1),
                    NpaConfig.growing_2d().perception_options(),
                    NpaConfig.growing_2d().with_(density_grad=False).perception_options(),
                    PerceptionOptions(state_grad=False, density_grad=True, eps0=0.07,
                                      position_features=True),
                    PerceptionOptions(state_grad=True, density_grad=False, hybrid_state_gradient=False,
                                      scale_equivariance=False, eps0=0.2)):
            cases.append((f"2d_c{c}", g, pos, st, 2, 1024, c, opt))
    gp = HashGridConfig(2, Boundary.Periodic, HashGridMode.Grid, (10, 10, 1), 0.2, 32)
    pp = workloads.uniform_positions_2d(1500, 2, -1.0, 1.0)
    sp = (rng.standard_normal(1500 * 4) * 0.3).astype(np.float32)
    cases.append(("periodic_grid", gp, pp, sp, 1, 1500, 4, NpaConfig.texture_2d().perception_options()))
    g3 = HashGridConfig.growing_3dgs().with_(eps=0.1)
    p3 = workloads.torus_positions(3000, 4)
    for c in (8, 32):
        s3 = (rng.standard_normal(3000 * c) * 0.3).astype(np.float32)
        cases.append((f"3d_c{c}", g3, p3, s3, 1, 3000, c, NpaConfig.growing_3dgs().perception_options()))
    return cases


@pytest.mark.parametrize("case", perception_cases(), ids=lambda c: c[0])
def test_perception_parity(oracle_mod, case):
    _, grid, pos, st, batch, n, c, opt = case
    gpu = ba.perceive_with_options(pos, st, batch, n, c, grid, opt)
    ref = oracle_mod.perceive_with_options(pos, st, batch, n, c, grid, opt)
    np.testing.assert_array_equal(gpu.density, ref["density"])
    np.testing.assert_array_equal(gpu.blurred_state, ref["blurred_state"])
    exact_keys = [] if (opt.log_norm_grad or opt.log_norm_density_grad) else ["features"]
    for key in ("features", "state_gradient", "density_gradient"):
        a, b = getattr(gpu, key), ref[key]
        np.testing.assert_allclose(a, b, rtol=RTOL, atol=ATOL, err_msg=key)
        if key in exact_keys:
            np.testing.assert_array_equal(a, b)


def test_mlp_bit_exact(oracle_mod):
    for (f, h, o) in ((64, 128, 18), (160, 256, 35), (13, 5, 3), (130, 100, 34)):
        cfg = NpaConfig(spatial_dims=2, state_dims=o - 2, hidden_dims=h)
        # pick a feature width by toggling options until it matches f
        rng = np.random.default_rng(f + h)
        rows = 1000
        feats = rng.standard_normal(rows * cfg.perception_dims()).astype(np.float32)
        w = NpaWeights(
            (rng.standard_normal(h * cfg.perception_dims()) * 0.2).astype(np.float32),
            (rng.standard_normal(h) * 0.1).astype(np.float32),
            (rng.standard_normal(cfg.update_dims() * h) * 0.2).astype(np.float32),
            (rng.standard_normal(cfg.update_dims()) * 0.1).astype(np.float32))
        model = NpaModel(cfg, w)
        gpu = model.forward_update_from_features(feats)
        ref = oracle_mod.forward_update(feats, rows, cfg.perception_dims(), h, cfg.update_dims(),
                                        w.w1, w.b1, w.w2, w.b2)
        np.testing.assert_array_equal(gpu, ref)


def test_euler_bit_exact(oracle_mod):
    rng = np.random.default_rng(5)
    for grid, c in ((HashGridConfig.growing_2d(), 16), (HashGridConfig.texture_2d(), 3),
                    (HashGridConfig.growing_3dgs(), 12)):
        n = 777
        pos = rng.uniform(-2, 2, size=(n, 4)).astype(np.float32)
        st = (rng.standard_normal(n * c) * 10).astype(np.float32)
        dx = rng.standard_normal((n, 4)).astype(np.float32)
        ds = (rng.standard_normal(n * c) * 10).astype(np.float32)
        mask = (rng.uniform(size=n) < 0.5).astype(np.float32)
        for m in (None, mask):
            a = ba.euler_step(pos, st, dx, ds, 1, n, c, grid, 0.37, m)
            b = oracle_mod.euler_step(pos, st, dx, ds, 1, n, c, grid, 0.37, m)
            np.testing.assert_array_equal(a[0], b[0])
            np.testing.assert_array_equal(a[1], b[1])


def test_euler_kats_on_gpu():
    from tests.test_oracle_kat import euler_mask_case

    cfg, pos, st, dx, ds, mask = euler_mask_case()
    npos, nst = ba.euler_step(pos, st, dx, ds, 1, 2, 1, cfg, 1.0, mask)
    assert npos[0, 0] == 0.5 and npos[1, 0] == np.float32(0.9) and list(nst) == [1.0, 1.0]


def test_sph_constants_on_gpu():
    from tests.test_oracle_kat import check_sph_constants, sph_constants_case

    cfg, pos, st = sph_constants_case()
    out = ba.perceive(pos, st, 1, 2, 2, cfg, True, True)
    check_sph_constants(out.density, out.blurred_state, out.state_gradient, out.density_gradient)


@pytest.mark.parametrize("mode", list(GaussianDecodeMode))
def test_decode_parity(oracle_mod, mode):
    rng = np.random.default_rng(int(mode))
    n, c = 5000, 32
    pos = rng.standard_normal((n, 4)).astype(np.float32)
    st = (rng.standard_normal(n * c) * 3).astype(np.float32)
    for sh in ((0, 1) if mode == GaussianDecodeMode.GaussianSh0Oriented else (0,)):
        cfg = GaussianDecodeConfig(mode=mode, sh_degree=sh)
        a = ba.decode_gaussians_3d_records(pos, st, c, cfg)
        b = oracle_mod.decode_gaussians(pos, st, c, cfg)
        np.testing.assert_allclose(a, b, rtol=RTOL, atol=ATOL)
    if mode == GaussianDecodeMode.GaussianSh0Oriented:
        # degree 2 needs 9 * 3 + 8 = 35 channels: the reference asserts, this reports StateShape
        with pytest.raises(ba.config.StateShape):
            ba.decode_gaussians_3d_records(pos, st, c, GaussianDecodeConfig(mode=mode, sh_degree=2))


@pytest.mark.parametrize("name", CASES)
def test_gpu_matches_reference_python_golden(name):
    z, grid, model = load_case(name)
    n = z["n"]
    out = ba.perceive_with_options(z["positions"], z["states"], 1, n, model.state_dims, grid,
                                   model.perception_options())
    np.testing.assert_allclose(out.features, z["features"], rtol=1e-4, atol=2e-5)
    m = NpaModel(model, NpaWeights(z["w1"], z["b1"], z["w2"], z["b2"]))
    st = m.step(z["positions"], z["states"], 1, n, grid, 1.0)
    np.testing.assert_allclose(st.next_states, z["next_states"], rtol=1e-4, atol=2e-5)


def make_model(w):
    return NpaModel(w.model, NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2, w.weights.b2))


# cfg0 / cfg2 (hidden width 128) run the step's MLP as two 192-thread blocks
# per SM (96-row tiles); cfg3 (hidden width 256) keeps one block per SM.
@pytest.mark.parametrize("name,batch,n", [("cfg0", 1, 4096), ("cfg2", 4, 4096), ("cfg2", 72, 4096),
                                          ("cfg3", 1, 4096)])
def test_step_parity(oracle_mod, name, batch, n):
    w = workloads.make(name, batch=batch, n=n, steps=1)
    m = make_model(w)
    gpu = m.step(w.positions, w.states, w.batch, w.n, w.grid, w.dt)
    ref = oracle_mod.step(w.model, w.weights, w.grid, w.positions, w.states, w.batch, w.n, w.dt)
    np.testing.assert_array_equal(gpu.density, ref["density"])
    np.testing.assert_allclose(gpu.features, ref["features"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gpu.ds, ref["ds"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gpu.dx, ref["dx"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gpu.next_states, ref["next_states"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gpu.next_positions, ref["next_positions"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("batch", [1, 8, 72])
def test_step_bit_exact_without_log_norm(oracle_mod, batch):
    w = workloads.make("cfg2", batch=batch, steps=1)
    w.model = w.model.with_(log_norm_grad=False, log_norm_density_grad=False)
    m = make_model(w)
    rng = np.random.default_rng(0)
    total = w.batch * w.n
    mask = (rng.uniform(size=total) < 0.7).astype(np.float32)
    gpu = m.step(w.positions, w.states, w.batch, w.n, w.grid, w.dt, mask)
    ref = oracle_mod.step(w.model, w.weights, w.grid, w.positions, w.states, w.batch, w.n, w.dt,
                          mask)
    for key in ("features", "ds", "dx", "next_states", "next_positions", "density"):
        np.testing.assert_array_equal(getattr(gpu, key), ref[key], err_msg=key)


@pytest.mark.parametrize("hidden", [3, 64, 100])
def test_step_mlp_shapes_bit_exact(oracle_mod, hidden):
    """The step's MLP stage at other hidden widths: 64 (a 192-row tile, one
    layer-2 / epilogue thread per row), 3 (the same shape, most hidden units
    padding) and 100 (padded to 128); three 1,000-particle rollouts, so the
    last tile is partly empty."""
    w = workloads.make("cfg2", batch=3, n=1000, steps=1)
    w.model = w.model.with_(log_norm_grad=False, log_norm_density_grad=False, hidden_dims=hidden)
    kw = workloads.kaiming_weights(w.model, hidden)
    rng = np.random.default_rng(hidden)
    w.weights = type(kw)(kw.w1, (rng.standard_normal(hidden) * 0.1).astype(np.float32), kw.w2,
                         (rng.standard_normal(w.model.update_dims()) * 0.01).astype(np.float32))
    m = make_model(w)
    gpu = m.step(w.positions, w.states, w.batch, w.n, w.grid, w.dt)
    ref = oracle_mod.step(w.model, w.weights, w.grid, w.positions, w.states, w.batch, w.n, w.dt)
    for key in ("features", "ds", "dx", "next_states", "next_positions", "density"):
        np.testing.assert_array_equal(getattr(gpu, key), ref[key], err_msg=key)


def test_3d_position_gates(oracle_mod):
    w = workloads.make("cfg3", n=2048, steps=1)
    w.model = w.model.with_(position_features=True)
    w.weights = workloads.kaiming_weights(w.model, 9)
    pos = w.positions.copy()
    pos[::3, 3] = 1.0  # anchored particles
    st = w.states.reshape(-1, 32).copy()
    st[:, 3] = np.linspace(2.0, 5.0, st.shape[0])  # liveness across the gate
    st[:, 7] = np.linspace(-0.05, 0.05, st.shape[0])  # signed distance across the gate
    m = make_model(w)
    gpu = m.step(pos, st.reshape(-1), 1, w.n, w.grid, w.dt)
    ref = oracle_mod.step(w.model, w.weights, w.grid, pos, st.reshape(-1), 1, w.n, w.dt)
    np.testing.assert_allclose(gpu.next_states, ref["next_states"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gpu.next_positions, ref["next_positions"], rtol=RTOL, atol=ATOL)


def normwise(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def test_rollout_64_steps_cfg0(oracle_mod):
    w = workloads.make("cfg0")
    m = make_model(w)
    trace = ba.run_rollout_from_particles(
        m, w.grid, ba.RolloutConfig(batch_size=1, particle_count=w.n, steps=64, dt=w.dt),
        w.positions, w.states)
    pos, st, _ = oracle_mod.rollout(w.model, w.weights, w.grid, w.positions, w.states, 1, w.n,
                                    64, w.dt)
    assert normwise(trace.states, st) <= 1e-3
    assert normwise(trace.positions, pos) <= 1e-3


def test_rollout_64_steps_bit_exact_without_log_norm(oracle_mod):
    w = workloads.make("cfg0")
    w.model = w.model.with_(log_norm_grad=False)
    m = make_model(w)
    trace = ba.run_rollout_from_particles(
        m, w.grid, ba.RolloutConfig(batch_size=1, particle_count=w.n, steps=64, dt=w.dt),
        w.positions, w.states)
    pos, st, _ = oracle_mod.rollout(w.model, w.weights, w.grid, w.positions, w.states, 1, w.n,
                                    64, w.dt)
    np.testing.assert_array_equal(trace.states, st)
    np.testing.assert_array_equal(trace.positions, pos)


def test_executor_graph_matches_eager():
    import torch

    w = workloads.make("cfg2", batch=4, steps=8)
    m = make_model(w)
    outs = []
    for use_graph in (False, True):
        ex = ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)
        ex.create_state(w.positions, w.states)
        s = torch.cuda.Stream()
        ex.step_state_many(8, w.dt, use_graph=use_graph, stream=s.cuda_stream)
        outs.append(ex.read_state())
        ex.close()
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])


def test_device_tensor_perception_matches_host():
    import torch

    w = workloads.make("cfg1", n=1 << 15, steps=1)
    host = ba.perceive_with_options(w.positions, w.states, 1, w.n, 32, w.grid, w.options)
    dev = ba.perceive_with_options(torch.from_numpy(w.positions).cuda(),
                                   torch.from_numpy(w.states).cuda(), 1, w.n, 32, w.grid,
                                   w.options)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev.features.cpu().numpy(), host.features)


def test_device_perception_runner_and_profiled_repeats():
    import torch

    w = workloads.make("cfg1", n=1 << 15, steps=1)
    host = ba.perceive_with_options(w.positions, w.states, 1, w.n, 32, w.grid, w.options)
    run = ba.DevicePerception(w.grid, w.options, 1, w.n, 32)
    d_pos = torch.from_numpy(w.positions).cuda()
    d_st = torch.from_numpy(w.states).cuda()
    feats, dens = run(d_pos, d_st)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(feats.cpu().numpy(), host.features)
    np.testing.assert_array_equal(dens.cpu().numpy(), host.density)
    run.features.zero_()
    phase, total = run.run_profiled(d_pos, d_st, 3)
    assert phase.shape == (3, 3) and np.all(phase > 0) and total >= phase.sum() * 0.5
    np.testing.assert_array_equal(run.features.cpu().numpy(), host.features)


def test_host_perception_output_selection_and_out_buffers():
    w = workloads.make("cfg1", n=1 << 14, steps=1)
    full = ba.perceive_with_options(w.positions, w.states, 1, w.n, 32, w.grid, w.options)
    out = (np.full(full.features.size, np.nan, np.float32),
           np.full(full.density.size, np.nan, np.float32))
    part = ba.perceive_with_options(w.positions, w.states, 1, w.n, 32, w.grid, w.options,
                                    outputs=(), out=out)
    assert part.features is out[0] and part.blurred_state is None
    np.testing.assert_array_equal(out[0], full.features)
    np.testing.assert_array_equal(out[1], full.density)


def _pinned_like(a):
    import torch

    p = torch.empty(a.size, dtype=torch.float32).pin_memory().numpy().reshape(a.shape)
    p[...] = a
    return p


@pytest.mark.parametrize("batch,n", [(67, 4096), (160, 4096), (1025, 256)])
def test_host_step_pipelined_over_rollout_chunks(oracle_mod, batch, n):
    """Page-locked buffers: the host step runs in rollout chunks (2 for 67
    rollouts, split 33 / 34; 5 for 160; 512 / 513 small rollouts for 1025)
    whose copies overlap the other chunks' kernels.  Every output equals the
    one-chunk step of pageable buffers bit for bit, and the first and last
    rollouts match the oracle."""
    w = workloads.make("cfg2", batch=batch, n=n, steps=1)
    m = make_model(w)
    whole = m.step(w.positions, w.states, w.batch, w.n, w.grid, w.dt)
    pos, st = _pinned_like(w.positions), _pinned_like(w.states)
    out = tuple(_pinned_like(np.full(a.shape, np.nan, np.float32))
                for a in (whole.next_positions, whole.next_states, whole.dx, whole.ds,
                          whole.features, whole.density))
    r = m.step(pos, st, w.batch, w.n, w.grid, w.dt, out=out)
    assert r.next_positions is out[0] and r.density is out[5]
    for key in ("next_positions", "next_states", "dx", "ds", "features", "density"):
        np.testing.assert_array_equal(getattr(r, key), getattr(whole, key), err_msg=key)
    C = w.state_dims
    for b in (0, batch - 1):
        sub = workloads.make("cfg2", batch=1, n=n, steps=1, first=b)
        ref = oracle_mod.step(sub.model, sub.weights, sub.grid, sub.positions, sub.states, 1,
                              sub.n, sub.dt)
        rows = slice(b * w.n, (b + 1) * w.n)
        np.testing.assert_allclose(r.next_positions[rows], ref["next_positions"].reshape(-1, 4),
                                   rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(r.next_states[b * w.n * C:(b + 1) * w.n * C],
                                   ref["next_states"], rtol=RTOL, atol=ATOL)


def test_host_step_reuses_buffers_across_sizes(oracle_mod):
    """Repeated host-buffer steps (growing and shrinking sizes) through the
    model's reusable device buffers match the oracle each time."""
    w = workloads.make("cfg2", batch=4, steps=1)
    m = make_model(w)
    for b in (1, 4, 2):
        sub = workloads.make("cfg2", batch=b, steps=1)
        out = (np.empty((b * sub.n, 4), np.float32), np.empty(b * sub.n * 16, np.float32))
        r = m.step(sub.positions, sub.states, b, sub.n, sub.grid, sub.dt, outputs=(), out=out)
        assert r.dx is None and r.features is None and r.next_positions is out[0]
        ref = oracle_mod.step(sub.model, sub.weights, sub.grid, sub.positions, sub.states, b,
                              sub.n, sub.dt)
        np.testing.assert_allclose(out[1], ref["next_states"], rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(out[0], ref["next_positions"], rtol=RTOL, atol=ATOL)


def test_host_calls_report_out_of_memory_under_an_allocation_cap():
    """The host-buffer entry points return OutOfMemory (not a crash) when their
    device allocations are refused; the cap is a test hook, lifted after."""
    from burn_automata_b200.config import OutOfMemory

    L = ba.load_library()
    w = workloads.make("cfg0", n=1024, steps=1)
    m = make_model(w)
    L.npa_debug_set_allocation_cap(4096)
    try:
        with pytest.raises(OutOfMemory):
            m.step(w.positions, w.states, 1, w.n, w.grid, w.dt)
        with pytest.raises(OutOfMemory):
            ba.perceive_with_options(w.positions, w.states, 1, w.n, 16, w.grid, w.options)
    finally:
        L.npa_debug_set_allocation_cap(0)
    r = m.step(w.positions, w.states, 1, w.n, w.grid, w.dt)
    assert np.isfinite(r.next_states).all()


@pytest.mark.parametrize("n", [8192])
def test_dense_cluster_step_bit_exact_without_log_norm(oracle_mod, n):
    """One tight cluster (thousands of particles per cell): density and
    perception take the warp-cooperative neighbour walk."""
    w = workloads.make("cfg4", n=n, components=1, steps=1)
    # 16 x 16 bins: mean occupancy >= 8 selects the cooperative kernels
    w.grid = w.grid.with_(grid_size=(16, 16, 1))
    w.model = w.model.with_(log_norm_grad=False, log_norm_density_grad=False)
    m = make_model(w)
    gpu = m.step(w.positions, w.states, 1, w.n, w.grid, w.dt)
    ref = oracle_mod.step(w.model, w.weights, w.grid, w.positions, w.states, 1, w.n, w.dt)
    for key in ("density", "features", "ds", "dx", "next_states", "next_positions"):
        np.testing.assert_array_equal(getattr(gpu, key), ref[key], err_msg=key)


@pytest.mark.parametrize("dim,c", [(2, 12), (2, 16), (3, 12), (3, 16)])
def test_dense_cluster_perception_sixteen_channel_threads(oracle_mod, dim, c):
    """Dense cells with 9 to 16 channels: the cooperative kernels run one
    thread per particle over all its channels (a partial chunk at C = 12)."""
    rng = np.random.Generator(np.random.PCG64(40 + dim))
    n = 4096
    pos = np.zeros((n, 4), np.float32)
    pos[:, :dim] = (rng.standard_normal((n, dim)) * 0.1).astype(np.float32)
    if dim == 2:
        grid = workloads.cfg0_grid().with_(grid_size=(16, 16, 1))
        opt = NpaConfig.growing_2d().perception_options()
    else:
        grid = HashGridConfig.growing_3dgs().with_(eps=0.06, grid_size=(8, 8, 8))
        opt = NpaConfig.growing_3dgs().perception_options()
    st = workloads.normal_states(n, c, 0.5, 5)
    gpu = ba.perceive_with_options(pos, st, 1, n, c, grid, opt)
    ref = oracle_mod.perceive_with_options(pos, st, 1, n, c, grid, opt)
    np.testing.assert_array_equal(gpu.density, ref["density"])
    np.testing.assert_allclose(gpu.features, ref["features"], rtol=RTOL, atol=ATOL)


def test_dense_cluster_perception_full_options(oracle_mod):
    """Dense cluster through the API perception (all outputs, density and state
    gradients, 2 and 4 channel chunks), cooperative kernels."""
    w = workloads.make("cfg4", n=4096, components=1, steps=1)
    w.grid = w.grid.with_(grid_size=(16, 16, 1))
    for c in (16, 32):
        st = workloads.normal_states(w.n, c, 0.5, 3)
        opt = NpaConfig.growing_2d().perception_options()
        gpu = ba.perceive_with_options(w.positions, st, 1, w.n, c, w.grid, opt)
        ref = oracle_mod.perceive_with_options(w.positions, st, 1, w.n, c, w.grid, opt)
        np.testing.assert_array_equal(gpu.density, ref["density"])
        np.testing.assert_allclose(gpu.features, ref["features"], rtol=RTOL, atol=ATOL)


def test_dense_cluster_batches_with_warps_across_rollouts(oracle_mod):
    """Dense cells in a batch of rollouts whose size is not a multiple of 32:
    some warps hold particles of two rollouts, and the cooperative walk of
    one rollout's cell group is staged by lanes of the other (their state
    rows must come from the walked rollout)."""
    b, n = 3, 2011
    w = workloads.make("cfg4", batch=b, n=n, components=1, steps=1)
    w.grid = w.grid.with_(grid_size=(8, 8, 1))  # ~31 particles per bin: cooperative kernels
    w.model = w.model.with_(log_norm_grad=False, log_norm_density_grad=False)
    opt = w.model.perception_options()
    gpu = ba.perceive_with_options(w.positions, w.states, b, n, w.state_dims, w.grid, opt)
    ref = oracle_mod.perceive_with_options(w.positions, w.states, b, n, w.state_dims, w.grid, opt)
    np.testing.assert_array_equal(gpu.density, ref["density"])
    np.testing.assert_array_equal(gpu.features, ref["features"])
    m = make_model(w)
    got = m.step(w.positions, w.states, b, n, w.grid, w.dt)
    want = oracle_mod.step(w.model, w.weights, w.grid, w.positions, w.states, b, n, w.dt)
    for key in ("features", "next_states", "next_positions"):
        np.testing.assert_array_equal(getattr(got, key), want[key], err_msg=key)


def test_mlp_feature_tile_bulk_copies_complete():
    """The MLP step kernel's bulk (TMA) copies of feature tiles all complete
    within their bounded waits: the device timeout counter stays 0 over
    executor steps of a batched and a single-rollout configuration."""
    L = ba.load_library()
    before = L.npa_bulk_copy_timeouts()
    for name, batch in (("cfg2", 32), ("cfg3", None)):
        w = workloads.make(name, batch=batch, steps=2)
        m = make_model(w)
        ex = ba.CudaAutomataExecutor(m, w.grid, w.batch, w.n)
        ex.create_state(w.positions, w.states)
        ex.step_state_many(3, w.dt, use_graph=False)
        pos, st = ex.read_state()
        assert np.isfinite(st).all()
        ex.close()
        m.close()
    assert L.npa_bulk_copy_timeouts() == before == 0
