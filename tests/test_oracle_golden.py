"""The CPU oracle against golden vectors produced by the reference's own
Python restatement (scripts/reference/selforg/validate_import_parity.py; see
tests/golden/make_golden.py).  That code runs in f64 over all pairs, so the
f32 oracle is compared with the reference's cross-implementation tolerance
style: absolute 2e-5 plus relative 1e-4."""

import json

import numpy as np
import pytest

from burn_automata_b200.config import Boundary, HashGridConfig, HashGridMode, NpaConfig
from burn_automata_b200.workloads import NpaWeightsHost

from tests.golden_cases import CASES, load_case


@pytest.mark.parametrize("name", CASES)
def test_oracle_perception_matches_reference_python(oracle_mod, name):
    z, grid, model = load_case(name)
    n, c = z["n"], model.state_dims
    out = oracle_mod.perceive_with_options(z["positions"], z["states"], 1, n, c, grid,
                                           model.perception_options())
    for key in ("density", "blurred_state", "state_gradient", "density_gradient", "features"):
        np.testing.assert_allclose(out[key], z[key], rtol=1e-4, atol=2e-5, err_msg=key)


@pytest.mark.parametrize("name", CASES)
def test_oracle_step_matches_reference_python(oracle_mod, name):
    z, grid, model = load_case(name)
    n, d = z["n"], model.spatial_dims
    w = NpaWeightsHost(z["w1"], z["b1"], z["w2"], z["b2"])
    st = oracle_mod.step(model, w, grid, z["positions"], z["states"], 1, n, 1.0)
    upd = oracle_mod.forward_update(z["features"].astype(np.float32), n, model.perception_dims(),
                                    model.hidden_dims, model.update_dims(), z["w1"], z["b1"],
                                    z["w2"], z["b2"])
    np.testing.assert_allclose(upd, z["update"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(st["next_states"], z["next_states"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(st["next_positions"][:, :d], z["next_positions"][:, :d],
                               rtol=1e-4, atol=2e-5)
