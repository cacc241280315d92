"""Loader for the committed golden fixtures (tests/golden/*.npz)."""

import json
from pathlib import Path

import numpy as np

from burn_automata_b200.config import Boundary, HashGridConfig, HashGridMode, NpaConfig

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["growing2d_c4", "texture2d_c4", "growing3d_c8"]


def load_case(name):
    raw = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(raw["meta"]))
    p = meta["params"]
    z = {k: raw[k] for k in raw.files if k != "meta"}
    z["n"] = p["n"]
    grid = HashGridConfig(p["dim"], Boundary[p["boundary"]], HashGridMode[p["mode"]],
                          tuple(p["grid"]), p["eps"], 32)
    model = NpaConfig(spatial_dims=p["dim"], state_dims=p["c"], hidden_dims=p["hidden"],
                      eps0=p["eps0"], alpha=p["alpha"])
    return z, grid, model
