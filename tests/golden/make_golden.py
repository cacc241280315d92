"""Generates tests/golden/*.npz from the reference's own Python restatement.

The reference ships a dependency-free SPH + MLP step in
scripts/reference/selforg/validate_import_parity.py (density :195,
perceive_second_pass :207, mlp :251, step_python :156).  This script imports
it from a checkout of mosure/burn_automata whose path is given in
$BURN_AUTOMATA_REF and records its outputs on small seeded inputs.  Run it
where the reference is present; the .npz files it writes are committed so the
tests never need the reference at run time.

That code evaluates in f64, iterates all pairs, and always takes the
state+density-gradient branch with moment correction, dt = 1 and mask = 1,
so the cases below enable both gradients.
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
def load_reference():
    if "BURN_AUTOMATA_REF" not in os.environ:
        sys.exit("set BURN_AUTOMATA_REF to a checkout of mosure/burn_automata")
    script = (Path(os.environ["BURN_AUTOMATA_REF"])
              / "scripts/reference/selforg/validate_import_parity.py")
    if not script.exists():
        sys.exit(f"reference script not found at {script}")
    spec = importlib.util.spec_from_file_location("validate_import_parity", script)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


CASES = {
    # growing_2d perception options (state + density gradients, both log norms)
    "growing2d_c4": dict(dim=2, n=48, c=4, hidden=16, eps=0.1, grid=[64, 64, 1],
                         boundary="Clamped", mode="Particle", spread=0.18, alpha=0.5, eps0=0.1,
                         seed=11),
    # periodic Grid-mode hashgrid (texture_2d layout)
    "texture2d_c4": dict(dim=2, n=48, c=4, hidden=16, eps=0.2, grid=[10, 10, 1],
                         boundary="Periodic", mode="Grid", spread=1.0, alpha=0.5, eps0=0.2,
                         seed=12),
    # 3D Particle-mode hashgrid
    "growing3d_c8": dict(dim=3, n=40, c=8, hidden=24, eps=0.35, grid=[8, 8, 8],
                         boundary="Clamped", mode="Particle", spread=0.3, alpha=1.0, eps0=0.1,
                         seed=13),
}


def make_case(ref, name, p):
    rng = np.random.Generator(np.random.PCG64(p["seed"]))
    n, c, d, h = p["n"], p["c"], p["dim"], p["hidden"]
    pos = np.zeros((n, 4), np.float32)
    pos[:, :d] = rng.uniform(-p["spread"], p["spread"], size=(n, d)).astype(np.float32)
    states = (rng.standard_normal(n * c) * 0.5).astype(np.float32)
    f = 2 * c + c * d + d
    o = d + c
    w1 = (rng.standard_normal((h, f)) * np.sqrt(2.0 / f)).astype(np.float32).reshape(-1)
    b1 = (rng.standard_normal(h) * 0.1).astype(np.float32)
    w2 = (rng.standard_normal((o, h)) * np.sqrt(2.0 / h)).astype(np.float32).reshape(-1)
    b2 = (rng.standard_normal(o) * 0.1).astype(np.float32)
    config = dict(state_dims=c, spatial_dims=d, hidden_dims=h, alpha=p["alpha"], eps0=p["eps0"],
                  state_grad=True, density_grad=True, log_norm_grad=True,
                  log_norm_density_grad=True, equivariance="ParticleDensityAndScale")
    grid = dict(dim=d, eps=p["eps"], grid_size=p["grid"], boundary=p["boundary"], mode=p["mode"])
    weights = dict(w1=w1.tolist(), b1=b1.tolist(), w2=w2.tolist(), b2=b2.tolist())
    plist = [list(map(float, row)) for row in pos]
    slist = list(map(float, states))
    rho = ref.density(plist, grid)
    blur, grad_s, grad_rho = ref.perceive_second_pass(plist, slist, rho, c, config, grid)
    features = []
    for i in range(n):
        features += slist[i * c:(i + 1) * c] + blur[i * c:(i + 1) * c]
        features += grad_s[i * c * d:(i + 1) * c * d] + grad_rho[i * d:(i + 1) * d]
    update = ref.mlp(features, config, weights)
    npos, nst = ref.step_python(plist, slist, config, grid, weights)
    out = dict(
        positions=pos, states=states, w1=w1, b1=b1, w2=w2, b2=b2,
        density=np.array(rho), blurred_state=np.array(blur), state_gradient=np.array(grad_s),
        density_gradient=np.array(grad_rho), features=np.array(features),
        update=np.array(update), next_positions=np.array(npos), next_states=np.array(nst),
        meta=np.array(json.dumps(dict(case=name, params=p, config=config, grid=grid))),
    )
    np.savez_compressed(HERE / f"{name}.npz", **out)
    return out


def main():
    ref = load_reference()
    for name, p in CASES.items():
        make_case(ref, name, p)
        print("wrote", name)


if __name__ == "__main__":
    main()
