"""The benchmark's measurement contract, checked without a GPU: the reference
arm's JSON line (the CPU port of the reference path timed on a bounded
sample), the algorithmic bytes per particle that the roofline divides by, and
the DRAM traffic constants against the committed ncu summaries they are
copied from."""

import json
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "particle-steps/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["config"]["workload"] == "cfg2"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_algorithmic_bytes_per_particle():
    import bench
    from burn_automata_b200 import workloads

    w = workloads.make("cfg2")
    # feature row 4 x 64, position read + write 32, own and next state 8 x 16, permutation 4
    assert bench.mlp_kernel_bytes(w.model) == 420
    # the whole step: positions 32, states 128, density 8, keys / permutation 16, bin offsets 4
    assert bench.step_bytes(w) == pytest.approx(188.0, abs=1e-3)
    w1 = workloads.make("cfg1", n=4096)
    # position 16, state 4 x 32, volume 4, feature row 4 x 130
    assert bench.perception_kernel_bytes(w1, 130) == 668


def _profile_dram_bytes(name):
    text = (ROOT / "profiles" / name).read_text()
    scale = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}

    def metric(key):
        m = re.search(rf"^{re.escape(key)}\s+([0-9.]+)\s+(\w+)", text, re.M)
        assert m, f"{key} missing from profiles/{name}"
        return float(m.group(1)) * scale[m.group(2)]

    return metric("dram__bytes_read.sum") + metric("dram__bytes_write.sum")


@pytest.mark.parametrize("key,profile,rows", [
    (("cfg2", "mlp_step_kernel"), "mlp_step_kernel_cfg2.txt", 1 << 20),
    (("cfg1", "perception_kernel"), "perception_kernel_cfg1.txt", 1 << 20),
])
def test_traffic_constants_match_the_profiles(key, profile, rows):
    import bench

    assert bench.NCU_TRAFFIC_PER_PARTICLE[key] * rows == pytest.approx(
        _profile_dram_bytes(profile), rel=1e-6)
