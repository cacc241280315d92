"""Checkpoint files (burn_automata_b200/checkpoint.py): round trip, the
shape and format checks, and a checkpoint made from the RolloutTrace JSON
that bpk.infer writes.  The resume itself (an executor continuing bit for bit
from a checkpoint) is checked on the GPU in test_checkpoint_gpu.py."""

import json

import numpy as np
import pytest

from burn_automata_b200 import checkpoint
from burn_automata_b200.bpk import trace_to_json
from burn_automata_b200.config import InvalidArgument
from burn_automata_b200.model import RolloutTrace


def make(b=2, n=5, c=3, lanes=True):
    rng = np.random.default_rng(0)
    return checkpoint.Checkpoint(
        rng.standard_normal((b * n, 4)).astype(np.float32),
        rng.standard_normal(b * n * c).astype(np.float32), b, n, c, step_index=17,
        update_prob=0.25, seed=2**63 + 5,
        lane_seeds=np.array([3, 2**40 + 1], np.uint64) if lanes else None)


@pytest.mark.parametrize("lanes", [True, False])
def test_round_trip(tmp_path, lanes):
    ck = make(lanes=lanes)
    path = str(tmp_path / "ck.npz")
    checkpoint.save(path, ck)
    got = checkpoint.load(path)
    np.testing.assert_array_equal(got.positions, ck.positions)
    np.testing.assert_array_equal(got.states, ck.states)
    assert (got.batch_size, got.particle_count, got.state_dims) == (2, 5, 3)
    assert (got.step_index, got.update_prob, got.seed) == (17, 0.25, 2**63 + 5)
    if lanes:
        np.testing.assert_array_equal(got.lane_seeds, ck.lane_seeds)
    else:
        assert got.lane_seeds is None


def test_rejects_bad_shapes_and_files(tmp_path):
    ck = make()
    ck.states = ck.states[:-1]
    with pytest.raises(InvalidArgument, match="states"):
        checkpoint.save(str(tmp_path / "a.npz"), ck)
    ck = make()
    ck.positions = ck.positions.astype(np.float64)
    with pytest.raises(InvalidArgument, match="positions"):
        checkpoint.save(str(tmp_path / "a.npz"), ck)
    ck = make()
    ck.step_index = 2**32
    with pytest.raises(InvalidArgument, match="step index"):
        checkpoint.save(str(tmp_path / "a.npz"), ck)
    bad = tmp_path / "b.npz"
    np.savez(bad, positions=np.zeros((1, 4), np.float32))
    with pytest.raises(InvalidArgument, match="not a rollout checkpoint"):
        checkpoint.load(str(bad))
    other = tmp_path / "c.npz"
    meta = {"format": "something/else"}
    np.savez(other, positions=np.zeros((1, 4), np.float32), states=np.zeros(1, np.float32),
             meta=np.frombuffer(json.dumps(meta).encode(), np.uint8))
    with pytest.raises(InvalidArgument, match="unknown checkpoint format"):
        checkpoint.load(str(other))


def test_from_trace_json(tmp_path):
    rng = np.random.default_rng(1)
    pos = rng.standard_normal((6, 4)).astype(np.float32)
    st = rng.standard_normal(12).astype(np.float32)
    trace = RolloutTrace(pos, st, 2, 3, 2, 4, np.zeros(4, np.float32))
    path = tmp_path / "trace.json"
    path.write_text(trace_to_json(trace))
    ck = checkpoint.from_trace(str(path))
    np.testing.assert_array_equal(ck.positions, pos)
    np.testing.assert_array_equal(ck.states, st)
    assert (ck.batch_size, ck.particle_count, ck.state_dims, ck.step_index) == (2, 3, 2, 0)
