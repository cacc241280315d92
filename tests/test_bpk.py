"""`.bpk` containers and manifests (crates/burn_automata/src/import.rs), after
the reference's tests/core/import_bridge.rs:3-42, plus a hand-built container
in the reference's serde layout and every decode error."""

import hashlib
import json
import struct

import numpy as np
import pytest

from burn_automata_b200 import bpk, workloads
from burn_automata_b200.config import (EquivarianceMode, HashGridConfig, InvalidModel,
                                       NpaConfig)
from burn_automata_b200.model import RolloutTrace


def manifest(config=None, grid=None, seed=123, source="binary-test"):
    config = config or NpaConfig.growing_2d()
    grid = grid or HashGridConfig.growing_2d()
    w = workloads.kaiming_weights(config, seed)
    return bpk.BpkModelManifest(config, grid, w.w1, w.b1, w.w2, w.b2, source=source)


def test_json_manifest_roundtrips(tmp_path):
    m = manifest(NpaConfig.growing_3dgs(), HashGridConfig.growing_3dgs(), 99, "unit-test")
    path = tmp_path / "manifest_roundtrip.json"
    assert bpk.save_manifest(path, m) is None
    loaded = bpk.load_manifest(path)
    assert loaded.format_version == 1 and loaded.model_kind == "npa"
    assert loaded.source == "unit-test"
    assert loaded.config == m.config and loaded.hashgrid == m.hashgrid
    loaded.validate()


def test_bpk_roundtrips_and_rejects_corruption(tmp_path):
    m = manifest()
    path = tmp_path / "manifest_roundtrip.bpk"
    digest = bpk.save_manifest(path, m)
    assert digest is not None and len(digest) == 64
    data = path.read_bytes()
    assert bpk.bpk_payload_sha256(data) == digest
    loaded = bpk.load_manifest(path)
    assert loaded.config == m.config
    np.testing.assert_array_equal(loaded.w1, m.w1)
    np.testing.assert_array_equal(loaded.b2, m.b2)
    bad = bytearray(data)
    bad[-1] = (bad[-1] + 1) % 256
    with pytest.raises(bpk.InvalidFormat, match="checksum"):
        bpk.decode_bpk_manifest(bytes(bad))


def serde_container(payload: bytes, version=1, length=None, digest=None) -> bytes:
    return (b"BAUTBPK1" + struct.pack("<IQ", version, len(payload) if length is None else length)
            + (digest or hashlib.sha256(payload).digest()) + payload)


def serde_payload(**override) -> bytes:
    """A manifest as serde_json writes it (field order, variant names, null)."""
    c = NpaConfig.growing_2d().with_(state_dims=2, hidden_dims=3, density_grad=False,
                                     state_grad=False)
    F, H, O = c.perception_dims(), c.hidden_dims, c.update_dims()
    d = {"format_version": 1, "model_kind": "npa", "source": None,
         "config": {"spatial_dims": 2, "state_dims": 2, "hidden_dims": 3, "eps0": 0.1,
                    "alpha": 0.5, "density_grad": False, "state_grad": False,
                    "log_norm_grad": True, "log_norm_density_grad": True, "stopgrad_pos": True,
                    "stopgrad_state": False, "equivariance": "None", "position_features": False,
                    "auxiliary_input_dims": 0, "decoder_dims": None, "output_dims": None},
         "hashgrid": {"dim": 2, "boundary": "Periodic", "mode": "Grid", "grid_size": [10, 10, 1],
                      "eps": 0.2, "max_particles_per_block": 32},
         "weights": {"w1": [0.25] * (F * H), "b1": [0.0, 1.0, -1.5], "w2": [0.5] * (O * H),
                     "b2": [1e-6] * O}}
    d.update(override)
    return json.dumps(d, separators=(",", ":")).encode()


def test_reads_a_serde_layout_container():
    m = bpk.decode_bpk_manifest(serde_container(serde_payload()))
    assert m.config.equivariance == EquivarianceMode.NoEquivariance
    assert m.hashgrid.boundary.name == "Periodic" and m.hashgrid.mode.name == "Grid"
    assert m.hashgrid.grid_size == (10, 10, 1)
    np.testing.assert_array_equal(m.b1, np.array([0.0, 1.0, -1.5], np.float32))
    assert m.b2.dtype == np.float32 and m.b2[0] == np.float32(1e-6)
    assert m.source is None and m.initialization is None
    # the same manifest as bare JSON (load_manifest_bytes without the magic)
    assert bpk.load_manifest_bytes(serde_payload()).config == m.config
    # serde defaults: equivariance / position_features / auxiliary dims may be absent
    d = json.loads(serde_payload())
    for k in ("equivariance", "position_features", "auxiliary_input_dims", "decoder_dims",
              "output_dims"):
        del d["config"][k]
    m2 = bpk.load_manifest_bytes(json.dumps(d).encode())
    assert m2.config.equivariance == EquivarianceMode.ParticleDensityAndScale


def test_decode_errors_in_reference_order():
    good = serde_container(serde_payload())
    with pytest.raises(bpk.InvalidFormat, match="shorter than header"):
        bpk.decode_bpk_manifest(good[:51])
    with pytest.raises(bpk.InvalidFormat, match="missing bpk magic"):
        bpk.decode_bpk_manifest(b"XAUTBPK1" + good[8:])
    with pytest.raises(bpk.InvalidFormat, match="unsupported bpk container version 2"):
        bpk.decode_bpk_manifest(serde_container(serde_payload(), version=2))
    with pytest.raises(bpk.InvalidFormat, match="length mismatch"):
        bpk.decode_bpk_manifest(good + b" ")
    with pytest.raises(bpk.InvalidFormat, match="not valid JSON"):
        bpk.decode_bpk_manifest(serde_container(b"{not json"))
    with pytest.raises(bpk.InvalidFormat, match="missing field `weights`"):
        d = json.loads(serde_payload())
        del d["weights"]
        bpk.decode_bpk_manifest(serde_container(json.dumps(d).encode()))
    with pytest.raises(bpk.InvalidFormat, match="unknown variant"):
        d = json.loads(serde_payload())
        d["hashgrid"]["mode"] = "Octree"
        bpk.decode_bpk_manifest(serde_container(json.dumps(d).encode()))
    with pytest.raises(InvalidModel, match="b1 len 2 != 3"):
        d = json.loads(serde_payload())
        d["weights"]["b1"] = [0.0, 1.0]
        bpk.decode_bpk_manifest(serde_container(json.dumps(d).encode()))
    with pytest.raises(bpk.InvalidFormat, match="not a bpk container"):
        bpk.bpk_payload_sha256(b"short")


def test_initialization_is_validated_and_kept():
    m = manifest()
    pos = workloads.uniform_positions_2d(8, 1)
    m.initialization = bpk.NpaParticleInitialization(pos, np.zeros(8 * 16, np.float32))
    back = bpk.decode_bpk_manifest(bpk.encode_bpk_manifest(m))
    np.testing.assert_array_equal(back.initialization.positions, pos)
    m.initialization = bpk.NpaParticleInitialization(pos, np.zeros(7, np.float32))
    with pytest.raises(InvalidModel, match="state values"):
        m.validate()
    m.initialization = bpk.NpaParticleInitialization(pos, np.full(8 * 16, np.nan, np.float32))
    with pytest.raises(InvalidModel, match="non-finite"):
        m.validate()


def test_trace_json_has_the_infer_fields():
    t = RolloutTrace(np.ones((2, 4), np.float32), np.arange(4, dtype=np.float32), 1, 2, 2, 3,
                     np.array([0.5, 0.25, 0.125], np.float32))
    d = json.loads(bpk.trace_to_json(t))
    assert list(d) == ["positions", "states", "batch_size", "particle_count", "state_dims",
                       "steps", "mean_dx"]
    assert d["positions"] == [[1.0] * 4] * 2 and d["mean_dx"] == [0.5, 0.25, 0.125]


@pytest.mark.gpu
def test_infer_from_a_bpk_matches_the_oracle(tmp_path, oracle_mod):
    w = workloads.make("cfg0", n=1024, steps=4)
    m = bpk.BpkModelManifest(w.model, w.grid, w.weights.w1, w.weights.b1, w.weights.w2,
                             w.weights.b2)
    m.initialization = bpk.NpaParticleInitialization(w.positions, w.states)
    path = tmp_path / "cfg0.bpk"
    bpk.save_manifest(path, m)
    out = tmp_path / "trace.json"
    trace = bpk.infer(bpk.load_manifest(path), None, None, steps=4, dt=w.dt, output=out)
    pos, st, mean_dx = oracle_mod.rollout(w.model, w.weights, w.grid, w.positions, w.states, 1,
                                          w.n, 4, w.dt)
    np.testing.assert_allclose(trace.states, st, rtol=1e-4, atol=1e-5)
    # f64 sum on the device vs the sequential f32 sum of the reference
    np.testing.assert_allclose(trace.mean_dx, mean_dx, rtol=1e-4)
    d = json.loads(out.read_text())
    assert d["steps"] == 4 and len(d["mean_dx"]) == 4 and len(d["positions"]) == w.n
