"""`.bpk` model containers and the `infer` trace export.

Restates crates/burn_automata/src/import.rs:16-30 and :370-537 (manifest,
container, load / save) and the JSON written by `burn_automata infer`
(crates/burn_automata/src/cli/commands/basic.rs:4-68), so catalog models saved
by the reference drive this package's kernels and its rollout traces can be
read by the reference's tooling.

Container layout (all integers little-endian):
    b"BAUTBPK1" | u32 container version (1) | u64 payload length |
    32-byte SHA-256 of the payload | payload (the manifest as JSON)
The manifest JSON uses the reference's serde field names: enum values are
their variant names, `None` is null, weights are flat f32 arrays.
"""

from __future__ import annotations

import hashlib
import json
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, List, Optional

import numpy as np

from .config import (Boundary, EquivarianceMode, HashGridConfig, HashGridMode, InvalidModel,
                     KernelError, NpaConfig)

BPK_MAGIC = b"BAUTBPK1"
BPK_CONTAINER_VERSION = 1
BPK_HEADER_LEN = 8 + 4 + 8 + 32


class InvalidFormat(KernelError):
    """AutomataError::InvalidFormat: not a readable container or manifest."""


@dataclass
class NpaParticleInitialization:
    """import.rs:32-64: initial particles stored with a model."""

    positions: np.ndarray  # [count, 4] f32
    states: np.ndarray  # [count * state_dims] f32

    def validate(self, config: NpaConfig) -> None:
        pos = np.asarray(self.positions, np.float32).reshape(-1, 4)
        st = np.asarray(self.states, np.float32).reshape(-1)
        if pos.shape[0] == 0:
            raise InvalidModel("particle initialization cannot be empty")
        if st.size != pos.shape[0] * config.state_dims:
            raise InvalidModel(f"particle initialization has {st.size} state values; expected "
                               f"{pos.shape[0]} positions * {config.state_dims} state dims")
        if not (np.isfinite(pos).all() and np.isfinite(st).all()):
            raise InvalidModel("particle initialization contains non-finite values")

    def particle_count(self) -> int:
        return int(np.asarray(self.positions).reshape(-1, 4).shape[0])


@dataclass
class BpkModelManifest:
    """import.rs:20-30."""

    config: NpaConfig
    hashgrid: HashGridConfig
    w1: np.ndarray
    b1: np.ndarray
    w2: np.ndarray
    b2: np.ndarray
    format_version: int = 1
    model_kind: str = "npa"
    source: Optional[str] = None
    initialization: Optional[NpaParticleInitialization] = None

    def weights(self):
        from .model import NpaWeights

        return NpaWeights(self.w1, self.b1, self.w2, self.b2)

    def into_model(self, device: int = 0):
        """An NpaModel on `device` with this manifest's config and weights."""
        from .model import NpaModel

        return NpaModel(self.config, self.weights(), device=device)

    def parameter_count(self) -> int:
        return int(self.w1.size + self.b1.size + self.w2.size + self.b2.size)

    def validate(self) -> None:
        """validate_manifest (import.rs:498-504): NpaWeights::validate
        (model.rs:77-107) and the initialization, if any."""
        c = self.config
        expected = (("w1", self.w1, c.hidden_dims * c.perception_dims()),
                    ("b1", self.b1, c.hidden_dims),
                    ("w2", self.w2, c.update_dims() * c.hidden_dims),
                    ("b2", self.b2, c.update_dims()))
        for name, arr, want in expected:
            if np.asarray(arr).size != want:
                raise InvalidModel(f"{name} len {np.asarray(arr).size} != {want}")
        if self.initialization is not None:
            self.initialization.validate(c)


# ---- JSON (serde) form ----

def _f32(x) -> float:
    """The shortest decimal that reads back as the same f32 (what serde_json
    writes for an f32), as a Python float."""
    return float(str(np.float32(x)))


def _f32_list(a) -> List[float]:
    return [float(str(v)) for v in np.asarray(a, np.float32).reshape(-1)]


def _config_to_json(c: NpaConfig) -> Dict[str, Any]:
    return {
        "spatial_dims": c.spatial_dims, "state_dims": c.state_dims,
        "hidden_dims": c.hidden_dims, "eps0": _f32(c.eps0),
        "alpha": _f32(c.alpha), "density_grad": c.density_grad,
        "state_grad": c.state_grad, "log_norm_grad": c.log_norm_grad,
        "log_norm_density_grad": c.log_norm_density_grad, "stopgrad_pos": c.stopgrad_pos,
        "stopgrad_state": c.stopgrad_state, "equivariance": _variant(c.equivariance),
        "position_features": c.position_features,
        "auxiliary_input_dims": c.auxiliary_input_dims, "decoder_dims": c.decoder_dims,
        "output_dims": c.output_dims,
    }


def _grid_to_json(g: HashGridConfig) -> Dict[str, Any]:
    return {"dim": g.dim, "boundary": _variant(g.boundary), "mode": _variant(g.mode),
            "grid_size": [int(v) for v in g.grid_size], "eps": _f32(g.eps),
            "max_particles_per_block": g.max_particles_per_block}


def manifest_to_json(m: BpkModelManifest) -> Dict[str, Any]:
    out: Dict[str, Any] = {
        "format_version": m.format_version, "model_kind": m.model_kind, "source": m.source,
        "config": _config_to_json(m.config), "hashgrid": _grid_to_json(m.hashgrid),
        "weights": {"w1": _f32_list(m.w1), "b1": _f32_list(m.b1), "w2": _f32_list(m.w2),
                    "b2": _f32_list(m.b2)},
    }
    if m.initialization is not None:  # skip_serializing_if = "Option::is_none"
        out["initialization"] = {
            "positions": [_f32_list(p) for p in
                          np.asarray(m.initialization.positions, np.float32).reshape(-1, 4)],
            "states": _f32_list(m.initialization.states)}
    return out


def _need(d: Dict[str, Any], key: str, where: str):
    if key not in d:
        raise InvalidFormat(f"missing field `{key}` in {where}")
    return d[key]


# Rust variant names that are not Python identifiers.
_RUST_NAMES = {("EquivarianceMode", "NoEquivariance"): "None"}


def _variant(value) -> str:
    return _RUST_NAMES.get((type(value).__name__, value.name), value.name)


def _enum(cls, value, where: str):
    for member in cls:
        if _variant(member) == value:
            return member
    raise InvalidFormat(f"unknown variant `{value}` for {where}")


def _config_from_json(d: Dict[str, Any]) -> NpaConfig:
    w = "config"
    return NpaConfig(
        spatial_dims=int(_need(d, "spatial_dims", w)), state_dims=int(_need(d, "state_dims", w)),
        hidden_dims=int(_need(d, "hidden_dims", w)), eps0=_f32(_need(d, "eps0", w)),
        alpha=_f32(_need(d, "alpha", w)), density_grad=bool(_need(d, "density_grad", w)),
        state_grad=bool(_need(d, "state_grad", w)),
        log_norm_grad=bool(_need(d, "log_norm_grad", w)),
        log_norm_density_grad=bool(_need(d, "log_norm_density_grad", w)),
        stopgrad_pos=bool(_need(d, "stopgrad_pos", w)),
        stopgrad_state=bool(_need(d, "stopgrad_state", w)),
        # #[serde(default)] fields
        equivariance=_enum(EquivarianceMode, d.get("equivariance", "ParticleDensityAndScale"),
                           "EquivarianceMode"),
        position_features=bool(d.get("position_features", False)),
        auxiliary_input_dims=int(d.get("auxiliary_input_dims", 0)),
        # Option<usize>: serde reads a missing key as None
        decoder_dims=d.get("decoder_dims"), output_dims=d.get("output_dims"))


def _grid_from_json(d: Dict[str, Any]) -> HashGridConfig:
    w = "hashgrid"
    gs = _need(d, "grid_size", w)
    if not isinstance(gs, list) or len(gs) != 3:
        raise InvalidFormat("hashgrid.grid_size must be an array of 3 integers")
    return HashGridConfig(dim=int(_need(d, "dim", w)),
                          boundary=_enum(Boundary, _need(d, "boundary", w), "Boundary"),
                          mode=_enum(HashGridMode, _need(d, "mode", w), "HashGridMode"),
                          grid_size=tuple(int(v) for v in gs), eps=_f32(_need(d, "eps", w)),
                          max_particles_per_block=int(_need(d, "max_particles_per_block", w)))


def manifest_from_json(d: Dict[str, Any]) -> BpkModelManifest:
    if not isinstance(d, dict):
        raise InvalidFormat("manifest must be a JSON object")
    wts = _need(d, "weights", "manifest")
    init = None
    if d.get("initialization") is not None:
        i = d["initialization"]
        init = NpaParticleInitialization(
            np.asarray(_need(i, "positions", "initialization"), np.float32).reshape(-1, 4),
            np.asarray(_need(i, "states", "initialization"), np.float32).reshape(-1))
    return BpkModelManifest(
        config=_config_from_json(_need(d, "config", "manifest")),
        hashgrid=_grid_from_json(_need(d, "hashgrid", "manifest")),
        w1=np.asarray(_need(wts, "w1", "weights"), np.float32),
        b1=np.asarray(_need(wts, "b1", "weights"), np.float32),
        w2=np.asarray(_need(wts, "w2", "weights"), np.float32),
        b2=np.asarray(_need(wts, "b2", "weights"), np.float32),
        format_version=int(_need(d, "format_version", "manifest")),
        model_kind=str(_need(d, "model_kind", "manifest")), source=d.get("source"),
        initialization=init)


def _payload(m: BpkModelManifest) -> bytes:
    # serde_json::to_vec: compact separators, struct field order
    return json.dumps(manifest_to_json(m), separators=(",", ":"), allow_nan=False).encode()


# ---- container ----

def encode_bpk_manifest(m: BpkModelManifest) -> bytes:
    """encode_bpk_manifest (import.rs:444-457)."""
    m.validate()
    payload = _payload(m)
    return (BPK_MAGIC + struct.pack("<IQ", BPK_CONTAINER_VERSION, len(payload)) +
            hashlib.sha256(payload).digest() + payload)


def decode_bpk_manifest(data: bytes) -> BpkModelManifest:
    """decode_bpk_manifest (import.rs:459-496), with its error order."""
    if len(data) < BPK_HEADER_LEN:
        raise InvalidFormat(f"bpk file is shorter than header: {len(data)} < {BPK_HEADER_LEN}")
    if not data.startswith(BPK_MAGIC):
        raise InvalidFormat("missing bpk magic")
    (version,) = struct.unpack_from("<I", data, 8)
    if version != BPK_CONTAINER_VERSION:
        raise InvalidFormat(f"unsupported bpk container version {version}")
    (payload_len,) = struct.unpack_from("<Q", data, 12)
    expected_len = BPK_HEADER_LEN + payload_len
    if len(data) != expected_len:
        raise InvalidFormat(
            f"bpk payload length mismatch: file {len(data)} != expected {expected_len}")
    payload = data[BPK_HEADER_LEN:]
    if hashlib.sha256(payload).digest() != data[20:52]:
        raise InvalidFormat("bpk sha256 checksum mismatch")
    m = _manifest_from_payload(payload)
    m.validate()
    return m


def _manifest_from_payload(payload: bytes) -> BpkModelManifest:
    try:
        d = json.loads(payload.decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise InvalidFormat(f"manifest is not valid JSON: {e}") from None
    return manifest_from_json(d)


def bpk_payload_sha256(data: bytes) -> str:
    """bpk_payload_sha256 (import.rs:506-513): the header's digest as hex."""
    if len(data) < BPK_HEADER_LEN or not data.startswith(BPK_MAGIC):
        raise InvalidFormat("not a bpk container")
    return data[20:52].hex()


def load_manifest_bytes(data: bytes) -> BpkModelManifest:
    """load_manifest_bytes (import.rs:383-390): a container, or a bare JSON manifest."""
    if data.startswith(BPK_MAGIC):
        return decode_bpk_manifest(data)
    m = _manifest_from_payload(data)
    m.validate()
    return m


def load_manifest(path) -> BpkModelManifest:
    return load_manifest_bytes(Path(path).read_bytes())


def is_bpk_path(path) -> bool:
    return Path(path).suffix.lower() == ".bpk"


def save_manifest(path, m: BpkModelManifest) -> Optional[str]:
    """save_manifest (import.rs:392-410): a container for `.bpk` paths (returns
    the payload's SHA-256 hex), pretty JSON otherwise (returns None)."""
    m.validate()
    path = Path(path)
    if path.parent:
        path.parent.mkdir(parents=True, exist_ok=True)
    if is_bpk_path(path):
        path.write_bytes(encode_bpk_manifest(m))
        return hashlib.sha256(_payload(m)).hexdigest()
    path.write_text(json.dumps(manifest_to_json(m), indent=2))
    return None


# ---- infer ----

def trace_to_json(trace) -> str:
    """The RolloutTrace JSON `burn_automata infer` writes
    (serde_json::to_string_pretty, cli/commands/basic.rs:63)."""
    pos = np.asarray(trace.positions, np.float32).reshape(-1, 4)
    mean_dx = trace.mean_dx if trace.mean_dx is not None else np.zeros(0, np.float32)
    return json.dumps({
        "positions": [_f32_list(p) for p in pos],
        "states": _f32_list(trace.states),
        "batch_size": int(trace.batch_size),
        "particle_count": int(trace.particle_count),
        "state_dims": int(trace.state_dims),
        "steps": int(trace.steps),
        "mean_dx": _f32_list(mean_dx),
    }, indent=2)


def infer(manifest: BpkModelManifest, positions, states, steps: int, dt: float = 1.0,
          batch_size: int = 1, output=None, device: int = 0):
    """`burn_automata infer --model <manifest>` on the GPU for given particles
    (the manifest's own initialization when positions is None): runs the
    rollout and, when `output` is set, writes the trace JSON there."""
    from .model import RolloutConfig, run_rollout_from_particles

    if positions is None:
        if manifest.initialization is None:
            raise InvalidModel("no particles given and the manifest has no initialization")
        positions = manifest.initialization.positions
        states = manifest.initialization.states
    pos = np.asarray(positions, np.float32).reshape(-1, 4)
    if pos.shape[0] % batch_size:
        raise InvalidFormat(f"{pos.shape[0]} particles do not split into {batch_size} rollouts")
    model = manifest.into_model(device)
    try:
        cfg = RolloutConfig(batch_size=batch_size, particle_count=pos.shape[0] // batch_size,
                            steps=steps, dt=dt)
        trace = run_rollout_from_particles(model, manifest.hashgrid, cfg, pos, states)
    finally:
        model.close()
    if output is not None:
        out = Path(output)
        if out.parent:
            out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(trace_to_json(trace))
    return trace
