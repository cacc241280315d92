"""The C ABI library loads, exports every entry point of include/npa_b200.h,
and reports the reference's error kinds for bad arguments.  Argument checks run
before any CUDA call, so these run without a GPU."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from burn_automata_b200 import _lib
from burn_automata_b200 import config as C
from burn_automata_b200 import kernels as K
from burn_automata_b200.config import GaussianDecodeConfig, GaussianDecodeMode, HashGridConfig
from tests.conftest import HAS_CUDA

HEADER = Path(__file__).resolve().parents[1] / "include" / "npa_b200.h"


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(npa_\w+)\s*\(", text, re.M)))


def test_library_exports_every_header_symbol(npa_lib):
    names = header_functions()
    assert len(names) >= 30
    for name in names:
        assert hasattr(npa_lib, name), name
    bound = {n for n, _, _ in _lib.SIGNATURES}
    assert set(names) == bound


def test_abi_version(npa_lib):
    assert npa_lib.npa_abi_version() == 1
    assert npa_lib.npa_status_string(7) == b"output shape"


def test_grid_validation_errors_match_reference_order():
    # config.rs:65-84: dim, then eps, then per-axis size / power of two
    with pytest.raises(C.InvalidDim):
        K.build_hashgrid(np.zeros((1, 4)), 1, 1, HashGridConfig.growing_2d().with_(dim=4))
    with pytest.raises(C.InvalidEps):
        K.build_hashgrid(np.zeros((1, 4)), 1, 1, HashGridConfig.growing_2d().with_(eps=0.0))
    with pytest.raises(C.InvalidEps):
        K.build_hashgrid(np.zeros((1, 4)), 1, 1, HashGridConfig.growing_2d().with_(eps=float("nan")))
    with pytest.raises(C.InvalidGridSize):
        K.build_hashgrid(np.zeros((1, 4)), 1, 1, HashGridConfig.growing_2d().with_(grid_size=(0, 4, 1)))
    with pytest.raises(C.ParticleModeRequiresPowerOfTwo):
        K.build_hashgrid(np.zeros((1, 4)), 1, 1, HashGridConfig.growing_2d().with_(grid_size=(6, 4, 1)))
    # Grid mode accepts non power-of-two sizes; the shape check fires next.
    with pytest.raises(C.PositionShape):
        K.build_hashgrid(np.zeros((3, 4)), 1, 2, HashGridConfig.texture_2d())


def test_shape_errors():
    cfg = HashGridConfig.growing_2d()
    with pytest.raises(C.PositionShape):
        K.perceive(np.zeros((3, 4)), np.zeros(4), 1, 2, 2, cfg, True, True)
    with pytest.raises(C.StateShape):
        K.perceive(np.zeros((2, 4)), np.zeros(5), 1, 2, 2, cfg, True, True)
    with pytest.raises(C.OutputShape):
        K.euler_step(np.zeros((2, 4)), np.zeros(4), np.zeros((1, 4)), np.zeros(4), 1, 2, 2, cfg,
                     1.0)
    with pytest.raises(C.OutputShape):
        K.euler_step(np.zeros((2, 4)), np.zeros(4), np.zeros((2, 4)), np.zeros(3), 1, 2, 2, cfg,
                     1.0)


def test_output_shape_on_caller_buffers(npa_lib):
    g = _lib.grid_c(HashGridConfig.growing_2d())
    pos = np.zeros((2, 4), np.float32)
    off = np.zeros(10, np.uint32)  # needs 4097
    perm = np.zeros(2, np.uint32)
    st = npa_lib.npa_build_hashgrid(ctypes.byref(g), pos.ctypes.data_as(_lib.f32p), 2, 1, 2,
                                    off.ctypes.data_as(_lib.u32p), off.shape[0],
                                    perm.ctypes.data_as(_lib.u32p),
                                    perm.ctypes.data_as(_lib.u32p), 2)
    assert st == 7


def test_decode_layout_errors_instead_of_panics():
    with pytest.raises(C.StateShape):
        K.decode_gaussians_3d_records(np.zeros((1, 4)), np.zeros(4), 4,
                                      GaussianDecodeConfig(mode=GaussianDecodeMode.GaussianSh0LearnedScale))
    with pytest.raises(C.StateShape):
        K.decode_gaussians_3d_records(np.zeros((1, 4)), np.zeros(10), 10,
                                      GaussianDecodeConfig(mode=GaussianDecodeMode.GaussianSh0Oriented))
    with pytest.raises(C.InvalidArgument):
        K.decode_gaussians_3d_records(np.zeros((1, 4)), np.zeros(8), 8,
                                      GaussianDecodeConfig(min_scale=1.0, max_scale=0.5))


def test_model_weight_validation():
    from burn_automata_b200.model import NpaModel, NpaWeights

    cfg = C.NpaConfig.growing_2d()
    w = NpaWeights.zeros(cfg)
    w.w1 = w.w1[:-1]
    with pytest.raises(C.InvalidModel):
        NpaModel(cfg, w)
    with pytest.raises(C.InvalidModel):
        NpaModel(cfg.with_(spatial_dims=4), NpaWeights.zeros(cfg))


@pytest.mark.skipif(HAS_CUDA, reason="checks the no-device path")
def test_valid_call_without_device_reports_no_device():
    with pytest.raises(C.NoDevice):
        K.build_hashgrid(np.zeros((2, 4)), 1, 2, HashGridConfig.growing_2d())


def test_errors_carry_the_reference_payloads():
    """KernelError's fields (config.rs:102-137) come across the C ABI through
    npa_last_error_detail, so a binding can rebuild the exact variant."""
    with pytest.raises(C.InvalidDim) as e:
        K.build_hashgrid(np.zeros((1, 4)), 1, 1, HashGridConfig.growing_2d().with_(dim=4))
    assert e.value.dim == 4
    with pytest.raises(C.InvalidEps) as e:
        K.build_hashgrid(np.zeros((1, 4)), 1, 1, HashGridConfig.growing_2d().with_(eps=-0.5))
    assert e.value.eps == -0.5
    with pytest.raises(C.ParticleModeRequiresPowerOfTwo) as e:
        K.build_hashgrid(np.zeros((1, 4)), 1, 1, HashGridConfig.growing_2d().with_(grid_size=(64, 6, 1)))
    assert (e.value.axis, e.value.value) == (1, 6)
    cfg = HashGridConfig.growing_2d()
    with pytest.raises(C.PositionShape) as e:
        K.perceive(np.zeros((3, 4)), np.zeros(4), 1, 2, 2, cfg, True, True)
    assert (e.value.positions, e.value.expected) == (3, 2)
    with pytest.raises(C.StateShape) as e:
        K.perceive(np.zeros((2, 4)), np.zeros(5), 1, 2, 2, cfg, True, True)
    assert (e.value.states, e.value.expected) == (5, 4)
    with pytest.raises(C.OutputShape) as e:
        K.euler_step(np.zeros((2, 4)), np.zeros(4), np.zeros((1, 4)), np.zeros(4), 1, 2, 2, cfg,
                     1.0)
    assert (e.value.actual, e.value.expected) == (1, 2)


def test_noalloc_hashgrid_validates_like_the_workspace_entry_point(npa_lib):
    """Bad arguments get the same status from npa_dev_build_hashgrid_noalloc
    as from npa_dev_build_hashgrid (checked before any CUDA call); only sizes
    above the fixed array's limit add NPA_ERR_UNSUPPORTED."""
    cases = [
        (HashGridConfig.growing_2d().with_(dim=5), 1, 10),
        (HashGridConfig.growing_2d().with_(eps=0.0), 1, 10),
        (HashGridConfig.growing_2d().with_(grid_size=(6, 64, 1)), 1, 10),
        (HashGridConfig.growing_2d(), -1, 10),
        (HashGridConfig.growing_2d(), 2, -3),
        (HashGridConfig.growing_2d().with_(grid_size=(1 << 15, 1 << 15, 1)), 8, 1),
    ]
    for cfg, batch, n in cases:
        g = _lib.grid_c(cfg)
        a = npa_lib.npa_dev_build_hashgrid(ctypes.byref(g), None, batch, n, None, None, None,
                                           None, 0, None)
        b = npa_lib.npa_dev_build_hashgrid_noalloc(ctypes.byref(g), None, batch, n, None, None,
                                                   None, None)
        assert a == b and a != 0, (cfg, batch, n, a, b)
    g = _lib.grid_c(HashGridConfig.growing_2d())
    assert npa_lib.npa_dev_build_hashgrid_noalloc(ctypes.byref(g), None, 3, 1 << 16, None, None,
                                                  None, None) == 24
