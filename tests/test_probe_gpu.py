"""The FP32 pipe probe behind `bench.py --fp32-ceiling` runs and reports a
rate within the pipe's limit (148 SMs x 128 lanes x the maximum clock)."""

import ctypes

import pytest

pytestmark = pytest.mark.gpu


def test_fp32_tile_probe_rate_is_plausible():
    import burn_automata_b200 as ba

    lib = ba.load_library()
    rate, ms = ctypes.c_double(0.0), ctypes.c_double(0.0)
    assert lib.npa_debug_fp32_tile_rate(50, ctypes.byref(rate), ctypes.byref(ms)) == 0
    assert ms.value > 0.0
    peak = 148 * 128 * 1965e6
    assert 0.05 * peak < rate.value <= 1.05 * peak
    assert lib.npa_debug_fp32_tile_rate(0, ctypes.byref(rate), ctypes.byref(ms)) != 0
