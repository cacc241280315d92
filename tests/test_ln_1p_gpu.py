"""f32::ln_1p on the device equals the host C library's log1pf bit for bit.

The reference's log-normalisation (crates/burn_automata_kernels/src/reference/
normalize.rs:60-69) calls f32::ln_1p, i.e. the host libm's log1pf, which is
not correctly rounded; the device reproduces it (csrc/host_log1p.cu).  Checked
here through the C ABI (npa_dev_ln_1p) against the host's own log1pf on every
float in [1, 2) -- where one in eight results differs from the correctly
rounded value -- every float in [1e-6, 2e-6), a stride over the whole
tabulated range [1e-6, FLT_MAX], and the range ends.
"""

import ctypes

import numpy as np
import pytest

from burn_automata_b200 import _lib

pytestmark = pytest.mark.gpu


def float_range(lo, hi, stride=1):
    a = np.array([lo], np.float32).view(np.uint32)[0]
    b = np.array([hi], np.float32).view(np.uint32)[0]
    return np.arange(a, b, stride, dtype=np.uint32).view(np.float32)


def device_ln_1p(torch, x):
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev)
    out = torch.empty_like(dx)
    _lib.check(L.npa_dev_ln_1p(dx.data_ptr(), dx.numel(), out.data_ptr(),
                               torch.cuda.current_stream(dev).cuda_stream), "npa_dev_ln_1p")
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_device_ln_1p_is_the_host_log1pf(oracle_mod):
    torch = pytest.importorskip("torch")
    inputs = np.concatenate([
        float_range(1.0, 2.0),
        float_range(1e-6, 2e-6),
        float_range(1e-6, np.finfo(np.float32).max, 97),
        np.array([1e-6, np.finfo(np.float32).max, np.inf], np.float32),
    ])
    got = device_ln_1p(torch, inputs)
    want = oracle_mod.ln_1p(inputs)
    bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, (f"{bad.size} of {inputs.size} differ, first inputs "
                           f"{inputs[bad[:5]].tolist()}")
    # the case is not trivial: the correctly rounded value differs on many of them
    cr = np.log1p(inputs[:1 << 23].astype(np.float64)).astype(np.float32)
    assert np.count_nonzero(cr != want[:1 << 23]) > 500_000
