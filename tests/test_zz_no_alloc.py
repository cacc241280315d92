"""The allocation-free hashgrid entry point (npa_dev_build_hashgrid_noalloc).

It serves callers that cannot allocate device memory themselves -- a host that
only holds buffers owned by another framework, or a loop that must not call
cudaMalloc because it synchronises the device -- by keeping the sort scratch in
a fixed array inside the library.  Here it is called through the C ABI and
its outputs are compared with the workspace-based entry point
(npa_dev_build_hashgrid), bit for bit as every hashgrid test, on two calls in a
row with different inputs (the shared array keeps the previous call's
contents, which must not leak into the next result).
"""

import ctypes

import numpy as np
import pytest

from burn_automata_b200 import _lib, workloads
from burn_automata_b200.config import HashGridConfig

pytestmark = pytest.mark.gpu

MAX_PARTICLES = 1 << 17


def run_both(torch, grid, positions, batch, n):
    L = _lib.lib()
    g = _lib.grid_c(grid)
    dev = torch.device("cuda", 0)
    pos = torch.from_numpy(np.ascontiguousarray(positions, np.float32)).to(dev)
    bins = batch * grid.cell_count() + 1
    outs = []
    for noalloc in (False, True):
        off = torch.full((bins,), 0xDEAD, dtype=torch.int32, device=dev)
        perm = torch.full((max(batch * n, 1),), -1, dtype=torch.int32, device=dev)
        inv = torch.full((max(batch * n, 1),), -1, dtype=torch.int32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        if noalloc:
            st = L.npa_dev_build_hashgrid_noalloc(ctypes.byref(g), pos.data_ptr(), batch, n,
                                                  off.data_ptr(), perm.data_ptr(),
                                                  inv.data_ptr(), stream)
        else:
            need = ctypes.c_size_t(0)
            _lib.check(L.npa_dev_hashgrid_workspace_size(ctypes.byref(g), batch, n,
                                                         ctypes.byref(need)))
            ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
            st = L.npa_dev_build_hashgrid(ctypes.byref(g), pos.data_ptr(), batch, n,
                                          off.data_ptr(), perm.data_ptr(), inv.data_ptr(),
                                          ws.data_ptr(), need.value, stream)
        _lib.check(st, "noalloc" if noalloc else "workspace")
        torch.cuda.synchronize()
        outs.append((off.cpu().numpy(), perm.cpu().numpy(), inv.cpu().numpy()))
    return outs


def test_noalloc_hashgrid_matches_workspace_entry_point_twice():
    """Batches of small rollouts: the per-rollout shared-memory sort, which
    takes only the sorted-record slices of the fixed array."""
    torch = pytest.importorskip("torch")
    first = workloads.make("cfg2", batch=32, steps=1)          # 131,072 particles: the limit
    second = workloads.make("cfg0", n=3000, steps=1, seed=5)  # smaller, different grid use
    for w in (first, second):
        a, b = run_both(torch, w.grid, w.positions, w.batch, w.n)
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)
    assert first.batch * first.n == MAX_PARTICLES


def test_noalloc_hashgrid_device_wide_sort_matches_twice():
    """Shapes that take the device-wide radix sort, whose key / value
    ping-pong buffers and tile histograms are carved from the fixed array:
    one 16,384-particle 3D rollout, then 2 x 65,536 particles on cfg1's
    262,144-cell grid (131,072 particles, the largest carve)."""
    torch = pytest.importorskip("torch")
    first = workloads.make("cfg3", steps=1)
    second = workloads.make("cfg1", batch=2, n=1 << 16, steps=1, seed=7)
    for w in (first, second):
        a, b = run_both(torch, w.grid, w.positions, w.batch, w.n)
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)
    assert second.batch * second.n == MAX_PARTICLES


def test_noalloc_hashgrid_rejects_sizes_beyond_its_limit():
    torch = pytest.importorskip("torch")
    L = _lib.lib()
    g = _lib.grid_c(HashGridConfig.growing_2d())
    dev = torch.device("cuda", 0)
    n = MAX_PARTICLES + 1
    pos = torch.zeros((n, 4), dtype=torch.float32, device=dev)
    off = torch.zeros(4097, dtype=torch.int32, device=dev)
    perm = torch.zeros(n, dtype=torch.int32, device=dev)
    st = L.npa_dev_build_hashgrid_noalloc(ctypes.byref(g), pos.data_ptr(), 1, n, off.data_ptr(),
                                          perm.data_ptr(), perm.data_ptr(), None)
    assert st == 24  # NPA_ERR_UNSUPPORTED
    assert b"131072" in L.npa_last_error_message()
