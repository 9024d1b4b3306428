"""loom_kernels_dot_noalloc: the dot reduction for callers that cannot give
the library device memory (no workspace argument; the per-CTA partials live
in a static device array inside the library).

Checked through the C ABI against the regular workspace entry
loom_kernels_dot on two calls in a row -- the first is large enough that the
entry caps its grid at the array's 4096 slots, the second is smaller and runs
over the first call's leftovers in the shared array -- with
the tolerance the other sum tests use:
|noalloc - dot| <= 1e-6 * max(1, log2 n) * max(|dot|, sqrt(sum (x_i*y_i)^2)).

This file is named to be collected last.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from loom_b200 import workloads

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _bind(pkg):
    fn = pkg.lib.loom_kernels_dot_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def test_noalloc_dot_matches_workspace_entry_on_two_calls(suite_pkg):
    noalloc = _bind(suite_pkg)
    dot = suite_pkg["dot"]
    for call, n in enumerate([(1 << 24) + 3, 1001]):
        inp = workloads.entry_inputs("dot", n, seed_offset=900 + call)
        x = torch.from_numpy(inp["x"]).cuda()
        y = torch.from_numpy(inp["y"]).cuda()
        expected = float(dot(x=x, y=y).item())
        out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        assert noalloc(_ptr(x), _ptr(y), n, _ptr(out), None) == 0
        torch.cuda.synchronize()
        got = float(out.item())
        v = inp["x"].astype(np.float64) * inp["y"]
        tol = 1e-6 * max(1.0, math.log2(n)) * max(abs(expected), math.sqrt(float(np.sum(v * v))))
        assert abs(got - expected) <= tol, (call, n, got, expected, tol)


def test_noalloc_dot_rejects_bad_arguments(suite_pkg):
    noalloc = _bind(suite_pkg)
    x = torch.zeros(16, device="cuda")
    out = torch.empty(1, device="cuda")
    assert noalloc(_ptr(x), _ptr(x), 0, _ptr(out), None) == 1      # n <= 0
    assert noalloc(None, _ptr(x), 16, _ptr(out), None) == 1        # null input
    assert noalloc(_ptr(x), _ptr(x), 16, None, None) == 1          # null output
