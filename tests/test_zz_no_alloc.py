"""loom_kernels_dot_noalloc: the dot reduction for callers that cannot give
the library device memory -- a framework that owns the GPU's memory through
its own allocator, a loop where cudaMalloc's possible device-wide
synchronisation is not allowed, a plain C caller with no workspace to pass.
The entry takes no workspace argument; its per-CTA partials live in a static
device array inside the library (4096 fp64 slots, 32 KiB).

Two calls in a row through the C ABI, each checked against the CPU oracle's
fp64 sum of the same fp32 products with the sum bar of the other tests,
|got - ref| <= 1e-6 * max(1, log2 n) * |ref|:

* n = 2^24 + 3 needs 8192 tiles, so the entry caps its grid at the array's
  4096 slots (each CTA walks two tiles) and fills every slot;
* n = 2^20 + 5 then runs a grid of 513 CTAs over the first call's leftovers:
  its finalize must read only the 513 partials this call wrote.  With the same
  grid as the workspace entry loom_kernels_dot, it must also give the same
  bits as that entry.

This file is named to be collected last.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from loom_b200 import workloads

pytestmark = pytest.mark.gpu

SLOTS = 4096
TILE = 2048          # elements per tile of a two-input reduction (256 threads x 2 float4)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _bind(pkg):
    fn = pkg.lib.loom_kernels_dot_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def test_noalloc_dot_matches_the_oracle_on_two_calls(suite_pkg, oracle):
    noalloc = _bind(suite_pkg)
    dot = suite_pkg["dot"]
    for call, n in enumerate([(1 << 24) + 3, (1 << 20) + 5]):
        tiles = -(-n // TILE)
        inp = workloads.entry_inputs("dot", n, seed_offset=900 + call)
        ref = oracle.run("dot", inp)
        x = torch.from_numpy(inp["x"]).cuda()
        y = torch.from_numpy(inp["y"]).cuda()
        out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        assert noalloc(_ptr(x), _ptr(y), n, _ptr(out), None) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        bar = 1e-6 * max(1.0, math.log2(n)) * abs(ref)
        assert abs(float(got[0]) - ref) <= bar, (call, n, float(got[0]), ref, bar)
        if tiles <= SLOTS:
            # same grid as the workspace entry: same bits
            assert 8 < tiles, tiles        # a grid that goes through the slots
            want = dot(x=x, y=y).cpu().numpy()
            assert got.view(np.uint32)[0] == want.view(np.uint32)[0], (call, got, want)
        else:
            assert call == 0


def test_noalloc_dot_rejects_bad_arguments(suite_pkg):
    noalloc = _bind(suite_pkg)
    x = torch.zeros(16, device="cuda")
    out = torch.empty(1, device="cuda")
    assert noalloc(_ptr(x), _ptr(x), 0, _ptr(out), None) == 1      # n <= 0
    assert noalloc(None, _ptr(x), 16, _ptr(out), None) == 1        # null input
    assert noalloc(_ptr(x), _ptr(x), 16, None, None) == 1          # null output
