"""The reference-style GPU baseline (baseline/loom_reference_style.cu): the
kernels the reference's CUDA backend generates for the suite entries under
its "none" and "cuda" profiles, restated by hand and timed beside the
product by bench.py.

CPU: the library builds for sm_100a, exports every entry of both profiles,
and sizes its workspace by the reference's formula (cuda_backend.ml:1674-1715).
GPU: every entry against the oracle on seeded inputs -- maps and max
bit-exact, sums within the reference's own tolerance (rtol 1e-4,
test/python/test_package.py:100,131) since the baseline accumulates in fp32,
with float atomics in the cuda profile.
"""

import math

import numpy as np
import pytest

from baseline import reference_style as rs
from loom_b200 import workloads


def _align(v, a=256):
    return (v + a - 1) // a * a


def _block_count(n, block=256):
    return max(1, min(-(-n // block), 4096))


@pytest.fixture(scope="module")
def lib():
    rs.build()
    return rs.ReferenceStyle()


def test_exports_every_entry_of_both_profiles(lib):
    for profile in rs.PROFILES:
        for entry in rs.PARAMS:
            assert (profile, entry) in lib.fns


@pytest.mark.parametrize("n", [0, 1, 4096, 4097, 1 << 20, (1 << 28) + 3])
def test_workspace_sizes_follow_the_reference_formula(lib, n):
    def tree(n, temps):
        if n <= 0:
            return 0
        b = 0
        for _ in range(temps):
            b = _align(b) + 4 * n
        parts = 4 * _block_count(n)
        return _align(_align(b) + parts) + parts

    want = {
        ("none", "saxpy"): 0, ("none", "relu"): 0, ("none", "affine_relu"): 0,
        ("none", "dot"): tree(n, 1), ("none", "l2_norm_sq"): tree(n, 1),
        ("none", "max_value"): tree(n, 0), ("none", "pipeline_sum"): tree(n, 2),
        ("cuda", "saxpy"): 0, ("cuda", "relu"): 0, ("cuda", "affine_relu"): 0,
        ("cuda", "dot"): 0, ("cuda", "l2_norm_sq"): 0, ("cuda", "pipeline_sum"): 0,
        ("cuda", "max_value"): tree(n, 0),
    }
    for (profile, entry), size in want.items():
        assert lib.workspace_size(profile, entry, n) == size, (profile, entry, n)


def _sum_scale(entry, inp):
    if entry == "dot":
        v = inp["x"].astype(np.float64) * inp["y"]
    elif entry == "l2_norm_sq":
        v = inp["x"].astype(np.float64) ** 2
    else:
        z = np.maximum(0.75 * inp["x"].astype(np.float64) + inp["y"], 0.0)
        v = z * inp["w"]
    return math.sqrt(float(np.sum(v * v)))


@pytest.mark.gpu
@pytest.mark.parametrize("profile", rs.PROFILES)
@pytest.mark.parametrize("n", [1, 5, 4096, 4099, (1 << 20) + 3])
def test_reference_style_matches_oracle(lib, oracle, profile, n):
    import torch
    for entry in rs.PARAMS:
        inp = workloads.entry_inputs(entry, n, seed_offset=17)
        dev = {k: (torch.from_numpy(v).cuda() if isinstance(v, np.ndarray) else v)
               for k, v in inp.items()}
        out = torch.empty(n if entry in rs.MAPS else 1, device="cuda")
        size = lib.workspace_size(profile, entry, n)
        ws = torch.empty(size, dtype=torch.uint8, device="cuda") if size else None
        assert lib.bind(profile, entry, n, out, ws, **dev)() == 0, (profile, entry)
        torch.cuda.synchronize()
        ref = oracle.run(entry, inp)
        if entry in rs.MAPS:
            got = out.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (profile, entry)
        elif entry == "max_value":
            assert float(out.cpu()[0]) == float(np.float32(ref)), (profile, entry)
        else:
            got = float(out.cpu()[0])
            tol = 1e-4 * max(abs(ref), _sum_scale(entry, inp))
            assert abs(got - ref) <= tol, (profile, entry, n, got, ref)


@pytest.mark.gpu
def test_reference_style_status_codes(lib):
    import torch
    x = torch.zeros(8, device="cuda")
    out = torch.zeros(8, device="cuda")
    for profile in rs.PROFILES:
        assert lib.bind(profile, "relu", -1, out, None, x=x)() == 1
        assert lib.bind(profile, "dot", 0, out, None, x=x, y=x)() == 1
        assert lib.bind(profile, "relu", 0, out, None, x=x)() == 0
    assert lib.bind("none", "dot", 8, out, None, x=x, y=x)() == 2   # needs a workspace
