"""Pinning the CPU oracle (CPU only).

1. The reference's own runtime expectations (test/python/test_package.py:66-131,
   test/python/test_cli.py:374-407): saxpy at n=4096, a=2.5 against a*x+y and
   dot against sum(x*y), rtol 1e-4 / atol 1e-5.
2. Exact-rational known answers for the rendering semantics: fmaf rounds
   once, relu/max follow CUDA's fmaxf, the clamp is exact, sums are the exact
   sum of the fp32 per-element values.
"""

import math
from fractions import Fraction

import numpy as np
import pytest

from loom_b200 import workloads
from oracle import loom_oracle as O


def round_f32(q: Fraction) -> np.float32:
    """Exact round-to-nearest-even of a rational to float32."""
    d = np.float32(float(q))
    cands = {float(d), float(np.nextafter(d, np.float32(-np.inf))),
             float(np.nextafter(d, np.float32(np.inf)))}

    def key(c):
        f = np.float32(c)
        return (abs(Fraction(c) - q), int(f.view(np.uint32)) & 1)

    return np.float32(min(cands, key=key))


def exact_fmaf(a, b, c) -> np.float32:
    return round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def test_reference_saxpy_expectation(oracle):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(4096).astype(np.float32)
    y = rng.standard_normal(4096).astype(np.float32)
    out = oracle.run("saxpy", {"a": 2.5, "x": x, "y": y})
    np.testing.assert_allclose(out, np.float32(2.5) * x + y, rtol=1e-4, atol=1e-5)


def test_reference_dot_expectation(oracle):
    rng = np.random.default_rng(1)
    x = rng.standard_normal(4096).astype(np.float32)
    y = rng.standard_normal(4096).astype(np.float32)
    s = oracle.run("dot", {"x": x, "y": y})
    np.testing.assert_allclose(s, float(np.sum(x * y, dtype=np.float32)), rtol=1e-4, atol=1e-5)


def test_saxpy_single_rounding_fmaf_exact(oracle):
    inp = workloads.entry_inputs("saxpy", 3000)
    x, y = inp["x"], inp["y"]
    # add cases where a*x + y differs between fused and unfused rounding
    x = np.concatenate([x, np.float32([1 + 2 ** -23, 1 - 2 ** -24, 3.0, 1e-30])])
    y = np.concatenate([y, np.float32([-1.0, 0.5, -7.5, 1.0])])
    out = oracle.run("saxpy", {"a": 2.5, "x": x, "y": y})
    expect = np.array([exact_fmaf(2.5, a, b) for a, b in zip(x, y)], dtype=np.float32)
    assert np.array_equal(out.view(np.uint32), expect.view(np.uint32))


def test_fused_differs_from_unfused_somewhere(oracle):
    # the oracle must not silently compute round(round(a*x)+y)
    inp = workloads.entry_inputs("saxpy", 1 << 16)
    out = oracle.run("saxpy", {"a": 2.5, "x": inp["x"], "y": inp["y"]})
    unfused = np.float32(2.5) * inp["x"] + inp["y"]
    assert np.any(out != unfused)


def test_relu_semantics(oracle):
    x = np.float32([-1.0, -0.0, 0.0, 1e-45, -1e-45, 2.0, np.inf, -np.inf, np.nan, 3.5])
    out = oracle.run("relu", {"x": x})
    expect = np.float32([0.0, 0.0, 0.0, 1e-45, 0.0, 2.0, np.inf, 0.0, 0.0, 3.5])
    assert np.array_equal(out.view(np.uint32), expect.view(np.uint32))  # +0.0 for -0.0


def test_affine_relu_exact(oracle):
    inp = workloads.entry_inputs("affine_relu", 2000)
    out = oracle.run("affine_relu", inp)
    z = np.array([exact_fmaf(0.75, a, b) for a, b in zip(inp["x"], inp["y"])], dtype=np.float32)
    expect = np.where(z > 0, z, np.float32(0.0)).astype(np.float32)
    assert np.array_equal(out.view(np.uint32), expect.view(np.uint32))


@pytest.mark.parametrize("entry", ["dot", "l2_norm_sq", "pipeline_sum"])
def test_sums_are_exact_sums_of_fp32_values(oracle, entry):
    inp = workloads.entry_inputs(entry, 10007)
    got = oracle.run(entry, inp)
    if entry == "dot":
        v = inp["x"] * inp["y"]
    elif entry == "l2_norm_sq":
        v = inp["x"] * inp["x"]
    else:
        z = np.array([exact_fmaf(0.75, a, b) for a, b in zip(inp["x"], inp["y"])],
                     dtype=np.float32)
        v = np.where(z > 0, z, np.float32(0.0)).astype(np.float32) * inp["w"]
    expect = math.fsum(float(t) for t in v.astype(np.float32))
    assert got == pytest.approx(expect, rel=1e-13, abs=1e-300)


def test_max_semantics(oracle):
    x = workloads.entry_inputs("max_value", 5000)["x"]
    assert oracle.run("max_value", {"x": x}) == float(np.max(x))
    with_nan = x.copy()
    with_nan[::7] = np.nan
    assert oracle.run("max_value", {"x": with_nan}) == float(np.nanmax(with_nan))
    assert oracle.run("max_value", {"x": np.float32([np.nan, np.nan])}) == -math.inf
    zeros = np.float32([-0.0, 0.0, -0.0])
    assert math.copysign(1.0, oracle.run("max_value", {"x": zeros})) == 1.0


def test_thread_count_does_not_change_results(oracle):
    inp = workloads.entry_inputs("pipeline_sum", 1 << 15)
    a = oracle.run("pipeline_sum", inp, threads=1)
    b = oracle.run("pipeline_sum", inp, threads=7)
    assert a == pytest.approx(b, rel=1e-15)
    m1 = oracle.run("affine_relu", inp, threads=1)
    m2 = oracle.run("affine_relu", inp, threads=5)
    assert np.array_equal(m1.view(np.uint32), m2.view(np.uint32))
