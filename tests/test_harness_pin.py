"""The oracle and the CUDA path against the reference's own numeric oracle.

``tests/golden/harness_outputs.npz`` holds what the reference harness's
``reference_output`` (``experiments/source/harness/run.py:1031-1099``, plain
PyTorch) returned on this repository's seeded inputs for the 33 kernels of
the harness's table and for the suite entries it covers (saxpy, relu, dot,
l2_norm_sq), at n = 4096, 65541 and 2^20 + 3; ``make_harness_outputs.py``
beside it made the file by importing that function from the reference.

The bar is the harness's own: ``torch.testing.assert_close`` at the kernel's
``verification_rtol`` / ``verification_atol`` (1e-4 / 1e-5 for all of them,
``run.py:1016-1017``), i.e. |actual - expected| <= atol + rtol * |expected|
elementwise, no NaN on either side.  The reference's PyTorch expressions
round differently from the generated kernels (no fmaf, fp32 sums), so this
pin is a tolerance pin; the bit-exact bar against the oracle is in
test_gpu_parity.py, test_workloads.py and the other GPU suites.

* CPU: the oracle meets the bar for every case and size (and a mistake
  planted in the oracle's inputs fails it);
* GPU: the suite package and the default build of the harness kernels meet
  it through the C ABI.
"""

import json
import os

import numpy as np
import pytest

from loom_b200 import workloads

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
META = json.load(open(os.path.join(GOLDEN, "harness_outputs.json")))
ARRAYS = dict(np.load(os.path.join(GOLDEN, "harness_outputs.npz")))
WL_DIR = os.path.join(GOLDEN, "sources", "workloads")
WL_TABLE = {w["name"]: w for w in json.load(open(os.path.join(WL_DIR, "workloads.json")))}


def case_inputs(case: dict, n: int):
    group, name = case["case"].split("/", 1)
    if group == "harness":
        w = WL_TABLE[name]
        return workloads.harness_inputs(w["tensor_inputs"], w["scalar_args"], n)
    return workloads.entry_inputs(name, n)


def harness_close(actual, expected, rtol, atol):
    """torch.testing.assert_close's float32 criterion; returns the largest
    |actual - expected| / (atol + rtol * |expected|) (<= 1 passes)."""
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert actual.shape == expected.shape
    assert not np.isnan(actual).any() and not np.isnan(expected).any()
    ratio = np.abs(actual - expected) / (atol + rtol * np.abs(expected))
    return float(ratio.max()) if ratio.size else 0.0


def stored(case: dict, n: int, full):
    """The elements of a full result that the fixture stored."""
    if case["result_kind"] == "scalar":
        return np.asarray([full], np.float32).reshape(1)
    return np.asarray(full, np.float32)[ARRAYS[f"indices/{n}"]]


def test_fixture_covers_the_harness_table_and_suite():
    names = [c["case"] for c in META["cases"]]
    assert len(names) == 37
    assert sorted(n for n in names if n.startswith("harness/")) == \
        sorted("harness/" + k for k in WL_TABLE)
    assert META["sizes"] == [4096, 65541, (1 << 20) + 3]
    assert all((c["rtol"], c["atol"]) == (1e-4, 1e-5) for c in META["cases"])


@pytest.fixture(scope="module")
def harness_oracle(suite_programs):
    from oracle.loom_oracle import Oracle
    from loom_b200 import tensor_ir as TI
    from test_workloads import _programs
    objs = [TI.program_to_json(p) for p in _programs().values()]
    return Oracle(objs, name="workloads_harness_pin"), Oracle(suite_programs, name="b200_suite")


def test_oracle_meets_the_reference_harness_oracle(harness_oracle):
    wl_oracle, suite_oracle = harness_oracle
    worst = {}
    for case in META["cases"]:
        group = case["case"].split("/", 1)[0]
        orc = wl_oracle if group == "harness" else suite_oracle
        for n in META["sizes"]:
            got = stored(case, n, orc.run(case["entry"], case_inputs(case, n)))
            r = harness_close(got, ARRAYS[f"{case['case']}/{n}"], case["rtol"], case["atol"])
            assert r <= 1.0, (case["case"], n, r)
            worst[case["case"]] = max(worst.get(case["case"], 0.0), r)
    # every case was compared; the oracle sits far inside the tolerance (the
    # largest ratio when the fixture was made was 9e-3, saxpy's unfused
    # a*x + y against the oracle's fmaf)
    assert len(worst) == 37
    assert max(worst.values()) < 0.05, max(worst.items(), key=lambda kv: kv[1])


def test_a_mistake_planted_in_the_oracle_fails_the_pin(harness_oracle):
    _, suite_oracle = harness_oracle
    case = next(c for c in META["cases"] if c["case"] == "suite/saxpy")
    n = 4096
    inp = case_inputs(case, n)
    inp["a"] = 2.5 * (1 + 1e-3)            # a scalar off by 0.1%
    got = stored(case, n, suite_oracle.run("saxpy", inp))
    assert harness_close(got, ARRAYS[f"suite/saxpy/{n}"], case["rtol"], case["atol"]) > 1.0
    case = next(c for c in META["cases"] if c["case"] == "suite/dot")
    inp = case_inputs(case, n)
    inp["x"] = inp["x"].copy()
    inp["x"][17] += np.float32(0.5)        # one input element changed
    got = stored(case, n, suite_oracle.run("dot", inp))
    assert harness_close(got, ARRAYS[f"suite/dot/{n}"], case["rtol"], case["atol"]) > 1.0


@pytest.mark.gpu
def test_cuda_path_meets_the_reference_harness_oracle(suite_pkg):
    import torch

    from loom_b200.build import build_project
    from loom_b200.loader import Package
    from test_gpu_parity import to_device
    from test_workloads import _programs

    wl_pkg = Package(build_project(WL_DIR, name="workloads"))
    progs = _programs()
    worst = 0.0
    for case in META["cases"]:
        group, name = case["case"].split("/", 1)
        pkg = wl_pkg if group == "harness" else suite_pkg
        entry = progs[name].entry_name if group == "harness" else name
        for n in META["sizes"]:
            inp = case_inputs(case, n)
            dev = {k: (to_device(v, 1) if isinstance(v, np.ndarray) else v)
                   for k, v in inp.items()}
            out = to_device(np.zeros(n, np.float32), 1) \
                if case["result_kind"] == "tensor" else None
            res = pkg[entry](out=out, **dev)
            torch.cuda.synchronize()
            full = res.cpu().numpy()
            got = stored(case, n, full if case["result_kind"] == "tensor" else float(full[0]))
            r = harness_close(got, ARRAYS[f"{case['case']}/{n}"], case["rtol"], case["atol"])
            assert r <= 1.0, (case["case"], n, r)
            worst = max(worst, r)
    assert worst < 0.05, worst
