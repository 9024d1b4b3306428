"""Broader bodies through the whole pipeline (Python source -> front end ->
B200 package -> CUDA) against the oracle: helper functions, clamps, soft
thresholds, sqrt, exp/log, division, select, negation, a tail if statement,
qualified primitives, unary plus and equality, maxes over maps and
multi-node chains (tests/golden/sources/cases/frontend_cases.py).

The project is packaged four times: with the reference's default flags;
with the flags that change how map bodies are rendered (soft-threshold and
predicated-select rewrites, the `if` clamp form, `__fdividef` for ratio
bodies; loom_b200.build.RENDER_FLAGS); with the TensorIR fusion passes; and
with the whole flag set of the reference harness's tuned CUDA profile
(loom_b200.build.CUDA_FIXED_FLAGS: the scalar and TensorIR rewrites too),
each checked against the oracle built from the same rewritten programs and
flags.

Bar: maps and max bit-exact, except `ratio_exp`, whose expf/logf are CUDA's
(up to 2 ulp / 1 ulp from the correctly rounded value; with the flags also
__fdividef, 2 ulp) against the host's libm and IEEE division, so it is
compared to a relative 1e-6 (about 8 ulp); sums as in test_gpu_parity:
1e-6 * max(1, log2 n) * max(|ref|, sqrt(sum v_i^2)).
"""

import math
import os

import numpy as np
import pytest
import torch

from loom_b200 import tensor_ir as TI
from loom_b200.build import CUDA_FIXED_FLAGS, FUSION_FLAGS, RENDER_FLAGS, build_project
from loom_b200.frontend import python_programs
from loom_b200.loader import Package

from test_gpu_parity import assert_bits, to_device

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = os.path.join(HERE, "golden", "sources", "cases")
SCALARS = {"lo": -0.5, "hi": 0.75, "s": 1.5, "a": 0.3, "t": 0.25, "k": 0.4}
SCALARS_BY_ENTRY = {"scaled_chain": {"a": 1.25}}


@pytest.fixture(scope="module", params=["default", "render_flags", "fusion", "cuda_fixed"])
def cases(request):
    from oracle.loom_oracle import Oracle
    src = os.path.join(CASES, "frontend_cases.py")
    if request.param == "default":
        progs = python_programs(src)
        pkg = Package(build_project(CASES))
        oracle = Oracle([TI.program_to_json(p) for p in progs], name="frontend_cases")
    elif request.param == "render_flags":
        progs = python_programs(src)
        pkg = Package(build_project(CASES, enabled=RENDER_FLAGS, name="frontend_cases_flags"))
        oracle = Oracle([TI.program_to_json(p) for p in progs], name="frontend_cases_flags",
                        enabled=RENDER_FLAGS)
    elif request.param == "fusion":
        # the reference's TensorIR fusion passes ahead of the backend: the
        # oracle evaluates the same fused programs
        progs = python_programs(src, FUSION_FLAGS)
        pkg = Package(build_project(CASES, enabled=FUSION_FLAGS, name="frontend_cases_fused"))
        oracle = Oracle([TI.program_to_json(p) for p in progs], name="frontend_cases_fused",
                        enabled=FUSION_FLAGS)
    else:
        progs = python_programs(src, CUDA_FIXED_FLAGS)
        pkg = Package(build_project(CASES, enabled=CUDA_FIXED_FLAGS,
                                    name="frontend_cases_cuda_fixed"))
        oracle = Oracle([TI.program_to_json(p) for p in progs],
                        name="frontend_cases_cuda_fixed", enabled=CUDA_FIXED_FLAGS)
    return pkg, oracle, {p.entry_name: p for p in progs}


def _values(entry, inp):
    x = inp.get("x").astype(np.float64)
    y = inp["y"].astype(np.float64) if "y" in inp else None
    if entry == "nested_helpers":
        return x * y
    if entry == "hypot_sum":
        return np.sqrt(x * x + y * y) + np.maximum(x, y) - np.minimum(x, 0.0)
    if entry == "scaled_chain":
        d = inp["a"] * x - y
        return d * d / (inp["w"].astype(np.float64) ** 2 + 1.0)
    if entry == "let_chain_sum":
        u = x * inp["a"]
        return u * (u - 1.0)
    raise KeyError(entry)


@pytest.mark.parametrize("n, offset", [(4099, 0), ((1 << 20) + 3, 1), (7, 2)])
def test_bodies_match_oracle(cases, n, offset):
    pkg, oracle, progs = cases
    rng = np.random.default_rng(n)
    for entry, prog in progs.items():
        inp = {}
        for p in prog.params:
            if isinstance(p, TI.TensorParam):
                inp[p.name] = rng.uniform(-2.0, 2.0, n).astype(np.float32)
            else:
                inp[p.name] = SCALARS_BY_ENTRY.get(entry, {}).get(p.name, SCALARS[p.name])
        ref = oracle.run(entry, inp)
        dev = {k: (to_device(v, offset) if isinstance(v, np.ndarray) else v)
               for k, v in inp.items()}
        out = None
        if prog.result_kind == "tensor":
            out = to_device(np.zeros(n, np.float32), offset)
        got = pkg[entry](out=out, **dev)
        torch.cuda.synchronize()
        got = got.cpu().numpy()
        if prog.result_kind == "tensor":
            if entry == "ratio_exp":
                np.testing.assert_allclose(got, ref, rtol=1e-6, atol=0)
            else:
                assert_bits(got, ref)
        elif prog.node(prog.result.id).kind == "max":
            assert float(got[0]) == float(np.float32(ref)), entry
        else:
            v = _values(entry, inp)
            tol = 1e-6 * max(1.0, math.log2(n)) * max(abs(ref), math.sqrt(float(np.sum(v * v))))
            assert abs(float(got[0]) - ref) <= tol, (entry, float(got[0]), ref, tol)
