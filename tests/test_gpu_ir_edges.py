"""TensorIR shapes that the reference produces (for instance under its
reduce-map-fusion flag, or for trivial entries) but the front end here does
not: a mapped dot reduction, a weighted mapped reduction over a map node and
a parameter with scalar captures, a producer used twice next to a dead node,
an identity entry, a plain sum over a parameter, a max over a map with a
double literal, one tensor bound to both inputs of a map2
(tests/golden/sources/ir/edge.tensor_ir.json).  CUDA results against the
oracle with the bar of test_gpu_parity."""

import json
import math
import os

import numpy as np
import pytest
import torch

from loom_b200.build import build_project
from loom_b200.loader import Package

from test_gpu_parity import assert_bits, to_device

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
IR_DIR = os.path.join(HERE, "golden", "sources", "ir")
SCALARS = {"scale": 1.5, "bias": -0.25}


@pytest.fixture(scope="module")
def edge():
    from oracle.loom_oracle import Oracle, load_programs
    progs = load_programs(os.path.join(IR_DIR, "edge.tensor_ir.json"))
    return Package(build_project(IR_DIR)), Oracle(progs, name="ir_edge_cases"), progs


def _mass(name, inp):
    x = inp["x"].astype(np.float64)
    if name == "mapped_dot":
        v = x * inp["y"]
    elif name == "weighted_mapped":
        v = (1.5 * x) * inp["w"]
    else:
        v = x
    return math.sqrt(float(np.sum(v * v)))


@pytest.mark.parametrize("n, offset", [(5, 0), (4096 + 7, 3), ((1 << 20) + 1, 1)])
def test_ir_edge_cases(edge, n, offset):
    pkg, oracle, progs = edge
    rng = np.random.default_rng(n + offset)
    for prog in progs:
        name = prog["entry_name"]
        inp = {}
        for p in prog["params"]:
            inp[p["name"]] = (rng.uniform(-2, 2, n).astype(np.float32)
                              if p["kind"] == "tensor1-f32" else SCALARS[p["name"]])
        ref = oracle.run(name, inp)
        dev = {k: (to_device(v, offset) if isinstance(v, np.ndarray) else v)
               for k, v in inp.items()}
        out = to_device(np.zeros(n, np.float32), offset) if prog["result"]["kind"] == "tensor" \
            else None
        got = pkg[name](out=out, **dev)
        torch.cuda.synchronize()
        got = got.cpu().numpy()
        if prog["result"]["kind"] == "tensor":
            assert_bits(got, ref)
        elif name == "max_of_map":
            assert float(got[0]) == float(np.float32(ref))
        else:
            tol = 1e-6 * max(1.0, math.log2(n)) * max(abs(ref), _mass(name, inp))
            assert abs(float(got[0]) - ref) <= tol, (name, float(got[0]), ref)
