"""Seeded random TensorIR programs (tests/golden/sources/random, written by
make_random_programs.py there): element-wise chains of 1-3 nodes over 1-3
tensors and 0-2 scalars, ending in a map, a plain or mapped sum, or a max.

CPU: the committed programs are what the generator writes, and the oracle
compiles them.
GPU: every program through the B200 package against the oracle, at ragged
sizes and offsets, with and without special values (signed zeros,
denormals, infinities, NaN) in the inputs.  Bar: maps and max bit-exact (NaN
only has to be NaN); sums within 1e-6 * max(1, log2 n) * max(|ref|,
sqrt(sum v_i^2)), where v_i are the per-element values from the program's
companion map `<name>_values`, and of the same class (NaN, +inf, -inf) when
the oracle's sum is not finite.
"""

import json
import math
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
RAND_DIR = os.path.join(HERE, "golden", "sources", "random")
RAND_IR = os.path.join(RAND_DIR, "random_programs.tensor_ir.json")
SCALARS = {"a": 1.25, "b": -0.5}
SPECIALS_MAP = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 3.4e38, -3.4e38,
                         1.2e-38], dtype=np.float32)
SPECIALS_SUM = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40], dtype=np.float32)


def _programs():
    with open(RAND_IR) as fh:
        return json.load(fh)


def test_committed_programs_match_generator(tmp_path):
    import shutil
    work = tmp_path / "random"
    work.mkdir()
    shutil.copy(os.path.join(RAND_DIR, "make_random_programs.py"), work)
    # the generator writes beside itself; point it at the repository's package
    env = dict(os.environ, PYTHONPATH=os.path.dirname(HERE))
    subprocess.run([sys.executable, str(work / "make_random_programs.py")], check=True,
                   env=env, capture_output=True)
    assert json.load(open(work / "random_programs.tensor_ir.json")) == _programs()


def test_oracle_compiles_random_programs():
    from oracle.loom_oracle import Oracle, load_programs
    progs = load_programs(RAND_IR)
    o = Oracle(progs, name="random_programs")
    n = 9
    for prog in progs:
        inp = {p["name"]: (np.linspace(-2, 2, n, dtype=np.float32)
                           if p["kind"] == "tensor1-f32" else SCALARS[p["name"]])
               for p in prog["params"]}
        o.run(prog["entry_name"], inp)


def _inputs(prog, n, rng, specials):
    inp = {}
    for p in prog["params"]:
        if p["kind"] != "tensor1-f32":
            inp[p["name"]] = SCALARS[p["name"]]
            continue
        v = rng.uniform(-2, 2, n).astype(np.float32)
        if specials is not None:
            hit = rng.random(n) < 0.02
            v[hit] = rng.choice(specials, int(hit.sum()))
        inp[p["name"]] = v
    return inp


def _same_class(got, ref):
    if math.isnan(ref):
        return math.isnan(got)
    return got == ref          # +inf or -inf


@pytest.mark.gpu
@pytest.mark.parametrize("n, offset, specials", [
    (1, 0, False), (3, 1, True), (17, 2, False), (4096 + 7, 3, True),
    (65536 + 5, 0, False), ((1 << 20) + 3, 2, True)])
def test_random_programs_match_oracle(n, offset, specials):
    import torch

    from loom_b200.build import build_project
    from loom_b200.loader import Package
    from oracle.loom_oracle import Oracle, load_programs
    from test_gpu_parity import assert_bits, to_device

    progs = load_programs(RAND_IR)
    pkg = Package(build_project(RAND_DIR))
    oracle = Oracle(progs, name="random_programs")
    rng = np.random.default_rng(1000 * n + offset)
    for prog in progs:
        name = prog["entry_name"]
        if name.endswith("_values"):
            continue
        kind = name.rsplit("_", 1)[1]
        pool = None if not specials else (SPECIALS_SUM if kind == "sum" else SPECIALS_MAP)
        inp = _inputs(prog, n, rng, pool)
        ref = oracle.run(name, inp)
        dev = {k: (to_device(v, offset) if isinstance(v, np.ndarray) else v)
               for k, v in inp.items()}
        out = to_device(np.zeros(n, np.float32), offset) if kind == "map" else None
        got = pkg[name](out=out, **dev)
        torch.cuda.synchronize()
        got = got.cpu().numpy()
        if kind == "map":
            assert_bits(got, ref)
        elif kind == "max":
            g, r = np.float32(got[0]), np.float32(ref)
            assert (np.isnan(g) and np.isnan(r)) or g.view(np.uint32) == r.view(np.uint32), \
                (name, n, g, r)
        else:
            g = float(got[0])
            if not math.isfinite(ref):
                assert _same_class(g, ref), (name, n, g, ref)
                continue
            vals = oracle.run(name + "_values", inp).astype(np.float64)
            scale = math.sqrt(float(np.sum(vals * vals)))
            tol = 1e-6 * max(1.0, math.log2(n)) * max(abs(ref), scale)
            assert abs(g - ref) <= tol, (name, n, g, ref, tol)
