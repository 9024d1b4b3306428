"""The restated scalar and TensorIR passes preserve what a program computes,
up to rounding: every entry of the seeded random project
tests/golden/sources/pass_programs (make_pass_programs.py) is lowered without
flags and with the pass flags, and both TensorIR programs are evaluated in
float64 on the same inputs.

The FrontIR the front end prints for these entries equals what the
reference's own Python frontend printed for them (committed fixture).

The passes re-associate sums and products and fold constants, so the two
evaluations differ by rounding only (relative 1e-9 of the magnitudes
involved); an operand swapped in a non-commutative operation, a min turned
into a max, a dropped term or a wrong weight would show as a large
difference.  Inputs are finite and every generated denominator is d*d + 1,
so x*0 -> 0 is exact here too.

On a GPU the project is also packaged with the flag set of the reference
harness's tuned CUDA profile and every entry is compared with the oracle
run on the same rewritten programs (maps bit-exact except bodies rendered
with __fdividef, sums to the suite's tolerance, max exact)."""

import math
import os
import re

import numpy as np
import pytest

from loom_b200 import tensor_ir as TI
from loom_b200.build import CUDA_FIXED_FLAGS
from loom_b200.frontend import python_programs
from loom_b200.frontend.normalize_passes import NORMALIZE_FLAGS
from loom_b200.frontend.passes import FUSE_FLAGS, TENSOR_BODY_FLAGS

HERE = os.path.dirname(os.path.abspath(__file__))
PROJECT = os.path.join(HERE, "golden", "sources", "pass_programs")
SOURCE = os.path.join(PROJECT, "pass_programs.py")
ALL_PASSES = (NORMALIZE_FLAGS + TENSOR_BODY_FLAGS + FUSE_FLAGS
              + ("reduce-map-fusion", "shape-use-simplify"))
SCALARS = {"a": 0.75, "b": -1.25}
# further flag sets of the reference harness's profiles
# (experiments/source/data/profiles/loom_profiles.json)
POINTWISE_GUARDED = ("scalar-const-fold", "if-simplify", "arith-reassociate", "branch-hoist",
                     "lambda-inline-small", "scalar-cse", "normalized-dce", "tensor-canonicalize",
                     "map-chain-collapse", "elementwise-fusion", "shape-use-simplify", "tensor-cse",
                     "materialization-choice", "branch-aware-fusion-guard",
                     "pointwise-materialization-guard", "elementwise-plan-specialize",
                     "pointwise-shape-plan", "multi-use-fusion-guard", "storage-reuse-pack",
                     "launch-bucket-specialize")
REDUCTION_CORE = ("scalar-const-fold", "if-simplify", "arith-reassociate", "lambda-inline-small",
                  "scalar-cse", "normalized-dce", "tensor-canonicalize", "reduction-input-simplify",
                  "reduction-body-normalize", "reduction-body-canonicalize",
                  "reduction-accumulator-shape", "reduction-reuse-hoist", "reduction-body-cse",
                  "reduce-map-fusion", "map-chain-collapse", "tensor-cse", "shape-use-simplify",
                  "materialization-choice", "reduction-materialization-choice",
                  "reduction-plan-specialize", "reduction-classify", "reduction-tree-plan",
                  "reduction-split-plan", "reduction-small-plan-specialize",
                  "reduction-stage-sizing", "reduction-stage-balance",
                  "reduction-partial-shape-pack", "reduction-class-aware-buckets",
                  "storage-reuse-pack", "launch-bucket-specialize")
# the late-fusion guard and clone flags, which no profile enables together
GUARDS = ("reduce-map-fusion", "map-chain-collapse", "small-producer-clone",
          "reduction-late-fusion-guard", "materialization-choice",
          "reduction-materialization-choice", "branchy-reduction-rescue", "scalar-hoist",
          "let-float")


def eval_expr(e, env):
    if isinstance(e, TI.SVar):
        return env[e.name]
    if isinstance(e, TI.SConstF32):
        return np.float64(e.value)
    if isinstance(e, TI.SConstBool):
        return np.bool_(e.value)
    if isinstance(e, TI.SUnary):
        v = eval_expr(e.expr, env)
        return {"neg": np.negative, "sqrt": np.sqrt, "exp": np.exp, "log": np.log}[e.op](v)
    if isinstance(e, TI.SSelect):
        return np.where(eval_expr(e.cond, env), eval_expr(e.then, env), eval_expr(e.els, env))
    a, b = eval_expr(e.lhs, env), eval_expr(e.rhs, env)
    return {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide,
            "min": np.minimum, "max": np.maximum, "cmplt": np.less, "cmple": np.less_equal,
            "cmpgt": np.greater, "cmpge": np.greater_equal, "cmpeq": np.equal}[e.op](a, b)


def evaluate(prog: TI.Program, inputs, n):
    """float64 value of the program and the magnitude that bounds its
    rounding (the sum of |terms| for a sum)."""
    values = {}

    def ref(r):
        return inputs[r.name] if isinstance(r, TI.ParamRef) else values[r.id]

    scalars = {k: np.float64(v) for k, v in inputs.items() if not isinstance(v, np.ndarray)}
    for node in prog.nodes:
        if isinstance(node, TI.Elementwise1D):
            env = dict(scalars)
            env.update({bd.name: ref(bd.source) for bd in node.inputs})
            values[node.id] = np.broadcast_to(eval_expr(node.body, env), (n,)).astype(np.float64)
            continue
        if isinstance(node.source, TI.PlainInput):
            terms = ref(node.source.input)
        else:
            env = dict(scalars)
            env.update({bd.name: ref(bd.source) for bd in node.source.inputs})
            terms = np.broadcast_to(eval_expr(node.source.body, env), (n,)).astype(np.float64)
        if node.kind == "sum":
            values[node.id] = (np.sum(terms), np.sum(np.abs(terms)))
        else:
            values[node.id] = (np.max(terms), np.max(np.abs(terms)))
    out = values[prog.result.id]
    if prog.result_kind == "tensor":
        return out, np.abs(out)
    return out


def _inputs(n, seed):
    rng = np.random.default_rng(seed)
    inp = {t: rng.standard_normal(n) for t in ("x", "y", "w")}
    inp.update(SCALARS)
    return inp


def test_front_ir_of_the_pass_programs_matches_the_reference_frontend():
    # tests/golden/pass_programs_front_ir.json holds what the reference's
    # Python frontend printed for every entry (make_front_ir.py), so the
    # programs the passes rewrite start from the reference's own FrontIR
    import json
    from loom_b200.frontend import front_ir
    golden = json.load(open(os.path.join(HERE, "golden", "pass_programs_front_ir.json")))
    with open(SOURCE, encoding="utf-8") as fh:
        src = fh.read()
    assert len(golden) == 40
    for entry, want in golden.items():
        assert front_ir(src, entry) == want, entry


@pytest.mark.parametrize("flags", [ALL_PASSES, tuple(CUDA_FIXED_FLAGS), POINTWISE_GUARDED,
                                   REDUCTION_CORE, GUARDS],
                         ids=["all_passes", "cuda_fixed", "pointwise_guarded", "reduction_core",
                              "guards"])
def test_passes_preserve_values(flags):
    plain = {p.entry_name: p for p in python_programs(SOURCE)}
    rewritten = {p.entry_name: p for p in python_programs(SOURCE, flags)}
    assert sorted(plain) == sorted(rewritten) and len(plain) == 40
    n = 2000
    changed = 0
    for name in sorted(plain):
        TI.validate(rewritten[name])
        inp = _inputs(n, seed=len(name) + int(name[1:]))
        want, mag = evaluate(plain[name], inp, n)
        got, _ = evaluate(rewritten[name], inp, n)
        tol = 1e-9 * (np.asarray(mag) + 1.0)
        assert np.all(np.abs(np.asarray(got) - np.asarray(want)) <= tol), name
        changed += TI.program_to_string(plain[name]) != TI.program_to_string(rewritten[name])
    assert changed >= 30                  # the passes do fire on these programs


@pytest.mark.gpu
def test_pass_programs_match_oracle_on_gpu():
    import torch

    from loom_b200.build import build_project
    from loom_b200.loader import Package
    from oracle.loom_oracle import Oracle
    from test_gpu_parity import assert_bits, to_device

    progs = {p.entry_name: p for p in python_programs(SOURCE, CUDA_FIXED_FLAGS)}
    pkg_dir = build_project(PROJECT, enabled=CUDA_FIXED_FLAGS, name="pass_programs_cuda_fixed")
    pkg = Package(pkg_dir)
    oracle = Oracle([TI.program_to_json(p) for p in progs.values()],
                    name="pass_programs_cuda_fixed", enabled=CUDA_FIXED_FLAGS)
    src = open(os.path.join(pkg_dir, "src-gen", "pass_programs_cuda_fixed.cu")).read()
    fast = {m.group(1) for m in re.finditer(r"struct LoomBody_(\w+) \{(.*?)\n\};", src, re.S)
            if "__fdividef" in m.group(2)}
    for n, offset in ((4099, 1), ((1 << 20) + 5, 0)):
        for name, prog in sorted(progs.items()):
            inp = {k: (v.astype(np.float32) if isinstance(v, np.ndarray) else v)
                   for k, v in _inputs(n, seed=n + int(name[1:])).items()}
            ref = oracle.run(name, inp)
            dev = {k: (to_device(v, offset) if isinstance(v, np.ndarray) else v)
                   for k, v in inp.items()}
            out = to_device(np.zeros(n, np.float32), offset) \
                if prog.result_kind == "tensor" else None
            got = pkg[name](out=out, **dev)
            torch.cuda.synchronize()
            got = got.cpu().numpy()
            if prog.result_kind == "tensor":
                if pkg[name].symbol in fast:
                    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-30)
                else:
                    assert_bits(got, ref)
            elif prog.node(prog.result.id).kind == "max":
                assert float(got[0]) == float(np.float32(ref)), name
            else:
                f64 = {k: (v.astype(np.float64) if isinstance(v, np.ndarray) else v)
                       for k, v in inp.items()}
                _, mag = evaluate(progs[name], f64, n)
                tol = 1e-6 * max(1.0, math.log2(n)) * max(abs(ref), float(mag))
                assert abs(float(got[0]) - ref) <= tol, (name, float(got[0]), ref, tol)
