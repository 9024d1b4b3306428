"""The reference harness's 33 supported kernels
(experiments/source/data/common/workloads.json) through this backend.

The fixtures under tests/golden/sources/workloads/ hold the FrontIR that the
reference's own Python frontend printed for each kernel's source
(tests/golden/make_workloads.py); this repository's front end printed the
same FrontIR for all of them when the fixtures were made.  Here that FrontIR
is lowered (normalize, tensorize), packaged for sm_100a and run:

* CPU: every kernel lowers to valid TensorIR, the package finds all 33
  entries, and the oracle compiles them;
* GPU: every kernel against the oracle on the harness's input distribution
  (N(0,1) tensors, the harness's scalar arguments), built three times: with
  the default flags, with the reference's fusion passes and body-rendering
  flags (loom_b200.build.FUSION_FLAGS + RENDER_FLAGS), and with the flag set
  of the harness's tuned CUDA profile (loom_b200.build.CUDA_FIXED_FLAGS,
  which adds the scalar and TensorIR rewrites).  Maps bit-exact (NaN
  only has to be NaN), except bodies rendered with __fdividef, which are
  within 2 ulp of the oracle's exact division and are compared at rtol 1e-6;
  sums within 1e-6 * max(1, log2 n) * |ref| (the relative bound the
  backend is specified to; ref is the oracle's fp64 sum of the per-element
  values, which a companion map of the reduced body also exposes).
"""

import copy
import json
import math
import os
import re

import numpy as np
import pytest

from loom_b200 import tensor_ir as TI
from loom_b200.artifact import discover_entries, load_front_ir_file
from loom_b200.build import CUDA_FIXED_FLAGS, FUSION_FLAGS, RENDER_FLAGS

HERE = os.path.dirname(os.path.abspath(__file__))
WL_DIR = os.path.join(HERE, "golden", "sources", "workloads")
TABLE = json.load(open(os.path.join(WL_DIR, "workloads.json")))
FLAGGED = tuple(FUSION_FLAGS) + tuple(RENDER_FLAGS)


def _programs(enabled=()):
    progs = {}
    for w in TABLE:
        for p in load_front_ir_file(os.path.join(WL_DIR, w["name"] + ".front_ir.json"), enabled):
            progs[w["name"]] = p
    return progs


def values_program(prog: TI.Program) -> TI.Program:
    """The per-element values a reduction folds, as a map program."""
    red = prog.node(prog.result.id)
    assert isinstance(red, TI.Reduce1D)
    nodes = [copy.deepcopy(n) for n in prog.nodes if n.id != red.id]
    if isinstance(red.source, TI.PlainInput):
        result = red.source.input
        if isinstance(result, TI.ParamRef):      # a plain sum over a parameter
            nodes.append(TI.Elementwise1D(red.id, (TI.InputBinding("v", result),), (),
                                          TI.SVar("v")))
            result = TI.NodeRef(red.id)
    else:
        src = red.source
        nodes.append(TI.Elementwise1D(red.id, src.inputs, src.scalar_params, src.body))
        result = TI.NodeRef(red.id)
    return TI.Program(prog.entry_name + "__values", prog.params, "tensor", result, nodes)


def test_fixtures_cover_the_harness_kernels():
    assert len(TABLE) == 33
    assert all(w["front_ir_matches_this_front_end"] for w in TABLE)


@pytest.mark.parametrize("enabled", [(), FLAGGED, tuple(CUDA_FIXED_FLAGS)],
                         ids=["default", "flags", "cuda_fixed"])
def test_workloads_lower_and_package(enabled):
    progs = _programs(enabled)
    assert len(progs) == 33
    for name, prog in progs.items():
        TI.validate(prog)
        w = next(t for t in TABLE if t["name"] == name)
        assert prog.result_kind == w["result_kind"]
        assert sorted(p.name for p in prog.tensor_params) == sorted(w["tensor_inputs"])
    assert len(discover_entries(WL_DIR, enabled=enabled)) == 33


def test_oracle_compiles_workloads_and_their_values():
    from oracle.loom_oracle import Oracle
    progs = _programs()
    objs = [TI.program_to_json(p) for p in progs.values()]
    objs += [TI.program_to_json(values_program(p)) for p in progs.values()
             if p.result_kind == "scalar"]
    Oracle(objs, name="workloads_cpu_check")


def _inputs(w, n, seed):
    rng = np.random.default_rng(seed)
    inp = {t: rng.standard_normal(n).astype(np.float32) for t in w["tensor_inputs"]}
    inp.update({k: float(v) for k, v in w["scalar_args"].items()})
    return inp


VARIANTS = {"default": ((), "workloads"), "flags": (FLAGGED, "workloads_flags"),
            "cuda_fixed": (tuple(CUDA_FIXED_FLAGS), "workloads_cuda_fixed")}


@pytest.mark.gpu
@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_workloads_match_oracle(variant):
    import torch

    from loom_b200.build import build_project
    from loom_b200.loader import Package
    from oracle.loom_oracle import Oracle
    from test_gpu_parity import assert_bits, to_device

    enabled, name = VARIANTS[variant]
    progs = _programs(enabled)
    pkg_dir = build_project(WL_DIR, enabled=enabled, name=name)
    pkg = Package(pkg_dir)
    objs = [TI.program_to_json(p) for p in progs.values()]
    objs += [TI.program_to_json(values_program(p)) for p in progs.values()
             if p.result_kind == "scalar"]
    oracle = Oracle(objs, name=name, enabled=enabled)
    # map bodies rendered with __fdividef (the ratio-book bodies under
    # cuda-pointwise-selected-tail-plan): CUDA's fast division is within 2 ulp
    # of IEEE division for these operands, the oracle divides exactly
    src = open(os.path.join(pkg_dir, "src-gen", name + ".cu")).read()
    fast = {m.group(1) for m in re.finditer(r"struct LoomBody_(\w+) \{(.*?)\n\};", src, re.S)
            if "__fdividef" in m.group(2)}
    for n, offset in ((4099, 1), ((1 << 20) + 3, 0)):
        for w in TABLE:
            prog = progs[w["name"]]
            entry = prog.entry_name
            inp = _inputs(w, n, seed=n + len(w["name"]))
            ref = oracle.run(entry, inp)
            dev = {k: (to_device(v, offset) if isinstance(v, np.ndarray) else v)
                   for k, v in inp.items()}
            out = to_device(np.zeros(n, np.float32), offset) if prog.result_kind == "tensor" \
                else None
            got = pkg[entry](out=out, **dev)
            torch.cuda.synchronize()
            got = got.cpu().numpy()
            if prog.result_kind == "tensor":
                if pkg[entry].symbol in fast:
                    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=0)
                else:
                    assert_bits(got, ref)
                continue
            tol = 1e-6 * max(1.0, math.log2(n)) * abs(ref)
            assert abs(float(got[0]) - ref) <= tol, (variant, w["name"], n, float(got[0]), ref)


LIMITATIONS = json.load(open(os.path.join(HERE, "golden", "workload_limitations.json")))


def test_unsupported_capability_cases_are_rejected():
    # the harness's unsupported cases (experiments/source/python/limitations):
    # where the reference frontend rejects one, this front end gave the same
    # message when the fixtures were made; where only loomc's later lowering
    # rejects one, its FrontIR is committed and this lowering must reject it
    from loom_b200.frontend import FrontendError, program_from_front_ir
    assert len(LIMITATIONS) == 6
    lim_dir = os.path.join(HERE, "golden", "sources", "workload_limitations")
    for name, rec in LIMITATIONS.items():
        if rec["reference_frontend_returncode"] != 0:
            assert rec["this_front_end_error"] == rec["reference_error"], name
            continue
        assert rec["front_ir_matches_this_front_end"], name
        front = json.load(open(os.path.join(lim_dir, name + ".front_ir.json")))
        with pytest.raises(FrontendError):
            program_from_front_ir(front)
