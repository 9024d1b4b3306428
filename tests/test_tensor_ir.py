"""TensorIR boundary: JSON reader/writer and validation."""

import json
import os

import pytest

from loom_b200 import tensor_ir as T

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "reference_ir", "l2_norm_sq_tensor_ir.json")


def _strip(o, drop=("metrics",)):
    if isinstance(o, dict):
        return {k: _strip(v, drop) for k, v in o.items() if k not in drop}
    if isinstance(o, list):
        return [_strip(v, drop) for v in o]
    return o


def test_reference_golden_loads_and_roundtrips():
    with open(GOLDEN) as fh:
        golden = json.load(fh)
    prog = T.program_from_json(golden)
    assert prog.entry_name == "l2_norm_sq"
    assert prog.result_kind == "scalar" and prog.result == T.NodeRef(1)
    assert T.program_to_json(prog) == golden


def test_suite_l2_norm_sq_matches_reference_golden(suite_programs):
    with open(GOLDEN) as fh:
        golden = json.load(fh)
    mine = [p for p in suite_programs if p["entry_name"] == "l2_norm_sq"][0]
    assert _strip(mine) == _strip(golden)


def test_suite_programs_roundtrip(suite_programs):
    for obj in suite_programs:
        prog = T.program_from_json(obj)
        assert T.program_from_json(T.program_to_json(prog)).nodes == prog.nodes


def test_structural_equality_of_expressions():
    a = T.SBinary("add", T.SBinary("mul", T.SVar("a"), T.SVar("x")), T.SVar("y"))
    b = T.SBinary("add", T.SBinary("mul", T.SVar("a"), T.SVar("x")), T.SVar("y"))
    assert a == b and hash(a) == hash(b)
    assert T.SConstF32(0.0) == T.SConstF32(-0.0)  # OCaml '=' on floats
    assert T.free_vars(a) == ["a", "x", "y"]


@pytest.mark.parametrize("mutate, message", [
    (lambda p: p["nodes"][0]["inputs"].__setitem__(0, {"name": "xi", "source": "nope"}),
     "not a tensor parameter"),
    (lambda p: p["nodes"][0]["body"].__setitem__("lhs", {"kind": "var", "name": "zz"}),
     "unbound variable"),
    (lambda p: p.__setitem__("result", {"kind": "scalar", "value": "node_0"}),
     "must be a reduction"),
    (lambda p: p["nodes"][1].__setitem__("reduce_kind", "mean"), "unknown reduce kind"),
])
def test_validation_rejects(suite_programs, mutate, message):
    prog = json.loads(json.dumps([p for p in suite_programs if p["entry_name"] == "dot"][0]))
    mutate(prog)
    with pytest.raises(T.TensorIRError, match=message):
        T.program_from_json(prog)
