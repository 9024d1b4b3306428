"""Front end (Python entry language -> FrontIR -> LoomLambda -> TensorIR)
against the reference's own outputs: FrontIR that the reference's Python
frontend printed for the same sources, its error messages, its golden
LoomLambda and TensorIR files.  All fixtures were produced by
tests/golden/make_golden.py."""

import glob
import json
import os

import pytest

from loom_b200 import tensor_ir as TI
from loom_b200.artifact import discover_entries, generate_package
from loom_b200.frontend import (FrontendError, front_ir, list_entries, loom_lambda,
                                program_from_front_ir)

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")
SUITE_SRC = os.path.join(ROOT, "loom_b200", "suite", "kernels.py")
CASES_SRC = os.path.join(GOLDEN, "sources", "cases", "frontend_cases.py")
ERRORS_SRC = os.path.join(GOLDEN, "sources", "errors", "frontend_errors.py")


def _read(path):
    with open(path) as fh:
        return fh.read()


def _golden_front(tag, entry):
    return json.load(open(os.path.join(GOLDEN, "front_ir", f"{tag}.{entry}.json")))


def _front_cases():
    out = []
    for path in sorted(glob.glob(os.path.join(GOLDEN, "front_ir", "*.json"))):
        tag, entry = os.path.basename(path)[:-5].split(".")
        if tag == "suite_kernels":
            out.append((SUITE_SRC, tag, entry))
        elif tag == "cases_frontend_cases":
            out.append((CASES_SRC, tag, entry))
    return out


@pytest.mark.parametrize("src, tag, entry", _front_cases(), ids=lambda v: str(v)[-30:])
def test_front_ir_matches_reference_frontend(src, tag, entry):
    assert front_ir(_read(src), entry) == _golden_front(tag, entry)


@pytest.mark.parametrize("tag, entry", [
    ("examples_saxpy", "saxpy"), ("examples_relu", "relu"), ("examples_dot", "dot"),
    ("examples_l2_norm_sq", "l2_norm_sq"), ("python_package_project_kernels", "saxpy"),
    ("python_package_project_kernels", "relu"), ("python_package_project_kernels", "dot")])
def test_reference_examples_have_the_suite_front_ir(tag, entry):
    # The reference's own examples and package fixture are the same programs as
    # the suite's; the reference frontend gave the same FrontIR for both.
    assert _golden_front(tag, entry) == front_ir(_read(SUITE_SRC), entry)


def test_error_messages_match_reference_frontend():
    errors = json.load(open(os.path.join(GOLDEN, "front_ir_errors.json")))
    src = _read(ERRORS_SRC)
    for entry, ref in errors.items():
        if ref["returncode"] == 0:
            fir = front_ir(src, entry)          # accepted by the frontend ...
            with pytest.raises(FrontendError):  # ... rejected when tensorized
                program_from_front_ir(fir)
            continue
        with pytest.raises(FrontendError) as info:
            front_ir(src, entry)
        assert ref["stderr"] == "Python frontend error: " + str(info.value)


def test_loom_lambda_matches_reference_golden():
    golden = json.load(open(os.path.join(GOLDEN, "reference_ir", "saxpy_loom_lambda.json")))
    assert loom_lambda(front_ir(_read(SUITE_SRC), "saxpy")) == golden


def test_tensor_ir_matches_reference_golden_with_metrics():
    golden = json.load(open(os.path.join(GOLDEN, "reference_ir", "l2_norm_sq_tensor_ir.json")))
    prog = program_from_front_ir(front_ir(_read(SUITE_SRC), "l2_norm_sq"))
    assert TI.program_to_json(prog) == golden


def test_suite_front_end_matches_hand_written_oracle_programs():
    def strip(o):
        if isinstance(o, dict):
            return {k: strip(v) for k, v in o.items() if k != "metrics"}
        if isinstance(o, list):
            return [strip(v) for v in o]
        return o

    hand = json.load(open(os.path.join(ROOT, "oracle", "suite_kernels.tensor_ir.json")))
    src = _read(SUITE_SRC)
    for obj in hand:
        prog = program_from_front_ir(front_ir(src, obj["entry_name"]))
        assert strip(TI.program_to_json(prog)) == strip(obj)


def test_metrics_and_shapes():
    src = _read(CASES_SRC)
    chain = program_from_front_ir(front_ir(src, "scaled_chain"))
    assert [n.metrics.estimated_uses for n in chain.nodes] == [1, 1, 1, 1]
    div_node = chain.nodes[2]
    assert div_node.metrics.has_div and div_node.metrics.div_count == 1
    soft = program_from_front_ir(front_ir(src, "soft_threshold")).nodes[0]
    assert soft.metrics.branch_count == 2 and soft.scalar_params == ("t",)
    lets = program_from_front_ir(front_ir(src, "tuple_lets")).nodes[0]
    assert lets.scalar_params == ("a",)     # p, q and scale are substituted
    assert [e["name"] for e in list_entries(src)] == sorted(e["name"] for e in list_entries(src))


def test_package_discovers_python_sources(tmp_path):
    res = generate_package(os.path.dirname(CASES_SRC), str(tmp_path), build=False)
    manifest = json.load(open(res.manifest_path))
    assert manifest["package_name"] == "frontend_cases"
    assert sorted(e["entry_name"] for e in manifest["entries"]) == sorted(
        e["name"] for e in list_entries(_read(CASES_SRC)))
    assert {e["symbol_name"] for e in manifest["entries"]} == {
        "loom_frontend_cases_" + e["name"] for e in list_entries(_read(CASES_SRC))}
    with pytest.raises(FrontendError):
        discover_entries(os.path.dirname(ERRORS_SRC))


def test_entry_listing_matches_reference_frontend():
    # the reference frontend's list-entries-json output (make_golden.py):
    # names in its order, parameter names and kinds
    listings = json.load(open(os.path.join(GOLDEN, "list_entries.json")))
    assert len(listings) == 3
    for rel, want in listings.items():
        path = os.path.join(ROOT, *rel.split("/"))
        assert list_entries(_read(path), path) == want["entries"], rel


def test_random_rejected_entries_give_the_reference_messages():
    # 40 seeded entries with one rejected construct each, at random depths
    # (sources/errors/make_random_errors.py): the same message, line and
    # column as the reference's Python frontend
    errors = json.load(open(os.path.join(GOLDEN, "random_errors.json")))
    src = _read(os.path.join(GOLDEN, "sources", "errors", "random_errors.py"))
    assert len(errors) == 40
    for entry, ref in errors.items():
        assert ref["returncode"] != 0, entry
        with pytest.raises(FrontendError) as info:
            front_ir(src, entry)
        assert ref["stderr"] == "Python frontend error: " + str(info.value), entry
