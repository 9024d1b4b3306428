"""The restated TensorIR passes (loom_b200/frontend/passes.py) on the suite
entries: what map-chain collapse, reduce-map fusion and shape-use
simplification make of them, derived by hand from the reference's passes
(src/loom_tensorize/tensor_passes.ml:103-335) and its materialisation policy
(materialization_policy.ml); that they are off by default; and that the
fused programs still compute the same values (the oracle on the fused and the
unfused TensorIR; bits may differ where fusion lets a product and an add
contract into one fmaf, as in the reference)."""

import os

import numpy as np
import pytest

from loom_b200 import tensor_ir as TI
from loom_b200 import workloads
from loom_b200.frontend import python_programs
from loom_b200.frontend.passes import allow_inline_producer, allow_inline_into_reduction

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SUITE_SRC = os.path.join(ROOT, "loom_b200", "suite", "kernels.py")
FUSE = ("map-chain-collapse", "reduce-map-fusion")


def _progs(enabled):
    return {p.entry_name: p for p in python_programs(SUITE_SRC, enabled)}


def test_passes_are_off_by_default():
    plain = _progs(())
    assert [type(n).__name__ for n in plain["dot"].nodes] == ["Elementwise1D", "Reduce1D"]
    assert isinstance(plain["dot"].nodes[1].source, TI.PlainInput)


def test_reduce_map_fusion_makes_a_mapped_dot():
    prog = _progs(FUSE)["dot"]
    assert len(prog.nodes) == 1
    red = prog.nodes[0]
    assert isinstance(red, TI.Reduce1D) and red.id == 1 and prog.result == TI.NodeRef(1)
    src = red.source
    assert isinstance(src, TI.MappedInput)
    assert [(b.name, b.source) for b in src.inputs] == [
        ("xi__r0", TI.ParamRef("x")), ("yi__r0", TI.ParamRef("y"))]
    assert src.scalar_params == ()
    assert src.body == TI.SBinary("mul", TI.SVar("xi__r0"), TI.SVar("yi__r0"))
    assert red.reduction_shape == "mapped"


def test_chain_collapse_then_reduce_fusion_on_the_pipeline():
    prog = _progs(FUSE)["pipeline_sum"]
    assert len(prog.nodes) == 1 and prog.nodes[0].id == 2
    src = prog.nodes[0].source
    assert [(b.name, b.source) for b in src.inputs] == [
        ("zi__xi__f0__r0", TI.ParamRef("x")), ("zi__yi__f0__r0", TI.ParamRef("y")),
        ("wi__r0", TI.ParamRef("w"))]
    assert src.scalar_params == ("a",)
    affine = TI.SBinary("add", TI.SBinary("mul", TI.SVar("a"), TI.SVar("zi__xi__f0__r0")),
                        TI.SVar("zi__yi__f0__r0"))
    relu = TI.SSelect(TI.SBinary("cmpgt", affine, TI.SConstF32(0.0)), affine, TI.SConstF32(0.0))
    assert src.body == TI.SBinary("mul", relu, TI.SVar("wi__r0"))
    assert prog.nodes[0].reduction_shape == "branchy-mapped"


def test_maps_keep_their_single_node():
    progs = _progs(FUSE)
    for name in ("saxpy", "relu", "affine_relu"):
        assert len(progs[name].nodes) == 1


def test_guards_keep_a_branchy_producer_materialised():
    # branch-aware-fusion-guard: a producer with a select and complexity >= 6
    m = TI.BodyMetrics(scalar_complexity=6, has_branch=True, branch_count=1)
    assert allow_inline_producer(("branch-aware-fusion-guard",), m, 1) == "disallow"
    assert allow_inline_producer((), m, 1) == "fuse"
    assert allow_inline_producer((), m, 2) == "clone"
    assert allow_inline_producer(("materialization-choice",), m, 2) == "disallow"
    assert allow_inline_into_reduction(("reduction-late-fusion-guard",), m, 1, 3) == "disallow"
    assert allow_inline_into_reduction(("reduction-materialization-choice",), m, 2, 0) == \
        "disallow"


def test_small_producer_clone_duplicates_a_shared_producer():
    # node_0 feeds node_1 twice (use count 2): cloned only under small-producer-clone
    d = TI.SVar("d")
    prog = TI.Program("twice", [TI.TensorParam("x")], "tensor", TI.NodeRef(1), [
        TI.Elementwise1D(0, (TI.InputBinding("xi", TI.ParamRef("x")),), (),
                         TI.SBinary("mul", TI.SVar("xi"), TI.SConstF32(3.0))),
        TI.Elementwise1D(1, (TI.InputBinding("d", TI.NodeRef(0)),
                             TI.InputBinding("e", TI.NodeRef(0))), (),
                         TI.SBinary("add", d, TI.SVar("e")))])
    from loom_b200.frontend.passes import apply_tensor_passes
    import copy
    kept = apply_tensor_passes(copy.deepcopy(prog), ("map-chain-collapse",))
    assert len(kept.nodes) == 2 and kept.nodes[1].inputs[0].source == TI.NodeRef(0)
    cloned = apply_tensor_passes(copy.deepcopy(prog), ("map-chain-collapse",
                                                       "small-producer-clone"))
    # cloned into both bindings; the producer stays (use count 2) until shape-use
    # simplification drops it as unreachable
    assert [b.name for b in cloned.nodes[-1].inputs] == ["d__xi__f0", "e__xi__f0"]
    assert len(cloned.nodes) == 2
    dropped = apply_tensor_passes(copy.deepcopy(prog), ("map-chain-collapse",
                                                        "small-producer-clone",
                                                        "shape-use-simplify"))
    assert [n.id for n in dropped.nodes] == [1]
    # the clone limit is the configuration's small_clone_nodes (tensor_passes.ml:
    # ~clone_complexity_limit); the producer has complexity 1
    from dataclasses import replace
    from loom_b200.optconfig import DEFAULT_CONFIG
    tight = replace(DEFAULT_CONFIG, small_clone_nodes=0)
    kept = apply_tensor_passes(copy.deepcopy(prog), ("map-chain-collapse",
                                                     "small-producer-clone"), tight)
    assert kept.nodes[1].inputs[0].source == TI.NodeRef(0)


@pytest.mark.parametrize("entry", ["dot", "l2_norm_sq", "max_value", "pipeline_sum",
                                   "affine_relu"])
def test_fused_programs_compute_the_same_values(entry):
    from oracle.loom_oracle import Oracle
    plain = Oracle([TI.program_to_json(_progs(())[entry])], name=f"pass_plain_{entry}")
    fused = Oracle([TI.program_to_json(_progs(FUSE)[entry])], name=f"pass_fused_{entry}")
    inp = workloads.entry_inputs(entry, 100003)
    a, b = plain.run(entry, inp), fused.run(entry, inp)
    if isinstance(a, np.ndarray):
        np.testing.assert_allclose(a, b, rtol=1e-6, atol=1e-6)
    else:
        assert b == pytest.approx(a, rel=1e-9)
