"""Optimisation flags and the tuning configuration as ``loomc`` reads them
(src/loom_core/optimizations.ml, optimization_config.ml), restated in
loom_b200/optconfig.py."""

import pytest

from loom_b200.build import CUDA_FIXED_FLAGS
from loom_b200.optconfig import (DEFAULT_CONFIG, FLAGS, OptionsError, config_from_json,
                                 in_catalogue_order, parse_cli_flags)


def test_catalogue():
    # optimizations.ml lists 70 flags; the harness's tuned CUDA profile uses
    # 47 of them
    assert len(FLAGS) == len(set(FLAGS)) == 70
    assert set(CUDA_FIXED_FLAGS) <= set(FLAGS)
    assert FLAGS[0] == "scalar-const-fold" and FLAGS[-1] == "cuda-selected-profile"


def test_cli_flags_enable_then_disable_in_catalogue_order():
    # optimization_config.ml:182-216
    got = parse_cli_flags(["tensor-cse", "normalized-dce", "scalar-const-fold", "tensor-cse"],
                          ["tensor-cse"])
    assert got == ["scalar-const-fold", "normalized-dce"]
    with pytest.raises(OptionsError, match="unknown optimization flag bogus in --enable-opt"):
        parse_cli_flags(["bogus"], [])
    with pytest.raises(OptionsError, match="unknown optimization flag bogus in --disable-opt"):
        parse_cli_flags([], ["bogus"])
    assert in_catalogue_order(["cuda-selected-profile", "if-simplify"]) == \
        ["if-simplify", "cuda-selected-profile"]


def test_default_config_is_the_reference_current_json():
    cfg = DEFAULT_CONFIG.to_json()
    assert (cfg["version"], cfg["small_inline_nodes"], cfg["small_clone_nodes"]) == (9, 20, 12)
    assert cfg["reduction_stage_medium_threshold"] == 4096
    assert cfg["elementwise_buckets"][0] == {"max_n": 131072, "block_size": 256, "num_warps": 4}
    assert cfg["source_path"] is None


def _minimal(**extra):
    obj = {"version": 1, "small_inline_nodes": 5, "reduction_precombine_max_body_complexity": 7,
           "single_block_reduction_threshold": 9,
           "elementwise_buckets": [{"max_n": 10, "block_size": 128, "num_warps": 4}],
           "reduction_buckets": []}
    obj.update(extra)
    return obj


def test_loaded_config_defaults_come_from_the_builtin_configuration():
    # optimization_config.ml:96-177: an omitted optional field takes the
    # built-in value (:5-40), not the current.json one
    cfg = config_from_json(_minimal(), "x.json")
    assert cfg.small_inline_nodes == 5 and cfg.source_path == "x.json"
    assert cfg.reduction_stage_medium_threshold == 8192      # built-in, not 4096
    assert cfg.small_reduction_program_count == 8            # built-in, not 4
    assert cfg.small_clone_nodes == 12
    assert cfg.reduction_buckets == ()
    assert config_from_json(_minimal(small_clone_nodes=3)).small_clone_nodes == 3


@pytest.mark.parametrize("obj, message", [
    ([], "expected JSON object in Loom optimization config"),
    ({k: v for k, v in _minimal().items() if k != "reduction_buckets"},
     "missing Loom optimization config field reduction_buckets"),
    (_minimal(version=1.0), "expected integer field version"),
    (_minimal(small_clone_nodes=True), "expected integer field small_clone_nodes"),
    (_minimal(elementwise_buckets={}), "expected list field elementwise_buckets"),
    (_minimal(elementwise_buckets=[{"max_n": 1, "block_size": 2}]),
     "missing Loom optimization config field num_warps"),
])
def test_config_errors(obj, message):
    with pytest.raises(OptionsError, match=message):
        config_from_json(obj)
