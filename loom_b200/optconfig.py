"""Loom's optimisation flags and tuning configuration, as ``loomc`` reads
them from its command line.

* ``FLAGS``: every flag of the reference's catalogue, in catalogue order
  (``src/loom_core/optimizations.ml:1-1045``).  ``--enable-opt`` and
  ``--disable-opt`` take these names only; the enabled set is reported in
  catalogue order (``optimization_config.ml:182-216``).
* ``OptConfig``: the tuning configuration (``optimization_config.ml:5-40``,
  ``:85-180``).  Without ``--opt-config`` it holds the values of the
  reference's ``configs/optimizations/current.json``, the file ``loomc``
  loads by default; a file given with ``--opt-config`` is read with the
  reference's rules: six required fields, the others defaulting to the
  built-in configuration, integers only.

Of the configuration, the front end's passes use ``small_inline_nodes``,
``small_clone_nodes``, the four fusion-guard thresholds and
``reduction_body_cse_min_occurrences``; the launch buckets and reduction
thresholds steer the reference's own kernel plans, which the B200 plan
replaces, and are recorded in the manifest only.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field, fields, replace
from typing import List, Optional, Sequence

FLAGS = (
    "scalar-const-fold", "normalized-dce", "if-simplify", "let-float", "lambda-inline-small",
    "scalar-cse", "arith-reassociate", "branch-hoist", "tensor-canonicalize",
    "reduction-input-simplify", "shape-use-simplify", "map-chain-collapse", "reduce-map-fusion",
    "small-producer-clone", "reduction-body-normalize", "tensor-cse", "elementwise-fusion",
    "scalar-hoist", "materialization-choice", "reduction-accumulator-shape",
    "reduction-reuse-hoist", "reduction-body-cse", "reduction-materialization-choice",
    "reduction-late-fusion-guard", "branch-aware-fusion-guard",
    "pointwise-materialization-guard", "reduction-plan-specialize",
    "elementwise-plan-specialize", "reduction-precombine", "reduction-two-phase",
    "launch-bucket-specialize", "reduction-classify", "reduction-tree-plan",
    "reduction-split-plan", "reduction-stage-sizing", "reduction-stage-balance",
    "reduction-partial-shape-pack", "reduction-class-aware-buckets",
    "reduction-small-plan-specialize", "reduction-body-canonicalize", "branchy-reduction-rescue",
    "temp-lifetime-pack", "storage-reuse-pack", "multi-use-fusion-guard", "pointwise-shape-plan",
    "shared-body-trait-analysis", "triton-reduction-instruction-select",
    "triton-pointwise-instruction-select", "triton-small-reduction-tail-tune",
    "cuda-reduction-norm-plan", "cuda-reduction-dot-plan", "cuda-reduction-weighted-product-plan",
    "cuda-reduction-pipeline-plan", "cuda-pointwise-small-shape-plan", "cuda-body-trait-analysis",
    "cuda-reduction-instruction-select", "cuda-specialized-combine",
    "cuda-pointwise-instruction-select", "cuda-pointwise-medium-plan",
    "cuda-pointwise-predicated-select", "cuda-pointwise-affine-vector-tail",
    "cuda-book-filter-register-plan", "cuda-pointwise-vectorize", "cuda-pointwise-tail-tune",
    "cuda-pointwise-selected-tail-plan", "cuda-reduction-shuffle", "cuda-reduction-tail-tune",
    "cuda-reduction-medium-tail-plan", "cuda-async-wrapper-return", "cuda-selected-profile")

_ORDER = {f: i for i, f in enumerate(FLAGS)}


class OptionsError(ValueError):
    """A flag or configuration ``loomc`` would reject."""


def in_catalogue_order(flags: Sequence[str]) -> List[str]:
    """Unique flags, in catalogue order (unknown names last, as given)."""
    seen = []
    for f in flags:
        if f not in seen:
            seen.append(f)
    return sorted(seen, key=lambda f: (_ORDER.get(f, len(FLAGS)), seen.index(f)))


def parse_cli_flags(enable: Sequence[str], disable: Sequence[str]) -> List[str]:
    """The enabled set: every ``--enable-opt`` flag, then every
    ``--disable-opt`` flag removed; an unknown name is an error
    (optimization_config.ml:182-206)."""
    for kind, names in (("enable", enable), ("disable", disable)):
        for name in names:
            if name not in _ORDER:
                raise OptionsError(f"unknown optimization flag {name} in --{kind}-opt")
    off = set(disable)
    return in_catalogue_order([f for f in enable if f not in off])


@dataclass(frozen=True)
class LaunchBucket:
    max_n: int
    block_size: int
    num_warps: int


def _buckets(*rows):
    return tuple(LaunchBucket(*r) for r in rows)


@dataclass(frozen=True)
class OptConfig:
    """Field order and names of optimization_config.ml:220-268."""
    version: int = 9
    small_inline_nodes: int = 20
    small_clone_nodes: int = 12
    reduction_precombine_max_body_complexity: int = 20
    single_block_reduction_threshold: int = 2048
    reduction_stage_split_threshold: int = 65536
    branchy_fusion_complexity_threshold: int = 6
    pointwise_materialization_complexity_threshold: int = 5
    materialize_multi_use_complexity_threshold: int = 4
    reduction_stage_medium_threshold: int = 4096
    reduction_stage_large_threshold: int = 131072
    small_direct_reduction_threshold: int = 131072
    small_partial_reduction_threshold: int = 262144
    small_reduction_program_count: int = 4
    branchy_small_reduction_threshold: int = 131072
    branchy_small_reduction_program_count: int = 4
    reduction_body_cse_min_occurrences: int = 2
    reduction_materialize_complexity_threshold: int = 5
    reduction_late_fusion_complexity_threshold: int = 8
    elementwise_buckets: tuple = _buckets((131072, 256, 4), (2097152, 512, 8),
                                          (2147483647, 1024, 8))
    reduction_buckets: tuple = _buckets((131072, 256, 4), (2097152, 512, 8),
                                        (2147483647, 1024, 8))
    source_path: Optional[str] = None

    def to_json(self) -> dict:
        out = {}
        for f in fields(self):
            v = getattr(self, f.name)
            if f.name.endswith("_buckets"):
                v = [{"max_n": b.max_n, "block_size": b.block_size, "num_warps": b.num_warps}
                     for b in v]
            out[f.name] = v
        return out


DEFAULT_CONFIG = OptConfig()

# The reference's built-in configuration (optimization_config.ml:5-40): what
# an optional field of a loaded file defaults to.
_BUILTIN = OptConfig(version=4, small_inline_nodes=18, reduction_precombine_max_body_complexity=18,
                     single_block_reduction_threshold=1024, reduction_stage_medium_threshold=8192,
                     reduction_stage_large_threshold=262144, small_direct_reduction_threshold=8192,
                     small_partial_reduction_threshold=131072, small_reduction_program_count=8,
                     reduction_buckets=_buckets((131072, 128, 4), (2097152, 256, 4),
                                                (2147483647, 512, 8)))
_REQUIRED = ("version", "small_inline_nodes", "reduction_precombine_max_body_complexity",
             "single_block_reduction_threshold", "elementwise_buckets", "reduction_buckets")


def _int(obj: dict, name: str) -> int:
    v = obj[name]
    if type(v) is not int:          # JSON 4.0 and true are not integers to Yojson
        raise OptionsError(f"expected integer field {name} in Loom optimization config")
    return v


def config_from_json(obj, source_path: Optional[str] = None) -> OptConfig:
    """optimization_config.ml:85-177."""
    if not isinstance(obj, dict):
        raise OptionsError("expected JSON object in Loom optimization config")
    for name in _REQUIRED:
        if name not in obj:
            raise OptionsError(f"missing Loom optimization config field {name}")
    values = {}
    for f in fields(OptConfig):
        name = f.name
        if name == "source_path" or name not in obj:
            continue
        if name.endswith("_buckets"):
            rows = obj[name]
            if not isinstance(rows, list):
                raise OptionsError(f"expected list field {name} in Loom optimization config")
            buckets = []
            for row in rows:
                if not isinstance(row, dict):
                    raise OptionsError("expected JSON object in Loom optimization config")
                for key in ("max_n", "block_size", "num_warps"):
                    if key not in row:
                        raise OptionsError(f"missing Loom optimization config field {key}")
                buckets.append(LaunchBucket(_int(row, "max_n"), _int(row, "block_size"),
                                            _int(row, "num_warps")))
            values[name] = tuple(buckets)
        else:
            values[name] = _int(obj, name)
    return replace(_BUILTIN, source_path=source_path, **values)


def load_config(path: str) -> OptConfig:
    with open(path, "r", encoding="utf-8") as fh:
        try:
            obj = json.load(fh)
        except ValueError as exc:
            raise OptionsError(f"{path}: {exc}") from None
    return config_from_json(obj, path)
