"""In-tree build of the shipped benchmark-suite package.

``build_suite()`` packages ``loom_b200/suite`` (the five workload
configurations of the hot path, module ``kernels``) into
``loom_b200/_built/b200_suite/`` with the reference's default flags (so the
plain entry points synchronise like the reference's); ``load_suite()`` loads
it.  The built ``.so`` stays in the tree so that it travels with the
repository to the GPU machine.
"""

from __future__ import annotations

import os

from . import artifact
from .loader import Package

HERE = os.path.dirname(os.path.abspath(__file__))
SUITE_PROJECT = os.path.join(HERE, "suite")
BUILT_DIR = os.path.join(HERE, "_built")
SUITE_DIR = os.path.join(BUILT_DIR, "b200_suite")


# Reference flags that change how map bodies are rendered; the body-coverage
# test project is also packaged with them (as frontend_cases_flags).
# the reference's TensorIR fusion passes (restated in loom_b200/frontend/passes.py)
FUSION_FLAGS = ["map-chain-collapse", "reduce-map-fusion", "shape-use-simplify"]
RENDER_FLAGS = ["cuda-pointwise-tail-tune", "cuda-pointwise-predicated-select",
                "cuda-pointwise-selected-tail-plan", "cuda-body-trait-analysis"]
# The flag set of the reference harness's tuned CUDA profile, "loom_cuda_fixed"
# (experiments/source/data/profiles/loom_profiles.json): its scalar and
# TensorIR passes (restated in loom_b200/frontend/), its fusion, and its
# rendering flags.
CUDA_FIXED_FLAGS = [
    "scalar-const-fold", "if-simplify", "arith-reassociate", "lambda-inline-small", "scalar-cse",
    "normalized-dce", "tensor-canonicalize", "reduction-input-simplify",
    "reduction-body-normalize", "reduction-body-canonicalize", "reduction-accumulator-shape",
    "reduction-reuse-hoist", "reduction-body-cse", "map-chain-collapse", "reduce-map-fusion",
    "shape-use-simplify", "tensor-cse", "materialization-choice",
    "reduction-materialization-choice", "reduction-plan-specialize", "reduction-classify",
    "reduction-tree-plan", "reduction-split-plan", "reduction-small-plan-specialize",
    "reduction-stage-sizing", "reduction-stage-balance", "reduction-partial-shape-pack",
    "reduction-class-aware-buckets", "shared-body-trait-analysis", "cuda-body-trait-analysis",
    "cuda-reduction-instruction-select", "cuda-reduction-tail-tune", "cuda-reduction-norm-plan",
    "cuda-reduction-dot-plan", "cuda-reduction-weighted-product-plan",
    "cuda-pointwise-small-shape-plan", "cuda-pointwise-medium-plan",
    "cuda-pointwise-predicated-select", "cuda-pointwise-selected-tail-plan",
    "cuda-pointwise-vectorize", "cuda-pointwise-tail-tune", "cuda-reduction-shuffle",
    "cuda-reduction-medium-tail-plan", "cuda-async-wrapper-return", "cuda-selected-profile",
    "storage-reuse-pack", "launch-bucket-specialize"]


def SUITE_OPTIONS() -> artifact.Options:
    """Reference default flags, plus the static-scratch variant of dot."""
    return artifact.Options(noalloc_entries=["dot"])


def _newest_source_mtime() -> float:
    newest = 0.0
    for root in (SUITE_PROJECT, os.path.join(HERE, "csrc"), HERE, os.path.join(HERE, "frontend")):
        for name in os.listdir(root):
            path = os.path.join(root, name)
            if os.path.isfile(path):
                newest = max(newest, os.path.getmtime(path))
    return newest


def suite_is_current() -> bool:
    lib = os.path.join(SUITE_DIR, "libb200_suite.so")
    return os.path.exists(lib) and os.path.getmtime(lib) >= _newest_source_mtime()


def build_suite(force: bool = False) -> artifact.PackageResult:
    if not force and suite_is_current():
        return None
    return artifact.generate_package(SUITE_PROJECT, SUITE_DIR, SUITE_OPTIONS())


def load_suite() -> Package:
    lib = os.path.join(SUITE_DIR, "libb200_suite.so")
    if not os.path.exists(lib):
        raise FileNotFoundError(
            f"{lib} is missing: build it with `python -c 'import loom_b200.build as b; "
            "b.build_suite()'` (needs nvcc)")
    return Package(SUITE_DIR)


def build_project(project_dir: str, force: bool = False, enabled=(), name: str = None) -> str:
    """Package any project into ``loom_b200/_built/<name>/`` (default: the
    package name) with the given reference flags, and return that directory;
    skipped when the library is newer than the project's sources and the
    backend."""
    pkg = name or artifact.package_name_of_root(project_dir)
    out = os.path.join(BUILT_DIR, pkg)
    lib = os.path.join(out, f"lib{pkg}.so")
    newest = _newest_source_mtime()
    for root, _, files in os.walk(project_dir):
        for f in files:
            newest = max(newest, os.path.getmtime(os.path.join(root, f)))
    if force or not os.path.exists(lib) or os.path.getmtime(lib) < newest:
        artifact.generate_package(project_dir, out, artifact.Options(enabled=list(enabled)),
                                  package_name=pkg)
    return out
