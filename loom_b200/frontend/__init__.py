"""Front end for Loom's Python entry language: source -> FrontIR -> LoomLambda
-> TensorIR, so that ``package`` and ``compile`` accept Python projects the
way ``loomc --target cuda`` does, without the OCaml toolchain."""

from __future__ import annotations

from typing import List, Tuple

from .. import tensor_ir as TI
from .lower import loom_lambda, program_from_front_ir, tensor_ir
from .python_front import FrontendError, front_ir, list_entries


def front_ir_stages(front: dict, enabled=(), cfg=None) -> Tuple[dict, dict, TI.Program]:
    """One FrontIR entry through normalize and tensorize: (FrontIR,
    LoomLambda, TensorIR), with the passes that `enabled` switches on and
    the thresholds of `cfg` (``loom_b200.optconfig.OptConfig``)."""
    lam = loom_lambda(front, enabled, cfg)
    return front, lam, tensor_ir(lam, enabled, cfg)


def python_stages(path: str, enabled=(), cfg=None) -> List[Tuple[dict, dict, TI.Program]]:
    """Every ``@loom.entry`` of a Python source file: its FrontIR, LoomLambda
    and TensorIR."""
    with open(path, "r", encoding="utf-8") as fh:
        src = fh.read()
    return [front_ir_stages(front_ir(src, e["name"], path), enabled, cfg)
            for e in list_entries(src, path)]


def python_programs(path: str, enabled=(), cfg=None) -> List[TI.Program]:
    """Every ``@loom.entry`` of a Python source file, lowered to TensorIR
    (with the passes that the flags in `enabled` switch on)."""
    return [prog for _, _, prog in python_stages(path, enabled, cfg)]


__all__ = ["FrontendError", "front_ir", "list_entries", "loom_lambda", "tensor_ir",
           "program_from_front_ir", "front_ir_stages", "python_stages", "python_programs"]
