"""Front end for Loom's Python entry language: source -> FrontIR -> LoomLambda
-> TensorIR, so that ``package`` and ``compile`` accept Python projects the
way ``loomc --target cuda`` does, without the OCaml toolchain."""

from __future__ import annotations

from typing import List, Tuple

from .. import tensor_ir as TI
from .lower import loom_lambda, program_from_front_ir, tensor_ir
from .python_front import FrontendError, front_ir, list_entries


def python_programs(path: str, enabled=()) -> List[TI.Program]:
    """Every ``@loom.entry`` of a Python source file, lowered to TensorIR
    (with the TensorIR passes that the flags in `enabled` switch on)."""
    with open(path, "r", encoding="utf-8") as fh:
        src = fh.read()
    return [program_from_front_ir(front_ir(src, e["name"], path), enabled)
            for e in list_entries(src, path)]


__all__ = ["FrontendError", "front_ir", "list_entries", "loom_lambda", "tensor_ir",
           "program_from_front_ir", "python_programs"]
