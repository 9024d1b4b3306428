"""B200 kernel plan: one fused streaming kernel per Loom entry.

The reference plans a list of steps per entry (one kernel per element-wise
node, a first-stage reduction plus a host loop of combine kernels, temporary
buffers for intermediates; ``src/loom_core/kernel_plan.ml``,
``src/loom_backend_cuda/cuda_plan.ml:763-1028``) and fuses only under
optimisation flags (``src/loom_tensorize/tensor_passes.ml:130-335``).

On B200 every supported entry is HBM-bound, so the plan is always the same
shape: the entry's result is computed by ONE kernel that reads each distinct
tensor parameter once and writes the result once.  Every element-wise node
reachable from the result is inlined into that kernel at *register* level:
each node is evaluated into its own ``float`` temporary, exactly as if it had
been materialised to an fp32 buffer, so fusing never changes a bit of a map
result (the substitution-style fusion of the reference can re-associate
``fmaf`` patterns across node boundaries; this never does).  Multi-use
producers are evaluated once per element and reused from the register.

The body traits and reduction family of the reference
(``src/loom_core/kernel_plan_common.ml:213-415``) are computed for the
manifest and plan dump; they do not change the kernel, since the same
streaming loop is optimal for every body here.
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from . import render
from .tensor_ir import (Elementwise1D, InputBinding, MappedInput, NodeRef, ParamRef,
                        PlainInput, Program, Reduce1D, SBinary, SSelect, ScalarExpr,
                        TensorIRError, complexity, expr_any, free_vars)

_IDENT = re.compile(r"[^A-Za-z0-9_]")


def c_ident(name: str) -> str:
    """User variable -> C identifier that cannot collide with generated names."""
    return "v_" + _IDENT.sub("_", name)


def sanitize_ident(text: str) -> str:
    """Symbol-name sanitiser (src/loom_backend_cuda/cuda_backend.ml:180-188)."""
    return "".join(ch if ch.isascii() and ch.isalnum() else "_" for ch in text.lower())


def symbol_name(module_name: str, entry_name: str) -> str:
    """``loom_<module>_<entry>`` (cuda_backend.ml:210-213)."""
    return f"loom_{module_name}_{sanitize_ident(entry_name)}"


@dataclass
class NodeBlock:
    """One inlined element-wise node: bind its inputs, evaluate, keep in a temp."""
    node_id: Optional[int]          # None for the mapped source of a reduction
    temp: str                       # C name of the fp32 result
    bindings: List[Tuple[str, str]]  # (C name of lambda var, C expression it reads)
    lines: List[str]                # render_value_lines output, target "value"
    body: ScalarExpr


@dataclass
class EntryPlan:
    program: Program
    module_name: str
    symbol: str
    kind: str                        # "map" | "reduce"
    reduce_kind: Optional[str]       # "sum" | "max" for reductions
    slots: List[str]                 # tensor params read by the kernel, in slot order
    scalar_args: List[str]           # scalar params captured by the body, in param order
    blocks: List[NodeBlock]
    result_expr: str                 # C expression of the per-element value
    traits: List[str] = field(default_factory=list)
    family: str = ""
    fused_node_ids: List[int] = field(default_factory=list)

    @property
    def workspace_symbol(self) -> str:
        return self.symbol + "_workspace_size"

    @property
    def uses_workspace(self) -> bool:
        return self.kind == "reduce"

    @property
    def bytes_per_element(self) -> int:
        """Algorithmic HBM bytes per element: each input read once, the
        tensor result written once (a scalar result is not counted)."""
        return 4 * (len(self.slots) + (1 if self.kind == "map" else 0))

    @property
    def result_kind(self) -> str:
        return self.program.result_kind


def _has_minmax(e):
    return expr_any(e, lambda x: isinstance(x, SBinary) and x.op in ("min", "max"))


def _has_div(e):
    return expr_any(e, lambda x: isinstance(x, SBinary) and x.op == "div")


def _has_mul(e):
    return expr_any(e, lambda x: isinstance(x, SBinary) and x.op == "mul")


def _has_select(e):
    return expr_any(e, lambda x: isinstance(x, SSelect))


def _has_addsub(e):
    return expr_any(e, lambda x: isinstance(x, SBinary) and x.op in ("add", "sub"))


def pointwise_traits(n_inputs: int, scalar_params, body) -> List[str]:
    """Body traits of an element-wise body (kernel_plan_common.ml:213-235)."""
    branch, div = _has_select(body), _has_div(body)
    t = []

    def add(cond, name):
        if cond and name not in t:
            t.append(name)

    add(n_inputs == 1 and bool(scalar_params) and branch, "threshold")
    add(n_inputs == 1 and not scalar_params and (branch or _has_minmax(body)), "simple-activation")
    add(n_inputs == 2 and div and not branch, "ratio-book")
    add(n_inputs == 2 and div and branch, "mixed-filter-ratio")
    add(n_inputs == 1 and branch, "activation-or-threshold")
    add(n_inputs == 2 and branch, "filter-or-book")
    add(n_inputs == 2 and not branch, "affine-vector-update")
    add(bool(scalar_params) and _has_addsub(body), "affine")
    add(_has_mul(body), "mul")
    add(div, "ratio")
    add(branch, "branch")
    add(_has_minmax(body), "clip")
    return t


def reduction_family(inputs, scalar_params, body) -> str:
    """Reduction family of a mapped body, following the base family of
    kernel_plan_common.ml:351-374 and the specialisations at :324-349."""
    from .tensor_ir import SVar
    if body is None:
        return "plain"
    names = [b.name for b in inputs]
    if len(names) == 1 and not scalar_params and isinstance(body, SBinary) and body.op == "mul" \
            and body.lhs == SVar(names[0]) and body.rhs == SVar(names[0]):
        return "norm-square"
    if len(names) == 2 and not scalar_params and isinstance(body, SBinary) and body.op == "mul" \
            and {body.lhs, body.rhs} == {SVar(names[0]), SVar(names[1])}:
        return "dot-product"
    if isinstance(body, SBinary) and body.op == "mul" and body.lhs == body.rhs \
            and isinstance(body.lhs, SBinary) and body.lhs.op == "sub" \
            and not _has_select(body) and not _has_div(body):
        return "delta-square"
    if _has_select(body):
        return "branchy"
    if _has_div(body):
        return "ratio"
    if scalar_params:
        return "weighted"
    return "mapped"


TRAIT_FLAGS = {"cuda-body-trait-analysis", "shared-body-trait-analysis"}


def node_render_flags(enabled, n_inputs: int, scalar_params, body) -> render.RenderFlags:
    """Rendering switches of one element-wise node under the enabled reference
    flags (the per-step derivation of src/loom_backend_cuda/cuda_backend.ml:
    1310-1345; body traits exist only under a trait-analysis flag,
    src/loom_backend_cuda/cuda_plan.ml:785-792)."""
    enabled = set(enabled or ())
    tail = "cuda-pointwise-tail-tune" in enabled
    pred = "cuda-pointwise-predicated-select" in enabled
    sel_tail = "cuda-pointwise-selected-tail-plan" in enabled
    traits = pointwise_traits(n_inputs, scalar_params, body) if enabled & TRAIT_FLAGS else []

    def has(t):
        return t in traits

    affine_threshold_clamp = has("affine") and has("threshold") and n_inputs == 1
    affine_clip_threshold = affine_threshold_clamp and has("clip")
    pred_body = pred and not (sel_tail and affine_clip_threshold) and (
        affine_threshold_clamp or not (has("threshold") and not has("clip")))
    return render.RenderFlags(
        tail_tune=tail,
        predicated_select=pred_body,
        fast_divide=sel_tail and has("ratio-book") and not has("branch"),
        eager_select_then=tail and has("mixed-filter-ratio"),
    )


class _Builder:
    def __init__(self, prog: Program, enabled=()):
        self.prog = prog
        self.enabled = set(enabled)
        self.slots: List[str] = []
        self.blocks: List[NodeBlock] = []
        self.temps: Dict[int, str] = {}
        self.scalars_used: set = set()
        self.fused: List[int] = []

    def slot_expr(self, param: str) -> str:
        if param not in self.slots:
            self.slots.append(param)
        return f"in[{self.slots.index(param)}]"

    def value(self, ref) -> str:
        if isinstance(ref, ParamRef):
            return self.slot_expr(ref.name)
        if ref.id in self.temps:
            return self.temps[ref.id]
        node = self.prog.node(ref.id)
        if not isinstance(node, Elementwise1D):
            raise TensorIRError(f"{self.prog.entry_name}: node_{ref.id} is not element-wise")
        temp = self.block(node.id, node.inputs, node.scalar_params, node.body)
        self.temps[node.id] = temp
        self.fused.append(node.id)
        return temp

    def block(self, node_id, inputs, scalar_params, body) -> str:
        bindings = []
        for b in inputs:
            bindings.append((c_ident(b.name), self.value(b.source)))
        self.scalars_used.update(scalar_params)
        # Mapped reduction bodies always render with the defaults
        # (cuda_backend.ml:1071-1085); element-wise nodes take the flags.
        flags = (node_render_flags(self.enabled, len(inputs), scalar_params, body)
                 if node_id is not None else render.DEFAULT_FLAGS)
        lines = render.render_value_lines(body, c_ident, flags=flags)
        temp = f"t{len(self.blocks)}"
        self.blocks.append(NodeBlock(node_id, temp, bindings, lines, body))
        return temp


def plan_entry(prog: Program, module_name: str, enabled=()) -> EntryPlan:
    """Plan one entry; `enabled` holds the reference optimisation flags (only
    the body-rendering ones change the generated code)."""
    b = _Builder(prog, enabled)
    traits: List[str] = []
    family = ""
    if prog.result_kind == "tensor":
        kind, rkind = "map", None
        result_expr = b.value(prog.result)
        if isinstance(prog.result, NodeRef):
            node = prog.node(prog.result.id)
            traits = pointwise_traits(len(node.inputs), node.scalar_params, node.body)
            family = "pointwise"
        else:
            family = "copy"
    else:
        red = prog.node(prog.result.id)
        assert isinstance(red, Reduce1D)
        kind, rkind = "reduce", red.kind
        if isinstance(red.source, PlainInput):
            result_expr = b.value(red.source.input)
            src = red.source.input
            if isinstance(src, NodeRef):
                n = prog.node(src.id)
                family = reduction_family(n.inputs, n.scalar_params, n.body)
            else:
                family = "plain"
        else:
            ms: MappedInput = red.source
            result_expr = b.block(None, ms.inputs, ms.scalar_params, ms.body)
            family = reduction_family(ms.inputs, ms.scalar_params, ms.body)
        traits = [f"reduce-{rkind}"]
    scalar_order = [p.name for p in prog.scalar_params if p.name in b.scalars_used]
    # Every scalar parameter the body reads must be an entry parameter.
    for s in b.scalars_used:
        if s not in [p.name for p in prog.scalar_params]:
            raise TensorIRError(f"{prog.entry_name}: body captures unknown scalar {s!r}")
    return EntryPlan(program=prog, module_name=module_name, symbol=symbol_name(module_name,
                     prog.entry_name), kind=kind, reduce_kind=rkind, slots=b.slots,
                     scalar_args=scalar_order, blocks=b.blocks, result_expr=result_expr,
                     traits=traits, family=family, fused_node_ids=b.fused)


def plan_to_json(plan: EntryPlan) -> dict:
    """The B200 plan, written to entries/<symbol>/cuda_plan.json."""
    return {
        "backend": "loom-b200",
        "arch": "sm_100a",
        "entry_name": plan.program.entry_name,
        "symbol_name": plan.symbol,
        "kernel_kind": plan.kind,
        "reduce_kind": plan.reduce_kind,
        "family": plan.family,
        "traits": plan.traits,
        "tensor_slots": plan.slots,
        "scalar_args": plan.scalar_args,
        "fused_nodes": [f"node_{i}" for i in plan.fused_node_ids],
        "launches_per_call": 1 if plan.kind == "map" else 2,
        "hbm_bytes_per_element": plan.bytes_per_element,
        "temporaries": 0,
        "workspace": "reduction partials + rank scratch" if plan.uses_workspace else "none",
    }
