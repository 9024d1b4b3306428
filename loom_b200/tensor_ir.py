"""TensorIR: the input boundary of the B200 backend.

This is the program form that Loom's front end hands to a backend after
tensorization: a list of 1D float32 nodes (``elementwise1d`` maps and
``reduce1d`` reductions) over one symbolic extent ``n``.  The data model and
its JSON form follow the reference's ``src/loom_core/tensor_ir.mli:1-114``
(types) and ``src/loom_core/tensor_ir.ml:119-252`` (JSON writer), so a
``tensor_ir.json`` written by ``loomc ... --emit tensor-ir`` loads here
unchanged, and a program written here reads back in the reference.

Scalar expressions are frozen dataclasses whose ``==`` is OCaml's
structural ``=`` (``expr_eq``), which the reference's pattern guards use
(``lhs = then_expr`` and the like) and the renderer and passes rely on.
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from typing import Iterable, List, Optional, Sequence, Tuple, Union

# ---------------------------------------------------------------------------
# scalar expressions (tensor_ir.mli:1-26)

UNARY_OPS = ("neg", "sqrt", "exp", "log")
BINARY_OPS = ("add", "sub", "mul", "div", "min", "max",
              "cmplt", "cmple", "cmpgt", "cmpge", "cmpeq")
COMPARE_OPS = ("cmplt", "cmple", "cmpgt", "cmpge", "cmpeq")


class _Expr:
    """Equality of scalar expressions is OCaml's structural ``=``
    (``expr_eq``); the hash agrees with it."""

    __slots__ = ()

    def __eq__(self, other):
        return expr_eq(self, other)

    def __ne__(self, other):
        return not expr_eq(self, other)

    def __hash__(self):
        return hash(_expr_key(self))


@dataclass(frozen=True, eq=False)
class SVar(_Expr):
    name: str


@dataclass(frozen=True, eq=False)
class SConstF32(_Expr):
    # The reference stores the literal as an OCaml float (a double); the
    # CUDA renderer prints it with "%.12g", so keep the double here.
    value: float


@dataclass(frozen=True, eq=False)
class SConstBool(_Expr):
    value: bool


@dataclass(frozen=True, eq=False)
class SUnary(_Expr):
    op: str
    expr: "ScalarExpr"


@dataclass(frozen=True, eq=False)
class SBinary(_Expr):
    op: str
    lhs: "ScalarExpr"
    rhs: "ScalarExpr"


@dataclass(frozen=True, eq=False)
class SSelect(_Expr):
    cond: "ScalarExpr"
    then: "ScalarExpr"
    els: "ScalarExpr"


def expr_eq(a, b) -> bool:
    """OCaml's structural ``=`` on two scalar expressions: constructors and
    fields compared recursively, floats as IEEE values (-0.0 = 0.0, a NaN
    equals nothing, not even itself -- Python's tuple comparison would let
    one NaN object equal itself, so no tuple comparison is used here)."""
    if type(a) is not type(b):
        return False
    if isinstance(a, SConstF32):
        return a.value == b.value
    if isinstance(a, SVar):
        return a.name == b.name
    if isinstance(a, SConstBool):
        return a.value == b.value
    if isinstance(a, SUnary):
        return a.op == b.op and expr_eq(a.expr, b.expr)
    if isinstance(a, SBinary):
        return a.op == b.op and expr_eq(a.lhs, b.lhs) and expr_eq(a.rhs, b.rhs)
    if isinstance(a, SSelect):
        return expr_eq(a.cond, b.cond) and expr_eq(a.then, b.then) and expr_eq(a.els, b.els)
    return a == b


def _expr_key(e):
    if isinstance(e, SConstF32):
        return ("f", e.value)          # hash(-0.0) == hash(0.0)
    if isinstance(e, SVar):
        return ("v", e.name)
    if isinstance(e, SConstBool):
        return ("b", e.value)
    if isinstance(e, SUnary):
        return ("u", e.op, _expr_key(e.expr))
    if isinstance(e, SBinary):
        return ("b2", e.op, _expr_key(e.lhs), _expr_key(e.rhs))
    return ("s", _expr_key(e.cond), _expr_key(e.then), _expr_key(e.els))


ScalarExpr = Union[SVar, SConstF32, SConstBool, SUnary, SBinary, SSelect]


def free_vars(expr: ScalarExpr) -> List[str]:
    """Sorted unique free variables (tensor_ir.ml:119-130)."""
    out = set()

    def walk(e):
        if isinstance(e, SVar):
            out.add(e.name)
        elif isinstance(e, SUnary):
            walk(e.expr)
        elif isinstance(e, SBinary):
            walk(e.lhs)
            walk(e.rhs)
        elif isinstance(e, SSelect):
            walk(e.cond)
            walk(e.then)
            walk(e.els)

    walk(expr)
    return sorted(out)


def complexity(expr: ScalarExpr) -> int:
    """Operator count, as ``kernel_plan_common.ml`` scores bodies."""
    if isinstance(expr, (SVar, SConstF32, SConstBool)):
        return 0
    if isinstance(expr, SUnary):
        return 1 + complexity(expr.expr)
    if isinstance(expr, SBinary):
        return 1 + complexity(expr.lhs) + complexity(expr.rhs)
    return 1 + complexity(expr.cond) + complexity(expr.then) + complexity(expr.els)


def expr_any(expr: ScalarExpr, pred) -> bool:
    if pred(expr):
        return True
    if isinstance(expr, SUnary):
        return expr_any(expr.expr, pred)
    if isinstance(expr, SBinary):
        return expr_any(expr.lhs, pred) or expr_any(expr.rhs, pred)
    if isinstance(expr, SSelect):
        return (expr_any(expr.cond, pred) or expr_any(expr.then, pred)
                or expr_any(expr.els, pred))
    return False


# ---------------------------------------------------------------------------
# program structure (tensor_ir.mli:27-105)

@dataclass(frozen=True)
class ParamRef:
    name: str


@dataclass(frozen=True)
class NodeRef:
    id: int


ValueRef = Union[ParamRef, NodeRef]


@dataclass(frozen=True)
class ScalarParam:
    name: str


@dataclass(frozen=True)
class TensorParam:
    name: str
    shape_symbol: str = "n"


Param = Union[ScalarParam, TensorParam]


@dataclass(frozen=True)
class InputBinding:
    name: str
    source: ValueRef


@dataclass
class BodyMetrics:
    scalar_complexity: int = 0
    has_branch: bool = False
    has_div: bool = False
    branch_count: int = 0
    div_count: int = 0
    repeated_subexpressions: int = 0
    estimated_uses: int = 0


@dataclass(frozen=True)
class PlainInput:
    input: ValueRef


@dataclass(frozen=True)
class MappedInput:
    inputs: Tuple[InputBinding, ...]
    scalar_params: Tuple[str, ...]
    body: ScalarExpr


ReductionSource = Union[PlainInput, MappedInput]


@dataclass
class Elementwise1D:
    id: int
    inputs: Tuple[InputBinding, ...]
    scalar_params: Tuple[str, ...]
    body: ScalarExpr
    shape_symbol: str = "n"
    metrics: BodyMetrics = field(default_factory=BodyMetrics)
    handling_hint: str = "no-preference"


@dataclass
class Reduce1D:
    id: int
    source: ReductionSource
    kind: str  # "sum" | "max"
    shape_symbol: str = "n"
    metrics: BodyMetrics = field(default_factory=BodyMetrics)
    reduction_shape: str = "plain"
    handling_hint: str = "no-preference"


Node = Union[Elementwise1D, Reduce1D]


@dataclass
class Program:
    entry_name: str
    params: List[Param]
    result_kind: str  # "tensor" | "scalar"
    result: ValueRef
    nodes: List[Node]

    def node(self, node_id: int) -> Node:
        for n in self.nodes:
            if n.id == node_id:
                return n
        raise TensorIRError(f"{self.entry_name}: reference to missing node_{node_id}")

    @property
    def tensor_params(self) -> List[TensorParam]:
        return [p for p in self.params if isinstance(p, TensorParam)]

    @property
    def scalar_params(self) -> List[ScalarParam]:
        return [p for p in self.params if isinstance(p, ScalarParam)]


class TensorIRError(ValueError):
    """A TensorIR document that the backend cannot accept."""


# ---------------------------------------------------------------------------
# JSON reader

def _expr_from_json(obj) -> ScalarExpr:
    kind = obj.get("kind")
    if kind == "var":
        return SVar(obj["name"])
    if kind == "f32":
        return SConstF32(float(obj["value"]))
    if kind == "bool":
        return SConstBool(bool(obj["value"]))
    if kind == "unary":
        if obj["op"] not in UNARY_OPS:
            raise TensorIRError(f"unknown unary op {obj['op']!r}")
        return SUnary(obj["op"], _expr_from_json(obj["expr"]))
    if kind == "binary":
        if obj["op"] not in BINARY_OPS:
            raise TensorIRError(f"unknown binary op {obj['op']!r}")
        return SBinary(obj["op"], _expr_from_json(obj["lhs"]), _expr_from_json(obj["rhs"]))
    if kind == "select":
        return SSelect(_expr_from_json(obj["cond"]), _expr_from_json(obj["then"]),
                       _expr_from_json(obj["else"]))
    raise TensorIRError(f"unknown scalar expression kind {kind!r}")


def _ref_from_json(text, param_names) -> ValueRef:
    # tensor_ir.ml:119-121 writes NodeRef as "node_<id>" and ParamRef as the name.
    if isinstance(text, int):
        return NodeRef(text)
    if text in param_names:
        return ParamRef(text)
    if text.startswith("node_") and text[5:].isdigit():
        return NodeRef(int(text[5:]))
    return ParamRef(text)


def _metrics_from_json(obj) -> BodyMetrics:
    if not obj:
        return BodyMetrics()
    return BodyMetrics(**{k: obj[k] for k in BodyMetrics.__dataclass_fields__ if k in obj})


def program_from_json(obj) -> Program:
    if isinstance(obj, (str, bytes)):
        obj = json.loads(obj)
    params: List[Param] = []
    for p in obj["params"]:
        if p["kind"] == "scalar-f32":
            params.append(ScalarParam(p["name"]))
        elif p["kind"] == "tensor1-f32":
            params.append(TensorParam(p["name"], p.get("shape_symbol", "n")))
        else:
            raise TensorIRError(f"unsupported parameter kind {p['kind']!r}")
    names = {p.name for p in params}
    nodes: List[Node] = []
    for n in obj["nodes"]:
        if n["kind"] == "elementwise1d":
            nodes.append(Elementwise1D(
                id=int(n["id"]),
                inputs=tuple(InputBinding(b["name"], _ref_from_json(b["source"], names))
                             for b in n["inputs"]),
                scalar_params=tuple(n.get("scalar_params", [])),
                body=_expr_from_json(n["body"]),
                shape_symbol=n.get("shape_symbol", "n"),
                metrics=_metrics_from_json(n.get("metrics")),
                handling_hint=n.get("handling_hint", "no-preference"),
            ))
        elif n["kind"] == "reduce1d":
            src = n["source"]
            if src["kind"] == "plain":
                source: ReductionSource = PlainInput(_ref_from_json(src["input"], names))
            elif src["kind"] == "mapped":
                source = MappedInput(
                    inputs=tuple(InputBinding(b["name"], _ref_from_json(b["source"], names))
                                 for b in src["inputs"]),
                    scalar_params=tuple(src.get("scalar_params", [])),
                    body=_expr_from_json(src["body"]),
                )
            else:
                raise TensorIRError(f"unknown reduction source kind {src['kind']!r}")
            kind = n["reduce_kind"]
            if kind not in ("sum", "max"):
                raise TensorIRError(f"unknown reduce kind {kind!r}")
            nodes.append(Reduce1D(
                id=int(n["id"]), source=source, kind=kind,
                shape_symbol=n.get("shape_symbol", "n"),
                metrics=_metrics_from_json(n.get("metrics")),
                reduction_shape=n.get("reduction_shape", "plain"),
                handling_hint=n.get("handling_hint", "no-preference"),
            ))
        else:
            raise TensorIRError(f"unknown node kind {n['kind']!r}")
    res = obj["result"]
    if res["kind"] not in ("tensor", "scalar"):
        raise TensorIRError(f"unknown result kind {res['kind']!r}")
    prog = Program(entry_name=obj["entry_name"], params=params, result_kind=res["kind"],
                   result=_ref_from_json(res["value"], names), nodes=nodes)
    validate(prog)
    return prog


def load_program(path) -> Program:
    with open(path, "r", encoding="utf-8") as fh:
        return program_from_json(json.load(fh))


# ---------------------------------------------------------------------------
# JSON writer (tensor_ir.ml:132-252)

def _expr_to_json(e: ScalarExpr):
    if isinstance(e, SVar):
        return {"kind": "var", "name": e.name}
    if isinstance(e, SConstF32):
        return {"kind": "f32", "value": e.value}
    if isinstance(e, SConstBool):
        return {"kind": "bool", "value": e.value}
    if isinstance(e, SUnary):
        return {"kind": "unary", "op": e.op, "expr": _expr_to_json(e.expr)}
    if isinstance(e, SBinary):
        return {"kind": "binary", "op": e.op, "lhs": _expr_to_json(e.lhs),
                "rhs": _expr_to_json(e.rhs)}
    return {"kind": "select", "cond": _expr_to_json(e.cond), "then": _expr_to_json(e.then),
            "else": _expr_to_json(e.els)}


def _ref_to_json(r: ValueRef) -> str:
    return r.name if isinstance(r, ParamRef) else f"node_{r.id}"


def _metrics_to_json(m: BodyMetrics):
    return {k: getattr(m, k) for k in BodyMetrics.__dataclass_fields__}


def program_to_json(prog: Program) -> dict:
    params = []
    for p in prog.params:
        if isinstance(p, ScalarParam):
            params.append({"kind": "scalar-f32", "name": p.name})
        else:
            params.append({"kind": "tensor1-f32", "name": p.name, "shape_symbol": p.shape_symbol})
    nodes = []
    for n in prog.nodes:
        if isinstance(n, Elementwise1D):
            nodes.append({
                "kind": "elementwise1d", "id": n.id, "shape_symbol": n.shape_symbol,
                "inputs": [{"name": b.name, "source": _ref_to_json(b.source)} for b in n.inputs],
                "scalar_params": list(n.scalar_params), "body": _expr_to_json(n.body),
                "metrics": _metrics_to_json(n.metrics), "handling_hint": n.handling_hint,
            })
        else:
            if isinstance(n.source, PlainInput):
                src = {"kind": "plain", "input": _ref_to_json(n.source.input)}
            else:
                src = {"kind": "mapped",
                       "inputs": [{"name": b.name, "source": _ref_to_json(b.source)}
                                  for b in n.source.inputs],
                       "scalar_params": list(n.source.scalar_params),
                       "body": _expr_to_json(n.source.body)}
            nodes.append({
                "kind": "reduce1d", "id": n.id, "shape_symbol": n.shape_symbol, "source": src,
                "reduce_kind": n.kind, "metrics": _metrics_to_json(n.metrics),
                "reduction_shape": n.reduction_shape, "handling_hint": n.handling_hint,
            })
    return {"entry_name": prog.entry_name, "params": params,
            "result": {"kind": prog.result_kind, "value": _ref_to_json(prog.result)},
            "nodes": nodes}


def program_to_string(prog: Program) -> str:
    return json.dumps(program_to_json(prog), indent=2)


# ---------------------------------------------------------------------------
# validation (the checks of src/loom_tensorize/validate.ml plus the
# structural rules the CUDA backend assumes)

def validate(prog: Program) -> None:
    names = [p.name for p in prog.params]
    if len(set(names)) != len(names):
        raise TensorIRError(f"{prog.entry_name}: duplicate parameter names")
    tensor_names = {p.name for p in prog.tensor_params}
    scalar_names = {p.name for p in prog.scalar_params}
    ids = [n.id for n in prog.nodes]
    if len(set(ids)) != len(ids):
        raise TensorIRError(f"{prog.entry_name}: duplicate node ids")
    by_id = {n.id: n for n in prog.nodes}

    def check_tensor_ref(ref: ValueRef, where: str):
        if isinstance(ref, ParamRef):
            if ref.name not in tensor_names:
                raise TensorIRError(f"{prog.entry_name}: {where} reads {ref.name!r}, "
                                    "which is not a tensor parameter")
        else:
            node = by_id.get(ref.id)
            if node is None:
                raise TensorIRError(f"{prog.entry_name}: {where} reads missing node_{ref.id}")
            if not isinstance(node, Elementwise1D):
                raise TensorIRError(f"{prog.entry_name}: {where} reads reduction node_{ref.id} "
                                    "as a tensor")

    def check_body(inputs, scalars, body, where):
        bound = {b.name for b in inputs} | set(scalars)
        for s in scalars:
            if s not in scalar_names:
                raise TensorIRError(f"{prog.entry_name}: {where} captures {s!r}, which is not "
                                    "a scalar parameter")
        for v in free_vars(body):
            if v not in bound:
                raise TensorIRError(f"{prog.entry_name}: {where} uses unbound variable {v!r}")
        for b in inputs:
            check_tensor_ref(b.source, where)

    for n in prog.nodes:
        where = f"node_{n.id}"
        if isinstance(n, Elementwise1D):
            if not n.inputs:
                raise TensorIRError(f"{prog.entry_name}: {where} has no tensor inputs")
            check_body(n.inputs, n.scalar_params, n.body, where)
            for b in n.inputs:
                if isinstance(b.source, NodeRef) and b.source.id >= n.id:
                    raise TensorIRError(f"{prog.entry_name}: {where} reads a later node")
        else:
            if isinstance(n.source, PlainInput):
                check_tensor_ref(n.source.input, where)
            else:
                if not n.source.inputs:
                    raise TensorIRError(f"{prog.entry_name}: {where} has no tensor inputs")
                check_body(n.source.inputs, n.source.scalar_params, n.source.body, where)
    if prog.result_kind == "tensor":
        check_tensor_ref(prog.result, "result")
    else:
        if not isinstance(prog.result, NodeRef) or not isinstance(by_id.get(prog.result.id), Reduce1D):
            raise TensorIRError(f"{prog.entry_name}: a scalar result must be a reduction node")
