"""Scalar-expression rewrites that the reference's TensorIR passes are built
from (``src/loom_tensorize/reduction_analysis.ml``), and OCaml's float
arithmetic for constant folding.

Every rewrite keys expressions by their *rank* (``scalar_rank``,
``reduction_analysis.ml:3-28``): a string in which a unary's operator does
not appear, compared byte-wise as OCaml's ``String.compare`` does.  Equality
in the guards is OCaml's structural ``=`` (``==`` on TensorIR expressions,
IEEE on floats).  Constants are folded in double precision, as OCaml
evaluates them; the CUDA renderer prints the result with ``%.12g``.
"""

from __future__ import annotations

import math
from typing import List, Sequence

from .. import tensor_ir as TI
from .lower import body_metrics, scalar_rank

_INF = float("inf")
_NAN = float("nan")

# --- OCaml float arithmetic (IEEE double; Python raises where OCaml does not) --


def f_div(a: float, b: float) -> float:
    if b == 0.0:
        if a == 0.0 or math.isnan(a):
            return _NAN
        return math.copysign(_INF, a) * math.copysign(1.0, b)
    return a / b


def f_sqrt(v: float) -> float:
    return _NAN if v < 0.0 else math.sqrt(v)


def f_exp(v: float) -> float:
    try:
        return math.exp(v)
    except OverflowError:
        return _INF


def f_log(v: float) -> float:
    if v == 0.0:
        return -_INF
    if v < 0.0:
        return _NAN
    return math.log(v)


def f_min(a: float, b: float) -> float:
    """``Stdlib.min``: ``if a <= b then a else b``."""
    return a if a <= b else b


def f_max(a: float, b: float) -> float:
    """``Stdlib.max``: ``if a >= b then a else b``."""
    return a if a >= b else b


FOLD_UNARY = {"neg": lambda v: -v, "sqrt": f_sqrt, "exp": f_exp, "log": f_log}
FOLD_FLOAT = {"add": lambda a, b: a + b, "sub": lambda a, b: a - b,
              "mul": lambda a, b: a * b, "div": f_div, "min": f_min, "max": f_max}
FOLD_COMPARE = {"cmplt": lambda a, b: a < b, "cmple": lambda a, b: a <= b,
                "cmpgt": lambda a, b: a > b, "cmpge": lambda a, b: a >= b,
                "cmpeq": lambda a, b: a == b}

# --- canonical operand order (reduction_analysis.ml:30-57) ---------------------

_COMMUTATIVE = ("add", "mul", "min", "max", "cmpeq")


def canonicalize(e: TI.ScalarExpr) -> TI.ScalarExpr:
    """Operands of +, *, min, max and == in rank order; a select that picks
    the larger (smaller) of the two compared values becomes max (min)."""
    if isinstance(e, TI.SUnary):
        return TI.SUnary(e.op, canonicalize(e.expr))
    if isinstance(e, TI.SBinary):
        lhs, rhs = canonicalize(e.lhs), canonicalize(e.rhs)
        if e.op in _COMMUTATIVE and scalar_rank(lhs) > scalar_rank(rhs):
            lhs, rhs = rhs, lhs
        return TI.SBinary(e.op, lhs, rhs)
    if isinstance(e, TI.SSelect):
        c, t, f = canonicalize(e.cond), canonicalize(e.then), canonicalize(e.els)
        if isinstance(c, TI.SBinary) and c.op in ("cmpgt", "cmplt"):
            larger = "max" if c.op == "cmpgt" else "min"
            smaller = "min" if c.op == "cmpgt" else "max"
            if t == c.lhs and f == c.rhs:
                return canonicalize(TI.SBinary(larger, c.lhs, c.rhs))
            if t == c.rhs and f == c.lhs:
                return canonicalize(TI.SBinary(smaller, c.lhs, c.rhs))
        return TI.SSelect(c, t, f)
    return e


# --- algebraic simplification (reduction_analysis.ml:293-343) ------------------


def _f(e):
    return e.value if isinstance(e, TI.SConstF32) else None


def _b(e):
    return e.value if isinstance(e, TI.SConstBool) else None


def simplify(e: TI.ScalarExpr) -> TI.ScalarExpr:
    """Constant folding and the identities x+0, 0+x, x-0, x*0, 0*x, x*1,
    1*x, x/1, min(x,x), max(x,x), and selects on a constant condition or with
    equal arms.  A float pattern ``0.0`` matches -0.0 too, as OCaml compares
    float patterns by value; x*0 folds to 0 whatever x is."""
    if isinstance(e, TI.SUnary):
        x = simplify(e.expr)
        v = _f(x)
        if v is not None:
            return TI.SConstF32(FOLD_UNARY[e.op](v))
        return TI.SUnary(e.op, x)
    if isinstance(e, TI.SBinary):
        op = e.op
        lhs, rhs = simplify(e.lhs), simplify(e.rhs)
        a, b = _f(lhs), _f(rhs)
        if a is not None and b is not None:
            if op in FOLD_FLOAT:
                return TI.SConstF32(FOLD_FLOAT[op](a, b))
            return TI.SConstBool(FOLD_COMPARE[op](a, b))
        if op == "cmpeq" and _b(lhs) is not None and _b(rhs) is not None:
            return TI.SConstBool(_b(lhs) == _b(rhs))
        if op == "add" and a == 0.0:
            return rhs
        if op == "add" and b == 0.0:
            return lhs
        if op == "sub" and b == 0.0:
            return lhs
        if op == "mul" and (a == 0.0 or b == 0.0):
            return TI.SConstF32(0.0)
        if op == "mul" and a == 1.0:
            return rhs
        if op == "mul" and b == 1.0:
            return lhs
        if op == "div" and b == 1.0:
            return lhs
        if op in ("min", "max") and lhs == rhs:
            return lhs
        return TI.SBinary(op, lhs, rhs)
    if isinstance(e, TI.SSelect):
        c, t, f = simplify(e.cond), simplify(e.then), simplify(e.els)
        cv = _b(c)
        if cv is True:
            return t
        if cv is False:
            return f
        if t == f:
            return t
        return TI.SSelect(c, t, f)
    return e


# --- products and reduction bodies (reduction_analysis.ml:59-138) -------------


def flatten_mul_terms(e) -> List[TI.ScalarExpr]:
    if isinstance(e, TI.SBinary) and e.op == "mul":
        return flatten_mul_terms(e.lhs) + flatten_mul_terms(e.rhs)
    return [e]


def rebuild_mul_terms(terms: Sequence[TI.ScalarExpr]) -> TI.ScalarExpr:
    if not terms:
        return TI.SConstF32(1.0)
    acc = terms[0]
    for t in terms[1:]:
        acc = TI.SBinary("mul", acc, t)
    return acc


def _is_scalar_param(scalar_params, e) -> bool:
    return isinstance(e, TI.SVar) and e.name in scalar_params


def _partition(pred, items):
    yes = [x for x in items if pred(x)]
    no = [x for x in items if not pred(x)]
    return yes, no


def normalize_mul_expr(scalar_params, e) -> TI.ScalarExpr:
    """A product's factors: the data factors in rank order, then the scalar
    parameters in rank order."""
    terms = [canonicalize(t) for t in flatten_mul_terms(e)]
    scalars, data = _partition(lambda t: _is_scalar_param(scalar_params, t), terms)
    order = lambda ts: sorted(ts, key=scalar_rank)
    return rebuild_mul_terms(order(data) + order(scalars))


def canonicalize_reduction_body(scalar_params, e) -> TI.ScalarExpr:
    if isinstance(e, TI.SUnary):
        return TI.SUnary(e.op, canonicalize_reduction_body(scalar_params, e.expr))
    if isinstance(e, TI.SBinary):
        lhs = canonicalize_reduction_body(scalar_params, e.lhs)
        rhs = canonicalize_reduction_body(scalar_params, e.rhs)
        if e.op == "mul":
            return normalize_mul_expr(scalar_params, TI.SBinary("mul", lhs, rhs))
        return canonicalize(TI.SBinary(e.op, lhs, rhs))
    if isinstance(e, TI.SSelect):
        return canonicalize(TI.SSelect(canonicalize_reduction_body(scalar_params, e.cond),
                                       canonicalize_reduction_body(scalar_params, e.then),
                                       canonicalize_reduction_body(scalar_params, e.els)))
    return e


def branchy_weighted_rescue_body(scalar_params, body) -> TI.ScalarExpr:
    """``c ? d*w1 : d*w2`` (one scalar weight per arm, equal data factors)
    becomes ``d * (c ? w1 : w2)``."""
    body = canonicalize_reduction_body(scalar_params, body)

    def split(e):
        factors = [canonicalize(t) for t in flatten_mul_terms(e)]
        scalars, data = _partition(lambda t: _is_scalar_param(scalar_params, t), factors)
        if not data or not scalars or len(scalars) != 1:
            return None
        return rebuild_mul_terms(data), scalars[0]

    if isinstance(body, TI.SSelect):
        a, b = split(body.then), split(body.els)
        if a is not None and b is not None and a[0] == b[0]:
            return rebuild_mul_terms([a[0], TI.SSelect(canonicalize(body.cond), a[1], b[1])])
    return body


def repeated_subexpressions(e) -> int:
    return body_metrics(0, e).repeated_subexpressions


def reduction_body_cse_expr(e) -> TI.ScalarExpr:
    """Bottom-up: x+x -> 2*x, x-x -> 0, a select with equal arms -> the arm
    (reduction_analysis.ml:345-365)."""
    if isinstance(e, TI.SUnary):
        e = TI.SUnary(e.op, reduction_body_cse_expr(e.expr))
    elif isinstance(e, TI.SBinary):
        e = TI.SBinary(e.op, reduction_body_cse_expr(e.lhs), reduction_body_cse_expr(e.rhs))
    elif isinstance(e, TI.SSelect):
        e = TI.SSelect(reduction_body_cse_expr(e.cond), reduction_body_cse_expr(e.then),
                       reduction_body_cse_expr(e.els))
    if isinstance(e, TI.SBinary) and e.lhs == e.rhs:
        if e.op == "add":
            return simplify(TI.SBinary("mul", TI.SConstF32(2.0), e.lhs))
        if e.op == "sub":
            return TI.SConstF32(0.0)
        if e.op == "mul":
            return simplify(TI.SBinary("mul", e.lhs, e.rhs))
    if isinstance(e, TI.SSelect) and e.then == e.els:
        return e.then
    return e


# --- body patterns and the metrics annotation uses (:238-282) ------------------


def classify_reduction_body_pattern(scalar_params, body) -> str:
    body = canonicalize_reduction_body(scalar_params, body)
    scalars, data = _partition(lambda t: _is_scalar_param(scalar_params, t),
                               flatten_mul_terms(body))
    tensor_term = lambda e: isinstance(e, TI.SVar) and e.name not in scalar_params
    difference = lambda e: isinstance(e, TI.SBinary) and e.op == "sub" and e.lhs != e.rhs
    if len(data) == 2:
        lhs, rhs = data
        if tensor_term(lhs) and tensor_term(rhs):
            return "weighted-dot-like" if scalars else "dot-like"
        if lhs == rhs and difference(lhs):
            return "weighted-squared-difference" if scalars else "squared-difference"
    return "generic"


def adjusted_reduction_body_metrics(scalar_params, use_count, body) -> TI.BodyMetrics:
    body = canonicalize_reduction_body(scalar_params, body)
    m = body_metrics(use_count, body)
    pattern = classify_reduction_body_pattern(scalar_params, body)
    if pattern == "dot-like":
        m.scalar_complexity, m.repeated_subexpressions = min(m.scalar_complexity, 1), 0
    elif pattern == "weighted-dot-like":
        m.scalar_complexity, m.repeated_subexpressions = min(m.scalar_complexity, 2), 0
    elif pattern == "squared-difference":
        m.scalar_complexity, m.repeated_subexpressions = max(2, m.scalar_complexity - 1), 0
    elif pattern == "weighted-squared-difference":
        m.scalar_complexity, m.repeated_subexpressions = max(3, m.scalar_complexity - 1), 0
    return m
