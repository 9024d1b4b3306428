"""Scalar-body rendering: TensorIR scalar expressions -> CUDA C++ statements.

The text a body renders to fixes its bitwise result (which products contract
into ``fmaf``, which selects become ``fmaxf``/``fminf``, which literals are
``double`` and so promote the arithmetic around them).  For a B200 build to
give the same bits as the reference's generated kernels, bodies are rendered
with the reference's rules, restated here:

* literals: ``cpp_float`` (``src/loom_backend_cuda/cuda_backend.ml:348-350``)
* expressions: ``render_scalar_expr_with`` (``cuda_backend.ml:446-527``),
  including the ``fmaf`` contraction patterns (``:471-491``) and the
  zero-max/min ternaries (``:502-513``, ``:352-363``)
* the select/clamp/square rewrites of ``render_value_lines``
  (``cuda_backend.ml:614-848``), with ``render_scalar_expr_replacing``
  (``:529-600``) for the guard form.

Deliberate differences, all outside the default flag set:

* the generated kernels are compiled with ``-fmad=false``: only the
  ``fmaf`` calls written here contract.  (The reference builds with nvcc's
  default ``-fmad=true``; its rendered text already spells every mul-add
  pattern as ``fmaf``, so the two agree except where a product reaches an add
  through a negation or a select.)
* ``cuda-plain-mul-add`` renders the same ``fmaf`` as the default: the
  reference prints ``a*b+c`` there and relies on nvcc's contraction, which
  gives the same bits.
* a literal whose ``%.12g`` text has an exponent or is not finite is printed
  as a valid C++ double literal (the reference would print e.g.
  ``1e-07.0f``, which does not compile).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, List, Optional

from .tensor_ir import (SBinary, SConstBool, SConstF32, SSelect, SUnary, SVar,
                        ScalarExpr)


@dataclass(frozen=True)
class RenderFlags:
    """CUDA body-rendering switches (reference optimisation flags)."""

    # cuda-pointwise-tail-tune: soft-threshold select rewrite (cuda_backend.ml:386-421)
    tail_tune: bool = False
    # cuda-pointwise-predicated-select: copysignf soft threshold (:423-444)
    predicated_select: bool = False
    # cuda-fast-divide policy: __fdividef (:498-501)
    fast_divide: bool = False
    # eager select-then form (:776-787)
    eager_select_then: bool = False


DEFAULT_FLAGS = RenderFlags()


def cpp_float(value: float) -> str:
    """Literal text for a float constant (cuda_backend.ml:348-350)."""
    if math.isnan(value):
        return "(0.0/0.0)"
    if math.isinf(value):
        return "(1.0/0.0)" if value > 0 else "(-1.0/0.0)"
    text = "%.12g" % value
    if "." in text:
        return text
    if "e" in text:
        return text  # double literal; see module docstring
    return text + ".0f"


def is_zero_const(e: ScalarExpr) -> bool:
    return isinstance(e, SConstF32) and e.value == 0.0


def is_inline_ternary_value(e: ScalarExpr) -> bool:
    return isinstance(e, (SVar, SConstF32, SConstBool))


def is_simple(e: ScalarExpr) -> bool:
    return isinstance(e, (SVar, SConstF32, SConstBool))


def _zero_max(text: str) -> str:
    return f"(({text}) > 0.0f ? {text} : 0.0f)"


def _zero_min(text: str) -> str:
    return f"(({text}) < 0.0f ? {text} : 0.0f)"


_CMP = {"cmplt": "<", "cmple": "<=", "cmpgt": ">", "cmpge": ">=", "cmpeq": "=="}


# --- soft-threshold select (cuda_backend.ml:365-421) -------------------------

def _is_negated(threshold, e) -> bool:
    if isinstance(e, SUnary) and e.op == "neg":
        return e.expr == threshold
    if isinstance(e, SBinary) and e.op == "sub":
        return is_zero_const(e.lhs) and e.rhs == threshold
    return False


def _gt_threshold(value, threshold, cond) -> bool:
    if isinstance(cond, SBinary) and cond.op == "cmpgt":
        return cond.lhs == value and cond.rhs == threshold
    if isinstance(cond, SBinary) and cond.op == "cmplt":
        return cond.lhs == threshold and cond.rhs == value
    return False


def _lt_neg_threshold(value, threshold, cond) -> bool:
    return (isinstance(cond, SBinary) and cond.op == "cmplt" and cond.lhs == value
            and _is_negated(threshold, cond.rhs))


def _add_uses(lhs, rhs, value, threshold) -> bool:
    return (lhs == value and rhs == threshold) or (lhs == threshold and rhs == value)


def soft_threshold_select(e):
    if not isinstance(e, SSelect):
        return None
    inner = e.els
    if (isinstance(e.then, SBinary) and e.then.op == "sub" and isinstance(inner, SSelect)
            and isinstance(inner.then, SBinary) and inner.then.op == "add"):
        value, threshold = e.then.lhs, e.then.rhs
        if (_gt_threshold(value, threshold, e.cond)
                and _lt_neg_threshold(value, threshold, inner.cond)
                and _add_uses(inner.then.lhs, inner.then.rhs, value, threshold)
                and is_zero_const(inner.els)):
            return value, threshold
    if (isinstance(e.then, SBinary) and e.then.op == "add" and isinstance(inner, SSelect)
            and isinstance(inner.then, SBinary) and inner.then.op == "sub"):
        value, threshold = inner.then.lhs, inner.then.rhs
        if value == e.then.lhs or value == e.then.rhs:
            if (_lt_neg_threshold(value, threshold, e.cond)
                    and _gt_threshold(value, threshold, inner.cond)
                    and _add_uses(e.then.lhs, e.then.rhs, value, threshold)
                    and is_zero_const(inner.els)):
                return value, threshold
    return None


def _soft_text(v: str, t: str) -> str:
    return (f"((({v}) > ({t})) ? (({v}) - ({t})) : ((({v}) < -({t})) ? (({v}) + ({t})) : "
            f"0.0f))")


# --- expressions -------------------------------------------------------------

class ExprRenderer:
    """``render_scalar_expr_with`` for one variable-naming function."""

    def __init__(self, var: Callable[[str], str], flags: RenderFlags = DEFAULT_FLAGS):
        self.var = var
        self.flags = flags

    def __call__(self, e: ScalarExpr) -> str:
        r = self
        if self.flags.tail_tune:
            st = soft_threshold_select(e)
            if st is not None:
                return _soft_text(r(st[0]), r(st[1]))
        if isinstance(e, SVar):
            return self.var(e.name)
        if isinstance(e, SConstF32):
            return cpp_float(e.value)
        if isinstance(e, SConstBool):
            return "true" if e.value else "false"
        if isinstance(e, SUnary):
            fn = {"neg": None, "sqrt": "sqrtf", "exp": "expf", "log": "logf"}[e.op]
            return f"(-({r(e.expr)}))" if fn is None else f"{fn}({r(e.expr)})"
        if isinstance(e, SSelect):
            return f"(({r(e.cond)}) ? ({r(e.then)}) : ({r(e.els)}))"
        op, lhs, rhs = e.op, e.lhs, e.rhs
        if op == "add":
            if isinstance(lhs, SBinary) and lhs.op == "mul":
                return f"fmaf({r(lhs.lhs)}, {r(lhs.rhs)}, {r(rhs)})"
            if isinstance(rhs, SBinary) and rhs.op == "mul":
                return f"fmaf({r(rhs.lhs)}, {r(rhs.rhs)}, {r(lhs)})"
            return f"(({r(lhs)}) + ({r(rhs)}))"
        if op == "sub":
            if isinstance(lhs, SBinary) and lhs.op == "mul":
                return f"fmaf({r(lhs.lhs)}, {r(lhs.rhs)}, -({r(rhs)}))"
            if isinstance(rhs, SBinary) and rhs.op == "mul":
                return f"fmaf(-({r(rhs.lhs)}), {r(rhs.rhs)}, {r(lhs)})"
            return f"(({r(lhs)}) - ({r(rhs)}))"
        if op == "mul":
            return f"(({r(lhs)}) * ({r(rhs)}))"
        if op == "div":
            if self.flags.fast_divide:
                return f"__fdividef({r(lhs)}, {r(rhs)})"
            return f"(({r(lhs)}) / ({r(rhs)}))"
        if op in ("min", "max"):
            tern = _zero_min if op == "min" else _zero_max
            fn = "fminf" if op == "min" else "fmaxf"
            if is_zero_const(lhs) and is_inline_ternary_value(rhs):
                return tern(r(rhs))
            if is_zero_const(rhs) and is_inline_ternary_value(lhs):
                return tern(r(lhs))
            return f"{fn}({r(lhs)}, {r(rhs)})"
        return f"(({r(lhs)}) {_CMP[op]} ({r(rhs)}))"


def render_replacing(var, replaced: ScalarExpr, replacement: str, e: ScalarExpr) -> str:
    """``render_scalar_expr_replacing`` (cuda_backend.ml:529-600): default
    rules, with every occurrence of ``replaced`` printed as ``replacement``."""
    def r(x):
        return render_replacing(var, replaced, replacement, x)

    if e == replaced:
        return replacement
    if isinstance(e, SVar):
        return var(e.name)
    if isinstance(e, SConstF32):
        return cpp_float(e.value)
    if isinstance(e, SConstBool):
        return "true" if e.value else "false"
    if isinstance(e, SUnary):
        fn = {"neg": None, "sqrt": "sqrtf", "exp": "expf", "log": "logf"}[e.op]
        return f"(-({r(e.expr)}))" if fn is None else f"{fn}({r(e.expr)})"
    if isinstance(e, SSelect):
        return f"(({r(e.cond)}) ? ({r(e.then)}) : ({r(e.els)}))"
    op, lhs, rhs = e.op, e.lhs, e.rhs
    if op == "add":
        if isinstance(lhs, SBinary) and lhs.op == "mul":
            return f"fmaf({r(lhs.lhs)}, {r(lhs.rhs)}, {r(rhs)})"
        if isinstance(rhs, SBinary) and rhs.op == "mul":
            return f"fmaf({r(rhs.lhs)}, {r(rhs.rhs)}, {r(lhs)})"
    if op == "sub":
        if isinstance(lhs, SBinary) and lhs.op == "mul":
            return f"fmaf({r(lhs.lhs)}, {r(lhs.rhs)}, -({r(rhs)}))"
        if isinstance(rhs, SBinary) and rhs.op == "mul":
            return f"fmaf(-({r(rhs.lhs)}), {r(rhs.rhs)}, {r(lhs)})"
    a, b = r(lhs), r(rhs)
    if op == "add":
        return f"(({a}) + ({b}))"
    if op == "sub":
        return f"(({a}) - ({b}))"
    if op == "mul":
        return f"(({a}) * ({b}))"
    if op == "div":
        return f"(({a}) / ({b}))"
    if op in ("min", "max"):
        tern = _zero_min if op == "min" else _zero_max
        fn = "fminf" if op == "min" else "fmaxf"
        if is_zero_const(lhs) and is_inline_ternary_value(rhs):
            return tern(b)
        if is_zero_const(rhs) and is_inline_ternary_value(lhs):
            return tern(a)
        return f"{fn}({a}, {b})"
    return f"(({a}) {_CMP[op]} ({b}))"


# --- statement forms (render_value_lines) ------------------------------------

def _contains(needle, e) -> bool:
    if e == needle:
        return True
    if isinstance(e, SUnary):
        return _contains(needle, e.expr)
    if isinstance(e, SBinary):
        return _contains(needle, e.lhs) or _contains(needle, e.rhs)
    if isinstance(e, SSelect):
        return _contains(needle, e.cond) or _contains(needle, e.then) or _contains(needle, e.els)
    return False


def select_clamps_compared_value(e):
    """(value, low, high) for the four clamp shapes (cuda_backend.ml:686-719)."""
    if not isinstance(e, SSelect) or not isinstance(e.cond, SBinary):
        return None
    c, t, el = e.cond, e.then, e.els
    if c.op == "cmplt" and isinstance(el, SSelect) and isinstance(el.cond, SBinary) \
            and el.cond.op == "cmpgt":
        lv, lb, hv, hb = c.lhs, c.rhs, el.cond.lhs, el.cond.rhs
        if lb == t and hb == el.then and lv == hv and lv == el.els:
            return lv, lb, hb
    if c.op == "cmpgt" and isinstance(el, SSelect) and isinstance(el.cond, SBinary) \
            and el.cond.op == "cmplt":
        hv, hb, lv, lb = c.lhs, c.rhs, el.cond.lhs, el.cond.rhs
        if hb == t and lb == el.then and hv == lv and hv == el.els:
            return hv, lb, hb
    if c.op == "cmplt" and isinstance(el, SBinary) and el.op == "min":
        lv, lb = c.lhs, c.rhs
        if lb == t and lv == el.lhs:
            return lv, lb, el.rhs
    if c.op == "cmpgt" and isinstance(el, SBinary) and el.op == "max":
        hv, hb = c.lhs, c.rhs
        if hb == t and hv == el.lhs:
            return hv, el.rhs, hb
    return None


def select_reuses_compared_subexpr(e):
    """(reused, op, reused_on_lhs, other, then, else) (cuda_backend.ml:665-684)."""
    if isinstance(e, SSelect) and isinstance(e.cond, SBinary) and e.cond.op in _CMP:
        c = e.cond
        if not is_simple(c.lhs) and _contains(c.lhs, e.then):
            return c.lhs, c.op, True, c.rhs, e.then, e.els
        if not is_simple(c.rhs) and _contains(c.rhs, e.then):
            return c.rhs, c.op, False, c.lhs, e.then, e.els
    return None


def select_reuses_compared_value(e):
    """(reused, op, reused_on_lhs, other, else) (cuda_backend.ml:614-635)."""
    if isinstance(e, SSelect) and isinstance(e.cond, SBinary) and e.cond.op in _CMP:
        c = e.cond
        if c.lhs == e.then:
            return c.lhs, c.op, True, c.rhs, e.els
        if c.rhs == e.then:
            return c.rhs, c.op, False, c.lhs, e.els
    return None


def minmax_for_reused_select(op: str, on_lhs: bool) -> Optional[str]:
    """cuda_backend.ml:637-645."""
    if op in ("cmplt", "cmple"):
        return "fminf" if on_lhs else "fmaxf"
    if op in ("cmpgt", "cmpge"):
        return "fmaxf" if on_lhs else "fminf"
    return None


def render_value_lines(body: ScalarExpr, var: Callable[[str], str], target: str = "value",
                       flags: RenderFlags = DEFAULT_FLAGS) -> List[str]:
    """Statements that declare ``float <target>`` = body (cuda_backend.ml:721-848)."""
    render = ExprRenderer(var, flags)
    clamp = select_clamps_compared_value(body)
    if clamp is not None:
        v, lo, hi = clamp
        raw = target + "_unclamped"
        if flags.tail_tune and not flags.predicated_select:
            return [f"float {target} = {render(v)};",
                    f"if ({target} < {render(lo)}) {target} = {render(lo)};",
                    f"if ({target} > {render(hi)}) {target} = {render(hi)};"]
        return [f"float {raw} = {render(v)};",
                f"float {target} = fminf(fmaxf({raw}, {render(lo)}), {render(hi)});"]
    if flags.predicated_select:
        st = soft_threshold_select(body)
        if st is not None:
            v, t = render(st[0]), render(st[1])
            return [f"float {target} = ((({t}) >= 0.0f) ? copysignf(fmaxf(fabsf({v}) - ({t}), "
                    f"0.0f), {v}) : ({_soft_text(v, t)}));"]
    sub = select_reuses_compared_subexpr(body)
    if sub is not None:
        reused, op, on_lhs, other, then_e, else_e = sub
        guard = target + "_guard"

        def rr(x):
            return render_replacing(var, reused, guard, x)

        lhs, rhs = (guard, rr(other)) if on_lhs else (rr(other), guard)
        lines = [f"float {guard} = {render(reused)};"]
        if flags.eager_select_then:
            cand = target + "_candidate"
            lines += [f"float {cand} = {rr(then_e)};",
                      f"float {target} = (({lhs}) {_CMP[op]} ({rhs})) ? {cand} : ({rr(else_e)});"]
        else:
            lines.append(f"float {target} = (({lhs}) {_CMP[op]} ({rhs})) ? ({rr(then_e)}) : "
                         f"({rr(else_e)});")
        return lines
    val = select_reuses_compared_value(body)
    if val is not None:
        reused, op, on_lhs, other, else_e = val
        sel = target + "_selected_value"
        lines = [f"float {sel} = {render(reused)};"]
        fn = minmax_for_reused_select(op, on_lhs)
        if fn is not None and else_e == other:
            lines.append(f"float {target} = {fn}({sel}, {render(other)});")
        else:
            lhs, rhs = (sel, render(other)) if on_lhs else (render(other), sel)
            lines.append(f"float {target} = (({lhs}) {_CMP[op]} ({rhs})) ? {sel} : "
                         f"({render(else_e)});")
        return lines
    if isinstance(body, SBinary) and body.op == "mul" and body.lhs == body.rhs \
            and not is_simple(body.lhs):
        fac = target + "_factor"
        return [f"float {fac} = {render(body.lhs)};", f"float {target} = {fac} * {fac};"]
    return [f"float {target} = {render(body)};"]
