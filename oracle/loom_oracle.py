"""CPU oracle for the Loom hot path -- TEST INFRASTRUCTURE, not product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg (and its ``--impl reference`` arm) may import this module.  It never runs
on the product path: the product is the CUDA code in ``loom_b200``.

What it restates
----------------
The reference has no CPU evaluator (``src/loom_stdlib/tensor1.ml:5-13``
raises "staged primitive"); the meaning of an entry is the CUDA its backend
emits.  This oracle restates that meaning as plain C, compiled by gcc with
strict IEEE float semantics (``-O2 -ffp-contract=off -fno-fast-math`` on
x86-64 SSE, so every ``float`` expression rounds exactly as CUDA's does):

* each scalar body is printed with the reference's emission rules --
  literals ``cpp_float`` (``src/loom_backend_cuda/cuda_backend.ml:348-350``),
  expressions ``render_scalar_expr_with`` (``:446-527``) with its ``fmaf``
  contraction patterns (``:471-491``) and zero ternaries (``:502-513``),
  statements ``render_value_lines`` (``:721-848``) with the clamp
  (``:686-719``), guard (``:665-684``, ``render_scalar_expr_replacing``
  ``:529-600``), reused-value min/max (``:614-645``) and square (``:831-841``)
  forms;
* each element-wise node is evaluated per element into an fp32 value, in node
  order, which is exactly the reference's unfused execution (one kernel per
  node writing an fp32 buffer; ``cuda_backend.ml:1308-1387``);
* ``reduce_sum`` is returned as an fp64 Neumaier-compensated sum of the fp32
  per-element values (the "fp64 reference sum" the tolerance is taken
  against); ``reduce_max`` folds with CUDA's ``fmaxf`` from ``-INFINITY``
  (``cuda_backend.ml:999-1005``), exact in any order.

The C math the rendered text calls is defined in ``oracle_semantics.h``.

Pinning
-------
The reference's generated code cannot be built here (its compiler is OCaml,
which this image lacks), so the oracle cannot be compared with the
reference's own outputs.  It is pinned instead by (tests/test_oracle.py):
the reference's own runtime tests' expectations (``test/python/
test_package.py:66-131``, ``test/python/test_cli.py:374-407``: saxpy and dot
at n=4096, rtol 1e-4 against a*x+y and sum(x*y)), exact-rational known
answers for the rendering semantics (single-rounding ``fmaf``, relu,
clamp), and the reference's golden TensorIR (``test/golden/
l2_norm_sq_tensor_ir.json``).  Bit-level parity with the reference's own
binaries is therefore unpinned; bit-level parity with the restated rules is
what the CUDA tests check.
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import math
import os
import subprocess
from typing import Dict, List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")

# ---------------------------------------------------------------------------
# rendering restatement (operates on TensorIR JSON dicts)

_CMP = {"cmplt": "<", "cmple": "<=", "cmpgt": ">", "cmpge": ">=", "cmpeq": "=="}


def cpp_float(value: float) -> str:
    """cuda_backend.ml:348-350 ("%.12g", '.0f' appended when there is no '.')."""
    if value != value:
        return "(0.0/0.0)"
    if value in (float("inf"), float("-inf")):
        return "(1.0/0.0)" if value > 0 else "(-1.0/0.0)"
    text = "%.12g" % value
    if "." in text or "e" in text:
        return text
    return text + ".0f"


def _eq(a, b) -> bool:
    """OCaml's structural '=' on two expressions: floats compare as IEEE
    values (-0.0 = 0.0, NaN equals nothing), everything else by value."""
    if a["kind"] != b["kind"]:
        return False
    k = a["kind"]
    if k == "f32":
        return float(a["value"]) == float(b["value"])
    if k in ("var",):
        return a["name"] == b["name"]
    if k == "bool":
        return bool(a["value"]) == bool(b["value"])
    if k == "unary":
        return a["op"] == b["op"] and _eq(a["expr"], b["expr"])
    if k == "binary":
        return a["op"] == b["op"] and _eq(a["lhs"], b["lhs"]) and _eq(a["rhs"], b["rhs"])
    return _eq(a["cond"], b["cond"]) and _eq(a["then"], b["then"]) and _eq(a["else"], b["else"])


def _is_zero(e) -> bool:
    return e["kind"] == "f32" and float(e["value"]) == 0.0


def _is_leaf(e) -> bool:
    return e["kind"] in ("var", "f32", "bool")


def _is_bin(e, op=None) -> bool:
    return e["kind"] == "binary" and (op is None or e["op"] == op)


def _soft_threshold(e):
    """(value, threshold) when e is a soft-threshold select
    (cuda_backend.ml:365-421), else None."""
    if e["kind"] != "select" or e["else"]["kind"] != "select":
        return None
    outer, inner = e, e["else"]

    def gt(v, t, c):      # v > t, also written t < v
        return _is_bin(c) and ((c["op"] == "cmpgt" and _eq(c["lhs"], v) and _eq(c["rhs"], t))
                               or (c["op"] == "cmplt" and _eq(c["lhs"], t) and _eq(c["rhs"], v)))

    def lt_neg(v, t, c):  # v < -t, the negation written -t or 0 - t
        if not (_is_bin(c, "cmplt") and _eq(c["lhs"], v)):
            return False
        m = c["rhs"]
        return ((m["kind"] == "unary" and m["op"] == "neg" and _eq(m["expr"], t))
                or (_is_bin(m, "sub") and _is_zero(m["lhs"]) and _eq(m["rhs"], t)))

    def sums(a, b, v, t):
        return (_eq(a, v) and _eq(b, t)) or (_eq(a, t) and _eq(b, v))

    if _is_bin(outer["then"], "sub") and _is_bin(inner["then"], "add"):
        v, t = outer["then"]["lhs"], outer["then"]["rhs"]
        if (gt(v, t, outer["cond"]) and lt_neg(v, t, inner["cond"])
                and sums(inner["then"]["lhs"], inner["then"]["rhs"], v, t)
                and _is_zero(inner["else"])):
            return v, t
    if _is_bin(outer["then"], "add") and _is_bin(inner["then"], "sub"):
        v, t = inner["then"]["lhs"], inner["then"]["rhs"]
        if ((_eq(v, outer["then"]["lhs"]) or _eq(v, outer["then"]["rhs"]))
                and lt_neg(v, t, outer["cond"]) and gt(v, t, inner["cond"])
                and sums(outer["then"]["lhs"], outer["then"]["rhs"], v, t)
                and _is_zero(inner["else"])):
            return v, t
    return None


def _soft_text(v, t):
    return f"((({v}) > ({t})) ? (({v}) - ({t})) : ((({v}) < -({t})) ? (({v}) + ({t})) : 0.0f))"


def render_expr(e, var, flags=None) -> str:
    """render_scalar_expr_with (cuda_backend.ml:446-527); `flags` may carry
    tail_tune (soft-threshold rewrite) and fast_divide."""
    flags = flags or {}

    def r(x):
        return render_expr(x, var, flags)

    if flags.get("tail_tune"):
        st = _soft_threshold(e)
        if st is not None:
            return _soft_text(r(st[0]), r(st[1]))
    k = e["kind"]
    if k == "var":
        return var(e["name"])
    if k == "f32":
        return cpp_float(float(e["value"]))
    if k == "bool":
        return "true" if e["value"] else "false"
    if k == "unary":
        inner = r(e["expr"])
        return {"neg": f"(-({inner}))", "sqrt": f"sqrtf({inner})",
                "exp": f"expf({inner})", "log": f"logf({inner})"}[e["op"]]
    if k == "select":
        return f"(({r(e['cond'])}) ? ({r(e['then'])}) : ({r(e['else'])}))"
    op, lhs, rhs = e["op"], e["lhs"], e["rhs"]
    if op == "add" and _is_bin(lhs, "mul"):
        return f"fmaf({r(lhs['lhs'])}, {r(lhs['rhs'])}, {r(rhs)})"
    if op == "add" and _is_bin(rhs, "mul"):
        return f"fmaf({r(rhs['lhs'])}, {r(rhs['rhs'])}, {r(lhs)})"
    if op == "sub" and _is_bin(lhs, "mul"):
        return f"fmaf({r(lhs['lhs'])}, {r(lhs['rhs'])}, -({r(rhs)}))"
    if op == "sub" and _is_bin(rhs, "mul"):
        return f"fmaf(-({r(rhs['lhs'])}), {r(rhs['rhs'])}, {r(lhs)})"
    if op == "div" and flags.get("fast_divide"):
        return f"__fdividef({r(lhs)}, {r(rhs)})"
    if op in ("add", "sub", "mul", "div"):
        sym = {"add": "+", "sub": "-", "mul": "*", "div": "/"}[op]
        return f"(({r(lhs)}) {sym} ({r(rhs)}))"
    if op in ("min", "max"):
        cmp_sym = "<" if op == "min" else ">"
        if _is_zero(lhs) and _is_leaf(rhs):
            t = r(rhs)
            return f"(({t}) {cmp_sym} 0.0f ? {t} : 0.0f)"
        if _is_zero(rhs) and _is_leaf(lhs):
            t = r(lhs)
            return f"(({t}) {cmp_sym} 0.0f ? {t} : 0.0f)"
        return f"{'fminf' if op == 'min' else 'fmaxf'}({r(lhs)}, {r(rhs)})"
    return f"(({r(lhs)}) {_CMP[op]} ({r(rhs)}))"


def render_replacing(e, var, replaced, replacement) -> str:
    """render_scalar_expr_replacing (cuda_backend.ml:529-600)."""
    if _eq(e, replaced):
        return replacement
    k = e["kind"]
    if k != "binary" or e["op"] not in ("add", "sub", "mul", "div", "min", "max", *_CMP):
        if k in ("var", "f32", "bool"):
            return render_expr(e, var)
        if k == "unary":
            inner = render_replacing(e["expr"], var, replaced, replacement)
            return {"neg": f"(-({inner}))", "sqrt": f"sqrtf({inner})",
                    "exp": f"expf({inner})", "log": f"logf({inner})"}[e["op"]]
        c = render_replacing(e["cond"], var, replaced, replacement)
        t = render_replacing(e["then"], var, replaced, replacement)
        f = render_replacing(e["else"], var, replaced, replacement)
        return f"(({c}) ? ({t}) : ({f}))"

    def r(x):
        return render_replacing(x, var, replaced, replacement)

    op, lhs, rhs = e["op"], e["lhs"], e["rhs"]
    if op == "add" and _is_bin(lhs, "mul"):
        return f"fmaf({r(lhs['lhs'])}, {r(lhs['rhs'])}, {r(rhs)})"
    if op == "add" and _is_bin(rhs, "mul"):
        return f"fmaf({r(rhs['lhs'])}, {r(rhs['rhs'])}, {r(lhs)})"
    if op == "sub" and _is_bin(lhs, "mul"):
        return f"fmaf({r(lhs['lhs'])}, {r(lhs['rhs'])}, -({r(rhs)}))"
    if op == "sub" and _is_bin(rhs, "mul"):
        return f"fmaf(-({r(rhs['lhs'])}), {r(rhs['rhs'])}, {r(lhs)})"
    a, b = r(lhs), r(rhs)
    if op in ("add", "sub", "mul", "div"):
        sym = {"add": "+", "sub": "-", "mul": "*", "div": "/"}[op]
        return f"(({a}) {sym} ({b}))"
    if op in ("min", "max"):
        cmp_sym = "<" if op == "min" else ">"
        if _is_zero(lhs) and _is_leaf(rhs):
            return f"(({b}) {cmp_sym} 0.0f ? {b} : 0.0f)"
        if _is_zero(rhs) and _is_leaf(lhs):
            return f"(({a}) {cmp_sym} 0.0f ? {a} : 0.0f)"
        return f"{'fminf' if op == 'min' else 'fmaxf'}({a}, {b})"
    return f"(({a}) {_CMP[op]} ({b}))"


def _contains(needle, e) -> bool:
    if _eq(needle, e):
        return True
    k = e["kind"]
    if k == "unary":
        return _contains(needle, e["expr"])
    if k == "binary":
        return _contains(needle, e["lhs"]) or _contains(needle, e["rhs"])
    if k == "select":
        return any(_contains(needle, e[x]) for x in ("cond", "then", "else"))
    return False


def _clamp(e):
    """select_clamps_compared_value (cuda_backend.ml:686-719)."""
    if e["kind"] != "select" or not _is_bin(e["cond"]):
        return None
    c, t, el = e["cond"], e["then"], e["else"]
    if c["op"] == "cmplt" and el["kind"] == "select" and _is_bin(el["cond"], "cmpgt"):
        if (_eq(c["rhs"], t) and _eq(el["cond"]["rhs"], el["then"])
                and _eq(c["lhs"], el["cond"]["lhs"]) and _eq(c["lhs"], el["else"])):
            return c["lhs"], c["rhs"], el["cond"]["rhs"]
    if c["op"] == "cmpgt" and el["kind"] == "select" and _is_bin(el["cond"], "cmplt"):
        if (_eq(c["rhs"], t) and _eq(el["cond"]["rhs"], el["then"])
                and _eq(c["lhs"], el["cond"]["lhs"]) and _eq(c["lhs"], el["else"])):
            return c["lhs"], el["cond"]["rhs"], c["rhs"]
    if c["op"] == "cmplt" and _is_bin(el, "min"):
        if _eq(c["rhs"], t) and _eq(c["lhs"], el["lhs"]):
            return c["lhs"], c["rhs"], el["rhs"]
    if c["op"] == "cmpgt" and _is_bin(el, "max"):
        if _eq(c["rhs"], t) and _eq(c["lhs"], el["lhs"]):
            return c["lhs"], el["rhs"], c["rhs"]
    return None


def value_lines(body, var, flags=None) -> List[str]:
    """render_value_lines (cuda_backend.ml:721-848); defines float `value`.
    `flags`: tail_tune, predicated_select, fast_divide, eager_select_then."""
    flags = flags or {}

    def R(x):
        return render_expr(x, var, flags)

    clamp = _clamp(body)
    if clamp is not None:
        v, lo, hi = clamp
        if flags.get("tail_tune") and not flags.get("predicated_select"):
            return [f"float value = {R(v)};",
                    f"if (value < {R(lo)}) value = {R(lo)};",
                    f"if (value > {R(hi)}) value = {R(hi)};"]
        return [f"float value_unclamped = {R(v)};",
                f"float value = fminf(fmaxf(value_unclamped, {R(lo)}), {R(hi)});"]
    if flags.get("predicated_select"):
        st = _soft_threshold(body)
        if st is not None:
            v, t = R(st[0]), R(st[1])
            return [f"float value = ((({t}) >= 0.0f) ? copysignf(fmaxf(fabsf({v}) - ({t}), "
                    f"0.0f), {v}) : ({_soft_text(v, t)}));"]
    if body["kind"] == "select" and _is_bin(body["cond"]) and body["cond"]["op"] in _CMP:
        c = body["cond"]
        # select_reuses_compared_subexpr (cuda_backend.ml:665-684)
        for reused, other, on_lhs in ((c["lhs"], c["rhs"], True), (c["rhs"], c["lhs"], False)):
            if not _is_leaf(reused) and _contains(reused, body["then"]):
                guard = "value_guard"
                o = render_replacing(other, var, reused, guard)
                lhs, rhs = (guard, o) if on_lhs else (o, guard)
                then_text = render_replacing(body['then'], var, reused, guard)
                else_text = render_replacing(body['else'], var, reused, guard)
                if flags.get("eager_select_then"):
                    return [f"float {guard} = {R(reused)};",
                            f"float value_candidate = {then_text};",
                            f"float value = (({lhs}) {_CMP[c['op']]} ({rhs})) ? value_candidate : "
                            f"({else_text});"]
                return [f"float {guard} = {R(reused)};",
                        f"float value = (({lhs}) {_CMP[c['op']]} ({rhs})) ? "
                        f"({then_text}) : ({else_text});"]
        # select_reuses_compared_value (cuda_backend.ml:614-645)
        for reused, other, on_lhs in ((c["lhs"], c["rhs"], True), (c["rhs"], c["lhs"], False)):
            if _eq(reused, body["then"]):
                sel = "value_selected_value"
                fn = None
                if c["op"] in ("cmplt", "cmple"):
                    fn = "fminf" if on_lhs else "fmaxf"
                elif c["op"] in ("cmpgt", "cmpge"):
                    fn = "fmaxf" if on_lhs else "fminf"
                lines = [f"float {sel} = {R(reused)};"]
                if fn is not None and _eq(body["else"], other):
                    lines.append(f"float value = {fn}({sel}, {R(other)});")
                else:
                    o = R(other)
                    lhs, rhs = (sel, o) if on_lhs else (o, sel)
                    lines.append(f"float value = (({lhs}) {_CMP[c['op']]} ({rhs})) ? {sel} : "
                                 f"({R(body['else'])});")
                return lines
    if _is_bin(body, "mul") and _eq(body["lhs"], body["rhs"]) and not _is_leaf(body["lhs"]):
        return [f"float value_factor = {R(body['lhs'])};",
                "float value = value_factor * value_factor;"]
    return [f"float value = {R(body)};"]


# ---------------------------------------------------------------------------
# C generation

def _cname(name: str) -> str:
    return "u_" + "".join(ch if ch.isalnum() or ch == "_" else "_" for ch in name)


def _ref(text, params):
    if text in params:
        return ("param", text)
    if isinstance(text, str) and text.startswith("node_") and text[5:].isdigit():
        return ("node", int(text[5:]))
    return ("param", text)


def _any(e, pred) -> bool:
    if pred(e):
        return True
    k = e["kind"]
    if k == "unary":
        return _any(e["expr"], pred)
    if k == "binary":
        return _any(e["lhs"], pred) or _any(e["rhs"], pred)
    if k == "select":
        return any(_any(e[x], pred) for x in ("cond", "then", "else"))
    return False


def map_node_flags(node: dict, enabled) -> dict:
    """Rendering switches of one elementwise node under the enabled reference
    flags: body traits (kernel_plan_common.ml:213-235, computed only under a
    trait-analysis flag, cuda_plan.ml:785-792) gate them as
    cuda_backend.ml:1310-1345 does."""
    enabled = set(enabled or ())
    body, n_in, scal = node["body"], len(node["inputs"]), list(node["scalar_params"])
    traits = set()
    if enabled & {"cuda-body-trait-analysis", "shared-body-trait-analysis"}:
        branch = _any(body, lambda x: x["kind"] == "select")
        div = _any(body, lambda x: _is_bin(x, "div"))
        minmax = _any(body, lambda x: _is_bin(x) and x["op"] in ("min", "max"))
        addsub = _any(body, lambda x: _is_bin(x) and x["op"] in ("add", "sub"))
        rules = [(n_in == 1 and bool(scal) and branch, "threshold"),
                 (n_in == 1 and not scal and (branch or minmax), "simple-activation"),
                 (n_in == 2 and div and not branch, "ratio-book"),
                 (n_in == 2 and div and branch, "mixed-filter-ratio"),
                 (n_in == 1 and branch, "activation-or-threshold"),
                 (n_in == 2 and branch, "filter-or-book"),
                 (n_in == 2 and not branch, "affine-vector-update"),
                 (bool(scal) and addsub, "affine"),
                 (div, "ratio"), (branch, "branch"), (minmax, "clip")]
        traits = {name for ok, name in rules if ok}
    tail = "cuda-pointwise-tail-tune" in enabled
    pred = "cuda-pointwise-predicated-select" in enabled
    sel = "cuda-pointwise-selected-tail-plan" in enabled
    atc = "affine" in traits and "threshold" in traits and n_in == 1
    return {"tail_tune": tail,
            "predicated_select": pred and not (sel and atc and "clip" in traits)
            and (atc or not ("threshold" in traits and "clip" not in traits)),
            "fast_divide": sel and "ratio-book" in traits and "branch" not in traits,
            "eager_select_then": tail and "mixed-filter-ratio" in traits}


def entry_c(prog: dict, enabled=()) -> str:
    """C for one entry: oracle_<entry>(tensors, scalars, n, out, result, threads)."""
    name = prog["entry_name"]
    params = {p["name"]: p for p in prog["params"]}
    tensors = [p["name"] for p in prog["params"] if p["kind"] == "tensor1-f32"]
    scalars = [p["name"] for p in prog["params"] if p["kind"] == "scalar-f32"]
    nodes = {n["id"]: n for n in prog["nodes"]}
    res_kind = prog["result"]["kind"]
    res = _ref(prog["result"]["value"], params)

    body: List[str] = []
    done: Dict[int, str] = {}

    def value_of(ref) -> str:
        kind, key = ref
        if kind == "param":
            return f"P_{tensors.index(key)}[i]"
        if key in done:
            return done[key]
        node = nodes[key]
        assert node["kind"] == "elementwise1d", "a reduction cannot feed a map"
        return emit_block(node["inputs"], node["body"], f"node_{key}", key,
                          map_node_flags(node, enabled))

    def emit_block(inputs, expr, label, key=None, flags=None) -> str:
        srcs = [(b["name"], value_of(_ref(b["source"], params))) for b in inputs]
        temp = f"T_{len(done)}_{len(body)}"
        body.append(f"    float {temp};")
        body.append(f"    {{ /* {label} */")
        for nm, src in srcs:
            body.append(f"      const float {_cname(nm)} = {src};")
        for line in value_lines(expr, _cname, flags):
            body.append("      " + line)
        body.append(f"      {temp} = value;")
        body.append("    }")
        if key is not None:
            done[key] = temp
        return temp

    if res_kind == "tensor":
        final = value_of(res)
        reduce_kind = None
    else:
        red = nodes[res[1]]
        reduce_kind = red["reduce_kind"]
        src = red["source"]
        if src["kind"] == "plain":
            final = value_of(_ref(src["input"], params))
        else:
            final = emit_block(src["inputs"], src["body"], "mapped source")

    out = [f"/* entry {name} */",
           f"int oracle_{name}(const float* const* tensors, const float* scalars, int64_t n, "
           "float* out, double* result, int threads) {"]
    for k, t in enumerate(tensors):
        out.append(f"  const float* P_{k} = tensors[{k}];")
    for k, s in enumerate(scalars):
        out.append(f"  const float {_cname(s)} = scalars[{k}];")
    out.append("  if (threads < 1) threads = 1;")
    if reduce_kind is None:
        out.append("  (void)result;")
        out.append("#pragma omp parallel for schedule(static) num_threads(threads)")
        out.append("  for (int64_t i = 0; i < n; ++i) {")
        out += body
        out.append(f"    out[i] = {final};")
        out.append("  }")
    else:
        out.append("  (void)out;")
        out.append("  oracle_acc accs[512];")
        out.append("  float maxes[512];")
        out.append("  if (threads > 512) threads = 512;")
        out.append("#pragma omp parallel num_threads(threads)")
        out.append("  {")
        out.append("    const int tid = omp_get_thread_num();")
        out.append("    const int nt = omp_get_num_threads();")
        out.append("    const int64_t lo = n * tid / nt, hi = n * (tid + 1) / nt;")
        out.append("    oracle_acc acc = {0.0, 0.0};")
        out.append("    float mx = -INFINITY;")
        out.append("    for (int64_t i = lo; i < hi; ++i) {")
        out += ["  " + line for line in body]
        if reduce_kind == "sum":
            out.append(f"      oracle_acc_add(&acc, (double){final});")
        else:
            out.append(f"      mx = fmaxf(mx, {final});")
        out.append("    }")
        out.append("    accs[tid] = acc;")
        out.append("    maxes[tid] = mx;")
        out.append("    if (tid == 0) threads = nt;")
        out.append("  }")
        if reduce_kind == "sum":
            out.append("  oracle_acc total = {0.0, 0.0};")
            out.append("  for (int t = 0; t < threads; ++t) {")
            out.append("    oracle_acc_add(&total, accs[t].sum);")
            out.append("    oracle_acc_add(&total, accs[t].comp);")
            out.append("  }")
            out.append("  *result = oracle_acc_value(&total);")
        else:
            out.append("  float m = -INFINITY;")
            out.append("  for (int t = 0; t < threads; ++t) m = fmaxf(m, maxes[t]);")
            out.append("  *result = (double)m;")
    out.append("  return 0;")
    out.append("}")
    out.append("")
    return "\n".join(out)


def program_c(programs: Sequence[dict], enabled=()) -> str:
    parts = ["/* Generated by oracle/loom_oracle.py -- test infrastructure. */",
             f"/* reference flags: {', '.join(sorted(enabled)) or 'none'} */",
             "#include <omp.h>", "#include <stdint.h>", '#include "oracle_semantics.h"', ""]
    parts += [entry_c(p, enabled) for p in programs]
    return "\n".join(parts)


GCC_FLAGS = ["-O2", "-std=c11", "-fopenmp", "-fPIC", "-shared", "-ffp-contract=off",
             "-fno-fast-math", "-fexcess-precision=standard", "-fno-unsafe-math-optimizations"]


def build(programs: Sequence[dict], name: str, build_dir: str = BUILD_DIR, enabled=()) -> str:
    """Write and compile the oracle for `programs`; returns the .so path."""
    os.makedirs(build_dir, exist_ok=True)
    src = program_c(programs, enabled)
    with open(os.path.join(HERE, "oracle_semantics.h"), "rb") as fh:
        digest = hashlib.sha256(src.encode() + fh.read()).hexdigest()[:12]
    so = os.path.join(build_dir, f"liboracle_{name}_{digest}.so")
    if os.path.exists(so):
        return so
    c_path = os.path.join(build_dir, f"oracle_{name}_{digest}.c")
    with open(c_path, "w", encoding="utf-8") as fh:
        fh.write(src)
    tmp = so + ".tmp"
    cmd = ["gcc", *GCC_FLAGS, f"-I{HERE}", "-o", tmp, c_path, "-lm"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed: {' '.join(cmd)}\n{proc.stderr}")
    os.replace(tmp, so)
    return so


class Oracle:
    """ctypes front of a compiled oracle library."""

    def __init__(self, programs: Sequence[dict], name: str = "programs",
                 build_dir: str = BUILD_DIR, enabled=()):
        self.programs = {p["entry_name"]: p for p in programs}
        self.path = build(list(programs), name, build_dir, enabled)
        self.lib = ctypes.CDLL(self.path)
        self.fns = {}
        for entry in self.programs:
            fn = getattr(self.lib, f"oracle_{entry}")
            fn.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_float),
                           ctypes.c_int64, ctypes.c_void_p, ctypes.POINTER(ctypes.c_double),
                           ctypes.c_int]
            fn.restype = ctypes.c_int
            self.fns[entry] = fn

    def result_kind(self, entry: str) -> str:
        return self.programs[entry]["result"]["kind"]

    def run(self, entry: str, inputs: Dict[str, object], threads: Optional[int] = None):
        """Evaluate `entry`.  Tensor inputs are float32 numpy arrays of one
        length n.  Returns a float32 array (tensor result) or a Python float
        (fp64 sum, or the exact max)."""
        prog = self.programs[entry]
        tnames = [p["name"] for p in prog["params"] if p["kind"] == "tensor1-f32"]
        snames = [p["name"] for p in prog["params"] if p["kind"] == "scalar-f32"]
        arrays = [np.ascontiguousarray(inputs[t], dtype=np.float32) for t in tnames]
        n = int(arrays[0].shape[0]) if arrays else 0
        for a in arrays:
            if a.shape[0] != n:
                raise ValueError("tensor inputs must share one length")
        ptrs = (ctypes.c_void_p * max(1, len(arrays)))(*[a.ctypes.data for a in arrays])
        scal = (ctypes.c_float * max(1, len(snames)))(*[float(inputs[s]) for s in snames])
        result = ctypes.c_double(0.0)
        threads = threads or (os.cpu_count() or 1)
        if prog["result"]["kind"] == "tensor":
            out = np.empty(n, dtype=np.float32)
            self.fns[entry](ptrs, scal, n, out.ctypes.data, ctypes.byref(result), threads)
            return out
        self.fns[entry](ptrs, scal, n, None, ctypes.byref(result), threads)
        return float(result.value)


def load_programs(path: str) -> List[dict]:
    with open(path, "r", encoding="utf-8") as fh:
        obj = json.load(fh)
    return obj if isinstance(obj, list) else [obj]
