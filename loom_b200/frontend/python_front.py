"""Python entry language -> FrontIR.

Reads Loom's Python entry language -- ``@loom.entry`` functions over
``float`` and ``loom.Tensor1`` parameters whose bodies use
``loom.Tensor1.map / map2 / reduce_sum / reduce_max``, lambdas, local
``def``s, assignments, tuple destructuring, conditional expressions,
arithmetic, comparisons and ``min / max / sqrt / exp / log / select`` -- and
produces FrontIR in the JSON form that Loom's own Python frontend prints
(``src/frontends/python/loom_frontend_python.py front-ir-json``), so the two
can be compared node for node (tests/test_frontend.py does, on committed
fixtures).  The accepted language and its error cases follow
``docs/design/language-specs.md`` and that frontend's behaviour.

FrontIR node kinds: var, float, bool, unit, tuple, if, lambda, let, prim,
tensor-prim, apply; types print as ``float``, ``bool``, ``unit``,
``tensor1<f32>``, ``(a -> b -> r)`` for functions and ``(a * b)`` for tuples.
"""

from __future__ import annotations

import ast
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

F = "float"
B = "bool"
U = "unit"
T = "tensor1<f32>"


class FrontendError(ValueError):
    """A Python entry outside the staged language."""


@dataclass(frozen=True)
class Fn:
    params: Tuple[object, ...]
    result: object


@dataclass(frozen=True)
class Tup:
    items: Tuple[object, ...]


def tname(ty) -> str:
    if isinstance(ty, Fn):
        return "(" + " -> ".join([tname(p) for p in ty.params] + [tname(ty.result)]) + ")"
    if isinstance(ty, Tup):
        return "(" + " * ".join(tname(i) for i in ty.items) + ")"
    return ty


def _where(node) -> str:
    return f"line {getattr(node, 'lineno', '?')}, column {getattr(node, 'col_offset', '?')}"


def _err(node, msg):
    raise FrontendError(f"{_where(node)}: {msg}")


def _dotted(node) -> str:
    if isinstance(node, ast.Name):
        return node.id
    if isinstance(node, ast.Attribute):
        return _dotted(node.value) + "." + node.attr
    return ""


_TENSOR_NAMES = {"Tensor1", "Tensor"}
_TENSOR_DOTTED = {"loom.Tensor1", "loom.Tensor", "Tensor1.t", "loom.Tensor1.t"}


def annotation_type(node):
    if node is None:
        raise FrontendError("missing Python type annotation")
    if isinstance(node, ast.Name):
        if node.id in ("float", "bool"):
            return node.id
        if node.id in _TENSOR_NAMES:
            return T
    if isinstance(node, ast.Attribute) and _dotted(node) in _TENSOR_DOTTED:
        return T
    if isinstance(node, ast.Subscript) and _dotted(node.value) in ("tuple", "Tuple"):
        sl = node.slice
        elts = sl.elts if isinstance(sl, ast.Tuple) else [sl]
        return Tup(tuple(annotation_type(e) for e in elts))
    raise FrontendError(f"unsupported Python type annotation: {ast.unparse(node)}")


def _is_entry(dec) -> bool:
    if isinstance(dec, ast.Call):
        return _is_entry(dec.func)
    return _dotted(dec) in ("loom.entry", "entry")


def _skippable(stmt) -> bool:
    if isinstance(stmt, (ast.Import, ast.ImportFrom)):
        return True
    return (isinstance(stmt, ast.Expr) and isinstance(stmt.value, ast.Constant)
            and isinstance(stmt.value.value, str))


# Python call name and arity -> FrontIR scalar primitive
_SCALAR_CALLS = {}
for _names, _arity, _op in ((("sqrt", "math.sqrt", "loom.sqrt"), 1, "fsqrt"),
                            (("exp", "math.exp", "loom.exp"), 1, "fexp"),
                            (("log", "math.log", "loom.log"), 1, "flog"),
                            (("min", "loom.min"), 2, "fmin"),
                            (("max", "loom.max"), 2, "fmax"),
                            (("select", "loom.select"), 3, "select")):
    for _n in _names:
        _SCALAR_CALLS[(_n, _arity)] = _op

# Tensor primitive call name -> (FrontIR op, expected lambda type, result type)
_TENSOR_CALLS = {}
for _prefix in ("loom.Tensor1.", "Tensor1."):
    _TENSOR_CALLS[_prefix + "map"] = ("tensor-map", Fn((F,), F), T)
    _TENSOR_CALLS[_prefix + "map2"] = ("tensor-map2", Fn((F, F), F), T)
    _TENSOR_CALLS[_prefix + "reduce_sum"] = ("tensor-reduce-sum", None, F)
    _TENSOR_CALLS[_prefix + "reduce_max"] = ("tensor-reduce-max", None, F)

_BINOPS = {ast.Add: "fadd", ast.Sub: "fsub", ast.Mult: "fmul", ast.Div: "fdiv"}
_CMPOPS = {ast.Lt: "fcmplt", ast.LtE: "fcmple", ast.Gt: "fcmpgt", ast.GtE: "fcmpge",
           ast.Eq: "fcmpeq"}


class _Translator:
    """One module's staged entries."""

    def __init__(self, tree: ast.Module):
        self.entries = {s.name: s for s in tree.body
                        if isinstance(s, ast.FunctionDef) and any(map(_is_entry, s.decorator_list))}

    # -- functions --------------------------------------------------------
    @staticmethod
    def _check_signature(fn):
        a = fn.args
        if a.posonlyargs or a.kwonlyargs or a.vararg or a.kwarg:
            _err(fn, "only positional Python parameters are supported in Loom entries")
        if a.defaults or a.kw_defaults:
            _err(fn, "default Python parameters are not supported in Loom entries")
        if fn.returns is None:
            _err(fn, "Loom entrypoints require a return annotation")

    def entry(self, name: str) -> dict:
        fn = self.entries.get(name)
        if fn is None:
            raise FrontendError(f'entry "{name}" not found')
        self._check_signature(fn)
        env: Dict[str, object] = {}
        params = []
        for arg in fn.args.args:
            ty = annotation_type(arg.annotation)
            if ty not in (F, T):
                _err(arg, f"unsupported entry parameter type {tname(ty)}")
            env[arg.arg] = ty
            params.append({"name": arg.arg, "type": tname(ty)})
        ret = annotation_type(fn.returns)
        body, body_ty = self.block(fn.body, env, fn.name)
        if tname(ret) != tname(body_ty):
            _err(fn, f"entry return annotation {tname(ret)} does not match inferred "
                     f"{tname(body_ty)}")
        return {"entry": fn.name, "params": params, "return_type": tname(ret), "body": body}

    def local_function(self, fn, env):
        self._check_signature(fn)
        inner = dict(env)
        params, ptypes = [], []
        for arg in fn.args.args:
            ty = annotation_type(arg.annotation)
            inner[arg.arg] = ty
            ptypes.append(ty)
            params.append({"name": arg.arg, "type": tname(ty)})
        ret = annotation_type(fn.returns)
        body, body_ty = self.block(fn.body, inner, fn.name)
        if tname(ret) != tname(body_ty):
            _err(fn, f"function return annotation {tname(ret)} does not match inferred "
                     f"{tname(body_ty)}")
        return {"kind": "lambda", "params": params, "body": body}, Fn(tuple(ptypes), ret)

    # -- statements -------------------------------------------------------
    def block(self, stmts: List[ast.stmt], env, owner):
        i = 0
        while i < len(stmts) and _skippable(stmts[i]):
            i += 1
        if i == len(stmts):
            raise FrontendError(f"{owner}: staged function body must return a value")
        first, rest = stmts[i], stmts[i + 1:]
        if isinstance(first, ast.Return):
            if rest:
                _err(rest[0], "statements after return are not supported in staged regions")
            if first.value is None:
                return {"kind": "unit"}, U
            return self.expr(first.value, env)
        if isinstance(first, ast.FunctionDef):
            value, fty = self.local_function(first, env)
            body, bty = self.block(rest, {**env, first.name: fty}, owner)
            return {"kind": "let", "pattern": {"kind": "var", "name": first.name,
                                               "type": tname(fty)},
                    "value": value, "body": body}, bty
        if isinstance(first, (ast.Assign, ast.AnnAssign)):
            if isinstance(first, ast.Assign):
                if len(first.targets) != 1:
                    _err(first, "parallel assignment is not supported in staged regions")
                target = first.targets[0]
            else:
                target = first.target
                if first.value is None:
                    _err(first, "annotation-only bindings are not supported in staged regions")
            value, vty = self.expr(first.value, env)
            if isinstance(first, ast.AnnAssign):
                ann = annotation_type(first.annotation)
                if tname(ann) != tname(vty):
                    _err(first, f"annotation {tname(ann)} does not match inferred {tname(vty)}")
            inner = dict(env)
            self.bind(target, vty, inner)
            body, bty = self.block(rest, inner, owner)
            return {"kind": "let", "pattern": self.pattern(target, vty), "value": value,
                    "body": body}, bty
        if isinstance(first, ast.If):
            if rest:
                _err(first, "statement-level if is only supported as a tail expression")
            cond, cty = self.expr(first.test, env)
            if cty != B:
                _err(first.test, "if condition must be bool")
            then, tty = self.block(first.body, dict(env), owner)
            other, oty = self.block(first.orelse, dict(env), owner)
            if tname(tty) != tname(oty):
                _err(first, "if branches must have the same staged type")
            return {"kind": "if", "cond": cond, "then": then, "else": other}, tty
        if isinstance(first, (ast.For, ast.While)):
            _err(first, "loops are not supported in staged regions")
        if isinstance(first, (ast.AugAssign, ast.Delete, ast.With, ast.Try, ast.Raise)):
            _err(first, "mutation, exceptions, and resource scopes are not supported in "
                        "staged regions")
        _err(first, "unsupported Python statement in staged region")

    def pattern(self, target, ty):
        if isinstance(target, ast.Name):
            return {"kind": "var", "name": target.id, "type": tname(ty)}
        if isinstance(target, ast.Tuple):
            if not isinstance(ty, Tup):
                _err(target, "tuple destructuring requires a tuple-producing expression")
            if len(target.elts) != len(ty.items):
                _err(target, "tuple pattern arity mismatch")
            return {"kind": "tuple",
                    "items": [self.pattern(t, i) for t, i in zip(target.elts, ty.items)]}
        _err(target, "unsupported assignment target in staged region")

    def bind(self, target, ty, env):
        if isinstance(target, ast.Name):
            env[target.id] = ty
        elif isinstance(target, ast.Tuple):
            if not isinstance(ty, Tup) or len(target.elts) != len(ty.items):
                _err(target, "tuple destructuring requires a matching tuple value")
            for t, i in zip(target.elts, ty.items):
                self.bind(t, i, env)
        else:
            _err(target, "unsupported assignment target in staged region")

    # -- expressions ------------------------------------------------------
    def expr(self, e, env, expected=None):
        if isinstance(e, ast.Name):
            if e.id not in env:
                _err(e, f"unknown staged variable {e.id}")
            return {"kind": "var", "name": e.id, "type": tname(env[e.id])}, env[e.id]
        if isinstance(e, ast.Constant):
            v = e.value
            if isinstance(v, bool):
                return {"kind": "bool", "value": v}, B
            if isinstance(v, (int, float)):
                return {"kind": "float", "value": float(v)}, F
            if v is None:
                return {"kind": "unit"}, U
            _err(e, "unsupported constant in staged region")
        if isinstance(e, ast.Tuple):
            parts = [self.expr(x, env) for x in e.elts]
            return {"kind": "tuple", "items": [p for p, _ in parts]}, Tup(tuple(t for _, t in parts))
        if isinstance(e, ast.IfExp):
            cond, cty = self.expr(e.test, env)
            if cty != B:
                _err(e.test, "conditional expression requires a bool condition")
            a, aty = self.expr(e.body, env)
            b, bty = self.expr(e.orelse, env)
            if tname(aty) != tname(bty):
                _err(e, "conditional branches must have the same staged type")
            return {"kind": "if", "cond": cond, "then": a, "else": b}, aty
        if isinstance(e, ast.Lambda):
            if not isinstance(expected, Fn):
                _err(e, "lambda expressions require an expected Loom function type")
            if len(e.args.args) != len(expected.params):
                _err(e, "lambda arity does not match expected Loom function type")
            inner = dict(env)
            params = []
            for arg, ty in zip(e.args.args, expected.params):
                inner[arg.arg] = ty
                params.append({"name": arg.arg, "type": tname(ty)})
            body, bty = self.expr(e.body, inner)
            if tname(bty) != tname(expected.result):
                _err(e, "lambda result type does not match expected Loom function type")
            return {"kind": "lambda", "params": params, "body": body}, expected
        if isinstance(e, ast.UnaryOp):
            v, vty = self.expr(e.operand, env)
            if vty != F:
                _err(e, "unary numeric operators require float operands")
            if isinstance(e.op, ast.USub):
                return {"kind": "prim", "op": "fneg", "args": [v]}, F
            if isinstance(e.op, ast.UAdd):
                return v, F
            _err(e, "unsupported unary operator in staged region")
        if isinstance(e, ast.BinOp):
            a, aty = self.expr(e.left, env)
            b, bty = self.expr(e.right, env)
            if aty != F or bty != F:
                _err(e, "binary numeric operators require float operands")
            op = _BINOPS.get(type(e.op))
            if op is None:
                _err(e, "unsupported binary operator in staged region")
            return {"kind": "prim", "op": op, "args": [a, b]}, F
        if isinstance(e, ast.Compare):
            if len(e.ops) != 1 or len(e.comparators) != 1:
                _err(e, "chained comparisons are not supported in staged regions")
            a, aty = self.expr(e.left, env)
            b, bty = self.expr(e.comparators[0], env)
            if aty != F or bty != F:
                _err(e, "scalar comparisons require float operands")
            op = _CMPOPS.get(type(e.ops[0]))
            if op is None:
                _err(e, "unsupported comparison operator in staged region")
            return {"kind": "prim", "op": op, "args": [a, b]}, B
        if isinstance(e, ast.Call):
            return self.call(e, env)
        if isinstance(e, ast.Attribute):
            _err(e, f"unsupported staged attribute access {_dotted(e)}")
        _err(e, "unsupported Python expression in staged region")

    def call(self, e: ast.Call, env):
        if e.keywords:
            _err(e, "keyword arguments are not supported in staged regions")
        name = _dotted(e.func)
        spec = _TENSOR_CALLS.get(name)
        if spec is not None:
            op, fty, rty = spec
            want = {"tensor-map": 2, "tensor-map2": 3}.get(op, 1)
            if len(e.args) != want:
                _err(e, {"tensor-map": "Tensor1.map expects a function and one tensor",
                         "tensor-map2": "Tensor1.map2 expects a function and two tensors"}.get(
                             op, f"{name} expects one tensor"))
            args = []
            if fty is not None:
                args.append(self.expr(e.args[0], env, fty)[0])
                tensor_args = e.args[1:]
            else:
                tensor_args = e.args
            for t in tensor_args:
                v, vty = self.expr(t, env)
                if vty != T:
                    if op == "tensor-map":
                        _err(t, "Tensor1.map expects a tensor argument")
                    if op == "tensor-map2":
                        _err(e, "Tensor1.map2 expects tensor arguments")
                    _err(t, f"{name} expects a tensor argument")
                args.append(v)
            return {"kind": "tensor-prim", "op": op, "args": args}, rty
        prim = _SCALAR_CALLS.get((name, len(e.args)))
        if prim is not None:
            return {"kind": "prim", "op": prim,
                    "args": [self.expr(a, env)[0] for a in e.args]}, F
        fn, fty = self.expr(e.func, env)
        args = [self.expr(a, env)[0] for a in e.args]
        if isinstance(fty, Fn) and len(args) <= len(fty.params):
            rty = fty.result if len(args) == len(fty.params) else \
                Fn(fty.params[len(args):], fty.result)
        else:
            rty = U
        return {"kind": "apply", "fn": fn, "args": args}, rty


def parse(source: str, filename: str = "<source>") -> _Translator:
    try:
        return _Translator(ast.parse(source, filename=filename))
    except SyntaxError as exc:
        raise FrontendError(str(exc)) from exc


def list_entries(source: str, filename: str = "<source>") -> List[dict]:
    """Entries of a module in name order, with parameter kinds."""
    tr = parse(source, filename)
    out = []
    for name in sorted(tr.entries):
        params = []
        for arg in tr.entries[name].args.args:
            ty = annotation_type(arg.annotation)
            if ty == F:
                params.append({"name": arg.arg, "kind": "scalar-f32"})
            elif ty == T:
                params.append({"name": arg.arg, "kind": "tensor1-f32"})
            else:
                _err(arg, f"unsupported entry parameter type {tname(ty)}")
        out.append({"name": name, "params": params})
    return out


def front_ir(source: str, entry: str, filename: str = "<source>") -> dict:
    return parse(source, filename).entry(entry)
