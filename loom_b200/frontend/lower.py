"""FrontIR -> LoomLambda -> TensorIR.

Restates the two front-end passes between a frontend and the backends, with
the default (empty) optimisation set:

* normalize (``src/loom_normalize/normalize.ml:1-280``): local function
  bindings are inlined where they are applied -- the arguments bind in the
  function's own closure environment, as there -- value ``let``s stay
  ``let``s, tuples are destructured away, a lambda that is not applied stays
  a lambda, and ``()`` becomes the variable ``()`` of type unit;
* tensorize (``src/loom_tensorize/tensorize.ml:1-282``): scalar lets are
  substituted into scalar bodies, every map/map2 becomes an ``elementwise1d``
  node whose scalar parameters are the body's free variables other than the
  lambda's own (sorted), every reduction a ``reduce1d`` over its plain input,
  numbered in creation order;
* annotate (``src/loom_tensorize/tensor_passes.ml:515-552`` with the metric
  definitions of ``src/loom_tensorize/reduction_analysis.ml:1-290``): use
  counts, body metrics and the reduction shape.

With optimisation flags, the reference's LoomLambda scalar passes run after
normalize (normalize_passes.py) and its TensorIR passes after tensorize
(passes.py).

The output is the TensorIR the reference hands its CUDA backend for the same
source, node for node (checked against the reference's golden TensorIR and
LoomLambda files in tests/test_frontend.py).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

from .. import tensor_ir as TI
from .python_front import FrontendError

# ---------------------------------------------------------------------------
# normalize: FrontIR -> LoomLambda (dicts in LoomLambda's JSON form)


class _Value:
    def __init__(self, expr):
        self.expr = expr


class _Tuple:
    def __init__(self, items):
        self.items = items


class _Function:
    def __init__(self, params, body, closure):
        self.params = params
        self.body = body
        self.closure = closure


def _var(name, ty):
    return {"kind": "var", "name": name, "type": ty}


def _as_expr(binding):
    if isinstance(binding, _Value):
        return binding.expr
    if isinstance(binding, _Tuple):
        raise FrontendError("tuple values must be destructured before LoomLambda normalization")
    env = dict(binding.closure)
    for p in binding.params:
        env[p["name"]] = _Value(_var(p["name"], p["type"]))
    return {"kind": "lambda", "params": [dict(p) for p in binding.params],
            "body": _norm(binding.body, env)}


def _norm_value(e, env):
    if e["kind"] == "tuple":
        items = []
        for item in e["items"]:
            v = _norm_value(item, env)
            items.append(v if isinstance(v, _Tuple) else _Value(v))
        return _Tuple(items)
    if e["kind"] == "var":
        b = env.get(e["name"])
        if isinstance(b, _Tuple):
            return b
        if b is not None:
            return _as_expr(b)
        return _var(e["name"], e["type"])
    return _norm(e, env)


def _bind_pattern(env, pattern, binding):
    if pattern["kind"] == "var":
        if pattern["name"] != "_":
            env[pattern["name"]] = binding
        return env
    if not isinstance(binding, _Tuple):
        raise FrontendError("tuple destructuring requires a tuple-producing expression during "
                            "normalization")
    if len(pattern["items"]) != len(binding.items):
        raise FrontendError("tuple pattern arity mismatch during normalization")
    for p, b in zip(pattern["items"], binding.items):
        env = _bind_pattern(env, p, b)
    return env


def _apply_function(closure, params, body, args):
    """Bind arguments to parameters in the function's closure environment
    (normalize.ml:98-122); too few arguments leave a lambda over the rest,
    too many apply the result to the extra ones."""
    env = dict(closure)
    for i, p in enumerate(params):
        if i >= len(args):
            return {"kind": "lambda", "params": [dict(q) for q in params[i:]],
                    "body": _norm(body, env)}
        v = _norm_value(args[i], env)
        env[p["name"]] = v if isinstance(v, _Tuple) else _Value(v)
    extra = args[len(params):]
    if not extra:
        return _norm(body, env)
    return {"kind": "apply", "fn": _norm(body, env), "args": [_norm(a, env) for a in extra]}


def _norm(e, env):
    k = e["kind"]
    if k == "var":
        b = env.get(e["name"])
        return _as_expr(b) if b is not None else _var(e["name"], e["type"])
    if k == "float":
        return {"kind": "float", "value": float(e["value"])}
    if k == "bool":
        return {"kind": "bool", "value": bool(e["value"])}
    if k == "unit":
        return _var("()", "unit")
    if k == "tuple":
        raise FrontendError("tuple expressions must be eliminated during normalization")
    if k == "let":
        pat, value = e["pattern"], e["value"]
        if pat["kind"] == "var" and value["kind"] == "lambda":
            inner = dict(env)
            inner[pat["name"]] = _Function(value["params"], value["body"], env)
            return _norm(e["body"], inner)
        v = _norm_value(value, env)
        if pat["kind"] == "var" and not isinstance(v, _Tuple):
            inner = dict(env)
            inner[pat["name"]] = _Value(_var(pat["name"], pat["type"]))
            return {"kind": "let", "name": pat["name"], "value": v, "body": _norm(e["body"], inner)}
        binding = v if isinstance(v, _Tuple) else _Value(v)
        return _norm(e["body"], _bind_pattern(dict(env), pat, binding))
    if k == "if":
        return {"kind": "if", "cond": _norm(e["cond"], env), "then": _norm(e["then"], env),
                "else": _norm(e["else"], env)}
    if k == "lambda":
        inner = dict(env)
        for p in e["params"]:
            inner[p["name"]] = _Value(_var(p["name"], p["type"]))
        return {"kind": "lambda", "params": [dict(p) for p in e["params"]],
                "body": _norm(e["body"], inner)}
    if k == "apply":
        fn, args = e["fn"], e["args"]
        if fn["kind"] == "var":
            b = env.get(fn["name"])
            if isinstance(b, _Function):
                return _apply_function(b.closure, b.params, b.body, args)
            head = _as_expr(b) if b is not None else _var(fn["name"], "unit")
            return {"kind": "apply", "fn": head, "args": [_norm(a, env) for a in args]}
        if fn["kind"] == "lambda":
            return _apply_function(env, fn["params"], fn["body"], args)
        return {"kind": "apply", "fn": _norm(fn, env), "args": [_norm(a, env) for a in args]}
    if k == "prim":
        return {"kind": "prim", "op": e["op"], "args": [_norm(a, env) for a in e["args"]]}
    if k == "tensor-prim":
        return {"kind": "tensor-prim", "op": e["op"], "args": [_norm(a, env) for a in e["args"]]}
    raise FrontendError(f"unknown FrontIR node kind {k!r}")


def loom_lambda(front: dict, enabled=(), cfg=None) -> dict:
    """FrontIR entry -> LoomLambda entry (JSON form of loomLambda.ml:74-137),
    after the scalar passes that `enabled` switches on (normalize.ml:195-258;
    normalize_passes.py)."""
    from ..optconfig import DEFAULT_CONFIG
    from .normalize_passes import apply_normalize_passes
    cfg = cfg or DEFAULT_CONFIG
    env = {p["name"]: _Value(_var(p["name"], p["type"])) for p in front["params"]}
    body = apply_normalize_passes(_norm(front["body"], env), enabled, cfg.small_inline_nodes)
    return {"entry": front["entry"], "params": [dict(p) for p in front["params"]],
            "return_type": front["return_type"], "body": body}


# ---------------------------------------------------------------------------
# tensorize: LoomLambda -> TensorIR

_PRIMS = {"fadd": ("b", "add"), "fsub": ("b", "sub"), "fmul": ("b", "mul"),
          "fdiv": ("b", "div"), "fmin": ("b", "min"), "fmax": ("b", "max"),
          "fneg": ("u", "neg"), "fsqrt": ("u", "sqrt"), "fexp": ("u", "exp"),
          "flog": ("u", "log"), "fcmplt": ("b", "cmplt"), "fcmple": ("b", "cmple"),
          "fcmpgt": ("b", "cmpgt"), "fcmpge": ("b", "cmpge"), "fcmpeq": ("b", "cmpeq"),
          "select": ("s", None)}


class _Scalar:                       # a scalar expression
    def __init__(self, expr):
        self.expr = expr


class _ScalarRef:                    # the result of a reduction
    def __init__(self, ref):
        self.ref = ref


class _Tensor:
    def __init__(self, ref):
        self.ref = ref


def _scalar_of(e, env) -> TI.ScalarExpr:
    k = e["kind"]
    if k == "var":
        b = env.get(e["name"])
        if isinstance(b, _Scalar):
            return b.expr
        if isinstance(b, _ScalarRef):
            raise FrontendError("reduction results cannot be captured inside scalar lambdas")
        if isinstance(b, _Tensor):
            raise FrontendError("tensor capture inside scalar lambdas is not supported")
        raise FrontendError(f"unbound scalar variable {e['name']}")
    if k == "float":
        return TI.SConstF32(float(e["value"]))
    if k == "bool":
        return TI.SConstBool(bool(e["value"]))
    if k == "let":
        v = _scalar_of(e["value"], env)
        return _scalar_of(e["body"], {**env, e["name"]: _Scalar(v)})
    if k == "if":
        return TI.SSelect(_scalar_of(e["cond"], env), _scalar_of(e["then"], env),
                          _scalar_of(e["else"], env))
    if k == "prim":
        args = [_scalar_of(a, env) for a in e["args"]]
        arity, op = _PRIMS[e["op"]]
        if arity == "u":
            if len(args) != 1:
                raise FrontendError("invalid unary primitive arity")
            return TI.SUnary(op, args[0])
        if arity == "b":
            if len(args) != 2:
                raise FrontendError("invalid binary primitive arity")
            return TI.SBinary(op, args[0], args[1])
        if len(args) != 3:
            raise FrontendError("invalid select primitive arity")
        return TI.SSelect(*args)
    if k == "apply":
        if e["fn"]["kind"] == "var":
            raise FrontendError(f"unknown function call inside scalar lambda: {e['fn']['name']}")
        raise FrontendError("unsupported higher-order function call inside scalar lambda")
    if k == "tensor-prim":
        raise FrontendError("tensor primitives are not allowed inside scalar lambdas")
    raise FrontendError("nested lambdas are not supported inside scalar lambdas")


class _Tensorizer:
    def __init__(self):
        self.nodes: List[TI.Node] = []

    def add(self, make):
        nid = len(self.nodes)
        self.nodes.append(make(nid))
        return nid

    def tensor(self, e, env) -> TI.ValueRef:
        v = self.compile(e, env)
        if not isinstance(v, _Tensor):
            raise FrontendError("expected a tensor expression")
        return v.ref

    def compile(self, e, env):
        k = e["kind"]
        if k == "var":
            if e["name"] not in env:
                raise FrontendError(f"unbound staged variable {e['name']}")
            return env[e["name"]]
        if k == "float":
            return _Scalar(TI.SConstF32(float(e["value"])))
        if k == "bool":
            return _Scalar(TI.SConstBool(bool(e["value"])))
        if k == "let":
            v = self.compile(e["value"], env)
            return self.compile(e["body"], {**env, e["name"]: v})
        if k == "if":
            return _Scalar(TI.SSelect(_scalar_of(e["cond"], env), _scalar_of(e["then"], env),
                                      _scalar_of(e["else"], env)))
        if k == "prim":
            return _Scalar(_scalar_of(e, env))
        if k == "apply":
            raise FrontendError("unsupported top-level function application in staged entry")
        if k == "lambda":
            raise FrontendError("unexpected lambda at top level during tensorization")
        op, args = e["op"], e["args"]
        if op in ("tensor-reduce-sum", "tensor-reduce-max") and len(args) == 1:
            src = self.tensor(args[0], env)
            kind = "sum" if op == "tensor-reduce-sum" else "max"
            return _ScalarRef(TI.NodeRef(self.add(lambda i: TI.Reduce1D(
                id=i, source=TI.PlainInput(src), kind=kind))))
        if op == "tensor-map" and len(args) == 2 and args[0]["kind"] == "lambda" \
                and len(args[0]["params"]) == 1:
            lam = args[0]
            src = self.tensor(args[1], env)
            p = lam["params"][0]["name"]
            body = _scalar_of(lam["body"], {**env, p: _Scalar(TI.SVar(p))})
            scalars = tuple(v for v in TI.free_vars(body) if v != p)
            return _Tensor(TI.NodeRef(self.add(lambda i: TI.Elementwise1D(
                id=i, inputs=(TI.InputBinding(p, src),), scalar_params=scalars, body=body))))
        if op == "tensor-map2" and len(args) == 3 and args[0]["kind"] == "lambda" \
                and len(args[0]["params"]) == 2:
            lam = args[0]
            a = self.tensor(args[1], env)
            b = self.tensor(args[2], env)
            p, q = lam["params"][0]["name"], lam["params"][1]["name"]
            body = _scalar_of(lam["body"], {**env, p: _Scalar(TI.SVar(p)), q: _Scalar(TI.SVar(q))})
            scalars = tuple(v for v in TI.free_vars(body) if v not in (p, q))
            return _Tensor(TI.NodeRef(self.add(lambda i: TI.Elementwise1D(
                id=i, inputs=(TI.InputBinding(p, a), TI.InputBinding(q, b)),
                scalar_params=scalars, body=body))))
        raise FrontendError("invalid tensor primitive application shape")


# --- annotation (metrics) ------------------------------------------------------

def scalar_rank(e) -> str:
    """Structural key of an expression; a unary's operator is not part of it
    (reduction_analysis.ml:3-28)."""
    if isinstance(e, TI.SVar):
        return "v:" + e.name
    if isinstance(e, TI.SConstF32):
        return "f:%0.12g" % e.value
    if isinstance(e, TI.SConstBool):
        return "b:" + ("true" if e.value else "false")
    if isinstance(e, TI.SUnary):
        return "u:" + scalar_rank(e.expr)
    if isinstance(e, TI.SBinary):
        return f"b:{e.op}:{scalar_rank(e.lhs)}:{scalar_rank(e.rhs)}"
    return f"s:{scalar_rank(e.cond)}:{scalar_rank(e.then)}:{scalar_rank(e.els)}"


def _children(e):
    if isinstance(e, TI.SUnary):
        return [e.expr]
    if isinstance(e, TI.SBinary):
        return [e.lhs, e.rhs]
    if isinstance(e, TI.SSelect):
        return [e.cond, e.then, e.els]
    return []


def _count(e, pred) -> int:
    return (1 if pred(e) else 0) + sum(_count(c, pred) for c in _children(e))


def body_metrics(uses: int, body) -> TI.BodyMetrics:
    counts: Dict[str, int] = {}

    def walk(e):
        if isinstance(e, (TI.SVar, TI.SConstF32, TI.SConstBool)):
            return
        key = scalar_rank(e)
        counts[key] = counts.get(key, 0) + 1
        for c in _children(e):
            walk(c)

    walk(body)
    is_sel = lambda x: isinstance(x, TI.SSelect)
    is_div = lambda x: isinstance(x, TI.SBinary) and x.op == "div"
    return TI.BodyMetrics(
        scalar_complexity=TI.complexity(body),
        has_branch=_count(body, is_sel) > 0,
        has_div=_count(body, is_div) > 0,
        branch_count=_count(body, is_sel),
        div_count=_count(body, is_div),
        repeated_subexpressions=sum(c - 1 for c in counts.values() if c > 1),
        estimated_uses=uses,
    )


def _use_counts(prog: TI.Program) -> Dict[int, int]:
    counts: Dict[int, int] = {}

    def add(ref):
        if isinstance(ref, TI.NodeRef):
            counts[ref.id] = counts.get(ref.id, 0) + 1

    for n in prog.nodes:
        if isinstance(n, TI.Elementwise1D):
            for b in n.inputs:
                add(b.source)
        elif isinstance(n.source, TI.PlainInput):
            add(n.source.input)
        else:
            for b in n.source.inputs:
                add(b.source)
    add(prog.result)
    return counts


def annotate(prog: TI.Program, enabled=(), cfg=None) -> TI.Program:
    """Metrics, reduction shapes and handling hints of every node
    (tensor_passes.ml:513-548); the hints depend on the materialisation flags
    in `enabled`."""
    from ..optconfig import DEFAULT_CONFIG
    from .passes import materialization_hint
    uses = _use_counts(prog)
    for n in prog.nodes:
        u = uses.get(n.id, 0)
        if isinstance(n, TI.Elementwise1D):
            n.metrics = body_metrics(u, n.body)
        else:
            if isinstance(n.source, TI.PlainInput):
                n.metrics = TI.BodyMetrics(estimated_uses=u)
                n.reduction_shape = "plain"
            else:
                b = n.source.body
                if "reduction-body-canonicalize" in enabled:
                    from .analysis import adjusted_reduction_body_metrics
                    n.metrics = adjusted_reduction_body_metrics(n.source.scalar_params, u, b)
                else:
                    n.metrics = body_metrics(u, b)
                has_sel = _count(b, lambda x: isinstance(x, TI.SSelect)) > 0
                has_div = _count(b, lambda x: isinstance(x, TI.SBinary) and x.op == "div") > 0
                n.reduction_shape = ("branchy-mapped" if has_sel else "ratio-mapped" if has_div
                                     else "weighted-mapped" if n.source.scalar_params
                                     else "mapped")
        n.handling_hint = materialization_hint(
            enabled, n.metrics, None if isinstance(n, TI.Elementwise1D) else n.reduction_shape,
            cfg or DEFAULT_CONFIG)
    return prog


def tensor_ir(lam: dict, enabled=(), cfg=None) -> TI.Program:
    """LoomLambda entry -> annotated, validated TensorIR program, after the
    restated TensorIR passes that `enabled` switches on (passes.py)."""
    from .passes import apply_tensor_passes
    env = {}
    params: List[TI.Param] = []
    for p in lam["params"]:
        if p["type"] == "float":
            env[p["name"]] = _Scalar(TI.SVar(p["name"]))
            params.append(TI.ScalarParam(p["name"]))
        elif p["type"] == "tensor1<f32>":
            env[p["name"]] = _Tensor(TI.ParamRef(p["name"]))
            params.append(TI.TensorParam(p["name"], "n"))
        else:
            raise FrontendError(f"unsupported entry parameter type {p['type']}")
    tz = _Tensorizer()
    res = tz.compile(lam["body"], env)
    if isinstance(res, _Tensor):
        kind, ref = "tensor", res.ref
    elif isinstance(res, _ScalarRef):
        kind, ref = "scalar", res.ref
    else:
        raise FrontendError("entry lowered to a scalar expression instead of a reduction result")
    prog = TI.Program(entry_name=lam["entry"], params=params, result_kind=kind, result=ref,
                      nodes=tz.nodes)
    from ..optconfig import DEFAULT_CONFIG
    cfg = cfg or DEFAULT_CONFIG
    prog = apply_tensor_passes(prog, enabled, cfg)
    annotate(prog, enabled, cfg)
    TI.validate(prog)
    return prog


def program_from_front_ir(front: dict, enabled=(), cfg=None) -> TI.Program:
    """FrontIR entry -> TensorIR, with the passes `enabled` switches on and
    the thresholds of `cfg` (an ``OptConfig``; the reference's defaults when
    None)."""
    return tensor_ir(loom_lambda(front, enabled, cfg), enabled, cfg)
