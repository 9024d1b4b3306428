"""The reference's LoomLambda scalar passes, for the Python front end.

`loomc` runs these on an entry's body right after normalisation when their
flags are enabled (``src/loom_normalize/normalize.ml:195-258``), in this
order: const-fold, if-simplify, arith-reassociate, let-float, branch-hoist,
lambda-inline-small, scalar-cse, dce, scalar-hoist, then const-fold,
if-simplify and dce once more.  Each function restates one pass of
``src/loom_normalize/normalize_scalar.ml`` on the JSON form of LoomLambda
(``src/loom_core/loomLambda.ml:74-121``), including what the passes do
not guard against: substitution is not capture-avoiding, scalar CSE keys
expressions by a fingerprint that prints floats with 12 significant digits,
and constants fold in double precision.

Tensorization substitutes scalar lets into the bodies, so of these passes
the ones that change the kernels are const-fold (folded literals),
if-simplify (branches with equal arms), arith-reassociate (sums and
products re-associated in fingerprint order, which changes the rounding),
scalar-cse (its fingerprint collisions) and dce (an unused let of a tensor
expression no longer creates a node).
"""

from __future__ import annotations

from typing import Dict, List, Sequence, Set, Tuple

from .analysis import FOLD_FLOAT, FOLD_UNARY, f_max, f_min

# configs/optimizations/current.json (the reference's defaults)
SMALL_INLINE_NODES = 20

NORMALIZE_FLAGS = ("scalar-const-fold", "if-simplify", "arith-reassociate", "let-float",
                   "branch-hoist", "lambda-inline-small", "scalar-cse", "normalized-dce",
                   "scalar-hoist")

_BINARY_FOLD = {"fadd": FOLD_FLOAT["add"], "fsub": FOLD_FLOAT["sub"], "fmul": FOLD_FLOAT["mul"],
                "fdiv": FOLD_FLOAT["div"], "fmin": f_min, "fmax": f_max}
_COMPARE_FOLD = {"fcmplt": lambda a, b: a < b, "fcmple": lambda a, b: a <= b,
                 "fcmpgt": lambda a, b: a > b, "fcmpge": lambda a, b: a >= b,
                 "fcmpeq": lambda a, b: a == b}
_UNARY_FOLD = {"fneg": FOLD_UNARY["neg"], "fsqrt": FOLD_UNARY["sqrt"],
               "fexp": FOLD_UNARY["exp"], "flog": FOLD_UNARY["log"]}


# --- constructors and structure ------------------------------------------------

def _let(name, value, body):
    return {"kind": "let", "name": name, "value": value, "body": body}


def _if(c, t, e):
    return {"kind": "if", "cond": c, "then": t, "else": e}


def _lam(params, body):
    return {"kind": "lambda", "params": params, "body": body}


def _prim(kind, op, args):
    return {"kind": kind, "op": op, "args": args}


def _map_children(e, f, lam_body=None):
    """Rebuild `e` with `f` applied to every direct child.  For a tensor
    primitive whose first argument is a lambda, that lambda's body goes
    through `lam_body` (default `f`) -- the passes treat it apart."""
    k = e["kind"]
    if k in ("var", "float", "bool"):
        return e
    if k == "let":
        return _let(e["name"], f(e["value"]), f(e["body"]))
    if k == "if":
        return _if(f(e["cond"]), f(e["then"]), f(e["else"]))
    if k == "lambda":
        return _lam(e["params"], f(e["body"]))
    if k == "apply":
        return {"kind": "apply", "fn": f(e["fn"]), "args": [f(a) for a in e["args"]]}
    if k == "prim":
        return _prim(k, e["op"], [f(a) for a in e["args"]])
    args = e["args"]
    if args and args[0]["kind"] == "lambda":
        head = _lam(args[0]["params"], (lam_body or f)(args[0]["body"]))
        return _prim(k, e["op"], [head] + [f(a) for a in args[1:]])
    return _prim(k, e["op"], [f(a) for a in args])


def ll_equal(a, b) -> bool:
    """OCaml's structural ``=`` on LoomLambda expressions (floats by IEEE
    value: -0.0 = 0.0, a NaN equals nothing)."""
    k = a["kind"]
    if k != b["kind"]:
        return False
    if k == "var":
        return a["name"] == b["name"] and a["type"] == b["type"]
    if k == "float":
        return float(a["value"]) == float(b["value"])
    if k == "bool":
        return bool(a["value"]) == bool(b["value"])
    if k == "let":
        return (a["name"] == b["name"] and ll_equal(a["value"], b["value"])
                and ll_equal(a["body"], b["body"]))
    if k == "if":
        return all(ll_equal(a[f], b[f]) for f in ("cond", "then", "else"))
    if k == "lambda":
        return ([(p["name"], p["type"]) for p in a["params"]]
                == [(p["name"], p["type"]) for p in b["params"]]
                and ll_equal(a["body"], b["body"]))
    if k == "apply":
        return (ll_equal(a["fn"], b["fn"]) and len(a["args"]) == len(b["args"])
                and all(ll_equal(x, y) for x, y in zip(a["args"], b["args"])))
    return (a["op"] == b["op"] and len(a["args"]) == len(b["args"])
            and all(ll_equal(x, y) for x, y in zip(a["args"], b["args"])))


def free_vars(e) -> Set[str]:
    """normalize_scalar.ml:6-25."""
    k = e["kind"]
    if k == "var":
        return {e["name"]}
    if k in ("float", "bool"):
        return set()
    if k == "let":
        return free_vars(e["value"]) | (free_vars(e["body"]) - {e["name"]})
    if k == "if":
        return free_vars(e["cond"]) | free_vars(e["then"]) | free_vars(e["else"])
    if k == "lambda":
        return free_vars(e["body"]) - {p["name"] for p in e["params"]}
    if k == "apply":
        out = free_vars(e["fn"])
        for a in e["args"]:
            out |= free_vars(a)
        return out
    out: Set[str] = set()
    for a in e["args"]:
        out |= free_vars(a)
    return out


def is_scalar_only(e) -> bool:
    """No lambda, application or tensor primitive, and every variable a
    float or a bool (normalize_scalar.ml:61-72)."""
    k = e["kind"]
    if k == "var":
        return e["type"] in ("float", "bool")
    if k in ("float", "bool"):
        return True
    if k == "let":
        return is_scalar_only(e["value"]) and is_scalar_only(e["body"])
    if k == "if":
        return all(is_scalar_only(e[f]) for f in ("cond", "then", "else"))
    if k == "prim":
        return all(is_scalar_only(a) for a in e["args"])
    return False


def expr_size(e) -> int:
    """normalize_scalar.ml:132-142."""
    k = e["kind"]
    if k in ("var", "float", "bool"):
        return 1
    if k == "let":
        return 1 + expr_size(e["value"]) + expr_size(e["body"])
    if k == "if":
        return 1 + sum(expr_size(e[f]) for f in ("cond", "then", "else"))
    if k == "lambda":
        return 1 + expr_size(e["body"])
    if k == "apply":
        return 1 + expr_size(e["fn"]) + sum(expr_size(a) for a in e["args"])
    return 1 + sum(expr_size(a) for a in e["args"])


def fingerprint(e) -> str:
    """normalize_scalar.ml:238-263."""
    k = e["kind"]
    if k == "var":
        return "v:" + e["name"]
    if k == "float":
        return "f:%0.12g" % float(e["value"])
    if k == "bool":
        return "b:" + ("true" if e["value"] else "false")
    if k == "let":
        return f"l:{e['name']}:{fingerprint(e['value'])}:{fingerprint(e['body'])}"
    if k == "if":
        return f"i:{fingerprint(e['cond'])}:{fingerprint(e['then'])}:{fingerprint(e['else'])}"
    if k == "lambda":
        return "fn:%s:%s" % (",".join(p["name"] for p in e["params"]), fingerprint(e["body"]))
    if k == "apply":
        return "app:%s:%s" % (fingerprint(e["fn"]), ",".join(fingerprint(a) for a in e["args"]))
    tag = "p" if k == "prim" else "t"
    return "%s:%s:%s" % (tag, e["op"], ",".join(fingerprint(a) for a in e["args"]))


def subst_var(name: str, replacement, e):
    """Replace the free occurrences of `name` (normalize_scalar.ml:265-306);
    not capture-avoiding."""
    k = e["kind"]
    if k == "var":
        return replacement if e["name"] == name else e
    if k in ("float", "bool"):
        return e
    rec = lambda x: subst_var(name, replacement, x)
    if k == "let":
        value = rec(e["value"])
        return _let(e["name"], value, e["body"] if e["name"] == name else rec(e["body"]))
    if k == "lambda":
        if any(p["name"] == name for p in e["params"]):
            return e
        return _lam(e["params"], rec(e["body"]))
    if k == "tensor-prim" and e["args"] and e["args"][0]["kind"] == "lambda":
        lam = e["args"][0]
        shadowed = any(p["name"] == name for p in lam["params"])
        head = _lam(lam["params"], lam["body"] if shadowed else rec(lam["body"]))
        return _prim(k, e["op"], [head] + [rec(a) for a in e["args"][1:]])
    return _map_children(e, rec)


# --- the passes ------------------------------------------------------------------

def _is_float(e):
    return float(e["value"]) if e["kind"] == "float" else None


def _is_bool(e):
    return bool(e["value"]) if e["kind"] == "bool" else None


def _eval_binary(op, lhs, rhs):
    a, b = _is_float(lhs), _is_float(rhs)
    if a is not None and b is not None:
        if op in _BINARY_FOLD:
            return {"kind": "float", "value": _BINARY_FOLD[op](a, b)}
        if op in _COMPARE_FOLD:
            return {"kind": "bool", "value": _COMPARE_FOLD[op](a, b)}
    if op == "fcmpeq" and _is_bool(lhs) is not None and _is_bool(rhs) is not None:
        return {"kind": "bool", "value": _is_bool(lhs) == _is_bool(rhs)}
    return None


def const_fold(env: Dict[str, dict], e):
    """normalize_scalar.ml:74-130.  A let bound to a constant is propagated
    into its body; the parameters of a tensor primitive's lambda are not
    removed from the environment, as there."""
    k = e["kind"]
    if k == "var":
        return env.get(e["name"], e)
    if k in ("float", "bool"):
        return e
    if k == "let":
        value = const_fold(env, e["value"])
        inner = dict(env)
        if value["kind"] in ("float", "bool"):
            inner[e["name"]] = value
        else:
            inner.pop(e["name"], None)
        return _let(e["name"], value, const_fold(inner, e["body"]))
    if k == "if":
        c, t, f = (const_fold(env, e[x]) for x in ("cond", "then", "else"))
        cv = _is_bool(c)
        if cv is True:
            return t
        if cv is False:
            return f
        return _if(c, t, f)
    if k == "lambda":
        inner = {n: v for n, v in env.items() if n not in {p["name"] for p in e["params"]}}
        return _lam(e["params"], const_fold(inner, e["body"]))
    if k == "prim":
        op = e["op"]
        args = [const_fold(env, a) for a in e["args"]]
        if op == "select" and len(args) == 3:
            cv = _is_bool(args[0])
            if cv is True:
                return args[1]
            if cv is False:
                return args[2]
            return _prim(k, op, args)
        if op in _UNARY_FOLD and len(args) == 1:
            v = _is_float(args[0])
            if v is not None:
                return {"kind": "float", "value": _UNARY_FOLD[op](v)}
            return _prim(k, op, args)
        if len(args) == 2:
            folded = _eval_binary(op, args[0], args[1])
            return folded if folded is not None else _prim(k, op, args)
        return _prim(k, op, args)
    return _map_children(e, lambda x: const_fold(env, x))


def if_simplify(e):
    """normalize_scalar.ml:144-172."""
    k = e["kind"]
    if k == "if":
        c, t, f = (if_simplify(e[x]) for x in ("cond", "then", "else"))
        cv = _is_bool(c)
        if cv is True:
            return t
        if cv is False:
            return f
        if ll_equal(t, f):
            return t
        return _if(c, t, f)
    if k == "prim" and e["op"] == "select" and len(e["args"]) == 3:
        c, t, f = (if_simplify(a) for a in e["args"])
        if ll_equal(t, f):
            return t
        return _prim(k, "select", [c, t, f])
    return _map_children(e, if_simplify)


def let_float(e):
    """``if c then (let x = v in a) else (let x = v in b)`` with the same
    scalar-only `v` becomes ``let x = v in if c then a else b``
    (normalize_scalar.ml:174-200); branch-hoist is the same pass."""
    if e["kind"] == "if":
        t, f = e["then"], e["else"]
        if (t["kind"] == "let" and f["kind"] == "let" and t["name"] == f["name"]
                and ll_equal(t["value"], f["value"]) and is_scalar_only(t["value"])):
            return _let(t["name"], let_float(t["value"]),
                        _if(let_float(e["cond"]), let_float(t["body"]), let_float(f["body"])))
    return _map_children(e, let_float)


branch_hoist = let_float


def lambda_inline_small(max_nodes: int, e):
    """A lambda applied to as many arguments as it has parameters, whose body
    has at most `max_nodes` nodes, becomes nested lets
    (normalize_scalar.ml:202-236)."""
    rec = lambda x: lambda_inline_small(max_nodes, x)
    if (e["kind"] == "apply" and e["fn"]["kind"] == "lambda"
            and len(e["fn"]["params"]) == len(e["args"])
            and expr_size(e["fn"]["body"]) <= max_nodes):
        out = rec(e["fn"]["body"])
        for p, a in reversed(list(zip(e["fn"]["params"], e["args"]))):
            out = _let(p["name"], rec(a), out)
        return out
    return _map_children(e, rec)


def arith_reassociate(e):
    """Sums and products flattened and rebuilt left-leaning in fingerprint
    order; the operands of min, max and == in fingerprint order
    (normalize_scalar.ml:308-355)."""
    if e["kind"] == "prim" and e["op"] in ("fadd", "fmul"):
        op = e["op"]
        flat: List[dict] = []

        def flatten(x):
            if x["kind"] == "prim" and x["op"] == op:
                for y in x["args"]:
                    flatten(y)
            else:
                flat.append(arith_reassociate(x))

        for a in e["args"]:
            flatten(a)
        flat.sort(key=fingerprint)
        if not flat:
            return _prim("prim", op, [])
        if len(flat) == 1:
            return flat[0]
        acc = _prim("prim", op, [flat[0], flat[1]])
        for x in flat[2:]:
            acc = _prim("prim", op, [acc, x])
        return acc
    if e["kind"] == "prim" and e["op"] in ("fmin", "fmax", "fcmpeq") and len(e["args"]) == 2:
        lhs, rhs = (arith_reassociate(a) for a in e["args"])
        if fingerprint(lhs) > fingerprint(rhs):
            lhs, rhs = rhs, lhs
        return _prim("prim", e["op"], [lhs, rhs])
    return _map_children(e, arith_reassociate)


def scalar_cse(seen: Dict[str, dict], e):
    """A let whose scalar-only value has the fingerprint of an earlier let's
    value is dropped and that earlier value substituted for its name
    (normalize_scalar.ml:357-383)."""
    if e["kind"] == "let":
        value = scalar_cse(seen, e["value"])
        if is_scalar_only(value):
            key = fingerprint(value)
            if key in seen:
                return scalar_cse(seen, subst_var(e["name"], seen[key], e["body"]))
            inner = dict(seen)
            inner[key] = value
            return _let(e["name"], value, scalar_cse(inner, e["body"]))
        return _let(e["name"], value, scalar_cse(seen, e["body"]))
    return _map_children(e, lambda x: scalar_cse(seen, x))


def dce(e):
    """Drop lets whose name the body does not use (normalize_scalar.ml:387-406)."""
    if e["kind"] == "let":
        value, body = dce(e["value"]), dce(e["body"])
        return _let(e["name"], value, body) if e["name"] in free_vars(body) else body
    return _map_children(e, dce)


def _wrap(hoisted: List[Tuple[str, dict]], body):
    for name, value in reversed(hoisted):
        body = _let(name, value, body)
    return body


def hoist_invariant_lets(bound: Set[str], e) -> Tuple[List[Tuple[str, dict]], dict]:
    """normalize_scalar.ml:408-476: the scalar-only lets that use none of
    `bound`, lifted out of `e` in order."""
    k = e["kind"]
    if k == "let":
        vh, value = hoist_invariant_lets(bound, e["value"])
        bh, body = hoist_invariant_lets(bound | {e["name"]}, e["body"])
        if is_scalar_only(value) and not (bound & free_vars(value)):
            return vh + [(e["name"], value)] + bh, body
        return vh + bh, _let(e["name"], value, body)
    if k == "if":
        ch, c = hoist_invariant_lets(bound, e["cond"])
        th, t = hoist_invariant_lets(bound, e["then"])
        fh, f = hoist_invariant_lets(bound, e["else"])
        return ch, _if(c, _wrap(th, t), _wrap(fh, f))
    if k in ("prim", "tensor-prim"):
        hoisted, args = [], []
        for a in e["args"]:
            h, a = hoist_invariant_lets(bound, a)
            hoisted += h
            args.append(a)
        return hoisted, _prim(k, e["op"], args)
    if k == "apply":
        hoisted, fn = hoist_invariant_lets(bound, e["fn"])
        args = []
        for a in e["args"]:
            h, a = hoist_invariant_lets(bound, a)
            hoisted += h
            args.append(a)
        return hoisted, {"kind": "apply", "fn": fn, "args": args}
    if k == "lambda":
        inner = bound | {p["name"] for p in e["params"]}
        h, body = hoist_invariant_lets(inner, e["body"])
        return [], _lam(e["params"], _wrap(h, body))
    return [], e


def scalar_hoist(e):
    """Loop-invariant scalar lets lifted out of map lambdas
    (normalize_scalar.ml:478-502)."""
    if (e["kind"] == "tensor-prim" and e["op"] in ("tensor-map", "tensor-map2")
            and e["args"] and e["args"][0]["kind"] == "lambda"):
        lam = e["args"][0]
        bound = {p["name"] for p in lam["params"]}
        hoisted, body = hoist_invariant_lets(bound, scalar_hoist(lam["body"]))
        out = _prim(e["kind"], e["op"], [_lam(lam["params"], body)]
                    + [scalar_hoist(a) for a in e["args"][1:]])
        for name, value in reversed(hoisted):
            out = _let(name, scalar_hoist(value), out)
        return out
    if e["kind"] == "tensor-prim":
        return _prim(e["kind"], e["op"], [scalar_hoist(a) for a in e["args"]])
    return _map_children(e, scalar_hoist)


def apply_normalize_passes(body, enabled: Sequence[str],
                           small_inline_nodes: int = SMALL_INLINE_NODES):
    """The passes `enabled` switches on, in the reference's order
    (normalize.ml:195-258)."""
    on = set(enabled)
    if "scalar-const-fold" in on:
        body = const_fold({}, body)
    if "if-simplify" in on:
        body = if_simplify(body)
    if "arith-reassociate" in on:
        body = arith_reassociate(body)
    if "let-float" in on:
        body = let_float(body)
    if "branch-hoist" in on:
        body = branch_hoist(body)
    if "lambda-inline-small" in on:
        body = lambda_inline_small(small_inline_nodes, body)
    if "scalar-cse" in on:
        body = scalar_cse({}, body)
    if "normalized-dce" in on:
        body = dce(body)
    if "scalar-hoist" in on:
        body = scalar_hoist(body)
    if "scalar-const-fold" in on:
        body = const_fold({}, body)
    if "if-simplify" in on:
        body = if_simplify(body)
    if "normalized-dce" in on:
        body = dce(body)
    return body
