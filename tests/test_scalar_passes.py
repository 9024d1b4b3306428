"""The reference's LoomLambda scalar passes (src/loom_normalize/
normalize_scalar.ml) and TensorIR body rewrites and CSE
(src/loom_tensorize/tensor_passes.ml, reduction_analysis.ml), restated in
loom_b200/frontend/normalize_passes.py, analysis.py and passes.py.

The reference's own tests hold no output of these passes (only a check that
the flags are accepted and reported, test/python/test_cli.py:511-540), so
each expectation here is worked out by hand from the OCaml source at the
cited lines -- including the behaviours that source does not guard against
(non-capture-avoiding substitution, x*0 folded to 0, a CSE key blind to
unary operators)."""

import math

import pytest

from loom_b200 import tensor_ir as TI
from loom_b200.build import CUDA_FIXED_FLAGS
from loom_b200.frontend import analysis as A
from loom_b200.frontend import normalize_passes as NP
from loom_b200.frontend import passes as P
from loom_b200.frontend import front_ir, loom_lambda, program_from_front_ir

# --- LoomLambda constructors ------------------------------------------------------


def V(name, ty="float"):
    return {"kind": "var", "name": name, "type": ty}


def F(v):
    return {"kind": "float", "value": v}


def B(v):
    return {"kind": "bool", "value": v}


def prim(op, *args):
    return {"kind": "prim", "op": op, "args": list(args)}


def let(name, value, body):
    return {"kind": "let", "name": name, "value": value, "body": body}


def if_(c, t, e):
    return {"kind": "if", "cond": c, "then": t, "else": e}


def lam(names, body):
    return {"kind": "lambda", "params": [{"name": n, "type": "float"} for n in names],
            "body": body}


def tmap(fn, src):
    return {"kind": "tensor-prim", "op": "tensor-map", "args": [fn, src]}


T = V("t", "tensor1<f32>")

# --- normalize_scalar.ml -----------------------------------------------------------


def test_const_fold_propagates_and_folds_in_double():
    # normalize_scalar.ml:74-130: a constant let propagates into its body and
    # stays (dce removes it); arithmetic folds in double precision
    e = let("a", prim("fadd", F(0.1), F(0.2)), prim("fmul", V("x"), V("a")))
    got = NP.const_fold({}, e)
    assert got == let("a", F(0.1 + 0.2), prim("fmul", V("x"), F(0.30000000000000004)))
    assert NP.dce(got) == prim("fmul", V("x"), F(0.30000000000000004))


def test_const_fold_branches_and_ocaml_float_semantics():
    assert NP.const_fold({}, if_(prim("fcmplt", F(1.0), F(2.0)), V("x"), V("y"))) == V("x")
    assert NP.const_fold({}, prim("select", B(False), V("x"), V("y"))) == V("y")
    # OCaml raises on none of these: 1/0 = inf, sqrt(-1) = nan, log 0 = -inf
    assert NP.const_fold({}, prim("fdiv", F(1.0), F(0.0)))["value"] == math.inf
    assert math.isnan(NP.const_fold({}, prim("fsqrt", F(-1.0)))["value"])
    assert NP.const_fold({}, prim("flog", F(0.0)))["value"] == -math.inf
    assert NP.const_fold({}, prim("fexp", F(1000.0)))["value"] == math.inf
    # Stdlib.min a b = if a <= b then a else b
    assert NP.const_fold({}, prim("fmin", F(math.nan), F(1.0)))["value"] == 1.0
    assert math.isnan(NP.const_fold({}, prim("fmin", F(1.0), F(math.nan)))["value"])
    # equality of two bools folds too
    assert NP.const_fold({}, prim("fcmpeq", B(True), B(True))) == B(True)


def test_const_fold_reaches_into_a_map_lambda_without_unbinding_its_params():
    # normalize_scalar.ml:121-129: the environment is not cleared of a tensor
    # primitive's lambda parameters, so an outer constant of the same name
    # replaces the parameter inside the body
    e = let("x", F(2.0), tmap(lam(["x"], prim("fadd", V("x"), F(1.0))), T))
    got = NP.const_fold({}, e)
    assert got["body"]["args"][0]["body"] == F(3.0)
    # a plain lambda does unbind them (:100-107)
    e2 = let("x", F(2.0), lam(["x"], prim("fadd", V("x"), F(1.0))))
    assert NP.const_fold({}, e2)["body"]["body"] == prim("fadd", V("x"), F(1.0))


def test_if_simplify_equal_arms():
    # normalize_scalar.ml:144-172 (OCaml '=': -0.0 equals 0.0)
    c = prim("fcmpgt", V("x"), F(0.0))
    assert NP.if_simplify(if_(c, V("y"), V("y"))) == V("y")
    assert NP.if_simplify(prim("select", c, F(-0.0), F(0.0))) == F(-0.0)
    nan = F(math.nan)
    kept = NP.if_simplify(prim("select", c, nan, nan))
    assert kept["kind"] == "prim"


def test_arith_reassociate_sorts_by_fingerprint():
    # normalize_scalar.ml:308-355: (y + x) + (b * a) is flattened; the
    # product's factors sort to a*b; then "p:fmul:..." < "v:x" < "v:y"
    e = prim("fadd", prim("fadd", V("y"), V("x")), prim("fmul", V("b"), V("a")))
    want = prim("fadd", prim("fadd", prim("fmul", V("a"), V("b")), V("x")), V("y"))
    assert NP.arith_reassociate(e) == want
    assert NP.arith_reassociate(prim("fmax", V("y"), V("x"))) == prim("fmax", V("x"), V("y"))
    # subtraction is not reordered
    assert NP.arith_reassociate(prim("fsub", V("y"), V("x"))) == prim("fsub", V("y"), V("x"))


def test_scalar_cse_substitutes_the_earlier_value():
    # normalize_scalar.ml:357-383: the later let is dropped and the earlier
    # *value* substituted for its name
    xy = prim("fmul", V("x"), V("y"))
    e = let("a", xy, let("b", xy, prim("fadd", V("a"), V("b"))))
    assert NP.scalar_cse({}, e) == let("a", xy, prim("fadd", V("a"), xy))
    # the fingerprint prints floats with 12 significant digits
    e = let("a", F(0.1000000000001), let("b", F(0.1000000000002), V("b")))
    assert NP.scalar_cse({}, e) == let("a", F(0.1000000000001), F(0.1000000000001))


def test_let_float_and_lambda_inline_small():
    # normalize_scalar.ml:174-200 and :202-236
    v = prim("fmul", V("s"), F(2.0))
    e = if_(V("c", "bool"), let("k", v, prim("fadd", V("k"), V("x"))),
            let("k", v, prim("fsub", V("k"), V("x"))))
    assert NP.let_float(e) == let("k", v, if_(V("c", "bool"), prim("fadd", V("k"), V("x")),
                                              prim("fsub", V("k"), V("x"))))
    app = {"kind": "apply", "fn": lam(["p"], prim("fmul", V("p"), F(2.0))), "args": [V("x")]}
    assert NP.lambda_inline_small(20, app) == let("p", V("x"), prim("fmul", V("p"), F(2.0)))
    assert NP.lambda_inline_small(2, app) == app       # body of 3 nodes


def test_dce_and_scalar_hoist():
    # normalize_scalar.ml:387-406: an unused let of a map goes
    e = let("u", tmap(lam(["x"], V("x")), T), tmap(lam(["x"], prim("fneg", V("x"))), T))
    assert NP.dce(e) == tmap(lam(["x"], prim("fneg", V("x"))), T)
    # normalize_scalar.ml:478-502: a let that uses no lambda parameter is
    # lifted out of the map
    k = prim("fmul", V("s"), F(2.0))
    e = tmap(lam(["x"], let("k", k, prim("fmul", V("x"), V("k")))), T)
    assert NP.scalar_hoist(e) == let("k", k, tmap(lam(["x"], prim("fmul", V("x"), V("k"))), T))


def test_normalize_pipeline_from_python_source():
    src = '''import loom


@loom.entry
def k(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    s = 2.0 * 3.0
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda xi, yi: yi * a + xi * s, x, y))
'''
    front = front_ir(src, "k")
    plain = program_from_front_ir(front)
    assert len(plain.nodes) == 3                    # the unused map is a node
    prog = program_from_front_ir(front, NP.NORMALIZE_FLAGS)
    assert len(prog.nodes) == 2                     # dce dropped it
    body = prog.nodes[0].body
    # s folded to 6.0; each product's factors sorted by fingerprint ("f:6" <
    # "v:xi", "v:a" < "v:yi"), then the sum's terms ("p:fmul:f:6,v:xi" <
    # "p:fmul:v:a,v:yi")
    assert body == TI.SBinary("add", TI.SBinary("mul", TI.SConstF32(6.0), TI.SVar("xi")),
                              TI.SBinary("mul", TI.SVar("a"), TI.SVar("yi")))
    lam_ = loom_lambda(front, NP.NORMALIZE_FLAGS)
    assert "let" not in str(lam_["body"])


# --- reduction_analysis.ml ------------------------------------------------------------

x, y, a, w = TI.SVar("x"), TI.SVar("y"), TI.SVar("a"), TI.SVar("w")
zero, one = TI.SConstF32(0.0), TI.SConstF32(1.0)


def b(op, l, r):
    return TI.SBinary(op, l, r)


def test_canonicalize_orders_operands_and_turns_selects_into_min_max():
    # reduction_analysis.ml:30-57
    assert A.canonicalize(b("add", y, b("mul", a, x))) == b("add", b("mul", a, x), y)
    assert A.canonicalize(b("sub", y, x)) == b("sub", y, x)
    relu = TI.SSelect(b("cmpgt", x, zero), x, zero)
    assert A.canonicalize(relu) == b("max", zero, x)            # "f:0" < "v:x"
    assert A.canonicalize(TI.SSelect(b("cmplt", x, y), y, x)) == b("max", x, y)
    assert A.canonicalize(TI.SSelect(b("cmpgt", x, y), y, x)) == b("min", x, y)
    # the rank ignores a unary's operator: sqrt x and exp x tie and keep order
    s, e = TI.SUnary("sqrt", x), TI.SUnary("exp", x)
    assert A.canonicalize(b("add", s, e)) == b("add", s, e)
    assert A.canonicalize(b("add", e, s)) == b("add", e, s)


def test_simplify_identities():
    # reduction_analysis.ml:293-343
    assert A.simplify(b("mul", x, one)) == x
    assert A.simplify(b("add", TI.SConstF32(-0.0), x)) == x     # float patterns match -0.0
    assert A.simplify(b("mul", x, zero)) == zero                 # whatever x is
    assert A.simplify(b("sub", zero, x)) == b("sub", zero, x)
    assert A.simplify(b("min", x, x)) == x
    assert A.simplify(b("mul", TI.SConstF32(2.0), TI.SConstF32(3.0))) == TI.SConstF32(6.0)
    assert A.simplify(TI.SSelect(TI.SConstBool(True), x, y)) == x
    assert A.simplify(TI.SSelect(b("cmpgt", x, y), y, y)) == y
    assert math.isnan(A.simplify(TI.SUnary("sqrt", TI.SConstF32(-1.0))).value)
    assert A.simplify(b("cmpeq", TI.SConstBool(False), TI.SConstBool(False))) == TI.SConstBool(True)


def test_reduction_body_rewrites():
    # reduction_analysis.ml:74-138: data factors first, then scalar weights
    assert A.canonicalize_reduction_body(("w",), b("mul", w, b("mul", y, x))) == \
        b("mul", b("mul", x, y), w)
    w1, w2 = TI.SVar("w1"), TI.SVar("w2")
    c = b("cmpgt", x, zero)
    body = TI.SSelect(c, b("mul", x, w1), b("mul", w2, x))
    assert A.branchy_weighted_rescue_body(("w1", "w2"), body) == \
        b("mul", x, TI.SSelect(c, w1, w2))
    # reduction_analysis.ml:345-365
    d = b("sub", x, y)
    assert A.reduction_body_cse_expr(b("add", d, d)) == b("mul", TI.SConstF32(2.0), d)
    assert A.reduction_body_cse_expr(b("sub", d, d)) == zero
    assert A.repeated_subexpressions(b("mul", d, d)) == 1


def test_adjusted_metrics_of_dot_like_bodies():
    # reduction_analysis.ml:238-282
    assert A.classify_reduction_body_pattern((), b("mul", x, y)) == "dot-like"
    assert A.classify_reduction_body_pattern(("w",), b("mul", w, b("mul", x, y))) == \
        "weighted-dot-like"
    d = b("sub", x, y)
    assert A.classify_reduction_body_pattern((), b("mul", d, d)) == "squared-difference"
    m = A.adjusted_reduction_body_metrics((), 1, b("mul", d, d))
    assert (m.scalar_complexity, m.repeated_subexpressions) == (2, 0)
    m = A.adjusted_reduction_body_metrics(("w",), 1, b("mul", w, b("mul", x, y)))
    assert m.scalar_complexity == 2


def test_ocaml_equality_has_no_identity_shortcut():
    nan = TI.SConstF32(math.nan)
    e = b("add", nan, x)
    assert e != e
    assert TI.SConstF32(-0.0) == zero and hash(TI.SConstF32(-0.0)) == hash(zero)


# --- tensor_passes.ml ---------------------------------------------------------------


def _prog(nodes, result):
    return TI.Program("p", [TI.TensorParam("t"), TI.ScalarParam("s")], "tensor", result, nodes)


def test_tensor_cse_merges_equal_nodes_and_redirects_uses():
    # tensor_passes.ml:440-513
    t = TI.ParamRef("t")
    n0 = TI.Elementwise1D(0, (TI.InputBinding("x", t),), (), b("mul", x, x))
    n1 = TI.Elementwise1D(1, (TI.InputBinding("x", t),), (), b("mul", x, x))
    n2 = TI.Elementwise1D(2, (TI.InputBinding("u", TI.NodeRef(0)), TI.InputBinding("v", TI.NodeRef(1))),
                          (), b("add", TI.SVar("u"), TI.SVar("v")))
    prog = P.tensor_cse(_prog([n0, n1, n2], TI.NodeRef(2)))
    assert [n.id for n in prog.nodes] == [0, 2]
    assert [bd.source for bd in prog.nodes[1].inputs] == [TI.NodeRef(0), TI.NodeRef(0)]
    # the key holds the body's rank, blind to the unary operator
    n0 = TI.Elementwise1D(0, (TI.InputBinding("x", t),), (), TI.SUnary("sqrt", x))
    n1 = TI.Elementwise1D(1, (TI.InputBinding("x", t),), (), TI.SUnary("exp", x))
    prog = P.tensor_cse(_prog([n0, n1], TI.NodeRef(1)))
    assert [n.id for n in prog.nodes] == [0] and prog.result == TI.NodeRef(0)


def test_tensor_pipeline_on_a_mapped_reduction():
    src = '''import loom


@loom.entry
def wdot(w: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda xi, yi: w * (yi * xi), x, y))
'''
    prog = program_from_front_ir(front_ir(src, "wdot"), CUDA_FIXED_FLAGS)
    (red,) = prog.nodes
    assert isinstance(red.source, TI.MappedInput)
    # inputs sorted by name; product as data factors then the weight
    assert [bd.name for bd in red.source.inputs] == ["xi__r0", "yi__r0"]
    assert red.source.body == b("mul", b("mul", TI.SVar("xi__r0"), TI.SVar("yi__r0")), w)
    # annotation under reduction-body-canonicalize: weighted dot-like metrics
    assert red.metrics.scalar_complexity == 2 and red.metrics.repeated_subexpressions == 0


@pytest.mark.parametrize("flags", [(), tuple(CUDA_FIXED_FLAGS)])
def test_passes_keep_programs_valid(flags):
    from loom_b200.frontend import python_programs
    import os
    here = os.path.dirname(os.path.abspath(__file__))
    progs = python_programs(os.path.join(here, "golden", "sources", "cases", "frontend_cases.py"),
                            flags)
    assert progs
    for p in progs:
        TI.validate(p)
