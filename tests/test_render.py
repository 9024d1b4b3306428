"""Body rendering: the product renderer (loom_b200/render.py) and the
oracle's independent restatement (oracle/loom_oracle.py) of the reference's
emission rules must print the same statements; spot checks pin the rules
themselves against the forms the reference prints
(src/loom_backend_cuda/cuda_backend.ml:446-848)."""

import random
import re

import pytest

from loom_b200 import render
from loom_b200 import tensor_ir as T
from oracle import loom_oracle as O

V, C = T.SVar, T.SConstF32


def B(op, lhs, rhs):
    return T.SBinary(op, lhs, rhs)


def product_lines(body):
    return render.render_value_lines(body, lambda n: "v_" + n)


def oracle_lines(body):
    return [re.sub(r"\bu_", "v_", ln) for ln in O.value_lines(T._expr_to_json(body),
                                                               lambda n: "u_" + n)]


@pytest.mark.parametrize("value, text", [
    (0.0, "0.0f"), (1.0, "1.0f"), (2.5, "2.5"), (0.75, "0.75"), (-0.0, "-0.0f"),
    (100000.0, "100000.0f"), (0.1, "0.1"), (1e-7, "1e-07"), (3.0e20, "3e+20"),
])
def test_cpp_float(value, text):
    assert render.cpp_float(value) == text
    assert O.cpp_float(value) == text


def test_saxpy_contracts_to_fmaf():
    body = B("add", B("mul", V("a"), V("xi")), V("yi"))
    assert product_lines(body) == ["float value = fmaf(v_a, v_xi, v_yi);"]


def test_sub_patterns():
    assert product_lines(B("sub", B("mul", V("a"), V("b")), V("c"))) == \
        ["float value = fmaf(v_a, v_b, -(v_c));"]
    assert product_lines(B("sub", V("c"), B("mul", V("a"), V("b")))) == \
        ["float value = fmaf(-(v_a), v_b, v_c);"]


def test_relu_select_becomes_fmaxf():
    body = T.SSelect(B("cmpgt", V("xi"), C(0.0)), V("xi"), C(0.0))
    assert product_lines(body) == ["float value_selected_value = v_xi;",
                                   "float value = fmaxf(value_selected_value, 0.0f);"]


def test_max_zero_ternary():
    assert product_lines(B("max", V("x"), C(0.0))) == \
        ["float value = ((v_x) > 0.0f ? v_x : 0.0f);"]
    assert product_lines(B("max", B("mul", V("x"), V("y")), C(0.0))) == \
        ["float value = fmaxf(((v_x) * (v_y)), 0.0f);"]


def test_clamp_form():
    body = T.SSelect(B("cmplt", V("x"), V("lo")), V("lo"),
                     T.SSelect(B("cmpgt", V("x"), V("hi")), V("hi"), V("x")))
    assert product_lines(body) == ["float value_unclamped = v_x;",
                                   "float value = fminf(fmaxf(value_unclamped, v_lo), v_hi);"]


def test_guard_form():
    e = B("add", B("mul", V("a"), V("x")), V("y"))
    body = T.SSelect(B("cmpgt", e, C(0.0)), e, C(0.0))
    assert product_lines(body) == [
        "float value_guard = fmaf(v_a, v_x, v_y);",
        "float value = ((value_guard) > (0.0f)) ? (value_guard) : (0.0f);"]


def test_square_form():
    d = B("sub", V("x"), V("y"))
    assert product_lines(B("mul", d, d)) == ["float value_factor = ((v_x) - (v_y));",
                                             "float value = value_factor * value_factor;"]


def _random_expr(rng, depth, names):
    if depth == 0 or rng.random() < 0.25:
        r = rng.random()
        if r < 0.6:
            return V(rng.choice(names))
        return C(rng.choice([0.0, 1.0, 0.5, 2.5, -1.0, 0.1, 3.0]))
    k = rng.random()
    if k < 0.12:
        return T.SUnary(rng.choice(["neg", "sqrt", "exp", "log"]), _random_expr(rng, depth - 1, names))
    if k < 0.3:
        c = B(rng.choice(list(O._CMP)), _random_expr(rng, depth - 1, names),
              _random_expr(rng, depth - 1, names))
        # bias toward the reuse/clamp shapes
        then = c.lhs if rng.random() < 0.5 else _random_expr(rng, depth - 1, names)
        return T.SSelect(c, then, _random_expr(rng, depth - 1, names))
    op = rng.choice(["add", "sub", "mul", "div", "min", "max", "add", "mul"])
    return B(op, _random_expr(rng, depth - 1, names), _random_expr(rng, depth - 1, names))


def test_two_restatements_agree_on_random_bodies():
    rng = random.Random(20260417)
    for _ in range(3000):
        body = _random_expr(rng, rng.randint(1, 5), ["x", "y", "a"])
        assert product_lines(body) == oracle_lines(body), body


FLAG_SETS = [dict(tail_tune=a, predicated_select=b, fast_divide=c, eager_select_then=d)
             for a in (False, True) for b in (False, True) for c in (False, True)
             for d in (False, True)]


def _soft(v, t):
    # x > t ? x - t : (x < -t ? x + t : 0), in both written orders
    return [T.SSelect(B("cmpgt", v, t), B("sub", v, t),
                      T.SSelect(B("cmplt", v, T.SUnary("neg", t)), B("add", v, t), C(0.0))),
            T.SSelect(B("cmplt", v, B("sub", C(0.0), t)), B("add", t, v),
                      T.SSelect(B("cmplt", t, v), B("sub", v, t), C(0.0)))]


def test_flagged_rendering_restatements_agree():
    rng = random.Random(7)
    bodies = _soft(V("x"), V("t")) + _soft(B("mul", V("a"), V("x")), V("t"))
    e = B("add", B("mul", V("a"), V("x")), V("y"))
    bodies.append(T.SSelect(B("cmpgt", e, C(0.0)), e, C(0.0)))      # guard (eager form)
    bodies.append(B("div", V("x"), B("add", V("y"), C(1.0))))          # divide
    bodies += [_random_expr(rng, rng.randint(1, 4), ["x", "y", "a", "t"]) for _ in range(400)]
    for fl in FLAG_SETS:
        rf = render.RenderFlags(**fl)
        for body in bodies:
            got = render.render_value_lines(body, lambda n: "v_" + n, flags=rf)
            ref = [re.sub(r"\bu_", "v_", ln) for ln in
                   O.value_lines(T._expr_to_json(body), lambda n: "u_" + n, fl)]
            assert got == ref, (fl, body)


def test_soft_threshold_forms():
    body = _soft(V("x"), V("t"))[0]
    plain = render.render_value_lines(body, lambda n: n)
    tuned = render.render_value_lines(body, lambda n: n, flags=render.RenderFlags(tail_tune=True))
    pred = render.render_value_lines(body, lambda n: n,
                                     flags=render.RenderFlags(predicated_select=True))
    assert plain != tuned and "copysignf(fmaxf(fabsf(x) - (t), 0.0f), x)" in pred[0]


def test_node_flag_derivation_restatements_agree():
    from loom_b200.plan import node_render_flags
    rng = random.Random(11)
    names = ["cuda-pointwise-tail-tune", "cuda-pointwise-predicated-select",
             "cuda-pointwise-selected-tail-plan", "cuda-body-trait-analysis"]
    for _ in range(600):
        n_in = rng.choice([1, 2])
        ins = ["x", "y"][:n_in]
        scal = sorted(rng.sample(["a", "t"], rng.randint(0, 2)))
        body = _random_expr(rng, rng.randint(1, 4), ins + scal)
        enabled = [f for f in names if rng.random() < 0.6]
        node = {"body": T._expr_to_json(body), "inputs": [{"name": i} for i in ins],
                "scalar_params": scal}
        mine = node_render_flags(enabled, n_in, scal, body)
        ref = O.map_node_flags(node, enabled)
        assert (mine.tail_tune, mine.predicated_select, mine.fast_divide,
                mine.eager_select_then) == (ref["tail_tune"], ref["predicated_select"],
                                            ref["fast_divide"], ref["eager_select_then"])


def test_literal_equality_is_ieee_as_in_ocaml():
    # The reference's pattern guards compare expressions with OCaml's
    # structural `=`, which compares floats as IEEE values: the literal -0.0
    # equals 0.0 (so `x > 0.0 ? x : -0.0` still reuses the compared value and
    # becomes fmaxf), and NaN equals nothing (so `x > nan ? x : nan` stays a
    # ternary).  Both restatements must follow that.
    neg_zero = T.SSelect(B("cmpgt", V("xi"), C(0.0)), V("xi"), C(-0.0))
    assert C(-0.0) == C(0.0) and C(float("nan")) != C(float("nan"))
    assert product_lines(neg_zero) == oracle_lines(neg_zero)
    assert "fmaxf" in product_lines(neg_zero)[-1]
    nan = float("nan")
    with_nan = T.SSelect(B("cmpgt", V("xi"), C(nan)), V("xi"), C(nan))
    assert product_lines(with_nan) == oracle_lines(with_nan)
    assert "fmaxf" not in "".join(product_lines(with_nan))
