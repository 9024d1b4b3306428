"""Seeded random entries for the scalar and TensorIR pass tests (make_pass_programs.py)."""

import loom


@loom.entry
def p000(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    m0 = loom.Tensor1.map2(lambda xi, yi: a, x, y)
    return m0


@loom.entry
def p001(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = -2.0
    c1 = 3.0
    m0 = loom.Tensor1.map2(lambda xi, yi: (xi if a < xi else a), x, y)
    m1 = loom.Tensor1.map(lambda v: ((c1 * (b * c1)) if (0.0 * (v * a)) > ((c0 - 1.5) * (c0 - 1.5)) else (c1 * (b * c1))), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: (-(a * -2.0)), m1, w))


@loom.entry
def p002(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = -2.0
    c1 = ((-0.5 * 0.5) + -0.5)
    s0 = ((a * 0.0) * (c0 if c1 >= b else -2.0))
    m0 = loom.Tensor1.map2(lambda xi, yi: (c1 * ((b - (b / (c1 * c1 + 1.0))) * max((b + c1), (-c1)))), x, y)
    m1 = loom.Tensor1.map(lambda v: 0.0, m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: ((c1 / (s0 * s0 + 1.0)) + c0), m1, w))


@loom.entry
def p003(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = (3.0 * (1.0 * 0.5))
    s0 = (min(b, 0.25) + (1.0 if 3.0 > b else 1.0))
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    m0 = loom.Tensor1.map2(lambda xi, yi: 3.0, x, y)
    m1 = loom.Tensor1.map(lambda v: (-(v * s0)), m0)
    return loom.Tensor1.reduce_max(m1)


@loom.entry
def p004(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    m0 = loom.Tensor1.map2(lambda xi, yi: yi, x, y)
    m1 = loom.Tensor1.map(lambda v: b, m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: min((-2.0 * 0.5), (q if q < q else q)), m1, w))


@loom.entry
def p005(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    m0 = loom.Tensor1.map2(lambda xi, yi: yi, x, y)
    m1 = loom.Tensor1.map(lambda v: ((v + a) - -0.5), m0)
    return m1


@loom.entry
def p006(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    c0 = (2.0 - (2.0 * 1.5))
    c1 = (1.0 + (-0.5 + 3.0))
    s0 = c1
    m0 = loom.Tensor1.map2(lambda xi, yi: max(((a - 1.5) + (a - 1.5)), b), x, y)
    m1 = loom.Tensor1.map(lambda v: ((c0 if 0.0 <= a else 0.0) if (0.25 - v) > (c0 if s0 < 3.0 else 2.0) else (c0 if 0.0 <= a else 0.0)), m0)
    return m1


@loom.entry
def p007(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((1.5 - 0.25) - 1.5)
    c1 = ((0.25 - -0.5) + c0)
    s0 = (c1 * (c1 * (b if b >= b else c0)))
    m0 = loom.Tensor1.map2(lambda xi, yi: (((1.0 if s0 < 1.0 else s0) * ((b if c0 >= s0 else s0) if (0.5 + a) < (3.0 - s0) else ((c1 - c0) * (c1 - c0)))) if (xi * (((3.0 + 3.0) if (-a) > (-0.5 if -0.5 > xi else xi) else (3.0 + 3.0)) * max(1.5, 0.25))) < (-((c1 * yi) - (s0 * 3.0))) else ((s0 if a < s0 else a) + ((((s0 - c1) * (s0 - c1)) - max(0.25, 1.5)) * (((s0 - c1) * (s0 - c1)) - max(0.25, 1.5))))), x, y)
    m1 = loom.Tensor1.map(lambda v: min((c0 * c1), ((b - 0.0) + (b - 0.0))), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: (b if 1.0 < b else 1.0), m1, w))


@loom.entry
def p008(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    s0 = ((3.0 + b) if max(b, -0.5) > ((-0.5 - b) * (-0.5 - b)) else min(a, b))
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    m0 = loom.Tensor1.map2(lambda xi, yi: ((-s0) + 1.5), x, y)
    m1 = loom.Tensor1.map(lambda v: ((a * (0.25 * -0.5)) + -0.5), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: (b * ((b if b <= s0 else b) * max(0.0, -0.5))), m1, w))


@loom.entry
def p009(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    c0 = (-2.0 - (0.0 * 0.25))
    m0 = loom.Tensor1.map2(lambda xi, yi: 0.5, x, y)
    m1 = loom.Tensor1.map(lambda v: c0, m0)
    return m1


@loom.entry
def p010(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    s0 = -0.5
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    m0 = loom.Tensor1.map2(lambda xi, yi: (yi if yi < 2.0 else 2.0), x, y)
    m1 = loom.Tensor1.map(lambda v: ((b * (v * a)) if (v if s0 >= 0.0 else 3.0) < ((s0 - -0.5) + (s0 - -0.5)) else (1.5 if v > s0 else 1.5)), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: p, m1, w))


@loom.entry
def p011(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    s0 = ((a if a <= b else a) * b)
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    m0 = loom.Tensor1.map2(lambda xi, yi: (((yi if b > yi else b) - (xi / ((a * s0) * (a * s0) + 1.0))) * ((yi if b > yi else b) - (xi / ((a * s0) * (a * s0) + 1.0)))), x, y)
    m1 = loom.Tensor1.map(lambda v: ((3.0 * 0.5) if min(v, b) > (2.0 if 2.0 < 1.0 else 1.0) else (3.0 * 0.5)), m0)
    return m1


@loom.entry
def p012(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((0.5 * -2.0) + -0.5)
    s0 = (-2.0 * ((b / (b * b + 1.0)) * max(a, b)))
    m0 = loom.Tensor1.map2(lambda xi, yi: b, x, y)
    m1 = loom.Tensor1.map(lambda v: (((a - b) * (a - b)) + (c0 * a)), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: (q * ((--0.5) * (c0 + c0))), m1, w))


@loom.entry
def p013(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    c0 = 2.0
    c1 = (0.0 * 1.5)
    s0 = min((c0 if b <= c1 else b), (c1 + a))
    m0 = loom.Tensor1.map2(lambda xi, yi: c0, x, y)
    m1 = loom.Tensor1.map(lambda v: (a - (1.5 + b)), m0)
    return m1


@loom.entry
def p014(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    s0 = (0.25 - (b * 3.0))
    m0 = loom.Tensor1.map2(lambda xi, yi: (xi if xi < xi else xi), x, y)
    return m0


@loom.entry
def p015(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((-2.0 + 2.0) - (0.25 * 3.0))
    c1 = 0.0
    m0 = loom.Tensor1.map2(lambda xi, yi: 0.5, x, y)
    m1 = loom.Tensor1.map(lambda v: 2.0, m0)
    return loom.Tensor1.reduce_max(m1)


@loom.entry
def p016(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    c0 = ((-2.0 + 0.5) * (-0.5 + 1.0))
    c1 = (2.0 * -2.0)
    m0 = loom.Tensor1.map2(lambda xi, yi: ((0.25 - c1) + max(c1, c0)), x, y)
    return m0


@loom.entry
def p017(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    s0 = (b if b > 1.0 else 1.0)
    m0 = loom.Tensor1.map2(lambda xi, yi: (xi if (2.0 * 2.0) > (yi - s0) else xi), x, y)
    return m0


@loom.entry
def p018(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((1.0 - 1.5) + 1.0)
    c1 = (2.0 - (-2.0 * 3.0))
    s0 = (c0 * ((0.25 if 1.0 > a else 0.25) * c0))
    m0 = loom.Tensor1.map2(lambda xi, yi: ((c1 + 2.0) + ((1.5 - s0) * (1.5 - s0))), x, y)
    return loom.Tensor1.reduce_max(m0)


@loom.entry
def p019(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((0.5 - 0.0) - (1.5 + 0.0))
    c1 = -0.5
    s0 = max((a + 1.5), (c1 - -2.0))
    m0 = loom.Tensor1.map2(lambda xi, yi: (a * -2.0), x, y)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: max(s0, c0), m0, w))


@loom.entry
def p020(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    c0 = ((3.0 - -2.0) + 3.0)
    s0 = (((c0 * (c0 * a)) - (c0 * 1.0)) + ((c0 * (c0 * a)) - (c0 * 1.0)))
    m0 = loom.Tensor1.map2(lambda xi, yi: (xi if xi < xi else xi), x, y)
    m1 = loom.Tensor1.map(lambda v: (((a - v) + (a - v)) / (b * b + 1.0)), m0)
    return m1


@loom.entry
def p021(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = 0.0
    m0 = loom.Tensor1.map2(lambda xi, yi: min(min(xi, (b + -0.5)), max((c0 if a < c0 else a), xi)), x, y)
    m1 = loom.Tensor1.map(lambda v: (3.0 + (-a)), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: c0, m1, w))


@loom.entry
def p022(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((1.5 + 3.0) * (1.5 * 0.25))
    c1 = 1.5
    s0 = a
    m0 = loom.Tensor1.map2(lambda xi, yi: ((c0 / (1.0 * 1.0 + 1.0)) * min(c0, c1)), x, y)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: ((c0 * 0.25) if (c0 * b) < ((2.0 - 0.0) * (2.0 - 0.0)) else (-0.5)), m0, w))


@loom.entry
def p023(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((0.25 * 0.25) + (0.5 + -0.5))
    c1 = 0.0
    s0 = a
    m0 = loom.Tensor1.map2(lambda xi, yi: ((a * ((1.0 - yi) * (c1 if a < c1 else a))) - 0.0), x, y)
    return loom.Tensor1.reduce_max(m0)


@loom.entry
def p024(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    m0 = loom.Tensor1.map2(lambda xi, yi: b, x, y)
    m1 = loom.Tensor1.map(lambda v: (((a if b > v else a) - max(1.0, b)) * ((a if b > v else a) - max(1.0, b))), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: q, m1, w))


@loom.entry
def p025(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    c0 = ((0.25 + 0.25) + (0.0 * 3.0))
    c1 = 2.0
    m0 = loom.Tensor1.map2(lambda xi, yi: yi, x, y)
    m1 = loom.Tensor1.map(lambda v: (c0 - (v if -0.5 >= a else v)), m0)
    return m1


@loom.entry
def p026(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    c0 = 0.25
    s0 = b
    m0 = loom.Tensor1.map2(lambda xi, yi: ((xi - 0.0) - (0.0 if 0.0 < xi else xi)), x, y)
    m1 = loom.Tensor1.map(lambda v: (a * (a * (b + s0))), m0)
    return m1


@loom.entry
def p027(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    s0 = (a * (a * (3.0 * b)))
    m0 = loom.Tensor1.map2(lambda xi, yi: (((0.5 if 0.5 > b else b) - (1.0 - -2.0)) - (a if a < xi else xi)), x, y)
    m1 = loom.Tensor1.map(lambda v: ((b * (s0 * s0)) if (v if a < a else b) < 3.0 else (-0.5 if -0.5 < -0.5 else -0.5)), m0)
    return m1


@loom.entry
def p028(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    s0 = a
    m0 = loom.Tensor1.map2(lambda xi, yi: ((2.0 - (b if 2.0 >= yi else yi)) + (2.0 - (b if 2.0 >= yi else yi))), x, y)
    m1 = loom.Tensor1.map(lambda v: ((b + s0) * (v / (v * v + 1.0))), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: (a if 1.0 > a else 1.0), m1, w))


@loom.entry
def p029(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    m0 = loom.Tensor1.map2(lambda xi, yi: ((b if yi < b else yi) - 3.0), x, y)
    m1 = loom.Tensor1.map(lambda v: a, m0)
    return m1


@loom.entry
def p030(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = 2.0
    s0 = c0
    m0 = loom.Tensor1.map2(lambda xi, yi: (1.5 * max(a, s0)), x, y)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: ((q if q < p else p) / ((s0 * (q * s0)) * (s0 * (q * s0)) + 1.0)), m0, w))


@loom.entry
def p031(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    c0 = 0.0
    c1 = ((-0.5 * 1.5) * -0.5)
    m0 = loom.Tensor1.map2(lambda xi, yi: (xi if -0.5 < (0.25 * c0) else b), x, y)
    m1 = loom.Tensor1.map(lambda v: ((c1 * (c1 * c0)) if (c0 * 2.0) >= (a * (v * b)) else (c1 + c0)), m0)
    return m1


@loom.entry
def p032(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    m0 = loom.Tensor1.map2(lambda xi, yi: (((xi - (yi if b >= 2.0 else yi)) + (xi - (yi if b >= 2.0 else yi))) - (yi + (1.5 * (3.0 * yi)))), x, y)
    m1 = loom.Tensor1.map(lambda v: (min(-0.5, v) if (b - b) < (a * (0.0 * b)) else v), m0)
    return m1


@loom.entry
def p033(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((0.5 * 0.25) + (1.5 + 1.0))
    c1 = 1.5
    m0 = loom.Tensor1.map2(lambda xi, yi: (3.0 * ((c1 if 0.25 < c1 else a) * 0.5)), x, y)
    return loom.Tensor1.reduce_max(m0)


@loom.entry
def p034(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = (1.0 - (1.0 - 1.0))
    m0 = loom.Tensor1.map2(lambda xi, yi: ((b * (-0.5 - xi)) + ((-0.5 * yi) if min(c0, -0.5) >= (a * (b * 0.5)) else (b if yi <= yi else 1.5))), x, y)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: ((a / (p * p + 1.0)) - 1.0), m0, w))


@loom.entry
def p035(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    s0 = ((min(a, b) - (a / (a * a + 1.0))) * (min(a, b) - (a / (a * a + 1.0))))
    m0 = loom.Tensor1.map2(lambda xi, yi: ((((xi / (s0 * s0 + 1.0)) / ((a + s0) * (a + s0) + 1.0)) - (s0 if s0 < s0 else s0)) + (((xi / (s0 * s0 + 1.0)) / ((a + s0) * (a + s0) + 1.0)) - (s0 if s0 < s0 else s0))), x, y)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: (q if b < q else b), m0, w))


@loom.entry
def p036(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = 1.5
    c1 = ((-2.0 - 3.0) * (-0.5 * c0))
    m0 = loom.Tensor1.map2(lambda xi, yi: c1, x, y)
    m1 = loom.Tensor1.map(lambda v: ((v + c0) if (c1 if b <= c1 else b) < ((b - v) * (b - v)) else (b - c0)), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: (c1 if p < c1 else p), m1, w))


@loom.entry
def p037(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> loom.Tensor1:
    s0 = (b * ((a * b) * b))
    m0 = loom.Tensor1.map2(lambda xi, yi: ((-1.5) - min(0.25, xi)), x, y)
    return m0


@loom.entry
def p038(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    c0 = ((1.0 * 0.0) + (1.5 + -0.5))
    c1 = ((0.25 + 0.5) + (0.25 - 0.25))
    s0 = (c1 if c1 < c1 else c1)
    m0 = loom.Tensor1.map2(lambda xi, yi: (a - (c1 - ((xi if xi > c0 else c0) * min(c0, b)))), x, y)
    m1 = loom.Tensor1.map(lambda v: ((c0 if a < c0 else a) + (a * (a * c0))), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: (q if q < s0 else s0), m1, w))


@loom.entry
def p039(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    s0 = min(a, (a if a < b else b))
    unused = loom.Tensor1.map(lambda xi: xi * a, x)
    m0 = loom.Tensor1.map2(lambda xi, yi: (a * min(((b if s0 >= s0 else s0) + (0.25 / (s0 * s0 + 1.0))), xi)), x, y)
    m1 = loom.Tensor1.map(lambda v: ((-3.0) if a >= (2.0 if 0.5 > 2.0 else 0.5) else (b - -0.5)), m0)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: ((-2.0 * (s0 * q)) - s0), m1, w))
