"""Seeded random entries over the structured forms of the entry language (make_front_programs.py)."""

import math

import loom


@loom.entry
def f000(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    p, q = (a * 1.0), 2.0
    s: float = ((a + -0.25) - log(q * q + 1.0))
    def h0(u: float) -> float:
        if u > (s * u):
            return (min(3.0, 3.0) if (a if s <= a else s) == a else (q - a))
        else:
            return exp(min((q - a), 3.0))
    def h1(u: float, v: float) -> float:
        if u > (2.0 + s):
            return h0(select(a > v, v, u))
        else:
            return ((a + s) - 1.0)
    m = loom.Tensor1.map2(lambda xi, yi: (h1((a if p >= -0.25 else a), log(a * a + 1.0)) * h0(a)), x, y)
    return m


@loom.entry
def f001(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    p, q = a, (a if 1.0 == a else a)
    s: float = loom.max(select(1.0 > a, q, 0.5), log(3.0 * 3.0 + 1.0))
    def h0(u: float, v: float) -> float:
        return ((+0.0) - (p if 2.0 >= u else a))
    def h1(u: float) -> float:
        return s
    def h2(u: float) -> float:
        if u > 1.0:
            return ((u - a) - h1(0.0))
        else:
            return a
    m = loom.Tensor1.map(h2, x)
    return m


@loom.entry
def f002(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = (a - a), (+1.0)
    s: float = loom.sqrt((a * p) * (a * p) + 1.0)
    def h0(u: float) -> float:
        return min((+q), q)
    def h1(u: float) -> float:
        return (u + (a * s))
    def h2(u: float) -> float:
        if u > u:
            return u
        else:
            return (+h0(s))
    m = loom.Tensor1.map2(lambda xi, yi: (select(a > select(s > p, yi, xi), 2.0, q) if 1.0 > (+0.0) else (+q)), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def f003(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = a, (a - a)
    def h0(u: float) -> float:
        return loom.max((q * q), (u * a))
    def h1(u: float, v: float) -> float:
        if u > p:
            return loom.max(math.sqrt(a * a + 1.0), (v if 0.5 < a else u))
        else:
            return min((a + v), (a - p))
    def h2(u: float, v: float) -> float:
        return a
    m = loom.Tensor1.map2(lambda xi, yi: p, x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def f004(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    p, q = loom.max(a, a), (a * a)
    s: float = (q if loom.sqrt(a * a + 1.0) >= math.sqrt(q * q + 1.0) else (q - a))
    def h0(u: float) -> float:
        if u > min(p, p):
            return ((0.0 if u > q else a) if (q if q <= s else u) <= 0.0 else (+a))
        else:
            return math.sqrt((1.0 - p) * (1.0 - p) + 1.0)
    def h1(u: float) -> float:
        if u > (1.0 - a):
            return p
        else:
            return (+(p if s > s else u))
    m = loom.Tensor1.map2(lambda xi, yi: p, x, y)
    return m


@loom.entry
def f005(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = a, select(a > a, a, a)
    def h0(u: float, v: float) -> float:
        if u > select(u > p, a, p):
            return log((u * u) * (u * u) + 1.0)
        else:
            return (+a)
    def h1(u: float, v: float) -> float:
        if u > (1.0 if u <= p else q):
            return ((a + q) + h0(p, u))
        else:
            return select((+v) > 0.0, h0(u, u), (u if a <= p else p))
    m = loom.Tensor1.map2(lambda xi, yi: (+xi), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def f006(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    def h0(u: float) -> float:
        if u > (a if u <= u else u):
            return select((u + u) > (a if a == 0.0 else 2.0), (u + a), (a - u))
        else:
            return select((0.0 + 3.0) > loom.max(u, u), (a * u), (a if u < a else a))
    def h1(u: float, v: float) -> float:
        if u > loom.max(1.0, u):
            return math.sqrt(0.5 * 0.5 + 1.0)
        else:
            return (select(v > -0.25, v, a) if 1.0 >= (u if 0.0 < u else 3.0) else v)
    m = loom.Tensor1.map2(lambda xi, yi: h0(min(loom.max(2.0, -0.25), select(a > 3.0, a, yi))), x, y)
    def total(t: loom.Tensor1) -> float:
        return loom.Tensor1.reduce_sum(t)
    return total(loom.Tensor1.map(lambda v: v * v, m))


@loom.entry
def f007(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    s: float = ((a * a) - (a + a))
    def h0(u: float) -> float:
        if u > (s * a):
            return u
        else:
            return (u * (a + u))
    m = loom.Tensor1.map(h0, x)
    def total(t: loom.Tensor1) -> float:
        return loom.Tensor1.reduce_sum(t)
    return total(loom.Tensor1.map(lambda v: v * v, m))


@loom.entry
def f008(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = (a + a), exp(min(a, 3.0))
    s: float = p
    def h0(u: float, v: float) -> float:
        return (+math.sqrt(q * q + 1.0))
    def h1(u: float) -> float:
        return (math.sqrt(0.0 * 0.0 + 1.0) + min(q, s))
    def h2(u: float, v: float) -> float:
        if u > a:
            return h1(q)
        else:
            return ((v + 3.0) + (s - v))
    m = loom.Tensor1.map2(lambda xi, yi: a, x, y)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f009(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    def h0(u: float) -> float:
        return ((a if a < a else 0.5) if (+u) == exp(min(3.0, 3.0)) else (3.0 if a <= a else a))
    def h1(u: float, v: float) -> float:
        return (h0(v) if (0.0 if v > u else u) <= (v if 0.5 >= v else u) else 3.0)
    m = loom.Tensor1.map2(h1, x, y)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f010(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    s: float = (exp(min(a, 3.0)) if math.sqrt(a * a + 1.0) > log(a * a + 1.0) else (3.0 * a))
    def h0(u: float, v: float) -> float:
        return v
    def h1(u: float) -> float:
        if u > (a if s > s else s):
            return (+s)
        else:
            return (0.0 - (a - u))
    def h2(u: float) -> float:
        return s
    m = loom.Tensor1.map(h1, x)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f011(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    p, q = (a if a >= a else a), loom.max(a, a)
    def h0(u: float) -> float:
        return ((a if a == u else q) if (-0.25 + u) >= (2.0 - u) else q)
    m = loom.Tensor1.map(h0, x)
    return m


@loom.entry
def f012(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = (0.5 - a), a
    def h0(u: float, v: float) -> float:
        if u > q:
            return (a * (u * v))
        else:
            return 3.0
    def h1(u: float) -> float:
        return loom.max((u + p), (u if a < q else u))
    def h2(u: float) -> float:
        return ((u - q) - math.sqrt(3.0 * 3.0 + 1.0))
    m = loom.Tensor1.map2(h0, x, y)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f013(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    p, q = (3.0 - a), (a * a)
    def h0(u: float) -> float:
        if u > (p + q):
            return min((a + a), (p - u))
        else:
            return ((0.0 + p) if min(-0.25, q) > u else q)
    def h1(u: float) -> float:
        return 0.5
    def h2(u: float, v: float) -> float:
        return h0(h0(p))
    m = loom.Tensor1.map(h0, x)
    return m


@loom.entry
def f014(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    s: float = a
    def h0(u: float) -> float:
        if u > (+3.0):
            return a
        else:
            return select((+u) > a, loom.max(0.5, a), (a - a))
    def h1(u: float) -> float:
        if u > u:
            return ((s * u) + a)
        else:
            return h0((s * a))
    m = loom.Tensor1.map(h1, x)
    return m


@loom.entry
def f015(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    s: float = select((0.0 if a == a else a) > (a if a >= a else a), (1.0 - 0.0), (+0.0))
    def h0(u: float) -> float:
        return ((a if a > -0.25 else s) + (-0.25 + s))
    m = loom.Tensor1.map(h0, x)
    def total(t: loom.Tensor1) -> float:
        return loom.Tensor1.reduce_sum(t)
    return total(loom.Tensor1.map(lambda v: v * v, m))


@loom.entry
def f016(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    def h0(u: float, v: float) -> float:
        return ((v if u <= u else a) if loom.sqrt(u * u + 1.0) <= select(a > u, a, u) else (v if v < u else u))
    m = loom.Tensor1.map2(h0, x, y)
    return m


@loom.entry
def f017(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = (a if a < a else a), (a if 1.0 == a else a)
    def h0(u: float, v: float) -> float:
        return (select(3.0 > q, v, v) + (3.0 - v))
    m = loom.Tensor1.map2(h0, x, y)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f018(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = (a + a), (a * 0.5)
    def h0(u: float, v: float) -> float:
        return select(log(q * q + 1.0) > (0.0 if q == v else q), (q if u < 1.0 else -0.25), (p * u))
    def h1(u: float) -> float:
        return a
    def h2(u: float) -> float:
        if u > (p + -0.25):
            return (+p)
        else:
            return h0(0.0, select(q > 3.0, q, a))
    m = loom.Tensor1.map(h1, x)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def f019(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    s: float = (a * exp(min(a, 3.0)))
    def h0(u: float) -> float:
        return a
    def h1(u: float) -> float:
        if u > (a - s):
            return (+h0(u))
        else:
            return h0((u if u <= s else u))
    m = loom.Tensor1.map2(lambda xi, yi: select(((+yi) - (xi if -0.25 > xi else s)) > h1((s - a)), (a * (a + xi)), 0.0), x, y)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f020(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    s: float = a
    def h0(u: float, v: float) -> float:
        return ((u + a) - (u + a))
    def h1(u: float) -> float:
        return h0(h0(u, s), (s - s))
    m = loom.Tensor1.map2(lambda xi, yi: (1.0 if (yi - (xi - yi)) >= ((yi + a) - (0.0 if s == 0.0 else a)) else h1(h0(a, a))), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def f021(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    def h0(u: float) -> float:
        if u > math.sqrt(u * u + 1.0):
            return ((u * 2.0) * (u + u))
        else:
            return math.sqrt((+a) * (+a) + 1.0)
    def h1(u: float, v: float) -> float:
        return (log(v * v + 1.0) if select(u > u, u, v) == u else h0(2.0))
    m = loom.Tensor1.map(h0, x)
    def total(t: loom.Tensor1) -> float:
        return loom.Tensor1.reduce_sum(t)
    return total(loom.Tensor1.map(lambda v: v * v, m))


@loom.entry
def f022(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    s: float = ((3.0 if a <= a else a) - (a - a))
    def h0(u: float) -> float:
        return (+(u - u))
    def h1(u: float) -> float:
        return select(h0(a) > (s if 0.0 < 1.0 else 0.0), exp(min(u, 3.0)), a)
    def h2(u: float) -> float:
        return math.sqrt(a * a + 1.0)
    m = loom.Tensor1.map(h0, x)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def f023(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = (1.0 - a), (a if 0.0 <= a else -0.25)
    def h0(u: float, v: float) -> float:
        return (+(2.0 if u == p else p))
    def h1(u: float) -> float:
        if u > (+u):
            return p
        else:
            return (0.5 + (1.0 + 1.0))
    m = loom.Tensor1.map2(h0, x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def f024(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = a, (a + a)
    s: float = (p if (p * q) >= (0.5 - q) else (a * 1.0))
    def h0(u: float) -> float:
        if u > (+s):
            return (s - q)
        else:
            return (p - loom.max(q, a))
    def h1(u: float) -> float:
        if u > log(s * s + 1.0):
            return (p if (p if 0.0 > q else u) < exp(min(0.5, 3.0)) else (s * p))
        else:
            return log((-0.25 if u > q else 1.0) * (-0.25 if u > q else 1.0) + 1.0)
    m = loom.Tensor1.map2(lambda xi, yi: yi, x, y)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f025(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = a, min(3.0, a)
    s: float = math.sqrt((q + 0.5) * (q + 0.5) + 1.0)
    def h0(u: float, v: float) -> float:
        return ((a - v) if (q if v == a else a) <= (v if v == s else u) else (2.0 if 0.0 <= q else q))
    def h1(u: float, v: float) -> float:
        if u > (q * 0.0):
            return ((s if s == 0.0 else s) - select(q > u, v, p))
        else:
            return v
    def h2(u: float, v: float) -> float:
        if u > q:
            return u
        else:
            return (+(2.0 * u))
    m = loom.Tensor1.map2(lambda xi, yi: log(((p + -0.25) if (2.0 if yi >= yi else s) <= min(xi, s) else (p - yi)) * ((p + -0.25) if (2.0 if yi >= yi else s) <= min(xi, s) else (p - yi)) + 1.0), x, y)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f026(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    def h0(u: float, v: float) -> float:
        return exp(min(select(a > v, v, 1.0), 3.0))
    def h1(u: float, v: float) -> float:
        if u > exp(min(a, 3.0)):
            return ((u if u == v else v) * h0(v, a))
        else:
            return ((+0.0) + h0(u, u))
    def h2(u: float, v: float) -> float:
        return ((v if v == a else u) if (v - a) == math.sqrt(0.0 * 0.0 + 1.0) else (v - u))
    m = loom.Tensor1.map2(h1, x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def f027(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    s: float = (+a)
    def h0(u: float) -> float:
        return exp(min((s * u), 3.0))
    m = loom.Tensor1.map2(lambda xi, yi: (((s * s) + loom.sqrt(s * s + 1.0)) + ((0.0 if a < a else a) if (a - s) == h0(s) else -0.25)), x, y)
    return m


@loom.entry
def f028(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    def h0(u: float) -> float:
        return (a - (+a))
    def h1(u: float, v: float) -> float:
        if u > (v * u):
            return (+(v - a))
        else:
            return math.sqrt((u * a) * (u * a) + 1.0)
    m = loom.Tensor1.map2(h1, x, y)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def f029(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    p, q = a, min(a, a)
    def h0(u: float, v: float) -> float:
        return select(select(v > p, u, q) > (1.0 * q), log(q * q + 1.0), (a - 2.0))
    def h1(u: float, v: float) -> float:
        return (q - (2.0 * p))
    m = loom.Tensor1.map2(h0, x, y)
    def total(t: loom.Tensor1) -> float:
        return loom.Tensor1.reduce_sum(t)
    return total(loom.Tensor1.map(lambda v: v * v, m))
