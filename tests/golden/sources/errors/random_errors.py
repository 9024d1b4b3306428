"""Seeded entries that the Loom entry language rejects (make_random_errors.py)."""

import math

import loom


@loom.entry
def e000(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: (xi ** 2.0), x)


@loom.entry
def e001(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: (undefined_name * a), x)


@loom.entry
def e002(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: (yi * max(yi, b=a)), x, y)


@loom.entry
def e003(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: max((xi - max(a, b=xi)), a), x, y)


@loom.entry
def e004(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: (1.0 if xi else a), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e005(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: (a * (xi - max(max(yi, b=xi), 1.5))), x, y)


@loom.entry
def e006(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: max(undefined_name, a), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e007(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: (yi + (((yi @ xi) * yi) + yi)), x, y)


@loom.entry
def e008(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: (not (a > xi)), x)


@loom.entry
def e009(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: ((a * (0.25 - (xi ** 2.0))) * 1.5), x)


@loom.entry
def e010(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: (1.0 if yi else a), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e011(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: (1.5 + abs(yi)), x, y)


@loom.entry
def e012(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: max(max(max(a, b=yi), 1.5), xi), x, y)


@loom.entry
def e013(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: (a * [a]), x, y)


@loom.entry
def e014(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: ([xi] * 1.5), x, y)


@loom.entry
def e015(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: (xi * (yi * abs(yi))), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e016(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: (-a if a > yi else True), x, y)


@loom.entry
def e017(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: ((0.25 - (a @ xi)) * a), x)


@loom.entry
def e018(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: (loom.Tensor1.reduce_sum(xi) - 0.25), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e019(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: max(a, b=yi), x, y)


@loom.entry
def e020(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: math.floor(a), x)


@loom.entry
def e021(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: max((1.0 if a else xi), a), x)


@loom.entry
def e022(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: max((yi.real), 0.25), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e023(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: (max(((a < yi < 1.0) * xi), xi) - xi), x, y)


@loom.entry
def e024(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: lambda_missing(yi), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e025(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: max(((a % 2.0) + 1.5), yi), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e026(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: (1.5 + ((lambda_missing(yi) + 0.25) * a)), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e027(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: (xi // yi), x, y)


@loom.entry
def e028(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: max((xi - (True + a)), xi), x)


@loom.entry
def e029(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: (undefined_name - yi), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e030(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: max(max(max((a // xi), a), 1.5), 0.25), x)


@loom.entry
def e031(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: (1.5 + (1.5 + (not (a > xi)))), x)


@loom.entry
def e032(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: max((max(undefined_name, 1.5) - 1.5), xi), x, y)


@loom.entry
def e033(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: lambda_missing(a), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e034(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: (((1.5 - loom.Tensor1.reduce_sum(xi)) - 1.5) - 1.5), x)


@loom.entry
def e035(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: ((xi - (a ** 2.0)) * 1.5), x)


@loom.entry
def e036(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: max(((a * (yi % 2.0)) - xi), xi), x, y)


@loom.entry
def e037(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: ((yi * max((-xi if xi > a else True), yi)) * 1.5), x, y)
    return loom.Tensor1.reduce_sum(m)


@loom.entry
def e038(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: ((a * (1.0 if a else xi)) - xi), x)


@loom.entry
def e039(a: float, x: loom.Tensor1, y: loom.Tensor1) -> float:
    m = loom.Tensor1.map2(lambda xi, yi: (xi - (math.floor(a) * 1.5)), x, y)
    return loom.Tensor1.reduce_sum(m)
