"""Loom entries written for the front-end and body-coverage tests: local
helper functions passed to maps and applied, tuple lets, annotated lets, clamps,
soft thresholds, square roots, exp/log, division, select, negation, a tail
if statement, qualified primitives (math.sqrt, loom.max ...), unary plus and
equality, and maxes of maps.  (Its FrontIR from the reference frontend is committed under
tests/golden/front_ir/; tests/golden/make_golden.py regenerates it.)"""

import math

import loom


@loom.entry
def nested_helpers(x: loom.Tensor1, y: loom.Tensor1) -> float:
    def mul(xi: float, yi: float) -> float:
        return xi * yi

    def total(t: loom.Tensor1) -> float:
        return loom.Tensor1.reduce_sum(t)

    return total(loom.Tensor1.map2(mul, x, y))


@loom.entry
def clamp_scale(lo: float, hi: float, s: float, x: loom.Tensor1) -> loom.Tensor1:
    def clamp(v: float) -> float:
        return lo if v < lo else (hi if v > hi else v)

    return loom.Tensor1.map(lambda xi: clamp(s * xi), x)


@loom.entry
def tuple_lets(a: float, x: loom.Tensor1) -> loom.Tensor1:
    p, q = a * 2.0, a + 1.0
    scale: float = p - q
    return loom.Tensor1.map(lambda xi: scale * xi + q, x)


@loom.entry
def soft_threshold(t: float, x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: xi - t if xi > t else (xi + t if xi < -t else 0.0), x)


@loom.entry
def hypot_sum(x: loom.Tensor1, y: loom.Tensor1) -> float:
    return loom.Tensor1.reduce_sum(
        loom.Tensor1.map2(lambda xi, yi: sqrt(xi * xi + yi * yi) + max(xi, yi) - min(xi, 0.0), x, y))


@loom.entry
def neg_max(x: loom.Tensor1) -> float:
    m = loom.Tensor1.map(lambda xi: -xi, x)
    return loom.Tensor1.reduce_max(m)


@loom.entry
def ratio_exp(x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: exp(xi) / (1.0 + log(yi * yi + 1.0)), x, y)


@loom.entry
def select_floor(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: select(xi >= 0.5, xi, 0.1), x)


@loom.entry
def scaled_chain(a: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    def affine(u: float, v: float) -> float:
        return a * u - v

    d = loom.Tensor1.map2(affine, x, y)
    sq = loom.Tensor1.map(lambda di: di * di, d)
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda s_, wi: s_ / (wi * wi + 1.0), sq, w))


@loom.entry
def tail_if(k: float, x: loom.Tensor1) -> loom.Tensor1:
    def gate(v: float) -> float:
        if v > k:
            return v - k
        else:
            return 0.0

    return loom.Tensor1.map(gate, x)


@loom.entry
def qualified_prims(x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(
        lambda xi, yi: loom.select(xi <= yi, math.sqrt(xi * xi + 1.0),
                                   loom.max(xi, yi) - loom.min(yi, 0.5)), x, y)


@loom.entry
def unary_and_eq(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: select(xi == 0.0, +xi, -xi * 0.5), x)


@loom.entry
def let_chain_sum(a: float, x: loom.Tensor1) -> float:
    def f(v: float) -> float:
        u: float = v * a
        w = u - 1.0
        return u * w

    return loom.Tensor1.reduce_sum(loom.Tensor1.map(f, x))


@loom.entry
def max_of_difference(x: loom.Tensor1, y: loom.Tensor1) -> float:
    return loom.Tensor1.reduce_max(loom.Tensor1.map2(lambda xi, yi: xi - yi, x, y))
