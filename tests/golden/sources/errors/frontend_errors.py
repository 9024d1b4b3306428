"""Entries outside Loom's staged language, one error each (front-end
negative tests)."""

import loom


@loom.entry
def with_loop(x: loom.Tensor1) -> loom.Tensor1:
    for _ in range(2):
        x = loom.Tensor1.map(lambda xi: xi, x)
    return x


@loom.entry
def tensor_capture(x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: xi + y, x)


@loom.entry
def chained(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: 1.0 if 0.0 < xi < 1.0 else 0.0, x)


@loom.entry
def keyword_call(x: loom.Tensor1) -> float:
    return loom.Tensor1.reduce_sum(t=x)


@loom.entry
def wrong_return(x: loom.Tensor1) -> float:
    return loom.Tensor1.map(lambda xi: xi, x)


@loom.entry
def unknown_call(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: tanh(xi), x)


@loom.entry
def tensor_branch(x: loom.Tensor1, k: float) -> loom.Tensor1:
    if k > 0.0:
        return loom.Tensor1.map(lambda xi: xi * k, x)
    else:
        return loom.Tensor1.map(lambda xi: xi, x)


@loom.entry
def power_op(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: xi ** 2.0, x)


@loom.entry
def aug_assign(a: float, x: loom.Tensor1) -> loom.Tensor1:
    b = a
    b += 1.0
    return loom.Tensor1.map(lambda xi: xi * b, x)


@loom.entry
def non_tail_if(a: float, x: loom.Tensor1) -> loom.Tensor1:
    def f(v: float) -> float:
        if v > a:
            w = v
        else:
            w = a
        return w

    return loom.Tensor1.map(f, x)


@loom.entry
def bool_not(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: select(not (xi > 0.0), xi, 0.0), x)


@loom.entry
def attribute_access(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: xi * x.shape, x)
