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
