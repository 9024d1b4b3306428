"""The B200 benchmark suite: the five workload configurations of the Loom
hot path, written in Loom's Python entry language (one module, ``kernels``).

saxpy / relu / dot / l2_norm_sq are the reference's own example entries
(examples/saxpy.py, examples/relu.py, examples/dot.py, examples/l2_norm_sq.py);
max_value is the reduce_max entry of the l2_norm_sq/reduce_max pair;
affine_relu and pipeline_sum are the two entries of the fused pipeline
package (z = relu(a*x + y), s = sum(z * w)).
"""

import loom


@loom.entry
def saxpy(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: a * xi + yi, x, y)


@loom.entry
def relu(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: xi if xi > 0.0 else 0.0, x)


@loom.entry
def dot(x: loom.Tensor1, y: loom.Tensor1) -> float:
    products = loom.Tensor1.map2(lambda xi, yi: xi * yi, x, y)
    return loom.Tensor1.reduce_sum(products)


@loom.entry
def l2_norm_sq(x: loom.Tensor1) -> float:
    squares = loom.Tensor1.map(lambda xi: xi * xi, x)
    return loom.Tensor1.reduce_sum(squares)


@loom.entry
def max_value(x: loom.Tensor1) -> float:
    return loom.Tensor1.reduce_max(x)


@loom.entry
def affine_relu(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(
        lambda xi, yi: (a * xi + yi) if (a * xi + yi) > 0.0 else 0.0, x, y)


@loom.entry
def pipeline_sum(a: float, x: loom.Tensor1, y: loom.Tensor1, w: loom.Tensor1) -> float:
    z = loom.Tensor1.map2(
        lambda xi, yi: (a * xi + yi) if (a * xi + yi) > 0.0 else 0.0, x, y)
    products = loom.Tensor1.map2(lambda zi, wi: zi * wi, z, w)
    return loom.Tensor1.reduce_sum(products)
