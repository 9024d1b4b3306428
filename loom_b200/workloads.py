"""The hot path's workload configurations and their seeded synthetic inputs.

Five configurations, each an entry of the ``kernels`` module of the shipped
suite package (``loom_b200/suite``):

  1. saxpy        map2  y_out = a*x + y,   a = 2.5,  x, y ~ U(-1, 1),   N = 2^24
  2. relu         map   max(x, 0),                   x ~ N(0, 1),      N = 2^26
  3. dot          sum(x*y) (fused map2 -> reduce),   x, y ~ U(-1, 1),  N = 2^28
  4. l2_norm_sq   sum(x*x) and max_value max(x) on one vector,
                  x ~ N(0, 1) with a seeded 1% of entries scaled by 1e3, N = 2^30
  5. affine_relu  z = relu(a*x + y) and pipeline_sum s = sum(relu(a*x + y)*w),
                  a = 0.75, x, y, w ~ U(-1, 1),  N = 2^10 ... 2^32

The base seed is the reference harness's (``experiments/source/data/tuning/
settings.json``: 20260417) and the k-th tensor input of a call adds
k*104729 (``experiments/source/harness/run.py`` seeds its inputs that way).
Inputs are generated on the host with numpy's PCG64, so the same arrays feed
both the GPU and the CPU oracle.  There is no public dataset for this path:
all data is synthetic with the shapes and distributions above.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

BASE_SEED = 20260417
INPUT_SEED_STRIDE = 104729


@dataclass(frozen=True)
class Config:
    name: str
    entries: Tuple[str, ...]     # suite entries exercised by this configuration
    n: int
    dist: str                    # "uniform" | "normal" | "normal_outliers"
    tensors: Tuple[str, ...]
    scalars: Tuple[Tuple[str, float], ...] = ()


CONFIGS: List[Config] = [
    Config("saxpy", ("saxpy",), 1 << 24, "uniform", ("x", "y"), (("a", 2.5),)),
    Config("relu", ("relu",), 1 << 26, "normal", ("x",)),
    Config("dot", ("dot",), 1 << 28, "uniform", ("x", "y")),
    Config("l2_norm_sq_max", ("l2_norm_sq", "max_value"), 1 << 30, "normal_outliers", ("x",)),
    Config("pipeline", ("affine_relu", "pipeline_sum"), 1 << 22, "uniform", ("x", "y", "w"),
           (("a", 0.75),)),
]

PIPELINE_SWEEP = [1 << 10, 1 << 14, 1 << 18, 1 << 22, 1 << 26, 1 << 30, 1 << 32]

# Entry -> (tensor params in call order, scalar params with their values, input distribution)
ENTRY_SPECS: Dict[str, Tuple[Tuple[str, ...], Tuple[Tuple[str, float], ...], str]] = {
    "saxpy": (("x", "y"), (("a", 2.5),), "uniform"),
    "relu": (("x",), (), "normal"),
    "dot": (("x", "y"), (), "uniform"),
    "l2_norm_sq": (("x",), (), "normal_outliers"),
    "max_value": (("x",), (), "normal_outliers"),
    "affine_relu": (("x", "y"), (("a", 0.75),), "uniform"),
    "pipeline_sum": (("x", "y", "w"), (("a", 0.75),), "uniform"),
}


def generate(dist: str, n: int, seed: int) -> np.ndarray:
    """n float32 values of distribution `dist` from PCG64(seed)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if dist == "uniform":
        out = rng.random(n, dtype=np.float32)
        out *= np.float32(2.0)
        out -= np.float32(1.0)
        return out
    if dist == "normal":
        return rng.standard_normal(n, dtype=np.float32)
    if dist == "normal_outliers":
        out = rng.standard_normal(n, dtype=np.float32)
        k = max(1, n // 100)
        idx = rng.choice(n, size=k, replace=False) if n <= (1 << 26) else \
            rng.integers(0, n, size=k)
        out[idx] *= np.float32(1e3)
        return out
    raise ValueError(f"unknown distribution {dist!r}")


def harness_inputs(tensor_inputs, scalar_args, n: int, seed_offset: int = 0) -> Dict[str, object]:
    """Seeded host inputs for one kernel of the reference harness's table
    (``experiments/source/data/common/workloads.json``).

    The harness draws every tensor from N(0, 1) with seed ``base + n +
    seed_offset + k*104729`` for the k-th tensor input and passes the table's
    scalar arguments as floats (``experiments/source/harness/run.py:941-960``;
    the ``+ n`` is its ``config["seed"] + size``).  It generates on the GPU
    with torch; these inputs keep the seeds and the distribution but come
    from numpy's PCG64 on the host, so the CPU oracle sees the same arrays.
    """
    seed = BASE_SEED + n + seed_offset
    out: Dict[str, object] = {}
    for k, name in enumerate(tensor_inputs):
        out[name] = generate("normal", n, seed + k * INPUT_SEED_STRIDE)
    for name, value in dict(scalar_args).items():
        out[name] = float(value)
    return out


def entry_inputs(entry: str, n: int, seed_offset: int = 0) -> Dict[str, object]:
    """Seeded host inputs for one suite entry (tensor k gets seed + k*104729)."""
    tensors, scalars, dist = ENTRY_SPECS[entry]
    out: Dict[str, object] = {}
    for k, name in enumerate(tensors):
        out[name] = generate(dist, n, BASE_SEED + seed_offset + k * INPUT_SEED_STRIDE)
    for name, value in scalars:
        out[name] = value
    return out
