"""Writes random_programs.tensor_ir.json: seeded random TensorIR programs for
the GPU parity test tests/test_gpu_random_programs.py.

Each program has 1-3 tensor parameters (x, y, w), 0-2 scalar parameters
(a, b) and a chain of 1-3 element-wise nodes, each reading parameters or
earlier nodes.  Its result is the last node (a map), or a sum or max over it
(a plain reduction) or over a further body of parameters and nodes (a mapped
reduction, the form the reference's reduce-map-fusion emits).  Every
reduction comes with a companion map entry, `<name>_values`, that returns the
reduced per-element values, so the test can size the sum's tolerance.

Bodies use the operators whose fp32 results are exactly rounded on both the
GPU and the host (add, sub, mul, div, min, max, neg, sqrt, comparisons and
select), so every map and max must match the oracle bit for bit.  Constants
include fractional ones, which the reference renders as double literals, and
-0.0, which its pattern guards treat as equal to 0.0.

Run from the repository root: python tests/golden/sources/random/make_random_programs.py
"""

import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(HERE))))
sys.path.insert(0, ROOT)

from loom_b200 import tensor_ir as TI  # noqa: E402
from loom_b200.frontend.lower import annotate  # noqa: E402

SEED = 20260417
N_PROGRAMS = 36
CONSTS = [0.0, -0.0, 1.0, -1.0, 2.0, 3.0, 0.5, 0.25, -0.75, 1.5, 0.001, 10.0]


def fexpr(rng, depth, names):
    """A float-valued expression over `names`."""
    if depth == 0 or rng.random() < 0.2:
        if rng.random() < 0.75:
            return TI.SVar(rng.choice(names))
        return TI.SConstF32(rng.choice(CONSTS))
    k = rng.random()
    if k < 0.12:
        return TI.SUnary(rng.choice(["neg", "sqrt"]), fexpr(rng, depth - 1, names))
    if k < 0.32:
        cond = TI.SBinary(rng.choice(TI.COMPARE_OPS), fexpr(rng, depth - 1, names),
                          fexpr(rng, depth - 1, names))
        then = cond.lhs if rng.random() < 0.4 else fexpr(rng, depth - 1, names)
        els = cond.rhs if rng.random() < 0.4 else fexpr(rng, depth - 1, names)
        return TI.SSelect(cond, then, els)
    op = rng.choice(["add", "sub", "mul", "div", "min", "max", "add", "mul"])
    return TI.SBinary(op, fexpr(rng, depth - 1, names), fexpr(rng, depth - 1, names))


def scalars_in(expr):
    return [v for v in dict.fromkeys(TI.free_vars(expr)) if v in ("a", "b")]


def body_node(rng, node_id, sources, uses_all=()):
    """An element-wise node over 1-2 of `sources` (parameter or node refs)."""
    k = 1 if len(sources) == 1 else rng.choice([1, 2, 2])
    picked = list(uses_all) or rng.sample(sources, k)
    picked = picked[:2] if len(picked) > 2 else picked
    bind = ["u", "v"][:len(picked)]
    names = bind + [s for s in ("a", "b") if rng.random() < 0.35]
    body = fexpr(rng, rng.randint(1, 4), names)
    # every binding is read by the body
    for b in bind:
        if b not in TI.free_vars(body):
            body = TI.SBinary(rng.choice(["add", "mul", "sub"]), body, TI.SVar(b))
    inputs = tuple(TI.InputBinding(b, s) for b, s in zip(bind, picked))
    return TI.Elementwise1D(node_id, inputs, tuple(scalars_in(body)), body)


def program(rng, index):
    n_tensors = rng.randint(1, 3)
    tensors = ["x", "y", "w"][:n_tensors]
    params_t = [TI.ParamRef(t) for t in tensors]
    nodes = []
    sources = list(params_t)
    unused = list(params_t)
    for j in range(rng.randint(1, 3)):
        need = unused[:2] if (j == 0 and len(unused) >= 2 and rng.random() < 0.5) else ()
        node = body_node(rng, j, sources, need)
        for b in node.inputs:
            if b.source in unused:
                unused.remove(b.source)
        nodes.append(node)
        sources.append(TI.NodeRef(j))
    last = TI.NodeRef(nodes[-1].id)
    r = rng.random()
    kind = "map" if r < 0.45 else ("sum" if r < 0.75 else "max")
    if unused and kind == "map":     # fold the unread parameters into the result
        node = body_node(rng, len(nodes), sources, [last] + unused[:1])
        nodes.append(node)
        unused = unused[1:]
        last = TI.NodeRef(node.id)
    name = f"rand{index:02d}_{kind}"
    programs = []
    if kind == "map":
        if unused:
            return []
        result, result_kind = last, "tensor"
    else:
        mapped = unused or rng.random() < 0.5
        if mapped:
            pick = [last] + unused[:1]
            src_node = body_node(rng, len(nodes), sources, pick)
            if unused[1:]:
                return []
            source = TI.MappedInput(src_node.inputs, src_node.scalar_params, src_node.body)
            values_nodes = nodes + [src_node]
            values_ref = TI.NodeRef(src_node.id)
        else:
            source = TI.PlainInput(last)
            values_nodes = list(nodes)
            values_ref = last
        red = TI.Reduce1D(len(nodes), source, kind)
        # companion: the per-element values the reduction folds
        params = scalar_params(values_nodes) + [TI.TensorParam(t) for t in tensors]
        programs.append(TI.Program(name + "_values", params, "tensor", values_ref,
                                   [TI.Elementwise1D(nd.id, nd.inputs, nd.scalar_params, nd.body)
                                    for nd in values_nodes]))
        nodes = nodes + [red]
        result, result_kind = TI.NodeRef(red.id), "scalar"
    params = scalar_params(nodes) + [TI.TensorParam(t) for t in tensors]
    programs.insert(0, TI.Program(name, params, result_kind, result, nodes))
    return programs


def scalar_params(nodes):
    seen = []
    for nd in nodes:
        sp = nd.scalar_params if isinstance(nd, TI.Elementwise1D) else getattr(
            nd.source, "scalar_params", ())
        for s in sp:
            if s not in seen:
                seen.append(s)
    return [TI.ScalarParam(s) for s in sorted(seen)]


def main():
    rng = random.Random(SEED)
    out = []
    index = 0
    while len([p for p in out if not p.entry_name.endswith("_values")]) < N_PROGRAMS:
        progs = program(rng, index)
        index += 1
        for p in progs:
            TI.validate(p)
            out.append(annotate(p))
    with open(os.path.join(HERE, "random_programs.tensor_ir.json"), "w") as fh:
        json.dump([TI.program_to_json(p) for p in out], fh, indent=1)
        fh.write("\n")
    with open(os.path.join(HERE, "loom-package.json"), "w") as fh:
        json.dump({"name": "random_programs"}, fh)
        fh.write("\n")
    print(len(out), "programs")


if __name__ == "__main__":
    main()
