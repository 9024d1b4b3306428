"""Regenerate pass_programs.py: seeded random Loom entries (Python entry
language) shaped to exercise the reference's scalar and TensorIR passes --
constant lets and constant subexpressions (const-fold), branches with equal
arms (if-simplify), sums and products in arbitrary order (arith-reassociate,
tensor-canonicalize), compare-and-pick branches (select -> min/max),
weighted products and repeated differences in reductions (the
reduction-body rewrites), unused maps (dce) and map chains (fusion).

Bodies use + - * / min max, negation, comparisons and conditionals only, with
every denominator of the form d*d + 1, so that a float64 evaluation is finite
and the CUDA kernels' bits are fully determined by the emission rules.

    python tests/golden/sources/pass_programs/make_pass_programs.py
"""

import os
import random

HERE = os.path.dirname(os.path.abspath(__file__))
COUNT = 40
SEED = 20260417
LITERALS = ("0.0", "1.0", "2.0", "0.5", "-0.5", "0.25", "1.5", "3.0", "-2.0")
COMPARE = ("<", "<=", ">", ">=")


class Gen:
    def __init__(self, rng):
        self.rng = rng

    def const(self, consts, depth=2):
        r = self.rng
        if depth == 0 or r.random() < 0.35:
            return r.choice(LITERALS + tuple(consts)) if consts else r.choice(LITERALS)
        op = r.choice(("+", "-", "*"))
        return f"({self.const(consts, depth - 1)} {op} {self.const(consts, depth - 1)})"

    def leaf(self, names):
        r = self.rng
        return r.choice(names) if r.random() < 0.75 else r.choice(LITERALS)

    def expr(self, names, depth):
        r = self.rng
        if depth == 0 or r.random() < 0.2:
            return self.leaf(names)
        kind = r.choices(("arith", "div", "minmax", "neg", "pick", "branch", "same", "weighted",
                          "square"), weights=(6, 1, 2, 1, 2, 2, 1, 2, 1))[0]
        sub = lambda: self.expr(names, depth - 1)
        if kind == "arith":
            return f"({sub()} {r.choice('+-*')} {sub()})"
        if kind == "div":
            d = sub()
            return f"({sub()} / ({d} * {d} + 1.0))"
        if kind == "minmax":
            return f"{r.choice(('min', 'max'))}({sub()}, {sub()})"
        if kind == "neg":
            return f"(-{sub()})"
        if kind == "pick":           # compare-and-pick: becomes min or max
            p, q = self.leaf(names), self.leaf(names)
            op = r.choice(COMPARE[0:1] + COMPARE[2:3])
            return f"({p} if {p} {op} {q} else {q})" if r.random() < 0.5 \
                else f"({q} if {p} {op} {q} else {p})"
        if kind == "branch":
            return f"({sub()} if {sub()} {r.choice(COMPARE)} {sub()} else {sub()})"
        if kind == "same":           # equal arms
            e = sub()
            return f"({e} if {sub()} > {sub()} else {e})"
        if kind == "weighted":
            return f"({self.leaf(names)} * ({sub()} * {sub()}))"
        d = f"({sub()} - {sub()})"
        return f"({d} * {d})" if r.random() < 0.5 else f"({d} + {d})"

    def entry(self, name):
        r = self.rng
        lines = []
        consts = []
        for i in range(r.randint(0, 2)):
            c = f"c{i}"
            lines.append(f"    {c} = {self.const(consts)}")
            consts.append(c)
        scalars = ["a", "b"] + consts
        if r.random() < 0.5:
            lines.append(f"    s0 = {self.expr(['a', 'b'] + consts, 2)}")
            scalars.append("s0")
        if r.random() < 0.3:
            lines.append("    unused = loom.Tensor1.map(lambda xi: xi * a, x)")
        depth = r.randint(2, 4)
        body = self.expr(["xi", "yi"] + scalars, depth)
        lines.append(f"    m0 = loom.Tensor1.map2(lambda xi, yi: {body}, x, y)")
        last = "m0"
        if r.random() < 0.6:
            lines.append(f"    m1 = loom.Tensor1.map(lambda v: {self.expr(['v'] + scalars, 2)}, m0)")
            last = "m1"
        kind = r.choices(("tensor", "sum", "max"), weights=(4, 4, 2))[0]
        if kind == "tensor":
            ret, rty = last, "loom.Tensor1"
        elif kind == "max":
            ret, rty = f"loom.Tensor1.reduce_max({last})", "float"
        else:
            red = self.expr(["p", "q"] + scalars, 2)
            ret = f"loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda p, q: {red}, {last}, w))"
            rty = "float"
        head = (f"@loom.entry\ndef {name}(a: float, b: float, x: loom.Tensor1, y: loom.Tensor1, "
                f"w: loom.Tensor1) -> {rty}:")
        return "\n".join([head] + lines + [f"    return {ret}"])


def main():
    gen = Gen(random.Random(SEED))
    parts = ['"""Seeded random entries for the scalar and TensorIR pass tests '
             '(make_pass_programs.py)."""', "", "import loom", ""]
    for i in range(COUNT):
        parts += ["", gen.entry(f"p{i:03d}"), ""]
    with open(os.path.join(HERE, "pass_programs.py"), "w") as fh:
        fh.write("\n".join(parts))
    with open(os.path.join(HERE, "loom-package.json"), "w") as fh:
        fh.write('{"name": "pass_programs"}\n')


if __name__ == "__main__":
    main()
