"""Regenerate front_programs.py and ../../front_programs_front_ir.json: seeded
random Loom entries built from the entry language's structured forms --
local helper functions (one or two parameters, some ending in an
if/else statement, some calling another helper), helpers passed to maps directly,
tuple and annotated lets, qualified primitives (math.sqrt, loom.max, ...),
select, unary plus, equality tests and tensor-level helpers -- with the
FrontIR the reference's Python frontend
(src/frontends/python/loom_frontend_python.py front-ir-json) prints for
each.  Square roots and logs take d*d + 1 and exponents min(d, 3), so a
float64 evaluation stays finite.  Nothing at test time reads the reference.
Run in a checkout that has it:

    python tests/golden/sources/front_programs/make_front_programs.py /path/to/reference
"""

import json
import os
import random
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_JSON = os.path.join(os.path.dirname(os.path.dirname(HERE)), "front_programs_front_ir.json")
COUNT = 30
SEED = 104729
LITS = ("0.5", "1.0", "2.0", "-0.25", "3.0", "0.0")


class Gen:
    def __init__(self, rng):
        self.r = rng

    def expr(self, names, depth, helpers=()):
        r = self.r
        if depth == 0 or r.random() < 0.2:
            return r.choice(names) if r.random() < 0.8 else r.choice(LITS)
        sub = lambda: self.expr(names, depth - 1, helpers)
        kind = r.choices(("arith", "call", "prim", "select", "ifexp", "plus", "eq"),
                         weights=(6, 3 if helpers else 0, 3, 1, 2, 1, 1))[0]
        if kind == "arith":
            return f"({sub()} {r.choice('+-*')} {sub()})"
        if kind == "call":
            h, arity = r.choice(helpers)
            return f"{h}({', '.join(sub() for _ in range(arity))})"
        if kind == "prim":
            d = sub()
            return r.choice((f"math.sqrt({d} * {d} + 1.0)", f"loom.max({d}, {sub()})",
                             f"min({d}, {sub()})", f"log({d} * {d} + 1.0)",
                             f"exp(min({d}, 3.0))", f"loom.sqrt({d} * {d} + 1.0)"))
        if kind == "select":
            return f"select({sub()} > {sub()}, {sub()}, {sub()})"
        if kind == "ifexp":
            return f"({sub()} if {sub()} {r.choice(('<', '<=', '>', '>='))} {sub()} else {sub()})"
        if kind == "plus":
            return f"(+{sub()})"
        return f"({sub()} if {sub()} == {sub()} else {sub()})"

    def helper(self, name, scalars, helpers):
        r = self.r
        arity = r.choice((1, 1, 2))
        params = ["u", "v"][:arity]
        sig = ", ".join(f"{p}: float" for p in params)
        lines = [f"    def {name}({sig}) -> float:"]
        if r.random() < 0.35:
            c = self.expr(params + scalars, 1)
            lines += [f"        if {params[0]} > {c}:",
                      f"            return {self.expr(params + scalars, 2, helpers)}",
                      "        else:",
                      f"            return {self.expr(params + scalars, 2, helpers)}"]
        else:
            lines += [f"        return {self.expr(params + scalars, 2, helpers)}"]
        return lines, (name, arity)

    def entry(self, name):
        r = self.r
        lines = []
        scalars = ["a"]
        if r.random() < 0.5:
            lines.append(f"    p, q = {self.expr(['a'], 1)}, {self.expr(['a'], 1)}")
            scalars += ["p", "q"]
        if r.random() < 0.4:
            lines.append(f"    s: float = {self.expr(scalars, 2)}")
            scalars.append("s")
        helpers = []
        for i in range(r.randint(1, 3)):
            body, h = self.helper(f"h{i}", scalars, tuple(helpers))
            lines += body
            helpers.append(h)
        one = [h for h in helpers if h[1] == 1]
        two = [h for h in helpers if h[1] == 2]
        if one and r.random() < 0.4:
            m0 = f"loom.Tensor1.map({r.choice(one)[0]}, x)"
        elif two and r.random() < 0.4:
            m0 = f"loom.Tensor1.map2({r.choice(two)[0]}, x, y)"
        else:
            m0 = (f"loom.Tensor1.map2(lambda xi, yi: "
                  f"{self.expr(['xi', 'yi'] + scalars, 3, tuple(helpers))}, x, y)")
        lines.append(f"    m = {m0}")
        kind = r.choices(("tensor", "sum", "max", "total"), weights=(3, 3, 2, 2))[0]
        if kind == "tensor":
            ret, rty = "m", "loom.Tensor1"
        elif kind == "max":
            ret, rty = "loom.Tensor1.reduce_max(m)", "float"
        elif kind == "sum":
            ret, rty = "loom.Tensor1.reduce_sum(m)", "float"
        else:
            lines += ["    def total(t: loom.Tensor1) -> float:",
                      "        return loom.Tensor1.reduce_sum(t)"]
            ret, rty = "total(loom.Tensor1.map(lambda v: v * v, m))", "float"
        head = f"@loom.entry\ndef {name}(a: float, x: loom.Tensor1, y: loom.Tensor1) -> {rty}:"
        return "\n".join([head] + lines + [f"    return {ret}"])


def main(ref: str) -> None:
    gen = Gen(random.Random(SEED))
    names = [f"f{i:03d}" for i in range(COUNT)]
    parts = ['"""Seeded random entries over the structured forms of the entry language '
             '(make_front_programs.py)."""', "", "import math", "", "import loom", ""]
    for n in names:
        parts += ["", gen.entry(n), ""]
    src = os.path.join(HERE, "front_programs.py")
    with open(src, "w") as fh:
        fh.write("\n".join(parts))
    with open(os.path.join(HERE, "loom-package.json"), "w") as fh:
        fh.write('{"name": "front_programs"}\n')
    frontend = os.path.join(ref, "src", "frontends", "python", "loom_frontend_python.py")
    table = {}
    for n in names:
        proc = subprocess.run([sys.executable, frontend, "front-ir-json", src, "--entry", n],
                              capture_output=True, text=True, check=True)
        table[n] = json.loads(proc.stdout)
    with open(OUT_JSON, "w") as fh:
        json.dump(table, fh, sort_keys=True)
        fh.write("\n")
    print(f"{len(table)} entries written")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to a checkout of the reference>")
    main(sys.argv[1])
