"""Regenerate random_errors.py and ../../random_errors.json: seeded entries
that each hold one construct the Loom entry language rejects (Python parses
all of them), placed at a random depth inside an otherwise valid map, map2 or
reduction body, together with the message (line and column included) that
the reference's Python frontend (src/frontends/python/loom_frontend_python.py
front-ir-json) prints for each.  Nothing at test time reads the reference.
Run in a checkout that has it:

    python tests/golden/sources/errors/make_random_errors.py /path/to/reference
"""

import json
import os
import random
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_JSON = os.path.join(os.path.dirname(os.path.dirname(HERE)), "random_errors.json")
COUNT = 40
SEED = 20260417

# one rejected construct each; {v} and {w} are scalar operands in scope
BAD = ("({v} ** 2.0)", "(not ({v} > {w}))", "({v} < {w} < 1.0)", "({v}.real)", "abs({v})",
       "math.floor({v})", "max({v}, {w}, 1.0)", "max({v}, b={w})", "(1.0 if {v} else {w})",
       "'s'", "(True + {v})", "({v} // {w})", "({v} % 2.0)", "(-{v} if {v} > {w} else True)",
       "loom.Tensor1.reduce_sum({v})", "undefined_name", "({v} @ {w})", "[{v}]", "({v}, {w})",
       "lambda_missing({v})")


def expr(rng, names, depth, bad):
    """A valid expression over `names` with `bad` spliced in at one leaf."""
    if depth == 0:
        return bad
    op = rng.choice(("+", "-", "*"))
    other = rng.choice(names + ["1.5", "0.25"])
    inner = expr(rng, names, depth - 1, bad)
    form = rng.randrange(3)
    if form == 0:
        return f"({inner} {op} {other})"
    if form == 1:
        return f"({other} {op} {inner})"
    return f"max({inner}, {other})"


def entry(rng, name):
    kind = rng.choice(("map", "map2", "sum"))
    names = ["xi", "a"] + (["yi"] if kind != "map" else [])
    v, w = rng.sample(names, 2)
    bad = rng.choice(BAD).format(v=v, w=w)
    body = expr(rng, names, rng.randint(0, 3), bad)
    head = f"@loom.entry\ndef {name}(a: float, x: loom.Tensor1, y: loom.Tensor1)"
    if kind == "map":
        return f"{head} -> loom.Tensor1:\n    return loom.Tensor1.map(lambda xi: {body}, x)\n"
    if kind == "map2":
        return (f"{head} -> loom.Tensor1:\n"
                f"    return loom.Tensor1.map2(lambda xi, yi: {body}, x, y)\n")
    return (f"{head} -> float:\n    m = loom.Tensor1.map2(lambda xi, yi: {body}, x, y)\n"
            f"    return loom.Tensor1.reduce_sum(m)\n")


def main(ref: str) -> None:
    rng = random.Random(SEED)
    names = [f"e{i:03d}" for i in range(COUNT)]
    parts = ['"""Seeded entries that the Loom entry language rejects '
             '(make_random_errors.py)."""', "", "import math", "", "import loom", ""]
    for n in names:
        parts += ["", entry(rng, n)]
    src = os.path.join(HERE, "random_errors.py")
    with open(src, "w") as fh:
        fh.write("\n".join(parts))
    frontend = os.path.join(ref, "src", "frontends", "python", "loom_frontend_python.py")
    table = {}
    for n in names:
        proc = subprocess.run([sys.executable, frontend, "front-ir-json", src, "--entry", n],
                              capture_output=True, text=True)
        table[n] = {"returncode": proc.returncode,
                    "stderr": proc.stderr.strip().splitlines()[-1] if proc.stderr.strip() else ""}
    with open(OUT_JSON, "w") as fh:
        json.dump(table, fh, indent=1, sort_keys=True)
        fh.write("\n")
    rejected = sum(t["returncode"] != 0 for t in table.values())
    print(f"{len(table)} entries, {rejected} rejected by the reference frontend")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to a checkout of the reference>")
    main(sys.argv[1])
