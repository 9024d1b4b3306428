"""Regenerate tests/golden/pass_programs_front_ir.json: the FrontIR that the
reference's Python frontend (src/frontends/python/loom_frontend_python.py
front-ir-json) prints for every entry of pass_programs.py.  Nothing at test
time reads the reference.  Run in a checkout that has it:

    python tests/golden/sources/pass_programs/make_front_ir.py /path/to/reference
"""

import json
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(os.path.dirname(os.path.dirname(HERE)), "pass_programs_front_ir.json")


def main(ref: str) -> None:
    frontend = os.path.join(ref, "src", "frontends", "python", "loom_frontend_python.py")
    src = os.path.join(HERE, "pass_programs.py")
    with open(src, encoding="utf-8") as fh:
        entries = re.findall(r"^def (p\d+)\(", fh.read(), re.M)
    table = {}
    for entry in entries:
        proc = subprocess.run([sys.executable, frontend, "front-ir-json", src, "--entry", entry],
                              capture_output=True, text=True, check=True)
        table[entry] = json.loads(proc.stdout)
    with open(OUT, "w") as fh:
        json.dump(table, fh, indent=None, sort_keys=True)
        fh.write("\n")
    print(f"{len(table)} entries written to {OUT}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to a checkout of the reference>")
    main(sys.argv[1])
