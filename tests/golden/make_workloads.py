"""Regenerate tests/golden/sources/workloads/ from the reference.

The reference's benchmark harness runs 33 supported kernels
(``experiments/source/data/common/workloads.json``), each a Python entry
under ``experiments/source/python/``.  For each one this script records:

* ``<name>.front_ir.json``: the FrontIR that the reference's own Python
  frontend (``src/frontends/python/loom_frontend_python.py front-ir-json``)
  prints for it -- the input of the B200 project built from this folder;
* in ``workloads.json``: the entry name, the harness's scalar arguments and
  tensor inputs, the result kind, and whether this repository's front end
  printed the same FrontIR from the same source when the fixture was made;
* ``../workload_limitations.json`` and ``../sources/workload_limitations/``:
  the harness's unsupported capability cases -- the reference frontend's
  error, or (where only loomc's later lowering rejects a case) its FrontIR,
  next to this front end's verdict.

Nothing at test time reads the reference.  Run in a checkout that has it:

    python tests/golden/make_workloads.py /path/to/reference
"""

import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "sources", "workloads")


def main(ref: str) -> None:
    sys.path.insert(0, ROOT)
    from loom_b200.frontend import front_ir

    frontend = os.path.join(ref, "src", "frontends", "python", "loom_frontend_python.py")
    spec = json.load(open(os.path.join(ref, "experiments", "source", "data", "common",
                                       "workloads.json")))
    os.makedirs(OUT, exist_ok=True)
    table = []
    for w in spec["supported_kernels"]:
        src = os.path.join(ref, "experiments", "source", "python", w["name"] + ".py")
        proc = subprocess.run([sys.executable, frontend, "front-ir-json", src, "--entry",
                               w["entry"]], capture_output=True, text=True, check=True)
        theirs = json.loads(proc.stdout)
        with open(src, encoding="utf-8") as fh:
            ours = front_ir(fh.read(), w["entry"])
        with open(os.path.join(OUT, w["name"] + ".front_ir.json"), "w") as fh:
            json.dump(theirs, fh, indent=1, sort_keys=True)
            fh.write("\n")
        table.append({"name": w["name"], "entry": w["entry"],
                      "scalar_args": w["scalar_args"], "tensor_inputs": w["tensor_inputs"],
                      "result_kind": w["result_kind"],
                      "front_ir_matches_this_front_end": ours == theirs})
    with open(os.path.join(OUT, "workloads.json"), "w") as fh:
        json.dump(table, fh, indent=1)
        fh.write("\n")
    with open(os.path.join(OUT, "loom-package.json"), "w") as fh:
        json.dump({"name": "workloads"}, fh)
        fh.write("\n")
    same = sum(t["front_ir_matches_this_front_end"] for t in table)
    print(f"{len(table)} workloads written to {OUT}; this front end matched {same}")

    # The harness's capability cases that the reference does not support
    # (experiments/source/python/limitations/*.py, entry "bad"): the
    # reference frontend's verdict, and this front end's, for each.
    from loom_b200.frontend import FrontendError, program_from_front_ir
    lim_dir = os.path.join(HERE, "sources", "workload_limitations")
    os.makedirs(lim_dir, exist_ok=True)
    limitations = {}
    src_dir = os.path.join(ref, "experiments", "source", "python", "limitations")
    for name in sorted(os.listdir(src_dir)):
        if not name.endswith(".py"):
            continue
        path = os.path.join(src_dir, name)
        proc = subprocess.run([sys.executable, frontend, "front-ir-json", path, "--entry", "bad"],
                              capture_output=True, text=True)
        with open(path, encoding="utf-8") as fh:
            text = fh.read()
        try:
            ours_front = front_ir(text, "bad", path)
            ours_error = None
        except FrontendError as exc:
            ours_front, ours_error = None, "Python frontend error: " + str(exc)
        rec = {"reference_frontend_returncode": proc.returncode}
        if proc.returncode == 0:
            # accepted by the frontend, rejected later by loomc's lowering
            theirs = json.loads(proc.stdout)
            stem = os.path.splitext(name)[0]
            with open(os.path.join(lim_dir, stem + ".front_ir.json"), "w") as fh:
                json.dump(theirs, fh, indent=1, sort_keys=True)
                fh.write("\n")
            rec["front_ir_matches_this_front_end"] = ours_front == theirs
            try:
                program_from_front_ir(theirs)
                rec["this_lowering_rejects"] = False
            except FrontendError:
                rec["this_lowering_rejects"] = True
        else:
            rec["reference_error"] = proc.stderr.strip().splitlines()[-1]
            rec["this_front_end_error"] = ours_error
        limitations[os.path.splitext(name)[0]] = rec
    with open(os.path.join(HERE, "workload_limitations.json"), "w") as fh:
        json.dump(limitations, fh, indent=1, sort_keys=True)
        fh.write("\n")
    print(f"{len(limitations)} limitation cases recorded")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to a checkout of the reference>")
    main(sys.argv[1])
