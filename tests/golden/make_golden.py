"""Regenerate the golden fixtures under tests/golden/ from the reference.

Run in a checkout that has the reference mounted (it is read-only data here;
nothing at test time reads it):

    python tests/golden/make_golden.py /path/to/reference

* ``reference_ir/``: the reference's own golden IR files
  (``test/golden/saxpy_loom_lambda.json``, ``test/golden/l2_norm_sq_tensor_ir.json``),
  copied verbatim;
* ``front_ir/<module>.<entry>.json``: FrontIR that the reference's Python
  frontend (``src/frontends/python/loom_frontend_python.py front-ir-json``)
  prints for the suite entries, for ``sources/cases/frontend_cases.py`` and for the
  reference's Python examples and package fixture;
* ``front_ir_errors.json``: the reference frontend's error message for each
  entry of ``sources/errors/frontend_errors.py``;
* ``list_entries.json``: its entry listing (``list-entries-json``) for the
  suite, the cases and the random pass programs.
"""

import json
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def main(ref: str) -> None:
    out_ir = os.path.join(HERE, "reference_ir")
    os.makedirs(out_ir, exist_ok=True)
    for name in ("saxpy_loom_lambda.json", "l2_norm_sq_tensor_ir.json"):
        shutil.copyfile(os.path.join(ref, "test", "golden", name), os.path.join(out_ir, name))
    frontend = os.path.join(ref, "src", "frontends", "python", "loom_frontend_python.py")
    sources = {
        os.path.join(ROOT, "loom_b200", "suite", "kernels.py"):
            ["saxpy", "relu", "dot", "l2_norm_sq", "max_value", "affine_relu", "pipeline_sum"],
        os.path.join(HERE, "sources", "cases", "frontend_cases.py"):
            ["nested_helpers", "clamp_scale", "tuple_lets", "soft_threshold", "hypot_sum",
             "neg_max", "ratio_exp", "select_floor", "scaled_chain", "tail_if",
             "qualified_prims", "unary_and_eq", "let_chain_sum", "max_of_difference"],
        os.path.join(ref, "examples", "saxpy.py"): ["saxpy"],
        os.path.join(ref, "examples", "relu.py"): ["relu"],
        os.path.join(ref, "examples", "dot.py"): ["dot"],
        os.path.join(ref, "examples", "l2_norm_sq.py"): ["l2_norm_sq"],
        os.path.join(ref, "experiments", "source", "python", "dot_pipeline.py"): ["dot_pipeline"],
        os.path.join(ref, "test", "fixtures", "python_package_project", "kernels.py"):
            ["saxpy", "relu", "dot"],
    }
    out_front = os.path.join(HERE, "front_ir")
    os.makedirs(out_front, exist_ok=True)
    for path, entries in sources.items():
        tag = os.path.basename(os.path.dirname(path)) + "_" + os.path.splitext(
            os.path.basename(path))[0]
        for entry in entries:
            proc = subprocess.run([sys.executable, frontend, "front-ir-json", path, "--entry", entry],
                                  capture_output=True, text=True, check=True)
            obj = json.loads(proc.stdout)
            with open(os.path.join(out_front, f"{tag}.{entry}.json"), "w") as fh:
                json.dump(obj, fh, indent=1, sort_keys=True)
                fh.write("\n")
    errors = {}
    bad = os.path.join(HERE, "sources", "errors", "frontend_errors.py")
    for entry in ("with_loop", "tensor_capture", "chained", "keyword_call", "wrong_return",
                  "unknown_call", "tensor_branch", "power_op", "aug_assign", "non_tail_if",
                  "bool_not", "attribute_access"):
        proc = subprocess.run([sys.executable, frontend, "front-ir-json", bad, "--entry", entry],
                              capture_output=True, text=True)
        errors[entry] = {"returncode": proc.returncode,
                         "stderr": proc.stderr.strip().splitlines()[-1] if proc.stderr.strip()
                         else ""}
    with open(os.path.join(HERE, "front_ir_errors.json"), "w") as fh:
        json.dump(errors, fh, indent=1, sort_keys=True)
        fh.write("\n")
    # the frontend's entry listing (list-entries-json) for the Python sources
    listings = {}
    for rel in (os.path.join("loom_b200", "suite", "kernels.py"),
                os.path.join("tests", "golden", "sources", "cases", "frontend_cases.py"),
                os.path.join("tests", "golden", "sources", "pass_programs", "pass_programs.py")):
        proc = subprocess.run([sys.executable, frontend, "list-entries-json",
                               os.path.join(ROOT, rel)], capture_output=True, text=True,
                              check=True)
        listings[rel.replace(os.sep, "/")] = json.loads(proc.stdout)
    with open(os.path.join(HERE, "list_entries.json"), "w") as fh:
        json.dump(listings, fh, indent=1, sort_keys=True)
        fh.write("\n")
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to a checkout of the reference>")
    main(sys.argv[1])
