"""Regenerate tests/golden/harness_outputs.npz and harness_outputs.json: the
reference's own numeric oracle evaluated on this repository's seeded inputs.

The reference has no CPU evaluation of its generated kernels.  Its one
numeric oracle is ``reference_output`` in its benchmark harness
(``experiments/source/harness/run.py:1031-1099``): a plain PyTorch
expression per kernel, which the harness compares with every generated
kernel's output under ``torch.testing.assert_close`` at the kernel's
``verification_rtol`` / ``verification_atol`` (defaults 1e-4 / 1e-5,
``run.py:1016-1017`` and ``:1109-1111``).  This script imports that function
from a checkout of the reference (it does not copy it), runs it with torch on
the CPU, and stores its results:

* for the 33 kernels of the harness's table
  (``experiments/source/data/common/workloads.json``, looked up by
  ``baseline_name`` as ``run.py:1569`` does), on the inputs of
  ``loom_b200.workloads.harness_inputs`` (the harness's seeds and N(0, 1)
  distribution, drawn on the host);
* for the suite entries the function covers (saxpy, relu, dot, l2_norm_sq),
  on the inputs of ``loom_b200.workloads.entry_inputs`` (this backend's
  configurations: uniform, normal, normal with 1% outliers);

at n = 4096 (the reference's package tests use 4096), 65541 and 2^20 + 3.
Scalar results are stored whole; tensor results whole at 4096 and at a fixed
seeded sample of 1024 indices, plus the first and last 16, at the larger
sizes.  The tests compare this repository's oracle (CPU) and CUDA path (GPU)
against these values at the harness's own tolerances.

The harness module imports matplotlib for its plots; where it is absent a
stub stands in for it inside this script only.  Nothing at test time reads
the reference.  Run in a checkout that has it:

    python tests/golden/make_harness_outputs.py /path/to/reference
"""

import importlib.util
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT_NPZ = os.path.join(HERE, "harness_outputs.npz")
OUT_JSON = os.path.join(HERE, "harness_outputs.json")

SIZES = [4096, 65541, (1 << 20) + 3]
FULL_UP_TO = 4096
SAMPLE = 1024
EDGE = 16
SAMPLE_SEED = 7919
SUITE_ENTRIES = ["saxpy", "relu", "dot", "l2_norm_sq"]


def sample_indices(n: int) -> np.ndarray:
    """Indices of a tensor result stored in the fixture (all of them up to
    FULL_UP_TO elements)."""
    if n <= FULL_UP_TO:
        return np.arange(n, dtype=np.int64)
    rng = np.random.default_rng(SAMPLE_SEED + n)
    mid = rng.choice(np.arange(EDGE, n - EDGE), size=SAMPLE, replace=False)
    return np.unique(np.concatenate([np.arange(EDGE), mid, np.arange(n - EDGE, n)])).astype(np.int64)


def _stub_matplotlib() -> None:
    try:
        import matplotlib  # noqa: F401
        return
    except ImportError:
        pass
    mpl = types.ModuleType("matplotlib")
    mpl.use = lambda *a, **k: None
    pyplot = types.ModuleType("matplotlib.pyplot")
    colors = types.ModuleType("matplotlib.colors")
    colors.TwoSlopeNorm = object
    mpl.pyplot, mpl.colors = pyplot, colors
    sys.modules.update({"matplotlib": mpl, "matplotlib.pyplot": pyplot,
                        "matplotlib.colors": colors})


def load_harness(ref: str):
    _stub_matplotlib()
    path = os.path.join(ref, "experiments", "source", "harness", "run.py")
    spec = importlib.util.spec_from_file_location("loom_reference_harness", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod      # its dataclasses look their module up
    spec.loader.exec_module(mod)
    return mod


def main(ref: str) -> None:
    sys.path.insert(0, ROOT)
    import torch

    from loom_b200 import workloads

    harness = load_harness(ref)
    table = json.load(open(os.path.join(ref, "experiments", "source", "data", "common",
                                        "workloads.json")))["supported_kernels"]
    cases = []      # (case name, reference kernel name, inputs-maker, tolerances, entry)
    for k in table:
        rtol, atol = harness.verification_tolerances(k)
        cases.append(("harness/" + k["name"], harness.logical_kernel_name(k), k["entry"],
                      ("harness", k["tensor_inputs"], k["scalar_args"]), rtol, atol,
                      k["result_kind"]))
    for e in SUITE_ENTRIES:
        rtol, atol = harness.verification_tolerances({})
        kind = "tensor" if e in ("saxpy", "relu") else "scalar"
        cases.append(("suite/" + e, e, e, ("suite", e), rtol, atol, kind))

    arrays = {}
    meta = {"reference_function": "experiments/source/harness/run.py:1031-1099 reference_output",
            "tolerances_from": "experiments/source/harness/run.py:1016-1017 verification_tolerances",
            "torch": torch.__version__, "sizes": SIZES, "cases": []}
    for n in SIZES:
        arrays[f"indices/{n}"] = sample_indices(n)
    for name, ref_kernel, entry, spec, rtol, atol, kind in cases:
        for n in SIZES:
            if spec[0] == "harness":
                inp = workloads.harness_inputs(spec[1], spec[2], n)
            else:
                inp = workloads.entry_inputs(spec[1], n)
            tin = {key: (torch.from_numpy(v) if isinstance(v, np.ndarray) else v)
                   for key, v in inp.items()}
            with torch.no_grad():
                out = harness.reference_output(ref_kernel, tin).numpy().astype(np.float32)
            if kind == "tensor":
                assert out.shape == (n,), (name, out.shape)
                out = out[arrays[f"indices/{n}"]]
            else:
                assert out.shape == (1,), (name, out.shape)
            arrays[f"{name}/{n}"] = out
        meta["cases"].append({"case": name, "reference_kernel": ref_kernel, "entry": entry,
                              "result_kind": kind, "rtol": rtol, "atol": atol})
    np.savez_compressed(OUT_NPZ, **arrays)
    with open(OUT_JSON, "w") as fh:
        json.dump(meta, fh, indent=1)
        fh.write("\n")
    print(f"wrote {len(meta['cases'])} cases x {len(SIZES)} sizes to {OUT_NPZ}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to a checkout of the reference>")
    main(sys.argv[1])
