"""The generated map bodies against the oracle on the CPU.

The CUDA source of a package holds one body functor per entry
(``struct LoomBody_<symbol>``: the element-wise chain, inlined, that the map
or reduction kernel applies to each element).  Its text comes from
loom_b200/render.py; the oracle renders its own C from the same emission
rules (oracle/loom_oracle.py), independently.  Here each body is compiled
for the host with g++ (``__device__`` defined away, no FMA contraction, as
nvcc builds the kernels with ``-fmad=false``) and run over seeded inputs:

* every map entry must give the oracle's bits (NaN only has to be NaN);
* the per-element values of every reduction must equal those of the
  oracle's map over the reduction's source, rendered with the default rules
  (a body fused into a reduction renders with them whatever the flags).

``+ - * /``, ``fmaf``, ``sqrtf``, ``fabsf`` and ``copysignf`` round the
same on the host as on the GPU; ``fminf`` and ``fmaxf`` take CUDA's NaN and
signed-zero ordering from oracle/oracle_semantics.h, which the GPU tests
check against the device.  ``expf``, ``logf`` and ``__fdividef`` are the
host's (exact division for the last) on both sides here, so for bodies that
call them this checks the rendered structure only; CUDA's versions differ
from the host's, and the GPU tests compare those bodies to a relative 1e-6.

So the CPU suite checks the renderer against the oracle over every test
project and flag set, without a GPU.
"""

import ctypes
import os
import re
import shutil
import subprocess

from pathlib import Path

import numpy as np
import pytest

from loom_b200 import artifact
from loom_b200 import tensor_ir as TI
from loom_b200.build import CUDA_FIXED_FLAGS, FUSION_FLAGS, RENDER_FLAGS

from test_workloads import values_program

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCES = os.path.join(HERE, "golden", "sources")
FLAGGED = tuple(FUSION_FLAGS) + tuple(RENDER_FLAGS)
BUILDS = [("cases", ()), ("cases", tuple(RENDER_FLAGS)), ("cases", tuple(FUSION_FLAGS)),
          ("cases", tuple(CUDA_FIXED_FLAGS)), ("workloads", ()), ("workloads", FLAGGED),
          ("workloads", tuple(CUDA_FIXED_FLAGS)), ("pass_programs", ()),
          ("pass_programs", tuple(CUDA_FIXED_FLAGS)), ("random", ()), ("ir", ())]
# CUDA's fminf/fmaxf (NaN and signed-zero ordering) as the oracle restates
# them; glibc's may return either zero for fmaxf(-0.0f, +0.0f)
PRELUDE = """#include "oracle_semantics.h"
#define __device__
#define __forceinline__ inline
"""
ORACLE_DIR = os.path.join(os.path.dirname(HERE), "oracle")

pytestmark = pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")


def _host_library(tmp, name, bodies):
    """One extern "C" runner per body: fills the scalar fields, then
    out[i] = body(inputs at i) for i in [0, n)."""
    lines = [PRELUDE]
    for sym, (text, fields, k) in bodies.items():
        lines.append(text)
        sets = "".join(f"  b.v_{f} = scalars[{j}];\n" for j, f in enumerate(fields))
        lines.append(
            f'extern "C" void run_{sym}(const float* const* ins, const float* scalars, '
            f"int64_t n, float* out) {{\n  LoomBody_{sym} b;\n{sets}"
            f"  for (int64_t i = 0; i < n; ++i) {{\n    float in[{max(k, 1)}];\n"
            f"    for (int j = 0; j < {k}; ++j) in[j] = ins[j][i];\n"
            f"    out[i] = b(in);\n  }}\n}}\n")
    src = tmp / f"{name}.cpp"
    src.write_text("\n".join(lines))
    lib = tmp / f"lib{name}.so"
    subprocess.run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared",
                    "-fPIC", f"-I{ORACLE_DIR}", "-o", str(lib), str(src)], check=True,
                   capture_output=True)
    return ctypes.CDLL(str(lib))


def _run(lib, sym, arrays, scalars, n):
    fn = getattr(lib, "run_" + sym)
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    ptrs = (ctypes.c_void_p * max(1, len(arrays)))(*[a.ctypes.data for a in arrays])
    sc = (ctypes.c_float * max(1, len(scalars)))(*scalars)
    out = np.empty(n, np.float32)
    fn(ptrs, sc, n, out.ctypes.data)
    return out


def _same_bits(got, ref):
    nan = np.isnan(ref)
    return (np.array_equal(np.isnan(got), nan)
            and np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32)))


@pytest.mark.parametrize("project, flags", BUILDS,
                         ids=[f"{p}-{len(f)}flags" for p, f in BUILDS])
def test_generated_bodies_match_the_oracle_on_the_host(tmp_path, project, flags):
    check_project(tmp_path, os.path.join(SOURCES, project), flags, project)


def test_structured_random_entries_on_the_host(tmp_path):
    # tests/golden/sources/front_programs without the two entries that the
    # reference's normalize rejects (tests/test_front_programs.py)
    src = open(os.path.join(SOURCES, "front_programs", "front_programs.py")).read()
    for entry in ("f000", "f020"):
        start = src.index(f"@loom.entry\ndef {entry}(")
        end = src.find("@loom.entry", start + 1)
        src = src[:start] + (src[end:] if end >= 0 else "")
    root = tmp_path / "front_programs"
    root.mkdir()
    (root / "front_programs.py").write_text(src)
    for flags in ((), tuple(CUDA_FIXED_FLAGS)):
        check_project(tmp_path / f"f{len(flags)}", str(root), flags, "front_programs")


def check_project(tmp_path, root, flags, project):
    """Package `root` with `flags` (sources only), compile its body functors
    for the host and compare every map's bits, and every reduction's
    per-element values, with the oracle's."""
    from oracle.loom_oracle import Oracle
    os.makedirs(tmp_path, exist_ok=True)
    opts = artifact.Options(enabled=list(flags), multi_gpu=False)
    res = artifact.generate_package(root, str(tmp_path / "pkg"), opts, build=False)
    src = open(res.source_path).read()
    structs = {m.group(1): m.group(0) for m in
               re.finditer(r"struct LoomBody_(\w+) \{.*?\n\};", src, re.S)}
    bundles = artifact.discover_entries(root, enabled=flags)
    maps, reductions, bodies = [], [], {}
    for b in bundles:
        sym = b.plan.symbol
        text = structs[sym]
        fields = re.findall(r"^\s*float v_(\w+);", text, re.M)
        k = int(re.search(r"kInputs = (\d+);", text).group(1))
        bodies[sym] = (text, fields, k)
        (maps if b.program.result_kind == "tensor" else reductions).append(b)
    assert maps or reductions
    lib = _host_library(Path(tmp_path), "bodies", bodies)
    # a reduction's body renders with the default rules whatever the flags
    # (the rendering flags select map kernels), so its values are checked
    # against an oracle map built without them
    oracle = Oracle([TI.program_to_json(b.program) for b in maps] or
                    [TI.program_to_json(values_program(reductions[0].program))],
                    name=f"host_{project}_{len(flags)}", enabled=flags)
    values = Oracle([TI.program_to_json(values_program(b.program)) for b in reductions] or
                    [TI.program_to_json(maps[0].program)],
                    name=f"host_{project}_{len(flags)}_values")
    rng = np.random.default_rng(len(bundles) + len(flags))
    n = 4099
    checked = 0
    for b in maps + reductions:
        prog = b.program
        inp = {p.name: (rng.standard_normal(n).astype(np.float32) * 2.0)
               for p in prog.tensor_params}
        for arr in inp.values():
            arr[:8] = [0.0, -0.0, 1.0, -1.0, 0.5, -2.0, 3.0, 0.25]
        inp.update({p.name: float(rng.uniform(-1.5, 1.5)) for p in prog.scalar_params})
        sym = b.plan.symbol
        text, fields, k = bodies[sym]
        slots = b.plan.slots
        assert len(slots) == k, sym
        arrays = [inp[s] for s in slots]
        scalars = [inp[f] for f in fields]
        got = _run(lib, sym, arrays, scalars, n)
        if prog.result_kind == "tensor":
            ref = np.asarray(oracle.run(prog.entry_name, inp), dtype=np.float32)
        else:
            ref = np.asarray(values.run(prog.entry_name + "__values", inp), dtype=np.float32)
        assert _same_bits(got, ref), (project, flags, prog.entry_name)
        checked += 1
    assert checked == len(maps) + len(reductions)
