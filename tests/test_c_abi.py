"""The generated header and library from plain C: a C11 program
(tests/c/abi_smoke.c) is compiled against `include/loom/b200_suite.h` and
linked twice -- against the shared suite library, and against a static
(`--kind static`) archive of the same package.  Building is checked on CPU;
running both binaries needs a GPU."""

import os
import shutil
import subprocess

import pytest

from loom_b200 import artifact
from loom_b200.build import SUITE_DIR, SUITE_PROJECT, SUITE_OPTIONS, build_suite

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "c", "abi_smoke.c")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, (cmd, proc.stdout, proc.stderr)
    return proc


@pytest.fixture(scope="module")
def binaries(tmp_path_factory):
    if shutil.which("gcc") is None or shutil.which("nvcc") is None:
        pytest.skip("needs gcc and nvcc")
    build_suite()
    out = tmp_path_factory.mktemp("c_abi")
    shared = str(out / "abi_smoke_shared")
    _run(["gcc", "-std=c11", "-O2", "-Wall", "-Werror", f"-I{os.path.join(ROOT, 'include')}",
          f"-I{CUDA}/include", SRC, "-o", shared, f"-L{SUITE_DIR}", "-lb200_suite",
          f"-Wl,-rpath,{SUITE_DIR}", f"-L{CUDA}/lib64", "-lcudart", "-lm"])
    opts = SUITE_OPTIONS()
    opts.kind = "static"
    res = artifact.generate_package(SUITE_PROJECT, str(out / "static_pkg"), opts)
    static = str(out / "abi_smoke_static")
    _run(["nvcc", "-O2", f"-I{os.path.join(str(out), 'static_pkg', 'include')}", SRC, "-o", static,
          res.artifact_path, "-lnccl", "-lm"])
    return shared, static


def test_c_programs_build(binaries):
    for path in binaries:
        assert os.path.exists(path)


@pytest.mark.gpu
def test_c_programs_run(binaries):
    for path in binaries:
        proc = subprocess.run([path], capture_output=True, text=True, timeout=120)
        assert proc.returncode == 0, (path, proc.returncode, proc.stderr)
        assert "abi_smoke ok" in proc.stdout
