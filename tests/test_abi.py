"""The drop-in C ABI, checked without a GPU: header text, exported symbols,
manifest contract and the host-side argument checks (which return before any
CUDA call, so they run on a CPU-only machine)."""

import ctypes
import json
import os
import re

import pytest

from loom_b200 import build as B
from loom_b200 import codegen
from loom_b200.artifact import discover_entries

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "loom", "b200_suite.h")


@pytest.fixture(scope="module")
def built():
    B.build_suite()
    return B.SUITE_DIR


@pytest.fixture(scope="module")
def lib(built):
    return ctypes.CDLL(os.path.join(built, "libb200_suite.so"))


def declared_symbols(path):
    with open(path) as fh:
        text = fh.read()
    return re.findall(r"^\s*(?:size_t|int)\s+(\w+)\(", text, flags=re.M)


def test_committed_header_is_the_generated_one(built):
    plans = [b.plan for b in discover_entries(B.SUITE_PROJECT)]
    assert open(HEADER).read() == codegen.render_header("b200_suite", plans, True,
                                                        B.SUITE_OPTIONS().noalloc_entries)
    assert open(os.path.join(built, "include", "loom", "b200_suite.h")).read() == \
        open(HEADER).read()


def test_library_exports_every_declared_symbol(lib):
    syms = declared_symbols(HEADER)
    assert len(syms) >= 7 * 6
    for s in syms:
        assert hasattr(lib, s), s


def test_reference_prototypes():
    text = open(HEADER).read()
    # the reference fixture's saxpy/relu/dot shapes (test/python/test_package.py:89-131)
    assert ("int loom_kernels_saxpy(float a, const float* x, const float* y, int64_t n, "
            "float* out, void* workspace, size_t workspace_size);") in text
    assert "int loom_kernels_saxpy_noworkspace(float a, const float* x, const float* y, " \
           "int64_t n, float* out);" in text
    assert ("int loom_kernels_dot(const float* x, const float* y, int64_t n, float* out, "
            "void* workspace, size_t workspace_size);") in text
    assert "loom_kernels_dot_noworkspace" not in text
    for code, value in (("OK", 0), ("INVALID_ARGUMENT", 1), ("WORKSPACE_TOO_SMALL", 2),
                        ("CUDA_ERROR", 3)):
        assert f"#define LOOM_STATUS_{code} {value}" in text


def test_manifest_contract(built):
    # fields the reference's tests and harness read (test_package.py:43-63, run.py:1797-1836)
    m = json.load(open(os.path.join(built, "manifest.json")))
    assert m["target_backend"] == "cuda" and m["artifact_kind"] == "shared"
    assert m["cuda_arch"] == "sm_100a"
    assert sorted(e["entry_name"] for e in m["entries"]) == sorted(
        ["saxpy", "relu", "dot", "l2_norm_sq", "max_value", "affine_relu", "pipeline_sum"])
    for e in m["entries"]:
        assert e["symbol_name"] == "loom_kernels_" + e["entry_name"]
        assert e["workspace_symbol"] == e["symbol_name"] + "_workspace_size"
        assert ("no_workspace_symbol" in e) == (e["result_kind"] == "tensor")
        for f in ("tensor_ir.json", "kernel_plan.json", "cuda_plan.json", "backend_analysis.json"):
            assert os.path.exists(os.path.join(built, "entries", e["symbol_name"], f))
    assert "enabled" in m["optimizations"]
    assert os.path.exists(m["header_path"]) and os.path.exists(m["source_path"])


def _ws(lib, sym):
    f = getattr(lib, sym)
    f.argtypes = [ctypes.c_int64]
    f.restype = ctypes.c_size_t
    return f


def test_workspace_sizes(lib):
    assert _ws(lib, "loom_kernels_saxpy_workspace_size")(4096) == 0
    assert _ws(lib, "loom_kernels_relu_workspace_size")(1 << 26) == 0
    dot = _ws(lib, "loom_kernels_dot_workspace_size")
    assert dot(4096) > 0
    assert dot(0) == 0 and dot(-5) == 0
    assert dot(1 << 30) <= 600 * 1024  # bounded: at most 65536 fp64 partials
    assert dot(1 << 30) >= dot(4096)


def test_host_side_argument_checks(lib):
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: every check returns first
    saxpy = lib.loom_kernels_saxpy
    saxpy.argtypes = [ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    saxpy.restype = ctypes.c_int
    assert saxpy(2.5, fake, fake, -1, fake, None, 0) == 1       # n < 0
    assert saxpy(2.5, None, fake, 16, fake, None, 0) == 1       # null input
    assert saxpy(2.5, fake, None, 16, fake, None, 0) == 1
    assert saxpy(2.5, fake, fake, 16, None, None, 0) == 1       # null out
    dot = lib.loom_kernels_dot
    dot.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                    ctypes.c_void_p, ctypes.c_size_t]
    dot.restype = ctypes.c_int
    assert dot(fake, fake, 0, fake, fake, 1 << 20) == 1         # reductions need n > 0
    assert dot(fake, fake, 4096, fake, None, 0) == 2            # no workspace
    assert dot(fake, fake, 4096, fake, fake, 16) == 2           # workspace too small
    nows = lib.loom_kernels_relu_noworkspace
    nows.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    nows.restype = ctypes.c_int
    assert nows(fake, 0, fake) == 0 and nows(fake, -3, fake) == 0  # fast form: n <= 0 is OK


def test_multi_gpu_argument_checks(lib):
    """The multi-GPU entries reject bad arguments before any CUDA or NCCL call."""
    fake = ctypes.c_void_p(0x10000)
    multi = lib.loom_kernels_dot_multi
    multi.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                      ctypes.c_void_p]
    multi.restype = ctypes.c_int
    arr = (ctypes.c_void_p * 2)(0x10000, 0x10000)
    shard = (ctypes.c_int64 * 2)(16, 16)
    assert multi(0, arr, arr, arr, shard, arr, arr, arr, None) == 1       # no devices
    assert multi(25, arr, arr, arr, shard, arr, arr, arr, None) == 1      # > 24 ranks
    assert multi(2, None, arr, arr, shard, arr, arr, arr, None) == 1      # no communicators
    nulls = (ctypes.c_void_p * 2)(0x10000, None)
    assert multi(2, arr, nulls, arr, shard, arr, arr, arr, None) == 1    # null shard input
    bad = (ctypes.c_int64 * 2)(16, -1)
    assert multi(2, arr, arr, arr, bad, arr, arr, arr, None) == 1        # negative shard
    sizes = (ctypes.c_size_t * 2)(8, 8)
    assert multi(2, arr, arr, arr, shard, arr, arr, sizes, None) == 2    # workspace too small
    dist = lib.loom_kernels_dot_dist
    dist.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                     ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
    dist.restype = ctypes.c_int
    assert dist(fake, fake, -1, fake, fake, 1 << 20, fake, None) == 1     # n_local < 0
    assert dist(fake, fake, 16, fake, fake, 1 << 20, None, None) == 1     # no communicator
    assert dist(fake, fake, 16, fake, fake, 8, fake, None) == 2           # workspace too small
    rdist = lib.loom_kernels_relu_dist
    rdist.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                      ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
    rdist.restype = ctypes.c_int
    assert rdist(None, 0, None, None, 0, None, None) == 0                 # empty map shard
    init = lib.loom_b200_suite_comm_init_rank
    init.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t]
    init.restype = ctypes.c_int
    handle = ctypes.c_void_p(0)
    assert init(ctypes.byref(handle), 2, 2, fake, 128) == 1               # rank out of range
    assert init(ctypes.byref(handle), 0, 0, fake, 128) == 1               # no ranks
    assert init(ctypes.byref(handle), 2, 0, fake, 4) == 1                 # id too short
