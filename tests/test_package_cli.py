"""`python -m loom_b200 package`, exercised the way the reference's own
package tests exercise `loomc package` (test/python/test_package.py:29-165):
a project with a `kernels` module holding saxpy, relu and dot is packaged as
a shared library and, with module/entry filters and an optimisation flag, as
a static archive; the artefact layout and manifest fields are checked on CPU,
and on a GPU the shared library is bound with plain ctypes and compared with
torch at the reference tests' tolerance (rtol 1e-4, atol 1e-5)."""

import ctypes
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

KERNELS = '''import loom


@loom.entry
def saxpy(a: float, x: loom.Tensor1, y: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map2(lambda xi, yi: a * xi + yi, x, y)


@loom.entry
def relu(x: loom.Tensor1) -> loom.Tensor1:
    return loom.Tensor1.map(lambda xi: xi if xi > 0.0 else 0.0, x)


@loom.entry
def dot(x: loom.Tensor1, y: loom.Tensor1) -> float:
    products = loom.Tensor1.map2(lambda xi, yi: xi * yi, x, y)
    return loom.Tensor1.reduce_sum(products)
'''


def _project(tmp_path):
    proj = tmp_path / "package_project"
    proj.mkdir()
    (proj / "kernels.py").write_text(KERNELS)
    return proj


def _package(*args):
    return subprocess.run([sys.executable, "-m", "loom_b200", "package", *args], cwd=ROOT,
                          capture_output=True, text=True)


@pytest.fixture(scope="module")
def shared_package(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("pkg_shared")
    proj = _project(tmp)
    out = tmp / "out"
    result = _package("--project", str(proj), "--out", str(out))
    assert result.returncode == 0, result.stderr
    return out


def test_package_shared_layout(shared_package):
    out = shared_package
    for rel in ("libpackage_project.so", "include/loom/package_project.h",
                "src-gen/package_project.cu", "manifest.json", "report.md",
                "entries/loom_kernels_saxpy/tensor_ir.json",
                "entries/loom_kernels_dot/kernel_plan.json",
                "entries/loom_kernels_dot/cuda_plan.json",
                "entries/loom_kernels_dot/backend_analysis.json"):
        assert (out / rel).exists(), rel
    manifest = json.loads((out / "manifest.json").read_text())
    assert manifest["target_backend"] == "cuda"
    assert manifest["artifact_kind"] == "shared"
    assert sorted(e["entry_name"] for e in manifest["entries"]) == ["dot", "relu", "saxpy"]
    by_name = {e["entry_name"]: e for e in manifest["entries"]}
    assert by_name["saxpy"]["no_workspace_symbol"] == "loom_kernels_saxpy_noworkspace"
    assert by_name["dot"]["workspace_symbol"] == "loom_kernels_dot_workspace_size"
    assert [p["kind"] for p in by_name["saxpy"]["params"]] == [
        "scalar-f32", "tensor1-f32", "tensor1-f32"]
    assert by_name["dot"]["result_kind"] == "scalar"


def test_package_static_with_filters(tmp_path):
    proj = _project(tmp_path)
    out = tmp_path / "out"
    result = _package("--project", str(proj), "--out", str(out), "--kind", "static",
                      "--input-kind", "python", "--module", "kernels", "--entry", "relu",
                      "--enable-opt", "elementwise-plan-specialize")
    assert result.returncode == 0, result.stderr
    manifest = json.loads((out / "manifest.json").read_text())
    assert (out / "libpackage_project.a").exists()
    assert manifest["target_backend"] == "cuda"
    assert manifest["artifact_kind"] == "static"
    assert manifest["optimizations"]["enabled"] == ["elementwise-plan-specialize"]
    assert len(manifest["entries"]) == 1
    assert manifest["entries"][0]["entry_name"] == "relu"
    assert manifest["entries"][0]["symbol_name"] == "loom_kernels_relu"


def test_package_rejects_another_arch(tmp_path):
    proj = _project(tmp_path)
    result = _package("--project", str(proj), "--out", str(tmp_path / "o"), "--cuda-arch",
                      "sm_90a")
    assert result.returncode != 0 and "sm_100a" in result.stderr


@pytest.mark.gpu
def test_package_shared_library_runtime(shared_package):
    import torch

    def ptr(t):
        return ctypes.c_void_p(t.data_ptr())

    lib = ctypes.CDLL(str(shared_package / "libpackage_project.so"))
    saxpy_ws = lib.loom_kernels_saxpy_workspace_size
    saxpy_ws.argtypes = [ctypes.c_longlong]
    saxpy_ws.restype = ctypes.c_size_t
    assert saxpy_ws(4096) == 0
    saxpy = lib.loom_kernels_saxpy
    saxpy.argtypes = [ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    saxpy.restype = ctypes.c_int
    n, a = 4096, 2.5
    x = torch.randn(n, device="cuda")
    y = torch.randn(n, device="cuda")
    out = torch.empty_like(x)
    assert saxpy(ctypes.c_float(a), ptr(x), ptr(y), n, ptr(out), None, 0) == 0
    torch.testing.assert_close(out, a * x + y, rtol=1e-4, atol=1e-5)

    dot_ws = lib.loom_kernels_dot_workspace_size
    dot_ws.argtypes = [ctypes.c_longlong]
    dot_ws.restype = ctypes.c_size_t
    size = dot_ws(n)
    assert size > 0
    dot = lib.loom_kernels_dot
    dot.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p,
                    ctypes.c_void_p, ctypes.c_size_t]
    dot.restype = ctypes.c_int
    s = torch.empty(1, device="cuda")
    ws = torch.empty(size, device="cuda", dtype=torch.uint8)
    assert dot(ptr(x), ptr(y), n, ptr(s), ptr(ws), size) == 0
    torch.testing.assert_close(s[0], torch.sum(x * y), rtol=1e-4, atol=1e-5)


@pytest.fixture(scope="module")
def async_package(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("pkg_async")
    proj = _project(tmp)
    out = tmp / "out"
    result = _package("--project", str(proj), "--out", str(out),
                      "--enable-opt", "cuda-async-wrapper-return")
    assert result.returncode == 0, result.stderr
    return out


def test_async_wrapper_return_drops_the_final_synchronise(async_package, shared_package):
    # cuda_backend.ml:2263-2267: with cuda-async-wrapper-return the plain entry
    # returns right after its launches instead of synchronising the device
    manifest = json.loads((async_package / "manifest.json").read_text())
    assert manifest["optimizations"]["honoured"] == ["cuda-async-wrapper-return"]
    src = (async_package / "src-gen" / "package_project.cu").read_text()
    sync_src = (shared_package / "src-gen" / "package_project.cu").read_text()

    def plain_entry(text, name):
        start = text.index(f'extern "C" int loom_kernels_{name}(')
        return text[start:text.index("\n}\n", start)]

    for name in ("saxpy", "dot"):
        assert "finish_sync" in plain_entry(sync_src, name)
        assert "finish_sync" not in plain_entry(src, name)


@pytest.mark.gpu
def test_async_wrapper_return_results_after_synchronise(async_package):
    import torch
    from loom_b200.loader import Package
    pkg = Package(str(async_package))
    x = torch.randn(1 << 20, device="cuda")
    y = torch.randn(1 << 20, device="cuda")
    s = pkg["dot"](x=x, y=y)          # the plain entry: returns without synchronising
    torch.cuda.synchronize()
    torch.testing.assert_close(s[0], torch.sum(x.double() * y.double()).float(),
                               rtol=1e-5, atol=1e-4)


def _compile(*args):
    return subprocess.run([sys.executable, "-m", "loom_b200", "compile", *args], cwd=ROOT,
                          capture_output=True, text=True)


def test_compile_emits_the_reference_artifact_set(tmp_path):
    # test/python/test_cli.py:328-368 (the CUDA target with --emit all)
    (tmp_path / "kernels.py").write_text(KERNELS)
    out = tmp_path / "out"
    result = _compile(str(tmp_path / "kernels.py"), "--entry", "saxpy", "--target", "cuda",
                      "--out", str(out), "--emit", "all")
    assert result.returncode == 0, result.stderr
    expected = {"front_ir.json", "lambda.sexp", "loom_lambda.json", "tensor_ir.json",
                "kernel_plan.json", "cuda_plan.json", "backend_analysis.json", "pipeline.json",
                "manifest.json", "report.md", "saxpy_cuda.cu", "saxpy_cuda.h", "libsaxpy.so"}
    assert expected <= {p.name for p in out.iterdir()}
    manifest = json.loads((out / "manifest.json").read_text())
    assert manifest["target_backend"] == "cuda" and manifest["mode"] == "compile"
    assert [e["entry_name"] for e in manifest["entries"]] == ["saxpy"]
    assert manifest["entries"][0]["result_kind"] == "tensor"
    pipeline = json.loads((out / "pipeline.json").read_text())
    assert {"front_ir", "loom_lambda", "tensor_ir", "kernel_plan", "cuda_plan"} <= set(pipeline)
    assert pipeline["loom_lambda"] == json.loads((out / "loom_lambda.json").read_text())
    assert pipeline["loom_lambda"]["entry"] == "saxpy"
    # test/python/test_cli.py:198: non-OCaml frontends have no raw lambda
    assert "unavailable for this frontend" in (out / "lambda.sexp").read_text()


def test_compile_emit_selects_dumps_and_rejects_triton_kinds(tmp_path):
    (tmp_path / "kernels.py").write_text(KERNELS)
    out = tmp_path / "only_tir"
    result = _compile(str(tmp_path / "kernels.py"), "--entry", "dot", "--target", "cuda",
                      "--out", str(out), "--emit", "tensor-ir")
    assert result.returncode == 0, result.stderr
    names = {p.name for p in out.iterdir()}
    assert "tensor_ir.json" in names and "pipeline.json" in names and "libdot.so" in names
    assert not names & {"front_ir.json", "loom_lambda.json", "kernel_plan.json", "cuda_plan.json"}
    # test/python/test_cli.py:284-301
    result = _compile(str(tmp_path / "kernels.py"), "--entry", "dot", "--target", "cuda",
                      "--out", str(tmp_path / "bad"), "--emit", "triton-plan")
    assert result.returncode != 0
    assert "--emit triton-plan cannot be used with --target cuda" in result.stderr


def test_package_entry_dirs_hold_the_loom_lambda(shared_package):
    # cuda_backend.ml:2272-2313: lambda.sexp and loom_lambda.json beside the
    # TensorIR of every entry
    d = shared_package / "entries" / "loom_kernels_saxpy"
    assert (d / "lambda.sexp").read_text() == "; unavailable\n"
    lam = json.loads((d / "loom_lambda.json").read_text())
    assert lam["entry"] == "saxpy" and lam["body"]["kind"] == "tensor-prim"


def _cli(*args):
    return subprocess.run([sys.executable, "-m", "loom_b200", *args], cwd=ROOT,
                          capture_output=True, text=True)


def test_list_entries_and_front_ir_commands(tmp_path):
    # test/python/test_cli.py:75-96
    src = tmp_path / "kernels.py"
    src.write_text(KERNELS)
    result = _cli("list-entries", str(src), "--input-kind", "python")
    assert result.returncode == 0, result.stderr
    assert "saxpy (a:scalar-f32, x:tensor1-f32, y:tensor1-f32)" in result.stdout
    result = _cli("front-ir", str(src), "--input-kind", "py", "--entry", "saxpy")
    assert result.returncode == 0, result.stderr
    payload = json.loads(result.stdout)
    assert payload["entry"] == "saxpy"
    assert [p["type"] for p in payload["params"]] == ["float", "tensor1<f32>", "tensor1<f32>"]
    # main.ml:191, :335 and :219-226
    fir = tmp_path / "saxpy.front_ir.json"
    fir.write_text(result.stdout)
    bad = _cli("list-entries", str(fir), "--input-kind", "front-ir")
    assert bad.returncode != 0
    assert "list-entries does not support --input-kind front-ir" in bad.stderr
    bad = _cli("compile", str(fir), "--entry", "relu", "--out", str(tmp_path / "o"))
    assert bad.returncode != 0
    assert "FrontIR entry saxpy does not match requested --entry relu" in bad.stderr


CSE_KERNEL = '''import loom


@loom.entry
def twice(x: loom.Tensor1, y: loom.Tensor1) -> float:
    return loom.Tensor1.reduce_sum(loom.Tensor1.map2(lambda xi, yi: (xi - yi) + (xi - yi), x, y))
'''


def test_flags_are_checked_and_reported_in_catalogue_order(tmp_path):
    # optimization_config.ml:182-206, :269-274; test/python/test_cli.py:511-540
    src = tmp_path / "kernels.py"
    src.write_text(KERNELS)
    bad = _cli("compile", str(src), "--entry", "saxpy", "--out", str(tmp_path / "b"),
               "--enable-opt", "no-such-flag")
    assert bad.returncode != 0
    assert "unknown optimization flag no-such-flag in --enable-opt" in bad.stderr
    out = tmp_path / "o"
    ok = _cli("compile", str(src), "--entry", "saxpy", "--out", str(out), "--emit", "tensor-ir",
              "--enable-opt", "normalized-dce", "--enable-opt", "scalar-const-fold",
              "--enable-opt", "tensor-cse", "--disable-opt", "tensor-cse")
    assert ok.returncode == 0, ok.stderr
    manifest = json.loads((out / "manifest.json").read_text())
    assert manifest["optimizations"]["enabled"] == ["scalar-const-fold", "normalized-dce"]
    assert manifest["optimizations"]["config"]["small_inline_nodes"] == 20
    assert "enabled optimizations: scalar-const-fold, normalized-dce" in \
        (out / "report.md").read_text()


def test_opt_config_file_steers_the_passes(tmp_path):
    # optimization_config.ml:85-180: required fields, integers only, the
    # others defaulting; the thresholds reach the restated passes
    from loom_b200.optconfig import DEFAULT_CONFIG
    src = tmp_path / "kernels.py"
    src.write_text(CSE_KERNEL)
    cfg = DEFAULT_CONFIG.to_json()
    del cfg["source_path"]
    flags = ["--enable-opt", "reduce-map-fusion", "--enable-opt", "reduction-body-cse"]

    def body(config_path=None):
        out = tmp_path / f"o{len(list(tmp_path.iterdir()))}"
        extra = ["--opt-config", str(config_path)] if config_path else []
        r = _cli("compile", str(src), "--entry", "twice", "--out", str(out), "--emit",
                 "tensor-ir", *flags, *extra)
        assert r.returncode == 0, r.stderr
        manifest = json.loads((out / "manifest.json").read_text())
        return json.loads((out / "tensor_ir.json").read_text()), manifest

    tir, _ = body()
    red = tir["nodes"][-1]
    assert red["source"]["body"]["op"] == "add"        # one repeat: below the default of 2
    cfg["reduction_body_cse_min_occurrences"] = 1
    path = tmp_path / "cfg.json"
    path.write_text(json.dumps(cfg))
    tir, manifest = body(path)
    body_ = tir["nodes"][-1]["source"]["body"]
    # x+x -> 2*x, then canonical order ("b:sub:..." < "f:2"): (x - y) * 2
    assert body_["op"] == "mul" and body_["rhs"] == {"kind": "f32", "value": 2.0}
    assert body_["lhs"]["op"] == "sub"
    assert manifest["optimizations"]["config"]["source_path"] == str(path)
    for broken, message in (({k: v for k, v in cfg.items() if k != "version"},
                             "missing Loom optimization config field version"),
                            ({**cfg, "small_inline_nodes": 20.0},
                             "expected integer field small_inline_nodes")):
        path.write_text(json.dumps(broken))
        r = _cli("compile", str(src), "--entry", "twice", "--out", str(tmp_path / "x"),
                 "--opt-config", str(path))
        assert r.returncode != 0 and message in r.stderr


def test_package_rejects_empty_and_unsupported_projects(tmp_path):
    # test/python/test_package.py:257-287: a project without entries, and one
    # whose entry calls an unknown function inside a lambda
    empty = tmp_path / "empty_project"
    empty.mkdir()
    (empty / "helpers.py").write_text("def helper(x):\n    return x + 1.0\n")
    r = _package("--project", str(empty), "--out", str(tmp_path / "o1"))
    assert r.returncode != 0 and "[@loom.entry]" in r.stderr
    bad = tmp_path / "unsupported_project"
    bad.mkdir()
    front = {"entry": "bad", "params": [{"name": "x", "type": "tensor1<f32>"}],
             "return_type": "tensor1<f32>",
             "body": {"kind": "tensor-prim", "op": "tensor-map", "args": [
                 {"kind": "lambda", "params": [{"name": "xi", "type": "float"}],
                  "body": {"kind": "apply",
                           "fn": {"kind": "var", "name": "bad_scalar", "type": "(float -> float)"},
                           "args": [{"kind": "var", "name": "xi", "type": "float"}]}},
                 {"kind": "var", "name": "x", "type": "tensor1<f32>"}]}}
    (bad / "bad.front_ir.json").write_text(json.dumps(front))
    r = _package("--project", str(bad), "--out", str(tmp_path / "o2"))
    assert r.returncode != 0
    assert "unknown function call inside scalar lambda: bad_scalar" in r.stderr


def test_compile_target_platform_and_autotune_checks(tmp_path):
    # test/python/test_cli.py:222-323 (the CUDA-target cases) and main.ml:392-424
    src = tmp_path / "kernels.py"
    src.write_text(KERNELS)
    r = _cli("compile", str(src), "--entry", "relu", "--backend", "cuda", "--out",
             str(tmp_path / "o"), "--emit", "tensor-ir", "--cuda-platform", "native")
    assert r.returncode == 0, r.stderr
    manifest = json.loads((tmp_path / "o" / "manifest.json").read_text())
    assert manifest["cuda_platform"] == "current"
    assert manifest["cuda_tuning"]["max_partials"] == 32768
    r = _cli("compile", str(src), "--entry", "relu", "--target", "cuda", "--out",
             str(tmp_path / "a"), "--autotune")
    assert r.returncode != 0
    assert "does not support Triton autotuning flags" in r.stderr
    r = _cli("compile", str(src), "--entry", "relu", "--out", str(tmp_path / "p"),
             "--cuda-platform", "fastest")
    assert r.returncode != 0 and "unknown CUDA platform fastest" in r.stderr
    r = _cli("compile", str(src), "--entry", "relu", "--target", "triton", "--out",
             str(tmp_path / "t"))
    assert r.returncode != 0 and "--target cuda only" in r.stderr


def test_compile_tensor_ir_input_has_no_front_end_dumps(tmp_path):
    # a TensorIR source enters after loomc's front end: no FrontIR or
    # LoomLambda to dump, and pipeline.json says so with nulls
    src = os.path.join(ROOT, "oracle", "suite_kernels.tensor_ir.json")
    out = tmp_path / "tir"
    r = _cli("compile", src, "--entry", "dot", "--out", str(out), "--emit", "all",
             "--input-kind", "tensor-ir")
    assert r.returncode == 0, r.stderr
    names = {p.name for p in out.iterdir()}
    assert {"tensor_ir.json", "kernel_plan.json", "cuda_plan.json", "backend_analysis.json",
            "lambda.sexp", "pipeline.json", "libdot.so"} <= names
    assert not names & {"front_ir.json", "loom_lambda.json"}
    pipeline = json.loads((out / "pipeline.json").read_text())
    assert pipeline["front_ir"] is None and pipeline["loom_lambda"] is None
    assert pipeline["tensor_ir"]["entry_name"] == "dot"
