"""Package and compile drivers: TensorIR entries -> lib<project>.so + header,
manifest, report and per-entry plan dumps.

Follows the artefact layout of the reference's CUDA packaging
(``src/loom_backend_cuda/cuda_backend.ml:2675-2816``):

* ``package``: ``<out>/include/loom/<pkg>.h``, ``<out>/src-gen/<pkg>.cu``,
  ``<out>/lib<pkg>.so`` (or ``.a``), ``<out>/manifest.json``,
  ``<out>/report.md`` and ``<out>/entries/<symbol>/*``;
* ``compile``: ``<out>/<entry>_cuda.h``, ``<out>/<entry>_cuda.cu``,
  ``<out>/lib<entry>.so``, ``manifest.json``, ``report.md``.

The nvcc line targets sm_100a only (``-gencode arch=compute_100a,
code=sm_100a``) and adds ``-fmad=false`` (see ``render.py``) and the NCCL
link for the multi-GPU entries.
"""

from __future__ import annotations

import json
import os
import shlex
import shutil
import subprocess
from dataclasses import dataclass, field
from pathlib import Path
from typing import Iterable, List, Optional, Sequence

from . import codegen
from .optconfig import DEFAULT_CONFIG, OptConfig, in_catalogue_order
from .plan import EntryPlan, plan_entry, plan_to_json, sanitize_ident
from .tensor_ir import (Program, TensorIRError, program_from_json, program_to_json,
                        program_to_string)

CSRC = Path(__file__).resolve().parent / "csrc"
CUDA_ARCH = "sm_100a"
GENCODE = "arch=compute_100a,code=sm_100a"

# Reference optimisation flags that change this backend's output: the async
# wrapper return, and the flags that change how map bodies are rendered (and
# so their bits).  The front-end pass flags below act before the backend;
# every other flag is accepted and recorded, as the B200 plan (always fused,
# always vectorised, deterministic reductions) does not depend on it.
HONOURED_FLAGS = {"cuda-async-wrapper-return", "cuda-pointwise-tail-tune",
                  "cuda-pointwise-predicated-select", "cuda-pointwise-selected-tail-plan",
                  "cuda-body-trait-analysis", "shared-body-trait-analysis"}
# The LoomLambda scalar passes, the TensorIR passes and the policy flags that
# steer fusion, which the front end applies to Python and FrontIR sources
# (frontend/normalize_passes.py, frontend/passes.py); TensorIR files are
# taken as given, as `loomc` ran its passes before writing them.
FRONTEND_PASS_FLAGS = {"map-chain-collapse", "elementwise-fusion", "small-producer-clone",
                       "reduce-map-fusion", "shape-use-simplify", "materialization-choice",
                       "reduction-materialization-choice", "reduction-late-fusion-guard",
                       "branch-aware-fusion-guard", "pointwise-materialization-guard",
                       # normalize_scalar.ml
                       "scalar-const-fold", "if-simplify", "arith-reassociate", "let-float",
                       "branch-hoist", "lambda-inline-small", "scalar-cse", "normalized-dce",
                       "scalar-hoist",
                       # tensor_passes.ml body rewrites and node CSE
                       "tensor-canonicalize", "reduction-input-simplify",
                       "reduction-body-normalize", "reduction-accumulator-shape",
                       "reduction-reuse-hoist", "branchy-reduction-rescue",
                       "reduction-body-canonicalize", "reduction-body-cse", "tensor-cse"}


class BuildError(RuntimeError):
    pass


@dataclass
class Options:
    enabled: List[str] = field(default_factory=list)
    multi_gpu: bool = True
    kind: str = "shared"          # "shared" | "static"
    nvcc: str = "nvcc"
    extra_nvcc_flags: List[str] = field(default_factory=list)
    # reduction entries that also get a <sym>_noalloc variant (static scratch)
    noalloc_entries: List[str] = field(default_factory=list)
    # the tuning configuration (``--opt-config``); its pass thresholds steer
    # the front end
    config: OptConfig = DEFAULT_CONFIG
    # ``--cuda-platform`` as recorded in the manifest; the sm_100a build is the
    # same for both
    cuda_platform: str = "generic"

    @property
    def async_return(self) -> bool:
        return "cuda-async-wrapper-return" in self.enabled

    def to_json(self) -> dict:
        """The reference's ``optimizations`` object (enabled flags in
        catalogue order, and the configuration; optimization_config.ml:269-274),
        with what each flag does here."""
        on = in_catalogue_order(self.enabled)
        return {"enabled": on, "config": self.config.to_json(),
                "honoured": [f for f in on if f in HONOURED_FLAGS],
                "tensor_ir_passes_for_python_sources": [f for f in on if f in FRONTEND_PASS_FLAGS],
                "no_effect_on_b200_plan": [f for f in on if f not in HONOURED_FLAGS
                                           and f not in FRONTEND_PASS_FLAGS]}


@dataclass
class EntryBundle:
    module_name: str
    source_file: str
    program: Program
    plan: EntryPlan
    # the FrontIR and LoomLambda entries it was lowered from (None for a
    # TensorIR source)
    front_ir: Optional[dict] = None
    loom_lambda: Optional[dict] = None


def module_name_of_file(path: str) -> str:
    base = os.path.basename(path)
    for suffix in (".tensor_ir.json", ".front_ir.json", ".json", ".py", ".ml", ".cpp"):
        if base.endswith(suffix):
            base = base[: -len(suffix)]
            break
    return sanitize_ident(base)


def load_entries_file(path: str) -> List[Program]:
    """A ``*.tensor_ir.json`` file holds one TensorIR program or a list."""
    with open(path, "r", encoding="utf-8") as fh:
        obj = json.load(fh)
    items = obj if isinstance(obj, list) else [obj]
    return [program_from_json(item) for item in items]


def _defines_entries(path: str) -> bool:
    with open(path, "r", encoding="utf-8") as fh:
        text = fh.read()
    return "loom.entry" in text or "@entry" in text


def load_front_ir_file(path: str, enabled: Sequence[str] = (),
                       cfg: OptConfig = DEFAULT_CONFIG) -> List[Program]:
    """A ``*.front_ir.json`` file: one FrontIR entry or a list, as any Loom
    frontend writes it (``loomc compile --input-kind front-ir``,
    ``src/loom_cli/main.ml:219-226``), lowered through normalize and
    tensorize here."""
    return [prog for _, _, prog in _front_ir_file_stages(path, enabled, cfg)]


def _front_ir_file_stages(path: str, enabled: Sequence[str], cfg: OptConfig = DEFAULT_CONFIG):
    from .frontend import front_ir_stages
    with open(path, "r", encoding="utf-8") as fh:
        obj = json.load(fh)
    return [front_ir_stages(e, enabled, cfg) for e in (obj if isinstance(obj, list) else [obj])]


def load_source_file(path: str, enabled: Sequence[str] = (), kind: str = "auto",
                     cfg: OptConfig = DEFAULT_CONFIG) -> List[Program]:
    """Programs of one source: a ``*.tensor_ir.json`` (one program or a list,
    taken as given), a ``*.front_ir.json`` (FrontIR entries), or a Python
    module of ``@loom.entry`` functions (through the front end); the last two
    with the TensorIR passes `enabled` switches on.  `kind` ("python",
    "front-ir", "tensor-ir") overrides the choice by file name."""
    return [prog for _, _, prog in load_source_stages(path, enabled, kind, cfg)]


def load_source_stages(path: str, enabled: Sequence[str] = (), kind: str = "auto",
                       cfg: OptConfig = DEFAULT_CONFIG):
    """As ``load_source_file``, with each program's FrontIR and LoomLambda
    entries: ``(front_ir, loom_lambda, program)``, the first two None for a
    TensorIR source."""
    if kind == "auto":
        kind = ("python" if path.endswith(".py") else
                "front-ir" if path.endswith(".front_ir.json") else "tensor-ir")
    if kind == "python":
        from .frontend import python_stages
        return python_stages(path, enabled, cfg)
    if kind == "front-ir":
        return _front_ir_file_stages(path, enabled, cfg)
    if kind == "tensor-ir":
        return [(None, None, prog) for prog in load_entries_file(path)]
    raise TensorIRError(f"unknown input kind {kind!r} (expected python, front-ir or tensor-ir)")


def discover_entries(project_root: str, module_filters: Sequence[str] = (),
                     entry_filters: Sequence[str] = (), enabled: Sequence[str] = (),
                     input_kind: str = "auto", cfg: OptConfig = DEFAULT_CONFIG
                     ) -> List[EntryBundle]:
    """Collect entries of a project (cuda_backend.ml:158-178, 307-326): every
    ``*.tensor_ir.json``, every ``*.front_ir.json`` and every Python module
    with ``@loom.entry`` functions below the root (only the Python modules
    when `input_kind` is "python"), skipping build and hidden dirs, in path
    order."""
    skip = {"_build", "build", ".venv", ".git", ".hg", ".svn", "node_modules", "__pycache__"}
    found: List[str] = []
    for dirpath, dirnames, filenames in os.walk(project_root):
        dirnames[:] = sorted(d for d in dirnames if d not in skip and not d.startswith("."))
        for name in sorted(filenames):
            path = os.path.join(dirpath, name)
            ir_file = name.endswith(".tensor_ir.json") or name.endswith(".front_ir.json")
            if ((ir_file and input_kind == "auto")
                    or (name.endswith(".py") and _defines_entries(path))):
                found.append(path)
    mfilt = [m.lower() for m in module_filters]
    efilt = [e.lower() for e in entry_filters]
    bundles: List[EntryBundle] = []
    for path in found:
        module = module_name_of_file(path)
        if mfilt and module.lower() not in mfilt:
            continue
        for front, lam, prog in load_source_stages(path, enabled, cfg=cfg):
            if efilt and prog.entry_name.lower() not in efilt:
                continue
            bundles.append(EntryBundle(module, path, prog, plan_entry(prog, module, enabled),
                                       front, lam))
    return bundles


def package_name_of_root(root: str) -> str:
    """``loom-package.json`` name, else the directory name (cuda_backend.ml:192-208)."""
    marker = os.path.join(root, "loom-package.json")
    if os.path.exists(marker):
        try:
            with open(marker, "r", encoding="utf-8") as fh:
                name = json.load(fh).get("name", "")
            if isinstance(name, str) and name.strip():
                return sanitize_ident(name)
        except (OSError, ValueError):
            pass
    return sanitize_ident(os.path.basename(os.path.abspath(root)))


def nvcc_command(opts: Options, include_dir: str, source: str, artifact: str,
                 object_only: bool = False) -> List[str]:
    cmd = [opts.nvcc, "-std=c++17", "-O3", "-gencode", GENCODE, "-fmad=false", "-lineinfo",
           "-Xptxas", "-O3", f"-I{include_dir}", f"-I{CSRC}"]
    if object_only:
        cmd += ["-c", "-Xcompiler", "-fPIC", "-o", artifact, source]
    else:
        cmd += ["-shared", "-Xcompiler", "-fPIC", "-o", artifact, source]
        if opts.multi_gpu:
            cmd.append("-lnccl")
    return cmd + list(opts.extra_nvcc_flags)


def _run(cmd: List[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise BuildError(f"command failed ({proc.returncode}): {shlex.join(cmd)}\n"
                         f"{proc.stdout}\n{proc.stderr}")


def build_artifact(opts: Options, include_dir: str, source: str, artifact: str) -> List[str]:
    if shutil.which(opts.nvcc) is None and not os.path.exists(opts.nvcc):
        raise BuildError("nvcc is required on PATH for the Loom B200 backend")
    if opts.kind == "shared":
        cmd = nvcc_command(opts, include_dir, source, artifact)
        _run(cmd)
        return [shlex.join(cmd)]
    obj = os.path.splitext(source)[0] + ".o"
    cmd = nvcc_command(opts, include_dir, source, obj, object_only=True)
    _run(cmd)
    ar = ["ar", "rcs", artifact, obj]
    _run(ar)
    return [shlex.join(cmd), shlex.join(ar)]


def _entry_json(b: EntryBundle, files: List[str], package: str, multi_gpu: bool) -> dict:
    p = b.plan
    d = {
        "entry_name": b.program.entry_name,
        "module_name": b.module_name,
        "source_file": b.source_file,
        "symbol_name": p.symbol,
        "workspace_symbol": p.workspace_symbol,
        "result_kind": b.program.result_kind,
        "params": [{"name": q.name, "kind": "scalar-f32"} if not hasattr(q, "shape_symbol")
                   else {"name": q.name, "kind": "tensor1-f32", "shape_symbol": q.shape_symbol}
                   for q in b.program.params],
        "kernel_count": 1,
        "temporary_count": 0,
        "generated_files": files,
    }
    if not p.uses_workspace:
        d["no_workspace_symbol"] = p.symbol + "_noworkspace"
    d["stream_symbol"] = p.symbol + "_stream"
    if multi_gpu:
        d["dist_symbol"] = p.symbol + "_dist"
        d["dist_workspace_symbol"] = p.symbol + "_dist_workspace_size"
        d["multi_symbol"] = p.symbol + "_multi"
    d["b200_plan"] = plan_to_json(p)
    return d


def _noalloc_symbols(bundles, opts) -> List[str]:
    return [b.plan.symbol + "_noalloc" for b in bundles
            if b.program.entry_name in opts.noalloc_entries]


def _manifest(mode, project_root, package, opts, artifact, header, source, entry_files,
              commands) -> str:
    obj = {
        "mode": mode,
        "target_backend": "cuda",
        "backend": "loom-b200",
        "project_root": project_root,
        "package_name": package,
        "artifact_kind": opts.kind,
        "cuda_arch": CUDA_ARCH,
        "cuda_platform": opts.cuda_platform,
        # the launch constants of loom_b200/csrc/loom_b200_device.cuh
        "cuda_tuning": {"block_size": 256, "finalize_threads": 1024, "max_partials": 32768,
                        "max_cluster_ctas": 8,
                        "map_float4_per_input_per_thread": {"one_input": 2, "more_inputs": 1},
                        "reduce_float4_per_input_per_thread": {"one_input": 4, "more_inputs": 2},
                        "grid": "one CTA per tile"},
        "artifact_path": artifact,
        "header_path": header,
        "source_path": source,
        "entries": [_entry_json(b, files, package, opts.multi_gpu) for b, files in entry_files],
        "optimizations": opts.to_json(),
        "build_commands": commands,
    }
    if opts.noalloc_entries:
        obj["noalloc_symbols"] = _noalloc_symbols([b for b, _ in entry_files], opts)
    if opts.multi_gpu:
        obj["comm_symbols"] = [line.split("(")[0].split()[-1]
                               for line in codegen.comm_prototypes(package)]
    return json.dumps(obj, indent=2)


def _report(title, project_root, package, opts, artifact, header, source, bundles,
            commands) -> str:
    lines = [title, "",
             f"- project root: `{project_root}`",
             "- pipeline: `TensorIR -> B200 fused plan -> sm_100a CUDA`",
             f"- package: `{package}`",
             f"- artifact kind: `{opts.kind}`",
             f"- CUDA arch: `{CUDA_ARCH}`",
             f"- artifact: `{artifact}`",
             f"- header: `{header}`",
             f"- source: `{source}`",
             f"- exported entrypoints: `{len(bundles)}`",
             "- enabled optimizations: " + (", ".join(in_catalogue_order(opts.enabled))
                                            if opts.enabled else "none"),
             ""]
    for b in bundles:
        p = b.plan
        lines += [f"## `{p.symbol}`", "",
                  f"- entrypoint: `{b.program.entry_name}`",
                  f"- source: `{b.source_file}`",
                  f"- result kind: `{b.program.result_kind}`",
                  f"- kernel: `{p.kind}`" + (f" ({p.reduce_kind})" if p.reduce_kind else ""),
                  f"- launches per call: `{1 if p.kind == 'map' else 2}`",
                  f"- fused nodes: `{len(p.fused_node_ids)}`",
                  f"- HBM bytes per element: `{p.bytes_per_element}`",
                  "- temporary allocations: `0`", ""]
    lines += ["## Build Commands", ""] + [f"- `{c}`" for c in commands] + [""]
    return "\n".join(lines)


def _write(path: str, text: str) -> None:
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "w", encoding="utf-8") as fh:
        fh.write(text)


def _backend_analysis(b: EntryBundle) -> str:
    return json.dumps({
        "entry_name": b.program.entry_name,
        "hbm_bytes_per_element": b.plan.bytes_per_element,
        "roofline": "hbm",
        "tensor_slots": b.plan.slots,
    }, indent=2)


def _write_entry_dir(out_dir: str, b: EntryBundle) -> List[str]:
    """``entries/<symbol>/`` (cuda_backend.ml:2272-2313): the OCaml raw
    lambda is unavailable (no OCaml frontend here); the LoomLambda is
    written when the entry came from a Python or FrontIR source."""
    sym = b.plan.symbol
    rel = os.path.join("entries", sym)
    files = {"lambda.sexp": "; unavailable\n"}
    if b.loom_lambda is not None:
        files["loom_lambda.json"] = json.dumps(b.loom_lambda, indent=2)
    files.update({
        "tensor_ir.json": program_to_string(b.program),
        "kernel_plan.json": json.dumps(plan_to_json(b.plan), indent=2),
        "cuda_plan.json": json.dumps(plan_to_json(b.plan), indent=2),
        "backend_analysis.json": _backend_analysis(b),
        "report.md": "\n".join([
            "# Loom Entry Report", "",
            f"- entrypoint: `{b.program.entry_name}`",
            f"- module: `{b.module_name}`",
            f"- source: `{b.source_file}`",
            "- pipeline: `TensorIR -> B200 fused plan -> sm_100a CUDA`",
            f"- exported symbol: `{sym}`",
            f"- workspace function: `{b.plan.workspace_symbol}`",
            f"- result kind: `{b.program.result_kind}`",
            "- generated kernels: `1`",
            "- temporary allocations: `0`", ""]),
    })
    out = []
    for name, text in files.items():
        _write(os.path.join(out_dir, rel, name), text)
        out.append(os.path.join(rel, name))
    return out


@dataclass
class PackageResult:
    project_root: str
    package_name: str
    artifact_path: str
    header_path: str
    source_path: str
    manifest_path: str
    report_path: str
    build_commands: List[str]


def generate_package(project_root: str, out_dir: str, opts: Optional[Options] = None,
                     module_filters: Sequence[str] = (), entry_filters: Sequence[str] = (),
                     build: bool = True, package_name: Optional[str] = None,
                     input_kind: str = "auto") -> PackageResult:
    """``loomc package --target cuda`` (cuda_backend.ml:2733-2816) for B200."""
    opts = opts or Options()
    project_root = os.path.abspath(project_root)
    package = package_name or package_name_of_root(project_root)
    bundles = discover_entries(project_root, module_filters, entry_filters, opts.enabled,
                               input_kind, opts.config)
    if not bundles:
        raise TensorIRError("no Loom entry bindings ([@loom.entry], @loom.entry, or LOOM_ENTRY) "
                            "matched the requested project selection")  # cuda_backend.ml:2761
    symbols = [b.plan.symbol for b in bundles]
    if len(set(symbols)) != len(symbols):
        raise TensorIRError("duplicate entry symbols in project: " + ", ".join(symbols))
    out_dir = os.path.abspath(out_dir)
    include_root = os.path.join(out_dir, "include")
    header = os.path.join(include_root, "loom", package + ".h")
    source = os.path.join(out_dir, "src-gen", package + ".cu")
    ext = "so" if opts.kind == "shared" else "a"
    artifact = os.path.join(out_dir, f"lib{package}.{ext}")
    plans = [b.plan for b in bundles]
    _write(header, codegen.render_header(package, plans, opts.multi_gpu, opts.noalloc_entries))
    _write(source, codegen.render_source(package, f"loom/{package}.h", plans,
                                         opts.async_return, opts.multi_gpu,
                                         opts.noalloc_entries))
    entry_files = [(b, _write_entry_dir(out_dir, b)) for b in bundles]
    commands = build_artifact(opts, include_root, source, artifact) if build else \
        [shlex.join(nvcc_command(opts, include_root, source, artifact))]
    manifest = os.path.join(out_dir, "manifest.json")
    report = os.path.join(out_dir, "report.md")
    _write(manifest, _manifest("package", project_root, package, opts, artifact, header, source,
                               entry_files, commands))
    _write(report, _report("# Loom Package Report", project_root, package, opts, artifact,
                           header, source, bundles, commands))
    return PackageResult(project_root, package, artifact, header, source, manifest, report,
                         commands)


# `loomc compile --emit <kind>` (src/loom_cli/main.ml:53-67); "all" is every
# kind the CUDA target writes (:241-268)
EMIT_KINDS = ("front-ir", "lambda", "loom-lambda", "tensor-ir", "kernel-plan", "cuda-plan",
              "backend-analysis", "cuda", "report")


def parse_emit(value: str) -> List[str]:
    """The kinds one ``--emit`` value selects, with the reference's errors
    (main.ml:53-67, 78-112)."""
    if value in ("triton-plan", "triton"):
        raise BuildError(f"--emit {value} cannot be used with --target cuda")
    if value == "all":
        return list(EMIT_KINDS)
    if value not in EMIT_KINDS:
        raise BuildError(f"unknown emit target {value}")
    return [value]


def compile_entry(source_file: str, entry_name: str, out_dir: str,
                  opts: Optional[Options] = None, build: bool = True,
                  input_kind: str = "auto", emit: Sequence[str] = EMIT_KINDS) -> PackageResult:
    """``loomc compile <file> --entry e --target cuda`` (src/loom_cli/main.ml:228-330,
    cuda_backend.ml:2675-2731): the IR dumps that `emit` selects, then
    ``pipeline.json`` and the header, source, library, manifest and report
    that the CUDA target always writes.  ``lambda.sexp`` says the OCaml raw
    lambda is unavailable, as the reference says for its non-OCaml
    frontends; ``front_ir.json`` and ``loom_lambda.json`` need a Python or
    FrontIR source."""
    opts = opts or Options()
    module = module_name_of_file(source_file)
    loaded = load_source_stages(source_file, opts.enabled, input_kind, opts.config)
    stages = [st for st in loaded if st[2].entry_name == entry_name]
    front_ir_file = input_kind == "front-ir" or (
        input_kind == "auto" and source_file.endswith(".front_ir.json"))
    if not stages and front_ir_file and len(loaded) == 1:
        # main.ml:219-226: a FrontIR file holds one entry, which must be the one asked for
        raise TensorIRError(f"FrontIR entry {loaded[0][0]['entry']} does not match requested "
                            f"--entry {entry_name}")
    if not stages:
        raise TensorIRError(f"entry {entry_name!r} not found in {source_file}")
    front, lam, prog = stages[0]
    b = EntryBundle(module, os.path.abspath(source_file), prog,
                    plan_entry(prog, module, opts.enabled), front, lam)
    out_dir = os.path.abspath(out_dir)
    plan_text = json.dumps(plan_to_json(b.plan), indent=2)
    dumps = {"front-ir": ("front_ir.json", None if front is None else json.dumps(front, indent=2)),
             "lambda": ("lambda.sexp", "; unavailable for this frontend\n"),
             "loom-lambda": ("loom_lambda.json",
                             None if lam is None else json.dumps(lam, indent=2)),
             "tensor-ir": ("tensor_ir.json", program_to_string(prog)),
             "kernel-plan": ("kernel_plan.json", plan_text),
             "cuda-plan": ("cuda_plan.json", plan_text),
             "backend-analysis": ("backend_analysis.json", _backend_analysis(b))}
    for kind in emit:
        name, text = dumps.get(kind, (None, None))
        if text is not None:
            _write(os.path.join(out_dir, name), text)
    _write(os.path.join(out_dir, "pipeline.json"), json.dumps({
        "front_ir": front, "loom_lambda": lam, "tensor_ir": program_to_json(prog),
        "kernel_plan": plan_to_json(b.plan), "cuda_plan": plan_to_json(b.plan),
        "optimizations": opts.to_json()}, indent=2))
    header = os.path.join(out_dir, f"{entry_name}_cuda.h")
    source = os.path.join(out_dir, f"{entry_name}_cuda.cu")
    artifact = os.path.join(out_dir, f"lib{entry_name}.so")
    package = b.plan.symbol
    _write(header, codegen.render_header(package, [b.plan], opts.multi_gpu))
    _write(source, codegen.render_source(package, os.path.basename(header), [b.plan],
                                         opts.async_return, opts.multi_gpu))
    commands = build_artifact(opts, out_dir, source, artifact) if build else \
        [shlex.join(nvcc_command(opts, out_dir, source, artifact))]
    files = [os.path.basename(p) for p in (header, source, artifact)]
    manifest = os.path.join(out_dir, "manifest.json")
    report = os.path.join(out_dir, "report.md")
    _write(manifest, _manifest("compile", os.path.dirname(b.source_file), package, opts,
                               artifact, header, source, [(b, files)], commands))
    _write(report, _report("# Loom CUDA Compile Report", os.path.dirname(b.source_file), package,
                           opts, artifact, header, source, [b], commands))
    return PackageResult(os.path.dirname(b.source_file), package, artifact, header, source,
                         manifest, report, commands)
