"""Command line with the shape of ``loomc compile|package --target cuda``
(``src/loom_cli/main.ml:305-346``, flags at ``:443-458``):

    python -m loom_b200 package --project DIR --out OUT [--kind shared|static]
                                [--input-kind auto|python] [--module M ...] [--entry E ...]
                                [--opt-config PATH] [--enable-opt FLAG ...]
                                [--disable-opt FLAG ...] [--no-multi-gpu]
    python -m loom_b200 compile FILE --entry E --target cuda --out OUT
                                [--emit KIND] [--input-kind auto|python|front-ir|tensor-ir]
                                [--opt-config PATH] [--enable-opt FLAG ...]
                                [--disable-opt FLAG ...]
    python -m loom_b200 list-entries FILE [--input-kind python]
    python -m loom_b200 front-ir FILE --entry E [--input-kind python]

Entries are read from ``*.tensor_ir.json`` files (the TensorIR the reference
front end dumps with ``--emit tensor-ir``), from ``*.front_ir.json`` files
(FrontIR, as any Loom frontend writes it) and from Python modules written in
the reference's entry language (``loom.entry`` functions); the last two are
lowered by ``loom_b200.frontend``; ``--cuda-arch`` is accepted for compatibility and
must name sm_100a.
"""

from __future__ import annotations

import argparse
import sys

from . import artifact
from .frontend import FrontendError
from .optconfig import DEFAULT_CONFIG, OptionsError, load_config, parse_cli_flags
from .tensor_ir import TensorIRError


def _options(ns) -> artifact.Options:
    """Flags and configuration as loomc reads them (optimization_config.ml:182-206):
    unknown flag names are errors; --opt-config replaces the default
    configuration."""
    enabled, disabled = [], []
    for item in ns.enable_opt or []:
        enabled += [f for f in item.split(",") if f]
    for item in ns.disable_opt or []:
        disabled += [f for f in item.split(",") if f]
    config = load_config(ns.opt_config) if ns.opt_config else DEFAULT_CONFIG
    platform = "current" if ns.cuda_platform.lower() in ("current", "native") else "generic"
    return artifact.Options(enabled=parse_cli_flags(enabled, disabled),
                            multi_gpu=not ns.no_multi_gpu,
                            kind=getattr(ns, "kind", "shared"), config=config,
                            cuda_platform=platform)


def _input_kind(value: str) -> str:
    """``--input-kind`` with the reference's spellings (main.ml:143-151)."""
    v = value.lower()
    kind = {"py": "python", "front_ir": "front-ir", "c++": "cpp"}.get(v, v)
    if kind not in ("auto", "python", "front-ir", "tensor-ir", "ocaml", "cpp"):
        raise artifact.BuildError(f"unknown input kind {value} (expected ocaml, python, cpp, "
                                  "or front-ir)")
    if kind in ("ocaml", "cpp"):
        raise artifact.BuildError(f"--input-kind {kind}: this backend reads Python, FrontIR "
                                  "and TensorIR sources (the OCaml and C++ frontends write "
                                  "FrontIR, which --input-kind front-ir takes)")
    return kind


def _read_python(path: str, kind: str, command: str) -> str:
    """The Python source that ``list-entries`` and ``front-ir`` read; a
    FrontIR input is refused with the reference's message (main.ml:191,
    :335)."""
    if kind == "front-ir":
        raise artifact.BuildError(f"{command} does not support --input-kind front-ir")
    if kind == "tensor-ir" or (kind == "auto" and not path.endswith(".py")):
        raise artifact.BuildError(f"{command} reads Python sources")
    with open(path, "r", encoding="utf-8") as fh:
        return fh.read()


def list_entries(path: str, kind: str) -> int:
    """``loomc list-entries`` (main.ml:166-201): one line per entry,
    ``name (param:kind, ...)``."""
    from .frontend import list_entries as entries
    src = _read_python(path, kind, "list-entries")
    for e in entries(src, path):
        params = ", ".join(f"{p['name']}:{p['kind']}" for p in e["params"])
        print(f"{e['name']} ({params})")
    return 0


def emit_front_ir(path: str, entry: str, kind: str) -> int:
    """``loomc front-ir`` (main.ml:332-338): the entry's FrontIR as JSON."""
    import json
    from .frontend import front_ir
    src = _read_python(path, kind, "front-ir command")
    print(json.dumps(front_ir(src, entry, path), indent=2))
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m loom_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)

    def common(p):
        p.add_argument("--out", required=True)
        # --backend is loomc's alias of --target (src/loom_cli/main.ml:422-424)
        p.add_argument("--target", "--backend", dest="target", default="cuda")
        p.add_argument("--cuda-arch", default="sm_100a")
        p.add_argument("--cuda-platform", default="generic")
        p.add_argument("--opt-config")
        p.add_argument("--enable-opt", action="append")
        p.add_argument("--disable-opt", action="append")
        p.add_argument("--no-multi-gpu", action="store_true")

    pk = sub.add_parser("package", help="package every entry of a project")
    pk.add_argument("--project", required=True)
    pk.add_argument("--kind", default="shared", choices=["shared", "static"])
    pk.add_argument("--module", action="append", default=[])
    pk.add_argument("--entry", action="append", default=[])
    pk.add_argument("--input-kind", default="auto")
    common(pk)

    cp = sub.add_parser("compile", help="compile one entry")
    cp.add_argument("file")
    cp.add_argument("--entry", required=True)
    cp.add_argument("--emit", default="all")
    cp.add_argument("--input-kind", default="auto")
    cp.add_argument("--autotune", action="store_true")
    cp.add_argument("--autotune-config")
    common(cp)

    le = sub.add_parser("list-entries", help="list the entries of a Python source")
    le.add_argument("file")
    le.add_argument("--input-kind", default="auto")

    fi = sub.add_parser("front-ir", help="print an entry's FrontIR")
    fi.add_argument("file")
    fi.add_argument("--entry", required=True)
    fi.add_argument("--input-kind", default="auto")

    ns = ap.parse_args(argv)
    try:
        if ns.cmd == "list-entries":
            return list_entries(ns.file, _input_kind(ns.input_kind))
        if ns.cmd == "front-ir":
            return emit_front_ir(ns.file, ns.entry, _input_kind(ns.input_kind))
    except (FrontendError, artifact.BuildError, OSError) as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 1
    if ns.cuda_arch not in ("sm_100a", "sm_100"):
        print(f"error: this backend targets sm_100a only (got {ns.cuda_arch})", file=sys.stderr)
        return 2
    # the reference's target, platform and autotuning checks (main.ml:392-412,
    # cuda_backend.ml:69-76)
    problem = None
    if ns.target.lower() != "cuda":
        problem = (f"this backend builds --target cuda only (got {ns.target}); the Triton "
                   "backend is not part of it")
    elif ns.cuda_platform.lower() not in ("generic", "portable", "current", "native"):
        problem = f"unknown CUDA platform {ns.cuda_platform} (expected generic or current)"
    elif getattr(ns, "autotune", False) or getattr(ns, "autotune_config", None):
        problem = "The generated CUDA backend does not support Triton autotuning flags"
    if problem:
        print(f"error: {problem}", file=sys.stderr)
        return 1
    try:
        if ns.cmd == "package":
            kind = _input_kind(ns.input_kind)
            if kind not in ("auto", "python"):
                raise artifact.BuildError(f"unknown package input kind {ns.input_kind} "
                                          "(expected ocaml, python, cpp, or auto)")
            res = artifact.generate_package(ns.project, ns.out, _options(ns), ns.module,
                                            ns.entry, input_kind=kind)
        else:
            res = artifact.compile_entry(ns.file, ns.entry, ns.out, _options(ns),
                                         input_kind=_input_kind(ns.input_kind),
                                         emit=artifact.parse_emit(ns.emit))
    except (TensorIRError, FrontendError, artifact.BuildError, OptionsError, OSError) as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 1
    print(res.artifact_path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
