"""CUDA source and C header generation for a Loom package on B200.

The generated package keeps the reference's C ABI (header layout of
``src/loom_backend_cuda/cuda_backend.ml:2315-2337``, prototypes of
``:875-896``, wrapper validation and status codes of ``:1828-1883`` and
``:2259-2267``) so ``lib<project>.so`` is a drop-in.  What differs is behind
the ABI: each entry instantiates the hand-written sm_100a kernels of
``csrc/loom_b200_device.cuh`` with a generated body functor.

Additive symbols (absent from the reference, declared after the reference
prototypes in the same header):

* ``<sym>_stream(..., void* stream)`` -- the same call, asynchronous on the
  given CUDA stream (the reference ABI always uses the legacy default stream),
  so callers can overlap copies and capture calls in CUDA graphs;
* ``<sym>_dist(..., int64_t n_local, ..., void* comm, void* stream)`` -- one
  rank's shard of a multi-GPU call (one process per GPU): maps run locally,
  reductions add one scalar NCCL collective;
* ``<sym>_multi(int ndev, void* const* comms, ...)`` -- one process driving
  ``ndev`` GPUs, one shard per device;
* ``loom_<pkg>_comm_*`` -- NCCL communicator set-up and tear-down for the two
  multi-GPU forms.
"""

from __future__ import annotations

from typing import List, Sequence

from .plan import EntryPlan, c_ident
from .tensor_ir import ScalarParam, TensorParam

# Names the generated C ABI uses for its own parameters, plus C/C++ keywords:
# a user parameter with one of these names is renamed p_<name> in C.
_RESERVED = {
    "n", "out", "workspace", "workspace_size", "stream", "comm", "n_local", "ndev", "comms",
    "shard_n", "host_result",
    "alignas", "alignof", "and", "asm", "auto", "bool", "break", "case", "catch", "char",
    "class", "const", "constexpr", "continue", "decltype", "default", "delete", "do", "double",
    "else", "enum", "explicit", "export", "extern", "false", "float", "for", "friend", "goto",
    "if", "inline", "int", "long", "mutable", "namespace", "new", "noexcept", "not", "nullptr",
    "operator", "or", "private", "protected", "public", "register", "return", "short",
    "signed", "sizeof", "static", "struct", "switch", "template", "this", "throw", "true",
    "try", "typedef", "typeid", "typename", "union", "unsigned", "using", "virtual", "void",
    "volatile", "while", "xor",
}


def cparam(name: str) -> str:
    """C name of an entry parameter in the generated ABI."""
    if name in _RESERVED or name.lower().startswith("loom"):
        return "p_" + name
    return name


STATUS_DEFINES = [
    ("LOOM_STATUS_OK", 0),
    ("LOOM_STATUS_INVALID_ARGUMENT", 1),
    ("LOOM_STATUS_WORKSPACE_TOO_SMALL", 2),
    ("LOOM_STATUS_CUDA_ERROR", 3),
    ("LOOM_STATUS_COMM_ERROR", 4),   # additive: NCCL failure in a multi-GPU entry
]


def _param_decls(plan: EntryPlan) -> List[str]:
    out = []
    for p in plan.program.params:
        if isinstance(p, ScalarParam):
            out.append(f"float {cparam(p.name)}")
        else:
            out.append(f"const float* {cparam(p.name)}")
    return out


def _multi_param_decls(plan: EntryPlan) -> List[str]:
    out = []
    for p in plan.program.params:
        if isinstance(p, ScalarParam):
            out.append(f"float {cparam(p.name)}")
        else:
            out.append(f"const float* const* {cparam(p.name)}")
    return out


def _arg_names(plan: EntryPlan) -> List[str]:
    return [cparam(p.name) for p in plan.program.params]


def header_prototypes(plan: EntryPlan, multi_gpu: bool = True) -> List[str]:
    """Prototypes for one entry: the reference's three, then the additive ones."""
    base = _param_decls(plan) + ["int64_t n", "float* out"]
    full = base + ["void* workspace", "size_t workspace_size"]
    protos = [
        f"size_t {plan.workspace_symbol}(int64_t n);",
        f"int {plan.symbol}({', '.join(full)});",
    ]
    if not plan.uses_workspace:
        protos.append(f"int {plan.symbol}_noworkspace({', '.join(base)});")
    protos.append(f"int {plan.symbol}_stream({', '.join(full + ['void* stream'])});")
    if multi_gpu:
        dist = _param_decls(plan) + ["int64_t n_local", "float* out", "void* workspace",
                                     "size_t workspace_size", "void* comm", "void* stream"]
        protos.append(f"size_t {plan.symbol}_dist_workspace_size(int64_t n_local);")
        protos.append(f"int {plan.symbol}_dist({', '.join(dist)});")
        multi = ["int ndev", "void* const* comms"] + _multi_param_decls(plan) + [
            "const int64_t* shard_n", "float* const* out", "void* const* workspace",
            "const size_t* workspace_size", "float* host_result"]
        protos.append(f"int {plan.symbol}_multi({', '.join(multi)});")
    return protos


def comm_prototypes(package: str) -> List[str]:
    p = f"loom_{package}_comm"
    return [
        f"int {p}_id_size(void);",
        f"int {p}_unique_id(void* id_out, size_t id_size);",
        f"int {p}_init_rank(void** comm_out, int nranks, int rank, const void* id, size_t id_size);",
        f"int {p}_init_all(void** comms_out, int ndev, const int* devices);",
        f"int {p}_destroy(void* comm);",
        f"int {p}_set_peer_exchange(void* comm, int enable);",
        f"int {p}_set_timeout_ms(void* comm, int64_t ms);",
        f"int {p}_peer_exchange(void* comm);",
        f"int {p}_check(void* comm);",
        f"int {p}_exchange_stats(void* comm, uint64_t* out, int reset);",
    ]


def noalloc_prototype(plan: EntryPlan) -> str:
    decls = _param_decls(plan) + ["int64_t n", "float* out", "void* stream"]
    return f"int {plan.symbol}_noalloc({', '.join(decls)});"


def render_header(package: str, plans: List[EntryPlan], multi_gpu: bool = True,
                  noalloc: Sequence[str] = ()) -> str:
    lines = ["#pragma once", "", "#include <stddef.h>", "#include <stdint.h>", "",
             "#ifdef __cplusplus", 'extern "C" {', "#endif", ""]
    lines.append("/* Status codes of Loom's CUDA packages (src/loom_backend_cuda/cuda_backend.ml:"
                 "2328-2331); COMM_ERROR is additive. */")
    for name, value in STATUS_DEFINES:
        lines.append(f"#define {name} {value}")
    lines += ["", f"/* Generated by the Loom B200 (sm_100a) backend for {package}. */", ""]
    for plan in plans:
        lines.append(f"/* {plan.program.entry_name}: the first "
                     f"{3 if not plan.uses_workspace else 2} prototypes replace the reference's "
                     "generated entry (src/loom_backend_cuda/cuda_backend.ml:875-896); "
                     "_stream, _dist and _multi are additive. */")
        lines += header_prototypes(plan, multi_gpu)
        if plan.program.entry_name in noalloc:
            lines.append(f"/* {plan.symbol}_noalloc: no counterpart in the reference.  The same "
                         "reduction for callers that cannot allocate device memory (no workspace "
                         f"argument): its per-CTA partials live in a static {NOALLOC_BYTES // 1024} KiB "
                         f"device array ({NOALLOC_SLOTS} slots) that the library holds on every GPU "
                         f"that loads it; the grid is capped at {NOALLOC_SLOTS} CTAs, so any n >= 1 "
                         "fits.  The first call on a device, and the first after its context is "
                         "re-created (cudaDeviceReset), looks the array up: make it before any "
                         "stream capture.  Calls that overlap on the GPU race on the array. */")
            lines.append(noalloc_prototype(plan))
    if multi_gpu:
        lines.append("")
        lines.append("/* Communicators for the _dist and _multi entries (additive; the reference has "
                     "no multi-GPU path): NCCL, plus a peer-memory scalar exchange where every GPU "
                     "reaches the others'. _set_peer_exchange switches paths (every rank alike); "
                     "an exchange waits at most _set_timeout_ms (30 s by default) for the other "
                     "ranks; _check reports one that gave up; _exchange_stats reads (and with "
                     "reset zeroes) the total and largest time this rank's exchanges waited, in ns, "
                     "and their number. */")
        lines += comm_prototypes(package)
    lines += ["", "#ifdef __cplusplus", "}", "#endif", ""]
    return "\n".join(lines)


# Reduction families whose values are never negative (an fp32 value times
# itself): the square families of the reference's reduction classification.
NONNEGATIVE_FAMILIES = ("norm-square", "delta-square")


def render_body_struct(plan: EntryPlan) -> str:
    k = len(plan.slots)
    name = f"LoomBody_{plan.symbol}"
    out = [f"// {plan.program.entry_name}: {plan.kind}"
           + (f" ({plan.reduce_kind})" if plan.reduce_kind else "")
           + f", slots [{', '.join(plan.slots)}], family {plan.family}",
           f"struct {name} {{",
           f"  static constexpr int kInputs = {k};",
           # a reduction over squares (x*x, (a-b)*(a-b)) never adds a negative
           # value, so its sums may add within a tile in fp32 (Chunking)
           "  static constexpr bool kNonNegative = "
           + ("true;" if plan.kind == "reduce" and plan.family in NONNEGATIVE_FAMILIES
              else "false;")]
    for s in plan.scalar_args:
        out.append(f"  float {c_ident(s)};")
    out.append("  __device__ __forceinline__ float operator()(const float* in) const {")
    for blk in plan.blocks:
        out.append(f"    float {blk.temp};")
        out.append("    {" + (f"  // node_{blk.node_id}" if blk.node_id is not None else
                              "  // mapped reduction source"))
        for cname, expr in blk.bindings:
            out.append(f"      const float {cname} = {expr};")
        for line in blk.lines:
            out.append("      " + line)
        out.append(f"      {blk.temp} = value;")
        out.append("    }")
    out.append(f"    return {plan.result_expr};")
    out += ["  }", "};", ""]
    return "\n".join(out)


def _validation(plan: EntryPlan, n_name: str = "n") -> List[str]:
    """Argument checks in the reference's order (cuda_backend.ml:1863-1883)."""
    lines = []
    if plan.kind == "reduce":
        lines.append(f"  if ({n_name} <= 0) return LOOM_STATUS_INVALID_ARGUMENT;")
    else:
        lines.append(f"  if ({n_name} < 0) return LOOM_STATUS_INVALID_ARGUMENT;")
    for p in plan.program.params:
        if isinstance(p, TensorParam):
            lines.append(f"  if ({cparam(p.name)} == nullptr) return LOOM_STATUS_INVALID_ARGUMENT;")
    lines.append("  if (out == nullptr) return LOOM_STATUS_INVALID_ARGUMENT;")
    return lines


def _body_setup(plan: EntryPlan, ptr_expr=lambda name: name) -> List[str]:
    name = f"LoomBody_{plan.symbol}"
    lines = [f"  {name} loom_body;"]
    for s in plan.scalar_args:
        lines.append(f"  loom_body.{c_ident(s)} = {cparam(s)};")
    ptrs = ", ".join(ptr_expr(cparam(p)) for p in plan.slots)
    lines.append(f"  const loomb::Ptrs<{len(plan.slots)}> loom_in = {{{{{ptrs}}}}};")
    return lines


def _op(plan: EntryPlan) -> str:
    return "loomb::SumOp" if plan.reduce_kind == "sum" else "loomb::MaxOp"


def render_entry(plan: EntryPlan, async_return: bool, multi_gpu: bool = True,
                 package: str = "") -> str:
    sym = plan.symbol
    decls = _param_decls(plan)
    args = _arg_names(plan)
    full = decls + ["int64_t n", "float* out", "void* workspace", "size_t workspace_size"]
    L: List[str] = []
    # workspace size (cuda_backend.ml:1674-1715 for the reference's carving)
    L.append(f'extern "C" size_t {plan.workspace_symbol}(int64_t n) {{')
    if plan.uses_workspace:
        L.append("  return loomb::reduce_workspace_bytes(n);")
    else:
        L.append("  (void)n;")
        L.append("  return 0;")
    L.append("}")
    L.append("")
    # stream form: validation + launch, never synchronises
    L.append(f'extern "C" int {sym}_stream({", ".join(full + ["void* stream"])}) {{')
    L += _validation(plan)
    L.append(f"  const size_t loom_needed = {plan.workspace_symbol}(n);")
    L.append("  if (loom_needed > 0 && (workspace == nullptr || workspace_size < "
             "loom_needed)) return LOOM_STATUS_WORKSPACE_TOO_SMALL;")
    if plan.kind == "map":
        L.append("  (void)workspace;")
        L.append("  (void)workspace_size;")
    L += _body_setup(plan)
    L.append("  cudaStream_t loom_stream = static_cast<cudaStream_t>(stream);")
    if plan.kind == "map":
        L.append("  return loomb::launch_map(out, loom_in, n, loom_body, loom_stream);")
    else:
        acc = "double" if plan.reduce_kind == "sum" else "float"
        L.append(f"  {acc}* loom_partials = reinterpret_cast<{acc}*>(loomb::workspace_base(workspace));")
        L.append(f"  return loomb::launch_reduce<{_op(plan)}>(loom_in, n, loom_body, loom_partials, "
                 "loomb::partial_capacity(n), out, nullptr, loom_stream);")
    L.append("}")
    L.append("")
    # the reference entry: legacy default stream, synchronous unless built with
    # cuda-async-wrapper-return (cuda_backend.ml:2259-2267)
    L.append(f'extern "C" int {sym}({", ".join(full)}) {{')
    call_args = ", ".join(args + ["n", "out", "workspace", "workspace_size", "nullptr"])
    L.append(f"  const int loom_status = {sym}_stream({call_args});")
    L.append("  if (loom_status != LOOM_STATUS_OK) return loom_status;")
    L.append("  return LOOM_STATUS_OK;" if async_return else "  return loomb::finish_sync();")
    L.append("}")
    L.append("")
    if not plan.uses_workspace:
        base = decls + ["int64_t n", "float* out"]
        L.append(f'extern "C" int {sym}_noworkspace({", ".join(base)}) {{')
        L.append("  if (n <= 0) return LOOM_STATUS_OK;")
        L.append(f"  return {sym}({', '.join(args + ['n', 'out', 'nullptr', '0'])});")
        L.append("}")
        L.append("")
    if multi_gpu:
        L += _render_dist(plan, async_return)
        L += _render_multi(plan, async_return)
    return "\n".join(L)


def _render_dist(plan: EntryPlan, async_return: bool) -> List[str]:
    sym = plan.symbol
    decls = _param_decls(plan) + ["int64_t n_local", "float* out", "void* workspace",
                                  "size_t workspace_size", "void* comm", "void* stream"]
    L = [f'extern "C" size_t {sym}_dist_workspace_size(int64_t n_local) {{']
    if plan.uses_workspace:
        L.append("  return loomb::reduce_workspace_bytes(n_local > 0 ? n_local : 1);")
    else:
        L.append("  (void)n_local;")
        L.append("  return 0;")
    L += ["}", ""]
    L.append(f'extern "C" int {sym}_dist({", ".join(decls)}) {{')
    if plan.kind == "map":
        args = ", ".join(_arg_names(plan) + ["n_local", "out", "workspace", "workspace_size",
                                              "stream"])
        L.append("  (void)comm;  // a map shard needs no communication")
        L.append("  if (n_local < 0) return LOOM_STATUS_INVALID_ARGUMENT;")
        L.append("  if (n_local == 0) return LOOM_STATUS_OK;  // an empty shard may have null pointers")
        L.append(f"  return {sym}_stream({args});")
    else:
        L.append("  if (n_local < 0) return LOOM_STATUS_INVALID_ARGUMENT;")
        for p in plan.program.params:
            if isinstance(p, TensorParam):
                L.append(f"  if (n_local > 0 && {cparam(p.name)} == nullptr) return "
                         "LOOM_STATUS_INVALID_ARGUMENT;")
        L.append("  if (out == nullptr || comm == nullptr) return LOOM_STATUS_INVALID_ARGUMENT;")
        L.append(f"  const size_t loom_needed = {sym}_dist_workspace_size(n_local);")
        L.append("  if (workspace == nullptr || workspace_size < loom_needed) "
                 "return LOOM_STATUS_WORKSPACE_TOO_SMALL;")
        L += _body_setup(plan)
        op = _op(plan)
        L.append(f"  return loomb::dist_reduce<{op}>(loom_in, n_local, loom_body, workspace, out, "
                 "static_cast<loomb::Comm*>(comm), static_cast<cudaStream_t>(stream));")
    L += ["}", ""]
    return L


def _render_multi(plan: EntryPlan, async_return: bool) -> List[str]:
    """One process, ``ndev`` GPUs: local shards on every device, then (for a
    reduction) the scalar exchange: through peer memory where the
    communicators set it up, else one grouped NCCL collective and the rank
    fold on every device."""
    sym = plan.symbol
    decls = ["int ndev", "void* const* comms"] + _multi_param_decls(plan) + [
        "const int64_t* shard_n", "float* const* out", "void* const* workspace",
        "const size_t* workspace_size", "float* host_result"]
    L = [f'extern "C" int {sym}_multi({", ".join(decls)}) {{']
    L.append("  if (ndev <= 0 || ndev > loomb::kMaxRanks || comms == nullptr || shard_n == nullptr"
             " || out == nullptr) return LOOM_STATUS_INVALID_ARGUMENT;")
    for p in plan.program.params:
        if isinstance(p, TensorParam):
            L.append(f"  if ({cparam(p.name)} == nullptr) return LOOM_STATUS_INVALID_ARGUMENT;")
    L.append("  for (int loom_d = 0; loom_d < ndev; ++loom_d) {")
    out_null = "out[loom_d] == nullptr" if plan.kind == "reduce" else \
        "(shard_n[loom_d] > 0 && out[loom_d] == nullptr)"
    L.append(f"    if (comms[loom_d] == nullptr || {out_null} || shard_n[loom_d] < 0) "
             "return LOOM_STATUS_INVALID_ARGUMENT;")
    for p in plan.program.params:
        if isinstance(p, TensorParam):
            L.append(f"    if (shard_n[loom_d] > 0 && {cparam(p.name)}[loom_d] == nullptr) "
                     "return LOOM_STATUS_INVALID_ARGUMENT;")
    if plan.uses_workspace:
        L.append("    if (workspace == nullptr || workspace_size == nullptr || workspace[loom_d] == nullptr"
                 f" || workspace_size[loom_d] < {sym}_dist_workspace_size(shard_n[loom_d])) "
                 "return LOOM_STATUS_WORKSPACE_TOO_SMALL;")
    L.append("  }")
    L.append("  loomb::DeviceGuard loom_guard;")
    if plan.kind != "map":
        L.append("  const bool loom_peer = loomb::all_peer_exchange(ndev, comms);")
    L.append("  for (int loom_d = 0; loom_d < ndev; ++loom_d) {")
    L.append("    loomb::Comm* loom_c = static_cast<loomb::Comm*>(comms[loom_d]);")
    L.append("    if (cudaSetDevice(loom_c->device) != cudaSuccess) return LOOM_STATUS_CUDA_ERROR;")
    args = [f"{cparam(p.name)}[loom_d]" if isinstance(p, TensorParam) else cparam(p.name)
            for p in plan.program.params]
    if plan.kind == "map":
        L.append("    if (shard_n[loom_d] == 0) continue;")
        L.append(f"    const int loom_status = {sym}_stream({', '.join(args)}, shard_n[loom_d], out[loom_d], "
                 "nullptr, 0, nullptr);")
        L.append("    if (loom_status != LOOM_STATUS_OK) return loom_status;")
        L.append("  }")
        L.append("  (void)workspace;")
        L.append("  (void)workspace_size;")
        L.append("  (void)host_result;")
    else:
        op = _op(plan)
        L += ["  " + line for line in _body_setup(plan, lambda name: f"{name}[loom_d]")]
        L.append("    // peer memory: reduce and exchange on each device in turn (each exchange")
        L.append("    // waits for the devices launched after it); NCCL: the local phase only")
        L.append(f"    const int loom_status = loom_peer")
        L.append(f"        ? loomb::dist_local_exchange<{op}>(loom_in, shard_n[loom_d], loom_body, "
                 "workspace[loom_d], out[loom_d], loom_c, nullptr)")
        L.append(f"        : loomb::dist_local<{op}>(loom_in, shard_n[loom_d], loom_body, "
                 "workspace[loom_d], nullptr);")
        L.append("    if (loom_status != LOOM_STATUS_OK) return loom_status;")
        L.append("  }")
        L.append("  if (!loom_peer) {")
        L.append(f"    const int loom_exchange = loomb::multi_nccl_exchange<{op}>(ndev, comms, "
                 "workspace, shard_n, out);")
        L.append("    if (loom_exchange != LOOM_STATUS_OK) return loom_exchange;")
        L.append("  }")
        L.append("  if (host_result != nullptr) {")
        L.append("    loomb::Comm* loom_c0 = static_cast<loomb::Comm*>(comms[0]);")
        L.append("    if (cudaSetDevice(loom_c0->device) != cudaSuccess) return LOOM_STATUS_CUDA_ERROR;")
        L.append("    if (cudaMemcpy(host_result, out[0], sizeof(float), cudaMemcpyDeviceToHost) != "
                 "cudaSuccess) return LOOM_STATUS_CUDA_ERROR;")
        L.append("  }")
    if not async_return:
        L.append("  for (int loom_d = 0; loom_d < ndev; ++loom_d) {")
        L.append("    loomb::Comm* loom_c = static_cast<loomb::Comm*>(comms[loom_d]);")
        L.append("    if (cudaSetDevice(loom_c->device) != cudaSuccess) return LOOM_STATUS_CUDA_ERROR;")
        L.append("    if (loomb::finish_sync() != LOOM_STATUS_OK) return LOOM_STATUS_CUDA_ERROR;")
        L.append("  }")
    L.append("  return LOOM_STATUS_OK;")
    L += ["}", ""]
    return L


def render_comm_api(package: str) -> str:
    p = f"loom_{package}_comm"
    return "\n".join([
        f'extern "C" int {p}_id_size(void) {{ return loomb::comm_id_size(); }}',
        f'extern "C" int {p}_unique_id(void* id_out, size_t id_size) {{',
        "  return loomb::comm_unique_id(id_out, id_size);",
        "}",
        f'extern "C" int {p}_init_rank(void** comm_out, int nranks, int rank, const void* id, '
        "size_t id_size) {",
        "  return loomb::comm_init_rank(comm_out, nranks, rank, id, id_size);",
        "}",
        f'extern "C" int {p}_init_all(void** comms_out, int ndev, const int* devices) {{',
        "  return loomb::comm_init_all(comms_out, ndev, devices);",
        "}",
        f'extern "C" int {p}_destroy(void* comm) {{ return loomb::comm_destroy(comm); }}',
        f'extern "C" int {p}_set_peer_exchange(void* comm, int enable) {{',
        "  return loomb::comm_set_peer_exchange(comm, enable);",
        "}",
        f'extern "C" int {p}_set_timeout_ms(void* comm, int64_t ms) {{',
        "  return loomb::comm_set_timeout_ms(comm, ms);",
        "}",
        f'extern "C" int {p}_peer_exchange(void* comm) {{ return loomb::comm_peer_exchange(comm); }}',
        f'extern "C" int {p}_check(void* comm) {{ return loomb::comm_check(comm); }}',
        f'extern "C" int {p}_exchange_stats(void* comm, uint64_t* out, int reset) {{',
        "  return loomb::comm_exchange_stats(comm, reinterpret_cast<unsigned long long*>(out), reset);",
        "}",
        "",
    ])


NOALLOC_SLOTS = 4096
NOALLOC_BYTES = 8 * NOALLOC_SLOTS     # one fp64 partial per CTA


def render_noalloc_scratch() -> str:
    """The static scratch array shared by every ``<sym>_noalloc`` entry of a
    package, and the per-context lookup of its device address (emitted once
    per generated source)."""
    return "\n".join([
        "// ---------------------------------------------------------------------------",
        "// Scratch for the _noalloc entries: callers that cannot allocate.",
        "//",
        "// Some callers have no way to give this library device memory: a host",
        "// application or plugin whose framework owns every byte of the GPU through",
        "// its own allocator, a latency-critical loop where cudaMalloc (which may",
        "// synchronise the whole device) is not allowed, or a C caller of the plain",
        "// ABI, whose reductions otherwise demand a sized workspace argument (only",
        "// maps have a _noworkspace form).  A _noalloc entry needs nothing but the",
        "// inputs and the 1-float output: its per-CTA partials go to the static",
        f"// array below, {NOALLOC_SLOTS} fp64 slots ({NOALLOC_BYTES // 1024} KiB), which every GPU that loads",
        "// the library holds until the process exits.",
        "//",
        "// Host code must not hand the array's name to a kernel: on the host it is",
        "// only a stand-in for the device symbol.  The entries look up the real",
        "// device address with cudaGetSymbolAddress, with the device current, once",
        "// per CUDA context: on the first call on each device, and again when that",
        "// device's context has been re-created since (after cudaDeviceReset the",
        "// module is loaded anew and the array may move), which the cache notices",
        "// by the context's unique id.  Make the first call on each device, and",
        "// the first after a reset, before any stream capture.",
        f"constexpr int kLoomNoallocSlots = {NOALLOC_SLOTS};",
        "static __device__ __align__(256) double loom_noalloc_scratch[kLoomNoallocSlots];",
        "",
        "namespace {",
        "using LoomCtxGetCurrent = CUresult (*)(CUcontext*);",
        "using LoomCtxGetId = CUresult (*)(CUcontext, unsigned long long*);",
        "",
        "struct LoomNoallocCache {",
        "  unsigned long long context_id;",
        "  void* address;",
        "};",
        "",
        "std::mutex loom_noalloc_mutex;",
        "LoomNoallocCache loom_noalloc_cache[loomb::kMaxDevices];",
        "LoomCtxGetCurrent loom_ctx_get_current = nullptr;",
        "LoomCtxGetId loom_ctx_get_id = nullptr;",
        "",
        "// Unique id of the calling thread's current CUDA context (0 when there is",
        "// none yet); the two driver functions are resolved through the runtime,",
        "// so the library does not link the driver library itself.  Called with",
        "// loom_noalloc_mutex held.",
        "bool loom_current_context_id(unsigned long long* id) {",
        "  if (loom_ctx_get_current == nullptr || loom_ctx_get_id == nullptr) {",
        "    void* get_current = nullptr;",
        "    void* get_id = nullptr;",
        "    cudaDriverEntryPointQueryResult q1, q2;",
        "    if (cudaGetDriverEntryPointByVersion(\"cuCtxGetCurrent\", &get_current, 12000,",
        "                                         cudaEnableDefault, &q1) != cudaSuccess ||",
        "        cudaGetDriverEntryPointByVersion(\"cuCtxGetId\", &get_id, 12000, cudaEnableDefault,",
        "                                         &q2) != cudaSuccess ||",
        "        q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess ||",
        "        get_current == nullptr || get_id == nullptr) {",
        "      cudaGetLastError();",
        "      return false;",
        "    }",
        "    loom_ctx_get_current = reinterpret_cast<LoomCtxGetCurrent>(get_current);",
        "    loom_ctx_get_id = reinterpret_cast<LoomCtxGetId>(get_id);",
        "  }",
        "  CUcontext ctx = nullptr;",
        "  if (loom_ctx_get_current(&ctx) != CUDA_SUCCESS) return false;",
        "  *id = 0;",
        "  return ctx == nullptr || loom_ctx_get_id(ctx, id) == CUDA_SUCCESS;",
        "}",
        "",
        "// Device address of loom_noalloc_scratch on device `dev` (the current one)",
        "// in its current context: looked up on the first call in each context.",
        "int loom_noalloc_scratch_on(int dev, void** address) {",
        "  if (dev < 0 || dev >= loomb::kMaxDevices) return LOOM_STATUS_CUDA_ERROR;",
        "  std::lock_guard<std::mutex> lock(loom_noalloc_mutex);",
        "  unsigned long long id = 0;",
        "  if (!loom_current_context_id(&id)) return LOOM_STATUS_CUDA_ERROR;",
        "  LoomNoallocCache& c = loom_noalloc_cache[dev];",
        "  if (id != 0 && c.address != nullptr && c.context_id == id) {",
        "    *address = c.address;",
        "    return LOOM_STATUS_OK;",
        "  }",
        "  // set-up in this context (cudaGetSymbolAddress also creates the device's",
        "  // primary context when the thread has none yet)",
        "  void* p = nullptr;",
        "  const cudaError_t err = cudaGetSymbolAddress(&p, loom_noalloc_scratch);",
        "  if (err != cudaSuccess || p == nullptr) {",
        "    cudaGetLastError();",
        "    return LOOM_STATUS_CUDA_ERROR;",
        "  }",
        "  if (id == 0 && !loom_current_context_id(&id)) return LOOM_STATUS_CUDA_ERROR;",
        "  c.context_id = id;",
        "  c.address = p;",
        "  *address = p;",
        "  return LOOM_STATUS_OK;",
        "}",
        "}  // namespace",
        "",
    ])


def render_noalloc(plan: EntryPlan) -> str:
    """The no-allocation variant of one reduction entry, over the shared
    scratch of ``render_noalloc_scratch``."""
    if plan.kind != "reduce":
        raise ValueError(f"{plan.program.entry_name}: only a reduction uses scratch memory")
    sym = plan.symbol
    decls = _param_decls(plan) + ["int64_t n", "float* out", "void* stream"]
    L = [
        f"// {sym}_noalloc -- {plan.program.entry_name} with its CTA partials in the shared",
        "// static scratch above (no workspace argument).  The grid is capped at the",
        f"// {NOALLOC_SLOTS} slots (for large n each CTA then walks several tiles), so every",
        "// n >= 1 fits; while n needs no more tiles than that, it launches the same",
        "// grid as the workspace entry and gives the same bits, past that it differs",
        "// only in rounding order.  Nothing in the array has to start at zero:",
        "// every slot the finalize kernel reads was written by the same call's",
        "// first kernel.  All calls of all _noalloc entries share the array, so two",
        "// calls whose kernels overlap on the GPU (different streams, no ordering",
        "// between them) race and corrupt each other's partials: keep calls",
        "// ordered on one stream.",
        f'extern "C" int {sym}_noalloc({", ".join(decls)}) {{',
    ]
    L += _validation(plan)
    L.append("  void* loom_scratch = nullptr;")
    L.append("  const int loom_status = loom_noalloc_scratch_on(loomb::current_device(), &loom_scratch);")
    L.append("  if (loom_status != LOOM_STATUS_OK) return loom_status;")
    L += _body_setup(plan)
    # the slot count is the array's, whatever the accumulator (fp64 for sums,
    # fp32 for max), so the grid cap is kLoomNoallocSlots for both
    acc = "double" if plan.reduce_kind == "sum" else "float"
    L.append(f"  return loomb::launch_reduce<{_op(plan)}>(loom_in, n, loom_body, "
             f"static_cast<{acc}*>(loom_scratch), (int64_t)kLoomNoallocSlots, out, nullptr, "
             "static_cast<cudaStream_t>(stream));")
    L += ["}", ""]
    return "\n".join(L)


def render_source(package: str, header_include: str, plans: List[EntryPlan],
                  async_return: bool, multi_gpu: bool = True,
                  noalloc: Sequence[str] = ()) -> str:
    parts = [
        f"// Generated by the Loom B200 (sm_100a) backend for {package}.",
        "// Body functors are generated; the kernels are the hand-written ones in",
        "// loom_b200_device.cuh.  Build: -gencode arch=compute_100a,code=sm_100a -fmad=false.",
        "#include <cuda_runtime.h>",
        "#include <math.h>",
        "#include <stddef.h>",
        "#include <stdint.h>",
        f'#include "{header_include}"',
        '#include "loom_b200_launch.cuh"',
    ]
    if noalloc:
        parts += ["#include <cuda.h>", "#include <mutex>"]
    if multi_gpu:
        parts.append('#include "loom_b200_comm.cuh"')
    parts += ["", "namespace {", ""]
    for plan in plans:
        parts.append(render_body_struct(plan))
    parts += ["}  // namespace", ""]
    for plan in plans:
        parts.append(render_entry(plan, async_return, multi_gpu, package))
    noalloc_plans = [p for p in plans if p.program.entry_name in noalloc]
    if noalloc_plans:
        parts.append(render_noalloc_scratch())
    for plan in noalloc_plans:
        parts.append(render_noalloc(plan))
    if multi_gpu:
        parts.append(render_comm_api(package))
    return "\n".join(parts)
