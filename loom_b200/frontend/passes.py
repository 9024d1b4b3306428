"""The reference's TensorIR fusion passes, for the Python front end.

`loomc` runs these after tensorization when their flags are enabled
(``src/loom_tensorize/tensor_passes.ml:595-620``); with them the TensorIR
that reaches a backend has producer maps folded into their consumers:

* ``fuse_program`` (``tensor_passes.ml:130-232``) -- under
  ``map-chain-collapse``, ``elementwise-fusion`` or ``small-producer-clone``:
  an element-wise producer is substituted into an element-wise consumer's
  body, its inputs renamed ``<binding>__<input>__f<i>``;
* ``reduce_map_fusion_program`` (``:251-335``) -- under
  ``reduce-map-fusion``: a reduction over an element-wise node becomes a
  mapped reduction (``MappedInput``), inputs renamed ``<input>__r<i>``;
* ``shape_use_simplify`` (``:103-112``) -- under ``shape-use-simplify``: nodes
  the result does not reach are dropped;

each gated by the materialisation policy
(``src/loom_tensorize/materialization_policy.ml:1-94``), and the handling
hints that annotation attaches (``materialization_hint``, ``:1-44``).  The
thresholds come from the optimisation configuration (``loom_b200/optconfig.py``).

and the body rewrites and node CSE (``:6-60``, ``:337-513``), applied before
and again after fusion (``:554-666``):

* ``tensor-canonicalize`` -- operands of +, *, min, max, == in rank order,
  compare-and-pick selects turned into min/max;
* ``reduction-input-simplify`` -- constant folding and algebraic identities;
* ``reduction-body-normalize`` / ``reduction-accumulator-shape``,
  ``reduction-reuse-hoist``, ``reduction-body-canonicalize``,
  ``branchy-reduction-rescue``, ``reduction-body-cse`` -- the same rewrites,
  and product reordering, on mapped-reduction bodies;
* ``tensor-cse`` -- nodes with equal keys merged.

The B200 plan inlines every element-wise chain into one kernel whether or
not the fusion passes ran, so those change the TensorIR (and its dump under
``entries/``), not the kernels, except for which rendering flags apply to a
body (a body fused into a reduction renders with the defaults).  The body
rewrites do change the kernels: a reordered sum or a folded constant rounds
differently, and the oracle, which evaluates the rewritten TensorIR, follows.
"""

from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

from .. import tensor_ir as TI
from . import analysis as A
from ..optconfig import DEFAULT_CONFIG, OptConfig
from .lower import _use_counts, body_metrics

# The thresholds come from the optimisation configuration (``--opt-config``;
# by default the values of the reference's configs/optimizations/current.json).

FUSE_FLAGS = ("map-chain-collapse", "elementwise-fusion", "small-producer-clone")


def _on(enabled: Sequence[str], flag: str) -> bool:
    return flag in enabled


# --- materialisation policy (materialization_policy.ml) -----------------------

def allow_inline_producer(enabled, m: TI.BodyMetrics, use_count: int,
                          cfg: OptConfig = DEFAULT_CONFIG) -> str:
    """"fuse", "clone" or "disallow" for an element-wise producer
    (materialization_policy.ml:46-68)."""
    branch_guard = (_on(enabled, "branch-aware-fusion-guard") and m.has_branch
                    and m.scalar_complexity >= cfg.branchy_fusion_complexity_threshold)
    pointwise_guard = (_on(enabled, "pointwise-materialization-guard")
                       and (m.has_branch or m.has_div)
                       and m.scalar_complexity
                       >= cfg.pointwise_materialization_complexity_threshold)
    if branch_guard or pointwise_guard:
        return "disallow"
    if use_count <= 1:
        return "fuse"
    if (_on(enabled, "materialization-choice")
            and m.scalar_complexity >= cfg.materialize_multi_use_complexity_threshold):
        return "disallow"
    return "clone"


def allow_inline_into_reduction(enabled, m: TI.BodyMetrics, use_count: int,
                                target_complexity: int,
                                cfg: OptConfig = DEFAULT_CONFIG) -> str:
    """The same decision for a producer feeding a reduction
    (materialization_policy.ml:70-94)."""
    late_guard = _on(enabled, "reduction-late-fusion-guard") and (
        m.scalar_complexity + target_complexity >= cfg.reduction_late_fusion_complexity_threshold
        or (m.has_branch and target_complexity > 0)
        or m.repeated_subexpressions >= cfg.reduction_body_cse_min_occurrences)
    if late_guard:
        return "disallow"
    if (_on(enabled, "reduction-materialization-choice")
            and (m.scalar_complexity >= cfg.reduction_materialize_complexity_threshold
                 or m.has_branch
                 or m.div_count > 0)
            and use_count > 1):
        return "disallow"
    return allow_inline_producer(enabled, m, use_count, cfg)


def materialization_hint(enabled, m: TI.BodyMetrics, reduction_shape,
                         cfg: OptConfig = DEFAULT_CONFIG) -> str:
    """The handling hint annotation attaches to a node
    (materialization_policy.ml:1-44)."""
    if not _on(enabled, "materialization-choice"):
        return "no-preference"
    if reduction_shape is not None and _on(enabled, "reduction-materialization-choice"):
        if reduction_shape == "branchy-mapped":
            return "prefer-materialize"
        if reduction_shape == "ratio-mapped" and (
                m.scalar_complexity >= cfg.reduction_materialize_complexity_threshold
                or m.div_count > 0):
            return "prefer-materialize"
        if reduction_shape == "weighted-mapped" and (
                m.repeated_subexpressions > 0 or m.estimated_uses > 1):
            return "prefer-clone"
        if m.estimated_uses <= 1:
            return "prefer-fuse"
        if (m.scalar_complexity >= cfg.reduction_materialize_complexity_threshold
                or m.repeated_subexpressions > 0):
            return "prefer-materialize"
        return "prefer-clone"
    if reduction_shape == "branchy-mapped":
        return "prefer-materialize"
    if reduction_shape == "ratio-mapped" and m.scalar_complexity >= 3:
        return "prefer-materialize"
    if m.estimated_uses <= 1:
        return "prefer-fuse"
    if m.scalar_complexity <= cfg.small_clone_nodes:
        return "prefer-clone"
    if m.has_branch or m.scalar_complexity >= cfg.materialize_multi_use_complexity_threshold:
        return "prefer-materialize"
    return "prefer-clone"


# --- expression helpers (reduction_analysis.ml:376-396) ------------------------

def substitute(name: str, replacement, e):
    if isinstance(e, TI.SVar):
        return replacement if e.name == name else e
    if isinstance(e, TI.SUnary):
        return TI.SUnary(e.op, substitute(name, replacement, e.expr))
    if isinstance(e, TI.SBinary):
        return TI.SBinary(e.op, substitute(name, replacement, e.lhs),
                          substitute(name, replacement, e.rhs))
    if isinstance(e, TI.SSelect):
        return TI.SSelect(substitute(name, replacement, e.cond),
                          substitute(name, replacement, e.then),
                          substitute(name, replacement, e.els))
    return e


def rename_vars(renamings: List[Tuple[str, str]], e):
    """Applies the renamings one after another, as the reference does."""
    for old, new in renamings:
        e = substitute(old, TI.SVar(new), e)
    return e


def _fresh(base: str, suffix: str, existing: Sequence[TI.InputBinding]) -> str:
    names = {b.name for b in existing}
    i = 0
    while f"{base}__{suffix}{i}" in names:
        i += 1
    return f"{base}__{suffix}{i}"


# --- the passes -----------------------------------------------------------------

def fuse_program(prog: TI.Program, enabled, allow_clone: bool = False,
                 cfg: OptConfig = DEFAULT_CONFIG) -> TI.Program:
    """Element-wise producers into element-wise consumers
    (tensor_passes.ml:130-232)."""
    uses = _use_counts(prog)
    done: Dict[int, TI.Elementwise1D] = {}
    fused = set()
    nodes = []
    for node in prog.nodes:
        if not isinstance(node, TI.Elementwise1D):
            done[node.id] = node
            nodes.append(node)
            continue
        inputs: List[TI.InputBinding] = []
        body = node.body
        scalars = list(node.scalar_params)
        for b in node.inputs:
            producer = done.get(b.source.id) if isinstance(b.source, TI.NodeRef) else None
            use_count = uses.get(b.source.id) if isinstance(b.source, TI.NodeRef) else None
            if not isinstance(producer, TI.Elementwise1D) or use_count is None:
                inputs.append(b)
                continue
            decision = allow_inline_producer(enabled, body_metrics(use_count, producer.body),
                                             use_count, cfg)
            if decision == "disallow" or (
                    decision == "clone"
                    and (not allow_clone
                         or TI.complexity(producer.body) > cfg.small_clone_nodes)):
                inputs.append(b)
                continue
            if use_count == 1:
                fused.add(producer.id)
            renamed, renamings = [], []
            for pi in producer.inputs:
                fresh = _fresh(f"{b.name}__{pi.name}", "f", inputs + renamed)
                renamed.append(TI.InputBinding(fresh, pi.source))
                renamings.append((pi.name, fresh))
            body = substitute(b.name, rename_vars(renamings, producer.body), body)
            inputs = inputs + renamed
            scalars = sorted(set(scalars) | set(producer.scalar_params))
        new = TI.Elementwise1D(node.id, tuple(inputs), tuple(scalars), body,
                               shape_symbol=node.shape_symbol, metrics=node.metrics,
                               handling_hint=node.handling_hint)
        done[node.id] = new
        nodes.append(new)
    prog.nodes = [n for n in nodes if n.id not in fused]
    return prog


def reduce_map_fusion_program(prog: TI.Program, enabled, allow_clone: bool = False,
                              cfg: OptConfig = DEFAULT_CONFIG) -> TI.Program:
    """A reduction over an element-wise node becomes a mapped reduction
    (tensor_passes.ml:251-335)."""
    uses = _use_counts(prog)
    by_id = {n.id: n for n in prog.nodes}
    fused = set()
    nodes = []
    for node in prog.nodes:
        src = node.source if isinstance(node, TI.Reduce1D) else None
        if not (isinstance(src, TI.PlainInput) and isinstance(src.input, TI.NodeRef)):
            nodes.append(node)
            continue
        producer = by_id.get(src.input.id)
        use_count = uses.get(src.input.id)
        if not isinstance(producer, TI.Elementwise1D) or use_count is None:
            nodes.append(node)
            continue
        decision = allow_inline_into_reduction(
            enabled, body_metrics(use_count, producer.body), use_count, 0, cfg)
        if decision == "disallow" or (
                decision == "clone"
                and (not allow_clone or TI.complexity(producer.body) > cfg.small_clone_nodes)):
            nodes.append(node)
            continue
        if use_count == 1:
            fused.add(producer.id)
        inputs, renamings = [], []
        for b in producer.inputs:
            fresh = _fresh(b.name, "r", inputs + list(producer.inputs))
            inputs.append(TI.InputBinding(fresh, b.source))
            renamings.append((b.name, fresh))
        node.source = TI.MappedInput(tuple(inputs), tuple(producer.scalar_params),
                                     rename_vars(renamings, producer.body))
        nodes.append(node)
    prog.nodes = [n for n in nodes
                  if not (isinstance(n, TI.Elementwise1D) and n.id in fused)]
    return prog


def shape_use_simplify(prog: TI.Program) -> TI.Program:
    """Drop the nodes the result does not reach (tensor_passes.ml:65-112)."""
    by_id = {n.id: n for n in prog.nodes}
    seen = set()
    stack = [prog.result]
    while stack:
        ref = stack.pop()
        if not isinstance(ref, TI.NodeRef) or ref.id in seen:
            continue
        seen.add(ref.id)
        n = by_id.get(ref.id)
        if isinstance(n, TI.Elementwise1D):
            stack.extend(b.source for b in n.inputs)
        elif isinstance(n, TI.Reduce1D):
            if isinstance(n.source, TI.PlainInput):
                stack.append(n.source.input)
            else:
                stack.extend(b.source for b in n.source.inputs)
    prog.nodes = [n for n in prog.nodes if n.id in seen]
    return prog


# --- body rewrites and CSE (tensor_passes.ml:6-60, 337-510) ----------------------

def _with_mapped(node: TI.Reduce1D, **changes) -> None:
    src = node.source
    node.source = TI.MappedInput(changes.get("inputs", src.inputs),
                                 changes.get("scalar_params", src.scalar_params),
                                 changes.get("body", src.body))


def _mapped(prog: TI.Program):
    return [n for n in prog.nodes
            if isinstance(n, TI.Reduce1D) and isinstance(n.source, TI.MappedInput)]


def canonicalize_program(prog: TI.Program) -> TI.Program:
    """tensor-canonicalize: scalar parameters sorted and unique, bodies in
    canonical operand order (tensor_passes.ml:6-33)."""
    for n in prog.nodes:
        if isinstance(n, TI.Elementwise1D):
            n.scalar_params = tuple(sorted(set(n.scalar_params)))
            n.body = A.canonicalize(n.body)
    for n in _mapped(prog):
        _with_mapped(n, scalar_params=tuple(sorted(set(n.source.scalar_params))),
                     body=A.canonicalize(n.source.body))
    return prog


def simplify_program(prog: TI.Program) -> TI.Program:
    """reduction-input-simplify: every body simplified (tensor_passes.ml:35-60)."""
    for n in prog.nodes:
        if isinstance(n, TI.Elementwise1D):
            n.body = A.simplify(n.body)
    for n in _mapped(prog):
        _with_mapped(n, body=A.simplify(n.source.body))
    return prog


def reduction_body_normalize(prog: TI.Program) -> TI.Program:
    """Mapped reductions: parameters sorted, inputs sorted by name, body
    canonicalised then simplified (tensor_passes.ml:337-358)."""
    for n in _mapped(prog):
        src = n.source
        _with_mapped(n, scalar_params=tuple(sorted(set(src.scalar_params))),
                     inputs=tuple(sorted(src.inputs, key=lambda b: b.name)),
                     body=A.simplify(A.canonicalize(src.body)))
    return prog


def reduction_reuse_hoist(prog: TI.Program) -> TI.Program:
    """tensor_passes.ml:360-376."""
    for n in _mapped(prog):
        _with_mapped(n, body=A.simplify(A.canonicalize(A.simplify(n.source.body))))
    return prog


def reduction_body_canonicalize(prog: TI.Program) -> TI.Program:
    """Products with data factors before scalar weights (tensor_passes.ml:378-394)."""
    for n in _mapped(prog):
        body = A.canonicalize_reduction_body(n.source.scalar_params, n.source.body)
        _with_mapped(n, body=A.canonicalize(A.simplify(body)))
    return prog


def branchy_reduction_rescue(prog: TI.Program) -> TI.Program:
    """tensor_passes.ml:396-412."""
    for n in _mapped(prog):
        body = A.branchy_weighted_rescue_body(n.source.scalar_params, n.source.body)
        _with_mapped(n, body=A.canonicalize(A.simplify(body)))
    return prog


def reduction_body_cse(prog: TI.Program, cfg: OptConfig = DEFAULT_CONFIG) -> TI.Program:
    """Bodies with at least ``reduction_body_cse_min_occurrences`` repeated
    subexpressions (tensor_passes.ml:414-438)."""
    for n in _mapped(prog):
        body = n.source.body
        if A.repeated_subexpressions(body) >= cfg.reduction_body_cse_min_occurrences:
            _with_mapped(n, body=A.canonicalize(A.simplify(A.reduction_body_cse_expr(body))))
    return prog


def _ref_key(ref: TI.ValueRef) -> str:
    return "p:" + ref.name if isinstance(ref, TI.ParamRef) else "n:%d" % ref.id


def _bindings_key(bindings) -> str:
    return "|".join(b.name + "=" + _ref_key(b.source) for b in bindings)


def _node_key(n: TI.Node) -> str:
    if isinstance(n, TI.Elementwise1D):
        return "e:%s:%s:%s:%s" % (n.shape_symbol, _bindings_key(n.inputs),
                                  ",".join(n.scalar_params), A.scalar_rank(n.body))
    if isinstance(n.source, TI.PlainInput):
        src = "p:" + _ref_key(n.source.input)
    else:
        src = "m:%s:%s:%s" % (_bindings_key(n.source.inputs), ",".join(n.source.scalar_params),
                              A.scalar_rank(n.source.body))
    return "r:%s:%s:%s" % (n.shape_symbol, n.kind, src)


def tensor_cse(prog: TI.Program) -> TI.Program:
    """A node whose key equals an earlier node's is dropped and its uses
    redirected to that node (tensor_passes.ml:440-513).  The key holds the
    body's rank, in which a unary's operator does not appear, so two maps of
    the same input that differ only in a unary operator merge, as there."""
    redirects: Dict[int, TI.ValueRef] = {}
    seen: Dict[str, int] = {}
    remap = lambda r: redirects.get(r.id, r) if isinstance(r, TI.NodeRef) else r
    keep = []
    for n in prog.nodes:
        if isinstance(n, TI.Elementwise1D):
            n.inputs = tuple(TI.InputBinding(b.name, remap(b.source)) for b in n.inputs)
        elif isinstance(n.source, TI.PlainInput):
            n.source = TI.PlainInput(remap(n.source.input))
        else:
            _with_mapped(n, inputs=tuple(TI.InputBinding(b.name, remap(b.source))
                                         for b in n.source.inputs))
        key = _node_key(n)
        if key in seen:
            redirects[n.id] = TI.NodeRef(seen[key])
            continue
        seen[key] = n.id
        keep.append(n)
    prog.nodes = keep
    prog.result = remap(prog.result)
    return prog


TENSOR_BODY_FLAGS = ("tensor-canonicalize", "reduction-input-simplify", "reduction-body-normalize",
                     "reduction-accumulator-shape", "reduction-reuse-hoist",
                     "branchy-reduction-rescue", "reduction-body-canonicalize",
                     "reduction-body-cse", "tensor-cse")


def _body_passes(prog: TI.Program, enabled, cfg: OptConfig) -> TI.Program:
    if _on(enabled, "tensor-canonicalize"):
        prog = canonicalize_program(prog)
    if _on(enabled, "reduction-input-simplify"):
        prog = simplify_program(prog)
    if _on(enabled, "reduction-body-normalize") or _on(enabled, "reduction-accumulator-shape"):
        prog = reduction_body_normalize(prog)
    if _on(enabled, "reduction-reuse-hoist"):
        prog = reduction_reuse_hoist(prog)
    if _on(enabled, "branchy-reduction-rescue"):
        prog = branchy_reduction_rescue(prog)
    if _on(enabled, "reduction-body-canonicalize"):
        prog = reduction_body_canonicalize(prog)
    if _on(enabled, "reduction-body-cse"):
        prog = reduction_body_cse(prog, cfg)
    return prog


def apply_tensor_passes(prog: TI.Program, enabled: Sequence[str],
                        cfg: OptConfig = DEFAULT_CONFIG) -> TI.Program:
    """The restated passes in the reference's order (tensor_passes.ml:554-666):
    the body rewrites, fusion, dead-node removal, node CSE, then the body
    rewrites once more."""
    enabled = tuple(enabled)
    prog = _body_passes(prog, enabled, cfg)
    clone = _on(enabled, "small-producer-clone")
    if any(_on(enabled, f) for f in FUSE_FLAGS):
        prog = fuse_program(prog, enabled, allow_clone=clone, cfg=cfg)
    if _on(enabled, "reduce-map-fusion"):
        prog = reduce_map_fusion_program(prog, enabled, allow_clone=clone, cfg=cfg)
    if _on(enabled, "shape-use-simplify"):
        prog = shape_use_simplify(prog)
    if _on(enabled, "tensor-cse"):
        prog = tensor_cse(prog)
    return _body_passes(prog, enabled, cfg)
