"""Optimisation pipeline between the frontend and the compiled program.

The pipeline is the reference's (src/forgeml/passes.py:410-430) pass for
pass, because its outcome is observable: the optimised graph, its pass
records and its slot plan are compared with the reference's one to one, and
the fusions decide which epilogues the native GEMM runs.  Passes, in order:

  eliminate_dead_nodes, fold_constants (results up to 64 MiB),
  eliminate_dead_nodes, simplify_algebra (identity reshapes and transposes,
  reshape-of-reshape, transpose pairs), common_subexpression_elimination
  (add / mul commutative), canonicalize_linear (matmul + 1-D bias ->
  linear), fuse_linear_gelu (gelu(linear | matmul [+ const bias]) ->
  fused_linear_gelu), fuse_shared_projections (constant-weight linears of one
  input -> one wide linear + narrow views: the fused QKV GEMM, constants
  ``<first>_shared_weight_<n>`` / ``<first>_shared_bias_<n>``, node
  ``<first>_shared_<n>``), eliminate_dead_nodes, schedule (six candidate
  topological orders; the one with the fewest planned bytes, ties broken by
  the order's node names).

Every pass maps a validated graph to a validated graph; ``_Edit`` carries the
bookkeeping they share (replacing, dropping and re-pointing nodes).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from forgeml_b200.forgeml.ir import Graph, GraphError, Node, TensorSpec
from forgeml_b200.forgeml.memory import VIEW_LIKE_OPS, plan_memory
from forgeml_b200.forgeml.ops import evaluate

FOLD_LIMIT_BYTES = 64 * 1024 * 1024


@dataclass(frozen=True)
class PassRecord:
    name: str
    nodes_before: int
    nodes_after: int


def _graph(base: Graph, nodes, constants, outputs=None) -> Graph:
    g = Graph(dict(base.inputs), constants, list(nodes), tuple(base.outputs if outputs is None else outputs),
              base.output_is_tuple)
    g.validate()
    return g


def _used_constants(constants: dict, nodes, outputs) -> dict:
    wanted = {i for n in nodes for i in n.inputs} | set(outputs)
    return {k: v for k, v in constants.items() if k in wanted}


def _readers(graph: Graph) -> dict[str, list[str]]:
    out: dict[str, list[str]] = {}
    for n in graph.nodes:
        for i in n.inputs:
            out.setdefault(i, []).append(n.name)
    return out


class _Renames:
    """Values replaced by other values (a removed node points at its stand-in)."""

    def __init__(self):
        self.to: dict[str, str] = {}

    def __call__(self, name: str) -> str:
        while name in self.to and self.to[name] != name:
            name = self.to[name]
        return name

    def node(self, n: Node) -> Node:
        return Node(n.name, n.op, tuple(self(i) for i in n.inputs), dict(n.attrs), n.spec)


# ------------------------------------------------------------------ passes
def eliminate_dead_nodes(graph: Graph) -> Graph:
    needed = set(graph.outputs)
    kept = []
    for n in reversed(graph.nodes):
        if n.name in needed:
            kept.append(n)
            needed.update(n.inputs)
    return _graph(graph, kept[::-1], {k: v for k, v in graph.constants.items() if k in needed})


def fold_constants(graph: Graph) -> Graph:
    known = dict(graph.constants)
    kept = []
    for n in graph.nodes:
        foldable = all(i in known for i in n.inputs)
        if foldable and n.op not in VIEW_LIKE_OPS:
            in_bytes = sum(known[i].numel() * known[i].element_size() for i in dict.fromkeys(n.inputs))
            foldable = n.spec.nbytes <= FOLD_LIMIT_BYTES and in_bytes <= FOLD_LIMIT_BYTES
        if not foldable:
            kept.append(n)
            continue
        try:
            with torch.inference_mode():
                known[n.name] = evaluate(n.op, tuple(known[i] for i in n.inputs), dict(n.attrs))
        except Exception as e:  # noqa: BLE001
            raise GraphError(f"constant folding failed at node {n.name!r}: {e}") from e
    return _graph(graph, kept, _used_constants(known, kept, graph.outputs))


def _transpose_pair(n: Node, rank: int) -> frozenset:
    return frozenset((n.attrs["dim0"] % rank, n.attrs["dim1"] % rank))


def simplify_algebra(graph: Graph) -> Graph:
    rn = _Renames()
    specs = graph.specs()
    kept: dict[str, Node] = {}
    for original in graph.nodes:
        n = rn.node(original)
        src = kept.get(n.inputs[0]) if n.inputs else None
        if n.op == "reshape":
            if specs[n.inputs[0]].shape == n.spec.shape:  # identity reshape
                rn.to[n.name] = n.inputs[0]
                continue
            if src is not None and src.op == "reshape":  # reshape of a reshape reads the source
                n = Node(n.name, "reshape", src.inputs, dict(n.attrs), n.spec)
        elif n.op == "transpose":
            rank = len(n.spec.shape)
            dims = _transpose_pair(n, rank)
            if len(dims) == 1:  # transpose(d, d)
                rn.to[n.name] = n.inputs[0]
                continue
            if src is not None and src.op == "transpose" and _transpose_pair(src, rank) == dims:
                rn.to[n.name] = rn(src.inputs[0])  # a transpose undoing the previous one
                continue
        kept[n.name] = n
    g = Graph(dict(graph.inputs), dict(graph.constants), list(kept.values()),
              tuple(rn(o) for o in graph.outputs), graph.output_is_tuple)
    g.validate()
    return eliminate_dead_nodes(g)


def _hashable(v):
    if isinstance(v, (tuple, list)):
        return tuple(_hashable(x) for x in v)
    if isinstance(v, dict):
        return tuple(sorted((k, _hashable(x)) for k, x in v.items()))
    return v


def common_subexpression_elimination(graph: Graph) -> Graph:
    rn = _Renames()
    first: dict[tuple, str] = {}
    kept = []
    for original in graph.nodes:
        n = rn.node(original)
        operands = tuple(sorted(n.inputs)) if n.op in ("add", "mul") else n.inputs
        key = (n.op, operands, _hashable(n.attrs), n.spec)
        if key in first:
            rn.to[n.name] = first[key]
            continue
        first[key] = n.name
        kept.append(n)
    outputs = tuple(rn(o) for o in graph.outputs)
    return _graph(graph, kept, _used_constants(graph.constants, kept, outputs), outputs)


def canonicalize_linear(graph: Graph) -> Graph:
    """add(matmul(x, W), b), b 1-D of the output width, the matmul read only
    there -> linear(x, W, b)."""
    readers = _readers(graph)
    nodes = {n.name: n for n in graph.nodes}
    specs = graph.specs()
    new, gone = {}, set()
    for n in graph.nodes:
        if n.op != "add":
            continue
        for mm_name, bias in ((n.inputs[0], n.inputs[1]), (n.inputs[1], n.inputs[0])):
            mm, bs = nodes.get(mm_name), specs.get(bias)
            if (mm is not None and mm.op == "matmul" and mm.name not in graph.outputs
                    and len(readers.get(mm.name, ())) == 1 and bs is not None and len(bs.shape) == 1
                    and bs.shape[0] == mm.spec.shape[1]):
                new[n.name] = Node(n.name, "linear", mm.inputs + (bias,), {}, n.spec)
                gone.add(mm.name)
                break
    kept = [new.get(n.name, n) for n in graph.nodes if n.name not in gone]
    return _graph(graph, kept, _used_constants(graph.constants, kept, graph.outputs))


def fuse_linear_gelu(graph: Graph) -> Graph:
    """gelu(linear | matmul) and gelu(add(matmul, constant 1-D bias)), each
    producer read only by the next -> fused_linear_gelu."""
    readers = _readers(graph)
    nodes = {n.name: n for n in graph.nodes}

    def private(n: Node) -> bool:
        return n.name not in graph.outputs and len(readers.get(n.name, ())) == 1

    new, gone = {}, set()
    for n in graph.nodes:
        if n.op != "gelu" or len(n.inputs) != 1:
            continue
        attrs = {"approximate": n.attrs.get("approximate", "none")}
        p = nodes.get(n.inputs[0])
        if p is None or not private(p):
            continue
        if p.op in ("linear", "matmul"):
            new[n.name] = Node(n.name, "fused_linear_gelu", p.inputs, attrs, n.spec)
            gone.add(p.name)
            continue
        if p.op != "add":
            continue
        pick = next(((nodes[a], b) for a, b in ((p.inputs[0], p.inputs[1]), (p.inputs[1], p.inputs[0]))
                     if a in nodes and nodes[a].op == "matmul" and b in graph.constants), None)
        if pick is None or not private(pick[0]):
            continue
        mm, bias = pick
        bt = graph.constants[bias]
        if bt.dim() == 1 and bt.shape[0] == mm.spec.shape[1] and len(mm.spec.shape) == 2:
            new[n.name] = Node(n.name, "fused_linear_gelu", (mm.inputs[0], mm.inputs[1], bias), attrs, n.spec)
            gone.update((mm.name, p.name))
    kept = [new.get(n.name, n) for n in graph.nodes if n.name not in gone]
    constants = _used_constants(graph.constants, kept, graph.outputs) if new else dict(graph.constants)
    return _graph(graph, kept, constants)


def fuse_shared_projections(graph: Graph) -> Graph:
    """Two or more linears with constant weights (and biases) reading the same
    input -> one wide linear over the concatenated weights, then one narrow
    view per original linear, in graph order (the fused QKV GEMM)."""
    position = {n.name: i for i, n in enumerate(graph.nodes)}
    families: dict[tuple[str, int], list[Node]] = {}
    for n in graph.nodes:
        if n.op == "linear" and all(i in graph.constants for i in n.inputs[1:]):
            families.setdefault((n.inputs[0], len(n.inputs)), []).append(n)
    families = {k: sorted(v, key=lambda m: position[m.name]) for k, v in families.items() if len(v) > 1}
    if not families:
        return _graph(graph, graph.nodes, dict(graph.constants))
    taken = set(graph.inputs) | set(graph.constants) | set(position)
    serial = [0]

    def unused(stem: str) -> str:
        while True:
            serial[0] += 1
            name = f"{stem}_{serial[0]}"
            if name not in taken:
                taken.add(name)
                return name

    constants = dict(graph.constants)
    specs = graph.specs()
    replacement: dict[str, list[Node]] = {}
    gone: set[str] = set()
    for members in families.values():
        lead = members[0]
        if len({constants[m.inputs[1]].dtype for m in members}) != 1:
            continue
        with_bias = len(lead.inputs) == 3
        if with_bias and len({constants[m.inputs[2]].dtype for m in members}) != 1:
            continue
        w = unused(f"{lead.name}_shared_weight")
        constants[w] = torch.cat([constants[m.inputs[1]] for m in members], dim=1).contiguous()
        ins = (lead.inputs[0], w)
        if with_bias:
            b = unused(f"{lead.name}_shared_bias")
            constants[b] = torch.cat([constants[m.inputs[2]] for m in members])
            ins += (b,)
        x = specs[lead.inputs[0]]
        wide_name = unused(f"{lead.name}_shared")
        width = sum(m.spec.shape[1] for m in members)
        block = [Node(wide_name, "linear", ins, {}, TensorSpec((x.shape[0], width), x.dtype, x.device))]
        start = 0
        for m in members:
            block.append(Node(m.name, "narrow", (wide_name,), {"dim": 1, "start": start, "length": m.spec.shape[1]},
                              m.spec))
            start += m.spec.shape[1]
            gone.add(m.name)
        replacement[lead.name] = block
    out = []
    for n in graph.nodes:
        if n.name in replacement:
            out.extend(replacement[n.name])
        elif n.name not in gone:
            out.append(n)
    return _graph(graph, out, constants)


# ------------------------------------------------------------------ scheduling
def _greedy_order(graph: Graph, priority) -> list[Node]:
    """A topological order that repeatedly runs the ready node of highest
    ``priority(node, original position, bytes its run frees)``."""
    position = {n.name: i for i, n in enumerate(graph.nodes)}
    nodes = {n.name: n for n in graph.nodes}
    specs = graph.specs()
    outputs = set(graph.outputs)
    readers: dict[str, set[str]] = {}
    for n in graph.nodes:
        for i in set(n.inputs):
            readers.setdefault(i, set()).add(n.name)
    blockers = {n.name: {i for i in n.inputs if i in position} for n in graph.nodes}
    reads_left = {k: len(v) for k, v in readers.items() if k in position}

    def frees(n: Node) -> int:
        return sum(specs[i].nbytes for i in set(n.inputs)
                   if i in position and i not in outputs and reads_left.get(i, 0) == 1)

    ready = [n for n in graph.nodes if not blockers[n.name]]
    order = []
    while ready:
        nxt = max(ready, key=lambda n: priority(n, position[n.name], frees(n)))
        ready.remove(nxt)
        order.append(nxt)
        for r in sorted(readers.get(nxt.name, ())):
            blockers[r].discard(nxt.name)
            if not blockers[r]:
                ready.append(nodes[r])
        for i in set(nxt.inputs):
            if i in reads_left:
                reads_left[i] -= 1
    if len(order) != len(graph.nodes):
        raise GraphError("graph contains a cycle")
    return order


_PRIORITIES = (
    lambda n, i, fr: (fr - n.spec.nbytes, -i),
    lambda n, i, fr: (fr - 2 * n.spec.nbytes, -i),
    lambda n, i, fr: (fr - n.spec.nbytes // 2, -i),
    lambda n, i, fr: (-n.spec.nbytes, fr, -i),
    lambda n, i, fr: (-i,),
    lambda n, i, fr: (i,),
)


def schedule(graph: Graph) -> Graph:
    candidates: dict[tuple, list[Node]] = {}
    for priority in _PRIORITIES:
        order = _greedy_order(graph, priority)
        candidates.setdefault(tuple(n.name for n in order), order)
    best = min(candidates.items(),
               key=lambda kv: (plan_memory(_graph(graph, kv[1], dict(graph.constants))).planned_bytes, kv[0]))[1]
    return _graph(graph, best, dict(graph.constants))


PIPELINE = (
    ("eliminate_dead_nodes", eliminate_dead_nodes),
    ("fold_constants", fold_constants),
    ("eliminate_dead_nodes", eliminate_dead_nodes),
    ("simplify_algebra", simplify_algebra),
    ("common_subexpression_elimination", common_subexpression_elimination),
    ("canonicalize_linear", canonicalize_linear),
    ("fuse_linear_gelu", fuse_linear_gelu),
    ("fuse_shared_projections", fuse_shared_projections),
    ("eliminate_dead_nodes", eliminate_dead_nodes),
    ("schedule", schedule),
)


def optimize(graph: Graph) -> tuple[Graph, list[PassRecord]]:
    graph.validate()
    g = graph.clone()
    records = []
    for name, run in PIPELINE:
        before = len(g.nodes)
        g = run(g)
        g.validate()
        records.append(PassRecord(name, before, len(g.nodes)))
    return g, records
