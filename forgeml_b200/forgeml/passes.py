"""Graph optimisation pipeline feeding the compiled forward pass.

Same pass sequence and outcomes as the reference (src/forgeml/passes.py:
410-430): dead-node elimination, constant folding (64 MiB cap), algebraic
simplification (identity reshapes/transposes, reshape chains, transpose
pairs), CSE (commutative add/mul), matmul+bias -> linear, linear/matmul(+bias)
-> fused_linear_gelu, shared-input linears -> one wide linear + narrow views
(the fused QKV GEMM; ``<leader>_shared_weight_<n>`` naming), and a
memory-aware topological schedule chosen among six candidate orders by planned
bytes (ties by node-name tuple).  Fusion patterns decide which GEMM epilogues
the native kernel runs, and the final order decides the slot plan, so both
follow the reference's rules exactly.
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


def _rebuild(graph: Graph, nodes: list[Node], constants: dict, outputs=None) -> Graph:
    g = Graph(inputs=dict(graph.inputs), constants=constants, nodes=nodes,
              outputs=tuple(graph.outputs if outputs is None else outputs), output_is_tuple=graph.output_is_tuple)
    g.validate()
    return g


def _consumers(graph: Graph) -> dict[str, list[str]]:
    out: dict[str, list[str]] = {}
    for n in graph.nodes:
        for i in n.inputs:
            out.setdefault(i, []).append(n.name)
    return out


def _follow(aliases: dict[str, str], name: str) -> str:
    while aliases.get(name, name) != name:
        name = aliases[name]
    return name


def _keep_used(constants: dict, nodes: list[Node], extra=()) -> dict:
    used = {i for n in nodes for i in n.inputs} | set(extra)
    return {k: v for k, v in constants.items() if k in used}


def eliminate_dead_nodes(graph: Graph) -> Graph:
    live = set(graph.outputs)
    kept = []
    for n in reversed(graph.nodes):
        if n.name in live:
            kept.append(n)
            live.update(n.inputs)
    kept.reverse()
    return _rebuild(graph, kept, {k: v for k, v in graph.constants.items() if k in live})


def fold_constants(graph: Graph) -> Graph:
    constants = dict(graph.constants)
    env = dict(constants)
    nodes = []
    for n in graph.nodes:
        if not all(i in env for i in n.inputs):
            nodes.append(n)
            continue
        in_bytes = sum(env[i].numel() * env[i].element_size() for i in dict.fromkeys(n.inputs))
        if n.op not in VIEW_LIKE_OPS and (n.spec.nbytes > FOLD_LIMIT_BYTES or in_bytes > FOLD_LIMIT_BYTES):
            nodes.append(n)
            continue
        try:
            with torch.inference_mode():
                val = evaluate(n.op, tuple(env[i] for i in n.inputs), dict(n.attrs))
        except Exception as e:  # noqa: BLE001
            raise GraphError(f"constant folding failed at node {n.name!r}: {e}") from e
        constants[n.name] = env[n.name] = val
    return _rebuild(graph, nodes, _keep_used(constants, nodes, graph.outputs))


def simplify_algebra(graph: Graph) -> Graph:
    aliases: dict[str, str] = {}
    kept: dict[str, Node] = {}
    nodes: list[Node] = []
    specs = graph.specs()
    for n in graph.nodes:
        n = Node(n.name, n.op, tuple(_follow(aliases, i) for i in n.inputs), dict(n.attrs), n.spec)
        if n.op == "reshape":
            if specs[n.inputs[0]].shape == n.spec.shape:
                aliases[n.name] = n.inputs[0]
                continue
            src = kept.get(n.inputs[0])
            if src is not None and src.op == "reshape":
                n = Node(n.name, "reshape", src.inputs, dict(n.attrs), n.spec)
        if n.op == "transpose":
            rank = len(n.spec.shape)
            dims = frozenset((n.attrs["dim0"] % rank, n.attrs["dim1"] % rank))
            if len(dims) == 1:
                aliases[n.name] = n.inputs[0]
                continue
            src = kept.get(n.inputs[0])
            if (src is not None and src.op == "transpose"
                    and frozenset((src.attrs["dim0"] % rank, src.attrs["dim1"] % rank)) == dims):
                aliases[n.name] = _follow(aliases, src.inputs[0])
                continue
        aliases[n.name] = n.name
        kept[n.name] = n
        nodes.append(n)
    outputs = tuple(_follow(aliases, o) for o in graph.outputs)
    g = Graph(inputs=dict(graph.inputs), constants=dict(graph.constants), nodes=nodes, outputs=outputs,
              output_is_tuple=graph.output_is_tuple)
    g.validate()
    return eliminate_dead_nodes(g)


def _frozen(v):
    if isinstance(v, (tuple, list)):
        return tuple(_frozen(x) for x in v)
    if isinstance(v, dict):
        return tuple(sorted((k, _frozen(x)) for k, x in v.items()))
    return v


def common_subexpression_elimination(graph: Graph) -> Graph:
    aliases: dict[str, str] = {}
    seen: dict[tuple, str] = {}
    nodes = []
    for n in graph.nodes:
        ins = tuple(_follow(aliases, i) for i in n.inputs)
        key = (n.op, tuple(sorted(ins)) if n.op in ("add", "mul") else ins, _frozen(n.attrs), n.spec)
        if key in seen:
            aliases[n.name] = seen[key]
            continue
        seen[key] = n.name
        aliases[n.name] = n.name
        nodes.append(Node(n.name, n.op, ins, dict(n.attrs), n.spec))
    outputs = tuple(_follow(aliases, o) for o in graph.outputs)
    return _rebuild(graph, nodes, _keep_used(graph.constants, nodes, outputs), outputs=outputs)


def canonicalize_linear(graph: Graph) -> Graph:
    """add(matmul(x, W), b) with a 1-D output-width b -> linear(x, W, b)."""
    cons = _consumers(graph)
    by = {n.name: n for n in graph.nodes}
    specs = graph.specs()
    repl: dict[str, Node] = {}
    drop: set[str] = set()
    for n in graph.nodes:
        if n.op != "add":
            continue
        for mm_name, bias in ((n.inputs[0], n.inputs[1]), (n.inputs[1], n.inputs[0])):
            mm = by.get(mm_name)
            bs = specs.get(bias)
            if (mm is None or mm.op != "matmul" or mm.name in graph.outputs or len(cons.get(mm.name, ())) != 1
                    or bs is None or len(bs.shape) != 1 or bs.shape[0] != mm.spec.shape[1]):
                continue
            repl[n.name] = Node(n.name, "linear", mm.inputs + (bias,), {}, n.spec)
            drop.add(mm.name)
            break
    nodes = [repl.get(n.name, n) for n in graph.nodes if n.name not in drop]
    return _rebuild(graph, nodes, _keep_used(graph.constants, nodes, graph.outputs))


def fuse_linear_gelu(graph: Graph) -> Graph:
    """gelu(linear|matmul) and gelu(add(matmul, const bias)) -> fused_linear_gelu."""
    cons = _consumers(graph)
    by = {n.name: n for n in graph.nodes}
    fused: dict[str, Node] = {}
    drop: set[str] = set()

    def single_use(node):
        return node.name not in graph.outputs and len(cons.get(node.name, ())) == 1

    for n in graph.nodes:
        if n.op != "gelu" or len(n.inputs) != 1:
            continue
        approx = {"approximate": n.attrs.get("approximate", "none")}
        p = by.get(n.inputs[0])
        if p is not None and p.op in ("linear", "matmul") and single_use(p):
            fused[n.name] = Node(n.name, "fused_linear_gelu", p.inputs, approx, n.spec)
            drop.add(p.name)
            continue
        if p is None or p.op != "add" or not single_use(p):
            continue
        mm, bias = None, None
        for cand, other in ((p.inputs[0], p.inputs[1]), (p.inputs[1], p.inputs[0])):
            c = by.get(cand)
            if c is not None and c.op == "matmul" and other in graph.constants:
                mm, bias = c, other
                break
        if mm is None or not single_use(mm):
            continue
        bt = graph.constants[bias]
        if bt.dim() != 1 or bt.shape[0] != mm.spec.shape[1] or len(mm.spec.shape) != 2:
            continue
        fused[n.name] = Node(n.name, "fused_linear_gelu", (mm.inputs[0], mm.inputs[1], bias), approx, n.spec)
        drop.update((mm.name, p.name))
    if not fused:
        return _rebuild(graph, list(graph.nodes), dict(graph.constants))
    nodes = [fused.get(n.name, n) for n in graph.nodes if n.name not in drop]
    return _rebuild(graph, nodes, _keep_used(graph.constants, nodes, graph.outputs))


def fuse_shared_projections(graph: Graph) -> Graph:
    """Linears with constant weights reading the same input -> one wide linear
    followed by one narrow view per original linear (e.g. Q, K, V)."""
    index = {n.name: i for i, n in enumerate(graph.nodes)}
    specs = graph.specs()
    groups: dict[tuple[str, int], list[Node]] = {}
    for n in graph.nodes:
        if n.op != "linear" or n.inputs[1] not in graph.constants:
            continue
        if len(n.inputs) == 3 and n.inputs[2] not in graph.constants:
            continue
        groups.setdefault((n.inputs[0], len(n.inputs)), []).append(n)
    groups = {k: v for k, v in groups.items() if len(v) >= 2}
    if not groups:
        return _rebuild(graph, list(graph.nodes), dict(graph.constants))
    taken = set(graph.inputs) | set(graph.constants) | set(index)
    constants = dict(graph.constants)
    counter = [0]

    def fresh(hint):
        while True:
            counter[0] += 1
            cand = f"{hint}_{counter[0]}"
            if cand not in taken:
                taken.add(cand)
                return cand

    emit: dict[str, list[Node]] = {}
    drop: set[str] = set()
    for members in groups.values():
        members.sort(key=lambda m: index[m.name])
        lead = members[0]
        if len({constants[m.inputs[1]].dtype for m in members}) != 1:
            continue
        if len(lead.inputs) == 3 and len({constants[m.inputs[2]].dtype for m in members}) > 1:
            continue
        xs = specs[lead.inputs[0]]
        wname = fresh(f"{lead.name}_shared_weight")
        constants[wname] = torch.cat([constants[m.inputs[1]] for m in members], dim=1).contiguous()
        ins = [lead.inputs[0], wname]
        if len(lead.inputs) == 3:
            bname = fresh(f"{lead.name}_shared_bias")
            constants[bname] = torch.cat([constants[m.inputs[2]] for m in members])
            ins.append(bname)
        width = sum(m.spec.shape[1] for m in members)
        wide = fresh(f"{lead.name}_shared")
        out = [Node(wide, "linear", tuple(ins), {}, TensorSpec((xs.shape[0], width), xs.dtype, xs.device))]
        off = 0
        for m in members:
            out.append(Node(m.name, "narrow", (wide,), {"dim": 1, "start": off, "length": m.spec.shape[1]}, m.spec))
            off += m.spec.shape[1]
            drop.add(m.name)
        emit[lead.name] = out
    nodes: list[Node] = []
    for n in graph.nodes:
        if n.name in emit:
            nodes.extend(emit[n.name])
        elif n.name not in drop:
            nodes.append(n)
    return _rebuild(graph, nodes, constants)


def _topo_order(graph: Graph, score) -> list[Node]:
    outputs = set(graph.outputs)
    index = {n.name: i for i, n in enumerate(graph.nodes)}
    by = {n.name: n for n in graph.nodes}
    cons: dict[str, set[str]] = {}
    waiting: dict[str, set[str]] = {}
    for n in graph.nodes:
        for i in set(n.inputs):
            cons.setdefault(i, set()).add(n.name)
        waiting[n.name] = {i for i in n.inputs if i in index}
    specs = graph.specs()
    remaining_uses = {k: len(v) for k, v in cons.items() if k in index}

    def freed(n: Node) -> int:
        return sum(specs[i].nbytes for i in set(n.inputs)
                   if i not in outputs and i in index and remaining_uses.get(i, 0) == 1)

    ready = [n for n in graph.nodes if not waiting[n.name]]
    order: list[Node] = []
    while ready:
        best = max(ready, key=lambda n: score(n, index[n.name], freed(n)))
        ready.remove(best)
        order.append(best)
        for c in sorted(cons.get(best.name, ())):
            waiting[c].discard(best.name)
            if not waiting[c]:
                ready.append(by[c])
        for i in set(best.inputs):
            if i in remaining_uses:
                remaining_uses[i] -= 1
    if len(order) != len(graph.nodes):
        raise GraphError("graph contains a cycle")
    return order


_SCHEDULE_SCORES = (
    lambda n, i, fr: (fr - n.spec.nbytes, -i),
    lambda n, i, fr: (fr - 2 * n.spec.nbytes, -i),
    lambda n, i, fr: (fr - n.spec.nbytes // 2, -i),
    lambda n, i, fr: (-n.spec.nbytes, fr, -i),
    lambda n, i, fr: (-i,),
    lambda n, i, fr: (i,),
)


def schedule(graph: Graph) -> Graph:
    orders, seen = [], set()
    for score in _SCHEDULE_SCORES:
        order = _topo_order(graph, score)
        key = tuple(n.name for n in order)
        if key not in seen:
            seen.add(key)
            orders.append(order)
    best = min(orders, key=lambda o: (plan_memory(_rebuild(graph, o, dict(graph.constants))).planned_bytes,
                                      tuple(n.name for n in o)))
    return _rebuild(graph, best, dict(graph.constants))


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
    work = graph.clone()
    records = []
    for name, fn in PIPELINE:
        before = len(work.nodes)
        work = fn(work)
        work.validate()
        records.append(PassRecord(name, before, len(work.nodes)))
    return work, records
