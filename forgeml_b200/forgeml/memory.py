"""Slot-arena memory planner.

Produces the same plan as the reference planner (src/forgeml/memory.py:59-138)
for the same graph -- identical slot ids, sizes, live intervals, aliases,
naive and planned bytes -- because the compiled model's slot views are part
of the drop-in contract.  The rules that must match:

* view ops (reshape, transpose, narrow) alias their first input, take no
  slot, and extend the live range of what they view to their own last use;
* graph outputs and ops without an ``out=`` writer get no slot;
* a node may reuse a slot whose current tenant's last use is strictly before
  the node's index, with equal dtype and device; among those it takes the
  smallest capacity that fits (lowest slot id on ties);
* a new slot is a flat 1-D buffer of ceil(nbytes / itemsize) elements.

``plan_memory(graph, out_capable=...)`` with a wider op set plans the
extension arena that the native backend uses for LayerNorm and SDPA outputs
(same rules, separate slots), leaving the reference-compatible plan intact.
"""

from __future__ import annotations

from dataclasses import dataclass

from forgeml_b200.forgeml.ir import Graph, TensorSpec

VIEW_LIKE_OPS = frozenset({"reshape", "transpose", "narrow"})
OUT_CAPABLE_OPS = frozenset(
    {"matmul", "linear", "add", "mul", "relu", "softmax", "gelu", "embedding", "fused_linear_gelu"}
)


@dataclass(frozen=True)
class Allocation:
    slot: int
    size_bytes: int
    first: int
    last: int


@dataclass
class MemoryPlan:
    allocations: dict[str, Allocation]
    aliases: dict[str, str]
    slot_specs: dict[int, TensorSpec]
    naive_bytes: int
    planned_bytes: int

    def to_dict(self) -> dict:
        return {
            "aliases": dict(self.aliases),
            "allocations": {
                k: {"slot": a.slot, "size_bytes": a.size_bytes, "first": a.first, "last": a.last}
                for k, a in self.allocations.items()
            },
            "slot_specs": {str(k): v.to_dict() for k, v in self.slot_specs.items()},
            "naive_bytes": self.naive_bytes,
            "planned_bytes": self.planned_bytes,
        }


def _last_uses(graph: Graph) -> dict[str, int]:
    """Index of the last node that reads each value, looking through views.

    Computed in one reverse sweep: a consumer that is a view op contributes the
    last use of the view itself (already known, since it comes later).
    """
    index = {n.name: i for i, n in enumerate(graph.nodes)}
    last = {n.name: i for i, n in enumerate(graph.nodes)}
    for node in reversed(graph.nodes):
        through = last[node.name] if node.op in VIEW_LIKE_OPS else index[node.name]
        for src in set(node.inputs):
            if src in last and through > last[src]:
                last[src] = through
    return last


def plan_memory(graph: Graph, out_capable: frozenset = OUT_CAPABLE_OPS) -> MemoryPlan:
    graph.validate()
    outputs = set(graph.outputs)
    last_use = _last_uses(graph)
    aliases: dict[str, str] = {}
    allocations: dict[str, Allocation] = {}
    slot_specs: dict[int, TensorSpec] = {}
    busy_until: dict[int, int] = {}
    naive = 0
    for i, node in enumerate(graph.nodes):
        if node.name in outputs:
            continue
        naive += node.spec.nbytes
        if node.op in VIEW_LIKE_OPS:
            aliases[node.name] = node.inputs[0]
            continue
        if node.op not in out_capable:
            continue
        need = node.spec.nbytes
        itemsize = node.spec.dtype.itemsize
        chosen, chosen_cap = None, None
        for slot, spec in slot_specs.items():  # insertion order == slot id order
            if busy_until[slot] >= i or spec.dtype != node.spec.dtype or spec.device != node.spec.device:
                continue
            cap = spec.shape[0] * spec.dtype.itemsize
            if cap >= need and (chosen is None or cap < chosen_cap):
                chosen, chosen_cap = slot, cap
        if chosen is None:
            chosen = len(slot_specs)
            slot_specs[chosen] = TensorSpec((-(-need // itemsize),), node.spec.dtype, node.spec.device)
        busy_until[chosen] = last_use[node.name]
        allocations[node.name] = Allocation(chosen, need, i, last_use[node.name])
    planned = sum(s.shape[0] * s.dtype.itemsize for s in slot_specs.values())
    return MemoryPlan(allocations, aliases, slot_specs, naive, planned)
