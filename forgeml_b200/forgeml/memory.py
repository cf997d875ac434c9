"""Slot-arena memory planner of the compiled forward pass.

The plan is part of the drop-in contract: for a given graph it must come out
exactly as the reference planner's (src/forgeml/memory.py:59-138) -- same
slot ids, sizes, live intervals, aliases, naive and planned bytes.  The rules
it has to share with the reference:

  * view ops (reshape, transpose, narrow) take no slot; they alias their
    first input and keep it live until their own last use;
  * graph outputs, and ops without an ``out=`` writer, take no slot;
  * a node may take a slot whose tenant's last use is strictly earlier than
    the node's position, of the same dtype and device; of those it takes the
    smallest that fits, the lowest slot id on ties;
  * otherwise it opens a new flat 1-D slot of ceil(nbytes / itemsize)
    elements.

``plan_slots`` implements them over plain (name, op, inputs, spec) entries,
so the native backend can plan its own execution program (fused nodes,
LayerNorm / SDPA outputs) with the same rules; ``plan_memory`` is the
reference-facing entry point over a validated Graph.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, NamedTuple

from forgeml_b200.forgeml.ir import Graph, TensorSpec

VIEW_LIKE_OPS = frozenset({"reshape", "transpose", "narrow"})
OUT_CAPABLE_OPS = frozenset(
    {"matmul", "linear", "add", "mul", "relu", "softmax", "gelu", "embedding", "fused_linear_gelu"})


class Entry(NamedTuple):
    name: str
    op: str
    inputs: tuple
    spec: TensorSpec


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
            "allocations": {k: {"slot": a.slot, "size_bytes": a.size_bytes, "first": a.first, "last": a.last}
                            for k, a in self.allocations.items()},
            "slot_specs": {str(k): v.to_dict() for k, v in self.slot_specs.items()},
            "naive_bytes": self.naive_bytes,
            "planned_bytes": self.planned_bytes,
        }


def last_reads(entries: list[Entry]) -> dict[str, int]:
    """Position of the last entry that reads each value, through views: a view
    read at position j keeps what it views alive until j as well.  A value
    nobody reads ends at its own position."""
    pos = {e.name: i for i, e in enumerate(entries)}
    end = dict(pos)
    for e in reversed(entries):  # a view's own end is final before its inputs are visited
        reach = end[e.name] if e.op in VIEW_LIKE_OPS else pos[e.name]
        for src in e.inputs:
            if src in end and end[src] < reach:
                end[src] = reach
    return end


class _Slots:
    """Open slots with the position until which each one is taken."""

    def __init__(self):
        self.specs: dict[int, TensorSpec] = {}
        self.taken_until: dict[int, int] = {}

    def fit(self, spec: TensorSpec, nbytes: int, at: int) -> int:
        best, best_cap = None, None
        for sid, s in self.specs.items():
            if self.taken_until[sid] >= at or s.dtype != spec.dtype or s.device != spec.device:
                continue
            cap = s.shape[0] * s.dtype.itemsize
            if cap >= nbytes and (best is None or cap < best_cap):
                best, best_cap = sid, cap
        if best is None:
            best = len(self.specs)
            self.specs[best] = TensorSpec((-(-nbytes // spec.dtype.itemsize),), spec.dtype, spec.device)
        return best


def plan_slots(entries: Iterable[Entry], outputs: Iterable[str],
               out_capable: frozenset = OUT_CAPABLE_OPS) -> MemoryPlan:
    entries = list(entries)
    outs = set(outputs)
    ends = last_reads(entries)
    slots = _Slots()
    allocations: dict[str, Allocation] = {}
    aliases: dict[str, str] = {}
    naive = 0
    for i, e in enumerate(entries):
        if e.name in outs:
            continue
        naive += e.spec.nbytes
        if e.op in VIEW_LIKE_OPS:
            aliases[e.name] = e.inputs[0]
        elif e.op in out_capable:
            sid = slots.fit(e.spec, e.spec.nbytes, i)
            slots.taken_until[sid] = ends[e.name]
            allocations[e.name] = Allocation(sid, e.spec.nbytes, i, ends[e.name])
    planned = sum(s.shape[0] * s.dtype.itemsize for s in slots.specs.values())
    return MemoryPlan(allocations, aliases, slots.specs, naive, planned)


def graph_entries(graph: Graph) -> list[Entry]:
    return [Entry(n.name, n.op, tuple(n.inputs), n.spec) for n in graph.nodes]


def plan_memory(graph: Graph, out_capable: frozenset = OUT_CAPABLE_OPS) -> MemoryPlan:
    """The reference-compatible slot plan of a (validated) graph."""
    graph.validate()
    return plan_slots(graph_entries(graph), graph.outputs, out_capable)
