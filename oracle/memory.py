"""Slot-planner oracle: restates src/forgeml/memory.py:59-138 as a plain
recursive computation (integer bookkeeping, small graphs only).

Rules restated:
  * view ops (reshape/transpose/narrow) alias their first input and extend the
    live range of what they view to their own last use (memory.py:72-99);
  * graph outputs get no slot (:108-109); non-out-capable ops get no slot;
  * a node may take a slot whose current tenant's last use is strictly before
    the node's index, with equal dtype and device (:121-123), choosing the
    smallest capacity that fits, lowest slot id on ties (:124-129);
  * a new slot is flat 1-D, ceil(nbytes / itemsize) elements (:133-134).
Returns the same dict shape as MemoryPlan.to_dict().
"""

from __future__ import annotations

import math

VIEW_OPS = {"reshape", "transpose", "narrow"}
OUT_CAPABLE = {"matmul", "linear", "add", "mul", "relu", "softmax", "gelu", "embedding", "fused_linear_gelu"}


def plan(nodes, outputs, out_capable=OUT_CAPABLE):
    """nodes: list of dicts {name, op, inputs, spec:{shape,dtype,device}}; dtype as str."""
    itemsize = {"float32": 4, "float16": 2, "bfloat16": 2, "float64": 8, "int64": 8, "int32": 4,
                "int16": 2, "int8": 1, "uint8": 1, "bool": 1}
    idx = {n["name"]: i for i, n in enumerate(nodes)}
    byname = {n["name"]: n for n in nodes}

    def nbytes(n):
        return math.prod(n["spec"]["shape"]) * itemsize[n["spec"]["dtype"]]

    def last_use(name):
        best = idx[name]
        for c in nodes:
            if name in c["inputs"]:
                best = max(best, last_use(c["name"]) if c["op"] in VIEW_OPS else idx[c["name"]])
        return best

    outputs = set(outputs)
    aliases, allocs, slots = {}, {}, {}  # slots: id -> [elements, dtype, device, busy_until]
    naive = 0
    for n in nodes:
        if n["name"] in outputs:
            continue
        naive += nbytes(n)
        if n["op"] in VIEW_OPS:
            aliases[n["name"]] = n["inputs"][0]
            continue
        if n["op"] not in out_capable:
            continue
        first, last, need = idx[n["name"]], last_use(n["name"]), nbytes(n)
        isz = itemsize[n["spec"]["dtype"]]
        fits = [
            (s[0] * itemsize[s[1]], sid)
            for sid, s in slots.items()
            if s[3] < first and s[1] == n["spec"]["dtype"] and s[2] == n["spec"]["device"]
            and s[0] * itemsize[s[1]] >= need
        ]
        if fits:
            sid = min(fits)[1]
        else:
            sid = len(slots)
            slots[sid] = [-(-need // isz), n["spec"]["dtype"], n["spec"]["device"], -1]
        slots[sid][3] = last
        allocs[n["name"]] = {"slot": sid, "size_bytes": need, "first": first, "last": last}
    return {
        "aliases": aliases,
        "allocations": allocs,
        "slot_specs": {str(k): {"shape": [v[0]], "dtype": v[1], "device": v[2]} for k, v in slots.items()},
        "naive_bytes": naive,
        "planned_bytes": sum(v[0] * itemsize[v[1]] for v in slots.values()),
    }
